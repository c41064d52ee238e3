"""The decode path as PyTorch dispatcher operators: torch.ops.mcb200.*.

Importing this module loads libmcb200_torch.so (csrc/torch_ops.cpp, C++ over the same libmcb200
C ABI that modelcore_b200.ops reaches through ctypes) and registers the operators' shape
functions, so that torch.compile can trace through them:

    torch.ops.mcb200.kv_append_rope(q, k, v, k_cache, v_cache, cache_seqlens, cos, sin,
                                    eps=None, scale=1.2, ring=False) -> q'
        rope + QK-norm + x scale of q (and, with k, of k) and the insert of k, v at each row's
        position (modelcore/components/attention.py:147-160, kernels/flash_attn.py:337-346);
        k, v, k_cache, v_cache all None for a layer that reads another layer's slot
    torch.ops.mcb200.kv_broadcast(src_k, src_v, dst_k, dst_v, src_row, dst_row_begin,
                                  dst_row_count, n_pos, dst_seqlens=None)
        KVCache.prefill / prefill_row's copy (modelcore/cache.py:75-119), in place
    torch.ops.mcb200.decode_attn(q, k_cache, v_cache, cache_seqlens, window=-1,
                                 softmax_scale=None, num_ctas=0, ring=False) -> y
        the attention of flash_attn_with_kvcache over one slot (kernels/flash_attn.py:348-366)
    torch.ops.mcb200.append_attn(q, k, v, k_cache, v_cache, cache_seqlens, cos, sin, eps=None,
                                 scale=1.2, window=-1, ring=False) -> y
        the two above in one launch where the plan allows it (a decode step), else two
    torch.ops.mcb200.kv_advance(cache_seqlens, n)
        KVCache.advance (modelcore/cache.py:62-73), in place
    torch.ops.mcb200.linear(x, weight, out, res=None, h_out=None, eps=None, gated=False, pdl=False)
        the decode step's projections (ops.linear's plain, residual, gated and norm-out modes),
        into out (and h_out)
    torch.ops.mcb200.add_rms_norm(x, delta, x_out, h_out, eps=None)
        the residual add and the next RMSNorm (ops.add_rms_norm), into x_out and h_out

bf16 slots only (the fp8 cache format is reached through modelcore_b200.ops).  The results are
those of the ctypes entry points bit for bit: one library does the work.  Without the built
library the import fails: there is no fallback.
"""
import os

import torch

from . import _native
from .build import TORCH_OPS_PATH

OPS = ("kv_append_rope", "kv_broadcast", "decode_attn", "append_attn", "kv_advance", "linear",
       "add_rms_norm")


def _register_fakes():
    def like_q(q, *args, **kwargs):
        return torch.empty(q.shape, dtype=q.dtype, device=q.device)

    def nothing(*args, **kwargs):
        return None

    for name, fn in (("kv_append_rope", like_q), ("decode_attn", like_q), ("append_attn", like_q),
                     ("kv_broadcast", nothing), ("kv_advance", nothing), ("linear", nothing),
                     ("add_rms_norm", nothing)):
        torch.library.register_fake(f"mcb200::{name}")(fn)


def _load():
    if not os.path.exists(TORCH_OPS_PATH):
        raise ImportError(f"{TORCH_OPS_PATH} is missing: build it with "
                          "`python -m modelcore_b200.build` (or __graft_entry__.build())")
    _native.load()  # libmcb200.so first, with its ABI-version check
    torch.ops.load_library(TORCH_OPS_PATH)
    _register_fakes()


_load()
