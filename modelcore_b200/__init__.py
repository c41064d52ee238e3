"""modelcore_b200 -- modelcore's KV-cache decode path on hand-written sm_100a CUDA kernels.

Public surface (mirrors modelcore's names for this path):
  KVCache                   modelcore.cache.KVCache on the B200 layout and kernels
  flash_attn                namespace with flash_attn_with_kvcache (modelcore.kernels.flash_attn's)
  flash_attn_with_kvcache   insert + split-K decode attention
  ModelManager              modelcore.ModelManager with the decode path installed (needs modelcore)
  install / uninstall       bind / unbind the B200 attention forward on a built modelcore model
  GraphDecoder              modelcore's Decoder stepping through a captured CUDA graph
  sample_next_token         modelcore.generate.sample_next_token on one libmcb200 kernel
  ops                       the torch-facing wrappers of the C ABI (include/mcb200.h)

The kernels live in libmcb200.so next to this file (build: `python -m modelcore_b200.build`).
The library is loaded on first use (any op, any KVCache) and its absence is an error: nothing
here has a CPU or pure-Python fallback.
"""
from . import _native, ops
from .cache import KVCache
from .flash_attn import flash_attn, flash_attn_with_kvcache
from .sampling import sample_next_token

__all__ = ["KVCache", "flash_attn", "flash_attn_with_kvcache", "ModelManager", "install",
           "uninstall", "GraphDecoder", "sample_next_token", "ops"]


def __getattr__(name):
    # modelcore-facing pieces import modelcore lazily: the kernels and KVCache do not need it.
    if name in ("install", "uninstall", "GraphDecoder", "attention_forward"):
        from . import integration
        return getattr(integration, name)
    if name == "ModelManager":
        from . import integration
        cls = integration.make_manager_class()
        globals()["ModelManager"] = cls
        return cls
    raise AttributeError(name)
