"""Drop-in for modelcore's `flash_attn` kernel namespace (modelcore/kernels/flash_attn.py:373-376).

`flash_attn_with_kvcache` keeps the reference signature and contract
(modelcore/kernels/flash_attn.py:306-366): k, v (when given) are written in place at each row's
positions [cache_seqlens[b], cache_seqlens[b] + T_new), cache_seqlens is NOT advanced, and the
result is a fresh (B, T_new, H, D) tensor.  Both halves run on libmcb200 kernels (the insert, then
the split-K decode attention); there is no host sync (the reference reads cache_seqlens back with
tolist(), flash_attn.py:332) and no mask tensor.  `causal` is ignored exactly as the reference's
SDPA path ignores it (the KV path is always causal), and so is window_size[1].

`flash_attn_func` (the training path, kv_cache is None) is outside the decode path: the namespace
forwards it to the reference's own implementation unchanged.

`install()` swaps the reference namespace's entry in place -- the same switch modelcore makes
when FA3 is available (flash_attn.py:71-86) -- so every Attention module picks it up.
"""
from types import SimpleNamespace

from . import ops


def flash_attn_with_kvcache(q, k_cache, v_cache, k=None, v=None, cache_seqlens=None,
                            causal=False, window_size=(-1, -1)):
    if cache_seqlens is None:
        raise RuntimeError("flash_attn_with_kvcache needs cache_seqlens")
    if (k is None) != (v is None):
        raise RuntimeError("pass both k and v, or neither")
    if k is not None:
        ops.kv_write(k, v, k_cache, v_cache, cache_seqlens)
    return ops.decode_attn(q, k_cache, v_cache, cache_seqlens, window=window_size[0])


def _reference_flash_attn_func(*args, **kwargs):
    from modelcore.kernels.flash_attn import flash_attn_func as ref
    return ref(*args, **kwargs)


flash_attn = SimpleNamespace(
    flash_attn_func=_reference_flash_attn_func,
    flash_attn_with_kvcache=flash_attn_with_kvcache,
)

_saved = {}


def install():
    """Route modelcore's flash_attn.flash_attn_with_kvcache to this implementation, process-wide.
    Returns the reference function it replaced (also restorable with uninstall())."""
    import modelcore.kernels.flash_attn as ref_mod
    ns = ref_mod.flash_attn
    if "with_kvcache" not in _saved:
        _saved["with_kvcache"] = ns.flash_attn_with_kvcache
    ns.flash_attn_with_kvcache = flash_attn_with_kvcache
    return _saved["with_kvcache"]


def uninstall():
    import modelcore.kernels.flash_attn as ref_mod
    if "with_kvcache" in _saved:
        ref_mod.flash_attn.flash_attn_with_kvcache = _saved.pop("with_kvcache")
