"""modelcore glue: the B200 decode path behind modelcore's own API.

    from modelcore_b200 import ModelManager          # instead of modelcore.ModelManager
    manager = ModelManager()
    model = manager.create_model(config, device=torch.device("cuda"), seed=0).to(torch.bfloat16)
    decoder = manager.new_decoder(model, prompts, max_tokens=512)   # modelcore's Decoder
    logits = decoder.step(tokens)                                    # or model(idx, kv_cache=...)

* `ModelManager` is modelcore.ModelManager with new_kv_cache returning modelcore_b200.KVCache on
  CUDA devices, and create_model / load_model installing the B200 attention forward on every
  Attention module of the model they return.  Everything else is the reference's.
* `install(model)` binds `attention_forward` to each modelcore Attention module (an instance
  attribute; the class and the catalog are untouched, modelcore/catalog.py:25 forbids
  re-registering "attention").  With kv_cache=None (training) the module's original forward runs.
* `GraphDecoder` is modelcore's Decoder whose steps replay a CUDA graph of the decode forward.
"""
import types

import torch

from . import ops, step
from .cache import KVCache
from .flash_attn import flash_attn_with_kvcache

_ORIGINAL_FORWARD = "_mcb_original_forward"
_FUSE_QKV = "_mcb_fuse_qkv"


def _fusable(attn, x):
    """The fused append applies when QK-norm is modelcore's RMSNorm and the position encoding is
    its RotaryEmbedding with bf16 tables on x's device."""
    from modelcore.components.norm import RMSNorm
    from modelcore.components.rotary import RotaryEmbedding
    rope = attn.rope
    return (isinstance(attn.norm, RMSNorm) and isinstance(rope, RotaryEmbedding)
            and rope.cos.dtype == torch.bfloat16 and rope.cos.device == x.device
            and attn.head_dim % 2 == 0 and attn.head_dim <= 256)


# The decode step's append and attention in one launch where the plan allows it (T = 1, a bf16
# slot, the split or persistent plan; ops.append_attn), with the bits of the two launches.
USE_FUSED_APPEND = True
# ... through the torch.ops.mcb200 operator (C++ over the same library: a third of the host cost
# of the ctypes call, which an eager, ungraphed decode step pays once per layer) for bf16 slots
USE_TORCH_OPS = True
_TORCH_OPS = None


def _torch_ops():
    global _TORCH_OPS
    if _TORCH_OPS is None:
        from . import torch_ops  # loads libmcb200_torch.so; fails loudly when it is missing
        _TORCH_OPS = torch.ops.mcb200
    return _TORCH_OPS


def attend(self, q, k, v, kv_cache):
    """The fused KV-cache branch of Attention.forward (modelcore/components/attention.py:144-178)
    from projected (B, T, H, D) q, k, v (k and v None for a consumer layer, produces_kv=False):
    one kernel does rope + RMSNorm + x1.2 for q and k and writes k, v into the layer's slot at each
    row's position, then the decode attention over the slot.  Returns y (B, T, Hq, D)."""
    T = q.size(1)
    k_cache, v_cache = kv_cache.get_slot_cache(self.kv_slot)
    k_scale, v_scale = kv_cache.get_slot_scales(self.kv_slot)
    ring = kv_cache.slot_ring(self.kv_slot)
    seqlens = kv_cache.cache_seqlens
    rope = self.rope
    kv_cache.check_room(T, rope.cos.size(1))
    if USE_FUSED_APPEND and USE_TORCH_OPS and k_scale is None:
        return _torch_ops().append_attn(q, k if self.produces_kv else None,
                                         v if self.produces_kv else None, k_cache, v_cache, seqlens,
                                         rope.cos, rope.sin, eps=self.norm.eps, scale=1.2,
                                         window=-1 if self.window is None else self.window, ring=ring)
    if USE_FUSED_APPEND:  # one launch where the plan allows it (ops.append_attn), else two
        return ops.append_attn(q, k if self.produces_kv else None, v if self.produces_kv else None,
                               k_cache, v_cache, seqlens, rope.cos, rope.sin, eps=self.norm.eps,
                               scale=1.2, window=self.window, ring=ring, k_scale=k_scale,
                               v_scale=v_scale)
    if self.produces_kv:
        q = ops.kv_append_rope(q, k, v, k_cache, v_cache, seqlens, rope.cos, rope.sin,
                               rotate_q=True, rotate_k=True, write_kv=True, eps=self.norm.eps,
                               scale=1.2, ring=ring, k_scale=k_scale, v_scale=v_scale)
    else:
        q = ops.kv_append_rope(q, None, None, None, None, seqlens, rope.cos, rope.sin,
                               rotate_q=True, rotate_k=False, write_kv=False,
                               eps=self.norm.eps, scale=1.2)
    return ops.decode_attn(q, k_cache, v_cache, seqlens, window=self.window, ring=ring,
                           k_scale=k_scale, v_scale=v_scale)


def attention_forward(self, x, idx, kv_cache, kv_bus=None, doc_args=None):
    """modelcore Attention.forward (modelcore/components/attention.py:135-184) with the KV-cache
    branch on libmcb200.  Same projections, hooks (`values` after c_v, `output` before c_proj),
    window and kv_slot semantics; same state-dict keys.

    Fused mode (RMSNorm QK-norm + RotaryEmbedding): one kernel does rope + norm + x1.2 for q and
    k and writes k, v into the slot at each row's position (a consumer layer, produces_kv=False,
    rotates only its q and reads the producer's slot, which the producer wrote earlier in the
    same forward); then the decode-attention kernel.  Composed mode (any other norm or position
    encoding): the module's own torch ops compute q, k as the reference does, then the insert and
    the attention run on libmcb200.  In both modes kv_bus is not used: consumers read the slot."""
    if kv_cache is None or not isinstance(kv_cache, KVCache):
        return getattr(self, _ORIGINAL_FORWARD)(x, idx, kv_cache, kv_bus, doc_args)
    B, T, C = x.size()
    fused = _fusable(self, x)
    qkv = None
    if fused and self.produces_kv and getattr(self, _FUSE_QKV, False):
        qkv = step.qkv_projection(self, x)  # q, k, v as views of one GEMM's output
    if qkv is not None:
        q, k, v = qkv
    else:
        q = self.c_q(x).view(B, T, self.n_head, self.head_dim)
    k_cache, v_cache = kv_cache.get_slot_cache(self.kv_slot)
    ring = kv_cache.slot_ring(self.kv_slot)
    seqlens = kv_cache.cache_seqlens
    if ring and not fused:
        raise RuntimeError("a window-ring KV cache needs modelcore's RotaryEmbedding + RMSNorm "
                           "attention (the fused append); build the cache without rings")
    if getattr(kv_cache, "kv_format", "bf16") == "fp8" and not fused:
        raise RuntimeError("an fp8 KV cache needs modelcore's RotaryEmbedding + RMSNorm attention "
                           "(the fused append quantizes); build the cache as bf16")
    if fused:
        if self.produces_kv:
            if qkv is None:
                k = self.c_k(x).view(B, T, self.n_kv_head, self.head_dim)
                v = self.c_v(x).view(B, T, self.n_kv_head, self.head_dim)
            v = self._hook("values", v, x, idx)
        else:
            k = v = None
        y = attend(self, q, k, v, kv_cache)
    else:
        kv_cache.check_room(T)
        if self.produces_kv:
            k = self.c_k(x).view(B, T, self.n_kv_head, self.head_dim)
            v = self.c_v(x).view(B, T, self.n_kv_head, self.head_dim)
            v = self._hook("values", v, x, idx)
            q, k = self.rope(q, k, kv_cache)
            q, k = self.norm(q), self.norm(k)
            q = q * 1.2
            k = k * 1.2
            y = flash_attn_with_kvcache(q, k_cache, v_cache, k=k, v=v, cache_seqlens=seqlens,
                                        causal=True, window_size=(self.window, 0))
        else:
            q = self.rope.apply_to_q(q, kv_cache)
            q = self.norm(q)
            q = q * 1.2
            y = flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens=seqlens, causal=True,
                                        window_size=(self.window, 0))
    y = self._hook("output", y, x)
    y = y.contiguous().view(B, T, -1)
    return self.c_proj(y)


def install(model, fuse_step=True):
    """Binds attention_forward to every modelcore Attention module of `model`; returns the
    number of modules changed.  With fuse_step, producer layers project q, k, v with one GEMM
    and, where the model's structure qualifies, the body runs modelcore_b200.step.stack_forward
    (residual add + norm and the gated MLP fused); fuse_step=False keeps modelcore's op-by-op
    forward around the libmcb200 attention.  Idempotent; a second call only changes fuse_step."""
    from modelcore.components.attention import Attention
    n = 0
    for m in model.modules():
        if isinstance(m, Attention):
            if not hasattr(m, _ORIGINAL_FORWARD):
                object.__setattr__(m, _ORIGINAL_FORWARD, m.forward)
                object.__setattr__(m, "forward", types.MethodType(attention_forward, m))
                n += 1
            object.__setattr__(m, _FUSE_QKV, bool(fuse_step))
    if fuse_step:
        step.install(model)
    else:
        step.uninstall(model)
    return n


def uninstall(model):
    from modelcore.components.attention import Attention
    step.uninstall(model)
    for m in model.modules():
        if isinstance(m, Attention) and hasattr(m, _ORIGINAL_FORWARD):
            object.__setattr__(m, "forward", getattr(m, _ORIGINAL_FORWARD))
            object.__delattr__(m, _ORIGINAL_FORWARD)
            object.__delattr__(m, _FUSE_QKV)


def _manager_base():
    from modelcore.manager import ModelManager as RefManager
    return RefManager


RING_CHUNK = 512  # tokens one forward may append to a window ring (longer inputs are chunked)


def ring_config(model, seq_len):
    """The window rings new_kv_cache builds with ring_window on: the slots whose every layer has
    a sliding window, one capacity for all of them (the largest window plus RING_CHUNK, rounded up
    to 128 positions), or none when that is not below seq_len.  Returns (slots, capacity, window)."""
    windows = {}
    for i, spec in enumerate(model.layer_specs()):
        if not hasattr(spec, "window") or not hasattr(spec, "kv_slot"):
            continue  # not an attention layer
        slot = i if spec.kv_slot is None else spec.kv_slot
        windows.setdefault(slot, []).append(spec.window)
    ring = sorted(s for s, ws in windows.items() if all(w is not None and w >= 0 for w in ws))
    if not ring:
        return (), 0, None
    wmax = max(max(windows[s]) for s in ring)
    cap = (wmax + RING_CHUNK + 127) // 128 * 128
    if cap >= seq_len:
        return (), 0, None
    return tuple(ring), cap, wmax


class _ManagerMixin:
    fuse_step = True  # install(model, fuse_step) for the models this manager returns
    # new_kv_cache keeps the slots of sliding-window layers as window rings (see ring_config):
    # cache memory in proportion to the window instead of the sequence length.  Off by default:
    # it needs the fused decode forward (chunked prefill) and is a layout modelcore does not have.
    ring_window = False
    # new_kv_cache's storage: "bf16" (modelcore's layout) or "fp8" (e4m3 with per-vector scales:
    # half the cache memory; an extension with its own parity rules)
    kv_format = "bf16"

    def create_model(self, *args, **kwargs):
        model = super().create_model(*args, **kwargs)
        install(model, fuse_step=self.fuse_step)
        return model

    def load_model(self, *args, **kwargs):
        model = super().load_model(*args, **kwargs)
        install(model, fuse_step=self.fuse_step)
        return model

    def new_kv_cache(self, model, *, batch_size, seq_len, device=None):
        """modelcore's new_kv_cache (modelcore/manager.py:286-291) returning the B200 KVCache
        for CUDA devices; the cache dtype is the model's activation dtype (bf16)."""
        from modelcore.stats import kv_cache_spec
        device = torch.device(device) if device is not None else model.get_device()
        if device.type != "cuda":
            return super().new_kv_cache(model, batch_size=batch_size, seq_len=seq_len, device=device)
        spec = kv_cache_spec(model.layer_specs())
        ring_slots, cap, wmax = ring_config(model, seq_len) if self.ring_window else ((), 0, None)
        if ring_slots and not step.decode_installed(model):
            raise RuntimeError("window rings need the fused decode forward (install with fuse_step)")
        return KVCache(batch_size=batch_size, seq_len=seq_len, device=device, dtype=torch.bfloat16,
                       ring_slots=ring_slots, ring_capacity=cap, ring_window=wmax,
                       kv_format=self.kv_format, **spec)

    def new_decoder(self, model, tokens, *, num_samples=1, max_tokens=None, device=None,
                    cuda_graph=False, batched_prefill=True):
        """modelcore's Decoder (modelcore/generate.py:37-94) over the B200 cache; with
        cuda_graph=True, a GraphDecoder (whose multi-prompt prefill is one batched forward unless
        batched_prefill=False)."""
        if cuda_graph:
            return GraphDecoder(model, self, tokens, num_samples=num_samples, max_tokens=max_tokens,
                                device=device, batched_prefill=batched_prefill)
        from modelcore.generate import Decoder
        return Decoder(model, self, tokens, num_samples=num_samples, max_tokens=max_tokens,
                       device=device)


def make_manager_class():
    return type("ModelManager", (_ManagerMixin, _manager_base()), {
        "__doc__": "modelcore.ModelManager with the B200 KV-cache decode path installed.",
        "__module__": __name__,
    })


class GraphDecoder:
    """modelcore's Decoder (same constructor, .logits, .step, .kv_cache) whose decode steps replay
    one CUDA graph of `model.forward(ids (B, 1), kv_cache)` instead of launching each op from
    Python.  The first step runs eagerly (it warms up cuBLAS and the kernels); the second
    captures the graph; every step after replays it.  The graph holds fixed pointers, so the
    cache must not be reallocated while it lives.

    greedy_steps(n) additionally keeps the argmax on the device: each replay feeds its own
    greedy token to the next step (no host round trip), returning the (B, n) tokens.
    step_greedy(tokens) is step() plus the greedy pick for a caller that drives every step from
    the host: the pinned-memory copy in, the forward, the pick and the pinned-memory copy out are
    one graph, and the call returns the next tokens on the host."""

    def __init__(self, model, manager, tokens, *, num_samples=1, max_tokens=None, device=None,
                 batched_prefill=True):
        self.model = model
        prompts = None if isinstance(tokens[0], int) else [list(p) for p in tokens]
        dev = torch.device(device) if device is not None else model.get_device()
        done = None
        if (batched_prefill and prompts is not None and len(prompts) > 1
                and step.decode_installed(model) and dev.type == "cuda"):
            done = self._batched_prefill(manager, prompts, num_samples, max_tokens, dev)
        if done is not None:
            self.kv_cache, self._logits = done
        else:
            from modelcore.generate import Decoder
            dec = Decoder(model, manager, tokens, num_samples=num_samples, max_tokens=max_tokens,
                          device=device)
            self.kv_cache, self._logits = dec.kv_cache, dec.logits
        if not isinstance(self.kv_cache, KVCache):
            raise RuntimeError("GraphDecoder needs the modelcore_b200 KVCache (a CUDA model)")
        self._graph = None
        self._greedy_graph = None
        self._eager_steps = 0
        B = self.kv_cache.batch_size
        dev = self.kv_cache.cache_seqlens.device
        self._ids = torch.zeros((B, 1), dtype=torch.long, device=dev)
        self._ids_host = torch.zeros((B, 1), dtype=torch.long).pin_memory()
        self._static_logits = None
        self._rt_graph = None
        self._next = torch.zeros((B, 1), dtype=torch.long, device=dev)
        # step_greedy's tokens go out through the same pinned buffer its column comes in by: a
        # caller that feeds the returned tokens straight back (a greedy loop) needs no host copy
        self._next_host = self._ids_host
        self._next_view = self._ids_host.view(-1)
        self._rt_done = torch.cuda.Event()
        # recorded after each step()'s copy out of _ids_host: the next step() waits on it before
        # overwriting that pinned buffer (the copy reads it when the stream reaches it, not when
        # it is enqueued)
        self._h2d_done = torch.cuda.Event()
        self.launches_per_step = None  # libmcb200 kernels recorded in one captured step

    @torch.inference_mode()
    def _batched_prefill(self, manager, prompts, num_samples, max_tokens, dev):
        """Decoder's multi-prompt prefill (modelcore/generate.py:64-79: every prompt prefilled
        alone at batch 1, then prefill_row into its right-ragged row) as one forward: the prompts
        right-padded into a (P, max_len) batch, one pass through the model (the tensor-core
        prefill attention, the projections at M = P x max_len), the LM head only at each prompt's
        last token, then every row cut back to its own length.  A row's padding positions hold
        keys no later query reads (each decode step overwrites the next one).  num_samples > 1
        copies each prompt's row into its samples' rows."""
        model = self.model
        P, S = len(prompts), num_samples
        lens = [len(p) for p in prompts]
        width = max(lens)
        kv_len = (width + max_tokens) if max_tokens is not None else model.config.sequence_len
        cache = manager.new_kv_cache(model, batch_size=P * S, seq_len=kv_len, device=dev)
        ids = torch.zeros((P, width), dtype=torch.long)
        for i, p in enumerate(prompts):
            ids[i, :len(p)] = torch.tensor(p, dtype=torch.long)
        ids = ids.to(dev)
        last = torch.tensor([n - 1 for n in lens], dtype=torch.long, device=dev)
        target = cache if S == 1 else manager.new_kv_cache(model, batch_size=P, seq_len=width,
                                                             device=dev)
        if not step._model_call_ok(model, ids, target):
            return None  # not the fused decode forward's model: modelcore's prefill runs
        target.check_room(width)
        logits = step.decode_forward(model, ids, target, last_positions=last)[:, 0, :]
        target.set_row_lengths(lens)
        if S > 1:
            for i, n in enumerate(lens):
                cache._copy_slots_from(target, i * S, S, n, src_row=i)
            cache.set_row_lengths([n for n in lens for _ in range(S)])
            logits = logits.repeat_interleave(S, dim=0)
        return cache, logits

    @property
    def logits(self):
        return self._logits

    def _room(self, n):
        self.kv_cache.check_room(n)

    def _capture(self, greedy):
        cache = self.kv_cache
        snap = cache.host_state()
        state_snap = dict(cache.state)
        g = torch.cuda.CUDAGraph()
        launches = ops.launch_count()
        with torch.inference_mode():
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            fused_pick = (greedy and step.decode_installed(self.model)
                          and step._model_call_ok(self.model, self._ids, cache))
            with torch.cuda.graph(g, stream=side):
                nxt = None
                if fused_pick:   # the LM-head epilogue writes the greedy ids into _ids
                    logits = step.decode_forward(self.model, self._ids, cache,
                                                 argmax_out=self._ids)[:, -1, :]
                else:
                    logits = self.model.forward(self._ids, kv_cache=cache)[:, -1, :]
                    if greedy:
                        nxt = torch.argmax(logits, dim=-1, keepdim=True)
                        self._ids.copy_(nxt)
            torch.cuda.current_stream().wait_stream(side)
        self.launches_per_step = ops.launch_count() - launches
        cache.restore_host_state(snap)
        cache.state.update(state_snap)
        return g, logits, nxt

    def _capture_sampling(self, temperature, top_k, generator):
        cache = self.kv_cache
        snap = cache.host_state()
        state_snap = dict(cache.state)
        g = torch.cuda.CUDAGraph()
        if generator is not None:
            g.register_generator_state(generator)
        B = cache.batch_size
        with torch.inference_mode():
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.graph(g, stream=side):
                if step.decode_installed(self.model) and step._model_call_ok(self.model, self._ids, cache):
                    logits = step.decode_forward(self.model, self._ids, cache)[:, -1, :]
                else:
                    logits = self.model.forward(self._ids, kv_cache=cache)[:, -1, :].float()
                u = torch.rand(B, generator=generator, dtype=torch.float32, device=self._ids.device)
                ops.sample(logits, u, temperature=temperature, top_k=top_k, out=self._ids)
            torch.cuda.current_stream().wait_stream(side)
        cache.restore_host_state(snap)
        cache.state.update(state_snap)
        return g, logits

    @torch.inference_mode()
    def sample_steps(self, n, *, temperature=1.0, top_k=None, generator=None, first_tokens=None,
                     out=None):
        """n device-resident sampled steps: step i feeds token t_i and draws t_{i+1} from its
        logits with sample_next_token's distribution (modelcore/generate.py:19-34: top_k,
        temperature; one mcb_sample launch on uniforms from `generator`, a CUDA torch.Generator or
        the default one); t_0 = first_tokens (default: drawn from the current logits).  Returns
        out (B, n) int64 holding t_0 .. t_{n-1}; .logits afterwards are those of the last step."""
        from .sampling import sample_next_token
        B = self.kv_cache.batch_size
        if first_tokens is None:
            first_tokens = sample_next_token(self._logits, generator, temperature, top_k)
        self._ids.copy_(first_tokens.view(-1, 1))
        if out is None:
            out = torch.empty((B, n), dtype=torch.long, device=self._ids.device)
        key = (float(temperature), top_k, id(generator))
        graphs = self.__dict__.setdefault("_sample_graphs", {})
        for i in range(n):
            out[:, i] = self._ids[:, 0]
            self._room(1)
            if key not in graphs and self._eager_steps == 0:
                logits = self._eager(self._ids.clone())
                self._ids.copy_(sample_next_token(logits, generator, temperature, top_k))
                self._logits = logits
                continue
            if key not in graphs:
                graphs[key] = self._capture_sampling(temperature, top_k, generator)
            graph, logits = graphs[key]
            graph.replay()
            self._replayed()
            self._logits = logits
        return out

    def _capture_roundtrip(self):
        cache = self.kv_cache
        snap = cache.host_state()
        state_snap = dict(cache.state)
        g = torch.cuda.CUDAGraph()
        with torch.inference_mode():
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            fused_pick = step.decode_installed(self.model) and step._model_call_ok(self.model, self._ids, cache)
            with torch.cuda.graph(g, stream=side):
                self._ids.copy_(self._ids_host, non_blocking=True)
                if fused_pick:
                    logits = step.decode_forward(self.model, self._ids, cache,
                                                 argmax_out=self._next)[:, -1, :]
                else:
                    logits = self.model.forward(self._ids, kv_cache=cache)[:, -1, :]
                    self._next.copy_(torch.argmax(logits, dim=-1, keepdim=True))
                self._next_host.copy_(self._next, non_blocking=True)
            torch.cuda.current_stream().wait_stream(side)
        cache.restore_host_state(snap)
        cache.state.update(state_snap)
        return g, logits

    @torch.inference_mode()
    def step_greedy(self, token_column):
        """step(token_column), then the greedy pick of the new logits (sample_next_token with
        temperature 0, modelcore/generate.py:23-24): returns the (B,) next tokens as a host int64
        tensor (a view of pinned memory, valid until the next call).  The host-to-device copy of
        the column, the decode forward with the pick fused into the LM-head epilogue and the
        device-to-host copy of the tokens replay as one CUDA graph.  The tokens come back in the
        pinned buffer the next column goes in by: passing the returned tensor itself as the next
        column skips the host copy."""
        self._room(1)
        if token_column is not self._next_view:
            self._h2d_done.synchronize()  # a step() may still be copying out of the buffer
            self._ids_host.copy_(torch.as_tensor(token_column, dtype=torch.long).view(-1, 1))
        if self._rt_graph is None and self._eager_steps == 0:
            self._ids.copy_(self._ids_host, non_blocking=True)
            self._logits = self._eager(self._ids.clone())
            self._next_host.copy_(torch.argmax(self._logits, dim=-1, keepdim=True).cpu())
            return self._next_view
        if self._rt_graph is None:
            self._rt_graph, self._rt_logits = self._capture_roundtrip()
        self._rt_graph.replay()
        self._replayed()
        self._rt_done.record()
        self._rt_done.synchronize()
        self._logits = self._rt_logits
        return self._next_view

    def _eager(self, ids):
        logits = self.model.forward(ids, kv_cache=self.kv_cache)[:, -1, :]
        self._eager_steps += 1
        return logits

    def _replayed(self):
        cache = self.kv_cache
        cache._host_lens += 1
        if cache._pos_uniform is not None:
            cache._pos_uniform += 1

    @torch.inference_mode()
    def step(self, token_column):
        """Advance every row by one position; returns the new (B, vocab) logits."""
        self._room(1)
        if isinstance(token_column, torch.Tensor) and token_column.is_cuda:
            self._ids.copy_(token_column.view(-1, 1))
        else:
            self._h2d_done.synchronize()
            self._ids_host.copy_(torch.as_tensor(token_column, dtype=torch.long).view(-1, 1))
            self._ids.copy_(self._ids_host, non_blocking=True)
            self._h2d_done.record()
        if self._graph is None and self._eager_steps == 0:
            self._logits = self._eager(self._ids.clone())
            return self._logits
        if self._graph is None:
            self._graph, self._static_logits, _ = self._capture(greedy=False)
        self._graph.replay()
        self._replayed()
        self._logits = self._static_logits
        return self._logits

    @torch.inference_mode()
    def greedy_steps(self, n, first_tokens=None, out=None):
        """n device-resident greedy steps.  Step i feeds token t_i and computes
        t_{i+1} = argmax(logits); t_0 = first_tokens (default: argmax of the current logits).
        Returns out (B, n) int64 on the device holding t_0 .. t_{n-1}, the same stream modelcore's
        greedy loop produces; .logits afterwards are those of the last step."""
        B = self.kv_cache.batch_size
        if first_tokens is None:
            first_tokens = torch.argmax(self._logits, dim=-1)
        self._ids.copy_(first_tokens.view(-1, 1))
        if out is None:
            out = torch.empty((B, n), dtype=torch.long, device=self._ids.device)
        for i in range(n):
            out[:, i] = self._ids[:, 0]
            self._room(1)
            if self._greedy_graph is None and self._eager_steps == 0:
                logits = self._eager(self._ids.clone())
                self._ids.copy_(torch.argmax(logits, dim=-1, keepdim=True))
                self._logits = logits
                continue
            if self._greedy_graph is None:
                self._greedy_graph, self._greedy_logits, _ = self._capture(greedy=True)
            self._greedy_graph.replay()
            self._replayed()
            self._logits = self._greedy_logits
        return out
