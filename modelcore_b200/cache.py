"""KVCache for the B200 decode path: modelcore's KVCache API and layout over libmcb200 kernels.

Same constructor, attributes and methods as modelcore.cache.KVCache (modelcore/cache.py:13-119):
k_cache / v_cache (n_slots, B, T_max, H_kv, D), cache_seqlens (B,) int32, state, reset, get_pos,
uniform_pos, get_slot_cache, advance, prefill, prefill_row -- so modelcore's Model, Decoder and
Attention use it unchanged.  Differences, all on the host side:

* Layout (piece 4 of the decode path): bf16 on a CUDA device only, base addresses 256-byte
  aligned (every (slot, row, position) vector then starts on a 16-byte boundary, which the TMA
  loads of the attention kernel require).  Anything else raises: there is no CPU path.
* A host mirror of every row's length (`_host_lens`) is kept by this class's own methods, so
  prefill_row's checks and the overflow checks never read cache_seqlens back (the reference syncs
  at modelcore/cache.py:102 and :118).  As in the reference, only KVCache's own methods may
  mutate cache_seqlens.
* prefill / prefill_row copy with one kernel that also sets cache_seqlens for the rows it fills.
"""
import numpy as np
import torch

from . import _native, ops

CACHE_ALIGN = 256


def _aligned_zeros(shape, device, dtype=torch.bfloat16):
    t = torch.zeros(shape, dtype=dtype, device=device)
    if t.numel() and t.data_ptr() % CACHE_ALIGN:
        raise RuntimeError(f"KV cache base {t.data_ptr():#x} is not {CACHE_ALIGN}-byte aligned")
    return t


class KVCache:
    """modelcore.cache.KVCache on the B200 layout.  ring_slots / ring_capacity: optional window
    rings -- slots read only by sliding-window layers keep ring_capacity positions (a multiple of
    128, below seq_len), position p at index p % ring_capacity, instead of seq_len; step_limit is
    then the most tokens one forward may append (ring_capacity minus the largest window of those
    layers), so every key a query can see is still resident.  The full-length slots stay in
    k_cache / v_cache, the rings in k_ring / v_ring; get_slot_cache and slot_ring resolve a slot.

    kv_format "fp8" (an extension; the reference stores the compute dtype) keeps every slot as
    float8 e4m3 with one fp32 scale per (row, position, kv head) vector -- half the bytes a key
    costs -- in k_scale / v_scale (n_slots, B, H_kv, T_max rounded up to 64) and k_ring_scale /
    v_ring_scale; get_slot_scales resolves them (None, None for bf16).  The fused append
    quantizes each new vector, the attention reads e4m3 x scale; head_dim 64 or 128."""

    def __init__(self, batch_size, n_kv_head, seq_len, head_dim, num_kv_slots, device, dtype,
                 ring_slots=(), ring_capacity=0, ring_window=None, kv_format="bf16"):
        _native.load()
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError(f"modelcore_b200.KVCache lives on a CUDA device, got {device}")
        if dtype != torch.bfloat16:
            raise RuntimeError(f"modelcore_b200.KVCache stores bf16, got {dtype}")
        if num_kv_slots and (head_dim % 8):
            raise RuntimeError(f"head_dim {head_dim} must be a multiple of 8 (16-byte cache rows)")
        if kv_format not in ("bf16", "fp8"):
            raise RuntimeError(f"kv_format must be 'bf16' or 'fp8', got {kv_format!r}")
        if kv_format == "fp8" and num_kv_slots and head_dim not in (64, 128):
            raise RuntimeError(f"an fp8 KV cache needs head_dim 64 or 128, got {head_dim}")
        self.kv_format = kv_format
        self.batch_size = batch_size
        self.max_seq_len = seq_len
        self.n_slots = num_kv_slots
        self.n_kv_head = n_kv_head
        self.head_dim = head_dim
        ring = sorted(set(int(x) for x in ring_slots)) if 0 < ring_capacity < seq_len else []
        if ring:
            assert ring_capacity % 128 == 0, "ring capacity must be a multiple of 128 positions"
            assert ring_window is not None and 0 <= ring_window < ring_capacity, \
                "a window ring needs the largest window of its layers, below the capacity"
        full = [x for x in range(num_kv_slots) if x not in ring]
        self._slots = {x: (False, i) for i, x in enumerate(full)}
        self._slots.update({x: (True, i) for i, x in enumerate(ring)})
        self.ring_capacity = ring_capacity if ring else 0
        self.step_limit = ring_capacity - ring_window if ring else None
        store = ops.FP8 if kv_format == "fp8" else torch.bfloat16
        self.k_cache = _aligned_zeros((len(full), batch_size, seq_len, n_kv_head, head_dim), device, store)
        self.v_cache = _aligned_zeros((len(full), batch_size, seq_len, n_kv_head, head_dim), device, store)
        rshape = (len(ring), batch_size, self.ring_capacity, n_kv_head, head_dim)
        self.k_ring = _aligned_zeros(rshape, device, store)
        self.v_ring = _aligned_zeros(rshape, device, store)
        self.k_scale = self.v_scale = self.k_ring_scale = self.v_ring_scale = None
        if kv_format == "fp8":
            self.k_scale = ops.fp8_scales(batch_size, n_kv_head, seq_len, device, n_slots=len(full))
            self.v_scale = torch.zeros_like(self.k_scale)
            self.k_ring_scale = ops.fp8_scales(batch_size, n_kv_head, self.ring_capacity, device,
                                               n_slots=len(ring))
            self.v_ring_scale = torch.zeros_like(self.k_ring_scale)
        self.cache_seqlens = torch.zeros(batch_size, dtype=torch.int32, device=device)
        self._pos_uniform = 0
        self._host_lens = np.zeros(batch_size, dtype=np.int64)
        self.state = {}

    # -- the reference API -------------------------------------------------------------------
    def reset(self):
        """Rows back to length 0; k/v are not zeroed (stale KV is unreachable: every kernel masks
        keys beyond a row's own position), as in modelcore/cache.py:38-45."""
        self.cache_seqlens.zero_()
        self.state = {}
        self._pos_uniform = 0
        self._host_lens[:] = 0

    def get_pos(self):
        assert self._pos_uniform is not None, \
            "get_pos() on a right-ragged KV cache; read cache_seqlens or check uniform_pos()"
        return self._pos_uniform

    def uniform_pos(self):
        return self._pos_uniform

    def get_slot_cache(self, slot):
        is_ring, i = self._slots[slot]
        if is_ring:
            return self.k_ring[i], self.v_ring[i]
        return self.k_cache[i], self.v_cache[i]

    def slot_ring(self, slot):
        """True when `slot` is a window ring (position p at index p % ring_capacity)."""
        return self._slots[slot][0]

    def get_slot_scales(self, slot):
        """The fp8 slot's (k_scale, v_scale), (B, H_kv, T_max rounded up to 64) each; (None, None)
        for a bf16 cache."""
        if self.kv_format != "fp8":
            return None, None
        is_ring, i = self._slots[slot]
        if is_ring:
            return self.k_ring_scale[i], self.v_ring_scale[i]
        return self.k_scale[i], self.v_scale[i]

    def cache_bytes(self):
        """Device bytes of the K and V storage (and the fp8 scales)."""
        n = 2 * (self.k_cache.numel() + self.k_ring.numel()) * self.k_cache.element_size()
        if self.kv_format == "fp8":
            n += 2 * (self.k_scale.numel() + self.k_ring_scale.numel()) * 4
        return n

    def _copy_slots_from(self, other, dst_row_begin, dst_row_count, n_pos, src_row=0):
        """Positions [0, n_pos) of other's row src_row into rows [dst_row_begin, +count), every
        slot, ring or not; cache_seqlens of those rows set to n_pos."""
        assert self.kv_format == other.kv_format, "prefill between caches of different formats"
        same_layout = (not self.ring_capacity and not other.ring_capacity)
        if same_layout:
            ops.kv_copy_rows(self.k_cache, self.v_cache, other.k_cache, other.v_cache, src_row=src_row,
                             dst_row_begin=dst_row_begin, dst_row_count=dst_row_count, n_pos=n_pos,
                             dst_seqlens=self.cache_seqlens)
            if self.kv_format == "fp8":
                self._copy_scales(self.k_scale, self.v_scale, other.k_scale, other.v_scale, src_row,
                                  dst_row_begin, dst_row_count, n_pos)
            return
        for slot in range(self.n_slots):
            d_ring, di = self._slots[slot]
            s_ring, si = other._slots[slot]
            dk, dv = (self.k_ring, self.v_ring) if d_ring else (self.k_cache, self.v_cache)
            sk, sv = (other.k_ring, other.v_ring) if s_ring else (other.k_cache, other.v_cache)
            n = n_pos
            if d_ring:
                assert s_ring and other.ring_capacity == self.ring_capacity or n_pos <= self.ring_capacity, \
                    "a window ring takes a longer prompt only from a ring of the same capacity"
                n = min(n_pos, self.ring_capacity)  # a ring holds positions p at p % capacity
            else:
                assert not s_ring, "a full-length slot cannot be filled from a window ring"
            ops.kv_copy_rows(dk[di:di + 1], dv[di:di + 1], sk[si:si + 1], sv[si:si + 1],
                             src_row=src_row, dst_row_begin=dst_row_begin,
                             dst_row_count=dst_row_count, n_pos=n, dst_seqlens=None)
            if self.kv_format == "fp8":
                dks, dvs = (self.k_ring_scale, self.v_ring_scale) if d_ring else (self.k_scale, self.v_scale)
                sks, svs = (other.k_ring_scale, other.v_ring_scale) if s_ring else (other.k_scale, other.v_scale)
                self._copy_scales(dks[di:di + 1], dvs[di:di + 1], sks[si:si + 1], svs[si:si + 1], src_row,
                                  dst_row_begin, dst_row_count, n)
        self.cache_seqlens[dst_row_begin:dst_row_begin + dst_row_count] = n_pos

    @staticmethod
    def _copy_scales(dk, dv, sk, sv, src_row, dst_row_begin, dst_row_count, n_pos):
        """The fp8 scales of positions [0, n_pos) of row src_row into the destination rows."""
        rows = slice(dst_row_begin, dst_row_begin + dst_row_count)
        dk[:, rows, :, :n_pos] = sk[:, src_row:src_row + 1, :, :n_pos]
        dv[:, rows, :, :n_pos] = sv[:, src_row:src_row + 1, :, :n_pos]

    def advance(self, num_tokens):
        """cache_seqlens += num_tokens on the device, and the host mirrors with it
        (modelcore/cache.py:62-73)."""
        ops.kv_advance(self.cache_seqlens, num_tokens)
        self._host_lens += num_tokens
        if self._pos_uniform is not None:
            self._pos_uniform += num_tokens

    def prefill(self, other):
        """Broadcast a batch-1 cache into every row (modelcore/cache.py:75-90): one kernel reads
        the source once, writes it to all rows and sets cache_seqlens."""
        assert self.get_pos() == 0, "Cannot prefill a non-empty KV cache"
        assert self.n_slots == other.n_slots and self.n_kv_head == other.n_kv_head and self.head_dim == other.head_dim
        assert self.max_seq_len >= other.max_seq_len
        other_pos = other.get_pos()
        if self.n_slots:
            self._copy_slots_from(other, 0, self.batch_size, other_pos)
        else:
            self.cache_seqlens.fill_(other_pos)
        self._pos_uniform = other_pos
        self._host_lens[:] = other_pos
        for key, value in other.state.items():
            self.state[key] = value.expand(self.batch_size, *([-1] * (value.dim() - 1))).clone()

    def prefill_row(self, row, other):
        """Copy a batch-1 prefilled cache into row `row` (modelcore/cache.py:92-119), checked
        against the host mirror instead of a device read."""
        assert other.batch_size == 1, "prefill_row copies from a batch=1 cache"
        assert 0 <= row < self.batch_size, f"row {row} out of range for batch_size {self.batch_size}"
        assert self._host_lens[row] == 0, "Cannot prefill a non-empty KV cache row"
        assert self.n_slots == other.n_slots and self.n_kv_head == other.n_kv_head and self.head_dim == other.head_dim
        other_pos = other.get_pos()
        assert other_pos <= self.max_seq_len, f"prompt of {other_pos} tokens exceeds cache length {self.max_seq_len}"
        if self.n_slots:
            self._copy_slots_from(other, row, 1, other_pos)
        else:
            self.cache_seqlens[row] = other_pos
        for key, value in other.state.items():
            buf = self.state.get(key)
            if buf is None:
                buf = value.new_zeros((self.batch_size,) + tuple(value.shape[1:]))
                self.state[key] = buf
            buf[row] = value[0]
        self._host_lens[row] = other_pos
        lens = self._host_lens
        self._pos_uniform = int(lens[0]) if bool((lens == lens[0]).all()) else None

    def set_row_lengths(self, lengths):
        """Sets every row's length (device and host mirror): after a batched ragged prefill that
        advanced all rows by the padded prompt length, each row keeps only its own prompt.
        Positions past a row's length hold stale keys the attention never reads."""
        lens = np.asarray(lengths, dtype=np.int64)
        assert lens.shape == (self.batch_size,), "one length per row"
        assert int(lens.max(initial=0)) <= self.max_seq_len, "length beyond the cache"
        self.cache_seqlens.copy_(torch.from_numpy(lens.astype(np.int32)), non_blocking=False)
        self._host_lens[:] = lens
        self._pos_uniform = int(lens[0]) if lens.size and bool((lens == lens[0]).all()) else None

    # -- host-side helpers ---------------------------------------------------------------------
    def host_lens(self):
        """Row lengths as this cache's methods have set them (no device read)."""
        return self._host_lens.copy()

    def max_len(self):
        return int(self._host_lens.max()) if self.batch_size else 0

    def check_room(self, num_tokens, rot_len=None):
        """Raises before a step that would write past T_max or past the rotary table (the
        reference asserts the latter at modelcore/components/rotary.py:55 and :62)."""
        end = self.max_len() + num_tokens
        assert end <= self.max_seq_len, \
            f"KV cache overflow: positions up to {end} > cache length {self.max_seq_len}"
        if rot_len is not None:
            assert end <= rot_len, \
                f"Sequence length grew beyond the rotary embeddings cache: {end} > {rot_len}"

    def host_state(self):
        """Snapshot of the host mirrors (used around CUDA-graph capture, which records kernels
        without running them)."""
        return (self._host_lens.copy(), self._pos_uniform)

    def restore_host_state(self, snap):
        self._host_lens[:] = snap[0]
        self._pos_uniform = snap[1]
