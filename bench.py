"""Decode benchmark of modelcore's KV-cache path on B200: tokens/s and KV-read HBM GB/s.

    python bench.py [--gpus N --steps K --warmup W]            # this implementation
    python bench.py --impl reference [--steps K --warmup W]    # the reference on the host CPU
    torchrun --nproc-per-node N bench.py --gpus N ...           # N > 1: one rank per GPU

Workload (measurement config 2): modelcore's README quickstart architecture (12 blocks, n_embd
768, 12 q / 12 kv heads of 64, gated SiLU MLP 2048, vocab 32768) with bf16 random-init weights
(seed 0); 64 prompts per GPU of 512 tokens uniform in [0, 32768) (seed 1); KV cache of 1024
positions; prefill through modelcore's Decoder, then greedy decode.  A step is one decode step of
all 64 rows (every layer, the LM head and the greedy pick).  Scaling is weak: every rank decodes
its own 64 rows (rows r*64 .. r*64+63 of one seeded 64*N-prompt batch) with no collective on the
hot path; the sampled tokens are gathered with NCCL at the end of the timed region.

value      64*N*K / max-over-ranks(device time of K CUDA-graph replays), tokens/s; the graph
           feeds each step's greedy token to the next on the device.
e2e        the same through the public step_greedy() call: per step a pinned host->device copy of the
           token column, the replayed step, and the device->host read of the greedy tokens; over
           the same contexts as `value` (the rows are rewound to where the timed steps began).
roofline   the decode-attention kernel: algorithmic KV bytes (exact keys per row and layer,
           2*Hkv*D*2 bytes each) / its mean launch time, timed with CUDA events on its stream
           over the 12 cache slots in rotation (1.6 GB, far above L2), against the measured HBM
           copy bandwidth in MEASURED_PEAKS.json.
kv_read_sweep  measurement config 5 (32 q / 8 kv heads of 128, lengths U[1, 32768] from seed 5,
           window -1 / 4096): one step = fused rope append + decode attention, timed on the device
           in CUDA graphs of consecutive steps on rotating groups of cache rows (no launch finds
           its keys in L2).  On N GPUs each batch is partitioned over the ranks (B / N rows each,
           balanced by length); time = max over ranks, bytes = sum.
kv_read_sweep_fp8  the same over an fp8 (e4m3) cache with per-vector scales (an opt-in cache
           format: bytes = e4m3 keys and values + fp32 scales), with the speed-up over bf16 (N=1).
gqa_decode measurement configs 3 and 4 (the 24 x 2048 GQA model with windows; config 4 with
           cross-layer KV sharing, a broadcast prefill and top-k sampling): a bounded sample of
           their decode steps through ModelManager, tokens/s and the KV bytes read per second; on
           N GPUs config 3's 128 rows and config 4's 256 rows are sharded over the ranks (strong
           scaling) and the timed region ends with the token gather.
kv_copies  (N=1) the broadcast prefill copy, the per-step append and the append of whole prompts
           (config 2's 64 x 512 tokens, config 3's 8,192) against the HBM copy roofline.
cpu_baseline   the reference's own code (modelcore, SDPA path, fp32) on the host cores, a bounded
           sample of the same workload (rank 0, N = 1); cpu_baseline_config5 the reference's
           flash_attn_with_kvcache on config 5 at batch 8; cpu_baseline_configs34 the reference's
           Decoder on configs 3 (one row of the mean context) and 4 (two rows), per-row tokens/s
           and KV GB/s.
reference_on_b200  (N=1) the reference's own decode path (modelcore's Decoder, KVCache and
           flash_attn_with_kvcache, its SDPA path, bf16) on the same GPU and config-2 rows.

Output: rank 0 prints every measurement but the headline as its own JSON line
{"bench_extra": name, "n_gpus": N, "data": ...}, then the headline line last (compact, with a
summary of the extras: kv_read_sweep_frac, gqa_decode_tokens_per_s, prefill_append_frac,
reference_on_b200_tokens_per_s).
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    # NCCL's init lines (one per rank, with the communicator's rank count) stay in the log, so a
    # reader of the run can count the ranks that joined.  A preset level below INFO (the GPU
    # boxes' environment sets VERSION, which prints one version line and no rank) is raised to
    # INFO, limited to the INIT subsystem unless the caller chose subsystems.  Set before torch
    # loads NCCL, which reads them once.
    if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
        os.environ["NCCL_DEBUG"] = "INFO"
    os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

ROWS_PER_GPU = 64
PROMPT_LEN = 512
DECODE_LEN = 512
CPU_SAMPLE_ROWS = 8
FALLBACK_HBM_GBS = 6650.0
# From an ncu capture of the split decode-attention kernel on config 2 (context 516):
NCU_READ_BYTES_PER_TILE_D64 = 16402   # 113.37 MB read / 6,912 fetched tiles
NCU_WRITE_BYTES_CFG2 = 3_500_000       # mean of the two captured launches
METRIC = "decode tokens/sec + KV-read HBM GB/s (% of peak) at 1/2/4/8 B200"


def _ensure_modelcore():
    try:
        import modelcore  # noqa: F401
    except ImportError:
        ref = os.path.join(REPO, "baseline", "_ref")
        if os.path.isdir(ref):
            sys.path.append(ref)
        import modelcore  # noqa: F401


def _bf16_peak():
    """Dense bf16 TFLOP/s measured on this pool (burst: a kernel timed alone), else fallback."""
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["bf16_tflops"])
    except Exception:
        return 1590.0


def _peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------------------------
# clocks during the timed region
class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id):
        self.gpu_id = gpu_id
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "25", "-i", str(self.gpu_id)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def mark(self, which):
        """Records the host time at which the timed region starts ('start') or ends ('end');
        the summary keeps the samples taken between the two marks (all, if too few)."""
        setattr(self, which, time.time())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        lo, hi = getattr(self, "start", 0.0), getattr(self, "end", float("inf"))
        inside = [ln for t, ln in self.lines if lo <= t <= hi + 0.05]
        if len(inside) < 3:
            inside = [ln for _, ln in self.lines]
        for line in inside:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                sm.append(float(parts[2]))
                mx = float(parts[3])
            except ValueError:
                continue
            for name, val in zip(names, parts[6:10]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------------------------
def _dist_setup(n_gpus):
    import datetime
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
        # every rank counts the communicator's members with one all_reduce and says so on stderr,
        # beside NCCL's own init lines
        t = torch.ones(1, device="cuda")
        dist.all_reduce(t)
        n = int(t.item())
        print(f"bench: rank {rank} of {world} on cuda:{local}: an NCCL all_reduce over the process group "
              f"counted {n} ranks", file=sys.stderr, flush=True)
        if n != world:
            raise SystemExit(f"the NCCL communicator holds {n} ranks, WORLD_SIZE={world}")
    return rank, world, local


def _max_over_ranks(x, world):
    import torch
    import torch.distributed as dist
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def _build_decoder(rank, world, steps_needed, fuse_step=True):
    import torch
    import modelcore_b200
    from modelcore_b200 import workloads
    mgr = modelcore_b200.ModelManager()
    mgr.fuse_step = fuse_step
    model = mgr.create_model(workloads.quickstart_config(), device=torch.device("cuda"), seed=0)
    model = model.to(torch.bfloat16).eval()
    from modelcore_b200.sharding import contiguous_rows
    all_prompts = workloads.prompts(ROWS_PER_GPU * world, PROMPT_LEN, seed=1)
    begin, end = contiguous_rows(ROWS_PER_GPU * world, world, rank)
    mine = all_prompts[begin:end].tolist()
    with torch.inference_mode():
        # one warm-up prefill of the same prompts and cache (kernel modules, cuBLAS heuristics for
        # these shapes, the allocator's blocks), then the timed one
        warm = mgr.new_decoder(model, mine, max_tokens=DECODE_LEN, cuda_graph=True)
        del warm
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        dec = mgr.new_decoder(model, mine, max_tokens=DECODE_LEN, cuda_graph=True)
        torch.cuda.synchronize()
        dec.prefill_ms = (time.perf_counter() - t0) * 1e3
    assert steps_needed <= DECODE_LEN, "more decode steps than the configured 512"
    return mgr, model, dec


def _per_prompt_prefill_ms(mgr, model, prompts):
    """The same prefill the reference's Decoder does (every prompt alone at batch 1, then
    prefill_row), on the B200 kernels: wall time in ms."""
    import torch
    with torch.inference_mode():
        # warm-up: the batch-1 shapes of this order (cuBLAS heuristics, kernel modules)
        warm = mgr.new_decoder(model, prompts[:2], max_tokens=DECODE_LEN, cuda_graph=True,
                               batched_prefill=False)
        del warm
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        mgr.new_decoder(model, prompts, max_tokens=DECODE_LEN, cuda_graph=True, batched_prefill=False)
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) * 1e3


def _attention_roofline(dec, peak, reps=4):
    """Mean device time of the decode-attention kernel on the bench's own cache (its current
    lengths): the 12 per-slot launches of one step are captured in a CUDA graph (so host launch
    cost is not timed) and replayed `reps` times between CUDA events on the replay stream; the
    12 slots hold 1.6 GB, far above L2.  Algorithmic bytes = exact keys x 2 x Hkv x D x 2.
    `kernel` is the template instance the library reports for these launches."""
    import torch
    from modelcore_b200 import ops
    cache = dec.kv_cache
    B, H, D, S = cache.batch_size, cache.n_kv_head, cache.head_dim, cache.n_slots
    q = torch.randn(B, 1, H, D, device="cuda").to(torch.bfloat16)
    lens = cache.host_lens()
    keys = int(sum(L + 1 for L in lens))
    bytes_per_launch = keys * 2 * H * D * 2
    out = torch.empty_like(q)
    for s in range(S):  # warm (allocates the cached workspace outside the capture)
        ops.decode_attn(q, cache.k_cache[s], cache.v_cache[s], cache.cache_seqlens, out=out)
    torch.cuda.synchronize()
    kernel = ops.last_attn_kernel()
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.graph(g, stream=side):
        for s in range(S):
            ops.decode_attn(q, cache.k_cache[s], cache.v_cache[s], cache.cache_seqlens, out=out)
    torch.cuda.current_stream().wait_stream(side)
    g.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * S)
    del g
    gbs = bytes_per_launch / (us * 1e-6) / 1e9
    # DRAM traffic per launch, scaled from an ncu capture of this kernel on this model (a shorter
    # context): NCU_READ_BYTES_PER_TILE_D64 read per fetched 64-key tile of one kv head (K and V)
    # plus NCU_WRITE_BYTES_CFG2 written (the outputs), times the tiles this launch fetches
    tiles = int(sum((L + 1 + 63) // 64 for L in lens)) * H
    traffic = tiles * NCU_READ_BYTES_PER_TILE_D64 + NCU_WRITE_BYTES_CFG2
    return {"bytes_per_launch": bytes_per_launch, "us_per_launch": us, "achieved_gbs": gbs,
            "frac": gbs / peak, "mean_context": keys / B, "traffic": traffic, "kernel": kernel,
            "tiles": tiles}


def _sum_over_ranks(x, world):
    import torch
    import torch.distributed as dist
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def _sweep_rows(B, rank, world):
    """Config 5's B rows (lengths U[1, 32768] from seed 5, each row's position = length - 1) and
    the ones this rank decodes: all of them on one GPU; with world > 1 an equal share balanced
    by length (sharding.balanced_rows)."""
    import numpy as np
    from modelcore_b200.sharding import balanced_rows
    lens = np.random.default_rng(5).integers(1, 32769, size=B) - 1
    if world == 1:
        return lens, lens
    mine = balanced_rows(lens.tolist(), world, equal_counts=True)[rank]
    return lens, lens[mine]


def _kv_read_sweep(peak, batches=(1, 8, 64, 256, 512), windows=(-1, 4096), fp8=False, rank=0,
                   world=1):
    """Config 5: fused rope append + decode attention per step.  Each (batch, window) point is
    timed on the device in a CUDA graph of consecutive steps, each on a different group of cache
    rows (kc[g*B:(g+1)*B]) so that no launch finds its keys in L2 (the groups cycled through hold
    more than the 126 MB L2 between two visits); attention alone and append + attention.
    fp8: the same over an e4m3 cache with per-vector scales (bytes = e4m3 keys and values plus
    their fp32 scales).
    world > 1: the batch is partitioned over the ranks (each decodes B / world rows, an equal
    share balanced by length; batches not divisible by world are skipped); a point's time is
    the max over ranks, its bytes the sum, its fraction against world x the per-GPU peak."""
    import torch
    from modelcore_b200 import ops
    Hq, Hkv, D, Tmax = 32, 8, 128, 32769
    stream = torch.cuda.current_stream()
    g = torch.Generator(device="cuda").manual_seed(5 + rank)
    batches = [B for B in batches if B % world == 0]
    rows = []
    if not batches:
        return rows
    max_b = max(batches) // world
    kc = torch.empty(max_b, Tmax, Hkv, D, device="cuda", dtype=ops.FP8 if fp8 else torch.bfloat16)
    vc = torch.empty_like(kc)
    for c in (kc, vc):
        for r in range(0, max_b, 8):   # a few rows at a time (an fp32 draw of all would not fit)
            c[r:r + 8] = torch.randn(c[r:r + 8].shape, device="cuda", generator=g).to(c.dtype)
    kscl = vscl = None
    if fp8:
        kscl = torch.ones(max_b, Hkv, ops.fp8_scale_tmax(Tmax), device="cuda", dtype=torch.float32)
        vscl = torch.ones_like(kscl)
    per_key = 2 * Hkv * (D + 4) if fp8 else 2 * Hkv * D * 2
    ang = torch.arange(Tmax + 1, device="cuda", dtype=torch.float32)[:, None] * \
        (100000.0 ** (-torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))[None]
    cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)

    def graph_us(fn, n):
        fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.graph(gr, stream=side):
            fn()
        stream.wait_stream(side)
        gr.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(3):
            gr.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del gr
        return e0.elapsed_time(e1) * 1e3 / (3 * n)

    for B in batches:
        _, lens = _sweep_rows(B, rank, world)
        b = int(lens.size)
        sl = torch.from_numpy(lens).to(torch.int32).cuda()
        q = torch.randn(b, 1, Hq, D, device="cuda", generator=g, dtype=torch.bfloat16)
        k = torch.randn(b, 1, Hkv, D, device="cuda", generator=g, dtype=torch.bfloat16)
        v = torch.randn(b, 1, Hkv, D, device="cuda", generator=g, dtype=torch.bfloat16)
        groups = max(1, min(16, max_b // b))
        kcs = [kc[i * b:(i + 1) * b] for i in range(groups)]
        vcs = [vc[i * b:(i + 1) * b] for i in range(groups)]
        kss = [kscl[i * b:(i + 1) * b] if fp8 else None for i in range(groups)]
        vss = [vscl[i * b:(i + 1) * b] if fp8 else None for i in range(groups)]
        for w in windows:
            keys = int(sum((L + 1) if w < 0 else min(L + 1, w + 1) for L in lens))
            nbytes = _sum_over_ranks(keys * per_key, world)
            torch.cuda.nvtx.range_push(f"sweep_b{B}_w{w}{'_fp8' if fp8 else ''}")
            qr = ops.kv_append_rope(q, k, v, kcs[0], vcs[0], sl, cos, sin, k_scale=kss[0], v_scale=vss[0])
            out = torch.empty_like(qr)
            n = 4 * groups

            def attn_only():
                for i in range(n):
                    j = i % groups
                    ops.decode_attn(qr, kcs[j], vcs[j], sl, window=w, out=out, k_scale=kss[j], v_scale=vss[j])

            def step():
                for i in range(n):
                    j = i % groups
                    qi = ops.kv_append_rope(q, k, v, kcs[j], vcs[j], sl, cos, sin, q_out=qr,
                                            k_scale=kss[j], v_scale=vss[j])
                    ops.decode_attn(qi, kcs[j], vcs[j], sl, window=w, out=out, k_scale=kss[j], v_scale=vss[j])

            _barrier(world)
            ta = _max_over_ranks(graph_us(attn_only, n), world)
            ts = _max_over_ranks(graph_us(step, n), world)
            torch.cuda.nvtx.range_pop()
            gbs = nbytes / (ta * 1e-6) / 1e9
            row = {"batch": B, "window": w, "mean_keys": round(nbytes / per_key / B, 1),
                   "attn_us": round(ta, 1), "step_us": round(ts, 1),
                   "kv_gbs": round(gbs, 1), "frac": round(gbs / (peak * world), 3)}
            if world > 1:
                row["rows_per_gpu"] = b
            rows.append(row)
    del kc, vc, kscl, vscl
    torch.cuda.empty_cache()
    return rows


def _with_speedup(rows8, rows16):
    """The fp8 sweep rows with the attention speed-up over the bf16 cache at the same point."""
    base = {(r["batch"], r["window"]): r["attn_us"] for r in rows16}
    out = []
    for r in rows8:
        r = dict(r)
        b = base.get((r["batch"], r["window"]))
        r["speedup_vs_bf16"] = round(b / r["attn_us"], 2) if b else None
        out.append(r)
    return out


def _gqa_decode(config, peak, steps=64, rank=0, world=1):
    """Configs 3 and 4, a bounded sample of their decode runs (the full runs are 1024 and 256
    steps): the 24-block GQA model (16 q / 4 kv heads of 128, windows of 1024 on three layers of
    four), bf16 random-init weights (seed 0), through ModelManager and the CUDA-graph decoder.
    Config 3: 128 prompts of U[1024, 8192] tokens (seed 2), prefilled one by one (prefill_row),
    `steps` greedy steps.  Config 4: odd layers read the preceding even layer's slot; one
    4,096-token prompt (seed 3) prefilled once and broadcast to 256 rows, `steps` steps sampled at
    temperature 1.0, top_k 50 (seed 4).
    world > 1 (strong scaling, one process per GPU, full weights on every rank): config 3's 128
    rows are partitioned by length (sharding.balanced_rows, an equal share per rank), config 4's
    256 rows are split evenly and every rank prefills the prompt itself and broadcasts it into its
    own rows.  The timed region ends with the gather of every rank's tokens (NCCL, the path's only
    collective); the step time is the max over ranks.
    kv_gbs: the KV bytes the steps' attention reads (every layer, its visible keys, all ranks) /
    the step time."""
    import numpy as np
    import torch
    import modelcore_b200
    from modelcore_b200 import workloads
    from modelcore_b200.sharding import balanced_rows, gather_tokens
    mgr = modelcore_b200.ModelManager()
    model = mgr.create_model(workloads.gqa_window_config(kv_share=(config == 4)), device=torch.device("cuda"),
                             seed=0).to(torch.bfloat16).eval()
    blocks = model.body.blocks
    windows = [b.mixer.window for b in blocks]
    Hkv, D = blocks[0].mixer.n_kv_head, blocks[0].mixer.head_dim
    stream = torch.cuda.current_stream()
    n_rows = 128 if config == 3 else 256
    with torch.inference_mode():
        t0 = time.perf_counter()
        if config == 3:
            lens = torch.randint(1024, 8193, (128,), generator=torch.Generator().manual_seed(2))
            toks = workloads.prompts(128, 8192, seed=2)
            mine = balanced_rows(lens.tolist(), world, equal_counts=True)[rank]
            prompts = [toks[i, :int(lens[i])].tolist() for i in mine]
            dec = mgr.new_decoder(model, prompts, max_tokens=steps + 8, cuda_graph=True, batched_prefill=False)
        else:
            prompt = workloads.prompts(1, 4096, seed=3)[0].tolist()
            dec = mgr.new_decoder(model, [prompt], num_samples=n_rows // world, max_tokens=steps + 8,
                                  cuda_graph=True)
        torch.cuda.synchronize()
        prefill_s = _max_over_ranks(time.perf_counter() - t0, world)
        gen = torch.Generator(device="cuda").manual_seed(4 + rank)

        def run(n):
            if config == 3:
                return dec.greedy_steps(n)
            return dec.sample_steps(n, temperature=1.0, top_k=50, generator=gen)

        run(3)  # eager step, graph capture, one replay
        before = dec.kv_cache.host_lens().astype(np.int64)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        _barrier(world)
        torch.cuda.nvtx.range_push(f"gqa_decode_cfg{config}")
        e0.record(stream)
        toks_out = run(steps)
        if world > 1:
            gather_tokens(toks_out)
        e1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    ms = _max_over_ranks(e0.elapsed_time(e1), world)
    B = int(before.size)
    keys = 0
    for i in range(steps):
        L = before + i  # the new token's position
        for w in windows:
            keys += int(np.minimum(L + 1, w + 1).sum()) if w >= 0 else int((L + 1).sum())
    kv_bytes = _sum_over_ranks(keys * 2 * Hkv * D * 2, world)
    ctx = _sum_over_ranks(float(before.sum()), world) / n_rows
    kv_gbs = kv_bytes / (ms * 1e-3) / 1e9
    out = {"workload": f"config {config}: 24 x 2048 GQA (16/4 heads of 128, window 1024 on 3 of 4 layers"
                       + (", odd layers sharing the even layer's slot" if config == 4 else "")
                       + f"), {n_rows} rows" + (f" over {world} GPUs ({B} per GPU)" if world > 1 else "")
                       + f", {steps} of the run's decode steps",
           "rows": n_rows, "n_gpus": world, "mean_context": round(ctx + steps / 2, 1),
           "tokens_per_s": round(n_rows * steps / (ms * 1e-3), 1), "ms_per_step": round(ms / steps, 3),
           "kv_gbs": round(kv_gbs, 1), "kv_frac_of_peak": round(kv_gbs / (peak * world), 3),
           "prefill_s": round(prefill_s, 2)}
    del dec, model
    torch.cuda.empty_cache()
    return out


def _prefill_append(peak, timed):
    """Piece 1 at T_new = P -- the append of whole prompts -- against the HBM copy roofline:
    config 2's prefill (64 rows x 512 tokens, 12 q / 12 kv heads of 64) and config 3's longest
    prompt (one row of 8,192 tokens, 16 q / 4 kv heads of 128), one attention layer's
    mcb_kv_append_rope each.  Algorithmic bytes: q, k, v read, the rotated q written, k' and v
    written into the slot, and the rotary rows of the P positions (cos and sin) read once."""
    import torch
    from modelcore_b200 import ops
    out = []
    for name, B, T, Hq, Hkv, D in (("config 2 prefill: 64 rows x 512 tokens, 12/12 heads of 64", 64, 512, 12, 12, 64),
                                   ("config 3 prompt: 1 row x 8192 tokens, 16/4 heads of 128", 1, 8192, 16, 4, 128)):
        g = torch.Generator(device="cuda").manual_seed(7)
        qkv = torch.randn(B, T, Hq + 2 * Hkv, D, device="cuda", generator=g, dtype=torch.bfloat16)
        q, k, v = qkv[:, :, :Hq], qkv[:, :, Hq:Hq + Hkv], qkv[:, :, Hq + Hkv:]  # views of one packed GEMM output
        kc = torch.zeros(B, 1024 if T <= 512 else T + 1024, Hkv, D, device="cuda", dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        sl = torch.zeros(B, dtype=torch.int32, device="cuda")
        ang = torch.arange(kc.size(1), device="cuda", dtype=torch.float32)[:, None] * \
            (100000.0 ** (-torch.arange(0, D, 2, device="cuda", dtype=torch.float32) / D))[None]
        cos, sin = ang.cos().to(torch.bfloat16), ang.sin().to(torch.bfloat16)
        q_out = torch.empty(B, T, Hq, D, device="cuda", dtype=torch.bfloat16)
        us = timed(lambda: ops.kv_append_rope(q, k, v, kc, vc, sl, cos, sin, q_out=q_out))
        nbytes = B * T * D * 2 * ((Hq + 2 * Hkv) + Hq + 2 * Hkv) + T * D * 2
        out.append({"workload": name, "bytes": nbytes, "us": round(us, 1),
                    "gbs": round(nbytes / us / 1e3, 1), "frac": round(nbytes / us / 1e3 / peak, 3)})
        del qkv, kc, vc, q_out
    torch.cuda.empty_cache()
    return out


def _copy_and_append(peak):
    """Piece 2 and piece 1 against the HBM copy roofline.

    kv_broadcast: config 4's prefill -> broadcast (12 slots of a 4,096-token batch-1 cache, 4 kv
    heads of 128, into 256 rows of a 4,352-position cache): algorithmic bytes = the source read
    once + every destination row written.  kv_append: config 5's per-step fused rope append at
    batch 512 (32 q / 8 kv heads of 128): q, k, v read, q' and the cache rows written, the rotary
    rows read.  prefill_append: the append of whole prompts (_prefill_append).  Each timed with
    CUDA events around single launches, L2 flushed before each, median of 5."""
    import torch
    import modelcore_b200
    from modelcore_b200 import ops
    out = {}
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    def timed(fn, reps=5):
        ts = []
        for i in range(reps + 1):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize()
            if i:
                ts.append(a.elapsed_time(b) * 1e3)
        return statistics.median(ts)

    S, P, H, D, B, Tmax = 12, 4096, 4, 128, 256, 4352
    src = modelcore_b200.KVCache(1, H, P, D, S, "cuda", torch.bfloat16)
    src.k_cache.normal_()
    src.v_cache.normal_()
    src.advance(P)
    dst = modelcore_b200.KVCache(B, H, Tmax, D, S, "cuda", torch.bfloat16)

    def bcast():
        ops.kv_copy_rows(dst.k_cache, dst.v_cache, src.k_cache, src.v_cache, src_row=0,
                         dst_row_begin=0, dst_row_count=B, n_pos=P, dst_seqlens=dst.cache_seqlens)
    us = timed(bcast)
    nbytes = 2 * S * P * H * D * 2 * (1 + B)
    out["kv_broadcast"] = {"workload": "config 4: 12 slots x 4096 positions x 4 x 128 -> 256 rows",
                           "bytes": nbytes, "us": round(us, 1),
                           "gbs": round(nbytes / us / 1e3, 1), "frac": round(nbytes / us / 1e3 / peak, 3)}
    del src, dst
    torch.cuda.empty_cache()

    B, Hq, Hkv, D, Tmax = 512, 32, 8, 128, 4096
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(B, 1, Hq, D, device="cuda", generator=g, dtype=torch.bfloat16)
    k = torch.randn(B, 1, Hkv, D, device="cuda", generator=g, dtype=torch.bfloat16)
    v = torch.randn(B, 1, Hkv, D, device="cuda", generator=g, dtype=torch.bfloat16)
    kc = torch.zeros(B, Tmax, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    sl = torch.randint(0, Tmax - 1, (B,), device="cuda", generator=g, dtype=torch.int32)
    cos = torch.randn(Tmax, D // 2, device="cuda", generator=g).to(torch.bfloat16)
    sin = torch.randn(Tmax, D // 2, device="cuda", generator=g).to(torch.bfloat16)
    q_out = torch.empty_like(q)
    us = timed(lambda: ops.kv_append_rope(q, k, v, kc, vc, sl, cos, sin, q_out=q_out))
    nbytes = 2 * (B * Hq * D * 2) + 2 * (2 * B * Hkv * D * 2) + 2 * B * (D // 2) * 2
    out["kv_append"] = {"workload": "config 5 step: batch 512, 32 q / 8 kv heads of 128",
                        "bytes": nbytes, "us": round(us, 2),
                        "gbs": round(nbytes / us / 1e3, 1), "frac": round(nbytes / us / 1e3 / peak, 3)}
    del q, k, v, kc, vc, q_out
    out["prefill_append"] = _prefill_append(peak, timed)
    del flush
    torch.cuda.empty_cache()
    return out


def _prefill(tflops_peak):
    """The tensor-core prefill attention (tcgen05) against the measured dense bf16 peak.

    config 3's longest prompt (8,192 tokens, 16 q / 4 kv heads of 128, full window and window
    1024) and config 2's prefill (64 prompts x 512 tokens, 12 / 12 heads of 64), each as one
    mcb_decode_attn call over an empty cache (the automatic prefill plan).  Algorithmic FLOPs =
    4 * D * Hq * (visible keys summed over queries): QK^T and PV, causal.  L2 flushed before
    each timed launch."""
    import torch
    from modelcore_b200 import ops
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    rows = []
    for name, B, T, Hq, Hkv, D, window in (("config 3 prompt, 8192 tokens", 1, 8192, 16, 4, 128, -1),
                                            ("config 3 prompt, 8192 tokens, window 1024", 1, 8192, 16, 4, 128, 1024),
                                            ("config 2 prefill, 64 prompts x 512 tokens", 64, 512, 12, 12, 64, -1)):
        g = torch.Generator(device="cuda").manual_seed(2)
        q = torch.randn(B, T, Hq, D, device="cuda", generator=g, dtype=torch.bfloat16)
        kc = torch.randn(B, T, Hkv, D, device="cuda", generator=g, dtype=torch.bfloat16)
        vc = torch.randn(B, T, Hkv, D, device="cuda", generator=g, dtype=torch.bfloat16)
        sl = torch.zeros(B, dtype=torch.int32, device="cuda")
        out = torch.empty_like(q)
        keys = sum(min(t + 1, window + 1) if window >= 0 else t + 1 for t in range(T))
        flops = 4 * D * Hq * B * keys
        ts = []
        for i in range(6):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            ops.decode_attn(q, kc, vc, sl, window=window, out=out)
            b.record(stream)
            torch.cuda.synchronize()
            if i:
                ts.append(a.elapsed_time(b) * 1e3)
        us = statistics.median(ts)
        rows.append({"workload": name, "kernel": ops.last_attn_kernel(), "us": round(us, 1),
                     "tflops": round(flops / us / 1e6, 1),
                     "frac": round(flops / us / 1e6 / tflops_peak, 3)})
        del q, kc, vc, out
    del flush
    torch.cuda.empty_cache()
    return rows


def _cpu_reference_decode(rows, steps, warmup, threads=None):
    """The reference itself (modelcore's Decoder over its KVCache and SDPA path, fp32 on the host
    cores) on `rows` of the same prompts; returns (tokens/s, seconds per step, cores)."""
    import torch
    _ensure_modelcore()
    import modelcore
    from modelcore_b200 import workloads
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    mgr = modelcore.ModelManager(runtime=modelcore.Runtime(compute_dtype=torch.float32))
    model = mgr.create_model(workloads.quickstart_config(), device=torch.device("cpu"), seed=0).eval()
    prompts = workloads.prompts(rows, PROMPT_LEN, seed=1).tolist()
    with torch.inference_mode():
        dec = mgr.new_decoder(model, prompts, max_tokens=DECODE_LEN)
        tok = torch.argmax(dec.logits, dim=-1)
        for _ in range(warmup):
            tok = torch.argmax(dec.step(tok.tolist()), dim=-1)
        t0 = time.perf_counter()
        for _ in range(steps):
            tok = torch.argmax(dec.step(tok.tolist()), dim=-1)
        dt = time.perf_counter() - t0
    return rows * steps / dt, dt / steps, threads


def _gpu_reference_decode(rows, steps, warmup):
    """The reference's own decode path on the same B200 (BASELINE's GPU comparison point): the
    stock modelcore ModelManager, KVCache, Decoder and flash_attn_with_kvcache (its SDPA path on
    this GPU), bf16, none of this repository's kernels, on `rows` of the same prompts; timed with
    CUDA events around `steps` greedy steps of its own loop (a host read of the tokens each step,
    as the reference's Decoder does).  Returns (tokens/s, ms per step, the attention path)."""
    import torch
    _ensure_modelcore()
    import modelcore
    from modelcore.kernels import flash_attn as ref_fa
    from modelcore_b200 import workloads
    mgr = modelcore.ModelManager(runtime=modelcore.Runtime(compute_dtype=torch.bfloat16))
    model = mgr.create_model(workloads.quickstart_config(), device=torch.device("cuda"), seed=0)
    model = model.to(torch.bfloat16).eval()
    prompts = workloads.prompts(rows, PROMPT_LEN, seed=1).tolist()
    with torch.inference_mode():
        dec = mgr.new_decoder(model, prompts, max_tokens=DECODE_LEN)
        tok = torch.argmax(dec.logits, dim=-1)
        for _ in range(warmup):
            tok = torch.argmax(dec.step(tok.tolist()), dim=-1)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            tok = torch.argmax(dec.step(tok.tolist()), dim=-1)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
    path = "FA3" if getattr(ref_fa, "USE_FA3", False) else "SDPA"
    del dec, model, mgr
    torch.cuda.empty_cache()
    return rows / (ms * 1e-3), ms, path


def _cpu_reference_gqa(config, steps=3, threads=None):
    """Configs 3 and 4 on the host cores through the reference itself (modelcore's Decoder,
    KVCache and SDPA path, fp32), at a reduced batch with the GPU run's per-row shapes: config 3
    one row, the seeded prompt (seed 2, as the GPU run's) whose length is closest to the rows'
    mean; config 4 the 4,096-token prompt (seed 3) broadcast to 2 rows, sampled at temperature
    1.0, top_k 50.  Prefill untimed; `steps` timed decode steps.  Per-row tokens/s, and KV GB/s by
    the GPU's formula (exact visible keys x 2 x Hkv x D x 2: the bf16 cache's bytes)."""
    import numpy as np
    import torch
    _ensure_modelcore()
    import modelcore
    from modelcore.generate import sample_next_token
    from modelcore_b200 import workloads
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    mgr = modelcore.ModelManager(runtime=modelcore.Runtime(compute_dtype=torch.float32))
    model = mgr.create_model(workloads.gqa_window_config(kv_share=(config == 4)), device=torch.device("cpu"),
                             seed=0).eval()
    blocks = model.body.blocks
    windows = [b.mixer.window for b in blocks]
    Hkv, D = blocks[0].mixer.n_kv_head, blocks[0].mixer.head_dim
    if config == 3:
        lens = torch.randint(1024, 8193, (128,), generator=torch.Generator().manual_seed(2))
        i = int(torch.argmin((lens.float() - lens.float().mean()).abs()))
        prompts, samples = [workloads.prompts(128, 8192, seed=2)[i, :int(lens[i])].tolist()], 1
    else:
        prompts, samples = [workloads.prompts(1, 4096, seed=3)[0].tolist()], 2
    gen = torch.Generator().manual_seed(4)
    with torch.inference_mode():
        dec = mgr.new_decoder(model, prompts, num_samples=samples, max_tokens=steps + 4)
        L0 = int(dec.kv_cache.cache_seqlens[0])
        rows = samples * len(prompts)

        def pick(logits):
            if config == 3:
                return torch.argmax(logits, dim=-1)
            return sample_next_token(logits, gen, temperature=1.0, top_k=50).view(-1)

        tok = pick(dec.logits)
        t0 = time.perf_counter()
        for _ in range(steps):
            tok = pick(dec.step(tok.tolist()))
        dt = time.perf_counter() - t0
    keys = 0
    for j in range(steps):
        L = L0 + j
        keys += rows * sum(min(L + 1, w + 1) if w >= 0 else L + 1 for w in windows)
    return {"config": config, "rows": rows, "context": L0, "steps": steps,
            "tokens_per_s": round(rows * steps / dt, 3), "per_row_tokens_per_s": round(steps / dt, 3),
            "kv_gbs": round(keys * 2 * Hkv * D * 2 / dt / 1e9, 3), "cores": threads,
            "sample": f"modelcore Decoder + SDPA path fp32 on {threads} threads ({_cpu_model()}), "
                      f"{rows} row(s) at context {L0}, {steps} timed steps, prefill untimed"}


def _cpu_reference_attention(B=8, windows=(-1, 4096), reps=2, threads=None):
    """Config 5 on the host cores through the reference's own kernel call: modelcore's
    flash_attn_with_kvcache on its SDPA path (modelcore/kernels/flash_attn.py:306-366), fp32,
    B rows of 32 q / 8 kv heads of 128 with the GPU sweep's lengths (U[1, 32768] from seed 5),
    one call = one decode step (the insert of one K/V per row + the attention over the cache).
    Per point: the call time, keys/s, tokens/s and the same algorithmic KV bytes as the GPU
    sweep (exact keys x 2 x Hkv x D x 2, i.e. the bf16 cache's bytes; the fp32 cache the CPU
    reads holds twice as many)."""
    import numpy as np
    import torch
    _ensure_modelcore()
    from modelcore.kernels.flash_attn import flash_attn as fa
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    Hq, Hkv, D, Tmax = 32, 8, 128, 32769
    lens = np.random.default_rng(5).integers(1, 32769, size=B) - 1
    g = torch.Generator().manual_seed(5)
    kc = torch.randn(B, Tmax, Hkv, D, generator=g)
    vc = torch.randn(B, Tmax, Hkv, D, generator=g)
    q = torch.randn(B, 1, Hq, D, generator=g)
    k = torch.randn(B, 1, Hkv, D, generator=g)
    v = torch.randn(B, 1, Hkv, D, generator=g)
    sl = torch.from_numpy(lens).to(torch.int32)
    rows = []
    with torch.inference_mode():
        for w in windows:
            call = lambda: fa.flash_attn_with_kvcache(q, kc, vc, k=k, v=v, cache_seqlens=sl, causal=True,
                                                     window_size=(w, 0))
            call()
            t0 = time.perf_counter()
            for _ in range(reps):
                call()
            dt = (time.perf_counter() - t0) / reps
            keys = int(sum((L + 1) if w < 0 else min(L + 1, w + 1) for L in lens))
            gbs = keys * 2 * Hkv * D * 2 / dt / 1e9
            rows.append({"batch": B, "window": w, "mean_keys": round(keys / B, 1),
                         "call_ms": round(dt * 1e3, 1), "keys_per_s": round(keys / dt),
                         "tokens_per_s": round(B / dt, 2), "kv_gbs": round(gbs, 2)})
    return {"value": rows, "unit": "per point", "cores": threads, "kind": "reference",
            "sample": f"config 5 at batch {B} (of 1-512), {reps} timed calls per window after one "
                      f"warm-up, modelcore flash_attn_with_kvcache SDPA path fp32 ({_cpu_model()})"}


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args):
    """--impl reference: the reference's CPU implementation on the host cores (rank 0 only), on
    the same 64 rows of config 2 the GPU decodes per rank (prefill untimed)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    rows = ROWS_PER_GPU
    tps, sps, cores = _cpu_reference_decode(rows, args.steps, args.warmup)
    sample = (f"the 64 rows of one GPU, 512-token prompts (prefill untimed), {args.steps} timed "
              f"greedy decode steps after {args.warmup} warm-up steps, modelcore Decoder + SDPA "
              f"path in fp32 on {cores} threads ({_cpu_model()})")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tps, 2), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded uniform token ids)",
        "config": _config(args.gpus),
        "cpu_baseline": {"value": round(tps, 2), "unit": "tokens/s", "cores": cores,
                         "kind": "reference", "sample": sample,
                         "per_row_tokens_per_s": round(tps / rows, 3)},
        "e2e": {"value": round(tps, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _config(n):
    return {"workload": "config 2: README quickstart model (12 x 768, 12/12 heads of 64), bf16 weights, "
                        "64 prompts x 512 tokens per GPU, KV cache 1024, greedy decode",
            "model": "modelcore quickstart 12x768", "global_batch": ROWS_PER_GPU * n,
            "seq_len": PROMPT_LEN + DECODE_LEN, "prompt_len": PROMPT_LEN,
            "parallelism": f"batch-sharded replicas x{n}",
            "l2": "inputs larger than L2: 1.2-2.4 GB of KV + 0.2 GB of weights per step per GPU"}


def run_prefill_only(args):
    """--prefill-only: the prefill-attention measurements alone (used for small ncu captures)."""
    import torch
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    _ensure_modelcore()
    print(json.dumps({"prefill_attention": _prefill(_bf16_peak())}), flush=True)


def run_sweep_only(args):
    """--sweep-only: the config-5 sweep alone (used for small ncu captures)."""
    import torch
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    peak, _ = _peaks()
    rows = _kv_read_sweep(peak, batches=tuple(args.sweep_batches), windows=tuple(args.sweep_windows))
    rows8 = _kv_read_sweep(peak, batches=tuple(args.sweep_batches), windows=tuple(args.sweep_windows), fp8=True)
    print(json.dumps({"kv_read_sweep": rows, "kv_read_sweep_fp8": _with_speedup(rows8, rows),
                      "peak_gbs": peak}), flush=True)


def _print_extras(extras, world):
    """The measurements beside the headline, one JSON line each, printed before it (the headline
    is the last line): {"bench_extra": name, "n_gpus": N, "data": ...}."""
    for name, obj in extras.items():
        if obj is not None:
            print(json.dumps({"bench_extra": name, "n_gpus": world, "data": obj}), flush=True)


def _sweep_summary(rows):
    return {f"b{r['batch']}_w{r['window']}": r["frac"] for r in rows} if rows else None


def run_b200(args):
    import torch
    _ensure_modelcore()
    import modelcore_b200
    from modelcore_b200 import step as _step
    _step.USE_FUSED_PROJ = args.linear == "fused"
    _step.USE_LINEAR_PROJ = args.linear in ("mcb", "mcb-norm")
    _step.USE_LINEAR_NORM_OUT = args.linear == "mcb"
    rank, world, local = _dist_setup(args.gpus)
    peak, peak_kind = _peaks()
    steps_needed = 1 + args.warmup + max(args.steps, args.e2e_steps or 0) + 2
    mgr, model, dec = _build_decoder(rank, world, steps_needed, fuse_step=args.step == "fused")
    cache = dec.kv_cache
    B = cache.batch_size

    # warm-up: the first step runs eagerly, the second captures the CUDA graph, the rest replay it
    with torch.inference_mode():
        dec.greedy_steps(1 + args.warmup)
    tokens = torch.empty((B, args.steps), dtype=torch.long, device="cuda")
    ctx_before = cache.host_lens().copy()

    _barrier(world)
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gpu_uuid = torch.cuda.get_device_properties(local).uuid
    with ClockSampler(f"GPU-{gpu_uuid}" if gpu_uuid else local) as clocks:
        time.sleep(0.3)  # let the sampler start before the timed region
        clocks.mark("start")
        torch.cuda.nvtx.range_push("timed_decode")
        e0.record(stream)
        with torch.inference_mode():
            dec.greedy_steps(args.steps, first_tokens=None, out=tokens)
            if world > 1:
                from modelcore_b200.sharding import gather_tokens
                gather_tokens(tokens)
        e1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        clocks.mark("end")
    ms = _max_over_ranks(e0.elapsed_time(e1), world)
    _barrier(world)
    ctx_after = cache.host_lens().copy()
    value = B * world * args.steps / (ms * 1e-3)
    kv_bytes_step = float(((ctx_before + ctx_after) / 2 + 1).sum()) * cache.n_slots * 2 * \
        cache.n_kv_head * cache.head_dim * 2

    # e2e: the public GraphDecoder.step_greedy() -- host token column in through pinned memory,
    # the forward, the greedy pick, the next tokens back in pinned memory and read on the host,
    # every step -- over the same context range as the timed steps: the rows are rewound to
    # where the timed region began (less the two untimed calls below); the positions decoded
    # again are overwritten by the steps' own appends, and no kernel reads past a row's length
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else args.steps
    with torch.inference_mode():
        cache.set_row_lengths(ctx_before - 2)
        host_tok = torch.argmax(dec.logits, dim=-1).cpu()
        for _ in range(2):  # the first call captures its graph: keep that out of the timing
            host_tok = dec.step_greedy(host_tok).clone()
        _barrier(world)
        t0 = time.perf_counter()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(e2e_steps):
            host_tok = dec.step_greedy(host_tok)
        f1.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    e2e_ms = _max_over_ranks(f0.elapsed_time(f1), world)
    e2e_value = B * world * e2e_steps / (e2e_ms * 1e-3)
    launches_per_step = dec.launches_per_step  # libmcb200 kernels in one captured step
    roof = _attention_roofline(dec, peak)
    prompt_prefill = {"workload": f"{B} prompts x {PROMPT_LEN} tokens per GPU, one forward "
                                  "(GraphDecoder batched ragged prefill)",
                      "batched_ms": round(dec.prefill_ms, 2)}
    if world == 1 and not args.no_sweep:
        from modelcore_b200 import workloads
        mine = workloads.prompts(ROWS_PER_GPU, PROMPT_LEN, seed=1).tolist()
        prompt_prefill["per_prompt_ms"] = round(_per_prompt_prefill_ms(mgr, model, mine), 2)
        prompt_prefill["per_prompt"] = "modelcore's Decoder order: each prompt at batch 1, then prefill_row"
    del dec, model, mgr, cache
    torch.cuda.empty_cache()

    # the other measurement configs: on one GPU all of them; on N GPUs the ones the path shards
    # (config 3 and 4 rows, config 5 batches partitioned over the ranks, no collective but the
    # token gather)
    extras = {}
    if not args.no_sweep:
        extras["kv_read_sweep"] = _kv_read_sweep(peak, batches=tuple(args.sweep_batches),
                                                 windows=tuple(args.sweep_windows), rank=rank, world=world)
        extras["gqa_decode"] = [_gqa_decode(c, peak, rank=rank, world=world) for c in (3, 4)]
        if world == 1:
            extras["kv_read_sweep_fp8"] = _with_speedup(
                _kv_read_sweep(peak, batches=tuple(args.sweep_batches), windows=tuple(args.sweep_windows),
                               fp8=True), extras["kv_read_sweep"])
            extras["kv_copies"] = _copy_and_append(peak)
            extras["prefill_attention"] = _prefill(_bf16_peak())
    extras["prompt_prefill"] = prompt_prefill
    if world == 1 and not args.no_sweep:
        # BASELINE's GPU comparison point: the reference's own decode path on this B200
        tps_ref, ms_ref, path = _gpu_reference_decode(ROWS_PER_GPU, 20, 3)
        extras["reference_on_b200"] = {
            "workload": f"config 2, {ROWS_PER_GPU} rows, 20 greedy steps after 3 warm-up steps",
            "impl": f"modelcore's own Decoder + KVCache + flash_attn_with_kvcache ({path} path), bf16",
            "tokens_per_s": round(tps_ref, 1), "ms_per_step": round(ms_ref, 3),
            "this_path_over_it": round(value / tps_ref, 1)}
    cpu = None
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        tps, sps, cores = _cpu_reference_decode(CPU_SAMPLE_ROWS, 5, 1)
        cpu = {"value": round(tps, 2), "unit": "tokens/s", "cores": cores, "kind": "reference",
               "per_row_tokens_per_s": round(tps / CPU_SAMPLE_ROWS, 3),
               "sample": f"{CPU_SAMPLE_ROWS} of the 64 rows, 512-token prompts, 5 timed greedy "
                         f"steps, modelcore Decoder + SDPA path fp32 ({_cpu_model()}); the "
                         f"--impl reference arm runs all 64 rows"}
        extras["cpu_baseline_config5"] = _cpu_reference_attention()
        extras["cpu_baseline_configs34"] = [_cpu_reference_gqa(3), _cpu_reference_gqa(4)]

    if rank != 0:
        return
    _print_extras(extras, world)
    sweep, gqa, copies = extras.get("kv_read_sweep"), extras.get("gqa_decode"), extras.get("kv_copies")
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded uniform token ids, random-init weights)",
        "config": _config(world),
        "decode_step": {"fused": "packed QKV and gate|up GEMMs; residual add + norm and silu * up "
                                 "on libmcb200",
                        "plain": "modelcore's op-by-op forward around the libmcb200 append and "
                                 "attention"}[args.step],
        "projections": {"mcb": "every projection on libmcb200 mcb_linear under programmatic "
                               "dependent launch: c_proj with the residual add and the next norm "
                               "in its epilogue, gate|up with silu * up in its epilogue",
                        "mcb-norm": "every projection on libmcb200 mcb_linear, c_proj with the "
                                    "residual add in its epilogue, the norm after it a launch "
                                    "of its own",
                        "fused": "libmcb200 mcb_linear with the norms and adds fused in, down_proj on cuBLAS",
                        "cublas": "torch F.linear (cuBLAS)"}[args.linear],
        "kv_read": {"bytes_per_step": int(kv_bytes_step),
                    "step_gbs": round(kv_bytes_step / (ms / args.steps * 1e-3) / 1e9, 1),
                    "attention_kernel_gbs": round(roof["achieved_gbs"], 1),
                    "attention_frac_of_peak": round(roof["frac"], 3),
                    "mean_context": round(roof["mean_context"], 1)},
        "roofline": {"bound": "hbm", "achieved": round(roof["achieved_gbs"], 1),
                     "peak": peak, "unit": "GB/s", "frac": round(roof["frac"], 4),
                     "traffic": roof["traffic"], "kernel": roof["kernel"],
                     "traffic_source": "scaled constant: DRAM bytes per fetched 64-key tile from an "
                                       "ncu capture of this kernel on this model, times the "
                                       f"{roof['tiles']} tiles of this launch",
                     "algorithmic_bytes_per_launch": roof["bytes_per_launch"],
                     "us_per_launch": round(roof["us_per_launch"], 2),
                     "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback"},
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": B * 8, "d2h_bytes_per_step": B * 8,
                "wall_s": round(wall, 4)},
        "gpu_launches": int(launches_per_step * args.steps) if launches_per_step else None,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
        "kv_read_sweep_frac": _sweep_summary(sweep),
        "gqa_decode_tokens_per_s": {f"config {c}": r["tokens_per_s"] for c, r in zip((3, 4), gqa)} if gqa else None,
        "prefill_append_frac": [r["frac"] for r in copies["prefill_append"]] if copies else None,
        "reference_on_b200_tokens_per_s": (extras["reference_on_b200"]["tokens_per_s"]
                                           if "reference_on_b200" in extras else None),
        "extras_printed_above": [k for k, v in extras.items() if v is not None],
    }
    return line


def main():
    ap = argparse.ArgumentParser(description="modelcore KV-cache decode benchmark (B200)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--e2e-steps", type=int, default=None,
                    help="steps of the end-to-end loop (default: --steps, over the same contexts)")
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--step", choices=("fused", "plain"), default="fused",
                    help="decode step around attention: fused (default) or modelcore's op-by-op")
    ap.add_argument("--linear", choices=("mcb", "mcb-norm", "cublas", "fused"), default="mcb",
                    help="decode projections: all on libmcb200's mcb_linear, c_proj with the "
                         "residual add and the next norm in its epilogue (default); the same with "
                         "the norm a launch of its own; all on cuBLAS; or mcb_linear with the "
                         "norms and adds fused in front")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep-only", action="store_true", help="run only the config-5 KV-read sweep")
    ap.add_argument("--prefill-only", action="store_true",
                    help="run only the prefill-attention measurements")
    ap.add_argument("--gqa-only", action="store_true",
                    help="run only the config-3 / config-4 decode measurements")
    ap.add_argument("--gqa-configs", type=int, nargs="+", choices=(3, 4), default=[3, 4],
                    help="with --gqa-only: which of configs 3 and 4 to run")
    ap.add_argument("--sweep-batches", type=int, nargs="+", default=[1, 8, 64, 256, 512])
    ap.add_argument("--sweep-windows", type=int, nargs="+", default=[-1, 4096])
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.sweep_only:
        run_sweep_only(args)
    elif args.prefill_only:
        run_prefill_only(args)
    elif args.gqa_only:
        import torch
        _ensure_modelcore()
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        peak, _ = _peaks()
        print(json.dumps({"gqa_decode": [_gqa_decode(c, peak) for c in args.gqa_configs]}), flush=True)
    else:
        line = run_b200(args)
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()
        if line is not None:  # rank 0: the headline last, after NCCL's teardown lines
            print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
