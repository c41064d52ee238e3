"""The multi-GPU host logic on CPU ranks (gloo, world size 2): row sharding, the token gather that
is the path's only collective, and a rank that leaves before the gather (failure detection on
the host, with a short process-group timeout -- no GPU involved)."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from modelcore_b200.sharding import balanced_rows, contiguous_rows, gather_tokens


def test_contiguous_rows_cover_every_row_once():
    for n in (1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            spans = [contiguous_rows(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - b for b, e in spans]
            assert max(sizes) - min(sizes) <= 1


def test_balanced_rows_balance_ragged_context():
    g = torch.Generator().manual_seed(2)
    lengths = torch.randint(1024, 8193, (128,), generator=g).tolist()  # config 3's prompt lengths
    for world in (2, 4, 8):
        parts = balanced_rows(lengths, world)
        assert sorted(i for p in parts for i in p) == list(range(128))
        loads = [sum(lengths[i] for i in p) for p in parts]
        assert max(loads) / (sum(lengths) / world) < 1.02
        eq = balanced_rows(lengths, world, equal_counts=True)
        assert sorted(i for p in eq for i in p) == list(range(128))
        assert all(len(p) == 128 // world for p in eq)
        loads = [sum(lengths[i] for i in p) for p in eq]
        assert max(loads) / (sum(lengths) / world) < 1.03
    with pytest.raises(ValueError):
        balanced_rows(lengths[:7], 2, equal_counts=True)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=6))
    try:
        begin, end = contiguous_rows(6, world, rank)
        tokens = torch.arange(begin, end, dtype=torch.int64)[:, None] * 100 + torch.arange(4)
        if mode == "leave" and rank == 1:
            results[rank] = "left"
            return  # leaves between steps, before the gather, with nothing in flight
        try:
            out = gather_tokens(tokens)
            results[rank] = out.tolist()
        except Exception as e:  # the surviving rank learns of it from the collective's error
            results[rank] = f"error: {type(e).__name__}"
    finally:
        if mode != "leave":
            dist.destroy_process_group()


def _run(mode):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, results)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(60)
            assert not p.is_alive()
        return dict(results)


def test_token_gather_concatenates_ranks_in_order():
    res = _run("gather")
    want = [[r * 100 + s for s in range(4)] for r in range(6)]
    assert res[0] == want and res[1] == want


def test_a_rank_that_leaves_before_the_gather_is_reported_not_waited_on():
    res = _run("leave")
    assert res[1] == "left"
    assert str(res[0]).startswith("error:")


@pytest.mark.parametrize("world,preset,expected", [("2", "VERSION", "INFO"), ("2", None, "INFO"),
                                                   ("2", "TRACE", "TRACE"), ("1", "VERSION", "VERSION")])
def test_bench_raises_nccl_logging_to_init_lines_at_more_than_one_rank(world, preset, expected):
    # bench.py's module top only touches the environment (stdlib imports): load it in a child
    import subprocess
    import sys
    env = {k: v for k, v in os.environ.items() if not k.startswith("NCCL_DEBUG")}
    env["WORLD_SIZE"] = world
    if preset is not None:
        env["NCCL_DEBUG"] = preset
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import os, runpy; runpy.run_path(os.path.join(%r, 'bench.py'), run_name='not_main'); "
            "print(os.environ.get('NCCL_DEBUG'), os.environ.get('NCCL_DEBUG_SUBSYS'))" % root)
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    level, subsys = out.stdout.split()
    assert level == expected
    assert subsys == ("INIT" if world == "2" else "None")
