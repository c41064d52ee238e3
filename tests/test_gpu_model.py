"""End-to-end parity through modelcore's own API on the GPU: the reference (modelcore's SDPA path,
unmodified) and the B200 path decode the same weights and prompts in bf16 on the same device.

* greedy token streams are identical for 64 steps (README quickstart architecture, awake weights)
* logits agree within LOGIT_TOL at every step
* multi-prompt right-ragged decode agrees on every reference test flavor that has attention
  (windows, cross-layer KV sharing, GQA, gates, value embeddings, smear, layer_norm QK-norm)
* the CUDA-graph decoder reproduces the eager decoder bit for bit
"""
import copy

import pytest
import torch

from conftest import have_modelcore, load_golden

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2


@pytest.fixture(scope="module")
def env():
    if not have_modelcore():
        raise RuntimeError("modelcore (the reference package) is not importable: install it into "
                           "baseline/_ref (__graft_entry__.build() does) to run the end-to-end parity tests")
    import modelcore
    import modelcore_b200
    return modelcore, modelcore_b200


def _pair(env, config, awake=True):
    modelcore, mcb = env
    from modelcore_b200 import workloads
    ref_mgr = modelcore.ModelManager()
    cpu = ref_mgr.create_model(config, device=torch.device("cpu"), seed=0)
    if awake:
        workloads.awaken(cpu)
    cpu.eval()
    ref = copy.deepcopy(cpu).to("cuda")
    mine = copy.deepcopy(cpu).to("cuda")
    assert mcb.install(mine) > 0
    return ref_mgr, ref, mcb.ModelManager(), mine


@torch.inference_mode()
def _greedy(mgr, model, prompts, steps):
    dec = mgr.new_decoder(model, prompts, max_tokens=steps)
    toks, logits = [], []
    for _ in range(steps):
        lg = dec.logits.float().clone()
        logits.append(lg)
        nxt = torch.argmax(lg, dim=-1)
        toks.append(nxt)
        dec.step(nxt.tolist())
    logits.append(dec.logits.float().clone())
    return torch.stack(toks, 1).cpu(), logits, dec


def test_quickstart_random_init_greedy_stream_matches_the_reference_for_64_steps(env):
    """Measurement config 1 as stated (README quickstart, modelcore's random init, seed 0;
    prompts 2 x 16 from seed 1): 64 greedy steps identical to the reference's on the same GPU."""
    from modelcore_b200 import workloads
    z = load_golden("decode_cfg1.npz")
    prompts = z["prompts"].tolist()
    ref_mgr, ref, mgr, mine = _pair(env, workloads.quickstart_config(), awake=False)
    t_ref, l_ref, _ = _greedy(ref_mgr, ref, prompts, 64)
    t_mine, l_mine, dec = _greedy(mgr, mine, prompts, 64)
    import modelcore_b200
    assert isinstance(dec.kv_cache, modelcore_b200.KVCache)
    assert torch.equal(t_ref, t_mine)
    assert max((a - b).abs().max().item() for a, b in zip(l_ref, l_mine)) <= LOGIT_TOL


@torch.inference_mode()
def _forced(mgr, model, prompts, columns):
    """Logits before each forced step (teacher forcing), plus the final ones."""
    dec = mgr.new_decoder(model, prompts, max_tokens=columns.shape[1])
    out = []
    for i in range(columns.shape[1]):
        out.append(dec.logits.float().clone())
        dec.step(columns[:, i].tolist())
    out.append(dec.logits.float().clone())
    return torch.stack(out, 1)


def test_quickstart_awake_decode_is_as_accurate_as_the_reference(env):
    """Config 1's model with modelcore's test wake-up (attention reaches the logits).  Its logits
    are small (lm_head init std 1e-3), so greedy top-2 margins are often below bf16 noise and the
    reference's own bf16 stream departs from its fp32 stream within a few steps.  So, under
    identical contexts (the reference's bf16 greedy tokens, forced on every path):
      * B200 logits are within 2e-2 of the reference evaluated in fp32 on the GPU, and no
        further from it than the reference's bf16 SDPA path (x1.25 + 1e-3);
      * wherever B200 and the reference pick different greedy tokens, the fp32 top-2 margin is
        within the two paths' combined error (a genuine near-tie)."""
    modelcore, mcb = env
    from modelcore_b200 import workloads
    z = load_golden("decode_cfg1.npz")
    prompts = z["prompts"].tolist()
    ref_mgr, ref, mgr, mine = _pair(env, workloads.quickstart_config(), awake=True)
    m32 = modelcore.ModelManager(runtime=modelcore.Runtime(compute_dtype=torch.float32))
    ref32 = m32.create_model(workloads.quickstart_config(), device=torch.device("cpu"), seed=0)
    ref32.load_state_dict({k: v.float().cpu() for k, v in ref.state_dict().items()})
    ref32 = ref32.to("cuda").eval()
    t_ref, _, _ = _greedy(ref_mgr, ref, prompts, 64)
    l_ref = _forced(ref_mgr, ref, prompts, t_ref)
    l_mine = _forced(mgr, mine, prompts, t_ref)
    l32 = _forced(m32, ref32, prompts, t_ref)
    err_mine = (l_mine - l32).abs().max().item()
    err_ref = (l_ref - l32).abs().max().item()
    top2 = torch.topk(l32, 2, dim=-1).values
    margin = top2[..., 0] - top2[..., 1]
    a_mine, a_ref, a32 = l_mine.argmax(-1), l_ref.argmax(-1), l32.argmax(-1)
    differ = a_mine != a_ref
    print(f"awake quickstart: max|B200 - fp32| = {err_mine:.3e}, max|ref bf16 - fp32| = {err_ref:.3e}; "
          f"greedy picks: B200 != ref at {int(differ.sum())}/{differ.numel()}, "
          f"B200 != fp32 at {int((a_mine != a32).sum())}, ref != fp32 at {int((a_ref != a32).sum())}")
    assert err_mine <= LOGIT_TOL
    assert err_mine <= 1.25 * err_ref + 1e-3
    assert bool((margin[differ] <= 2 * (err_mine + err_ref)).all())
    assert int((a_mine != a32).sum()) <= int((a_ref != a32).sum())


LM_HEAD_GAIN = 30.0  # lm_head x30: median fp32 top-2 margin 0.13 instead of 0.005 (1e-3 init std)


def test_awake_free_running_greedy_stream_against_the_reference_for_64_steps(env):
    """The north-star stream check on a model whose attention reaches the logits: config 1's
    architecture with modelcore's test wake-up and the lm_head scaled by LM_HEAD_GAIN (so top-2
    margins mostly clear bf16 noise).  modelcore's bf16 SDPA path and the B200 path each decode
    64 greedy steps from the same prompts, each feeding its own picks (free running).

    The streams must be identical, except at a genuine near-tie: if a row's streams part, then at
    the first step where they do (both contexts still identical there), the fp32 evaluation's
    top-2 margin must be within the two bf16 paths' combined error at that step.  The first
    divergence (step, row, margin) is printed either way."""
    modelcore, mcb = env
    from modelcore_b200 import workloads
    z = load_golden("decode_cfg1.npz")
    prompts = z["prompts"].tolist()
    ref_mgr, ref, mgr, mine = _pair(env, workloads.quickstart_config(), awake=True)
    with torch.no_grad():
        for m in (ref, mine):
            m.unembedding.lm_head.weight.mul_(LM_HEAD_GAIN)
    t_ref, _, _ = _greedy(ref_mgr, ref, prompts, 64)
    t_mine, _, _ = _greedy(mgr, mine, prompts, 64)
    differ = t_ref != t_mine
    if not bool(differ.any()):
        print("awake quickstart (lm_head x30): B200 and modelcore greedy streams identical for 64 steps")
        return
    m32 = modelcore.ModelManager(runtime=modelcore.Runtime(compute_dtype=torch.float32))
    ref32 = m32.create_model(workloads.quickstart_config(), device=torch.device("cpu"), seed=0)
    ref32.load_state_dict({k: v.float().cpu() for k, v in ref.state_dict().items()})
    ref32 = ref32.to("cuda").eval()
    for r in range(differ.shape[0]):
        if not bool(differ[r].any()):
            print(f"row {r}: identical for 64 steps")
            continue
        s = int(differ[r].nonzero()[0])
        cols = t_ref[:, :s]  # row r's context is identical on both paths up to step s
        l32 = _forced(m32, ref32, prompts, cols)[:, s]
        l_mine = _forced(mgr, mine, prompts, cols)[:, s]
        l_ref = _forced(ref_mgr, ref, prompts, cols)[:, s]
        top2 = torch.topk(l32[r], 2).values
        margin = (top2[0] - top2[1]).item()
        err = (l_mine[r] - l32[r]).abs().max().item() + (l_ref[r] - l32[r]).abs().max().item()
        gap = (l_mine[r] - l_ref[r]).abs().max().item()
        print(f"row {r}: first divergence at step {s}: fp32 top-2 margin {margin:.3e}, combined "
              f"bf16 error {err:.3e} (max |B200 - modelcore bf16| there {gap:.3e})")
        assert margin <= 2 * err, (r, s, margin, err)


def _attention_flavors():
    from modelcore.tests.conftest import FLAVORS
    out = []
    for name, make in FLAVORS.items():
        cfg = make()
        if any(b.params["mixer"].type == "attention" for b in cfg.body.params["blocks"]):
            out.append(name)
    return out


def _flavor_names():
    try:
        return _attention_flavors()
    except Exception:  # collection without modelcore: the env fixture reports it
        return ["plain_kvshare_win"]


@pytest.mark.parametrize("flavor", _flavor_names())
def test_multi_prompt_ragged_decode_matches_the_reference(env, flavor):
    """modelcore/tests/test_generate.py:298-320 run as reference-vs-B200 on the GPU: right-ragged
    prompts, fixed token columns, logits compared at every step."""
    from modelcore.tests.conftest import FLAVORS
    from modelcore.tests.test_generate import RAGGED_PROMPTS
    ref_mgr, ref, mgr, mine = _pair(env, FLAVORS[flavor]())
    steps = 12
    with torch.inference_mode():
        a = ref_mgr.new_decoder(ref, RAGGED_PROMPTS, max_tokens=steps)
        b = mgr.new_decoder(mine, RAGGED_PROMPTS, max_tokens=steps)
        assert b.kv_cache.cache_seqlens.tolist() == [len(p) for p in RAGGED_PROMPTS]
        for step in range(steps + 1):
            d = (a.logits.float() - b.logits.float()).abs().max().item()
            assert d <= LOGIT_TOL, (flavor, step, d)
            if step == steps:
                break
            column = [(step * 7 + i * 3) % 100 + 1 for i in range(len(RAGGED_PROMPTS))]
            a.step(column)
            b.step(column)
        assert b.kv_cache.cache_seqlens.tolist() == [len(p) + steps for p in RAGGED_PROMPTS]


def test_graph_decoder_reproduces_the_eager_decoder_bit_for_bit(env):
    modelcore, mcb = env
    from modelcore_b200 import workloads
    mgr = mcb.ModelManager()
    model = workloads.awaken(mgr.create_model(workloads.quickstart_config(n_layer=4),
                                              device=torch.device("cuda"), seed=0))
    model.eval()
    prompts = workloads.prompts(3, 20, seed=1).tolist()
    prompts[1] = prompts[1][:7]  # ragged rows
    eager = mgr.new_decoder(model, prompts, max_tokens=16)
    graph = mgr.new_decoder(model, prompts, max_tokens=16, cuda_graph=True)
    with torch.inference_mode():
        for step in range(10):
            col = [(step * 5 + i) % 1000 for i in range(3)]
            le = eager.step(col).clone()
            lg = graph.step(col).clone()
            assert torch.equal(le, lg), step
        assert graph.kv_cache.cache_seqlens.tolist() == eager.kv_cache.cache_seqlens.tolist()
        assert graph.kv_cache.host_lens().tolist() == eager.kv_cache.cache_seqlens.tolist()
        # device-resident greedy loop == host-driven greedy loop
        g2 = mgr.new_decoder(model, prompts, max_tokens=16, cuda_graph=True)
        e2 = mgr.new_decoder(model, prompts, max_tokens=16)
        dev_tokens = g2.greedy_steps(12).cpu()
        host = []
        for _ in range(12):
            nxt = torch.argmax(e2.logits, dim=-1)
            host.append(nxt.cpu())
            e2.step(nxt.tolist())
        assert torch.equal(dev_tokens, torch.stack(host, 1))


def test_graph_decoder_steps_fed_from_the_host_back_to_back(env):
    """GraphDecoder.step(list) copies the column through a pinned host buffer with a
    non-blocking copy; steps issued back to back, with nothing on the host waiting for the GPU in
    between, must each see their own column (the buffer is not overwritten before its copy ran)."""
    modelcore, mcb = env
    from modelcore_b200 import workloads
    mgr = mcb.ModelManager()
    model = workloads.awaken(mgr.create_model(workloads.quickstart_config(n_layer=4),
                                              device=torch.device("cuda"), seed=0)).eval()
    prompts = workloads.prompts(64, 200, seed=1).tolist()
    cols = [[(s * 131 + i * 7) % 30000 for i in range(64)] for s in range(12)]
    with torch.inference_mode():
        eager = mgr.new_decoder(model, prompts, max_tokens=16)
        want = [eager.step(c).clone() for c in cols]
        graph = mgr.new_decoder(model, prompts, max_tokens=16, cuda_graph=True)
        got = [graph.step(c).clone() for c in cols]  # no host read in between
        torch.cuda.synchronize()
    for s, (a, b) in enumerate(zip(want, got)):
        assert torch.equal(a, b), s


def test_config4_broadcast_and_kv_sharing_decode_matches_the_reference(env):
    """Config 4's structure at reduced depth and width of prompt: one prompt prefilled once,
    broadcast to every row, odd layers reading the even layers' slots, windowed layers."""
    from modelcore_b200 import workloads
    cfg = workloads.gqa_window_config(n_layer=4, kv_share=True, window=64)
    ref_mgr, ref, mgr, mine = _pair(env, cfg)
    prompt = workloads.prompts(1, 150, seed=3)[0].tolist()
    with torch.inference_mode():
        a = ref_mgr.new_decoder(ref, prompt, num_samples=4, max_tokens=40)
        b = mgr.new_decoder(mine, prompt, num_samples=4, max_tokens=40)
        assert b.kv_cache.get_pos() == 150 and b.kv_cache.n_slots == 2
        for step in range(40):
            d = (a.logits.float() - b.logits.float()).abs().max().item()
            assert d <= LOGIT_TOL, (step, d)
            col = [(step * 11 + i) % 30000 for i in range(4)]
            a.step(col)
            b.step(col)
