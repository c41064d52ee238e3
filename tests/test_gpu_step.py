"""GPU parity of the decode-step kernels either side of attention, called through the C ABI
(modelcore_b200.ops): the residual add fused with the next RMSNorm, and GatedMLP's silu(gate) * up.

Bars: the add and silu * up are bit-exact against torch's own CUDA ops (one bf16 rounding per op,
the same fp32 formulas); the norm is bit-exact against the CPU oracle, which restates the kernel's
fp32 summation order, and within one bf16 ulp of torch's F.rms_norm and of the reference's golden
vectors."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import load_golden
from oracle import kv_path as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from modelcore_b200 import ops
    return ops


def dev_bf16(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).cuda()


def host_bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def ulps(a, b):
    return np.abs(a.astype(np.int32) - b.astype(np.int32))


@pytest.mark.parametrize("C", [40, 768, 2048, 4096])
def test_add_rms_norm_against_the_reference_golden_vectors(ops, C):
    z = load_golden("step_fused.npz")
    x, d = dev_bf16(z[f"x_C{C}"]), dev_bf16(z[f"delta_C{C}"])
    s, h = ops.add_rms_norm(x, d)
    torch.cuda.synchronize()
    assert np.array_equal(host_bits(s), z[f"sum_C{C}"])
    assert ulps(host_bits(h), z[f"norm_C{C}"]).max() <= 1
    assert np.array_equal(host_bits(h), O.add_rms_norm(z[f"x_C{C}"], z[f"delta_C{C}"])[1])
    _, h0 = ops.add_rms_norm(x)
    assert np.array_equal(host_bits(h0), O.add_rms_norm(z[f"x_C{C}"])[1])
    assert ulps(host_bits(h0), z[f"norm_only_C{C}"]).max() <= 1


@pytest.mark.parametrize("rows,C", [(1, 8), (3, 264), (64, 768), (129, 2048), (1000, 1536),
                                    (7, 4096)])
def test_add_rms_norm_is_bit_exact_against_the_oracle(ops, rows, C):
    g = torch.Generator(device="cuda").manual_seed(rows * 7919 + C)
    x = (torch.randn(rows, C, device="cuda", generator=g) * 4).to(torch.bfloat16)
    d = torch.randn(rows, C, device="cuda", generator=g).to(torch.bfloat16)
    s, h = ops.add_rms_norm(x, d)
    torch.cuda.synchronize()
    os_, oh = O.add_rms_norm(host_bits(x), host_bits(d))
    assert np.array_equal(host_bits(s), os_)
    assert np.array_equal(host_bits(h), oh)
    # against torch's CUDA ops: the add exactly, the norm within one ulp on rare elements
    s_t = x + d
    assert torch.equal(s, s_t)
    diff = ulps(host_bits(h), host_bits(F.rms_norm(s_t, (C,))))
    assert diff.max() <= 1
    assert (diff != 0).mean() <= 5e-3


def test_add_rms_norm_in_place_with_strided_rows(ops):
    """x_out may alias x (the residual stream updated in place); rows may be strided views."""
    rows, C = 33, 768
    g = torch.Generator(device="cuda").manual_seed(5)
    wide = (torch.randn(rows, 2 * C, device="cuda", generator=g) * 2).to(torch.bfloat16)
    x = wide[:, C:]
    d = torch.randn(rows, 3 * C, device="cuda", generator=g).to(torch.bfloat16)[:, :C]
    want_s, want_h = O.add_rms_norm(host_bits(x), host_bits(d), eps=1e-5)
    left = wide[:, :C].clone()
    h = torch.empty(rows, 2 * C, device="cuda", dtype=torch.bfloat16)[:, :C]
    s, h = ops.add_rms_norm(x, d, eps=1e-5, x_out=x, h_out=h)
    torch.cuda.synchronize()
    assert s.data_ptr() == x.data_ptr()
    assert np.array_equal(host_bits(x), want_s)
    assert np.array_equal(host_bits(h), want_h)
    assert torch.equal(wide[:, :C], left)


@pytest.mark.parametrize("rows,H", [(16, 2048), (1, 8), (64, 5632), (333, 2048)])
def test_gated_silu_is_bit_exact_against_torch(ops, rows, H):
    g = torch.Generator(device="cuda").manual_seed(rows + H)
    gu = (torch.randn(rows, 2 * H, device="cuda", generator=g) * 5).to(torch.bfloat16)
    gate, up = gu[:, :H], gu[:, H:]      # the two halves of one fused gate|up projection
    out = ops.gated_silu(gate, up)
    torch.cuda.synchronize()
    assert torch.equal(out, F.silu(gate) * up)
    assert ulps(host_bits(out), O.gated_silu(host_bits(gate), host_bits(up))).max() <= 1


def test_gated_silu_against_the_reference_golden_vectors(ops):
    z = load_golden("step_fused.npz")
    out = ops.gated_silu(dev_bf16(z["gate"]), dev_bf16(z["up"]))
    torch.cuda.synchronize()
    assert ulps(host_bits(out), z["gated"]).max() <= 1


def test_step_kernels_reject_unsupported_shapes(ops):
    from modelcore_b200._native import McbError
    x = torch.zeros(4, 12, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(McbError, match="multiple of 8"):
        ops.add_rms_norm(x)
    with pytest.raises(McbError, match="at most 4096"):
        ops.add_rms_norm(torch.zeros(2, 4104, device="cuda", dtype=torch.bfloat16))
    y = torch.zeros(4, 24, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(McbError, match="16-byte"):
        ops.add_rms_norm(y[:, 1:17])
    with pytest.raises(McbError, match="multiple of 8"):
        ops.gated_silu(x, x)


def test_embed_rms_norm_against_the_reference_and_the_oracle(ops):
    z = load_golden("step_fused.npz")
    ids = torch.from_numpy(z["ids"]).cuda()
    x, h = ops.embed_rms_norm(ids, dev_bf16(z["wte"]))
    torch.cuda.synchronize()
    ox, oh = O.embed_rms_norm(z["ids"], z["wte"])
    assert np.array_equal(host_bits(x), ox) and np.array_equal(host_bits(h), oh)
    assert ulps(host_bits(x), z["embed_x"]).max() <= 1
    assert ulps(host_bits(h), z["embed_h"]).max() <= 1


def test_embed_rms_norm_against_torch_and_out_of_range_ids(ops):
    g = torch.Generator(device="cuda").manual_seed(11)
    table = (torch.randn(5000, 2048, device="cuda", generator=g) * 0.8).to(torch.bfloat16)
    ids = torch.randint(0, 5000, (64, 1), device="cuda", generator=g)
    x, h = ops.embed_rms_norm(ids, table)
    x_t = F.rms_norm(table[ids], (2048,))
    assert (ulps(host_bits(x), host_bits(x_t)) != 0).mean() <= 5e-3
    assert ulps(host_bits(h), host_bits(F.rms_norm(x, (2048,)))).max() <= 1
    assert ops.device_error()[0] == 0
    bad = ids.clone()
    bad[3, 0] = 5000
    bad[7, 0] = -1
    xb, hb = ops.embed_rms_norm(bad, table)
    code, what = ops.device_error()
    assert code == 4, what
    assert not xb[3].any() and not hb[7].any()
    assert torch.equal(xb[5], x[5])


def _softcap_torch(lg, V, cap):
    f = lg[..., :V].float()
    return f if cap is None else cap * torch.tanh(f / cap)


@pytest.mark.parametrize("rows,Vp,V,cap", [(64, 32768, 32768, 15.0), (9, 1024, 1000, 15.0),
                                           (5, 1024, 1001, 30.0), (3, 512, 512, None)])
def test_softcap_argmax_is_bit_exact_against_torch(ops, rows, Vp, V, cap):
    """LMHead's crop + .float() + softcap as torch computes it on the GPU, and torch.argmax."""
    g = torch.Generator(device="cuda").manual_seed(rows + V)
    lg = (torch.randn(rows, Vp, device="cuda", generator=g) * 20).to(torch.bfloat16)
    lg[0, 17] = lg[0, 900 % V] = 200.0    # a tie at the maximum: the first index wins
    ids = torch.empty(rows, dtype=torch.int64, device="cuda")
    out = ops.softcap_argmax(lg, V, cap, argmax_out=ids)
    want = _softcap_torch(lg, V, cap)
    assert out.shape == (rows, V)
    assert torch.equal(out, want)
    assert torch.equal(ids, torch.argmax(want, dim=-1))
    assert ids[0].item() == 17
    only = torch.zeros(rows, 1, dtype=torch.int64, device="cuda")
    assert ops.softcap_argmax(lg, V, cap, want_logits=False, argmax_out=only) is None
    assert torch.equal(only[:, 0], ids)


@pytest.mark.parametrize("rows,V", [(1, 50257), (2, 32768), (300, 4096), (40, 7)])
def test_softcap_argmax_rows_split_over_a_cluster(ops, rows, V):
    """Rows split over up to 8 CTAs (fewer than 296 rows) or one CTA each: ties across the split
    go to the first index, a NaN anywhere wins, an all -inf row picks index 0."""
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + V)
    lg = (torch.randn(rows, V, device="cuda", generator=g) * 20).to(torch.bfloat16)
    lg[0, V - 1] = lg[0, V // 3] = 300.0      # equal maxima in different CTAs of the row
    if rows > 1:
        lg[1, V - 2] = float("nan")
        lg[1, 1] = 300.0
    if rows > 2:
        lg[rows - 1] = float("-inf")
    ids = torch.empty(rows, dtype=torch.int64, device="cuda")
    out = ops.softcap_argmax(lg, V, 15.0, argmax_out=ids)
    want = _softcap_torch(lg, V, 15.0)
    assert torch.equal(out.nan_to_num(7.0), want.nan_to_num(7.0))
    assert torch.equal(ids, torch.argmax(want, dim=-1))
    assert ids[0].item() == V // 3
    if rows > 1:
        assert ids[1].item() == V - 2
    if rows > 2:
        assert ids[rows - 1].item() == 0


def test_softcap_argmax_against_the_reference_lm_head(ops):
    z = load_golden("step_fused.npz")
    lg = dev_bf16(z["head_logits_bf16"])
    ids = torch.empty(lg.shape[0], dtype=torch.int64, device="cuda")
    out = ops.softcap_argmax(lg, 1000, 15, argmax_out=ids).cpu().numpy()
    f32 = lambda a: a.view(np.int32).astype(np.int64)
    assert np.abs(f32(out) - f32(z["head_out"])).max() <= 4
    assert np.array_equal(ids.cpu().numpy(), np.argmax(z["head_out"], axis=-1))
    # numpy's float32 tanh against the device's tanhf: a few ulps
    assert np.abs(f32(out) - f32(O.softcap_logits(z["head_logits_bf16"], 1000, 15))).max() <= 4
    nocap = ops.softcap_argmax(lg, 1000, None).cpu().numpy()
    assert np.array_equal(nocap, z["head_out_nocap"])


# ---------------------------------------------------------------------------------------------
# the fused decode step through modelcore's API (bf16 weights: the fused path's precondition)
LOGIT_TOL = 2e-2


@pytest.fixture(scope="module")
def env():
    from conftest import have_modelcore
    if not have_modelcore():
        raise RuntimeError("modelcore (the reference package) is not importable: install it into "
                           "baseline/_ref to run the end-to-end tests")
    import modelcore
    import modelcore_b200
    return modelcore, modelcore_b200


def _models(env, config):
    """The reference model, the fused B200 model and the op-by-op B200 model, all with the same
    awake bf16 weights on the GPU, plus an fp32 copy of the reference for the error yardstick."""
    import copy
    modelcore, mcb = env
    from modelcore_b200 import step, workloads
    mgr = modelcore.ModelManager()
    cpu = workloads.awaken(mgr.create_model(config, device=torch.device("cpu"), seed=0)).eval()
    ref = copy.deepcopy(cpu).to("cuda", torch.bfloat16)
    fused = copy.deepcopy(cpu).to("cuda", torch.bfloat16)
    plain = copy.deepcopy(cpu).to("cuda", torch.bfloat16)
    mcb.install(fused, fuse_step=True)
    mcb.install(plain, fuse_step=False)
    assert step.installed(fused) and not step.installed(plain)
    assert step.decode_installed(fused) and not step.decode_installed(plain)
    m32 = modelcore.ModelManager(runtime=modelcore.Runtime(compute_dtype=torch.float32))
    ref32 = m32.create_model(config, device=torch.device("cpu"), seed=0)
    ref32.load_state_dict({k: v.float().cpu() for k, v in ref.state_dict().items()})
    return (mgr, ref), (mcb.ModelManager(), fused), (mcb.ModelManager(), plain), (m32, ref32.to("cuda").eval())


@torch.inference_mode()
def _forced(mgr, model, prompts, columns):
    dec = mgr.new_decoder(model, prompts, max_tokens=columns.shape[1])
    out = []
    for i in range(columns.shape[1]):
        out.append(dec.logits.float().clone())
        dec.step(columns[:, i].tolist())
    out.append(dec.logits.float().clone())
    return torch.stack(out, 1)


def _configs():
    from modelcore_b200 import workloads
    return {
        "quickstart": lambda: workloads.quickstart_config(n_layer=4),
        "gqa_window": lambda: workloads.gqa_window_config(n_layer=4, window=16),
        "kv_share": lambda: workloads.gqa_window_config(n_layer=4, kv_share=True, window=16),
    }


@pytest.mark.parametrize("name", ["quickstart", "gqa_window", "kv_share"])
def test_fused_step_decode_is_as_accurate_as_the_reference(env, name):
    """Right-ragged prompts, fixed token columns (teacher forcing): the fused step's logits are
    within LOGIT_TOL of the fp32 reference and no further from it than the reference's own bf16
    forward (x1.25 + 1e-3); the op-by-op B200 path is the same bar's control."""
    from modelcore.tests.test_generate import RAGGED_PROMPTS
    (rm, ref), (fm, fused), (pm, plain), (m32, ref32) = _models(env, _configs()[name]())
    steps = 12
    cols = torch.tensor([[(s * 7 + i * 3) % 100 + 1 for s in range(steps)]
                         for i in range(len(RAGGED_PROMPTS))])
    l32 = _forced(m32, ref32, RAGGED_PROMPTS, cols)
    l_ref = _forced(rm, ref, RAGGED_PROMPTS, cols)
    l_fused = _forced(fm, fused, RAGGED_PROMPTS, cols)
    l_plain = _forced(pm, plain, RAGGED_PROMPTS, cols)
    e_ref = (l_ref - l32).abs().max().item()
    e_fused = (l_fused - l32).abs().max().item()
    e_plain = (l_plain - l32).abs().max().item()
    print(f"{name}: max|logits - fp32|: reference bf16 {e_ref:.3e}, fused {e_fused:.3e}, "
          f"op-by-op {e_plain:.3e}")
    assert e_fused <= LOGIT_TOL
    assert e_fused <= 1.25 * e_ref + 1e-3


PROJ_MODES = ["cublas", "linear", "linear_norm_out", "fused_proj"]


def _set_proj_mode(step, monkeypatch, mode):
    """cublas: every projection on cuBLAS; linear: every projection on mcb_linear, c_proj with the
    residual add in its epilogue (USE_LINEAR_PROJ) and the norm after it a launch of its own;
    linear_norm_out: the same with c_proj's norm in its epilogue too (USE_LINEAR_NORM_OUT, the
    default); fused_proj: the projections on mcb_linear with the norms and adds fused into them
    (USE_FUSED_PROJ)."""
    monkeypatch.setattr(step, "USE_FUSED_PROJ", mode == "fused_proj")
    monkeypatch.setattr(step, "USE_LINEAR_PROJ", mode in ("linear", "linear_norm_out"))
    monkeypatch.setattr(step, "USE_LINEAR_NORM_OUT", mode == "linear_norm_out")


@pytest.mark.parametrize("mode", PROJ_MODES)
def test_fused_step_launches_and_graph_replay(env, mode, monkeypatch):
    """One decode step of the fused 4-layer quickstart launches the libmcb200 kernels it should
    (per layer: the projections it runs, the add + norms, silu * up, append, attention; plus the
    embedding, the last add + norm, the advance and the LM-head epilogue),
    and the CUDA-graph decoder reproduces the eager fused decoder bit for bit."""
    modelcore, mcb = env
    from modelcore_b200 import integration, ops, step, workloads
    _set_proj_mode(step, monkeypatch, mode)
    fused_proj = mode == "fused_proj"
    mgr = mcb.ModelManager()
    model = workloads.awaken(mgr.create_model(workloads.quickstart_config(n_layer=4),
                                              device=torch.device("cuda"), seed=0))
    model = model.to(torch.bfloat16).eval()
    prompts = workloads.prompts(3, 20, seed=1).tolist()
    prompts[2] = prompts[2][:9]
    eager = mgr.new_decoder(model, prompts, max_tokens=16)
    graph = mgr.new_decoder(model, prompts, max_tokens=16, cuda_graph=True)
    cols = [[1, 2, 3]] + [[(s * 5 + i) % 1000 for i in range(3)] for s in range(1, 7)]
    with torch.inference_mode():
        n0 = ops.launch_count()
        eager.step(cols[0])
        per_step = ops.launch_count() - n0
        # the append runs inside the attention launch (integration.USE_FUSED_APPEND; these rows
        # take the split plan) or as its own launch
        append = 0 if integration.USE_FUSED_APPEND else 1
        if fused_proj:
            # the embedding; per layer q|k|v (add + norm inside), append, c_proj (+ residual),
            # gate|up (norm inside), silu * up (down_proj is cuBLAS); the final add + norm, the
            # advance, the LM-head epilogue
            attn_launches = per_step - (1 + 4 * (4 + append) + 1 + 1 + 1)
        elif mode == "linear":
            # embedding + first norm, per layer q|k|v, c_proj (+ residual), the norm, gate|up
            # with silu * up in its epilogue, down_proj, the add + norm and the append, the
            # advance, the LM-head epilogue
            attn_launches = per_step - (1 + 4 * (6 + append) + 1 + 1)
        elif mode == "linear_norm_out":
            # the same with the norm inside c_proj's launch, where the device schedules it
            if not all(step._NORM_OUT_OK.values()):
                pytest.skip("the device does not schedule mcb_linear's norm-out clusters")
            attn_launches = per_step - (1 + 4 * (5 + append) + 1 + 1)
        else:
            # embedding + first norm, per layer two add + norms, silu * up and the append, the
            # advance, the LM-head epilogue
            attn_launches = per_step - (1 + 4 * (3 + append) + 1 + 1)
        assert attn_launches == 4, per_step           # one per layer
        graph.step(cols[0])                           # eager: the graph decoder's first step
        for col in cols[1:]:                          # capture, then replays
            assert torch.equal(eager.step(col), graph.step(col))
        # the device-resident greedy loop (greedy pick fused into the LM-head epilogue) equals
        # the host-driven loop over torch.argmax
        g2 = mgr.new_decoder(model, prompts, max_tokens=16, cuda_graph=True)
        e2 = mgr.new_decoder(model, prompts, max_tokens=16)
        dev_tokens = g2.greedy_steps(12).cpu()
        host = []
        for _ in range(12):
            nxt = torch.argmax(e2.logits, dim=-1)
            host.append(nxt.cpu())
            e2.step(nxt.tolist())
        assert torch.equal(dev_tokens, torch.stack(host, 1))
        assert torch.equal(g2.logits, e2.logits)
        # step_greedy: host column in, host greedy tokens out, one graph per step
        g3 = mgr.new_decoder(model, prompts, max_tokens=16, cuda_graph=True)
        e3 = mgr.new_decoder(model, prompts, max_tokens=16)
        tok = torch.argmax(e3.logits, dim=-1).cpu()
        for _ in range(8):
            nxt = g3.step_greedy(tok).clone()
            want = torch.argmax(e3.step(tok.tolist()), dim=-1).cpu()
            assert torch.equal(nxt, want)
            assert torch.equal(g3.logits, e3.logits)
            tok = nxt
        # the returned tensor fed straight back as the next column (no host copy: the tokens
        # come back in the buffer the column goes in by) gives the same stream
        g4 = mgr.new_decoder(model, prompts, max_tokens=16, cuda_graph=True)
        e4 = mgr.new_decoder(model, prompts, max_tokens=16)
        tok = torch.argmax(e4.logits, dim=-1).cpu()
        out = g4.step_greedy(tok)
        for _ in range(8):
            want = torch.argmax(e4.step(tok.tolist()), dim=-1).cpu()
            assert torch.equal(out, want)
            assert torch.equal(g4.logits, e4.logits)
            tok = want
            again = g4.step_greedy(out)
            assert again is out  # the same pinned view, now holding the next tokens
            out = again


def test_packed_weights_follow_the_parameters(env):
    """The packed [Wq; Wk; Wv] and [Wg; Wu] are the Parameters' own storage: the state dict keeps
    its keys and shapes, load_state_dict lands in the packed buffer, and replacing the storage
    (model.to) re-packs on the next forward."""
    modelcore, mcb = env
    from modelcore_b200 import workloads
    mgr = mcb.ModelManager()
    model = workloads.awaken(mgr.create_model(workloads.quickstart_config(n_layer=2),
                                              device=torch.device("cuda"), seed=0))
    model = model.to(torch.bfloat16).eval()
    keys = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    prompts = workloads.prompts(2, 8, seed=3).tolist()

    def logits():
        with torch.inference_mode():
            return mgr.new_decoder(model, prompts, max_tokens=4).step([5, 6]).float().clone()

    first = logits()
    attn = model.body.blocks[0].mixer
    wq, wk = attn.c_q.weight, attn.c_k.weight
    assert wk.data_ptr() == wq.data_ptr() + wq.numel() * wq.element_size()
    assert {k: tuple(v.shape) for k, v in model.state_dict().items()} == keys
    # new weights through load_state_dict: the fused forward sees them
    sd = {k: v.clone() for k, v in model.state_dict().items()}
    with torch.no_grad():
        for k in sd:
            if k.endswith(("c_k.weight", "gate_proj.weight")):
                sd[k].mul_(-1.5)
    model.load_state_dict(sd)
    changed = logits()
    control = copy_with_plain_forward(env, model)
    assert (changed - first).abs().max().item() > 0
    assert (changed - control).abs().max().item() <= LOGIT_TOL
    # storage replaced: re-packed on the next forward
    model.to(torch.float32).to(torch.bfloat16)
    again = logits()
    assert torch.equal(again, changed)


def copy_with_plain_forward(env, model):
    import copy
    _, mcb = env
    other = copy.deepcopy(model)
    mcb.install(other, fuse_step=False)
    with torch.inference_mode():
        from modelcore_b200 import workloads
        prompts = workloads.prompts(2, 8, seed=3).tolist()
        return mcb.ModelManager().new_decoder(other, prompts, max_tokens=4).step([5, 6]).float().clone()


@pytest.mark.parametrize("mode", PROJ_MODES)
def test_fused_step_projection_paths_are_as_accurate(env, mode, monkeypatch):
    """The same bar with every decode projection on cuBLAS, with q|k|v and c_proj (+ residual)
    on libmcb200's mcb_linear (USE_LINEAR_PROJ, body_forward_linear), and with the projections on
    mcb_linear with the norms and residual adds fused into them (USE_FUSED_PROJ,
    body_forward_proj)."""
    from modelcore.tests.test_generate import RAGGED_PROMPTS
    from modelcore_b200 import step
    _set_proj_mode(step, monkeypatch, mode)
    (rm, ref), (fm, fused), _, (m32, ref32) = _models(env, _configs()["quickstart"]())
    cols = torch.tensor([[(s * 7 + i * 3) % 100 + 1 for s in range(8)]
                         for i in range(len(RAGGED_PROMPTS))])
    l_fused = _forced(fm, fused, RAGGED_PROMPTS, cols)
    l32 = _forced(m32, ref32, RAGGED_PROMPTS, cols)
    l_ref = _forced(rm, ref, RAGGED_PROMPTS, cols)
    e_ref = (l_ref - l32).abs().max().item()
    e_fused = (l_fused - l32).abs().max().item()
    assert e_fused <= LOGIT_TOL
    assert e_fused <= 1.25 * e_ref + 1e-3


@pytest.mark.parametrize("samples", [1, 3])
def test_batched_prefill_matches_per_prompt_prefill(env, samples):
    """GraphDecoder's one-forward ragged prefill against modelcore's per-prompt prefill
    (Decoder, batch-1 forwards + prefill_row): same row lengths, logits within LOGIT_TOL, and the
    first decode steps' logits too (the caches hold the same keys up to GEMM summation order)."""
    modelcore, mcb = env
    from modelcore_b200 import workloads
    mgr = mcb.ModelManager()
    model = workloads.awaken(mgr.create_model(workloads.quickstart_config(n_layer=4),
                                              device=torch.device("cuda"), seed=0))
    model = model.to(torch.bfloat16).eval()
    prompts = workloads.prompts(5, 150, seed=4).tolist()
    for i, n in enumerate((150, 3, 77, 128, 1)):
        prompts[i] = prompts[i][:n]
    with torch.inference_mode():
        fast = mgr.new_decoder(model, prompts, num_samples=samples, max_tokens=8, cuda_graph=True)
        slow = mgr.new_decoder(model, prompts, num_samples=samples, max_tokens=8, cuda_graph=True,
                               batched_prefill=False)
        assert fast.kv_cache.cache_seqlens.tolist() == slow.kv_cache.cache_seqlens.tolist()
        assert fast.kv_cache.host_lens().tolist() == slow.kv_cache.cache_seqlens.tolist()
        assert (fast.logits - slow.logits).abs().max().item() <= LOGIT_TOL
        for s in range(4):
            col = [(s * 13 + r) % 500 for r in range(5 * samples)]
            a, b = fast.step(col), slow.step(col)
            assert (a - b).abs().max().item() <= LOGIT_TOL, s
