"""Writes the golden fixtures under tests/golden/ by running the reference (modelcore) itself.

    python tests/golden/make_golden.py [--ref PATH]

PATH is a directory from which `import modelcore` loads the reference: the MODELCORE_REF_PATH
environment variable, else the repository's baseline/_ref install of it.  The fixtures are small
.npz files; bf16 tensors are stored as uint16 bit patterns.  Every value written is what the
reference's own code returned for the stated inputs, so the oracle (oracle/kv_path.py) is pinned
against the reference through tests/test_oracle_golden.py, and the GPU tests compare the CUDA path
against the same numbers without needing the reference at run time.

Fixtures:
  rope_norm_D{64,128}.npz   RotaryEmbedding._cos_sin on a right-ragged cache + apply_rotary_emb +
                            RMSNorm(eps=None) + x1.2 in bf16 (modelcore/components/rotary.py:43-67,
                            rope.py:4-12, norm.py:43-44, attention.py:147-150)
  kv_attn_*.npz             flash_attn_with_kvcache's SDPA path in fp32 on bf16-representable
                            inputs: the cache after the insert and the attention output
                            (modelcore/kernels/flash_attn.py:306-366), ragged and uniform rows,
                            windows -1 / 8, T_new 1 / 3, MHA and GQA
  prefill.npz               KVCache.prefill broadcast and prefill_row (modelcore/cache.py:75-119)
  step_fused.npz            Block's residual add + RMSNorm(eps=None) in bf16 (modelcore/components/
                            block.py:57-59, norm.py:43-44) for C in 40 / 768 / 2048 / 4096, and
                            GatedMLP's act(gate) * up with activation "silu" in bf16
                            (modelcore/components/mlp.py:89-90); TokenEmbedding without smear
                            then the first norm (embedding.py:71-75); LMHead with softcap 15 and
                            without (unembedding.py:50-56): its bf16 logits and fp32 outputs
  v2_llama*.npz             modelcore's own real-weight goldens (modelcore/tests/goldens/v2_llama.pt,
                            v2_llama_kvshare_win_gated_block.pt: awake weights, an input (2, 12) and
                            the full-forward logits the v2 code produced), passed through modelcore's
                            own v2 -> v3 upgrade (config.upgrade.upgrade_v2_to_v3 and
                            convert.convert_state_v2_to_v3, the path test_v3_migration.py:43-52
                            checks bit-exact): the v3 config as JSON, the v3 state (fp32) and the
                            golden idx / logits.  The goldens ship in the reference's source tree
                            only (not in its installed package): --ref-src names that tree
  decode_cfg1.npz           the README quickstart model (fp32, seed 0), prompts (2, 16) from seed 1,
                            64 greedy steps through Decoder: the token streams, for the plain
                            random init and for the awake init of
                            modelcore/tests/test_generate.py:187-201
"""
import argparse
import os
import sys
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _import_reference(path):
    sys.path.insert(0, path)
    import torch  # noqa: F401
    import modelcore  # noqa: F401
    return modelcore


def bits(t):
    """bf16 tensor -> uint16 numpy bits."""
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def bf16_representable(t):
    import torch
    return t.to(torch.bfloat16).to(torch.float32)


def make_rope_norm(out_dir):
    import torch
    from modelcore.cache import KVCache
    from modelcore.components.norm import RMSNorm
    from modelcore.components.rope import apply_rotary_emb
    from modelcore.components.rotary import RotaryEmbedding
    from modelcore.runtime import Runtime

    for D in (64, 128):
        g = torch.Generator().manual_seed(100 + D)
        rot = RotaryEmbedding(head_dim=D, sequence_len=64, over_compute=2,
                              runtime=Runtime(compute_dtype=torch.bfloat16))
        rot.init_weights()
        B, T, H = 3, 2, 5
        cache = KVCache(batch_size=B, n_kv_head=H, seq_len=128, head_dim=D, num_kv_slots=1,
                        device="cpu", dtype=torch.bfloat16)
        seqlens = torch.tensor([5, 40, 117], dtype=torch.int32)
        cache.cache_seqlens.copy_(seqlens)
        cache._pos_uniform = None
        x = (torch.randn(B, T, H, D, generator=g) * 2.0).to(torch.bfloat16)
        cos, sin = rot._cos_sin(T, cache)
        y = apply_rotary_emb(x, cos, sin)
        n = RMSNorm(eps=None)(y)
        z = n * 1.2
        np.savez_compressed(os.path.join(out_dir, f"rope_norm_D{D}.npz"),
                 x=bits(x), seqlens=seqlens.numpy(), cos_table=bits(rot.cos[0, :, 0]),
                 sin_table=bits(rot.sin[0, :, 0]), rope=bits(y), norm=bits(n), out=bits(z))


def make_kv_attn(out_dir):
    import torch
    import modelcore.kernels.flash_attn as fa

    cases = [
        # name, seqlens, Hq, Hkv, D, T_new, window, Tmax
        ("ragged_mha_d16_t1_wfull", [4, 17, 31, 9], 4, 4, 16, 1, -1, 48),
        ("ragged_mha_d16_t1_w8", [4, 17, 31, 9], 4, 4, 16, 1, 8, 48),
        ("ragged_mha_d16_t3_wfull", [4, 17, 31, 9], 4, 4, 16, 3, -1, 48),
        ("ragged_mha_d16_t3_w8", [4, 17, 31, 9], 4, 4, 16, 3, 8, 48),
        ("uniform_mha_d16_t1_w8", [13, 13], 4, 4, 16, 1, 8, 48),
        ("ragged_gqa_d64_t1_wfull", [0, 5, 70, 129], 8, 2, 64, 1, -1, 160),
        ("ragged_gqa_d128_t1_w33", [1, 40, 100], 8, 2, 128, 1, 33, 128),
        ("ragged_gqa_d128_t2_wfull", [3, 64, 65], 16, 4, 128, 2, -1, 80),
        ("uniform_mha_d64_t1_wfull", [77, 77], 12, 12, 64, 1, -1, 96),
        ("ragged_mha_d32_t1_w0", [6, 2], 4, 4, 32, 1, 0, 16),
        ("ragged_gqa_d256_t1_w20", [30, 7], 4, 1, 256, 1, 20, 40),
    ]
    fa._override_impl = "sdpa"
    for name, seqlens, Hq, Hkv, D, T, window, Tmax in cases:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        B = len(seqlens)
        r = lambda *s: bf16_representable(torch.randn(*s, generator=g))
        k_cache = torch.zeros(B, Tmax, Hkv, D)
        v_cache = torch.zeros_like(k_cache)
        for i, L in enumerate(seqlens):
            k_cache[i, :L] = r(L, Hkv, D)
            v_cache[i, :L] = r(L, Hkv, D)
        # stale garbage past each row's content: must be unreachable (test_kernels.py:487-498)
        for i, L in enumerate(seqlens):
            k_cache[i, L + T:] = bf16_representable(torch.full((Tmax - L - T, Hkv, D), 3.0))
            v_cache[i, L + T:] = bf16_representable(torch.full((Tmax - L - T, Hkv, D), -3.0))
        q, k, v = r(B, T, Hq, D), r(B, T, Hkv, D), r(B, T, Hkv, D)
        cs = torch.tensor(seqlens, dtype=torch.int32)
        kc0, vc0 = k_cache.clone(), v_cache.clone()
        y = fa.flash_attn_with_kvcache(q, k_cache, v_cache, k=k, v=v, cache_seqlens=cs,
                                       causal=True, window_size=(window, 0))
        b16 = lambda t: bits(t.to(torch.bfloat16))
        np.savez_compressed(os.path.join(out_dir, f"kv_attn_{name}.npz"),
                 seqlens=cs.numpy(), window=np.int64(window), q=b16(q), k=b16(k), v=b16(v),
                 k_cache_before=b16(kc0), v_cache_before=b16(vc0),
                 k_cache_after=b16(k_cache), v_cache_after=b16(v_cache), y=y.numpy())
    fa._override_impl = None


def make_prefill(out_dir):
    import torch
    from modelcore.cache import KVCache

    g = torch.Generator().manual_seed(7)
    S, H, D = 2, 2, 16

    def filled(n):
        c = KVCache(batch_size=1, n_kv_head=H, seq_len=n, head_dim=D, num_kv_slots=S, device="cpu",
                    dtype=torch.float32)
        c.k_cache.copy_(bf16_representable(torch.randn(c.k_cache.shape, generator=g)))
        c.v_cache.copy_(bf16_representable(torch.randn(c.v_cache.shape, generator=g)))
        c.advance(n)
        return c

    src = filled(7)
    dst = KVCache(batch_size=4, n_kv_head=H, seq_len=24, head_dim=D, num_kv_slots=S, device="cpu",
                  dtype=torch.float32)
    dst.prefill(src)
    a, b = filled(5), filled(11)
    rows = KVCache(batch_size=3, n_kv_head=H, seq_len=24, head_dim=D, num_kv_slots=S, device="cpu",
                   dtype=torch.float32)
    rows.prefill_row(1, a)
    rows.prefill_row(2, b)
    b16 = lambda t: bits(t.to(torch.bfloat16))
    np.savez_compressed(os.path.join(out_dir, "prefill.npz"),
             src_k=b16(src.k_cache), src_v=b16(src.v_cache), bcast_k=b16(dst.k_cache),
             bcast_v=b16(dst.v_cache), bcast_seqlens=dst.cache_seqlens.numpy(),
             row_a_k=b16(a.k_cache), row_a_v=b16(a.v_cache), row_b_k=b16(b.k_cache),
             row_b_v=b16(b.v_cache), rows_k=b16(rows.k_cache), rows_v=b16(rows.v_cache),
             rows_seqlens=rows.cache_seqlens.numpy())


def make_step_fused(out_dir):
    import torch
    from modelcore.components.mlp import GatedMLP
    from modelcore.components.norm import RMSNorm

    out = {}
    norm = RMSNorm(eps=None)
    g = torch.Generator().manual_seed(zlib.crc32(b"step_fused"))
    for C in (40, 768, 2048, 4096):
        rows = 37
        x = (torch.randn(rows, C, generator=g) * 3).to(torch.bfloat16)
        d = (torch.randn(rows, C, generator=g) * 0.5).to(torch.bfloat16)
        x1 = x + d
        out[f"x_C{C}"], out[f"delta_C{C}"] = bits(x), bits(d)
        out[f"sum_C{C}"], out[f"norm_C{C}"] = bits(x1), bits(norm(x1))
        out[f"norm_only_C{C}"] = bits(norm(x))
    mlp = GatedMLP(n_embd=64, activation="silu", hidden_dim=2048)
    gate = (torch.randn(16, 2048, generator=g) * 6).to(torch.bfloat16)
    up = torch.randn(16, 2048, generator=g).to(torch.bfloat16)
    out["gate"], out["up"], out["gated"] = bits(gate), bits(up), bits(mlp.act(gate) * up)
    # TokenEmbedding (no smear) + the first block's norm
    from modelcore.components.embedding import TokenEmbedding
    from modelcore.components.unembedding import LMHead
    from modelcore.runtime import Runtime
    emb = TokenEmbedding(padded_vocab_size=1024, n_embd=768, norm=norm, smear=False,
                         runtime=Runtime(compute_dtype=torch.bfloat16))
    emb.init_weights()
    ids = torch.randint(0, 1024, (3, 7), generator=g)
    ids[0, 0], ids[2, 6] = 0, 1023
    with torch.no_grad():
        xe = emb(ids)
    out["wte"], out["ids"], out["embed_x"], out["embed_h"] = (bits(emb.wte.weight), ids.numpy(),
                                                              bits(xe), bits(norm(xe)))
    # LMHead: norm, projection, crop, .float(), softcap
    head = LMHead(n_embd=64, vocab_size=1000, padded_vocab_size=1024, norm=norm, softcap=15)
    with torch.no_grad():
        head.lm_head.weight.copy_(torch.randn(1024, 64, generator=g) * 3)
    head = head.to(torch.bfloat16)
    xh = torch.randn(9, 64, generator=g).to(torch.bfloat16)
    out["head_x"] = bits(xh)
    with torch.no_grad():
        out["head_logits_bf16"] = bits(head.lm_head(head.norm(xh)))
        out["head_out"] = head(xh).numpy()
        head.softcap = None
        out["head_out_nocap"] = head(xh).numpy()
    np.savez_compressed(os.path.join(out_dir, "step_fused.npz"), **out)


def quickstart_config():
    from modelcore import ComponentSpec, ModelConfig
    head_dim = 64
    return ModelConfig(
        sequence_len=1024, vocab_size=32768, n_embd=768, pad_vocab_size_to=64, template="base",
        shared={"rope": ComponentSpec("rotary", {"head_dim": head_dim, "over_compute": 10}),
                "norm": ComponentSpec("rms_norm", {"eps": None})},
        input=ComponentSpec("token_embedding", {"smear": False}),
        body=ComponentSpec("stack", {"features": [], "blocks": [
            ComponentSpec("block", {
                "layer_idx": i, "features": [],
                "mixer": ComponentSpec("attention", {"n_head": 12, "n_kv_head": 12, "head_dim": head_dim,
                                                     "window": -1, "kv_slot": None, "produces_kv": True,
                                                     "features": []}),
                "ffn": ComponentSpec("gated_mlp", {"activation": "silu", "hidden_dim": 2048}),
            })
            for i in range(12)
        ]}),
        output=ComponentSpec("lm_head", {"softcap": 15}),
    )


def make_decode_cfg1(out_dir, steps=64):
    import torch
    from modelcore import ModelManager
    from modelcore.generate import sample_next_token

    manager = ModelManager()
    out = {}
    for variant in ("random", "awake"):
        model = manager.create_model(quickstart_config(), device=torch.device("cpu"), seed=0)
        if variant == "awake":
            g = torch.Generator().manual_seed(1)
            with torch.no_grad():
                for p in model.parameters():
                    if p.numel() and p.abs().sum() == 0:
                        p.copy_(torch.randn(p.shape, generator=g) * 0.1)
        model.eval()
        prompts = torch.randint(0, 32768, (2, 16), generator=torch.Generator().manual_seed(1))
        dec = manager.new_decoder(model, prompts.tolist(), max_tokens=steps)
        toks, margins = [], []
        for _ in range(steps):
            logits = dec.logits
            top2 = torch.topk(logits, 2, dim=-1).values
            margins.append((top2[:, 0] - top2[:, 1]).numpy())
            nxt = sample_next_token(logits, rng=None, temperature=0.0)[:, 0]
            toks.append(nxt.numpy())
            dec.step(nxt.tolist())
        out[f"{variant}_tokens"] = np.stack(toks, axis=1)
        out[f"{variant}_margins"] = np.stack(margins, axis=1).astype(np.float32)
        out["prompts"] = prompts.numpy()
    np.savez_compressed(os.path.join(out_dir, "decode_cfg1.npz"), **out)


V2_GOLDENS = ("v2_llama.pt", "v2_llama_kvshare_win_gated_block.pt")


def make_v2_goldens(out_dir, ref_src):
    """The reference's real-weight goldens in v3 form (see the module docstring).  The upgraded
    model's own fp32 forward is checked against the golden logits (within 1e-5: the goldens are
    bit-exact on the CPU that wrote them, fp32 BLAS order differs elsewhere) before anything is
    written."""
    import json
    import torch
    from modelcore import ModelConfig, ModelManager, Runtime
    from modelcore.config.upgrade import upgrade_v2_to_v3
    from modelcore.convert import convert_state_v2_to_v3

    gdir = os.path.join(ref_src, "modelcore", "tests", "goldens")
    for name in V2_GOLDENS:
        golden = torch.load(os.path.join(gdir, name), map_location="cpu")
        cfg = upgrade_v2_to_v3(golden["config"])
        state = convert_state_v2_to_v3(golden["state"])
        mgr = ModelManager(runtime=Runtime(compute_dtype=torch.float32))
        model = mgr.create_model(ModelConfig.from_dict(cfg), device=torch.device("cpu"), seed=0)
        model.load_state_dict(state)
        with torch.no_grad():  # bit-exact on the CPU that wrote them; within fp32 BLAS noise here
            err = (model.eval()(golden["idx"]) - golden["logits"]).abs().max().item()
        assert err <= 1e-5, (name, err)
        out = {"config_json": np.frombuffer(json.dumps(cfg).encode(), dtype=np.uint8),
               "idx": golden["idx"].numpy(), "logits": golden["logits"].numpy(),
               "state_keys": np.array(sorted(state))}
        for i, key in enumerate(sorted(state)):
            out[f"state_{i}"] = state[key].float().numpy()
        np.savez_compressed(os.path.join(out_dir, name.replace(".pt", ".npz")), **out)


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--ref", default=os.environ.get("MODELCORE_REF_PATH",
                                                    os.path.join(REPO, "baseline", "_ref")))
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--ref-src", default=os.environ.get("MODELCORE_REFERENCE_SRC",
                                                        os.path.join(os.path.dirname(REPO), "reference")),
                    help="the reference's source tree (its tests/goldens are not installed)")
    ap.add_argument("--skip-decode", action="store_true")
    ap.add_argument("--only-v2", action="store_true", help="write only the v2_*.npz fixtures")
    args = ap.parse_args()
    os.environ.setdefault("MODELCORE_DTYPE", "float32")
    _import_reference(args.ref)
    import torch
    torch.manual_seed(0)
    make_v2_goldens(args.out, args.ref_src)
    if args.only_v2:
        print("wrote fixtures to", args.out)
        return
    make_rope_norm(args.out)
    make_kv_attn(args.out)
    make_prefill(args.out)
    make_step_fused(args.out)
    if not args.skip_decode:
        make_decode_cfg1(args.out)
    print("wrote fixtures to", args.out)


if __name__ == "__main__":
    main()
