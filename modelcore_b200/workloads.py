"""The measured workloads as modelcore config trees and seeded synthetic inputs.

  quickstart_config()        12 blocks x n_embd 768, 12 q / 12 kv heads of 64, full window, gated
                             SiLU MLP 2048, rms_norm QK-norm, rotary, softcap 15, vocab 32768
                             (modelcore README quickstart; measurement configs 1 and 2)
  gqa_window_config()        24 blocks x n_embd 2048, 16 q / 4 kv heads of 128, gated MLP 5632,
                             window 1024 on layers i % 4 != 3 and full context on i % 4 == 3
                             (config 3); kv_share=True makes every odd layer a consumer
                             (produces_kv=False) of the preceding even layer's slot (config 4),
                             with explicit kv_slot = i // 2 on every layer -- modelcore's validator
                             requires contiguous slots (modelcore/config/validate.py:166-168)
  awaken(model)              modelcore's own test wake-up (modelcore/tests/test_generate.py:187-201):
                             every zero-initialised parameter gets N(0, 0.1) values, so attention
                             actually reaches the logits
  prompts(B, P, seed)        token ids uniform in [0, 32768) from a seeded torch.Generator

There is no public dataset behind these numbers: inputs are seeded synthetic tokens of the
configured shapes, weights are random-init of the named architecture.
"""
import torch


def quickstart_config(n_layer=12, sequence_len=1024):
    from modelcore import ComponentSpec, ModelConfig
    head_dim = 64
    return ModelConfig(
        sequence_len=sequence_len, vocab_size=32768, n_embd=768, pad_vocab_size_to=64, template="base",
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
            for i in range(n_layer)
        ]}),
        output=ComponentSpec("lm_head", {"softcap": 15}),
    )


def gqa_window_config(n_layer=24, kv_share=False, window=1024, sequence_len=1024, over_compute=10):
    from modelcore import ComponentSpec, ModelConfig
    head_dim = 128
    blocks = []
    for i in range(n_layer):
        w = -1 if i % 4 == 3 else window
        if kv_share:
            slot, produces = i // 2, (i % 2 == 0)
        else:
            slot, produces = None, True
        blocks.append(ComponentSpec("block", {
            "layer_idx": i, "features": [],
            "mixer": ComponentSpec("attention", {"n_head": 16, "n_kv_head": 4, "head_dim": head_dim,
                                                 "window": w, "kv_slot": slot, "produces_kv": produces,
                                                 "features": []}),
            "ffn": ComponentSpec("gated_mlp", {"activation": "silu", "hidden_dim": 5632}),
        }))
    return ModelConfig(
        sequence_len=sequence_len, vocab_size=32768, n_embd=2048, pad_vocab_size_to=64, template="base",
        shared={"rope": ComponentSpec("rotary", {"head_dim": head_dim, "over_compute": over_compute}),
                "norm": ComponentSpec("rms_norm", {"eps": None})},
        input=ComponentSpec("token_embedding", {"smear": False}),
        body=ComponentSpec("stack", {"features": [], "blocks": blocks}),
        output=ComponentSpec("lm_head", {"softcap": 15}),
    )


@torch.no_grad()
def awaken(model, seed=0):
    g = torch.Generator().manual_seed(seed + 1)
    for p in model.parameters():
        if p.numel() and p.abs().sum() == 0:
            p.copy_(torch.randn(p.shape, generator=g).to(p.dtype).to(p.device) * 0.1)
    return model


def prompts(batch, length, seed, vocab=32768):
    return torch.randint(0, vocab, (batch, length), generator=torch.Generator().manual_seed(seed))
