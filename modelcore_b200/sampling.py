"""sample_next_token on libmcb200: modelcore/generate.py:19-34 with the same signature.

The reference draws with torch.multinomial from softmax(topk(logits) / T); here one kernel
(mcb_sample) selects the top-k, forms the softmax and draws by the inverse CDF at a uniform taken
from `rng` (torch.rand), so the draw has the reference's distribution; the exact token for a given
generator state differs from torch.multinomial's, as it would between any two sampler
implementations.  temperature == 0 is the greedy pick (the first index of the row maximum)."""
import torch

from . import ops


@torch.inference_mode()
def sample_next_token(logits, rng, temperature=1.0, top_k=None):
    """Sample a single next token from given logits of shape (B, vocab_size). Returns (B, 1)."""
    assert temperature >= 0.0, "temperature must be non-negative"
    logits = logits if logits.dtype == torch.float32 else logits.float()
    B = logits.size(0)
    if temperature == 0.0:
        u = torch.zeros(B, dtype=torch.float32, device=logits.device)
        return ops.sample(logits, u, temperature=0.0)
    if rng is None or rng.device.type == logits.device.type:
        u = torch.rand(B, generator=rng, dtype=torch.float32, device=logits.device)
    else:  # a host generator: draw on the host, copy the B uniforms over
        u = torch.rand(B, generator=rng, dtype=torch.float32).to(logits.device)
    return ops.sample(logits, u, temperature=temperature, top_k=top_k)
