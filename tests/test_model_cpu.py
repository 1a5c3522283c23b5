"""PackedDecoder's host-side model code on the CPU (reference / float32 linear modes).

The KV-cache decode path must give the logits a full prefill of the same
tokens gives (attention mask, RoPE positions, cache writes), and the
reference's bf16 formulation stays within bf16 tolerance of float32.
"""
import torch

from epure.synthetic import DecoderShapes

TINY = DecoderShapes("tiny", 2, 256, 512, 4, 2, 64, 300)


def _model(mode):
    from epure.model import PackedDecoder
    m = PackedDecoder(TINY, device="cpu", seed=5, max_len=32, linear_mode="fp32")
    return m if mode == "fp32" else m.share_weights(mode)


def test_cached_decode_equals_prefill():
    m = _model("fp32")
    g = torch.Generator().manual_seed(0)
    toks = torch.randint(0, TINY.vocab, (10,), generator=g)
    m.prefill(toks[:6])
    step_logits = []
    for t in range(6, 10):
        step_logits.append(m.step(toks[t:t + 1], torch.tensor([t])))
    for t in range(6, 10):
        fresh = _model("fp32")
        full = fresh.prefill(toks[:t + 1])
        assert torch.allclose(step_logits[t - 6], full, rtol=1e-4, atol=1e-5), t


def test_reference_bf16_close_to_fp32():
    f32 = _model("fp32")
    ref = f32.share_weights("reference")
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, TINY.vocab, (8,), generator=g)
    a, b = ref.prefill(prompt), f32.prefill(prompt)
    assert float((a - b).abs().max() / b.abs().max()) <= 3e-2
