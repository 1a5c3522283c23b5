"""PackedCausalLM on the CPU: the training model and the decoder agree.

The whole-sequence causal forward of PackedCausalLM (the fine-tuning model)
gives, at the last position, the logits that PackedDecoder.prefill gives for
the same prompt and stores (both in the reference's materialize formulation
on the CPU); make_trainable(mode="both") finds every projection's scales and
codebook; a ScaleTuner loop lowers the loss and leaves the indices alone.
"""
import torch

from epure.finetune import ScaleTuner, make_trainable
from epure.model import PackedCausalLM, PackedDecoder
from epure.synthetic import DecoderShapes


def _decoder(name, seed=1):
    return PackedDecoder(DecoderShapes(name, 2, 256, 512, 4, 2, 64, 100), device="cpu", seed=seed,
                         max_len=64, linear_mode="reference", fp32_logits=False)


def test_last_position_matches_decoder_prefill():
    for name in ("qwen3-tiny", "llama3-tiny"):
        dec = _decoder(name)
        ids = torch.randint(0, 100, (12,), generator=torch.Generator().manual_seed(2))
        want = dec.prefill(ids).float()
        got = PackedCausalLM(dec, "reference").logits(ids[None])[0, -1].float()
        err = float((got - want).abs().max() / want.abs().max())
        assert err <= 2e-2, (name, err)


def test_make_trainable_finds_every_projection():
    model = PackedCausalLM(_decoder("qwen3-tiny"), "ours")
    params = make_trainable(model, "both")
    assert len(params) == 2 * 7 * 2
    assert all(p.dtype == torch.float32 and p.requires_grad for p in params)


def test_scale_tuner_lowers_the_loss_on_cpu():
    model = PackedCausalLM(_decoder("llama3-tiny", seed=4), "ours")
    tuner = ScaleTuner(model, mode="both", lr=3e-3, device=torch.device("cpu"))
    ids = torch.randint(0, 100, (2, 24), generator=torch.Generator().manual_seed(5))
    losses = [tuner.step(ids) for _ in range(6)]
    assert losses[-1] < losses[0] - 0.02, losses
    tuner.finish()
