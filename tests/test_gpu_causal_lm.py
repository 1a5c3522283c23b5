"""Whole-model compressed-state fine-tuning on the GPU (epure.model.PackedCausalLM).

A 2-layer Qwen3-shaped model (q/k RMSNorm, tied lm_head, GQA) and a 2-layer
Llama-shaped one, with make_trainable(mode="both"): one forward + next-token
cross-entropy + backward through libepq.so's packed GEMM forward and fused
backward, against torch autograd of the reference formulation (every packed
linear as F.linear over materialize(bf16), fp32 scales and codebooks) on the
same stores and tokens.  The losses agree to 2e-3 relative; every dscale /
dcb within 5e-2 of the largest reference entry (both sides round activations
and their gradients to bf16, through 2 blocks, attention and the vocabulary
softmax); a ScaleTuner loop lowers the loss on a repeated batch, and the
indices never move.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _rel(a, b):
    a, b = a.detach().double().reshape(-1), b.detach().double().reshape(-1)
    return float((a - b).abs().max() / b.abs().max())


def _model(name, seed):
    from epure.model import PackedDecoder
    from epure.synthetic import DecoderShapes
    shapes = DecoderShapes(name, 2, 512, 1024, 8, 2, 64, 1000)
    return PackedDecoder(shapes, device=DEV, seed=seed, max_len=128, fused_glue=False)


def _grads(params):
    return [p.grad.detach().clone() for p in params]


@pytest.mark.parametrize("name", ["qwen3-small", "llama3-small"])
def test_whole_model_gradients_match_reference_autograd(name):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from epure import _native
    from epure.finetune import make_trainable, snapshot_indices, verify_frozen
    from epure.model import PackedCausalLM
    dec = _model(name, seed=5)
    ours = PackedCausalLM(dec, "ours")
    ref = PackedCausalLM(dec, "reference")        # the same stores: shared parameters
    params = make_trainable(ours, "both")
    assert len(params) == 2 * 7 * 2
    snap = snapshot_indices(ours)
    g = torch.Generator(device=DEV).manual_seed(11)
    ids = torch.randint(0, 1000, (2, 96), generator=g, device=DEV)

    loss_o = ours(ids).loss
    loss_o.backward()
    g_ours = _grads(params)
    for p in params:
        p.grad = None
    loss_r = ref(ids).loss
    loss_r.backward()
    g_ref = _grads(params)

    assert abs(float(loss_o) - float(loss_r)) <= 2e-3 * abs(float(loss_r))
    for i, (a, b) in enumerate(zip(g_ours, g_ref)):
        assert float(b.abs().max()) > 0, i
        assert _rel(a, b) <= 5e-2, (i, _rel(a, b))
    verify_frozen(ours, snap)
    assert _native.device_error() == 0


def test_scale_tuner_lowers_the_loss():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from epure.finetune import ScaleTuner
    from epure.model import PackedCausalLM
    model = PackedCausalLM(_model("qwen3-small", seed=9), "ours")
    tuner = ScaleTuner(model, mode="both", lr=3e-3, device=torch.device(DEV))
    g = torch.Generator(device=DEV).manual_seed(3)
    ids = torch.randint(0, 1000, (2, 64), generator=g, device=DEV)
    losses = [tuner.step(ids) for _ in range(8)]
    assert losses[-1] < losses[0] - 0.05, losses
    tuner.finish()                                 # raises if an index moved
