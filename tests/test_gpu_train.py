"""The compressed-state fine-tuning step (epure.train.PackedTrainStep) on the GPU.

A 2-layer stack of small decoder shapes with fp32 scales and codebooks (what
make_trainable(mode="both") holds) runs one step through libepq.so; torch
autograd of the reference formulation (F.linear over materialize(bf16),
fp32 parameters, the same injected output gradients) gives the same parameter
and input gradients within bf16 tolerance (3e-2 relative per tensor: both
sides round every activation and activation gradient to bf16), and the
indices never change.
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _rel(a, b):
    a, b = a.detach().double().reshape(-1), b.detach().double().reshape(-1)
    return float((a - b).abs().max() / b.abs().max())


def test_train_step_matches_autograd():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from epure import _native, synthetic
    from epure.synthetic import DecoderShapes
    from epure.train import PackedTrainStep
    shapes = DecoderShapes("small", 2, 512, 1024, 4, 2, 128, 1000)
    stack = synthetic.LinearStack(shapes, device=DEV, seed=3, gpu_layout="mma16",
                                  scale_dtype=torch.float32, cb_dtype=torch.float32)
    before = [{n: st.index_rows().clone() for n, st in b.items()} for b in stack.blocks]
    m = 96
    trainer = PackedTrainStep(stack, m, device=DEV, seed=1)
    x = (torch.randn(m, 512, device=DEV)).to(torch.bfloat16)
    dx = trainer.step(x)

    # reference: autograd of F.linear(h, materialize(bf16)) with fp32 parameters
    params = []
    for b in stack.blocks:
        params.append({n: (st.index_rows().long(), st.cb.float().clone().requires_grad_(True),
                           st.scale.float().clone().requires_grad_(True), st) for n, st in b.items()})

    def weight(p):
        idx, cb, sc, st = p
        w = cb.to(torch.bfloat16)[idx].reshape(st.out_features, -1)
        return w * sc.to(torch.bfloat16).repeat_interleave(st.group, dim=1)

    h0 = x.clone().requires_grad_(True)
    h = h0
    loss = 0
    for pb in params:
        q = F.linear(h, weight(pb["q_proj"]))
        k = F.linear(h, weight(pb["k_proj"]))
        v = F.linear(h, weight(pb["v_proj"]))
        o = F.linear(q, weight(pb["o_proj"]))
        gt = F.linear(o, weight(pb["gate_proj"]))
        u = F.linear(o, weight(pb["up_proj"]))
        h = F.linear(u, weight(pb["down_proj"]))
        loss = loss + (k.float() * trainer.dk.float()).sum() + (v.float() * trainer.dv.float()).sum() \
            + (gt.float() * trainer.dg.float()).sum()
    loss = loss + (h.float() * trainer.dout.float()).sum()
    loss.backward()

    assert _rel(dx.float(), h0.grad.float()) <= 3e-2
    for li, pb in enumerate(params):
        for name, (_, cb, sc, st) in pb.items():
            dscale, dcb = trainer.grads[li][name]
            assert _rel(dscale, sc.grad) <= 3e-2, (li, name)
            assert _rel(dcb, cb.grad.reshape(-1)) <= 3e-2, (li, name)
    for b, snap in zip(stack.blocks, before):
        for n, st in b.items():
            assert torch.equal(st.index_rows(), snap[n])
    assert _native.device_error() == 0
