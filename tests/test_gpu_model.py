"""Whole-model greedy decoding around the packed linears (epure.model.PackedDecoder).

* The decoder with libepq.so's kernels ("ours") gives the same logits as the
  same model in float32 (weights cb * scale exactly) within bf16 tolerance.
* The fused decode launches (RMSNorm prologue, residual / SiLU epilogues) give
  the logits of the same block written with torch glue.
* The CUDA-graphed greedy loop emits exactly the tokens of the eager loop.
* Greedy top-1 agreement over 256 decode steps (128-token prompt of uniform
  random ids) on the Qwen3-1.7B and Llama-3-8B shapes, teacher-forced on the
  reference's own greedy sequence (``F.linear(x, materialize(bf16))``,
  runtime.py:123-124, with the block in torch ops).  Ours decodes the
  reference's bf16 weight bit for bit, so the two differ only in the fp32
  summation order of each linear.  With random weights the logits are nearly
  flat, and any change of summation order flips some argmaxes: the same
  reference block with every linear computed exactly (float64, then rounded
  to bf16 -- the "exact control") agrees with the reference on ~95 % of the
  steps, not 99 %.  The test therefore asserts that ours agrees with the
  reference about as well as the exact control does (flip counts are small
  and noisy: within 8 of 256 steps), that every step where ours and the
  reference differ is a near-tie of the reference's own logits (their gap
  is within twice ours' logit deviation there), and that ours is no further
  from the float32 model than the reference is.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from epure import _native
    _native.load_library()
    yield
    assert _native.device_error() == 0


def _small():
    from epure.synthetic import DecoderShapes
    return DecoderShapes("small", 2, 512, 1024, 8, 2, 64, 1000)


def test_small_model_logits_vs_fp32():
    from epure.model import PackedDecoder
    ours = PackedDecoder(_small(), device=DEV, seed=3, max_len=64)
    ref32 = ours.share_weights("fp32")
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, 1000, (16,), generator=g)
    a, b = ours.prefill(prompt), ref32.prefill(prompt)
    assert float((a - b).abs().max() / b.abs().max()) <= 2e-2
    tok = torch.tensor([5], device=DEV)
    for t in range(6):
        pos = torch.tensor([16 + t], device=DEV)
        a, b = ours.step(tok, pos), ref32.step(tok, pos)
        assert float((a - b).abs().max() / b.abs().max()) <= 2e-2, t
        tok = torch.argmax(b).view(1)


@pytest.mark.parametrize("shape", ["small", "qwen3"])
def test_fused_glue_matches_torch_glue(shape):
    """The decode glue kernels (include/epq_decode.h) against the same block in torch ops."""
    from epure.model import PackedDecoder
    from epure.synthetic import DecoderShapes
    sh = _small() if shape == "small" else DecoderShapes("qwen3-test", 2, 512, 1024, 8, 4, 128, 1000)
    fused = PackedDecoder(sh, device=DEV, seed=6, max_len=64)
    plain = fused.share_weights("ours")
    plain.fused_glue = False
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, 1000, (10,), generator=g)
    fused.prefill(prompt)
    plain.prefill(prompt)
    tok = torch.tensor([7], device=DEV)
    for t in range(12):
        pos = torch.tensor([10 + t], device=DEV)
        a, b = fused.step(tok, pos), plain.step(tok, pos)
        assert float((a - b).abs().max() / b.abs().max()) <= 1e-2, (shape, t)
        tok = torch.argmax(b).view(1)


def test_graph_matches_eager():
    from epure.model import PackedDecoder
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, 1000, (12,), generator=g)
    eager = PackedDecoder(_small(), device=DEV, seed=4, max_len=64)
    want = eager.generate(prompt, 20, graph=False)
    graphed = eager.share_weights("ours").capture()
    got = graphed.generate(prompt, 20, graph=True)
    assert torch.equal(got.cpu(), want.cpu())


def _exact_control(dec):
    """The reference block with each linear computed exactly (float64) and rounded
    to bf16: a valid implementation of the reference's arithmetic that differs
    from it only in summation order."""
    import types
    ctl = dec.share_weights("reference")

    def lin(self, x, stores):
        return [(x.double() @ st.materialize(x.dtype).double().T).to(x.dtype) for st in stores]

    ctl._lin = types.MethodType(lin, ctl)
    return ctl


@pytest.mark.parametrize("model", ["qwen3-1.7b", "llama3-8b"])
def test_greedy_agreement_256(model):
    from epure import synthetic
    from epure.model import PackedDecoder
    shapes = synthetic.SHAPES[model]
    ours = PackedDecoder(shapes, device=DEV, seed=11, max_len=128 + 256)
    ref = ours.share_weights("reference")
    f32 = ours.share_weights("fp32")
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, shapes.vocab, (128,), generator=g)
    seq = ref.generate(prompt, 256, graph=False).cpu()
    l_ref = ref.teacher_forced_logits(prompt, seq)
    l_ours = ours.teacher_forced_logits(prompt, seq)
    p_ref, p_ours = l_ref.argmax(-1).cpu(), l_ours.argmax(-1).cpu()
    p_ctl = _exact_control(ours).teacher_forced_argmax(prompt, seq)
    l32 = f32.teacher_forced_logits(prompt, seq)
    p_f32 = l32.argmax(-1).cpu()
    assert torch.equal(p_ref, seq)                    # the reference reproduces itself
    agree = lambda a, b: float((a == b).float().mean())          # noqa: E731
    ours_ref, ctl_ref = agree(p_ours, p_ref), agree(p_ctl, p_ref)
    ours_f32, ref_f32 = agree(p_ours, p_f32), agree(p_ref, p_f32)
    # steps where ours differs from the reference: the reference's own logit gap
    # between the two tokens against the size of ours' logit deviation there
    rows = (p_ours != p_ref).nonzero().flatten()
    gap = (l_ref[rows, p_ref[rows]] - l_ref[rows, p_ours[rows]]).abs()
    dev = (l_ours[rows] - l_ref[rows]).abs().amax(-1)
    rel_ours = float(((l_ours - l32).abs().amax(-1) / l32.abs().amax(-1)).max())
    rel_ref = float(((l_ref - l32).abs().amax(-1) / l32.abs().amax(-1)).max())
    print(f"{model}: top-1 agreement over 256 steps: ours~reference {ours_ref:.4f}  "
          f"exact-control~reference {ctl_ref:.4f}  ours~fp32 {ours_f32:.4f}  reference~fp32 {ref_f32:.4f}; "
          f"flips {len(rows)}, largest reference gap at a flip {float(gap.max()) if len(rows) else 0:.4f}; "
          f"logit max rel err vs fp32: ours {rel_ours:.2e} reference {rel_ref:.2e}")
    # the flip counts of two implementations that differ only in summation order are
    # small (~5-15 of 256) and noisy: allow ours 8 more flips than the exact control
    assert ours_ref >= min(0.99, ctl_ref - 8 / 256)
    assert bool((gap <= 2 * dev + 1e-6).all())          # every flip is a near-tie of the reference
    assert ours_f32 >= ref_f32 - 0.01
    assert rel_ours <= max(1.1 * rel_ref, 1e-2)
