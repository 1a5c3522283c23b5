"""The decode program (epq_program_*: a whole decode token as one persistent
kernel) against the same steps launched one by one.

* Linear steps reuse the fused GEMV's arithmetic: a program of the four fused
  linear kinds (q/k/v with the RMSNorm prologue, o and down into the residual
  stream, gate/up with SiLU * up) gives BIT-identical results to the same
  epq_decode_linear calls, at Llama-3-8B widths.
* The attention step matches epq_attn_rope_decode to bf16 rounding (only the
  split merge order differs) and writes the same cache rows.
* A PackedDecoder with the program decodes the same tokens as the five-launch
  path, logits within 2e-2, in and out of a CUDA graph, reproducibly.
* A position past the KV cache zeroes the attention, writes no cache row and
  sets bit 4 of epq_device_error (child process: the flag stays set).
"""
import math

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


def _rel(a, b):
    return float((a.float() - b.float()).abs().max() / b.float().abs().max())


def _stack(layers=1):
    from epure import synthetic
    return synthetic.LinearStack(synthetic.SHAPES["llama3-8b"], layers=layers, device=DEV, seed=3,
                                 gpu_layout="mma16")


def test_program_linears_bit_identical_to_decode_linear():
    from epure import _native
    b = _stack(1).blocks[0]
    bf = torch.bfloat16
    g = torch.Generator(device=DEV).manual_seed(1)
    h0 = torch.randn(1, 4096, generator=g, device=DEV).to(bf)
    a0 = torch.randn(1, 4096, generator=g, device=DEV).to(bf)

    def bufs():
        return dict(h=h0.clone(), att=a0.clone(), q=torch.empty(1, 4096, dtype=bf, device=DEV),
                    k=torch.empty(1, 1024, dtype=bf, device=DEV), v=torch.empty(1, 1024, dtype=bf, device=DEV),
                    act=torch.empty(1, 14336, dtype=bf, device=DEV))

    want = bufs()
    _native.decode_linear(want["h"], [b["q_proj"], b["k_proj"], b["v_proj"]], prologue=_native.PRO_RMSNORM,
                          outs=[want["q"], want["k"], want["v"]], eps=1e-5)
    _native.decode_linear(want["att"], [b["o_proj"]], epilogue=_native.EPI_RESIDUAL, outs=[want["h"]])
    _native.decode_linear(want["h"], [b["gate_proj"], b["up_proj"]], prologue=_native.PRO_RMSNORM,
                          epilogue=_native.EPI_SILU_MUL, outs=[want["act"]], eps=1e-5)
    _native.decode_linear(want["act"], [b["down_proj"]], epilogue=_native.EPI_RESIDUAL, outs=[want["h"]])

    got = bufs()
    prog = _native.DecodeProgram(DEV)
    prog.linear(got["h"], [b["q_proj"], b["k_proj"], b["v_proj"]], [got["q"], got["k"], got["v"]],
                prologue=_native.PRO_RMSNORM, eps=1e-5)
    prog.linear(got["att"], [b["o_proj"]], [got["h"]], epilogue=_native.EPI_RESIDUAL)
    prog.linear(got["h"], [b["gate_proj"], b["up_proj"]], [got["act"]], prologue=_native.PRO_RMSNORM,
                epilogue=_native.EPI_SILU_MUL, eps=1e-5)
    prog.linear(got["act"], [b["down_proj"]], [got["h"]], epilogue=_native.EPI_RESIDUAL)
    prog.finalize()
    prog.run()
    torch.cuda.synchronize()
    for name in ("q", "k", "v", "act", "h"):
        assert torch.equal(got[name], want[name]), name
    # a second run over the same buffers repeats the same arithmetic
    h1 = got["h"].clone()
    got["h"].copy_(h0)
    prog.run()
    torch.cuda.synchronize()
    assert torch.equal(got["h"], h1)


@pytest.mark.parametrize("heads,kv,hd,qk", [(32, 8, 128, False), (16, 8, 128, True), (8, 8, 64, False),
                                            (16, 2, 64, True)])
@pytest.mark.parametrize("P", [0, 5, 130])
def test_program_attention_matches_attn_rope_decode(heads, kv, hd, qk, P):
    from epure import _native
    L = 160
    g = torch.Generator(device=DEV).manual_seed(P + heads)
    bf = torch.bfloat16
    q = torch.randn(heads, hd, generator=g, device=DEV).to(bf)
    k = torch.randn(kv, hd, generator=g, device=DEV).to(bf)
    v = torch.randn(kv, hd, generator=g, device=DEV).to(bf)
    kc = torch.randn(L, kv, hd, generator=g, device=DEV).to(bf)
    vc = torch.randn(L, kv, hd, generator=g, device=DEV).to(bf)
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, device=DEV, dtype=torch.float64) / hd))
    ang = torch.arange(L, device=DEV, dtype=torch.float64)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang).float(), torch.sin(ang).float()
    pos = torch.tensor([P], device=DEV)
    ws = _native.attn_decode_workspace(heads, kv, hd, DEV)
    kc2, vc2 = kc.clone(), vc.clone()
    want = _native.attn_rope_decode(q, k, v, pos, cos, sin, kc2, vc2, qk, 1e-6, 1.0 / math.sqrt(hd), ws)
    out = torch.empty(heads, hd, dtype=bf, device=DEV)
    prog = _native.DecodeProgram(DEV)
    prog.attention(q, k, v, pos, cos, sin, kc, vc, qk, 1e-6, 1.0 / math.sqrt(hd), out)
    prog.finalize()
    prog.run()
    torch.cuda.synchronize()
    assert _rel(out, want) <= 1e-2
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)


def _decoders(name="llama3-8b", layers=4, max_len=96):
    from epure.model import PackedDecoder
    from epure.synthetic import SHAPES
    one = PackedDecoder(SHAPES[name], layers=layers, device=DEV, seed=5, max_len=max_len, program=True)
    other = PackedDecoder(SHAPES[name], layers=layers, device=DEV, seed=5, max_len=max_len, program=False,
                          stack=one.stack, embed=one.embed, lm_head=one.lm_head)
    assert one.use_program and not other.use_program
    return one, other


@pytest.mark.parametrize("name", ["llama3-8b", "qwen3-1.7b"])
def test_decoder_program_matches_launches(name):
    one, other = _decoders(name)
    g = torch.Generator().manual_seed(7)
    prompt = torch.randint(0, one.shapes.vocab, (24,), generator=g)
    tokens = torch.randint(0, one.shapes.vocab, (12,), generator=g)
    a = one.teacher_forced_logits(prompt, tokens)
    b = other.teacher_forced_logits(prompt, tokens)
    assert _rel(a, b) <= 2e-2
    assert (a.argmax(-1) == b.argmax(-1)).float().mean() >= 0.75
    # reproducible: the same prompt again gives the same logits bit for bit
    assert torch.equal(one.teacher_forced_logits(prompt, tokens), a)


def test_decoder_program_in_a_graph():
    one, other = _decoders("qwen3-1.7b", layers=3)
    prompt = torch.randint(0, one.shapes.vocab, (16,), generator=torch.Generator().manual_seed(2))
    one.capture()
    got = one.generate(prompt, 10, graph=True).cpu()
    want = one.generate(prompt, 10, graph=False).cpu()
    assert torch.equal(got, want)


_PAST_CACHE_CHILD = r"""
import math, sys, torch
sys.path.insert(0, sys.argv[1])
from epure import _native
dev = "cuda:0"
heads, kv, hd, L = 16, 8, 128, 32
g = torch.Generator(device=dev).manual_seed(0)
bf = torch.bfloat16
q = torch.randn(heads, hd, generator=g, device=dev).to(bf)
k = torch.randn(kv, hd, generator=g, device=dev).to(bf)
v = torch.randn(kv, hd, generator=g, device=dev).to(bf)
kc = torch.randn(L, kv, hd, generator=g, device=dev).to(bf)
vc = kc.clone()
cos = torch.ones(L, hd // 2, device=dev)
sin = torch.zeros(L, hd // 2, device=dev)
pos = torch.tensor([L], device=dev)
out = torch.full((heads, hd), 1.0, dtype=bf, device=dev)
k0, v0 = kc.clone(), vc.clone()
prog = _native.DecodeProgram(dev)
prog.attention(q, k, v, pos, cos, sin, kc, vc, False, 1e-6, 1.0 / math.sqrt(hd), out)
prog.finalize()
assert _native.device_error() == 0
prog.run()
torch.cuda.synchronize()
assert torch.equal(kc, k0) and torch.equal(vc, v0), "cache written past its capacity"
assert not out.any(), "attention output not zeroed"
flag = _native.device_error()
pos.fill_(L - 1)
prog.run()           # the same program still serves an in-range position afterwards
torch.cuda.synchronize()
assert out.float().abs().sum() > 0
print("FLAG", flag)
"""


def test_program_position_past_cache_is_refused():
    import subprocess
    import sys
    from conftest import PKG
    r = subprocess.run([sys.executable, "-c", _PAST_CACHE_CHILD, PKG], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "FLAG 16" in r.stdout, r.stdout
