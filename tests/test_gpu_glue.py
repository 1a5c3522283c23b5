"""The decode-step glue kernels (include/epq_decode.h) against torch on the GPU."""
import math

import pytest
import torch
import torch.nn.functional as F

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


@pytest.mark.parametrize("n", [2048, 4096, 8192, 1000])
@pytest.mark.parametrize("with_add", [False, True])
def test_add_rmsnorm(n, with_add):
    from epure import _native
    g = torch.Generator(device=DEV).manual_seed(n)
    x = torch.randn(3, n, generator=g, device=DEV).to(torch.bfloat16)
    add = torch.randn(3, n, generator=g, device=DEV).to(torch.bfloat16) if with_add else None
    h = torch.empty_like(x)
    y = _native.add_rmsnorm(x, add=add, h_out=h, eps=1e-6)
    hw = (x.float() + add.float()).to(torch.bfloat16) if with_add else x
    yw = (hw.float() * torch.rsqrt(hw.float().pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    assert torch.equal(h, hw)
    assert _rel(y, yw) <= 1e-2


@pytest.mark.parametrize("heads,kv,hd", [(32, 8, 128), (16, 8, 128), (8, 2, 64), (64, 8, 128), (4, 4, 128)])
@pytest.mark.parametrize("P", [0, 1, 17, 300])
def test_attn_decode_vs_sdpa(heads, kv, hd, P):
    from epure import _native
    g = torch.Generator(device=DEV).manual_seed(P + heads)
    L = 320
    q = torch.randn(heads, hd, generator=g, device=DEV).to(torch.bfloat16)
    kc = torch.randn(L, kv, hd, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(L, kv, hd, generator=g, device=DEV).to(torch.bfloat16)
    pos = torch.tensor([P], device=DEV)
    ws = _native.attn_decode_workspace(heads, kv, hd, DEV)
    got = _native.attn_decode(q, kc, vc, pos, 1.0 / math.sqrt(hd), ws)
    got2 = _native.attn_decode(q, kc, vc, pos, 1.0 / math.sqrt(hd), ws)       # workspace reused
    plain = _native.attn_decode(q, kc, vc, pos, 1.0 / math.sqrt(hd), None)    # one CTA per head
    k = kc[:P + 1].float().repeat_interleave(heads // kv, dim=1).transpose(0, 1)
    v = vc[:P + 1].float().repeat_interleave(heads // kv, dim=1).transpose(0, 1)
    want = F.scaled_dot_product_attention(q.float()[:, None], k, v, scale=1.0 / math.sqrt(hd))[:, 0]
    assert _rel(got, want) <= 1e-2
    assert torch.equal(got, got2)
    assert _rel(plain, want) <= 1e-2


def test_argmax_matches_torch_with_ties():
    from epure import _native
    g = torch.Generator(device=DEV).manual_seed(5)
    ws = _native.argmax_workspace(DEV)
    out = torch.zeros(1, dtype=torch.long, device=DEV)
    for n in (1, 7, 1000, 128256, 151936):
        x = torch.randn(n, generator=g, device=DEV)
        if n > 10:
            x[n // 3] = x[n - 2] = x.max() + 1          # a tie: the first index wins
        _native.argmax(x, out, ws)
        assert int(out) == int(torch.argmax(x)), n


def test_silu_mul_and_rope():
    from epure import _native
    g = torch.Generator(device=DEV).manual_seed(6)
    a = torch.randn(6144, generator=g, device=DEV).to(torch.bfloat16)
    b = torch.randn(6144, generator=g, device=DEV).to(torch.bfloat16)
    want = (F.silu(a.float()) * b.float()).to(torch.bfloat16)
    assert _rel(_native.silu_mul(a, b), want) <= 1e-2
    # RoPE + KV write at position 5 against the torch formulation of epure.model
    H, KV, hd, L = 4, 2, 128, 16
    q = torch.randn(1, H, hd, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(1, KV, hd, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(1, KV, hd, generator=g, device=DEV).to(torch.bfloat16)
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, device=DEV, dtype=torch.float64) / hd))
    ang = torch.arange(L, device=DEV, dtype=torch.float64)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang).float(), torch.sin(ang).float()
    kc = torch.zeros(L, KV, hd, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    pos = torch.tensor([5], device=DEV)

    def rms(t):
        return (t.float() * torch.rsqrt(t.float().pow(2).mean(-1, keepdim=True) + 1e-6)).to(t.dtype)

    def rope(t):
        c, s = cos[pos][:, None, :], sin[pos][:, None, :]
        tf = t.float()
        x1, x2 = tf[..., :hd // 2], tf[..., hd // 2:]
        return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(t.dtype)

    qw, kw = rope(rms(q)), rope(rms(k))
    qq = q.clone()
    _native.rope_kv(qq, k, v, pos, cos, sin, kc, vc, True, 1e-6)
    assert _rel(qq, qw) <= 1e-2
    assert _rel(kc[5], kw[0]) <= 1e-2
    assert torch.equal(vc[5], v[0])


@pytest.mark.parametrize("heads,kv,hd,qk", [(32, 8, 128, False), (16, 8, 128, True), (8, 2, 64, True)])
def test_attn_rope_matches_two_kernels(heads, kv, hd, qk):
    """epq_attn_rope_decode == epq_rope_kv followed by epq_attn_decode."""
    from epure import _native
    g = torch.Generator(device=DEV).manual_seed(heads + hd)
    L, P = 64, 40
    q = torch.randn(heads, hd, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(kv, hd, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(kv, hd, generator=g, device=DEV).to(torch.bfloat16)
    kc = torch.randn(L, kv, hd, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(L, kv, hd, generator=g, device=DEV).to(torch.bfloat16)
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2, device=DEV, dtype=torch.float64) / hd))
    ang = torch.arange(L, device=DEV, dtype=torch.float64)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang).float(), torch.sin(ang).float()
    pos = torch.tensor([P], device=DEV)
    ws = _native.attn_decode_workspace(heads, kv, hd, DEV)
    kc2, vc2, q2 = kc.clone(), vc.clone(), q.clone().view(1, heads, hd)
    _native.rope_kv(q2, k.view(1, kv, hd), v.view(1, kv, hd), pos, cos, sin, kc2, vc2, qk, 1e-6)
    want = _native.attn_decode(q2.view(heads, hd), kc2, vc2, pos, 1.0 / math.sqrt(hd), ws)
    got = _native.attn_rope_decode(q, k, v, pos, cos, sin, kc, vc, qk, 1e-6, 1.0 / math.sqrt(hd), ws)
    assert _rel(got, want) <= 1e-2
    assert _rel(kc[P], kc2[P]) <= 1e-2 and torch.equal(vc[P], vc2[P])
    assert torch.equal(kc[:P], kc2[:P])


_PAST_CACHE_CHILD = r"""
import math, sys, torch
sys.path.insert(0, sys.argv[1])
from epure import _native
dev = "cuda:0"
heads, kv, hd, L = 16, 8, 128, 32
g = torch.Generator(device=dev).manual_seed(0)
q = torch.randn(heads, hd, generator=g, device=dev).to(torch.bfloat16)
k = torch.randn(kv, hd, generator=g, device=dev).to(torch.bfloat16)
v = torch.randn(kv, hd, generator=g, device=dev).to(torch.bfloat16)
kc = torch.randn(L, kv, hd, generator=g, device=dev).to(torch.bfloat16)
vc = kc.clone()
cos = torch.ones(L, hd // 2, device=dev)
sin = torch.zeros(L, hd // 2, device=dev)
ws = _native.attn_decode_workspace(heads, kv, hd, dev)
k0, v0 = kc.clone(), vc.clone()
assert _native.device_error() == 0
out = _native.attn_rope_decode(q, k, v, torch.tensor([L], device=dev), cos, sin, kc, vc, False, 1e-6,
                               1.0 / math.sqrt(hd), ws)
torch.cuda.synchronize()
assert torch.equal(kc, k0) and torch.equal(vc, v0), "cache written past its capacity"
assert not out.any(), "attention output not zeroed"
flag = _native.device_error()
# the same workspace still serves an in-range call afterwards
_native.attn_rope_decode(q, k, v, torch.tensor([L - 1], device=dev), cos, sin, kc, vc, False, 1e-6,
                         1.0 / math.sqrt(hd), ws)
torch.cuda.synchronize()
print("FLAG", flag)
"""


def test_position_past_cache_is_refused():
    """A device-side position at the KV cache's capacity writes nothing to the cache,
    zeroes the attention output and sets bit 4 of epq_device_error.  Run in a child
    process, because the flag stays set for the rest of that process."""
    import subprocess
    import sys
    from conftest import PKG
    r = subprocess.run([sys.executable, "-c", _PAST_CACHE_CHILD, PKG], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "FLAG 16" in r.stdout, r.stdout


def test_decoder_refuses_more_tokens_than_its_cache():
    from epure.model import PackedDecoder
    from epure.synthetic import DecoderShapes
    dec = PackedDecoder(DecoderShapes("tiny", 1, 256, 512, 4, 2, 64, 100), device=DEV, seed=1, max_len=16)
    with pytest.raises(ValueError, match="max_len"):
        dec.generate(torch.arange(10), 7, graph=False)
    with pytest.raises(ValueError, match="max_len"):
        dec.prefill(torch.arange(17))
