"""The block's fused residual + norm + AdaLN modulation pass (tm_residual_norm).

``r = x + y * gate`` (stored, rounded to bf16), then ``norm(r) * (1 + scale)
+ shift`` for up to two modulations, with AdaLN parameter rows per frame
(``table[p] + ts[frame, p]``).  Checked against a torch fp32 restatement of
kv_cache.py:2201-2204 / 2601-2640 (the residual must match to one bf16 ulp;
the normalised outputs within the bf16 rounding of the output) at the
model's widths (video 4096, audio 2048) and others (1280, 1024), at the
token counts of 1 / 8 GPUs and of the audio stream, for RMSNorm and
LayerNorm, with and without the residual input and the gate.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0") if torch.cuda.is_available() else None


@pytest.fixture(scope="module", autouse=True)
def _device():
    if DEV is None:
        pytest.skip("no CUDA device")
    torch.cuda.set_device(DEV)
    yield
    from taomate_b200 import _lib
    assert _lib.device_error() == 0, "a kernel set the device error flag"


def _rel(a, b):
    a, b = a.double(), b.double()
    return float(torch.linalg.norm(a - b) / torch.linalg.norm(b))


def _params(table, ts, L, D, fs, p):
    """[L, D] fp32 values of AdaLN parameter p for tokens 0..L-1 (frame = t // fs)."""
    rows = torch.arange(L, device=DEV) // fs
    return table[p].float()[None] + ts[0, rows, p * D:(p + 1) * D].float()


CASES = [  # (L, D, frames' tokens, norm, with y, with gate, outputs)
    (1152, 4096, 384, "rms", True, True, 2),
    (144, 4096, 384, "rms", True, True, 2),
    (1152, 4096, 384, "rms", False, False, 1),
    (25, 2048, 1, "rms", True, True, 1),
    (144, 4096, 384, "layer", False, False, 1),
    (96, 1280, 32, "rms", True, True, 2),
    (40, 1024, 8, "layer", True, False, 0),
]


@pytest.mark.parametrize("L,D,fs,norm,with_y,with_gate,n_out", CASES)
def test_residual_norm_vs_torch(L, D, fs, norm, with_y, with_gate, n_out):
    from taomate_b200.block import AdaParams, residual_norm
    g = torch.Generator().manual_seed(L + D + n_out)
    r_ = lambda *s: torch.randn(*s, generator=g).to(DEV, torch.bfloat16)
    n = 6
    F = (L + fs - 1) // fs
    x, y = r_(1, L, D), r_(1, L, D)
    table, ts = r_(n, D) * 0.1, r_(1, F, n * D) * 0.1
    prm = AdaParams(table, ts, L, n, D, fs, 0)
    xo = torch.empty_like(x) if with_y else None
    outs = [torch.empty_like(x) for _ in range(n_out)]
    mods = [(1, 0), (4, 3)][:n_out]
    residual_norm(x, y if with_y else None, prm if with_gate else None, 2 if with_gate else -1,
                  xo, [(o, prm, sc, sh) for o, (sc, sh) in zip(outs, mods)], norm=norm,
                  eps=1e-6)
    torch.cuda.synchronize()
    v = x[0].float()
    if with_y:
        yy = y[0].float()
        if with_gate:
            yy = yy * _params(table, ts, L, D, fs, 2)
        v = (v + yy).to(torch.bfloat16).float()
        assert (xo[0].float() - v).abs().max() <= v.abs().max() * 2 ** -7
        assert _rel(xo[0], v) < 1e-3
    if norm == "rms":
        h = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-6)
    else:
        m = v.mean(-1, keepdim=True)
        h = (v - m) * torch.rsqrt((v - m).pow(2).mean(-1, keepdim=True) + 1e-6)
    for o, (sc, sh) in zip(outs, mods):
        ref = h * (1 + _params(table, ts, L, D, fs, sc)) + _params(table, ts, L, D, fs, sh)
        assert _rel(o[0], ref) < 2.5e-3


def test_residual_norm_rows_beyond_one_wave():
    """More rows than one wave of CTAs (one per row) fit on the GPU."""
    from taomate_b200.block import AdaParams, residual_norm
    L, D = 4 * 148 * 4 + 3, 2048
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, L, D, generator=g).to(DEV, torch.bfloat16)
    out = torch.empty_like(x)
    residual_norm(x, outs=[(out, None, -1, -1)], eps=1e-6)
    v = x[0].float()
    ref = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-6)
    assert _rel(out[0], ref) < 2.5e-3


@pytest.mark.parametrize("n", [8, 4096 * 3, 1152 * 16384])
def test_gelu_tanh_vs_torch(n):
    """tm_gelu_tanh in place against torch's tanh GELU of the same bf16 input
    computed in fp32 (one bf16 rounding of the result each)."""
    from taomate_b200.block import gelu_tanh_
    g = torch.Generator().manual_seed(n)
    x = (torch.randn(n, generator=g) * 3).to(DEV, torch.bfloat16)
    ref = torch.nn.functional.gelu(x.float(), approximate="tanh")
    gelu_tanh_(x)
    assert (x.float() - ref).abs().max() <= ref.abs().max() * 2 ** -7
    assert _rel(x, ref) < 3e-3


def test_feed_forward_gelu_epilogue():
    """The block's FFN (bias + tanh GELU fused into the first GEMM) against an
    fp64 restatement, and the unfused path (no bias: tm_gelu_tanh) against the
    same restatement."""
    from taomate_b200.block import feed_forward

    class _Lin(torch.nn.Module):
        def __init__(self, w, b):
            super().__init__()
            self.weight, self.bias = w, b

    class _FF(torch.nn.Module):
        def __init__(self, w1, b1, w2, b2):
            super().__init__()
            p = torch.nn.Module()
            p.proj = _Lin(w1, b1)
            self.net = [p, None, _Lin(w2, b2)]

    g = torch.Generator().manual_seed(7)
    r_ = lambda *s: torch.randn(*s, generator=g).to(DEV, torch.bfloat16)
    D, I = 1024, 4096
    x = r_(1, 300, D)
    w1, b1, w2, b2 = r_(I, D) * 0.05, r_(I) * 0.05, r_(D, I) * 0.02, r_(D) * 0.02
    for bias in (True, False):
        ff = _FF(w1, b1 if bias else None, w2, b2)
        out = feed_forward(ff, x)
        h = x.double() @ w1.double().t() + (b1.double() if bias else 0)
        ref = torch.nn.functional.gelu(h, approximate="tanh") @ w2.double().t() + b2.double()
        assert out.shape == (1, 300, D)
        assert _rel(out, ref) < 5e-3
