"""GPU parity of the layer-glue kernels (csrc/norm.cu) against fp32 torch
references of the reference's CUDA boundary (model/layers.py:28-115):
flashinfer.norm.rmsnorm, flashinfer.norm.fused_add_rmsnorm and
flashinfer.activation.silu_and_mul.  Outputs are one rounding of an fp32
result, so they may differ from the torch reference by one unit in the last
place of the output type (bf16: 2^-7 relative, fp16: 2^-10); the residual
that fused_add_rmsnorm stores is one rounding of an exact fp32 sum and must
match bit for bit."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

RTOL = {torch.bfloat16: 2.0**-7, torch.float16: 2.0**-10}
EPS = 1e-6


def _rms_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def _assert_ulp(got: torch.Tensor, want_f32: torch.Tensor, dtype) -> None:
    got = got.float().cpu()
    want = want_f32.cpu()
    bound = RTOL[dtype] * want.abs() + 1e-6
    err = (got - want).abs()
    assert bool((err <= bound).all()), f"max |err| {float(err.max()):.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("rows", "hidden"), [(1, 8), (7, 136), (64, 2048), (5, 1024), (3, 8192), (300, 2056)])
def test_rmsnorm(nqt, cuda, dtype, rows, hidden):
    g = torch.Generator().manual_seed(rows * 7 + hidden)
    wide = (torch.randn(rows, hidden + 24, generator=g) * 3).to(dtype).to(cuda)
    x = wide[:, 8: 8 + hidden]  # row stride hidden + 24, 16-byte aligned start
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(dtype).to(cuda)
    out_wide = torch.zeros(rows, hidden + 40, dtype=dtype, device=cuda)
    out = out_wide[:, 16: 16 + hidden]
    nqt.kernels.rmsnorm(x, w, EPS, out=out)
    _assert_ulp(out, _rms_ref(x, w, EPS), dtype)
    # the padding around the strided output is untouched
    assert bool((out_wide[:, :16] == 0).all()) and bool((out_wide[:, 16 + hidden:] == 0).all())
    # default (contiguous) output
    _assert_ulp(nqt.kernels.rmsnorm(x.contiguous(), w, EPS), _rms_ref(x, w, EPS), dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("rows", "hidden"), [(1, 8), (64, 2048), (9, 1000), (256, 1024), (2, 8192)])
def test_fused_add_rmsnorm(nqt, cuda, dtype, rows, hidden):
    g = torch.Generator().manual_seed(rows * 11 + hidden)
    x = (torch.randn(rows, hidden, generator=g) * 0.5).to(dtype)
    r = (torch.randn(rows, hidden, generator=g) * 4).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, generator=g)).to(dtype)
    xd, rd, wd = x.to(cuda), r.to(cuda), w.to(cuda)
    nqt.kernels.fused_add_rmsnorm_(xd, rd, wd, EPS)
    s = x.float() + r.float()
    assert torch.equal(rd.cpu(), s.to(dtype)), "residual must be the rounded fp32 sum"
    _assert_ulp(xd, _rms_ref(s, w, EPS), dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("rows", "d"), [(1, 8), (64, 6144), (3, 24), (256, 3072), (17, 2056)])
def test_silu_and_mul(nqt, cuda, dtype, rows, d):
    g = torch.Generator().manual_seed(rows * 13 + d)
    wide = (torch.randn(rows, 2 * d + 16, generator=g) * 3).to(dtype).to(cuda)
    gate_up = wide[:, : 2 * d]  # row stride 2d + 16
    out = nqt.kernels.silu_and_mul(gate_up)
    gf, uf = gate_up[:, :d].float(), gate_up[:, d:].float()
    _assert_ulp(out, torch.nn.functional.silu(gf) * uf, dtype)
    out_wide = torch.zeros(rows, d + 8, dtype=dtype, device=cuda)
    nqt.kernels.silu_and_mul(gate_up, out=out_wide[:, :d])
    _assert_ulp(out_wide[:, :d], torch.nn.functional.silu(gf) * uf, dtype)
    assert bool((out_wide[:, d:] == 0).all())


def test_glue_rejects_bad_shapes(nqt, cuda):
    x = torch.zeros(4, 12, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(nqt.NqtError):
        nqt.kernels.rmsnorm(x, torch.ones(12, dtype=torch.bfloat16, device=cuda), EPS)
    big = torch.zeros(2, 8200, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(nqt.NqtError):
        nqt.kernels.rmsnorm(big, torch.ones(8200, dtype=torch.bfloat16, device=cuda), EPS)
    with pytest.raises(nqt.NqtError):
        nqt.kernels.fused_add_rmsnorm_(x, x, torch.ones(12, dtype=torch.bfloat16, device=cuda), EPS)
