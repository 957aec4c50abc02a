"""GPU: the FP8 block-scaled gate/up path (csrc/gemm_fp8.cu, csrc/norm.cu)
against the CPU oracle (oracle/fp8.py), which is pinned to the reference's
quantize_fp8_weight_blocks by tests/golden/fp8.pt.

* quantisers (weight blocks, activation rows, the fused add + RMSNorm):
  bit-exact e4m3 bytes and scales;
* the GEMM: the kernel accumulates each 128-K block in fp32 on the tensor
  cores and promotes it with fp32 scales, the oracle in float64 rounded once
  to bf16, so an output differs from the oracle's by at most one bf16 ulp
  (2^-7 |y|, plus 1e-5 of the largest |y| where the sum cancels), the mean
  error stays within 2^-10 of the mean |y|, and at least 97 % of the outputs
  are bit-equal; SwiGLU outputs (two bf16 roundings before silu * up) within
  2^-6 |y| plus the same absolute term.
"""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from oracle import fp8 as ofp8

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "fp8.pt"


def _bytes(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.uint8).cpu()


def test_weight_quantiser_reproduces_the_reference_fixture(nqt, cuda):
    g = torch.load(GOLDEN)
    q, s = nqt.kernels.quantize_fp8_weight_blocks(g["weight"].to(cuda))
    assert torch.equal(_bytes(q), g["q"])
    assert torch.equal(s.cpu(), g["scales"])


@pytest.mark.parametrize("shape", [(128, 128), (384, 1024), (1024, 2048)])
def test_weight_quantiser_matches_the_oracle(nqt, cuda, shape):
    gen = torch.Generator().manual_seed(shape[0])
    w = (torch.randn(*shape, generator=gen) * torch.logspace(-6, 6, shape[1] // 128).repeat_interleave(128)).to(
        torch.bfloat16)
    q, s = nqt.kernels.quantize_fp8_weight_blocks(w.to(cuda))
    want_q, want_s = ofp8.quantize_weight_blocks(w)
    assert torch.equal(s.cpu(), want_s)
    assert torch.equal(_bytes(q), want_q.view(torch.uint8))


def test_weight_quantiser_rejects_what_the_reference_rejects(nqt, cuda):
    with pytest.raises(ValueError, match="divisible by 128"):
        nqt.kernels.quantize_fp8_weight_blocks(torch.zeros(128, 200, dtype=torch.bfloat16, device=cuda))
    with pytest.raises(ValueError, match="contiguous matrix"):
        nqt.kernels.quantize_fp8_weight_blocks(torch.zeros(256, 256, dtype=torch.bfloat16, device=cuda)[:, :128])


@pytest.mark.parametrize("m", [1, 64, 200])
def test_row_quantiser_matches_the_oracle(nqt, cuda, m):
    gen = torch.Generator().manual_seed(m)
    x = (torch.randn(m, 2048, generator=gen) * torch.logspace(-5, 5, m).view(m, 1)).to(torch.bfloat16)
    x[0, 256:384] = 0.0
    if m > 2:
        x[1, :128] = torch.finfo(torch.bfloat16).max
        x[2, 5] = -torch.finfo(torch.bfloat16).tiny
    q, s = nqt.kernels.fp8_quantize_rows(x.to(cuda))
    want_q, want_s = ofp8.quantize_rows(x)
    assert torch.equal(s.cpu(), want_s)
    assert torch.equal(_bytes(q), want_q.view(torch.uint8))


def test_fused_add_rmsnorm_fp8_is_the_norm_then_the_row_quantiser(nqt, cuda):
    gen = torch.Generator(device=cuda).manual_seed(7)
    rows, hidden = 64, 2048
    o = torch.randn(rows, hidden, generator=gen, device=cuda).to(torch.bfloat16)
    res = (torch.randn(rows, hidden, generator=gen, device=cuda) * 4).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, generator=gen, device=cuda)).to(torch.bfloat16)
    o_ref, res_ref = o.clone(), res.clone()
    nqt.kernels.fused_add_rmsnorm_(o_ref, res_ref, w, 1e-6)
    q_ref, s_ref = nqt.kernels.fp8_quantize_rows(o_ref)
    q = torch.empty(rows, hidden, dtype=torch.float8_e4m3fn, device=cuda)
    s = torch.empty(hidden // 128, rows, dtype=torch.float32, device=cuda)
    x = o.clone()
    nqt.kernels.fused_add_rmsnorm_fp8_(x, res, w, 1e-6, q, s, write_x=True)
    torch.cuda.synchronize()
    assert torch.equal(res, res_ref)
    assert torch.equal(x, o_ref)
    assert torch.equal(_bytes(q), _bytes(q_ref))
    assert torch.equal(s, s_ref)
    # the CPU oracle on the GPU's normed rows gives the same bytes
    oq, os_ = ofp8.quantize_rows(o_ref.cpu())
    assert torch.equal(_bytes(q), oq.view(torch.uint8)) and torch.equal(s.cpu(), os_)


def _check(got: torch.Tensor, want: torch.Tensor, rtol: float, what: str, equal_frac: float | None) -> None:
    got, want = got.float().cpu(), want.float()
    err = (got - want).abs()
    atol = 1e-5 * float(want.abs().max())
    worst = float((err - (rtol * want.abs() + atol)).max())
    assert worst <= 0, f"{what}: max |err| {float(err.max()):.3e} over the bound by {worst:.3e}"
    assert float(err.mean()) <= 2.0 ** -10 * float(want.abs().mean()) + atol, f"{what}: mean |err| {float(err.mean())}"
    if equal_frac is not None:
        frac = float((got == want).float().mean())
        assert frac >= equal_frac, f"{what}: only {frac:.3f} of the outputs are bit-equal"


def _operands(m: int, n: int, k: int, seed: int):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=gen).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=gen) * k ** -0.5 * torch.logspace(-1, 1, k // 128).repeat_interleave(128)).to(
        torch.bfloat16)
    return x, w


@pytest.mark.parametrize("m,n,k,split", [
    (1, 128, 128, 0), (17, 384, 640, 0), (64, 1024, 2048, 0), (64, 1024, 2048, 2), (64, 1024, 2048, 3),
    (100, 256, 1024, 4), (128, 512, 2048, 0), (130, 256, 512, 0), (300, 384, 1280, 0), (64, 1024, 2048, 0x401),
    (64, 1024, 2048, 0x201), (32, 2048, 2048, 0x308),
    (64, 12288, 2048, 0), (20, 12288, 2048, 0),  # 96 tiles: K split over 3 CTAs, two CTAs per SM
    (1000, 512, 2048, 0),  # prefill-scale rows (the mixed batch with the FP8 gate/up): many token chunks
])
def test_gemm_plain_matches_the_blockscaled_oracle(nqt, cuda, m, n, k, split):
    x, w = _operands(m, n, k, m * 7 + n)
    weight = nqt.kernels.Fp8BlockWeight(w.to(cuda))
    xq, xs = nqt.kernels.fp8_quantize_rows(x.to(cuda))
    y = nqt.kernels.linear_fp8(xq, xs, weight, split=split)
    torch.cuda.synchronize()
    assert nqt.kernels.read_status(cuda) == 0
    wq, ws = ofp8.quantize_weight_blocks(w)
    oxq, oxs = ofp8.quantize_rows(x)
    want = ofp8.gemm_blockscaled(oxq, oxs, wq, ws).to(torch.bfloat16)
    _check(y, want, 2.0 ** -7, f"m={m} n={n} k={k} split={split:#x}", 0.97)


@pytest.mark.parametrize("m,split", [(64, 0), (64, 2), (7, 0), (200, 0), (1000, 0)])
def test_gemm_swiglu_matches_the_oracle(nqt, cuda, m, split):
    ffn, hidden = 1536, 2048
    x, w = _operands(m, 2 * ffn, hidden, 100 + m)
    weight = nqt.kernels.Fp8BlockWeight(w.to(cuda), gate_up=True)
    xq, xs = nqt.kernels.fp8_quantize_rows(x.to(cuda))
    y = nqt.kernels.linear_fp8(xq, xs, weight, split=split)
    torch.cuda.synchronize()
    assert nqt.kernels.read_status(cuda) == 0
    assert y.shape == (m, ffn)
    want = ofp8.gate_up_fp8(x, w)
    _check(y, want, 2.0 ** -6, f"swiglu m={m} split={split}", None)


def test_talker_gate_up_shape_end_to_end(nqt, cuda):
    """The talker's gate/up at B = 64 (hidden 2048, FFN 6144), from the fused norm's output."""

    rows, hidden, ffn = 64, 2048, 6144
    gen = torch.Generator(device=cuda).manual_seed(9)
    o = torch.randn(rows, hidden, generator=gen, device=cuda).to(torch.bfloat16)
    res = torch.randn(rows, hidden, generator=gen, device=cuda).to(torch.bfloat16)
    ln = (1 + 0.05 * torch.randn(hidden, generator=gen, device=cuda)).to(torch.bfloat16)
    w = (torch.randn(2 * ffn, hidden, generator=gen, device=cuda) * hidden ** -0.5).to(torch.bfloat16)
    weight = nqt.kernels.Fp8BlockWeight(w, gate_up=True)
    q = torch.empty(rows, hidden, dtype=torch.float8_e4m3fn, device=cuda)
    s = torch.empty(hidden // 128, rows, dtype=torch.float32, device=cuda)
    x = o.clone()
    nqt.kernels.fused_add_rmsnorm_fp8_(x, res, ln, 1e-6, q, s, write_x=True)
    y = nqt.kernels.linear_fp8(q, s, weight)
    torch.cuda.synchronize()
    assert nqt.kernels.read_status(cuda) == 0
    want = ofp8.gate_up_fp8(x.cpu(), w.cpu())
    _check(y, want, 2.0 ** -6, "talker gate_up", None)
    # the FP8 path stays close to the bf16 path it replaces (quantisation error only)
    ref16 = x.float() @ w.float().T
    g, u = ref16[:, :ffn].to(torch.bfloat16).float(), ref16[:, ffn:].to(torch.bfloat16).float()
    bf16_path = g / (1 + torch.exp(-g)) * u
    rel = float((y.float() - bf16_path).norm() / bf16_path.norm())
    assert rel < 0.08, rel


def test_gemm_rejects_bad_arguments(nqt, cuda):
    w = nqt.kernels.Fp8BlockWeight(torch.zeros(256, 256, dtype=torch.bfloat16, device=cuda))
    xq = torch.zeros(4, 256, dtype=torch.float8_e4m3fn, device=cuda)
    xs = torch.ones(2, 4, dtype=torch.float32, device=cuda)
    with pytest.raises(ValueError):
        nqt.kernels.linear_fp8(xq[:, :128], xs, w)
    with pytest.raises(ValueError):
        nqt.kernels.linear_fp8(xq, xs[:1], w)
    with pytest.raises(nqt.NqtError):
        nqt.kernels.linear_fp8(xq, xs, w, split=9)
    with pytest.raises(TypeError):
        nqt.kernels.linear_fp8(xq, xs, object())


def test_split_k_sum_is_deterministic(nqt, cuda):
    """The split-K tile sum adds the partials in rank order whichever CTA completes the tile's ticket, so
    repeated launches give identical bits."""

    x, w = _operands(64, 12288, 2048, 77)
    weight = nqt.kernels.Fp8BlockWeight(w.to(cuda), gate_up=True)
    xq, xs = nqt.kernels.fp8_quantize_rows(x.to(cuda))
    first = nqt.kernels.linear_fp8(xq, xs, weight).clone()
    for _ in range(8):
        assert torch.equal(nqt.kernels.linear_fp8(xq, xs, weight), first)
    assert nqt.kernels.read_status(cuda) == 0
