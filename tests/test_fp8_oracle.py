"""CPU: the FP8 block-scaled gate/up oracle (oracle/fp8.py) against the
reference's own quantize_fp8_weight_blocks output (tests/golden/fp8.pt, made
by tests/golden/make_golden.py) and against the formula it restates."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from oracle import fp8 as ofp8

GOLDEN = Path(__file__).resolve().parent / "golden" / "fp8.pt"


def test_weight_quantiser_matches_the_reference_output_bit_for_bit():
    g = torch.load(GOLDEN)
    q, scales = ofp8.quantize_weight_blocks(g["weight"])
    assert torch.equal(scales, g["scales"])
    assert torch.equal(q.view(torch.uint8), g["q"])
    # the fixture covers the clamp, exact power-of-two boundaries and underflow to zero
    assert float(g["scales"][0, 0]) == 2.0 ** -22 and float(g["scales"][0, 2]) == 2.0 ** -3
    assert float(g["scales"][0, 5]) == 1.0
    assert int((g["q"].view(2, 128, 6, 128)[0, :, 4] & 0x7F).count_nonzero()) == 0  # +-0 only


def test_exact_exponent_equals_the_fp32_log2_formula_for_every_bf16_amax():
    """The oracle (and the kernel) take ceil(log2(x)) from the float's bits; the reference computes
    pow(2, ceil(log2(max(amax, 1e-4) / 448))) in fp32 tensors.  Both agree on every positive finite bf16."""

    bits = torch.arange(0x0001, 0x7F80, dtype=torch.int32).to(torch.int16)
    amax = bits.view(torch.bfloat16).float()
    want = torch.pow(2.0, torch.ceil(torch.log2(amax.clamp(1e-4) / 448.0)))
    got = torch.from_numpy(ofp8.weight_block_scales(amax.numpy()))
    assert torch.equal(got, want)


def test_activation_rule_round_trips_within_e4m3_precision():
    g = torch.Generator().manual_seed(2)
    x = (torch.randn(9, 512, generator=g) * torch.logspace(-4, 4, 9).view(9, 1)).to(torch.bfloat16)
    x[3, 128:256] = 0.0  # an all-zero block: factor 1, scale 1
    q, s = ofp8.quantize_rows(x)
    assert s.shape == (4, 9) and float(s[1, 3]) == 1.0
    assert int((q.view(torch.uint8)[3, 128:256] & 0x7F).count_nonzero()) == 0
    deq = q.float().view(9, 4, 128) * s.T.reshape(9, 4, 1)
    xf = x.float().view(9, 4, 128)
    # e4m3 keeps 3 mantissa bits: relative error <= 2^-4 for normal values, absolute below the subnormal step
    err = (deq - xf).abs()
    bound = 2.0 ** -4 * xf.abs() + 2.0 ** -9 * s.T.reshape(9, 4, 1)
    assert bool((err <= bound).all())
    # each block's largest element lands on +-448
    top = q.float().view(9, 4, 128).abs().amax(dim=2)
    nonzero = xf.abs().amax(dim=2) > 0
    assert bool((top[nonzero] == 448.0).all())


def test_blockscaled_product_equals_the_dequantised_product():
    g = torch.Generator().manual_seed(4)
    x = torch.randn(5, 384, generator=g).to(torch.bfloat16)
    w = (torch.randn(256, 384, generator=g) * 0.03).to(torch.bfloat16)
    xq, xs = ofp8.quantize_rows(x)
    wq, ws = ofp8.quantize_weight_blocks(w)
    y = ofp8.gemm_blockscaled(xq, xs, wq, ws)
    xd = xq.double().view(5, 3, 128) * xs.T.double().reshape(5, 3, 1)
    wd = wq.double().view(256, 3, 128) * ws.double().view(2, 1, 3, 1).expand(2, 128, 3, 1).reshape(256, 3, 1)
    assert torch.allclose(y, xd.view(5, 384) @ wd.view(256, 384).T, rtol=1e-12, atol=1e-12)
    out = ofp8.swiglu(y)
    assert out.shape == (5, 128) and out.dtype == torch.bfloat16
    assert np.isfinite(out.float().numpy()).all()
