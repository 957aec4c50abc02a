"""CPU restatement of the reference's FP8 block-scaled gate/up path.

Test infrastructure only: the GPU tests, ``smoke()`` and the bench's CPU arms
use it as the checker; the product never imports it.

* ``quantize_weight_blocks`` follows quantize_fp8_weight_blocks
  (model/layers.py:11-25): per 128 x 128 block, amax in fp32 clamped to 1e-4,
  s = 2^ceil(log2(amax / 448)), q = e4m3(w / s).  The exponent is taken from the
  float's bits (exact); ``tests/test_fp8_oracle.py`` checks it against the
  fp32 log2 / ceil / pow formula for every bf16 amax, and the golden fixture
  ``tests/golden/fp8.pt`` pins the whole function to the reference's own output.
* ``quantize_rows`` is the activation rule of the GEMM the reference calls on a
  bf16 input (model/layers.py:242-256, flashinfer fp8_blockscale_gemm_sm90).
  FlashInfer is a dependency outside the reference tree (flashinfer-python
  0.6.16.post2, pyproject.toml:27); its rule is restated from the published
  source of the version importable here (0.6.11.post2, scale_1x128_kernel):
  per token per 128 elements, f = 448 / amax (1 when amax = 0) in fp32,
  q = e4m3(x * f), dequantisation scale 1 / f.  Not pinned by a reference test
  (the library GEMM only runs on sm90).
* ``gemm_blockscaled`` is the exact block-scaled product
  sum_b (Xq_b . Wq_b^T) * sx[b, t] * sw[row / 128, b] in float64, rounded once
  to bf16; ``swiglu`` is silu(bf16 g) * bf16 u (model/layers.py:28-40) on the
  [gate | up] halves of that product.

e4m3 conversion is torch's float8_e4m3fn cast (round to nearest even), the
cast the reference itself uses.
"""

from __future__ import annotations

import numpy as np
import torch

E4M3_MAX = np.float32(448.0)


def ceil_log2(x: np.ndarray) -> np.ndarray:
    """ceil(log2(x)) of positive normal float32 values, exactly (exponent + 1 unless a power of two)."""

    bits = np.asarray(x, dtype=np.float32).view(np.uint32)
    e = ((bits >> 23) & 0xFF).astype(np.int64) - 127
    return np.where((bits & 0x7FFFFF) != 0, e + 1, e)


def weight_block_scales(amax: np.ndarray) -> np.ndarray:
    """Power-of-two block scales from block amax values (float32)."""

    x = np.maximum(np.asarray(amax, dtype=np.float32), np.float32(1e-4)) / E4M3_MAX
    return np.ldexp(np.float32(1.0), ceil_log2(x).astype(np.int32)).astype(np.float32)


def quantize_weight_blocks(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(q [n, k] float8_e4m3fn, scales [n / 128, k / 128] float32) of a bf16 [n, k] weight."""

    n, k = weight.shape
    if n % 128 or k % 128:
        raise ValueError("dimensions must be multiples of 128")
    blocks = weight.float().view(n // 128, 128, k // 128, 128)
    amax = blocks.abs().amax(dim=(1, 3)).numpy()
    scales = torch.from_numpy(weight_block_scales(amax))
    q = (blocks / scales.view(n // 128, 1, k // 128, 1)).to(torch.float8_e4m3fn)
    return q.view(n, k).contiguous(), scales


def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(q [m, k] float8_e4m3fn, scale [k / 128, m] float32) of a bf16 [m, k] activation."""

    m, k = x.shape
    if k % 128:
        raise ValueError("k must be a multiple of 128")
    xf = x.float().numpy().reshape(m, k // 128, 128)
    amax = np.abs(xf).max(axis=2)
    with np.errstate(divide="ignore"):
        f = np.where(amax != 0, E4M3_MAX / np.where(amax != 0, amax, np.float32(1)), np.float32(1)).astype(np.float32)
    scaled = (xf * f[:, :, None]).astype(np.float32)
    q = torch.from_numpy(scaled.reshape(m, k)).to(torch.float8_e4m3fn)
    inv = (np.float32(1) / f).astype(np.float32)
    return q, torch.from_numpy(np.ascontiguousarray(inv.T))


def gemm_blockscaled(xq: torch.Tensor, xscale: torch.Tensor, wq: torch.Tensor, wscale: torch.Tensor) -> torch.Tensor:
    """Exact block-scaled product in float64: Y [m, n]."""

    m, k = xq.shape
    n = wq.shape[0]
    kb = k // 128
    xd = xq.double().view(m, kb, 128)
    wd = wq.double().view(n, kb, 128)
    sx = xscale.double()[:, :m]                          # [kb, m]
    sw = wscale.double().repeat_interleave(128, dim=0)   # [n, kb]
    y = torch.zeros(m, n, dtype=torch.float64)
    for b in range(kb):
        y += (xd[:, b] @ wd[:, b].T) * sx[b][:, None] * sw[:, b][None, :]
    return y


def swiglu(y: torch.Tensor) -> torch.Tensor:
    """silu(g) * u on bf16-rounded halves of a [m, 2d] gate_up product, rounded to bf16."""

    d = y.shape[1] // 2
    g = y[:, :d].to(torch.bfloat16).float()
    u = y[:, d:].to(torch.bfloat16).float()
    return (g / (1.0 + torch.exp(-g)) * u).to(torch.bfloat16)


def gate_up_fp8(x: torch.Tensor, w_gate_up: torch.Tensor) -> torch.Tensor:
    """The reference's FP8 MLP input half, end to end: quantise the weight and the bf16 input, block-scaled
    product, SwiGLU.  x bf16 [m, hidden], w_gate_up bf16 [2 * ffn, hidden] -> bf16 [m, ffn]."""

    wq, ws = quantize_weight_blocks(w_gate_up)
    xq, xs = quantize_rows(x)
    return swiglu(gemm_blockscaled(xq, xs, wq, ws))
