"""GPU: the weight-streaming tcgen05 GEMM (nqt_gemm_bf16 on nqt_gemm_pack_weight
layouts) against a torch
fp32 reference on the decoder projection shapes (talker M=64, code predictor
M=256, ragged M), every epilogue and every cluster split."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(x, w, bias=None):
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    return y


def _close(got, want):
    # one bf16 rounding of the output plus fp32 accumulation-order differences
    err = (got.float() - want).abs()
    tol = 2.0 ** -7 * want.abs() + 1e-2
    assert bool((err <= tol).all()), (err.max().item(), (err - tol).max().item())


SHAPES = [
    (64, 4096, 2048),   # talker qkv
    (64, 2048, 2048),   # talker o
    (64, 2048, 6144),   # talker down
    (64, 3072, 2048),   # talker codec head
    (256, 2048, 1024),  # cp qkv
    (256, 1024, 3072),  # cp down
    (37, 1024, 512),    # ragged rows (TMA zero fill)
    (1, 256, 128),
]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_plain_matches_fp32_reference(nqt, cuda, m, n, k):
    g = torch.Generator(device=cuda).manual_seed(m * 7 + n + k)
    x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=cuda) * k ** -0.5).to(torch.bfloat16)
    y = nqt.kernels.linear(x, nqt.kernels.PackedWeight(w))
    torch.cuda.synchronize()
    _close(y, _ref(x, w))
    assert nqt.kernels.read_status(cuda) == 0


@pytest.mark.parametrize("split", [1, 2, 3, 5, 8])
def test_every_k_split_gives_the_same_result(nqt, cuda, split):
    # one CTA per tile, and clusters of 2..8 CTAs splitting K (uneven slices at 3 and 5) reduced
    # through distributed shared memory; called twice: nothing carries over between calls
    g = torch.Generator(device=cuda).manual_seed(11)
    x = torch.randn(64, 2048, generator=g, device=cuda).to(torch.bfloat16)
    w = (torch.randn(1024, 2048, generator=g, device=cuda) * 2048 ** -0.5).to(torch.bfloat16)
    pw = nqt.kernels.PackedWeight(w)
    want = _ref(x, w)
    for _ in range(2):
        y = nqt.kernels.linear(x, pw, split=split)
        torch.cuda.synchronize()
        _close(y, want)
    assert nqt.kernels.read_status(cuda) == 0


def test_split_beyond_the_cluster_limit_is_rejected(nqt, cuda):
    x = torch.randn(64, 512, device=cuda).to(torch.bfloat16)
    pw = nqt.kernels.PackedWeight((torch.randn(256, 512, device=cuda) * 0.05).to(torch.bfloat16))
    with pytest.raises(nqt.NqtError):
        nqt.kernels.linear(x, pw, split=9)


def test_bias_epilogue(nqt, cuda):
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(256, 2048, generator=g, device=cuda).to(torch.bfloat16)
    w = (torch.randn(1024, 2048, generator=g, device=cuda) * 2048 ** -0.5).to(torch.bfloat16)
    b = torch.randn(1024, generator=g, device=cuda).to(torch.bfloat16)
    y = nqt.kernels.linear(x, nqt.kernels.PackedWeight(w), b)
    torch.cuda.synchronize()
    _close(y, _ref(x, w, b))


@pytest.mark.parametrize("m,f,k", [(64, 6144, 2048), (256, 3072, 1024), (20, 128, 256)])
def test_silu_mul_epilogue_equals_gemm_then_silu_and_mul(nqt, cuda, m, f, k):
    g = torch.Generator(device=cuda).manual_seed(f + m)
    x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
    w = (torch.randn(2 * f, k, generator=g, device=cuda) * k ** -0.5).to(torch.bfloat16)
    fused = nqt.kernels.linear(x, nqt.kernels.PackedWeight(w, gate_up=True))
    gate_up = nqt.kernels.linear(x, nqt.kernels.PackedWeight(w))
    unfused = nqt.kernels.silu_and_mul(gate_up)
    torch.cuda.synchronize()
    # same accumulation per output element, same roundings: identical up to the K-split order
    err = (fused.float() - unfused.float()).abs()
    assert bool((err <= 2.0 ** -7 * unfused.float().abs() + 1e-2).all()), err.max().item()
    ref = _ref(x, w)
    want = torch.nn.functional.silu(ref[:, :f].bfloat16().float()) * ref[:, f:].bfloat16().float()
    _close(fused, want)


def test_graph_capture_and_rejects_bad_shapes(nqt, cuda):
    x = torch.randn(64, 512, device=cuda).to(torch.bfloat16)
    w = (torch.randn(256, 512, device=cuda) * 0.05).to(torch.bfloat16)
    out = torch.empty(64, 256, dtype=torch.bfloat16, device=cuda)
    pw = nqt.kernels.PackedWeight(w)
    nqt.kernels.linear(x, pw, out=out)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        nqt.kernels.linear(x, pw, out=out)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    _close(out, _ref(x, w))
    with pytest.raises(ValueError):
        nqt.kernels.PackedWeight(w[:200])  # n not a multiple of 128
    with pytest.raises(nqt.NqtError):
        nqt.kernels.linear(torch.randn(300, 512, device=cuda).to(torch.bfloat16), pw)  # m > 256


def test_packed_layout_is_the_swizzled_tile_order(nqt, cuda):
    # tile (t, kb) row r chunk c holds W[128 t + r, 64 kb + 8 c : +8] at chunk c ^ (r % 8)
    n, k = 256, 128
    w = torch.arange(n * k, device=cuda, dtype=torch.float32).remainder(251).to(torch.bfloat16).view(n, k)
    packed = nqt.kernels.PackedWeight(w).data.view(n // 128, k // 64, 128, 8, 8).cpu()
    wc = w.cpu().view(n // 128, 128, k // 64, 8, 8)
    for t in range(n // 128):
        for kb in range(k // 64):
            for r in (0, 1, 7, 8, 127):
                for c in range(8):
                    assert torch.equal(packed[t, kb, r, c ^ (r % 8)], wc[t, r, kb, c])
