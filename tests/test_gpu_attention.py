"""GPU parity: QK norm/RoPE + paged K/V write, paged decode, causal prefill and
the code-predictor kernels against the CPU oracle (through the C ABI)."""

from __future__ import annotations

import pytest
import torch

from oracle import attention as oatt
from tests._paged import make_paged

pytestmark = pytest.mark.gpu

ATOL = 2e-2  # bf16 attention outputs


def _decode_case(nqt, cuda, lens, *, page_size=16, hq=16, hkv=8, d=128, seed=0, strided=False):
    cache, indptr, indices, last = make_paged(lens, page_size=page_size, hkv=hkv, d=d, seed=seed)
    g = torch.Generator().manual_seed(seed + 1)
    rows = len(lens)
    if strided:  # q as a view of a packed qkv projection, like layers.py:296-306
        qkv = torch.randn(rows, hq * d + 2 * hkv * d, generator=g).to(torch.bfloat16)
        q_cpu = qkv[:, : hq * d].view(rows, hq, d)
        q_dev = qkv.to(cuda)[:, : hq * d].view(rows, hq, d)
    else:
        q_cpu = torch.randn(rows, hq, d, generator=g).to(torch.bfloat16)
        q_dev = q_cpu.to(cuda)
    ws = torch.zeros(nqt.lib().nqt_decode_workspace_bytes(rows, hq, d), dtype=torch.uint8, device=cuda)
    out = nqt.batch_decode_paged(q_dev, cache.to(cuda), indptr.to(cuda), indices.to(cuda), last.to(cuda), ws)
    torch.cuda.synchronize()
    want = oatt.paged_decode(q_cpu.float(), cache.float(), indptr, indices, last)
    return out.float().cpu(), want


@pytest.mark.parametrize(
    "lens",
    [
        [int(x) for x in torch.randint(16, 513, (8,), generator=torch.Generator().manual_seed(0))],  # config 1
        [1, 15, 16, 17, 31, 32, 33],
        [4096],
        [1],
        [2048, 1, 700, 64, 3, 1999],
    ],
)
def test_decode_matches_oracle(nqt, cuda, lens):
    got, want = _decode_case(nqt, cuda, lens)
    assert torch.isfinite(got).all()
    torch.testing.assert_close(got, want, atol=ATOL, rtol=0)
    assert nqt.kernels.read_status(cuda) == 0


def test_decode_config2_shapes(nqt, cuda):
    lens = torch.randint(64, 2049, (64,), generator=torch.Generator().manual_seed(2)).tolist()
    got, want = _decode_case(nqt, cuda, lens, seed=2, strided=True)
    torch.testing.assert_close(got, want, atol=ATOL, rtol=0)


@pytest.mark.parametrize("page_size", [32, 64, 128])
def test_decode_page_sizes(nqt, cuda, page_size):
    got, want = _decode_case(nqt, cuda, [5, 130, 333, 1024], page_size=page_size, seed=3)
    torch.testing.assert_close(got, want, atol=ATOL, rtol=0)


@pytest.mark.parametrize(("hq", "hkv", "d"), [(16, 8, 64), (8, 8, 128), (16, 4, 128), (8, 2, 64), (6, 3, 128)])
def test_decode_head_layouts(nqt, cuda, hq, hkv, d):
    got, want = _decode_case(nqt, cuda, [77, 300, 16], hq=hq, hkv=hkv, d=d, seed=4)
    torch.testing.assert_close(got, want, atol=ATOL, rtol=0)


def test_decode_golden_fixture(nqt, cuda, golden):
    g = golden("attention.pt")["paged"]
    cache = g["cache"].to(cuda)
    rows = g["q_decode"].shape[0]
    ws = torch.zeros(nqt.lib().nqt_decode_workspace_bytes(rows, 16, 128), dtype=torch.uint8, device=cuda)
    out = nqt.batch_decode_paged(g["q_decode"].to(torch.bfloat16).to(cuda), cache, g["indptr"].to(cuda),
                                 g["indices"].to(cuda), g["last_page_len"].to(cuda), ws)
    torch.testing.assert_close(out.float().cpu(), g["decode_out"], atol=ATOL, rtol=0)


def test_decode_bad_page_id_reports_status(nqt, cuda):
    cache, indptr, indices, last = make_paged([40, 40], seed=5)
    indices[1] = cache.shape[0] + 7  # outside the pool: read as zeros, flagged, no fault
    nqt.kernels.clear_status(cuda)
    ws = torch.zeros(nqt.lib().nqt_decode_workspace_bytes(2, 16, 128), dtype=torch.uint8, device=cuda)
    q = torch.randn(2, 16, 128).to(torch.bfloat16)
    out = nqt.batch_decode_paged(q.to(cuda), cache.to(cuda), indptr.to(cuda), indices.to(cuda), last.to(cuda), ws)
    torch.cuda.synchronize()
    assert nqt.kernels.read_status(cuda) & 0x1
    assert torch.isfinite(out.float()).all()
    nqt.kernels.clear_status(cuda)


def _prefill_case(nqt, cuda, lens, qo_lens, *, page_size=16, hq=16, hkv=8, d=128, seed=0):
    cache, indptr, indices, last = make_paged(lens, page_size=page_size, hkv=hkv, d=d, seed=seed)
    qo_indptr = torch.tensor([0, *torch.tensor(qo_lens).cumsum(0).tolist()], dtype=torch.int32)
    g = torch.Generator().manual_seed(seed + 1)
    q = torch.randn(int(qo_indptr[-1]), hq, d, generator=g).to(torch.bfloat16)
    out = nqt.batch_prefill_paged(q.to(cuda), cache.to(cuda), qo_indptr.to(cuda), indptr.to(cuda),
                                  indices.to(cuda), last.to(cuda))
    torch.cuda.synchronize()
    want = oatt.paged_prefill(q.float(), cache.float(), qo_indptr, indptr, indices, last)
    return out.float().cpu(), want


@pytest.mark.parametrize(
    ("lens", "qo_lens"),
    [
        ([37, 1, 300, 128], [37, 1, 45, 128]),
        ([16, 17, 64, 65], [1, 17, 33, 2]),
        ([1024, 700], [1024, 500]),
        ([5, 200, 33], [0, 64, 33]),
    ],
)
def test_prefill_matches_oracle(nqt, cuda, lens, qo_lens):
    got, want = _prefill_case(nqt, cuda, lens, qo_lens)
    assert torch.isfinite(got).all()
    torch.testing.assert_close(got, want, atol=ATOL, rtol=0)


def test_prefill_ragged_query_tile_pairs(nqt, cuda):
    # a CTA computes two query tiles of 128 / G tokens: chunks that end inside the first tile, exactly
    # at its end, inside and at the end of the second, over short and long contexts, one key block of
    # context or none
    lens = [129, 1, 94, 65, 227, 128, 256, 257, 1033, 64, 191]
    qo_lens = [129, 1, 30, 65, 100, 128, 1, 257, 333, 64, 127]
    got, want = _prefill_case(nqt, cuda, lens, qo_lens, seed=9)
    assert torch.isfinite(got).all()
    torch.testing.assert_close(got, want, atol=ATOL, rtol=0)


@pytest.mark.parametrize("seed", range(6))
def test_prefill_random_batches(nqt, cuda, seed):
    # seeded random batches: 1-9 sequences, chunks of 1-400 tokens over 0-600 tokens of context, the
    # four GQA groups the kernel takes (128 / G tokens per query tile) and three page sizes
    g = torch.Generator().manual_seed(1000 + seed)
    hq, hkv = [(8, 8), (16, 8), (16, 4), (16, 2)][seed % 4]
    page_size = [16, 32, 64][seed % 3]
    b = int(torch.randint(1, 10, (1,), generator=g))
    qo_lens = torch.randint(1, 401, (b,), generator=g).tolist()
    ctx = torch.randint(0, 601, (b,), generator=g).tolist()
    lens = [q + c for q, c in zip(qo_lens, ctx)]
    got, want = _prefill_case(nqt, cuda, lens, qo_lens, page_size=page_size, hq=hq, hkv=hkv, seed=seed)
    assert torch.isfinite(got).all()
    torch.testing.assert_close(got, want, atol=ATOL, rtol=0)


def test_prefill_output_without_a_tensor_map_layout(nqt, cuda):
    # full query tiles normally leave through a TMA store; an output whose token stride is not a
    # multiple of 16 bytes cannot take a tensor map, so every tile goes through the row stores.
    # Both layouts must hold the same values, and the padding columns stay untouched
    lens, qo_lens = [300, 257, 128], [256, 257, 128]
    cache, indptr, indices, last = make_paged(lens, seed=11)
    qo_indptr = torch.tensor([0, *torch.tensor(qo_lens).cumsum(0).tolist()], dtype=torch.int32)
    tokens = int(qo_indptr[-1])
    q = torch.randn(tokens, 16, 128, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16).to(cuda)
    args = (cache.to(cuda), qo_indptr.to(cuda), indptr.to(cuda), indices.to(cuda), last.to(cuda))
    dense = nqt.batch_prefill_paged(q, *args)
    padded = torch.full((tokens, 16 * 128 + 4), 7.0, dtype=torch.bfloat16, device=cuda)
    view = padded[:, : 16 * 128].view(tokens, 16, 128)
    assert view.stride(0) % 8 != 0
    nqt.batch_prefill_paged(q, *args, out=view)
    torch.cuda.synchronize()
    assert torch.equal(view, dense)
    assert bool((padded[:, 16 * 128:] == 7.0).all())


@pytest.mark.parametrize(("hq", "hkv", "d", "page_size"), [(16, 8, 64, 16), (8, 8, 128, 32), (16, 2, 128, 64)])
def test_prefill_layouts(nqt, cuda, hq, hkv, d, page_size):
    got, want = _prefill_case(nqt, cuda, [90, 260], [90, 31], hq=hq, hkv=hkv, d=d, page_size=page_size, seed=7)
    torch.testing.assert_close(got, want, atol=ATOL, rtol=0)


def test_prefill_golden_fixture(nqt, cuda, golden):
    g = golden("attention.pt")["paged"]
    out = nqt.batch_prefill_paged(g["q_prefill"].to(torch.bfloat16).to(cuda), g["cache"].to(cuda),
                                  g["qo_indptr"].to(cuda), g["indptr"].to(cuda), g["indices"].to(cuda),
                                  g["last_page_len"].to(cuda))
    torch.testing.assert_close(out.float().cpu(), g["prefill_out"], atol=ATOL, rtol=0)


def _qk_inputs(tokens, hq, hkv, d, seed):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(tokens, (hq + 2 * hkv) * d, generator=g).to(torch.bfloat16)
    qw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    return qkv, qw, kw


def _split(qkv, hq, hkv, d):
    t = qkv.shape[0]
    return (qkv[:, : hq * d].view(t, hq, d), qkv[:, hq * d: (hq + hkv) * d].view(t, hkv, d),
            qkv[:, (hq + hkv) * d:].view(t, hkv, d))


def test_qk_norm_rope_paged_write(nqt, cuda):
    tokens, hq, hkv, d, P, pages = 40, 16, 8, 128, 16, 12
    qkv, qw, kw = _qk_inputs(tokens, hq, hkv, d, 11)
    g = torch.Generator().manual_seed(12)
    positions = torch.randint(0, 4096, (tokens,), generator=g)
    slots = torch.randperm(pages * P, generator=g)[:tokens]
    wp, wo = slots // P, slots % P
    cache = torch.zeros(pages, 2, P, hkv, d, dtype=torch.bfloat16)
    q_cpu, k_cpu, v_cpu = _split(qkv.clone(), hq, hkv, d)
    oatt.qk_norm_rope_paged_(q_cpu, k_cpu, v_cpu, qw, kw, positions, 1e-6, 1e6, cache, wp, wo)
    qkv_dev = qkv.to(cuda)
    q, k, v = _split(qkv_dev, hq, hkv, d)
    cache_dev = torch.zeros(pages, 2, P, hkv, d, dtype=torch.bfloat16, device=cuda)
    nqt.paired_qk_norm_rope_paged_cache_(q, k, v, qw.to(cuda), kw.to(cuda), positions.to(cuda), 1e-6, 1e6,
                                         cache_dev, wp.to(cuda), wo.to(cuda))
    torch.cuda.synchronize()
    for got, want in ((q.cpu(), q_cpu), (k.cpu(), k_cpu), (cache_dev.cpu(), cache)):
        diff = (got.float() - want.float()).abs()
        assert diff.max().item() <= 2.0 ** -7 and (diff > 0).float().mean().item() < 0.01
    # V is copied bit for bit; cached K equals the in-place rotated K
    assert torch.equal(cache_dev[wp.to(cuda), 1, wo.to(cuda)].cpu(), v_cpu)
    assert torch.equal(cache_dev[wp.to(cuda), 0, wo.to(cuda)], k)


def test_qk_norm_rope_dense_rounding_modes(nqt, cuda):
    tokens, hq, hkv, d = 9, 16, 8, 64
    for round_to_input in (True, False):
        qkv, qw, kw = _qk_inputs(tokens, hq, hkv, d, 21)
        positions = torch.arange(tokens) * 3
        q_cpu, k_cpu, v_cpu = _split(qkv.clone(), hq, hkv, d)
        kc = torch.zeros(tokens, 16, hkv, d, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        oatt.qk_norm_rope_dense_(q_cpu, k_cpu, v_cpu, qw, kw, positions, 1e-6, 1e6,
                                 None if round_to_input else kc, vc, 5, round_to_input=round_to_input)
        q, k, v = _split(qkv.to(cuda), hq, hkv, d)
        kcd, vcd = kc.zero_().to(cuda), torch.zeros_like(vc, device=cuda)
        if round_to_input:
            nqt.paired_qk_norm_rope_(q, k, qw.to(cuda), kw.to(cuda), positions.to(cuda), 1e-6, 1e6)
        else:
            nqt.paired_qk_norm_rope_dense_cache_(q, k, v, qw.to(cuda), kw.to(cuda), positions.to(cuda), 1e-6, 1e6,
                                                 kcd, vcd, 5)
            assert torch.equal(kcd[:, 5], k) and torch.equal(vcd[:, 5].cpu(), v_cpu)
        for got, want in ((q.cpu(), q_cpu), (k.cpu(), k_cpu)):
            diff = (got.float() - want.float()).abs()
            assert diff.max().item() <= 2.0 ** -7 and (diff > 0).float().mean().item() < 0.01


def test_cp_fused_decode_matches_oracle(nqt, cuda):
    rows, hq, hkv, d, cap = 256, 16, 8, 64, 16
    g = torch.Generator().manual_seed(31)
    for cache_pos in (0, 1, 7, 15):
        qkv, qw, kw = _qk_inputs(rows, hq, hkv, d, 32 + cache_pos)
        kc = torch.randn(rows, cap, hkv, d, generator=g).to(torch.bfloat16)
        vc = torch.randn(rows, cap, hkv, d, generator=g).to(torch.bfloat16)
        positions = torch.full((rows,), cache_pos, dtype=torch.long)
        q_cpu, k_cpu, v_cpu = _split(qkv.clone(), hq, hkv, d)
        kc_cpu, vc_cpu = kc.clone(), vc.clone()
        oatt.qk_norm_rope_dense_(q_cpu, k_cpu, v_cpu, qw, kw, positions, 1e-6, 1e6, kc_cpu, vc_cpu, cache_pos,
                                 round_to_input=False)
        want = oatt.short_cache_attention(q_cpu, kc_cpu, vc_cpu, cache_pos + 1)
        q, k, v = _split(qkv.to(cuda), hq, hkv, d)
        kcd, vcd = kc.to(cuda), vc.to(cuda)
        out = nqt.cp_decode_attention_(q, k, v, qw.to(cuda), kw.to(cuda), positions.to(cuda), 1e-6, 1e6, kcd, vcd,
                                       cache_pos)
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float().cpu(), want, atol=ATOL, rtol=0)
        diff = (kcd.cpu().float() - kc_cpu.float()).abs()
        assert diff.max().item() <= 2.0 ** -7
        assert torch.equal(vcd.cpu(), vc_cpu)


def test_short_cache_golden_fixture(nqt, cuda, golden):
    g = golden("attention.pt")["short_cache"]
    out = nqt.decode_attn_nhd_short_cache(g["q"].to(torch.bfloat16).to(cuda), g["k_cache"].to(torch.bfloat16).to(cuda),
                                          g["v_cache"].to(torch.bfloat16).to(cuda), g["length"])
    torch.testing.assert_close(out.float().cpu(), g["out"], atol=ATOL, rtol=0)


def test_decode_overlapping_the_kv_write_sees_each_new_token(nqt, cuda):
    """The decode step's order (attend, executor/talker_kv.py:104-130): the K/V write of each row's one new
    token, then the decode launch.  With overlap_kv_write the decode stages page ids and streams the older
    tiles while the write kernel still runs; the new token (in each row's last tile) and q must still be
    the written ones, so the result equals the oracle on the updated cache and, bit for bit, the launch
    that waits for the write kernel first."""
    hq, hkv, d, P = 16, 8, 128, 16
    g = torch.Generator().manual_seed(21)
    lens = torch.randint(1, 1500, (48,), generator=g).tolist() + [1, 16, 17, 32, 33, 2047, 2048, 2049]
    rows = len(lens)
    cache, indptr, indices, last = make_paged(lens, page_size=P, hkv=hkv, d=d, seed=21)
    pos = torch.tensor(lens) - 1
    wp = indices[indptr[:-1].long() + pos // P].long()
    wo = pos % P
    cache_dev = cache.to(cuda)
    meta = [x.to(cuda) for x in (indptr, indices, last)]
    ws = torch.zeros(nqt.lib().nqt_decode_workspace_bytes(rows, hq, d), dtype=torch.uint8, device=cuda)
    out_a = torch.empty(rows, hq, d, dtype=torch.bfloat16, device=cuda)
    out_b = torch.empty_like(out_a)
    for step in range(4):
        qkv, qw, kw = _qk_inputs(rows, hq, hkv, d, 100 + step)
        qkv = qkv.to(cuda)
        q, k, v = _split(qkv, hq, hkv, d)
        nqt.paired_qk_norm_rope_paged_cache_(q, k, v, qw.to(cuda), kw.to(cuda), pos.to(cuda), 1e-6, 1e6,
                                             cache_dev, wp.to(cuda), wo.to(cuda))
        nqt.batch_decode_paged(q, cache_dev, *meta, ws, out=out_a, plan=step == 0, overlap_kv_write=True)
        nqt.batch_decode_paged(q, cache_dev, *meta, ws, out=out_b, plan=False)
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b), step
        want = oatt.paged_decode(q.float().cpu(), cache_dev.float().cpu(), indptr, indices, last)
        torch.testing.assert_close(out_a.float().cpu(), want, atol=ATOL, rtol=0)
    assert nqt.kernels.read_status(cuda) == 0
