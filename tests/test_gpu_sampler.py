"""GPU parity of the fused sampler: the noise entry against the CPU oracle
(sampled ids bit-exact, filtered probabilities within 1e-5), and the
production Philox draw's contract (replayable, row-local, offset-sensitive)."""

from __future__ import annotations

import pytest
import torch

from oracle import sampler as osamp

pytestmark = pytest.mark.gpu

PROB_ATOL = 1e-5


def _to(c, cuda):
    seen = c["seen_token_mask"]
    return dict(
        logits=c["logits"].to(cuda),
        temperature=c["temperature"].to(cuda),
        top_k=c["top_k"].to(cuda),
        top_p=c["top_p"].to(cuda),
        seed=c["seed"].to(cuda),
        offset=c["offset"].to(cuda),
        repetition_penalty=c["repetition_penalty"].to(cuda) if seen is not None else None,
        seen_token_mask=seen.to(cuda) if seen is not None else None,
    )


def _tie_explained(c, row, d, probs, ids, noise, token):
    """A token that differs from the oracle's on a row with ties: the kept sets (top-k, then top-p) may
    hold different members of a tie group, since torch orders tied values arbitrarily; the multisets of kept
    values must agree and the kernel's token must win the race over its own ranks."""

    scaled = osamp.scaled_rows(c["logits"][row: row + 1], c["temperature"][row: row + 1],
                               None if c["repetition_penalty"] is None else c["repetition_penalty"][row: row + 1],
                               None if c["seen_token_mask"] is None else c["seen_token_mask"][row: row + 1])[0]
    k = d[0]
    kept_k = ids[row, :k][probs[row, :k] > 0].long()
    kept_o = d[2][d[1] > 0]
    if not torch.equal(torch.sort(scaled[kept_k]).values, torch.sort(scaled[kept_o]).values):
        return False
    race = probs[row, :k] / noise[row, :k]
    return int(ids[row, int(torch.argmax(race))]) == token


def _check_case(nqt, cuda, c, kernel_dtype=None):
    """Kernel vs oracle on one case.  The oracle's Exp(1) noise belongs to
    torch.topk's rank positions; torch orders exactly tied values arbitrarily
    while the kernel ranks them by token id, so the noise is handed to the
    kernel by token id (the identity permutation when the row has no ties).
    With ``kernel_dtype`` the kernel reads the logits in that type (values the
    type holds exactly) and computes in fp32 as the oracle does."""

    details = osamp.row_details(c["logits"], c["temperature"], c["top_k"], c["top_p"], c["seed"], c["offset"],
                                repetition_penalty=c["repetition_penalty"], seen_token_mask=c["seen_token_mask"])
    want = osamp.sample_logits(c["logits"], c["temperature"], c["top_k"], c["top_p"], c["seed"], c["offset"],
                               repetition_penalty=c["repetition_penalty"], seen_token_mask=c["seen_token_mask"])
    rows, vocab = c["logits"].shape
    a = _to(c, cuda)
    extra = {}
    if kernel_dtype is not None:
        assert torch.equal(c["logits"].to(kernel_dtype).float(), c["logits"])
        a["logits"] = a["logits"].to(kernel_dtype)
        extra["round_scaled_to_input"] = False

    def run(noise):
        return nqt.sample_rows(
            a["logits"], a["temperature"], a["top_k"], a["top_p"], a["seed"], a["offset"],
            repetition_penalty=a["repetition_penalty"], seen_token_mask=a["seen_token_mask"],
            noise=noise.to(cuda), return_probs=True, **extra,
        )

    _, _, ids_k = run(torch.ones(rows, vocab))
    ids_k = ids_k.cpu().long()
    noise = torch.full((rows, vocab), 1.0e30)
    for row, d in enumerate(details):
        if d is None:
            continue
        pos = {int(t): i for i, t in enumerate(d[2])}
        for r in range(d[0]):
            i = pos.get(int(ids_k[row, r]))
            if i is not None:
                noise[row, r] = d[3][i]
    tokens, probs, ids = run(noise)
    torch.cuda.synchronize()
    if kernel_dtype is None:
        assert tokens.cpu().tolist() == want.tolist(), c.get("name")
    else:
        # values of a 2-byte type tie: a differing token must be explained by the tie order
        t_k = tokens.cpu()
        for row in (t_k != want).nonzero().flatten().tolist():
            assert details[row] is not None and _tie_explained(c, row, details[row], probs.cpu(), ids.cpu(),
                                                                noise, int(t_k[row])), row
    scaled_all = osamp.scaled_rows(c["logits"], c["temperature"], c["repetition_penalty"], c["seen_token_mask"]) \
        if kernel_dtype is not None else None
    for row, d in enumerate(details):
        if d is None:
            continue
        k = d[0]
        if kernel_dtype is not None:
            # tie-agnostic: the ranked values equal the oracle's top-k values, ordered by (value desc, token
            # asc), and the probabilities agree as multisets
            sc, kid = scaled_all[row], ids[row, :k].cpu().long()
            v = sc[kid]
            assert torch.equal(v, torch.sort(sc[d[2]], descending=True).values), row
            assert bool(((v[:-1] > v[1:]) | ((v[:-1] == v[1:]) & (kid[:-1] < kid[1:]))).all()), row
            torch.testing.assert_close(torch.sort(probs[row, :k].cpu()).values, torch.sort(d[1]).values,
                                       atol=PROB_ATOL, rtol=0)
            continue
        got_ids = ids[row, :k].cpu().long()
        pos = {int(t): i for i, t in enumerate(d[2])}
        shared = [r for r in range(k) if int(got_ids[r]) in pos]
        # only exact ties at the k-th value may be chosen differently
        assert len(shared) >= k - int((d[1] == d[1][-1]).sum()), (c.get("name"), row)
        got_p = probs[row, shared].cpu()
        want_p = d[1][[pos[int(got_ids[r])] for r in shared]]
        torch.testing.assert_close(got_p, want_p, atol=PROB_ATOL, rtol=0)


def test_noise_entry_matches_oracle_on_golden_cases(nqt, cuda, golden):
    for c in golden("sampler.pt")["cases"]:
        _check_case(nqt, cuda, c)
        # and the oracle itself reproduces the reference's ids on these inputs
        assert c["tokens"].tolist() == osamp.sample_logits(
            c["logits"], c["temperature"], c["top_k"], c["top_p"], c["seed"], c["offset"],
            repetition_penalty=c["repetition_penalty"], seen_token_mask=c["seen_token_mask"]).tolist()


@pytest.mark.parametrize("seed", range(4))
def test_noise_entry_matches_oracle_random(nqt, cuda, seed):
    g = torch.Generator().manual_seed(100 + seed)
    rows, vocab = 64, 3072
    c = {
        "logits": torch.randn(rows, vocab, generator=g) * 2.0,
        "temperature": torch.rand(rows, generator=g) * 1.5 + 0.05,
        "top_k": torch.randint(0, 200, (rows,), generator=g, dtype=torch.int32),
        "top_p": torch.rand(rows, generator=g) * 0.9 + 0.1,
        "seed": torch.randint(0, 2**62, (rows,), generator=g),
        "offset": torch.randint(0, 2**40, (rows,), generator=g),
        "repetition_penalty": torch.rand(rows, generator=g) + 0.5,
        "seen_token_mask": torch.rand(rows, vocab, generator=g) < 0.05,
    }
    c["temperature"][::9] = 0.0
    c["top_p"][::5] = 1.0
    _check_case(nqt, cuda, c)


def test_bf16_ties_pick_lowest_token_id(nqt, cuda):
    # bf16 logits have ties; the kernel ranks equal values by token id and a tied pick is value-equal
    g = torch.Generator().manual_seed(9)
    logits = (torch.randn(16, 3072, generator=g) * 2).to(torch.bfloat16)
    args = dict(temperature=torch.full((16,), 0.9), top_k=torch.full((16,), 50, dtype=torch.int32),
                top_p=torch.full((16,), 0.95), seed=torch.arange(16), offset=torch.zeros(16, dtype=torch.long))
    tokens, probs, ids = nqt.sample_rows(logits.to(cuda), *(v.to(cuda) for v in args.values()), return_probs=True)
    scaled = (logits / 0.9).to(torch.bfloat16).float()  # round_scaled_to_input: no seen mask, bf16 row
    for row in range(16):
        r_ids = ids[row, :50].cpu().long()
        vals = scaled[row, r_ids]
        assert bool((vals[:-1] >= vals[1:]).all())
        for i in range(49):
            if vals[i] == vals[i + 1]:
                assert r_ids[i] < r_ids[i + 1]
        assert float(vals[-1]) >= float(torch.topk(scaled[row], 50).values[-1])
    assert tokens.shape == (16,)


def _draw(nqt, cuda, logits, seed, offset, **kw):
    rows = logits.shape[0]
    return nqt.sample_rows(logits.to(cuda), torch.full((rows,), 1.0, device=cuda),
                           torch.full((rows,), kw.get("k", 0), dtype=torch.int32, device=cuda),
                           torch.full((rows,), kw.get("p", 1.0), device=cuda), seed.to(cuda), offset.to(cuda)).cpu()


def test_philox_draw_is_replayable_row_local_and_offset_sensitive(nqt, cuda):
    logits = torch.zeros(2, 32)
    first = _draw(nqt, cuda, logits, torch.tensor([41, 42]), torch.tensor([0, 6]))
    assert torch.equal(first, _draw(nqt, cuda, logits, torch.tensor([41, 42]), torch.tensor([0, 6])))
    seen_change = 0
    for off in range(1, 9):
        changed = _draw(nqt, cuda, logits, torch.tensor([41, 42]), torch.tensor([off, 6]))
        assert changed[1] == first[1]
        seen_change += int(changed[0] != first[0])
    assert seen_change >= 6
    # batch row position does not matter: singletons and permutations agree
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(9, 300, generator=g)
    seeds = torch.arange(9) * 7 + 1
    offs = torch.arange(9) * 512
    batched = _draw(nqt, cuda, logits, seeds, offs, k=40, p=0.9)
    single = torch.cat([_draw(nqt, cuda, logits[i: i + 1], seeds[i: i + 1], offs[i: i + 1], k=40, p=0.9)
                        for i in range(9)])
    assert torch.equal(batched, single)
    perm = torch.randperm(9, generator=g)
    permuted = _draw(nqt, cuda, logits[perm], seeds[perm], offs[perm], k=40, p=0.9)
    assert torch.equal(permuted, batched[perm])


def test_philox_draw_follows_the_distribution(nqt, cuda):
    probs = torch.tensor([0.4, 0.3, 0.2, 0.1, 0.0, 0.0, 0.0, 0.0])
    logits = torch.log(probs.clamp_min(1e-30)).expand(20000, 8).contiguous()
    tokens = _draw(nqt, cuda, logits, torch.full((20000,), 5), torch.arange(20000) * 32)
    freq = torch.bincount(tokens, minlength=8).float() / 20000
    assert freq[4:].sum() == 0
    assert (freq[:4] - probs[:4]).abs().max() < 0.015


def test_greedy_penalty_and_seen_update(nqt, cuda):
    # tests/job_separation/test_sampling.py:79-93 and test_cuda_graph_sampling.py:11-36, on the kernel
    seen = torch.tensor([[True, False], [False, False]], device=cuda)
    tokens = nqt.sample_talker_cuda_graph(
        torch.tensor([[10.0, 9.0], [10.0, 9.0]], device=cuda), torch.zeros(2, device=cuda),
        torch.zeros(2, dtype=torch.int32, device=cuda), torch.ones(2, device=cuda),
        torch.tensor([31, 32], device=cuda), torch.tensor([7, 8], device=cuda), torch.tensor([2.0, 1.0], device=cuda),
        seen, update_seen=True)
    assert tokens.cpu().tolist() == [1, 0]
    assert seen.cpu().tolist() == [[True, True], [True, False]]
    tokens = nqt.sample_logits_cuda_graph(
        torch.tensor([[0.0, 3.0, 1.0], [4.0, 0.0, 1.0]], device=cuda), torch.zeros(2, device=cuda),
        torch.ones(2, dtype=torch.int32, device=cuda), torch.ones(2, device=cuda), torch.tensor([7, 11], device=cuda),
        torch.tensor([0, 32], device=cuda))
    assert tokens.cpu().tolist() == [1, 0]
    t = nqt.sample_logits_stateless(torch.tensor([[1.0, 3.0, 2.0]], device=cuda), torch.zeros(1, device=cuda),
                                    torch.zeros(1, dtype=torch.int32, device=cuda), torch.ones(1, device=cuda),
                                    torch.tensor([99], device=cuda), torch.tensor([100], device=cuda))
    assert t.cpu().tolist() == [1]


def test_code_predictor_strided_offsets(nqt, cuda):
    g = torch.Generator().manual_seed(5)
    logits = torch.randn(256, 2048, generator=g).to(torch.bfloat16).to(cuda)
    offsets = (torch.arange(256).view(-1, 1) * 512 + torch.arange(1, 16).view(1, -1) * 32).to(cuda)
    args = (torch.full((256,), 0.9, device=cuda), torch.full((256,), 50, dtype=torch.int32, device=cuda),
            torch.ones(256, device=cuda), torch.arange(256, device=cuda))
    col = nqt.sample_code_predictor_cuda_graph(logits, *args, offsets[:, 3])
    dense = nqt.sample_code_predictor_cuda_graph(logits, *args, offsets[:, 3].contiguous())
    assert torch.equal(col, dense)


def _shaped_rows(g, rows, vocab):
    """Tie-free row shapes that stress the small-k candidate search: masked (-inf) vocab, one dominant
    logit, a tight cluster of 70 near-equal leaders (the refinement level), a plain row, a narrow and a
    wide spread, a boosted block of 100."""

    logits = torch.randn(rows, vocab, generator=g) * 2.0
    logits[0::8, : vocab // 3] = float("-inf")
    logits[1::8, 7] += 60.0
    logits[2::8, 200:270] = 5.0 + torch.randn(logits[2::8, 200:270].shape, generator=g) * 1e-3
    logits[4::8] *= 1e-3
    logits[5::8] *= 40.0
    logits[6::8, :100] += 9.0
    return logits


@pytest.mark.parametrize("top_k", [1, 2, 17, 50, 63, 64, 65])
def test_small_k_candidate_search_matches_oracle_on_shaped_rows(nqt, cuda, top_k):
    g = torch.Generator().manual_seed(300 + top_k)
    rows, vocab = 64, 2048
    c = {
        "logits": _shaped_rows(g, rows, vocab),
        "temperature": torch.rand(rows, generator=g) * 1.5 + 0.05,
        "top_k": torch.full((rows,), top_k, dtype=torch.int32),
        "top_p": torch.where(torch.arange(rows) % 2 == 0, torch.ones(rows), torch.rand(rows, generator=g) * 0.9 + 0.1),
        "seed": torch.randint(0, 2**62, (rows,), generator=g),
        "offset": torch.randint(0, 2**40, (rows,), generator=g),
        "repetition_penalty": None,
        "seen_token_mask": None,
    }
    _check_case(nqt, cuda, c)


def test_small_k_path_with_penalty(nqt, cuda):
    g = torch.Generator().manual_seed(77)
    rows, vocab = 64, 3072
    c = {
        "logits": _shaped_rows(g, rows, vocab),
        "temperature": torch.full((rows,), 0.9),
        "top_k": torch.full((rows,), 50, dtype=torch.int32),
        "top_p": torch.full((rows,), 0.95),
        "seed": torch.arange(rows),
        "offset": torch.arange(rows) * 512,
        "repetition_penalty": torch.full((rows,), 1.05),
        "seen_token_mask": torch.rand(rows, vocab, generator=g) < 0.02,
    }
    _check_case(nqt, cuda, c)


@pytest.mark.parametrize("top_k", [20, 64, 65, 300])
def test_tied_rows_rank_by_value_then_token_id(nqt, cuda, top_k):
    # flat rows and integer-valued rows: every boundary is a tie, so the top-k set and its order are
    # fixed by (value desc, token id asc); the kept probabilities are the softmax of those values
    g = torch.Generator().manual_seed(top_k)
    rows, vocab = 16, 2048
    logits = torch.randn(rows, vocab, generator=g).mul(1.5).round()
    logits[::4] = 0.25
    temperature = torch.full((rows,), 1.0)
    tokens, probs, ids = nqt.sample_rows(
        logits.to(cuda), temperature.to(cuda), torch.full((rows,), top_k, dtype=torch.int32, device=cuda),
        torch.ones(rows, device=cuda), torch.arange(rows, device=cuda), torch.zeros(rows, dtype=torch.long, device=cuda),
        return_probs=True)
    ids, probs = ids.cpu().long(), probs.cpu()
    for row in range(rows):
        order = sorted(range(vocab), key=lambda i: (-float(logits[row, i]), i))[:top_k]
        assert ids[row, :top_k].tolist() == order, row
        want = torch.softmax(logits[row, order], dim=0)
        torch.testing.assert_close(probs[row, :top_k], want, atol=PROB_ATOL, rtol=0)
        assert int(tokens[row]) in order


@pytest.mark.parametrize("rows", [400, 800, 2048])
def test_warps_per_row_variants_match_oracle(nqt, cuda, rows):
    # the launch gives a row 8, 4, 2 or 1 warps depending on the batch; each width against the oracle
    g = torch.Generator().manual_seed(rows)
    vocab = 2048
    c = {
        "logits": _shaped_rows(g, rows, vocab),
        "temperature": torch.rand(rows, generator=g) * 1.5 + 0.05,
        "top_k": torch.randint(1, 80, (rows,), generator=g, dtype=torch.int32),
        "top_p": torch.where(torch.arange(rows) % 2 == 0, torch.ones(rows), torch.rand(rows, generator=g) * 0.9 + 0.1),
        "seed": torch.randint(0, 2**62, (rows,), generator=g),
        "offset": torch.randint(0, 2**40, (rows,), generator=g),
        "repetition_penalty": torch.rand(rows, generator=g) + 0.5,
        "seen_token_mask": torch.rand(rows, vocab, generator=g) < 0.03,
    }
    c["temperature"][::11] = 0.0
    _check_case(nqt, cuda, c)


# ---- 2-byte logits: 32-bit rank keys -------------------------------------------------------------
# Rows of bf16 / fp16 logits whose y is not rounded to the logits type rank their candidates with 32-bit
# keys (20-bit penalised value, 12-bit token); fp32 logits holding the same values take the 64-bit ranking.
# Both compute in fp32, so the ranks must agree exactly.


def _mixed_case(g, rows, vocab, dtype=torch.bfloat16):
    """Rows of every kind the fast paths meet: plain penalised rows (the stacked-step workload), greedy,
    k = 1 / 17 / 64 / 65 / 0, top-p off and 0.5, penalty below one and 1.5, masked vocab, ties, a dominant
    logit, NaN and +inf."""

    logits = (torch.randn(rows, vocab, generator=g) * 2.0)
    kind = torch.arange(rows) % 16
    logits[kind == 8, : vocab // 3] = float("-inf")
    logits[kind == 9] = logits[kind == 9].mul(0.75).round()
    logits[kind == 10, 11] += 30.0
    logits[kind == 6, 5] = float("nan")
    logits[kind == 7, 9] = float("inf")
    temperature = torch.full((rows,), 0.9)
    temperature[kind == 0] = 0.0
    temperature[kind == 12] = 1.7
    top_k = torch.full((rows,), 50, dtype=torch.int32)
    top_k[kind == 1] = 64
    top_k[kind == 2] = 65
    top_k[kind == 3] = 0
    top_k[kind == 11] = 1
    top_k[kind == 13] = 17
    top_p = torch.full((rows,), 0.95)
    top_p[kind == 4] = 1.0
    top_p[kind == 14] = 0.5
    penalty = torch.full((rows,), 1.05)
    penalty[kind == 5] = 0.8
    penalty[kind == 15] = 1.5
    return {
        "logits": logits.to(dtype),
        "temperature": temperature,
        "top_k": top_k,
        "top_p": top_p,
        "seed": torch.randint(0, 2**62, (rows,), generator=g),
        "offset": torch.randint(0, 2**40, (rows,), generator=g),
        "repetition_penalty": penalty,
        "seen_token_mask": torch.rand(rows, vocab, generator=g) < 0.02,
    }


def _sample(nqt, a, sl=slice(None), noise=None, probs=False):
    return nqt.sample_rows(
        a["logits"][sl], a["temperature"][sl], a["top_k"][sl], a["top_p"][sl], a["seed"][sl], a["offset"][sl],
        repetition_penalty=None if a["repetition_penalty"] is None else a["repetition_penalty"][sl],
        seen_token_mask=None if a["seen_token_mask"] is None else a["seen_token_mask"][sl],
        round_scaled_to_input=False, noise=None if noise is None else noise[sl], return_probs=probs)


@pytest.mark.parametrize("rows", [64, 2048])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_seen", [True, False])
def test_rank_keys_match_the_64_bit_ranking(nqt, cuda, rows, dtype, with_seen):
    """The same values as 2-byte and as fp32 logits: identical ranks (token ids in rank order), the
    probabilities within 1e-6, and the same draws, both from the production Philox stream and from the
    noise entry, except where two ranks' p / E agree to rounding (the softmax sums in another order)."""

    g = torch.Generator().manual_seed(rows + int(with_seen) + (7 if dtype == torch.float16 else 0))
    c = _mixed_case(g, rows, 3072, dtype)
    if not with_seen:
        c["repetition_penalty"] = c["seen_token_mask"] = None
    a = {k: (v.to(cuda) if v is not None else None) for k, v in c.items()}
    f = dict(a, logits=a["logits"].float())
    t2, tf = _sample(nqt, a), _sample(nqt, f)
    torch.cuda.synchronize()
    assert int((t2 != tf).sum()) <= 2
    noise = torch.empty(rows, 3072).exponential_(generator=g).to(cuda)
    t1, p1, i1 = _sample(nqt, a, noise=noise, probs=True)
    t2, p2, i2 = _sample(nqt, f, noise=noise, probs=True)
    torch.cuda.synchronize()
    assert torch.equal(i1, i2)
    torch.testing.assert_close(p1, p2, atol=1e-6, rtol=0, equal_nan=True)  # NaN rows: NaN on both
    for row in (t1 != t2).nonzero().flatten().tolist():
        r1 = int((i1[row] == t1[row]).nonzero()[0])
        r2 = int((i1[row] == t2[row]).nonzero()[0])
        s1 = float(p1[row, r1] / noise[row, r1])
        s2 = float(p1[row, r2] / noise[row, r2])
        assert abs(s1 - s2) <= 1e-6 * max(s1, s2), (row, s1, s2)


def test_bf16_rows_match_oracle(nqt, cuda):
    g = torch.Generator().manual_seed(33)
    rows = 2048
    c = _mixed_case(g, rows, 3072)
    # finite rows without whole tie groups: torch.topk keeps an arbitrary part of a tie group at the k-th
    # value, so NaN / +inf rows and integer-valued rows are covered against the 64-bit ranking above
    kind = torch.arange(rows) % 16
    redo = (kind == 6) | (kind == 7) | (kind == 9)
    c["logits"][redo] = (torch.randn(int(redo.sum()), 3072, generator=g) * 2.0).to(torch.bfloat16)
    c["logits"] = c["logits"].float()  # bf16 values: the oracle computes on them in fp32, the kernel reads bf16
    _check_case(nqt, cuda, c, kernel_dtype=torch.bfloat16)


def test_rank_keys_on_unaligned_rows_and_seen_update(nqt, cuda):
    # rows that do not start on 16 bytes take the general path; update_seen marks each drawn token once
    g = torch.Generator().manual_seed(44)
    rows = 512
    c = _mixed_case(g, rows, 3072)
    a = {k: v.to(cuda) for k, v in c.items()}
    wide = torch.full((rows, 3080), float("-inf"), dtype=torch.bfloat16, device=cuda)
    wide[:, 4:3076] = a["logits"]
    t_shift = _sample(nqt, dict(a, logits=wide[:, 4:3076]))
    t_plain = _sample(nqt, a)
    assert torch.equal(t_shift, t_plain)
    seen = a["seen_token_mask"].clone()
    tokens = nqt.sample_rows(a["logits"], a["temperature"], a["top_k"], a["top_p"], a["seed"], a["offset"],
                             repetition_penalty=a["repetition_penalty"], seen_token_mask=seen, update_seen=True,
                             round_scaled_to_input=False)
    torch.cuda.synchronize()
    assert torch.equal(tokens, t_plain)
    idx = torch.arange(rows, device=cuda)
    assert bool(seen[idx, tokens].all())
    assert int(seen.ne(a["seen_token_mask"]).sum()) == int((~a["seen_token_mask"][idx, tokens]).sum())
