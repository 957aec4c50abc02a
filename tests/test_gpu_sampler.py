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


def _check_case(nqt, cuda, c):
    """Kernel vs oracle on one case.  The oracle's Exp(1) noise belongs to
    torch.topk's rank positions; torch orders exactly tied values arbitrarily
    while the kernel ranks them by token id, so the noise is handed to the
    kernel by token id (the identity permutation when the row has no ties)."""

    details = osamp.row_details(c["logits"], c["temperature"], c["top_k"], c["top_p"], c["seed"], c["offset"],
                                repetition_penalty=c["repetition_penalty"], seen_token_mask=c["seen_token_mask"])
    want = osamp.sample_logits(c["logits"], c["temperature"], c["top_k"], c["top_p"], c["seed"], c["offset"],
                               repetition_penalty=c["repetition_penalty"], seen_token_mask=c["seen_token_mask"])
    rows, vocab = c["logits"].shape
    a = _to(c, cuda)

    def run(noise):
        return nqt.sample_rows(
            a["logits"], a["temperature"], a["top_k"], a["top_p"], a["seed"], a["offset"],
            repetition_penalty=a["repetition_penalty"], seen_token_mask=a["seen_token_mask"],
            noise=noise.to(cuda), return_probs=True,
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
    assert tokens.cpu().tolist() == want.tolist(), c.get("name")
    for row, d in enumerate(details):
        if d is None:
            continue
        k = d[0]
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
