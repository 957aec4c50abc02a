"""CPU: the oracle against the reference's own outputs (tests/golden/*.pt,
made by tests/golden/make_golden.py) and the reference tests' known answers."""

from __future__ import annotations

import pytest
import torch

from oracle import attention as oatt
from oracle import planner as oplan
from oracle import sampler as osamp


# ---------------------------------------------------------------- sampler
def _args(c):
    return (c["logits"], c["temperature"], c["top_k"], c["top_p"], c["seed"], c["offset"])


def test_sampler_tokens_match_reference(golden):
    for c in golden("sampler.pt")["cases"]:
        tokens = osamp.sample_logits(*_args(c), repetition_penalty=c["repetition_penalty"],
                                     seen_token_mask=c["seen_token_mask"])
        assert tokens.tolist() == c["tokens"].tolist(), c["name"]


def test_sampler_filtered_probabilities_match_reference(golden):
    for c in golden("sampler.pt")["cases"]:
        details = osamp.row_details(*_args(c), repetition_penalty=c["repetition_penalty"],
                                    seen_token_mask=c["seen_token_mask"])
        sampled = [d for d in details if d is not None]
        assert len(sampled) == len(c["multinomial_probs"]), c["name"]
        for d, ref_probs in zip(sampled, c["multinomial_probs"], strict=True):
            assert torch.equal(d[1], ref_probs), c["name"]


def test_exponential_race_noise_reproduces_multinomial(golden):
    # the parity mechanism of the GPU noise entry: argmax(p / E) == multinomial(p, 1)
    for c in golden("sampler.pt")["cases"]:
        details = osamp.row_details(*_args(c), repetition_penalty=c["repetition_penalty"],
                                    seen_token_mask=c["seen_token_mask"])
        for row, d in enumerate(details):
            if d is not None:
                assert d[4] == int(c["tokens"][row]), (c["name"], row)


def test_sampler_known_answers():
    # tests/job_separation/test_sampling.py:64-76
    t = osamp.sample_logits(torch.tensor([[1.0, 3.0, 2.0]]), torch.zeros(1), torch.zeros(1, dtype=torch.int32),
                            torch.ones(1), torch.tensor([99]), torch.tensor([100]))
    assert t.tolist() == [1]
    # tests/job_separation/test_sampling.py:79-93 (greedy rows still see the penalty)
    t = osamp.sample_logits(torch.tensor([[10.0, 9.0], [10.0, 9.0]]), torch.zeros(2),
                            torch.zeros(2, dtype=torch.int32), torch.ones(2), torch.tensor([31, 32]),
                            torch.tensor([7, 8]), repetition_penalty=torch.tensor([2.0, 1.0]),
                            seen_token_mask=torch.tensor([[True, False], [False, False]]))
    assert t.tolist() == [1, 0]
    # tests/model_optimization/test_cuda_graph_sampling.py:11-36
    t = osamp.sample_logits(torch.tensor([[0.0, 3.0, 1.0], [4.0, 0.0, 1.0]]), torch.zeros(2),
                            torch.ones(2, dtype=torch.int32), torch.ones(2), torch.tensor([7, 11]),
                            torch.tensor([0, 32]))
    assert t.tolist() == [1, 0]


def test_sampler_row_local_and_offset_sensitive():
    # tests/job_separation/test_sampling.py:11-25
    logits = torch.zeros((2, 32))
    kw = dict(temperature=torch.ones(2), top_k=torch.full((2,), 32, dtype=torch.int32), top_p=torch.ones(2),
              seed=torch.tensor([41, 42]), offset=torch.tensor([0, 6]))
    first = osamp.sample_logits(logits, **kw)
    assert torch.equal(first, osamp.sample_logits(logits, **kw))
    changed = osamp.sample_logits(logits, **{**kw, "offset": torch.tensor([1, 6])})
    assert first[0] != changed[0] and first[1] == changed[1]


# ---------------------------------------------------------------- planner
def replay_planner_script(data, on_step):
    """Replay the reference's op script on the host oracle; on_step(step, meta_or_error)."""

    pool = oplan.HostPagePool(data["total_pages"], data["page_size"], data["scratch"])
    for step in data["steps"]:
        op = step["op"]
        if op == "add":
            pool.add_request(step["rid"])
            continue
        if op == "remove":
            pool.remove_request(step["rid"])
            continue
        try:
            meta = pool.metadata(step["rows"], step["advances"], step["capture_rows"], step["token_capacity"],
                                 op == "prefill")
        except (ValueError, oplan.KVAllocationError) as error:
            on_step(step, error)
            continue
        on_step(step, meta)
        for rid, ok in zip(step["rows"], step["publish"], strict=True):
            (pool.publish if ok else pool.discard)(rid)
    return pool


def test_planner_metadata_matches_reference(golden):
    data = golden("planner.pt")
    checked = {"meta": 0, "error": 0}

    def on_step(step, got):
        if "error" in step:
            assert isinstance(got, Exception) and type(got).__name__ == step["error"]
            checked["error"] += 1
            return
        assert not isinstance(got, Exception), got
        for key in ("qo_indptr", "paged_kv_indptr", "paged_kv_indices", "paged_kv_last_page_len", "position_ids",
                    "write_pages", "write_offsets"):
            assert got[key] == step[key], key
        for new, pages, rid in zip(got["new_pages"], step["publication_pages"], step["rows"], strict=True):
            assert pages[len(pages) - len(new):] == new
        checked["meta"] += 1

    pool = replay_planner_script(data, on_step)
    assert checked["meta"] >= 30 and checked["error"] > 0
    for rid, state in data["final"].items():
        assert pool.pages[rid] == state["pages"] and pool.length[rid] == state["length"]
    assert len(pool.free) == data["free_pages"]


def test_planner_known_answers():
    # tests/model_optimization/test_talker_kv_metadata.py:17-56
    pool = oplan.HostPagePool(16, 4, 4)
    pool.add_request("a")
    pool.add_request("b")
    meta = pool.metadata(["a", "b"], [3, 2], 4, 8, True)
    assert meta["qo_indptr"] == [0, 3, 5, 5, 5]
    assert meta["position_ids"] == [0, 1, 2, 0, 1, 0, 0, 0]
    assert meta["write_offsets"][:5] == [0, 1, 2, 0, 1]
    assert len(set(meta["paged_kv_indices"][-2:])) == 2
    pad = set(zip(meta["write_pages"][5:], meta["write_offsets"][5:], strict=True))
    assert len(pad) == 3 and not pad & set(zip(meta["write_pages"][:5], meta["write_offsets"][:5], strict=True))
    # :59-89 decode after a published 3-token prefill
    pool = oplan.HostPagePool(16, 4, 2)
    pool.add_request("a")
    pool.metadata(["a"], [3], 1, 4, True)
    pool.publish("a")
    meta = pool.metadata(["a"], [1], 2, 2, False)
    assert meta["position_ids"] == [3, 0] and meta["write_offsets"][0] == 3
    assert meta["write_pages"][1] == pool.scratch[1]
    # :92-119 capacity errors
    pool = oplan.HostPagePool(16, 4, 1)
    pool.add_request("a")
    with pytest.raises(ValueError, match="CUDA Graph rows exceed"):
        pool.metadata(["a"], [1], 2, 2, False)
    with pytest.raises(ValueError, match="token capacity exceeds"):
        pool.metadata(["a"], [1], 1, 8, True)


def test_allocator_rollback_and_recycling():
    # tests/model_optimization/test_staging_cache_rng.py:102-136
    pool = oplan.HostPagePool(3, 4, 0)
    pool.add_request("a")
    pool.add_request("b")
    with pytest.raises(oplan.KVAllocationError):
        pool.reserve(["a", "b"], [1, 9])
    assert len(pool.free) == 3
    for i in range(12):
        rid = f"r{i}"
        pool.add_request(rid)
        pool.reserve([rid], [9])
        pool.publish(rid)
        assert not pool.free
        pool.remove_request(rid)
        assert len(pool.free) == 3


# ---------------------------------------------------------------- attention
def test_norm_rope_matches_reference_math(golden):
    g = golden("attention.pt")["norm_rope"]
    for name, x, w in (("q", g["q"], g["q_weight"]), ("k", g["k"], g["k_weight"])):
        got = oatt.norm_rope(x, w, g["positions"], g["eps"], g["theta"], round_norm=True).to(torch.bfloat16)
        want = g[f"{name}_out"]
        diff = (got.float() - want.float()).abs()
        # identical math with a different inv_freq / FMA order: normalised values are O(1), so the
        # rounding error is at most one bf16 ulp at magnitude 1-2 (2^-7), and it is rare
        assert diff.max().item() <= 2.0 ** -7
        assert (diff > 0).float().mean().item() < 0.01


def test_paged_decode_and_prefill_match_reference_math(golden):
    g = golden("attention.pt")["paged"]
    cache = g["cache"].float()
    dec = oatt.paged_decode(g["q_decode"], cache, g["indptr"], g["indices"], g["last_page_len"])
    torch.testing.assert_close(dec, g["decode_out"], atol=1e-5, rtol=1e-5)
    pre = oatt.paged_prefill(g["q_prefill"], cache, g["qo_indptr"], g["indptr"], g["indices"], g["last_page_len"])
    torch.testing.assert_close(pre, g["prefill_out"], atol=1e-5, rtol=1e-5)


def test_short_cache_matches_reference_math(golden):
    g = golden("attention.pt")["short_cache"]
    out = oatt.short_cache_attention(g["q"], g["k_cache"], g["v_cache"], g["length"])
    torch.testing.assert_close(out, g["out"], atol=1e-5, rtol=1e-5)
