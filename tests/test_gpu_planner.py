"""GPU planner parity: the reference's op script (tests/golden/planner.pt)
replayed through the device planner must give bit-identical metadata,
allocation and final state; pool exhaustion reserves nothing."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


class Buffers:
    """Static metadata buffers shaped like a binding's (capture rows, token capacity)."""

    def __init__(self, rows, tokens, total_pages, device):
        self.qo_indptr = torch.zeros(rows + 1, dtype=torch.int32, device=device)
        self.kv_indptr = torch.zeros(rows + 1, dtype=torch.int32, device=device)
        self.kv_indices = torch.zeros(total_pages + rows, dtype=torch.int32, device=device)
        self.last_page_len = torch.zeros(rows, dtype=torch.int32, device=device)
        self.position_ids = torch.zeros(tokens, dtype=torch.long, device=device)
        self.write_pages = torch.zeros(tokens, dtype=torch.long, device=device)
        self.write_offsets = torch.zeros(tokens, dtype=torch.long, device=device)


def _planner(nqt, data, cuda, capture_rows, token_capacity):
    return nqt.DevicePagePlanner(total_pages=data["total_pages"], page_size=data["page_size"], slots=16,
                                 max_pages_per_slot=data["total_pages"], scratch_page_count=data["scratch"],
                                 capture_rows=capture_rows, token_capacity=token_capacity, device=cuda)


def test_device_planner_replays_reference_script(nqt, cuda, golden):
    data = golden("planner.pt")
    planners = {}
    # one planner state shared by prefill (24 tokens) and decode (4 tokens) captures: use one pool,
    # two planner views over the same state tensor
    base = _planner(nqt, data, cuda, 4, 24)
    dec = _planner(nqt, data, cuda, 4, 4)
    dec.state = base.state
    dec._slot_of = base._slot_of
    dec._free_slots = base._free_slots
    planners = {"prefill": base, "decode": dec}
    bufs = {"prefill": Buffers(4, 24, data["total_pages"], cuda), "decode": Buffers(4, 4, data["total_pages"], cuda)}
    matched = errors = 0
    for step in data["steps"]:
        if step["op"] == "add":
            base.add_request(step["rid"])
            continue
        if step["op"] == "remove":
            base.remove_request(step["rid"])
            continue
        kind = step["op"]
        pl, b = planners[kind], bufs[kind]
        free_before = base.free_pages()
        pl.set_rows([base.slot(r) for r in step["rows"]], step["advances"])
        pl.status.zero_()
        pl.plan_into(qo_indptr=b.qo_indptr, kv_indptr=b.kv_indptr, kv_indices=b.kv_indices,
                     last_page_len=b.last_page_len, position_ids=b.position_ids, write_pages=b.write_pages,
                     write_offsets=b.write_offsets, prefill=kind == "prefill")
        torch.cuda.synchronize()
        status = int(pl.status.item())
        if "error" in step:
            # KVAllocationError -> pool exhausted; ValueError -> tokens exceed the capture.  Either way
            # the device reserves nothing and flags the step.
            assert status & (0x4 | 0x20), step
            assert base.free_pages() == free_before
            assert int(pl.pending[0, 0]) == -1
            errors += 1
            continue
        assert status == 0, step
        n = len(step["paged_kv_indices"])
        got = {
            "paged_kv_indptr": b.kv_indptr.tolist(),
            "paged_kv_indices": b.kv_indices[:n].tolist(),
            "paged_kv_last_page_len": b.last_page_len.tolist(),
            "position_ids": b.position_ids.tolist(),
            "write_pages": b.write_pages.tolist(),
            "write_offsets": b.write_offsets.tolist(),
        }
        if kind == "prefill":
            got["qo_indptr"] = b.qo_indptr.tolist()
        for key, value in got.items():
            assert value == step[key], (key, step)
        publish = torch.zeros(4, dtype=torch.int32)
        publish[: len(step["publish"])] = torch.tensor([int(x) for x in step["publish"]], dtype=torch.int32)
        pl.commit(publish.to(cuda))
        matched += 1
    torch.cuda.synchronize()
    assert matched >= 30 and errors > 0
    for rid, state in data["final"].items():
        pages, length, _ = base.request_state(rid)
        assert list(pages) == state["pages"] and length == state["length"]
    assert base.free_pages() == data["free_pages"]


def test_device_planner_large_pool_decode_growth(nqt, cuda):
    # 64 rows over a 32768-page pool, 40 decode steps: matches the host oracle step by step
    from oracle import planner as oplan

    total, P, rows = 32768, 16, 64
    pl = nqt.DevicePagePlanner(total_pages=total, page_size=P, slots=rows, max_pages_per_slot=256,
                               scratch_page_count=rows, capture_rows=rows, token_capacity=rows, device=cuda)
    host = oplan.HostPagePool(total, P, rows)
    g = torch.Generator().manual_seed(1)
    lens = torch.randint(1, 200, (rows,), generator=g).tolist()
    slots = [pl.add_request(f"r{i}") for i in range(rows)]
    for i in range(rows):
        host.add_request(f"r{i}")
    # prefill everyone through the host oracle's allocation order, mirrored on the device by import
    for i, n in enumerate(lens):
        new = host.reserve([f"r{i}"], [n])[0]
        host.publish(f"r{i}")
        pl.import_pages(slots[i], torch.tensor(new), n)
    b = Buffers(rows, rows, total, cuda)
    pl.set_rows(slots, [1] * rows)
    for _ in range(40):
        meta = host.metadata([f"r{i}" for i in range(rows)], [1] * rows, rows, rows, False)
        pl.plan_into(qo_indptr=b.qo_indptr, kv_indptr=b.kv_indptr, kv_indices=b.kv_indices,
                     last_page_len=b.last_page_len, position_ids=b.position_ids, write_pages=b.write_pages,
                     write_offsets=b.write_offsets, prefill=False)
        pl.commit(True)
        for i in range(rows):
            host.publish(f"r{i}")
        assert b.kv_indptr.tolist() == meta["paged_kv_indptr"]
        assert b.kv_indices[: len(meta["paged_kv_indices"])].tolist() == meta["paged_kv_indices"]
        assert b.write_pages.tolist() == meta["write_pages"]
        assert b.write_offsets.tolist() == meta["write_offsets"]
        assert b.position_ids.tolist() == meta["position_ids"]
    assert int(pl.status.item()) == 0
    assert pl.free_pages() == len(host.free)


def test_device_planner_exhaustion_reserves_nothing(nqt, cuda):
    # tests/model_optimization/test_staging_cache_rng.py:102-117 on the device
    pl = nqt.DevicePagePlanner(total_pages=8, page_size=4, slots=4, max_pages_per_slot=8, scratch_page_count=2,
                               capture_rows=2, token_capacity=8, device=cuda)
    a, b = pl.add_request("a"), pl.add_request("b")
    buf = Buffers(2, 8, 8, cuda)

    def plan(advances):
        pl.set_rows([a, b], advances)
        pl.plan_into(qo_indptr=buf.qo_indptr, kv_indptr=buf.kv_indptr, kv_indices=buf.kv_indices,
                     last_page_len=buf.last_page_len, position_ids=buf.position_ids, write_pages=buf.write_pages,
                     write_offsets=buf.write_offsets, prefill=True)

    plan([4, 4])  # 1 + 1 pages
    pl.commit(True)
    plan([4, 4])  # 2 + 2 pages total, 2 free left
    pl.commit(True)
    assert pl.free_pages() == 2
    plan([5, 3])  # a needs +2, b needs +1: 3 > 2 free
    pl.commit(True)  # rows the plan did not reserve are skipped
    with pytest.raises(nqt.KVAllocationError):
        pl.check()
    assert pl.free_pages() == 2
    assert pl.request_state("a")[1] == 8 and pl.request_state("b")[1] == 8
    # the failed step's metadata puts every row on its scratch page
    assert buf.kv_indices[:2].tolist() == [0, 1] and buf.last_page_len.tolist() == [1, 1]
    assert buf.qo_indptr.tolist() == [0, 0, 0]
    # a second commit of a consumed plan changes nothing
    plan([1, 1])
    pl.commit(True)
    pl.commit(True)
    assert pl.request_state("a")[1] == 9 and pl.request_state("b")[1] == 9
    assert int(pl.status.item()) == 0


def test_mixed_step_churn_keeps_the_pool_stationary(nqt, cuda):
    # config-4 mechanics at toy size: prefill chunks + decode rows + device-side request replacement
    from importlib import import_module

    ts = import_module("nari-qwen3-tts_b200.talker_step")
    shape = ts.TalkerShape(num_layers=2, hidden=256, ffn=512, vocab=512, codec_vocab=384, eos_id=400)
    ctx = torch.randint(32, 400, (16,), generator=torch.Generator().manual_seed(4)).tolist()
    step = ts.TalkerMixedStep(shape=shape, chunks=[100, 37, 5], decode_contexts=ctx, churn_rows=4,
                              total_pages=2048, page_size=16, device=cuda, seed=0)
    step.admit(scatter_seed=1)
    free0 = step.dec.free_pages()
    slot_of = {f"decode{i}": step.dec.slot(f"decode{i}") for i in range(16)}
    for i in range(6):
        step.forward()
        torch.cuda.synchronize()
        assert int(step.dec.status.item()) == 0 and nqt.kernels.read_status(cuda) == 0
        assert step.dec.free_pages() == free0
    for i, n in enumerate(ctx):  # replaced requests come back at the same length
        pages, length, _ = step.dec.request_state(f"decode{i}")
        assert length == n and len(pages) == (n + 15) // 16
    assert torch.isfinite(step._x.float()).all()
    assert set(slot_of.values()) == {step.dec.slot(f"decode{i}") for i in range(16)}
