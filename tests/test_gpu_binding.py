"""GPU: the TalkerAttentionContext drop-in (plan / select_layer / attend) with
host metadata from the oracle's builder and with device metadata from the
GPU planner, eagerly and replayed from a CUDA graph."""

from __future__ import annotations

import pytest
import torch

from oracle import attention as oatt
from oracle import planner as oplan
from tests._paged import FakeAttention

pytestmark = pytest.mark.gpu


def _binding(nqt, cuda, storage, rows, tokens):
    return nqt.binding_factory(storage=storage, capture_batch_size=rows, token_capacity=tokens, num_qo_heads=16,
                               num_kv_heads=8, head_dim=128, page_size=16, total_pages=storage.shape[1],
                               workspace=torch.empty(16, dtype=torch.uint8, device=cuda), shared_plan_state=None,
                               device=cuda, dtype=torch.bfloat16, slot=0, metadata=None)


def _meta(nqt, m, prefill):
    def t(x, dt):
        return torch.tensor(x, dtype=dt).pin_memory()

    return nqt.TalkerAttentionMetadata(
        qo_indptr=t(m["qo_indptr"], torch.int32) if prefill else None,
        paged_kv_indptr=t(m["paged_kv_indptr"], torch.int32),
        paged_kv_indices=t(m["paged_kv_indices"], torch.int32),
        paged_kv_last_page_len=t(m["paged_kv_last_page_len"], torch.int32),
        position_ids=t(m["position_ids"], torch.long),
        write_pages=t(m["write_pages"], torch.long),
        write_offsets=t(m["write_offsets"], torch.long),
        padding_pages=(),
    )


def _oracle_attend(cache, m, q, k, v, attn, prefill):
    q, k = q.clone(), k.clone()
    oatt.qk_norm_rope_paged_(q, k, v, attn.q_norm.weight.cpu(), attn.k_norm.weight.cpu(),
                             torch.tensor(m["position_ids"]), 1e-6, 1e6, cache, torch.tensor(m["write_pages"]),
                             torch.tensor(m["write_offsets"]))
    indptr = torch.tensor(m["paged_kv_indptr"])
    indices = torch.tensor(m["paged_kv_indices"])
    last = torch.tensor(m["paged_kv_last_page_len"])
    if prefill:
        return oatt.paged_prefill(q.float(), cache.float(), torch.tensor(m["qo_indptr"]), indptr, indices, last)
    return oatt.paged_decode(q.float(), cache.float(), indptr, indices, last)


def test_binding_prefill_then_decode_with_graph_replay(nqt, cuda):
    layers, pages, P = 2, 64, 16
    g = torch.Generator().manual_seed(0)
    storage_cpu = torch.zeros(layers, pages, 2, P, 8, 128, dtype=torch.bfloat16)
    storage = storage_cpu.to(cuda)
    attn = FakeAttention((1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).to(cuda),
                         (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).to(cuda))
    pool = oplan.HostPagePool(pages, P, 12)
    for r in ("a", "b", "c"):
        pool.add_request(r)
    # prefill 3 rows (capture 4 rows / 160 tokens)
    m = pool.metadata(["a", "b", "c"], [40, 7, 100], 4, 160, True)
    pre = _binding(nqt, cuda, storage, 4, 160)
    pre.plan(_meta(nqt, m, True))
    for layer in range(layers):
        qkv = torch.randn(160, 32 * 128, generator=g).to(torch.bfloat16)
        q, k, v = qkv[:, :2048].view(160, 16, 128), qkv[:, 2048:3072].view(160, 8, 128), qkv[:, 3072:].view(160, 8, 128)
        want = _oracle_attend(storage_cpu[layer], m, q, k, v, attn, True)
        pre.select_layer(layer)
        qd = qkv.to(cuda)
        got = pre.attend(attn, qd[:, :2048].view(160, 16, 128), qd[:, 2048:3072].view(160, 8, 128),
                         qd[:, 3072:].view(160, 8, 128))
        torch.testing.assert_close(got[:147].float().cpu(), want[:147], atol=2e-2, rtol=0)
    for r in ("a", "b", "c"):
        pool.publish(r)
    torch.testing.assert_close(storage.cpu().float(), storage_cpu.float(), atol=2.0 ** -7, rtol=2.0 ** -7)
    storage_cpu.copy_(storage.cpu())

    # decode: capture attend for layer 0 once, replay with fresh metadata each step
    dec = _binding(nqt, cuda, storage, 4, 4)
    q_static = torch.zeros(4, 32 * 128, dtype=torch.bfloat16, device=cuda)
    steps = []
    for _ in range(3):
        m = pool.metadata(["a", "b", "c"], [1, 1, 1], 4, 4, False)
        steps.append(m)
        for r in ("a", "b", "c"):
            pool.publish(r)
    dec.plan(_meta(nqt, steps[0], False))
    dec.select_layer(0)

    def step():
        return dec.attend(attn, q_static[:, :2048].view(4, 16, 128), q_static[:, 2048:3072].view(4, 8, 128),
                          q_static[:, 3072:].view(4, 8, 128))

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()  # warm-up (writes the step-0 token; redone below on replay)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    for m in steps:
        qkv = torch.randn(4, 32 * 128, generator=g).to(torch.bfloat16)
        q, k, v = qkv[:, :2048].view(4, 16, 128), qkv[:, 2048:3072].view(4, 8, 128), qkv[:, 3072:].view(4, 8, 128)
        want = _oracle_attend(storage_cpu[0], m, q, k, v, attn, False)
        dec.plan(_meta(nqt, m, False))
        q_static.copy_(qkv.to(cuda))
        graph.replay()
        torch.testing.assert_close(out[:3].float().cpu(), want[:3], atol=2e-2, rtol=0)
    assert nqt.kernels.read_status(cuda) == 0


def test_binding_rejects_oversized_metadata(nqt, cuda):
    storage = torch.zeros(1, 8, 2, 16, 8, 128, dtype=torch.bfloat16, device=cuda)
    b = _binding(nqt, cuda, storage, 2, 2)
    m = nqt.TalkerAttentionMetadata(
        qo_indptr=None, paged_kv_indptr=torch.zeros(3, dtype=torch.int32),
        paged_kv_indices=torch.zeros(20, dtype=torch.int32), paged_kv_last_page_len=torch.ones(2, dtype=torch.int32),
        position_ids=torch.zeros(2, dtype=torch.long), write_pages=torch.zeros(2, dtype=torch.long),
        write_offsets=torch.zeros(2, dtype=torch.long), padding_pages=())
    with pytest.raises(ValueError, match="exceeds its captured buffer"):
        b.plan(m)
    with pytest.raises(IndexError):
        b.select_layer(1)


def _empty_meta(nqt, rows, prefill):
    return nqt.TalkerAttentionMetadata(
        qo_indptr=torch.zeros(rows + 1, dtype=torch.int32) if prefill else None,
        paged_kv_indptr=torch.arange(rows + 1, dtype=torch.int32),
        paged_kv_indices=torch.arange(rows, dtype=torch.int32),
        paged_kv_last_page_len=torch.ones(rows, dtype=torch.int32),
        position_ids=torch.zeros(rows, dtype=torch.long), write_pages=torch.arange(rows, dtype=torch.long),
        write_offsets=torch.zeros(rows, dtype=torch.long), padding_pages=())


def test_binding_kind_is_fixed_by_its_first_plan(nqt, cuda):
    """The reference decode binding rejects packed query metadata and the
    prefill binding requires it (executor/talker_kv.py:176-177, 260-261)."""

    storage = torch.zeros(1, 8, 2, 16, 8, 128, dtype=torch.bfloat16, device=cuda)
    dec = _binding(nqt, cuda, storage, 2, 2)
    dec.plan(_empty_meta(nqt, 2, False))
    with pytest.raises(ValueError, match="Talker decode cannot contain packed query metadata"):
        dec.plan(_empty_meta(nqt, 2, True))
    pre = _binding(nqt, cuda, storage, 2, 2)
    pre.plan(_empty_meta(nqt, 2, True))
    with pytest.raises(ValueError, match="Talker prefill requires packed query metadata"):
        pre.plan(_empty_meta(nqt, 2, False))
    fixed = nqt.B200TalkerBinding(storage=storage, capture_batch_size=2, token_capacity=2, num_qo_heads=16,
                                  num_kv_heads=8, head_dim=128, page_size=16, total_pages=8, device=cuda,
                                  dtype=torch.bfloat16, mode="prefill")
    with pytest.raises(ValueError, match="Talker prefill requires packed query metadata"):
        fixed.plan(_empty_meta(nqt, 2, False))


def test_bindings_share_the_slot_workspace(nqt, cuda):
    """Two decode bindings of one slot keep their split-KV plans in the slot's
    workspace (like the reference's per-slot FlashInfer workspace); planning
    before each run keeps both correct."""

    g = torch.Generator().manual_seed(5)
    pages, P = 96, 16
    storage_cpu = torch.randn(1, pages, 2, P, 8, 128, generator=g).to(torch.bfloat16)
    storage = storage_cpu.to(cuda)
    attn = FakeAttention(torch.ones(128, dtype=torch.bfloat16, device=cuda),
                         torch.ones(128, dtype=torch.bfloat16, device=cuda))
    workspace = torch.empty(64 << 20, dtype=torch.uint8, device=cuda)

    def make(rows):
        return nqt.binding_factory(storage=storage, capture_batch_size=rows, token_capacity=rows, num_qo_heads=16,
                                   num_kv_heads=8, head_dim=128, page_size=P, total_pages=pages, workspace=workspace,
                                   shared_plan_state=None, device=cuda, dtype=torch.bfloat16, slot=0, metadata=None)

    a, b = make(2), make(3)
    assert a.decode_workspace.data_ptr() == workspace.data_ptr() == b.decode_workspace.data_ptr()
    pool = oplan.HostPagePool(pages, P, 3)
    for r, n in (("x", 700), ("y", 33), ("z", 400)):
        pool.add_request(r)
        pool.reserve([r], [n])
        pool.publish(r)
    cases = ((a, ["x", "y"], 2), (b, ["x", "y", "z"], 3), (a, ["y", "z"], 2))
    for binding, rids, rows in cases:
        m = pool.metadata(rids, [1] * rows, rows, rows, False)
        binding.plan(_meta(nqt, m, False))
        binding.select_layer(0)
        qkv = torch.randn(rows, 32 * 128, generator=g).to(torch.bfloat16)
        q, k, v = qkv[:, :2048].view(rows, 16, 128), qkv[:, 2048:3072].view(rows, 8, 128), qkv[:, 3072:].view(rows, 8, 128)
        want = _oracle_attend(storage_cpu[0], m, q, k, v, attn, False)
        qd = qkv.to(cuda)
        got = binding.attend(attn, qd[:, :2048].view(rows, 16, 128), qd[:, 2048:3072].view(rows, 8, 128),
                             qd[:, 3072:].view(rows, 8, 128))
        torch.testing.assert_close(got.float().cpu(), want, atol=2e-2, rtol=0)
        for r in rids:
            pool.discard(r)
        storage_cpu.copy_(storage.cpu())
    assert nqt.kernels.read_status(cuda) == 0


def test_binding_replays_the_reference_paged_talker_kv(nqt, cuda, golden):
    """The calls the reference's own PagedTalkerKV makes on a custom binding
    (factory kwargs, then plan() with its prefill / decode / capture metadata;
    recorded by tests/golden/make_golden.py) replayed on B200TalkerBinding:
    every plan is accepted and every attend matches the oracle."""

    fx = golden("binding.pt")
    shape = fx["factories"][0]["storage_shape"]
    g = torch.Generator().manual_seed(8)
    storage_cpu = torch.randn(*shape, generator=g).to(torch.bfloat16)
    storage = storage_cpu.to(cuda)
    workspace = torch.empty(fx["factories"][0]["workspace_bytes"], dtype=torch.uint8, device=cuda)
    bindings = [nqt.binding_factory(storage=storage, workspace=workspace, shared_plan_state=object(), device=cuda,
                                    dtype=torch.bfloat16, **f["scalars"]) for f in fx["factories"]]
    attn = FakeAttention((1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).to(cuda),
                         (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16).to(cuda))
    for call in fx["calls"]:
        binding = bindings[call["binding"]]
        meta = nqt.TalkerAttentionMetadata(**{k: call[k] for k in call["fields"]})
        binding.plan(meta)
        prefill = meta.qo_indptr is not None
        m = {k: (v.tolist() if isinstance(v, torch.Tensor) else v) for k, v in call.items()}
        tokens = binding.token_capacity
        valid = m["qo_indptr"][-1] if prefill else tokens
        for layer in range(shape[0]):
            binding.select_layer(layer)
            qkv = torch.randn(tokens, 32 * 128, generator=g).to(torch.bfloat16)
            q, k, v = (qkv[:, :2048].view(tokens, 16, 128), qkv[:, 2048:3072].view(tokens, 8, 128),
                       qkv[:, 3072:].view(tokens, 8, 128))
            want = _oracle_attend(storage_cpu[layer], m, q, k, v, attn, prefill)
            qd = qkv.to(cuda)
            got = binding.attend(attn, qd[:, :2048].view(tokens, 16, 128), qd[:, 2048:3072].view(tokens, 8, 128),
                                 qd[:, 3072:].view(tokens, 8, 128))
            torch.testing.assert_close(got[:valid].float().cpu(), want[:valid], atol=2e-2, rtol=0)
        storage_cpu.copy_(storage.cpu())
    assert nqt.kernels.read_status(cuda) == 0
