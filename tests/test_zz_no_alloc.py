"""GPU: nqt_decode_attention_noalloc, the decode entry point that allocates
nothing, against nqt_decode_attention with a caller workspace.

It exists for callers that cannot allocate device memory (their device
memory belongs to another runtime's allocator, or they may only pass
pointers to buffers they already hold); its scratch is a fixed array inside
libnqt.  This file is collected last so that a run stopping at the first
failure has run every other test first; it also passes alone in a fresh
process.  Two calls in a row on different inputs check that the shared
scratch left by one call does not leak into the next."""

from __future__ import annotations

import pytest
import torch

from tests._paged import make_paged

pytestmark = pytest.mark.gpu


def _noalloc(lib_mod, q, cache, indptr, indices, last, out, status):
    rows, hq, d = q.shape
    lib_mod.call(
        "nqt_decode_attention_noalloc",
        q.data_ptr(), q.stride(0), q.stride(1),
        cache.data_ptr(), cache.shape[0], cache.shape[2],
        indptr.data_ptr(), indices.data_ptr(), last.data_ptr(),
        rows, hq, cache.shape[3], d, d ** -0.5,
        out.data_ptr(), out.stride(0), out.stride(1),
        status.data_ptr(), lib_mod.stream_handle(q.device),
    )


def test_noalloc_decode_matches_workspace_decode_twice(nqt, cuda):
    from importlib import import_module

    lib_mod = import_module("nari-qwen3-tts_b200._lib")
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    cases = [
        ([int(x) for x in torch.randint(16, 513, (8,), generator=torch.Generator().manual_seed(0))], 0),
        (torch.randint(64, 2049, (64,), generator=torch.Generator().manual_seed(1)).tolist(), 1),
    ]
    for lens, seed in cases:  # two calls in a row, different shapes and data
        cache, indptr, indices, last = make_paged(lens, seed=seed)
        cache, indptr, indices, last = cache.to(cuda), indptr.to(cuda), indices.to(cuda), last.to(cuda)
        q = torch.randn(len(lens), 16, 128, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16).to(cuda)
        ws = torch.zeros(nqt.lib().nqt_decode_workspace_bytes(len(lens), 16, 128), dtype=torch.uint8, device=cuda)
        want = nqt.batch_decode_paged(q, cache, indptr, indices, last, ws)
        got = torch.full_like(want, float("nan"))
        _noalloc(lib_mod, q, cache, indptr, indices, last, got, status)
        torch.cuda.synchronize()
        # same kernels and the same split (both cap the split CTAs above the 2-per-SM grid), and the split
        # partials are combined in a fixed order: the outputs are identical, well inside the 2e-2 tolerance
        assert torch.equal(got, want)
        assert int(status.item()) == 0
    assert nqt.lib().nqt_decode_noalloc_scratch_bytes() < 8 * 1024 * 1024


def test_noalloc_rejects_shapes_beyond_its_scratch(nqt, cuda):
    from importlib import import_module

    lib_mod = import_module("nari-qwen3-tts_b200._lib")
    cache, indptr, indices, last = make_paged([16] * 4, seed=3)
    cache, indptr, indices, last = cache.to(cuda), indptr.to(cuda), indices.to(cuda), last.to(cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    q = torch.zeros(2000, 16, 128, dtype=torch.bfloat16, device=cuda)  # more rows than the scratch holds
    out = torch.zeros_like(q)
    with pytest.raises(lib_mod.NqtError, match="capacity"):
        _noalloc(lib_mod, q, cache, indptr, indices, last, out, status)
