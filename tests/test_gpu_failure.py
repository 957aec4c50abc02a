"""GPU failure path without a fault: a decode launch whose bounded waits give
up (the test-only NQT_DECODE_SHORT_WAIT flag makes every pipeline wait give
up at once) must report NQT_DEV_TIMEOUT, exit cleanly, and leave the plan's
split-KV fix-up state settled so the next launches on the same plan match the
oracle.  Nothing here traps, faults or hangs: the short waits end by
themselves and the launch still waits for its own copies before exiting."""

from __future__ import annotations

import pytest
import torch

from oracle import attention as oatt
from tests._paged import make_paged

pytestmark = pytest.mark.gpu

ATOL = 2e-2


def test_decode_timeout_leaves_plan_usable(nqt, cuda):
    # long ragged rows: far more 16-token tiles than split CTAs, so most rows are split
    lens = torch.randint(300, 3000, (24,), generator=torch.Generator().manual_seed(11)).tolist()
    cache, indptr, indices, last = make_paged(lens, seed=11)
    rows, hq, d = len(lens), 16, 128
    q = torch.randn(rows, hq, d, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    dev = dict(cache=cache.to(cuda), indptr=indptr.to(cuda), indices=indices.to(cuda), last=last.to(cuda))
    ws = torch.zeros(nqt.lib().nqt_decode_workspace_bytes(rows, hq, d), dtype=torch.uint8, device=cuda)
    want = oatt.paged_decode(q.float(), cache.float(), indptr, indices, last)
    qd = q.to(cuda)

    def run(*, plan, short_wait=False):
        return nqt.batch_decode_paged(qd, dev["cache"], dev["indptr"], dev["indices"], dev["last"], ws, plan=plan,
                                      short_wait=short_wait)

    nqt.kernels.clear_status(cuda)
    torch.testing.assert_close(run(plan=True).float().cpu(), want, atol=ATOL, rtol=0)
    assert nqt.kernels.read_status(cuda) == 0
    # one launch gives up on its waits
    run(plan=False, short_wait=True)
    torch.cuda.synchronize()
    assert nqt.kernels.read_status(cuda) & nqt._lib.NQT_DEV_TIMEOUT
    nqt.kernels.clear_status(cuda)
    # the next launches on the same plan are correct and report nothing
    for _ in range(2):
        torch.testing.assert_close(run(plan=False).float().cpu(), want, atol=ATOL, rtol=0)
        assert nqt.kernels.read_status(cuda) == 0


def test_decode_timeouts_in_a_row(nqt, cuda):
    # enough tiles per CTA that some copy is still in flight when its short wait gives up
    lens = [5000, 17, 1200, 2047, 64] + torch.randint(1000, 4000, (19,), generator=torch.Generator().manual_seed(15)).tolist()
    cache, indptr, indices, last = make_paged(lens, seed=13)
    rows, hq, d = len(lens), 16, 128
    q = torch.randn(rows, hq, d, generator=torch.Generator().manual_seed(14)).to(torch.bfloat16)
    ws = torch.zeros(nqt.lib().nqt_decode_workspace_bytes(rows, hq, d), dtype=torch.uint8, device=cuda)
    args = (q.to(cuda), cache.to(cuda), indptr.to(cuda), indices.to(cuda), last.to(cuda), ws)
    nqt.batch_decode_paged(*args, plan=True, short_wait=True)
    for _ in range(3):
        nqt.batch_decode_paged(*args, plan=False, short_wait=True)
    torch.cuda.synchronize()
    assert nqt.kernels.read_status(cuda) & nqt._lib.NQT_DEV_TIMEOUT
    nqt.kernels.clear_status(cuda)
    want = oatt.paged_decode(q.float(), cache.float(), indptr, indices, last)
    torch.testing.assert_close(nqt.batch_decode_paged(*args, plan=False).float().cpu(), want, atol=ATOL, rtol=0)
    assert nqt.kernels.read_status(cuda) == 0
