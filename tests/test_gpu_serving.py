"""GPU: the config-5 serving worker at toy depth (2 talker layers): every
admitted request is prefilled, decoded and retired by the device completion
rule after exactly its audio frame count, the page pool returns to its
starting occupancy, and time-to-first-frame is measured for each request."""

from __future__ import annotations

from importlib import import_module

import pytest
import torch

@pytest.mark.gpu
def test_worker_serves_every_request_its_frames(nqt, cuda):
    serving = import_module("nari-qwen3-tts_b200.serving")
    ts = import_module("nari-qwen3-tts_b200.talker_step")
    worker = serving.ServingWorker(shape=ts.TalkerShape(num_layers=2), slots=16, pool_tokens=16 * 1024,
                                   prefill_tokens=256, device=cuda, seed=1)
    worker.capture()
    free0 = worker.step.planner.free_pages()
    requests = serving.poisson_requests(rate=40.0, horizon=0.5, seed=3, audio_seconds=(0.5, 2.0))
    assert requests, "the arrival stream is empty"
    rep = worker.run(requests, horizon=0.5)
    torch.cuda.synchronize()
    assert rep.admitted == rep.finished == len(requests)
    assert all(r.emitted == r.frames for r in requests)
    assert rep.frames == sum(r.frames for r in requests)
    assert len(rep.ttff) == len(requests) and min(rep.ttff) > 0
    assert all(r.first_frame >= r.arrival and r.done >= r.first_frame for r in requests)
    assert worker.step.planner.free_pages() == free0
    assert nqt.kernels.read_status(cuda) == 0 and int(worker.step.planner.status.item()) == 0


def test_round_robin_router_partitions_the_arrival_stream():
    serving = import_module("nari-qwen3-tts_b200.serving")
    everything = serving.poisson_requests(rate=20.0 * 4, horizon=5.0, seed=9)
    parts = [serving.poisson_requests(rate=20.0, horizon=5.0, seed=9, rank=r, world=4) for r in range(4)]
    ids = sorted(r.rid for p in parts for r in p)
    assert ids == [r.rid for r in everything]
    for p in parts:
        assert all(0 < r.frames <= 240 and 20 <= r.text_tokens <= 200 for r in p)
