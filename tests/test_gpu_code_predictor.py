"""GPU: one code-predictor frame (executor/code_predictor.py:160-235) on the
sm_100a kernels against the CPU port (oracle/code_predictor.py).

Sampling is discontinuous, so the frame is checked in two halves:
* teacher-forced: the CPU port replays the GPU frame's codes and its
  per-group logits must match the GPU's within a bf16 tolerance, and the
  codec embedding sum (bf16 gathers + adds) bit-exactly;
* sampling: each GPU code is the fused sampler's draw on the GPU logits of
  its group (a replay of the same draw) and lies inside the reference's
  filtered top-k support of those logits.
"""

from __future__ import annotations

import importlib

import pytest
import torch

from oracle import sampler as osamp
from oracle.code_predictor import CpuCodePredictorFrame

pytestmark = pytest.mark.gpu

ROWS = 8


@pytest.fixture(scope="module")
def frame(nqt, cuda):
    cp = importlib.import_module("nari-qwen3-tts_b200.code_predictor")
    f = cp.CodePredictorFrame(rows=ROWS, device=cuda, seed=3)
    g = torch.Generator(device=cuda).manual_seed(5)
    f.past_hidden.copy_(torch.randn(ROWS, f.shape.talker_hidden, generator=g, device=cuda))
    f.layer0_token.copy_(torch.randint(0, f.shape.vocab, (ROWS,), generator=g, device=cuda))
    f.set_frame(7)
    codes = f.forward().clone()
    torch.cuda.synchronize()
    assert nqt.kernels.read_status(cuda) == 0
    return f, codes


def test_teacher_forced_logits_and_codec_sum_match_the_cpu_port(frame):
    f, codes = frame
    port = CpuCodePredictorFrame(f.cpu_weights(), heads=f.shape.num_heads, kv_heads=f.shape.num_kv_heads,
                                 head_dim=f.shape.head_dim, groups=f.shape.groups, eps=f.shape.eps,
                                 theta=f.shape.rope_theta)
    frames, logits, codec_sum = port.frame(
        f.past_hidden.cpu(), f.layer0_token.cpu(), temperature=f.temperature.cpu(), top_k=f.top_k.cpu(),
        top_p=f.top_p.cpu(), seed=f.seed.cpu(), offsets=f.offsets.cpu(), forced_tokens=codes.cpu())
    assert torch.equal(frames, codes.cpu())
    gpu = f.logits.float().cpu()
    err = (gpu - logits).abs()
    scale = logits.abs().max().item()
    # bf16 activations through 5 layers x 16 depth steps: GEMM accumulation order differs (cuBLAS vs CPU),
    # so logits agree to a few bf16 ulps of their magnitude, not bit-exactly
    assert err.max().item() <= 0.05 * max(scale, 1.0), (err.max().item(), scale)
    assert err.mean().item() <= 0.01 * max(scale, 1.0), (err.mean().item(), scale)
    assert torch.equal(f.codec_sum.cpu(), codec_sum.to(torch.bfloat16))


def test_codes_are_the_fused_sampler_draws_inside_the_filtered_support(nqt, frame):
    f, codes = frame
    for group in range(1, f.shape.groups):
        logits = f.logits[group - 1]
        redraw = nqt.sample_rows(logits, f.temperature, f.top_k, f.top_p, f.seed, f.offsets[:, group - 1],
                                 round_scaled_to_input=False)
        assert torch.equal(redraw, codes[:, group]), group
        host = logits.float().cpu()
        for row in range(ROWS):
            scaled = host[row] / float(f.temperature[row])
            probs, ids = osamp.filtered_probs(scaled, int(f.top_k[row]), float(f.top_p[row]))
            support = set(ids[probs > 0].tolist())
            assert int(codes[row, group]) in support, (group, row)


def test_graph_replay_and_host_step_reproduce_the_eager_frame(frame):
    f, codes = frame
    f.capture(warmup=1)
    f.replay()
    torch.cuda.synchronize()
    assert torch.equal(f.frames, codes)
    host = f.step(f.past_hidden.cpu(), f.layer0_token.cpu())
    assert torch.equal(host, codes.cpu())
    # another frame index draws with other offsets (row-local Philox streams move)
    f.set_frame(8)
    f.replay()
    torch.cuda.synchronize()
    assert not torch.equal(f.frames, codes)
    assert torch.equal(f.frames[:, 0], codes[:, 0])
