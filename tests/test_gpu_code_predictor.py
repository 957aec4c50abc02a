"""GPU: one code-predictor frame (executor/code_predictor.py:160-235) on the
sm_100a kernels against the CPU port (oracle/code_predictor.py).

Sampling is discontinuous, so the frame is checked in parts:
* per layer, teacher-forced: the CPU port runs each decoder layer of every
  depth step from the GPU's own residual stream and frame cache; the residual
  after the layer must agree within 2e-2 + 2^-6 (|x| + max |x|) (mean within
  half a bf16 ulp of the mean magnitude), the K / V row it wrote within the
  same element bound (mean within one ulp of the mean magnitude), the step's
  final norm within one bf16 rounding (1e-2 + 2^-7 |x|, mean within half an
  ulp of the mean magnitude) and the group's logits within one bf16 rounding
  (1e-2 + 2^-7 |x|, mean <= 1e-3);
* whole frame: the CPU port replays the GPU frame's codes and its per-group
  logits stay within a few bf16 ulps of their magnitude after 16 chained depth
  steps, and the codec embedding sum (bf16 gathers + adds) is bit-exact;
* sampling: each GPU code is the fused sampler's draw on the GPU logits of
  its group (a replay of the same draw) and lies inside the reference's
  filtered top-k support of those logits;
* the fused glue between depth steps (nqt_cp_codec_step) equals the six ops
  it replaces bit for bit.
"""

from __future__ import annotations

import importlib

import pytest
import torch
import torch.nn.functional as F

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
    trace: list = []
    codes = f.forward(trace).clone()
    torch.cuda.synchronize()
    assert nqt.kernels.read_status(cuda) == 0
    return f, codes, trace


def _close(bad, got, want, atol, rtol, mean_tol, what):
    """Append to ``bad`` each bound that ``got`` breaks (all are reported at the end of the test)."""
    err = (got - want).abs()
    worst = float((err - (atol + rtol * want.abs())).max())
    if worst > 0:
        bad.append(f"{what}: max |err| {float(err.max()):.3e} exceeds the bound by {worst:.3e}")
    if float(err.mean()) > mean_tol:
        bad.append(f"{what}: mean |err| {float(err.mean()):.3e} over mean |x| {float(want.abs().mean()):.3e}")


def test_depth_layers_teacher_forced_match_the_cpu_port(frame):
    f, codes, trace = frame
    s = f.shape
    port = CpuCodePredictorFrame(f.cpu_weights(), heads=s.num_heads, kv_heads=s.num_kv_heads, head_dim=s.head_dim,
                                 groups=s.groups, eps=s.eps, theta=s.rope_theta)
    lm_head = f.lm_head.float().cpu()
    ln_final = f.ln_final.float().cpu()
    bad: list[str] = []
    for pos, (residuals, cache, hidden) in enumerate(trace):
        cache = cache.cpu()
        after = trace[pos + 1][1].cpu() if pos + 1 < len(trace) else f.kv_cache.cpu()
        for layer in range(s.num_layers):
            cache_list = [(cache[i, :, 0].clone(), cache[i, :, 1].clone()) for i in range(s.num_layers)]
            x_in = residuals[layer].float().cpu()
            want = port.depth_layer(x_in, layer, cache_list, pos)
            # every bf16 intermediate (o, the residual sums, m) rounds on either side of a boundary when the
            # two GEMM accumulation orders differ, so about half the elements move by one bf16 ulp
            # (~2^-7 |x|): the mean bound is half an ulp of the mean magnitude; an intermediate larger than
            # the residual element it feeds (the MLP or attention output before the add) rounds at its own
            # ulp, so the element bound carries one ulp of the largest magnitude as well
            got_r = residuals[layer + 1].float().cpu()
            _close(bad, got_r, want, 2e-2 + 2.0**-6 * float(want.abs().max()), 2.0**-6,
                   2.0**-10 + 2.0**-8 * float(want.abs().mean()), f"position {pos} layer {layer}")
            for kind in range(2):  # the K / V row this layer wrote (a GEMM, a norm and RoPE from its input)
                # the GPU normalises the fp32 residual sum, the port the rounded one: a one-ulp input
                # difference carries through the projection, so the mean bound is one ulp of the mean magnitude
                want_kv = cache_list[layer][kind][:, pos].float()
                _close(bad, after[layer, :, kind, pos].float(), want_kv,
                       2e-2 + 2.0**-6 * float(want_kv.abs().max()), 2.0**-6,
                       2.0**-10 + 2.0**-7 * float(want_kv.abs().mean()), f"position {pos} layer {layer} cache write")
        if hidden is None:
            continue
        final = residuals[-1].float().cpu()
        want_h = (final * torch.rsqrt(final.pow(2).mean(-1, keepdim=True) + s.eps) * ln_final).to(torch.bfloat16)
        got = hidden.float().cpu()
        # the GPU's fused add + norm normalises the fp32 sum, the check the rounded residual: half an ulp of
        # the mean magnitude on average
        _close(bad, got, want_h.float(), 1e-2, 2.0**-7, 2.0**-10 + 2.0**-8 * float(want_h.float().abs().mean()),
               f"depth step {pos} final norm")
        want_logits = (got @ lm_head[pos - 1].T).to(torch.bfloat16).float()
        _close(bad, f.logits[pos - 1].float().cpu(), want_logits, 1e-2, 2.0**-7, 1e-3, f"group {pos} logits")
    assert not bad, f"{len(bad)} bounds broken:\n" + "\n".join(bad[:12])


def test_frame_logits_and_codec_sum_match_the_cpu_port(frame):
    f, codes, _ = frame
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
    f, codes, _ = frame
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
            # torch.topk leaves the order of tied values unspecified: a cut through a tie group may keep a
            # different member of it
            vmin = min(float(scaled[t]) for t in support)
            support |= set((scaled == vmin).nonzero().flatten().tolist())
            assert int(codes[row, group]) in support, (group, row)


def test_graph_replay_and_host_step_reproduce_the_eager_frame(frame):
    f, codes, _ = frame
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


@pytest.mark.parametrize("accumulate,with_next", [(True, True), (False, True), (True, False)])
def test_codec_step_equals_the_unfused_ops(nqt, cuda, accumulate, with_next):
    """nqt_cp_codec_step against the six ops it replaces: the frame's code column, the codec embedding sum
    (bf16 add), the next step's input and its rmsnorm - all bit for bit."""

    g = torch.Generator(device=cuda).manual_seed(11)
    rows, vocab, th, hd = 37, 2048, 2048, 1024
    tokens = torch.randint(0, vocab, (rows,), generator=g, device=cuda)
    emb = (0.5 * torch.randn(vocab, th, generator=g, device=cuda)).to(torch.bfloat16)
    proj = torch.randn(vocab, hd, generator=g, device=cuda).to(torch.bfloat16)
    ln = (1 + 0.1 * torch.randn(hd, generator=g, device=cuda)).to(torch.bfloat16)
    sum0 = torch.randn(rows, th, generator=g, device=cuda).to(torch.bfloat16)
    frames = torch.zeros(rows, 16, dtype=torch.long, device=cuda)
    codec_sum, res, h = sum0.clone(), torch.zeros(rows, hd, dtype=torch.bfloat16, device=cuda), \
        torch.zeros(rows, hd, dtype=torch.bfloat16, device=cuda)
    nqt.kernels.cp_codec_step(tokens, frames[:, 5], emb, codec_sum, accumulate=accumulate,
                              proj_emb=proj if with_next else None, ln=ln, eps=1e-6, residual=res, h=h)
    torch.cuda.synchronize()
    assert torch.equal(frames[:, 5], tokens) and int(frames[:, :5].abs().sum()) == 0
    want_sum = sum0 + F.embedding(tokens, emb) if accumulate else F.embedding(tokens, emb)
    assert torch.equal(codec_sum, want_sum)
    if with_next:
        x = F.embedding(tokens, proj)
        assert torch.equal(res, x)
        assert torch.equal(h, nqt.kernels.rmsnorm(x, ln, 1e-6))
    # an id outside the vocabulary: status bit, the row left as it was
    nqt.kernels.clear_status(cuda)
    bad = tokens.clone()
    bad[3] = vocab
    before = codec_sum.clone()
    nqt.kernels.cp_codec_step(bad, frames[:, 6], emb, codec_sum, proj_emb=None)
    torch.cuda.synchronize()
    assert nqt.kernels.read_status(cuda) & nqt._lib.NQT_DEV_BAD_TOKEN
    assert torch.equal(codec_sum[3], before[3])
    nqt.kernels.clear_status(cuda)
