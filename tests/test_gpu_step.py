"""GPU parity of the benchmarked compositions: one talker decode step
(TalkerDecodeStep, BASELINE config 2 widths) and one mixed prefill + decode
step (TalkerMixedStep, config 4 widths), each at 2 layers, against the CPU
oracle's restatement of the reference layer (oracle/talker_step.py).

The decode step runs with both gate/up paths: the reference's production FP8
path (the default; oracle/fp8.py restates its quantisation rules) and bf16.
On the FP8 path the oracle's MLP also starts from the GPU's e4m3 rows and
scales (its own quantisation of its MLP input must stay within one e4m3 step
plus 2e-2 of the GPU's after dequantisation, scales within 2^-7, >= 95 % of
the bytes equal), since one bf16 ulp at an e4m3 rounding boundary moves a
whole e4m3 step.

Teacher-forced: the oracle runs each layer from the GPU's own input to that
layer (the step's trace), so the check sees this layer's error only:
  * hidden state / residual after each layer: |err| <= 2e-2 + 2^-6 |want|
    and mean |err| <= 2e-3 (bf16 rounding at every module boundary plus the
    2e-2 attention tolerance);
  * logits of the codec head: |err| <= 1e-2 + 2^-7 |want| (one bf16 rounding), and the
    suppress mask of forward_logits (columns past the code-predictor vocabulary
    except EOS, and EOS on rows before step 2) exactly;
  * the K/V the step wrote: within 2^-7 relative + 2e-2 (RoPE cancellation);
  * sampled ids through the sampler's noise entry: bit-exact against the
    reference CPU sampler (oracle/sampler.py) on the step's logits, penalty
    and seen mask, except on rows where a top-k / top-p cut runs through tied
    logits (the reference's torch.topk leaves their order unspecified): there
    the id must lie in the support extended by the tie group; the seen mask, the terminal flags and the request slots'
    step and RNG offset after the step.
"""

from __future__ import annotations

from importlib import import_module

import pytest
import torch

from oracle import fp8 as ofp8
from oracle import sampler as osamp
from oracle import step_control as octl
from oracle import talker_step as ostep

pytestmark = pytest.mark.gpu

LAYERS = 2


def _cpu(t):
    return t.detach().float().cpu()


def _close(got, want, atol, rtol, mean_tol, what):
    err = (got - want).abs()
    bound = atol + rtol * want.abs()
    worst = float((err - bound).max())
    assert worst <= 0, f"{what}: max |err| {float(err.max()):.3e} exceeds the bound by {worst:.3e}"
    assert float(err.mean()) <= mean_tol, f"{what}: mean |err| {float(err.mean()):.3e}"


def _layer_weights(w, layer, shape):
    nxt = w.ln_final if layer + 1 == shape.num_layers else w.ln_in[layer + 1]
    a = w.attn[layer]
    return dict(w_qkv=_cpu(w.w_qkv[layer]), w_o=_cpu(w.w_o[layer]), w_gate_up=_cpu(w.w_gate_up[layer]),
                w_down=_cpu(w.w_down[layer]), ln_post=_cpu(w.ln_post[layer]), ln_next=_cpu(nxt),
                q_norm=a.q_norm.weight.cpu(), k_norm=a.k_norm.weight.cpu(), eps=shape.eps, theta=shape.rope_theta,
                heads=shape.num_heads, kv_heads=shape.num_kv_heads, head_dim=shape.head_dim)


def _meta(b, prefix=""):
    rows = b.capture_batch_size
    indptr = b.paged_kv_indptr.cpu()
    out = {
        prefix + "pos": b.position_ids.cpu(), prefix + "wp": b.write_pages.cpu(), prefix + "wo": b.write_offsets.cpu(),
        prefix + "indptr": indptr, prefix + "indices": b.paged_kv_indices[: int(indptr[rows])].cpu(),
        prefix + "last": b.paged_kv_last_page_len.cpu(),
    }
    if prefix:
        out[prefix + "qo_indptr"] = b.qo_indptr.cpu()
    return out


def _tie_support(scaled: torch.Tensor, d) -> tuple[set[int], bool]:
    """(ids a conforming sampler may keep, whether the kept set depends on the order of tied values) for one
    row of oracle details.  The reference ranks with torch.topk, whose order among equal values is unspecified
    (the CUDA sampler uses value descending, token id ascending), so a top-k or top-p cut through a group of
    tied values - common with bf16 logits - keeps an implementation-defined subset of the group."""

    kept = {int(t) for t, q in zip(d[2], d[1], strict=True) if q > 0}
    vmin = min(float(scaled[t]) for t in kept)
    tied = set((scaled == vmin).nonzero().flatten().tolist())
    return kept | tied, not tied <= kept


def _check_logits(step, got, hidden):
    """Codec head + suppress mask of forward_logits against the oracle (first decode step: EOS suppressed)."""

    s = step.shape
    want = octl.mask_logits(ostep.head_logits(hidden, _cpu(step.weights.w_head)), s.codec_vocab, s.eos_id,
                            [True] * got.shape[0])
    finite = torch.isfinite(want)
    assert torch.equal(torch.isfinite(got), finite) and bool((got[~finite] < 0).all())
    _close(got[finite], want[finite], 1e-2, 2.0**-7, 1e-3, "codec head logits")


def _check_layers(step, trace, storage0, meta, prefill_rows=0):
    shape, w = step.shape, step.weights
    x0, r0 = _cpu(trace[0][0]), _cpu(trace[0][1])
    want_x0 = ostep._round(ostep.rmsnorm(r0, _cpu(w.ln_in[0]), shape.eps))
    _close(x0, want_x0, 1e-2, 2.0**-7, 1e-3, "input norm")
    for layer in range(shape.num_layers):
        cache = storage0[layer].clone()
        x_in, r_in = _cpu(trace[layer][0]), _cpu(trace[layer][1])
        fp8 = len(trace[layer + 1]) == 4  # (x, residual, e4m3 MLP rows, scales) on the FP8 path
        rows = (trace[layer + 1][2].cpu(), trace[layer + 1][3].cpu()) if fp8 else None
        probe: dict = {}
        want_x, want_r = ostep.layer_forward(x_in, r_in, cache=cache, meta=meta, prefill_rows=prefill_rows,
                                             gate_up_fp8=fp8, fp8_rows=rows, probe=probe,
                                             **_layer_weights(w, layer, shape))
        if fp8:
            # the oracle's own quantisation of its MLP input against the GPU's (inputs may differ by a bf16 ulp)
            # (a block's amax moving by one ulp rescales the whole block, so compare dequantised values: one e4m3
            # step, 2^-3 relative, plus the subnormal step, plus the 2e-2 the MLP inputs may differ by)
            oq, os_ = ofp8.quantize_rows(probe["mlp_in"].to(torch.bfloat16))
            assert bool(((os_ - rows[1]).abs() <= 2.0**-7 * os_.abs()).all()), f"layer {layer} activation scales"
            t = oq.shape[0]
            deq_o = oq.float().view(t, -1, 128) * os_.T.reshape(t, -1, 1)
            deq_g = rows[0].float().view(t, -1, 128) * rows[1].T.reshape(t, -1, 1)
            bound = 2.0**-3 * deq_o.abs() + 2.0**-9 * os_.T.reshape(t, -1, 1) + 2e-2
            assert bool(((deq_g - deq_o).abs() <= bound).all()), f"layer {layer}: e4m3 MLP input beyond one step"
            same = float((oq.view(torch.uint8) == rows[0].view(torch.uint8)).float().mean())
            assert same >= 0.95, f"layer {layer}: only {same:.4f} of the e4m3 MLP input bytes agree"
        got_x, got_r = _cpu(trace[layer + 1][0]), _cpu(trace[layer + 1][1])
        _close(got_r, want_r, 2e-2, 2.0**-6, 2e-3, f"layer {layer} residual")
        _close(got_x, want_x, 2e-2, 2.0**-6, 2e-3, f"layer {layer} normed output")
        # the K/V rows this step wrote (rotated K, raw V)
        keys = [k for k in ("pre_", "") if k + "wp" in meta]
        live = step.storage[layer].cpu()
        for key in keys:
            wp, wo = meta[key + "wp"], meta[key + "wo"]
            n = wp.shape[0] if key else (x_in.shape[0] - prefill_rows)
            # RoPE output x1 cos - x2 sin can be much smaller than its inputs: one bf16 ulp of |x| < 4 absolute
            _close(live[wp[:n], :, wo[:n]].float(), cache[wp[:n], :, wo[:n]].float(), 2e-2, 2.0**-7, 1e-3,
                   f"layer {layer} K/V write")


@pytest.mark.parametrize("gate_up", ["fp8", "bf16"])
def test_talker_decode_step_matches_oracle(nqt, cuda, gate_up):
    ts = import_module("nari-qwen3-tts_b200.talker_step")
    shape = ts.TalkerShape(num_layers=LAYERS)
    rows = 64
    g = torch.Generator().manual_seed(21)
    contexts = torch.randint(64, 2049, (rows,), generator=g).tolist()
    pages = sum((n + 16) // 16 for n in contexts) + 2 * rows + 64
    step = ts.TalkerDecodeStep(shape=shape, batch=rows, total_pages=pages, page_size=16,
                               max_pages_per_seq=(2048 + 64) // 16 + 1, device=cuda, seed=21, publish=False,
                               gate_up=gate_up)
    step.admit(contexts, scatter_seed=21)
    step.hidden_in.copy_(torch.randn(rows, shape.hidden, generator=g).to(torch.bfloat16).to(cuda))
    storage0 = step.storage.cpu()
    ctl = step.control
    seen0, off0, step0 = step.seen.cpu(), ctl.slot_offset.cpu(), ctl.slot_step.cpu()
    nqt.kernels.clear_status(cuda)

    trace: list = []
    step.forward(trace)
    torch.cuda.synchronize()
    meta = _meta(step.binding)
    assert meta["pos"].tolist() == contexts  # one new token after each context
    _check_layers(step, trace, storage0, meta)
    logits = _cpu(trace[-1])
    _check_logits(step, logits, _cpu(trace[-2][0]))
    assert torch.equal(step.offset.cpu(), off0)  # staged from the request slots

    # sampled ids through the noise entry: the oracle's Exp(1) noise, handed over by token id
    temp, top_k, top_p = step.temperature.cpu(), step.top_k.cpu(), step.top_p.cpu()
    pen, seed = step.penalty.cpu(), step.seed.cpu()
    kw = dict(repetition_penalty=pen, seen_token_mask=seen0)
    details = osamp.row_details(logits, temp, top_k, top_p, seed, off0, **kw)
    want = osamp.sample_logits(logits, temp, top_k, top_p, seed, off0, **kw)
    _, _, ids_k = nqt.sample_rows(trace[-1], step.temperature, step.top_k, step.top_p, step.seed, step.offset,
                                  repetition_penalty=step.penalty, seen_token_mask=seen0.to(cuda),
                                  noise=torch.ones(rows, shape.vocab, device=cuda), return_probs=True)
    ids_k = ids_k.cpu().long()
    noise = torch.full((rows, shape.vocab), 1.0e30)
    for row, d in enumerate(details):
        pos = {int(t): i for i, t in enumerate(d[2])}
        for r in range(d[0]):
            i = pos.get(int(ids_k[row, r]))
            if i is not None:
                noise[row, r] = d[3][i]
    # replay the same step (its reservation was discarded) with the noise entry
    step.seen.copy_(seen0.to(cuda))
    ctl.slot_offset.copy_(off0.to(cuda))
    ctl.slot_step.copy_(step0.to(cuda))
    step.sample_noise = noise.to(cuda)
    trace2: list = []
    tokens = step.forward(trace2).cpu()
    torch.cuda.synchronize()
    assert torch.equal(trace2[-1], trace[-1]), "the step is not deterministic"
    scaled = osamp.scaled_rows(logits, temp, pen, seen0)
    for row, d in enumerate(details):
        support, ambiguous = _tie_support(scaled[row], d)
        if ambiguous:  # a cut through tied values: the draw lies in the tie-extended support
            assert int(tokens[row]) in support, row
        else:
            assert int(tokens[row]) == int(want[row]), row
    expect_seen = seen0.clone()
    expect_seen[torch.arange(rows), tokens] = True
    assert torch.equal(step.seen.cpu(), expect_seen)
    assert torch.equal(ctl.slot_offset.cpu(), off0 + ts.FRAME_OFFSET_STRIDE)
    assert torch.equal(ctl.slot_step.cpu(), step0 + 1)
    assert not bool(ctl.terminal.cpu().any())  # EOS is suppressed on the first steps, no limit
    assert nqt.kernels.read_status(cuda) == 0 and int(step.planner.status.item()) == 0


def test_talker_mixed_step_matches_oracle(nqt, cuda):
    ts = import_module("nari-qwen3-tts_b200.talker_step")
    shape = ts.TalkerShape(num_layers=LAYERS)
    g = torch.Generator().manual_seed(31)
    chunks = [37, 128, 5, 300]
    decode_ctx = torch.randint(32, 700, (20,), generator=g).tolist()
    step = ts.TalkerMixedStep(shape=shape, chunks=chunks, decode_contexts=decode_ctx, churn_rows=4, total_pages=2048,
                              page_size=16, device=cuda, seed=31)
    step.admit(scatter_seed=31)
    step.hidden_in.copy_(torch.randn(step.tokens, shape.hidden, generator=g).to(torch.bfloat16).to(cuda))
    storage0 = step.storage.cpu()
    seen0, off0 = step.seen.cpu(), step.control.slot_offset.cpu()
    nqt.kernels.clear_status(cuda)

    trace: list = []
    tokens = step.forward(trace).cpu()
    torch.cuda.synchronize()
    meta = {**_meta(step.pre_b, "pre_"), **_meta(step.dec_b)}
    assert meta["pre_qo_indptr"].tolist() == [0, *torch.tensor(chunks).cumsum(0).tolist()]
    _check_layers(step, trace, storage0, meta, prefill_rows=step.t_pre)
    final = _cpu(trace[-2][0])
    sampled = final.index_select(0, step._sample_rows.cpu())
    logits = _cpu(trace[-1])
    _check_logits(step, logits, sampled)
    # the production draw: every sampled id lies in the reference sampler's filtered support
    details = osamp.row_details(logits, step.temperature.cpu(), step.top_k.cpu(), step.top_p.cpu(), step.seed.cpu(),
                                off0, repetition_penalty=step.penalty.cpu(), seen_token_mask=seen0)
    scaled = osamp.scaled_rows(logits, step.temperature.cpu(), step.penalty.cpu(), seen0)
    for row, d in enumerate(details):
        support, _ = _tie_support(scaled[row], d)
        assert int(tokens[row]) in support, row
    expect_seen = seen0.clone()
    expect_seen[torch.arange(step.rows), tokens] = True
    assert torch.equal(step.seen.cpu(), expect_seen)
    assert torch.equal(step.control.slot_offset.cpu(), off0 + ts.FRAME_OFFSET_STRIDE)
    assert not bool(step.control.terminal.cpu().any())
    assert nqt.kernels.read_status(cuda) == 0
