"""CPU port of one talker step: the teacher-forced layer used by the step
parity tests, and the timed CPU baseline.

The reference has no CPU talker attention (attend() always runs Triton +
FlashInfer), so its "CPU torch path" for this step is restated here with
the oracle pieces: the host page allocator and metadata builder
(oracle/planner.py, = executor/cache.py + executor/talker_kv.py:403-480),
RMSNorm / QK-norm + RoPE + paged K/V write / paged decode and causal
prefill attention in fp32 (oracle/attention.py), fp32 torch GEMMs for the
projections and MLP, and the reference CPU sampler semantics
(oracle/sampler.py).

``layer_forward`` is one decoder layer in the order of the reference's
captured step (model/components.py:37-90 with model/layers.py:28-115,
296-317): QKV projection, attend (QK norm + RoPE + K/V write, attention),
O projection, fused residual add + post-attention RMSNorm, gate/up,
SiLU * up, down, fused residual add + the next layer's input RMSNorm.  It
rounds to bf16 wherever the bf16 step materialises a tensor (each GEMM
output, the attention output, the residual, each norm output), so a
teacher-forced comparison with the GPU step sees only accumulation-order and
attention-tolerance differences.  The fused add + RMSNorm follows FlashInfer's
fused_add_rmsnorm: the sum is kept in fp32 for the norm and stored to the
residual rounded.

``CpuTalkerStep.time_step`` runs the whole step - the planner, every
decoder layer for every row, the head and the sampler - on the host cores.
Only ``layers_resident`` layers of weights and KV are held (the port cycles
through them), which changes no arithmetic.  Test and baseline
infrastructure only; the product never imports it.
"""

from __future__ import annotations

import time

import torch

from . import attention as oatt
from . import fp8 as ofp8
from . import planner as oplan
from . import sampler as osamp

BF16 = torch.bfloat16


def _round(x: torch.Tensor) -> torch.Tensor:
    return x.to(BF16).float()


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """fp32 RMSNorm (model/layers.py:110-115 / flashinfer.norm.rmsnorm), unrounded."""

    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """(normed bf16, residual bf16) of flashinfer.norm.fused_add_rmsnorm (model/layers.py:42-77)."""

    r = x.float() + residual.float()
    return _round(rmsnorm(r, w, eps)), _round(r)


def layer_forward(x, residual, *, w_qkv, w_o, w_gate_up, w_down, ln_post, ln_next, q_norm, k_norm, eps, theta,
                  heads, kv_heads, head_dim, cache, meta, prefill_rows=0, gate_up_fp8=False, fp8_rows=None,
                  probe=None):
    """One decoder layer, teacher-forced.

    x: the layer's normed input, residual: the residual stream (both [T, hidden],
    bf16 values).  cache: the layer view [pages, 2, P, Hkv, D] bf16 (written in
    place).  meta: dict of CPU tensors for the step's rows - for a decode
    group ``pos, wp, wo, indptr, indices, last``; with ``prefill_rows`` > 0 the
    first ``prefill_rows`` tokens form a prefill group described by
    ``pre_*`` keys (``pre_qo_indptr`` included) and the rest the decode group.
    ``gate_up_fp8``: the gate/up projection takes the reference's FP8 path (128 x 128 weight blocks, per-token
    128-element activation blocks, oracle/fp8.py) instead of bf16; ``fp8_rows`` = (e4m3 rows, scales) replaces
    the quantised MLP input (teacher forcing at the quantisation step).  ``probe``, a dict, receives the MLP
    input ("mlp_in", bf16 values).
    Returns (next normed input, residual), bf16 values in fp32 tensors.
    """

    h, hkv, d = heads, kv_heads, head_dim
    t = x.shape[0]
    qkv = _round(x.float() @ w_qkv.float().T)
    q = qkv[:, : h * d].reshape(t, h, d).to(BF16)
    k = qkv[:, h * d: (h + hkv) * d].reshape(t, hkv, d).to(BF16)
    v = qkv[:, (h + hkv) * d:].reshape(t, hkv, d).to(BF16)
    attn = torch.zeros(t, h, d)
    groups = []
    if prefill_rows:
        groups.append(("pre_", 0, prefill_rows, True))
    groups.append(("", prefill_rows, t, False))
    for key, lo, hi, is_prefill in groups:
        if hi == lo:
            continue
        qs, ks = q[lo:hi].clone(), k[lo:hi].clone()
        oatt.qk_norm_rope_paged_(qs, ks, v[lo:hi], q_norm, k_norm, meta[key + "pos"], eps, theta, cache,
                                 meta[key + "wp"], meta[key + "wo"])
        if is_prefill:
            attn[lo:hi] = oatt.paged_prefill(qs.float(), cache, meta["pre_qo_indptr"], meta["pre_indptr"],
                                             meta["pre_indices"], meta["pre_last"])
        else:
            attn[lo:hi] = oatt.paged_decode(qs.float(), cache, meta["indptr"], meta["indices"], meta["last"])
    o = _round(_round(attn).reshape(t, h * d) @ w_o.float().T)
    x2, residual = add_rmsnorm(o, residual, ln_post, eps)
    if probe is not None:
        probe["mlp_in"] = x2
    if gate_up_fp8:
        xq, xs = fp8_rows if fp8_rows is not None else ofp8.quantize_rows(x2.to(BF16))
        wq, ws = ofp8.quantize_weight_blocks(w_gate_up.to(BF16))
        act = ofp8.swiglu(ofp8.gemm_blockscaled(xq, xs, wq, ws)).float()
    else:
        gu = _round(x2 @ w_gate_up.float().T)
        ffn = gu.shape[1] // 2
        act = _round(torch.nn.functional.silu(gu[:, :ffn]) * gu[:, ffn:])
    m = _round(act @ w_down.float().T)
    return add_rmsnorm(m, residual, ln_next, eps)


def head_logits(x: torch.Tensor, w_head: torch.Tensor) -> torch.Tensor:
    """Codec head on the final normed hidden state, rounded to bf16 like the step's GEMM."""

    return _round(x.float() @ w_head.float().T)


class CpuTalkerStep:
    def __init__(self, *, contexts, num_layers=28, hidden=2048, heads=16, kv_heads=8, head_dim=128, ffn=6144,
                 vocab=3072, page_size=16, layers_resident=2, seed=0, eps=1e-6, theta=1.0e6) -> None:
        g = torch.Generator().manual_seed(seed)
        self.contexts = list(contexts)
        self.batch = len(contexts)
        self.num_layers = num_layers
        self.hidden, self.heads, self.kv_heads, self.head_dim, self.ffn = hidden, heads, kv_heads, head_dim, ffn
        self.vocab, self.page_size, self.eps, self.theta = vocab, page_size, eps, theta
        self.layers_resident = layers_resident
        qkv_out = (heads + 2 * kv_heads) * head_dim

        def w(o, i):
            return torch.randn(o, i, generator=g) * i**-0.5

        self.w_qkv = [w(qkv_out, hidden) for _ in range(layers_resident)]
        self.w_o = [w(hidden, heads * head_dim) for _ in range(layers_resident)]
        self.w_gu = [w(2 * ffn, hidden) for _ in range(layers_resident)]
        self.w_down = [w(hidden, ffn) for _ in range(layers_resident)]
        self.w_head = w(vocab, hidden)
        self.norm = torch.ones(hidden)
        self.qk_norm = torch.ones(head_dim, dtype=torch.bfloat16)
        pages = sum((n + 64 + page_size - 1) // page_size for n in contexts) + self.batch
        self.pool = oplan.HostPagePool(pages + self.batch, page_size, self.batch)
        self.cache = [torch.randn(pages + self.batch, 2, page_size, kv_heads, head_dim, generator=g).to(torch.bfloat16)
                      for _ in range(layers_resident)]
        for i, n in enumerate(contexts):
            self.pool.add_request(f"r{i}")
            self.pool.reserve([f"r{i}"], [n])
            self.pool.publish(f"r{i}")
        self.seen = torch.zeros(self.batch, vocab, dtype=torch.bool)
        self.seen.scatter_(1, torch.randint(0, vocab, (self.batch, 64), generator=g), True)
        self.offset = torch.zeros(self.batch, dtype=torch.long)

    def _layer(self, layer, x, residual, meta):
        i = layer % self.layers_resident
        return layer_forward(x, residual, w_qkv=self.w_qkv[i], w_o=self.w_o[i], w_gate_up=self.w_gu[i],
                             w_down=self.w_down[i], ln_post=self.norm, ln_next=self.norm, q_norm=self.qk_norm,
                             k_norm=self.qk_norm, eps=self.eps, theta=self.theta, heads=self.heads,
                             kv_heads=self.kv_heads, head_dim=self.head_dim, cache=self.cache[i], meta=meta)

    def time_step(self, *, layers: int | None = None) -> dict:
        """Run one whole step (all rows; ``layers`` decoder layers, by default
        all of them) and return the seconds spent in each part."""

        layers = self.num_layers if layers is None else layers
        rids = [f"r{i}" for i in range(self.batch)]
        rows = self.batch
        t0 = time.perf_counter()
        m = self.pool.metadata(rids, [1] * rows, rows, rows, False)
        meta = {
            "indptr": torch.tensor(m["paged_kv_indptr"], dtype=torch.int32),
            "indices": torch.tensor(m["paged_kv_indices"], dtype=torch.int32),
            "last": torch.tensor(m["paged_kv_last_page_len"], dtype=torch.int32),
            "pos": torch.tensor(m["position_ids"]),
            "wp": torch.tensor(m["write_pages"]),
            "wo": torch.tensor(m["write_offsets"]),
        }
        t1 = time.perf_counter()
        residual = _round(torch.randn(rows, self.hidden))
        x = _round(rmsnorm(residual, self.norm, self.eps))
        for layer in range(layers):
            x, residual = self._layer(layer, x, residual, meta)
        t2 = time.perf_counter()
        logits = head_logits(x, self.w_head)
        tokens = osamp.sample_logits(
            logits, torch.full((rows,), 0.9), torch.full((rows,), 50, dtype=torch.int32), torch.full((rows,), 0.95),
            torch.arange(rows), self.offset, repetition_penalty=torch.full((rows,), 1.05),
            seen_token_mask=self.seen)
        self.seen[torch.arange(rows), tokens] = True
        t3 = time.perf_counter()
        # discard the reservation so every step sees the same lengths (a stationary workload)
        for rid in rids:
            self.pool.discard(rid)
        self.offset += 512
        return {"planner_s": t1 - t0, "layers_s": t2 - t1, "head_sampler_s": t3 - t2, "step_s": t3 - t0,
                "layers": layers}
