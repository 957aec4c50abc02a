"""CPU port of one talker decode step, timed as the CPU baseline.

The reference has no CPU talker attention (attend() always runs Triton +
FlashInfer), so its "CPU torch path" for this step is restated here with
the oracle pieces: the host page allocator and metadata builder
(oracle/planner.py, = executor/cache.py + executor/talker_kv.py:403-480),
RMSNorm / QK-norm + RoPE + paged K/V write / paged decode attention in fp32
(oracle/attention.py), fp32 torch GEMMs for the projections and MLP, and the
reference CPU sampler semantics (oracle/sampler.py).

``CpuTalkerStep.time_step`` runs a bounded sample of the step - the planner,
``rows`` rows through ``layers`` of the decoder layers and the head +
sampler - and extrapolates to the full step (all layers, all rows) because
every term is linear in rows and layers.  Test and baseline infrastructure
only; the product never imports it.
"""

from __future__ import annotations

import time

import torch

from . import attention as oatt
from . import planner as oplan
from . import sampler as osamp


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

    @staticmethod
    def _rms(x, w, eps):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w

    def _layer(self, layer, x, meta, rows):
        h, hkv, d = self.heads, self.kv_heads, self.head_dim
        qkv = self._rms(x, self.norm, self.eps) @ self.w_qkv[layer].T
        q = qkv[:, : h * d].reshape(rows, h, d).to(torch.bfloat16)
        k = qkv[:, h * d: (h + hkv) * d].reshape(rows, hkv, d).to(torch.bfloat16)
        v = qkv[:, (h + hkv) * d:].reshape(rows, hkv, d).to(torch.bfloat16)
        oatt.qk_norm_rope_paged_(q, k, v, self.qk_norm, self.qk_norm, meta["pos"], self.eps, self.theta,
                                 self.cache[layer], meta["wp"], meta["wo"])
        attn = oatt.paged_decode(q.float(), self.cache[layer], meta["indptr"], meta["indices"], meta["last"])
        x = x + attn.reshape(rows, h * d) @ self.w_o[layer].T
        gu = self._rms(x, self.norm, self.eps) @ self.w_gu[layer].T
        act = torch.nn.functional.silu(gu[:, : self.ffn]) * gu[:, self.ffn:]
        return x + act @ self.w_down[layer].T

    def time_step(self, *, rows: int | None = None, layers: int = 1) -> dict:
        """Run one sampled step; returns the measured parts and the
        extrapolated full-step seconds."""

        rows = rows or self.batch
        rids = [f"r{i}" for i in range(self.batch)]
        t0 = time.perf_counter()
        m = self.pool.metadata(rids, [1] * self.batch, self.batch, self.batch, False)
        t1 = time.perf_counter()
        sel = slice(0, rows)
        nsel = m["paged_kv_indptr"][rows]
        meta = {
            "indptr": torch.tensor(m["paged_kv_indptr"][: rows + 1], dtype=torch.int32),
            "indices": torch.tensor(m["paged_kv_indices"][:nsel], dtype=torch.int32),
            "last": torch.tensor(m["paged_kv_last_page_len"][sel], dtype=torch.int32),
            "pos": torch.tensor(m["position_ids"][sel]),
            "wp": torch.tensor(m["write_pages"][sel]),
            "wo": torch.tensor(m["write_offsets"][sel]),
        }
        x = torch.randn(rows, self.hidden)
        t2 = time.perf_counter()
        for i in range(layers):
            x = self._layer(i % self.layers_resident, x, meta, rows)
        t3 = time.perf_counter()
        logits = self._rms(x, self.norm, self.eps) @ self.w_head.T
        tokens = osamp.sample_logits(
            logits, torch.full((rows,), 0.9), torch.full((rows,), 50, dtype=torch.int32), torch.full((rows,), 0.95),
            torch.arange(rows), self.offset[sel], repetition_penalty=torch.full((rows,), 1.05),
            seen_token_mask=self.seen[sel])
        self.seen[torch.arange(rows), tokens] = True
        t4 = time.perf_counter()
        # discard the reservation so every sampled step sees the same lengths (a stationary sample)
        for rid in rids:
            self.pool.discard(rid)
        self.offset += 512
        scale_rows = self.batch / rows
        full = (t1 - t0) + scale_rows * ((t3 - t2) * self.num_layers / layers + (t4 - t3))
        return {"planner_s": t1 - t0, "layers_s": t3 - t2, "head_sampler_s": t4 - t3, "full_step_s": full,
                "rows": rows, "layers": layers}
