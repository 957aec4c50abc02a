"""CPU port of one code-predictor frame (test and baseline infrastructure
only; the product never imports it).

Restates the reference's whole_frame (executor/code_predictor.py:160-235)
and its fused depth step (model/components.py:254-356) with the oracle
pieces: QK RMSNorm + RoPE + dense cache write (oracle/attention.py
qk_norm_rope_dense_), one-query short-cache attention
(short_cache_attention), and the reference's CPU sampler semantics
(oracle/sampler.py).  Activations are rounded to bf16 at the same op
boundaries as the reference's bf16 module path (GEMM outputs, norm outputs,
the residual stream), arithmetic inside an op is fp32.

``forced_tokens`` teacher-forces the residual tokens so that the per-group
logits can be compared with the GPU frame's independent of sampling.
"""

from __future__ import annotations

import time

import torch
import torch.nn.functional as F

from . import attention as oatt
from . import sampler as osamp

BF16 = torch.bfloat16


def _bf(x: torch.Tensor) -> torch.Tensor:
    return x.to(BF16).float()


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return _bf(x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w)


class CpuCodePredictorFrame:
    """``weights`` maps the GPU frame's attribute names to CPU tensors (any
    float dtype): w_in, b_in, w_qkv[L], w_o[L], w_gate_up[L], w_down[L],
    ln_in[L], ln_post[L], q_norm[L], k_norm[L], ln_final, lm_head,
    codec_embedding, layer0_embedding."""

    def __init__(self, weights: dict, *, heads=16, kv_heads=8, head_dim=64, groups=16, eps=1e-6,
                 theta=1.0e6) -> None:
        self.w = {k: ([t.float() for t in v] if isinstance(v, list) else v.float()) for k, v in weights.items()}
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.groups, self.eps, self.theta = groups, eps, theta
        self.layers = len(self.w["w_qkv"])
        w_in, b_in = self.w["w_in"], self.w["b_in"]
        # executor/code_predictor.py:73-88: projections of the embedding tables, rounded to the model dtype
        self.projected_layer0 = _bf(self.w["layer0_embedding"] @ w_in.T + b_in)
        self.projected_residual = [_bf(self.w["codec_embedding"][i] @ w_in.T + b_in) for i in range(groups - 2)]

    @classmethod
    def random(cls, *, layers=5, hidden=1024, heads=16, kv_heads=8, head_dim=64, ffn=3072, vocab=2048, groups=16,
               talker_hidden=2048, seed=0):
        g = torch.Generator().manual_seed(seed)

        def w(o, i):
            return (torch.randn(o, i, generator=g) * i**-0.5).to(BF16)

        qkv = (heads + 2 * kv_heads) * head_dim
        weights = {
            "w_in": w(hidden, talker_hidden), "b_in": torch.zeros(hidden, dtype=BF16),
            "w_qkv": [w(qkv, hidden) for _ in range(layers)], "w_o": [w(hidden, heads * head_dim) for _ in range(layers)],
            "w_gate_up": [w(2 * ffn, hidden) for _ in range(layers)], "w_down": [w(hidden, ffn) for _ in range(layers)],
            "ln_in": [torch.ones(hidden, dtype=BF16)] * layers, "ln_post": [torch.ones(hidden, dtype=BF16)] * layers,
            "q_norm": [torch.ones(head_dim, dtype=BF16)] * layers, "k_norm": [torch.ones(head_dim, dtype=BF16)] * layers,
            "ln_final": torch.ones(hidden, dtype=BF16),
            "lm_head": torch.stack([w(vocab, hidden) for _ in range(groups - 1)]),
            "codec_embedding": (0.02 * torch.randn(groups - 1, vocab, talker_hidden, generator=g)).to(BF16),
            "layer0_embedding": (0.02 * torch.randn(vocab, talker_hidden, generator=g)).to(BF16),
        }
        return cls(weights, heads=heads, kv_heads=kv_heads, head_dim=head_dim, groups=groups)

    def _depth_step(self, x: torch.Tensor, cache: list, cache_pos: int, final_norm: bool) -> torch.Tensor:
        for layer in range(self.layers):
            x = self.depth_layer(x, layer, cache, cache_pos)
        return _rms(x, self.w["ln_final"], self.eps) if final_norm else x

    def depth_layer(self, x: torch.Tensor, layer: int, cache: list, cache_pos: int) -> torch.Tensor:
        """One decoder layer of a depth step on the residual stream x (model/components.py:300-350):
        RMSNorm, QKV, QK norm + RoPE + dense cache write, short-cache attention, O, residual add (rounded),
        RMSNorm, gate/up, SiLU * up, down, residual add.  Writes cache[layer] at cache_pos."""

        w = self.w
        rows = x.shape[0]
        hq, hkv, d = self.heads, self.kv_heads, self.head_dim
        positions = torch.full((rows,), cache_pos, dtype=torch.long)
        h = _rms(x, w["ln_in"][layer], self.eps)
        qkv = _bf(h @ w["w_qkv"][layer].T)
        q = qkv[:, : hq * d].reshape(rows, hq, d).to(BF16)
        k = qkv[:, hq * d: (hq + hkv) * d].reshape(rows, hkv, d).to(BF16)
        v = qkv[:, (hq + hkv) * d:].reshape(rows, hkv, d).to(BF16)
        kc, vc = cache[layer]
        oatt.qk_norm_rope_dense_(q, k, v, w["q_norm"][layer].to(BF16), w["k_norm"][layer].to(BF16), positions,
                                 self.eps, self.theta, kc, vc, cache_pos, round_to_input=False)
        attn = _bf(oatt.short_cache_attention(q, kc, vc, cache_pos + 1))
        x = _bf(x + _bf(attn.reshape(rows, hq * d) @ w["w_o"][layer].T))
        h = _rms(x, w["ln_post"][layer], self.eps)
        gu = _bf(h @ w["w_gate_up"][layer].T)
        ffn = gu.shape[1] // 2
        act = _bf(F.silu(gu[:, :ffn]) * gu[:, ffn:])
        x = _bf(x + _bf(act @ w["w_down"][layer].T))
        return x

    def frame(self, past_hidden, layer0_token, *, temperature, top_k, top_p, seed, offsets, forced_tokens=None):
        """Returns (frames [rows, groups], logits [groups-1, rows, vocab] fp32, codec_sum fp32)."""

        w = self.w
        rows = past_hidden.shape[0]
        cache = [(torch.zeros(rows, self.groups, self.kv_heads, self.head_dim, dtype=BF16),
                  torch.zeros(rows, self.groups, self.kv_heads, self.head_dim, dtype=BF16))
                 for _ in range(self.layers)]
        hidden0 = _bf(_bf(past_hidden.float()) @ w["w_in"].T + w["b_in"])
        self._depth_step(hidden0, cache, 0, final_norm=False)
        frames = torch.zeros(rows, self.groups, dtype=torch.long)
        frames[:, 0] = layer0_token
        codec_sum = w["layer0_embedding"][layer0_token].clone()
        x = self.projected_layer0[layer0_token]
        logits_all = []
        for group in range(1, self.groups):
            hidden = self._depth_step(x, cache, group, final_norm=True)
            logits = _bf(hidden @ w["lm_head"][group - 1].T)
            logits_all.append(logits)
            if forced_tokens is not None:
                token = forced_tokens[:, group].long()
            else:
                token = osamp.sample_logits(logits, temperature, top_k, top_p, seed, offsets[:, group - 1])
            frames[:, group] = token
            codec_sum = _bf(codec_sum + w["codec_embedding"][group - 1][token])
            if group < self.groups - 1:
                x = self.projected_residual[group - 1][token]
        return frames, torch.stack(logits_all), codec_sum

    def time_frame(self, rows: int) -> float:
        """Seconds for one sampled frame of ``rows`` rows (T 0.9, top-k 50)."""

        past = torch.randn(rows, self.w["w_in"].shape[1])
        layer0 = torch.randint(0, self.w["layer0_embedding"].shape[0], (rows,))
        offsets = torch.arange(1, self.groups).unsqueeze(0).expand(rows, -1) * 32
        t0 = time.perf_counter()
        self.frame(past, layer0, temperature=torch.full((rows,), 0.9), top_k=torch.full((rows,), 50, dtype=torch.int32),
                   top_p=torch.ones(rows), seed=torch.arange(rows), offsets=offsets)
        return time.perf_counter() - t0
