"""One code-predictor frame (15 residual codebooks) of a batch of rows,
captured as one CUDA graph: the reference's whole_frame
(executor/code_predictor.py:160-235) on the sm_100a kernels.

    hidden0 = small_to_mtp_projection(past_hidden)          # talker 2048 -> 1024
    depth step at cache position 0 (fills the dense frame cache)
    for group in 1..15:
        depth step at cache position `group` on the projected embedding of the
        previous token -> final RMSNorm -> logits = hidden @ lm_head[group-1]^T
        token = fused sampler (row-local Philox, offsets frame*512 + group*32)
        codec_sum += codec_embedding[group-1](token)

A depth step runs 5 decoder layers; each layer's attention is one fused launch
(QK RMSNorm + RoPE, K/V write into the dense cache at the step's position,
short-cache GQA attention: nqt_cp_decode_attention), the glue is the fused
add + RMSNorm and SwiGLU kernels and the projections are cuBLAS calls.
Between depth steps one launch (nqt_cp_codec_step) writes the frame's code,
adds the codec embedding to the sum and prepares the next step's input and
its first norm, in place of six torch / glue ops.  Weights are random (bf16).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import kernels
from .sampling import sample_rows

CODEBOOK_STRIDE = 32  # contract/rng.py: PHILOX_CODEBOOK_STRIDE
FRAME_STRIDE = 512


@dataclass(frozen=True)
class CodePredictorShape:
    num_layers: int = 5
    hidden: int = 1024
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 64
    ffn: int = 3072
    vocab: int = 2048
    groups: int = 16
    talker_hidden: int = 2048
    rope_theta: float = 1.0e6
    eps: float = 1e-6


class CodePredictorFrame:
    def __init__(self, *, shape: CodePredictorShape = CodePredictorShape(), rows: int = 256,
                 device: torch.device | str = "cuda", seed: int = 0) -> None:
        self.shape = s = shape
        self.rows = rows
        self.device = dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)
        bf16 = torch.bfloat16

        def w(out_f, in_f):
            return (torch.randn(out_f, in_f, generator=g, device=dev) * in_f**-0.5).to(bf16)

        def norm_w(n):
            return (1.0 + 0.05 * torch.randn(n, generator=g, device=dev)).to(bf16)

        qkv_out = (s.num_heads + 2 * s.num_kv_heads) * s.head_dim
        L = s.num_layers
        self.w_in = w(s.hidden, s.talker_hidden)  # small_to_mtp_projection
        self.b_in = (0.01 * torch.randn(s.hidden, generator=g, device=dev)).to(bf16)
        self.w_qkv = [w(qkv_out, s.hidden) for _ in range(L)]
        self.w_o = [w(s.hidden, s.num_heads * s.head_dim) for _ in range(L)]
        self.w_gate_up = [w(2 * s.ffn, s.hidden) for _ in range(L)]
        self.w_down = [w(s.hidden, s.ffn) for _ in range(L)]
        self.ln_in = [norm_w(s.hidden) for _ in range(L)]
        self.ln_post = [norm_w(s.hidden) for _ in range(L)]
        self.q_norm = [norm_w(s.head_dim) for _ in range(L)]
        self.k_norm = [norm_w(s.head_dim) for _ in range(L)]
        self.ln_final = norm_w(s.hidden)
        self.lm_head = torch.stack([w(s.vocab, s.hidden) for _ in range(s.groups - 1)])
        # codec embeddings (talker width) and their projections to the predictor width
        self.codec_embedding = (0.02 * torch.randn(s.groups - 1, s.vocab, s.talker_hidden, generator=g,
                                                   device=dev)).to(bf16)
        self.layer0_embedding = (0.02 * torch.randn(s.vocab, s.talker_hidden, generator=g, device=dev)).to(bf16)
        self.projected_layer0 = F.linear(self.layer0_embedding, self.w_in, self.b_in)
        self.projected_residual = torch.stack(
            [F.linear(self.codec_embedding[i], self.w_in, self.b_in) for i in range(s.groups - 2)])
        # dense frame cache [layers, rows, 2, positions, kv_heads, head_dim] (executor/code_predictor.py:90-110)
        self.kv_cache = torch.zeros((L, rows, 2, s.groups, s.num_kv_heads, s.head_dim), dtype=bf16, device=dev)
        # static graph inputs / outputs
        self.past_hidden = torch.zeros(rows, s.talker_hidden, dtype=bf16, device=dev)
        self.layer0_token = torch.zeros(rows, dtype=torch.long, device=dev)
        self.temperature = torch.full((rows,), 0.9, device=dev)
        self.top_k = torch.full((rows,), 50, dtype=torch.int32, device=dev)
        self.top_p = torch.ones(rows, device=dev)
        self.seed = torch.arange(rows, dtype=torch.long, device=dev)
        self.offsets = torch.zeros(rows, s.groups - 1, dtype=torch.long, device=dev)
        self.positions = torch.arange(s.groups, device=dev).unsqueeze(0).expand(rows, -1).contiguous()
        self.frames = torch.zeros(rows, s.groups, dtype=torch.long, device=dev)
        self.codec_sum = torch.zeros(rows, s.talker_hidden, dtype=bf16, device=dev)
        self._act = torch.empty(rows, s.ffn, dtype=bf16, device=dev)
        self._residual = torch.empty(rows, s.hidden, dtype=bf16, device=dev)
        self._h = torch.empty(rows, s.hidden, dtype=bf16, device=dev)  # a depth step's first normed input
        self._token = torch.zeros(rows, dtype=torch.long, device=dev)
        # per-group logits stay resident (one [rows, vocab] slab per residual codebook)
        self.logits = torch.empty(s.groups - 1, rows, s.vocab, dtype=bf16, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self._host_in: tuple[torch.Tensor, torch.Tensor] | None = None
        self._host_frames: torch.Tensor | None = None

    def set_frame(self, frame_index: int) -> None:
        """RNG offsets of one frame: frame * 512 + group * 32 (contract/rng.py:33-41)."""

        groups = torch.arange(1, self.shape.groups, device=self.device)
        self.offsets.copy_((frame_index * FRAME_STRIDE + groups * CODEBOOK_STRIDE).unsqueeze(0).expand(self.rows, -1))

    def _depth_step(self, x: torch.Tensor | None, cache_pos: int, final_norm: bool,
                    residuals: list | None = None) -> torch.Tensor:
        """Five layers on one token per row at `cache_pos` (model/components.py:254-356).  ``x`` None: the
        input is already in the residual buffer and its first norm in ``_h`` (written by cp_codec_step).
        ``residuals`` (parity tests) receives the residual stream before each layer and after the last."""

        s = self.shape
        hq, hkv, d = s.num_heads, s.num_kv_heads, s.head_dim
        rows = self.rows
        residual = self._residual
        if x is None:
            h = self._h
        else:
            residual.copy_(x)
            h = kernels.rmsnorm(x, self.ln_in[0], s.eps, out=self._h)
        for layer in range(s.num_layers):
            if residuals is not None:
                residuals.append(residual.clone())
            qkv = F.linear(h, self.w_qkv[layer])
            q = qkv[:, : hq * d].view(rows, hq, d)
            k = qkv[:, hq * d: (hq + hkv) * d].view(rows, hkv, d)
            v = qkv[:, (hq + hkv) * d:].view(rows, hkv, d)
            attn = kernels.cp_decode_attention_(
                q, k, v, self.q_norm[layer], self.k_norm[layer], self.positions[:, cache_pos], s.eps, s.rope_theta,
                self.kv_cache[layer, :, 0], self.kv_cache[layer, :, 1], cache_pos)
            o = F.linear(attn.view(rows, hq * d), self.w_o[layer])
            kernels.fused_add_rmsnorm_(o, residual, self.ln_post[layer], s.eps)
            gate_up = F.linear(o, self.w_gate_up[layer])
            kernels.silu_and_mul(gate_up, out=self._act)
            m = F.linear(self._act, self.w_down[layer])
            last = layer + 1 == s.num_layers
            if last and not final_norm:
                residual.add_(m)
                if residuals is not None:
                    residuals.append(residual.clone())
                return residual
            kernels.fused_add_rmsnorm_(m, residual, self.ln_final if last else self.ln_in[layer + 1], s.eps)
            h = m
        if residuals is not None:
            residuals.append(residual.clone())
        return h

    def forward(self, trace: list | None = None) -> torch.Tensor:
        """The frame body (what capture() records).  ``trace``, for parity tests
        of an eager frame: receives per depth step (the residual stream before
        each layer and after the last, a copy of the frame cache before the
        step, the output hidden state or None for position 0)."""

        s = self.shape
        hidden0 = F.linear(self.past_hidden, self.w_in, self.b_in)
        residuals = [] if trace is not None else None
        cache_before = self.kv_cache.clone() if trace is not None else None
        self._depth_step(hidden0, 0, final_norm=False, residuals=residuals)
        if trace is not None:
            trace.append((residuals, cache_before, None))
        # codebook 0 (the talker's token): the frame's first code, the codec sum, the next step's input + norm
        kernels.cp_codec_step(self.layer0_token, self.frames[:, 0], self.layer0_embedding, self.codec_sum,
                              accumulate=False, proj_emb=self.projected_layer0, ln=self.ln_in[0], eps=s.eps,
                              residual=self._residual, h=self._h)
        for group in range(1, s.groups):
            cache_before = self.kv_cache.clone() if trace is not None else None
            residuals = [] if trace is not None else None
            hidden = self._depth_step(None, group, final_norm=True, residuals=residuals)
            if trace is not None:
                trace.append((residuals, cache_before, hidden.clone()))
            logits = torch.matmul(hidden, self.lm_head[group - 1].t(), out=self.logits[group - 1])
            sample_rows(logits, self.temperature, self.top_k, self.top_p, self.seed, self.offsets[:, group - 1],
                        round_scaled_to_input=False, out=self._token)
            last = group == s.groups - 1
            kernels.cp_codec_step(self._token, self.frames[:, group], self.codec_embedding[group - 1], self.codec_sum,
                                  proj_emb=None if last else self.projected_residual[group - 1], ln=self.ln_in[0],
                                  eps=s.eps, residual=self._residual, h=self._h)
        return self.frames

    def capture(self, warmup: int = 2) -> None:
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self.forward()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.forward()

    def replay(self) -> None:
        self.graph.replay()

    def step(self, past_hidden: torch.Tensor, layer0_token: torch.Tensor) -> torch.Tensor:
        """One frame from host inputs: pinned H2D of the talker hidden state
        and the layer-0 token, graph replay, D2H of the frame's codes."""

        if self._host_in is None:
            self._host_in = (torch.empty_like(self.past_hidden, device="cpu").pin_memory(),
                             torch.empty_like(self.layer0_token, device="cpu").pin_memory())
            self._host_frames = torch.empty_like(self.frames, device="cpu").pin_memory()
        h_hidden, h_token = self._host_in
        h_hidden.copy_(past_hidden)
        h_token.copy_(layer0_token)
        self.past_hidden.copy_(h_hidden, non_blocking=True)
        self.layer0_token.copy_(h_token, non_blocking=True)
        self.graph.replay()
        self._host_frames.copy_(self.frames, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self._host_frames

    def h2d_bytes(self) -> int:
        return self.past_hidden.numel() * self.past_hidden.element_size() + self.layer0_token.numel() * 8

    def d2h_bytes(self) -> int:
        return self.frames.numel() * 8

    def cpu_weights(self) -> dict:
        """The weights as CPU tensors, keyed like the attributes (for a CPU check)."""

        names = ("w_in", "b_in", "w_qkv", "w_o", "w_gate_up", "w_down", "ln_in", "ln_post", "q_norm", "k_norm",
                 "ln_final", "lm_head", "codec_embedding", "layer0_embedding")
        out = {}
        for n in names:
            v = getattr(self, n)
            out[n] = [t.cpu() for t in v] if isinstance(v, list) else v.cpu()
        return out

    def weight_bytes(self) -> int:
        tensors = [*self.w_qkv, *self.w_o, *self.w_gate_up, *self.w_down]
        return sum(t.numel() * t.element_size() for t in tensors)


__all__ = ["CodePredictorFrame", "CodePredictorShape"]
