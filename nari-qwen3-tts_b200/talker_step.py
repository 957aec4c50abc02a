"""One talker decode step of a continuously batched request set, end to end
on the device and captured as one CUDA graph.

The step mirrors the reference's captured decode op (executor/talker.py:477-492
with the layer loop of model/components.py:74-90):

    GPU planner: reserve pages, metadata, split-KV partition   (planner.py)
    input RMSNorm
    for each layer:
        QKV projection (cuBLAS)
        attend: QK RMSNorm + RoPE + paged K/V write, paged decode (talker_kv.py)
        O projection (cuBLAS), fused residual add + RMSNorm
        gate/up (cuBLAS), SiLU * up, down (cuBLAS), fused add + RMSNorm (next norm)
    codec head (cuBLAS), fused sampler with the seen-mask update, commit,
    RNG offsets += 512 (executor/talker.py:606)

There is no host round trip inside the step.  ``step()`` is the host-facing
call: it copies the step's inputs from pinned host memory, replays the
graph and returns the sampled tokens to the host.

Weights are random (bf16); GEMMs are plain library calls (torch -> cuBLAS).
The suppress-token mask of forward_logits (executor/talker.py:241-243) is
not applied.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import kernels
from .planner import DevicePagePlanner
from .sampling import sample_rows
from .talker_kv import B200TalkerBinding

FRAME_OFFSET_STRIDE = 512  # contract/rng.py: 16 codebooks x 32


@dataclass(frozen=True)
class TalkerShape:
    num_layers: int = 28
    hidden: int = 2048
    num_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 6144
    vocab: int = 3072
    rope_theta: float = 1.0e6
    eps: float = 1e-6


class _Norm:
    def __init__(self, weight: torch.Tensor, eps: float) -> None:
        self.weight = weight
        self.variance_epsilon = eps


class _AttentionParams:
    """What attend() reads from a layer's Attention module."""

    def __init__(self, q_weight, k_weight, eps, theta) -> None:
        self.q_norm = _Norm(q_weight, eps)
        self.k_norm = _Norm(k_weight, eps)
        self.rope_theta = theta


class TalkerDecodeStep:
    def __init__(
        self,
        *,
        shape: TalkerShape = TalkerShape(),
        batch: int = 64,
        total_pages: int = 32768,
        page_size: int = 16,
        max_pages_per_seq: int = 512,
        device: torch.device | str = "cuda",
        seed: int = 0,
        publish: bool = True,
    ) -> None:
        self.shape = s = shape
        # publish=False discards each step's reservation after the step, so every
        # step sees the same context lengths (a stationary benchmark workload)
        self.publish = publish
        self.batch = batch
        self.page_size = page_size
        self.device = dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)
        bf16 = torch.bfloat16

        def w(out_f, in_f):
            return (torch.randn(out_f, in_f, generator=g, device=dev) * in_f**-0.5).to(bf16)

        def norm_w(n):
            return (1.0 + 0.05 * torch.randn(n, generator=g, device=dev)).to(bf16)

        qkv_out = (s.num_heads + 2 * s.num_kv_heads) * s.head_dim
        self.w_qkv = [w(qkv_out, s.hidden) for _ in range(s.num_layers)]
        self.w_o = [w(s.hidden, s.num_heads * s.head_dim) for _ in range(s.num_layers)]
        self.w_gate_up = [w(2 * s.ffn, s.hidden) for _ in range(s.num_layers)]
        self.w_down = [w(s.hidden, s.ffn) for _ in range(s.num_layers)]
        self.ln_in = [norm_w(s.hidden) for _ in range(s.num_layers)]
        self.ln_post = [norm_w(s.hidden) for _ in range(s.num_layers)]
        self.ln_final = norm_w(s.hidden)
        self.w_head = w(s.vocab, s.hidden)
        self.attn = [_AttentionParams(norm_w(s.head_dim), norm_w(s.head_dim), s.eps, s.rope_theta)
                     for _ in range(s.num_layers)]

        # paged KV pool [layers, pages, 2, P, Hkv, D], filled with N(0, 1) data
        self.storage = torch.empty((s.num_layers, total_pages, 2, page_size, s.num_kv_heads, s.head_dim),
                                   dtype=bf16, device=dev)
        for layer in range(s.num_layers):
            self.storage[layer].normal_(generator=g)
        self.planner = DevicePagePlanner(total_pages=total_pages, page_size=page_size, slots=batch,
                                         max_pages_per_slot=max_pages_per_seq, scratch_page_count=batch,
                                         capture_rows=batch, token_capacity=batch, device=dev,
                                         num_qo_heads=s.num_heads, head_dim=s.head_dim)
        self.binding = B200TalkerBinding(storage=self.storage, capture_batch_size=batch, token_capacity=batch,
                                         num_qo_heads=s.num_heads, num_kv_heads=s.num_kv_heads, head_dim=s.head_dim,
                                         page_size=page_size, total_pages=total_pages, device=dev, dtype=bf16)
        # static step buffers (graph inputs and outputs)
        self.hidden_in = torch.zeros(batch, s.hidden, dtype=bf16, device=dev)
        self.temperature = torch.full((batch,), 0.9, device=dev)
        self.top_k = torch.full((batch,), 50, dtype=torch.int32, device=dev)
        self.top_p = torch.full((batch,), 0.95, device=dev)
        self.penalty = torch.full((batch,), 1.05, device=dev)
        self.seed = torch.arange(batch, dtype=torch.long, device=dev)
        self.offset = torch.zeros(batch, dtype=torch.long, device=dev)
        self.seen = torch.zeros(batch, s.vocab, dtype=torch.bool, device=dev)
        self.tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self._x = torch.empty(batch, s.hidden, dtype=bf16, device=dev)
        self._residual = torch.empty(batch, s.hidden, dtype=bf16, device=dev)
        self._act = torch.empty(batch, s.ffn, dtype=bf16, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.contexts: list[int] = []
        # pinned host staging for step()
        self._h_hidden = torch.empty(batch, s.hidden, dtype=bf16).pin_memory()
        self._h_tokens = torch.empty(batch, dtype=torch.long).pin_memory()

    # ---------------------------------------------------------------- requests
    def admit(self, contexts: list[int], *, scatter_seed: int = 0) -> None:
        """Admit len(contexts) requests whose KV already fills `contexts[i]`
        tokens, on pages scattered by a seeded permutation of the pool."""

        if len(contexts) != self.batch:
            raise ValueError("admit one context per batch row")
        P = self.page_size
        g = torch.Generator().manual_seed(scatter_seed)
        scratch = self.planner.scratch_pages.numel()
        perm = (torch.randperm(self.planner.total_pages - scratch, generator=g) + scratch).to(torch.int32)
        pos = 0
        slots = []
        for i, n in enumerate(contexts):
            pages = (n + P - 1) // P
            slot = self.planner.add_request(f"row{i}")
            self.planner.import_pages(slot, perm[pos: pos + pages], n)
            pos += pages
            slots.append(slot)
        self.planner.set_rows(slots, [1] * self.batch)
        self.contexts = list(contexts)
        # repetition-penalty history: 64 recent ids per row
        ids = torch.randint(0, self.shape.vocab, (self.batch, 64), generator=g)
        self.seen.zero_()
        self.seen.scatter_(1, ids.to(self.device), True)

    # ---------------------------------------------------------------- step body
    def forward(self) -> torch.Tensor:
        s = self.shape
        b = self.binding
        self.planner.plan(b, prefill=False)
        x, residual = self._x, self._residual
        residual.copy_(self.hidden_in)
        kernels.rmsnorm(self.hidden_in, self.ln_in[0], s.eps, out=x)
        hq, hkv, d = s.num_heads, s.num_kv_heads, s.head_dim
        rows = self.batch
        for layer in range(s.num_layers):
            b.select_layer(layer)
            qkv = F.linear(x, self.w_qkv[layer])
            q = qkv[:, : hq * d].view(rows, hq, d)
            k = qkv[:, hq * d: (hq + hkv) * d].view(rows, hkv, d)
            v = qkv[:, (hq + hkv) * d:].view(rows, hkv, d)
            attn = b.attend(self.attn[layer], q, k, v)
            o = F.linear(attn.view(rows, hq * d), self.w_o[layer])
            kernels.fused_add_rmsnorm_(o, residual, self.ln_post[layer], s.eps)
            gate_up = F.linear(o, self.w_gate_up[layer])
            kernels.silu_and_mul(gate_up, out=self._act)
            m = F.linear(self._act, self.w_down[layer])
            nxt = self.ln_final if layer + 1 == s.num_layers else self.ln_in[layer + 1]
            kernels.fused_add_rmsnorm_(m, residual, nxt, s.eps)
            x = m
        logits = F.linear(x, self.w_head)
        sample_rows(logits, self.temperature, self.top_k, self.top_p, self.seed, self.offset,
                    repetition_penalty=self.penalty, seen_token_mask=self.seen, update_seen=True,
                    round_scaled_to_input=False, out=self.tokens)
        self.planner.commit(self.publish)
        self.offset.add_(FRAME_OFFSET_STRIDE)
        return self.tokens

    def capture(self, warmup: int = 2) -> None:
        """Capture forward() into a CUDA graph (after eager warm-ups, like
        TorchCaptureDriver, executor/cuda_graph.py:59-77).  Warm-ups advance
        the request state like real steps."""

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

    def step(self, hidden: torch.Tensor) -> torch.Tensor:
        """Host-facing step: ``hidden`` [batch, hidden] bf16 host tensor in,
        sampled token ids (host int64 [batch]) out."""

        self._h_hidden.copy_(hidden)
        self.hidden_in.copy_(self._h_hidden, non_blocking=True)
        self.graph.replay()
        self._h_tokens.copy_(self.tokens, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self._h_tokens

    # ---------------------------------------------------------------- accounting
    def attention_bytes_per_layer(self) -> int:
        """Algorithmic HBM bytes of one decode-attention launch at the current
        lengths: K and V of every cached token plus the new one, q in, out."""

        s = self.shape
        kv = sum(n + 1 for n in self.contexts) * 2 * s.num_kv_heads * s.head_dim * 2
        qo = 2 * self.batch * s.num_heads * s.head_dim * 2
        return kv + qo

    def weight_bytes(self) -> int:
        tensors = [*self.w_qkv, *self.w_o, *self.w_gate_up, *self.w_down, self.w_head]
        return sum(t.numel() * t.element_size() for t in tensors)


__all__ = ["TalkerDecodeStep", "TalkerShape"]
