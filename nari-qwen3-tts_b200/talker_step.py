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
        gate/up (FP8 GEMM with SwiGLU fused, or cuBLAS + SiLU * up), down (cuBLAS),
        fused add + RMSNorm (next norm)
    codec head (cuBLAS), suppress mask, fused sampler with the seen-mask update,
    device completion rule (terminal flags, step and RNG offset += 512), commit

The rows' sampling parameters are gathered on the device from a per-request
slot table (step_control.py) at the start of the step instead of being staged
from the host (executor/talker.py:527-563), and termination is decided on the
device (engine/pipeline.py:583-609) instead of by a host read of each token.

There is no host round trip inside the step.  ``step()`` is the host-facing
call: it copies the step's inputs from pinned host memory, replays the
graph and returns the sampled tokens to the host.

Weights are random (bf16).  The decode step's gate/up projection takes the
reference's production FP8 path by default (``gate_up="fp8"``: 128 x 128 e4m3
weight blocks, the post-attention norm writing e4m3 activation blocks, the
block-scaled tcgen05 GEMM with SwiGLU fused); ``gate_up="bf16"`` keeps it in
bf16.  The mixed step defaults to bf16: its gate/up multiplies thousands of
prefill tokens, where the FP8 kernel (built to stream weights for decode-sized
batches) is slower than cuBLAS.  The other projections are library calls
(torch -> cuBLAS), as in the reference.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import kernels
from .planner import DevicePagePlanner
from .sampling import sample_rows
from .step_control import EOS_NEVER, DeviceStepControl, RequestSampling, eos_from
from .talker_kv import B200TalkerBinding, batch_decode_paged, batch_prefill_paged

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
    codec_vocab: int = 2048  # the code predictor's vocabulary: talker logits past it are suppressed
    eos_id: int = 2150       # codec EOS token (inside the suppressed range, kept live)
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


class TalkerWeights:
    """Random-init bf16 weights of the talker decoder (the shapes of
    model/components.py:60-90 and model/layers.py:273-294)."""

    def __init__(self, shape: TalkerShape, device: torch.device, generator: torch.Generator) -> None:
        s, g, dev, bf16 = shape, generator, device, torch.bfloat16

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

    def bytes(self) -> int:
        tensors = [*self.w_qkv, *self.w_o, *self.w_gate_up, *self.w_down, self.w_head]
        return sum(t.numel() * t.element_size() for t in tensors)


def _kv_pool(shape: TalkerShape, total_pages: int, page_size: int, device, generator) -> torch.Tensor:
    """Paged KV pool [layers, pages, 2, P, Hkv, D] filled with N(0, 1) data."""

    storage = torch.empty((shape.num_layers, total_pages, 2, page_size, shape.num_kv_heads, shape.head_dim),
                          dtype=torch.bfloat16, device=device)
    for layer in range(shape.num_layers):
        storage[layer].normal_(generator=generator)
    return storage


class GateUpFp8:
    """The reference's production gate/up for a step's rows (executor/build.py:73 requires it on every talker
    layer; model/layers.py:195-270): the weights quantised once into 128 x 128 e4m3 blocks, the post-attention
    add + RMSNorm writing e4m3 rows with per-128 scales, and the block-scaled tcgen05 GEMM with SwiGLU fused."""

    def __init__(self, weights: TalkerWeights, shape: TalkerShape, rows: int, device: torch.device) -> None:
        self.weights = [kernels.Fp8BlockWeight(w, gate_up=True) for w in weights.w_gate_up]
        self.q = torch.empty(rows, shape.hidden, dtype=torch.float8_e4m3fn, device=device)
        self.scale = torch.empty(shape.hidden // 128, rows, dtype=torch.float32, device=device)
        # the split-K workspace is made here, outside any graph capture
        self.workspace = kernels.fp8_gemm_workspace(device, rows, 2 * shape.ffn, shape.hidden)

    def bytes(self) -> int:
        return sum(w.data.numel() + w.scale.numel() * 4 for w in self.weights)


def _mlp_block(weights: TalkerWeights, shape: TalkerShape, layer: int, o: torch.Tensor, residual: torch.Tensor,
               act: torch.Tensor, fp8: GateUpFp8 | None = None) -> torch.Tensor:
    """residual += o; MLP(norm(residual)); residual += mlp; returns the next layer's normed input.  With ``fp8``
    the gate/up projection takes the reference's FP8 path."""

    if fp8 is None:
        kernels.fused_add_rmsnorm_(o, residual, weights.ln_post[layer], shape.eps)
        gate_up = F.linear(o, weights.w_gate_up[layer])
        kernels.silu_and_mul(gate_up, out=act)
    else:
        kernels.fused_add_rmsnorm_fp8_(o, residual, weights.ln_post[layer], shape.eps, fp8.q, fp8.scale)
        kernels.linear_fp8(fp8.q, fp8.scale, fp8.weights[layer], out=act, workspace=fp8.workspace)
    m = F.linear(act, weights.w_down[layer])
    nxt = weights.ln_final if layer + 1 == shape.num_layers else weights.ln_in[layer + 1]
    kernels.fused_add_rmsnorm_(m, residual, nxt, shape.eps)
    return m


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
        gate_up: str = "fp8",
    ) -> None:
        if gate_up not in ("fp8", "bf16"):
            raise ValueError("gate_up is 'fp8' (the reference's production path) or 'bf16'")
        self.shape = s = shape
        self.gate_up = gate_up
        # publish=False discards each step's reservation after the step, so every
        # step sees the same context lengths (a stationary benchmark workload)
        self.publish = publish
        self.batch = batch
        self.page_size = page_size
        self.device = dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(seed)
        bf16 = torch.bfloat16
        self.weights = TalkerWeights(s, dev, g)
        self.storage = _kv_pool(s, total_pages, page_size, dev, g)
        self.planner = DevicePagePlanner(total_pages=total_pages, page_size=page_size, slots=batch,
                                         max_pages_per_slot=max_pages_per_seq, scratch_page_count=batch,
                                         capture_rows=batch, token_capacity=batch, device=dev,
                                         num_qo_heads=s.num_heads, head_dim=s.head_dim)
        self.binding = B200TalkerBinding(storage=self.storage, capture_batch_size=batch, token_capacity=batch,
                                         num_qo_heads=s.num_heads, num_kv_heads=s.num_kv_heads, head_dim=s.head_dim,
                                         page_size=page_size, total_pages=total_pages, device=dev, dtype=bf16,
                                         mode="decode")
        # static step buffers (graph inputs and outputs)
        self.hidden_in = torch.zeros(batch, s.hidden, dtype=bf16, device=dev)
        # request state on the device: row i serves request slot i
        self.control = DeviceStepControl(slots=batch, rows=batch, device=dev, vocab=s.vocab,
                                         codec_vocab=s.codec_vocab, eos_id=s.eos_id)
        self.seen = torch.zeros(batch, s.vocab, dtype=torch.bool, device=dev)
        self.tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self._x = torch.empty(batch, s.hidden, dtype=bf16, device=dev)
        self._residual = torch.empty(batch, s.hidden, dtype=bf16, device=dev)
        self._act = torch.empty(batch, s.ffn, dtype=bf16, device=dev)
        self.fp8 = GateUpFp8(self.weights, s, batch, dev) if gate_up == "fp8" else None
        self.graph: torch.cuda.CUDAGraph | None = None
        self.contexts: list[int] = []
        # parity hook: Exp(1) noise [batch, vocab] for the sampler's noise entry instead of the Philox draw
        self.sample_noise: torch.Tensor | None = None
        # pinned host staging for step()
        self._h_hidden = torch.empty(batch, s.hidden, dtype=bf16).pin_memory()
        self._h_tokens = torch.empty(batch, dtype=torch.long).pin_memory()
        self._h_terminal = torch.empty(batch, dtype=torch.uint8).pin_memory()

    # ---------------------------------------------------------------- requests
    # the rows' staged sampling parameters (written by the step itself)
    temperature = property(lambda self: self.control.temperature)
    top_k = property(lambda self: self.control.top_k)
    top_p = property(lambda self: self.control.top_p)
    penalty = property(lambda self: self.control.penalty)
    seed = property(lambda self: self.control.seed)
    offset = property(lambda self: self.control.offset)
    terminal = property(lambda self: self.control.terminal)

    def admit(self, contexts: list[int], *, scatter_seed: int = 0, sampling: RequestSampling | None = None,
              max_tokens: int = EOS_NEVER, ignore_eos: bool = False) -> None:
        """Admit len(contexts) requests whose KV already fills `contexts[i]`
        tokens, on pages scattered by a seeded permutation of the pool.  Every
        request gets ``sampling`` (default T 0.9, top-k 50, top-p 0.95,
        penalty 1.05, seed = row, offset 0) and the completion limits."""

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
        for i in range(self.batch):
            req = sampling or RequestSampling(temperature=0.9, top_k=50, top_p=0.95, repetition_penalty=1.05, seed=i)
            self.control.set_request(i, req, max_tokens=max_tokens, eos_from_step=eos_from(ignore_eos=ignore_eos))
        self.control.set_rows(list(range(self.batch)))
        # repetition-penalty history: 64 recent ids per row
        ids = torch.randint(0, self.shape.vocab, (self.batch, 64), generator=g)
        self.seen.zero_()
        self.seen.scatter_(1, ids.to(self.device), True)

    # ---------------------------------------------------------------- step body
    def _mlp_rows(self) -> tuple:
        """The layer's FP8 MLP input (e4m3 rows, scales) for a parity trace; empty on the bf16 path."""

        return () if self.fp8 is None else (self.fp8.q.clone(), self.fp8.scale.clone())

    def forward(self, trace: list | None = None) -> torch.Tensor:
        """The step body (what capture() records).  ``trace``, for parity
        tests of an eager step: receives (normed input, residual) before the
        first layer and after every layer - plus, on the FP8 path, the layer's
        e4m3 MLP input rows and their scales - then the logits."""

        s = self.shape
        b = self.binding
        ctl = self.control
        ctl.stage()
        self.planner.plan(b, prefill=False)
        x, residual = self._x, self._residual
        w = self.weights
        residual.copy_(self.hidden_in)
        kernels.rmsnorm(self.hidden_in, w.ln_in[0], s.eps, out=x)
        hq, hkv, d = s.num_heads, s.num_kv_heads, s.head_dim
        rows = self.batch
        if trace is not None:
            trace.append((x.clone(), residual.clone()))
        for layer in range(s.num_layers):
            b.select_layer(layer)
            qkv = F.linear(x, w.w_qkv[layer])
            q = qkv[:, : hq * d].view(rows, hq, d)
            k = qkv[:, hq * d: (hq + hkv) * d].view(rows, hkv, d)
            v = qkv[:, (hq + hkv) * d:].view(rows, hkv, d)
            attn = b.attend(w.attn[layer], q, k, v)
            o = F.linear(attn.view(rows, hq * d), w.w_o[layer])
            x = _mlp_block(w, s, layer, o, residual, self._act, self.fp8)
            if trace is not None:
                trace.append((x.clone(), residual.clone()) + self._mlp_rows())
        self.last_hidden = x  # the final normed hidden state (the code predictor's input)
        logits = ctl.mask_logits(F.linear(x, w.w_head))
        if trace is not None:
            trace.append(logits.clone())
        sample_rows(logits, ctl.temperature, ctl.top_k, ctl.top_p, ctl.seed, ctl.offset,
                    repetition_penalty=ctl.penalty, seen_token_mask=self.seen, update_seen=True,
                    round_scaled_to_input=False, noise=self.sample_noise, out=self.tokens)
        ctl.finish(self.tokens, offset_stride=FRAME_OFFSET_STRIDE)
        self.planner.commit(self.publish)
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

    def step(self, hidden: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Host-facing step: ``hidden`` [batch, hidden] bf16 host tensor in;
        sampled token ids (host int64 [batch]) and terminal flags (host uint8
        [batch], the device completion rule) out."""

        self._h_hidden.copy_(hidden)
        self.hidden_in.copy_(self._h_hidden, non_blocking=True)
        self.graph.replay()
        self._h_tokens.copy_(self.tokens, non_blocking=True)
        self._h_terminal.copy_(self.control.terminal, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return self._h_tokens, self._h_terminal

    def d2h_bytes(self) -> int:
        return self.batch * (8 + 1)

    # ---------------------------------------------------------------- accounting
    def attention_bytes_per_layer(self) -> int:
        """Algorithmic HBM bytes of one decode-attention launch at the current
        lengths: K and V of every cached token plus the new one, q in, out."""

        s = self.shape
        kv = sum(n + 1 for n in self.contexts) * 2 * s.num_kv_heads * s.head_dim * 2
        qo = 2 * self.batch * s.num_heads * s.head_dim * 2
        return kv + qo

    def weight_bytes(self) -> int:
        """Weight bytes one step streams (the FP8 gate/up in place of its bf16 copy)."""

        total = self.weights.bytes()
        if self.fp8 is not None:
            total += self.fp8.bytes() - sum(w.numel() * w.element_size() for w in self.weights.w_gate_up)
        return total


class TalkerMixedStep:
    """One step of a mixed continuous batch: chunked
    prefills and decode rows in the same step, one CUDA graph.

    Rows [0, n_prefill) are prefill chunks (their tokens first in the packed
    token order), rows [n_prefill, n_prefill + n_decode) decode one token each.
    Each step: the GPU planner plans both groups (two views of one page pool),
    every layer runs one QKV GEMM over all tokens, QK-norm/RoPE + KV write for
    both groups, the tcgen05 causal prefill for the chunks and the split-KV
    decode for the decode rows, then the shared O projection and MLP; the last
    token of each chunk and every decode row are sampled.  Then ``churn_rows``
    decode requests finish and are replaced on the device: their pages are
    released and new requests of the same lengths are admitted through the
    planner's allocation path (lowest free pages first).  Reservations of the
    step itself are discarded, so the workload is stationary.
    """

    def __init__(self, *, shape: TalkerShape = TalkerShape(), chunks: list[int], decode_contexts: list[int],
                 churn_rows: int = 24, total_pages: int, page_size: int = 16, device: torch.device | str = "cuda",
                 seed: int = 0, gate_up: str = "bf16") -> None:
        if gate_up not in ("fp8", "bf16"):
            raise ValueError("gate_up is 'fp8' (the reference's production path) or 'bf16'")
        self.shape = s = shape
        self.gate_up = gate_up
        self.device = dev = torch.device(device)
        self.page_size = P = page_size
        self.chunks = list(chunks)
        self.decode_contexts = list(decode_contexts)
        self.n_pre, self.n_dec = len(chunks), len(decode_contexts)
        self.rows = self.n_pre + self.n_dec
        self.t_pre = sum(chunks)
        self.tokens = self.t_pre + self.n_dec
        self.churn_rows = churn_rows
        g = torch.Generator(device=dev).manual_seed(seed)
        self.weights = TalkerWeights(s, dev, g)
        self.storage = _kv_pool(s, total_pages, page_size, dev, g)
        max_len = max(max(chunks), max(decode_contexts)) + 1
        # scratch pages: the largest prefill chunk set or the decode rows (executor/build.py:40-54)
        scratch = max((self.t_pre + P - 1) // P, self.n_dec, churn_rows)
        self.dec = DevicePagePlanner(total_pages=total_pages, page_size=P, slots=self.rows,
                                     max_pages_per_slot=(max_len + P - 1) // P + 1, scratch_page_count=scratch,
                                     capture_rows=self.n_dec, token_capacity=self.n_dec, device=dev,
                                     num_qo_heads=s.num_heads, head_dim=s.head_dim)
        self.pre = self.dec.view(capture_rows=self.n_pre, token_capacity=self.t_pre)
        self.adm = self.dec.view(capture_rows=churn_rows, token_capacity=0)
        common = dict(storage=self.storage, num_qo_heads=s.num_heads, num_kv_heads=s.num_kv_heads,
                      head_dim=s.head_dim, page_size=P, total_pages=total_pages, device=dev, dtype=torch.bfloat16)
        self.pre_b = B200TalkerBinding(capture_batch_size=self.n_pre, token_capacity=self.t_pre, mode="prefill",
                                       **common)
        self.dec_b = B200TalkerBinding(capture_batch_size=self.n_dec, token_capacity=self.n_dec, mode="decode",
                                       **common)
        # allocation-only metadata sink of the admission step
        self._adm_indptr = torch.zeros(churn_rows + 1, dtype=torch.int32, device=dev)
        self._adm_indices = torch.zeros(total_pages + churn_rows, dtype=torch.int32, device=dev)
        self._adm_last = torch.zeros(churn_rows, dtype=torch.int32, device=dev)
        self._churn_base = torch.zeros(1, dtype=torch.long, device=dev)
        self._churn_range = torch.arange(churn_rows, dtype=torch.long, device=dev)
        self._replacement_len = torch.tensor(decode_contexts, dtype=torch.int32, device=dev)
        bf16 = torch.bfloat16
        self.hidden_in = torch.zeros(self.tokens, s.hidden, dtype=bf16, device=dev)
        self._x = torch.empty(self.tokens, s.hidden, dtype=bf16, device=dev)
        self._residual = torch.empty(self.tokens, s.hidden, dtype=bf16, device=dev)
        self._attn = torch.empty(self.tokens, s.num_heads * s.head_dim, dtype=bf16, device=dev)
        self._act = torch.empty(self.tokens, s.ffn, dtype=bf16, device=dev)
        self.fp8 = GateUpFp8(self.weights, s, self.tokens, dev) if gate_up == "fp8" else None
        ends = torch.tensor(chunks).cumsum(0) - 1
        self._sample_rows = torch.cat([ends, self.t_pre + torch.arange(self.n_dec)]).to(dev)
        n = self.rows
        # request state on the device: row i serves request slot i
        self.control = DeviceStepControl(slots=n, rows=n, device=dev, vocab=s.vocab, codec_vocab=s.codec_vocab,
                                         eos_id=s.eos_id)
        self.seen = torch.zeros(n, s.vocab, dtype=torch.bool, device=dev)
        self.out_tokens = torch.zeros(n, dtype=torch.long, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        # parity hook: Exp(1) noise [rows, vocab] for the sampler's noise entry instead of the Philox draw
        self.sample_noise: torch.Tensor | None = None

    temperature = property(lambda self: self.control.temperature)
    top_k = property(lambda self: self.control.top_k)
    top_p = property(lambda self: self.control.top_p)
    penalty = property(lambda self: self.control.penalty)
    seed = property(lambda self: self.control.seed)
    offset = property(lambda self: self.control.offset)
    terminal = property(lambda self: self.control.terminal)

    def admit(self, *, scatter_seed: int = 0) -> None:
        """Prefill rows start empty; decode rows get their contexts on scattered pages.  Every row samples
        with T 0.9, top-k 50, top-p 0.95, penalty 1.05; prefill rows never terminate (their completion is
        not a decode step, engine/pipeline.py:583-593), decode rows end on EOS."""

        P = self.page_size
        gen = torch.Generator().manual_seed(scatter_seed)
        scratch = self.dec.scratch_pages.numel()
        perm = (torch.randperm(self.dec.total_pages - scratch, generator=gen) + scratch).to(torch.int32)
        pre_slots = [self.dec.add_request(f"prefill{i}") for i in range(self.n_pre)]
        dec_slots, pos = [], 0
        for i, n in enumerate(self.decode_contexts):
            slot = self.dec.add_request(f"decode{i}")
            pages = (n + P - 1) // P
            self.dec.import_pages(slot, perm[pos: pos + pages], n)
            pos += pages
            dec_slots.append(slot)
        self.pre.set_rows(pre_slots, self.chunks)
        self.dec.set_rows(dec_slots, [1] * self.n_dec)
        for i in range(self.rows):
            prefill = i < self.n_pre
            self.control.set_request(i, RequestSampling(0.9, 50, 0.95, 1.05, seed=i), max_tokens=EOS_NEVER,
                                     eos_from_step=EOS_NEVER if prefill else eos_from(ignore_eos=False))
        self.control.set_rows(list(range(self.rows)))
        ids = torch.randint(0, self.shape.vocab, (self.rows, 64), generator=gen)
        self.seen.zero_()
        self.seen.scatter_(1, ids.to(self.device), True)

    _mlp_rows = TalkerDecodeStep._mlp_rows

    def forward(self, trace: list | None = None) -> torch.Tensor:
        """The step body; ``trace`` as in TalkerDecodeStep.forward (over all
        packed tokens, prefill chunks first)."""

        s, w = self.shape, self.weights
        hq, hkv, d = s.num_heads, s.num_kv_heads, s.head_dim
        tp, nd, T = self.t_pre, self.n_dec, self.tokens
        ctl = self.control
        ctl.stage()
        self.pre.plan(self.pre_b, prefill=True)
        self.dec.plan(self.dec_b, prefill=False)
        x, residual = self._x, self._residual
        residual.copy_(self.hidden_in)
        kernels.rmsnorm(self.hidden_in, w.ln_in[0], s.eps, out=x)
        if trace is not None:
            trace.append((x.clone(), residual.clone()))
        for layer in range(s.num_layers):
            cache = self.storage[layer]
            qkv = F.linear(x, w.w_qkv[layer])
            q = qkv[:, : hq * d].view(T, hq, d)
            k = qkv[:, hq * d: (hq + hkv) * d].view(T, hkv, d)
            v = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
            a = w.attn[layer]
            for b, lo, hi in ((self.pre_b, 0, tp), (self.dec_b, tp, T)):
                kernels.paired_qk_norm_rope_paged_cache_(
                    q[lo:hi], k[lo:hi], v[lo:hi], a.q_norm.weight, a.k_norm.weight, b.position_ids, s.eps,
                    s.rope_theta, cache, b.write_pages, b.write_offsets)
            attn = self._attn.view(T, hq, d)
            batch_prefill_paged(q[:tp], cache, self.pre_b.qo_indptr, self.pre_b.paged_kv_indptr,
                                self.pre_b.paged_kv_indices, self.pre_b.paged_kv_last_page_len, batch=self.n_pre,
                                out=attn[:tp])
            batch_decode_paged(q[tp:], cache, self.dec_b.paged_kv_indptr, self.dec_b.paged_kv_indices,
                               self.dec_b.paged_kv_last_page_len, self.dec_b.decode_workspace, batch_capacity=nd,
                               out=attn[tp:], plan=False)
            o = F.linear(self._attn, w.w_o[layer])
            x = _mlp_block(w, s, layer, o, residual, self._act, self.fp8)
            if trace is not None:
                trace.append((x.clone(), residual.clone()) + self._mlp_rows())
        logits = ctl.mask_logits(F.linear(x.index_select(0, self._sample_rows), w.w_head))
        if trace is not None:
            trace.append(logits.clone())
        sample_rows(logits, ctl.temperature, ctl.top_k, ctl.top_p, ctl.seed, ctl.offset,
                    repetition_penalty=ctl.penalty, seen_token_mask=self.seen, update_seen=True,
                    round_scaled_to_input=False, noise=self.sample_noise, out=self.out_tokens)
        ctl.finish(self.out_tokens, offset_stride=FRAME_OFFSET_STRIDE)
        self.pre.commit(False)
        self.dec.commit(False)
        # churn: churn_rows decode requests finish and new ones of the same lengths are admitted
        slots = (self._churn_base + self._churn_range) % nd
        self.adm.row_slot.copy_(slots + self.n_pre)
        self.adm.row_advance.copy_(self._replacement_len.index_select(0, slots))
        self.adm.release_rows()
        self.adm.plan_into(qo_indptr=None, kv_indptr=self._adm_indptr, kv_indices=self._adm_indices,
                           last_page_len=self._adm_last, position_ids=None, write_pages=None, write_offsets=None,
                           prefill=True)
        self.adm.commit(True)
        self._churn_base.add_(self.churn_rows)
        return self.out_tokens

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

    def prefill_flops_per_layer(self) -> int:
        """Causal prefill FLOPs of one layer: 2 (QK^T, PV) x 2 x Hq x D per visible (query, key) pair."""

        s = self.shape
        pairs = sum(n * (n + 1) // 2 for n in self.chunks)
        return 4 * s.num_heads * s.head_dim * pairs

    def decode_bytes_per_layer(self) -> int:
        s = self.shape
        return sum(n + 1 for n in self.decode_contexts) * 2 * s.num_kv_heads * s.head_dim * 2


__all__ = ["TalkerDecodeStep", "TalkerMixedStep", "TalkerShape", "TalkerWeights"]
