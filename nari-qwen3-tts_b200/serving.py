"""Box-level serving simulation of one GPU: a continuously
batched talker + code-predictor worker built from this path's parts.

Per step the worker admits the requests that have arrived (one captured
prefill per request: the GPU planner reserves its pages, the causal prefill
attention writes its KV, the request joins the decode rows), replays the
captured talker decode step over its 64 request slots (GPU planner, paged
decode attention, fused sampler, device request control) and the captured
code-predictor frame for the same rows, and feeds each frame's codec
embedding sum back as the next talker input.  A request's audio length is its
``max_tokens`` in the device request table, so the device completion rule
(engine/pipeline.py:583-609) ends it; the host only reads the step's terminal
flags (one device-to-host copy per step).

This is a measurement harness of the path, not the reference's engine: there
is no text frontend, codec decoder or network I/O.  Time is wall-clock on the
host with the GPU work of each step synchronised, so the reported
time-to-first-frame includes queueing behind the running step.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from . import kernels
from .code_predictor import CodePredictorFrame
from .sampling import sample_rows
from .step_control import EOS_NEVER, RequestSampling
from .talker_kv import B200TalkerBinding
from .talker_step import TalkerDecodeStep, TalkerShape, _mlp_block

FRAMES_PER_SECOND = 12


@dataclass
class Request:
    rid: int
    arrival: float          # seconds after the worker's start
    text_tokens: int        # prefill length
    frames: int             # audio frames to emit
    slot: int = -1
    first_frame: float = math.nan
    done: float = math.nan
    emitted: int = 0


def poisson_requests(*, rate: float, horizon: float, seed: int, rank: int = 0, world: int = 1,
                     text_range=(20, 200), audio_seconds=(2.0, 20.0)) -> list[Request]:
    """The box's arrival stream (Poisson, ``rate`` requests/s per GPU, seeded) routed round-robin: rank r
    serves requests r, r + world, ...  Text lengths and audio durations are uniform."""

    g = torch.Generator().manual_seed(seed)
    t, out, i = 0.0, [], 0
    total_rate = rate * world
    while True:
        t += float(torch.empty(1).exponential_(total_rate, generator=g))
        if t >= horizon:
            break
        text = int(torch.randint(text_range[0], text_range[1] + 1, (1,), generator=g))
        secs = float(torch.empty(1).uniform_(audio_seconds[0], audio_seconds[1], generator=g))
        if i % world == rank:
            out.append(Request(rid=i, arrival=t, text_tokens=text, frames=max(1, round(secs * FRAMES_PER_SECOND))))
        i += 1
    return out


class TalkerPrefill:
    """One request's chunked prefill (up to ``tokens`` tokens) over a decode step's weights, KV pool and
    request slots, captured as one CUDA graph; the first token is drawn from the last position."""

    def __init__(self, step: TalkerDecodeStep, tokens: int = 256) -> None:
        s, dev = step.shape, step.device
        self.step, self.tokens = step, tokens
        self.planner = step.planner.view(capture_rows=1, token_capacity=tokens)
        self.binding = B200TalkerBinding(storage=step.storage, capture_batch_size=1, token_capacity=tokens,
                                         num_qo_heads=s.num_heads, num_kv_heads=s.num_kv_heads, head_dim=s.head_dim,
                                         page_size=step.page_size, total_pages=step.planner.total_pages, device=dev,
                                         dtype=torch.bfloat16, mode="prefill")
        bf16 = torch.bfloat16
        self.hidden_in = torch.zeros(tokens, s.hidden, dtype=bf16, device=dev)
        self._x = torch.empty(tokens, s.hidden, dtype=bf16, device=dev)
        self._residual = torch.empty(tokens, s.hidden, dtype=bf16, device=dev)
        self._act = torch.empty(tokens, s.ffn, dtype=bf16, device=dev)
        self.last_index = torch.zeros(1, dtype=torch.long, device=dev)
        self.temperature = torch.full((1,), 0.9, device=dev)
        self.top_k = torch.full((1,), 50, dtype=torch.int32, device=dev)
        self.top_p = torch.full((1,), 0.95, device=dev)
        self.seed = torch.zeros(1, dtype=torch.long, device=dev)
        self.offset = torch.zeros(1, dtype=torch.long, device=dev)
        self.token = torch.zeros(1, dtype=torch.long, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None

    def forward(self) -> torch.Tensor:
        s, w, b = self.step.shape, self.step.weights, self.binding
        hq, hkv, d, T = s.num_heads, s.num_kv_heads, s.head_dim, self.tokens
        self.planner.plan(b, prefill=True)
        residual = self._residual
        residual.copy_(self.hidden_in)
        x = kernels.rmsnorm(self.hidden_in, w.ln_in[0], s.eps, out=self._x)
        for layer in range(s.num_layers):
            b.select_layer(layer)
            qkv = F.linear(x, w.w_qkv[layer])
            attn = b.attend(w.attn[layer], qkv[:, : hq * d].view(T, hq, d), qkv[:, hq * d: (hq + hkv) * d].view(T, hkv, d),
                            qkv[:, (hq + hkv) * d:].view(T, hkv, d))
            o = F.linear(attn.view(T, hq * d), w.w_o[layer])
            x = _mlp_block(w, s, layer, o, residual, self._act)
        logits = F.linear(x.index_select(0, self.last_index), w.w_head)
        sample_rows(logits, self.temperature, self.top_k, self.top_p, self.seed, self.offset,
                    round_scaled_to_input=False, out=self.token)
        self.planner.commit(True)
        return self.token

    def capture(self) -> None:
        stream = torch.cuda.Stream(self.step.device)
        stream.wait_stream(torch.cuda.current_stream(self.step.device))
        # warm-ups on a throw-away request in slot 0's place: plan and discard
        with torch.cuda.stream(stream):
            self.planner.set_rows([-1], [0])
            self.forward()
        torch.cuda.current_stream(self.step.device).wait_stream(stream)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.forward()

    def run(self, slot: int, length: int, seed: int) -> None:
        if not 0 < length <= self.tokens:
            raise ValueError("prefill length outside the captured capacity")
        self.planner.set_rows([slot], [length])
        self.last_index.fill_(length - 1)
        self.seed.fill_(seed)
        self.graph.replay()


@dataclass
class WorkerReport:
    frames: int = 0
    steps: int = 0
    finished: int = 0
    admitted: int = 0
    elapsed: float = 0.0
    ttff: list = field(default_factory=list)
    busy_rows: list = field(default_factory=list)


class ServingWorker:
    """One GPU of the box: ``slots`` concurrent requests (the captured decode batch)."""

    def __init__(self, *, shape: TalkerShape = TalkerShape(), slots: int = 64, pool_tokens: int = 128 * 1024,
                 prefill_tokens: int = 256, device: torch.device | str = "cuda", seed: int = 0) -> None:
        dev = torch.device(device)
        self.device, self.slots = dev, slots
        page = 16
        self.step = TalkerDecodeStep(shape=shape, batch=slots, total_pages=pool_tokens // page, page_size=page,
                                     max_pages_per_seq=(prefill_tokens + 20 * FRAMES_PER_SECOND + 2 * page) // page + 1,
                                     device=dev, seed=seed, publish=True)
        self.prefill = TalkerPrefill(self.step, prefill_tokens)
        self.cp = CodePredictorFrame(rows=slots, device=dev, seed=seed + 1)
        self.active: dict[int, Request] = {}   # slot -> request
        self.rid_of_slot: dict[int, str] = {}
        self.frame_index = 0

    def _rows(self) -> list[int]:
        return [slot if slot in self.active else -1 for slot in range(self.slots)]

    def capture(self) -> None:
        st = self.step
        st.control.set_rows([-1] * self.slots)
        st.planner.set_rows([-1] * self.slots, [0] * self.slots)
        st.capture(warmup=1)
        self.prefill.capture()
        self.cp.capture(warmup=1)

    def _admit(self, req: Request, t_now: float) -> None:
        st = self.step
        rid = f"req{req.rid}"
        slot = st.planner.add_request(rid)
        req.slot = slot
        self.rid_of_slot[slot] = rid
        self.prefill.run(slot, req.text_tokens, seed=req.rid)
        st.control.set_request(slot, RequestSampling(0.9, 50, 0.95, 1.05, seed=req.rid),
                               max_tokens=req.frames, eos_from_step=EOS_NEVER)
        st.seen[slot].zero_()
        self.active[slot] = req

    def _retire(self, slot: int, t_now: float) -> None:
        req = self.active.pop(slot)
        req.done = t_now
        self.step.planner.remove_request(self.rid_of_slot.pop(slot))

    def run(self, requests: list[Request], *, horizon: float) -> WorkerReport:
        """Serve ``requests`` (arrival times relative to the start) until every one admitted before
        ``horizon`` has finished.  Returns frames, steps and time-to-first-frame per request."""

        st, cp, rep = self.step, self.cp, WorkerReport()
        pending = sorted(requests, key=lambda r: r.arrival)
        queue: list[Request] = []
        h_terminal = torch.empty(self.slots, dtype=torch.uint8).pin_memory()
        t0 = time.perf_counter()
        while True:
            now = time.perf_counter() - t0
            while pending and pending[0].arrival <= now:
                queue.append(pending.pop(0))
            while queue and len(self.active) < self.slots:
                self._admit(queue.pop(0), now)
                rep.admitted += 1
            if not self.active:
                if not pending and not queue:
                    break
                if pending:
                    time.sleep(max(0.0, min(pending[0].arrival - now, 0.001)))
                continue
            rows = self._rows()
            st.control.set_rows(rows)
            st.planner.set_rows(rows, [1 if s >= 0 else 0 for s in rows])
            st.replay()
            cp.past_hidden.copy_(st.last_hidden)
            cp.layer0_token.copy_(st.tokens)
            cp.set_frame(self.frame_index)
            cp.replay()
            st.hidden_in.copy_(cp.codec_sum)
            h_terminal.copy_(st.control.terminal, non_blocking=True)
            torch.cuda.current_stream(self.device).synchronize()
            now = time.perf_counter() - t0
            self.frame_index += 1
            rep.steps += 1
            rep.busy_rows.append(len(self.active))
            for slot in list(self.active):
                req = self.active[slot]
                req.emitted += 1
                rep.frames += 1
                if req.emitted == 1:
                    req.first_frame = now
                    rep.ttff.append(now - req.arrival)
                if h_terminal[slot]:
                    self._retire(slot, now)
                    rep.finished += 1
        rep.elapsed = time.perf_counter() - t0
        return rep


__all__ = ["Request", "ServingWorker", "TalkerPrefill", "WorkerReport", "poisson_requests"]
