"""Device-side request control of a talker step (libnqt ``nqt_step_stage``,
``nqt_talker_logits_mask``, ``nqt_step_finish``).

The reference stages every row's sampling parameters from host rows into
device buffers before each replay (executor/talker.py:527-563), masks the
codec head's logits in forward_logits (executor/talker.py:170-183, 241-243)
and decides termination on the host by reading each sampled token
(engine/pipeline.py:583-609).  Here the per-request state is a slot table on
the device, written once when a request is admitted or its EOS rule changes;
a captured step gathers its rows' parameters, masks the logits and computes
terminal flags and the next step / RNG offset on the device.  The host reads
the tokens and terminal flags of a step with one device-to-host copy.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import call, ptr
from .kernels import device_status

EOS_NEVER = 2**31 - 1  # eos_from while EOS is suppressed indefinitely
TALKER_FRAME_OFFSET_STRIDE = 512  # contract/rng.py: 16 codebooks x 32


def eos_from(*, ignore_eos: bool, terminal_continuation: bool = False, input_finished: bool = True,
             token_count: int = 0) -> int:
    """First generation step at which EOS may end a request
    (engine/input_builder.py:60-70): never with ignore_eos or while a terminal
    continuation's input is unfinished; else max(2, token_count - 1) for a
    terminal continuation and 2 otherwise."""

    if ignore_eos:
        return EOS_NEVER
    if not terminal_continuation:
        return 2
    if not input_finished:
        return EOS_NEVER
    return max(2, token_count - 1)


@dataclass(frozen=True)
class RequestSampling:
    """One request's sampling parameters (executor/rows.py:16-53)."""

    temperature: float
    top_k: int
    top_p: float
    repetition_penalty: float
    seed: int
    offset: int = 0


class DeviceStepControl:
    """Slot table of request state plus the step's row buffers on one device."""

    def __init__(self, *, slots: int, rows: int, device: torch.device | str, vocab: int, codec_vocab: int,
                 eos_id: int) -> None:
        if not 0 <= codec_vocab <= vocab or eos_id >= vocab:
            raise ValueError("the code-predictor vocabulary and the EOS id must lie inside the talker vocabulary")
        dev = torch.device(device)
        self.device, self.slots, self.rows = dev, slots, rows
        self.vocab, self.codec_vocab, self.eos_id = vocab, codec_vocab, eos_id
        f32, i32, i64 = torch.float32, torch.int32, torch.long
        # slot table
        self.slot_temperature = torch.zeros(slots, dtype=f32, device=dev)
        self.slot_top_k = torch.ones(slots, dtype=i32, device=dev)
        self.slot_top_p = torch.ones(slots, dtype=f32, device=dev)
        self.slot_penalty = torch.ones(slots, dtype=f32, device=dev)
        self.slot_seed = torch.zeros(slots, dtype=i64, device=dev)
        self.slot_offset = torch.zeros(slots, dtype=i64, device=dev)
        self.slot_step = torch.zeros(slots, dtype=i32, device=dev)
        self.slot_max_tokens = torch.zeros(slots, dtype=i32, device=dev)
        self.slot_eos_from = torch.full((slots,), EOS_NEVER, dtype=i32, device=dev)
        # the step's rows: which slot each row serves, staged parameters, outputs
        self.row_slot = torch.full((rows,), -1, dtype=i32, device=dev)
        self.temperature = torch.zeros(rows, dtype=f32, device=dev)
        self.top_k = torch.ones(rows, dtype=i32, device=dev)
        self.top_p = torch.ones(rows, dtype=f32, device=dev)
        self.penalty = torch.ones(rows, dtype=f32, device=dev)
        self.seed = torch.zeros(rows, dtype=i64, device=dev)
        self.offset = torch.zeros(rows, dtype=i64, device=dev)
        self.suppress_eos = torch.ones(rows, dtype=torch.uint8, device=dev)
        self.terminal = torch.zeros(rows, dtype=torch.uint8, device=dev)
        self.n_terminal = torch.zeros(1, dtype=i32, device=dev)

    # ---------------------------------------------------------------- host side: admission
    def set_request(self, slot: int, sampling: RequestSampling, *, max_tokens: int, eos_from_step: int,
                    generation_step: int = 0) -> None:
        """Write one slot (at admission, or when its parameters change)."""

        if not 0 <= slot < self.slots:
            raise IndexError("request slot outside the table")
        self.slot_temperature[slot] = sampling.temperature
        self.slot_top_k[slot] = sampling.top_k
        self.slot_top_p[slot] = sampling.top_p
        self.slot_penalty[slot] = sampling.repetition_penalty
        self.slot_seed[slot] = sampling.seed
        self.slot_offset[slot] = sampling.offset
        self.slot_step[slot] = generation_step
        self.slot_max_tokens[slot] = max_tokens
        self.slot_eos_from[slot] = eos_from_step

    def set_eos_from(self, slot: int, eos_from_step: int) -> None:
        """A request's EOS rule changed (e.g. its streamed input finished)."""

        self.slot_eos_from[slot] = eos_from_step

    def set_rows(self, slots: list[int] | torch.Tensor) -> None:
        """Rows of the next steps (row r serves slots[r]; missing rows are padding)."""

        row_slot = torch.full((self.rows,), -1, dtype=torch.int32)
        s = torch.as_tensor(slots, dtype=torch.int32)
        row_slot[: s.numel()] = s
        self.row_slot.copy_(row_slot)

    # ---------------------------------------------------------------- device side: inside the step
    def stage(self) -> None:
        """Gather each row's sampling parameters and EOS-suppression flag."""

        dev = self.device
        call("nqt_step_stage", ptr(self.row_slot), self.rows, self.slots,
             ptr(self.slot_temperature), ptr(self.slot_top_k), ptr(self.slot_top_p), ptr(self.slot_penalty),
             ptr(self.slot_seed), ptr(self.slot_offset), ptr(self.slot_step), ptr(self.slot_eos_from),
             ptr(self.temperature), ptr(self.top_k), ptr(self.top_p), ptr(self.penalty), ptr(self.seed),
             ptr(self.offset), ptr(self.suppress_eos), ptr(device_status(dev)), _lib.stream_handle(dev))

    def mask_logits(self, logits: torch.Tensor) -> torch.Tensor:
        """The codec head's suppress mask, in place (forward_logits)."""

        if logits.ndim != 2 or logits.shape[0] != self.rows or logits.shape[1] != self.vocab or logits.stride(1) != 1:
            raise ValueError("logits must be [rows, vocab] with unit vocab stride")
        call("nqt_talker_logits_mask", ptr(logits), _lib.dtype_code(logits.dtype), logits.stride(0), self.rows,
             self.vocab, self.codec_vocab, self.eos_id, ptr(self.suppress_eos), _lib.stream_handle(logits.device))
        return logits

    def finish(self, tokens: torch.Tensor, *, offset_stride: int = TALKER_FRAME_OFFSET_STRIDE) -> torch.Tensor:
        """Terminal flags of the step's rows; advances each live row's step and RNG offset."""

        if tokens.dtype != torch.long or tokens.shape != (self.rows,) or not tokens.is_contiguous():
            raise ValueError("tokens must be contiguous int64 [rows]")
        dev = self.device
        call("nqt_step_finish", ptr(self.row_slot), self.rows, self.slots, ptr(tokens), self.eos_id,
             ptr(self.slot_step), ptr(self.slot_max_tokens), ptr(self.slot_eos_from), ptr(self.slot_offset),
             int(offset_stride), ptr(self.terminal), ptr(self.n_terminal), ptr(device_status(dev)),
             _lib.stream_handle(dev))
        return self.terminal


__all__ = ["DeviceStepControl", "EOS_NEVER", "RequestSampling", "TALKER_FRAME_OFFSET_STRIDE", "eos_from"]
