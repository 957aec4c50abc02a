"""CPU restatement of the talker step's request control (test infrastructure
only; the product never imports it).

* staging - TalkerExecutor._stage_sampling_rows (executor/talker.py:527-563):
  row r takes its request's temperature, top_k, top_p, repetition_penalty,
  seed and offset; padding rows take 0, 1, 1.0, 1.0, 0, 0;
* EOS suppression - the input builder's _suppress_decode_eos
  (engine/input_builder.py:60-70): suppressed with ignore_eos, before step 2,
  and for a terminal continuation while its input is unfinished or before
  step token_count - 1;
* logits mask - forward_logits (executor/talker.py:170-183, 241-243):
  columns >= the code-predictor vocabulary are -inf except EOS, and EOS is
  -inf on suppressed rows;
* completion - SynthesisPipeline (engine/pipeline.py:583-609), decode steps:
  reached_limit = step + 1 >= effective_max_output_tokens; eos = token ==
  codec_eos_token_id unless suppressed, ignore_eos or reached_limit;
  terminal = eos or reached_limit; the next sampling offset is offset + 512.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class RequestState:
    temperature: float
    top_k: int
    top_p: float
    repetition_penalty: float
    seed: int
    offset: int
    generation_step: int
    max_output_tokens: int
    ignore_eos: bool = False
    terminal_continuation: bool = False
    input_finished: bool = True
    token_count: int = 0


def suppress_decode_eos(s: RequestState) -> bool:
    if s.ignore_eos:
        return True
    if s.generation_step < 2:
        return True
    if not s.terminal_continuation:
        return False
    return not s.input_finished or s.generation_step < s.token_count - 1


def stage(rows: list[RequestState | None]) -> dict:
    out = {"temperature": [], "top_k": [], "top_p": [], "penalty": [], "seed": [], "offset": [], "suppress": []}
    for s in rows:
        if s is None:
            vals = (0.0, 1, 1.0, 1.0, 0, 0, True)
        else:
            vals = (s.temperature, s.top_k, s.top_p, s.repetition_penalty, s.seed, s.offset, suppress_decode_eos(s))
        for key, v in zip(out, vals, strict=True):
            out[key].append(v)
    return out


def mask_logits(logits: torch.Tensor, codec_vocab: int, eos_id: int, suppress: list[bool]) -> torch.Tensor:
    out = logits.clone()
    mask = torch.zeros(logits.shape[1], dtype=torch.bool)
    mask[codec_vocab:] = True
    if eos_id >= 0:
        mask[eos_id] = False
    out = out.masked_fill(mask.unsqueeze(0), -torch.inf)
    if eos_id >= 0:
        out[:, eos_id] = out[:, eos_id].masked_fill(torch.tensor(suppress), -torch.inf)
    return out


def finish(rows: list[RequestState | None], tokens: list[int], eos_id: int) -> list[bool]:
    terminal = []
    for s, token in zip(rows, tokens, strict=True):
        if s is None:
            terminal.append(False)
            continue
        reached_limit = s.generation_step + 1 >= s.max_output_tokens
        eos = False
        if not suppress_decode_eos(s) and not s.ignore_eos and not reached_limit:
            eos = int(token) == eos_id
        terminal.append(eos or reached_limit)
        s.generation_step += 1
        s.offset += 512
    return terminal
