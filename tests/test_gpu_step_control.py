"""GPU parity of the device-side request control (csrc/step_control.cu)
against the CPU restatement of the reference's staging, EOS-suppression,
logits-mask and completion rules (oracle/step_control.py): staged parameters,
masked logits and terminal flags exact, slot state advanced like the host's."""

from __future__ import annotations

import random
from importlib import import_module

import pytest
import torch

from oracle import step_control as octl

pytestmark = pytest.mark.gpu


def _random_states(n, rng):
    states = []
    for i in range(n):
        states.append(octl.RequestState(
            temperature=rng.choice([0.0, 0.9, 1.3]), top_k=rng.choice([0, 1, 50, 80]), top_p=rng.choice([0.8, 1.0]),
            repetition_penalty=rng.choice([1.0, 1.05]), seed=rng.randrange(2**62), offset=rng.randrange(2**40) * 32,
            generation_step=rng.randrange(0, 12), max_output_tokens=rng.randrange(1, 14),
            ignore_eos=rng.random() < 0.15, terminal_continuation=rng.random() < 0.4,
            input_finished=rng.random() < 0.6, token_count=rng.randrange(0, 10)))
    return states


def test_stage_mask_finish_match_the_reference_rules(nqt, cuda):
    sc = import_module("nari-qwen3-tts_b200.step_control")
    rng = random.Random(3)
    slots, rows, vocab, codec_vocab, eos_id = 40, 32, 3072, 2048, 2150
    states = _random_states(slots, rng)
    ctl = sc.DeviceStepControl(slots=slots, rows=rows, device=cuda, vocab=vocab, codec_vocab=codec_vocab,
                               eos_id=eos_id)
    for i, s in enumerate(states):
        ctl.set_request(i, sc.RequestSampling(s.temperature, s.top_k, s.top_p, s.repetition_penalty, s.seed,
                                              s.offset),
                        max_tokens=s.max_output_tokens, generation_step=s.generation_step,
                        eos_from_step=sc.eos_from(ignore_eos=s.ignore_eos,
                                                  terminal_continuation=s.terminal_continuation,
                                                  input_finished=s.input_finished, token_count=s.token_count))
    row_slots = rng.sample(range(slots), rows - 3)  # three padding rows at the end
    ctl.set_rows(row_slots)
    nqt.kernels.clear_status(cuda)
    for step in range(4):
        row_states = [states[s] for s in row_slots] + [None] * 3
        ctl.stage()
        want = octl.stage(row_states)
        assert ctl.temperature.cpu().tolist() == pytest.approx(want["temperature"])
        assert ctl.top_k.cpu().tolist() == want["top_k"]
        assert ctl.top_p.cpu().tolist() == pytest.approx(want["top_p"])
        assert ctl.penalty.cpu().tolist() == pytest.approx(want["penalty"])
        assert ctl.seed.cpu().tolist() == want["seed"]
        assert ctl.offset.cpu().tolist() == want["offset"]
        assert [bool(x) for x in ctl.suppress_eos.cpu().tolist()] == want["suppress"]
        logits = (torch.randn(rows, vocab) * 3).to(torch.bfloat16)
        got = ctl.mask_logits(logits.to(cuda)).cpu()
        assert torch.equal(got, octl.mask_logits(logits, codec_vocab, eos_id, want["suppress"]))
        # half of the live rows draw EOS this step
        tokens = torch.tensor([eos_id if rng.random() < 0.5 else rng.randrange(codec_vocab) for _ in range(rows)])
        terminal = ctl.finish(tokens.to(cuda)).cpu()
        assert [bool(x) for x in terminal.tolist()] == octl.finish(row_states, tokens.tolist(), eos_id), step
    assert ctl.slot_step.cpu().tolist() == [s.generation_step for s in states]
    assert ctl.slot_offset.cpu().tolist() == [s.offset for s in states]
    assert nqt.kernels.read_status(cuda) == 0


def test_step_control_is_graph_capturable(nqt, cuda):
    sc = import_module("nari-qwen3-tts_b200.step_control")
    ctl = sc.DeviceStepControl(slots=4, rows=4, device=cuda, vocab=64, codec_vocab=48, eos_id=50)
    for i in range(4):
        ctl.set_request(i, sc.RequestSampling(0.9, 5, 1.0, 1.0, i, 0), max_tokens=3, eos_from_step=0)
    ctl.set_rows([0, 1, 2, 3])
    tokens = torch.tensor([50, 1, 50, 2], device=cuda)
    logits = torch.zeros(4, 64, device=cuda)
    ctl.stage()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ctl.stage()
        ctl.mask_logits(logits)
        ctl.finish(tokens)
    ctl.slot_step.zero_()
    ctl.slot_offset.zero_()
    seen = []
    for _ in range(3):
        graph.replay()
        seen.append(ctl.terminal.cpu().tolist())
    # EOS rows end at once; the others reach max_tokens = 3 on their third step
    assert seen == [[1, 0, 1, 0], [1, 0, 1, 0], [1, 1, 1, 1]]
    assert ctl.slot_offset.cpu().tolist() == [1536] * 4
    assert bool(torch.isinf(logits[:, 48:50]).all()) and bool((logits[:, 50] == 0).all())
