"""Sampler entry points with the reference's call surfaces, on one fused
sm_100a kernel (libnqt ``nqt_sample_rows``).

* ``sample_talker_cuda_graph`` - executor/sampling.py:156-198
* ``sample_logits_cuda_graph`` - executor/sampling.py:201-239
* ``sample_code_predictor_cuda_graph`` - executor/sampling.py:305-336
* ``sample_logits_stateless`` - model/sampling.py:127-225 (validation and
  semantics of the reference; the draw is the kernel's Philox race)

All rows go through one launch; each row's draw depends only on its own
(seed, offset), so a request samples the same token whatever its batch row
(the property the reference buys with one FlashInfer call per row).
Nothing here synchronises with the host except ``sample_logits_stateless``'s
validation, which the reference performs too.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import call, ptr
from .kernels import device_status

MAX_FUSED_RESIDUAL_TOP_K = 64
MAX_CODE_PREDICTOR_TOP_K = MAX_FUSED_RESIDUAL_TOP_K


def _rows(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return t if (t.dtype == dtype and t.is_contiguous()) else t.to(dtype).contiguous()


def sample_rows(
    logits: torch.Tensor,
    temperature: torch.Tensor,
    top_k: torch.Tensor,
    top_p: torch.Tensor,
    seed: torch.Tensor,
    offset: torch.Tensor,
    *,
    repetition_penalty: torch.Tensor | None = None,
    seen_token_mask: torch.Tensor | None = None,
    update_seen: bool = False,
    round_scaled_to_input: bool | None = None,
    noise: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    return_probs: bool = False,
):
    """One fused launch over all rows.  Returns int64 tokens [rows] (and, with
    ``return_probs``, the filtered probabilities and their token ids in rank
    order, [rows, vocab] each)."""

    if logits.ndim != 2 or logits.stride(-1) != 1:
        raise ValueError("logits must be [rows, vocab] with unit vocab stride")
    rows, vocab = logits.shape
    device = _lib.require_cuda(logits, temperature, top_k, top_p, seed, offset, repetition_penalty, seen_token_mask)
    if seen_token_mask is not None:
        if seen_token_mask.shape != logits.shape or seen_token_mask.stride(-1) != 1:
            raise ValueError("seen_token_mask must match the logits shape")
        if seen_token_mask.dtype not in (torch.bool, torch.uint8):
            raise TypeError("seen_token_mask must use torch.bool")
    if update_seen and seen_token_mask is None:
        raise ValueError("update_seen needs a seen_token_mask")
    if round_scaled_to_input is None:
        round_scaled_to_input = seen_token_mask is None and logits.dtype in (torch.bfloat16, torch.float16)
    temperature = _rows(temperature, torch.float32)
    top_k = _rows(top_k, torch.int32)
    top_p = _rows(top_p, torch.float32)
    penalty = None if repetition_penalty is None else _rows(repetition_penalty, torch.float32)
    tokens = out if out is not None else torch.empty(rows, dtype=torch.long, device=device)
    probs = ids = None
    if return_probs:
        probs = torch.empty((rows, vocab), dtype=torch.float32, device=device)
        ids = torch.empty((rows, vocab), dtype=torch.int32, device=device)
    seen_u8 = None if seen_token_mask is None else seen_token_mask.view(torch.uint8)
    common_tail = (
        ptr(penalty),
        ptr(seen_u8),
        0 if seen_u8 is None else seen_u8.stride(0),
        1 if update_seen else 0,
        1 if round_scaled_to_input else 0,
        ptr(tokens),
        ptr(probs),
        ptr(ids),
        ptr(device_status(device)),
        _lib.stream_handle(device),
    )
    if noise is None:
        seed = _rows(seed, torch.long)
        if offset.dtype != torch.long or offset.ndim != 1:
            offset = offset.to(torch.long)
        call(
            "nqt_sample_rows",
            ptr(logits), _lib.dtype_code(logits.dtype), logits.stride(0), rows, vocab,
            ptr(temperature), ptr(top_k), ptr(top_p),
            ptr(seed), ptr(offset), offset.stride(0),
            *common_tail,
        )
    else:
        if noise.ndim != 2 or noise.shape[0] != rows or noise.shape[1] < vocab or noise.dtype != torch.float32 \
                or noise.stride(-1) != 1:
            raise ValueError("noise must be float32 [rows, vocab] with unit stride")
        call(
            "nqt_sample_rows_noise",
            ptr(logits), _lib.dtype_code(logits.dtype), logits.stride(0), rows, vocab,
            ptr(temperature), ptr(top_k), ptr(top_p),
            ptr(noise), noise.stride(0),
            *common_tail,
        )
    if return_probs:
        return tokens, probs, ids
    return tokens


def sample_talker_cuda_graph(
    logits: torch.Tensor,
    temperature: torch.Tensor,
    top_k: torch.Tensor,
    top_p: torch.Tensor,
    seed: torch.Tensor,
    offset: torch.Tensor,
    repetition_penalty: torch.Tensor,
    seen_token_mask: torch.Tensor,
    *,
    update_seen: bool = False,
) -> torch.Tensor:
    """Talker draw with the repetition penalty on the seen mask; greedy rows
    (temperature 0) take the first argmax of the penalised logits.  With
    ``update_seen`` the sampled tokens are also marked in the mask (the
    reference does that with a separate scatter, executor/talker.py:373)."""

    if not logits.is_cuda:
        raise ValueError("sample_talker_cuda_graph requires CUDA logits")
    return sample_rows(
        logits,
        temperature,
        top_k,
        top_p,
        seed,
        offset,
        repetition_penalty=repetition_penalty,
        seen_token_mask=seen_token_mask,
        update_seen=update_seen,
        round_scaled_to_input=False,
    )


def sample_logits_cuda_graph(
    logits: torch.Tensor,
    temperature: torch.Tensor,
    top_k: torch.Tensor,
    top_p: torch.Tensor,
    seed: torch.Tensor,
    offset: torch.Tensor,
) -> torch.Tensor:
    """General-route draw from logits (no penalty)."""

    return sample_rows(logits, temperature, top_k, top_p, seed, offset, round_scaled_to_input=False)


def sample_code_predictor_cuda_graph(
    logits: torch.Tensor,
    temperature: torch.Tensor,
    top_k: torch.Tensor,
    top_p: torch.Tensor,
    seed: torch.Tensor,
    offset: torch.Tensor,
) -> torch.Tensor:
    """Residual-codebook draw; ``offset`` may be a strided column of the
    [rows, groups] offset table (executor/code_predictor.py:222-229)."""

    return sample_rows(logits, temperature, top_k, top_p, seed, offset, round_scaled_to_input=False)


def _require_rows(name: str, value: torch.Tensor, rows: int) -> None:
    if value.ndim != 1 or value.shape[0] != rows:
        raise ValueError(f"{name} must be a row vector with {rows} entries")


def _validate(logits, temperature, top_k, top_p, seed, offset, repetition_penalty, seen_token_mask) -> None:
    """The reference's contract and domain checks (model/sampling.py:8-52, 98-124)."""

    if not logits.is_floating_point():
        raise TypeError("logits must be a floating-point tensor")
    for name, value in (("temperature", temperature), ("top_p", top_p), ("repetition_penalty", repetition_penalty)):
        if not value.is_floating_point():
            raise TypeError(f"{name} must be a floating-point tensor")
    for name, value, dtype in (("top_k", top_k, torch.int32), ("seed", seed, torch.long), ("offset", offset, torch.long)):
        if value.dtype != dtype:
            raise TypeError(f"{name} must use {dtype}, got {value.dtype}")
    tensors = {
        "temperature": temperature,
        "top_k": top_k,
        "top_p": top_p,
        "seed": seed,
        "offset": offset,
        "repetition_penalty": repetition_penalty,
        "seen_token_mask": seen_token_mask,
    }
    mismatched = [name for name, value in tensors.items() if value is not None and value.device != logits.device]
    if mismatched:
        raise ValueError(f"logits and {', '.join(mismatched)} must share one device")
    if seen_token_mask is not None and seen_token_mask.dtype != torch.bool:
        raise TypeError("seen_token_mask must use torch.bool")
    for name, value in (("temperature", temperature), ("top_p", top_p), ("repetition_penalty", repetition_penalty)):
        if not bool(torch.all(torch.isfinite(value))):
            raise ValueError(f"{name} must contain only finite values")
    for name, value in (("temperature", temperature), ("top_k", top_k), ("seed", seed), ("offset", offset)):
        if torch.any(value < 0):
            raise ValueError(f"{name} must be non-negative")
    if torch.any((top_p <= 0) | (top_p > 1)):
        raise ValueError("top_p must be in (0, 1]")
    if torch.any(repetition_penalty <= 0):
        raise ValueError("repetition_penalty must be positive")


def sample_logits_stateless(
    logits: torch.Tensor,
    temperature: torch.Tensor,
    top_k: torch.Tensor,
    top_p: torch.Tensor,
    seed: torch.Tensor,
    offset: torch.Tensor,
    *,
    repetition_penalty: torch.Tensor | None = None,
    seen_token_mask: torch.Tensor | None = None,
    any_greedy: bool | None = None,
    any_top_k_zero: bool | None = None,
    all_top_k_zero: bool | None = None,
) -> torch.Tensor:
    """Validated stateless sampling (model/sampling.py:127-225) on the fused
    kernel.  The optional hints are accepted and ignored, like the reference."""

    del any_greedy, any_top_k_zero, all_top_k_zero
    if logits.ndim != 2 or logits.shape[0] < 1:
        raise ValueError("logits must have shape (rows, vocabulary)")
    rows = logits.shape[0]
    for name, value in (("temperature", temperature), ("top_k", top_k), ("top_p", top_p), ("seed", seed), ("offset", offset)):
        _require_rows(name, value, rows)
    if repetition_penalty is None:
        repetition_penalty = torch.ones_like(temperature)
    _require_rows("repetition_penalty", repetition_penalty, rows)
    _validate(logits, temperature, top_k, top_p, seed, offset, repetition_penalty, seen_token_mask)
    if seen_token_mask is not None and seen_token_mask.shape != logits.shape:
        raise ValueError("seen_token_mask must match the logits shape")
    return sample_rows(
        logits.contiguous(),
        temperature,
        top_k,
        top_p,
        seed,
        offset,
        repetition_penalty=repetition_penalty if seen_token_mask is not None else None,
        seen_token_mask=seen_token_mask.contiguous() if seen_token_mask is not None else None,
    )


__all__ = [
    "MAX_CODE_PREDICTOR_TOP_K",
    "MAX_FUSED_RESIDUAL_TOP_K",
    "sample_code_predictor_cuda_graph",
    "sample_logits_cuda_graph",
    "sample_logits_stateless",
    "sample_rows",
    "sample_talker_cuda_graph",
]
