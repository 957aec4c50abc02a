"""CPU restatement of the talker / code-predictor attention math.

Follows, in fp32 on the CPU:
  * paired QK RMSNorm + RoPE + paged K/V write - model/kernels.py:15-91
    (norm in fp32, x * inv_rms * w, rounded to the element type, then RoPE
    with inv_freq = exp(-ln(theta) * 2i / D); rotated K and raw V stored at
    cache[write_pages[t], 0/1, write_offsets[t], h]);
  * the dense variants - model/kernels.py:163-248 (rounding only when
    round_to_input);
  * paged decode / causal prefill - the FlashInfer wrappers bound at
    executor/talker_kv.py:140-306: row b attends over
    (n_pages - 1) * P + last_page_len tokens, prefill query i of a qo_len
    chunk sees KV positions <= kv_len - qo_len + i; GQA head h reads KV
    head h // (Hq / Hkv) (model/components.py:236-252);
  * short-cache CP attention - model/kernels.py:408-463.
Test infrastructure only (see the package docstring).
"""

from __future__ import annotations

import math

import torch


def rope_inv_freq(head_dim: int, theta: float) -> torch.Tensor:
    i = torch.arange(head_dim // 2, dtype=torch.float64)
    return torch.exp(-math.log(theta) * (2.0 * i / head_dim)).to(torch.float32)


def norm_rope(x: torch.Tensor, weight: torch.Tensor, positions: torch.Tensor, eps: float, theta: float,
              *, round_norm: bool) -> torch.Tensor:
    """x [T, H, D] (any float dtype) -> rotated fp32 [T, H, D] before the final cast."""

    xf = x.float()
    d = xf.shape[-1]
    half = d // 2
    ss = (xf * xf).sum(dim=-1, keepdim=True)
    inv_rms = 1.0 / torch.sqrt(ss / d + eps)
    y = xf * inv_rms * weight.float()
    if round_norm:
        y = y.to(x.dtype).float()
    angle = positions.to(torch.float32).view(-1, 1, 1) * rope_inv_freq(d, theta).view(1, 1, half)
    cos, sin = torch.cos(angle), torch.sin(angle)
    first, second = y[..., :half], y[..., half:]
    return torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)


def qk_norm_rope_paged_(q, k, v, q_weight, k_weight, positions, eps, theta, layer_cache, write_pages, write_offsets):
    """In-place restatement of paired_qk_norm_rope_paged_cache_ on CPU tensors."""

    qr = norm_rope(q, q_weight, positions, eps, theta, round_norm=True).to(q.dtype)
    kr = norm_rope(k, k_weight, positions, eps, theta, round_norm=True).to(k.dtype)
    q.copy_(qr)
    k.copy_(kr)
    for t in range(q.shape[0]):
        page, off = int(write_pages[t]), int(write_offsets[t])
        layer_cache[page, 0, off] = kr[t]
        layer_cache[page, 1, off] = v[t]
    return q, k


def qk_norm_rope_dense_(q, k, v, q_weight, k_weight, positions, eps, theta, key_cache, value_cache, cache_position,
                        *, round_to_input: bool):
    qr = norm_rope(q, q_weight, positions, eps, theta, round_norm=round_to_input).to(q.dtype)
    kr = norm_rope(k, k_weight, positions, eps, theta, round_norm=round_to_input).to(k.dtype)
    q.copy_(qr)
    k.copy_(kr)
    if key_cache is not None:
        key_cache[:, cache_position] = kr
        value_cache[:, cache_position] = v
    return q, k


def kv_length(indptr, last_page_len, page_size: int, b: int) -> int:
    n = int(indptr[b + 1]) - int(indptr[b])
    return 0 if n == 0 else (n - 1) * page_size + int(last_page_len[b])


def gather_kv(layer_cache, indptr, indices, last_page_len, b: int):
    """Dense K, V [kv_len, Hkv, D] (fp32) of row b from the paged layer view."""

    page_size = layer_cache.shape[2]
    pages = indices[int(indptr[b]): int(indptr[b + 1])].long()
    kv_len = kv_length(indptr, last_page_len, page_size, b)
    k = layer_cache[pages, 0].reshape(-1, *layer_cache.shape[3:])[:kv_len].float()
    v = layer_cache[pages, 1].reshape(-1, *layer_cache.shape[3:])[:kv_len].float()
    return k, v


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, visible: torch.Tensor | None):
    """q [Tq, Hq, D], k/v [Tk, Hkv, D] fp32; visible [Tq, Tk] bool or None."""

    group = q.shape[1] // k.shape[1]
    kk = k.repeat_interleave(group, dim=1)
    vv = v.repeat_interleave(group, dim=1)
    scores = torch.einsum("qhd,khd->hqk", q.float(), kk) * scale
    if visible is not None:
        scores = scores.masked_fill(~visible.unsqueeze(0), float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return torch.einsum("hqk,khd->qhd", probs, vv)


def paged_decode(q, layer_cache, indptr, indices, last_page_len, sm_scale=None) -> torch.Tensor:
    """FlashInfer decode semantics; returns fp32 [B, Hq, D]."""

    rows, hq, d = q.shape
    scale = sm_scale if sm_scale is not None else d ** -0.5
    out = torch.zeros(rows, hq, d)
    for b in range(rows):
        k, v = gather_kv(layer_cache, indptr, indices, last_page_len, b)
        if k.shape[0] == 0:
            continue
        out[b] = _attend(q[b: b + 1], k, v, scale, None)[0]
    return out


def paged_prefill(q, layer_cache, qo_indptr, indptr, indices, last_page_len, sm_scale=None) -> torch.Tensor:
    """FlashInfer causal prefill semantics; returns fp32 [T, Hq, D]."""

    tokens, hq, d = q.shape
    scale = sm_scale if sm_scale is not None else d ** -0.5
    out = torch.zeros(tokens, hq, d)
    for b in range(len(qo_indptr) - 1):
        q0, q1 = int(qo_indptr[b]), int(qo_indptr[b + 1])
        if q1 == q0:
            continue
        k, v = gather_kv(layer_cache, indptr, indices, last_page_len, b)
        qo_len, kv_len = q1 - q0, k.shape[0]
        qi = torch.arange(qo_len).view(-1, 1)
        kj = torch.arange(kv_len).view(1, -1)
        visible = kj <= (kv_len - qo_len + qi)
        out[q0:q1] = _attend(q[q0:q1], k, v, scale, visible)
    return out


def short_cache_attention(q, key_cache, value_cache, cache_length: int) -> torch.Tensor:
    """CP one-query attention over cache positions [0, cache_length); fp32 [rows, Hq, D]."""

    rows, hq, d = q.shape
    out = torch.zeros(rows, hq, d)
    for r in range(rows):
        out[r] = _attend(q[r: r + 1], key_cache[r, :cache_length].float(), value_cache[r, :cache_length].float(),
                         d ** -0.5, None)[0]
    return out
