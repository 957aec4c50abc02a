"""Attention-math entry points with the reference's names and contracts.

Each function validates its arguments the way the reference does
(model/kernels.py) and raises the same exception types before any launch,
then calls the sm_100a kernel through libnqt's C ABI on torch's current
stream.  There is no CPU path: non-CUDA tensors are rejected.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import call, ptr


def _status_for(device: torch.device) -> torch.Tensor:
    return device_status(device)


_STATUS: dict[int, torch.Tensor] = {}


def device_status(device: torch.device) -> torch.Tensor:
    """Per-device int32 status word that kernels OR error bits into."""

    index = device.index if device.index is not None else torch.cuda.current_device()
    word = _STATUS.get(index)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
        _STATUS[index] = word
    return word


def read_status(device: torch.device) -> int:
    """Host read of the status word (synchronises); 0 means no device error."""

    return int(device_status(device).item())


def clear_status(device: torch.device) -> None:
    device_status(device).zero_()


def paired_qk_norm_rope_paged_cache_(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    query_weight: torch.Tensor,
    key_weight: torch.Tensor,
    position_ids: torch.Tensor,
    epsilon: float,
    rope_theta: float,
    layer_cache: torch.Tensor,
    write_pages: torch.Tensor,
    write_offsets: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Normalise/rotate QK in place and stage K/V into the paged cache.

    Contract of model/kernels.py:94-160: per (token, head) fp32 RMSNorm,
    times the weight, rounded to the element type, then RoPE; rotated K and
    raw V land in layer_cache[write_pages[t], 0/1, write_offsets[t]].
    """

    if query.ndim != 3 or key.ndim != 3 or value.ndim != 3:
        raise ValueError("Qwen3-TTS QKV tensors must have rank three")
    tokens, query_heads, head_dim = query.shape
    if key.shape != value.shape or key.shape[0] != tokens or key.shape[2] != head_dim:
        raise ValueError("Qwen3-TTS QKV shapes are incompatible")
    key_heads = key.shape[1]
    if query.device.type != "cuda" or not (query.device == key.device == value.device == layer_cache.device):
        raise ValueError("paired QKV paged staging requires one CUDA device")
    if not (query.dtype == key.dtype == value.dtype == layer_cache.dtype):
        raise TypeError("paired QKV paged staging requires one dtype")
    if head_dim % 2 or query_weight.shape != (head_dim,) or key_weight.shape != (head_dim,):
        raise ValueError("QK norm weights must match an even head dimension")
    if position_ids.shape != (tokens,) or write_pages.shape != (tokens,) or write_offsets.shape != (tokens,):
        raise ValueError("paged QKV metadata must contain one entry per token")
    if layer_cache.ndim != 5 or layer_cache.shape[1] != 2 or layer_cache.shape[3:] != (key_heads, head_dim):
        raise ValueError("paged QKV cache has an invalid layout")
    if not all(tensor.stride(-1) == 1 for tensor in (query, key, value, layer_cache)):
        raise ValueError("QKV and paged cache must be contiguous per head")
    if not layer_cache.is_contiguous():
        raise ValueError("paged QKV cache must be contiguous")
    for t in (position_ids, write_pages, write_offsets):
        if t.dtype != torch.long or not t.is_contiguous():
            raise TypeError("paged QKV metadata must be contiguous int64")
    if query_weight.dtype != query.dtype or key_weight.dtype != query.dtype:
        query_weight = query_weight.to(query.dtype)
        key_weight = key_weight.to(query.dtype)
    if tokens == 0:
        return query, key
    device = query.device
    call(
        "nqt_qk_norm_rope_paged_kv_write",
        ptr(query), query.stride(0), query.stride(1),
        ptr(key), key.stride(0), key.stride(1),
        ptr(value), value.stride(0), value.stride(1),
        ptr(query_weight.contiguous()), ptr(key_weight.contiguous()),
        ptr(position_ids), ptr(write_pages), ptr(write_offsets),
        ptr(layer_cache), layer_cache.shape[0], layer_cache.shape[2],
        tokens, query_heads, key_heads, head_dim,
        float(epsilon), float(rope_theta), _lib.dtype_code(query.dtype),
        ptr(device_status(device)), _lib.stream_handle(device),
    )
    return query, key


def _validate_qk(query, key, query_weight, key_weight, positions):
    if query.ndim != 3 or key.ndim != 3:
        raise ValueError("QK tensors must have shape [tokens, heads, head_dim]")
    tokens, query_heads, head_dim = query.shape
    if key.shape[0] != tokens or key.shape[2] != head_dim or head_dim % 2:
        raise ValueError("QK shapes are incompatible")
    key_heads = key.shape[1]
    if query.device.type != "cuda" or key.device != query.device or query.dtype != key.dtype:
        raise ValueError("paired QK transform requires one CUDA dtype/device")
    if query.stride(-1) != 1 or key.stride(-1) != 1:
        raise ValueError("QK tensors must be contiguous per head")
    if positions.shape != (tokens,) or positions.device != query.device:
        raise ValueError("positions must contain one CUDA value per token")
    if query_weight.shape != (head_dim,) or key_weight.shape != (head_dim,):
        raise ValueError("QK norm weights must match head_dim")
    return tokens, query_heads, key_heads, head_dim


def paired_qk_norm_rope_(
    query: torch.Tensor,
    key: torch.Tensor,
    query_weight: torch.Tensor,
    key_weight: torch.Tensor,
    positions: torch.Tensor,
    epsilon: float,
    rope_theta: float,
) -> tuple[torch.Tensor, torch.Tensor]:
    """QK transform with the bf16 rounding boundary (model/kernels.py:275-332)."""

    tokens, query_heads, key_heads, head_dim = _validate_qk(query, key, query_weight, key_weight, positions)
    if tokens == 0:
        return query, key
    positions = positions.to(torch.long)
    device = query.device
    call(
        "nqt_qk_norm_rope_dense",
        ptr(query), query.stride(0), query.stride(1),
        ptr(key), key.stride(0), key.stride(1),
        None, 0, 0,
        ptr(query_weight.to(query.dtype).contiguous()), ptr(key_weight.to(query.dtype).contiguous()),
        ptr(positions), positions.stride(0),
        None, None, 0, 0, 0, 0,
        tokens, query_heads, key_heads, head_dim,
        float(epsilon), float(rope_theta), 1, _lib.dtype_code(query.dtype),
        ptr(device_status(device)), _lib.stream_handle(device),
    )
    return query, key


def paired_qk_norm_rope_dense_cache_(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    query_weight: torch.Tensor,
    key_weight: torch.Tensor,
    positions: torch.Tensor,
    epsilon: float,
    rope_theta: float,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    cache_position: int,
) -> tuple[torch.Tensor, torch.Tensor]:
    """One-token QK transform plus dense CP cache write (model/kernels.py:335-405)."""

    tokens, query_heads, key_heads, head_dim = _validate_qk(query, key, query_weight, key_weight, positions)
    expected = (tokens, key_cache.shape[1], key_heads, head_dim)
    if value.shape != (tokens, key_heads, head_dim) or key_cache.shape != expected or value_cache.shape != expected:
        raise ValueError("dense CP QKV cache shape mismatch")
    if not 0 <= cache_position < key_cache.shape[1]:
        raise ValueError("dense CP cache position is invalid")
    if not (value.device == key_cache.device == value_cache.device == query.device):
        raise ValueError("dense CP QKV cache requires one CUDA device")
    if not (value.dtype == key_cache.dtype == value_cache.dtype == query.dtype):
        raise TypeError("dense CP QKV cache requires one dtype")
    if key_cache.stride() != value_cache.stride() or key_cache.stride(-1) != 1 or value.stride(-1) != 1:
        raise ValueError("dense CP caches must share a layout with unit head_dim stride")
    if tokens == 0:
        return query, key
    positions = positions.to(torch.long)
    device = query.device
    call(
        "nqt_qk_norm_rope_dense",
        ptr(query), query.stride(0), query.stride(1),
        ptr(key), key.stride(0), key.stride(1),
        ptr(value), value.stride(0), value.stride(1),
        ptr(query_weight.to(query.dtype).contiguous()), ptr(key_weight.to(query.dtype).contiguous()),
        ptr(positions), positions.stride(0),
        ptr(key_cache), ptr(value_cache), key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
        int(cache_position),
        tokens, query_heads, key_heads, head_dim,
        float(epsilon), float(rope_theta), 0, _lib.dtype_code(query.dtype),
        ptr(device_status(device)), _lib.stream_handle(device),
    )
    return query, key


def decode_attn_nhd_short_cache(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    cache_length: int,
) -> torch.Tensor:
    """Short-cache one-query attention (model/kernels.py:466-520)."""

    if not isinstance(cache_length, int) or isinstance(cache_length, bool) or not 1 <= cache_length <= 16:
        raise ValueError("short-cache attention requires cache_length in [1, 16]")
    squeeze = query.ndim == 4
    if squeeze:
        if query.shape[1] != 1:
            raise ValueError("short-cache attention supports one query token")
        query = query.squeeze(1)
    if query.ndim != 3 or key_cache.ndim != 4 or key_cache.shape != value_cache.shape:
        raise ValueError("short-cache QKV ranks are invalid")
    rows, query_heads, head_dim = query.shape
    cache_rows, capacity, key_heads, cache_head_dim = key_cache.shape
    if (cache_rows, cache_head_dim) != (rows, head_dim) or cache_length > capacity:
        raise ValueError("short-cache QKV shapes are incompatible")
    if query_heads % key_heads or query.device.type != "cuda":
        raise ValueError("short-cache attention requires compatible CUDA heads")
    if key_cache.stride() != value_cache.stride() or key_cache.stride(-1) != 1 or query.stride(-1) != 1:
        raise ValueError("short-cache tensors must be contiguous per head with one cache layout")
    output = torch.empty((rows, query_heads, head_dim), dtype=query.dtype, device=query.device)
    device = query.device
    call(
        "nqt_cp_short_attention",
        ptr(query), query.stride(0), query.stride(1),
        ptr(key_cache), ptr(value_cache), key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
        cache_length, rows, query_heads, key_heads, head_dim, 1.0 / (head_dim**0.5),
        ptr(output), output.stride(0), output.stride(1),
        ptr(device_status(device)), _lib.stream_handle(device),
    )
    return output.unsqueeze(1) if squeeze else output


def cp_decode_attention_(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    query_weight: torch.Tensor,
    key_weight: torch.Tensor,
    positions: torch.Tensor,
    epsilon: float,
    rope_theta: float,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    cache_position: int,
) -> torch.Tensor:
    """Fused code-predictor decode step: the dense-cache QK transform and
    write of ``paired_qk_norm_rope_dense_cache_`` followed by
    ``decode_attn_nhd_short_cache`` over ``cache_position + 1`` positions,
    in one launch (model/components.py:309-345).  Returns [rows, Hq, D]."""

    tokens, query_heads, key_heads, head_dim = _validate_qk(query, key, query_weight, key_weight, positions)
    expected = (tokens, key_cache.shape[1], key_heads, head_dim)
    if value.shape != (tokens, key_heads, head_dim) or key_cache.shape != expected or value_cache.shape != expected:
        raise ValueError("dense CP QKV cache shape mismatch")
    if not 0 <= cache_position < key_cache.shape[1]:
        raise ValueError("dense CP cache position is invalid")
    if not (value.dtype == key_cache.dtype == value_cache.dtype == query.dtype == torch.bfloat16):
        raise TypeError("fused CP attention requires bf16 tensors")
    if key_cache.stride() != value_cache.stride() or key_cache.stride(-1) != 1 or value.stride(-1) != 1:
        raise ValueError("dense CP caches must share a layout with unit head_dim stride")
    positions = positions.to(torch.long)
    output = torch.empty((tokens, query_heads, head_dim), dtype=query.dtype, device=query.device)
    device = query.device
    call(
        "nqt_cp_decode_attention",
        ptr(query), query.stride(0), query.stride(1),
        ptr(key), key.stride(0), key.stride(1),
        ptr(value), value.stride(0), value.stride(1),
        ptr(query_weight.to(query.dtype).contiguous()), ptr(key_weight.to(query.dtype).contiguous()),
        ptr(positions), positions.stride(0),
        ptr(key_cache), ptr(value_cache), key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
        key_cache.shape[1], int(cache_position),
        tokens, query_heads, key_heads, head_dim,
        float(epsilon), float(rope_theta), 1.0 / (head_dim**0.5),
        ptr(output), output.stride(0), output.stride(1),
        ptr(device_status(device)), _lib.stream_handle(device),
    )
    return output


__all__ = [
    "Fp8BlockWeight",
    "PackedWeight",
    "clear_status",
    "cp_codec_step",
    "cp_decode_attention_",
    "decode_attn_nhd_short_cache",
    "device_status",
    "paired_qk_norm_rope_",
    "paired_qk_norm_rope_dense_cache_",
    "fp8_gemm_workspace",
    "fp8_quantize_rows",
    "fused_add_rmsnorm_",
    "fused_add_rmsnorm_fp8_",
    "linear",
    "linear_fp8",
    "paired_qk_norm_rope_paged_cache_",
    "quantize_fp8_weight_blocks",
    "read_status",
    "rmsnorm",
    "silu_and_mul",
]


# ---------------------------------------------------------------- layer glue
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """RMSNorm over the last dim (flashinfer.norm.rmsnorm at model/layers.py:80-100)."""

    if x.stride(-1) != 1 or weight.dtype != x.dtype:
        raise ValueError("rmsnorm needs rows contiguous in the hidden dim and a weight of the input dtype")
    flat = x.reshape(-1, x.shape[-1])
    if out is None:
        out = torch.empty_like(flat)
    call("nqt_rmsnorm", ptr(flat), flat.stride(0), ptr(weight), ptr(out), out.stride(0), flat.shape[0],
         flat.shape[1], float(eps), _lib.dtype_code(x.dtype), _lib.stream_handle(x.device))
    return out.view(x.shape)


def fused_add_rmsnorm_(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float) -> None:
    """In place: residual <- x + residual; x <- rmsnorm(residual) * weight
    (flashinfer.norm.fused_add_rmsnorm at model/layers.py:42-77)."""

    if not (x.is_contiguous() and residual.is_contiguous()) or x.shape != residual.shape:
        raise ValueError("fused_add_rmsnorm needs contiguous tensors of one shape")
    hidden = x.shape[-1]
    call("nqt_fused_add_rmsnorm", ptr(x), ptr(residual), ptr(weight), x.numel() // hidden, hidden, float(eps),
         _lib.dtype_code(x.dtype), _lib.stream_handle(x.device))


def silu_and_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """silu(gate) * up for gate_up = [gate | up] (model/layers.py:28-39)."""

    d = gate_up.shape[-1] // 2
    flat = gate_up.reshape(-1, 2 * d)
    if out is None:
        out = torch.empty((flat.shape[0], d), dtype=gate_up.dtype, device=gate_up.device)
    call("nqt_silu_and_mul", ptr(flat), flat.stride(0), ptr(out), out.stride(0), flat.shape[0], d,
         _lib.dtype_code(gate_up.dtype), _lib.stream_handle(gate_up.device))
    return out.view(*gate_up.shape[:-1], d)


GEMM_PLAIN = 0
GEMM_BIAS = 1
GEMM_SILU_MUL = 2


class PackedWeight:
    """A weight [n, k] laid out once for nqt_gemm_bf16: contiguous 16 KB
    tiles in the MMA's swizzled order (``gate_up`` interleaves the two
    halves of a gate_up weight in 64-row blocks for the silu_mul epilogue)."""

    def __init__(self, weight: torch.Tensor, *, gate_up: bool = False) -> None:
        if weight.dim() != 2 or weight.dtype != torch.bfloat16 or weight.stride(1) != 1:
            raise ValueError("pack a bf16 [n, k] weight with unit stride along k")
        n, k = weight.shape
        if n % 128 or k % 64 or (gate_up and n % 256):
            raise ValueError("packed weights need n % 128 == 0 (256 for gate_up) and k % 64 == 0")
        self.n, self.k, self.gate_up = n, k, gate_up
        self.data = torch.empty(n * k, dtype=torch.bfloat16, device=weight.device)
        call("nqt_gemm_pack_weight", ptr(weight), weight.stride(0), n, k, 1 if gate_up else 0, ptr(self.data),
             _lib.stream_handle(weight.device))

    @property
    def shape(self) -> tuple[int, int]:
        return (self.n, self.k)


def linear(x: torch.Tensor, weight: PackedWeight, bias: torch.Tensor | None = None, *,
           out: torch.Tensor | None = None, split: int = 0) -> torch.Tensor:
    """x [m, k] @ W[n, k]^T (+ bias) on the weight-streaming tcgen05 GEMM
    (the decoder projections, model/layers.py:195-270).  A ``gate_up`` packed
    weight gives silu(gate) * up, [m, n / 2].  ``split``: CTAs (one cluster)
    sharing each 128-row tile's K, 1..8; 0 picks the largest that keeps the
    grid within one CTA per SM."""

    if not isinstance(weight, PackedWeight):
        raise TypeError("linear takes a PackedWeight")
    if x.dim() != 2 or x.shape[1] != weight.k:
        raise ValueError("linear needs x [m, k] matching the weight")
    if x.dtype != torch.bfloat16:
        raise TypeError("linear computes in bf16")
    if x.stride(1) != 1:
        raise ValueError("linear needs unit stride along k")
    if weight.gate_up and bias is not None:
        raise ValueError("the silu_mul epilogue takes no bias")
    m = x.shape[0]
    cols = weight.n // 2 if weight.gate_up else weight.n
    if out is None:
        out = torch.empty((m, cols), dtype=torch.bfloat16, device=x.device)
    elif out.shape != (m, cols) or out.dtype != torch.bfloat16 or out.stride(1) != 1:
        raise ValueError("linear output must be bf16 [m, n] with unit column stride")
    epilogue = GEMM_SILU_MUL if weight.gate_up else (GEMM_BIAS if bias is not None else GEMM_PLAIN)
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.shape != (weight.n,) or not bias.is_contiguous()):
        raise ValueError("linear bias must be contiguous bf16 [n]")
    call("nqt_gemm_bf16", ptr(x), x.stride(0), ptr(weight.data), ptr(out), out.stride(0), ptr(bias),
         m, weight.n, weight.k, epilogue, int(split), ptr(device_status(x.device)), _lib.stream_handle(x.device))
    return out


def cp_codec_step(tokens: torch.Tensor, frames_col: torch.Tensor, codec_emb: torch.Tensor, codec_sum: torch.Tensor,
                  *, accumulate: bool = True, proj_emb: torch.Tensor | None = None, ln: torch.Tensor | None = None,
                  eps: float = 1e-6, residual: torch.Tensor | None = None, h: torch.Tensor | None = None) -> None:
    """The code-predictor frame's glue after a codebook's tokens are sampled (executor/code_predictor.py:
    160-235), one launch: frames_col <- tokens; codec_sum (+)= codec_emb[tokens]; with ``proj_emb``,
    residual <- proj_emb[tokens] and h <- rmsnorm(residual) * ln (the next depth step's input)."""

    rows = tokens.shape[0]
    if tokens.dtype != torch.long or frames_col.dtype != torch.long or frames_col.shape[0] != rows:
        raise TypeError("cp_codec_step takes int64 tokens and an int64 frames column")
    if codec_emb.dtype != torch.bfloat16 or not codec_emb.is_contiguous() or not codec_sum.is_contiguous() \
            or codec_sum.shape != (rows, codec_emb.shape[1]):
        raise ValueError("cp_codec_step needs contiguous bf16 codec_emb [vocab, H] and codec_sum [rows, H]")
    hidden = 0
    if proj_emb is not None:
        hidden = proj_emb.shape[1]
        for t in (proj_emb, ln, residual, h):
            if t is None or not t.is_contiguous() or t.dtype != torch.bfloat16:
                raise ValueError("cp_codec_step needs contiguous bf16 proj_emb, ln, residual and h")
        if residual.shape != (rows, hidden) or h.shape != (rows, hidden) or proj_emb.shape[0] != codec_emb.shape[0]:
            raise ValueError("cp_codec_step: residual / h must be [rows, hidden] and the tables share the vocab")
    call("nqt_cp_codec_step", ptr(tokens), rows, ptr(frames_col), frames_col.stride(0), ptr(codec_emb),
         codec_emb.shape[0], codec_emb.shape[1], ptr(codec_sum), 1 if accumulate else 0, ptr(proj_emb), ptr(ln),
         hidden, float(eps), ptr(residual), ptr(h), _lib.dtype_code(codec_emb.dtype), ptr(device_status(tokens.device)),
         _lib.stream_handle(tokens.device))


# ---------------------------------------------------------------- FP8 block-scaled gate/up
def quantize_fp8_weight_blocks(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise a row-major bf16 matrix into 128 x 128 e4m3 blocks with power-of-two scales, on the GPU
    (model/layers.py:11-25: s = 2^ceil(log2(max(amax, 1e-4) / 448)), q = e4m3(w / s)).  Returns
    (q [n, k] float8_e4m3fn, scales [n / 128, k / 128] float32), the reference's layouts."""

    if weight.ndim != 2 or not weight.is_contiguous():
        raise ValueError("FP8 block quantization requires a contiguous matrix")
    rows, columns = weight.shape
    if rows % 128 or columns % 128:
        raise ValueError(
            f"FP8 block quantization requires dimensions divisible by 128, got {tuple(weight.shape)}")
    if weight.dtype != torch.bfloat16:
        raise TypeError("FP8 block quantization takes a bf16 weight")
    q = torch.empty((rows, columns), dtype=torch.float8_e4m3fn, device=weight.device)
    scales = torch.empty((rows // 128, columns // 128), dtype=torch.float32, device=weight.device)
    call("nqt_fp8_quantize_weight_blocks", ptr(weight), weight.stride(0), rows, columns, ptr(q), q.stride(0),
         ptr(scales), _lib.stream_handle(weight.device))
    return q, scales


def fp8_quantize_rows(x: torch.Tensor, *, out: torch.Tensor | None = None,
                      scale: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per token, per 128-element block: f = 448 / amax (1 when amax = 0), q = e4m3(x * f), scale 1 / f - the
    bf16-input rule of the reference's FP8 gate/up GEMM (model/layers.py:242-256).  Returns (q [m, k]
    float8_e4m3fn, scale [k / 128, m] float32: a block's tokens contiguous)."""

    if x.dim() != 2 or x.dtype != torch.bfloat16 or x.stride(1) != 1:
        raise ValueError("fp8_quantize_rows takes bf16 [m, k] with unit stride along k")
    m, k = x.shape
    if k % 128:
        raise ValueError("fp8_quantize_rows needs k % 128 == 0")
    if out is None:
        out = torch.empty((m, k), dtype=torch.float8_e4m3fn, device=x.device)
    if scale is None:
        scale = torch.empty((k // 128, m), dtype=torch.float32, device=x.device)
    if out.shape != (m, k) or out.dtype != torch.float8_e4m3fn or out.stride(1) != 1:
        raise ValueError("fp8_quantize_rows output must be float8_e4m3fn [m, k] with unit column stride")
    if scale.dim() != 2 or scale.shape[0] != k // 128 or scale.shape[1] < m or scale.stride(1) != 1 \
            or scale.dtype != torch.float32:
        raise ValueError("fp8_quantize_rows scale must be float32 [k / 128, >= m] with unit column stride")
    call("nqt_fp8_quantize_rows", ptr(x), x.stride(0), m, k, ptr(out), out.stride(0), ptr(scale), scale.stride(0),
         _lib.stream_handle(x.device))
    return out, scale


def fused_add_rmsnorm_fp8_(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                           q: torch.Tensor, scale: torch.Tensor, *, write_x: bool = False) -> None:
    """residual <- x + residual; the normed row rmsnorm(residual) * weight (bf16) is quantised into q / scale
    by the fp8_quantize_rows rule (and written to x when ``write_x``): the post-attention norm feeding the
    FP8 gate/up GEMM."""

    if not (x.is_contiguous() and residual.is_contiguous()) or x.shape != residual.shape or x.dim() != 2:
        raise ValueError("fused_add_rmsnorm_fp8 needs contiguous [rows, hidden] tensors of one shape")
    rows, hidden = x.shape
    if q.shape != (rows, hidden) or q.dtype != torch.float8_e4m3fn or q.stride(1) != 1:
        raise ValueError("fused_add_rmsnorm_fp8 q must be float8_e4m3fn [rows, hidden]")
    if scale.dtype != torch.float32 or scale.dim() != 2 or scale.shape[0] != hidden // 128 or \
            scale.shape[1] < rows or scale.stride(1) != 1:
        raise ValueError("fused_add_rmsnorm_fp8 scale must be float32 [hidden / 128, >= rows]")
    call("nqt_fused_add_rmsnorm_fp8", ptr(x), ptr(residual), ptr(weight), rows, hidden, float(eps), ptr(q),
         q.stride(0), ptr(scale), scale.stride(0), 1 if write_x else 0, _lib.dtype_code(x.dtype),
         _lib.stream_handle(x.device))


class Fp8BlockWeight:
    """A bf16 weight [n, k] quantised once (quantize_fp8_weight_blocks) and packed for nqt_gemm_fp8.
    ``gate_up`` interleaves the gate and up halves in 64-row blocks for the SwiGLU epilogue.  Keeps the
    reference-layout ``q`` and ``scale`` (the GEMM reads ``scale`` directly)."""

    def __init__(self, weight: torch.Tensor, *, gate_up: bool = False) -> None:
        n, k = weight.shape
        if gate_up and n % 256:
            raise ValueError("a gate_up weight needs n % 256 == 0")
        self.n, self.k, self.gate_up = n, k, gate_up
        self.q, self.scale = quantize_fp8_weight_blocks(weight)
        self.data = torch.empty(n * k, dtype=torch.uint8, device=weight.device)
        call("nqt_gemm_fp8_pack_weight", ptr(self.q), self.q.stride(0), n, k, 1 if gate_up else 0, ptr(self.data),
             _lib.stream_handle(weight.device))

    @property
    def shape(self) -> tuple[int, int]:
        return (self.n, self.k)


_FP8_WORKSPACE: dict[tuple[int, int, int, int, int], torch.Tensor] = {}


def fp8_gemm_workspace(device: torch.device, m: int, n: int, k: int, split: int = 0) -> torch.Tensor | None:
    """The split-K workspace nqt_gemm_fp8 needs for this shape (None when it needs none): one zeroed buffer
    per (device, shape), because a workspace's tickets are laid out for one launch shape (another shape's
    partials would land on them).  Call it once outside graph capture for every shape a captured step uses;
    a first call inside capture would allocate."""

    nbytes = ctypes.c_int64(0)
    call("nqt_gemm_fp8_workspace_bytes", m, n, k, int(split), ctypes.addressof(nbytes))
    if nbytes.value == 0:
        return None
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, m, n, k, int(split))
    ws = _FP8_WORKSPACE.get(key)
    if ws is None:
        ws = torch.zeros(nbytes.value, dtype=torch.uint8, device=torch.device("cuda", index))
        _FP8_WORKSPACE[key] = ws
    return ws


def linear_fp8(xq: torch.Tensor, xscale: torch.Tensor, weight: Fp8BlockWeight, *, out: torch.Tensor | None = None,
               split: int = 0, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Block-scaled FP8 product Y = sum_b (Xq_b . Wq_b^T) * xscale[b, t] * wscale[row / 128, b] on the tcgen05
    weight-streaming GEMM (the reference's FP8 gate/up, model/layers.py:242-256); a ``gate_up`` weight gives
    silu(gate) * up, [m, n / 2].  ``split``: bits 0-7 CTAs sharing each tile's K (0 automatic), bits 8-11 K
    blocks per copy stage (0 automatic).  ``workspace``: the split-K buffer (fp8_gemm_workspace by default;
    one launch at a time per buffer)."""

    if not isinstance(weight, Fp8BlockWeight):
        raise TypeError("linear_fp8 takes an Fp8BlockWeight")
    if xq.dim() != 2 or xq.shape[1] != weight.k or xq.dtype != torch.float8_e4m3fn or xq.stride(1) != 1:
        raise ValueError("linear_fp8 needs xq float8_e4m3fn [m, k] matching the weight")
    m = xq.shape[0]
    if xscale.dtype != torch.float32 or xscale.dim() != 2 or xscale.shape[0] != weight.k // 128 or \
            xscale.shape[1] < m or xscale.stride(1) != 1:
        raise ValueError("linear_fp8 xscale must be float32 [k / 128, >= m]")
    cols = weight.n // 2 if weight.gate_up else weight.n
    if out is None:
        out = torch.empty((m, cols), dtype=torch.bfloat16, device=xq.device)
    elif out.shape != (m, cols) or out.dtype != torch.bfloat16 or out.stride(1) != 1:
        raise ValueError("linear_fp8 output must be bf16 [m, n] with unit column stride")
    epilogue = GEMM_SILU_MUL if weight.gate_up else GEMM_PLAIN
    if workspace is None:
        workspace = fp8_gemm_workspace(xq.device, m, weight.n, weight.k, split)
    call("nqt_gemm_fp8", ptr(xq), xq.stride(0), ptr(xscale), xscale.stride(0), ptr(weight.data), ptr(weight.scale),
         ptr(out), out.stride(0), m, weight.n, weight.k, epilogue, 1 if weight.gate_up else 0, int(split),
         ptr(workspace), 0 if workspace is None else workspace.numel(), ptr(device_status(xq.device)),
         _lib.stream_handle(xq.device))
    return out
