"""ctypes binding of libnqt.so (the C ABI declared in include/nqt.h).

There is no fallback: if the library is missing or CUDA is unavailable the
call raises.  ``lib()`` loads the in-tree library once per process.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libnqt.so"

NQT_OK = 0
NQT_ERR_ARG = -1
NQT_ERR_CUDA = -2
NQT_ERR_CAPACITY = -3
NQT_ERR_UNSUPPORTED = -4

NQT_DEV_BAD_PAGE = 0x1
NQT_DEV_TIMEOUT = 0x2
NQT_DEV_KV_EXHAUSTED = 0x4
NQT_DEV_BAD_SLOT = 0x8
NQT_DEV_TABLE_FULL = 0x10
NQT_DEV_CAPACITY = 0x20
NQT_DEV_BAD_TOKEN = 0x40

NQT_BF16 = 0
NQT_F16 = 1
NQT_F32 = 2

P = c_void_p
I = c_int
L = c_int64
F = c_float
Z = c_size_t

# name -> (restype, argtypes); mirrors include/nqt.h one to one.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "nqt_abi_version": (I, []),
    "nqt_last_error": (ctypes.c_char_p, []),
    "nqt_qk_norm_rope_paged_kv_write": (
        I,
        [P, L, L, P, L, L, P, L, L, P, P, P, P, P, P, I, I, I, I, I, I, F, F, I, P, P],
    ),
    "nqt_qk_norm_rope_dense": (
        I,
        [P, L, L, P, L, L, P, L, L, P, P, P, L, P, P, L, L, L, I, I, I, I, I, F, F, I, I, P, P],
    ),
    "nqt_decode_workspace_bytes": (Z, [I, I, I]),
    "nqt_decode_plan": (I, [P, P, I, I, I, I, I, P, Z, P]),
    "nqt_decode_attention": (
        I,
        [P, L, L, P, I, I, P, P, P, I, I, I, I, I, F, P, L, L, P, Z, P, P],
    ),
    "nqt_decode_attention_ex": (
        I,
        [P, L, L, P, I, I, P, P, P, I, I, I, I, I, F, P, L, L, P, Z, I, P, P],
    ),
    "nqt_decode_attention_noalloc": (
        I,
        [P, L, L, P, I, I, P, P, P, I, I, I, I, F, P, L, L, P, P],
    ),
    "nqt_decode_noalloc_scratch_bytes": (Z, []),
    "nqt_prefill_attention": (
        I,
        [P, L, L, P, I, I, P, P, P, P, I, I, I, I, I, F, P, L, L, P, P],
    ),
    "nqt_cp_decode_attention": (
        I,
        [P, L, L, P, L, L, P, L, L, P, P, P, L, P, P, L, L, L, I, I, I, I, I, I, F, F, F, P, L, L, P, P],
    ),
    "nqt_cp_short_attention": (I, [P, L, L, P, P, L, L, L, I, I, I, I, I, F, P, L, L, P, P]),
    "nqt_sample_rows": (
        I,
        [P, I, L, I, I, P, P, P, P, P, L, P, P, L, I, I, P, P, P, P, P],
    ),
    "nqt_sample_rows_noise": (
        I,
        [P, I, L, I, I, P, P, P, P, L, P, P, L, I, I, P, P, P, P, P],
    ),
    "nqt_planner_state_bytes": (Z, [I, I, I]),
    "nqt_planner_init": (I, [P, I, I, I, I, P]),
    "nqt_plan_step": (
        I,
        [P, I, I, I, I, P, P, I, I, P, I, I, P, P, P, I, P, P, P, P, P, P, Z, I, I, P, P],
    ),
    "nqt_plan_commit": (I, [P, I, I, I, P, P, P, I, P, P, P]),
    "nqt_plan_release": (I, [P, I, I, I, P, I, P, P]),
    "nqt_plan_import": (I, [P, I, I, I, I, P, I, I, I, P, P]),
    "nqt_rmsnorm": (I, [P, L, P, P, L, I, I, F, I, P]),
    "nqt_fused_add_rmsnorm": (I, [P, P, P, I, I, F, I, P]),
    "nqt_silu_and_mul": (I, [P, L, P, L, I, I, I, P]),
    "nqt_gemm_pack_weight": (I, [P, L, I, I, I, P, P]),
    "nqt_gemm_bf16": (I, [P, L, P, P, L, P, I, I, I, I, I, P, P]),
    "nqt_cp_codec_step": (I, [P, I, P, L, P, I, I, P, I, P, P, I, F, P, P, I, P, P]),
    "nqt_fp8_quantize_weight_blocks": (I, [P, L, I, I, P, L, P, P]),
    "nqt_fp8_quantize_rows": (I, [P, L, I, I, P, L, P, L, P]),
    "nqt_fused_add_rmsnorm_fp8": (I, [P, P, P, I, I, F, P, L, P, L, I, I, P]),
    "nqt_gemm_fp8_pack_weight": (I, [P, L, I, I, I, P, P]),
    "nqt_gemm_fp8_workspace_bytes": (I, [I, I, I, I, P]),
    "nqt_gemm_fp8": (I, [P, L, P, L, P, P, P, L, I, I, I, I, I, I, P, L, P, P]),
    "nqt_step_stage": (I, [P, I, I, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P]),
    "nqt_talker_logits_mask": (I, [P, I, L, I, I, I, I, P, P]),
    "nqt_step_finish": (I, [P, I, I, P, I, P, P, P, P, L, P, P, P, P]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NqtError(RuntimeError):
    """A libnqt entry point returned a negative status."""

    def __init__(self, name: str, code: int, detail: str = "") -> None:
        names = {
            NQT_ERR_ARG: "invalid argument",
            NQT_ERR_CUDA: "CUDA error",
            NQT_ERR_CAPACITY: "capacity exceeded",
            NQT_ERR_UNSUPPORTED: "unsupported shape",
        }
        message = f"{name} failed: {names.get(code, code)}"
        if detail:
            message += f" ({detail})"
        super().__init__(message)
        self.code = code


def lib() -> ctypes.CDLL:
    """Load libnqt.so (once).  Raises if it has not been built."""

    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


# kernels each entry point launches (nqt_plan_step adds the split-KV plan when given a workspace)
KERNELS_PER_CALL = {
    "nqt_decode_attention_noalloc": 2,
}
_launches = 0


def reset_launch_count() -> None:
    global _launches
    _launches = 0


def launch_count() -> int:
    """libnqt kernel launches issued since the last reset (graph capture included)."""

    return _launches


def call(name: str, *args) -> int:
    """Invoke an entry point and raise NqtError on a negative status."""

    global _launches
    fn = getattr(lib(), name)
    rc = fn(*args)
    if not name.endswith(("_bytes", "_version", "_error")):
        n = KERNELS_PER_CALL.get(name, 1)
        if name == "nqt_plan_step" and args[20] is not None:
            n = 2
        _launches += n
    if isinstance(rc, int) and rc < 0:
        detail = ""
        if rc == NQT_ERR_CUDA:
            detail = (lib().nqt_last_error() or b"").decode(errors="replace")
        raise NqtError(name, rc, detail)
    return rc


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device | None = None) -> int:
    """Raw cudaStream_t of torch's current stream (what graph capture records)."""

    if not torch.cuda.is_available():
        raise RuntimeError("libnqt kernels need a CUDA device; none is available")
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return NQT_BF16
    if dtype == torch.float16:
        return NQT_F16
    if dtype == torch.float32:
        return NQT_F32
    raise TypeError(f"unsupported element type {dtype}")


def require_cuda(*tensors: torch.Tensor | None) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError("libnqt kernels require CUDA tensors on one device")
        if device is None:
            device = t.device
        elif t.device != device:
            raise ValueError("libnqt kernels require CUDA tensors on one device")
    if device is None:
        raise ValueError("no tensor given")
    return device
