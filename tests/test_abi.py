"""CPU: libnqt.so loads and exports exactly what include/nqt.h declares, and
the ctypes signatures agree with the header (no compute calls: no GPU)."""

from __future__ import annotations

import re
from pathlib import Path

HEADER = Path(__file__).resolve().parents[1] / "include" / "nqt.h"


def header_prototypes() -> dict[str, int]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    protos = {}
    for m in re.finditer(r"^\s*(?:const\s+)?[\w\s\*]+?\b(nqt_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.M | re.S):
        args = m.group(2).strip()
        protos[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    return protos


def test_header_declares_the_hot_path():
    protos = header_prototypes()
    for name in ("nqt_qk_norm_rope_paged_kv_write", "nqt_decode_plan", "nqt_decode_attention",
                 "nqt_prefill_attention", "nqt_cp_decode_attention", "nqt_sample_rows", "nqt_sample_rows_noise",
                 "nqt_plan_step", "nqt_plan_commit"):
        assert name in protos


def test_library_exports_every_declared_symbol(nqt):
    lib = nqt.lib()
    for name in header_prototypes():
        assert hasattr(lib, name), name


def test_ctypes_signatures_match_header(nqt):
    from importlib import import_module

    sigs = import_module("nari-qwen3-tts_b200._lib").SIGNATURES
    protos = header_prototypes()
    assert set(sigs) == set(protos)
    for name, count in protos.items():
        assert len(sigs[name][1]) == count, name


def test_host_only_entry_points(nqt):
    lib = nqt.lib()
    assert lib.nqt_abi_version() == 1
    assert lib.nqt_decode_workspace_bytes(64, 16, 128) > 64 * 4
    assert lib.nqt_decode_workspace_bytes(0, 16, 128) == 0
    assert lib.nqt_planner_state_bytes(32768, 64, 256) >= 32768 // 8 + 64 * 256 * 4
    # argument errors are reported before any launch, without a device
    for name in ("nqt_decode_attention", "nqt_prefill_attention", "nqt_sample_rows", "nqt_plan_step",
                 "nqt_qk_norm_rope_paged_kv_write", "nqt_cp_decode_attention"):
        assert getattr(lib, name)(*null_args(name)) == -1, name


def null_args(name):
    import ctypes
    from importlib import import_module

    sigs = import_module("nari-qwen3-tts_b200._lib").SIGNATURES
    out = []
    for t in sigs[name][1]:
        out.append(None if t in (ctypes.c_void_p, ctypes.c_char_p) else 0)
    return out
