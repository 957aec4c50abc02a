"""Talker attention binding on the sm_100a kernels: the drop-in for the
reference's FlashInfer bindings behind ``PagedTalkerKV(binding_factory=...)``.

``B200TalkerBinding`` implements the ``TalkerAttentionContext`` protocol
(executor/talker_kv.py:28-43): ``plan(metadata)``, ``select_layer(i)``,
``attend(attention, q, k, v)`` and ``advance_sequence_lengths()``.  It is
constructed with exactly the keyword arguments ``PagedTalkerKV._binding``
passes to a custom factory (executor/talker_kv.py:358-382) and serves both
capture kinds: metadata with ``qo_indptr`` is a ragged causal prefill,
without it a one-query decode (the two reference classes,
FlashInferPrefillBinding :140-226 and FlashInferDecodeBinding :229-306).

The factory is called with the same arguments for both kinds, so a binding
takes its kind from its first ``plan``: after that, prefill metadata on a
decode binding raises the reference decode binding's ValueError and decode
metadata on a prefill binding the reference prefill binding's.

Differences by design:
  * ``plan`` accepts host (pinned) or device metadata.  It copies it into
    the static buffers on the current stream and builds the split-KV
    partition on the device, so there is no host plan, no signature cache
    and nothing to invalidate: every ``plan`` rewrites the partition.
  * the split-KV plan and partials live at the start of the factory's
    per-slot ``workspace`` (the buffer the reference hands FlashInfer).
    Bindings of one slot share it the way the reference's do: a binding's
    ``plan`` must come before its replay, which the executor already does
    (executor/talker.py plans before every replay).  Without a workspace, or
    with one smaller than ``nqt_decode_workspace_bytes`` (about 10.6 MB at
    64 rows, 16 heads, D 128), the binding allocates its own.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Protocol

import torch

from . import _lib
from ._lib import call, ptr
from .kernels import device_status, paired_qk_norm_rope_paged_cache_

# nqt_decode_attention_ex flags (include/nqt.h NQT_DECODE_OVERLAP_KV_WRITE, NQT_DECODE_SHORT_WAIT)
DECODE_OVERLAP_KV_WRITE = 0x1
DECODE_SHORT_WAIT = 0x2


@dataclass(frozen=True, slots=True)
class TalkerAttentionMetadata:
    """Same fields as executor/talker_kv.py:15-25."""

    qo_indptr: torch.Tensor | None
    paged_kv_indptr: torch.Tensor
    paged_kv_indices: torch.Tensor
    paged_kv_last_page_len: torch.Tensor
    position_ids: torch.Tensor
    write_pages: torch.Tensor
    write_offsets: torch.Tensor
    padding_pages: tuple[int, ...]
    reuse_attention_plan: bool = True


class TalkerAttentionContext(Protocol):
    metadata: TalkerAttentionMetadata | None

    def plan(self, metadata: TalkerAttentionMetadata) -> None: ...

    def select_layer(self, index: int) -> None: ...

    def attend(self, attention: object, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> torch.Tensor: ...

    def advance_sequence_lengths(self) -> None: ...


def batch_decode_paged(
    query: torch.Tensor,
    layer_cache: torch.Tensor,
    kv_indptr: torch.Tensor,
    kv_indices: torch.Tensor,
    last_page_len: torch.Tensor,
    workspace: torch.Tensor,
    *,
    batch_capacity: int | None = None,
    sm_scale: float | None = None,
    out: torch.Tensor | None = None,
    plan: bool = True,
    overlap_kv_write: bool = False,
    short_wait: bool = False,
) -> torch.Tensor:
    """Paged GQA decode attention, one query per row (FlashInfer decode
    wrapper semantics: all (n_pages - 1) * P + last_page_len tokens).

    ``overlap_kv_write``: the kernel issued just before on this stream writes
    no KV tile but each row's last, and neither the page table nor the plan
    (the one-token-per-row K/V write of a decode step, or another decode
    launch on the same plan); the decode kernel then stages page ids and
    streams the older tiles while that kernel finishes.

    ``short_wait`` exists for failure-path tests only: the launch's pipeline
    waits give up at once, it reports NQT_DEV_TIMEOUT and its output is
    undefined, but the plan stays usable for the next launch."""

    rows, hq, d = query.shape
    pages, kinds, page_size, hkv, d2 = layer_cache.shape
    if kinds != 2 or d2 != d or hq % hkv:
        raise ValueError("paged decode shapes are incompatible")
    if query.dtype != torch.bfloat16 or layer_cache.dtype != torch.bfloat16:
        raise TypeError("paged decode runs on bf16 query and cache")
    if not layer_cache.is_contiguous() or query.stride(-1) != 1:
        raise ValueError("paged cache must be contiguous and query contiguous per head")
    cap = batch_capacity or rows
    device = _lib.require_cuda(query, layer_cache, kv_indptr, kv_indices, last_page_len, workspace)
    if out is None:
        out = torch.empty((rows, hq, d), dtype=query.dtype, device=device)
    stream = _lib.stream_handle(device)
    if plan:
        call(
            "nqt_decode_plan",
            ptr(kv_indptr), ptr(last_page_len), rows, cap, page_size, hq, d,
            ptr(workspace), workspace.numel() * workspace.element_size(), stream,
        )
    call(
        "nqt_decode_attention_ex",
        ptr(query), query.stride(0), query.stride(1),
        ptr(layer_cache), pages, page_size,
        ptr(kv_indptr), ptr(kv_indices), ptr(last_page_len),
        rows, cap, hq, hkv, d,
        float(sm_scale if sm_scale is not None else d**-0.5),
        ptr(out), out.stride(0), out.stride(1),
        ptr(workspace), workspace.numel() * workspace.element_size(),
        # a plan made just above is the previous kernel: it must be complete before anything is read
        (DECODE_OVERLAP_KV_WRITE if overlap_kv_write and not plan else 0) | (DECODE_SHORT_WAIT if short_wait else 0),
        ptr(device_status(device)), stream,
    )
    return out


def batch_prefill_paged(
    query: torch.Tensor,
    layer_cache: torch.Tensor,
    qo_indptr: torch.Tensor,
    kv_indptr: torch.Tensor,
    kv_indices: torch.Tensor,
    last_page_len: torch.Tensor,
    *,
    batch: int | None = None,
    sm_scale: float | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Ragged causal prefill over paged KV (FlashInfer prefill wrapper
    semantics, causal=True: query i of a qo_len chunk sees KV positions
    <= kv_len - qo_len + i)."""

    tokens, hq, d = query.shape
    pages, kinds, page_size, hkv, d2 = layer_cache.shape
    if kinds != 2 or d2 != d or hq % hkv:
        raise ValueError("paged prefill shapes are incompatible")
    if query.dtype != torch.bfloat16 or layer_cache.dtype != torch.bfloat16:
        raise TypeError("paged prefill runs on bf16 query and cache")
    if not layer_cache.is_contiguous() or query.stride(-1) != 1:
        raise ValueError("paged cache must be contiguous and query contiguous per head")
    rows = batch if batch is not None else qo_indptr.shape[0] - 1
    device = _lib.require_cuda(query, layer_cache, qo_indptr, kv_indptr, kv_indices, last_page_len)
    if out is None:
        out = torch.empty((tokens, hq, d), dtype=query.dtype, device=device)
    if tokens == 0:
        return out
    call(
        "nqt_prefill_attention",
        ptr(query), query.stride(0), query.stride(1),
        ptr(layer_cache), pages, page_size,
        ptr(qo_indptr), ptr(kv_indptr), ptr(kv_indices), ptr(last_page_len),
        rows, tokens, hq, hkv, d,
        float(sm_scale if sm_scale is not None else d**-0.5),
        ptr(out), out.stride(0), out.stride(1),
        ptr(device_status(device)), _lib.stream_handle(device),
    )
    return out


class B200TalkerBinding:
    """Attention context for one (capture key, slot) on the sm_100a kernels."""

    def __init__(
        self,
        *,
        storage: torch.Tensor,
        capture_batch_size: int,
        token_capacity: int,
        num_qo_heads: int,
        num_kv_heads: int,
        head_dim: int,
        page_size: int,
        total_pages: int,
        workspace: torch.Tensor | None = None,
        shared_plan_state: object | None = None,
        device: torch.device,
        dtype: torch.dtype,
        slot: int | None = None,
        metadata: TalkerAttentionMetadata | None = None,
        mode: str | None = None,
    ) -> None:
        """``mode`` ("decode" or "prefill") fixes the binding's kind up front;
        by default the first ``plan`` fixes it."""

        del shared_plan_state, slot  # no shared host plan: see the module docstring
        if mode not in (None, "decode", "prefill"):
            raise ValueError("mode must be 'decode', 'prefill' or None")
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("B200TalkerBinding requires a CUDA device")
        if workspace is not None and (workspace.dtype is not torch.uint8 or workspace.device != device):
            raise ValueError("Talker workspace must be a uint8 tensor on the execution device")
        if storage.ndim != 6 or storage.shape[2] != 2:
            raise ValueError("paged KV storage must be [layers, pages, 2, page_size, kv_heads, head_dim]")
        self.storage = storage
        self.capture_batch_size = capture_batch_size
        self.token_capacity = token_capacity
        self.num_qo_heads = num_qo_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.page_size = page_size
        self.total_pages = total_pages
        self.device = device
        self.dtype = dtype
        self.position_ids = torch.zeros(token_capacity, dtype=torch.long, device=device)
        self.write_pages = torch.zeros(token_capacity, dtype=torch.long, device=device)
        self.write_offsets = torch.zeros(token_capacity, dtype=torch.long, device=device)
        self.qo_indptr = torch.zeros(capture_batch_size + 1, dtype=torch.int32, device=device)
        self.paged_kv_indptr = torch.zeros(capture_batch_size + 1, dtype=torch.int32, device=device)
        self.paged_kv_indices = torch.zeros(total_pages + capture_batch_size, dtype=torch.int32, device=device)
        self.paged_kv_last_page_len = torch.ones(capture_batch_size, dtype=torch.int32, device=device)
        nbytes = _lib.lib().nqt_decode_workspace_bytes(capture_batch_size, num_qo_heads, head_dim)
        if mode == "prefill":
            self.decode_workspace = torch.empty(0, dtype=torch.uint8, device=device)
        elif workspace is not None and workspace.is_contiguous() and workspace.numel() >= nbytes:
            self.decode_workspace = workspace[:nbytes]
        else:
            self.decode_workspace = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        self.metadata: TalkerAttentionMetadata | None = None
        self._mode = mode
        self._prefill = mode == "prefill"
        self._layer_index = 0
        if metadata is not None:
            self.plan(metadata)

    # -- plan ------------------------------------------------------------------------
    def plan(self, metadata: TalkerAttentionMetadata) -> None:
        if metadata.paged_kv_indices.numel() > self.paged_kv_indices.numel():
            raise ValueError("Talker page metadata exceeds its captured buffer")
        if metadata.position_ids.shape != self.position_ids.shape:
            raise ValueError("Talker position metadata does not match the captured token capacity")
        if metadata.paged_kv_indptr.shape != self.paged_kv_indptr.shape:
            raise ValueError("Talker page metadata does not match the captured batch size")
        prefill = metadata.qo_indptr is not None
        self._fix_mode(prefill)
        with torch.cuda.device(self.device):
            self._copy(self.position_ids, metadata.position_ids)
            self._copy(self.write_pages, metadata.write_pages)
            self._copy(self.write_offsets, metadata.write_offsets)
            self._copy(self.paged_kv_indptr, metadata.paged_kv_indptr)
            n = metadata.paged_kv_indices.numel()
            self._copy(self.paged_kv_indices[:n], metadata.paged_kv_indices)
            self._copy(self.paged_kv_last_page_len, metadata.paged_kv_last_page_len)
            if prefill:
                self._copy(self.qo_indptr, metadata.qo_indptr)
            self._prefill = prefill
            self.metadata = metadata
            self.device_plan()

    def _fix_mode(self, prefill: bool) -> None:
        # the reference bindings' checks (executor/talker_kv.py:176-177, 260-261)
        if self._mode == "decode" and prefill:
            raise ValueError("Talker decode cannot contain packed query metadata")
        if self._mode == "prefill" and not prefill:
            raise ValueError("Talker prefill requires packed query metadata")
        if self._mode is None:
            self._mode = "prefill" if prefill else "decode"

    def device_plan(self) -> None:
        """Build the split-KV partition from the staged buffers (device only)."""

        if self._prefill:
            return
        call(
            "nqt_decode_plan",
            ptr(self.paged_kv_indptr), ptr(self.paged_kv_last_page_len),
            self.capture_batch_size, self.capture_batch_size, self.page_size,
            self.num_qo_heads, self.head_dim,
            ptr(self.decode_workspace), self.decode_workspace.numel(),
            _lib.stream_handle(self.device),
        )

    def bind_device_metadata(self, *, prefill: bool, padding_pages: tuple[int, ...] = ()) -> None:
        """Mark the static buffers (written in place by the GPU planner) as
        this step's metadata, without copies."""

        self._fix_mode(prefill)
        self._prefill = prefill
        self.metadata = TalkerAttentionMetadata(
            qo_indptr=self.qo_indptr if prefill else None,
            paged_kv_indptr=self.paged_kv_indptr,
            paged_kv_indices=self.paged_kv_indices,
            paged_kv_last_page_len=self.paged_kv_last_page_len,
            position_ids=self.position_ids,
            write_pages=self.write_pages,
            write_offsets=self.write_offsets,
            padding_pages=padding_pages,
        )

    @staticmethod
    def _copy(dst: torch.Tensor, src: torch.Tensor) -> None:
        non_blocking = src.device.type == "cuda" or src.is_pinned()
        dst.copy_(src.to(dst.dtype) if src.dtype != dst.dtype else src, non_blocking=non_blocking)

    # -- layer loop --------------------------------------------------------------------
    def select_layer(self, index: int) -> None:
        if not 0 <= index < self.storage.shape[0]:
            raise IndexError("Talker layer index exceeds paged KV storage")
        self._layer_index = index

    def attend(self, attention: object, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> torch.Tensor:
        layer = self.storage[self._layer_index]
        query, key = paired_qk_norm_rope_paged_cache_(
            query,
            key,
            value,
            attention.q_norm.weight,
            attention.k_norm.weight,
            self.position_ids,
            attention.q_norm.variance_epsilon,
            float(attention.rope_theta),
            layer,
            self.write_pages,
            self.write_offsets,
        )
        return self._run(query, layer).to(query.dtype)

    def _run(self, query: torch.Tensor, layer: torch.Tensor) -> torch.Tensor:
        if self._prefill:
            return batch_prefill_paged(
                query.to(self.dtype),
                layer,
                self.qo_indptr,
                self.paged_kv_indptr,
                self.paged_kv_indices,
                self.paged_kv_last_page_len,
                batch=self.capture_batch_size,
            )
        # attend() has just written each row's one new token (its last tile) with the K/V write kernel
        return batch_decode_paged(
            query.to(self.dtype),
            layer,
            self.paged_kv_indptr,
            self.paged_kv_indices,
            self.paged_kv_last_page_len,
            self.decode_workspace,
            batch_capacity=self.capture_batch_size,
            plan=False,
            overlap_kv_write=True,
        )

    @staticmethod
    def advance_sequence_lengths() -> None:
        # Replay proposes a KV publication; the engine owns committed lengths.
        return None


def binding_factory(**kwargs) -> B200TalkerBinding:
    """``PagedTalkerKV(binding_factory=binding_factory)`` hook."""

    return B200TalkerBinding(**kwargs)


__all__ = [
    "B200TalkerBinding",
    "TalkerAttentionContext",
    "TalkerAttentionMetadata",
    "batch_decode_paged",
    "batch_prefill_paged",
    "binding_factory",
]
