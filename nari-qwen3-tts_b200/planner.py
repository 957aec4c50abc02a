"""GPU planner: the page pool and the per-step attention metadata live on the
device (libnqt ``nqt_plan_*``), replacing ``PagedTalkerKV._metadata`` and
``PagedKVAllocator.reserve`` (executor/talker_kv.py:403-480,
executor/cache.py:86-212) for steps that must not round-trip to the host.

The host keeps only request bookkeeping: request id -> slot, and which rows
the next step covers.  Page ids, lengths and the free pool never leave the
device.  Allocation order is the reference's (rows in order, lowest free
page first), so for the same history the device produces the same page
tables, indptr, last-page lengths, positions and write slots as the
reference's host builder.

Step protocol (mirrors reserve -> replay -> publish/discard):
    planner.plan(binding, rows=[slot...], advances=[n...], prefill=...)
    ... run the captured step ...
    planner.commit(publish)     # publish all (or a per-row mask) / discard
Device errors (pool exhausted, bad slot) are reported in ``status`` and the
step's rows fall back to scratch pages, so nothing reads or writes outside
the pool; ``check()`` reads the status on the host when the caller chooses.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import call, ptr


class KVAllocationError(RuntimeError):
    pass


class DevicePagePlanner:
    def __init__(
        self,
        *,
        total_pages: int,
        page_size: int,
        slots: int,
        max_pages_per_slot: int,
        scratch_page_count: int,
        capture_rows: int,
        token_capacity: int,
        device: torch.device,
        num_qo_heads: int = 16,
        head_dim: int = 128,
    ) -> None:
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("DevicePagePlanner requires a CUDA device")
        if scratch_page_count < 1 or scratch_page_count > total_pages:
            raise ValueError("scratch page count must be a positive integer within the pool")
        if capture_rows > scratch_page_count:
            raise ValueError("Talker CUDA Graph rows exceed executor-private scratch pages")
        if token_capacity > scratch_page_count * page_size:
            raise ValueError("Talker token capacity exceeds executor-private scratch slots")
        self.total_pages = total_pages
        self.page_size = page_size
        self.slots = slots
        self.max_pages = max_pages_per_slot
        self.capture_rows = capture_rows
        self.token_capacity = token_capacity
        self.device = device
        self.num_qo_heads = num_qo_heads
        self.head_dim = head_dim
        lib = _lib.lib()
        self.state = torch.zeros(lib.nqt_planner_state_bytes(total_pages, slots, max_pages_per_slot),
                                 dtype=torch.uint8, device=device)
        # the reference claims the lowest pages as scratch (executor/cache.py:103-112)
        self.scratch_pages = torch.arange(scratch_page_count, dtype=torch.int32, device=device)
        self.padding_pages = tuple(range(scratch_page_count))
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.row_slot = torch.full((capture_rows,), -1, dtype=torch.int32, device=device)
        self.row_advance = torch.zeros(capture_rows, dtype=torch.int32, device=device)
        self.row_publish = torch.ones(capture_rows, dtype=torch.int32, device=device)
        self.pending = torch.zeros((capture_rows, max_pages_per_slot + 1), dtype=torch.int32, device=device)
        self._free_slots = list(range(slots))
        self._slot_of: dict[str, int] = {}
        with torch.cuda.device(device):
            call("nqt_planner_init", ptr(self.state), total_pages, slots, max_pages_per_slot,
                 scratch_page_count, _lib.stream_handle(device))

    def view(self, *, capture_rows: int, token_capacity: int) -> "DevicePagePlanner":
        """Another step shape (rows, token capacity) over the same page pool and
        request slots, with its own row and pending buffers: e.g. the prefill and
        the decode half of a mixed batch.  token_capacity 0 = allocation only."""

        if capture_rows > self.scratch_pages.numel():
            raise ValueError("Talker CUDA Graph rows exceed executor-private scratch pages")
        if token_capacity > self.scratch_pages.numel() * self.page_size:
            raise ValueError("Talker token capacity exceeds executor-private scratch slots")
        other = object.__new__(DevicePagePlanner)
        other.__dict__.update(self.__dict__)
        other.capture_rows = capture_rows
        other.token_capacity = token_capacity
        other.row_slot = torch.full((capture_rows,), -1, dtype=torch.int32, device=self.device)
        other.row_advance = torch.zeros(capture_rows, dtype=torch.int32, device=self.device)
        other.row_publish = torch.ones(capture_rows, dtype=torch.int32, device=self.device)
        other.pending = torch.zeros((capture_rows, self.max_pages + 1), dtype=torch.int32, device=self.device)
        return other

    # -- request bookkeeping (host) -------------------------------------------------
    def add_request(self, request_id: str) -> int:
        if not isinstance(request_id, str) or not request_id:
            raise ValueError("request_id must be a non-empty string")
        if request_id in self._slot_of:
            raise ValueError(f"request {request_id!r} already owns KV state")
        if not self._free_slots:
            raise KVAllocationError("no free request slot")
        slot = self._free_slots.pop(0)
        self._slot_of[request_id] = slot
        return slot

    def slot(self, request_id: str) -> int:
        try:
            return self._slot_of[request_id]
        except KeyError as error:
            raise KeyError(f"unknown Talker KV request {request_id!r}") from error

    def remove_request(self, request_id: str) -> None:
        slot = self.slot(request_id)
        self.release([slot])
        del self._slot_of[request_id]
        self._free_slots.append(slot)
        self._free_slots.sort()

    def release_rows(self) -> None:
        """Release every page of the slots in ``row_slot`` (device list, graph-capturable)."""

        with torch.cuda.device(self.device):
            call("nqt_plan_release", ptr(self.state), self.total_pages, self.slots, self.max_pages,
                 ptr(self.row_slot), self.capture_rows, ptr(self.status), _lib.stream_handle(self.device))

    def release(self, slots: list[int]) -> None:
        if not slots:
            return
        lst = torch.tensor(slots, dtype=torch.int32).to(self.device, non_blocking=True)
        with torch.cuda.device(self.device):
            call("nqt_plan_release", ptr(self.state), self.total_pages, self.slots, self.max_pages,
                 ptr(lst), len(slots), ptr(self.status), _lib.stream_handle(self.device))

    def import_pages(self, slot: int, pages: torch.Tensor, seq_len: int, pos_start: int | None = None) -> None:
        """Install an existing page list for ``slot`` (KV written elsewhere)."""

        pages = pages.to(device=self.device, dtype=torch.int32).contiguous()
        with torch.cuda.device(self.device):
            call("nqt_plan_import", ptr(self.state), self.total_pages, self.slots, self.max_pages,
                 int(slot), ptr(pages), pages.numel(), int(seq_len), int(seq_len if pos_start is None else pos_start),
                 ptr(self.status), _lib.stream_handle(self.device))

    # -- per step (device) ---------------------------------------------------------
    def set_rows(self, slots: list[int] | torch.Tensor, advances: list[int] | torch.Tensor) -> None:
        """Host helper: load the next step's rows (padding rows get slot -1)."""

        n = len(slots)
        if n > self.capture_rows or len(advances) != n:
            raise ValueError("Talker request rows do not fit the capture")
        row_slot = torch.full((self.capture_rows,), -1, dtype=torch.int32)
        row_adv = torch.zeros(self.capture_rows, dtype=torch.int32)
        row_slot[:n] = torch.as_tensor(slots, dtype=torch.int32)
        row_adv[:n] = torch.as_tensor(advances, dtype=torch.int32)
        self.row_slot.copy_(row_slot, non_blocking=True)
        self.row_advance.copy_(row_adv, non_blocking=True)

    def plan(self, binding, *, prefill: bool) -> None:
        """Reserve pages and write the step's metadata straight into the
        binding's static buffers, plus its split-KV partition (decode)."""

        if binding.capture_batch_size != self.capture_rows or binding.token_capacity != self.token_capacity:
            raise ValueError("binding capture shape differs from the planner's")
        with torch.cuda.device(self.device):
            call(
                "nqt_plan_step",
                ptr(self.state), self.total_pages, self.slots, self.max_pages, self.page_size,
                ptr(self.row_slot), ptr(self.row_advance), self.capture_rows, self.token_capacity,
                ptr(self.scratch_pages), self.scratch_pages.numel(), 1 if prefill else 0,
                ptr(binding.qo_indptr), ptr(binding.paged_kv_indptr), ptr(binding.paged_kv_indices),
                binding.paged_kv_indices.numel(),
                ptr(binding.paged_kv_last_page_len), ptr(binding.position_ids), ptr(binding.write_pages),
                ptr(binding.write_offsets), ptr(self.pending),
                None if prefill else ptr(binding.decode_workspace),
                0 if prefill else binding.decode_workspace.numel(),
                self.num_qo_heads, self.head_dim,
                ptr(self.status), _lib.stream_handle(self.device),
            )
        binding.bind_device_metadata(prefill=prefill, padding_pages=self.padding_pages)

    def plan_into(self, *, qo_indptr, kv_indptr, kv_indices, last_page_len, position_ids, write_pages,
                  write_offsets, prefill: bool, decode_workspace: torch.Tensor | None = None) -> None:
        """Same as ``plan`` with explicit output buffers (token buffers None:
        allocation only)."""

        with torch.cuda.device(self.device):
            call(
                "nqt_plan_step",
                ptr(self.state), self.total_pages, self.slots, self.max_pages, self.page_size,
                ptr(self.row_slot), ptr(self.row_advance), self.capture_rows, max(self.token_capacity, 1),
                ptr(self.scratch_pages), self.scratch_pages.numel(), 1 if prefill else 0,
                ptr(qo_indptr), ptr(kv_indptr), ptr(kv_indices), kv_indices.numel(),
                ptr(last_page_len), ptr(position_ids), ptr(write_pages), ptr(write_offsets), ptr(self.pending),
                ptr(decode_workspace), 0 if decode_workspace is None else decode_workspace.numel(),
                self.num_qo_heads, self.head_dim,
                ptr(self.status), _lib.stream_handle(self.device),
            )

    def commit(self, publish: bool | torch.Tensor = True) -> None:
        """Publish (True) or discard (False) the last plan, or per row with an
        int32 mask; device only, graph-capturable."""

        if isinstance(publish, torch.Tensor):
            self.row_publish.copy_(publish.to(torch.int32), non_blocking=True)
        else:
            self.row_publish.fill_(1 if publish else 0)
        with torch.cuda.device(self.device):
            call("nqt_plan_commit", ptr(self.state), self.total_pages, self.slots, self.max_pages,
                 ptr(self.row_slot), ptr(self.row_advance), ptr(self.row_publish), self.capture_rows,
                 ptr(self.pending), ptr(self.status), _lib.stream_handle(self.device))

    # -- inspection (host reads; synchronising) --------------------------------------
    def check(self) -> int:
        """Raise KVAllocationError if the device reported pool exhaustion."""

        status = int(self.status.item())
        if status & _lib.NQT_DEV_KV_EXHAUSTED:
            self.status.zero_()
            raise KVAllocationError("Talker KV page pool exhausted; the step reserved nothing")
        return status

    def _views(self):
        words = (self.total_pages + 31) // 32

        def a256(x: int) -> int:
            return (x + 255) // 256 * 256

        raw = self.state
        off = 0
        bitmap = raw[off: off + 4 * words].view(torch.int32)
        off = a256(off + 4 * words)
        seq_len = raw[off: off + 4 * self.slots].view(torch.int32)
        off = a256(off + 4 * self.slots)
        pos_start = raw[off: off + 4 * self.slots].view(torch.int32)
        off = a256(off + 4 * self.slots)
        n_pages = raw[off: off + 4 * self.slots].view(torch.int32)
        off = a256(off + 4 * self.slots)
        table = raw[off: off + 4 * self.slots * self.max_pages].view(torch.int32).view(self.slots, self.max_pages)
        return bitmap, seq_len, pos_start, n_pages, table

    def free_pages(self) -> int:
        bitmap = self._views()[0].cpu().numpy().view("uint32")
        return int(sum(bin(int(w)).count("1") for w in bitmap))

    def request_state(self, request_id: str) -> tuple[tuple[int, ...], int, int]:
        """(page_indices, sequence_length, position_start) of a request."""

        _, seq_len, pos_start, n_pages, table = self._views()
        s = self.slot(request_id)
        n = int(n_pages[s].item())
        return tuple(int(x) for x in table[s, :n].tolist()), int(seq_len[s].item()), int(pos_start[s].item())


__all__ = ["DevicePagePlanner", "KVAllocationError"]
