"""CPU restatement of the paged KV allocator and the talker metadata builder.

``HostPagePool`` follows PagedKVAllocator (executor/cache.py:86-212): a
sorted free list, scratch pages claimed first (:103-112), reserve serving
rows in order with the lowest free pages (:135-184), publish appending the
pages and advancing length/position (:199-207), discard returning the new
pages (:208-211), remove returning every page (:127-133).

``metadata`` follows PagedTalkerKV._metadata (executor/talker_kv.py:403-480):
indptr over proposed page counts, the proposed page lists, last_page_len =
total % P or P, per-token write page/offset and position, padding rows on
scratch page [row] with last_page_len 1 (prefill: qo_len 0; decode: one
write to slot 0, position 0), spare token slots spread over the scratch
pages.  Pure Python on small cases; test infrastructure only.
"""

from __future__ import annotations


class KVAllocationError(RuntimeError):
    pass


class HostPagePool:
    def __init__(self, total_pages: int, page_size: int, scratch_count: int) -> None:
        self.total_pages = total_pages
        self.page_size = page_size
        self.free = list(range(total_pages))
        self.scratch = tuple(self.free[:scratch_count])
        del self.free[:scratch_count]
        self.pages: dict[str, list[int]] = {}
        self.length: dict[str, int] = {}
        self.position: dict[str, int] = {}
        self.pending: dict[str, tuple[list[int], int]] = {}

    def add_request(self, rid: str) -> None:
        if rid in self.pages:
            raise ValueError(f"request {rid!r} already owns KV state")
        self.pages[rid] = []
        self.length[rid] = 0
        self.position[rid] = 0

    def remove_request(self, rid: str) -> None:
        self.free.extend(self.pages.pop(rid))
        self.free.sort()
        del self.length[rid], self.position[rid]

    def reserve(self, rids, advances) -> list[list[int]]:
        """New pages per row; raises KVAllocationError (and reserves nothing) on exhaustion."""

        allocated: list[int] = []
        out: list[list[int]] = []
        try:
            for rid, adv in zip(rids, advances, strict=True):
                need = (self.length[rid] + adv + self.page_size - 1) // self.page_size
                missing = need - len(self.pages[rid])
                if missing > len(self.free):
                    raise KVAllocationError(f"needs {missing} pages, {len(self.free)} free")
                new = self.free[:missing]
                del self.free[:missing]
                allocated.extend(new)
                out.append(new)
        except KVAllocationError:
            self.free.extend(allocated)
            self.free.sort()
            raise
        for rid, adv, new in zip(rids, advances, out, strict=True):
            self.pending[rid] = (new, adv)
        return out

    def publish(self, rid: str) -> None:
        new, adv = self.pending.pop(rid)
        self.pages[rid].extend(new)
        self.length[rid] += adv
        self.position[rid] += adv

    def discard(self, rid: str) -> None:
        new, _ = self.pending.pop(rid)
        self.free.extend(new)
        self.free.sort()

    def metadata(self, rids, advances, capture_rows: int, token_capacity: int, prefill: bool) -> dict:
        """Reserve and build the step's metadata as plain lists.

        Capture checks come first, as in prepare_prefill / prepare_decode and
        _validate_scratch_capacity (executor/talker_kv.py:397-401, 485-527)."""

        if len(rids) != len(advances) or not rids or len(rids) > capture_rows:
            raise ValueError("Talker request rows do not fit the capture")
        if prefill and sum(advances) > token_capacity:
            raise ValueError("Talker prefill tokens exceed the capture")
        if capture_rows > len(self.scratch):
            raise ValueError("Talker CUDA Graph rows exceed executor-private scratch pages")
        if token_capacity > len(self.scratch) * self.page_size:
            raise ValueError("Talker token capacity exceeds executor-private scratch slots")
        new_pages = self.reserve(rids, advances)
        p = self.page_size
        indptr, indices, last, positions, wpages, woffs, qo = [0], [], [], [], [], [], [0]
        for row in range(capture_rows):
            if row < len(rids):
                rid, adv = rids[row], advances[row]
                prior = self.length[rid]
                pages = self.pages[rid] + new_pages[row]
                total = prior + adv
                indices.extend(pages)
                indptr.append(len(indices))
                last.append(total % p or p)
                for i in range(adv):
                    absolute = prior + i
                    wpages.append(pages[absolute // p])
                    woffs.append(absolute % p)
                    positions.append(self.position[rid] + i)
                if prefill:
                    qo.append(qo[-1] + adv)
            else:
                scratch = self.scratch[row]
                indices.append(scratch)
                indptr.append(len(indices))
                last.append(1)
                if prefill:
                    qo.append(qo[-1])
                else:
                    wpages.append(scratch)
                    woffs.append(0)
                    positions.append(0)
        while len(positions) < token_capacity:
            slot = len(positions) - sum(advances)
            positions.append(0)
            wpages.append(self.scratch[slot // p])
            woffs.append(slot % p)
        if len(positions) != token_capacity:
            raise ValueError("Talker KV metadata exceeds the captured token capacity")
        return {
            "qo_indptr": qo if prefill else None,
            "paged_kv_indptr": indptr,
            "paged_kv_indices": indices,
            "paged_kv_last_page_len": last,
            "position_ids": positions,
            "write_pages": wpages,
            "write_offsets": woffs,
            "new_pages": new_pages,
        }
