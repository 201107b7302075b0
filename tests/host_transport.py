"""A host-memory stand-in for the kvx transport, for testing the connector's host logic on CPU. TEST ONLY.

It implements the transport surface CudaIpcConnectorWorker calls, with kvx_copy's byte map (include/kvx.h)
performed by memmove over CPU caches in this process, and it checks every range it touches against the registered
caches, so a wrong offset, head or block id in what the connector asks for either lands the wrong bytes or raises.
`fail` injects the two failures a transport can report: refused when posted, or failed in flight.
"""

from __future__ import annotations

import ctypes
from itertools import count


class HostStatusWord:
    """A status word in plain memory: bit 2 once a host store skipped a row."""

    opened = 0

    def __init__(self):
        self.value = 0
        HostStatusWord.opened += 1

    def bits(self) -> int:
        return self.value

    def close(self):
        HostStatusWord.opened -= 1


class HostTransport:
    fail: str | None = None  # "posted" or "in flight"
    instances: list["HostTransport"] = []

    def __init__(self, kv_caches):
        self.caches = list(kv_caches)
        self.spans = [(c.data_ptr(), c.numel() * c.element_size()) for c in self.caches]
        self.regions = []
        for cache in self.caches:
            itemsize = cache.element_size()
            for part in cache:
                head = part.stride(1) * itemsize if cache.dim() == 5 else 0
                self.regions.append((part.data_ptr(), part.stride(0) * itemsize, head))
        self.num_blocks = int(self.caches[0].size(1))
        self.exported = {"regions": self.regions, "num_blocks": self.num_blocks, "spans": self.spans}
        self.ids = count()
        self.pending: dict[int, list] = {}
        self.opened = 0
        self.closed: list[tuple] = []  # (exported, posts made by then) of every mapping closed
        self.posts: list[tuple] = []  # (layer, number of jobs) of every post, for tests to inspect
        self.stores: list[tuple] = []  # (number of peer targets, rows) of every store
        HostTransport.instances.append(self)

    def bind_thread(self):
        pass

    def ready_marker(self):
        return None

    def open(self, exported):
        self.opened += 1
        return exported

    def close(self, exported):
        self.opened -= 1
        self.closed.append((exported, len(self.posts)))

    def drain(self):
        pass

    def _tables(self, tables, layer):
        out = [self.exported, *tables]
        if layer is None:
            return out
        start, n = layer
        return [dict(t, regions=t["regions"][start : start + n]) for t in out]

    @staticmethod
    def _rows(table, block_ids, first_head, num_heads, latents):
        rows = []
        for addr, block_bytes, head_bytes in table["regions"]:
            if head_bytes:
                start, length = addr + first_head * head_bytes, num_heads * head_bytes
            elif latents:
                start, length = addr, block_bytes
            else:
                continue
            rows += [(start + b * block_bytes, length) for b in block_ids]
        return rows

    @staticmethod
    def _check(table, block_ids, rows):
        if any(b < 0 or b >= table["num_blocks"] for b in block_ids):
            raise RuntimeError("block id outside the cache")
        for addr, length in rows:
            if not any(lo <= addr and addr + length <= lo + n for lo, n in table["spans"]):
                raise RuntimeError("a row outside registered memory")

    def _pairs(self, tables, jobs, layer):
        caches = self._tables(tables, layer)
        for job in jobs:
            src, dst = caches[job.src], caches[job.dst]
            s_rows = self._rows(src, job.src_block_ids, job.src_first_head, job.num_heads, job.latents)
            d_rows = self._rows(dst, job.dst_block_ids, job.dst_first_head, job.num_heads, job.latents)
            self._check(src, job.src_block_ids, s_rows)
            self._check(dst, job.dst_block_ids, d_rows)
            assert [n for _, n in s_rows] == [n for _, n in d_rows]
            yield from zip(d_rows, s_rows)

    def job_bytes(self, tables, jobs, layer=None):
        return sum(n for (_, n), _ in self._pairs(tables, jobs, layer))

    def relay_ring(self):
        return [f"ring-{id(self)}-{slot}" for slot in range(64)]

    def open_ring(self, handles):
        return list(handles)

    def post(self, tables, jobs, ready, layer=None, flags=None, save=False, relay=False, mark=None, after=None,
             engine_order=False):
        """Host copies land when posted, so a mark needs no event and a wait on one is already satisfied."""
        if HostTransport.fail == "posted":
            raise RuntimeError("the transport refused the copy")
        for (dst, n), (src, _) in list(self._pairs(tables, jobs, layer)):
            ctypes.memmove(dst, src, n)
        self.posts.append((layer, len(jobs)))
        handle = next(self.ids)
        self.pending[handle] = [1]  # done on the second poll
        return handle

    def fences(self, ready):
        """An empty post per stream the GPU transport copies on (two load streams, save, relay)."""
        return [self.post([], [], ready) for _ in range(4)]

    def fence(self, ready):
        """Host stores are synchronous: a handle that completes like a post's, copying nothing."""
        handle = next(self.ids)
        self.pending[handle] = [1]
        return handle

    # The fused store-and-push, on host memory: kvx_store's byte map with slots and block maps.

    def new_block_map(self):
        import torch

        return torch.full((self.num_blocks,), -1, dtype=torch.int32)

    def map_blocks(self, block_map, local_ids, remote_ids):
        for i, b in enumerate(local_ids):
            block_map[b] = -1 if remote_ids is None else remote_ids[i]

    def push_target(self, table, first_region, share, block_map, block_size):
        k = table["regions"][first_region]
        v = table["regions"][first_region + 1] if k[2] else None
        heads = (share.remote_head, share.num_heads, share.local_head) if k[2] else (0, 1, 0)
        return {"k": k, "v": v, "heads": heads, "block_map": block_map, "block_size": block_size, "table": table}

    def status_word(self):
        return HostStatusWord()

    def store(self, cache, key, value, slot_mapping, targets, async_push=False, status=None):
        """kvx_store's byte map; a row whose mapped block lies past a target's cache is skipped and reported in
        `status` (bit 2), as the kernel does."""
        self.stores.append((len(targets), key.shape[0]))
        latents = value is None
        block = cache.size(2) if latents else cache.size(3)
        itemsize = key.element_size()
        row = (key.size(-1) if latents else key.size(-1)) * itemsize  # one head's (or latent's) bytes
        heads = 1 if latents else key.size(1)
        parts = [(key, 0)] if latents else [(key, 0), (value, 1)]
        for t, slot in enumerate(slot_mapping.tolist()):
            if slot < 0:
                continue
            b, off = divmod(int(slot), block)
            for rows, part in parts:
                for h in range(heads):
                    src = rows.data_ptr() + (t * heads + h) * row
                    local = cache[part, b] if latents else cache[part, b, h]
                    ctypes.memmove(local.data_ptr() + off * row, src, row)
                    for target in targets:
                        first, count, dst_first = target["heads"]
                        mapped = int(target["block_map"][b])
                        if mapped < 0 or not first <= h < first + count:
                            continue
                        if mapped >= target["table"]["num_blocks"]:
                            if status is not None:
                                status.value = 2
                            continue
                        addr, block_bytes, head_bytes = target["k"] if part == 0 else target["v"]
                        dst = addr + mapped * block_bytes + (h - first + dst_first) * head_bytes + off * row
                        self._check(target["table"], [mapped], [(dst, row)])
                        ctypes.memmove(dst, src, row)

    def done(self, handle):
        if HostTransport.fail == "in flight":
            raise RuntimeError("copy failed in flight")
        state = self.pending[handle]
        if state[0]:
            state[0] -= 1
            return False
        return True

    def wait(self, handle):
        pass

    def release(self, handle):
        self.pending.pop(handle, None)
