"""The connector's transport on CUDA devices: a rank's cache exported over CUDA IPC, peers' caches mapped, one kvx
launch per load on a side stream, completion by event, announced by a doorbell the transfer thread sleeps on.

It replaces the NIXL agent under NixlConnectorWorker call for call: register_memory/get_agent_metadata
(nixl_connector.py:240-244) -> `exported`; add_remote_agent (:510) -> open; initialize_xfer + transfer (:411-420)
-> post; check_xfer_state (:431) -> done; release_xfer_handle (:437) -> release; remove_remote_agent -> close.
"""

from __future__ import annotations

import os
import time

import torch

from lean_vllm_b200 import _native, envs
from lean_vllm_b200.kv_transfer import transport
from lean_vllm_b200.kv_transfer.transport import CacheTable, CopyJob

ENGINES = {"auto": _native.ENGINE_AUTO, "lsu": _native.ENGINE_LSU, "tma": _native.ENGINE_TMA}
RELAY_RING = 64  # interprocess events a decode rank marks its relayed parts with, reused in turn

# This process's own ring events by IPC handle, with their device: a peer rank in the same process on the same GPU
# uses them directly (CUDA cannot open an IPC handle in the process that exported it).
_OWN_RING_EVENTS: dict[str, tuple] = {}


class KvxTransport:
    def __init__(self, kv_caches: list[torch.Tensor]):
        if not kv_caches or not all(c.is_cuda for c in kv_caches):
            raise RuntimeError("CudaIpcConnector moves CUDA memory: every KV cache must be on a CUDA device")
        self.device = kv_caches[0].device
        if any(c.device != self.device for c in kv_caches):
            raise RuntimeError("one rank's KV caches must share one device")
        _native.lib()  # fail loudly here, at registration, if libkvx.so is missing
        self.local = CacheTable.from_tensors(kv_caches)
        engine = ENGINES.get(envs.LEAN_VLLM_KVX_ENGINE, _native.ENGINE_AUTO)
        self.engine = engine
        self.flags = _native.flags(engine)
        # A per-layer save runs beside the prefill's kernels: hold it to a few SMs.
        self.save_flags = _native.flags(engine, sm_budget=min(max(envs.LEAN_VLLM_KVX_SAVE_SMS, 0), 255))
        with torch.cuda.device(self.device):
            # Loads alternate between two streams: each writes its own blocks, so a launch may start while the one
            # before it drains, and a launch's tail no longer leaves SMs idle between consecutive loads.
            self.load_streams = [torch.cuda.Stream(device=self.device), torch.cuda.Stream(device=self.device)]
            self._lane = 0
            # Per-layer saves go first when SMs free up between the prefill's kernels.
            self.save_stream = torch.cuda.Stream(device=self.device, priority=-10)
            # A relayed load's copy from peer decode ranks runs beside the next loads' copies from the producer.
            self.relay_stream = torch.cuda.Stream(device=self.device)
        # Rung after every post: the transfer thread sleeps on it instead of polling copies in flight.
        self.doorbell = transport.Doorbell()
        # One IPC handle per layer tensor; each region as (tensor, byte offset in it, block bytes, head bytes).
        bases = [c.data_ptr() for c in kv_caches]
        spans = [(c.data_ptr(), c.data_ptr() + c.numel() * c.element_size()) for c in kv_caches]
        regions = []
        for addr, block_bytes, head_bytes in self.local.regions:
            index = next(i for i, (lo, hi) in enumerate(spans) if lo <= addr < hi)
            regions.append([index, addr - bases[index], block_bytes, head_bytes])
        with torch.cuda.device(self.device):
            handles = [transport.export(base).hex() for base in bases]
        self.exported = {
            "handles": handles,
            "regions": regions,
            "num_blocks": self.local.num_blocks,
            "device": self.device.index,
            "pid": os.getpid(),
        }

    def relay_ring(self) -> list[str]:
        """IPC handles (hex) of this rank's ring of interprocess events, created on first use: a relayed load's own
        part is marked with one (post's `mark`), and the peer decode ranks' copies of that part wait on it."""
        if getattr(self, "_ring", None) is None:
            with torch.cuda.device(self.device):
                self._ring = [torch.cuda.Event(interprocess=True) for _ in range(RELAY_RING)]
                self._ring_handles = [e.ipc_handle().hex() for e in self._ring]
            for handle, event in zip(self._ring_handles, self._ring):
                _OWN_RING_EVENTS[handle] = (event, self.device.index)
        return self._ring_handles

    def open_ring(self, handles: list[str]) -> list:
        """A peer rank's ring events, opened once -- or used directly when the peer lives in this process on this
        GPU. A peer in this process on another GPU gets no ring (an empty list): a stream waiting on such an event
        object crashed the process on this pool's B200s, so its parts are copied once it says they landed."""
        out = []
        for handle in handles:
            own = _OWN_RING_EVENTS.get(handle)
            if own is None:
                out.append(torch.cuda.Event.from_ipc_handle(self.device, bytes.fromhex(handle)))
            elif own[1] == self.device.index:
                out.append(own[0])
            else:
                return []
        return out

    def split_sms(self):
        """Relayed loads: copies from the producer and from peer decode ranks run at once on two streams, so each
        is held to half the SMs (a TMA copy CTA fills most of an SM's shared memory; a few dozen SMs already keep
        one NVLink direction full)."""
        half = max(1, torch.cuda.get_device_properties(self.device).multi_processor_count // 2)
        self.flags = _native.flags(self.engine, sm_budget=min(half, 255))

    def bind_thread(self):
        """CUDA's current device is per thread: the transfer thread works on the cache's device."""
        torch.cuda.set_device(self.device)

    def ready_marker(self):
        """An event after everything queued so far on the engine's stream (the reference's ready event, :266)."""
        return torch.cuda.current_stream(self.device).record_event()

    def open(self, exported: dict) -> CacheTable:
        bases = [transport.open_mapping(bytes.fromhex(h)) for h in exported["handles"]]
        regions = [(bases[i] + offset, block_bytes, head_bytes) for i, offset, block_bytes, head_bytes in
                   exported["regions"]]
        return CacheTable(regions, exported["num_blocks"])

    def close(self, exported: dict):
        for h in exported["handles"]:
            transport.close_mapping(bytes.fromhex(h))

    @staticmethod
    def _caches(local: CacheTable, tables: list[CacheTable], layer) -> list[CacheTable]:
        caches = [local, *tables]
        if layer is None:
            return caches
        start, count = layer
        return [CacheTable(c.regions[start : start + count], c.num_blocks) for c in caches]

    def job_bytes(self, tables: list[CacheTable], jobs: list[CopyJob], layer=None) -> int:
        """Bytes the jobs move (validated like the launch): the reference's descriptor-length sum (:421). Cache 0 of
        every job is this rank's own; cache k is tables[k-1]."""
        return transport.job_bytes(self._caches(self.local, tables, layer), jobs)

    def post(self, tables: list[CacheTable], jobs: list[CopyJob], ready, layer=None,
             flags: int | None = None, save: bool = False, relay: bool = False, mark: int | None = None,
             after: list | None = None, engine_order: bool = False) -> transport.Transfer:
        """One launch for all jobs, after `ready`, on a side stream. `layer` = (first region, region count)
        restricts every cache to one layer's regions. A push of a save (`save`) runs on the high-priority save
        stream, in order with the save's earlier pushes (a block pushed again must land after its older copy);
        `flags` holds a per-layer push to its SM budget. A relayed load's copy from its peers (`relay`) runs on a
        stream of its own, beside later loads' copies from the producer. Other loads alternate between the two load
        streams. `after`: events (a peer's ring) the launch also waits for; `mark`: the slot of this rank's ring
        recorded after the launch, for peers to wait on. `engine_order` (with `ready` None): the launch waits for
        everything queued so far on the calling thread's current stream, through the library's own event -- what a
        ready_marker would give, without creating one."""
        event = ready.cuda_event if ready is not None else 0
        if save or relay:
            stream = self.save_stream if save else self.relay_stream
        elif mark is not None:
            # A relayed load's own part: one stream for all of them, so with the peers' copies on the relay stream
            # two copies run at once, each on its half of the SMs (split_sms), as in the device-timed relay.
            stream = self.load_streams[0]
        else:
            stream = self.load_streams[self._lane]
            self._lane ^= 1
        if mark is not None:
            self.relay_ring()  # before the launch: a mark must never fail after the copy went out
        for peer_event in after or ():
            stream.wait_event(peer_event)
        engine = torch._C._cuda_getCurrentRawStream(self.device.index) if engine_order else None
        xfer = self._post_on(stream, tables, jobs, event, layer, flags, engine)
        if mark is not None:
            self._ring[mark].record(stream)
        return xfer

    def _post_on(self, stream, tables, jobs, event, layer=None, flags=None, after_stream=None) -> transport.Transfer:
        if torch.cuda.current_device() != self.device.index:
            # A launch goes to the calling thread's current device: an engine thread that posts for a rank whose
            # cache sits on another GPU (several ranks in one process) launches on the cache's device.
            with torch.cuda.device(self.device):
                return self._post_on(stream, tables, jobs, event, layer, flags, after_stream)
        xfer = transport.transfer(self._caches(self.local, tables, layer), jobs, stream.cuda_stream, event,
                                  self.flags if flags is None else flags, after_stream)
        self.doorbell.ring_after(stream.cuda_stream)
        return xfer

    def fences(self, ready) -> list:
        """One empty transfer after `ready` on every stream this transport copies on: once all have completed,
        nothing queued before `ready` on any of them still reads or writes a peer's memory."""
        event = ready.cuda_event if ready is not None else 0
        return [self._post_on(s, [], [], event)
                for s in (*self.load_streams, self.save_stream, self.relay_stream)]

    def fence(self, ready) -> transport.Transfer:
        """A transfer of nothing that completes once `ready` has: what a save whose layers were all stored fused
        (on the engine's stream) waits for before its decode instance hears that every byte landed."""
        return self.post([], [], ready, save=True)

    # The fused store-and-push (kvx_store), on the engine's stream.

    def new_block_map(self) -> torch.Tensor:
        """A device map from this cache's block ids to a decode instance's, all -1 (no block saved)."""
        return torch.full((self.local.num_blocks,), -1, dtype=torch.int32, device=self.device)

    def map_blocks(self, block_map: torch.Tensor, local_ids, remote_ids):
        """Enter (or with remote_ids None, clear) blocks of a save, in order on the engine's stream."""
        index = torch.as_tensor(list(local_ids), dtype=torch.long).to(self.device, non_blocking=True)
        if remote_ids is None:
            block_map.index_fill_(0, index, -1)
        else:
            block_map.index_copy_(0, index, torch.as_tensor(list(remote_ids), dtype=torch.int32).to(
                self.device, non_blocking=True))

    def push_target(self, table: CacheTable, first_region: int, share, block_map: torch.Tensor, block_size: int):
        """One decode rank's cache for one layer (its regions from first_region) as a store destination."""
        from lean_vllm_b200.attention.kvx_cache import PushTarget

        k_region = table.regions[first_region]
        v_region = table.regions[first_region + 1] if k_region[2] else None
        return PushTarget.of_regions(k_region, v_region, block_size, table.num_blocks, None,
                                     src_first_head=share.remote_head if k_region[2] else 0,
                                     num_heads=share.num_heads if k_region[2] else 1,
                                     dst_first_head=share.local_head if k_region[2] else 0, block_map=block_map)

    def status_word(self) -> transport.StatusWord:
        """A status word for a store whose rows also go to peers (kvx_status_open)."""
        return transport.StatusWord()

    def store(self, cache: torch.Tensor, key: torch.Tensor, value, slot_mapping: torch.Tensor, targets: list,
              async_push: bool = False, status: transport.StatusWord | None = None):
        """The layer's store into `cache` (HND keys/values, or latents when value is None) and every target;
        `status` gets bit 2 if a row was skipped because its slot lies past a cache. With `async_push`, one launch
        on the engine's stream writes the local cache (what attention waits for) and a second on the save stream,
        after it and held to the save SM budget, writes the targets from the same rows (KVX_STORE_PEERS_ONLY): the
        NVLink writes leave the prefill's critical path."""
        from lean_vllm_b200.attention.kvx_cache import store_kvcache, store_latents

        word = status.address if status is not None else 0

        def launch(push_to, stream=None, flags=0):
            if value is None:
                store_latents(key, cache[0], slot_mapping, push_to=push_to, stream=stream, flags=flags, status=word)
            else:
                view = cache.transpose(2, 3)  # (2, blocks, tokens, heads, dim), as the attention backend sees it
                store_kvcache(key, value, view[0], view[1], slot_mapping, push_to=push_to, stream=stream,
                              flags=flags, status=word)

        if not targets or not async_push:
            launch(targets)
            return
        launch([])
        self.save_stream.wait_event(torch.cuda.current_stream(self.device).record_event())
        for tensor in (key, value, slot_mapping):
            if tensor is not None:
                tensor.record_stream(self.save_stream)  # the engine may free them once its own store is queued
        budget = min(max(envs.LEAN_VLLM_KVX_SAVE_SMS, 0), 255)
        launch(targets, self.save_stream.cuda_stream, _native.flags(sm_budget=budget) | _native.STORE_PEERS_ONLY)

    def done(self, xfer: transport.Transfer) -> bool:
        return xfer.done()

    def wait(self, xfer: transport.Transfer):
        while not xfer.done():
            time.sleep(1e-4)

    def release(self, xfer: transport.Transfer):
        xfer.release()

    def drain(self):
        """Waits for everything queued on the cache's device, by any thread: before peers' mappings close."""
        torch.cuda.synchronize(self.device)

    def shutdown(self):
        """After every transfer was waited for: rings still queued then find the doorbell closed."""
        self.doorbell.close()
