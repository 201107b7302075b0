"""The kvx transport: torch-facing wrappers over the C ABI (include/kvx.h).

Stands where NixlConnector's NIXL agent stands (lean_vllm/kv_transfer/nixl_connector.py:50-57): it exports a rank's
cache for peers (register_memory + agent metadata, :240-244), maps a peer's cache (add_remote_agent, :510), posts a
block copy (initialize_xfer + transfer, :411-420), and polls it (check_xfer_state, :431). Every data-moving call is
a CUDA kernel of libkvx.so; nothing here copies bytes on the host.
"""

from __future__ import annotations

import array
import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

from lean_vllm_b200 import _native
from lean_vllm_b200._native import Cache, IpcHandle, Job, Region, check, lib


_I32P = ctypes.POINTER(ctypes.c_int32)
assert array.array("i").itemsize == 4


def _ids(block_ids):
    """Block ids as (keep-alive buffer, int32* for the ABI, count). A list goes through array.array (a few us for
    hundreds of ids; numpy's ctypes accessor costs more than the rest of a launch's marshalling)."""
    if isinstance(block_ids, np.ndarray):
        a = np.ascontiguousarray(block_ids.reshape(-1), dtype=np.int32)
        return a, a.ctypes.data_as(_I32P), int(a.size)
    buf = array.array("i", block_ids)
    n = len(buf)
    return buf, ((ctypes.c_int32 * n).from_buffer(buf) if n else None), n


@dataclass
class CacheTable:
    """One rank's cache as kvx sees it: (addr, block_bytes, head_bytes) per K, V or latent region, in model order,
    plus the block count every region shares. `addrs` are device addresses in this process (a peer's are its
    kvx_ipc_open mapping)."""

    regions: list[tuple[int, int, int]]
    num_blocks: int
    _struct: Cache | None = field(default=None, repr=False, compare=False)
    _array: object = field(default=None, repr=False, compare=False)

    @classmethod
    def from_tensors(cls, kv_caches) -> "CacheTable":
        """Regions of per-layer caches, as register_kv_caches derives them (nixl_connector.py:224-235): a key/value
        layer is (2, blocks, heads, tokens, dim) HND, a latent layer (1, blocks, tokens, dim)."""
        regions, num_blocks = [], None
        for cache in kv_caches:
            if cache.dim() not in (4, 5):
                raise ValueError(f"a layer cache is 5-D (keys/values, HND) or 4-D (latents), not {cache.dim()}-D")
            if not cache.is_cuda:
                raise ValueError("kvx moves device memory; this cache is on the host")
            itemsize = cache.element_size()
            # What a share copies must be contiguous: a head's tokens (HND) or a whole latent block.
            if cache.stride(-1) != 1 or cache.stride(-2) != cache.size(-1):
                raise ValueError("each head's tokens (or each latent block) must be contiguous: an HND cache")
            for part in cache:
                head = part.stride(1) * itemsize if cache.dim() == 5 else 0
                regions.append((part.data_ptr(), part.stride(0) * itemsize, head))
            if num_blocks is None:
                num_blocks = cache.size(1)
            elif cache.size(1) != num_blocks:
                raise ValueError("every layer must hold the same number of blocks")
        return cls(regions, num_blocks or 0)

    def struct(self) -> Cache:
        if self._struct is None:
            array = (Region * max(len(self.regions), 1))(*[Region(a, b, h) for a, b, h in self.regions])
            self._array = array
            self._struct = Cache(ctypes.cast(array, ctypes.POINTER(Region)), len(self.regions), self.num_blocks)
        return self._struct


@dataclass
class CopyJob:
    """One READ: blocks of one request for one head share (kvx_job)."""

    src: int  # index of the source CacheTable in the call's list
    dst: int
    src_block_ids: object
    dst_block_ids: object
    src_first_head: int = 0
    dst_first_head: int = 0
    num_heads: int = 0
    latents: bool = False


_CACHE_ARRAYS: dict[tuple, tuple] = {}  # ids of a list of tables -> (the tables, their kvx_cache array)


def _cache_array(caches: list[CacheTable]):
    """The kvx_cache array of a list of tables, built once per list of the same (long-lived) tables: the entry
    holds the tables, so their ids cannot be reused while it exists."""
    key = tuple(map(id, caches))
    entry = _CACHE_ARRAYS.get(key)
    if entry is None or any(a is not b for a, b in zip(entry[0], caches)):
        if len(_CACHE_ARRAYS) >= 256:
            _CACHE_ARRAYS.clear()
        entry = _CACHE_ARRAYS[key] = (tuple(caches), (Cache * max(len(caches), 1))(*[c.struct() for c in caches]))
    return entry[1]


def _marshal(caches: list[CacheTable], jobs: list[CopyJob]):
    cache_array = _cache_array(caches)
    keep = [cache_array]
    job_array = (Job * max(len(jobs), 1))()
    for k, job in enumerate(jobs):
        src_buf, src_ptr, n_src = _ids(job.src_block_ids)
        dst_buf, dst_ptr, n_dst = _ids(job.dst_block_ids)
        if n_src != n_dst:
            raise ValueError(f"job {k} pairs {n_src} source blocks with {n_dst} destination blocks")
        keep += [src_buf, dst_buf, src_ptr, dst_ptr]
        job_array[k] = Job(
            job.src,
            job.dst,
            src_ptr,
            dst_ptr,
            n_src,
            job.src_first_head,
            job.dst_first_head,
            job.num_heads,
            int(job.latents),
        )
    keep.append(job_array)
    return cache_array, job_array, keep


def copy(caches: list[CacheTable], jobs: list[CopyJob], stream: int = 0, flags: int = 0) -> None:
    """Launches the paged-block copy of `jobs` on `stream` (a cudaStream_t as int)."""
    if not jobs:
        return
    cache_array, job_array, _keep = _marshal(caches, jobs)
    check(lib().kvx_copy(cache_array, len(caches), job_array, len(jobs), flags, stream))


def job_bytes(caches: list[CacheTable], jobs: list[CopyJob]) -> int:
    """Bytes the jobs move: the reference's descriptor-length sum (nixl_connector.py:421)."""
    if not jobs:
        return 0
    cache_array, job_array, _keep = _marshal(caches, jobs)
    out = ctypes.c_uint64()
    check(lib().kvx_job_bytes(cache_array, len(caches), job_array, len(jobs), ctypes.byref(out)))
    return out.value


class StatusWord:
    """A status word (kvx_status_open): 4 bytes of pinned host memory every device writes directly. A launch given
    one sets error bits there only if it fails without faulting; read it once the launch's event has completed."""

    def __init__(self):
        out = ctypes.c_void_p()
        check(lib().kvx_status_open(ctypes.byref(out)))
        self.address = out.value

    def bits(self) -> int:
        out = ctypes.c_int32()
        check(lib().kvx_status_read(self.address, ctypes.byref(out)))
        return out.value

    def close(self):
        """After every launch given the word has completed."""
        if self.address:
            check(lib().kvx_status_close(self.address))
            self.address = 0


class Transfer:
    """A posted copy and the event after it (a NIXL xfer handle), with a status word of its own."""

    def __init__(self, handle: int):
        self._handle = ctypes.c_void_p(handle)

    def done(self) -> bool:
        """True once every byte has landed; raises KvxDeviceError if one of this transfer's copies gave up."""
        return check(lib().kvx_check_xfer(self._handle)) == _native.KVX_OK

    def status_address(self) -> int:
        """The device-visible address of this transfer's status word (for kvx_wait_selftest in tests)."""
        out = ctypes.c_void_p()
        check(lib().kvx_xfer_status(self._handle, ctypes.byref(out)))
        return out.value

    def release(self):
        if self._handle:
            check(lib().kvx_release_xfer(self._handle))
            self._handle = ctypes.c_void_p(0)


def transfer(caches: list[CacheTable], jobs: list[CopyJob], stream: int, wait_event: int = 0,
             flags: int = 0, after_stream: int | None = None) -> Transfer:
    """Waits (on the stream) for `wait_event` -- or, given `after_stream`, for everything queued on that stream so
    far (kvx_transfer_after; 0 is the legacy default stream) -- launches the copy, records completion."""
    cache_array, job_array, _keep = _marshal(caches, jobs)
    out = ctypes.c_void_p()
    if after_stream is None:
        check(lib().kvx_transfer(cache_array, len(caches), job_array, len(jobs), flags, wait_event or None,
                                 stream or None, ctypes.byref(out)))
    else:
        check(lib().kvx_transfer_after(cache_array, len(caches), job_array, len(jobs), flags, after_stream or None,
                                       stream or None, ctypes.byref(out)))
    return Transfer(out.value)


class Doorbell:
    """An eventfd rung from a stream once the work queued before each ring has ended (kvx_doorbell_*): a thread
    polls `fd` beside its sockets and sleeps until a transfer lands."""

    def __init__(self):
        bell, fd = ctypes.c_int(), ctypes.c_int()
        check(lib().kvx_doorbell_open(ctypes.byref(bell), ctypes.byref(fd)))
        self.id, self.fd = bell.value, fd.value

    def ring_after(self, stream: int):
        check(lib().kvx_doorbell_ring_after(self.id, stream or None))

    def clear(self):
        """Takes the rings so far; the fd polls readable again at the next one."""
        try:
            os.eventfd_read(self.fd)
        except BlockingIOError:
            pass

    def close(self):
        if self.id:
            check(lib().kvx_doorbell_close(self.id))
            self.id = self.fd = 0


def pack(src: CacheTable, block_ids, first_head: int, num_heads: int, latents: bool, staging: int,
         staging_bytes: int, stream: int = 0, flags: int = 0) -> None:
    _keep, ids, n = _ids(block_ids)
    check(lib().kvx_pack(ctypes.byref(src.struct()), ids, n,
                         first_head, num_heads, int(latents), staging, staging_bytes, flags, stream))


def scatter(staging: int, staging_bytes: int, dst: CacheTable, block_ids, first_head: int, num_heads: int,
            latents: bool, stream: int = 0, flags: int = 0) -> None:
    _keep, ids, n = _ids(block_ids)
    check(lib().kvx_scatter(staging, staging_bytes, ctypes.byref(dst.struct()), ids, n, first_head, num_heads,
                            int(latents), flags, stream))


def push(dst: int, src: int, nbytes: int, stream: int = 0, flags: int = 0) -> None:
    check(lib().kvx_push(dst, src, nbytes, flags, stream))


def export(ptr: int) -> bytes:
    """An IPC handle for the allocation holding device address `ptr`, as bytes for a handshake."""
    handle = IpcHandle()
    check(lib().kvx_ipc_export(ptr, ctypes.byref(handle)))
    return handle.to_bytes()


def open_mapping(blob: bytes) -> int:
    """This process's address for a peer's exported pointer (on the current device)."""
    handle = IpcHandle.from_bytes(blob)
    out = ctypes.c_void_p()
    check(lib().kvx_ipc_open(ctypes.byref(handle), ctypes.byref(out)))
    return out.value or 0


def close_mapping(blob: bytes) -> None:
    check(lib().kvx_ipc_close(ctypes.byref(IpcHandle.from_bytes(blob))))


def enable_peer_access(device: int, peer: int) -> bool:
    out = ctypes.c_int()
    check(lib().kvx_enable_peer_access(device, peer, ctypes.byref(out)))
    return bool(out.value)


def launch_count() -> int:
    return int(lib().kvx_launch_count())


def wait_selftest(limit_us: int, code: int = 4, stream: int = 0, status: int = 0) -> None:
    """Launches the bounded-wait self-test (kvx_wait_selftest): after limit_us the device word has bit `code` set
    (4, the self-test's own; 1 stands in for a stuck copy), and so has the status word at `status` when given -- a
    transfer's own (Transfer.status_address), whose check then fails as if one of its copies had given up."""
    check(lib().kvx_wait_selftest(limit_us, code, status or None, stream or None))


def device_error() -> int:
    """Reads and clears, atomically on the device, the current device's diagnostic error word."""
    out = ctypes.c_int()
    check(lib().kvx_device_error(ctypes.byref(out)))
    return out.value
