"""A cross-process host transport for CPU tests: caches live in /dev/shm files, which a peer maps. TEST ONLY.

The kvx transport exports a CUDA IPC handle per layer tensor and the peer maps it; this stand-in exports the shared
file behind each layer tensor instead, and the peer maps that file, so CudaIpcConnectorWorker's cross-process logic
(handshakes, mapped tables, reader notifications, pushes) runs between real processes without a GPU. Copies follow
kvx_copy's byte map through tests/host_transport.HostTransport.
"""

from __future__ import annotations

import mmap
import os
import uuid

import numpy as np
import torch

from tests.host_transport import HostTransport

_files: dict[int, tuple[str, int]] = {}  # tensor data_ptr -> (file, bytes), for caches made by shared_cache


def shared_cache(shape, fill: torch.Tensor | None = None, directory: str = "/dev/shm") -> torch.Tensor:
    """A bf16 tensor whose storage is a file other processes can map."""
    path = os.path.join(directory, f"kvx-test-{os.getpid()}-{uuid.uuid4().hex[:8]}")
    count = int(np.prod(shape))
    array = np.memmap(path, dtype=np.int16, mode="w+", shape=(count,))
    tensor = torch.from_numpy(array).view(torch.bfloat16).view(*shape)
    if fill is not None:
        tensor.copy_(fill)
    _files[tensor.data_ptr()] = (path, count * 2)
    tensor._kvx_keepalive = array  # the memmap must outlive the tensor's use
    return tensor


def remove_files():
    """Unlinks this process's shared cache files (mappings stay valid until they are closed)."""
    for path, _ in list(_files.values()):
        try:
            os.unlink(path)
        except FileNotFoundError:
            pass
    _files.clear()


class ShmTransport(HostTransport):
    def __init__(self, kv_caches):
        super().__init__(kv_caches)
        files = []
        for cache in self.caches:
            path, size = _files[cache.data_ptr()]
            files.append((path, size, cache.data_ptr()))
        regions = []
        for addr, block_bytes, head_bytes in self.regions:
            index = next(i for i, (_, size, base) in enumerate(files) if base <= addr < base + size)
            regions.append((index, addr - files[index][2], block_bytes, head_bytes))
        self.exported = dict(self.exported, files=[(p, s) for p, s, _ in files], relative=regions, pid=os.getpid())
        self._maps: dict[str, tuple] = {}

    def open(self, exported):
        self.opened += 1
        if exported.get("pid") == os.getpid():
            return exported
        bases = []
        for path, size in exported["files"]:
            if path not in self._maps:
                fd = os.open(path, os.O_RDWR)
                m = mmap.mmap(fd, size)
                os.close(fd)
                buffer = np.frombuffer(m, dtype=np.uint8)
                self._maps[path] = (m, buffer)
            bases.append(self._maps[path][1].ctypes.data)
        regions = [(bases[i] + off, bb, hb) for i, off, bb, hb in exported["relative"]]
        spans = [(bases[i], size) for i, (_, size) in enumerate(exported["files"])]
        return {"regions": regions, "num_blocks": exported["num_blocks"], "spans": spans}
