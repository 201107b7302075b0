"""ctypes binding of the C oracle (oracle/kvx_oracle.c). TEST INFRASTRUCTURE ONLY.

Used by tests/ as a second restatement of the reference's load, and by bench.py as the timed CPU baseline
(a NIXL READ restated as one memmove per descriptor row, rows spread over host threads).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

from oracle.kv_oracle import Region, Share

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libkvx_oracle.so")


class _Region(ctypes.Structure):
    _fields_ = [("addr", ctypes.c_uint64), ("block_bytes", ctypes.c_uint64), ("head_bytes", ctypes.c_uint64)]


def build() -> str:
    """Compile the C oracle with its Makefile if the library is missing or older than its source."""
    src = os.path.join(HERE, "kvx_oracle.c")
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        handle = ctypes.CDLL(LIB_PATH)
        handle.kvx_oracle_head_shares.restype = ctypes.c_int
        handle.kvx_oracle_head_shares.argtypes = [ctypes.c_int] * 4 + [ctypes.POINTER(ctypes.c_int), ctypes.c_int]
        handle.kvx_oracle_block_descs.restype = ctypes.c_int64
        handle.kvx_oracle_block_descs.argtypes = [
            ctypes.POINTER(_Region),
            ctypes.c_int,
            ctypes.POINTER(ctypes.c_int32),
            ctypes.c_int,
            ctypes.c_int,
            ctypes.c_int,
            ctypes.c_int,
            ctypes.POINTER(ctypes.c_uint64),
            ctypes.POINTER(ctypes.c_uint64),
            ctypes.c_int64,
        ]
        handle.kvx_oracle_read.restype = ctypes.c_int64
        handle.kvx_oracle_read.argtypes = [ctypes.POINTER(ctypes.c_uint64)] * 3 + [ctypes.c_int64, ctypes.c_int]
        _lib = handle
    return _lib


def head_shares(rank: int, tp_size: int, remote_tp_size: int, num_heads: int) -> list[Share]:
    out = (ctypes.c_int * (4 * 64))()
    n = lib().kvx_oracle_head_shares(rank, tp_size, remote_tp_size, num_heads, out, 64)
    return [Share(*out[4 * i : 4 * i + 4]) for i in range(n)]


def block_descs(regions: list[Region], block_ids, first_head: int, num_heads: int, latents: bool):
    """(addr, len) uint64 arrays, region-major."""
    table = (_Region * max(len(regions), 1))(*[_Region(r.addr, r.block_bytes, r.head_bytes) for r in regions])
    ids = np.ascontiguousarray(np.asarray(list(block_ids), dtype=np.int32))
    cap = max(len(regions) * len(ids), 1)
    addr = np.empty(cap, dtype=np.uint64)
    length = np.empty(cap, dtype=np.uint64)
    n = lib().kvx_oracle_block_descs(
        table,
        len(regions),
        ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
        len(ids),
        first_head,
        num_heads,
        int(latents),
        addr.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
        length.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
        cap,
    )
    return addr[:n].copy(), length[:n].copy()


def read(dst: np.ndarray, src: np.ndarray, length: np.ndarray, threads: int = 1) -> int:
    """memmove each row; returns bytes moved."""
    dst = np.ascontiguousarray(dst, dtype=np.uint64)
    src = np.ascontiguousarray(src, dtype=np.uint64)
    length = np.ascontiguousarray(length, dtype=np.uint64)
    assert dst.shape == src.shape == length.shape
    p = ctypes.POINTER(ctypes.c_uint64)
    moved = lib().kvx_oracle_read(
        dst.ctypes.data_as(p), src.ctypes.data_as(p), length.ctypes.data_as(p), len(dst), threads
    )
    if moved < 0:
        raise RuntimeError("kvx_oracle_read could not start its threads")
    return moved
