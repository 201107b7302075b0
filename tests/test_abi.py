"""The C ABI library loads without a GPU and exports every entry point include/kvx.h declares."""

import ctypes
import os
import re

import pytest

from lean_vllm_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared() -> set[str]:
    with open(os.path.join(ROOT, "include", "kvx.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(kvx_\w+)\s*\(", text))


def test_the_header_declares_the_bound_symbols():
    assert declared() == set(_native.SIGNATURES)


def test_the_library_loads_and_exports_every_declared_symbol():
    if not os.path.exists(_native.LIB_PATH):
        pytest.skip("libkvx.so is not built here")
    lib = _native.lib()
    for name in declared():
        assert getattr(lib, name) is not None
    assert lib.kvx_abi_version() == 1
    assert lib.kvx_last_error() == b""


def test_a_missing_library_raises_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIB_PATH", str(tmp_path / "libkvx.so"))
    with pytest.raises(_native.KvxUnavailable, match="is not built"):
        _native.lib()


def test_host_validation_runs_without_a_device():
    """Argument checks happen before any CUDA call, so they answer here too."""
    if not os.path.exists(_native.LIB_PATH):
        pytest.skip("libkvx.so is not built here")
    from lean_vllm_b200.kv_transfer.transport import CacheTable, CopyJob, job_bytes

    src = CacheTable([(1 << 40, 4096, 512), (2 << 40, 4096, 512)], 10)
    dst = CacheTable([(3 << 40, 2048, 512), (4 << 40, 2048, 512)], 6)
    assert job_bytes([src, dst], [CopyJob(0, 1, [9, 0], [5, 1], 2, 0, 4)]) == 2 * 2 * 4 * 512
    with pytest.raises(_native.KvxRangeError, match="destination block id 6"):
        job_bytes([src, dst], [CopyJob(0, 1, [9], [6], 2, 0, 4)])
    with pytest.raises(_native.KvxRangeError, match="pass the end of a block"):
        job_bytes([src, dst], [CopyJob(0, 1, [0], [0], 0, 1, 4)])
    with pytest.raises(_native.KvxError, match="outside the 2 given"):
        job_bytes([src, dst], [CopyJob(0, 2, [0], [0], 0, 0, 1)])


def test_flags_word():
    assert _native.flags() == 0
    assert _native.flags(_native.ENGINE_TMA, 1 << 15, 2) == 2 | (15 << 8) | (2 << 16)
    with pytest.raises(ValueError):
        _native.flags(tile_bytes=3000)


def test_ipc_handle_round_trips_as_bytes():
    h = _native.IpcHandle()
    h.offset, h.device, h.pid, h.ptr = 4096, 3, 77, 1 << 40
    back = _native.IpcHandle.from_bytes(h.to_bytes())
    assert (back.offset, back.device, back.pid, back.ptr) == (4096, 3, 77, 1 << 40)
    assert ctypes.sizeof(h) == 64 + 8 + 8 + 4 + 4 + 8


def test_a_doorbell_opens_and_closes_without_a_device():
    """Doorbells are host objects: opening gives a quiet non-blocking eventfd; a closed one refuses rings."""
    if not os.path.exists(_native.LIB_PATH):
        pytest.skip("libkvx.so is not built here")
    import select

    from lean_vllm_b200.kv_transfer.transport import Doorbell

    a, b = Doorbell(), Doorbell()
    assert a.id != b.id and a.fd != b.fd
    assert select.select([a.fd], [], [], 0)[0] == []  # not rung
    a.clear()  # nothing to take: no error, no block
    bell = a.id
    a.close()
    assert a.id == 0
    with pytest.raises(_native.KvxError, match="no open doorbell"):
        _native.check(_native.lib().kvx_doorbell_ring_after(bell, None))
    with pytest.raises(_native.KvxError, match="no open doorbell"):
        _native.check(_native.lib().kvx_doorbell_close(bell))
    b.close()


def test_the_wait_selftest_checks_its_limit_before_launching():
    if not os.path.exists(_native.LIB_PATH):
        pytest.skip("libkvx.so is not built here")
    for bad in (0, -5, 10_000_001):
        with pytest.raises(_native.KvxError, match="limit"):
            _native.check(_native.lib().kvx_wait_selftest(bad, None))
