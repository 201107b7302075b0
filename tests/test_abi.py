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
    assert lib.kvx_abi_version() == _native.ABI_VERSION == 2
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
    with pytest.raises(_native.KvxRangeError, match="pass the end of a block"):  # no int32 wrap-around
        job_bytes([src, dst], [CopyJob(0, 1, [0], [0], 2**31 - 1, 0, 2**31 - 1)])
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
    assert ctypes.sizeof(h) == 64 + 8 + 8 + 4 + 4 + 8 + 16


def test_a_handle_with_this_pid_but_another_process_s_nonce_is_not_taken_for_local_memory():
    """Prefill and decode in separate containers can share a pid (each namespace has its own 1, 2, ...): a handle
    is used as a pointer of this process only when its pid AND its 16-byte process nonce both match. With the nonce
    wrong, kvx_ipc_open goes the IPC way -- which, with no device here, fails loudly instead of returning the
    other process's raw address -- and kvx_ipc_close finds no mapping to drop."""
    if not os.path.exists(_native.LIB_PATH):
        pytest.skip("libkvx.so is not built here")
    lib = _native.lib()
    h = _native.IpcHandle()
    h.pid, h.ptr, h.device = os.getpid(), 0xDEAD0000, 0
    for i in range(16):
        h.nonce[i] = i + 1  # not this process's nonce
    out = ctypes.c_void_p()
    rc = lib.kvx_ipc_open(ctypes.byref(h), ctypes.byref(out))
    assert rc < 0 and out.value != 0xDEAD0000
    assert lib.kvx_ipc_close(ctypes.byref(h)) < 0


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


def test_a_process_that_leaves_a_doorbell_open_still_exits_cleanly():
    """A process that ends on an exception before its connector shut down leaves its doorbell open: the library
    stops the doorbell's watcher at exit rather than abort (std::terminate on a joinable thread)."""
    if not os.path.exists(_native.LIB_PATH):
        pytest.skip("libkvx.so is not built here")
    import subprocess
    import sys

    code = ("from lean_vllm_b200.kv_transfer.transport import Doorbell\n"
            "bells = [Doorbell(), Doorbell()]\n"
            "raise SystemExit(3)\n")
    done = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert done.returncode == 3, done.stderr[-2000:]
    assert "terminate" not in done.stderr


def test_the_wait_selftest_checks_its_limit_before_launching():
    if not os.path.exists(_native.LIB_PATH):
        pytest.skip("libkvx.so is not built here")
    for bad in (0, -5, 10_000_001):
        with pytest.raises(_native.KvxError, match="limit"):
            _native.check(_native.lib().kvx_wait_selftest(bad, 4, None, None))
    for bad in (0, 2, 3, 8):
        with pytest.raises(_native.KvxError, match="the self-test's"):
            _native.check(_native.lib().kvx_wait_selftest(1000, bad, None, None))


C_CLIENT = r"""
#include <stdio.h>
#include <string.h>
#include "kvx.h"

/* What a C host binding does: describe caches and jobs in host memory and ask the library. */
int main(void) {
    kvx_region src_regions[2] = {{1ull << 40, 4096, 512}, {2ull << 40, 4096, 512}};
    kvx_region dst_regions[2] = {{3ull << 40, 2048, 512}, {4ull << 40, 2048, 512}};
    kvx_cache caches[2] = {{src_regions, 2, 10}, {dst_regions, 2, 6}};
    int32_t src_ids[2] = {9, 0}, dst_ids[2] = {5, 1}, bad_ids[1] = {6};
    kvx_job job = {0, 1, src_ids, dst_ids, 2, 2, 0, 4, 0};
    uint64_t bytes = 0;
    unsigned char box[4096];
    uint64_t lens[2];
    if (kvx_abi_version() != KVX_ABI_VERSION) return 1;
    if (kvx_job_bytes(caches, 2, &job, 1, &bytes) != KVX_OK || bytes != 2 * 2 * 4 * 512) return 2;
    job.dst_block_ids = bad_ids;
    job.src_block_ids = src_ids;
    job.n_blocks = 1;
    if (kvx_job_bytes(caches, 2, &job, 1, &bytes) != KVX_ERR_RANGE) return 3;
    if (strstr(kvx_last_error(), "destination block id 6") == NULL) return 4;
    /* One process as both ranks of a two-rank mailbox. */
    if (kvx_mailbox_bytes(2, 64) > sizeof box) return 5;
    memset(box, 0, sizeof box);
    if (kvx_mailbox_post(box, 2, 1, 64, 1, "done", 4, 1.0) != KVX_OK) return 6;
    if (kvx_mailbox_collect(box, 2, 64, 1, lens, 1.0) != KVX_OK || lens[1] != 4) return 7;
    if (memcmp(box + 64 + kvx_mailbox_stride(64) + 16, "done", 4) != 0) return 8;
    if (kvx_mailbox_release(box, 1) != KVX_OK) return 9;
    if (kvx_mailbox_post(box, 2, 1, 64, 3, "", 0, 0.05) != KVX_ERR_TIMEOUT) return 10; /* step 2 was never read */
    puts("ok");
    return 0;
}
"""


@pytest.mark.parametrize("compiler, standard, suffix", [("gcc", "-std=c99", ".c"), ("g++", "-std=c++17", ".cpp")],
                         ids=["c99", "c++17"])
def test_a_plain_client_compiles_against_the_header_and_runs_without_a_device(tmp_path, compiler, standard, suffix):
    """The boundary is C: the header compiles as strict C99 (and, through its extern "C" block, as C++17), and a
    program linked to libkvx.so gets the same answers the ctypes binding gets (host validation and the step mailbox
    need no GPU)."""
    import shutil
    import subprocess

    if not os.path.exists(_native.LIB_PATH):
        pytest.skip("libkvx.so is not built here")
    if shutil.which(compiler) is None:
        pytest.skip(f"no {compiler}")
    source = tmp_path / f"client{suffix}"
    source.write_text(C_CLIENT)
    binary = tmp_path / "client"
    lib_dir = os.path.dirname(_native.LIB_PATH)
    subprocess.run([compiler, standard, "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", os.path.join(ROOT, "include"),
                    str(source), "-o", str(binary), "-L", lib_dir, "-lkvx", f"-Wl,-rpath,{lib_dir}"],
                   check=True, capture_output=True, text=True)
    run = subprocess.run([str(binary)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.strip() == "ok", (run.returncode, run.stdout, run.stderr)


def test_the_binding_passes_as_many_arguments_as_each_prototype_takes():
    """The ctypes table and the header agree entry by entry -- parameter count and return type -- so a prototype
    that gains or loses a parameter cannot be called with the old argument list, nor a 64-bit result truncated."""
    with open(os.path.join(ROOT, "include", "kvx.h")) as f:
        text = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    found = re.findall(r"^(int|uint64_t|const char \*)\s*(kvx_\w+)\s*\(([^)]*)\)\s*;", text, flags=re.M)
    assert {name for _, name, _ in found} == set(_native.SIGNATURES)
    returns = {"int": ctypes.c_int, "uint64_t": ctypes.c_uint64, "const char *": ctypes.c_char_p}
    for ret, name, params in found:
        params = params.strip()
        count = 0 if params in ("", "void") else params.count(",") + 1
        argtypes, restype = _native.SIGNATURES[name]
        assert len(argtypes) == count, name
        assert restype is returns[ret], name
