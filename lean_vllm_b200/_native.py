"""ctypes binding of libkvx.so, the C ABI declared in include/kvx.h.

There is no fallback: if the library is missing or cannot load, every call raises KvxUnavailable, naming the build
step. The binding holds no torch types; callers pass raw device addresses and cudaStream_t values.
"""

from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkvx.so")

ABI_VERSION = 2  # KVX_ABI_VERSION of include/kvx.h

KVX_OK = 0
KVX_PENDING = 1
KVX_ERR_INVALID = -1
KVX_ERR_CUDA = -2
KVX_ERR_RANGE = -3
KVX_ERR_DEVICE = -4
KVX_ERR_TIMEOUT = -5

# Status word bits (kvx_status_open): what a launch reports when it fails without faulting.
STATUS_COPY_WAIT = 1  # a copy's bounded wait ran out: not every byte landed
STATUS_PAST_CACHE = 2  # a store row whose slot or block lies past its cache was skipped
STATUS_SELFTEST = 4  # kvx_wait_selftest gave up, as designed

STORE_SERIAL = 1  # kvx_store flag: a plain launch, no overlap with the kernel before it
STORE_PEERS_ONLY = 4  # kvx_store flag: only the peer destinations are written (destination 0 places their rows)

ENGINE_AUTO = 0
ENGINE_LSU = 1
ENGINE_TMA = 2


class KvxError(RuntimeError):
    """A kvx call returned an error status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"kvx error {code}: {message}")
        self.code = code


class KvxRangeError(KvxError):
    """A block id or head range outside its cache (nixl_connector.py:398-399)."""


class KvxDeviceError(KvxError):
    """A transfer's copy gave up a bounded wait, so its bytes did not all land (its own status word says so)."""


class KvxTimeout(KvxError):
    """A host wait ran out: a rank that never posted its step to the mailbox."""


class KvxUnavailable(RuntimeError):
    """libkvx.so is not built or cannot be loaded."""


class Region(ctypes.Structure):
    _fields_ = [("addr", ctypes.c_uint64), ("block_bytes", ctypes.c_uint64), ("head_bytes", ctypes.c_uint64)]


class Cache(ctypes.Structure):
    _fields_ = [("regions", ctypes.POINTER(Region)), ("n_regions", ctypes.c_int32), ("num_blocks", ctypes.c_int32)]


class Job(ctypes.Structure):
    _fields_ = [
        ("src_cache", ctypes.c_int32),
        ("dst_cache", ctypes.c_int32),
        ("src_block_ids", ctypes.POINTER(ctypes.c_int32)),
        ("dst_block_ids", ctypes.POINTER(ctypes.c_int32)),
        ("n_blocks", ctypes.c_int32),
        ("src_first_head", ctypes.c_int32),
        ("dst_first_head", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("latents", ctypes.c_int32),
    ]


class IpcHandle(ctypes.Structure):
    _fields_ = [
        ("handle", ctypes.c_ubyte * 64),
        ("offset", ctypes.c_uint64),
        ("alloc_bytes", ctypes.c_uint64),
        ("device", ctypes.c_int32),
        ("pid", ctypes.c_int32),
        ("ptr", ctypes.c_uint64),
        ("nonce", ctypes.c_ubyte * 16),
    ]

    def to_bytes(self) -> bytes:
        return ctypes.string_at(ctypes.addressof(self), ctypes.sizeof(self))

    @classmethod
    def from_bytes(cls, data: bytes) -> "IpcHandle":
        if len(data) != ctypes.sizeof(cls):
            raise ValueError(f"an IPC handle is {ctypes.sizeof(cls)} bytes, not {len(data)}")
        return cls.from_buffer_copy(data)


class StoreDest(ctypes.Structure):
    _fields_ = [
        ("k_cache", ctypes.c_uint64),
        ("v_cache", ctypes.c_uint64),
        ("block_stride", ctypes.c_int64),
        ("token_stride", ctypes.c_int64),
        ("head_stride", ctypes.c_int64),
        ("block_size", ctypes.c_int32),
        ("num_blocks", ctypes.c_int32),
        ("slot_mapping", ctypes.c_void_p),
        ("slot_bytes", ctypes.c_int32),
        ("src_first_head", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("dst_first_head", ctypes.c_int32),
        ("block_map", ctypes.c_void_p),
        ("block_map_len", ctypes.c_int32),
        ("pad_", ctypes.c_int32),
    ]


# Every symbol include/kvx.h declares, with its argtypes and restype.
_P = ctypes.c_void_p
SIGNATURES: dict[str, tuple[list, object]] = {
    "kvx_abi_version": ([], ctypes.c_int),
    "kvx_last_error": ([], ctypes.c_char_p),
    "kvx_ipc_export": ([_P, ctypes.POINTER(IpcHandle)], ctypes.c_int),
    "kvx_ipc_open": ([ctypes.POINTER(IpcHandle), ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "kvx_ipc_close": ([ctypes.POINTER(IpcHandle)], ctypes.c_int),
    "kvx_enable_peer_access": ([ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "kvx_copy": ([ctypes.POINTER(Cache), ctypes.c_int, ctypes.POINTER(Job), ctypes.c_int, ctypes.c_int, _P],
                 ctypes.c_int),
    "kvx_pack": ([ctypes.POINTER(Cache), ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int, _P, ctypes.c_uint64, ctypes.c_int, _P], ctypes.c_int),
    "kvx_push": ([_P, _P, ctypes.c_uint64, ctypes.c_int, _P], ctypes.c_int),
    "kvx_scatter": ([_P, ctypes.c_uint64, ctypes.POINTER(Cache), ctypes.POINTER(ctypes.c_int32), ctypes.c_int,
                     ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P], ctypes.c_int),
    "kvx_store": ([_P, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.POINTER(StoreDest), ctypes.c_int, _P, ctypes.c_int, _P], ctypes.c_int),
    "kvx_transfer": ([ctypes.POINTER(Cache), ctypes.c_int, ctypes.POINTER(Job), ctypes.c_int, ctypes.c_int, _P, _P,
                      ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "kvx_transfer_after": ([ctypes.POINTER(Cache), ctypes.c_int, ctypes.POINTER(Job), ctypes.c_int, ctypes.c_int, _P,
                            _P, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "kvx_check_xfer": ([_P], ctypes.c_int),
    "kvx_release_xfer": ([_P], ctypes.c_int),
    "kvx_xfer_status": ([_P, ctypes.POINTER(_P)], ctypes.c_int),
    "kvx_status_open": ([ctypes.POINTER(_P)], ctypes.c_int),
    "kvx_status_close": ([_P], ctypes.c_int),
    "kvx_status_read": ([_P, ctypes.POINTER(ctypes.c_int32)], ctypes.c_int),
    "kvx_doorbell_open": ([ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "kvx_doorbell_ring_after": ([ctypes.c_int, _P], ctypes.c_int),
    "kvx_doorbell_close": ([ctypes.c_int], ctypes.c_int),
    "kvx_mailbox_stride": ([ctypes.c_uint64], ctypes.c_uint64),
    "kvx_mailbox_bytes": ([ctypes.c_int, ctypes.c_uint64], ctypes.c_uint64),
    "kvx_mailbox_post": ([_P, ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, _P, ctypes.c_uint64,
                          ctypes.c_double], ctypes.c_int),
    "kvx_mailbox_collect": ([_P, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64),
                             ctypes.c_double], ctypes.c_int),
    "kvx_mailbox_release": ([_P, ctypes.c_uint64], ctypes.c_int),
    "kvx_job_bytes": ([ctypes.POINTER(Cache), ctypes.c_int, ctypes.POINTER(Job), ctypes.c_int,
                       ctypes.POINTER(ctypes.c_uint64)], ctypes.c_int),
    "kvx_device_error": ([ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "kvx_wait_selftest": ([ctypes.c_int, ctypes.c_int, _P, _P], ctypes.c_int),
    "kvx_launch_count": ([], ctypes.c_uint64),
}

_lib = None


def lib():
    """The loaded library; raises KvxUnavailable if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise KvxUnavailable(
                f"{LIB_PATH} is not built; run `python -c 'import __graft_entry__ as g; g.build()'` "
                "or `python -m lean_vllm_b200.build`"
            )
        try:
            handle = ctypes.CDLL(LIB_PATH)
        except OSError as error:
            raise KvxUnavailable(f"cannot load {LIB_PATH}: {error}") from error
        for name, (argtypes, restype) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = argtypes
            fn.restype = restype
        if handle.kvx_abi_version() != ABI_VERSION:
            raise KvxUnavailable(f"{LIB_PATH} has ABI {handle.kvx_abi_version()}, expected {ABI_VERSION}; rebuild it")
        _lib = handle
    return _lib


def check(rc: int) -> int:
    """Raises for an error status; returns KVX_OK or KVX_PENDING."""
    if rc >= 0:
        return rc
    message = lib().kvx_last_error().decode(errors="replace")
    raise {KVX_ERR_RANGE: KvxRangeError, KVX_ERR_TIMEOUT: KvxTimeout, KVX_ERR_DEVICE: KvxDeviceError}.get(
        rc, KvxError)(rc, message)


def flags(engine: int = ENGINE_AUTO, tile_bytes: int = 0, ctas_per_sm: int = 0, sm_budget: int = 0) -> int:
    """kvx_copy's flags word: engine, tile size (a power of two, 0 for the default), CTAs per SM, and how many SMs
    the grid may cover (0 for all; a copy beside compute can be held to a few)."""
    log_tile = 0
    if tile_bytes:
        log_tile = tile_bytes.bit_length() - 1
        if 1 << log_tile != tile_bytes:
            raise ValueError(f"tile_bytes {tile_bytes} is not a power of two")
    if not 0 <= ctas_per_sm < 256 or not 0 <= sm_budget < 256:
        raise ValueError("ctas_per_sm and sm_budget are 0..255")
    return engine | (log_tile << 8) | (ctas_per_sm << 16) | (sm_budget << 24)
