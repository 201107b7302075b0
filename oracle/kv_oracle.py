"""CPU oracle for the prefill->decode KV-cache transfer. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module, and only as the checker or
as the timed CPU baseline. The product path (lean_vllm_b200) never imports it and has no CPU fallback.

It restates, in plain Python and numpy, what lean-vLLM's NixlConnector computes for one load
(lean_vllm/kv_transfer/nixl_connector.py):

* head_shares     -- nixl_connector.py:69-77. Which producer ranks hold a consumer rank's key/value heads.
* block_descs     -- nixl_connector.py:89-108. The (address, length, device) rows of one side of a READ.
* read_rows       -- a NIXL READ as a byte copy of each (local, remote) row pair; the reference's CPU tests model
                     it the same way (tests/test_nixl_connector.py:83-89).
* plan_load       -- nixl_connector.py:388-421 (_start): the shares of one ReqToRecv, the rows of each share, the
                     reader count each producer rank waits for (:400-402) and the byte count (:421).
* expected_decode -- the tests' closed form of the result (tests/test_nixl_connector.py:223-226):
                     dst[:, local_ids] = src[:, remote_ids] on every rank's heads together.

Parity is pinned against golden fixtures made by running the reference connector itself over a memmove agent
(tests/golden/make_golden.py), and against the reference tests' own known answers.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np


class Share(NamedTuple):
    """The heads one consumer rank takes from one producer rank (nixl_connector.py:60-66)."""

    remote_rank: int
    remote_head: int  # first head, counted among the producer rank's own
    local_head: int  # where it lands, counted among the consumer rank's own
    num_heads: int


def head_shares(rank: int, tp_size: int, remote_tp_size: int, num_heads: int) -> list[Share]:
    """Overlap of consumer rank `rank`'s heads with each producer rank's, heads split evenly on both sides.

    Follows nixl_connector.py:69-77: the consumer rank holds heads [rank*h, (rank+1)*h) with h = num_heads/tp_size;
    producer rank q holds [q*g, (q+1)*g) with g = num_heads/remote_tp_size; one share per non-empty intersection.
    """
    mine = num_heads // tp_size
    theirs = num_heads // remote_tp_size
    lo, hi = rank * mine, (rank + 1) * mine
    out = []
    q = lo // theirs
    while q * theirs < hi:
        a = max(lo, q * theirs)
        b = min(hi, (q + 1) * theirs)
        out.append(Share(q, a - q * theirs, a - lo, b - a))
        q += 1
    return out


def lcm_heads(tp_size: int, remote_tp_size: int) -> int:
    """Pseudo-head count for latent caches, which every rank holds whole (nixl_connector.py:473-476)."""
    return math.lcm(tp_size, remote_tp_size)


@dataclass(frozen=True)
class Region:
    """One K, V or latent tensor as a read addresses it (nixl_connector.py:80-86)."""

    addr: int  # of block 0
    block_bytes: int  # stride between blocks
    head_bytes: int  # one head's tokens within a block; 0 for latents


def regions_of(caches) -> list[Region]:
    """Regions of a list of per-layer caches, as register_kv_caches derives them (nixl_connector.py:224-235).

    A cache is (2, blocks, heads, tokens, dim) for keys/values (HND) or (1, blocks, tokens, dim) for latents; each
    leading part is one region. Works on numpy arrays and torch tensors alike.
    """
    out = []
    for cache in caches:
        if hasattr(cache, "data_ptr"):  # torch
            itemsize = cache.element_size()
            for part in cache:
                head = part.stride(1) * itemsize if cache.dim() == 5 else 0
                out.append(Region(part.data_ptr(), part.stride(0) * itemsize, head))
        else:  # numpy
            for part in cache:
                head = part.strides[1] if cache.ndim == 5 else 0
                out.append(Region(part.ctypes.data, part.strides[0], head))
    return out


def block_descs(
    regions: list[Region], block_ids, first_head: int, num_heads: int, latents: bool, device_id: int = 0
) -> np.ndarray:
    """(address, length, device) rows, region-major, as nixl_connector.py:89-108 builds them.

    A key/value region contributes, per block, `num_heads` heads from `first_head`; a latent region contributes
    whole blocks if `latents`, else nothing.
    """
    ids = [int(b) for b in block_ids]
    rows = []
    for region in regions:
        if region.head_bytes:
            base = region.addr + first_head * region.head_bytes
            length = num_heads * region.head_bytes
        elif latents:
            base, length = region.addr, region.block_bytes
        else:
            continue
        for b in ids:
            rows.append((base + b * region.block_bytes, length, device_id))
    if not rows:
        return np.empty((0, 3), dtype=np.uint64)
    return np.asarray(rows, dtype=np.uint64)


def read_rows(local: np.ndarray, remote: np.ndarray) -> int:
    """A READ: copy each remote row's bytes to the local row paired with it. Returns the bytes moved."""
    assert local.shape == remote.shape
    moved = 0
    for (dst, length, _), (src, rlen, _) in zip(local.tolist(), remote.tolist()):
        assert length == rlen, "paired rows differ in length"
        ctypes.memmove(int(dst), int(src), int(length))
        moved += int(length)
    return moved


def place_rows(region_array: np.ndarray, block_ids, rows: np.ndarray, first_head: int, num_heads: int,
               latents: bool) -> int:
    """The scatter half of a staged transfer: contiguous staging rows, in block_descs order, written into one
    region's blocks. Row i of `rows` lands where block_descs([region], block_ids, first_head, num_heads, latents)
    row i points (nixl_connector.py:89-108), i.e. a READ whose remote side is the staging buffer. `region_array` is
    one K, V or latent tensor of a layer: (blocks, heads, tokens, dim) or (blocks, tokens, dim). Returns the bytes
    placed."""
    head_bytes = region_array.strides[1] if region_array.ndim == 4 else 0
    region = Region(region_array.ctypes.data, region_array.strides[0], head_bytes)
    local = block_descs([region], block_ids, first_head, num_heads, latents)
    rows = np.ascontiguousarray(rows)
    if len(local) == 0:
        return 0
    length = int(local[0, 1])
    assert rows.nbytes == length * len(local), "staging rows and block_descs rows differ in size"
    remote = np.asarray([(rows.ctypes.data + i * length, length, 0) for i in range(len(local))], dtype=np.uint64)
    return read_rows(local, remote)


@dataclass
class PlannedRead:
    """One READ the consumer rank posts: rows on both sides plus the notification the producer rank counts."""

    share: Share
    local: np.ndarray
    remote: np.ndarray
    readers: int  # consumer ranks that overlap this producer rank (nixl_connector.py:400-401)


def plan_load(
    rank: int,
    tp_size: int,
    remote_tp_size: int,
    num_heads: int,
    local_regions: list[Region],
    remote_regions_by_rank: dict[int, list[Region]],
    local_block_ids,
    remote_block_ids,
) -> tuple[list[PlannedRead], int]:
    """The reads one consumer rank posts for one ReqToRecv, and their byte count, as _start does
    (nixl_connector.py:388-421). `num_heads` is every rank's heads together, or 0 for a latent-only model."""
    heads = num_heads or lcm_heads(tp_size, remote_tp_size)
    shares = head_shares(rank, tp_size, remote_tp_size, heads)
    reads, total = [], 0
    for i, share in enumerate(shares):
        readers = len(head_shares(share.remote_rank, remote_tp_size, tp_size, heads))
        args = (share.num_heads, i == 0)  # latents come whole from the first producer rank only
        local = block_descs(local_regions, local_block_ids, share.local_head, *args)
        remote = block_descs(remote_regions_by_rank[share.remote_rank], remote_block_ids, share.remote_head, *args)
        reads.append(PlannedRead(share, local, remote, readers))
        total += int(local[:, 1].sum()) if len(local) else 0
    return reads, total


def rank_slice(full, rank: int, tp_size: int):
    """One rank's heads of a full (every rank's heads) key/value cache; a latent cache is whole on every rank."""
    if len(full.shape) == 4:
        return full
    heads = full.shape[2] // tp_size
    return full[:, :, rank * heads : (rank + 1) * heads]


def load_between(
    prefill_layers: list[np.ndarray],
    decode_layers: list[np.ndarray],
    prefill_tp: int,
    decode_tp: int,
    local_ids,
    remote_ids,
    copy=None,
) -> tuple[list[list[np.ndarray]], list[int]]:
    """Every decode rank's load of one request from every prefill rank, on host arrays.

    `prefill_layers`/`decode_layers` hold every rank's heads together (HND key/value or latent layers). Each side is
    split into per-rank contiguous arrays; each decode rank plans its reads as _start does and performs them with
    `copy(local_rows, remote_rows)` (default read_rows). Returns the decode ranks' layers and bytes per decode rank.
    """
    copy = copy or read_rows
    mla = prefill_layers[0].ndim == 4
    heads = 0 if mla else prefill_layers[0].shape[2]

    def split(layers, tp):
        out = []
        for rank in range(tp):
            if mla:
                out.append([np.array(a, copy=True, order="C") for a in layers])
            else:  # always a fresh array: the inputs are never written
                per = heads // tp
                out.append([np.array(a[:, :, rank * per : (rank + 1) * per], copy=True, order="C") for a in layers])
        return out

    producers = split(prefill_layers, prefill_tp)
    consumers = split(decode_layers, decode_tp)
    remote_regions = {q: regions_of(producers[q]) for q in range(prefill_tp)}
    moved = []
    for rank in range(decode_tp):
        reads, total = plan_load(
            rank, decode_tp, prefill_tp, heads, regions_of(consumers[rank]), remote_regions, local_ids, remote_ids
        )
        for read in reads:
            copy(read.local, read.remote)
        moved.append(total)
    return consumers, moved


def store_kvcache(key: np.ndarray, value: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, slot_mapping) -> None:
    """The per-token cache store, as TorchAttention.store_kvcache (attention/torch_backend.py:34-48): row t of
    key/value [tokens, heads, dim] goes to block slot // block_size, token slot % block_size of the caches, given as
    (blocks, block_size, heads, dim) views (an HND cache's transposed view works, the writes go through); slot -1
    skips the row."""
    block_size = k_cache.shape[1]
    for t, slot in enumerate(np.asarray(slot_mapping).tolist()):
        if slot < 0:
            continue
        block, offset = divmod(int(slot), block_size)
        k_cache[block, offset] = key[t]
        v_cache[block, offset] = value[t]


def store_latents(latent: np.ndarray, latent_cache: np.ndarray, slot_mapping) -> None:
    """TorchAttention.store_latents (attention/torch_backend.py:50-60): row t of latent [tokens, dim] goes to flat
    slot t of the (blocks, block_size, dim) cache; slot -1 skips."""
    flat = latent_cache.reshape(-1, latent_cache.shape[-1])
    for t, slot in enumerate(np.asarray(slot_mapping).tolist()):
        if slot >= 0:
            flat[int(slot)] = latent[t]


def expected_decode(prefill_full: np.ndarray, decode_full: np.ndarray, local_ids, remote_ids) -> np.ndarray:
    """The decode instance's full cache after the load: remote blocks copied onto local ones, all heads.

    The closed form the reference tests assert (tests/test_nixl_connector.py:223-226). Arrays may be any dtype; bf16
    caches are compared as uint16 bit patterns.
    """
    out = decode_full.copy()
    if len(local_ids):
        out[:, list(local_ids)] = prefill_full[:, list(remote_ids)]
    return out
