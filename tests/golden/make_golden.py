"""Generates the golden fixtures in this folder by running lean-vLLM's own NixlConnectorWorker.

Run it where the reference checkout is importable (REFERENCE_ROOT, default: a "reference" folder beside this
repository):

    python tests/golden/make_golden.py

The reference's NIXL agent is replaced by MemmoveAgent below, which performs a READ as one memmove per descriptor
row over host memory, the way the reference's CPU tests model NIXL. Everything else -- head_shares, block_descs,
the ZMQ handshake, reader counting, byte counting -- is the reference's own code. The fixtures record the inputs, the
decode ranks' caches after the load, the byte counts, head_shares answers and raw block_descs rows. The GPU box does
not have the reference; tests there read only these files.
"""

from __future__ import annotations

import hashlib
import json
import os
import socket
import sys
from dataclasses import dataclass
from time import monotonic, sleep

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REFERENCE_ROOT = os.environ.get("REFERENCE_ROOT", os.path.join(HERE, "..", "..", "..", "reference"))
sys.dont_write_bytecode = True  # the reference tree is read-only
sys.path.insert(0, REFERENCE_ROOT)

from lean_vllm.kv_transfer import (  # noqa: E402
    KVConnectorMetadata,
    KVOutputAggregator,
    KVTransferConfig,
    ReqToRecv,
    nixl_connector,
)
from lean_vllm.kv_transfer.nixl_connector import NixlConnectorWorker, Region, block_descs, head_shares  # noqa: E402

sys.path.insert(0, os.path.join(HERE, "..", ".."))
from oracle.memmove_agent import MemmoveAgent  # noqa: E402  (the NIXL stand-in the reference's tests describe)


nixl_connector.make_agent = MemmoveAgent


@dataclass
class Cfg:
    kv_transfer: KVTransferConfig
    tensor_parallel_size: int = 1
    kvcache_block_size: int = 4
    kv_cache_layout: str = "HND"


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def seeded(shape, seed: int) -> torch.Tensor:
    generator = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=generator).to(torch.bfloat16)


def rank_part(full: torch.Tensor, rank: int, tp: int) -> torch.Tensor:
    if full.dim() == 4:
        return full.clone()
    heads = full.shape[2] // tp
    return full[:, :, rank * heads : (rank + 1) * heads].clone()


def side(role, tp, layers, block, port, engine_id, workers):
    out = []
    for rank in range(tp):
        cfg = Cfg(KVTransferConfig(kv_role=role, kv_port=port, engine_id=engine_id), tp, block)
        worker = NixlConnectorWorker(cfg, rank)
        worker.register_kv_caches([rank_part(full, rank, tp) for full in layers])
        out.append(worker)
    workers.extend(out)
    return out


def wait_for(worker, timeout=20.0):
    deadline = monotonic() + timeout
    while monotonic() < deadline:
        if output := worker.get_finished():
            return output
        sleep(0.002)
    raise AssertionError("no transfer finished")


def run_load(prefill_layers, decode_layers, prefill_tp, decode_tp, block, local_ids, remote_ids):
    """Runs one load through the reference workers; returns (per decode rank caches, per rank bytes)."""
    workers = []
    try:
        port = free_port()
        producers = side("kv_producer", prefill_tp, prefill_layers, block, port, "prefill", workers)
        consumers = side("kv_consumer", decode_tp, decode_layers, block, free_port(), "decode", workers)
        for producer in producers:
            producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(remote_ids)}))
        req = ReqToRecv(list(local_ids), list(remote_ids), "p-1", "prefill", "127.0.0.1", port, prefill_tp)
        for consumer in consumers:
            consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": req}))
        outputs = [wait_for(c) for c in consumers]
        aggregate = KVOutputAggregator(decode_tp).aggregate(outputs)
        assert aggregate.finished_recving == {"d-1"}, aggregate
        per_rank_bytes = [o.recv_stats["d-1"].num_bytes for o in outputs]
        sent = KVOutputAggregator(prefill_tp).aggregate([wait_for(p) for p in producers])
        assert sent.finished_sending == {"p-1"}
        caches = [[c.clone() for c in consumer.kv_caches] for consumer in consumers]
        return caches, per_rank_bytes
    finally:
        for worker in workers:
            worker.shutdown()


def as_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def full_from_ranks(rank_caches: list[torch.Tensor], mla: bool) -> torch.Tensor:
    return rank_caches[0] if mla else torch.cat(rank_caches, dim=2)


TP_PAIRS = [(1, 1), (2, 2), (1, 2), (2, 1), (1, 4), (4, 1), (2, 4), (4, 2), (4, 6), (6, 4), (2, 3)]


def small_cases(arrays: dict, meta: dict):
    """The reference tests' own shapes (12 blocks of 4 tokens, 12 heads of 8, latents 6 wide)."""
    blocks, block, heads, dim, latent = 12, 4, 12, 8, 6
    local, remote = [0, 5, 3], [7, 2, 9]
    cases = []
    for mla in (False, True):
        shape = (1, blocks, block, latent) if mla else (2, blocks, heads, block, dim)
        prefill, decode = seeded(shape, 0), seeded(shape, 1)
        key = "lat" if mla else "kv"
        arrays[f"small_{key}_prefill"] = as_bits(prefill)
        arrays[f"small_{key}_decode"] = as_bits(decode)
        for ptp, dtp in TP_PAIRS:
            caches, nbytes = run_load([prefill], [decode], ptp, dtp, block, local, remote)
            full = full_from_ranks([c[0] for c in caches], mla)
            name = f"small_{key}_tp{ptp}to{dtp}"
            arrays[name] = as_bits(full)
            cases.append(dict(name=name, mla=mla, prefill_tp=ptp, decode_tp=dtp, bytes_per_rank=nbytes))
    # A prefix hit: one block read of three, TP2 -> TP1 (tests/test_nixl_connector.py:256-267).
    shape = (2, blocks, heads, block, dim)
    prefill, decode = seeded(shape, 0), seeded(shape, 1)
    caches, nbytes = run_load([prefill], [decode], 2, 1, block, [8], [3])
    arrays["small_kv_prefix_hit"] = as_bits(caches[0][0])
    cases.append(dict(name="small_kv_prefix_hit", mla=False, prefill_tp=2, decode_tp=1, bytes_per_rank=nbytes,
                      local=[8], remote=[3]))
    # Nothing to read (a full prefix hit, :270-278).
    caches, nbytes = run_load([prefill], [decode], 1, 1, block, [], [])
    arrays["small_kv_empty"] = as_bits(caches[0][0])
    cases.append(dict(name="small_kv_empty", mla=False, prefill_tp=1, decode_tp=1, bytes_per_rank=nbytes,
                      local=[], remote=[]))
    meta["small"] = dict(blocks=blocks, block=block, heads=heads, dim=dim, latent=latent, local=local,
                         remote=remote, seeds=[0, 1], cases=cases)


def model_shaped_cases(meta: dict):
    """Qwen3-shaped key/value layers (8 heads of 128, 256-token blocks) and DeepSeek-V2-Lite-shaped latents (576
    wide, 64-token pages), two layers each, 10 blocks. Recorded as SHA-256 digests of the bf16 bit patterns."""
    blocks = 10
    local, remote = [9, 0, 4, 6, 1], [2, 7, 3, 8, 5]
    specs = [
        ("qwen_kv", False, (2, blocks, 8, 256, 128), [(1, 1), (2, 4), (1, 2), (4, 2)], 256),
        ("dsv2_lat", True, (1, blocks, 64, 576), [(1, 1), (1, 2), (2, 1)], 64),
    ]
    for key, mla, shape, pairs, block in specs:
        cases = []
        prefill = [seeded(shape, 10 + i) for i in range(2)]
        decode = [seeded(shape, 20 + i) for i in range(2)]
        inputs = dict(
            prefill=[hashlib.sha256(as_bits(t).tobytes()).hexdigest() for t in prefill],
            decode=[hashlib.sha256(as_bits(t).tobytes()).hexdigest() for t in decode],
        )
        for ptp, dtp in pairs:
            caches, nbytes = run_load(prefill, decode, ptp, dtp, block, local, remote)
            digests = []
            for layer in range(2):
                full = full_from_ranks([c[layer] for c in caches], mla)
                digests.append(hashlib.sha256(as_bits(full).tobytes()).hexdigest())
            cases.append(dict(name=f"{key}_tp{ptp}to{dtp}", mla=mla, prefill_tp=ptp, decode_tp=dtp,
                              bytes_per_rank=nbytes, layer_sha256=digests))
        meta[key] = dict(shape=list(shape), block=block, layers=2, prefill_seeds=[10, 11], decode_seeds=[20, 21],
                         local=local, remote=remote, input_sha256=inputs, cases=cases)


def shares_table(meta: dict):
    rows = []
    for heads in (8, 12, 24):
        sizes = [t for t in (1, 2, 3, 4, 6, 8, 12, 24) if heads % t == 0]
        for tp in sizes:
            for rtp in sizes:
                for rank in range(tp):
                    rows.append([rank, tp, rtp, heads, [list(s) for s in head_shares(rank, tp, rtp, heads)]])
    meta["head_shares"] = rows


def descs_table(meta: dict):
    """Raw block_descs rows on synthetic regions (addresses are plain integers here)."""
    regions = [Region(1 << 20, 4096, 512), Region(3 << 20, 4096, 512), Region(5 << 20, 1152, 0)]
    cases = []
    for first, num, latents in ((0, 8, False), (2, 3, True), (7, 1, True), (0, 0, False)):
        rows = block_descs(regions, [3, 0, 11, 5], first, num, latents, 1)
        cases.append(dict(first_head=first, num_heads=num, latents=latents, rows=rows.tolist()))
    meta["block_descs"] = dict(regions=[[r.addr, r.block_bytes, r.head_bytes] for r in regions],
                               block_ids=[3, 0, 11, 5], device_id=1, cases=cases)


def store_cases(arrays: dict, meta: dict):
    """The reference's per-token cache store (TorchAttention.store_kvcache / store_latents,
    attention/torch_backend.py:34-60, the CPU path of the Triton kernels in triton_cache.py) on NHD and HND caches
    and on latents, with padding slots (-1)."""
    from lean_vllm.attention.torch_backend import TorchAttention

    blocks, block, heads, dim, latent, tokens = 6, 4, 3, 8, 6, 10
    g = torch.Generator().manual_seed(5)
    slots = torch.randperm(blocks * block, generator=g)[:tokens].clone()
    slots[[2, 7]] = -1
    key = torch.randn(tokens, heads, dim, generator=g).to(torch.bfloat16)
    value = torch.randn(tokens, heads, dim, generator=g).to(torch.bfloat16)
    lat = torch.randn(tokens, latent, generator=g).to(torch.bfloat16)
    arrays["store_slots"] = slots.numpy().astype(np.int64)
    arrays["store_key"], arrays["store_value"], arrays["store_latent"] = as_bits(key), as_bits(value), as_bits(lat)
    for layout in ("NHD", "HND"):
        shape = (2, blocks, block, heads, dim) if layout == "NHD" else (2, blocks, heads, block, dim)
        cache = seeded(shape, 6)
        arrays[f"store_{layout}_before"] = as_bits(cache)
        view = cache if layout == "NHD" else cache.transpose(2, 3)  # what bind_kv_cache hands the backend
        TorchAttention.store_kvcache(None, key, value, view[0], view[1], slots)
        arrays[f"store_{layout}_after"] = as_bits(cache)
    cache = seeded((1, blocks, block, latent), 7)
    arrays["store_latent_before"] = as_bits(cache)
    TorchAttention.store_latents(None, lat, cache[0], slots)
    arrays["store_latent_after"] = as_bits(cache)
    meta["store"] = dict(blocks=blocks, block=block, heads=heads, dim=dim, latent=latent, tokens=tokens,
                         reference="lean_vllm/attention/torch_backend.py:34-60")


def main():
    arrays: dict = {}
    meta: dict = {"generator": "tests/golden/make_golden.py", "reference": "lean_vllm/kv_transfer/nixl_connector.py"}
    shares_table(meta)
    descs_table(meta)
    small_cases(arrays, meta)
    model_shaped_cases(meta)
    store_cases(arrays, meta)
    np.savez_compressed(os.path.join(HERE, "kv_transfer_small.npz"), **arrays)
    with open(os.path.join(HERE, "kv_transfer_golden.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote", len(arrays), "arrays and", len(meta), "tables")


if __name__ == "__main__":
    main()
