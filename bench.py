"""Benchmark of the KV-cache transfer path: GB/s and ms per 8k-token request.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload pair|hetero|mla] [--mode pull|push]
                    [--engine auto|lsu|tma]
    python bench.py --impl reference ...      # the reference's CPU transfer path (restated in oracle/), host cores

Workloads (the benchmark's configurations; seeded N(0,1) bf16 caches, block ids from seeded shuffled free lists):
  pair    Qwen3-8B-shaped KV (36 layers x {K,V}, 8 KV heads x 128, 256-token blocks, HND), prefill TP1 -> decode TP1,
          64 requests, prompt lengths uniform in [1024, 8192]. N=1: same-device loopback on cuda:0 (HBM-bound);
          N even: N/2 independent pairs (ranks 2p -> 2p+1) over NVLink.
  hetero  Qwen3-8B-shaped KV, prefill TP2 -> decode TP4 (head resharding), 128 requests, lengths log-uniform in
          [512, 16384]; one group per 6 GPUs (prefill on the group's first 2 ranks, decode on its last 4).
  mla     DeepSeek-V2-Lite-shaped latents (27 layers x 576, 64-token pages), prefill TP1 -> decode TP2 (each decode
          rank takes a whole copy), 64 requests, lengths uniform in [2048, 16384]; one group per 3 GPUs.

One step moves every block of every request once: on each launching rank one kvx_copy with one job per (request,
head share). Groups are independent (weak scaling); no collective touches the data path.

`value` is device-timed (CUDA events on the launching stream, max over ranks) with the caches resident in HBM:
payload GB/s summed over decode ranks (the reference's byte count, nixl_connector.py:421 + base.py:106-108).
`e2e` times the same loads through the connector's public API (CudaIpcConnectorWorker.start_load_kv ->
get_finished) by the host clock. The caches exceed L2 by far, so no flush is needed between steps.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
import time
from dataclasses import dataclass

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from lean_vllm_b200 import envs  # noqa: E402  (settings only: no torch, no library load)

METRIC = "KV transfer GB/s & ms per 8k-token request"
BYTES_8K_REQUEST = 32 * 36 * 2 * 8 * 256 * 128 * 2  # 1,207,959,552: 32 blocks x 36 layers x K/V x 512 KiB
NVLINK_GBS = 900.0  # NVLink 5, per direction per GPU (nominal): the north star's link peak, the N >= 2 denominator


@dataclass(frozen=True)
class Workload:
    name: str
    layers: int
    kv_heads: int  # every rank's heads together; 0 for latents
    head_dim: int  # latent width for latents
    block: int
    prefill_tp: int
    decode_tp: int
    n_requests: int
    lengths: tuple  # (distribution, lo, hi)

    @property
    def mla(self) -> bool:
        return self.kv_heads == 0

    @property
    def group_size(self) -> int:
        return self.prefill_tp + self.decode_tp

    def describe(self) -> str:
        if self.mla:
            return f"{self.layers} layers x latent {self.head_dim}, page {self.block} tokens, bf16"
        return f"{self.layers} layers x {{K,V}}, {self.kv_heads} KV heads x {self.head_dim}, block {self.block} tokens, bf16, HND"


WORKLOADS = {
    "pair": Workload("qwen3-8b-kv", 36, 8, 128, 256, 1, 1, 64, ("uniform", 1024, 8192)),
    "hetero": Workload("qwen3-8b-kv", 36, 8, 128, 256, 2, 4, 128, ("loguniform", 512, 16384)),
    "mla": Workload("dsv2-lite-latent", 27, 0, 576, 64, 1, 2, 64, ("uniform", 2048, 16384)),
}


def workload(seed: int = 0, n_requests: int | None = None, spec: Workload = WORKLOADS["pair"]):
    """Prompt lengths and per-request (src, dst) block ids from seeded shuffled free lists. A smaller n_requests
    takes a prefix of the same draw."""
    rng = np.random.default_rng(seed)
    dist, lo, hi = spec.lengths
    if dist == "uniform":
        lengths = rng.integers(lo, hi + 1, size=spec.n_requests)
    else:
        lengths = np.exp(rng.uniform(np.log(lo), np.log(hi), size=spec.n_requests)).astype(np.int64)
    lengths = lengths[: n_requests or spec.n_requests]
    counts = [math.ceil(int(n) / spec.block) for n in lengths]
    total = sum(counts)
    num_blocks = total + max(8, total // 16)  # slack, so ids are spread over a larger cache
    src_free, dst_free = rng.permutation(num_blocks), rng.permutation(num_blocks)
    reqs, at = [], 0
    for c in counts:
        reqs.append((src_free[at : at + c].astype(np.int32), dst_free[at : at + c].astype(np.int32)))
        at += c
    return lengths, reqs, num_blocks


def chunk_bytes(spec: Workload, heads: int) -> int:
    if spec.mla:
        return spec.block * spec.head_dim * 2
    return heads * spec.block * spec.head_dim * 2


def request_bytes(n_blocks: int, spec: Workload = WORKLOADS["pair"]) -> int:
    """Payload of n_blocks for one decode rank holding every head (TP1)."""
    parts = 1 if spec.mla else 2
    return n_blocks * spec.layers * parts * chunk_bytes(spec, spec.kv_heads)


# ------------------------------------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi clock and throttle samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        self.out.flush()
        with open(self.out.name) as f:
            rows = [line.strip().split(", ") for line in f if line.strip()]
        os.unlink(self.out.name)
        sms, max_mhz, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for row in rows:
            if len(row) < 9:
                continue
            try:
                sms.append(float(row[1]))
                max_mhz = float(row[2])
            except ValueError:
                continue
            for name, value in zip(names, row[5:9]):
                if value.strip().lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sms)), "sm_max_mhz": max_mhz, "reasons": sorted(reasons),
                "samples": len(sms)}


# ------------------------------------------------------------------------------------------------ CPU baseline


def cpu_baseline(reqs, spec: Workload = WORKLOADS["pair"], seconds: float = 10.0, threads: int | None = None) -> dict:
    """The reference's CPU transfer path, restated in C (oracle/kvx_oracle.c): per request, block_descs rows for
    both sides, then one memmove per row, rows spread over host threads. Timed on a bounded sample: the first
    requests of the workload (at most 96 blocks) on host caches of the same shape (TP1 -> TP1), repeated for
    ~`seconds`."""
    from oracle import c_oracle
    from oracle.kv_oracle import Region

    threads = threads or len(os.sched_getaffinity(0))
    sample, blocks = [], 0
    for src, dst in reqs:
        if blocks + len(src) > 96 and sample:
            break
        sample.append((src, dst))
        blocks += len(src)
    nb = blocks
    if spec.mla:
        shape = (1, nb, spec.block, spec.head_dim)
    else:
        shape = (2, nb, spec.kv_heads, spec.block, spec.head_dim)
    src_caches = [np.full(shape, 0x3F80, dtype=np.uint16) for _ in range(spec.layers)]
    dst_caches = [np.zeros(shape, dtype=np.uint16) for _ in range(spec.layers)]
    for a in dst_caches:
        a.fill(1)  # touch every page before timing

    def regions(caches):
        return [Region(part.ctypes.data, part.strides[0], 0 if spec.mla else part.strides[1])
                for c in caches for part in c]

    src_r, dst_r = regions(src_caches), regions(dst_caches)
    remap, at = [], 0
    rng = np.random.default_rng(1)
    src_perm, dst_perm = rng.permutation(nb), rng.permutation(nb)
    for src, _ in sample:  # the sample's ids on sample-sized caches, still shuffled
        n = len(src)
        remap.append((src_perm[at : at + n], dst_perm[at : at + n]))
        at += n
    c_oracle.lib()
    heads = spec.kv_heads
    moved, reps = 0, 0
    start = time.perf_counter()
    while True:
        for src_ids, dst_ids in remap:
            d_addr, d_len = c_oracle.block_descs(dst_r, dst_ids, 0, heads, spec.mla)
            s_addr, _ = c_oracle.block_descs(src_r, src_ids, 0, heads, spec.mla)
            moved += c_oracle.read(d_addr, s_addr, d_len, threads)
        reps += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds or reps >= 200:
            break
    gbs = moved / elapsed / 1e9
    assert int(dst_caches[0][0, remap[0][1][0]].reshape(-1)[0]) == 0x3F80  # the copy happened
    return {
        "value": round(gbs, 3),
        "unit": "GB/s",
        "cores": threads,
        "kind": "port",
        "sample": (f"first {len(sample)} requests of the workload ({nb} blocks, {request_bytes(nb, spec) / 1e9:.2f} GB)"
                   f" on host caches of the same shape, {reps} passes in {elapsed:.1f} s; C restatement of "
                   "block_descs + one memmove per row, rows split over threads"),
        "ms_per_8k_request": round(BYTES_8K_REQUEST / (gbs * 1e9) * 1e3, 3),
        "host_cpus": os.cpu_count(),
    }


# ------------------------------------------------------------------------------------------------ topology


@dataclass
class Role:
    group: int
    side: str  # "prefill", "decode" or "idle" (or "both" for the 1-GPU loopback)
    tp_rank: int


def role_of(rank: int, world: int, spec: Workload) -> Role:
    if world == 1:
        if spec.group_size != 2:
            raise SystemExit(f"the {spec.name} workload needs {spec.group_size} GPUs")
        return Role(0, "both", 0)
    groups = world // spec.group_size
    if groups == 0:
        raise SystemExit(f"the {spec.name} workload needs {spec.group_size} GPUs per group, got {world}")
    group, index = divmod(rank, spec.group_size)
    if group >= groups:
        return Role(group, "idle", 0)
    if index < spec.prefill_tp:
        return Role(group, "prefill", index)
    return Role(group, "decode", index - spec.prefill_tp)


def plan(spec: Workload, role: Role, reqs, mode: str):
    """What one rank launches: (peers, jobs). Cache 0 of every job list is this rank's own cache; cache k >= 1 is
    peers[k-1] = (side, tp_rank) of the same group. Pull: a decode rank takes each of its shares from the prefill
    rank holding it. Push: a prefill rank writes every share it holds into each decode rank that reads it. Latent
    caches come whole from the first share only, as the reference reads them (nixl_connector.py:403)."""
    from lean_vllm_b200.kv_transfer.shares import head_shares, split_heads
    from lean_vllm_b200.kv_transfer.transport import CopyJob

    heads = split_heads(spec.kv_heads, spec.decode_tp, spec.prefill_tp)
    peers, jobs = [], []
    if role.side == "both":  # loopback: cache 0 is the source, cache 1 the destination
        shares = head_shares(0, 1, 1, heads)
        peers = [("decode", 0)]
        jobs = [CopyJob(0, 1, s, d, sh.remote_head, sh.local_head, sh.num_heads, i == 0)
                for s, d in reqs for i, sh in enumerate(shares)]
    elif role.side == "decode" and mode == "pull":
        shares = head_shares(role.tp_rank, spec.decode_tp, spec.prefill_tp, heads)
        for sh in shares:
            if ("prefill", sh.remote_rank) not in peers:
                peers.append(("prefill", sh.remote_rank))
        jobs = [CopyJob(1 + peers.index(("prefill", sh.remote_rank)), 0, s, d, sh.remote_head, sh.local_head,
                        sh.num_heads, i == 0) for s, d in reqs for i, sh in enumerate(shares)]
    elif role.side == "prefill" and mode == "push":
        for decode_rank in range(spec.decode_tp):
            shares = head_shares(decode_rank, spec.decode_tp, spec.prefill_tp, heads)
            mine = [(i, sh) for i, sh in enumerate(shares) if sh.remote_rank == role.tp_rank]
            if not mine:
                continue
            peers.append(("decode", decode_rank))
            jobs += [CopyJob(0, len(peers), s, d, sh.remote_head, sh.local_head, sh.num_heads, i == 0)
                     for s, d in reqs for i, sh in mine]
    return peers, jobs


RELAY_CHUNKS = 8  # request chunks a relayed step is pipelined over (--relay-chunks)


def plan_relay(spec: Workload, role: Role, reqs):
    """A decode rank's relayed latent load (LEAN_VLLM_KVX_RELAY): (peers, its own part of every request's blocks
    from the prefill rank, the other decode ranks' parts from them). Parts are contiguous 1/decode_tp slices of each
    request's blocks, as the connector cuts them."""
    from lean_vllm_b200.kv_transfer.transport import CopyJob

    from lean_vllm_b200.kv_transfer.cuda_ipc_connector import relay_parts

    peers = [("prefill", 0)] + [("decode", r) for r in range(spec.decode_tp) if r != role.tp_rank]
    own, others = [], []
    for s, d in reqs:
        parts = relay_parts(len(d), spec.decode_tp)
        me = role.tp_rank
        first, end = parts[me]
        if end > first:
            own.append(CopyJob(1, 0, s[first:end], d[first:end], 0, 0, 0, True))
        for r, (first, end) in enumerate(parts):
            if r != me and end > first:
                k = 1 + peers.index(("decode", r))
                others.append(CopyJob(k, 0, d[first:end], d[first:end], 0, 0, 0, True))
    return peers, own, others


def alloc_cache(spec: Workload, tp: int, num_blocks: int, device, fill: bool, seed: int):
    import torch

    if spec.mla:
        shape = (1, num_blocks, spec.block, spec.head_dim)
    else:
        shape = (2, num_blocks, spec.kv_heads // tp, spec.block, spec.head_dim)
    g = torch.Generator(device=device).manual_seed(seed)
    layers = []
    for _ in range(spec.layers):
        t = torch.empty(shape, dtype=torch.bfloat16, device=device)
        if fill:
            t.normal_(generator=g)
        else:
            t.zero_()
        layers.append(t)
    return layers


def load_traffic() -> dict:
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


def block_digests(layers, ids, first_head: int, num_heads: int, mla: bool, chunk: int = 128):
    """Per (layer, K|V or latent part, block) of `ids`: the sum and a position-weighted sum (odd 64-bit weights,
    wrapping) of the block's share -- heads [first_head, +num_heads), or the whole latent block -- as int16 words.
    Shape [layers, parts, len(ids), 2], on the cache's device. Every word of every listed block enters the digest
    and any single changed word changes the weighted sum (odd weights are invertible mod 2^64), so equal digests on
    both sides of a transfer mean every moved block landed where it should."""
    import torch

    device = layers[0].device
    index = torch.as_tensor(np.asarray(ids, dtype=np.int64), device=device)
    out = []
    weights = None
    for layer in layers:
        per_layer = []
        for at in range(0, len(ids), chunk):
            part = layer.index_select(1, index[at : at + chunk])
            if not mla:
                part = part[:, :, first_head : first_head + num_heads]
            flat = part.contiguous().view(torch.int16).reshape(part.shape[0], part.shape[1], -1).to(torch.int64)
            if weights is None or weights.numel() != flat.shape[-1]:
                weights = torch.arange(flat.shape[-1], device=device, dtype=torch.int64) * 2654435761 * 2 + 1
            per_layer.append(torch.stack([flat.sum(-1), (flat * weights).sum(-1)], -1))
        out.append(torch.cat(per_layer, 1))
    return torch.stack(out)


def measure_peer_copy(src_device: int, dst_device: int, nbytes: int = 1 << 30, reps: int = 5) -> float | None:
    """GB/s of one event-timed device-to-device copy of `nbytes` from src_device's memory into dst_device's, issued
    on dst_device (a copy engine pulling over NVLink, as cudaMemcpyPeerAsync does with peer access on), best of
    `reps`. No kvx kernel and no library kernel touches peer memory. None if the two cannot reach each other."""
    import torch

    from lean_vllm_b200.kv_transfer import transport

    if not transport.enable_peer_access(dst_device, src_device):
        return None
    src = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{src_device}")
    dst = torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{dst_device}")
    src.fill_(1)
    torch.cuda.synchronize(src_device)
    best = float("inf")
    with torch.cuda.device(dst_device):
        stream = torch.cuda.current_stream()
        for _ in range(reps + 1):
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            dst.copy_(src, non_blocking=True)
            end.record(stream)
            end.synchronize()
            best = min(best, start.elapsed_time(end))
    del src, dst
    torch.cuda.empty_cache()
    return nbytes / (best * 1e-3) / 1e9


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    from lean_vllm_b200._native import ENGINE_AUTO, ENGINE_LSU, ENGINE_TMA, flags
    from lean_vllm_b200.kv_transfer import transport
    from lean_vllm_b200.kv_transfer.shares import head_shares, split_heads
    from lean_vllm_b200.kv_transfer.transport import CacheTable, CopyJob

    spec = WORKLOADS[args.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}; launch N>1 with torchrun")
    role = role_of(rank, world, spec)
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    gloo = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
        gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=300))

    engine = {"auto": ENGINE_AUTO, "lsu": ENGINE_LSU, "tma": ENGINE_TMA}[args.engine]
    # Relayed: the copies from the prefill rank and from the peers run at once on two streams, half the SMs each.
    relay_sms = torch.cuda.get_device_properties(local_rank).multi_processor_count // 2 if args.relay else 0
    if args.relay and args.relay_sms >= 0:  # an explicit SM budget per relay stream (0: every SM)
        relay_sms = args.relay_sms
    copy_flags = flags(engine, args.tile_bytes, args.ctas_per_sm, relay_sms)
    lengths, reqs, num_blocks = workload(args.seed, args.requests, spec)
    step_blocks = sum(len(s) for s, _ in reqs)
    heads = split_heads(spec.kv_heads, spec.decode_tp, spec.prefill_tp)
    loopback = role.side == "both"
    groups = 1 if loopback else world // spec.group_size
    # --peer-device: one process, the destination cache on another GPU, peer access instead of IPC (the NVLink
    # path in a single process, for profilers that take one process).
    peer_mode = loopback and args.peer_device is not None
    dst_device = launch_device = device
    if peer_mode:
        dst_device = torch.device("cuda", args.peer_device)
        launch_device = dst_device if args.mode == "pull" else device
        other = device if args.mode == "pull" else dst_device
        if not transport.enable_peer_access(launch_device.index, other.index):
            raise SystemExit(f"cuda:{launch_device.index} cannot reach cuda:{other.index} directly")

    src = dst = None
    if role.side in ("prefill", "both"):
        src = alloc_cache(spec, spec.prefill_tp, num_blocks, device, fill=True, seed=1000 + rank)
    if role.side in ("decode", "both"):
        dst = alloc_cache(spec, spec.decode_tp, num_blocks, dst_device, fill=False, seed=0)
    torch.cuda.synchronize(device)
    torch.cuda.synchronize(dst_device)
    torch.cuda.set_device(launch_device)

    # Exchange every rank's cache description; map the peers this rank launches against.
    mine = src if role.side == "prefill" else dst
    info = [None] * world
    if world > 1:
        exported = [transport.export(t.data_ptr()) for t in mine] if mine is not None else []
        table = CacheTable.from_tensors(mine) if mine is not None else None
        dist.all_gather_object(info, (role.side, role.group, role.tp_rank, exported,
                                      table.regions if table else None, table.num_blocks if table else 0),
                               group=gloo)

    def rank_of(group: int, side: str, tp_rank: int) -> int:
        return group * spec.group_size + (tp_rank if side == "prefill" else spec.prefill_tp + tp_rank)

    opened: list[bytes] = []

    def peer_table(peer: int) -> CacheTable:
        _, _, _, blobs, regions, nb = info[peer]
        parts = 1 if spec.mla else 2
        out = []
        for layer, blob in enumerate(blobs):  # one exported tensor per layer: its K region, then V (or the latent)
            first = regions[parts * layer][0]
            here = transport.open_mapping(blob)
            opened.append(blob)
            for addr, bb, hb in regions[parts * layer : parts * layer + parts]:
                out.append((here + (addr - first), bb, hb))
        return CacheTable(out, nb)

    # Jobs: one per (request, share) on the launching rank; its peers' caches mapped over CUDA IPC.
    relay = args.relay and spec.mla and spec.decode_tp > 1 and not loopback
    if args.relay and not relay:
        raise SystemExit("--relay applies to the MLA workload's decode ranks (--workload mla, N >= 3)")
    relay_jobs = []
    relay_chunks = []  # (own-part jobs, peer-part jobs) per chunk of the step's requests
    if relay and role.side == "decode":
        chunk = max(1, -(-len(reqs) // (args.relay_chunks or RELAY_CHUNKS)))
        for first in range(0, len(reqs), chunk):
            peers, own, others = plan_relay(spec, role, reqs[first : first + chunk])
            relay_chunks.append((own, others))
        jobs = [j for own, _ in relay_chunks for j in own]
        relay_jobs = [j for _, others in relay_chunks for j in others]
    elif relay:
        peers, jobs = [], []
    else:
        peers, jobs = plan(spec, role, reqs, args.mode)
    launching = bool(jobs) or bool(relay_jobs)
    if loopback:
        caches = [CacheTable.from_tensors(src), CacheTable.from_tensors(dst)]
    elif launching:
        own = dst if role.side == "decode" else src
        caches = [CacheTable.from_tensors(own)] + [peer_table(rank_of(role.group, side, tp_rank))
                                                   for side, tp_rank in peers]
    else:
        caches = []
    my_bytes = (transport.job_bytes(caches, jobs) if jobs else 0) + \
        (transport.job_bytes(caches, relay_jobs) if relay_jobs else 0)
    stream = torch.cuda.Stream(device=launch_device)
    sid = stream.cuda_stream
    peer_stream = torch.cuda.Stream(device=launch_device)  # relayed: the copies from peer decode ranks

    # Relayed: one interprocess event per chunk on each decode rank, recorded once its own part of the chunk has
    # landed; its peers' second stream waits on it (on the GPU) before pulling that part from it. The host only
    # agrees that every rank recorded this step's events before any wait is enqueued -- it never waits for a copy.
    chunk_events, peer_events = [], []
    if relay:
        if role.side == "decode":
            chunk_events = [torch.cuda.Event(interprocess=True) for _ in relay_chunks]
        handles = [None] * world
        dist.all_gather_object(handles, (role.group, role.side, role.tp_rank,
                                         [e.ipc_handle() for e in chunk_events]), group=gloo)
        if role.side == "decode":
            peer_events = [[torch.cuda.Event.from_ipc_handle(launch_device, h) for h in hs]
                           for g, side, r, hs in handles if g == role.group and side == "decode" and r != role.tp_rank]

    def step():
        if not relay:
            if jobs:
                transport.copy(caches, jobs, sid, copy_flags)
            return
        # Pipelined by chunks of requests: every own part goes out from the prefill rank on the first stream, each
        # followed by its event; a chunk's parts from the peers go on the second stream once their events passed.
        for (own, _), event in zip(relay_chunks, chunk_events):
            if own:
                transport.copy(caches, own, sid, copy_flags)
            event.record(stream)
        dist.barrier(group=gloo)  # every decode rank has recorded this step's events
        for c, (_, others) in enumerate(relay_chunks):
            for events in peer_events:
                peer_stream.wait_event(events[c])
            if others:
                transport.copy(caches, others, peer_stream.cuda_stream, copy_flags)
        stream.wait_stream(peer_stream)  # the step ends when both streams have
        dist.barrier(group=gloo)  # every wait is enqueued before any rank records the events again

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()

    # The copy-engine peer copy between the pair's GPUs, measured on the consumer's side: reported beside the
    # link's nominal peak, never used as the denominator.
    peer_copy = None
    if world > 1 and role.side == "decode" and role.tp_rank == 0:
        producer = rank_of(role.group, "prefill", 0) % torch.cuda.device_count()
        peer_copy = measure_peer_copy(producer, local_rank)
        torch.cuda.set_device(launch_device)
    elif peer_mode:
        peer_copy = measure_peer_copy(device.index, dst_device.index)
        torch.cuda.set_device(launch_device)
    barrier()

    for _ in range(args.warmup):
        step()
    barrier()

    launches0 = transport.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(launch_device.index) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        barrier()
    launches = transport.launch_count() - launches0
    elapsed_ms = start.elapsed_time(end) if launching else 0.0
    stats = torch.tensor([elapsed_ms, float(launches), float(my_bytes), peer_copy or 0.0], device=device,
                         dtype=torch.float64)
    if world > 1:
        gathered = [torch.zeros_like(stats) for _ in range(world)]
        dist.all_gather(gathered, stats)
        stats_all = torch.stack(gathered).cpu().numpy()
    else:
        stats_all = stats.cpu().numpy()[None]
    max_ms = float(stats_all[:, 0].max())
    total_launches = int(stats_all[:, 1].sum())
    step_bytes_total = float(stats_all[:, 2].sum())  # payload per step over all decode ranks of all groups
    peer_copies = [float(v) for v in stats_all[:, 3] if v > 0]

    # Correctness over every byte the step moved: every block of every request, each decode rank's heads against
    # the producer rank that holds them. One GPU: the blocks compared outright. N GPUs: per-(layer, part, block)
    # digests of each share computed on both sides and compared.
    all_src = np.concatenate([s for s, _ in reqs])
    all_dst = np.concatenate([d for _, d in reqs])

    def verify() -> tuple[bool, int]:
        ok = True
        if loopback:
            s_index = torch.as_tensor(all_src, dtype=torch.long, device=src[0].device)
            d_index = torch.as_tensor(all_dst, dtype=torch.long, device=dst[0].device)
            for a, b in zip(src, dst):
                ok &= bool(torch.equal(a.index_select(1, s_index), b.index_select(1, d_index).to(a.device)))
            return ok, int(len(all_src) * len(src))
        if world == 1:
            return ok, 0
        mine_digests = {}
        if role.side == "decode":
            for i, sh in enumerate(head_shares(role.tp_rank, spec.decode_tp, spec.prefill_tp, heads)):
                if spec.mla and i:
                    continue
                mine_digests[(role.tp_rank, i)] = block_digests(dst, all_dst, sh.local_head, sh.num_heads,
                                                                spec.mla).cpu()
        elif role.side == "prefill":
            for decode_rank in range(spec.decode_tp):
                for i, sh in enumerate(head_shares(decode_rank, spec.decode_tp, spec.prefill_tp, heads)):
                    if sh.remote_rank != role.tp_rank or (spec.mla and i):
                        continue
                    mine_digests[(decode_rank, i)] = block_digests(src, all_src, sh.remote_head, sh.num_heads,
                                                                   spec.mla).cpu()
        every = [None] * world
        dist.all_gather_object(every, (role.group, role.side, mine_digests), group=gloo)
        checked = 0
        for group in range(groups):
            got = {k: v for g, side, d in every if g == group and side == "decode" for k, v in d.items()}
            want = {k: v for g, side, d in every if g == group and side == "prefill" for k, v in d.items()}
            ok &= bool(got) and got.keys() == want.keys() and all(torch.equal(got[k], want[k]) for k in got)
            checked += sum(v.shape[0] * v.shape[2] for v in got.values())
        return ok, checked

    ok, checked = verify()

    # e2e: the same loads through the connector's public API.
    e2e_ms, e2e_bytes = None, 0
    e2e_ok = None
    if args.steps and not args.no_e2e and not peer_mode:
        # The decode caches start from zeros, so the check after these loads sees what the connector moved.
        if dst is not None:
            for layer in dst:
                layer.zero_()
            torch.cuda.synchronize(dst[0].device)
        e2e_launches0 = transport.launch_count()
        e2e_ms, e2e_bytes = e2e_connector(args, spec, world, rank, role, src, dst, reqs, gloo)
        e2e_launches = transport.launch_count() - e2e_launches0
        e2e_ok, _ = verify()
        e = torch.tensor([e2e_ms, float(e2e_bytes), float(e2e_launches)], device=device, dtype=torch.float64)
        if world > 1:
            gathered = [torch.zeros_like(e) for _ in range(world)]
            dist.all_gather(gathered, e)
            e_all = torch.stack(gathered).cpu().numpy()
        else:
            e_all = e.cpu().numpy()[None]
        e2e_ms, e2e_bytes = float(e_all[:, 0].max()), int(e_all[:, 1].sum())
        e2e_launches = int(e_all[:, 2].sum())  # every rank's (a pull's producers launch none)

    ok_t = torch.tensor([0.0 if ok else 1.0, 0.0 if e2e_ok in (True, None) else 1.0], device=device,
                        dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ok_t, op=dist.ReduceOp.MAX)
    clock_summary = clocks.summary()
    # One GPU: the per-token store (a12) and the layer-wise push beside a prefill (a13), each in a child process of
    # its own once this run's caches are freed, so this line carries them from the same run.
    extras = {}
    if loopback and not peer_mode and not args.no_extras and rank == 0:
        src = dst = mine = None  # the caches: the children need the memory
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        extras = measure_extras(args)

    if rank == 0:
        ms_per_step = max_ms / args.steps
        gbs = step_bytes_total / (ms_per_step * 1e-3) / 1e9
        per_group_bytes = step_bytes_total / groups
        ms_8k = BYTES_8K_REQUEST / (per_group_bytes / (ms_per_step * 1e-3)) * 1e3
        peaks = {}
        peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
        if os.path.exists(peaks_path):
            with open(peaks_path) as f:
                peaks = json.load(f)
        traffic = load_traffic().get("loopback" if loopback and not peer_mode else f"{args.workload}-{args.mode}")
        if loopback and not peer_mode:
            hbm = peaks.get("hbm_gbs", 6650.0)
            achieved = 2 * step_bytes_total / (ms_per_step * 1e-3) / 1e9
            roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(achieved / hbm, 4),
                        "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks else "fallback",
                        "traffic": traffic.get("bytes_per_launch") if traffic else None,
                        "algorithmic_bytes_per_launch": int(2 * step_bytes_total)}
        else:
            # The busiest GPU's NVLink direction: each producer sends its decode ranks' shares of its heads.
            per_group = step_bytes_total / groups
            egress = per_group / spec.prefill_tp  # TP splits heads evenly; latents: each decode rank pulls whole
            if spec.mla:
                egress = per_group  # one producer feeds every decode rank a whole copy
                if relay:  # ... or, relayed, each byte once; every decode rank still takes a whole copy in
                    egress = per_group / spec.decode_tp
            ingress = per_group / spec.decode_tp
            link_bytes = max(egress, ingress)
            achieved = link_bytes / (ms_per_step * 1e-3) / 1e9
            roofline = {"bound": "nvlink", "achieved": round(achieved, 1), "peak": NVLINK_GBS, "unit": "GB/s",
                        "frac": round(achieved / NVLINK_GBS, 4),
                        "peak_source": "nominal NVLink 5 per direction per GPU (900 GB/s), the north star's peak",
                        "peer_copy_gbs_measured": round(min(peer_copies), 1) if peer_copies else None,
                        "peer_copy_method": "1 GiB device-to-device copy on the consumer GPU's stream from the "
                                            "producer GPU's memory (copy engine, peer access), CUDA events, best of "
                                            "5; min over pairs",
                        "busiest_link": "producer egress" if egress >= ingress else "decode ingress",
                        "link_bytes_per_step": int(link_bytes),
                        "traffic": traffic.get("bytes_per_launch") if traffic else None,
                        "nvlink_rx_bytes_per_launch": traffic.get("nvlink_rx_bytes_per_launch") if traffic else None,
                        "algorithmic_bytes_per_launch": int(per_group / (spec.decode_tp if args.mode == "pull"
                                                                         else spec.prefill_tp))}
        line = {
            "metric": METRIC,
            "value": round(gbs, 2),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "ms_per_8k_request": round(ms_8k, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: seeded N(0,1) bf16 caches, seeded shuffled block tables",
            "config": {
                "workload": (f"{spec.name}/peer-1process-cuda0-to-cuda{args.peer_device}" if peer_mode else
                             f"{spec.name}/loopback-1gpu" if loopback else
                             f"{spec.name}/{groups}x-tp{spec.prefill_tp}to{spec.decode_tp}"),
                "shape": spec.describe(),
                "requests_per_step": len(reqs),
                "prompt_lengths": f"{spec.lengths[0]} [{spec.lengths[1]}, {spec.lengths[2]}], seed {args.seed}",
                "blocks_per_step_per_group": step_blocks,
                "payload_bytes_per_step": int(step_bytes_total),
                "groups": groups,
                "mode": "loopback" if loopback else args.mode + (" relayed" if relay else ""),
                "relay_chunks": (args.relay_chunks or RELAY_CHUNKS) if relay else None,
                "relay_sms_per_stream": (relay_sms or "all") if relay else None,
                "engine": args.engine,
                "tile_bytes": args.tile_bytes or "default", "ctas_per_sm": args.ctas_per_sm or "default",
                "parallelism": ("1 GPU" if loopback else
                                f"{groups} independent prefill TP{spec.prefill_tp} -> decode TP{spec.decode_tp} groups"),
                "l2": f"no flush: each step moves {step_bytes_total / 1e9:.1f} GB, far beyond the 126 MB L2",
            },
            "roofline": roofline,
            "gpu_launches": total_launches,
            "clocks": clock_summary,
            "correct": bool(ok_t[0].item() == 0.0),
            "correct_covers": (f"every moved block of every request ({checked} (layer, block) pairs"
                               + (": compared outright)" if loopback else
                                  ": per-(layer, part, block) digests of each head share on both sides)")),
        }
        if e2e_ms is not None:
            ids_bytes = 2 * 4 * step_blocks * spec.decode_tp * groups
            line["e2e"] = {"value": round(e2e_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                           "ms_per_step": round(e2e_ms, 4),
                           "h2d_bytes_per_step": ids_bytes, "d2h_bytes_per_step": 0,
                           "bytes_reported_by_connector": e2e_bytes,
                           "kvx_launches_per_step": round(e2e_launches / (1 + max(args.steps // 2, 2)), 1),
                           "correct": bool(ok_t[1].item() == 0.0),
                           "correct_covers": "every moved block again, checked after these loads into zeroed "
                                             "decode caches",
                           "batch_bytes": envs.LEAN_VLLM_KVX_BATCH_BYTES,
                           "path": (f"CudaIpcConnectorWorker.start_load_kv({len(reqs)} ReqToRecv from host lists) -> "
                                    "get_finished() until every load finished_recving; the first load launched "
                                    "by start_load_kv itself, the rest planned by the transfer thread into "
                                    "launches of up to batch_bytes on two alternating streams, block ids carried "
                                    "in each launch; the thread woken by a doorbell when a copy lands; each "
                                    "transfer's result read from its status word in mapped host memory (written "
                                    "by the device only on failure), so no device-to-host copy is made")}
        line.update(extras)
        if loopback and not peer_mode and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(reqs, spec, seconds=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        for blob in opened:
            transport.close_mapping(blob)
        dist.destroy_process_group()


def child_line(argv: list[str], timeout: float = 600.0) -> dict:
    """The JSON line a child run of this script prints, or why there is none."""
    try:
        run = subprocess.run([sys.executable, os.path.abspath(__file__), *argv], capture_output=True, text=True,
                             timeout=timeout, cwd=ROOT)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"bench.py {' '.join(argv)} ran past {timeout:.0f} s"}
    lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
    if run.returncode or not lines:
        return {"unavailable": f"bench.py {' '.join(argv)} exited {run.returncode}: {run.stderr.strip()[-300:]}"}
    return json.loads(lines[-1])


def measure_extras(args) -> dict:
    """The store and the layer-wise push, measured by child runs of this script on the same GPU."""
    out = {}
    store = child_line(["--store", "--steps", str(max(args.steps, 10)), "--warmup", str(max(args.warmup, 3)),
                        "--seed", str(args.seed)])
    if "unavailable" in store:
        out["store"] = store
    else:
        out["store"] = {"metric": store["metric"], "value": store["value"], "unit": store["unit"],
                        "ms_per_step": store["ms_per_step"], "us_per_launch": round(store["ms_per_step"] / 36 * 1e3, 2),
                        "roofline": store["roofline"], "frac_of_same_bytes_copy": store["frac_of_same_bytes_copy"],
                        "correct": store["correct"], "clocks": store["clocks"],
                        "workload": "36 kvx_store launches of an 8192-token Qwen3-8B prefill step, graph-replayed",
                        "command": f"python bench.py --store --steps {max(args.steps, 10)} --warmup "
                                   f"{max(args.warmup, 3)}"}
    layerwise = child_line(["--layerwise", "--steps", "3", "--warmup", "1", "--seed", str(args.seed)])
    if "unavailable" in layerwise:
        out["layerwise"] = layerwise
    else:
        out["layerwise"] = {"metric": layerwise["metric"], "exposed_fraction": layerwise["value"],
                            "ms_compute_alone": layerwise["ms_compute_alone"],
                            "ms_until_last_byte_landed": layerwise["ms_until_last_byte_landed"],
                            "prefill_tflops": layerwise["prefill_tflops"], "correct": layerwise["correct"],
                            "workload": layerwise["config"]["workload"],
                            "command": "python bench.py --layerwise --steps 3 --warmup 1"}
    return out


def e2e_connector(args, spec, world, rank, role, src, dst, reqs, gloo):
    """Times a step's loads through CudaIpcConnectorWorker (host clock, consumer side, median over steps): each
    group's prefill ranks hold the source cache and its decode ranks load every request, shares and all. The 1-GPU
    loopback runs both workers in this process. Returns (ms per step, bytes the connector counted here)."""
    import torch
    import torch.distributed as dist

    from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVTransferConfig, ReqToRecv
    from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker

    @dataclass
    class WorkerConfig:
        kv_transfer: KVTransferConfig
        tensor_parallel_size: int = 1
        kvcache_block_size: int = spec.block
        kv_cache_layout: str = "HND"
        kvx_relay: bool = bool(args.relay)

    base_port = args.kv_port + 16 * role.group
    producer_worker = consumer_worker = None
    if role.side in ("prefill", "both"):
        kv = KVTransferConfig(kv_role="kv_producer", kv_port=base_port, engine_id=f"bench-prefill-{role.group}")
        producer_worker = CudaIpcConnectorWorker(WorkerConfig(kv, spec.prefill_tp), role.tp_rank)
        producer_worker.register_kv_caches(src)
    if role.side in ("decode", "both"):
        kv = KVTransferConfig(kv_role="kv_consumer", kv_port=base_port + 8, engine_id=f"bench-decode-{role.group}")
        consumer_worker = CudaIpcConnectorWorker(WorkerConfig(kv, spec.decode_tp), role.tp_rank)
        consumer_worker.register_kv_caches(dst)

    def one_step(tag: str) -> tuple[float, int]:
        sends = {f"{tag}-{i}": s.tolist() for i, (s, _) in enumerate(reqs)}
        recvs = {f"{tag}-{i}": ReqToRecv(d.tolist(), s.tolist(), f"{tag}-{i}", f"bench-prefill-{role.group}",
                                         "127.0.0.1", base_port, spec.prefill_tp) for i, (s, d) in enumerate(reqs)}
        if world > 1:
            dist.barrier(group=gloo)
        torch.cuda.synchronize()
        if producer_worker is not None:
            producer_worker.start_load_kv(KVConnectorMetadata(reqs_to_send=sends))
        t0 = time.perf_counter()
        nbytes = 0
        if consumer_worker is not None:
            consumer_worker.start_load_kv(KVConnectorMetadata(reqs_to_recv=recvs))
            pending = set(recvs)
            deadline = time.monotonic() + 120
            while pending and time.monotonic() < deadline:
                out = consumer_worker.get_finished()
                if out.failed_recving:
                    raise RuntimeError(f"connector loads failed: {sorted(out.failed_recving)[:3]}")
                for rid in out.finished_recving:
                    nbytes += out.recv_stats[rid].num_bytes
                pending -= out.finished_recving
                if pending:
                    time.sleep(50e-6)
            if pending:
                raise RuntimeError(f"{len(pending)} connector loads did not finish")
        elapsed = (time.perf_counter() - t0) * 1e3
        if producer_worker is not None:  # every held request is released once all its readers have notified
            left, deadline = set(sends), time.monotonic() + 60
            while left and time.monotonic() < deadline:
                left -= producer_worker.get_finished().finished_sending
                if left:
                    time.sleep(1e-3)
            if left:
                raise RuntimeError(f"{len(left)} held requests were never released")
        return (elapsed if consumer_worker is not None else 0.0), nbytes

    try:
        one_step("warm")
        times, nbytes = [], 0
        for s in range(max(args.steps // 2, 2)):
            ms, nbytes = one_step(f"s{s}")
            times.append(ms)
    finally:
        for worker in (producer_worker, consumer_worker):
            if worker is not None:
                worker.shutdown()
    return (float(np.median(times)) if consumer_worker is not None else 0.0), nbytes


# Qwen3-8B per layer: q 4096x4096, k and v 4096x1024, o 4096x4096, MLP 3 x 4096x12288 = 193e6 weights, 2 FLOPs
# each per token (attention scores left out, so the stand-in is, if anything, shorter than the real layer).
LAYER_FLOPS_PER_TOKEN = 2 * 193e6


def token_slots(block_ids, length: int, block: int) -> np.ndarray:
    """The cache slot of each of a request's tokens, given its block table."""
    t = np.arange(int(length))
    return np.asarray(block_ids, dtype=np.int64)[t // block] * block + t % block


def row_digest(layers, slots):
    """Position-weighted digest of the keys and values at the given slots, every layer."""
    import torch

    device = layers[0].device
    index = torch.as_tensor(slots, device=device, dtype=torch.long)
    out = []
    for layer in range(len(layers)):
        view = layers[layer].transpose(2, 3)  # (2, blocks, tokens, heads, dim)
        part = view[:, index // view.size(2), index % view.size(2)]
        flat = part.contiguous().view(torch.int16).reshape(-1).to(torch.int64)
        weights = torch.arange(flat.numel(), device=device, dtype=torch.int64) % 65521 + 1
        out += [int(flat.sum().item()), int((flat * weights).sum().item())]
    return out


def run_layerwise(args) -> None:
    """Layer-by-layer push during a synthetic prefill, through the connector's per-layer save (save_kv_layer).

    The prefill instance prefills the workload's first requests in steps of at most 8192 tokens; each layer of a
    step is a bf16 GEMM with Qwen3-8B's per-layer FLOPs for the step's tokens (the calibrated stand-in for the real
    layer), after which the engine calls save_kv_layer, which pushes that layer's blocks of the step's requests into
    the decode instance's blocks on a high-priority stream held to a few SMs. The same prefill runs without saves.
    Reported: compute time alone, with saves, until the last byte landed, and the exposed transfer time (the
    latter minus compute alone) as a fraction of compute alone."""
    import torch
    import torch.distributed as dist

    from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVTransferConfig, ReqToRecv
    from lean_vllm_b200.kv_transfer.base import ReqToSave
    from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker

    spec = WORKLOADS["pair"]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    role = role_of(rank, world, spec)
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    gloo = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
        gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=300))
    lengths, reqs, num_blocks = workload(args.seed, args.requests or 16, spec)
    steps, current, tokens = [], [], 0  # whole requests per step, at most 8192 tokens each
    for i, n in enumerate(lengths):
        if current and tokens + int(n) > 8192:
            steps.append(current)
            current, tokens = [], 0
        current.append(i)
        tokens += int(n)
    steps.append(current)

    @dataclass
    class WorkerConfig:
        kv_transfer: KVTransferConfig
        tensor_parallel_size: int = 1
        kvcache_block_size: int = spec.block
        kv_cache_layout: str = "HND"
        kvx_accept_push: bool = False

    base_port = args.kv_port + 16 * role.group
    src = dst = producer = consumer = None
    if role.side in ("prefill", "both"):
        src = alloc_cache(spec, 1, num_blocks, device, fill=True, seed=1000 + rank)
        producer = CudaIpcConnectorWorker(WorkerConfig(KVTransferConfig(
            kv_role="kv_producer", kv_port=base_port, engine_id=f"lw-prefill-{role.group}")), 0)
        producer.register_kv_caches(src)
    if role.side in ("decode", "both"):
        dst = alloc_cache(spec, 1, num_blocks, device, fill=False, seed=0)
        consumer = CudaIpcConnectorWorker(WorkerConfig(KVTransferConfig(
            kv_role="kv_consumer", kv_port=base_port + 8, engine_id=f"lw-decode-{role.group}"),
            kvx_accept_push=True), 0)
        consumer.register_kv_caches(dst)
    # A multiple of 128 wide, so the GEMM runs at tensor-core speed like the real layer's projections.
    hidden, width = 4096, int(LAYER_FLOPS_PER_TOKEN / (2 * 4096)) // 128 * 128
    if producer is not None:
        a = torch.randn(8192, hidden, device=device, dtype=torch.bfloat16)
        w = torch.randn(hidden, width, device=device, dtype=torch.bfloat16) * 0.01
        out = torch.empty(8192, width, device=device, dtype=torch.bfloat16)
        if args.fused:  # each layer's new keys/values, stored through the connector (store_kv)
            new_k = torch.randn(8192, spec.kv_heads, spec.head_dim, device=device).to(torch.bfloat16)
            new_v = torch.randn(8192, spec.kv_heads, spec.head_dim, device=device).to(torch.bfloat16)
            step_slots = [torch.as_tensor(np.concatenate([token_slots(reqs[i][0], lengths[i], spec.block)
                                                          for i in step]), device=device) for step in steps]
    torch.cuda.synchronize()

    def sync_all():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(group=gloo)

    def iteration(tag: str, saves: bool) -> tuple[float, float]:
        """Returns (ms of compute, ms until the last push landed) on the prefill side (0 elsewhere)."""
        ids = {i: f"{tag}-{i}" for i in range(len(reqs))}
        if consumer is not None and saves:
            consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={
                ids[i]: ReqToRecv(reqs[i][1].tolist(), reqs[i][0].tolist(), ids[i], f"lw-prefill-{role.group}",
                                  "127.0.0.1", base_port, 1, pushed=True) for i in range(len(reqs))}))
        sync_all()
        compute_ms = landed_ms = 0.0
        if producer is not None:
            stream = torch.cuda.current_stream()
            start, compute_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            landed = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for si, step in enumerate(steps):
                n_tokens = int(sum(int(lengths[i]) for i in step))
                if saves:
                    producer.start_load_kv(KVConnectorMetadata(reqs_to_save={
                        ids[i]: ReqToSave(reqs[i][0].tolist(), reqs[i][1].tolist(), f"lw-decode-{role.group}",
                                          "127.0.0.1", base_port + 8, 1, num_tokens=int(lengths[i])) for i in step},
                        save_progress={ids[i]: int(lengths[i]) for i in step}))  # whole prompts in this step
                    if tag == "warm-b" and step is steps[0]:
                        # First contact maps the decode cache on the transfer thread (once per decode instance);
                        # every later save finds it mapped and is ready at once.
                        deadline = time.monotonic() + 30
                        for i in step:
                            save = producer._saves[ids[i]]
                            while not (save.ready or save.failed) and time.monotonic() < deadline:
                                time.sleep(1e-4)
                            if not save.ready:
                                raise RuntimeError("the decode instance could not be mapped")
                for layer in range(spec.layers):
                    torch.matmul(a[:n_tokens], w, out=out[:n_tokens])
                    if args.fused:  # the layer's store, which also pushes the rows of every mapped save
                        producer.store_kv(layer, new_k[:n_tokens], new_v[:n_tokens], step_slots[si])
                    elif saves:
                        producer.save_kv_layer(layer)
                if saves:
                    producer.wait_for_save()
                    producer.start_load_kv(KVConnectorMetadata(reqs_to_send={ids[i]: reqs[i][0].tolist()
                                                                              for i in step}))
            compute_end.record(stream)
            landed.record(producer.transport.save_stream)
            landed.synchronize()
            torch.cuda.synchronize()
            compute_ms = start.elapsed_time(compute_end)
            landed_ms = max(compute_ms, start.elapsed_time(landed))
        if saves:
            for worker, field_name in ((producer, "finished_sending"), (consumer, "finished_recving")):
                if worker is None:
                    continue
                left, deadline = set(ids.values()), time.monotonic() + 120
                while left and time.monotonic() < deadline:
                    out_ = worker.get_finished()
                    if out_.failed_recving:
                        raise RuntimeError("a pushed load failed")
                    left -= getattr(out_, field_name)
                    time.sleep(1e-3)
                if left:
                    raise RuntimeError(f"{len(left)} pushed requests did not finish")
        sync_all()
        return compute_ms, landed_ms

    try:
        iteration("warm-a", False)
        iteration("warm-b", True)
        alone = [iteration(f"c{k}", False)[0] for k in range(args.steps)]
        both = [iteration(f"s{k}", True) for k in range(args.steps)]
        ok = True
        samples = range(len(reqs))  # every request

        def check(layers, ids, i):
            if args.fused:  # the stored rows only: a last block's tail past the prompt is never written
                return row_digest(layers, token_slots(ids, lengths[i], spec.block))
            return block_digests(layers, ids, 0, 8, False).cpu().tolist()

        if world == 1:
            ok = all(check(dst, reqs[i][1], i) == check(src, reqs[i][0], i) for i in samples)
        else:
            mine = [check(src, reqs[i][0], i) if src is not None else check(dst, reqs[i][1], i)
                    for i in samples] if role.side != "idle" else None
            every = [None] * world
            dist.all_gather_object(every, (role.group, role.side, mine), group=gloo)
            for g in range(world // spec.group_size):
                got = [m for gg, side, m in every if gg == g and side == "decode"]
                want = [m for gg, side, m in every if gg == g and side == "prefill"]
                ok &= got == want
    finally:
        for worker in (producer, consumer):
            if worker is not None:
                worker.shutdown()
    stats = torch.tensor([float(np.median(alone)), float(np.median([c for c, _ in both])),
                          float(np.median([ld for _, ld in both]))], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    if rank == 0:
        t_alone, t_with, t_landed = (float(x) for x in stats.cpu())
        payload = request_bytes(sum(len(s) for s, _ in reqs), spec)
        flops = LAYER_FLOPS_PER_TOKEN * spec.layers * float(sum(int(x) for x in lengths))
        line = {
            "metric": "layerwise push during prefill: exposed transfer time",
            "value": round((t_landed - t_alone) / t_alone, 5),
            "unit": "fraction of prefill compute time",
            "higher_is_better": False,
            "n_gpus": world,
            "steps": args.steps,
            "ms_compute_alone": round(t_alone, 3),
            "ms_compute_with_saves": round(t_with, 3),
            "ms_until_last_byte_landed": round(t_landed, 3),
            "exposed_ms": round(t_landed - t_alone, 3),
            "compute_slowdown": round(t_with / t_alone - 1, 5),
            "payload_bytes": payload,
            "prefill_tflops": round(flops / (t_alone * 1e-3) / 1e12, 1),
            "config": {"workload": f"{spec.name}/{'loopback-1gpu' if world == 1 else 'pair'} layerwise push",
                       "requests": len(reqs), "prefill_steps": len(steps),
                       "push": ("fused into each layer's store (store_kv)" if args.fused else
                                "save_kv_layer after each layer"),
                       "layer_stand_in": f"bf16 GEMM [tokens x 4096] @ [4096 x {width}] per layer",
                       "save_sms": int(os.environ.get("LEAN_VLLM_KVX_SAVE_SMS", "16"))},
            "correct": bool(ok),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_store(args) -> None:
    """The per-token cache store (store_kvcache, one kvx_store launch per layer) for one 8192-token prefill step of
    a Qwen3-8B-shaped model: 36 layers, each with its own new keys/values [8192, 8, 128] bf16 and its own HND cache,
    slots from a seeded shuffled block table. With --peer-device the same launches also push every row into a
    decode cache on that GPU (the fused store-and-push). Beside it, the torch indexing store (the reference's
    TorchAttention.store_kvcache, attention/torch_backend.py:34-48) on the same inputs."""
    import torch

    from lean_vllm_b200.attention.kvx_cache import PushTarget, store_kvcache
    from lean_vllm_b200.kv_transfer import transport

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    tokens, heads, dim, block, layers, nb = 8192, 8, 128, 256, 36, 48
    g = torch.Generator(device=device).manual_seed(args.seed)
    keys = [torch.randn(tokens, heads, dim, device=device, generator=g).to(torch.bfloat16) for _ in range(layers)]
    values = [torch.randn(tokens, heads, dim, device=device, generator=g).to(torch.bfloat16) for _ in range(layers)]
    caches = [torch.zeros(2, nb, heads, block, dim, device=device, dtype=torch.bfloat16) for _ in range(layers)]
    blocks = torch.randperm(nb, device=device, generator=g)[: tokens // block]
    slots = (blocks[:, None] * block + torch.arange(block, device=device)[None, :]).reshape(-1).contiguous()
    targets = [[] for _ in range(layers)]
    if args.peer_device is not None:
        peer = torch.device("cuda", args.peer_device)
        if not transport.enable_peer_access(0, peer.index):
            raise SystemExit(f"cuda:0 cannot reach cuda:{peer.index} directly")
        peer_caches = [torch.zeros(2, nb, heads, block, dim, device=peer, dtype=torch.bfloat16)
                       for _ in range(layers)]
        peer_slots = torch.flip(slots, [0]).contiguous()  # another block table on the decode side
        targets = [[PushTarget.of(c.transpose(2, 3)[0], c.transpose(2, 3)[1], peer_slots)] for c in peer_caches]
        torch.cuda.synchronize(peer)

    from lean_vllm_b200._native import STORE_SERIAL

    store_flags = (STORE_SERIAL if args.serial else 0) | (args.ctas_per_sm << 16)

    def ours():
        for layer in range(layers):
            view = caches[layer].transpose(2, 3)
            store_kvcache(keys[layer], values[layer], view[0], view[1], slots, push_to=targets[layer],
                          flags=store_flags)

    def torch_indexing():
        b, o = slots // block, slots % block
        for layer in range(layers):
            view = caches[layer].transpose(2, 3)
            view[0][b, o] = keys[layer]
            view[1][b, o] = values[layer]

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / steps

    ms_eager = timed(ours, args.steps)  # one Python call and launch per layer, as an eager engine issues them
    # The same 36 launches captured once and replayed: the kernels' own time, as a graph-captured engine runs them.
    graph = torch.cuda.CUDAGraph()
    capture = torch.cuda.Stream()
    capture.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(capture):
        ours()
        torch.cuda.synchronize()
        captured0 = transport.launch_count()
        with torch.cuda.graph(graph, stream=capture):
            ours()
        per_replay = transport.launch_count() - captured0  # kvx_store launches each replay runs
    torch.cuda.synchronize()
    with ClockSampler(0) as clocks:
        ms = timed(graph.replay, args.steps)
    ms_torch = timed(torch_indexing, max(args.steps // 4, 2))
    # Calibration: the same bytes per launch as a plain device copy (cudaMemcpyAsync of each layer's keys and values,
    # 33.5 MB read + 33.5 MB written), 36 launches replayed from a graph the same way: what a launch of this size
    # reaches at best, ramp and drain included.
    flat_src = [torch.cat([k.reshape(-1), v.reshape(-1)]) for k, v in zip(keys, values)]
    flat_dst = [torch.empty_like(f) for f in flat_src]
    copy_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(capture):
        for d, f in zip(flat_dst, flat_src):
            d.copy_(f)
        torch.cuda.synchronize()
        with torch.cuda.graph(copy_graph, stream=capture):
            for d, f in zip(flat_dst, flat_src):
                d.copy_(f)
    torch.cuda.synchronize()
    ms_copy = timed(copy_graph.replay, args.steps)
    del flat_src, flat_dst, copy_graph
    # Correctness: every layer's cache holds its rows at the slots (and the peer's at its slots).
    ok = True
    for layer in (0, layers - 1):
        view = caches[layer].transpose(2, 3)
        ok &= torch.equal(view[0][slots // block, slots % block], keys[layer])
        ok &= torch.equal(view[1][slots // block, slots % block], values[layer])
        if args.peer_device is not None:
            pv = peer_caches[layer].transpose(2, 3)
            ps = peer_slots.to(peer)
            ok &= torch.equal(pv[0][ps // block, ps % block], keys[layer].to(peer))
    rows = 2 * tokens * heads * dim * 2  # keys and values of one layer
    hbm_bytes = layers * (2 * rows + tokens * 8)  # read rows and slots, write rows
    peaks = {}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            peaks = json.load(f)
    hbm = peaks.get("hbm_gbs", 6650.0)
    if args.peer_device is None:
        roofline = {"bound": "hbm", "achieved": round(hbm_bytes / (ms * 1e-3) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                    "frac": round(hbm_bytes / (ms * 1e-3) / 1e9 / hbm, 4), "algorithmic_bytes_per_launch":
                    hbm_bytes // layers, "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)"}
    else:
        link = layers * rows
        roofline = {"bound": "nvlink", "achieved": round(link / (ms * 1e-3) / 1e9, 1), "peak": NVLINK_GBS,
                    "unit": "GB/s", "frac": round(link / (ms * 1e-3) / 1e9 / NVLINK_GBS, 4),
                    "link_bytes_per_launch": link // layers, "hbm_bytes_per_launch": hbm_bytes // layers,
                    "peak_source": "measured peer copy per direction on this pool (nominal 900 GB/s)"}
    line = {
        "metric": "KV cache store (store_kvcache) GB/s" + (" fused with push" if args.peer_device is not None else ""),
        "value": round(hbm_bytes / (ms * 1e-3) / 1e9, 1),
        "unit": "GB/s (HBM bytes read + written)",
        "higher_is_better": True,
        "n_gpus": 1 if args.peer_device is None else 2,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) bf16 rows, seeded shuffled block table",
        "config": {"workload": "qwen3-8b-kv/store-8192-token-step", "layers": layers, "tokens": tokens,
                   "shape": "8 KV heads x 128, block 256, HND",
                   "push": f"cuda:{args.peer_device}" if args.peer_device is not None else None,
                   "launch": "plain" if args.serial else "programmatic (overlaps the previous store's drain)",
                   "ctas_per_sm": args.ctas_per_sm or "default"},
        "roofline": roofline,
        "ms_per_step_eager": round(ms_eager, 4),
        "timing": "CUDA graph of the step's 36 store launches, replayed; ms_per_step_eager issues them one by one",
        "same_bytes_device_copy_ms_per_step": round(ms_copy, 4),
        "frac_of_same_bytes_copy": round(ms_copy / ms, 4),
        "torch_indexing_ms_per_step": round(ms_torch, 4),
        "speedup_vs_torch_indexing": round(ms_torch / ms_eager, 2),
        "gpu_launches": per_replay * args.steps,
        "clocks": clocks.summary(),
        "correct": bool(ok),
    }
    print(json.dumps(line), flush=True)


def run_poisson(args) -> None:
    """The arrival-rate sweep through the connector's public API: Qwen3-8B-shaped KV, prefill TP1 ->
    decode TP1 (a pair over NVLink at N=2, the same GPU at N=1), requests arriving as a Poisson process at each rate
    in --rates, prompt lengths log-normal with median 2048 and sigma 1.0 (a choice: the configuration gives no sigma),
    clipped to [128, 32768]. The decode side allocates each request's blocks from a free list and returns them when
    its load finishes; the prefill side holds random source blocks. Per rate: p50/p99 of each load's latency (from
    its start_load_kv to the get_finished that reports it, host clock) and the bytes moved over the wall time."""
    import torch
    import torch.distributed as dist

    from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVTransferConfig, ReqToRecv
    from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker

    spec = WORKLOADS["pair"]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    role = role_of(rank, world, spec)
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    gloo = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
        gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=600))
    pool = 1024  # blocks per side: 38.7 GB
    rates = [float(r) for r in args.rates.split(",")]
    # The decode loop below stands in for an engine calling get_finished as often as it can: it sleeps 20 us between
    # calls, and a 1 us timer slack (this process only; Linux's default is 50 us) keeps each sleep near that.
    import ctypes

    ctypes.CDLL(None, use_errno=True).prctl(29, 1000, 0, 0, 0)  # PR_SET_TIMERSLACK, in ns

    @dataclass
    class WorkerConfig:
        kv_transfer: KVTransferConfig
        tensor_parallel_size: int = 1
        kvcache_block_size: int = spec.block
        kv_cache_layout: str = "HND"

    base_port = args.kv_port + 16 * role.group
    producer = consumer = None
    if role.side in ("prefill", "both"):
        src = alloc_cache(spec, 1, pool, device, fill=True, seed=7)
        producer = CudaIpcConnectorWorker(WorkerConfig(KVTransferConfig(
            kv_role="kv_producer", kv_port=base_port, engine_id=f"ps-prefill-{role.group}")), 0)
        producer.register_kv_caches(src)
    if role.side in ("decode", "both"):
        dst = alloc_cache(spec, 1, pool, device, fill=False, seed=0)
        consumer = CudaIpcConnectorWorker(WorkerConfig(KVTransferConfig(
            kv_role="kv_consumer", kv_port=base_port + 8, engine_id=f"ps-decode-{role.group}")), 0)
        consumer.register_kv_caches(dst)
    torch.cuda.synchronize()
    results = []

    def warm_up():
        """One load before timing: the first handshake maps every layer of the producer's cache once."""
        if producer is not None:
            producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"warm": [0, 1]}))
        if world > 1:
            dist.barrier(group=gloo)
        if consumer is not None:
            consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={"warm": ReqToRecv(
                [0, 1], [0, 1], "warm", f"ps-prefill-{role.group}", "127.0.0.1", base_port, 1)}))
            deadline = time.monotonic() + 60
            while not consumer.get_finished().finished_recving and time.monotonic() < deadline:
                time.sleep(1e-3)
        if world > 1:
            dist.barrier(group=gloo)

    try:
        warm_up()
        for rate in rates:
            rng = np.random.default_rng(int(rate * 1000) + args.seed)
            n = int(min(max(rate * args.poisson_seconds, 24), 400))  # 24 at least: a p50 worth reading
            lengths = np.clip(np.exp(rng.normal(np.log(2048), 1.0, size=n)), 128, 32768).astype(np.int64)
            arrivals = np.cumsum(rng.exponential(1.0 / rate, size=n))
            blocks = [math.ceil(int(x) / spec.block) for x in lengths]
            srcs = [rng.choice(pool, size=b, replace=False).astype(np.int32) for b in blocks]
            ids = [f"r{rate}-{i}" for i in range(n)]
            if producer is not None:
                producer.start_load_kv(KVConnectorMetadata(reqs_to_send={ids[i]: srcs[i].tolist() for i in range(n)}))
            if world > 1:
                dist.barrier(group=gloo)
            latency, in_flight, moved = [], [], 0
            if consumer is not None:
                free = list(rng.permutation(pool))
                pending, started, waiting = {}, {}, list(range(n))
                t0 = time.perf_counter()
                while waiting or pending:
                    now = time.perf_counter() - t0
                    due = [i for i in waiting if arrivals[i] <= now and len(free) >= blocks[i]]
                    if due:
                        reqs = {}
                        for i in due:
                            waiting.remove(i)
                            local = [int(free.pop()) for _ in range(blocks[i])]
                            pending[ids[i]] = (i, local)
                            started[ids[i]] = time.perf_counter()
                            reqs[ids[i]] = ReqToRecv(local, srcs[i].tolist(), ids[i], f"ps-prefill-{role.group}",
                                                     "127.0.0.1", base_port, 1)
                        consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv=reqs))
                    out = consumer.get_finished()
                    if out.failed_recving:
                        raise RuntimeError(f"loads failed: {sorted(out.failed_recving)[:3]}")
                    for rid in out.finished_recving:
                        i, local = pending.pop(rid)
                        latency.append((time.perf_counter() - started[rid]) * 1e3)
                        in_flight.append(out.recv_stats[rid].seconds * 1e3)
                        moved += out.recv_stats[rid].num_bytes
                        free.extend(local)
                    time.sleep(20e-6)
                wall = time.perf_counter() - t0
                results.append({"rate_req_per_s": rate, "requests": n, "p50_ms": round(float(np.percentile(latency, 50)), 3),
                                "p99_ms": round(float(np.percentile(latency, 99)), 3),
                                "mean_ms": round(float(np.mean(latency)), 3),
                                # the connector's own stats: from posting the copy to seeing it landed
                                "p50_posted_to_landed_ms": round(float(np.percentile(in_flight, 50)), 3),
                                # the host path around the copy: start_load_kv to posting, and landing to the
                                # get_finished that reports it
                                "p50_host_ms": round(float(np.percentile(np.subtract(latency, in_flight), 50)), 3),
                                "offered_gb_per_s": round(moved / float(arrivals[-1]) / 1e9, 2),
                                "moved_gb_per_s": round(moved / wall / 1e9, 2), "bytes": moved,
                                "mean_prompt_tokens": int(lengths.mean())})
            if world > 1:
                dist.barrier(group=gloo)
            if producer is not None:  # every held request released once read
                left, deadline = set(ids), time.monotonic() + 60
                while left and time.monotonic() < deadline:
                    left -= producer.get_finished().finished_sending
                    time.sleep(1e-3)
    finally:
        for worker in (producer, consumer):
            if worker is not None:
                worker.shutdown()
    every = [None] * world
    if world > 1:
        dist.all_gather_object(every, results, group=gloo)
    else:
        every = [results]
    if rank == 0:
        pairs = [r for r in every if r]  # one list of rate rows per decode rank (per pair)
        line = {"metric": "KV transfer latency under Poisson arrivals (connector API)", "unit": "ms",
                "higher_is_better": False, "n_gpus": world,
                "config": {"workload": f"{spec.name}/{'loopback-1gpu' if world == 1 else 'pair'} poisson",
                           "pairs": len(pairs),
                           "prompt_lengths": "log-normal, median 2048, sigma 1.0, clipped [128, 32768]",
                           "decode_pool_blocks": pool, "get_finished_poll_us": 20,
                           "inline_loads": bool(envs.LEAN_VLLM_KVX_INLINE_LOADS)},
                "rates": pairs[0]}
        if len(pairs) > 1:  # every pair runs the same seeded arrivals at once: the spread shows any interference
            line["p50_ms_by_pair"] = {str(row["rate_req_per_s"]): [p[i]["p50_ms"] for p in pairs]
                                      for i, row in enumerate(pairs[0])}
            line["p99_ms_by_pair"] = {str(row["rate_req_per_s"]): [p[i]["p99_ms"] for p in pairs]
                                      for i, row in enumerate(pairs[0])}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_staged(args) -> None:
    """The three-kernel path the north star names, stage by stage: kvx_pack gathers each request's blocks into a
    contiguous staging buffer (block_descs row order), kvx_push moves the buffer to a staging buffer on the decode
    GPU (--peer-device; the same GPU otherwise), kvx_scatter writes it into the decode cache's blocks. Qwen3-8B
    shape, the workload's first --requests requests (16 by default, so that both caches and both buffers fit). Each
    stage is timed with CUDA events over --steps repetitions; pack and scatter are HBM-bound (read + write), the push
    NVLink-bound (or HBM-bound on one GPU)."""
    import torch

    from lean_vllm_b200._native import ENGINE_AUTO, ENGINE_LSU, ENGINE_TMA, flags
    from lean_vllm_b200.kv_transfer import transport
    from lean_vllm_b200.kv_transfer.transport import CacheTable

    spec = WORKLOADS["pair"]
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peer = torch.device("cuda", args.peer_device) if args.peer_device is not None else device
    if peer != device and not transport.enable_peer_access(0, peer.index):
        raise SystemExit(f"cuda:0 cannot reach cuda:{peer.index} directly")
    engine = {"auto": ENGINE_AUTO, "lsu": ENGINE_LSU, "tma": ENGINE_TMA}[args.engine]
    copy_flags = flags(engine, args.tile_bytes, args.ctas_per_sm)
    lengths, reqs, num_blocks = workload(args.seed, args.requests or 16, spec)
    src = alloc_cache(spec, 1, num_blocks, device, fill=True, seed=3)
    dst = alloc_cache(spec, 1, num_blocks, peer, fill=False, seed=0)
    per_request = [request_bytes(len(s), spec) for s, _ in reqs]
    total = sum(per_request)
    offsets = np.concatenate([[0], np.cumsum(per_request)]).astype(np.int64)
    staging = torch.empty(total, dtype=torch.uint8, device=device)
    landing = torch.empty(total, dtype=torch.uint8, device=peer)
    src_t, dst_t = CacheTable.from_tensors(src), CacheTable.from_tensors(dst)
    heads = spec.kv_heads

    def pack():
        for (s, _), off, n in zip(reqs, offsets, per_request):
            transport.pack(src_t, s, 0, heads, False, staging.data_ptr() + int(off), n, 0, copy_flags)

    def push():
        transport.push(landing.data_ptr(), staging.data_ptr(), total, 0, copy_flags)

    def scatter():  # on the decode GPU, which owns both the landing buffer and the cache
        for (_, d), off, n in zip(reqs, offsets, per_request):
            transport.scatter(landing.data_ptr() + int(off), n, dst_t, d, 0, heads, False, 0, copy_flags)

    def timed(fn, on):
        with torch.cuda.device(on):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize(on)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(args.steps):
                fn()
            end.record()
            torch.cuda.synchronize(on)
            return start.elapsed_time(end) / args.steps

    with ClockSampler(0) as clocks:
        ms = {"pack": timed(pack, device), "push": timed(push, device), "scatter": timed(scatter, peer)}
    torch.cuda.synchronize(peer)
    ok = all(digest(dst, d, 0, heads, False, peer) == digest(src, s, 0, heads, False, device)
             for s, d in (reqs[0], reqs[-1]))
    peaks = {}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            peaks = json.load(f)
    hbm = peaks.get("hbm_gbs", 6650.0)
    stages = {}
    for name, t in ms.items():
        moved = 2 * total if name != "push" or peer == device else total
        bound, peak = ("nvlink", NVLINK_GBS) if name == "push" and peer != device else ("hbm", hbm)
        achieved = moved / (t * 1e-3) / 1e9
        stages[name] = {"ms": round(t, 4), "payload_gb_per_s": round(total / (t * 1e-3) / 1e9, 1),
                        "roofline": {"bound": bound, "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                                     "frac": round(achieved / peak, 4), "algorithmic_bytes": moved}}
    line = {
        "metric": "staged KV transfer (pack -> push -> scatter) GB/s",
        "value": round(total / (sum(ms.values()) * 1e-3) / 1e9, 1),
        "unit": "GB/s payload through all three stages",
        "higher_is_better": True,
        "n_gpus": 1 if peer == device else 2,
        "steps": args.steps,
        "warmup": args.warmup,
        "config": {"workload": f"{spec.name}/staged-{len(reqs)}-requests", "payload_bytes": total,
                   "requests": len(reqs), "decode_device": f"cuda:{peer.index}", "engine": args.engine},
        "stages": stages,
        "clocks": clocks.summary(),
        "correct": bool(ok),
    }
    print(json.dumps(line), flush=True)


def run_step_exchange(args) -> None:
    """ModelRunner.kv_connector_step's per-step exchange of connector outputs between one instance's tensor-parallel
    ranks (engine/model_runner.py:637-649), host only: every rank runs --steps steps with a stub connector, rank 0
    times each step (start to its aggregated output). Two exchanges: the reference's gloo gather_object, and the
    shared-memory step mailbox; two loads: quiet steps (nothing finished anywhere, the common case) and busy steps
    (every rank reports 4 finished loads each step). Launch under torchrun with --gpus N for N ranks."""
    import torch.distributed as dist

    from lean_vllm_b200.kv_transfer.base import KVConnectorOutput, KVTransferStats
    from lean_vllm_b200.kv_transfer.step import KVConnectorStep

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world < 2:
        raise SystemExit("--step-exchange needs torchrun with 2 or more ranks")
    dist.init_process_group("gloo")

    class Stub:
        def __init__(self, busy):
            self.busy, self.n = busy, 0

        def start_load_kv(self, metadata):
            pass

        def get_finished(self):
            if not self.busy:
                return KVConnectorOutput()
            self.n += 1
            ids = {f"req-{self.n}-{i}" for i in range(4)}
            return KVConnectorOutput(finished_recving=ids, recv_stats={r: KVTransferStats(1e-3, 1 << 28) for r in ids})

    results = {}
    for exchange in ("gather", "mailbox"):
        for load in ("quiet", "busy"):
            step = KVConnectorStep(Stub(load == "busy"), rank, world, exchange=exchange)
            times = []
            for i in range(args.warmup + args.steps):
                t0 = time.perf_counter()
                step(None)
                if i >= args.warmup:
                    times.append((time.perf_counter() - t0) * 1e6)
            step.close()
            dist.barrier()
            results[f"{exchange}/{load}"] = {"p50_us": round(float(np.median(times)), 1),
                                             "p99_us": round(float(np.percentile(times, 99)), 1)}
    if rank == 0:
        print(json.dumps({"metric": "kv_connector_step exchange latency (rank 0, per step)", "unit": "us",
                          "higher_is_better": False, "ranks": world, "steps": args.steps, "warmup": args.warmup,
                          "config": {"workload": "stub connector; quiet = nothing finished, busy = 4 loads per rank "
                                                 "per step", "host_cores": os.cpu_count()},
                          "results": results}), flush=True)
    dist.destroy_process_group()


def run_copy_engine(args) -> None:
    """A copy-engine baseline for the transfer kernel: the same loads as one cudaMemcpyAsync per (layer, K|V, block)
    chunk -- what a DMA transport such as the reference's NIXL/UCX path issues per descriptor row
    (nixl_connector.py:404-420) -- on the decode GPU's stream, against one kvx_copy launch for the same jobs. Qwen3-8B
    shape, the workload's first --requests requests (4 by default), destination on --peer-device (NVLink) or the same
    GPU. Both are timed with CUDA events; the copy-engine line also reports the host time spent issuing."""
    import ctypes
    import glob

    import torch

    from lean_vllm_b200.kv_transfer import transport
    from lean_vllm_b200.kv_transfer.transport import CacheTable, CopyJob

    spec = WORKLOADS["pair"]
    src_dev = torch.device("cuda", 0)
    dst_dev = torch.device("cuda", args.peer_device) if args.peer_device is not None else src_dev
    if dst_dev != src_dev and not transport.enable_peer_access(dst_dev.index, src_dev.index):
        raise SystemExit(f"cuda:{dst_dev.index} cannot reach cuda:{src_dev.index} directly")
    lengths, reqs, num_blocks = workload(args.seed, args.requests or 4, spec)
    src = alloc_cache(spec, 1, num_blocks, src_dev, fill=True, seed=3)
    dst = alloc_cache(spec, 1, num_blocks, dst_dev, fill=False, seed=0)
    payload = sum(request_bytes(len(s), spec) for s, _ in reqs)
    candidates = glob.glob(os.path.join(os.path.dirname(os.path.dirname(torch.__file__)), "nvidia", "cuda_runtime",
                                        "lib", "libcudart.so*"))
    cudart = ctypes.CDLL(candidates[0])
    cudart.cudaMemcpyAsync.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int,
                                       ctypes.c_void_p]
    cudart.cudaMemcpyAsync.restype = ctypes.c_int
    chunk = spec.kv_heads * spec.block * spec.head_dim * 2
    rows = []  # (dst address, src address) per chunk, block_descs order
    for s_ids, d_ids in reqs:
        for layer in range(spec.layers):
            for part in range(2):
                for s_id, d_id in zip(s_ids, d_ids):
                    rows.append((dst[layer][part, int(d_id)].data_ptr(), src[layer][part, int(s_id)].data_ptr()))
    torch.cuda.set_device(dst_dev)
    stream = torch.cuda.Stream(device=dst_dev)

    def ce():
        for d, s_ in rows:
            rc = cudart.cudaMemcpyAsync(d, s_, chunk, 4, stream.cuda_stream)  # cudaMemcpyDefault
            if rc:
                raise RuntimeError(f"cudaMemcpyAsync failed with {rc}")

    tables = [CacheTable.from_tensors(dst), CacheTable.from_tensors(src)]
    jobs = [CopyJob(1, 0, s, d, 0, 0, spec.kv_heads) for s, d in reqs]

    def kvx():
        transport.copy(tables, jobs, stream.cuda_stream)

    def timed(fn):
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                fn()
            stream.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            t0 = time.perf_counter()
            for _ in range(args.steps):
                fn()
            host = (time.perf_counter() - t0) * 1e3 / args.steps
            end.record(stream)
            stream.synchronize()
            return start.elapsed_time(end) / args.steps, host

    with ClockSampler(dst_dev.index) as clocks:
        ms_ce, host_ce = timed(ce)
        ms_kvx, host_kvx = timed(kvx)
    ok = digest(dst, reqs[-1][1], 0, spec.kv_heads, False, dst_dev) == digest(src, reqs[-1][0], 0, spec.kv_heads,
                                                                           False, src_dev)
    line = {
        "metric": "KV transfer GB/s: one cudaMemcpyAsync per chunk (copy engines) vs one kvx_copy launch",
        "unit": "GB/s payload", "higher_is_better": True, "steps": args.steps, "warmup": args.warmup,
        "config": {"workload": f"{spec.name}/{len(reqs)}-requests", "payload_bytes": payload, "chunks": len(rows),
                   "chunk_bytes": chunk, "path": "NVLink pull" if dst_dev != src_dev else "same GPU"},
        "copy_engine": {"ms": round(ms_ce, 4), "gb_per_s": round(payload / (ms_ce * 1e-3) / 1e9, 1),
                        "host_issue_ms": round(host_ce, 4),
                        "host_us_per_memcpy": round(host_ce * 1e3 / len(rows), 3)},
        "kvx_copy": {"ms": round(ms_kvx, 4), "gb_per_s": round(payload / (ms_kvx * 1e-3) / 1e9, 1),
                     "host_issue_ms": round(host_kvx, 4), "launches": 1},
        "clocks": clocks.summary(),
        "correct": bool(ok),
    }
    print(json.dumps(line), flush=True)


REFERENCE_PATH = os.path.join(ROOT, "baseline", "_ref")  # the reference, pip-installed here (git-ignored)
REFERENCE_SECONDS = 180.0  # the reference worker leg's timed budget: its per-step sample shrinks to fit it


def host_rank_caches(spec: Workload, tp: int, num_blocks: int, seed: int | None):
    """One side's caches on the host, per rank (torch CPU bf16, HND or latents): rank r holds heads
    [r*H/tp, (r+1)*H/tp), latents whole. With a seed every block gets distinct contents (a seeded random block
    pattern, stamped with the layer and block index); without one, zeros."""
    import torch

    ranks = []
    g = torch.Generator().manual_seed(seed or 0)
    for rank in range(tp):
        layers = []
        for layer in range(spec.layers):
            shape = ((1, num_blocks, spec.block, spec.head_dim) if spec.mla else
                     (2, num_blocks, spec.kv_heads // tp, spec.block, spec.head_dim))
            t = torch.zeros(shape, dtype=torch.bfloat16)
            if seed is not None:
                words = t.view(torch.int16)
                pattern = torch.randint(-(1 << 15), 1 << 15, (shape[0], 1, *shape[2:]), generator=g,
                                        dtype=torch.int16)
                words.copy_(pattern.expand_as(words))
                stamp = words.reshape(shape[0], num_blocks, -1)
                stamp[:, :, 0] = torch.arange(num_blocks, dtype=torch.int16)
                stamp[:, :, 1] = layer * 16 + rank
            layers.append(t)
        ranks.append(layers)
    return ranks


def reference_worker_leg(spec: Workload, reqs, producers, consumers, steps: int, warmup: int) -> dict:
    """The reference's own transfer path, unmodified: lean-vLLM's NixlConnectorWorker (imported from the pip-installed
    reference in baseline/_ref) as every prefill and decode rank in this process, over host caches, with NIXL
    replaced by the memmove agent the reference's CPU tests describe (oracle/memmove_agent.py). A step hands every
    request over on the producer ranks and loads it on the decode ranks (start_load_kv, then get_finished until all
    have landed), as tests/test_nixl_connector.py:33-115 drives them. Returns the leg's numbers, or why it could not
    run."""
    import socket
    from dataclasses import dataclass as plain_dataclass

    if not os.path.isdir(os.path.join(REFERENCE_PATH, "lean_vllm")):
        return {"unavailable": f"the reference is not installed in {os.path.relpath(REFERENCE_PATH, ROOT)}"}
    if REFERENCE_PATH not in sys.path:
        sys.path.insert(0, REFERENCE_PATH)
    try:
        from lean_vllm.kv_transfer import KVConnectorMetadata, KVTransferConfig, ReqToRecv
        from lean_vllm.kv_transfer import nixl_connector
    except Exception as error:  # noqa: BLE001
        return {"unavailable": f"importing the reference failed: {type(error).__name__}: {error}"}
    from oracle.memmove_agent import MemmoveAgent

    nixl_connector.make_agent = MemmoveAgent

    @plain_dataclass
    class Cfg:
        kv_transfer: object
        tensor_parallel_size: int
        kvcache_block_size: int
        kv_cache_layout: str = "HND"

    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    if port + spec.prefill_tp > 65535:
        port -= 64
    prefill_ranks, decode_ranks = [], []
    try:
        for rank, layers in enumerate(producers):
            kv = KVTransferConfig(kv_role="kv_producer", kv_port=port, engine_id="ref-prefill")
            worker = nixl_connector.NixlConnectorWorker(Cfg(kv, spec.prefill_tp, spec.block), rank)
            worker.register_kv_caches(layers)
            prefill_ranks.append(worker)
        for rank, layers in enumerate(consumers):
            kv = KVTransferConfig(kv_role="kv_consumer", kv_port=port + 64, engine_id="ref-decode")
            worker = nixl_connector.NixlConnectorWorker(Cfg(kv, spec.decode_tp, spec.block), rank)
            worker.register_kv_caches(layers)
            decode_ranks.append(worker)

        def step(tag: str, sample) -> tuple[float, int]:
            sends = {f"{tag}-{i}": [int(b) for b in s] for i, (s, _) in enumerate(sample)}
            recvs = {f"{tag}-{i}": ReqToRecv([int(b) for b in d], [int(b) for b in s], f"{tag}-{i}", "ref-prefill",
                                             "127.0.0.1", port, spec.prefill_tp) for i, (s, d) in enumerate(sample)}
            for worker in prefill_ranks:
                worker.start_load_kv(KVConnectorMetadata(reqs_to_send=sends))
            started = time.perf_counter()
            for worker in decode_ranks:
                worker.start_load_kv(KVConnectorMetadata(reqs_to_recv=recvs))
            nbytes, waiting = 0, [set(recvs) for _ in decode_ranks]
            deadline = time.monotonic() + 1800
            while any(waiting) and time.monotonic() < deadline:
                for left, worker in zip(waiting, decode_ranks):
                    out = worker.get_finished()
                    if out.failed_recving:
                        raise RuntimeError(f"reference loads failed: {sorted(out.failed_recving)[:3]}")
                    for request_id in out.finished_recving:
                        nbytes += out.recv_stats[request_id].num_bytes
                    left -= out.finished_recving
                if any(waiting):
                    time.sleep(1e-3)
            elapsed = time.perf_counter() - started
            if any(waiting):
                raise RuntimeError("reference loads did not finish")
            left, deadline = set(sends), time.monotonic() + 60  # held blocks released once every reader reported
            while left and time.monotonic() < deadline:
                for worker in prefill_ranks:
                    left -= worker.get_finished().finished_sending
                time.sleep(1e-3)
            return elapsed, nbytes

        for k in range(min(warmup, 1)):  # the first handshake; nothing else warms up
            step(f"warm{k}", reqs[:1])
        # A full step on the whole workload if the timed steps fit the budget, else the largest prefix that does.
        probe_s, probe_bytes = step("probe", reqs[: max(1, len(reqs) // 8)])
        per_byte = probe_s / max(probe_bytes, 1)
        total = sum(request_bytes(len(s), spec) for s, _ in reqs)
        sample = reqs
        if per_byte * total * steps > REFERENCE_SECONDS:
            budget = REFERENCE_SECONDS / steps / per_byte
            sample, acc = [], 0
            for s, d in reqs:
                acc += request_bytes(len(s), spec)
                if acc > budget and sample:
                    break
                sample.append((s, d))
        times, moved = [], 0
        for k in range(steps):
            seconds, moved = step(f"s{k}", sample)
            times.append(seconds)
        seconds = float(np.median(times))
        gbs = moved / seconds / 1e9
        # The decode caches hold the producer's blocks (rank 0's share of the last request of the sample).
        import torch

        s_ids, d_ids = sample[-1]
        heads = spec.kv_heads // spec.decode_tp if not spec.mla else None
        landed = consumers[0][0][:, list(d_ids)]
        sent = producers[0][0][:, list(s_ids)]
        if heads is not None and spec.prefill_tp == 1:
            sent = sent[:, :, :heads]
        # Bit patterns, not values: random words include bf16 NaNs, which compare unequal to themselves.
        correct = bool(torch.equal(landed.view(torch.int16), sent.view(torch.int16))) if spec.prefill_tp == 1 else None
        return {
            "value": round(gbs, 3), "unit": "GB/s", "kind": "reference",
            "ms_per_step": round(seconds * 1e3, 3), "steps": steps,
            "cores": spec.decode_tp,
            "sample": (f"{len(sample)} of the workload's {len(reqs)} requests per step ({moved / 1e9:.2f} GB)"
                       + ("" if len(sample) == len(reqs) else f", cut to fit {REFERENCE_SECONDS:.0f} s of timed steps")),
            "same_config": len(sample) == len(reqs),
            "path": ("lean_vllm.kv_transfer.nixl_connector.NixlConnectorWorker (the installed reference, unmodified): "
                     f"{spec.prefill_tp} prefill + {spec.decode_tp} decode ranks in one process, one transfer thread "
                     "each; NIXL replaced by the reference tests' memmove agent (one memmove per descriptor row)"),
            "correct": correct,
        }
    except Exception as error:  # noqa: BLE001 - the arm reports what stopped it rather than no line at all
        return {"unavailable": f"the reference worker leg failed: {type(error).__name__}: {error}"}
    finally:
        for worker in prefill_ranks + decode_ranks:
            worker.shutdown()


def port_leg(spec: Workload, reqs, producers, consumers, steps: int, threads: int) -> dict:
    """The same loads by the C restatement of the reference's path (oracle/kvx_oracle.c: block_descs rows for both
    sides, one memmove per row, rows split over `threads` host threads), on the same host caches."""
    from oracle import c_oracle
    from oracle.kv_oracle import Region, head_shares, lcm_heads

    import torch

    def regions(layers):
        out = []
        for t in layers:
            for part in t:
                head = part.stride(1) * 2 if t.dim() == 5 else 0
                out.append(Region(part.data_ptr(), part.stride(0) * 2, head))
        return out

    c_oracle.lib()
    src_regions = [regions(layers) for layers in producers]
    dst_regions = [regions(layers) for layers in consumers]
    heads = spec.kv_heads or lcm_heads(spec.decode_tp, spec.prefill_tp)
    times, moved = [], 0
    for _ in range(max(steps, 1)):
        started, moved = time.perf_counter(), 0
        for s_ids, d_ids in reqs:
            for rank in range(spec.decode_tp):
                for i, share in enumerate(head_shares(rank, spec.decode_tp, spec.prefill_tp, heads)):
                    d_addr, d_len = c_oracle.block_descs(dst_regions[rank], d_ids, share.local_head, share.num_heads,
                                                         i == 0)
                    s_addr, _ = c_oracle.block_descs(src_regions[share.remote_rank], s_ids, share.remote_head,
                                                     share.num_heads, i == 0)
                    moved += c_oracle.read(d_addr, s_addr, d_len, threads)
        times.append(time.perf_counter() - started)
    seconds = float(np.median(times))
    return {"value": round(moved / seconds / 1e9, 3), "unit": "GB/s", "kind": "port", "cores": threads,
            "ms_per_step": round(seconds * 1e3, 3), "steps": max(steps, 1),
            "sample": f"all {len(reqs)} requests per step ({moved / 1e9:.2f} GB) on the same host caches",
            "path": "C restatement of block_descs + one memmove per row, rows split over every host thread"}


def run_reference(args) -> None:
    """The reference arm, on the box's host cores: the reference's own NixlConnectorWorker pair (the primary value,
    kind "reference") and the C restatement beside it (kind "port"), on the same host caches of the workload -- the
    whole workload when host RAM allows. Rank 0 alone runs; other ranks exit."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import psutil

    spec = WORKLOADS[args.workload]
    lengths, reqs, num_blocks = workload(args.seed, args.requests, spec)
    layer_bytes = (num_blocks * spec.block * spec.head_dim * 2 * (1 if spec.mla else 2 * spec.kv_heads))
    need = 2 * spec.layers * layer_bytes  # both sides; the ranks of a side split one side's bytes
    available = psutil.virtual_memory().available
    ram_note = f"{need / 1e9:.1f} GB of host caches, {available / 1e9:.1f} GB available"
    if need > 0.6 * available:  # the largest prefix of the workload whose caches fit comfortably
        n = len(reqs)
        while n > 1:
            n -= max(1, n // 8)
            _, reqs, num_blocks = workload(args.seed, n, spec)
            layer_bytes = (num_blocks * spec.block * spec.head_dim * 2 * (1 if spec.mla else 2 * spec.kv_heads))
            if 2 * spec.layers * layer_bytes <= 0.6 * available:
                break
        ram_note += f": cut to the first {len(reqs)} requests"
    producers = host_rank_caches(spec, spec.prefill_tp, num_blocks, seed=args.seed + 1)
    consumers = host_rank_caches(spec, spec.decode_tp, num_blocks, seed=None)
    threads = len(os.sched_getaffinity(0))
    legs = {"reference": reference_worker_leg(spec, reqs, producers, consumers, max(args.steps, 1), args.warmup),
            "port": port_leg(spec, reqs, producers, consumers, min(max(args.steps, 1), 5), threads)}
    primary = legs["reference"] if "value" in legs["reference"] else legs["port"]
    gbs = primary["value"]
    line = {
        "metric": METRIC,
        "impl": "reference",
        "value": gbs,
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_8k_request": round(BYTES_8K_REQUEST / (gbs * 1e9) * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded bf16 host caches (distinct per block), seeded shuffled block tables",
        # The same workload our arm names at this N, so the two lines compare.
        "config": {"workload": (f"{spec.name}/loopback-1gpu" if args.gpus == 1 else
                                f"{spec.name}/{args.gpus // spec.group_size}x-tp{spec.prefill_tp}to{spec.decode_tp}"),
                   "shape": spec.describe(),
                   "requests_per_step": len(reqs),
                   "prompt_lengths": f"{spec.lengths[0]} [{spec.lengths[1]}, {spec.lengths[2]}], seed {args.seed}",
                   "mode": "pull",
                   "host_ram": ram_note,
                   "host_cpus": os.cpu_count()},
        "legs": legs,
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": primary["cores"], "kind": primary["kind"],
                         "sample": primary["sample"]},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=sorted(WORKLOADS), default="pair")
    p.add_argument("--mode", choices=["pull", "push"], default="pull")
    p.add_argument("--engine", choices=["auto", "lsu", "tma"], default="auto")
    p.add_argument("--tile-bytes", type=int, default=0)
    p.add_argument("--ctas-per-sm", type=int, default=0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--requests", type=int, default=0, help="a prefix of the workload's requests (small cases)")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true", help="skip the connector end-to-end timing")
    p.add_argument("--no-extras", action="store_true",
                   help="N=1: skip the store and layer-wise push measurements added to the line")
    p.add_argument("--kv-port", type=int, default=24600, help="first handshake port of the e2e connectors")
    p.add_argument("--peer-device", type=int, default=None,
                   help="N=1 only: put the destination cache on this GPU (one process, peer access over NVLink)")
    p.add_argument("--layerwise", action="store_true",
                   help="measure the per-layer push beside a synthetic prefill (exposed transfer time)")
    p.add_argument("--store", action="store_true", help="measure the per-token cache store (and fused push)")
    p.add_argument("--serial", action="store_true", help="with --store: plain launches (KVX_STORE_SERIAL)")
    p.add_argument("--fused", action="store_true",
                   help="with --layerwise: each layer stores new rows through store_kv, which pushes them too")
    p.add_argument("--poisson", action="store_true", help="latency under Poisson arrivals at 1-64 requests/s")
    p.add_argument("--staged", action="store_true", help="the pack -> push -> scatter path, stage by stage")
    p.add_argument("--relay-chunks", type=int, default=0, help="with --relay: request chunks per step (0: 8)")
    p.add_argument("--relay-sms", type=int, default=-1,
                   help="with --relay: SMs each of the two copy streams may use (default half; 0: every SM)")
    p.add_argument("--relay", action="store_true",
                   help="MLA workload: each decode rank pulls its part from the prefill rank, the rest from its peers")
    p.add_argument("--copy-engine", action="store_true",
                   help="baseline: one cudaMemcpyAsync per chunk (copy engines) against one kvx_copy launch")
    p.add_argument("--step-exchange", action="store_true",
                   help="host only: kv_connector_step's per-step output exchange, gloo gather vs step mailbox")
    p.add_argument("--rates", default="1,4,16,64", help="arrival rates for --poisson, requests per second")
    p.add_argument("--poisson-seconds", type=float, default=6.0, help="arrival window per rate")
    args = p.parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    elif args.step_exchange:
        run_step_exchange(args)
    elif args.copy_engine:
        run_copy_engine(args)
    elif args.poisson:
        run_poisson(args)
    elif args.staged:
        run_staged(args)
    elif args.store:
        run_store(args)
    elif args.layerwise:
        run_layerwise(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
