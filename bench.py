"""Benchmark of the KV-cache transfer path: GB/s and ms per 8k-token request.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--mode pull|push] [--engine auto|lsu|tma]
    python bench.py --impl reference ...      # the reference's CPU transfer path (restated in oracle/), host cores

Workload: Qwen3-8B-shaped paged KV (36 layers x {K, V}, 8 KV heads x 128 dims, 256-token blocks, bf16, HND),
64 requests with prompt lengths uniform in [1024, 8192], source and destination block ids drawn from seeded
shuffled free lists, N(0,1) bf16 values. One step moves every block of every request once: one kvx_copy launch
with one job per request.

  N = 1   same-device loopback on cuda:0 (source and destination caches on one GPU): HBM-bound.
  N even  N/2 prefill->decode pairs (ranks 2p -> 2p+1), one process per GPU, caches mapped over CUDA IPC; the
          decode rank pulls (or, with --mode push, the prefill rank pushes) over NVLink. Pairs are independent
          (weak scaling); no collective touches the data path.

`value` is device-timed (CUDA events on the launching stream, max over ranks) with the caches resident in HBM;
`e2e` times the same transfers through the public transport call (host block tables marshalled per step, launch,
completion polled with the transfer's event) by the host clock. The caches exceed L2 many times over, so no flush
is needed between steps.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "KV transfer GB/s & ms per 8k-token request"
SHAPE = dict(layers=36, kv_heads=8, head_dim=128, block=256, itemsize=2)
BYTES_8K_REQUEST = 32 * 36 * 2 * 8 * 256 * 128 * 2  # 1,207,959,552: 32 blocks x 36 layers x K/V x 512 KiB
NVLINK_PEER_GBS = 770.0  # measured peer copy per direction on this pool's B200s (nominal 900)


def workload(seed: int = 0, n_requests: int = 64, lo: int = 1024, hi: int = 8192, block: int = 256):
    """Prompt lengths and per-request (src, dst) block ids from seeded shuffled free lists."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(lo, hi + 1, size=64)[:n_requests]  # a prefix of the same draw when fewer are asked
    counts = [math.ceil(int(n) / block) for n in lengths]
    total = sum(counts)
    num_blocks = total + max(8, total // 16)  # slack, so ids are spread over a larger cache
    src_free, dst_free = rng.permutation(num_blocks), rng.permutation(num_blocks)
    reqs, at = [], 0
    for c in counts:
        reqs.append((src_free[at : at + c].astype(np.int32), dst_free[at : at + c].astype(np.int32)))
        at += c
    return lengths, reqs, num_blocks


def chunk_bytes(kv_heads: int) -> int:
    return kv_heads * SHAPE["block"] * SHAPE["head_dim"] * SHAPE["itemsize"]


def request_bytes(n_blocks: int, kv_heads: int = SHAPE["kv_heads"]) -> int:
    return n_blocks * SHAPE["layers"] * 2 * chunk_bytes(kv_heads)


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


def cpu_baseline(lengths, reqs, seconds: float = 10.0, threads: int | None = None) -> dict:
    """The reference's CPU transfer path, restated in C (oracle/kvx_oracle.c): per request, block_descs rows for
    both sides, then one memmove per row, rows spread over host threads. Timed on a bounded sample: the first
    requests of the workload (at most 96 blocks) on host caches of the same shape, repeated for ~`seconds`."""
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
    layers = SHAPE["layers"]
    shape = (2, nb, SHAPE["kv_heads"], SHAPE["block"], SHAPE["head_dim"])
    src_caches = [np.full(shape, 0x3F80, dtype=np.uint16) for _ in range(layers)]
    dst_caches = [np.zeros(shape, dtype=np.uint16) for _ in range(layers)]
    for a in dst_caches:
        a.fill(1)  # touch every page before timing

    def regions(caches):
        return [Region(part.ctypes.data, part.strides[0], part.strides[1]) for c in caches for part in c]

    src_r, dst_r = regions(src_caches), regions(dst_caches)
    # Remap the sample's ids onto the sample-sized caches, keeping the shuffled order.
    remap, at = [], 0
    rng = np.random.default_rng(1)
    src_perm, dst_perm = rng.permutation(nb), rng.permutation(nb)
    for src, _ in sample:
        n = len(src)
        remap.append((src_perm[at : at + n], dst_perm[at : at + n]))
        at += n
    c_oracle.lib()
    moved, reps = 0, 0
    start = time.perf_counter()
    while True:
        for src_ids, dst_ids in remap:
            d_addr, d_len = c_oracle.block_descs(dst_r, dst_ids, 0, SHAPE["kv_heads"], False)
            s_addr, _ = c_oracle.block_descs(src_r, src_ids, 0, SHAPE["kv_heads"], False)
            moved += c_oracle.read(d_addr, s_addr, d_len, threads)
        reps += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds or reps >= 200:
            break
    gbs = moved / elapsed / 1e9
    # Spot-check the copy: the first request's first destination chunk holds the source pattern.
    assert int(dst_caches[0][0, remap[0][1][0], 0, 0, 0]) == 0x3F80
    return {
        "value": round(gbs, 3),
        "unit": "GB/s",
        "cores": threads,
        "kind": "port",
        "sample": (f"first {len(sample)} requests of the workload ({nb} blocks, {request_bytes(nb) / 1e9:.2f} GB) on "
                   f"host caches of the same shape, {reps} passes in {elapsed:.1f} s; C restatement of "
                   "block_descs + one memmove per row, rows split over threads"),
        "ms_per_8k_request": round(BYTES_8K_REQUEST / (gbs * 1e9) * 1e3, 3),
        "host_cpus": os.cpu_count(),
    }


# ------------------------------------------------------------------------------------------------ GPU arm


def alloc_cache(num_blocks: int, device, fill: bool, seed: int):
    import torch

    shape = (2, num_blocks, SHAPE["kv_heads"], SHAPE["block"], SHAPE["head_dim"])
    layers = []
    g = torch.Generator(device=device).manual_seed(seed)
    for _ in range(SHAPE["layers"]):
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


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    from lean_vllm_b200._native import ENGINE_AUTO, ENGINE_LSU, ENGINE_TMA, flags
    from lean_vllm_b200.kv_transfer import transport
    from lean_vllm_b200.kv_transfer.transport import CacheTable, CopyJob

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}; launch N>1 with torchrun")
    if world > 1 and world % 2:
        raise SystemExit("N > 1 runs prefill->decode pairs, so N must be even")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    gloo = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
        gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=180))

    engine = {"auto": ENGINE_AUTO, "lsu": ENGINE_LSU, "tma": ENGINE_TMA}[args.engine]
    copy_flags = flags(engine, args.tile_bytes, args.ctas_per_sm)
    lengths, reqs, num_blocks = workload(args.seed, args.requests)
    step_blocks = sum(len(s) for s, _ in reqs)
    step_bytes = request_bytes(step_blocks)
    pairs = max(world // 2, 1)
    loopback = world == 1
    producer = loopback or rank % 2 == 0
    consumer = loopback or rank % 2 == 1
    active = loopback or (consumer if args.mode == "pull" else producer)

    src = alloc_cache(num_blocks, device, fill=True, seed=1000 + rank) if producer else None
    dst = alloc_cache(num_blocks, device, fill=False, seed=0) if consumer else None
    torch.cuda.synchronize()

    # Each side's cache as a CacheTable in the launching process: peers' caches through CUDA IPC.
    mine = src if producer and not loopback else dst
    handles = None
    if not loopback:
        exported = [transport.export(t.data_ptr()) for t in mine]
        table = CacheTable.from_tensors(mine)
        info = [None] * world
        dist.all_gather_object(info, (exported, table.regions, table.num_blocks), group=gloo)
        peer = rank ^ 1
        handles = info[peer][0]
        if active:
            transport.enable_peer_access(local_rank, local_rank ^ 1)
            peer_regions = []
            for layer, blob in enumerate(handles):  # one exported tensor per layer: its K region, then V
                k_addr = info[peer][1][2 * layer][0]
                k_here = transport.open_mapping(blob)
                for addr, bb, hb in info[peer][1][2 * layer : 2 * layer + 2]:
                    peer_regions.append((k_here + (addr - k_addr), bb, hb))
            peer_table = CacheTable(peer_regions, info[peer][2])
            if producer:
                caches = [CacheTable.from_tensors(src), peer_table]
            else:
                caches = [peer_table, CacheTable.from_tensors(dst)]
    else:
        caches = [CacheTable.from_tensors(src), CacheTable.from_tensors(dst)]

    jobs = [CopyJob(0, 1, s, d, 0, 0, SHAPE["kv_heads"]) for s, d in reqs] if active else []
    stream = torch.cuda.Stream(device=device)
    sid = stream.cuda_stream

    def step():
        if jobs:
            transport.copy(caches, jobs, sid, copy_flags)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()

    launches0 = transport.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        barrier()
    launches = transport.launch_count() - launches0
    elapsed_ms = start.elapsed_time(end) if active else 0.0
    t = torch.tensor([elapsed_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    launch_total = torch.tensor([launches], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(launch_total)

    # Correctness spot-check after timing: the first and last requests' blocks landed bit for bit (across a pair,
    # by comparing position-weighted digests computed on each side).
    def digest(layers, ids):
        index = torch.as_tensor(ids, device=device, dtype=torch.long)
        out = []
        for layer in (0, SHAPE["layers"] - 1):
            flat = layers[layer][:, index].contiguous().view(torch.int16).reshape(-1).to(torch.int64)
            weights = torch.arange(flat.numel(), device=device, dtype=torch.int64) % 65521 + 1
            out += [int(flat.sum().item()), int((flat * weights).sum().item())]
        return out

    ok = True
    checks = [(reqs[0][0], reqs[0][1]), (reqs[-1][0], reqs[-1][1])]
    if loopback:
        ok = all(digest(dst, d) == digest(src, s) for s, d in checks)
    else:
        mine_digest = [digest(src, s) if producer else digest(dst, d) for s, d in checks]
        digests = [None] * world
        dist.all_gather_object(digests, mine_digest, group=gloo)
        ok = digests[rank] == digests[rank ^ 1]

    # e2e: the same loads through the connector's public API (start_load_kv -> get_finished), host clock.
    e2e_ms, e2e_bytes = None, 0
    if args.steps and not args.no_e2e:
        e2e_ms, e2e_bytes = e2e_connector(args, world, rank, src, dst, reqs, barrier, gloo, device)
        e = torch.tensor([e2e_ms], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(e, op=dist.ReduceOp.MAX)
        e2e_ms = float(e.item())

    ok_t = torch.tensor([0.0 if ok else 1.0], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(ok_t, op=dist.ReduceOp.MAX)
    clock_summary = clocks.summary()

    if rank == 0:
        ms_per_step = max_ms / args.steps
        total_bytes = step_bytes * pairs
        gbs = total_bytes / (ms_per_step * 1e-3) / 1e9
        per_pair_gbs = step_bytes / (ms_per_step * 1e-3) / 1e9
        ms_8k = BYTES_8K_REQUEST / (per_pair_gbs * 1e9) * 1e3
        peaks = {}
        peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
        if os.path.exists(peaks_path):
            with open(peaks_path) as f:
                peaks = json.load(f)
        traffic = load_traffic().get("loopback" if loopback else args.mode)
        if loopback:
            hbm = peaks.get("hbm_gbs", 6650.0)
            achieved = 2 * step_bytes / (ms_per_step * 1e-3) / 1e9
            roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(achieved / hbm, 4),
                        "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                        "traffic": traffic.get("bytes_per_launch") if traffic else None,
                        "algorithmic_bytes_per_launch": 2 * step_bytes}
        else:
            achieved = per_pair_gbs
            roofline = {"bound": "nvlink", "achieved": round(achieved, 1), "peak": NVLINK_PEER_GBS, "unit": "GB/s",
                        "frac": round(achieved / NVLINK_PEER_GBS, 4),
                        "peak_source": "measured peer copy per direction (nominal 900)",
                        "traffic": traffic.get("bytes_per_launch") if traffic else None,
                        "algorithmic_bytes_per_launch": step_bytes}
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
                "workload": ("qwen3-8b-kv/loopback-1gpu" if loopback else f"qwen3-8b-kv/{pairs}x-pair-tp1to1"),
                "shape": "36 layers x {K,V}, 8 KV heads x 128, block 256 tokens, bf16, HND",
                "requests_per_step": len(reqs),
                "prompt_lengths": f"uniform [1024, 8192], seed {args.seed}",
                "blocks_per_step_per_pair": step_blocks,
                "bytes_per_step_per_pair": step_bytes,
                "pairs": pairs,
                "mode": "loopback" if loopback else args.mode,
                "engine": args.engine,
                "parallelism": "1 GPU" if loopback else f"{pairs} independent prefill->decode pairs",
                "l2": f"no flush: each step reads and writes {2 * step_bytes / 1e9:.1f} GB, far beyond the 126 MB L2",
            },
            "roofline": roofline,
            "gpu_launches": int(launch_total.item()),
            "clocks": clock_summary,
            "correct": bool(ok_t.item() == 0.0),
        }
        if e2e_ms is not None:
            ids_bytes = 2 * 4 * step_blocks
            line["e2e"] = {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                           "ms_per_step": round(e2e_ms, 4),
                           "h2d_bytes_per_step": ids_bytes * pairs, "d2h_bytes_per_step": 0,
                           "bytes_reported_by_connector": e2e_bytes,
                           "path": ("CudaIpcConnectorWorker.start_load_kv(64 ReqToRecv from host lists) -> "
                                    "get_finished() until all 64 finished_recving; one kvx launch per load, block "
                                    "ids carried in the launch, completion by event query")}
        if loopback and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(lengths, reqs, seconds=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        if handles is not None and active:
            for blob in handles:
                transport.close_mapping(blob)
        dist.destroy_process_group()


def e2e_connector(args, world, rank, src, dst, reqs, barrier, gloo, device):
    """Times the step's loads through CudaIpcConnectorWorker (host clock, per step, consumer side): a producer
    worker holds the source cache and a consumer worker loads every request. N=1 runs both in this process; a pair
    runs the producer on rank 2p and the consumer on rank 2p+1. Returns (ms per step, bytes the connector counted)."""
    import torch
    import torch.distributed as dist
    from dataclasses import dataclass

    from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVTransferConfig, ReqToRecv
    from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker

    @dataclass
    class WorkerConfig:
        kv_transfer: KVTransferConfig
        tensor_parallel_size: int = 1
        kvcache_block_size: int = SHAPE["block"]
        kv_cache_layout: str = "HND"

    base_port = args.kv_port + 16 * (rank // 2)
    loopback = world == 1
    producer_worker = consumer_worker = None
    if loopback or rank % 2 == 0:
        kv = KVTransferConfig(kv_role="kv_producer", kv_port=base_port, engine_id="bench-prefill")
        producer_worker = CudaIpcConnectorWorker(WorkerConfig(kv), 0)
        producer_worker.register_kv_caches(src)
    if loopback or rank % 2 == 1:
        kv = KVTransferConfig(kv_role="kv_consumer", kv_port=base_port + 8, engine_id="bench-decode")
        consumer_worker = CudaIpcConnectorWorker(WorkerConfig(kv), 0)
        consumer_worker.register_kv_caches(dst)

    def one_step(tag: str) -> tuple[float, int]:
        sends = {f"{tag}-{i}": s.tolist() for i, (s, _) in enumerate(reqs)}
        recvs = {f"{tag}-{i}": ReqToRecv(d.tolist(), s.tolist(), f"{tag}-{i}", "bench-prefill", "127.0.0.1",
                                         base_port, 1) for i, (s, d) in enumerate(reqs)}
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
        if producer_worker is not None:  # every held request is released once its reader has notified
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
    return float(np.median(times)), nbytes


def run_reference(args) -> None:
    """The reference arm: the reference's CPU transfer path (C restatement in oracle/, all host threads)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    lengths, reqs, num_blocks = workload(args.seed)
    cpu_seconds = max(2.0, min(args.cpu_seconds, 40.0 / max(args.steps + args.warmup, 1)))
    for _ in range(args.warmup):
        cpu_baseline(lengths, reqs, seconds=0.5)
    results = [cpu_baseline(lengths, reqs, seconds=cpu_seconds) for _ in range(max(args.steps, 1))]
    gbs = float(np.median([r["value"] for r in results]))
    base = results[0]
    line = {
        "metric": METRIC,
        "impl": "reference",
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_8k_request": round(BYTES_8K_REQUEST / (gbs * 1e9) * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: bf16-sized host caches, seeded shuffled block tables",
        "config": {"workload": "qwen3-8b-kv (reference CPU transfer path)", "requests": "bounded sample per step",
                   "prompt_lengths": f"uniform [1024, 8192], seed {args.seed}"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": base["cores"], "kind": "port",
                         "sample": base["sample"]},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--mode", choices=["pull", "push"], default="pull")
    p.add_argument("--engine", choices=["auto", "lsu", "tma"], default="auto")
    p.add_argument("--tile-bytes", type=int, default=0)
    p.add_argument("--ctas-per-sm", type=int, default=0)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--requests", type=int, default=64, help="a prefix of the 64 requests (small profiling cases)")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true", help="skip the connector end-to-end timing")
    p.add_argument("--kv-port", type=int, default=24600, help="first handshake port of the e2e connectors")
    args = p.parse_args(argv)
    if args.warmup < 3 and args.impl == "ours" and args.steps > 0:
        print("note: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
