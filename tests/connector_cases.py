"""Shared set-up for the connector tests: worker halves of a prefill and a decode instance in one process.

Mirrors the reference's own connector tests (tests/test_nixl_connector.py): CPU-sized caches of 12 blocks of 4
tokens, 12 heads of 8 (which split over 1, 2, 3, 4 and 6 ranks) or 6-wide latents, seeded torch.randn -> bf16, and
loads of blocks [7, 2, 9] into [0, 5, 3]. The same cases run on CPU over tests/host_transport.py and on a GPU over
the kvx transport.
"""

from __future__ import annotations

import socket
from dataclasses import dataclass
from time import monotonic, sleep

import torch

from lean_vllm_b200.kv_transfer import KVConnectorOutput, KVTransferConfig, ReqToRecv
from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker

NUM_BLOCKS, BLOCK, HEAD_DIM, LATENT_DIM = 12, 4, 8, 6
NUM_HEADS = 12
TP_PAIRS = [(1, 1), (2, 2), (1, 2), (2, 1), (1, 4), (4, 1), (2, 4), (4, 2), (4, 6), (6, 4), (2, 3)]


@dataclass
class WorkerConfig:
    kv_transfer: KVTransferConfig
    tensor_parallel_size: int = 1
    kvcache_block_size: int = BLOCK
    kv_cache_layout: str = "HND"
    kvx_accept_push: bool = False


_handed_out: set[int] = set()


def free_port(span: int = 8) -> int:
    """A port p with p .. p+span-1 free now and not handed out before in this process: an instance's ranks bind
    kv_port + rank, so two instances need disjoint spans."""
    for _ in range(200):
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            base = s.getsockname()[1]
        ports = range(base, base + span)
        if base + span > 65535 or any(p in _handed_out for p in ports):
            continue
        socks = []
        try:
            for p in ports:
                sock = socket.socket()
                socks.append(sock)
                sock.bind(("127.0.0.1", p))
        except OSError:
            continue
        finally:
            for sock in socks:
                sock.close()
        _handed_out.update(ports)
        return base
    raise RuntimeError("no free port span")


def full_cache(seed: int, mla: bool) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    shape = (1, NUM_BLOCKS, BLOCK, LATENT_DIM) if mla else (2, NUM_BLOCKS, NUM_HEADS, BLOCK, HEAD_DIM)
    return torch.randn(*shape, generator=g).to(torch.bfloat16)


def rank_cache(full: torch.Tensor, rank: int, tp_size: int) -> torch.Tensor:
    if full.dim() == 4:
        return full.clone()
    per = NUM_HEADS // tp_size
    return full[:, :, rank * per : (rank + 1) * per].clone()


class Sides:
    """Creates instances (lists of worker halves) and shuts them all down at the end."""

    def __init__(self, device: str = "cpu"):
        self.device = device
        self.workers: list[CudaIpcConnectorWorker] = []

    def make(self, role: str, tp_size: int, full, port: int = 0, engine_id: str = "prefill",
             accept_push: bool = False):
        """An instance of tp_size ranks; `full` is one layer's cache (every rank's heads) or a list of layers."""
        port = port or free_port()
        layers = full if isinstance(full, list) else [full]
        side = []
        for rank in range(tp_size):
            kv = KVTransferConfig(kv_connector="CudaIpcConnector", kv_role=role, kv_port=port, engine_id=engine_id)
            config = WorkerConfig(kv, tensor_parallel_size=tp_size, kvx_accept_push=accept_push)
            worker = CudaIpcConnectorWorker(config, rank)
            worker.register_kv_caches([rank_cache(layer, rank, tp_size).to(self.device) for layer in layers])
            side.append(worker)
        self.workers.extend(side)
        return side

    def close(self):
        for worker in self.workers:
            worker.shutdown()


def recv(producers, local, remote, **overrides) -> ReqToRecv:
    kv = producers[0].kv_transfer
    fields = dict(local_block_ids=local, remote_block_ids=remote, remote_request_id="p-1",
                  remote_engine_id=kv.engine_id, remote_host=kv.kv_ip, remote_port=kv.kv_port,
                  remote_tp_size=len(producers))
    fields.update(overrides)
    return ReqToRecv(**fields)


def wait_for(worker, timeout: float = 10.0) -> KVConnectorOutput:
    deadline = monotonic() + timeout
    while monotonic() < deadline:
        output = worker.get_finished()
        if output:
            return output
        sleep(0.002)
    raise AssertionError("no transfer finished")
