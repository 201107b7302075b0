"""The connector between separate processes on CPU: two gloo ranks, a prefill instance and a decode instance, each a
process with its caches in shared files (tests/shm_transport.py). Covers the cross-process handshake, a pull with
its reader notification and release, and a push with its announcement -- the N>1 paths bench.py drives on GPUs."""

import os
import socket
from dataclasses import dataclass
from time import monotonic, sleep

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


BLOCKS, BLOCK, HEADS, DIM = 10, 4, 4, 8


@dataclass
class Cfg:
    kv_transfer: object
    tensor_parallel_size: int = 1
    kvcache_block_size: int = BLOCK
    kv_cache_layout: str = "HND"
    kvx_accept_push: bool = True


def _full(seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(2, BLOCKS, HEADS, BLOCK, DIM, generator=g).to(torch.bfloat16) for _ in range(2)]


def _wait(worker, field, want, timeout=20.0):
    got, deadline = set(), monotonic() + timeout
    while got != want and monotonic() < deadline:
        out = worker.get_finished()
        if out.failed_recving:
            raise AssertionError(f"failed: {out.failed_recving}")
        got |= getattr(out, field)
        sleep(0.005)
    assert got == want, (field, got, want)


def _rank(rank: int, world: int, master_port: int, kv_port: int, failures):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(master_port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVTransferConfig, ReqToRecv, cuda_ipc_connector
        from lean_vllm_b200.kv_transfer.base import ReqToSave
        from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker
        from tests.shm_transport import ShmTransport, shared_cache

        cuda_ipc_connector.make_transport = ShmTransport
        layers = _full(100 if rank == 0 else 200)
        caches = [shared_cache(t.shape, t) for t in layers]
        role = "kv_producer" if rank == 0 else "kv_consumer"
        kv = KVTransferConfig(kv_role=role, kv_port=kv_port + 10 * rank, engine_id=f"e{rank}")
        worker = CudaIpcConnectorWorker(Cfg(kv), 0)
        worker.register_kv_caches(caches)
        dist.barrier()

        # Pull: the decode rank copies blocks [7, 2] of the prefill rank into its [0, 5].
        if rank == 0:
            worker.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-pull": [7, 2]}))
            _wait(worker, "finished_sending", {"p-pull"})
        else:
            worker.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-pull": ReqToRecv(
                [0, 5], [7, 2], "p-pull", "e0", "127.0.0.1", kv_port, 1)}))
            _wait(worker, "finished_recving", {"d-pull"})
            prefill = _full(100)
            for layer in range(2):
                assert torch.equal(caches[layer][:, [0, 5]], prefill[layer][:, [7, 2]]), layer
        dist.barrier()

        # Push with its announcement: the decode rank announces [1, 8]; the prefill rank pushes its [3, 4] there.
        if rank == 1:
            worker.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-push": ReqToRecv(
                [1, 8], [], "push-1", "", "127.0.0.1", kv_port, 1, pushed=True)}))
        dist.barrier()
        if rank == 0:
            worker.start_load_kv(KVConnectorMetadata(reqs_to_save={"p-push": ReqToSave([3, 4], push_id="push-1")}))
            sleep(0.1)
            worker.save_kv_layer(0)
            worker.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-push": [3, 4]}))
            _wait(worker, "finished_sending", {"p-push"})
        else:
            _wait(worker, "finished_recving", {"d-push"})
            prefill = _full(100)
            for layer in range(2):
                assert torch.equal(caches[layer][:, [1, 8]], prefill[layer][:, [3, 4]]), layer
        dist.barrier()
        worker.shutdown()
        dist.destroy_process_group()
    except BaseException as error:  # noqa: BLE001 - reported to the parent
        failures.put(f"rank {rank}: {type(error).__name__}: {error}")
        raise
    finally:
        from tests.shm_transport import remove_files

        remove_files()


def test_pull_and_announced_push_between_two_processes():
    if not os.path.isdir("/dev/shm"):
        pytest.skip("needs /dev/shm")
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    master_port, kv_port = _free_port(), _free_port()  # the same for both ranks
    procs = [ctx.Process(target=_rank, args=(r, 2, master_port, kv_port, failures)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    errors = []
    while not failures.empty():
        errors.append(failures.get())
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


LATENT = 6


def _latents(seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(1, BLOCKS, BLOCK, LATENT, generator=g).to(torch.bfloat16) for _ in range(2)]


def _relay_rank(rank: int, world: int, master_port: int, kv_port: int, failures):
    """Rank 0 a prefill instance (TP1), ranks 1-2 one decode instance (TP2) relaying MLA latents between them."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(master_port), LEAN_VLLM_KVX_RELAY="1")
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVTransferConfig, ReqToRecv, cuda_ipc_connector
        from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker
        from tests.shm_transport import ShmTransport, shared_cache

        cuda_ipc_connector.make_transport = ShmTransport
        producer = rank == 0
        layers = _latents(300 if producer else 400 + rank)
        caches = [shared_cache(t.shape, t) for t in layers]
        kv = KVTransferConfig(kv_role="kv_producer" if producer else "kv_consumer",
                              kv_port=kv_port if producer else kv_port + 10, engine_id="p" if producer else "d")
        worker = CudaIpcConnectorWorker(Cfg(kv, tensor_parallel_size=1 if producer else 2), 0 if producer else rank - 1)
        worker.register_kv_caches(caches)
        dist.barrier()
        local, remote = [0, 5, 3, 8, 1], [7, 2, 9, 4, 6]
        if producer:
            worker.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-relay": remote}))
            _wait(worker, "finished_sending", {"p-relay"})  # both decode ranks read their part
        else:
            worker.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-relay": ReqToRecv(
                local, remote, "p-relay", "p", "127.0.0.1", kv_port, 1)}))
            _wait(worker, "finished_recving", {"d-relay"})
            prefill = _latents(300)
            for layer in range(2):
                assert torch.equal(caches[layer][:, local], prefill[layer][:, remote]), layer
        dist.barrier()
        worker.shutdown()
        dist.destroy_process_group()
    except BaseException as error:  # noqa: BLE001 - reported to the parent
        failures.put(f"rank {rank}: {type(error).__name__}: {error}")
        raise
    finally:
        from tests.shm_transport import remove_files

        remove_files()


def test_a_relayed_latent_load_between_three_processes():
    """Each decode rank (its own process) pulls its part from the prefill process and the other part from its peer
    process, through shared-file caches: both end with every latent block, the producer frees after both reads."""
    if not os.path.isdir("/dev/shm"):
        pytest.skip("needs /dev/shm")
    ctx = mp.get_context("spawn")
    failures = ctx.Queue()
    master_port, kv_port = _free_port(), _free_port()
    procs = [ctx.Process(target=_relay_rank, args=(r, 3, master_port, kv_port, failures)) for r in range(3)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    errors = []
    while not failures.empty():
        errors.append(failures.get())
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
