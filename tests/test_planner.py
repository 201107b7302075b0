"""The connector's per-load byte count and id checks (CudaIpcConnectorWorker._job_bytes) against libkvx's own
planner (kvx_job_bytes): the same bytes for every share shape, the same refusals for ids outside a cache. Host only:
the planner reads region tables and ids, never device memory."""

import os
import random
from dataclasses import dataclass

import pytest
import torch

from lean_vllm_b200 import _native
from lean_vllm_b200.kv_transfer import KVTransferConfig
from lean_vllm_b200.kv_transfer import transport as kvx
from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker, _Remote
from lean_vllm_b200.kv_transfer.transport import CacheTable, CopyJob

pytestmark = pytest.mark.skipif(not os.path.exists(_native.LIB_PATH), reason="libkvx.so is not built here")


@dataclass
class Cfg:
    kv_transfer: KVTransferConfig
    tensor_parallel_size: int = 1
    kvcache_block_size: int = 16
    kv_cache_layout: str = "HND"


class PlannerOnly:
    """The transport surface _job_bytes uses, over fake addresses: libkvx plans without touching memory."""

    def __init__(self, local: CacheTable):
        self.local = local

    def job_bytes(self, tables, jobs, layer=None):
        return kvx.job_bytes([self.local, *tables], jobs)


def table(base, layers, heads, block, dim, latent, num_blocks):
    regions = []
    for layer in range(layers):
        if latent:
            regions.append((base + layer * (1 << 30), block * dim * 2, 0))
        else:
            for part in range(2):
                block_bytes = heads * block * dim * 2
                regions.append((base + (2 * layer + part) * (1 << 30), block_bytes, block * dim * 2))
    return CacheTable(regions, num_blocks)


@pytest.mark.parametrize("latent", [False, True], ids=["kv", "latents"])
def test_the_connector_counts_what_the_planner_counts(latent):
    rng = random.Random(5)
    for _ in range(60):
        layers, heads, dim = rng.randint(1, 4), rng.choice([2, 4, 8]), rng.choice([8, 64, 128])
        local_blocks, remote_blocks = rng.randint(4, 40), rng.randint(4, 40)
        local = table(1 << 40, layers, heads, 16, dim, latent, local_blocks)
        remote_table = table(2 << 40, layers, heads, 16, dim, latent, remote_blocks)
        worker = CudaIpcConnectorWorker(Cfg(KVTransferConfig(kv_role="kv_consumer")), 0)
        worker.kv_caches = [torch.empty(2 if not latent else 1, local_blocks, 1, 1, 1)]
        worker.transport = PlannerOnly(local)
        remote = _Remote("p", 1, remote_blocks, {}, remote_table, None)
        n = rng.randint(0, 6)
        src = [rng.randrange(remote_blocks) for _ in range(n)]
        dst = [rng.randrange(local_blocks) for _ in range(n)]
        first, count = rng.randint(0, heads - 1), 0
        count = rng.randint(1, heads - first)
        job = CopyJob(1, 0, src, dst, first, first, count, latents=rng.random() < 0.5)
        want = kvx.job_bytes([local, remote_table], [job])
        assert worker._job_bytes(remote, job) == want
        assert worker._job_bytes(remote, job) == want  # the cached per-block figure gives the same
        if n:
            bad_src = CopyJob(1, 0, src[:-1] + [remote_blocks], dst, first, first, count, job.latents)
            with pytest.raises(_native.KvxRangeError):
                kvx.job_bytes([local, remote_table], [bad_src])
            with pytest.raises(RuntimeError, match="past the producer's"):
                worker._job_bytes(remote, bad_src)
            bad_dst = CopyJob(1, 0, src, dst[:-1] + [-1], first, first, count, job.latents)
            with pytest.raises(_native.KvxRangeError):
                kvx.job_bytes([local, remote_table], [bad_dst])
            with pytest.raises(RuntimeError, match="past this rank's"):
                worker._job_bytes(remote, bad_dst)
        worker._context.term()
        os.close(worker._wake)  # never registered, so never shut down
