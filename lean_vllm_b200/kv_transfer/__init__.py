"""The KV connector API and the CUDA-IPC connector: a drop-in for lean_vllm.kv_transfer (reference __init__.py:1-45).

`CONNECTORS` maps a kv_transfer_config `kv_connector` name to its scheduler and worker halves, exactly as the
reference's factory does; the worker half is imported lazily so the scheduler half (engine process) needs no CUDA.
"""

from lean_vllm_b200.kv_transfer.base import (
    KVConnectorMetadata,
    KVConnectorOutput,
    KVConnectorScheduler,
    KVConnectorWorker,
    KVOutputAggregator,
    KVTransferConfig,
    KVTransferStats,
    ReqToRecv,
    check_kv_transfer_params,
)
from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorScheduler, CudaIpcConnectorWorker
from lean_vllm_b200.kv_transfer.step import KVConnectorStep

__all__ = [
    "CONNECTORS",
    "KVConnectorMetadata",
    "KVConnectorOutput",
    "KVConnectorScheduler",
    "KVConnectorStep",
    "KVConnectorWorker",
    "KVOutputAggregator",
    "KVTransferConfig",
    "KVTransferStats",
    "ReqToRecv",
    "check_kv_transfer_params",
    "create_scheduler_connector",
    "create_worker_connector",
    "parse_kv_transfer_config",
]

CONNECTORS = {"CudaIpcConnector": (CudaIpcConnectorScheduler, CudaIpcConnectorWorker)}


def parse_kv_transfer_config(value) -> KVTransferConfig:
    kv_transfer = KVTransferConfig.parse(value)
    if kv_transfer.kv_connector not in CONNECTORS:
        raise ValueError(f"unknown kv_connector {kv_transfer.kv_connector!r}, expected one of {sorted(CONNECTORS)}")
    return kv_transfer


def create_scheduler_connector(config) -> KVConnectorScheduler:
    return CONNECTORS[config.kv_transfer.kv_connector][0](config)


def create_worker_connector(config, rank: int) -> KVConnectorWorker:
    return CONNECTORS[config.kv_transfer.kv_connector][1](config, rank)
