"""A pytest plugin for running the reference's own connector tests against this package. TEST ONLY.

Loaded into a pytest run of a lean-vLLM checkout's test files (`-p kvx_reference_swap`), it puts this package's
connector halves under the reference's "NixlConnector" entry of CONNECTORS (kv_transfer/__init__.py:31-45), the
one name the reference's tests configure, so every engine they build gets CudaIpcConnectorScheduler (and the worker
half). At the end of the session it writes how many scheduler halves were made to the file named by
KVX_SWAP_REPORT, so the caller can tell the swap took effect.
"""

import os

import lean_vllm.kv_transfer as ref_kv

from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorScheduler, CudaIpcConnectorWorker

_made = []


class _Counted(CudaIpcConnectorScheduler):
    def __init__(self, config):
        _made.append(config)
        super().__init__(config)


ref_kv.CONNECTORS["NixlConnector"] = (_Counted, CudaIpcConnectorWorker)


def pytest_sessionfinish(session, exitstatus):
    report = os.environ.get("KVX_SWAP_REPORT")
    if report:
        with open(report, "w") as f:
            f.write(str(len(_made)))
