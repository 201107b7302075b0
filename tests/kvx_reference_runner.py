"""The reference engine's model runner, set up for end-to-end tests of this connector on CPU. TEST ONLY.

Importing this module prepares a lean-vLLM checkout (KVX_REFERENCE_ROOT) in the importing process:
- CudaIpcConnector joins the reference's CONNECTORS table;
- the connector's transport is the cross-process host one (tests/shm_transport.py);
- LLMEngine's ModelRunner becomes SharedCacheModelRunner, which allocates each layer's KV cache in a shared file
  under KVX_TEST_CACHE_DIR, so a peer process can map the bytes.

The engine starts its other tensor-parallel ranks by spawning ModelRunner. Each spawned rank unpickles this
module's class, and so imports this module and gets the same setup. A rank of any tensor-parallel size therefore
runs the real model with this connector.
"""

import os
import sys

import torch

torch._dynamo.config.disable = True  # the reference compiles a few layers; this image has no OpenMP for inductor
if os.environ["KVX_REFERENCE_ROOT"] not in sys.path:
    sys.path.insert(0, os.environ["KVX_REFERENCE_ROOT"])

import lean_vllm.kv_transfer as ref_kv  # noqa: E402
from lean_vllm.engine import llm_engine, model_runner  # noqa: E402

from lean_vllm_b200.kv_transfer import cuda_ipc_connector  # noqa: E402
from lean_vllm_b200.kv_transfer.cuda_ipc_connector import (  # noqa: E402
    CudaIpcConnectorScheduler,
    CudaIpcConnectorWorker,
)
from tests.shm_transport import ShmTransport, shared_cache  # noqa: E402

ref_kv.CONNECTORS["CudaIpcConnector"] = (CudaIpcConnectorScheduler, CudaIpcConnectorWorker)
cuda_ipc_connector.make_transport = ShmTransport


class SharedCacheModelRunner(model_runner.ModelRunner):
    """The reference's ModelRunner, with its KV caches allocated in shared files. With KVX_TEST_STEP=mailbox its
    kv_connector_step is this package's KVConnectorStep, wired in as a maintainer would: the ranks' outputs reach
    rank 0 through the shared-memory step mailbox instead of gather_object."""

    def kv_connector_step(self, metadata):
        if os.environ.get("KVX_TEST_STEP") != "mailbox":
            return super().kv_connector_step(metadata)
        if getattr(self, "_kv_step", None) is None:  # every rank gets here on the same step, through call()
            from lean_vllm_b200.kv_transfer import KVConnectorStep

            self._kv_step = KVConnectorStep(self.kv_connector, self.rank, self.world_size,
                                            group=getattr(self, "call_group", None))
        return self._kv_step(metadata)

    def allocate_kv_cache(self):
        def shared_empty(shape, **_):
            assert torch.get_default_dtype() == torch.bfloat16
            return shared_cache(tuple(shape), directory=os.environ["KVX_TEST_CACHE_DIR"])

        empty, torch.empty = torch.empty, shared_empty
        try:
            super().allocate_kv_cache()
        finally:
            torch.empty = empty


llm_engine.ModelRunner = SharedCacheModelRunner
