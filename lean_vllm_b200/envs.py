"""Environment variables this package reads, parsed at access (the names lean-vLLM's envs.py uses where shared)."""

import os
from collections.abc import Callable
from typing import Any

environment_variables: dict[str, Callable[[], Any]] = {
    # Seconds a prefill instance holds a request's KV blocks for decode instances to read (lean_vllm/envs.py:31).
    "LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT": lambda: float(os.getenv("LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT", "480")),
    # kvx copy engine for connector transfers: "auto", "lsu" or "tma".
    "LEAN_VLLM_KVX_ENGINE": lambda: os.getenv("LEAN_VLLM_KVX_ENGINE", "auto").lower(),
}


def __getattr__(name: str):
    if name in environment_variables:
        return environment_variables[name]()
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def __dir__():
    return list(environment_variables)
