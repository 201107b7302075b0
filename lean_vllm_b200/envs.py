"""Environment variables this package reads, parsed at access (the names lean-vLLM's envs.py uses where shared)."""

import os
from collections.abc import Callable
from typing import Any

environment_variables: dict[str, Callable[[], Any]] = {
    # Seconds a prefill instance holds a request's KV blocks for decode instances to read (lean_vllm/envs.py:31).
    "LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT": lambda: float(os.getenv("LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT", "480")),
    # kvx copy engine for connector transfers: "auto", "lsu" or "tma".
    "LEAN_VLLM_KVX_ENGINE": lambda: os.getenv("LEAN_VLLM_KVX_ENGINE", "auto").lower(),
    # A decode (kv_consumer) rank also answers handshakes on kv_port + rank, so prefill ranks can push into it.
    "LEAN_VLLM_KVX_ACCEPT_PUSH": lambda: os.getenv("LEAN_VLLM_KVX_ACCEPT_PUSH", "0").strip().lower()
    not in ("", "0", "false"),
    # A decode instance of several ranks loading MLA latents (replicated on every rank) splits the copy: each rank
    # pulls 1/tp of the blocks from the prefill rank, then the rest from its peer decode ranks, so the prefill GPU
    # sends each byte once. Its ranks then answer handshakes on kv_port + rank, as with ACCEPT_PUSH.
    "LEAN_VLLM_KVX_RELAY": lambda: os.getenv("LEAN_VLLM_KVX_RELAY", "0").strip().lower() not in ("", "0", "false"),
    # 1: store_kv's push to the decode ranks runs as a second launch on the save stream (the local store stays on
    # the engine's stream); 0 (default): one launch on the engine's stream writes both. Measured beside a 1.4 PFLOP/s
    # prefill the two are within run-to-run noise (0.5-0.9 % exposed), so the simpler one is the default.
    "LEAN_VLLM_KVX_FUSED_ASYNC": lambda: os.getenv("LEAN_VLLM_KVX_FUSED_ASYNC", "0").strip().lower()
    not in ("", "0", "false"),
    # Behind copies in flight, loads planned in one pass of the transfer thread share a copy launch until they add
    # up to this many bytes (a load that finds none of its rank's copies in flight launches at once, for its
    # latency). 2 GiB: on one B200, 64 Qwen3-8B-shaped loads went from 64 launches to 17 and their end-to-end rate
    # from 0.944 to 0.967 of the device-timed copy.
    "LEAN_VLLM_KVX_BATCH_BYTES": lambda: int(os.getenv("LEAN_VLLM_KVX_BATCH_BYTES", str(2 << 30))),
    # 1 (default): when none of a decode rank's copies is in flight, start_load_kv launches the step's first load
    # itself if its producer ranks are already mapped, instead of waking the transfer thread to do it; the thread
    # still plans every other load, polls the copy and notifies the producers. 0: every load goes to the thread.
    "LEAN_VLLM_KVX_INLINE_LOADS": lambda: os.getenv("LEAN_VLLM_KVX_INLINE_LOADS", "1").strip().lower()
    not in ("", "0", "false"),
    # SMs a per-layer save's copy may use while the prefill computes (0: every SM).
    "LEAN_VLLM_KVX_SAVE_SMS": lambda: int(os.getenv("LEAN_VLLM_KVX_SAVE_SMS", "16")),
}


def __getattr__(name: str):
    if name in environment_variables:
        return environment_variables[name]()
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def __dir__():
    return list(environment_variables)
