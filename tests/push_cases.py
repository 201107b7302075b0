"""The layer-by-layer push (save_kv_layer) scenarios, shared by the CPU (host transport) and GPU (kvx) tests.

A prefill instance holding a request's KV in blocks [7, 2, 9] pushes it into a decode instance's blocks [0, 5, 3]:
the same bytes the reference's pull lands (tests/test_nixl_connector.py:217-226), so the same golden results apply.
"""

from __future__ import annotations

from time import monotonic, sleep

from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVOutputAggregator, ReqToRecv
from lean_vllm_b200.kv_transfer.base import ReqToSave
from tests.connector_cases import wait_for

LOCAL, REMOTE = [0, 5, 3], [7, 2, 9]


def save_req(consumers) -> ReqToSave:
    kv = consumers[0].kv_transfer
    return ReqToSave(list(REMOTE), list(LOCAL), kv.engine_id, kv.kv_ip, kv.kv_port, len(consumers))


def pushed_recv(producers) -> ReqToRecv:
    kv = producers[0].kv_transfer
    return ReqToRecv(list(LOCAL), list(REMOTE), "p-1", kv.engine_id, kv.kv_ip, kv.kv_port, len(producers),
                     pushed=True)


def wait_ready(producer, request_id="p-1", timeout=10.0):
    deadline = monotonic() + timeout
    while monotonic() < deadline:
        with producer._lock:
            save = producer._saves.get(request_id)
            if save is not None and (save.ready or save.failed):
                return save.ready
        sleep(0.002)
    raise AssertionError("the push never connected")


def run_push(producers, consumers, layers_to_save, decode_first: bool = True):
    """Saves the listed layers on every producer rank, hands the request over, and returns the aggregated outputs
    of both sides."""
    if decode_first:
        for consumer in consumers:
            consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": pushed_recv(producers)}))
    for producer in producers:
        producer.start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save_req(consumers)}))
    for producer in producers:
        assert wait_ready(producer)
    for layer in layers_to_save:  # as the engine would, after each layer's store
        for producer in producers:
            producer.save_kv_layer(layer)
    for producer in producers:
        producer.wait_for_save()
        producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    if not decode_first:
        for consumer in consumers:
            consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": pushed_recv(producers)}))
    sent = KVOutputAggregator(len(producers)).aggregate([wait_for(p) for p in producers])
    recved = KVOutputAggregator(len(consumers)).aggregate([wait_for(c) for c in consumers])
    return sent, recved
