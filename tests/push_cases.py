"""The layer-by-layer push (save_kv_layer) scenarios, shared by the CPU (host transport) and GPU (kvx) tests.

A prefill instance holding a request's KV in blocks [7, 2, 9] pushes it into a decode instance's blocks [0, 5, 3]:
the same bytes the reference's pull lands (tests/test_nixl_connector.py:217-226), so the same golden results apply.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from time import monotonic, sleep

from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVOutputAggregator, KVTransferConfig, ReqToRecv
from lean_vllm_b200.kv_transfer.base import ReqToSave
from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorScheduler
from tests.connector_cases import BLOCK, full_cache, wait_for

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
    for producer in producers:  # the whole prompt is computed in this step
        producer.start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save_req(consumers)},
                                                   save_progress={"p-1": len(REMOTE) * BLOCK}))
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


@dataclass
class Seq:
    """The Sequence fields the scheduler half reads."""

    request_id: str
    num_prompt_tokens: int
    block_table: list
    kv_transfer_params: dict
    num_cached_tokens: int = 0
    finish_reason: str | None = None
    num_scheduled_tokens: int = 0


@dataclass
class SchedConfig:
    kv_transfer: KVTransferConfig
    tensor_parallel_size: int = 1
    kvcache_block_size: int = BLOCK


@dataclass
class Flow:
    producers: list
    consumers: list
    prefill_half: CudaIpcConnectorScheduler
    decode_half: CudaIpcConnectorScheduler
    outputs: dict = field(default_factory=dict)

    def decode_admits(self, push_id="push-1", blocks=(0, 5, 3), cached=0):
        kv = self.producers[0].kv_transfer
        seq = Seq("d-1", len(blocks) * BLOCK, list(blocks), {
            "do_remote_prefill": True, "kv_push": True, "remote_request_id": push_id, "remote_engine_id": "",
            "remote_host": kv.kv_ip, "remote_port": kv.kv_port, "tp_size": len(self.producers),
            "remote_block_ids": []}, num_cached_tokens=cached * BLOCK)
        assert self.decode_half.get_num_new_matched_tokens(seq, seq.num_cached_tokens) == (
            seq.num_prompt_tokens - seq.num_cached_tokens, True)
        self.decode_half.update_state_after_alloc(seq, seq.num_prompt_tokens)
        meta = self.decode_half.build_connector_meta()
        for c in self.consumers:
            c.start_load_kv(meta)

    def prefill_runs(self, push_id="push-1", blocks=(7, 2, 9), layers=(0,)):
        seq = Seq("p-1", len(blocks) * BLOCK, list(blocks), {"do_remote_decode": True, "kv_push_id": push_id})
        assert self.prefill_half.get_num_new_matched_tokens(seq, 0) == (0, False)
        seq.num_scheduled_tokens = seq.num_prompt_tokens  # the engine schedules the whole prompt in this step
        meta = self.prefill_half.build_connector_meta()
        assert "p-1" in meta.reqs_to_save and meta.save_progress == {"p-1": seq.num_prompt_tokens}
        for p in self.producers:
            p.start_load_kv(meta)
        sleep(0.05)
        for layer in layers:
            for p in self.producers:
                p.save_kv_layer(layer)
        seq.finish_reason = "length"
        hold, params = self.prefill_half.request_finished(seq)
        assert hold and params["do_remote_prefill"]
        meta = self.prefill_half.build_connector_meta()
        for p in self.producers:
            p.start_load_kv(meta)

    def results(self):
        sent = KVOutputAggregator(len(self.producers)).aggregate([wait_for(p) for p in self.producers])
        recved = KVOutputAggregator(len(self.consumers)).aggregate([wait_for(c) for c in self.consumers])
        return sent, recved


def make_flow(sides, prefill_tp, decode_tp, mla=False) -> Flow:
    producers = sides.make("kv_producer", prefill_tp, full_cache(0, mla), engine_id="prefill")
    consumers = sides.make("kv_consumer", decode_tp, full_cache(1, mla), engine_id="decode", accept_push=True)
    p_half = CudaIpcConnectorScheduler(SchedConfig(producers[0].kv_transfer, prefill_tp))
    d_half = CudaIpcConnectorScheduler(SchedConfig(consumers[0].kv_transfer, decode_tp))
    return Flow(producers, consumers, p_half, d_half)
