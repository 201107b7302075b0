"""Relayed latent loads (LEAN_VLLM_KVX_RELAY): a decode instance of several ranks loading MLA latents, which every
rank holds whole, pulls 1/tp of the blocks per rank from the prefill rank and the rest from its peer decode ranks --
the same bytes the reference's pull lands (each decode rank reading everything from the first producer rank,
nixl_connector.py:403), with the prefill GPU sending each byte once. CPU caches over the host transport."""

import numpy as np
import pytest

from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVOutputAggregator, cuda_ipc_connector
from tests.connector_cases import TP_PAIRS, Sides, full_cache, recv, wait_for
from tests.helpers import bits, full_of
from tests.host_transport import HostTransport

LOCAL, REMOTE = [0, 5, 3], [7, 2, 9]


@pytest.fixture(autouse=True)
def host_transport(monkeypatch):
    monkeypatch.setattr(cuda_ipc_connector, "make_transport", HostTransport)
    monkeypatch.setattr(HostTransport, "fail", None)
    monkeypatch.setenv("LEAN_VLLM_KVX_RELAY", "1")


@pytest.fixture
def sides():
    s = Sides("cpu")
    yield s
    s.close()


def load(producers, consumers):
    for producer in producers:
        producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    for consumer in consumers:
        consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, list(LOCAL),
                                                                              list(REMOTE))}))
    recved = KVOutputAggregator(len(consumers)).aggregate([wait_for(c) for c in consumers])
    sent = KVOutputAggregator(len(producers)).aggregate([wait_for(p) for p in producers])
    return sent, recved


@pytest.mark.parametrize("prefill_tp, decode_tp", [pair for pair in TP_PAIRS if pair[1] > 1])
def test_relayed_latents_land_what_the_reference_s_pull_lands(sides, golden, prefill_tp, decode_tp):
    _, arrays = golden
    producers = sides.make("kv_producer", prefill_tp, full_cache(0, True))
    consumers = sides.make("kv_consumer", decode_tp, full_cache(1, True), engine_id="decode")
    sent, recved = load(producers, consumers)
    assert recved.finished_recving == {"d-1"} and sent.finished_sending == {"p-1"}
    assert np.array_equal(bits(full_of([c.kv_caches[0] for c in consumers], True)),
                          arrays[f"small_lat_tp{prefill_tp}to{decode_tp}"])
    # Each decode rank's part from the prefill rank, then the others' parts from its peers: two launches (one if
    # its own part is empty); the byte count is the reference's, the whole payload on every rank.
    parts = [len(LOCAL) * (r + 1) // decode_tp - len(LOCAL) * r // decode_tp for r in range(decode_tp)]
    assert [len(c.transport.posts) for c in consumers] == [2 if n else 1 for n in parts]
    per_rank = len(LOCAL) * consumers[0].kv_caches[0][0, 0].numel() * 2
    assert recved.recv_stats["d-1"].num_bytes == per_rank * decode_tp


def test_keys_and_values_are_not_relayed(sides, golden):
    """Heads are split between decode ranks, so nothing is replicated: the plain pull, one launch per rank."""
    _, arrays = golden
    producers = sides.make("kv_producer", 2, full_cache(0, False))
    consumers = sides.make("kv_consumer", 4, full_cache(1, False), engine_id="decode")
    sent, recved = load(producers, consumers)
    assert recved.finished_recving == {"d-1"}
    assert [len(c.transport.posts) for c in consumers] == [1] * 4
    assert np.array_equal(bits(full_of([c.kv_caches[0] for c in consumers], False)), arrays["small_kv_tp2to4"])


def test_a_rank_whose_part_fails_fails_the_load_on_every_rank(sides):
    """Decode rank 1 cannot copy its part: it tells its peers, every rank reports the load failed (the instance
    prefills the prompt itself), and the producer's blocks are still released."""
    producers = sides.make("kv_producer", 1, full_cache(0, True))
    consumers = sides.make("kv_consumer", 2, full_cache(1, True), engine_id="decode")

    def refused(*args, **kwargs):
        raise RuntimeError("the transport refused the copy")

    consumers[1].transport.post = refused
    sent, recved = load(producers, consumers)
    assert recved.failed_recving == {"d-1"} and not recved.finished_recving
    assert sent.finished_sending == {"p-1"}


def test_a_peer_that_never_reports_its_part_fails_the_load_after_the_wait(sides, monkeypatch):
    monkeypatch.setattr(cuda_ipc_connector, "RELAY_WAIT", 0.3)
    producers = sides.make("kv_producer", 1, full_cache(0, True))
    consumers = sides.make("kv_consumer", 2, full_cache(1, True), engine_id="decode")
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, list(LOCAL), list(REMOTE))}))
    out = wait_for(consumers[0])  # rank 1 never gets the load
    assert out.failed_recving == {"d-1"}


def test_part_messages_nobody_reads_are_dropped_after_the_wait(sides, monkeypatch):
    """A peer's part for a load this rank never had stays only twice RELAY_WAIT."""
    monkeypatch.setattr(cuda_ipc_connector, "RELAY_WAIT", 0.1)
    from time import monotonic, sleep

    producers = sides.make("kv_producer", 1, full_cache(0, True))
    consumers = sides.make("kv_consumer", 2, full_cache(1, True), engine_id="decode")
    sent, recved = load(producers, consumers)
    assert recved.finished_recving == {"d-1"}
    worker = consumers[0]
    worker._handle(b"peer", {"op": "part", "request": "never-here", "rank": 1, "ok": True})
    assert "never-here" in worker._parts
    deadline = monotonic() + 5
    while "never-here" in worker._parts and monotonic() < deadline:
        sleep(0.02)
    assert "never-here" not in worker._parts and not worker._parts_seen


def test_a_peer_s_slot_that_comes_before_this_rank_starts_the_load_is_kept(sides, golden):
    """Decode rank 1 starts, posts its part and announces its ring slot well before rank 0 even gets the load: rank 0
    still finds the slot when it starts, copies rank 1's part, and both land the reference's result."""
    from time import sleep

    _, arrays = golden
    producers = sides.make("kv_producer", 1, full_cache(0, True))
    consumers = sides.make("kv_consumer", 2, full_cache(1, True), engine_id="decode")
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    consumers[1].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, list(LOCAL), list(REMOTE))}))
    sleep(0.3)  # rank 1's slot and landed messages are waiting at rank 0
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, list(LOCAL), list(REMOTE))}))
    recved = KVOutputAggregator(2).aggregate([wait_for(c) for c in consumers])
    assert recved.finished_recving == {"d-1"}
    assert np.array_equal(bits(full_of([c.kv_caches[0] for c in consumers], True)), arrays["small_lat_tp1to2"])
    assert KVOutputAggregator(1).aggregate([wait_for(p) for p in producers]).finished_sending == {"p-1"}


def test_a_peer_without_an_open_ring_is_copied_from_once_its_part_landed(sides, golden, monkeypatch):
    """A peer decode rank in this process on another GPU gets no ring (its event objects are not waited on across
    GPUs in one process): this rank copies its part once it said the part landed, and the load lands the reference's
    result all the same."""
    _, arrays = golden
    monkeypatch.setattr(HostTransport, "open_ring", lambda self, handles: [])
    producers = sides.make("kv_producer", 1, full_cache(0, True))
    consumers = sides.make("kv_consumer", 2, full_cache(1, True), engine_id="decode")
    sent, recved = load(producers, consumers)
    assert recved.finished_recving == {"d-1"} and sent.finished_sending == {"p-1"}
    assert np.array_equal(bits(full_of([c.kv_caches[0] for c in consumers], True)), arrays["small_lat_tp1to2"])
