"""Loads launched by the engine thread (LEAN_VLLM_KVX_INLINE_LOADS): once a decode rank has mapped its producer ranks
and none of its copies is in flight, start_load_kv launches the step's first load itself, and the transfer thread
only polls it and notifies the producers. The landed bytes are the reference's (the golden fixtures), and every
case the fast path does not cover goes to the transfer thread as before. CPU caches over the host transport."""

import threading
from time import monotonic, sleep

import numpy as np
import pytest

from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVOutputAggregator, cuda_ipc_connector
from tests.connector_cases import Sides, full_cache, recv, wait_for
from tests.helpers import bits, full_of
from tests.host_transport import HostTransport

LOCAL, REMOTE = [0, 5, 3], [7, 2, 9]


@pytest.fixture(autouse=True)
def host_transport(monkeypatch):
    monkeypatch.setattr(cuda_ipc_connector, "make_transport", HostTransport)
    monkeypatch.setattr(HostTransport, "fail", None)


@pytest.fixture
def sides():
    s = Sides("cpu")
    yield s
    s.close()


def threads_posting(consumers, monkeypatch) -> list:
    """Records, per post of the consumers' loads, the name of the thread that made it."""
    seen = []
    original = HostTransport.post

    def post(self, *args, **kwargs):
        if self in [c.transport for c in consumers]:
            seen.append(threading.current_thread().name)
        return original(self, *args, **kwargs)

    monkeypatch.setattr(HostTransport, "post", post)
    return seen


def warm(producers, consumers):
    """A first load that maps every producer rank (the handshake), after which the consumers' caches are put back
    as they were, so the next load's result can be compared with the fixtures."""
    before = [c.kv_caches[0].clone() for c in consumers]
    load(producers, consumers, "warm", [1], [4])
    for cache, old in zip([c.kv_caches[0] for c in consumers], before):
        cache.copy_(old)


def load(producers, consumers, request_id="p-1", local=LOCAL, remote=REMOTE, **overrides):
    for producer in producers:
        producer.start_load_kv(KVConnectorMetadata(reqs_to_send={request_id: list(remote)}))
    for consumer in consumers:
        req = recv(producers, list(local), list(remote), remote_request_id=request_id, **overrides)
        consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={f"d-{request_id}": req}))
    recved = KVOutputAggregator(len(consumers)).aggregate([wait_for(c) for c in consumers])
    sent = KVOutputAggregator(len(producers)).aggregate([wait_for(p) for p in producers])
    return sent, recved


@pytest.mark.parametrize("prefill_tp, decode_tp, mla", [(2, 1, False), (1, 2, False), (2, 4, False), (1, 2, True)])
def test_a_load_to_mapped_producers_launches_from_the_engine_thread(sides, golden, monkeypatch, prefill_tp,
                                                                    decode_tp, mla):
    _, arrays = golden
    producers = sides.make("kv_producer", prefill_tp, full_cache(0, mla))
    consumers = sides.make("kv_consumer", decode_tp, full_cache(1, mla), engine_id="decode")
    posting = threads_posting(consumers, monkeypatch)
    warm(producers, consumers)
    assert posting and all(name.startswith("kvx-ipc-") for name in posting)  # first contact: the thread
    posting.clear()
    sent, recved = load(producers, consumers)
    assert recved.finished_recving == {"d-p-1"} and sent.finished_sending == {"p-1"}
    assert posting == [threading.current_thread().name] * decode_tp
    name = f"small_{'lat' if mla else 'kv'}_tp{prefill_tp}to{decode_tp}"
    assert np.array_equal(bits(full_of([c.kv_caches[0] for c in consumers], mla)), arrays[name])
    # The reference's byte count, and every producer rank heard from its readers (it released the blocks).
    assert recved.recv_stats["d-p-1"].num_bytes > 0


def test_the_switch_off_sends_every_load_to_the_transfer_thread(sides, golden, monkeypatch):
    _, arrays = golden
    monkeypatch.setenv("LEAN_VLLM_KVX_INLINE_LOADS", "0")
    producers = sides.make("kv_producer", 2, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    posting = threads_posting(consumers, monkeypatch)
    warm(producers, consumers)
    posting.clear()
    sent, recved = load(producers, consumers)
    assert recved.finished_recving == {"d-p-1"} and sent.finished_sending == {"p-1"}
    assert posting and all(name.startswith("kvx-ipc-") for name in posting)
    assert np.array_equal(bits(full_of([c.kv_caches[0] for c in consumers], False)), arrays["small_kv_tp2to1"])


def test_a_bad_block_id_goes_to_the_thread_and_fails_only_its_load(sides, monkeypatch):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    posting = threads_posting(consumers, monkeypatch)
    warm(producers, consumers)
    posting.clear()
    before = consumers[0].kv_caches[0].clone()
    sent, recved = load(producers, consumers, remote=[7, 2, 40])  # block 40 lies past the producer's 12
    assert recved.failed_recving == {"d-p-1"} and not posting
    assert sent.finished_sending == {"p-1"}  # the failed reader still counts: the producer frees the blocks
    assert np.array_equal(bits(consumers[0].kv_caches[0]), bits(before))


def test_a_producer_under_another_engine_id_is_not_read_from_here(sides, monkeypatch):
    """The mapping names the engine that answered the handshake; a load naming another engine id goes to the
    thread, whose handshake sees the mismatch."""
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    posting = threads_posting(consumers, monkeypatch)
    warm(producers, consumers)
    posting.clear()
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    req = recv(producers, list(LOCAL), list(REMOTE), remote_engine_id="some-other-prefill")
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-p-1": req}))
    assert wait_for(consumers[0]).failed_recving == {"d-p-1"}  # the producer, another engine, never hears
    assert all(name.startswith("kvx-ipc-") for name in posting)


def test_behind_a_copy_in_flight_the_next_loads_go_to_the_thread(sides, monkeypatch):
    """The fast path is for latency: with a copy of this rank still in flight, a new step's loads are the thread's
    to plan, so they share launches."""
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    posting = threads_posting(consumers, monkeypatch)
    warm(producers, consumers)
    posting.clear()
    worker = consumers[0]
    with worker._lock:
        worker._launches_in_flight += 1  # as if a copy were still landing
    try:
        sent, recved = load(producers, consumers)
    finally:
        with worker._lock:
            worker._launches_in_flight -= 1
    assert recved.finished_recving == {"d-p-1"}
    assert posting and all(name.startswith("kvx-ipc-") for name in posting)


def test_the_in_flight_count_returns_to_zero(sides):
    producers = sides.make("kv_producer", 2, full_cache(0, False))
    consumers = sides.make("kv_consumer", 2, full_cache(1, False), engine_id="decode")
    warm(producers, consumers)
    load(producers, consumers)
    assert [c._launches_in_flight for c in consumers] == [0, 0]


def test_a_copy_launched_here_is_waited_for_at_shutdown(sides, monkeypatch):
    """shutdown right after start_load_kv: the thread takes the engine thread's launch before it closes the peer
    mappings, and waits for it."""
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    warm(producers, consumers)
    waited = []
    original = HostTransport.wait
    monkeypatch.setattr(HostTransport, "wait", lambda self, handle: (waited.append(handle), original(self, handle)))
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-p-1": recv(producers, list(LOCAL),
                                                                                list(REMOTE))}))
    consumers[0].shutdown()
    assert waited


def test_get_finished_reports_a_load_launched_here_without_the_transfer_thread(sides, golden, monkeypatch):
    """The engine thread's own query: with the transfer thread's polling switched off on the decode rank, a load
    launched by start_load_kv still comes back from get_finished once its copy has landed, with the reference's
    bytes in place, and the rank counts no copy in flight afterwards."""
    _, arrays = golden
    producers = sides.make("kv_producer", 2, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    warm(producers, consumers)
    worker = consumers[0]
    monkeypatch.setattr(worker, "_poll_loads", lambda notes: None)
    for producer in producers:
        producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    worker.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-p-1": recv(producers, list(LOCAL), list(REMOTE))}))
    out = wait_for(worker)
    assert out.finished_recving == {"d-p-1"} and not out.failed_recving
    assert out.recv_stats["d-p-1"].num_bytes > 0
    assert worker._launches_in_flight == 0
    assert np.array_equal(bits(full_of([worker.kv_caches[0]], False)), arrays["small_kv_tp2to1"])


def test_each_load_is_reported_once_whichever_thread_sees_it_land(sides):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    warm(producers, consumers)
    worker = consumers[0]
    seen: dict = {}
    for i in range(40):
        producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={f"p-{i}": list(REMOTE)}))
        worker.start_load_kv(KVConnectorMetadata(reqs_to_recv={
            f"d-{i}": recv(producers, list(LOCAL), list(REMOTE), remote_request_id=f"p-{i}")}))
        if i % 3 == 0:  # sometimes the thread gets there first
            sleep(0.01)
        out = worker.get_finished()
        for rid in out.finished_recving:
            seen[rid] = seen.get(rid, 0) + 1
        assert not out.failed_recving
    deadline = monotonic() + 10
    while len(seen) < 40 and monotonic() < deadline:
        for rid in worker.get_finished().finished_recving:
            seen[rid] = seen.get(rid, 0) + 1
        sleep(0.002)
    assert seen == {f"d-{i}": 1 for i in range(40)}
    left = {f"p-{i}" for i in range(40)}  # and every producer request was released by its reader's notification
    deadline = monotonic() + 10
    while left and monotonic() < deadline:
        left -= producers[0].get_finished().finished_sending
        sleep(0.002)
    assert not left
    assert worker._launches_in_flight == 0
