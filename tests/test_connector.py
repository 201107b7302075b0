"""CudaIpcConnector's worker halves on CPU caches over a host-memory transport: the reference connector's behaviour,
case by case (tests/test_nixl_connector.py), with the results checked against the golden fixtures recorded from the
reference connector itself."""

import socket
from time import monotonic, sleep

import numpy as np
import pytest
import torch

from lean_vllm_b200.kv_transfer import (
    KVConnectorMetadata,
    KVConnectorOutput,
    KVOutputAggregator,
    ReqToRecv,
    cuda_ipc_connector,
)
from lean_vllm_b200.kv_transfer.shares import Share, head_shares
from tests.connector_cases import (
    NUM_BLOCKS,
    TP_PAIRS,
    Sides,
    free_port,
    full_cache,
    rank_cache,
    recv,
    wait_for,
)
from tests.helpers import bits, full_of
from tests.host_transport import HostTransport


@pytest.fixture(autouse=True)
def host_transport(monkeypatch):
    monkeypatch.setattr(cuda_ipc_connector, "make_transport", HostTransport)
    monkeypatch.setattr(HostTransport, "fail", None)
    monkeypatch.setattr(HostTransport, "instances", [])


@pytest.fixture
def sides():
    s = Sides("cpu")
    yield s
    s.close()


def test_each_rank_s_shares_are_the_overlap_of_its_heads_with_each_producer_rank_s():
    assert head_shares(0, 1, 1, 8) == [Share(0, 0, 0, 8)]
    assert head_shares(3, 4, 2, 8) == [Share(1, 2, 0, 2)]
    assert head_shares(1, 2, 4, 8) == [Share(2, 0, 0, 2), Share(3, 0, 2, 2)]
    assert head_shares(1, 6, 4, 12) == [Share(0, 2, 0, 1), Share(1, 0, 1, 1)]


def test_shares_match_the_reference_on_every_split(golden):
    meta, _ = golden
    for rank, tp, rtp, heads, shares in meta["head_shares"]:
        assert head_shares(rank, tp, rtp, heads) == [Share(*s) for s in shares]


@pytest.mark.parametrize("mla", [False, True], ids=["kv", "latents"])
@pytest.mark.parametrize("prefill_tp, decode_tp", TP_PAIRS)
def test_each_decode_rank_gets_its_heads_whatever_the_two_sizes(sides, golden, prefill_tp, decode_tp, mla):
    _, arrays = golden
    prefill, decode = full_cache(0, mla), full_cache(1, mla)
    key = "lat" if mla else "kv"
    assert np.array_equal(bits(prefill), arrays[f"small_{key}_prefill"])  # the reference's inputs, bit for bit
    producers = sides.make("kv_producer", prefill_tp, prefill)
    consumers = sides.make("kv_consumer", decode_tp, decode, engine_id="decode")
    for producer in producers:
        producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [7, 2, 9]}))
    for consumer in consumers:
        consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0, 5, 3], [7, 2, 9])}))
    outputs = [wait_for(c) for c in consumers]
    assert KVOutputAggregator(decode_tp).aggregate(outputs).finished_recving == {"d-1"}
    got = full_of([c.kv_caches[0] for c in consumers], mla)
    assert np.array_equal(bits(got), arrays[f"small_{key}_tp{prefill_tp}to{decode_tp}"])
    assert KVOutputAggregator(prefill_tp).aggregate([wait_for(p) for p in producers]).finished_sending == {"p-1"}


def test_a_producer_rank_waits_for_every_decode_rank_that_reads_it(sides):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 2, full_cache(1, False), engine_id="decode")
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [4]}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4])}))
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    sleep(0.05)
    assert not producers[0].get_finished(), "freed while decode rank 1 has yet to read"
    consumers[1].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4])}))
    assert wait_for(consumers[1]).finished_recving == {"d-1"}
    assert wait_for(producers[0]) == KVConnectorOutput(finished_sending={"p-1"})


def test_a_copy_before_the_hand_over_frees_the_blocks_once_it_comes(sides):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4])}))
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    sleep(0.05)
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [4]}))
    assert producers[0].get_finished() == KVConnectorOutput(finished_sending={"p-1"})


def test_only_the_blocks_not_cached_here_are_copied(sides, golden):
    _, arrays = golden
    prefill, decode = full_cache(0, False), full_cache(1, False)
    producers = sides.make("kv_producer", 2, prefill)
    consumers = sides.make("kv_consumer", 1, decode, engine_id="decode")
    for producer in producers:
        producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [1, 2, 3]}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [8], [3])}))
    stats = wait_for(consumers[0]).recv_stats["d-1"]
    assert stats.num_bytes == 2 * 12 * 4 * 8 * 2  # one block of keys and values, bf16 (the reference's answer)
    assert np.array_equal(bits(consumers[0].kv_caches[0]), arrays["small_kv_prefix_hit"])


def test_a_full_prefix_hit_copies_nothing_but_still_frees_the_producer_s_blocks(sides):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    before = consumers[0].kv_caches[0].clone()
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [4]}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [], [])}))
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    assert wait_for(producers[0]).finished_sending == {"p-1"}
    assert torch.equal(consumers[0].kv_caches[0], before)


def test_an_absent_producer_fails_the_load(sides, monkeypatch):
    monkeypatch.setattr(cuda_ipc_connector, "HANDSHAKE_TIMEOUT", 0.2)
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    req = ReqToRecv([0], [4], "p-1", "prefill", "127.0.0.1", free_port())
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": req}))
    assert wait_for(consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})


@pytest.mark.parametrize(
    "overrides, message",
    [
        (dict(remote_engine_id="before-a-restart"), "is engine prefill, not before-a-restart"),
        (dict(remote_tp_size=2), "runs tp_size 1, not 2"),
        (dict(remote_block_ids=[NUM_BLOCKS]), "past the producer's"),
    ],
)
def test_a_producer_that_does_not_match_the_request_fails_the_load(sides, caplog, overrides, message):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4], **overrides)}))
    assert wait_for(consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})
    assert message in caplog.text


def test_a_producer_of_another_model_fails_the_load(sides, caplog):
    producers = sides.make("kv_producer", 1, full_cache(0, True))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4])}))
    assert wait_for(consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})
    assert "serve the same model, dtype and block size" in caplog.text


def test_a_producer_on_another_node_fails_the_load(sides, caplog):
    """CUDA IPC mappings only work within one node, so a producer elsewhere is refused at the handshake."""
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    producers[0].node = "another-node"
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4])}))
    assert wait_for(consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})
    assert "runs on another node" in caplog.text


def test_a_copy_refused_when_posted_fails_the_load_and_tells_the_producer(sides):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    HostTransport.fail = "posted"
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [4]}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4])}))
    assert wait_for(consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})
    assert wait_for(producers[0]) == KVConnectorOutput(finished_sending={"p-1"})


def test_a_copy_failing_in_flight_fails_the_load_and_leaves_the_blocks_to_expire(sides, monkeypatch):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    HostTransport.fail = "in flight"
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [4]}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4])}))
    assert wait_for(consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})
    sleep(0.05)
    assert not producers[0].get_finished()
    monkeypatch.setenv("LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT", "0")
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [4]}))  # handed over again, to expire now
    sleep(0.01)
    assert producers[0].get_finished() == KVConnectorOutput(finished_sending={"p-1"}, expired_sending={"p-1"})


def test_a_second_request_reuses_the_handshake(sides):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    for request_id, block in (("p-1", 4), ("p-2", 5)):
        producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={request_id: [block]}))
        req = recv(producers, [block], [block], remote_request_id=request_id)
        consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={request_id: req}))
        assert wait_for(consumers[0]).finished_recving == {request_id}
    assert len(consumers[0]._remotes) == 1 and consumers[0].transport.opened == 1


def test_a_restarted_producer_is_asked_afresh_and_the_old_mapping_closed(sides):
    first = sides.make("kv_producer", 1, full_cache(0, False), engine_id="prefill-a")
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(first, [0], [4])}))
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    first[0].shutdown()
    sleep(0.05)
    second = sides.make("kv_producer", 1, full_cache(2, False), port=first[0].kv_transfer.kv_port,
                        engine_id="prefill-b")
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-2": recv(second, [1], [4])}))
    deadline = monotonic() + 5
    while not consumers[0]._retired and monotonic() < deadline:
        sleep(0.002)
    # A copy queued before the swap may still read the old mapping: it stays open until the engine thread polls.
    sleep(0.05)
    transport = consumers[0].transport
    assert transport.opened == 2 and not transport.closed
    assert wait_for(consumers[0]).finished_recving == {"d-2"}
    while transport.opened != 1 and monotonic() < deadline:
        consumers[0].get_finished()
        sleep(0.002)
    assert transport.opened == 1 and not consumers[0]._retired
    (exported, posts_by_then), = transport.closed
    assert exported["spans"] == [list(span) for span in first[0].transport.spans]  # the first producer's
    assert transport.posts[posts_by_then - 4 : posts_by_then] == [(None, 0)] * 4  # a fence on every stream first
    assert torch.equal(consumers[0].kv_caches[0][:, 1], rank_cache(full_cache(2, False), 0, 1)[:, 4])


def test_a_replaced_mapping_the_engine_never_polled_past_closes_at_shutdown(sides):
    first = sides.make("kv_producer", 1, full_cache(0, False), engine_id="prefill-a")
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(first, [0], [4])}))
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    first[0].shutdown()
    sleep(0.05)
    second = sides.make("kv_producer", 1, full_cache(2, False), port=first[0].kv_transfer.kv_port,
                        engine_id="prefill-b")
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-2": recv(second, [1], [4])}))
    deadline = monotonic() + 5
    while not consumers[0]._retired and monotonic() < deadline:
        sleep(0.002)
    sleep(0.05)
    transport = consumers[0].transport
    assert transport.opened == 2  # no poll since the swap: still open
    consumers[0].shutdown()  # waits for the device (the host transport's drain), then closes every mapping
    assert transport.opened == 0 and len(transport.closed) == 2


@pytest.mark.parametrize("failure", ["posted", "in flight"])
def test_a_replaced_mapping_whose_fences_fail_stays_open(sides, failure):
    """If the transport cannot show that the streams ran past the swap, the old mapping is never closed: one kept
    open costs address space, one closed under a copy faults it."""
    first = sides.make("kv_producer", 1, full_cache(0, False), engine_id="prefill-a")
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(first, [0], [4])}))
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    first[0].shutdown()
    sleep(0.05)
    second = sides.make("kv_producer", 1, full_cache(2, False), port=first[0].kv_transfer.kv_port,
                        engine_id="prefill-b")
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-2": recv(second, [1], [4])}))
    deadline = monotonic() + 5
    while not consumers[0]._retired and monotonic() < deadline:
        sleep(0.002)
    sleep(0.05)  # the load's own post is made in the pass that swapped the mapping
    HostTransport.fail = failure
    while consumers[0]._retired and monotonic() < deadline:
        consumers[0].get_finished()
        sleep(0.002)
    assert not consumers[0]._retired
    assert consumers[0].transport.opened == 2 and not consumers[0].transport.closed


def test_malformed_messages_are_dropped_and_the_rank_keeps_serving(sides, caplog):
    """Garbage, and messages whose fields do not parse, reach a producer rank's socket; each is dropped with a
    warning, and the rank still answers handshakes and counts readers."""
    import json

    import zmq

    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    context = zmq.Context()
    sock = context.socket(zmq.DEALER)
    try:
        sock.connect(f"tcp://127.0.0.1:{producers[0].kv_transfer.kv_port}")
        for message in (b"not json", b"[1, 2]", {"op": "part", "request": "x", "rank": "one", "ok": True},
                        {"op": "saved", "request": "x", "rank": [0]}, {"op": "expect", "push_id": "p", "tp_size": 0},
                        {"op": "expect", "push_id": "p", "block_ids": ["a"]}, {"op": "notify", "message": "no-colon"}):
            sock.send(message if isinstance(message, bytes) else json.dumps(message).encode())
        sleep(0.1)
    finally:
        sock.close(linger=0)
        context.term()
    assert producers[0]._thread.is_alive()
    assert not producers[0]._expects
    assert "ignoring a malformed KV message" in caplog.text
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [4]}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4])}))
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    assert wait_for(producers[0]).finished_sending == {"p-1"}


def test_loads_that_finish_together_notify_their_producer_in_one_message(sides, monkeypatch):
    """Two loads started in one step share a launch and land together: the producer rank gets one message carrying
    both reader notifications (one socket send, not one per load) and frees both requests."""
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    sent = []
    send = consumers[0]._send
    monkeypatch.setattr(consumers[0], "_send", lambda key, message: (sent.append(message), send(key, message))[1])
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [4], "p-2": [5]}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={
        "d-1": recv(producers, [0], [4], remote_request_id="p-1"),
        "d-2": recv(producers, [1], [5], remote_request_id="p-2")}))
    done, deadline = set(), monotonic() + 10
    while done != {"d-1", "d-2"} and monotonic() < deadline:
        done |= consumers[0].get_finished().finished_recving
        sleep(0.002)
    assert done == {"d-1", "d-2"}
    freed, deadline = set(), monotonic() + 10
    while freed != {"p-1", "p-2"} and monotonic() < deadline:
        freed |= producers[0].get_finished().finished_sending
        sleep(0.002)
    assert freed == {"p-1", "p-2"}
    notes = [m for m in sent if m.get("op") == "notify"]
    assert len(notes) == 1 and sorted(notes[0]["messages"]) == ["p-1:1", "p-2:1"]


def test_an_unexpected_error_in_a_step_is_logged_once_and_the_thread_carries_on(sides, caplog):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    worker = consumers[0]

    def broken():
        raise ZeroDivisionError("planted in a test")

    worker._poll_waits = broken  # runs every pass of the transfer thread
    sleep(0.1)
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [4]}))
    worker.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4])}))
    assert wait_for(worker).finished_recving == {"d-1"}
    assert worker._thread.is_alive()
    assert caplog.text.count("hit an unexpected error in broken") == 1


def test_two_kv_both_instances_load_from_each_other_at_once(sides):
    """kv_both (the reference's default role): each instance holds a prefill the other loads, and both loads start
    together, so their handshakes cross -- each rank answers the other's while it waits for its own reply. Both
    loads land bit for bit and both held requests are freed."""
    a = sides.make("kv_both", 1, full_cache(0, False), engine_id="engine-a")
    b = sides.make("kv_both", 1, full_cache(1, False), engine_id="engine-b")
    before_a, before_b = a[0].kv_caches[0].clone(), b[0].kv_caches[0].clone()
    a[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"pa": [4]}))
    b[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"pb": [6]}))
    a[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"from-b": recv(b, [2], [6], remote_request_id="pb")}))
    b[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"from-a": recv(a, [3], [4], remote_request_id="pa")}))
    got_a, got_b, deadline = KVConnectorOutput(), KVConnectorOutput(), monotonic() + 10
    while monotonic() < deadline and not (got_a.finished_recving and got_a.finished_sending and
                                          got_b.finished_recving and got_b.finished_sending):
        for worker, got in ((a[0], got_a), (b[0], got_b)):
            out = worker.get_finished()
            got.finished_recving |= out.finished_recving
            got.finished_sending |= out.finished_sending
        sleep(0.002)
    assert got_a.finished_recving == {"from-b"} and got_a.finished_sending == {"pa"}
    assert got_b.finished_recving == {"from-a"} and got_b.finished_sending == {"pb"}
    assert torch.equal(a[0].kv_caches[0][:, 2], before_b[:, 6])
    assert torch.equal(b[0].kv_caches[0][:, 3], before_a[:, 4])


def test_a_taken_port_is_named(sides):
    with socket.socket() as taken:
        taken.bind(("127.0.0.1", 0))
        with pytest.raises(RuntimeError, match="pick another kv_port"):
            sides.make("kv_producer", 1, full_cache(0, False), port=taken.getsockname()[1])


def test_a_consumer_serves_nothing(sides):
    assert sides.make("kv_consumer", 1, full_cache(1, False))[0]._server is None


def test_an_nhd_cache_is_refused():
    from lean_vllm_b200.kv_transfer import KVTransferConfig
    from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker
    from tests.connector_cases import WorkerConfig

    with pytest.raises(AssertionError, match="needs HND caches"):
        CudaIpcConnectorWorker(WorkerConfig(KVTransferConfig(), kv_cache_layout="NHD"), 0)


def test_many_requests_in_one_step_each_finish(sides):
    prefill, decode = full_cache(0, False), full_cache(1, False)
    producers = sides.make("kv_producer", 2, prefill)
    consumers = sides.make("kv_consumer", 2, decode, engine_id="decode")
    pairs = {f"r{i}": ([i], [NUM_BLOCKS - 1 - i]) for i in range(6)}
    for producer in producers:
        producer.start_load_kv(KVConnectorMetadata(reqs_to_send={f"r{i}": [NUM_BLOCKS - 1 - i] for i in range(6)}))
    for consumer in consumers:
        consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={
            rid: recv(producers, local, remote, remote_request_id=rid) for rid, (local, remote) in pairs.items()}))
    done = set()
    aggregator = KVOutputAggregator(2)
    for _ in range(200):
        done |= aggregator.aggregate([c.get_finished() for c in consumers]).finished_recving
        if len(done) == 6:
            break
        sleep(0.005)
    assert done == set(pairs)
    expected = decode.clone()
    for local, remote in pairs.values():
        expected[:, local] = prefill[:, remote]
    assert torch.equal(full_of([c.kv_caches[0] for c in consumers], False), expected)
