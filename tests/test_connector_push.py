"""The per-layer save (push) on CPU caches over the host transport: protocol, catch-up of layers no hook pushed,
failures, and bit-exact results against the reference's golden pulls."""

from time import monotonic, sleep

import numpy as np
import pytest
import torch

from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVConnectorOutput, cuda_ipc_connector
from tests.connector_cases import BLOCK, TP_PAIRS, Sides, full_cache, wait_for
from tests.helpers import bits, full_of
from tests.host_transport import HostTransport
from tests.push_cases import LOCAL, REMOTE, pushed_recv, run_push, save_req, wait_ready


@pytest.fixture(autouse=True)
def host_transport(monkeypatch):
    monkeypatch.setattr(cuda_ipc_connector, "make_transport", HostTransport)
    monkeypatch.setattr(HostTransport, "fail", None)


@pytest.fixture
def sides():
    s = Sides("cpu")
    yield s
    s.close()


@pytest.mark.parametrize("mla", [False, True], ids=["kv", "latents"])
@pytest.mark.parametrize("prefill_tp, decode_tp", TP_PAIRS)
def test_a_pushed_request_lands_what_the_reference_s_pull_lands(sides, golden, prefill_tp, decode_tp, mla):
    _, arrays = golden
    producers = sides.make("kv_producer", prefill_tp, full_cache(0, mla))
    consumers = sides.make("kv_consumer", decode_tp, full_cache(1, mla), engine_id="decode", accept_push=True)
    sent, recved = run_push(producers, consumers, layers_to_save=[0])
    assert sent.finished_sending == {"p-1"} and recved.finished_recving == {"d-1"}
    key = "lat" if mla else "kv"
    got = full_of([c.kv_caches[0] for c in consumers], mla)
    assert np.array_equal(bits(got), arrays[f"small_{key}_tp{prefill_tp}to{decode_tp}"])
    # The decode side counts its own heads' bytes, as a pull would.
    per_rank = 2 * 3 * (12 // decode_tp) * 4 * 8 * 2 if not mla else 3 * 4 * 6 * 2
    assert all(stats.num_bytes == per_rank * decode_tp for stats in recved.recv_stats.values())


def test_each_layer_is_pushed_by_its_own_hook_and_the_rest_at_hand_over(sides):
    layers = [full_cache(10 + i, False) for i in range(3)]
    producers = sides.make("kv_producer", 1, layers)
    consumers = sides.make("kv_consumer", 2, [full_cache(20 + i, False) for i in range(3)], engine_id="decode",
                           accept_push=True)
    sent, recved = run_push(producers, consumers, layers_to_save=[0, 1])  # layer 2's hook never ran
    assert sent.finished_sending == {"p-1"} and recved.finished_recving == {"d-1"}
    posts = producers[0].transport.posts
    assert [layer for layer, _ in posts] == [(0, 2), (2, 2), (4, 2)]  # one launch per layer: K and V regions
    assert all(jobs == 2 for _, jobs in posts)  # one job per decode rank
    for layer in range(3):
        got = full_of([c.kv_caches[layer] for c in consumers], False)
        want = full_cache(20 + layer, False)
        want[:, LOCAL] = layers[layer][:, REMOTE]
        assert torch.equal(got, want), layer


def test_an_engine_without_layer_hooks_pushes_everything_in_one_launch_at_hand_over(sides):
    layers = [full_cache(30 + i, False) for i in range(2)]
    producers = sides.make("kv_producer", 2, layers)
    consumers = sides.make("kv_consumer", 1, [full_cache(40 + i, False) for i in range(2)], engine_id="decode",
                           accept_push=True)
    sent, recved = run_push(producers, consumers, layers_to_save=[])
    assert sent.finished_sending == {"p-1"} and recved.finished_recving == {"d-1"}
    assert all([layer for layer, _ in p.transport.posts] == [None] for p in producers)
    got = consumers[0].kv_caches
    for layer in range(2):
        want = full_cache(40 + layer, False)
        want[:, LOCAL] = layers[layer][:, REMOTE]
        assert torch.equal(got[layer], want)


def test_the_landing_word_may_come_before_the_decode_side_waits(sides, golden):
    _, arrays = golden
    producers = sides.make("kv_producer", 2, full_cache(0, False))
    consumers = sides.make("kv_consumer", 4, full_cache(1, False), engine_id="decode", accept_push=True)
    sent, recved = run_push(producers, consumers, layers_to_save=[0], decode_first=False)
    assert recved.finished_recving == {"d-1"}
    assert np.array_equal(bits(full_of([c.kv_caches[0] for c in consumers], False)), arrays["small_kv_tp2to4"])


def test_a_decode_instance_that_does_not_answer_fails_the_push_and_its_wait(sides, monkeypatch):
    monkeypatch.setattr(cuda_ipc_connector, "HANDSHAKE_TIMEOUT", 0.2)
    monkeypatch.setenv("LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT", "0.5")
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")  # does not accept pushes
    before = consumers[0].kv_caches[0].clone()
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": pushed_recv(producers)}))
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save_req(consumers)}))
    producers[0].save_kv_layer(0)
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    assert wait_for(producers[0]) == KVConnectorOutput(finished_sending={"p-1"})  # the blocks are freed
    assert wait_for(consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})  # and the decode side prefills
    assert torch.equal(consumers[0].kv_caches[0], before)


def test_a_save_into_a_decode_instance_that_restarted_fails_and_its_old_mapping_outlives_what_was_queued(sides):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    first = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode-a", accept_push=True)
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save_req(first)},
                                                   save_progress={"p-1": len(REMOTE) * BLOCK}))
    assert wait_ready(producers[0])
    producers[0].save_kv_layer(0)  # queued into decode-a's blocks
    first[0].shutdown()
    sleep(0.05)
    second = sides.make("kv_consumer", 1, full_cache(2, False), port=first[0].kv_transfer.kv_port,
                        engine_id="decode-b", accept_push=True)
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_save={"p-2": save_req(second)}))
    assert wait_ready(producers[0], "p-2")
    assert producers[0]._saves["p-1"].failed  # its decode instance is gone: nothing more is pushed into it
    transport = producers[0].transport
    sleep(0.05)
    assert transport.opened == 2 and not transport.closed  # the engine thread has not polled since the swap
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    assert wait_for(producers[0]).finished_sending == {"p-1"}  # its blocks are freed
    deadline = monotonic() + 5
    while transport.opened != 1 and monotonic() < deadline:
        producers[0].get_finished()
        sleep(0.002)
    assert transport.opened == 1 and len(transport.closed) == 1
    while "p-1" not in second[0]._saved and monotonic() < deadline:
        sleep(0.002)
    assert second[0]._saved["p-1"] == {0: False}  # the instance now at that port hears "not ok", and ignores it


def test_a_landing_word_no_wait_takes_is_dropped_at_the_timeout(sides, monkeypatch):
    import json

    import zmq

    monkeypatch.setenv("LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT", "0.3")
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode", accept_push=True)
    context = zmq.Context()
    sock = context.socket(zmq.DEALER)
    try:
        sock.connect(f"tcp://127.0.0.1:{consumers[0].kv_transfer.kv_port}")
        sock.send(json.dumps({"op": "saved", "request": "aborted", "rank": 0, "ok": True}).encode())
        deadline = monotonic() + 5
        while "aborted" not in consumers[0]._saved and monotonic() < deadline:
            sleep(0.002)
        assert consumers[0]._saved["aborted"] == {0: True}  # kept: its wait may come later
        while "aborted" in consumers[0]._saved and monotonic() < deadline:
            sleep(0.01)
        assert "aborted" not in consumers[0]._saved and not consumers[0]._saved_seen
    finally:
        sock.close(linger=0)
        context.term()


def test_a_push_refused_when_posted_tells_the_decode_side_it_failed(sides):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode", accept_push=True)
    HostTransport.fail = "posted"
    sent, recved = run_push(producers, consumers, layers_to_save=[0])
    assert sent.finished_sending == {"p-1"}
    assert recved.failed_recving == {"d-1"}


def test_a_push_failing_in_flight_tells_the_decode_side_it_failed(sides):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode", accept_push=True)
    HostTransport.fail = "in flight"
    sent, recved = run_push(producers, consumers, layers_to_save=[0])
    assert sent.finished_sending == {"p-1"}
    assert recved.failed_recving == {"d-1"}


def test_a_save_that_is_never_handed_over_expires(sides, monkeypatch):
    monkeypatch.setenv("LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT", "0.3")
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode", accept_push=True)
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": pushed_recv(producers)}))
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save_req(consumers)}))
    producers[0].save_kv_layer(0)  # the prefill is then aborted: no hand-over
    assert wait_for(consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})
    deadline = monotonic() + 2.0  # the producer checks its deadlines at least every IDLE_WAIT
    while producers[0]._saves and monotonic() < deadline:
        sleep(0.005)
    assert not producers[0]._saves


def test_hooks_without_saves_launch_nothing(sides):
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    producers[0].save_kv_layer(0)
    producers[0].wait_for_save()
    assert producers[0].transport.posts == []


def test_a_consumer_that_accepts_pushes_serves_handshakes(sides):
    assert sides.make("kv_consumer", 1, full_cache(1, False), accept_push=True)[0]._server is not None


def test_a_chunked_prefill_pushes_what_each_chunk_fills_and_the_partial_block_again(sides):
    """A prompt prefilled in three chunks (ending mid-block): each chunk's per-layer push copies the blocks that
    chunk filled from the first one not yet final -- the partly filled block goes again with the next chunk -- and
    the decode blocks end up equal to the prefill's final blocks, with nothing left for hand-over."""
    from lean_vllm_b200.kv_transfer.base import ReqToSave
    from tests.connector_cases import BLOCK

    layers = [full_cache(50 + i, False) for i in range(2)]
    producers = sides.make("kv_producer", 1, [t.clone() for t in layers])
    consumers = sides.make("kv_consumer", 1, [full_cache(60 + i, False) for i in range(2)], engine_id="decode",
                           accept_push=True)
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": pushed_recv(producers)}))
    kv = consumers[0].kv_transfer
    tokens = 3 * BLOCK - 1  # the last block holds one token less
    save = ReqToSave(list(REMOTE), list(LOCAL), kv.engine_id, kv.kv_ip, kv.kv_port, 1, num_tokens=tokens)
    producer = producers[0]
    chunks = [(0, BLOCK + 1), (BLOCK + 1, 2 * BLOCK + 1), (2 * BLOCK + 1, tokens)]  # each ends inside a block
    for step, (begin, end) in enumerate(chunks):
        meta = KVConnectorMetadata(reqs_to_save={"p-1": save} if step == 0 else {}, save_progress={"p-1": end})
        producer.start_load_kv(meta)
        if step == 0:
            from tests.push_cases import wait_ready

            assert wait_ready(producer)
        for layer, cache in enumerate(producer.kv_caches):
            # The chunk's rows land in the prefill's blocks (new values), then the layer's hook runs.
            for position in range(begin, end):
                block, offset = REMOTE[position // BLOCK], position % BLOCK
                cache[:, block, :, offset] = float(100 * layer + position)
            producer.save_kv_layer(layer)
    posts = [p for p in producer.transport.posts]
    producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    assert wait_for(producer).finished_sending == {"p-1"}
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    assert producer.transport.posts == posts  # every layer's blocks were final after the last chunk: no catch-up
    assert len(posts) == 3 * 2  # one per chunk per layer
    for layer in range(2):
        got, have = consumers[0].kv_caches[layer], producer.kv_caches[layer]
        for i, (d, s) in enumerate(zip(LOCAL, REMOTE)):
            rows = BLOCK if i < 2 else BLOCK - 1
            assert torch.equal(got[:, d, :, :rows], have[:, s, :, :rows]), (layer, i)


def test_without_progress_a_layer_hook_pushes_nothing_and_hand_over_pushes_everything(sides):
    """Metadata that never says how far the prefill got (an engine whose scheduler half does not report it): the
    per-layer hooks cannot know which blocks are final, so the whole request goes at hand-over, in one launch."""
    producers = sides.make("kv_producer", 1, [full_cache(70 + i, False) for i in range(2)])
    consumers = sides.make("kv_consumer", 1, [full_cache(80 + i, False) for i in range(2)], engine_id="decode",
                           accept_push=True)
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": pushed_recv(producers)}))
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save_req(consumers)}))
    from tests.push_cases import wait_ready

    assert wait_ready(producers[0])
    for layer in range(2):
        producers[0].save_kv_layer(layer)
    assert producers[0].transport.posts == []
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    assert [layer for layer, _ in producers[0].transport.posts] == [None]
    for layer in range(2):
        assert torch.equal(consumers[0].kv_caches[layer][:, LOCAL], producers[0].kv_caches[layer][:, REMOTE])


def test_a_layer_whose_last_chunk_was_not_hooked_is_finished_at_hand_over(sides):
    """Layer 1's hook did not run for the second chunk: hand-over pushes that layer's blocks from the first one
    not yet final; layer 0, complete, is not copied again."""
    from lean_vllm_b200.kv_transfer.base import ReqToSave
    from tests.connector_cases import BLOCK
    from tests.push_cases import wait_ready

    producers = sides.make("kv_producer", 1, [full_cache(90 + i, False) for i in range(2)])
    consumers = sides.make("kv_consumer", 1, [full_cache(95 + i, False) for i in range(2)], engine_id="decode",
                           accept_push=True)
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": pushed_recv(producers)}))
    kv = consumers[0].kv_transfer
    producer = producers[0]
    save = ReqToSave(list(REMOTE), list(LOCAL), kv.engine_id, kv.kv_ip, kv.kv_port, 1)
    producer.start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save}, save_progress={"p-1": BLOCK + 3}))
    assert wait_ready(producer)
    producer.save_kv_layer(0)
    producer.save_kv_layer(1)
    producer.start_load_kv(KVConnectorMetadata(save_progress={"p-1": 3 * BLOCK}))
    producer.save_kv_layer(0)  # layer 1's hook never runs for this chunk
    producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    layer_posts = [layer for layer, _ in producer.transport.posts]
    assert layer_posts == [(0, 2), (2, 2), (0, 2), (2, 2)]  # 2 hooks, 1 hook, then layer 1 at hand-over
    for layer in range(2):
        assert torch.equal(consumers[0].kv_caches[layer][:, LOCAL], producer.kv_caches[layer][:, REMOTE])
