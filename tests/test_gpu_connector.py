"""CudaIpcConnector on CUDA devices with the kvx transport: the reference connector's cases bit for bit against its
golden results, in one process on one GPU (producer ranks used by pointer), and across processes and GPUs over real
CUDA IPC mappings when the box has two or more GPUs."""

import multiprocessing as mp
from time import monotonic, sleep

import numpy as np
import pytest
import torch

from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVConnectorOutput, KVOutputAggregator, KVTransferConfig
from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker
from tests.conftest import gpu_count
from tests.connector_cases import (
    NUM_BLOCKS,
    TP_PAIRS,
    Sides,
    WorkerConfig,
    free_port,
    full_cache,
    rank_cache,
    recv,
    wait_for,
)
from tests.helpers import bits, full_of

pytestmark = pytest.mark.gpu


@pytest.fixture
def sides():
    s = Sides("cuda")
    yield s
    s.close()


@pytest.mark.parametrize("mla", [False, True], ids=["kv", "latents"])
@pytest.mark.parametrize("prefill_tp, decode_tp", TP_PAIRS)
def test_each_decode_rank_gets_its_heads_on_the_gpu(sides, golden, prefill_tp, decode_tp, mla):
    _, arrays = golden
    prefill, decode = full_cache(0, mla), full_cache(1, mla)
    producers = sides.make("kv_producer", prefill_tp, prefill)
    consumers = sides.make("kv_consumer", decode_tp, decode, engine_id="decode")
    for producer in producers:
        producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [7, 2, 9]}))
    for consumer in consumers:
        consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0, 5, 3], [7, 2, 9])}))
    outputs = [wait_for(c) for c in consumers]
    assert KVOutputAggregator(decode_tp).aggregate(outputs).finished_recving == {"d-1"}
    got = full_of([c.kv_caches[0].cpu() for c in consumers], mla)
    key = "lat" if mla else "kv"
    assert np.array_equal(bits(got), arrays[f"small_{key}_tp{prefill_tp}to{decode_tp}"])
    assert KVOutputAggregator(prefill_tp).aggregate([wait_for(p) for p in producers]).finished_sending == {"p-1"}


def test_the_byte_count_and_a_prefix_hit_on_the_gpu(sides, golden):
    _, arrays = golden
    producers = sides.make("kv_producer", 2, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    for producer in producers:
        producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [1, 2, 3]}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [8], [3])}))
    stats = wait_for(consumers[0]).recv_stats["d-1"]
    assert stats.num_bytes == 2 * 12 * 4 * 8 * 2
    assert np.array_equal(bits(consumers[0].kv_caches[0].cpu()), arrays["small_kv_prefix_hit"])


def test_a_block_id_past_the_producer_s_fails_without_a_launch(sides, caplog):
    from lean_vllm_b200.kv_transfer import transport

    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    before = transport.launch_count()
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [NUM_BLOCKS])}))
    assert wait_for(consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})
    assert transport.launch_count() == before
    assert "past the producer's" in caplog.text


def test_the_load_waits_on_the_gpu_for_the_step_that_still_writes_its_blocks(sides):
    """No host synchronisation: the copy waits on its stream for the event recorded at start_load_kv."""
    prefill, decode = full_cache(0, False), full_cache(1, False)
    producers = sides.make("kv_producer", 1, prefill)
    consumers = sides.make("kv_consumer", 1, decode, engine_id="decode")
    cache = consumers[0].kv_caches[0]
    torch.cuda._sleep(50_000_000)  # a step still in flight on the engine's stream ...
    cache[:, 0].fill_(3.0)  # ... that writes the block the load is about to fill
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0], [4])}))
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    assert torch.equal(cache[:, 0].cpu(), prefill[:, 4])


@pytest.mark.parametrize("decode_tp", [2, 4])
def test_relayed_latents_land_what_the_reference_s_pull_lands_on_the_gpu(sides, golden, monkeypatch, decode_tp):
    """LEAN_VLLM_KVX_RELAY on one GPU: each decode rank pulls its part of the latent pages from the producer, marks
    that launch in its ring of events and tells its peers at once; each peer's copy of the part waits on the mark on
    the GPU. Two loads in a row (the second reuses the ring) land the reference's result bit for bit."""
    monkeypatch.setenv("LEAN_VLLM_KVX_RELAY", "1")
    _, arrays = golden
    producers = sides.make("kv_producer", 1, full_cache(0, True))
    consumers = sides.make("kv_consumer", decode_tp, full_cache(1, True), engine_id="decode")
    for tag in ("1", "2"):
        for producer in producers:
            producer.start_load_kv(KVConnectorMetadata(reqs_to_send={f"p-{tag}": [7, 2, 9]}))
        for consumer in consumers:
            consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={f"d-{tag}": recv(
                producers, [0, 5, 3], [7, 2, 9], remote_request_id=f"p-{tag}")}))
        outputs = [wait_for(c) for c in consumers]
        assert KVOutputAggregator(decode_tp).aggregate(outputs).finished_recving == {f"d-{tag}"}
        for consumer in consumers:  # latents are whole on every decode rank
            assert np.array_equal(bits(consumer.kv_caches[0].cpu()), arrays["small_lat_tp1to2"])
        assert KVOutputAggregator(1).aggregate([wait_for(p) for p in producers]).finished_sending == {f"p-{tag}"}


def test_a_copy_that_gave_up_fails_its_load_alone_and_the_next_load_lands(sides, golden):
    """The first load's launch is made to look stuck: the bounded-wait self-test writes "gave up" (1) into that
    launch's own status word, as a copy whose bytes did not all land would. That load fails (the engine prefills
    it) and the producer's blocks expire rather than be freed under a possible late write; the next load on the
    same device, posted after it with nothing cleared in between, lands bit for bit."""
    from lean_vllm_b200.kv_transfer import transport

    _, arrays = golden
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
    kvx = consumers[0].transport
    real_post, real_done, stuck, flagged = kvx.post, kvx.done, [], []

    def post(tables, jobs, ready, **kw):
        xfer = real_post(tables, jobs, ready, **kw)
        if not stuck:
            stuck.append(xfer)
        return xfer

    def done(xfer):
        # Before the host first reads the first launch's word, the self-test writes "gave up" into it (on a stream
        # of its own, waited for here), standing in for that launch's copy.
        if stuck and xfer is stuck[0] and not flagged:
            side = torch.cuda.Stream()
            transport.wait_selftest(2_000, code=1, stream=side.cuda_stream, status=xfer.status_address())
            side.synchronize()
            flagged.append(True)
        return real_done(xfer)

    kvx.post, kvx.done = post, done
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [7, 2, 9]}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, [0, 5, 3], [7, 2, 9])}))
    assert wait_for(consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})
    assert producers[0].get_finished().finished_sending == set()  # no reader notified: expiry frees them
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-2": [7, 2, 9]}))
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={
        "d-2": recv(producers, [0, 5, 3], [7, 2, 9], remote_request_id="p-2")}))
    out = wait_for(consumers[0])
    assert out.finished_recving == {"d-2"} and not out.failed_recving
    assert np.array_equal(bits(consumers[0].kv_caches[0].cpu()), arrays["small_kv_tp1to1"])
    assert wait_for(producers[0]).finished_sending == {"p-2"}
    transport.device_error()  # the diagnostic word saw the stand-in; leave it clear for the tests after this one


def _producer(conn, device: int, kv_port: int, tp_size: int, rank: int, mla: bool):
    torch.cuda.set_device(device)
    kv = KVTransferConfig(kv_connector="CudaIpcConnector", kv_role="kv_producer", kv_port=kv_port,
                          engine_id="engine")
    worker = CudaIpcConnectorWorker(WorkerConfig(kv, tensor_parallel_size=tp_size), rank)
    worker.register_kv_caches([rank_cache(full_cache(0, mla), rank, tp_size).cuda()])
    worker.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": [7, 2, 9]}))
    conn.send("ready")
    deadline = monotonic() + 120
    while monotonic() < deadline and not worker.get_finished().finished_sending:
        sleep(0.01)
    conn.send("sent")
    worker.shutdown()


CROSS = [(1, 1, False), (1, 1, True), (2, 1, False), (1, 2, False), (1, 2, True), (2, 2, False), (2, 4, False)]


@pytest.mark.multigpu
@pytest.mark.parametrize("prefill_tp, decode_tp, mla", CROSS)
def test_a_load_between_processes_on_different_gpus(golden, prefill_tp, decode_tp, mla):
    """Producer ranks in spawned processes on their own GPUs, decode ranks in this process on the next GPUs: the
    copies run over real CUDA IPC mappings and NVLink (the reference's two-GPU read, tests/test_kv_transfer.py:58)."""
    if gpu_count() < prefill_tp + decode_tp:
        pytest.skip(f"needs {prefill_tp + decode_tp} GPUs")
    _, arrays = golden
    kv_port = free_port()
    ctx = mp.get_context("spawn")
    procs, conns = [], []
    for rank in range(prefill_tp):
        parent, child = ctx.Pipe()
        proc = ctx.Process(target=_producer, args=(child, rank, kv_port, prefill_tp, rank, mla))
        proc.start()
        procs.append(proc)
        conns.append(parent)
    consumers = []
    try:
        for conn in conns:
            assert conn.poll(120) and conn.recv() == "ready"
        for rank in range(decode_tp):
            device = prefill_tp + rank
            torch.cuda.set_device(device)
            kv = KVTransferConfig(kv_connector="CudaIpcConnector", kv_role="kv_consumer", engine_id="decode")
            worker = CudaIpcConnectorWorker(WorkerConfig(kv, tensor_parallel_size=decode_tp), rank)
            worker.register_kv_caches([rank_cache(full_cache(1, mla), rank, decode_tp).to(device)])
            consumers.append(worker)
        req_fields = dict(remote_request_id="p-1", remote_engine_id="engine", remote_host="127.0.0.1",
                          remote_port=kv_port, remote_tp_size=prefill_tp)
        from lean_vllm_b200.kv_transfer import ReqToRecv

        for worker in consumers:
            torch.cuda.set_device(worker.kv_caches[0].device)
            worker.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": ReqToRecv([0, 5, 3], [7, 2, 9],
                                                                                      **req_fields)}))
        outputs = [wait_for(w, timeout=60) for w in consumers]
        assert KVOutputAggregator(decode_tp).aggregate(outputs).finished_recving == {"d-1"}
        got = full_of([w.kv_caches[0].cpu() for w in consumers], mla)
        key = "lat" if mla else "kv"
        assert np.array_equal(bits(got), arrays[f"small_{key}_tp{prefill_tp}to{decode_tp}"])
        for conn in conns:  # every producer rank frees its blocks once all its readers told it
            assert conn.poll(60) and conn.recv() == "sent"
    finally:
        for worker in consumers:
            worker.shutdown()
        for proc in procs:
            proc.join(timeout=60)
            if proc.is_alive():
                proc.kill()


@pytest.mark.multigpu
@pytest.mark.parametrize("decode_tp", [2, 4])
def test_a_relayed_latent_load_between_processes(golden, monkeypatch, decode_tp):
    """LEAN_VLLM_KVX_RELAY with the producer in a spawned process and the decode ranks on their own GPUs: each
    decode rank pulls its part of the latent blocks from the producer over CUDA IPC, then the others' parts from its
    peer decode ranks (in this process: peer access, no IPC), and lands what the reference's pull lands."""
    if gpu_count() < 1 + decode_tp:
        pytest.skip(f"needs {1 + decode_tp} GPUs")
    monkeypatch.setenv("LEAN_VLLM_KVX_RELAY", "1")
    _, arrays = golden
    kv_port, decode_port = free_port(), free_port()
    ctx = mp.get_context("spawn")
    parent, child = ctx.Pipe()
    proc = ctx.Process(target=_producer, args=(child, 0, kv_port, 1, 0, True))
    proc.start()
    consumers = []
    try:
        assert parent.poll(120) and parent.recv() == "ready"
        for rank in range(decode_tp):
            device = 1 + rank
            torch.cuda.set_device(device)
            kv = KVTransferConfig(kv_connector="CudaIpcConnector", kv_role="kv_consumer", kv_port=decode_port,
                                  engine_id="decode")
            worker = CudaIpcConnectorWorker(WorkerConfig(kv, tensor_parallel_size=decode_tp), rank)
            worker.register_kv_caches([rank_cache(full_cache(1, True), rank, decode_tp).to(device)])
            consumers.append(worker)
        from lean_vllm_b200.kv_transfer import ReqToRecv

        for worker in consumers:
            torch.cuda.set_device(worker.kv_caches[0].device)
            worker.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": ReqToRecv(
                [0, 5, 3], [7, 2, 9], "p-1", "engine", "127.0.0.1", kv_port, 1)}))
        outputs = [wait_for(w, timeout=60) for w in consumers]
        assert KVOutputAggregator(decode_tp).aggregate(outputs).finished_recving == {"d-1"}
        got = full_of([w.kv_caches[0].cpu() for w in consumers], True)
        assert np.array_equal(bits(got), arrays[f"small_lat_tp1to{decode_tp}"])
        assert parent.poll(60) and parent.recv() == "sent"
    finally:
        for worker in consumers:
            worker.shutdown()
        proc.join(timeout=60)
        if proc.is_alive():
            proc.kill()


@pytest.mark.multigpu
def test_a_load_the_engine_thread_launches_for_a_cache_on_another_gpu_lands(golden, monkeypatch):
    """Two ranks in one process: the producer's cache on cuda:0, the decode rank's on cuda:1, the calling thread's
    current device cuda:0. Once the producer is mapped, start_load_kv launches the next load itself -- on the decode
    cache's device, ordered after that device's current stream -- and it lands the reference's bytes."""
    if gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    import threading

    from lean_vllm_b200.kv_transfer.kvx_transport import KvxTransport

    _, arrays = golden
    torch.cuda.set_device(0)
    posting = []
    original = KvxTransport.post

    def post(self, *args, **kwargs):
        if self.device.index == 1 and not kwargs.get("save"):
            posting.append(threading.current_thread().name)
        return original(self, *args, **kwargs)

    monkeypatch.setattr(KvxTransport, "post", post)
    producers_side, consumers_side = Sides("cuda:0"), Sides("cuda:1")
    try:
        producers = producers_side.make("kv_producer", 1, full_cache(0, False))
        consumers = consumers_side.make("kv_consumer", 1, full_cache(1, False), engine_id="decode")
        before = consumers[0].kv_caches[0].clone()
        for request_id, local, remote in (("warm", [1], [4]), ("p-1", [0, 5, 3], [7, 2, 9])):
            producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={request_id: list(remote)}))
            consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={
                f"d-{request_id}": recv(producers, list(local), list(remote), remote_request_id=request_id)}))
            assert wait_for(consumers[0]).finished_recving == {f"d-{request_id}"}
            assert wait_for(producers[0]).finished_sending == {request_id}
            if request_id == "warm":
                consumers[0].kv_caches[0].copy_(before)  # the fixture's state before its load
        assert posting[0].startswith("kvx-ipc-") and posting[-1] == threading.current_thread().name
        assert torch.cuda.current_device() == 0
        assert np.array_equal(bits(consumers[0].kv_caches[0]), arrays["small_kv_tp1to1"])
    finally:
        consumers_side.close()
        producers_side.close()
