"""kv_connector_step (ModelRunner.kv_connector_step, engine/model_runner.py:637-649) with the shared-memory step
mailbox: the same aggregated outputs on rank 0 as the reference's gloo gather_object, step for step, at 2 and 4
ranks; the mailbox's ordering (a rank waits for rank 0's read of the step before), overflow and timeouts."""

import os
import random
import socket
import threading
import time
import uuid

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from lean_vllm_b200 import _native
from lean_vllm_b200.kv_transfer.base import KVConnectorOutput, KVOutputAggregator, KVTransferStats
from lean_vllm_b200.kv_transfer.step import KVConnectorStep, StepMailbox, decode, encode

pytestmark = pytest.mark.skipif(not os.path.exists(_native.LIB_PATH), reason="libkvx.so is not built here")


def _path():
    return f"/dev/shm/kvx-step-test-{os.getpid()}-{uuid.uuid4().hex[:8]}"


def test_encode_and_decode_round_trip():
    out = KVConnectorOutput({"a"}, {"b", "c"}, {"d"}, {"a"}, {"b": KVTransferStats(0.5, 12)})
    assert decode(encode(out)) == out
    assert encode(KVConnectorOutput()) == b"" and decode(b"") == KVConnectorOutput()


def test_a_rank_posts_the_next_step_only_after_rank_0_read_the_last():
    path = _path()
    boxes = [StepMailbox(path, 3, r, 64, create=(r == 0)) for r in range(3)]
    os.unlink(path)
    try:
        boxes[1].post(1, b"one")
        boxes[2].post(1, b"")
        assert boxes[0].collect(1) == [b"", b"one", b""]
        later = threading.Thread(target=boxes[1].post, args=(2, b"two"))
        later.start()
        time.sleep(0.1)
        assert later.is_alive()  # slot 1 still holds step 1 until rank 0 releases it
        boxes[0].release(1)
        later.join(timeout=5)
        assert not later.is_alive()
        boxes[2].post(2, b"z" * 64)  # a full slot
        assert boxes[0].collect(2) == [b"", b"two", b"z" * 64]
    finally:
        for box in boxes:
            box.close()


def test_an_oversized_output_and_a_silent_rank_raise():
    path = _path()
    boxes = [StepMailbox(path, 2, r, 64, create=(r == 0)) for r in range(2)]
    os.unlink(path)
    try:
        with pytest.raises(_native.KvxRangeError, match="does not fit"):
            boxes[1].post(1, b"x" * 65, timeout=0.1)
        started = time.monotonic()
        with pytest.raises(_native.KvxTimeout, match="rank 1 did not post step 1"):
            boxes[0].collect(1, timeout=0.3)
        assert time.monotonic() - started < 5
        with pytest.raises(_native.KvxTimeout, match="rank 0 did not read step 1"):
            boxes[1].post(2, b"", timeout=0.2)  # step 1 was never read
    finally:
        for box in boxes:
            box.close()


def script(world: int, steps: int, seed: int):
    """Per rank, per step: a KVConnectorOutput. Each request finishes on every rank, at its own step per rank; some
    fail on one rank; producers' sends finish the same way, some expired."""
    rng = random.Random(seed)
    outs = [[KVConnectorOutput() for _ in range(steps)] for _ in range(world)]
    for k in range(40):
        failing = rng.randrange(world) if k % 7 == 0 else -1
        expired = k % 5 == 0
        for rank in range(world):
            step = rng.randrange(steps)
            o = outs[rank][step]
            if k % 2:
                o.finished_sending.add(f"s{k}")
                if expired:
                    o.expired_sending.add(f"s{k}")
            elif rank == failing:
                o.failed_recving.add(f"r{k}")
            else:
                o.finished_recving.add(f"r{k}")
                o.recv_stats[f"r{k}"] = KVTransferStats(rng.random(), rng.randrange(1, 1 << 20))
    return outs


class Scripted:
    """A connector worker half that reports a scripted output each step."""

    def __init__(self, outputs):
        self.outputs, self.step, self.started = outputs, 0, []

    def start_load_kv(self, metadata):
        self.started.append(metadata)

    def get_finished(self):
        out = self.outputs[self.step]
        self.step += 1
        return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, steps, seed, results):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        outs = script(world, steps, seed)[rank]
        got = {}
        for exchange in ("gather", "mailbox"):
            step = KVConnectorStep(Scripted(outs), rank, world, exchange=exchange, timeout=30.0)
            got[exchange] = [step({"step": i}) for i in range(steps)]
            step.close()
            dist.barrier()
        if rank == 0:
            results.put(("ok", [(encode(a), encode(b)) for a, b in zip(got["gather"], got["mailbox"])]))
        else:
            assert all(x is None for x in got["gather"] + got["mailbox"])
        dist.destroy_process_group()
    except BaseException as error:  # noqa: BLE001 - reported to the parent
        results.put(("error", f"rank {rank}: {type(error).__name__}: {error}"))
        raise


@pytest.mark.parametrize("world", [2, 4])
def test_the_mailbox_aggregates_what_the_reference_gather_does(world):
    steps, seed = 25, 11
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, steps, seed, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    messages = []
    while not results.empty():
        messages.append(results.get())
    errors = [m for kind, m in messages if kind == "error"]
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    (pairs,) = [m for kind, m in messages if kind == "ok"]
    # Both exchanges give rank 0 the same thing every step, and that is the reference aggregator over all ranks.
    aggregator = KVOutputAggregator(world)
    outs = script(world, steps, seed)
    finished = set()
    for i, (gathered, mailed) in enumerate(pairs):
        assert decode(gathered) == decode(mailed), i
        want = aggregator.aggregate([outs[r][i] for r in range(world)])
        assert decode(mailed) == want, i
        finished |= want.finished_recving | want.failed_recving | want.finished_sending
    assert len(finished) == 40  # every request completed once all its ranks reported it


def test_a_single_rank_returns_its_own_output():
    outs = script(1, 3, 5)[0]
    step = KVConnectorStep(Scripted(outs), 0, 1)
    assert [step({}) for _ in range(3)] == outs
