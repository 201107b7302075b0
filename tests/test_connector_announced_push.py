"""The push with its block-ID exchange, end to end through both connector halves on CPU (host transport).

A proxy sends the decode request first with "kv_push": its scheduler half admits it and its worker ranks announce
the allocated blocks to the prefill ranks under the push id. The prefill request carries "kv_push_id": its
scheduler half turns its admission into a ReqToSave, its workers push as layers are computed (or at hand-over),
and the decode ranks finish once every byte has landed -- the reference's engine loop needs no change.
"""

from time import sleep

import numpy as np
import pytest

from lean_vllm_b200.kv_transfer import KVConnectorOutput, cuda_ipc_connector
from tests.connector_cases import BLOCK, Sides, full_cache, wait_for
from tests.helpers import bits, full_of
from tests.host_transport import HostTransport
from tests.push_cases import Seq, make_flow


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
@pytest.mark.parametrize("prefill_tp, decode_tp", [(1, 1), (2, 4), (4, 2), (2, 3)])
def test_an_announced_push_lands_what_the_reference_s_pull_lands(sides, golden, prefill_tp, decode_tp, mla):
    _, arrays = golden
    flow = make_flow(sides, prefill_tp, decode_tp, mla)
    flow.decode_admits()
    sleep(0.05)  # the announcements reach the prefill ranks before they prefill
    flow.prefill_runs()
    sent, recved = flow.results()
    assert sent.finished_sending == {"p-1"} and recved.finished_recving == {"d-1"}
    key = "lat" if mla else "kv"
    got = full_of([c.kv_caches[0] for c in flow.consumers], mla)
    assert np.array_equal(bits(got), arrays[f"small_{key}_tp{prefill_tp}to{decode_tp}"])


def test_a_prefill_that_ends_before_the_announcement_pushes_everything_when_it_comes(sides, golden):
    _, arrays = golden
    flow = make_flow(sides, 2, 4)
    flow.prefill_runs()  # no decode rank has announced: the layer hook pushes nothing
    sleep(0.05)
    assert all(p.transport.posts == [] for p in flow.producers)
    flow.decode_admits()
    sent, recved = flow.results()
    assert sent.finished_sending == {"p-1"} and recved.finished_recving == {"d-1"}
    assert np.array_equal(bits(full_of([c.kv_caches[0] for c in flow.consumers], False)), arrays["small_kv_tp2to4"])


def test_blocks_the_decode_instance_already_caches_are_not_pushed(sides):
    flow = make_flow(sides, 1, 1)
    before = flow.consumers[0].kv_caches[0].clone()
    flow.decode_admits(cached=1)  # block 0 is a local prefix hit: only 5 and 3 are written
    sleep(0.05)
    flow.prefill_runs()
    sent, recved = flow.results()
    assert recved.finished_recving == {"d-1"}
    got, prefill = flow.consumers[0].kv_caches[0], full_cache(0, False)
    assert bool((got[:, 0] == before[:, 0]).all())
    assert bool((got[:, [5, 3]] == prefill[:, [2, 9]]).all())
    assert recved.recv_stats["d-1"].num_bytes == 2 * 2 * 12 * 4 * 8 * 2  # two blocks of keys and values


def test_a_decode_request_whose_prefill_never_comes_fails_after_the_timeout(sides, monkeypatch):
    monkeypatch.setenv("LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT", "0.3")
    flow = make_flow(sides, 1, 1)
    flow.decode_admits()
    assert wait_for(flow.consumers[0]) == KVConnectorOutput(failed_recving={"d-1"})
    sleep(0.1)
    assert not flow.producers[0]._expects  # the unclaimed announcement expired too


def test_a_prefill_whose_decode_instance_never_announces_frees_its_blocks_at_the_timeout(sides, monkeypatch):
    monkeypatch.setenv("LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT", "0.3")
    flow = make_flow(sides, 1, 1)
    flow.prefill_runs()
    assert wait_for(flow.producers[0]) == KVConnectorOutput(finished_sending={"p-1"}, expired_sending={"p-1"})


def test_an_announcement_of_the_wrong_length_fails_both_sides(sides):
    flow = make_flow(sides, 1, 1)
    flow.decode_admits(blocks=(0, 5))  # a 2-block decode prompt for a 3-block prefill
    sleep(0.05)
    flow.prefill_runs()
    sent, recved = flow.results()
    assert sent.finished_sending == {"p-1"}
    assert recved.failed_recving == {"d-1"}


def test_a_pull_request_still_checks_its_block_count(sides):
    flow = make_flow(sides, 1, 1)
    seq = Seq("d-2", 3 * BLOCK, [0, 1, 2], {"do_remote_prefill": True, "remote_request_id": "x",
                                              "remote_engine_id": "e", "remote_host": "h", "remote_port": 1,
                                              "remote_block_ids": [4, 5]})
    assert flow.decode_half.get_num_new_matched_tokens(seq, 0) == (0, False)


def test_crossing_handshakes_do_not_deadlock(sides, monkeypatch):
    """A decode rank handshakes a prefill rank (to announce) while that prefill rank handshakes it (to map it):
    each must answer the other while it waits, or both stall until the timeout and the load fails."""
    monkeypatch.setattr(cuda_ipc_connector, "HANDSHAKE_TIMEOUT", 0.5)
    for attempt in range(4):
        flow = make_flow(sides, 2, 4)
        flow.prefill_runs(push_id=f"push-{attempt}")
        flow.decode_admits(push_id=f"push-{attempt}")  # announcements race the prefill ranks' mapping
        sent, recved = flow.results()
        assert sent.finished_sending == {"p-1"} and recved.finished_recving == {"d-1"}, attempt
