"""The fused store-and-push through the worker (store_kv / store_latents) on CPU caches over the host transport:
the layer's new rows land in the local cache and, for a save mapped before its first store, in the decode ranks'
blocks in the same call; hand-over then copies only what no store wrote (prefix-cache hits)."""

from time import sleep

import pytest
import torch

from lean_vllm_b200.kv_transfer import KVConnectorMetadata, ReqToRecv, cuda_ipc_connector
from lean_vllm_b200.kv_transfer.base import ReqToSave
from oracle.kv_oracle import store_kvcache as oracle_store
from tests.connector_cases import BLOCK, HEAD_DIM, LATENT_DIM, NUM_HEADS, Sides, full_cache, rank_cache, wait_for
from tests.helpers import bits, full_of
from tests.host_transport import HostStatusWord, HostTransport
from tests.push_cases import wait_ready

LOCAL, REMOTE = [7, 2, 9], [0, 5, 3]  # the prefill's blocks and the decode instance's


@pytest.fixture(autouse=True)
def host_transport(monkeypatch):
    monkeypatch.setattr(cuda_ipc_connector, "make_transport", HostTransport)
    monkeypatch.setattr(HostTransport, "fail", None)


@pytest.fixture
def sides():
    s = Sides("cpu")
    yield s
    s.close()


def rows(seed, tokens, heads, mla):
    g = torch.Generator().manual_seed(seed)
    shape = (tokens, LATENT_DIM) if mla else (tokens, heads, HEAD_DIM)
    return torch.randn(*shape, generator=g).to(torch.bfloat16), torch.randn(*shape, generator=g).to(torch.bfloat16)


def slots_of(blocks, first_block=0):
    return torch.tensor([b * BLOCK + o for b in blocks[first_block:] for o in range(BLOCK)], dtype=torch.int64)


def save_and_recv(producers, consumers, cached_blocks=0):
    kv_d, kv_p = consumers[0].kv_transfer, producers[0].kv_transfer
    save = ReqToSave(list(LOCAL), list(REMOTE), kv_d.engine_id, kv_d.kv_ip, kv_d.kv_port, len(consumers),
                     cached_blocks=cached_blocks)
    recv = ReqToRecv(list(REMOTE), list(LOCAL), "p-1", kv_p.engine_id, kv_p.kv_ip, kv_p.kv_port, len(producers),
                     pushed=True)
    for c in consumers:
        c.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv}))
    for p in producers:
        p.start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save}))
        assert wait_ready(p)


def hand_over(producers, consumers):
    for p in producers:
        p.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(LOCAL)}))
    sent = [wait_for(p) for p in producers]
    recved = [wait_for(c) for c in consumers]
    return sent, recved


@pytest.mark.parametrize("mla", [False, True], ids=["kv", "latents"])
@pytest.mark.parametrize("prefill_tp, decode_tp", [(1, 1), (2, 4), (4, 2), (1, 3)])
def test_a_fused_store_lands_the_new_rows_in_the_decode_blocks(sides, prefill_tp, decode_tp, mla):
    prefill, decode = full_cache(0, mla), full_cache(1, mla)
    producers = sides.make("kv_producer", prefill_tp, prefill)
    consumers = sides.make("kv_consumer", decode_tp, decode, engine_id="decode", accept_push=True)
    save_and_recv(producers, consumers)
    key, value = rows(5, 3 * BLOCK, NUM_HEADS, mla)  # every head's new rows: each prefill rank stores its slice
    slots = slots_of(LOCAL)
    for rank, p in enumerate(producers):
        if mla:
            p.store_latents(0, key, slots)
        else:
            per = NUM_HEADS // prefill_tp
            p.store_kv(0, key[:, rank * per : (rank + 1) * per].contiguous(),
                       value[:, rank * per : (rank + 1) * per].contiguous(), slots)
    sent, recved = hand_over(producers, consumers)
    assert all(s.finished_sending == {"p-1"} for s in sent) and all(r.finished_recving == {"d-1"} for r in recved)
    assert all(p.transport.posts == [] for p in producers)  # nothing left to copy at hand-over
    # The prefill's own cache holds the rows (the plain store), and the decode blocks now equal its blocks.
    full_prefill = full_of([p.kv_caches[0] for p in producers], mla)
    expected = prefill.clone()
    if mla:
        expected[0].reshape(-1, LATENT_DIM)[slots] = key
    else:
        e = bits(expected)
        oracle_store(bits(key), bits(value), e[0].swapaxes(1, 2), e[1].swapaxes(1, 2), slots.numpy())
        expected = torch.from_numpy(e.view("int16")).view(torch.bfloat16)
    assert torch.equal(full_prefill, expected)
    got = full_of([c.kv_caches[0] for c in consumers], mla)
    want = decode.clone()
    want[:, REMOTE] = expected[:, LOCAL]
    assert torch.equal(got, want)


def test_prefix_hit_blocks_are_copied_at_hand_over(sides):
    """Block 7 was a prefix-cache hit on the prefill side: no store writes it, so hand-over copies that block alone."""
    prefill, decode = full_cache(0, False), full_cache(1, False)
    producers = sides.make("kv_producer", 1, prefill)
    consumers = sides.make("kv_consumer", 1, decode, engine_id="decode", accept_push=True)
    save_and_recv(producers, consumers, cached_blocks=1)
    key, value = rows(6, 2 * BLOCK, NUM_HEADS, False)
    producers[0].store_kv(0, key, value, slots_of(LOCAL, first_block=1))
    hand_over(producers, consumers)
    assert producers[0].transport.posts == [(None, 1)]  # one copy of the first block, every layer
    got, have = consumers[0].kv_caches[0], producers[0].kv_caches[0]
    assert torch.equal(got[:, REMOTE], have[:, LOCAL])


def test_a_save_mapped_after_its_first_store_is_not_fused(sides):
    """Rows stored before the decode ranks were mapped never reached them, so such a save pushes whole layers."""
    prefill, decode = full_cache(0, False), full_cache(1, False)
    producers = sides.make("kv_producer", 1, prefill)
    consumers = sides.make("kv_consumer", 1, decode, engine_id="decode", accept_push=True)
    kv_d, kv_p = consumers[0].kv_transfer, producers[0].kv_transfer
    key, value = rows(7, 3 * BLOCK, NUM_HEADS, False)
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_save={
        "p-1": ReqToSave(list(LOCAL), list(REMOTE), kv_d.engine_id, kv_d.kv_ip, kv_d.kv_port, 1)}))
    with producers[0]._lock:
        producers[0]._saves["p-1"].ready = False  # as if the first handshake were still in flight
    producers[0].store_kv(0, key, value, slots_of(LOCAL))
    assert producers[0].transport.stores == [(0, 12)]
    with producers[0]._lock:
        producers[0]._saves["p-1"].ready = True
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": ReqToRecv(
        list(REMOTE), list(LOCAL), "p-1", kv_p.engine_id, kv_p.kv_ip, kv_p.kv_port, 1, pushed=True)}))
    hand_over(producers, consumers)
    assert producers[0].transport.posts == [(None, 1)]  # the whole cache, at hand-over
    assert torch.equal(consumers[0].kv_caches[0][:, REMOTE], producers[0].kv_caches[0][:, LOCAL])


def test_a_finished_save_leaves_the_block_map(sides):
    """After hand-over the prefill's blocks go back to the engine: a later store into them must not reach the old
    decode blocks."""
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode", accept_push=True)
    save_and_recv(producers, consumers)
    key, value = rows(8, 3 * BLOCK, NUM_HEADS, False)
    producers[0].store_kv(0, key, value, slots_of(LOCAL))
    hand_over(producers, consumers)
    landed = consumers[0].kv_caches[0].clone()
    key2, value2 = rows(9, 3 * BLOCK, NUM_HEADS, False)
    producers[0].store_kv(0, key2, value2, slots_of(LOCAL))  # the blocks, reused by another request
    assert torch.equal(consumers[0].kv_caches[0], landed)
    assert producers[0].transport.stores[-1] == (0, 12)


def test_a_store_with_no_saves_is_the_plain_store(sides, golden):
    _, arrays = golden
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    cache = producers[0].kv_caches[0]
    before = bits(cache).copy()
    key, value = rows(10, 5, NUM_HEADS, False)
    slots = torch.tensor([3, 17, -1, 40, 0])
    producers[0].store_kv(0, key, value, slots)
    oracle_store(bits(key), bits(value), before[0].swapaxes(1, 2), before[1].swapaxes(1, 2), slots.numpy())
    assert (bits(cache) == before).all()


def test_a_re_admitted_prefill_starts_its_save_over(sides):
    """A preempted prefill is admitted again in new blocks: the new ReqToSave replaces the old one."""
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode", accept_push=True)
    save_and_recv(producers, consumers)
    kv_d = consumers[0].kv_transfer
    producers[0].store_kv(0, *rows(11, 3 * BLOCK, NUM_HEADS, False), slots_of(LOCAL))
    new_local = [1, 4, 6]
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_save={
        "p-1": ReqToSave(new_local, list(REMOTE), kv_d.engine_id, kv_d.kv_ip, kv_d.kv_port, 1)}))
    sleep(0.05)
    key, value = rows(12, 3 * BLOCK, NUM_HEADS, False)
    producers[0].store_kv(0, key, value, slots_of(new_local))
    for p in producers:
        p.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": new_local}))
    assert wait_for(producers[0]).finished_sending == {"p-1"}
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    assert torch.equal(consumers[0].kv_caches[0][:, REMOTE], producers[0].kv_caches[0][:, new_local])


def test_rank_cache_helper_slices_heads():
    full = full_cache(0, False)
    assert torch.equal(torch.cat([rank_cache(full, r, 3) for r in range(3)], dim=2), full)


def test_a_fully_fused_save_is_reported_only_after_its_stores_land(sides):
    """Every layer stored fused: nothing is copied at hand-over, but the decode ranks hear of the request only once
    the engine stream's stores have landed (a fence on the hand-over's ready marker)."""
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode", accept_push=True)
    save_and_recv(producers, consumers)
    key, value = rows(5, 3 * BLOCK, NUM_HEADS, False)
    producers[0].store_kv(0, key, value, slots_of(LOCAL))
    held = []
    transport = producers[0].transport
    real_fence = transport.fence

    def slow_fence(ready):
        handle = real_fence(ready)
        transport.pending[handle] = [10**9]  # the stores are still running
        held.append(handle)
        return handle

    transport.fence = slow_fence
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(LOCAL)}))
    sleep(0.3)
    assert len(held) == 1 and transport.posts == []
    assert consumers[0].get_finished().finished_recving == set()
    assert producers[0].get_finished().finished_sending == set()
    transport.pending[held[0]] = [0]  # landed
    assert wait_for(producers[0]).finished_sending == {"p-1"}
    assert wait_for(consumers[0]).finished_recving == {"d-1"}


def test_decode_blocks_past_the_decode_cache_fail_the_save_before_any_store(sides):
    """A decode instance that names blocks its cache does not have: the prefill rank refuses the save when it maps
    the decode ranks (before any block map names those ids), stores only locally, and the decode instance hears
    "not ok" at hand-over and prefills."""
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode", accept_push=True)
    kv_d, kv_p = consumers[0].kv_transfer, producers[0].kv_transfer
    num_blocks = consumers[0].kv_caches[0].size(1)
    bad = [0, num_blocks, 3]
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": ReqToRecv(
        bad, list(LOCAL), "p-1", kv_p.engine_id, kv_p.kv_ip, kv_p.kv_port, 1, pushed=True)}))
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_save={
        "p-1": ReqToSave(list(LOCAL), bad, kv_d.engine_id, kv_d.kv_ip, kv_d.kv_port, 1)}))
    assert wait_ready(producers[0]) is False
    producers[0].store_kv(0, *rows(13, 3 * BLOCK, NUM_HEADS, False), slots_of(LOCAL))
    assert producers[0].transport.stores[-1] == (0, 3 * BLOCK)  # local only
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(LOCAL)}))
    assert wait_for(producers[0]).finished_sending == {"p-1"}
    assert wait_for(consumers[0]).failed_recving == {"d-1"}


def test_a_fused_store_that_skipped_rows_fails_its_save(sides, monkeypatch):
    """The device-side check behind the host's: if a store skips a row because its decode block lies past the
    decode rank's cache (its status word set), the save fails before the decode instance is told its blocks are
    full. The host's range check is bypassed here so that the store itself meets the bad id."""
    monkeypatch.setattr(cuda_ipc_connector, "_ids_fit", lambda ids, num_blocks: True)
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode", accept_push=True)
    kv_d, kv_p = consumers[0].kv_transfer, producers[0].kv_transfer
    num_blocks = consumers[0].kv_caches[0].size(1)
    bad = [0, num_blocks, 3]
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": ReqToRecv(
        bad, list(LOCAL), "p-1", kv_p.engine_id, kv_p.kv_ip, kv_p.kv_port, 1, pushed=True)}))
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_save={
        "p-1": ReqToSave(list(LOCAL), bad, kv_d.engine_id, kv_d.kv_ip, kv_d.kv_port, 1)}))
    assert wait_ready(producers[0])
    opened = HostStatusWord.opened
    producers[0].store_kv(0, *rows(14, 3 * BLOCK, NUM_HEADS, False), slots_of(LOCAL))
    assert producers[0].transport.stores[-1] == (1, 3 * BLOCK)  # fused, one decode rank
    assert HostStatusWord.opened == opened + 1
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(LOCAL)}))
    assert wait_for(producers[0]).finished_sending == {"p-1"}
    assert wait_for(consumers[0]).failed_recving == {"d-1"}
    assert HostStatusWord.opened == opened  # the save let go of its store's word
