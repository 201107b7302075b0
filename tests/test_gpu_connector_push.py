"""The per-layer save (push) on CUDA devices with the kvx transport, in one process on one GPU: bit for bit against
the reference's golden pulls, layer launches on the bounded SM budget, and the ordering after each layer's store."""

import numpy as np
import pytest
import torch

from lean_vllm_b200.kv_transfer import KVConnectorMetadata
from tests.connector_cases import BLOCK, Sides, full_cache, wait_for
from tests.helpers import bits, full_of
from tests.push_cases import LOCAL, REMOTE, pushed_recv, run_push, save_req, wait_ready

pytestmark = pytest.mark.gpu


@pytest.fixture
def sides():
    s = Sides("cuda")
    yield s
    s.close()


@pytest.mark.parametrize("mla", [False, True], ids=["kv", "latents"])
@pytest.mark.parametrize("prefill_tp, decode_tp", [(1, 1), (2, 4), (4, 2), (4, 6), (1, 2)])
def test_a_pushed_request_lands_what_the_reference_s_pull_lands_on_the_gpu(sides, golden, prefill_tp, decode_tp,
                                                                           mla):
    _, arrays = golden
    producers = sides.make("kv_producer", prefill_tp, full_cache(0, mla))
    consumers = sides.make("kv_consumer", decode_tp, full_cache(1, mla), engine_id="decode", accept_push=True)
    sent, recved = run_push(producers, consumers, layers_to_save=[0])
    assert sent.finished_sending == {"p-1"} and recved.finished_recving == {"d-1"}
    key = "lat" if mla else "kv"
    got = full_of([c.kv_caches[0].cpu() for c in consumers], mla)
    assert np.array_equal(bits(got), arrays[f"small_{key}_tp{prefill_tp}to{decode_tp}"])


@pytest.mark.parametrize("hooks", [[0, 1, 2], [0, 2], []], ids=["every-layer", "some-layers", "no-hooks"])
def test_layers_pushed_by_hooks_and_at_hand_over_land_bit_for_bit(sides, hooks):
    layers = [full_cache(10 + i, False) for i in range(3)]
    producers = sides.make("kv_producer", 2, layers)
    consumers = sides.make("kv_consumer", 1, [full_cache(20 + i, False) for i in range(3)], engine_id="decode",
                           accept_push=True)
    sent, recved = run_push(producers, consumers, layers_to_save=hooks)
    assert sent.finished_sending == {"p-1"} and recved.finished_recving == {"d-1"}
    for layer in range(3):
        want = full_cache(20 + layer, False)
        want[:, LOCAL] = layers[layer][:, REMOTE]
        assert torch.equal(consumers[0].kv_caches[layer].cpu(), want), layer


def test_a_layer_is_pushed_only_after_its_store_on_the_engine_stream(sides):
    """save_kv_layer records an event on the engine's stream: a store still queued behind a long kernel is what
    lands, not the bytes before it."""
    producers = sides.make("kv_producer", 1, full_cache(0, False))
    consumers = sides.make("kv_consumer", 1, full_cache(1, False), engine_id="decode", accept_push=True)
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": pushed_recv(producers)}))
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save_req(consumers)},
                                                   save_progress={"p-1": 3 * BLOCK}))
    assert wait_ready(producers[0])
    cache = producers[0].kv_caches[0]
    torch.cuda._sleep(50_000_000)  # the layer's attention, still running ...
    cache[:, REMOTE] = 7.0  # ... before its store writes the blocks
    producers[0].save_kv_layer(0)
    producers[0].start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    assert wait_for(producers[0]).finished_sending == {"p-1"}
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    assert bool((consumers[0].kv_caches[0][:, LOCAL] == 7.0).all())


def test_a_per_layer_save_launch_is_held_to_its_sm_budget(sides, monkeypatch):
    """The save's launch covers at most LEAN_VLLM_KVX_SAVE_SMS SMs (the grid is capped), and still lands every byte."""
    monkeypatch.setenv("LEAN_VLLM_KVX_SAVE_SMS", "2")
    big = torch.randn(2, 16, 12, 64, 128).to(torch.bfloat16)
    producers = sides.make("kv_producer", 1, big)
    consumers = sides.make("kv_consumer", 1, torch.zeros_like(big), engine_id="decode", accept_push=True)
    assert producers[0].transport.save_flags >> 24 == 2
    sent, recved = run_push(producers, consumers, layers_to_save=[0])
    assert recved.finished_recving == {"d-1"}
    want = torch.zeros_like(big)
    want[:, LOCAL] = big[:, REMOTE]
    assert torch.equal(consumers[0].kv_caches[0].cpu(), want)


@pytest.mark.parametrize("prefill_tp, decode_tp, mla", [(1, 1, False), (2, 4, False), (1, 2, True)])
def test_an_announced_push_through_both_halves_on_the_gpu(sides, golden, prefill_tp, decode_tp, mla):
    """The decode request is admitted first and its ranks announce their blocks; the prefill's admission turns into
    a ReqToSave; the bytes land as the reference's pull lands them."""
    from time import sleep

    from tests.push_cases import make_flow

    _, arrays = golden
    flow = make_flow(sides, prefill_tp, decode_tp, mla)
    flow.decode_admits()
    sleep(0.1)
    flow.prefill_runs()
    sent, recved = flow.results()
    assert sent.finished_sending == {"p-1"} and recved.finished_recving == {"d-1"}
    key = "lat" if mla else "kv"
    got = full_of([c.kv_caches[0].cpu() for c in flow.consumers], mla)
    assert np.array_equal(bits(got), arrays[f"small_{key}_tp{prefill_tp}to{decode_tp}"])


@pytest.mark.parametrize("split", [False, True], ids=["one-launch", "push-on-save-stream"])
@pytest.mark.parametrize("prefill_tp, decode_tp, mla", [(1, 1, False), (2, 4, False), (4, 2, False),
                                                        (1, 2, True)])
def test_a_fused_store_lands_the_new_rows_in_the_decode_blocks_on_the_gpu(sides, monkeypatch, prefill_tp, decode_tp,
                                                                          mla, split):
    """store_kv writes each rank's new rows into its own cache and, through the block map, into every decode rank's
    blocks -- in one kvx_store launch, or (LEAN_VLLM_KVX_FUSED_ASYNC) the local half on the engine's stream and the
    push half on the save stream; hand-over then has nothing left to copy."""
    monkeypatch.setenv("LEAN_VLLM_KVX_FUSED_ASYNC", "1" if split else "0")
    from lean_vllm_b200.kv_transfer import ReqToRecv
    from lean_vllm_b200.kv_transfer.base import ReqToSave
    from tests.connector_cases import HEAD_DIM, LATENT_DIM, NUM_HEADS

    prefill, decode = full_cache(0, mla), full_cache(1, mla)
    producers = sides.make("kv_producer", prefill_tp, prefill)
    consumers = sides.make("kv_consumer", decode_tp, decode, engine_id="decode", accept_push=True)
    kv_d, kv_p = consumers[0].kv_transfer, producers[0].kv_transfer
    local, remote = [7, 2, 9], [0, 5, 3]
    for c in consumers:
        c.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": ReqToRecv(
            remote, local, "p-1", kv_p.engine_id, kv_p.kv_ip, kv_p.kv_port, prefill_tp, pushed=True)}))
    for p in producers:
        p.start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": ReqToSave(
            local, remote, kv_d.engine_id, kv_d.kv_ip, kv_d.kv_port, decode_tp)}))
        assert wait_ready(p)
    g = torch.Generator().manual_seed(3)
    shape = (3 * BLOCK, LATENT_DIM) if mla else (3 * BLOCK, NUM_HEADS, HEAD_DIM)
    key = torch.randn(*shape, generator=g).to(torch.bfloat16).cuda()
    value = torch.randn(*shape, generator=g).to(torch.bfloat16).cuda()
    slots = torch.tensor([b * BLOCK + o for b in local for o in range(BLOCK)], device="cuda")
    for rank, p in enumerate(producers):
        if mla:
            p.store_latents(0, key, slots)
        else:
            per = NUM_HEADS // prefill_tp
            p.store_kv(0, key[:, rank * per : (rank + 1) * per].contiguous(),
                       value[:, rank * per : (rank + 1) * per].contiguous(), slots)
    for p in producers:
        p.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": local}))
    assert all(wait_for(p).finished_sending == {"p-1"} for p in producers)
    assert all(wait_for(c).finished_recving == {"d-1"} for c in consumers)
    have = full_of([p.kv_caches[0].cpu() for p in producers], mla)
    got = full_of([c.kv_caches[0].cpu() for c in consumers], mla)
    want = decode.clone()
    want[:, remote] = have[:, local]
    assert torch.equal(got, want)
    if mla:
        assert torch.equal(have[0].reshape(-1, LATENT_DIM)[slots.cpu()], key.cpu())
    else:
        assert torch.equal(have[0].transpose(1, 2).reshape(-1, NUM_HEADS, HEAD_DIM)[slots.cpu()], key.cpu())


def test_a_chunked_prefill_lands_its_final_blocks_on_the_gpu(sides):
    """Three chunks ending inside blocks, each written on the engine's stream behind a long kernel before its layer
    hooks run: every chunk re-pushes the partly filled block on the save stream, in order, so the decode blocks
    end equal to the prefill's final ones."""
    from lean_vllm_b200.kv_transfer.base import ReqToSave

    producers = sides.make("kv_producer", 1, [full_cache(50 + i, False) for i in range(2)])
    consumers = sides.make("kv_consumer", 1, [full_cache(60 + i, False) for i in range(2)], engine_id="decode",
                           accept_push=True)
    consumers[0].start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": pushed_recv(producers)}))
    kv = consumers[0].kv_transfer
    tokens = 3 * BLOCK - 1
    save = ReqToSave(list(REMOTE), list(LOCAL), kv.engine_id, kv.kv_ip, kv.kv_port, 1, num_tokens=tokens)
    producer = producers[0]
    for step, (begin, end) in enumerate([(0, BLOCK + 1), (BLOCK + 1, 2 * BLOCK + 1), (2 * BLOCK + 1, tokens)]):
        producer.start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save} if step == 0 else {},
                                                   save_progress={"p-1": end}))
        if step == 0:
            assert wait_ready(producer)
        for layer, cache in enumerate(producer.kv_caches):
            torch.cuda._sleep(5_000_000)  # the layer's compute, still running when the hook is called
            for position in range(begin, end):
                cache[:, REMOTE[position // BLOCK], :, position % BLOCK] = float(100 * layer + position)
            producer.save_kv_layer(layer)
    producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(REMOTE)}))
    assert wait_for(producer).finished_sending == {"p-1"}
    assert wait_for(consumers[0]).finished_recving == {"d-1"}
    for layer in range(2):
        got, have = consumers[0].kv_caches[layer].cpu(), producer.kv_caches[layer].cpu()
        for i, (d, s) in enumerate(zip(LOCAL, REMOTE)):
            rows = BLOCK if i < 2 else BLOCK - 1
            assert torch.equal(got[:, d, :, :rows], have[:, s, :, :rows]), (layer, i)
