"""The worker half against the reference's own, on generated loads: lean-vLLM's NixlConnectorWorker (over the
memmove NIXL agent of tests/golden/make_golden.py) and CudaIpcConnectorWorker (over the host transport) load the same
blocks between the same caches, for any pair of tensor-parallel sizes, keys/values or latents, any block ids and
any prefix hit. The decode ranks' caches must end bit for bit equal, and each rank must count the same bytes. The
same loads also run as pushes (this package's ReqToSave, written by the prefill ranks at hand-over): the decode
caches must end as the reference's pull leaves them. And as relayed loads (LEAN_VLLM_KVX_RELAY: latents split
between decode ranks, each pulling its part and copying the rest from its peers), which must land the same bytes.

The golden fixtures pin a few such loads; this runs as many as hypothesis draws. Skipped where no reference
checkout is present (REFERENCE_ROOT)."""

import importlib.util
import os

import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

HERE = os.path.dirname(os.path.abspath(__file__))
REFERENCE_ROOT = os.environ.get("REFERENCE_ROOT", os.path.join(HERE, "..", "..", "reference"))
if not os.path.isdir(os.path.join(REFERENCE_ROOT, "lean_vllm")):
    pytest.skip("no lean-vLLM reference checkout", allow_module_level=True)

from lean_vllm_b200.kv_transfer import KVConnectorMetadata, ReqToRecv, cuda_ipc_connector  # noqa: E402
from lean_vllm_b200.kv_transfer.base import ReqToSave  # noqa: E402
from tests.connector_cases import Sides, free_port, recv, wait_for  # noqa: E402
from tests.host_transport import HostTransport  # noqa: E402

BLOCKS, BLOCK, HEADS, DIM, LATENT = 12, 4, 12, 8, 6
TP_SIZES = [(1, 1), (2, 2), (1, 2), (2, 1), (1, 4), (4, 1), (2, 4), (4, 2), (4, 6), (6, 4), (2, 3), (3, 6), (6, 1)]


def _reference():
    """tests/golden/make_golden.py as a module, loaded once: the reference's worker over a memmove agent."""
    import sys

    if "kvx_make_golden" not in sys.modules:
        os.environ.setdefault("REFERENCE_ROOT", REFERENCE_ROOT)
        spec = importlib.util.spec_from_file_location("kvx_make_golden",
                                                      os.path.join(HERE, "golden", "make_golden.py"))
        module = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = module  # its dataclasses look their module up while it runs
        spec.loader.exec_module(module)
        # Its ranks bind port + rank: take ports whose whole span is free and never handed out before, as this
        # package's side does, so many loads in a row do not collide.
        module.free_port = free_port
    return sys.modules["kvx_make_golden"]


@st.composite
def loads(draw):
    prefill_tp, decode_tp = draw(st.sampled_from(TP_SIZES))
    mla = draw(st.booleans())
    layers = draw(st.integers(1, 2))
    n = draw(st.integers(0, 6))
    remote = draw(st.lists(st.integers(0, BLOCKS - 1), min_size=n, max_size=n, unique=True))
    local = draw(st.lists(st.integers(0, BLOCKS - 1), min_size=n, max_size=n, unique=True))
    hits = draw(st.integers(0, n))  # leading blocks the decode instance already holds: not read
    mode = draw(st.sampled_from(["pull", "push", "relay"]))
    return prefill_tp, decode_tp, mla, layers, local[hits:], remote[hits:], draw(st.integers(0, 1 << 16)), mode


@settings(max_examples=40, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(loads())
def test_a_load_lands_what_the_reference_worker_lands(load):
    prefill_tp, decode_tp, mla, n_layers, local, remote, seed, mode = load
    ref = _reference()
    shape = (1, BLOCKS, BLOCK, LATENT) if mla else (2, BLOCKS, HEADS, BLOCK, DIM)
    prefill = [ref.seeded(shape, seed + i) for i in range(n_layers)]
    decode = [ref.seeded(shape, seed + 100 + i) for i in range(n_layers)]
    want, want_bytes = ref.run_load(prefill, decode, prefill_tp, decode_tp, BLOCK, local, remote)

    make_transport, fail = cuda_ipc_connector.make_transport, HostTransport.fail
    cuda_ipc_connector.make_transport, HostTransport.fail = HostTransport, None
    relay = os.environ.get("LEAN_VLLM_KVX_RELAY")
    os.environ["LEAN_VLLM_KVX_RELAY"] = "1" if mode == "relay" else "0"
    sides = Sides("cpu")
    try:
        producers = sides.make("kv_producer", prefill_tp, [p.clone() for p in prefill])
        consumers = sides.make("kv_consumer", decode_tp, [d.clone() for d in decode], engine_id="decode",
                               accept_push=mode == "push")
        if mode in ("pull", "relay"):
            for producer in producers:
                producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(remote)}))
            for consumer in consumers:
                consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": recv(producers, list(local),
                                                                                    list(remote))}))
        else:  # the decode side waits; the prefill ranks push everything at hand-over (no per-layer hooks)
            kv_p, kv_d = producers[0].kv_transfer, consumers[0].kv_transfer
            for consumer in consumers:
                consumer.start_load_kv(KVConnectorMetadata(reqs_to_recv={"d-1": ReqToRecv(
                    list(local), list(remote), "p-1", kv_p.engine_id, kv_p.kv_ip, kv_p.kv_port, prefill_tp,
                    pushed=True)}))
            save = ReqToSave(list(remote), list(local), kv_d.engine_id, kv_d.kv_ip, kv_d.kv_port, decode_tp)
            for producer in producers:
                producer.start_load_kv(KVConnectorMetadata(reqs_to_save={"p-1": save}))
                producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"p-1": list(remote)}))
        outputs = [wait_for(consumer) for consumer in consumers]
        assert all(out.finished_recving == {"d-1"} for out in outputs)
        assert [out.recv_stats["d-1"].num_bytes for out in outputs] == want_bytes
        for rank, consumer in enumerate(consumers):
            for got, expected in zip(consumer.kv_caches, want[rank]):
                assert torch.equal(got.view(torch.int16), expected.view(torch.int16)), (rank, load)
    finally:
        sides.close()
        cuda_ipc_connector.make_transport, HostTransport.fail = make_transport, fail
        if relay is None:
            os.environ.pop("LEAN_VLLM_KVX_RELAY", None)
        else:
            os.environ["LEAN_VLLM_KVX_RELAY"] = relay
