"""Properties the connector's arithmetic must keep for every size, checked over generated cases (hypothesis):
head shares tile each consumer rank's heads exactly once from the right producer heads, readers count the same
overlaps from the other side, relay parts partition a load's blocks, per-layer save spans leave every block
pushed in its final state once the prompt is done -- whatever the chunking -- the native planner's byte count
and range checks agree with the oracle's block_descs, the store oracle writes what the reference's torch store
writes, and head shares, reader counts, descriptor rows, the output aggregator, the pull-mode scheduler half and the
request-params and --kv-transfer-config checks agree with the reference's own functions."""

from hypothesis import event, given, settings
from hypothesis import strategies as st

from lean_vllm_b200.kv_transfer.cuda_ipc_connector import _cdiv, relay_parts
from lean_vllm_b200.kv_transfer.shares import head_shares, readers_of, split_heads


@st.composite
def splits(draw):
    tp = draw(st.integers(1, 8))
    remote_tp = draw(st.integers(1, 8))
    base = split_heads(0, tp, remote_tp)  # the least count both sizes divide
    return tp, remote_tp, base * draw(st.integers(1, 4))


@settings(max_examples=300, deadline=None)
@given(splits())
def test_shares_tile_every_consumer_rank_s_heads_from_the_producer_that_holds_them(case):
    tp, remote_tp, heads = case
    per_local, per_remote = heads // tp, heads // remote_tp
    for rank in range(tp):
        covered = []
        for share in head_shares(rank, tp, remote_tp, heads):
            assert share.num_heads > 0
            for k in range(share.num_heads):
                global_head = rank * per_local + share.local_head + k
                assert global_head == share.remote_rank * per_remote + share.remote_head + k
                assert 0 <= share.remote_head + k < per_remote
                covered.append(share.local_head + k)
        assert covered == list(range(per_local))  # each local head once, in order


@settings(max_examples=300, deadline=None)
@given(splits())
def test_a_producer_rank_counts_as_readers_exactly_the_consumer_ranks_that_take_its_heads(case):
    tp, remote_tp, heads = case
    for remote_rank in range(remote_tp):
        takers = [r for r in range(tp) if any(s.remote_rank == remote_rank for s in head_shares(r, tp, remote_tp, heads))]
        assert readers_of(remote_rank, remote_tp, tp, heads) == len(takers)


@settings(max_examples=300, deadline=None)
@given(st.integers(0, 200), st.integers(1, 8))
def test_relay_parts_partition_a_load_s_blocks(n, tp):
    parts = relay_parts(n, tp)
    assert parts[0][0] == 0 and parts[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
    assert max(e - s for s, e in parts) - min(e - s for s, e in parts) <= 1  # balanced


class _Req:
    def __init__(self, blocks, tokens):
        self.local_block_ids = list(range(blocks))
        self.num_tokens = tokens


class _Save:
    def __init__(self, req):
        self.req, self.progress, self.layer_blocks = req, None, {}


@settings(max_examples=300, deadline=None)
@given(st.integers(1, 9), st.integers(1, 300), st.data())
def test_per_layer_spans_end_with_every_block_final_whatever_the_chunking(block, tokens, data):
    """Drive CudaIpcConnectorWorker._layer_span as save_kv_layer does, chunk by chunk: every block is pushed after
    its last write, no block is pushed again once final, and nothing is left for hand-over."""
    from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker

    blocks = _cdiv(tokens, block)
    worker = CudaIpcConnectorWorker.__new__(CudaIpcConnectorWorker)
    worker.block_size = block
    save = _Save(_Req(blocks, tokens))
    cuts = sorted(set(data.draw(st.lists(st.integers(1, tokens - 1), max_size=6)) if tokens > 1 else []))
    last_pushed_at = {}  # block -> chunk index of its last push
    last_written_at = {}  # block -> chunk index of its last write
    done = 0
    for chunk, end in enumerate(cuts + [tokens]):
        for position in range(done, end):
            last_written_at[position // block] = chunk
        done = end
        save.progress = end
        final_before = save.layer_blocks.get(0, 0)
        start, stop, final = worker._layer_span(save, 0)
        assert start == final_before  # a block once final is never pushed again
        for b in range(start, stop):
            last_pushed_at[b] = chunk
        save.layer_blocks[0] = final
    assert save.layer_blocks[0] == blocks  # hand-over finds nothing left
    assert all(last_pushed_at[b] >= last_written_at[b] for b in range(blocks))


@st.composite
def planner_cases(draw):
    """Region tables for both sides of a job (keys/values or latent layers), and one job whose ids and head range
    may fall outside them. Addresses are never touched: only the host planner runs."""
    layers = draw(st.lists(st.sampled_from(["kv", "latent"]), min_size=1, max_size=4))
    head_bytes = draw(st.integers(1, 512))
    src_heads, dst_heads = draw(st.integers(1, 8)), draw(st.integers(1, 8))
    page = draw(st.integers(1, 4096))
    src_blocks, dst_blocks = draw(st.integers(1, 12)), draw(st.integers(1, 12))

    def table(heads, base):
        regions = []
        for i, kind in enumerate(layers):
            for part in ((0, 1) if kind == "kv" else (0,)):
                addr = base + (2 * i + part) * (1 << 32)
                regions.append((addr, heads * head_bytes, head_bytes) if kind == "kv" else (addr, page, 0))
        return regions

    n = draw(st.integers(0, 6) if draw(st.integers(0, 9)) == 0 else st.integers(1, 6))  # empty loads now and then
    bad_id, bad_heads = draw(st.integers(0, 4)) == 0, draw(st.integers(0, 4)) == 0  # mostly valid jobs
    src_ids = draw(st.lists(st.integers(-1 if bad_id else 0, src_blocks if bad_id else src_blocks - 1),
                            min_size=n, max_size=n))
    dst_ids = draw(st.lists(st.integers(-1 if bad_id else 0, dst_blocks if bad_id else dst_blocks - 1),
                            min_size=n, max_size=n))
    if bad_heads:
        src_head, dst_head, heads = draw(st.integers(0, 9)), draw(st.integers(0, 9)), draw(st.integers(0, 9))
    else:
        heads = draw(st.integers(0, min(src_heads, dst_heads)))
        src_head, dst_head = draw(st.integers(0, src_heads - heads)), draw(st.integers(0, dst_heads - heads))
    job = (src_head, dst_head, heads, draw(st.booleans()))
    return (table(src_heads, 1 << 44), src_blocks), (table(dst_heads, 1 << 45), dst_blocks), src_ids, dst_ids, job


@settings(max_examples=400, deadline=None)
@given(planner_cases())
def test_the_native_planner_counts_and_refuses_what_the_oracle_says(case):
    """kvx_job_bytes (the planner every launch runs) against block_descs: the same byte count for any tables and
    job, and a range error exactly where a block id or head range falls outside a cache."""
    import os

    import pytest

    from lean_vllm_b200 import _native
    from lean_vllm_b200.kv_transfer.transport import CacheTable, CopyJob, job_bytes
    from oracle.kv_oracle import Region, block_descs

    if not os.path.exists(_native.LIB_PATH):
        pytest.skip("libkvx.so is not built here")
    (src_regions, src_blocks), (dst_regions, dst_blocks), src_ids, dst_ids, (src_head, dst_head, heads, latents) = case
    job = CopyJob(0, 1, src_ids, dst_ids, src_head, dst_head, heads, latents)
    tables = [CacheTable(src_regions, src_blocks), CacheTable(dst_regions, dst_blocks)]
    ids_out = any(not 0 <= b < src_blocks for b in src_ids) or any(not 0 <= b < dst_blocks for b in dst_ids)
    heads_out = any(h and (first + heads) * h > block
                    for regions, first in ((src_regions, src_head), (dst_regions, dst_head))
                    for _, block, h in regions)
    if src_ids and (ids_out or heads_out):
        event("refused: " + ("block id" if ids_out else "head range"))
        with pytest.raises(_native.KvxRangeError):
            job_bytes(tables, [job])
        return
    rows = block_descs([Region(*r) for r in src_regions], src_ids, src_head, heads, latents)
    expected = int(rows[:, 1].sum()) if len(rows) else 0
    event("counted: " + ("nothing" if expected == 0 else "bytes"))
    assert job_bytes(tables, [job]) == expected


def _reference_kv():
    """The reference checkout's kv_transfer package (REFERENCE_ROOT, else a "reference" folder beside this
    repository), or None."""
    import importlib
    import os
    import sys

    root = os.environ.get("REFERENCE_ROOT", os.path.join(os.path.dirname(__file__), "..", "..", "reference"))
    if not os.path.isdir(os.path.join(root, "lean_vllm")):
        return None
    sys.path.insert(0, root)
    try:
        return importlib.import_module("lean_vllm.kv_transfer.base")
    except ImportError:
        return None
    finally:
        sys.path.remove(root)


@st.composite
def rank_outputs(draw):
    """A few steps of every rank's output: request ids from a small pool, each rank reporting any of them."""
    world = draw(st.integers(1, 4))
    pool = ["r0", "r1", "r2", "r3", "r4"]
    ids = st.sets(st.sampled_from(pool), max_size=3)
    steps = []
    for _ in range(draw(st.integers(1, 4))):
        step = []
        for _ in range(world):
            recving, failed = draw(ids), draw(ids)
            stats = {rid: (draw(st.floats(0, 5, allow_nan=False)), draw(st.integers(0, 1 << 40))) for rid in recving}
            step.append((draw(ids), recving, failed, draw(ids), stats))
        steps.append(step)
    return world, steps


@settings(max_examples=300, deadline=None)
@given(rank_outputs())
def test_the_aggregator_matches_the_reference_s_on_any_rank_outputs(case):
    """KVOutputAggregator against the reference's own (kv_transfer/base.py:125-165), step after step: the same
    finished, failed and expired sets and the same merged stats (slowest rank's time, every rank's bytes)."""
    import pytest

    from lean_vllm_b200.kv_transfer.base import KVConnectorOutput, KVOutputAggregator, KVTransferStats

    ref = _reference_kv()
    if ref is None:
        pytest.skip("no lean-vLLM reference checkout")
    world, steps = case
    ours, theirs = KVOutputAggregator(world), ref.KVOutputAggregator(world)
    for step in steps:
        mine = ours.aggregate([KVConnectorOutput(set(s), set(r), set(f), set(e),
                                                 {k: KVTransferStats(*v) for k, v in st_.items()})
                               for s, r, f, e, st_ in step])
        ref_out = theirs.aggregate([ref.KVConnectorOutput(set(s), set(r), set(f), set(e),
                                                          {k: ref.KVTransferStats(*v) for k, v in st_.items()})
                                    for s, r, f, e, st_ in step])
        assert mine.finished_sending == ref_out.finished_sending
        assert mine.finished_recving == ref_out.finished_recving
        assert mine.failed_recving == ref_out.failed_recving
        assert mine.expired_sending == ref_out.expired_sending
        assert {k: (v.seconds, v.num_bytes) for k, v in mine.recv_stats.items()} == \
            {k: (v.seconds, v.num_bytes) for k, v in ref_out.recv_stats.items()}


@st.composite
def scheduler_events(draw):
    """A request as both scheduler halves see it (pull mode): its prompt and block table, prefix hits here, the
    kv_transfer_params it arrives with (the block count sometimes wrong), and how it finishes."""
    block = 16
    prompt = draw(st.integers(1, 200))
    blocks = -(-prompt // block)
    table = draw(st.lists(st.integers(0, 999), min_size=blocks, max_size=blocks + 1, unique=True))
    cached = draw(st.integers(0, blocks - 1 if prompt % block == 0 else blocks)) * block
    cached = min(cached, (prompt - 1) // block * block)  # the last prompt token is always computed here
    remote = draw(st.lists(st.integers(0, 999), min_size=blocks, max_size=blocks)) if draw(st.integers(0, 4)) else \
        draw(st.lists(st.integers(0, 999), max_size=blocks + 2))
    params = {"do_remote_prefill": draw(st.booleans()), "do_remote_decode": draw(st.booleans()),
              "remote_request_id": "p-1", "remote_engine_id": draw(st.sampled_from(["e1", "e2"])),
              "remote_block_ids": remote, "remote_host": "10.0.0.1", "remote_port": draw(st.integers(1, 65535)),
              "tp_size": draw(st.integers(1, 8))}
    return block, prompt, table, cached, params, draw(st.sampled_from(["length", "stop", "abort", None]))


@settings(max_examples=300, deadline=None)
@given(scheduler_events())
def test_the_scheduler_half_matches_the_reference_s_in_pull_mode(event):
    """CudaIpcConnectorScheduler against the reference's NixlConnectorScheduler (nixl_connector.py:111-168) on the
    same request: the same admission answer, the same load (ids, remote request, engine, address, tp_size), the
    same step metadata and the same hand-over params."""
    import copy
    import importlib
    import types

    import pytest

    from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorScheduler

    if _reference_kv() is None:
        pytest.skip("no lean-vLLM reference checkout")
    nixl = importlib.import_module("lean_vllm.kv_transfer.nixl_connector")
    block, prompt, table, cached, params, finish = event
    kv = types.SimpleNamespace(engine_id="this-engine", kv_ip="10.0.0.2", kv_port=15000)
    config = types.SimpleNamespace(kv_transfer=kv, kvcache_block_size=block, tensor_parallel_size=2)
    results = []
    for half in (CudaIpcConnectorScheduler(config), nixl.NixlConnectorScheduler(config)):
        seq = types.SimpleNamespace(request_id="r", num_prompt_tokens=prompt, block_table=list(table),
                                    num_cached_tokens=cached, kv_transfer_params=copy.deepcopy(params),
                                    finish_reason=finish, num_scheduled_tokens=0)
        matched = half.get_num_new_matched_tokens(seq, cached)
        if matched[1]:
            half.update_state_after_alloc(seq, matched[0])
        meta = half.build_connector_meta()
        loads = {rid: (list(r.local_block_ids), list(r.remote_block_ids), r.remote_request_id, r.remote_engine_id,
                       r.remote_host, r.remote_port, r.remote_tp_size) for rid, r in meta.reqs_to_recv.items()}
        handed = half.request_finished(seq)
        sends = half.build_connector_meta().reqs_to_send
        results.append((matched, loads, dict(meta.reqs_to_send), handed, {k: list(v) for k, v in sends.items()},
                        seq.kv_transfer_params))
    assert results[0] == results[1]


@settings(max_examples=400, deadline=None)
@given(st.dictionaries(
    st.sampled_from(["do_remote_prefill", "do_remote_decode", "remote_block_ids", "remote_request_id",
                     "remote_engine_id", "remote_host", "remote_port", "tp_size", "kv_push", "kv_push_id"]),
    st.one_of(st.booleans(), st.integers(-2, 70000), st.text(max_size=4), st.none(),
              st.lists(st.integers(0, 9), max_size=3), st.lists(st.text(max_size=2), max_size=2))),
    st.sampled_from(["kv_producer", "kv_consumer", "kv_both", None]))
def test_request_params_are_judged_as_the_reference_judges_them(params, role):
    """check_kv_transfer_params (what the API server asks before admitting a request) gives the reference's answer,
    word for word, on any params object and engine role."""
    import pytest

    from lean_vllm_b200.kv_transfer.base import KVTransferConfig, check_kv_transfer_params

    ref = _reference_kv()
    if ref is None:
        pytest.skip("no lean-vLLM reference checkout")
    ours = KVTransferConfig(kv_role=role) if role else None
    theirs = ref.KVTransferConfig(kv_role=role) if role else None
    assert check_kv_transfer_params(dict(params), ours) == ref.check_kv_transfer_params(dict(params), theirs)


@settings(max_examples=300, deadline=None)
@given(st.dictionaries(
    st.sampled_from(["kv_connector", "kv_role", "kv_ip", "kv_port", "engine_id", "kv_buffer_device"]),
    st.one_of(st.sampled_from(["kv_producer", "kv_consumer", "kv_both", "NixlConnector"]), st.integers(-1, 70000),
              st.text(max_size=3), st.none(), st.floats(allow_nan=False, allow_infinity=False), st.booleans())))
def test_kv_transfer_config_parses_as_the_reference_parses_it(value):
    """--kv-transfer-config JSON: accepted or refused exactly when the reference's is, with the same fields (the
    connector name's default and the random engine id aside)."""
    import json

    import pytest
    from pydantic import ValidationError

    from lean_vllm_b200.kv_transfer.base import KVTransferConfig

    ref = _reference_kv()
    if ref is None:
        pytest.skip("no lean-vLLM reference checkout")
    text = json.dumps(value)
    got = []
    for cls in (KVTransferConfig, ref.KVTransferConfig):
        try:
            config = cls.parse(text)
        except ValidationError:
            got.append("refused")
            continue
        got.append((config.kv_role, config.kv_ip, config.kv_port, config.engine_id if "engine_id" in value else None,
                    config.kv_connector if "kv_connector" in value else None))
    assert got[0] == got[1]


@st.composite
def store_steps(draw):
    """A step's rows for a paged cache: shape, layout (NHD, or HND seen through its transposed view), and distinct
    slots with -1 padding among them, as an engine's slot mapping has."""
    blocks, block, heads, dim = draw(st.integers(1, 5)), draw(st.integers(1, 8)), draw(st.integers(1, 4)), \
        draw(st.integers(1, 8))
    slots = draw(st.lists(st.one_of(st.integers(0, blocks * block - 1), st.just(-1)), max_size=blocks * block))
    seen, distinct = set(), []
    for slot in slots:  # an engine never maps two rows of a step to one slot: repeats become padding
        distinct.append(slot if slot < 0 or slot not in seen else -1)
        seen.add(slot)
    slots = distinct
    return blocks, block, heads, dim, slots, draw(st.sampled_from(["NHD", "HND"])), draw(st.integers(0, 1 << 16))


@settings(max_examples=200, deadline=None)
@given(store_steps())
def test_the_store_oracle_writes_what_the_reference_s_torch_store_writes(step):
    """oracle.kv_oracle.store_kvcache / store_latents -- what the kvx_store GPU tests are checked against -- against
    the reference's TorchAttention store (attention/torch_backend.py:34-60) on any shape, layout and slot mapping."""
    import importlib

    import numpy as np
    import pytest
    import torch

    from oracle.kv_oracle import store_kvcache, store_latents

    if _reference_kv() is None:
        pytest.skip("no lean-vLLM reference checkout")
    torch_store = importlib.import_module("lean_vllm.attention.torch_backend").TorchAttention
    blocks, block, heads, dim, slots, layout, seed = step
    g = torch.Generator().manual_seed(seed)
    n = len(slots)
    key, value = (torch.randn(n, heads, dim, generator=g).to(torch.bfloat16) for _ in range(2))
    shape = (2, blocks, block, heads, dim) if layout == "NHD" else (2, blocks, heads, block, dim)
    cache = torch.randn(*shape, generator=g).to(torch.bfloat16)

    def views(c):
        return (c[0], c[1]) if layout == "NHD" else (c[0].transpose(1, 2), c[1].transpose(1, 2))

    theirs = cache.clone()
    torch_store.store_kvcache(None, key, value, *views(theirs), torch.tensor(slots, dtype=torch.long))
    mine = cache.clone().view(torch.int16).numpy()
    k_view, v_view = (mine[0], mine[1]) if layout == "NHD" else (mine[0].swapaxes(1, 2), mine[1].swapaxes(1, 2))
    store_kvcache(key.view(torch.int16).numpy(), value.view(torch.int16).numpy(), k_view, v_view, slots)
    assert np.array_equal(mine, theirs.view(torch.int16).numpy())

    latent = torch.randn(n, dim, generator=g).to(torch.bfloat16)
    lat_cache = torch.randn(blocks, block, dim, generator=g).to(torch.bfloat16)
    theirs_lat = lat_cache.clone()
    torch_store.store_latents(None, latent, theirs_lat, torch.tensor(slots, dtype=torch.long))
    mine_lat = lat_cache.clone().view(torch.int16).numpy()
    store_latents(latent.view(torch.int16).numpy(), mine_lat, slots)
    assert np.array_equal(mine_lat, theirs_lat.view(torch.int16).numpy())


@settings(max_examples=500, deadline=None)
@given(st.integers(1, 8), st.integers(1, 8), st.integers(1, 32), st.data())
def test_head_shares_and_reader_counts_are_the_reference_s(tp, remote_tp, multiple, data):
    """head_shares and the reader count a producer rank waits for, against the reference's own functions
    (nixl_connector.py:60-77, 400-401) on any split: every consumer rank of any pair of tensor-parallel sizes, up
    to 256 heads (the golden table holds 372 splits of these)."""
    import importlib

    import pytest

    if _reference_kv() is None:
        pytest.skip("no lean-vLLM reference checkout")
    nixl = importlib.import_module("lean_vllm.kv_transfer.nixl_connector")
    heads = split_heads(0, tp, remote_tp) * multiple
    rank = data.draw(st.integers(0, tp - 1))
    ours = head_shares(rank, tp, remote_tp, heads)
    theirs = nixl.head_shares(rank, tp, remote_tp, heads)
    assert [tuple(s) for s in ours] == [tuple(s) for s in theirs]
    for share in theirs:
        assert readers_of(share.remote_rank, remote_tp, tp, heads) == \
            len(nixl.head_shares(share.remote_rank, remote_tp, tp, heads))


@settings(max_examples=300, deadline=None)
@given(st.lists(st.tuples(st.integers(1, 1 << 40), st.integers(1, 1 << 20), st.sampled_from([0, 16, 512, 65536])),
                min_size=0, max_size=6),
       st.lists(st.integers(0, 4096), max_size=8), st.integers(0, 8), st.integers(0, 8), st.booleans())
def test_the_oracle_s_descriptor_rows_are_the_reference_s(regions, block_ids, first_head, num_heads, latents):
    """oracle.kv_oracle.block_descs -- the byte map every parity check here rests on -- against the reference's own
    block_descs (nixl_connector.py:89-108): the same (address, length, device) rows in the same order."""
    import importlib

    import numpy as np
    import pytest

    from oracle.kv_oracle import Region, block_descs

    if _reference_kv() is None:
        pytest.skip("no lean-vLLM reference checkout")
    nixl = importlib.import_module("lean_vllm.kv_transfer.nixl_connector")
    ours = block_descs([Region(*r) for r in regions], block_ids, first_head, num_heads, latents, device_id=3)
    theirs = nixl.block_descs([nixl.Region(*r) for r in regions], block_ids, first_head, num_heads, latents, 3)
    assert ours.shape == theirs.shape and np.array_equal(ours.astype(np.uint64), theirs)
