"""bench.py's sharding plan on CPU: for every workload, group count and pull/push mode, the jobs all ranks launch
move each decode rank's heads of every requested block exactly once, from the right prefill rank."""

import dataclasses

import numpy as np
import pytest

import bench


def tiny(spec: bench.Workload) -> bench.Workload:
    """Same topology and head split, small caches."""
    return dataclasses.replace(spec, layers=2, head_dim=8 if not spec.mla else 6, block=4, n_requests=6,
                               lengths=("uniform", 1, 11))


def caches(spec, tp, num_blocks, seed):
    rng = np.random.default_rng(seed)
    if spec.mla:
        shape = (1, num_blocks, spec.block, spec.head_dim)
    else:
        shape = (2, num_blocks, spec.kv_heads // tp, spec.block, spec.head_dim)
    return [rng.integers(0, 1 << 16, size=shape, dtype=np.uint16) for _ in range(spec.layers)]


def apply(job, src_layers, dst_layers, mla):
    """kvx_copy's byte map (include/kvx.h) on host arrays."""
    for s_layer, d_layer in zip(src_layers, dst_layers):
        for sb, db in zip(job.src_block_ids, job.dst_block_ids):
            if mla:
                if job.latents:
                    d_layer[:, db] = s_layer[:, sb]
            else:
                d_layer[:, db, job.dst_first_head : job.dst_first_head + job.num_heads] = \
                    s_layer[:, sb, job.src_first_head : job.src_first_head + job.num_heads]


CASES = [("pair", 2), ("pair", 8), ("hetero", 6), ("hetero", 8), ("mla", 3), ("mla", 8)]


@pytest.mark.parametrize("mode", ["pull", "push"])
@pytest.mark.parametrize("name, world", CASES)
def test_every_decode_rank_receives_exactly_its_heads(name, world, mode):
    spec = tiny(bench.WORKLOADS[name])
    _, reqs, num_blocks = bench.workload(3, None, spec)
    roles = [bench.role_of(r, world, spec) for r in range(world)]
    groups = world // spec.group_size
    assert sum(r.side == "decode" for r in roles) == groups * spec.decode_tp
    assert sum(r.side == "prefill" for r in roles) == groups * spec.prefill_tp
    mem = {}
    for rank, role in enumerate(roles):
        if role.side == "prefill":
            mem[rank] = caches(spec, spec.prefill_tp, num_blocks, seed=rank)
        elif role.side == "decode":
            mem[rank] = caches(spec, spec.decode_tp, num_blocks, seed=100 + rank)
    before = {rank: [a.copy() for a in layers] for rank, layers in mem.items()}

    def rank_of(group, side, tp_rank):
        return group * spec.group_size + (tp_rank if side == "prefill" else spec.prefill_tp + tp_rank)

    launched = 0
    for rank, role in enumerate(roles):
        peers, jobs = bench.plan(spec, role, reqs, mode)
        launched += bool(jobs)
        for job in jobs:
            tables = [mem.get(rank)] + [mem[rank_of(role.group, side, tp)] for side, tp in peers]
            apply(job, tables[job.src], tables[job.dst], spec.mla)
    assert launched == groups * (spec.decode_tp if mode == "pull" else spec.prefill_tp)

    # Expected: on every rank's heads together, dst[:, d] = src[:, s] for every request.
    heads = spec.kv_heads
    for group in range(groups):
        prefill_full = []
        for layer in range(spec.layers):
            parts = [before[rank_of(group, "prefill", q)][layer] for q in range(spec.prefill_tp)]
            prefill_full.append(parts[0] if spec.mla else np.concatenate(parts, axis=2))
        for r in range(spec.decode_tp):
            rank = rank_of(group, "decode", r)
            for layer in range(spec.layers):
                want = before[rank][layer].copy()
                for s, d in reqs:
                    if spec.mla:
                        want[:, d] = prefill_full[layer][:, s]
                    else:
                        per = heads // spec.decode_tp
                        want[:, d] = prefill_full[layer][:, s, r * per : (r + 1) * per]
                assert np.array_equal(mem[rank][layer], want), (group, r, layer)
    for rank, role in enumerate(roles):  # producers are only read
        if role.side == "prefill":
            assert all(np.array_equal(a, b) for a, b in zip(mem[rank], before[rank]))


def test_ranks_past_the_last_whole_group_stay_idle():
    spec = bench.WORKLOADS["hetero"]
    roles = [bench.role_of(r, 8, spec) for r in range(8)]
    assert [r.side for r in roles] == ["prefill"] * 2 + ["decode"] * 4 + ["idle"] * 2


def test_the_loopback_copies_whole_blocks_of_every_head():
    spec = tiny(bench.WORKLOADS["pair"])
    _, reqs, _ = bench.workload(0, None, spec)
    peers, jobs = bench.plan(spec, bench.role_of(0, 1, spec), reqs, "pull")
    assert peers == [("decode", 0)] and len(jobs) == len(reqs)
    assert all((j.src_first_head, j.dst_first_head, j.num_heads) == (0, 0, spec.kv_heads) for j in jobs)


def test_workload_draws_are_seeded_and_prefix_stable():
    a = bench.workload(0)
    b = bench.workload(0, 5)
    assert len(a[1]) == 64 and len(b[1]) == 5
    assert list(a[0][:5]) == list(b[0])  # the same prompt lengths
    ids = np.concatenate([s for s, _ in a[1]])
    assert len(set(ids.tolist())) == len(ids) and ids.max() < a[2]  # distinct source blocks inside the cache
    assert bench.request_bytes(32) == bench.BYTES_8K_REQUEST


@pytest.mark.parametrize("world", [3, 8])
def test_a_relayed_mla_load_lands_every_block_on_every_decode_rank(world):
    """--relay: each decode rank's own part from the prefill rank, then (after every rank's part landed) the others'
    parts from its peers; every decode rank ends with every requested latent block, the prefill rank sends each
    block once."""
    spec = tiny(bench.WORKLOADS["mla"])
    _, reqs, num_blocks = bench.workload(3, None, spec)
    roles = [bench.role_of(r, world, spec) for r in range(world)]
    groups = world // spec.group_size

    def rank_of(group, side, tp_rank):
        return group * spec.group_size + (tp_rank if side == "prefill" else spec.prefill_tp + tp_rank)

    mem = {rank: caches(spec, 1, num_blocks, seed=rank) for rank, role in enumerate(roles) if role.side != "idle"}
    before = {rank: [a.copy() for a in layers] for rank, layers in mem.items()}
    plans = {rank: bench.plan_relay(spec, role, reqs) for rank, role in enumerate(roles) if role.side == "decode"}
    sent_from_prefill = 0
    for phase in (1, 2):
        for rank, (peers, own, others) in plans.items():
            role = roles[rank]
            for job in own if phase == 1 else others:
                tables = [mem[rank]] + [mem[rank_of(role.group, side, tp)] for side, tp in peers]
                apply(job, tables[job.src], tables[job.dst], True)
                sent_from_prefill += len(job.src_block_ids) if phase == 1 else 0
    assert sent_from_prefill == groups * sum(len(d) for _, d in reqs)  # each block leaves the prefill GPU once
    for group in range(groups):
        prefill = before[rank_of(group, "prefill", 0)]
        for r in range(spec.decode_tp):
            rank = rank_of(group, "decode", r)
            for layer in range(spec.layers):
                want = before[rank][layer].copy()
                for s, d in reqs:
                    want[:, d] = prefill[layer][:, s]
                assert np.array_equal(mem[rank][layer], want), (group, r, layer)


def test_the_command_line_parses_every_mode():
    """Every mode's flags parse (argparse only; the modes themselves need GPUs)."""
    import contextlib
    import io

    with contextlib.redirect_stdout(io.StringIO()) as out, pytest.raises(SystemExit) as done:
        bench.main(["--help"])
    assert done.value.code == 0
    for flag in ("--relay", "--staged", "--store", "--poisson", "--layerwise", "--copy-engine", "--step-exchange",
                 "--impl", "--peer-device", "--serial"):
        assert flag in out.getvalue(), flag


@pytest.mark.parametrize("name", ["pair", "hetero", "mla"])
def test_the_reference_arm_s_legs_land_the_same_bytes(name):
    """bench.py's reference arm on tiny caches: the reference's own NixlConnectorWorker ranks (installed in
    baseline/_ref, NIXL replaced by the memmove agent) and the C restatement each move every request's blocks, with
    the reference's byte count, and the decode caches they leave are the same."""
    import os

    if not os.path.isdir(os.path.join(bench.REFERENCE_PATH, "lean_vllm")):
        pytest.skip("the reference is not installed in baseline/_ref")
    spec = tiny(bench.WORKLOADS[name])
    _, reqs, num_blocks = bench.workload(0, None, spec)
    producers = bench.host_rank_caches(spec, spec.prefill_tp, num_blocks, seed=1)
    by_reference = bench.host_rank_caches(spec, spec.decode_tp, num_blocks, seed=None)
    by_port = bench.host_rank_caches(spec, spec.decode_tp, num_blocks, seed=None)
    ref = bench.reference_worker_leg(spec, reqs, producers, by_reference, steps=1, warmup=1)
    port = bench.port_leg(spec, reqs, producers, by_port, steps=1, threads=2)
    assert "value" in ref, ref
    assert ref["kind"] == "reference" and port["kind"] == "port" and ref["same_config"]
    import torch

    for ref_rank, port_rank in zip(by_reference, by_port):
        for x, y in zip(ref_rank, port_rank):
            assert torch.equal(x.view(torch.int16), y.view(torch.int16))  # bit patterns: NaN words compare too
