"""The CPU oracle against the golden fixtures recorded from the reference connector itself.

Pins both restatements (oracle/kv_oracle.py in Python, oracle/kvx_oracle.c in C) before any GPU result is checked
against them.
"""

import numpy as np
import pytest
import torch

from oracle import c_oracle
from oracle.kv_oracle import (
    Region,
    Share,
    block_descs,
    expected_decode,
    head_shares,
    load_between,
)
from tests.helpers import bits, full_of, seeded, sha


def test_head_shares_match_the_reference_on_every_split(golden):
    meta, _ = golden
    assert len(meta["head_shares"]) > 300
    for rank, tp, rtp, heads, shares in meta["head_shares"]:
        expected = [Share(*s) for s in shares]
        assert head_shares(rank, tp, rtp, heads) == expected, (rank, tp, rtp, heads)
        assert c_oracle.head_shares(rank, tp, rtp, heads) == expected, (rank, tp, rtp, heads)


def test_head_shares_known_answers_of_the_reference_tests():
    # tests/test_nixl_connector.py:199-204
    assert head_shares(0, 1, 1, 8) == [Share(0, 0, 0, 8)]
    assert head_shares(3, 4, 2, 8) == [Share(1, 2, 0, 2)]
    assert head_shares(1, 2, 4, 8) == [Share(2, 0, 0, 2), Share(3, 0, 2, 2)]
    assert head_shares(1, 6, 4, 12) == [Share(0, 2, 0, 1), Share(1, 0, 1, 1)]


def test_block_descs_rows_match_the_reference(golden):
    meta, _ = golden
    table = meta["block_descs"]
    regions = [Region(*r) for r in table["regions"]]
    for case in table["cases"]:
        rows = block_descs(regions, table["block_ids"], case["first_head"], case["num_heads"], case["latents"],
                           table["device_id"])
        assert rows.tolist() == case["rows"]
        addr, length = c_oracle.block_descs(regions, table["block_ids"], case["first_head"], case["num_heads"],
                                            case["latents"])
        assert addr.tolist() == [r[0] for r in case["rows"]]
        assert length.tolist() == [r[1] for r in case["rows"]]


def _c_copy(threads):
    def copy(local, remote):
        if len(local):
            c_oracle.read(local[:, 0], remote[:, 0], local[:, 1], threads)

    return copy


@pytest.mark.parametrize("copy", [None, _c_copy(1), _c_copy(4)], ids=["python", "c-1thread", "c-4threads"])
def test_every_small_case_matches_the_reference_bit_for_bit(golden, copy):
    meta, arrays = golden
    small = meta["small"]
    for case in small["cases"]:
        key = "lat" if case["mla"] else "kv"
        prefill, decode = arrays[f"small_{key}_prefill"], arrays[f"small_{key}_decode"]
        local, remote = case.get("local", small["local"]), case.get("remote", small["remote"])
        consumers, moved = load_between([prefill], [decode], case["prefill_tp"], case["decode_tp"], local, remote,
                                        copy)
        full = full_of([c[0] for c in consumers], case["mla"])
        assert np.array_equal(full, arrays[case["name"]]), case["name"]
        assert moved == case["bytes_per_rank"], case["name"]
        assert np.array_equal(full, expected_decode(prefill, decode, local, remote)), case["name"]


def test_the_reference_s_byte_count_known_answer(golden):
    # tests/test_nixl_connector.py:264: one block of keys and values, 12 heads of 4 tokens x 8, bf16.
    meta, _ = golden
    case = next(c for c in meta["small"]["cases"] if c["name"] == "small_kv_prefix_hit")
    assert case["bytes_per_rank"] == [2 * 12 * 4 * 8 * 2]


@pytest.mark.parametrize("key", ["qwen_kv", "dsv2_lat"])
def test_model_shaped_cases_match_the_reference_digests(golden, key):
    meta, _ = golden
    spec = meta[key]
    shape = tuple(spec["shape"])
    prefill = [seeded(shape, s) for s in spec["prefill_seeds"]]
    decode = [seeded(shape, s) for s in spec["decode_seeds"]]
    assert [sha(t) for t in prefill] == spec["input_sha256"]["prefill"]
    assert [sha(t) for t in decode] == spec["input_sha256"]["decode"]
    p_bits, d_bits = [bits(t) for t in prefill], [bits(t) for t in decode]
    for case in spec["cases"]:
        consumers, moved = load_between(p_bits, d_bits, case["prefill_tp"], case["decode_tp"], spec["local"],
                                        spec["remote"], _c_copy(4))
        assert moved == case["bytes_per_rank"], case["name"]
        for layer in range(spec["layers"]):
            full = full_of([c[layer] for c in consumers], case["mla"])
            assert sha(full) == case["layer_sha256"][layer], (case["name"], layer)


def test_a_planted_offset_error_is_caught(golden):
    """The fixtures can tell a wrong head offset: shift the consumer's first head by one and the result differs."""
    meta, arrays = golden
    prefill, decode = arrays["small_kv_prefill"], arrays["small_kv_decode"]

    def shifted(local, remote):
        local = local.copy()
        local[:, 0] += np.uint64(8 * 4 * 2)  # one head further on
        mask = np.ones(len(local), bool)
        mask[-3:] = False  # keep the last rows in bounds
        from oracle.kv_oracle import read_rows

        read_rows(local[mask], remote[mask])

    consumers, _ = load_between([prefill], [decode], 2, 4, [0, 5, 3], [7, 2, 9], shifted)
    assert not np.array_equal(full_of([c[0] for c in consumers], False), arrays["small_kv_tp2to4"])


def test_bf16_bits_round_trip():
    t = seeded((3, 5), 7)
    assert torch.equal(torch.from_numpy(bits(t).view(np.int16)).view(torch.bfloat16), t)


@pytest.mark.parametrize("latents", [False, True], ids=["kv", "latent"])
def test_place_rows_is_the_closed_form_of_a_scatter(latents):
    """The oracle's staged scatter writes row i of the staging buffer into block ids[i] (heads first..first+n), the
    same result as numpy indexing -- the reference tests' closed form -- so it can judge kvx_scatter alone."""
    from oracle.kv_oracle import place_rows

    rng = np.random.default_rng(5)
    shape = (12, 16, 576) if latents else (12, 4, 16, 8)
    region = rng.integers(0, 1 << 16, size=shape, dtype=np.uint16)
    ids = [11, 0, 5, 7]
    first, n = (0, 0) if latents else (1, 2)
    rows = rng.integers(0, 1 << 16, size=(len(ids), *(shape[1:] if latents else (n, *shape[2:]))), dtype=np.uint16)
    want = region.copy()
    if latents:
        want[ids] = rows
    else:
        want[ids, first : first + n] = rows
    moved = place_rows(region, ids, rows, first, n, latents)
    assert moved == rows.nbytes
    assert np.array_equal(region, want)
