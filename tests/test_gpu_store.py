"""kvx_store through the C ABI: the per-token cache store bit for bit against the reference's torch store (golden
fixtures and the oracle), and the fused store-and-push into peers' caches with head resharding and latent
replication."""

import numpy as np
import pytest
import torch

from lean_vllm_b200.attention.kvx_cache import PushTarget, store_kvcache, store_latents
from lean_vllm_b200.kv_transfer import transport
from oracle.kv_oracle import store_kvcache as oracle_store
from tests.helpers import bits, from_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("slot_dtype", [torch.int64, torch.int32])
@pytest.mark.parametrize("layout", ["NHD", "HND"])
def test_the_store_matches_the_reference(golden, layout, slot_dtype):
    _, arrays = golden
    key = from_bits(arrays["store_key"]).cuda()
    value = from_bits(arrays["store_value"]).cuda()
    slots = torch.from_numpy(arrays["store_slots"]).to(slot_dtype).cuda()
    cache = from_bits(arrays[f"store_{layout}_before"]).cuda()
    view = cache if layout == "NHD" else cache.transpose(2, 3)
    store_kvcache(key, value, view[0], view[1], slots)
    torch.cuda.synchronize()
    assert np.array_equal(bits(cache), arrays[f"store_{layout}_after"])


def test_the_latent_store_matches_the_reference(golden):
    _, arrays = golden
    cache = from_bits(arrays["store_latent_before"]).cuda()
    store_latents(from_bits(arrays["store_latent"]).cuda(), cache[0],
                  torch.from_numpy(arrays["store_slots"]).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(bits(cache), arrays["store_latent_after"])


def _qwen_step(tokens=3000, blocks=40, heads=8, seed=0, hnd=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    key = torch.randn(tokens, heads, 128, generator=g, device="cuda").to(torch.bfloat16)
    value = torch.randn(tokens, heads, 128, generator=g, device="cuda").to(torch.bfloat16)
    shape = (2, blocks, heads, 256, 128) if hnd else (2, blocks, 256, heads, 128)
    cache = torch.randn(*shape, generator=g, device="cuda").to(torch.bfloat16)
    slots = torch.randperm(blocks * 256, generator=g, device="cuda")[:tokens]
    slots[::97] = -1
    return key, value, cache, slots


@pytest.mark.parametrize("hnd", [True, False], ids=["HND", "NHD"])
def test_a_model_sized_store_matches_the_oracle(hnd):
    key, value, cache, slots = _qwen_step(hnd=hnd)
    expected = bits(cache).copy()
    e_view = expected if not hnd else expected.swapaxes(2, 3)
    oracle_store(bits(key), bits(value), e_view[0], e_view[1], slots.cpu().numpy())
    view = cache.transpose(2, 3) if hnd else cache
    store_kvcache(key, value, view[0], view[1], slots)
    torch.cuda.synchronize()
    assert np.array_equal(bits(cache), expected)


def test_the_fused_store_also_writes_each_peer_s_heads_into_its_own_slots():
    """TP1 prefill -> TP2 decode: the store writes all 8 heads locally and heads 0-3 / 4-7 into two 4-head decode
    caches at their own (shuffled) slots, in the same launch. Every expected cache comes from the oracle's store
    (the reference's torch store, restated) on host copies: no kvx kernel computes what is expected."""
    key, value, cache, slots = _qwen_step(tokens=2000)
    peers = [torch.zeros(2, 30, 4, 256, 128, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    peer_slots = [torch.randperm(30 * 256, device="cuda")[:2000] for _ in range(2)]
    peer_slots[1][5] = -1
    targets = [PushTarget.of(p.transpose(2, 3)[0], p.transpose(2, 3)[1], s, src_first_head=4 * r, num_heads=4)
               for r, (p, s) in enumerate(zip(peers, peer_slots))]
    k_bits, v_bits = bits(key), bits(value)
    expected_local = bits(cache).copy()
    ev = expected_local.swapaxes(2, 3)  # (2, blocks, tokens, heads, dim), as the store addresses an HND cache
    oracle_store(k_bits, v_bits, ev[0], ev[1], slots.cpu().numpy())
    expected_peers = []
    for r, (p, s) in enumerate(zip(peers, peer_slots)):
        e = bits(p).copy()
        pv = e.swapaxes(2, 3)
        oracle_store(np.ascontiguousarray(k_bits[:, 4 * r : 4 * r + 4]), np.ascontiguousarray(v_bits[:, 4 * r : 4 * r + 4]),
                     pv[0], pv[1], s.cpu().numpy())
        expected_peers.append(e)
    before = transport.launch_count()
    word = transport.StatusWord()
    view = cache.transpose(2, 3)
    store_kvcache(key, value, view[0], view[1], slots, push_to=targets, status=word.address)
    torch.cuda.synchronize()
    assert transport.launch_count() - before == 1
    assert word.bits() == 0
    word.close()
    assert np.array_equal(bits(cache), expected_local)
    for p, e in zip(peers, expected_peers):
        assert np.array_equal(bits(p), e)


def test_the_fused_latent_store_replicates_to_every_decode_rank():
    g = torch.Generator(device="cuda").manual_seed(3)
    latent = torch.randn(1000, 576, generator=g, device="cuda").to(torch.bfloat16)
    local = torch.zeros(1, 40, 64, 576, device="cuda", dtype=torch.bfloat16)
    slots = torch.randperm(40 * 64, device="cuda")[:1000]
    peers = [torch.zeros(1, 50, 64, 576, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    peer_slots = [torch.randperm(50 * 64, device="cuda")[:1000].to(torch.int32) for _ in range(3)]
    store_latents(latent, local[0], slots, push_to=[PushTarget.of(p[0], None, s) for p, s in zip(peers, peer_slots)])
    torch.cuda.synchronize()
    assert torch.equal(local[0].reshape(-1, 576)[slots], latent)
    for p, s in zip(peers, peer_slots):
        assert torch.equal(p[0].reshape(-1, 576)[s.long()], latent)


def test_a_slot_past_the_cache_is_skipped_and_flagged_in_the_launch_s_status_word():
    key, value, cache, slots = _qwen_step(tokens=64, blocks=4)
    slots[10] = 4 * 256  # one past the last slot
    expected = bits(cache).copy()
    keep = slots.cpu().numpy().copy()
    keep[10] = -1  # the row the kernel must skip
    ev = expected.swapaxes(2, 3)
    oracle_store(bits(key), bits(value), ev[0], ev[1], keep)
    assert transport.device_error() == 0
    word = transport.StatusWord()
    view = cache.transpose(2, 3)
    store_kvcache(key, value, view[0], view[1], slots, status=word.address)
    torch.cuda.synchronize()
    assert word.bits() == 2
    word.close()
    assert transport.device_error() == 2
    assert transport.device_error() == 0  # read and cleared
    assert np.array_equal(bits(cache), expected)


def test_a_peer_block_map_entry_past_the_peer_cache_is_flagged_not_written():
    """A fused push whose block map sends a row to a block past the decode rank's cache skips that row and says so
    in the store's status word -- what fails the save before the decode instance is told its blocks are full."""
    key, value, cache, slots = _qwen_step(tokens=300, blocks=8)
    peer = torch.zeros(2, 4, 8, 256, 128, device="cuda", dtype=torch.bfloat16)
    block_map = torch.full((8,), -1, dtype=torch.int32, device="cuda")
    block_map[:] = torch.tensor([0, 1, 2, 3, 9, -1, -1, -1], dtype=torch.int32)  # block 4 -> 9: past 4 blocks
    target = PushTarget.of(peer.transpose(2, 3)[0], peer.transpose(2, 3)[1], None, block_map=block_map)
    word = transport.StatusWord()
    view = cache.transpose(2, 3)
    store_kvcache(key, value, view[0], view[1], slots, push_to=[target], status=word.address)
    torch.cuda.synchronize()
    hit = bool(((slots >= 4 * 256) & (slots < 5 * 256)).any())
    assert word.bits() == (2 if hit else 0)
    word.close()
    transport.device_error()
    expected = np.zeros(bits(peer).shape, dtype=np.uint16)
    s = slots.cpu().numpy()
    mapped = np.full_like(s, -1)
    table = block_map.cpu().numpy()
    for t, slot in enumerate(s.tolist()):
        if slot >= 0 and table[slot // 256] >= 0 and table[slot // 256] < 4:
            mapped[t] = table[slot // 256] * 256 + slot % 256
    ev = expected.swapaxes(2, 3)
    oracle_store(bits(key), bits(value), ev[0], ev[1], mapped)
    assert np.array_equal(bits(peer), expected)


def test_bad_arguments_raise_before_a_launch():
    key, value, cache, slots = _qwen_step(tokens=16, blocks=2)
    view = cache.transpose(2, 3)
    with pytest.raises(ValueError, match="slots for"):
        store_kvcache(key, value, view[0], view[1], slots[:5])
    with pytest.raises(TypeError):
        store_kvcache(key, value, view[0], view[1], slots.float())
    bad = PushTarget.of(view[0], view[1], slots, src_first_head=6, num_heads=4)
    from lean_vllm_b200._native import KvxRangeError

    with pytest.raises(KvxRangeError, match="heads"):
        store_kvcache(key, value, view[0], view[1], slots, push_to=[bad])


@pytest.mark.parametrize("serial", [False, True], ids=["programmatic", "plain"])
def test_chained_stores_see_what_the_kernels_before_them_wrote(serial):
    """Stores launch with programmatic stream serialization: each may be scheduled while the kernel before it
    drains, but reads nothing before that kernel has completed. A chain where every store reads the cache the
    previous store (or a torch kernel) just wrote must equal the same chain run one launch at a time."""
    from lean_vllm_b200._native import STORE_SERIAL

    flags = STORE_SERIAL if serial else 0
    g = torch.Generator(device="cuda").manual_seed(3)
    blocks, block, heads, dim, hops = 24, 16, 4, 128, 12
    tokens = blocks * block
    caches = [torch.zeros(2, blocks, block, heads, dim, dtype=torch.bfloat16, device="cuda") for _ in range(hops)]
    perms = [torch.randperm(tokens, device="cuda", generator=g) for _ in range(hops)]
    rows = torch.randn(tokens, heads, dim, device="cuda", generator=g).to(torch.bfloat16)
    key, value = rows * 2, rows - 1  # torch kernels right before the first store
    for hop in range(hops):
        store_kvcache(key, value, caches[hop][0], caches[hop][1], perms[hop], flags=flags)
        # The next hop's rows are this cache, as stored: token i of the flat (blocks * block) view.
        key, value = caches[hop][0].reshape(tokens, heads, dim), caches[hop][1].reshape(tokens, heads, dim)
    torch.cuda.synchronize()
    want_k, want_v = rows * 2, rows - 1
    for hop in range(hops):
        k = torch.empty_like(want_k)
        k[perms[hop]] = want_k
        v = torch.empty_like(want_v)
        v[perms[hop]] = want_v
        assert torch.equal(caches[hop][0].reshape(tokens, heads, dim), k), hop
        assert torch.equal(caches[hop][1].reshape(tokens, heads, dim), v), hop
        want_k, want_v = k, v


@pytest.mark.parametrize("head_dim", [128, 12], ids=["aligned", "unaligned"])
def test_rows_strided_across_tokens_store_like_contiguous_ones(head_dim):
    """Keys and values as views into a wider per-token tensor (a fused qkv output), with 16-byte vectors and, for a
    24-byte head row (12 bf16), 8-byte ones."""
    g = torch.Generator(device="cuda").manual_seed(9)
    tokens, heads, blocks, block = 777, 4, 16, 64
    qkv = torch.randn(tokens, 3 * heads, head_dim, generator=g, device="cuda").to(torch.bfloat16)
    key, value = qkv[:, heads : 2 * heads], qkv[:, 2 * heads :]
    assert key.stride(0) == 3 * heads * head_dim
    cache = torch.randn(2, blocks, heads, block, head_dim, generator=g, device="cuda").to(torch.bfloat16)
    slots = torch.randperm(blocks * block, generator=g, device="cuda")[:tokens]
    slots[3::50] = -1
    expected = bits(cache).copy()
    e_view = expected.swapaxes(2, 3)
    oracle_store(bits(key.contiguous()), bits(value.contiguous()), e_view[0], e_view[1], slots.cpu().numpy())
    view = cache.transpose(2, 3)
    store_kvcache(key, value, view[0], view[1], slots)
    torch.cuda.synchronize()
    assert np.array_equal(bits(cache), expected)


@pytest.mark.parametrize("block", [24, 64], ids=["block24", "block64"])
def test_block_sizes_that_are_not_powers_of_two_divide(block):
    """A 24-token block takes the general slot arithmetic (divide), a 64-token block the shift-and-mask one."""
    g = torch.Generator(device="cuda").manual_seed(21)
    tokens, heads, dim, blocks = 500, 2, 64, 30
    key = torch.randn(tokens, heads, dim, generator=g, device="cuda").to(torch.bfloat16)
    value = torch.randn(tokens, heads, dim, generator=g, device="cuda").to(torch.bfloat16)
    cache = torch.randn(2, blocks, heads, block, dim, generator=g, device="cuda").to(torch.bfloat16)
    slots = torch.randperm(blocks * block, generator=g, device="cuda")[:tokens]
    slots[::31] = -1
    expected = bits(cache).copy()
    e_view = expected.swapaxes(2, 3)
    oracle_store(bits(key), bits(value), e_view[0], e_view[1], slots.cpu().numpy())
    view = cache.transpose(2, 3)
    store_kvcache(key, value, view[0], view[1], slots)
    torch.cuda.synchronize()
    assert np.array_equal(bits(cache), expected)


def test_a_peers_only_store_writes_the_peers_and_not_the_local_cache():
    """KVX_STORE_PEERS_ONLY: destination 0's slots (and block map) still place the peers' rows, but destination 0
    itself is left as it was -- the push half of a store whose local half ran on the engine's stream."""
    from lean_vllm_b200._native import STORE_PEERS_ONLY

    key, value, cache, slots = _qwen_step(tokens=700)
    peer = torch.zeros(2, 40, 8, 256, 128, device="cuda", dtype=torch.bfloat16)  # room for every used block
    block_map = torch.full((40,), -1, dtype=torch.int32, device="cuda")
    used = torch.unique(slots[slots >= 0] // 256)
    block_map[used] = torch.arange(used.numel(), dtype=torch.int32, device="cuda")
    target = PushTarget.of(peer.transpose(2, 3)[0], peer.transpose(2, 3)[1], None, block_map=block_map)
    before = cache.clone()
    view = cache.transpose(2, 3)
    store_kvcache(key, value, view[0], view[1], slots, push_to=[target], flags=STORE_PEERS_ONLY)
    torch.cuda.synchronize()
    assert torch.equal(cache, before)
    # The oracle's store of the same rows into a host copy of the peer at the mapped slots.
    expected = np.zeros(bits(peer).shape, dtype=np.uint16)
    ev = expected.swapaxes(2, 3)
    table = block_map.cpu().numpy()
    s = slots.cpu().numpy()
    mapped = np.where(s >= 0, table[np.clip(s, 0, None) // 256].astype(np.int64) * 256 + s % 256, -1)
    oracle_store(bits(key), bits(value), ev[0], ev[1], mapped)
    assert np.array_equal(bits(peer), expected)


@pytest.mark.parametrize("tokens, heads, dim, block, layout, strided", [
    (8192, 8, 128, 256, "HND", False),  # a Qwen3-8B prefill step: full stages of 8 tokens
    (777, 8, 128, 256, "HND", False),   # a last stage with 1 token
    (300, 4, 128, 64, "NHD", False),    # NHD: a token's heads together, one bulk store per row
    (513, 2, 64, 16, "HND", True),      # rows strided across tokens (a fused qkv): one load per token
    (5, 8, 128, 256, "HND", False),     # fewer tokens than SMs
])
def test_the_store_matches_the_oracle_across_shapes(tokens, heads, dim, block, layout, strided):
    """The store on a Qwen3-8B prefill step, ragged token counts, NHD, rows strided across tokens and fewer tokens
    than SMs, each against the oracle's store on a host copy: padding slots skipped, everything else in place, the
    status word clear."""
    g = torch.Generator(device="cuda").manual_seed(tokens + heads)
    if strided:
        qkv = torch.randn(tokens, 3 * heads, dim, generator=g, device="cuda").to(torch.bfloat16)
        key, value = qkv[:, heads : 2 * heads], qkv[:, 2 * heads :]
    else:
        key = torch.randn(tokens, heads, dim, generator=g, device="cuda").to(torch.bfloat16)
        value = torch.randn(tokens, heads, dim, generator=g, device="cuda").to(torch.bfloat16)
    blocks = -(-tokens // block) + 3
    shape = (2, blocks, heads, block, dim) if layout == "HND" else (2, blocks, block, heads, dim)
    cache = torch.randn(*shape, generator=g, device="cuda").to(torch.bfloat16)
    slots = torch.randperm(blocks * block, generator=g, device="cuda")[:tokens]
    slots[::13] = -1
    expected = bits(cache).copy()
    ev = expected.swapaxes(2, 3) if layout == "HND" else expected
    oracle_store(bits(key.contiguous()), bits(value.contiguous()), ev[0], ev[1], slots.cpu().numpy())
    view = cache.transpose(2, 3) if layout == "HND" else cache
    word = transport.StatusWord()
    store_kvcache(key, value, view[0], view[1], slots, status=word.address)
    torch.cuda.synchronize()
    assert word.bits() == 0
    word.close()
    assert np.array_equal(bits(cache), expected)


def test_a_prefill_step_of_latents_stores_like_the_oracle():
    from oracle.kv_oracle import store_latents as oracle_latents

    g = torch.Generator(device="cuda").manual_seed(17)
    latent = torch.randn(2049, 576, generator=g, device="cuda").to(torch.bfloat16)
    cache = torch.randn(1, 40, 64, 576, generator=g, device="cuda").to(torch.bfloat16)
    slots = torch.randperm(40 * 64, generator=g, device="cuda")[:2049]
    slots[7::101] = -1
    expected = bits(cache).copy()
    oracle_latents(bits(latent), expected[0], slots.cpu().numpy())
    store_latents(latent, cache[0], slots)
    torch.cuda.synchronize()
    assert np.array_equal(bits(cache), expected)
