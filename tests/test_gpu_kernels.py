"""The kvx kernels through the C ABI, bit for bit against the reference's golden results and the CPU oracle.

Every comparison here is exact (torch.equal on bf16 bit patterns): the path moves bytes and must not change one.
"""

import numpy as np
import pytest
import torch

from lean_vllm_b200._native import ENGINE_LSU, ENGINE_TMA, KvxDeviceError, KvxError, KvxRangeError, flags
from lean_vllm_b200.kv_transfer import transport
from lean_vllm_b200.kv_transfer.shares import head_shares, split_heads
from lean_vllm_b200.kv_transfer.transport import CacheTable, CopyJob
from oracle.kv_oracle import load_between
from tests.helpers import bits, from_bits, full_of, rank_part, seeded, sha

pytestmark = pytest.mark.gpu

ENGINES = {"auto": 0, "lsu": flags(ENGINE_LSU), "tma": flags(ENGINE_TMA)}


def load_on_gpu(prefill_layers, decode_layers, prefill_tp, decode_tp, local, remote, engine_flags, device="cuda"):
    """Every decode rank pulls its shares from every prefill rank: one kvx_copy per decode rank, each job one
    share (nixl_connector.py:396-421). All ranks' caches live on one GPU here."""
    mla = prefill_layers[0].dim() == 4
    heads = split_heads(0 if mla else prefill_layers[0].shape[2], decode_tp, prefill_tp)
    producers = [[rank_part(layer, q, prefill_tp).to(device) for layer in prefill_layers] for q in range(prefill_tp)]
    consumers = [[rank_part(layer, r, decode_tp).to(device) for layer in decode_layers] for r in range(decode_tp)]
    tables = [CacheTable.from_tensors(p) for p in producers]
    moved = []
    for rank in range(decode_tp):
        local_table = CacheTable.from_tensors(consumers[rank])
        caches = [local_table] + tables
        jobs = [
            CopyJob(1 + s.remote_rank, 0, remote, local, s.remote_head, s.local_head, s.num_heads, latents=(i == 0))
            for i, s in enumerate(head_shares(rank, decode_tp, prefill_tp, heads))
        ]
        moved.append(transport.job_bytes(caches, jobs))
        transport.copy(caches, jobs, torch.cuda.current_stream().cuda_stream, engine_flags)
    torch.cuda.synchronize()
    return [[c.cpu() for c in layers] for layers in consumers], moved


@pytest.mark.parametrize("engine", list(ENGINES))
def test_every_small_case_matches_the_reference(golden, engine):
    meta, arrays = golden
    small = meta["small"]
    for case in small["cases"]:
        key = "lat" if case["mla"] else "kv"
        prefill = from_bits(arrays[f"small_{key}_prefill"])
        decode = from_bits(arrays[f"small_{key}_decode"])
        local, remote = case.get("local", small["local"]), case.get("remote", small["remote"])
        consumers, moved = load_on_gpu([prefill], [decode], case["prefill_tp"], case["decode_tp"], local, remote,
                                       ENGINES[engine])
        full = full_of([c[0] for c in consumers], case["mla"])
        assert np.array_equal(bits(full), arrays[case["name"]]), case["name"]
        assert moved == case["bytes_per_rank"], case["name"]


@pytest.mark.parametrize("engine", list(ENGINES))
@pytest.mark.parametrize("key", ["qwen_kv", "dsv2_lat"])
def test_model_shaped_cases_match_the_reference_digests(golden, key, engine):
    meta, _ = golden
    spec = meta[key]
    shape = tuple(spec["shape"])
    prefill = [seeded(shape, s) for s in spec["prefill_seeds"]]
    decode = [seeded(shape, s) for s in spec["decode_seeds"]]
    assert [sha(t) for t in prefill] == spec["input_sha256"]["prefill"]
    for case in spec["cases"]:
        consumers, moved = load_on_gpu(prefill, decode, case["prefill_tp"], case["decode_tp"], spec["local"],
                                       spec["remote"], ENGINES[engine])
        assert moved == case["bytes_per_rank"], case["name"]
        for layer in range(spec["layers"]):
            assert sha(full_of([c[layer] for c in consumers], case["mla"])) == case["layer_sha256"][layer]


def _odd_layers(mla, seed, blocks=9):
    """Shapes whose heads or latent blocks are not 16-byte multiples, so the kernel falls back to narrow vectors."""
    shape = (1, blocks, 5, 7) if mla else (2, blocks, 6, 5, 3)  # 70-byte latent blocks; 30-byte heads
    return [seeded(shape, seed + i) for i in range(3)]


@pytest.mark.parametrize("mla", [False, True], ids=["kv", "latents"])
@pytest.mark.parametrize("prefill_tp, decode_tp", [(1, 1), (2, 3), (3, 2), (1, 6)])
def test_unaligned_shapes_against_the_oracle(mla, prefill_tp, decode_tp):
    prefill, decode = _odd_layers(mla, 0), _odd_layers(mla, 10)
    local, remote = [8, 0, 4, 2], [1, 6, 0, 8]
    consumers, moved = load_on_gpu(prefill, decode, prefill_tp, decode_tp, local, remote, 0)
    expected, expected_moved = load_between([bits(t) for t in prefill], [bits(t) for t in decode], prefill_tp,
                                            decode_tp, local, remote)
    assert moved == expected_moved
    for rank in range(decode_tp):
        for layer in range(3):
            assert np.array_equal(bits(consumers[rank][layer]), expected[rank][layer]), (rank, layer)


def _qwen_like(num_blocks, layers, heads=8, seed=0, device="cuda"):
    g = torch.Generator(device=device).manual_seed(seed)
    return [torch.randn(2, num_blocks, heads, 256, 128, generator=g, device=device).to(torch.bfloat16)
            for _ in range(layers)]


@pytest.mark.parametrize("engine", list(ENGINES))
def test_a_many_request_batch_in_one_call_matches_torch_indexing(engine):
    """64 requests of random lengths, one job each, shuffled block tables; the result must equal torch's own index
    copy, and every block no request names must keep its bytes."""
    rng = np.random.default_rng(0)
    num_blocks, layers = 160, 3
    src, dst = _qwen_like(num_blocks, layers, seed=1), _qwen_like(num_blocks, layers, seed=2)
    before = [d.clone() for d in dst]
    lengths = rng.integers(1, 5, size=64)
    free_src, free_dst = rng.permutation(num_blocks), rng.permutation(num_blocks)
    jobs, at = [], 0
    for n in lengths:
        if at + n > num_blocks:
            break
        jobs.append(CopyJob(0, 1, free_src[at : at + n], free_dst[at : at + n], 0, 0, 8))
        at += n
    caches = [CacheTable.from_tensors(src), CacheTable.from_tensors(dst)]
    transport.copy(caches, jobs, torch.cuda.current_stream().cuda_stream, ENGINES[engine])
    torch.cuda.synchronize()
    s_ids = torch.tensor(np.concatenate([j.src_block_ids for j in jobs]), device="cuda", dtype=torch.long)
    d_ids = torch.tensor(np.concatenate([j.dst_block_ids for j in jobs]), device="cuda", dtype=torch.long)
    untouched = torch.ones(num_blocks, dtype=torch.bool, device="cuda")
    untouched[d_ids] = False
    for layer in range(layers):
        assert torch.equal(dst[layer][:, d_ids], src[layer][:, s_ids])
        assert torch.equal(dst[layer][:, untouched], before[layer][:, untouched])


def test_more_jobs_and_blocks_than_one_launch_holds():
    """Past the launch's capacity (96 job pieces, 1536 blocks a piece) the library splits into several launches."""
    num_blocks, layers = 2000, 2
    src = [torch.randn(2, num_blocks, 1, 16, 8, device="cuda").to(torch.bfloat16) for _ in range(layers)]
    dst = [torch.zeros_like(s) for s in src]  # 150 small jobs land here, on disjoint blocks
    big = [torch.zeros_like(s) for s in src]  # one 1700-block job lands here
    perm = torch.randperm(num_blocks).numpy()
    jobs = [CopyJob(0, 1, perm[k * 10 : (k + 1) * 10], np.arange(k * 10, (k + 1) * 10), 0, 0, 1) for k in range(150)]
    jobs.append(CopyJob(0, 2, perm[:1700], perm[::-1][:1700].copy(), 0, 0, 1))
    caches = [CacheTable.from_tensors(t) for t in (src, dst, big)]
    before = transport.launch_count()
    transport.copy(caches, jobs, 0, 0)
    torch.cuda.synchronize()
    assert transport.launch_count() - before >= 3
    expect = {1: [torch.zeros_like(s) for s in src], 2: [torch.zeros_like(s) for s in src]}
    for job in jobs:
        for layer in range(layers):
            expect[job.dst][layer][:, torch.as_tensor(job.dst_block_ids, dtype=torch.long)] = src[layer][
                :, torch.as_tensor(job.src_block_ids, dtype=torch.long)]
    for layer in range(layers):
        assert torch.equal(dst[layer], expect[1][layer])
        assert torch.equal(big[layer], expect[2][layer])


@pytest.mark.parametrize("layers, n_jobs, blocks_per_job", [(40, 8, 16), (41, 8, 16), (40, 9, 14), (40, 8, 17)])
@pytest.mark.parametrize("engine", ["lsu", "tma"])
def test_launches_at_and_past_the_compact_parameter_block_match_torch_indexing(layers, n_jobs, blocks_per_job,
                                                                             engine):
    """A launch that fits the compact parameter block (8 jobs, 160 region slots, 256 block ids) goes out with it;
    one region, job or id more and it takes the full block. Both sides of each limit land what torch indexing of the
    source says, and leave every other block alone."""
    rng = np.random.default_rng(layers * 100 + n_jobs * 10 + blocks_per_job)
    num_blocks = n_jobs * blocks_per_job + 4
    g = torch.Generator(device="cuda").manual_seed(9)
    src = [torch.randn(2, num_blocks, 2, 16, 64, generator=g, device="cuda").to(torch.bfloat16) for _ in range(layers)]
    dst = [torch.randn(2, num_blocks, 2, 16, 64, generator=g, device="cuda").to(torch.bfloat16) for _ in range(layers)]
    before = [d.clone() for d in dst]
    src_order, dst_order = rng.permutation(num_blocks), rng.permutation(num_blocks)
    b = blocks_per_job
    fixed = [([int(x) for x in src_order[j * b : (j + 1) * b]], [int(x) for x in dst_order[j * b : (j + 1) * b]])
             for j in range(n_jobs)]  # each job its own destinations
    jobs = [CopyJob(1, 0, s_ids, d_ids, 0, 0, 2) for s_ids, d_ids in fixed]
    caches = [CacheTable.from_tensors(dst), CacheTable.from_tensors(src)]
    transport.copy(caches, jobs, torch.cuda.current_stream().cuda_stream, ENGINES[engine])
    torch.cuda.synchronize()
    for s_layer, d_layer, old in zip(src, dst, before):
        expected = old.clone()
        for s_ids, d_ids in fixed:
            expected[:, d_ids] = s_layer[:, s_ids]
        assert torch.equal(d_layer, expected)


def test_out_of_range_blocks_and_heads_raise_before_any_launch():
    src = [torch.zeros(2, 4, 2, 16, 8, device="cuda", dtype=torch.bfloat16)]
    dst = [torch.zeros(2, 4, 2, 16, 8, device="cuda", dtype=torch.bfloat16)]
    caches = [CacheTable.from_tensors(src), CacheTable.from_tensors(dst)]
    before = transport.launch_count()
    with pytest.raises(KvxRangeError, match="outside the cache"):
        transport.copy(caches, [CopyJob(0, 1, [4], [0], 0, 0, 2)])
    with pytest.raises(KvxRangeError, match="outside the cache"):
        transport.copy(caches, [CopyJob(0, 1, [0], [-1], 0, 0, 2)])
    with pytest.raises(KvxRangeError, match="pass the end of a block"):
        transport.copy(caches, [CopyJob(0, 1, [0], [0], 1, 0, 2)])
    with pytest.raises(KvxError, match="latent on one side only"):
        lat = CacheTable.from_tensors([torch.zeros(1, 4, 16, 16, device="cuda", dtype=torch.bfloat16)] * 2)
        transport.copy([caches[0], lat], [CopyJob(0, 1, [0], [0], 0, 0, 1)])
    assert transport.launch_count() == before


def test_empty_jobs_launch_nothing():
    src = [torch.zeros(2, 4, 2, 16, 8, device="cuda", dtype=torch.bfloat16)]
    caches = [CacheTable.from_tensors(src), CacheTable.from_tensors([torch.ones_like(src[0])])]
    before = transport.launch_count()
    transport.copy(caches, [CopyJob(0, 1, [], [], 0, 0, 2), CopyJob(0, 1, [1], [2], 0, 0, 0)])
    assert transport.launch_count() == before


@pytest.mark.parametrize("engine", list(ENGINES))
def test_pack_push_scatter_lands_what_torch_indexing_of_the_source_says(engine):
    """Gather into a staging buffer, push it to a second buffer, scatter into the destination's blocks. The staging
    buffer must hold the rows in block_descs order and the destination must equal torch indexing of the source
    (`dst[:, d_ids, 2:4] = src[:, s_ids, 1:3]`, the reference tests' closed form): no kvx kernel computes what is
    expected. Untouched blocks and heads keep their values."""
    f = ENGINES[engine]
    src = _qwen_like(24, 2, heads=4, seed=3)
    dst = _qwen_like(24, 2, heads=4, seed=4)
    s_ids, d_ids = [5, 17, 2, 9], [0, 23, 11, 6]
    expected = [d.clone() for d in dst]
    for e, s in zip(expected, src):
        e[:, d_ids, 2:4] = s[:, s_ids, 1:3]
    src_t, dst_t = CacheTable.from_tensors(src), CacheTable.from_tensors(dst)
    chunk = 2 * 256 * 128 * 2
    staging = torch.empty(4 * len(s_ids) * chunk, dtype=torch.uint8, device="cuda")
    landing = torch.empty_like(staging)
    transport.pack(src_t, s_ids, 1, 2, False, staging.data_ptr(), staging.numel(), 0, f)
    transport.push(landing.data_ptr(), staging.data_ptr(), staging.numel(), 0, f)
    transport.scatter(landing.data_ptr(), landing.numel(), dst_t, d_ids, 2, 2, False, 0, f)
    torch.cuda.synchronize()
    for layer in range(2):
        assert torch.equal(dst[layer], expected[layer])
    rows = landing.view(torch.bfloat16).view(4, len(s_ids), 2, 256, 128)  # (region, block, head, token, dim)
    for r in range(4):
        layer, part = divmod(r, 2)
        assert torch.equal(rows[r], src[layer][part][s_ids, 1:3])


@pytest.mark.parametrize("latents", [False, True], ids=["kv", "latent"])
def test_scatter_alone_matches_the_oracle_s_placement(latents):
    """kvx_scatter from a staging buffer filled by torch (not by kvx_pack) in block_descs row order, against the
    oracle's placement on host copies: the scatter is pinned by itself, not through another kvx kernel."""
    import oracle.kv_oracle as oracle

    g = torch.Generator().manual_seed(11)
    if latents:
        dst = [torch.randn(1, 20, 64, 576, generator=g).to(torch.bfloat16) for _ in range(3)]
        first, count = 0, 0
    else:
        dst = [torch.randn(2, 20, 4, 32, 64, generator=g).to(torch.bfloat16) for _ in range(3)]
        first, count = 1, 2
    ids = [19, 0, 7, 3, 12]
    regions = [part for layer in dst for part in layer]
    chunk_shape = regions[0][0].shape if latents else regions[0][0, first : first + count].shape
    rows = torch.randn(len(regions), len(ids), *chunk_shape, generator=g).to(torch.bfloat16)
    expected = [bits(d).copy() for d in dst]
    for r, region_rows in enumerate(rows):
        layer, part = divmod(r, len(dst[0]))
        oracle.place_rows(expected[layer][part], ids, bits(region_rows), first, count, latents)
    on_gpu = [d.cuda() for d in dst]
    staging = rows.cuda().contiguous()
    transport.scatter(staging.data_ptr(), staging.numel() * 2, CacheTable.from_tensors(on_gpu), ids, first, count,
                      latents)
    torch.cuda.synchronize()
    for got, want in zip(on_gpu, expected):
        assert np.array_equal(bits(got), want)


def test_a_staging_buffer_too_small_is_refused():
    src = CacheTable.from_tensors([torch.zeros(2, 4, 2, 16, 8, device="cuda", dtype=torch.bfloat16)])
    staging = torch.empty(1024, dtype=torch.uint8, device="cuda")
    with pytest.raises(KvxRangeError, match="staging needs"):
        transport.pack(src, [0, 1, 2], 0, 2, False, staging.data_ptr(), staging.numel())


def test_a_transfer_waits_for_its_ready_event_and_reports_completion():
    """The load waits on the stream for the event recorded where the blocks were allocated (the reference's
    ready.synchronize, nixl_connector.py:266, 394-395), then reports done through its own event."""
    src = _qwen_like(8, 2, seed=5)
    dst = [torch.zeros_like(s) for s in src]
    side = torch.cuda.Stream()
    main = torch.cuda.current_stream()
    torch.cuda._sleep(20_000_000)  # the "step in flight" that still owns dst's blocks
    for d in dst:
        d.fill_(1.0)  # ... and writes them after the sleep
    ready = main.record_event()
    xfer = transport.transfer([CacheTable.from_tensors(src), CacheTable.from_tensors(dst)],
                              [CopyJob(0, 1, [1, 2], [3, 4], 0, 0, 8)], side.cuda_stream, ready.cuda_event)
    while not xfer.done():
        pass
    xfer.release()
    for s, d in zip(src, dst):
        assert torch.equal(d[:, [3, 4]], s[:, [1, 2]])
        assert bool((d[:, [0, 1, 2, 5, 6, 7]] == 1.0).all())


@pytest.mark.parametrize("on_default_stream", [False, True])
def test_a_transfer_after_a_stream_waits_for_what_was_queued_there(on_default_stream):
    """kvx_transfer_after: no ready event from the caller; the library's own event, recorded on the engine's stream,
    orders the copy after the writes queued there -- on a stream of the engine's or the legacy default stream (0),
    and again for a second transfer reusing the same event while the first still waits."""
    src = _qwen_like(8, 2, seed=6)
    dst = [torch.zeros_like(s) for s in src]
    side = torch.cuda.Stream()
    engine = torch.cuda.default_stream() if on_default_stream else torch.cuda.Stream()
    caches = [CacheTable.from_tensors(src), CacheTable.from_tensors(dst)]
    with torch.cuda.stream(engine):
        torch.cuda._sleep(20_000_000)  # the "step in flight" that still owns dst's blocks
        for d in dst:
            d.fill_(1.0)  # ... and writes them after the sleep
        first = transport.transfer(caches, [CopyJob(0, 1, [1, 2], [3, 4], 0, 0, 8)], side.cuda_stream,
                                   after_stream=engine.cuda_stream)
        torch.cuda._sleep(20_000_000)
        for d in dst:
            d[:, [6]] = 2.0
        second = transport.transfer(caches, [CopyJob(0, 1, [5], [6], 0, 0, 8)], side.cuda_stream,
                                    after_stream=engine.cuda_stream)
    while not (first.done() and second.done()):
        pass
    first.release()
    second.release()
    torch.cuda.synchronize()
    for s, d in zip(src, dst):
        assert torch.equal(d[:, [3, 4]], s[:, [1, 2]])
        assert torch.equal(d[:, [6]], s[:, [5]])
        assert bool((d[:, [0, 1, 2, 5, 7]] == 1.0).all())


def test_a_doorbell_rings_once_the_stream_work_before_it_ends():
    """kvx_doorbell_ring_after: the eventfd turns readable only after the copy queued before the ring landed."""
    import select

    src = _qwen_like(8, 2, seed=6)
    dst = [torch.zeros_like(s) for s in src]
    bell = transport.Doorbell()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(50_000_000)  # tens of ms at B200 clocks
    xfer = transport.transfer([CacheTable.from_tensors(src), CacheTable.from_tensors(dst)],
                              [CopyJob(0, 1, [1, 2], [3, 4], 0, 0, 8)], stream.cuda_stream)
    bell.ring_after(stream.cuda_stream)
    assert select.select([bell.fd], [], [], 0)[0] == []  # the sleep still runs
    assert select.select([bell.fd], [], [], 10.0)[0] == [bell.fd]
    assert xfer.done()  # the ring came after the copy's completion event
    bell.clear()
    assert select.select([bell.fd], [], [], 0)[0] == []
    xfer.release()
    bell.close()
    for s, d in zip(src, dst):
        assert torch.equal(d[:, [3, 4]], s[:, [1, 2]])


def test_ipc_export_and_open_in_the_same_process_is_the_pointer_itself():
    t = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    view = t[4096:]
    blob = transport.export(view.data_ptr())
    assert transport.open_mapping(blob) == view.data_ptr()
    transport.close_mapping(blob)


def test_the_device_error_word_starts_clear():
    assert transport.device_error() == 0


def test_a_bounded_wait_that_runs_out_reports_and_leaves_the_context_usable():
    """The failure path every TMA copy relies on, made to happen: an mbarrier waited on for bytes that never come
    gives up after its limit and leaves code 4 in the device word; the device then copies as before."""
    import time

    assert transport.device_error() == 0
    started = time.monotonic()
    transport.wait_selftest(20_000)  # 20 ms
    torch.cuda.synchronize()
    assert time.monotonic() - started < 5
    assert transport.device_error() == 4
    assert transport.device_error() == 0  # read and cleared
    src = _qwen_like(4, 1, seed=8)
    dst = [torch.zeros_like(s) for s in src]
    transport.copy([CacheTable.from_tensors(src), CacheTable.from_tensors(dst)], [CopyJob(0, 1, [1, 2], [0, 3], 0, 0, 8)])
    torch.cuda.synchronize()
    assert torch.equal(dst[0][:, [0, 3]], src[0][:, [1, 2]])


def test_a_copy_that_gave_up_fails_its_own_transfer_and_no_other():
    """A TMA copy whose bounded wait ran out ends with its bytes not all landed, and only its status word says so.
    The self-test writes that bit (1) into transfer B's word without copying anything: B's check fails, while A
    (posted before, on the same device and stream) and C (posted after) report their bytes landed -- with no call
    that clears anything in between. The device's diagnostic word saw the bit too, and reading it changes no
    transfer's result."""
    src = _qwen_like(4, 1, seed=9)
    dsts = [[torch.zeros_like(s) for s in src] for _ in range(3)]
    stream = torch.cuda.current_stream().cuda_stream
    assert transport.device_error() == 0
    xfers = []
    for k, dst in enumerate(dsts):
        xfers.append(transport.transfer([CacheTable.from_tensors(src), CacheTable.from_tensors(dst)],
                                        [CopyJob(0, 1, [1, 2], [0, 3], 0, 0, 8)], stream))
        if k == 1:
            transport.wait_selftest(20_000, code=1, stream=stream, status=xfers[1].status_address())  # 20 ms
    torch.cuda.synchronize()
    assert xfers[0].done()
    with pytest.raises(KvxDeviceError, match="gave up a bounded wait"):
        xfers[1].done()
    assert xfers[2].done()
    assert transport.device_error() == 1
    assert xfers[2].done() and xfers[0].done()  # judged by their own words, before and after the read
    for xfer in xfers:
        xfer.release()
    for dst in dsts:
        assert torch.equal(dst[0][:, [0, 3]], src[0][:, [1, 2]])


def test_status_words_start_clear_and_come_back_clear():
    """A word handed out again after a failure starts at zero: a new transfer never inherits an old one's bits."""
    word = transport.StatusWord()
    stream = torch.cuda.current_stream().cuda_stream
    transport.wait_selftest(1_000, code=1, stream=stream, status=word.address)
    torch.cuda.synchronize()
    assert word.bits() == 1
    assert transport.device_error() == 1
    word.close()
    words = [transport.StatusWord() for _ in range(64)]  # the pool hands the freed word out again, zeroed
    assert all(w.bits() == 0 for w in words)
    for w in words:
        w.close()
