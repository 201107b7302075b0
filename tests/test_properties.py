"""Properties the connector's arithmetic must keep for every size, checked over generated cases (hypothesis):
head shares tile each consumer rank's heads exactly once from the right producer heads, readers count the same
overlaps from the other side, relay parts partition a load's blocks, and per-layer save spans leave every block
pushed in its final state once the prompt is done -- whatever the chunking."""

from hypothesis import given, settings
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
