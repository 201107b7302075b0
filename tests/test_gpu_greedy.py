"""Greedy decode after a transfer is token-identical to a colocated run.

The reference checks this with a real Qwen3 checkpoint through two engines (tests/test_disagg_e2e.py:94-124); there
is no checkpoint or reference engine on the GPU box, so this runs a tiny random-init decoder (Qwen3-like: RMSNorm,
GQA attention over an HND paged KV cache, SwiGLU) whose prefill writes its KV with the kvx store kernel. The prompt's
blocks then move to a decode instance's cache -- other block ids, TP1 -> TP2 head split -- through
CudaIpcConnector, and greedy decoding from the moved blocks must pick the same tokens as decoding in place. The
splits cover TP1 -> TP1, TP1 -> TP2 and the benchmark's heterogeneous TP2 -> TP4, an MLA model whose cache holds
latents (replicated to every decode rank), and a control where one decode rank misses its share.
"""

import math

import pytest
import torch

from lean_vllm_b200.attention.kvx_cache import store_kvcache, store_latents
from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVOutputAggregator, KVTransferConfig, ReqToRecv
from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker
from tests.connector_cases import WorkerConfig, free_port, wait_for

pytestmark = pytest.mark.gpu

VOCAB, HIDDEN, HEADS, KV_HEADS, HEAD_DIM, LAYERS, BLOCK = 512, 256, 8, 4, 32, 3, 16


class TinyDecoder:
    """Random-init decoder; its KV lives in per-layer HND caches (2, blocks, kv heads, BLOCK, HEAD_DIM)."""

    def __init__(self, seed=0, kv_heads=KV_HEADS):
        self.kv_heads = kv_heads
        g = torch.Generator(device="cuda").manual_seed(seed)

        def w(*shape):
            return (torch.randn(*shape, generator=g, device="cuda") / math.sqrt(shape[0])).to(torch.bfloat16)

        self.embed = w(VOCAB, HIDDEN) * 8
        self.layers = [dict(qkv=w(HIDDEN, (HEADS + 2 * kv_heads) * HEAD_DIM), o=w(HEADS * HEAD_DIM, HIDDEN),
                            up=w(HIDDEN, 2 * 4 * HIDDEN), down=w(4 * HIDDEN, HIDDEN)) for _ in range(LAYERS)]
        self.head = w(HIDDEN, VOCAB)

    @staticmethod
    def norm(x):
        x32 = x.float()
        return (x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype)

    def forward(self, tokens, positions, caches, block_table, cache_len):
        """One step over `tokens` at `positions`: store their KV, attend causally over the whole cached prefix."""
        x = self.embed[tokens]
        slots = torch.tensor([block_table[p // BLOCK] * BLOCK + p % BLOCK for p in positions.tolist()],
                             device="cuda")
        for layer, cache in zip(self.layers, caches):
            h = self.norm(x)
            kvh = self.kv_heads
            q, k, v = (h @ layer["qkv"]).split([HEADS * HEAD_DIM, kvh * HEAD_DIM, kvh * HEAD_DIM], -1)
            q = q.view(-1, HEADS, HEAD_DIM)
            k = k.reshape(-1, kvh, HEAD_DIM).contiguous()
            v = v.reshape(-1, kvh, HEAD_DIM).contiguous()
            view = cache.transpose(2, 3)  # (2, blocks, tokens, heads, dim)
            store_kvcache(k, v, view[0], view[1], slots)
            # Gather the sequence's keys/values from its blocks, then causal attention (GQA).
            n_blocks = -(-cache_len // BLOCK)
            ids = torch.tensor(block_table[:n_blocks], device="cuda")
            keys = view[0][ids].reshape(-1, kvh, HEAD_DIM)[:cache_len]
            values = view[1][ids].reshape(-1, kvh, HEAD_DIM)[:cache_len]
            keys = keys.repeat_interleave(HEADS // kvh, 1).transpose(0, 1)
            values = values.repeat_interleave(HEADS // kvh, 1).transpose(0, 1)
            mask = positions[:, None] >= torch.arange(cache_len, device="cuda")[None, :]
            attn = torch.nn.functional.scaled_dot_product_attention(q.transpose(0, 1), keys, values,
                                                                    attn_mask=mask)
            x = x + attn.transpose(0, 1).reshape(-1, HEADS * HEAD_DIM) @ layer["o"]
            gate, up = (self.norm(x) @ layer["up"]).chunk(2, -1)
            x = x + (torch.nn.functional.silu(gate) * up) @ layer["down"]
        return self.norm(x) @ self.head

    def greedy(self, caches, block_table, prompt_len, first_token, steps):
        out, token = [], first_token
        for i in range(steps):
            pos = prompt_len + i
            logits = self.forward(torch.tensor([token], device="cuda"), torch.tensor([pos], device="cuda"), caches,
                                  block_table, pos + 1)
            token = int(logits[-1].argmax())
            out.append(token)
        return out


def cache(blocks, heads=KV_HEADS):
    return [torch.zeros(2, blocks, heads, BLOCK, HEAD_DIM, device="cuda", dtype=torch.bfloat16)
            for _ in range(LAYERS)]


def move(prefill_rank_caches, decode_rank_caches, prefill_table, decode_table, prompt_blocks, skip_rank=None):
    """Loads the prompt's blocks from every prefill rank into every decode rank through CudaIpcConnector (each
    decode rank takes its head shares; latents whole). `skip_rank` leaves one decode rank without its load."""
    port = free_port()
    prefill_tp, decode_tp = len(prefill_rank_caches), len(decode_rank_caches)
    workers, producers, consumers = [], [], []
    try:
        for rank, caches in enumerate(prefill_rank_caches):
            w = CudaIpcConnectorWorker(WorkerConfig(KVTransferConfig(kv_role="kv_producer", kv_port=port,
                                                                     engine_id="p"), prefill_tp, BLOCK), rank)
            w.register_kv_caches(caches)
            workers.append(w)
            producers.append(w)
        for rank, caches in enumerate(decode_rank_caches):
            w = CudaIpcConnectorWorker(WorkerConfig(KVTransferConfig(kv_role="kv_consumer", engine_id="d"),
                                                    decode_tp, BLOCK), rank)
            w.register_kv_caches(caches)
            workers.append(w)
            consumers.append(w)
        for w in producers:
            w.start_load_kv(KVConnectorMetadata(reqs_to_send={"r": prefill_table[:prompt_blocks]}))
        loading = [c for rank, c in enumerate(consumers) if rank != skip_rank]
        for c in loading:
            c.start_load_kv(KVConnectorMetadata(reqs_to_recv={"r": ReqToRecv(
                decode_table[:prompt_blocks], prefill_table[:prompt_blocks], "r", "p", "127.0.0.1", port,
                prefill_tp)}))
        outputs = [wait_for(c) for c in loading]
        assert KVOutputAggregator(len(loading)).aggregate(outputs).finished_recving == {"r"}
    finally:
        for w in workers:
            w.shutdown()


def split_heads_of(caches, tp):
    """One TP rank's contiguous slice of every layer's KV heads (HND), as a TP engine's rank holds its cache."""
    per = caches[0].size(2) // tp
    return [[c[:, :, r * per : (r + 1) * per].contiguous() for c in caches] for r in range(tp)]


@pytest.mark.parametrize("prefill_tp, decode_tp", [(1, 1), (1, 2), (2, 4)], ids=["tp1-tp1", "tp1-tp2", "tp2-tp4"])
def test_greedy_decode_after_a_transfer_is_token_identical(prefill_tp, decode_tp):
    """The prefill's cache is split over prefill_tp ranks as a TP engine holds it, moved to decode_tp ranks with
    head resharding (TP2 -> TP4 is the benchmark's heterogeneous split: each decode rank takes 2 of 8 KV heads from
    one prefill rank), and decoding from the moved blocks picks the colocated run's tokens."""
    model = TinyDecoder(kv_heads=8)
    g = torch.Generator().manual_seed(1)
    prompt_len = 150  # 10 blocks, the last one partly filled
    prompt = torch.randint(0, VOCAB, (prompt_len,), generator=g).cuda()
    n_blocks = -(-(prompt_len + 40) // BLOCK)
    prefill_table = torch.randperm(40, generator=g)[:n_blocks].tolist()
    decode_table = torch.randperm(48, generator=g)[:n_blocks].tolist()

    prefill_caches = cache(40, 8)
    logits = model.forward(prompt, torch.arange(prompt_len, device="cuda"), prefill_caches, prefill_table, prompt_len)
    first = int(logits[-1].argmax())
    decode_rank_caches = [cache(48, 8 // decode_tp) for _ in range(decode_tp)]
    move(split_heads_of(prefill_caches, prefill_tp), decode_rank_caches, prefill_table, decode_table,
         -(-prompt_len // BLOCK))
    decode_caches = [torch.cat([decode_rank_caches[r][layer] for r in range(decode_tp)], dim=2)
                     for layer in range(LAYERS)]  # every decode rank's heads, as one TP1 cache

    colocated = model.greedy(prefill_caches, prefill_table, prompt_len, first, 24)
    disaggregated = model.greedy(decode_caches, decode_table, prompt_len, first, 24)
    assert colocated == disaggregated
    assert len(set(colocated)) > 1  # a real decode, not one token repeated


def test_a_dropped_share_changes_the_tokens():
    """The check's control: TP2 -> TP4 with decode rank 3 never loading its share (its two KV heads stay zero). The
    decode then differs from the colocated run, so token identity above means every share landed."""
    model = TinyDecoder(kv_heads=8)
    g = torch.Generator().manual_seed(1)
    prompt_len = 150
    prompt = torch.randint(0, VOCAB, (prompt_len,), generator=g).cuda()
    n_blocks = -(-(prompt_len + 40) // BLOCK)
    prefill_table = torch.randperm(40, generator=g)[:n_blocks].tolist()
    decode_table = torch.randperm(48, generator=g)[:n_blocks].tolist()
    prefill_caches = cache(40, 8)
    logits = model.forward(prompt, torch.arange(prompt_len, device="cuda"), prefill_caches, prefill_table, prompt_len)
    first = int(logits[-1].argmax())
    decode_rank_caches = [cache(48, 2) for _ in range(4)]
    move(split_heads_of(prefill_caches, 2), decode_rank_caches, prefill_table, decode_table,
         -(-prompt_len // BLOCK), skip_rank=3)
    decode_caches = [torch.cat([decode_rank_caches[r][layer] for r in range(4)], dim=2) for layer in range(LAYERS)]
    colocated = model.greedy(prefill_caches, prefill_table, prompt_len, first, 24)
    assert model.greedy(decode_caches, decode_table, prompt_len, first, 24) != colocated


LATENT, ROPE = 64, 16  # an MLA layer's cached latent per token: c_kv (LATENT) and k_pe (ROPE), 160 bytes in bf16


class TinyLatentDecoder(TinyDecoder):
    """A random-init decoder with multi-head latent attention (DeepSeek-V2-like): per token each layer caches one
    latent row [c_kv | k_pe] in a (1, blocks, BLOCK, LATENT + ROPE) cache, whole on every rank; keys and values of
    every head are expanded from it at attention time."""

    def __init__(self, seed=0):
        super().__init__(seed=seed, kv_heads=1)
        g = torch.Generator(device="cuda").manual_seed(seed + 7)

        def w(*shape):
            return (torch.randn(*shape, generator=g, device="cuda") / math.sqrt(shape[0])).to(torch.bfloat16)

        for layer in self.layers:
            layer.update(q=w(HIDDEN, HEADS * (HEAD_DIM + ROPE)), latent=w(HIDDEN, LATENT + ROPE),
                         uk=w(LATENT, HEADS * HEAD_DIM), uv=w(LATENT, HEADS * HEAD_DIM))

    def forward(self, tokens, positions, caches, block_table, cache_len):
        x = self.embed[tokens]
        slots = torch.tensor([block_table[p // BLOCK] * BLOCK + p % BLOCK for p in positions.tolist()],
                             device="cuda")
        for layer, cache in zip(self.layers, caches):
            h = self.norm(x)
            q = (h @ layer["q"]).view(-1, HEADS, HEAD_DIM + ROPE)
            store_latents((h @ layer["latent"]).contiguous(), cache[0], slots)
            n_blocks = -(-cache_len // BLOCK)
            ids = torch.tensor(block_table[:n_blocks], device="cuda")
            rows = cache[0][ids].reshape(-1, LATENT + ROPE)[:cache_len]
            c_kv, k_pe = rows[:, :LATENT], rows[:, LATENT:]
            keys = torch.cat([(c_kv @ layer["uk"]).view(-1, HEADS, HEAD_DIM),
                              k_pe[:, None, :].expand(-1, HEADS, ROPE)], -1).transpose(0, 1)
            values = torch.cat([(c_kv @ layer["uv"]).view(-1, HEADS, HEAD_DIM),
                                torch.zeros(cache_len, HEADS, ROPE, device="cuda", dtype=x.dtype)], -1).transpose(0, 1)
            mask = positions[:, None] >= torch.arange(cache_len, device="cuda")[None, :]
            attn = torch.nn.functional.scaled_dot_product_attention(q.transpose(0, 1), keys, values, attn_mask=mask)
            x = x + attn.transpose(0, 1)[..., :HEAD_DIM].reshape(-1, HEADS * HEAD_DIM) @ layer["o"]
            gate, up = (self.norm(x) @ layer["up"]).chunk(2, -1)
            x = x + (torch.nn.functional.silu(gate) * up) @ layer["down"]
        return self.norm(x) @ self.head


def latent_cache(blocks):
    return [torch.zeros(1, blocks, BLOCK, LATENT + ROPE, device="cuda", dtype=torch.bfloat16) for _ in range(LAYERS)]


def test_greedy_decode_after_a_latent_transfer_is_token_identical_on_every_decode_rank():
    """MLA: prefill TP1 -> decode TP2, latents replicated whole to both decode ranks; decoding from either rank's
    moved latents picks the colocated run's tokens."""
    model = TinyLatentDecoder()
    g = torch.Generator().manual_seed(2)
    prompt_len = 170
    prompt = torch.randint(0, VOCAB, (prompt_len,), generator=g).cuda()
    n_blocks = -(-(prompt_len + 40) // BLOCK)
    prefill_table = torch.randperm(40, generator=g)[:n_blocks].tolist()
    decode_table = torch.randperm(48, generator=g)[:n_blocks].tolist()
    prefill_caches = latent_cache(40)
    logits = model.forward(prompt, torch.arange(prompt_len, device="cuda"), prefill_caches, prefill_table, prompt_len)
    first = int(logits[-1].argmax())
    decode_rank_caches = [latent_cache(48) for _ in range(2)]
    move([prefill_caches], decode_rank_caches, prefill_table, decode_table, -(-prompt_len // BLOCK))
    colocated = model.greedy(prefill_caches, prefill_table, prompt_len, first, 24)
    assert len(set(colocated)) > 1
    for rank_caches in decode_rank_caches:
        assert model.greedy([c.clone() for c in rank_caches], decode_table, prompt_len, first, 24) == colocated
