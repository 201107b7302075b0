"""Greedy decode after a transfer is token-identical to a colocated run.

The reference checks this with a real Qwen3 checkpoint through two engines (tests/test_disagg_e2e.py:94-124); there
is no checkpoint or reference engine on the GPU box, so this runs a tiny random-init decoder (Qwen3-like: RMSNorm,
GQA attention over an HND paged KV cache, SwiGLU) whose prefill writes its KV with the kvx store kernel. The prompt's
blocks then move to a decode instance's cache -- other block ids, TP1 -> TP2 head split -- through
CudaIpcConnector, and greedy decoding from the moved blocks must pick the same tokens as decoding in place.
"""

import math

import pytest
import torch

from lean_vllm_b200.attention.kvx_cache import store_kvcache
from lean_vllm_b200.kv_transfer import KVConnectorMetadata, KVOutputAggregator, KVTransferConfig, ReqToRecv
from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorWorker
from tests.connector_cases import WorkerConfig, free_port, wait_for

pytestmark = pytest.mark.gpu

VOCAB, HIDDEN, HEADS, KV_HEADS, HEAD_DIM, LAYERS, BLOCK = 512, 256, 8, 4, 32, 3, 16


class TinyDecoder:
    """Random-init decoder; its KV lives in per-layer HND caches (2, blocks, kv heads, BLOCK, HEAD_DIM)."""

    def __init__(self, seed=0):
        g = torch.Generator(device="cuda").manual_seed(seed)

        def w(*shape):
            return (torch.randn(*shape, generator=g, device="cuda") / math.sqrt(shape[0])).to(torch.bfloat16)

        self.embed = w(VOCAB, HIDDEN) * 8
        self.layers = [dict(qkv=w(HIDDEN, (HEADS + 2 * KV_HEADS) * HEAD_DIM), o=w(HEADS * HEAD_DIM, HIDDEN),
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
            q, k, v = (h @ layer["qkv"]).split([HEADS * HEAD_DIM, KV_HEADS * HEAD_DIM, KV_HEADS * HEAD_DIM], -1)
            q = q.view(-1, HEADS, HEAD_DIM)
            k = k.reshape(-1, KV_HEADS, HEAD_DIM).contiguous()
            v = v.reshape(-1, KV_HEADS, HEAD_DIM).contiguous()
            view = cache.transpose(2, 3)  # (2, blocks, tokens, heads, dim)
            store_kvcache(k, v, view[0], view[1], slots)
            # Gather the sequence's keys/values from its blocks, then causal attention (GQA).
            n_blocks = -(-cache_len // BLOCK)
            ids = torch.tensor(block_table[:n_blocks], device="cuda")
            keys = view[0][ids].reshape(-1, KV_HEADS, HEAD_DIM)[:cache_len]
            values = view[1][ids].reshape(-1, KV_HEADS, HEAD_DIM)[:cache_len]
            keys = keys.repeat_interleave(HEADS // KV_HEADS, 1).transpose(0, 1)
            values = values.repeat_interleave(HEADS // KV_HEADS, 1).transpose(0, 1)
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


@pytest.mark.parametrize("decode_tp", [1, 2])
def test_greedy_decode_after_a_transfer_is_token_identical(decode_tp):
    model = TinyDecoder()
    g = torch.Generator().manual_seed(1)
    prompt_len = 150  # 10 blocks, the last one partly filled
    prompt = torch.randint(0, VOCAB, (prompt_len,), generator=g).cuda()
    n_blocks = -(-(prompt_len + 40) // BLOCK)
    prefill_table = torch.randperm(40, generator=g)[:n_blocks].tolist()
    decode_table = torch.randperm(48, generator=g)[:n_blocks].tolist()

    prefill_caches = cache(40)
    logits = model.forward(prompt, torch.arange(prompt_len, device="cuda"), prefill_caches, prefill_table, prompt_len)
    first = int(logits[-1].argmax())

    # Move the prompt's blocks: prefill TP1 -> decode TP decode_tp (each decode rank takes its KV heads).
    prompt_blocks = -(-prompt_len // BLOCK)
    port = free_port()
    producer = CudaIpcConnectorWorker(WorkerConfig(KVTransferConfig(kv_role="kv_producer", kv_port=port,
                                                                    engine_id="p"), 1, BLOCK), 0)
    producer.register_kv_caches(prefill_caches)
    per = KV_HEADS // decode_tp
    decode_rank_caches = [cache(48, per) for _ in range(decode_tp)]
    consumers = []
    try:
        for rank in range(decode_tp):
            c = CudaIpcConnectorWorker(WorkerConfig(KVTransferConfig(kv_role="kv_consumer", engine_id="d"),
                                                    decode_tp, BLOCK), rank)
            c.register_kv_caches(decode_rank_caches[rank])
            consumers.append(c)
        producer.start_load_kv(KVConnectorMetadata(reqs_to_send={"r": prefill_table[:prompt_blocks]}))
        for c in consumers:
            c.start_load_kv(KVConnectorMetadata(reqs_to_recv={"r": ReqToRecv(
                decode_table[:prompt_blocks], prefill_table[:prompt_blocks], "r", "p", "127.0.0.1", port, 1)}))
        outputs = [wait_for(c) for c in consumers]
        assert KVOutputAggregator(decode_tp).aggregate(outputs).finished_recving == {"r"}
    finally:
        for w in [producer, *consumers]:
            w.shutdown()
    decode_caches = [torch.cat([decode_rank_caches[r][layer] for r in range(decode_tp)], dim=2)
                     for layer in range(LAYERS)]  # every decode rank's heads, as one TP1 cache

    colocated = model.greedy(prefill_caches, prefill_table, prompt_len, first, 24)
    disaggregated = model.greedy(decode_caches, decode_table, prompt_len, first, 24)
    assert colocated == disaggregated
    assert len(set(colocated)) > 1  # a real decode, not one token repeated
