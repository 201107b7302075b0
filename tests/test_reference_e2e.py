"""Disaggregated prefill end to end with the reference's real engine and model: a prefill and a decode LLMEngine of
lean-vLLM, each in its own process, on a small random-weight Qwen3 on CPU, with CudaIpcConnector registered in the
reference's connector table (as a maintainer registers it) carrying the KV between them.

It follows the reference's own check (tests/test_disagg_e2e.py:1-7, 94-124). The decode engine recomputes only the
last prompt token, attending to the pulled KV. Its greedy tokens must therefore equal the prefill engine's when that
engine runs the same prompt split the same way: all but one token, then that one. The prefill engine frees every
held block once the decode engine has them. Both directions run: the reference's pull, and this package's push with
the block ids announced by the decode instance. A TP2 prefill engine feeding a TP1 decode engine runs too: there the
two engines' tokens are not comparable (different summation orders), so the decode rank instead compares every
pulled token row, head by head, with the producer rank that computed it.

What runs on CPU here: the reference engine (scheduler, block manager, model runner, torch attention backend) and
this package's connector halves, handshake, reader counting and release. The byte copy is the host transport's
memmove over caches in shared files (tests/shm_transport.py, as the multi-process tests use); the sm_100a kernels under it are checked against the
oracle by the GPU tests. The checkpoint and its word-level tokenizer are written here with seeded random weights:
there is no network to fetch one. Skipped where no reference checkout is present (REFERENCE_ROOT)."""

import json
import multiprocessing as mp
import os
from time import sleep

import pytest

REFERENCE_ROOT = os.path.abspath(
    os.environ.get("REFERENCE_ROOT", os.path.join(os.path.dirname(__file__), "..", "..", "reference")))
if not os.path.isdir(os.path.join(REFERENCE_ROOT, "lean_vllm")):
    pytest.skip("no lean-vLLM reference checkout", allow_module_level=True)

VOCAB = 256  # word-level tokens "t0".."t255", then "<eos>" and "<pad>"
PROMPT = [(7 * i + 3) % VOCAB for i in range(90)]  # five 16-token blocks and a bit
MAX_TOKENS = 16
ENGINE_ARGS = dict(enforce_eager=True, kvcache_memory_gb=0.01, max_model_len=256, max_num_batched_tokens=256)


def make_checkpoint(folder: str):
    """A two-layer Qwen3 in the Hugging Face layout (config.json, model.safetensors, a word-level tokenizer.json):
    4 query heads and 2 KV heads of 32, seeded random bf16 weights. Written directly, without transformers."""
    import torch
    from safetensors.torch import save_file
    from tokenizers import Tokenizer, models, pre_tokenizers

    os.makedirs(folder, exist_ok=True)
    # "<pad>" is never produced by the prompt; it makes the table even, as a TP2 engine splits it in halves.
    words = Tokenizer(models.WordLevel({f"t{i}": i for i in range(VOCAB)} | {"<eos>": VOCAB, "<pad>": VOCAB + 1},
                                       unk_token="t0"))
    words.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    words.save(os.path.join(folder, "tokenizer.json"))
    with open(os.path.join(folder, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "eos_token": "<eos>", "unk_token": "t0"}, f)
    hidden, inner, heads, kv_heads, dim, layers = 64, 128, 4, 2, 32, 2
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump({"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "vocab_size": VOCAB + 2,
                   "hidden_size": hidden, "intermediate_size": inner, "num_hidden_layers": layers,
                   "num_attention_heads": heads, "num_key_value_heads": kv_heads, "head_dim": dim,
                   "max_position_embeddings": 512, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0,
                   "hidden_act": "silu", "attention_bias": False, "tie_word_embeddings": False,
                   "eos_token_id": VOCAB, "bos_token_id": VOCAB, "dtype": "bfloat16"}, f)
    generator = torch.Generator().manual_seed(0)

    def weight(*shape):
        return (torch.randn(*shape, generator=generator) * 0.1).to(torch.bfloat16)

    tensors = {"model.embed_tokens.weight": weight(VOCAB + 2, hidden), "lm_head.weight": weight(VOCAB + 2, hidden),
               "model.norm.weight": torch.ones(hidden, dtype=torch.bfloat16)}
    for i in range(layers):
        at = f"model.layers.{i}."
        tensors |= {
            at + "self_attn.q_proj.weight": weight(heads * dim, hidden),
            at + "self_attn.k_proj.weight": weight(kv_heads * dim, hidden),
            at + "self_attn.v_proj.weight": weight(kv_heads * dim, hidden),
            at + "self_attn.o_proj.weight": weight(hidden, heads * dim),
            at + "self_attn.q_norm.weight": torch.ones(dim, dtype=torch.bfloat16),
            at + "self_attn.k_norm.weight": torch.ones(dim, dtype=torch.bfloat16),
            at + "mlp.gate_proj.weight": weight(inner, hidden),
            at + "mlp.up_proj.weight": weight(inner, hidden),
            at + "mlp.down_proj.weight": weight(hidden, inner),
            at + "input_layernorm.weight": torch.ones(hidden, dtype=torch.bfloat16),
            at + "post_attention_layernorm.weight": torch.ones(hidden, dtype=torch.bfloat16),
        }
    save_file(tensors, os.path.join(folder, "model.safetensors"), metadata={"format": "pt"})


def _engine(model: str, cache_folder: str, **kwargs):
    """A reference LLMEngine on CPU with CudaIpcConnector in its connector table and its KV caches in shared files,
    on every tensor-parallel rank (tests/kvx_reference_runner.py)."""
    os.environ["LEAN_VLLM_DEVICE"] = "cpu"
    os.environ["KVX_REFERENCE_ROOT"] = REFERENCE_ROOT
    os.environ["KVX_TEST_CACHE_DIR"] = cache_folder
    import tests.kvx_reference_runner  # noqa: F401 - the setup, in this process and every rank it spawns
    from lean_vllm.engine.llm_engine import LLMEngine

    return LLMEngine(model, **ENGINE_ARGS, **kwargs)


def _prefill(conn, model: str, cache_folder: str, kv_port: int, push_id: str | None, tp: int):
    # The prompt runs split n-1 + 1 where the split is comparable (TP1). The reference engine at TP > 1 cannot run a
    # chunk that samples nothing (its logits gather reshapes zero rows), so there the prompt runs whole.
    split = dict(long_prefill_token_threshold=len(PROMPT) - 1) if tp == 1 else {}
    if tp > 1:  # the ranks' connector outputs reach rank 0 through KVConnectorStep's mailbox, not gather_object
        os.environ["KVX_TEST_STEP"] = "mailbox"
    engine = _engine(model, cache_folder, enable_prefix_caching=False, tensor_parallel_size=tp, **split,
                     kv_transfer_config=json.dumps(dict(kv_connector="CudaIpcConnector", kv_role="kv_producer",
                                                        kv_port=kv_port)))
    from lean_vllm.sampling_params import SamplingParams

    params = {"do_remote_decode": True}
    if push_id is not None:  # the decode request came first and waits: push into the blocks it announces
        conn.send("serving")
        conn.recv()
        params["kv_push_id"] = push_id
    engine.add_request(list(PROMPT), SamplingParams(temperature=0, max_tokens=1, kv_transfer_params=params), "p-1")
    result = None
    while result is None:
        result = next((output.kv_transfer_params for output in engine.step()[0] if output.finished), None)
    conn.send(result)
    while not engine.is_finished():  # until the decode engine has the blocks and they are let go
        engine.step()
        sleep(0.001)
    step = getattr(engine.model_runner, "_kv_step", None)  # KVConnectorStep, where it replaced the gather
    conn.send((engine.scheduler.block_manager.usage, step.exchange if step is not None else None))
    conn.recv()  # the decode side has compared its copy with the freed blocks: they may be reused now
    reference = None
    if tp == 1:  # across sizes the tokens are not comparable (see the test)
        reference = engine.generate([list(PROMPT)], SamplingParams(temperature=0, max_tokens=MAX_TOKENS),
                                    use_tqdm=False)[0]["token_ids"]
    conn.send(reference)
    engine.exit()  # the other ranks leave their loop before this process ends


def _pulled_bytes_match(worker, req, positions: int) -> bool:
    """This decode rank's copy of the first `positions` prompt tokens against every producer rank's blocks, mapped
    here by the handshake: each head share of head_shares, token rows compared byte for byte, every layer, K and V."""
    import ctypes

    from lean_vllm_b200.kv_transfer.shares import head_shares, split_heads

    heads = split_heads(worker.num_heads, worker.tp_size, req.remote_tp_size)
    block = worker.block_size
    compared = 0
    for share in head_shares(worker.rank, worker.tp_size, req.remote_tp_size, heads):
        remote = worker._remotes[(req.remote_host, req.remote_port + share.remote_rank)].table["regions"]
        for (mine, my_block, my_head), (theirs, their_block, their_head) in zip(worker.transport.regions, remote):
            row = my_head // block  # one token of one head
            for i, (local, src) in enumerate(zip(req.local_block_ids, req.remote_block_ids)):
                tokens = min(block, positions - i * block)
                for k in range(share.num_heads if tokens > 0 else 0):
                    a = mine + local * my_block + (share.local_head + k) * my_head
                    b = theirs + src * their_block + (share.remote_head + k) * their_head
                    if ctypes.string_at(a, tokens * row) != ctypes.string_at(b, tokens * row):
                        return False
                    compared += tokens * row
    return compared > 0


def _decode(conn, model: str, cache_folder: str, kv_port: int, tp: int):
    os.environ["LEAN_VLLM_KVX_ACCEPT_PUSH"] = "1"  # serves on kv_port, so a prefill engine may push into it
    if tp > 1:  # the load ends once both ranks report it, through KVConnectorStep's mailbox
        os.environ["KVX_TEST_STEP"] = "mailbox"
    engine = _engine(model, cache_folder, tensor_parallel_size=tp, kv_transfer_config=json.dumps(
        dict(kv_connector="CudaIpcConnector", kv_role="kv_consumer", kv_port=kv_port)))
    from lean_vllm.sampling_params import SamplingParams

    worker, loads = engine.model_runner.kv_connector, {}
    start_load_kv = worker.start_load_kv

    def recording(metadata):  # what the scheduler half asked this rank to load
        loads.update(metadata.reqs_to_recv)
        start_load_kv(metadata)

    worker.start_load_kv = recording
    params = conn.recv()
    sampling_params = SamplingParams(temperature=0, max_tokens=MAX_TOKENS, kv_transfer_params=params)
    outputs = engine.generate([list(PROMPT)], sampling_params, use_tqdm=False)
    # A prometheus counter: its total over labels.
    prefill_tokens = sum(sample.value for family in engine.metrics.prefill_tokens.collect()
                         for sample in family.samples if sample.name.endswith("_total"))
    # The last prompt token's slot was recomputed here, so the copy is compared up to it.
    (req,) = loads.values()
    match = None if req.pushed else _pulled_bytes_match(worker, req, len(PROMPT) - 1)  # this rank's heads
    step = getattr(engine.model_runner, "_kv_step", None)
    conn.send((outputs[0]["token_ids"], prefill_tokens, match, step.exchange if step is not None else None))
    engine.exit()


def _receive(conn, process, what: str, timeout: float = 300.0):
    """The child's next message; fails as soon as the child has died rather than at the timeout."""
    for _ in range(int(timeout / 0.1)):
        if conn.poll(0.1):
            return conn.recv()
        if not process.is_alive():
            raise AssertionError(f"{what}: its process exited with {process.exitcode}")
    raise AssertionError(what)


def _free_port() -> int:
    """A port whose span (kv_port + rank for every rank) is free and was not handed out before here."""
    from tests.connector_cases import free_port

    return free_port()


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    folder = str(tmp_path_factory.mktemp("qwen3-random"))
    make_checkpoint(folder)
    return folder


@pytest.mark.parametrize("mode, prefill_tp, decode_tp", [("pull", 1, 1), ("push", 1, 1), ("pull", 2, 1),
                                                         ("pull", 1, 2), ("push", 1, 2)],
                         ids=["pull", "push", "pull-tp2-to-tp1", "pull-tp1-to-tp2", "push-tp1-to-tp2"])
def test_the_reference_decode_engine_continues_from_the_kv_this_connector_carried(checkpoint, tmp_path, mode,
                                                                                  prefill_tp, decode_tp):
    """Pull: the prefill finishes, hands its kv_transfer_params over, and the decode engine reads the blocks. Push:
    the decode request is admitted first (kv_push, no block ids) and announces its blocks; the prefill engine,
    given the same push id, writes them (all at hand-over: the reference model calls no per-layer hook). With a TP2
    prefill engine, each of its ranks holds one of the two KV heads, and the TP1 decode rank takes a share from each
    (head_shares); that engine's ranks hand rank 0 their connector outputs through KVConnectorStep's shared-memory
    mailbox, wired into the reference's ModelRunner as a maintainer would. A TP1 prefill engine feeding a TP2 decode
    engine has each decode rank pull its own head and the load end once both ranks report it, through the same
    mailbox. Every pull is also checked byte for byte against the producer ranks' blocks (on decode rank 0)."""
    caches = tmp_path / "caches"
    caches.mkdir()
    prefill_port, decode_port = _free_port(), _free_port()
    push_id = "push-1" if mode == "push" else None
    ctx = mp.get_context("spawn")
    prefill_conn, prefill_child = ctx.Pipe()
    decode_conn, decode_child = ctx.Pipe()
    prefill = ctx.Process(target=_prefill, args=(prefill_child, checkpoint, str(caches), prefill_port, push_id,
                                                 prefill_tp))
    decode = ctx.Process(target=_decode, args=(decode_child, checkpoint, str(caches), decode_port, decode_tp))
    for process in (prefill, decode):
        process.start()
    try:
        if push_id is None:
            params = _receive(prefill_conn, prefill, "the prefill engine never handed off")
            assert params["do_remote_prefill"] and params["remote_port"] == prefill_port
            assert params["tp_size"] == prefill_tp
            decode_conn.send(params)
        else:
            assert _receive(prefill_conn, prefill, "the prefill engine never came up") == "serving"
            decode_conn.send({"do_remote_prefill": True, "kv_push": True, "remote_request_id": push_id,
                              "remote_engine_id": "", "remote_host": "127.0.0.1", "remote_port": prefill_port,
                              "tp_size": prefill_tp, "remote_block_ids": []})
            prefill_conn.send("go")
            _receive(prefill_conn, prefill, "the prefill engine never finished its request")
        token_ids, num_prefill_tokens, bytes_match, decode_exchange = _receive(decode_conn, decode,
                                                                               "the decode engine never finished")
        assert decode_exchange == ("mailbox" if decode_tp > 1 else None)
        usage, exchange = _receive(prefill_conn, prefill, "the prefill engine kept its blocks")
        assert usage == 0.0  # every held block freed
        assert exchange == ("mailbox" if prefill_tp > 1 else None)
        prefill_conn.send("compared")
        reference = _receive(prefill_conn, prefill, "the prefill engine's own run never finished")
    finally:
        for process in (prefill, decode):
            process.join(timeout=60)
            if process.is_alive():
                process.kill()
    assert num_prefill_tokens == 1  # only the last prompt token ran here; the rest came from the prefill engine
    assert len(token_ids) == MAX_TOKENS or token_ids[-1] == VOCAB
    if mode == "pull":
        assert bytes_match  # every head of every pulled token, bit for bit, from the rank that computed it
    if prefill_tp == decode_tp:
        assert token_ids == reference
    # Across tensor-parallel sizes the two engines sum in different orders, so their greedy tokens may differ in
    # bf16; the bytes above are the exact check there.
