"""Disaggregated prefill end to end with the reference's real engine and model: a prefill and a decode LLMEngine of
lean-vLLM, each in its own process, on a small random-weight Qwen3 on CPU, with CudaIpcConnector registered in the
reference's connector table (as INTEGRATION.md does) carrying the KV between them.

It follows the reference's own check (tests/test_disagg_e2e.py:1-7, 94-124). The decode engine recomputes only the
last prompt token, attending to the pulled KV. Its greedy tokens must therefore equal the prefill engine's when that
engine runs the same prompt split the same way: all but one token, then that one. The prefill engine frees every
held block once the decode engine has them. Both directions run: the reference's pull, and this package's push with
the block ids announced by the decode instance.

What runs on CPU here: the reference engine (scheduler, block manager, model runner, torch attention backend) and
this package's connector halves, handshake, reader counting and release. The byte copy is the host transport's
memmove over caches in shared files (tests/shm_transport.py, as the multi-process tests use); the sm_100a kernels under it are checked against the
oracle by the GPU tests. The checkpoint and its word-level tokenizer are written here with seeded random weights:
there is no network to fetch one. Skipped where no reference checkout is present (REFERENCE_ROOT)."""

import json
import multiprocessing as mp
import os
import socket
import sys
from time import sleep

import pytest

REFERENCE_ROOT = os.path.abspath(
    os.environ.get("REFERENCE_ROOT", os.path.join(os.path.dirname(__file__), "..", "..", "reference")))
if not os.path.isdir(os.path.join(REFERENCE_ROOT, "lean_vllm")):
    pytest.skip("no lean-vLLM reference checkout", allow_module_level=True)

VOCAB = 256  # word-level tokens "t0".."t255", then "<eos>"
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
    words = Tokenizer(models.WordLevel({f"t{i}": i for i in range(VOCAB)} | {"<eos>": VOCAB}, unk_token="t0"))
    words.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    words.save(os.path.join(folder, "tokenizer.json"))
    with open(os.path.join(folder, "tokenizer_config.json"), "w") as f:
        json.dump({"tokenizer_class": "PreTrainedTokenizerFast", "eos_token": "<eos>", "unk_token": "t0"}, f)
    hidden, inner, heads, kv_heads, dim, layers = 64, 128, 4, 2, 32, 2
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump({"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "vocab_size": VOCAB + 1,
                   "hidden_size": hidden, "intermediate_size": inner, "num_hidden_layers": layers,
                   "num_attention_heads": heads, "num_key_value_heads": kv_heads, "head_dim": dim,
                   "max_position_embeddings": 512, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0,
                   "hidden_act": "silu", "attention_bias": False, "tie_word_embeddings": False,
                   "eos_token_id": VOCAB, "bos_token_id": VOCAB, "dtype": "bfloat16"}, f)
    generator = torch.Generator().manual_seed(0)

    def weight(*shape):
        return (torch.randn(*shape, generator=generator) * 0.1).to(torch.bfloat16)

    tensors = {"model.embed_tokens.weight": weight(VOCAB + 1, hidden), "lm_head.weight": weight(VOCAB + 1, hidden),
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
    """A reference LLMEngine on CPU with CudaIpcConnector in its connector table, its KV caches in shared files."""
    os.environ["LEAN_VLLM_DEVICE"] = "cpu"
    import torch

    torch._dynamo.config.disable = True  # the reference compiles a few layers; this image has no OpenMP for inductor
    sys.path.insert(0, REFERENCE_ROOT)
    import lean_vllm.kv_transfer as ref_kv
    from lean_vllm.engine import model_runner
    from lean_vllm.engine.llm_engine import LLMEngine

    from lean_vllm_b200.kv_transfer import cuda_ipc_connector
    from lean_vllm_b200.kv_transfer.cuda_ipc_connector import CudaIpcConnectorScheduler, CudaIpcConnectorWorker
    from tests.shm_transport import ShmTransport, shared_cache

    ref_kv.CONNECTORS["CudaIpcConnector"] = (CudaIpcConnectorScheduler, CudaIpcConnectorWorker)
    cuda_ipc_connector.make_transport = ShmTransport
    allocate = model_runner.ModelRunner.allocate_kv_cache

    def shared_empty(shape, **_):
        assert torch.get_default_dtype() == torch.bfloat16
        return shared_cache(tuple(shape), directory=cache_folder)

    def allocate_shared(self):  # the engine's own allocation, with each layer's tensor in a shared file
        empty, torch.empty = torch.empty, shared_empty
        try:
            allocate(self)
        finally:
            torch.empty = empty

    model_runner.ModelRunner.allocate_kv_cache = allocate_shared
    return LLMEngine(model, **ENGINE_ARGS, **kwargs)


def _prefill(conn, model: str, cache_folder: str, kv_port: int, push_id: str | None):
    engine = _engine(model, cache_folder, enable_prefix_caching=False, long_prefill_token_threshold=len(PROMPT) - 1,
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
    conn.send(engine.scheduler.block_manager.usage)
    reference = engine.generate([list(PROMPT)], SamplingParams(temperature=0, max_tokens=MAX_TOKENS), use_tqdm=False)
    conn.send(reference[0]["token_ids"])


def _decode(conn, model: str, cache_folder: str, kv_port: int):
    os.environ["LEAN_VLLM_KVX_ACCEPT_PUSH"] = "1"  # serves on kv_port, so a prefill engine may push into it
    engine = _engine(model, cache_folder, kv_transfer_config=json.dumps(
        dict(kv_connector="CudaIpcConnector", kv_role="kv_consumer", kv_port=kv_port)))
    from lean_vllm.sampling_params import SamplingParams

    params = conn.recv()
    sampling_params = SamplingParams(temperature=0, max_tokens=MAX_TOKENS, kv_transfer_params=params)
    outputs = engine.generate([list(PROMPT)], sampling_params, use_tqdm=False)
    # A prometheus counter: its total over labels.
    prefill_tokens = sum(sample.value for family in engine.metrics.prefill_tokens.collect()
                         for sample in family.samples if sample.name.endswith("_total"))
    conn.send((outputs[0]["token_ids"], prefill_tokens))


def _receive(conn, process, what: str, timeout: float = 300.0):
    """The child's next message; fails as soon as the child has died rather than at the timeout."""
    for _ in range(int(timeout / 0.1)):
        if conn.poll(0.1):
            return conn.recv()
        if not process.is_alive():
            raise AssertionError(f"{what}: its process exited with {process.exitcode}")
    raise AssertionError(what)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    folder = str(tmp_path_factory.mktemp("qwen3-random"))
    make_checkpoint(folder)
    return folder


@pytest.mark.parametrize("mode", ["pull", "push"])
def test_the_reference_decode_engine_continues_from_the_kv_this_connector_carried(checkpoint, tmp_path, mode):
    """Pull: the prefill finishes, hands its kv_transfer_params over, and the decode engine reads the blocks. Push:
    the decode request is admitted first (kv_push, no block ids) and announces its blocks; the prefill engine,
    given the same push id, writes them (all at hand-over: the reference model calls no per-layer hook)."""
    caches = tmp_path / "caches"
    caches.mkdir()
    prefill_port, decode_port = _free_port(), _free_port()
    push_id = "push-1" if mode == "push" else None
    ctx = mp.get_context("spawn")
    prefill_conn, prefill_child = ctx.Pipe()
    decode_conn, decode_child = ctx.Pipe()
    prefill = ctx.Process(target=_prefill, args=(prefill_child, checkpoint, str(caches), prefill_port, push_id))
    decode = ctx.Process(target=_decode, args=(decode_child, checkpoint, str(caches), decode_port))
    for process in (prefill, decode):
        process.start()
    try:
        if push_id is None:
            params = _receive(prefill_conn, prefill, "the prefill engine never handed off")
            assert params["do_remote_prefill"] and params["remote_port"] == prefill_port
            decode_conn.send(params)
        else:
            assert _receive(prefill_conn, prefill, "the prefill engine never came up") == "serving"
            decode_conn.send({"do_remote_prefill": True, "kv_push": True, "remote_request_id": push_id,
                              "remote_engine_id": "", "remote_host": "127.0.0.1", "remote_port": prefill_port,
                              "tp_size": 1, "remote_block_ids": []})
            prefill_conn.send("go")
            _receive(prefill_conn, prefill, "the prefill engine never finished its request")
        token_ids, num_prefill_tokens = _receive(decode_conn, decode, "the decode engine never finished")
        assert _receive(prefill_conn, prefill, "the prefill engine kept its blocks") == 0.0  # all freed
        reference = _receive(prefill_conn, prefill, "the prefill engine's own run never finished")
    finally:
        for process in (prefill, decode):
            process.join(timeout=60)
            if process.is_alive():
                process.kill()
    assert num_prefill_tokens == 1  # only the last prompt token ran here; the rest came from the prefill engine
    assert len(token_ids) == MAX_TOKENS or token_ids[-1] == VOCAB
    assert token_ids == reference
