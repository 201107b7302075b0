"""The drop-in, proven against the reference's own engine code: lean-vLLM's Scheduler, BlockManager and
LLMEngine step loop (imported from a reference checkout, unmodified) drive CudaIpcConnector through the reference's
connector factory, exactly as a maintainer registers it. Runs on CPU: the runner is a stub whose model "computes"
a deterministic KV row per (token, position) into the worker's caches, and the transport is the host one.

A prefill engine finishes a request with do_remote_decode, holds its blocks and returns kv_transfer_params; a decode
engine admits the request with those params, waits (WAITING_FOR_REMOTE_KVS) while the worker pulls the blocks,
resumes at the last prompt token and finishes; the prefill engine frees its blocks once the read is reported. The
decode cache then holds, bit for bit, the prefill's KV of every prompt position.

Skipped where no reference checkout is present (set REFERENCE_ROOT to point at one)."""

import os
import socket
import sys
import time
from dataclasses import dataclass

import pytest
import torch

# A lean-vLLM checkout: REFERENCE_ROOT, else a "reference" folder beside this repository.
REFERENCE_ROOT = os.environ.get("REFERENCE_ROOT", os.path.join(os.path.dirname(__file__), "..", "..", "reference"))
if not os.path.isdir(os.path.join(REFERENCE_ROOT, "lean_vllm")):
    pytest.skip("no lean-vLLM reference checkout", allow_module_level=True)
sys.path.insert(0, REFERENCE_ROOT)
try:
    import lean_vllm.kv_transfer as ref_kv
    from lean_vllm.engine.llm_engine import LLMEngine
    from lean_vllm.engine.metrics import Metrics
    from lean_vllm.engine.scheduler import Scheduler
    from lean_vllm.engine.sequence import Sequence, SequenceStatus
    from lean_vllm.sampling_params import SamplingParams
except ImportError as error:  # a dependency of the reference engine is missing here
    pytest.skip(f"the reference engine does not import: {error}", allow_module_level=True)
finally:
    sys.path.remove(REFERENCE_ROOT)

from lean_vllm_b200.kv_transfer import KVConnectorStep, KVTransferConfig, cuda_ipc_connector  # noqa: E402
from lean_vllm_b200.kv_transfer.cuda_ipc_connector import (  # noqa: E402
    CudaIpcConnectorScheduler,
    CudaIpcConnectorWorker,
)
from tests.host_transport import HostTransport  # noqa: E402

BLOCK, HEADS, DIM, LAYERS, BLOCKS = 8, 4, 16, 3, 32


@dataclass
class EngineConfig:
    """What the reference Scheduler and the connector halves read from an engine's Config."""

    kv_transfer: object
    num_kvcache_blocks: int = BLOCKS
    kvcache_block_size: int = BLOCK
    max_num_seqs: int = 4
    max_num_batched_tokens: int = 256
    max_model_len: int = 1024
    eos: int = 2
    enable_chunked_prefill: bool = True
    enable_prefix_caching: bool = True
    prefix_caching_hash_algo: str = "sha256"
    scheduling_policy: str = "fcfs"
    long_prefill_token_threshold: int = 0
    async_scheduling: bool = False
    tensor_parallel_size: int = 1
    speculative: object = None
    kv_cache_layout: str = "HND"
    kvx_accept_push: bool = False


def kv_row(token: int, position: int, layer: int, part: int) -> torch.Tensor:
    """The stub model's key (part 0) or value (part 1) of one token at one position: (heads, dim), exact in bf16."""
    grid = torch.arange(HEADS * DIM, dtype=torch.float32).reshape(HEADS, DIM)
    return ((grid + token * 3 + position * 5 + layer * 7 + part * 11) % 97).to(torch.bfloat16)


class Tokens:
    def __init__(self, token_ids):
        self.token_ids = token_ids

    def tolist(self):
        return self.token_ids


class StubRunner:
    """ModelRunner's call() surface: kv_connector_step through this package's KVConnectorStep, and a run() that
    stores each scheduled token's KV into the paged caches by the sequence's block table."""

    step_kind = "eager"

    def __init__(self, config, caches, layer_hooks=False):
        self.caches = caches
        self.layer_hooks = layer_hooks  # call save_kv_layer after each layer's store, as an engine with hooks does
        self.batches: list = []  # (request, tokens scheduled) of every batch run
        self.worker = CudaIpcConnectorWorker(config, 0)
        self.worker.register_kv_caches(caches)
        self.kv_step = KVConnectorStep(self.worker, 0, 1)

    def call(self, method, *args):
        return getattr(self, method)(*args)

    def kv_connector_step(self, metadata):
        return self.kv_step(metadata)

    def run(self, seqs):
        sampled = []
        self.batches.append([(seq.request_id, seq.num_scheduled_tokens) for seq in seqs])
        for seq in seqs:
            begin = seq.num_cached_tokens
            end = begin + seq.num_scheduled_tokens
            for layer, cache in enumerate(self.caches):
                for position in range(begin, end):
                    block, offset = seq.block_table[position // BLOCK], position % BLOCK
                    for part in range(2):
                        cache[part, block, :, offset, :] = kv_row(seq.token_ids[position], position, layer, part)
                if self.layer_hooks:
                    self.worker.save_kv_layer(layer)
            if end >= seq.num_planned_tokens:  # the scheduler's sampling rows: a finished prefill or a decode step
                sampled.append(100 + len(seq.token_ids))
        return Tokens(sampled)

    def shutdown(self):
        self.worker.shutdown()


class Engine(LLMEngine):
    """The reference's production step loop (step/_launch/_reconcile), with the stub runner."""

    tokenizer = None

    def __init__(self, config, runner):
        # What LLMEngine.__init__ sets on Sequence from the Config (llm_engine.py:131-133); the fixture restores them.
        Sequence.block_size = config.kvcache_block_size
        Sequence.enable_prefix_caching = config.enable_prefix_caching
        Sequence.hash_algo = config.prefix_caching_hash_algo
        self.config = config
        self.scheduler = Scheduler(config)
        self.model_runner = runner
        self.metrics = Metrics()
        self.in_flight = None
        self.profiler = None
        self.output_processor = None
        self.ps = []

    def add(self, prompt, params, request_id):
        seq = Sequence(prompt, params, request_id)
        self.scheduler.add(seq)
        return seq


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture
def engines(monkeypatch):
    monkeypatch.setitem(ref_kv.CONNECTORS, "CudaIpcConnector", (CudaIpcConnectorScheduler, CudaIpcConnectorWorker))
    monkeypatch.setattr(cuda_ipc_connector, "make_transport", HostTransport)
    monkeypatch.setattr(HostTransport, "fail", None)
    for name in ("block_size", "enable_prefix_caching", "hash_algo"):
        monkeypatch.setattr(Sequence, name, getattr(Sequence, name))  # restored after the test
    made = []

    def make(role, engine_id, accept_push=False, layer_hooks=False, max_batched=256):
        kv = KVTransferConfig(kv_connector="CudaIpcConnector", kv_role=role, kv_ip="127.0.0.1", kv_port=free_port(),
                              engine_id=engine_id)
        config = EngineConfig(kv, kvx_accept_push=accept_push, max_num_batched_tokens=max_batched)
        caches = [torch.zeros(2, BLOCKS, HEADS, BLOCK, DIM, dtype=torch.bfloat16) for _ in range(LAYERS)]
        engine = Engine(config, StubRunner(config, caches, layer_hooks))
        made.append(engine)
        return engine

    yield make
    for engine in made:
        engine.model_runner.shutdown()


def step_until(engines_to_step, done, timeout=20.0):
    deadline = time.monotonic() + timeout
    outputs = []
    while not done(outputs):
        assert time.monotonic() < deadline, "the engines did not get there"
        for engine in engines_to_step:
            outputs += engine.step()[0]
        time.sleep(0.002)
    return outputs


def test_the_reference_engine_runs_a_disaggregated_request_through_the_connector(engines):
    prefill, decode = engines("kv_producer", "prefill-engine"), engines("kv_consumer", "decode-engine")
    prompt = [40 + (i * 13) % 50 for i in range(21)]  # 21 tokens: three blocks, the last partial

    # Prefill: one token, then the connector holds the blocks and hands back what the decode side pulls.
    prefill_seq = prefill.add(prompt, SamplingParams(max_tokens=1, ignore_eos=True,
                                                     kv_transfer_params={"do_remote_decode": True}), "p-1")
    outputs = step_until([prefill], lambda out: any(o.finished for o in out))
    params = next(o.kv_transfer_params for o in outputs if o.finished)
    assert params["do_remote_prefill"] and params["remote_engine_id"] == "prefill-engine"
    assert params["remote_block_ids"] == list(prefill_seq.block_table[:3])
    assert not prefill.is_finished()  # the blocks are held for the reader

    # Decode: admitted, waits for the blocks, then computes only its last prompt token and decodes.
    decode_seq = decode.add(prompt, SamplingParams(max_tokens=3, ignore_eos=True, kv_transfer_params=params), "d-1")
    decode.step()
    assert decode_seq.status == SequenceStatus.WAITING_FOR_REMOTE_KVS
    dst_blocks = list(decode_seq.block_table[:3])  # freed (and the table cleared) when the request finishes
    step_until([prefill, decode], lambda out: decode.is_finished() and prefill.is_finished())
    assert decode_seq.is_finished and len(decode_seq.token_ids) == len(prompt) + 3
    assert prefill.scheduler.block_manager.free_block_queue.num_free_blocks == BLOCKS  # released once read

    # Every prompt position's KV in the decode cache is the prefill's, bit for bit.
    src_blocks = params["remote_block_ids"]
    for layer in range(LAYERS):
        src = prefill.model_runner.caches[layer][:, src_blocks].transpose(2, 3).reshape(2, 3 * BLOCK, HEADS, DIM)
        dst = decode.model_runner.caches[layer][:, dst_blocks].transpose(2, 3).reshape(2, 3 * BLOCK, HEADS, DIM)
        assert torch.equal(src[:, : len(prompt)].view(torch.int16), dst[:, : len(prompt)].view(torch.int16)), layer
    # The reference's metrics saw one load of the connector's byte count: 3 blocks x 2 x 3 layers x 4 heads x 8 x 16.
    registry = decode.metrics.registry
    assert registry.get_sample_value("lean_vllm:kv_transfers_total") == 1.0
    assert registry.get_sample_value("lean_vllm:kv_transfer_bytes_sum") == 3 * 2 * LAYERS * HEADS * BLOCK * DIM * 2


def test_a_load_from_an_absent_prefill_instance_prefills_on_the_decode_side(engines, monkeypatch):
    monkeypatch.setattr(cuda_ipc_connector, "HANDSHAKE_TIMEOUT", 0.3)
    decode = engines("kv_consumer", "decode-engine")
    prompt = list(range(30, 47))
    params = {"do_remote_prefill": True, "do_remote_decode": False, "remote_request_id": "gone",
              "remote_engine_id": "prefill-engine", "remote_block_ids": [4, 5, 6], "remote_host": "127.0.0.1",
              "remote_port": free_port(), "tp_size": 1}
    seq = decode.add(prompt, SamplingParams(max_tokens=2, ignore_eos=True, kv_transfer_params=params), "d-2")
    decode.step()
    blocks = list(seq.block_table[:3])
    step_until([decode], lambda out: decode.is_finished())
    assert seq.is_finished and len(seq.token_ids) == len(prompt) + 2
    assert decode.metrics.registry.get_sample_value("lean_vllm:kv_transfer_failures_total") == 1.0
    # It prefilled the whole prompt itself: its cache holds its own KV at every prompt position.
    for layer in range(LAYERS):
        got = decode.model_runner.caches[layer][:, blocks].transpose(2, 3).reshape(2, 3 * BLOCK, HEADS, DIM)
        for position in (0, len(prompt) - 1):
            assert torch.equal(got[0, position], kv_row(prompt[position], position, layer, 0))


@pytest.mark.parametrize("layer_hooks, chunk", [(False, 256), (True, 256), (True, 6)],
                         ids=["at-hand-over", "per-layer", "per-layer-chunked"])
def test_the_reference_engine_runs_a_pushed_request_with_its_block_ids_exchanged(engines, layer_hooks, chunk):
    """Push mode through the same unmodified engine code: the proxy sends the decode request first (kv_push, no
    block ids) and the prefill request with the same push id; the decode engine admits and waits while its worker
    announces the allocated blocks; the prefill engine's scheduler half turns its admission into a save, and the
    prefill writes the decode blocks (per layer from save_kv_layer, or all at hand-over) before freeing its own.
    With a 6-token step budget the prompt is prefilled in chunks that end inside blocks: each chunk's hooks push
    what it filled (the scheduler half reports each step's progress), and the result is the same."""
    prefill = engines("kv_producer", "prefill-engine", layer_hooks=layer_hooks, max_batched=chunk)
    decode = engines("kv_consumer", "decode-engine", accept_push=True)
    prompt = [60 + (i * 7) % 40 for i in range(19)]
    push_id = "push-7"
    decode_params = {"do_remote_prefill": True, "kv_push": True, "remote_request_id": push_id,
                     "remote_engine_id": "", "remote_host": "127.0.0.1",
                     "remote_port": prefill.config.kv_transfer.kv_port, "tp_size": 1, "remote_block_ids": []}
    assert ref_kv.check_kv_transfer_params(decode_params, decode.config.kv_transfer) is None  # the server accepts it
    decode_seq = decode.add(prompt, SamplingParams(max_tokens=2, ignore_eos=True, kv_transfer_params=decode_params),
                            "d-7")
    decode.step()
    assert decode_seq.status == SequenceStatus.WAITING_FOR_REMOTE_KVS
    dst_blocks = list(decode_seq.block_table[:3])
    prefill_params = {"do_remote_decode": True, "kv_push_id": push_id}
    assert ref_kv.check_kv_transfer_params(prefill_params, prefill.config.kv_transfer) is None
    prefill_seq = prefill.add(prompt, SamplingParams(max_tokens=1, ignore_eos=True,
                                                     kv_transfer_params=prefill_params), "p-7")
    prefill.step()
    src_blocks = list(prefill_seq.block_table[:3])
    if chunk < len(prompt):  # let the first chunk's save find the decode ranks mapped before the next chunk runs
        worker = prefill.model_runner.worker
        deadline = time.monotonic() + 10
        while not worker._saves["p-7"].ready and time.monotonic() < deadline:
            time.sleep(0.002)
    step_until([prefill, decode], lambda out: decode.is_finished() and prefill.is_finished())
    if chunk < len(prompt):
        posts = prefill.model_runner.worker.transport.posts
        assert sum(1 for layer, _ in posts if layer is not None) >= 2 * LAYERS  # per-layer pushes of later chunks
    assert decode_seq.is_finished and len(decode_seq.token_ids) == len(prompt) + 2
    assert prefill.scheduler.block_manager.free_block_queue.num_free_blocks == BLOCKS
    for layer in range(LAYERS):
        src = prefill.model_runner.caches[layer][:, src_blocks].transpose(2, 3).reshape(2, 3 * BLOCK, HEADS, DIM)
        dst = decode.model_runner.caches[layer][:, dst_blocks].transpose(2, 3).reshape(2, 3 * BLOCK, HEADS, DIM)
        assert torch.equal(src[:, : len(prompt)].view(torch.int16), dst[:, : len(prompt)].view(torch.int16)), layer
    assert decode.metrics.registry.get_sample_value("lean_vllm:kv_transfers_total") == 1.0


def test_blocks_the_decode_engine_already_caches_are_not_pulled_again(engines):
    """The decode engine served the same prompt before, so its prefix cache holds the leading full blocks: the
    reference scheduler admits the remote request with those blocks cached, the connector's load covers only the
    rest (the reference's own rule, nixl_connector.py:134-146), and the decode cache still ends equal, position for
    position, to the prefill's KV."""
    prefill, decode = engines("kv_producer", "prefill-engine"), engines("kv_consumer", "decode-engine")
    prompt = [40 + (i * 11) % 50 for i in range(21)]  # 21 tokens: two full blocks and a partial one
    decode.add(prompt, SamplingParams(max_tokens=1, ignore_eos=True), "warm")  # computed here, published
    step_until([decode], lambda out: decode.is_finished())
    prefill.add(prompt, SamplingParams(max_tokens=1, ignore_eos=True, kv_transfer_params={"do_remote_decode": True}),
                "p-2")
    outputs = step_until([prefill], lambda out: any(o.finished for o in out))
    params = next(o.kv_transfer_params for o in outputs if o.finished)
    worker = decode.model_runner.worker
    seen = []
    real_start = worker.start_load_kv

    def recording(metadata):
        seen.extend(metadata.reqs_to_recv.values())
        return real_start(metadata)

    worker.start_load_kv = recording
    seq = decode.add(prompt, SamplingParams(max_tokens=2, ignore_eos=True, kv_transfer_params=params), "d-2")
    decode.step()
    dst_blocks = list(seq.block_table[:3])
    assert seq.num_cached_tokens == 2 * BLOCK  # the trailing partial block always recomputes
    (req,) = seen
    assert req.local_block_ids == dst_blocks[2:] and req.remote_block_ids == params["remote_block_ids"][2:]
    step_until([prefill, decode], lambda out: decode.is_finished() and prefill.is_finished())
    src_blocks = params["remote_block_ids"]
    for layer in range(LAYERS):
        src = prefill.model_runner.caches[layer][:, src_blocks].transpose(2, 3).reshape(2, 3 * BLOCK, HEADS, DIM)
        dst = decode.model_runner.caches[layer][:, dst_blocks].transpose(2, 3).reshape(2, 3 * BLOCK, HEADS, DIM)
        assert torch.equal(src[:, : len(prompt)].view(torch.int16), dst[:, : len(prompt)].view(torch.int16)), layer
    # The connector counted the one block it read: 2 parts x layers x heads x block x dim x 2 bytes.
    assert decode.metrics.registry.get_sample_value("lean_vllm:kv_transfer_bytes_sum") == \
        2 * LAYERS * HEADS * BLOCK * DIM * 2


def test_an_abort_mid_load_frees_the_decode_blocks_once_the_load_ended(engines):
    """The decode request is aborted right after its load started: the reference scheduler keeps its blocks (the
    loader may still be writing them) until the connector reports the load over, then frees them; the prefill
    side still has its blocks read and released."""
    prefill, decode = engines("kv_producer", "prefill-engine"), engines("kv_consumer", "decode-engine")
    prompt = [45 + (i * 7) % 40 for i in range(20)]
    prefill.add(prompt, SamplingParams(max_tokens=1, ignore_eos=True, kv_transfer_params={"do_remote_decode": True}),
                "p-3")
    outputs = step_until([prefill], lambda out: any(o.finished for o in out))
    params = next(o.kv_transfer_params for o in outputs if o.finished)
    decode.add(prompt, SamplingParams(max_tokens=2, ignore_eos=True, kv_transfer_params=params), "d-3")
    decode.step()
    assert decode.scheduler.abort("d-3")
    assert decode.scheduler.block_manager.free_block_queue.num_free_blocks < BLOCKS  # held for the loader
    step_until([prefill, decode], lambda out: decode.is_finished() and prefill.is_finished())
    assert decode.scheduler.block_manager.free_block_queue.num_free_blocks == BLOCKS
    assert prefill.scheduler.block_manager.free_block_queue.num_free_blocks == BLOCKS


def test_an_abort_while_pushed_holds_the_decode_blocks_until_the_pushes_landed(engines):
    """Push mode: the decode request is aborted while it waits for the prefill to write its blocks. The reference
    scheduler keeps them (the prefill may still be pushing into them) until the connector reports the wait over,
    which it does once the prefill has said every push landed; then both sides have freed everything."""
    prefill = engines("kv_producer", "prefill-engine")
    decode = engines("kv_consumer", "decode-engine", accept_push=True)
    prompt = [50 + (i * 3) % 40 for i in range(21)]
    push_id = "push-9"
    decode_params = {"do_remote_prefill": True, "kv_push": True, "remote_request_id": push_id,
                     "remote_engine_id": "", "remote_host": "127.0.0.1",
                     "remote_port": prefill.config.kv_transfer.kv_port, "tp_size": 1, "remote_block_ids": []}
    decode.add(prompt, SamplingParams(max_tokens=2, ignore_eos=True, kv_transfer_params=decode_params), "d-9")
    decode.step()
    assert decode.scheduler.abort("d-9")
    assert decode.scheduler.block_manager.free_block_queue.num_free_blocks < BLOCKS  # held for the pushes
    prefill.add(prompt, SamplingParams(max_tokens=1, ignore_eos=True,
                                       kv_transfer_params={"do_remote_decode": True, "kv_push_id": push_id}), "p-9")
    step_until([prefill, decode], lambda out: decode.is_finished() and prefill.is_finished())
    assert decode.scheduler.block_manager.free_block_queue.num_free_blocks == BLOCKS
    assert prefill.scheduler.block_manager.free_block_queue.num_free_blocks == BLOCKS
    assert prefill.model_runner.worker.transport.posts  # the prefill did push into the held blocks


def test_the_prefill_s_released_blocks_stay_in_its_prefix_cache(engines):
    """Once the decode side has read them, the prefill engine frees the held blocks into its prefix cache: the same
    prompt served again there finds its full blocks cached."""
    prefill, decode = engines("kv_producer", "prefill-engine"), engines("kv_consumer", "decode-engine")
    prompt = [50 + (i * 5) % 30 for i in range(21)]
    prefill.add(prompt, SamplingParams(max_tokens=1, ignore_eos=True, kv_transfer_params={"do_remote_decode": True}),
                "p-4")
    outputs = step_until([prefill], lambda out: any(o.finished for o in out))
    params = next(o.kv_transfer_params for o in outputs if o.finished)
    decode.add(prompt, SamplingParams(max_tokens=1, ignore_eos=True, kv_transfer_params=params), "d-4")
    step_until([prefill, decode], lambda out: decode.is_finished() and prefill.is_finished())
    prefill.add(prompt, SamplingParams(max_tokens=1, ignore_eos=True), "again")
    prefill.step()
    assert prefill.model_runner.batches[-1] == [("again", len(prompt) - 2 * BLOCK)]  # two full blocks were hits
