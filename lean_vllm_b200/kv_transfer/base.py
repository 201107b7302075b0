"""The KV connector API of lean-vLLM (lean_vllm/kv_transfer/base.py), restated for this package.

Names, fields, defaults and semantics match the reference so that the connector here is a drop-in: a scheduler half
in the engine and a worker half per rank, KVConnectorMetadata down each step, KVConnectorOutput back, and the
aggregator's all-ranks rule. Objects of the reference's own classes work with the connector too (it only reads
attributes), which is how it plugs into an unmodified lean-vLLM engine.
"""

from __future__ import annotations

import uuid
from abc import ABC, abstractmethod
from collections import Counter
from dataclasses import dataclass, field
from typing import Literal

from pydantic import BaseModel, ConfigDict, TypeAdapter, ValidationError
from pydantic.dataclasses import dataclass as pydantic_dataclass

DEFAULT_CONNECTOR = "CudaIpcConnector"


@pydantic_dataclass(config=ConfigDict(extra="forbid"), slots=True)
class KVTransferConfig:
    """--kv-transfer-config as JSON (reference base.py:17-41). kv_producer serves prefilled KV, kv_consumer loads
    it, kv_both does either per request. Unknown keys are rejected."""

    kv_connector: str = DEFAULT_CONNECTOR
    kv_role: Literal["kv_producer", "kv_consumer", "kv_both"] = "kv_both"
    kv_ip: str = "127.0.0.1"  # where a producer answers handshakes, and the address it hands to consumers
    kv_port: int = 14579  # rank r answers on kv_port + r
    engine_id: str = field(default_factory=lambda: uuid.uuid4().hex)

    @classmethod
    def parse(cls, value) -> "KVTransferConfig":
        if isinstance(value, KVTransferConfig):
            return value
        adapter = TypeAdapter(cls)
        if isinstance(value, (str, bytes)):
            return adapter.validate_json(value)
        return adapter.validate_python(value)

    @property
    def is_producer(self) -> bool:
        return self.kv_role != "kv_consumer"

    @property
    def is_consumer(self) -> bool:
        return self.kv_role != "kv_producer"


class _RemotePrefill(BaseModel):
    """The kv_transfer_params a decode request must carry to load a remote prefill (reference base.py:43-53)."""

    model_config = ConfigDict(strict=True)  # wire input: a port given as "1" is refused

    remote_block_ids: list[int]
    remote_request_id: str
    remote_engine_id: str
    remote_host: str
    remote_port: int
    tp_size: int = 1


def check_kv_transfer_params(params, kv_transfer: KVTransferConfig | None) -> str | None:
    """Why an engine cannot honour a request's kv_transfer_params, or None (reference base.py:56-72)."""
    if not isinstance(params, dict):
        return "kv_transfer_params must be an object"
    if kv_transfer is None:
        return "kv_transfer_params needs an engine started with kv_transfer_config"
    role = kv_transfer.kv_role
    if params.get("do_remote_decode") and not kv_transfer.is_producer:
        return f"do_remote_decode needs kv_role kv_producer or kv_both, not {role}"
    if not params.get("do_remote_prefill"):
        return None
    if not kv_transfer.is_consumer:
        return f"do_remote_prefill needs kv_role kv_consumer or kv_both, not {role}"
    try:
        _RemotePrefill.model_validate(params)
    except ValidationError as error:
        first = error.errors()[0]
        where = ".".join(str(part) for part in first["loc"])
        return f"do_remote_prefill needs {where}: {first['msg']}"
    return None


@dataclass(slots=True)
class ReqToRecv:
    """A remote prefill's blocks and the local blocks they land in, aligned (reference base.py:75-85).

    `pushed` is this package's extension: the prefill instance writes the blocks itself, layer by layer as it
    computes them (ReqToSave on its side), and this rank only waits for its word that they have landed."""

    local_block_ids: list[int]
    remote_block_ids: list[int]
    remote_request_id: str
    remote_engine_id: str
    remote_host: str
    remote_port: int
    remote_tp_size: int = 1
    pushed: bool = False
    skip_blocks: int = 0  # pushed with no remote_block_ids: the prompt's leading blocks already cached here


@dataclass(slots=True)
class ReqToSave:
    """This package's extension (no counterpart in the reference): a request being prefilled here whose blocks are
    pushed, layer by layer during the prefill, into a decode instance's already allocated blocks. `local_block_ids`
    are this instance's, `remote_block_ids` the decode instance's, aligned; `remote_*` name the decode instance
    (its kv_ip, kv_port, engine_id and tensor-parallel size). With `push_id` and no remote_block_ids, the decode
    instance is not known yet: its ranks announce themselves and their blocks under that id."""

    local_block_ids: list[int]
    remote_block_ids: list[int] | None = None
    remote_engine_id: str = ""
    remote_host: str = ""
    remote_port: int = 0
    remote_tp_size: int = 1
    push_id: str | None = None
    cached_blocks: int = 0  # leading local blocks that were prefix-cache hits: no store of this prefill writes them
    num_tokens: int | None = None  # the prompt's tokens (None: every block full), so the last block's end is known


@dataclass(slots=True)
class KVConnectorMetadata:
    """One step's instructions for every worker half (reference base.py:88-96). `reqs_to_save` (requests this step
    prefills whose KV is pushed layer by layer) is this package's extension; it defaults to empty, so metadata built
    by the reference's scheduler half behaves exactly as there."""

    reqs_to_recv: dict[str, ReqToRecv] = field(default_factory=dict)
    reqs_to_send: dict[str, list[int]] = field(default_factory=dict)  # held blocks a decode instance may now read
    reqs_to_save: dict[str, ReqToSave] = field(default_factory=dict)
    # Of each request being saved: how many prompt tokens have KV once this step's layers have run. A per-layer save
    # pushes the blocks those tokens fill (a chunked prefill's later chunks push again what they add); without it,
    # everything is pushed at hand-over.
    save_progress: dict[str, int] = field(default_factory=dict)

    def __bool__(self):
        return bool(self.reqs_to_recv) or bool(self.reqs_to_send) or bool(self.reqs_to_save) or \
            bool(self.save_progress)


@dataclass(slots=True)
class KVTransferStats:
    """One load, from posting to the last byte landing (reference base.py:99-108)."""

    seconds: float
    num_bytes: int

    def merge(self, other: "KVTransferStats") -> "KVTransferStats":
        """Ranks load side by side: the slowest sets the time; bytes add up."""
        return KVTransferStats(max(self.seconds, other.seconds), self.num_bytes + other.num_bytes)


@dataclass(slots=True)
class KVConnectorOutput:
    """What a worker half finished since its last report (reference base.py:111-122)."""

    finished_sending: set[str] = field(default_factory=set)
    finished_recving: set[str] = field(default_factory=set)
    failed_recving: set[str] = field(default_factory=set)
    expired_sending: set[str] = field(default_factory=set)  # of finished_sending: freed with no consumer read
    recv_stats: dict[str, KVTransferStats] = field(default_factory=dict)  # of finished_recving

    def __bool__(self):
        return bool(self.finished_sending) or bool(self.finished_recving) or bool(self.failed_recving)


class KVOutputAggregator:
    """Per-request completion over all ranks: done once every rank reported it, failed if any rank's load failed
    (reference base.py:125-165)."""

    def __init__(self, world_size: int):
        self.world_size = world_size
        self._sent: Counter[str] = Counter()
        self._recved: Counter[str] = Counter()
        self._failed: set[str] = set()
        self._expired: set[str] = set()
        self._stats: dict[str, KVTransferStats] = {}

    def aggregate(self, outputs) -> KVConnectorOutput:
        result = KVConnectorOutput()
        for output in outputs:
            self._failed.update(output.failed_recving)
            self._expired.update(output.expired_sending)
            for request_id, stats in output.recv_stats.items():
                earlier = self._stats.get(request_id)
                self._stats[request_id] = stats if earlier is None else earlier.merge(stats)
            for request_id in output.finished_sending:
                self._sent[request_id] += 1
                if self._sent[request_id] < self.world_size:
                    continue
                del self._sent[request_id]
                result.finished_sending.add(request_id)
                if request_id in self._expired:
                    self._expired.remove(request_id)
                    result.expired_sending.add(request_id)
            for request_id in set(output.finished_recving) | set(output.failed_recving):
                self._recved[request_id] += 1
                if self._recved[request_id] < self.world_size:
                    continue
                del self._recved[request_id]
                stats = self._stats.pop(request_id, None)
                if request_id in self._failed:
                    self._failed.remove(request_id)
                    result.failed_recving.add(request_id)
                    continue
                result.finished_recving.add(request_id)
                if stats is not None:
                    result.recv_stats[request_id] = stats
        return result


class KVConnectorScheduler(ABC):
    """The engine's half; every method runs on the engine thread between steps (reference base.py:168-185)."""

    @abstractmethod
    def get_num_new_matched_tokens(self, seq, num_computed_tokens: int) -> tuple[int, bool]:
        """Prompt tokens past num_computed_tokens whose KV can come from elsewhere, and whether it loads async."""

    @abstractmethod
    def update_state_after_alloc(self, seq, num_external_tokens: int):
        """seq holds blocks for its prompt now; queue the load into those not already cached here."""

    @abstractmethod
    def build_connector_meta(self) -> KVConnectorMetadata:
        """This step's metadata for the workers; resets what it hands over."""

    @abstractmethod
    def request_finished(self, seq) -> tuple[bool, dict | None]:
        """Whether to hold seq's blocks until the workers report them sent, and the kv_transfer_params to return."""


class KVConnectorWorker(ABC):
    """One rank's half: moves blocks between this rank's KV cache and another instance's (reference base.py:188-204).

    save_kv_layer/wait_for_save are this package's optional layer-by-layer hooks (vLLM's names); the reference has
    no per-layer save, so they default to doing nothing.
    """

    @abstractmethod
    def register_kv_caches(self, kv_caches: list):
        """Each layer's cache, block index on dim 1, in model order. Called once, before any step."""

    @abstractmethod
    def start_load_kv(self, metadata: KVConnectorMetadata):
        """Start this step's loads and expose this step's sends. Must not block on the network."""

    @abstractmethod
    def get_finished(self) -> KVConnectorOutput:
        """Transfers finished on this rank since the last call."""

    def save_kv_layer(self, layer_index: int):
        """Called after layer `layer_index` stored this step's keys/values; may start moving them."""

    def wait_for_save(self):
        """Called at the end of a step's forward pass: saves started this step are ordered before what follows."""

    def shutdown(self):
        pass
