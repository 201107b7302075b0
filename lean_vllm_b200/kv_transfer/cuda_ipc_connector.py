"""CudaIpcConnector: the decode instance copies a finished prefill's blocks GPU to GPU over NVLink with kvx kernels.

A drop-in for lean-vLLM's NixlConnector (lean_vllm/kv_transfer/nixl_connector.py) on one NVSwitch node. The scheduler
half, the kv_transfer_params it returns, the handshake on kv_port + rank, the head shares between any two
tensor-parallel sizes, reader counting and the release/expiry rules are the reference's. What changes is below the
worker: instead of registering memory with a NIXL agent and posting one-sided READs, each rank exports its cache
through CUDA IPC in the handshake reply, maps the producer ranks' caches, and posts one kvx kernel launch per load
(a load finding none of the rank's copies in flight launches at once; behind copies in flight, the loads planned in
one pass share launches of up to 2 GiB), which gathers the shares' blocks from every
producer rank's HBM over NVLink and scatters them into its own blocks.
The launch waits on the stream for the load's ready event (no host synchronisation); a native watcher rings an
eventfd once the copy's event completes, and the transfer thread sleeps on that, its ZMQ socket and its work queue
together, so it wakes when a copy lands or a message or a load arrives rather than polling on a timer; and a
consumer rank tells each producer rank it read from once its bytes have landed (the NIXL notification's role) over
the same ZMQ channel as the handshake, in one message for all the loads that landed in one pass.

It adds a layer-by-layer push the reference does not have (its docs list vLLM's save_kv_layer as unsupported,
docs/disaggregated-prefill.md:29-30): given ReqToSave entries naming a decode instance's allocated blocks, a
prefill rank copies each layer's blocks into them from save_kv_layer while later layers compute, on a few SMs.
"""

from __future__ import annotations

import json
import logging
import os
import queue
import threading
from dataclasses import dataclass, field
from time import monotonic

import zmq

from lean_vllm_b200 import envs
from lean_vllm_b200.kv_transfer.base import (
    KVConnectorMetadata,
    KVConnectorOutput,
    KVConnectorScheduler,
    KVConnectorWorker,
    KVTransferStats,
    ReqToRecv,
    ReqToSave,
)
from lean_vllm_b200.kv_transfer.holds import Holds
from lean_vllm_b200.kv_transfer.shares import Share, head_shares, readers_of, split_heads
from lean_vllm_b200.kv_transfer.transport import CopyJob

logger = logging.getLogger(__name__)

HANDSHAKE_TIMEOUT = 5.0  # ZMQ never refuses a connect; an absent producer is one that does not answer
IDLE_WAIT = 0.01  # the transfer thread's longest sleep: deadlines are checked at least this often
BELL_WAIT = 0.001  # its sleep with copies in flight whose completion rings its doorbell (a safety net only)
BUSY_WAIT = 0.0002  # and with copies in flight on a transport without a doorbell, which it must poll
RELAY_WAIT = 60.0  # seconds a relayed load waits for its peer decode ranks' parts before it fails
RELAY_RING = 64  # slots of a decode rank's ring of relay events (kvx_transport.RELAY_RING)


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


def relay_parts(n_blocks: int, tp_size: int) -> list[tuple[int, int]]:
    """A relayed load's parts: decode rank r pulls block positions [first, end) of part r from the producer, the
    other parts from its peers. Contiguous, balanced to a block, and empty where there are fewer blocks than ranks."""
    return [(n_blocks * r // tp_size, n_blocks * (r + 1) // tp_size) for r in range(tp_size)]


def _ids_fit(block_ids, num_blocks: int) -> bool:
    """Every id names one of a cache's num_blocks blocks (no ids fit any cache)."""
    ids = list(block_ids or ())
    return not ids or (min(ids) >= 0 and max(ids) < num_blocks)


def _peer_mismatch(reply: dict, key, req, layout: dict, node: str) -> str | None:
    """Why a peer's handshake reply cannot serve this load, or None. The fields both sides of a deployment compare
    (nixl_connector.py:490-501, plus the node: CUDA IPC reaches only GPUs of one machine)."""
    where = f"{key[0]}:{key[1]}"
    checks = (
        (bool(req.remote_engine_id) and reply["engine_id"] != req.remote_engine_id,
         lambda: f"{where} is engine {reply['engine_id']}, not {req.remote_engine_id}"),
        (reply["tp_size"] != req.remote_tp_size,
         lambda: f"{where} runs tp_size {reply['tp_size']}, not {req.remote_tp_size}"),
        (reply["layout"] != json.loads(json.dumps(layout)),  # as the JSON round trip left the peer's
         lambda: f"{where} lays its KV cache out as {reply['layout']}, this engine as {layout}; "
                 "serve the same model, dtype and block size"),
        (reply.get("node") != node, lambda: f"{where} runs on another node; CUDA IPC needs both on one node"),
    )
    return next((message() for failed, message in checks if failed), None)


def node_id() -> str:
    """Identifies this machine's boot: CUDA IPC mappings work only between processes of one node."""
    try:
        with open("/proc/sys/kernel/random/boot_id") as f:
            return f.read().strip()
    except OSError:
        return os.uname().nodename


def make_transport(kv_caches):
    """The kvx transport for caches on a CUDA device (the reference's make_agent, nixl_connector.py:50-57)."""
    from lean_vllm_b200.kv_transfer.kvx_transport import KvxTransport

    return KvxTransport(kv_caches)


def _request_kind(params) -> str | None:
    """What a request's kv_transfer_params ask of this instance: "save" (a prefill whose decode instance waits for
    pushed blocks), "pull" (a decode that reads a finished prefill's blocks), "pushed" (a decode whose blocks will be
    pushed to it), or None (nothing to transfer)."""
    if not params:
        return None
    if params.get("do_remote_decode") and params.get("kv_push_id"):
        return "save"
    if params.get("do_remote_prefill"):
        return "pushed" if params.get("kv_push") else "pull"
    return None


class CudaIpcConnectorScheduler(KVConnectorScheduler):
    """The engine's half (the reference's NixlConnectorScheduler, nixl_connector.py:111-168): it admits loads,
    hands each step's work to the worker ranks as metadata, and describes a finished prefill's blocks to the proxy.

    Push mode adds two optional kv_transfer_params keys the reference does not have. A decode request sent before
    its prefill carries "kv_push": true (with remote_block_ids empty): it is admitted, allocated and left waiting,
    and its worker ranks announce its blocks to the prefill ranks. The prefill request carries "kv_push_id" (the
    decode request's remote_request_id): at its admission -- the reference scheduler asks the connector about every
    request right after allocating its blocks (engine/scheduler.py:193-196) -- this half hands the workers a
    ReqToSave, and they push the blocks as they are computed.
    """

    def __init__(self, config):
        self.kv_transfer = config.kv_transfer
        self.block_size = config.kvcache_block_size
        self.tp_size = config.tensor_parallel_size
        self._reqs_to_recv: dict[str, ReqToRecv] = {}
        self._reqs_to_send: dict[str, list[int]] = {}
        self._reqs_to_save: dict[str, ReqToSave] = {}
        self._saving: dict[str, object] = {}  # request -> its sequence while its prompt is prefilled under a save

    def _prompt_blocks(self, seq) -> int:
        return _cdiv(seq.num_prompt_tokens, self.block_size)

    def get_num_new_matched_tokens(self, seq, num_computed_tokens: int) -> tuple[int, bool]:
        """(tokens the decode instance will receive instead of computing, whether they arrive asynchronously)."""
        kind = _request_kind(seq.kv_transfer_params)
        if kind == "save":
            self._begin_save(seq, num_computed_tokens)
            return 0, False
        if kind is None or (kind == "pull" and not self._load_fits(seq)):
            return 0, False
        # Any split of heads between the two instances works: shares cover every tp_size pair.
        return seq.num_prompt_tokens - num_computed_tokens, True

    def _begin_save(self, seq, num_computed_tokens: int):
        """A prefill whose decode instance waits for a push: its blocks are allocated now, so they are saved."""
        self._reqs_to_save[seq.request_id] = ReqToSave(
            list(seq.block_table[: self._prompt_blocks(seq)]), push_id=str(seq.kv_transfer_params["kv_push_id"]),
            cached_blocks=num_computed_tokens // self.block_size, num_tokens=seq.num_prompt_tokens)
        self._saving[seq.request_id] = seq

    def _load_fits(self, seq) -> bool:
        """A pull must name one remote block per prompt block; otherwise the prompt is prefilled here."""
        params = seq.kv_transfer_params
        wanted, named = self._prompt_blocks(seq), len(params["remote_block_ids"])
        if named == wanted:
            return True
        logger.warning("prefilling %s here instead: %d remote blocks for a %d-block prompt", seq.request_id,
                       named, wanted)
        params["do_remote_prefill"] = False
        return False

    def update_state_after_alloc(self, seq, num_external_tokens: int):
        params = seq.kv_transfer_params
        params["do_remote_prefill"] = False  # one load per request: a preempted one recomputes
        skip = seq.num_cached_tokens // self.block_size  # blocks this instance already holds are not loaded again
        table = list(seq.block_table)
        if params.get("kv_push"):  # the producer learns the blocks from the workers' announcement
            local, remote = table[skip : self._prompt_blocks(seq)], []
        else:
            local, remote = table[skip:], list(params["remote_block_ids"][skip:])
        self._reqs_to_recv[seq.request_id] = ReqToRecv(
            local_block_ids=local, remote_block_ids=remote, remote_request_id=params["remote_request_id"],
            remote_engine_id=params["remote_engine_id"], remote_host=params["remote_host"],
            remote_port=params["remote_port"], remote_tp_size=params.get("tp_size", 1),
            pushed=bool(params.get("kv_push")), skip_blocks=skip if params.get("kv_push") else 0)

    def build_connector_meta(self) -> KVConnectorMetadata:
        """The step's work for the worker ranks. Built once per step after scheduling (engine/scheduler.py:147,
        260-263), so each saved prompt's progress -- its tokens with KV once this step runs -- lets per-layer
        saves push exactly what the step's chunk fills."""
        progress = {}
        for request_id, seq in list(self._saving.items()):
            progress[request_id] = min(seq.num_cached_tokens + seq.num_scheduled_tokens, seq.num_prompt_tokens)
            if progress[request_id] >= seq.num_prompt_tokens:
                del self._saving[request_id]
        metadata = KVConnectorMetadata(self._reqs_to_recv, self._reqs_to_send, self._reqs_to_save, progress)
        self._reqs_to_recv, self._reqs_to_send, self._reqs_to_save = {}, {}, {}
        return metadata

    def request_finished(self, seq) -> tuple[bool, dict | None]:
        """(whether the engine must keep the request's blocks for readers, the params a decode instance needs).
        Only a prefill that ran to its token (length or stop) hands over; an aborted one frees its blocks."""
        self._saving.pop(seq.request_id, None)
        params = seq.kv_transfer_params
        if not (params and params.get("do_remote_decode")) or seq.finish_reason not in ("length", "stop"):
            return False, None
        blocks = list(seq.block_table[: self._prompt_blocks(seq)])
        self._reqs_to_send[seq.request_id] = blocks
        return True, self._decode_params(seq.request_id, blocks)

    def _decode_params(self, request_id: str, blocks: list[int]) -> dict:
        """Where a decode instance reads this prefill's blocks from: the kv_transfer_params wire dict the proxy
        carries to it (nixl_connector.py:159-168, disagg_proxy.py:57-71)."""
        kv = self.kv_transfer
        where = {"remote_engine_id": kv.engine_id, "remote_host": kv.kv_ip, "remote_port": kv.kv_port,
                 "tp_size": self.tp_size}
        return {"do_remote_prefill": True, "do_remote_decode": False, "remote_request_id": request_id,
                "remote_block_ids": blocks, **where}


@dataclass(slots=True)
class _Remote:
    """A peer rank as its handshake described it, with its cache mapped here."""

    engine_id: str
    tp_size: int
    num_blocks: int
    exported: dict
    table: object  # the transport's view of the peer rank's cache, mapped into this process
    sock: object  # DEALER kept open for notifications
    per_block: dict = field(default_factory=dict)  # (share, latents) -> bytes one block of a load moves
    ring: list = field(default_factory=list)  # a peer decode rank's relay events, opened here (relayed loads)


@dataclass(slots=True)
class _Retired:
    """A peer rank's mapping replaced after the peer restarted under a new engine id. Copies and stores queued
    before the swap may still read or write it, so it closes only once every stream that can carry them has run
    past the swap: the engine's stream (its marker, recorded when the engine thread next polls) and each of the
    transport's streams (an empty transfer posted after that)."""

    remote: _Remote
    passed: bool = False  # the engine thread polled since: nothing it queues from then on names the mapping
    marker: object = None  # the engine stream's event at that poll
    fences: list | None = None  # empty transfers after the marker, one per transport stream


@dataclass(slots=True)
class _Batch:
    """One launch shared by the loads planned in one pass of the transfer thread."""

    xfer: object
    refs: int  # loads not yet finished with it; released at zero
    done: bool = False
    error: Exception | None = None


@dataclass(slots=True)
class _Relay:
    """A relayed latent load on one decode rank: its part of the blocks from the prefill rank, the rest from the
    other decode ranks of its instance once each has its own part."""

    parts: list  # (first, end) block positions of each decode rank's part
    transfer: _Batch | None = None  # the copy of the peers' parts
    waiting_since: float = field(default_factory=monotonic)
    ready: object = None  # the load's ready event: the peers' copy writes the same freshly allocated blocks
    own_done: bool = False  # this rank's own part has landed (or it had none)
    copied: bool = False  # the copy of the peers' parts has landed (or there was nothing to copy)
    peer_failed: bool = False  # a peer's part failed or never came: the load fails once nothing of it is in flight


@dataclass(slots=True)
class _Load:
    """One request's pull: one kernel launch over every share."""

    req: ReqToRecv
    transfer: _Batch | None = None
    request_id: str = ""
    notify: list = field(default_factory=list)  # (remote key, message, rank) to send once the bytes have landed
    unnotified: set = field(default_factory=set)  # producer ranks no notification has reached
    started: float = field(default_factory=monotonic)
    num_bytes: int = 0
    failed: bool = False
    relay: _Relay | None = None
    reported: bool = False  # launched by the engine thread, which saw it land and reported it (under the lock)


@dataclass(slots=True)
class _Save:
    """A request this producer rank pushes, layer by layer, into a decode instance's blocks."""

    req: ReqToSave
    targets: list  # (remote key, decode rank, [(share index, Share)]): the decode ranks that take heads from here
    tables: list = field(default_factory=list)  # their caches, mapped here, aligned with targets
    ready: bool = False  # every target mapped
    failed: bool = False
    progress: int | None = None  # prompt tokens with KV as of the latest step (None: unknown, push at hand-over)
    layer_blocks: dict = field(default_factory=dict)  # layer -> leading blocks already pushed in their final state
    inflight: int = 0  # launches not yet landed
    handed_over: bool = False  # the prefill is over (engine thread): no more per-layer pushes
    finishing: bool = False  # what was left is queued (transfer thread): done once nothing is in flight
    started: float = field(default_factory=monotonic)
    ready_marker: object = None  # the engine stream's event at hand-over, which the catch-up pushes wait for
    finish_seen: bool = False  # the transfer thread took the hand-over (and its ready_marker)
    fused: bool | None = None  # decided at its first store_kv: its rows go to the decode ranks with every store
    stored: set = field(default_factory=set)  # layers whose new rows store_kv pushed
    mapped: bool = False  # its blocks are in its decode instance's block map
    words: list = field(default_factory=list)  # _StoreWord of every fused store that wrote its rows


@dataclass(slots=True)
class _StoreWord:
    """The status word of one fused store launch, shared by the saves whose rows it pushed. Read once a save's
    last push or fence has completed (every store before it on the engine's stream has then completed too); closed
    when the last of those saves is done with it."""

    word: object
    refs: int


@dataclass(slots=True)
class _Wait:
    """A pushed load on a decode rank: it waits for every producer rank holding its heads to say they landed."""

    req: ReqToRecv
    expected: set
    num_bytes: int
    started: float = field(default_factory=monotonic)


class CudaIpcConnectorWorker(KVConnectorWorker):
    """One rank's half, as NixlConnectorWorker (nixl_connector.py:195-520) with the kvx transport under it.

    Pull (the reference's contract): a decode rank copies its heads of a finished prefill's blocks from every
    producer rank holding them, then notifies each. Push (this package's per-layer save): a prefill rank given
    ReqToSave in its metadata copies each layer's blocks into the decode ranks' blocks from save_kv_layer, beside the
    prefill's compute, and once the request is handed over and every copy has landed it tells each decode rank (which
    holds a ReqToRecv with pushed=True) and frees the blocks.
    """

    def __init__(self, config, rank: int):
        if config.kv_cache_layout != "HND":
            raise AssertionError("CudaIpcConnector copies heads out of blocks, so needs HND caches")
        self.kv_transfer = config.kv_transfer
        self.rank = rank
        self.tp_size = config.tensor_parallel_size
        self.block_size = config.kvcache_block_size
        self.accept_push = bool(getattr(config, "kvx_accept_push", False)) or envs.LEAN_VLLM_KVX_ACCEPT_PUSH
        self.relay = bool(getattr(config, "kvx_relay", False)) or envs.LEAN_VLLM_KVX_RELAY
        self.kv_caches: list = []
        self.num_heads = 0  # every rank's key heads together; 0 for a latent-only model
        self.layout: dict = {}
        self.layer_regions: list[tuple[int, int]] = []  # (first region, count) of each layer
        self.transport = None
        self.node = node_id()
        self._lock = threading.Lock()  # guards the maps below that both threads touch
        self._holds = Holds()  # producer: handed-over blocks kept for their readers; under the lock
        self._saves: dict[str, _Save] = {}  # producer: requests pushed layer by layer
        self._saved: dict[str, dict] = {}  # decode: request -> {producer rank: landed ok}, may precede the wait
        self._saved_seen: dict[str, float] = {}  # request -> when its first landing word came; under the lock
        self._push_ids: dict[str, str] = {}  # producer: push id -> request id, for saves awaiting their decode ranks
        self._expects: dict[str, dict] = {}  # producer: push id -> a decode rank's announcement, may come first
        self._finished = KVConnectorOutput()
        self._queue: queue.Queue = queue.Queue()
        self._wake = os.eventfd(0, os.EFD_NONBLOCK | os.EFD_CLOEXEC)  # written after every put: wakes the thread
        self._context = zmq.Context()
        self._context.setsockopt(zmq.LINGER, 0)
        self._server = None
        self._deferred: list = []  # messages that came while a handshake wait answered handshakes only
        self._remotes: dict[tuple[str, int], _Remote] = {}  # transfer thread only
        self._mapped: dict[tuple[str, int], tuple] = {}  # key -> (engine id, table, blocks, _Remote); locked
        self._launches_in_flight = 0  # load launches (either thread's) not yet seen landed; under the lock
        self._retired: list[_Retired] = []  # replaced mappings not yet closed; both threads, under the lock
        self._loads: dict[str, _Load] = {}  # transfer thread only
        self._inline: dict[str, _Load] = {}  # engine thread only: the loads it launched, until one side reports them
        self._share_plans: dict[int, list] = {}  # producer TP size -> [(Share, readers)] (engine thread)
        self.inline_loads = envs.LEAN_VLLM_KVX_INLINE_LOADS
        self._waits: dict[str, _Wait] = {}  # transfer thread only
        self._pushes: list = []  # (transfer, [saves]) in flight; both threads, under the lock
        self._relays: dict[str, _Load] = {}  # transfer thread only: loads past their own part, waiting for peers'
        self._parts: dict[str, dict] = {}  # request -> {decode rank: its part landed}; under the lock
        self._part_slots: dict[str, dict] = {}  # request -> {decode rank: ring slot marking its part, -1: none}
        self._ring_next = 0  # the next slot of this rank's relay ring (transfer thread only)
        self._parts_seen: dict[str, float] = {}  # request -> when its first part message came (transfer thread)
        self._block_maps: dict[tuple, object] = {}  # decode instance -> local block id -> its block id (engine thread)
        self._map_updates: list = []  # (instance, local ids, remote ids or None) for the engine thread to apply
        self._thread: threading.Thread | None = None
        self._errors_seen: dict = {}  # (step, error type) -> times the transfer thread hit it

    # -------------------------------------------------------------------------------------------- engine thread

    def register_kv_caches(self, kv_caches: list):
        self.kv_caches = list(kv_caches)
        layers, at = [], 0
        for cache in self.kv_caches:
            if cache.dim() == 5:  # keys and values, (2, block, head, token, dim)
                _, _, heads, tokens, dim = cache.shape
                self.num_heads = heads * self.tp_size
                layers.append(["kv", str(cache.dtype), self.num_heads, tokens, dim])
            else:  # latents, (1, block, token, dim)
                layers.append(["latent", str(cache.dtype), *cache.shape[2:]])
            self.layer_regions.append((at, cache.size(0)))
            at += cache.size(0)
        # What a peer must match: every rank's heads together, so the two sides may split them differently.
        self.layout = {"block_size": self.block_size, "layers": layers}
        self.transport = make_transport(self.kv_caches)
        if self.relay and self.tp_size > 1 and self.num_heads == 0 and hasattr(self.transport, "split_sms"):
            self.transport.split_sms()  # relayed latent loads copy on two streams at once
        kv = self.kv_transfer
        if kv.is_producer or self.accept_push or (self.relay and self.tp_size > 1):
            port = kv.kv_port + self.rank
            server = self._context.socket(zmq.ROUTER)
            try:
                server.bind(f"tcp://{kv.kv_ip}:{port}")
            except zmq.ZMQError as error:
                server.close()
                raise RuntimeError(f"cannot serve KV on {kv.kv_ip}:{port}: {error}; pick another kv_port") from error
            self._server = server
        self._thread = threading.Thread(target=self._run, name=f"kvx-ipc-{self.rank}", daemon=True)
        self._thread.start()

    def start_load_kv(self, metadata: KVConnectorMetadata):
        for request_id, req in getattr(metadata, "reqs_to_save", {}).items():
            with self._lock:
                old = self._saves.get(request_id)
                if old is not None and list(old.req.local_block_ids) == list(req.local_block_ids):
                    continue
                if old is not None:  # re-admitted after a preemption, in new blocks: start over
                    self._forget_fused(old)
                    self._saves.pop(request_id)
                    for entry in old.words:  # a store that wrote it may still run: its word is left open
                        entry.refs -= 1
                if req.remote_block_ids is None:  # its decode ranks announce themselves under req.push_id
                    self._saves[request_id] = _Save(req, [])
                    self._push_ids[str(req.push_id)] = request_id
                    self._put(("connect", request_id))
                    continue
                save = self._saves[request_id] = _Save(req, self._targets(req))
                # Decode ranks mapped by an earlier handshake: ready now, so this step's first layer is pushed by
                # its own hook. First contact goes to the transfer thread, never blocking this one on the network.
                mapped = [self._mapped.get(key) for key, _, _ in save.targets]
                if all(m is not None and m[0] == req.remote_engine_id for m in mapped):
                    if not all(_ids_fit(req.remote_block_ids, m[2]) for m in mapped):
                        save.failed = True  # its decode ranks hear "not ok" at hand-over
                        logger.warning("the decode blocks of %s lie past a decode rank's cache; not pushing them",
                                       request_id)
                        continue
                    save.tables = [m[1] for m in mapped]
                    save.ready = True
                    continue
            self._put(("connect", request_id))
        progress = getattr(metadata, "save_progress", None)
        if progress:
            with self._lock:
                for request_id, tokens in progress.items():
                    save = self._saves.get(request_id)
                    if save is not None:
                        save.progress = int(tokens)
        if metadata.reqs_to_send:
            deadline = monotonic() + envs.LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT
            finishing = []
            with self._lock:
                for request_id in metadata.reqs_to_send:
                    save = self._saves.get(request_id)
                    if save is not None:  # pushed: it finishes once its copies land, not by readers
                        save.handed_over = True
                        finishing.append(request_id)
                    elif self._holds.hold(request_id, deadline):  # every reader reported before the hand-over
                        self._finished.finished_sending.add(request_id)
            if finishing:
                ready = self.transport.ready_marker()
                for request_id in finishing:
                    self._put(("finish", request_id, ready))
        if metadata.reqs_to_recv:
            # Freshly allocated blocks may still be written by a step in flight; the copy waits for it on the GPU.
            # One queue item for the step's loads: the transfer thread plans them in one pass, so they share launches.
            loads = list(metadata.reqs_to_recv.items())
            if self._post_here(*loads[0]):
                loads = loads[1:]
            if loads:
                self._put(("loads", self.transport.ready_marker(), loads))

    def _post_here(self, request_id: str, req: ReqToRecv) -> bool:
        """Launches one load from the engine thread when none of this rank's copies is in flight and every producer
        rank it reads is mapped with the engine id it names: its copy starts without waiting for the transfer thread
        to wake. The thread then polls it and notifies the producers as for its own loads. Anything else -- a pushed
        or relayed load, a producer not yet mapped, an empty share, a bad block id, a refused launch -- returns False
        and the load goes to the thread, which plans it from the start (and fails it, if it must)."""
        if not self.inline_loads or getattr(req, "pushed", False) or self._relaying():
            return False
        try:
            shares = self._share_plan(req.remote_tp_size)
            keys = [(req.remote_host, req.remote_port + share.remote_rank) for share, _ in shares]
            with self._lock:
                if self._launches_in_flight:
                    return False
                # Read under the lock: a mapping _retire drops after this stays open until this engine thread has
                # polled again (get_finished) and every transport stream has run past that poll.
                remotes = [self._mapped.get(key) for key in keys]
            if not all(m is not None and (not req.remote_engine_id or m[0] == req.remote_engine_id) for m in remotes):
                return False
            load = _Load(req, request_id=request_id)
            jobs, tables = [], []
            for i, ((share, readers), key, mapped) in enumerate(zip(shares, keys, remotes)):
                job = CopyJob(len(tables) + 1, 0, req.remote_block_ids, req.local_block_ids, share.remote_head,
                              share.local_head, share.num_heads, i == 0)
                nbytes = self._job_bytes(mapped[3], job)
                if nbytes == 0:
                    return False
                tables.append(mapped[1])
                jobs.append(job)
                load.notify.append((key, f"{req.remote_request_id}:{readers}", share.remote_rank))
                load.unnotified.add(share.remote_rank)
                load.num_bytes += nbytes
            if not jobs:
                return False
            load.started = monotonic()
            # After the engine's stream as it stands (this is the engine thread): no ready event to create.
            load.transfer = _Batch(self.transport.post(tables, jobs, None, engine_order=True), 1)
        except Exception as error:  # noqa: BLE001 - the transfer thread plans it again and reports what is wrong
            logger.debug("load %s goes to the transfer thread: %s", request_id, error)
            return False
        with self._lock:
            self._launches_in_flight += 1
        self._inline[request_id] = load
        self._put(("posted", request_id, load))
        return True

    def _share_plan(self, remote_tp: int) -> list:
        """This rank's shares of a producer instance of `remote_tp` ranks, each with its reader count (the
        notification's), computed once per producer TP size: both depend on nothing else."""
        plan = self._share_plans.get(remote_tp)
        if plan is None:
            heads = split_heads(self.num_heads, self.tp_size, remote_tp)
            plan = self._share_plans[remote_tp] = [
                (share, readers_of(share.remote_rank, remote_tp, self.tp_size, heads))
                for share in head_shares(self.rank, self.tp_size, remote_tp, heads)]
        return plan

    def _finish_inline(self):
        """Engine thread, in get_finished: a load it launched whose copy has landed is reported here and now, without
        waiting for the transfer thread to wake (under a busy engine that can take a GIL switch interval). The
        thread still notifies its producers and lets the launch go; it lets it go under the lock, so the query here
        never meets a released transfer. A copy that failed is left to the thread."""
        with self._lock:
            for request_id, load in list(self._inline.items()):
                shared = load.transfer
                if shared is None or shared.done or load.failed:  # the thread has taken it from here
                    del self._inline[request_id]
                    continue
                try:
                    landed = self.transport.done(shared.xfer)
                except Exception:  # noqa: BLE001 - its own failure: the thread fails the load
                    del self._inline[request_id]
                    continue
                if landed:
                    del self._inline[request_id]
                    self._mark_landed(shared, locked=True)
                    load.reported = True
                    self._finished.finished_recving.add(request_id)
                    self._finished.recv_stats[request_id] = KVTransferStats(monotonic() - load.started,
                                                                            load.num_bytes)

    def save_kv_layer(self, layer_index: int):
        """Pushes layer `layer_index` of every request being saved whose decode ranks are mapped -- the blocks this
        step's chunk filled (its metadata's save_progress), from the first one not yet pushed in its final state --
        in one launch on the side stream after the layer's store (an event on the engine's stream), held to a few
        SMs. A block a chunk leaves partly filled is pushed again with the next chunk."""
        with self._lock:
            active = []
            for s in self._saves.values():
                if not s.ready or s.failed or s.handed_over or layer_index in s.stored or s.progress is None:
                    continue
                start, end, final = self._layer_span(s, layer_index)
                if end > start:
                    active.append((s, start, end))
                    s.layer_blocks[layer_index] = final
                    s.inflight += 1
            if not active:
                return
        saves = [entry[0] for entry in active]
        try:
            tables, jobs = self._push_jobs(active)
            ready = self.transport.ready_marker()
            xfer = self.transport.post(tables, jobs, ready, layer=self.layer_regions[layer_index],
                                       flags=self._save_flags(), save=True)
        except Exception as error:  # noqa: BLE001 - a failed save fails its loads, never the step
            logger.warning("pushing layer %d failed: %s", layer_index, error)
            with self._lock:
                for save in saves:
                    save.inflight -= 1
                    save.failed = True
            return
        with self._lock:
            self._pushes.append((xfer, saves))

    def wait_for_save(self):
        """Saves are ordered after their layers on the GPU and awaited on the transfer thread: nothing to do."""

    def get_finished(self) -> KVConnectorOutput:
        """What finished since the last call: the transfer thread fills the output as loads land and readers
        report; here held blocks past the abort timeout are given back, and the output is handed to the engine."""
        self._mark_swaps_passed()
        if self._inline:
            self._finish_inline()
        timeout = envs.LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT
        now = monotonic()
        with self._lock:
            for request_id in self._holds.expire(now):
                logger.warning("freeing the KV blocks of %s, which no decode instance read in %.0f s",
                               request_id, timeout)
                self._finished.finished_sending.add(request_id)
                self._finished.expired_sending.add(request_id)
            self._holds.forget_strays(now, timeout)
            out, self._finished = self._finished, KVConnectorOutput()
        return out

    def _mark_swaps_passed(self):
        """Every store and push the engine thread queued naming a replaced mapping is on a stream by now: the
        engine stream's event here is what the mapping's close waits for."""
        with self._lock:
            swapped = [r for r in self._retired if not r.passed]
        if not swapped:
            return
        marker = self.transport.ready_marker()
        with self._lock:
            for retired in swapped:
                retired.marker, retired.passed = marker, True

    def shutdown(self):
        """Stops the transfer thread -- which waits for the copies in flight before it closes any peer mapping --
        then the wake-up descriptor and the sockets. A second call does nothing."""
        if self._wake < 0:
            return
        if self._thread is not None:
            self._put(None)
            self._thread.join(timeout=10)
        wake, self._wake = self._wake, -1
        os.close(wake)
        self._context.term()

    def _relaying(self) -> bool:
        """Latent-only loads on a decode instance of several ranks are relayed (LEAN_VLLM_KVX_RELAY)."""
        return self.relay and self.tp_size > 1 and self.num_heads == 0

    def _heads(self, req) -> int:
        return split_heads(self.num_heads, self.tp_size, req.remote_tp_size)

    def _targets(self, req: ReqToSave) -> list:
        """The decode ranks that take heads from this rank, with those shares (seen from each decode rank)."""
        heads = self._heads(req)
        targets = []
        for decode_rank in range(req.remote_tp_size):
            shares = head_shares(decode_rank, req.remote_tp_size, self.tp_size, heads)
            mine = [(i, share) for i, share in enumerate(shares) if share.remote_rank == self.rank]
            if mine:
                targets.append(((req.remote_host, req.remote_port + decode_rank), decode_rank, mine))
        return targets

    def _layer_span(self, save: _Save, layer: int) -> tuple[int, int, int]:
        """Lock held. For a per-layer push of `layer`: the blocks [start, end) the save's progress has filled and not
        yet pushed in their final state, and how many leading blocks are final once they land."""
        total = len(save.req.local_block_ids)
        tokens = save.req.num_tokens if save.req.num_tokens is not None else total * self.block_size
        done = min(save.progress, tokens)
        end = min(_cdiv(done, self.block_size), total)
        final = end if done >= tokens else min(done // self.block_size, total)
        return save.layer_blocks.get(layer, 0), end, final

    def _push_jobs(self, spans: list) -> tuple[list, list]:
        """Copy jobs to every target decode rank for each (save, first block, end block) span."""
        tables, jobs = [], []
        for save, start, end in spans:
            local = list(save.req.local_block_ids)[start:end]
            remote = list(save.req.remote_block_ids)[start:end]
            for (key, _, mine), table in zip(save.targets, save.tables):
                tables.append(table)
                k = len(tables)
                for i, share in mine:
                    jobs.append(CopyJob(0, k, local, remote, share.remote_head, share.local_head, share.num_heads,
                                        i == 0))
        return tables, jobs

    # Fused store-and-push: the attention layer's store writes the decode ranks' blocks too.

    @staticmethod
    def _instance(req) -> tuple:
        return (req.remote_host, req.remote_port, req.remote_engine_id)

    def _forget_fused(self, save: _Save):
        """Lock held. Its blocks leave the block map before the engine can hand them to another request."""
        if save.mapped:
            self._map_updates.append((self._instance(save.req), list(save.req.local_block_ids), None))
            save.mapped = False

    def store_kv(self, layer_index: int, key, value, slot_mapping):
        """Stores this step's keys/values [tokens, heads, dim] of layer `layer_index` into this rank's cache by
        slot (the reference's store_kvcache, attention/triton_cache.py:58-81), and in the same pass into the decode
        ranks' blocks of every request being saved whose decode instance was mapped at its first store. An engine
        calls this in place of the backend's store; it then needs no save_kv_layer for those layers."""
        targets, word = self._fused_targets(layer_index, latents=False)
        self.transport.store(self.kv_caches[layer_index], key, value, slot_mapping, targets,
                             async_push=envs.LEAN_VLLM_KVX_FUSED_ASYNC, status=word)

    def store_latents(self, layer_index: int, latent, slot_mapping):
        """store_kv for an MLA layer's latents [tokens, 576] (attention/triton_cache.py:84-91); every decode rank
        takes a whole copy."""
        targets, word = self._fused_targets(layer_index, latents=True)
        self.transport.store(self.kv_caches[layer_index], latent, None, slot_mapping, targets,
                             async_push=envs.LEAN_VLLM_KVX_FUSED_ASYNC, status=word)

    def _fused_targets(self, layer_index: int, latents: bool) -> tuple[list, object]:
        """The peer destinations of this layer's store, and the status word the store reports into (None without
        peers): every save whose rows the store writes holds the word until it finishes."""
        with self._lock:
            updates, self._map_updates = self._map_updates, []
            groups: dict[tuple, _Save] = {}
            served: list[_Save] = []
            for save in self._saves.values():
                if save.failed or save.handed_over:
                    continue
                if save.fused is None:
                    save.fused = save.ready  # mapped before its first store, or never fused
                if not save.fused:
                    continue
                save.stored.add(layer_index)
                served.append(save)
                if not save.mapped:
                    updates.append((self._instance(save.req), list(save.req.local_block_ids),
                                    list(save.req.remote_block_ids)))
                    save.mapped = True
                groups.setdefault(self._instance(save.req), save)
        for instance, local_ids, remote_ids in updates:
            block_map = self._block_maps.get(instance)
            if block_map is None:
                block_map = self._block_maps[instance] = self.transport.new_block_map()
            self.transport.map_blocks(block_map, local_ids, remote_ids)
        targets = []
        start, _ = self.layer_regions[layer_index]
        for instance, save in groups.items():
            for (_, _, mine), table in zip(save.targets, save.tables):
                for i, share in mine:
                    if latents and i:
                        continue  # latents come whole from the first producer rank only
                    targets.append(self.transport.push_target(table, start, share, self._block_maps[instance],
                                                              self.block_size))
        if not targets:
            return targets, None
        word = _StoreWord(self.transport.status_word(), len(served))
        with self._lock:
            for save in served:
                save.words.append(word)
        return targets, word.word

    def _save_flags(self):
        return getattr(self.transport, "save_flags", None)

    # -------------------------------------------------------------------------------------------- transfer thread

    def _put(self, item):
        self._queue.put(item)
        if self._wake >= 0:  # closed at shutdown
            os.eventfd_write(self._wake, 1)

    def _run(self):
        try:
            self.transport.bind_thread()
            bell = getattr(self.transport, "doorbell", None)
            poller = zmq.Poller()
            poller.register(self._wake, zmq.POLLIN)
            if bell is not None:
                poller.register(bell.fd, zmq.POLLIN)
            if self._server is not None:
                poller.register(self._server, zmq.POLLIN)
            while True:
                busy = self._loads or self._pushes or self._relays
                if self._queue.empty():
                    # Sleep until a load is queued, a message comes, or (doorbell) a copy lands.
                    wait = (BELL_WAIT if bell is not None else BUSY_WAIT) if busy else IDLE_WAIT
                    poller.poll(wait * 1000)
                try:
                    os.eventfd_read(self._wake)  # before the queue is read: a put after this wakes the next poll
                except BlockingIOError:
                    pass
                if bell is not None:
                    bell.clear()  # before the copies are queried: a ring after this wakes the next poll
                items = []
                while True:
                    try:
                        items.append(self._queue.get_nowait())
                    except queue.Empty:
                        break
                if None in items:
                    for item in items:  # copies the engine thread launched: _close waits for them to land
                        if item is not None and item[0] == "posted":
                            self._loads[item[1]] = item[2]
                    return
                batch: list = []
                for item in items:
                    if item[0] == "loads":
                        for request_id, req in item[2]:
                            self._guarded(self._start, request_id, req, item[1], batch)
                    elif item[0] == "posted":  # launched by the engine thread (_post_here): polled from here on
                        self._loads[item[1]] = item[2]
                    elif item[0] == "connect":
                        self._guarded(self._connect, item[1])
                    elif item[0] == "finish":
                        self._guarded(self._finish, *item[1:])
                self._guarded(self._post_loads, batch)
                if self._server is not None:
                    self._guarded(self._serve)
                for poll in (self._poll, self._poll_relays, self._poll_pushes, self._poll_waits,
                             self._poll_retired):  # retired mappings last: after every post this pass made
                    self._guarded(poll)
        except zmq.ContextTerminated:
            pass
        finally:
            self._close()

    def _guarded(self, step, *args):
        """One step of the transfer thread. An error nothing below expected is logged (once per kind) and the thread
        goes on serving: if it ended, every load on this rank would wait for ever, since a decode engine has no
        deadline on a pull. Closing the context still ends the thread."""
        try:
            step(*args)
        except zmq.ContextTerminated:
            raise
        except Exception as error:  # noqa: BLE001
            kind = (getattr(step, "__name__", str(step)), type(error).__name__)  # bounded: no request ids
            times = self._errors_seen[kind] = self._errors_seen.get(kind, 0) + 1
            if times == 1:
                logger.exception("the KV transfer thread hit an unexpected error in %s and carries on", kind[0])
            elif times & (times - 1) == 0:  # 2, 4, 8, ...: a recurring error stays visible without flooding
                logger.warning("the KV transfer thread has hit %s in %s %d times", kind[1], kind[0], times)

    def _close(self):
        released = set()
        for load in self._loads.values():
            if load.transfer is not None and id(load.transfer) not in released:
                released.add(id(load.transfer))
                self.transport.wait(load.transfer.xfer)  # bytes still landing in blocks the engine would reuse
                self.transport.release(load.transfer.xfer)
        for xfer, _ in self._pushes:
            self.transport.wait(xfer)
            self.transport.release(xfer)
        for load in self._relays.values():
            if load.relay.transfer is not None:
                self.transport.wait(load.relay.transfer.xfer)
                self.transport.release(load.relay.transfer.xfer)
        drain = getattr(self.transport, "drain", None)
        if drain is not None:
            try:
                drain()  # the engine's own stores into peers' blocks, on streams this thread does not track
            except Exception as error:  # noqa: BLE001 - a device that failed runs nothing more: close regardless
                logger.warning("waiting for the device before closing KV mappings failed: %s", error)
        with self._lock:
            retired, self._retired = self._retired, []
        for entry in retired:
            for fence in entry.fences or []:
                self.transport.release(fence)
            self.transport.close(entry.remote.exported)
        for remote in self._remotes.values():
            self.transport.close(remote.exported)
            remote.sock.close()
        if self._server is not None:
            self._server.close()
        if hasattr(self.transport, "shutdown"):
            self.transport.shutdown()

    # Serving: handshakes, and the notifications that end reads (producer) or pushes (decode).

    def _serve(self, answer_only: bool = False):
        """Answers handshakes and takes notifications. While this thread waits for a peer's handshake reply it
        calls this with answer_only: handshakes are answered (the peer may be waiting on this rank at the same time,
        which would otherwise deadlock both until the timeout) and everything else is kept for later."""
        if not answer_only and self._deferred:
            deferred, self._deferred = self._deferred, []
            for identity, message in deferred:
                self._handle_one(identity, message)
        while True:
            try:
                identity, raw = self._server.recv_multipart(zmq.NOBLOCK)
            except zmq.Again:
                return
            except ValueError:
                continue
            try:
                message = json.loads(raw)
                message.get("op")
            except (ValueError, AttributeError):
                message = {}
            if answer_only and message.get("op") != "handshake":
                self._deferred.append((identity, message))
                continue
            self._handle_one(identity, message)

    def _handle_one(self, identity, message: dict):
        """A peer's message whose fields do not parse is dropped with a warning: it must not end this thread."""
        try:
            self._handle(identity, message)
        except zmq.ContextTerminated:
            raise
        except Exception as error:  # noqa: BLE001 - whatever a peer sends must not end this thread
            logger.warning("ignoring a malformed KV message %.200r: %s", message, error)

    def _handle(self, identity, message: dict):
        op = message.get("op")
        if op == "notify":  # one "req:readers" notification, or several a reader batched into one message
            batch = message.get("messages")
            for note in batch if isinstance(batch, list) else [message.get("message", "")]:
                self._count(str(note))
            return
        if op == "expect":
            push_id = str(message.get("push_id"))
            # Parsed here, so one that does not parse is dropped before _connect (which also runs from the queue).
            expect = {"skip": int(message.get("skip", 0)), "block_ids": [int(b) for b in message.get("block_ids", [])],
                      "engine_id": str(message.get("engine_id", "")), "host": str(message.get("host", "")),
                      "port": int(message.get("port", 0)), "tp_size": int(message.get("tp_size", 1))}
            if expect["tp_size"] < 1 or expect["skip"] < 0:
                raise ValueError("an announcement with tp_size below 1 or a negative skip")
            with self._lock:
                self._expects.setdefault(push_id, expect)
                request_id = self._push_ids.get(push_id)
            if request_id is not None:
                self._connect(request_id)
            return
        if op == "part":  # a peer decode rank posted its part (its ring slot), or its part landed (ok or not)
            request, rank = str(message.get("request")), int(message.get("rank", -1))
            with self._lock:
                if "slot" in message:
                    self._part_slots.setdefault(request, {})[rank] = int(message["slot"])
                if "ok" in message:
                    self._parts.setdefault(request, {})[rank] = bool(message["ok"])
            self._parts_seen.setdefault(request, monotonic())
            return
        if op == "saved":
            request = str(message.get("request"))
            with self._lock:
                self._saved.setdefault(request, {})[int(message.get("rank", -1))] = bool(message.get("ok"))
                self._saved_seen.setdefault(request, monotonic())
            return
        if op == "handshake":
            reply = {
                "ok": True,
                "engine_id": self.kv_transfer.engine_id,
                "tp_size": self.tp_size,
                "layout": self.layout,
                "num_blocks": int(self.kv_caches[0].size(1)),
                "exported": self.transport.exported,
                "node": self.node,
            }
            if self._relaying():
                reply["relay_ring"] = self.transport.relay_ring()
        else:
            reply = {"ok": False, "error": f"unknown op {op!r}"}
        try:
            self._server.send_multipart([identity, json.dumps(reply).encode()], zmq.NOBLOCK)
        except zmq.Again:
            logger.warning("a KV handshake went unanswered: its peer is not reading")

    def _count(self, message: str):
        try:
            request_id, readers = message.rsplit(":", 1)
            readers = int(readers)
        except ValueError:
            logger.warning("ignoring a malformed KV notification %r", message)
            return
        with self._lock:
            if self._holds.reported(request_id, readers, monotonic()):
                self._finished.finished_sending.add(request_id)

    # Pull: plan the step's loads, launch them (small ones together), then poll each launch once per pass.

    def _start(self, request_id: str, req: ReqToRecv, ready, batch: list):
        """Plans one load (handshakes, shares, byte count); `_post_loads` launches the batch."""
        if getattr(req, "pushed", False):
            self._start_wait(request_id, req)
            return
        load = self._loads[request_id] = _Load(req, request_id=request_id)
        try:
            heads = self._heads(req)
            shares: list[Share] = head_shares(self.rank, self.tp_size, req.remote_tp_size, heads)
            load.unnotified = {share.remote_rank for share in shares}
            if self._relaying():
                # Latents are whole on every decode rank: this rank pulls its part from the prefill rank and the
                # others' parts from them, so each byte crosses the prefill GPU's links once.
                load.relay = _Relay(relay_parts(len(req.local_block_ids), self.tp_size), ready=ready)
                for peer in range(self.tp_size):
                    if peer != self.rank:
                        self._handshake(self._peer_req(), peer)
            jobs, tables = [], []
            for i, share in enumerate(shares):
                remote = self._handshake(req, share.remote_rank)
                readers = readers_of(share.remote_rank, req.remote_tp_size, self.tp_size, heads)
                key = (req.remote_host, req.remote_port + share.remote_rank)
                message = f"{req.remote_request_id}:{readers}"
                # Latents come whole from the first producer rank only (nixl_connector.py:403).
                job = CopyJob(1, 0, req.remote_block_ids, req.local_block_ids, share.remote_head, share.local_head,
                              share.num_heads, i == 0)
                nbytes = self._job_bytes(remote, job)
                if load.relay is not None and i == 0:  # the whole payload counts; only this rank's part is read
                    load.num_bytes += nbytes
                    first, end = load.relay.parts[self.rank]
                    job = CopyJob(1, 0, req.remote_block_ids[first:end], req.local_block_ids[first:end],
                                  share.remote_head, share.local_head, share.num_heads, True)
                    nbytes = self._job_bytes(remote, job)
                    load.num_bytes -= nbytes
                if nbytes == 0:
                    self._notify(key, message)  # nothing to read from this rank, but it must count this reader
                    load.unnotified.discard(share.remote_rank)
                    continue
                tables.append(remote.table)
                job.src = len(tables)
                jobs.append(job)
                load.notify.append((key, message, share.remote_rank))
                load.num_bytes += nbytes
            load.started = monotonic()
            if not jobs and load.relay is not None:  # an empty part: nothing to mark, nothing to land
                del self._loads[request_id]
                self._relay_posted(load, -1)
                self._relay_landed(load)
                return
            if jobs:
                batch.append((load, tables, jobs, ready))
                # A load that finds none of this rank's copies in flight launches at once: its latency is the
                # device's alone. Behind copies in flight, loads share launches of up to BATCH_BYTES: fewer launches
                # leave fewer ramps and tails between them, and the device stays busy while later loads are planned.
                # A relayed load launches at once too: its peers wait for its part to land before they copy theirs.
                if (sum(entry[0].num_bytes for entry in batch) >= envs.LEAN_VLLM_KVX_BATCH_BYTES
                        or load.relay is not None or not self._copies_in_flight()):
                    self._post_loads(batch)
                    batch.clear()
        except Exception as error:  # noqa: BLE001 - every failure of a load becomes failed_recving
            self._fail(load, error)

    def _mark_landed(self, shared: _Batch, locked: bool = False):
        """The one place a launch is marked landed: the in-flight count drops once, whichever thread saw it."""
        if not locked:
            with self._lock:
                return self._mark_landed(shared, locked=True)
        if not shared.done:
            shared.done = True
            self._launches_in_flight -= 1

    def _copies_in_flight(self) -> bool:
        with self._lock:
            return self._launches_in_flight > 0

    def _job_bytes(self, remote: _Remote, job: CopyJob) -> int:
        """What the job moves: the reference's descriptor-length sum (nixl_connector.py:421). The bytes of one block
        come from the transport's planner once per producer rank and share (it checks the heads and regions); every
        load's block ids are range-checked here, as the planner would, so a bad id fails its own load before any
        launch."""
        src, dst = job.src_block_ids, job.dst_block_ids
        if len(src) != len(dst):
            raise ValueError(f"{len(src)} source blocks for {len(dst)} destination blocks")
        if not src:
            return 0
        if min(src) < 0 or max(src) >= remote.num_blocks:
            raise RuntimeError(f"a block id past the producer's {remote.num_blocks} blocks")
        local_blocks = int(self.kv_caches[0].size(1))
        if min(dst) < 0 or max(dst) >= local_blocks:
            raise RuntimeError(f"a block id past this rank's {local_blocks} blocks")
        key = (job.src_first_head, job.dst_first_head, job.num_heads, job.latents)
        per_block = remote.per_block.get(key)
        if per_block is None:
            one = CopyJob(job.src, job.dst, [0], [0], job.src_first_head, job.dst_first_head, job.num_heads,
                          job.latents)
            per_block = remote.per_block[key] = self.transport.job_bytes([remote.table], [one])
        return per_block * len(src)

    def _post_loads(self, batch: list):
        """One launch for every load planned in this pass that waits on the same ready event: their jobs share one
        kernel and one completion event, which each load polls."""
        groups: dict[int, list] = {}
        for entry in batch:
            groups.setdefault(id(entry[3]), []).append(entry)
        for entries in groups.values():
            tables, jobs, index = [], [], {}
            for _, load_tables, load_jobs, _ in entries:
                for job in load_jobs:
                    table = load_tables[job.src - 1]
                    if id(table) not in index:
                        tables.append(table)
                        index[id(table)] = len(tables)
                    jobs.append(CopyJob(index[id(table)], 0, job.src_block_ids, job.dst_block_ids, job.src_first_head,
                                        job.dst_first_head, job.num_heads, job.latents))
            relayed = [load for load, *_ in entries if load.relay is not None]
            slot = None
            if relayed:  # the launch is marked in this rank's ring, so the peers' copies of its part wait on the GPU
                slot, self._ring_next = self._ring_next, (self._ring_next + 1) % RELAY_RING
            try:
                shared = _Batch(self.transport.post(tables, jobs, entries[0][3], mark=slot), len(entries))
            except Exception as error:  # noqa: BLE001 - refused when posted: these loads fail, producers hear now
                for load, *_ in entries:
                    self._fail(load, error)
                continue
            with self._lock:
                self._launches_in_flight += 1
            for load, *_ in entries:
                load.transfer = shared
            for load in relayed:
                self._relay_posted(load, slot)

    def _poll(self):
        notes: dict[tuple, list] = {}  # producer rank -> the notifications of every load this pass finished
        try:
            self._poll_loads(notes)
        finally:
            for key, messages in notes.items():
                self._notify(key, *messages)

    def _poll_loads(self, notes: dict):
        queried: set[int] = set()  # launches asked once this pass: the loads sharing one finish together
        for request_id, load in list(self._loads.items()):
            try:
                if not self._landed(load, queried, notes):
                    continue
            except Exception as error:  # noqa: BLE001 - one load's trouble is that load's, never the others'
                if load.transfer is not None and not load.transfer.done:
                    self._note_error("_poll_loads", error)  # its copy may still write the blocks: ask again
                    continue
                self._fail(load, RuntimeError(f"finishing the load failed: {error}"), in_flight=True)
            del self._loads[request_id]
            if load.relay is not None and request_id in self._relays:
                self._relay_landed(load)  # the rest of the load is _poll_relays'
                continue
            self._finish_load(request_id, load)

    def _landed(self, load: _Load, queried: set, notes: dict) -> bool:
        """Whether the load's launch has ended (asked once per pass per launch); once it has, the launch is let go
        and, unless the copy failed, each producer rank's notification queued."""
        if load.transfer is None:
            return True
        shared = load.transfer
        if not shared.done and id(shared) not in queried:
            queried.add(id(shared))
            try:
                landed = self.transport.done(shared.xfer)
            except Exception as error:  # noqa: BLE001 - this launch's own failure (its status word, or CUDA)
                landed = True
                shared.error = shared.error or error
            if landed:
                self._mark_landed(shared)
        if not shared.done:
            return False
        if shared.error is not None:
            self._fail(load, RuntimeError(f"a kvx copy failed in flight: {shared.error}"), in_flight=True)
        load.transfer = None
        shared.refs -= 1
        if shared.refs == 0:
            with self._lock:  # the engine thread may be asking about it (_finish_inline)
                self.transport.release(shared.xfer)
        if not load.failed:
            for key, message, remote_rank in load.notify:
                notes.setdefault(key, []).append(message)
                load.unnotified.discard(remote_rank)
        return True

    def _note_error(self, where: str, error: Exception):
        """Counts an unexpected error the thread recovered from, logging it as _guarded does."""
        kind = (where, type(error).__name__)
        times = self._errors_seen[kind] = self._errors_seen.get(kind, 0) + 1
        if times == 1 or times & (times - 1) == 0:
            logger.warning("the KV transfer thread hit %s in %s (%d times): %s", kind[1], where, times, error)

    def _finish_load(self, request_id: str, load: _Load):
        if load.relay is not None:
            if load.failed:
                self._send_part(request_id, False)  # the peers' loads fail too, and prefill as this one does
            with self._lock:
                self._parts.pop(request_id, None)
                self._part_slots.pop(request_id, None)
            self._parts_seen.pop(request_id, None)
        with self._lock:
            if load.reported:  # the engine thread saw it land and reported it
                return
            if load.failed:
                self._finished.failed_recving.add(request_id)
            else:
                self._finished.finished_recving.add(request_id)
                self._finished.recv_stats[request_id] = KVTransferStats(monotonic() - load.started, load.num_bytes)

    # Relay: a decode rank's own part landed; the other parts come from its peer decode ranks.

    def _peer_req(self):
        """A peer decode rank of this instance as _handshake addresses a producer."""
        kv = self.kv_transfer
        return ReqToRecv([], [], "", kv.engine_id, kv.kv_ip, kv.kv_port, self.tp_size)

    def _send_part(self, request_id: str, ok: bool):
        kv = self.kv_transfer
        for peer in range(self.tp_size):
            if peer != self.rank:
                self._send((kv.kv_ip, kv.kv_port + peer), {"op": "part", "request": request_id, "rank": self.rank,
                                                             "ok": ok})

    def _relay_posted(self, load: _Load, slot: int):
        """Own part launched (marked with `slot` of this rank's ring; -1: nothing to wait for): the peers may queue
        their copies of it now, and this load is _poll_relays' from here on."""
        kv = self.kv_transfer
        for peer in range(self.tp_size):
            if peer != self.rank:
                self._send((kv.kv_ip, kv.kv_port + peer), {"op": "part", "request": load.request_id,
                                                             "rank": self.rank, "slot": slot})
        load.relay.waiting_since = monotonic()
        self._relays[load.request_id] = load

    def _relay_landed(self, load: _Load):
        """Own part landed: the peers learn whether their copies of it hold the producer's bytes."""
        load.relay.own_done = True
        self._send_part(load.request_id, not load.failed)

    def _poll_relays(self):
        """Relayed loads past their own part's launch. The copy of the peers' parts is queued as soon as every peer
        has said where its part's launch is marked (its ring slot), and waits for those marks and for the load's
        ready event on the GPU. The load ends once its own part and that copy have landed and every peer has said
        its part landed; any failure fails it on every rank, once nothing of it is still in flight."""
        timeout = RELAY_WAIT
        now = monotonic()
        for request_id, seen in list(self._parts_seen.items()):
            # Parts for a load this rank finished (or never had) long ago: nobody will read them.
            if request_id not in self._relays and request_id not in self._loads and seen + 2 * timeout < now:
                del self._parts_seen[request_id]
                with self._lock:
                    self._parts.pop(request_id, None)
                    self._part_slots.pop(request_id, None)
        peers = [r for r in range(self.tp_size) if r != self.rank]
        for request_id, load in list(self._relays.items()):
            relay = load.relay
            with self._lock:
                landed = dict(self._parts.get(request_id, {}))
                slots = dict(self._part_slots.get(request_id, {}))
            # A peer's failure is kept apart from this rank's own: its own part still lands and notifies the
            # producer, and the load fails when it ends.
            if any(landed.get(r) is False for r in peers) and not relay.peer_failed:
                relay.peer_failed = True
                logger.warning("a peer decode rank could not load its part of %s, so it prefills here",
                               load.req.remote_request_id)
            if relay.transfer is None and not relay.copied and not load.failed and not relay.peer_failed:
                # A peer whose ring is not open here (in this process on another GPU) is copied from once its part
                # landed; the others as soon as their launches are marked.
                if all(r in slots for r in peers) and all(self._peer_ring(r) or landed.get(r) is True
                                                          or relay.parts[r][1] <= relay.parts[r][0] for r in peers):
                    self._copy_peer_parts(load, slots)
                elif relay.waiting_since + timeout < now:
                    relay.peer_failed = True
                    logger.warning("the peer decode ranks never reported their parts of %s",
                                   load.req.remote_request_id)
            if relay.transfer is not None:
                try:
                    if not self.transport.done(relay.transfer.xfer):
                        continue
                except Exception as error:  # noqa: BLE001
                    logger.warning("copying the peers' parts of %s failed in flight: %s", load.req.remote_request_id,
                                   error)
                    load.failed = True
                self.transport.release(relay.transfer.xfer)
                relay.transfer = None
                relay.copied = True
            if not relay.own_done:
                continue  # its own copy may still write the blocks
            healthy = not load.failed and not relay.peer_failed
            if healthy and not relay.copied:
                continue
            if healthy and not all(landed.get(r) is True for r in peers):
                if relay.waiting_since + timeout >= now:
                    continue
                relay.peer_failed = True
                logger.warning("the peer decode ranks never said their parts of %s landed",
                               load.req.remote_request_id)
            load.failed = load.failed or relay.peer_failed
            del self._relays[request_id]
            self._finish_load(request_id, load)

    def _peer_ring(self, rank: int) -> list:
        kv = self.kv_transfer
        remote = self._remotes.get((kv.kv_ip, kv.kv_port + rank))
        return remote.ring if remote is not None else []

    def _copy_peer_parts(self, load: _Load, slots: dict):
        """Queues the copy of every peer's part from its cache into this rank's blocks, after the peers' ring marks
        and the load's ready event."""
        kv = self.kv_transfer
        relay = load.relay
        tables, jobs, marks = [], [], []
        local = list(load.req.local_block_ids)
        for r, slot in sorted(slots.items()):
            first, end = relay.parts[r]
            if end <= first:
                continue
            remote = self._remotes[(kv.kv_ip, kv.kv_port + r)]
            tables.append(remote.table)
            jobs.append(CopyJob(len(tables), 0, local[first:end], local[first:end], 0, 0, 0, True))
            if slot >= 0 and remote.ring:
                marks.append(remote.ring[slot])
        if not jobs:
            relay.copied = True
            return
        try:
            relay.transfer = _Batch(self.transport.post(tables, jobs, relay.ready, relay=True, after=marks), 1)
        except Exception as error:  # noqa: BLE001
            logger.warning("copying the peers' parts of %s failed: %s", load.req.remote_request_id, error)
            load.failed = True

    def _send(self, key, message: dict):
        remote = self._remotes.get(key)
        if remote is None:
            return
        try:
            remote.sock.send(json.dumps(message).encode(), zmq.NOBLOCK)
        except zmq.ZMQError as error:  # the peer times out instead
            logger.debug("notifying %s:%d failed: %s", key[0], key[1], error)

    def _notify(self, key, *messages: str):
        """Reader notifications for one producer rank (the NIXL notification's role): the loads that finished in one
        pass of this thread share one message, which costs a socket send rather than one per load."""
        if len(messages) == 1:
            self._send(key, {"op": "notify", "message": messages[0]})
        elif messages:
            self._send(key, {"op": "notify", "messages": list(messages)})

    def _fail(self, load: _Load, error: Exception, in_flight: bool = False):
        req = load.req
        if load.relay is not None and not load.failed:
            self._send_part(load.request_id, False)
        if not load.failed:
            logger.warning("loading the KV of %s from %s:%d failed, so it prefills here: %s",
                           req.remote_request_id, req.remote_host, req.remote_port, error)
        load.failed = True
        if in_flight:
            return  # bytes may still be landing from those ranks: their blocks expire at the timeout instead
        # Producer ranks no copy reached free their blocks now rather than at the timeout, where they are known.
        for remote_rank in list(load.unnotified):
            key = (req.remote_host, req.remote_port + remote_rank)
            remote = self._remotes.get(key)
            if remote is not None and remote.engine_id == req.remote_engine_id:
                readers = readers_of(remote_rank, req.remote_tp_size, self.tp_size, self._heads(req))
                self._notify(key, f"{req.remote_request_id}:{readers}")
            load.unnotified.discard(remote_rank)
        load.notify = []

    # Push, producer side: map the decode ranks, catch up on layers no save_kv_layer pushed, report landing.

    def _connect(self, request_id: str):
        """Maps the decode ranks of a save (once its decode instance is known), then advances it."""
        with self._lock:
            save = self._saves.get(request_id)
            if save is None or save.ready or save.failed:
                return
            if save.req.remote_block_ids is None:
                expect = self._expects.pop(str(save.req.push_id), None)
                if expect is None:
                    return  # its decode ranks have not announced themselves yet
                self._push_ids.pop(str(save.req.push_id), None)
                skip, remote_ids = expect["skip"], expect["block_ids"]
                local_ids = list(save.req.local_block_ids)[skip:]
                save.req = ReqToSave(local_ids, remote_ids, expect["engine_id"], expect["host"], expect["port"],
                                     expect["tp_size"], save.req.push_id, max(save.req.cached_blocks - skip, 0))
                save.targets = self._targets(save.req)
                if len(local_ids) != len(remote_ids):
                    save.failed = True  # still mapped below, so the decode ranks hear that nothing comes
                    logger.warning("the decode instance announced %d blocks for %s, which has %d here",
                                   len(remote_ids), request_id, len(local_ids))
        try:
            remotes = [self._handshake(save.req, decode_rank) for _, decode_rank, _ in save.targets]
            if not all(_ids_fit(save.req.remote_block_ids, r.num_blocks) for r in remotes):
                # Checked here, before any block map names them: a store would skip such rows on the device.
                raise RuntimeError("a decode block id lies past the decode rank's cache")
            with self._lock:
                save.tables = [r.table for r in remotes]
                save.ready = not save.failed
        except Exception as error:  # noqa: BLE001
            logger.warning("cannot push the KV of %s to %s:%d, so the decode instance prefills it: %s",
                           request_id, save.req.remote_host, save.req.remote_port, error)
            with self._lock:
                save.failed = True
        self._advance(request_id)

    def _finish(self, request_id: str, ready):
        with self._lock:
            save = self._saves.get(request_id)
            if save is not None:
                save.ready_marker = ready
                save.finish_seen = True
        self._advance(request_id)

    def _advance(self, request_id: str):
        """A handed-over save whose decode ranks are mapped: push the layers no save_kv_layer reached (all of them
        for an engine without layer hooks) and let it finish once they land. One whose mapping failed finishes at
        once; one still waiting for its decode instance waits (and expires at the timeout)."""
        with self._lock:
            save = self._saves.get(request_id)
            if save is None or not save.finish_seen or save.finishing:
                return
            if not save.failed and not save.ready:
                return
            total = len(save.req.local_block_ids)
            # What no per-layer push covered: each layer's blocks from its first one not pushed in its final state.
            starts: dict[int, list] = {}
            if not save.failed:
                for layer in range(len(self.layer_regions)):
                    if layer not in save.stored and save.layer_blocks.get(layer, 0) < total:
                        starts.setdefault(save.layer_blocks.get(layer, 0), []).append(layer)
                        save.layer_blocks[layer] = total
            # Fused stores wrote only this prefill's new rows: prefix-cache hits need a copy of their own.
            cached = 0
            if not save.failed and save.stored:
                cached = min(save.req.cached_blocks, total)
            ready = save.ready_marker
        posts = []  # (layer or None for all, first block, end block)
        for start, layers in sorted(starts.items()):
            if len(layers) == len(self.layer_regions):
                posts.append((None, start, total))  # one launch for every layer
            else:
                posts += [(layer, start, total) for layer in layers]
        if cached:
            posts.append((None, 0, cached))
        missing = bool(starts)
        for layer, start, end in posts:
            with self._lock:
                save.inflight += 1
            try:
                tables, jobs = self._push_jobs([(save, start, end)])
                region = None if layer is None else self.layer_regions[layer]
                xfer = self.transport.post(tables, jobs, ready, layer=region, save=True)
            except Exception as error:  # noqa: BLE001
                logger.warning("pushing the KV of %s failed: %s", request_id, error)
                with self._lock:
                    save.inflight -= 1
                    save.failed = True
                break
            with self._lock:
                self._pushes.append((xfer, [save]))
        if save.stored and not (missing or cached) and not save.failed:
            # Every layer was stored fused, on the engine's stream: the decode ranks hear once those stores landed.
            try:
                xfer = self.transport.fence(ready)
            except Exception as error:  # noqa: BLE001
                logger.warning("waiting for the stores of %s failed: %s", request_id, error)
                with self._lock:
                    save.failed = True
            else:
                with self._lock:
                    save.inflight += 1
                    self._pushes.append((xfer, [save]))
        with self._lock:
            save.finishing = True

    def _poll_pushes(self):
        with self._lock:
            pushes = list(self._pushes)
        for entry in pushes:
            xfer, saves = entry
            try:
                if not self.transport.done(xfer):
                    continue
                failed = False
            except Exception as error:  # noqa: BLE001
                logger.warning("a kvx push failed in flight: %s", error)
                failed = True
            self.transport.release(xfer)
            with self._lock:
                self._pushes.remove(entry)
                for save in saves:
                    save.inflight -= 1
                    save.failed |= failed
        timeout = envs.LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT
        now = monotonic()
        with self._lock:
            done = [(rid, s) for rid, s in self._saves.items() if s.finishing and s.inflight == 0]
            stale = [(rid, s) for rid, s in self._saves.items()
                     if not s.finishing and s.inflight == 0 and s.started + timeout < now]
            for request_id, save in done:
                del self._saves[request_id]
                self._forget_fused(save)
                if self._settle_words(save):
                    save.failed = True
                    logger.warning("a fused store skipped rows of %s that lie past a decode rank's cache, so the "
                                   "decode instance prefills it", request_id)
                self._finished.finished_sending.add(request_id)  # every byte landed, or none will
            for request_id, save in stale:
                # Never handed over (an aborted prefill), or handed over to a decode instance that never announced
                # itself: the held blocks are freed as the reference frees unread ones.
                del self._saves[request_id]
                self._forget_fused(save)
                self._push_ids.pop(str(save.req.push_id), None)
                self._settle_words(save)  # idle past the abort timeout: its stores have long completed
                save.failed = True
                if save.handed_over:
                    self._finished.finished_sending.add(request_id)
                    self._finished.expired_sending.add(request_id)
            for push_id, expect in list(self._expects.items()):
                if expect.setdefault("_seen", now) + timeout < now:
                    del self._expects[push_id]  # announced for a prefill that never came here
        for request_id, save in done + stale:
            tag = save.req.push_id or request_id
            for key, _, _ in save.targets:
                self._send(key, {"op": "saved", "request": tag, "rank": self.rank, "ok": not save.failed})

    @staticmethod
    def _settle_words(save: _Save) -> bool:
        """Lock held, once every store that wrote the save's rows has completed: whether one of them skipped a row
        (its status word is set). The save lets go of each word; the last save to do so closes it."""
        skipped = False
        for entry in save.words:
            skipped |= entry.word.bits() != 0
            entry.refs -= 1
            if entry.refs == 0:
                entry.word.close()
        save.words = []
        return skipped

    # Push, decode side: wait for every producer rank holding this rank's heads.

    def _start_wait(self, request_id: str, req: ReqToRecv):
        heads = self._heads(req)
        shares = head_shares(self.rank, self.tp_size, req.remote_tp_size, heads)
        if not req.remote_block_ids:
            # The prefill instance does not know where to push yet: announce these blocks to every producer rank
            # holding this rank's heads, under the push id (the load's remote_request_id).
            kv = self.kv_transfer
            announcement = {"op": "expect", "push_id": req.remote_request_id, "block_ids": list(req.local_block_ids),
                            "skip": req.skip_blocks, "engine_id": kv.engine_id, "host": kv.kv_ip,
                            "port": kv.kv_port, "tp_size": self.tp_size}
            try:
                for share in shares:
                    self._handshake(req, share.remote_rank, fresh=True)
                    self._send((req.remote_host, req.remote_port + share.remote_rank), announcement)
            except Exception as error:  # noqa: BLE001
                logger.warning("cannot announce %s to %s:%d, so it prefills here: %s", req.remote_request_id,
                               req.remote_host, req.remote_port, error)
                with self._lock:
                    self._finished.failed_recving.add(request_id)
                return
        num_bytes = 0
        for i, share in enumerate(shares):
            for cache in self.kv_caches:
                if cache.dim() == 5:
                    num_bytes += 2 * len(req.local_block_ids) * share.num_heads * cache[0, 0, 0].numel() * \
                        cache.element_size()
                elif i == 0:
                    num_bytes += len(req.local_block_ids) * cache[0, 0].numel() * cache.element_size()
        self._waits[request_id] = _Wait(req, {share.remote_rank for share in shares}, num_bytes)

    def _poll_waits(self):
        timeout = envs.LEAN_VLLM_KV_ABORT_REQUEST_TIMEOUT
        now = monotonic()
        for request_id, wait in list(self._waits.items()):
            with self._lock:
                saved = self._saved.get(wait.req.remote_request_id, {})
                complete = wait.expected <= set(saved)
                ok = complete and all(saved[rank] for rank in wait.expected)
                if complete:
                    self._saved.pop(wait.req.remote_request_id, None)
                    self._saved_seen.pop(wait.req.remote_request_id, None)
            if not complete and wait.started + timeout >= now:
                continue
            del self._waits[request_id]
            with self._lock:
                if ok:
                    self._finished.finished_recving.add(request_id)
                    self._finished.recv_stats[request_id] = KVTransferStats(now - wait.started, wait.num_bytes)
                else:
                    logger.warning("the pushed KV of %s did not land, so it prefills here", wait.req.remote_request_id)
                    self._finished.failed_recving.add(request_id)
        awaited = {wait.req.remote_request_id for wait in self._waits.values()}
        with self._lock:
            for request, seen in list(self._saved_seen.items()):
                if request not in awaited and seen + timeout < now:
                    # Landing words no wait here took (an aborted decode request, or one for the instance that ran
                    # on this port before): dropped as unread prefill blocks are.
                    del self._saved_seen[request]
                    self._saved.pop(request, None)

    def _handshake(self, req, remote_rank: int, fresh: bool = False) -> _Remote:
        """The peer rank's cache, asked for once per peer and mapped here, checked to match this engine. An empty
        remote_engine_id accepts whichever engine answers; `fresh` asks again even if one is mapped, to see a
        restart (for a load that names no engine id)."""
        key = (req.remote_host, req.remote_port + remote_rank)
        known = self._remotes.get(key)
        if known is not None:
            if fresh:
                still = self._ask(key)["engine_id"] == known.engine_id
            else:
                still = not req.remote_engine_id or known.engine_id == req.remote_engine_id
            if still:
                return known
            self._retire(key, known)  # the peer restarted under a new engine id: ask afresh
        sock = self._dealer(key)
        try:
            reply = self._round_trip(sock, key)
            problem = _peer_mismatch(reply, key, req, self.layout, self.node)
            if problem:
                raise RuntimeError(problem)
            remote = _Remote(reply["engine_id"], reply["tp_size"], reply["num_blocks"], reply["exported"],
                             self.transport.open(reply["exported"]), sock)
            if reply.get("relay_ring") and self._relaying():
                remote.ring = self.transport.open_ring(reply["relay_ring"])
        except BaseException:
            sock.close()
            raise
        self._remotes[key] = remote  # its socket stays open for notifications
        with self._lock:
            self._mapped[key] = (remote.engine_id, remote.table, remote.num_blocks, remote)
        return remote

    def _dealer(self, key):
        sock = self._context.socket(zmq.DEALER)
        sock.rcvtimeo = sock.sndtimeo = int(HANDSHAKE_TIMEOUT * 1000)
        sock.connect(f"tcp://{key[0]}:{key[1]}")
        return sock

    def _round_trip(self, sock, key) -> dict:
        """Sends a handshake and returns the peer's accepted reply. While waiting, handshakes addressed to this rank
        are answered (the peer may be waiting on this rank at the same time, which would otherwise hold both until
        the timeout)."""
        sock.send(json.dumps({"op": "handshake"}).encode())
        deadline = monotonic() + HANDSHAKE_TIMEOUT
        while not sock.poll(timeout=2):
            if self._server is not None:
                self._serve(answer_only=True)
            if monotonic() > deadline:
                raise ConnectionError(f"{key[0]}:{key[1]} did not answer the handshake")
        reply = json.loads(sock.recv())
        if not reply.get("ok"):
            raise RuntimeError(reply.get("error", "handshake refused"))
        return reply

    def _retire(self, key, remote: _Remote):
        """Drops a peer rank that restarted under a new engine id. Its old mapping stays open until nothing queued
        can reach it (_poll_retired); saves pushing into it fail now, so no later store or push names it."""
        del self._remotes[key]
        remote.sock.close()
        with self._lock:
            self._mapped.pop(key, None)
            for save in self._saves.values():
                if any(table is remote.table for table in save.tables):
                    save.failed = True  # its decode instance is gone: the one now at that port hears "not ok"
            self._retired.append(_Retired(remote))

    def _poll_retired(self):
        """Closes replaced mappings once the engine thread has polled since the swap and every transport stream has
        run past that poll's marker."""
        with self._lock:
            retired = [r for r in self._retired if r.passed]
        for entry in retired:
            close = False
            try:
                if entry.fences is None:
                    entry.fences = list(self.transport.fences(entry.marker))
                    continue
                if not all(self.transport.done(fence) for fence in entry.fences):
                    continue
                close = True
            except Exception as error:  # noqa: BLE001 - a mapping kept open is harmless; one closed early is not
                logger.warning("keeping a replaced KV mapping open: %s", error)
            for fence in entry.fences or []:  # none when the transport refused to post them
                self.transport.release(fence)
            if close:
                self.transport.close(entry.remote.exported)
            with self._lock:
                self._retired.remove(entry)

    def _ask(self, key) -> dict:
        """One handshake round trip on a socket of its own, for its reply only."""
        sock = self._dealer(key)
        try:
            return self._round_trip(sock, key)
        finally:
            sock.close()
