/*
 * kvx -- B200-native KV-cache transfer for disaggregated prefill -> decode (C ABI).
 *
 * This library replaces the NIXL/UCX transport under lean-vLLM's NixlConnector
 * (lean_vllm/kv_transfer/nixl_connector.py) on one NVSwitch node. Each entry point below names the NIXL agent call
 * (or the reference code) it stands in for. All functions are plain C: pointers, sizes and int status codes; no
 * exceptions cross the boundary. `stream` is a cudaStream_t passed as void* (0 is the legacy default stream).
 *
 * A transfer is described exactly as NixlConnectorWorker describes its READs:
 *   - a cache is a list of regions, one per K, V or latent tensor of one layer (Region, nixl_connector.py:80-86);
 *   - a job is one READ of one request: the blocks to take from one producer rank's cache (src) and where they
 *     land in a consumer rank's cache (dst), and which heads (one Share of head_shares, nixl_connector.py:60-77);
 *   - job j copies, for every region r and every i < n_blocks, num_heads*head_bytes bytes from
 *       src.regions[r].addr + src_block_ids[i]*src.block_bytes + src_first_head*src.head_bytes
 *     to
 *       dst.regions[r].addr + dst_block_ids[i]*dst.block_bytes + dst_first_head*dst.head_bytes,
 *     or whole blocks for latent regions (head_bytes == 0) when `latents` is set, nothing for them otherwise --
 *     the byte map of block_descs (nixl_connector.py:89-108) applied to both sides of the READ (:404-417).
 * Block ids and region tables are read from host memory at call time and travel inside the kernel launch, so no
 * call here needs device scratch memory or a host-to-device copy of its own.
 */
#ifndef KVX_H
#define KVX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KVX_ABI_VERSION 2

/* Status codes. Every entry point returns one; kvx_last_error() describes the last failure on this thread. */
#define KVX_OK 0
#define KVX_PENDING 1          /* kvx_check_xfer: still in flight (NIXL's "PROC", nixl_connector.py:434) */
#define KVX_ERR_INVALID (-1)   /* a bad argument */
#define KVX_ERR_CUDA (-2)      /* a CUDA call failed */
#define KVX_ERR_RANGE (-3)     /* a block id or head range outside its cache (nixl_connector.py:398-399) */
#define KVX_ERR_DEVICE (-4)    /* a transfer's copy gave up a bounded wait (its status word says so) */
#define KVX_ERR_TIMEOUT (-5)   /* a host wait ran out (a rank that never posted its step) */

/* kvx_copy/kvx_transfer/kvx_pack/kvx_push/kvx_scatter flags word: bits 0-7 engine (below), bits 8-15 log2 of the
 * tile size (0: 32 KiB), bits 16-23 CTAs per SM (0: 1 for TMA, 2 for LSU), bits 24-31 how many SMs the grid may
 * cover (0: every SM; a copy that runs beside compute can be held to a few). */
/* Copy engines (low byte of flags). */
#define KVX_ENGINE_AUTO 0      /* TMA bulk copies when every address and length is 16-byte aligned, else LSU */
#define KVX_ENGINE_LSU 1       /* vectorised ld/st through the SMs' load/store units */
#define KVX_ENGINE_TMA 2       /* cp.async.bulk global->smem->global, one issuing thread per CTA */

/* One K, V or latent tensor of one layer. Mirrors Region (nixl_connector.py:80-86). */
typedef struct kvx_region {
    uint64_t addr;        /* device address of block 0 (this process's mapping; a peer's via kvx_ipc_open) */
    uint64_t block_bytes; /* bytes between consecutive blocks */
    uint64_t head_bytes;  /* bytes of one head's tokens in a block; 0 for latents */
} kvx_region;

/* One side of a transfer: a cache's regions, in model order. Mirrors the `regions` list a handshake carries
 * (nixl_connector.py:360) and the local self.regions (:235). */
typedef struct kvx_cache {
    const kvx_region *regions; /* host array of n_regions */
    int32_t n_regions;
    int32_t num_blocks;        /* blocks per region; every block id must be below it (nixl_connector.py:398) */
} kvx_cache;

/* One READ: one request's blocks for one head share. Mirrors the arguments of the two block_descs calls and the
 * READ posted in NixlConnectorWorker._start (nixl_connector.py:403-420). */
typedef struct kvx_job {
    int32_t src_cache;              /* index into the caches array */
    int32_t dst_cache;
    const int32_t *src_block_ids;   /* host array of n_blocks (remote_block_ids) */
    const int32_t *dst_block_ids;   /* host array of n_blocks (local_block_ids) */
    int32_t n_blocks;
    int32_t src_first_head;         /* Share.remote_head */
    int32_t dst_first_head;         /* Share.local_head */
    int32_t num_heads;              /* Share.num_heads */
    int32_t latents;                /* nonzero: whole latent blocks too (the first share, nixl_connector.py:403) */
} kvx_job;

/* CUDA IPC export of a device allocation, carried in the handshake reply in place of NIXL agent metadata. */
typedef struct kvx_ipc_handle {
    unsigned char handle[64]; /* cudaIpcMemHandle_t of the allocation holding the pointer */
    uint64_t offset;          /* of the pointer within that allocation */
    uint64_t alloc_bytes;     /* size of that allocation */
    int32_t device;           /* exporting device ordinal, in the exporter's numbering */
    int32_t pid;              /* exporting process ... */
    uint64_t ptr;             /* the exported pointer, valid in the exporting process only */
    unsigned char nonce[16];  /* ... and 16 random bytes drawn once per process: an importer whose pid AND nonce
                                 match uses `ptr` directly (a pid alone repeats across PID namespaces) */
} kvx_ipc_handle;

/* Opaque in-flight transfer: a launch plus the event recorded after it (a NIXL xfer handle, :411-418). */
typedef struct kvx_xfer *kvx_xfer_t;

/* ---- library ---- */
int kvx_abi_version(void);
/* The last failure's description on the calling thread (empty if none). */
const char *kvx_last_error(void);

/* ---- memory registration and the handshake ---- */

/* Exports the allocation holding `ptr` for another process on this node.
 * Replaces agent.get_reg_descs/register_memory/get_agent_metadata (nixl_connector.py:240-244). */
int kvx_ipc_export(const void *ptr, kvx_ipc_handle *out);

/* Maps a peer's exported allocation into this process on the current device and returns the exported pointer's
 * address here. Reference-counted per allocation: a second open of the same allocation returns the same mapping.
 * An allocation of this process is returned as is, with peer access from the current device enabled when it
 * lives on another device (refused if the two cannot reach each other directly).
 * Replaces agent.add_remote_agent (nixl_connector.py:510). */
int kvx_ipc_open(const kvx_ipc_handle *handle, void **out_ptr);

/* Drops one reference taken by kvx_ipc_open; unmaps at zero. Replaces agent.remove_remote_agent (:337, :486). */
int kvx_ipc_close(const kvx_ipc_handle *handle);

/* Whether `device` can load and store `peer`'s memory directly (NVLink/NVSwitch); enables it if so. */
int kvx_enable_peer_access(int device, int peer, int *out_can_access);

/* ---- the three kernels ---- */

/* Paged-block copy, one launch for all jobs, stream-ordered: gather from src blocks, head resharding, scatter into
 * dst blocks. Either side may be another GPU's memory (a kvx_ipc_open mapping): a consumer-side launch pulls over
 * NVLink, a producer-side launch pushes. This is the data movement of one or more NIXL READs (:411-420). */
int kvx_copy(const kvx_cache *caches, int n_caches, const kvx_job *jobs, int n_jobs, int flags, void *stream);

/* Gathers one job's chunks (region-major, then block) into the contiguous buffer `staging`, which must hold
 * n_chunks*chunk_bytes bytes; `staging` may be a peer's mapping (pack-and-push in one pass).
 * Chunk (region r, block i) lands at staging + (r*n_blocks + i)*chunk_bytes, the row order of block_descs. */
int kvx_pack(const kvx_cache *src, const int32_t *src_block_ids, int n_blocks, int first_head, int num_heads,
             int latents, void *staging, uint64_t staging_bytes, int flags, void *stream);

/* Moves `bytes` contiguous bytes from `src` to `dst`, either of which may be a peer mapping (the push of a packed
 * staging buffer over NVLink). */
int kvx_push(void *dst, const void *src, uint64_t bytes, int flags, void *stream);

/* The inverse of kvx_pack: scatters a staging buffer in kvx_pack's order into dst blocks. */
int kvx_scatter(const void *staging, uint64_t staging_bytes, const kvx_cache *dst, const int32_t *dst_block_ids,
                int n_blocks, int first_head, int num_heads, int latents, int flags, void *stream);

/* ---- the per-token cache store, alone or fused with the push ---- */

/* One cache a store writes: the local paged cache, or a peer's (a decode rank's blocks, mapped with kvx_ipc_open).
 * Strides are in bytes and address the cache as (block, token, head, dim), so NHD and HND caches both work, as the
 * reference's store kernel reads them (attention/triton_cache.py:32-36, 66). */
typedef struct kvx_store_dest {
    uint64_t k_cache;            /* device address of block 0's keys (or latents) */
    uint64_t v_cache;            /* device address of block 0's values; 0 for latents */
    int64_t block_stride;        /* bytes between blocks */
    int64_t token_stride;        /* bytes between a block's tokens */
    int64_t head_stride;         /* bytes between heads (unused for latents) */
    int32_t block_size;          /* tokens per block */
    int32_t num_blocks;          /* slots at or past num_blocks*block_size are skipped and flagged (device error 2) */
    const void *slot_mapping;    /* device array of num_tokens slots (block*block_size + offset); -1 skips */
    int32_t slot_bytes;          /* 4 (int32) or 8 (int64) */
    int32_t src_first_head;      /* this destination takes source heads [src_first_head, +num_heads) ... */
    int32_t num_heads;
    int32_t dst_first_head;      /* ... and stores them from its head dst_first_head */
    const int32_t *block_map;    /* destinations after the first: if set, a device array mapping destination 0's
                                    block ids to this cache's (-1 skips), used instead of slot_mapping: the row of
                                    destination-0 slot s lands at block_map[s / block_size] * block_size +
                                    s % block_size (both caches then share block_size) */
    int32_t block_map_len;       /* entries of block_map; a block id past it is skipped and flagged (error 2) */
    int32_t pad_;
} kvx_store_dest;

/* kvx_store flags: bits 16-23 CTAs per SM (0: as many as fit), bits 24-31 SM budget, as for copies; and */
#define KVX_STORE_SERIAL 1     /* a plain launch: no overlap with the kernel before it on the stream */
#define KVX_STORE_PEERS_ONLY 4 /* destination 0 is not written (its slots still place the peers' rows): the push
                                  half of a store whose local half ran on another stream */

/* Scatters num_tokens rows of keys and values [token][head][head_bytes] (or latents, with value = NULL and
 * num_heads = 1) into each destination's slots, one pass over the rows: destination 0 is the local cache
 * (store_kvcache / store_latents, attention/triton_cache.py:9-91); destinations 1..8 may be peers' caches, which
 * makes this the fused store-and-push of a layer-by-layer transfer. Strides of the rows are in bytes. `status` (may be
 * NULL) is a status word (kvx_status_open) that gets bit 2 when a row was skipped because its slot, or its block
 * map entry, lies past a destination's cache -- what a fused push checks before it reports the peer's blocks full. */
int kvx_store(const void *key, const void *value, int64_t key_stride, int64_t value_stride, int num_tokens,
              int num_heads, int head_bytes, const kvx_store_dest *dests, int n_dests, int32_t *status, int flags,
              void *stream);

/* ---- transfers with completion (post, poll, release) ---- */

/* kvx_copy after `wait_event` (a cudaEvent_t as void*, may be 0) has passed on `stream`, then records a completion
 * event. Replaces initialize_xfer("READ") + transfer (nixl_connector.py:411-420); the wait replaces the host
 * synchronisation on the ready event (:394-395) with a stream wait. */
int kvx_transfer(const kvx_cache *caches, int n_caches, const kvx_job *jobs, int n_jobs, int flags,
                 void *wait_event, void *stream, kvx_xfer_t *out);

/* kvx_transfer ordered after everything queued so far on `after_stream` (a cudaStream_t as void*; 0 is the legacy
 * default stream): an event this library keeps per device is recorded there and waited for on `stream`, so the
 * caller needs no event of its own. The reference's ready event (nixl_connector.py:266), for a caller that posts
 * the transfer on the thread that runs the engine's stream. */
int kvx_transfer_after(const kvx_cache *caches, int n_caches, const kvx_job *jobs, int n_jobs, int flags,
                       void *after_stream, void *stream, kvx_xfer_t *out);

/* KVX_OK once the transfer's copies have landed, KVX_PENDING while in flight, <0 on failure: KVX_ERR_CUDA if the
 * launch failed, KVX_ERR_DEVICE if one of ITS copies gave up a bounded wait (bit 1 of its own status word, read from
 * host memory once the transfer's event has completed: no copy, no stream). A failure elsewhere on the device fails
 * no other transfer. Replaces check_xfer_state (nixl_connector.py:431). */
int kvx_check_xfer(kvx_xfer_t xfer);

/* Frees the handle and its status word (waits for nothing: release a transfer once it completed, or once the device
 * has finished everything queued before it). Replaces release_xfer_handle (nixl_connector.py:437). */
int kvx_release_xfer(kvx_xfer_t xfer);

/* The transfer's status word (see kvx_status_open), for a test that stands in a failure of this transfer alone
 * (kvx_wait_selftest). Valid until kvx_release_xfer. No reference counterpart: NIXL keeps per-xfer state inside the
 * agent. */
int kvx_xfer_status(kvx_xfer_t xfer, int32_t **out_word);

/* ---- status words ---- */

/* A status word: 4 bytes of pinned host memory mapped into every device at the same address. A kernel given one
 * writes an error bit there only when it fails without faulting (1: a copy's bounded wait ran out; 2: a store row
 * whose slot or block lies past its cache was skipped), and the host reads it once the launch's completion event has
 * completed. Opened zeroed; close it only after every launch given it has completed. kvx_transfer holds one per
 * transfer; kvx_store takes one from its caller. Up to 65,536 are open at once. No reference counterpart (NIXL
 * reports per-xfer state through check_xfer_state, nixl_connector.py:431). */
int kvx_status_open(int32_t **out_word);
int kvx_status_close(int32_t *word);
int kvx_status_read(const int32_t *word, int32_t *out_bits);

/* ---- completion doorbells ---- */

/* A doorbell: a non-blocking eventfd (`out_fd`, readable while rung) and a native watcher thread that rings it when
 * the stream work before a kvx_doorbell_ring_after has ended. A transfer thread sleeps in poll() on it, on its
 * sockets and on its work queue together, and wakes within microseconds of a copy landing, instead of querying
 * every transfer on a timer (the reference polls check_xfer_state every 1 ms, nixl_connector.py:43, :431). */
int kvx_doorbell_open(int *out_id, int *out_fd);

/* Rings doorbell `id` (adds 1 to its eventfd) once the work queued on `stream` so far has ended: records an event
 * there, which the watcher queries every few microseconds. `stream` never waits for anything. */
int kvx_doorbell_ring_after(int id, void *stream);

/* Stops the watcher (rings not yet due are dropped) and closes the eventfd. */
int kvx_doorbell_close(int id);

/* ---- the per-step exchange of connector outputs between one instance's ranks ---- */

/* A step mailbox: host shared memory (a file every rank of one engine instance maps) through which each rank hands
 * rank 0 its KVConnectorOutput every step, replacing the gloo gather_object of ModelRunner.kv_connector_step
 * (engine/model_runner.py:637-649). Layout, all little-endian uint64 words: at 0 `consumed` (the last step rank 0
 * has read); rank r's slot at 64 + r * kvx_mailbox_stride(slot_bytes): `seq` (the last step it posted), `len`, then
 * `len` payload bytes (at most slot_bytes). A rank with nothing to report posts len 0. Waits spin, then sleep, and
 * give up with KVX_ERR_TIMEOUT after timeout_s seconds. */
uint64_t kvx_mailbox_stride(uint64_t slot_bytes);
uint64_t kvx_mailbox_bytes(int world, uint64_t slot_bytes);

/* Rank `rank` (1 <= rank < world) posts step `seq` (1, 2, ...): waits until rank 0 has read step seq - 1, copies
 * `len` bytes of `data` into its slot, then publishes seq (release). */
int kvx_mailbox_post(void *box, int world, int rank, uint64_t slot_bytes, uint64_t seq, const void *data,
                     uint64_t len, double timeout_s);

/* Rank 0 waits until every other rank has posted step `seq` (acquire) and writes each slot's length to lens[rank]
 * (lens[0] = 0); the payloads are then readable in place until kvx_mailbox_release. */
int kvx_mailbox_collect(void *box, int world, uint64_t slot_bytes, uint64_t seq, uint64_t *lens, double timeout_s);

/* Rank 0 is done reading step `seq`: the other ranks may post seq + 1. */
int kvx_mailbox_release(void *box, uint64_t seq);

/* ---- diagnostics ---- */

/* Bytes kvx_copy would move for these jobs: the sum of descriptor lengths the reference counts
 * (nixl_connector.py:421). Validates like kvx_copy; launches nothing. */
int kvx_job_bytes(const kvx_cache *caches, int n_caches, const kvx_job *jobs, int n_jobs, uint64_t *out_bytes);

/* Reads and clears, in one atomic step on the device, the diagnostic error word of the current device: 0, or the OR
 * of the errors kernels recorded since the last read -- 1 a copy's bounded TMA wait ran out (its bytes did not all
 * land), 2 a store slot or block id past its cache (skipped), 4 kvx_wait_selftest gave up as designed. Runs on a
 * stream of the library's own and waits on no other. Transfers are judged by their own status words, not by this
 * word: reading it (or not) changes no transfer's result. */
int kvx_device_error(int *out_code);

/* Runs, on `stream`, the bounded wait that guards every TMA copy against a transfer that never arrives: one
 * thread waits on an mbarrier armed for bytes no copy will bring, gives up after limit_us (1 us .. 10 s) and
 * records `code` in the device word and in `status` when given (kvx_xfer_status): 4 (the self-test's own bit), or 1
 * to stand in for a stuck copy of that transfer. Nothing is copied, nothing faults or hangs; for tests of the
 * failure path. */
int kvx_wait_selftest(int limit_us, int code, int32_t *status, void *stream);

/* Kernel launches issued by this process so far (all entry points), for launch accounting. */
uint64_t kvx_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* KVX_H */
