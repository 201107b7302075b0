// kvx: B200-native paged KV-cache transfer (the C ABI of include/kvx.h).
//
// One kernel family moves paged KV blocks: gather by source block table, head resharding, scatter by destination
// block table, in a single pass over HBM or NVLink. A launch's whole description -- region tables of both caches,
// block ids, head shares -- travels in the kernel's parameter space (up to 32 KB, CUDA >= 12.1), so a transfer needs
// no device scratch memory and no host-to-device copy besides the launch itself.
//
// Work decomposition. Job j (one READ: one request x one head share) covers n_regions x n_blocks contiguous chunks
// of chunk_bytes (HND caches keep a share's heads of one block contiguous). Chunks are cut into tiles of
// tile_bytes; a launch numbers all tiles of all its jobs consecutively and a persistent grid of
// (SM count x CTAs per SM) walks them with a grid stride. Two engines copy a tile:
//   LSU -- every thread moves VEC-byte vectors (16 when all addresses and lengths allow) with streaming loads,
//          UNROLL vectors in flight per thread;
//   TMA -- one thread per CTA runs a STAGES-deep ring of cp.async.bulk global->shared loads (mbarrier completion)
//          and cp.async.bulk shared->global stores (bulk-group completion); data never enters registers.
// Either side may be another GPU's memory mapped with cudaIpcOpenMemHandle: a launch on the consumer pulls over
// NVLink, a launch on the producer pushes. Every bulk load lands in the issuing CTA's own shared memory.
//
// Status. A launch that can fail on the device without faulting -- a copy whose bounded wait ran out, a store row
// whose slot lies past its cache -- reports it in a status word of its own: 4 bytes of pinned host memory mapped into
// every device (kvx_status_open), written by the kernel only on failure and read by the host once the launch's event
// has completed, with no copy and no stream of its own. Each transfer holds one, so a failure fails that transfer
// alone. The same bits are also OR-ed into a per-device word, a diagnostic read and cleared by kvx_device_error.

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <condition_variable>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <type_traits>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <sched.h>
#include <sys/eventfd.h>
#include <sys/prctl.h>
#include <time.h>
#include <unistd.h>

#include <nvtx3/nvToolsExt.h>

#include "kvx.h"

namespace {

// ------------------------------------------------------------------------------------------------ errors

thread_local std::string t_error;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_error = buf;
    return code;
}

#define KVX_CUDA(call)                                                                                  \
    do {                                                                                                \
        cudaError_t e_ = (call);                                                                        \
        if (e_ != cudaSuccess) return fail(KVX_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

std::atomic<uint64_t> g_launches{0};

// An NVTX range around each entry point that launches work, so a timeline (nsys, ncu's range view) shows which call
// queued which kernels. Without a tool attached, NVTX calls are no-ops.
struct Range {
    explicit Range(const char *name) { nvtxRangePushA(name); }
    ~Range() { nvtxRangePop(); }
};

// ------------------------------------------------------------------------------------------------ launch params

constexpr int kMaxRegions = 512;  // region slots per launch, over all caches it touches
constexpr int kMaxCacheRegions = 256;
constexpr int kMaxJobs = 96;      // job pieces per launch
constexpr int kMaxIds = 3072;     // block ids per launch (source and destination)

struct DevJob {
    uint64_t tile_start;    // first tile of this job in the launch's numbering
    uint64_t chunk_bytes;   // bytes per (region, block)
    uint64_t src_head_off;  // src_first_head * head_bytes
    uint64_t dst_head_off;
    uint32_t src_region0;   // slot of this job's first source region
    uint32_t dst_region0;
    uint32_t n_regions;
    uint32_t n_blocks;
    uint32_t ids_off;       // source ids at ids[ids_off], destination ids at ids[ids_off + n_blocks]
    uint32_t tiles_per_chunk;
};

template <int J, int R, int I>
struct ParamsOf {
    static constexpr int kJobs = J, kRegions = R, kIds = I;
    uint64_t total_tiles;
    uint32_t n_jobs;
    uint32_t tile_bytes;
    int32_t error_code;  // written to the status words when a bounded wait runs out
    uint32_t pad;
    int32_t *status;     // this launch's status word (mapped host memory), or null
    DevJob jobs[J];
    uint64_t addr[R];         // region base (block 0)
    uint64_t block_bytes[R];  // region block stride
    int32_t ids[I];
};
// Every launch is packed into the full block; one that fits the compact block is launched with that instead. Measured
// on B200 (driver 580): on a stream's first ~200 launches, and after the host idled, a launch's host cost grows with
// its parameter block (~18 us for 26 KB, ~6 us up to 4 KB); a connector's single-request loads fit 4 KB.
using Params = ParamsOf<kMaxJobs, kMaxRegions, kMaxIds>;
using SmallParams = ParamsOf<8, 160, 256>;
static_assert(sizeof(Params) <= 32764, "kernel parameter space is 32764 bytes");
static_assert(sizeof(SmallParams) <= 4096, "the compact parameter block stays within 4 KB");

// Errors kernels record, as bits: a copy's bounded TMA wait ran out (its bytes did not all land), a store slot or
// block id past its cache (skipped), the wait self-test gave up. Each goes into the launch's status word, when it
// has one, and into the device's diagnostic word (read and cleared by kvx_device_error).
constexpr int kErrCopyWait = 1;
constexpr int kErrPastCache = 2;
constexpr int kErrSelftest = 4;
__device__ int g_device_error;

// Records `code` for a launch. A status word is only ever given one code per launch, so a plain store suffices (no
// atomic reaches host memory); the host reads it after the launch's completion event, which orders the store.
__device__ __forceinline__ void report(int32_t *status, int code) {
    atomicOr(&g_device_error, code);
    if (status) *reinterpret_cast<volatile int32_t *>(status) = code;
}

struct Tile {
    const char *src;
    char *dst;
    uint32_t len;
};

// Locates tile t of the launch. `j` is a cursor into the job list that only moves forward, since each CTA visits
// tiles in increasing order.
template <class P>
__device__ __forceinline__ Tile locate(const P &p, uint64_t t, uint32_t &j) {
    while (j + 1 < p.n_jobs && t >= p.jobs[j + 1].tile_start) ++j;
    const DevJob &job = p.jobs[j];
    const uint64_t lt = t - job.tile_start;
    const uint64_t chunk = lt / job.tiles_per_chunk;
    const uint64_t sub = lt - chunk * job.tiles_per_chunk;
    const uint32_t r = (uint32_t)(chunk / job.n_blocks);
    const uint32_t i = (uint32_t)(chunk - (uint64_t)r * job.n_blocks);
    const int64_t sid = p.ids[job.ids_off + i];
    const int64_t did = p.ids[job.ids_off + job.n_blocks + i];
    const uint32_t sr = job.src_region0 + r, dr = job.dst_region0 + r;
    const uint64_t off = sub * p.tile_bytes;
    Tile tile;
    tile.src = reinterpret_cast<const char *>(p.addr[sr] + (uint64_t)sid * p.block_bytes[sr] + job.src_head_off + off);
    tile.dst = reinterpret_cast<char *>(p.addr[dr] + (uint64_t)did * p.block_bytes[dr] + job.dst_head_off + off);
    const uint64_t rest = job.chunk_bytes - off;
    tile.len = (uint32_t)(rest < p.tile_bytes ? rest : p.tile_bytes);
    return tile;
}

// ------------------------------------------------------------------------------------------------ LSU engine

template <int VEC>
struct Vec;
template <>
struct Vec<16> {
    using T = uint4;
    static __device__ __forceinline__ T load(const void *p) {
        T v;
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "l"(p));
        return v;
    }
    static __device__ __forceinline__ void store(void *p, T v) {
        asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
    }
};
template <>
struct Vec<8> {
    using T = uint2;
    static __device__ __forceinline__ T load(const void *p) { return __ldg(reinterpret_cast<const uint2 *>(p)); }
    static __device__ __forceinline__ void store(void *p, T v) { *reinterpret_cast<uint2 *>(p) = v; }
};
template <>
struct Vec<4> {
    using T = uint32_t;
    static __device__ __forceinline__ T load(const void *p) { return __ldg(reinterpret_cast<const uint32_t *>(p)); }
    static __device__ __forceinline__ void store(void *p, T v) { *reinterpret_cast<uint32_t *>(p) = v; }
};
template <>
struct Vec<2> {
    using T = unsigned short;
    static __device__ __forceinline__ T load(const void *p) {
        return __ldg(reinterpret_cast<const unsigned short *>(p));
    }
    static __device__ __forceinline__ void store(void *p, T v) { *reinterpret_cast<unsigned short *>(p) = v; }
};
template <>
struct Vec<1> {
    using T = unsigned char;
    static __device__ __forceinline__ T load(const void *p) { return __ldg(reinterpret_cast<const unsigned char *>(p)); }
    static __device__ __forceinline__ void store(void *p, T v) { *reinterpret_cast<unsigned char *>(p) = v; }
};

constexpr int kLsuThreads = 512;
constexpr int kLsuUnroll = 4;

template <int VEC, class P>
__global__ void __launch_bounds__(kLsuThreads) kvx_copy_lsu(const __grid_constant__ P p) {
    using V = Vec<VEC>;
    uint32_t j = 0;
    for (uint64_t t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
        const Tile tile = locate(p, t, j);
        const uint32_t n = tile.len / VEC;
        for (uint32_t base = threadIdx.x; base < n; base += kLsuThreads * kLsuUnroll) {
            typename V::T r[kLsuUnroll];
#pragma unroll
            for (int u = 0; u < kLsuUnroll; ++u) {
                const uint32_t k = base + u * kLsuThreads;
                if (k < n) r[u] = V::load(tile.src + (uint64_t)k * VEC);
            }
#pragma unroll
            for (int u = 0; u < kLsuUnroll; ++u) {
                const uint32_t k = base + u * kLsuThreads;
                if (k < n) V::store(tile.dst + (uint64_t)k * VEC, r[u]);
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------ TMA engine

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // a bulk load that has not landed after 2 s is an error

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait on an mbarrier phase: false if it did not complete by `deadline` (globaltimer ns).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t deadline) {
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() > deadline) return false;
    }
    return true;
}

__device__ __forceinline__ void bulk_load(uint32_t smem, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void bulk_store(void *dst, uint32_t smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

constexpr int kTmaStages = 4;

// The failure path of every TMA wait, on demand: an mbarrier armed for 16 bytes that no copy will bring, waited on
// with the same bounded wait the copy kernels use. It gives up after `limit_ns`, records `code` in the device word
// (and in `status`, when given) and returns -- the status a stuck copy would leave -- without copying, faulting or
// hanging anything.
__global__ void __launch_bounds__(32) kvx_wait_selftest_kernel(uint64_t limit_ns, int code, int32_t *status) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    const uint32_t b = smem_u32(&bar);
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(b) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(16u) : "memory");
    if (!mbar_wait(b, 0, globaltimer() + limit_ns)) report(status, code);
}

// Reads and clears the device's diagnostic word in one atomic step, into mapped host memory: a bit a kernel sets
// meanwhile is either taken here or left for the next read, never lost.
__global__ void __launch_bounds__(32) kvx_take_device_error_kernel(int32_t *out) {
    if (threadIdx.x == 0) *reinterpret_cast<volatile int32_t *>(out) = atomicExch(&g_device_error, 0);
}

template <class P>
__global__ void __launch_bounds__(32) kvx_copy_tma(const __grid_constant__ P p) {
    extern __shared__ __align__(128) unsigned char ring[];
    __shared__ __align__(8) uint64_t full[kTmaStages];
    if (threadIdx.x != 0) return;  // one issuing thread; the rest of the warp has nothing to do

    const uint64_t mine =
        p.total_tiles > blockIdx.x ? (p.total_tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    if (mine == 0) return;
    for (int s = 0; s < kTmaStages; ++s)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[s])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");

    char *dst_of[kTmaStages];
    uint32_t len_of[kTmaStages];
    uint32_t load_cursor = 0;
    const uint32_t stage_bytes = p.tile_bytes;

    auto issue = [&](uint64_t k) {
        const int s = (int)(k % kTmaStages);
        const Tile tile = locate(p, blockIdx.x + k * gridDim.x, load_cursor);
        dst_of[s] = tile.dst;
        len_of[s] = tile.len;
        bulk_load(smem_u32(ring + (size_t)s * stage_bytes), tile.src, tile.len, smem_u32(&full[s]));
    };

    const uint64_t prologue = mine < kTmaStages ? mine : kTmaStages;
    for (uint64_t k = 0; k < prologue; ++k) issue(k);

    uint64_t landed = 0;  // loads waited for
    bool ok = true;
    for (uint64_t k = 0; k < mine; ++k) {
        const int s = (int)(k % kTmaStages);
        if (!mbar_wait(smem_u32(&full[s]), (uint32_t)((k / kTmaStages) & 1), globaltimer() + kWaitLimitNs)) {
            ok = false;
            break;
        }
        landed = k + 1;
        bulk_store(dst_of[s], smem_u32(ring + (size_t)s * stage_bytes), len_of[s]);
        // Refill the stage of tile k-1 once its store has read shared memory; tile k's store may still be reading.
        if (k >= 1 && k - 1 + kTmaStages < mine) {
            bulk_wait_read<1>();
            issue(k - 1 + kTmaStages);
        }
    }
    if (!ok) {
        report(p.status, p.error_code);
        // Loads issued but not waited for may still be writing shared memory: give each a bounded wait.
        const uint64_t issued = mine < landed + kTmaStages ? mine : landed + kTmaStages;
        const uint64_t drain = globaltimer() + kWaitLimitNs;
        for (uint64_t k = landed; k < issued; ++k)
            if (!mbar_wait(smem_u32(&full[k % kTmaStages]), (uint32_t)((k / kTmaStages) & 1), drain)) break;
    }
    bulk_wait_all();
}

// ------------------------------------------------------------------------------------------------ store kernel

// The per-token cache store (the reference's store_kvcache/store_latents), optionally fused with the push: each
// source row [token][head] is read once and written to every destination whose head range holds it. Thread t of
// the flattened space (token, K|V, head, vector) moves one VEC-byte vector, so reads of a token's rows are
// contiguous and each (token, head) row lands as one contiguous run of head_bytes in every cache.
constexpr int kMaxStoreDests = 9;  // the local cache and up to 8 decode ranks

struct StoreDest {
    uint64_t k, v;
    int64_t block_stride, token_stride, head_stride;
    const void *slots;
    const int32_t *block_map;
    int32_t block_size, num_blocks, slot_bytes, src_first_head, num_heads, dst_first_head, block_map_len;
    int32_t block_shift;  // log2(block_size) when it is a power of two (the usual 16, 64, 256), else -1
};

struct StoreParams {
    uint64_t key, value;
    int64_t key_stride, value_stride;
    int32_t num_tokens, num_heads, head_bytes, n_dests;
    int32_t peers_only, pad_;  // KVX_STORE_PEERS_ONLY: destination 0 places rows but is not written
    int32_t *status;           // this launch's status word (mapped host memory), or null
    StoreDest dests[kMaxStoreDests];
};

__device__ __forceinline__ int32_t load_slot(const StoreDest &dst, uint32_t token) {
    return dst.slot_bytes == 8 ? (int32_t) static_cast<const int64_t *>(dst.slots)[token]
                               : static_cast<const int32_t *>(dst.slots)[token];
}

// Destination d's slot for a row whose destination-0 slot is first_slot (-1: no slot, skip). Slots are below 2^31
// (the host checks num_blocks * block_size), so the arithmetic runs in 32 bits.
__device__ __forceinline__ int32_t resolve_slot(const StoreParams &p, int d, uint32_t token, int32_t first_slot) {
    const StoreDest &dst = p.dests[d];
    if (d == 0) return first_slot;
    if (!dst.block_map) return load_slot(dst, token);
    if (first_slot < 0) return -1;
    const uint32_t block_size0 = (uint32_t)p.dests[0].block_size;
    const int32_t shift0 = p.dests[0].block_shift;
    const uint32_t b = shift0 >= 0 ? (uint32_t)first_slot >> shift0 : (uint32_t)first_slot / block_size0;
    if (b >= (uint32_t)dst.block_map_len) {
        report(p.status, kErrPastCache);
        return -1;
    }
    const int32_t mapped = dst.block_map[b];  // a block no save covers maps to -1
    return mapped < 0 ? -1 : mapped * dst.block_size + (first_slot - (int32_t)(b * block_size0));
}

// One destination as one thread sees it from its fixed (K|V, head, vector) position, computed once per thread so
// that storing a vector costs a slot check, a shift and one address multiply-add: the kernels are bound by issue
// rate, not bytes, when every field is re-read per token.
struct StoreLane {
    uint64_t base;  // the position's address at block 0, token 0; 0 when the head is not this destination's
    int64_t block_stride, token_stride;
    int32_t limit;  // num_blocks * block_size
    int32_t shift;  // log2(block_size), or -1
    uint32_t block_size;
};

__device__ __forceinline__ StoreLane lane_of(const StoreDest &dst, uint32_t part, int32_t head, uint32_t byte_in_row) {
    StoreLane l;
    const bool mine = head >= dst.src_first_head && head < dst.src_first_head + dst.num_heads;
    l.base = mine ? (part ? dst.v : dst.k) + (int64_t)(head - dst.src_first_head + dst.dst_first_head) * dst.head_stride +
                        byte_in_row
                  : 0;
    l.block_stride = dst.block_stride;
    l.token_stride = dst.token_stride;
    l.limit = dst.num_blocks * dst.block_size;
    l.shift = dst.block_shift;
    l.block_size = (uint32_t)dst.block_size;
    return l;
}

// FAST: the destination's block size is a power of two and its block and token strides are below 2^32, so a slot
// becomes an address with a shift, a mask and two 32x32->64-bit multiply-adds (the usual paged cache).
template <int VEC, bool FAST>
__device__ __forceinline__ void put(const StoreLane &l, int32_t slot, typename Vec<VEC>::T data, int32_t *status) {
    if (slot < 0) return;  // padding: no cache slot
    if (slot >= l.limit) {
        report(status, kErrPastCache);  // a slot past the cache: skipped, never written
        return;
    }
    uint64_t at;
    if (FAST) {
        const uint32_t block = (uint32_t)slot >> l.shift;
        const uint32_t offset = (uint32_t)slot & (l.block_size - 1);
        at = l.base + (uint64_t)block * (uint32_t)l.block_stride + (uint64_t)offset * (uint32_t)l.token_stride;
    } else {
        const uint32_t block = l.shift >= 0 ? (uint32_t)slot >> l.shift : (uint32_t)slot / l.block_size;
        const uint32_t offset = (uint32_t)slot - block * l.block_size;
        at = l.base + (uint64_t)block * l.block_stride + (uint64_t)offset * l.token_stride;
    }
    Vec<VEC>::store(reinterpret_cast<char *>(at), data);
}

template <int VEC>
__device__ __forceinline__ void store_row(const StoreParams &p, const StoreDest &dst, int32_t slot, uint32_t part,
                                          int32_t head, uint32_t byte_in_row, typename Vec<VEC>::T data) {
    if (slot < 0) return;  // padding: no cache slot
    if (slot >= dst.num_blocks * dst.block_size) {
        report(p.status, kErrPastCache);  // a slot past the cache: skipped, never written
        return;
    }
    const uint32_t block = dst.block_shift >= 0 ? (uint32_t)slot >> dst.block_shift
                                                : (uint32_t)slot / (uint32_t)dst.block_size;
    const uint32_t offset = (uint32_t)slot - block * (uint32_t)dst.block_size;
    const uint64_t base = part ? dst.v : dst.k;
    char *out = reinterpret_cast<char *>(base + (uint64_t)block * dst.block_stride +
                                         (uint64_t)offset * dst.token_stride +
                                         (int64_t)(head - dst.src_first_head + dst.dst_first_head) * dst.head_stride) +
                byte_in_row;
    Vec<VEC>::store(out, data);
}

constexpr int kStoreThreads = 256;
constexpr int kStoreUnroll = 4;  // tokens each thread loads before it stores any: bytes in flight per SM

// Each thread owns fixed positions within a token's rows -- (K|V, head, vector), decoded once -- and sweeps tokens:
// a CTA covers `tpp` tokens per pass (one when a token's rows exceed the CTA), kStoreUnroll passes in flight. The
// rows and their destination-0 slots load together; each further destination resolves the slots of all tokens in
// flight before it stores any, so every dependent load is one round trip per batch, not per token.
//
// Launched with programmatic stream serialization (unless flags ask for a plain launch): the grid may be scheduled
// while the kernel before it on the stream drains; it lets the next such launch start at once (launch_dependents),
// decodes its positions from the parameters, and waits for the previous kernel's completion and memory
// (griddepcontrol.wait) before it reads any row, slot or block map. Per-layer stores thus overlap each other's
// launch, ramp and set-up; with an ordinary kernel before or after, ordering is the plain stream's.
template <int VEC, bool FAST>
__global__ void __launch_bounds__(kStoreThreads, 5) kvx_store_kernel(const __grid_constant__ StoreParams p) {
    using V = Vec<VEC>;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint32_t vecs = (uint32_t)p.head_bytes / VEC;  // per (token, head) row
    const uint32_t parts = p.value ? 2u : 1u;
    const uint32_t per_token = parts * (uint32_t)p.num_heads * vecs;
    const bool packed = per_token <= blockDim.x;
    const uint32_t tpp = packed ? blockDim.x / per_token : 1;  // tokens per CTA pass
    const uint32_t lane_token = packed ? threadIdx.x / per_token : 0;
    if (lane_token >= tpp) return;  // threads past the last whole token of the pass
    const uint32_t token_step = gridDim.x * tpp;
    const uint32_t n = (uint32_t)p.num_tokens;
    for (uint32_t w = packed ? threadIdx.x % per_token : threadIdx.x; w < per_token;
         w += packed ? per_token : blockDim.x) {
        const uint32_t vec = w % vecs;
        const int32_t head = (int32_t)((w / vecs) % (uint32_t)p.num_heads);
        const uint32_t part = w / (vecs * (uint32_t)p.num_heads);
        const uint64_t row0 = part ? p.value : p.key;
        const int64_t row_stride = part ? p.value_stride : p.key_stride;
        const uint32_t byte_in_row = vec * VEC;
        const char *in_row = reinterpret_cast<const char *>(row0 + (uint64_t)head * p.head_bytes + byte_in_row);
        const StoreLane lane0 = lane_of(p.dests[0], part, head, byte_in_row);
        const bool peers_only = p.peers_only != 0;
        const void *slots0 = p.dests[0].slots;
        const bool wide0 = p.dests[0].slot_bytes == 8;
        // Everything above reads only this launch's parameters, so it runs while the kernel before it drains; rows,
        // slots and block maps are read only once that kernel has completed and its memory is visible.
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (uint32_t t0 = blockIdx.x * tpp + lane_token; t0 < n; t0 += token_step * kStoreUnroll) {
            typename V::T data[kStoreUnroll];
            int32_t first[kStoreUnroll];
#pragma unroll
            for (int u = 0; u < kStoreUnroll; ++u) {
                const uint32_t t = t0 + u * token_step;
                first[u] = -1;
                if (t < n) {
                    data[u] = V::load(FAST ? in_row + (uint64_t)t * (uint32_t)row_stride : in_row + (int64_t)t * row_stride);
                    first[u] = wide0 ? (int32_t) static_cast<const int64_t *>(slots0)[t]
                                     : static_cast<const int32_t *>(slots0)[t];
                }
            }
            if (lane0.base && !peers_only) {
#pragma unroll
                for (int u = 0; u < kStoreUnroll; ++u) put<VEC, FAST>(lane0, first[u], data[u], p.status);
            }
            for (int d = 1; d < p.n_dests; ++d) {
                const StoreDest &dst = p.dests[d];
                if (head < dst.src_first_head || head >= dst.src_first_head + dst.num_heads) continue;
                int32_t slot[kStoreUnroll];
#pragma unroll
                for (int u = 0; u < kStoreUnroll; ++u) {
                    const uint32_t t = t0 + u * token_step;
                    slot[u] = t < n ? resolve_slot(p, d, t, first[u]) : -1;
                }
#pragma unroll
                for (int u = 0; u < kStoreUnroll; ++u) store_row<VEC>(p, dst, slot[u], part, head, byte_in_row, data[u]);
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------ host side

struct DeviceInfo {
    int sms = 0;
    size_t tma_smem_set[2] = {};  // dynamic shared memory allowed for kvx_copy_tma<Params, SmallParams>
    int store_ctas_per_sm[5][2] = {};  // resident kvx_store_kernel<16, 8, 4, 2, 1; FAST> CTAs per SM
};

std::mutex g_mutex;
std::map<int, DeviceInfo> g_devices;

int device_info(DeviceInfo **out) {
    int dev;
    KVX_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceInfo &info = g_devices[dev];
    if (info.sms == 0) KVX_CUDA(cudaDeviceGetAttribute(&info.sms, cudaDevAttrMultiProcessorCount, dev));
    *out = &info;
    return KVX_OK;
}

// One contiguous run of a job's regions with a single chunk size, cut to the launch capacity.
struct Piece {
    int src_cache, dst_cache;
    int r0, nr;
    uint64_t chunk, src_head_off, dst_head_off;
    const int32_t *src_ids, *dst_ids;
    int nb;
};

uint64_t low_bit(uint64_t x) { return x & (~x + 1); }

int plan(const kvx_cache *caches, int n_caches, const kvx_job *jobs, int n_jobs, std::vector<Piece> &pieces,
         uint64_t &bytes, uint64_t &align_bits) {
    if (n_jobs < 0 || n_caches < 0) return fail(KVX_ERR_INVALID, "negative job or cache count");
    if (n_jobs > 0 && (!jobs || !caches)) return fail(KVX_ERR_INVALID, "null jobs or caches");
    for (int c = 0; c < n_caches; ++c) {
        const kvx_cache &cache = caches[c];
        if (cache.n_regions < 0 || cache.n_regions > kMaxCacheRegions)
            return fail(KVX_ERR_INVALID, "cache %d has %d regions; at most %d", c, cache.n_regions, kMaxCacheRegions);
        if (cache.n_regions > 0 && !cache.regions) return fail(KVX_ERR_INVALID, "cache %d has no region table", c);
        if (cache.num_blocks < 0) return fail(KVX_ERR_INVALID, "cache %d has a negative block count", c);
    }
    bytes = 0;
    align_bits = 0;
    for (int j = 0; j < n_jobs; ++j) {
        const kvx_job &job = jobs[j];
        if (job.src_cache < 0 || job.src_cache >= n_caches || job.dst_cache < 0 || job.dst_cache >= n_caches)
            return fail(KVX_ERR_INVALID, "job %d names a cache outside the %d given", j, n_caches);
        if (job.n_blocks < 0) return fail(KVX_ERR_INVALID, "job %d has a negative block count", j);
        if (job.n_blocks == 0) continue;
        if (!job.src_block_ids || !job.dst_block_ids) return fail(KVX_ERR_INVALID, "job %d has null block ids", j);
        const kvx_cache &src = caches[job.src_cache], &dst = caches[job.dst_cache];
        if (src.n_regions != dst.n_regions)
            return fail(KVX_ERR_INVALID, "job %d pairs caches of %d and %d regions", j, src.n_regions, dst.n_regions);
        for (int i = 0; i < job.n_blocks; ++i) {
            if (job.src_block_ids[i] < 0 || job.src_block_ids[i] >= src.num_blocks)
                return fail(KVX_ERR_RANGE, "job %d: source block id %d outside the cache's %d blocks", j,
                            job.src_block_ids[i], src.num_blocks);
            if (job.dst_block_ids[i] < 0 || job.dst_block_ids[i] >= dst.num_blocks)
                return fail(KVX_ERR_RANGE, "job %d: destination block id %d outside the cache's %d blocks", j,
                            job.dst_block_ids[i], dst.num_blocks);
        }
        int run_start = -1;
        uint64_t run_chunk = 0, run_soff = 0, run_doff = 0;
        auto close_run = [&](int end) {
            if (run_start >= 0 && run_chunk > 0)
                pieces.push_back(Piece{job.src_cache, job.dst_cache, run_start, end - run_start, run_chunk, run_soff,
                                       run_doff, job.src_block_ids, job.dst_block_ids, job.n_blocks});
            run_start = -1;
        };
        for (int r = 0; r < src.n_regions; ++r) {
            const kvx_region &a = src.regions[r], &b = dst.regions[r];
            if (!a.addr || !b.addr) return fail(KVX_ERR_INVALID, "job %d: region %d has a null address", j, r);
            if ((a.head_bytes == 0) != (b.head_bytes == 0))
                return fail(KVX_ERR_INVALID, "job %d: region %d is latent on one side only", j, r);
            uint64_t chunk, soff = 0, doff = 0;
            if (a.head_bytes) {
                if (a.head_bytes != b.head_bytes)
                    return fail(KVX_ERR_INVALID, "job %d: region %d heads are %llu and %llu bytes", j, r,
                                (unsigned long long)a.head_bytes, (unsigned long long)b.head_bytes);
                if (job.num_heads < 0 || job.src_first_head < 0 || job.dst_first_head < 0)
                    return fail(KVX_ERR_INVALID, "job %d: negative head range", j);
                if (((uint64_t)job.src_first_head + (uint64_t)job.num_heads) * a.head_bytes > a.block_bytes ||
                    ((uint64_t)job.dst_first_head + (uint64_t)job.num_heads) * b.head_bytes > b.block_bytes)
                    return fail(KVX_ERR_RANGE, "job %d: heads [%d, +%d) / [%d, +%d) pass the end of a block", j,
                                job.src_first_head, job.num_heads, job.dst_first_head, job.num_heads);
                chunk = (uint64_t)job.num_heads * a.head_bytes;
                soff = (uint64_t)job.src_first_head * a.head_bytes;
                doff = (uint64_t)job.dst_first_head * b.head_bytes;
            } else if (job.latents) {
                if (a.block_bytes != b.block_bytes)
                    return fail(KVX_ERR_INVALID, "job %d: latent region %d blocks are %llu and %llu bytes", j, r,
                                (unsigned long long)a.block_bytes, (unsigned long long)b.block_bytes);
                chunk = a.block_bytes;
            } else {
                chunk = 0;  // latents come from another share
            }
            if (chunk == 0) {
                close_run(r);
                continue;
            }
            align_bits |= a.addr | b.addr | a.block_bytes | b.block_bytes | soff | doff | chunk;
            bytes += chunk * (uint64_t)job.n_blocks;
            if (run_start >= 0 && (chunk != run_chunk || soff != run_soff || doff != run_doff)) close_run(r);
            if (run_start < 0) {
                run_start = r;
                run_chunk = chunk;
                run_soff = soff;
                run_doff = doff;
            }
        }
        close_run(src.n_regions);
    }
    return KVX_OK;
}

struct Config {
    int engine;       // KVX_ENGINE_LSU or KVX_ENGINE_TMA
    int vec;          // LSU vector bytes
    uint32_t tile_bytes;
    int ctas_per_sm;
    int sm_budget;    // SMs the grid may cover (0: all)
};

// flags: bits 0-7 engine, bits 8-15 log2(tile bytes) (0: default), bits 16-23 CTAs per SM (0: default),
// bits 24-31 SM budget (0: every SM) -- a copy that runs beside compute can be held to a few SMs.
int choose(int flags, uint64_t align_bits, Config &cfg) {
    const int engine = flags & 0xff;
    if (engine != KVX_ENGINE_AUTO && engine != KVX_ENGINE_LSU && engine != KVX_ENGINE_TMA)
        return fail(KVX_ERR_INVALID, "unknown engine %d", engine);
    const uint64_t lb = align_bits ? low_bit(align_bits) : 16;
    cfg.vec = (int)std::min<uint64_t>(lb, 16);
    const bool tma_ok = cfg.vec == 16;
    if (engine == KVX_ENGINE_TMA && !tma_ok)
        return fail(KVX_ERR_INVALID, "the TMA engine needs 16-byte aligned addresses and lengths");
    cfg.engine = (engine == KVX_ENGINE_LSU || !tma_ok) ? KVX_ENGINE_LSU : KVX_ENGINE_TMA;
    const int log_tile = (flags >> 8) & 0xff;
    if (log_tile > 24) return fail(KVX_ERR_INVALID, "tile of 2^%d bytes", log_tile);  // before any shift by it
    const int ctas = (flags >> 16) & 0xff;
    cfg.sm_budget = (flags >> 24) & 0xff;
    if (cfg.engine == KVX_ENGINE_TMA) {
        cfg.tile_bytes = log_tile ? (1u << log_tile) : (32u << 10);
        cfg.ctas_per_sm = ctas ? ctas : 1;
        if (cfg.tile_bytes < 16 || cfg.tile_bytes * kTmaStages > (200u << 10))
            return fail(KVX_ERR_INVALID, "TMA tile of %u bytes does not fit %d stages", cfg.tile_bytes, kTmaStages);
    } else {
        cfg.tile_bytes = log_tile ? (1u << log_tile) : (32u << 10);
        cfg.ctas_per_sm = ctas ? ctas : 2;
        if (cfg.tile_bytes < (uint32_t)cfg.vec) return fail(KVX_ERR_INVALID, "tile smaller than a vector");
    }
    return KVX_OK;
}

template <class P>
int launch_as(const P &p, const Config &cfg, DeviceInfo *info, unsigned grid, cudaStream_t stream) {
    if (cfg.engine == KVX_ENGINE_TMA) {
        const size_t smem = (size_t)cfg.tile_bytes * kTmaStages;
        size_t &allowed = info->tma_smem_set[std::is_same<P, SmallParams>::value ? 1 : 0];
        if (allowed < smem) {
            KVX_CUDA(cudaFuncSetAttribute(kvx_copy_tma<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
            allowed = smem;
        }
        kvx_copy_tma<P><<<grid, 32, smem, stream>>>(p);
    } else {
        switch (cfg.vec) {
            case 16: kvx_copy_lsu<16, P><<<grid, kLsuThreads, 0, stream>>>(p); break;
            case 8: kvx_copy_lsu<8, P><<<grid, kLsuThreads, 0, stream>>>(p); break;
            case 4: kvx_copy_lsu<4, P><<<grid, kLsuThreads, 0, stream>>>(p); break;
            case 2: kvx_copy_lsu<2, P><<<grid, kLsuThreads, 0, stream>>>(p); break;
            default: kvx_copy_lsu<1, P><<<grid, kLsuThreads, 0, stream>>>(p); break;
        }
    }
    return KVX_OK;
}

// Launches the packed block `p`, of which the first n_regions region slots and n_ids block ids are in use: as the
// compact block when everything fits it.
int launch(Params &p, int n_regions, int n_ids, const Config &cfg, cudaStream_t stream) {
    if (p.total_tiles == 0) return KVX_OK;
    DeviceInfo *info;
    if (int rc = device_info(&info)) return rc;
    const int sms = cfg.sm_budget > 0 && cfg.sm_budget < info->sms ? cfg.sm_budget : info->sms;
    const uint64_t cap = (uint64_t)sms * cfg.ctas_per_sm;
    const unsigned grid = (unsigned)std::min<uint64_t>(p.total_tiles, cap);
    p.error_code = kErrCopyWait;
    int rc;
    if (p.n_jobs <= (uint32_t)SmallParams::kJobs && n_regions <= SmallParams::kRegions &&
        n_ids <= SmallParams::kIds) {
        thread_local SmallParams small;
        small.total_tiles = p.total_tiles;
        small.n_jobs = p.n_jobs;
        small.tile_bytes = p.tile_bytes;
        small.error_code = p.error_code;
        small.pad = 0;
        small.status = p.status;
        std::memcpy(small.jobs, p.jobs, sizeof(DevJob) * p.n_jobs);
        std::memcpy(small.addr, p.addr, sizeof(uint64_t) * n_regions);
        std::memcpy(small.block_bytes, p.block_bytes, sizeof(uint64_t) * n_regions);
        std::memcpy(small.ids, p.ids, sizeof(int32_t) * n_ids);
        rc = launch_as(small, cfg, info, grid, stream);
    } else {
        rc = launch_as(p, cfg, info, grid, stream);
    }
    if (rc) return rc;
    KVX_CUDA(cudaGetLastError());
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return KVX_OK;
}

// Packs pieces into as few launches as the parameter space allows and launches them in order on `stream`.
int run(const kvx_cache *caches, int n_caches, const std::vector<Piece> &pieces, const Config &cfg,
        int32_t *status, cudaStream_t stream) {
    thread_local std::vector<Params> storage(1);
    Params &p = storage[0];
    std::vector<int> slot(n_caches, -1);
    int n_regions = 0, n_ids = 0;
    auto reset = [&] {
        p.total_tiles = 0;
        p.n_jobs = 0;
        p.tile_bytes = cfg.tile_bytes;
        p.status = status;  // every launch of one call reports into the call's word
        std::fill(slot.begin(), slot.end(), -1);
        n_regions = 0;
        n_ids = 0;
    };
    reset();
    auto region_slot = [&](int c) -> int {
        if (slot[c] >= 0) return slot[c];
        const kvx_cache &cache = caches[c];
        if (n_regions + cache.n_regions > Params::kRegions) return -1;
        for (int r = 0; r < cache.n_regions; ++r) {
            p.addr[n_regions + r] = cache.regions[r].addr;
            p.block_bytes[n_regions + r] = cache.regions[r].block_bytes;
        }
        slot[c] = n_regions;
        n_regions += cache.n_regions;
        return slot[c];
    };
    const int max_blocks = Params::kIds / 2;
    for (const Piece &piece : pieces) {
        for (int b0 = 0; b0 < piece.nb; b0 += max_blocks) {
            const int nb = std::min(max_blocks, piece.nb - b0);
            for (int attempt = 0; attempt < 2; ++attempt) {
                int s = -1, d = -1;
                const bool room = p.n_jobs < (uint32_t)Params::kJobs && n_ids + 2 * nb <= Params::kIds &&
                                  (s = region_slot(piece.src_cache)) >= 0 && (d = region_slot(piece.dst_cache)) >= 0;
                if (!room) {
                    if (attempt == 1) return fail(KVX_ERR_INVALID, "a job piece does not fit one launch");
                    if (int rc = launch(p, n_regions, n_ids, cfg, stream)) return rc;
                    reset();
                    continue;
                }
                DevJob &job = p.jobs[p.n_jobs++];
                job.tile_start = p.total_tiles;
                job.chunk_bytes = piece.chunk;
                job.src_head_off = piece.src_head_off;
                job.dst_head_off = piece.dst_head_off;
                job.src_region0 = (uint32_t)(s + piece.r0);
                job.dst_region0 = (uint32_t)(d + piece.r0);
                job.n_regions = (uint32_t)piece.nr;
                job.n_blocks = (uint32_t)nb;
                job.ids_off = (uint32_t)n_ids;
                job.tiles_per_chunk = (uint32_t)((piece.chunk + cfg.tile_bytes - 1) / cfg.tile_bytes);
                std::memcpy(&p.ids[n_ids], piece.src_ids + b0, sizeof(int32_t) * nb);
                std::memcpy(&p.ids[n_ids + nb], piece.dst_ids + b0, sizeof(int32_t) * nb);
                n_ids += 2 * nb;
                p.total_tiles += (uint64_t)piece.nr * nb * job.tiles_per_chunk;
                break;
            }
        }
    }
    return launch(p, n_regions, n_ids, cfg, stream);
}

int copy_impl(const kvx_cache *caches, int n_caches, const kvx_job *jobs, int n_jobs, int flags,
              cudaStream_t stream, int32_t *status = nullptr) {
    std::vector<Piece> pieces;
    uint64_t bytes, align_bits;
    if (int rc = plan(caches, n_caches, jobs, n_jobs, pieces, bytes, align_bits)) return rc;
    if (pieces.empty()) return KVX_OK;
    Config cfg;
    if (int rc = choose(flags, align_bits, cfg)) return rc;
    return run(caches, n_caches, pieces, cfg, status, stream);
}

// A staging buffer in kvx_pack's order, as a cache of the same region count: region r starts where the rows of
// regions before it end, and block i of it sits at i * chunk_bytes(r).
int staging_cache(const kvx_cache *cache, int n_blocks, int num_heads, int latents, uint64_t staging,
                  uint64_t staging_bytes, std::vector<kvx_region> &regions, std::vector<int32_t> &identity) {
    if (!cache || cache->n_regions < 0 || (cache->n_regions > 0 && !cache->regions))
        return fail(KVX_ERR_INVALID, "null cache");
    if (n_blocks < 0 || num_heads < 0) return fail(KVX_ERR_INVALID, "negative block or head count");
    if (!staging && n_blocks > 0) return fail(KVX_ERR_INVALID, "null staging buffer");
    regions.resize(cache->n_regions);
    uint64_t at = 0;
    for (int r = 0; r < cache->n_regions; ++r) {
        const kvx_region &a = cache->regions[r];
        uint64_t chunk = a.head_bytes ? (uint64_t)num_heads * a.head_bytes : (latents ? a.block_bytes : 0);
        regions[r].addr = staging + at;
        regions[r].block_bytes = chunk ? chunk : 1;
        regions[r].head_bytes = a.head_bytes;
        at += chunk * (uint64_t)n_blocks;
    }
    if (at > staging_bytes)
        return fail(KVX_ERR_RANGE, "staging needs %llu bytes, has %llu", (unsigned long long)at,
                    (unsigned long long)staging_bytes);
    identity.resize(n_blocks);
    for (int i = 0; i < n_blocks; ++i) identity[i] = i;
    return KVX_OK;
}

// Open IPC mappings in this process, by (device, allocation handle).
struct Mapping {
    void *base;
    int refs;
};
std::map<std::pair<int, std::string>, Mapping> g_mappings;

typedef int (*GetAddressRangeFn)(unsigned long long *, size_t *, unsigned long long);

int allocation_of(const void *ptr, uint64_t *base, size_t *size) {
    static GetAddressRangeFn fn = nullptr;
    if (!fn) {
        void *sym = nullptr;
        cudaDriverEntryPointQueryResult q;
        KVX_CUDA(cudaGetDriverEntryPoint("cuMemGetAddressRange", &sym, cudaEnableDefault, &q));
        if (!sym || q != cudaDriverEntryPointSuccess) return fail(KVX_ERR_CUDA, "cuMemGetAddressRange not found");
        fn = reinterpret_cast<GetAddressRangeFn>(sym);
    }
    unsigned long long b = 0;
    size_t s = 0;
    const int rc = fn(&b, &s, (unsigned long long)(uintptr_t)ptr);
    if (rc != 0) return fail(KVX_ERR_CUDA, "cuMemGetAddressRange failed with %d: not a device allocation", rc);
    *base = b;
    *size = s;
    return KVX_OK;
}

struct Xfer {
    cudaEvent_t done;
    int device;
    int32_t *status;  // the transfer's own status word
};

// ------------------------------------------------------------------------------------------------ doorbells

// A ring is an event recorded on the caller's stream; the doorbell's watcher thread queries its pending events
// every few microseconds (outside any interpreter lock) and writes the eventfd when one completes. Measured on B200
// with driver 580: a CUDA host callback (cudaLaunchHostFunc) or a blocking-sync event wakes a sleeping thread
// ~350-390 us after the work before it ends, a query loop ~15-45 us; the caller's stream never waits on a callback.
constexpr long kBellPollNs = 5000;

struct Bell {
    int fd = -1;
    std::mutex mu;
    std::condition_variable cv;
    std::vector<std::pair<cudaEvent_t, int>> pending;  // (event, device), guarded by mu
    bool stop = false;
    std::thread watcher;

    // A doorbell its owner never closed (a process leaving on an exception) is stopped when the registry goes at
    // exit: destroying a thread that can still be joined would end the process with std::terminate.
    ~Bell() {
        if (!watcher.joinable()) return;
        {
            std::lock_guard<std::mutex> lock(mu);
            stop = true;
        }
        cv.notify_one();
        watcher.join();
        if (fd >= 0) close(fd);
    }
};

void watch(Bell *bell) {
    prctl(PR_SET_TIMERSLACK, 1000UL, 0, 0, 0);  // a 5 us sleep stays near 5 us (the default slack is 50 us)
    int current = -1;
    std::vector<std::pair<cudaEvent_t, int>> items, ended;
    std::unique_lock<std::mutex> lock(bell->mu);
    while (true) {
        bell->cv.wait(lock, [bell] { return bell->stop || !bell->pending.empty(); });
        if (bell->stop) return;
        items = bell->pending;
        lock.unlock();
        ended.clear();
        for (const auto &item : items) {
            if (item.second != current && cudaSetDevice(item.second) == cudaSuccess) current = item.second;
            if (cudaEventQuery(item.first) != cudaErrorNotReady) ended.push_back(item);  // done, or failed: wake
        }
        (void)cudaGetLastError();
        if (!ended.empty()) {
            const uint64_t one = 1;
            (void)!write(bell->fd, &one, sizeof one);  // non-blocking; a full counter stays readable
            for (const auto &item : ended) cudaEventDestroy(item.first);
        }
        lock.lock();
        for (const auto &item : ended)
            bell->pending.erase(std::find(bell->pending.begin(), bell->pending.end(), item));
        if (!bell->pending.empty() && !bell->stop) {
            lock.unlock();
            const timespec pause{0, kBellPollNs};
            nanosleep(&pause, nullptr);
            lock.lock();
        }
    }
}

// ------------------------------------------------------------------------------------------------ step mailbox

constexpr uint64_t kMailboxHeader = 64;

uint64_t *mailbox_word(void *box, uint64_t offset) {
    return reinterpret_cast<uint64_t *>(static_cast<char *>(box) + offset);
}

uint64_t slot_offset(int rank, uint64_t slot_bytes) {
    return kMailboxHeader + (uint64_t)rank * ((16 + slot_bytes + 63) / 64 * 64);
}

double seconds_now() {
    timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec + t.tv_nsec * 1e-9;
}

// Waits until *word >= want (acquire): spins with yields for ~50 us, then sleeps 20 us at a time.
bool wait_word(const uint64_t *word, uint64_t want, double timeout_s) {
    const double deadline = seconds_now() + timeout_s;
    for (int spin = 0;; ++spin) {
        if (__atomic_load_n(word, __ATOMIC_ACQUIRE) >= want) return true;
        if (spin < 2000) {
            sched_yield();
            continue;
        }
        if (seconds_now() > deadline) return false;
        const timespec pause{0, 20000};
        nanosleep(&pause, nullptr);
    }
}

std::mutex g_bells_mu;
std::map<int, std::shared_ptr<Bell>> g_bells;  // open doorbells by id; ids are never reused
int g_next_bell = 1;

std::shared_ptr<Bell> find_bell(int id) {
    std::lock_guard<std::mutex> lock(g_bells_mu);
    auto it = g_bells.find(id);
    return it == g_bells.end() ? nullptr : it->second;
}

// ------------------------------------------------------------------------------------------------ status words

// One pinned host allocation of status words, mapped into every device (portable + mapped): with unified addressing
// a word has the same address on the host and on every device, so a kernel given it writes the host's memory
// directly. Words are handed out one at a time and zeroed when handed out; a word goes back only after the launches
// given it have completed, so no kernel still writes a word that is handed out again.
constexpr int kStatusWords = 1 << 16;

struct StatusPool {
    std::mutex mu;
    int32_t *words = nullptr;
    std::vector<int32_t> free;  // indices of words not in use
    std::vector<char> used;
};
StatusPool g_status;

int status_open(int32_t **out) {
    std::lock_guard<std::mutex> lock(g_status.mu);
    if (!g_status.words) {
        void *host = nullptr;
        KVX_CUDA(cudaHostAlloc(&host, kStatusWords * sizeof(int32_t), cudaHostAllocMapped | cudaHostAllocPortable));
        void *dev = nullptr;
        const cudaError_t e = cudaHostGetDevicePointer(&dev, host, 0);
        if (e != cudaSuccess || dev != host) {
            cudaFreeHost(host);
            return fail(KVX_ERR_CUDA, "status words are not mapped at their host address (%s)",
                        e == cudaSuccess ? "no unified addressing" : cudaGetErrorString(e));
        }
        std::memset(host, 0, kStatusWords * sizeof(int32_t));
        g_status.words = static_cast<int32_t *>(host);
        g_status.used.assign(kStatusWords, 0);
        g_status.free.reserve(kStatusWords);
        for (int i = kStatusWords - 1; i >= 0; --i) g_status.free.push_back(i);
    }
    if (g_status.free.empty()) return fail(KVX_ERR_RANGE, "all %d status words are in use", kStatusWords);
    const int i = g_status.free.back();
    g_status.free.pop_back();
    g_status.used[i] = 1;
    *reinterpret_cast<volatile int32_t *>(g_status.words + i) = 0;
    *out = g_status.words + i;
    return KVX_OK;
}

int status_close(int32_t *word) {
    std::lock_guard<std::mutex> lock(g_status.mu);
    const ptrdiff_t i = g_status.words ? word - g_status.words : -1;
    if (i < 0 || i >= kStatusWords || !g_status.used[i]) return fail(KVX_ERR_INVALID, "not an open status word");
    g_status.used[i] = 0;
    g_status.free.push_back((int32_t)i);
    return KVX_OK;
}

int32_t status_bits(const int32_t *word) { return *reinterpret_cast<const volatile int32_t *>(word); }

// A non-blocking stream of the library's own per device, for reading the diagnostic word without waiting on anyone
// else's streams.
std::mutex g_probe_mu;
std::map<int, cudaStream_t> g_probe_streams;

int probe_stream(int device, cudaStream_t *out) {
    std::lock_guard<std::mutex> lock(g_probe_mu);
    cudaStream_t &s = g_probe_streams[device];
    if (!s) KVX_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *out = s;
    return KVX_OK;
}

// ------------------------------------------------------------------------------------------------ process identity

// 16 random bytes drawn once per process: an IPC handle from this process carries them, so a handle is taken for
// this process's own memory only when its pid AND its nonce match. Processes in separate PID namespaces (containers)
// can share a pid; they do not share a nonce.
const unsigned char *process_nonce() {
    static unsigned char nonce[16];
    static std::once_flag once;
    std::call_once(once, [] {
        size_t got = 0;
        if (FILE *f = std::fopen("/dev/urandom", "rb")) {
            got = std::fread(nonce, 1, sizeof nonce, f);
            std::fclose(f);
        }
        if (got != sizeof nonce) {  // no urandom: mix what differs between processes
            timespec t;
            clock_gettime(CLOCK_REALTIME, &t);
            uint64_t mix[2] = {(uint64_t)t.tv_sec * 1000000007ull ^ (uint64_t)getpid(),
                               (uint64_t)t.tv_nsec ^ (uint64_t)(uintptr_t)&got};
            std::memcpy(nonce, mix, sizeof nonce);
        }
    });
    return nonce;
}

bool same_process(const kvx_ipc_handle *h) {
    return h->pid == (int32_t)getpid() && std::memcmp(h->nonce, process_nonce(), sizeof h->nonce) == 0;
}

}  // namespace

// ================================================================================================ C ABI

extern "C" {

int kvx_abi_version(void) { return KVX_ABI_VERSION; }

const char *kvx_last_error(void) { return t_error.c_str(); }

uint64_t kvx_launch_count(void) { return g_launches.load(); }

int kvx_ipc_export(const void *ptr, kvx_ipc_handle *out) {
    if (!ptr || !out) return fail(KVX_ERR_INVALID, "null pointer");
    cudaPointerAttributes attr;
    KVX_CUDA(cudaPointerGetAttributes(&attr, ptr));
    if (attr.type != cudaMemoryTypeDevice) return fail(KVX_ERR_INVALID, "not device memory");
    uint64_t base;
    size_t size;
    if (int rc = allocation_of(ptr, &base, &size)) return rc;
    cudaIpcMemHandle_t handle;
    KVX_CUDA(cudaIpcGetMemHandle(&handle, reinterpret_cast<void *>(base)));
    std::memset(out, 0, sizeof *out);
    static_assert(sizeof(handle) <= sizeof(out->handle), "handle size");
    std::memcpy(out->handle, &handle, sizeof handle);
    out->offset = (uint64_t)(uintptr_t)ptr - base;
    out->alloc_bytes = size;
    out->device = attr.device;
    out->pid = (int32_t)getpid();
    out->ptr = (uint64_t)(uintptr_t)ptr;
    std::memcpy(out->nonce, process_nonce(), sizeof out->nonce);
    return KVX_OK;
}

int kvx_ipc_open(const kvx_ipc_handle *h, void **out_ptr) {
    if (!h || !out_ptr) return fail(KVX_ERR_INVALID, "null pointer");
    int dev;
    KVX_CUDA(cudaGetDevice(&dev));
    if (same_process(h)) {  // our own allocation: CUDA IPC cannot reopen it, and need not
        if (h->device != dev) {  // ... but a kernel on this device reaches it only with peer access on
            int can = 0;
            if (int rc = kvx_enable_peer_access(dev, h->device, &can)) return rc;
            if (!can)
                return fail(KVX_ERR_INVALID, "device %d cannot reach device %d's memory directly", dev, h->device);
        }
        *out_ptr = reinterpret_cast<void *>(h->ptr);
        return KVX_OK;
    }
    const auto key = std::make_pair(dev, std::string(reinterpret_cast<const char *>(h->handle), 64));
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_mappings.find(key);
    if (it == g_mappings.end()) {
        cudaIpcMemHandle_t handle;
        std::memcpy(&handle, h->handle, sizeof handle);
        void *base = nullptr;
        KVX_CUDA(cudaIpcOpenMemHandle(&base, handle, cudaIpcMemLazyEnablePeerAccess));
        it = g_mappings.emplace(key, Mapping{base, 0}).first;
    }
    it->second.refs += 1;
    *out_ptr = static_cast<char *>(it->second.base) + h->offset;
    return KVX_OK;
}

int kvx_ipc_close(const kvx_ipc_handle *h) {
    if (!h) return fail(KVX_ERR_INVALID, "null pointer");
    if (same_process(h)) return KVX_OK;
    int dev;
    KVX_CUDA(cudaGetDevice(&dev));
    const auto key = std::make_pair(dev, std::string(reinterpret_cast<const char *>(h->handle), 64));
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_mappings.find(key);
    if (it == g_mappings.end()) return fail(KVX_ERR_INVALID, "handle not open on this device");
    if (--it->second.refs == 0) {
        void *base = it->second.base;
        g_mappings.erase(it);
        KVX_CUDA(cudaIpcCloseMemHandle(base));
    }
    return KVX_OK;
}

int kvx_enable_peer_access(int device, int peer, int *out_can_access) {
    if (!out_can_access) return fail(KVX_ERR_INVALID, "null pointer");
    *out_can_access = 0;
    if (device == peer) {
        *out_can_access = 1;
        return KVX_OK;
    }
    int can = 0;
    KVX_CUDA(cudaDeviceCanAccessPeer(&can, device, peer));
    if (!can) return KVX_OK;
    int prev;
    KVX_CUDA(cudaGetDevice(&prev));
    KVX_CUDA(cudaSetDevice(device));
    cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
        (void)cudaGetLastError();
        e = cudaSuccess;
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return fail(KVX_ERR_CUDA, "cudaDeviceEnablePeerAccess: %s", cudaGetErrorString(e));
    *out_can_access = 1;
    return KVX_OK;
}

int kvx_copy(const kvx_cache *caches, int n_caches, const kvx_job *jobs, int n_jobs, int flags, void *stream) {
    Range range("kvx_copy");
    return copy_impl(caches, n_caches, jobs, n_jobs, flags, static_cast<cudaStream_t>(stream));
}

int kvx_job_bytes(const kvx_cache *caches, int n_caches, const kvx_job *jobs, int n_jobs, uint64_t *out_bytes) {
    if (!out_bytes) return fail(KVX_ERR_INVALID, "null pointer");
    std::vector<Piece> pieces;
    uint64_t bytes, align_bits;
    if (int rc = plan(caches, n_caches, jobs, n_jobs, pieces, bytes, align_bits)) return rc;
    *out_bytes = bytes;
    return KVX_OK;
}

int kvx_pack(const kvx_cache *src, const int32_t *src_block_ids, int n_blocks, int first_head, int num_heads,
             int latents, void *staging, uint64_t staging_bytes, int flags, void *stream) {
    Range range("kvx_pack");
    std::vector<kvx_region> regions;
    std::vector<int32_t> identity;
    if (int rc = staging_cache(src, n_blocks, num_heads, latents, (uint64_t)(uintptr_t)staging, staging_bytes,
                               regions, identity))
        return rc;
    const kvx_cache caches[2] = {*src, kvx_cache{regions.data(), src->n_regions, n_blocks}};
    const kvx_job job = {0, 1, src_block_ids, identity.data(), n_blocks, first_head, 0, num_heads, latents};
    return copy_impl(caches, 2, &job, 1, flags, static_cast<cudaStream_t>(stream));
}

int kvx_scatter(const void *staging, uint64_t staging_bytes, const kvx_cache *dst, const int32_t *dst_block_ids,
                int n_blocks, int first_head, int num_heads, int latents, int flags, void *stream) {
    Range range("kvx_scatter");
    std::vector<kvx_region> regions;
    std::vector<int32_t> identity;
    if (int rc = staging_cache(dst, n_blocks, num_heads, latents, (uint64_t)(uintptr_t)staging, staging_bytes,
                               regions, identity))
        return rc;
    const kvx_cache caches[2] = {kvx_cache{regions.data(), dst->n_regions, n_blocks}, *dst};
    const kvx_job job = {0, 1, identity.data(), dst_block_ids, n_blocks, 0, first_head, num_heads, latents};
    return copy_impl(caches, 2, &job, 1, flags, static_cast<cudaStream_t>(stream));
}

int kvx_push(void *dst, const void *src, uint64_t bytes, int flags, void *stream) {
    Range range("kvx_push");
    if (bytes == 0) return KVX_OK;
    if (!dst || !src) return fail(KVX_ERR_INVALID, "null pointer");
    const kvx_region a = {(uint64_t)(uintptr_t)src, bytes, 0}, b = {(uint64_t)(uintptr_t)dst, bytes, 0};
    const kvx_cache caches[2] = {{&a, 1, 1}, {&b, 1, 1}};
    const int32_t zero = 0;
    const kvx_job job = {0, 1, &zero, &zero, 1, 0, 0, 0, 1};
    return copy_impl(caches, 2, &job, 1, flags, static_cast<cudaStream_t>(stream));
}

int kvx_store(const void *key, const void *value, int64_t key_stride, int64_t value_stride, int num_tokens,
              int num_heads, int head_bytes, const kvx_store_dest *dests, int n_dests, int32_t *status, int flags,
              void *stream) {
    Range range("kvx_store");
    if (!key || !dests) return fail(KVX_ERR_INVALID, "null rows or destinations");
    if (num_tokens < 0 || num_heads < 1 || head_bytes < 1)
        return fail(KVX_ERR_INVALID, "bad row shape: %d tokens, %d heads of %d bytes", num_tokens, num_heads,
                    head_bytes);
    if (n_dests < 1 || n_dests > kMaxStoreDests)
        return fail(KVX_ERR_INVALID, "%d destinations; 1 to %d", n_dests, kMaxStoreDests);
    StoreParams p{};
    p.key = (uint64_t)(uintptr_t)key;
    p.value = (uint64_t)(uintptr_t)value;
    p.key_stride = key_stride;
    p.value_stride = value_stride;
    p.num_tokens = num_tokens;
    p.num_heads = num_heads;
    p.head_bytes = head_bytes;
    p.n_dests = n_dests;
    p.peers_only = (flags & KVX_STORE_PEERS_ONLY) ? 1 : 0;
    p.status = status;
    uint64_t align_bits = p.key | p.value | (uint64_t)key_stride | (uint64_t)value_stride | (uint64_t)head_bytes;
    for (int d = 0; d < n_dests; ++d) {
        const kvx_store_dest &s = dests[d];
        if (!s.k_cache || (!value) != (!s.v_cache))
            return fail(KVX_ERR_INVALID, "destination %d: keys and values must match the rows given", d);
        if (s.block_size < 1 || s.num_blocks < 0 || (s.slot_bytes != 4 && s.slot_bytes != 8))
            return fail(KVX_ERR_INVALID, "destination %d: bad block size, block count or slot width", d);
        if (s.block_map && (d == 0 || s.block_size != dests[0].block_size || s.block_map_len < 0))
            return fail(KVX_ERR_INVALID, "destination %d: a block map needs a later destination of equal block size",
                        d);
        if (num_tokens > 0 && !s.slot_mapping && !s.block_map)
            return fail(KVX_ERR_INVALID, "destination %d: null slots", d);
        if (s.src_first_head < 0 || s.num_heads < 0 || s.dst_first_head < 0 ||
            (int64_t)s.src_first_head + s.num_heads > num_heads)
            return fail(KVX_ERR_RANGE, "destination %d: heads [%d, +%d) of %d", d, s.src_first_head, s.num_heads,
                        num_heads);
        if (s.block_stride < 0 || s.token_stride < 0 || s.head_stride < 0)
            return fail(KVX_ERR_INVALID, "destination %d: negative stride", d);
        if ((int64_t)s.num_blocks * s.block_size >= (int64_t)1 << 31)
            return fail(KVX_ERR_INVALID, "destination %d: more than 2^31 slots", d);
        int32_t shift = -1;
        for (int k = 0; k < 31; ++k)
            if (s.block_size == (1 << k)) shift = k;
        p.dests[d] = StoreDest{s.k_cache, s.v_cache, s.block_stride, s.token_stride, s.head_stride, s.slot_mapping,
                               s.block_map, s.block_size, s.num_blocks, s.slot_bytes, s.src_first_head, s.num_heads,
                               s.dst_first_head, s.block_map_len, shift};
        align_bits |= s.k_cache | s.v_cache | (uint64_t)s.block_stride | (uint64_t)s.token_stride |
                      (uint64_t)s.head_stride;
    }
    if (num_tokens == 0) return KVX_OK;
    const int vec = (int)std::min<uint64_t>(low_bit(align_bits), 16);
    DeviceInfo *info;
    if (int rc = device_info(&info)) return rc;
    const int sm_budget = (flags >> 24) & 0xff;
    const int sms = sm_budget > 0 && sm_budget < info->sms ? sm_budget : info->sms;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = (flags & KVX_STORE_SERIAL) ? 0 : 1;

    // Destination 0 with a power-of-two block size and strides below 2^32, and row strides below 2^32: the kernel's
    // address arithmetic then stays in 32-bit multiplies.
    const kvx_store_dest &d0 = dests[0];
    auto small = [](int64_t v) { return v >= 0 && v < ((int64_t)1 << 32); };
    const bool fast = p.dests[0].block_shift >= 0 && small(d0.block_stride) && small(d0.token_stride) &&
                      small(key_stride) && small(value_stride);
    const uint32_t parts = value ? 2u : 1u;

    int vi = 0;
    while ((16 >> vi) != vec) ++vi;
    void (*kernel)(StoreParams) =
        fast ? (vec == 16 ? kvx_store_kernel<16, true>
                : vec == 8 ? kvx_store_kernel<8, true>
                : vec == 4 ? kvx_store_kernel<4, true>
                : vec == 2 ? kvx_store_kernel<2, true>
                           : kvx_store_kernel<1, true>)
             : (vec == 16 ? kvx_store_kernel<16, false>
                : vec == 8 ? kvx_store_kernel<8, false>
                : vec == 4 ? kvx_store_kernel<4, false>
                : vec == 2 ? kvx_store_kernel<2, false>
                           : kvx_store_kernel<1, false>);
    int &occupancy = info->store_ctas_per_sm[vi][fast ? 1 : 0];
    if (occupancy == 0) {
        int occ = 0;
        KVX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, kStoreThreads, 0));
        occupancy = occ > 0 ? occ : 1;
    }
    const int ctas_per_sm = ((flags >> 16) & 0xff) ? ((flags >> 16) & 0xff) : occupancy;
    const uint64_t per_token = (uint64_t)parts * num_heads * (head_bytes / vec);
    const uint64_t tpp = per_token <= kStoreThreads ? kStoreThreads / per_token : 1;
    const uint64_t passes = ((uint64_t)num_tokens + tpp - 1) / tpp;
    // One resident wave: every CTA is on an SM from the start and sweeps its tokens; none waits for a second wave.
    cfg.gridDim = dim3((unsigned)std::min<uint64_t>(passes, (uint64_t)sms * ctas_per_sm));
    cfg.blockDim = dim3(kStoreThreads);
    KVX_CUDA(cudaLaunchKernelEx(&cfg, kernel, p));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return KVX_OK;
}

int kvx_transfer(const kvx_cache *caches, int n_caches, const kvx_job *jobs, int n_jobs, int flags,
                 void *wait_event, void *stream, kvx_xfer_t *out) {
    Range range("kvx_transfer");
    if (!out) return fail(KVX_ERR_INVALID, "null pointer");
    *out = nullptr;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int device;
    KVX_CUDA(cudaGetDevice(&device));
    int32_t *status = nullptr;
    if (int rc = status_open(&status)) return rc;
    cudaEvent_t done = nullptr;
    int rc = KVX_OK;
    cudaError_t e = cudaSuccess;
    const uint64_t launches_before = g_launches.load();
    if (wait_event) e = cudaStreamWaitEvent(s, static_cast<cudaEvent_t>(wait_event), 0);
    if (e == cudaSuccess) rc = copy_impl(caches, n_caches, jobs, n_jobs, flags, s, status);
    if (e == cudaSuccess && rc == KVX_OK) e = cudaEventCreateWithFlags(&done, cudaEventDisableTiming);
    if (e == cudaSuccess && rc == KVX_OK) e = cudaEventRecord(done, s);
    if (e != cudaSuccess || rc != KVX_OK) {
        if (done) cudaEventDestroy(done);
        if (rc == KVX_OK) rc = fail(KVX_ERR_CUDA, "posting a transfer: %s", cudaGetErrorString(e));
        // A launch that went out before the failure may still write the word: then it stays out of circulation
        // (one word lost) rather than reach a later transfer.
        if (g_launches.load() == launches_before) {
            const std::string why = t_error;
            (void)status_close(status);
            t_error = why;
        }
        return rc;
    }
    *out = reinterpret_cast<kvx_xfer_t>(new Xfer{done, device, status});
    return KVX_OK;
}

// One event per device for kvx_transfer_after: recorded on the caller's stream and waited for on the copy stream
// under one lock, so every wait captures its own record (a wait is bound to the record before it, not to later ones).
std::mutex g_after_mu;
std::map<int, cudaEvent_t> g_after_events;

int kvx_transfer_after(const kvx_cache *caches, int n_caches, const kvx_job *jobs, int n_jobs, int flags,
                       void *after_stream, void *stream, kvx_xfer_t *out) {
    if (!out) return fail(KVX_ERR_INVALID, "null pointer");
    *out = nullptr;
    int device;
    KVX_CUDA(cudaGetDevice(&device));
    {
        std::lock_guard<std::mutex> lock(g_after_mu);
        cudaEvent_t &after = g_after_events[device];
        if (!after) KVX_CUDA(cudaEventCreateWithFlags(&after, cudaEventDisableTiming));
        KVX_CUDA(cudaEventRecord(after, static_cast<cudaStream_t>(after_stream)));
        KVX_CUDA(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), after, 0));
    }
    return kvx_transfer(caches, n_caches, jobs, n_jobs, flags, nullptr, stream, out);
}

int kvx_check_xfer(kvx_xfer_t xfer) {
    if (!xfer) return fail(KVX_ERR_INVALID, "null transfer");
    Xfer *x = reinterpret_cast<Xfer *>(xfer);
    const cudaError_t e = cudaEventQuery(x->done);
    if (e == cudaErrorNotReady) {
        (void)cudaGetLastError();
        return KVX_PENDING;
    }
    if (e != cudaSuccess) return fail(KVX_ERR_CUDA, "transfer failed: %s", cudaGetErrorString(e));
    // The event says the launch ended. A TMA copy that gave up a bounded wait ends too, with its bytes not all
    // landed, and says so only in the transfer's status word, which the completed event has made visible here.
    if (status_bits(x->status) & kErrCopyWait)
        return fail(KVX_ERR_DEVICE, "a copy of this transfer on device %d gave up a bounded wait, so not every byte "
                    "landed", x->device);
    return KVX_OK;
}

int kvx_release_xfer(kvx_xfer_t xfer) {
    if (!xfer) return KVX_OK;
    Xfer *x = reinterpret_cast<Xfer *>(xfer);
    const cudaError_t e = cudaEventDestroy(x->done);
    // A transfer is released once it has completed, or once nothing will ask about it again after the device
    // finished (the caller waits first): its word may then go to another transfer.
    (void)status_close(x->status);
    delete x;
    if (e != cudaSuccess) return fail(KVX_ERR_CUDA, "cudaEventDestroy: %s", cudaGetErrorString(e));
    return KVX_OK;
}

int kvx_doorbell_open(int *out_id, int *out_fd) {
    if (!out_id || !out_fd) return fail(KVX_ERR_INVALID, "null pointer");
    auto bell = std::make_shared<Bell>();
    bell->fd = eventfd(0, EFD_NONBLOCK | EFD_CLOEXEC);
    if (bell->fd < 0) return fail(KVX_ERR_INVALID, "eventfd: %s", strerror(errno));
    try {
        bell->watcher = std::thread(watch, bell.get());
    } catch (const std::exception &error) {
        close(bell->fd);
        return fail(KVX_ERR_INVALID, "doorbell thread: %s", error.what());
    }
    std::lock_guard<std::mutex> lock(g_bells_mu);
    const int id = g_next_bell++;
    g_bells[id] = bell;
    *out_id = id;
    *out_fd = bell->fd;
    return KVX_OK;
}

int kvx_doorbell_ring_after(int id, void *stream) {
    auto bell = find_bell(id);
    if (!bell) return fail(KVX_ERR_INVALID, "no open doorbell %d", id);
    int device;
    KVX_CUDA(cudaGetDevice(&device));
    cudaEvent_t mark;
    KVX_CUDA(cudaEventCreateWithFlags(&mark, cudaEventDisableTiming));
    const cudaError_t e = cudaEventRecord(mark, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        cudaEventDestroy(mark);
        return fail(KVX_ERR_CUDA, "doorbell ring: %s", cudaGetErrorString(e));
    }
    {
        std::lock_guard<std::mutex> lock(bell->mu);
        bell->pending.emplace_back(mark, device);
    }
    bell->cv.notify_one();
    return KVX_OK;
}

int kvx_doorbell_close(int id) {
    std::shared_ptr<Bell> bell;
    {
        std::lock_guard<std::mutex> lock(g_bells_mu);
        auto it = g_bells.find(id);
        if (it == g_bells.end()) return fail(KVX_ERR_INVALID, "no open doorbell %d", id);
        bell = it->second;
        g_bells.erase(it);
    }
    {
        std::lock_guard<std::mutex> lock(bell->mu);
        bell->stop = true;
    }
    bell->cv.notify_one();
    bell->watcher.join();  // returns within one poll interval
    for (const auto &item : bell->pending) cudaEventDestroy(item.first);  // rings that never came
    bell->pending.clear();
    close(bell->fd);
    return KVX_OK;
}

uint64_t kvx_mailbox_stride(uint64_t slot_bytes) { return (16 + slot_bytes + 63) / 64 * 64; }

uint64_t kvx_mailbox_bytes(int world, uint64_t slot_bytes) {
    return world < 1 ? 0 : slot_offset(world, slot_bytes);
}

int kvx_mailbox_post(void *box, int world, int rank, uint64_t slot_bytes, uint64_t seq, const void *data,
                     uint64_t len, double timeout_s) {
    if (!box || rank < 1 || rank >= world || seq < 1 || (len && !data))
        return fail(KVX_ERR_INVALID, "mailbox post: rank %d of %d, step %llu", rank, world, (unsigned long long)seq);
    if (len > slot_bytes)
        return fail(KVX_ERR_RANGE, "a step output of %llu bytes does not fit a %llu-byte mailbox slot",
                    (unsigned long long)len, (unsigned long long)slot_bytes);
    if (!wait_word(mailbox_word(box, 0), seq - 1, timeout_s))
        return fail(KVX_ERR_TIMEOUT, "rank 0 did not read step %llu within %.1f s", (unsigned long long)(seq - 1),
                    timeout_s);
    const uint64_t at = slot_offset(rank, slot_bytes);
    if (len) memcpy(static_cast<char *>(box) + at + 16, data, len);
    __atomic_store_n(mailbox_word(box, at + 8), len, __ATOMIC_RELAXED);
    __atomic_store_n(mailbox_word(box, at), seq, __ATOMIC_RELEASE);
    return KVX_OK;
}

int kvx_mailbox_collect(void *box, int world, uint64_t slot_bytes, uint64_t seq, uint64_t *lens, double timeout_s) {
    if (!box || !lens || world < 1 || seq < 1) return fail(KVX_ERR_INVALID, "mailbox collect: bad arguments");
    lens[0] = 0;
    for (int rank = 1; rank < world; ++rank) {
        const uint64_t at = slot_offset(rank, slot_bytes);
        if (!wait_word(mailbox_word(box, at), seq, timeout_s))
            return fail(KVX_ERR_TIMEOUT, "rank %d did not post step %llu within %.1f s", rank,
                        (unsigned long long)seq, timeout_s);
        lens[rank] = __atomic_load_n(mailbox_word(box, at + 8), __ATOMIC_RELAXED);
        if (lens[rank] > slot_bytes) return fail(KVX_ERR_RANGE, "rank %d posted a corrupt length", rank);
    }
    return KVX_OK;
}

int kvx_mailbox_release(void *box, uint64_t seq) {
    if (!box) return fail(KVX_ERR_INVALID, "null mailbox");
    __atomic_store_n(mailbox_word(box, 0), seq, __ATOMIC_RELEASE);
    return KVX_OK;
}

int kvx_wait_selftest(int limit_us, int code, int32_t *status, void *stream) {
    if (limit_us < 1 || limit_us > 10000000) return fail(KVX_ERR_INVALID, "limit %d us: 1 us to 10 s", limit_us);
    if (code != kErrSelftest && code != kErrCopyWait)
        return fail(KVX_ERR_INVALID, "code %d: %d (the self-test's) or %d (a stuck copy's)", code, kErrSelftest,
                    kErrCopyWait);
    kvx_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>((uint64_t)limit_us * 1000, code,
                                                                               status);
    KVX_CUDA(cudaGetLastError());
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return KVX_OK;
}

int kvx_device_error(int *out_code) {
    if (!out_code) return fail(KVX_ERR_INVALID, "null pointer");
    int device;
    KVX_CUDA(cudaGetDevice(&device));
    cudaStream_t s;
    if (int rc = probe_stream(device, &s)) return rc;
    int32_t *word;
    if (int rc = status_open(&word)) return rc;
    kvx_take_device_error_kernel<<<1, 32, 0, s>>>(word);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) {
        g_launches.fetch_add(1, std::memory_order_relaxed);
        *out_code = status_bits(word);
    }
    (void)status_close(word);  // the kernel has completed, or never ran
    if (e != cudaSuccess) return fail(KVX_ERR_CUDA, "reading the device error word: %s", cudaGetErrorString(e));
    return KVX_OK;
}

int kvx_status_open(int32_t **out_word) {
    if (!out_word) return fail(KVX_ERR_INVALID, "null pointer");
    return status_open(out_word);
}

int kvx_status_close(int32_t *word) { return status_close(word); }

int kvx_status_read(const int32_t *word, int32_t *out_bits) {
    if (!word || !out_bits) return fail(KVX_ERR_INVALID, "null pointer");
    *out_bits = status_bits(word);
    return KVX_OK;
}

int kvx_xfer_status(kvx_xfer_t xfer, int32_t **out_word) {
    if (!xfer || !out_word) return fail(KVX_ERR_INVALID, "null pointer");
    *out_word = reinterpret_cast<Xfer *>(xfer)->status;
    return KVX_OK;
}

}  // extern "C"
