/*
 * CPU oracle for the prefill->decode KV-cache transfer, in plain C. TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this library, as the checker or as the
 * timed CPU baseline. The product library (lean_vllm_b200/libkvx.so) does not link it and has no CPU fallback.
 *
 * It restates lean-vLLM's NixlConnector load (lean_vllm/kv_transfer/nixl_connector.py):
 *   kvx_oracle_head_shares  -- head_shares, nixl_connector.py:69-77
 *   kvx_oracle_block_descs  -- block_descs, nixl_connector.py:89-108 (region-major rows)
 *   kvx_oracle_read         -- a READ as one memmove per (local, remote) row pair, as the reference's CPU tests
 *                              model NIXL (tests/test_nixl_connector.py:83-89); rows are split over `threads`
 *                              POSIX threads, since the rows of one READ are disjoint.
 * Build: oracle/Makefile -> oracle/_build/libkvx_oracle.so.
 */
#include <pthread.h>
#include <stdint.h>
#include <string.h>

typedef struct {
    uint64_t addr;        /* of block 0 */
    uint64_t block_bytes; /* between blocks */
    uint64_t head_bytes;  /* one head's tokens in a block; 0 for latents */
} kvx_oracle_region;

/* Writes up to `max` shares as (remote_rank, remote_head, local_head, num_heads) int quadruples; returns the count. */
int kvx_oracle_head_shares(int rank, int tp_size, int remote_tp_size, int num_heads, int *out, int max) {
    int mine = num_heads / tp_size, theirs = num_heads / remote_tp_size;
    int lo = rank * mine, hi = (rank + 1) * mine, n = 0;
    for (int q = lo / theirs; q * theirs < hi; ++q) {
        int a = lo > q * theirs ? lo : q * theirs;
        int b = hi < (q + 1) * theirs ? hi : (q + 1) * theirs;
        if (n < max) {
            out[4 * n + 0] = q;
            out[4 * n + 1] = a - q * theirs;
            out[4 * n + 2] = a - lo;
            out[4 * n + 3] = b - a;
        }
        ++n;
    }
    return n;
}

/* Region-major (addr, len) rows; returns the number of rows written (at most `max`). */
int64_t kvx_oracle_block_descs(const kvx_oracle_region *regions, int n_regions, const int32_t *ids, int n_blocks,
                               int first_head, int num_heads, int latents, uint64_t *addr, uint64_t *len,
                               int64_t max) {
    int64_t n = 0;
    for (int r = 0; r < n_regions; ++r) {
        uint64_t base, length;
        if (regions[r].head_bytes) {
            base = regions[r].addr + (uint64_t)first_head * regions[r].head_bytes;
            length = (uint64_t)num_heads * regions[r].head_bytes;
        } else if (latents) {
            base = regions[r].addr;
            length = regions[r].block_bytes;
        } else {
            continue;
        }
        for (int i = 0; i < n_blocks; ++i) {
            if (n < max) {
                addr[n] = base + (uint64_t)ids[i] * regions[r].block_bytes;
                len[n] = length;
            }
            ++n;
        }
    }
    return n;
}

typedef struct {
    const uint64_t *dst, *src, *len;
    int64_t lo, hi;
} read_span;

static void *read_worker(void *arg) {
    const read_span *s = (const read_span *)arg;
    for (int64_t i = s->lo; i < s->hi; ++i)
        memmove((void *)(uintptr_t)s->dst[i], (const void *)(uintptr_t)s->src[i], (size_t)s->len[i]);
    return 0;
}

/* Copies row i's len[i] bytes from src[i] to dst[i] for every row; returns the bytes moved, or -1 on a thread error.
 * Rows are divided into `threads` contiguous spans of equal byte weight. */
int64_t kvx_oracle_read(const uint64_t *dst, const uint64_t *src, const uint64_t *len, int64_t n, int threads) {
    enum { MAX_THREADS = 256 };
    int64_t total = 0;
    for (int64_t i = 0; i < n; ++i) total += (int64_t)len[i];
    if (threads < 1) threads = 1;
    if (threads > MAX_THREADS) threads = MAX_THREADS;
    if (threads == 1 || n < 2) {
        read_span s = {dst, src, len, 0, n};
        read_worker(&s);
        return total;
    }
    pthread_t tid[MAX_THREADS];
    read_span spans[MAX_THREADS];
    int64_t row = 0, acc = 0;
    int used = 0;
    for (int t = 0; t < threads && row < n; ++t) {
        int64_t goal = total * (t + 1) / threads;
        int64_t start = row;
        while (row < n && (acc < goal || row == start)) acc += (int64_t)len[row++];
        if (t == threads - 1) row = n;
        spans[used] = (read_span){dst, src, len, start, row};
        if (pthread_create(&tid[used], 0, read_worker, &spans[used]) != 0) {
            for (int k = 0; k < used; ++k) pthread_join(tid[k], 0);
            return -1;
        }
        ++used;
    }
    for (int k = 0; k < used; ++k) pthread_join(tid[k], 0);
    return total;
}
