/* bucket.cu: token bucketing for the expert kernels.
 *
 * Replaces the reference's per-token expert loop (engine/src/moe_layer.c:79-83, prefill = T calls) and
 * the batched template of its MLX path (engine/hybrid/hybrid.py:177-189: unique experts + inverse index,
 * tokens sorted by expert) with a histogram + prefix scan + scatter on the GPU. Every (token, slot) pair
 * p = t*(k+1) + j (j = k is the shared expert) lands in its expert's bucket (slots whose expert id is outside
 * [0, E) are skipped: the experts another GPU owns); the active buckets and the
 * work items of the gate/up and down kernels are listed so those kernels run a compact grid.
 * Numerics do not depend on the order of pairs inside a bucket (every pair is an independent MMA column).
 */
#include "qe_common.cuh"
#include "qe_kernels.h"

namespace {

constexpr int kThreads = 1024;

/* Exclusive scan of n ints in place by one warp (n <= a few thousand). Returns the total. */
__device__ int warp_exclusive_scan(int *a, int n, int lane) {
    const int per = (n + 31) / 32;
    const int b0 = lane * per, b1 = min(n, b0 + per);
    int local = 0;
    for (int i = b0; i < b1; i++) local += a[i];
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(QE_FULL, incl, o);
        if (lane >= o) incl += v;
    }
    int run = incl - local;
    for (int i = b0; i < b1; i++) {
        const int v = a[i];
        a[i] = run;
        run += v;
    }
    return __shfl_sync(QE_FULL, incl, 31);
}

/* two compact arrays of E+2 ints after the six per-expert arrays */
__device__ __forceinline__ int *cnt_tmp(int *sm, int E) { return sm + 6 * (E + 2); }

__global__ void __launch_bounds__(kThreads) bucket_kernel(const int32_t *__restrict__ idx, int T, int E, int k,
                                                          int shared_tokens, int shared_first, int tiles_gu,
                                                          int tiles_sh_gu, int tiles_dn, int chunk, QeBuckets b) {
    extern __shared__ int sm[];
    int *cnt = sm;                 /* [E+1] */
    int *off = cnt + (E + 1);      /* [E+2] */
    int *cur = off + (E + 2);      /* [E+1] */
    int *flag = cur + (E + 1);     /* [E+2] active-slot scan */
    int *igu = flag + (E + 2);     /* [E+2] */
    int *idn = igu + (E + 2);      /* [E+2] */
    const int tid = threadIdx.x, lane = tid & 31;
    for (int e = tid; e <= E; e += kThreads) cnt[e] = 0;
    __syncthreads();
    const int npairs = T * k;
    for (int q = tid; q < npairs; q += kThreads) {
        const int e = idx[q];
        if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (tid == 0) cnt[E] = shared_tokens;   /* rows shared_first.. of the batch, or 0 (computed elsewhere) */
    __syncthreads();
    for (int e = tid; e <= E; e += kThreads) {
        off[e] = cnt[e];
        const int active = cnt[e] > 0;
        flag[e] = active;
        const int chunks = (cnt[e] + chunk - 1) / chunk;
        igu[e] = chunks * (e == E ? tiles_sh_gu : tiles_gu);
        idn[e] = chunks * tiles_dn;
    }
    __syncthreads();
    if (tid < 32) {
        const int total = warp_exclusive_scan(off, E + 1, lane);
        if (lane == 0) off[E + 1] = total;
    } else if (tid < 64) {
        const int na = warp_exclusive_scan(flag, E + 1, lane);
        if (lane == 0) flag[E + 1] = na;
    }
    __syncthreads();
    /* active slots in expert order: slot_expert[a] = e; their work-item counts, compacted and scanned in
     * shared memory (igu/idn are reused as the compact arrays: entry a <= e, written after a barrier) */
    int *cgu = cnt_tmp(sm, E);                  /* [E+2] compact gate/up item counts */
    int *cdn = cgu + (E + 2);                   /* [E+2] compact down item counts   */
    for (int e = tid; e <= E; e += kThreads) {
        cur[e] = off[e];
        if (cnt[e] > 0) {
            const int a = flag[e];
            b.slot_expert[a] = e;
            cgu[a] = igu[e];
            cdn[a] = idn[e];
        }
    }
    __syncthreads();
    const int na = flag[E + 1];
    if (tid < 32) {
        const int tot = warp_exclusive_scan(cgu, na, lane);
        if (lane == 0) cgu[na] = tot;
    } else if (tid < 64) {
        const int tot = warp_exclusive_scan(cdn, na, lane);
        if (lane == 0) cdn[na] = tot;
    }
    __syncthreads();
    /* with one gate/up tile per expert, the items are the chunks themselves: list them (at most one per pair) */
    if (b.chunks && tiles_gu == 1 && tiles_sh_gu == 1) {
        for (int e = tid; e <= E; e += kThreads) {
            const int n = cnt[e];
            if (n == 0) continue;
            const int base = cgu[flag[e]];
            for (int c = 0, n0 = 0; n0 < n; c++, n0 += chunk)
                b.chunks[base + c] = make_int4(e, off[e] + n0, min(chunk, n - n0), 0);
        }
    }
    for (int a = tid; a <= na; a += kThreads) {
        b.slot_items[a] = cgu[a];
        b.slot_items[(E + 2) + a] = cdn[a];
    }
    if (tid == 0) {
        b.n_active[0] = na;
        b.n_active[1] = cgu[na];
        b.n_active[2] = cdn[na];
    }
    /* scatter the pairs into their buckets */
    for (int q = tid; q < npairs; q += kThreads) {
        const int e = idx[q];
        if (e < 0 || e >= E) continue;
        const int t = q / k, j = q % k;
        const int pos = atomicAdd(&cur[e], 1);
        b.pairs[pos] = t * (k + 1) + j;
    }
    for (int t = tid; t < shared_tokens; t += kThreads) b.pairs[off[E] + t] = (shared_first + t) * (k + 1) + k;
    for (int e = tid; e <= E; e += kThreads) {
        b.counts[e] = cnt[e];
        b.offsets[e] = off[e];
    }
    if (tid == 0) b.offsets[E + 1] = off[E + 1];
}

}  // namespace

int qe_launch_bucket(const int32_t *idx, int T, int E, int k, int shared_tokens, int tiles_gu, int tiles_sh_gu,
                     int tiles_dn, int chunk, const QeBuckets *b, cudaStream_t s, int shared_first) {
    if (shared_first < 0 || shared_tokens < 0 || shared_first + shared_tokens > T)
        QE_FAIL("bucket: shared rows [%d, %d) outside the batch of %d", shared_first, shared_first + shared_tokens, T);
    const size_t smem = sizeof(int) * (size_t)(8 * (E + 2));
    bucket_kernel<<<1, kThreads, smem, s>>>(idx, T, E, k, shared_tokens, shared_first, tiles_gu, tiles_sh_gu, tiles_dn,
                                            chunk, *b);
    QE_CHECK(cudaGetLastError());
    return 0;
}
