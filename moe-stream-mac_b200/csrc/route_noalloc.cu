/* route_noalloc.cu: fp32-router routing that allocates no device memory.
 *
 * qe_moe_route and qe_moe_forward keep their logits in a workspace the library grows with cudaMalloc.
 * Some callers cannot let a library allocate: a host framework whose caching allocator already holds the
 * device memory (a cudaMalloc from the side can fail although the framework has room), or a decode loop
 * that cannot afford the device-wide synchronisation cudaMalloc/cudaFree may cause. This entry point
 * takes every input and output as a device pointer and keeps its only scratch, the logits, in a fixed
 * file-scope device array.
 *
 * The array is QE_NOALLOC_LOGITS floats (4 MiB) on every GPU that loads the library, held until the
 * process exits. All calls on a device share it, so calls that overlap on the GPU (different streams, or
 * threads) race; the router kernel rewrites every logit a call uses, so nothing needs clearing between
 * calls. Host code cannot use the array's name as a device address: the first call on each device looks
 * the address up with cudaGetSymbolAddress (with that device current) and caches it, so that first call
 * should come before any stream capture.
 */
#include <atomic>

#include "qe_common.cuh"
#include "qe_kernels.h"
#include "../../include/qe_moe.h"

#define QE_NOALLOC_LOGITS (1u << 20)

static __device__ __align__(256) float qe_noalloc_logits[QE_NOALLOC_LOGITS];

/* device address of qe_noalloc_logits, per device; atomic, since two host threads may make their first calls on a
 * device at the same time (both then store the same address) */
static std::atomic<float *> g_noalloc_logits[64];

extern "C" int qe_route_f32_noalloc(const float *router_w, const float *router_bias, const float *x, int T, int hidden,
                                    int E, int top_k, int32_t *idx, float *score, void *stream) {
    if (!router_w || !x || !idx || !score) QE_FAIL("route_noalloc: null pointer");
    if (T < 1 || hidden < 1 || hidden > 8192) QE_FAIL("route_noalloc: T=%d hidden=%d out of range", T, hidden);
    if (E < 1 || E > 512 || top_k < 1 || top_k > 16 || top_k > E)
        QE_FAIL("route_noalloc: E=%d top_k=%d out of range", E, top_k);
    if ((size_t)T * (size_t)(E + 1) > QE_NOALLOC_LOGITS)
        QE_FAIL("route_noalloc: T*(E+1) = %zu logits exceed the fixed %u-float scratch (T <= %u at E=%d)",
                (size_t)T * (size_t)(E + 1), QE_NOALLOC_LOGITS, QE_NOALLOC_LOGITS / (unsigned)(E + 1), E);
    int dev = 0;
    QE_CHECK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) QE_FAIL("route_noalloc: device %d out of range", dev);
    float *logits = g_noalloc_logits[dev].load(std::memory_order_acquire);
    if (!logits) {
        void *p = nullptr;
        QE_CHECK(cudaGetSymbolAddress(&p, qe_noalloc_logits));
        logits = static_cast<float *>(p);
        g_noalloc_logits[dev].store(logits, std::memory_order_release);
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (qe_launch_router_f32(router_w, router_bias, x, T, hidden, E, logits, nullptr, nullptr, nullptr, s) < 0)
        return -1;
    return qe_launch_route_topk(logits, E + 1, T, E, top_k, idx, score, nullptr, s);
}
