// qmm_linear_splitk_static: the split-K GEMM with its f32 partial-sum scratch
// in a file-scope device array instead of a caller-provided workspace.
//
// Who needs it: code that runs as a custom op or plug-in inside a host that
// owns all device memory through its own pool and hands plug-ins no allocator
// (an inference server's or framework's extension interface), where a private
// cudaMalloc would fall outside the host's memory budget; and latency-critical
// paths that must not pay the device-wide synchronization cudaMalloc/cudaFree
// can imply.  This entry point allocates nothing: the scratch is part of the
// library's device image, so every GPU that loads the library holds its 16 MiB
// until the process exits.  In host code the array's name is only a host-side
// stand-in, so its device address is resolved once per device, with that
// device current, by cudaGetSymbolAddress, and that address is what the
// kernels get.
//
// Contract (also stated in include/qmm.h):
//   - at most kStaticScratchBytes (16 MiB) of scratch: splits * m * n * 4 bytes;
//     larger requests fail with QMM_ERR_UNSUPPORTED before anything is launched;
//   - the scratch keeps whatever the last call left in it; nothing has to
//     start at zero, because every split writes its whole partial tile before
//     the reduction reads it;
//   - all calls on a device share the one scratch array, so calls that may
//     overlap on the GPU (different streams, host threads, processes sharing a
//     context) race; order them on one stream;
//   - the first call on a device resolves the scratch address (a runtime
//     call, not a stream operation): make it before any stream capture;
//   - the address is kept for the life of the process: after a
//     cudaDeviceReset (or anything else that destroys the device's primary
//     context) the library's device image is loaded anew and this entry point
//     must not be called again in that process.
#include <mutex>

#include "qmm_internal.h"

namespace qmm {
namespace {

constexpr uint64_t kStaticScratchBytes = 16ull << 20;
constexpr int kMaxScratchDevices = 64;

static __device__ __align__(256) float g_static_scratch[kStaticScratchBytes / sizeof(float)];

std::mutex g_scratch_mutex;
void *g_scratch_addr[kMaxScratchDevices] = {};

qmm_status static_scratch(void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "no CUDA device");
    if (dev < 0 || dev >= kMaxScratchDevices)
        return fail(QMM_ERR_UNSUPPORTED, "device %d is beyond the %d devices the static scratch serves", dev,
                    kMaxScratchDevices);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "static scratch address");
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return QMM_OK;
}

}  // namespace
}  // namespace qmm

extern "C" {

uint64_t qmm_static_scratch_bytes(void) { return qmm::kStaticScratchBytes; }

qmm_status qmm_linear_splitk_static(const qmm_weight *w, const uint16_t *x, int64_t m,
                                    const qmm_epilogue *ep, uint16_t *y, int32_t splits, void *stream) {
    if (!w) return qmm::fail(QMM_ERR_INVALID_ARGUMENT, "null weight");
    if (splits < 1 || splits > 16)
        return qmm::fail(QMM_ERR_INVALID_ARGUMENT, "split count %d is not in [1, 16]", splits);
    if (m < 0 || w->n <= 0) return qmm::fail(QMM_ERR_BAD_SHAPE, "%lld tokens of %lld outputs", (long long)m,
                                             (long long)w->n);
    // splits * m * n * 4 bytes, compared without forming a product that could
    // wrap: m * n must be at most the scratch's floats divided by the splits.
    const uint64_t floats = qmm::kStaticScratchBytes / sizeof(float) / (uint64_t)splits;
    if (splits > 1 && m > 0 && (uint64_t)m > floats / (uint64_t)w->n)
        return qmm::fail(QMM_ERR_UNSUPPORTED,
                         "split-k with %d splits of %lld x %lld needs more than the static scratch's %llu bytes "
                         "(use qmm_linear_splitk with a caller workspace, or fewer splits)",
                         splits, (long long)m, (long long)w->n, (unsigned long long)qmm::kStaticScratchBytes);
    const uint64_t need = qmm_splitk_workspace_bytes(w, m, splits);
    if (need > qmm::kStaticScratchBytes)
        return qmm::fail(QMM_ERR_UNSUPPORTED,
                         "split-k with %d splits of %lld x %lld needs %llu bytes of scratch; the static scratch "
                         "holds %llu (use qmm_linear_splitk with a caller workspace, or fewer splits)",
                         splits, (long long)m, (long long)w->n, (unsigned long long)need,
                         (unsigned long long)qmm::kStaticScratchBytes);
    void *scratch = nullptr;
    if (need > 0) {
        qmm_status s = qmm::static_scratch(&scratch);
        if (s != QMM_OK) return s;
    }
    return qmm_linear_splitk(w, x, m, ep, y, splits, scratch, qmm::kStaticScratchBytes, stream);
}

}  // extern "C"
