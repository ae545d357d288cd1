// C ABI of libqmm (include/qmm.h): argument validation, kernel dispatch,
// error reporting.
//
// Validation mirrors image-forger's `Linear::load` (src/quant.rs:43-77) and
// the shape checks of its Qmm/Dequantize custom ops (src/quant.rs:438-451,
// 505-513, 589-598).  Dispatch mirrors `Module::forward` (src/quant.rs:115-124):
// layouts the fused kernels cover run fused; anything else returns
// QMM_ERR_UNSUPPORTED so the caller dequantizes and runs a dense GEMM, the way
// the reference falls back to `self.dense()?.forward(x)` (src/quant.rs:121).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>

#include "qmm_common.cuh"
#include "qmm_internal.h"

namespace qmm {

// The device-side error word that bounded waits write (see qmm_common.cuh).
__device__ uint32_t g_device_error = 0;

namespace {
thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {};
uint32_t *g_err_addr[kMaxDevices] = {};
std::mutex g_dev_mutex;

int current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    return dev;
}
}  // namespace

qmm_status fail(qmm_status status, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return status;
}

qmm_status cuda_fail(cudaError_t e, const char *what) {
    return fail(QMM_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

uint32_t *device_error_word() {
    const int dev = current_device();
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (!g_err_addr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess)
            g_err_addr[dev] = static_cast<uint32_t *>(p);
    }
    return g_err_addr[dev];
}

std::atomic<int> g_sm_budget{0};

int sm_count() {
    const int dev = current_device();
    if (g_sm_count[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        g_sm_count[dev] = n;
    }
    const int budget = g_sm_budget.load(std::memory_order_relaxed);
    return budget > 0 && budget < g_sm_count[dev] ? budget : g_sm_count[dev];
}

void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

namespace {
std::atomic<int32_t> g_weights_immutable{0};
}  // namespace

bool weights_immutable() { return g_weights_immutable.load(std::memory_order_relaxed) != 0; }

bool gemv_pdl_enabled() {
    static const bool on = [] {
        const char *v = getenv("QMM_GEMV_PDL");
        return !(v && v[0] == '0' && v[1] == '\0');
    }();
    return on;
}

}  // namespace qmm

using qmm::fail;

// An empty kernel whose attributes report the architecture the library's
// device code was built for (qmm_binary_version).
__global__ void qmm_arch_probe_kernel() {}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// qmm_activation in the low byte, optionally QMM_EPILOGUE_RESIDUAL_MUL.
static bool valid_activation(int32_t a) {
    const int32_t act = a & 0xFF;
    return (a & ~(0xFF | QMM_EPILOGUE_RESIDUAL_MUL)) == 0 && act >= QMM_ACT_NONE && act <= QMM_ACT_SILU;
}

static qmm_status check_device() {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return qmm::cuda_fail(e, "no CUDA device");
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (major != 10) return fail(QMM_ERR_CUDA, "device %d is not sm_100 (compute capability %d.x)", dev, major);
    return QMM_OK;
}

extern "C" {

int32_t qmm_abi_version(void) { return QMM_ABI_VERSION; }

const char *qmm_last_error(void) { return qmm::t_last_error.c_str(); }

uint64_t qmm_launch_count(void) { return qmm::g_launches.load(std::memory_order_relaxed); }

qmm_status qmm_binary_version(int32_t *binary_version, int32_t *ptx_version) {
    if (!binary_version || !ptx_version) return fail(QMM_ERR_INVALID_ARGUMENT, "null output pointer");
    cudaFuncAttributes attr{};
    cudaError_t e = cudaFuncGetAttributes(&attr, qmm_arch_probe_kernel);
    if (e != cudaSuccess) return qmm::cuda_fail(e, "kernel attributes");
    *binary_version = attr.binaryVersion;
    *ptx_version = attr.ptxVersion;
    return QMM_OK;
}

qmm_status qmm_debug_gemm_stall(int32_t withhold_block, uint64_t wait_limit_ns) {
    if (withhold_block < -1) return fail(QMM_ERR_INVALID_ARGUMENT, "withheld block %d", withhold_block);
    if (wait_limit_ns != 0 && (wait_limit_ns < 1000000ull || wait_limit_ns > qmm::kWaitLimitNs))
        return fail(QMM_ERR_INVALID_ARGUMENT, "wait limit %llu ns is outside [1 ms, 4 s]",
                    (unsigned long long)wait_limit_ns);
    qmm_status s = check_device();
    if (s != QMM_OK) return s;
    return qmm::gemm_set_stall(withhold_block, wait_limit_ns);
}

int32_t qmm_set_weights_immutable(int32_t on) {
    return qmm::g_weights_immutable.exchange(on ? 1 : 0, std::memory_order_relaxed);
}

int32_t qmm_set_sm_budget(int32_t sms) {
    const int prev = qmm::g_sm_budget.exchange(sms > 0 ? sms : 0, std::memory_order_relaxed);
    return prev;
}

qmm_status qmm_infer_layout(int64_t input, int64_t output, int64_t scales_rows,
                            int64_t scales_cols, int64_t packed_rows, int64_t packed_words,
                            int32_t *bits_out, int32_t *group_out) {
    if (!bits_out || !group_out) return fail(QMM_ERR_INVALID_ARGUMENT, "null output pointer");
    if (input <= 0 || output <= 0)
        return fail(QMM_ERR_BAD_SHAPE, "a %lld->%lld linear has no weights", (long long)input,
                    (long long)output);
    const int64_t groups = scales_cols;
    if (scales_rows != output || groups <= 0 || input % groups != 0)
        return fail(QMM_ERR_BAD_SHAPE, "scales [%lld, %lld] do not match a %lld->%lld linear",
                    (long long)scales_rows, (long long)scales_cols, (long long)input,
                    (long long)output);
    const int64_t bits = packed_words * 32 / input;
    if (packed_rows != output || packed_words * 32 != bits * input ||
        !(bits == 2 || bits == 4 || bits == 8))
        return fail(QMM_ERR_BAD_SHAPE,
                    "packed weight [%lld, %lld] is not 2-, 4- or 8-bit for %lld inputs",
                    (long long)packed_rows, (long long)packed_words, (long long)input);
    *bits_out = (int32_t)bits;
    *group_out = (int32_t)(input / groups);
    return QMM_OK;
}

qmm_status qmm_validate(const qmm_weight *w) {
    if (!w) return fail(QMM_ERR_INVALID_ARGUMENT, "null weight");
    if (!w->packed || !w->scales || !w->biases)
        return fail(QMM_ERR_INVALID_ARGUMENT, "weight has a null packed/scales/biases pointer");
    if (w->n <= 0 || w->k <= 0) return fail(QMM_ERR_BAD_SHAPE, "weight is %lldx%lld", (long long)w->n, (long long)w->k);
    if (!(w->bits == 2 || w->bits == 4 || w->bits == 8))
        return fail(QMM_ERR_BAD_SHAPE, "%d-bit codes are not 2-, 4- or 8-bit", w->bits);
    if (w->group <= 0 || w->k % w->group != 0)
        return fail(QMM_ERR_BAD_SHAPE, "group %d does not divide %lld inputs", w->group, (long long)w->k);
    if ((w->k * w->bits) % 32 != 0)
        return fail(QMM_ERR_BAD_SHAPE, "%lld %d-bit codes do not fill whole words", (long long)w->k, w->bits);
    if (!aligned16(w->packed))
        return fail(QMM_ERR_MISALIGNED, "packed weights are not 16-byte aligned");
    return QMM_OK;
}

qmm_status qmm_dequantize(const qmm_weight *w, void *dst, int32_t dtype, void *stream) {
    qmm_status s = qmm_validate(w);
    if (s != QMM_OK) return s;
    if (!dst) return fail(QMM_ERR_INVALID_ARGUMENT, "null destination");
    if (dtype != QMM_DTYPE_BF16 && dtype != QMM_DTYPE_F32)
        return fail(QMM_ERR_INVALID_ARGUMENT, "dequantize does not support dtype %d", dtype);
    if (!aligned16(dst)) return fail(QMM_ERR_MISALIGNED, "destination is not 16-byte aligned");
    if ((s = check_device()) != QMM_OK) return s;
    return qmm::launch_dequantize(*w, dst, dtype, static_cast<cudaStream_t>(stream));
}

qmm_status qmm_linear_ex(const qmm_weight *w, const uint16_t *x, int64_t m,
                         const qmm_epilogue *ep, uint16_t *y, int32_t path, void *stream) {
    qmm_status s = qmm_validate(w);
    if (s != QMM_OK) return s;
    if (m < 0) return fail(QMM_ERR_BAD_SHAPE, "negative token count %lld", (long long)m);
    if (m == 0) return QMM_OK;
    if (!x || !y) return fail(QMM_ERR_INVALID_ARGUMENT, "null x or y");
    if (path < QMM_PATH_AUTO || path > QMM_PATH_GEMM_F16)
        return fail(QMM_ERR_INVALID_ARGUMENT, "unknown path %d", path);
    qmm_epilogue e = ep ? *ep : qmm_epilogue{nullptr, nullptr, nullptr, QMM_ACT_NONE};
    if (!valid_activation(e.activation))
        return fail(QMM_ERR_INVALID_ARGUMENT, "unknown activation %d", e.activation);
    if (!aligned16(x) || !aligned16(y) || (e.residual && !aligned16(e.residual)))
        return fail(QMM_ERR_MISALIGNED, "x, y and residual must be 16-byte aligned");
    {
        const uintptr_t xb = reinterpret_cast<uintptr_t>(x), yb = reinterpret_cast<uintptr_t>(y);
        const uintptr_t xe = xb + (uintptr_t)(m * w->k * 2), ye = yb + (uintptr_t)(m * w->n * 2);
        if (xb < ye && yb < xe) return fail(QMM_ERR_INVALID_ARGUMENT, "y overlaps x");
    }
    if ((s = check_device()) != QMM_OK) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (path == QMM_PATH_AUTO)
        path = (m <= 16 && (qmm::gemv_mma_supported(*w, m) || qmm::gemv_tma_supported(*w, m) ||
                            qmm::gemv_supported(*w, m)))
                   ? QMM_PATH_GEMV
                   : QMM_PATH_GEMM;
    if (path == QMM_PATH_GEMV) {
        if (qmm::gemv_mma_supported(*w, m)) return qmm::launch_gemv_mma(*w, x, m, e, y, st);
        if (qmm::gemv_tma_supported(*w, m)) return qmm::launch_gemv_tma(*w, x, m, e, y, st);
        if (!qmm::gemv_supported(*w, m))
            return fail(QMM_ERR_UNSUPPORTED,
                        "gemv: %d-bit, group %d, k=%lld, m=%lld is outside the kernel's layouts",
                        w->bits, w->group, (long long)w->k, (long long)m);
        return qmm::launch_gemv(*w, x, m, e, y, st);
    }
    if (!qmm::gemm_supported(*w))
        return fail(QMM_ERR_UNSUPPORTED,
                    "gemm: %d-bit, group %d, k=%lld is outside the kernel's layouts (needs 4/8-bit, "
                    "k %% 64 == 0, group 32 or a multiple of 64)",
                    w->bits, w->group, (long long)w->k);
    return qmm::launch_gemm(*w, x, m, e, y, path == QMM_PATH_GEMM_PAIR, 1, nullptr, st, path == QMM_PATH_GEMM_F16);
}

int32_t qmm_gemm_splits(const qmm_weight *w, int64_t m) {
    if (!w || qmm_validate(w) != QMM_OK) return 1;
    return qmm::gemm_recommended_splits(*w, m);
}

uint64_t qmm_splitk_workspace_bytes(const qmm_weight *w, int64_t m, int32_t splits) {
    if (!w || m <= 0 || splits <= 1 || w->n <= 0) return 0;
    return (uint64_t)splits * (uint64_t)m * (uint64_t)w->n * 4u;
}

qmm_status qmm_linear_splitk(const qmm_weight *w, const uint16_t *x, int64_t m, const qmm_epilogue *ep,
                             uint16_t *y, int32_t splits, void *workspace, uint64_t workspace_bytes,
                             void *stream) {
    qmm_status s = qmm_validate(w);
    if (s != QMM_OK) return s;
    if (m < 0) return fail(QMM_ERR_BAD_SHAPE, "negative token count %lld", (long long)m);
    if (m == 0) return QMM_OK;
    if (!x || !y) return fail(QMM_ERR_INVALID_ARGUMENT, "null x or y");
    if (splits < 1 || splits > 16) return fail(QMM_ERR_INVALID_ARGUMENT, "split count %d is not in [1, 16]", splits);
    qmm_epilogue e = ep ? *ep : qmm_epilogue{nullptr, nullptr, nullptr, QMM_ACT_NONE};
    if (!valid_activation(e.activation))
        return fail(QMM_ERR_INVALID_ARGUMENT, "unknown activation %d", e.activation);
    if (!aligned16(x) || !aligned16(y) || (e.residual && !aligned16(e.residual)))
        return fail(QMM_ERR_MISALIGNED, "x, y and residual must be 16-byte aligned");
    {
        const uintptr_t xb = reinterpret_cast<uintptr_t>(x), yb = reinterpret_cast<uintptr_t>(y);
        const uintptr_t xe = xb + (uintptr_t)(m * w->k * 2), ye = yb + (uintptr_t)(m * w->n * 2);
        if (xb < ye && yb < xe) return fail(QMM_ERR_INVALID_ARGUMENT, "y overlaps x");
    }
    if (!qmm::gemm_supported(*w))
        return fail(QMM_ERR_UNSUPPORTED, "gemm: %d-bit, group %d, k=%lld is outside the kernel's layouts",
                    w->bits, w->group, (long long)w->k);
    if (splits > 1) {
        if ((w->k / 64) % splits != 0)
            return fail(QMM_ERR_INVALID_ARGUMENT, "%d splits do not divide %lld k-blocks of 64", splits,
                        (long long)(w->k / 64));
        if (w->n % 4 != 0) return fail(QMM_ERR_UNSUPPORTED, "split-k needs n %% 4 == 0 (n = %lld)", (long long)w->n);
        const uint64_t need = qmm_splitk_workspace_bytes(w, m, splits);
        if (!workspace || workspace_bytes < need)
            return fail(QMM_ERR_INVALID_ARGUMENT, "split-k workspace of %llu bytes is smaller than %llu",
                        (unsigned long long)workspace_bytes, (unsigned long long)need);
        if (!aligned16(workspace)) return fail(QMM_ERR_MISALIGNED, "split-k workspace is not 16-byte aligned");
        const uintptr_t wb = reinterpret_cast<uintptr_t>(workspace), we = wb + (uintptr_t)need;
        const uintptr_t yb = reinterpret_cast<uintptr_t>(y), ye = yb + (uintptr_t)(m * w->n * 2);
        const uintptr_t xb = reinterpret_cast<uintptr_t>(x), xe = xb + (uintptr_t)(m * w->k * 2);
        if ((wb < ye && yb < we) || (wb < xe && xb < we))
            return fail(QMM_ERR_INVALID_ARGUMENT, "split-k workspace overlaps x or y");
    }
    if ((s = check_device()) != QMM_OK) return s;
    return qmm::launch_gemm(*w, x, m, e, y, false, splits, static_cast<float *>(workspace),
                            static_cast<cudaStream_t>(stream));
}

qmm_status qmm_linear(const qmm_weight *w, const uint16_t *x, int64_t m, const qmm_epilogue *ep,
                      uint16_t *y, void *stream) {
    return qmm_linear_ex(w, x, m, ep, y, QMM_PATH_AUTO, stream);
}

qmm_status qmm_device_error(void *stream, uint32_t *code_out) {
    if (!code_out) return fail(QMM_ERR_INVALID_ARGUMENT, "null output pointer");
    qmm_status s = check_device();
    if (s != QMM_OK) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return qmm::cuda_fail(e, "stream synchronize");
    uint32_t v = 0, zero = 0;
    e = cudaMemcpyFromSymbol(&v, qmm::g_device_error, sizeof v);
    if (e != cudaSuccess) return qmm::cuda_fail(e, "read device error word");
    if (v != 0) {
        e = cudaMemcpyToSymbol(qmm::g_device_error, &zero, sizeof zero);
        if (e != cudaSuccess) return qmm::cuda_fail(e, "clear device error word");
    }
    *code_out = v;
    return v == 0 ? QMM_OK : fail(QMM_ERR_TIMEOUT, "device-side wait expired (code %u)", v);
}

}  // extern "C"
