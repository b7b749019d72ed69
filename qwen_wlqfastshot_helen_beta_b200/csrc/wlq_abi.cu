// extern "C" entry points of libwlq_b200.so: argument validation, error
// reporting and dispatch to the sm_100a kernels.  Mirrors the checks and the
// optional-argument handling of csrc/vllm_binding.cpp:253-453 (NULL = absent,
// chunk_m from bits) and adds the dtype / alignment / shape checks that the
// reference leaves to the caller.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "wlq_common.cuh"
#include "wlq_internal.h"

namespace wlq {

static thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return WLQ_OK;
    return fail(WLQ_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

namespace {
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];
int g_cc_major[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

int current_device(int* dev) {
    const cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return check_cuda(e, "cudaGetDevice");
    if (*dev < 0 || *dev >= kMaxDevices) return fail(WLQ_ERR_DEVICE, "device index %d out of range", *dev);
    std::call_once(g_dev_once[*dev], [d = *dev]() {
        cudaDeviceGetAttribute(&g_sm_count[d], cudaDevAttrMultiProcessorCount, d);
        cudaDeviceGetAttribute(&g_cc_major[d], cudaDevAttrComputeCapabilityMajor, d);
    });
    return WLQ_OK;
}

int require_sm100() {
    int dev = 0;
    int rc = current_device(&dev);
    if (rc) return rc;
    if (g_cc_major[dev] != 10)
        return fail(WLQ_ERR_DEVICE, "device %d has compute capability %d.x; this build runs sm_100a only", dev,
                    g_cc_major[dev]);
    return WLQ_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Shared validation of the quantized-linear arguments.
// lorah (the low-rank input h = A x, fp32 [M, r]) or loraA (A itself, [r, K]
// in act_dtype, for the GEMV to compute h) carries the DoRA input; at most one
// of them is given.
int build_args(const char* fn, const void* x, const int32_t* q, const void* lut, void* out,
               const int32_t* off, const void* ccols, const void* cvals, const void* loraB,
               const float* lorah, const void* loraA, const void* gamma, float scale, int r, int M, int N, int K,
               int bits, int wpr, int G, int goff, int lut_format, int dtype, LinearArgs& a) {
    if (M < 0 || N < 0 || K < 0) return fail(WLQ_ERR_INVALID_ARG, "%s: negative size (M=%d N=%d K=%d)", fn, M, N, K);
    if (bits != 4)
        return fail(WLQ_ERR_UNSUPPORTED, "%s: only 4-bit indices are supported by the fused kernels (bits=%d)", fn, bits);
    if (dtype != WLQ_DTYPE_F16 && dtype != WLQ_DTYPE_BF16)
        return fail(WLQ_ERR_UNSUPPORTED, "%s: act_dtype must be WLQ_DTYPE_F16 or WLQ_DTYPE_BF16 (got %d)", fn, dtype);
    if (lut_format != WLQ_LUT_F16 && lut_format != WLQ_LUT_PREPACKED)
        return fail(WLQ_ERR_INVALID_ARG, "%s: lut_format must be WLQ_LUT_F16 or WLQ_LUT_PREPACKED (got %d)", fn,
                    lut_format);
    if (M > 0 && N > 0 && K > 0 && (!x || !q || !lut || !out))
        return fail(WLQ_ERR_INVALID_ARG, "%s: x, q_packed, lut_c and out are required", fn);
    const int64_t need_wpr = words_per_row(K, bits);
    if (wpr != need_wpr)
        return fail(WLQ_ERR_INVALID_ARG, "%s: words_per_row=%d but K=%d needs %lld (row-aligned layout)", fn, wpr, K,
                    (long long)need_wpr);
    if (G < 0 || goff < 0 || (G > 0 && goff >= G))
        return fail(WLQ_ERR_INVALID_ARG, "%s: bad codebook grouping (group_size=%d, group_offset=%d)", fn, G, goff);
    if (!aligned(q, 16) || !aligned(lut, 16))
        return fail(WLQ_ERR_ALIGNMENT, "%s: q_packed and lut_c must be 16-byte aligned", fn);
    if (!aligned(x, 2) || !aligned(out, 2)) return fail(WLQ_ERR_ALIGNMENT, "%s: x/out must be 2-byte aligned", fn);
    const bool has_outl = off && ccols && cvals;
    if (has_outl && lut_format == WLQ_LUT_PREPACKED && K > 65535)
        return fail(WLQ_ERR_UNSUPPORTED, "%s: prepacked outliers hold uint16 columns; K=%d is too large", fn, K);
    if (lorah && loraA) return fail(WLQ_ERR_INVALID_ARG, "%s: give lora_h or lora_A, not both", fn);
    const bool dora = loraB && (lorah || loraA) && gamma && r > 0;
    a.q = reinterpret_cast<const uint32_t*>(q);
    a.lut = reinterpret_cast<const uint16_t*>(lut);
    a.x = x;
    a.out = out;
    a.off = has_outl ? off : nullptr;
    a.ccols = has_outl ? ccols : nullptr;
    a.cvals = has_outl ? cvals : nullptr;
    a.loraB = dora ? reinterpret_cast<const uint16_t*>(loraB) : nullptr;
    a.lorah = dora ? lorah : nullptr;
    a.loraA = dora ? reinterpret_cast<const uint16_t*>(loraA) : nullptr;
    a.gamma = dora ? reinterpret_cast<const uint16_t*>(gamma) : nullptr;
    a.scale = scale;
    a.r = dora ? r : 0;
    a.M = M;
    a.N = N;
    a.K = K;
    a.wpr = wpr;
    a.group_size = G;
    a.group_offset = goff;
    a.ngroups = G > 0 ? (K + goff + G - 1) / G : 1;
    a.chunk_m = chunk_m_for_bits(bits);
    a.ncsr = (K + a.chunk_m - 1) / a.chunk_m;
    a.dtype = dtype;
    a.lut_prepacked = lut_format == WLQ_LUT_PREPACKED;
    return WLQ_OK;
}
}  // namespace

bool gemv_preferred(int M, int N, int K, bool prepacked, const void* x) {
    if (M <= 16) return true;
    // 17..32 tokens: the GEMV (weights streamed once, one launch) unless the
    // tensor-core GEMM's 128-row tiles fill the device
    const bool gemv_ok = M <= 32 && prepacked && K % 8 == 0 && aligned(x, 16);
    return gemv_ok && (N + 127) / 128 < device_sm_count();
}

int device_sm_count() {
    int dev = 0;
    if (current_device(&dev) != WLQ_OK) return 148;
    return g_sm_count[dev] > 0 ? g_sm_count[dev] : 148;
}

}  // namespace wlq

using namespace wlq;

extern "C" {

const char* wlq_last_error(void) { return g_last_error; }

int wlq_abi_version(void) { return WLQ_ABI_VERSION; }

int wlq_gemv(const int32_t* q_packed, const void* lut_c, const void* x, void* out, const int32_t* chunk_offsets,
             const void* chunk_cols, const void* chunk_vals, const void* lora_B, const float* lora_h,
             const void* dora_gamma, float lora_scale, int r, int M, int N, int K, int bits, int words_per_row,
             int lut_group_size, int lut_group_offset, int lut_format, int act_dtype, wlq_stream_t stream) {
    g_last_error[0] = '\0';
    LinearArgs a;
    int rc = build_args("wlq_gemv", x, q_packed, lut_c, out, chunk_offsets, chunk_cols, chunk_vals, lora_B, lora_h,
                        nullptr, dora_gamma, lora_scale, r, M, N, K, bits, words_per_row, lut_group_size, lut_group_offset,
                        lut_format, act_dtype, a);
    if (rc) return rc;
    if (M > 16) return fail(WLQ_ERR_INVALID_ARG, "wlq_gemv: M must be 1..16 (got %d); use wlq_gemm", M);
    if (M == 0 || N == 0) return WLQ_OK;
    if ((rc = require_sm100())) return rc;
    return launch_gemv(a, reinterpret_cast<cudaStream_t>(stream));
}

int wlq_gemv_lora_a(const int32_t* q_packed, const void* lut_c, const void* x, void* out,
                    const int32_t* chunk_offsets, const void* chunk_cols, const void* chunk_vals, const void* lora_B,
                    const void* lora_A, const void* dora_gamma, float lora_scale, int r, int M, int N, int K, int bits,
                    int words_per_row, int lut_group_size, int lut_group_offset, int lut_format, int act_dtype,
                    wlq_stream_t stream) {
    g_last_error[0] = '\0';
    LinearArgs a;
    int rc = build_args("wlq_gemv_lora_a", x, q_packed, lut_c, out, chunk_offsets, chunk_cols, chunk_vals, lora_B,
                        nullptr, lora_A, dora_gamma, lora_scale, r, M, N, K, bits, words_per_row, lut_group_size,
                        lut_group_offset, lut_format, act_dtype, a);
    if (rc) return rc;
    if (M > 32) return fail(WLQ_ERR_INVALID_ARG, "wlq_gemv_lora_a: M must be 1..32 (got %d)", M);
    if (M == 0 || N == 0) return WLQ_OK;
    if ((rc = require_sm100())) return rc;
    return launch_gemv(a, reinterpret_cast<cudaStream_t>(stream));
}

int wlq_gemm(const void* X, const int32_t* q_packed, const void* lut_c, void* out, const int32_t* chunk_offsets,
             const void* chunk_cols, const void* chunk_vals, const float* lora_H, const void* lora_B,
             const void* dora_gamma, float lora_scale, int r, int M, int N, int K, int bits, int words_per_row,
             int lut_group_size, int lut_group_offset, int lut_format, int act_dtype, wlq_stream_t stream) {
    g_last_error[0] = '\0';
    LinearArgs a;
    int rc = build_args("wlq_gemm", X, q_packed, lut_c, out, chunk_offsets, chunk_cols, chunk_vals, lora_B, lora_H,
                        nullptr, dora_gamma, lora_scale, r, M, N, K, bits, words_per_row, lut_group_size, lut_group_offset,
                        lut_format, act_dtype, a);
    if (rc) return rc;
    if (M == 0 || N == 0) return WLQ_OK;
    if ((rc = require_sm100())) return rc;
    if (gemv_preferred(M, N, K, a.lut_prepacked, X)) return launch_gemv(a, reinterpret_cast<cudaStream_t>(stream));
    return launch_gemm(a, reinterpret_cast<cudaStream_t>(stream));
}

size_t wlq_gemm_workspace_bytes(int device) {
    g_last_error[0] = '\0';
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) return 0;
    if (device != prev && cudaSetDevice(device) != cudaSuccess) return 0;
    const size_t b = gemm_workspace_bytes();
    if (device != prev) cudaSetDevice(prev);
    return b;
}

int wlq_gemm_streamk(const void* X, const int32_t* q_packed, const void* lut_c, void* out,
                     const int32_t* chunk_offsets, const void* chunk_cols, const void* chunk_vals,
                     const float* lora_H, const void* lora_B, const void* dora_gamma, float lora_scale, int r, int M,
                     int N, int K, int bits, int words_per_row, int lut_group_size, int lut_group_offset,
                     int lut_format, int act_dtype, void* workspace, size_t workspace_bytes, wlq_stream_t stream) {
    g_last_error[0] = '\0';
    LinearArgs a;
    int rc = build_args("wlq_gemm_streamk", X, q_packed, lut_c, out, chunk_offsets, chunk_cols, chunk_vals, lora_B,
                        lora_H, nullptr, dora_gamma, lora_scale, r, M, N, K, bits, words_per_row, lut_group_size,
                        lut_group_offset, lut_format, act_dtype, a);
    if (rc) return rc;
    if (workspace && !aligned(workspace, 256))
        return fail(WLQ_ERR_ALIGNMENT, "wlq_gemm_streamk: the workspace must be 256-byte aligned");
    if (M == 0 || N == 0) return WLQ_OK;
    if ((rc = require_sm100())) return rc;
    if (gemv_preferred(M, N, K, a.lut_prepacked, X)) return launch_gemv(a, reinterpret_cast<cudaStream_t>(stream));
    a.ws = workspace;
    a.ws_bytes = workspace ? workspace_bytes : 0;
    return launch_gemm(a, reinterpret_cast<cudaStream_t>(stream));
}

int wlq_gemm_streamk_noalloc(const void* X, const int32_t* q_packed, const void* lut_c, void* out,
                             const int32_t* chunk_offsets, const void* chunk_cols, const void* chunk_vals,
                             const float* lora_H, const void* lora_B, const void* dora_gamma, float lora_scale,
                             int r, int M, int N, int K, int bits, int words_per_row, int lut_group_size,
                             int lut_group_offset, int lut_format, int act_dtype, wlq_stream_t stream) {
    g_last_error[0] = '\0';
    LinearArgs a;
    int rc = build_args("wlq_gemm_streamk_noalloc", X, q_packed, lut_c, out, chunk_offsets, chunk_cols, chunk_vals,
                        lora_B, lora_H, nullptr, dora_gamma, lora_scale, r, M, N, K, bits, words_per_row,
                        lut_group_size, lut_group_offset, lut_format, act_dtype, a);
    if (rc) return rc;
    if (M == 0 || N == 0) return WLQ_OK;
    if ((rc = require_sm100())) return rc;
    // up to 16 tokens the GEMV runs: it needs no scratch
    if (gemv_preferred(M, N, K, a.lut_prepacked, X)) return launch_gemv(a, reinterpret_cast<cudaStream_t>(stream));
    return launch_gemm_noalloc(a, reinterpret_cast<cudaStream_t>(stream));
}

int wlq_lora_h(const void* X, const void* lora_A, float* H, int M, int K, int r, int act_dtype,
               wlq_stream_t stream) {
    g_last_error[0] = '\0';
    if (M < 0 || K < 0 || r < 0) return fail(WLQ_ERR_INVALID_ARG, "wlq_lora_h: negative size (M=%d K=%d r=%d)", M, K, r);
    if (act_dtype != WLQ_DTYPE_F16 && act_dtype != WLQ_DTYPE_BF16)
        return fail(WLQ_ERR_UNSUPPORTED, "wlq_lora_h: act_dtype must be WLQ_DTYPE_F16 or WLQ_DTYPE_BF16 (got %d)",
                    act_dtype);
    if (M == 0 || r == 0) return WLQ_OK;
    if (!X || !lora_A || !H) return fail(WLQ_ERR_INVALID_ARG, "wlq_lora_h: X, lora_A and H are required");
    if (!aligned(X, 2) || !aligned(lora_A, 2) || !aligned(H, 4))
        return fail(WLQ_ERR_ALIGNMENT, "wlq_lora_h: misaligned pointer");
    int rc = require_sm100();
    if (rc) return rc;
    return launch_lora_h(X, lora_A, H, M, K, r, act_dtype, reinterpret_cast<cudaStream_t>(stream));
}

int wlq_dequant(const int32_t* q_packed, const void* lut_c, void* W_out, const int32_t* chunk_offsets,
                const uint16_t* chunk_cols, const uint8_t* chunk_vals, int N, int K, int bits, int words_per_row,
                int lut_group_size, int lut_group_offset, wlq_stream_t stream) {
    g_last_error[0] = '\0';
    if (N < 0 || K < 0) return fail(WLQ_ERR_INVALID_ARG, "wlq_dequant: negative size");
    if (bits < 1 || bits > 4) return fail(WLQ_ERR_UNSUPPORTED, "wlq_dequant: bits must be 1..4 (got %d)", bits);
    if (N == 0 || K == 0) return WLQ_OK;
    if (!q_packed || !lut_c || !W_out) return fail(WLQ_ERR_INVALID_ARG, "wlq_dequant: q_packed, lut_c, W_out required");
    if (words_per_row != wlq::words_per_row(K, bits))
        return fail(WLQ_ERR_INVALID_ARG, "wlq_dequant: words_per_row=%d does not match K=%d, bits=%d", words_per_row, K,
                    bits);
    if (lut_group_size < 0 || lut_group_offset < 0 || (lut_group_size > 0 && lut_group_offset >= lut_group_size))
        return fail(WLQ_ERR_INVALID_ARG, "wlq_dequant: bad codebook grouping");
    if (!aligned(q_packed, 4) || !aligned(lut_c, 2) || !aligned(W_out, 2))
        return fail(WLQ_ERR_ALIGNMENT, "wlq_dequant: misaligned pointer");
    int rc = require_sm100();
    if (rc) return rc;
    const bool has_outl = chunk_offsets && chunk_cols && chunk_vals;
    const int chunk_m = chunk_m_for_bits(bits);
    const int ngroups = lut_group_size > 0 ? (K + lut_group_offset + lut_group_size - 1) / lut_group_size : 1;
    return launch_dequant(reinterpret_cast<const uint32_t*>(q_packed), reinterpret_cast<const uint16_t*>(lut_c),
                          reinterpret_cast<uint16_t*>(W_out), has_outl ? chunk_offsets : nullptr,
                          has_outl ? chunk_cols : nullptr, has_outl ? chunk_vals : nullptr, N, K, bits, words_per_row,
                          lut_group_size, lut_group_offset, ngroups, chunk_m, (K + chunk_m - 1) / chunk_m,
                          reinterpret_cast<cudaStream_t>(stream));
}

int wlq_prepack_lut(const void* lut_c, void* lut_out, int64_t n_codebooks, int act_dtype, wlq_stream_t stream) {
    g_last_error[0] = '\0';
    if (n_codebooks < 0) return fail(WLQ_ERR_INVALID_ARG, "wlq_prepack_lut: negative count");
    if (n_codebooks == 0) return WLQ_OK;
    if (!lut_c || !lut_out) return fail(WLQ_ERR_INVALID_ARG, "wlq_prepack_lut: null pointer");
    if (act_dtype != WLQ_DTYPE_F16 && act_dtype != WLQ_DTYPE_BF16)
        return fail(WLQ_ERR_UNSUPPORTED, "wlq_prepack_lut: act_dtype %d", act_dtype);
    if (!aligned(lut_c, 16) || !aligned(lut_out, 16))
        return fail(WLQ_ERR_ALIGNMENT, "wlq_prepack_lut: pointers must be 16-byte aligned");
    const char* a = static_cast<const char*>(lut_c);
    const char* b = static_cast<const char*>(lut_out);
    if (a < b + n_codebooks * 32 && b < a + n_codebooks * 32)
        return fail(WLQ_ERR_INVALID_ARG, "wlq_prepack_lut: input and output overlap");
    int rc = require_sm100();
    if (rc) return rc;
    return launch_prepack_lut(reinterpret_cast<const uint16_t*>(lut_c), reinterpret_cast<uint32_t*>(lut_out),
                              n_codebooks, act_dtype, reinterpret_cast<cudaStream_t>(stream));
}

int wlq_prepack_outliers(const int32_t* q_packed, const void* lut_c, const int32_t* chunk_offsets,
                         const uint16_t* chunk_cols, const uint8_t* chunk_vals, int64_t nnz, int N, int K, int bits,
                         int words_per_row, int lut_group_size, int lut_group_offset, int act_dtype,
                         uint32_t* cols_out, float* delta_out, wlq_stream_t stream) {
    g_last_error[0] = '\0';
    if (nnz < 0 || N < 0 || K < 0) return fail(WLQ_ERR_INVALID_ARG, "wlq_prepack_outliers: negative size");
    if (bits != 4) return fail(WLQ_ERR_UNSUPPORTED, "wlq_prepack_outliers: 4-bit indices only (bits=%d)", bits);
    if (K > 65535) return fail(WLQ_ERR_UNSUPPORTED, "wlq_prepack_outliers: K=%d exceeds uint16 columns", K);
    if (act_dtype != WLQ_DTYPE_F16 && act_dtype != WLQ_DTYPE_BF16)
        return fail(WLQ_ERR_UNSUPPORTED, "wlq_prepack_outliers: act_dtype %d", act_dtype);
    if (words_per_row != wlq::words_per_row(K, bits))
        return fail(WLQ_ERR_INVALID_ARG, "wlq_prepack_outliers: words_per_row does not match K");
    if (lut_group_size < 0 || lut_group_offset < 0 || (lut_group_size > 0 && lut_group_offset >= lut_group_size))
        return fail(WLQ_ERR_INVALID_ARG, "wlq_prepack_outliers: bad codebook grouping");
    if (nnz == 0 || N == 0) return WLQ_OK;
    if (!q_packed || !lut_c || !chunk_offsets || !chunk_cols || !chunk_vals || !cols_out || !delta_out)
        return fail(WLQ_ERR_INVALID_ARG, "wlq_prepack_outliers: null pointer");
    int rc = require_sm100();
    if (rc) return rc;
    const int chunk_m = chunk_m_for_bits(bits);
    const int ngroups = lut_group_size > 0 ? (K + lut_group_offset + lut_group_size - 1) / lut_group_size : 1;
    return launch_prepack_outliers(reinterpret_cast<const uint32_t*>(q_packed), reinterpret_cast<const uint16_t*>(lut_c),
                                   chunk_offsets, chunk_cols, chunk_vals, N, K, words_per_row, lut_group_size,
                                   lut_group_offset, ngroups, chunk_m, (K + chunk_m - 1) / chunk_m, act_dtype,
                                   cols_out, delta_out, reinterpret_cast<cudaStream_t>(stream));
}

int wlq_init_workspaces(int64_t max_N, int64_t max_K, int device) {
    g_last_error[0] = '\0';
    if (max_N < 0 || max_K < 0 || device < 0) return fail(WLQ_ERR_INVALID_ARG, "wlq_init_workspaces: bad arguments");
    return WLQ_OK;
}

size_t wlq_tp_buffer_bytes(int world, int max_N) {
    if (world < 1 || world > 8 || max_N < 0) return 0;
    return tp_layout(world, max_N).total;
}

int wlq_tp_buffer_alloc(size_t bytes, void** ptr_out, unsigned char handle_out[64]) {
    g_last_error[0] = '\0';
    if (!ptr_out || !handle_out || bytes == 0) return fail(WLQ_ERR_INVALID_ARG, "wlq_tp_buffer_alloc: bad arguments");
    int rc = require_sm100();
    if (rc) return rc;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return check_cuda(e, "wlq_tp_buffer_alloc: cudaMalloc");
    if ((e = cudaMemset(p, 0, bytes)) != cudaSuccess || (e = cudaDeviceSynchronize()) != cudaSuccess) {
        cudaFree(p);
        return check_cuda(e, "wlq_tp_buffer_alloc: clear");
    }
    cudaIpcMemHandle_t h;
    static_assert(sizeof(h) == 64, "IPC handle size");
    if ((e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
        cudaFree(p);
        return check_cuda(e, "wlq_tp_buffer_alloc: cudaIpcGetMemHandle");
    }
    memcpy(handle_out, &h, 64);
    *ptr_out = p;
    return WLQ_OK;
}

int wlq_tp_buffer_open(const unsigned char handle[64], void** ptr_out) {
    g_last_error[0] = '\0';
    if (!handle || !ptr_out) return fail(WLQ_ERR_INVALID_ARG, "wlq_tp_buffer_open: bad arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, 64);
    return check_cuda(cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess), "wlq_tp_buffer_open");
}

int wlq_tp_buffer_close(void* peer_ptr) {
    g_last_error[0] = '\0';
    return check_cuda(cudaIpcCloseMemHandle(peer_ptr), "wlq_tp_buffer_close");
}

int wlq_tp_buffer_free(void* ptr) {
    g_last_error[0] = '\0';
    return check_cuda(cudaFree(ptr), "wlq_tp_buffer_free");
}

int wlq_tp_error(void* local_buf, unsigned int* flags_out, int clear) {
    g_last_error[0] = '\0';
    if (!local_buf || !flags_out) return fail(WLQ_ERR_INVALID_ARG, "wlq_tp_error: bad arguments");
    unsigned int v = 0;
    cudaError_t e = cudaMemcpy(&v, local_buf, sizeof(v), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(local_buf, 0, sizeof(v));
    if (e != cudaSuccess) return check_cuda(e, "wlq_tp_error");
    *flags_out = v;
    return WLQ_OK;
}

int wlq_gemv_allreduce(const int32_t* q_packed, const void* lut_c, const void* x, void* out,
                       const int32_t* chunk_offsets, const void* chunk_cols, const void* chunk_vals,
                       const void* lora_B, const float* lora_h, const void* lora_A, const void* dora_gamma,
                       float lora_scale, int r, int M, int N, int K, int bits, int words_per_row, int lut_group_size,
                       int lut_group_offset, int lut_format, int act_dtype, void* const* tp_bufs, int tp_rank,
                       int tp_world, int max_N, wlq_stream_t stream) {
    g_last_error[0] = '\0';
    LinearArgs a;
    int rc = build_args("wlq_gemv_allreduce", x, q_packed, lut_c, out, chunk_offsets, chunk_cols, chunk_vals, lora_B,
                        lora_h, lora_A, dora_gamma, lora_scale, r, M, N, K, bits, words_per_row, lut_group_size,
                        lut_group_offset, lut_format, act_dtype, a);
    if (rc) return rc;
    if (M > 16) return fail(WLQ_ERR_INVALID_ARG, "wlq_gemv_allreduce: M must be 1..16 (got %d)", M);
    if (tp_world < 2 || tp_world > 8 || tp_rank < 0 || tp_rank >= tp_world || !tp_bufs)
        return fail(WLQ_ERR_INVALID_ARG, "wlq_gemv_allreduce: bad rank %d of %d", tp_rank, tp_world);
    if (N > max_N) return fail(WLQ_ERR_CAPACITY, "wlq_gemv_allreduce: N=%d exceeds the buffers' max_N=%d", N, max_N);
    for (int q = 0; q < tp_world; ++q)
        if (!tp_bufs[q] || !aligned(tp_bufs[q], 256))
            return fail(WLQ_ERR_INVALID_ARG, "wlq_gemv_allreduce: buffer of rank %d missing or misaligned", q);
    if (M == 0 || N == 0) return WLQ_OK;
    if ((rc = require_sm100())) return rc;
    a.tp_world = tp_world;
    a.tp_rank = tp_rank;
    a.tp_nmax = max_N;
    for (int q = 0; q < tp_world; ++q) a.tp_bufs[q] = tp_bufs[q];
    return launch_gemv(a, reinterpret_cast<cudaStream_t>(stream));
}

int wlq_device_error(int device, unsigned int* flags_out, int clear) {
    g_last_error[0] = '\0';
    if (!flags_out || device < 0) return fail(WLQ_ERR_INVALID_ARG, "wlq_device_error: bad arguments");
    return read_device_error(device, flags_out, clear);
}

}  // extern "C"
