// Host-side plumbing shared by the translation units of libwlq_b200.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/wlq_b200.h"

namespace wlq {

// Records `msg` as this thread's last error and returns `code`.
int fail(int code, const char* fmt, ...);
// Maps a CUDA error to WLQ_ERR_CUDA with its name, or returns WLQ_OK.
int check_cuda(cudaError_t e, const char* what);

// Arguments of one quantized-linear call, already validated.
struct LinearArgs {
    const uint32_t* q;       // [N * wpr]
    const uint16_t* lut;     // fp16 bits, [N, ngroups, 16]
    const void* x;           // [M, K] act dtype
    void* out;               // [M, N] act dtype
    const int32_t* off;      // [N, ncsr + 1] or null
    const void* ccols;       // [nnz] uint16 columns, or uint32 records when prepacked; or null
    const void* cvals;       // [nnz] e5m2 bytes, or float32 corrections when prepacked; or null
    const uint16_t* loraB;   // fp16 [N, r] or null
    const float* lorah;      // fp32 [M, r] or null
    const uint16_t* loraA = nullptr;  // act dtype [r, K]: the GEMV computes h = A x (lorah null)
    const uint16_t* gamma;   // fp16 [N] or null
    float scale;
    int r;                   // 0 when the DoRA term is off
    int M, N, K;
    int wpr;
    int group_size;          // 0 = one codebook per row
    int group_offset;
    int ngroups;             // codebooks per row
    int chunk_m;             // outlier chunk width (512 for 4-bit)
    int ncsr;                // outlier chunks per row
    int dtype;               // WLQ_DTYPE_*
    bool lut_prepacked;      // WLQ_LUT_PREPACKED codebooks
    // stream-K workspace of the tensor-core GEMM (wlq_gemm_streamk): flags
    // then partial tiles; null = data-parallel schedule only
    void* ws = nullptr;
    size_t ws_bytes = 0;
    // fused tensor-parallel all-reduce (wlq_gemv_allreduce); tp_world = 1: off
    int tp_world = 1, tp_rank = 0, tp_nmax = 0;
    void* tp_bufs[8] = {};   // every rank's communication buffer (this process's mappings)
};

// Layout of a tensor-parallel communication buffer (one per rank, shared
// through CUDA IPC): error word, per-tile call counters (local use), then
// [2][world][16][max_N] 8-byte slots, each an fp32 value and the epoch of the
// call that wrote it.
struct TpLayout {
    size_t err, counters, data, total;
    int stride;  // 8-byte words per (parity, source rank, token) row of the data region
};
constexpr size_t tp_round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
// The data region holds, per parity, source rank and token, eight 8-byte words
// per 16-row tile (two 16-bit values and a 32-bit epoch each), written in
// 16-byte pairs: the stride is even and holds every tile's eight words.
constexpr TpLayout tp_layout(int world, int max_N) {
    const size_t tiles = (size_t)(max_N + 15) / 16;
    TpLayout l{};
    l.err = 0;
    l.counters = 128;
    l.data = tp_round_up(l.counters + 4 * tiles, 256);
    const size_t words = 8 * tiles > (size_t)max_N ? 8 * tiles : (size_t)max_N;
    l.stride = (int)tp_round_up(words, 2);
    l.total = tp_round_up(l.data + 2ull * world * 16 * (size_t)l.stride * 8, 256);
    return l;
}


int launch_gemv(const LinearArgs& a, cudaStream_t stream);
int launch_gemm(const LinearArgs& a, cudaStream_t stream);
// Workspace bytes of the stream-K schedule on the current device: flags plus
// one partial tile of the largest CTA shape per SM.
size_t gemm_workspace_bytes();
// The stream-K GEMM on the library's static scratch (wlq_gemm_streamk_noalloc).
int launch_gemm_noalloc(const LinearArgs& a, cudaStream_t stream);
int launch_lora_h(const void* X, const void* A, float* H, int M, int K, int r, int dtype, cudaStream_t stream);
int launch_prepack_outliers(const uint32_t* q, const uint16_t* lut, const int32_t* off, const uint16_t* ccols,
                            const uint8_t* cvals, int N, int K, int wpr, int group_size, int goff, int ngroups,
                            int chunk_m, int ncsr, int dtype, uint32_t* recs, float* delta, cudaStream_t stream);
int launch_prepack_lut(const uint16_t* in, uint32_t* out, int64_t n, int dtype, cudaStream_t stream);
int launch_dequant(const uint32_t* q, const uint16_t* lut, uint16_t* W, const int32_t* off,
                   const uint16_t* ccols, const uint8_t* cvals, int N, int K, int bits, int wpr,
                   int group_size, int group_offset, int ngroups, int chunk_m, int ncsr,
                   cudaStream_t stream);

// Reads (and optionally clears) the device error word of `device`.
int read_device_error(int device, unsigned int* flags, int clear);

// 2-D tensor map (TMA descriptor) of a row-major [outer, inner] array with
// rows of row_bytes, box box_inner x box_outer elements; rejected shapes give
// WLQ_ERR_CUDA.  Loads past the array's edges read zeros.
int encode_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz, const char* what);

// Multiprocessor count of the current device (cached per device).
int device_sm_count();

// Whether M tokens of an [N, K] layer run on the GEMV-class kernel (M <= 16;
// 17..32 when the prepacked layout and 16-byte rows allow it and the
// tensor-core GEMM would not fill the device) rather than the GEMM.
bool gemv_preferred(int M, int N, int K, bool prepacked, const void* x);

}  // namespace wlq
