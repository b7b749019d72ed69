// Dense dequantisation W[N,K] = codebook[q] with outliers replaced; the
// bit-exact counterpart of dequant_patch_metalog_kernel
// (csrc/gemm_kernel.cu:322-445).  HBM-bound: 0.5 B of indices read and 2 B of
// fp16 written per weight for 4-bit.  One thread owns one index word (8
// columns for 4-bit), so the codebook gather and the outlier overwrite of
// those columns happen in registers before a single 16-byte store; no
// ordering between threads is needed.
#include "wlq_common.cuh"
#include "wlq_internal.h"

namespace wlq {

template <int BITS>
__global__ void __launch_bounds__(256) dequant_kernel(const uint32_t* __restrict__ q,
                                                      const uint16_t* __restrict__ lut,
                                                      uint16_t* __restrict__ W,
                                                      const int32_t* __restrict__ off,
                                                      const uint16_t* __restrict__ ccols,
                                                      const uint8_t* __restrict__ cvals, int N, int K,
                                                      int wpr, int G, int goff, int ngroups, int chunk_m,
                                                      int ncsr, int words_used, int vec_store) {
    constexpr int SPW = BITS == 3 ? 10 : 32 / BITS;
    constexpr int KCB = 1 << BITS;
    constexpr uint32_t MASK = (1u << BITS) - 1u;
    const int64_t total = (int64_t)N * words_used;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(idx / words_used);
        const int w = (int)(idx - (int64_t)row * words_used);
        const uint32_t word = __ldg(q + (int64_t)row * wpr + w);
        const int col0 = w * SPW;
        uint16_t v[SPW];
        const uint16_t* lrow = lut + (int64_t)row * ngroups * KCB;
#pragma unroll
        for (int s = 0; s < SPW; ++s) {
            const int col = col0 + s;
            const uint32_t sym = (word >> (BITS * s)) & MASK;
            const int g = G > 0 ? (col + goff) / G : 0;
            v[s] = col < K ? __ldg(lrow + g * KCB + sym) : (uint16_t)0;
        }
        if (off != nullptr) {
            // A word never straddles an outlier chunk: chunk_m is a multiple of
            // the symbols per word (512 = 64 words of 8, 640 = 64 words of 10).
            const int c = col0 / chunk_m;
            const int64_t ob = (int64_t)row * (ncsr + 1) + c;
            const int a = __ldg(off + ob), b = __ldg(off + ob + 1);
            const int lc0 = col0 - c * chunk_m;
            for (int i = a; i < b; ++i) {
                const int lc = (int)__ldg(ccols + i) - lc0;
                if (lc >= 0 && lc < SPW && col0 + lc < K) {
                    const uint16_t ov = fp8_byte_to_f16_bits(__ldg(cvals + i));
#pragma unroll
                    for (int s = 0; s < SPW; ++s)
                        if (s == lc) v[s] = ov;
                }
            }
        }
        uint16_t* dst = W + (int64_t)row * K + col0;
        if (BITS == 4 && vec_store && col0 + 8 <= K) {
            uint4 pk;
            pk.x = (uint32_t)v[0] | ((uint32_t)v[1] << 16);
            pk.y = (uint32_t)v[2] | ((uint32_t)v[3] << 16);
            pk.z = (uint32_t)v[4] | ((uint32_t)v[5] << 16);
            pk.w = (uint32_t)v[6] | ((uint32_t)v[7] << 16);
            *reinterpret_cast<uint4*>(dst) = pk;
        } else {
#pragma unroll
            for (int s = 0; s < SPW; ++s)
                if (col0 + s < K) dst[s] = v[s];
        }
    }
}

int launch_dequant(const uint32_t* q, const uint16_t* lut, uint16_t* W, const int32_t* off,
                   const uint16_t* ccols, const uint8_t* cvals, int N, int K, int bits, int wpr,
                   int group_size, int group_offset, int ngroups, int chunk_m, int ncsr,
                   cudaStream_t stream) {
    if (N == 0 || K == 0) return WLQ_OK;
    const int spw = symbols_per_word(bits);
    const int words_used = (K + spw - 1) / spw;
    const int64_t total = (int64_t)N * words_used;
    const int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    const int64_t cap = (int64_t)device_sm_count() * 16;
    if (blocks > cap) blocks = cap;
    const int vec = (K % 8 == 0) && ((reinterpret_cast<uintptr_t>(W) & 15) == 0);
#define WLQ_DQ(B)                                                                                  \
    dequant_kernel<B><<<(unsigned)blocks, threads, 0, stream>>>(q, lut, W, off, ccols, cvals, N, K, \
                                                                 wpr, group_size, group_offset,    \
                                                                 ngroups, chunk_m, ncsr, words_used, vec)
    switch (bits) {
        case 1: WLQ_DQ(1); break;
        case 2: WLQ_DQ(2); break;
        case 3: WLQ_DQ(3); break;
        case 4: WLQ_DQ(4); break;
        default: return fail(WLQ_ERR_UNSUPPORTED, "wlq_dequant: bits must be 1..4, got %d", bits);
    }
#undef WLQ_DQ
    return check_cuda(cudaGetLastError(), "dequant_kernel launch");
}

}  // namespace wlq
