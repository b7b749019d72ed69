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

// ---------------------------------------------------------------------------
// Codebook prepacking (WLQ_LUT_PREPACKED): 16 fp16 entries -> entries in the
// MMA type (fp16 unchanged, bf16 rounded to nearest even) split into byte
// planes {lo[4], hi[4]}, the layout the GEMV/GEMM lookups permute from.
// ---------------------------------------------------------------------------
namespace wlq {

template <typename T>
__global__ void prepack_lut_kernel(const uint16_t* __restrict__ in, uint32_t* __restrict__ out, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint4 a = ldg_nc_v4(in + i * 16), b = ldg_nc_v4(in + i * 16 + 8);
        uint32_t e[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        if (!ActTraits<T>::kIsF16) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&e[k]));
                const __nv_bfloat162 v = __float22bfloat162_rn(f);
                e[k] = *reinterpret_cast<const uint32_t*>(&v);
            }
        }
        LutPlanes P;
        make_planes(e, P);
        uint4* dst = reinterpret_cast<uint4*>(out + i * 8);
        dst[0] = make_uint4(P.lo[0], P.lo[1], P.lo[2], P.lo[3]);
        dst[1] = make_uint4(P.hi[0], P.hi[1], P.hi[2], P.hi[3]);
    }
}

int launch_prepack_lut(const uint16_t* in, uint32_t* out, int64_t n, int dtype, cudaStream_t stream) {
    const int threads = 256;
    int64_t blocks = (n + threads - 1) / threads;
    const int64_t cap = (int64_t)device_sm_count() * 8;
    if (blocks > cap) blocks = cap;
    if (dtype == WLQ_DTYPE_BF16)
        prepack_lut_kernel<__nv_bfloat16><<<(unsigned)blocks, threads, 0, stream>>>(in, out, n);
    else
        prepack_lut_kernel<__half><<<(unsigned)blocks, threads, 0, stream>>>(in, out, n);
    return check_cuda(cudaGetLastError(), "prepack_lut_kernel launch");
}

}  // namespace wlq

// ---------------------------------------------------------------------------
// Outlier prepacking (WLQ_LUT_PREPACKED): chunk-CSR entries -> global column
// (uint16) and the float32 correction w_outlier - codebook value as the MMA
// sees it (codebook entry rounded to the MMA type), in the same order, so the
// forward kernels add d * x without re-reading indices or codebooks.
// ---------------------------------------------------------------------------
namespace wlq {

template <typename T>
__global__ void prepack_outliers_kernel(const uint32_t* __restrict__ q, const uint16_t* __restrict__ lut,
                                        const int32_t* __restrict__ off, const uint16_t* __restrict__ ccols,
                                        const uint8_t* __restrict__ cvals, int N, int K, int wpr, int log2G,
                                        bool grouped, int goff, int ngroups, int chunk_m, int ncsr,
                                        uint32_t* __restrict__ recs, float* __restrict__ delta) {
    for (int row = blockIdx.x * blockDim.x + threadIdx.x; row < N; row += gridDim.x * blockDim.x) {
        const int32_t* ro = off + (int64_t)row * (ncsr + 1);
        for (int cc = 0; cc < ncsr; ++cc) {
            for (int i = ro[cc]; i < ro[cc + 1]; ++i) {
                const int col = cc * chunk_m + ccols[i];
                float d = 0.f;
                uint32_t vbits = 0u;
                if (col < K) {
                    const uint32_t sym = (q[(int64_t)row * wpr + (col >> 3)] >> (4 * (col & 7))) & 15u;
                    const int grp = grouped ? (col + goff) >> log2G : 0;
                    const uint16_t lb = lut[((int64_t)row * ngroups + grp) * 16 + sym];
                    const float wl = ActTraits<T>::bits_to_f32(ActTraits<T>::from_f16_bits(lb));
                    const uint16_t ob = fp8_byte_to_f16_bits(cvals[i]);
                    d = f16_bits_to_f32(ob) - wl;
                    vbits = ActTraits<T>::from_f16_bits(ob);  // exact: e5m2 fits both types
                }
                recs[i] = (col < K ? (uint32_t)col : 0xFFFFu) | (vbits << 16);  // 0xFFFF: dropped (past K)
                delta[i] = d;
            }
        }
        // order the row by column (the builders of the reference layout emit
        // sorted chunks, so this is one pass; entries stay inside their chunk's
        // index range because chunks partition the columns)
        for (int i = ro[0] + 1; i < ro[ncsr]; ++i) {
            const uint32_t c = recs[i];
            if ((recs[i - 1] & 0xFFFFu) <= (c & 0xFFFFu)) continue;
            const float d = delta[i];
            int k = i - 1;
            while (k >= ro[0] && (recs[k] & 0xFFFFu) > (c & 0xFFFFu)) {
                recs[k + 1] = recs[k];
                delta[k + 1] = delta[k];
                --k;
            }
            recs[k + 1] = c;
            delta[k + 1] = d;
        }
    }
}

int launch_prepack_outliers(const uint32_t* q, const uint16_t* lut, const int32_t* off, const uint16_t* ccols,
                            const uint8_t* cvals, int N, int K, int wpr, int group_size, int goff, int ngroups,
                            int chunk_m, int ncsr, int dtype, uint32_t* recs, float* delta, cudaStream_t stream) {
    int log2G = 0;
    if (group_size > 0) {
        while ((1 << log2G) < group_size) ++log2G;
        if ((1 << log2G) != group_size)
            return fail(WLQ_ERR_UNSUPPORTED, "wlq_prepack_outliers: group_size must be a power of two");
    }
    const int threads = 128;
    const int blocks = (N + threads - 1) / threads;
    if (dtype == WLQ_DTYPE_BF16)
        prepack_outliers_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(
            q, lut, off, ccols, cvals, N, K, wpr, log2G, group_size > 0, goff, ngroups, chunk_m, ncsr, recs, delta);
    else
        prepack_outliers_kernel<__half><<<blocks, threads, 0, stream>>>(
            q, lut, off, ccols, cvals, N, K, wpr, log2G, group_size > 0, goff, ngroups, chunk_m, ncsr, recs, delta);
    return check_cuda(cudaGetLastError(), "prepack_outliers_kernel launch");
}

}  // namespace wlq
