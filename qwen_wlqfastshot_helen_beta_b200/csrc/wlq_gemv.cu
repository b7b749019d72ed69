// Decode GEMV for M = 1..16 token rows over 4-bit LUT-quantised weights, with
// outlier replacement and the DoRA epilogue fused.  Replaces
// gemv_chunk_csr_kernel + reduce_split_k_dora_kernel
// (csrc/gemv_kernel.cu:86-353) and, for 2 <= M <= 16, the wmma kernel
// (csrc/gemm_kernel.cu:32-294).
//
// The kernel is HBM-bound (0.5 B of indices per weight, +0.25 B with 128-wide
// per-group codebooks), so the design goal is the fewest instructions per
// weight:
//  * the tensor core does the multiply-accumulate: weights are the A operand
//    of mma.m16n8k16 (16 output rows x 16 k), tokens the 8-wide B operand;
//    one MMA retires 256 weights for up to 8 tokens;
//  * the codebook lookup runs in registers through byte permutes (LutPlanes),
//    no shared memory traffic per weight;
//  * the A fragment's k order is free (the same permutation is applied to x):
//    lane (g, t) owns rows g and g+8 and the 32 consecutive columns
//    [32t, 32t+32) of every 128-wide chunk, so it reads 16 contiguous bytes of
//    each of its rows per chunk with one 128-bit load;
//  * K is split over the 4 warps of a CTA and over the CTAs of a thread-block
//    cluster; partial sums meet in shared memory and, across the cluster, in
//    distributed shared memory, so no global workspace and no second launch.
// Outliers REPLACE the codebook weight (csrc/gemm_kernel.cu:204-228); here the
// replacement is applied as (w_outlier - w_codebook) * x after the MMA loop,
// the same arithmetic as csrc/gemv_kernel.cu:262-288.
#include "wlq_common.cuh"
#include "wlq_internal.h"

namespace wlq {

namespace {

constexpr int kWarps = 4;
constexpr int kRowsPerTile = 16;
constexpr int kChunk = 128;  // k columns per warp iteration

struct GemvParams {
    const uint32_t* q;
    const uint16_t* lut;
    const void* x;
    void* out;
    const int32_t* off;
    const uint16_t* ccols;
    const uint8_t* cvals;
    const uint16_t* loraB;
    const float* lorah;
    const uint16_t* gamma;
    float scale;
    int r, M, N, K, wpr, G, goff, ngroups, chunk_m, ncsr;
    int kchunks;          // ceil(K / 128)
    int chunks_per_warp;  // K split granularity
    int xvec;             // rows of x are 16-byte aligned (K % 8 == 0)
};

template <typename T>
__device__ __forceinline__ void load_planes(const uint16_t* __restrict__ lut, int64_t entry, bool valid,
                                            LutPlanes& P) {
    uint32_t e[8];
    if (valid) {
        const uint4 a = ldg_nc_v4(lut + entry * 16);
        const uint4 b = ldg_nc_v4(lut + entry * 16 + 8);
        e[0] = a.x; e[1] = a.y; e[2] = a.z; e[3] = a.w;
        e[4] = b.x; e[5] = b.y; e[6] = b.z; e[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = 0u;
    }
    if (!ActTraits<T>::kIsF16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t lo = ActTraits<T>::from_f16_bits((uint16_t)(e[i] & 0xFFFFu));
            const uint32_t hi = ActTraits<T>::from_f16_bits((uint16_t)(e[i] >> 16));
            e[i] = lo | (hi << 16);
        }
    }
    make_planes(e, P);
}

// 32 consecutive activations of one token starting at column k (zero beyond
// K or for an absent token).
template <typename T>
__device__ __forceinline__ void load_x32(const T* __restrict__ x, int tok, int M, int K, int k, int xvec,
                                         uint4 xv[4]) {
#pragma unroll
    for (int v = 0; v < 4; ++v) xv[v] = make_uint4(0u, 0u, 0u, 0u);
    if (tok >= M) return;
    const T* xr = x + (int64_t)tok * K;
    if (xvec) {  // K % 8 == 0: each 8-wide group is wholly inside or outside K
#pragma unroll
        for (int v = 0; v < 4; ++v)
            if (k + 8 * v + 8 <= K) xv[v] = ldg_nc_v4(xr + k + 8 * v);
        return;
    }
    const uint16_t* xs = reinterpret_cast<const uint16_t*>(xr);
#pragma unroll
    for (int v = 0; v < 4; ++v) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int k0 = k + 8 * v + 2 * j;
            const uint32_t lo = k0 < K ? (uint32_t)__ldg(xs + k0) : 0u;
            const uint32_t hi = k0 + 1 < K ? (uint32_t)__ldg(xs + k0 + 1) : 0u;
            w[j] = lo | (hi << 16);
        }
        xv[v] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

template <typename T, int MT, bool GROUPED>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(const GemvParams p) {
    constexpr int NT = MT / 8;  // n8 tiles of tokens
    __shared__ float red[kWarps][kRowsPerTile][MT];
    __shared__ float part[kRowsPerTile * MT];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;
    const int row0 = blockIdx.x * kRowsPerTile + g;
    const int row1 = row0 + 8;
    const bool v0 = row0 < p.N;
    const bool v1 = row1 < p.N;
    const uint32_t* q0 = p.q + (int64_t)(v0 ? row0 : 0) * p.wpr;
    const uint32_t* q1 = p.q + (int64_t)(v1 ? row1 : 0) * p.wpr;
    const T* x = reinterpret_cast<const T*>(p.x);

    const int slice = blockIdx.y * kWarps + warp;
    const int c_begin = slice * p.chunks_per_warp;
    const int c_end = min(p.kchunks, c_begin + p.chunks_per_warp);

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;

    LutPlanes P0, P1;
    int cur_grp = -1;
    if (!GROUPED) {
        load_planes<T>(p.lut, v0 ? row0 : 0, v0, P0);
        load_planes<T>(p.lut, v1 ? row1 : 0, v1, P1);
    }

    // software pipeline: the next chunk's index words are in flight while
    // the current chunk is dequantised and multiplied
    uint4 w0n = make_uint4(0u, 0u, 0u, 0u), w1n = w0n;
    auto load_words = [&](int c, uint4& a, uint4& b) {
        const int wi = c * (kChunk / 8) + 4 * t;
        const bool in = wi < p.wpr;
        a = (v0 && in) ? ldg_stream_v4(q0 + wi) : make_uint4(0u, 0u, 0u, 0u);
        b = (v1 && in) ? ldg_stream_v4(q1 + wi) : make_uint4(0u, 0u, 0u, 0u);
    };
    if (c_begin < c_end) load_words(c_begin, w0n, w1n);

    for (int c = c_begin; c < c_end; ++c) {
        const uint4 w0 = w0n, w1 = w1n;
        if (c + 1 < c_end) load_words(c + 1, w0n, w1n);
        const int kl = c * kChunk + 32 * t;  // first column of this lane
        uint4 xa[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j) load_x32<T>(x, 8 * j + g, p.M, p.K, kl, p.xvec, xa[j]);
        if (GROUPED) {
            // lanes past K multiply zero activations; clamp their group so the
            // codebook read stays inside the row
            const int grp = min((kl + p.goff) / p.G, p.ngroups - 1);
            if (grp != cur_grp) {
                cur_grp = grp;
                load_planes<T>(p.lut, (int64_t)(v0 ? row0 : 0) * p.ngroups + grp, v0, P0);
                load_planes<T>(p.lut, (int64_t)(v1 ? row1 : 0) * p.ngroups + grp, v1, P1);
            }
        }
        const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w};
        const uint32_t wb[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int ws = 0; ws < 4; ++ws) {
            uint32_t sa, ca, sb, cb;
            lut_selectors(wa[ws], sa, ca);
            lut_selectors(wb[ws], sb, cb);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t a[4];
                lut4(P0, sa, ca, a[0], a[2]);
                lut4(P1, sb, cb, a[1], a[3]);
                sa >>= 16; ca >>= 16; sb >>= 16; cb >>= 16;
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const uint32_t b0 = h ? xa[j][ws].z : xa[j][ws].x;
                    const uint32_t b1 = h ? xa[j][ws].w : xa[j][ws].y;
                    Mma16816<T>::run(acc[j], a, b0, b1);
                }
            }
        }
    }

    // outlier replacement for this warp's K range: (w_outlier - w_codebook) * x
    if (p.off != nullptr && c_begin < c_end) {
        const int kb = c_begin * kChunk;
        const int ke = min(p.K, c_end * kChunk);
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int row = rr ? row1 : row0;
            if (!(rr ? v1 : v0)) continue;
            const uint32_t* qr = rr ? q1 : q0;
            const int cc_lo = kb / p.chunk_m;
            const int cc_hi = (ke - 1) / p.chunk_m;
            for (int cc = cc_lo; cc <= cc_hi; ++cc) {
                const int64_t ob = (int64_t)row * (p.ncsr + 1) + cc;
                const int ia = __ldg(p.off + ob), ib = __ldg(p.off + ob + 1);
                for (int i = ia; i < ib; ++i) {
                    const int col = cc * p.chunk_m + (int)__ldg(p.ccols + i);
                    if (col < kb || col >= ke) continue;
                    const uint32_t sym = (__ldg(qr + (col >> 3)) >> (4 * (col & 7))) & 15u;
                    const int grp = GROUPED ? (col + p.goff) / p.G : 0;
                    const uint16_t lb = __ldg(p.lut + ((int64_t)row * p.ngroups + grp) * 16 + sym);
                    // the codebook value the MMA used (rounded to bf16 on the bf16 path)
                    const float wl = ActTraits<T>::bits_to_f32(ActTraits<T>::from_f16_bits(lb));
                    const float wo = f16_bits_to_f32(fp8_byte_to_f16_bits(__ldg(p.cvals + i)));
                    const float d = wo - wl;
#pragma unroll
                    for (int j = 0; j < NT; ++j)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int m = 8 * j + 2 * t + e;
                            if (m < p.M) acc[j][2 * rr + e] += d * ActTraits<T>::to_f32(x[(int64_t)m * p.K + col]);
                        }
                }
            }
        }
    }

    // reduce the 4 warps' partial tiles
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        red[warp][g][8 * j + 2 * t] = acc[j][0];
        red[warp][g][8 * j + 2 * t + 1] = acc[j][1];
        red[warp][g + 8][8 * j + 2 * t] = acc[j][2];
        red[warp][g + 8][8 * j + 2 * t + 1] = acc[j][3];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kRowsPerTile * MT; e += blockDim.x) {
        const int rl = e / MT, tk = e % MT;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) s += red[w][rl][tk];
        part[e] = s;
    }

    const bool clustered = gridDim.y > 1;
    if (clustered) {
        // all CTAs of the cluster publish `part`; rank 0 sums them through
        // distributed shared memory and writes the output
        cluster_sync_all();
    } else {
        __syncthreads();
    }
    const uint32_t rank = clustered ? cluster_ctarank() : 0u;
    if (rank == 0) {
        const uint32_t nranks = clustered ? cluster_nctarank() : 1u;
        const bool dora = p.r > 0;
        for (int e = threadIdx.x; e < kRowsPerTile * MT; e += blockDim.x) {
            const int rl = e % kRowsPerTile, tk = e / kRowsPerTile;  // rows fastest: coalesced stores
            const int n = blockIdx.x * kRowsPerTile + rl;
            if (n >= p.N || tk >= p.M) continue;
            const int pe = rl * MT + tk;
            float s = part[pe];
            if (clustered) {
                const uint32_t a = smem_u32(&part[pe]);
                for (uint32_t q = 1; q < nranks; ++q) s += ld_shared_cluster_f32(mapa_shared(a, q));
            }
            if (dora) {
                float l = 0.f;
                const float* h = p.lorah + (int64_t)tk * p.r;
                const uint16_t* B = p.loraB + (int64_t)n * p.r;
                for (int j = 0; j < p.r; ++j) l += __ldg(h + j) * f16_bits_to_f32(__ldg(B + j));
                s = (s + p.scale * l) * f16_bits_to_f32(__ldg(p.gamma + n));
            }
            reinterpret_cast<T*>(p.out)[(int64_t)tk * p.N + n] = ActTraits<T>::from_f32(s);
        }
    }
    if (clustered) cluster_sync_all();  // keep every CTA's `part` alive until rank 0 is done
}

template <typename T, int MT, bool GROUPED>
int launch_variant(const GemvParams& p, int row_tiles, int cs, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)row_tiles, (unsigned)cs, 1);
    cfg.blockDim = dim3(kWarps * 32, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)cs;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cs > 1 ? 1 : 0;
    return check_cuda(cudaLaunchKernelEx(&cfg, gemv_kernel<T, MT, GROUPED>, p), "gemv_kernel launch");
}

template <typename T>
int dispatch(const GemvParams& p, int row_tiles, int cs, cudaStream_t stream) {
    const bool grouped = p.G > 0;
    if (p.M <= 8) {
        return grouped ? launch_variant<T, 8, true>(p, row_tiles, cs, stream)
                       : launch_variant<T, 8, false>(p, row_tiles, cs, stream);
    }
    return grouped ? launch_variant<T, 16, true>(p, row_tiles, cs, stream)
                   : launch_variant<T, 16, false>(p, row_tiles, cs, stream);
}

}  // namespace

int launch_gemv(const LinearArgs& a, cudaStream_t stream) {
    if (a.M == 0 || a.N == 0) return WLQ_OK;
    if (a.M > 16) return fail(WLQ_ERR_INVALID_ARG, "wlq_gemv: M must be <= 16, got %d", a.M);
    if (a.group_size > 0 && (a.group_size % 32 != 0 || a.group_offset % 32 != 0))
        return fail(WLQ_ERR_UNSUPPORTED,
                    "wlq_gemv: per-group codebooks need group_size and group_offset multiples of 32 "
                    "(got %d, %d)", a.group_size, a.group_offset);
    GemvParams p;
    p.q = a.q; p.lut = a.lut; p.x = a.x; p.out = a.out;
    p.off = a.off; p.ccols = a.ccols; p.cvals = a.cvals;
    p.loraB = a.loraB; p.lorah = a.lorah; p.gamma = a.gamma; p.scale = a.scale; p.r = a.r;
    p.M = a.M; p.N = a.N; p.K = a.K; p.wpr = a.wpr; p.G = a.group_size; p.goff = a.group_offset;
    p.ngroups = a.ngroups; p.chunk_m = a.chunk_m; p.ncsr = a.ncsr;
    p.kchunks = (a.K + kChunk - 1) / kChunk;
    p.xvec = (a.K % 8 == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);

    const int row_tiles = (a.N + kRowsPerTile - 1) / kRowsPerTile;
    // Split K over a cluster until about 4 CTAs per SM are in flight, keeping
    // at least 2 chunks per warp.
    const int sms = device_sm_count();
    int cs = 1;
    while (cs < 8 && (int64_t)row_tiles * cs < 4LL * sms && p.kchunks >= 2 * kWarps * (cs + 1)) ++cs;
    p.chunks_per_warp = (p.kchunks + kWarps * cs - 1) / (kWarps * cs);
    if (a.dtype == WLQ_DTYPE_BF16) return dispatch<__nv_bfloat16>(p, row_tiles, cs, stream);
    return dispatch<__half>(p, row_tiles, cs, stream);
}

}  // namespace wlq
