// The DoRA low-rank input H = X A^T (fp32 [M, r]) for calls that do not fold
// it into the decode GEMV: the prefill GEMM and rank above what the GEMV
// folds.  Replaces the library GEMM plus cast the reference runs before every
// GEMM op, F.linear(x, lora_A).float() (vllm_wlq/linear_method.py:984).
//
// HBM-bound on X (M K 2 bytes; A is r K 2 bytes, re-read from L2 by every
// token tile).  A CTA computes 64 tokens x 64 ranks on the tensor core
// (mma.m16n8k16, tokens the A operand, ranks the B operand, both K-contiguous
// so ldmatrix reads them without transposition) over a 3-stage cp.async ring
// of 64-column k tiles, rows of 128 bytes with the 16-byte chunk index XORed
// with row % 8 (conflict-free ldmatrix).  Few token tiles (small M) split K
// across a thread-block cluster; the partial tiles meet in distributed shared
// memory and are summed in rank order, so the result does not depend on the
// split's schedule.  No workspace, one launch.  H stays in fp32: the
// reference rounds it to fp16 first.
#include "wlq_common.cuh"
#include "wlq_internal.h"

namespace wlq {

namespace {

constexpr int kHTok = 64;      // tokens per CTA: 4 warps x 16
constexpr int kHRank = 64;     // ranks per CTA; gridDim.z covers larger r
constexpr int kHK = 64;        // k columns per stage
constexpr int kHStages = 3;
constexpr int kHTile = 64 * 128;                      // bytes of one 64 x 64 tile of 16-bit values
constexpr int kHSmem = kHStages * 2 * kHTile;         // X and A tiles per stage
constexpr int kHPartStride = kHRank + 4;              // fp32 partial tile row stride (floats)
constexpr int kHMaxSplit = 16;  // above 8: a non-portable cluster size
static_assert(kHTok * kHPartStride * 4 <= kHSmem, "the partial tile reuses the ring");

struct HParams {
    const uint16_t* X;  // [M, K] act dtype
    const uint16_t* A;  // [r, K] act dtype
    float* H;           // [M, r]
    int M, K, r;
    int ktiles, ktiles_per_rank;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr) : "memory");
}

// byte offset of 16-byte chunk `ch` of row `row` in a swizzled tile
__device__ __forceinline__ uint32_t hswz(int row, int ch) { return (uint32_t)(row * 128 + (((ch ^ row) & 7) << 4)); }

template <typename T>
__global__ void __launch_bounds__(128) lora_h_kernel(const HParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int m0 = blockIdx.x * kHTok;
    const int j0 = blockIdx.z * kHRank;
    const int kt0 = blockIdx.y * p.ktiles_per_rank;
    const int kt1 = min(p.ktiles, kt0 + p.ktiles_per_rank);
    const uint32_t sb = smem_u32(smem);
    auto xs = [&](int s) { return sb + (uint32_t)(s * 2 * kHTile); };
    auto as = [&](int s) { return sb + (uint32_t)(s * 2 * kHTile + kHTile); };

    // ranks of this CTA in MMA n-tile pairs (16 ranks each): only these rows
    // of A are loaded and multiplied
    const int npairs = min(4, (p.r - j0 + 15) / 16);
    // k tile kt into stage s: 512 16-byte pieces of X (4 per thread) and the
    // 16 npairs rows of A; rows past M or r and columns past K (K % 8 == 0)
    // read as zero
    auto issue = [&](int kt, int s) {
        if (kt < kt1) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int e = threadIdx.x + 128 * i;
                const int row = e >> 3, ch = e & 7;
                const int k = kt * kHK + ch * 8;
                const bool kok = k < p.K;
                const bool xok = kok && m0 + row < p.M;
                cp_async16(xs(s) + hswz(row, ch), p.X + (xok ? (int64_t)(m0 + row) * p.K + k : 0), xok);
                if (row < 16 * npairs) {
                    const bool aok = kok && j0 + row < p.r;
                    cp_async16(as(s) + hswz(row, ch), p.A + (aok ? (int64_t)(j0 + row) * p.K + k : 0), aok);
                }
            }
        }
        cp_async_commit();
    };

    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;

#pragma unroll
    for (int j = 0; j < kHStages - 1; ++j) issue(kt0 + j, j);
    int st = 0;
    for (int kt = kt0; kt < kt1; ++kt) {
        cp_async_wait<kHStages - 2>();  // this thread's pieces of tile kt have landed
        __syncthreads();                // ... and everyone's; the stage read last iteration is free
        issue(kt + kHStages - 1, st == 0 ? kHStages - 1 : st - 1);
#pragma unroll
        for (int kk = 0; kk < kHK / 16; ++kk) {
            uint32_t a[4];
            {
                const int row = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
                ldsm_x4(xs(st) + hswz(row, 2 * kk + (lane >> 4)), a[0], a[1], a[2], a[3]);
            }
#pragma unroll
            for (int np = 0; np < 4; ++np) {  // ranks 16 np .. +15: two MMA n-tiles
                if (np >= npairs) break;
                const int row = np * 16 + (lane & 7) + 8 * (lane >> 4);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(as(st) + hswz(row, 2 * kk + ((lane >> 3) & 1)), b0, b1, b2, b3);
                Mma16816<T>::run(acc[2 * np], a, b0, b1);
                Mma16816<T>::run(acc[2 * np + 1], a, b2, b3);
            }
        }
        st = st + 1 == kHStages ? 0 : st + 1;
    }

    if (gridDim.y == 1) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int m = m0 + warp * 16 + g + 8 * (e >> 1);
                const int j = j0 + nt * 8 + 2 * t + (e & 1);
                if (m < p.M && j < p.r) p.H[(int64_t)m * p.r + j] = acc[nt][e];
            }
        return;
    }
    // K split over the cluster: partial tiles through distributed shared
    // memory, summed in rank order; rank q writes the token rows m with
    // m % nranks == q
    cp_async_wait<0>();
    __syncthreads();  // the ring is idle: it holds the partial tile now
    float* part = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e)
            part[(warp * 16 + g + 8 * (e >> 1)) * kHPartStride + nt * 8 + 2 * t + (e & 1)] = acc[nt][e];
    cluster_sync_all();
    const uint32_t rank = cluster_ctarank(), nranks = cluster_nctarank();
    for (int e = threadIdx.x; e < kHTok * kHRank; e += blockDim.x) {
        const int row = e / kHRank, col = e % kHRank;
        const int m = m0 + row, j = j0 + col;
        if ((uint32_t)row % nranks != rank || m >= p.M || j >= p.r) continue;
        const uint32_t addr = smem_u32(part + row * kHPartStride + col);
        float s = 0.f;
        for (uint32_t q = 0; q < nranks; ++q) s += ld_shared_cluster_f32(mapa_shared(addr, q));
        p.H[(int64_t)m * p.r + j] = s;
    }
    cluster_sync_all();  // keep every rank's partial tile alive until all reads are done
}

// Rows of X or A that are not 16-byte aligned (K % 8 != 0): one CTA per
// token, a warp per rank, fp32 accumulation.
template <typename T>
__global__ void __launch_bounds__(128) lora_h_rows_kernel(const HParams p) {
    const int m = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const T* x = reinterpret_cast<const T*>(p.X) + (int64_t)m * p.K;
    for (int j = warp; j < p.r; j += 4) {
        const T* a = reinterpret_cast<const T*>(p.A) + (int64_t)j * p.K;
        float s = 0.f;
        for (int k = lane; k < p.K; k += 32) s += ActTraits<T>::to_f32(x[k]) * ActTraits<T>::to_f32(a[k]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
        if (lane == 0) p.H[(int64_t)m * p.r + j] = s;
    }
}

// Returns kHRefused (the error cleared) when the device refuses a cluster of
// more than 8 CTAs; the caller retries at 8.
constexpr int kHRefused = -1;

template <typename T>
int launch_h(const HParams& p, int gx, int ks, int gz, bool vec, cudaStream_t stream) {
    if (!vec) {
        lora_h_rows_kernel<T><<<p.M, 128, 0, stream>>>(p);
        return check_cuda(cudaGetLastError(), "lora_h_rows_kernel launch");
    }
    auto kern = lora_h_kernel<T>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kHSmem);
    if (e != cudaSuccess) return check_cuda(e, "lora_h_kernel smem attribute");
    if (ks > 8) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return kHRefused;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)gx, (unsigned)ks, (unsigned)gz);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.dynamicSmemBytes = kHSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)ks;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ks > 1 ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess && ks > 8 &&
        (e == cudaErrorInvalidClusterSize || e == cudaErrorLaunchOutOfResources || e == cudaErrorInvalidValue ||
         e == cudaErrorNotSupported)) {
        cudaGetLastError();
        return kHRefused;
    }
    return check_cuda(e, "lora_h_kernel launch");
}

}  // namespace

int launch_lora_h(const void* X, const void* A, float* H, int M, int K, int r, int dtype, cudaStream_t stream) {
    if (M == 0 || r == 0) return WLQ_OK;
    if (K == 0) return check_cuda(cudaMemsetAsync(H, 0, (size_t)M * r * sizeof(float), stream), "lora_h clear");
    HParams p;
    p.X = static_cast<const uint16_t*>(X);
    p.A = static_cast<const uint16_t*>(A);
    p.H = H;
    p.M = M;
    p.K = K;
    p.r = r;
    p.ktiles = (K + kHK - 1) / kHK;
    const bool vec = K % 8 == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(A) & 15) == 0;
    const int gx = (M + kHTok - 1) / kHTok;
    const int gz = (r + kHRank - 1) / kHRank;
    // split K over a cluster (up to 16 CTAs) while the grid still fits in one
    // wave of four CTAs per SM (their shared-memory limit) -- the kernel is
    // bound by the latency of its loads, so every resident CTA counts, and a
    // second partial wave costs more than the split saves -- keeping at least
    // two k tiles per rank; no rank left empty
    const int sms = device_sm_count();
    auto plan = [&](int cap) {
        int ks = 1;
        while (ks < cap && (int64_t)gx * gz * (ks + 1) <= 4LL * sms && p.ktiles >= 2 * (ks + 1)) ++ks;
        p.ktiles_per_rank = (p.ktiles + ks - 1) / ks;
        return (p.ktiles + p.ktiles_per_rank - 1) / p.ktiles_per_rank;
    };
    auto run = [&](int ks) {
        return dtype == WLQ_DTYPE_BF16 ? launch_h<__nv_bfloat16>(p, gx, ks, gz, vec, stream)
                                       : launch_h<__half>(p, gx, ks, gz, vec, stream);
    };
    int rc = run(plan(kHMaxSplit));
    if (rc == kHRefused) rc = run(plan(8));
    return rc;
}

}  // namespace wlq
