// Prefill GEMM for M > 16 token rows over 4-bit LUT-quantised weights, with
// outlier replacement and the DoRA epilogue fused, on the sm_100a tensor
// cores (tcgen05, accumulators in TMEM).  Replaces the reference's
// dequant_patch_metalog + at::mm_out + fused_dora_epilogue sequence
// (csrc/gemm_kernel.cu:296-526, csrc/vllm_binding.cpp:355-393), which
// materialises the whole dequantised weight in HBM before a cuBLAS GEMM.
//
// One CTA computes a (NACC x 128) x 128 tile of out = gamma * (X W^T + s H B^T):
//   warp 0      TMA producer of the activation tiles (64 k x 128 tokens,
//               128-byte swizzle);
//   warp 1      allocates TMEM and issues tcgen05.mma from one thread;
//   warp 2      TMA producer of the 128 x 64 index tiles and their codebooks
//               (a deep ring of its own, so dequantisation never waits on it);
//   warps 3..18 four threads per weight row: LUT lookups in registers (byte
//               permutes, as in the decode GEMV) written as the K-major
//               128-byte-swizzled bf16/f16 tile the MMA reads, outlier values
//               patched in, then the epilogue (TMEM -> gamma -> global).
// The DoRA low-rank term runs as extra K steps: the dequant warps write
// s * H (tokens x r) and B (rows x r) into a stage's operand buffers, so it
// accumulates into the same TMEM tile with no separate epilogue pass.
// Every mbarrier wait is bounded; a wait that runs out sets the device error
// word (wlq_device_error) and the CTA winds down, releasing its TMEM.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "wlq_common.cuh"
#include "wlq_internal.h"
#include "wlq_sm100.cuh"

namespace wlq {

namespace {

constexpr int kBK = 64;           // k per stage: one 128-byte swizzle row of 16-bit values
constexpr int kTileM = 128;       // tokens per accumulator (MMA M)
constexpr int kDeq = 512;         // dequant / epilogue threads (warps 3 ..)
constexpr int kDeqWarps = kDeq / 32;

// Work split for a tile of BN weight rows (128 or 256) over the kDeq dequant
// threads: kTpr threads per row, kColsT columns of a step each (at most 32:
// one codebook group), epilogue column chunks per warp and accumulator.
template <int BN>
struct Tile {
    static constexpr int kTpr = kDeq / BN;
    static constexpr int kColsT = kBK / kTpr;
    static constexpr int kWordsT = kColsT / 8;
    static constexpr int kCcPerWarp = BN / 32 / (kDeqWarps / 4);
    static_assert(kColsT <= 32 && kWordsT >= 1, "one codebook group per thread and step");
};
constexpr int kDeqBase = 96;      // warps 0..2: activation producer, MMA, index producer
constexpr int kThreads = kDeqBase + kDeq;
constexpr int kWin = 8;           // reference layout: outliers per (row, chunk) held in registers
constexpr int kSmemLimit = 227 * 1024;

struct GemmParams {
    CUtensorMap tm_x;    // X [M, K], box 64 x 128, 128-byte swizzle
    CUtensorMap tm_q;    // indices [N, wpr] u32, box 8 x 128
    CUtensorMap tm_lut;  // per-group codebooks [N, ngroups * 8] u32, box 8*NPG x 128
    const uint16_t* lut; // per-row codebooks (ungrouped)
    void* out;
    const int32_t* off;
    const void* ccols;   // uint16 chunk-local columns, or uint32 records column | value << 16 (prepacked)
    const void* cvals;   // e5m2 bytes (reference layout); unused when prepacked
    const uint16_t* loraB;
    const float* lorah;
    const uint16_t* gamma;
    float scale;
    int r, M, N, K, ngroups, goff, log2G, chunk_m, ncsr;
    int ksteps;          // ceil(K / 64)
    int lsteps;          // ceil(r / 64) low-rank steps after the K steps
    uint32_t mul16, mul31;
    int vec_out;         // rows of out are 16-byte aligned
    // schedule: tile t = n tile * mtiles + token tile; the first dp_tiles run
    // whole (CTA b takes b, b + G, ...); the k steps of the rest are split
    // evenly over the first sk_ctas CTAs (stream-K), whose partial tiles meet
    // through the workspace
    int mtiles, dp_tiles, sk_ctas;
    int sk_iters;        // (tiles - dp_tiles) * steps
    float* ws_part;      // [sk_ctas][NACC * 128][BN] fp32 partial tiles (stream-K only)
    uint32_t* ws_flag;   // [sk_ctas] partial-ready flags, zero between launches
};

// Shared-memory plan of one CTA: three rings, each slot 1024-byte aligned
// (the swizzle atom): activation tiles (SX slots, filled by TMA, freed by the
// MMAs), weight tiles (SW slots, written by the dequant threads, freed by the
// MMAs) and index/codebook tiles (SI slots, filled by TMA, freed by the
// dequant threads).  The last ring is small per slot and deep, so the
// dequant inputs arrive long before they are needed; then the mbarriers, the
// TMEM address and gamma.
template <int NACC, int NPG, int BN>
struct Plan {
    static constexpr int kX = kTileM * kBK * 2;          // one accumulator's activation tile
    static constexpr int kXStage = NACC * kX;
    static constexpr int kWStage = BN * kBK * 2;
    static constexpr int kIdx = BN * 32;                   // BN rows x 8 index words
    static constexpr int kTma = kIdx + BN * 32 * NPG;      // + codebooks: the bytes TMA lands
    static constexpr int kIStage = kTma;
    // activation tiles take ~2500 cycles to land (L2), so their ring is the
    // deepest that fits; the index ring is consumed at the dequant pace and
    // gets what is left (at least 2 slots)
    static constexpr int kSX = BN == 256 ? 3 : (NACC == 2 ? 4 : 6);
    static constexpr int kSW = BN == 256 ? (NPG == 2 ? 2 : 3) : ((NACC == 2 && NPG == 2) ? 3 : 4);
    static constexpr int kBudget = kSmemLimit - 2048;
    static constexpr int kSIfit = (kBudget - kSX * kXStage - kSW * kWStage) / kIStage;
    static constexpr int kSI = kSIfit > 8 ? 8 : kSIfit;
    static constexpr int kXOff = 0;
    static constexpr int kWOff = kSX * kXStage;
    static constexpr int kIOff = kWOff + kSW * kWStage;
    static constexpr int kBarOff = kIOff + kSI * kIStage;
    static constexpr int kGammaOff = kBarOff + 512;
    static constexpr int kAlloc = kGammaOff + 4 * BN + 1024;  // barriers + gamma, alignment slack
    static_assert(kSI >= 2, "shared memory too small for the index ring");
    static_assert(kTma % 1024 == 0, "slots stay 1024-byte aligned");
};

__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ void sts16(uint32_t a, uint16_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"(v) : "memory");
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (ActTraits<T>::kIsF16) {
        return (uint32_t)__half_as_ushort(__float2half_rn(a)) | ((uint32_t)__half_as_ushort(__float2half_rn(b)) << 16);
    } else {
        return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a)) |
               ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b)) << 16);
    }
}

// Byte address of element k (0..63) of a 128-byte row at `row_addr` (row
// index `row`) in a K-major tile with the 128-byte swizzle: the 16-byte chunk
// index is XORed with row % 8 (the layout TMA writes and tcgen05 reads).
__device__ __forceinline__ uint32_t sw128_elem(uint32_t row_addr, int row, int k) {
    return row_addr + ((((k >> 3) ^ row) & 7) << 4) + ((k & 7) << 1);
}

// Work of one CTA: data-parallel tiles first (b, b + G, ... < dp_tiles, whole
// K), then its contiguous share of the stream-K iterations (k steps of the
// remaining tiles, in tile order; CTAs b < sk_ctas only).  A unit is one tile
// and a step range [s0, s1) of it; every warp role walks the same sequence.
struct Units {
    int dp_next, it, it1;  // next data-parallel tile; this CTA's stream-K iteration range
    __device__ __forceinline__ void init(const GemmParams& p) {
        const int b = (int)blockIdx.x;
        dp_next = b;
        it = b < p.sk_ctas ? (int)((long long)b * p.sk_iters / p.sk_ctas) : 0;
        it1 = b < p.sk_ctas ? (int)((long long)(b + 1) * p.sk_iters / p.sk_ctas) : 0;
    }
    __device__ __forceinline__ bool next(const GemmParams& p, int& tile, int& s0, int& s1) {
        const int steps = p.ksteps + p.lsteps;
        if (dp_next < p.dp_tiles) {
            tile = dp_next;
            s0 = 0;
            s1 = steps;
            dp_next += (int)gridDim.x;
            return true;
        }
        if (it < it1) {
            const int t = it / steps;
            tile = p.dp_tiles + t;
            s0 = it - t * steps;
            s1 = min(steps, s0 + (it1 - it));
            it += s1 - s0;
            return true;
        }
        return false;
    }
};

// The stream-K CTA that owns iteration i (sk_ctas CTAs over sk_iters).
__device__ __forceinline__ int sk_owner(const GemmParams& p, int i) {
    return (int)(((long long)(i + 1) * p.sk_ctas + p.sk_iters - 1) / p.sk_iters) - 1;
}

__device__ __forceinline__ void bar_sync_deq() {  // the kDeq dequant / epilogue threads
    asm volatile("bar.sync 1, %0;" ::"n"(kDeq) : "memory");
}
__device__ __forceinline__ void st_release_u32(uint32_t* a, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* a) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}
__device__ __forceinline__ float4 ldcg_f4(const float* a) {  // L2 only: another SM wrote it
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(a));
    return v;
}

template <typename T, int NACC, int NPG, bool PREPACKED, int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ GemmParams p) {
    using P = Plan<NACC, NPG, BN>;
    constexpr int kTpr = Tile<BN>::kTpr, kColsT = Tile<BN>::kColsT, kWordsT = Tile<BN>::kWordsT;
    constexpr bool GROUPED = NPG > 0;
    constexpr int SX = P::kSX, SW = P::kSW, SI = P::kSI;
    constexpr int kPartFloats = NACC * kTileM * BN;  // one partial tile in the stream-K workspace
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sb = (raw + 1023u) & ~1023u;
    uint8_t* sgen = smem_raw + (sb - raw);
    const uint32_t bars = sb + P::kBarOff;
    auto xfull = [&](int s) { return bars + 8u * s; };                    // activations landed / slot handed over
    auto xempty = [&](int s) { return bars + 8u * (SX + s); };            // MMAs done with the slot
    auto wfull = [&](int s) { return bars + 8u * (2 * SX + s); };         // weight tile written
    auto wempty = [&](int s) { return bars + 8u * (2 * SX + SW + s); };   // MMAs done with the slot
    auto ifull = [&](int s) { return bars + 8u * (2 * SX + 2 * SW + s); };           // index tile landed
    auto iempty = [&](int s) { return bars + 8u * (2 * SX + 2 * SW + SI + s); };     // dequant done with it
    const uint32_t acc_full = bars + 8u * (2 * SX + 2 * SW + 2 * SI);  // a unit's MMAs are done
    const uint32_t acc_empty = acc_full + 8u;                           // its epilogue has read TMEM
    const uint32_t tmem_slot = acc_full + 16u;
    float* gam = reinterpret_cast<float*>(sgen + P::kGammaOff);  // gamma of the current unit's tile rows
    auto xslot = [&](int s) { return sb + P::kXOff + s * P::kXStage; };
    auto wslot = [&](int s) { return sb + P::kWOff + s * P::kWStage; };
    auto islot = [&](int s) { return sb + P::kIOff + s * P::kIStage; };

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // token tiles vary fastest in the tile order, so the CTAs resident at
    // one time read several activation tiles instead of all hitting one
    const int mtiles = p.mtiles;
    const int steps = p.ksteps + p.lsteps;
    const bool dora = p.r > 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SX; ++s) {
            mbar_init(xfull(s), 1);
            mbar_init(xempty(s), 1);
        }
        for (int s = 0; s < SW; ++s) {
            mbar_init(wfull(s), kDeqWarps);
            mbar_init(wempty(s), 1);
        }
        for (int s = 0; s < SI; ++s) {
            mbar_init(ifull(s), 1);
            mbar_init(iempty(s), kDeqWarps);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, kDeqWarps);
        mbar_fence_init();
        tma_prefetch_desc(&p.tm_x);
        tma_prefetch_desc(&p.tm_q);
        if (GROUPED) tma_prefetch_desc(&p.tm_lut);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, NACC * BN);
        tmem_relinquish();
    }
    tc_fence_before_sync();
    __syncthreads();
    tc_fence_after_sync();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sgen + P::kBarOff + (tmem_slot - bars));

    auto group_at = [&](int col) { return min((col + p.goff) >> p.log2G, p.ngroups - 1); };
    Units U;
    U.init(p);
    int tile, s0, s1;

    if (warp == 0) {
        // ------------------------------------------------ activation producer
        if (lane == 0) {
            int g = 0;  // steps issued over all units
            bool ok = true;
            while (ok && U.next(p, tile, s0, s1)) {
                const int m0 = (tile % mtiles) * (NACC * kTileM);
                for (int j = s0; j < s1; ++j) {
                    const int s = g % SX, u = g / SX;
                    if (u > 0 && !mbar_wait(xempty(s), (u - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    ++g;
                    if (j < p.ksteps) {
                        mbar_arrive_expect_tx(xfull(s), (uint32_t)P::kXStage);
#pragma unroll
                        for (int a = 0; a < NACC; ++a)
                            tma_load_2d(xslot(s) + a * P::kX, &p.tm_x, xfull(s), j * kBK, m0 + a * kTileM);
                    } else {
                        mbar_arrive(xfull(s));  // low-rank step: the dequant threads write the slot
                    }
                }
            }
            // no copy may still be landing when the CTA exits (matters only
            // after a wait ran out): the last use of each slot has completed
            for (int j = g > SX ? g - SX : 0; j < g; ++j) mbar_wait(xfull(j % SX), (j / SX) & 1);
        }
    } else if (warp == 2) {
        // ------------------------------------------- index/codebook producer
        if (lane == 0) {
            int g = 0;  // index tiles issued over all units
            bool ok = true;
            while (ok && U.next(p, tile, s0, s1)) {
                const int n0 = (tile / mtiles) * BN;
                for (int j = s0; j < min(s1, p.ksteps); ++j) {
                    const int s = g % SI, u = g / SI;
                    if (u > 0 && !mbar_wait(iempty(s), (u - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    ++g;
                    mbar_arrive_expect_tx(ifull(s), (uint32_t)P::kTma);
                    tma_load_2d(islot(s), &p.tm_q, ifull(s), j * (kBK / 8), n0);
                    if constexpr (GROUPED)
                        tma_load_2d(islot(s) + P::kIdx, &p.tm_lut, ifull(s), group_at(j * kBK) * 8, n0);
                }
            }
            for (int j = g > SI ? g - SI : 0; j < g; ++j) mbar_wait(ifull(j % SI), (j / SI) & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issue
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(ActTraits<T>::kIsF16 ? 0u : 1u, kTileM, BN);
            int gx = 0, gw = 0, u = 0;
            bool ok = true;
            while (ok && U.next(p, tile, s0, s1)) {
                // the previous unit's epilogue has read the accumulators
                if (u > 0 && !mbar_wait(acc_empty, (u - 1) & 1)) break;
                tc_fence_after_sync();
                for (int j = s0; j < s1; ++j, ++gx, ++gw) {
                    const int sx = gx % SX, sw = gw % SW;
                    if (!mbar_wait(xfull(sx), (gx / SX) & 1) || !mbar_wait(wfull(sw), (gw / SW) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after_sync();
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint64_t bdesc = umma_desc_sw128(wslot(sw) + kk * 32);
#pragma unroll
                        for (int a = 0; a < NACC; ++a)
                            umma_f16(tmem + a * BN, umma_desc_sw128(xslot(sx) + a * P::kX + kk * 32), bdesc, idesc,
                                     (j != s0 || kk != 0) ? 1u : 0u);
                    }
                    umma_commit(xempty(sx));
                    umma_commit(wempty(sw));
                }
                umma_commit(acc_full);  // completes once every MMA of the unit has
                ++u;
            }
        }
    } else {
        // ------------------------------------------------------- dequant rows
        // kTpr threads per weight row, the row's threads adjacent lanes of
        // one warp: thread (nl, part) owns columns [kColsT part, +kColsT) of
        // every step (kWordsT index words, one codebook: groups are >= 32
        // columns and 32-aligned)
        const int td = threadIdx.x - kDeqBase;
        const int nl = td / kTpr;
        const int part = td % kTpr;
        const int col0 = kColsT * part;
        const uint32_t m16 = p.mul16, m31 = p.mul31;
        const uint32_t* recs = reinterpret_cast<const uint32_t*>(p.ccols);
        const int ksteps_per_chunk = p.chunk_m / kBK;
        bool ok = true;
        int gx = 0, gw = 0, gi = 0, u = 0;

        while (U.next(p, tile, s0, s1)) {
            const int n0 = (tile / mtiles) * BN;
            const int m0 = (tile % mtiles) * (NACC * kTileM);
            const int n = n0 + nl;
            const bool nv = n < p.N;

            LutPlanes PR;  // per-row codebook (ungrouped)
            if (!GROUPED) load_planes<T, PREPACKED>(p.lut, n, nv, PR);
            // the tile's gamma (read by every epilogue thread after the
            // barrier before the epilogue; the previous unit's readers are
            // past the barrier that ends its epilogue)
            if (td < BN) gam[td] = (dora && n0 + td < p.N) ? f16_bits_to_f32(__ldg(p.gamma + n0 + td)) : 1.f;

            // outliers of this row from column k0 = 64 s0 on.  Prepacked
            // layout: the row's records are sorted by column; each of the
            // row's threads keeps the next three in registers (x0 next), so a
            // step without an outlier costs one compare, and a consumed record
            // is replaced by one loaded two consumptions earlier.  Reference
            // layout: each thread keeps the first kWin entries of the current
            // chunk in registers, the next chunk's prefetched one chunk ahead.
            const bool outl = p.off != nullptr && nv && s0 < p.ksteps;
            const int32_t* orow = p.off + (int64_t)(nv ? n : 0) * (p.ncsr + 1);
            int ob = 0, oe = 0, one = 0, row_end = 0;
            uint32_t wc[kWin], wv[kWin], nc[kWin], nvv[kWin];
            auto ld_rec = [&](int i) { return i < row_end ? __ldg(recs + i) : 0xFFFFu; };  // 0xFFFF: none (K <= 65535)
            uint32_t x0 = 0xFFFFu, x1 = 0xFFFFu, x2 = 0xFFFFu;
            int xi = 0;  // index of x0
            auto load_win = [&](int base, uint32_t (&c)[kWin], uint32_t (&v)[kWin]) {
#pragma unroll
                for (int e = 0; e < kWin; ++e) {
                    const int i = base + e;
                    const bool in = i < row_end;
                    c[e] = in ? (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(p.ccols) + i) : 0xFFFFu;
                    v[e] = in ? (uint32_t)__ldg(reinterpret_cast<const uint8_t*>(p.cvals) + i) : 0u;
                }
            };
            int chunk = (s0 * kBK) / p.chunk_m;  // reference layout: chunk of the current step
            int chunk_left = ksteps_per_chunk - (s0 % ksteps_per_chunk);
            if (outl) {
                row_end = __ldg(orow + p.ncsr);
                ob = __ldg(orow + chunk);
                if constexpr (PREPACKED) {
                    xi = ob;  // the chunk's entries are in its index range, sorted: skip those left of k0
                    x0 = ld_rec(xi);
                    while ((x0 & 0xFFFFu) < (uint32_t)(s0 * kBK)) x0 = ld_rec(++xi);
                    x1 = ld_rec(xi + 1);
                    x2 = ld_rec(xi + 2);
                } else {
                    oe = __ldg(orow + chunk + 1);
                    one = chunk + 2 <= p.ncsr ? __ldg(orow + chunk + 2) : oe;
                    load_win(ob, wc, wv);
                    load_win(oe, nc, nvv);
                }
            }

            // replaces the weight at column kl (0..63) of this step: v is the
            // value in the MMA type (prepacked) or the e5m2 byte
            auto patch = [&](uint32_t wrow, int kl, uint32_t v) {
                const uint32_t a = sw128_elem(wrow, nl, kl);
                if (PREPACKED)
                    sts16(a, (uint16_t)v);
                else
                    sts16(a, ActTraits<T>::from_f16_bits(fp8_byte_to_f16_bits((uint8_t)v)));
            };

            // after a wait ran out (ok false) the warps skip all work but keep
            // walking the units, so every named barrier below is reached by
            // all dequant warps
            for (int j = s0; j < s1; ++j, ++gx, ++gw) {
                if (!ok) continue;
                const int sw = gw % SW, uw = gw / SW;
                if (uw > 0 && !mbar_wait(wempty(sw), (uw - 1) & 1)) { ok = false; continue; }
                const uint32_t wrow = wslot(sw) + nl * 128;
                if (j < p.ksteps) {
                    const int si = gi % SI;
                    if (!mbar_wait(ifull(si), (gi / SI) & 1)) { ok = false; continue; }
                    const int k0 = j * kBK;
                    uint32_t words[kWordsT];
                    if constexpr (kWordsT == 4) {
                        const uint4 w4 = lds128(islot(si) + nl * 32 + col0 / 2);
                        words[0] = w4.x; words[1] = w4.y; words[2] = w4.z; words[3] = w4.w;
                    } else {
                        const uint2 w2 = lds64(islot(si) + nl * 32 + col0 / 2);
                        words[0] = w2.x; words[1] = w2.y;
                    }
                    LutPlanes PL;
                    if constexpr (GROUPED) {
                        const int slot = NPG == 2 ? group_at(k0 + col0) - group_at(k0) : 0;
                        planes_from_smem<T, PREPACKED>(islot(si) + P::kIdx + nl * (32 * NPG) + 32 * slot, PL);
                    } else {
                        PL = PR;
                    }
#pragma unroll
                    for (int wi = 0; wi < kWordsT; ++wi) {
                        const uint32_t w = words[wi];
                        const uint32_t sa = w & 0x77777777u;
                        const uint32_t ca = lop_and_or(mulhi(w, m31), 0x44444444u, 0x32103210u);
                        uint32_t o0, o1, o2, o3;
                        lookup4(PL, sa, ca, o0, o1);
                        lookup4(PL, mulhi(sa, m16), mulhi(ca, m16), o2, o3);
                        sts128(wrow + ((((col0 / 8 + wi) ^ nl) & 7) << 4), o0, o1, o2, o3);
                    }
                    if constexpr (PREPACKED) {
                        const uint32_t kend = (uint32_t)min(k0 + kBK, p.K);
                        while ((x0 & 0xFFFFu) < kend) {  // sorted: nothing below k0 is left
                            const int kl = (int)(x0 & 0xFFFFu) - k0;
                            if ((uint32_t)(kl - col0) < (uint32_t)kColsT) patch(wrow, kl, x0 >> 16);
                            ++xi;
                            x0 = x1;
                            x1 = x2;
                            x2 = ld_rec(xi + 2);
                        }
                    } else if (outl) {
                        if (chunk_left == 0) {  // entering the next chunk: rotate the windows
                            ++chunk;
                            chunk_left = ksteps_per_chunk;
                            ob = oe;
                            oe = one;
                            one = chunk + 2 <= p.ncsr ? __ldg(orow + chunk + 2) : oe;
#pragma unroll
                            for (int e = 0; e < kWin; ++e) {
                                wc[e] = nc[e];
                                wv[e] = nvv[e];
                            }
                            load_win(oe, nc, nvv);
                        }
                        --chunk_left;
                        // this thread's columns in the chunk-local numbering
                        const int cbase = k0 - chunk * p.chunk_m + col0;
                        uint32_t hits = 0;
#pragma unroll
                        for (int e = 0; e < kWin; ++e)
                            hits |= (ob + e < oe && (uint32_t)((int)wc[e] - cbase) < (uint32_t)kColsT) ? 1u << e : 0u;
                        while (hits) {
                            const int e = __ffs(hits) - 1;
                            hits &= hits - 1;
                            uint32_t cw = wc[0], vw = wv[0];
#pragma unroll
                            for (int q = 1; q < kWin; ++q)
                                if (q == e) {
                                    cw = wc[q];
                                    vw = wv[q];
                                }
                            patch(wrow, (int)cw - cbase + col0, vw);
                        }
                        for (int i = ob + kWin; i < oe; ++i) {  // more than kWin outliers in this chunk
                            const int kl = (int)__ldg(reinterpret_cast<const uint16_t*>(p.ccols) + i) - cbase;
                            if ((uint32_t)kl < (uint32_t)kColsT)
                                patch(wrow, kl + col0, (uint32_t)__ldg(reinterpret_cast<const uint8_t*>(p.cvals) + i));
                        }
                    }
                    fence_proxy_async_smem();  // generic-proxy tile writes -> tensor core
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(iempty(si));
                        mbar_arrive(wfull(sw));
                    }
                    ++gi;
                } else {
                    // low-rank step: X <- s * H (tokens x r), W <- B (rows x r), zero
                    // past r; the dequant threads share the 16-byte chunks of both
                    const int sx = gx % SX;
                    if (!mbar_wait(xfull(sx), (gx / SX) & 1)) { ok = false; continue; }  // slot handed over
                    const int j0 = (j - p.ksteps) * kBK;
#pragma unroll 1
                    for (int c = td; c < NACC * kTileM * 8; c += kDeq) {
                        const int rx = c >> 3, ch = c & 7, a = rx / kTileM, rr = rx % kTileM;
                        const int m = m0 + rx;
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const int jj = j0 + 8 * ch + e;
                            f[e] = (m < p.M && jj < p.r) ? p.scale * __ldg(p.lorah + (int64_t)m * p.r + jj) : 0.f;
                        }
                        sts128(xslot(sx) + a * P::kX + rr * 128 + (((ch ^ rr) & 7) << 4), pack2<T>(f[0], f[1]),
                               pack2<T>(f[2], f[3]), pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
                    }
#pragma unroll 1
                    for (int c = td; c < BN * 8; c += kDeq) {
                        const int rw = c >> 3, ch = c & 7;
                        const int nw = n0 + rw;
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const int jj = j0 + 8 * ch + e;
                            f[e] = (nw < p.N && jj < p.r) ? f16_bits_to_f32(__ldg(p.loraB + (int64_t)nw * p.r + jj)) : 0.f;
                        }
                        sts128(wslot(sw) + rw * 128 + (((ch ^ rw) & 7) << 4), pack2<T>(f[0], f[1]), pack2<T>(f[2], f[3]),
                               pack2<T>(f[4], f[5]), pack2<T>(f[6], f[7]));
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(wfull(sw));
                }
            }

            // ------------------------------------------------------ epilogue
            // warp w reads TMEM lanes 32 (w % 4) .. +31; the kTpr warps of a
            // lane quarter split the tile's columns.  A unit covering the
            // whole tile stores gamma * acc; one covering its first steps
            // (the tile's "head") waits for the CTAs that ran its later steps
            // -- at the start of their ranges -- and adds their partial tiles
            // in CTA order; any other unit writes its partial tile to its
            // CTA's workspace slot and raises its flag.
            if (ok && !mbar_wait(acc_full, u & 1)) ok = false;
            tc_fence_after_sync();
            bar_sync_deq();  // this unit's gamma is written
            const bool whole = s0 == 0 && s1 == steps;
            const bool head = s0 == 0 && !whole;
            int q_lo = 0, q_hi = -1;  // contributing CTAs of a head unit
            if (head) {
                const int it0 = (tile - p.dp_tiles) * steps;
                q_lo = (int)blockIdx.x + 1;
                q_hi = sk_owner(p, it0 + steps - 1);
                if (td == 0) {
                    const uint64_t t0 = globaltimer_ns();
                    for (int q = q_lo; q <= q_hi && ok; ++q) {
                        while (ld_acquire_u32(p.ws_flag + q) == 0u) {
                            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                                atomicOr(&g_wlq_device_error, kErrWaitTimeout);
                                ok = false;
                                break;
                            }
                            __nanosleep(256);
                        }
                        p.ws_flag[q] = 0u;  // consumed; each CTA writes one partial per launch at most
                    }
                }
                bar_sync_deq();
            }
            const int qd = warp & 3;
            constexpr int kCcPerWarp = Tile<BN>::kCcPerWarp;
            const int c_lo = ((warp - kDeqBase / 32) >> 2) * kCcPerWarp;
            T* out = reinterpret_cast<T*>(p.out);
            // partial tiles are stored thread-major -- float4 i4 of column
            // chunk cc, accumulator a of dequant warp wd at float4 index
            // (((wd NACC + a) kCcPerWarp + cc - c_lo) 8 + i4) 32 + lane -- so
            // every warp access is 512 contiguous bytes; the head reads them
            // back with the same mapping (same kernel, same shape)
            const int wd = warp - kDeqBase / 32;
            float4* mine = reinterpret_cast<float4*>(p.ws_part + (size_t)blockIdx.x * kPartFloats);
#pragma unroll
            for (int a = 0; a < NACC; ++a) {
                const int row = a * kTileM + 32 * qd + lane;  // token row within the tile
                const int m = m0 + row;
#pragma unroll 1
                for (int cc = c_lo; cc < c_lo + kCcPerWarp; ++cc) {
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * qd) << 16) + a * BN + 32 * cc, v);
                    tmem_ld_wait();
                    if (!ok) continue;
                    const size_t pbase = (size_t)(((wd * NACC + a) * kCcPerWarp + (cc - c_lo)) * 8) * 32 + lane;
                    if (!whole && !head) {  // partial tile into this CTA's slot
#pragma unroll
                        for (int i = 0; i < 32; i += 4)
                            mine[pbase + (size_t)(i / 4) * 32] =
                                make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                                            __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
                        continue;
                    }
                    if (head) {
#pragma unroll 1
                        for (int q = q_lo; q <= q_hi; ++q) {
                            const float* src = p.ws_part + (size_t)q * kPartFloats + 4 * pbase;
#pragma unroll
                            for (int i0 = 0; i0 < 32; i0 += 16) {  // 16 values in flight
                                float4 w[4];
#pragma unroll
                                for (int e = 0; e < 4; ++e) w[e] = ldcg_f4(src + (size_t)((i0 + 4 * e) / 4) * 128);
#pragma unroll
                                for (int e = 0; e < 4; ++e) {
                                    const int i = i0 + 4 * e;
                                    v[i] = __float_as_uint(__uint_as_float(v[i]) + w[e].x);
                                    v[i + 1] = __float_as_uint(__uint_as_float(v[i + 1]) + w[e].y);
                                    v[i + 2] = __float_as_uint(__uint_as_float(v[i + 2]) + w[e].z);
                                    v[i + 3] = __float_as_uint(__uint_as_float(v[i + 3]) + w[e].w);
                                }
                            }
                        }
                    }
                    if (m >= p.M) continue;
                    const int nb = n0 + 32 * cc;
                    T* orow_out = out + (int64_t)m * p.N + nb;
                    const float* gm = gam + 32 * cc;
                    if (p.vec_out && nb + 32 <= p.N) {
#pragma unroll
                        for (int q4 = 0; q4 < 4; ++q4) {
                            uint32_t w[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int i = 8 * q4 + 2 * e;
                                w[e] = pack2<T>(__uint_as_float(v[i]) * gm[i], __uint_as_float(v[i + 1]) * gm[i + 1]);
                            }
                            *reinterpret_cast<uint4*>(orow_out + 8 * q4) = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (nb + i < p.N) orow_out[i] = ActTraits<T>::from_f32(__uint_as_float(v[i]) * gm[i]);
                    }
                }
            }
            if (!whole && !head) {
                // publish the partial: every thread's stores, then the flag
                __threadfence();
                bar_sync_deq();
                if (td == 0) st_release_u32(p.ws_flag + blockIdx.x, 1u);
            }
            // the accumulators are free for the next unit
            tc_fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
            bar_sync_deq();  // every epilogue read of gamma is done
            ++u;
        }
    }

    tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after_sync();
        tmem_dealloc(tmem, NACC * BN);
    }
}

// ---------------------------------------------------------------- host side
template <typename T, int NACC, int NPG, bool PREPACKED, int BN>
int launch_tiles(const GemmParams& p, int grid, cudaStream_t stream) {
    using P = Plan<NACC, NPG, BN>;
    auto kern = gemm_kernel<T, NACC, NPG, PREPACKED, BN>;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P::kAlloc);
    if (e != cudaSuccess) return check_cuda(e, "gemm_kernel smem attribute");
    kern<<<(unsigned)grid, kThreads, P::kAlloc, stream>>>(p);
    return check_cuda(cudaGetLastError(), "gemm_kernel launch");
}

template <typename T, int NACC, int BN>
int dispatch_npg(const GemmParams& p, int grid, int npg, bool prepacked, cudaStream_t stream) {
    switch (npg) {
        case 0: return prepacked ? launch_tiles<T, NACC, 0, true, BN>(p, grid, stream)
                                 : launch_tiles<T, NACC, 0, false, BN>(p, grid, stream);
        case 1: return prepacked ? launch_tiles<T, NACC, 1, true, BN>(p, grid, stream)
                                 : launch_tiles<T, NACC, 1, false, BN>(p, grid, stream);
        default: return prepacked ? launch_tiles<T, NACC, 2, true, BN>(p, grid, stream)
                                  : launch_tiles<T, NACC, 2, false, BN>(p, grid, stream);
    }
}

// CTA shapes built: 256 tokens x 256 or 128 rows, 128 tokens x 128 rows
template <typename T>
int dispatch_shape(const GemmParams& p, int grid, int nacc, int bn, int npg, bool prepacked, cudaStream_t stream) {
    if (nacc == 2)
        return bn == 256 ? dispatch_npg<T, 2, 256>(p, grid, npg, prepacked, stream)
                         : dispatch_npg<T, 2, 128>(p, grid, npg, prepacked, stream);
    return dispatch_npg<T, 1, 128>(p, grid, npg, prepacked, stream);
}

constexpr int kMinSkIters = 4;         // k steps per stream-K CTA at least
constexpr double kUnitOverhead = 2.0;  // a unit's epilogue and pipeline restart, in k steps

// One launch shape and schedule.
struct Sched {
    int nacc, bn;
    int grid, mtiles, dp_tiles, sk_ctas;
    int sk_iters;
    double cost;  // estimated time, arbitrary units
};

// Schedule of one CTA shape: data-parallel when the tiles fill whole waves
// (or there is no workspace); otherwise the last full wave and the remainder
// run stream-K over up to one CTA per SM, as many as the workspace holds
// partial tiles for.  The estimate counts the k steps on the busiest CTA (a
// step of the 256 x 256 shape = 1, scaled by the shape's size and its
// measured relative efficiency) plus the stream-K fix-up: the head CTA of a
// tile reads the other CTAs' partial tiles from L2 (about a step's time per
// 64 KB partial).
Sched plan_shape(int nacc, int bn, double eff, int M, int N, int steps, int sms, size_t ws_part_bytes) {
    Sched s{};
    s.nacc = nacc;
    s.bn = bn;
    s.mtiles = (M + nacc * kTileM - 1) / (nacc * kTileM);
    const int tiles = s.mtiles * ((N + bn - 1) / bn);
    const double step = (double)(nacc * kTileM) * bn / (256.0 * 256.0) / eff;
    const size_t part = (size_t)nacc * kTileM * bn * 4;
    const int fit = (int)(ws_part_bytes / part);
    const double dp_cost = (double)((tiles + sms - 1) / sms) * (steps + kUnitOverhead) * step;
    if (fit < 2 || tiles % sms == 0) {  // data-parallel
        s.grid = tiles;
        s.dp_tiles = tiles;
        s.cost = dp_cost;
        return s;
    }
    const int waves = tiles / sms;
    s.dp_tiles = waves > 0 ? (waves - 1) * sms : 0;
    const int sk_tiles = tiles - s.dp_tiles;
    s.sk_iters = sk_tiles * steps;
    long long ctas = s.sk_iters / kMinSkIters;
    if (ctas > sms) ctas = sms;
    if (ctas > fit) ctas = fit;
    if (ctas < 1) ctas = 1;
    s.sk_ctas = (int)ctas;
    s.grid = s.dp_tiles > 0 ? sms : s.sk_ctas;
    const double per_cta = (double)s.sk_iters / s.sk_ctas;
    const double units = per_cta / steps + 1.0;           // units per stream-K CTA
    const double readers = (double)s.sk_ctas / sk_tiles;  // CTAs per tile
    const double fixup = (readers > 1.0 ? readers - 1.0 : 0.0) * (double)part / 65536.0 + (double)part / 65536.0;
    s.cost = (double)(s.dp_tiles / sms) * (steps + kUnitOverhead) * step +
             (per_cta + units * kUnitOverhead) * step + fixup * 0.25;
    if (s.cost >= dp_cost) {  // stream-K does not pay: data-parallel
        s.grid = tiles;
        s.dp_tiles = tiles;
        s.sk_ctas = 0;
        s.sk_iters = 0;
        s.cost = dp_cost;
    }
    return s;
}

// M > 16 shapes the TMA path cannot take run as decode GEMVs over 16-token slices.
int gemm_by_slices(const LinearArgs& a, cudaStream_t stream) {
    const size_t es = 2;
    for (int m = 0; m < a.M; m += 16) {
        LinearArgs s = a;
        s.M = a.M - m < 16 ? a.M - m : 16;
        s.x = static_cast<const char*>(a.x) + (size_t)m * a.K * es;
        s.out = static_cast<char*>(a.out) + (size_t)m * a.N * es;
        if (a.lorah) s.lorah = a.lorah + (size_t)m * a.r;
        const int rc = launch_gemv(s, stream);
        if (rc) return rc;
    }
    return WLQ_OK;
}

}  // namespace

int launch_gemm(const LinearArgs& a, cudaStream_t stream) {
    if (a.M == 0 || a.N == 0) return WLQ_OK;
    int log2G = 0;
    if (a.group_size > 0) {
        while ((1 << log2G) < a.group_size) ++log2G;
        if ((1 << log2G) != a.group_size || a.group_size < 32 || a.group_offset % 32 != 0)
            return fail(WLQ_ERR_UNSUPPORTED,
                        "wlq_gemm: per-group codebooks need a power-of-two group_size >= 32 and a group_offset "
                        "multiple of 32 (got %d, %d)", a.group_size, a.group_offset);
    }
    const bool tma_ok = a.K % 8 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
                        (a.off == nullptr || a.chunk_m % kBK == 0);
    if (!tma_ok) return gemm_by_slices(a, stream);

    // CTA shape: 256 tokens x 256 rows needs the least dequantisation and the
    // least activation traffic per FLOP; smaller shapes fill the GPU when the
    // problem is small.  Pick the schedule with the least estimated time
    // (relative efficiency of each shape measured on B200).
    const int sms = device_sm_count();
    const int steps = (a.K + kBK - 1) / kBK + (a.r > 0 ? (a.r + kBK - 1) / kBK : 0);
    const size_t flag_bytes = ((size_t)sms * 4 + 255) / 256 * 256;
    const size_t part_bytes = a.ws != nullptr && a.ws_bytes > flag_bytes ? a.ws_bytes - flag_bytes : 0;
    struct Shape { int nacc, bn; double eff; };
    const Shape shapes[3] = {{2, 256, 1.0}, {2, 128, 0.85}, {1, 128, 0.55}};
    Sched sc{};
    sc.cost = 1e300;
    for (const Shape& sh : shapes) {
        const Sched c = plan_shape(sh.nacc, sh.bn, sh.eff, a.M, a.N, steps, sms, part_bytes);
        if (c.cost < sc.cost * (1.0 - 1e-9)) sc = c;
    }
    const int nacc = sc.nacc, bn = sc.bn;

    GemmParams p;
    memset(&p, 0, sizeof(p));
    const CUtensorMapDataType xdt =
        a.dtype == WLQ_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    int rc = encode_2d(&p.tm_x, xdt, a.x, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2, kBK, kTileM,
                       CU_TENSOR_MAP_SWIZZLE_128B, "X");
    if (rc) return rc;
    rc = encode_2d(&p.tm_q, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.q, (uint64_t)a.wpr, (uint64_t)a.N, (uint64_t)a.wpr * 4,
                   kBK / 8, (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_NONE, "q_packed");
    if (rc) return rc;
    // codebooks per 64-column step: 1 when groups of >= 64 columns align with
    // the steps, else 2 (a step then spans at most two groups)
    const int npg = a.group_size == 0 ? 0 : (a.group_size >= kBK && a.group_offset % kBK == 0) ? 1 : 2;
    if (npg > 0) {
        rc = encode_2d(&p.tm_lut, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.lut, (uint64_t)a.ngroups * 8, (uint64_t)a.N,
                       (uint64_t)a.ngroups * 32, 8 * npg, (uint32_t)bn, CU_TENSOR_MAP_SWIZZLE_NONE, "lut_c");
        if (rc) return rc;
    }
    p.lut = a.lut; p.out = a.out; p.off = a.off; p.ccols = a.ccols; p.cvals = a.cvals;
    p.loraB = a.loraB; p.lorah = a.lorah; p.gamma = a.gamma; p.scale = a.scale;
    p.r = a.r; p.M = a.M; p.N = a.N; p.K = a.K;
    p.ngroups = a.ngroups; p.goff = a.group_offset; p.log2G = log2G;
    p.chunk_m = a.chunk_m; p.ncsr = a.ncsr;
    p.ksteps = (a.K + kBK - 1) / kBK;
    p.lsteps = a.r > 0 ? (a.r + kBK - 1) / kBK : 0;
    p.mul16 = 1u << 16;
    p.mul31 = 1u << 31;
    p.vec_out = (a.N % 8 == 0) && ((reinterpret_cast<uintptr_t>(a.out) & 15) == 0);
    p.mtiles = sc.mtiles;
    p.dp_tiles = sc.dp_tiles;
    p.sk_ctas = sc.sk_ctas;
    p.sk_iters = sc.sk_iters;
    if (sc.sk_ctas > 0) {
        p.ws_flag = static_cast<uint32_t*>(a.ws);
        p.ws_part = reinterpret_cast<float*>(static_cast<char*>(a.ws) + flag_bytes);
    }

    if (a.dtype == WLQ_DTYPE_BF16)
        return dispatch_shape<__nv_bfloat16>(p, sc.grid, nacc, bn, npg, a.lut_prepacked, stream);
    return dispatch_shape<__half>(p, sc.grid, nacc, bn, npg, a.lut_prepacked, stream);
}

size_t gemm_workspace_bytes() {
    const int sms = device_sm_count();
    return ((size_t)sms * 4 + 255) / 256 * 256 + (size_t)sms * (2 * kTileM) * 256 * 4;
}

// ------------------------------------------- stream-K without allocation
// Scratch of wlq_gemm_streamk_noalloc: a file-scope device array, so callers
// that cannot allocate device memory still get the stream-K schedule.  Every
// GPU that loads the library holds it (zero-filled at load) until the process
// exits; all calls on a device share it.
static __device__ __align__(256) unsigned char g_static_scratch[WLQ_GEMM_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_static_mu;
void* g_static_ptr[64] = {};  // device address of g_static_scratch, per device
}  // namespace

int launch_gemm_noalloc(const LinearArgs& a0, cudaStream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return check_cuda(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(WLQ_ERR_DEVICE, "wlq_gemm_streamk_noalloc: device %d out of range", dev);
    void* scratch = nullptr;
    {
        // set-up once per device, with that device current: in host code the
        // array's name is only a stand-in, so the kernels get its device
        // address from the runtime
        std::lock_guard<std::mutex> lock(g_static_mu);
        if (!g_static_ptr[dev]) {
            void* ptr = nullptr;
            e = cudaGetSymbolAddress(&ptr, g_static_scratch);
            if (e != cudaSuccess) return check_cuda(e, "wlq_gemm_streamk_noalloc: cudaGetSymbolAddress");
            g_static_ptr[dev] = ptr;
        }
        scratch = g_static_ptr[dev];
    }
    // the scratch this call's schedule needs: the schedule a full workspace
    // would give (flags plus one partial tile per stream-K CTA)
    const int sms = device_sm_count();
    const size_t flag_bytes = ((size_t)sms * 4 + 255) / 256 * 256;
    const int steps = (a0.K + kBK - 1) / kBK + (a0.r > 0 ? (a0.r + kBK - 1) / kBK : 0);
    const size_t full_part = gemm_workspace_bytes() - flag_bytes;
    const struct { int nacc, bn; double eff; } shapes[3] = {{2, 256, 1.0}, {2, 128, 0.85}, {1, 128, 0.55}};
    Sched sc{};
    sc.cost = 1e300;
    for (const auto& sh : shapes) {
        const Sched c = plan_shape(sh.nacc, sh.bn, sh.eff, a0.M, a0.N, steps, sms, full_part);
        if (c.cost < sc.cost * (1.0 - 1e-9)) sc = c;
    }
    const size_t need = sc.sk_ctas > 0 ? flag_bytes + (size_t)sc.sk_ctas * sc.nacc * kTileM * sc.bn * 4 : 0;
    if (need > WLQ_GEMM_STATIC_SCRATCH_BYTES)
        return fail(WLQ_ERR_CAPACITY,
                    "wlq_gemm_streamk_noalloc: M=%d N=%d K=%d needs %zu bytes of stream-K scratch, more than the "
                    "library's static %zu; use wlq_gemm_streamk with a workspace", a0.M, a0.N, a0.K, need,
                    (size_t)WLQ_GEMM_STATIC_SCRATCH_BYTES);
    // the flags must start at zero: a call that gave up waiting may have
    // left some set
    e = cudaMemsetAsync(scratch, 0, flag_bytes, stream);
    if (e != cudaSuccess) return check_cuda(e, "wlq_gemm_streamk_noalloc: clearing the flags");
    LinearArgs a = a0;
    a.ws = scratch;
    a.ws_bytes = WLQ_GEMM_STATIC_SCRATCH_BYTES;
    return launch_gemm(a, stream);
}

int read_device_error(int device, unsigned int* flags, int clear) {
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return check_cuda(e, "cudaGetDevice");
    if (device != prev && (e = cudaSetDevice(device)) != cudaSuccess) return check_cuda(e, "cudaSetDevice");
    // only this translation unit's kernels wait on mbarriers
    unsigned int v = 0;
    const int rc = tu_device_error(&v, clear);
    if (device != prev) cudaSetDevice(prev);
    if (rc) return rc;
    *flags = v;
    return WLQ_OK;
}

}  // namespace wlq
