// The decode GEMV kernel template and its launch helpers, shared by
// wlq_gemv.cu (low-rank input h given) and wlq_gemv_fold.cu (h = A x computed
// in the kernel); the design notes are at the top of wlq_gemv.cu.
#pragma once
#include <atomic>

#include "wlq_common.cuh"
#include "wlq_internal.h"

namespace wlq {
namespace gemv {

constexpr int kWarps = 4;
constexpr int kRowsPerTile = 16;
constexpr int kChunk = 128;  // k columns per warp iteration
constexpr int kMaxTp = 8;    // ranks of a fused all-reduce
constexpr int kMaxGemvM = 32;  // token rows of one launch: 1, 2 or 4 eight-token MMA tiles
constexpr int kMaxSplit = 16;  // CTAs of a K-split cluster (above 8: a non-portable cluster size)

// compile-time flag for generic lambdas
template <bool B> struct BoolTag { static constexpr bool value = B; };

struct GemvParams {
    const uint32_t* q;
    const uint16_t* lut;
    const void* x;
    void* out;
    const int32_t* off;
    const void* ccols;  // uint16 chunk-local columns, or uint32 records (prepacked)
    const void* cvals;  // e5m2 bytes, or float32 corrections (prepacked)
    const uint16_t* loraB;
    const float* lorah;    // [M, r] fp32, or null when the kernel computes h (loraA)
    const uint16_t* loraA; // [r, K] in the activation type (RT > 0)
    const uint16_t* gamma;
    float scale;
    int r, M, N, K, wpr, G, goff, ngroups, chunk_m, ncsr;
    int log2G;             // group_size = 1 << log2G when grouped
    int kchunks;           // ceil(K / 128)
    int chunks_per_rank;   // K split across the cluster
    int x_stride;          // shared-memory row stride of staged activations (elements)
    int x_bytes;           // bytes of dynamic shared memory before the ring (staged activations)
    uint32_t mul16, mul31; // 1<<16 and 1<<31, runtime values so mul.hi stays a multiply
    // fused tensor-parallel all-reduce (row-parallel layers), tp_world > 1
    int tp_world, tp_rank, tp_nmax;
    int tp_stride;                        // words per (parity, rank, token) row of each rank's slots
    unsigned long long* tp_data[kMaxTp];  // each rank's slots [2 parities][world][16 tokens][tp_stride]:
                                          // per tile eight words of two 16-bit values | epoch << 32
    uint32_t* tp_counters;       // this rank's per-tile call counters [tiles]
    uint32_t* tp_err;            // this rank's error word
};

// Codebook value of symbol q of one (row, group) as the MMA saw it.
template <typename T, bool PREPACKED>
__device__ __forceinline__ float codebook_value(const uint16_t* __restrict__ lut, int64_t entry, uint32_t q) {
    if (PREPACKED) {
        const uint8_t* rec = reinterpret_cast<const uint8_t*>(lut + entry * 16);
        const uint16_t bits = (uint16_t)(__ldg(rec + q) | ((uint16_t)__ldg(rec + 16 + q) << 8));
        return ActTraits<T>::bits_to_f32(bits);
    }
    return ActTraits<T>::bits_to_f32(ActTraits<T>::from_f16_bits(__ldg(lut + entry * 16 + q)));
}

// An 8-column activation piece at a constant byte offset from a chunk's
// base: shared memory (staged) or global through L1.
template <bool XSMEM, int OFF>
__device__ __forceinline__ uint4 x8_at(uint32_t sa, const uint16_t* gp) {
    if constexpr (XSMEM) return lds128_at<OFF>(sa);
    else return ldg_keep_v4_at<OFF>(gp);
}

// Issues the staging of x[0:M, kb:kb+cols) into shared memory as one
// cp.async group (the caller waits for it), rows padded by 8 elements (16
// bytes) so the per-token rows fall in different banks; columns past K read
// as zero.  16-byte cp.async when rows of x are 16-byte aligned.
template <typename T, bool XVEC>
__device__ __forceinline__ void stage_x_issue(uint16_t* xs, const T* __restrict__ x, int M, int K, int kb, int cols,
                                              int stride) {
    const uint16_t* xg = reinterpret_cast<const uint16_t*>(x);
    const int pieces = cols / 8;
    for (int e = threadIdx.x; e < M * pieces; e += blockDim.x) {
        const int m = e / pieces, pc = e - m * pieces;
        const int k = kb + 8 * pc;
        uint16_t* dst = xs + m * stride + 8 * pc;
        if (XVEC && k + 8 <= K) {
            const uint32_t sa = smem_u32(dst);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sa), "l"(xg + (int64_t)m * K + k) : "memory");
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[j] = k + j < K ? xg[(int64_t)m * K + k + j] : (uint16_t)0;
        }
    }
    cp_async_commit();
}

// Sum over the cluster's ranks of one partial-tile element, rank 0 first:
// the remote loads are all issued before the adds.
template <int MAXR>
__device__ __forceinline__ float cluster_sum_n(uint32_t a, uint32_t nranks) {
    float v[MAXR];
#pragma unroll
    for (int q = 0; q < MAXR; ++q)
        v[q] = (uint32_t)q < nranks ? ld_shared_cluster_f32(mapa_shared(a, (uint32_t)q)) : 0.f;
    float s = v[0];
#pragma unroll
    for (int q = 1; q < MAXR; ++q) s += v[q];
    return s;
}
__device__ __forceinline__ float cluster_sum(const float* own, uint32_t nranks) {
    if (nranks == 1) return *own;
    const uint32_t a = smem_u32(own);
    // the portable sizes (<= 8) keep to 8 loads in flight; adding zeros past
    // nranks leaves the sum unchanged
    return nranks <= 8 ? cluster_sum_n<8>(a, nranks) : cluster_sum_n<kMaxSplit>(a, nranks);
}

// Per-warp shared-memory ring of S stages, filled by cp.async (no register
// scoreboards held by prefetches).  A stage holds one 128-column chunk: the
// index words of the warp's 16 rows (16 x 64 B), with per-group codebooks
// NSLOT codebooks per row (16 x NSLOT x 32 B, slot s holding group g0 + s
// where g0 is the group of the chunk's first column), and when the kernel
// computes h = A x, the warp's 32-column block of A (RT x 16 rows x 64 B).
template <int NSLOT, int RT>
struct Ring {
    static constexpr int kIdxBytes = kRowsPerTile * 64;
    static constexpr int kPlaneBytes = kRowsPerTile * NSLOT * 32;
    static constexpr int kABytes = RT * 16 * 64;
    static constexpr int kStageBytes = kIdxBytes + kPlaneBytes + kABytes;
};

// 16-byte slot accesses that reach the other GPUs' memory and are never
// cached or merged.  Each 8-byte half is written and read whole (single-copy
// atomic) and carries its own epoch, so a reader that sees one half of a
// pair early simply reads the pair again.
__device__ __forceinline__ void st_slot2(unsigned long long* a, unsigned long long v0, unsigned long long v1) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(a), "l"(v0), "l"(v1) : "memory");
}
__device__ __forceinline__ void ld_slot2(const unsigned long long* a, unsigned long long& v0, unsigned long long& v1) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v0), "=l"(v1) : "l"(a) : "memory");
}

// Row-parallel epilogue with the all-reduce fused, for one warp's 16-row
// tile (cluster rank 0).  First every lane finishes its elements of the tile
// (the K-split sum over the cluster, times the row's DoRA magnitude) in place
// in the warp's own partial tile, rounded to the activation type -- what a
// rank's output would carry into an all-reduce after the GEMV.  Then the
// values go out packed two to an 8-byte word with the call's 32-bit epoch;
// two words (rows 4pg .. 4pg + 3 of one token) go to every other rank in one
// 16-byte store.  A reader knows a word is complete once its epoch matches:
// no fences and no separate flags on the way (a system-scope fence per tile
// cost ~25 us per call over NVLink), and four values per store instead of
// one.  Epochs come from a per-tile call counter that advances identically
// on every rank, so CUDA graph replays need no host input; slots alternate by
// epoch parity, and a rank cannot run two calls ahead on a tile because each
// call waits for all ranks' values of the previous one.  Every rank adds the
// same rounded values in rank order, so all ranks hold the same result bit
// for bit.  The waits share one 2 s deadline; when it passes the error word
// is set and the output is undefined.
template <typename T, int MT>
__device__ void tp_allreduce_tile(const GemvParams& p, float (*part)[MT], uint32_t nranks, int tile_row0, int lane,
                                  float gam) {
    // lane owns elements e = lane + 32 i: row e % 16 (= lane % 16, whose
    // magnitude `gam` is), token e / 16.  Only this warp reads or writes its
    // own tile here; the other cluster ranks' tiles are only read.
#pragma unroll
    for (int e = lane; e < kRowsPerTile * MT; e += 32) {
        const int rl = e % kRowsPerTile, tk = e / kRowsPerTile;
        const int n = tile_row0 + rl;
        float v = 0.f;
        if (n < p.N && tk < p.M) v = cluster_sum(&part[rl][tk], nranks) * gam;
        part[rl][tk] = ActTraits<T>::to_f32(ActTraits<T>::from_f32(v));
    }
    __syncwarp();
    // pair pr = (token tk, group pg): words 2pg and 2pg + 1 of the token's
    // eight, word w holding rows 2w and 2w + 1 of the tile
    constexpr int kPairs = 4 * MT;
    constexpr int kPer = (kPairs + 31) / 32;
    const int tile = tile_row0 / kRowsPerTile;
    const int world = p.tp_world, me = p.tp_rank;
    uint32_t cnt = lane == 0 ? p.tp_counters[tile] + 1u : 0u;
    cnt = __shfl_sync(0xFFFFFFFFu, cnt, 0);
    const int par = (int)(cnt & 1u);
    const unsigned long long tag = (unsigned long long)cnt << 32;
    auto slot_of = [&](int src, int tk, int pg) {
        return ((int64_t)(par * world + src) * kRowsPerTile + tk) * p.tp_stride + tile * 8 + 2 * pg;
    };
    auto bits = [](float v) {  // v is exactly representable in T
        const T t = ActTraits<T>::from_f32(v);
        return (unsigned long long)*reinterpret_cast<const uint16_t*>(&t);
    };
    unsigned long long mine[kPer][2];
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int pr = lane + 32 * i;
        const int tk = pr >> 2, pg = pr & 3;
        mine[i][0] = mine[i][1] = 0ull;
        if (pr >= kPairs || tk >= p.M) continue;
        mine[i][0] = tag | bits(part[4 * pg][tk]) | (bits(part[4 * pg + 1][tk]) << 16);
        mine[i][1] = tag | bits(part[4 * pg + 2][tk]) | (bits(part[4 * pg + 3][tk]) << 16);
        const int64_t slot = slot_of(me, tk, pg);
        for (int q = 0; q < world; ++q)
            if (q != me) st_slot2(p.tp_data[q] + slot, mine[i][0], mine[i][1]);
    }
    const uint64_t deadline = globaltimer_ns() + 2000000000ull;
    bool ok = true;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int pr = lane + 32 * i;
        const int tk = pr >> 2, pg = pr & 3;
        if (pr >= kPairs || tk >= p.M) continue;
        float s[4] = {0.f, 0.f, 0.f, 0.f};
        for (int q = 0; q < world; ++q) {
            unsigned long long w0 = mine[i][0], w1 = mine[i][1];
            if (q != me) {
                const unsigned long long* a = p.tp_data[me] + slot_of(q, tk, pg);
                ld_slot2(a, w0, w1);
                while (((uint32_t)(w0 >> 32) != cnt || (uint32_t)(w1 >> 32) != cnt) && ok) {
                    if (globaltimer_ns() > deadline) ok = false;  // a rank never arrived: give up
                    else ld_slot2(a, w0, w1);
                }
            }
            s[0] += ActTraits<T>::bits_to_f32((uint16_t)w0);
            s[1] += ActTraits<T>::bits_to_f32((uint16_t)(w0 >> 16));
            s[2] += ActTraits<T>::bits_to_f32((uint16_t)w1);
            s[3] += ActTraits<T>::bits_to_f32((uint16_t)(w1 >> 16));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = tile_row0 + 4 * pg + j;
            if (n < p.N) reinterpret_cast<T*>(p.out)[(int64_t)tk * p.N + n] = ActTraits<T>::from_f32(s[j]);
        }
    }
    if (!ok) atomicOr(p.tp_err, 1u);
    __syncwarp();
    if (lane == 0) p.tp_counters[tile] = cnt;
}

// RT > 0: the low-rank input h = A x (r <= 16 RT) is computed here.  Each
// chunk's 128 columns are four 32-column blocks; a warp multiplies the blocks
// it is assigned (all four warps of a 4-warp CTA take block w of every chunk;
// see h_duty for 16 warps), staged through its ring, with the activations on
// the tensor core (A rows are the MMA's A operand, tokens its B operand);
// after the main loop the warps' partial h meet in shared memory and each
// warp adds s B h for its rows.  With the K
// range split over a cluster each rank adds the term for its own range, and
// the split-K reduction sums them.
template <typename T, int NT, int NSLOT, bool PREPACKED, bool XVEC, bool XSMEM, int S, int RT, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 16 / WARPS) gemv_kernel(const GemvParams p) {
    constexpr bool GROUPED = NSLOT > 0;
    constexpr int MT = 8 * NT;
    using R = Ring<NSLOT, RT>;
    static_assert(S >= 2, "ring needs two stages");
    static_assert(RT == 0 || XVEC, "h = A x in the kernel needs 16-byte aligned rows");
    static_assert(S * R::kStageBytes >= RT * 16 * MT * 4, "the partial h reuses the ring");
    static_assert(WARPS == 4 || WARPS == 16, "4 warps (4 CTAs per SM) or 16 (one CTA per SM)");
    extern __shared__ __align__(128) uint8_t smem[];  // [x stage (XSMEM)][WARPS][S] ring stages
    __shared__ float part[WARPS][kRowsPerTile][MT];   // per-warp partial tile

    const int warp = threadIdx.x >> 5;
    // the next launch in the stream (a programmatic dependent launch) may
    // begin its weight prologue on the SMs this grid's CTAs leave
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;
    const int tile_row0 = (blockIdx.x * WARPS + warp) * kRowsPerTile;
    // computing h = A x: every chunk's 128 columns are split into four
    // 32-column blocks; warp w takes block w % 4 of the chunks whose offset
    // in the CTA's range is w / 4 modulo WARPS / 4 (every chunk with 4 warps)
    constexpr int kHPhases = WARPS / 4;
    const int hblk = warp & 3, hphase = warp >> 2;
    auto h_duty = [&](int c) { return kHPhases == 1 || (c - blockIdx.y * p.chunks_per_rank) % kHPhases == hphase; };
    const int row0 = tile_row0 + g;
    const bool v0 = row0 < p.N;
    const bool v1 = row0 + 8 < p.N;
    const T* x = reinterpret_cast<const T*>(p.x);
    const uint32_t m16 = p.mul16, m31 = p.mul31;
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem);  // [M][x_stride] activations of this rank's K range
    const uint32_t ring = smem_u32(smem + p.x_bytes) + (uint32_t)(warp * S * R::kStageBytes);

    const int c_begin = blockIdx.y * p.chunks_per_rank;
    const int c_end = min(p.kchunks, c_begin + p.chunks_per_rank);

    // codebook group of a column (clamped: columns past K meet zero activations)
    auto group_at = [&](int col) { return min((col + p.goff) >> p.log2G, p.ngroups - 1); };
    // codebook slot of this lane's 32 columns within a chunk: the same for
    // every chunk when groups are at most a chunk wide (a chunk then starts on
    // a group boundary plus goff % G).  Columns past K may land on a slot the
    // chunk did not load; it was zero-filled and their activations are zero.
    const int lane_slot = p.G <= kChunk ? ((p.goff & (p.G - 1)) + 32 * t) >> p.log2G : 0;

    // The lane's part of every ring copy is fixed for the whole K range: the
    // 16-byte piece q4 = lane % 4 of index rows lane / 4 and lane / 4 + 8, its
    // codebook slot and half, and (computing h) its rows of A.  Their sources
    // at chunk 0 and their byte counts (16, or 0 to zero-fill a row past N or
    // a rank past r) are set once; a chunk inside K then costs one wide
    // multiply-add per copy and no integer/logic instruction.  Chunks past
    // c_full (a ragged K end) take the checked path.
    const int q4 = lane & 3;
    const int ir = lane >> 2;
    const int c_full = p.K / kChunk;
    const bool iok0 = tile_row0 + ir < p.N, iok1 = tile_row0 + ir + 8 < p.N;
    const uint32_t ioff0 = iok0 ? (uint32_t)(tile_row0 + ir) * (uint32_t)p.wpr + 4u * q4 : 0u;
    const uint32_t ioff1 = iok1 ? (uint32_t)(tile_row0 + ir + 8) * (uint32_t)p.wpr + 4u * q4 : 0u;
    const uint32_t qn0 = iok0 ? 16u : 0u, qn1 = iok1 ? 16u : 0u;
    const uint32_t idst = (uint32_t)(ir * 64 + q4 * 16);
    constexpr int kSlots = GROUPED ? NSLOT : 1;
    const int ls = (lane >> 1) % kSlots, lhalf = lane & 1;  // codebook slot and half of this lane
    // groups at most a chunk wide: chunk c's first group is c * (128 / G) +
    // goff / G and the chunk spans the same number of groups every time
    const bool cb_fixed = GROUPED && p.G <= kChunk;
    const uint32_t cb_step = cb_fixed ? (uint32_t)(kChunk >> p.log2G) * 32u : 0u;  // codebook bytes per chunk
    const int cb_used = cb_fixed ? (kChunk >> p.log2G) + ((p.goff & (p.G - 1)) != 0 ? 1 : 0) : 0;
    bool lok[kSlots];
    uint32_t loff[kSlots], ldst[kSlots], lnf[kSlots];
#pragma unroll
    for (int i = 0; i < kSlots; ++i) {
        const int r = (lane + 32 * i) / (2 * kSlots);
        lok[i] = tile_row0 + r < p.N;
        loff[i] = lok[i] ? ((uint32_t)(tile_row0 + r) * (uint32_t)p.ngroups + ls) * 16u + 8u * lhalf : 0u;
        ldst[i] = (uint32_t)(R::kIdxBytes + (r * kSlots + ls) * 32 + lhalf * 16);
        lnf[i] = lok[i] && ls < cb_used ? 16u : 0u;
    }
    const uint16_t* lbase = p.lut + (cb_fixed ? (uint32_t)(p.goff >> p.log2G) * 16u : 0u);
    constexpr int kAPieces = RT > 0 ? 2 * RT : 1;
    uint32_t aoff[kAPieces], an[kAPieces];
    bool aok[kAPieces];
#pragma unroll
    for (int i = 0; i < kAPieces; ++i) {
        const int ar = ir + 8 * i;
        aok[i] = RT > 0 && ar < p.r;
        aoff[i] = aok[i] ? (uint32_t)ar * (uint32_t)p.K + 32u * hblk + 8u * q4 : 0u;
        an[i] = aok[i] ? 16u : 0u;
    }

    // chunk c into ring stage st; one commit group per lane per chunk, empty
    // past the rank's range
    auto issue = [&](int c, int st) {
        if (c < c_end) {
            const uint32_t base = ring + (uint32_t)(st * R::kStageBytes);
            const uint32_t cu = (uint32_t)c;
            if (c < c_full) {
                cp_async16_n(base + idst, ptr_mad(p.q + ioff0, cu, 64u), qn0);
                cp_async16_n(base + idst + 8 * 64, ptr_mad(p.q + ioff1, cu, 64u), qn1);
                if constexpr (GROUPED) {
                    if (cb_fixed) {
#pragma unroll
                        for (int i = 0; i < NSLOT; ++i)
                            cp_async16_n(base + ldst[i], ptr_mad(lbase + loff[i], cu, cb_step), lnf[i]);
                    } else {
                        const int g0 = (c * kChunk + p.goff) >> p.log2G;
                        const int used = ((c * kChunk + kChunk - 1 + p.goff) >> p.log2G) - g0 + 1;
#pragma unroll
                        for (int i = 0; i < NSLOT; ++i)
                            cp_async16_n(base + ldst[i], ptr_mad(p.lut + loff[i], (uint32_t)g0, 32u),
                                         lok[i] && ls < used ? 16u : 0u);
                    }
                }
                if (RT > 0 && h_duty(c)) {
#pragma unroll
                    for (int i = 0; i < 2 * RT; ++i)
                        cp_async16_n(base + R::kIdxBytes + R::kPlaneBytes + (ir + 8 * i) * 64 + q4 * 16,
                                     ptr_mad(p.loraA + aoff[i], cu, 2u * kChunk), an[i]);
                }
            } else {
                const uint32_t wi = cu * (kChunk / 8);  // first index word of the chunk
                const bool wok = (int)(wi + 4u * q4) < p.wpr;
                const bool ok0 = iok0 && wok, ok1 = iok1 && wok;
                cp_async16(base + idst, p.q + (ok0 ? ioff0 + wi : 0u), ok0);
                cp_async16(base + idst + 8 * 64, p.q + (ok1 ? ioff1 + wi : 0u), ok1);
                if constexpr (GROUPED) {
                    const int g0 = group_at(c * kChunk);
                    const int used = group_at(c * kChunk + kChunk - 1) - g0 + 1;
                    const bool sok = ls < used;
#pragma unroll
                    for (int i = 0; i < NSLOT; ++i) {
                        const bool ok = lok[i] && sok;
                        cp_async16(base + ldst[i], p.lut + (ok ? loff[i] + (uint32_t)g0 * 16u : 0u), ok);
                    }
                }
                if (RT > 0 && h_duty(c)) {
                    // rows [0, 16 RT) of A, columns [128c + 32b, +32) of this
                    // warp's block b; rows past r and columns past K (K % 8
                    // == 0) read as zero
                    const uint32_t ca = cu * kChunk;
                    const bool cok = (int)(ca + 32u * hblk + 8u * q4) < p.K;
#pragma unroll
                    for (int i = 0; i < 2 * RT; ++i) {
                        const bool ok = aok[i] && cok;
                        cp_async16(base + R::kIdxBytes + R::kPlaneBytes + (ir + 8 * i) * 64 + q4 * 16,
                                   p.loraA + (ok ? aoff[i] + ca : 0u), ok);
                    }
                }
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int j = 0; j < S - 1; ++j) issue(c_begin + j, j);
    const int kb0 = c_begin * kChunk;

    // per-row codebooks (no grouping) stay in registers for the whole K range
    LutPlanes PR0, PR1;
    if (!GROUPED) {
        load_planes<T, PREPACKED>(p.lut, row0, v0, PR0);
        load_planes<T, PREPACKED>(p.lut, row0 + 8, v1, PR1);
    }

    float acc[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;

    // this row's outlier range (prepacked layout), loaded before the
    // activation staging wait so the latency overlaps it
    const bool o_has = p.off != nullptr && c_begin < c_end && tile_row0 + (lane & 15) < p.N;
    int o_ia = 0, o_ib = 0;
    if (PREPACKED && o_has) {
        const int32_t* ro = p.off + (int64_t)(tile_row0 + (lane & 15)) * (p.ncsr + 1);
        o_ia = __ldg(ro + c_begin * kChunk / p.chunk_m);
        o_ib = __ldg(ro + (min(p.K, c_end * kChunk) - 1) / p.chunk_m + 1);
    }
    // DoRA magnitude of the row this lane finishes in the epilogue
    const int erow = tile_row0 + (lane & 15);
    const float gam = (p.r > 0 && erow < p.N) ? f16_bits_to_f32(__ldg(p.gamma + erow)) : 1.f;

    // DoRA low-rank term s * B h on the tensor core, once per output tile
    // (cluster rank 0), into the accumulators before the main loop: A = the
    // tile's 16 rows of B (k = rank index), the B operand = s * h per token,
    // both rounded to the MMA type
    const uint16_t* B0 = p.r > 0 ? p.loraB + (int64_t)(v0 ? row0 : 0) * p.r : p.loraB;
    const uint16_t* B1 = p.r > 0 ? p.loraB + (int64_t)(v1 ? row0 + 8 : 0) * p.r : p.loraB;
    auto bval = [&](const uint16_t* Br, bool ok, int k) -> uint32_t {  // one 16-bit element of B
        return (ok && k < p.r) ? (uint32_t)ActTraits<T>::from_f16_bits(__ldg(Br + k)) : 0u;
    };
    // with h computed here: the tile's B fragments now, h's accumulators
    uint32_t bfrag[RT > 0 ? RT : 1][4];
    float hacc[RT > 0 ? RT : 1][NT][4];
    if constexpr (RT > 0) {
#pragma unroll
        for (int rt = 0; rt < RT; ++rt) {
            const int k0 = 16 * rt + 2 * t, k8 = k0 + 8;
            bfrag[rt][0] = bval(B0, v0, k0) | (bval(B0, v0, k0 + 1) << 16);
            bfrag[rt][1] = bval(B1, v1, k0) | (bval(B1, v1, k0 + 1) << 16);
            bfrag[rt][2] = bval(B0, v0, k8) | (bval(B0, v0, k8 + 1) << 16);
            bfrag[rt][3] = bval(B1, v1, k8) | (bval(B1, v1, k8 + 1) << 16);
#pragma unroll
            for (int tt = 0; tt < NT; ++tt)
#pragma unroll
                for (int i = 0; i < 4; ++i) hacc[rt][tt][i] = 0.f;
        }
    }
    // Everything above reads weights only.  The activations, h and the
    // output follow the previous kernel in stream order: launched as a
    // programmatic dependent launch, this grid starts while the previous one
    // drains and waits here for it to complete (a no-op otherwise).
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // this rank's activations into shared memory (XSMEM), waited for after
    // the low-rank MMA; larger slices are read through L1
    if (XSMEM) stage_x_issue<T, XVEC>(xs, x, p.M, p.K, kb0, p.chunks_per_rank * kChunk, p.x_stride);
    if (RT == 0 && p.r > 0 && (gridDim.y == 1 || cluster_ctarank() == 0u)) {
        for (int kb = 0; kb < p.r; kb += 16) {
            uint32_t a[4];
            const int k0 = kb + 2 * t, k8 = kb + 2 * t + 8;
            a[0] = bval(B0, v0, k0) | (bval(B0, v0, k0 + 1) << 16);
            a[1] = bval(B1, v1, k0) | (bval(B1, v1, k0 + 1) << 16);
            a[2] = bval(B0, v0, k8) | (bval(B0, v0, k8 + 1) << 16);
            a[3] = bval(B1, v1, k8) | (bval(B1, v1, k8 + 1) << 16);
#pragma unroll
            for (int tt = 0; tt < NT; ++tt) {
                const int tok = 8 * tt + g;
                const float* h = p.lorah + (int64_t)(tok < p.M ? tok : 0) * p.r;
                auto hv = [&](int k) { return (tok < p.M && k < p.r) ? p.scale * __ldg(h + k) : 0.f; };
                const T h0 = ActTraits<T>::from_f32(hv(k0)), h1 = ActTraits<T>::from_f32(hv(k0 + 1));
                const T h8 = ActTraits<T>::from_f32(hv(k8)), h9 = ActTraits<T>::from_f32(hv(k8 + 1));
                const uint32_t b0 = (uint32_t)*reinterpret_cast<const uint16_t*>(&h0) |
                                    ((uint32_t)*reinterpret_cast<const uint16_t*>(&h1) << 16);
                const uint32_t b1 = (uint32_t)*reinterpret_cast<const uint16_t*>(&h8) |
                                    ((uint32_t)*reinterpret_cast<const uint16_t*>(&h9) << 16);
                Mma16816<T>::run(acc[tt], a, b0, b1);
            }
        }
    }

    // this lane's first outlier entries (prepacked layout: global columns
    // and ready corrections), loaded before the activation wait; lanes l and
    // l+16 take alternate entries of row l % 16, four in flight per lane
    const uint32_t* orec = reinterpret_cast<const uint32_t*>(p.ccols);
    const float* odel = reinterpret_cast<const float*>(p.cvals);
    int ocol[4];
    float odl[4];
    auto load_outliers = [&](int i0, int ib) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = i0 + 2 * u;
            ocol[u] = i < ib ? (int)(__ldg(orec + i) & 0xFFFFu) : -1;
            odl[u] = i < ib ? __ldg(odel + i) : 0.f;
        }
    };
    if (PREPACKED && o_has) load_outliers(o_ia + (lane >> 4), o_ib);
    if (XSMEM) {
        cp_async_wait<0>();  // the staged activations (and the ring's first chunks)
        __syncthreads();
    }
    bool tok_ok[NT];
    const uint16_t* xrow[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        tok_ok[j] = 8 * j + g < p.M;
        const int tok = tok_ok[j] ? 8 * j + g : 0;
        xrow[j] = XSMEM ? xs + tok * p.x_stride + 32 * t  // this lane's 32 columns of chunk c_begin
                        : reinterpret_cast<const uint16_t*>(x) + (int64_t)tok * p.K + kb0 + 32 * t;
    }

    // activations run one k-step pair ahead of their use
    auto lds_x8 = [&](int tt, int off) -> uint4 {
        if (!tok_ok[tt]) return make_uint4(0u, 0u, 0u, 0u);
        const int k = kb0 + 32 * t + off;  // global column of this 8-wide piece
        if constexpr (XSMEM) {
            return *reinterpret_cast<const uint4*>(xrow[tt] + off);
        } else if constexpr (XVEC) {
            return k + 8 <= p.K ? ldg_keep_v4(xrow[tt] + off) : make_uint4(0u, 0u, 0u, 0u);
        } else {
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t lo = k + 2 * j < p.K ? (uint32_t)__ldg(xrow[tt] + off + 2 * j) : 0u;
                const uint32_t hi = k + 2 * j + 1 < p.K ? (uint32_t)__ldg(xrow[tt] + off + 2 * j + 1) : 0u;
                w[j] = lo | (hi << 16);
            }
            return make_uint4(w[0], w[1], w[2], w[3]);
        }
    };
    auto x_at = [&](int m, int col) -> float {  // activation of token m at global column col
        return XSMEM ? ActTraits<T>::bits_to_f32(xs[m * p.x_stride + col - kb0])
                     : ActTraits<T>::to_f32(x[(int64_t)m * p.K + col]);
    };
    // outlier replacement over this rank's K range, done before the main
    // loop so its dependent loads overlap the ring fill instead of trailing
    // it: lanes l and l+16 share tile row l % 16 and take alternate entries
    // of its chunk-CSR range; the sums seed the warp's partial tile
    {
        const int kb = c_begin * kChunk;
        const int ke = min(p.K, c_end * kChunk);
        const int rl = lane & 15;
        const int row = tile_row0 + rl;
        float os[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) os[m] = 0.f;
        if (PREPACKED && o_has) {
            // each batch of four entries is in registers before its
            // activations are read; the next batch loads meanwhile
            const int ib = o_ib;
            for (int i0 = o_ia + (lane >> 4); i0 < ib; i0 += 8) {
                int col[4];
                float d[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    col[u] = ocol[u];
                    d[u] = odl[u];
                }
                if (i0 + 8 < ib) load_outliers(i0 + 8, ib);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    if (col[u] < kb || col[u] >= ke) continue;
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                        if (m < p.M) os[m] += d[u] * x_at(m, col[u]);
                }
            }
        } else if (!PREPACKED && o_has) {
            const int32_t* ro = p.off + (int64_t)row * (p.ncsr + 1);
            int cc = kb / p.chunk_m;
            const int cc_hi = (ke - 1) / p.chunk_m;
            int bound = __ldg(ro + cc + 1);  // end of chunk cc
            const int ib = __ldg(ro + cc_hi + 1);
            for (int i = __ldg(ro + cc) + (lane >> 4); i < ib; i += 2) {
                while (i >= bound) bound = __ldg(ro + (++cc) + 1);  // entries are chunk-ordered
                const int col = cc * p.chunk_m + (int)__ldg(reinterpret_cast<const uint16_t*>(p.ccols) + i);
                if (col < kb || col >= ke) continue;
                const uint32_t sym = (__ldg(p.q + (int64_t)row * p.wpr + (col >> 3)) >> (4 * (col & 7))) & 15u;
                const int grp = GROUPED ? ((col + p.goff) >> p.log2G) : 0;
                const float wl = codebook_value<T, PREPACKED>(p.lut, (int64_t)row * p.ngroups + grp, sym);
                const float d =
                    f16_bits_to_f32(fp8_byte_to_f16_bits(__ldg(reinterpret_cast<const uint8_t*>(p.cvals) + i))) - wl;
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    if (m < p.M) os[m] += d * x_at(m, col);
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) os[m] += __shfl_down_sync(0xFFFFFFFFu, os[m], 16);
        if (lane < 16) {
#pragma unroll
            for (int m = 0; m < MT; ++m) part[warp][rl][m] = os[m];  // the MMA tile is added at publish
        }
        __syncwarp();
    }

    uint4 xnext[NT];
#pragma unroll
    for (int tt = 0; tt < NT; ++tt) xnext[tt] = c_begin < c_end ? lds_x8(tt, 0) : make_uint4(0u, 0u, 0u, 0u);

    // Unchecked activation sources for chunks inside K (16-byte aligned
    // rows): token rows past M read token 0's row, whose products land only
    // in output columns that are never stored.  Shared-memory addresses
    // (XSMEM) or global pointers of this lane's 8-column pieces at chunk
    // c_begin: the lookup's (columns 32t..) and the h MMA's (32w + 8t).
    uint32_t xsa[NT], xfa[NT];
    const uint16_t* xga[NT];
    const uint16_t* xgf[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        const int tok = 8 * j + g < p.M ? 8 * j + g : 0;
        xsa[j] = XSMEM ? smem_u32(xs + tok * p.x_stride + 32 * t) : 0u;
        xfa[j] = XSMEM ? smem_u32(xs + tok * p.x_stride + 32 * hblk + 8 * t) : 0u;
        xga[j] = reinterpret_cast<const uint16_t*>(x) + (int64_t)tok * p.K + kb0 + 32 * t;
        xgf[j] = reinterpret_cast<const uint16_t*>(x) + (int64_t)tok * p.K + kb0 + 32 * hblk + 8 * t;
    }
    // codebook slot offset of this lane's rows within a stage (fixed slots)
    const uint32_t pl_off0 = (uint32_t)(R::kIdxBytes + lane_slot * 32 + g * (kSlots * 32));

    // One chunk: FULL when the chunk and the next one (or none) lie inside
    // K, so that no activation load needs a column check.
    auto chunk = [&](int c, uint32_t base, auto full_tag) {
        constexpr bool FULL = decltype(full_tag)::value;
        const uint32_t cu = (uint32_t)(c - c_begin);
        const uint4 w0 = lds128(base + g * 64 + 16 * t);
        const uint4 w1 = lds128(base + (g + 8) * 64 + 16 * t);
        LutPlanes P0, P1;
        if (GROUPED) {
            uint32_t pb;
            if (cb_fixed) {
                pb = base + pl_off0;
            } else {
                const int s = group_at(c * kChunk + 32 * t) - group_at(c * kChunk);
                pb = base + R::kIdxBytes + s * 32 + g * (NSLOT * 32);
            }
            planes_from_smem<T, PREPACKED>(pb, P0);
            planes_from_smem<T, PREPACKED>(pb + 8 * (kSlots * 32), P1);
        } else {
            P0 = PR0;
            P1 = PR1;
        }
        uint32_t xsc[NT] = {};
        const uint16_t* xgc[NT] = {};
        if constexpr (FULL) {
#pragma unroll
            for (int tt = 0; tt < NT; ++tt) {
                if constexpr (XSMEM) xsc[tt] = mad_u32(cu, 2u * kChunk, xsa[tt]);
                else xgc[tt] = static_cast<const uint16_t*>(ptr_mad(xga[tt], cu, 2u * kChunk));
            }
        }
        const uint32_t ra[4] = {w0.x, w0.y, w0.z, w0.w};
        const uint32_t rb[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int ws = 0; ws < 4; ++ws) {
            uint4 xv[NT];
#pragma unroll
            for (int tt = 0; tt < NT; ++tt) {
                xv[tt] = xnext[tt];
                // next pair: this chunk's ws+1, or the next chunk's first
                if constexpr (FULL) {
                    // byte offsets 16, 32, 48 in this chunk, then the next
                    // chunk's first piece (ws is a constant once unrolled)
                    if (ws == 0) xnext[tt] = x8_at<XSMEM, 16>(xsc[tt], xgc[tt]);
                    else if (ws == 1) xnext[tt] = x8_at<XSMEM, 32>(xsc[tt], xgc[tt]);
                    else if (ws == 2) xnext[tt] = x8_at<XSMEM, 48>(xsc[tt], xgc[tt]);
                    else if (c + 1 < c_end) xnext[tt] = x8_at<XSMEM, 2 * kChunk>(xsc[tt], xgc[tt]);
                } else {
                    const int kn = (c - c_begin) * kChunk + (ws < 3 ? 8 * (ws + 1) : kChunk);
                    if (ws < 3 || c + 1 < c_end) xnext[tt] = lds_x8(tt, kn);
                }
            }
            const uint32_t sa = ra[ws] & 0x77777777u;
            const uint32_t ca = lop_and_or(mulhi(ra[ws], m31), 0x44444444u, 0x32103210u);
            const uint32_t sb = rb[ws] & 0x77777777u;
            const uint32_t cb2 = lop_and_or(mulhi(rb[ws], m31), 0x44444444u, 0x32103210u);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t a[4];
                if (h == 0) {
                    lookup4(P0, sa, ca, a[0], a[2]);
                    lookup4(P1, sb, cb2, a[1], a[3]);
                } else {
                    lookup4(P0, mulhi(sa, m16), mulhi(ca, m16), a[0], a[2]);
                    lookup4(P1, mulhi(sb, m16), mulhi(cb2, m16), a[1], a[3]);
                }
#pragma unroll
                for (int tt = 0; tt < NT; ++tt) {
                    const uint32_t b0 = h ? xv[tt].z : xv[tt].x;
                    const uint32_t b1 = h ? xv[tt].w : xv[tt].y;
                    Mma16816<T>::run(acc[tt], a, b0, b1);
                }
            }
        }
        if (RT > 0 && h_duty(c)) {
            // h += A[:, block] x[block]: lane (g, t) holds columns [8t, 8t+8)
            // of the block for A rows g, g+8 and token g (the k order inside
            // each MMA is the same permutation for both operands)
            const int col = c * kChunk + 32 * hblk + 8 * t;
            uint4 xa[NT];
#pragma unroll
            for (int tt = 0; tt < NT; ++tt) {
                if constexpr (FULL) {
                    if constexpr (XSMEM) xa[tt] = lds128(mad_u32(cu, 2u * kChunk, xfa[tt]));
                    else xa[tt] = ldg_keep_v4(ptr_mad(xgf[tt], cu, 2u * kChunk));
                } else if (!tok_ok[tt] || col >= p.K) {
                    xa[tt] = make_uint4(0u, 0u, 0u, 0u);
                } else if constexpr (XSMEM) {
                    xa[tt] = *reinterpret_cast<const uint4*>(xs + (8 * tt + g) * p.x_stride + (col - kb0));
                } else {
                    xa[tt] = ldg_keep_v4(reinterpret_cast<const uint16_t*>(x) + (int64_t)(8 * tt + g) * p.K + col);
                }
            }
            const uint32_t ab = base + R::kIdxBytes + R::kPlaneBytes;
#pragma unroll
            for (int rt = 0; rt < RT; ++rt) {
                const uint4 a0 = lds128(ab + (16 * rt + g) * 64 + 16 * t);
                const uint4 a8 = lds128(ab + (16 * rt + g + 8) * 64 + 16 * t);
                const uint32_t fa[4] = {a0.x, a8.x, a0.y, a8.y};
                const uint32_t fb[4] = {a0.z, a8.z, a0.w, a8.w};
#pragma unroll
                for (int tt = 0; tt < NT; ++tt) {
                    Mma16816<T>::run(hacc[rt][tt], fa, xa[tt].x, xa[tt].y);
                    Mma16816<T>::run(hacc[rt][tt], fb, xa[tt].z, xa[tt].w);
                }
            }
        }
    };

    int st = 0;
    for (int c = c_begin; c < c_end; ++c) {
        cp_async_wait<S - 2>();  // this lane's copies of chunk c have landed
        __syncwarp();            // ... and every lane's; the previous stage is free
        issue(c + S - 1, st == 0 ? S - 1 : st - 1);
        const uint32_t base = ring + (uint32_t)(st * R::kStageBytes);
        st = st + 1 == S ? 0 : st + 1;
        if ((XVEC || XSMEM) && (c + 1 < c_full || (c + 1 == c_end && c < c_full)))
            chunk(c, base, BoolTag<true>{});
        else
            chunk(c, base, BoolTag<false>{});
    }
    if constexpr (RT > 0) {
        // the warps' partial h [16 RT][MT] meet in their (now idle) rings;
        // each warp then adds s B h for its rows, h in the MMA type
        __syncwarp();  // every lane's last ring reads are done
        float* hmine = reinterpret_cast<float*>(smem + p.x_bytes + warp * S * R::kStageBytes);
#pragma unroll
        for (int rt = 0; rt < RT; ++rt)
#pragma unroll
            for (int tt = 0; tt < NT; ++tt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    hmine[(16 * rt + g) * MT + 8 * tt + 2 * t + e] = hacc[rt][tt][e];
                    hmine[(16 * rt + g + 8) * MT + 8 * tt + 2 * t + e] = hacc[rt][tt][2 + e];
                }
        __syncthreads();
        auto warp_part = [&](int w) {
            return reinterpret_cast<const float*>(smem + p.x_bytes + w * S * R::kStageBytes);
        };
        auto hsum = [&](int k, int tok) -> float {  // s * h[k][tok] over the CTA's K range
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < WARPS; ++w) v += warp_part(w)[k * MT + tok];
            return p.scale * v;
        };
        auto pack = [](float lo, float hi) -> uint32_t {
            const T l = ActTraits<T>::from_f32(lo), h = ActTraits<T>::from_f32(hi);
            return (uint32_t)*reinterpret_cast<const uint16_t*>(&l) |
                   ((uint32_t)*reinterpret_cast<const uint16_t*>(&h) << 16);
        };
#pragma unroll
        for (int rt = 0; rt < RT; ++rt) {
            const int k0 = 16 * rt + 2 * t, k8 = k0 + 8;
#pragma unroll
            for (int tt = 0; tt < NT; ++tt) {
                const int tok = 8 * tt + g;
                const uint32_t b0 = pack(hsum(k0, tok), hsum(k0 + 1, tok));
                const uint32_t b1 = pack(hsum(k8, tok), hsum(k8 + 1, tok));
                Mma16816<T>::run(acc[tt], bfrag[rt], b0, b1);
            }
        }
    }
    // publish this warp's partial tile
#pragma unroll
    for (int tt = 0; tt < NT; ++tt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            part[warp][g][8 * tt + 2 * t + e] += acc[tt][e];
            part[warp][g + 8][8 * tt + 2 * t + e] += acc[tt][2 + e];
        }
    __syncwarp();

    const bool clustered = gridDim.y > 1;
    if (clustered) cluster_sync_all();  // every rank's partial tiles are visible cluster-wide
    const uint32_t rank = clustered ? cluster_ctarank() : 0u;
    const uint32_t nranks = clustered ? cluster_nctarank() : 1u;
    if (p.tp_world > 1) {
        // tiles past N (the grid's last CTA) have no epochs or slots
        if (rank == 0 && tile_row0 < p.N) tp_allreduce_tile<T, MT>(p, part[warp], nranks, tile_row0, lane, gam);
    } else {
        // every rank finishes the tile rows rl with rl % nranks == rank; the
        // sum over ranks is in rank order, so the result does not depend on
        // which rank computes it.  s * B h is already in the tile.
        for (int e = lane; e < kRowsPerTile * MT; e += 32) {
            const int rl = e % kRowsPerTile, tk = e / kRowsPerTile;  // rl == lane % 16
            const int n = tile_row0 + rl;
            if (n >= p.N || tk >= p.M || (uint32_t)rl % nranks != rank) continue;
            const float s = cluster_sum(&part[warp][rl][tk], nranks) * gam;
            reinterpret_cast<T*>(p.out)[(int64_t)tk * p.N + n] = ActTraits<T>::from_f32(s);
        }
    }
    if (clustered) cluster_sync_all();  // keep every rank's tiles alive until all reads are done
}

constexpr int kStages = 3;  // measured: 3 >= 4 > 6 (more stages cost occupancy, not latency)

// One CTA of 16 warps per SM: the whole SM's shared memory holds the
// activations of the CTA's K range (up to 16 tokens x ~3.5K columns) beside
// a 2-stage ring per warp, where 4 CTAs of 4 warps would have to read them
// through L1.  Its 16 warps share one staged copy.
constexpr int kBigWarps = 16;
constexpr int kBigStages = 2;
// shared memory one block may hold (static + dynamic) on sm_100
constexpr size_t kMaxBlockSmem = 227 * 1024;
// static shared memory of the kernel (the per-warp partial tiles)
constexpr size_t gemv_static_smem(int nt, int warps) { return sizeof(float) * warps * kRowsPerTile * 8 * nt; }

// codebook slots a 128-column chunk needs per row: 1 without grouping
// (registers, no slot), 2 for groups of >= 128 columns, 4 for 32 and 64
inline int codebook_slots(int G) { return G == 0 ? 0 : G >= kChunk ? 2 : 4; }

// bytes of one warp's ring stage (host side of Ring<NSLOT, RT>)
inline int ring_stage_bytes(int slots, int rt) { return kRowsPerTile * 64 + kRowsPerTile * slots * 32 + rt * 16 * 64; }

// Clusters of the launch shape `cfg` that the device holds at once (cached
// per kernel, shape and shared memory size; 0 for a non-portable size the
// device refuses).
int clusters_that_fit(const void* kern, const cudaLaunchConfig_t& cfg, int* fit);

// Split forced by wlq_gemv_set_split (0 = chosen per call) and the split of
// this thread's last launch (wlq_gemv_last_split) and its warps per CTA
// (wlq_gemv_last_warps).
extern std::atomic<int> g_forced_split;
// Programmatic dependent launch of the GEMV (wlq_gemv_set_overlap), off by
// default.
extern std::atomic<int> g_overlap;
extern thread_local int g_last_split;
extern thread_local int g_last_warps;

// Returned by a launch whose non-portable cluster size (> 8) the device
// refused (the error is cleared): the caller retries at 8 CTAs or fewer.
constexpr int kRetryPortable = -1;

// The errors with which the runtime refuses a cluster size above the portable
// 8 CTAs (as opposed to a failure of the call itself).
inline bool cluster_size_refused(cudaError_t e) {
    return e == cudaErrorInvalidClusterSize || e == cudaErrorLaunchOutOfResources ||
           e == cudaErrorInvalidValue || e == cudaErrorNotSupported;
}

// Launches one variant; with `fit` set, reports instead how many of its
// clusters the device holds at once (INT_MAX when it runs without clusters).
template <typename T, int NT, int NSLOT, bool PREPACKED, bool XVEC, bool XSMEM, int RT, int STAGES = kStages,
          int WARPS = kWarps>
int launch_variant(const GemvParams& p, int ctas, int cs, cudaStream_t stream, int* fit = nullptr) {
    auto kern = gemv_kernel<T, NT, NSLOT, PREPACKED, XVEC, XSMEM, STAGES, RT, WARPS>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas, (unsigned)cs, 1);
    cfg.blockDim = dim3(WARPS * 32, 1, 1);
    const size_t smem = (size_t)p.x_bytes + (size_t)WARPS * STAGES * Ring<NSLOT, RT>::kStageBytes;
    // the default limit covers static + dynamic shared memory up to 48 KB
    constexpr size_t kStatic = gemv_static_smem(NT, WARPS);
    if (smem + kStatic > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return check_cuda(e, "gemv_kernel smem attribute");
    }
    if (cs > 8) {  // clusters above the portable size of 8
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) {
            if (!cluster_size_refused(e)) return check_cuda(e, "gemv_kernel cluster size attribute");
            cudaGetLastError();
            if (fit) {
                *fit = 0;
                return WLQ_OK;
            }
            return kRetryPortable;
        }
    }
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];  // clusters split K: cs CTAs along y
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)cs;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cs > 1 ? 1 : 0;
    if (fit) {
        if (cfg.numAttrs == 0) {
            *fit = 0x7FFFFFFF;
            return WLQ_OK;
        }
        return clusters_that_fit(reinterpret_cast<const void*>(kern), cfg, fit);
    }
    // Programmatic dependent launch, when the caller opted in
    // (wlq_gemv_set_overlap; measured: 439.0 -> 413.6 us over the 16 decode
    // configurations, every one faster).  The grid may start as soon as every
    // CTA of the previous grid has started (each triggers on entry), so its
    // CTAs only take SM room that grid no longer needs; its weight prologue
    // then runs before the previous kernel's writes are visible, which is why
    // the caller must guarantee that kernel wrote none of this layer's
    // weights.  Not for the fused all-reduce, whose calls must not overlap.
    if (p.tp_world <= 1 && g_overlap.load(std::memory_order_relaxed) != 0) {
        attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
        ++cfg.numAttrs;
    }
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess && cs > 8 && cluster_size_refused(e)) {
        cudaGetLastError();
        return kRetryPortable;
    }
    return check_cuda(e, "gemv_kernel launch");
}

// Launches the kernel that computes h = A x itself (p.loraA, r <= 16 rt,
// rt = 1 or 2; prepacked codebooks and outliers, 16-byte aligned rows).
// Defined in wlq_gemv_fold.cu.
// stages2: a 2-stage ring, which lets the activations of 16 tokens be staged
// beside the larger stages of this kernel.
// big: one 16-warp CTA per SM with the activations staged (kBigWarps; r <= 32
// and at most 16 tokens).
int launch_fold(const GemvParams& p, int rt, bool bf16, bool xsmem, bool stages2, bool big, int ctas, int cs,
                cudaStream_t stream, int* fit = nullptr);

}  // namespace gemv
}  // namespace wlq
