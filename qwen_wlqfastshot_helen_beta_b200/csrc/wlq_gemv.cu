// Decode GEMV for M = 1..32 token rows over 4-bit LUT-quantised weights, with
// outlier replacement and the DoRA epilogue fused.  Replaces
// gemv_chunk_csr_kernel + reduce_split_k_dora_kernel
// (csrc/gemv_kernel.cu:86-353) and, for 2 <= M <= 16, the wmma kernel
// (csrc/gemm_kernel.cu:32-294).
//
// HBM-bound: 0.5 B of indices per weight (+0.25 B with 128-wide per-group
// codebooks).  On B200 the integer/logic pipe retires 64 lanes per clock per
// SM, so the lookup must stay near 2 such instructions per weight:
//  * the tensor core does the multiply-accumulate: weights are the A operand
//    of mma.m16n8k16 (16 output rows x 16 k), tokens the 8-wide B operand;
//  * the codebook lookup runs in registers through byte permutes (LutPlanes):
//    8 permutes per 4 weights plus 2 logic ops per 8; the shifts that feed
//    the upper index halves run as mul.hi on the FMA pipe;
//  * codebooks arrive as byte planes already in the MMA type ("prepacked",
//    wlq_prepack_lut) so the hot loop never converts or rebuilds them; the
//    reference fp16 layout is accepted too and rebuilt per lane;
//  * the A fragment's k order is free (the same permutation is applied to x):
//    lane (g, t) owns rows g and g+8 and the 32 consecutive columns
//    [32t, 32t+32) of every 128-wide chunk, i.e. 16 contiguous bytes of each
//    of its rows per chunk;
//  * index words and codebooks stream through a per-warp shared-memory ring
//    filled with cp.async (kStages chunks in flight): prefetches hold no
//    registers or scoreboards, and a chunk is read with one 128-bit shared
//    load per row;
//  * the CTA stages its K range of the activations in shared memory once
//    (cp.async) when it fits, so the B fragments are short-latency loads:
//    4-warp CTAs (4 per SM) where that fits beside their rings, else one
//    16-warp CTA per SM that holds up to ~112 KB of activations for all its
//    warps (also where neither shape splits K);
//  * each warp owns a 16-row tile; K is split only across the CTAs of a
//    thread-block cluster, whose partial tiles meet in distributed shared
//    memory: no global workspace, no second launch;
//  * with wlq_gemv_set_overlap on, a launch is a programmatic dependent
//    launch: it reads only weights before griddepcontrol.wait.
// Outliers REPLACE the codebook weight (csrc/gemm_kernel.cu:204-228).  Before
// the MMA loop, so that its dependent loads overlap the ring's first chunks,
// each warp adds (w_outlier - w_codebook) * x for the outliers of its tile
// (the arithmetic of csrc/gemv_kernel.cu:262-288): two lanes per row walk the
// row's chunk-CSR entries, accumulate in registers and combine with one
// shuffle, seeding the warp's partial tile.
#include <atomic>
#include <mutex>
#include <utility>
#include <vector>

#include "wlq_gemv_kernel.cuh"

namespace wlq {

using namespace gemv;

namespace {

template <typename T, int NT, int NSLOT, bool PREPACKED>
int dispatch_x(const GemvParams& p, bool xvec, bool xsmem, int ctas, int cs, cudaStream_t stream, int* fit) {
    if (xsmem)
        return xvec ? launch_variant<T, NT, NSLOT, PREPACKED, true, true, 0>(p, ctas, cs, stream, fit)
                    : launch_variant<T, NT, NSLOT, PREPACKED, false, true, 0>(p, ctas, cs, stream, fit);
    return xvec ? launch_variant<T, NT, NSLOT, PREPACKED, true, false, 0>(p, ctas, cs, stream, fit)
                : launch_variant<T, NT, NSLOT, PREPACKED, false, false, 0>(p, ctas, cs, stream, fit);
}

template <typename T, int NT, int NSLOT>
int dispatch_fmt(const GemvParams& p, bool prepacked, bool xvec, bool xsmem, int ctas, int cs, cudaStream_t stream,
                 int* fit) {
    return prepacked ? dispatch_x<T, NT, NSLOT, true>(p, xvec, xsmem, ctas, cs, stream, fit)
                     : dispatch_x<T, NT, NSLOT, false>(p, xvec, xsmem, ctas, cs, stream, fit);
}

template <typename T, int NT>
int dispatch_slots(const GemvParams& p, bool prepacked, bool xvec, bool xsmem, int ctas, int cs,
                   cudaStream_t stream, int* fit) {
    switch (codebook_slots(p.G)) {
        case 0: return dispatch_fmt<T, NT, 0>(p, prepacked, xvec, xsmem, ctas, cs, stream, fit);
        case 2: return dispatch_fmt<T, NT, 2>(p, prepacked, xvec, xsmem, ctas, cs, stream, fit);
        default: return dispatch_fmt<T, NT, 4>(p, prepacked, xvec, xsmem, ctas, cs, stream, fit);
    }
}

// 17..32 tokens (four 8-token MMA tiles): prepacked layout, 16-byte rows
template <typename T>
int dispatch32(const GemvParams& p, bool xsmem, int ctas, int cs, cudaStream_t stream, int* fit) {
    switch (codebook_slots(p.G)) {
        case 0:
            return xsmem ? launch_variant<T, 4, 0, true, true, true, 0>(p, ctas, cs, stream, fit)
                         : launch_variant<T, 4, 0, true, true, false, 0>(p, ctas, cs, stream, fit);
        case 2:
            return xsmem ? launch_variant<T, 4, 2, true, true, true, 0>(p, ctas, cs, stream, fit)
                         : launch_variant<T, 4, 2, true, true, false, 0>(p, ctas, cs, stream, fit);
        default:
            return xsmem ? launch_variant<T, 4, 4, true, true, true, 0>(p, ctas, cs, stream, fit)
                         : launch_variant<T, 4, 4, true, true, false, 0>(p, ctas, cs, stream, fit);
    }
}

// one 16-warp CTA per SM with the activations staged: prepacked layout,
// 16-byte aligned rows, at most 16 tokens
template <typename T, int NT>
int dispatch_big(const GemvParams& p, int ctas, int cs, cudaStream_t stream, int* fit) {
    switch (codebook_slots(p.G)) {
        case 0: return launch_variant<T, NT, 0, true, true, true, 0, kBigStages, kBigWarps>(p, ctas, cs, stream, fit);
        case 2: return launch_variant<T, NT, 2, true, true, true, 0, kBigStages, kBigWarps>(p, ctas, cs, stream, fit);
        default: return launch_variant<T, NT, 4, true, true, true, 0, kBigStages, kBigWarps>(p, ctas, cs, stream, fit);
    }
}

template <typename T>
int dispatch(const GemvParams& p, bool prepacked, bool xvec, bool xsmem, bool big, int ctas, int cs,
             cudaStream_t stream, int* fit) {
    if (big)
        return p.M <= 8 ? dispatch_big<T, 1>(p, ctas, cs, stream, fit) : dispatch_big<T, 2>(p, ctas, cs, stream, fit);
    if (p.M > 16) return dispatch32<T>(p, xsmem, ctas, cs, stream, fit);
    return p.M <= 8 ? dispatch_slots<T, 1>(p, prepacked, xvec, xsmem, ctas, cs, stream, fit)
                    : dispatch_slots<T, 2>(p, prepacked, xvec, xsmem, ctas, cs, stream, fit);
}

// One launch shape: K split over cs CTAs; activations staged in shared
// memory or read through L1.
struct Plan {
    int cs;
    bool xsmem, stages2;
    bool big;  // one 16-warp CTA per SM (kBigWarps) instead of 4-warp CTAs
};

struct FitKey {
    const void* kern;
    unsigned cx, cy;
    size_t smem;
    int dev;
};

}  // namespace

namespace gemv {

std::atomic<int> g_forced_split{0};
std::atomic<int> g_overlap{0};
thread_local int g_last_split = 0;
thread_local int g_last_warps = 0;

int clusters_that_fit(const void* kern, const cudaLaunchConfig_t& cfg, int* fit) {
    static std::mutex mu;
    static std::vector<std::pair<FitKey, int>> cache;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return check_cuda(e, "cudaGetDevice");
    const FitKey key{kern, cfg.attrs[0].val.clusterDim.x, cfg.attrs[0].val.clusterDim.y, cfg.dynamicSmemBytes, dev};
    std::lock_guard<std::mutex> lock(mu);
    for (const auto& kv : cache)
        if (kv.first.kern == key.kern && kv.first.cx == key.cx && kv.first.cy == key.cy &&
            kv.first.smem == key.smem && kv.first.dev == key.dev) {
            *fit = kv.second;
            return WLQ_OK;
        }
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess) {
        // a cluster size the device or driver does not run: none fits; the
        // refusal is cached, so the query runs once per shape
        if (key.cy <= 8 || !cluster_size_refused(e)) return check_cuda(e, "cudaOccupancyMaxActiveClusters");
        cudaGetLastError();  // clears this call's (non-sticky) error only
        n = 0;
    }
    cache.emplace_back(key, n);
    *fit = n;
    return WLQ_OK;
}

}  // namespace gemv

int launch_gemv(const LinearArgs& a, cudaStream_t stream) {
    if (a.M == 0 || a.N == 0) return WLQ_OK;
    if (a.M > kMaxGemvM) return fail(WLQ_ERR_INVALID_ARG, "wlq_gemv: M must be <= %d, got %d", kMaxGemvM, a.M);
    if (a.M > 16 && (!a.lut_prepacked || a.K % 8 != 0 || (reinterpret_cast<uintptr_t>(a.x) & 15) != 0))
        return fail(WLQ_ERR_UNSUPPORTED, "wlq_gemv: 17..%d tokens need the prepacked layout and 16-byte aligned rows",
                    kMaxGemvM);
    int log2G = 0;
    if (a.group_size > 0) {
        while ((1 << log2G) < a.group_size) ++log2G;
        if ((1 << log2G) != a.group_size || a.group_size < 32 || a.group_offset % 32 != 0)
            return fail(WLQ_ERR_UNSUPPORTED,
                        "wlq_gemv: per-group codebooks need a power-of-two group_size >= 32 and a group_offset "
                        "multiple of 32 (got %d, %d)", a.group_size, a.group_offset);
    }
    GemvParams p;
    p.q = a.q; p.lut = a.lut; p.x = a.x; p.out = a.out;
    p.off = a.off; p.ccols = a.ccols; p.cvals = a.cvals;
    p.loraB = a.loraB; p.lorah = a.lorah; p.loraA = a.loraA; p.gamma = a.gamma; p.scale = a.scale; p.r = a.r;
    p.M = a.M; p.N = a.N; p.K = a.K; p.wpr = a.wpr; p.G = a.group_size; p.goff = a.group_offset;
    p.ngroups = a.ngroups; p.chunk_m = a.chunk_m; p.ncsr = a.ncsr;
    p.log2G = log2G;
    p.kchunks = (a.K + kChunk - 1) / kChunk;
    p.mul16 = 1u << 16;
    p.mul31 = 1u << 31;
    p.tp_world = a.tp_world;
    p.tp_rank = a.tp_rank;
    p.tp_nmax = a.tp_nmax;
    if (a.tp_world > 1) {
        const TpLayout l = tp_layout(a.tp_world, a.tp_nmax);
        p.tp_stride = l.stride;
        for (int q = 0; q < a.tp_world; ++q) {
            char* b = static_cast<char*>(a.tp_bufs[q]);
            p.tp_data[q] = reinterpret_cast<unsigned long long*>(b + l.data);
        }
        char* mine = static_cast<char*>(a.tp_bufs[a.tp_rank]);
        p.tp_counters = reinterpret_cast<uint32_t*>(mine + l.counters);
        p.tp_err = reinterpret_cast<uint32_t*>(mine + l.err);
    }
    const bool xvec = (a.K % 8 == 0) && ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0);
    // h = A x in the kernel: r <= 16 rt
    const int rt = a.loraA != nullptr && a.r > 0 ? (a.r + 15) / 16 : 0;
    if (rt > 0) {
        if (a.r > 48) return fail(WLQ_ERR_UNSUPPORTED, "wlq_gemv: h = A x in the kernel needs r <= 48 (r=%d)", a.r);
        if (a.M > 16 && a.r > 16)
            return fail(WLQ_ERR_UNSUPPORTED, "wlq_gemv: h = A x in the kernel for more than 16 tokens needs r <= 16");
        if (!a.lut_prepacked)
            return fail(WLQ_ERR_UNSUPPORTED, "wlq_gemv: h = A x in the kernel needs the prepacked layout");
        if (!xvec || (reinterpret_cast<uintptr_t>(a.loraA) & 15) != 0)
            return fail(WLQ_ERR_ALIGNMENT, "wlq_gemv: h = A x in the kernel needs K %% 8 == 0 and 16-byte aligned "
                        "x and lora_A");
    }
    const bool bf16 = a.dtype == WLQ_DTYPE_BF16;
    const int tiles = (a.N + kRowsPerTile - 1) / kRowsPerTile;
    const int ctas4 = (tiles + kWarps - 1) / kWarps;
    const int ctas16 = (tiles + kBigWarps - 1) / kBigWarps;
    const int slots = codebook_slots(p.G);
    // r <= 48 (rt = 3) always runs a 2-stage ring: three stages of its larger
    // A blocks would leave no room for 4 CTAs per SM
    const int stages = rt == 3 ? 2 : kStages;
    const int ring_bytes = kWarps * stages * ring_stage_bytes(slots, rt);
    // one 16-warp CTA per SM: prepacked layout, 16-byte aligned rows, at most
    // 16 tokens and r <= 32
    const bool big_ok = a.lut_prepacked && xvec && a.M <= 16 && rt <= 2;
    const size_t big_fixed = (size_t)kBigWarps * kBigStages * ring_stage_bytes(slots, rt) +
                             gemv_static_smem(a.M <= 8 ? 1 : 2, kBigWarps);

    auto configure = [&](int cs, bool big) {
        Plan pl;
        pl.cs = cs;
        pl.big = big;
        p.chunks_per_rank = (p.kchunks + cs - 1) / cs;
        p.x_stride = p.chunks_per_rank * kChunk + 8;
        const int64_t x_bytes = ((int64_t)a.M * p.x_stride * 2 + 127) / 128 * 128;
        if (big) {  // the activations must fit beside the 16 rings
            pl.xsmem = (size_t)x_bytes + big_fixed <= kMaxBlockSmem;
            pl.stages2 = false;
            p.x_bytes = pl.xsmem ? (int)x_bytes : 0;
            return pl;
        }
        // stage the rank's activations in shared memory when 4 CTAs per SM
        // still fit beside the rings; larger slices are read through L1.
        // Computing h (larger stages) for 9..16 tokens, a 2-stage ring when
        // that lets the activations be staged.
        pl.xsmem = x_bytes + ring_bytes <= 48 * 1024;
        pl.stages2 = rt == 3 ||
                     (rt > 0 && a.M > 8 && !pl.xsmem && x_bytes + ring_bytes / kStages * 2 <= 48 * 1024);
        if (rt != 3) pl.xsmem = pl.xsmem || pl.stages2;
        p.x_bytes = pl.xsmem ? (int)x_bytes : 0;
        return pl;
    };
    auto run = [&](const Plan& pl, int* fit) {
        const int ctas = pl.big ? ctas16 : ctas4;
        if (rt > 0) return launch_fold(p, rt, bf16, pl.xsmem, pl.stages2, pl.big, ctas, pl.cs, stream, fit);
        return bf16 ? dispatch<__nv_bfloat16>(p, a.lut_prepacked, xvec, pl.xsmem, pl.big, ctas, pl.cs, stream, fit)
                    : dispatch<__half>(p, a.lut_prepacked, xvec, pl.xsmem, pl.big, ctas, pl.cs, stream, fit);
    };

    // Split K over a cluster (up to 16 CTAs) until about 16 warps per SM are
    // in flight (4 CTAs of 4 warps, or one of 16), keeping at least 2 chunks
    // per rank, and at least 4 above 8 ranks (measured: a 14-way split of 28
    // chunks lost to the wider reduction, a 16-way split of 148 won 15 %);
    // then take the largest split (down to none) whose clusters the device
    // holds in one wave.  4-warp CTAs first; where their activations would
    // have to come through L1, 16-warp CTAs that stage them instead.  A split
    // forced through wlq_gemv_set_split replaces the choice.
    const int forced = g_forced_split.load(std::memory_order_relaxed);
    const int sms = device_sm_count();
    auto chunks_ok = [&](int cs) { return p.kchunks >= (cs > 8 ? 4 : 2) * cs; };
    auto search = [&](bool big, Plan& out) {
        const int ctas = big ? ctas16 : ctas4;
        const int64_t target = big ? (int64_t)sms : 4LL * sms;
        int cs_max = 1;
        while (cs_max < kMaxSplit && (int64_t)ctas * cs_max < target && chunks_ok(cs_max + 1)) ++cs_max;
        out = configure(1, big);
        for (int cs = cs_max; cs > 1; --cs) {
            const Plan c = configure(cs, big);
            if (big && !c.xsmem) continue;
            int fit = 0;
            const int rc = run(c, &fit);  // a refused non-portable size reports fit = 0 (cached)
            if (rc) return rc;
            if (ctas <= fit) {
                out = c;
                break;
            }
        }
        return (int)WLQ_OK;
    };
    Plan pl;
    if (forced > 0) {
        if (forced > kMaxSplit || forced > p.kchunks)
            return fail(WLQ_ERR_INVALID_ARG, "wlq_gemv: forced split %d needs 1..%d and at most %d chunks of 128 "
                        "columns", forced, kMaxSplit, p.kchunks);
        pl = configure(forced, false);
        if (!pl.xsmem && big_ok) {
            const Plan b = configure(forced, true);
            if (b.xsmem) pl = b;
        }
    } else {
        int rc = search(false, pl);
        if (rc) return rc;
        // measured: 16-warp CTAs also win where neither shape splits K
        // (gate_up at M = 1: 43.4 -> 41.2 us), and lose where both split it
        if (big_ok && (!pl.xsmem || pl.cs == 1)) {
            Plan b;
            rc = search(true, b);
            if (rc) return rc;
            if (b.xsmem && (!pl.xsmem || b.cs == 1)) pl = b;
        }
    }
    configure(pl.cs, pl.big);
    int rc = run(pl, nullptr);
    if (rc == kRetryPortable && forced == 0) {
        // the launch refused a non-portable cluster size: once more at 8 CTAs
        // or fewer (4-warp CTAs when the 16-warp ones cannot stage that slice)
        int cs = pl.cs > 8 ? 8 : pl.cs;
        while (cs > 1 && p.kchunks < 2 * cs) --cs;
        pl = configure(cs, pl.big);
        if (pl.big && !pl.xsmem) pl = configure(cs, false);
        rc = run(pl, nullptr);
    }
    if (rc == kRetryPortable)
        return fail(WLQ_ERR_CUDA, "wlq_gemv: the device refused a cluster of %d CTAs", pl.cs);
    if (rc == WLQ_OK) {
        g_last_split = pl.cs;
        g_last_warps = pl.big ? kBigWarps : kWarps;
    }
    return rc;
}

}  // namespace wlq

extern "C" {

int wlq_gemv_set_split(int cs) {
    if (cs < 0 || cs > wlq::gemv::kMaxSplit)
        return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_gemv_set_split: %d is outside 0..%d", cs, wlq::gemv::kMaxSplit);
    wlq::gemv::g_forced_split.store(cs, std::memory_order_relaxed);
    return WLQ_OK;
}

int wlq_gemv_last_split(void) { return wlq::gemv::g_last_split; }

int wlq_gemv_last_warps(void) { return wlq::gemv::g_last_warps; }

int wlq_gemv_set_overlap(int on) {
    if (on != 0 && on != 1) return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_gemv_set_overlap: expected 0 or 1, got %d", on);
    wlq::gemv::g_overlap.store(on, std::memory_order_relaxed);
    return WLQ_OK;
}

int wlq_gemv_get_overlap(void) { return wlq::gemv::g_overlap.load(std::memory_order_relaxed); }

}  // extern "C"
