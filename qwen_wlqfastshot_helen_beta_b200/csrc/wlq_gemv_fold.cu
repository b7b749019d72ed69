// Instantiations of the decode GEMV that computes the DoRA low-rank input
// h = A x itself (RT = 1 for r <= 16, 2 for r <= 32, 3 for r <= 48): the
// F.linear(x, A) and
// .float() launches that precede every reference GEMV
// (vllm_wlq/linear_method.py:962-963) folded into the one kernel.  Prepacked
// codebooks and outliers and 16-byte aligned rows only, as the load path
// always produces; kept in their own translation unit so the two halves of
// the GEMV compile in parallel.
#include "wlq_gemv_kernel.cuh"

namespace wlq {
namespace gemv {

namespace {

template <typename T, int NT, int NSLOT>
int fold_x(const GemvParams& p, int rt, bool xsmem, bool stages2, bool big, int ctas, int cs, cudaStream_t stream,
           int* fit) {
    if (big) {  // one 16-warp CTA per SM, activations staged (r <= 32)
        if (rt == 1) return launch_variant<T, NT, NSLOT, true, true, true, 1, kBigStages, kBigWarps>(p, ctas, cs,
                                                                                                      stream, fit);
        return launch_variant<T, NT, NSLOT, true, true, true, 2, kBigStages, kBigWarps>(p, ctas, cs, stream, fit);
    }
    if (rt == 3)  // r <= 48 (a fused qkv of three rank-16 adapters): always a 2-stage ring
        return xsmem ? launch_variant<T, NT, NSLOT, true, true, true, 3, 2>(p, ctas, cs, stream, fit)
                     : launch_variant<T, NT, NSLOT, true, true, false, 3, 2>(p, ctas, cs, stream, fit);
    if constexpr (NT == 2) {
        if (stages2 && xsmem)  // 16 tokens staged beside a 2-stage ring
            return rt == 1 ? launch_variant<T, NT, NSLOT, true, true, true, 1, 2>(p, ctas, cs, stream, fit)
                           : launch_variant<T, NT, NSLOT, true, true, true, 2, 2>(p, ctas, cs, stream, fit);
    }
    if (rt == 1)
        return xsmem ? launch_variant<T, NT, NSLOT, true, true, true, 1>(p, ctas, cs, stream, fit)
                     : launch_variant<T, NT, NSLOT, true, true, false, 1>(p, ctas, cs, stream, fit);
    return xsmem ? launch_variant<T, NT, NSLOT, true, true, true, 2>(p, ctas, cs, stream, fit)
                 : launch_variant<T, NT, NSLOT, true, true, false, 2>(p, ctas, cs, stream, fit);
}

template <typename T, int NT>
int fold_slots(const GemvParams& p, int rt, bool xsmem, bool stages2, bool big, int ctas, int cs,
               cudaStream_t stream, int* fit) {
    switch (codebook_slots(p.G)) {
        case 0: return fold_x<T, NT, 0>(p, rt, xsmem, stages2, big, ctas, cs, stream, fit);
        case 2: return fold_x<T, NT, 2>(p, rt, xsmem, stages2, big, ctas, cs, stream, fit);
        default: return fold_x<T, NT, 4>(p, rt, xsmem, stages2, big, ctas, cs, stream, fit);
    }
}

// 17..32 tokens: rank <= 16 only
template <typename T>
int fold32(const GemvParams& p, bool xsmem, int ctas, int cs, cudaStream_t stream, int* fit) {
    switch (codebook_slots(p.G)) {
        case 0:
            return xsmem ? launch_variant<T, 4, 0, true, true, true, 1>(p, ctas, cs, stream, fit)
                         : launch_variant<T, 4, 0, true, true, false, 1>(p, ctas, cs, stream, fit);
        case 2:
            return xsmem ? launch_variant<T, 4, 2, true, true, true, 1>(p, ctas, cs, stream, fit)
                         : launch_variant<T, 4, 2, true, true, false, 1>(p, ctas, cs, stream, fit);
        default:
            return xsmem ? launch_variant<T, 4, 4, true, true, true, 1>(p, ctas, cs, stream, fit)
                         : launch_variant<T, 4, 4, true, true, false, 1>(p, ctas, cs, stream, fit);
    }
}

template <typename T>
int fold_tokens(const GemvParams& p, int rt, bool xsmem, bool stages2, bool big, int ctas, int cs,
                cudaStream_t stream, int* fit) {
    if (p.M > 16) return fold32<T>(p, xsmem, ctas, cs, stream, fit);
    return p.M <= 8 ? fold_slots<T, 1>(p, rt, xsmem, false, big, ctas, cs, stream, fit)
                    : fold_slots<T, 2>(p, rt, xsmem, stages2, big, ctas, cs, stream, fit);
}

}  // namespace

int launch_fold(const GemvParams& p, int rt, bool bf16, bool xsmem, bool stages2, bool big, int ctas, int cs,
                cudaStream_t stream, int* fit) {
    return bf16 ? fold_tokens<__nv_bfloat16>(p, rt, xsmem, stages2, big, ctas, cs, stream, fit)
                : fold_tokens<__half>(p, rt, xsmem, stages2, big, ctas, cs, stream, fit);
}

}  // namespace gemv
}  // namespace wlq
