// Load-time host codecs of libwlq_b200.so: index repacking, Elias-Fano and
// mask outlier decoding to chunk-CSR, fp16 -> e5m2 bytes, and a host
// dequantiser for computing the DoRA scale without a GPU.  These run once per
// layer at load time (the reference's csrc/vllm_binding.cpp:82-236 and the
// numpy paths of vllm_wlq/linear_method.py:186-338); nothing here is on the
// forward path.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/wlq_b200.h"

namespace wlq {
int fail(int code, const char* fmt, ...);
}

namespace {

inline int64_t spw_of(int bits) { return bits == 3 ? 10 : 32 / bits; }

inline int64_t wpr_of(int64_t K, int bits) {
    const int64_t spw = spw_of(bits);
    return ((K + spw - 1) / spw + 3) / 4 * 4;
}

// Reads symbol `i` of a continuous stream (0 past its end).
inline uint32_t stream_symbol(const uint32_t* src, int64_t n_src, int64_t i, int bits, int64_t spw) {
    const int64_t w = i / spw;
    if (w >= n_src) return 0u;
    return (src[w] >> (uint32_t)(bits * (i - w * spw))) & ((1u << bits) - 1u);
}

// Sub-matrix [r0,r1) x [c0,c1) of the continuous [N_full, K_full] stream into
// row-aligned words.
void repack_slice(const uint32_t* src, int64_t n_src, int64_t K_full, int bits, int64_t r0, int64_t r1, int64_t c0,
                  int64_t c1, uint32_t* dst) {
    const int64_t spw = spw_of(bits);
    const int64_t K = c1 - c0;
    const int64_t wpr = wpr_of(K, bits);
    const int64_t rows = r1 - r0;
    std::memset(dst, 0, (size_t)(rows * wpr) * sizeof(uint32_t));
    // fast path: 4-bit rows that start on a word boundary of the stream
    const bool word_aligned = bits == 4 && ((K_full % 8) == 0) && ((c0 % 8) == 0);
    for (int64_t r = 0; r < rows; ++r) {
        uint32_t* out = dst + r * wpr;
        const int64_t base = (r0 + r) * K_full + c0;
        if (word_aligned) {
            const int64_t w0 = base / 8;
            const int64_t full = K / 8;
            for (int64_t w = 0; w < full; ++w) out[w] = (w0 + w) < n_src ? src[w0 + w] : 0u;
            for (int64_t k = full * 8; k < K; ++k)
                out[k / 8] |= stream_symbol(src, n_src, base + k, 4, 8) << (uint32_t)(4 * (k % 8));
            continue;
        }
        for (int64_t k = 0; k < K; ++k)
            out[k / spw] |= stream_symbol(src, n_src, base + k, bits, spw) << (uint32_t)(bits * (k % spw));
    }
}

inline uint32_t read_bits(const uint32_t* d, int64_t nw, int64_t pos, int n) {
    if (n <= 0) return 0u;
    const int64_t w = pos >> 5;
    if (w >= nw) return 0u;
    const int o = (int)(pos & 31);
    uint64_t v = (uint64_t)d[w] >> o;
    if (n > 32 - o && w + 1 < nw) v |= (uint64_t)d[w + 1] << (32 - o);
    return (uint32_t)(v & ((1ull << n) - 1ull));
}

// Decodes every EF tile, calling emit(row, col) in tile order and, within a
// tile, in increasing position.  Matches csrc/vllm_binding.cpp:130-167,
// including its handling of a stream that ends early (the remaining elements
// keep the last high part).
template <typename Emit>
void ef_walk(const int64_t* meta, int64_t n_tiles, const uint32_t* bs, int64_t n_words, int64_t tile,
             int64_t tiles_x, Emit&& emit) {
    const int64_t U = tile * tile;
    const int64_t nbits = n_words * 32;
    for (int64_t t = 0; t < n_tiles; ++t) {
        const int64_t start = meta[2 * t];
        const int64_t m = meta[2 * t + 1];
        if (m <= 0) continue;
        int L = 0;
        if (U > m) {
            L = (int)std::floor(std::log2((double)U / (double)m));
            if (L < 0) L = 0;
        }
        const int64_t br = (t / tiles_x) * tile, bc = (t % tiles_x) * tile;
        int64_t cur = start + m * L;
        int64_t high = 0;
        for (int64_t i = 0; i < m; ++i) {
            const uint32_t low = L > 0 ? read_bits(bs, n_words, start + i * L, L) : 0u;
            // skip zeros a word at a time, stop after the terminating one
            while (cur < nbits) {
                const uint32_t word = bs[cur >> 5] >> (cur & 31);
                const int avail = 32 - (int)(cur & 31);
                if (word == 0u) {
                    high += avail;
                    cur += avail;
                    continue;
                }
                const int z = __builtin_ctz(word);
                high += z;
                cur += z + 1;
                break;
            }
            const int64_t local = (high << L) | (int64_t)low;
            emit(br + local / tile, bc + local % tile);
        }
    }
}

// Row-ordered (row, col) outlier positions -> chunk-CSR with a counting pass;
// positions of one row must arrive in increasing column order.
template <typename Pos>
int64_t positions_to_csr(const Pos& pos, int64_t n, int64_t N, int64_t K, int64_t chunk_m, int32_t* offsets,
                         uint16_t* cols) {
    const int64_t nc = (K + chunk_m - 1) / chunk_m;
    std::vector<int64_t> cnt((size_t)(N * nc), 0);
    for (int64_t i = 0; i < n; ++i) {
        int64_t r, c;
        pos(i, r, c);
        cnt[(size_t)(r * nc + c / chunk_m)]++;
    }
    int64_t run = 0;
    for (int64_t r = 0; r < N; ++r) {
        offsets[r * (nc + 1)] = (int32_t)run;
        for (int64_t c = 0; c < nc; ++c) {
            const int64_t k = cnt[(size_t)(r * nc + c)];
            cnt[(size_t)(r * nc + c)] = run;  // becomes the fill cursor
            run += k;
            offsets[r * (nc + 1) + c + 1] = (int32_t)run;
        }
    }
    if (cols) {
        for (int64_t i = 0; i < n; ++i) {
            int64_t r, c;
            pos(i, r, c);
            cols[cnt[(size_t)(r * nc + c / chunk_m)]++] = (uint16_t)(c % chunk_m);
        }
    }
    return run;
}

}  // namespace

extern "C" {

int64_t wlq_words_per_row(int64_t K, int bits) {
    if (bits < 1 || bits > 4 || K < 0) return -1;
    return wpr_of(K, bits);
}

int wlq_repack_q_indices_row_aligned(const int32_t* src, int64_t n_src, int64_t N, int64_t K, int bits, int32_t* dst,
                                     int64_t dst_capacity, int64_t* words_per_row) {
    if (bits < 1 || bits > 4 || N < 0 || K < 0 || n_src < 0)
        return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_repack_q_indices_row_aligned: bad arguments");
    const int64_t wpr = wpr_of(K, bits);
    if (words_per_row) *words_per_row = wpr;
    if (!dst) return WLQ_OK;
    if (dst_capacity < N * wpr)
        return wlq::fail(WLQ_ERR_CAPACITY, "wlq_repack_q_indices_row_aligned: need %lld words", (long long)(N * wpr));
    repack_slice(reinterpret_cast<const uint32_t*>(src), n_src, K, bits, 0, N, 0, K, reinterpret_cast<uint32_t*>(dst));
    return WLQ_OK;
}

// Rows [r0,r1) x columns [c0,c1) of a continuous [N_full, K_full] stream, for
// the tensor-parallel shard of a layer (vllm_wlq/linear_method.py:724, 753-761, 792).
int wlq_repack_q_indices_slice(const int32_t* src, int64_t n_src, int64_t N_full, int64_t K_full, int bits, int64_t r0,
                               int64_t r1, int64_t c0, int64_t c1, int32_t* dst, int64_t dst_capacity,
                               int64_t* words_per_row) {
    if (bits < 1 || bits > 4 || r0 < 0 || r1 < r0 || r1 > N_full || c0 < 0 || c1 < c0 || c1 > K_full)
        return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_repack_q_indices_slice: bad slice");
    const int64_t wpr = wpr_of(c1 - c0, bits);
    if (words_per_row) *words_per_row = wpr;
    if (!dst) return WLQ_OK;
    if (dst_capacity < (r1 - r0) * wpr) return wlq::fail(WLQ_ERR_CAPACITY, "wlq_repack_q_indices_slice: capacity");
    repack_slice(reinterpret_cast<const uint32_t*>(src), n_src, K_full, bits, r0, r1, c0, c1,
                 reinterpret_cast<uint32_t*>(dst));
    return WLQ_OK;
}

int wlq_decode_ef_to_chunk_csr(const int64_t* tile_meta, int64_t n_tiles, const int32_t* bitstream, int64_t n_words,
                               int64_t N, int64_t K, int64_t tile_size, int64_t chunk_m, int32_t* offsets,
                               uint16_t* cols, int64_t cols_capacity, int64_t* nnz) {
    if (!tile_meta && n_tiles > 0) return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_decode_ef_to_chunk_csr: tile_meta");
    if (N < 0 || K < 0 || tile_size <= 0 || chunk_m <= 0 || chunk_m > 65536 || !offsets)
        return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_decode_ef_to_chunk_csr: bad arguments");
    const int64_t tiles_x = (K + tile_size - 1) / tile_size;
    const uint32_t* bs = reinterpret_cast<const uint32_t*>(bitstream);
    std::vector<int64_t> pos;
    ef_walk(tile_meta, n_tiles, bs, n_words, tile_size, tiles_x, [&](int64_t r, int64_t c) {
        if (r < N && c < K) pos.push_back(r * K + c);
    });
    // tiles are visited band by band, so one row's positions interleave with
    // the other rows of its band: order them (row, col) as the reference does
    std::sort(pos.begin(), pos.end());
    const int64_t n = (int64_t)pos.size();
    if (nnz) *nnz = n;
    if (cols && cols_capacity < n) return wlq::fail(WLQ_ERR_CAPACITY, "wlq_decode_ef_to_chunk_csr: need %lld", (long long)n);
    positions_to_csr([&](int64_t i, int64_t& r, int64_t& c) { r = pos[i] / K; c = pos[i] % K; }, n, N, K, chunk_m,
                     offsets, cols);
    return WLQ_OK;
}

// EF tiles -> sorted flat positions r*K + c (the row-major order of the
// outlier value list), for slicing before the CSR is built
// (vllm_wlq/linear_method.py:243-281).
int wlq_decode_ef_positions(const int64_t* tile_meta, int64_t n_tiles, const int32_t* bitstream, int64_t n_words,
                            int64_t N, int64_t K, int64_t tile_size, int64_t* positions, int64_t capacity,
                            int64_t* count) {
    if ((!tile_meta && n_tiles > 0) || N < 0 || K < 0 || tile_size <= 0)
        return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_decode_ef_positions: bad arguments");
    const int64_t tiles_x = (K + tile_size - 1) / tile_size;
    std::vector<int64_t> pos;
    ef_walk(tile_meta, n_tiles, reinterpret_cast<const uint32_t*>(bitstream), n_words, tile_size, tiles_x,
            [&](int64_t r, int64_t c) {
                if (r < N && c < K) pos.push_back(r * K + c);
            });
    std::sort(pos.begin(), pos.end());
    pos.erase(std::unique(pos.begin(), pos.end()), pos.end());
    if (count) *count = (int64_t)pos.size();
    if (!positions) return WLQ_OK;
    if (capacity < (int64_t)pos.size()) return wlq::fail(WLQ_ERR_CAPACITY, "wlq_decode_ef_positions: capacity");
    std::copy(pos.begin(), pos.end(), positions);
    return WLQ_OK;
}

int wlq_build_chunk_csr(const uint8_t* mask, int64_t N, int64_t K, int64_t chunk_m, int32_t* offsets, uint16_t* cols,
                        int64_t cols_capacity, int64_t* nnz) {
    if ((!mask && N * K > 0) || N < 0 || K < 0 || chunk_m <= 0 || chunk_m > 65536 || !offsets)
        return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_build_chunk_csr: bad arguments");
    int64_t n = 0;
    for (int64_t i = 0; i < N * K; ++i) n += mask[i] != 0;
    if (nnz) *nnz = n;
    if (cols && cols_capacity < n) return wlq::fail(WLQ_ERR_CAPACITY, "wlq_build_chunk_csr: need %lld", (long long)n);
    std::vector<int64_t> pos;
    pos.reserve((size_t)n);
    for (int64_t i = 0; i < N * K; ++i)
        if (mask[i]) pos.push_back(i);
    positions_to_csr([&](int64_t i, int64_t& r, int64_t& c) { r = pos[i] / K; c = pos[i] % K; }, n, N, K, chunk_m,
                     offsets, cols);
    return WLQ_OK;
}

// Sorted flat positions (r*K + c) -> chunk-CSR.
int wlq_positions_to_chunk_csr(const int64_t* positions, int64_t n, int64_t N, int64_t K, int64_t chunk_m,
                               int32_t* offsets, uint16_t* cols) {
    if ((!positions && n > 0) || N < 0 || K <= 0 || chunk_m <= 0 || chunk_m > 65536 || !offsets)
        return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_positions_to_chunk_csr: bad arguments");
    for (int64_t i = 0; i < n; ++i)
        if (positions[i] < 0 || positions[i] >= N * K || (i > 0 && positions[i] <= positions[i - 1]))
            return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_positions_to_chunk_csr: positions must be sorted, unique, in range");
    positions_to_csr([&](int64_t i, int64_t& r, int64_t& c) { r = positions[i] / K; c = positions[i] % K; }, n, N, K,
                     chunk_m, offsets, cols);
    return WLQ_OK;
}

int wlq_fp16_to_fp8_bytes(const uint16_t* src, int64_t n, uint8_t* dst) {
    if ((!src || !dst) && n > 0) return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_fp16_to_fp8_bytes: null pointer");
    for (int64_t i = 0; i < n; ++i) {
        const int32_t v = ((int32_t)src[i] + 0x80) >> 8;
        dst[i] = (uint8_t)(v > 255 ? 255 : v);
    }
    return WLQ_OK;
}

int wlq_dequant_host(const int32_t* q_packed, const uint16_t* lut_c, uint16_t* W_out, const int32_t* chunk_offsets,
                     const uint16_t* chunk_cols, const uint8_t* chunk_vals, int64_t N, int64_t K, int bits,
                     int64_t words_per_row, int64_t lut_group_size, int64_t lut_group_offset) {
    if (bits < 1 || bits > 4 || N < 0 || K < 0 || words_per_row != wpr_of(K, bits) || lut_group_size < 0 ||
        lut_group_offset < 0)
        return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_dequant_host: bad arguments");
    if (N == 0 || K == 0) return WLQ_OK;
    if (!q_packed || !lut_c || !W_out) return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_dequant_host: null pointer");
    const int64_t spw = spw_of(bits);
    const int64_t kcb = (int64_t)1 << bits;
    const uint32_t msk = (1u << bits) - 1u;
    const int64_t ng = lut_group_size > 0 ? (K + lut_group_offset + lut_group_size - 1) / lut_group_size : 1;
    const int64_t chunk_m = bits == 3 ? 640 : 512;
    const int64_t nc = (K + chunk_m - 1) / chunk_m;
    const uint32_t* q = reinterpret_cast<const uint32_t*>(q_packed);
    for (int64_t n = 0; n < N; ++n) {
        const uint32_t* qr = q + n * words_per_row;
        uint16_t* wr = W_out + n * K;
        for (int64_t k = 0; k < K; ++k) {
            const uint32_t s = (qr[k / spw] >> (uint32_t)(bits * (k % spw))) & msk;
            const int64_t g = lut_group_size > 0 ? (k + lut_group_offset) / lut_group_size : 0;
            wr[k] = lut_c[(n * ng + g) * kcb + s];
        }
        if (chunk_offsets && chunk_cols && chunk_vals) {
            for (int64_t c = 0; c < nc; ++c) {
                for (int32_t i = chunk_offsets[n * (nc + 1) + c]; i < chunk_offsets[n * (nc + 1) + c + 1]; ++i) {
                    const int64_t col = c * chunk_m + chunk_cols[i];
                    if (col < K) wr[col] = (uint16_t)((uint16_t)chunk_vals[i] << 8);
                }
            }
        }
    }
    return WLQ_OK;
}

}  // extern "C"

namespace {
// IEEE-754 binary16 -> binary32 (exact) and binary32 -> bfloat16 (round to
// nearest even), from the formats' bit layouts.
float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        float v = std::ldexp((float)man, -24);
        std::memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (ex == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex + 112u) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}
uint16_t f32_to_bf16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    if ((x & 0x7F800000u) == 0x7F800000u && (x & 0x7FFFFFu)) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}
}  // namespace

extern "C" int wlq_prepack_lut_host(const uint16_t* lut_c, uint16_t* lut_out, int64_t n_codebooks, int act_dtype) {
    if (n_codebooks < 0 || (n_codebooks > 0 && (!lut_c || !lut_out)) ||
        (act_dtype != WLQ_DTYPE_F16 && act_dtype != WLQ_DTYPE_BF16))
        return wlq::fail(WLQ_ERR_INVALID_ARG, "wlq_prepack_lut_host: bad arguments");
    for (int64_t i = 0; i < n_codebooks; ++i) {
        uint16_t e[16];
        for (int k = 0; k < 16; ++k) {
            const uint16_t v = lut_c[i * 16 + k];
            e[k] = act_dtype == WLQ_DTYPE_BF16 ? f32_to_bf16(f16_to_f32(v)) : v;
        }
        uint8_t* o = reinterpret_cast<uint8_t*>(lut_out + i * 16);
        for (int k = 0; k < 16; ++k) {
            o[k] = (uint8_t)(e[k] & 0xFFu);        // lo planes: entry k at byte k
            o[16 + k] = (uint8_t)(e[k] >> 8);      // hi planes
        }
    }
    return WLQ_OK;
}
