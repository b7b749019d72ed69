/*
 * wlq_oracle.c -- CPU restatement of the reference's WLQ linear-method arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product path (the package, its
 * CUDA kernels, its C ABI) may link, load or call this file.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs
 * use it, and there only as the checker.
 *
 * Every function names the reference file:line whose behaviour it restates
 * (paths are relative to the reference project root).  Integer and byte work
 * is bit-exact; the layer forward is evaluated in double precision.
 *
 * Pinned against golden vectors produced by the reference's own Python code
 * (tests/golden/make_golden.py) and, on the GPU box, against the reference's
 * own CUDA kernels compiled from source (oracle/build_ref.sh).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

/* ------------------------------------------------------------------------ */
/* IEEE-754 binary16 / bfloat16 conversions, written from the format spec.   */
/* ------------------------------------------------------------------------ */

float orc_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    const uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        /* zero or subnormal: value = man * 2^-24, exact in binary32 */
        float v = ldexpf((float)man, -24);
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
    const int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        const uint32_t m = man | 0x800000u;
        const uint32_t s = (uint32_t)(14 - e);
        uint32_t q = m >> s;
        const uint32_t r = m & ((1u << s) - 1u);
        const uint32_t halfway = 1u << (s - 1u);
        if (r > halfway || (r == halfway && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t r = man & 0x1FFFu;
    if (r > 0x1000u || (r == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

float orc_bf16_to_f32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7F800000u) == 0x7F800000u && (x & 0x7FFFFFu)) return (uint16_t)((x >> 16) | 0x40u);
    x += 0x7FFFu + ((x >> 16) & 1u);
    return (uint16_t)(x >> 16);
}

/* ------------------------------------------------------------------------ */
/* Index packing                                                             */
/* ------------------------------------------------------------------------ */

/* symbols per 32-bit word: 10 for 3-bit, 32/bits otherwise
 * (vllm_wlq/linear_method.py:316, csrc/vllm_binding.cpp:208) */
int64_t orc_symbols_per_word(int bits) { return bits == 3 ? 10 : 32 / bits; }

/* words per row rounded up to a multiple of 4, so each row starts 16-byte
 * aligned (vllm_wlq/linear_method.py:329-330, csrc/vllm_binding.cpp:209-210) */
int64_t orc_words_per_row(int64_t K, int bits) {
    const int64_t spw = orc_symbols_per_word(bits);
    const int64_t raw = (K + spw - 1) / spw;
    return ((raw + 3) / 4) * 4;
}

/* Continuous on-disk stream -> [N,K] symbols.  Symbol i of the row-major
 * matrix sits in word i/spw at bit offset bits*(i%spw), least significant
 * first; symbols past the end of the stream read as 0 only in the C++
 * repacker, the numpy unpacker requires the full stream
 * (vllm_wlq/linear_method.py:315-323). */
int orc_unpack_continuous(const uint32_t* words, int64_t n_words, int64_t N, int64_t K,
                          int bits, uint8_t* idx_out) {
    const int64_t spw = orc_symbols_per_word(bits);
    const uint32_t mask = (1u << bits) - 1u;
    const int64_t total = N * K;
    if ((total + spw - 1) / spw > n_words) return -1;
    for (int64_t i = 0; i < total; ++i) {
        const uint32_t w = words[i / spw];
        idx_out[i] = (uint8_t)((w >> (uint32_t)(bits * (i % spw))) & mask);
    }
    return 0;
}

/* [N,K] symbols -> row-aligned words [N*wpr], zero padded
 * (vllm_wlq/linear_method.py:326-338). */
void orc_pack_row_aligned(const uint8_t* idx, int64_t N, int64_t K, int bits, uint32_t* out) {
    const int64_t spw = orc_symbols_per_word(bits);
    const int64_t wpr = orc_words_per_row(K, bits);
    const uint32_t mask = (1u << bits) - 1u;
    memset(out, 0, (size_t)(N * wpr) * sizeof(uint32_t));
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k = 0; k < K; ++k) {
            const uint32_t s = idx[n * K + k] & mask;
            out[n * wpr + k / spw] |= s << (uint32_t)(bits * (k % spw));
        }
    }
}

/* Continuous stream -> row-aligned words directly; symbols beyond the
 * stream read as 0 (csrc/vllm_binding.cpp:198-236). */
void orc_repack_row_aligned(const uint32_t* src, int64_t n_src, int64_t N, int64_t K, int bits,
                            uint32_t* out) {
    const int64_t spw = orc_symbols_per_word(bits);
    const int64_t wpr = orc_words_per_row(K, bits);
    const uint32_t mask = (1u << bits) - 1u;
    memset(out, 0, (size_t)(N * wpr) * sizeof(uint32_t));
    int64_t g = 0;
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k = 0; k < K; ++k, ++g) {
            const int64_t sw = g / spw;
            const uint32_t s = sw < n_src ? (src[sw] >> (uint32_t)(bits * (g % spw))) & mask : 0u;
            out[n * wpr + k / spw] |= s << (uint32_t)(bits * (k % spw));
        }
    }
}

/* Row-aligned words -> [N,K] symbols, the in-kernel read of the reference
 * (csrc/gemv_kernel.cu:133-137,168-189; csrc/gemm_kernel.cu:352-426). */
void orc_unpack_row_aligned(const uint32_t* q, int64_t N, int64_t K, int bits, int64_t wpr,
                            uint8_t* idx) {
    const int64_t spw = orc_symbols_per_word(bits);
    const uint32_t mask = (1u << bits) - 1u;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k)
            idx[n * K + k] = (uint8_t)((q[n * wpr + k / spw] >> (uint32_t)(bits * (k % spw))) & mask);
}

/* ------------------------------------------------------------------------ */
/* Outliers                                                                  */
/* ------------------------------------------------------------------------ */

/* fp16 outlier value -> e5m2 byte: (u16 + 0x80) >> 8, clamped to 0..255
 * (vllm_wlq/linear_method.py:306-308, 519-521). */
void orc_fp16_to_fp8_bytes(const uint16_t* h, int64_t n, uint8_t* out) {
    for (int64_t i = 0; i < n; ++i) {
        int32_t v = ((int32_t)h[i] + 0x80) >> 8;
        if (v < 0) v = 0;
        if (v > 255) v = 255;
        out[i] = (uint8_t)v;
    }
}

/* Dense boolean mask [N,K] -> chunk-CSR.  offsets[N,nc+1] hold global running
 * positions, cols hold the column local to its chunk, entries in row-major
 * (row, column) order (vllm_wlq/linear_method.py:284-312).  Returns nnz. */
int64_t orc_build_chunk_csr(const uint8_t* mask, int64_t N, int64_t K, int64_t chunk_m,
                            int32_t* offsets, uint16_t* cols) {
    const int64_t nc = (K + chunk_m - 1) / chunk_m;
    int64_t pos = 0;
    for (int64_t n = 0; n < N; ++n) {
        int32_t* row_off = offsets + n * (nc + 1);
        row_off[0] = (int32_t)pos;
        for (int64_t c = 0; c < nc; ++c) {
            const int64_t k0 = c * chunk_m;
            const int64_t k1 = k0 + chunk_m < K ? k0 + chunk_m : K;
            for (int64_t k = k0; k < k1; ++k) {
                if (mask[n * K + k]) {
                    if (cols) cols[pos] = (uint16_t)(k - k0);
                    ++pos;
                }
            }
            row_off[c + 1] = (int32_t)pos;
        }
    }
    return pos;
}

/* Bit reader used by the Elias-Fano low parts: n_bits from bit_pos, LSB first,
 * spilling into the next word when present (csrc/vllm_binding.cpp:82-92). */
static uint32_t orc_read_bits(const uint32_t* data, int64_t total_words, int64_t bit_pos, int n_bits) {
    if (n_bits <= 0) return 0;
    const int64_t w = bit_pos >> 5;
    const int off = (int)(bit_pos & 31);
    uint64_t v = (uint64_t)data[w] >> off;
    const int got = 32 - off;
    if (n_bits > got && w + 1 < total_words) v |= (uint64_t)data[w + 1] << got;
    return (uint32_t)(v & ((1ull << n_bits) - 1ull));
}

/* Low-part width of one Elias-Fano tile: floor(log2(U/m)) when U > m, else 0
 * (csrc/vllm_binding.cpp:140-144; vllm_wlq/linear_method.py:212, 263). */
static int orc_ef_low_bits(int64_t U, int64_t m) {
    if (m <= 0 || U <= m) return 0;
    int L = (int)floor(log2((double)U / (double)m));
    return L < 0 ? 0 : L;
}

static int orc_cmp_u64(const void* a, const void* b) {
    const uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

/* Elias-Fano tiles -> chunk-CSR, the loader's C++ codec
 * (csrc/vllm_binding.cpp:94-196).  Tiles are row-major over the grid padded
 * to whole tiles; positions outside [N,K] are dropped; coordinates are sorted
 * by (row, col) before the CSR is built.  `cols` may be NULL to count only.
 * Returns the number of kept outliers, or -1 if cap is too small. */
int64_t orc_decode_ef_to_chunk_csr(const int64_t* meta, int64_t n_tiles, const uint32_t* bs,
                                   int64_t n_words, int64_t N, int64_t K, int64_t tile,
                                   int64_t chunk_m, int32_t* offsets, uint16_t* cols, int64_t cap) {
    const int64_t pad_w = (tile - (K % tile)) % tile;
    const int64_t tiles_x = (K + pad_w) / tile;
    const int64_t U = tile * tile;
    const int64_t nc = (K + chunk_m - 1) / chunk_m;
    int64_t total = 0;
    for (int64_t t = 0; t < n_tiles; ++t) total += meta[2 * t + 1];
    memset(offsets, 0, (size_t)(N * (nc + 1)) * sizeof(int32_t));
    if (total == 0) return 0;
    uint64_t* coords = (uint64_t*)malloc((size_t)total * sizeof(uint64_t));
    int64_t kept = 0;
    for (int64_t t = 0; t < n_tiles; ++t) {
        const int64_t start = meta[2 * t];
        const int64_t m = meta[2 * t + 1];
        if (m <= 0) continue;
        const int64_t base_r = (t / tiles_x) * tile;
        const int64_t base_c = (t % tiles_x) * tile;
        const int L = orc_ef_low_bits(U, m);
        int64_t cur = start + m * L;
        int64_t high = 0;
        for (int64_t i = 0; i < m; ++i) {
            const uint32_t low = L > 0 ? orc_read_bits(bs, n_words, start + i * L, L) : 0u;
            while (cur < n_words * 32) {
                const uint32_t bit = (bs[cur >> 5] >> (cur & 31)) & 1u;
                ++cur;
                if (bit == 0u) ++high;
                else break;
            }
            const int64_t local = (high << L) | (int64_t)low;
            const int64_t r = base_r + local / tile;
            const int64_t c = base_c + local % tile;
            if (r < N && c < K) coords[kept++] = ((uint64_t)r << 32) | (uint64_t)c;
        }
    }
    qsort(coords, (size_t)kept, sizeof(uint64_t), orc_cmp_u64);
    if (cols && kept > cap) { free(coords); return -1; }
    for (int64_t i = 0; i < kept; ++i) {
        const int64_t r = (int64_t)(coords[i] >> 32);
        const int64_t c = (int64_t)(coords[i] & 0xFFFFFFFFull);
        if (cols) cols[i] = (uint16_t)(c % chunk_m);
        offsets[r * (nc + 1) + c / chunk_m + 1] += 1;
    }
    int32_t running = 0;
    for (int64_t r = 0; r < N; ++r) {
        int32_t* ro = offsets + r * (nc + 1);
        ro[0] = running;
        for (int64_t c = 0; c < nc; ++c) {
            running += ro[c + 1];
            ro[c + 1] = running;
        }
    }
    free(coords);
    return kept;
}

/* Elias-Fano tiles -> dense mask [H,W] (vllm_wlq/linear_method.py:243-281).
 * Unlike the C++ codec this decoder writes into the padded grid and crops,
 * so the same positions survive. */
int orc_decode_ef_mask(const int64_t* meta, const uint32_t* bs, int64_t n_words, int64_t H,
                       int64_t W, int64_t tile, uint8_t* mask) {
    const int64_t pad_h = (tile - (H % tile)) % tile;
    const int64_t pad_w = (tile - (W % tile)) % tile;
    const int64_t ty = (H + pad_h) / tile, tx = (W + pad_w) / tile;
    const int64_t U = tile * tile;
    memset(mask, 0, (size_t)(H * W));
    for (int64_t t = 0; t < ty * tx; ++t) {
        const int64_t start = meta[2 * t];
        const int64_t m = meta[2 * t + 1];
        if (m <= 0) continue;
        const int L = orc_ef_low_bits(U, m);
        int64_t cur = start + m * L, high = 0, found = 0;
        while (found < m) {
            if (cur >= n_words * 32) return -1;
            const uint32_t bit = (bs[cur >> 5] >> (cur & 31)) & 1u;
            ++cur;
            if (bit == 0u) { ++high; continue; }
            const uint32_t low = L > 0 ? orc_read_bits(bs, n_words, start + found * L, L) : 0u;
            const int64_t local = (high << L) | (int64_t)low;
            const int64_t r = (t / tx) * tile + local / tile;
            const int64_t c = (t % tx) * tile + local % tile;
            if (local < U && r < H && c < W) mask[r * W + c] = 1;
            ++found;
        }
    }
    return 0;
}

/* Elias-Fano ENCODER for test data.  The reference ships no encoder (its
 * checkpoints are produced elsewhere); this writes exactly the layout the
 * decoders above read: per tile, m low parts of L bits each, LSB first, then
 * the unary-coded high parts (gap zeros followed by a one).  meta[t] =
 * (start_bit, m).  Returns the number of 32-bit words used, or -1 if the
 * stream capacity is too small. */
int64_t orc_encode_ef(const uint8_t* mask, int64_t H, int64_t W, int64_t tile, int64_t* meta,
                      uint32_t* bs, int64_t cap_words) {
    const int64_t pad_h = (tile - (H % tile)) % tile;
    const int64_t pad_w = (tile - (W % tile)) % tile;
    const int64_t ty = (H + pad_h) / tile, tx = (W + pad_w) / tile;
    const int64_t U = tile * tile;
    memset(bs, 0, (size_t)cap_words * sizeof(uint32_t));
    int64_t bit = 0;
    int64_t* loc = (int64_t*)malloc((size_t)U * sizeof(int64_t));
    for (int64_t t = 0; t < ty * tx; ++t) {
        const int64_t r0 = (t / tx) * tile, c0 = (t % tx) * tile;
        int64_t m = 0;
        for (int64_t i = 0; i < U; ++i) {
            const int64_t r = r0 + i / tile, c = c0 + i % tile;
            if (r < H && c < W && mask[r * W + c]) loc[m++] = i;
        }
        meta[2 * t] = bit;
        meta[2 * t + 1] = m;
        if (m == 0) continue;
        const int L = orc_ef_low_bits(U, m);
        const int64_t need = bit + m * L + m + ((U - 1) >> L) + 1;
        if ((need + 31) / 32 > cap_words) { free(loc); return -1; }
        for (int64_t i = 0; i < m; ++i) {
            const uint64_t low = (uint64_t)loc[i] & ((1ull << L) - 1ull);
            for (int b = 0; b < L; ++b, ++bit)
                if ((low >> b) & 1ull) bs[bit >> 5] |= 1u << (bit & 31);
        }
        int64_t prev = 0;
        for (int64_t i = 0; i < m; ++i) {
            const int64_t hi = loc[i] >> L;
            bit += hi - prev;
            bs[bit >> 5] |= 1u << (bit & 31);
            ++bit;
            prev = hi;
        }
    }
    free(loc);
    return (bit + 31) / 32;
}

/* ------------------------------------------------------------------------ */
/* Dequantization and the layer forward                                      */
/* ------------------------------------------------------------------------ */

/* Dense W[N,K] as fp16 bit patterns: LUT gather, then outlier positions
 * overwritten by the e5m2 byte shifted into the high byte of an fp16
 * (csrc/gemm_kernel.cu:322-445).  lut layout: group_size == 0 -> [N, 2^bits]
 * (the reference's per-row codebook); group_size > 0 -> [N, ngroups, 2^bits]
 * with column k in group (k + group_offset) / group_size (the per-group
 * codebook of the benchmark recipe; no reference counterpart). */
void orc_dequant(const uint32_t* q, int64_t wpr, const uint16_t* lut, int64_t N, int64_t K,
                 int bits, int64_t group_size, int64_t group_offset, const int32_t* offsets,
                 const uint16_t* cols, const uint8_t* vals, int64_t chunk_m, uint16_t* W) {
    const int64_t spw = orc_symbols_per_word(bits);
    const int64_t kcb = (int64_t)1 << bits;
    const uint32_t mask = (1u << bits) - 1u;
    const int64_t ngroups = group_size > 0 ? (K + group_offset + group_size - 1) / group_size : 1;
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k = 0; k < K; ++k) {
            const uint32_t s = (q[n * wpr + k / spw] >> (uint32_t)(bits * (k % spw))) & mask;
            const int64_t g = group_size > 0 ? (k + group_offset) / group_size : 0;
            W[n * K + k] = lut[(n * ngroups + g) * kcb + s];
        }
        if (offsets && cols && vals) {
            const int64_t nc = (K + chunk_m - 1) / chunk_m;
            for (int64_t c = 0; c < nc; ++c) {
                const int32_t a = offsets[n * (nc + 1) + c], b = offsets[n * (nc + 1) + c + 1];
                for (int32_t i = a; i < b; ++i) {
                    const int64_t col = c * chunk_m + cols[i];
                    if (col < K) W[n * K + col] = (uint16_t)((uint16_t)vals[i] << 8);
                }
            }
        }
    }
}

/* y[m,n] = gamma[n] * (sum_k W[n,k] x[m,k] + s * sum_r h[m,r] B[n,r]) in
 * double precision; W is fp16 bits [N,K], x float [M,K], h float [M,r],
 * B / gamma fp16 bits.  With B, h or gamma NULL the DoRA terms are skipped,
 * as in the reference (csrc/gemv_kernel.cu:305-317, csrc/gemm_kernel.cu:271-293,
 * csrc/gemm_kernel.cu:447-473). */
void orc_forward_f64(const uint16_t* W, const float* x, int64_t M, int64_t N, int64_t K,
                     const float* h, const uint16_t* B, const uint16_t* gamma, int64_t r,
                     double s, double* y) {
    const int dora = (h && B && gamma && r > 0);
    double* wrow = (double*)malloc((size_t)K * sizeof(double));
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t k = 0; k < K; ++k) wrow[k] = (double)orc_f16_to_f32(W[n * K + k]);
        for (int64_t m = 0; m < M; ++m) {
            double acc = 0.0;
            const float* xr = x + m * K;
            for (int64_t k = 0; k < K; ++k) acc += wrow[k] * (double)xr[k];
            if (dora) {
                double l = 0.0;
                for (int64_t j = 0; j < r; ++j) l += (double)h[m * r + j] * (double)orc_f16_to_f32(B[n * r + j]);
                acc = (acc + s * l) * (double)orc_f16_to_f32(gamma[n]);
            }
            y[m * N + n] = acc;
        }
    }
    free(wrow);
}
