/*
 * wlq_b200.h -- C ABI of the B200 (sm_100a) WLQ 4-bit LUT linear path.
 *
 * Plain pointers and sizes only; no framework types.  Every GPU entry point
 * takes device pointers and a CUDA stream (cudaStream_t, passed as an opaque
 * pointer), validates its arguments on the host, enqueues its kernels on that
 * stream and returns a status code; it never synchronises and never
 * allocates device memory.  On failure wlq_last_error() returns a message for
 * the calling thread.  Each declaration cites the reference interface it
 * replaces (paths relative to the reference project root).
 *
 * Data layout (the reference's device layout, vllm_wlq/linear_method.py:326-338,
 * 655-667):
 *   q_packed      int32 [N * words_per_row]; 4-bit indices, 8 per word, least
 *                 significant nibble first; words_per_row = roundup4(ceil(K/8)).
 *   lut_c         fp16; lut_group_size == 0: [N, 16], one codebook per output
 *                 row (the reference); lut_group_size > 0: [N, ngroups, 16]
 *                 with column k in group (k + lut_group_offset) / lut_group_size
 *                 and ngroups = ceil((K + lut_group_offset) / lut_group_size).
 *   chunk_offsets int32 [N, ceil(K/512) + 1], global running offsets;
 *   chunk_cols    uint16 [nnz], column local to its 512-wide chunk;
 *   chunk_vals    uint8  [nnz], e5m2 byte = high byte of the fp16 value.
 *                 Outliers REPLACE the codebook weight (all three NULL = none).
 *   lora_B        fp16 [N, r]; lora_h / lora_H fp32 [M, r] (= A x);
 *   dora_gamma    fp16 [N]; lora_scale = lora_alpha / r.  The DoRA term is
 *                 applied only when lora_B, lora_h/H and dora_gamma are all
 *                 non-NULL and r > 0 (csrc/gemv_kernel.cu:440).
 *   x / X, out    [M, K] / [M, N], row-major, act_dtype (fp16 or bf16).
 *
 * out[m, n] = gamma[n] * (sum_k W[n,k] x[m,k] + s * sum_j h[m,j] B[n,j]),
 * W the codebook weights with outliers replaced, accumulated in fp32.
 */
#ifndef WLQ_B200_H
#define WLQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define WLQ_API __attribute__((visibility("default")))
#else
#define WLQ_API
#endif

typedef void* wlq_stream_t; /* a cudaStream_t; NULL = the legacy default stream */

enum wlq_status {
    WLQ_OK = 0,
    WLQ_ERR_INVALID_ARG = 1, /* NULL required pointer, bad size */
    WLQ_ERR_UNSUPPORTED = 2, /* bits / dtype / group layout this build does not run */
    WLQ_ERR_ALIGNMENT = 3,   /* pointer not aligned as the layout requires */
    WLQ_ERR_CUDA = 4,        /* a CUDA runtime call or launch failed */
    WLQ_ERR_CAPACITY = 5,    /* caller's output buffer too small */
    WLQ_ERR_DEVICE = 6       /* the current device is not sm_100 */
};

enum wlq_dtype { WLQ_DTYPE_F16 = 0, WLQ_DTYPE_BF16 = 1 };

/* Layout of the codebooks and outliers given to wlq_gemv / wlq_gemm.
 * WLQ_LUT_F16: the reference's layout (16 fp16 entries per codebook; outliers
 * as chunk-local columns and e5m2 bytes).
 * WLQ_LUT_PREPACKED: the load-time layout for one act_dtype, made once by
 * wlq_prepack_lut (codebooks: entries rounded to the MMA type, bytes split
 * into planes; same size and indexing) and wlq_prepack_outliers (chunk_cols
 * then points to uint32 records, column | outlier value bits in the MMA type
 * << 16, each row's entries in ascending column order, and chunk_vals to
 * float32 corrections w_outlier - codebook value; chunk_offsets unchanged),
 * so the kernels never convert codebooks or look up outlier codebook values. */
enum wlq_lut_format { WLQ_LUT_F16 = 0, WLQ_LUT_PREPACKED = 1 };

/* Message of the last failed call on this thread ("" if none). */
WLQ_API const char* wlq_last_error(void);
/* ABI revision of this header. */
WLQ_API int wlq_abi_version(void);
#define WLQ_ABI_VERSION 1

/* ---------------------------------------------------------------- GPU --- */

/* Decode GEMV for M = 1..16 token rows, DoRA update and outlier replacement
 * fused.  Replaces launch_gemv_chunk_csr (csrc/gemv_kernel.cu:396-414) and
 * gemv_forward (csrc/vllm_binding.cpp:253-315), which handle M = 1 only and
 * need a split-K workspace; this one needs none.  bits must be 4. */
WLQ_API int wlq_gemv(const int32_t* q_packed, const void* lut_c, const void* x, void* out,
             const int32_t* chunk_offsets, const void* chunk_cols, const void* chunk_vals,
             const void* lora_B, const float* lora_h, const void* dora_gamma, float lora_scale,
             int r, int M, int N, int K, int bits, int words_per_row, int lut_group_size,
             int lut_group_offset, int lut_format, int act_dtype, wlq_stream_t stream);

/* wlq_gemv with the DoRA low-rank input computed inside the kernel: lora_A
 * ([r, K] in act_dtype, r <= 32) takes the place of lora_h = A x.  Needs
 * WLQ_LUT_PREPACKED and 16-byte aligned rows of x and lora_A (K % 8 == 0).
 * Folds the two launches that precede every reference GEMV,
 * F.linear(x, lora_A).float() (vllm_wlq/linear_method.py:962-963), into the
 * GEMV; h is kept in fp32 instead of being rounded to fp16 first. */
WLQ_API int wlq_gemv_lora_a(const int32_t* q_packed, const void* lut_c, const void* x, void* out,
             const int32_t* chunk_offsets, const void* chunk_cols, const void* chunk_vals,
             const void* lora_B, const void* lora_A, const void* dora_gamma, float lora_scale,
             int r, int M, int N, int K, int bits, int words_per_row, int lut_group_size,
             int lut_group_offset, int lut_format, int act_dtype, wlq_stream_t stream);

/* Batched forward for any M >= 1: M <= 16 runs the GEMV-class kernel, larger
 * M the tcgen05 tensor-core GEMM with dequantisation, outlier replacement and
 * the DoRA epilogue fused.  chunk_cols / chunk_vals: uint16 columns and e5m2
 * bytes (WLQ_LUT_F16) or the prepacked records and corrections
 * (WLQ_LUT_PREPACKED).  Replaces launch_gemm_metalog_dora
 * (csrc/gemm_kernel.cu:527-547) and the M >= 16 dequantise + cuBLAS +
 * epilogue composition of gemm_forward (csrc/vllm_binding.cpp:318-419). */
WLQ_API int wlq_gemm(const void* X, const int32_t* q_packed, const void* lut_c, void* out,
             const int32_t* chunk_offsets, const void* chunk_cols, const void* chunk_vals,
             const float* lora_H, const void* lora_B, const void* dora_gamma, float lora_scale,
             int r, int M, int N, int K, int bits, int words_per_row, int lut_group_size,
             int lut_group_offset, int lut_format, int act_dtype, wlq_stream_t stream);

/* wlq_gemm with a stream-K schedule for the tensor-core path (M > 16 rows
 * that the GEMV does not take): when the output tiles do not fill whole
 * waves of one CTA per SM, the k steps of the last wave and the remainder are
 * split evenly over the SMs and the partial tiles are summed through
 * `workspace` (fp32, in a fixed CTA order, so results do not depend on
 * timing).  `workspace` is device memory of workspace_bytes, 256-byte aligned,
 * zero-filled before its first use and kept between calls (every call leaves
 * its flags zero again); wlq_gemm_workspace_bytes(device) bytes always
 * suffice, less restricts the split.  Calls that share a workspace must not
 * run concurrently (one stream, or one workspace per stream).  NULL or too
 * small a workspace gives wlq_gemm's data-parallel schedule.  Replaces the same
 * reference composition as wlq_gemm (csrc/vllm_binding.cpp:355-393), where
 * cuBLAS picks split-K schedules internally. */
WLQ_API size_t wlq_gemm_workspace_bytes(int device);
WLQ_API int wlq_gemm_streamk(const void* X, const int32_t* q_packed, const void* lut_c, void* out,
             const int32_t* chunk_offsets, const void* chunk_cols, const void* chunk_vals,
             const float* lora_H, const void* lora_B, const void* dora_gamma, float lora_scale,
             int r, int M, int N, int K, int bits, int words_per_row, int lut_group_size,
             int lut_group_offset, int lut_format, int act_dtype, void* workspace, size_t workspace_bytes,
             wlq_stream_t stream);

/* wlq_gemm_streamk for callers that cannot allocate device memory: a host
 * runtime reaching this library through FFI (cgo, JNI, ctypes) with no device
 * allocator of its own, or a serving loop that must not call cudaMalloc on
 * its hot path because cudaMalloc synchronises the device and cannot be
 * recorded while a stream is being captured.  It allocates nothing: its
 * stream-K scratch (flags and partial tiles) is a static array of
 * WLQ_GEMM_STATIC_SCRATCH_BYTES inside the library, which every GPU that
 * loads the library holds until the process exits.  Same arguments and
 * results as wlq_gemm_streamk without the workspace.  The first call on a
 * device looks the array's device address up (cudaGetSymbolAddress, with
 * that device current): make it before any stream capture.  Each call
 * clears the scratch's flags on `stream` first; the array keeps the last
 * call's partial tiles.  Calls on one device share the array: calls that
 * overlap on the GPU (several streams, or several threads) race and give
 * wrong results.  A problem whose schedule needs more scratch than the
 * array holds is refused with WLQ_ERR_CAPACITY (on a 148-SM B200 every
 * schedule fits: 148 partial tiles of 256 KB plus flags).  No counterpart in
 * the reference, whose GEMM path allocates through ATen. */
#define WLQ_GEMM_STATIC_SCRATCH_BYTES (40u * 1024u * 1024u)
WLQ_API int wlq_gemm_streamk_noalloc(const void* X, const int32_t* q_packed, const void* lut_c, void* out,
             const int32_t* chunk_offsets, const void* chunk_cols, const void* chunk_vals,
             const float* lora_H, const void* lora_B, const void* dora_gamma, float lora_scale,
             int r, int M, int N, int K, int bits, int words_per_row, int lut_group_size,
             int lut_group_offset, int lut_format, int act_dtype, wlq_stream_t stream);

/* DoRA low-rank input H = X lora_A^T, fp32 [M, r], for the calls that do not
 * compute it inside the decode GEMV (the prefill GEMM; rank above 48).  X
 * [M, K] and lora_A [r, K] in act_dtype; tensor cores, fp32 accumulation, no
 * workspace.  Replaces the library GEMM and cast before every reference GEMM
 * op, F.linear(x, lora_A).float() (vllm_wlq/linear_method.py:984); H is not
 * rounded to fp16 first. */
WLQ_API int wlq_lora_h(const void* X, const void* lora_A, float* H, int M, int K, int r, int act_dtype,
                       wlq_stream_t stream);

/* Codebooks -> WLQ_LUT_PREPACKED layout for act_dtype: n_codebooks x 16 fp16
 * entries in, the same number of 32-byte records out (may not alias).  Done
 * once at load time; no reference counterpart (the reference converts per
 * call inside its kernels). */
WLQ_API int wlq_prepack_lut(const void* lut_c, void* lut_out, int64_t n_codebooks, int act_dtype,
                            wlq_stream_t stream);

/* Outliers -> the WLQ_LUT_PREPACKED outlier stream for act_dtype: per chunk-CSR
 * entry a uint32 record (global column in the low 16 bits, K <= 65535, 0xFFFF
 * for an entry past K; the outlier value rounded to the MMA type in the high
 * 16 bits) and the float32 correction w_outlier - codebook value with the
 * codebook entry rounded to the MMA type.  Within each row the entries are
 * reordered by ascending column (they stay inside their chunk's index range;
 * the reference's builders already emit that order).  Inputs are in the
 * reference layout (fp16 codebooks).  No reference counterpart (the reference
 * re-reads the index word and codebook per outlier,
 * csrc/gemv_kernel.cu:262-288). */
WLQ_API int wlq_prepack_outliers(const int32_t* q_packed, const void* lut_c, const int32_t* chunk_offsets,
                                 const uint16_t* chunk_cols, const uint8_t* chunk_vals, int64_t nnz, int N,
                                 int K, int bits, int words_per_row, int lut_group_size, int lut_group_offset,
                                 int act_dtype, uint32_t* cols_out, float* delta_out, wlq_stream_t stream);

/* Dense fp16 W[N, K] (codebook gather, then outliers overwritten), bit-exact
 * with the reference.  bits 1..4.  Replaces launch_dequant_patch_metalog
 * (csrc/gemm_kernel.cu:475-489) and dequant_w0 (csrc/vllm_binding.cpp:421-453). */
WLQ_API int wlq_dequant(const int32_t* q_packed, const void* lut_c, void* W_out,
                const int32_t* chunk_offsets, const uint16_t* chunk_cols, const uint8_t* chunk_vals,
                int N, int K, int bits, int words_per_row, int lut_group_size, int lut_group_offset,
                wlq_stream_t stream);

/* Kept for interface parity with init_workspaces (csrc/vllm_binding.cpp:241-251):
 * the kernels of this library need no workspace, so this only validates. */
WLQ_API int wlq_init_workspaces(int64_t max_N, int64_t max_K, int device);

/* ------------------------------------------------ tensor parallelism --- */
/* Row-parallel layers (o, down) need the sum of every rank's partial output.
 * wlq_gemv_allreduce fuses that all-reduce into the GEMV epilogue over NVLink
 * peer memory: each rank stores its gamma-scaled tile into every other rank's
 * communication buffer, every value tagged with the call's epoch in the same
 * 8-byte store, then waits (bounded, 2 s) until its own slots hold every
 * rank's values of this epoch and sums them in rank order.  Each rank
 * allocates one buffer of
 * wlq_tp_buffer_bytes(world, max_N) with wlq_tp_buffer_alloc, exchanges the
 * 64-byte IPC handles with the other ranks (any host channel) and maps theirs
 * with wlq_tp_buffer_open.  All ranks must issue the same sequence of calls,
 * on one stream per rank, one call after another: the per-tile epoch
 * counters and the value slots of a buffer are shared by every call made
 * with it (o and down alike), so two calls in flight at once on one rank
 * (concurrent streams, or a call overlapping the previous one through
 * programmatic dependent launch) race; use one buffer set per stream.
 * No reference counterpart: the reference leaves the all-reduce to vLLM's
 * NCCL call after the layer (vllm: model_executor/layers/linear.py:1558-1559). */
WLQ_API size_t wlq_tp_buffer_bytes(int world, int max_N);
/* cudaMalloc'd and zeroed on the current device; handle_out receives the
 * cudaIpcMemHandle_t (64 bytes).  Setup only: the one allocating entry point
 * besides the codec helpers. */
WLQ_API int wlq_tp_buffer_alloc(size_t bytes, void** ptr_out, unsigned char handle_out[64]);
WLQ_API int wlq_tp_buffer_open(const unsigned char handle[64], void** ptr_out);
WLQ_API int wlq_tp_buffer_close(void* peer_ptr);
WLQ_API int wlq_tp_buffer_free(void* ptr);
/* Reads (and optionally clears) the error word of this rank's buffer: bit 0
 * set when a fused all-reduce gave up waiting for a rank (its output is then
 * undefined).  Synchronous. */
WLQ_API int wlq_tp_error(void* local_buf, unsigned int* flags_out, int clear);
/* wlq_gemv (M <= 16) on this rank's K shard with the all-reduce of out over
 * the tp_world ranks fused; tp_bufs[q] is rank q's buffer as mapped in this
 * process (tp_bufs[tp_rank] the local one), max_N the N it was sized for.
 * The DoRA input is lora_h, or lora_A (this rank's K columns of A) as in
 * wlq_gemv_lora_a; the other one is null. */
WLQ_API int wlq_gemv_allreduce(const int32_t* q_packed, const void* lut_c, const void* x, void* out,
             const int32_t* chunk_offsets, const void* chunk_cols, const void* chunk_vals,
             const void* lora_B, const float* lora_h, const void* lora_A, const void* dora_gamma,
             float lora_scale,
             int r, int M, int N, int K, int bits, int words_per_row, int lut_group_size,
             int lut_group_offset, int lut_format, int act_dtype, void* const* tp_bufs, int tp_rank,
             int tp_world, int max_N, wlq_stream_t stream);

/* Test and tuning hook of the decode GEMV's K split: wlq_gemv_set_split(cs)
 * makes every later wlq_gemv / wlq_gemv_lora_a / wlq_gemm-as-GEMV launch of
 * the process split K over a cluster of exactly cs CTAs (1..16, at most one
 * per 128-column chunk; above 8 a non-portable cluster size the device must
 * accept), 0 restores the per-call choice.  wlq_gemv_last_split() returns the
 * split of the calling thread's last successful GEMV launch and
 * wlq_gemv_last_warps() its CTA shape: 4 (warps per CTA, 4 CTAs per SM) or 16
 * (one CTA per SM, chosen where 4-warp CTAs could not keep the activations in
 * shared memory, or where neither shape splits K).  No reference counterpart
 * (the reference's split-K is internal, csrc/gemv_kernel.cu:422-428). */
WLQ_API int wlq_gemv_set_split(int cs);
WLQ_API int wlq_gemv_last_split(void);
WLQ_API int wlq_gemv_last_warps(void);

/* Opt-in overlap of consecutive decode GEMV launches in a stream (process
 * wide; off by default).  With wlq_gemv_set_overlap(1), every later
 * wlq_gemv / wlq_gemv_lora_a / wlq_gemm-as-GEMV launch (not the fused
 * all-reduce) is a programmatic dependent launch: it may start while the
 * kernel before it in the stream is still running and read its WEIGHTS
 * (q_packed, codebooks, outlier records and offsets, lora_A / lora_B, gamma)
 * before that kernel's writes are visible; activations, h and out are only
 * touched after the previous kernel has completed.  Enable it only where no
 * kernel launched immediately before a GEMV call in the same stream writes
 * that layer's weights -- true for inference once the weights are loaded and
 * the device synchronised -- and keep it off while weights are being written
 * (loading, prepacking).  wlq_gemv_get_overlap() returns the setting.  No
 * reference counterpart (the reference launches its kernels plainly). */
WLQ_API int wlq_gemv_set_overlap(int on);
WLQ_API int wlq_gemv_get_overlap(void);

/* Device error word of `device`: bit 0 (WLQ_DEVERR_WAIT_TIMEOUT) is set when
 * a pipeline wait inside a tensor-core GEMM kernel gave up (the kernel then
 * abandons its tile and its output is undefined).  Synchronous; clears the
 * word when `clear` is non-zero.  No reference counterpart: the reference
 * kernels have no bounded waits. */
#define WLQ_DEVERR_WAIT_TIMEOUT 1u
WLQ_API int wlq_device_error(int device, unsigned int* flags_out, int clear);

/* ---------------------------------------------------------------- CPU --- */
/* Load-time codecs (host memory). */

/* roundup4(ceil(K / symbols_per_word)) (vllm_wlq/linear_method.py:326-331). */
WLQ_API int64_t wlq_words_per_row(int64_t K, int bits);

/* Continuous on-disk index stream -> row-aligned words [N * words_per_row];
 * symbols beyond n_src words read as 0.  Replaces repack_q_indices_row_aligned
 * (csrc/vllm_binding.cpp:198-236). */
WLQ_API int wlq_repack_q_indices_row_aligned(const int32_t* src, int64_t n_src, int64_t N, int64_t K,
                                     int bits, int32_t* dst, int64_t dst_capacity,
                                     int64_t* words_per_row);

/* Rows [r0,r1) x columns [c0,c1) of a continuous [N_full, K_full] index stream
 * -> row-aligned words: the tensor-parallel shard of a layer.  Replaces the
 * unpack / slice / pack sequence of vllm_wlq/linear_method.py:724, 753-761, 792. */
WLQ_API int wlq_repack_q_indices_slice(const int32_t* src, int64_t n_src, int64_t N_full, int64_t K_full, int bits,
                               int64_t r0, int64_t r1, int64_t c0, int64_t c1, int32_t* dst,
                               int64_t dst_capacity, int64_t* words_per_row);

/* Elias-Fano tiles -> sorted, unique flat outlier positions r*K + c, the
 * row-major order of the outlier value list; positions may be NULL to count.
 * Replaces decode_elias_fano (vllm_wlq/linear_method.py:243-281) where the
 * mask is needed for tensor-parallel slicing. */
WLQ_API int wlq_decode_ef_positions(const int64_t* tile_meta, int64_t n_tiles, const int32_t* bitstream,
                            int64_t n_words, int64_t N, int64_t K, int64_t tile_size, int64_t* positions,
                            int64_t capacity, int64_t* count);

/* Sorted unique flat positions -> chunk-CSR (vllm_wlq/linear_method.py:284-303). */
WLQ_API int wlq_positions_to_chunk_csr(const int64_t* positions, int64_t n, int64_t N, int64_t K, int64_t chunk_m,
                               int32_t* offsets, uint16_t* cols);

/* Elias-Fano tiles -> chunk-CSR.  offsets [N, ceil(K/chunk_m)+1]; cols may be
 * NULL to count only (nnz returned either way).  Replaces
 * decode_ef_to_chunk_csr (csrc/vllm_binding.cpp:94-196). */
WLQ_API int wlq_decode_ef_to_chunk_csr(const int64_t* tile_meta, int64_t n_tiles, const int32_t* bitstream,
                               int64_t n_words, int64_t N, int64_t K, int64_t tile_size,
                               int64_t chunk_m, int32_t* offsets, uint16_t* cols,
                               int64_t cols_capacity, int64_t* nnz);

/* Dense outlier mask [N, K] (0/1 bytes) -> chunk-CSR.  Replaces
 * build_chunk_csr (vllm_wlq/linear_method.py:284-312). */
WLQ_API int wlq_build_chunk_csr(const uint8_t* mask, int64_t N, int64_t K, int64_t chunk_m,
                        int32_t* offsets, uint16_t* cols, int64_t cols_capacity, int64_t* nnz);

/* fp16 outlier values -> e5m2 bytes, (u16 + 0x80) >> 8 clamped
 * (vllm_wlq/linear_method.py:306-308, 519-521). */
WLQ_API int wlq_fp16_to_fp8_bytes(const uint16_t* src, int64_t n, uint8_t* dst);

/* Host twin of wlq_prepack_lut. */
WLQ_API int wlq_prepack_lut_host(const uint16_t* lut_c, uint16_t* lut_out, int64_t n_codebooks, int act_dtype);

/* Host twin of wlq_dequant, for loading without a GPU (the reference's
 * gather fallback, vllm_wlq/linear_method.py:608-623). */
WLQ_API int wlq_dequant_host(const int32_t* q_packed, const uint16_t* lut_c, uint16_t* W_out,
                     const int32_t* chunk_offsets, const uint16_t* chunk_cols,
                     const uint8_t* chunk_vals, int64_t N, int64_t K, int bits,
                     int64_t words_per_row, int64_t lut_group_size, int64_t lut_group_offset);

#ifdef __cplusplus
}
#endif

#endif /* WLQ_B200_H */
