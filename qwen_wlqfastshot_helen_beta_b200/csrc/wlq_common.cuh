// Shared device helpers for the WLQ sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/wlq_b200.h"

namespace wlq {

// Symbols of a 4-bit index word: 8, least significant nibble first
// (vllm_wlq/linear_method.py:315-338).
constexpr int kSymPerWord4 = 8;

// Chunk width of the chunk-CSR outlier layout: 640 columns for 3-bit, else
// 512 (csrc/vllm_binding.cpp:279).
__host__ __device__ inline int chunk_m_for_bits(int bits) { return bits == 3 ? 640 : 512; }

__host__ __device__ inline int symbols_per_word(int bits) { return bits == 3 ? 10 : 32 / bits; }

__host__ __device__ inline int64_t words_per_row(int64_t K, int bits) {
    const int64_t spw = symbols_per_word(bits);
    return (((K + spw - 1) / spw) + 3) / 4 * 4;
}

// Activation element types the kernels accept.
template <typename T> struct ActTraits;
template <> struct ActTraits<__half> {
    static constexpr bool kIsF16 = true;
    static __device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
    static __device__ __forceinline__ float bits_to_f32(uint16_t b) { return __half2float(__ushort_as_half(b)); }
    static __device__ __forceinline__ __half from_f32(float v) { return __float2half_rn(v); }
    // fp16 LUT entry -> this type (identity for fp16)
    static __device__ __forceinline__ uint16_t from_f16_bits(uint16_t b) { return b; }
};
template <> struct ActTraits<__nv_bfloat16> {
    static constexpr bool kIsF16 = false;
    static __device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ float bits_to_f32(uint16_t b) { return __bfloat162float(__ushort_as_bfloat16(b)); }
    static __device__ __forceinline__ __nv_bfloat16 from_f32(float v) { return __float2bfloat16_rn(v); }
    static __device__ __forceinline__ uint16_t from_f16_bits(uint16_t b) {
        const float f = __half2float(__ushort_as_half(b));
        return __bfloat16_as_ushort(__float2bfloat16_rn(f));
    }
};

__device__ __forceinline__ float f16_bits_to_f32(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// The e5m2 outlier byte is the high byte of an fp16 (csrc/gemv_kernel.cu:273).
__device__ __forceinline__ uint16_t fp8_byte_to_f16_bits(uint8_t v) { return (uint16_t)((uint16_t)v << 8); }

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// Activations: re-read by every warp on the SM, keep them in L1.
__device__ __forceinline__ uint4 ldg_keep_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::evict_last.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// Streaming load of weight index data: read once, do not keep in L1.
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// 16-byte global -> shared copy that bypasses L1; writes zeros when !ok.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0)
                 : "memory");
}
// The same with the byte count given (16, or 0 to zero-fill): a lane whose
// count is fixed for a whole loop keeps it in a register.
__device__ __forceinline__ void cp_async16_n(uint32_t dst, const void* src, uint32_t n) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
// base + i * stride as one wide multiply-add (the FMA pipe, not the
// integer/logic pipe that the lookups keep busy).
__device__ __forceinline__ const void* ptr_mad(const void* base, uint32_t i, uint32_t stride) {
    uint64_t d;
    asm("mad.wide.u32 %0, %1, %2, %3;" : "=l"(d) : "r"(i), "r"(stride), "l"(reinterpret_cast<uint64_t>(base)));
    return reinterpret_cast<const void*>(d);
}
__device__ __forceinline__ uint32_t mad_u32(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("mad.lo.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a)
                 : "memory");
    return r;
}
// ... at a constant byte offset, folded into the instruction's address
template <int OFF>
__device__ __forceinline__ uint4 lds128_at(uint32_t a) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4+%5];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(a), "n"(OFF) : "memory");
    return r;
}
template <int OFF>
__device__ __forceinline__ uint4 ldg_keep_v4_at(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::evict_last.v4.u32 {%0,%1,%2,%3}, [%4+%5];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "n"(OFF));
    return r;
}


// ---------------------------------------------------------------------------
// In-register 16-entry LUT.
//
// A 16-entry table of 16-bit values is held as four byte planes: lo[0..1]
// hold the low bytes of entries 0..7, lo[2..3] of entries 8..15, hi[] the high
// bytes.  A byte permute (prmt) with a 3-bit selector picks one byte out of
// two registers, so four lookups per plane-half, one more permute to choose
// the half by bit 3 of the index, and two permutes to interleave low and high
// bytes give two packed 16-bit pairs for four indices.
// ---------------------------------------------------------------------------
struct LutPlanes {
    uint32_t lo[4];
    uint32_t hi[4];
};

// e[i] packs entries 2i (low half) and 2i+1 (high half).
__device__ __forceinline__ void make_planes(const uint32_t e[8], LutPlanes& p) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        p.lo[j] = __byte_perm(e[2 * j], e[2 * j + 1], 0x6420);
        p.hi[j] = __byte_perm(e[2 * j], e[2 * j + 1], 0x7531);
    }
}

// x >> 16 and x >> 1 on the FMA pipe (mul.hi by a runtime power of two).
__device__ __forceinline__ uint32_t mulhi(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.hi.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
    return d;
}
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t o) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(m), "r"(o));  // (a & m) | o
    return d;
}

// (T[q0],T[q1]) and (T[q2],T[q3]) for the four indices in the low 16 bits.
__device__ __forceinline__ void lookup4(const LutPlanes& p, uint32_t sel, uint32_t csel, uint32_t& o01,
                                        uint32_t& o23) {
    const uint32_t la = prmt(p.lo[0], p.lo[1], sel);
    const uint32_t lb = prmt(p.lo[2], p.lo[3], sel);
    const uint32_t ha = prmt(p.hi[0], p.hi[1], sel);
    const uint32_t hb = prmt(p.hi[2], p.hi[3], sel);
    const uint32_t lo = prmt(la, lb, csel);
    const uint32_t hi = prmt(ha, hb, csel);
    o01 = prmt(lo, hi, 0x5140u);
    o23 = prmt(lo, hi, 0x7362u);
}

// Codebook planes of one (row, group): prepacked (8 words: lo[4], hi[4]) or
// the reference's 16 fp16 entries, converted and permuted here.
template <typename T, bool PREPACKED>
__device__ __forceinline__ void planes_from_words(const uint4 a, const uint4 b, LutPlanes& P) {
    if (PREPACKED) {
        P.lo[0] = a.x; P.lo[1] = a.y; P.lo[2] = a.z; P.lo[3] = a.w;
        P.hi[0] = b.x; P.hi[1] = b.y; P.hi[2] = b.z; P.hi[3] = b.w;
        return;
    }
    uint32_t e[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (!ActTraits<T>::kIsF16) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&e[i]));
            const __nv_bfloat162 v = __float22bfloat162_rn(f);
            e[i] = *reinterpret_cast<const uint32_t*>(&v);
        }
    }
    make_planes(e, P);
}

template <typename T, bool PREPACKED>
__device__ __forceinline__ void load_planes(const uint16_t* __restrict__ lut, int64_t entry, bool valid,
                                            LutPlanes& P) {
    uint4 a = make_uint4(0u, 0u, 0u, 0u), b = a;
    if (valid) {  // the 4 lanes sharing a codebook read it in one request
        a = ldg_stream_v4(lut + entry * 16);
        b = ldg_stream_v4(lut + entry * 16 + 8);
    }
    planes_from_words<T, PREPACKED>(a, b, P);
}

template <typename T, bool PREPACKED>
__device__ __forceinline__ void planes_from_smem(uint32_t addr, LutPlanes& P) {
    planes_from_words<T, PREPACKED>(lds128(addr), lds128(addr + 16), P);
}

// ---------------------------------------------------------------------------
// Warp-level tensor-core MMA (m16n8k16, fp32 accumulate).
// ---------------------------------------------------------------------------
template <typename T> struct Mma16816;
template <> struct Mma16816<__half> {
    static __device__ __forceinline__ void run(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <> struct Mma16816<__nv_bfloat16> {
    static __device__ __forceinline__ void run(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

// ---------------------------------------------------------------------------
// Thread-block cluster helpers (distributed shared memory).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ float ld_shared_cluster_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

}  // namespace wlq
