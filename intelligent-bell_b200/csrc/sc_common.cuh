// sc_common.cuh — shared device helpers for the sm_100a KV-restore kernels.
//
// Everything here is elementwise, HBM-bound integer/half arithmetic: 16-byte vector
// loads of INT8 codes, exact int8 -> fp16 conversion by exponent-bias arithmetic,
// fp16/fp32 dequantisation and the rotate-half RoPE step, packed 16-byte stores.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "sc_internal.h"

namespace sc {

// ---------------------------------------------------------------------------------------
// Unsigned 32-bit division by a run-time constant (Granlund-Montgomery round-up method).
// Valid for numerators < 2^31, which every launch guarantees (rows < 2^31).
// ---------------------------------------------------------------------------------------
struct FastDiv {
    uint32_t d;
    uint32_t m;
    uint32_t s;
};

inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f{d, 0u, 0u};
    uint32_t l = 0;
    while ((1ull << l) < d) ++l;
    f.s = l;
    // m = floor(2^32 * (2^l - d) / d) + 1
    f.m = static_cast<uint32_t>(((1ull << 32) * ((1ull << l) - d)) / d + 1ull);
    return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
    const uint32_t t = __umulhi(n, f.m);
    return (t + n) >> f.s;
}

// ---------------------------------------------------------------------------------------
// Memory access.  Inputs are read once: non-coherent loads that do not allocate in L1.
// Tuning knobs (compile-time): SC_LOAD_L2_PREFETCH adds a 256-byte L2 prefetch hint to
// the input loads; SC_STORE_STREAMING marks output stores evict-first.
// ---------------------------------------------------------------------------------------
#ifndef SC_LOAD_L2_PREFETCH
#define SC_LOAD_L2_PREFETCH 0
#endif
#ifndef SC_STORE_STREAMING
#define SC_STORE_STREAMING 0
#endif

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
    uint4 r;
#if SC_LOAD_L2_PREFETCH
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
#else
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
#endif
    return r;
}

__device__ __forceinline__ void st_v4(void* p, const uint4& v) {
#if SC_STORE_STREAMING
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
#else
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
#endif
}

// One 32-byte store (a full L2 sector per lane); the address must be 32-byte aligned.
__device__ __forceinline__ void st_v8(void* p, const uint32_t (&v)[8]) {
#if SC_STORE_STREAMING
    asm volatile("st.global.cs.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
#else
    asm volatile("st.global.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
#endif
}

__device__ __forceinline__ void st_v2(void* p, const uint2& v) {
    asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

template <typename T>
__device__ __forceinline__ T bit_cast_u32(uint32_t u);
template <>
__device__ __forceinline__ __half2 bit_cast_u32<__half2>(uint32_t u) {
    return *reinterpret_cast<__half2*>(&u);
}
__device__ __forceinline__ uint32_t u32_of(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ uint32_t u32_of(__nv_bfloat162 h) {
    return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------------------------------
// Exact int8 -> fp16 for four codes packed in one 32-bit word.
// Flip the sign bit so each byte holds code+128 in [0, 255]; splice each byte under the
// fp16 exponent pattern 0x64 (0x64XX == 1024 + XX exactly) and subtract 1152 = 1024+128.
// Three integer/half instructions per two codes, no type-conversion unit involved.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void i8x4_to_h2(uint32_t w, __half2& lo, __half2& hi) {
    const uint32_t u = w ^ 0x80808080u;
    const uint32_t a = __byte_perm(u, 0x64646464u, 0x4140);
    const uint32_t b = __byte_perm(u, 0x64646464u, 0x4342);
    const __half2 bias = bit_cast_u32<__half2>(0x64806480u);  // (1152, 1152)
    lo = __hsub2(bit_cast_u32<__half2>(a), bias);
    hi = __hsub2(bit_cast_u32<__half2>(b), bias);
}

// Output packing: two fp32 values -> one 32-bit word of the output dtype (RN-even).
template <typename OutT>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    return u32_of(__floats2half2_rn(a, b));
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    return u32_of(__floats2bfloat162_rn(a, b));
}

template <typename OutT>
__device__ __forceinline__ OutT from_float(float a);
template <>
__device__ __forceinline__ __half from_float<__half>(float a) {
    return __float2half_rn(a);
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float a) {
    return __float2bfloat16_rn(a);
}

template <typename ScaleT>
__device__ __forceinline__ float scale_to_float(ScaleT s);
template <>
__device__ __forceinline__ float scale_to_float<__half>(__half s) {
    return __half2float(s);
}
template <>
__device__ __forceinline__ float scale_to_float<float>(float s) {
    return s;
}

// cos/sin of one relative shift for frequency f, rounded like the reference's tables:
// angle = fp32(dp * inv_freq) (one fp32 multiply); cos/sin of the angle rounded to fp16.
// Returns the fp16 values widened back to fp32.
//
// Fast path: sincosf is within 2 ulp of the true value, so when v - 4 ulp and v + 4 ulp
// round to the same fp16 value, that value is the fp16 rounding of the true cos/sin.
// Otherwise (the value lies next to an fp16 rounding tie) both are evaluated in double,
// rounded to fp32 and then to fp16.  Both paths give the same fp16 values as evaluating
// in double everywhere.
__device__ __forceinline__ bool fp16_settled(float v, __half& out) {
    const float margin = fmaxf(fabsf(v) * 4.76837158203125e-07f, 1.0e-30f);  // >= 4 ulp
    const __half lo = __float2half_rn(v - margin);
    const __half hi = __float2half_rn(v + margin);
    out = __float2half_rn(v);
    return __half_as_ushort(lo) == __half_as_ushort(hi);
}

__device__ __forceinline__ void rope_cs(float dp, float inv_freq, float& c, float& s) {
    const float angle = __fmul_rn(dp, inv_freq);
    float sf, cf;
    sincosf(angle, &sf, &cf);
    __half ch, sh;
    const bool ok_c = fp16_settled(cf, ch);
    const bool ok_s = fp16_settled(sf, sh);
    if (!(ok_c && ok_s)) {
        double sd, cd;
        sincos(static_cast<double>(angle), &sd, &cd);
        ch = __float2half_rn(static_cast<float>(cd));
        sh = __float2half_rn(static_cast<float>(sd));
    }
    c = __half2float(ch);
    s = __half2float(sh);
}

// The rotate-half pair: o1 = x1 c - x2 s, o2 = x2 c + x1 s, rounded like torch's separate
// multiply and add (each product rounded to fp32, then the sum).  kExact: x1, x2, c and s
// are all fp16 values, so both products are exact in fp32 and one fma per output gives the
// same bits with fewer instructions.  Otherwise (fp32 intermediate) the products carry up to
// 29 significant bits and are rounded explicitly, which an fma would skip.
template <bool kExact>
__device__ __forceinline__ void rotate_pair(float x1, float x2, float c, float s, float& o1,
                                            float& o2) {
    if constexpr (kExact) {
        o1 = fmaf(x1, c, -(x2 * s));
        o2 = fmaf(x2, c, x1 * s);
    } else {
        o1 = __fadd_rn(__fmul_rn(x1, c), -__fmul_rn(x2, s));
        o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    }
}

// cos/sin of a 16-frequency slice, read four at a time.
//   CsShared: the block's table in shared memory (16-byte aligned float4 reads).
//   CsRegs:   values the thread holds itself (per-token tables).
struct CsShared {
    const float4* c;
    const float4* s;
    __device__ __forceinline__ float4 cos4(int w) const { return c[w]; }
    __device__ __forceinline__ float4 sin4(int w) const { return s[w]; }
};
struct CsRegs {
    const float* c;
    const float* s;
    __device__ __forceinline__ float4 cos4(int w) const {
        return make_float4(c[4 * w], c[4 * w + 1], c[4 * w + 2], c[4 * w + 3]);
    }
    __device__ __forceinline__ float4 sin4(int w) const {
        return make_float4(s[4 * w], s[4 * w + 1], s[4 * w + 2], s[4 * w + 3]);
    }
};

// ---------------------------------------------------------------------------------------
// One 16-frequency slice of one row: 16 key codes of the first half (a) and their 16
// rotate-half partners of the second half (b), the row scale, the slice's cos/sin.
// Writes 16 outputs at o1 (first half) and 16 at o2 (second half), one 32-byte store
// each (o1 and o2 must be 32-byte aligned).
//   X16 = true : x = fp16(q*s) first (reference eager arithmetic; exact because q*s is
//                exact in fp32 and __hmul2_rn rounds it once)
//   X16 = false: x = q*s kept in fp32
// ---------------------------------------------------------------------------------------
template <typename OutT, typename ScaleT, bool X16, typename CS>
__device__ __forceinline__ void rope_slice_store(const uint4& a, const uint4& b, ScaleT scale,
                                                 const CS& cs, void* o1, void* o2) {
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
    const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
    const float sf = scale_to_float<ScaleT>(scale);
    uint32_t r1[8], r2[8];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        __half2 qa[2], qb[2];
        i8x4_to_h2(aw[w], qa[0], qa[1]);
        i8x4_to_h2(bw[w], qb[0], qb[1]);
        const float4 c4 = cs.cos4(w);
        const float4 s4 = cs.sin4(w);
        const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
        const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            float2 x1, x2;
            if constexpr (X16 && sizeof(ScaleT) == 2) {
                const __half2 s2 = __half2half2(*reinterpret_cast<const __half*>(&scale));
                x1 = __half22float2(__hmul2_rn(qa[k], s2));
                x2 = __half22float2(__hmul2_rn(qb[k], s2));
            } else {
                const float2 fa = __half22float2(qa[k]);
                const float2 fb = __half22float2(qb[k]);
                x1 = make_float2(__fmul_rn(fa.x, sf), __fmul_rn(fa.y, sf));
                x2 = make_float2(__fmul_rn(fb.x, sf), __fmul_rn(fb.y, sf));
                if constexpr (X16) {
                    x1 = __half22float2(__floats2half2_rn(x1.x, x1.y));
                    x2 = __half22float2(__floats2half2_rn(x2.x, x2.y));
                }
            }
            const float c0 = cv[2 * k], c1 = cv[2 * k + 1], s0 = sv[2 * k], s1 = sv[2 * k + 1];
            float o1a, o1b, o2a, o2b;
            rotate_pair<X16>(x1.x, x2.x, c0, s0, o1a, o2a);
            rotate_pair<X16>(x1.y, x2.y, c1, s1, o1b, o2b);
            r1[w * 2 + k] = pack2<OutT>(o1a, o1b);
            r2[w * 2 + k] = pack2<OutT>(o2a, o2b);
        }
    }
    st_v8(o1, r1);
    st_v8(o2, r2);
}

// 16 value codes -> 16 outputs of cvt(q*s), one 32-byte store.
template <typename OutT, typename ScaleT>
__device__ __forceinline__ void value_slice_store(const uint4& a, ScaleT scale, void* o) {
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
    uint32_t r[8];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        __half2 q[2];
        i8x4_to_h2(aw[w], q[0], q[1]);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            if constexpr (sizeof(ScaleT) == 2 && std::is_same<OutT, __half>::value) {
                const __half2 s2 = __half2half2(*reinterpret_cast<const __half*>(&scale));
                r[w * 2 + k] = u32_of(__hmul2_rn(q[k], s2));
            } else {
                const float sf = scale_to_float<ScaleT>(scale);
                const float2 f = __half22float2(q[k]);
                r[w * 2 + k] = pack2<OutT>(__fmul_rn(f.x, sf), __fmul_rn(f.y, sf));
            }
        }
    }
    st_v8(o, r);
}

}  // namespace sc
