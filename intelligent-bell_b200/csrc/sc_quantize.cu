// sc_quantize.cu — per-(token, head) absmax INT8 quantisation (the offload twin of the
// restore kernels).  Bit-exact with the reference's CPU arithmetic:
//   amax  = max |x| (fp32)
//   scale = fp16(max(amax / 127, eps))      IEEE fp32 division by 127
//   q     = clamp(round_half_even(x / float(scale)), -127, 127)   IEEE fp32 division
//
// Vector path: a row is G lanes x V x 32 bytes (G = head_dim * sizeof(x) / (32 V), a power of
// two <= 32, V 256-bit loads per lane); the absmax is reduced with G-lane xor shuffles; each
// lane writes 32 V / sizeof(x) codes with 32-byte (or smaller) stores.  Codes come from packed
// fp32x2 arithmetic; rounding to an integer is done by adding 1.5 * 2^23 (the fp32 add rounds
// half to even and leaves the integer in the low mantissa byte).  For fp16/bf16 inputs with
// fp16 scales, two products that bracket x / scale give the exact code with no tie test
// (pair_codes2); otherwise x * (1/scale) is exact unless the quotient lies within 2^-14 of a
// half-integer, where the lane redoes the IEEE division (fast_codes2).
// Generic path: one warp per row, any strides, two passes over the row.
#include <type_traits>

#include "sc_common.cuh"

namespace sc {
namespace {

// Threads per block of the generic path.
constexpr int kQThreads = 256;
// Vector path, per input width: threads per block and the grid (1: capped at the resident
// blocks, each block walking rows with a grid stride; 0: one block per tile of rows).
// Measured on [458,752 tokens, 4, 128] (us, fp16 / bf16 / fp32 input): 256 threads capped
// 109.5 / 108.6 / 182.5; 128 threads one block per tile 106.2 / 106.9 / 193.0; 128 capped
// 117.5 / 116.5 / 183.0; 256 one block per tile 113.1 / 114.7 / 205.8.
#ifndef SC_QUANT_THREADS_16
#define SC_QUANT_THREADS_16 128
#endif
#ifndef SC_QUANT_GRID_CAP_16
#define SC_QUANT_GRID_CAP_16 0
#endif
#ifndef SC_QUANT_THREADS_32
#define SC_QUANT_THREADS_32 256
#endif
#ifndef SC_QUANT_GRID_CAP_32
#define SC_QUANT_GRID_CAP_32 1
#endif
template <typename InT>
struct QuantShape {
    static constexpr bool k32 = std::is_same<InT, float>::value;
    static constexpr int threads = k32 ? SC_QUANT_THREADS_32 : SC_QUANT_THREADS_16;
    static constexpr bool cap = k32 ? SC_QUANT_GRID_CAP_32 : SC_QUANT_GRID_CAP_16;
};

#ifndef SC_QUANT_MAX_V
#define SC_QUANT_MAX_V 2
#endif
// Resident blocks per SM the vector kernel is compiled for, per input type (the register
// cap follows; 0 leaves the register count to the compiler).
#ifndef SC_QUANT_MB_F16
#define SC_QUANT_MB_F16 0
#endif
#ifndef SC_QUANT_MB_BF16
#define SC_QUANT_MB_BF16 0
#endif
#ifndef SC_QUANT_MB_F32
#define SC_QUANT_MB_F32 1
#endif
template <typename InT>
struct QuantMinBlocks {
    static constexpr int value = std::is_same<InT, __half>::value           ? SC_QUANT_MB_F16
                                 : std::is_same<InT, __nv_bfloat16>::value ? SC_QUANT_MB_BF16
                                                                           : SC_QUANT_MB_F32;
};
static_assert(SC_QUANT_MAX_V == 1 || SC_QUANT_MAX_V == 2 || SC_QUANT_MAX_V == 4,
              "SC_QUANT_MAX_V is 1, 2 or 4");

struct QuantParams {
    int32_t rows;  // n_tokens * n_heads (< 2^31)
    int32_t H, D, G;
    FastDiv divH;
    const void* x;
    int64_t x_t, x_h, x_d;
    int8_t* q;
    int64_t q_t, q_h, q_d;
    void* s;
    int64_t s_t, s_h;
    float eps;
};

template <typename InT>
__device__ __forceinline__ float in_to_float(InT v);
template <>
__device__ __forceinline__ float in_to_float<__half>(__half v) {
    return __half2float(v);
}
template <>
__device__ __forceinline__ float in_to_float<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float in_to_float<float>(float v) {
    return v;
}

__device__ __forceinline__ float quant_scale(float amax, float eps, bool f16_scale) {
    float s = __fdiv_rn(amax, 127.0f);
    s = (s < eps) ? eps : s;  // clamp(min=eps); a NaN stays NaN as in torch.clamp
    return f16_scale ? __half2float(__float2half_rn(s)) : s;
}

// int8 bit pattern of round_half_even(clamp(y, -127, 127)): adding 1.5 * 2^23 rounds to an
// integer (half to even) and leaves it in the low mantissa byte.
__device__ __forceinline__ uint32_t byte_of(float y) {
    y = fminf(fmaxf(y, -127.0f), 127.0f);
    return __float_as_uint(__fadd_rn(y, 12582912.0f)) & 0xffu;
}

// Exact code: IEEE division, as the reference (clamping before or after rounding gives the
// same integer in [-127, 127]).
__device__ __forceinline__ uint32_t code_byte(float x, float scale) {
    return byte_of(__fdiv_rn(x, scale));
}

// Fast codes.  y = RN(x * RN(1/scale)) is within 2^-16 of the true quotient x / scale
// whenever |x / scale| < 128 (two roundings of 2^-24 relative each), and RN(x / scale)
// is within half an ulp (<= 2^-18) of the true quotient, so when y is farther than
// kTieBand from every half-integer both round to the same integer.  Scales outside
// [2^-126, 2^125] (whose reciprocal would be subnormal, with fewer bits) always take the
// exact path.  For a finite row the
// quotient is also below 127.5 in magnitude (the fp16 scale is amax/127 up to a relative
// 2^-11, or 0.3 % in the fp16 subnormal range, or the larger eps), so the rounded value
// needs no clamp.  n = (y + 1.5*2^23) - 1.5*2^23 is y rounded half to even, the sum's
// low byte is n as int8, and |y - n| > 0.5 - kTieBand flags a quotient near a half-integer,
// for which the caller redoes the IEEE division.
constexpr float kTieBand = 6.103515625e-05f;  // 2^-14
constexpr float kRound = 12582912.0f;          // 1.5 * 2^23

__device__ __forceinline__ void fast_codes2(float2 x, float2 rcp2, uint32_t& t0, uint32_t& t1,
                                            bool& tie) {
    const float2 m2 = make_float2(kRound, kRound);
    const float2 y = __fmul2_rn(x, rcp2);
    const float2 t = __fadd2_rn(y, m2);
    const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
    const float2 r = __fadd2_rn(y, make_float2(-n.x, -n.y));
    tie |= fabsf(r.x) > 0.5f - kTieBand;
    tie |= fabsf(r.y) > 0.5f - kTieBand;
    t0 = __float_as_uint(t.x);
    t1 = __float_as_uint(t.y);
}

// Codes for 16-bit inputs with fp16 scales, with no tie test.  x and s have at most 11
// significant bits, so x - (m + 1/2) s is a multiple of min(ulp(x), ulp(s) / 2): a quotient
// q = x / s (|q| <= 127.5) that is not itself a half-integer lies at least 2^-19 |q| from
// every half-integer.  rcp_lo and rcp_hi bracket 1 / s within 1.5 * 2^-22 relative
// (rcp_lo * s < 1 < rcp_hi * s), so the exact products x * rcp_lo and x * rcp_hi (one fma
// each, rounded to an integer by adding 1.5 * 2^23) both round to the integer nearest q
// unless q is exactly a half-integer, when they are its two neighbours.  t1 + t2 then lies
// in [2^24, 2^25), where the fp32 grid step is 2: the sum is exact when t1 = t2 and rounds
// half to even onto 2 * (the even neighbour) otherwise, which is rint_even(q) either way.
// RN(x / s) rounds to the same integer because it is within 2^-24 |q| of q.  The low byte
// of the sum's bits is that integer as int8 (the sum is 2^24 + 2 * (2^22 + n)).
constexpr float kPairLo = 0x1.fffff8p-1f;  // 1 - 2^-22
constexpr float kPairHi = 0x1.000004p+0f;  // 1 + 2^-22

__device__ __forceinline__ void pair_codes2(float2 x, float2 lo2, float2 hi2, uint32_t& c0,
                                            uint32_t& c1) {
    const float2 m2 = make_float2(kRound, kRound);
    const float2 s = __fadd2_rn(__ffma2_rn(x, lo2, m2), __ffma2_rn(x, hi2, m2));
    c0 = __float_as_uint(s.x);
    c1 = __float_as_uint(s.y);
}

// Low bytes of four words -> one word.
__device__ __forceinline__ uint32_t pack_low_bytes(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// 32-byte non-coherent load (one 256-bit access; the address must be 32-byte aligned).
__device__ __forceinline__ void ld_stream_v8(const void* p, uint32_t* w) {
    asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]),
                   "=r"(w[6]), "=r"(w[7])
                 : "l"(p));
}

// Largest |x| of the elements packed in w (fp32 words or 16-bit pairs).  For 16-bit types
// the maximum is taken in the input type, which is exact (widening to fp32 is monotone).
template <typename InT, int NW>
__device__ __forceinline__ float lane_absmax(const uint32_t (&w)[NW]) {
    if constexpr (std::is_same<InT, float>::value) {
        float m = 0.0f;
#pragma unroll
        for (int k = 0; k < NW; ++k) m = fmaxf(m, fabsf(__uint_as_float(w[k])));
        return m;
    } else if constexpr (std::is_same<InT, __half>::value) {
        __half2 m = __habs2(bit_cast_u32<__half2>(w[0]));
#pragma unroll
        for (int k = 1; k < NW; ++k) m = __hmax2(m, __habs2(bit_cast_u32<__half2>(w[k])));
        return fmaxf(__low2float(m), __high2float(m));
    } else {
        __nv_bfloat162 m = __habs2(*reinterpret_cast<const __nv_bfloat162*>(&w[0]));
#pragma unroll
        for (int k = 1; k < NW; ++k)
            m = __hmax2(m, __habs2(*reinterpret_cast<const __nv_bfloat162*>(&w[k])));
        return fmaxf(__low2float(m), __high2float(m));
    }
}

// Elements k and k+1 (k even) of the packed words as floats.
template <typename InT>
__device__ __forceinline__ float2 pair_at(const uint32_t* w, int k) {
    if constexpr (std::is_same<InT, float>::value) {
        return make_float2(__uint_as_float(w[k]), __uint_as_float(w[k + 1]));
    } else if constexpr (std::is_same<InT, __half>::value) {
        return __half22float2(bit_cast_u32<__half2>(w[k / 2]));
    } else {
        // bf16 -> fp32 is a 16-bit left shift of the bit pattern.
        const uint32_t u = w[k / 2];
        return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
    }
}

// The lane's V x 32 input bytes of `row` into w, and the row's token and head.
template <typename InT, int V>
__device__ __forceinline__ void fetch_row(const QuantParams& p, int64_t row, int lane,
                                          uint32_t* w, int64_t& t, int64_t& h) {
    constexpr int E = 32 * V / static_cast<int>(sizeof(InT));
    const uint32_t ti = fdiv(static_cast<uint32_t>(row), p.divH);
    t = ti;
    h = static_cast<int64_t>(static_cast<uint32_t>(row) - ti * static_cast<uint32_t>(p.H));
    const char* xp = reinterpret_cast<const char*>(
        reinterpret_cast<const InT*>(p.x) + t * p.x_t + h * p.x_h + lane * E);
#pragma unroll
    for (int v = 0; v < V; ++v) ld_stream_v8(xp + 32 * v, w + 8 * v);
}

// Codes and scale of one row from the lane's words w and the row's absmax m.
template <typename InT, typename ScaleT, int V>
__device__ __forceinline__ void convert_store(const QuantParams& p, uint32_t* w, float m,
                                              int64_t t, int64_t h, int lane) {
    constexpr int E = 32 * V / static_cast<int>(sizeof(InT));
    constexpr bool kF16Scale = std::is_same<ScaleT, __half>::value;
    // 16-bit input and fp16 scale: two-product rule, no tie test (pair_codes2)
    constexpr bool kPairRule = kF16Scale && !std::is_same<InT, float>::value;
    const float sc = quant_scale(m, p.eps, kF16Scale);
    const float rcp = __frcp_rn(sc);
    // zero, tiny, huge or non-finite scale: exact path
    bool tie = !(sc >= 0x1p-126f && sc <= 0x1p125f);
    // Codes are packed four to a word as they are made, so only the packed words stay live.
    uint32_t packed[E / 4];
    if constexpr (kPairRule) {
        const float lo = __fmul_rn(rcp, kPairLo), hi = __fmul_rn(rcp, kPairHi);
        const float2 lo2 = make_float2(lo, lo), hi2 = make_float2(hi, hi);
#pragma unroll
        for (int k = 0; k < E; k += 4) {
            uint32_t c0, c1, c2, c3;
            pair_codes2(pair_at<InT>(w, k), lo2, hi2, c0, c1);
            pair_codes2(pair_at<InT>(w, k + 2), lo2, hi2, c2, c3);
            packed[k / 4] = pack_low_bytes(c0, c1, c2, c3);
        }
    } else {
        const float2 rcp2 = make_float2(rcp, rcp);
#pragma unroll
        for (int k = 0; k < E; k += 4) {
            uint32_t c0, c1, c2, c3;
            fast_codes2(pair_at<InT>(w, k), rcp2, c0, c1, tie);
            fast_codes2(pair_at<InT>(w, k + 2), rcp2, c2, c3, tie);
            packed[k / 4] = pack_low_bytes(c0, c1, c2, c3);
        }
    }
    if (tie) {  // rare: reload the lane's input (keeps the fast path's registers free)
        int64_t t2, h2;
        fetch_row<InT, V>(p, t * p.H + h, lane, w, t2, h2);
#pragma unroll
        for (int k = 0; k < E; k += 4) {
            const float2 x0 = pair_at<InT>(w, k), x1 = pair_at<InT>(w, k + 2);
            packed[k / 4] = pack_low_bytes(code_byte(x0.x, sc), code_byte(x0.y, sc),
                                           code_byte(x1.x, sc), code_byte(x1.y, sc));
        }
    }
    int8_t* qp = p.q + t * p.q_t + h * p.q_h + lane * E;
    if constexpr (E >= 32) {
#pragma unroll
        for (int c = 0; c < E / 32; ++c)
            st_v8(qp + 32 * c, *reinterpret_cast<const uint32_t(*)[8]>(packed + 8 * c));
    } else if constexpr (E == 16) {
        st_v4(qp, make_uint4(packed[0], packed[1], packed[2], packed[3]));
    } else {
        st_v2(qp, make_uint2(packed[0], packed[1]));
    }
    if (lane == 0) {
        ScaleT* sp = reinterpret_cast<ScaleT*>(p.s) + t * p.s_t + h * p.s_h;
        if constexpr (kF16Scale)
            *sp = __float2half_rn(sc);
        else
            *sp = sc;
    }
}

// Vector path: each lane owns V x 32 bytes of a row (E = 32 V / sizeof(x) elements, V
// 256-bit loads in flight per lane); G lanes (a power of two <= 32) cover the row.  Larger
// V shares the per-row work (scale, reciprocal, shuffles, addressing) among more elements.
template <typename InT, typename ScaleT, int V>
__global__ void __launch_bounds__(QuantShape<InT>::threads, QuantMinBlocks<InT>::value)
    quant_vec(const __grid_constant__ QuantParams p) {
    constexpr int NW = 8 * V;
    const int G = p.G;
    const int lane = threadIdx.x % G;
    const int RB = blockDim.x / G;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * RB;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * RB; base < p.rows; base += stride) {
        const int64_t row = base + threadIdx.x / G;
        const bool active = row < p.rows;
        uint32_t w[NW];
        int64_t t = 0, h = 0;
        float m = 0.0f;
        if (active) {
            fetch_row<InT, V>(p, row, lane, w, t, h);
            m = lane_absmax<InT>(w);
        }
        for (int o = G >> 1; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (active) convert_store<InT, ScaleT, V>(p, w, m, t, h, lane);
    }
}

template <typename InT, typename ScaleT>
__global__ void __launch_bounds__(kQThreads) quant_generic(const __grid_constant__ QuantParams p) {
    constexpr bool kF16Scale = std::is_same<ScaleT, __half>::value;
    const int warps = blockDim.x / 32;
    const int lane = threadIdx.x & 31;
    for (int64_t row = static_cast<int64_t>(blockIdx.x) * warps + threadIdx.x / 32; row < p.rows;
         row += static_cast<int64_t>(gridDim.x) * warps) {
        const int64_t t = row / p.H, h = row % p.H;
        const InT* xp = reinterpret_cast<const InT*>(p.x) + t * p.x_t + h * p.x_h;
        float m = 0.0f;
        for (int d = lane; d < p.D; d += 32) m = fmaxf(m, fabsf(in_to_float<InT>(xp[d * p.x_d])));
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        const float sc = quant_scale(m, p.eps, kF16Scale);
        int8_t* qp = p.q + t * p.q_t + h * p.q_h;
        for (int d = lane; d < p.D; d += 32)
            qp[d * p.q_d] = static_cast<int8_t>(code_byte(in_to_float<InT>(xp[d * p.x_d]), sc));
        if (lane == 0) {
            ScaleT* sp = reinterpret_cast<ScaleT*>(p.s) + t * p.s_t + h * p.s_h;
            if constexpr (kF16Scale)
                *sp = __float2half_rn(sc);
            else
                *sp = sc;
        }
    }
}

template <typename K>
int resident_blocks(K kernel, int threads) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, 0) != cudaSuccess || n <= 0)
        n = 1;
    return n;
}

// Grids are sized to the work, capped (cap = true) at exactly the resident blocks (no
// partial wave).
template <typename K>
cudaError_t launch_rows(K kern, const QuantParams& p, int threads, int rows_per_block, bool cap,
                        cudaStream_t stream) {
    const int64_t need = (static_cast<int64_t>(p.rows) + rows_per_block - 1) / rows_per_block;
    const int64_t lim = cap ? static_cast<int64_t>(sm_count()) * resident_blocks(kern, threads) : need;
    kern<<<static_cast<int>(need < lim ? need : lim), threads, 0, stream>>>(p);
    return cudaGetLastError();
}

// v = 0: generic path; v = 1, 2, 4: vector path with v 32-byte vectors per lane.
template <typename InT, typename ScaleT>
cudaError_t launch_quant(const QuantParams& p, int v, cudaStream_t stream) {
    constexpr int T = QuantShape<InT>::threads;
    constexpr bool C = QuantShape<InT>::cap;
    const int rb = T / p.G;
    switch (v) {
        case 1: return launch_rows(quant_vec<InT, ScaleT, 1>, p, T, rb, C, stream);
        case 2: return launch_rows(quant_vec<InT, ScaleT, 2>, p, T, rb, C, stream);
        case 4: return launch_rows(quant_vec<InT, ScaleT, 4>, p, T, rb, C, stream);
        default: return launch_rows(quant_generic<InT, ScaleT>, p, kQThreads, kQThreads / 32, true, stream);
    }
}

template <typename InT>
cudaError_t launch_quant_s(const QuantParams& p, int v, bool f16_scale, cudaStream_t s) {
    return f16_scale ? launch_quant<InT, __half>(p, v, s) : launch_quant<InT, float>(p, v, s);
}

template <typename InT, typename ScaleT>
cudaError_t preload_quant_in() {
    cudaFuncAttributes attr;
    cudaError_t e = cudaFuncGetAttributes(&attr, quant_vec<InT, ScaleT, 1>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, quant_vec<InT, ScaleT, 2>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, quant_vec<InT, ScaleT, 4>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, quant_generic<InT, ScaleT>);
    return e;
}

}  // namespace

cudaError_t preload_quantize_kernels(bool f32_scales) {
    cudaError_t e = preload_quant_in<__half, __half>();
    if (e == cudaSuccess) e = preload_quant_in<__nv_bfloat16, __half>();
    if (e == cudaSuccess) e = preload_quant_in<float, __half>();
    if (f32_scales) {
        if (e == cudaSuccess) e = preload_quant_in<__half, float>();
        if (e == cudaSuccess) e = preload_quant_in<__nv_bfloat16, float>();
        if (e == cudaSuccess) e = preload_quant_in<float, float>();
    }
    return e;
}

}  // namespace sc

using namespace sc;

extern "C" int32_t sc_quantize_int8(int64_t n_tokens, int32_t n_heads, int32_t head_dim,
                                    const void* x, int32_t x_dtype, const int64_t* x_strides,
                                    float eps, int8_t* q_out, const int64_t* q_strides,
                                    void* scale_out, int32_t scale_dtype,
                                    const int64_t* s_strides, uint32_t flags, void* stream) {
    if (n_tokens < 0 || n_heads < 0 || head_dim < 0)
        return set_error(SC_ERR_INVALID_ARGUMENT, "negative size");
    if (x_dtype != SC_DTYPE_F16 && x_dtype != SC_DTYPE_BF16 && x_dtype != SC_DTYPE_F32)
        return set_error(SC_ERR_INVALID_DTYPE, "input dtype code %d: float16/bfloat16/float32",
                         x_dtype);
    if (scale_dtype != SC_DTYPE_F16 && scale_dtype != SC_DTYPE_F32)
        return set_error(SC_ERR_INVALID_DTYPE, "scale dtype code %d: float16 or float32",
                         scale_dtype);
    const int64_t rows = size_product(n_tokens, n_heads);
    if (rows >= (int64_t(1) << 31))
        return set_error(SC_ERR_INVALID_ARGUMENT, "%lld rows; split the call below 2^31",
                         (long long)rows);
    if (rows == 0 || head_dim == 0) {
        if (rows != 0 && head_dim == 0)
            return set_error(SC_ERR_INVALID_ARGUMENT, "head_dim must be positive");
        return ok();
    }
    if (!x || !q_out || !scale_out || !x_strides || !q_strides || !s_strides)
        return set_error(SC_ERR_INVALID_ARGUMENT, "null pointer argument");

    QuantParams p{};
    p.rows = static_cast<int32_t>(rows);
    p.H = n_heads;
    p.D = head_dim;
    p.divH = make_fastdiv(static_cast<uint32_t>(n_heads));
    p.x = x;
    p.x_t = x_strides[0], p.x_h = x_strides[1], p.x_d = x_strides[2];
    p.q = q_out;
    p.q_t = q_strides[0], p.q_h = q_strides[1], p.q_d = q_strides[2];
    p.s = scale_out;
    p.s_t = s_strides[0], p.s_h = s_strides[1];
    p.eps = eps;

    // Vector path: V x 32 bytes of input per lane (V 256-bit loads), G = row_bytes / (32 V)
    // lanes per row (a power of two <= 32), 32-byte aligned input rows, code rows aligned to
    // the lane's store (E = 32 V / sizeof(x) bytes, at most 32).  The largest V that fits
    // (up to SC_QUANT_MAX_V) is taken.
    const int es = x_dtype == SC_DTYPE_F32 ? 4 : 2;
    const int64_t row_bytes = static_cast<int64_t>(head_dim) * es;
    auto al = [](const void* ptr, int a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
    auto st_ok = [](int64_t st, int64_t size, int64_t a) { return size <= 1 || st % a == 0; };
    const bool in_ok = p.x_d == 1 && al(x, 32) && st_ok(p.x_t * es, n_tokens, 32) &&
                       st_ok(p.x_h * es, n_heads, 32) && p.q_d == 1;
    int v = 0;
    for (int cand = SC_QUANT_MAX_V; cand >= 1 && v == 0 && in_ok && !(flags & SC_FLAG_FORCE_GENERIC);
         cand /= 2) {
        const int64_t lane_bytes = 32 * cand;
        const int64_t g = row_bytes / lane_bytes;
        const int qa = static_cast<int>(lane_bytes / es < 32 ? lane_bytes / es : 32);
        if (row_bytes % lane_bytes == 0 && g >= 1 && g <= 32 && (g & (g - 1)) == 0 &&
            al(q_out, qa) && st_ok(p.q_t, n_tokens, qa) && st_ok(p.q_h, n_heads, qa)) {
            v = cand;
            p.G = static_cast<int>(g);
        }
    }
    if (v == 0) p.G = 32;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool f16s = scale_dtype == SC_DTYPE_F16;
    cudaError_t e;
    switch (x_dtype) {
        case SC_DTYPE_F16: e = launch_quant_s<__half>(p, v, f16s, s); break;
        case SC_DTYPE_BF16: e = launch_quant_s<__nv_bfloat16>(p, v, f16s, s); break;
        default: e = launch_quant_s<float>(p, v, f16s, s); break;
    }
    if (e != cudaSuccess) return cuda_error(e, "quantize launch");
    return ok();
}
