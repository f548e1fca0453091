// sc_quantize.cu — per-(token, head) absmax INT8 quantisation (the offload twin of the
// restore kernels).  Bit-exact with the reference's CPU arithmetic:
//   amax  = max |x| (fp32)
//   scale = fp16(max(amax / 127, eps))      IEEE fp32 division by 127
//   q     = clamp(round_half_even(x / float(scale)), -127, 127)   IEEE fp32 division
//
// Vector path: a row is G lanes x 16 bytes (G = head_dim * sizeof(x) / 16, a power of two
// <= 32); the absmax is reduced with G-lane xor shuffles; each lane writes 16/sizeof(x)
// codes with one store.  Rounding to an integer is done by adding 1.5 * 2^23 (the fp32
// add rounds half to even and leaves the integer in the low mantissa byte), so no
// float->int conversion instruction is needed.
// Generic path: one warp per row, any strides, two passes over the row.
#include <type_traits>

#include "sc_common.cuh"

namespace sc {
namespace {

constexpr int kQThreads = 256;

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

// Unpack one 16-byte vector into E = 16 / sizeof(InT) floats.
template <typename InT>
__device__ __forceinline__ void unpack16(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    if constexpr (std::is_same<InT, float>::value) {
#pragma unroll
        for (int k = 0; k < 4; ++k) f[k] = __uint_as_float(w[k]);
    } else if constexpr (std::is_same<InT, __half>::value) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 p = __half22float2(bit_cast_u32<__half2>(w[k]));
            f[2 * k] = p.x;
            f[2 * k + 1] = p.y;
        }
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            // bf16 -> fp32 is a 16-bit left shift of the bit pattern.
            f[2 * k] = __uint_as_float(w[k] << 16);
            f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
        }
    }
}

__device__ __forceinline__ float quant_scale(float amax, float eps, bool f16_scale) {
    float s = __fdiv_rn(amax, 127.0f);
    s = (s < eps) ? eps : s;  // clamp(min=eps); a NaN stays NaN as in torch.clamp
    return f16_scale ? __half2float(__float2half_rn(s)) : s;
}

// Round-half-even of a value clamped to [-127, 127], returned as the int8 bit pattern.
__device__ __forceinline__ uint32_t code_byte(float x, float scale) {
    float y = __fdiv_rn(x, scale);
    y = fminf(fmaxf(y, -127.0f), 127.0f);
    return __float_as_uint(__fadd_rn(y, 12582912.0f)) & 0xffu;
}

template <typename InT, typename ScaleT>
__global__ void __launch_bounds__(kQThreads) quant_vec(const __grid_constant__ QuantParams p) {
    constexpr int E = 16 / sizeof(InT);
    const int G = p.G;
    const int lane = threadIdx.x % G;
    const int RB = blockDim.x / G;
    constexpr bool kF16Scale = std::is_same<ScaleT, __half>::value;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * RB; base < p.rows;
         base += static_cast<int64_t>(gridDim.x) * RB) {
        const int64_t row = base + threadIdx.x / G;
        const bool active = row < p.rows;
        float f[E];
        int64_t t = 0, h = 0;
        float m = 0.0f;
        if (active) {
            const uint32_t ti = fdiv(static_cast<uint32_t>(row), p.divH);
            t = ti;
            h = static_cast<int64_t>(static_cast<uint32_t>(row) - ti * static_cast<uint32_t>(p.H));
            const InT* xp = reinterpret_cast<const InT*>(p.x) + t * p.x_t + h * p.x_h + lane * E;
            unpack16<InT>(ld_stream_v4(xp), f);
#pragma unroll
            for (int k = 0; k < E; ++k) m = fmaxf(m, fabsf(f[k]));
        }
        for (int o = G >> 1; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (!active) continue;
        const float sc = quant_scale(m, p.eps, kF16Scale);
        uint32_t b[E];
#pragma unroll
        for (int k = 0; k < E; ++k) b[k] = code_byte(f[k], sc);
        int8_t* qp = p.q + t * p.q_t + h * p.q_h + lane * E;
        if constexpr (E == 8) {
            const uint32_t lo = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
            const uint32_t hi = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
            st_v2(qp, make_uint2(lo, hi));
        } else {
            *reinterpret_cast<uint32_t*>(qp) = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
        }
        if (lane == 0) {
            ScaleT* sp = reinterpret_cast<ScaleT*>(p.s) + t * p.s_t + h * p.s_h;
            if constexpr (kF16Scale)
                *sp = __float2half_rn(sc);
            else
                *sp = sc;
        }
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

template <typename InT, typename ScaleT>
cudaError_t launch_quant(const QuantParams& p, bool vec, cudaStream_t stream) {
    const int cap = sm_count() * (2048 / kQThreads);
    if (vec) {
        const int threads = kQThreads;
        const int rb = threads / p.G;
        const int64_t need = (static_cast<int64_t>(p.rows) + rb - 1) / rb;
        const int grid = static_cast<int>(need < cap ? need : cap);
        quant_vec<InT, ScaleT><<<grid, threads, 0, stream>>>(p);
    } else {
        const int64_t need = (static_cast<int64_t>(p.rows) + 7) / 8;
        const int grid = static_cast<int>(need < cap ? need : cap);
        quant_generic<InT, ScaleT><<<grid, kQThreads, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

template <typename InT>
cudaError_t launch_quant_s(const QuantParams& p, bool vec, bool f16_scale, cudaStream_t s) {
    return f16_scale ? launch_quant<InT, __half>(p, vec, s) : launch_quant<InT, float>(p, vec, s);
}

}  // namespace
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
    const int64_t rows = n_tokens * n_heads;
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

    const int es = x_dtype == SC_DTYPE_F32 ? 4 : 2;
    const int E = 16 / es;
    const int64_t row_bytes = static_cast<int64_t>(head_dim) * es;
    int G = static_cast<int>(row_bytes / 16);
    bool vec = !(flags & SC_FLAG_FORCE_GENERIC) && row_bytes % 16 == 0 && G >= 1 && G <= 32 &&
               (G & (G - 1)) == 0;
    auto al = [](const void* ptr, int a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; };
    auto st_ok = [](int64_t st, int64_t size, int64_t a) { return size <= 1 || st % a == 0; };
    if (vec) {
        vec = p.x_d == 1 && al(x, 16) && st_ok(p.x_t * es, n_tokens, 16) &&
              st_ok(p.x_h * es, n_heads, 16) && p.q_d == 1 && al(q_out, E) &&
              st_ok(p.q_t, n_tokens, E) && st_ok(p.q_h, n_heads, E);
    }
    p.G = vec ? G : 32;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool f16s = scale_dtype == SC_DTYPE_F16;
    cudaError_t e;
    switch (x_dtype) {
        case SC_DTYPE_F16: e = launch_quant_s<__half>(p, vec, f16s, s); break;
        case SC_DTYPE_BF16: e = launch_quant_s<__nv_bfloat16>(p, vec, f16s, s); break;
        default: e = launch_quant_s<float>(p, vec, f16s, s); break;
    }
    if (e != cudaSuccess) return cuda_error(e, "quantize launch");
    return ok();
}
