// sc_shift.cu — relative RoPE shift of already dequantised keys (fp16 / bf16 in and out):
// the key rotation of MultiLayerKVInjector.apply_rope_shift
// (speccache/serving/kv_injector.py:246-283), used when keys are injected into the cache
// with a shift (inject_layer_kv, kv_injector.py:285-301).
//
// Arithmetic, as the reference: x in fp32, fp16 cos/sin tables of the shift expanded to
// both halves,
//   out[i]       = cvt(RN(x[i]       * cos[i]) - RN(x[i + D/2] * sin[i]))
//   out[i + D/2] = cvt(RN(x[i + D/2] * cos[i]) + RN(x[i]       * sin[i]))
// with each product and the sum rounded separately (no contraction), so the result equals
// the reference's bit for bit given the same tables, subnormal products included.
//
// Vector path: a thread owns F = 16 (or 8) frequencies of one (token, head) row (packed fp32x2
// arithmetic, two frequencies per instruction): two 32-byte
// (16-byte) loads - the slice and its rotate-half partner - and two stores; one-shot blocks.  The
// table of a host-side shift travels in the kernel parameters and is copied to shared
// memory; device tables ([1 | T, D/2] fp16) are read per row.  Generic path: one thread per
// (row, frequency), any strides.  A thread reads both halves before writing them, so the
// shift may run in place (out == x with the same strides).
#include "sc_common.cuh"

namespace sc {
namespace {

// Threads per block.  Smaller one-shot blocks start streaming sooner after the table copy
// and barrier: 32 layers of Llama-3-8B keys take 156 us with 64- or 128-thread blocks, 167 us
// with 256, 175 us with 512 and 193 us with 1024.
#ifndef SC_SHIFT_THREADS
#define SC_SHIFT_THREADS 128
#endif
constexpr int kSThreads = SC_SHIFT_THREADS;
// Widest vector slice (frequencies per thread) the launcher may pick: 16 or 8.
#ifndef SC_SHIFT_MAX_F
#define SC_SHIFT_MAX_F 16
#endif

struct ShiftParams {
    int32_t rows;  // n_tokens * n_heads (< 2^31)
    int32_t H, D, S;  // S = (D / 2) / F slices of F frequencies per row (vector path)
    FastDiv divH, divS;
    const void* x;
    int64_t x_t, x_h, x_d;
    void* out;
    int64_t o_t, o_h, o_d;
    const __half* cos;  // device tables, or null: host table in `tab`
    const __half* sin;
    int64_t cs_t, cs_d;
    uint32_t tab[kMaxHeadDim / 2];  // half2(cos, sin) per frequency
};

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__half>(__half v) {
    return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}

// Two packed 16-bit values as floats (exact).
template <typename T>
__device__ __forceinline__ float2 to_f2(uint32_t w);
template <>
__device__ __forceinline__ float2 to_f2<__half>(uint32_t w) {
    return __half22float2(bit_cast_u32<__half2>(w));
}
template <>
__device__ __forceinline__ float2 to_f2<__nv_bfloat16>(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ void shift_pair(float x1, float x2, float c, float s, float& o1,
                                           float& o2) {
    o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
}

// 16 consecutive 16-bit values (32 bytes, 32-byte aligned).  A plain (coherent) load: the
// shift may run in place.
__device__ __forceinline__ void ld_v8(const void* p, uint32_t* w) {
    asm volatile("ld.global.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]),
                   "=r"(w[6]), "=r"(w[7])
                 : "l"(p));
}

// F consecutive 16-bit values (F = 8: one 16-byte access, F = 16: one 32-byte access).
template <int F>
__device__ __forceinline__ void load_f(const void* p, uint32_t* w) {
    if constexpr (F == 16) {
        ld_v8(p, w);
    } else {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
    }
}

template <int F>
__device__ __forceinline__ void store_f(void* p, uint32_t* w) {
    if constexpr (F == 16) {
        st_v8(p, *reinterpret_cast<const uint32_t(*)[8]>(w));
    } else {
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

template <typename InT, typename OutT, int F>
__global__ void __launch_bounds__(kSThreads) shift_vec(const __grid_constant__ ShiftParams p) {
    constexpr int NW = F / 2;  // 32-bit words per half-slice
    __shared__ __align__(16) float s_cos[kMaxHeadDim / 2];
    __shared__ __align__(16) float s_sin[kMaxHeadDim / 2];
    const int half = p.D >> 1;
    if (p.cos == nullptr) {
        for (int f = threadIdx.x; f < half; f += blockDim.x) {
            const __half2 cs = bit_cast_u32<__half2>(p.tab[f]);
            s_cos[f] = __low2float(cs);
            s_sin[f] = __high2float(cs);
        }
        __syncthreads();
    }
    const int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (w >= static_cast<int64_t>(p.rows) * p.S) return;
    const uint32_t row = fdiv(static_cast<uint32_t>(w), p.divS);
    const int j = static_cast<int>(static_cast<uint32_t>(w) - row * static_cast<uint32_t>(p.S));
    const uint32_t t = fdiv(row, p.divH);
    const int64_t h = static_cast<int64_t>(row) - static_cast<int64_t>(t) * p.H;
    const int f0 = j * F;
    const InT* xp = reinterpret_cast<const InT*>(p.x) + t * p.x_t + h * p.x_h + f0;
    uint32_t aw[NW], bw[NW];
    load_f<F>(xp, aw);
    load_f<F>(xp + half, bw);
    uint32_t cw[NW], sw[NW];
    if (p.cos != nullptr) {
        load_f<F>(p.cos + t * p.cs_t + f0, cw);
        load_f<F>(p.sin + t * p.cs_t + f0, sw);
    }
    uint32_t lo[NW], hi[NW];
#pragma unroll
    for (int k = 0; k < NW; ++k) {
        // Two frequencies at once in packed fp32x2: each product and sum is still rounded
        // once (RN), as in shift_pair; x2 * (-s) = -(x2 * s) exactly.
        float2 c, ns, s;
        if (p.cos == nullptr) {
            c = *reinterpret_cast<const float2*>(&s_cos[f0 + 2 * k]);
            s = *reinterpret_cast<const float2*>(&s_sin[f0 + 2 * k]);
        } else {
            c = __half22float2(bit_cast_u32<__half2>(cw[k]));
            s = __half22float2(bit_cast_u32<__half2>(sw[k]));
        }
        ns = make_float2(-s.x, -s.y);
        const float2 a = to_f2<InT>(aw[k]), b = to_f2<InT>(bw[k]);
        const float2 o1 = __fadd2_rn(__fmul2_rn(a, c), __fmul2_rn(b, ns));
        const float2 o2 = __fadd2_rn(__fmul2_rn(b, c), __fmul2_rn(a, s));
        lo[k] = pack2<OutT>(o1.x, o1.y);
        hi[k] = pack2<OutT>(o2.x, o2.y);
    }
    OutT* op = reinterpret_cast<OutT*>(p.out) + t * p.o_t + h * p.o_h + f0;
    store_f<F>(op, lo);
    store_f<F>(op + half, hi);
}

template <typename InT, typename OutT>
__global__ void __launch_bounds__(kSThreads) shift_generic(const __grid_constant__ ShiftParams p) {
    const int half = p.D >> 1;
    const int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (w >= static_cast<int64_t>(p.rows) * half) return;
    const int64_t row = w / half;
    const int f = static_cast<int>(w - row * half);
    const int64_t t = row / p.H, h = row - t * p.H;
    const InT* xp = reinterpret_cast<const InT*>(p.x) + t * p.x_t + h * p.x_h;
    float c, s;
    if (p.cos == nullptr) {
        const __half2 cs = bit_cast_u32<__half2>(p.tab[f]);
        c = __low2float(cs);
        s = __high2float(cs);
    } else {
        c = __half2float(p.cos[t * p.cs_t + f * p.cs_d]);
        s = __half2float(p.sin[t * p.cs_t + f * p.cs_d]);
    }
    float o1, o2;
    shift_pair(to_f(xp[f * p.x_d]), to_f(xp[(f + half) * p.x_d]), c, s, o1, o2);
    OutT* op = reinterpret_cast<OutT*>(p.out) + t * p.o_t + h * p.o_h;
    op[f * p.o_d] = from_float<OutT>(o1);
    op[(f + half) * p.o_d] = from_float<OutT>(o2);
}

// width: frequencies per thread of the vector path (16 or 8), or 0 for the generic path.
template <typename InT, typename OutT>
cudaError_t launch_shift(const ShiftParams& p, int width, cudaStream_t stream) {
    const int64_t work = static_cast<int64_t>(p.rows) * (width ? p.S : p.D / 2);
    const unsigned blocks = static_cast<unsigned>((work + kSThreads - 1) / kSThreads);
    if (width == 16)
        shift_vec<InT, OutT, 16><<<blocks, kSThreads, 0, stream>>>(p);
    else if (width == 8)
        shift_vec<InT, OutT, 8><<<blocks, kSThreads, 0, stream>>>(p);
    else
        shift_generic<InT, OutT><<<blocks, kSThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

template <typename InT>
cudaError_t launch_shift_in(const ShiftParams& p, int32_t out_dtype, int width, cudaStream_t s) {
    return out_dtype == SC_DTYPE_F16 ? launch_shift<InT, __half>(p, width, s)
                                     : launch_shift<InT, __nv_bfloat16>(p, width, s);
}

template <typename InT, typename OutT>
cudaError_t preload_shift_io() {
    cudaFuncAttributes attr;
    cudaError_t e = cudaFuncGetAttributes(&attr, shift_vec<InT, OutT, 16>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, shift_vec<InT, OutT, 8>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, shift_generic<InT, OutT>);
    return e;
}

}  // namespace

cudaError_t preload_shift_kernels() {
    cudaError_t e = preload_shift_io<__half, __half>();
    if (e == cudaSuccess) e = preload_shift_io<__half, __nv_bfloat16>();
    if (e == cudaSuccess) e = preload_shift_io<__nv_bfloat16, __half>();
    if (e == cudaSuccess) e = preload_shift_io<__nv_bfloat16, __nv_bfloat16>();
    return e;
}

}  // namespace sc

using namespace sc;

extern "C" int32_t sc_rope_shift_keys(int64_t n_tokens, int32_t n_heads, int32_t head_dim,
                                      const void* x, int32_t x_dtype, const int64_t* x_strides,
                                      const void* cos_delta, const void* sin_delta,
                                      const int64_t* cs_strides, double delta_p,
                                      double theta_base, const float* inv_freq, void* out,
                                      int32_t out_dtype, const int64_t* out_strides,
                                      void* stream) {
    if (n_tokens < 0 || n_heads < 0 || head_dim < 0)
        return set_error(SC_ERR_INVALID_ARGUMENT, "negative size");
    if (head_dim % 2 != 0)
        return set_error(SC_ERR_INVALID_ARGUMENT, "head_dim must be even, got %d", head_dim);
    if (head_dim > kMaxHeadDim)
        return set_error(SC_ERR_UNSUPPORTED, "head_dim %d exceeds %d", head_dim, kMaxHeadDim);
    for (int32_t dt : {x_dtype, out_dtype})
        if (dt != SC_DTYPE_F16 && dt != SC_DTYPE_BF16)
            return set_error(SC_ERR_INVALID_DTYPE, "key dtype code %d: float16 or bfloat16", dt);
    const int64_t rows = size_product(n_tokens, n_heads);
    if (rows >= (int64_t(1) << 31) / (head_dim > 2 ? head_dim / 2 : 1))
        return set_error(SC_ERR_INVALID_ARGUMENT, "%lld rows in one call; split it",
                         (long long)rows);
    if (rows == 0 || head_dim == 0) return ok();
    if (!x || !out || !x_strides || !out_strides)
        return set_error(SC_ERR_INVALID_ARGUMENT, "null pointer argument");
    if ((cos_delta == nullptr) != (sin_delta == nullptr))
        return set_error(SC_ERR_INVALID_ARGUMENT, "give both cos and sin tables or neither");
    if (cos_delta && !cs_strides)
        return set_error(SC_ERR_INVALID_ARGUMENT, "null table strides");

    ShiftParams p{};
    p.rows = static_cast<int32_t>(rows);
    p.H = n_heads;
    p.D = head_dim;
    p.divH = make_fastdiv(static_cast<uint32_t>(n_heads));
    p.x = x;
    p.x_t = x_strides[0], p.x_h = x_strides[1], p.x_d = x_strides[2];
    p.out = out;
    p.o_t = out_strides[0], p.o_h = out_strides[1], p.o_d = out_strides[2];
    p.cos = static_cast<const __half*>(cos_delta);
    p.sin = static_cast<const __half*>(sin_delta);
    if (cos_delta) {
        p.cs_t = cs_strides[0], p.cs_d = cs_strides[1];
    } else {
        host_cos_sin_table(head_dim, static_cast<float>(delta_p), theta_base, inv_freq, p.tab);
    }
    // Vector path: 16 (or 8) frequencies per thread, 32-byte (16-byte) aligned slices of x,
    // out and the tables; otherwise the generic path.
    const int half = head_dim / 2;
    auto fits = [&](int f) {
        const int bytes = 2 * f;
        auto al = [&](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) % bytes) == 0; };
        auto st = [&](int64_t stride, int64_t size) { return size <= 1 || stride % f == 0; };
        bool ok = half % f == 0 && p.x_d == 1 && p.o_d == 1 && al(x) && al(out) &&
                  st(p.x_t, n_tokens) && st(p.x_h, n_heads) && st(p.o_t, n_tokens) &&
                  st(p.o_h, n_heads);
        if (ok && cos_delta)
            ok = p.cs_d == 1 && al(cos_delta) && al(sin_delta) && st(p.cs_t, n_tokens);
        return ok;
    };
    const int width = SC_SHIFT_MAX_F >= 16 && fits(16) ? 16 : (fits(8) ? 8 : 0);
    p.S = width ? half / width : 1;
    p.divS = make_fastdiv(static_cast<uint32_t>(p.S));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaError_t e = x_dtype == SC_DTYPE_F16
                              ? launch_shift_in<__half>(p, out_dtype, width, s)
                              : launch_shift_in<__nv_bfloat16>(p, out_dtype, width, s);
    if (e != cudaSuccess) return cuda_error(e, "key shift launch");
    return ok();
}
