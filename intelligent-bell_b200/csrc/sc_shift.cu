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
// Vector path: a thread owns 8 frequencies of one (token, head) row: two 16-byte loads (the
// slice and its rotate-half partner), 16 outputs, two 16-byte stores; one-shot blocks.  The
// table of a host-side shift travels in the kernel parameters and is copied to shared
// memory; device tables ([1 | T, D/2] fp16) are read per row.  Generic path: one thread per
// (row, frequency), any strides.  A thread reads both halves before writing them, so the
// shift may run in place (out == x with the same strides).
#include "sc_common.cuh"

namespace sc {
namespace {

constexpr int kSThreads = 256;

struct ShiftParams {
    int32_t rows;  // n_tokens * n_heads (< 2^31)
    int32_t H, D, S;  // S = (D / 2) / 8 slices of 8 frequencies per row (vector path)
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

__device__ __forceinline__ void shift_pair(float x1, float x2, float c, float s, float& o1,
                                           float& o2) {
    o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
}

template <typename InT, typename OutT>
__global__ void __launch_bounds__(kSThreads) shift_vec(const __grid_constant__ ShiftParams p) {
    __shared__ float s_cos[kMaxHeadDim / 2];
    __shared__ float s_sin[kMaxHeadDim / 2];
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
    const int f0 = j * 8;
    const InT* xp = reinterpret_cast<const InT*>(p.x) + t * p.x_t + h * p.x_h + f0;
    const uint4 a = *reinterpret_cast<const uint4*>(xp);
    const uint4 b = *reinterpret_cast<const uint4*>(xp + half);
    float c[8], s[8];
    if (p.cos == nullptr) {
#pragma unroll
        for (int k = 0; k < 8; ++k) c[k] = s_cos[f0 + k], s[k] = s_sin[f0 + k];
    } else {
        const uint4 cv = *reinterpret_cast<const uint4*>(p.cos + t * p.cs_t + f0);
        const uint4 sv = *reinterpret_cast<const uint4*>(p.sin + t * p.cs_t + f0);
        const uint32_t cw[4] = {cv.x, cv.y, cv.z, cv.w}, sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 cc = __half22float2(bit_cast_u32<__half2>(cw[k]));
            const float2 ss = __half22float2(bit_cast_u32<__half2>(sw[k]));
            c[2 * k] = cc.x, c[2 * k + 1] = cc.y, s[2 * k] = ss.x, s[2 * k + 1] = ss.y;
        }
    }
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
    uint32_t lo[4], hi[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const InT* ap = reinterpret_cast<const InT*>(&aw[k]);
        const InT* bp = reinterpret_cast<const InT*>(&bw[k]);
        float o1a, o2a, o1b, o2b;
        shift_pair(to_f(ap[0]), to_f(bp[0]), c[2 * k], s[2 * k], o1a, o2a);
        shift_pair(to_f(ap[1]), to_f(bp[1]), c[2 * k + 1], s[2 * k + 1], o1b, o2b);
        lo[k] = pack2<OutT>(o1a, o1b);
        hi[k] = pack2<OutT>(o2a, o2b);
    }
    OutT* op = reinterpret_cast<OutT*>(p.out) + t * p.o_t + h * p.o_h + f0;
    *reinterpret_cast<uint4*>(op) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *reinterpret_cast<uint4*>(op + half) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
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

template <typename InT, typename OutT>
cudaError_t launch_shift(const ShiftParams& p, bool vec, cudaStream_t stream) {
    const int64_t work = static_cast<int64_t>(p.rows) * (vec ? p.S : p.D / 2);
    const int64_t blocks = (work + kSThreads - 1) / kSThreads;
    if (vec)
        shift_vec<InT, OutT><<<static_cast<unsigned>(blocks), kSThreads, 0, stream>>>(p);
    else
        shift_generic<InT, OutT><<<static_cast<unsigned>(blocks), kSThreads, 0, stream>>>(p);
    return cudaGetLastError();
}

template <typename InT>
cudaError_t launch_shift_in(const ShiftParams& p, int32_t out_dtype, bool vec, cudaStream_t s) {
    return out_dtype == SC_DTYPE_F16 ? launch_shift<InT, __half>(p, vec, s)
                                     : launch_shift<InT, __nv_bfloat16>(p, vec, s);
}

template <typename InT, typename OutT>
cudaError_t preload_shift_io() {
    cudaFuncAttributes attr;
    cudaError_t e = cudaFuncGetAttributes(&attr, shift_vec<InT, OutT>);
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
    const int64_t rows = n_tokens * n_heads;
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
    // Vector path: 8 frequencies per thread, 16-byte aligned slices of x, out and the tables.
    const int half = head_dim / 2;
    auto al = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    auto st8 = [](int64_t st, int64_t size) { return size <= 1 || st % 8 == 0; };
    bool vec = half % 8 == 0 && p.x_d == 1 && p.o_d == 1 && al(x) && al(out) &&
               st8(p.x_t, n_tokens) && st8(p.x_h, n_heads) && st8(p.o_t, n_tokens) &&
               st8(p.o_h, n_heads);
    if (vec && cos_delta)
        vec = p.cs_d == 1 && al(cos_delta) && al(sin_delta) && st8(p.cs_t, n_tokens);
    p.S = half / 8 > 0 ? half / 8 : 1;
    p.divS = make_fastdiv(static_cast<uint32_t>(p.S));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaError_t e = x_dtype == SC_DTYPE_F16 ? launch_shift_in<__half>(p, out_dtype, vec, s)
                                                  : launch_shift_in<__nv_bfloat16>(p, out_dtype, vec, s);
    if (e != cudaSuccess) return cuda_error(e, "key shift launch");
    return ok();
}
