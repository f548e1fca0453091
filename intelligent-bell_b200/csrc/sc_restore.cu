// sc_restore.cu — fused INT8 K dequant + relative RoPE shift and V dequant (dense layout),
// plus the cos/sin table kernel.
//
// Vector path (head_dim % 32 == 0, unit dim stride, 16-byte aligned input rows and
// 32-byte aligned output rows):
//   a row is one (layer, token, head) vector of head_dim int8 codes.  Thread j of a row
//   owns the 16-frequency slice j: it loads bytes [16j, 16j+16) of the first half and
//   their rotate-half partners [D/2+16j, D/2+16j+16) with two 16-byte loads, so the
//   rotation needs no data from other lanes.  The same thread does the V row slice.
//   Each 16-output run is written with one 32-byte store, i.e. one full L2 sector.
//   Blocks are one-shot tiles of consecutive rows (no grid-stride loop): each thread
//   issues the loads of its SC_ROWS_PER_THREAD row-slices, then converts and stores them.
//   On B200 this streams 9-10 % faster than a persistent grid walking the same rows.
//   The cos/sin table of a single shift is computed once on the host (double cos/sin of
//   the fp32 angle, rounded to fp32 then fp16, like the reference's tables), travels in the
//   kernel parameters, and is unpacked into shared memory by every block; a shift read from
//   device memory is expanded per block; per-token tables are read per row.
// Generic path: any strides, any even head_dim <= 1024, one thread per (row, frequency).
#include <math.h>
#include <string.h>

#include <type_traits>

#include "sc_common.cuh"

namespace sc {
namespace {

// Threads per block.  128-thread blocks (8 resident per SM at 64 registers) restore the
// 32-layer Llama-3-8B batch in 241 us against 245 us with 256-thread blocks (4 per SM).
#ifndef SC_DENSE_THREADS
#define SC_DENSE_THREADS 128
#endif
constexpr int kThreads = SC_DENSE_THREADS;
// Resident blocks per SM the register allocation aims for (vector kernel).
#ifndef SC_DENSE_MIN_BLOCKS
#define SC_DENSE_MIN_BLOCKS 8
#endif
// Row-slices per thread (all their loads are issued before the first store).
#ifndef SC_ROWS_PER_THREAD
#define SC_ROWS_PER_THREAD 1
#endif
// Stage SC_DENSE_ROUNDS rounds of rows per block in shared memory with cp.async before
// converting any (1), instead of loading SC_ROWS_PER_THREAD rows into registers (0).
#ifndef SC_DENSE_CPASYNC
#define SC_DENSE_CPASYNC 0
#endif
#ifndef SC_DENSE_ROUNDS
#define SC_DENSE_ROUNDS 4
#endif

struct DenseParams {
    int32_t rows;  // n_layers * n_tokens * n_heads  (< 2^31)
    int32_t D;
    int32_t P;  // 16-frequency slices per half row: D / 32 (vector path)
    int32_t has_k, has_v;
    int32_t cs_kind;  // 0: shift in device memory, 1: one table row, 2: one table row per
                      // token, 3: table computed on the host (in `tab`)
    FastDiv divH, divT;
    int32_t H, T;
    const int8_t* kq;
    const void* ks;
    const int8_t* vq;
    const void* vs;
    void* ko;
    void* vo;
    int64_t kq_s[4], ks_s[3], vq_s[4], vs_s[3], ko_s[4], vo_s[4];  // [l, t, h(, d)]
    const __half* cos;
    const __half* sin;
    int64_t cs_t, cs_d;
    const float* dp_dev;
    // cs_kind 0: float inverse frequencies; cs_kind 3: half2(cos, sin) per frequency.
    uint32_t tab[kMaxHeadDim / 2];
};

__device__ __forceinline__ void row_coords(const DenseParams& p, uint32_t row, int64_t& l,
                                           int64_t& t, int64_t& h) {
    const uint32_t lt = fdiv(row, p.divH);
    h = static_cast<int64_t>(row - lt * static_cast<uint32_t>(p.H));
    const uint32_t li = fdiv(lt, p.divT);
    t = static_cast<int64_t>(lt - li * static_cast<uint32_t>(p.T));
    l = static_cast<int64_t>(li);
}

// Fill the block's shared cos/sin table for a single shift (cs_kind 0, 1 or 3).
__device__ __forceinline__ void fill_shared_table(const DenseParams& p, float* s_cos,
                                                  float* s_sin) {
    const int half = p.D >> 1;
    if (p.cs_kind == 3) {
        for (int f = threadIdx.x; f < half; f += blockDim.x) {
            const float2 cs = __half22float2(bit_cast_u32<__half2>(p.tab[f]));
            s_cos[f] = cs.x;
            s_sin[f] = cs.y;
        }
    } else if (p.cs_kind == 1) {
        for (int f = threadIdx.x; f < half; f += blockDim.x) {
            s_cos[f] = __half2float(p.cos[f * p.cs_d]);
            s_sin[f] = __half2float(p.sin[f * p.cs_d]);
        }
    } else {
        const float dp = *p.dp_dev;
        for (int f = threadIdx.x; f < half; f += blockDim.x) {
            float c, s;
            rope_cs(dp, __uint_as_float(p.tab[f]), c, s);
            s_cos[f] = c;
            s_sin[f] = s;
        }
    }
    __syncthreads();
}

// What one thread carries from the load of a row-slice to its store: the codes and
// scales only (store addresses are recomputed from the row index).
template <typename ScaleT>
struct RowLoad {
    uint4 ka, kb, va, vb;
    ScaleT ksc, vsc;
    int32_t row;  // -1 when past the end
};

template <typename ScaleT>
__device__ __forceinline__ void load_row(const DenseParams& p, int64_t row, int j,
                                         RowLoad<ScaleT>& r) {
    if (row >= p.rows) {
        r.row = -1;
        return;
    }
    r.row = static_cast<int32_t>(row);
    int64_t l, t, h;
    row_coords(p, static_cast<uint32_t>(row), l, t, h);
    const int half = p.D >> 1;
    if (p.has_k) {
        const int8_t* base = p.kq + l * p.kq_s[0] + t * p.kq_s[1] + h * p.kq_s[2] + j * 16;
        r.ka = ld_stream_v4(base);
        r.kb = ld_stream_v4(base + half);
        r.ksc = reinterpret_cast<const ScaleT*>(p.ks)[l * p.ks_s[0] + t * p.ks_s[1] + h * p.ks_s[2]];
    }
    if (p.has_v) {
        const int8_t* base = p.vq + l * p.vq_s[0] + t * p.vq_s[1] + h * p.vq_s[2] + j * 16;
        r.va = ld_stream_v4(base);
        r.vb = ld_stream_v4(base + half);
        r.vsc = reinterpret_cast<const ScaleT*>(p.vs)[l * p.vs_s[0] + t * p.vs_s[1] + h * p.vs_s[2]];
    }
}

__device__ __forceinline__ void load_token_cs(const DenseParams& p, int64_t t, int j, float* c,
                                              float* s) {
    const __half* cp = p.cos + t * p.cs_t + j * 16;
    const __half* sp = p.sin + t * p.cs_t + j * 16;
    const uint4 c0 = ld_stream_v4(cp), c1 = ld_stream_v4(cp + 8);
    const uint4 s0 = ld_stream_v4(sp), s1 = ld_stream_v4(sp + 8);
    const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const float2 cf = __half22float2(bit_cast_u32<__half2>(cw[k]));
        const float2 sf = __half22float2(bit_cast_u32<__half2>(sw[k]));
        c[2 * k] = cf.x;
        c[2 * k + 1] = cf.y;
        s[2 * k] = sf.x;
        s[2 * k + 1] = sf.y;
    }
}

template <typename OutT, typename ScaleT, bool X16, bool PER_TOKEN>
__device__ __forceinline__ void store_row(const DenseParams& p, const RowLoad<ScaleT>& r, int j,
                                          const CsShared& cs) {
    if (r.row < 0) return;
    int64_t l, t, h;
    row_coords(p, static_cast<uint32_t>(r.row), l, t, h);
    const int half = p.D >> 1;
    if (p.has_k) {
        OutT* o = reinterpret_cast<OutT*>(p.ko) + (l * p.ko_s[0] + t * p.ko_s[1] + h * p.ko_s[2] + j * 16);
        if constexpr (PER_TOKEN) {
            float ct[16], st[16];
            load_token_cs(p, t, j, ct, st);
            rope_slice_store<OutT, ScaleT, X16>(r.ka, r.kb, r.ksc, CsRegs{ct, st}, o, o + half);
        } else {
            rope_slice_store<OutT, ScaleT, X16>(r.ka, r.kb, r.ksc, cs, o, o + half);
        }
    }
    if (p.has_v) {
        OutT* o = reinterpret_cast<OutT*>(p.vo) + (l * p.vo_s[0] + t * p.vo_s[1] + h * p.vo_s[2] + j * 16);
        value_slice_store<OutT, ScaleT>(r.va, r.vsc, o);
        value_slice_store<OutT, ScaleT>(r.vb, r.vsc, o + half);
    }
}

// Where a block's cos/sin come from (a template parameter, so each order compiles alone):
enum CsMode : int {
    kCsCopied = 0,  // host-computed or caller's single row: filled into shared memory first
    kCsDevice = 1,  // shift read from device memory: expanded (double sincos) while the
                    // block's loads are in flight
    kCsToken = 2,   // one table row per token, read per row from global memory
};

// One-shot tile: block b owns rows [b * RB * R, (b + 1) * RB * R); each thread loads its R
// row-slices, then converts and stores them.
#if SC_DENSE_CPASYNC
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
#endif

template <typename OutT, typename ScaleT, bool X16, int CSM>
__global__ void __launch_bounds__(kThreads, SC_DENSE_MIN_BLOCKS)
    dense_restore_vec(const __grid_constant__ DenseParams p) {
    __shared__ __align__(16) float s_cos[kMaxHeadDim / 2];
    __shared__ __align__(16) float s_sin[kMaxHeadDim / 2];
#if SC_DENSE_CPASYNC
    {
        constexpr int NR = SC_DENSE_ROUNDS;
        constexpr bool kPerToken = CSM == kCsToken;
        __shared__ __align__(16) uint4 s_codes[NR][4][kThreads];
        const int tid = threadIdx.x;
        const int P = p.P;
        const int j = tid % P;
        const int rl = tid / P;
        const int RB = blockDim.x / P;
        const int half = p.D >> 1;
        const int64_t row0 = static_cast<int64_t>(blockIdx.x) * RB * NR + rl;
        ScaleT ksc[NR], vsc[NR];
#pragma unroll
        for (int k = 0; k < NR; ++k) {
            const int64_t row = row0 + k * RB;
            if (row >= p.rows) continue;
            int64_t l, t, h;
            row_coords(p, static_cast<uint32_t>(row), l, t, h);
            if (p.has_k) {
                const int8_t* base = p.kq + l * p.kq_s[0] + t * p.kq_s[1] + h * p.kq_s[2] + j * 16;
                cp_async16(&s_codes[k][0][tid], base);
                cp_async16(&s_codes[k][1][tid], base + half);
                ksc[k] = reinterpret_cast<const ScaleT*>(p.ks)[l * p.ks_s[0] + t * p.ks_s[1] + h * p.ks_s[2]];
            }
            if (p.has_v) {
                const int8_t* base = p.vq + l * p.vq_s[0] + t * p.vq_s[1] + h * p.vq_s[2] + j * 16;
                cp_async16(&s_codes[k][2][tid], base);
                cp_async16(&s_codes[k][3][tid], base + half);
                vsc[k] = reinterpret_cast<const ScaleT*>(p.vs)[l * p.vs_s[0] + t * p.vs_s[1] + h * p.vs_s[2]];
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        if constexpr (CSM != kCsToken) fill_shared_table(p, s_cos, s_sin);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        const CsShared cs{reinterpret_cast<const float4*>(s_cos + j * 16),
                          reinterpret_cast<const float4*>(s_sin + j * 16)};
#pragma unroll
        for (int k = 0; k < NR; ++k) {
            const int64_t row = row0 + k * RB;
            if (row >= p.rows) continue;
            RowLoad<ScaleT> r;
            r.row = static_cast<int32_t>(row);
            r.ka = s_codes[k][0][tid];
            r.kb = s_codes[k][1][tid];
            r.va = s_codes[k][2][tid];
            r.vb = s_codes[k][3][tid];
            r.ksc = ksc[k];
            r.vsc = vsc[k];
            store_row<OutT, ScaleT, X16, kPerToken>(p, r, j, cs);
        }
        return;
    }
#endif
    constexpr int R = SC_ROWS_PER_THREAD;
    constexpr bool kPerToken = CSM == kCsToken;
    const int P = p.P;
    const int j = threadIdx.x % P;
    const int rl = threadIdx.x / P;
    const int RB = blockDim.x / P;
    if constexpr (CSM == kCsCopied) fill_shared_table(p, s_cos, s_sin);
    const CsShared cs{reinterpret_cast<const float4*>(s_cos + j * 16),
                      reinterpret_cast<const float4*>(s_sin + j * 16)};
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * RB * R + rl;
    RowLoad<ScaleT> buf[R];
#pragma unroll
    for (int k = 0; k < R; ++k) load_row<ScaleT>(p, row0 + k * RB, j, buf[k]);
    if constexpr (CSM == kCsDevice) fill_shared_table(p, s_cos, s_sin);
#pragma unroll
    for (int k = 0; k < R; ++k) store_row<OutT, ScaleT, X16, kPerToken>(p, buf[k], j, cs);
}

// Stride-generic path: one thread per (row, frequency f), both halves of the pair.
struct GenericStrides {
    int64_t rows;
    int64_t kq_d, vq_d, ko_d, vo_d;
};

template <typename OutT, typename ScaleT, bool X16>
__global__ void __launch_bounds__(kThreads)
    dense_restore_generic(const __grid_constant__ DenseParams p, const GenericStrides g) {
    __shared__ float s_cos[kMaxHeadDim / 2];
    __shared__ float s_sin[kMaxHeadDim / 2];
    if (p.cs_kind != 2) fill_shared_table(p, s_cos, s_sin);
    const int half = p.D >> 1;
    const int64_t total = g.rows * half;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t row = i / half;
        const int f = static_cast<int>(i - row * half);
        const int64_t h = row % p.H;
        const int64_t lt = row / p.H;
        const int64_t t = lt % p.T;
        const int64_t l = lt / p.T;
        if (p.has_k) {
            const int8_t* kb = p.kq + l * p.kq_s[0] + t * p.kq_s[1] + h * p.kq_s[2];
            const float sf = scale_to_float<ScaleT>(
                reinterpret_cast<const ScaleT*>(p.ks)[l * p.ks_s[0] + t * p.ks_s[1] + h * p.ks_s[2]]);
            float x1 = __fmul_rn(static_cast<float>(kb[f * g.kq_d]), sf);
            float x2 = __fmul_rn(static_cast<float>(kb[(f + half) * g.kq_d]), sf);
            if constexpr (X16) {
                x1 = __half2float(__float2half_rn(x1));
                x2 = __half2float(__float2half_rn(x2));
            }
            float c, s;
            if (p.cs_kind == 2) {
                c = __half2float(p.cos[t * p.cs_t + f * p.cs_d]);
                s = __half2float(p.sin[t * p.cs_t + f * p.cs_d]);
            } else {
                c = s_cos[f];
                s = s_sin[f];
            }
            OutT* o = reinterpret_cast<OutT*>(p.ko) + l * p.ko_s[0] + t * p.ko_s[1] + h * p.ko_s[2];
            float o1, o2;
            rotate_pair<X16>(x1, x2, c, s, o1, o2);
            o[f * g.ko_d] = from_float<OutT>(o1);
            o[(f + half) * g.ko_d] = from_float<OutT>(o2);
        }
        if (p.has_v) {
            const int8_t* vb = p.vq + l * p.vq_s[0] + t * p.vq_s[1] + h * p.vq_s[2];
            const float sf = scale_to_float<ScaleT>(
                reinterpret_cast<const ScaleT*>(p.vs)[l * p.vs_s[0] + t * p.vs_s[1] + h * p.vs_s[2]]);
            OutT* o = reinterpret_cast<OutT*>(p.vo) + l * p.vo_s[0] + t * p.vo_s[1] + h * p.vo_s[2];
            o[f * g.vo_d] = from_float<OutT>(__fmul_rn(static_cast<float>(vb[f * g.vq_d]), sf));
            o[(f + half) * g.vo_d] =
                from_float<OutT>(__fmul_rn(static_cast<float>(vb[(f + half) * g.vq_d]), sf));
        }
    }
}

template <typename OutT>
__global__ void __launch_bounds__(kThreads)
    rope_table_kernel(const float* __restrict__ dp, int64_t n, int half,
                      const __grid_constant__ DenseParams p, OutT* cos_out, OutT* sin_out) {
    const int64_t total = n * half;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / half;
        const int f = static_cast<int>(i - r * half);
        const float angle = __fmul_rn(dp[r], __uint_as_float(p.tab[f]));
        double sd, cd;
        sincos(static_cast<double>(angle), &sd, &cd);
        const float c = static_cast<float>(cd), s = static_cast<float>(sd);
        if constexpr (std::is_same<OutT, float>::value) {
            cos_out[i] = c;
            sin_out[i] = s;
        } else {
            cos_out[i] = from_float<OutT>(c);
            sin_out[i] = from_float<OutT>(s);
        }
    }
}

void fill_inv_freq(DenseParams& p, int head_dim, double theta, const float* inv_freq) {
    float tmp[kMaxHeadDim / 2];
    if (inv_freq == nullptr) {
        default_inv_freq(head_dim, theta, tmp);
        inv_freq = tmp;
    }
    for (int i = 0; i < head_dim / 2; ++i) memcpy(&p.tab[i], &inv_freq[i], sizeof(float));
}

// cos/sin of one shift as the reference tabulates them: angle = fp32(dp * inv_freq) (one
// fp32 multiply), cos/sin in double, rounded to fp32 and then to fp16.  A few recent tables
// are kept per host thread (keyed by the shift, head_dim and the inverse frequencies), so
// restoring many layers with one shift computes the table once.
struct HostTable {
    uint32_t dp_bits = 0;
    int head_dim = 0;
    uint64_t freq_hash = 0;
    bool valid = false;
    uint32_t tab[kMaxHeadDim / 2];
};

uint64_t hash_freqs(const float* f, int n) {
    uint64_t h = 1469598103934665603ull;  // FNV-1a over the float bit patterns
    for (int i = 0; i < n; ++i) {
        uint32_t b;
        memcpy(&b, &f[i], sizeof(b));
        h = (h ^ b) * 1099511628211ull;
    }
    return h;
}

void fill_host_table(uint32_t* out_tab, int head_dim, float dp, double theta, const float* inv_freq) {
    float tmp[kMaxHeadDim / 2];
    if (inv_freq == nullptr) {
        default_inv_freq(head_dim, theta, tmp);
        inv_freq = tmp;
    }
    const int half = head_dim / 2;
    uint32_t dp_bits;
    memcpy(&dp_bits, &dp, sizeof(dp_bits));
    const uint64_t fh = hash_freqs(inv_freq, half);
    constexpr int kEntries = 4;
    thread_local HostTable cache[kEntries];
    thread_local int next_slot = 0;
    for (int e = 0; e < kEntries; ++e) {
        const HostTable& c = cache[e];
        if (c.valid && c.dp_bits == dp_bits && c.head_dim == head_dim && c.freq_hash == fh) {
            memcpy(out_tab, c.tab, sizeof(uint32_t) * half);
            return;
        }
    }
    HostTable& c = cache[next_slot];
    next_slot = (next_slot + 1) % kEntries;
    for (int i = 0; i < half; ++i) {
        const volatile float angle = dp * inv_freq[i];  // one rounding, no contraction
        const __half cv = __float2half_rn(static_cast<float>(cos(static_cast<double>(angle))));
        const __half sv = __float2half_rn(static_cast<float>(sin(static_cast<double>(angle))));
        const __half2 cs = __halves2half2(cv, sv);
        memcpy(&c.tab[i], &cs, sizeof(uint32_t));
    }
    c.dp_bits = dp_bits;
    c.head_dim = head_dim;
    c.freq_hash = fh;
    c.valid = true;
    memcpy(out_tab, c.tab, sizeof(uint32_t) * half);
}

// Resident blocks per SM of `kernel`, cached per device in the caller's `cache` (one cache
// per kernel instantiation: every instantiation has its own register count).
template <typename K>
int blocks_per_sm(K kernel, int threads, int (&cache)[64]) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, 0) != cudaSuccess ||
        n <= 0)
        n = 1;
    if (dev >= 0 && dev < 64) cache[dev] = n;
    return n;
}

inline bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }
inline bool stride_ok(int64_t stride, int64_t size, int64_t align) {
    return size <= 1 || (stride % align) == 0;
}

template <typename OutT, typename ScaleT, bool X16, int CSM>
cudaError_t launch_vec(const DenseParams& p, cudaStream_t stream) {
    auto kern = dense_restore_vec<OutT, ScaleT, X16, CSM>;
    const int threads = (kThreads / p.P) * p.P;
    const int64_t per_block = static_cast<int64_t>(threads / p.P) *
                              (SC_DENSE_CPASYNC ? SC_DENSE_ROUNDS : SC_ROWS_PER_THREAD);
    const int64_t grid = (static_cast<int64_t>(p.rows) + per_block - 1) / per_block;
    kern<<<static_cast<unsigned>(grid), threads, 0, stream>>>(p);
    return cudaGetLastError();
}

template <typename OutT, typename ScaleT, bool X16>
cudaError_t launch_generic(const DenseParams& p, const GenericStrides& g, cudaStream_t stream) {
    auto kern = dense_restore_generic<OutT, ScaleT, X16>;
    const int64_t total = g.rows * (p.D / 2);
    const int64_t need = (total + kThreads - 1) / kThreads;
    static int occupancy[64] = {0};  // this instantiation's resident blocks per SM, per device
    const int64_t cap = static_cast<int64_t>(sm_count()) * blocks_per_sm(kern, kThreads, occupancy);
    const int grid = static_cast<int>(need < cap ? (need > 0 ? need : 1) : cap);
    kern<<<grid, kThreads, 0, stream>>>(p, g);
    return cudaGetLastError();
}

template <typename OutT, typename ScaleT>
cudaError_t dispatch(const DenseParams& p, const GenericStrides& g, bool vec, bool x16,
                     cudaStream_t stream) {
    if (vec) {
        const int mode = p.cs_kind == 2 ? kCsToken : (p.cs_kind == 0 ? kCsDevice : kCsCopied);
        if (mode == kCsToken)
            return x16 ? launch_vec<OutT, ScaleT, true, kCsToken>(p, stream)
                       : launch_vec<OutT, ScaleT, false, kCsToken>(p, stream);
        if (mode == kCsDevice)
            return x16 ? launch_vec<OutT, ScaleT, true, kCsDevice>(p, stream)
                       : launch_vec<OutT, ScaleT, false, kCsDevice>(p, stream);
        return x16 ? launch_vec<OutT, ScaleT, true, kCsCopied>(p, stream)
                   : launch_vec<OutT, ScaleT, false, kCsCopied>(p, stream);
    }
    return x16 ? launch_generic<OutT, ScaleT, true>(p, g, stream)
               : launch_generic<OutT, ScaleT, false>(p, g, stream);
}

template <typename K>
cudaError_t load_kernel(K kern) {
    cudaFuncAttributes attr;
    return cudaFuncGetAttributes(&attr, kern);
}

template <typename OutT, typename ScaleT>
cudaError_t preload_dense_ts() {
    cudaError_t e = load_kernel(dense_restore_vec<OutT, ScaleT, true, kCsCopied>);
    if (e == cudaSuccess) e = load_kernel(dense_restore_vec<OutT, ScaleT, false, kCsCopied>);
    if (e == cudaSuccess) e = load_kernel(dense_restore_vec<OutT, ScaleT, true, kCsDevice>);
    if (e == cudaSuccess) e = load_kernel(dense_restore_vec<OutT, ScaleT, false, kCsDevice>);
    if (e == cudaSuccess) e = load_kernel(dense_restore_vec<OutT, ScaleT, true, kCsToken>);
    if (e == cudaSuccess) e = load_kernel(dense_restore_vec<OutT, ScaleT, false, kCsToken>);
    if (e == cudaSuccess) e = load_kernel(dense_restore_generic<OutT, ScaleT, true>);
    if (e == cudaSuccess) e = load_kernel(dense_restore_generic<OutT, ScaleT, false>);
    return e;
}

}  // namespace

cudaError_t preload_dense_kernels() {
    cudaError_t e = preload_dense_ts<__half, __half>();
    if (e == cudaSuccess) e = preload_dense_ts<__half, float>();
    if (e == cudaSuccess) e = preload_dense_ts<__nv_bfloat16, __half>();
    if (e == cudaSuccess) e = preload_dense_ts<__nv_bfloat16, float>();
    if (e == cudaSuccess) e = load_kernel(rope_table_kernel<__half>);
    if (e == cudaSuccess) e = load_kernel(rope_table_kernel<__nv_bfloat16>);
    if (e == cudaSuccess) e = load_kernel(rope_table_kernel<float>);
    return e;
}

void host_cos_sin_table(int head_dim, float dp, double theta, const float* inv_freq,
                        uint32_t* tab) {
    fill_host_table(tab, head_dim, dp, theta, inv_freq);
}

}  // namespace sc

using namespace sc;

extern "C" int32_t sc_rope_cos_sin_delta(const float* delta_pos, int64_t n, int32_t head_dim,
                                         double theta_base, const float* inv_freq,
                                         void* cos_out, void* sin_out, int32_t out_dtype,
                                         void* stream) {
    if (head_dim <= 0 || (head_dim & 1))
        return set_error(SC_ERR_INVALID_ARGUMENT, "head_dim must be even, got %d", head_dim);
    if (head_dim > kMaxHeadDim)
        return set_error(SC_ERR_UNSUPPORTED, "head_dim %d exceeds %d", head_dim, kMaxHeadDim);
    if (n < 0) return set_error(SC_ERR_INVALID_ARGUMENT, "n must be >= 0, got %lld", (long long)n);
    if (n == 0) return ok();
    if (!delta_pos || !cos_out || !sin_out)
        return set_error(SC_ERR_INVALID_ARGUMENT, "null pointer argument");
    DenseParams p{};
    p.D = head_dim;
    fill_inv_freq(p, head_dim, theta_base, inv_freq);
    const int half = head_dim / 2;
    const int64_t total = size_product(n, half);
    if (total >= (int64_t(1) << 40))
        return set_error(SC_ERR_INVALID_ARGUMENT, "n = %lld table rows is too many", (long long)n);
    const int64_t need = (total + kThreads - 1) / kThreads;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
    const int grid = static_cast<int>(need < cap ? need : cap);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (out_dtype) {
        case SC_DTYPE_F16:
            rope_table_kernel<__half><<<grid, kThreads, 0, s>>>(
                delta_pos, n, half, p, static_cast<__half*>(cos_out), static_cast<__half*>(sin_out));
            break;
        case SC_DTYPE_BF16:
            rope_table_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(
                delta_pos, n, half, p, static_cast<__nv_bfloat16*>(cos_out),
                static_cast<__nv_bfloat16*>(sin_out));
            break;
        case SC_DTYPE_F32:
            rope_table_kernel<float><<<grid, kThreads, 0, s>>>(
                delta_pos, n, half, p, static_cast<float*>(cos_out), static_cast<float*>(sin_out));
            break;
        default:
            return set_error(SC_ERR_INVALID_DTYPE, "unsupported table dtype code %d", out_dtype);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "rope_table_kernel launch");
    return ok();
}

extern "C" int32_t sc_dequant_rope_kv(
    int32_t n_layers, int64_t n_tokens, int32_t n_heads, int32_t head_dim, const int8_t* k_quant,
    const int64_t* kq_strides, const void* k_scale, const int64_t* ks_strides,
    const int8_t* v_quant, const int64_t* vq_strides, const void* v_scale,
    const int64_t* vs_strides, int32_t scale_dtype, const void* cos_delta, const void* sin_delta,
    const int64_t* cs_strides, double delta_p, const float* delta_p_dev, double theta_base,
    const float* inv_freq, void* k_out, const int64_t* ko_strides, void* v_out,
    const int64_t* vo_strides, int32_t out_dtype, uint32_t flags, void* stream) {
    if (n_layers < 0 || n_tokens < 0 || n_heads < 0)
        return set_error(SC_ERR_INVALID_ARGUMENT, "negative size (layers=%d tokens=%lld heads=%d)",
                         n_layers, (long long)n_tokens, n_heads);
    if (head_dim <= 0 || (head_dim & 1))
        return set_error(SC_ERR_INVALID_ARGUMENT,
                         "head_dim must be even for RoPE half-pairing, got head_dim=%d", head_dim);
    if (head_dim > kMaxHeadDim)
        return set_error(SC_ERR_UNSUPPORTED, "head_dim %d exceeds %d", head_dim, kMaxHeadDim);
    if (out_dtype != SC_DTYPE_F16 && out_dtype != SC_DTYPE_BF16)
        return set_error(SC_ERR_INVALID_DTYPE, "output dtype code %d: float16 or bfloat16 only",
                         out_dtype);
    if (scale_dtype != SC_DTYPE_F16 && scale_dtype != SC_DTYPE_F32)
        return set_error(SC_ERR_INVALID_DTYPE, "scale dtype code %d: float16 or float32 only",
                         scale_dtype);
    const int64_t rows = size_product(n_layers, n_tokens, n_heads);
    if (rows == 0) return ok();  // empty tensors may carry null pointers
    const bool has_k = k_quant != nullptr, has_v = v_quant != nullptr;
    if (!has_k && !has_v) return set_error(SC_ERR_INVALID_ARGUMENT, "neither K nor V given");
    if (has_k && (!k_scale || !k_out || !kq_strides || !ks_strides || !ko_strides))
        return set_error(SC_ERR_INVALID_ARGUMENT, "K given without its scale/output/strides");
    if (has_v && (!v_scale || !v_out || !vq_strides || !vs_strides || !vo_strides))
        return set_error(SC_ERR_INVALID_ARGUMENT, "V given without its scale/output/strides");
    if ((cos_delta == nullptr) != (sin_delta == nullptr))
        return set_error(SC_ERR_INVALID_ARGUMENT, "cos_delta and sin_delta must both be given");
    if (cos_delta && !cs_strides)
        return set_error(SC_ERR_INVALID_ARGUMENT, "cos/sin tables given without strides");
    if (rows >= (int64_t(1) << 31))
        return set_error(SC_ERR_INVALID_ARGUMENT,
                         "%lld rows in one call; split the call below 2^31 rows", (long long)rows);

    DenseParams p{};
    p.rows = static_cast<int32_t>(rows);
    p.D = head_dim;
    p.P = head_dim / 32;
    p.has_k = has_k;
    p.has_v = has_v;
    p.H = n_heads;
    p.T = static_cast<int32_t>(n_tokens);
    p.divH = make_fastdiv(static_cast<uint32_t>(n_heads));
    p.divT = make_fastdiv(static_cast<uint32_t>(n_tokens));
    p.kq = k_quant;
    p.ks = k_scale;
    p.vq = v_quant;
    p.vs = v_scale;
    p.ko = k_out;
    p.vo = v_out;
    GenericStrides g{};
    g.rows = rows;
    if (has_k) {
        for (int i = 0; i < 4; ++i) p.kq_s[i] = kq_strides[i], p.ko_s[i] = ko_strides[i];
        for (int i = 0; i < 3; ++i) p.ks_s[i] = ks_strides[i];
        g.kq_d = kq_strides[3];
        g.ko_d = ko_strides[3];
    }
    if (has_v) {
        for (int i = 0; i < 4; ++i) p.vq_s[i] = vq_strides[i], p.vo_s[i] = vo_strides[i];
        for (int i = 0; i < 3; ++i) p.vs_s[i] = vs_strides[i];
        g.vq_d = vq_strides[3];
        g.vo_d = vo_strides[3];
    }
    if (cos_delta) {
        p.cos = static_cast<const __half*>(cos_delta);
        p.sin = static_cast<const __half*>(sin_delta);
        p.cs_t = cs_strides[0];
        p.cs_d = cs_strides[1];
        p.cs_kind = (p.cs_t == 0 || n_tokens == 1) ? 1 : 2;
    } else {
        if (delta_p_dev != nullptr) {
            p.cs_kind = 0;  // shift known on the device only: expand per block
            p.dp_dev = delta_p_dev;
            fill_inv_freq(p, head_dim, theta_base, inv_freq);
        } else {
            p.cs_kind = 3;
            fill_host_table(p.tab, head_dim, static_cast<float>(delta_p), theta_base, inv_freq);
        }
    }

    // Vector path eligibility: 16-byte aligned row starts, unit dim stride, D % 32 == 0.
    bool vec = !(flags & SC_FLAG_FORCE_GENERIC) && (head_dim % 32 == 0);
    const int64_t sizes[3] = {n_layers, n_tokens, n_heads};
    // Inputs: 16-byte row starts.  Outputs: 32-byte row starts (one 32-byte store per lane).
    auto rows_ok = [&](const void* base, const int64_t* st, int64_t align_elems, uintptr_t align_bytes) {
        if ((reinterpret_cast<uintptr_t>(base) % align_bytes) != 0 || st[3] != 1) return false;
        for (int i = 0; i < 3; ++i)
            if (!stride_ok(st[i], sizes[i], align_elems)) return false;
        return true;
    };
    if (vec && has_k) vec = rows_ok(k_quant, kq_strides, 16, 16) && rows_ok(k_out, ko_strides, 16, 32);
    if (vec && has_v) vec = rows_ok(v_quant, vq_strides, 16, 16) && rows_ok(v_out, vo_strides, 16, 32);
    if (vec && p.cs_kind == 2)
        vec = aligned16(cos_delta) && aligned16(sin_delta) && p.cs_d == 1 && (p.cs_t % 8) == 0;

    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool x16 = !(flags & SC_FLAG_FP32_INTERMEDIATE);
    cudaError_t e;
    if (out_dtype == SC_DTYPE_F16)
        e = scale_dtype == SC_DTYPE_F16 ? dispatch<__half, __half>(p, g, vec, x16, s)
                                        : dispatch<__half, float>(p, g, vec, x16, s);
    else
        e = scale_dtype == SC_DTYPE_F16 ? dispatch<__nv_bfloat16, __half>(p, g, vec, x16, s)
                                        : dispatch<__nv_bfloat16, float>(p, g, vec, x16, s);
    if (e != cudaSuccess) return cuda_error(e, "dense restore launch");
    return ok();
}
