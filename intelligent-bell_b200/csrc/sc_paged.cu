// sc_paged.cu — ragged, paged restore: page-table gather + INT8 dequant + relative RoPE
// shift, written straight into contiguous per-request caches.
//
// Work unit: one block per (request, page, chunk of the page's rows): one-shot blocks, no
// persistent loop.  A block first reads its request's length and exits at once if its page
// lies past it; otherwise it reads the page id, output offset and shift together (one memory
// latency for the three).  It then issues the copies of all its rows at once: each thread
// owns a 16-frequency slice of one row per round (16 key codes of the first half and their
// rotate-half partners, the same for V: four 16-byte pieces) and copies them into its own
// shared-memory slots with cp.async, for SC_PAGED_ROUNDS rounds of threads / (D/32) rows,
// and loads the rows' scales into registers.  While those are in flight it builds the
// cos/sin table of the request's (or page's) shift in shared memory (single-precision
// sincos, double precision only where the fp16 rounding is not settled, rounded like the
// reference's fp16 tables), then waits for its own copies (cp.async.wait_group: a thread
// reads only the slots it filled, so no barrier guards the data) and converts and stores
// every row, each 16 outputs with one 32-byte store.
//
// Why this shape (measured on B200, ragged batch of 64 requests, 275K tokens):
// * one-shot blocks launched in order beat a persistent kernel over the same tiles: a
//   persistent version that walked only the live tiles, prefetched each page's metadata a
//   tile ahead and pipelined 2-4 tiles of copies per block reached 4.8-5.8 TB/s, against
//   6.2 TB/s for one-shot blocks (more stages in flight made it slower; its per-tile search,
//   records and barriers made it issue-bound at 68 % DRAM throughput);
// * staging every round's rows before converting any: 6.22 -> 6.47 TB/s over loading each
//   round into registers in turn (the rounds' loads no longer wait for each other); loading
//   two rows per thread into registers instead was slower (5.63 TB/s, register-bound);
// * what is left is mostly the page order: with the metadata loads replaced by arithmetic,
//   a uniform batch streams 6.54 TB/s when its pages are scrambled like the shuffled page
//   table's and 6.68 TB/s when they are in order, against 6.50-6.51 TB/s for this kernel (a
//   64 KB page of codes spreads thinly over the DRAM channels, so scattered pages open more
//   DRAM rows than consecutive ones).  Loading the metadata together with the length, or
//   prefetching its lines into L1 beside it, measured no gain (the empty blocks of a ragged
//   batch then wait for, or issue, more).
//
// Device-side checks never fault: a page id outside the pool, a bad sequence length or an
// output range outside out_numel makes the block skip the work and OR a status bit into
// the caller's status word.
#include "sc_common.cuh"

namespace sc {
namespace {

// Threads per block, rounds of rows per block and resident blocks per SM the register
// allocation aims for: 128 threads x 4 rounds = 128 rows at head_dim 128 (32 KB of codes
// staged per block).
#ifndef SC_PAGED_THREADS
#define SC_PAGED_THREADS 128
#endif
constexpr int kPThreads = SC_PAGED_THREADS;
#ifndef SC_PAGED_ROUNDS
#define SC_PAGED_ROUNDS 4
#endif
constexpr int kRounds = SC_PAGED_ROUNDS;
#ifndef SC_PAGED_MIN_BLOCKS
#define SC_PAGED_MIN_BLOCKS 5
#endif


// Read-only scalar loads kept in program order (volatile), so that metadata loads issued
// together are not sunk past the early-exit branches that follow them.
__device__ __forceinline__ int32_t ld_meta(const int32_t* ptr) {
    int32_t v;
    asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(ptr));
    return v;
}
__device__ __forceinline__ int64_t ld_meta(const int64_t* ptr) {
    int64_t v;
    asm volatile("ld.global.nc.b64 %0, [%1];" : "=l"(v) : "l"(ptr));
    return v;
}
__device__ __forceinline__ float ld_meta(const float* ptr) {
    float v;
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(ptr));
    return v;
}

// L2 prefetch size hint on the staging copies (0: none, 128 or 256 bytes).
#ifndef SC_PAGED_L2_PREFETCH
#define SC_PAGED_L2_PREFETCH 0
#endif

// 16 bytes global -> shared, cached in L2 only; the copy completes asynchronously.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
#if SC_PAGED_L2_PREFETCH == 256
    asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
#elif SC_PAGED_L2_PREFETCH == 128
    asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
#else
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
#endif
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

struct PagedParams {
    int32_t R, max_pages, page, H, D, P;
    int32_t chunks;  // blocks per page (page * H rows split into chunks of RB * kRounds rows)
    int64_t n_pool_pages;
    FastDiv divH;
    const int8_t* kq;
    const __half* ks;
    const int8_t* vq;
    const __half* vs;
    const int32_t* table;
    int64_t table_stride;
    const int32_t* seq_lens;
    int32_t seq_r;          // request stride of seq_lens (0: one length for every request)
    const float* dp;
    int64_t dp_r, dp_pg;    // shift of (request r, page pg): dp[r * dp_r + pg * dp_pg]
    int64_t sc_skew;        // scale rows added per request (packed codes, wider scale layout)
    void* ko;
    void* vo;
    const uint64_t* ko_ptrs;  // per-request output buffers (device), or null: ko/vo + out_off
    const uint64_t* vo_ptrs;
    int64_t ptr_off;          // with ko_ptrs / vo_ptrs: first element written of each buffer
    const int64_t* out_off;
    int64_t o_t, o_h;
    int64_t out_numel;
    int32_t* status;
    float inv_freq[kMaxHeadDim / 2];
};

// Output element offset of slice j of page-row `row` (token tok0 + row / H, head row % H).
__device__ __forceinline__ int64_t page_out_offset(const PagedParams& p, int32_t row, int j,
                                                   int64_t off, int tok0) {
    const uint32_t c = fdiv(static_cast<uint32_t>(row), p.divH);
    const int64_t h = row - static_cast<int64_t>(c) * p.H;
    return off + (tok0 + static_cast<int64_t>(c)) * p.o_t + h * p.o_h + j * 16;
}

// kPtrs: request r writes its own buffers (ko_ptrs[r], vo_ptrs[r]) from offset 0; otherwise
// ko / vo + out_off[r].  A separate instantiation keeps the offset path's output base in the
// kernel parameters (holding it in registers measured 9 % slower).
template <typename OutT, bool X16, bool kPtrs>
__global__ void __launch_bounds__(kPThreads, SC_PAGED_MIN_BLOCKS)
    paged_restore(const __grid_constant__ PagedParams p) {
    __shared__ __align__(16) float s_cos[kMaxHeadDim / 2];
    __shared__ __align__(16) float s_sin[kMaxHeadDim / 2];
    // This thread's slots: [round][K first half, K second half, V first, V second][thread].
    __shared__ __align__(16) uint4 s_codes[kRounds][4][kPThreads];
    const int tid = threadIdx.x;
    const int P = p.P;
    const int j = tid % P;
    const int rl = tid / P;
    const int RB = blockDim.x / P;
    const int half = p.D >> 1;
    const bool has_k = p.kq != nullptr, has_v = p.vq != nullptr;

    const int64_t task = blockIdx.x / p.chunks;
    const int chunk = static_cast<int>(blockIdx.x - task * p.chunks);
    const int r = static_cast<int>(task / p.max_pages);
    const int pg = static_cast<int>(task - static_cast<int64_t>(r) * p.max_pages);
    const bool reporter = chunk == 0 && tid == 0;
    // The length alone first: a block past its request's length exits after one load.
    const int len = ld_meta(p.seq_lens + r * p.seq_r);
    if (len < 0 || static_cast<int64_t>(len) > static_cast<int64_t>(p.max_pages) * p.page) {
        if (reporter && pg == 0) atomicOr(p.status, SC_STATUS_BAD_SEQ_LEN);
        return;
    }
    const int tok0 = pg * p.page;
    if (tok0 >= len) return;
    const int n_tok = min(p.page, len - tok0);
    const int64_t rows = static_cast<int64_t>(n_tok) * p.H;
    const int64_t row_begin = static_cast<int64_t>(chunk) * RB * kRounds;
    if (row_begin >= rows) return;
    // Page id, output offset and shift together: one memory latency for the three (all in
    // bounds: r < R, pg < max_pages <= table stride).
    const int32_t page_id = ld_meta(p.table + static_cast<int64_t>(r) * p.table_stride + pg);
    void* ko_r = nullptr;
    void* vo_r = nullptr;
    int64_t off = 0;
    if constexpr (kPtrs) {
        if (has_k) ko_r = reinterpret_cast<void*>(ld_meta(reinterpret_cast<const int64_t*>(p.ko_ptrs) + r));
        if (has_v) vo_r = reinterpret_cast<void*>(ld_meta(reinterpret_cast<const int64_t*>(p.vo_ptrs) + r));
        off = p.ptr_off;
    } else {
        off = ld_meta(p.out_off + r);
    }
    const float dp = has_k ? ld_meta(p.dp + r * p.dp_r + pg * p.dp_pg) : 0.0f;
    if (page_id < 0 || page_id >= p.n_pool_pages) {
        if (reporter) atomicOr(p.status, SC_STATUS_BAD_PAGE_ID);
        return;
    }
    {
        // Output range of this page: rows tok0 .. tok0+n_tok-1, heads 0 .. H-1.
        const int64_t first = off + static_cast<int64_t>(tok0) * p.o_t;
        const int64_t last = first + static_cast<int64_t>(n_tok - 1) * p.o_t +
                             static_cast<int64_t>(p.H - 1) * p.o_h + p.D;
        const bool misaligned =
            kPtrs && ((reinterpret_cast<uintptr_t>(ko_r) | reinterpret_cast<uintptr_t>(vo_r)) & 31) != 0;
        if ((off & 15) != 0 || misaligned || first < 0 || last > p.out_numel || p.o_t < 0 ||
            p.o_h < 0) {
            if (reporter) atomicOr(p.status, SC_STATUS_BAD_OUT_OFFSET);
            return;
        }
    }

    // Every round's rows in flight at once: codes into this thread's slots, scales into
    // registers.
    const int64_t prow0 = static_cast<int64_t>(page_id) * p.page * p.H + row_begin + rl;
    const int64_t srow0 = prow0 + r * p.sc_skew;
    __half ksc[kRounds], vsc[kRounds];
#pragma unroll
    for (int round = 0; round < kRounds; ++round) {
        if (row_begin + static_cast<int64_t>(round) * RB + rl < rows) {
            const int64_t prow = prow0 + static_cast<int64_t>(round) * RB;
            const int64_t srow = srow0 + static_cast<int64_t>(round) * RB;
            const int64_t src = prow * p.D + j * 16;
            if (has_k) {
                cp_async16(&s_codes[round][0][tid], p.kq + src);
                cp_async16(&s_codes[round][1][tid], p.kq + src + half);
                ksc[round] = p.ks[srow];
            }
            if (has_v) {
                cp_async16(&s_codes[round][2][tid], p.vq + src);
                cp_async16(&s_codes[round][3][tid], p.vq + src + half);
                vsc[round] = p.vs[srow];
            }
        }
    }
    cp_async_commit();
    if (has_k) {
        for (int f = tid; f < half; f += blockDim.x) rope_cs(dp, p.inv_freq[f], s_cos[f], s_sin[f]);
        __syncthreads();
    }
    cp_async_wait_all();
    const CsShared cs{reinterpret_cast<const float4*>(s_cos + j * 16),
                      reinterpret_cast<const float4*>(s_sin + j * 16)};
#pragma unroll
    for (int round = 0; round < kRounds; ++round) {
        const int64_t row = row_begin + static_cast<int64_t>(round) * RB + rl;
        if (row >= rows) continue;
        const int64_t oo = page_out_offset(p, static_cast<int32_t>(row), j, off, tok0);
        if (has_k) {
            OutT* o = reinterpret_cast<OutT*>(kPtrs ? ko_r : p.ko) + oo;
            rope_slice_store<OutT, __half, X16>(s_codes[round][0][tid], s_codes[round][1][tid],
                                               ksc[round], cs, o, o + half);
        }
        if (has_v) {
            OutT* o = reinterpret_cast<OutT*>(kPtrs ? vo_r : p.vo) + oo;
            value_slice_store<OutT, __half>(s_codes[round][2][tid], vsc[round], o);
            value_slice_store<OutT, __half>(s_codes[round][3][tid], vsc[round], o + half);
        }
    }
}

template <typename OutT, bool X16>
cudaError_t launch(const PagedParams& p, cudaStream_t stream) {
    const int threads = (kPThreads / p.P) * p.P;
    const int64_t blocks = static_cast<int64_t>(p.R) * p.max_pages * p.chunks;
    if (p.ko_ptrs != nullptr || p.vo_ptrs != nullptr)
        paged_restore<OutT, X16, true><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(p);
    else
        paged_restore<OutT, X16, false><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(p);
    return cudaGetLastError();
}

// Scattered pieces from a device-accessible source (the pipeline's mapped pinned scale slab)
// into a packed staging buffer: piece (t, i) of the output, n pieces per row, is piece
// ids[i] of source row t (src_blocks pieces per row).  One warp per piece, four 16-byte loads
// in flight per lane.  Reading pinned host memory from the SMs moves many small pieces at
// PCIe rate (measured on B200: 8192 scattered 1 KiB pieces in 0.17 ms, 49 GB/s), where one
// copy-engine command per piece costs about 4 us each.
__global__ void __launch_bounds__(256)
    gather_pieces(const uint4* __restrict__ src, int64_t src_blocks, uint4* __restrict__ dst,
                  const int32_t* __restrict__ ids, int32_t n, int64_t n_pieces, int32_t piece16,
                  int32_t* status) {
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= n_pieces) return;
    const int64_t t = warp / n;
    const int32_t b = ids[warp - t * n];
    if (b < 0 || b >= src_blocks) {
        if (lane == 0) atomicOr(status, SC_STATUS_BAD_PAGE_ID);
        return;
    }
    const uint4* s = src + (t * src_blocks + b) * piece16;
    uint4* d = dst + warp * piece16;
    for (int o = lane; o < piece16; o += 128) {
        uint4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (o + 32 * k < piece16) v[k] = s[o + 32 * k];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (o + 32 * k < piece16) d[o + 32 * k] = v[k];
    }
}

// Staged pieces into scattered blocks of a device-accessible destination (the pipeline's
// mapped pinned slabs): piece (t, i) of the source (row pitch src_pitch pieces) goes to piece
// t * dst_pitch + ids[i] of the destination.  The ids travel in the kernel parameters (at most
// kMaxScatterIds per launch), so no upload precedes the kernel.  One warp per piece, four
// 16-byte loads in flight per lane; SM stores into pinned host memory reach 51-53 GB/s over
// PCIe whatever the piece size or order (measured on B200), where a device-to-host copy per
// piece costs about 5 us of copy-engine time each.
struct ScatterParams {
    const uint4* src;
    uint4* dst;
    int64_t src_pitch, dst_pitch, bound;
    int32_t n, rows, piece16;
    int32_t* status;
    int32_t ids[kMaxScatterIds];
};

__global__ void __launch_bounds__(256) scatter_pieces(const __grid_constant__ ScatterParams p) {
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= static_cast<int64_t>(p.rows) * p.n) return;
    const int32_t t = static_cast<int32_t>(warp / p.n);
    const int32_t i = static_cast<int32_t>(warp - static_cast<int64_t>(t) * p.n);
    const int32_t b = p.ids[i];
    if (b < 0 || b >= p.bound) {
        if (lane == 0) atomicOr(p.status, SC_STATUS_BAD_PAGE_ID);
        return;
    }
    const uint4* s = p.src + (t * p.src_pitch + i) * p.piece16;
    uint4* d = p.dst + (t * p.dst_pitch + b) * p.piece16;
    for (int o = lane; o < p.piece16; o += 128) {
        uint4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (o + 32 * k < p.piece16) v[k] = s[o + 32 * k];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (o + 32 * k < p.piece16) d[o + 32 * k] = v[k];
    }
}

}  // namespace

cudaError_t preload_paged_kernels() {
    cudaFuncAttributes attr;
    cudaError_t e = cudaFuncGetAttributes(&attr, gather_pieces);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, scatter_pieces);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore<__half, true, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore<__half, false, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore<__nv_bfloat16, true, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore<__nv_bfloat16, false, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore<__half, true, true>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore<__half, false, true>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore<__nv_bfloat16, true, true>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore<__nv_bfloat16, false, true>);
    return e;
}

int32_t launch_paged(const PagedArgs& a) {
    if (a.n_requests < 0 || a.max_pages < 0 || a.page_size <= 0 || a.n_heads <= 0 ||
        a.n_pool_pages < 0)
        return set_error(SC_ERR_INVALID_ARGUMENT, "invalid paged geometry");
    if (a.head_dim <= 0 || a.head_dim % 32 != 0 || a.head_dim > kMaxHeadDim)
        return set_error(SC_ERR_UNSUPPORTED,
                         "paged restore needs head_dim a multiple of 32 up to %d, got %d",
                         kMaxHeadDim, a.head_dim);
    if (a.out_dtype != SC_DTYPE_F16 && a.out_dtype != SC_DTYPE_BF16)
        return set_error(SC_ERR_INVALID_DTYPE, "output dtype code %d: float16 or bfloat16 only",
                         a.out_dtype);
    if (a.n_requests == 0 || a.max_pages == 0) return ok();
    const bool has_k = a.pool_kq != nullptr, has_v = a.pool_vq != nullptr;
    if (!has_k && !has_v) return set_error(SC_ERR_INVALID_ARGUMENT, "neither K nor V given");
    const bool ptrs = a.k_out_ptrs != nullptr || a.v_out_ptrs != nullptr;
    if ((has_k && (!a.pool_ks || !(ptrs ? a.k_out_ptrs : a.k_out))) ||
        (has_v && (!a.pool_vs || !(ptrs ? a.v_out_ptrs : a.v_out))))
        return set_error(SC_ERR_INVALID_ARGUMENT, "pool tensor given without scale or output");
    if (!a.page_table || !a.seq_lens || (!ptrs && !a.out_offsets) || !a.status ||
        (has_k && !a.delta_p))
        return set_error(SC_ERR_INVALID_ARGUMENT, "null page table / lengths / offsets / status");
    if (a.delta_p_per_page < 0 || a.delta_p_per_page > 2)
        return set_error(SC_ERR_INVALID_ARGUMENT, "delta_p_per_page %d", a.delta_p_per_page);
    if (a.page_table_stride < a.max_pages)
        return set_error(SC_ERR_INVALID_ARGUMENT, "page_table_stride %lld < max_pages %d",
                         (long long)a.page_table_stride, a.max_pages);
    if (a.out_strides[2] != 1 || a.out_strides[0] % 16 != 0 || a.out_strides[1] % 16 != 0)
        return set_error(SC_ERR_INVALID_ARGUMENT,
                         "output strides must be [t, h, 1] with t, h multiples of 16 elements");
    auto al = [](const void* ptr, uintptr_t n) { return (reinterpret_cast<uintptr_t>(ptr) % n) == 0; };
    if ((has_k && (!al(a.pool_kq, 16) || (!ptrs && !al(a.k_out, 32)))) ||
        (has_v && (!al(a.pool_vq, 16) || (!ptrs && !al(a.v_out, 32)))))
        return set_error(SC_ERR_INVALID_ARGUMENT,
                         "pools must be 16-byte and outputs 32-byte aligned");
    if (static_cast<int64_t>(a.page_size) * a.n_heads >= (int64_t(1) << 31))
        return set_error(SC_ERR_INVALID_ARGUMENT, "page_size * n_heads too large");

    const int64_t rows_per_block = static_cast<int64_t>(kPThreads / (a.head_dim / 32)) * SC_PAGED_ROUNDS;
    const int64_t chunks = (static_cast<int64_t>(a.page_size) * a.n_heads + rows_per_block - 1) /
                           rows_per_block;
    if (size_product(a.n_requests, a.max_pages, chunks) >= (int64_t(1) << 31))
        return set_error(SC_ERR_INVALID_ARGUMENT, "too many (request, page) blocks in one call");

    PagedParams p{};
    p.chunks = static_cast<int32_t>(chunks);
    p.R = a.n_requests;
    p.max_pages = a.max_pages;
    p.page = a.page_size;
    p.H = a.n_heads;
    p.D = a.head_dim;
    p.P = a.head_dim / 32;
    p.n_pool_pages = a.n_pool_pages;
    p.divH = make_fastdiv(static_cast<uint32_t>(a.n_heads));
    p.kq = a.pool_kq;
    p.ks = static_cast<const __half*>(a.pool_ks);
    p.vq = a.pool_vq;
    p.vs = static_cast<const __half*>(a.pool_vs);
    p.table = a.page_table;
    p.table_stride = a.page_table_stride;
    p.seq_lens = a.seq_lens;
    p.seq_r = a.seq_len_shared ? 0 : 1;
    p.dp = a.delta_p;
    p.dp_r = a.delta_p_per_page == 0 ? 1 : a.delta_p_per_page == 1 ? a.max_pages : 0;
    p.dp_pg = a.delta_p_per_page == 0 ? 0 : 1;
    p.sc_skew = a.scale_request_skew;
    p.ko = a.k_out;
    p.vo = a.v_out;
    p.ko_ptrs = a.k_out_ptrs;
    p.vo_ptrs = a.v_out_ptrs;
    p.ptr_off = a.out_ptr_offset;
    p.out_off = a.out_offsets;
    p.o_t = a.out_strides[0];
    p.o_h = a.out_strides[1];
    p.out_numel = a.out_numel;
    p.status = a.status;
    if (a.inv_freq)
        for (int i = 0; i < a.head_dim / 2; ++i) p.inv_freq[i] = a.inv_freq[i];
    else
        default_inv_freq(a.head_dim, a.theta_base, p.inv_freq);
    const bool x16 = !(a.flags & SC_FLAG_FP32_INTERMEDIATE);
    cudaError_t e;
    if (a.out_dtype == SC_DTYPE_F16)
        e = x16 ? launch<__half, true>(p, a.stream) : launch<__half, false>(p, a.stream);
    else
        e = x16 ? launch<__nv_bfloat16, true>(p, a.stream)
                : launch<__nv_bfloat16, false>(p, a.stream);
    if (e != cudaSuccess) return cuda_error(e, "paged restore launch");
    return ok();
}

int32_t launch_gather_pieces(const void* src, int64_t src_blocks, void* dst, const int32_t* ids,
                             int32_t n, int32_t rows, int64_t piece_bytes, int32_t* status,
                             cudaStream_t stream) {
    if (!src || !dst || !ids || !status || n < 0 || rows < 0 || src_blocks <= 0 ||
        piece_bytes <= 0 || piece_bytes % 16 != 0 || piece_bytes / 16 > (int64_t(1) << 30) ||
        (reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) % 16 != 0)
        return set_error(SC_ERR_INVALID_ARGUMENT, "invalid piece gather");
    const int64_t n_pieces = static_cast<int64_t>(rows) * n;
    if (n_pieces == 0) return ok();
    const int64_t blocks = (n_pieces * 32 + 255) / 256;
    if (blocks >= (int64_t(1) << 31)) return set_error(SC_ERR_INVALID_ARGUMENT, "too many pieces");
    gather_pieces<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const uint4*>(src), src_blocks, static_cast<uint4*>(dst), ids, n, n_pieces,
        static_cast<int32_t>(piece_bytes / 16), status);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "piece gather launch");
    return ok();
}

int32_t launch_scatter_pieces(const void* src, int64_t src_pitch, void* dst, int64_t dst_pitch,
                              int64_t bound, const int32_t* ids, int32_t n, int32_t rows,
                              int64_t piece_bytes, int32_t* status, cudaStream_t stream) {
    if (!src || !dst || !ids || !status || n < 0 || rows < 0 || bound <= 0 || src_pitch < n ||
        dst_pitch < bound || piece_bytes <= 0 || piece_bytes % 16 != 0 ||
        piece_bytes / 16 > (int64_t(1) << 30) ||
        (reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) % 16 != 0)
        return set_error(SC_ERR_INVALID_ARGUMENT, "invalid piece scatter");
    ScatterParams p{};
    p.dst = static_cast<uint4*>(dst);
    p.src_pitch = src_pitch;
    p.dst_pitch = dst_pitch;
    p.bound = bound;
    p.rows = rows;
    p.piece16 = static_cast<int32_t>(piece_bytes / 16);
    p.status = status;
    for (int32_t i0 = 0; i0 < n; i0 += kMaxScatterIds) {
        p.n = n - i0 < kMaxScatterIds ? n - i0 : kMaxScatterIds;
        p.src = static_cast<const uint4*>(src) + static_cast<int64_t>(i0) * p.piece16;
        for (int32_t i = 0; i < p.n; ++i) p.ids[i] = ids[i0 + i];
        const int64_t blocks = (static_cast<int64_t>(rows) * p.n * 32 + 255) / 256;
        if (blocks == 0) continue;
        scatter_pieces<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(p);
        const cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_error(e, "piece scatter launch");
    }
    return ok();
}

}  // namespace sc

extern "C" int32_t sc_restore_paged(int32_t n_requests, int32_t max_pages, int32_t page_size,
                                    int32_t n_heads, int32_t head_dim, int64_t n_pool_pages,
                                    const int8_t* pool_kq, const void* pool_ks,
                                    const int8_t* pool_vq, const void* pool_vs,
                                    const int32_t* page_table, int64_t page_table_stride,
                                    const int32_t* seq_lens, const float* delta_p,
                                    int32_t delta_p_per_page, double theta_base,
                                    const float* inv_freq, void* k_out, void* v_out,
                                    const int64_t* out_offsets, const int64_t* out_strides,
                                    int64_t out_numel, int32_t out_dtype, int32_t* status,
                                    uint32_t flags, void* stream) {
    if (!out_strides) return sc::set_error(SC_ERR_INVALID_ARGUMENT, "null out_strides");
    if (delta_p_per_page != 0 && delta_p_per_page != 1)
        return sc::set_error(SC_ERR_INVALID_ARGUMENT, "delta_p_per_page must be 0 or 1, got %d",
                             delta_p_per_page);
    sc::PagedArgs a{};
    a.n_requests = n_requests;
    a.max_pages = max_pages;
    a.page_size = page_size;
    a.n_heads = n_heads;
    a.head_dim = head_dim;
    a.n_pool_pages = n_pool_pages;
    a.pool_kq = pool_kq;
    a.pool_ks = pool_ks;
    a.pool_vq = pool_vq;
    a.pool_vs = pool_vs;
    a.page_table = page_table;
    a.page_table_stride = page_table_stride;
    a.seq_lens = seq_lens;
    a.delta_p = delta_p;
    a.delta_p_per_page = delta_p_per_page;
    a.theta_base = theta_base;
    a.inv_freq = inv_freq;
    a.k_out = k_out;
    a.v_out = v_out;
    a.out_offsets = out_offsets;
    for (int i = 0; i < 3; ++i) a.out_strides[i] = out_strides[i];
    a.out_numel = out_numel;
    a.out_dtype = out_dtype;
    a.status = status;
    a.flags = flags;
    a.stream = static_cast<cudaStream_t>(stream);
    return sc::launch_paged(a);
}
