// sc_paged.cu — ragged, paged restore: page-table gather + INT8 dequant + relative RoPE
// shift, written straight into contiguous per-request caches.
//
// Per row (one token-head of a page), each thread owns a 16-frequency slice: it reads 16
// codes of the first half and their rotate-half partners (two 16-byte pieces per tensor),
// converts them with the row's scale and the request's (or page's) cos/sin table, and
// writes each 16 outputs with one 32-byte store.  The table is built in shared memory
// (single-precision sincos, double precision only where the fp16 rounding is not settled,
// rounded like the reference's fp16 tables).  Two kernels share that per-row work:
//
// * paged_restore_stream (the default): persistent blocks walk only the live tiles (a tile
//   is TR = threads / (D/32) consecutive rows of one page).  Every block reads the request
//   lengths, counts each request's tiles and scans the counts in shared memory, then takes
//   an equal share of the tiles.  Each thread stages its own row-slice of the next tiles in
//   shared memory with cp.async (SC_PSTREAM_STAGES tiles in flight per block, no register
//   cost, no barrier on the data: a thread reads only what it copied, after
//   cp.async.wait_group), and the page id, shift and output offset of the page after the
//   current one are loaded a page ahead.  So no block is launched for pages past a request's
//   end, no block waits on metadata before its first load, and the bytes in flight per SM
//   are bounded by shared memory instead of registers.
// * paged_restore (SC_FLAG_PAGED_ONE_SHOT, more than kMaxStreamRequests requests, odd
//   page * heads, scale arrays not 4-byte aligned): one-shot blocks, one per (request,
//   page, chunk of the page's rows).  A block first reads its request's length and exits
//   at once if its page lies past it; otherwise it reads the page id, output offset and
//   shift together (one memory latency for the three), builds the table, then walks
//   SC_PAGED_ROUNDS groups of rows, loading each row-slice into registers.
//
// Device-side checks never fault: a page id outside the pool, a bad sequence length or an
// output range outside out_numel makes the block skip the work and OR a status bit into
// the caller's status word.
#include "sc_common.cuh"

namespace sc {
namespace {

// Threads per block (128-thread blocks at 8 per SM measured within 1 % either way).
#ifndef SC_PAGED_THREADS
#define SC_PAGED_THREADS 256
#endif
constexpr int kPThreads = SC_PAGED_THREADS;
#ifndef SC_PAGED_MIN_BLOCKS
#define SC_PAGED_MIN_BLOCKS 4
#endif
#ifndef SC_PAGED_ROWS_PER_THREAD
#define SC_PAGED_ROWS_PER_THREAD 1
#endif
// Build the block's cos/sin table before issuing the page loads (1) or while they are in
// flight (0).
#ifndef SC_PAGED_TABLE_FIRST
#define SC_PAGED_TABLE_FIRST 1
#endif
// Consecutive row groups a block walks (its cos/sin table is built once for all of them).
#ifndef SC_PAGED_ROUNDS
#define SC_PAGED_ROUNDS 2
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

struct PagedParams {
    int32_t R, max_pages, page, H, D, P;
    int32_t chunks;  // blocks per page (page * H rows split into chunks of RB * rows/thread)
    int32_t tile_rows, tiles_per_page;  // streaming kernel: rows per tile, tiles per full page
    int64_t n_pool_pages;
    FastDiv divH;
    const int8_t* kq;
    const __half* ks;
    const int8_t* vq;
    const __half* vs;
    const int32_t* table;
    int64_t table_stride;
    const int32_t* seq_lens;
    const float* dp;
    int32_t dp_per_page;
    void* ko;
    void* vo;
    const uint64_t* ko_ptrs;  // per-request output buffers (device), or null: ko/vo + out_off
    const uint64_t* vo_ptrs;
    const int64_t* out_off;
    int64_t o_t, o_h;
    int64_t out_numel;
    int32_t* status;
    float inv_freq[kMaxHeadDim / 2];
};

// What a thread carries from the load of a row-slice to its store: codes, scales and the
// row index (the output address is recomputed at the store).
struct PageRow {
    uint4 ka, kb, va, vb;
    __half ksc, vsc;
    int32_t row;  // -1 when past the page's rows
};

__device__ __forceinline__ void load_page_row(const PagedParams& p, int64_t row, int64_t rows,
                                              int j, int half, int64_t pbase, int64_t sbase,
                                              bool has_k, bool has_v, PageRow& r) {
    if (row >= rows) {
        r.row = -1;
        return;
    }
    r.row = static_cast<int32_t>(row);
    const int64_t src = pbase + row * p.D + j * 16;
    if (has_k) {
        r.ka = ld_stream_v4(p.kq + src);
        r.kb = ld_stream_v4(p.kq + src + half);
        r.ksc = p.ks[sbase + row];
    }
    if (has_v) {
        r.va = ld_stream_v4(p.vq + src);
        r.vb = ld_stream_v4(p.vq + src + half);
        r.vsc = p.vs[sbase + row];
    }
}

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
    constexpr int RT = SC_PAGED_ROWS_PER_THREAD;
    const int P = p.P;
    const int j = threadIdx.x % P;
    const int rl = threadIdx.x / P;
    const int RB = blockDim.x / P;
    const int half = p.D >> 1;
    const bool has_k = p.kq != nullptr, has_v = p.vq != nullptr;

    const int64_t task = blockIdx.x / p.chunks;
    const int chunk = static_cast<int>(blockIdx.x - task * p.chunks);
    const int r = static_cast<int>(task / p.max_pages);
    const int pg = static_cast<int>(task - static_cast<int64_t>(r) * p.max_pages);
    const bool reporter = chunk == 0 && threadIdx.x == 0;
    // The length alone first: a block past its request's length exits after one load.
    const int len = p.seq_lens[r];
    if (len < 0 || static_cast<int64_t>(len) > static_cast<int64_t>(p.max_pages) * p.page) {
        if (reporter && pg == 0) atomicOr(p.status, SC_STATUS_BAD_SEQ_LEN);
        return;
    }
    const int tok0 = pg * p.page;
    if (tok0 >= len) return;
    const int n_tok = min(p.page, len - tok0);
    const int64_t rows = static_cast<int64_t>(n_tok) * p.H;
    const int64_t row_begin = static_cast<int64_t>(chunk) * RB * RT * SC_PAGED_ROUNDS;
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
    } else {
        off = ld_meta(p.out_off + r);
    }
    const float dp_blk = has_k ? ld_meta(p.dp + (p.dp_per_page ? task : r)) : 0.0f;
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
    auto block_dp = [&] { return dp_blk; };
#if SC_PAGED_TABLE_FIRST
    if (has_k) {
        const float dp = block_dp();
        for (int f = threadIdx.x; f < half; f += blockDim.x) rope_cs(dp, p.inv_freq[f], s_cos[f], s_sin[f]);
        __syncthreads();
    }
#endif
    const CsShared cs{reinterpret_cast<const float4*>(s_cos + j * 16),
                      reinterpret_cast<const float4*>(s_sin + j * 16)};
    const int64_t pbase = static_cast<int64_t>(page_id) * p.page * p.H * p.D;
    const int64_t sbase = static_cast<int64_t>(page_id) * p.page * p.H;
    for (int round = 0; round < SC_PAGED_ROUNDS; ++round) {
    const int64_t group = row_begin + static_cast<int64_t>(round) * RB * RT;
    if (group >= rows) break;  // uniform across the block
    PageRow buf[RT];
#pragma unroll
    for (int k = 0; k < RT; ++k)
        load_page_row(p, group + k * RB + rl, rows, j, half, pbase, sbase, has_k, has_v, buf[k]);
    if (!SC_PAGED_TABLE_FIRST && round == 0 && has_k) {
        // The table is built while the first loads are in flight.
        const float dp = block_dp();
        for (int f = threadIdx.x; f < half; f += blockDim.x) rope_cs(dp, p.inv_freq[f], s_cos[f], s_sin[f]);
        __syncthreads();
    }
#pragma unroll
    for (int k = 0; k < RT; ++k) {
        if (buf[k].row < 0) continue;
        const int64_t oo = page_out_offset(p, buf[k].row, j, off, tok0);
        if (has_k) {
            OutT* o = reinterpret_cast<OutT*>(kPtrs ? ko_r : p.ko) + oo;
            rope_slice_store<OutT, __half, X16>(buf[k].ka, buf[k].kb, buf[k].ksc, cs, o, o + half);
        }
        if (has_v) {
            OutT* o = reinterpret_cast<OutT*>(kPtrs ? vo_r : p.vo) + oo;
            value_slice_store<OutT, __half>(buf[k].va, buf[k].vsc, o);
            value_slice_store<OutT, __half>(buf[k].vb, buf[k].vsc, o + half);
        }
    }
    }
}

// ---------------------------------------------------------------------------------------
// Streaming kernel
// ---------------------------------------------------------------------------------------
#ifndef SC_PSTREAM_THREADS
#define SC_PSTREAM_THREADS 256
#endif
#ifndef SC_PSTREAM_STAGES
#define SC_PSTREAM_STAGES 3
#endif
#ifndef SC_PSTREAM_MIN_BLOCKS
#define SC_PSTREAM_MIN_BLOCKS 3
#endif
constexpr int kSThreads = SC_PSTREAM_THREADS;
constexpr int kStages = SC_PSTREAM_STAGES;
static_assert(kStages >= 2, "the streaming kernel needs at least two stages");
constexpr int kMaxStreamRequests = 1024;

// What the issuing side records for the converting side, per stage (written by thread 0).
struct StreamTile {
    int32_t r;       // request
    int32_t tok0;    // first token of the tile's page
    int32_t row0;    // first page row of the tile
    int32_t n_rows;  // rows to convert (0: none)
    float dp;        // the shift of the tile's request (or page)
    int32_t pad;
    int64_t off;     // output element offset of the request (offset mode)
    uint64_t ko, vo;  // the request's output buffers (pointer mode)
};

struct alignas(16) StreamShared {
    uint4 codes[kStages][4][kSThreads];      // K first half, K second half, V first, V second
    uint32_t scales[kStages][2][kSThreads];  // K, V: the 4-byte pair holding the row's scale
    StreamTile tile[kStages];
    alignas(16) float cos_[kMaxHeadDim / 2];
    alignas(16) float sin_[kMaxHeadDim / 2];
    int32_t lens[kMaxStreamRequests];
    int32_t first_tile[kMaxStreamRequests + 1];  // exclusive prefix of the tiles per request
    int32_t warp_sum[kSThreads / 32];
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ int32_t request_tiles(int32_t len, const PagedParams& p) {
    if (len <= 0) return 0;
    const int32_t np = (len + p.page - 1) / p.page;
    const int32_t rows_last = (len - (np - 1) * p.page) * p.H;
    return (np - 1) * p.tiles_per_page + (rows_last + p.tile_rows - 1) / p.tile_rows;
}

// A page of the walk and its metadata, loaded ahead of use.
struct PageRef {
    int32_t r, pg;  // r < 0: past the last page
    int32_t pid;
    float dp;
    int64_t off;
    uint64_t ko, vo;
};

template <bool kPtrs>
__device__ __forceinline__ void load_page(const PagedParams& p, int32_t r, int32_t pg, bool has_k,
                                          bool has_v, PageRef& q) {
    q.r = r;
    q.pg = pg;
    if (r < 0) return;
    q.pid = ld_meta(p.table + static_cast<int64_t>(r) * p.table_stride + pg);
    q.dp = has_k ? ld_meta(p.dp + (p.dp_per_page ? static_cast<int64_t>(r) * p.max_pages + pg : r)) : 0.0f;
    if constexpr (kPtrs) {
        q.ko = has_k ? static_cast<uint64_t>(ld_meta(reinterpret_cast<const int64_t*>(p.ko_ptrs) + r)) : 0;
        q.vo = has_v ? static_cast<uint64_t>(ld_meta(reinterpret_cast<const int64_t*>(p.vo_ptrs) + r)) : 0;
        q.off = 0;
    } else {
        q.off = ld_meta(p.out_off + r);
        q.ko = q.vo = 0;
    }
}

// The page after (r, pg) in the walk: the next page of r, else page 0 of the next request
// with tiles; r = -1 past the end.
__device__ __forceinline__ void next_page(const StreamShared& sm, const PagedParams& p,
                                          int32_t r, int32_t pg, int32_t& nr, int32_t& npg) {
    const int32_t np = (sm.lens[r] + p.page - 1) / p.page;
    if (pg + 1 < np) {
        nr = r;
        npg = pg + 1;
        return;
    }
    int32_t q = r + 1;
    while (q < p.R && sm.first_tile[q + 1] == sm.first_tile[q]) ++q;
    nr = q < p.R ? q : -1;
    npg = 0;
}

template <typename OutT, bool X16, bool kPtrs>
__global__ void __launch_bounds__(kSThreads, SC_PSTREAM_MIN_BLOCKS)
    paged_restore_stream(const __grid_constant__ PagedParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    StreamShared& sm = *reinterpret_cast<StreamShared*>(smem_raw);
    const int tid = threadIdx.x;
    const int P = p.P;
    const int j = tid % P;
    const int rl = tid / P;  // < tile_rows: blockDim.x == tile_rows * P
    const int half = p.D >> 1;
    const int TR = p.tile_rows;
    const bool has_k = p.kq != nullptr, has_v = p.vq != nullptr;
    const int R = p.R;

    // 1. Lengths (a bad one counts as empty; block 0 reports it).
    for (int r = tid; r < R; r += blockDim.x) {
        int32_t len = p.seq_lens[r];
        if (len < 0 || static_cast<int64_t>(len) > static_cast<int64_t>(p.max_pages) * p.page) {
            if (blockIdx.x == 0) atomicOr(p.status, SC_STATUS_BAD_SEQ_LEN);
            len = 0;
        }
        sm.lens[r] = len;
    }
    __syncthreads();
    // 2. Exclusive scan of the tiles per request: thread t owns requests [t*per, t*per+per).
    const int per = (R + blockDim.x - 1) / blockDim.x;
    const int r0 = min(R, tid * per), r1 = min(R, r0 + per);
    int32_t local = 0;
    for (int r = r0; r < r1; ++r) local += request_tiles(sm.lens[r], p);
    const int lane = tid & 31, warp = tid >> 5, n_warps = (blockDim.x + 31) >> 5;
    int32_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31 || tid == blockDim.x - 1) sm.warp_sum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int32_t w = lane < n_warps ? sm.warp_sum[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int32_t v = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += v;
        }
        if (lane < n_warps) sm.warp_sum[lane] = w;  // inclusive totals per warp
    }
    __syncthreads();
    int32_t run = incl - local + (warp > 0 ? sm.warp_sum[warp - 1] : 0);
    for (int r = r0; r < r1; ++r) {
        sm.first_tile[r] = run;
        run += request_tiles(sm.lens[r], p);
    }
    if (tid == 0) sm.first_tile[R] = sm.warp_sum[n_warps - 1];
    __syncthreads();
    const int32_t total = sm.first_tile[R];
    const int32_t t_begin = static_cast<int32_t>(static_cast<int64_t>(total) * blockIdx.x / gridDim.x);
    const int32_t t_end = static_cast<int32_t>(static_cast<int64_t>(total) * (blockIdx.x + 1) / gridDim.x);
    if (t_begin >= t_end) return;  // uniform across the block

    // 3. The walk starts at the request holding t_begin (last r with first_tile[r] <= t_begin).
    int32_t lo = 0, hi = R - 1;
    while (lo < hi) {
        const int32_t mid = (lo + hi + 1) >> 1;
        if (sm.first_tile[mid] <= t_begin) lo = mid;
        else hi = mid - 1;
    }
    int32_t wr = lo;
    const int32_t lt = t_begin - sm.first_tile[wr];
    int32_t wpg = lt / p.tiles_per_page;
    int32_t wc = lt - wpg * p.tiles_per_page;
    PageRef cur, nxt;
    load_page<kPtrs>(p, wr, wpg, has_k, has_v, cur);
    {
        int32_t nr, npg;
        next_page(sm, p, wr, wpg, nr, npg);
        load_page<kPtrs>(p, nr, npg, has_k, has_v, nxt);
    }
    bool cur_checked = false, cur_ok = false;

    // Issue the copies of the walk's current tile into stage s, record it, step the walk.
    auto issue = [&](int s) {
        const int32_t len = sm.lens[wr];
        const int32_t tok0 = wpg * p.page;
        const int32_t n_tok = min(p.page, len - tok0);
        if (!cur_checked) {
            cur_checked = true;
            cur_ok = true;
            if (cur.pid < 0 || cur.pid >= p.n_pool_pages) {
                cur_ok = false;
                if (tid == 0) atomicOr(p.status, SC_STATUS_BAD_PAGE_ID);
            } else {
                const int64_t first = cur.off + static_cast<int64_t>(tok0) * p.o_t;
                const int64_t last = first + static_cast<int64_t>(n_tok - 1) * p.o_t +
                                     static_cast<int64_t>(p.H - 1) * p.o_h + p.D;
                const bool misaligned = kPtrs && ((cur.ko | cur.vo) & 31) != 0;
                if ((cur.off & 15) != 0 || misaligned || first < 0 || last > p.out_numel ||
                    p.o_t < 0 || p.o_h < 0) {
                    cur_ok = false;
                    if (tid == 0) atomicOr(p.status, SC_STATUS_BAD_OUT_OFFSET);
                }
            }
        }
        const int32_t rows_pg = n_tok * p.H;
        const int32_t row0 = wc * TR;
        const int32_t n = cur_ok ? min(TR, rows_pg - row0) : 0;
        if (rl < n) {
            const int64_t prow = static_cast<int64_t>(cur.pid) * p.page * p.H + row0 + rl;
            const int64_t src = prow * p.D + j * 16;
            if (has_k) {
                cp_async16(&sm.codes[s][0][tid], p.kq + src);
                cp_async16(&sm.codes[s][1][tid], p.kq + src + half);
                cp_async4(&sm.scales[s][0][tid], p.ks + (prow & ~int64_t(1)));
            }
            if (has_v) {
                cp_async16(&sm.codes[s][2][tid], p.vq + src);
                cp_async16(&sm.codes[s][3][tid], p.vq + src + half);
                cp_async4(&sm.scales[s][1][tid], p.vs + (prow & ~int64_t(1)));
            }
        }
        if (tid == 0) {
            StreamTile& t = sm.tile[s];
            t.r = wr;
            t.tok0 = tok0;
            t.row0 = row0;
            t.n_rows = n;
            t.dp = cur.dp;
            t.off = cur.off;
            t.ko = cur.ko;
            t.vo = cur.vo;
        }
        // step: next tile of the page, else the next page (whose metadata is in flight)
        const int32_t tiles_pg = (rows_pg + TR - 1) / TR;
        if (++wc == tiles_pg) {
            wc = 0;
            cur = nxt;
            wr = cur.r;
            wpg = cur.pg;
            cur_checked = false;
            if (wr >= 0) {
                int32_t nr, npg;
                next_page(sm, p, wr, wpg, nr, npg);
                load_page<kPtrs>(p, nr, npg, has_k, has_v, nxt);
            }
        }
    };

    const CsShared cs{reinterpret_cast<const float4*>(sm.cos_ + j * 16),
                      reinterpret_cast<const float4*>(sm.sin_ + j * 16)};
    uint32_t table_bits = 0;
    bool table_valid = false;
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
        if (t_begin + s < t_end) issue(s);
        cp_async_commit();
    }
    int stage = 0;
    for (int32_t i = t_begin; i < t_end; ++i) {
        __syncthreads();  // tile i-1 is consumed: its stage, its record and the table are free
        if (i + kStages - 1 < t_end) issue(stage == 0 ? kStages - 1 : stage - 1);
        cp_async_commit();
        cp_async_wait<kStages - 1>();  // this thread's copies of tile i have landed
        const StreamTile& t = sm.tile[stage];
        const int32_t n_rows = t.n_rows;
        const float dp = t.dp;
        if (has_k && n_rows > 0 && (!table_valid || __float_as_uint(dp) != table_bits)) {
            // uniform: every thread reads the same record
            for (int f = tid; f < half; f += blockDim.x) rope_cs(dp, p.inv_freq[f], sm.cos_[f], sm.sin_[f]);
            __syncthreads();
            table_bits = __float_as_uint(dp);
            table_valid = true;
        }
        if (rl < n_rows) {
            const int32_t row = t.row0 + rl;
            const uint32_t c = fdiv(static_cast<uint32_t>(row), p.divH);
            const int64_t h = row - static_cast<int64_t>(c) * p.H;
            const int64_t oo = (kPtrs ? 0 : t.off) + (t.tok0 + static_cast<int64_t>(c)) * p.o_t +
                               h * p.o_h + j * 16;
            const bool odd = (row & 1) != 0;  // page * H is even, so the pool row has row's parity
            if (has_k) {
                const uint32_t pr = sm.scales[stage][0][tid];
                const __half sc = __ushort_as_half(static_cast<unsigned short>(odd ? pr >> 16 : pr & 0xffffu));
                OutT* o = reinterpret_cast<OutT*>(kPtrs ? reinterpret_cast<void*>(t.ko) : p.ko) + oo;
                rope_slice_store<OutT, __half, X16>(sm.codes[stage][0][tid], sm.codes[stage][1][tid], sc,
                                                   cs, o, o + half);
            }
            if (has_v) {
                const uint32_t pr = sm.scales[stage][1][tid];
                const __half sc = __ushort_as_half(static_cast<unsigned short>(odd ? pr >> 16 : pr & 0xffffu));
                OutT* o = reinterpret_cast<OutT*>(kPtrs ? reinterpret_cast<void*>(t.vo) : p.vo) + oo;
                value_slice_store<OutT, __half>(sm.codes[stage][2][tid], sc, o);
                value_slice_store<OutT, __half>(sm.codes[stage][3][tid], sc, o + half);
            }
        }
        stage = stage + 1 == kStages ? 0 : stage + 1;
    }
    cp_async_wait<0>();  // no copy outlives the block
}

// Per-instantiation launch state: dynamic shared memory opted in and resident blocks per SM,
// per device.
struct StreamLaunchState {
    int occupancy[64] = {0};
};

template <typename OutT, bool X16, bool kPtrs>
cudaError_t launch_stream(const PagedParams& p, int64_t max_tiles, cudaStream_t stream) {
    auto kern = paged_restore_stream<OutT, X16, kPtrs>;
    static StreamLaunchState state;
    // Always kSThreads: when P does not divide it, threads past tile_rows * P own no row.
    const int threads = kSThreads;
    const size_t smem = sizeof(StreamShared);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int occ = (dev >= 0 && dev < 64) ? state.occupancy[dev] : 0;
    if (occ <= 0) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
        if (e != cudaSuccess) return e;
        if (occ <= 0) occ = 1;
        if (dev >= 0 && dev < 64) state.occupancy[dev] = occ;
    }
    const int64_t cap = static_cast<int64_t>(sm_count()) * occ;
    const int64_t grid = max_tiles < cap ? (max_tiles > 0 ? max_tiles : 1) : cap;
    kern<<<static_cast<unsigned>(grid), threads, smem, stream>>>(p);
    return cudaGetLastError();
}

template <typename OutT, bool X16>
cudaError_t launch(const PagedParams& p, bool streaming, int64_t max_tiles, cudaStream_t stream) {
    const bool ptrs = p.ko_ptrs != nullptr || p.vo_ptrs != nullptr;
    if (streaming)
        return ptrs ? launch_stream<OutT, X16, true>(p, max_tiles, stream)
                    : launch_stream<OutT, X16, false>(p, max_tiles, stream);
    const int threads = (kPThreads / p.P) * p.P;
    const int64_t blocks = static_cast<int64_t>(p.R) * p.max_pages * p.chunks;
    if (ptrs)
        paged_restore<OutT, X16, true><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(p);
    else
        paged_restore<OutT, X16, false><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t preload_paged_kernels() {
    cudaFuncAttributes attr;
    cudaError_t e = cudaFuncGetAttributes(&attr, paged_restore_stream<__half, true, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore_stream<__half, false, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore_stream<__nv_bfloat16, true, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore_stream<__nv_bfloat16, false, false>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore_stream<__half, true, true>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore_stream<__half, false, true>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore_stream<__nv_bfloat16, true, true>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&attr, paged_restore_stream<__nv_bfloat16, false, true>);
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

    const int64_t rows_per_block = static_cast<int64_t>(kPThreads / (a.head_dim / 32)) *
                                   SC_PAGED_ROWS_PER_THREAD * SC_PAGED_ROUNDS;
    const int64_t chunks = (static_cast<int64_t>(a.page_size) * a.n_heads + rows_per_block - 1) /
                           rows_per_block;
    if (static_cast<int64_t>(a.n_requests) * a.max_pages * chunks >= (int64_t(1) << 31))
        return set_error(SC_ERR_INVALID_ARGUMENT, "too many (request, page) blocks in one call");

    // Streaming kernel: tiles of kSThreads / P rows; the scale pairs it copies need page * H
    // even (a pair never reaches past the pool) and 4-byte aligned scale arrays.
    const int32_t tile_rows = kSThreads / (a.head_dim / 32);
    const int64_t tiles_per_page = (static_cast<int64_t>(a.page_size) * a.n_heads + tile_rows - 1) / tile_rows;
    const int64_t max_tiles = static_cast<int64_t>(a.n_requests) * a.max_pages * tiles_per_page;
    const bool streaming =
        !(a.flags & SC_FLAG_PAGED_ONE_SHOT) && a.n_requests <= kMaxStreamRequests &&
        (static_cast<int64_t>(a.page_size) * a.n_heads) % 2 == 0 && max_tiles < (int64_t(1) << 31) &&
        (!has_k || al(a.pool_ks, 4)) && (!has_v || al(a.pool_vs, 4));

    PagedParams p{};
    p.chunks = static_cast<int32_t>(chunks);
    p.tile_rows = tile_rows;
    p.tiles_per_page = static_cast<int32_t>(tiles_per_page);
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
    p.dp = a.delta_p;
    p.dp_per_page = a.delta_p_per_page;
    p.ko = a.k_out;
    p.vo = a.v_out;
    p.ko_ptrs = a.k_out_ptrs;
    p.vo_ptrs = a.v_out_ptrs;
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
        e = x16 ? launch<__half, true>(p, streaming, max_tiles, a.stream)
                : launch<__half, false>(p, streaming, max_tiles, a.stream);
    else
        e = x16 ? launch<__nv_bfloat16, true>(p, streaming, max_tiles, a.stream)
                : launch<__nv_bfloat16, false>(p, streaming, max_tiles, a.stream);
    if (e != cudaSuccess) return cuda_error(e, "paged restore launch");
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
