// sc_internal.h — host-side internals shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "speccache_b200.h"

namespace sc {

// Record a message for sc_last_error() on this host thread and return `code`.
int32_t set_error(int32_t code, const char* fmt, ...)
#if defined(__GNUC__)
    __attribute__((format(printf, 2, 3)))
#endif
    ;

// Clear the per-thread message (successful call).
int32_t ok();

// Map a CUDA error to SC_ERR_CUDA with context.
int32_t cuda_error(cudaError_t e, const char* what);

// Streaming multiprocessor count of the current device (cached per device).
int sm_count();

// Compute float32 inverse frequencies 1/theta^(2i/D) (double pow rounded to float32)
// when the caller gives none.  `out` has room for head_dim/2 values.
void default_inv_freq(int32_t head_dim, double theta, float* out);

// cos/sin of one shift as the reference tabulates them (angle = fp32(dp * inv_freq), cos and
// sin in double rounded to fp32 then fp16), packed as half2(cos, sin) per frequency into
// tab[head_dim / 2]; inv_freq may be null (then 1/theta^(2i/D)).  Recent tables are cached
// per host thread.
void host_cos_sin_table(int head_dim, float dp, double theta, const float* inv_freq,
                        uint32_t* tab);

// Largest head_dim handled by any kernel (the inverse-frequency table travels as a
// kernel parameter of head_dim/2 floats).
constexpr int kMaxHeadDim = 1024;

// a * b * c of non-negative sizes, or INT64_MAX when the product does not fit: a caller's
// absurd sizes then fail the size limits instead of wrapping past them.
inline int64_t size_product(int64_t a, int64_t b, int64_t c = 1) {
    int64_t ab = 0, abc = 0;
    if (__builtin_mul_overflow(a, b, &ab) || __builtin_mul_overflow(ab, c, &abc)) return INT64_MAX;
    return abc;
}

// Paged restore launch shared by sc_restore_paged and the host pipeline.
struct PagedArgs {
    int32_t n_requests, max_pages, page_size, n_heads, head_dim;
    int64_t n_pool_pages;
    const int8_t* pool_kq;
    const void* pool_ks;
    const int8_t* pool_vq;
    const void* pool_vs;
    const int32_t* page_table;
    int64_t page_table_stride;
    const int32_t* seq_lens;
    int32_t seq_len_shared;  // 1: seq_lens[0] is every request's length
    const float* delta_p;
    // 0: delta_p[r]; 1: delta_p[r * max_pages + page]; 2: delta_p[page] (shared by requests)
    int32_t delta_p_per_page;
    // Rows added to request r's scale index per request (r * scale_request_skew): lets the
    // requests' codes be packed in a staging pool while their scales keep a wider layout.
    int64_t scale_request_skew;
    double theta_base;
    const float* inv_freq;  // host, may be null
    void* k_out;
    void* v_out;
    // Per-request output buffers (device arrays of n_requests addresses, 32-byte aligned); when
    // given, request r writes from element out_ptr_offset of its own buffers and out_offsets is
    // not read.
    const uint64_t* k_out_ptrs;
    const uint64_t* v_out_ptrs;
    int64_t out_ptr_offset;
    const int64_t* out_offsets;
    int64_t out_strides[3];
    int64_t out_numel;
    int32_t out_dtype;
    int32_t* status;
    uint32_t flags;
    cudaStream_t stream;
};

int32_t launch_paged(const PagedArgs& a);

// Gather rows x n pieces of piece_bytes (a multiple of 16) from a device-accessible source
// laid out [rows][src_blocks] pieces into dst [rows][n]: piece (t, i) is piece ids[i] of
// source row t.  An id outside [0, src_blocks) skips its piece and ORs SC_STATUS_BAD_PAGE_ID
// into *status.
int32_t launch_gather_pieces(const void* src, int64_t src_blocks, void* dst, const int32_t* ids,
                             int32_t n, int32_t rows, int64_t piece_bytes, int32_t* status,
                             cudaStream_t stream);

// Scatter rows x n pieces of piece_bytes (a multiple of 16) from src (row pitch src_pitch
// pieces) into a device-accessible destination: piece (t, i) goes to piece
// t * dst_pitch + ids[i].  The ids (host array, each in [0, bound)) are passed in the launch
// parameters, kMaxScatterIds per launch; an id outside [0, bound) skips its piece and ORs
// SC_STATUS_BAD_PAGE_ID into *status.
constexpr int32_t kMaxScatterIds = 960;
int32_t launch_scatter_pieces(const void* src, int64_t src_pitch, void* dst, int64_t dst_pitch,
                              int64_t bound, const int32_t* ids, int32_t n, int32_t rows,
                              int64_t piece_bytes, int32_t* status, cudaStream_t stream);

// Load the kernels the pipeline launches (paged restore; quantize with fp16 scales) on the
// current device now.  CUDA loads a kernel's module lazily at its first launch, and that
// load waits for the device to go idle, which would make a first restore or offload enqueued
// behind other work block the host.
cudaError_t preload_paged_kernels();
cudaError_t preload_quantize_kernels(bool f32_scales);  // fp16-scale kernels, + fp32 if asked
cudaError_t preload_dense_kernels();
cudaError_t preload_shift_kernels();

}  // namespace sc
