/*
 * speccache_b200.h — C ABI of the B200 (sm_100a) KV-restore library for SpecCache Path-1.
 *
 * Library: libspeccache_b200.so (built in-tree next to the Python package).
 *
 * Conventions shared by every entry point
 * ---------------------------------------
 *  - Plain pointers, sizes and element strides only; no framework types.
 *  - Device pointers are CUDA device (or managed) addresses on the current device.
 *    ``stream`` is a ``cudaStream_t`` passed as ``void*`` (NULL = legacy default stream).
 *  - Work is enqueued on ``stream`` and never synchronised by the library (the pipeline's
 *    explicit synchronise call excepted).
 *  - Every call returns an ``sc_status``; nothing throws across the ABI and nothing
 *    aborts the process.  ``sc_last_error()`` returns a per-thread message for the last
 *    failing call on that thread.
 *  - Stride arrays are host arrays, counted in elements.
 *  - Thread safety: calls on distinct streams may run concurrently from distinct host
 *    threads; one ``sc_pipeline`` object must be driven by one thread at a time.
 *
 * Arithmetic contract (parity with the reference's eager path)
 * ------------------------------------------------------------
 *  Keys:    x = fp16(q * s)  [rounded to fp16 first, speccache/kernels/reference.py:257]
 *           out[i]       = cvt(x[i]      * cos[i] - x[i+D/2] * sin[i])
 *           out[i + D/2] = cvt(x[i+D/2]  * cos[i] + x[i]     * sin[i])   (fp32 math)
 *           with SC_FLAG_FP32_INTERMEDIATE the fp16 rounding of x is skipped
 *           (the arithmetic of speccache/kernels/triton_rope_kv.py:150-158).
 *  Values:  out = cvt(q * s)                                        (reference.py:302)
 *  Tables:  cos/sin[i] = fp16(cos|sin(fp32(dp) * inv_freq[i])),
 *           inv_freq[i] = 1 / theta^(2i/D) in float32             (reference.py:151-164)
 *  Quantize: scale = fp16(max(amax / 127, eps)) with IEEE division,
 *            q = clamp(round_half_even(x / scale), -127, 127)       (reference.py:200-204)
 *  cvt is round-to-nearest-even into the output dtype (fp16, or bf16 as an extension).
 */
#ifndef SPECCACHE_B200_H
#define SPECCACHE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SC_ABI_VERSION 1

/* Every entry point is exported with default visibility; the library is built with
 * -fvisibility=hidden so that nothing else leaks out of it. */
#if defined(__GNUC__)
#define SC_API __attribute__((visibility("default")))
#else
#define SC_API
#endif

/* Status codes.  The Python layer maps them to the reference's exception types. */
typedef enum sc_status {
    SC_OK = 0,
    SC_ERR_INVALID_ARGUMENT = 1, /* shape / size / stride / alignment problem (ValueError) */
    SC_ERR_INVALID_DTYPE = 2,    /* unsupported dtype code (TypeError)                     */
    SC_ERR_CUDA = 3,             /* a CUDA runtime call failed (RuntimeError)              */
    SC_ERR_OUT_OF_RANGE = 4,     /* a device-side index check tripped (page id, length)    */
    SC_ERR_TIMEOUT = 5,          /* a bounded wait ran out                                 */
    SC_ERR_HOST_ALLOC = 6,       /* pinned host allocation failed                          */
    SC_ERR_UNSUPPORTED = 7       /* valid request the library does not implement           */
} sc_status;

/* Element type codes. */
typedef enum sc_dtype {
    SC_DTYPE_F16 = 0,
    SC_DTYPE_BF16 = 1,
    SC_DTYPE_F32 = 2
} sc_dtype;

/* Flags for the restore entry points. */
#define SC_FLAG_FP32_INTERMEDIATE 0x1u /* keep q*s in fp32 before the rotation            */
#define SC_FLAG_FORCE_GENERIC 0x2u     /* use the stride-generic kernel (testing aid)      */

/* Device status bits written (atomicOr) by the paged kernels into a caller-given word. */
#define SC_STATUS_BAD_PAGE_ID 0x1    /* page-table entry outside [0, n_pool_pages)          */
#define SC_STATUS_BAD_SEQ_LEN 0x2    /* seq_len < 0 or > max_pages * page_size              */
#define SC_STATUS_BAD_OUT_OFFSET 0x4 /* offset not a multiple of 16 or rows beyond out_numel */

/* Message for the last failing call on this host thread ("" if none). */
SC_API const char* sc_last_error(void);

/* SC_ABI_VERSION of the loaded library. */
SC_API int32_t sc_abi_version(void);

/* Load every kernel of the library on the current device now.  CUDA loads a kernel's module
 * lazily at its first launch, and that load waits for the device to go idle, so a first call
 * enqueued behind running work would block the calling thread until that work ends; call this
 * once per device at start-up to avoid it (sc_pipeline_create does it for its own kernels). */
SC_API int32_t sc_preload_kernels(void);

/*
 * cos/sin tables for relative RoPE shifts.
 * Replaces compute_rope_cos_sin_delta (speccache/kernels/reference.py:122-165).
 *
 *  delta_pos  device float32 [n] (the shifts, already converted to float32)
 *  inv_freq   host float32 [head_dim/2], or NULL to compute 1/theta^(2i/D) here
 *  cos_out, sin_out  device [n, head_dim/2] contiguous, dtype out_dtype (F16 | BF16 | F32)
 */
SC_API int32_t sc_rope_cos_sin_delta(const float* delta_pos, int64_t n, int32_t head_dim,
                              double theta_base, const float* inv_freq, void* cos_out,
                              void* sin_out, int32_t out_dtype, void* stream);

/*
 * Fused INT8 K dequant + relative RoPE shift and INT8 V dequant, one launch for both.
 * Replaces triton_fused_k_dequant_rope_shift (speccache/kernels/triton_rope_kv.py:243-345),
 * dequant_value (triton_rope_kv.py:352-411) and dequant_kv_cache (triton_rope_kv.py:414-427).
 *
 * Geometry: n_layers x n_tokens x n_heads rows of head_dim (head_dim even).
 *  k_quant / v_quant  int8, strides [layer, token, head, dim]; either may be NULL to skip it
 *  k_scale / v_scale  scale_dtype (F16 as in the reference, or F32), strides [layer, token, head]
 *  cos_delta/sin_delta  fp16 tables, strides [token, dim]; token stride 0 broadcasts one
 *                     row ([1, D/2]); a non-zero token stride gives one row per token
 *                     ([T, D/2]).  Pass NULL for both to use delta_p instead.
 *  delta_p            the shift when no table is given (converted to float32 like the
 *                     reference); if delta_p_dev (device float32 scalar) is non-NULL it
 *                     is read on the device instead.
 *  theta_base, inv_freq  as for sc_rope_cos_sin_delta (only used without tables)
 *  k_out / v_out      out_dtype (F16 | BF16), strides [layer, token, head, dim]
 */
SC_API int32_t sc_dequant_rope_kv(int32_t n_layers, int64_t n_tokens, int32_t n_heads,
                           int32_t head_dim, const int8_t* k_quant, const int64_t* kq_strides,
                           const void* k_scale, const int64_t* ks_strides,
                           const int8_t* v_quant, const int64_t* vq_strides,
                           const void* v_scale, const int64_t* vs_strides, int32_t scale_dtype,
                           const void* cos_delta, const void* sin_delta,
                           const int64_t* cs_strides, double delta_p, const float* delta_p_dev,
                           double theta_base, const float* inv_freq, void* k_out,
                           const int64_t* ko_strides, void* v_out, const int64_t* vo_strides,
                           int32_t out_dtype, uint32_t flags, void* stream);

/*
 * Per-token-shift restore that allocates no device memory.  No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc (an engine that has
 * reserved the device's memory for its own pools, or a request path that must not risk
 * the device synchronisation cudaMalloc/cudaFree can cause).
 *
 * Same work as building cos/sin tables for delta_p_tokens (device float32 [n_tokens],
 * one shift per token) with sc_rope_cos_sin_delta and passing them to sc_dequant_rope_kv,
 * but the two tables live in a fixed array inside the library (4 MiB per GPU that loads
 * it, held until exit) instead of caller-allocated buffers.  Limit: n_tokens * head_dim/2
 * <= 1,048,576 (e.g. 16384 tokens at head_dim 128); larger calls are rejected with
 * SC_ERR_INVALID_ARGUMENT.  Keys are required, values optional; other arguments as for
 * sc_dequant_rope_kv.  The first call on a device looks up the array's device address
 * (make it before any stream capture) and keeps it for the life of the process, so a
 * cudaDeviceReset after that first call is not supported.  Calls share the array: calls
 * that overlap on the GPU race.  Arguments are all checked before the array is written, so
 * a refused call leaves it untouched.
 */
SC_API int32_t sc_dequant_rope_kv_token_shifts_noalloc(
    int32_t n_layers, int64_t n_tokens, int32_t n_heads, int32_t head_dim, const int8_t* k_quant,
    const int64_t* kq_strides, const void* k_scale, const int64_t* ks_strides,
    const int8_t* v_quant, const int64_t* vq_strides, const void* v_scale,
    const int64_t* vs_strides, int32_t scale_dtype, const float* delta_p_tokens,
    double theta_base, const float* inv_freq, void* k_out, const int64_t* ko_strides,
    void* v_out, const int64_t* vo_strides, int32_t out_dtype, uint32_t flags, void* stream);

/*
 * Relative RoPE shift of already dequantised keys (float16 / bfloat16 in and out).
 * Replaces the rotation of MultiLayerKVInjector.apply_rope_shift
 * (speccache/serving/kv_injector.py:246-283), which inject_layer_kv applies before appending
 * keys to the cache (kv_injector.py:285-301).
 *
 *  x, out     [n_tokens, n_heads, head_dim] (head_dim even), dtypes x_dtype / out_dtype
 *             (F16 | BF16), element strides [token, head, dim]; out may be x itself (same
 *             strides) for an in-place shift, no other overlap
 *  cos_delta/sin_delta  fp16 tables, strides [token, dim]; token stride 0 broadcasts one row
 *             ([1, D/2]), a non-zero one gives one row per token ([T, D/2]); NULL for both to
 *             use delta_p (the table as sc_rope_cos_sin_delta computes it from theta_base,
 *             inv_freq)
 *  out = cvt(RN(x * cos) -/+ RN(x_partner * sin)): the reference's fp32 arithmetic, each
 *  product and the sum rounded once, bit-exact given the same tables.
 */
SC_API int32_t sc_rope_shift_keys(int64_t n_tokens, int32_t n_heads, int32_t head_dim,
                                  const void* x, int32_t x_dtype, const int64_t* x_strides,
                                  const void* cos_delta, const void* sin_delta,
                                  const int64_t* cs_strides, double delta_p, double theta_base,
                                  const float* inv_freq, void* out, int32_t out_dtype,
                                  const int64_t* out_strides, void* stream);

/*
 * Per-(token, head) absmax INT8 quantisation (the offload twin).
 * Replaces quantize_kv_int8 / quantize_symmetric_int8 (speccache/kernels/reference.py:179-209).
 *
 *  x        [n_tokens, n_heads, head_dim], dtype x_dtype (F16 | BF16 | F32), strides [t, h, d]
 *  q_out    int8, strides [t, h, d]
 *  scale_out  dtype scale_dtype (F16 as in the reference, or F32), strides [t, h]
 */
SC_API int32_t sc_quantize_int8(int64_t n_tokens, int32_t n_heads, int32_t head_dim, const void* x,
                         int32_t x_dtype, const int64_t* x_strides, float eps, int8_t* q_out,
                         const int64_t* q_strides, void* scale_out, int32_t scale_dtype,
                         const int64_t* s_strides, uint32_t flags, void* stream);

/*
 * Ragged, paged restore: gather each request's pages from a device page pool, dequantise,
 * shift keys by the request's (or page's) delta_p and write contiguous per-request caches.
 * Replaces the host gather of PinnedKVPool.get_coalesced_views
 * (speccache/cache/pinned_pool.py:392-464) followed by the per-chunk kernels of
 * SpecCacheEngine.execute_async_dma_and_rope (speccache/cache/engine.py:441-601).
 *
 *  pool_kq / pool_vq   int8  [n_pool_pages, page_size, n_heads, head_dim] contiguous
 *  pool_ks / pool_vs   fp16  [n_pool_pages, page_size, n_heads] contiguous
 *  page_table          device int32 [n_requests, page_table_stride] (first max_pages used)
 *  seq_lens            device int32 [n_requests]
 *  delta_p             device float32 [n_requests] or, with delta_p_per_page,
 *                      [n_requests, max_pages]
 *  out_offsets         device int64 [n_requests]: element offset of request r's token 0
 *                      (a multiple of 16 elements: rows are written 32 bytes at a time)
 *  out_strides         [token, head, dim] of the outputs (dim stride 1, others multiples
 *                      of 16 elements; outputs 32-byte aligned)
 *  out_numel           elements in each of k_out / v_out; a request whose rows would
 *                      fall outside is skipped and flagged (SC_STATUS_BAD_OUT_OFFSET)
 *  status              device int32 word; SC_STATUS_* bits are OR-ed in when an entry is
 *                      rejected (the offending page is skipped, nothing faults).  Required.
 */
SC_API int32_t sc_restore_paged(int32_t n_requests, int32_t max_pages, int32_t page_size,
                         int32_t n_heads, int32_t head_dim, int64_t n_pool_pages,
                         const int8_t* pool_kq, const void* pool_ks, const int8_t* pool_vq,
                         const void* pool_vs, const int32_t* page_table,
                         int64_t page_table_stride, const int32_t* seq_lens,
                         const float* delta_p, int32_t delta_p_per_page, double theta_base,
                         const float* inv_freq, void* k_out, void* v_out,
                         const int64_t* out_offsets, const int64_t* out_strides,
                         int64_t out_numel, int32_t out_dtype, int32_t* status, uint32_t flags,
                         void* stream);

/*
 * Multi-layer pinned-host -> GPU restore pipeline.
 * Replaces the pinned slabs of MultiLayerKVInjector (speccache/serving/kv_injector.py:171-215)
 * and its reconstruct_and_inject_multi_layer (kv_injector.py:392-498), and the
 * double-buffered DMA loop of SpecCacheEngine.execute_async_dma_and_rope
 * (speccache/cache/engine.py:441-601).
 *
 * Host slabs (pinned, owned by the pipeline), per layer l and block b:
 *    k_quant/v_quant  int8 [n_layers, n_blocks, chunk_size, n_heads, head_dim]
 *    k_scale/v_scale  fp16 [n_layers, n_blocks, chunk_size, n_heads]
 * The v_quant slab directly follows the k_quant slab in one allocation, and v_scale follows
 * k_scale; the scale slab is mapped pinned memory.  A restore stages the scales of every
 * layer on the pipeline's transfer stream: one 2-D copy for a run of consecutive block ids,
 * one gather kernel reading the mapped slab for a list in several runs.  It then cuts its
 * block list into stages of at most 64 MiB of K and V codes over all layers (the last stage
 * one block) and, per stage, copies the codes of every layer with one 3-D copy per run of
 * consecutive block ids within the stage into one of n_slots device staging slots, and runs
 * one restore kernel for the stage's blocks of every layer on compute_stream once its copy
 * event has fired, so stage s+1's copy overlaps stage s's kernel.  Every copy command costs a
 * few microseconds of copy-engine time beyond its bytes, so a block list in r runs costs
 * about r + stages commands.  A restore of fewer than 8 blocks that fits one stage is one
 * launch; from 8 blocks on the last block has a stage of its own.  With
 * SC_PIPE_PER_LAYER (or where a copy pitch exceeds the device's limit) it goes layer by
 * layer instead: per layer and run one 2-D copy of the K and V codes, one launch per layer.
 */
typedef struct sc_pipeline sc_pipeline;

#define SC_PIPE_NUMA_LOCAL 0x1u /* allocate the slabs from a thread bound to the GPU's NUMA node */
#define SC_PIPE_WRITE_COMBINED 0x2u /* pin the slabs write-combined: faster DMA reads on some
                                       hosts, very slow host reads (write-only use) */
#define SC_PIPE_PER_LAYER 0x4u /* always restore layer by layer (no block stages); for
                                  comparisons and tests */
#define SC_PIPE_SPLIT_KV_COPIES 0x8u /* block stages move a run's K and V codes as two 2-D copies
                                        (the form a slab beyond the device's copy pitch takes)
                                        instead of one 3-D copy; for comparisons and tests */

SC_API int32_t sc_pipeline_create(int32_t device, int32_t n_layers, int64_t n_blocks,
                           int32_t chunk_size, int32_t n_heads, int32_t head_dim,
                           int64_t max_restore_blocks, int32_t n_slots, uint32_t flags,
                           sc_pipeline** out);

/* Pinned host slab addresses (see layout above). */
SC_API int32_t sc_pipeline_host_slabs(const sc_pipeline* p, int8_t** k_quant, void** k_scale,
                               int8_t** v_quant, void** v_scale);

/*
 * Enqueue one restore of n_blocks blocks for every layer.
 *  block_ids, delta_ps  host int32 [n_blocks]; delta_ps[i] shifts block i's keys
 *  k_out, v_out         host arrays of n_layers device pointers; token i*chunk_size+c of
 *                       layer l goes to k_out[l] + (i*chunk_size + c)*st + h*sh + d
 *  out_strides          [token, head, dim] (dim stride 1)
 *  out_numel            elements of each k_out[l] / v_out[l] buffer (bounds check)
 * Returns once everything is enqueued; completion is ordered on compute_stream.  The host
 * waits only when four earlier restores still have their metadata upload queued (each upload
 * follows the previous restore's kernels).
 */
SC_API int32_t sc_pipeline_restore(sc_pipeline* p, const int32_t* block_ids, const int32_t* delta_ps,
                            int32_t n_blocks, double theta_base, const float* inv_freq,
                            void* const* k_out, void* const* v_out, const int64_t* out_strides,
                            int64_t out_numel, int32_t out_dtype, void* compute_stream);

/*
 * Enqueue the offload of n_blocks freshly computed K/V blocks of one layer into the slabs:
 * quantize on the GPU (sc_quantize_int8 arithmetic, bit-exact with the reference) into one of
 * two device staging slots on compute_stream, then move codes and scales to the pinned slabs
 * on the pipeline's transfer stream, so the next layer's quantize overlaps this layer's
 * transfer: for consecutive block ids one 2-D copy of the codes (K and V as its two rows) and
 * one of the scales; for a list in several runs one scatter kernel writing every block into
 * the mapped slabs (a copy command per run costs about 5 us; SM stores into pinned memory run
 * at the PCIe rate whatever the block order).  A list that names a block twice goes by copies
 * in list order, so the later chunk wins.  Replaces the cold-miss offload of the
 * reference runner: quantize_kv_int8 + .cpu() + PinnedKVPool.write_block
 * (speccache/serving/pipeline.py:506-524, speccache/cache/pinned_pool.py:275-367).
 *  k, v       device [n_blocks * chunk_size, n_heads, head_dim], dtype x_dtype (F16|BF16|F32),
 *             strides [token, head, dim]; block i's tokens go to slab block block_ids[i]
 *  block_ids  host int32 [n_blocks]
 * Offloads and restores share the transfer stream, so a restore enqueued after an offload
 * reads the offloaded blocks.  The host may read the slabs after sc_pipeline_synchronize.
 */
SC_API int32_t sc_pipeline_offload(sc_pipeline* p, int32_t layer, const int32_t* block_ids,
                                   int32_t n_blocks, const void* k, const int64_t* k_strides,
                                   const void* v, const int64_t* v_strides, int32_t x_dtype,
                                   void* compute_stream);

/* Wait (bounded by timeout_s, polling) for the last restore and offload; SC_ERR_TIMEOUT if
 * it ran out. */
SC_API int32_t sc_pipeline_synchronize(sc_pipeline* p, double timeout_s);

/* Make `stream` wait on the GPU (the host does not wait) until the restores and offloads
 * enqueued so far have completed, their copies included: work enqueued on `stream` afterwards
 * sees the restored caches and the offloaded slabs.  No counterpart in the reference (its
 * loops synchronise the device instead). */
SC_API int32_t sc_pipeline_join(sc_pipeline* p, void* stream);

/* Read and clear the device status word of the pipeline's kernels (synchronises). */
SC_API int32_t sc_pipeline_status(sc_pipeline* p, int32_t* status_bits);

/* How sc_pipeline_restore would run a restore of n_blocks blocks: the kernel launches it
 * issues (one per block stage: 1 for a restore of fewer than 8 blocks that fits one stage;
 * one per layer when the stages are off) into *launches.  No device work.  No counterpart in the reference (it
 * launches two kernels per chunk and layer). */
SC_API int32_t sc_pipeline_restore_launches(const sc_pipeline* p, int32_t n_blocks,
                                            int32_t* launches);

/* The work a restore (offload = 0) or an offload of one layer (offload = 1) of this block list
 * would enqueue: the kernel launches (restore: one per block stage, plus the scale gather of a
 * list in several runs; offload: the K and V quantize, plus the scatter kernels of a list in
 * several runs) into *launches and the copy commands (metadata upload included) into *copies.
 * No device work.  No counterpart in the reference. */
SC_API int32_t sc_pipeline_plan(const sc_pipeline* p, int32_t offload, const int32_t* block_ids,
                                int32_t n_blocks, int32_t* launches, int32_t* copies);

SC_API int32_t sc_pipeline_destroy(sc_pipeline* p);

/*
 * Sharing a device buffer between the processes of one machine (CUDA IPC), for the gather of
 * head shards onto one GPU: the owner exports the buffer, each other rank imports it and
 * passes the returned pointer (plus its shard's head offset) as the output of its restore,
 * so its kernel stores the shard into the owner's memory over NVLink.  No counterpart in
 * the reference (it has no multi-GPU path); this is the optional last row of the restore's
 * multi-GPU design.  Order the owner's reads after the writers' completion on the host
 * (writer stream synchronised, then a barrier).
 *
 *  sc_ipc_export: handle_out receives SC_IPC_HANDLE_BYTES bytes, offset_out the byte
 *                 offset of dev_ptr inside its allocation
 *  sc_ipc_import: maps the allocation on the current device with peer access enabled;
 *                 base_out is what sc_ipc_close takes, ptr_out = base + offset
 */
#define SC_IPC_HANDLE_BYTES 64
SC_API int32_t sc_ipc_export(const void* dev_ptr, void* handle_out, int64_t* offset_out);
SC_API int32_t sc_ipc_import(const void* handle, int64_t offset, void** base_out, void** ptr_out);
SC_API int32_t sc_ipc_close(void* base);

#ifdef __cplusplus
}
#endif

#endif /* SPECCACHE_B200_H */
