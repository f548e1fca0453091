// sc_noalloc.cu — per-token-shift restore that allocates no device memory.
//
// Who needs this: callers that cannot call cudaMalloc.  A serving engine that reserves
// (nearly) all device memory for its own pools at start-up has nothing left for a fresh
// cudaMalloc, and a request path that must not stall cannot afford cudaMalloc/cudaFree,
// which may synchronise the device.  The regular per-token path needs two scratch tables
// (cos and sin, one row per token) that the caller or the Python layer allocates; this
// entry point keeps them in a fixed array that lives in the library instead.
//
// The array is file-scope `static __device__`, so every GPU that loads the library holds
// it (4 MiB) until the process exits.  Host code cannot use the symbol as a device address:
// the first call on a device, with that device current, looks the address up with
// cudaGetSymbolAddress and caches it for that device.  Make that first call before any
// stream capture.  The cached address belongs to the device's primary context: after a
// cudaDeviceReset it would be stale, so resetting a device after its first call here is not
// supported.  All calls share the array and it keeps the last call's tables; the tables
// are rewritten in full for every token a call uses, so nothing needs clearing, but calls
// whose work overlaps on the GPU (different streams, or different host threads) race on it.
#include <mutex>

#include "sc_internal.h"

#include <cuda_fp16.h>

namespace {

// cos and sin tables, each up to kMaxEntries = n_tokens * head_dim / 2 fp16 values.
constexpr int64_t kMaxEntries = int64_t(1) << 20;
static __device__ __align__(256) __half g_token_tables[2 * kMaxEntries];

constexpr int kMaxDevices = 64;
void* g_table_addr[kMaxDevices] = {nullptr};
std::mutex g_table_mutex;

// Device address of the static tables on the current device (looked up once per device).
int32_t table_address(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return sc::cuda_error(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices)
        return sc::set_error(SC_ERR_UNSUPPORTED, "device ordinal %d above %d", dev, kMaxDevices - 1);
    std::lock_guard<std::mutex> lock(g_table_mutex);
    if (g_table_addr[dev] == nullptr) {
        void* ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_token_tables);
        if (e != cudaSuccess) return sc::cuda_error(e, "cudaGetSymbolAddress(token tables)");
        g_table_addr[dev] = ptr;
    }
    *out = g_table_addr[dev];
    return SC_OK;
}

}  // namespace

extern "C" int32_t sc_dequant_rope_kv_token_shifts_noalloc(
    int32_t n_layers, int64_t n_tokens, int32_t n_heads, int32_t head_dim, const int8_t* k_quant,
    const int64_t* kq_strides, const void* k_scale, const int64_t* ks_strides,
    const int8_t* v_quant, const int64_t* vq_strides, const void* v_scale,
    const int64_t* vs_strides, int32_t scale_dtype, const float* delta_p_tokens,
    double theta_base, const float* inv_freq, void* k_out, const int64_t* ko_strides,
    void* v_out, const int64_t* vo_strides, int32_t out_dtype, uint32_t flags, void* stream) {
    // Every argument is checked before the shared tables are touched, so a call that is
    // refused never overwrites tables that a call still running on the GPU is reading.
    if (n_layers < 0 || n_tokens < 0 || n_heads < 0)
        return sc::set_error(SC_ERR_INVALID_ARGUMENT, "negative size (layers=%d tokens=%lld heads=%d)",
                             n_layers, (long long)n_tokens, n_heads);
    if (head_dim <= 0 || (head_dim & 1))
        return sc::set_error(SC_ERR_INVALID_ARGUMENT,
                             "head_dim must be even for RoPE half-pairing, got head_dim=%d", head_dim);
    if (head_dim > sc::kMaxHeadDim)
        return sc::set_error(SC_ERR_UNSUPPORTED, "head_dim %d exceeds %d", head_dim, sc::kMaxHeadDim);
    if (out_dtype != SC_DTYPE_F16 && out_dtype != SC_DTYPE_BF16)
        return sc::set_error(SC_ERR_INVALID_DTYPE, "output dtype code %d: float16 or bfloat16 only",
                             out_dtype);
    if (scale_dtype != SC_DTYPE_F16 && scale_dtype != SC_DTYPE_F32)
        return sc::set_error(SC_ERR_INVALID_DTYPE, "scale dtype code %d: float16 or float32 only",
                             scale_dtype);
    // An entry count is at least n_tokens (head_dim >= 2), so this bound comes first and the
    // product below cannot overflow.
    const int64_t entries = n_tokens > kMaxEntries ? kMaxEntries + 1 : n_tokens * (head_dim / 2);
    if (entries > kMaxEntries)
        return sc::set_error(SC_ERR_INVALID_ARGUMENT,
                             "n_tokens * head_dim / 2 = %lld exceeds the fixed table capacity of "
                             "%lld entries (e.g. 16384 tokens at head_dim 128); split the call "
                             "along the tokens",
                             (long long)entries, (long long)kMaxEntries);
    if (k_quant == nullptr)
        return sc::set_error(SC_ERR_INVALID_ARGUMENT, "keys are required (the shift applies to K)");
    if (delta_p_tokens == nullptr)
        return sc::set_error(SC_ERR_INVALID_ARGUMENT, "null delta_p_tokens");
    if (!k_scale || !k_out || !kq_strides || !ks_strides || !ko_strides)
        return sc::set_error(SC_ERR_INVALID_ARGUMENT, "K given without its scale/output/strides");
    if (v_quant && (!v_scale || !v_out || !vq_strides || !vs_strides || !vo_strides))
        return sc::set_error(SC_ERR_INVALID_ARGUMENT, "V given without its scale/output/strides");
    if (sc::size_product(n_layers, n_tokens, n_heads) >= (int64_t(1) << 31))
        return sc::set_error(SC_ERR_INVALID_ARGUMENT, "too many rows in one call; split it below 2^31");
    if (n_layers == 0 || n_tokens == 0 || n_heads == 0) return sc::ok();
    void* tables = nullptr;
    const int32_t rc = table_address(&tables);
    if (rc != SC_OK) return rc;
    __half* cos_tab = static_cast<__half*>(tables);
    __half* sin_tab = cos_tab + kMaxEntries;
    int32_t r = sc_rope_cos_sin_delta(delta_p_tokens, n_tokens, head_dim, theta_base, inv_freq,
                                      cos_tab, sin_tab, SC_DTYPE_F16, stream);
    if (r != SC_OK) return r;
    const int64_t cs_strides[2] = {head_dim / 2, 1};
    return sc_dequant_rope_kv(n_layers, n_tokens, n_heads, head_dim, k_quant, kq_strides, k_scale,
                              ks_strides, v_quant, vq_strides, v_scale, vs_strides, scale_dtype,
                              cos_tab, sin_tab, cs_strides, 0.0, nullptr, theta_base, nullptr,
                              k_out, ko_strides, v_out, vo_strides, out_dtype, flags, stream);
}
