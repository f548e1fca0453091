// sc_pipeline.cpp — multi-layer pinned-host -> GPU KV restore pipeline.
//
// Host side of the restore path (the reference drives the same steps from Python:
// speccache/serving/kv_injector.py:392-498 and speccache/cache/engine.py:441-601):
//   * pinned slabs [L, B, chunk, H, D] int8 and [L, B, chunk, H] fp16 (cudaHostAlloc,
//     optionally from a thread bound to the GPU's NUMA node);
//   * K and V code slabs are one pinned allocation (V right after K), and so are the scale
//     slabs (mapped, so kernels can read them); a restore first stages every layer's scales
//     of its blocks on the pipeline's own transfer stream: one 2-D copy (2 x n_layers rows)
//     for a list of consecutive block ids, one gather kernel reading the mapped slab for a
//     list in several runs;
//   * every copy command costs about 4 us of copy-engine time beyond its bytes, whatever
//     its size or shape (the rows of a 2-D or 3-D copy cost nothing extra), and spreading
//     commands over several streams does not overlap that cost (measured on B200: 8192
//     copies of 64 KiB take 43 ms against 9.7 ms for the same bytes in one 2-D copy).  So the
//     codes move in as few commands as the block list allows;
//   * block stages (the default where the copy pitches allow): the restore's block list is
//     cut into stages of at most 64 MiB of K and V codes over all layers; a stage's codes go
//     with one 3-D copy per run of consecutive block ids (rows: every layer at the slab's
//     layer pitch; slices: K then V) into one of a ring of device slots, and one paged-kernel
//     launch restores the stage, the layers being its requests.  A restore of n blocks in r
//     runs costs about r + stages copy commands, so a scattered block list costs one copy
//     per run rather than one per run and layer.  The last stage is one block, so that only
//     its kernel remains after the last copy; a restore of fewer than 8 blocks that fits one
//     stage is one copy per run and one launch;
//   * an event per slot joins the transfer stream to the caller's compute stream; a second
//     event per slot releases the slot for stage s + n_slots;
//   * layer by layer (SC_PIPE_PER_LAYER, or where a pitch exceeds the device's limit): per
//     layer, K and V codes of each run with one 2-D copy of two rows into a slot, one
//     paged-kernel launch per layer.
// The offload runs the other way: the quantize kernel writes a device staging buffer on
// the compute stream, an event hands it to the transfer stream, and D2H copies (consecutive
// block ids) or one scatter kernel writing the mapped slabs (a list in several runs) fill the
// slabs.
// Nothing on the host waits during a restore or an offload while fewer than four earlier
// restores still have their metadata upload queued (each upload follows the previous
// restore's kernels; the host metadata buffers form a ring of four); sc_pipeline_synchronize
// polls events with a deadline.
#include <errno.h>
#include <sched.h>
#include <sys/prctl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <vector>

#include "sc_internal.h"

namespace {

struct Meta {  // one upload per restore: identity-table length and per-block shifts
    int32_t seq_len;
    int32_t pad;
    int64_t out_offset;
    float delta_p[1];  // [max_restore_blocks]
};

// K and V codes of one block stage (all layers) in a slot.  A small restore is one copy per
// run and one kernel launch (per-layer launches and events cost about 8 us of host time per
// layer, more than the copies of a restore of a few blocks take).
constexpr size_t kStageBytes = size_t(64) << 20;
// Block stages are off where one block's codes over all layers exceed this (a slot holds at
// least one block).
constexpr size_t kMaxStageBytes = size_t(256) << 20;

// Restores of fewer blocks than this that fit one stage stay one stage; from this many on,
// the last block gets its own stage.
constexpr int64_t kSplitLastMin = 8;

// Blocks per stage of an n-block restore with at most `cap` blocks per stage.  The last stage
// is one block: its kernel is the only one left after the last copy, while every other
// stage's kernel runs under the next stage's copy (tens of times longer).  The n - 1 blocks
// before it go in as few stages of at most cap blocks as possible, of nearly equal size.  A
// restore of fewer than kSplitLastMin blocks that fits one stage is one stage: there the
// extra copy command and launch cost about what the shorter tail saves.
void stage_sizes(int64_t n, int64_t cap, std::vector<int32_t>& out) {
    out.clear();
    if (n <= 0) return;
    if (n <= cap && (n < kSplitLastMin || cap < 2)) {
        out.push_back(static_cast<int32_t>(n));
        return;
    }
    const int64_t front = n - 1;
    const int64_t n_front = (front + cap - 1) / cap;
    for (int64_t i = 0; i < n_front; ++i)
        out.push_back(static_cast<int32_t>(front / n_front + (i < front % n_front ? 1 : 0)));
    out.push_back(1);
}

// Whether a block list names a block twice.  An offload of such a list goes by copies, in
// list order, so the last of the duplicates wins as with the reference's block-by-block
// writes (pinned_pool.py:275-367); the scatter kernel would write them at once.
bool has_duplicates(const int32_t* ids, int32_t n) {
    std::vector<int32_t> v(ids, ids + n);
    std::sort(v.begin(), v.end());
    return std::adjacent_find(v.begin(), v.end()) != v.end();
}

size_t meta_bytes(int64_t max_blocks) {
    return sizeof(Meta) + sizeof(float) * static_cast<size_t>(max_blocks > 1 ? max_blocks - 1 : 0);
}

// Host metadata buffers per path: a restore fills the next one while the uploads of up to
// kMetaRing - 1 earlier restores may still be queued behind their predecessors' kernels, so
// the host waits only when kMetaRing restores are in flight.
constexpr int kMetaRing = 4;

size_t round_up64(size_t n) { return (n + 63) / 64 * 64; }

// Bind the calling thread to the CPUs local to `device` (best effort); returns true and
// the previous mask in `old` if the binding was changed.
bool bind_to_device_numa(int device, cpu_set_t* old) {
    char bus[32] = {0};
    if (cudaDeviceGetPCIBusId(bus, sizeof(bus), device) != cudaSuccess) return false;
    for (char* c = bus; *c; ++c)
        if (*c >= 'A' && *c <= 'F') *c = static_cast<char>(*c - 'A' + 'a');
    char path[160];
    snprintf(path, sizeof(path), "/sys/bus/pci/devices/%s/local_cpulist", bus);
    FILE* f = fopen(path, "r");
    if (!f) {
        // sysfs uses a 4-digit domain; the runtime may print 8 digits.
        if (strlen(bus) > 12) {
            snprintf(path, sizeof(path), "/sys/bus/pci/devices/%s/local_cpulist", bus + 4);
            f = fopen(path, "r");
        }
        if (!f) return false;
    }
    char list[1024] = {0};
    const bool got = fgets(list, sizeof(list), f) != nullptr;
    fclose(f);
    if (!got) return false;
    cpu_set_t set;
    CPU_ZERO(&set);
    int count = 0;
    char* save = nullptr;  // strtok_r: pipelines may be created from several threads at once
    for (char* tok = strtok_r(list, ",\n", &save); tok; tok = strtok_r(nullptr, ",\n", &save)) {
        int a = 0, b = 0;
        if (sscanf(tok, "%d-%d", &a, &b) == 2) {
            for (int c = a; c <= b && c < CPU_SETSIZE; ++c) CPU_SET(c, &set), ++count;
        } else if (sscanf(tok, "%d", &a) == 1 && a < CPU_SETSIZE) {
            CPU_SET(a, &set), ++count;
        }
    }
    if (count == 0) return false;
    if (sched_getaffinity(0, sizeof(cpu_set_t), old) != 0) return false;
    return sched_setaffinity(0, sizeof(cpu_set_t), &set) == 0;
}

double now_s() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

}  // namespace

struct sc_pipeline {
    int device = 0;
    int32_t L = 0, chunk = 0, H = 0, D = 0, n_slots = 0;
    int64_t B = 0, max_blocks = 0;
    uint32_t flags = 0;
    int8_t* h_kq = nullptr;
    uint16_t* h_ks = nullptr;
    int8_t* h_vq = nullptr;
    uint16_t* h_vs = nullptr;
    uint8_t* h_meta = nullptr;  // kMetaRing buffers of meta_stride bytes
    size_t meta_stride = 0;
    // per slot: block stages use d_kq[s] alone ([2][L][m][block]); layer by layer, d_vq[s] =
    // d_kq[s] + stage codes in the same allocation
    std::vector<int8_t*> d_kq, d_vq;
    uint16_t* d_sc = nullptr;         // scales of every layer: [2][L][max_blocks * chunk * H]
    bool codes_2d = false, scales_2d = false;  // pitches within the device's copy limit
    int32_t* d_table = nullptr;
    Meta* d_meta = nullptr;
    int32_t* d_status = nullptr;
    cudaStream_t transfer = nullptr;
    std::vector<cudaEvent_t> ready, slot_free;
    std::vector<bool> slot_used;
    cudaEvent_t meta_uploaded[kMetaRing] = {}, done = nullptr;
    bool meta_used[kMetaRing] = {};
    int meta_next = 0;
    bool any_restore = false;
    // block stages: at most stage_cap blocks per stage (0 = mode unavailable); stage_3d: K and
    // V codes of a run in one 3-D copy (else one 2-D copy each)
    int64_t stage_cap = 0;
    bool stage_3d = false;
    std::vector<int32_t> stages;  // the current restore's stage sizes
    // The slabs as the device addresses them (mapped pinned memory): the scale gather of
    // restores and the scatter of offloads in more than one run read and write through them;
    // null where a slab is not mapped (or, for the scales, where one block's scales of a layer
    // are not a multiple of 16 bytes).
    int8_t* d_hkq = nullptr;
    uint16_t* d_hks = nullptr;
    // kMetaRing host buffers, each seq[max stages] | dps[max_blocks] | ids[max_blocks] |
    // k_out[L] | v_out[L]
    uint8_t* h_stage_meta = nullptr;
    uint8_t* d_stage_meta = nullptr;
    size_t stage_meta_bytes = 0, stage_meta_stride = 0, off_dps = 0, off_ids = 0, off_kp = 0,
           off_vp = 0;
    cudaEvent_t stage_meta_uploaded[kMetaRing] = {};
    bool stage_meta_used[kMetaRing] = {};
    int stage_meta_next = 0;
    // offload: quantize into one of two device staging slots (K then V codes in one
    // allocation, K then V scales in another), then D2H into the slabs
    int8_t* o_codes[2] = {nullptr, nullptr};
    uint16_t* o_scales[2] = {nullptr, nullptr};
    cudaEvent_t o_ready[2] = {nullptr, nullptr}, o_free[2] = {nullptr, nullptr};
    bool o_used[2] = {false, false};
    int o_next = 0, o_last = 0;
    bool offload_scales_2d = false;
    bool any_offload = false;
};

namespace {

void release(sc_pipeline* p) {
    if (!p) return;
    DeviceGuard g(p->device);
    if (p->transfer) cudaStreamSynchronize(p->transfer);
    if (p->done && p->any_restore) cudaEventSynchronize(p->done);
    for (auto e : p->ready) cudaEventDestroy(e);
    for (auto e : p->slot_free) cudaEventDestroy(e);
    if (p->any_offload && p->o_free[p->o_last]) cudaEventSynchronize(p->o_free[p->o_last]);
    for (int i = 0; i < kMetaRing; ++i) {
        if (p->meta_uploaded[i]) cudaEventDestroy(p->meta_uploaded[i]);
        if (p->stage_meta_uploaded[i]) cudaEventDestroy(p->stage_meta_uploaded[i]);
    }
    cudaFree(p->d_stage_meta);
    cudaFreeHost(p->h_stage_meta);
    if (p->done) cudaEventDestroy(p->done);
    for (int s = 0; s < 2; ++s) {
        if (p->o_ready[s]) cudaEventDestroy(p->o_ready[s]);
        if (p->o_free[s]) cudaEventDestroy(p->o_free[s]);
        cudaFree(p->o_codes[s]);
        cudaFree(p->o_scales[s]);
    }
    if (p->transfer) cudaStreamDestroy(p->transfer);
    for (auto x : p->d_kq) cudaFree(x);  // d_vq[s], where set, lies in the same allocation
    cudaFree(p->d_sc);
    cudaFree(p->d_table);
    cudaFree(p->d_meta);
    cudaFree(p->d_status);
    cudaFreeHost(p->h_kq);  // h_vq lies in the same allocation
    cudaFreeHost(p->h_ks);  // and h_vs in this one
    cudaFreeHost(p->h_meta);
    delete p;
}

}  // namespace

using sc::cuda_error;
using sc::set_error;

extern "C" int32_t sc_pipeline_create(int32_t device, int32_t n_layers, int64_t n_blocks,
                                      int32_t chunk_size, int32_t n_heads, int32_t head_dim,
                                      int64_t max_restore_blocks, int32_t n_slots,
                                      uint32_t flags, sc_pipeline** out) {
    if (!out) return set_error(SC_ERR_INVALID_ARGUMENT, "null output handle");
    *out = nullptr;
    if (n_layers <= 0 || n_blocks <= 0 || chunk_size <= 0 || n_heads <= 0 || n_slots <= 0 ||
        max_restore_blocks <= 0 || max_restore_blocks > n_blocks)
        return set_error(SC_ERR_INVALID_ARGUMENT,
                         "invalid pipeline geometry (layers=%d blocks=%lld chunk=%d heads=%d "
                         "slots=%d max_restore=%lld)",
                         n_layers, (long long)n_blocks, chunk_size, n_heads, n_slots,
                         (long long)max_restore_blocks);
    if (head_dim <= 0 || head_dim % 32 != 0 || head_dim > sc::kMaxHeadDim)
        return set_error(SC_ERR_UNSUPPORTED, "head_dim must be a multiple of 32 up to %d",
                         sc::kMaxHeadDim);
    if (max_restore_blocks >= (int64_t(1) << 31) / chunk_size)
        return set_error(SC_ERR_INVALID_ARGUMENT, "max_restore_blocks too large");
    // Block ids are int32, and the slabs' codes must stay well inside size_t: sizes off by
    // orders of magnitude fail here instead of wrapping into a small allocation.
    if (n_blocks >= (int64_t(1) << 31) || n_slots > 64 ||
        sc::size_product(sc::size_product(n_layers, n_blocks, chunk_size), n_heads, head_dim) >=
            (int64_t(1) << 44))
        return set_error(SC_ERR_INVALID_ARGUMENT,
                         "pipeline too large (layers=%d blocks=%lld chunk=%d heads=%d "
                         "head_dim=%d slots=%d)",
                         n_layers, (long long)n_blocks, chunk_size, n_heads, head_dim, n_slots);
    auto* p = new sc_pipeline();
    p->device = device;
    p->L = n_layers;
    p->B = n_blocks;
    p->chunk = chunk_size;
    p->H = n_heads;
    p->D = head_dim;
    p->max_blocks = max_restore_blocks;
    p->n_slots = n_slots;
    p->flags = flags;
    DeviceGuard g(device);
    if (!g.ok) {
        delete p;
        return set_error(SC_ERR_CUDA, "cudaSetDevice(%d) failed", device);
    }
    const size_t row = static_cast<size_t>(chunk_size) * n_heads;
    const size_t slab_codes = static_cast<size_t>(n_layers) * n_blocks * row * head_dim;
    const size_t slab_scales = static_cast<size_t>(n_layers) * n_blocks * row;
    cpu_set_t old;
    const bool bound = (flags & SC_PIPE_NUMA_LOCAL) && bind_to_device_numa(device, &old);
    cudaError_t e = cudaSuccess;
    void* ptr = nullptr;
    const unsigned slab_flags = cudaHostAllocPortable |
                                ((flags & SC_PIPE_WRITE_COMBINED) ? cudaHostAllocWriteCombined : 0u);
    // Host-side fault injection for tests: with SC_FAILPOINT_HOST_ALLOC=k set, the k-th pinned
    // allocation of this call reports failure (the error and clean-up paths run as for a real
    // cudaHostAlloc failure).
    const char* fp = getenv("SC_FAILPOINT_HOST_ALLOC");
    const int fail_at = fp ? atoi(fp) : 0;
    int n_alloc = 0;
    auto halloc = [&](size_t bytes, void** dst, unsigned hflags) {
        *dst = nullptr;  // a failed allocation must not leave the previous address behind
        if (e != cudaSuccess) return;
        if (++n_alloc == fail_at) {
            e = cudaErrorMemoryAllocation;
            return;
        }
        e = cudaHostAlloc(dst, bytes, hflags);
        if (e == cudaSuccess) memset(*dst, 0, bytes);  // first touch on the bound thread
    };
    halloc(2 * slab_codes, &ptr, slab_flags | cudaHostAllocMapped), p->h_kq = static_cast<int8_t*>(ptr);
    if (e == cudaSuccess) p->h_vq = p->h_kq + slab_codes;
    halloc(2 * slab_scales * 2, &ptr, slab_flags | cudaHostAllocMapped),
        p->h_ks = static_cast<uint16_t*>(ptr);
    if (e == cudaSuccess) p->h_vs = p->h_ks + slab_scales;
    p->meta_stride = round_up64(meta_bytes(max_restore_blocks));
    halloc(kMetaRing * p->meta_stride, &ptr, cudaHostAllocPortable), p->h_meta = static_cast<uint8_t*>(ptr);
    if (bound) sched_setaffinity(0, sizeof(cpu_set_t), &old);
    if (e != cudaSuccess) {
        const int32_t rc = set_error(SC_ERR_HOST_ALLOC, "cudaHostAlloc of %zu-byte slabs failed: %s",
                                     slab_codes, cudaGetErrorString(e));
        cudaGetLastError();
        release(p);
        return rc;
    }
    const size_t stage_codes = static_cast<size_t>(max_restore_blocks) * row * head_dim;
    const size_t stage_scales = static_cast<size_t>(max_restore_blocks) * row;
    int max_pitch = 0;
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&max_pitch, cudaDevAttrMaxPitch, device);
    const size_t mp = static_cast<size_t>(max_pitch);
    const size_t blk_codes = row * head_dim;
    {
        // Block stages need the copies' pitches within the device's limit: the slab's layer
        // pitch and the slot's row (one layer of a stage) for the codes, the slabs' and the
        // staging's rows for the scales.
        const size_t per_block = 2 * static_cast<size_t>(n_layers) * blk_codes;
        int64_t cap = static_cast<int64_t>(kStageBytes / per_block);
        if (cap < 1) cap = 1;
        if (cap > max_restore_blocks) cap = max_restore_blocks;
        const bool pitches = static_cast<size_t>(n_blocks) * blk_codes <= mp &&
                             static_cast<size_t>(cap) * blk_codes <= mp &&
                             static_cast<size_t>(n_blocks) * row * 2 <= mp && stage_scales * 2 <= mp;
        if (!(flags & SC_PIPE_PER_LAYER) && pitches && per_block <= kMaxStageBytes)
            p->stage_cap = cap;
        // One 3-D copy per run moves K and V (slices at the K -> V slab distance) where that
        // distance is within the limit too; otherwise one 2-D copy each.
        p->stage_3d = slab_codes <= mp && !(flags & SC_PIPE_SPLIT_KV_COPIES);
    }
    const size_t slot_bytes = p->stage_cap > 0
                                  ? static_cast<size_t>(p->stage_cap) * 2 * n_layers * blk_codes
                                  : 2 * stage_codes;
    for (int s = 0; s < n_slots && e == cudaSuccess; ++s) {
        int8_t* kv = nullptr;
        e = cudaMalloc(&kv, slot_bytes);
        p->d_kq.push_back(kv);
        p->d_vq.push_back(kv && p->stage_cap == 0 ? kv + stage_codes : nullptr);
    }
    if (e == cudaSuccess)
        e = cudaMalloc(&p->d_sc, 2 * static_cast<size_t>(n_layers) * stage_scales * 2);
    if (e == cudaSuccess) {
        p->codes_2d = slab_codes <= mp && stage_codes <= mp;
        p->scales_2d = static_cast<size_t>(n_blocks) * row * 2 <= mp && stage_scales * 2 <= mp;
        p->offload_scales_2d = slab_scales * 2 <= mp && stage_scales * 2 <= mp;
    }
    if (e == cudaSuccess && p->stage_cap > 0) {
        // The stage count grows with the block count, so the largest restore has the most.
        stage_sizes(max_restore_blocks, p->stage_cap, p->stages);
        const size_t max_stages = p->stages.size();
        p->off_dps = (max_stages * 4 + 7) / 8 * 8;
        p->off_ids = p->off_dps + (static_cast<size_t>(max_restore_blocks) * 4 + 7) / 8 * 8;
        p->off_kp = p->off_ids + (static_cast<size_t>(max_restore_blocks) * 4 + 7) / 8 * 8;
        p->off_vp = p->off_kp + static_cast<size_t>(n_layers) * 8;
        p->stage_meta_bytes = p->off_vp + static_cast<size_t>(n_layers) * 8;
        p->stage_meta_stride = round_up64(p->stage_meta_bytes);
        e = cudaMalloc(&p->d_stage_meta, p->stage_meta_bytes);
        if (e == cudaSuccess)
            e = cudaHostAlloc(&p->h_stage_meta, kMetaRing * p->stage_meta_stride,
                              cudaHostAllocPortable);
        for (int i = 0; i < kMetaRing && e == cudaSuccess; ++i)
            e = cudaEventCreateWithFlags(&p->stage_meta_uploaded[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) {
        // The piece kernels move 16-byte units: one block's codes of a layer always are a
        // multiple of 16 bytes (head_dim is a multiple of 32); its scales (chunk x heads fp16)
        // must be too.  A slab that is not mapped goes by copies.
        void* mapped = nullptr;
        if (cudaHostGetDevicePointer(&mapped, p->h_kq, 0) == cudaSuccess)
            p->d_hkq = static_cast<int8_t*>(mapped);
        else
            cudaGetLastError();
        if ((row * 2) % 16 == 0 && cudaHostGetDevicePointer(&mapped, p->h_ks, 0) == cudaSuccess)
            p->d_hks = static_cast<uint16_t*>(mapped);
        else
            cudaGetLastError();
    }
    // Identity page table: a stage's pool holds n_layers x (at most stage_cap) pages.
    int64_t table_len = max_restore_blocks;
    if (static_cast<int64_t>(n_layers) * p->stage_cap > table_len)
        table_len = static_cast<int64_t>(n_layers) * p->stage_cap;
    if (e == cudaSuccess) e = cudaMalloc(&p->d_table, sizeof(int32_t) * table_len);
    if (e == cudaSuccess) e = cudaMalloc(&p->d_meta, meta_bytes(max_restore_blocks));
    if (e == cudaSuccess) e = cudaMalloc(&p->d_status, sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMemset(p->d_status, 0, sizeof(int32_t));
    if (e == cudaSuccess) {
        std::vector<int32_t> ident(static_cast<size_t>(table_len));
        for (int64_t i = 0; i < table_len; ++i) ident[i] = static_cast<int32_t>(i);
        e = cudaMemcpy(p->d_table, ident.data(), sizeof(int32_t) * ident.size(),
                       cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = sc::preload_paged_kernels();
    if (e == cudaSuccess) e = sc::preload_quantize_kernels(false);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->transfer, cudaStreamNonBlocking);
    for (int s = 0; s < n_slots && e == cudaSuccess; ++s) {
        cudaEvent_t a = nullptr, b = nullptr;
        e = cudaEventCreateWithFlags(&a, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&b, cudaEventDisableTiming);
        p->ready.push_back(a), p->slot_free.push_back(b), p->slot_used.push_back(false);
    }
    for (int i = 0; i < kMetaRing && e == cudaSuccess; ++i)
        e = cudaEventCreateWithFlags(&p->meta_uploaded[i], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->done, cudaEventDisableTiming);
    for (int s = 0; s < 2 && e == cudaSuccess; ++s) {
        e = cudaEventCreateWithFlags(&p->o_ready[s], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->o_free[s], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaMalloc(&p->o_codes[s], 2 * stage_codes);
        if (e == cudaSuccess) e = cudaMalloc(&p->o_scales[s], 2 * stage_scales * 2);
    }
    if (e != cudaSuccess) {
        const int32_t rc = cuda_error(e, "pipeline device set-up");
        release(p);
        return rc;
    }
    *out = p;
    return sc::ok();
}

extern "C" int32_t sc_pipeline_host_slabs(const sc_pipeline* p, int8_t** k_quant, void** k_scale,
                                          int8_t** v_quant, void** v_scale) {
    if (!p) return set_error(SC_ERR_INVALID_ARGUMENT, "null pipeline");
    if (k_quant) *k_quant = p->h_kq;
    if (k_scale) *k_scale = p->h_ks;
    if (v_quant) *v_quant = p->h_vq;
    if (v_scale) *v_scale = p->h_vs;
    return sc::ok();
}

namespace {

// Block stages: stage s holds the blocks at positions [i0, i0 + m) of the restore for every
// layer; the layers are the requests of one paged restore (request l writes layer l from
// token i0 * chunk).  The stage's K and V codes are staged [2][L][m][block] in a slot by one
// 3-D copy per run of consecutive block ids within the stage (rows: layers at the slab's
// layer pitch; slices: K then V), every layer's scales [2][L][n][chunk * H] up front (one
// 2-D copy for a single run, else one gather kernel over the mapped slab); the kernel reaches
// a stage's scales through a per-request skew of (n - m) pages.  The transfer stream fills slot s % n_slots while the compute stream
// restores the stages in the other slots.
int32_t restore_block_stages(sc_pipeline* p, const int32_t* block_ids, const int32_t* delta_ps,
                             int32_t n, double theta_base, const float* inv_freq,
                             void* const* k_out, void* const* v_out, const int64_t* out_strides,
                             int64_t out_numel, int32_t out_dtype, cudaStream_t cs) {
    const int L = p->L;
    for (int l = 0; l < L; ++l)
        if (((reinterpret_cast<uintptr_t>(k_out[l]) | reinterpret_cast<uintptr_t>(v_out[l])) & 31) != 0)
            return set_error(SC_ERR_INVALID_ARGUMENT, "outputs must be 32-byte aligned (layer %d)", l);
    const size_t row = static_cast<size_t>(p->chunk) * p->H;
    const size_t blk_codes = row * p->D, blk_scales = row;
    stage_sizes(n, p->stage_cap, p->stages);
    const size_t n_stages = p->stages.size();
    cudaError_t e = cudaSuccess;
    // The next host metadata buffer may still feed an upload kMetaRing restores back.
    const int ms = p->stage_meta_next;
    if (p->stage_meta_used[ms]) e = cudaEventSynchronize(p->stage_meta_uploaded[ms]);
    if (e != cudaSuccess) return cuda_error(e, "waiting for an earlier metadata upload");
    uint8_t* hm = p->h_stage_meta + static_cast<size_t>(ms) * p->stage_meta_stride;
    int32_t* seq = reinterpret_cast<int32_t*>(hm);
    float* dps = reinterpret_cast<float*>(hm + p->off_dps);
    int32_t* ids = reinterpret_cast<int32_t*>(hm + p->off_ids);
    uint64_t* kp = reinterpret_cast<uint64_t*>(hm + p->off_kp);
    uint64_t* vp = reinterpret_cast<uint64_t*>(hm + p->off_vp);
    for (size_t s = 0; s < n_stages; ++s) seq[s] = p->stages[s] * p->chunk;
    int32_t runs = n > 0 ? 1 : 0;
    for (int32_t i = 0; i < n; ++i) {
        dps[i] = static_cast<float>(delta_ps[i]);
        ids[i] = block_ids[i];
        if (i > 0 && block_ids[i] != block_ids[i - 1] + 1) ++runs;
    }
    for (int l = 0; l < L; ++l) {
        kp[l] = reinterpret_cast<uint64_t>(k_out[l]);
        vp[l] = reinterpret_cast<uint64_t>(v_out[l]);
    }
    // The slots, the scales and the metadata on the device may still be read by the previous
    // restore's kernels.
    if (p->any_restore) e = cudaStreamWaitEvent(p->transfer, p->done, 0);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(p->d_stage_meta, hm, p->stage_meta_bytes, cudaMemcpyHostToDevice,
                            p->transfer);
    if (e == cudaSuccess) e = cudaEventRecord(p->stage_meta_uploaded[ms], p->transfer);
    if (e != cudaSuccess) return cuda_error(e, "metadata upload");
    p->stage_meta_used[ms] = true;
    p->stage_meta_next = (ms + 1) % kMetaRing;
    // Runs of consecutive block ids among positions [lo, hi): fn(first block, position, length).
    auto for_runs = [&](int32_t lo, int32_t hi, auto&& fn) {
        for (int32_t i = lo; i < hi && e == cudaSuccess;) {
            int32_t rn = 1;
            while (i + rn < hi && block_ids[i + rn] == block_ids[i] + rn) ++rn;
            fn(static_cast<size_t>(block_ids[i]), static_cast<size_t>(i), static_cast<size_t>(rn));
            i += rn;
        }
    };
    if (runs > 1 && p->d_hks) {
        // Every layer's scales of every block by one gather kernel on the transfer stream,
        // reading the mapped slab: one launch instead of one copy command per run.
        const int32_t rc = sc::launch_gather_pieces(
            p->d_hks, p->B, p->d_sc, reinterpret_cast<const int32_t*>(p->d_stage_meta + p->off_ids),
            n, 2 * L, static_cast<int64_t>(blk_scales) * 2, p->d_status, p->transfer);
        if (rc != SC_OK) return rc;
    } else {
        for_runs(0, n, [&](size_t b0, size_t i, size_t rn) {
            e = cudaMemcpy2DAsync(p->d_sc + i * blk_scales, static_cast<size_t>(n) * blk_scales * 2,
                                  p->h_ks + b0 * blk_scales,
                                  static_cast<size_t>(p->B) * blk_scales * 2, rn * blk_scales * 2,
                                  2 * static_cast<size_t>(L), cudaMemcpyHostToDevice, p->transfer);
        });
        if (e != cudaSuccess) return cuda_error(e, "scale copies");
    }
    const size_t src_pitch = static_cast<size_t>(p->B) * blk_codes;
    const size_t slab_codes = static_cast<size_t>(L) * src_pitch;
    int32_t i0 = 0;
    for (size_t si = 0; si < n_stages; ++si) {
        const int32_t m = p->stages[si];
        const int s = static_cast<int>(si % static_cast<size_t>(p->n_slots));
        if (p->slot_used[s]) e = cudaStreamWaitEvent(p->transfer, p->slot_free[s], 0);
        int8_t* slot = p->d_kq[s];
        const size_t dst_pitch = static_cast<size_t>(m) * blk_codes;
        const size_t v_off = static_cast<size_t>(L) * dst_pitch;  // V codes of the stage
        for_runs(i0, i0 + m, [&](size_t b0, size_t i, size_t rn) {
            const size_t j = i - static_cast<size_t>(i0);
            if (p->stage_3d) {
                cudaMemcpy3DParms c = {};
                c.srcPtr = make_cudaPitchedPtr(p->h_kq, src_pitch, src_pitch, static_cast<size_t>(L));
                c.srcPos = make_cudaPos(b0 * blk_codes, 0, 0);
                c.dstPtr = make_cudaPitchedPtr(slot, dst_pitch, dst_pitch, static_cast<size_t>(L));
                c.dstPos = make_cudaPos(j * blk_codes, 0, 0);
                c.extent = make_cudaExtent(rn * blk_codes, static_cast<size_t>(L), 2);
                c.kind = cudaMemcpyHostToDevice;
                e = cudaMemcpy3DAsync(&c, p->transfer);
            } else {
                for (int kv = 0; kv < 2 && e == cudaSuccess; ++kv)
                    e = cudaMemcpy2DAsync(slot + kv * v_off + j * blk_codes, dst_pitch,
                                          p->h_kq + kv * slab_codes + b0 * blk_codes, src_pitch,
                                          rn * blk_codes, static_cast<size_t>(L),
                                          cudaMemcpyHostToDevice, p->transfer);
            }
        });
        if (e == cudaSuccess) e = cudaEventRecord(p->ready[s], p->transfer);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, p->ready[s], 0);
        if (e != cudaSuccess) return cuda_error(e, "block-stage copies");
        sc::PagedArgs a{};
        a.n_requests = L;
        a.max_pages = m;
        a.page_size = p->chunk;
        a.n_heads = p->H;
        a.head_dim = p->D;
        a.n_pool_pages = static_cast<int64_t>(L) * m;
        a.pool_kq = slot;
        a.pool_vq = slot + v_off;
        // Scales of layer l, stage page j: row (l * n + i0 + j) of d_sc's K half, i.e. pool
        // page l * m + j plus a skew of l * (n - m) pages.
        a.pool_ks = p->d_sc + static_cast<size_t>(i0) * blk_scales;
        a.pool_vs = p->d_sc + (static_cast<size_t>(L) * n + i0) * blk_scales;
        a.scale_request_skew = static_cast<int64_t>(n - m) * static_cast<int64_t>(blk_scales);
        a.page_table = p->d_table;  // identity: page j of layer l is pool page l * m + j
        a.page_table_stride = m;
        a.seq_lens = reinterpret_cast<const int32_t*>(p->d_stage_meta) + si;
        a.seq_len_shared = 1;
        a.delta_p = reinterpret_cast<const float*>(p->d_stage_meta + p->off_dps) + i0;
        a.delta_p_per_page = 2;  // block i0 + j's shift, the same for every layer
        a.theta_base = theta_base;
        a.inv_freq = inv_freq;
        a.k_out_ptrs = reinterpret_cast<const uint64_t*>(p->d_stage_meta + p->off_kp);
        a.v_out_ptrs = reinterpret_cast<const uint64_t*>(p->d_stage_meta + p->off_vp);
        a.out_ptr_offset = static_cast<int64_t>(i0) * p->chunk * out_strides[0];
        for (int i = 0; i < 3; ++i) a.out_strides[i] = out_strides[i];
        a.out_numel = out_numel;
        a.out_dtype = out_dtype;
        a.status = p->d_status;
        a.stream = cs;
        const int32_t rc = sc::launch_paged(a);
        if (rc != SC_OK) return rc;
        e = cudaEventRecord(p->slot_free[s], cs);
        if (e != cudaSuccess) return cuda_error(e, "restore enqueue");
        p->slot_used[s] = true;
        i0 += m;
    }
    e = cudaEventRecord(p->done, cs);
    if (e != cudaSuccess) return cuda_error(e, "restore enqueue");
    p->any_restore = true;
    return sc::ok();
}

}  // namespace

extern "C" int32_t sc_pipeline_restore_launches(const sc_pipeline* p, int32_t n_blocks,
                                                int32_t* launches) {
    if (!p || !launches) return set_error(SC_ERR_INVALID_ARGUMENT, "null argument");
    if (n_blocks < 0 || n_blocks > p->max_blocks)
        return set_error(SC_ERR_INVALID_ARGUMENT, "n_blocks %d outside [0, %lld]", n_blocks,
                         (long long)p->max_blocks);
    if (n_blocks == 0)
        *launches = 0;
    else if (p->stage_cap > 0 && n_blocks <= p->stage_cap &&
             (n_blocks < kSplitLastMin || p->stage_cap < 2))
        *launches = 1;
    else if (p->stage_cap > 0)  // the stages of stage_sizes(): the front ones and a last block
        *launches = static_cast<int32_t>((n_blocks - 1 + p->stage_cap - 1) / p->stage_cap + 1);
    else
        *launches = p->L;
    return sc::ok();
}

extern "C" int32_t sc_pipeline_plan(const sc_pipeline* p, int32_t offload,
                                    const int32_t* block_ids, int32_t n_blocks,
                                    int32_t* launches, int32_t* copies) {
    if (!p || !launches || !copies || (n_blocks > 0 && !block_ids))
        return set_error(SC_ERR_INVALID_ARGUMENT, "null argument");
    if (n_blocks < 0 || n_blocks > p->max_blocks)
        return set_error(SC_ERR_INVALID_ARGUMENT, "n_blocks %d outside [0, %lld]", n_blocks,
                         (long long)p->max_blocks);
    for (int32_t i = 0; i < n_blocks; ++i)
        if (block_ids[i] < 0 || block_ids[i] >= p->B)
            return set_error(SC_ERR_INVALID_ARGUMENT, "block id %d outside [0, %lld)",
                             block_ids[i], (long long)p->B);
    *launches = 0;
    *copies = 0;
    if (n_blocks == 0) return sc::ok();
    // Runs of consecutive block ids among positions [lo, hi).
    auto runs_in = [&](int32_t lo, int32_t hi) {
        int32_t r = hi > lo ? 1 : 0;
        for (int32_t i = lo + 1; i < hi; ++i) r += block_ids[i] != block_ids[i - 1] + 1;
        return r;
    };
    const int32_t runs = runs_in(0, n_blocks);
    if (offload) {  // sc_pipeline_offload: quantize K and V, then scatter kernels or copies
        if (runs > 1 && p->d_hkq && p->d_hks && !has_duplicates(block_ids, n_blocks)) {
            *launches = 2 + 2 * ((n_blocks + sc::kMaxScatterIds - 1) / sc::kMaxScatterIds);
        } else {
            *launches = 2;
            *copies = runs * ((p->codes_2d ? 1 : 2) + (p->offload_scales_2d ? 1 : 2));
        }
        return sc::ok();
    }
    if (p->stage_cap > 0) {  // block stages: metadata upload, scales, per stage its runs
        std::vector<int32_t> st;
        stage_sizes(n_blocks, p->stage_cap, st);
        const bool gather = runs > 1 && p->d_hks;
        *launches = static_cast<int32_t>(st.size()) + (gather ? 1 : 0);
        *copies = 1 + (gather ? 0 : runs);
        int32_t i0 = 0;
        for (const int32_t m : st) {
            *copies += runs_in(i0, i0 + m) * (p->stage_3d ? 1 : 2);
            i0 += m;
        }
    } else {  // layer by layer
        *launches = p->L;
        *copies = 1 + (p->scales_2d ? runs : 2 * p->L * runs) + p->L * runs * (p->codes_2d ? 1 : 2);
    }
    return sc::ok();
}

extern "C" int32_t sc_pipeline_restore(sc_pipeline* p, const int32_t* block_ids,
                                       const int32_t* delta_ps, int32_t n_blocks,
                                       double theta_base, const float* inv_freq,
                                       void* const* k_out, void* const* v_out,
                                       const int64_t* out_strides, int64_t out_numel,
                                       int32_t out_dtype, void* compute_stream) {
    if (!p) return set_error(SC_ERR_INVALID_ARGUMENT, "null pipeline");
    if (n_blocks == 0) return sc::ok();
    if (n_blocks < 0 || n_blocks > p->max_blocks)
        return set_error(SC_ERR_INVALID_ARGUMENT, "n_blocks %d outside [0, %lld]", n_blocks,
                         (long long)p->max_blocks);
    if (!block_ids || !delta_ps || !k_out || !v_out || !out_strides)
        return set_error(SC_ERR_INVALID_ARGUMENT, "null argument");
    for (int32_t i = 0; i < n_blocks; ++i)
        if (block_ids[i] < 0 || block_ids[i] >= p->B)
            return set_error(SC_ERR_INVALID_ARGUMENT, "block id %d outside [0, %lld)",
                             block_ids[i], (long long)p->B);
    for (int32_t l = 0; l < p->L; ++l)
        if (!k_out[l] || !v_out[l])
            return set_error(SC_ERR_INVALID_ARGUMENT, "null output pointer for layer %d", l);
    DeviceGuard g(p->device);
    if (!g.ok) return set_error(SC_ERR_CUDA, "cudaSetDevice(%d) failed", p->device);
    cudaStream_t cs = static_cast<cudaStream_t>(compute_stream);
    if (p->stage_cap > 0)
        return restore_block_stages(p, block_ids, delta_ps, n_blocks, theta_base, inv_freq, k_out,
                                    v_out, out_strides, out_numel, out_dtype, cs);
    cudaError_t e = cudaSuccess;

    // Metadata: the next host buffer may still feed an upload kMetaRing restores back.
    const int ms = p->meta_next;
    if (p->meta_used[ms]) e = cudaEventSynchronize(p->meta_uploaded[ms]);
    if (e != cudaSuccess) return cuda_error(e, "waiting for an earlier metadata upload");
    Meta* hm = reinterpret_cast<Meta*>(p->h_meta + static_cast<size_t>(ms) * p->meta_stride);
    hm->seq_len = n_blocks * p->chunk;
    hm->out_offset = 0;
    for (int32_t i = 0; i < n_blocks; ++i) hm->delta_p[i] = static_cast<float>(delta_ps[i]);
    // The device copy may still be read by the previous restore's last kernels.
    if (p->any_restore) e = cudaStreamWaitEvent(p->transfer, p->done, 0);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(p->d_meta, hm, meta_bytes(n_blocks), cudaMemcpyHostToDevice,
                            p->transfer);
    if (e == cudaSuccess) e = cudaEventRecord(p->meta_uploaded[ms], p->transfer);
    if (e != cudaSuccess) return cuda_error(e, "metadata upload");
    p->meta_used[ms] = true;
    p->meta_next = (ms + 1) % kMetaRing;

    const size_t row = static_cast<size_t>(p->chunk) * p->H;
    const size_t blk_codes = row * p->D, blk_scales = row;
    const size_t slab_codes = static_cast<size_t>(p->L) * p->B * blk_codes;
    const size_t stage_codes = static_cast<size_t>(p->max_blocks) * blk_codes;
    const size_t stage_scales = static_cast<size_t>(p->max_blocks) * blk_scales;
    // Runs of consecutive block ids: fn(first block, position in the restore, length).
    auto for_runs = [&](auto&& fn) {
        for (int32_t i = 0; i < n_blocks && e == cudaSuccess;) {
            int32_t n = 1;
            while (i + n < n_blocks && block_ids[i + n] == block_ids[i] + n) ++n;
            fn(static_cast<size_t>(block_ids[i]), static_cast<size_t>(i), static_cast<size_t>(n));
            i += n;
        }
    };
    // Scales of every layer (rows t = 0..2L-1: K scales of layer t, then V scales of layer
    // t - L; the V slab follows the K slab, so one source pitch covers both).
    const size_t src_pitch_s = static_cast<size_t>(p->B) * blk_scales * 2;
    for_runs([&](size_t b0, size_t dst, size_t n) {
        if (p->scales_2d) {
            e = cudaMemcpy2DAsync(p->d_sc + dst * blk_scales, stage_scales * 2,
                                  p->h_ks + b0 * blk_scales, src_pitch_s, n * blk_scales * 2,
                                  2 * static_cast<size_t>(p->L), cudaMemcpyHostToDevice,
                                  p->transfer);
        } else {
            for (int32_t t = 0; t < 2 * p->L && e == cudaSuccess; ++t)
                e = cudaMemcpyAsync(p->d_sc + t * stage_scales + dst * blk_scales,
                                    p->h_ks + t * (src_pitch_s / 2) + b0 * blk_scales,
                                    n * blk_scales * 2, cudaMemcpyHostToDevice, p->transfer);
        }
    });
    for (int32_t l = 0; l < p->L && e == cudaSuccess; ++l) {
        const int s = l % p->n_slots;
        if (p->slot_used[s]) e = cudaStreamWaitEvent(p->transfer, p->slot_free[s], 0);
        const size_t lay_codes = static_cast<size_t>(l) * p->B * blk_codes;
        // K and V codes of the layer: rows 0 and 1 of one 2-D copy (V slab = K slab +
        // slab_codes on the host, V staging = K staging + stage_codes on the device).
        for_runs([&](size_t b0, size_t dst, size_t n) {
            int8_t* d = p->d_kq[s] + dst * blk_codes;
            const int8_t* h = p->h_kq + lay_codes + b0 * blk_codes;
            if (p->codes_2d) {
                e = cudaMemcpy2DAsync(d, stage_codes, h, slab_codes, n * blk_codes, 2,
                                      cudaMemcpyHostToDevice, p->transfer);
            } else {
                e = cudaMemcpyAsync(d, h, n * blk_codes, cudaMemcpyHostToDevice, p->transfer);
                if (e == cudaSuccess)
                    e = cudaMemcpyAsync(d + stage_codes, h + slab_codes, n * blk_codes,
                                        cudaMemcpyHostToDevice, p->transfer);
            }
        });
        if (e == cudaSuccess) e = cudaEventRecord(p->ready[s], p->transfer);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, p->ready[s], 0);
        if (e != cudaSuccess) break;
        sc::PagedArgs a{};
        a.n_requests = 1;
        a.max_pages = n_blocks;
        a.page_size = p->chunk;
        a.n_heads = p->H;
        a.head_dim = p->D;
        a.n_pool_pages = n_blocks;
        a.pool_kq = p->d_kq[s];
        a.pool_ks = p->d_sc + static_cast<size_t>(l) * stage_scales;
        a.pool_vq = p->d_vq[s];
        a.pool_vs = p->d_sc + static_cast<size_t>(p->L + l) * stage_scales;
        a.page_table = p->d_table;
        a.page_table_stride = p->max_blocks;
        a.seq_lens = &p->d_meta->seq_len;
        a.delta_p = p->d_meta->delta_p;
        a.delta_p_per_page = 1;
        a.theta_base = theta_base;
        a.inv_freq = inv_freq;
        a.k_out = k_out[l];
        a.v_out = v_out[l];
        a.out_offsets = &p->d_meta->out_offset;
        for (int i = 0; i < 3; ++i) a.out_strides[i] = out_strides[i];
        a.out_numel = out_numel;
        a.out_dtype = out_dtype;
        a.status = p->d_status;
        a.flags = 0;
        a.stream = cs;
        const int32_t rc = sc::launch_paged(a);
        if (rc != SC_OK) return rc;
        e = cudaEventRecord(p->slot_free[s], cs);
        p->slot_used[s] = true;
    }
    if (e == cudaSuccess) e = cudaEventRecord(p->done, cs);
    if (e != cudaSuccess) return cuda_error(e, "restore enqueue");
    p->any_restore = true;
    return sc::ok();
}

extern "C" int32_t sc_pipeline_offload(sc_pipeline* p, int32_t layer, const int32_t* block_ids,
                                       int32_t n_blocks, const void* k, const int64_t* k_strides,
                                       const void* v, const int64_t* v_strides, int32_t x_dtype,
                                       void* compute_stream) {
    if (!p) return set_error(SC_ERR_INVALID_ARGUMENT, "null pipeline");
    if (n_blocks == 0) return sc::ok();
    if (layer < 0 || layer >= p->L)
        return set_error(SC_ERR_INVALID_ARGUMENT, "layer %d outside [0, %d)", layer, p->L);
    if (n_blocks < 0 || n_blocks > p->max_blocks)
        return set_error(SC_ERR_INVALID_ARGUMENT, "n_blocks %d outside [0, %lld]", n_blocks,
                         (long long)p->max_blocks);
    if (!block_ids || !k || !v || !k_strides || !v_strides)
        return set_error(SC_ERR_INVALID_ARGUMENT, "null argument");
    for (int32_t i = 0; i < n_blocks; ++i)
        if (block_ids[i] < 0 || block_ids[i] >= p->B)
            return set_error(SC_ERR_INVALID_ARGUMENT, "block id %d outside [0, %lld)",
                             block_ids[i], (long long)p->B);
    DeviceGuard g(p->device);
    if (!g.ok) return set_error(SC_ERR_CUDA, "cudaSetDevice(%d) failed", p->device);
    cudaStream_t cs = static_cast<cudaStream_t>(compute_stream);
    const int64_t n_tok = static_cast<int64_t>(n_blocks) * p->chunk;
    cudaError_t e = cudaSuccess;
    const size_t row = static_cast<size_t>(p->chunk) * p->H;
    const size_t blk_codes = row * p->D, blk_scales = row;
    const size_t stage_codes = static_cast<size_t>(p->max_blocks) * blk_codes;
    const size_t stage_scales = static_cast<size_t>(p->max_blocks) * blk_scales;
    const size_t slab_codes = static_cast<size_t>(p->L) * p->B * blk_codes;
    const size_t slab_scales = static_cast<size_t>(p->L) * p->B * blk_scales;
    // Staging slot s may still feed the copies of the offload before last: wait for them
    // on the compute stream (layer l+1's quantize overlaps layer l's copies).
    const int s = p->o_next;
    if (p->o_used[s]) e = cudaStreamWaitEvent(cs, p->o_free[s], 0);
    if (e != cudaSuccess) return cuda_error(e, "ordering the offload staging slot");
    int8_t* okq = p->o_codes[s];
    int8_t* ovq = okq + stage_codes;
    uint16_t* oks = p->o_scales[s];
    uint16_t* ovs = oks + stage_scales;
    const int64_t q_st[3] = {static_cast<int64_t>(p->H) * p->D, p->D, 1};
    const int64_t s_st[2] = {p->H, 1};
    int32_t rc = sc_quantize_int8(n_tok, p->H, p->D, k, x_dtype, k_strides, 1e-5f, okq, q_st,
                                  oks, SC_DTYPE_F16, s_st, 0, cs);
    if (rc != SC_OK) return rc;
    rc = sc_quantize_int8(n_tok, p->H, p->D, v, x_dtype, v_strides, 1e-5f, ovq, q_st, ovs,
                          SC_DTYPE_F16, s_st, 0, cs);
    if (rc != SC_OK) return rc;
    e = cudaEventRecord(p->o_ready[s], cs);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p->transfer, p->o_ready[s], 0);
    const size_t lay_codes = static_cast<size_t>(layer) * p->B * blk_codes;
    const size_t lay_scales = static_cast<size_t>(layer) * p->B * blk_scales;
    int32_t runs = 1;
    for (int32_t i = 1; i < n_blocks; ++i) runs += block_ids[i] != block_ids[i - 1] + 1;
    if (e == cudaSuccess && runs > 1 && p->d_hkq && p->d_hks &&
        !has_duplicates(block_ids, n_blocks)) {
        // A list in several runs: one scatter kernel writes every block's K and V codes into
        // the mapped slab (rows: K, V), one its scales, on the transfer stream, instead of two
        // copy commands per run.
        const int64_t lb = static_cast<int64_t>(p->L) * p->B;  // K -> V slab distance, blocks
        rc = sc::launch_scatter_pieces(okq, p->max_blocks, p->d_hkq + lay_codes, lb, p->B,
                                       block_ids, n_blocks, 2, static_cast<int64_t>(blk_codes),
                                       p->d_status, p->transfer);
        if (rc == SC_OK)
            rc = sc::launch_scatter_pieces(oks, p->max_blocks, p->d_hks + lay_scales, lb, p->B,
                                           block_ids, n_blocks, 2,
                                           static_cast<int64_t>(blk_scales) * 2, p->d_status,
                                           p->transfer);
        if (rc != SC_OK) return rc;
    } else {
        // Per run: K and V codes as the two rows of one 2-D copy (host pitch slab_codes,
        // device pitch stage_codes), and the same for the scales.
        for (int32_t i = 0; i < n_blocks && e == cudaSuccess;) {
            int32_t n = 1;
            while (i + n < n_blocks && block_ids[i + n] == block_ids[i] + n) ++n;
            const size_t b0 = static_cast<size_t>(block_ids[i]);
            const size_t src = static_cast<size_t>(i);
            int8_t* hc = p->h_kq + lay_codes + b0 * blk_codes;
            const int8_t* dc = okq + src * blk_codes;
            if (p->codes_2d) {
                e = cudaMemcpy2DAsync(hc, slab_codes, dc, stage_codes, n * blk_codes, 2,
                                      cudaMemcpyDeviceToHost, p->transfer);
            } else {
                e = cudaMemcpyAsync(hc, dc, n * blk_codes, cudaMemcpyDeviceToHost, p->transfer);
                if (e == cudaSuccess)
                    e = cudaMemcpyAsync(hc + slab_codes, dc + stage_codes, n * blk_codes,
                                        cudaMemcpyDeviceToHost, p->transfer);
            }
            uint16_t* hs = p->h_ks + lay_scales + b0 * blk_scales;
            const uint16_t* ds = oks + src * blk_scales;
            if (e == cudaSuccess && p->offload_scales_2d) {
                e = cudaMemcpy2DAsync(hs, slab_scales * 2, ds, stage_scales * 2,
                                      n * blk_scales * 2, 2, cudaMemcpyDeviceToHost, p->transfer);
            } else if (e == cudaSuccess) {
                e = cudaMemcpyAsync(hs, ds, n * blk_scales * 2, cudaMemcpyDeviceToHost,
                                    p->transfer);
                if (e == cudaSuccess)
                    e = cudaMemcpyAsync(hs + slab_scales, ds + stage_scales, n * blk_scales * 2,
                                        cudaMemcpyDeviceToHost, p->transfer);
            }
            i += n;
        }
    }
    if (e == cudaSuccess) e = cudaEventRecord(p->o_free[s], p->transfer);
    if (e != cudaSuccess) return cuda_error(e, "offload enqueue");
    p->o_used[s] = true;
    p->o_last = s;
    p->o_next = (s + 1) % 2;
    p->any_offload = true;
    return sc::ok();
}

namespace {
// Holds the calling thread's timer slack at 1 us for the scope: with the default 50 us slack a
// short sleep returns 50-100 us late, which restores of a few milliseconds would see as
// latency.  The previous slack is put back on exit.
struct TightTimerSlack {
    long prev = -1;
    TightTimerSlack() {
        prev = prctl(PR_GET_TIMERSLACK, 0, 0, 0, 0);
        if (prev > 0) prctl(PR_SET_TIMERSLACK, 1000UL, 0, 0, 0);
    }
    ~TightTimerSlack() {
        if (prev > 0) prctl(PR_SET_TIMERSLACK, static_cast<unsigned long>(prev), 0, 0, 0);
    }
};

// Polls without sleeping for the first millisecond, then every 20 us with a 1 us timer slack
// (measured on the GPU hosts: with 50 us sleeps at the default slack, a 1.3 ms restore's
// completion was seen 50-110 us late).
int32_t wait_event(cudaEvent_t ev, double deadline, double timeout_s, const char* what) {
    const double spin_until = now_s() + 1e-3;
    TightTimerSlack slack;
    for (;;) {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return SC_OK;
        if (e != cudaErrorNotReady) return cuda_error(e, what);
        const double t = now_s();
        if (t >= deadline)
            return set_error(SC_ERR_TIMEOUT, "%s not complete after %.3f s", what, timeout_s);
        if (t < spin_until)
            sched_yield();
        else
            usleep(20);
    }
}
}  // namespace

extern "C" int32_t sc_pipeline_synchronize(sc_pipeline* p, double timeout_s) {
    if (!p) return set_error(SC_ERR_INVALID_ARGUMENT, "null pipeline");
    DeviceGuard g(p->device);
    const double deadline = now_s() + (timeout_s > 0 ? timeout_s : 0);
    if (p->any_restore) {
        const int32_t rc = wait_event(p->done, deadline, timeout_s, "restore");
        if (rc != SC_OK) return rc;
    }
    if (p->any_offload) {
        const int32_t rc = wait_event(p->o_free[p->o_last], deadline, timeout_s, "offload");
        if (rc != SC_OK) return rc;
    }
    return sc::ok();
}

extern "C" int32_t sc_pipeline_join(sc_pipeline* p, void* stream) {
    if (!p) return set_error(SC_ERR_INVALID_ARGUMENT, "null pipeline");
    DeviceGuard g(p->device);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (p->any_restore) e = cudaStreamWaitEvent(st, p->done, 0);
    if (e == cudaSuccess && p->any_offload) e = cudaStreamWaitEvent(st, p->o_free[p->o_last], 0);
    if (e != cudaSuccess) return cuda_error(e, "joining the pipeline");
    return sc::ok();
}

extern "C" int32_t sc_pipeline_status(sc_pipeline* p, int32_t* status_bits) {
    if (!p || !status_bits) return set_error(SC_ERR_INVALID_ARGUMENT, "null argument");
    const int32_t rc = sc_pipeline_synchronize(p, 60.0);
    if (rc != SC_OK) return rc;
    DeviceGuard g(p->device);
    int32_t v = 0;
    cudaError_t e = cudaMemcpy(&v, p->d_status, sizeof(int32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(p->d_status, 0, sizeof(int32_t));
    if (e != cudaSuccess) return cuda_error(e, "reading pipeline status");
    *status_bits = v;
    return v == 0 ? sc::ok() : set_error(SC_ERR_OUT_OF_RANGE, "device status bits 0x%x", v);
}

extern "C" int32_t sc_pipeline_destroy(sc_pipeline* p) {
    release(p);
    return sc::ok();
}
