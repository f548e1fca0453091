/*
 * c_abi_consumer.c — a C11 program that uses the library through its C ABI only (no Python,
 * no torch in the process), the way a cgo / JNI / N-API binding would.
 *
 * It quantizes seeded float32 K and V [T, H, D] on the GPU (sc_quantize_int8, fp16 scales),
 * restores them (sc_dequant_rope_kv: K shifted by delta_p with the cos/sin table built by the
 * library, V plain, fp16 out, one launch), checks a rejected call's status and message, then
 * drives the pinned-host pipeline the way an engine binding would (sc_pipeline_create, the
 * slabs filled through sc_pipeline_host_slabs, sc_pipeline_plan, sc_pipeline_restore of a
 * scattered block list, sc_pipeline_synchronize, sc_pipeline_status), and writes inputs and
 * outputs to a file that the Python test compares with the oracle.
 *
 *   c_abi_consumer <out.bin> <T> <H> <D> <delta_p> <theta>
 *
 * File layout (little endian): int32 T, H, D; float64 delta_p, theta; then float32 xk[T*H*D],
 * xv[T*H*D]; int8 kq[T*H*D], vq[T*H*D]; uint16 ks[T*H], vs[T*H]; uint16 ko[T*H*D], vo[T*H*D]
 * (fp16 bit patterns).  Then the pipeline: int32 L, B, C, PH, PD, n, launches, copies; int32
 * ids[n], shifts[n]; int8 K and V code slabs [L*B*C*PH*PD] each; uint16 K and V scale slabs
 * [L*B*C*PH] each; uint16 K and V outputs [L*n*C*PH*PD] each.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "speccache_b200.h"

#define CHECK_CUDA(call)                                                             \
    do {                                                                             \
        cudaError_t e_ = (call);                                                     \
        if (e_ != cudaSuccess) {                                                     \
            fprintf(stderr, "%s failed: %s\n", #call, cudaGetErrorString(e_));      \
            return 2;                                                                \
        }                                                                            \
    } while (0)

#define CHECK_SC(call)                                                               \
    do {                                                                             \
        int32_t rc_ = (call);                                                        \
        if (rc_ != SC_OK) {                                                          \
            fprintf(stderr, "%s returned %d: %s\n", #call, rc_, sc_last_error());   \
            return 3;                                                                \
        }                                                                            \
    } while (0)

/* 64-bit linear congruential generator (Knuth's MMIX constants): uniform in [-4, 4). */
static float next_value(uint64_t* state) {
    *state = *state * 6364136223846793005ULL + 1442695040888963407ULL;
    return (float)((double)(*state >> 11) * (1.0 / 9007199254740992.0) * 8.0 - 4.0);
}

static int write_all(FILE* f, const void* p, size_t n) { return fwrite(p, 1, n, f) == n ? 0 : 1; }

int main(int argc, char** argv) {
    if (argc != 7) {
        fprintf(stderr, "usage: %s <out.bin> <T> <H> <D> <delta_p> <theta>\n", argv[0]);
        return 1;
    }
    const int32_t T = atoi(argv[2]), H = atoi(argv[3]), D = atoi(argv[4]);
    const double delta_p = atof(argv[5]), theta = atof(argv[6]);
    if (T <= 0 || H <= 0 || D <= 0 || D % 2 != 0) {
        fprintf(stderr, "bad geometry\n");
        return 1;
    }
    if (sc_abi_version() != SC_ABI_VERSION) {
        fprintf(stderr, "ABI version %d, header %d\n", sc_abi_version(), SC_ABI_VERSION);
        return 4;
    }
    const size_t n = (size_t)T * H * D, rows = (size_t)T * H;

    float* xk = malloc(n * sizeof(float));
    float* xv = malloc(n * sizeof(float));
    int8_t* kq = malloc(n);
    int8_t* vq = malloc(n);
    uint16_t* ks = malloc(rows * 2);
    uint16_t* vs = malloc(rows * 2);
    uint16_t* ko = malloc(n * 2);
    uint16_t* vo = malloc(n * 2);
    if (!xk || !xv || !kq || !vq || !ks || !vs || !ko || !vo) return 5;
    uint64_t state = 20260611ULL;
    for (size_t i = 0; i < n; ++i) xk[i] = next_value(&state);
    for (size_t i = 0; i < n; ++i) xv[i] = next_value(&state);
    for (int32_t h = 0; h < H; ++h) xk[(size_t)h * D] = 0.0f;              /* token 0, dim 0 */
    for (int32_t d = 0; d < D; ++d) xv[(size_t)(H - 1) * D + d] = 0.0f;    /* a zero row */

    float *d_xk, *d_xv;
    int8_t *d_kq, *d_vq;
    void *d_ks, *d_vs, *d_ko, *d_vo;
    CHECK_CUDA(cudaMalloc((void**)&d_xk, n * sizeof(float)));
    CHECK_CUDA(cudaMalloc((void**)&d_xv, n * sizeof(float)));
    CHECK_CUDA(cudaMalloc((void**)&d_kq, n));
    CHECK_CUDA(cudaMalloc((void**)&d_vq, n));
    CHECK_CUDA(cudaMalloc(&d_ks, rows * 2));
    CHECK_CUDA(cudaMalloc(&d_vs, rows * 2));
    CHECK_CUDA(cudaMalloc(&d_ko, n * 2));
    CHECK_CUDA(cudaMalloc(&d_vo, n * 2));
    CHECK_CUDA(cudaMemcpy(d_xk, xk, n * sizeof(float), cudaMemcpyHostToDevice));
    CHECK_CUDA(cudaMemcpy(d_xv, xv, n * sizeof(float), cudaMemcpyHostToDevice));

    cudaStream_t stream;
    CHECK_CUDA(cudaStreamCreate(&stream));
    const int64_t x_st[3] = {(int64_t)H * D, D, 1};
    const int64_t s_st[2] = {H, 1};
    CHECK_SC(sc_quantize_int8(T, H, D, d_xk, SC_DTYPE_F32, x_st, 1e-5f, d_kq, x_st, d_ks,
                              SC_DTYPE_F16, s_st, 0, stream));
    CHECK_SC(sc_quantize_int8(T, H, D, d_xv, SC_DTYPE_F32, x_st, 1e-5f, d_vq, x_st, d_vs,
                              SC_DTYPE_F16, s_st, 0, stream));

    const int64_t q_st[4] = {(int64_t)T * H * D, (int64_t)H * D, D, 1};
    const int64_t sc_st[3] = {(int64_t)T * H, H, 1};
    CHECK_SC(sc_dequant_rope_kv(1, T, H, D, d_kq, q_st, d_ks, sc_st, d_vq, q_st, d_vs, sc_st,
                                SC_DTYPE_F16, NULL, NULL, NULL, delta_p, NULL, theta, NULL, d_ko,
                                q_st, d_vo, q_st, SC_DTYPE_F16, 0, stream));

    /* A rejected call: odd head_dim.  It must return an error and leave a message. */
    const int32_t rc = sc_dequant_rope_kv(1, T, H, D - 1, d_kq, q_st, d_ks, sc_st, NULL, NULL,
                                          NULL, NULL, SC_DTYPE_F16, NULL, NULL, NULL, delta_p,
                                          NULL, theta, NULL, d_ko, q_st, NULL, NULL,
                                          SC_DTYPE_F16, 0, stream);
    if (rc == SC_OK || sc_last_error()[0] == '\0') {
        fprintf(stderr, "odd head_dim was accepted (rc %d)\n", rc);
        return 6;
    }
    printf("rejected call: rc=%d message=\"%s\"\n", rc, sc_last_error());

    CHECK_CUDA(cudaStreamSynchronize(stream));
    CHECK_CUDA(cudaMemcpy(kq, d_kq, n, cudaMemcpyDeviceToHost));
    CHECK_CUDA(cudaMemcpy(vq, d_vq, n, cudaMemcpyDeviceToHost));
    CHECK_CUDA(cudaMemcpy(ks, d_ks, rows * 2, cudaMemcpyDeviceToHost));
    CHECK_CUDA(cudaMemcpy(vs, d_vs, rows * 2, cudaMemcpyDeviceToHost));
    CHECK_CUDA(cudaMemcpy(ko, d_ko, n * 2, cudaMemcpyDeviceToHost));
    CHECK_CUDA(cudaMemcpy(vo, d_vo, n * 2, cudaMemcpyDeviceToHost));

    FILE* f = fopen(argv[1], "wb");
    if (!f) return 7;
    const int32_t geo[3] = {T, H, D};
    const double sh[2] = {delta_p, theta};
    int bad = write_all(f, geo, sizeof geo) | write_all(f, sh, sizeof sh) |
              write_all(f, xk, n * 4) | write_all(f, xv, n * 4) | write_all(f, kq, n) |
              write_all(f, vq, n) | write_all(f, ks, rows * 2) | write_all(f, vs, rows * 2) |
              write_all(f, ko, n * 2) | write_all(f, vo, n * 2);
    if (bad) return 8;

    /* The pipeline: 3 layers x 12 blocks of 16 tokens x 2 heads x 64, fp16 out.  Nine scattered
     * blocks in six runs: the scales come by the gather kernel, and from eight blocks on the
     * last block has a stage of its own (two launches). */
    enum { PL = 3, PB = 12, PC = 16, PH = 2, PD = 64, PN = 9 };
    const int32_t ids[PN] = {4, 0, 1, 5, 9, 10, 11, 2, 7};
    const int32_t shifts[PN] = {-300, 12, 12, 4000, -7, 0, 65000, 1, -4096};
    const size_t slab = (size_t)PL * PB * PC * PH * PD, slab_s = (size_t)PL * PB * PC * PH;
    const size_t per_layer = (size_t)PN * PC * PH * PD;
    sc_pipeline* pipe = NULL;
    CHECK_SC(sc_pipeline_create(0, PL, PB, PC, PH, PD, PB, 2, 0, &pipe));
    int8_t *h_kq, *h_vq;
    void *h_ks, *h_vs;
    CHECK_SC(sc_pipeline_host_slabs(pipe, &h_kq, &h_ks, &h_vq, &h_vs));
    for (size_t i = 0; i < slab; ++i) h_kq[i] = (int8_t)((int)(next_value(&state) * 31.75f));
    for (size_t i = 0; i < slab; ++i) h_vq[i] = (int8_t)((int)(next_value(&state) * 31.75f));
    /* fp16 scales (1 + m/1024) * 2^-8: exponent field 7, mantissa m */
    for (size_t i = 0; i < slab_s; ++i)
        ((uint16_t*)h_ks)[i] = (uint16_t)(0x1C00u | ((unsigned)((next_value(&state) + 4.0f) * 128.0f) & 1023u));
    for (size_t i = 0; i < slab_s; ++i)
        ((uint16_t*)h_vs)[i] = (uint16_t)(0x1C00u | ((unsigned)((next_value(&state) + 4.0f) * 128.0f) & 1023u));
    int32_t launches = 0, copies = 0;
    CHECK_SC(sc_pipeline_plan(pipe, 0, ids, PN, &launches, &copies));
    void* d_pk[PL];
    void* d_pv[PL];
    for (int l = 0; l < PL; ++l) {
        CHECK_CUDA(cudaMalloc(&d_pk[l], per_layer * 2));
        CHECK_CUDA(cudaMalloc(&d_pv[l], per_layer * 2));
    }
    const int64_t out_st[3] = {(int64_t)PH * PD, PD, 1};
    CHECK_SC(sc_pipeline_restore(pipe, ids, shifts, PN, theta, NULL, d_pk, d_pv, out_st,
                                 (int64_t)per_layer, SC_DTYPE_F16, stream));
    CHECK_SC(sc_pipeline_synchronize(pipe, 30.0));
    CHECK_CUDA(cudaStreamSynchronize(stream));
    int32_t status = -1;
    CHECK_SC(sc_pipeline_status(pipe, &status));
    if (status != 0) {
        fprintf(stderr, "pipeline status %d\n", status);
        return 9;
    }
    uint16_t* pko = malloc(PL * per_layer * 2);
    uint16_t* pvo = malloc(PL * per_layer * 2);
    if (!pko || !pvo) return 5;
    for (int l = 0; l < PL; ++l) {
        CHECK_CUDA(cudaMemcpy(pko + l * per_layer, d_pk[l], per_layer * 2, cudaMemcpyDeviceToHost));
        CHECK_CUDA(cudaMemcpy(pvo + l * per_layer, d_pv[l], per_layer * 2, cudaMemcpyDeviceToHost));
    }
    const int32_t pgeo[8] = {PL, PB, PC, PH, PD, PN, launches, copies};
    bad = write_all(f, pgeo, sizeof pgeo) | write_all(f, ids, sizeof ids) |
          write_all(f, shifts, sizeof shifts) | write_all(f, h_kq, slab) | write_all(f, h_vq, slab) |
          write_all(f, h_ks, slab_s * 2) | write_all(f, h_vs, slab_s * 2) |
          write_all(f, pko, PL * per_layer * 2) | write_all(f, pvo, PL * per_layer * 2);
    bad |= fclose(f) != 0;
    printf("pipeline: %d launches, %d copies\n", launches, copies);
    for (int l = 0; l < PL; ++l) {
        cudaFree(d_pk[l]);
        cudaFree(d_pv[l]);
    }
    free(pko);
    free(pvo);
    CHECK_SC(sc_pipeline_destroy(pipe));

    CHECK_CUDA(cudaStreamDestroy(stream));
    cudaFree(d_xk);
    cudaFree(d_xv);
    cudaFree(d_kq);
    cudaFree(d_vq);
    cudaFree(d_ks);
    cudaFree(d_vs);
    cudaFree(d_ko);
    cudaFree(d_vo);
    free(xk);
    free(xv);
    free(kq);
    free(vq);
    free(ks);
    free(vs);
    free(ko);
    free(vo);
    if (bad) return 8;
    printf("ok T=%d H=%d D=%d\n", T, H, D);
    return 0;
}
