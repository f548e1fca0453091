/*
 * c_abi_consumer.c — a C11 program that uses the library through its C ABI only (no Python,
 * no torch in the process), the way a cgo / JNI / N-API binding would.
 *
 * It quantizes seeded float32 K and V [T, H, D] on the GPU (sc_quantize_int8, fp16 scales),
 * restores them (sc_dequant_rope_kv: K shifted by delta_p with the cos/sin table built by the
 * library, V plain, fp16 out, one launch), checks a rejected call's status and message, and
 * writes inputs and outputs to a file that the Python test compares with the oracle.
 *
 *   c_abi_consumer <out.bin> <T> <H> <D> <delta_p> <theta>
 *
 * File layout (little endian): int32 T, H, D; float64 delta_p, theta; then float32 xk[T*H*D],
 * xv[T*H*D]; int8 kq[T*H*D], vq[T*H*D]; uint16 ks[T*H], vs[T*H]; uint16 ko[T*H*D], vo[T*H*D]
 * (fp16 bit patterns).
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
    bad |= fclose(f) != 0;

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
