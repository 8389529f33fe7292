/* A C99 caller of include/tecoops.h that runs one paged decode step on the GPU, the way
 * a C executor written against the reference header (teco/interface/include/tecoops.h)
 * would: tecoopsReshapeAndCache writes each sequence's new K/V into the paged cache,
 * tecoopsFlashAttention attends over the cache, and the result is checked against a
 * plain fp32 loop on the host (max-abs <= 2e-2, mean-abs <= 2e-3 on bf16 data).
 * Built and run by tests/test_c_header.py (GPU part). */
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "tecoops.h"

#define B 3
#define HQ 8
#define HKV 2
#define D 128
#define BS 16
#define PAGES_PER_SEQ 8
#define NB (B * PAGES_PER_SEQ + 4)

#define CK(x)                                                                    \
    do {                                                                         \
        if (!(x)) {                                                              \
            fprintf(stderr, "%s:%d: %s\n", __FILE__, __LINE__, #x);              \
            return 1;                                                            \
        }                                                                        \
    } while (0)

static uint16_t to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest even */
    return (uint16_t)(u >> 16);
}
static float from_bf16(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static float urand(uint32_t *s) {
    *s = *s * 1664525u + 1013904223u;
    return ((*s >> 8) * (1.0f / 16777216.0f)) * 2.f - 1.f;
}

int main(void) {
    static uint16_t kc[NB * HKV * BS * D], vc[NB * HKV * BS * D];
    static uint16_t q[B * HQ * D], knew[B * HKV * D], vnew[B * HKV * D], out[B * HQ * D];
    int ctx[B] = {37, 100, 127}; /* tokens already cached; the new one goes at ctx[b] */
    int kv_lens[B], q_lens[B] = {1, 1, 1}, bt[B * PAGES_PER_SEQ];
    int64_t slot[B];
    uint32_t seed = 12345u;
    size_t i;
    int b, h, j, d;
    for (i = 0; i < sizeof(kc) / 2; ++i) kc[i] = to_bf16(urand(&seed));
    for (i = 0; i < sizeof(vc) / 2; ++i) vc[i] = to_bf16(urand(&seed));
    for (i = 0; i < sizeof(q) / 2; ++i) q[i] = to_bf16(urand(&seed));
    for (i = 0; i < sizeof(knew) / 2; ++i) knew[i] = to_bf16(urand(&seed));
    for (i = 0; i < sizeof(vnew) / 2; ++i) vnew[i] = to_bf16(urand(&seed));
    for (b = 0; b < B; ++b) {
        for (j = 0; j < PAGES_PER_SEQ; ++j) bt[b * PAGES_PER_SEQ + j] = NB - 1 - (b * PAGES_PER_SEQ + j);
        kv_lens[b] = ctx[b] + 1;
        slot[b] = (int64_t)bt[b * PAGES_PER_SEQ + ctx[b] / BS] * BS + ctx[b] % BS;
    }

    void *dkc, *dvc, *dq, *dk, *dv, *dout, *dbt, *dql, *dkl, *dslot;
    CK(cudaMalloc(&dkc, sizeof(kc)) == cudaSuccess && cudaMalloc(&dvc, sizeof(vc)) == cudaSuccess);
    CK(cudaMalloc(&dq, sizeof(q)) == cudaSuccess && cudaMalloc(&dout, sizeof(out)) == cudaSuccess);
    CK(cudaMalloc(&dk, sizeof(knew)) == cudaSuccess && cudaMalloc(&dv, sizeof(vnew)) == cudaSuccess);
    CK(cudaMalloc(&dbt, sizeof(bt)) == cudaSuccess && cudaMalloc(&dslot, sizeof(slot)) == cudaSuccess);
    CK(cudaMalloc(&dql, sizeof(q_lens)) == cudaSuccess && cudaMalloc(&dkl, sizeof(kv_lens)) == cudaSuccess);
    cudaMemcpy(dkc, kc, sizeof(kc), cudaMemcpyHostToDevice);
    cudaMemcpy(dvc, vc, sizeof(vc), cudaMemcpyHostToDevice);
    cudaMemcpy(dq, q, sizeof(q), cudaMemcpyHostToDevice);
    cudaMemcpy(dk, knew, sizeof(knew), cudaMemcpyHostToDevice);
    cudaMemcpy(dv, vnew, sizeof(vnew), cudaMemcpyHostToDevice);
    cudaMemcpy(dbt, bt, sizeof(bt), cudaMemcpyHostToDevice);
    cudaMemcpy(dslot, slot, sizeof(slot), cudaMemcpyHostToDevice);
    cudaMemcpy(dql, q_lens, sizeof(q_lens), cudaMemcpyHostToDevice);
    cudaMemcpy(dkl, kv_lens, sizeof(kv_lens), cudaMemcpyHostToDevice);

    tecoopsHandle_t hd;
    tecoopsTensorDescriptor_t btD, qD, cD;
    int bt_dims[2] = {B, PAGES_PER_SEQ}, q_dims[3] = {B, HQ, D}, c_dims[4] = {NB, HKV, BS, D};
    CK(tecoopsCreate(&hd) == TECOOPS_STATUS_SUCCESS);
    CK(tecoopsCreateTensorDescriptor(&btD) == TECOOPS_STATUS_SUCCESS);
    CK(tecoopsCreateTensorDescriptor(&qD) == TECOOPS_STATUS_SUCCESS);
    CK(tecoopsCreateTensorDescriptor(&cD) == TECOOPS_STATUS_SUCCESS);
    CK(tecoopsSetTensorNdDescriptor(btD, TECOOPS_DATA_INT32, 2, bt_dims, NULL) == TECOOPS_STATUS_SUCCESS);
    CK(tecoopsSetTensorNdDescriptor(qD, TECOOPS_DATA_BFLOAT16, 3, q_dims, NULL) == TECOOPS_STATUS_SUCCESS);
    CK(tecoopsSetTensorNdDescriptor(cD, TECOOPS_DATA_BFLOAT16, 4, c_dims, NULL) == TECOOPS_STATUS_SUCCESS);
    CK(tecoopsReshapeAndCache(hd, dk, dv, (const int64_t *)dslot, dkc, dvc, B, HKV, D, NB, BS) ==
       TECOOPS_STATUS_SUCCESS);
    CK(tecoopsFlashAttention(hd, 1, ctx[B - 1] + 1, NB, (const int *)dql, (const int *)dkl, btD, dbt,
                             qD, dq, cD, dkc, cD, dvc, qD, dout, NULL) == TECOOPS_STATUS_SUCCESS);
    int code = -1;
    CK(tecoopsGetDeviceErrorStatus(hd, &code) == TECOOPS_STATUS_SUCCESS && code == 0);
    CK(cudaMemcpy(out, dout, sizeof(out), cudaMemcpyDeviceToHost) == cudaSuccess);

    /* host reference: the new token is attended at position ctx[b] */
    double max_err = 0.0, sum_err = 0.0;
    for (b = 0; b < B; ++b) {
        for (h = 0; h < HQ; ++h) {
            const int kvh = h / (HQ / HKV), S = kv_lens[b];
            float sc[128], m = -INFINITY, l = 0.f, o[D];
            for (j = 0; j < S; ++j) {
                const uint16_t *kr;
                if (j == ctx[b]) {
                    kr = knew + ((size_t)b * HKV + kvh) * D;
                } else {
                    const int pg = bt[b * PAGES_PER_SEQ + j / BS];
                    kr = kc + (((size_t)pg * HKV + kvh) * BS + j % BS) * D;
                }
                float dot = 0.f;
                for (d = 0; d < D; ++d) dot += from_bf16(q[((size_t)b * HQ + h) * D + d]) * from_bf16(kr[d]);
                sc[j] = dot / sqrtf((float)D);
                if (sc[j] > m) m = sc[j];
            }
            for (d = 0; d < D; ++d) o[d] = 0.f;
            for (j = 0; j < S; ++j) {
                const float p = expf(sc[j] - m);
                const uint16_t *vr;
                if (j == ctx[b]) {
                    vr = vnew + ((size_t)b * HKV + kvh) * D;
                } else {
                    const int pg = bt[b * PAGES_PER_SEQ + j / BS];
                    vr = vc + (((size_t)pg * HKV + kvh) * BS + j % BS) * D;
                }
                l += p;
                for (d = 0; d < D; ++d) o[d] += p * from_bf16(vr[d]);
            }
            for (d = 0; d < D; ++d) {
                const double e = fabs((double)from_bf16(out[((size_t)b * HQ + h) * D + d]) - o[d] / l);
                if (e > max_err) max_err = e;
                sum_err += e;
            }
        }
    }
    const double mean_err = sum_err / (B * HQ * D);
    printf("decode step from C: max_abs %.3e mean_abs %.3e\n", max_err, mean_err);
    CK(max_err <= 2e-2 && mean_err <= 2e-3);
    tecoopsDestroyTensorDescriptor(btD);
    tecoopsDestroyTensorDescriptor(qD);
    tecoopsDestroyTensorDescriptor(cD);
    tecoopsDestroy(hd);
    printf("c99 gpu client OK\n");
    return 0;
}
