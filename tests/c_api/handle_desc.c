/* Plain C99 client of include/tecoops.h: compiled with gcc -std=c99 -pedantic and
 * linked against libteco_ops.so by tests/test_c_header.py.  It exercises the
 * handle, stream and tensor-descriptor API (host only, no GPU needed) and the
 * argument checks of the two hot-path operators, the way a C program written against
 * the reference header (teco/interface/include/tecoops.h) would. */
#include <stdio.h>
#include <string.h>

#include "tecoops.h"

#define CHECK(cond)                                                   \
    do {                                                              \
        if (!(cond)) {                                                \
            fprintf(stderr, "%s:%d: %s\n", __FILE__, __LINE__, #cond); \
            return 1;                                                 \
        }                                                             \
    } while (0)

int main(void) {
    tecoopsHandle_t h = NULL;
    tecoopsTensorDescriptor_t d = NULL;
    sdaaStream_t s = NULL;
    int dims[3] = {5, 4, 128}, got[3] = {0, 0, 0}, strides[3] = {0, 0, 0}, nb = 0;
    tecoopsDataType_t dt = TECOOPS_DATA_FLOAT;

    CHECK(tecoopsCreate(NULL) == TECOOPS_STATUS_BAD_PARAM);
    CHECK(tecoopsCreate(&h) == TECOOPS_STATUS_SUCCESS && h != NULL);
    CHECK(tecoopsSetStream(h, NULL) == TECOOPS_STATUS_SUCCESS);
    CHECK(tecoopsGetStream(h, &s) == TECOOPS_STATUS_SUCCESS && s == NULL);
    CHECK(strcmp(tecoopsGetErrorString(TECOOPS_STATUS_BAD_PARAM), "TECOOPS_STATUS_BAD_PARAM") == 0);

    CHECK(tecoopsCreateTensorDescriptor(&d) == TECOOPS_STATUS_SUCCESS);
    CHECK(tecoopsSetTensorNdDescriptor(d, TECOOPS_DATA_BFLOAT16, 3, dims, NULL) ==
          TECOOPS_STATUS_SUCCESS);
    CHECK(tecoopsGetTensorNdDescriptor(d, 3, &dt, &nb, got, strides) == TECOOPS_STATUS_SUCCESS);
    CHECK(dt == TECOOPS_DATA_BFLOAT16 && nb == 3);
    CHECK(got[0] == 5 && got[1] == 4 && got[2] == 128);
    CHECK(strides[0] == 512 && strides[1] == 128 && strides[2] == 1);
    CHECK(tecoopsSetTensorNdDescriptor(d, TECOOPS_DATA_HALF, 0, dims, NULL) ==
          TECOOPS_STATUS_BAD_PARAM);

    /* argument checks run on the host before anything is launched */
    CHECK(tecoopsReshapeAndCache(NULL, NULL, NULL, NULL, NULL, NULL, 1, 1, 128, 1, 16) ==
          TECOOPS_STATUS_NOT_INITIALIZED);
    CHECK(tecoopsReshapeAndCache(h, NULL, NULL, NULL, NULL, NULL, 1, 1, 128, 1, 16) ==
          TECOOPS_STATUS_BAD_PARAM);
    CHECK(tecoopsFlashAttention(h, 1, 1, 1, NULL, NULL, NULL, NULL, d, NULL, d, NULL, d, NULL, d,
                                NULL, NULL) == TECOOPS_STATUS_BAD_PARAM);

    CHECK(tecoopsDestroyTensorDescriptor(d) == TECOOPS_STATUS_SUCCESS);
    CHECK(tecoopsDestroy(h) == TECOOPS_STATUS_SUCCESS);
    printf("c99 client OK\n");
    return 0;
}
