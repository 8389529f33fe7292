// Dequantise-and-compact of an e4m3 paged cache for the tcgen05 prefill.
//
// The prefill kernel contracts 16-bit tiles on the tensor cores.  For an e4m3 cache
// (a tecoopsFlashAttentionEx extension) the pages a batch references are first
// copied into a workspace cache of the query's 16-bit type, value = e4m3 * scale
// (e4m3 is exact in fp16 / bf16, the product is rounded once), laid out
// [batch * pages_per_seq, Hkv, block_size, D] with sequence b's i-th page at
// b * pages_per_seq + i, and a matching block table.  Prefill is compute-bound, so
// this extra pass over the referenced K/V bytes costs a few percent of its time.
//
// One thread per 16 e4m3 bytes (one 16-byte load, two 16-byte stores); pages past a
// sequence's kv_len are skipped, block-table entries outside the pool give zeros.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "ual/kernels/common.cuh"
#include "ual/kernels/launchers.h"

namespace tecoops {
namespace kern {

namespace {

template <typename T>
__device__ __forceinline__ uint32_t e4m3x2_scaled(uint32_t pair, float scale) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)pair, __NV_E4M3);
    const float a = __half2float(__half(__half_raw{h.x})) * scale;
    const float b = __half2float(__half(__half_raw{h.y})) * scale;
    return Elem<T>::pack2(a, b);
}

template <typename T>
__global__ void __launch_bounds__(256) kv_dequant_compact_kernel(KvDequantParams p) {
    // work item: (b, page i, kv head h, 16-byte chunk c) over both caches
    const int chunks = p.block_size * p.head_dim / 16;   // per (page, head)
    const int64_t per_page = (int64_t)p.num_kv_heads * chunks;
    const int64_t per_seq = (int64_t)p.pages_per_seq * per_page;
    const int64_t total = (int64_t)p.batch * per_seq;
    for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < total;
         w += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(w / per_seq);
        int64_t r = w - (int64_t)b * per_seq;
        const int i = (int)(r / per_page);
        r -= (int64_t)i * per_page;
        const int h = (int)(r / chunks);
        const int c = (int)(r - (int64_t)h * chunks);
        if (c == 0 && h == 0) p.bt_out[(int64_t)b * p.pages_per_seq + i] = b * p.pages_per_seq + i;
        if (i * p.block_size >= __ldg(p.kv_seq_lens + b)) continue;   // past kv_len
        const int blk = i < p.block_table_dim ? __ldg(p.block_table + (int64_t)b * p.block_table_dim + i)
                                              : -1;
        // element (row, col) of chunk c: row = c / (D/16), cols 16*(c % (D/16)) ..
        const int row = c / (p.head_dim / 16);
        const int col = (c - row * (p.head_dim / 16)) * 16;
        const int64_t dst = (((int64_t)(b * p.pages_per_seq + i) * p.num_kv_heads + h) *
                                 p.block_size + row) * p.head_dim + col;
        uint4 kq = make_uint4(0, 0, 0, 0), vq = make_uint4(0, 0, 0, 0);
        if (blk >= 0 && blk < p.num_pages) {
            const int64_t src =
                p.kv_layout == 0
                    ? (((int64_t)blk * p.num_kv_heads + h) * p.block_size + row) * p.head_dim + col
                    : (((int64_t)blk * p.block_size + row) * p.num_kv_heads + h) * p.head_dim + col;
            kq = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(p.key_cache) + src));
            vq = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint8_t *>(p.value_cache) + src));
        }
        const uint32_t kw[4] = {kq.x, kq.y, kq.z, kq.w}, vw[4] = {vq.x, vq.y, vq.z, vq.w};
        uint32_t ko[8], vo[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            ko[2 * q] = e4m3x2_scaled<T>(kw[q] & 0xffffu, p.k_scale);
            ko[2 * q + 1] = e4m3x2_scaled<T>(kw[q] >> 16, p.k_scale);
            vo[2 * q] = e4m3x2_scaled<T>(vw[q] & 0xffffu, p.v_scale);
            vo[2 * q + 1] = e4m3x2_scaled<T>(vw[q] >> 16, p.v_scale);
        }
        uint4 *kd = reinterpret_cast<uint4 *>(static_cast<T *>(p.key_out) + dst);
        uint4 *vd = reinterpret_cast<uint4 *>(static_cast<T *>(p.value_out) + dst);
        kd[0] = make_uint4(ko[0], ko[1], ko[2], ko[3]);
        kd[1] = make_uint4(ko[4], ko[5], ko[6], ko[7]);
        vd[0] = make_uint4(vo[0], vo[1], vo[2], vo[3]);
        vd[1] = make_uint4(vo[4], vo[5], vo[6], vo[7]);
    }
}

}  // namespace

size_t kv_dequant_workspace_bytes(int batch, int pages_per_seq, int num_kv_heads, int block_size,
                                  int head_dim) {
    const size_t pages = (size_t)batch * pages_per_seq;
    const size_t cache = pages * num_kv_heads * block_size * head_dim * 2;   // 16-bit
    return 2 * cache + pages * sizeof(int) + 512;
}

cudaError_t launch_kv_dequant(const KvDequantParams &p, bool bf16, int num_sms,
                              cudaStream_t stream) {
    if (p.head_dim % 16 != 0) return cudaErrorInvalidValue;
    const int64_t total = (int64_t)p.batch * p.pages_per_seq * p.num_kv_heads * p.block_size *
                          p.head_dim / 16;
    if (total == 0) return cudaSuccess;
    int64_t grid = (total + 255) / 256;
    const int64_t cap = (int64_t)num_sms * 8;
    if (grid > cap) grid = cap;
    if (bf16)
        kv_dequant_compact_kernel<__nv_bfloat16><<<(unsigned)grid, 256, 0, stream>>>(p);
    else
        kv_dequant_compact_kernel<__half><<<(unsigned)grid, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace kern
}  // namespace tecoops
