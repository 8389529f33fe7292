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
// One CTA per page of the compact cache; each thread moves up to 4 chunks of 16 e4m3
// bytes per iteration (one 16-byte load, two 16-byte stores each, all loads first); pages
// past a sequence's kv_len are skipped, block-table entries outside the pool give zeros.
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

// One CTA per (sequence b, page i) of the compact cache: the page's kv_len check and
// block-table entry are read once, then every thread converts its 16-byte chunks of all
// KV heads of the page (K and V) with all its loads in flight before the first store.
template <typename T, int PER>
__global__ void __launch_bounds__(256) kv_dequant_compact_kernel(KvDequantParams p) {
    const int bi = blockIdx.x;                 // b * pages_per_seq + i
    const int b = bi / p.pages_per_seq;
    const int i = bi - b * p.pages_per_seq;
    if (threadIdx.x == 0) p.bt_out[bi] = bi;
    // the length and the block-table entry are loaded together (one round trip)
    const int kv_len = __ldg(p.kv_seq_lens + b);
    const int blk =
        i < p.block_table_dim ? __ldg(p.block_table + (int64_t)b * p.block_table_dim + i) : -1;
    if (i * p.block_size >= kv_len) return;   // past kv_len: not read
    const bool valid = blk >= 0 && blk < p.num_pages;   // ids outside the pool give zeros
    const int dch = p.head_dim / 16;                    // 16-byte e4m3 chunks per row
    const int chunks = p.num_kv_heads * p.block_size * dch;   // per page, per cache
    const uint8_t *kc = static_cast<const uint8_t *>(p.key_cache);
    const uint8_t *vc = static_cast<const uint8_t *>(p.value_cache);
    for (int c0 = threadIdx.x; c0 < chunks; c0 += 256 * PER) {
        uint4 kq[PER], vq[PER];
        int64_t dst[PER];
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            const int c = c0 + u * 256;
            kq[u] = vq[u] = make_uint4(0, 0, 0, 0);
            dst[u] = -1;
            if (c < chunks) {
                // chunk c = (h, row, col / 16) of the page in [Hkv, bs, D] order
                const int h = c / (p.block_size * dch);
                const int rem = c - h * p.block_size * dch;
                const int row = rem / dch;
                const int col = (rem - row * dch) * 16;
                dst[u] = (((int64_t)bi * p.num_kv_heads + h) * p.block_size + row) * p.head_dim +
                         col;
                if (valid) {
                    const int64_t src =
                        p.kv_layout == 0
                            ? (((int64_t)blk * p.num_kv_heads + h) * p.block_size + row) *
                                      p.head_dim + col
                            : (((int64_t)blk * p.block_size + row) * p.num_kv_heads + h) *
                                      p.head_dim + col;
                    kq[u] = __ldg(reinterpret_cast<const uint4 *>(kc + src));
                    vq[u] = __ldg(reinterpret_cast<const uint4 *>(vc + src));
                }
            }
        }
#pragma unroll
        for (int u = 0; u < PER; ++u) {
            if (dst[u] < 0) continue;
            const uint32_t kw[4] = {kq[u].x, kq[u].y, kq[u].z, kq[u].w};
            const uint32_t vw[4] = {vq[u].x, vq[u].y, vq[u].z, vq[u].w};
            uint32_t ko[8], vo[8];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                ko[2 * q] = e4m3x2_scaled<T>(kw[q] & 0xffffu, p.k_scale);
                ko[2 * q + 1] = e4m3x2_scaled<T>(kw[q] >> 16, p.k_scale);
                vo[2 * q] = e4m3x2_scaled<T>(vw[q] & 0xffffu, p.v_scale);
                vo[2 * q + 1] = e4m3x2_scaled<T>(vw[q] >> 16, p.v_scale);
            }
            uint4 *kd = reinterpret_cast<uint4 *>(static_cast<T *>(p.key_out) + dst[u]);
            uint4 *vd = reinterpret_cast<uint4 *>(static_cast<T *>(p.value_out) + dst[u]);
            kd[0] = make_uint4(ko[0], ko[1], ko[2], ko[3]);
            kd[1] = make_uint4(ko[4], ko[5], ko[6], ko[7]);
            vd[0] = make_uint4(vo[0], vo[1], vo[2], vo[3]);
            vd[1] = make_uint4(vo[4], vo[5], vo[6], vo[7]);
        }
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
    (void)num_sms;
    if (p.head_dim % 16 != 0) return cudaErrorInvalidValue;
    const int64_t pages = (int64_t)p.batch * p.pages_per_seq;
    if (pages == 0) return cudaSuccess;
    if (pages > 0x7fffffff) return cudaErrorInvalidValue;
    if (bf16)
        kv_dequant_compact_kernel<__nv_bfloat16, 4><<<(unsigned)pages, 256, 0, stream>>>(p);
    else
        kv_dequant_compact_kernel<__half, 4><<<(unsigned)pages, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace kern
}  // namespace tecoops
