// Shape-generic paged attention (any head_dim <= 256, any block_size, any GQA
// ratio).  It serves shapes the tuned kernels do not cover (block_size not a
// multiple of 16, head_dim outside {64, 128}); it is a GPU kernel, not a
// host fallback.
//
// Semantics: reference golden test/zoo/teco/flash_attention/flash_attention.py:79-140
// (bottom-right causal: row i of a sequence with q_len L and kv_len S attends keys
// j <= S - L + i; scale 1/sqrt(D); q head h reads kv head h / (Hq/Hkv)).
//
// One warp per (query row, q head).  Keys are taken 32 at a time, one key per
// lane for the dot product, then the lanes switch to owning head dimensions for
// the P.V accumulation; online softmax in the exp2 domain.  The options of
// tecoopsFlashAttentionEx (scale, causal, window, log-sum-exp output) bound the
// key range [lo, end) of each row.  Caches in either page layout, 16-bit or e4m3
// (dequantised with k_scale / v_scale).
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <type_traits>

#include "ual/kernels/common.cuh"
#include "ual/kernels/launchers.h"

namespace tecoops {
namespace kern {

// cache element -> float (e4m3: exact via f16, times the scale)
template <typename T, typename C>
__device__ __forceinline__ float cache_to_float(C x, float scale) {
    if constexpr (std::is_same<C, uint8_t>::value) {
        const __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)x, __NV_E4M3);
        return __half2float(__half(h)) * scale;
    } else {
        (void)scale;
        return Elem<T>::to_float(x);
    }
}

template <typename T, typename C>
__global__ void __launch_bounds__(128) fa_generic_kernel(AttnShape s) {
    constexpr int kMaxD = 256;
    __shared__ float qs[4][kMaxD];
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t pair = (int64_t)blockIdx.x * 4 + warp;
    if (pair >= (int64_t)s.total_q * s.num_heads) return;
    const int row = (int)(pair / s.num_heads);
    const int h = (int)(pair - (int64_t)row * s.num_heads);
    const int D = s.head_dim;

    // locate the sequence of this row
    int b = 0, start = 0;
    for (; b < s.batch; ++b) {
        const int L = __ldg(s.q_seq_lens + b);
        if (row < start + L) break;
        start += L;
    }
    T *out = static_cast<T *>(s.out) + ((int64_t)row * s.num_heads + h) * D;
    if (b >= s.batch) {   // row beyond sum(q_seq_lens): leave zeros
        for (int d = lane; d < D; d += 32) out[d] = Elem<T>::from_float(0.f);
        if (s.lse != nullptr && lane == 0) s.lse[(int64_t)h * s.total_q + row] = -INFINITY;
        return;
    }
    const int L = __ldg(s.q_seq_lens + b);
    const int S = __ldg(s.kv_seq_lens + b);
    const int i = row - start;
    const int off = S - L;
    // admissible keys [lo, end)
    int end = s.causal ? off + i + 1 : (s.window_right >= 0 ? off + i + s.window_right + 1 : S);
    if (end > S) end = S;
    const int lo = s.window_left >= 0 ? max(0, off + i - s.window_left) : 0;
    const int kvh = h / (s.num_heads / s.num_kv_heads);

    const T *q = static_cast<const T *>(s.q) + ((int64_t)row * s.num_heads + h) * D;
    for (int d = lane; d < D; d += 32) qs[warp][d] = Elem<T>::to_float(q[d]);
    __syncwarp();

    const C *kc = static_cast<const C *>(s.key_cache);
    const C *vc = static_cast<const C *>(s.value_cache);
    const int *bt = s.block_table + (int64_t)b * s.block_table_dim;
    const int64_t page_stride = (int64_t)s.num_kv_heads * s.block_size * D;
    // [pages, Hkv, bs, D] or [pages, bs, Hkv, D]
    const int64_t head_off = s.kv_layout == 0 ? (int64_t)kvh * s.block_size * D : (int64_t)kvh * D;
    const int64_t row_stride = s.kv_layout == 0 ? D : (int64_t)s.num_kv_heads * D;
    const float ks = s.cache_fp8 ? s.k_scale : 1.f, vs = s.cache_fp8 ? s.v_scale : 1.f;

    float m = -INFINITY, l = 0.f;
    float acc[kMaxD / 32];
#pragma unroll
    for (int k = 0; k < kMaxD / 32; ++k) acc[k] = 0.f;

    for (int j0 = lo; j0 < end; j0 += 32) {
        const int j = j0 + lane;
        float x = -INFINITY;
        int64_t my_off = 0;
        if (j < end) {
            int blk = __ldg(bt + j / s.block_size);
            if (blk < 0 || blk >= s.num_pages) blk = 0;   // bad page id: stay in bounds
            my_off = (int64_t)blk * page_stride + head_off + (int64_t)(j % s.block_size) * row_stride;
            float dot = 0.f;
            for (int d = 0; d < D; ++d) dot += qs[warp][d] * cache_to_float<T>(kc[my_off + d], ks);
            x = dot * s.scale_log2;
        }
        float cm = x;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
        const float m_new = fmaxf(m, cm);
        const float alpha = exp2f(m - m_new);
        const float pj = (j < end) ? exp2f(x - m_new) : 0.f;
        float ps = pj;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        l = l * alpha + ps;
        m = m_new;
#pragma unroll
        for (int k = 0; k < kMaxD / 32; ++k) acc[k] *= alpha;
        const int nvalid = min(32, end - j0);
        for (int t = 0; t < nvalid; ++t) {
            const float pt = __shfl_sync(0xffffffffu, pj, t);
            const int64_t off = __shfl_sync(0xffffffffu, my_off, t);
#pragma unroll
            for (int k = 0; k < kMaxD / 32; ++k) {
                const int d = lane + 32 * k;
                if (d < D) acc[k] += pt * cache_to_float<T>(vc[off + d], vs);
            }
        }
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
    if (s.lse != nullptr && lane == 0)
        s.lse[(int64_t)h * s.total_q + row] = l > 0.f ? (m + log2f(l)) * 0.6931471805599453f
                                                      : -INFINITY;
#pragma unroll
    for (int k = 0; k < kMaxD / 32; ++k) {
        const int d = lane + 32 * k;
        if (d < D) out[d] = Elem<T>::from_float(acc[k] * inv);
    }
}

cudaError_t launch_generic_attention(const AttnShape &s, bool bf16, cudaStream_t stream) {
    if (s.head_dim > 256 || s.head_dim <= 0) return cudaErrorInvalidValue;
    const int64_t pairs = (int64_t)s.total_q * s.num_heads;
    if (pairs == 0) return cudaSuccess;
    const unsigned grid = (unsigned)((pairs + 3) / 4);
    if (s.cache_fp8) {
        if (bf16)
            fa_generic_kernel<__nv_bfloat16, uint8_t><<<grid, 128, 0, stream>>>(s);
        else
            fa_generic_kernel<__half, uint8_t><<<grid, 128, 0, stream>>>(s);
    } else if (bf16) {
        fa_generic_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 128, 0, stream>>>(s);
    } else {
        fa_generic_kernel<__half, __half><<<grid, 128, 0, stream>>>(s);
    }
    return cudaGetLastError();
}

}  // namespace kern
}  // namespace tecoops
