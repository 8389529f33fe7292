// reshape_and_cache for sm_100a: scatter key/value rows into the paged cache.
//
// Semantics follow the reference kernel
// teco/ual/kernel/reshape_and_cache/reshape_and_cache_fp16.scpp:47-96 and its CPU
// golden test/zoo/teco/reshape_and_cache/reshape_and_cache.cpp:136-147:
//   for token t, slot = slot_mapping[t]; slot < 0 -> skip;
//   blk = slot / block_size, off = slot % block_size;
//   for head h: key_cache[blk][h][off][:] = key[t][h][:]   (same for value)
// The copy is a bit-exact move of 2-byte words.
//
// B200 design: the reference issues 2*H blocking 256-byte DMA copies per token
// on 32 cores.  Here the whole [T, H, D] row space is flattened into 16-byte
// vectors; each thread moves UNROLL vectors of K and of V per iteration with all
// loads issued before any store (memory-level parallelism), loads bypass L1
// (read-once data), consecutive lanes touch consecutive 16-byte pieces of the
// same 256-byte head row, so both the reads and the scattered writes are whole
// 32-byte sectors.  The K/V loads do not wait for the slot_mapping load (only the
// stores need the slot), so a pass costs one DRAM round trip, not two; a launch
// that fits in 8 CTAs of 256 per SM takes one pass with every load in flight at
// once (2 vectors per thread below half that size), larger ones stride over a
// grid of 8 CTAs per SM.  64-bit offsets throughout (caches beyond 2^31
// elements).
//
// Extensions: the cache strides cover both page layouts ([NB, H, bs, D] and
// vLLM's [NB, bs, H, D]); an e4m3 cache stores e4m3(x / scale) with IEEE division
// and round-to-nearest-even, saturated to the finite range (+-448), 16 elements
// per thread (32 bytes read, 16 written).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "ual/args/reshape_and_cache_args.h"

namespace tecoops {
namespace kern {

using ual::args::ReshapeAndCacheArgs;

__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st16(void *p, const uint4 &v) {
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Unsigned 32-bit division by a run-time constant d >= 1 for n < 2^31 (round-up
// reciprocal, Granlund-Montgomery): with s = ceil(log2 d) and
// magic = floor(2^32 (2^s - d) / d) + 1, n / d = (umulhi(n, magic) + n) >> s; the sum
// stays below 2^32 because n < 2^31.
struct FastDiv {
    uint32_t magic, shift, d;
};
static inline FastDiv make_fastdiv(uint32_t d) {
    uint32_t s = 0;
    while (s < 32 && (1ull << s) < d) ++s;
    FastDiv f;
    f.magic = (uint32_t)((((1ull << 32) * ((1ull << s) - d)) / d) + 1);
    f.shift = s;
    f.d = d;
    return f;
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f) {
    return (__umulhi(n, f.magic) + n) >> f.shift;
}

// Vectorised path: head_size*2 bytes is a multiple of 16 and every base pointer
// and token stride is 16-byte aligned; fewer than 2^31 vectors (32-bit indices).
template <int UNROLL>
__global__ void __launch_bounds__(256) reshape_and_cache_vec16_kernel(
    const uint8_t *__restrict__ key, const uint8_t *__restrict__ value,
    const int64_t *__restrict__ slot_mapping, uint8_t *__restrict__ key_cache,
    uint8_t *__restrict__ value_cache, uint32_t total_vecs, FastDiv per_token, FastDiv per_head,
    FastDiv per_block, int64_t num_slots, int64_t key_stride_b, int64_t value_stride_b,
    int64_t block_stride_b, int64_t head_stride_b, int64_t entry_stride_b) {
    const uint32_t step = gridDim.x * blockDim.x;
    for (uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < total_vecs;
         i0 += step * UNROLL) {
        uint4 kv[UNROLL], vv[UNROLL];
        int64_t dst[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            const uint32_t i = i0 + (uint32_t)u * step;
            dst[u] = -1;
            if (i < total_vecs) {
                const uint32_t t = fdiv(i, per_token);
                const uint32_t r = i - t * per_token.d;
                const uint32_t h = fdiv(r, per_head);
                const uint32_t c = r - h * per_head.d;
                const int64_t slot = __ldg(slot_mapping + t);
                // K/V loads independent of the slot: in flight with the slot load
                kv[u] = ld_stream16(key + (int64_t)t * key_stride_b + (int64_t)r * 16);
                vv[u] = ld_stream16(value + (int64_t)t * value_stride_b + (int64_t)r * 16);
                if (slot >= 0 && slot < num_slots) {
                    const uint32_t s32 = (uint32_t)slot;   // num_slots < 2^31 on this path
                    const uint32_t blk = fdiv(s32, per_block);
                    const uint32_t off = s32 - blk * per_block.d;
                    dst[u] = (int64_t)blk * block_stride_b + (int64_t)h * head_stride_b +
                             (int64_t)off * entry_stride_b + (int64_t)c * 16;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
            if (dst[u] >= 0) {
                st16(key_cache + dst[u], kv[u]);
                st16(value_cache + dst[u], vv[u]);
            }
        }
    }
}

// Generic path: any head_size / alignment, 2-byte words.
__global__ void __launch_bounds__(256) reshape_and_cache_u16_kernel(
    const uint16_t *__restrict__ key, const uint16_t *__restrict__ value,
    const int64_t *__restrict__ slot_mapping, uint16_t *__restrict__ key_cache,
    uint16_t *__restrict__ value_cache, int64_t total, int head_size, int heads, int block_size,
    int64_t num_slots, int64_t key_stride, int64_t value_stride, int64_t block_stride,
    int64_t head_stride, int64_t entry_stride) {
    const int64_t per_token = (int64_t)head_size * heads;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / per_token;
        const int r = (int)(i - t * per_token);
        const int h = r / head_size;
        const int d = r - h * head_size;
        const int64_t slot = __ldg(slot_mapping + t);
        if (slot < 0 || slot >= num_slots) continue;
        const int64_t blk = slot / block_size;
        const int64_t off = slot - blk * block_size;
        const int64_t o = blk * block_stride + h * head_stride + off * entry_stride + d;
        key_cache[o] = key[t * key_stride + r];
        value_cache[o] = value[t * value_stride + r];
    }
}

template <typename Tin>
__device__ __forceinline__ float in_to_float(Tin x) {
    if constexpr (std::is_same<Tin, __half>::value)
        return __half2float(x);
    else
        return __bfloat162float(x);
}

// two floats -> e4m3x2 (first value in the low byte), saturating
__device__ __forceinline__ uint32_t e4m3x2(float a, float b) {
    return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}

// 8 consecutive 16-bit inputs (one 16-byte vector) / scale -> 8 e4m3 bytes
template <typename Tin>
__device__ __forceinline__ uint2 quant8(const uint4 &v, float scale) {
    const Tin *e = reinterpret_cast<const Tin *>(&v);
    uint32_t w[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t p0 = e4m3x2(__fdiv_rn(in_to_float(e[4 * i]), scale),
                                   __fdiv_rn(in_to_float(e[4 * i + 1]), scale));
        const uint32_t p1 = e4m3x2(__fdiv_rn(in_to_float(e[4 * i + 2]), scale),
                                   __fdiv_rn(in_to_float(e[4 * i + 3]), scale));
        w[i] = p0 | (p1 << 16);
    }
    return make_uint2(w[0], w[1]);
}

// e4m3 cache, vectorised: one unit = 16 elements of one (token, head) row.
// Strides: key/value in elements (16-bit), cache in bytes.
template <typename Tin>
__global__ void __launch_bounds__(256) reshape_and_cache_fp8_kernel(
    const uint8_t *__restrict__ key, const uint8_t *__restrict__ value,
    const int64_t *__restrict__ slot_mapping, uint8_t *__restrict__ key_cache,
    uint8_t *__restrict__ value_cache, int64_t total_units, int units_per_head, int heads,
    int block_size, int64_t num_slots, int64_t key_stride, int64_t value_stride,
    int64_t block_stride, int64_t head_stride, int64_t entry_stride, float k_scale,
    float v_scale) {
    const int64_t units_per_token = (int64_t)units_per_head * heads;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total_units;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / units_per_token;
        const int r = (int)(i - t * units_per_token);
        const int h = r / units_per_head;
        const int c = r - h * units_per_head;
        const int64_t slot = __ldg(slot_mapping + t);
        if (slot < 0 || slot >= num_slots) continue;
        const int64_t blk = slot / block_size;
        const int64_t off = slot - blk * block_size;
        const int64_t dst = blk * block_stride + h * head_stride + off * entry_stride + c * 16;
        const uint8_t *kp = key + (t * key_stride + (int64_t)r * 16) * 2;
        const uint8_t *vp = value + (t * value_stride + (int64_t)r * 16) * 2;
        const uint2 k0 = quant8<Tin>(ld_stream16(kp), k_scale);
        const uint2 k1 = quant8<Tin>(ld_stream16(kp + 16), k_scale);
        const uint2 v0 = quant8<Tin>(ld_stream16(vp), v_scale);
        const uint2 v1 = quant8<Tin>(ld_stream16(vp + 16), v_scale);
        st16(key_cache + dst, make_uint4(k0.x, k0.y, k1.x, k1.y));
        st16(value_cache + dst, make_uint4(v0.x, v0.y, v1.x, v1.y));
    }
}

// e4m3 cache, any head_size / alignment: one element per thread
template <typename Tin>
__global__ void __launch_bounds__(256) reshape_and_cache_fp8_scalar_kernel(
    const Tin *__restrict__ key, const Tin *__restrict__ value,
    const int64_t *__restrict__ slot_mapping, uint8_t *__restrict__ key_cache,
    uint8_t *__restrict__ value_cache, int64_t total, int head_size, int heads, int block_size,
    int64_t num_slots, int64_t key_stride, int64_t value_stride, int64_t block_stride,
    int64_t head_stride, int64_t entry_stride, float k_scale, float v_scale) {
    const int64_t per_token = (int64_t)head_size * heads;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / per_token;
        const int r = (int)(i - t * per_token);
        const int h = r / head_size;
        const int d = r - h * head_size;
        const int64_t slot = __ldg(slot_mapping + t);
        if (slot < 0 || slot >= num_slots) continue;
        const int64_t blk = slot / block_size;
        const int64_t off = slot - blk * block_size;
        const int64_t o = blk * block_stride + h * head_stride + off * entry_stride + d;
        key_cache[o] = (uint8_t)(e4m3x2(__fdiv_rn(in_to_float(key[t * key_stride + r]), k_scale),
                                        0.f) & 0xffu);
        value_cache[o] = (uint8_t)(
            e4m3x2(__fdiv_rn(in_to_float(value[t * value_stride + r]), v_scale), 0.f) & 0xffu);
    }
}

static inline bool aligned16(const void *p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

static cudaError_t launch_fp8(const ReshapeAndCacheArgs &a, int num_sms, cudaStream_t stream) {
    const int64_t num_slots = (int64_t)a.num_blocks * a.block_size;
    const float ks = a.k_scale > 0.f ? a.k_scale : 1.f, vs = a.v_scale > 0.f ? a.v_scale : 1.f;
    const bool vec = (a.size_per_head % 16 == 0) && aligned16(a.key) && aligned16(a.value) &&
                     aligned16(a.key_cache) && aligned16(a.value_cache) &&
                     ((a.key_stride * 2) % 16 == 0) && ((a.value_stride * 2) % 16 == 0) &&
                     (a.block_stride % 16 == 0) && (a.head_stride % 16 == 0) &&
                     (a.entry_stride % 16 == 0);
    const int64_t cap = (int64_t)num_sms * 8;
    if (vec) {
        const int uph = a.size_per_head / 16;
        const int64_t total = (int64_t)a.num_tokens * a.num_kv_heads * uph;
        int64_t grid = (total + 255) / 256;
        if (grid > cap) grid = cap;
        auto kfn = a.cache_fp8 == 2 ? reshape_and_cache_fp8_kernel<__nv_bfloat16>
                                    : reshape_and_cache_fp8_kernel<__half>;
        kfn<<<(unsigned)grid, 256, 0, stream>>>(
            static_cast<const uint8_t *>(a.key), static_cast<const uint8_t *>(a.value),
            a.slot_mapping, static_cast<uint8_t *>(a.key_cache),
            static_cast<uint8_t *>(a.value_cache), total, uph, a.num_kv_heads, a.block_size,
            num_slots, a.key_stride, a.value_stride, a.block_stride, a.head_stride,
            a.entry_stride, ks, vs);
    } else {
        const int64_t total = (int64_t)a.num_tokens * a.num_kv_heads * a.size_per_head;
        int64_t grid = (total + 255) / 256;
        if (grid > cap) grid = cap;
        if (a.cache_fp8 == 2)
            reshape_and_cache_fp8_scalar_kernel<__nv_bfloat16><<<(unsigned)grid, 256, 0, stream>>>(
                static_cast<const __nv_bfloat16 *>(a.key),
                static_cast<const __nv_bfloat16 *>(a.value), a.slot_mapping,
                static_cast<uint8_t *>(a.key_cache), static_cast<uint8_t *>(a.value_cache), total,
                a.size_per_head, a.num_kv_heads, a.block_size, num_slots, a.key_stride,
                a.value_stride, a.block_stride, a.head_stride, a.entry_stride, ks, vs);
        else
            reshape_and_cache_fp8_scalar_kernel<__half><<<(unsigned)grid, 256, 0, stream>>>(
                static_cast<const __half *>(a.key), static_cast<const __half *>(a.value),
                a.slot_mapping, static_cast<uint8_t *>(a.key_cache),
                static_cast<uint8_t *>(a.value_cache), total, a.size_per_head, a.num_kv_heads,
                a.block_size, num_slots, a.key_stride, a.value_stride, a.block_stride,
                a.head_stride, a.entry_stride, ks, vs);
    }
    return cudaGetLastError();
}

cudaError_t launch_reshape_and_cache(const ReshapeAndCacheArgs &a, int num_sms,
                                     cudaStream_t stream) {
    if (a.num_tokens <= 0) return cudaSuccess;
    if (a.cache_fp8) return launch_fp8(a, num_sms, stream);
    const int eb = a.elem_bytes;
    const int64_t num_slots = (int64_t)a.num_blocks * a.block_size;
    const int row_bytes = a.size_per_head * eb;
    const bool vec = (row_bytes % 16 == 0) && aligned16(a.key) && aligned16(a.value) &&
                     aligned16(a.key_cache) && aligned16(a.value_cache) &&
                     ((a.key_stride * eb) % 16 == 0) && ((a.value_stride * eb) % 16 == 0);
    const int64_t total_vec = vec ? (int64_t)a.num_tokens * a.num_kv_heads * (row_bytes / 16) : 0;
    if (vec && total_vec < (1ll << 31) && num_slots < (1ll << 31)) {
        const int vecs_per_head = row_bytes / 16;
        const uint32_t total = (uint32_t)total_vec;
        const int threads = 256;
        // resident CTAs per SM of each instantiation (register-limited), looked up once
        static int resident[2] = {0, 0};
        if (resident[0] == 0) {
            int r2 = 0, r4 = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r2, reshape_and_cache_vec16_kernel<2>,
                                                          threads, 0);
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r4, reshape_and_cache_vec16_kernel<4>,
                                                          threads, 0);
            resident[0] = r2 > 0 ? r2 : 4;
            resident[1] = r4 > 0 ? r4 : 4;
        }
        // one pass with every load in flight when the launch fits the resident CTAs:
        // 2 vectors per thread below half of that, 4 otherwise; larger T strides over
        // exactly the resident grid
        const int64_t cap2 = (int64_t)num_sms * resident[0];
        const int64_t cap4 = (int64_t)num_sms * resident[1];
        const bool small = total <= cap2 * threads * 2;
        const int unroll = small ? 2 : 4;
        const int64_t cap = small ? cap2 : cap4;
        const int64_t want = ((int64_t)total + (int64_t)threads * unroll - 1) /
                             ((int64_t)threads * unroll);
        const int64_t grid = want < 1 ? 1 : (want < cap ? want : cap);
        auto kfn = small ? reshape_and_cache_vec16_kernel<2> : reshape_and_cache_vec16_kernel<4>;
        kfn<<<(unsigned)grid, threads, 0, stream>>>(
            static_cast<const uint8_t *>(a.key), static_cast<const uint8_t *>(a.value),
            a.slot_mapping, static_cast<uint8_t *>(a.key_cache),
            static_cast<uint8_t *>(a.value_cache), total,
            make_fastdiv((uint32_t)(vecs_per_head * a.num_kv_heads)),
            make_fastdiv((uint32_t)vecs_per_head), make_fastdiv((uint32_t)a.block_size),
            num_slots, a.key_stride * eb, a.value_stride * eb, a.block_stride * eb,
            a.head_stride * eb, a.entry_stride * eb);
    } else {
        const int64_t total = (int64_t)a.num_tokens * a.num_kv_heads * a.size_per_head;
        int64_t grid = (total + 255) / 256;
        const int64_t cap = (int64_t)num_sms * 8;
        if (grid > cap) grid = cap;
        reshape_and_cache_u16_kernel<<<(unsigned)grid, 256, 0, stream>>>(
            static_cast<const uint16_t *>(a.key), static_cast<const uint16_t *>(a.value),
            a.slot_mapping, static_cast<uint16_t *>(a.key_cache),
            static_cast<uint16_t *>(a.value_cache), total, a.size_per_head, a.num_kv_heads,
            a.block_size, num_slots, a.key_stride, a.value_stride, a.block_stride,
            a.head_stride, a.entry_stride);
    }
    return cudaGetLastError();
}

}  // namespace kern
}  // namespace tecoops
