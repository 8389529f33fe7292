// Device helpers shared by the attention kernels: 2-byte element traits,
// warp-level MMA / ldmatrix wrappers, cp.async with zero fill, and the
// per-sequence start offset computed from the device array of lengths.
#ifndef TECOOPS_B200_UAL_KERNELS_COMMON_CUH_
#define TECOOPS_B200_UAL_KERNELS_COMMON_CUH_

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace tecoops {
namespace kern {

// ---- element traits ---------------------------------------------------------
template <typename T>
struct Elem;

template <>
struct Elem<__half> {
    static __device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
    static __device__ __forceinline__ uint32_t pack2(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    }
    static __device__ __forceinline__ __half from_float(float x) { return __float2half_rn(x); }
    static __device__ __forceinline__ float2 unpack2(uint32_t u) {
        __half2 h = *reinterpret_cast<__half2 *>(&u);
        return __half22float2(h);
    }
};

template <>
struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_float(__nv_bfloat16 x) {
        return __bfloat162float(x);
    }
    static __device__ __forceinline__ uint32_t pack2(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t *>(&h);
    }
    static __device__ __forceinline__ __nv_bfloat16 from_float(float x) {
        return __float2bfloat16_rn(x);
    }
    static __device__ __forceinline__ float2 unpack2(uint32_t u) {
        __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162 *>(&u);
        return __bfloat1622float2(h);
    }
};

// ---- warp MMA m16n8k16, fp32 accumulate --------------------------------------
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4],
                                                 uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// 16-byte cp.async (L2 only); src_bytes == 0 zero-fills the destination.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

// Start row of sequence `b` in the packed varlen Q/O tensors:
// sum(q_seq_lens[0:b]).  Whole-warp cooperative; every lane gets the result.
__device__ __forceinline__ int warp_seq_start(const int *__restrict__ lens, int b) {
    const int lane = threadIdx.x & 31;
    int acc = 0;
    for (int i = lane; i < b; i += 32) acc += __ldg(lens + i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

}  // namespace kern
}  // namespace tecoops

#endif  // TECOOPS_B200_UAL_KERNELS_COMMON_CUH_
