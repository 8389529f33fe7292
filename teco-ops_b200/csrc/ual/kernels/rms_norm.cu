// rms_norm (optionally fused with the residual add) for sm_100a.
//
// Semantics: reference kernel teco/ual/kernel/rms_norm/rms_norm_fp16.scpp and its
// CPU golden test/zoo/teco/rms_norm/rms_norm.cpp (cpuCompute):
//   without residual: y = x * rstd * w,      rstd = 1 / sqrt(sum(x^2) / D + eps)
//   with residual:    h = x + r (fp32), residual_out = round(h),
//                     rstd from sum(h^2) of the unrounded h,
//                     y = float(round(h)) * rstd * w
// all arithmetic in fp32, one rounding to the 16-bit type per stored value.
//
// B200 design: bandwidth-bound (2 or 4 row passes of 2 bytes per element).  Each
// row is read once: its 16-byte vectors stay in registers between the sum of
// squares and the scaling, so DRAM traffic is exactly the algorithmic bytes.
//   hidden_size <= 2048: one warp per row, 8 rows per 256-thread CTA;
//   larger: one 256-thread CTA per row (warp sums combined through shared memory);
//   hidden_size not a multiple of 8 or unaligned rows: a scalar two-pass kernel.
// Loads of x / r bypass L1 (read once); the weight vector is read through the
// read-only path and stays in L1/L2 across rows.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "ual/args/rms_norm_args.h"
#include "ual/kernels/common.cuh"

namespace tecoops {
namespace kern {

using ual::args::ElemType;
using ual::args::RmsNormArgs;

namespace {

__device__ __forceinline__ uint4 ld_once16(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const T *e = reinterpret_cast<const T *>(&w[i]);
        f[2 * i] = Elem<T>::to_float(e[0]);
        f[2 * i + 1] = Elem<T>::to_float(e[1]);
    }
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    return make_uint4(Elem<T>::pack2(f[0], f[1]), Elem<T>::pack2(f[2], f[3]),
                      Elem<T>::pack2(f[4], f[5]), Elem<T>::pack2(f[6], f[7]));
}

template <typename T>
__device__ __forceinline__ float round_trip(float x) {
    return Elem<T>::to_float(Elem<T>::from_float(x));
}

__device__ __forceinline__ float warp_sum(float s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}

// One row held in registers as VPT 16-byte vectors per thread; THREADS threads
// (32: a warp per row; 256: a CTA per row) share the row.
template <typename T, int VPT, int THREADS, bool RES>
__device__ __forceinline__ void row_norm(const RmsNormArgs &a, int row, int t) {
    const int D = a.hidden_size;
    const int nvec = D >> 3;
    const T *x = static_cast<const T *>(a.input) + (int64_t)row * a.stride;
    const T *r = RES ? static_cast<const T *>(a.residual) + (int64_t)row * D : nullptr;
    float h[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int v = t + i * THREADS;
        if (v < nvec) {
            unpack8<T>(ld_once16(x + v * 8), h[i]);
            if (RES) {
                float rr[8];
                unpack8<T>(ld_once16(r + v * 8), rr);
#pragma unroll
                for (int e = 0; e < 8; ++e) h[i][e] += rr[e];
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) ss += h[i][e] * h[i][e];
        }
    }
    ss = warp_sum(ss);
    if (THREADS > 32) {
        __shared__ float part[THREADS / 32];
        __syncthreads();   // a previous row's readers are done with `part`
        if ((t & 31) == 0) part[t >> 5] = ss;
        __syncthreads();
        ss = 0.f;
#pragma unroll
        for (int w = 0; w < THREADS / 32; ++w) ss += part[w];
    }
    const float rstd = 1.0f / sqrtf(ss / (float)D + a.eps);
    T *y = static_cast<T *>(a.output) + (int64_t)row * D;
    T *ro = RES ? static_cast<T *>(a.residual_out) + (int64_t)row * D : nullptr;
    const T *w = static_cast<const T *>(a.weight);
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
        const int v = t + i * THREADS;
        if (v < nvec) {
            float wf[8], o[8];
            unpack8<T>(__ldg(reinterpret_cast<const uint4 *>(w) + v), wf);
            if (RES) {
                const uint4 hp = pack8<T>(h[i]);
                *reinterpret_cast<uint4 *>(ro + v * 8) = hp;
                unpack8<T>(hp, h[i]);   // the output uses the rounded residual sum
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = h[i][e] * rstd * wf[e];
            *reinterpret_cast<uint4 *>(y + v * 8) = pack8<T>(o);
        }
    }
}

template <typename T, int VPT, bool RES>
__global__ void __launch_bounds__(256) rms_norm_warp_kernel(RmsNormArgs a) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= a.num_tokens) return;
    row_norm<T, VPT, 32, RES>(a, row, threadIdx.x & 31);
}

// CTA per row, software-pipelined over the CTA's rows: the raw vectors of the next row
// are loaded before this row's block-wide sum, so their DRAM latency overlaps the
// reduction barrier and the stores instead of following them.
template <typename T, int VPT, bool RES>
__global__ void __launch_bounds__(256) rms_norm_cta_kernel(RmsNormArgs a) {
    const int t = threadIdx.x;
    const int D = a.hidden_size;
    const int nvec = D >> 3;
    __shared__ float part[8];
    uint4 xr[VPT], rr[VPT];
    auto load_row = [&](int row) {
        const T *x = static_cast<const T *>(a.input) + (int64_t)row * a.stride;
        const T *r = RES ? static_cast<const T *>(a.residual) + (int64_t)row * D : nullptr;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int v = t + i * 256;
            if (v < nvec) {
                xr[i] = ld_once16(x + v * 8);
                if (RES) rr[i] = ld_once16(r + v * 8);
            }
        }
    };
    int row = blockIdx.x;
    if (row < a.num_tokens) load_row(row);
    for (; row < a.num_tokens; row += gridDim.x) {
        float h[VPT][8];
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            if (t + i * 256 < nvec) {
                unpack8<T>(xr[i], h[i]);
                if (RES) {
                    float rf[8];
                    unpack8<T>(rr[i], rf);
#pragma unroll
                    for (int e = 0; e < 8; ++e) h[i][e] += rf[e];
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) ss += h[i][e] * h[i][e];
            }
        }
        const int next = row + (int)gridDim.x;
        if (next < a.num_tokens) load_row(next);   // in flight during the sum and stores
        ss = warp_sum(ss);
        __syncthreads();   // the previous row's readers are done with `part`
        if ((t & 31) == 0) part[t >> 5] = ss;
        __syncthreads();
        ss = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) ss += part[w];
        const float rstd = 1.0f / sqrtf(ss / (float)D + a.eps);
        T *y = static_cast<T *>(a.output) + (int64_t)row * D;
        T *ro = RES ? static_cast<T *>(a.residual_out) + (int64_t)row * D : nullptr;
        const uint4 *w = reinterpret_cast<const uint4 *>(a.weight);
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
            const int v = t + i * 256;
            if (v < nvec) {
                float wf[8], o[8];
                unpack8<T>(__ldg(w + v), wf);
                if (RES) {
                    const uint4 hp = pack8<T>(h[i]);
                    *reinterpret_cast<uint4 *>(ro + v * 8) = hp;
                    unpack8<T>(hp, h[i]);   // the output uses the rounded residual sum
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] = h[i][e] * rstd * wf[e];
                *reinterpret_cast<uint4 *>(y + v * 8) = pack8<T>(o);
            }
        }
    }
}

// any hidden_size / alignment: two passes over global memory, CTA per row
template <typename T>
__global__ void __launch_bounds__(256) rms_norm_scalar_kernel(RmsNormArgs a) {
    __shared__ float part[8];
    const int D = a.hidden_size;
    const bool res = a.residual != nullptr;
    for (int row = blockIdx.x; row < a.num_tokens; row += gridDim.x) {
        const T *x = static_cast<const T *>(a.input) + (int64_t)row * a.stride;
        const T *r = res ? static_cast<const T *>(a.residual) + (int64_t)row * D : nullptr;
        float ss = 0.f;
        for (int d = threadIdx.x; d < D; d += 256) {
            float hv = Elem<T>::to_float(x[d]);
            if (res) hv += Elem<T>::to_float(r[d]);
            ss += hv * hv;
        }
        ss = warp_sum(ss);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
        __syncthreads();
        ss = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) ss += part[w];
        const float rstd = 1.0f / sqrtf(ss / (float)D + a.eps);
        T *y = static_cast<T *>(a.output) + (int64_t)row * D;
        const T *w = static_cast<const T *>(a.weight);
        for (int d = threadIdx.x; d < D; d += 256) {
            float hv = Elem<T>::to_float(x[d]);
            if (res) {
                hv = round_trip<T>(hv + Elem<T>::to_float(r[d]));
                static_cast<T *>(a.residual_out)[(int64_t)row * D + d] = Elem<T>::from_float(hv);
            }
            y[d] = Elem<T>::from_float(hv * rstd * Elem<T>::to_float(w[d]));
        }
    }
}

inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T, bool RES>
cudaError_t launch_t(const RmsNormArgs &a, cudaStream_t stream) {
    const int D = a.hidden_size;
    const bool vec = D % 8 == 0 && a.stride % 8 == 0 && al16(a.input) && al16(a.weight) &&
                     al16(a.output) && (!RES || (al16(a.residual) && al16(a.residual_out)));
    const int nvec = D / 8;
    if (vec && nvec <= 32 * 8) {   // warp per row
        const unsigned grid = (unsigned)((a.num_tokens + 7) / 8);
        if (nvec <= 32)
            rms_norm_warp_kernel<T, 1, RES><<<grid, 256, 0, stream>>>(a);
        else if (nvec <= 64)
            rms_norm_warp_kernel<T, 2, RES><<<grid, 256, 0, stream>>>(a);
        else if (nvec <= 128)
            rms_norm_warp_kernel<T, 4, RES><<<grid, 256, 0, stream>>>(a);
        else
            rms_norm_warp_kernel<T, 8, RES><<<grid, 256, 0, stream>>>(a);
        return cudaGetLastError();
    }
    int64_t cap = (int64_t)a.num_sms * 8;
    const unsigned grid = (unsigned)(a.num_tokens < cap ? a.num_tokens : cap);
    if (vec && nvec <= 256 * 8) {   // CTA per row, up to 16384 columns
        if (nvec <= 256 * 2)
            rms_norm_cta_kernel<T, 2, RES><<<grid, 256, 0, stream>>>(a);
        else if (nvec <= 256 * 4)
            rms_norm_cta_kernel<T, 4, RES><<<grid, 256, 0, stream>>>(a);
        else
            rms_norm_cta_kernel<T, 8, RES><<<grid, 256, 0, stream>>>(a);
        return cudaGetLastError();
    }
    rms_norm_scalar_kernel<T><<<grid, 256, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_rms_norm(const RmsNormArgs &a, cudaStream_t stream) {
    if (a.num_tokens <= 0) return cudaSuccess;
    const bool res = a.residual != nullptr;
    if (a.dtype == ElemType::BF16)
        return res ? launch_t<__nv_bfloat16, true>(a, stream)
                   : launch_t<__nv_bfloat16, false>(a, stream);
    return res ? launch_t<__half, true>(a, stream) : launch_t<__half, false>(a, stream);
}

}  // namespace kern
}  // namespace tecoops
