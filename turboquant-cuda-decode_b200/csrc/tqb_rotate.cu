// tqb_rotate.cu — query rotation prologue of the decode path.
//
// q_rot[b, h, :] = float(q[b, h, :]) @ R, R = Pi^T a [D, D] fp32 matrix, in
// one kernel: the reference launcher does it as a cast plus a cuBLAS fp32
// GEMM plus a copy (reference/soa_decode_v1.py:535-538).  The rows are
// independent 128-deep dot products: CUDA-core FMAs, fp32 accumulation in k
// order (the GEMM is 64 MFLOP at the c1 shape; the launch and the round trip
// of q through HBM, not the arithmetic, are what the fused kernel saves).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tqb_common.cuh"
#include "tqb_internal.h"

namespace tqb {

namespace {

constexpr int kRotRows = 16;                 // query rows per CTA
constexpr int kRotThreads = 256;             // output dim j = t % 128, rows (t / 128) * 8 .. + 7
constexpr int kRotSmem = (kHeadDim * kHeadDim + kRotRows * kHeadDim) * 4;  // R + rows: 72 KB

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

// CTA: kRotRows rows r = b * Hq + h.  R (64 KB) and the rows are staged in
// shared memory with every load in flight at once; thread t then computes
// output dim t % 128 of 8 rows (R read conflict-free, the rows as broadcast
// float4).
template <typename T>
__global__ void __launch_bounds__(kRotThreads) rotate_kernel(const RotateParams P) {
    extern __shared__ __align__(16) float rsm[];
    float* Rs = rsm;                          // [128][128]
    float* qs = rsm + kHeadDim * kHeadDim;    // [kRotRows][128]
    const int t = threadIdx.x;
    const int64_t rows = (int64_t)P.B * P.Hq;
    const int64_t r0 = (int64_t)blockIdx.x * kRotRows;
    const float4* R4 = reinterpret_cast<const float4*>(P.rot);
#pragma unroll
    for (int e = t; e < kHeadDim * kHeadDim / 4; e += kRotThreads)
        reinterpret_cast<float4*>(Rs)[e] = __ldg(R4 + e);
    const T* q = static_cast<const T*>(P.q);
#pragma unroll
    for (int e = t; e < kRotRows * kHeadDim; e += kRotThreads) {
        const int i = e / kHeadDim, d = e % kHeadDim;
        const int64_t r = r0 + i;
        float v = 0.0f;
        if (r < rows) {
            const int64_t b = r / P.Hq, h = r % P.Hq;
            v = to_f32<T>(q[b * P.qsb + h * P.qsh + d]);
        }
        qs[e] = v;
    }
    __syncthreads();
    const int j = t % kHeadDim, i0 = (t / kHeadDim) * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; i++) acc[i] = 0.0f;
#pragma unroll 2
    for (int k0 = 0; k0 < kHeadDim; k0 += 4) {
        const float r0k = Rs[(k0 + 0) * kHeadDim + j], r1k = Rs[(k0 + 1) * kHeadDim + j];
        const float r2k = Rs[(k0 + 2) * kHeadDim + j], r3k = Rs[(k0 + 3) * kHeadDim + j];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 x = *reinterpret_cast<const float4*>(qs + (i0 + i) * kHeadDim + k0);
            acc[i] = fmaf(x.x, r0k, acc[i]);
            acc[i] = fmaf(x.y, r1k, acc[i]);
            acc[i] = fmaf(x.z, r2k, acc[i]);
            acc[i] = fmaf(x.w, r3k, acc[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int64_t r = r0 + i0 + i;
        if (r < rows) {
            const int64_t b = r / P.Hq, h = r % P.Hq;
            P.out[b * P.osb + h * P.osh + j] = acc[i];
        }
    }
}

}  // namespace

template <typename T>
static int launch_rotate_t(const RotateParams& P, int64_t grid, cudaStream_t stream) {
    auto kern = rotate_kernel<T>;
    // 72 KB of dynamic shared memory: opt in on each device this thread uses
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kRotSmem) != cudaSuccess)
            return report_launch(cudaGetLastError());
        configured_dev = dev;
    }
    kern<<<(unsigned)grid, kRotThreads, kRotSmem, stream>>>(P);
    return report_launch(cudaGetLastError());
}

int launch_rotate(const RotateParams& P, cudaStream_t stream) {
    const int64_t rows = (int64_t)P.B * P.Hq;
    if (rows == 0) return TQB_OK;
    const int64_t grid = (rows + kRotRows - 1) / kRotRows;
    switch (P.dtype) {
        case TQB_DTYPE_F32: return launch_rotate_t<float>(P, grid, stream);
        case TQB_DTYPE_F16: return launch_rotate_t<__half>(P, grid, stream);
        case TQB_DTYPE_BF16: return launch_rotate_t<__nv_bfloat16>(P, grid, stream);
        default: return TQB_ERR_INVALID_ARG;
    }
}

}  // namespace tqb
