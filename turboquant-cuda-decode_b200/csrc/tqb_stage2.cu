// tqb_stage2.cu — split merge (Stage2) and cross-GPU partial merge.
//
// Stage2 (reference: baseline/stage2.py:8-55): for each (b, h), an online
// log-sum-exp merge over the non-empty splits of mid_o,
//     out = sum_s w_s O_s / sum_s w_s,  w_s = exp(lse_s - max),
//     lse = max + ln(sum_s w_s).
// The merge reads 33.8 MB at the B64x4K workload (mostly from L2, written by
// Stage1 just before) against 1 MB written: a latency-bound streaming pass.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tqb_common.cuh"
#include "tqb_internal.h"

namespace tqb {

namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kSplitsPerPass = 8;  // splits whose loads a warp keeps in flight at once

// Output element conversion (round to nearest even, as torch's .to(dtype)).
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// One CTA of 4 warps per (b, h).  Warp w merges the non-empty splits
// s = w, w + 4, w + 8, ... of (b, h): lane l owns dims l, l+32, l+64, l+96,
// so each split row is read as four coalesced 128-byte runs, and the warp
// issues the loads of up to kSplitsPerPass splits before using any of them.
// The four warps' (max, sum, acc) then combine through shared memory.  Same
// log-sum-exp algebra as the reference's running merge.
template <typename OutT>
__global__ void __launch_bounds__(kHeadDim, 8) stage2_kernel(const Stage2Params P) {
    constexpr int kParts = kHeadDim / 32;  // warps per CTA
    __shared__ float s_acc[kParts][kHeadDim];
    __shared__ float s_max[kParts], s_sum[kParts];
    const int64_t item = blockIdx.x;  // b * Hq + h
    const int b = (int)(item / P.Hq), h = (int)(item % P.Hq);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nsp = P.nsplits ? min(__ldg(P.nsplits + b), P.S) : P.S;
    const int L = __ldg(P.seq_lens + b);
    const int split_len = nsp > 0 ? (L + nsp - 1) / nsp : 0;
    // split s is non-empty iff split_len * s < L (its end is min(.., L))
    const int nvalid = split_len > 0 ? min(nsp, (L + split_len - 1) / split_len) : 0;
    const float* row0 = P.mid + (int64_t)b * P.msb + (int64_t)h * P.msh;

    float m = -INFINITY, sum = 0.0f, acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int s0 = warp; s0 < nvalid; s0 += kParts * kSplitsPerPass) {
        float ls[kSplitsPerPass], os[kSplitsPerPass][4];
#pragma unroll
        for (int k = 0; k < kSplitsPerPass; k++) {
            const int s = s0 + kParts * k;
            const float* row = row0 + (int64_t)s * P.mss;
            ls[k] = s < nvalid ? __ldg(row + kHeadDim) : -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) os[k][j] = s < nvalid ? __ldg(row + lane + 32 * j) : 0.0f;
        }
        float mn = m;
#pragma unroll
        for (int k = 0; k < kSplitsPerPass; k++) mn = fmaxf(mn, ls[k]);
        const float scale = m == -INFINITY ? 0.0f : expf(m - mn);
        sum *= scale;
#pragma unroll
        for (int j = 0; j < 4; j++) acc[j] *= scale;
#pragma unroll
        for (int k = 0; k < kSplitsPerPass; k++) {
            const float w = ls[k] == -INFINITY ? 0.0f : expf(ls[k] - mn);
            sum += w;
#pragma unroll
            for (int j = 0; j < 4; j++) acc[j] += w * os[k][j];
        }
        m = mn;
    }
#pragma unroll
    for (int j = 0; j < 4; j++) s_acc[warp][lane + 32 * j] = acc[j];
    if (lane == 0) {
        s_max[warp] = m;
        s_sum[warp] = sum;
    }
    __syncthreads();
    const int d = threadIdx.x;
    float gmax = -INFINITY;
#pragma unroll
    for (int p = 0; p < kParts; p++) gmax = fmaxf(gmax, s_max[p]);
    float o = 0.0f, wsum = 0.0f;
#pragma unroll
    for (int p = 0; p < kParts; p++) {
        const float w = s_max[p] == -INFINITY ? 0.0f : expf(s_max[p] - gmax);
        o += w * s_acc[p][d];
        wsum += w * s_sum[p];
    }
    OutT* out = static_cast<OutT*>(P.out) + (int64_t)b * P.osb + (int64_t)h * P.osh;
    out[d] = from_f32<OutT>(__fdiv_rn(o, wsum));
    if (d == 0) P.lse[(int64_t)b * P.lsb + h] = gmax + logf(wsum);
}

// Cross-GPU merge of G (O, LSE) partials laid out [G, B, Hq, D+1]; parts
// with LSE = -inf (an empty KV range) are skipped.
__global__ void __launch_bounds__(kWarpsPerCta * 32) merge_kernel(const MergeParams P) {
    const int lane = threadIdx.x & 31;
    const int64_t item = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    const int64_t BH = (int64_t)P.B * P.Hq;
    if (item >= BH) return;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float rmax = -INFINITY, rsum = 0.0f;
    for (int gp = 0; gp < P.G; gp++) {
        const float* row = P.partials + ((int64_t)gp * BH + item) * (kHeadDim + 1);
        const float slse = __ldg(row + kHeadDim);
        if (slse == -INFINITY) continue;
        const float nmax = fmaxf(rmax, slse);
        const float old_scale = expf(rmax - nmax);
        const float w = expf(slse - nmax);
#pragma unroll
        for (int j = 0; j < 4; j++) acc[j] = acc[j] * old_scale + w * __ldg(row + lane + 32 * j);
        rsum = rsum * old_scale + w;
        rmax = nmax;
    }
    float* out = P.out + item * kHeadDim;
#pragma unroll
    for (int j = 0; j < 4; j++) out[lane + 32 * j] = __fdiv_rn(acc[j], rsum);
    if (lane == 0 && P.lse) P.lse[item] = rmax + logf(rsum);
}

}  // namespace

int launch_stage2(const Stage2Params& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.B * P.Hq;
    if (items == 0) return TQB_OK;
    switch (P.out_dtype) {
        case TQB_DTYPE_F32: stage2_kernel<float><<<(unsigned)items, kHeadDim, 0, stream>>>(P); break;
        case TQB_DTYPE_F16: stage2_kernel<__half><<<(unsigned)items, kHeadDim, 0, stream>>>(P); break;
        case TQB_DTYPE_BF16: stage2_kernel<__nv_bfloat16><<<(unsigned)items, kHeadDim, 0, stream>>>(P); break;
        default: return TQB_ERR_INVALID_ARG;
    }
    return report_launch(cudaGetLastError());
}

int launch_merge(const MergeParams& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.B * P.Hq;
    if (items == 0) return TQB_OK;
    const int64_t grid = (items + kWarpsPerCta - 1) / kWarpsPerCta;
    merge_kernel<<<(unsigned)grid, kWarpsPerCta * 32, 0, stream>>>(P);
    return report_launch(cudaGetLastError());
}

}  // namespace tqb
