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
#include "tqb_merge_row.cuh"

namespace tqb {

namespace {

constexpr int kWarpsPerCta = 8;

// Output element conversion (round to nearest even, as torch's .to(dtype)).
template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// One CTA of 4 warps per (b, h): merge_row (tqb_merge_row.cuh) merges the
// row's non-empty splits; thread d writes output dim d, thread 0 the LSE.
template <typename OutT>
__global__ void __launch_bounds__(kHeadDim, 8) stage2_kernel(const Stage2Params P) {
    pdl_trigger();
    pdl_wait();  // Stage1's partials, when it ran just before on the stream
    const int64_t item = blockIdx.x;  // b * Hq + h
    const int b = (int)(item / P.Hq), h = (int)(item % P.Hq);
    float o, lse;
    merge_row(P, b, h, &o, &lse);
    OutT* out = static_cast<OutT*>(P.out) + (int64_t)b * P.osb + (int64_t)h * P.osh;
    out[threadIdx.x] = from_f32<OutT>(o);
    if (threadIdx.x == 0) P.lse[(int64_t)b * P.lsb + h] = lse;
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

// Attention sinks (reference/soa_decode_v1.py:134-145): split 0 of a
// non-empty sequence starts its online softmax at m = s, l = 1, i.e. counts
// one more token of logit s = sinks[h] and value 0.  From split 0's (O, LSE)
// that is LSE' = ln(e^LSE + e^s), O' = O e^(LSE - LSE').  One warp per
// (b, h); split 0 is unwritten, and left alone, when seq_len <= 0.  A sink of
// -inf leaves the row bit-identical (factor 1, LSE + ln 1).
__global__ void __launch_bounds__(kWarpsPerCta * 32) sink_fold_kernel(const SinkParams P) {
    const int lane = threadIdx.x & 31;
    const int64_t item = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (item >= (int64_t)P.B * P.Hq) return;
    const int b = (int)(item / P.Hq), h = (int)(item % P.Hq);
    if (P.seq_lens[b] <= 0) return;
    float* row = P.mid + (int64_t)b * P.msb + (int64_t)h * P.msh;  // split 0
    const float lse0 = row[kHeadDim];
    const float s = __ldg(P.sinks + h);
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; j++) v[j] = row[lane + 32 * j];
    __syncwarp();  // every lane has read the LSE before lane 0 rewrites it
    const float mx = fmaxf(lse0, s);
    const float e0 = expf(lse0 - mx), es = expf(s - mx);
    const float sum = e0 + es;
    const float f = __fdiv_rn(e0, sum);
#pragma unroll
    for (int j = 0; j < 4; j++) row[lane + 32 * j] = v[j] * f;
    if (lane == 0) row[kHeadDim] = mx + logf(sum);
}

}  // namespace

int launch_stage2(const Stage2Params& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.B * P.Hq;
    if (items == 0) return TQB_OK;
    switch (P.out_dtype) {
        case TQB_DTYPE_F32: return report_launch(launch_pdl(stage2_kernel<float>, dim3((unsigned)items), dim3(kHeadDim), 0, stream, P));
        case TQB_DTYPE_F16: return report_launch(launch_pdl(stage2_kernel<__half>, dim3((unsigned)items), dim3(kHeadDim), 0, stream, P));
        case TQB_DTYPE_BF16:
            return report_launch(launch_pdl(stage2_kernel<__nv_bfloat16>, dim3((unsigned)items), dim3(kHeadDim), 0, stream, P));
        default: return TQB_ERR_INVALID_ARG;
    }
}

int launch_merge(const MergeParams& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.B * P.Hq;
    if (items == 0) return TQB_OK;
    const int64_t grid = (items + kWarpsPerCta - 1) / kWarpsPerCta;
    merge_kernel<<<(unsigned)grid, kWarpsPerCta * 32, 0, stream>>>(P);
    return report_launch(cudaGetLastError());
}

int launch_fold_sinks(const SinkParams& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.B * P.Hq;
    if (items == 0) return TQB_OK;
    const int64_t grid = (items + kWarpsPerCta - 1) / kWarpsPerCta;
    sink_fold_kernel<<<(unsigned)grid, kWarpsPerCta * 32, 0, stream>>>(P);
    return report_launch(cudaGetLastError());
}

}  // namespace tqb
