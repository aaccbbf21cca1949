// tqb_stage2.cu — split merge (Stage2) and cross-GPU partial merge.
//
// Stage2 (reference: baseline/stage2.py:8-55): for each (b, h), an online
// log-sum-exp merge over the non-empty splits of mid_o,
//     out = sum_s w_s O_s / sum_s w_s,  w_s = exp(lse_s - max),
//     lse = max + ln(sum_s w_s).
// The merge reads 33.8 MB at the B64x4K workload (mostly from L2, written by
// Stage1 just before) against 1 MB written: a latency-bound streaming pass.
#include <cuda_runtime.h>

#include "tqb_common.cuh"
#include "tqb_internal.h"

namespace tqb {

namespace {

constexpr int kWarpsPerCta = 8;
constexpr int kFastSplits = 32;  // split counts served with all loads in flight

// One CTA of 128 threads per (b, h), thread d owning output dim d: every
// split row is read as one coalesced 512-byte run by the CTA, and each thread
// has all of its split loads in flight at once (the partials are mostly
// L2-resident right after Stage1).  Two passes so that no load waits on the
// previous split's result: (1) the maximum LSE over the non-empty splits,
// (2) sum_s w_s O_s and sum_s w_s with w_s = exp(LSE_s - max).  Same algebra
// as the reference's running merge.
__global__ void __launch_bounds__(kHeadDim) stage2_kernel(const Stage2Params P) {
    const int64_t item = blockIdx.x;  // b * Hq + h
    const int b = (int)(item / P.Hq), h = (int)(item % P.Hq);
    const int d = threadIdx.x;
    const int nsp = P.nsplits ? min(__ldg(P.nsplits + b), P.S) : P.S;
    const int L = __ldg(P.seq_lens + b);
    const int split_len = nsp > 0 ? (L + nsp - 1) / nsp : 0;
    // split s is non-empty iff split_len * s < L (its end is min(.., L))
    const int nvalid = split_len > 0 ? min(nsp, (L + split_len - 1) / split_len) : 0;
    const float* row0 = P.mid + (int64_t)b * P.msb + (int64_t)h * P.msh;

    float gmax = -INFINITY, acc = 0.0f, wsum = 0.0f;
    if (nvalid <= kFastSplits) {
        // Every load in flight at once: kFastSplits predicated (LSE, O) pairs.
        float ls[kFastSplits], os[kFastSplits];
#pragma unroll
        for (int s = 0; s < kFastSplits; s++) {
            const float* row = row0 + (int64_t)s * P.mss;
            ls[s] = s < nvalid ? __ldg(row + kHeadDim) : -INFINITY;
            os[s] = s < nvalid ? __ldg(row + d) : 0.0f;
        }
#pragma unroll
        for (int s = 0; s < kFastSplits; s++) gmax = fmaxf(gmax, ls[s]);
#pragma unroll
        for (int s = 0; s < kFastSplits; s++) {
            const float w = s < nvalid ? expf(ls[s] - gmax) : 0.0f;
            acc += w * os[s];
            wsum += w;
        }
    } else {
#pragma unroll 16
        for (int s = 0; s < nvalid; s++) gmax = fmaxf(gmax, __ldg(row0 + (int64_t)s * P.mss + kHeadDim));
#pragma unroll 16
        for (int s = 0; s < nvalid; s++) {
            const float* row = row0 + (int64_t)s * P.mss;
            const float w = expf(__ldg(row + kHeadDim) - gmax);
            acc += w * __ldg(row + d);
            wsum += w;
        }
    }
    float* out = P.out + (int64_t)b * P.osb + (int64_t)h * P.osh;
    out[d] = __fdiv_rn(acc, wsum);
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
    stage2_kernel<<<(unsigned)items, kHeadDim, 0, stream>>>(P);
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
