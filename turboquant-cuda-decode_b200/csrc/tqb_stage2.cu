// tqb_stage2.cu — split merge (Stage2) and cross-GPU partial merge.
//
// Stage2 (reference: baseline/stage2.py:8-55): for each (b, h), an online
// log-sum-exp merge over the non-empty splits of mid_o,
//     out = sum_s w_s O_s / sum_s w_s,  w_s = exp(lse_s - max),
//     lse = max + ln(sum_s w_s).
// The merge reads 33.8 MB at the B64x4K workload against 0.13 MB written, so
// it is an HBM-bound streaming pass: one warp per (b, h), each lane owning 4
// of the 128 dims, coalesced 128-byte row reads per split.
#include <cuda_runtime.h>

#include "tqb_common.cuh"
#include "tqb_internal.h"

namespace tqb {

namespace {

constexpr int kWarpsPerCta = 8;

// Two passes per (b, h) so that every load is independent of the previous
// split's result: (1) lane s of a 32-split chunk reads LSE_s, the warp forms
// the max and the weights w_s = exp(LSE_s - max); (2) every lane reads its 4
// dims of all splits (unrolled, loads in flight together) and accumulates
// w_s * O_s.  Same algebra as the reference's running merge.
__global__ void __launch_bounds__(kWarpsPerCta * 32) stage2_kernel(const Stage2Params P) {
    const int lane = threadIdx.x & 31;
    const int64_t item = (int64_t)blockIdx.x * kWarpsPerCta + (threadIdx.x >> 5);
    if (item >= (int64_t)P.B * P.Hq) return;
    const int b = (int)(item / P.Hq), h = (int)(item % P.Hq);
    const int nsp = P.nsplits ? min(__ldg(P.nsplits + b), P.S) : P.S;
    const int L = __ldg(P.seq_lens + b);
    const int split_len = nsp > 0 ? (L + nsp - 1) / nsp : 0;
    const float* row0 = P.mid + (int64_t)b * P.msb + (int64_t)h * P.msh;
    auto nonempty = [&](int s) { return s < nsp && split_len * s < min(split_len * (s + 1), L); };

    float gmax = -INFINITY;
    for (int s0 = 0; s0 < nsp; s0 += 32) {
        const int s = s0 + lane;
        const float l = nonempty(s) ? __ldg(row0 + (int64_t)s * P.mss + kHeadDim) : -INFINITY;
        gmax = fmaxf(gmax, warp_max_xor(l, 1, 16));
    }
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float wsum = 0.0f;
    for (int s0 = 0; s0 < nsp; s0 += 32) {
        const int s = s0 + lane;
        const bool ok = nonempty(s);
        const float l = ok ? __ldg(row0 + (int64_t)s * P.mss + kHeadDim) : -INFINITY;
        const float wl = ok ? expf(l - gmax) : 0.0f;
        wsum += warp_sum_xor(wl, 1, 16);
        const int n = min(32, nsp - s0);
#pragma unroll 8
        for (int k = 0; k < n; k++) {
            const float w = __shfl_sync(0xffffffffu, wl, k);
            const float* row = row0 + (int64_t)(s0 + k) * P.mss;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float v = __ldg(row + lane + 32 * j);
                acc[j] += w * (w != 0.0f ? v : 0.0f);
            }
        }
    }
    float* out = P.out + (int64_t)b * P.osb + (int64_t)h * P.osh;
#pragma unroll
    for (int j = 0; j < 4; j++) out[lane + 32 * j] = __fdiv_rn(acc[j], wsum);
    if (lane == 0) P.lse[(int64_t)b * P.lsb + h] = gmax + logf(wsum);
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
    const int64_t grid = (items + kWarpsPerCta - 1) / kWarpsPerCta;
    stage2_kernel<<<(unsigned)grid, kWarpsPerCta * 32, 0, stream>>>(P);
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
