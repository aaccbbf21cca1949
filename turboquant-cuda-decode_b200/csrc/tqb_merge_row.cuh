// tqb_merge_row.cuh — the Stage2 merge of one (b, h) row, shared by the
// Stage2 kernel and the sequence-parallel exchange kernel.
//
// Online log-sum-exp merge over the non-empty splits of mid_o
// (baseline/stage2.py:8-55): out = sum_s w_s O_s / sum_s w_s with
// w_s = exp(lse_s - max), lse = max + ln(sum_s w_s); the exponentials and the
// logarithm run on the hardware base-2 units (as Triton's tl.exp / tl.log in
// the reference's Stage2 do).  Called by all threads of a CTA of kWarps
// warps (warp w merges splits w, w + kWarps, ... with the loads of
// kSplitsPerPass splits in flight, lane l owning dims l, l+32, l+64, l+96;
// the kWarps partial states combine through shared memory).  Thread d < 128
// returns output dim d in *o, and every thread the row's LSE in *lse_out.
// Stage2 uses 4 warps per row (many rows, few splits each); the
// sequence-parallel exchange 16 (few rows, many splits each).
#pragma once

#include "tqb_common.cuh"
#include "tqb_internal.h"

namespace tqb {

constexpr int kSplitsPerPass = 4;  // splits whose loads a warp keeps in flight at once

template <int kParts = kHeadDim / 32>
__device__ __forceinline__ void merge_row(const Stage2Params& P, int b, int h, float* o, float* lse_out) {
    static_assert(kParts * 32 >= kHeadDim, "one thread per output dim");
    __shared__ float s_acc[kParts][kHeadDim];
    __shared__ float s_max[kParts], s_sum[kParts];
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
        const float scale = m == -INFINITY ? 0.0f : ex2_approx((m - mn) * kLog2e);
        sum *= scale;
#pragma unroll
        for (int j = 0; j < 4; j++) acc[j] *= scale;
#pragma unroll
        for (int k = 0; k < kSplitsPerPass; k++) {
            const float w = ls[k] == -INFINITY ? 0.0f : ex2_approx((ls[k] - mn) * kLog2e);
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
    const int d = threadIdx.x < kHeadDim ? threadIdx.x : kHeadDim - 1;
    float gmax = -INFINITY;
#pragma unroll
    for (int p = 0; p < kParts; p++) gmax = fmaxf(gmax, s_max[p]);
    float acc_d = 0.0f, wsum = 0.0f;
#pragma unroll
    for (int p = 0; p < kParts; p++) {
        const float w = s_max[p] == -INFINITY ? 0.0f : ex2_approx((s_max[p] - gmax) * kLog2e);
        acc_d += w * s_acc[p][d];
        wsum += w * s_sum[p];
    }
    *o = __fdiv_rn(acc_d, wsum);
    *lse_out = gmax + lg2_approx(wsum) * kLn2;
}

}  // namespace tqb
