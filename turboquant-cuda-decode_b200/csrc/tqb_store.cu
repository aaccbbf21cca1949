// tqb_store.cu — sm_100a TurboQuant cache store (all presets, SoA and AoS).
//
// Reference: _tq_fused_store_mse in reference/soa_store.py:223-373 (SoA) and
// reference/aos_store.py:221-340 (AoS).  Half a warp per token-head, each
// lane owning 8 consecutive dims, one kernel instance per layout:
//   1. bucketise y (rotated unit key) against the 15 midpoints with the
//      reference's 4-step binary search, `y >= mid` going right (:306-316);
//   2. pack two codes per byte, low nibble = even dim (:319-325);
//   3. SoA with norm correction: stored norm = fp16(|k| * (1/sqrt(sum c^2 +
//      1e-16))) (:343-353); AoS: fp16(|k|);
//   4. values: min/max, scale = max((max-min)/15, 1e-8), code =
//      clamp(trunc((v-min)/scale + 0.5), 0, 15), fp16 scale and zero (:85-116).
// All fp32 steps use explicitly rounded intrinsics, and the 128-term sum of
// squared centroids follows the reference's summation order (eight strided
// running sums combined pairwise, the order numpy applies when the reference
// kernel runs interpreted), so the written bytes are bit-identical to the
// reference store for the same kernel inputs.
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "tqb_common.cuh"
#include "tqb_internal.h"

namespace tqb {

namespace {

constexpr int kStoreWarps = 8;

// a / b rounded to nearest even, from y = RN(1/b): Markstein's FMA
// iteration (P. Markstein, "Computation of elementary functions on the IBM
// RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990).  q0 = RN(a y)
// is within 1.5 ulp of a/b; the first correction makes it faithful, after
// which the residual a - b q1 is exact and the second correction rounds
// correctly.  Holds for b and 1/b normal and a quotient far from the
// subnormal range; below that the store maps every candidate to code 0.
__device__ __forceinline__ float div_rn_by_rcp(float a, float b, float y) {
    const float q0 = __fmul_rn(a, y);
    const float r0 = __fmaf_rn(-b, q0, a);
    const float q1 = __fmaf_rn(r0, y, q0);
    const float r1 = __fmaf_rn(-b, q1, a);
    return __fmaf_rn(r1, y, q1);
}

// Byte stores of a little-endian value (3-bit streams, 2-byte-aligned slots).
__device__ __forceinline__ void st_bytes3(uint8_t* p, uint32_t v) {
    p[0] = (uint8_t)v;
    p[1] = (uint8_t)(v >> 8);
    p[2] = (uint8_t)(v >> 16);
}
__device__ __forceinline__ void st_u16x2(uint8_t* p, uint32_t v) {
    reinterpret_cast<unsigned short*>(p)[0] = (unsigned short)v;
    reinterpret_cast<unsigned short*>(p)[1] = (unsigned short)(v >> 16);
}

// One instance per cache layout L, so each carries only its own key and
// slot code.  A token-head takes 16 lanes, 8 consecutive dims per lane
// (dims 8m .. 8m + 7 on lane m of the half-warp), so a warp stores two
// token-heads and the per-row reductions are 4 shuffle levels.  The
// midpoints and the squared centroids sit in shared memory.
template <int L>
__global__ void __launch_bounds__(kStoreWarps * 32) store_kernel(const StoreParams P) {
    constexpr bool k8 = layout_fp8_keys(L), k3 = layout_3bit_keys(L), v3 = layout_3bit_values(L);
    constexpr int nc = k3 ? 8 : kNumCentroids;
    constexpr unsigned kFull = 0xffffffffu;
    __shared__ float4 sq[2 * kStoreWarps][kHeadDim / 4];  // squared centroids of each row
    __shared__ float smid[kNumCentroids], scsq[kNumCentroids];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, m = lane & 15, half = lane >> 4;
    if constexpr (!k8) {
        if (threadIdx.x < nc - 1) smid[threadIdx.x] = __ldg(P.mids + threadIdx.x);
        if (P.norm_correction && threadIdx.x < nc) {
            const float cv = __ldg(P.cents + threadIdx.x);
            scsq[threadIdx.x] = __fmul_rn(cv, cv);
        }
        __syncthreads();
    }
    // N x H < 2^31 (checked on the host): 32-bit index arithmetic.  A warp
    // past the end leaves as a whole; a half past the end, or on a padding
    // token, computes on the last row and stores nothing, so every shuffle
    // runs on all 32 lanes.
    const uint32_t total = (uint32_t)P.N * (uint32_t)P.H;
    const uint32_t w0 = (blockIdx.x * kStoreWarps + (uint32_t)warp) * 2u;
    if (w0 >= total) return;
    const uint32_t pid0 = w0 + (uint32_t)half;
    const bool live = pid0 < total;
    const uint32_t pid = live ? pid0 : total - 1;
    const uint32_t tok = pid / (uint32_t)P.H, h = pid - tok * (uint32_t)P.H;
    const int32_t slot = __ldg(P.slots + tok);
    const bool write = live && slot >= 0;  // slot < 0: padding token (reference/soa_store.py:275-277)
    const uint32_t blk = (uint32_t)max(slot, 0) / kBlockSize, off = (uint32_t)max(slot, 0) % kBlockSize;

    const float4* yp = reinterpret_cast<const float4*>(P.y + (size_t)pid * kHeadDim) + 2 * m;
    const float4* vp4 = reinterpret_cast<const float4*>(P.value + (size_t)pid * kHeadDim) + 2 * m;
    const float4 ya = __ldg(yp), yb = __ldg(yp + 1), va = __ldg(vp4), vb = __ldg(vp4 + 1);
    uint32_t klo = 0, khi = 0;  // key codes: dims 8m .. 8m+3 in klo, 8m+4 .. 8m+7 in khi (FP8: bytes)
    uint32_t kbits = 0;         // 4-bit: 8 nibbles; 3-bit: 24 bits
    float vn = 0.0f;
    if constexpr (k8) {
        // FP8 keys (reference/soa_store.py:187-194): the raw key cast to e4m3
        // with round-to-nearest-even and saturation to +-448, the conversion
        // the compiled reference issues on sm_90 and later.
        auto cvt2 = [](float a, float b) {
            return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
        };
        klo = cvt2(ya.x, ya.y) | (cvt2(ya.z, ya.w) << 16);
        khi = cvt2(yb.x, yb.y) | (cvt2(yb.z, yb.w) << 16);
    } else {
        // -- keys: bucketise + pack.  The reference's binary search
        // (reference/soa_store.py:305-316; `y >= mid` goes right, 4 steps, or
        // 3 for 8 centroids) visits the midpoints of a complete binary tree:
        // 7, then 3 or 11, then idx + 1, then idx (3-bit: 3, idx + 1, idx),
        // never reaching the clamp at nc - 2, so this walk is the same search.
        vn = __ldg(P.norms + pid);
        const float ys[8] = {ya.x, ya.y, ya.z, ya.w, yb.x, yb.y, yb.z, yb.w};
        int idx[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int i;
            if constexpr (k3) {
                i = ys[j] >= smid[3] ? 4 : 0;
            } else {
                i = ys[j] >= smid[7] ? 8 : 0;
                i += ys[j] >= smid[i + 3] ? 4 : 0;
            }
            i += ys[j] >= smid[i + 1] ? 2 : 0;
            i += ys[j] >= smid[i] ? 1 : 0;
            idx[j] = i;
            kbits |= (uint32_t)i << ((k3 ? 3 : 4) * j);
        }

        if (P.norm_correction) {
            // 8 strided running sums r_i = c^2[i] + c^2[i+8] + ... + c^2[i+120]
            // in that order (the row's lanes m = 0..15 in turn), then
            // ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7))
            float4* row = sq[2 * warp + half];
            row[2 * m] = make_float4(scsq[idx[0]], scsq[idx[1]], scsq[idx[2]], scsq[idx[3]]);
            row[2 * m + 1] = make_float4(scsq[idx[4]], scsq[idx[5]], scsq[idx[6]], scsq[idx[7]]);
            __syncwarp();
            const float* rs = reinterpret_cast<const float*>(row) + (m & 7);
            float r = rs[0];
#pragma unroll
            for (int k = 1; k < 16; k++) r = __fadd_rn(r, rs[8 * k]);  // r_{m & 7}
            const float r1 = __shfl_down_sync(kFull, r, 1);
            const float pr = __fadd_rn(r, r1);  // valid on even m < 8
            const float pr2 = __shfl_down_sync(kFull, pr, 2);
            const float qd = __fadd_rn(pr, pr2);  // valid on m = 0, 4
            const float qd4 = __shfl_down_sync(kFull, qd, 4);
            float nsq = __fadd_rn(qd, qd4);  // valid on m = 0
            nsq = __shfl_sync(kFull, nsq, lane & 16);
            nsq = __fadd_rn(nsq, 1e-16f);
            vn = __fmul_rn(vn, __frcp_rn(__fsqrt_rn(nsq)));  // RN(1/x) = RN(1 / x)
        }
    }

    // -- values: quantise + pack --
    const float vs[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
    float vmin = vs[0], vmax = vs[0];
#pragma unroll
    for (int j = 1; j < 8; j++) {
        vmin = fminf(vmin, vs[j]);
        vmax = fmaxf(vmax, vs[j]);
    }
#pragma unroll
    for (int o = 1; o < 16; o <<= 1) {
        vmin = fminf(vmin, __shfl_xor_sync(kFull, vmin, o));
        vmax = fmaxf(vmax, __shfl_xor_sync(kFull, vmax, o));
    }
    // 3-bit values (reference/soa_store.py:49-84): 7 levels, codes packed
    // little-endian at bit 3d; 4-bit: 15 levels, two codes per byte.
    // scale = max((max - min) / levels, 1e-8): a range below 1e-7 ends at the
    // floor, so the division only matters for normal ranges, where the FMA
    // iteration on RN(1/levels) is exact; an infinite range stays infinite.
    constexpr int vtop = v3 ? 7 : 15;
    constexpr float kRcpTop = 1.0f / (float)vtop;  // correctly rounded at compile time
    const float range = __fsub_rn(vmax, vmin);
    float scale = range < INFINITY ? div_rn_by_rcp(range, (float)vtop, kRcpTop) : range;
    scale = scale > 1e-8f ? scale : 1e-8f;
    float qv[8];
    if (isfinite(scale)) {  // uniform over the half-warp
        const float y = __frcp_rn(scale);
#pragma unroll
        for (int j = 0; j < 8; j++) qv[j] = div_rn_by_rcp(__fsub_rn(vs[j], vmin), scale, y);
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) qv[j] = __fdiv_rn(__fsub_rn(vs[j], vmin), scale);
    }
    uint32_t vbits = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        int q = __float2int_rz(__fadd_rn(qv[j], 0.5f));
        q = q < 0 ? 0 : (q > vtop ? vtop : q);
        vbits |= (uint32_t)q << ((v3 ? 3 : 4) * j);
    }
    if (!write) return;

    // -- write --
    uint8_t* base = P.cache + (size_t)blk * (size_t)P.block_bytes;
    const unsigned short vn_h = __half_as_ushort(__float2half_rn(vn));
    const unsigned short sc_h = __half_as_ushort(__float2half_rn(scale));
    const unsigned short zr_h = __half_as_ushort(__float2half_rn(vmin));
    if constexpr (L == TQB_LAYOUT_SOA_K8) {
        // 4-byte aligned rows (checked on the host): two words of e4m3 bytes
        uint8_t* dp = base + (size_t)off * ((size_t)P.H * kK8DataBytes) + (size_t)h * kK8DataBytes;
        reinterpret_cast<uint32_t*>(dp)[2 * m] = klo;
        reinterpret_cast<uint32_t*>(dp)[2 * m + 1] = khi;
        reinterpret_cast<uint32_t*>(dp + kK8KeyBytes)[m] = vbits;
        if (m == 0) {
            unsigned short* meta = reinterpret_cast<unsigned short*>(
                base + (size_t)kBlockSize * P.H * kK8DataBytes) + (size_t)h * 2 * kBlockSize;
            meta[off] = sc_h;
            meta[kBlockSize + off] = zr_h;
        }
    } else if constexpr (L == TQB_LAYOUT_SOA_K3V3 || L == TQB_LAYOUT_SOA_K3) {
        constexpr int row = v3 ? kK3V3DataBytes : kK3DataBytes;
        uint8_t* dp = base + (size_t)off * ((size_t)P.H * row) + (size_t)h * row;
        st_bytes3(dp + 3 * m, kbits);  // dims 8m .. 8m+7 = bits 24m .. 24m+23 of the stream
        if constexpr (v3)
            st_bytes3(dp + kK3KeyBytes + 3 * m, vbits);
        else
            st_u16x2(dp + kK3KeyBytes + 4 * m, vbits);
        if (m == 0) {
            unsigned short* meta = reinterpret_cast<unsigned short*>(
                base + (size_t)kBlockSize * P.H * row) + (size_t)h * 3 * kBlockSize;
            meta[off] = vn_h;
            meta[kBlockSize + off] = sc_h;
            meta[2 * kBlockSize + off] = zr_h;
        }
    } else if constexpr (L == TQB_LAYOUT_SOA) {
        uint8_t* dp = base + (size_t)off * ((size_t)P.H * kDataBytes) + (size_t)h * kDataBytes;
        st_u16x2(dp + 4 * m, kbits);
        st_u16x2(dp + kKBytes + 4 * m, vbits);
        if (m == 0) {
            unsigned short* meta = reinterpret_cast<unsigned short*>(
                base + (size_t)kBlockSize * P.H * kDataBytes) + (size_t)h * 3 * kBlockSize;
            meta[off] = vn_h;
            meta[kBlockSize + off] = sc_h;
            meta[2 * kBlockSize + off] = zr_h;
        }
    } else {
        // AoS slot (layout_is_aos): [key codes | fp16 norm | value codes |
        // fp16 scale | fp16 zero], 2-byte aligned, so 16-bit and byte stores
        // (reference/aos_store.py:26-116, :183-203, :296-325).
        uint8_t* sp = base + (size_t)off * P.pos_stride + (size_t)h * P.head_stride;
        if constexpr (k8) {  // e4m3 bytes of dims 8m .. 8m + 7
            st_u16x2(sp + 8 * m, klo);
            st_u16x2(sp + 8 * m + 4, khi);
        } else if constexpr (k3) {
            st_bytes3(sp + 3 * m, kbits);
        } else {
            st_u16x2(sp + 4 * m, kbits);
        }
        uint8_t* vq = sp + aos_val_off(L);
        if constexpr (v3)
            st_bytes3(vq + 3 * m, vbits);
        else
            st_u16x2(vq + 4 * m, vbits);
        if (m == 0) {
            // AoS stores the raw norm (no folding, reference/aos_store.py:317-325);
            // e4m3 keys have none.
            if constexpr (!k8) {
                const unsigned short raw = __half_as_ushort(__float2half_rn(__ldg(P.norms + pid)));
                reinterpret_cast<unsigned short*>(sp + aos_norm_off(L))[0] = raw;
            }
            reinterpret_cast<unsigned short*>(sp + aos_scale_off(L))[0] = sc_h;
            reinterpret_cast<unsigned short*>(sp + aos_scale_off(L) + 2)[0] = zr_h;
        }
    }
}

}  // namespace

template <int L>
void launch_store_t(const StoreParams& P, unsigned grid, cudaStream_t stream) {
    store_kernel<L><<<grid, kStoreWarps * 32, 0, stream>>>(P);
}

int launch_store(const StoreParams& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.N * P.H;
    if (items == 0) return TQB_OK;
    const unsigned grid = (unsigned)((items + 2 * kStoreWarps - 1) / (2 * kStoreWarps));
    switch (P.layout) {
        case TQB_LAYOUT_SOA: launch_store_t<TQB_LAYOUT_SOA>(P, grid, stream); break;
        case TQB_LAYOUT_SOA_K8: launch_store_t<TQB_LAYOUT_SOA_K8>(P, grid, stream); break;
        case TQB_LAYOUT_SOA_K3: launch_store_t<TQB_LAYOUT_SOA_K3>(P, grid, stream); break;
        case TQB_LAYOUT_SOA_K3V3: launch_store_t<TQB_LAYOUT_SOA_K3V3>(P, grid, stream); break;
        case TQB_LAYOUT_AOS: launch_store_t<TQB_LAYOUT_AOS>(P, grid, stream); break;
        case TQB_LAYOUT_AOS_K8: launch_store_t<TQB_LAYOUT_AOS_K8>(P, grid, stream); break;
        case TQB_LAYOUT_AOS_K3: launch_store_t<TQB_LAYOUT_AOS_K3>(P, grid, stream); break;
        case TQB_LAYOUT_AOS_K3V3: launch_store_t<TQB_LAYOUT_AOS_K3V3>(P, grid, stream); break;
        default: return TQB_ERR_INVALID_ARG;
    }
    return report_launch(cudaGetLastError());
}

}  // namespace tqb
