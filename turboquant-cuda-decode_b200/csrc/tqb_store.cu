// tqb_store.cu — sm_100a TurboQuant cache store (all presets, SoA and AoS).
//
// Reference: _tq_fused_store_mse in reference/soa_store.py:223-373 (SoA) and
// reference/aos_store.py:221-340 (AoS).  One warp per token-head, each lane
// owning 4 consecutive dims, one kernel instance per layout:
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

// One instance per cache layout L, so each carries only its own key and
// slot code.  The midpoints and the squared centroids sit in shared memory.
template <int L>
__global__ void __launch_bounds__(kStoreWarps * 32) store_kernel(const StoreParams P) {
    constexpr bool k8 = layout_fp8_keys(L), k3 = layout_3bit_keys(L), v3 = layout_3bit_values(L);
    constexpr int nc = k3 ? 8 : kNumCentroids;
    __shared__ float sq[kStoreWarps][kHeadDim];
    __shared__ float smid[kNumCentroids], scsq[kNumCentroids];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if constexpr (!k8) {
        if (threadIdx.x < nc - 1) smid[threadIdx.x] = __ldg(P.mids + threadIdx.x);
        if (P.norm_correction && threadIdx.x < nc) {
            const float cv = __ldg(P.cents + threadIdx.x);
            scsq[threadIdx.x] = __fmul_rn(cv, cv);
        }
        __syncthreads();
    }
    // N x H < 2^31 (checked on the host): 32-bit index arithmetic
    const uint32_t pid = blockIdx.x * kStoreWarps + (uint32_t)warp;
    if (pid >= (uint32_t)P.N * (uint32_t)P.H) return;
    const uint32_t tok = pid / (uint32_t)P.H, h = pid - tok * (uint32_t)P.H;
    const int32_t slot = __ldg(P.slots + tok);
    if (slot < 0) return;  // padding token (reference/soa_store.py:275-277)
    const uint32_t blk = (uint32_t)slot / kBlockSize, off = (uint32_t)slot % kBlockSize;

    const float4 yv = __ldg(reinterpret_cast<const float4*>(P.y + (size_t)pid * kHeadDim) + lane);
    const float4 vv = __ldg(reinterpret_cast<const float4*>(P.value + (size_t)pid * kHeadDim) + lane);
    uint32_t kpack = 0;
    float vn = 0.0f;
    if constexpr (k8) {
        // FP8 keys (reference/soa_store.py:187-194): the raw key cast to e4m3
        // with round-to-nearest-even and saturation to +-448, the conversion
        // the compiled reference issues on sm_90 and later.
        const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(yv.x, yv.y), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(yv.z, yv.w), __NV_SATFINITE, __NV_E4M3);
        kpack = (uint32_t)lo | ((uint32_t)hi << 16);
    } else {
        // -- keys: bucketise + pack.  The reference's binary search
        // (reference/soa_store.py:305-316; `y >= mid` goes right, 4 steps, or
        // 3 for 8 centroids) visits the midpoints of a complete binary tree:
        // 7, then 3 or 11, then idx + 1, then idx (3-bit: 3, idx + 1, idx),
        // never reaching the clamp at nc - 2, so this walk is the same search.
        vn = __ldg(P.norms + pid);
        const float ys[4] = {yv.x, yv.y, yv.z, yv.w};
        int idx[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
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
        }
        kpack = k3 ? (uint32_t)(idx[0] | (idx[1] << 3) | (idx[2] << 6) | (idx[3] << 9))  // 12 bits, dim 4 lane at bit 0
                   : (uint32_t)(idx[0] | (idx[1] << 4) | (idx[2] << 8) | (idx[3] << 12));

        if (P.norm_correction) {
#pragma unroll
            for (int j = 0; j < 4; j++) sq[warp][4 * lane + j] = scsq[idx[j]];
            __syncwarp();
            float r = 0.0f;
            if (lane < 8) {
                r = sq[warp][lane];
                for (int i = 8 + lane; i < kHeadDim; i += 8) r = __fadd_rn(r, sq[warp][i]);
            }
            // ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7))
            const float r1 = __shfl_down_sync(0xffffffffu, r, 1);
            const float pr = __fadd_rn(r, r1);  // valid on even lanes < 8
            const float pr2 = __shfl_down_sync(0xffffffffu, pr, 2);
            const float qd = __fadd_rn(pr, pr2);  // valid on lanes 0, 4
            const float qd4 = __shfl_down_sync(0xffffffffu, qd, 4);
            float nsq = __fadd_rn(qd, qd4);       // valid on lane 0
            nsq = __shfl_sync(0xffffffffu, nsq, 0);
            nsq = __fadd_rn(nsq, 1e-16f);
            vn = __fmul_rn(vn, __frcp_rn(__fsqrt_rn(nsq)));  // RN(1/x) = RN(1 / x)
        }
    }

    // -- values: quantise + pack --
    const float vs[4] = {vv.x, vv.y, vv.z, vv.w};
    float vmin = fminf(fminf(vs[0], vs[1]), fminf(vs[2], vs[3]));
    float vmax = fmaxf(fmaxf(vs[0], vs[1]), fmaxf(vs[2], vs[3]));
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        vmin = fminf(vmin, __shfl_xor_sync(0xffffffffu, vmin, o));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
    }
    // 3-bit values (reference/soa_store.py:49-84): 7 levels, codes packed
    // little-endian at bit 3d; 4-bit: 15 levels, two codes per byte.
    constexpr int vtop = v3 ? 7 : 15;
    float scale = __fdiv_rn(__fsub_rn(vmax, vmin), (float)vtop);
    scale = scale > 1e-8f ? scale : 1e-8f;
    float qv[4];
    if (isfinite(scale)) {  // uniform over the warp
        const float y = __frcp_rn(scale);
#pragma unroll
        for (int j = 0; j < 4; j++) qv[j] = div_rn_by_rcp(__fsub_rn(vs[j], vmin), scale, y);
    } else {
#pragma unroll
        for (int j = 0; j < 4; j++) qv[j] = __fdiv_rn(__fsub_rn(vs[j], vmin), scale);
    }
    uint32_t vpack = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        int q = __float2int_rz(__fadd_rn(qv[j], 0.5f));
        q = q < 0 ? 0 : (q > vtop ? vtop : q);
        vpack |= (uint32_t)q << ((v3 ? 3 : 4) * j);
    }

    // -- write --
    uint8_t* base = P.cache + blk * P.block_bytes;
    const unsigned short vn_h = __half_as_ushort(__float2half_rn(vn));
    const unsigned short sc_h = __half_as_ushort(__float2half_rn(scale));
    const unsigned short zr_h = __half_as_ushort(__float2half_rn(vmin));
    if constexpr (L == TQB_LAYOUT_SOA_K8) {
        uint8_t* dp = base + off * ((int64_t)P.H * kK8DataBytes) + (int64_t)h * kK8DataBytes;
        reinterpret_cast<uint32_t*>(dp)[lane] = kpack;  // dims 4 lane .. 4 lane + 3
        reinterpret_cast<unsigned short*>(dp + kK8KeyBytes)[lane] = (unsigned short)vpack;
        if (lane == 0) {
            unsigned short* meta = reinterpret_cast<unsigned short*>(
                base + (int64_t)kBlockSize * P.H * kK8DataBytes) + (int64_t)h * 2 * kBlockSize;
            meta[off] = sc_h;
            meta[kBlockSize + off] = zr_h;
        }
    } else if constexpr (L == TQB_LAYOUT_SOA_K3V3) {
        uint8_t* dp = base + off * ((int64_t)P.H * kK3V3DataBytes) + (int64_t)h * kK3V3DataBytes;
        // keys and values: lanes 2m and 2m+1 hold dims 8m .. 8m+7, bytes
        // 3m .. 3m+2 of each 48-byte stream
        const uint32_t kup = __shfl_down_sync(0xffffffffu, kpack, 1);
        const uint32_t vup = __shfl_down_sync(0xffffffffu, vpack, 1);
        if ((lane & 1) == 0) {
            const uint32_t k24 = kpack | (kup << 12), v24 = vpack | (vup << 12);
            uint8_t* kb = dp + 3 * (lane >> 1);
            uint8_t* vb = dp + kK3KeyBytes + 3 * (lane >> 1);
            kb[0] = (uint8_t)k24; kb[1] = (uint8_t)(k24 >> 8); kb[2] = (uint8_t)(k24 >> 16);
            vb[0] = (uint8_t)v24; vb[1] = (uint8_t)(v24 >> 8); vb[2] = (uint8_t)(v24 >> 16);
        }
        if (lane == 0) {
            unsigned short* meta = reinterpret_cast<unsigned short*>(
                base + (int64_t)kBlockSize * P.H * kK3V3DataBytes) + (int64_t)h * 3 * kBlockSize;
            meta[off] = vn_h;
            meta[kBlockSize + off] = sc_h;
            meta[2 * kBlockSize + off] = zr_h;
        }
    } else if constexpr (L == TQB_LAYOUT_SOA_K3) {
        uint8_t* dp = base + off * ((int64_t)P.H * kK3DataBytes) + (int64_t)h * kK3DataBytes;
        // Lanes 2m and 2m+1 hold dims 8m .. 8m+7 = bits 24m .. 24m+23 of the
        // little-endian 3-bit stream, i.e. bytes 3m .. 3m+2.
        const uint32_t up = __shfl_down_sync(0xffffffffu, kpack, 1);
        if ((lane & 1) == 0) {
            const uint32_t p24 = kpack | (up << 12);
            uint8_t* kb = dp + 3 * (lane >> 1);
            kb[0] = (uint8_t)p24;
            kb[1] = (uint8_t)(p24 >> 8);
            kb[2] = (uint8_t)(p24 >> 16);
        }
        reinterpret_cast<unsigned short*>(dp + kK3KeyBytes)[lane] = (unsigned short)vpack;
        if (lane == 0) {
            unsigned short* meta = reinterpret_cast<unsigned short*>(
                base + (int64_t)kBlockSize * P.H * kK3DataBytes) + (int64_t)h * 3 * kBlockSize;
            meta[off] = vn_h;
            meta[kBlockSize + off] = sc_h;
            meta[2 * kBlockSize + off] = zr_h;
        }
    } else if constexpr (L == TQB_LAYOUT_SOA) {
        uint8_t* dp = base + off * ((int64_t)P.H * kDataBytes) + (int64_t)h * kDataBytes;
        reinterpret_cast<unsigned short*>(dp)[lane] = (unsigned short)kpack;
        reinterpret_cast<unsigned short*>(dp + kKBytes)[lane] = (unsigned short)vpack;
        if (lane == 0) {
            unsigned short* meta = reinterpret_cast<unsigned short*>(
                base + (int64_t)kBlockSize * P.H * kDataBytes) + (int64_t)h * 3 * kBlockSize;
            meta[off] = vn_h;
            meta[kBlockSize + off] = sc_h;
            meta[2 * kBlockSize + off] = zr_h;
        }
    } else {
        // AoS slot (layout_is_aos): [key codes | fp16 norm | value codes |
        // fp16 scale | fp16 zero], 2-byte aligned, so 16-bit and byte stores
        // (reference/aos_store.py:26-116, :183-203, :296-325).
        uint8_t* sp = base + off * P.pos_stride + (int64_t)h * P.head_stride;
        const uint32_t kup = __shfl_down_sync(0xffffffffu, kpack, 1);
        const uint32_t vup = __shfl_down_sync(0xffffffffu, vpack, 1);
        if constexpr (k8) {  // e4m3 bytes of dims 4 lane .. 4 lane + 3
            reinterpret_cast<unsigned short*>(sp)[2 * lane] = (unsigned short)kpack;
            reinterpret_cast<unsigned short*>(sp)[2 * lane + 1] = (unsigned short)(kpack >> 16);
        } else if constexpr (k3) {  // lanes 2m and 2m+1: bytes 3m .. 3m+2 of the 3-bit stream
            if ((lane & 1) == 0) {
                const uint32_t k24 = kpack | (kup << 12);
                uint8_t* kb = sp + 3 * (lane >> 1);
                kb[0] = (uint8_t)k24; kb[1] = (uint8_t)(k24 >> 8); kb[2] = (uint8_t)(k24 >> 16);
            }
        } else {
            reinterpret_cast<unsigned short*>(sp)[lane] = (unsigned short)kpack;
        }
        uint8_t* vp = sp + aos_val_off(L);
        if constexpr (v3) {
            if ((lane & 1) == 0) {
                const uint32_t v24 = vpack | (vup << 12);
                uint8_t* vb = vp + 3 * (lane >> 1);
                vb[0] = (uint8_t)v24; vb[1] = (uint8_t)(v24 >> 8); vb[2] = (uint8_t)(v24 >> 16);
            }
        } else {
            reinterpret_cast<unsigned short*>(vp)[lane] = (unsigned short)vpack;
        }
        if (lane == 0) {
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
    const unsigned grid = (unsigned)((items + kStoreWarps - 1) / kStoreWarps);
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
