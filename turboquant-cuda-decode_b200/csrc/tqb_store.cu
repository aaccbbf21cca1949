// tqb_store.cu — sm_100a TurboQuant cache store (all presets, SoA and AoS).
//
// Reference: _tq_fused_store_mse in reference/soa_store.py:223-373 (SoA) and
// reference/aos_store.py:221-340 (AoS).  One warp per token-head, each lane
// owning 4 consecutive dims:
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

__global__ void __launch_bounds__(kStoreWarps * 32) store_kernel(const StoreParams P) {
    __shared__ float sq[kStoreWarps][kHeadDim];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t pid = (int64_t)blockIdx.x * kStoreWarps + warp;
    if (pid >= (int64_t)P.N * P.H) return;
    const int tok = (int)(pid / P.H), h = (int)(pid % P.H);
    const int32_t slot = __ldg(P.slots + tok);
    if (slot < 0) return;  // padding token (reference/soa_store.py:275-277)
    const int64_t blk = slot / kBlockSize, off = slot % kBlockSize;

    const float4 yv = __ldg(reinterpret_cast<const float4*>(P.y + pid * kHeadDim) + lane);
    const bool k8 = layout_fp8_keys(P.layout);
    const bool k3 = layout_3bit_keys(P.layout);
    uint32_t kpack = 0;
    float vn = 0.0f;
    if (k8) {
        // FP8 keys (reference/soa_store.py:187-194): the raw key cast to e4m3
        // with round-to-nearest-even and saturation to +-448, the conversion
        // the compiled reference issues on sm_90 and later.
        const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(yv.x, yv.y), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(yv.z, yv.w), __NV_SATFINITE, __NV_E4M3);
        kpack = (uint32_t)lo | ((uint32_t)hi << 16);
    } else {
    // -- keys: bucketise + pack --
    const float ys[4] = {yv.x, yv.y, yv.z, yv.w};
    // 3-bit keys: 8 centroids, 3 search steps (reference/soa_store.py:305-314
    // with MSE_BITS = 3)
    const int nc = k3 ? 8 : kNumCentroids, steps = k3 ? 3 : 4;
    int idx[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
        int lo = 0, hi = nc - 1;
#pragma unroll
        for (int it = 0; it < 4; it++) {
            if (it >= steps) break;
            const int mid = (lo + hi) >> 1;
            const int safe = mid < nc - 2 ? mid : nc - 2;
            const bool right = ys[j] >= __ldg(P.mids + safe);
            lo = right ? mid + 1 : lo;
            hi = right ? hi : mid;
        }
        idx[j] = lo < nc - 1 ? lo : nc - 1;
    }
    kpack = k3 ? (uint32_t)(idx[0] | (idx[1] << 3) | (idx[2] << 6) | (idx[3] << 9))  // 12 bits, dim 4 lane at bit 0
               : (uint32_t)(idx[0] | (idx[1] << 4) | (idx[2] << 8) | (idx[3] << 12));

    vn = __ldg(P.norms + pid);
    if (P.norm_correction) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float cv = __ldg(P.cents + idx[j]);
            sq[warp][4 * lane + j] = __fmul_rn(cv, cv);
        }
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
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(nsq));
        vn = __fmul_rn(vn, inv);
    }
    }  // 4-bit keys

    // -- values: quantise + pack --
    const float4 vv = __ldg(reinterpret_cast<const float4*>(P.value + pid * kHeadDim) + lane);
    const float vs[4] = {vv.x, vv.y, vv.z, vv.w};
    float vmin = fminf(fminf(vs[0], vs[1]), fminf(vs[2], vs[3]));
    float vmax = fmaxf(fmaxf(vs[0], vs[1]), fmaxf(vs[2], vs[3]));
    for (int o = 1; o < 32; o <<= 1) {
        vmin = fminf(vmin, __shfl_xor_sync(0xffffffffu, vmin, o));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
    }
    // 3-bit values (reference/soa_store.py:49-84): 7 levels, codes packed
    // little-endian at bit 3d; 4-bit: 15 levels, two codes per byte.
    const bool v3 = layout_3bit_values(P.layout);
    const int vtop = v3 ? 7 : 15;
    float scale = __fdiv_rn(__fsub_rn(vmax, vmin), v3 ? 7.0f : 15.0f);
    scale = scale > 1e-8f ? scale : 1e-8f;
    uint32_t vpack = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const float t = __fadd_rn(__fdiv_rn(__fsub_rn(vs[j], vmin), scale), 0.5f);
        int q = __float2int_rz(t);
        q = q < 0 ? 0 : (q > vtop ? vtop : q);
        vpack |= (uint32_t)q << ((v3 ? 3 : 4) * j);
    }

    // -- write --
    uint8_t* base = P.cache + blk * P.block_bytes;
    const unsigned short vn_h = __half_as_ushort(__float2half_rn(vn));
    const unsigned short sc_h = __half_as_ushort(__float2half_rn(scale));
    const unsigned short zr_h = __half_as_ushort(__float2half_rn(vmin));
    if (P.layout == TQB_LAYOUT_SOA_K8) {
        uint8_t* dp = base + off * ((int64_t)P.H * kK8DataBytes) + (int64_t)h * kK8DataBytes;
        reinterpret_cast<uint32_t*>(dp)[lane] = kpack;  // dims 4 lane .. 4 lane + 3
        reinterpret_cast<unsigned short*>(dp + kK8KeyBytes)[lane] = (unsigned short)vpack;
        if (lane == 0) {
            unsigned short* meta = reinterpret_cast<unsigned short*>(
                base + (int64_t)kBlockSize * P.H * kK8DataBytes) + (int64_t)h * 2 * kBlockSize;
            meta[off] = sc_h;
            meta[kBlockSize + off] = zr_h;
        }
    } else if (P.layout == TQB_LAYOUT_SOA_K3V3) {
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
    } else if (P.layout == TQB_LAYOUT_SOA_K3) {
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
    } else if (P.layout == TQB_LAYOUT_SOA) {
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
        const int L = P.layout;
        const uint32_t kup = __shfl_down_sync(0xffffffffu, kpack, 1);
        const uint32_t vup = __shfl_down_sync(0xffffffffu, vpack, 1);
        if (k8) {  // e4m3 bytes of dims 4 lane .. 4 lane + 3
            reinterpret_cast<unsigned short*>(sp)[2 * lane] = (unsigned short)kpack;
            reinterpret_cast<unsigned short*>(sp)[2 * lane + 1] = (unsigned short)(kpack >> 16);
        } else if (k3) {  // lanes 2m and 2m+1: bytes 3m .. 3m+2 of the 3-bit stream
            if ((lane & 1) == 0) {
                const uint32_t k24 = kpack | (kup << 12);
                uint8_t* kb = sp + 3 * (lane >> 1);
                kb[0] = (uint8_t)k24; kb[1] = (uint8_t)(k24 >> 8); kb[2] = (uint8_t)(k24 >> 16);
            }
        } else {
            reinterpret_cast<unsigned short*>(sp)[lane] = (unsigned short)kpack;
        }
        uint8_t* vp = sp + aos_val_off(L);
        if (v3) {
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
            if (!k8) {
                const unsigned short raw = __half_as_ushort(__float2half_rn(__ldg(P.norms + pid)));
                reinterpret_cast<unsigned short*>(sp + aos_norm_off(L))[0] = raw;
            }
            reinterpret_cast<unsigned short*>(sp + aos_scale_off(L))[0] = sc_h;
            reinterpret_cast<unsigned short*>(sp + aos_scale_off(L) + 2)[0] = zr_h;
        }
    }
}

}  // namespace

int launch_store(const StoreParams& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.N * P.H;
    if (items == 0) return TQB_OK;
    const int64_t grid = (items + kStoreWarps - 1) / kStoreWarps;
    store_kernel<<<(unsigned)grid, kStoreWarps * 32, 0, stream>>>(P);
    return report_launch(cudaGetLastError());
}

}  // namespace tqb
