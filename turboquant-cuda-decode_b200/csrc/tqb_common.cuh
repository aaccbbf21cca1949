// tqb_common.cuh — shared device helpers for the sm_100a TurboQuant kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace tqb {

constexpr int kHeadDim = 128;
constexpr int kBlockSize = 16;        // tokens per physical page
constexpr int kKBytes = kHeadDim / 2; // packed 4-bit K codes per token-head
constexpr int kVBytes = kHeadDim / 2; // packed 4-bit V codes per token-head
constexpr int kDataBytes = kKBytes + kVBytes;
constexpr int kSlotBytes = kDataBytes + 6; // + knorm, vscale, vzero (fp16)
// FP8-key layout (TQB_LAYOUT_SOA_K8): 128 e4m3 key bytes + 64 V bytes, then
// vscale and vzero in the block's meta region.
constexpr int kK8KeyBytes = kHeadDim;
constexpr int kK8DataBytes = kK8KeyBytes + kVBytes;  // 192
constexpr int kSlotBytesK8 = kK8DataBytes + 4;       // 196
// 3-bit-key layout (TQB_LAYOUT_SOA_K3): 48 packed key bytes + 64 V bytes,
// then knorm, vscale, vzero in the meta region; 8 centroids.
constexpr int kK3KeyBytes = kHeadDim * 3 / 8;        // 48
constexpr int kK3DataBytes = kK3KeyBytes + kVBytes;  // 112
constexpr int kSlotBytesK3 = kK3DataBytes + 6;       // 118
// 3-bit keys and values (TQB_LAYOUT_SOA_K3V3): 48 + 48 data bytes + meta.
constexpr int kV3Bytes = kHeadDim * 3 / 8;           // 48
constexpr int kK3V3DataBytes = kK3KeyBytes + kV3Bytes;  // 96
constexpr int kSlotBytesK3V3 = kK3V3DataBytes + 6;   // 102
constexpr int kNumCentroids = 16;

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---------------------------------------------------------------------------
// Tensor-core MMA: D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col).
// Fragment ownership (lane = 4*g + c): A {a0a1: row g, cols 2c..2c+1;
// a2a3: row g+8; a4a5: row g, cols 2c+8..; a6a7: row g+8, cols 2c+8..},
// B {b0b1: rows 2c..2c+1, col g; b2b3: rows 2c+8.., col g},
// D {d0d1: row g, cols 2c..2c+1; d2d3: row g+8}.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                          uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// (x & m) | o in one LOP3.
__device__ __forceinline__ uint32_t and_or(uint32_t x, uint32_t m, uint32_t o) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(x), "r"(m), "r"(o));
    return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) {
    return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) {
    return *reinterpret_cast<__half2*>(&u);
}

// Exact fp16 integers from nibbles: (x & mask) | 0x6400 per half gives
// 1024 + n (low nibble) or 1024 + 16 n (high nibble); subtracting 1024 is
// exact.
__device__ __forceinline__ uint32_t nib_to_h2(uint32_t x, uint32_t mask) {
    const uint32_t magic = 0x64006400u;
    __half2 v = u32_as_h2(and_or(x, mask, magic));
    return h2_as_u32(__hsub2(v, u32_as_h2(magic)));
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

__device__ __forceinline__ float warp_max_xor(float v, int from, int to) {
    for (int o = from; o <= to; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum_xor(float v, int from, int to) {
    for (int o = from; o <= to; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Power-of-two exponent e such that max_abs * 2^e lies in [2^14, 2^15):
// scaling fp16 operands this way keeps hi/lo splits away from both overflow
// and the subnormal range.  Read from the exponent bits (for a normal
// max_abs = m * 2^(E-126), m in [0.5, 1), e = 15 - (E - 126)); 0 for zero and
// non-finite inputs; clamped to [-100, 100] (a subnormal max_abs).
__device__ __forceinline__ int fp16_scale_exp(float max_abs) {
    const int be = (int)((__float_as_uint(max_abs) >> 23) & 0xFFu);
    if (!(max_abs > 0.0f) || be == 0xFF) return 0;
    const int e = 15 - (be - 126);
    return e < -100 ? -100 : (e > 100 ? 100 : e);
}

// 2^e for integer e in [-126, 127], built from the exponent bits.
__device__ __forceinline__ float exp2i(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// Programmatic dependent launch (PTX griddepcontrol, sm_90 and later).  A
// kernel launched by launch_pdl may be scheduled while the kernel before it
// on the stream is still running; pdl_wait blocks until that kernel has
// completed and its memory operations are visible, so it comes before the
// first global access.  pdl_trigger lets the next kernel be scheduled once
// every CTA of this one has issued it.  Both are no-ops in a kernel launched
// without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

#ifdef __CUDACC__
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}
#endif

// Hardware reciprocal and base-2 logarithm (relative error about 2^-23).
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float lg2_approx(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}
// Hardware 2^x (relative error about 2^-22; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}


// Eight 3-bit fields (bits 3i .. 3i+2 of h, 24 bits) to eight nibbles
// (bits 4i .. 4i+2): halves, then quarters, then pairs move apart.
__device__ __forceinline__ uint32_t spread3to4(uint32_t h) {
    const uint32_t z = (h & 0xFFFu) | ((h & 0xFFF000u) << 4);
    const uint32_t w = (z & 0x003F003Fu) | ((z & 0x0FC00FC0u) << 2);
    return (w & 0x07070707u) | ((w & 0x38383838u) << 1);
}

// Bits [o, o + 6) of the little-endian 96-bit stream k.x | k.y | k.z (o a
// compile-time constant after unrolling, o + 6 <= 96).
__device__ __forceinline__ uint32_t bits6(const uint4& k, int o) {
    const int i = o >> 5;
    const uint32_t lo = i == 0 ? k.x : i == 1 ? k.y : k.z;
    const uint32_t hi = i == 0 ? k.y : i == 1 ? k.z : 0u;
    return __funnelshift_r(lo, hi, (uint32_t)(o & 31)) & 63u;
}

// Two e4m3 bytes (low byte first) to an exact f16x2 (low half first).
__device__ __forceinline__ uint32_t fp8x2_to_h2(uint32_t two) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two, __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

}  // namespace tqb
