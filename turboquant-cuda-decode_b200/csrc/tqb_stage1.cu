// tqb_stage1.cu — sm_100a Stage1 of the TurboQuant 4bit_nc decode.
//
// What it computes (reference: reference/soa_decode_v1.py:43-314 for the SoA
// cache, reference/aos_decode.py:43-313 for the AoS cache): for every
// (sequence b, query head h, KV split s) the softmax-normalised partial
// output over the split's tokens and its natural-log LSE,
//     score_t = knorm_t * (q_rot[b,h] . c[idx_t]) * attn_scale
//     O       = sum_t exp(score_t - m) * V_t / sum_t exp(score_t - m)
//     LSE     = m + ln(sum_t exp(score_t - m))
// with K_t = centroids[idx_t] * knorm_t and V_t = vidx_t * vscale_t + vzero_t.
//
// How (B200 design, not a translation of the reference kernels):
//  * One warp owns one work item (b, KV head, split) and serves all Hq/Hk
//    query heads of its GQA group; 8 warps per CTA, persistent grid.  With
//    the KV head as the fastest item index, the 8 warps of a CTA read the 8
//    interleaved 128-byte head slices of the same 16-token pages, so each
//    17 KB page streams from HBM as one contiguous run.
//  * The warp walks the split one 16-token page at a time with 128/64/32-bit
//    streaming loads into a two-page register ring.  One lane per CTA asks
//    L2 for whole blocks kPrefetchPages ahead (cp.async.bulk.prefetch.L2,
//    one request per 17 KB block), so DRAM latency is covered without
//    spending registers on a deeper ring; the first pages of a warp's next
//    item are requested while it finishes the current one.
//  * Q.K runs on the tensor cores as D[row, n] = K[row, :] . Qpack[:, n]
//    (mma.m16n8k16; the contraction is 8 columns wide per token, so the
//    register-operand MMA is used rather than tcgen05, whose smem operands
//    would have to hold the dequantised K).  The 8 N columns are 4 query heads x {Q_hi, Q_lo}
//    (fp16 split of the power-of-two scaled fp32 query); the 16 M rows are 8
//    tokens x {C_hi, C_lo} (fp16 split of the scaled centroid).  The four
//    partial products add up, per lane, to the fp32-accurate dot product
//    (the single fp16 MMA of the reference's V2 kernel does not meet 1e-4).
//    A byte of packed K (two 4-bit codes) maps to {C_hi pair, C_lo pair}
//    through a 256-entry table with one copy per lane in shared memory
//    (bank-conflict free); one PRMT forms the table offset from the byte and
//    the lane, and each table load is exactly half of an A fragment.
//  * Softmax runs in the exp2 domain on the MMA accumulators; each lane owns
//    one query head and two tokens of the page, so the row max is three
//    shuffles.
//  * P.V runs on the tensor cores as D[dim, n] = Vq[dim, token] . W[token, n]
//    with dims as M.  The raw 4-bit codes are used as fp16 subnormals
//    (code * 2^-20, mantissa bits 4-7) with one AND (plus a shift for the
//    low nibble), so the operand is exact and costs no conversion;
//    W = p * vscale is split into fp16 hi/lo across the N columns, so the
//    product is fp32-accurate; the vzero term sum_t p_t * vzero_t is added
//    per head in fp32.
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include "tqb_common.cuh"
#include "tqb_internal.h"

namespace tqb {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kLutStride = 256;              // bytes per table entry (all copies)
constexpr float kLazy = 8.0f;                // lazy-rescale slack (log2 units)
constexpr float kWMax = 32768.0f;            // largest W kept on the lazy path
constexpr int kLutBytes = 256 * kLutStride;  // 64 KB
constexpr int kPrefetchPages = 3;            // L2 prefetch distance in pages
constexpr int kMinBlocksNT1 = 2;             // CTAs per SM for one n-tile

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint4 ld_stream_v4(const uint8_t* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ld_stream_v2(const uint8_t* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n"
                 : "=r"(r.x), "=r"(r.y)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ld_stream_u32(const uint8_t* p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];\n" : "=r"(r) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ld_stream_u16(const uint8_t* p) {
    unsigned short r;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];\n" : "=h"(r) : "l"(p));
    return r;
}
// L2 prefetch of `bytes` (multiple of 16) from a 16-byte aligned address,
// one bulk request.
__device__ __forceinline__ void prefetch_l2_bulk(const uint8_t* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(addr));
    return r;
}

// One page's worth of a lane's operands.
struct PageRegs {
    uint4 k0, k1;         // K bytes [16c, 16c+16) of tokens 2g and 2g+1
    uint4 k0b, k1b;       // FP8 keys: K bytes [32c, 32c+32) are k0|k0b and k1|k1b
    uint2 v[4];           // V bytes [8g, 8g+8) of tokens 4c .. 4c+3
    uint32_t kn, vs, vz;  // fp16 pairs (tokens 2g, 2g+1): knorm, vscale, vzero
};

// Byte offsets, inside one physical block, of a lane's operands for KV head
// kvh (fixed for a work item).  Token rows are `row` bytes apart.
struct LaneOffsets {
    uint32_t k0;    // K bytes of token 2g (token 2g+1: + row)
    uint32_t v0;    // V bytes of token 4c (token 4c+j: + j * row)
    uint32_t meta;  // SoA: knorm pair; AoS: slot metadata of token 2g
    uint32_t row;   // bytes between consecutive tokens of a page
};

template <int LAYOUT>
__device__ __forceinline__ LaneOffsets lane_offsets(const Stage1Params& P, int kvh, int lane) {
    const int g = lane >> 2, c = lane & 3;
    LaneOffsets o;
    if (LAYOUT == TQB_LAYOUT_SOA_K3V3) {
        const uint32_t tok = (uint32_t)P.Hk * kK3V3DataBytes;
        const uint32_t head = (uint32_t)kvh * kK3V3DataBytes;
        o.row = tok;
        o.k0 = (2 * g) * tok + head + 12 * c;
        o.v0 = (4 * c) * tok + head + kK3KeyBytes + 6 * g;  // dims 16g .. 16g+15 = 6 value bytes
        o.meta = kBlockSize * tok + (uint32_t)kvh * (3 * kBlockSize * 2) + 4 * g;
    } else if (LAYOUT == TQB_LAYOUT_SOA_K3) {
        const uint32_t tok = (uint32_t)P.Hk * kK3DataBytes;
        const uint32_t head = (uint32_t)kvh * kK3DataBytes;
        o.row = tok;
        o.k0 = (2 * g) * tok + head + 12 * c;  // dims 32c .. 32c+31 = key bytes 12c .. 12c+11
        o.v0 = (4 * c) * tok + head + kK3KeyBytes + 8 * g;
        o.meta = kBlockSize * tok + (uint32_t)kvh * (3 * kBlockSize * 2) + 4 * g;
    } else if (LAYOUT == TQB_LAYOUT_SOA_K8) {
        const uint32_t tok = (uint32_t)P.Hk * kK8DataBytes;
        const uint32_t head = (uint32_t)kvh * kK8DataBytes;
        o.row = tok;
        o.k0 = (2 * g) * tok + head + 32 * c;
        o.v0 = (4 * c) * tok + head + kK8KeyBytes + 8 * g;
        o.meta = kBlockSize * tok + (uint32_t)kvh * (2 * kBlockSize * 2) + 4 * g;
    } else if (LAYOUT == TQB_LAYOUT_SOA) {
        const uint32_t tok = (uint32_t)P.Hk * kDataBytes;
        const uint32_t head = (uint32_t)kvh * kDataBytes;
        o.row = tok;
        o.k0 = (2 * g) * tok + head + 16 * c;
        o.v0 = (4 * c) * tok + head + kKBytes + 8 * g;
        o.meta = kBlockSize * tok + (uint32_t)kvh * (3 * kBlockSize * 2) + 4 * g;
    } else {
        // AoS slot [key codes | fp16 norm | value codes | fp16 vscale | vzero]
        // (layout_is_aos): keys of dims 32c .. 32c+31 are 16 bytes (4-bit), 12
        // (3-bit) or 32 (e4m3) at that multiple of c; values of dims 16g ..
        // 16g+15 are 8 bytes (4-bit) or 6 (3-bit).
        const uint32_t pos = (uint32_t)P.pos_stride, hs = (uint32_t)P.head_stride * kvh;
        constexpr uint32_t kKeyLane = layout_fp8_keys(LAYOUT) ? 32 : layout_3bit_keys(LAYOUT) ? 12 : 16;
        constexpr uint32_t kValLane = layout_3bit_values(LAYOUT) ? 6 : 8;
        o.row = pos;
        o.k0 = (2 * g) * pos + hs + kKeyLane * c;
        o.v0 = (4 * c) * pos + hs + aos_val_off(LAYOUT) + kValLane * g;
        o.meta = (2 * g) * pos + hs + aos_norm_off(LAYOUT);
    }
    return o;
}

// Whole physical block into L2 with one bulk request (lane 0 of the warp
// that serves KV head 0, whose block holds every head of the page).
__device__ __forceinline__ void prefetch_block(const uint8_t* block, uint32_t bytes, bool leader) {
    if (leader) prefetch_l2_bulk(block, bytes);
}


// AoS slots are only 2-byte aligned: gather with 16-bit loads.
__device__ __forceinline__ uint32_t ld2x16(const uint8_t* p) {
    return ld_stream_u16(p) | (ld_stream_u16(p + 2) << 16);
}

template <int LAYOUT>
__device__ __forceinline__ void load_page(PageRegs& r, const uint8_t* base, const LaneOffsets& o) {
    if (LAYOUT == TQB_LAYOUT_SOA_K3V3) {
        const uint8_t* k = base + o.k0;
        const uint8_t* v = base + o.v0;
        const uint8_t* m = base + o.meta;
        r.k0 = make_uint4(ld_stream_u32(k), ld_stream_u32(k + 4), ld_stream_u32(k + 8), 0u);
        r.k1 = make_uint4(ld_stream_u32(k + o.row), ld_stream_u32(k + o.row + 4), ld_stream_u32(k + o.row + 8), 0u);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            // 16 3-bit codes (6 bytes, 2-byte aligned) spread to the nibble
            // layout of the 4-bit values (low nibble = even dim)
            const uint8_t* vj = v + j * o.row;
            const uint32_t a = ld_stream_u16(vj), b = ld_stream_u16(vj + 2), cc = ld_stream_u16(vj + 4);
            r.v[j] = make_uint2(spread3to4((a | (b << 16)) & 0xFFFFFFu), spread3to4((b >> 8) | (cc << 8)));
        }
        r.kn = ld_stream_u32(m);
        r.vs = ld_stream_u32(m + 2 * kBlockSize);
        r.vz = ld_stream_u32(m + 4 * kBlockSize);
    } else if (LAYOUT == TQB_LAYOUT_SOA_K3) {
        const uint8_t* k = base + o.k0;
        const uint8_t* v = base + o.v0;
        const uint8_t* m = base + o.meta;
        r.k0 = make_uint4(ld_stream_u32(k), ld_stream_u32(k + 4), ld_stream_u32(k + 8), 0u);
        r.k1 = make_uint4(ld_stream_u32(k + o.row), ld_stream_u32(k + o.row + 4), ld_stream_u32(k + o.row + 8), 0u);
#pragma unroll
        for (int j = 0; j < 4; j++) r.v[j] = ld_stream_v2(v + j * o.row);
        r.kn = ld_stream_u32(m);
        r.vs = ld_stream_u32(m + 2 * kBlockSize);
        r.vz = ld_stream_u32(m + 4 * kBlockSize);
    } else if (LAYOUT == TQB_LAYOUT_SOA_K8) {
        const uint8_t* k = base + o.k0;
        const uint8_t* v = base + o.v0;
        const uint8_t* m = base + o.meta;
        r.k0 = ld_stream_v4(k);
        r.k0b = ld_stream_v4(k + 16);
        r.k1 = ld_stream_v4(k + o.row);
        r.k1b = ld_stream_v4(k + o.row + 16);
#pragma unroll
        for (int j = 0; j < 4; j++) r.v[j] = ld_stream_v2(v + j * o.row);
        r.kn = 0x3C003C00u;  // no key norm: fp16 1.0 for both tokens
        r.vs = ld_stream_u32(m);
        r.vz = ld_stream_u32(m + 2 * kBlockSize);
    } else if (LAYOUT == TQB_LAYOUT_SOA) {
        const uint8_t* k = base + o.k0;
        const uint8_t* v = base + o.v0;
        const uint8_t* m = base + o.meta;
        r.k0 = ld_stream_v4(k);
        r.k1 = ld_stream_v4(k + o.row);
#pragma unroll
        for (int j = 0; j < 4; j++) r.v[j] = ld_stream_v2(v + j * o.row);
        r.kn = ld_stream_u32(m);
        r.vs = ld_stream_u32(m + 2 * kBlockSize);
        r.vz = ld_stream_u32(m + 4 * kBlockSize);
    } else {
        // AoS slots are only 2-byte aligned: 16-bit gathers.
        const uint8_t* s0 = base + o.k0;
        const uint8_t* s1 = s0 + o.row;
        if (layout_fp8_keys(LAYOUT)) {
            r.k0 = make_uint4(ld2x16(s0), ld2x16(s0 + 4), ld2x16(s0 + 8), ld2x16(s0 + 12));
            r.k0b = make_uint4(ld2x16(s0 + 16), ld2x16(s0 + 20), ld2x16(s0 + 24), ld2x16(s0 + 28));
            r.k1 = make_uint4(ld2x16(s1), ld2x16(s1 + 4), ld2x16(s1 + 8), ld2x16(s1 + 12));
            r.k1b = make_uint4(ld2x16(s1 + 16), ld2x16(s1 + 20), ld2x16(s1 + 24), ld2x16(s1 + 28));
        } else if (layout_3bit_keys(LAYOUT)) {
            r.k0 = make_uint4(ld2x16(s0), ld2x16(s0 + 4), ld2x16(s0 + 8), 0u);
            r.k1 = make_uint4(ld2x16(s1), ld2x16(s1 + 4), ld2x16(s1 + 8), 0u);
        } else {
            r.k0 = make_uint4(ld2x16(s0), ld2x16(s0 + 4), ld2x16(s0 + 8), ld2x16(s0 + 12));
            r.k1 = make_uint4(ld2x16(s1), ld2x16(s1 + 4), ld2x16(s1 + 8), ld2x16(s1 + 12));
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint8_t* sv = base + o.v0 + j * o.row;
            if (layout_3bit_values(LAYOUT)) {
                // 16 3-bit codes (6 bytes) spread to the nibble layout of the
                // 4-bit values (low nibble = even dim)
                const uint32_t a = ld_stream_u16(sv), b = ld_stream_u16(sv + 2), cc = ld_stream_u16(sv + 4);
                r.v[j] = make_uint2(spread3to4((a | (b << 16)) & 0xFFFFFFu), spread3to4((b >> 8) | (cc << 8)));
            } else {
                r.v[j] = make_uint2(ld2x16(sv), ld2x16(sv + 4));
            }
        }
        const uint8_t* m0 = base + o.meta;
        const uint8_t* m1 = m0 + o.row;
        constexpr int kSc = aos_scale_off(LAYOUT) - aos_norm_off(LAYOUT);  // scale, relative to the norm
        r.kn = layout_fp8_keys(LAYOUT) ? 0x3C003C00u  // no key norm: fp16 1.0 for both tokens
                                       : (ld_stream_u16(m0) | (ld_stream_u16(m1) << 16));
        r.vs = ld_stream_u16(m0 + kSc) | (ld_stream_u16(m1 + kSc) << 16);
        r.vz = ld_stream_u16(m0 + kSc + 2) | (ld_stream_u16(m1 + kSc + 2) << 16);
    }
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Running softmax / output state of one lane for one work item.
template <int NT>
struct ItemState {
    uint32_t qf[NT][16];  // Q.K B fragments
    float kfac[NT];       // score factor of this lane's head
    float m_run[NT], l_part[NT], z_part[NT];
    float acc[NT][8][4];  // P.V accumulators (codes scaled by 2^-20)
};

// Table entry load at byte offset `off` from the table start.
__device__ __forceinline__ uint2 lut_v2(const uint8_t* lut, uint32_t off) {
    return *reinterpret_cast<const uint2*>(lut + off);
}

// One 16-token page of one work item.
template <int NT, int LAYOUT>
__device__ __forceinline__ void process_page(ItemState<NT>& st, const PageRegs& cur, bool page_ok,
                                             int tok0, int start, int end, const uint8_t* lut,
                                             uint32_t lut_base, uint32_t lut_sel_src, int g, int c) {
    const bool va = page_ok && tok0 >= start && tok0 < end;
    const bool vb = page_ok && tok0 + 1 >= start && tok0 + 1 < end;

    // -- Q.K on the tensor cores --
    // Two M tiles per page: tile 0 = tokens 2g (even), tile 1 = tokens 2g+1.
    // Inside a tile, row g carries the C_hi part of the token and row g+8 its
    // C_lo part, so one table load ({C_hi pair, C_lo pair} of a byte) is
    // exactly half of an A fragment and the two parts add up per lane
    // afterwards.  The two tiles are independent accumulator chains.
    float dq[NT][2][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int mt = 0; mt < 2; mt++)
#pragma unroll
            for (int k = 0; k < 4; k++) dq[nt][mt][k] = 0.0f;
    float csq0 = 0.0f, csq1 = 0.0f;  // AoS: partial sums of c^2
    // AoS Lloyd-Max keys: the table entries carry the squared centroid sums
    // for the in-kernel norm correction.
    constexpr bool kNormCorr = layout_is_aos(LAYOUT) && !layout_fp8_keys(LAYOUT);
    if (layout_fp8_keys(LAYOUT)) {
        // FP8 keys convert exactly to fp16, so one M tile holds the whole
        // page: row g = token 2g, row g+8 = token 2g+1; k columns map to the
        // same dims 32c + 4ks + {0,1 | 2,3} as the query fragments.  Even and
        // odd ks accumulate in the two tiles' registers (two chains).
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
            const uint32_t w0 = word_of(ks < 4 ? cur.k0 : cur.k0b, ks & 3);
            const uint32_t w1 = word_of(ks < 4 ? cur.k1 : cur.k1b, ks & 3);
            const uint32_t a0 = fp8x2_to_h2(w0 & 0xFFFFu), a1 = fp8x2_to_h2(w1 & 0xFFFFu);
            const uint32_t a2 = fp8x2_to_h2(w0 >> 16), a3 = fp8x2_to_h2(w1 >> 16);
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
                mma_16816(dq[nt][ks & 1], a0, a1, a2, a3, st.qf[nt][2 * ks], st.qf[nt][2 * ks + 1]);
        }
    } else {
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
        const uint32_t w0 = word_of(cur.k0, ks >> 1), w1 = word_of(cur.k1, ks >> 1);
        const uint32_t jA = 2 * (ks & 1), jB = jA + 1;
        // (byte << 8) | this lane's copy offset, in one PRMT
        uint32_t ia, ib, ic, id;
        if (layout_3bit_keys(LAYOUT)) {
            // 3-bit keys: the dim pairs 32c + 4ks + {0,1} and {2,3} are the
            // 6-bit fields at bits 12ks and 12ks + 6 of the lane's 96 bits;
            // entry (pair << 8) + this lane's copy offset, as below.
            ia = (bits6(cur.k0, 12 * ks) << 8) + lut_sel_src;
            ib = (bits6(cur.k0, 12 * ks + 6) << 8) + lut_sel_src;
            ic = (bits6(cur.k1, 12 * ks) << 8) + lut_sel_src;
            id = (bits6(cur.k1, 12 * ks + 6) << 8) + lut_sel_src;
        } else {
            ia = prmt(w0, lut_sel_src, 0x5504u | (jA << 4));  // token 2g, dims k-lo
            ib = prmt(w0, lut_sel_src, 0x5504u | (jB << 4));  // token 2g, dims k-hi
            ic = prmt(w1, lut_sel_src, 0x5504u | (jA << 4));  // token 2g+1
            id = prmt(w1, lut_sel_src, 0x5504u | (jB << 4));
        }
        uint2 e0, e1, e2, e3;
        if (!kNormCorr) {
            e0 = lut_v2(lut, ia);
            e1 = lut_v2(lut, ib);
            e2 = lut_v2(lut, ic);
            e3 = lut_v2(lut, id);
        } else {
            const uint4 f0 = lds_v4(lut_base + ia), f1 = lds_v4(lut_base + ib);
            const uint4 f2 = lds_v4(lut_base + ic), f3 = lds_v4(lut_base + id);
            e0 = make_uint2(f0.x, f0.y);
            e1 = make_uint2(f1.x, f1.y);
            e2 = make_uint2(f2.x, f2.y);
            e3 = make_uint2(f3.x, f3.y);
            csq0 += __uint_as_float(f0.z) + __uint_as_float(f1.z);
            csq1 += __uint_as_float(f2.z) + __uint_as_float(f3.z);
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            // A = {C_hi kA, C_lo kA, C_hi kB, C_lo kB}; B = Q columns of dims
            // 32c + 4ks + {0,1 | 2,3}
            mma_16816(dq[nt][0], e0.x, e0.y, e1.x, e1.y, st.qf[nt][2 * ks], st.qf[nt][2 * ks + 1]);
            mma_16816(dq[nt][1], e2.x, e2.y, e3.x, e3.y, st.qf[nt][2 * ks], st.qf[nt][2 * ks + 1]);
        }
    }
    }  // 4-bit keys
    float kn0 = half_bits_to_float(cur.kn), kn1 = half_bits_to_float(cur.kn >> 16);
    if (kNormCorr) {
        // Norm correction c / |c| (reference/aos_decode.py:199-206).
        csq0 = warp_sum_xor(csq0, 1, 2);
        csq1 = warp_sum_xor(csq1, 1, 2);
        kn0 = kn0 * rsqrtf(csq0 + 1e-16f);
        kn1 = kn1 * rsqrtf(csq1 + 1e-16f);
    }
    const float vs0 = va ? half_bits_to_float(cur.vs) : 0.0f;
    const float vs1 = vb ? half_bits_to_float(cur.vs >> 16) : 0.0f;
    const float vz0 = va ? half_bits_to_float(cur.vz) : 0.0f;
    const float vz1 = vb ? half_bits_to_float(cur.vz >> 16) : 0.0f;

    // -- online softmax (exp2 domain), exact rescale --
    uint32_t bw0[NT], bw1[NT];
    float alpha[NT];
    bool rescale = false;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        // columns 2c / 2c+1: Q_hi / Q_lo parts of head c; rows g / g+8:
        // C_hi / C_lo parts of the token
        // FP8 keys: columns 2c / 2c+1 = Q_hi / Q_lo of head c, rows g / g+8
        // = tokens 2g / 2g+1, chains ks even / odd
        const float d0 = layout_fp8_keys(LAYOUT)
                             ? (dq[nt][0][0] + dq[nt][0][1]) + (dq[nt][1][0] + dq[nt][1][1])
                             : (dq[nt][0][0] + dq[nt][0][2]) + (dq[nt][0][1] + dq[nt][0][3]);
        const float d1 = layout_fp8_keys(LAYOUT)
                             ? (dq[nt][0][2] + dq[nt][0][3]) + (dq[nt][1][2] + dq[nt][1][3])
                             : (dq[nt][1][0] + dq[nt][1][2]) + (dq[nt][1][1] + dq[nt][1][3]);
        float s0 = d0 * kn0 * st.kfac[nt];
        float s1 = d1 * kn1 * st.kfac[nt];
        s0 = va ? s0 : -INFINITY;
        s1 = vb ? s1 : -INFINITY;
        const float tmax = warp_max_xor(fmaxf(s0, s1), 4, 16);
        const float mold = st.m_run[nt];
        // Lazy reference max: it only moves when a score exceeds it by more
        // than kLazy (log2 units), so most pages need no rescale; p <= 2^kLazy.
        float mref = tmax > mold + kLazy ? tmax : mold;
        float mref_e = mref == -INFINITY ? 0.0f : mref;  // page with no valid token
        float p0 = ex2(s0 - mref_e), p1 = ex2(s1 - mref_e);
        float w0 = p0 * vs0, w1 = p1 * vs1;
        // W must stay inside fp16: a huge V scale falls back to the exact max.
        if (__any_sync(0xffffffffu, fmaxf(w0, w1) > kWMax)) {
            mref = fmaxf(mold, tmax);
            mref_e = mref == -INFINITY ? 0.0f : mref;
            p0 = ex2(s0 - mref_e);
            p1 = ex2(s1 - mref_e);
            w0 = p0 * vs0;
            w1 = p1 * vs1;
        }
        // The first page has nothing to rescale (accumulators are 0).
        alpha[nt] = (mold == -INFINITY || mref == mold) ? 1.0f : ex2(mold - mref);
        rescale |= alpha[nt] != 1.0f;
        st.l_part[nt] = st.l_part[nt] * alpha[nt] + (p0 + p1);
        st.z_part[nt] = st.z_part[nt] * alpha[nt] + (p0 * vz0 + p1 * vz1);
        st.m_run[nt] = mref;
        const __half2 wh = __floats2half2_rn(w0, w1);
        const __half2 wl = __floats2half2_rn(w0 - __low2float(wh), w1 - __high2float(wh));
        // Transpose W into the B fragment of P.V: lane (g, c) takes tokens
        // {4c, 4c+1} from lane 8c + (g>>1) and {4c+2, 4c+3} from lane
        // 8c + 4 + (g>>1), part g&1.
        const int srcA = 8 * c + (g >> 1);
        const uint32_t hA = __shfl_sync(0xffffffffu, h2_as_u32(wh), srcA);
        const uint32_t lA = __shfl_sync(0xffffffffu, h2_as_u32(wl), srcA);
        const uint32_t hB = __shfl_sync(0xffffffffu, h2_as_u32(wh), srcA + 4);
        const uint32_t lB = __shfl_sync(0xffffffffu, h2_as_u32(wl), srcA + 4);
        bw0[nt] = (g & 1) ? lA : hA;
        bw1[nt] = (g & 1) ? lB : hB;
    }
    if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int k = 0; k < 4; k++) st.acc[nt][i][k] *= alpha[nt];
    }

    // -- P.V on the tensor cores; codes enter as exact fp16 subnormals --
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int wi = i >> 2, bi = i & 3;
        const uint32_t sel = (uint32_t)(bi | (bi << 4) | ((4 + bi) << 8) | ((4 + bi) << 12));
        const uint32_t x0 = wi ? cur.v[0].y : cur.v[0].x;
        const uint32_t x1 = wi ? cur.v[1].y : cur.v[1].x;
        const uint32_t x2 = wi ? cur.v[2].y : cur.v[2].x;
        const uint32_t x3 = wi ? cur.v[3].y : cur.v[3].x;
        const uint32_t p01 = prmt(x0, x1, sel), p23 = prmt(x2, x3, sel);
        // Both nibbles enter as code * 2^-20 (mantissa bits 4-7): the
        // tensor cores keep these subnormals exact, while codes at 2^-24
        // lose bits.
        const uint32_t a0 = (p01 << 4) & 0x00F000F0u;  // row g:   low nibble
        const uint32_t a1 = p01 & 0x00F000F0u;         // row g+8: high nibble
        const uint32_t a2 = (p23 << 4) & 0x00F000F0u;
        const uint32_t a3 = p23 & 0x00F000F0u;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) mma_16816(st.acc[nt][i], a0, a1, a2, a3, bw0[nt], bw1[nt]);
    }
}

template <int NT, int LAYOUT>
__global__ void __launch_bounds__(kThreads, NT == 1 ? kMinBlocksNT1 : 1)
    stage1_kernel(const Stage1Params P) {
    // Shared memory: the K table (256 entries x 256 bytes: SoA keeps 32 lane
    // copies of {C_hi pair, C_lo pair}; AoS keeps 16 copies that also carry
    // the byte's squared centroid sum for the in-kernel norm correction),
    // then one output staging row set per warp.
    constexpr bool kNormCorr = layout_is_aos(LAYOUT) && !layout_fp8_keys(LAYOUT);
    constexpr bool kFp8 = layout_fp8_keys(LAYOUT);
    constexpr int kEntry = kNormCorr ? 16 : 8;
    constexpr int kCopies = kLutStride / kEntry;
    extern __shared__ __align__(1024) uint8_t smem[];
    pdl_trigger();
    pdl_wait();  // the kernel before on the stream (e.g. the previous step's Stage2 reading mid_o)
    float* stage_all = reinterpret_cast<float*>(smem + kLutBytes);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;

    // ---- centroid table -------------------------------------------------
    // (FP8 keys need no table: their fp16 form is exact, scale exponent 0.)
    // 3-bit keys: 8 centroids, table entries for the 64 6-bit dim pairs.
    constexpr bool kKey3 = layout_3bit_keys(LAYOUT);
    constexpr int kNc = kKey3 ? 8 : kNumCentroids;
    constexpr int kPairs = kKey3 ? 64 : 256;
    constexpr int kLowBits = kKey3 ? 3 : 4;
    float cmax = 0.0f;
    if (!kFp8) {
#pragma unroll
        for (int k = 0; k < kNc; k++) cmax = fmaxf(cmax, fabsf(__ldg(P.cents + k)));
    }
    const int ec = kFp8 ? 0 : fp16_scale_exp(cmax);
    const float cscale = exp2i(ec);
    for (int e = tid; !kFp8 && e < kPairs * kCopies; e += kThreads) {
        const int byte = e / kCopies;
        const float a = __ldg(P.cents + (byte & (kNc - 1))), b = __ldg(P.cents + (byte >> kLowBits));
        const float clo = a * cscale, chi = b * cscale;
        const __half2 h = __floats2half2_rn(clo, chi);
        const __half2 l = __floats2half2_rn(clo - __low2float(h), chi - __high2float(h));
        uint8_t* dst = smem + (size_t)e * kEntry;
        if (!kNormCorr) {
            *reinterpret_cast<uint2*>(dst) = make_uint2(h2_as_u32(h), h2_as_u32(l));
        } else {
            *reinterpret_cast<uint4*>(dst) =
                make_uint4(h2_as_u32(h), h2_as_u32(l), __float_as_uint(a * a + b * b), 0u);
        }
    }
    __syncthreads();

    const uint32_t lut_base = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    // PRMT source: byte 0 = this lane's copy offset inside an entry, byte 1 = 0.
    const uint32_t lut_sel_src = (uint32_t)(lane % kCopies) * kEntry;
    float* stage = stage_all + warp * (NT * 4 * (kHeadDim + 1));

    // Work item -> (b, s, kvh) and its token range; false for an empty split.
    struct ItemRange { int b, s, kvh, start, end; };
    auto decode_item = [&](uint32_t item, ItemRange& r) {
        const uint32_t rest = P.div_hk.div(item);
        r.kvh = (int)(item - rest * (uint32_t)P.Hk);
        const uint32_t bq = P.div_s.div(rest);
        r.s = (int)(rest - bq * (uint32_t)P.S);
        r.b = (int)bq;
        const int nsp = P.nsplits ? min(__ldg(P.nsplits + r.b), P.S) : P.S;
        if (r.s >= nsp) return false;
        // Tokens past the block-table row are outside the sequence's pages.
        const int L = min(__ldg(P.seq_lens + r.b), P.max_blocks * kBlockSize);
        const int split_len = (L + nsp - 1) / nsp;
        r.start = split_len * r.s;
        r.end = min(r.start + split_len, L);
        return r.start < r.end;
    };
    const uint32_t nblocks_all = (P.num_blocks > 0 && P.num_blocks < 0x7fffffff) ? (uint32_t)P.num_blocks : 0x7fffffffu;
    const uint32_t item_stride = gridDim.x * kWarps;

    for (uint32_t item = blockIdx.x * kWarps + warp; item < (uint32_t)P.num_items; item += item_stride) {
        ItemRange ir;
        if (!decode_item(item, ir)) continue;  // empty split: left unwritten
        const int b = ir.b, s = ir.s, kvh = ir.kvh, start = ir.start, end = ir.end;
        // Ask L2 for the first two pages of this warp's next item now, so
        // the item boundary does not stall on DRAM.
        {
            ItemRange nx;
            const uint32_t nitem = item + item_stride;
            if (nitem < (uint32_t)P.num_items && decode_item(nitem, nx)) {
                const int np0 = nx.start / kBlockSize, np1 = min(np0 + 1, (nx.end - 1) / kBlockSize);
                const int32_t* nrow = P.bt + (int64_t)nx.b * P.bt_stride;
                const int id0 = __ldg(nrow + np0), id1 = __ldg(nrow + np1);
                const uint32_t bb = (uint32_t)P.block_bytes;
                const bool nlead = lane == 0 && nx.kvh == 0 &&
                                   ((reinterpret_cast<uintptr_t>(P.cache) | bb) & 15) == 0;
                if ((uint32_t)id0 < nblocks_all) prefetch_block(P.cache + (uint64_t)(uint32_t)id0 * bb, bb, nlead);
                if ((uint32_t)id1 < nblocks_all && np1 != np0)
                    prefetch_block(P.cache + (uint64_t)(uint32_t)id1 * bb, bb, nlead);
            }
        }

        const int p_first = start / kBlockSize, p_last = (end - 1) / kBlockSize;
        const int32_t* bt_row = P.bt + (int64_t)b * P.bt_stride;
        const LaneOffsets off = lane_offsets<LAYOUT>(P, kvh, lane);
        const uint8_t* cache = P.cache;
        const uint32_t block_bytes = (uint32_t)P.block_bytes;
        const uint32_t nblocks = nblocks_all;
        // One lane per page prefetches whole blocks: lane 0 of the warp of KV
        // head 0 (the warps of a CTA share the (b, s) of their items).  The
        // bulk form needs a 16-byte aligned block.
        const bool pf_leader = lane == 0 && kvh == 0 &&
                               ((reinterpret_cast<uintptr_t>(cache) | block_bytes) & 15) == 0;
        // Block ids of pages [w0, w0 + 32), one per lane; an id outside
        // [0, num_blocks) masks its page, whose loads then read block 0.
        int w0 = p_first;
        int blk_reg = (p_first + lane <= p_last) ? __ldg(bt_row + p_first + lane) : 0;
        auto valid_blk = [&](int id) { return (uint32_t)id < nblocks; };
        auto blk_of = [&](int pp) { return __shfl_sync(0xffffffffu, blk_reg, pp - w0); };
        auto block_ptr = [&](int id) {
            return cache + (uint64_t)(valid_blk(id) ? (uint32_t)id : 0u) * block_bytes;
        };

        // Start the first page's loads before the query prologue.
        PageRegs ra, rb;
        bool ok_a, ok_b = false;
        {
            const int id = blk_of(p_first);
            ok_a = valid_blk(id);
            load_page<LAYOUT>(ra, block_ptr(id), off);
#pragma unroll
            for (int d = 1; d <= kPrefetchPages; d++)
                if (p_first + d <= p_last) prefetch_block(block_ptr(blk_of(p_first + d)), block_bytes, pf_leader);
        }

        // ---- query fragments (B operand of Q.K) --------------------------
        // Lane (g, c) supplies column n = g (head g>>1 of the n-tile, part
        // g&1) for dims 32c .. 32c+31, in k order 32c + 4ks + {0,1 | 2,3}.
        ItemState<NT> st;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int hl = (g >> 1) + 4 * nt;
            float qv[32];
            float amax = 0.0f;
            if (hl < P.G) {
                const float* qp = P.q + (int64_t)b * P.qsb + (int64_t)(kvh * P.G + hl) * P.qsh + 32 * c;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(qp) + j);
                    qv[4 * j] = v.x; qv[4 * j + 1] = v.y; qv[4 * j + 2] = v.z; qv[4 * j + 3] = v.w;
                }
#pragma unroll
                for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(qv[j]));
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) qv[j] = 0.0f;
            }
            amax = warp_max_xor(amax, 1, 2);
            const int eq = fp16_scale_exp(amax);
            const float qscale = exp2i(eq);
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const float x0 = qv[2 * j] * qscale, x1 = qv[2 * j + 1] * qscale;
                const __half2 h = __floats2half2_rn(x0, x1);
                const __half2 l = __floats2half2_rn(x0 - __low2float(h), x1 - __high2float(h));
                st.qf[nt][j] = (g & 1) ? h2_as_u32(l) : h2_as_u32(h);
            }
            // Score factor of this lane's softmax head (c + 4 nt), whose
            // scale exponent lives on lane 8c.
            const int eq_head = __shfl_sync(0xffffffffu, eq, 8 * c);
            st.kfac[nt] = P.attn_scale * kLog2e * exp2i(-eq_head) * exp2i(-ec);
            st.m_run[nt] = -INFINITY;
            st.l_part[nt] = 0.0f;
            st.z_part[nt] = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int k = 0; k < 4; k++) st.acc[nt][i][k] = 0.0f;
        }

        // ---- page loop: two-page register ring, L2 prefetch further on ----
        // Issues the loads of page pp into `r` and the L2 prefetch of page
        // pp + kPrefetchPages.
        auto stage_page = [&](PageRegs& r, bool& ok, int pp) {
            if (pp + kPrefetchPages - w0 >= 32) {  // refill the block-id window
                w0 = pp;
                blk_reg = (pp + lane <= p_last) ? __ldg(bt_row + pp + lane) : 0;
            }
            const int id = blk_of(pp);
            ok = valid_blk(id);
            load_page<LAYOUT>(r, block_ptr(id), off);
            if (pp + kPrefetchPages <= p_last)
                prefetch_block(block_ptr(blk_of(pp + kPrefetchPages)), block_bytes, pf_leader);
        };
        for (int p = p_first; p <= p_last; p += 2) {
            if (p + 1 <= p_last) stage_page(rb, ok_b, p + 1);
            process_page<NT, LAYOUT>(st, ra, ok_a, p * kBlockSize + 2 * g, start, end, smem, lut_base,
                                     lut_sel_src, g, c);
            if (p + 1 > p_last) break;
            if (p + 2 <= p_last) stage_page(ra, ok_a, p + 2);
            process_page<NT, LAYOUT>(st, rb, ok_b, (p + 1) * kBlockSize + 2 * g, start, end, smem, lut_base,
                                     lut_sel_src, g, c);
        }

        // ---- epilogue: normalise, stage, coalesced write -------------------
        constexpr float kCodeScale = 1048576.0f;  // 2^20: undo the subnormal code scale
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            float l = warp_sum_xor(st.l_part[nt], 4, 16);
            l = l > 0.0f ? l : 1.0f;  // safe_l (reference/soa_decode_v1.py:311)
            const float z = warp_sum_xor(st.z_part[nt], 4, 16);
            const float inv = rcp_approx(l);
            const int hl = c + 4 * nt;
            float* row = stage + hl * (kHeadDim + 1);
            if (hl < P.G) {
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float lo = (st.acc[nt][i][0] + st.acc[nt][i][1]) * kCodeScale + z;
                    const float hi = (st.acc[nt][i][2] + st.acc[nt][i][3]) * kCodeScale + z;
                    row[16 * g + 2 * i] = lo * inv;
                    row[16 * g + 2 * i + 1] = hi * inv;
                }
                if (g == 0) row[kHeadDim] = (st.m_run[nt] + lg2_approx(l)) * kLn2;
            }
        }
        __syncwarp();
        const int nheads = min(P.G, NT * 4);
        for (int hl = 0; hl < nheads; hl++) {
            float* dst = P.mid + (int64_t)b * P.msb + (int64_t)(kvh * P.G + hl) * P.msh + (int64_t)s * P.mss;
            const float* src = stage + hl * (kHeadDim + 1);
            for (int j = lane; j <= kHeadDim; j += 32) dst[j] = src[j];
        }
        __syncwarp();
    }
}

template <int NT, int LAYOUT>
int launch_t(const Stage1Params& P, cudaStream_t stream, int num_sms) {
    const size_t smem = kLutBytes + (size_t)kWarps * NT * 4 * (kHeadDim + 1) * sizeof(float);
    auto kern = stage1_kernel<NT, LAYOUT>;
    static thread_local int configured_dev = -1;  // per template instance
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return report_launch(cudaGetLastError());
        configured_dev = dev;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    const int64_t need = (P.num_items + kWarps - 1) / kWarps;
    const int64_t grid = need < (int64_t)num_sms * per_sm ? need : (int64_t)num_sms * per_sm;
    if (grid <= 0) return TQB_OK;
    return report_launch(launch_pdl(kern, dim3((unsigned)grid), dim3(kThreads), smem, stream, P));
}

}  // namespace

// TQB_STAGE1_KERNEL=regs selects the register-ring kernel for an SoA cache
// too (the TMA page-ring kernel is the default there); read on every call.
bool stage1_register_kernel_forced() {
    const char* v = getenv("TQB_STAGE1_KERNEL");
    return v != nullptr && strcmp(v, "regs") == 0;
}

int launch_stage1(const Stage1Params& P, cudaStream_t stream, int num_sms) {
    if (stage1_ring_supported(P) && !stage1_register_kernel_forced()) {
        const int rc = launch_stage1_ring(P, stream, num_sms);
        if (rc != TQB_ERR_UNSUPPORTED) return rc;  // else: tensor maps refused, use the register kernel
    }
    switch (P.layout) {
        case TQB_LAYOUT_AOS_K8:
            return P.G <= 4 ? launch_t<1, TQB_LAYOUT_AOS_K8>(P, stream, num_sms)
                            : launch_t<2, TQB_LAYOUT_AOS_K8>(P, stream, num_sms);
        case TQB_LAYOUT_AOS_K3:
            return P.G <= 4 ? launch_t<1, TQB_LAYOUT_AOS_K3>(P, stream, num_sms)
                            : launch_t<2, TQB_LAYOUT_AOS_K3>(P, stream, num_sms);
        case TQB_LAYOUT_AOS_K3V3:
            return P.G <= 4 ? launch_t<1, TQB_LAYOUT_AOS_K3V3>(P, stream, num_sms)
                            : launch_t<2, TQB_LAYOUT_AOS_K3V3>(P, stream, num_sms);
        default:
            break;
    }
    if (P.layout == TQB_LAYOUT_SOA_K8)
        return P.G <= 4 ? launch_t<1, TQB_LAYOUT_SOA_K8>(P, stream, num_sms)
                        : launch_t<2, TQB_LAYOUT_SOA_K8>(P, stream, num_sms);
    if (P.layout == TQB_LAYOUT_SOA_K3)
        return P.G <= 4 ? launch_t<1, TQB_LAYOUT_SOA_K3>(P, stream, num_sms)
                        : launch_t<2, TQB_LAYOUT_SOA_K3>(P, stream, num_sms);
    if (P.layout == TQB_LAYOUT_SOA_K3V3)
        return P.G <= 4 ? launch_t<1, TQB_LAYOUT_SOA_K3V3>(P, stream, num_sms)
                        : launch_t<2, TQB_LAYOUT_SOA_K3V3>(P, stream, num_sms);
    const bool soa = P.layout == TQB_LAYOUT_SOA;
    if (P.G <= 4) return soa ? launch_t<1, TQB_LAYOUT_SOA>(P, stream, num_sms)
                             : launch_t<1, TQB_LAYOUT_AOS>(P, stream, num_sms);
    return soa ? launch_t<2, TQB_LAYOUT_SOA>(P, stream, num_sms)
               : launch_t<2, TQB_LAYOUT_AOS>(P, stream, num_sms);
}

}  // namespace tqb
