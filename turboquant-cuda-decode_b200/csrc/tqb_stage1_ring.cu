// tqb_stage1_ring.cu — sm_100a Stage1 for the SoA cache, fed by a TMA page ring.
//
// Same result as the register-ring kernel in tqb_stage1.cu (reference:
// reference/soa_decode_v1.py:43-314): per (sequence b, query head h, split s)
// the normalised partial output and natural-log LSE of the split's tokens.
//
// Structure (one CTA per SM, persistent):
//  * A CTA holds kGroups groups.  A group is 8 compute warps plus one
//    producer warp.  The group walks "tiles" of 8 consecutive work items
//    (b, s, KV head; head fastest), one item per compute warp, so with Hk = 8
//    the 8 warps share every page of one (b, s) split.
//  * The producer warps (two per group) move each page of the tile into a kStages-deep
//    shared-memory ring with TMA (CTA-local loads only): one cp.async.bulk.tensor of
//    the tile's head slices (a 4-D tensor map over [block][head][token][128 B]
//    with a box of {128 B, 16 tokens, 8 heads}; narrower runs use boxes of
//    4/2/1 heads) plus one cp.async.bulk of their metadata, all completing on
//    the stage's "full" mbarrier.  The compute warps release a
//    stage through its "empty" mbarrier.  Loads therefore need no registers
//    and no per-page address arithmetic in the compute warps, and up to
//    kStages pages per group are in flight, independently of the math.
//  * In shared memory a head's 16 token rows are one 2 KB column, written
//    with the 128-byte swizzle (16-byte chunk j of token t lands at chunk
//    j ^ (t & 7)).  The compute lanes own tokens tau(g) =
//    {0,4,2,6,8,12,10,14}[g] and tau(g)+1, so every K (LDS.128), V (LDS.64)
//    and metadata load of a page is free of bank conflicts; the PV operand
//    tokens of lane (g, c) are then {2c, 2c+1, 2c+8, 2c+9}, the natural k
//    order of mma.m16n8k16.
//  * The tile's query rows (fp32, one tensor copy of G rows per item) land in
//    a per-group query area with its own full/empty barrier pair, ahead of
//    the tile.
//  * The math per page is the register kernel's: Q.K and P.V on the tensor
//    cores with fp16 hi/lo splits (fp32-accurate), online softmax in the
//    exp2 domain with a lazy reference max.
//  * Every mbarrier wait is bounded (kWaitCycles); a wait that runs out bumps
//    a device counter (tqb_wait_timeouts) and the warp leaves its loops, so a
//    protocol fault ends the kernel instead of hanging the GPU.
#include <cuda.h>  // CUtensorMap and its enums; the encoder is fetched at run time
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "tqb_common.cuh"
#include "tqb_internal.h"

namespace tqb {

// Number of bounded mbarrier waits that ran out (read by tqb_wait_timeouts).
__device__ unsigned int g_wait_timeouts = 0;
// Grid barrier of the fused query rotation (stage1 with rot != nullptr): the
// cooperative-groups arrival scheme, block 0 adds 2^31 - (grid - 1) and every
// other block 1, so bit 31 flips once per launch and the word never needs a
// reset.  Two such launches never interleave their arrivals: each is a
// cooperative launch of one CTA per SM, so the next starts only after every
// CTA of the previous one has ended.
__device__ unsigned int g_rot_barrier = 0;

namespace {

constexpr int kGroupWarps = 8;                                 // compute warps per group
constexpr int kColBytes = kBlockSize * kDataBytes;             // 2048: one head's page column
constexpr int kMetaSlot = 3 * kBlockSize * 2;                  // 96 B: knorm, vscale, vzero
constexpr int kMetaOff = kGroupWarps * kColBytes;              // 16384
constexpr int kStageBytes = 17408;                             // data + metadata, 1024-aligned
static_assert(kMetaOff + kGroupWarps * kMetaSlot <= kStageBytes && kStageBytes % 1024 == 0, "stage");
constexpr int kQRowBytes = kHeadDim * 4;                       // one fp32 query row
constexpr int kStgBytes = 2 * kQRowBytes;                      // per-warp output staging
constexpr int kLutStride = 256;                                // bytes per table entry
constexpr int kLutCopies = 32;                                 // one copy per lane
constexpr int kAosSlot = 134;                                   // AoS bytes per (token, head)
constexpr int kAosHead = kBlockSize * kAosSlot;                 // 2144: one head's slots of a page
constexpr int kK8Head = kBlockSize * kSlotBytesK8;              // 3136: one head's share of an FP8-key block
constexpr int kK8StageBytes = 25600;                           // 8 x 3136, 1024-aligned
static_assert(kGroupWarps * kK8Head <= kK8StageBytes && kK8StageBytes % 1024 == 0, "FP8-key stage");
// Bytes of one ring stage, and of one head's page in it (SoA: 2048 data +
// 96 metadata, AoS: 16 slots, FP8 keys: 16 x 192 data + 64 metadata, 3-bit
// keys: 16 x 112 (or 96 with 3-bit values) data + 96 metadata).
// Both families of a preset take the same bytes per (token, head), so a
// head's page is 16 slots' worth: 2144 (4-bit), 3136 (FP8 keys), 1888 (3-bit
// keys) or 1632 (3-bit keys and values).
__host__ __device__ constexpr int stage_bytes(int layout) {
    return layout_fp8_keys(layout) ? kK8StageBytes : kStageBytes;
}
__host__ __device__ constexpr int head_page_bytes(int layout) { return kBlockSize * aos_slot_bytes(layout); }
static_assert(head_page_bytes(TQB_LAYOUT_SOA_K8) == kK8Head && head_page_bytes(TQB_LAYOUT_AOS) == kAosHead &&
                  kBlockSize * kSlotBytesK3 == head_page_bytes(TQB_LAYOUT_SOA_K3) &&
                  kBlockSize * kSlotBytesK3V3 == head_page_bytes(TQB_LAYOUT_SOA_K3V3),
              "head page bytes");
// Shared-memory bytes per head of a page: 3-bit-key blocks land row by row,
// token row t at t * row + 16 * (t >> 1) (112 bytes of padding in all), so
// that the eight token rows tau(g) the compute warps read at once start 4
// banks apart (a whole block copied unchanged has rows 896 or 768 bytes
// apart, all on the same banks).
constexpr int kK3RowPad = 16 * (kBlockSize / 2 - 1);  // 112
__host__ __device__ constexpr int head_stride_bytes(int layout) {
    return layout == TQB_LAYOUT_SOA_K3 || layout == TQB_LAYOUT_SOA_K3V3 ? head_page_bytes(layout) + kK3RowPad
                                                                        : head_page_bytes(layout);
}
static_assert(kGroupWarps * head_stride_bytes(TQB_LAYOUT_SOA_K3) <= kStageBytes &&
                  head_stride_bytes(TQB_LAYOUT_SOA_K3) % 16 == 0 && head_stride_bytes(TQB_LAYOUT_SOA_K3V3) % 16 == 0,
              "3-bit-key stage");
static_assert(kBlockSize * kDataBytes + kMetaSlot == kAosHead, "SoA and AoS heads take the same page bytes");
constexpr int kLutBytes = 256 * kLutStride;                    // 64 KB
constexpr int kLutAddr = 0x10000;                              // shared address of the table
constexpr int kDynBase = 0x400;  // shared address of dynamic shared memory (1 KB reserved below it)
constexpr int kBarStride = 128;                                // barrier block per group
constexpr int kProducersPerGroup = 2;  // the issue handoff is unambiguous for two
constexpr int kSplitCost = 16;         // per-split weight in tokens (query rows, epilogue)
constexpr long long kWaitCycles = 2000000000LL;                // ~1 s at 1.9 GHz
constexpr float kLazy = 8.0f;                                  // lazy-rescale slack (log2)
constexpr float kWMax = 32768.0f;                              // largest W on the lazy path

// Warp roles: kGroups x 8 compute warps (whole warpgroups) and one producer
// warpgroup whose warps feed the groups, two per group taking turns page by
// page.
// setmaxnreg moves registers from the producer warpgroup to the compute
// warpgroups; the shares add up to at most the launch allocation
// (kThreads x kLaunchRegs), so every setmaxnreg.inc can be satisfied.
template <int NT, int LAYOUT = TQB_LAYOUT_SOA>
struct Cfg {
    static constexpr bool kTable = !layout_fp8_keys(LAYOUT);  // FP8 keys convert without the K table
    static constexpr int kGroups = NT == 1 ? 2 : 1;
    static constexpr int kStages = 3;
    static constexpr int kHeadsPerWarp = 4 * NT;
    static constexpr int kQBytes = kGroupWarps * kHeadsPerWarp * kQRowBytes;
    static constexpr int kRingBytes = kStages * stage_bytes(LAYOUT);
    static constexpr int kComputeWarps = kGroups * kGroupWarps;
    static constexpr int kWarps = kComputeWarps + 4;
    static constexpr int kThreads = kWarps * 32;
    static constexpr int kLaunchRegs = NT == 1 ? 96 : 168;     // 65536 / kThreads, rounded down to 8
    static constexpr int kProducerRegs = 32;
    static constexpr int kComputeRegs = NT == 1 ? 112 : 232;
    static_assert(kThreads * kLaunchRegs <= 65536, "launch registers");
    static_assert(kComputeWarps * 32 * kComputeRegs + 128 * kProducerRegs <= kThreads * kLaunchRegs,
                  "register split exceeds the launch allocation");
    // Dynamic shared memory, which starts at shared address kDynBase: the K
    // table sits at shared address 0x10000, so a PRMT of (table page 0x01,
    // K byte, lane copy offset) is its complete LDS address.  Below it: group
    // 0's ring and the barrier blocks; above it: the query areas and group
    // 1's ring.  Every ring stage and query area is 1024-byte aligned.
    // Without the table (FP8 keys) the query areas start at the first 1 KB
    // boundary after the barrier blocks.
    static constexpr int kLutOff = kLutAddr - kDynBase;            // 64512
    static constexpr int kBarOff = kRingBytes;                     // after group 0's ring
    static constexpr int kHighOff = kTable ? kLutOff + kLutBytes   // 130048
                                           : (kBarOff + kGroups * kBarStride + 1023) / 1024 * 1024;
    static __host__ __device__ constexpr int ring_off(int gi) { return gi == 0 ? 0 : kHighOff + kQBytes; }
    static __host__ __device__ constexpr int q_off(int gi) { return gi == 0 ? kHighOff : kHighOff + kQBytes + kRingBytes; }
    // Output staging: 1 KB per compute warp (two fp32 rows of 128) after the
    // rest, never written by a copy engine.
    static constexpr int kStgOff = kGroups == 1 ? kHighOff + kQBytes : kHighOff + 2 * kQBytes + kRingBytes;
    static constexpr int kSmem = kStgOff + kComputeWarps * kStgBytes;
    static_assert(!kTable || kBarOff + kGroups * kBarStride <= kLutOff, "barriers below the table");
    static_assert(8 * (2 * kStages + 2) + 4 * kStages + 12 <= 96 && 96 + 12 <= kBarStride, "barrier block");
    static_assert((16 * kStages + 16 + 4 * kStages + 4) % 8 == 0, "handoff barrier alignment");
    static_assert(kSmem <= 232448, "shared memory per CTA");
};

// Tensor maps of one launch (kernel parameters, __grid_constant__):
// page[i] covers the SoA data region as [block][head][token][128 B] (dims
// innermost first: 128 B, token, head, block) with a box of 8 >> i heads and
// the 128-byte swizzle; query covers q_rot as [B][Hq][128 fp32] with a box of
// G rows.
struct RingMaps {
    CUtensorMap page[4];
    CUtensorMap query;
};

// ---- mbarrier / bulk-copy primitives (PTX ISA 8.x, sm_90+) -----------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits until every lane has observed the completion of the phase of `bar`
// with the given parity.  Warp-uniform result: false (and one count in
// g_wait_timeouts per warp) when kWaitCycles pass first.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    const long long t0 = clock64();
    for (uint32_t i = 1;; i++) {
        if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
        // the clock bound is checked every 64 polls (each try_wait already
        // holds the warp for a while when the phase is incomplete)
        if ((i & 63u) == 0 && __any_sync(0xffffffffu, clock64() - t0 > kWaitCycles)) {
            if ((threadIdx.x & 31) == 0) atomicAdd(&g_wait_timeouts, 1u);
            return false;
        }
    }
}
// Global -> shared bulk copy completing on `bar` (16-byte aligned, size a
// multiple of 16).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;\n" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
// Tensor-map copies (global -> shared, completing on `bar`).
// The page data is read exactly once: its copies carry an L2 evict-first
// policy so the stream does not push the partials (mid_o, read back by
// Stage2 right after) out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3, %4, %5}], [%6], %7;\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4}], [%5];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
        : "memory");
}
// Table entry at a shared address (the table is constant once built).
__device__ __forceinline__ uint2 lut_ld(uint32_t a) {
    uint2 r;
    asm("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "r"(a));
    return r;
}

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
    return r;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 r;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "r"(a));
    return r;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t r;
    asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(r) : "r"(a));
    return r;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    unsigned short r;
    asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(r) : "r"(a));
    return r;
}
// 16 / 8 bytes at a 2-byte aligned shared address (AoS slots are 134 bytes):
// the covering aligned words, funnel-shifted into place.
__device__ __forceinline__ uint4 lds128_a2(uint32_t a) {
    const uint32_t b = a & ~3u, sh = (a & 3u) * 8u;
    const uint32_t w0 = lds32(b), w1 = lds32(b + 4), w2 = lds32(b + 8), w3 = lds32(b + 12), w4 = lds32(b + 16);
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                      __funnelshift_r(w3, w4, sh));
}
// 4-byte-aligned reads (AoS FP8-key slots are 196 bytes).
__device__ __forceinline__ uint4 lds128_a4(uint32_t a) {
    return make_uint4(lds32(a), lds32(a + 4), lds32(a + 8), lds32(a + 12));
}
__device__ __forceinline__ uint2 lds64_a4(uint32_t a) { return make_uint2(lds32(a), lds32(a + 4)); }
// 12 bytes at a 2-byte-aligned address (AoS 3-bit key codes), in .x .. .z.
__device__ __forceinline__ uint4 lds96_a2(uint32_t a) {
    const uint32_t b = a & ~3u, sh = (a & 3u) * 8u;
    const uint32_t w0 = lds32(b), w1 = lds32(b + 4), w2 = lds32(b + 8), w3 = lds32(b + 12);
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh), 0u);
}
__device__ __forceinline__ uint2 lds64_a2(uint32_t a) {
    const uint32_t b = a & ~3u, sh = (a & 3u) * 8u;
    const uint32_t w0 = lds32(b), w1 = lds32(b + 4), w2 = lds32(b + 8);
    return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}
__device__ __forceinline__ float4 lds_f4(uint32_t a) {
    const uint4 u = lds128(a);
    return make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Work item -> (b, s, KV head) and its token range [start, end); false when
// the item does not exist or its split is empty (left unwritten).
struct ItemInfo {
    int b, s, kvh, start, end;
};
__device__ __forceinline__ bool decode_item(const Stage1Params& P, uint32_t item, ItemInfo& r) {
    r.b = r.s = r.kvh = r.start = r.end = 0;
    if (item >= (uint32_t)P.num_items) return false;
    const uint32_t rest = P.div_hk.div(item);
    r.kvh = (int)(item - rest * (uint32_t)P.Hk);
    const uint32_t bq = P.div_s.div(rest);
    r.s = (int)(rest - bq * (uint32_t)P.S);
    r.b = (int)bq;
    const int nsp = P.nsplits ? min(__ldg(P.nsplits + r.b), P.S) : P.S;
    if (r.s >= nsp) return false;
    const int L = min(__ldg(P.seq_lens + r.b), P.max_blocks * kBlockSize);
    // ceil(L / nsp); the uniform split count divides by its invariant divisor
    const int split_len = P.nsplits ? (L + nsp - 1) / nsp : (int)P.div_s.div((uint32_t)(L + nsp - 1));
    r.start = split_len * r.s;
    r.end = min(r.start + split_len, L);
    return r.start < r.end;
}

// Lanes 0-7 decode the 8 items of tile t (lane l: item 8t + l); returns the
// lane's page count (0 for lanes >= 8 and empty items) in `np` and the
// tile's page count (max over its items) as the result.
__device__ __forceinline__ int tile_items(const Stage1Params& P, uint32_t t, int lane, ItemInfo& ir, int& np) {
    np = 0;
    if (lane < kGroupWarps && decode_item(P, t * kGroupWarps + lane, ir))
        np = (ir.end - 1) / kBlockSize - ir.start / kBlockSize + 1;
    else
        ir.b = ir.s = ir.kvh = ir.start = ir.end = 0;
    int m = np;
#pragma unroll
    for (int o = 1; o < kGroupWarps; o <<= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    return __shfl_sync(0xffffffffu, m, 0);  // uniform over the warp
}

// ---------------------------------------------------------------------------
// Balanced tile ranges.  The items (b, s, KV head) in order are weighted and
// cut into gridDim.x * kGroups ranges of equal weight; group g takes the
// tiles whose first item starts inside its range: a contiguous run of tiles.
// Weights: with many tiles per group, each item weighs its split's token
// count plus kSplitCost, so ranges carry about equal work whatever the
// spread of sequence lengths; with at most two non-empty tiles per group
// (a small batch, e.g. one rank's share of a data-parallel batch), each
// non-empty item weighs 1, so every group takes one or two tiles: equal
// token weights would let a range catch a short tile and a long one.  Empty
// splits weigh nothing either way.  Every CTA derives the same cut from
// seq_lens (and nsplits), so no state is shared between CTAs or launches.
// ---------------------------------------------------------------------------
struct SeqSplit {
    int L, sl, ne;  // clamped length, split length, non-empty splits
};
__device__ __forceinline__ SeqSplit seq_split_of(const Stage1Params& P, int len, int nsplit) {
    SeqSplit r{0, 1, 0};
    const int nsp = min(nsplit, P.S);
    const int L = min(len, P.max_blocks * kBlockSize);
    if (nsp <= 0 || L <= 0) return r;
    r.L = L;
    r.sl = (L + nsp - 1) / nsp;  // ceil(L / nsp), the split rule of decode_item
    r.ne = (L + r.sl - 1) / r.sl;
    return r;
}
__device__ __forceinline__ SeqSplit seq_split(const Stage1Params& P, int b) {
    return seq_split_of(P, __ldg(P.seq_lens + b), P.nsplits ? __ldg(P.nsplits + b) : P.S);
}
__device__ __forceinline__ long long seq_weight(const Stage1Params& P, const SeqSplit& q, bool by_count) {
    return by_count ? (long long)P.Hk * q.ne : (long long)P.Hk * ((long long)q.L + (long long)kSplitCost * q.ne);
}
__device__ __forceinline__ long long warp_sum_ll(long long v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
// Tile of the first item of sequence b whose start weight reaches r (>= 1,
// at most the sequence's weight): split s* = the last split starting below
// r, then the KV head in it.
__device__ __forceinline__ uint32_t cut_tile(const Stage1Params& P, const SeqSplit& q, int b, long long r,
                                             uint32_t num_tiles, bool by_count) {
    const long long unit = by_count ? (long long)P.Hk : (long long)P.Hk * (q.sl + kSplitCost);
    const long long ss = min((long long)(q.ne - 1), (r - 1) / unit);
    const long long a = unit * ss;
    const long long per =
        by_count ? 1 : (long long)(min((int)(ss + 1) * q.sl, q.L) - (int)ss * q.sl) + kSplitCost;
    const long long kv = (r - a + per - 1) / per;  // in [1, Hk]
    const long long item = ((long long)b * P.S + ss) * P.Hk + kv;
    return (uint32_t)min((long long)num_tiles, (item + kGroupWarps - 1) / kGroupWarps);
}
// Tile walk of group gi of this CTA: tiles first, first + stride, ... below
// end, in res[0..2].  A batch whose sequences all have the same length and
// split count is cut into equal contiguous tile ranges (already balanced;
// consecutive tiles are consecutive splits of one sequence, so the compute
// warps keep their query fragments across them); any other batch takes the
// contiguous ranges of the weight cut.  One warp (compact loops:
// this code runs once, cold, ahead of every other warp's first tile).
__device__ void tile_walk(const Stage1Params& P, int gi, int groups_per_cta, uint32_t num_tiles, uint32_t (&res)[3],
                          int lane) {
    const uint32_t cuts = gridDim.x * (uint32_t)groups_per_cta;
    const uint32_t g = blockIdx.x * (uint32_t)groups_per_cta + (uint32_t)gi;
    long long tot = 0, cnt = 0;
    int lmin = 0x7fffffff, lmax = -0x7fffffff, nmin = 0x7fffffff, nmax = -0x7fffffff;
#pragma unroll 1
    for (int b0 = 0; b0 < P.B; b0 += 32) {
        const int b = b0 + lane;
        if (b < P.B) {
            const int len = __ldg(P.seq_lens + b), nsp = P.nsplits ? __ldg(P.nsplits + b) : P.S;
            const SeqSplit q = seq_split_of(P, len, nsp);
            tot += seq_weight(P, q, false);
            cnt += seq_weight(P, q, true);
            lmin = min(lmin, len);
            lmax = max(lmax, len);
            nmin = min(nmin, nsp);
            nmax = max(nmax, nsp);
        }
    }
    tot = warp_sum_ll(tot);
    cnt = warp_sum_ll(cnt);
    if (__reduce_min_sync(0xffffffffu, lmin) == __reduce_max_sync(0xffffffffu, lmax) &&
        __reduce_min_sync(0xffffffffu, nmin) == __reduce_max_sync(0xffffffffu, nmax)) {
        // contiguous ranges: consecutive tiles of a group are consecutive
        // splits of one sequence, so its warps keep their query fragments
        res[0] = (uint32_t)((uint64_t)g * num_tiles / cuts);
        res[1] = (uint32_t)((uint64_t)(g + 1) * num_tiles / cuts);
        res[2] = 1u;
        return;
    }
    res[2] = 1u;
    const bool by_count = cnt <= 2LL * kGroupWarps * (long long)cuts;  // <= 2 non-empty tiles per group
    if (by_count) tot = cnt;
    const long long qt = tot / (long long)cuts, rt = tot % (long long)cuts;
#pragma unroll 1
    for (int k = 0; k < 2; k++) {
        // cut g + k: the tile of the first item whose start weight reaches
        // floor((g + k) * tot / cuts); weight 0 is tile 0, the last cut (or
        // every cut when nothing has a token) the end
        const uint32_t gk = g + (uint32_t)k;
        const long long tgt = qt * gk + rt * gk / (long long)cuts;  // no overflow
        uint32_t t = num_tiles;
        if (tot > 0 && gk < cuts && tgt == 0) t = 0;
        if (tot > 0 && gk < cuts && tgt > 0) {
            long long base = 0;
#pragma unroll 1
            for (int b0 = 0; b0 < P.B; b0 += 32) {
                const int b = b0 + lane;
                SeqSplit q{0, 1, 0};
                if (b < P.B) q = seq_split(P, b);
                const long long w = seq_weight(P, q, by_count);
                long long incl = w;
#pragma unroll 1
                for (int o = 1; o < 32; o <<= 1) {
                    const long long v = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += v;
                }
                const long long excl = base + incl - w;
                const bool here = w > 0 && excl < tgt && tgt <= base + incl;
                const uint32_t m = __ballot_sync(0xffffffffu, here);
                if (m) {
                    const uint32_t tl = here ? cut_tile(P, q, b, tgt - excl, num_tiles, by_count) : 0u;
                    t = __shfl_sync(0xffffffffu, tl, __ffs(m) - 1);
                    break;
                }
                base += __shfl_sync(0xffffffffu, incl, 31);
            }
        }
        res[k] = t;
    }
}

// Shared-memory map of one group.
struct GroupSmem {
    uint32_t ring, qarea, bars, stg;
    template <int LAYOUT>
    __device__ uint32_t stage(int s) const { return ring + (uint32_t)s * (uint32_t)stage_bytes(LAYOUT); }
    __device__ uint32_t full(int s) const { return bars + 8u * s; }
    template <int NS>
    __device__ uint32_t empty(int s) const { return bars + 8u * (NS + s); }
    template <int NS>
    __device__ uint32_t q_full() const { return bars + 16u * NS; }
    template <int NS>
    __device__ uint32_t q_empty() const { return bars + 16u * NS + 8; }
    template <int NS>
    __device__ uint32_t vmask(int s) const { return bars + 16u * NS + 16 + 4u * s; }
    // Issue-order handoff between the group's producers: phase G completes
    // when page G (counted over all tiles) has been announced on its slot.
    template <int NS>
    __device__ uint32_t issued() const { return bars + 16u * NS + 16 + 4u * NS + 4u; }
    // The group's tile walk {first, end, stride} (written once before the
    // roles split).
    __device__ uint32_t tiles() const { return bars + 96u; }
};

// ---------------------------------------------------------------------------
// Fused query rotation (P.rot set; the one-group-per-warpgroup layout, GQA
// <= 4): before the roles split, the CTA computes rows [r0, r1) of
// q_out = float(rq) @ rot (an equal share of the B * Hq rows per CTA) with
// the arithmetic of the rotation kernel (tqb_rotate.cu: fp32 FMAs in k order,
// so the rows are bit-identical to it).  rot (64 KB) is staged in group 1's
// ring and query area, the input rows in group 0's query area, 32 at a time;
// the producers' TMA copies overwrite both only after the CTA barrier that
// ends the prologue.
// ---------------------------------------------------------------------------
template <int NT>
__device__ void rotate_share(const Stage1Params& P, uint8_t* smem, int tid) {
    using C = Cfg<NT>;
    static_assert(NT == 1, "the fused rotation stages rot in group 1's ring");
    static_assert(C::q_off(1) + C::kQBytes - C::ring_off(1) >= kHeadDim * kHeadDim * 4, "rot staging");
    static_assert(C::kQBytes >= 32 * kQRowBytes, "row staging");
    constexpr int kChunk = 32;
    float* rs = reinterpret_cast<float*>(smem + C::ring_off(1));
    float* qs = reinterpret_cast<float*>(smem + C::q_off(0));
    const int64_t rows = (int64_t)P.B * P.Hq;
    const int64_t per = (rows + gridDim.x - 1) / gridDim.x;
    const int64_t r0 = (int64_t)blockIdx.x * per, r1 = min(rows, r0 + per);
    if (r0 >= r1) return;  // uniform over the CTA
    const float4* R4 = reinterpret_cast<const float4*>(P.rot);
    for (int e = tid; e < kHeadDim * kHeadDim / 4; e += C::kThreads)
        reinterpret_cast<float4*>(rs)[e] = __ldg(R4 + e);
    const int j = tid % kHeadDim;
    for (int64_t c0 = r0; c0 < r1; c0 += kChunk) {
        const int n = (int)min((int64_t)kChunk, r1 - c0);
        __syncthreads();  // rot staged / the previous chunk's rows read
        for (int e = tid; e < n * kHeadDim; e += C::kThreads) {
            const int64_t r = c0 + e / kHeadDim;
            const int64_t off = (r / P.Hq) * P.rqsb + (r % P.Hq) * P.rqsh + e % kHeadDim;
            float v;
            if (P.rq_dtype == TQB_DTYPE_F16)
                v = __half2float(static_cast<const __half*>(P.rq)[off]);
            else if (P.rq_dtype == TQB_DTYPE_BF16)
                v = __bfloat162float(static_cast<const __nv_bfloat16*>(P.rq)[off]);
            else
                v = static_cast<const float*>(P.rq)[off];
            qs[e] = v;
        }
        __syncthreads();
        for (int i = tid / kHeadDim; i < n; i += C::kThreads / kHeadDim) {
            float acc = 0.0f;
#pragma unroll 8
            for (int k = 0; k < kHeadDim; k++) acc = fmaf(qs[i * kHeadDim + k], rs[k * kHeadDim + j], acc);
            const int64_t r = c0 + i;
            P.q_out[(r / P.Hq) * P.qsb + (r % P.Hq) * P.qsh + j] = acc;
        }
    }
}

// Producer 0 of a group, before its first query copy: wait (bounded) until
// every CTA's rotated rows are written (bit 31 of the barrier word differs
// from the value this CTA's arrival saw).
__device__ __forceinline__ bool rot_barrier_wait(uint32_t seen, int lane) {
    int ok = 1;
    if (lane == 0) {
        const long long t0 = clock64();
        for (;;) {
            uint32_t v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(&g_rot_barrier) : "memory");
            if ((v ^ seen) & 0x80000000u) break;
            if (clock64() - t0 > kWaitCycles) {
                atomicAdd(&g_wait_timeouts, 1u);
                ok = 0;
                break;
            }
            __nanosleep(64);
        }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    // the rows came from other CTAs through the generic proxy; the tensor
    // copies that read them are async-proxy operations
    asm volatile("fence.proxy.async.global;\n" ::: "memory");
    return ok != 0;
}

// ---------------------------------------------------------------------------
// Producer warp: query rows and pages of each tile into the group's ring.
// Runs at kProducerRegs registers, so run parameters live one run per lane
// and block ids are fetched one stage ahead into a single register.
// ---------------------------------------------------------------------------
template <int NT, int LAYOUT>
__device__ __forceinline__ void produce(const Stage1Params& P, const RingMaps& M, const GroupSmem& gs, int gi,
                                        int lane, int pj, int npj) {
    using C = Cfg<NT, LAYOUT>;
    constexpr bool kWholeBlock = LAYOUT != TQB_LAYOUT_SOA;  // pages copied as whole blocks
    // ... row by row, rows padded apart (SoA 3-bit keys; AoS slots are copied whole)
    constexpr bool kRowCopies = LAYOUT == TQB_LAYOUT_SOA_K3 || LAYOUT == TQB_LAYOUT_SOA_K3V3;
    constexpr uint32_t kHeadPage = (uint32_t)head_page_bytes(LAYOUT);
    constexpr uint32_t kHeadStride = (uint32_t)head_stride_bytes(LAYOUT);
    constexpr uint32_t kDps = layout_3bit_values(LAYOUT) ? kK3V3DataBytes : kK3DataBytes;
    constexpr int NS = C::kStages;
    const uint32_t t_end = lds32(gs.tiles() + 4u), t_stride = lds32(gs.tiles() + 8u);
    const uint32_t tok_bytes = (uint32_t)P.Hk * kDataBytes;
    const uint32_t nblocks = (P.num_blocks > 0 && P.num_blocks < 0x7fffffff) ? (uint32_t)P.num_blocks : 0x7fffffffu;
    // The group's two producer warps take turns: producer pj copies the pages
    // whose group-wide index is pj (mod 2), and producer 0 also the query rows.  Both
    // walk every page, so the slot phases they track stay exact, and a page
    // is announced on its slot only after the previous page was (the
    // `issued` handoff): every slot's previous use was therefore announced,
    // and its release before that one observed, when a producer waits for a
    // release, so no wait can alias an older phase of the same parity.  The
    // copies themselves are issued after the handoff and overlap.
    // Every tile starts at ring slot 0; bit s of `uses` is the parity of the
    // number of pages slot s has taken so far, `used` marks slots in use.
    uint32_t tq = 0, uses = 0, used = 0;
    uint32_t gpage = 0;  // pages of this group so far, over all tiles
    bool abort = false;
    const uint64_t stream_policy = l2_evict_first_policy();

    // Query rows of a tile (lanes 0-7: its items) into the query area, once
    // the compute warps have released the previous tile's rows.
    auto issue_query = [&](const ItemInfo& x, int npx) {
        if (pj != 0) return true;
        const uint32_t vit = __ballot_sync(0xffffffffu, npx > 0) & 0xFFu;
        if (!mbar_wait(gs.q_empty<NS>(), (tq & 1u) ^ 1u)) return false;
        if (lane == 0) mbar_arrive_tx(gs.q_full<NS>(), (uint32_t)__popc(vit) * P.G * kQRowBytes);
        __syncwarp();
        if (lane < kGroupWarps && npx > 0)  // item `lane`: its G query rows, one tensor copy
            tma_load_3d(gs.qarea + (uint32_t)(lane * C::kHeadsPerWarp) * kQRowBytes, &M.query, 0, x.kvh * P.G, x.b,
                        gs.q_full<NS>());
        tq++;
        return true;
    };
    // Next tile of this group with at least one page (or t >= t_end).
    auto next_tile = [&](uint32_t t, ItemInfo& x, int& npx, int& np_tile) {
        for (; t < t_end; t += t_stride)
            if ((np_tile = tile_items(P, t, lane, x, npx)) > 0) return t;
        return t;
    };

    ItemInfo ir;
    int np = 0, np_tile = 0;
    uint32_t t = next_tile(lds32(gs.tiles()), ir, np, np_tile);
    if (P.rot != nullptr && pj == 0 && t < t_end) {
        // fused rotation: the query rows are written by every CTA's prologue
        const uint32_t base = gs.bars - (uint32_t)gi * kBarStride - C::kBarOff;
        if (!rot_barrier_wait(lds32(base + C::kBarOff + 112u), lane)) abort = true;
    }
    if (t < t_end && !abort && !issue_query(ir, np)) abort = true;
    while (t < t_end && !abort) {
        // The next tile is decoded now; its query rows go out once page 0 of
        // this tile has been released (the compute warps have read this
        // tile's rows by then), well before they are needed.
        ItemInfo irn;
        int npn = 0, np_tile_n = 0;
        const uint32_t tn = next_tile(t + t_stride, irn, npn, np_tile_n);
        // When every item of the next tile keeps its sequence and KV head,
        // the query area already holds its rows (the compute warps keep
        // their fragments): no copy, and no handoff on the query barriers.
        const bool same_rows =
            tn < t_end && __all_sync(0xffffffffu, lane >= kGroupWarps || (np > 0 && npn > 0 && irn.b == ir.b &&
                                                                           irn.kvh == ir.kvh));
        bool next_query_sent = tn >= t_end || same_rows;
        // Runs of consecutive items sharing one (b, s): their head slices are
        // adjacent in every token row, so one copy per row serves a run.
        const int key = np > 0 ? ir.b * P.S + ir.s : -1 - lane;
        const int key_prev = __shfl_up_sync(0xffffffffu, key, 1);
        const int key_next = __shfl_down_sync(0xffffffffu, key, 1);
        const bool leader = np > 0 && (lane == 0 || key_prev != key);
        const bool last = np > 0 && (lane == kGroupWarps - 1 || key_next != key);
        const uint32_t lmask = __ballot_sync(0xffffffffu, leader) & 0xFFu;
        const uint32_t emask = __ballot_sync(0xffffffffu, last) & 0xFFu;
        const int nruns = __popc(lmask);
        // Lane r < nruns describes run r: first warp (column), width, pages,
        // first KV head and block-table position.
        const int col = lane < nruns ? (int)__fns(lmask, 0, lane + 1) : 0;
        const int r_np = __shfl_sync(0xffffffffu, np, col);
        const int r_b = __shfl_sync(0xffffffffu, ir.b, col);
        const int r_pf = __shfl_sync(0xffffffffu, ir.start, col) / kBlockSize;
        const int r_kvh = __shfl_sync(0xffffffffu, ir.kvh, col);
        const int r_nw = lane < nruns ? __ffs(emask >> col) : 0;
        const int32_t* r_bt = P.bt + (int64_t)r_b * P.bt_stride + r_pf;
        const int np_r = lane < nruns ? r_np : 0;
        int next_id = np_r > 0 ? __ldg(r_bt) : 0;

        // ---- pages ---------------------------------------------------------
        int slot = 0;
        for (int k = 0; k < np_tile; k++) {
            const int id = next_id;
            next_id = k + 1 < np_r ? __ldg(r_bt + k + 1) : 0;  // lands while we wait
            const bool here = k < np_r;
            const bool ok = (uint32_t)id < nblocks;
            const uint32_t bytes =
                __reduce_add_sync(0xffffffffu, here ? (uint32_t)r_nw * kHeadPage : 0u);
            const uint32_t vm = __reduce_or_sync(0xffffffffu, (here && ok) ? ((1u << r_nw) - 1u) << col : 0u);
            const uint32_t my_id = ok ? (uint32_t)id : 0u;  // a masked page copies block 0
            if (k == NS && !next_query_sent) {
                if (!issue_query(irn, npn)) { abort = true; break; }
                next_query_sent = true;
            }
            // strict alternation over the group's global page count: each
            // producer's previous page is gpage - 2, so the handoff barrier is
            // at most one phase behind the one waited for
            const bool mine = gpage % (uint32_t)npj == (uint32_t)pj;
            if (mine && gpage > 0 && !mbar_wait(gs.issued<NS>(), (gpage - 1) & 1u)) { abort = true; break; }
            if (mine && !mbar_wait(gs.empty<NS>(slot), ((uses >> slot) & 1u) ^ 1u)) { abort = true; break; }
            if (mine && lane == 0) {
                sts32(gs.vmask<NS>(slot), vm);
                mbar_arrive_tx(gs.full(slot), bytes);
                mbar_arrive(gs.issued<NS>());  // page gpage announced: the next producer may go
            }
            __syncwarp();
            // Lane r < nruns copies run r: its head slices as boxes of 8/4/2/1
            // heads (one box when the run is a whole group) and its metadata
            // (SoA), or its whole block, unchanged, in one bulk copy (AoS and
            // FP8 keys: a run is all Hk heads of one (b, s), Hk dividing 8).
            if (kRowCopies) {
                // 3-bit keys: run r's block as 8 pairs of token rows (rows
                // 2m and 2m + 1 at 2m * row + 16m, one copy) and its metadata
                // after them, lanes 0-7 a pair each, lane 8 the metadata.
                if (mine) {
                    for (int r = 0; r < nruns; r++) {
                        const int rcol = __shfl_sync(0xffffffffu, col, r);
                        const uint32_t rid = __shfl_sync(0xffffffffu, my_id, r);
                        const int rhere = __shfl_sync(0xffffffffu, here ? r_nw : 0, r);
                        if (rhere > 0 && lane <= kBlockSize / 2) {
                            const uint32_t rowb = (uint32_t)rhere * kDps;  // a run is a whole block: Hk heads
                            const uint32_t dst = gs.template stage<LAYOUT>(slot) + (uint32_t)rcol * kHeadStride;
                            const uint8_t* src = P.cache + (uint64_t)rid * (uint64_t)P.block_bytes;
                            if (lane < kBlockSize / 2)
                                bulk_g2s(dst + (uint32_t)(2 * lane) * rowb + 16u * (uint32_t)lane,
                                         src + (uint32_t)(2 * lane) * rowb, 2u * rowb, gs.full(slot), stream_policy);
                            else
                                bulk_g2s(dst + kBlockSize * rowb + (uint32_t)kK3RowPad, src + kBlockSize * rowb,
                                         (uint32_t)rhere * kMetaSlot, gs.full(slot), stream_policy);
                        }
                    }
                }
            } else if (kWholeBlock && mine && here) {
                bulk_g2s(gs.template stage<LAYOUT>(slot) + (uint32_t)col * kHeadPage,
                         P.cache + (uint64_t)my_id * (uint64_t)P.block_bytes, (uint32_t)r_nw * kHeadPage, gs.full(slot),
                         stream_policy);
            } else if (mine && here) {
                const uint32_t dst = gs.template stage<LAYOUT>(slot);
                int off = 0;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int box = kGroupWarps >> i;
                    if (r_nw & box) {
                        tma_load_4d(dst + (uint32_t)(col + off) * kColBytes, &M.page[i], 0, 0, r_kvh + off,
                                    (int)my_id, gs.full(slot), stream_policy);
                        off += box;
                    }
                }
                const uint8_t* blk = P.cache + (uint64_t)my_id * (uint64_t)P.block_bytes;
                bulk_g2s(dst + kMetaOff + (uint32_t)col * kMetaSlot,
                         blk + kBlockSize * tok_bytes + (uint32_t)r_kvh * kMetaSlot, (uint32_t)r_nw * kMetaSlot,
                         gs.full(slot), stream_policy);
            }
            uses ^= 1u << slot;
            used |= 1u << slot;
            gpage++;
            if (++slot == NS) slot = 0;
        }
        if (!abort && !next_query_sent && !issue_query(irn, npn)) abort = true;
        t = tn;
        ir = irn;
        np = npn;
        np_tile = np_tile_n;
    }
    if (abort) {
        // Let the copies already issued land before the CTA can exit: the
        // last phase of every slot in use, then the last query rows.
        for (int sl = 0; sl < NS; sl++)
            if (((used >> sl) & 1u) && !mbar_wait(gs.full(sl), ((uses >> sl) & 1u) ^ 1u)) break;
        if (pj == 0 && tq > 0) mbar_wait(gs.q_full<NS>(), (tq - 1) & 1u);
    }
}

// ---------------------------------------------------------------------------
// Compute warp
// ---------------------------------------------------------------------------
template <int NT>
struct ItemState {
    uint32_t qf[NT][16];  // Q.K B fragments
    float kfac[NT];       // score factor of this lane's head
    float m_run[NT], l_part[NT], z_part[NT];
    float acc[NT][8][4];  // P.V accumulators (codes scaled by 2^-20)
};

// Per-lane byte offsets inside a stage (fixed for the kernel); the swizzle
// puts 16-byte chunk j of token t at chunk j ^ (t & 7) of its 128-byte row.
struct LaneSmem {
    uint32_t k0, k1;  // K bytes [16c, 16c+16) of tokens tau(g), tau(g)+1
    uint32_t v0, v1;  // V bytes [8g, 8g+8) of tokens 2c, 2c+1 (2c+8, 2c+9: + 1024)
    uint32_t meta;    // SoA: knorm pair of tokens tau(g), tau(g)+1 (vscale +32, vzero +64);
                      // AoS: knorm of token tau(g) (token tau(g)+1: + row)
    uint32_t row;     // AoS: bytes between consecutive tokens of a page
};

template <int NT, int LAYOUT>
__device__ __forceinline__ void page_math(ItemState<NT>& st, const uint32_t sb, const LaneSmem& o, bool page_ok,
                                          int tok0, int start, int end, uint32_t lut_sel_src, int g,
                                          int c, int src_a, uint32_t release_bar, float csq_unscale) {
    // Every ring byte this lane uses is read first and the slot released, so
    // its next page is fetched while this one is computed.  The arrive has
    // release semantics: the reads above it are performed before the
    // producer can observe the arrival.
    constexpr bool kAos = layout_is_aos(LAYOUT);
    constexpr bool kFp8 = layout_fp8_keys(LAYOUT);
    constexpr bool kKey3 = layout_3bit_keys(LAYOUT);
    constexpr bool kVal3 = layout_3bit_values(LAYOUT);
    uint4 k0, k1, k0b, k1b;
    uint32_t kn, vsp, vzp;
    uint2 v[4];
    if constexpr (kAos) {
        // AoS slot [key codes | fp16 knorm (Lloyd-Max keys) | value codes |
        // vscale | vzero] (offsets by layout); o.meta = the slot of token
        // tau(g), token tau(g)+1 one row (o.row) further.  Slots are 2-byte
        // (4-byte for FP8 keys) aligned: keys of dims [32c, 32c+32) are read
        // realigned.  V is read (and the slot released) after Q.K.
        if constexpr (kFp8) {
            k0 = lds128_a4(sb + o.k0);
            k0b = lds128_a4(sb + o.k0 + 16u);
            k1 = lds128_a4(sb + o.k1);
            k1b = lds128_a4(sb + o.k1 + 16u);
        } else if constexpr (kKey3) {
            k0 = lds96_a2(sb + o.k0);
            k1 = lds96_a2(sb + o.k1);
        } else {
            k0 = lds128_a2(sb + o.k0);
            k1 = lds128_a2(sb + o.k1);
        }
        const uint32_t m0 = sb + o.meta, m1 = m0 + o.row;
        constexpr uint32_t kNo = (uint32_t)aos_norm_off(LAYOUT), kSc = (uint32_t)aos_scale_off(LAYOUT);
        kn = kFp8 ? 0x3C003C00u : __byte_perm(lds16(m0 + kNo), lds16(m1 + kNo), 0x5410);
        vsp = __byte_perm(lds16(m0 + kSc), lds16(m1 + kSc), 0x5410);
        vzp = __byte_perm(lds16(m0 + kSc + 2), lds16(m1 + kSc + 2), 0x5410);
    } else if constexpr (kKey3) {
        // whole block [16 tokens][Hk][K 48 (3-bit) | V 64 (or 48, 3-bit)] +
        // [Hk][knorm 16 | vscale 16 | vzero 16]: key bits of dims
        // [32c, 32c+32) = bytes [12c, 12c+12) of tokens tau(g), tau(g)+1
        k0 = make_uint4(lds32(sb + o.k0), lds32(sb + o.k0 + 4u), lds32(sb + o.k0 + 8u), 0u);
        k1 = make_uint4(lds32(sb + o.k1), lds32(sb + o.k1 + 4u), lds32(sb + o.k1 + 8u), 0u);
        kn = lds32(sb + o.meta);
        vsp = lds32(sb + o.meta + 32u);
        vzp = lds32(sb + o.meta + 64u);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t va = sb + (j & 1 ? o.v1 : o.v0) + (j & 2 ? (o.row << 3) + 64u : 0u);
            if constexpr (layout_3bit_values(LAYOUT)) {
                // 16 3-bit codes (6 bytes, 2-byte aligned) spread to the
                // nibble layout of the 4-bit values (low nibble = even dim)
                const uint32_t a = lds16(va), b = lds16(va + 2u), cc = lds16(va + 4u);
                v[j] = make_uint2(spread3to4((a | (b << 16)) & 0xFFFFFFu), spread3to4((b >> 8) | (cc << 8)));
            } else {
                v[j] = lds64(va);
            }
        }
        mbar_arrive(release_bar);
    } else if constexpr (kFp8) {
        // whole block [16 tokens][Hk][K 128 e4m3 | V 64] + [Hk][vscale 16 |
        // vzero 16]: key bytes [32c, 32c+32) of tokens tau(g), tau(g)+1
        k0 = lds128(sb + o.k0);
        k0b = lds128(sb + o.k0 + 16u);
        k1 = lds128(sb + o.k1);
        k1b = lds128(sb + o.k1 + 16u);
        kn = 0x3C003C00u;  // no key norm: fp16 1.0 for both tokens
        vsp = lds32(sb + o.meta);
        vzp = lds32(sb + o.meta + 32u);
        // V is read (and the slot released) after Q.K, as for AoS
    } else if constexpr (LAYOUT == TQB_LAYOUT_SOA) {
        k0 = lds128(sb + o.k0);
        k1 = lds128(sb + o.k1);
        kn = lds32(sb + o.meta);
        vsp = lds32(sb + o.meta + 32);
        vzp = lds32(sb + o.meta + 64);
        v[0] = lds64(sb + o.v0);
        v[1] = lds64(sb + o.v1);
        v[2] = lds64(sb + o.v0 + 8u * kDataBytes);
        v[3] = lds64(sb + o.v1 + 8u * kDataBytes);
    }
    if constexpr (LAYOUT == TQB_LAYOUT_SOA) mbar_arrive(release_bar);
    const bool va = page_ok && tok0 >= start && tok0 < end;
    const bool vb = page_ok && tok0 + 1 >= start && tok0 + 1 < end;

    // -- Q.K: M tile 0 = token tau(g) (rows g: C_hi, g+8: C_lo), tile 1 = tau(g)+1
    float dq[NT][2][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int mt = 0; mt < 2; mt++)
#pragma unroll
            for (int k = 0; k < 4; k++) dq[nt][mt][k] = 0.0f;
    // AoS: Gram products of each M tile with its own C_hi rows (the A
    // fragment's C_hi registers are exactly the B fragment of A_hi^T):
    // D[g][g] = sum C_hi^2 and D[g+8][g] = sum C_lo C_hi of token row g.
    float dcs[2][4];
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
        for (int k = 0; k < 4; k++) dcs[mt][k] = 0.0f;
    if constexpr (kFp8) {
        // e4m3 converts exactly to fp16, so one M tile holds the page: row g
        // = token tau(g), row g+8 = token tau(g)+1, k columns the dims
        // 32c + 4ks + {0,1 | 2,3} of the query fragments.  Even and odd ks
        // accumulate in the two tiles' registers (two chains).
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
            const uint32_t w0 = word_of(ks < 4 ? k0 : k0b, ks & 3), w1 = word_of(ks < 4 ? k1 : k1b, ks & 3);
            const uint32_t a0 = fp8x2_to_h2(w0 & 0xFFFFu), a1 = fp8x2_to_h2(w1 & 0xFFFFu);
            const uint32_t a2 = fp8x2_to_h2(w0 >> 16), a3 = fp8x2_to_h2(w1 >> 16);
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
                mma_16816(dq[nt][ks & 1], a0, a1, a2, a3, st.qf[nt][2 * ks], st.qf[nt][2 * ks + 1]);
        }
        if constexpr (kAos) {
            v[0] = lds64_a4(sb + o.v0);
            v[1] = lds64_a4(sb + o.v1);
            v[2] = lds64_a4(sb + o.v0 + (o.row << 3));
            v[3] = lds64_a4(sb + o.v1 + (o.row << 3));
        } else {
            v[0] = lds64(sb + o.v0);
            v[1] = lds64(sb + o.v1);
            v[2] = lds64(sb + o.v0 + (o.row << 3));
            v[3] = lds64(sb + o.v1 + (o.row << 3));
        }
        mbar_arrive(release_bar);
    } else {
    // 3-bit keys: table address 0x10000 | (6-bit field << 8) | lane copy offset
    const uint32_t lut_lane = __byte_perm(lut_sel_src, 0u, 0x4140u);
#pragma unroll
    for (int ks = 0; ks < 8; ks++) {
        const uint32_t w0 = word_of(k0, ks >> 1), w1 = word_of(k1, ks >> 1);
        const uint32_t jA = 2 * (ks & 1), jB = jA + 1;
        uint2 e0, e1, e2, e3;
        if constexpr (kKey3) {
            // dim pairs 32c + 4ks + {0,1} and {2,3}: the 6-bit fields at bits
            // 12ks and 12ks + 6 of the lane's 96 bits
            e0 = lut_ld((bits6(k0, 12 * ks) << 8) + lut_lane);
            e1 = lut_ld((bits6(k0, 12 * ks + 6) << 8) + lut_lane);
            e2 = lut_ld((bits6(k1, 12 * ks) << 8) + lut_lane);
            e3 = lut_ld((bits6(k1, 12 * ks + 6) << 8) + lut_lane);
        } else {
            // address 0x10000 | (K byte << 8) | lane copy offset, in one PRMT
            e0 = lut_ld(prmt(w0, lut_sel_src, 0x6504u | (jA << 4)));
            e1 = lut_ld(prmt(w0, lut_sel_src, 0x6504u | (jB << 4)));
            e2 = lut_ld(prmt(w1, lut_sel_src, 0x6504u | (jA << 4)));
            e3 = lut_ld(prmt(w1, lut_sel_src, 0x6504u | (jB << 4)));
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            mma_16816(dq[nt][0], e0.x, e0.y, e1.x, e1.y, st.qf[nt][2 * ks], st.qf[nt][2 * ks + 1]);
            mma_16816(dq[nt][1], e2.x, e2.y, e3.x, e3.y, st.qf[nt][2 * ks], st.qf[nt][2 * ks + 1]);
        }
        if constexpr (kAos) {  // Lloyd-Max AoS keys (the FP8 ones take the branch above)
            mma_16816(dcs[0], e0.x, e0.y, e1.x, e1.y, e0.x, e1.x);
            mma_16816(dcs[1], e2.x, e2.y, e3.x, e3.y, e2.x, e3.x);
        }
    }
    }  // table-decoded keys
    float kn0 = half_bits_to_float(kn), kn1 = half_bits_to_float(kn >> 16);
    if constexpr (kAos && !kFp8) {
        // norm correction c / |c| (reference/aos_decode.py:199-206), with
        // sum c^2 = sum (C_hi + C_lo)^2 = D[g][g] + 2 D[g+8][g] (+ sum C_lo^2,
        // 2^-22 of it, dropped); lane 4g + g/2 holds column g, element g & 1
        const int j = g & 1, owner = 4 * g + (g >> 1);
        const float o0 = (j ? dcs[0][1] : dcs[0][0]) + 2.0f * (j ? dcs[0][3] : dcs[0][2]);
        const float o1 = (j ? dcs[1][1] : dcs[1][0]) + 2.0f * (j ? dcs[1][3] : dcs[1][2]);
        const float csq0 = __shfl_sync(0xffffffffu, o0, owner) * csq_unscale;
        const float csq1 = __shfl_sync(0xffffffffu, o1, owner) * csq_unscale;
        kn0 *= rsqrtf(csq0 + 1e-16f);
        kn1 *= rsqrtf(csq1 + 1e-16f);
#pragma unroll
        for (int jv = 0; jv < 4; jv++) {
            const uint32_t va_ = sb + (jv & 1 ? o.v1 : o.v0) + (jv & 2 ? (o.row << 3) : 0u);
            if constexpr (kVal3) {
                // 16 3-bit codes (6 bytes, 2-byte aligned) spread to nibbles
                const uint32_t a = lds16(va_), b = lds16(va_ + 2u), cc = lds16(va_ + 4u);
                v[jv] = make_uint2(spread3to4((a | (b << 16)) & 0xFFFFFFu), spread3to4((b >> 8) | (cc << 8)));
            } else {
                v[jv] = lds64_a2(va_);
            }
        }
        mbar_arrive(release_bar);
    }
    const float vs0 = va ? half_bits_to_float(vsp) : 0.0f;
    const float vs1 = vb ? half_bits_to_float(vsp >> 16) : 0.0f;
    const float vz0 = va ? half_bits_to_float(vzp) : 0.0f;
    const float vz1 = vb ? half_bits_to_float(vzp >> 16) : 0.0f;

    // -- online softmax (exp2 domain), lazy reference max: a page is weighted
    //    against the running reference m_run while no score exceeds it by
    //    more than kLazy (log2 units) and no weight leaves fp16; only then is
    //    the exact row max formed (three shuffles) and the state rescaled.
    uint32_t bw0[NT], bw1[NT];
    float alpha[NT];
    bool rescale = false;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        // columns 2c / 2c+1: Q_hi / Q_lo parts of head c; rows g / g+8:
        // C_hi / C_lo parts of the token (FP8 keys: tokens tau(g) / tau(g)+1,
        // chains ks even / odd)
        const float d0 = kFp8 ? (dq[nt][0][0] + dq[nt][0][1]) + (dq[nt][1][0] + dq[nt][1][1])
                              : (dq[nt][0][0] + dq[nt][0][2]) + (dq[nt][0][1] + dq[nt][0][3]);
        const float d1 = kFp8 ? (dq[nt][0][2] + dq[nt][0][3]) + (dq[nt][1][2] + dq[nt][1][3])
                              : (dq[nt][1][0] + dq[nt][1][2]) + (dq[nt][1][1] + dq[nt][1][3]);
        float s0 = d0 * kn0 * st.kfac[nt];
        float s1 = d1 * kn1 * st.kfac[nt];
        s0 = va ? s0 : -INFINITY;
        s1 = vb ? s1 : -INFINITY;
        const float mold = st.m_run[nt];
        const float mold_e = mold == -INFINITY ? 0.0f : mold;
        float p0 = ex2(s0 - mold_e), p1 = ex2(s1 - mold_e);
        float w0 = p0 * vs0, w1 = p1 * vs1;
        float mref = mold;
        const bool over = fmaxf(s0, s1) > mold + kLazy || fmaxf(w0, w1) > kWMax;
        if (__any_sync(0xffffffffu, over)) {
            mref = fmaxf(mold, warp_max_xor(fmaxf(s0, s1), 4, 16));
            const float mref_e = mref == -INFINITY ? 0.0f : mref;
            p0 = ex2(s0 - mref_e);
            p1 = ex2(s1 - mref_e);
            w0 = p0 * vs0;
            w1 = p1 * vs1;
        }
        alpha[nt] = (mold == -INFINITY || mref == mold) ? 1.0f : ex2(mold - mref);
        rescale |= alpha[nt] != 1.0f;
        st.l_part[nt] = st.l_part[nt] * alpha[nt] + (p0 + p1);
        st.z_part[nt] = st.z_part[nt] * alpha[nt] + (p0 * vz0 + p1 * vz1);
        st.m_run[nt] = mref;
        const __half2 wh = __floats2half2_rn(w0, w1);
        const __half2 wl = __floats2half2_rn(w0 - __low2float(wh), w1 - __high2float(wh));
        // B fragment of P.V: lane (g, c) takes tokens {2c, 2c+1} from lane
        // src_a (the owner of tau = 2c for head g>>1) and {2c+8, 2c+9} from
        // lane src_a + 16, part g&1 (hi / lo).
        const uint32_t hA = __shfl_sync(0xffffffffu, h2_as_u32(wh), src_a);
        const uint32_t lA = __shfl_sync(0xffffffffu, h2_as_u32(wl), src_a);
        const uint32_t hB = __shfl_sync(0xffffffffu, h2_as_u32(wh), src_a + 16);
        const uint32_t lB = __shfl_sync(0xffffffffu, h2_as_u32(wl), src_a + 16);
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

    // -- P.V: rows g / g+8 = low / high nibble of V byte i&3 of word i>>2,
    //    k = tokens 2c, 2c+1, 2c+8, 2c+9; codes enter as exact fp16
    //    subnormals code * 2^-20 (mantissa bits 4-7).  Taking the low
    //    nibble in place (code * 2^-24) saves the shift but is not exact on
    //    the tensor cores: 36 % of the c1 partials changed, by up to 3.8e-5.
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int wi = i >> 2, bi = i & 3;
        const uint32_t sel = (uint32_t)(bi | (bi << 4) | ((4 + bi) << 8) | ((4 + bi) << 12));
        const uint32_t x0 = wi ? v[0].y : v[0].x;
        const uint32_t x1 = wi ? v[1].y : v[1].x;
        const uint32_t x2 = wi ? v[2].y : v[2].x;
        const uint32_t x3 = wi ? v[3].y : v[3].x;
        const uint32_t p01 = prmt(x0, x1, sel), p23 = prmt(x2, x3, sel);
        const uint32_t a0 = (p01 << 4) & 0x00F000F0u;  // row g:   low nibble
        const uint32_t a1 = p01 & 0x00F000F0u;         // row g+8: high nibble
        const uint32_t a2 = (p23 << 4) & 0x00F000F0u;
        const uint32_t a3 = p23 & 0x00F000F0u;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) mma_16816(st.acc[nt][i], a0, a1, a2, a3, bw0[nt], bw1[nt]);
    }
}

// Partial output rows of one item: lane (g, c) holds dims 16g .. 16g+15 of
// head c + 4 nt.  They pass through this warp's 1 KB staging area two heads
// at a time, as [2 heads][128] fp32 (16-byte chunk j of row r at chunk
// j ^ r: conflict-free both ways), and are written back as 128-byte
// coalesced runs.
template <int NT>
__device__ __forceinline__ void epilogue(const Stage1Params& P, const ItemState<NT>& st, uint32_t col, int b, int s,
                                         int kvh, int g, int c, int lane) {
    constexpr float kCodeScale = 1048576.0f;  // 2^20: undo the subnormal code scale
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        float l = warp_sum_xor(st.l_part[nt], 4, 16);
        l = l > 0.0f ? l : 1.0f;  // safe_l (reference/soa_decode_v1.py:311)
        const float z = warp_sum_xor(st.z_part[nt], 4, 16);
        const float inv = rcp_approx(l);
        // the lane's 16 outputs, formed once (not inside the per-pass branch,
        // which the warp issues twice)
        float val[8][2];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            val[i][0] = ((st.acc[nt][i][0] + st.acc[nt][i][1]) * kCodeScale + z) * inv;
            val[i][1] = ((st.acc[nt][i][2] + st.acc[nt][i][3]) * kCodeScale + z) * inv;
        }
        const int heads = min(4, P.G - 4 * nt);
#pragma unroll
        for (int pass = 0; pass < 2; pass++) {
            const int r = c & 1;  // staging row of this lane's head
            if ((c >> 1) == pass) {
#pragma unroll
                for (int j = 0; j < 4; j++)  // dims 16g + 4j .. 16g + 4j + 3
                    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};\n" ::"r"(
                                     col + (uint32_t)r * 512u + ((uint32_t)((4 * g + j) ^ r) << 4)),
                                 "f"(val[2 * j][0]), "f"(val[2 * j][1]), "f"(val[2 * j + 1][0]),
                                 "f"(val[2 * j + 1][1])
                                 : "memory");
            }
            __syncwarp();
#pragma unroll
            for (int rr = 0; rr < 2; rr++) {
                const int hl = 2 * pass + rr;
                if (hl < heads) {
                    float* dst = P.mid + (int64_t)b * P.msb + (int64_t)(kvh * P.G + 4 * nt + hl) * P.msh +
                                 (int64_t)s * P.mss;
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        dst[32 * q + lane] = __uint_as_float(
                            lds32(col + (uint32_t)rr * 512u + ((uint32_t)((8 * q + (lane >> 2)) ^ rr) << 4) +
                                  4u * (lane & 3)));
                }
            }
            __syncwarp();  // the area is rewritten by the next pass
        }
        if (g == 0 && c + 4 * nt < P.G) {
            float* dst = P.mid + (int64_t)b * P.msb + (int64_t)(kvh * P.G + c + 4 * nt) * P.msh + (int64_t)s * P.mss;
            dst[kHeadDim] = (st.m_run[nt] + lg2_approx(l)) * kLn2;
        }
    }
}

// One page from ring slot S (a compile-time constant, so every shared and
// barrier address below is a register plus an immediate).
template <int NT, int LAYOUT, int S>
__device__ __forceinline__ bool page_step(ItemState<NT>& st, const GroupSmem& gs, const LaneSmem& o, uint32_t& cbits,
                                          int k, int my_np, int w, int tok_first, int start, int end,
                                          uint32_t lut_sel_src, int g, int c, int src_a, float csq_unscale) {
    constexpr int NS = Cfg<NT, LAYOUT>::kStages;
    if (!mbar_wait(gs.full(S), (cbits >> S) & 1u)) return false;
    cbits ^= 1u << S;
    // all 32 lanes arrive on the slot's release barrier (no branch on the lane)
    if (k < my_np) {
        const bool page_ok = (lds32(gs.vmask<NS>(S)) >> w) & 1u;
        page_math<NT, LAYOUT>(st, (uint32_t)(S * stage_bytes(LAYOUT)), o, page_ok, tok_first + k * kBlockSize, start, end,
                      lut_sel_src, g, c, src_a, gs.empty<NS>(S), csq_unscale);
    } else {
        mbar_arrive(gs.empty<NS>(S));
    }
    return true;
}

template <int NT, int LAYOUT>
__device__ __forceinline__ void consume(const Stage1Params& P, const GroupSmem& gs, int gi, int w, int lane,
                                        int ec) {
    using C = Cfg<NT, LAYOUT>;
    constexpr int NS = C::kStages;
    const int g = lane >> 2, c = lane & 3;
    const uint32_t t_first = lds32(gs.tiles()), t_end = lds32(gs.tiles() + 4u), t_stride = lds32(gs.tiles() + 8u);
    // PRMT source: byte 0 = this lane's copy offset, byte 1 = table page 0x01, byte 2 = 0
    const uint32_t lut_sel_src = (uint32_t)(lane % kLutCopies) * 8u | ((uint32_t)(kLutAddr >> 16) << 8);
    // the table's centroids are scaled by 2^ec: sums of their squares by 2^(2 ec)
    const float csq_unscale = exp2i(-2 * ec);
    const int tau = 8 * (g >> 2) + 2 * ((g >> 1) & 1) + 4 * (g & 1);
    LaneSmem o;
    if constexpr (LAYOUT == TQB_LAYOUT_SOA) {
        auto sw = [](int t, int chunk) { return (uint32_t)(t * kDataBytes + ((chunk ^ (t & 7)) << 4)); };
        const uint32_t colw = gs.ring + (uint32_t)w * kColBytes;  // shared address of this warp's column
        o.k0 = colw + sw(tau, c);
        o.k1 = colw + sw(tau + 1, c);
        o.v0 = colw + sw(2 * c, 4 + (g >> 1)) + 8u * (g & 1);
        o.v1 = colw + sw(2 * c + 1, 4 + (g >> 1)) + 8u * (g & 1);
        o.meta = gs.ring + kMetaOff + (uint32_t)w * kMetaSlot + 2u * tau;
        o.row = 0;
    } else if constexpr (LAYOUT == TQB_LAYOUT_SOA_K3 || LAYOUT == TQB_LAYOUT_SOA_K3V3) {
        // The page's block of run [w - kvh, w - kvh + Hk) sits unchanged at
        // (w - kvh) * 16 * slot bytes of the stage: [16 tokens][Hk][K 48 | V]
        // then [Hk][knorm 16 | vscale 16 | vzero 16] fp16.
        constexpr uint32_t kDps = layout_3bit_values(LAYOUT) ? kK3V3DataBytes : kK3DataBytes;
        constexpr uint32_t kValLane = layout_3bit_values(LAYOUT) ? 6u : 8u;  // V bytes of dims 16g .. 16g+15
        // Rows sit padded apart (token t at t * row + 16 * (t >> 1)); tokens
        // 2m and 2m+1 share a pad, so o.k1 = o.k0 + row, and tokens 2c+8,
        // 2c+9 are 8 rows and 64 pad bytes after 2c, 2c+1.
        const int kvh = w % P.Hk;
        const uint32_t row = (uint32_t)P.Hk * kDps;
        const uint32_t run = gs.ring + (uint32_t)(w - kvh) * (uint32_t)head_stride_bytes(LAYOUT);
        const uint32_t head = run + (uint32_t)kvh * kDps;
        o.k0 = head + (uint32_t)tau * row + 8u * (uint32_t)tau + 12u * c;
        o.k1 = o.k0 + row;
        o.v0 = head + (uint32_t)(2 * c) * row + 16u * c + kK3KeyBytes + kValLane * g;
        o.v1 = o.v0 + row;
        o.meta = run + (uint32_t)kBlockSize * row + (uint32_t)kK3RowPad + (uint32_t)kvh * kMetaSlot + 2u * tau;
        o.row = row;
    } else if constexpr (LAYOUT == TQB_LAYOUT_SOA_K8) {
        // The page's block of run [w - kvh, w - kvh + Hk) sits unchanged at
        // (w - kvh) * 3136 bytes of the stage: [16 tokens][Hk][K 128 | V 64]
        // then [Hk][vscale 16 | vzero 16] fp16.
        const int kvh = w % P.Hk;
        const uint32_t row = (uint32_t)P.Hk * kK8DataBytes;
        const uint32_t run = gs.ring + (uint32_t)(w - kvh) * kK8Head;
        const uint32_t head = run + (uint32_t)kvh * kK8DataBytes;
        o.k0 = head + (uint32_t)tau * row + 32u * c;
        o.k1 = o.k0 + row;
        o.v0 = head + (uint32_t)(2 * c) * row + kK8KeyBytes + 8u * g;
        o.v1 = o.v0 + row;
        o.meta = run + (uint32_t)kBlockSize * row + (uint32_t)kvh * (2 * kBlockSize * 2) + 2u * tau;
        o.row = row;
    } else {
        // AoS: the page's block of run [w - kvh, w - kvh + Hk) sits unchanged
        // at (w - kvh) * 16 slots of the stage: [16 tokens][Hk][slot] (134,
        // 196, 118 or 102 bytes).  A lane's key bytes of dims [32c, 32c+32)
        // are 16 (4-bit), 32 (e4m3) or 12 (3-bit) bytes at that multiple of
        // c; its value codes of dims [16g, 16g+16) 8 (4-bit) or 6 (3-bit) bytes.
        constexpr uint32_t kSlot = (uint32_t)aos_slot_bytes(LAYOUT);
        constexpr uint32_t kKeyLane = layout_fp8_keys(LAYOUT) ? 32u : layout_3bit_keys(LAYOUT) ? 12u : 16u;
        constexpr uint32_t kValLane = layout_3bit_values(LAYOUT) ? 6u : 8u;
        const int kvh = w % P.Hk;
        const uint32_t row = (uint32_t)P.Hk * kSlot;
        const uint32_t head = gs.ring + (uint32_t)(w - kvh) * (kBlockSize * kSlot) + (uint32_t)kvh * kSlot;
        o.k0 = head + (uint32_t)tau * row + kKeyLane * c;
        o.k1 = o.k0 + row;
        o.v0 = head + (uint32_t)(2 * c) * row + (uint32_t)aos_val_off(LAYOUT) + kValLane * g;
        o.v1 = o.v0 + row;
        o.meta = head + (uint32_t)tau * row;  // the slot; fields at their offsets
        o.row = row;
    }
    // Owner of token 2c in the Q.K layout: tau(g') = 2c for g' = bitswap(c).
    const int src_a = 4 * (((c & 1) << 1) | (c >> 1)) + (g >> 1);
    uint32_t tq = 0;     // tiles done (query-barrier phase)
    uint32_t cbits = 0;  // bit s: parity of the pages slot s has delivered
    // The query fragments (and score factors) stay from one tile to the
    // next while the item's sequence and KV head do not change.
    ItemState<NT> st;
    int prev_b = -1, prev_kvh = -1;
    // lanes 0-7: (b, KV head) of item `lane` of the previous non-empty tile
    // (b = -1: none or empty), the test the producer makes for the rows
    int lane_b = -1, lane_kvh = -1;

    for (uint32_t t = t_first; t < t_end; t += t_stride) {
        ItemInfo ir;
        int np;
        const int np_tile = tile_items(P, t, lane, ir, np);
        if (np_tile == 0) continue;
        const int b = __shfl_sync(0xffffffffu, ir.b, w);
        const int s = __shfl_sync(0xffffffffu, ir.s, w);
        const int kvh = __shfl_sync(0xffffffffu, ir.kvh, w);
        const int start = __shfl_sync(0xffffffffu, ir.start, w);
        const int end = __shfl_sync(0xffffffffu, ir.end, w);
        const int my_np = __shfl_sync(0xffffffffu, np, w);

        // ---- query fragments from the tile's query rows ---------------------
        // Every item keeps its sequence and KV head: the producer copied no
        // rows and neither side uses the query barriers (its own test, on the
        // same items).  One warp's item keeping them: its fragments stay.
        const bool same_rows = __all_sync(0xffffffffu, lane >= kGroupWarps || (np > 0 && lane_b >= 0 &&
                                                                              ir.b == lane_b && ir.kvh == lane_kvh));
        lane_b = np > 0 ? ir.b : -1;
        lane_kvh = ir.kvh;
        if (!same_rows && !mbar_wait(gs.q_full<NS>(), tq & 1u)) return;
        const bool reuse = b == prev_b && kvh == prev_kvh;
        prev_b = my_np > 0 ? b : -1;
        prev_kvh = kvh;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            if (!reuse) {
                // Lanes g and g^1 share a head and dims 32c .. 32c+31 but keep the
                // hi (even g) or lo (odd g) parts: each converts 16 of the 32
                // floats and the pair swaps the halves the other keeps.
                const int hl = (g >> 1) + 4 * nt;
                const bool odd = g & 1;
                float qv[16];
                float amax = 0.0f;
                if (my_np > 0 && hl < P.G) {
                    const uint32_t qa = gs.qarea + (uint32_t)(w * C::kHeadsPerWarp + hl) * kQRowBytes + 128u * c +
                                        (odd ? 64u : 0u);
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float4 f = lds_f4(qa + 16u * j);
                        qv[4 * j] = f.x; qv[4 * j + 1] = f.y; qv[4 * j + 2] = f.z; qv[4 * j + 3] = f.w;
                    }
#pragma unroll
                    for (int j = 0; j < 16; j++) amax = fmaxf(amax, fabsf(qv[j]));
                } else {
#pragma unroll
                    for (int j = 0; j < 16; j++) qv[j] = 0.0f;
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
                amax = warp_max_xor(amax, 1, 2);
                const int eq = fp16_scale_exp(amax);
                const float qscale = exp2i(eq);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float x0 = qv[2 * j] * qscale, x1 = qv[2 * j + 1] * qscale;
                    const __half2 h = __floats2half2_rn(x0, x1);
                    const __half2 l = __floats2half2_rn(x0 - __low2float(h), x1 - __high2float(h));
                    const uint32_t keep = odd ? h2_as_u32(l) : h2_as_u32(h);
                    const uint32_t got = __shfl_xor_sync(0xffffffffu, odd ? h2_as_u32(h) : h2_as_u32(l), 4);
                    st.qf[nt][j] = odd ? got : keep;      // fragments 0-7: floats of the even lane
                    st.qf[nt][8 + j] = odd ? keep : got;  // fragments 8-15: floats of the odd lane
                }
                const int eq_head = __shfl_sync(0xffffffffu, eq, 8 * c);
                st.kfac[nt] = P.attn_scale * kLog2e * exp2i(-eq_head) * exp2i(-ec);
            }
            st.m_run[nt] = -INFINITY;
            st.l_part[nt] = 0.0f;
            st.z_part[nt] = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int k = 0; k < 4; k++) st.acc[nt][i][k] = 0.0f;
        }
        if (!same_rows) {
            mbar_arrive(gs.q_empty<NS>());  // all 32 lanes
            tq++;
        }

        // ---- pages: slot S of the ring holds pages k = S (mod NS) ------------
        const int tok_first = (start / kBlockSize) * kBlockSize + tau;
        for (int k = 0; k < np_tile; k += NS) {
            if (!page_step<NT, LAYOUT, 0>(st, gs, o, cbits, k, my_np, w, tok_first, start, end, lut_sel_src, g, c, src_a, csq_unscale))
                return;
            if (k + 1 < np_tile && !page_step<NT, LAYOUT, 1>(st, gs, o, cbits, k + 1, my_np, w, tok_first, start, end,
                                                     lut_sel_src, g, c, src_a, csq_unscale))
                return;
            if (k + 2 < np_tile && !page_step<NT, LAYOUT, 2>(st, gs, o, cbits, k + 2, my_np, w, tok_first, start, end,
                                                     lut_sel_src, g, c, src_a, csq_unscale))
                return;
        }
        if (my_np > 0) epilogue<NT>(P, st, gs.stg + (uint32_t)w * kStgBytes, b, s, kvh, g, c, lane);
    }
}

template <int NT, int LAYOUT>
__global__ void __launch_bounds__(Cfg<NT>::kThreads, 1)
    stage1_ring_kernel(const Stage1Params P, const __grid_constant__ RingMaps M) {
    using C = Cfg<NT, LAYOUT>;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_trigger();
    pdl_wait();  // the kernel before on the stream (e.g. the previous step's Stage2 reading mid_o)

    // ---- K table: 256 entries x 32 lane copies of {C_hi pair, C_lo pair} ----
    // (FP8 keys: no table, no centroids, no scale; 3-bit keys: 8 centroids,
    // entry = 6-bit field of two codes, low code in bits 0-2)
    constexpr bool kKey3 = layout_3bit_keys(LAYOUT);
    constexpr int kNc = C::kTable ? (kKey3 ? 8 : kNumCentroids) : 0;
    float cmax = 0.0f;
#pragma unroll
    for (int k = 0; k < kNc; k++) cmax = fmaxf(cmax, fabsf(__ldg(P.cents + k)));
    const int ec = C::kTable ? fp16_scale_exp(cmax) : 0;
    const float cscale = exp2i(ec);
    // The last kGroups warps plan the groups' tile walks (reading seq_lens)
    // while the others build the table.
    const uint32_t num_tiles = (uint32_t)((P.num_items + kGroupWarps - 1) / kGroupWarps);
    const int planner = warp - (C::kWarps - C::kGroups);  // group planned by this warp, if >= 0
    uint32_t walk[3] = {0u, 0u, 0u};
    if (planner >= 0)
        tile_walk(P, planner, C::kGroups, num_tiles, walk, lane);
    else if (C::kTable)
        for (int e = tid; e < 256 * kLutCopies; e += C::kThreads - 32 * C::kGroups) {
        const int byte = e / kLutCopies;
        const int ilo = kKey3 ? (byte & 7) : (byte & 15), ihi = kKey3 ? ((byte >> 3) & 7) : (byte >> 4);
        const float clo = __ldg(P.cents + ilo) * cscale, chi = __ldg(P.cents + ihi) * cscale;
        const __half2 h = __floats2half2_rn(clo, chi);
        const __half2 l = __floats2half2_rn(clo - __low2float(h), chi - __high2float(h));
        *reinterpret_cast<uint2*>(smem + C::kLutOff + (size_t)e * 8) = make_uint2(h2_as_u32(h), h2_as_u32(l));
        }

    const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    if (base != (uint32_t)kDynBase) {  // the table address above assumes this window layout
        if (tid == 0) atomicAdd(&g_wait_timeouts, 1u);
        return;
    }
    const bool producer = warp >= C::kComputeWarps;
    // producer warp p of the producer warpgroup feeds group p % kGroups as its
    // producer p / kGroups (two per group; with one group warps 2-3 idle)
    const int gi = producer ? (warp - C::kComputeWarps) % C::kGroups : warp / kGroupWarps;
    GroupSmem gs;
    gs.ring = base + (uint32_t)C::ring_off(gi);
    gs.qarea = base + (uint32_t)C::q_off(gi);
    gs.stg = base + (uint32_t)(C::kStgOff + gi * kGroupWarps * kStgBytes);
    gs.bars = base + C::kBarOff + (uint32_t)gi * kBarStride;
    if (planner >= 0 && lane == 0) {
        const uint32_t tiles = base + C::kBarOff + (uint32_t)planner * kBarStride + 96u;
        sts32(tiles, walk[0]);
        sts32(tiles + 4u, walk[1]);
        sts32(tiles + 8u, walk[2]);
    }
    if (tid < C::kGroups) {
        GroupSmem gb;
        gb.bars = base + C::kBarOff + (uint32_t)tid * kBarStride;
        for (int s = 0; s < C::kStages; s++) {
            mbar_init(gb.full(s), 1);
            mbar_init(gb.template empty<C::kStages>(s), kGroupWarps * 32);  // every compute lane arrives
        }
        mbar_init(gb.template q_full<C::kStages>(), 1);
        mbar_init(gb.template q_empty<C::kStages>(), kGroupWarps * 32);
        mbar_init(gb.template issued<C::kStages>(), 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    }
    __syncthreads();

    if constexpr (NT == 1 && C::kTable) {  // the fused rotation (not for FP8 keys)
        if (P.rot != nullptr) {
            rotate_share<NT>(P, smem, tid);
            // generic writes to the ring and query areas, before the tensor
            // copies (async proxy) that will overwrite them
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            __syncthreads();
            if (tid == 0) {
                __threadfence();  // this CTA's rows, before its arrival
                const uint32_t seen =
                    atomicAdd(&g_rot_barrier, blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1) : 1u);
                sts32(base + C::kBarOff + 112u, seen);
            }
            __syncthreads();
        }
    }

    if (producer) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(C::kProducerRegs));
        const int pj = (warp - C::kComputeWarps) / C::kGroups;
        if (pj < kProducersPerGroup) produce<NT, LAYOUT>(P, M, gs, gi, lane, pj, kProducersPerGroup);
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(C::kComputeRegs));
        consume<NT, LAYOUT>(P, gs, gi, warp % kGroupWarps, lane, ec);
    }
}

// True when the compiled kernel launches with enough registers per thread
// for its setmaxnreg split (otherwise a setmaxnreg.inc could wait forever,
// so the ring kernel is not used).
template <int NT, int LAYOUT>
bool ring_registers_ok() {
    using C = Cfg<NT, LAYOUT>;
    static int ok = -1;
    if (ok < 0) {
        cudaFuncAttributes a{};
        ok = cudaFuncGetAttributes(&a, stage1_ring_kernel<NT, LAYOUT>) == cudaSuccess &&
             (int64_t)a.numRegs * C::kThreads >=
                 (int64_t)C::kComputeWarps * 32 * C::kComputeRegs + 128 * C::kProducerRegs &&
             a.maxThreadsPerBlock >= C::kThreads;
        if (!ok) cudaGetLastError();
    }
    return ok == 1;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime
// (no link-time dependency on libcuda).
EncodeTiledFn encoder() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
        else
            cudaGetLastError();
    }
    return fn;
}

// Tensor maps of the page data (SoA) and query rows of one launch; false
// when the driver rejects them.
bool encode_maps(const Stage1Params& P, RingMaps& M) {
    EncodeTiledFn enc = encoder();
    if (!enc) return false;
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (P.layout == TQB_LAYOUT_SOA) {  // AoS pages are plain bulk copies
        const cuuint64_t nblk = P.num_blocks > 0 ? (cuuint64_t)P.num_blocks : (cuuint64_t)0x7fffffff;
        const cuuint64_t dims[4] = {(cuuint64_t)kDataBytes, (cuuint64_t)kBlockSize, (cuuint64_t)P.Hk, nblk};
        const cuuint64_t strides[3] = {(cuuint64_t)P.Hk * kDataBytes, (cuuint64_t)kDataBytes,
                                       (cuuint64_t)P.block_bytes};
        for (int i = 0; i < 4; i++) {
            const int heads = (kGroupWarps >> i) < P.Hk ? (kGroupWarps >> i) : P.Hk;
            const cuuint32_t box[4] = {(cuuint32_t)kDataBytes, (cuuint32_t)kBlockSize, (cuuint32_t)heads, 1};
            if (enc(&M.page[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t*>(P.cache), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
                return false;
        }
    }
    const cuuint64_t qdims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)P.Hq, (cuuint64_t)P.B};
    const cuuint64_t qstr[2] = {(cuuint64_t)P.qsh * 4, (cuuint64_t)P.qsb * 4};
    const cuuint32_t qbox[3] = {(cuuint32_t)kHeadDim, (cuuint32_t)P.G, 1};
    return enc(&M.query, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(P.q), qdims, qstr, qbox, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT, int LAYOUT>
int launch_ring_t(const Stage1Params& P, const RingMaps& M, cudaStream_t stream, int num_sms) {
    using C = Cfg<NT, LAYOUT>;
    auto kern = stage1_ring_kernel<NT, LAYOUT>;
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) != cudaSuccess)
            return report_launch(cudaGetLastError());
        configured_dev = dev;
    }
    if (P.rot != nullptr) {
        // Fused query rotation: every SM's CTA takes a share of the rows and
        // the grid barrier needs all of them resident at once, which a
        // cooperative launch guarantees (or refuses).
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)num_sms);
        cfg.blockDim = dim3(C::kThreads);
        cfg.dynamicSmemBytes = C::kSmem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, P, M);
        if (e == cudaErrorCooperativeLaunchTooLarge) {
            cudaGetLastError();
            return TQB_ERR_UNSUPPORTED;  // the caller rotates in a kernel of its own
        }
        return report_launch(e);
    }
    const int64_t tiles = (P.num_items + kGroupWarps - 1) / kGroupWarps;
    const int64_t need = (tiles + C::kGroups - 1) / C::kGroups;
    const int64_t grid = need < num_sms ? need : num_sms;
    if (grid <= 0) return TQB_OK;
    return report_launch(launch_pdl(kern, dim3((unsigned)grid), dim3(C::kThreads), C::kSmem, stream, P, M));
}

}  // namespace

bool stage1_ring_supported(const Stage1Params& P) {
    const bool soa = P.layout == TQB_LAYOUT_SOA;
    // AoS (every preset): a tile's runs are whole blocks (Hk divides 8) of
    // packed slots, each copied as one run of Hk * 16 slots.
    const bool aos_ok = layout_is_aos(P.layout) && kGroupWarps % P.Hk == 0 &&
                        P.head_stride == aos_slot_bytes(P.layout) &&
                        P.pos_stride == (int64_t)P.Hk * aos_slot_bytes(P.layout);
    // FP8 keys (SoA blocks): whole blocks too, Hk * 3136 bytes.
    const bool k8_ok = P.layout == TQB_LAYOUT_SOA_K8 && kGroupWarps % P.Hk == 0 &&
                       P.block_bytes >= (int64_t)kBlockSize * P.Hk * kSlotBytesK8;
    // 3-bit keys (SoA blocks): whole blocks, Hk * 1888 (or 1632) bytes.
    const bool k3_ok = (P.layout == TQB_LAYOUT_SOA_K3 || P.layout == TQB_LAYOUT_SOA_K3V3) &&
                       kGroupWarps % P.Hk == 0 && P.block_bytes >= (int64_t)P.Hk * head_page_bytes(P.layout);
    bool regs_ok = false;
    if (soa)
        regs_ok = P.G <= 4 ? ring_registers_ok<1, TQB_LAYOUT_SOA>() : ring_registers_ok<2, TQB_LAYOUT_SOA>();
    else if (aos_ok && P.layout == TQB_LAYOUT_AOS)
        regs_ok = P.G <= 4 ? ring_registers_ok<1, TQB_LAYOUT_AOS>() : ring_registers_ok<2, TQB_LAYOUT_AOS>();
    else if (aos_ok && P.layout == TQB_LAYOUT_AOS_K8)
        regs_ok = P.G <= 4 ? ring_registers_ok<1, TQB_LAYOUT_AOS_K8>() : ring_registers_ok<2, TQB_LAYOUT_AOS_K8>();
    else if (aos_ok && P.layout == TQB_LAYOUT_AOS_K3)
        regs_ok = P.G <= 4 ? ring_registers_ok<1, TQB_LAYOUT_AOS_K3>() : ring_registers_ok<2, TQB_LAYOUT_AOS_K3>();
    else if (aos_ok)
        regs_ok = P.G <= 4 ? ring_registers_ok<1, TQB_LAYOUT_AOS_K3V3>() : ring_registers_ok<2, TQB_LAYOUT_AOS_K3V3>();
    else if (k8_ok)
        regs_ok = P.G <= 4 ? ring_registers_ok<1, TQB_LAYOUT_SOA_K8>() : ring_registers_ok<2, TQB_LAYOUT_SOA_K8>();
    else if (k3_ok && P.layout == TQB_LAYOUT_SOA_K3)
        regs_ok = P.G <= 4 ? ring_registers_ok<1, TQB_LAYOUT_SOA_K3>() : ring_registers_ok<2, TQB_LAYOUT_SOA_K3>();
    else if (k3_ok)
        regs_ok = P.G <= 4 ? ring_registers_ok<1, TQB_LAYOUT_SOA_K3V3>() : ring_registers_ok<2, TQB_LAYOUT_SOA_K3V3>();
    // Query rows are copied by a tensor map: 16-byte row strides, >= one row.
    return regs_ok && (soa || aos_ok || k8_ok || k3_ok) && P.G >= 1 && P.G <= 8 &&
           (reinterpret_cast<uintptr_t>(P.cache) & 15) == 0 && (P.block_bytes & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(P.q) & 15) == 0 && P.qsh >= kHeadDim && (P.qsh & 3) == 0 &&
           P.qsb >= P.qsh && (P.qsb & 3) == 0 && encoder() != nullptr;
}

int launch_stage1_ring(const Stage1Params& P, cudaStream_t stream, int num_sms) {
    RingMaps M;
    if (!encode_maps(P, M)) return TQB_ERR_UNSUPPORTED;
    if (P.layout == TQB_LAYOUT_SOA)
        return P.G <= 4 ? launch_ring_t<1, TQB_LAYOUT_SOA>(P, M, stream, num_sms)
                        : launch_ring_t<2, TQB_LAYOUT_SOA>(P, M, stream, num_sms);
    if (P.layout == TQB_LAYOUT_SOA_K8) {
        if (P.rot != nullptr) return TQB_ERR_UNSUPPORTED;  // no rotation prologue in this instance
        return P.G <= 4 ? launch_ring_t<1, TQB_LAYOUT_SOA_K8>(P, M, stream, num_sms)
                        : launch_ring_t<2, TQB_LAYOUT_SOA_K8>(P, M, stream, num_sms);
    }
    if (P.layout == TQB_LAYOUT_AOS_K8) {
        if (P.rot != nullptr) return TQB_ERR_UNSUPPORTED;  // no rotation prologue in this instance
        return P.G <= 4 ? launch_ring_t<1, TQB_LAYOUT_AOS_K8>(P, M, stream, num_sms)
                        : launch_ring_t<2, TQB_LAYOUT_AOS_K8>(P, M, stream, num_sms);
    }
    if (P.layout == TQB_LAYOUT_AOS_K3)
        return P.G <= 4 ? launch_ring_t<1, TQB_LAYOUT_AOS_K3>(P, M, stream, num_sms)
                        : launch_ring_t<2, TQB_LAYOUT_AOS_K3>(P, M, stream, num_sms);
    if (P.layout == TQB_LAYOUT_AOS_K3V3)
        return P.G <= 4 ? launch_ring_t<1, TQB_LAYOUT_AOS_K3V3>(P, M, stream, num_sms)
                        : launch_ring_t<2, TQB_LAYOUT_AOS_K3V3>(P, M, stream, num_sms);
    if (P.layout == TQB_LAYOUT_SOA_K3)
        return P.G <= 4 ? launch_ring_t<1, TQB_LAYOUT_SOA_K3>(P, M, stream, num_sms)
                        : launch_ring_t<2, TQB_LAYOUT_SOA_K3>(P, M, stream, num_sms);
    if (P.layout == TQB_LAYOUT_SOA_K3V3)
        return P.G <= 4 ? launch_ring_t<1, TQB_LAYOUT_SOA_K3V3>(P, M, stream, num_sms)
                        : launch_ring_t<2, TQB_LAYOUT_SOA_K3V3>(P, M, stream, num_sms);
    return P.G <= 4 ? launch_ring_t<1, TQB_LAYOUT_AOS>(P, M, stream, num_sms)
                    : launch_ring_t<2, TQB_LAYOUT_AOS>(P, M, stream, num_sms);
}

int read_wait_timeouts(unsigned int* count, bool reset) {
    cudaError_t e = cudaMemcpyFromSymbol(count, g_wait_timeouts, sizeof(unsigned int));
    if (e == cudaSuccess && reset) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(unsigned int));
    }
    return e == cudaSuccess ? TQB_OK : report_launch(e);
}

}  // namespace tqb
