// tqb_p2p.cu — sequence-parallel exchange of split-KV partials over peer
// memory (NVLink P2P), fused with the Stage2 merge on the sending side and
// with the cross-range merge on the receiving side.
//
// Every rank owns one exchange buffer (plain cudaMalloc, shared with the
// other ranks of the node through CUDA IPC handles; plain stores only):
//     recv  [2 parities][G ranks][cap_rows][D+1] {fp32 value, u32 epoch}
//     done  uint32                                     merge CTAs finished (local)
//     step  uint64                                     last epoch merged (local)
// Every element of a row travels as one aligned 8-byte store of its value
// and the low 32 bits of the call's epoch (the low-latency protocol of
// NCCL's "LL" transport): an aligned 8-byte access is single-copy atomic,
// so a receiver that reads the epoch it expects holds the value written with
// it.  No fence and no separate flag orders the data (a system-scope fence
// costs several microseconds per step on this path).
// Call k of a rank (epoch k + 1) uses parity k & 1.  The epoch is either
// given by the host (1, 2, ... on every rank) or, with epoch 0 in the call,
// kept on the device in `step`: both kernels of a call use step + 1, and the
// merge's last CTA stores it back.  Device epochs need no host value per
// step, so a whole decode step (Stage1, exchange, merge) can be captured
// once in a CUDA graph and replayed.  One buffer uses one of the two forms
// from the start (a zero-filled buffer); they are not mixed.
//  * tqb_sp_exchange: one CTA per (b, h) merges the rank's own splits (the
//    Stage2 algebra) and stores the tagged row straight into slot [rank] of
//    every rank's recv buffer.
//  * tqb_sp_merge: one CTA per (b, h); thread d reads element d (and the
//    LSE) of the row from every rank, re-reading an element until its tag
//    holds the epoch (about a second at most), then merges the G rows with
//    the LSE algebra, skipping ranges whose LSE is -inf (no local token).  A
//    wait that gives up adds one to a device counter (read by
//    tqb_wait_timeouts) and writes NaN.
// The receiving side waits on other GPUs only, never on a kernel of its own
// GPU, so nothing depends on CTAs being co-resident.  Two parities suffice:
// a rank is at most one call ahead of another (its merge needs the other's
// rows of the same call), so call k + 2 never overwrites rows call k reads;
// a tag of epoch + 2 (an overrun) is not the expected one and ends in the
// timeout path rather than in a merge of overwritten values.
#include <cuda_runtime.h>

#include "tqb_common.cuh"
#include "tqb_internal.h"
#include "tqb_merge_row.cuh"

namespace tqb {

__device__ unsigned int g_p2p_timeouts = 0;

namespace {

constexpr long long kP2PWaitCycles = 2000000000LL;  // ~1 s at 1.9 GHz
constexpr int kRow = kHeadDim + 1;                   // floats per (O, LSE) row
// The exchange merges one (b, h) row per CTA over all of the rank's splits
// (74 per row in the bench's long-context config, for only B * Hq rows):
// 16 warps keep every split's loads of a row in flight at once.
constexpr int kExchangeWarps = 16;

// One tagged element: {value bits, epoch low bits}, an aligned 8-byte
// relaxed store / load at system scope (single-copy atomic).
__device__ __forceinline__ void st_tagged(uint2* p, float v, uint32_t tag) {
    asm volatile("st.relaxed.sys.global.v2.b32 [%0], {%1, %2};\n" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag)
                 : "memory");
}
__device__ __forceinline__ uint2 ld_tagged(const uint2* p) {
    uint2 r;
    asm volatile("ld.relaxed.sys.global.v2.b32 {%0, %1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "l"(p) : "memory");
    return r;
}

// Exchange-buffer layout (bytes).
struct P2PLayout {
    int64_t recv_bytes, done_off, step_off, total;
    __host__ __device__ P2PLayout(int world, int64_t cap_rows) {
        recv_bytes = 2 * (int64_t)world * cap_rows * kRow * 8;
        done_off = recv_bytes;
        step_off = done_off + 8;
        total = step_off + 8;
    }
};
__device__ __forceinline__ uint2* recv_row(void* buf, int parity, int src, int world, int64_t cap_rows,
                                           int64_t item) {
    return static_cast<uint2*>(buf) + (((int64_t)parity * world + src) * cap_rows + item) * kRow;
}
__device__ __forceinline__ unsigned long long* step_slot(void* buf, const P2PLayout& L) {
    return reinterpret_cast<unsigned long long*>(static_cast<char*>(buf) + L.step_off);
}
// The step counter is written by an earlier kernel on this GPU (stream
// order): read it from L2, not from a line an earlier launch left in L1.
__device__ __forceinline__ unsigned long long call_epoch(unsigned long long given, void* own, const P2PLayout& L) {
    return given ? given : __ldcg(step_slot(own, L)) + 1ull;
}

// One CTA (kExchangeWarps warps) per (b, h): Stage2 merge of the local
// splits, then the tagged row to every rank (threads 0-127).
__global__ void __launch_bounds__(kExchangeWarps * 32) sp_exchange_kernel(const SpExchangeParams P) {
    pdl_trigger();
    pdl_wait();  // the local Stage1's partials
    const int64_t item = blockIdx.x;  // b * Hq + h
    const int b = (int)(item / P.s2.Hq), h = (int)(item % P.s2.Hq);
    const P2PLayout L(P.world, P.cap_rows);
    const unsigned long long epoch = call_epoch(P.epoch, P.buffers[P.rank], L);
    const int parity = (int)((epoch - 1) & 1);
    const uint32_t tag = (uint32_t)epoch;
    float o, lse;
    merge_row<kExchangeWarps>(P.s2, b, h, &o, &lse);
    const int d = threadIdx.x;
    if (d < kHeadDim) {
        for (int r = 0; r < P.world; r++) {
            uint2* row = recv_row(P.buffers[r], parity, P.rank, P.world, P.cap_rows, item);
            st_tagged(row + d, o, tag);
            if (d == 0) st_tagged(row + kHeadDim, lse, tag);
        }
    }
}

// One CTA (128 threads) per (b, h): thread d gathers element d and the LSE
// of this row from every rank (waiting for this epoch's tags), then merges
// them; the last CTA advances the device epoch.
__global__ void __launch_bounds__(kHeadDim) sp_merge_kernel(const SpMergeParams P) {
    pdl_trigger();
    pdl_wait();  // the local exchange (its reads of step happen before this kernel stores it)
    const int64_t item = blockIdx.x;
    const int b = (int)(item / P.Hq), h = (int)(item % P.Hq);
    const int d = threadIdx.x;
    const P2PLayout L(P.world, P.cap_rows);
    const unsigned long long epoch = call_epoch(P.epoch, P.buffer, L);
    const int parity = (int)((epoch - 1) & 1);
    const uint32_t tag = (uint32_t)epoch;
    float val[kP2PMaxRanks], lse[kP2PMaxRanks];
    uint32_t missing = 0;  // bit 2r: value of rank r, bit 2r+1: its LSE
#pragma unroll
    for (int r = 0; r < kP2PMaxRanks; r++) {
        val[r] = 0.0f;
        lse[r] = -INFINITY;
        if (r < P.world) {
            const uint2* row = recv_row(P.buffer, parity, r, P.world, P.cap_rows, item);
            const uint2 x = ld_tagged(row + d), y = ld_tagged(row + kHeadDim);
            val[r] = __uint_as_float(x.x);
            lse[r] = __uint_as_float(y.x);
            missing |= (x.y != tag ? 1u : 0u) << (2 * r);
            missing |= (y.y != tag ? 1u : 0u) << (2 * r + 1);
        }
    }
    if (missing) {
        const long long t0 = clock64();
        while (missing) {
            __nanosleep(32);
#pragma unroll
            for (int r = 0; r < kP2PMaxRanks; r++) {
                if (!((missing >> (2 * r)) & 3u)) continue;
                const uint2* row = recv_row(P.buffer, parity, r, P.world, P.cap_rows, item);
                if ((missing >> (2 * r)) & 1u) {
                    const uint2 x = ld_tagged(row + d);
                    val[r] = __uint_as_float(x.x);
                    if (x.y == tag) missing &= ~(1u << (2 * r));
                }
                if ((missing >> (2 * r + 1)) & 1u) {
                    const uint2 y = ld_tagged(row + kHeadDim);
                    lse[r] = __uint_as_float(y.x);
                    if (y.y == tag) missing &= ~(1u << (2 * r + 1));
                }
            }
            if (clock64() - t0 > kP2PWaitCycles) break;
        }
    }
    const bool ok = __syncthreads_and(missing == 0);
    float* out = P.out + (int64_t)b * P.osb + (int64_t)h * P.osh;
    if (!ok) {
        out[d] = __int_as_float(0x7fffffff);
        if (d == 0) {
            atomicAdd(&g_p2p_timeouts, 1u);
            if (P.lse) P.lse[(int64_t)b * P.lsb + h] = __int_as_float(0x7fffffff);
        }
    } else {
        float acc = 0.0f, rmax = -INFINITY, rsum = 0.0f;
#pragma unroll
        for (int r = 0; r < kP2PMaxRanks; r++) {
            if (r >= P.world || lse[r] == -INFINITY) continue;  // no token of this range
            const float nmax = fmaxf(rmax, lse[r]);
            const float old_scale = expf(rmax - nmax);
            const float w = expf(lse[r] - nmax);
            acc = acc * old_scale + w * val[r];
            rsum = rsum * old_scale + w;
            rmax = nmax;
        }
        out[d] = __fdiv_rn(acc, rsum);
        if (d == 0 && P.lse) P.lse[(int64_t)b * P.lsb + h] = rmax + logf(rsum);
    }
    if (!P.epoch && d == 0) {
        // device epochs: every CTA has read step before the last one (the
        // one that finds all others counted in `done`) stores this epoch
        unsigned int* done = reinterpret_cast<unsigned int*>(static_cast<char*>(P.buffer) + L.done_off);
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0u;
            *step_slot(P.buffer, L) = epoch;
        }
    }
}

}  // namespace

int64_t p2p_buffer_bytes(int world, int64_t cap_rows) { return P2PLayout(world, cap_rows).total; }

int launch_sp_exchange(const SpExchangeParams& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.s2.B * P.s2.Hq;
    if (items == 0) return TQB_OK;
    return report_launch(launch_pdl(sp_exchange_kernel, dim3((unsigned)items), dim3(kExchangeWarps * 32), 0, stream, P));
}

int launch_sp_merge(const SpMergeParams& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.B * P.Hq;
    if (items == 0) return TQB_OK;
    return report_launch(launch_pdl(sp_merge_kernel, dim3((unsigned)items), dim3(kHeadDim), 0, stream, P));
}

int read_p2p_timeouts(unsigned int* count, bool reset) {
    cudaError_t e = cudaMemcpyFromSymbol(count, g_p2p_timeouts, sizeof(unsigned int));
    if (e == cudaSuccess && reset) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_p2p_timeouts, &zero, sizeof(unsigned int));
    }
    return e == cudaSuccess ? TQB_OK : report_launch(e);
}

}  // namespace tqb
