// tqb_p2p.cu — sequence-parallel exchange of split-KV partials over peer
// memory (NVLink P2P), fused with the Stage2 merge on the sending side and
// with the cross-range merge on the receiving side.
//
// Every rank owns one exchange buffer (plain cudaMalloc, shared with the
// other ranks of the node through CUDA IPC handles; plain stores only):
//     recv  [2 parities][G ranks][cap_rows][D+1] fp32   (O, LSE) rows
//     flags [2 parities][G ranks] uint64               epoch received
//     done  uint32                                     CTAs finished (local)
//     step  uint64                                     last epoch sent (local)
// Call k of a rank (epoch k + 1) uses parity k & 1.  The epoch is either
// given by the host (1, 2, ... on every rank) or, with epoch 0 in the call,
// kept on the device in `step`: the exchange reads step + 1 and its last CTA
// stores it back, the merge reads step.  Device epochs need no host value
// per step, so a whole decode step (Stage1, exchange, merge) can be
// captured once in a CUDA graph and replayed.  One buffer uses one of the
// two forms from the start (a zero-filled buffer); they are not mixed.
//  * tqb_sp_exchange: one CTA per (b, h) merges the rank's own splits (the
//    Stage2 algebra) and stores the row straight into slot [rank] of every
//    rank's recv buffer; every thread then fences at system scope, and the
//    CTA that finishes last (a self-resetting counter) publishes the epoch
//    into flags[parity][rank] of every rank with a system-scope release store.
//  * tqb_sp_merge: each CTA waits (acquire loads, about a second at most)
//    until every rank's flag for this parity holds the epoch, then merges the
//    G rows of its (b, h) with the LSE algebra, skipping ranges whose LSE is
//    -inf (no local token).  A wait that gives up adds one to a device
//    counter (read by tqb_wait_timeouts) and writes NaN.
// The receiving side waits on other GPUs only, never on a kernel of its own
// GPU, so nothing depends on CTAs being co-resident.  Two parities suffice:
// a rank is at most one call ahead of another (its merge needs the other's
// rows of the same call), so call k + 2 never overwrites rows call k reads.
#include <cuda_runtime.h>

#include "tqb_common.cuh"
#include "tqb_internal.h"
#include "tqb_merge_row.cuh"

namespace tqb {

__device__ unsigned int g_p2p_timeouts = 0;

namespace {

constexpr long long kP2PWaitCycles = 2000000000LL;  // ~1 s at 1.9 GHz
constexpr int kRow = kHeadDim + 1;                   // floats per (O, LSE) row

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];\n" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Exchange-buffer layout (bytes).
struct P2PLayout {
    int64_t recv_bytes, flags_off, done_off, step_off, total;
    __host__ __device__ P2PLayout(int world, int64_t cap_rows) {
        recv_bytes = 2 * (int64_t)world * cap_rows * kRow * 4;
        flags_off = (recv_bytes + 7) / 8 * 8;
        done_off = flags_off + 2 * (int64_t)world * 8;
        step_off = done_off + 8;
        total = step_off + 8;
    }
};
__device__ __forceinline__ unsigned long long* step_slot(void* buf, const P2PLayout& L) {
    return reinterpret_cast<unsigned long long*>(static_cast<char*>(buf) + L.step_off);
}
// The step counter is written by an earlier kernel on this GPU (stream
// order): read it from L2, not from a line an earlier launch left in L1.
__device__ __forceinline__ unsigned long long ld_cg_u64(const unsigned long long* p) {
    return __ldcg(p);
}
__device__ __forceinline__ float* recv_slot(void* buf, int parity, int src, int world, int64_t cap_rows) {
    return static_cast<float*>(buf) + ((int64_t)parity * world + src) * cap_rows * kRow;
}
__device__ __forceinline__ unsigned long long* flag_slot(void* buf, const P2PLayout& L, int parity, int src,
                                                         int world) {
    return reinterpret_cast<unsigned long long*>(static_cast<char*>(buf) + L.flags_off) + (int64_t)parity * world +
           src;
}

// One CTA (128 threads) per (b, h): Stage2 merge of the local splits, the
// row to every rank, then the epoch from the last CTA.
__global__ void __launch_bounds__(kHeadDim) sp_exchange_kernel(const SpExchangeParams P) {
    const int64_t item = blockIdx.x;  // b * Hq + h
    const int b = (int)(item / P.s2.Hq), h = (int)(item % P.s2.Hq);
    float o, lse;
    merge_row(P.s2, b, h, &o, &lse);
    const P2PLayout L(P.world, P.cap_rows);
    // Device epochs: every CTA reads step before the last CTA advances it
    // (the last CTA is the one that finds all others counted in `done`).
    const unsigned long long epoch = P.epoch ? P.epoch : ld_cg_u64(step_slot(P.buffers[P.rank], L)) + 1ull;
    const int parity = (int)((epoch - 1) & 1);
    const int d = threadIdx.x;
    for (int r = 0; r < P.world; r++) {
        float* row = recv_slot(P.buffers[r], parity, P.rank, P.world, P.cap_rows) + item * kRow;
        row[d] = o;
        if (d == 0) row[kHeadDim] = lse;
    }
    // every thread's stores reach every GPU before this CTA counts as done
    __threadfence_system();
    __syncthreads();
    if (d == 0) {
        unsigned int* done = reinterpret_cast<unsigned int*>(static_cast<char*>(P.buffers[P.rank]) + L.done_off);
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            // the last CTA: all rows of this rank are visible; publish the epoch
            __threadfence_system();
            *done = 0u;  // ready for the next call (a later launch on this stream)
            if (!P.epoch) *step_slot(P.buffers[P.rank], L) = epoch;
            for (int r = 0; r < P.world; r++)
                st_release_sys_u64(flag_slot(P.buffers[r], L, parity, P.rank, P.world), epoch);
        }
    }
}

// One CTA (128 threads) per (b, h): wait for every rank's rows of this
// epoch, then merge them.
__global__ void __launch_bounds__(kHeadDim) sp_merge_kernel(const SpMergeParams P) {
    __shared__ int s_ok;
    const int64_t item = blockIdx.x;
    const int b = (int)(item / P.Hq), h = (int)(item % P.Hq);
    const P2PLayout L(P.world, P.cap_rows);
    // device epochs: this rank's exchange, earlier on this stream, stored it
    const unsigned long long epoch = P.epoch ? P.epoch : ld_cg_u64(step_slot(P.buffer, L));
    const int parity = (int)((epoch - 1) & 1);
    if (threadIdx.x == 0) {
        int ok = 1;
        for (int r = 0; r < P.world && ok; r++) {
            const unsigned long long* f = flag_slot(P.buffer, L, parity, r, P.world);
            // A flag of this parity holds epoch - 2 (not yet sent) or epoch
            // (sent).  Anything else (epoch + 2: the peer already overwrote
            // these rows with a later step) is not ready either, so it ends
            // in the timeout path (NaN and a counted timeout) rather than a
            // merge of overwritten rows.
            if (ld_acquire_sys_u64(f) == epoch) continue;
            const long long t0 = clock64();
            for (;;) {
                if (ld_acquire_sys_u64(f) == epoch) break;
                if (clock64() - t0 > kP2PWaitCycles) {
                    atomicAdd(&g_p2p_timeouts, 1u);
                    ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        s_ok = ok;
    }
    __syncthreads();
    const int d = threadIdx.x;
    float* out = P.out + (int64_t)b * P.osb + (int64_t)h * P.osh;
    if (!s_ok) {
        out[d] = __int_as_float(0x7fffffff);
        if (d == 0 && P.lse) P.lse[(int64_t)b * P.lsb + h] = __int_as_float(0x7fffffff);
        return;
    }
    float acc = 0.0f, rmax = -INFINITY, rsum = 0.0f;
    for (int r = 0; r < P.world; r++) {
        const float* row = recv_slot(P.buffer, parity, r, P.world, P.cap_rows) + item * kRow;
        const float slse = row[kHeadDim];
        if (slse == -INFINITY) continue;  // no token of this range
        const float nmax = fmaxf(rmax, slse);
        const float old_scale = expf(rmax - nmax);
        const float w = expf(slse - nmax);
        acc = acc * old_scale + w * row[d];
        rsum = rsum * old_scale + w;
        rmax = nmax;
    }
    out[d] = __fdiv_rn(acc, rsum);
    if (d == 0 && P.lse) P.lse[(int64_t)b * P.lsb + h] = rmax + logf(rsum);
}

}  // namespace

int64_t p2p_buffer_bytes(int world, int64_t cap_rows) { return P2PLayout(world, cap_rows).total; }

int launch_sp_exchange(const SpExchangeParams& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.s2.B * P.s2.Hq;
    if (items == 0) return TQB_OK;
    sp_exchange_kernel<<<(unsigned)items, kHeadDim, 0, stream>>>(P);
    return report_launch(cudaGetLastError());
}

int launch_sp_merge(const SpMergeParams& P, cudaStream_t stream) {
    const int64_t items = (int64_t)P.B * P.Hq;
    if (items == 0) return TQB_OK;
    sp_merge_kernel<<<(unsigned)items, kHeadDim, 0, stream>>>(P);
    return report_launch(cudaGetLastError());
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
