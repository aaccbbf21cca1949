// tqb_internal.h — kernel parameter blocks shared by the launchers and the
// C-ABI front end (tqb_api.cu).  Not part of the public interface.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tqb.h"

namespace tqb {

// ---- cache layout traits (tqb_layout values) ------------------------------
// Key codes: 4-bit Lloyd-Max (SOA, AOS), 3-bit Lloyd-Max (*_K3, *_K3V3) or
// e4m3 bytes (*_K8); value codes 4-bit, or 3-bit for *_K3V3.
__host__ __device__ constexpr bool layout_is_aos(int l) {
    return l == TQB_LAYOUT_AOS || l == TQB_LAYOUT_AOS_K8 || l == TQB_LAYOUT_AOS_K3 || l == TQB_LAYOUT_AOS_K3V3;
}
__host__ __device__ constexpr bool layout_fp8_keys(int l) {
    return l == TQB_LAYOUT_SOA_K8 || l == TQB_LAYOUT_AOS_K8;
}
__host__ __device__ constexpr bool layout_3bit_keys(int l) {
    return l == TQB_LAYOUT_SOA_K3 || l == TQB_LAYOUT_SOA_K3V3 || l == TQB_LAYOUT_AOS_K3 || l == TQB_LAYOUT_AOS_K3V3;
}
__host__ __device__ constexpr bool layout_3bit_values(int l) {
    return l == TQB_LAYOUT_SOA_K3V3 || l == TQB_LAYOUT_AOS_K3V3;
}
__host__ __device__ constexpr bool layout_valid(int l) { return l >= TQB_LAYOUT_SOA && l <= TQB_LAYOUT_AOS_K3V3; }
// AoS cache slot, one per (token, KV head) (reference/aos_store.py:26-116,
// :145-340): [key codes | fp16 key norm (Lloyd-Max keys only) | value codes |
// fp16 value scale | fp16 value zero].  The stored norm is the raw |k|; the
// decoder applies the norm correction c / |c| itself.
__host__ __device__ constexpr int aos_key_bytes(int l) {
    return layout_fp8_keys(l) ? 128 : layout_3bit_keys(l) ? 48 : 64;
}
__host__ __device__ constexpr int aos_norm_off(int l) { return aos_key_bytes(l); }  // absent for e4m3 keys
__host__ __device__ constexpr int aos_val_off(int l) { return aos_key_bytes(l) + (layout_fp8_keys(l) ? 0 : 2); }
__host__ __device__ constexpr int val_code_bytes(int l) { return layout_3bit_values(l) ? 48 : 64; }
__host__ __device__ constexpr int aos_scale_off(int l) { return aos_val_off(l) + val_code_bytes(l); }
__host__ __device__ constexpr int aos_slot_bytes(int l) { return aos_scale_off(l) + 4; }
static_assert(aos_slot_bytes(TQB_LAYOUT_AOS) == 134 && aos_slot_bytes(TQB_LAYOUT_AOS_K8) == 196 &&
                  aos_slot_bytes(TQB_LAYOUT_AOS_K3) == 118 && aos_slot_bytes(TQB_LAYOUT_AOS_K3V3) == 102,
              "AoS slot sizes of the reference presets");

// Division of 32-bit unsigned n < 2^31 by a fixed divisor d >= 1 with a
// multiply-high and a shift (Granlund & Montgomery, "Division by invariant
// integers using multiplication", 1994): with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (umulhi(n, m) + n) >> l.
struct FastDiv {
    uint32_t d, m, l;
    FastDiv() : d(1), m(0), l(0) {}
    explicit FastDiv(uint32_t div) : d(div) {
        l = 0;
        while ((1ull << l) < div) l++;
        m = (uint32_t)((((1ull << l) - div) << 32) / div + 1);
    }
#ifdef __CUDACC__
    __device__ __forceinline__ uint32_t div(uint32_t n) const { return (__umulhi(n, m) + n) >> l; }
#endif
};

struct Stage1Params {
    const float* q;
    int64_t qsb, qsh;
    const uint8_t* cache;
    int64_t block_bytes, pos_stride, head_stride;
    int layout;
    const int32_t* bt;
    int64_t bt_stride;
    int max_blocks;      // entries per block-table row
    int64_t num_blocks;  // physical blocks (0: unchecked)
    const int32_t* seq_lens;
    const int32_t* nsplits;
    const float* cents;
    float* mid;
    int64_t msb, msh, mss;
    int B, Hq, Hk, G, S;
    float attn_scale;
    int64_t num_items;  // B * S * Hk work items, KV head fastest (< 2^31)
    FastDiv div_hk, div_s;
    // Fused query rotation (the page-ring kernel only; rot == nullptr: off):
    // q_out[b, h, :] = float(rq[b, h, :]) @ rot, written by the kernel's
    // prologue before its producers load the rows from q (== q_out).
    const void* rq;
    int rq_dtype;  // TQB_DTYPE_*
    int64_t rqsb, rqsh;
    const float* rot;  // [D, D] row-major
    float* q_out;
};

struct Stage2Params {
    const float* mid;
    int64_t msb, msh, mss;
    const int32_t* seq_lens;
    const int32_t* nsplits;
    void* out;      // [B, Hq, D] of out_dtype
    int out_dtype;  // TQB_DTYPE_*
    int64_t osb, osh;
    float* lse;
    int64_t lsb;
    int B, Hq, S;
};

// Attention sinks folded into split 0 of mid_o (tqb_stage2.cu).
struct SinkParams {
    float* mid;
    int64_t msb, msh;
    const int32_t* seq_lens;
    const float* sinks;  // [Hq]
    int B, Hq;
};

// Sequence-parallel exchange over peer memory (tqb_p2p.cu).
constexpr int kP2PMaxRanks = 8;
struct SpExchangeParams {
    Stage2Params s2;  // this rank's splits (out/lse unused)
    int rank, world;
    int64_t cap_rows;
    void* buffers[kP2PMaxRanks];  // every rank's exchange buffer, mapped here
    unsigned long long epoch;
};
struct SpMergeParams {
    void* buffer;  // this rank's exchange buffer
    int world, B, Hq;
    int64_t cap_rows;
    unsigned long long epoch;
    float* out;
    int64_t osb, osh;
    float* lse;
    int64_t lsb;
};

// q_rot[b, h, :] = float(q[b, h, :]) @ rot (rot [D, D] row-major fp32).
struct RotateParams {
    const void* q;
    int dtype;  // TQB_DTYPE_* of q
    int64_t qsb, qsh;
    const float* rot;
    float* out;
    int64_t osb, osh;
    int B, Hq;
};

struct MergeParams {
    const float* partials;
    int G, B, Hq;
    float* out;
    float* lse;
};

struct StoreParams {
    const float* y;
    const float* norms;
    const float* value;
    const float* mids;
    const float* cents;
    const int32_t* slots;
    uint8_t* cache;
    int layout;
    int64_t block_bytes, pos_stride, head_stride;
    int N, H;
    int norm_correction;
};

// Records the CUDA error text for tqb_last_error_detail(); returns
// TQB_OK or TQB_ERR_LAUNCH.
int report_launch(cudaError_t e);
// Sets the text tqb_last_error_detail() returns on this thread.
void set_error_detail(const char* msg);

int launch_stage1(const Stage1Params& p, cudaStream_t stream, int num_sms);
// SoA Stage1 fed by the TMA page ring (tqb_stage1_ring.cu); supported when
// the cache and query rows are 16-byte aligned.
bool stage1_ring_supported(const Stage1Params& p);
// TQB_STAGE1_KERNEL=regs in the environment (read on every call) selects the
// register-ring kernel for caches the page ring also serves.
bool stage1_register_kernel_forced();
int launch_stage1_ring(const Stage1Params& p, cudaStream_t stream, int num_sms);
// Reads (and optionally clears) the count of bounded device waits that ran
// out on the current device.
int read_wait_timeouts(unsigned int* count, bool reset);
int launch_stage2(const Stage2Params& p, cudaStream_t stream);
int launch_merge(const MergeParams& p, cudaStream_t stream);
int launch_fold_sinks(const SinkParams& p, cudaStream_t stream);
int launch_rotate(const RotateParams& p, cudaStream_t stream);
int64_t p2p_buffer_bytes(int world, int64_t cap_rows);
int launch_sp_exchange(const SpExchangeParams& p, cudaStream_t stream);
int launch_sp_merge(const SpMergeParams& p, cudaStream_t stream);
int read_p2p_timeouts(unsigned int* count, bool reset);
int launch_store(const StoreParams& p, cudaStream_t stream);

}  // namespace tqb
