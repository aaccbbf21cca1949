// tqb_noalloc.cu — tqb_decode_static: Stage1 + Stage2 with the split
// partials in a file-scope device buffer instead of a caller-provided mid_o.
//
// The partial buffer is a static __device__ array of kStaticPartialRows rows
// of D+1 floats (8192 x 129 fp32 = 4,227,072 bytes, 256-byte aligned) in this
// library's module; its address is looked up once per device with
// cudaGetSymbolAddress while that device is current.  A call whose
// batch * num_q_heads * num_splits exceeds kStaticPartialRows is rejected
// with TQB_ERR_UNSUPPORTED.  Nothing in the buffer must start at zero: Stage2
// reads exactly the rows Stage1 wrote in the same call.  Calls that overlap
// on a device (different streams, or host threads) share the buffer and race.
//
// The per-device address slots are atomics: two host threads that make their
// first call on one device at the same time both look the address up and
// both store it; the lookups return the same address, so either store wins
// with the same value.
#include <cuda_runtime.h>
#include <stdio.h>

#include <atomic>

#include "tqb_common.cuh"
#include "tqb_internal.h"

namespace {

constexpr int64_t kStaticPartialRows = 8192;
constexpr int kMaxStaticDevices = 64;

__device__ __align__(256) float g_static_partials[kStaticPartialRows * (tqb::kHeadDim + 1)];

std::atomic<float*> g_static_ptr[kMaxStaticDevices] = {};

int fail(int code, const char* msg) {
    tqb::set_error_detail(msg);
    return code;
}

}  // namespace

extern "C" int tqb_decode_static(const tqb_decode_static_args* a, cudaStream_t stream) {
    if (a == nullptr) return fail(TQB_ERR_INVALID_ARG, "args is NULL");
    const tqb_stage1_args& s = a->stage1;
    const int64_t rows = (int64_t)s.batch * s.num_q_heads * s.num_splits;
    if (s.batch < 0 || s.num_q_heads <= 0 || s.num_splits <= 0 || s.head_dim != tqb::kHeadDim)
        return fail(TQB_ERR_INVALID_ARG, "batch/heads/splits must be positive and head_dim 128");
    if (rows > kStaticPartialRows) {
        char msg[160];
        snprintf(msg, sizeof(msg),
                 "batch*num_q_heads*num_splits = %lld exceeds the static partial buffer (%lld rows of 129 floats)",
                 (long long)rows, (long long)kStaticPartialRows);
        return fail(TQB_ERR_UNSUPPORTED, msg);
    }
    if (s.batch == 0) return TQB_OK;
    if (a->output == nullptr || a->lse == nullptr) return fail(TQB_ERR_INVALID_ARG, "output and lse are required");

    // The device that owns the output; its static buffer address, once.
    int dev = -1, prev = -1;
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, a->output) != cudaSuccess || attr.type != cudaMemoryTypeDevice ||
        cudaGetDevice(&prev) != cudaSuccess) {
        cudaGetLastError();
        return fail(TQB_ERR_INVALID_ARG, "output is not device memory");
    }
    dev = attr.device;
    if (dev < 0 || dev >= kMaxStaticDevices) return fail(TQB_ERR_UNSUPPORTED, "device ordinal out of range");
    float* mid = g_static_ptr[dev].load(std::memory_order_acquire);
    if (mid == nullptr) {
        if (prev != dev && cudaSetDevice(dev) != cudaSuccess) {
            cudaGetLastError();
            return fail(TQB_ERR_CUDA, "cannot select the device owning output");
        }
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_partials);
        if (prev != dev) cudaSetDevice(prev);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            return fail(TQB_ERR_CUDA, "cudaGetSymbolAddress of the static partial buffer failed");
        }
        mid = static_cast<float*>(p);
        g_static_ptr[dev].store(mid, std::memory_order_release);
    }

    tqb_stage1_args s1 = s;
    s1.mid_o = mid;
    s1.mid_stride_s = tqb::kHeadDim + 1;
    s1.mid_stride_h = (int64_t)s.num_splits * s1.mid_stride_s;
    s1.mid_stride_b = (int64_t)s.num_q_heads * s1.mid_stride_h;
    const int rc = tqb_stage1(&s1, stream);  // sets the error detail itself
    if (rc != TQB_OK) return rc;
    tqb_stage2_args s2{};
    s2.mid_o = mid;
    s2.mid_stride_b = s1.mid_stride_b;
    s2.mid_stride_h = s1.mid_stride_h;
    s2.mid_stride_s = s1.mid_stride_s;
    s2.seq_lens = s.seq_lens;
    s2.num_splits_per_seq = s.num_splits_per_seq;
    s2.output = a->output;
    s2.out_stride_b = a->out_stride_b;
    s2.out_stride_h = a->out_stride_h;
    s2.lse = a->lse;
    s2.lse_stride_b = a->lse_stride_b;
    s2.batch = s.batch;
    s2.num_q_heads = s.num_q_heads;
    s2.head_dim = s.head_dim;
    s2.num_splits = s.num_splits;
    return tqb_stage2(&s2, stream);
}
