// tqb_api.cu — the C ABI (include/tqb.h): argument validation, error
// reporting and dispatch to the kernels.  No allocation happens here or in
// any kernel; every buffer is owned by the caller.
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include "tqb_common.cuh"
#include "tqb_internal.h"

namespace {

thread_local char g_detail[256] = "";

int fail(int code, const char* fmt, const char* what) {
    snprintf(g_detail, sizeof(g_detail), fmt, what);
    return code;
}

#define TQB_REQUIRE(cond, code, msg)                   \
    do {                                               \
        if (!(cond)) return fail((code), "%s", (msg)); \
    } while (0)

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};

// Makes the device that owns `ptr` current for the duration of a call (the
// library may run beside another CUDA runtime instance, e.g. torch's, whose
// notion of the current device it must not depend on).
struct DeviceGuard {
    int prev = -1, dev = -1;
    bool ok = true;
    explicit DeviceGuard(const void* ptr) {
        cudaPointerAttributes attr{};
        if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess || attr.type != cudaMemoryTypeDevice) {
            cudaGetLastError();  // clear the sticky-free error of a failed query
            ok = (cudaGetDevice(&dev) == cudaSuccess);
            return;
        }
        dev = attr.device;
        if (cudaGetDevice(&prev) != cudaSuccess) { ok = false; return; }
        if (prev != dev && cudaSetDevice(dev) != cudaSuccess) ok = false;
    }
    ~DeviceGuard() {
        if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    }
};

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return -1;
    if (dev < kMaxDevices && g_sm_count[dev] > 0) return g_sm_count[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        return -1;
    if (dev < kMaxDevices) g_sm_count[dev] = n;
    return n;
}

}  // namespace

namespace tqb {
void set_error_detail(const char* msg) { snprintf(g_detail, sizeof(g_detail), "%s", msg); }

int report_launch(cudaError_t e) {
    if (e == cudaSuccess) return TQB_OK;
    snprintf(g_detail, sizeof(g_detail), "kernel launch: %s", cudaGetErrorString(e));
    return TQB_ERR_LAUNCH;
}
}  // namespace tqb

// AoS slot strides (bytes): token-major ([16][Hk][slot], the reference's own
// cache) or head-major ([Hk][16][slot]: vLLM's (blocks, H, N, C) storage seen
// through kv_cache.transpose(1, 2), reference/turboquant_attn.py:565), with
// every slot (of `slot` bytes) of a block inside the block stride.
static bool aos_strides_ok(int64_t block, int64_t ps, int64_t hs, int64_t hk, int64_t slot) {
    const bool token_major = hs >= slot && ps >= hk * hs;
    const bool head_major = ps >= slot && hs >= tqb::kBlockSize * ps;
    const int64_t extent = (tqb::kBlockSize - 1) * ps + (hk - 1) * hs + slot;
    return (token_major || head_major) && block >= extent && extent < (int64_t(1) << 31);
}

extern "C" {

int tqb_version(void) { return TQB_VERSION; }

int tqb_wait_timeouts(unsigned int* count, int reset) {
    g_detail[0] = '\0';
    TQB_REQUIRE(count != nullptr, TQB_ERR_INVALID_ARG, "count is NULL");
    unsigned int ring = 0, p2p = 0;
    if (tqb::read_wait_timeouts(&ring, reset != 0) != TQB_OK) return TQB_ERR_CUDA;
    if (tqb::read_p2p_timeouts(&p2p, reset != 0) != TQB_OK) return TQB_ERR_CUDA;
    *count = ring + p2p;
    return TQB_OK;
}

const char* tqb_strerror(int status) {
    switch (status) {
        case TQB_OK: return "ok";
        case TQB_ERR_INVALID_ARG: return "invalid argument";
        case TQB_ERR_UNSUPPORTED: return "unsupported shape or configuration";
        case TQB_ERR_ALIGNMENT: return "misaligned pointer or stride";
        case TQB_ERR_LAUNCH: return "kernel launch failed";
        case TQB_ERR_CUDA: return "CUDA runtime error";
        default: return "unknown tqb status";
    }
}

const char* tqb_last_error_detail(void) { return g_detail; }

// Validates Stage1 arguments and fills p (for batch > 0).
static int stage1_check(const tqb_stage1_args* a, tqb::Stage1Params& p) {
    TQB_REQUIRE(a != nullptr, TQB_ERR_INVALID_ARG, "args is NULL");
    TQB_REQUIRE(a->batch >= 0 && a->num_q_heads > 0 && a->num_kv_heads > 0 && a->num_splits > 0,
                TQB_ERR_INVALID_ARG, "batch/heads/num_splits must be positive");
    TQB_REQUIRE(a->head_dim == tqb::kHeadDim, TQB_ERR_UNSUPPORTED, "head_dim must be 128");
    TQB_REQUIRE(a->block_size == tqb::kBlockSize, TQB_ERR_UNSUPPORTED, "block_size must be 16");
    TQB_REQUIRE(tqb::layout_valid(a->layout), TQB_ERR_INVALID_ARG, "layout must be a tqb_layout value");
    const bool k8 = a->layout == TQB_LAYOUT_SOA_K8, v3 = a->layout == TQB_LAYOUT_SOA_K3V3;
    const bool k3 = a->layout == TQB_LAYOUT_SOA_K3 || v3;
    TQB_REQUIRE(tqb::layout_fp8_keys(a->layout) ||
                    a->n_centroids == (tqb::layout_3bit_keys(a->layout) ? 8 : tqb::kNumCentroids),
                TQB_ERR_UNSUPPORTED, "n_centroids must be 16 (4-bit keys) or 8 (3-bit keys)");
    TQB_REQUIRE(a->num_q_heads % a->num_kv_heads == 0, TQB_ERR_INVALID_ARG,
                "num_q_heads must be a multiple of num_kv_heads");
    const int G = a->num_q_heads / a->num_kv_heads;
    TQB_REQUIRE(G <= 8, TQB_ERR_UNSUPPORTED, "GQA group size must be <= 8");
    if (a->batch == 0) return TQB_OK;
    TQB_REQUIRE(a->q_rot && a->kv_cache && a->block_table && a->seq_lens &&
                    (a->centroids || tqb::layout_fp8_keys(a->layout)) && a->mid_o,
                TQB_ERR_INVALID_ARG, "a required pointer is NULL");
    TQB_REQUIRE(aligned(a->q_rot, 16) && a->q_stride_b % 4 == 0 && a->q_stride_h % 4 == 0,
                TQB_ERR_ALIGNMENT, "q_rot must be 16-byte aligned with strides multiple of 4");
    TQB_REQUIRE(aligned(a->mid_o, 4), TQB_ERR_ALIGNMENT, "mid_o must be 4-byte aligned");
    TQB_REQUIRE(a->mid_stride_s >= tqb::kHeadDim + 1 && a->mid_stride_h >= 0 && a->mid_stride_b >= 0,
                TQB_ERR_INVALID_ARG, "mid_o split stride must be >= head_dim + 1");
    TQB_REQUIRE(a->max_blocks_per_seq > 0 && a->block_table_stride >= a->max_blocks_per_seq,
                TQB_ERR_INVALID_ARG, "block_table row stride must be >= max_blocks_per_seq");
    const int64_t hk = a->num_kv_heads;
    if (k8) {
        TQB_REQUIRE(aligned(a->kv_cache, 16), TQB_ERR_ALIGNMENT, "SoA kv_cache must be 16-byte aligned");
        TQB_REQUIRE(a->cache_stride_block >= tqb::kBlockSize * hk * tqb::kSlotBytesK8 &&
                        a->cache_stride_block % 16 == 0,
                    TQB_ERR_ALIGNMENT, "FP8-key block stride must be >= 16*Hk*196 bytes and a multiple of 16");
    } else if (k3) {
        TQB_REQUIRE(aligned(a->kv_cache, 16), TQB_ERR_ALIGNMENT, "SoA kv_cache must be 16-byte aligned");
        TQB_REQUIRE(a->cache_stride_block >= tqb::kBlockSize * hk * (v3 ? tqb::kSlotBytesK3V3 : tqb::kSlotBytesK3) &&
                        a->cache_stride_block % 16 == 0,
                    TQB_ERR_ALIGNMENT, "3-bit-key block stride must be >= 16*Hk*slot bytes (118, or 102 with "
                                       "3-bit values) and a multiple of 16");
    } else if (a->layout == TQB_LAYOUT_SOA) {
        TQB_REQUIRE(aligned(a->kv_cache, 16), TQB_ERR_ALIGNMENT, "SoA kv_cache must be 16-byte aligned");
        TQB_REQUIRE(a->cache_stride_block >= tqb::kBlockSize * hk * tqb::kSlotBytes &&
                        a->cache_stride_block % 16 == 0,
                    TQB_ERR_ALIGNMENT, "SoA block stride must be >= 16*Hk*134 bytes and a multiple of 16");
    } else {
        TQB_REQUIRE(aligned(a->kv_cache, 2) && a->cache_stride_block % 2 == 0 &&
                        a->cache_stride_pos % 2 == 0 && a->cache_stride_head % 2 == 0,
                    TQB_ERR_ALIGNMENT, "AoS cache pointer and strides must be even");
        TQB_REQUIRE(aos_strides_ok(a->cache_stride_block, a->cache_stride_pos, a->cache_stride_head, hk,
                                   tqb::aos_slot_bytes(a->layout)),
                    TQB_ERR_INVALID_ARG,
                    "AoS strides must describe [blocks, 16, Hk, >= slot] slots (slot 134, 196, 118 or 102 bytes "
                    "by layout), token- or head-major");
    }
    p.q = a->q_rot;
    p.qsb = a->q_stride_b;
    p.qsh = a->q_stride_h;
    p.cache = a->kv_cache;
    p.block_bytes = a->cache_stride_block;
    p.pos_stride = a->cache_stride_pos;
    p.head_stride = a->cache_stride_head;
    p.layout = a->layout;
    p.bt = a->block_table;
    p.bt_stride = a->block_table_stride;
    p.max_blocks = a->max_blocks_per_seq;
    p.num_blocks = a->num_blocks;
    p.seq_lens = a->seq_lens;
    p.nsplits = a->num_splits_per_seq;
    p.cents = a->centroids;
    p.mid = a->mid_o;
    p.msb = a->mid_stride_b;
    p.msh = a->mid_stride_h;
    p.mss = a->mid_stride_s;
    p.B = a->batch;
    p.Hq = a->num_q_heads;
    p.Hk = a->num_kv_heads;
    p.G = G;
    p.S = a->num_splits;
    p.attn_scale = a->attn_scale > 0.0f ? a->attn_scale : 1.0f / sqrtf((float)tqb::kHeadDim);
    p.num_items = (int64_t)a->batch * a->num_splits * a->num_kv_heads;
    TQB_REQUIRE(p.num_items < (int64_t(1) << 31), TQB_ERR_UNSUPPORTED,
                "batch * num_splits * num_kv_heads must be < 2^31");
    p.div_hk = tqb::FastDiv((uint32_t)a->num_kv_heads);
    p.div_s = tqb::FastDiv((uint32_t)a->num_splits);
    return TQB_OK;
}

int tqb_stage1(const tqb_stage1_args* a, cudaStream_t stream) {
    g_detail[0] = '\0';
    tqb::Stage1Params p{};
    const int rc = stage1_check(a, p);
    if (rc != TQB_OK || a->batch == 0) return rc;
    DeviceGuard guard(a->mid_o);
    TQB_REQUIRE(guard.ok, TQB_ERR_CUDA, "cannot select the device owning mid_o");
    const int nsm = sm_count();
    TQB_REQUIRE(nsm > 0, TQB_ERR_CUDA, "cannot query the current CUDA device");
    return tqb::launch_stage1(p, stream, nsm);
}

int tqb_stage1_rotated(const tqb_rotate_args* r, const tqb_stage1_args* a, cudaStream_t stream) {
    g_detail[0] = '\0';
    TQB_REQUIRE(r != nullptr && a != nullptr, TQB_ERR_INVALID_ARG, "args is NULL");
    TQB_REQUIRE(r->q_rot == a->q_rot && r->out_stride_b == a->q_stride_b && r->out_stride_h == a->q_stride_h &&
                    r->batch == a->batch && r->num_q_heads == a->num_q_heads && r->head_dim == a->head_dim,
                TQB_ERR_INVALID_ARG,
                "the rotation's output must be Stage1's q_rot (same pointer, strides, batch and heads)");
    TQB_REQUIRE(r->query_dtype == TQB_DTYPE_F32 || r->query_dtype == TQB_DTYPE_F16 ||
                    r->query_dtype == TQB_DTYPE_BF16,
                TQB_ERR_INVALID_ARG, "query_dtype must be TQB_DTYPE_F32, TQB_DTYPE_F16 or TQB_DTYPE_BF16");
    tqb::Stage1Params p{};
    int rc = stage1_check(a, p);
    if (rc != TQB_OK || a->batch == 0) return rc;
    TQB_REQUIRE(r->query && r->rotation, TQB_ERR_INVALID_ARG, "query or rotation is NULL");
    TQB_REQUIRE(aligned(r->query, r->query_dtype == TQB_DTYPE_F32 ? 4 : 2) && aligned(r->rotation, 16),
                TQB_ERR_ALIGNMENT, "query must be aligned to its element size, rotation to 16 bytes");
    DeviceGuard guard(a->mid_o);
    TQB_REQUIRE(guard.ok, TQB_ERR_CUDA, "cannot select the device owning mid_o");
    const int nsm = sm_count();
    TQB_REQUIRE(nsm > 0, TQB_ERR_CUDA, "cannot query the current CUDA device");
    // One kernel where the page ring runs with a group of at most 4 query
    // heads per KV head (its rotation prologue stages the 64 KB rotation in
    // a ring it has not started yet); otherwise the rotation kernel, then
    // Stage1.
    if (p.G <= 4 && !tqb::stage1_register_kernel_forced() && tqb::stage1_ring_supported(p)) {
        tqb::Stage1Params pr = p;
        pr.rq = r->query;
        pr.rq_dtype = r->query_dtype;
        pr.rqsb = r->q_stride_b;
        pr.rqsh = r->q_stride_h;
        pr.rot = r->rotation;
        pr.q_out = r->q_rot;
        rc = tqb::launch_stage1_ring(pr, stream, nsm);
        if (rc != TQB_ERR_UNSUPPORTED) return rc;
        g_detail[0] = '\0';
    }
    rc = tqb_rotate_query(r, stream);
    if (rc != TQB_OK) return rc;
    return tqb::launch_stage1(p, stream, nsm);
}

// Stage2 with the output written as `dtype` to `out` (a->output ignored).
static int stage2_impl(const tqb_stage2_args* a, void* out, int dtype, cudaStream_t stream) {
    g_detail[0] = '\0';
    TQB_REQUIRE(a != nullptr, TQB_ERR_INVALID_ARG, "args is NULL");
    TQB_REQUIRE(dtype == TQB_DTYPE_F32 || dtype == TQB_DTYPE_F16 || dtype == TQB_DTYPE_BF16, TQB_ERR_INVALID_ARG,
                "out_dtype must be TQB_DTYPE_F32, TQB_DTYPE_F16 or TQB_DTYPE_BF16");
    TQB_REQUIRE(a->batch >= 0 && a->num_q_heads > 0 && a->num_splits > 0, TQB_ERR_INVALID_ARG,
                "batch/heads/num_splits must be positive");
    TQB_REQUIRE(a->head_dim == tqb::kHeadDim, TQB_ERR_UNSUPPORTED, "head_dim must be 128");
    TQB_REQUIRE((int64_t)a->batch * a->num_q_heads < (int64_t(1) << 31), TQB_ERR_UNSUPPORTED,
                "batch * num_q_heads must be < 2^31");
    if (a->batch == 0) return TQB_OK;
    TQB_REQUIRE(a->mid_o && a->seq_lens && out && a->lse, TQB_ERR_INVALID_ARG, "a required pointer is NULL");
    TQB_REQUIRE(aligned(a->mid_o, 4) && aligned(out, dtype == TQB_DTYPE_F32 ? 4 : 2) && aligned(a->lse, 4),
                TQB_ERR_ALIGNMENT, "buffers must be aligned to their element size");
    DeviceGuard guard(out);
    TQB_REQUIRE(guard.ok, TQB_ERR_CUDA, "cannot select the device owning output");
    tqb::Stage2Params p{};
    p.mid = a->mid_o;
    p.msb = a->mid_stride_b;
    p.msh = a->mid_stride_h;
    p.mss = a->mid_stride_s;
    p.seq_lens = a->seq_lens;
    p.nsplits = a->num_splits_per_seq;
    p.out = out;
    p.out_dtype = dtype;
    p.osb = a->out_stride_b;
    p.osh = a->out_stride_h;
    p.lse = a->lse;
    p.lsb = a->lse_stride_b;
    p.B = a->batch;
    p.Hq = a->num_q_heads;
    p.S = a->num_splits;
    return tqb::launch_stage2(p, stream);
}

int tqb_stage2(const tqb_stage2_args* a, cudaStream_t stream) {
    return stage2_impl(a, a ? a->output : nullptr, TQB_DTYPE_F32, stream);
}

int tqb_stage2_typed(const tqb_stage2_args* a, int out_dtype, void* output, cudaStream_t stream) {
    return stage2_impl(a, output, out_dtype, stream);
}

int tqb_fold_sinks(const tqb_sink_args* a, cudaStream_t stream) {
    g_detail[0] = '\0';
    TQB_REQUIRE(a != nullptr, TQB_ERR_INVALID_ARG, "args is NULL");
    TQB_REQUIRE(a->batch >= 0 && a->num_q_heads > 0, TQB_ERR_INVALID_ARG, "batch/heads must be positive");
    TQB_REQUIRE(a->head_dim == tqb::kHeadDim, TQB_ERR_UNSUPPORTED, "head_dim must be 128");
    TQB_REQUIRE((int64_t)a->batch * a->num_q_heads < (int64_t(1) << 31), TQB_ERR_UNSUPPORTED,
                "batch * num_q_heads must be < 2^31");
    if (a->batch == 0) return TQB_OK;
    TQB_REQUIRE(a->mid_o && a->seq_lens && a->sinks, TQB_ERR_INVALID_ARG, "a required pointer is NULL");
    TQB_REQUIRE(aligned(a->mid_o, 4) && aligned(a->seq_lens, 4) && aligned(a->sinks, 4), TQB_ERR_ALIGNMENT,
                "buffers must be aligned to their element size");
    DeviceGuard guard(a->mid_o);
    TQB_REQUIRE(guard.ok, TQB_ERR_CUDA, "cannot select the device owning mid_o");
    tqb::SinkParams p{};
    p.mid = a->mid_o;
    p.msb = a->mid_stride_b;
    p.msh = a->mid_stride_h;
    p.seq_lens = a->seq_lens;
    p.sinks = a->sinks;
    p.B = a->batch;
    p.Hq = a->num_q_heads;
    return tqb::launch_fold_sinks(p, stream);
}

// ---- sequence-parallel exchange over peer memory --------------------------

int64_t tqb_p2p_buffer_bytes(int32_t world, int64_t cap_rows) {
    if (world < 1 || world > tqb::kP2PMaxRanks || cap_rows < 0) return -1;
    return tqb::p2p_buffer_bytes(world, cap_rows);
}

int tqb_p2p_alloc(int64_t bytes, void** ptr) {
    g_detail[0] = '\0';
    TQB_REQUIRE(ptr != nullptr && bytes > 0, TQB_ERR_INVALID_ARG, "ptr is NULL or bytes <= 0");
    *ptr = nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, (size_t)bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, (size_t)bytes);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        cudaGetLastError();
        tqb::set_error_detail(cudaGetErrorString(e));
        return TQB_ERR_CUDA;
    }
    *ptr = p;
    return TQB_OK;
}

int tqb_p2p_free(void* ptr) {
    g_detail[0] = '\0';
    if (!ptr) return TQB_OK;
    const cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess) {
        cudaGetLastError();
        tqb::set_error_detail(cudaGetErrorString(e));
        return TQB_ERR_CUDA;
    }
    return TQB_OK;
}

int tqb_ipc_export(const void* ptr, void* handle) {
    g_detail[0] = '\0';
    TQB_REQUIRE(ptr && handle, TQB_ERR_INVALID_ARG, "ptr or handle is NULL");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess) {
        cudaGetLastError();
        tqb::set_error_detail(cudaGetErrorString(e));
        return TQB_ERR_CUDA;
    }
    static_assert(sizeof(h) == TQB_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    return TQB_OK;
}

int tqb_ipc_import(const void* handle, void** ptr) {
    g_detail[0] = '\0';
    TQB_REQUIRE(ptr && handle, TQB_ERR_INVALID_ARG, "ptr or handle is NULL");
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        cudaGetLastError();
        tqb::set_error_detail(cudaGetErrorString(e));
        return TQB_ERR_CUDA;
    }
    return TQB_OK;
}

int tqb_ipc_close(void* ptr) {
    g_detail[0] = '\0';
    if (!ptr) return TQB_OK;
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) {
        cudaGetLastError();
        tqb::set_error_detail(cudaGetErrorString(e));
        return TQB_ERR_CUDA;
    }
    return TQB_OK;
}

int tqb_sp_exchange(const tqb_sp_exchange_args* a, cudaStream_t stream) {
    g_detail[0] = '\0';
    TQB_REQUIRE(a != nullptr, TQB_ERR_INVALID_ARG, "args is NULL");
    const tqb_stage2_args* s = &a->stage2;
    TQB_REQUIRE(a->world >= 1 && a->world <= TQB_P2P_MAX_RANKS && a->rank >= 0 && a->rank < a->world,
                TQB_ERR_INVALID_ARG, "rank/world out of range");
    TQB_REQUIRE(s->batch >= 0 && s->num_q_heads > 0 && s->num_splits > 0, TQB_ERR_INVALID_ARG,
                "batch/heads/num_splits must be positive");
    TQB_REQUIRE(s->head_dim == tqb::kHeadDim, TQB_ERR_UNSUPPORTED, "head_dim must be 128");
    TQB_REQUIRE((int64_t)s->batch * s->num_q_heads <= a->cap_rows && a->cap_rows < (int64_t(1) << 31),
                TQB_ERR_INVALID_ARG, "batch * num_q_heads exceeds cap_rows");
    if (s->batch == 0) return TQB_OK;
    TQB_REQUIRE(s->mid_o && s->seq_lens, TQB_ERR_INVALID_ARG, "a required pointer is NULL");
    for (int r = 0; r < a->world; r++)
        TQB_REQUIRE(a->buffers[r] && aligned(a->buffers[r], 8), TQB_ERR_INVALID_ARG,
                    "every rank's exchange buffer must be given (8-byte aligned)");
    DeviceGuard guard(a->buffers[a->rank]);
    TQB_REQUIRE(guard.ok, TQB_ERR_CUDA, "cannot select the device owning this rank's buffer");
    tqb::SpExchangeParams p{};
    p.s2.mid = s->mid_o;
    p.s2.msb = s->mid_stride_b;
    p.s2.msh = s->mid_stride_h;
    p.s2.mss = s->mid_stride_s;
    p.s2.seq_lens = s->seq_lens;
    p.s2.nsplits = s->num_splits_per_seq;
    p.s2.B = s->batch;
    p.s2.Hq = s->num_q_heads;
    p.s2.S = s->num_splits;
    p.rank = a->rank;
    p.world = a->world;
    p.cap_rows = a->cap_rows;
    for (int r = 0; r < a->world; r++) p.buffers[r] = a->buffers[r];
    p.epoch = a->epoch;
    return tqb::launch_sp_exchange(p, stream);
}

int tqb_sp_merge(const tqb_sp_merge_args* a, cudaStream_t stream) {
    g_detail[0] = '\0';
    TQB_REQUIRE(a != nullptr, TQB_ERR_INVALID_ARG, "args is NULL");
    TQB_REQUIRE(a->world >= 1 && a->world <= TQB_P2P_MAX_RANKS, TQB_ERR_INVALID_ARG, "world out of range");
    TQB_REQUIRE(a->batch >= 0 && a->num_q_heads > 0, TQB_ERR_INVALID_ARG, "batch/heads must be positive");
    TQB_REQUIRE(a->head_dim == tqb::kHeadDim, TQB_ERR_UNSUPPORTED, "head_dim must be 128");
    TQB_REQUIRE((int64_t)a->batch * a->num_q_heads <= a->cap_rows && a->cap_rows < (int64_t(1) << 31),
                TQB_ERR_INVALID_ARG, "batch * num_q_heads exceeds cap_rows");
    if (a->batch == 0) return TQB_OK;
    TQB_REQUIRE(a->buffer && a->output && aligned(a->buffer, 8) && aligned(a->output, 4), TQB_ERR_INVALID_ARG,
                "buffer/output NULL or misaligned");
    DeviceGuard guard(a->output);
    TQB_REQUIRE(guard.ok, TQB_ERR_CUDA, "cannot select the device owning output");
    tqb::SpMergeParams p{};
    p.buffer = a->buffer;
    p.world = a->world;
    p.B = a->batch;
    p.Hq = a->num_q_heads;
    p.cap_rows = a->cap_rows;
    p.epoch = a->epoch;
    p.out = a->output;
    p.osb = a->out_stride_b;
    p.osh = a->out_stride_h;
    p.lse = a->lse;
    p.lsb = a->lse_stride_b;
    return tqb::launch_sp_merge(p, stream);
}

int tqb_rotate_query(const tqb_rotate_args* a, cudaStream_t stream) {
    g_detail[0] = '\0';
    TQB_REQUIRE(a != nullptr, TQB_ERR_INVALID_ARG, "args is NULL");
    TQB_REQUIRE(a->query_dtype == TQB_DTYPE_F32 || a->query_dtype == TQB_DTYPE_F16 ||
                    a->query_dtype == TQB_DTYPE_BF16,
                TQB_ERR_INVALID_ARG, "query_dtype must be TQB_DTYPE_F32, TQB_DTYPE_F16 or TQB_DTYPE_BF16");
    TQB_REQUIRE(a->batch >= 0 && a->num_q_heads > 0, TQB_ERR_INVALID_ARG, "batch/heads must be positive");
    TQB_REQUIRE(a->head_dim == tqb::kHeadDim, TQB_ERR_UNSUPPORTED, "head_dim must be 128");
    TQB_REQUIRE((int64_t)a->batch * a->num_q_heads < (int64_t(1) << 31), TQB_ERR_UNSUPPORTED,
                "batch * num_q_heads must be < 2^31");
    if (a->batch == 0) return TQB_OK;
    TQB_REQUIRE(a->query && a->rotation && a->q_rot, TQB_ERR_INVALID_ARG, "a required pointer is NULL");
    TQB_REQUIRE(aligned(a->query, a->query_dtype == TQB_DTYPE_F32 ? 4 : 2) && aligned(a->rotation, 16) &&
                    aligned(a->q_rot, 4),
                TQB_ERR_ALIGNMENT, "query/q_rot must be aligned to their element size, rotation to 16 bytes");
    DeviceGuard guard(a->q_rot);
    TQB_REQUIRE(guard.ok, TQB_ERR_CUDA, "cannot select the device owning q_rot");
    tqb::RotateParams p{};
    p.q = a->query;
    p.dtype = a->query_dtype;
    p.qsb = a->q_stride_b;
    p.qsh = a->q_stride_h;
    p.rot = a->rotation;
    p.out = a->q_rot;
    p.osb = a->out_stride_b;
    p.osh = a->out_stride_h;
    p.B = a->batch;
    p.Hq = a->num_q_heads;
    return tqb::launch_rotate(p, stream);
}

int tqb_merge_partials(const tqb_merge_args* a, cudaStream_t stream) {
    g_detail[0] = '\0';
    TQB_REQUIRE(a != nullptr, TQB_ERR_INVALID_ARG, "args is NULL");
    TQB_REQUIRE(a->num_parts > 0 && a->batch >= 0 && a->num_q_heads > 0, TQB_ERR_INVALID_ARG,
                "num_parts/batch/heads must be positive");
    TQB_REQUIRE(a->head_dim == tqb::kHeadDim, TQB_ERR_UNSUPPORTED, "head_dim must be 128");
    if (a->batch == 0) return TQB_OK;
    TQB_REQUIRE(a->partials && a->output, TQB_ERR_INVALID_ARG, "a required pointer is NULL");
    TQB_REQUIRE(aligned(a->partials, 4) && aligned(a->output, 4) && aligned(a->lse, 4),
                TQB_ERR_ALIGNMENT, "buffers must be 4-byte aligned");
    DeviceGuard guard(a->output);
    TQB_REQUIRE(guard.ok, TQB_ERR_CUDA, "cannot select the device owning output");
    tqb::MergeParams p{};
    p.partials = a->partials;
    p.G = a->num_parts;
    p.B = a->batch;
    p.Hq = a->num_q_heads;
    p.out = a->output;
    p.lse = a->lse;
    const int rc = tqb::launch_merge(p, stream);
    if (rc != TQB_OK) return rc;
    return TQB_OK;
}

int tqb_store(const tqb_store_args* a, cudaStream_t stream) {
    g_detail[0] = '\0';
    TQB_REQUIRE(a != nullptr, TQB_ERR_INVALID_ARG, "args is NULL");
    TQB_REQUIRE(a->num_tokens >= 0 && a->num_kv_heads > 0, TQB_ERR_INVALID_ARG,
                "num_tokens must be >= 0 and num_kv_heads > 0");
    TQB_REQUIRE(a->head_dim == tqb::kHeadDim, TQB_ERR_UNSUPPORTED, "head_dim must be 128");
    TQB_REQUIRE(a->block_size == tqb::kBlockSize, TQB_ERR_UNSUPPORTED, "block_size must be 16");
    TQB_REQUIRE(tqb::layout_valid(a->layout), TQB_ERR_INVALID_ARG, "layout must be a tqb_layout value");
    const bool k8 = a->layout == TQB_LAYOUT_SOA_K8, v3 = a->layout == TQB_LAYOUT_SOA_K3V3;
    const bool k3 = a->layout == TQB_LAYOUT_SOA_K3 || v3;
    const bool fp8 = tqb::layout_fp8_keys(a->layout);
    TQB_REQUIRE(fp8 || a->n_centroids == (tqb::layout_3bit_keys(a->layout) ? 8 : tqb::kNumCentroids),
                TQB_ERR_UNSUPPORTED, "n_centroids must be 16, or 8 for 3-bit keys");
    TQB_REQUIRE(!(fp8 && a->norm_correction), TQB_ERR_INVALID_ARG,
                "the FP8-key layouts have no norm correction");
    if (a->num_tokens == 0) return TQB_OK;
    TQB_REQUIRE((int64_t)a->num_tokens * a->num_kv_heads < ((int64_t)1 << 31), TQB_ERR_UNSUPPORTED,
                "num_tokens x num_kv_heads must be below 2^31");
    TQB_REQUIRE(a->y && a->value && a->slot_mapping && a->kv_cache && (fp8 || (a->norms && a->midpoints)),
                TQB_ERR_INVALID_ARG, "a required pointer is NULL");
    TQB_REQUIRE(!a->norm_correction || a->centroids, TQB_ERR_INVALID_ARG,
                "norm_correction requires centroids");
    TQB_REQUIRE(aligned(a->y, 16) && aligned(a->value, 16), TQB_ERR_ALIGNMENT,
                "y and value must be 16-byte aligned");
    TQB_REQUIRE(aligned(a->kv_cache, 2) && a->cache_stride_block % 2 == 0, TQB_ERR_ALIGNMENT,
                "kv_cache and its block stride must be even");
    const int64_t hk = a->num_kv_heads;
    if (k8) {
        TQB_REQUIRE(a->cache_stride_block >= tqb::kBlockSize * hk * tqb::kSlotBytesK8 &&
                        a->cache_stride_block % 4 == 0,
                    TQB_ERR_INVALID_ARG, "FP8-key block stride must be >= 16*Hk*196 bytes and a multiple of 4");
        TQB_REQUIRE(aligned(a->kv_cache, 4), TQB_ERR_ALIGNMENT, "FP8-key kv_cache must be 4-byte aligned");
    } else if (k3) {
        TQB_REQUIRE(a->cache_stride_block >= tqb::kBlockSize * hk * (v3 ? tqb::kSlotBytesK3V3 : tqb::kSlotBytesK3),
                    TQB_ERR_INVALID_ARG, "3-bit-key block stride must be >= 16*Hk*slot bytes (118, or 102 with 3-bit values)");
    } else if (a->layout == TQB_LAYOUT_SOA) {
        TQB_REQUIRE(a->cache_stride_block >= tqb::kBlockSize * hk * tqb::kSlotBytes,
                    TQB_ERR_INVALID_ARG, "SoA block stride must be >= 16*Hk*134 bytes");
    } else {
        TQB_REQUIRE(a->cache_stride_pos % 2 == 0 && a->cache_stride_head % 2 == 0, TQB_ERR_ALIGNMENT,
                    "AoS strides must be even");
        TQB_REQUIRE(aos_strides_ok(a->cache_stride_block, a->cache_stride_pos, a->cache_stride_head, hk,
                                   tqb::aos_slot_bytes(a->layout)),
                    TQB_ERR_INVALID_ARG,
                    "AoS strides must describe [blocks, 16, Hk, >= slot] slots (slot 134, 196, 118 or 102 bytes "
                    "by layout), token- or head-major");
    }
    DeviceGuard guard(a->kv_cache);
    TQB_REQUIRE(guard.ok, TQB_ERR_CUDA, "cannot select the device owning kv_cache");
    tqb::StoreParams p{};
    p.y = a->y;
    p.norms = a->norms;
    p.value = a->value;
    p.mids = a->midpoints;
    p.cents = a->centroids;
    p.slots = a->slot_mapping;
    p.cache = a->kv_cache;
    p.layout = a->layout;
    p.block_bytes = a->cache_stride_block;
    p.pos_stride = a->cache_stride_pos;
    p.head_stride = a->cache_stride_head;
    p.N = a->num_tokens;
    p.H = a->num_kv_heads;
    p.norm_correction = a->norm_correction;
    const int rc = tqb::launch_store(p, stream);
    if (rc != TQB_OK) return rc;
    return TQB_OK;
}

}  // extern "C"
