/*
 * tqb.h — C ABI of the B200-native TurboQuant `turboquant_4bit_nc` decode path.
 *
 * The library (libtqb.so) holds hand-written sm_100a kernels for the decode
 * Stage1 (split-KV partial attention over the 4-bit paged cache), the Stage2
 * log-sum-exp merge, the cross-GPU merge of partial results, and the cache
 * store.  Every entry point:
 *   - takes plain device pointers, sizes and byte/element strides (no torch
 *     types), and the CUDA stream to launch on;
 *   - launches asynchronously;
 *   - returns TQB_OK (0) or a negative tqb_status; tqb_strerror() names it
 *     and tqb_last_error_detail() says which argument was rejected (per
 *     calling thread).
 * Memory: the decode, store and merge entry points allocate no device
 * memory; the caller owns every buffer.  Two exceptions are named here:
 * tqb_p2p_alloc allocates the sequence-parallel exchange buffer (that is its
 * purpose), and tqb_decode_static uses a static partial buffer that the
 * library holds on every device it runs on (4,227,072 bytes, a module-scope
 * __device__ array, not an allocation per call).
 * Library state: a per-device cache of device attributes and tensor-map
 * support, the per-device address of tqb_decode_static's buffer, and device
 * counters of bounded waits that gave up (tqb_wait_timeouts).  Calls on
 * different streams may run concurrently, except tqb_decode_static calls on
 * one device (they share its buffer).
 *
 * Reference interfaces replaced (paths inside zben777/turboquant-cuda-decode):
 *   tqb_stage1   <- launch_soa_v1_stage1 / launch_aos_v1_stage1
 *                   (baseline/triton_v1.py:90-97,145-152),
 *                   launch_tq4_v2_stage1 (baseline/triton_v2.py:569-577),
 *                   tq4_cuda_vN pybind entry (cuda/tq4_cuda_v9_bind.cpp:3-8,
 *                   cuda/tq4_cuda_v9.cu:276-306), and the Stage1 launch inside
 *                   triton_turboquant_decode_attention
 *                   (reference/soa_decode_v1.py:563-608)
 *   tqb_stage2   <- launch_stage2 (baseline/stage2.py:58-81),
 *                   tq4_cuda_v7_stage2 (cuda/tq4_cuda_v7.cu:56-76)
 *   tqb_merge_partials  (no counterpart: the reference is single-GPU; this
 *                   merges per-GPU (O, LSE) partials with the same algebra as
 *                   baseline/stage2.py:44-55)
 *   tqb_store    <- triton_turboquant_store kernel launch
 *                   (reference/soa_store.py:494-524, reference/aos_store.py:420-447)
 *   tqb_rotate_query <- the launcher's query cast + rotation GEMM + copy,
 *                   q_rot = (query.float() @ PiT).contiguous()
 *                   (reference/soa_decode_v1.py:535-538)
 *   tqb_stage2_typed <- the Stage2 launch plus the final output.to(query.dtype)
 *                   (reference/soa_decode_v1.py:625-643)
 */
#ifndef TQB_H_
#define TQB_H_

#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TQB_VERSION 1000 /* 1.0.0 */

typedef enum tqb_status {
    TQB_OK = 0,
    TQB_ERR_INVALID_ARG = -1,  /* null pointer, bad size or stride */
    TQB_ERR_UNSUPPORTED = -2,  /* shape outside the kernels' envelope */
    TQB_ERR_ALIGNMENT = -3,    /* pointer or stride misaligned */
    TQB_ERR_LAUNCH = -4,       /* cudaGetLastError after the launch */
    TQB_ERR_CUDA = -5          /* other CUDA runtime failure */
} tqb_status;

typedef enum tqb_dtype {
    TQB_DTYPE_F32 = 0,
    TQB_DTYPE_F16 = 1,
    TQB_DTYPE_BF16 = 2
} tqb_dtype;

typedef enum tqb_layout {
    TQB_LAYOUT_SOA = 0,    /* block = [16 tok][Hk][K64|V64] + [Hk][3][16] fp16 meta */
    TQB_LAYOUT_AOS = 1,    /* slot  = [K64 | knorm | V64 | vscale | vzero] */
    /* turboquant_k8v4 (FP8 keys, reference/config.py:21-25, SoA form of
     * reference/soa_store.py:125-221): block = [16 tok][Hk][K128 e4m3 | V64]
     * + [Hk][2][16] fp16 meta (vscale, vzero); 196 bytes per token-head.  The
     * query is not rotated and the centroids are unused (may be NULL). */
    TQB_LAYOUT_SOA_K8 = 2,
    /* turboquant_k3v4_nc (3-bit keys, reference/config.py:31-35): block =
     * [16 tok][Hk][K48 | V64] + [Hk][3][16] fp16 meta (knorm, vscale, vzero),
     * 118 bytes per token-head; key dim d at bits 3d..3d+2 of its 48 bytes
     * (little-endian, reference/soa_store.py:330-340); 8 centroids. */
    TQB_LAYOUT_SOA_K3 = 3,
    /* turboquant_3bit_nc (reference/config.py:36-40): as TQB_LAYOUT_SOA_K3
     * with 3-bit values too: [16 tok][Hk][K48 | V48] + [Hk][3][16] fp16 meta,
     * 102 bytes per token-head; value dim d at bits 3d..3d+2 of its 48 bytes,
     * v = code * vscale + vzero with codes 0..7. */
    TQB_LAYOUT_SOA_K3V3 = 4,
    /* AoS forms of the three presets above (reference/aos_store.py:26-340,
     * reference/aos_decode.py:43-313): one slot per (token, KV head),
     * [key codes | fp16 key norm | value codes | fp16 vscale | fp16 vzero],
     * addressed like TQB_LAYOUT_AOS through the position and head strides.
     * TQB_LAYOUT_AOS_K8: 128 e4m3 key bytes, no norm, 64 value bytes: 196
     * bytes.  TQB_LAYOUT_AOS_K3: 48 bytes of 3-bit keys, the raw norm, 64
     * value bytes: 118 bytes.  TQB_LAYOUT_AOS_K3V3: as AOS_K3 with 48 bytes of
     * 3-bit values: 102 bytes.  Like TQB_LAYOUT_AOS, the Lloyd-Max forms store
     * the raw |k| and Stage1 applies the norm correction c / |c|. */
    TQB_LAYOUT_AOS_K8 = 5,
    TQB_LAYOUT_AOS_K3 = 6,
    TQB_LAYOUT_AOS_K3V3 = 7
} tqb_layout;

/*
 * Stage1: mid_o[b, h, s, 0:D] = softmax-normalised partial output of split s
 * of sequence b for query head h; mid_o[b, h, s, D] = natural-log LSE.
 * Split rule (reference/soa_decode_v1.py:104-110): split_len =
 * ceil(seq_len / n_s), split s covers [s*split_len, min((s+1)*split_len,
 * seq_len)); empty splits are left unwritten, exactly like the reference.
 * n_s = num_splits, or num_splits_per_seq[b] when that array is given
 * (entries s >= n_s are left unwritten too).
 */
typedef struct tqb_stage1_args {
    const float* q_rot;          /* [B, Hq, D] fp32, unit inner stride */
    int64_t q_stride_b;          /* elements */
    int64_t q_stride_h;          /* elements */
    const uint8_t* kv_cache;     /* [num_blocks, block_size, Hk, slot] uint8 */
    int32_t layout;              /* tqb_layout */
    int64_t cache_stride_block;  /* bytes between physical blocks */
    int64_t cache_stride_pos;    /* bytes between tokens (AoS only) */
    int64_t cache_stride_head;   /* bytes between KV heads (AoS only) */
    int64_t num_blocks;          /* physical blocks (0: skip the range check) */
    const int32_t* block_table;  /* [B, max_blocks_per_seq] */
    int64_t block_table_stride;  /* elements between rows */
    int32_t max_blocks_per_seq;
    const int32_t* seq_lens;     /* [B] */
    const float* centroids;      /* [n_centroids] fp32 Lloyd-Max codebook */
    int32_t n_centroids;         /* 16 (4-bit keys) or 8 (3-bit keys); unused for e4m3 keys */
    const float* pair_lut;       /* optional [256, 2]; accepted, not needed */
    const int32_t* num_splits_per_seq; /* optional [B] */
    float* mid_o;                /* [B, Hq, S, D+1] fp32, unit inner stride */
    int64_t mid_stride_b;        /* elements */
    int64_t mid_stride_h;
    int64_t mid_stride_s;
    int32_t batch;               /* B */
    int32_t num_q_heads;         /* Hq */
    int32_t num_kv_heads;        /* Hk; Hq % Hk == 0, Hq / Hk <= 8 */
    int32_t head_dim;            /* D, must be 128 */
    int32_t block_size;          /* must be 16 */
    int32_t num_splits;          /* S: split count, and the mid_o split extent */
    float attn_scale;            /* <= 0 selects 1/sqrt(D) */
} tqb_stage1_args;

int tqb_stage1(const tqb_stage1_args* args, cudaStream_t stream);

/*
 * Stage2: merge the non-empty splits of mid_o into output[b, h, 0:D] and
 * lse[b, h] (baseline/stage2.py:33-58).  A sequence with no non-empty split
 * (seq_len 0) gets output NaN and lse -inf, as in the reference.
 */
typedef struct tqb_stage2_args {
    const float* mid_o;
    int64_t mid_stride_b, mid_stride_h, mid_stride_s; /* elements */
    const int32_t* seq_lens;
    const int32_t* num_splits_per_seq; /* optional [B] */
    float* output;                     /* [B, Hq, D] */
    int64_t out_stride_b, out_stride_h;
    float* lse;                        /* [B, Hq] */
    int64_t lse_stride_b;
    int32_t batch, num_q_heads, head_dim, num_splits;
} tqb_stage2_args;

int tqb_stage2(const tqb_stage2_args* args, cudaStream_t stream);

/*
 * Stage2 with the output written directly in `out_dtype` (a tqb_dtype) to
 * `output` (args->output is ignored; its strides, in elements, still apply):
 * the fp32 result rounded to nearest even, bit-identical to Stage2 followed
 * by the launcher's output.to(query.dtype) (reference/soa_decode_v1.py:643).
 */
int tqb_stage2_typed(const tqb_stage2_args* args, int out_dtype, void* output, cudaStream_t stream);

/*
 * Attention sinks: folds the per-head sink logit sinks[h] (natural-log units,
 * like the scaled scores) into split 0 of mid_o for every sequence with
 * seq_len > 0, as one extra token of value 0.  Stage1 followed by this call
 * equals the reference Stage1 with USE_SINKS (reference/soa_decode_v1.py:
 * 134-145, 565-605: split 0 starts its online softmax at m = sinks[h],
 * l = 1); a sink of -inf leaves the row unchanged.  Stream-ordered after
 * Stage1, before Stage2 (or the cross-GPU merge).
 */
typedef struct tqb_sink_args {
    float* mid_o;                      /* [B, Hq, S, D + 1]; split 0 rewritten in place */
    int64_t mid_stride_b, mid_stride_h; /* elements */
    const int32_t* seq_lens;           /* [B] */
    const float* sinks;                /* [Hq] fp32 */
    int32_t batch, num_q_heads, head_dim;
} tqb_sink_args;

int tqb_fold_sinks(const tqb_sink_args* args, cudaStream_t stream);

/*
 * Query rotation: q_rot[b, h, :] = float(query[b, h, :]) @ rotation, with
 * rotation = Pi^T, a [D, D] row-major fp32 matrix, accumulated in fp32 (the
 * launcher's cast + GEMM + copy, reference/soa_decode_v1.py:535-538, in one
 * kernel).  query: [B, Hq, D] of query_dtype with unit stride over D.
 */
typedef struct tqb_rotate_args {
    const void* query;
    int32_t query_dtype;               /* tqb_dtype */
    int64_t q_stride_b, q_stride_h;    /* elements */
    const float* rotation;             /* [D, D] row-major, 16-byte aligned */
    float* q_rot;                      /* [B, Hq, D] */
    int64_t out_stride_b, out_stride_h;
    int32_t batch, num_q_heads, head_dim;
} tqb_rotate_args;

int tqb_rotate_query(const tqb_rotate_args* args, cudaStream_t stream);

/*
 * Query rotation fused into Stage1 (reference/soa_decode_v1.py:535-608, the
 * launcher's cast + rotation GEMM + copy followed by the Stage1 launch; the
 * reference's unified attention rotates inside its kernel,
 * reference/soa_unified.py:88-124).  rot describes the rotation exactly as
 * for tqb_rotate_query, and its output must be Stage1's query: rot->q_rot ==
 * s1->q_rot with the same strides, batch and heads.  On return q_rot holds
 * float(query) @ rotation (bit-identical to tqb_rotate_query) and mid_o the
 * Stage1 result.  Where the page-ring Stage1 serves the cache (4-bit or
 * 3-bit-key SoA, or 4-bit AoS, the whole-block forms with Hk dividing 8; not
 * FP8 keys, whose query the reference does not rotate) and the GQA group is
 * at most 4, this is ONE kernel: a
 * cooperative launch of one CTA per SM whose prologue rotates an equal
 * share of the rows, followed by a grid barrier (a static counter of the
 * library, bounded wait); otherwise tqb_rotate_query then tqb_stage1 on the
 * same stream.  Fused calls on one device must not overlap in time (issue
 * them on one stream): they share that counter.
 */
int tqb_stage1_rotated(const tqb_rotate_args* rot, const tqb_stage1_args* s1, cudaStream_t stream);

/*
 * Cross-GPU merge: partials[g, b, h, 0:D] / partials[g, b, h, D] are the
 * (O, LSE) of G disjoint KV ranges (one per GPU, already gathered into this
 * GPU's memory).  Ranges whose LSE is -inf (no tokens) are skipped.
 */
typedef struct tqb_merge_args {
    const float* partials;       /* [G, B, Hq, D+1] contiguous */
    int32_t num_parts;           /* G */
    int32_t batch, num_q_heads, head_dim;
    float* output;               /* [B, Hq, D] contiguous */
    float* lse;                  /* [B, Hq] contiguous, may be NULL */
} tqb_merge_args;

int tqb_merge_partials(const tqb_merge_args* args, cudaStream_t stream);

/*
 * Store: quantise N tokens x H heads into the paged cache
 * (reference/soa_store.py:223-373, reference/aos_store.py:221-340).
 * Inputs are the kernel inputs of the reference launcher: y = rotated unit
 * keys (x / (|x| + 1e-8)) @ PiT, the key norms |x|, and the raw values, all
 * fp32 [N*H, D].  Bucketising, packing, norm folding (SoA,
 * norm_correction=1) and value quantisation are bit-exact with the
 * reference arithmetic.  Negative slot_mapping entries are skipped.
 * Other presets: TQB_LAYOUT_SOA_K3 / _K3V3 take the same inputs with 8
 * centroids and 7 midpoints (3-bit keys; _K3V3 also quantises values to 7
 * levels); TQB_LAYOUT_SOA_K8 takes the raw keys in y, cast to e4m3 (round to
 * nearest even, saturating at +-448, reference/soa_store.py:125-221), with
 * norms, midpoints and centroids unused (may be NULL) and no norm correction.
 */
typedef struct tqb_store_args {
    const float* y;              /* [N*H, D] */
    const float* norms;          /* [N*H] */
    const float* value;          /* [N*H, D] */
    const float* midpoints;      /* [n_centroids - 1] */
    const float* centroids;      /* [n_centroids] */
    const int32_t* slot_mapping; /* [N] */
    uint8_t* kv_cache;
    int32_t layout;              /* tqb_layout */
    int64_t cache_stride_block, cache_stride_pos, cache_stride_head; /* bytes */
    int64_t num_blocks;          /* 0: skip the range check */
    int32_t num_tokens;          /* N */
    int32_t num_kv_heads;        /* H */
    int32_t head_dim;            /* 128 */
    int32_t block_size;          /* 16 */
    int32_t n_centroids;         /* 16 (8 for the 3-bit-key layouts; ignored for K8) */
    int32_t norm_correction;     /* SoA: fold 1/|c| into the stored norm */
} tqb_store_args;

int tqb_store(const tqb_store_args* args, cudaStream_t stream);

const char* tqb_strerror(int status);
const char* tqb_last_error_detail(void);
int tqb_version(void);

/*
 * Allocation-free decode (no reference counterpart): Stage1 + Stage2 with
 * the split partials kept in a static device buffer of the library instead
 * of a caller-provided mid_o (stage1.mid_o and its strides are ignored).
 * For callers that cannot allocate per call: a C or C++ host without a
 * caching allocator (cudaMalloc/cudaFree synchronise the device on every
 * step) and serving loops whose device memory is planned up front.
 * Limit: batch * num_q_heads * num_splits <= 8192 (8192 rows of 129 floats,
 * 4,227,072 bytes per device); larger calls return TQB_ERR_UNSUPPORTED.  The
 * buffer address is looked up on the first call on each device; make that
 * first call before any stream capture.  Calls that overlap on one device
 * share the buffer and race: serialise them.
 */
typedef struct tqb_decode_static_args {
    tqb_stage1_args stage1;      /* as for tqb_stage1; mid_o fields ignored */
    float* output;               /* [B, Hq, D] */
    int64_t out_stride_b, out_stride_h;
    float* lse;                  /* [B, Hq] */
    int64_t lse_stride_b;
} tqb_decode_static_args;

int tqb_decode_static(const tqb_decode_static_args* args, cudaStream_t stream);

/*
 * Sequence-parallel exchange over peer memory (no reference counterpart: the
 * reference is single-GPU).  Each rank of one node allocates an exchange
 * buffer of tqb_p2p_buffer_bytes(world, cap_rows) bytes with tqb_p2p_alloc,
 * exports it with tqb_ipc_export, and maps every other rank's buffer with
 * tqb_ipc_import (the handles travel over the caller's own channel).  Per
 * decode step, after the local Stage1:
 *   tqb_sp_exchange: Stage2 of this rank's splits, each merged (O, LSE) row
 *     stored straight into every rank's buffer over NVLink, then the step's
 *     epoch published to every rank;
 *   tqb_sp_merge: waits (bounded, about a second) for every rank's epoch and
 *     merges the G rows per (b, h) into output / lse (the cross-range merge
 *     of tqb_merge_partials).
 * epoch is 1 on the first step and grows by one per step, identically on all
 * ranks; consecutive steps alternate between two row sets, so a rank may run
 * one step ahead of another.  epoch 0 keeps the epoch on the device instead
 * (a counter in the rank's buffer that the exchange advances and the merge
 * reads): no per-step host value, so Stage1 + exchange + merge can be
 * captured in one CUDA graph and replayed.  A buffer uses host epochs or
 * device epochs from its first step on, never both.  A merge whose wait gives
 * up writes NaN and counts in tqb_wait_timeouts.  Every rank must call both,
 * in the same order.
 */
#define TQB_P2P_MAX_RANKS 8
#define TQB_IPC_HANDLE_BYTES 64

int64_t tqb_p2p_buffer_bytes(int32_t world, int64_t cap_rows); /* -1 when out of range */
int tqb_p2p_alloc(int64_t bytes, void** ptr);                   /* zero-filled device memory */
int tqb_p2p_free(void* ptr);
int tqb_ipc_export(const void* ptr, void* handle);              /* handle: TQB_IPC_HANDLE_BYTES */
int tqb_ipc_import(const void* handle, void** ptr);
int tqb_ipc_close(void* ptr);

typedef struct tqb_sp_exchange_args {
    tqb_stage2_args stage2;            /* this rank's Stage2 inputs; output/lse ignored */
    int32_t rank, world;               /* world <= TQB_P2P_MAX_RANKS */
    int64_t cap_rows;                  /* rows per slot, >= batch * num_q_heads, same on all ranks */
    void* buffers[TQB_P2P_MAX_RANKS];  /* every rank's buffer as mapped in this process */
    uint64_t epoch;                    /* >= 1: host epoch; 0: device epoch */
} tqb_sp_exchange_args;

int tqb_sp_exchange(const tqb_sp_exchange_args* args, cudaStream_t stream);

typedef struct tqb_sp_merge_args {
    void* buffer;                      /* this rank's exchange buffer */
    int32_t world, batch, num_q_heads, head_dim;
    int64_t cap_rows;
    uint64_t epoch;                    /* the exchange's epoch, or 0 with device epochs */
    float* output;                     /* [B, Hq, D] */
    int64_t out_stride_b, out_stride_h;
    float* lse;                        /* [B, Hq], may be NULL */
    int64_t lse_stride_b;
} tqb_sp_merge_args;

int tqb_sp_merge(const tqb_sp_merge_args* args, cudaStream_t stream);

/* Diagnostics (no reference counterpart).  The page-ring Stage1 kernel paces
 * its TMA page ring with mbarrier waits that give up after about a second; each
 * wait that gives up adds one to a per-device counter (the kernel then ends
 * early and its mid_o is not valid).  Copies the counter of the current
 * device into *count and clears it when `reset` is non-zero.  Synchronous:
 * waits for the device's outstanding work. */
int tqb_wait_timeouts(unsigned int* count, int reset);

#ifdef __cplusplus
}
#endif

#endif /* TQB_H_ */
