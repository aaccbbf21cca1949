/*
 * tq_oracle.c — CPU restatement of the TurboQuant `turboquant_4bit_nc`
 * store, decode Stage1 and Stage2 merge.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
 * compared against (and the timed CPU baseline in bench.py).  The product
 * library never links, loads or calls it.
 *
 * Parity of this restatement is pinned against the reference's own Triton
 * kernels run under TRITON_INTERPRET=1 (fixtures in tests/golden/, produced by
 * tests/golden/make_golden.py).  All arithmetic is fp32 in the reference's
 * operation order, so the store is bit-exact and Stage1 agrees with the
 * interpreted reference to fp32 reassociation.
 *
 * Reference citations are paths inside zben777/turboquant-cuda-decode.
 *
 * Build: see oracle/Makefile (gcc -O2 -fopenmp -shared -fPIC).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define TQO_LAYOUT_SOA 0
#define TQO_LAYOUT_AOS 1

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32 (IEEE binary16, round-to-nearest-even)                      */
/* ------------------------------------------------------------------------ */

static float half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) { /* inf / nan */
        return (uint16_t)(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
    }
    if (absx >= 0x477FF000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7C00u);
    }
    if (absx < 0x38800000u) { /* below the smallest normal half: subnormal */
        if (absx < 0x33000000u) return (uint16_t)sign; /* < 2^-25 -> 0 */
        uint32_t e = absx >> 23;
        uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126 - e; /* 14 + (113 - e) ... value = m * 2^(e-150) */
        /* half subnormal unit is 2^-24: result = m * 2^(e-150+24) */
        uint32_t sh = shift; /* = 150 - 24 - e  = 126 - e */
        uint32_t q = m >> sh;
        uint32_t rem = m & ((1u << sh) - 1u);
        uint32_t halfway = 1u << (sh - 1);
        if (rem > halfway || (rem == halfway && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (absx >> 23) - 127 + 15;
    uint32_t m = absx & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

float tqo_half_to_float(uint16_t h) { return half_to_float(h); }
uint16_t tqo_float_to_half(float f) { return float_to_half(f); }

/* numpy's float32 sum of a contiguous run of n <= 128 values (8 running
 * partial sums, then a fixed pairwise combine).  The Triton interpreter
 * lowers tl.sum to np.sum, so this is the reference's summation order for
 * the 128-wide reductions of reference/soa_store.py:348. */
static float np_sum_f32(const float* a, int n) {
    if (n < 8) {
        float s = 0.0f; /* numpy starts from -0.0; identical for these sums */
        for (int i = 0; i < n; i++) s += a[i];
        return s;
    }
    float r[8];
    for (int j = 0; j < 8; j++) r[j] = a[j];
    int i;
    for (i = 8; i < n - (n % 8); i += 8)
        for (int j = 0; j < 8; j++) r[j] += a[i + j];
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; i++) res += a[i];
    return res;
}

/* ------------------------------------------------------------------------ */
/* Store: bucketize + pack + folded norm + value quantise                    */
/* reference/soa_store.py:223-373 (SoA), reference/aos_store.py:221-340 (AoS) */
/* ------------------------------------------------------------------------ */

/* Binary-search bucketize over the 15 midpoints, `y >= mid` goes right
 * (reference/soa_store.py:306-316). */
static int bucketize(float y, const float* mids, int n_centroids, int bits) {
    int lo = 0, hi = n_centroids - 1;
    for (int it = 0; it < bits; it++) {
        int mid = (lo + hi) >> 1;
        int safe = mid < n_centroids - 2 ? mid : n_centroids - 2;
        if (y >= mids[safe]) lo = mid + 1; else hi = mid;
    }
    return lo < n_centroids - 1 ? lo : n_centroids - 1;
}

/* Value quantiser (reference/soa_store.py:85-116): min/max, scale =
 * max((max-min)/15, 1e-8), q = clamp(int((v-min)/scale + 0.5), 0, 15). */
static void quantise_value(const float* v, int D, uint8_t* packed,
                           uint16_t* scale_h, uint16_t* zero_h) {
    float vmin = INFINITY, vmax = -INFINITY;
    for (int d = 0; d < D; d++) {
        vmin = v[d] < vmin ? v[d] : vmin;
        vmax = v[d] > vmax ? v[d] : vmax;
    }
    volatile float range = vmax - vmin;
    float scale = range / 15.0f;
    scale = scale > 1e-8f ? scale : 1e-8f;
    for (int j = 0; j < D / 2; j++) {
        int q2[2];
        for (int k = 0; k < 2; k++) {
            volatile float t = (v[2 * j + k] - vmin);
            volatile float u = t / scale;
            volatile float w = u + 0.5f;
            int q = (int)w; /* fptosi: truncation toward zero */
            q = q < 0 ? 0 : q;
            q = q > 15 ? 15 : q;
            q2[k] = q;
        }
        packed[j] = (uint8_t)((q2[0] & 0xF) | ((q2[1] & 0xF) << 4));
    }
    *scale_h = float_to_half(scale);
    *zero_h = float_to_half(vmin);
}

/*
 * tqo_store — write N*H token-heads into the paged cache.
 *   y        [N*H, D] fp32 rotated unit keys (x_hat @ PiT, computed by caller)
 *   norms    [N*H]    fp32 key norms
 *   value    [N*H, D] fp32 values
 *   slot_mapping [N]  int32 (negative = skip, reference/soa_store.py:275-277)
 *   block_bytes       bytes per physical block (= 16*H*134 for SoA)
 *   aos_stride_pos / aos_stride_head: AoS byte strides (ignored for SoA)
 * Returns 0.
 */
int tqo_store(int layout, const float* y, const float* norms, const float* value,
              int N, int H, int D, const float* mids, const float* cents,
              int bits, const int32_t* slot_mapping, uint8_t* cache,
              int64_t block_bytes, int64_t aos_stride_pos, int64_t aos_stride_head,
              int block_size, int norm_correction) {
    const int n_c = 1 << bits;
    const int kbytes = D * bits / 8, vbytes = D / 2;
    const int64_t data_per_slot = kbytes + vbytes;
    const int64_t meta_off = (int64_t)block_size * H * data_per_slot;
    float* tmp = (float*)malloc(sizeof(float) * (size_t)D);
    for (int64_t pid = 0; pid < (int64_t)N * H; pid++) {
        int tok = (int)(pid / H), h = (int)(pid % H);
        int32_t slot = slot_mapping[tok];
        if (slot < 0) continue;
        int64_t blk = slot / block_size, off = slot % block_size;
        const float* yv = y + pid * D;
        int idx[512];
        for (int d = 0; d < D; d++) idx[d] = bucketize(yv[d], mids, n_c, bits);
        uint8_t kpacked[256];
        for (int j = 0; j < D / 2; j++)
            kpacked[j] = (uint8_t)((idx[2 * j] & 0xF) | ((idx[2 * j + 1] & 0xF) << 4));
        float vn = norms[pid];
        if (norm_correction) {
            for (int d = 0; d < D; d++) {
                float c = cents[idx[d]];
                tmp[d] = c * c;
            }
            volatile float nsq = np_sum_f32(tmp, D) + 1e-16f;
            volatile float sq = sqrtf(nsq);
            volatile float inv = 1.0f / sq;
            vn = vn * inv;
        }
        uint16_t vn_h = float_to_half(vn);
        uint8_t vpacked[256];
        uint16_t sc_h, zr_h;
        quantise_value(value + pid * D, D, vpacked, &sc_h, &zr_h);
        uint8_t* blockp = cache + blk * block_bytes;
        if (layout == TQO_LAYOUT_SOA) {
            /* data region [token][head][K|V]; meta [head][field][token] fp16
             * (reference/soa_store.py:286-300) */
            uint8_t* dp = blockp + off * H * data_per_slot + (int64_t)h * data_per_slot;
            memcpy(dp, kpacked, (size_t)kbytes);
            memcpy(dp + kbytes, vpacked, (size_t)vbytes);
            uint16_t* meta = (uint16_t*)(blockp + meta_off) + (int64_t)h * 3 * block_size;
            meta[0 * block_size + off] = vn_h;
            meta[1 * block_size + off] = sc_h;
            meta[2 * block_size + off] = zr_h;
        } else {
            /* AoS slot [K | knorm fp16 | V | scale fp16 | zero fp16]
             * (reference/aos_store.py:296-340); the stored norm is the raw
             * key norm (no folding). */
            uint8_t* sp = blockp + off * aos_stride_pos + (int64_t)h * aos_stride_head;
            memcpy(sp, kpacked, (size_t)kbytes);
            uint16_t raw = float_to_half(norms[pid]);
            memcpy(sp + kbytes, &raw, 2);
            memcpy(sp + kbytes + 2, vpacked, (size_t)vbytes);
            memcpy(sp + kbytes + 2 + vbytes, &sc_h, 2);
            memcpy(sp + kbytes + 2 + vbytes + 2, &zr_h, 2);
        }
    }
    free(tmp);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Stage1 (split-KV partial attention)                                       */
/* reference/soa_decode_v1.py:43-314 (SoA), reference/aos_decode.py:43-313   */
/* ------------------------------------------------------------------------ */

#define BLOCK_KV 4

typedef struct {
    int layout;
    const uint8_t* cache;
    int64_t block_bytes, aos_stride_pos, aos_stride_head;
    int Hk, D, block_size;
} cache_desc;

/* Decode one token-head: K centroid values (not yet scaled by the norm),
 * the K norm, and V = idx*scale + zero. */
static void decode_token(const cache_desc* c, const float* cents, int64_t blk,
                         int off, int kvh, float* kc, float* knorm,
                         float* vv) {
    const int D = c->D, kbytes = D / 2, vbytes = D / 2;
    const uint8_t* bp = c->cache + blk * c->block_bytes;
    const uint8_t *kp, *vp;
    uint16_t kn_h, sc_h, zr_h;
    if (c->layout == TQO_LAYOUT_SOA) {
        const int64_t dps = kbytes + vbytes;
        kp = bp + (int64_t)off * c->Hk * dps + (int64_t)kvh * dps;
        vp = kp + kbytes;
        const uint16_t* meta = (const uint16_t*)(bp + (int64_t)c->block_size * c->Hk * dps)
                               + (int64_t)kvh * 3 * c->block_size;
        kn_h = meta[off];
        sc_h = meta[c->block_size + off];
        zr_h = meta[2 * c->block_size + off];
    } else {
        kp = bp + (int64_t)off * c->aos_stride_pos + (int64_t)kvh * c->aos_stride_head;
        memcpy(&kn_h, kp + kbytes, 2);
        vp = kp + kbytes + 2;
        memcpy(&sc_h, vp + vbytes, 2);
        memcpy(&zr_h, vp + vbytes + 2, 2);
    }
    for (int j = 0; j < kbytes; j++) {
        kc[2 * j] = cents[kp[j] & 0xF];
        kc[2 * j + 1] = cents[(kp[j] >> 4) & 0xF];
    }
    if (c->layout == TQO_LAYOUT_AOS) {
        /* NORM_CORRECTION in the decoder: c / sqrt(sum c^2 + 1e-16)
         * (reference/aos_decode.py:199-206) */
        float sq[512];
        for (int d = 0; d < D; d++) sq[d] = kc[d] * kc[d];
        volatile float nsq = np_sum_f32(sq, D) + 1e-16f;
        volatile float s = sqrtf(nsq);
        volatile float inv = 1.0f / s;
        for (int d = 0; d < D; d++) kc[d] = kc[d] * inv;
    }
    *knorm = half_to_float(kn_h);
    float sc = half_to_float(sc_h), zr = half_to_float(zr_h);
    for (int j = 0; j < vbytes; j++) {
        vv[2 * j] = (float)(vp[j] & 0xF) * sc + zr;
        vv[2 * j + 1] = (float)((vp[j] >> 4) & 0xF) * sc + zr;
    }
}

/*
 * tqo_stage1 — mid_o[b, h, s, 0:D] = normalised partial O of split s,
 * mid_o[b, h, s, D] = natural-log LSE.  Empty splits are not written
 * (reference/soa_decode_v1.py:109-110).
 *   num_splits_per_seq: optional [B] array; split count of sequence b (the
 *   uniform count S otherwise).  S is also the mid_o split extent.
 */
int tqo_stage1(int layout, const float* q_rot, int64_t sqb, int64_t sqh,
               const uint8_t* cache, int64_t block_bytes, int64_t aos_stride_pos,
               int64_t aos_stride_head, const int32_t* block_table, int64_t bt_stride,
               const int32_t* seq_lens, const int32_t* num_splits_per_seq,
               const float* cents, float* mid_o, int64_t smb, int64_t smh,
               int64_t sms, int B, int Hq, int Hk, int D, int block_size, int S,
               float attn_scale, int nthreads) {
    if (D > 512 || D % 2) return -1;
    cache_desc c = {layout, cache, block_bytes, aos_stride_pos, aos_stride_head,
                    Hk, D, block_size};
    const int G = Hq / Hk;
    const int64_t n_items = (int64_t)B * Hq * S;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 4)
#endif
    for (int64_t it = 0; it < n_items; it++) {
        const int s = (int)(it % S);
        const int h = (int)((it / S) % Hq);
        const int b = (int)(it / ((int64_t)S * Hq));
        const int nsp = num_splits_per_seq ? num_splits_per_seq[b] : S;
        if (s >= nsp) continue;
        const int seq_len = seq_lens[b];
        /* split rule, reference/soa_decode_v1.py:104-110 */
        const int split_len = (seq_len + nsp - 1) / nsp;
        const int start = split_len * s;
        const int end = start + split_len < seq_len ? start + split_len : seq_len;
        if (start >= end) continue;
        const int kvh = h / G;
        const float* q = q_rot + (int64_t)b * sqb + (int64_t)h * sqh;
        float m = -INFINITY, l = 0.0f;
        float acc[512], kc[BLOCK_KV][512], vv[BLOCK_KV][512], prod[512];
        for (int d = 0; d < D; d++) acc[d] = 0.0f;
        for (int n0 = start; n0 < end; n0 += BLOCK_KV) {
            float score[BLOCK_KV];
            int valid[BLOCK_KV];
            for (int i = 0; i < BLOCK_KV; i++) {
                const int t = n0 + i;
                valid[i] = t < end;
                if (!valid[i]) { score[i] = -INFINITY; continue; }
                const int64_t blk = block_table[(int64_t)b * bt_stride + t / block_size];
                float knorm;
                decode_token(&c, cents, blk, t % block_size, kvh, kc[i], &knorm, vv[i]);
                /* term1 = sum(q * c) (reference/soa_decode_v1.py:241-244) */
                for (int d = 0; d < D; d++) prod[d] = q[d] * kc[i][d];
                float term1 = np_sum_f32(prod, D);
                /* scores = norm * term1 * ATTN_SCALE (:253) */
                volatile float t1 = knorm * term1;
                score[i] = t1 * attn_scale;
            }
            /* online softmax update (:259-307) */
            float tmax = score[0];
            for (int i = 1; i < BLOCK_KV; i++) tmax = score[i] > tmax ? score[i] : tmax;
            const float n_e_max = tmax > m ? tmax : m;
            const float re_scale = expf(m - n_e_max);
            float p[BLOCK_KV];
            for (int i = 0; i < BLOCK_KV; i++) p[i] = expf(score[i] - n_e_max);
            for (int d = 0; d < D; d++) {
                float sum = 0.0f;
                int first = 1;
                for (int i = 0; i < BLOCK_KV; i++) {
                    volatile float term = valid[i] ? p[i] * vv[i][d] : 0.0f * p[i];
                    if (first) { sum = term; first = 0; } else sum = sum + term;
                }
                volatile float scaled = acc[d] * re_scale;
                acc[d] = scaled + sum;
            }
            float psum = 0.0f;
            for (int i = 0; i < BLOCK_KV; i++) psum = psum + p[i];
            volatile float ls = l * re_scale;
            l = ls + psum;
            m = n_e_max;
        }
        /* epilogue (:310-314) */
        const float safe_l = l > 0.0f ? l : 1.0f;
        float* o = mid_o + (int64_t)b * smb + (int64_t)h * smh + (int64_t)s * sms;
        for (int d = 0; d < D; d++) o[d] = acc[d] / safe_l;
        o[D] = m + logf(safe_l);
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Stage2: LSE merge over the non-empty splits (baseline/stage2.py:8-55)     */
/* ------------------------------------------------------------------------ */

int tqo_stage2(const float* mid_o, int64_t smb, int64_t smh, int64_t sms,
               const int32_t* seq_lens, const int32_t* num_splits_per_seq,
               float* out, int64_t sob, int64_t soh, float* lse, int64_t slb,
               int B, int Hq, int S, int D, int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
    for (int64_t it = 0; it < (int64_t)B * Hq; it++) {
        const int b = (int)(it / Hq), h = (int)(it % Hq);
        const int nsp = num_splits_per_seq ? num_splits_per_seq[b] : S;
        const int seq_len = seq_lens[b];
        float acc[512];
        for (int d = 0; d < D; d++) acc[d] = 0.0f;
        float rmax = -INFINITY, rsum = 0.0f;
        for (int s = 0; s < nsp; s++) {
            const int split_len = (seq_len + nsp - 1) / nsp;
            const int start = split_len * s;
            const int end = start + split_len < seq_len ? start + split_len : seq_len;
            if (end <= start) continue;
            const float* v = mid_o + (int64_t)b * smb + (int64_t)h * smh + (int64_t)s * sms;
            const float slse = v[D];
            const float nmax = rmax > slse ? rmax : slse;
            const float old_scale = expf(rmax - nmax);
            const float w = expf(slse - nmax);
            for (int d = 0; d < D; d++) {
                volatile float a = acc[d] * old_scale;
                volatile float bb = w * v[d];
                acc[d] = a + bb;
            }
            volatile float rs = rsum * old_scale;
            rsum = rs + w;
            rmax = nmax;
        }
        float* o = out + (int64_t)b * sob + (int64_t)h * soh;
        for (int d = 0; d < D; d++) o[d] = acc[d] / rsum;
        lse[(int64_t)b * slb + h] = rmax + logf(rsum);
    }
    return 0;
}
