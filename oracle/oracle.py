"""CPU oracle for the TurboQuant ``turboquant_4bit_nc`` decode path.

TEST INFRASTRUCTURE ONLY: this module is the checker the CUDA path is compared
against, and the timed CPU baseline of ``bench.py``.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs import it; the product
package never does.

Two independent restatements live here:

* ``store``/``stage1``/``stage2`` call ``libtqoracle.so`` (``tq_oracle.c``), an
  fp32 restatement in the reference's own operation order.  Its parity is
  pinned against the reference's Triton kernels run under
  ``TRITON_INTERPRET=1`` (``tests/golden/*.npz``).
* ``stage1_np``/``stage2_np`` are vectorised float64 numpy restatements of the
  same algorithm, used to cross-check the C code and for large configs.

Reference citations are paths inside zben777/turboquant-cuda-decode.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libtqoracle.so"

LAYOUT_SOA = 0
LAYOUT_AOS = 1
LAYOUT_SOA_K8 = 2  # turboquant_k8v4: [16][Hk][K128 e4m3 | V64] + [Hk][2][16] fp16 meta
LAYOUT_SOA_K3 = 3  # turboquant_k3v4_nc: [16][Hk][K48 3-bit | V64] + [Hk][3][16] fp16 meta
LAYOUT_SOA_K3V3 = 4  # turboquant_3bit_nc: [16][Hk][K48 3-bit | V48 3-bit] + [Hk][3][16] fp16 meta
# AoS forms of the presets: one slot per (token, KV head), [key codes | fp16
# raw norm (Lloyd-Max keys only) | value codes | fp16 vscale | fp16 vzero]
LAYOUT_AOS_K8 = 5    # [K128 e4m3 | V64 | sc | zr] = 196 bytes
LAYOUT_AOS_K3 = 6    # [K48 | norm | V64 | sc | zr] = 118 bytes
LAYOUT_AOS_K3V3 = 7  # [K48 | norm | V48 | sc | zr] = 102 bytes
AOS_PRESETS = (LAYOUT_AOS_K8, LAYOUT_AOS_K3, LAYOUT_AOS_K3V3)
HEAD_DIM = 128
BLOCK_SIZE = 16
SLOT_BYTES = 134  # 64 K + 64 V + 3 fp16 metadata

_lib = None


def build(force: bool = False) -> Path:
    """Compile ``libtqoracle.so`` with ``oracle/Makefile``."""
    if force or not LIB_PATH.exists() or (
        LIB_PATH.stat().st_mtime < (HERE / "tq_oracle.c").stat().st_mtime
    ):
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        i64, i32, vp, f32 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_float
        _lib.tqo_store.argtypes = [i32, vp, vp, vp, i32, i32, i32, vp, vp, i32, vp, vp,
                                   i64, i64, i64, i32, i32]
        _lib.tqo_stage1.argtypes = [i32, vp, i64, i64, vp, i64, i64, i64, vp, i64, vp, vp,
                                    vp, vp, i64, i64, i64, i32, i32, i32, i32, i32, i32,
                                    f32, i32]
        _lib.tqo_stage2.argtypes = [vp, i64, i64, i64, vp, vp, vp, i64, i64, vp, i64,
                                    i32, i32, i32, i32, i32]
        for f in (_lib.tqo_store, _lib.tqo_stage1, _lib.tqo_stage2):
            f.restype = ctypes.c_int
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---------------------------------------------------------------------------
# Layout helpers (baseline/common.py:79-224; reference/soa_decode_v1.py:168-188)
# ---------------------------------------------------------------------------


def block_bytes(hk: int, block_size: int = BLOCK_SIZE) -> int:
    """Bytes per physical block: [block_size, Hk, 134] uint8."""
    return block_size * hk * SLOT_BYTES


def soa_meta_offset(hk: int, block_size: int = BLOCK_SIZE, d: int = HEAD_DIM) -> int:
    """Byte offset of the SoA metadata region inside a block."""
    return block_size * hk * d


def split_range(seq_len: int, num_splits: int, s: int) -> tuple[int, int]:
    """Reference split rule (reference/soa_decode_v1.py:104-107)."""
    split_len = -(-seq_len // num_splits)
    start = split_len * s
    return start, min(start + split_len, seq_len)


# ---------------------------------------------------------------------------
# C restatement
# ---------------------------------------------------------------------------


def store(layout, y, norms, value, midpoints, centroids, slot_mapping, cache,
          norm_correction=True, bits=4):
    """In-place store of N*H token-heads (reference/soa_store.py:223-373,
    reference/aos_store.py:221-340).  ``y``/``norms``/``value`` are the kernel
    inputs ``[N*H, D]``, ``[N*H]``, ``[N*H, D]`` fp32; ``cache`` is the
    ``[num_blocks, 16, H, 134]`` uint8 array, modified in place."""
    assert cache.dtype == np.uint8 and cache.flags.c_contiguous
    N = slot_mapping.shape[0]
    H = cache.shape[2]
    D = y.shape[-1]
    y, norms, value = _c(y, np.float32), _c(norms, np.float32), _c(value, np.float32)
    mids, cents = _c(midpoints, np.float32), _c(centroids, np.float32)
    slots = _c(slot_mapping, np.int32)
    st = [s * cache.itemsize for s in cache.strides]
    rc = lib().tqo_store(layout, _ptr(y), _ptr(norms), _ptr(value), N, H, D, _ptr(mids),
                         _ptr(cents), bits, _ptr(slots), _ptr(cache), st[0], st[1], st[2],
                         cache.shape[1], int(norm_correction))
    assert rc == 0


def stage1(q_rot, cache, block_table, seq_lens, centroids, num_splits, *,
           layout=LAYOUT_SOA, num_splits_per_seq=None, mid_o=None, attn_scale=None,
           nthreads=0):
    """fp32 Stage1 in the reference's order.  Returns ``mid_o [B,Hq,S,D+1]``;
    entries of empty splits keep their initial value (NaN when allocated
    here), as the reference leaves them unwritten."""
    q = _c(q_rot, np.float32)
    B, Hq, D = q.shape
    cache = np.ascontiguousarray(cache)
    Hk = cache.shape[2]
    bt = _c(block_table, np.int32)
    sl = _c(seq_lens, np.int32)
    cents = _c(centroids, np.float32)
    nsp = None if num_splits_per_seq is None else _c(num_splits_per_seq, np.int32)
    if mid_o is None:
        mid_o = np.full((B, Hq, num_splits, D + 1), np.nan, dtype=np.float32)
    assert mid_o.dtype == np.float32 and mid_o.flags.c_contiguous
    scale = np.float32(1.0 / np.sqrt(D)) if attn_scale is None else np.float32(attn_scale)
    rc = lib().tqo_stage1(layout, _ptr(q), q.strides[0] // 4, q.strides[1] // 4, _ptr(cache),
                          cache.strides[0], cache.strides[1], cache.strides[2], _ptr(bt),
                          bt.strides[0] // 4, _ptr(sl), _ptr(nsp), _ptr(cents), _ptr(mid_o),
                          mid_o.strides[0] // 4, mid_o.strides[1] // 4, mid_o.strides[2] // 4,
                          B, Hq, Hk, D, cache.shape[1], num_splits, float(scale), nthreads)
    assert rc == 0
    return mid_o


def stage2(mid_o, seq_lens, num_splits_per_seq=None, nthreads=0):
    """LSE merge over non-empty splits (baseline/stage2.py:8-55).
    Returns ``(output [B,Hq,D], lse [B,Hq])``."""
    mid = _c(mid_o, np.float32)
    B, Hq, S, D1 = mid.shape
    D = D1 - 1
    sl = _c(seq_lens, np.int32)
    nsp = None if num_splits_per_seq is None else _c(num_splits_per_seq, np.int32)
    out = np.empty((B, Hq, D), np.float32)
    lse = np.empty((B, Hq), np.float32)
    rc = lib().tqo_stage2(_ptr(mid), mid.strides[0] // 4, mid.strides[1] // 4,
                          mid.strides[2] // 4, _ptr(sl), _ptr(nsp), _ptr(out),
                          out.strides[0] // 4, out.strides[1] // 4, _ptr(lse),
                          lse.strides[0] // 4, B, Hq, S, D, nthreads)
    assert rc == 0
    return out, lse


# ---------------------------------------------------------------------------
# Independent float64 numpy restatement
# ---------------------------------------------------------------------------


def _e4m3_values() -> np.ndarray:
    """Value of every e4m3 (OCP "fn" variant) byte: 1 sign, 4 exponent bits
    (bias 7), 3 mantissa bits; exponent 0 is subnormal (m / 8 * 2^-6);
    0x7F / 0xFF are NaN, no infinities."""
    b = np.arange(256)
    e, m = (b >> 3) & 0xF, b & 7
    mag = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * 2.0 ** (e - 7.0))
    v = np.where(b & 0x80, -mag, mag)
    v[(b & 0x7F) == 0x7F] = np.nan
    return v


E4M3 = _e4m3_values()


def e4m3_encode(x) -> np.ndarray:
    """float -> e4m3 byte, round to nearest, ties to the even code, finite
    values beyond 448 saturated to +-448 (the "rn.satfinite" conversion the
    compiled reference store issues, reference/soa_store.py:192-193)."""
    x = np.asarray(x, np.float64)
    mags = E4M3[:0x7F]                  # codes 0..126, increasing
    a = np.minimum(np.abs(x), 448.0)
    hi = np.clip(np.searchsorted(mags, a, side="left"), 1, 126)
    lo = hi - 1
    dlo, dhi = a - mags[lo], mags[hi] - a
    pick_hi = (dhi < dlo) | ((dhi == dlo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo)
    code = np.where(a == 0.0, 0, code)
    sign = np.signbit(x).astype(np.int64)  # values rounding to zero keep their sign
    out = (code | (sign << 7)).astype(np.uint8)
    return np.where(np.isnan(x), np.uint8(0x7F), out).astype(np.uint8)


def _quantise_value_np(v, bits=4):
    """Value quantiser of the reference store in fp32 (4-bit:
    reference/soa_store.py:85-116; 3-bit: :49-60): returns codes and the
    fp16 scale/zero."""
    v = np.asarray(v, np.float32)
    top = (1 << bits) - 1
    vmin, vmax = v.min(-1, keepdims=True), v.max(-1, keepdims=True)
    scale = (vmax - vmin) / np.float32(top)
    scale = np.where(scale > np.float32(1e-8), scale, np.float32(1e-8)).astype(np.float32)
    t = ((v - vmin) / scale + np.float32(0.5)).astype(np.float32)
    q = np.clip(np.trunc(t), 0, top).astype(np.uint8)
    return q, scale[..., 0].astype(np.float16), vmin[..., 0].astype(np.float16)


def store_k8_np(key, value, slot_mapping, cache):
    """FP8-key store (turboquant_k8v4, reference/soa_store.py:125-221) into
    ``cache [nb, 16, H, 196]`` in place: e4m3 key bytes, 4-bit values
    (low nibble = even dim), fp16 vscale/vzero in the meta region."""
    nb, bs, H, slot = cache.shape
    flat = cache.reshape(nb, bs * H * slot)
    D = HEAD_DIM
    dps = D + D // 2
    key = np.asarray(key, np.float32).reshape(-1, H, D)
    value = np.asarray(value, np.float32).reshape(-1, H, D)
    meta_off = bs * H * dps
    for t, s in enumerate(np.asarray(slot_mapping)):
        if s < 0:
            continue
        blk, off = int(s) // bs, int(s) % bs
        q, sc, zr = _quantise_value_np(value[t])
        for h in range(H):
            base = off * H * dps + h * dps
            flat[blk, base : base + D] = e4m3_encode(key[t, h])
            flat[blk, base + D : base + dps] = q[h, 0::2] | (q[h, 1::2] << 4)
            m = meta_off + h * 2 * bs * 2
            flat[blk, m + 2 * off : m + 2 * off + 2] = np.frombuffer(sc[h].tobytes(), np.uint8)
            flat[blk, m + 2 * bs + 2 * off : m + 2 * bs + 2 * off + 2] = np.frombuffer(zr[h].tobytes(), np.uint8)


def _pack3(codes) -> np.ndarray:
    """128 3-bit codes -> 48 bytes, code d at bits 3d..3d+2 (little-endian)."""
    stream = 0
    for d, x in enumerate(np.asarray(codes)):
        stream |= int(x) << (3 * d)
    return np.frombuffer(stream.to_bytes(len(codes) * 3 // 8, "little"), np.uint8)


def store_k3_np(y, norms, value, midpoints, centroids, slot_mapping, cache, vbits=4):
    """3-bit-key store (turboquant_k3v4_nc; reference/soa_store.py:223-373
    with MSE_BITS = 3) into ``cache [nb, 16, H, 118]`` in place, from the
    kernel inputs (rotated unit keys ``y [N*H, D]``, key norms, values):
    3-step binary search over the 7 midpoints with ``y >= mid`` going right,
    codes packed little-endian at bit 3d, stored norm = fp16(|k| /
    sqrt(sum c^2 + 1e-16)) in fp32 (the sum in numpy's float32 order, as the
    interpreted reference computes it), values as the 4-bit store, or with
    ``vbits=3`` (turboquant_3bit_nc) 7 levels packed like the keys."""
    nb, bs, H, slot = cache.shape
    flat = cache.reshape(nb, bs * H * slot)
    D = HEAD_DIM
    kbytes, dps = D * 3 // 8, D * 3 // 8 + D * vbits // 8
    mids = np.asarray(midpoints, np.float32)
    c = np.asarray(centroids, np.float32)
    y = np.asarray(y, np.float32).reshape(-1, H, D)
    norms = np.asarray(norms, np.float32).reshape(-1, H)
    value = np.asarray(value, np.float32).reshape(-1, H, D)
    meta_off = bs * H * dps
    for t, s_ in enumerate(np.asarray(slot_mapping)):
        if s_ < 0:
            continue
        blk, off = int(s_) // bs, int(s_) % bs
        q, sc, zr = _quantise_value_np(value[t], vbits)
        for h in range(H):
            lo = np.zeros(D, np.int64)
            hi = np.full(D, 7, np.int64)
            for _ in range(3):
                mid = (lo + hi) >> 1
                right = y[t, h] >= mids[np.minimum(mid, 6)]
                lo = np.where(right, mid + 1, lo)
                hi = np.where(right, hi, mid)
            idx = np.minimum(lo, 7)
            base = off * H * dps + h * dps
            flat[blk, base : base + kbytes] = _pack3(idx)
            flat[blk, base + kbytes : base + dps] = _pack3(q[h]) if vbits == 3 else q[h, 0::2] | (q[h, 1::2] << 4)
            cv = c[idx]
            nsq = np.float32((cv * cv).astype(np.float32).sum(dtype=np.float32)) + np.float32(1e-16)
            vn = np.float32(norms[t, h] * (np.float32(1.0) / np.sqrt(nsq, dtype=np.float32)))
            m = meta_off + h * 3 * bs * 2
            for f, val in enumerate((np.float16(vn), sc[h], zr[h])):
                flat[blk, m + f * 2 * bs + 2 * off : m + f * 2 * bs + 2 * off + 2] = np.frombuffer(
                    np.float16(val).tobytes(), np.uint8)


def _aos_geometry(layout):
    """(key bytes, has norm, value bits) of an AoS preset slot."""
    return {LAYOUT_AOS_K8: (128, False, 4), LAYOUT_AOS_K3: (48, True, 4), LAYOUT_AOS_K3V3: (48, True, 3)}[layout]


def aos_slot_bytes(layout) -> int:
    kb, has_norm, vbits = _aos_geometry(layout)
    return kb + (2 if has_norm else 0) + HEAD_DIM * vbits // 8 + 4


def _bucketize(y, mids, nc, steps):
    """The reference store's binary search over the sorted midpoints,
    ``y >= mid`` going right (reference/aos_store.py:280-295)."""
    lo = np.zeros(y.shape, np.int64)
    hi = np.full(y.shape, nc - 1, np.int64)
    for _ in range(steps):
        mid = (lo + hi) >> 1
        right = y >= mids[np.minimum(mid, nc - 2)]
        lo = np.where(right, mid + 1, lo)
        hi = np.where(right, hi, mid)
    return np.minimum(lo, nc - 1)


def store_aos_np(layout, y, norms, value, midpoints, slot_mapping, cache):
    """AoS store of the FP8-key and 3-bit presets (reference/aos_store.py:
    145-219 FP8, :221-340 MSE with MSE_BITS = 3, values :26-116) into
    ``cache [nb, 16, H, slot]`` in place.  ``y`` is the raw key for
    ``LAYOUT_AOS_K8`` (cast to e4m3, nearest even, saturating) and the
    rotated unit key for the 3-bit forms, whose slot stores the raw norm
    fp16(|k|) (the decoder applies the norm correction)."""
    kb, has_norm, vbits = _aos_geometry(layout)
    D = HEAD_DIM
    nb, bs, H, slot = cache.shape
    y = np.asarray(y, np.float32).reshape(-1, H, D)
    value = np.asarray(value, np.float32).reshape(-1, H, D)
    if has_norm:
        norms = np.asarray(norms, np.float32).reshape(-1, H)
        mids = np.asarray(midpoints, np.float32)
    voff = kb + (2 if has_norm else 0)
    vbytes = D * vbits // 8
    for t, s_ in enumerate(np.asarray(slot_mapping)):
        if s_ < 0:
            continue
        blk, off = int(s_) // bs, int(s_) % bs
        q, sc, zr = _quantise_value_np(value[t], vbits)
        for h in range(H):
            dst = cache[blk, off, h]
            if layout == LAYOUT_AOS_K8:
                dst[:kb] = e4m3_encode(y[t, h])
            else:
                dst[:kb] = _pack3(_bucketize(y[t, h], mids, 8, 3))
                dst[kb:kb + 2] = np.frombuffer(np.float16(norms[t, h]).tobytes(), np.uint8)
            dst[voff:voff + vbytes] = _pack3(q[h]) if vbits == 3 else q[h, 0::2] | (q[h, 1::2] << 4)
            dst[voff + vbytes:voff + vbytes + 2] = np.frombuffer(sc[h].tobytes(), np.uint8)
            dst[voff + vbytes + 2:voff + vbytes + 4] = np.frombuffer(zr[h].tobytes(), np.uint8)


def _unpack3(b, n=HEAD_DIM):
    """Little-endian 3-bit codes of the byte rows ``b [m, 3n/8]``."""
    b = np.asarray(b, np.int64)
    bit = 3 * np.arange(n)
    b0, b1 = b[:, bit // 8], b[:, np.minimum(bit // 8 + 1, b.shape[1] - 1)]
    return ((b0 | (b1 << 8)) >> (bit % 8)) & 7


def decode_kv_np(cache, block_ids, offs, kvh, centroids, layout=LAYOUT_SOA):
    """Dequantise tokens (block_ids[i], offs[i]) of KV head ``kvh``.
    Returns ``K [n, D]`` (centroid*norm, norm correction applied for AoS) and
    ``V [n, D]`` in float64."""
    nb, bs, Hk, slot = cache.shape
    D = HEAD_DIM
    if layout in AOS_PRESETS:
        # reference/aos_decode.py:153-299: e4m3 keys as they are; 3-bit keys
        # c[idx] / |c| * norm (NORM_CORRECTION); values code * scale + zero
        kb, has_norm, vbits = _aos_geometry(layout)
        slots = cache[block_ids, offs, kvh].astype(np.uint8)  # [n, slot]
        voff = kb + (2 if has_norm else 0)
        vbytes = D * vbits // 8
        sc = slots[:, voff + vbytes:voff + vbytes + 2].copy().view(np.float16)[:, 0].astype(np.float64)
        zr = slots[:, voff + vbytes + 2:voff + vbytes + 4].copy().view(np.float16)[:, 0].astype(np.float64)
        vb = slots[:, voff:voff + vbytes]
        vidx = (_unpack3(vb) if vbits == 3 else np.stack([vb & 0xF, vb >> 4], -1).reshape(-1, D)).astype(np.float64)
        V = vidx * sc[:, None] + zr[:, None]
        if layout == LAYOUT_AOS_K8:
            return E4M3[slots[:, :kb]], V
        c = np.asarray(centroids, np.float64)
        kc = c[_unpack3(slots[:, :kb])]
        kc = kc / np.sqrt((kc * kc).sum(-1, keepdims=True) + 1e-16)
        knorm = slots[:, kb:kb + 2].copy().view(np.float16)[:, 0].astype(np.float64)
        return kc * knorm[:, None], V
    flat = cache.reshape(nb, bs * Hk * slot)
    if layout == LAYOUT_SOA_K8:
        dps = D + D // 2  # 128 e4m3 key bytes + 64 V bytes
        base = offs * Hk * dps + kvh * dps
        kb = flat[block_ids[:, None], base[:, None] + np.arange(D)]
        vb = flat[block_ids[:, None], base[:, None] + D + np.arange(D // 2)]
        meta = flat[:, bs * Hk * dps :].copy().view(np.float16).reshape(nb, Hk, 2, bs)
        vsc = meta[block_ids, kvh, 0, offs].astype(np.float64)
        vz = meta[block_ids, kvh, 1, offs].astype(np.float64)
        vidx = np.stack([vb & 0xF, vb >> 4], -1).reshape(-1, D).astype(np.float64)
        return E4M3[kb], vidx * vsc[:, None] + vz[:, None]
    c = np.asarray(centroids, np.float64)
    if layout in (LAYOUT_SOA_K3, LAYOUT_SOA_K3V3):
        v3 = layout == LAYOUT_SOA_K3V3
        kbytes = D * 3 // 8                          # 48 packed key bytes
        dps = kbytes + (D * 3 // 8 if v3 else D // 2)  # + 48 (3-bit) or 64 (4-bit) V bytes
        base = offs * Hk * dps + kvh * dps
        kb = flat[block_ids[:, None], base[:, None] + np.arange(kbytes)].astype(np.int64)
        vb = flat[block_ids[:, None], base[:, None] + kbytes + np.arange(dps - kbytes)].astype(np.int64)
        meta = flat[:, bs * Hk * dps :].copy().view(np.float16).reshape(nb, Hk, 3, bs)
        knorm = meta[block_ids, kvh, 0, offs].astype(np.float64)
        vsc = meta[block_ids, kvh, 1, offs].astype(np.float64)
        vz = meta[block_ids, kvh, 2, offs].astype(np.float64)
        bit = 3 * np.arange(D)
        b0, b1 = kb[:, bit // 8], kb[:, np.minimum(bit // 8 + 1, kbytes - 1)]
        kidx = ((b0 | (b1 << 8)) >> (bit % 8)) & 7
        if v3:
            c0, c1 = vb[:, bit // 8], vb[:, np.minimum(bit // 8 + 1, kbytes - 1)]
            vidx = (((c0 | (c1 << 8)) >> (bit % 8)) & 7).astype(np.float64)
        else:
            vidx = np.stack([vb & 0xF, vb >> 4], -1).reshape(-1, D).astype(np.float64)
        return c[kidx] * knorm[:, None], vidx * vsc[:, None] + vz[:, None]
    if layout == LAYOUT_SOA:
        dps = D  # 64 K + 64 V bytes
        base = offs * Hk * dps + kvh * dps
        kb = flat[block_ids[:, None], base[:, None] + np.arange(D // 2)]
        vb = flat[block_ids[:, None], base[:, None] + D // 2 + np.arange(D // 2)]
        meta = flat[:, soa_meta_offset(Hk, bs, D):].view(np.float16).reshape(nb, Hk, 3, bs)
        knorm = meta[block_ids, kvh, 0, offs].astype(np.float64)
        vsc = meta[block_ids, kvh, 1, offs].astype(np.float64)
        vz = meta[block_ids, kvh, 2, offs].astype(np.float64)
    else:
        slots = cache[block_ids, offs, kvh]  # [n, 134]
        kb = slots[:, : D // 2]
        knorm = slots[:, D // 2 : D // 2 + 2].copy().view(np.float16)[:, 0].astype(np.float64)
        vb = slots[:, D // 2 + 2 : D + 2]
        vsc = slots[:, D + 2 : D + 4].copy().view(np.float16)[:, 0].astype(np.float64)
        vz = slots[:, D + 4 : D + 6].copy().view(np.float16)[:, 0].astype(np.float64)
    kidx = np.stack([kb & 0xF, kb >> 4], -1).reshape(-1, D)
    vidx = np.stack([vb & 0xF, vb >> 4], -1).reshape(-1, D).astype(np.float64)
    kc = c[kidx]
    if layout == LAYOUT_AOS:
        kc = kc / np.sqrt((kc * kc).sum(-1, keepdims=True) + 1e-16)
    K = kc * knorm[:, None]
    V = vidx * vsc[:, None] + vz[:, None]
    return K, V


def stage1_np(q_rot, cache, block_table, seq_lens, centroids, num_splits, *,
              layout=LAYOUT_SOA, num_splits_per_seq=None, attn_scale=None, sinks=None):
    """float64 restatement of Stage1 (two-pass softmax per split).

    ``sinks`` ([Hq] logits): split 0 starts its softmax at m = sinks[h],
    l = 1 with a zero accumulator (reference/soa_decode_v1.py:134-145), i.e.
    one extra token of logit sinks[h] and value 0 in split 0."""
    q = np.asarray(q_rot, np.float64)
    B, Hq, D = q.shape
    Hk = cache.shape[2]
    G = Hq // Hk
    bs = cache.shape[1]
    scale = 1.0 / np.sqrt(D) if attn_scale is None else attn_scale
    mid = np.full((B, Hq, num_splits, D + 1), np.nan, np.float64)
    for b in range(B):
        nsp = num_splits if num_splits_per_seq is None else int(num_splits_per_seq[b])
        L = int(seq_lens[b])
        for kvh in range(Hk):
            for s in range(nsp):
                t0, t1 = split_range(L, nsp, s)
                if t0 >= t1:
                    continue
                toks = np.arange(t0, t1)
                blk = np.asarray(block_table[b])[toks // bs].astype(np.int64)
                K, V = decode_kv_np(cache, blk, toks % bs, kvh, centroids, layout)
                qs = q[b, kvh * G : (kvh + 1) * G]  # [G, D]
                sc = qs @ K.T * scale  # [G, n]
                m = sc.max(-1, keepdims=True)
                sk = None
                if sinks is not None and s == 0:
                    sk = np.asarray(sinks, np.float64)[kvh * G : (kvh + 1) * G, None]
                    m = np.maximum(m, sk)
                p = np.exp(sc - m)
                l = p.sum(-1, keepdims=True)
                if sk is not None:
                    l = l + np.exp(sk - m)
                mid[b, kvh * G : (kvh + 1) * G, s, :D] = (p @ V) / l
                mid[b, kvh * G : (kvh + 1) * G, s, D] = (m + np.log(l))[:, 0]
    return mid


def stage2_np(mid_o, seq_lens, num_splits_per_seq=None):
    mid = np.asarray(mid_o, np.float64)
    B, Hq, S, D1 = mid.shape
    out = np.empty((B, Hq, D1 - 1))
    lse = np.empty((B, Hq))
    for b in range(B):
        nsp = S if num_splits_per_seq is None else int(num_splits_per_seq[b])
        keep = [s for s in range(nsp) if split_range(int(seq_lens[b]), nsp, s)[0]
                < split_range(int(seq_lens[b]), nsp, s)[1]]
        if not keep:
            out[b] = np.nan
            lse[b] = -np.inf
            continue
        ls = mid[b][:, keep, D1 - 1]  # [Hq, k]
        m = ls.max(-1, keepdims=True)
        w = np.exp(ls - m)
        out[b] = (w[..., None] * mid[b][:, keep, : D1 - 1]).sum(1) / w.sum(-1, keepdims=True)
        lse[b] = (m + np.log(w.sum(-1, keepdims=True)))[:, 0]
    return out, lse


def merge_np(partials):
    """Merge G per-range partials ``[G, B, Hq, D+1]`` (O, natural-log LSE in
    the last slot) into (O [B, Hq, D], LSE [B, Hq]) in float64.  The split
    merge's running log-sum-exp algebra (reference baseline/stage2.py:37-52)
    applied across KV ranges; a part with LSE = -inf (an empty range) is
    skipped, and a row with no part left gives NaN / -inf."""
    p = np.asarray(partials, np.float64)
    G, B, Hq, D1 = p.shape
    lse = p[..., D1 - 1]                       # [G, B, Hq]
    keep = np.isfinite(lse) | (lse > 0)
    m = np.where(keep, lse, -np.inf).max(0)    # [B, Hq]
    with np.errstate(invalid="ignore", divide="ignore"):
        w = np.where(keep, np.exp(lse - m[None]), 0.0)
        num = (w[..., None] * np.where(keep[..., None], p[..., : D1 - 1], 0.0)).sum(0)
        den = w.sum(0)
        out = num / den[..., None]
        return out, m + np.log(den)


def default_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
