"""The CPU oracle against the reference's own outputs (CPU only).

The golden vectors were produced by the reference Triton kernels run under
TRITON_INTERPRET=1 (tests/golden/make_golden.py).  These tests pin the two
oracle restatements (fp32 C, float64 numpy) before either is trusted as the
checker of the CUDA path.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN_CASES, assert_close
from oracle import oracle as O

# The fp32 restatement follows the reference operation order; what remains
# is exp/log rounding and numpy-vs-C summation of 4-token tiles.
ORACLE_ATOL = 2e-6


def _written(mid):
    return ~np.isnan(mid[..., 0])


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_stage1_soa_matches_reference(golden, name):
    z = golden[name]
    S = int(z["num_splits"])
    got = O.stage1(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], S)
    ref = z["mid_o_soa_v1"]
    # Same splits written (empty splits stay untouched in both).
    assert np.array_equal(_written(got), _written(ref))
    w = _written(ref)
    assert np.abs(got - ref)[w].max() <= ORACLE_ATOL


@pytest.mark.parametrize("name", [n for n in GOLDEN_CASES if n != "ragged_gqa8_hk2"])
def test_stage1_aos_matches_reference(golden, name):
    z = golden[name]
    S = int(z["num_splits"])
    got = O.stage1(z["q_rot"], z["kv_cache_aos"], z["block_table"], z["seq_lens"], z["centroids"], S,
                   layout=O.LAYOUT_AOS)
    ref = z["mid_o_aos_v1"]
    w = _written(ref)
    assert np.array_equal(_written(got), w)
    assert np.abs(got - ref)[w].max() <= ORACLE_ATOL


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_numpy_restatement_matches_reference(golden, name):
    z = golden[name]
    S = int(z["num_splits"])
    got = O.stage1_np(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], S)
    ref = z["mid_o_soa_v1"]
    w = _written(ref)
    assert np.array_equal(~np.isnan(got[..., 0]), w)
    assert np.abs(got - ref)[w].max() <= ORACLE_ATOL


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_stage2_matches_reference(golden, name):
    z = golden[name]
    out, lse = O.stage2(z["mid_o_soa_v1"], z["seq_lens"])
    assert_close(out, z["out_stage2"], atol=1e-6, rtol=0, what="stage2 out")
    assert_close(lse, z["lse_stage2"], atol=1e-6, rtol=0, what="stage2 lse")
    o2, l2 = O.stage2_np(z["mid_o_soa_v1"], z["seq_lens"])
    assert_close(o2, z["out_stage2"], atol=1e-6, rtol=0, what="stage2_np out")


def test_numpy_sinks_match_reference(golden_sinks):
    """Attention sinks: the float64 restatement with sinks against the
    reference Stage1 run with USE_SINKS=1 (a -inf sink, a dominating sink,
    ragged lengths with empty splits), and Stage2 on it."""
    z = golden_sinks
    S = int(z["num_splits"])
    got = O.stage1_np(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], S,
                      sinks=z["sinks"])
    ref = z["mid_o_soa_v1_sinks"]
    w = _written(ref)
    assert np.array_equal(~np.isnan(got[..., 0]), w)
    assert np.abs(got - ref)[w].max() <= ORACLE_ATOL
    # only split 0 moves; the -inf sink leaves its head's rows unchanged
    plain = z["mid_o_soa_v1"]
    assert np.array_equal(np.nan_to_num(plain[:, :, 1:]), np.nan_to_num(ref[:, :, 1:]))
    assert np.array_equal(plain[:, 0, 0], ref[:, 0, 0])
    o2, l2 = O.stage2_np(ref, z["seq_lens"])
    assert_close(o2, z["out_stage2_sinks"], atol=1e-6, rtol=0, what="stage2_np out (sinks)")
    assert_close(l2, z["lse_stage2_sinks"], atol=1e-6, rtol=0, what="stage2_np lse (sinks)")


def test_store_bit_exact(golden_store):
    z = golden_store
    for layout, key, nc in ((O.LAYOUT_SOA, "kv_cache_soa", True), (O.LAYOUT_AOS, "kv_cache_aos", False)):
        cache = z["cache_before"].copy()
        O.store(layout, z["y"], z["norms"], z["value"].reshape(-1, 128), z["midpoints"],
                z["centroids"], z["slot_mapping"], cache, norm_correction=nc)
        assert np.array_equal(cache, z[key]), f"{key}: {(cache != z[key]).sum()} bytes differ"


def test_golden_cache_is_store_output(golden):
    """The fixture caches were written by the reference store: every stored
    metadata value is finite and norms/scales positive (the store's
    self-check, validation/store_decode.py:70-86), on in-range tokens."""
    z = golden["c0"]
    kv = z["kv_cache"]
    nb, bs, hk, _ = kv.shape
    meta = kv.reshape(nb, -1)[:, bs * hk * 128:].copy().view(np.float16).reshape(nb, hk, 3, bs)
    assert np.isfinite(meta).all()
    assert (meta[:, :, 0] > 0).all() and (meta[:, :, 1] > 0).all()


def test_v2_fixed_fails_the_parity_bar(golden):
    """Documents why the kernel splits fp16 operands: the reference's own
    single-fp16-MMA V2 kernel misses the 1e-4 + 2e-3*|ref| bar."""
    z = golden["c0"]
    ref, v2 = z["mid_o_soa_v1"], z["mid_o_v2"]
    w = _written(ref)
    frac = (np.abs(v2 - ref) > 1e-4 + 2e-3 * np.abs(ref))[w].mean()
    assert frac > 0.001


def test_e4m3_encode_matches_torch_cast():
    """The FP8 key cast of the oracle (round to nearest even, saturate to
    +-448) against torch's float8_e4m3fn conversion of the clamped value,
    ties, subnormals, signed zeros and out-of-range values included."""
    import torch
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100000) * 50, rng.standard_normal(50000) * 0.01,
                        [0.0, -0.0, 448, 449, 464, 465, 500, -600, 1e-9, -2e-4, 2.0 ** -10, 3 * 2.0 ** -10,
                         17.0, 19.0, -17.0]]).astype(np.float32)
    ref = torch.from_numpy(np.clip(x, -448, 448)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(O.e4m3_encode(x), ref)


def test_k8v4_store_oracle_against_reference(golden_k8):
    """FP8-key store: value codes and the fp16 scale/zero are bit-identical
    to the reference store's; the key bytes are the e4m3 cast with
    round-to-nearest-even and saturation (the compiled reference's
    conversion on sm_90+).  The fixture's own key bytes came from the Triton
    interpreter, whose FP8 cast rounds ties up, flushes subnormals and wraps
    on overflow, so they are not compared."""
    import torch
    z = golden_k8
    cache = z["cache_before"].copy()
    O.store_k8_np(z["key"], z["value"], z["slot_mapping"], cache)
    nb, bs, hk, slot = cache.shape
    keymask = np.zeros(bs * hk * slot, bool)
    for o in range(bs):
        for h in range(hk):
            keymask[o * hk * 192 + h * 192 : o * hk * 192 + h * 192 + 128] = True
    got, ref = cache.reshape(nb, -1), z["kv_cache"].reshape(nb, -1)
    assert np.array_equal(got[:, ~keymask], ref[:, ~keymask])
    sm = z["slot_mapping"]
    for t in range(len(sm)):
        blk, off = int(sm[t]) // bs, int(sm[t]) % bs
        for h in range(hk):
            k = torch.from_numpy(np.clip(z["key"][t, h], -448, 448)).to(torch.float8_e4m3fn)
            b0 = off * hk * 192 + h * 192
            assert np.array_equal(got[blk, b0 : b0 + 128], k.view(torch.uint8).numpy())


def test_k8v4_stage1_numpy_matches_reference(golden_k8):
    """FP8-key Stage1 restatement against the reference SoA Stage1 run with
    KEY_FP8=1 on the unrotated fp16 query; keys up to 448 make scores large,
    so the bound is relative as well (float64 oracle vs fp32 reference)."""
    z = golden_k8
    mid = O.stage1_np(z["query"], z["kv_cache"], z["block_table"], z["seq_lens"], None, int(z["num_splits"]),
                      layout=O.LAYOUT_SOA_K8)
    ref = z["mid_o"]
    w = _written(ref)
    assert np.array_equal(~np.isnan(mid[..., 0]), w)
    assert (np.abs(mid - ref)[w] <= ORACLE_ATOL + 1e-6 * np.abs(ref)[w]).all()
    o2, l2 = O.stage2_np(ref, z["seq_lens"])
    assert_close(o2, z["out_stage2"], atol=1e-6, rtol=0, what="stage2_np out (k8v4)")


def test_k3v4_oracle_against_reference(golden_k3):
    """3-bit keys (turboquant_k3v4_nc): the oracle store is bit-identical to
    the reference store (3-bit bucketize and little-endian packing, the
    norm-corrected fp16 norm, 4-bit values), the Stage1 restatement matches
    the reference SoA Stage1 with MSE_BITS=3, and the 3-bit codebook equals
    the reference's."""
    import tqb
    z = golden_k3
    assert np.array_equal(tqb.get_centroids(128, 3).numpy(), z["centroids"])
    cache = z["cache_before"].copy()
    O.store_k3_np(z["y"], z["norms"], z["value"], z["midpoints"], z["centroids"], z["slot_mapping"], cache)
    assert np.array_equal(cache, z["kv_cache"]), f"{(cache != z['kv_cache']).sum()} bytes differ"
    mid = O.stage1_np(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"],
                      int(z["num_splits"]), layout=O.LAYOUT_SOA_K3)
    ref = z["mid_o"]
    w = _written(ref)
    assert np.array_equal(~np.isnan(mid[..., 0]), w)
    assert np.abs(mid - ref)[w].max() <= ORACLE_ATOL


def test_k3v3_oracle_against_reference():
    """3-bit keys and values (turboquant_3bit_nc): the oracle store is
    bit-identical to the reference store (values: 7 levels, packed like the
    keys) and the Stage1 restatement matches the reference SoA Stage1 with
    MSE_BITS=3 and VQB=3."""
    from conftest import load_golden
    z = load_golden("k3v3_ragged")
    cache = z["cache_before"].copy()
    O.store_k3_np(z["y"], z["norms"], z["value"], z["midpoints"], z["centroids"], z["slot_mapping"], cache, vbits=3)
    assert np.array_equal(cache, z["kv_cache"]), f"{(cache != z['kv_cache']).sum()} bytes differ"
    mid = O.stage1_np(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"],
                      int(z["num_splits"]), layout=O.LAYOUT_SOA_K3V3)
    ref = z["mid_o"]
    w = _written(ref)
    assert np.array_equal(~np.isnan(mid[..., 0]), w)
    assert np.abs(mid - ref)[w].max() <= ORACLE_ATOL


@pytest.mark.parametrize("name,layout", [("aos_k8v4_ragged", O.LAYOUT_AOS_K8), ("aos_k3v4_ragged", O.LAYOUT_AOS_K3),
                                         ("aos_k3v3_ragged", O.LAYOUT_AOS_K3V3)])
def test_aos_presets_oracle_against_reference(name, layout):
    """AoS forms of the FP8-key and 3-bit presets (reference/aos_store.py,
    reference/aos_decode.py): the oracle's AoS store reproduces the
    reference store's bytes (for FP8 keys: the value codes, scale and zero;
    the key bytes are the hardware e4m3 cast, as for the SoA form, because
    the interpreter's FP8 cast differs), and the Stage1 restatement matches
    the reference AoS V1 Stage1 (KEY_FP8=1, or MSE_BITS=3 with VQB 4 / 3 and
    the in-kernel norm correction)."""
    import torch
    from conftest import load_golden
    z = load_golden(name)
    cache = z["cache_before"].copy()
    if layout == O.LAYOUT_AOS_K8:
        O.store_aos_np(layout, z["key"], None, z["value"], None, z["slot_mapping"], cache)
        got, ref = cache.copy(), z["kv_cache"]
        assert np.array_equal(got[..., 128:], ref[..., 128:]), "value bytes / scale / zero differ"
        sm = z["slot_mapping"]
        for t in range(len(sm)):
            blk, off = int(sm[t]) // 16, int(sm[t]) % 16
            for h in range(cache.shape[2]):
                k = torch.from_numpy(np.clip(z["key"][t, h], -448, 448)).to(torch.float8_e4m3fn)
                assert np.array_equal(got[blk, off, h, :128], k.view(torch.uint8).numpy())
        q = z["query"]
    else:
        O.store_aos_np(layout, z["y"], z["norms"], z["value"], z["midpoints"], z["slot_mapping"], cache)
        assert np.array_equal(cache, z["kv_cache"]), f"{(cache != z['kv_cache']).sum()} bytes differ"
        q = z["q_rot"]
    mid = O.stage1_np(q, z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], int(z["num_splits"]),
                      layout=layout)
    ref = z["mid_o"]
    w = _written(ref)
    assert np.array_equal(~np.isnan(mid[..., 0]), w)
    assert (np.abs(mid - ref)[w] <= ORACLE_ATOL + 1e-6 * np.abs(ref)[w]).all(), np.abs(mid - ref)[w].max()
    o2, l2 = O.stage2_np(ref, z["seq_lens"])
    assert_close(o2, z["out_stage2"], atol=1e-6, rtol=0, what=f"stage2_np out ({name})")
