"""turboquant_k3v4_nc (3-bit keys, 4-bit values) and turboquant_3bit_nc
(3-bit keys and values), both with norm correction, on the GPU.

The cache is the reference's SoA form with 3-bit keys: per token-head 48
packed key bytes (dim d at bits 3d..3d+2, little-endian) and 64 value bytes,
then the fp16 knorm, v-scale and v-zero in the block's meta region; the
3-bit-value preset packs its values the same way (48 bytes).  Bars:
the store bit-exact against the reference store's bytes, Stage1 and Stage2
within 1e-4 + 2e-3 |ref| against the reference's own outputs and the
float64 oracle.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import assert_close, load_golden
from oracle import oracle as O
import tqb
from tqb import compat

pytestmark = pytest.mark.gpu

SENTINEL = -12345.0

# (layout, golden fixture, value bits, bytes per token-head)
PRESETS = [("soa_k3", "k3v4_ragged", 4, 118), ("soa_k3v3", "k3v3_ragged", 3, 102)]
LAYOUT_ID = {"soa_k3": O.LAYOUT_SOA_K3, "soa_k3v3": O.LAYOUT_SOA_K3V3}


@pytest.fixture(autouse=True)
def no_wait_timeouts(cuda_device):
    tqb.wait_timeouts(reset=True)
    yield
    torch.cuda.synchronize()
    assert tqb.wait_timeouts(reset=True) == 0, "a bounded device wait gave up"


def _dev(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _stage1(dev, q_rot, cache, bt, lens, cents, S, layout):
    q = _dev(q_rot, dev)
    mid = torch.full((q.shape[0], q.shape[1], S, 129), SENTINEL, device=dev)
    tqb.stage1(q, _dev(cache, dev), _dev(bt, dev), _dev(lens, dev), _dev(cents, dev), mid, layout=layout)
    torch.cuda.synchronize()
    return mid.cpu().numpy()


def _check(got, ref, what):
    written = ~np.isnan(ref[..., 0])
    assert np.all(got[~written] == SENTINEL), f"{what}: wrote into an empty split"
    assert_close(got[written], ref[written], what=what)


@pytest.mark.parametrize("layout,name,vbits,slot", PRESETS)
def test_store_bit_exact_vs_reference(cuda_device, layout, name, vbits, slot):
    z = load_golden(name)
    dev = cuda_device
    cache = _dev(z["cache_before"], dev)
    tqb.store(_dev(z["y"], dev), _dev(z["norms"], dev), _dev(z["value"], dev), cache, _dev(z["slot_mapping"], dev),
              _dev(z["midpoints"], dev), _dev(z["centroids"], dev), layout=layout, norm_correction=True)
    torch.cuda.synchronize()
    got = cache.cpu().numpy()
    assert np.array_equal(got, z["kv_cache"]), f"{(got != z['kv_cache']).sum()} bytes differ"


@pytest.mark.parametrize("layout,name,vbits,slot", PRESETS)
def test_stage1_and_stage2_vs_reference_golden(cuda_device, layout, name, vbits, slot):
    z = load_golden(name)
    dev = cuda_device
    S = int(z["num_splits"])
    got = _stage1(dev, z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], S, layout)
    _check(got, z["mid_o"], f"{name} Stage1")
    mid = torch.from_numpy(np.where(np.isnan(z["mid_o"]), 0.0, got).astype(np.float32)).to(dev)
    B, Hq = mid.shape[:2]
    out = torch.empty(B, Hq, 128, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    tqb.stage2(mid, _dev(z["seq_lens"], dev), out, lse)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), z["out_stage2"], what=f"{name} Stage2 out")
    assert_close(lse.cpu().numpy(), z["lse_stage2"], what=f"{name} Stage2 lse")


@pytest.mark.parametrize("layout,name,vbits,slot", PRESETS)
@pytest.mark.parametrize("hq,hk", [(32, 8), (16, 2), (8, 1)])
def test_stage1_gqa_vs_oracle(cuda_device, hq, hk, layout, name, vbits, slot):
    """GQA 4 and 8, ragged lengths, a cache written by the oracle store."""
    rng = np.random.default_rng(51 + hq + hk)
    lens = [1, 45, 300, 517]
    B = len(lens)
    pages = [max(1, math.ceil(n / 16)) for n in lens]
    nblk = sum(pages) + 3
    cache = rng.integers(0, 256, size=(nblk, 16, hk, slot), dtype=np.uint8)
    perm = rng.permutation(nblk)
    bt = np.zeros((B, max(pages)), np.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    slots = np.concatenate([bt[b, np.arange(n) // 16] * 16 + np.arange(n) % 16
                            for b, n in enumerate(lens)]).astype(np.int32)
    cents = tqb.get_centroids(128, 3).numpy()
    mids = ((cents[:-1] + cents[1:]) * 0.5).astype(np.float32)
    key = rng.standard_normal((len(slots) * hk, 128)).astype(np.float32)
    norms = np.linalg.norm(key, axis=1).astype(np.float32)
    R = np.linalg.qr(rng.standard_normal((128, 128)))[0].astype(np.float32)
    y = ((key / norms[:, None]) @ R).astype(np.float32)
    val = rng.standard_normal((len(slots) * hk, 128)).astype(np.float32)
    O.store_k3_np(y, norms, val, mids, cents, slots, cache, vbits=vbits)
    q = rng.standard_normal((B, hq, 128)).astype(np.float32)
    S = 5
    ref = O.stage1_np(q, cache, bt, np.asarray(lens, np.int32), cents, S, layout=LAYOUT_ID[layout])
    _check(_stage1(cuda_device, q, cache, bt, np.asarray(lens, np.int32), cents, S, layout), ref,
           f"{name} Stage1 Hq{hq}/Hk{hk}")


@pytest.mark.parametrize("layout,name,vbits,slot", PRESETS)
def test_launchers_store_and_decode(cuda_device, layout, name, vbits, slot):
    """The reference-named launchers with ``mse_bits=3``: store raw keys
    (norm, rotation, 3-bit bucketize), then decode a bf16 query; the decode
    is checked against the oracle on the cache the store wrote."""
    dev = cuda_device
    rng = np.random.default_rng(13)
    lens = [200, 33, 0, 129]
    B, Hq, Hk, S = len(lens), 32, 8, 6
    pages = [max(1, math.ceil(n / 16)) for n in lens]
    nblk = sum(pages) + 2
    cache = _dev(rng.integers(0, 256, size=(nblk, 16, Hk, slot), dtype=np.uint8), dev)
    perm = rng.permutation(nblk)
    bt = np.zeros((B, max(pages)), np.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    slots = np.concatenate([bt[b, np.arange(n) // 16] * 16 + np.arange(n) % 16
                            for b, n in enumerate(lens)]).astype(np.int32)
    cents = tqb.get_centroids(128, 3)
    mids = tqb.get_midpoints(cents)
    Pi = torch.from_numpy(np.linalg.qr(rng.standard_normal((128, 128)))[0].astype(np.float32))
    key = torch.from_numpy(rng.standard_normal((len(slots), Hk, 128)).astype(np.float32))
    val = torch.from_numpy(rng.standard_normal((len(slots), Hk, 128)).astype(np.float32))
    compat.triton_turboquant_store(key.to(dev), val.to(dev), cache, _dev(slots, dev), Pi.T.contiguous().to(dev),
                                   mids.to(dev), 3, 50, vbits, centroids=cents.to(dev), norm_correction=True)
    torch.cuda.synchronize()
    stored = cache.cpu().numpy()
    query = torch.from_numpy(rng.standard_normal((B, Hq, 128)).astype(np.float32)).to(torch.bfloat16)
    q_rot = (query.float() @ Pi.T).numpy()
    mid = O.stage1_np(q_rot, stored, bt, np.asarray(lens, np.int32), cents.numpy(), S, layout=LAYOUT_ID[layout])
    ref_out, ref_lse = O.stage2_np(mid, np.asarray(lens, np.int32))
    lse = torch.empty(B, Hq, device=dev)
    out = compat.triton_turboquant_decode_attention(
        query.to(dev), cache, _dev(bt, dev), _dev(np.asarray(lens, np.int32), dev), Pi.to(dev), cents.to(dev),
        1.0 / math.sqrt(128), 3, 50, vbits, norm_correction=True, max_num_kv_splits=S, lse_buf=lse)
    torch.cuda.synchronize()
    live = np.asarray(lens) > 0
    got = out.float().cpu().numpy()
    ref16 = torch.from_numpy(ref_out[live].astype(np.float32)).to(torch.bfloat16).float().numpy()
    from conftest import RTOL
    assert_close(got[live], ref16, rtol=RTOL + 2.0 ** -7, what=f"{name} decode out")
    assert_close(lse.cpu().numpy()[live], ref_lse[live], what=f"{name} decode lse")
    assert np.all(np.isnan(got[~live]))


def _k3_case(seed, lens, hq, hk, slot, vbits, pool_extra=3):
    rng = np.random.default_rng(seed)
    B = len(lens)
    pages = [max(1, math.ceil(n / 16)) for n in lens]
    nblk = sum(pages) + pool_extra
    cache = rng.integers(0, 256, size=(nblk, 16, hk, slot), dtype=np.uint8)
    perm = rng.permutation(nblk)
    bt = np.zeros((B, max(pages)), np.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    slots = np.concatenate([bt[b, np.arange(n) // 16] * 16 + np.arange(n) % 16
                            for b, n in enumerate(lens)]).astype(np.int32)
    cents = tqb.get_centroids(128, 3).numpy()
    mids = ((cents[:-1] + cents[1:]) * 0.5).astype(np.float32)
    key = rng.standard_normal((len(slots) * hk, 128)).astype(np.float32)
    norms = np.linalg.norm(key, axis=1).astype(np.float32)
    R = np.linalg.qr(rng.standard_normal((128, 128)))[0].astype(np.float32)
    y = ((key / norms[:, None]) @ R).astype(np.float32)
    val = rng.standard_normal((len(slots) * hk, 128)).astype(np.float32)
    O.store_k3_np(y, norms, val, mids, cents, slots, cache, vbits=vbits)
    q = rng.standard_normal((B, hq, 128)).astype(np.float32)
    return q, cache, bt, np.asarray(lens, np.int32), cents


@pytest.mark.parametrize("layout,name,vbits,slot", PRESETS)
@pytest.mark.parametrize("hq,hk", [(32, 8), (8, 2), (4, 1), (12, 4), (16, 8), (20, 4)])
@pytest.mark.parametrize("kernel", ["default", "regs"])
def test_stage1_page_ring_and_register_kernel(cuda_device, hq, hk, kernel, layout, name, vbits, slot, monkeypatch):
    """3-bit keys on both Stage1 kernels: the TMA page ring (GQA <= 4 with Hk
    dividing 8: whole blocks per page, keys decoded through the 6-bit-field
    table, 3-bit values spread to nibbles) and the register-ring kernel
    (TQB_STAGE1_KERNEL=regs, and GQA-5 always).  Ragged lengths with an empty
    sequence and a split of more than 32 pages, against the float64 oracle."""
    if kernel == "regs":
        monkeypatch.setenv("TQB_STAGE1_KERNEL", "regs")
    lens = [1, 0, 1100, 45, 300, 517, 2100]
    q, cache, bt, sl, cents = _k3_case(91 + hq + 5 * hk + vbits, lens, hq, hk, slot, vbits, pool_extra=7)
    S = 6
    ref = O.stage1_np(q, cache, bt, sl, cents, S, layout=LAYOUT_ID[layout])
    _check(_stage1(cuda_device, q, cache, bt, sl, cents, S, layout), ref, f"{name} Stage1 Hq{hq}/Hk{hk} ({kernel})")


@pytest.mark.parametrize("layout,name,vbits,slot", PRESETS)
def test_c1_3bit_decode_vs_oracle(cuda_device, layout, name, vbits, slot):
    """The c1 shape (B64 x 4096, Hq32/Hk8, S32) with 3-bit keys (and
    values), on the page ring: every partial, then Stage2, against the
    float64 oracle on a cache written by the sm_100a store from seeded K/V."""
    dev = cuda_device
    B, L, Hq, Hk, S = 64, 4096, 32, 8, 32
    gen = torch.Generator(device=dev).manual_seed(29 + vbits)
    pages = L // 16
    nblk = B * pages
    bt = torch.randperm(nblk, device=dev, generator=gen).view(B, pages).to(torch.int32)
    kv = torch.zeros(nblk, 16, Hk, slot, dtype=torch.uint8, device=dev)
    cents = tqb.get_centroids(128, 3).to(dev)
    mids = ((cents[:-1] + cents[1:]) * 0.5).contiguous()
    tok = torch.arange(L, device=dev)
    for b in range(B):  # one sequence per store call
        slots = (bt[b, tok // 16] * 16 + tok % 16).to(torch.int32)
        key = torch.randn(L * Hk, 128, device=dev, generator=gen)
        norms = key.norm(dim=1)
        y = (key / norms[:, None]).contiguous()  # unit keys (the rotation does not matter here)
        val = torch.randn(L * Hk, 128, device=dev, generator=gen)
        tqb.store(y, norms, val, kv, slots, mids, cents, layout=layout)
    q = torch.randn(B, Hq, 128, device=dev, generator=gen)
    sl = torch.full((B,), L, dtype=torch.int32, device=dev)
    mid = torch.full((B, Hq, S, 129), SENTINEL, device=dev)
    tqb.stage1(q, kv, bt, sl, cents, mid, layout=layout)
    out = torch.empty(B, Hq, 128, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    tqb.stage2(mid, sl, out, lse)
    torch.cuda.synchronize()
    ref = O.stage1_np(q.cpu().numpy(), kv.cpu().numpy(), bt.cpu().numpy(), sl.cpu().numpy(), cents.cpu().numpy(), S,
                      layout=LAYOUT_ID[layout])
    _check(mid.cpu().numpy(), ref, f"c1 {name} Stage1")
    ref_out, ref_lse = O.stage2_np(ref, sl.cpu().numpy())
    assert_close(out.cpu().numpy(), ref_out, what=f"c1 {name} Stage2 out")
    assert_close(lse.cpu().numpy(), ref_lse, what=f"c1 {name} Stage2 lse")
