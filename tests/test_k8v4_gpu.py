"""turboquant_k8v4 (FP8 keys, 4-bit values) on the GPU.

The cache is the reference's SoA form for FP8 keys (reference/soa_store.py:
125-221): per token-head 128 e4m3 key bytes and 64 value bytes, then the
fp16 v-scale and v-zero in the block's meta region.  Bars: the store
bit-exact against the oracle store (which is pinned to the reference's value
bytes and to the hardware e4m3 cast of the key), Stage1 and Stage2 within
1e-4 + 2e-3 |ref| against the reference's own Stage1 output and the float64
oracle.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import RTOL, assert_close
from oracle import oracle as O
import tqb
from tqb import compat

pytestmark = pytest.mark.gpu

SENTINEL = -12345.0


@pytest.fixture(autouse=True)
def no_wait_timeouts(cuda_device):
    tqb.wait_timeouts(reset=True)
    yield
    torch.cuda.synchronize()
    assert tqb.wait_timeouts(reset=True) == 0, "a bounded device wait gave up"


def _k8_case(seed, B, Hq, Hk, lens, pool_extra=3):
    """Seeded FP8-key cache written by the oracle store, shuffled block pool,
    random bytes in unused slots."""
    rng = np.random.default_rng(seed)
    pages = [max(1, math.ceil(n / 16)) for n in lens]
    nblk = sum(pages) + pool_extra
    cache = rng.integers(0, 256, size=(nblk, 16, Hk, 196), dtype=np.uint8)
    perm = rng.permutation(nblk)
    bt = np.zeros((B, max(pages)), np.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    slots = np.concatenate([bt[b, np.arange(n) // 16] * 16 + np.arange(n) % 16
                            for b, n in enumerate(lens)]).astype(np.int32)
    key = (rng.standard_normal((len(slots), Hk, 128)) * 3.0).astype(np.float32)
    val = rng.standard_normal((len(slots), Hk, 128)).astype(np.float32)
    O.store_k8_np(key, val, slots, cache)
    q = (rng.standard_normal((B, Hq, 128)) * 0.5).astype(np.float32)
    return dict(query=q, kv_cache=cache, block_table=bt, seq_lens=np.asarray(lens, np.int32))


def _dev(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _stage1(dev, z, S):
    q = _dev(z["query"], dev).float()
    mid = torch.full((q.shape[0], q.shape[1], S, 129), SENTINEL, device=dev)
    tqb.stage1(q, _dev(z["kv_cache"], dev), _dev(z["block_table"], dev), _dev(z["seq_lens"], dev), None, mid,
               layout="soa_k8")
    torch.cuda.synchronize()
    return mid.cpu().numpy()


def _check(got, ref, what):
    written = ~np.isnan(ref[..., 0])
    assert np.all(got[~written] == SENTINEL), f"{what}: wrote into an empty split"
    assert_close(got[written], ref[written], what=what)


def test_store_bit_exact(cuda_device, golden_k8):
    """The FP8-key store kernel against the oracle store on the reference's
    inputs (e4m3 keys with round-to-nearest-even and saturation, 4-bit
    values, fp16 scale/zero), padding and overflowing keys included."""
    z = golden_k8
    dev = cuda_device
    ref = z["cache_before"].copy()
    O.store_k8_np(z["key"], z["value"], z["slot_mapping"], ref)
    cache = _dev(z["cache_before"], dev)
    n, hk = z["key"].shape[:2]
    tqb.store(_dev(z["key"].reshape(n * hk, 128), dev), None, _dev(z["value"].reshape(n * hk, 128), dev), cache,
              _dev(z["slot_mapping"], dev), None, layout="soa_k8", norm_correction=False)
    torch.cuda.synchronize()
    got = cache.cpu().numpy()
    assert np.array_equal(got, ref), f"{(got != ref).sum()} bytes differ"


def test_stage1_vs_reference_golden(cuda_device, golden_k8):
    """Stage1 on the reference's FP8-key cache against the reference SoA
    Stage1 with KEY_FP8=1 (ragged lengths, an empty split, GQA-4), then
    Stage2 against the reference Stage2."""
    z = golden_k8
    dev = cuda_device
    S = int(z["num_splits"])
    got = _stage1(dev, z, S)
    _check(got, z["mid_o"], "k8v4 Stage1")
    mid = torch.from_numpy(np.where(np.isnan(z["mid_o"]), 0.0, got).astype(np.float32)).to(dev)
    B, Hq = mid.shape[:2]
    out = torch.empty(B, Hq, 128, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    tqb.stage2(mid, _dev(z["seq_lens"], dev), out, lse)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), z["out_stage2"], what="k8v4 Stage2 out")
    assert_close(lse.cpu().numpy(), z["lse_stage2"], what="k8v4 Stage2 lse")


@pytest.mark.parametrize("hq,hk", [(32, 8), (16, 2), (8, 1)])
def test_stage1_gqa_vs_oracle(cuda_device, hq, hk):
    """GQA 4 and 8 (one and two head tiles per warp), ragged lengths with
    splits starting mid-page, against the float64 oracle."""
    lens = [1, 45, 300, 517]
    z = _k8_case(31 + hq + hk, len(lens), hq, hk, lens)
    S = 5
    ref = O.stage1_np(z["query"], z["kv_cache"], z["block_table"], z["seq_lens"], None, S, layout=O.LAYOUT_SOA_K8)
    _check(_stage1(cuda_device, z, S), ref, f"k8v4 Stage1 Hq{hq}/Hk{hk}")


def test_launchers_store_and_decode(cuda_device):
    """The reference-named launchers with ``key_fp8=True``: the store from
    fp16 keys/values (bit-exact against the oracle store), then the decode on
    an fp16 query (no rotation) into fp16, against the oracle's Stage1 and
    Stage2 on the same cache."""
    dev = cuda_device
    rng = np.random.default_rng(12)
    lens = [200, 33, 0, 129]
    B, Hq, Hk, S = len(lens), 32, 8, 6
    pages = [max(1, math.ceil(n / 16)) for n in lens]
    nblk = sum(pages) + 2
    before = rng.integers(0, 256, size=(nblk, 16, Hk, 196), dtype=np.uint8)
    perm = rng.permutation(nblk)
    bt = np.zeros((B, max(pages)), np.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    slots = np.concatenate([bt[b, np.arange(n) // 16] * 16 + np.arange(n) % 16
                            for b, n in enumerate(lens)]).astype(np.int32)
    key = torch.from_numpy(rng.standard_normal((len(slots), Hk, 128)) * 3.0).to(torch.float16)
    val = torch.from_numpy(rng.standard_normal((len(slots), Hk, 128))).to(torch.float16)
    ref_cache = before.copy()
    O.store_k8_np(key.float().numpy(), val.float().numpy(), slots, ref_cache)
    cache = _dev(before, dev)
    compat.triton_turboquant_store(key.to(dev), val.to(dev), cache, _dev(slots, dev), None, None, 8, 128, 4,
                                   key_fp8=True)
    torch.cuda.synchronize()
    assert np.array_equal(cache.cpu().numpy(), ref_cache)

    query = torch.from_numpy(rng.standard_normal((B, Hq, 128)) * 0.5).to(torch.float16)
    mid = O.stage1_np(query.float().numpy(), ref_cache, bt, np.asarray(lens, np.int32), None, S,
                      layout=O.LAYOUT_SOA_K8)
    ref_out, ref_lse = O.stage2_np(mid, np.asarray(lens, np.int32))
    lse = torch.empty(B, Hq, device=dev)
    out = compat.triton_turboquant_decode_attention(
        query.to(dev), cache, _dev(bt, dev), _dev(np.asarray(lens, np.int32), dev), None, None,
        1.0 / math.sqrt(128), 8, 128, 4, key_fp8=True, max_num_kv_splits=S, lse_buf=lse)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16
    live = np.asarray(lens) > 0
    got = out.float().cpu().numpy()
    ref16 = torch.from_numpy(ref_out[live].astype(np.float32)).to(torch.float16).float().numpy()
    assert_close(got[live], ref16, rtol=RTOL + 2.0 ** -10, what="k8v4 decode out")
    assert_close(lse.cpu().numpy()[live], ref_lse[live], what="k8v4 decode lse")
    assert np.all(np.isnan(got[~live]))


@pytest.mark.parametrize("hq,hk", [(32, 8), (8, 2), (4, 1), (12, 4), (16, 8), (8, 8), (20, 4)])
@pytest.mark.parametrize("kernel", ["default", "regs"])
def test_stage1_page_ring_and_register_kernel(cuda_device, hq, hk, kernel, monkeypatch):
    """FP8 keys on both Stage1 kernels: the TMA page ring (GQA <= 4 with Hk
    dividing 8: whole FP8 blocks per page, e4m3 converted in registers) and
    the register-ring kernel (TQB_STAGE1_KERNEL=regs, and GQA-5 always).
    Ragged lengths with an empty sequence, a split of more than 32 pages and
    splits starting mid-page, against the float64 oracle."""
    if kernel == "regs":
        monkeypatch.setenv("TQB_STAGE1_KERNEL", "regs")
    lens = [1, 0, 1100, 45, 300, 517, 2100]
    z = _k8_case(71 + hq + 3 * hk, len(lens), hq, hk, lens, pool_extra=7)
    S = 6
    ref = O.stage1_np(z["query"], z["kv_cache"], z["block_table"], z["seq_lens"], None, S, layout=O.LAYOUT_SOA_K8)
    _check(_stage1(cuda_device, z, S), ref, f"k8v4 Stage1 Hq{hq}/Hk{hk} ({kernel})")


def test_c1_fp8_decode_vs_oracle(cuda_device):
    """The c1 shape (B64 x 4096, Hq32/Hk8, S32) with FP8 keys, on the page
    ring: every partial, then Stage2, against the float64 oracle on the
    same cache (written by the FP8-key store from seeded N(0,1) K/V)."""
    dev = cuda_device
    B, L, Hq, Hk, S = 64, 4096, 32, 8, 32
    gen = torch.Generator(device=dev).manual_seed(23)
    pages = L // 16
    nblk = B * pages
    bt = torch.randperm(nblk, device=dev, generator=gen).view(B, pages).to(torch.int32)
    kv = torch.zeros(nblk, 16, Hk, 196, dtype=torch.uint8, device=dev)
    tok = torch.arange(L, device=dev)
    for b in range(B):  # one sequence per store call
        slots = (bt[b, tok // 16] * 16 + tok % 16).to(torch.int32)
        key = torch.randn(L * Hk, 128, device=dev, generator=gen) * 3.0
        val = torch.randn(L * Hk, 128, device=dev, generator=gen)
        tqb.store(key, None, val, kv, slots, None, None, layout="soa_k8", norm_correction=False)
    q = torch.randn(B, Hq, 128, device=dev, generator=gen) * 0.5
    sl = torch.full((B,), L, dtype=torch.int32, device=dev)
    mid = torch.full((B, Hq, S, 129), SENTINEL, device=dev)
    tqb.stage1(q, kv, bt, sl, None, mid, layout="soa_k8")
    out = torch.empty(B, Hq, 128, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    tqb.stage2(mid, sl, out, lse)
    torch.cuda.synchronize()
    ref = O.stage1_np(q.cpu().numpy(), kv.cpu().numpy(), bt.cpu().numpy(), sl.cpu().numpy(), None, S,
                      layout=O.LAYOUT_SOA_K8)
    _check(mid.cpu().numpy(), ref, "c1 FP8 Stage1")
    ref_out, ref_lse = O.stage2_np(ref, sl.cpu().numpy())
    assert_close(out.cpu().numpy(), ref_out, what="c1 FP8 Stage2 out")
    assert_close(lse.cpu().numpy(), ref_lse, what="c1 FP8 Stage2 lse")
