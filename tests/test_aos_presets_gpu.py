"""AoS forms of the FP8-key and 3-bit presets on the GPU.

The reference's AoS cache for ``turboquant_k8v4``, ``turboquant_k3v4_nc``
and ``turboquant_3bit_nc`` (reference/aos_store.py:26-340,
reference/aos_decode.py:43-313): one slot per (token, KV head), [key codes |
raw fp16 key norm (3-bit keys) | value codes | fp16 vscale | fp16 vzero], 196,
118 or 102 bytes.  Bars: the store bit-exact against the oracle store (itself
pinned to the reference store's bytes), Stage1 and Stage2 within
1e-4 + 2e-3 |ref| against the reference's own AoS Stage1 output on the
fixture cache and against the float64 oracle on fresh seeded caches, through
the C ABI and through the reference-named launchers.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import RTOL, assert_close, load_golden
from oracle import oracle as O
import tqb
from tqb import compat, compat_aos

pytestmark = pytest.mark.gpu

SENTINEL = -12345.0
PRESETS = {  # fixture, C-ABI layout name, oracle layout, (key_fp8, mse_bits, value_quant_bits)
    "k8": ("aos_k8v4_ragged", "aos_k8", O.LAYOUT_AOS_K8, (True, 8, 4)),
    "k3": ("aos_k3v4_ragged", "aos_k3", O.LAYOUT_AOS_K3, (False, 3, 4)),
    "k3v3": ("aos_k3v3_ragged", "aos_k3v3", O.LAYOUT_AOS_K3V3, (False, 3, 3)),
}


@pytest.fixture(autouse=True)
def no_wait_timeouts(cuda_device):
    tqb.wait_timeouts(reset=True)
    yield
    torch.cuda.synchronize()
    assert tqb.wait_timeouts(reset=True) == 0, "a bounded device wait gave up"


def _dev(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def _written_check(got, ref, what):
    written = ~np.isnan(ref[..., 0])
    assert np.all(got[~written] == SENTINEL), f"{what}: wrote into an empty split"
    assert_close(got[written], ref[written], what=what)


@pytest.mark.parametrize("preset", list(PRESETS))
def test_store_bit_exact(cuda_device, preset):
    """The store kernel on the fixture's store inputs writes the oracle
    store's bytes (the oracle is pinned to the reference store)."""
    name, lay, olay, _ = PRESETS[preset]
    z = load_golden(name)
    dev = cuda_device
    ref = z["cache_before"].copy()
    kv = _dev(z["cache_before"], dev)
    if preset == "k8":
        H = kv.shape[2]
        y = z["key"].reshape(-1, 128)
        O.store_aos_np(olay, z["key"], None, z["value"], None, z["slot_mapping"], ref)
        tqb.store(_dev(y, dev), None, _dev(z["value"].reshape(-1, 128), dev), kv, _dev(z["slot_mapping"], dev),
                  None, None, layout=lay, norm_correction=False)
    else:
        O.store_aos_np(olay, z["y"], z["norms"], z["value"], z["midpoints"], z["slot_mapping"], ref)
        tqb.store(_dev(z["y"], dev), _dev(z["norms"], dev), _dev(z["value"], dev), kv, _dev(z["slot_mapping"], dev),
                  _dev(z["midpoints"], dev), _dev(z["centroids"], dev), layout=lay, norm_correction=False)
    torch.cuda.synchronize()
    got = kv.cpu().numpy()
    assert np.array_equal(got, ref), f"{(got != ref).sum()} bytes differ from the oracle store"
    if preset != "k8":  # the 3-bit forms equal the reference store byte for byte
        assert np.array_equal(got, z["kv_cache"])


@pytest.mark.parametrize("preset", list(PRESETS))
def test_stage1_vs_reference_golden(cuda_device, preset):
    """Stage1 on the reference-written AoS cache against the reference AoS
    V1 Stage1 output, then Stage2 against the reference Stage2."""
    name, lay, _, _ = PRESETS[preset]
    z = load_golden(name)
    dev = cuda_device
    q = z["query"] if preset == "k8" else z["q_rot"]
    S = int(z["num_splits"])
    B, Hq = q.shape[:2]
    mid = torch.full((B, Hq, S, 129), SENTINEL, device=dev)
    cents = None if preset == "k8" else _dev(z["centroids"], dev)
    sl = _dev(z["seq_lens"], dev)
    tqb.stage1(_dev(q, dev), _dev(z["kv_cache"], dev), _dev(z["block_table"], dev), sl, cents, mid, layout=lay)
    torch.cuda.synchronize()
    got = mid.cpu().numpy()
    _written_check(got, z["mid_o"], f"{preset} AoS Stage1 vs reference")
    out = torch.empty(B, Hq, 128, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    tqb.stage2(mid, sl, out, lse)
    torch.cuda.synchronize()
    live = z["seq_lens"] > 0
    assert_close(out.cpu().numpy()[live], z["out_stage2"][live], what=f"{preset} Stage2 out")
    assert_close(lse.cpu().numpy()[live], z["lse_stage2"][live], what=f"{preset} Stage2 lse")


@pytest.mark.parametrize("hq,hk", [(32, 8), (16, 2)])
@pytest.mark.parametrize("preset", list(PRESETS))
def test_launchers_vs_oracle(cuda_device, preset, hq, hk):
    """The reference-named store and decode launchers on an AoS cache of
    each preset (GQA-4 and GQA-8, ragged lengths with an empty sequence and a
    split longer than 32 pages), against the float64 oracle on the same
    cache: the store by compat.triton_turboquant_store(layout="aos"), the
    decode by compat_aos.triton_turboquant_decode_attention (query cast and
    rotation, Stage1, Stage2)."""
    name, lay, olay, (fp8, mse_bits, vbits) = PRESETS[preset]
    dev = cuda_device
    rng = np.random.default_rng(500 + hq + len(preset))
    lens = [700, 33, 0, 1100, 16]
    B = len(lens)
    pages = [max(1, math.ceil(n / 16)) for n in lens]
    nblk = sum(pages) + 5
    slot = O.aos_slot_bytes(olay)
    kv = _dev(rng.integers(0, 256, size=(nblk, 16, hk, slot), dtype=np.uint8), dev)
    perm = rng.permutation(nblk)
    bt = np.zeros((B, max(pages)), np.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    slots = np.concatenate([bt[b, np.arange(n) // 16] * 16 + np.arange(n) % 16 for b, n in enumerate(lens)])
    ntok = len(slots)
    key = torch.from_numpy((rng.standard_normal((ntok, hk, 128)) * (3.0 if fp8 else 1.0)).astype(np.float32)).to(dev)
    val = torch.from_numpy(rng.standard_normal((ntok, hk, 128)).astype(np.float32)).to(dev)
    Pi = torch.from_numpy(np.linalg.qr(rng.standard_normal((128, 128)))[0].astype(np.float32)).to(dev)
    cents = tqb.get_centroids(128, 3 if mse_bits == 3 else 4).to(dev)
    mids = tqb.get_midpoints(cents)
    compat.triton_turboquant_store(key, val, kv, _dev(slots.astype(np.int32), dev), Pi.T.contiguous(), mids,
                                   mse_bits, 128 if fp8 else 50, vbits, key_fp8=fp8, centroids=cents,
                                   norm_correction=False, layout="aos")
    query = torch.from_numpy(rng.standard_normal((B, hq, 128)).astype(np.float32)).to(dev)
    S = 8
    lse = torch.empty(B, hq, device=dev)
    out = compat_aos.triton_turboquant_decode_attention(
        query, kv, _dev(bt, dev), _dev(np.asarray(lens, np.int32), dev), Pi, cents, 1.0 / math.sqrt(128),
        mse_bits, 128 if fp8 else 50, vbits, key_fp8=fp8, norm_correction=not fp8, max_num_kv_splits=S,
        lse_buf=lse)
    torch.cuda.synchronize()
    q_ref = query.cpu().numpy() if fp8 else (query @ Pi.T).cpu().numpy()
    mid = O.stage1_np(q_ref, kv.cpu().numpy(), bt, np.asarray(lens), cents.cpu().numpy(), S, layout=olay)
    ref_out, ref_lse = O.stage2_np(mid, np.asarray(lens))
    live = np.asarray(lens) > 0
    assert_close(out.cpu().numpy()[live], ref_out[live], what=f"{preset} GQA-{hq // hk} decode out")
    assert_close(lse.cpu().numpy()[live], ref_lse[live], what=f"{preset} GQA-{hq // hk} decode lse")


def test_aos_presets_reject_wrong_slot(cuda_device):
    """A cache whose slots are smaller than the preset's AoS slot is
    rejected on the host with the reason."""
    dev = cuda_device
    kv = torch.zeros(4, 16, 2, 134, dtype=torch.uint8, device=dev)  # 134 < 196
    q = torch.zeros(1, 4, 128, device=dev)
    mid = torch.empty(1, 4, 2, 129, device=dev)
    with pytest.raises(tqb.TqbError, match="AoS strides"):
        tqb.stage1(q, kv, torch.zeros(1, 2, dtype=torch.int32, device=dev),
                   torch.tensor([20], dtype=torch.int32, device=dev), None, mid, layout="aos_k8")


@pytest.mark.parametrize("hq,hk", [(32, 8), (8, 2), (4, 1), (12, 4), (20, 4)])
@pytest.mark.parametrize("kernel", ["default", "regs"])
@pytest.mark.parametrize("preset", list(PRESETS))
def test_stage1_page_ring_and_register_kernel(cuda_device, preset, hq, hk, kernel, monkeypatch):
    """The AoS presets on both Stage1 kernels: the TMA page ring (Hk dividing
    8: whole blocks of packed slots per page, realigned shared loads, the
    norm correction of the 3-bit forms in the kernel) and the register-ring
    kernel (TQB_STAGE1_KERNEL=regs).  GQA 1-5, ragged lengths with an empty
    sequence and a split of more than 32 pages, against the float64 oracle
    on a cache written by the oracle's AoS store."""
    if kernel == "regs":
        monkeypatch.setenv("TQB_STAGE1_KERNEL", "regs")
    _, lay, olay, (fp8, _, vbits) = PRESETS[preset]
    rng = np.random.default_rng(600 + hq + 7 * hk + vbits + (50 if fp8 else 0))
    lens = [1, 0, 1100, 45, 300, 517, 2100]
    B = len(lens)
    pages = [max(1, math.ceil(n / 16)) for n in lens]
    nblk = sum(pages) + 7
    slot = O.aos_slot_bytes(olay)
    cache = rng.integers(0, 256, size=(nblk, 16, hk, slot), dtype=np.uint8)
    perm = rng.permutation(nblk)
    bt = np.zeros((B, max(pages)), np.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    slots = np.concatenate([bt[b, np.arange(n) // 16] * 16 + np.arange(n) % 16 for b, n in enumerate(lens)])
    n = len(slots)
    cents = tqb.get_centroids(128, 3).numpy()
    mids = ((cents[:-1] + cents[1:]) * 0.5).astype(np.float32)
    val = rng.standard_normal((n * hk, 128)).astype(np.float32)
    if fp8:
        y = (rng.standard_normal((n * hk, 128)) * 3.0).astype(np.float32)
        norms = None
    else:
        key = rng.standard_normal((n * hk, 128)).astype(np.float32)
        norms = np.linalg.norm(key, axis=1).astype(np.float32)
        y = (key / norms[:, None]).astype(np.float32)
    O.store_aos_np(olay, y, norms, val, None if fp8 else mids, slots.astype(np.int32), cache)
    q = rng.standard_normal((B, hq, 128)).astype(np.float32)
    S = 6
    ref = O.stage1_np(q, cache, bt, np.asarray(lens, np.int32), None if fp8 else cents, S, layout=olay)
    dev = cuda_device
    mid = torch.full((B, hq, S, 129), SENTINEL, device=dev)
    tqb.stage1(_dev(q, dev), _dev(cache, dev), _dev(bt, dev), _dev(np.asarray(lens, np.int32), dev),
               None if fp8 else _dev(cents, dev), mid, layout=lay)
    torch.cuda.synchronize()
    _written_check(mid.cpu().numpy(), ref, f"{preset} AoS Stage1 Hq{hq}/Hk{hk} ({kernel})")
