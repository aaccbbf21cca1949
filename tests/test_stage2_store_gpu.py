"""Stage2 merge, cross-GPU partial merge and the store kernel (GPU)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, assert_close
from oracle import oracle as O
import tqb

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_stage2_vs_reference_golden(cuda_device, golden, name):
    z = golden[name]
    dev = cuda_device
    mid = torch.from_numpy(z["mid_o_soa_v1"]).to(dev)  # NaN in empty splits: must be skipped
    sl = torch.from_numpy(z["seq_lens"]).to(dev)
    B, Hq, S, D1 = mid.shape
    out = torch.empty(B, Hq, D1 - 1, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    tqb.stage2(mid, sl, out, lse)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), z["out_stage2"], what="stage2 out")
    assert_close(lse.cpu().numpy(), z["lse_stage2"], what="stage2 lse")


def test_stage2_empty_sequence_and_per_seq_splits(cuda_device):
    rng = np.random.default_rng(0)
    B, Hq, S = 4, 8, 6
    lens = np.array([0, 5, 100, 64], np.int32)
    nsp = np.array([3, 6, 4, 6], np.int32)
    mid = rng.standard_normal((B, Hq, S, 129)).astype(np.float32)
    dev = cuda_device
    out = torch.empty(B, Hq, 128, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    tqb.stage2(torch.from_numpy(mid).to(dev), torch.from_numpy(lens).to(dev), out, lse,
               num_splits_per_seq=torch.from_numpy(nsp).to(dev))
    torch.cuda.synchronize()
    ro, rl = O.stage2(mid, lens, nsp)
    assert_close(out.cpu().numpy(), ro, what="out")
    assert_close(lse.cpu().numpy(), rl, what="lse")
    assert np.isnan(out.cpu().numpy()[0]).all() and np.isneginf(lse.cpu().numpy()[0]).all()


def test_merge_partials_equals_single_pass(cuda_device):
    """Merging per-range (O, LSE) partials equals merging all splits at once
    (the identity behind the sequence-parallel path)."""
    rng = np.random.default_rng(1)
    G, B, Hq = 4, 3, 16
    parts = rng.standard_normal((G, B, Hq, 129)).astype(np.float32)
    parts[2, 1, :, 128] = -np.inf  # an empty range
    parts[2, 1, :, :128] = np.nan
    dev = cuda_device
    out = torch.empty(B, Hq, 128, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    tqb.merge_partials(torch.from_numpy(parts).to(dev), out, lse)
    torch.cuda.synchronize()
    lse_p = parts[..., 128]
    m = np.max(np.where(np.isneginf(lse_p), -np.inf, lse_p), axis=0)
    w = np.where(np.isneginf(lse_p), 0.0, np.exp(lse_p - m))
    ref = np.nansum(w[..., None] * np.nan_to_num(parts[..., :128]), axis=0) / w.sum(0)[..., None]
    assert_close(out.cpu().numpy(), ref, what="merge out")
    assert_close(lse.cpu().numpy(), m + np.log(w.sum(0)), what="merge lse")


@pytest.mark.parametrize("layout,key", [("soa", "kv_cache_soa"), ("aos", "kv_cache_aos")])
def test_store_bit_exact_vs_reference(cuda_device, golden_store, layout, key):
    z = golden_store
    dev = cuda_device
    cache = torch.from_numpy(z["cache_before"].copy()).to(dev)
    tqb.store(torch.from_numpy(z["y"]).to(dev), torch.from_numpy(z["norms"]).to(dev),
              torch.from_numpy(z["value"].reshape(-1, 128).copy()).to(dev), cache,
              torch.from_numpy(z["slot_mapping"]).to(dev), torch.from_numpy(z["midpoints"]).to(dev),
              torch.from_numpy(z["centroids"]).to(dev), layout=layout, norm_correction=(layout == "soa"))
    torch.cuda.synchronize()
    got = cache.cpu().numpy()
    assert np.array_equal(got, z[key]), f"{(got != z[key]).sum()} bytes differ"


@pytest.mark.parametrize("layout,key", [("soa", "kv_cache_soa"), ("aos", "kv_cache_aos")])
def test_store_through_vllm_view(cuda_device, golden_store, layout, key):
    """The store into vLLM's cache view, ``kv_cache.transpose(1, 2)`` of
    ``(blocks, H, N, C)`` storage (reference/turboquant_attn.py:565).  SoA
    writes a block's raw bytes from its base, so the storage holds exactly
    the reference bytes; AoS writes slot (t, h) through the view's strides,
    so the view reads back as the reference cache."""
    z = golden_store
    dev = cuda_device
    before = z["cache_before"]
    nb, bs, hk, slot = before.shape
    if layout == "soa":
        storage = torch.from_numpy(before.reshape(nb, hk, bs, slot).copy()).to(dev)  # same bytes
    else:
        storage = torch.from_numpy(before.transpose(0, 2, 1, 3).copy()).to(dev)  # head-major slots
    view = storage.transpose(1, 2)
    assert not view.is_contiguous()
    tqb.store(torch.from_numpy(z["y"]).to(dev), torch.from_numpy(z["norms"]).to(dev),
              torch.from_numpy(z["value"].reshape(-1, 128).copy()).to(dev), view,
              torch.from_numpy(z["slot_mapping"]).to(dev), torch.from_numpy(z["midpoints"]).to(dev),
              torch.from_numpy(z["centroids"]).to(dev), layout=layout, norm_correction=(layout == "soa"))
    torch.cuda.synchronize()
    if layout == "soa":
        got = storage.cpu().numpy().reshape(nb, bs, hk, slot)
    else:
        got = view.cpu().numpy()
    assert np.array_equal(got, z[key]), f"{(got != z[key]).sum()} bytes differ"


def test_store_bit_exact_vs_oracle_large(cuda_device):
    """Thousands of random token-heads, including near-midpoint values."""
    rng = np.random.default_rng(7)
    N, H, nb = 2000, 8, 160
    cents = tqb.get_centroids(128, 4)
    mids = tqb.get_midpoints(cents).numpy()
    y = rng.standard_normal((N * H, 128)).astype(np.float32) * np.float32(0.09)
    pick = rng.random(y.shape) < 0.05  # land exactly on a midpoint: `>=` goes right
    y[pick] = mids[rng.integers(0, 15, pick.sum())]
    norms = np.abs(rng.standard_normal(N * H)).astype(np.float32) * 11
    val = rng.standard_normal((N * H, 128)).astype(np.float32) * rng.uniform(0.01, 50, (N * H, 1)).astype(np.float32)
    slots = rng.permutation(nb * 16)[:N].astype(np.int32)
    slots[::97] = -1
    base = rng.integers(0, 256, (nb, 16, H, 134), dtype=np.uint8)
    ref = base.copy()
    O.store(O.LAYOUT_SOA, y, norms, val, mids, cents.numpy(), slots, ref, norm_correction=True)
    dev = cuda_device
    cache = torch.from_numpy(base).to(dev)
    tqb.store(*(torch.from_numpy(a).to(dev) for a in (y, norms, val)), cache,
              torch.from_numpy(slots).to(dev), torch.from_numpy(mids).to(dev), cents.to(dev))
    torch.cuda.synchronize()
    got = cache.cpu().numpy()
    assert np.array_equal(got, ref), f"{(got != ref).sum()} bytes differ"


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_stage2_typed_output_equals_cast(cuda_device, golden, dtype):
    """A 16-bit Stage2 output is the fp32 merge rounded to nearest even:
    bit-identical to merging into fp32 and casting (the launcher's
    output.to(query.dtype), reference/soa_decode_v1.py:643)."""
    z = golden["ragged_gqa4"]
    dev = cuda_device
    mid = torch.from_numpy(z["mid_o_soa_v1"]).to(dev)
    sl = torch.from_numpy(z["seq_lens"]).to(dev)
    B, Hq = mid.shape[:2]
    o32 = torch.empty(B, Hq, 128, device=dev)
    l32 = torch.empty(B, Hq, device=dev)
    tqb.stage2(mid, sl, o32, l32)
    o16 = torch.empty(B, Hq, 128, dtype=dtype, device=dev)
    l16 = torch.empty(B, Hq, device=dev)
    tqb.stage2(mid, sl, o16, l16)
    torch.cuda.synchronize()
    assert torch.equal(o16.view(torch.int16), o32.to(dtype).view(torch.int16))
    assert torch.equal(l16, l32)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_rotate_query_vs_torch(cuda_device, dtype):
    """Cast + rotation in one kernel against the launcher's
    query.float() @ PiT (reference/soa_decode_v1.py:535-538), on a strided
    query view; fp32 accumulation, so only the summation order differs."""
    dev = cuda_device
    g = torch.Generator(device=dev).manual_seed(5)
    big = torch.randn(37, 40, 128, generator=g, device=dev).to(dtype)
    q = big[:, 3:35]  # [37, 32, 128], batch stride 40*128
    PiT = torch.linalg.qr(torch.randn(128, 128, generator=g, device=dev))[0].contiguous()
    ref = q.double() @ PiT.double()
    got = tqb.rotate_query(q, PiT)
    out = torch.full((37, 36, 128), -7.0, device=dev)
    tqb.rotate_query(q, PiT, out=out[:, 2:34])
    torch.cuda.synchronize()
    err = (got.double() - ref).abs().max().item()
    assert err <= 1e-5 * max(1.0, ref.abs().max().item()), err
    assert torch.equal(out[:, 2:34], got)
    assert torch.all(out[:, :2] == -7.0) and torch.all(out[:, 34:] == -7.0)


def _value_edge_rows(rng, n, top):
    """Value rows that stress the quantiser's division (v - min) / scale:
    quotients a few ulps either side of every k + 1/2 (where the code
    changes), constant rows (scale clamped to 1e-8), tiny (1e-30) and huge
    (1e37) magnitudes, and plain rows at scales from 1e-6 to 1e6."""
    rows = np.empty((n, 128), np.float32)
    for i in range(n):
        kind = i % 5
        s = np.float32(10.0 ** rng.uniform(-6, 6))
        if kind == 0:
            vmin, vmax = np.float32(-rng.uniform(0.1, 3) * s), np.float32(rng.uniform(0.1, 3) * s)
            scale = np.float32((vmax - vmin) / np.float32(top))
            k = rng.integers(0, top, 126)
            a = ((k + 0.5) * np.float64(scale)).astype(np.float32)
            a = np.nextafter(a, np.float32(np.inf) * rng.choice([-1, 1], 126)).astype(np.float32)
            a[::3] = ((k[::3] + 0.5) * np.float64(scale)).astype(np.float32)
            rows[i, :126] = np.minimum(np.maximum(vmin + a, vmin), vmax)
            rows[i, 126:] = (vmin, vmax)
        elif kind == 1:
            rows[i] = np.float32(rng.standard_normal())
        elif kind == 2:
            rows[i] = rng.standard_normal(128).astype(np.float32) * np.float32(1e-30)
        elif kind == 3:
            rows[i] = rng.uniform(-1, 1, 128).astype(np.float32) * np.float32(1e37)
        else:
            rows[i] = rng.standard_normal(128).astype(np.float32) * s
    return rows


@pytest.mark.parametrize("layout", ["soa", "soa_k8", "soa_k3", "soa_k3v3", "aos"])
def test_store_value_rounding_edges(cuda_device, layout):
    """The store's value codes at the rounding edges of (v - min) / scale,
    bit-exact against the oracle's IEEE float32 division (the kernel divides
    by a correctly rounded reciprocal plus two FMA corrections)."""
    rng = np.random.default_rng(11)
    H, N, nb = 4, 1200, 320
    k3 = layout in ("soa_k3", "soa_k3v3")
    top = 7 if layout == "soa_k3v3" else 15
    val = _value_edge_rows(rng, N * H, top)
    y = (rng.standard_normal((N * H, 128)) * (3.0 if layout == "soa_k8" else 0.09)).astype(np.float32)
    norms = np.abs(rng.standard_normal(N * H)).astype(np.float32) * 7
    cents = tqb.get_centroids(128, 3 if k3 else 4).numpy()
    mids = ((cents[:-1] + cents[1:]) * 0.5).astype(np.float32) if k3 else tqb.get_midpoints(
        torch.from_numpy(cents)).numpy()
    slots = rng.permutation(nb * 16)[:N].astype(np.int32)
    slots[::89] = -1
    slot_bytes = {"soa": 134, "aos": 134, "soa_k8": 196, "soa_k3": 118, "soa_k3v3": 102}[layout]
    base = rng.integers(0, 256, (nb, 16, H, slot_bytes), dtype=np.uint8)
    ref = base.copy()
    if layout == "soa_k8":
        O.store_k8_np(y.reshape(N, H, 128), val.reshape(N, H, 128), slots, ref)
    elif k3:
        O.store_k3_np(y, norms, val, mids, cents, slots, ref, vbits=3 if layout == "soa_k3v3" else 4)
    else:
        lay = O.LAYOUT_SOA if layout == "soa" else O.LAYOUT_AOS
        O.store(lay, y, norms, val, mids, cents, slots, ref, norm_correction=layout == "soa")
    dev = cuda_device
    cache = torch.from_numpy(base).to(dev)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    if layout == "soa_k8":
        tqb.store(d(y), None, d(val), cache, d(slots), None, None, layout=layout, norm_correction=False)
    else:
        tqb.store(d(y), d(norms), d(val), cache, d(slots), d(mids), d(cents), layout=layout,
                  norm_correction=layout != "aos")
    torch.cuda.synchronize()
    got = cache.cpu().numpy()
    assert np.array_equal(got, ref), f"{(got != ref).sum()} bytes differ from the oracle store"
