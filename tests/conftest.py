"""Shared fixtures.  GPU tests carry ``@pytest.mark.gpu``; everything else runs
on a CPU-only host."""

from __future__ import annotations

import sys
from pathlib import Path

import math

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "turboquant-cuda-decode_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"

for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN_CASES = ["c0", "ragged_gqa4", "ragged_gqa8_hk1", "ragged_gqa8_hk2"]

# Parity bar of the decode path: |got - ref| <= ATOL + RTOL * |ref|
# (1e-4 absolute, 2e-3 relative) on Stage1 O and LSE and on Stage2.
ATOL = 1e-4
RTOL = 2e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA GPUs")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden():
    return {name: load_golden(name) for name in GOLDEN_CASES}


@pytest.fixture(scope="session")
def golden_store():
    return load_golden("store_small")


@pytest.fixture(scope="session")
def golden_k8():
    """turboquant_k8v4 (FP8 keys): the reference FP8 store and SoA Stage1."""
    return load_golden("k8v4_ragged")


@pytest.fixture(scope="session")
def golden_k3():
    """turboquant_k3v4_nc (3-bit keys): the reference store and SoA Stage1."""
    return load_golden("k3v4_ragged")


@pytest.fixture(scope="session")
def golden_sinks():
    """SoA Stage1 of the reference with and without attention sinks."""
    return load_golden("sinks_gqa4")


def assert_close(got, ref, atol=ATOL, rtol=RTOL, what=""):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    same_special = (np.isnan(got) & np.isnan(ref)) | (np.isinf(ref) & (got == ref))
    with np.errstate(invalid="ignore"):
        err = np.abs(got - ref)
        bad = ~same_special & ~(err <= atol + rtol * np.abs(ref))
    if bad.any():
        i = np.argwhere(bad)[0]
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.size} elements outside {atol}+{rtol}*|ref|; "
            f"max err {np.nanmax(err):.3e}; first bad {tuple(i)} got {got[tuple(i)]} ref {ref[tuple(i)]}")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def random_case(seed, B, Hq, Hk, seq_lens, pool_extra=3, block_stride_pad=0, layout="soa"):
    """Seeded cache written by the CPU oracle store (reference semantics),
    shuffled block pool, random garbage in unused slots.  ``layout="aos"``
    writes the AoS cache as the reference AoS store does (the norm correction
    is applied by the AoS decode, not folded into the stored norm)."""
    import tqb
    from oracle import oracle as O
    from tqb import layout as L

    rng = np.random.default_rng(seed)
    pages = [max(1, math.ceil(n / 16)) for n in seq_lens]
    nblk = sum(pages) + pool_extra
    slot = L.SLOT_SIZE
    cache = rng.integers(0, 256, size=(nblk, 16, Hk, slot), dtype=np.uint8)
    perm = rng.permutation(nblk)
    bt = np.zeros((B, max(pages)), np.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    cents = tqb.get_centroids(128, 4).numpy()
    mids = tqb.get_midpoints(tqb.get_centroids(128, 4)).numpy()
    ntok = int(sum(seq_lens))
    slots = np.concatenate([bt[b, np.arange(n) // 16] * 16 + np.arange(n) % 16 for b, n in enumerate(seq_lens)]).astype(np.int32)
    key = rng.standard_normal((ntok * Hk, 128)).astype(np.float32)
    norms = np.linalg.norm(key, axis=1).astype(np.float32)
    R = np.linalg.qr(rng.standard_normal((128, 128)))[0].astype(np.float32)
    y = ((key / (norms[:, None] + 1e-8)) @ R).astype(np.float32)
    val = rng.standard_normal((ntok * Hk, 128)).astype(np.float32)
    if layout == "soa":
        O.store(O.LAYOUT_SOA, y, norms, val, mids, cents, slots, cache, norm_correction=True)
    else:
        O.store(O.LAYOUT_AOS, y, norms, val, mids, cents, slots, cache, norm_correction=False)
    q = rng.standard_normal((B, Hq, 128)).astype(np.float32)
    return dict(q_rot=q, kv_cache=cache, block_table=bt, seq_lens=np.asarray(seq_lens, np.int32),
                centroids=cents)
