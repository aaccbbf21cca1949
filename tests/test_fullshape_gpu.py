"""Parity at the benchmark configurations' full shapes (GPU).

The other GPU tests run small shapes; these run the shapes every bench number
comes from, so each Stage1 kernel instance walks its page ring over as many
tiles as it does in the bench:

* c1  B64 x 4096, Hq32/Hk8 (GQA-4), 32 splits; SoA on both Stage1 kernels
      and AoS.  The cache is written by this library's store and checked
      byte for byte against the oracle store on the same inputs first.
* c3  B256 x 8192, Hq64/Hk8 (GQA-8, the ring kernel's two-item-per-warp
      instance), 32 splits.
* c2  B128 ragged, seq_lens U[512, 16384] (seeded), per-sequence splits
      min(32, ceil(len / 512)), fully shuffled block pool; on one GPU, and
      as the 8 data-parallel ranks' shares, each decoded on its own.
* c4  B4 x 131072 over 8 sequence-parallel ranks emulated on one GPU, 74
      local splits per rank; one rank's partials against the oracle on its
      share, and every rank's merged result (peer-memory exchange kernels)
      against the oracle's single-range decode.
* c1 against the reference's own Triton SoA V1 Stage1 run on the same GPU
  and inputs, when a reference checkout was placed under baseline/_ref
  (baseline/install_ref.py); skipped otherwise.

Bar: |got - ref| <= 1e-4 + 2e-3 |ref| (conftest.ATOL/RTOL) on Stage1 O and
LSE and on the Stage2 output and LSE; the store bit-exact.
"""

from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import ROOT, assert_close
from oracle import oracle as O
import tqb
from tqb import sharding

pytestmark = pytest.mark.gpu

SENTINEL = -12345.0
D = 128


def _rotation(seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    q, r = torch.linalg.qr(torch.randn(D, D, generator=g, dtype=torch.float64))
    return (q * torch.sign(torch.diagonal(r))[None, :]).to(torch.float32)


def _build(dev, seed, lens, Hq, Hk, layout="soa", keep_inputs=False, pool_extra=0):
    """Seeded N(0,1) keys/values of every token of every sequence written by
    this library's store into a shuffled block pool.  With ``keep_inputs``
    the store's fp32 inputs come back too (for the oracle store)."""
    B = len(lens)
    pages = [max(1, math.ceil(n / 16)) for n in lens]
    nblk = sum(pages) + pool_extra
    perm = torch.randperm(nblk, generator=torch.Generator().manual_seed(seed)).to(torch.int32)
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    bt = bt.to(dev)
    cents = tqb.get_centroids(128, 4).to(dev)
    mids = tqb.get_midpoints(cents)
    R = _rotation(seed + 1).to(dev)
    kv = torch.zeros(nblk, 16, Hk, 134, dtype=torch.uint8, device=dev)
    gen = torch.Generator(device=dev).manual_seed(seed + 2)
    kept = []
    for b in range(B):
        n = lens[b]
        tok = torch.arange(n, device=dev)
        slots = (bt[b, tok // 16].long() * 16 + tok % 16).to(torch.int32)
        for s0 in range(0, n, 8192):
            m = min(8192, n - s0)
            key = torch.randn(m * Hk, D, generator=gen, device=dev)
            val = torch.randn(m * Hk, D, generator=gen, device=dev)
            norms = key.norm(dim=1)
            y = ((key / (norms[:, None] + 1e-8)) @ R).contiguous()
            tqb.store(y, norms, val, kv, slots[s0 : s0 + m], mids, cents, layout=layout,
                      norm_correction=(layout == "soa"))
            if keep_inputs:
                kept.append((y.cpu().numpy(), norms.cpu().numpy(), val.cpu().numpy(),
                             slots[s0 : s0 + m].cpu().numpy()))
    q = torch.randn(B, Hq, D, generator=gen, device=dev).to(torch.bfloat16).float()
    q_rot = (q @ R).contiguous()
    torch.cuda.synchronize(dev)
    return dict(kv=kv, bt=bt, sl=torch.tensor(lens, dtype=torch.int32, device=dev), cents=cents, mids=mids,
                q=q_rot, lens=list(lens), kept=kept, layout=layout, Hq=Hq, Hk=Hk)


def _host(w):
    return dict(q=w["q"].cpu().numpy(), kv=w["kv"].cpu().numpy(), bt=w["bt"].cpu().numpy(),
                sl=w["sl"].cpu().numpy(), cents=w["cents"].cpu().numpy())


def _decode_gpu(w, S, nsp=None):
    dev = w["q"].device
    B, Hq = w["q"].shape[:2]
    mid = torch.full((B, Hq, S, D + 1), SENTINEL, device=dev)
    out = torch.empty(B, Hq, D, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    nsp_t = None if nsp is None else torch.tensor(nsp, dtype=torch.int32, device=dev)
    tqb.wait_timeouts(reset=True)
    tqb.stage1(w["q"], w["kv"], w["bt"], w["sl"], w["cents"], mid, layout=w["layout"], num_splits_per_seq=nsp_t)
    tqb.stage2(mid, w["sl"], out, lse, num_splits_per_seq=nsp_t)
    torch.cuda.synchronize(dev)
    assert tqb.wait_timeouts(reset=True) == 0, "a bounded device wait gave up"
    return mid.cpu().numpy(), out.cpu().numpy(), lse.cpu().numpy()


def _decode_oracle(h, S, layout="soa", nsp=None):
    lay = O.LAYOUT_SOA if layout == "soa" else O.LAYOUT_AOS
    nsp_a = None if nsp is None else np.asarray(nsp, np.int32)
    mid = O.stage1(h["q"], h["kv"], h["bt"], h["sl"], h["cents"], S, layout=lay, num_splits_per_seq=nsp_a)
    out, lse = O.stage2(mid, h["sl"], num_splits_per_seq=nsp_a)
    return mid, out, lse


def _written(lens, S, nsp=None):
    """[B, S] mask of the splits Stage1 writes (the reference split rule)."""
    m = np.zeros((len(lens), S), bool)
    for b, n in enumerate(lens):
        ns = S if nsp is None else int(nsp[b])
        for s in range(ns):
            t0, t1 = O.split_range(int(n), ns, s)
            m[b, s] = t1 > t0
    return m


def _check(got, ref, lens, S, nsp=None, what=""):
    gmid, gout, glse = got
    rmid, rout, rlse = ref
    wm = _written(lens, S, nsp)
    gm, rm = gmid.transpose(0, 2, 1, 3)[wm], rmid.transpose(0, 2, 1, 3)[wm]  # [written, Hq, D+1]
    assert_close(gm[..., :D], rm[..., :D], what=f"{what} Stage1 O")
    assert_close(gm[..., D], rm[..., D], what=f"{what} Stage1 LSE")
    assert np.all(gmid.transpose(0, 2, 1, 3)[~wm] == SENTINEL), f"{what}: an empty split was written"
    live = np.asarray(lens) > 0
    assert_close(gout[live], rout[live], what=f"{what} Stage2 output")
    assert_close(glse[live], rlse[live], what=f"{what} Stage2 LSE")


@pytest.fixture(scope="module")
def c1_soa(cuda_device):
    return _build(cuda_device, 11, [4096] * 64, 32, 8, "soa", keep_inputs=True)


@pytest.fixture(scope="module")
def c1_soa_host(c1_soa):
    return _host(c1_soa)


@pytest.fixture(scope="module")
def c1_soa_oracle(c1_soa_host):
    return _decode_oracle(c1_soa_host, 32)


def _store_matches_oracle(w, h):
    ref = np.zeros_like(h["kv"])
    lay = O.LAYOUT_SOA if w["layout"] == "soa" else O.LAYOUT_AOS
    for y, norms, val, slots in w["kept"]:
        O.store(lay, y, norms, val, w["mids"].cpu().numpy(), h["cents"], slots, ref,
                norm_correction=(w["layout"] == "soa"))
    diff = np.flatnonzero(ref.reshape(-1) != h["kv"].reshape(-1))
    assert diff.size == 0, f"{diff.size} cache bytes differ from the oracle store; first at byte {diff[0]}"


def test_c1_store_bit_exact(c1_soa, c1_soa_host):
    """The c1 cache (2,097,152 token-heads) written by this library's store
    equals the oracle store's bytes on the same inputs."""
    _store_matches_oracle(c1_soa, c1_soa_host)


@pytest.mark.parametrize("kernel", ["ring", "regs"])
def test_c1_soa_decode(c1_soa, c1_soa_oracle, kernel, monkeypatch):
    monkeypatch.setenv("TQB_STAGE1_KERNEL", kernel)
    got = _decode_gpu(c1_soa, 32)
    _check(got, c1_soa_oracle, c1_soa["lens"], 32, what=f"c1 SoA ({kernel})")


def test_c1_aos_decode(cuda_device):
    w = _build(cuda_device, 12, [4096] * 64, 32, 8, "aos", keep_inputs=True)
    h = _host(w)
    _store_matches_oracle(w, h)
    got = _decode_gpu(w, 32)
    _check(got, _decode_oracle(h, 32, layout="aos"), w["lens"], 32, what="c1 AoS")


def test_c3_gqa8_decode(cuda_device):
    """Full c3: B256 x 8192, 64 query heads over 8 KV heads, 32 splits."""
    w = _build(cuda_device, 13, [8192] * 256, 64, 8, "soa")
    h = _host(w)
    got = _decode_gpu(w, 32)
    _check(got, _decode_oracle(h, 32), w["lens"], 32, what="c3")


@pytest.fixture(scope="module")
def c2_ragged(cuda_device):
    """The c2 batch (B128, seq_lens U[512, 16384], splits min(32,
    ceil(len/512)), shuffled pool with spare blocks) and its oracle decode."""
    lens = np.random.default_rng(20261201).integers(512, 16384 + 1, size=128).tolist()
    nsp = [min(32, math.ceil(n / 512)) for n in lens]
    w = _build(cuda_device, 14, lens, 32, 8, "soa", pool_extra=64)
    h = _host(w)
    return w, nsp, _decode_oracle(h, 32, nsp=nsp)


def test_c2_ragged_decode(c2_ragged):
    """Full c2 on one GPU."""
    w, nsp, ref = c2_ragged
    got = _decode_gpu(w, 32, nsp=nsp)
    _check(got, ref, w["lens"], 32, nsp=nsp, what="c2")


def test_c2_data_parallel_rank_shares(c2_ragged):
    """c2 split over 8 data-parallel ranks as the 8-GPU bench splits it
    (sharding.plan_batch): each rank's share of 16 sequences is decoded on
    its own, as one rank does.  A share has so few non-empty tiles that the
    Stage1 tile walk cuts it by item count (at most two tiles per group),
    the cut none of the one-GPU shapes reach."""
    w, nsp, ref = c2_ragged
    lens = w["lens"]
    B, Hq = len(lens), w["Hq"]
    mid = np.full((B, Hq, 32, D + 1), SENTINEL, np.float32)
    out = np.empty((B, Hq, D), np.float32)
    lse = np.empty((B, Hq), np.float32)
    plan = sharding.plan_batch(lens, 8)
    assert sorted(i for r in plan for i in r) == list(range(B))
    dev = w["q"].device
    for idx in plan:
        it = torch.tensor(idx, dtype=torch.long, device=dev)
        part = dict(w, q=w["q"][it].contiguous(), bt=w["bt"][it].contiguous(), sl=w["sl"][it].contiguous(),
                    lens=[lens[i] for i in idx])
        m, o, l = _decode_gpu(part, 32, nsp=[nsp[i] for i in idx])
        mid[idx], out[idx], lse[idx] = m, o, l
    _check((mid, out, lse), ref, lens, 32, nsp=nsp, what="c2 rank shares")


def test_c4_sequence_parallel_8_ranks(cuda_device):
    """Full c4: B4 x 131072 split over 8 emulated SP ranks with 74 local
    splits each; rank 3's partials against the oracle on its share, and the
    merge of all ranks (the peer-memory exchange kernels) on every rank
    against the oracle's decode of the whole sequence."""
    dev = cuda_device
    world, S_local, lens = 8, 74, [131072] * 4
    w = _build(dev, 15, lens, 32, 8, "soa")
    h = _host(w)
    ranks = sharding.P2PExchange.emulated(world, len(lens), 32, dev)
    try:
        mids = []
        for r in range(world):
            bt, sl, _ = sharding.sp_shard(w["bt"], lens, world, r)
            mid = torch.full((len(lens), 32, S_local, D + 1), SENTINEL, device=dev)
            tqb.stage1(w["q"], w["kv"], bt, sl, w["cents"], mid)
            mids.append((mid, sl, bt))
        torch.cuda.synchronize(dev)
        mid3, sl3, bt3 = mids[3]
        ref3 = O.stage1(h["q"], h["kv"], bt3.cpu().numpy(), sl3.cpu().numpy(), h["cents"], S_local)
        assert_close(mid3.cpu().numpy(), ref3, what="c4 rank 3 Stage1 partials")
        tqb.wait_timeouts(reset=True)
        for r in range(world):
            ranks[r].send(mids[r][0], mids[r][1])
        outs = []
        for r in range(world):
            out = torch.empty(len(lens), 32, D, device=dev)
            lse = torch.empty(len(lens), 32, device=dev)
            ranks[r].recv(out, lse)
            outs.append((out, lse))
        torch.cuda.synchronize(dev)
        assert tqb.wait_timeouts(reset=True) == 0
        _, rout, rlse = _decode_oracle(h, 32)
        for r, (out, lse) in enumerate(outs):
            assert_close(out.cpu().numpy(), rout, what=f"c4 SP8 rank {r} merged output")
            assert_close(lse.cpu().numpy(), rlse, what=f"c4 SP8 rank {r} merged LSE")
    finally:
        ranks[0].close()


REF_CHECKOUT = ROOT / "baseline" / "_ref" / "turboquant-cuda-decode"


@pytest.mark.skipif(not (REF_CHECKOUT / "baseline" / "triton_v1.py").is_file(),
                    reason="no reference checkout under baseline/_ref (baseline/install_ref.py places it)")
def test_c1_against_reference_triton_soa_v1(c1_soa):
    """The reference's own SoA V1 Stage1 (its Triton kernel through its
    harness launcher, compiled for this GPU) and this library's Stage1 on
    the same c1 inputs: the north star's parity bar, on the GPU."""
    import importlib

    if str(REF_CHECKOUT) not in sys.path:
        sys.path.insert(0, str(REF_CHECKOUT))
    tv1 = importlib.import_module("baseline.triton_v1")
    w = c1_soa
    ref = torch.full((64, 32, 32, D + 1), float("nan"), device=w["q"].device)
    tv1.launch_soa_v1_stage1(w["q"], w["kv"], w["bt"], w["sl"], w["cents"], ref)
    got = _decode_gpu(w, 32)[0]
    ref = ref.cpu().numpy()
    assert_close(got[..., :D], ref[..., :D], what="c1 Stage1 O vs reference SoA V1")
    assert_close(got[..., D], ref[..., D], what="c1 Stage1 LSE vs reference SoA V1")
