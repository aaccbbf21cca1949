"""Query rotation fused into Stage1 (tqb_stage1_rotated), on the GPU.

The fused path (one cooperative launch of the page-ring kernel whose prologue
rotates the rows, for SoA caches and GQA <= 4) must give exactly what the
two-launch path gives: tqb_rotate_query, then tqb_stage1.  Both rotate with
fp32 FMAs in the same k order, so q_rot and every partial are compared bit
for bit; the decode itself is checked against the CPU oracle.  Also: the
fused call recorded in a CUDA graph and replayed, and the shapes that take
the two-launch path inside tqb_stage1_rotated (GQA-8, the register kernel).
"""

from __future__ import annotations


import numpy as np
import pytest
import torch

from conftest import assert_close, random_case
from oracle import oracle as O
import tqb
from tqb import ops

pytestmark = pytest.mark.gpu

SENTINEL = -12345.0


@pytest.fixture(autouse=True)
def no_wait_timeouts(cuda_device):
    tqb.wait_timeouts(reset=True)
    yield
    torch.cuda.synchronize()
    assert tqb.wait_timeouts(reset=True) == 0, "a bounded device wait gave up"


def _same(a, b):
    return bool(((a == b) | (torch.isnan(a) & torch.isnan(b))).all())


def _case(dev, seed, B, Hq, Hk, lens, qdtype):
    c = random_case(seed, B, Hq, Hk, lens)
    rng = np.random.default_rng(seed + 1)
    rot = torch.from_numpy(np.linalg.qr(rng.standard_normal((128, 128)))[0].astype(np.float32)).to(dev)
    query = torch.from_numpy(rng.standard_normal((B, Hq, 128)).astype(np.float32)).to(dev).to(qdtype)
    t = {k: torch.from_numpy(np.ascontiguousarray(c[k])).to(dev) for k in
         ("kv_cache", "block_table", "seq_lens", "centroids")}
    return c, t, query, rot


def _two_launch(t, query, rot, S):
    q_rot = ops.rotate_query(query, rot)
    mid = torch.full((query.shape[0], query.shape[1], S, 129), SENTINEL, device=query.device)
    ops.stage1(q_rot, t["kv_cache"], t["block_table"], t["seq_lens"], t["centroids"], mid)
    return q_rot, mid


def _fused(t, query, rot, S):
    q_rot = torch.full(query.shape, -1.0, dtype=torch.float32, device=query.device)
    mid = torch.full((query.shape[0], query.shape[1], S, 129), SENTINEL, device=query.device)
    ops.stage1(q_rot, t["kv_cache"], t["block_table"], t["seq_lens"], t["centroids"], mid, query=query,
               rotation=rot)
    return q_rot, mid


@pytest.mark.parametrize("qdtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(3, 32, 8, [300, 17, 1024], 8), (64, 32, 8, [512] * 64, 32),
                                   (5, 16, 4, [700, 1, 0, 2000, 64], 6), (2, 4, 1, [129, 64], 3)])
def test_fused_rotation_matches_two_launches(cuda_device, qdtype, shape):
    B, Hq, Hk, lens, S = shape
    c, t, query, rot = _case(cuda_device, 700 + B, B, Hq, Hk, lens, qdtype)
    qa, ma = _two_launch(t, query, rot, S)
    qb, mb = _fused(t, query, rot, S)
    torch.cuda.synchronize()
    assert torch.equal(qa, qb), "fused q_rot differs from tqb_rotate_query"
    assert _same(ma, mb), "fused Stage1 differs from the two-launch path"
    # and the decode against the oracle on the same rotated query
    ref = O.stage1(qa.cpu().numpy(), c["kv_cache"], c["block_table"], c["seq_lens"], c["centroids"], S)
    got = mb.cpu().numpy()
    written = ~np.isnan(ref[..., 0])
    assert np.all(got[~written] == SENTINEL)
    assert_close(got[written], ref[written], what="fused Stage1 vs oracle")


def test_fused_rotation_graph_replay(cuda_device):
    """The cooperative fused launch recorded in a CUDA graph; three replays
    with new queries written into the captured input."""
    dev = cuda_device
    B, Hq, Hk, lens, S = 8, 32, 8, [900, 33, 2500, 128, 4096, 1, 640, 77], 16
    c, t, query, rot = _case(dev, 731, B, Hq, Hk, lens, torch.bfloat16)
    q_rot = torch.empty(B, Hq, 128, device=dev)
    mid = torch.full((B, Hq, S, 129), SENTINEL, device=dev)

    def call():
        ops.stage1(q_rot, t["kv_cache"], t["block_table"], t["seq_lens"], t["centroids"], mid, query=query,
                   rotation=rot)

    call()
    torch.cuda.synchronize()
    cap = torch.cuda.Stream(dev)
    with torch.cuda.stream(cap):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            call()
    gen = torch.Generator(device=dev).manual_seed(5)
    for step in range(3):
        query.copy_(torch.randn(B, Hq, 128, generator=gen, device=dev).to(torch.bfloat16))
        g.replay()
        torch.cuda.synchronize()
        qa, ma = _two_launch(t, query, rot, S)
        torch.cuda.synchronize()
        assert torch.equal(qa, q_rot), f"replay {step}: q_rot differs"
        assert _same(ma, mid), f"replay {step}: partials differ"
    del g


@pytest.mark.parametrize("case", ["gqa8", "regs", "aos"])
def test_rotated_entry_two_launch_fallbacks(cuda_device, case, monkeypatch):
    """Where the fused kernel does not apply (GQA-8, the register kernel
    forced, an AoS cache whose slots the page ring does not copy whole),
    tqb_stage1_rotated runs the rotation kernel then Stage1: same results."""
    dev = cuda_device
    if case == "regs":
        monkeypatch.setenv("TQB_STAGE1_KERNEL", "regs")
    if case == "aos":
        lens = [300, 17, 1024]
        z = random_case(741, 3, 24, 6, lens, layout="aos")  # Hk = 6 does not divide 8: register kernel
        rng = np.random.default_rng(742)
        rot = torch.from_numpy(np.linalg.qr(rng.standard_normal((128, 128)))[0].astype(np.float32)).to(dev)
        query = torch.from_numpy(rng.standard_normal((3, 24, 128)).astype(np.float32)).to(dev)
        t = {k: torch.from_numpy(np.ascontiguousarray(z[k])).to(dev) for k in
             ("kv_cache", "block_table", "seq_lens", "centroids")}
        qa = ops.rotate_query(query, rot)
        ma = torch.full((3, 24, 4, 129), SENTINEL, device=dev)
        ops.stage1(qa, t["kv_cache"], t["block_table"], t["seq_lens"], t["centroids"], ma, layout="aos")
        qb = torch.empty_like(qa)
        mb = torch.full_like(ma, SENTINEL)
        ops.stage1(qb, t["kv_cache"], t["block_table"], t["seq_lens"], t["centroids"], mb, layout="aos",
                   query=query, rotation=rot)
    else:
        Hq, Hk = (64, 8) if case == "gqa8" else (32, 8)
        c, t, query, rot = _case(dev, 745, 4, Hq, Hk, [1000, 5, 300, 2049], torch.float16)
        qa, ma = _two_launch(t, query, rot, 8)
        qb, mb = _fused(t, query, rot, 8)
    torch.cuda.synchronize()
    assert torch.equal(qa, qb) and _same(ma, mb)


def test_rotated_entry_rejects_mismatched_output(cuda_device):
    dev = cuda_device
    c, t, query, rot = _case(dev, 751, 2, 32, 8, [64, 64], torch.float32)
    q_rot = torch.empty(2, 32, 128, device=dev)
    mid = torch.empty(2, 32, 2, 129, device=dev)
    with pytest.raises(tqb.TqbError):
        ops.stage1(q_rot, t["kv_cache"], t["block_table"], t["seq_lens"], t["centroids"], mid,
                   query=query[:1], rotation=rot)
