"""Multi-GPU sharding on the GPU.  With one GPU, every rank of a DP / TP / SP
layout runs in turn on cuda:0 and the results are reassembled (SP through
the tqb_merge_partials kernel); with two or more GPUs, SP also runs as one
process per GPU over NCCL.  All compare with the single-process CPU oracle
over the whole sequence at the conftest tolerance."""

from __future__ import annotations

import socket

import numpy as np
import pytest
import torch

from conftest import assert_close, random_case
from oracle import oracle as O
import tqb
from tqb import sharding

pytestmark = pytest.mark.gpu


def _full_ref(c):
    mid = O.stage1(c["q_rot"], c["kv_cache"], c["block_table"], c["seq_lens"], c["centroids"], 1)
    return O.stage2(mid, c["seq_lens"])


def _dev(c, k, dev):
    return torch.from_numpy(np.ascontiguousarray(c[k])).to(dev)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sp_ranks_merged_by_kernel(cuda_device, world):
    lens = [1000, 17, 4100, 1]
    c = random_case(100 + world, len(lens), 32, 8, lens)
    dev = cuda_device
    parts = []
    for r in range(world):
        bt, sl, _ = sharding.sp_shard(_dev(c, "block_table", dev), lens, world, r)
        parts.append(sharding.local_partial(_dev(c, "q_rot", dev), _dev(c, "kv_cache", dev), bt, sl,
                                            _dev(c, "centroids", dev), 16))
    out = torch.empty(len(lens), 32, 128, device=dev)
    lse = torch.empty(len(lens), 32, device=dev)
    tqb.merge_partials(torch.stack(parts).contiguous(), out, lse)
    ref_out, ref_lse = _full_ref(c)
    assert_close(out.cpu().numpy(), ref_out, what=f"SP{world} output")
    assert_close(lse.cpu().numpy(), ref_lse, what=f"SP{world} lse")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_ranks_reassembled(cuda_device, world):
    lens = [300, 77, 1024]
    c = random_case(200 + world, len(lens), 64, 8, lens)
    dev = cuda_device
    outs = []
    for r in range(world):
        kv = sharding.tp_shard_cache(_dev(c, "kv_cache", dev), world, r)
        q = sharding.tp_shard_query(_dev(c, "q_rot", dev), 8, world, r).contiguous()
        part = sharding.local_partial(q, kv, _dev(c, "block_table", dev), _dev(c, "seq_lens", dev),
                                      _dev(c, "centroids", dev), 4)
        outs.append(part)
    got = torch.cat(outs, dim=1).cpu().numpy()  # heads back in order
    ref_out, ref_lse = _full_ref(c)
    assert_close(got[..., :128], ref_out, what=f"TP{world} output")
    assert_close(got[..., 128], ref_lse, what=f"TP{world} lse")


def test_dp_ranks_reassembled(cuda_device):
    lens = [700, 30, 2000, 512, 513, 90, 1600]
    c = random_case(300, len(lens), 32, 8, lens)
    dev = cuda_device
    world = 4
    plan = sharding.plan_batch(lens, world)
    got = np.empty((len(lens), 32, 129), np.float32)
    for r in range(world):
        idx = torch.tensor(plan[r], dtype=torch.long)
        part = sharding.local_partial(_dev(c, "q_rot", dev)[idx.to(dev)].contiguous(), _dev(c, "kv_cache", dev),
                                      _dev(c, "block_table", dev)[idx.to(dev)].contiguous(),
                                      _dev(c, "seq_lens", dev)[idx.to(dev)].contiguous(), _dev(c, "centroids", dev), 8)
        got[plan[r]] = part.cpu().numpy()
    ref_out, ref_lse = _full_ref(c)
    assert_close(got[..., :128], ref_out, what="DP output")
    assert_close(got[..., 128], ref_lse, what="DP lse")


@pytest.mark.parametrize("device_epochs", [False, True])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_sp_p2p_exchange_emulated(cuda_device, world, device_epochs):
    """The peer-memory SP exchange with every rank of one process on one GPU
    (local buffers, no IPC): all ranks send, then all merge; three steps, so
    both row sets and growing epochs are used (host epochs, or the epochs the
    device keeps in each buffer)."""
    lens = [1000, 17, 4100, 1, 0]
    c = random_case(200 + world, len(lens), 32, 8, lens)
    dev = cuda_device
    ranks = sharding.P2PExchange.emulated(world, len(lens), 32, dev, device_epochs=device_epochs)
    ref_out, ref_lse = _full_ref(c)
    live = np.asarray(lens) > 0
    try:
        mids = []
        for r in range(world):
            bt, sl, _ = sharding.sp_shard(_dev(c, "block_table", dev), lens, world, r)
            mid = torch.empty(len(lens), 32, 16, 129, device=dev)
            tqb.stage1(_dev(c, "q_rot", dev), _dev(c, "kv_cache", dev), bt, sl, _dev(c, "centroids", dev), mid)
            mids.append((mid, sl))
        tqb.wait_timeouts(reset=True)
        for step in range(3):
            for r in range(world):
                ranks[r].send(*mids[r])
            outs = []
            for r in range(world):
                out = torch.full((len(lens), 32, 128), -1.0, device=dev)
                lse = torch.empty(len(lens), 32, device=dev)
                ranks[r].recv(out, lse)
                outs.append((out, lse))
            torch.cuda.synchronize()
            assert tqb.wait_timeouts(reset=True) == 0
            for r, (out, lse) in enumerate(outs):
                got = out.cpu().numpy()
                assert_close(got[live], ref_out[live], what=f"P2P SP{world} step {step} rank {r} output")
                assert_close(lse.cpu().numpy()[live], ref_lse[live], what=f"P2P SP{world} rank {r} lse")
                assert np.all(np.isnan(got[~live])), "a sequence without tokens merges to NaN"
    finally:
        ranks[0].close()


def test_sp_p2p_device_epochs_graph_replay(cuda_device):
    """Device epochs make the exchange graph-capturable: one CUDA graph holds
    every emulated rank's exchange and then every rank's merge; three
    replays, each checked against the single-range oracle."""
    world, lens = 4, [900, 33, 2500]
    c = random_case(210, len(lens), 32, 8, lens)
    dev = cuda_device
    ranks = sharding.P2PExchange.emulated(world, len(lens), 32, dev, device_epochs=True)
    ref_out, ref_lse = _full_ref(c)
    try:
        mids = []
        for r in range(world):
            bt, sl, _ = sharding.sp_shard(_dev(c, "block_table", dev), lens, world, r)
            mid = torch.empty(len(lens), 32, 8, 129, device=dev)
            tqb.stage1(_dev(c, "q_rot", dev), _dev(c, "kv_cache", dev), bt, sl, _dev(c, "centroids", dev), mid)
            mids.append((mid, sl))
        outs = [(torch.empty(len(lens), 32, 128, device=dev), torch.empty(len(lens), 32, device=dev))
                for _ in range(world)]
        torch.cuda.synchronize()
        tqb.wait_timeouts(reset=True)
        cap = torch.cuda.Stream(dev)
        with torch.cuda.stream(cap):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                for r in range(world):
                    ranks[r].send(*mids[r])
                for r in range(world):
                    ranks[r].recv(*outs[r])
        for step in range(3):
            for o, l in outs:
                o.fill_(-1.0)
            g.replay()
            torch.cuda.synchronize()
            assert tqb.wait_timeouts(reset=True) == 0
            for r, (o, l) in enumerate(outs):
                assert_close(o.cpu().numpy(), ref_out, what=f"graph step {step} rank {r} output")
                assert_close(l.cpu().numpy(), ref_lse, what=f"graph step {step} rank {r} lse")
        del g
    finally:
        ranks[0].close()


def test_sp_p2p_merge_gives_up_on_a_missing_rank(cuda_device):
    """A rank whose peer never sends: the merge's bounded wait (about a
    second) gives up, the rows come out NaN, the device counter read by
    tqb_wait_timeouts counts it, and the context stays usable."""
    dev = cuda_device
    B, Hq = 2, 32
    ranks = sharding.P2PExchange.emulated(2, B, Hq, dev)
    try:
        lens = [40, 9]
        c = random_case(321, len(lens), Hq, 8, lens)
        mid = torch.empty(B, Hq, 4, 129, device=dev)
        sl = _dev(c, "seq_lens", dev)
        tqb.stage1(_dev(c, "q_rot", dev), _dev(c, "kv_cache", dev), _dev(c, "block_table", dev), sl,
                   _dev(c, "centroids", dev), mid)
        tqb.wait_timeouts(reset=True)
        ranks[0].send(mid, sl)  # rank 1 never sends this epoch
        out = torch.zeros(B, Hq, 128, device=dev)
        lse = torch.zeros(B, Hq, device=dev)
        ranks[0].recv(out, lse)
        torch.cuda.synchronize()
        assert tqb.wait_timeouts(reset=True) >= 1
        assert torch.isnan(out).all() and torch.isnan(lse).all()
        # the device is still fine: a full step of both ranks completes
        ranks[1].epoch = ranks[0].epoch - 1  # resynchronise the ranks' step counters
        ranks[1].send(mid, sl)
        ranks[0].recv(out, lse)
        torch.cuda.synchronize()
        assert tqb.wait_timeouts(reset=True) == 0 and torch.isfinite(out).all()
    finally:
        ranks[0].close()


@pytest.mark.multigpu
def test_sp_nccl_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    import _dist_workers as W

    lens = [2000, 33, 700]
    c = random_case(400, len(lens), 32, 8, lens)
    case = tmp_path / "case.npz"
    np.savez(case, **c)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(W.sp_nccl_worker, args=(2, port, str(case), str(tmp_path), 8), nprocs=2,
                       start_method="spawn", join=True)
    ref_out, ref_lse = _full_ref(c)
    for r in range(2):
        with np.load(tmp_path / f"nccl{r}.npz") as z:
            assert_close(z["out"], ref_out, what=f"NCCL SP rank {r} output")
            assert_close(z["lse"], ref_lse, what=f"NCCL SP rank {r} lse")


@pytest.mark.multigpu
def test_sp_p2p_two_gpus(tmp_path):
    """The peer-memory SP exchange between two processes on two GPUs (IPC
    handles swapped over NCCL, rows stored over NVLink), three steps."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    import _dist_workers as W

    lens = [2000, 33, 700]
    c = random_case(401, len(lens), 32, 8, lens)
    case = tmp_path / "case.npz"
    np.savez(case, **c)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(W.sp_p2p_worker, args=(2, port, str(case), str(tmp_path), 8), nprocs=2,
                       start_method="spawn", join=True)
    ref_out, ref_lse = _full_ref(c)
    for r in range(2):
        with np.load(tmp_path / f"p2p{r}.npz") as z:
            assert int(z["timeouts"]) == 0
            for step in range(3):
                assert_close(z["out"][step], ref_out, what=f"P2P SP rank {r} step {step} output")
                assert_close(z["lse"][step], ref_lse, what=f"P2P SP rank {r} step {step} lse")
