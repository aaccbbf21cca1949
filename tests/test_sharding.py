"""Multi-GPU sharding: the plans (host logic) and, with world size 2 on the
CPU over gloo, the SP exchange + merge and the DP gather, checked against the
single-process oracle.  The merged SP output must equal full attention over
the whole sequence within fp32 reassociation (the conftest tolerance)."""

from __future__ import annotations

import socket

import numpy as np
import pytest

from conftest import assert_close, random_case
from oracle import oracle as O
from tqb import sharding


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_plan_batch_covers_and_balances():
    rng = np.random.default_rng(0)
    lens = rng.integers(512, 16385, size=128).tolist()
    for world in (1, 2, 4, 8):
        plan = sharding.plan_batch(lens, world)
        assert sorted(b for p in plan for b in p) == list(range(128))
        loads = [sum(lens[b] for b in p) for p in plan]
        # LPT bound: no rank exceeds the mean by more than the longest sequence
        assert max(loads) <= sum(lens) / world + max(lens)
        assert all(p == sorted(p) for p in plan)


def test_plan_kv_heads():
    assert sharding.plan_kv_heads(64, 8, 8) == [(r, r + 1, 8 * r, 8 * r + 8) for r in range(8)]
    assert sharding.plan_kv_heads(32, 8, 2) == [(0, 4, 0, 16), (4, 8, 16, 32)]
    with pytest.raises(ValueError):
        sharding.plan_kv_heads(32, 8, 3)


@pytest.mark.parametrize("n,world", [(131072, 8), (1000, 4), (17, 8), (0, 2), (16, 3), (4097, 2)])
def test_plan_sequence_is_page_aligned_partition(n, world):
    ranges = sharding.plan_sequence(n, world)
    assert len(ranges) == world
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    for t0, t1 in ranges:
        assert t0 <= t1 and (t0 == t1 or t0 % 16 == 0)


def _spawn(fn, world, *args):
    import torch.multiprocessing as mp

    mp.start_processes(fn, args=(world, _free_port()) + args, nprocs=world, start_method="spawn", join=True)


def test_sp_gloo_world2_matches_single_process(tmp_path):
    import _dist_workers as W

    lens = [300, 17, 1024, 1]
    c = random_case(77, len(lens), 32, 8, lens)
    case = tmp_path / "case.npz"
    np.savez(case, **c)
    _spawn(W.sp_oracle_worker, 2, str(case), str(tmp_path), 4)
    full = O.stage1(c["q_rot"], c["kv_cache"], c["block_table"], c["seq_lens"], c["centroids"], 1)
    ref_out, ref_lse = O.stage2(full, c["seq_lens"])
    for r in range(2):
        with np.load(tmp_path / f"rank{r}.npz") as z:
            assert z["parts"].shape == (2, len(lens), 32, 129)
            assert_close(z["out"], ref_out, what=f"SP rank {r} output")
            assert_close(z["lse"], ref_lse, what=f"SP rank {r} lse")
    # the 1-token sequence lives on rank 0 only: rank 1's part is empty (-inf)
    with np.load(tmp_path / "rank0.npz") as z:
        assert np.all(np.isneginf(z["parts"][1, 3, :, 128]))


def test_dp_gloo_world2_gathers_in_plan_order(tmp_path):
    import _dist_workers as W

    _spawn(W.dp_gather_worker, 2, str(tmp_path))
    lens = [700, 30, 4000, 512, 512, 90, 1600]
    plan = sharding.plan_batch(lens, 2)
    want = np.array([[b, lens[b]] for p in plan for b in p], np.float32)
    for r in range(2):
        np.testing.assert_array_equal(np.load(tmp_path / f"dp{r}.npy"), want)
