"""Worker bodies for the multi-process sharding tests (imported by spawned
children, so they live outside the test modules)."""

from __future__ import annotations

import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for _p in (str(ROOT), str(ROOT / "turboquant-cuda-decode_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)


def _init(rank: int, world: int, port: int, backend: str):
    import torch.distributed as dist

    dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))


def sp_oracle_worker(rank: int, world: int, port: int, case_path: str, out_dir: str, local_splits: int):
    """SP on CPU: this rank's token range through the oracle (Stage1 +
    Stage2), all-gather of the partials over gloo, oracle merge."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from oracle import oracle as O
    from tqb import sharding

    _init(rank, world, port, "gloo")
    try:
        with np.load(case_path) as z:
            c = {k: z[k] for k in z.files}
        bt, lens, _ = sharding.sp_shard(torch.from_numpy(c["block_table"]), c["seq_lens"].tolist(), world, rank)
        mid = O.stage1(c["q_rot"], c["kv_cache"], bt.numpy(), lens.numpy(), c["centroids"], local_splits)
        out, lse = O.stage2(mid, lens.numpy())
        part = sharding.pack_partial(torch.from_numpy(np.asarray(out, np.float32)),
                                     torch.from_numpy(np.asarray(lse, np.float32)))
        parts = sharding.gather_partials(part)
        mo, ml = O.merge_np(parts.numpy())
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), out=mo, lse=ml, parts=parts.numpy())
    finally:
        dist.destroy_process_group()


def dp_gather_worker(rank: int, world: int, port: int, out_dir: str):
    """DP on CPU: each rank's rows gathered back in plan order over gloo."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from tqb import sharding

    _init(rank, world, port, "gloo")
    try:
        lens = [700, 30, 4000, 512, 512, 90, 1600]
        plan = sharding.plan_batch(lens, world)
        mine = torch.tensor([[float(b), float(lens[b])] for b in plan[rank]]).reshape(-1, 2)
        got = sharding.gather_rows(mine, [len(p) for p in plan])
        np.save(os.path.join(out_dir, f"dp{rank}.npy"), got.numpy())
    finally:
        dist.destroy_process_group()


def sp_nccl_worker(rank: int, world: int, port: int, case_path: str, out_dir: str, local_splits: int):
    """SP on GPUs: this rank's pages on cuda:rank, sp_decode over NCCL."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from tqb import sharding

    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl")
    try:
        dev = torch.device("cuda", rank)
        with np.load(case_path) as z:
            c = {k: z[k] for k in z.files}
        bt, lens, _ = sharding.sp_shard(torch.from_numpy(c["block_table"]), c["seq_lens"].tolist(), world, rank)
        out, lse = sharding.sp_decode(torch.from_numpy(c["q_rot"]).to(dev), torch.from_numpy(c["kv_cache"]).to(dev),
                                      bt.to(dev), lens.to(dev), torch.from_numpy(c["centroids"]).to(dev),
                                      local_splits=local_splits)
        torch.cuda.synchronize(dev)
        np.savez(os.path.join(out_dir, f"nccl{rank}.npz"), out=out.cpu().numpy(), lse=lse.cpu().numpy())
    finally:
        dist.destroy_process_group()


def sp_p2p_worker(rank: int, world: int, port: int, case_path: str, out_dir: str, local_splits: int):
    """SP on GPUs with the exchange over peer memory (sp_decode_p2p), three steps."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import tqb
    from tqb import sharding

    torch.cuda.set_device(rank)
    _init(rank, world, port, "nccl")
    try:
        dev = torch.device("cuda", rank)
        with np.load(case_path) as z:
            c = {k: z[k] for k in z.files}
        bt, lens, _ = sharding.sp_shard(torch.from_numpy(c["block_table"]), c["seq_lens"].tolist(), world, rank)
        B = lens.shape[0]
        ex = sharding.P2PExchange(B, 32, dev)
        tqb.wait_timeouts(reset=True)
        outs, lses = [], []
        try:
            for _ in range(3):
                out, lse = sharding.sp_decode_p2p(ex, torch.from_numpy(c["q_rot"]).to(dev),
                                                  torch.from_numpy(c["kv_cache"]).to(dev), bt.to(dev), lens.to(dev),
                                                  torch.from_numpy(c["centroids"]).to(dev),
                                                  local_splits=local_splits)
                outs.append(out.cpu().numpy())
                lses.append(lse.cpu().numpy())
            timeouts = tqb.wait_timeouts(reset=True)
        finally:
            ex.close()
        np.savez(os.path.join(out_dir, f"p2p{rank}.npz"), out=np.stack(outs), lse=np.stack(lses), timeouts=timeouts)
    finally:
        dist.destroy_process_group()
