#!/usr/bin/env python
"""Benchmark of the TurboQuant 4bit_nc decode hot path (Stage1 + Stage2).

One JSON line on rank 0.  A "step" is one decode pass of one attention layer
over the whole batch: Stage1 (split-KV partial attention over the 4-bit
paged cache) followed by the Stage2 split merge, inputs resident in HBM.
``value`` is decode tokens/s (sequences decoded per second, summed over all
ranks) from CUDA events around exactly ``--steps`` steps, max over ranks.

Default workload (``--config c1``): the reference's fixed Qwen3-4B shape,
B=64, context 4096, 32 Q / 8 KV heads, D=128, block 16, 32 splits, SoA cache
written by the sm_100a store from seeded N(0,1) keys/values and a seeded
random rotation, shuffled physical block pool.  Under torchrun each rank
runs its own copy (data-parallel over batch, weak scaling, no collective on
the data path).

``--impl reference`` times the reference algorithm on the host CPU (the
fp32 C restatement in ``oracle/``, all host threads) on the same workload.

At N=1 the c1 line also carries, from the same process:

* ``parity``: this library's Stage1 partials and Stage2 output/LSE of the
  timed workload against the CPU oracle (the same inputs, the full c1
  workload), with the decode bar |got - ref| <= 1e-4 + 2e-3 |ref|;
* ``reference_gpu``: the reference's own Stage1 kernels (Triton AoS V1, SoA
  V1 and V2-fixed, CUDA V9 and V7 built for sm_100a) on the same B200 and
  the same inputs, loaded from the reference checkout that
  ``baseline/install_ref.py`` places under ``baseline/_ref/``, timed with the
  reference's protocol (``benchmarks/stage1.py:32-43,508-527``: 20 warm-up
  launches, 100 timed, 5 rounds in rotated order, median) beside this
  library's Stage1, and checked against the reference SoA V1 output;
* ``reference_interpreter``: the reference SoA V1 and V2-fixed Stage1 under
  ``TRITON_INTERPRET=1`` on the host CPU, a bounded subset of the c1 grid,
  with the per-program rate and the full-grid time extrapolated from it.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "turboquant-cuda-decode_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

CONFIGS = {
    # name: (B, seq_len, Hq, Hk, splits); c1 is the headline (DP, weak
    # scaling: one c1 workload per GPU); c2-c4 are the sharded configs
    # (fixed total work split over the GPUs: strong scaling).
    "c1": dict(B=64, L=4096, Hq=32, Hk=8, S=32,
               workload="Qwen3-4B decode Stage1+Stage2, B64 x 4096 ctx, Hq32/Hk8, D128, bs16, 32 splits"),
    "c2": dict(B=128, Lmin=512, Lmax=16384, Hq=32, Hk=8, S=32, split_tokens=512, parallel="dp",
               workload="ragged paged batch: B128, seq_lens U[512,16384] (seeded), Hq32/Hk8, "
                        "splits min(32, ceil(len/512)), shuffled block pool; DP by batch (LPT-balanced)"),
    "c3": dict(B=256, L=8192, Hq=64, Hk=8, S=32, parallel="tp",
               workload="Llama-3-70B-shaped decode: B256 x 8192 ctx, Hq64/Hk8 (GQA-8), 32 splits; "
                        "TP by KV head"),
    "c4": dict(B=4, L=131072, Hq=32, Hk=8, S=74, parallel="sp",
               workload="long-context decode: B4 x 131072 ctx, Hq32/Hk8; SP split-KV, merged rows exchanged "
                        "over peer memory (NVLink P2P) and merged; 74 local splits per GPU: 4 x 74 x 8 KV heads = 296 tiles, "
                        "one per Stage1 group on 148 SMs (the reference config's 16 leave most SMs idle; "
                        "the merge kernel combines any split count)"),
}
FALLBACK_HBM_GBS = 6650.0
# The arithmetic each cache layout computes in, by its key/value code suffix.
LAYOUT_DTYPE = {
    "_k4": "f32 (4-bit K/V codes, fp16-split tensor-core MMA, fp32 accumulate)",
    "_k8": "f32 (e4m3 K, 4-bit V codes, fp16 tensor-core MMA, fp32 accumulate)",
    "_k3": "f32 (3-bit K / 4-bit V codes, fp16-split tensor-core MMA, fp32 accumulate)",
    "_k3v3": "f32 (3-bit K/V codes, fp16-split tensor-core MMA, fp32 accumulate)",
}
# The Stage1 kernel each layout runs on (Hk dividing 8, as in every config).
STAGE1_KERNEL = {
    "soa": "tqb stage1_ring_kernel (TMA page ring: tensor-map page copies)",
    "aos": "tqb stage1_ring_kernel (TMA page ring: whole AoS blocks by bulk copy)",
    "soa_k8": "tqb stage1_ring_kernel (TMA page ring: whole FP8-key blocks by bulk copy)",
    "soa_k3": "tqb stage1_ring_kernel (TMA page ring: 3-bit-key blocks as padded row pairs by bulk copy)",
    "soa_k3v3": "tqb stage1_ring_kernel (TMA page ring: 3-bit-key blocks as padded row pairs by bulk copy)",
    "aos_k8": "tqb stage1_ring_kernel (TMA page ring: whole AoS FP8-key blocks by bulk copy)",
    "aos_k3": "tqb stage1_ring_kernel (TMA page ring: whole AoS 3-bit-key blocks by bulk copy)",
    "aos_k3v3": "tqb stage1_ring_kernel (TMA page ring: whole AoS 3-bit-key blocks by bulk copy)",
}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="c1",
                    help="one of " + ", ".join(sorted(CONFIGS)) + "; a comma-separated list of the sharded "
                         "configs (c2,c3,c4) runs them one after another in one process, one line each")
    ap.add_argument("--layout", choices=["soa", "aos", "soa_k8", "soa_k3", "soa_k3v3", "aos_k8", "aos_k3", "aos_k3v3"],
                    default="soa",
                    help="cache layout; soa_k8 = the turboquant_k8v4 preset (FP8 keys, 4-bit values), "
                         "soa_k3 = turboquant_k3v4_nc (3-bit keys, 4-bit values), soa_k3v3 = "
                         "turboquant_3bit_nc (3-bit keys and values); aos_* = the same presets in the AoS "
                         "slot layout; the presets run one GPU, c1 or c3's shape")
    ap.add_argument("--seed", type=int, default=20261201)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--splits", type=int, default=None,
                    help="override the config's (local) KV split count")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own kernels on the GPU")
    ap.add_argument("--no-interpreter", action="store_true",
                    help="skip the reference-under-TRITON_INTERPRET CPU sample")
    ap.add_argument("--interp-child", default=None, help=argparse.SUPPRESS)
    args = ap.parse_args()
    cfgs = args.config.split(",")
    for c in cfgs:
        if c not in CONFIGS:
            ap.error(f"unknown config {c!r}")
    if len(cfgs) > 1 and "c1" in cfgs:
        ap.error("c1 runs alone; lists are for the sharded configs c2, c3, c4")
    if args.splits is not None and len(cfgs) == 1:
        CONFIGS[args.config] = dict(CONFIGS[args.config], S=args.splits)
    return args


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------


def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------


def orthogonal(seed: int, d: int = 128) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    q, r = torch.linalg.qr(torch.randn(d, d, generator=g, dtype=torch.float64))
    return (q * torch.sign(torch.diagonal(r))[None, :]).to(torch.float32)


def build_workload(cfg: dict, seed: int, dev: torch.device, layout: str):
    """Seeded cache written by the sm_100a store, plus decode inputs."""
    import tqb
    from tqb import layout as L

    B, Lc, Hq, Hk, S = cfg["B"], cfg["L"], cfg["Hq"], cfg["Hk"], cfg["S"]
    pages = math.ceil(Lc / L.BLOCK_SIZE)
    nblk = B * pages
    gen = torch.Generator(device=dev).manual_seed(seed)
    cents = tqb.get_centroids(128, 4).to(dev)
    mids = tqb.get_midpoints(cents)
    R = orthogonal(seed + 1).to(dev)
    perm = torch.randperm(nblk, generator=torch.Generator().manual_seed(seed + 2)).to(torch.int32)
    bt = perm.reshape(B, pages).to(dev)
    k8, k3, v3 = layout.endswith("_k8"), layout.endswith(("_k3", "_k3v3")), layout.endswith("_k3v3")
    if k3:  # 3-bit keys: 8 centroids
        cents = tqb.get_centroids(128, 3).to(dev)
        mids = tqb.get_midpoints(cents)
    slot = L.K8_SLOT_SIZE if k8 else (L.K3V3_SLOT_SIZE if v3 else L.K3_SLOT_SIZE if k3 else L.SLOT_SIZE)
    kv = torch.zeros(nblk, L.BLOCK_SIZE, Hk, slot, dtype=torch.uint8, device=dev)
    chunk = 8192
    tok_b = torch.arange(Lc, device=dev)
    for b in range(B):
        slots_b = (bt[b, tok_b // 16].long() * 16 + tok_b % 16).to(torch.int32)
        for s0 in range(0, Lc, chunk):
            n = min(chunk, Lc - s0)
            key = torch.randn(n, Hk, 128, generator=gen, device=dev)
            val = torch.randn(n, Hk, 128, generator=gen, device=dev)
            if k8:  # keys at 3x unit scale spread over the e4m3 range
                tqb.triton_turboquant_store(key * 3.0, val, kv, slots_b[s0:s0 + n], None, None, 8, 128, 4,
                                            key_fp8=True)
            else:
                tqb.triton_turboquant_store(key, val, kv, slots_b[s0:s0 + n], R, mids, 3 if k3 else 4,
                                            50 if k3 else 66, 3 if v3 else 4, centroids=cents,
                                            norm_correction=(layout != "aos"), layout=layout)
    query = torch.randn(B, Hq, 128, generator=gen, device=dev).to(torch.bfloat16)
    # FP8 keys score against the unrotated query
    q_rot = query.float().contiguous() if k8 else (query.float() @ R).contiguous()
    seq_lens = torch.full((B,), Lc, dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)
    return dict(kv=kv, bt=bt, seq_lens=seq_lens, cents=cents, R=R, query=query, q_rot=q_rot,
                B=B, Hq=Hq, Hk=Hk, S=S, L=Lc, layout=layout)


def c1_config(cfg: dict, layout: str, B: int, L: int, S: int, world: int, cache_mb: float) -> dict:
    """The `config` object of the c1 line; the reference arm prints the same."""
    return {"workload": cfg["workload"], "layout": layout,
            "per_gpu_batch": B, "global_batch": world * B, "seq_len": L,
            "num_splits": S, "parallelism": f"dp{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (cache %.0f MB per GPU vs 126 MB L2); no flush" % cache_mb}


def algorithmic_bytes(w) -> int:
    """Bytes Stage1 must move: the cache slots of every token-head (134 B;
    196 B with FP8 keys), the fp32 query, the block-table entries used,
    seq_lens, the centroid table, and the fp32 mid_o write."""
    B, Hq, Hk, S, Lc = w["B"], w["Hq"], w["Hk"], w["S"], w["L"]
    cache = B * Lc * Hk * {"_k8": 196, "_k3": 118, "3v3": 102}.get(w["layout"][-3:], 134)
    q = B * Hq * 128 * 4
    bt = B * math.ceil(Lc / 16) * 4
    mid = B * Hq * S * 129 * 4
    return cache + q + bt + B * 4 + 16 * 4 + mid


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML)
# ---------------------------------------------------------------------------


class ClockSampler:
    REASONS = {
        "hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
        "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, dev: torch.device, period_s: float = 0.002):
        self.samples = []
        self.period = period_s
        self._stop = threading.Event()
        self._t = None
        self.window = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            try:  # map the CUDA device to its NVML handle by UUID
                uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
                self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            except Exception:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
                ids = [int(x) for x in vis.split(",") if x.strip().isdigit()]
                idx = ids[dev.index] if dev.index < len(ids) else dev.index
                self.h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:  # pragma: no cover - NVML missing
            self.nvml = None
            self.max_mhz = None

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM)
                reasons = self._reasons(self.h)
                self.samples.append((time.perf_counter(), mhz, reasons))
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.nvml is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self):
        if self._t is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        inside = [s for s in self.samples if self.window and self.window[0] <= s[0] <= self.window[1]]
        use = inside if inside else self.samples
        mask = 0
        for _, _, r in use:
            mask |= r
        reasons = [k for k, bit in self.REASONS.items() if mask & bit]
        return {"sm_mhz": statistics.median(m for _, m, _ in use), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(use),
                "window": "timed region" if inside else "warm-up + timed region"}


# ---------------------------------------------------------------------------
# measured numbers committed under profiles/
# ---------------------------------------------------------------------------


def measured_peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(config: str, layout: str):
    """DRAM bytes per Stage1 launch from the committed ncu summary, if any."""
    p = ROOT / "profiles" / f"stage1_{layout}_{config}.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
    return float(m.group(1)) if m else None


# ---------------------------------------------------------------------------
# CPU baseline (reference algorithm on the host cores)
# ---------------------------------------------------------------------------


def measure_store(w, dev, peak: float, reps: int = 20) -> dict:
    """The sm_100a store (4-bit SoA, norm correction) on a prefill-sized
    batch: 32768 tokens x Hk heads of rotated unit keys, norms and values,
    scattered into a shuffled block pool; 305 MB of fp32 inputs at Hk = 8,
    larger than the 126 MB L2.  CUDA events around `reps` launches after 3
    warm-up launches; bytes = the fp32 y / value / norm reads, the slot
    index, and the 134-byte slot written per token-head."""
    import tqb

    N, H = 32768, w["Hk"]
    gen = torch.Generator(device=dev).manual_seed(7)
    y = torch.nn.functional.normalize(torch.randn(N * H, 128, device=dev, generator=gen), dim=1)
    norms = torch.rand(N * H, device=dev, generator=gen) * 10 + 1
    val = torch.randn(N * H, 128, device=dev, generator=gen)
    cache = torch.zeros(N // 16, 16, H, 134, dtype=torch.uint8, device=dev)
    slots = torch.randperm(N, device=dev, generator=gen).to(torch.int32)
    mids = tqb.get_midpoints(w["cents"])
    for _ in range(3):
        tqb.store(y, norms, val, cache, slots, mids, w["cents"])
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    a.record()
    for _ in range(reps):
        tqb.store(y, norms, val, cache, slots, mids, w["cents"])
    b.record()
    torch.cuda.synchronize(dev)
    us = a.elapsed_time(b) / reps * 1e3
    per_th = 128 * 4 * 2 + 4 + 134
    alg = N * H * per_th + N * 4
    return {"token_heads": N * H, "us_per_launch": us, "token_heads_per_s": N * H / (us * 1e-6),
            "algorithmic_bytes_per_launch": alg, "bytes_per_token_head": per_th,
            "achieved_gbs": alg / (us * 1e-6) / 1e9, "frac_of_peak": alg / (us * 1e-6) / 1e9 / peak,
            "kernel": "tqb store_kernel (half a warp per token-head, 4-bit SoA with norm correction)"}


def cpu_baseline(w, min_seconds=10.0):
    """The C restatement of the reference Stage1 + Stage2 on the host cores,
    repeated over the full workload for about ``min_seconds``.  Returns the
    baseline record and the last repetition's (mid_o, output, lse), which
    the parity check compares with the GPU results."""
    from oracle import oracle as O

    cores = O.default_threads()
    q = w["q_rot"].cpu().numpy()
    kv = w["kv"].cpu().numpy()
    bt = w["bt"].cpu().numpy()
    sl = w["seq_lens"].cpu().numpy()
    cents = w["cents"].cpu().numpy()
    lay = O.LAYOUT_SOA if w["layout"] == "soa" else O.LAYOUT_AOS
    reps = 0
    t0 = time.perf_counter()
    while True:
        mid = O.stage1(q, kv, bt, sl, cents, w["S"], layout=lay, nthreads=cores)
        out, lse = O.stage2(mid, sl, nthreads=cores)
        reps += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    dt = (time.perf_counter() - t0) / reps
    rec = {"value": w["B"] / dt, "unit": "tok/s", "cores": cores, "kind": "port",
           "sample": f"full B{w['B']} x {w['L']} workload, Stage1+Stage2, fp32 C restatement "
                     f"of reference/soa_decode_v1.py + baseline/stage2.py, {reps} rep(s), "
                     f"{dt * 1e3:.1f} ms each"}
    return rec, (mid, out, lse)


PARITY_ATOL, PARITY_RTOL = 1e-4, 2e-3  # the decode bar: |got - ref| <= 1e-4 + 2e-3 |ref|


def _compare(got: np.ndarray, ref: np.ndarray) -> dict:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    both_nan = np.isnan(got) & np.isnan(ref)
    err = np.where(both_nan, 0.0, np.abs(got - ref))
    bad = ~(err <= PARITY_ATOL + PARITY_RTOL * np.abs(ref))
    return {"max_abs": float(np.nanmax(err)) if err.size else 0.0, "n_bad": int(bad.sum()), "n": int(got.size)}


def parity_vs_oracle(mid, out, lse, oracle_res) -> dict:
    """This library's results of the timed workload against the oracle's,
    element by element, with the decode bar."""
    rmid, rout, rlse = oracle_res
    gmid = mid.cpu().numpy()
    res = {"bar": f"|got - ref| <= {PARITY_ATOL} + {PARITY_RTOL}|ref|",
           "against": "CPU oracle (C restatement of the reference Stage1/Stage2), same inputs, full workload",
           "stage1_o": _compare(gmid[..., :128], rmid[..., :128]),
           "stage1_lse": _compare(gmid[..., 128], rmid[..., 128]),
           "stage2_output": _compare(out.cpu().numpy(), rout),
           "stage2_lse": _compare(lse.cpu().numpy(), rlse)}
    res["n_bad"] = sum(v["n_bad"] for v in res.values() if isinstance(v, dict))
    res["max_abs"] = max(v["max_abs"] for v in res.values() if isinstance(v, dict))
    return res


# ---------------------------------------------------------------------------
# The reference's own kernels on the same GPU (from baseline/_ref)
# ---------------------------------------------------------------------------

REF_CHECKOUT = ROOT / "baseline" / "_ref" / "turboquant-cuda-decode"
REF_NATIVE = {"CUDA V9": ("tq4_cuda_v9_ext", ROOT / "baseline" / "_ref" / "build_v9", "tq4_cuda_v9"),
              "CUDA V7": ("tq4_cuda_v7_ext", ROOT / "baseline" / "_ref" / "build_v7", "tq4_cuda_v7_stage1")}


def _reference_harness():
    """The reference's harness modules (baseline/triton_v1.py, triton_v2.py,
    common.py), imported from the checkout copy under baseline/_ref with the
    harness's own vLLM import stubs.  Raises FileNotFoundError without it."""
    import importlib

    if not (REF_CHECKOUT / "baseline" / "triton_v1.py").is_file():
        raise FileNotFoundError("no reference checkout under baseline/_ref (baseline/install_ref.py places it)")
    if str(REF_CHECKOUT) not in sys.path:
        sys.path.insert(0, str(REF_CHECKOUT))
    tv1 = importlib.import_module("baseline.triton_v1")
    tv2 = importlib.import_module("baseline.triton_v2")
    common = importlib.import_module("baseline.common")
    return tv1, tv2, common


def _reference_native(label: str):
    import importlib.machinery
    import importlib.util

    mod, folder, fn = REF_NATIVE[label]
    so = sorted(folder.glob(f"{mod}*.so"))
    if not so:
        raise FileNotFoundError(f"{label}: no {mod}*.so under baseline/_ref (baseline/install_ref.py builds it)")
    loader = importlib.machinery.ExtensionFileLoader(mod, str(so[0]))
    spec = importlib.util.spec_from_file_location(mod, str(so[0]), loader=loader)
    m = importlib.util.module_from_spec(spec)
    loader.exec_module(m)
    return getattr(m, fn)


def _event_time_ms(fn, warmup: int, iters: int) -> float:
    """benchmarks/stage1.py:32-43: warm-up launches, then `iters` launches
    between two events, mean per launch."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def reference_gpu(w, dev, ours: dict, warmup=20, iters=100, rounds=5) -> dict:
    """Time the reference's Stage1 kernels and this library's Stage1 on the
    same inputs with the reference's protocol (benchmarks/stage1.py:508-527:
    every round times each runner in a rotated order; the median over
    rounds is reported), and check each against the reference SoA V1.
    ``ours`` maps a label to (launch function, the mid_o it writes)."""
    tv1, tv2, common = _reference_harness()
    q, kv, bt, sl, cents = w["q_rot"], w["kv"], w["bt"], w["seq_lens"], w["cents"]
    B, Hq, S = w["B"], w["Hq"], w["S"]
    pair_lut = common.build_pair_lut(cents)
    aos = common.convert_soa_to_aos_kv_cache(kv, cents)
    outs = {}

    def buf():
        return torch.full((B, Hq, S, 129), float("nan"), device=dev)

    runners = []

    def add(label, fn):
        outs[label] = buf()
        runners.append((label, fn))

    add("AoS Triton V1", lambda: tv1.launch_aos_v1_stage1(q, aos, bt, sl, cents, outs["AoS Triton V1"]))
    add("SoA Triton V1", lambda: tv1.launch_soa_v1_stage1(q, kv, bt, sl, cents, outs["SoA Triton V1"]))
    add("SoA Triton V2-fixed",
        lambda: tv2.launch_tq4_v2_stage1(q, kv, bt, sl, cents, pair_lut, outs["SoA Triton V2-fixed"]))
    unavailable = {}
    for label in REF_NATIVE:
        try:
            fn = _reference_native(label)
        except Exception as e:  # recorded, not fatal: the Triton kernels still run
            unavailable[label] = str(e).splitlines()[0][:300]
            continue
        add(label, (lambda f, lab: (lambda: f(q, kv, bt, sl, cents, outs[lab])))(fn, label))
    for label, (fn, out) in ours.items():  # this library: a launcher and the buffer it writes
        outs[label] = out
        runners.append((label, fn))
    for _, fn in runners:  # compile / load and produce the outputs
        fn()
    torch.cuda.synchronize(dev)
    ref = outs["SoA Triton V1"]
    parity = {}
    for label, o in outs.items():
        if label == "SoA Triton V1":
            continue
        d_o = (o[..., :128] - ref[..., :128]).abs()
        d_l = (o[..., 128] - ref[..., 128]).abs()
        within = (o - ref).abs() <= PARITY_ATOL + PARITY_RTOL * ref.abs()
        parity[label] = {"output_max_abs": float(d_o.max()), "output_mean_abs": float(d_o.mean()),
                         "lse_max_abs": float(d_l.max()), "lse_mean_abs": float(d_l.mean()),
                         "n_bad": int((~within).sum()), "finite": bool(torch.isfinite(o).all())}
    samples = {label: [] for label, _ in runners}
    for r in range(rounds):
        k = r % len(runners)
        for label, fn in runners[k:] + runners[:k]:
            samples[label].append(_event_time_ms(fn, warmup, iters))
    med = {label: statistics.median(v) * 1e3 for label, v in samples.items()}
    v2 = med["SoA Triton V2-fixed"]
    res = {"protocol": f"benchmarks/stage1.py: {warmup} warm-up + {iters} timed launches per runner, "
                       f"{rounds} rounds in rotated order, median; no L2 flush (cache 281 MB > 126 MB L2)",
           "source": "unmodified reference checkout under baseline/_ref (Triton kernels through the "
                     "reference harness launchers; CUDA V9/V7 built from cuda/*.cu for sm_100a)",
           "median_us": med, "rounds_us": {k: [x * 1e3 for x in v] for k, v in samples.items()},
           "speedup_vs_v2_fixed": {label: v2 / t for label, t in med.items()},
           "parity_vs_soa_v1": parity}
    if unavailable:
        res["unavailable"] = unavailable
    del aos
    return res


def interpreter_sample(w, timeout_s: int = 240) -> dict:
    """Run the reference SoA V1 and V2-fixed Stage1 under TRITON_INTERPRET=1
    on the host CPU, in a child process (the interpreter is chosen when the
    kernels are defined), over a bounded subset of the c1 grid."""
    import subprocess
    import tempfile

    try:
        _reference_harness_path_ok = (REF_CHECKOUT / "baseline" / "triton_v1.py").is_file()
        if not _reference_harness_path_ok:
            return {"unavailable": "no reference checkout under baseline/_ref"}
        with tempfile.TemporaryDirectory() as td:
            np.savez(Path(td) / "w.npz", q=w["q_rot"].cpu().numpy(), kv=w["kv"].cpu().numpy(),
                     bt=w["bt"].cpu().numpy(), sl=w["seq_lens"].cpu().numpy(), cents=w["cents"].cpu().numpy())
            env = dict(os.environ, TRITON_INTERPRET="1", CUDA_VISIBLE_DEVICES="")
            res = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--interp-child", td], env=env,
                                 capture_output=True, text=True, timeout=timeout_s)
            lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
            if res.returncode != 0 or not lines:
                return {"unavailable": f"interpreter child rc={res.returncode}: "
                                       f"{(res.stderr or res.stdout).strip().splitlines()[-1:]}"}
            return json.loads(lines[-1])
    except Exception as e:
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}


def _interp_child(folder: str) -> None:
    """Child of interpreter_sample: the reference launchers with the grid cut
    to a prefix of batch row 0 (the same programs the full launch runs for
    that row; every c1 program covers 128 tokens of one sequence)."""
    tv1, tv2, common = _reference_harness()
    with np.load(Path(folder) / "w.npz") as z:
        q, kv, bt, sl, cents = (torch.from_numpy(z[k]) for k in ("q", "kv", "bt", "sl", "cents"))
    B, Hq, _ = q.shape
    Hk, S = kv.shape[2], 32
    pair_lut = common.build_pair_lut(cents)
    mid = torch.full((B, Hq, S, 129), float("nan"))

    class Prefix:  # kernel[grid] with the grid replaced by a prefix of it
        def __init__(self, kern, grid):
            self.kern, self.grid = kern, grid

        def __getitem__(self, grid):
            return self.kern[self.grid]

    out = {"cores": os.cpu_count(), "threads_used": 1,
           "note": "Triton interpreter (numpy, one thread); full-grid times are EXTRAPOLATED from the subset's "
                   "per-program rate; c1 Stage1 programs all cover 128 tokens"}
    for label, mod, attr, sub, full, call in (
        ("SoA Triton V1", tv1, "_soa_stage1", (1, 1, S), B * Hq * S,
         lambda: tv1.launch_soa_v1_stage1(q, kv, bt, sl, cents, mid)),
        ("SoA Triton V2-fixed", tv2, "tq4_decode_stage1_v2", (1, 2, S), B * Hk * S,
         lambda: tv2.launch_tq4_v2_stage1(q, kv, bt, sl, cents, pair_lut, mid)),
    ):
        real = getattr(mod, attr)
        setattr(mod, attr, Prefix(real, (1, 1, 1)))
        call()  # first call: interpreter set-up, not timed
        setattr(mod, attr, Prefix(real, sub))
        t0 = time.perf_counter()
        call()
        dt = time.perf_counter() - t0
        setattr(mod, attr, real)
        n = sub[0] * sub[1] * sub[2]
        out[label] = {"grid_subset": list(sub), "programs": n, "seconds": dt, "s_per_program": dt / n,
                      "full_grid_programs": full, "extrapolated_stage1_s": dt / n * full,
                      "extrapolated_tok_per_s": B / (dt / n * full)}
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# main
# ---------------------------------------------------------------------------


def build_workload_cpu(cfg: dict, seed: int, layout: str):
    """Host-only copy of the workload for the reference arm: seeded numpy
    keys/values written by the oracle store (reference store semantics)."""
    from oracle import oracle as O
    import tqb

    B, Lc, Hq, Hk, S = cfg["B"], cfg["L"], cfg["Hq"], cfg["Hk"], cfg["S"]
    pages = math.ceil(Lc / 16)
    nblk = B * pages
    rng = np.random.default_rng(seed)
    cents = tqb.get_centroids(128, 4).numpy()
    mids = tqb.get_midpoints(tqb.get_centroids(128, 4)).numpy()
    R = orthogonal(seed + 1).numpy()
    bt = rng.permutation(nblk).astype(np.int32).reshape(B, pages)
    kv = np.zeros((nblk, 16, Hk, 134), np.uint8)
    lay = O.LAYOUT_SOA if layout == "soa" else O.LAYOUT_AOS
    tok = np.arange(Lc)
    for b in range(B):
        slots = (bt[b, tok // 16].astype(np.int64) * 16 + tok % 16).astype(np.int32)
        key = rng.standard_normal((Lc * Hk, 128), dtype=np.float32)
        val = rng.standard_normal((Lc * Hk, 128), dtype=np.float32)
        norms = np.linalg.norm(key, axis=1).astype(np.float32)
        y = ((key / (norms[:, None] + np.float32(1e-8))) @ R).astype(np.float32)
        O.store(lay, y, norms, val, mids, cents, slots, kv, norm_correction=(layout == "soa"))
    q = rng.standard_normal((B, Hq, 128), dtype=np.float32)
    q_rot = (q @ R).astype(np.float32)
    return dict(q_rot=q_rot, kv=kv, bt=bt, seq_lens=np.full(B, Lc, np.int32), cents=cents,
                B=B, Hq=Hq, Hk=Hk, S=S, L=Lc, layout=layout)


def run_reference(args, world, rank):
    """--impl reference: the reference algorithm on the host CPU cores (the
    fp32 C restatement of reference/soa_decode_v1.py:43-314 and
    baseline/stage2.py:8-55).  Rank 0 only; other ranks exit without work."""
    if rank != 0:
        return
    if args.config != "c1":
        print(json.dumps({"impl": "reference", "unavailable": "the CPU reference arm runs the c1 headline config only"}),
              flush=True)
        return
    if args.layout not in ("soa", "aos"):
        print(json.dumps({"impl": "reference", "unavailable": "the CPU reference arm restates the 4-bit key presets only"}),
              flush=True)
        return
    from oracle import oracle as O

    cfg = CONFIGS[args.config]
    w = build_workload_cpu(cfg, args.seed, args.layout)
    cores = O.default_threads()
    lay = O.LAYOUT_SOA if args.layout == "soa" else O.LAYOUT_AOS

    def step():
        mid = O.stage1(w["q_rot"], w["kv"], w["bt"], w["seq_lens"], w["cents"], w["S"], layout=lay,
                       nthreads=cores)
        O.stage2(mid, w["seq_lens"], nthreads=cores)

    for _ in range(args.warmup):  # the same untimed warm-up count as the GPU arm
        step()
    steps = args.steps
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    # One host runs this arm whatever N is: its rate is per host, and the
    # whole-job value at N GPUs is that same host's rate.
    value = w["B"] / dt
    line = {
        "impl": "reference", "metric": "decode_tokens_per_s", "value": value, "unit": "tok/s",
        "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) K/V written by the oracle store, seeded rotation)",
        "config": c1_config(cfg, args.layout, w["B"], w["L"], w["S"], world, w["kv"].nbytes / 1e6),
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": f"the full B{w['B']} x {w['L']} workload per step, {steps} step(s) after "
                                   f"{args.warmup} warm-up, fp32 C restatement of the reference Stage1+Stage2, "
                                   f"{cores} threads"},
    }
    if world > 1:
        line["note"] = (f"CPU arm: rank 0's host alone runs it (one host, {cores} threads); its value is the "
                        "per-host rate, not scaled by the {world} GPUs of the job").replace("{world}", str(world))
    print(json.dumps(line), flush=True)


def _store_random_pages(kv, bt_row, n_tok, Hk, gen, dev, cents, mids, R):
    """Seeded N(0,1) K/V for the first n_tok tokens of one sequence, written
    by the sm_100a store into the pages bt_row lists."""
    import tqb

    chunk = 8192
    tok = torch.arange(n_tok, device=dev)
    slots = (bt_row[tok // 16].long() * 16 + tok % 16).to(torch.int32)
    for s0 in range(0, n_tok, chunk):
        n = min(chunk, n_tok - s0)
        key = torch.randn(n, Hk, 128, generator=gen, device=dev)
        val = torch.randn(n, Hk, 128, generator=gen, device=dev)
        tqb.triton_turboquant_store(key, val, kv, slots[s0:s0 + n], R, mids, 4, 66, 4, centroids=cents,
                                    norm_correction=True, layout="soa")


def build_sharded(cfg: dict, seed: int, dev: torch.device, world: int, rank: int):
    """This rank's share of a c2/c3/c4 workload (SoA cache on this GPU)."""
    import tqb
    from tqb import sharding

    par = cfg["parallel"]
    Hq, Hk, S = cfg["Hq"], cfg["Hk"], cfg["S"]
    if par == "dp":
        lens_all = np.random.default_rng(seed).integers(cfg["Lmin"], cfg["Lmax"] + 1, size=cfg["B"]).tolist()
        mine = sharding.plan_batch(lens_all, world)[rank]
        lens = [lens_all[b] for b in mine]
        nsp = [min(S, math.ceil(n / cfg["split_tokens"])) for n in lens]
        total_seqs = cfg["B"]
    elif par == "tp":
        kv0, kv1, q0, q1 = sharding.plan_kv_heads(Hq, Hk, world)[rank]
        Hq, Hk = q1 - q0, kv1 - kv0
        lens, nsp, total_seqs = [cfg["L"]] * cfg["B"], None, cfg["B"]
    else:  # sp
        t0, t1 = sharding.plan_sequence(cfg["L"], world)[rank]
        lens, nsp, total_seqs = [t1 - t0] * cfg["B"], None, cfg["B"]
    B = len(lens)
    gen = torch.Generator(device=dev).manual_seed(seed + 7919 * rank)
    cents = tqb.get_centroids(128, 4).to(dev)
    mids = tqb.get_midpoints(cents)
    R = orthogonal(seed + 1).to(dev)
    pages = [max(1, math.ceil(n / 16)) for n in lens]
    nblk = sum(pages)
    perm = torch.randperm(nblk, generator=torch.Generator().manual_seed(seed + 2 + rank)).to(torch.int32)
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]]
        k += pages[b]
    bt = bt.to(dev)
    kv = torch.zeros(nblk, 16, Hk, 134, dtype=torch.uint8, device=dev)
    for b in range(B):
        _store_random_pages(kv, bt[b], lens[b], Hk, gen, dev, cents, mids, R)
    q_rot = (torch.randn(B, Hq, 128, generator=gen, device=dev).to(torch.bfloat16).float() @ R).contiguous()
    torch.cuda.synchronize(dev)
    return dict(kv=kv, bt=bt, seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev), cents=cents,
                q_rot=q_rot, B=B, Hq=Hq, Hk=Hk, S=S, lens=lens, total_seqs=total_seqs,
                nsplits=None if nsp is None else torch.tensor(nsp, dtype=torch.int32, device=dev))


def run_sharded(args, world, rank, local):
    """c2 / c3 / c4: the sharded configs, strong-scaled over the GPUs.  The
    timed step is this rank's Stage1 + Stage2 (a CUDA graph) and, for SP, the
    NCCL all-gather of the partials and the merge kernel; the step time is
    the maximum over ranks."""
    import tqb
    from tqb import sharding

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    w = build_sharded(cfg, args.seed, dev, world, rank)
    B, Hq, S = w["B"], w["Hq"], w["S"]
    mid = torch.empty(B, Hq, S, 129, device=dev)
    out = torch.empty(B, Hq, 128, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    fout = torch.empty(B, Hq, 128, device=dev)
    flse = torch.empty(B, Hq, device=dev)

    sp = cfg["parallel"] == "sp"
    # SP: the local Stage2, the exchange of the merged rows and the
    # cross-range merge are the peer-memory exchange (tqb_sp_exchange +
    # tqb_sp_merge: rows stored straight into every rank's buffer over
    # NVLink), not Stage2 + NCCL all-gather + merge kernel.  Its epochs are
    # kept on the device, so the whole step is one CUDA graph.
    ex = sharding.P2PExchange(B, Hq, dev, device_epochs=True) if sp else None

    def local_step():
        tqb.stage1(w["q_rot"], w["kv"], w["bt"], w["seq_lens"], w["cents"], mid, num_splits_per_seq=w["nsplits"])
        if sp:
            ex.step(mid, w["seq_lens"], fout, flse, num_splits_per_seq=w["nsplits"])
        else:
            tqb.stage2(mid, w["seq_lens"], out, lse, num_splits_per_seq=w["nsplits"])

    cap = torch.cuda.Stream(dev)
    with torch.cuda.stream(cap):
        local_step()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            local_step()
    torch.cuda.synchronize(dev)

    def step():
        g.replay()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    K = args.steps
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(K):
        step()
    b_.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    ms = max_over_ranks(a.elapsed_time(b_) / K, world)
    a1, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    mid2 = torch.empty_like(mid)
    a1.record()
    for _ in range(K):
        tqb.stage1(w["q_rot"], w["kv"], w["bt"], w["seq_lens"], w["cents"], mid2, num_splits_per_seq=w["nsplits"])
    b1.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    s1_ms = max_over_ranks(a1.elapsed_time(b1) / K, world)
    cache_bytes = sum(w["lens"]) * w["Hk"] * 134
    if rank == 0:
        peak, peak_kind = measured_peak_hbm()
        line = {
            "metric": "decode_tokens_per_s", "value": w["total_seqs"] / (ms * 1e-3), "unit": "tok/s",
            "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32 (4-bit K/V codes)",
            "data": "synthetic (seeded N(0,1) K/V written by the sm_100a store)",
            "config": {"workload": cfg["workload"], "layout": "soa", "global_batch": w["total_seqs"],
                       "parallelism": f"{cfg['parallel']}{world}", "rank0_batch": B, "rank0_heads": Hq,
                       "rank0_cache_bytes": cache_bytes},
            "gpus_active": world, "nccl_ranks": world,
            "stage1_us_max_over_ranks": s1_ms * 1e3,
            "rest_of_step_us": (ms - s1_ms) * 1e3,
            "rank0_stage1_hbm_gbs": cache_bytes / (s1_ms * 1e-3) / 1e9,
            "rank0_stage1_frac_of_peak": cache_bytes / (s1_ms * 1e-3) / 1e9 / peak,
            "peak_source": peak_kind,
            "timing": ("step = CUDA-graph replay of the local Stage1 + the peer-memory exchange "
                       "(Stage2 rows to every rank over NVLink, then the merge; device epochs)" if sp else
                       "step = CUDA-graph replay of the local Stage1+Stage2") + ", CUDA events, max over ranks",
            "e2e": None, "e2e_note": "the end-to-end leg is measured on the c1 headline config",
        }
        print(json.dumps(line), flush=True)
    del g
    if ex is not None:
        ex.close()


def measure_e2e(args, w, dev, world: int, B: int, Hq: int, S: int) -> dict:
    """End to end through tqb.triton_turboquant_decode_attention with host
    buffers.  A step copies its inputs (query, block table, seq_lens: packed
    in one pinned host buffer, one copy) to the device, calls the API
    (fused query cast + rotation, Stage1, Stage2 writing bf16) on typed views
    of the device copy, and copies the bf16 output back to pinned host
    memory.  Every step does both copies.

    Three forms, same work per step:
      * ``value``: each of two buffer sets records its step (the two copies
        and the API call) once as a CUDA graph, and the graphs are replayed
        on two streams, so one step's copies overlap the other step's
        kernels, as a serving loop with two batches in flight;
      * ``serial_graph``: one buffer set, its graph replayed back to back;
      * ``serial_eager``: the Python call every step, one stream.
    Device time by CUDA events over `e2e_steps` steps, max over ranks."""
    import tqb
    import tqb.compat_aos  # noqa: F401  (the AoS launcher)

    k8, k3, v3 = args.layout.endswith("_k8"), args.layout.endswith(("_k3", "_k3v3")), args.layout.endswith("_k3v3")
    srcs = [w["query"], w["bt"], w["seq_lens"]]
    offs, n = [], 0
    for t in srcs:
        offs.append(n)
        n += (t.numel() * t.element_size() + 255) // 256 * 256

    def views(buf):
        return [buf[o:o + t.numel() * t.element_size()].view(t.dtype).view(t.shape) for o, t in zip(offs, srcs)]

    def make_set():
        hbuf = torch.empty(n, dtype=torch.uint8).pin_memory()
        for h, t in zip(views(hbuf), srcs):
            h.copy_(t.cpu())
        st = {"hbuf": hbuf, "dbuf": torch.empty(n, dtype=torch.uint8, device=dev),
              "hout": torch.empty(B, Hq, 128, dtype=torch.bfloat16).pin_memory(),
              "mbuf": torch.empty(B, Hq, S, 129, device=dev),
              "obuf": torch.empty(B, Hq, 128, dtype=w["query"].dtype, device=dev),  # vLLM's workspace: query dtype
              "lbuf": torch.empty(B, Hq, device=dev)}
        st["dq"], st["dbt"], st["dsl"] = views(st["dbuf"])
        return st

    decode = tqb.compat_aos.triton_turboquant_decode_attention if args.layout.startswith("aos") \
        else tqb.triton_turboquant_decode_attention

    def e2e_step(st):
        st["dbuf"].copy_(st["hbuf"], non_blocking=True)
        o = decode(
            st["dq"], w["kv"], st["dbt"], st["dsl"], w["R"].T, w["cents"], 1.0 / math.sqrt(128),
            8 if k8 else 3 if k3 else 4, 128 if k8 else 50 if k3 else 66, 3 if v3 else 4,
            key_fp8=k8, norm_correction=not k8, PiT=w["R"],
            mid_o_buf=st["mbuf"], output_buf=st["obuf"], lse_buf=st["lbuf"], max_num_kv_splits=S)
        st["hout"].copy_(o, non_blocking=True)

    K = args.e2e_steps
    sets = [make_set(), make_set()]
    streams = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
    # the output every step must reproduce (the computation is deterministic)
    with torch.cuda.stream(streams[0]):
        e2e_step(sets[0])
    streams[0].synchronize()
    expected = sets[0]["hout"].clone()

    def timed(run) -> float:
        torch.cuda.synchronize(dev)
        barrier(world)
        torch.cuda.synchronize(dev)
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream(dev)
        a.record(cur)
        for sm in streams:
            sm.wait_event(a)
        run()
        for sm in streams:
            cur.wait_stream(sm)
        b_.record(cur)
        torch.cuda.synchronize(dev)
        barrier(world)
        return max_over_ranks(a.elapsed_time(b_), world) / K

    # eager, one stream (the launches from Python every step)
    for _ in range(3):
        with torch.cuda.stream(streams[0]):
            e2e_step(sets[0])

    def run_eager():
        with torch.cuda.stream(streams[0]):
            for _ in range(K):
                e2e_step(sets[0])

    eager_ms = timed(run_eager)
    # each buffer set's step recorded once as a graph on its own stream
    graphs = []
    for st, sm in zip(sets, streams):
        with torch.cuda.stream(sm):
            e2e_step(st)
            sm.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=sm):
                e2e_step(st)
        graphs.append(g)
    torch.cuda.synchronize(dev)
    for _ in range(3):
        for g, sm in zip(graphs, streams):
            with torch.cuda.stream(sm):
                g.replay()

    def run_serial():
        with torch.cuda.stream(streams[0]):
            for _ in range(K):
                graphs[0].replay()

    def run_pipelined():
        for i in range(K):
            with torch.cuda.stream(streams[i % 2]):
                graphs[i % 2].replay()

    serial_ms = timed(run_serial)
    for st_ in sets:
        st_["hout"].zero_()
    piped_ms = timed(run_pipelined)
    del graphs
    # the last step of each buffer set, copied back to the host, against the
    # eager output: a race between the pipelined steps would show here
    same = [bool(torch.equal(st_["hout"].view(torch.int16), expected.view(torch.int16))) for st_ in sets]
    if not all(same):
        raise RuntimeError(f"e2e: the pipelined steps' outputs differ from the eager output ({same})")
    st = sets[0]
    h2d = st["hbuf"].numel()  # the packed buffer, padding included
    d2h = st["hout"].numel() * st["hout"].element_size()
    return {"value": world * B / (piped_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": piped_ms, "steps": K,
            "output_check": "the last pipelined step of each buffer set equals the eager output bit for bit",
            "serial_graph": {"value": world * B / (serial_ms * 1e-3), "ms_per_step": serial_ms},
            "serial_eager": {"value": world * B / (eager_ms * 1e-3), "ms_per_step": eager_ms},
            "path": "tqb.triton_turboquant_decode_attention (fused query cast + rotation, Stage1, Stage2 "
                    "writing bf16); per step one H2D copy of query/block_table/seq_lens from one pinned "
                    "host buffer and one D2H copy of the bf16 output to pinned memory; value: each of two "
                    "buffer sets' steps (copies + API call) recorded once as a CUDA graph, replayed "
                    "alternately on two streams (two steps in flight); serial_graph: one graph, one "
                    "stream; serial_eager: the Python call every step"}


def main():
    args = parse_args()
    if args.interp_child:
        _interp_child(args.interp_child)
        return
    args.warmup = max(3, args.warmup)
    world, rank, local = dist_init()
    preset = args.layout not in ("soa", "aos")
    if preset and (args.config not in ("c1", "c3") or world > 1):
        raise SystemExit("the FP8 / 3-bit preset layouts run on one GPU: the c1 workload, or c3's GQA-8 "
                         "shape unsharded")
    if args.impl == "ours" and args.config != "c1" and not preset:
        for c in args.config.split(","):
            args.config = c
            run_sharded(args, world, rank, local)
            barrier(world)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    import tqb

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    if args.config == "c3":  # a preset cache at c3's GQA-8 shape, on one GPU
        cfg = dict(cfg, workload=cfg["workload"].replace("TP by KV head", "one GPU, unsharded"))
    w = build_workload(cfg, args.seed + 1000 * rank, dev, args.layout)
    B, Hq, S = w["B"], w["Hq"], w["S"]
    mid = torch.empty(B, Hq, S, 129, device=dev)
    out = torch.empty(B, Hq, 128, device=dev)
    lse = torch.empty(B, Hq, device=dev)

    def stage1_call():
        tqb.stage1(w["q_rot"], w["kv"], w["bt"], w["seq_lens"], w["cents"], mid, layout=args.layout)

    def step():
        stage1_call()
        tqb.stage2(mid, w["seq_lens"], out, lse)

    # The decode step is captured once as a CUDA graph (as a serving engine
    # launches it) and replayed: the timed region holds the GPU work without
    # the Python argument marshalling between launches.  Stage1 alone is
    # timed the same way for the roofline.
    cap = torch.cuda.Stream(dev)
    with torch.cuda.stream(cap):
        step()
        torch.cuda.synchronize(dev)
        g_step, g_s1 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_step, stream=cap):
            step()
        with torch.cuda.graph(g_s1, stream=cap):
            stage1_call()
    torch.cuda.synchronize(dev)

    clocks = ClockSampler(dev)
    clocks.start()
    for _ in range(args.warmup):
        g_step.replay()
    torch.cuda.synchronize(dev)
    barrier(world)
    torch.cuda.synchronize(dev)
    K = args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    start.record()
    for i in range(K):
        g_step.replay()
    end.record()
    torch.cuda.synchronize(dev)
    w1 = time.perf_counter()
    barrier(world)
    # Stage1 alone (same inputs, K launches back to back)
    a1, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a1.record()
    for i in range(K):
        g_s1.replay()
    b1.record()
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks.mark(w0, w1)
    clocks.stop()
    step_ms_local, s1_ms_local = start.elapsed_time(end) / K, a1.elapsed_time(b1) / K
    total_ms = max_over_ranks(step_ms_local * K, world)
    s1_avg_ms = max_over_ranks(s1_ms_local, world)
    # Stage2 (+ the launch between) per rank, then the max: the difference of
    # the two maxima would also carry the spread between GPUs
    s2_ms = max_over_ranks(step_ms_local - s1_ms_local, world)
    ms_per_step = total_ms / K
    value = world * B / (ms_per_step * 1e-3)
    del g_step

    # -- the reference's own kernels on this GPU, same inputs, its protocol --
    ref_gpu = None
    single_c1 = world == 1 and args.config == "c1"
    if single_c1 and args.layout == "soa" and not args.no_reference_gpu:
        mid_eager = torch.empty_like(mid)
        ours = {"tqb (graph replay)": (g_s1.replay, mid),
                "tqb (compat.launch_soa_v1_stage1)":
                    ((lambda: tqb.compat.launch_soa_v1_stage1(w["q_rot"], w["kv"], w["bt"], w["seq_lens"],
                                                              w["cents"], mid_eager)), mid_eager)}
        try:
            ref_gpu = reference_gpu(w, dev, ours)
        except Exception as e:  # the reference not placed, or its kernels refused: say so in the line
            ref_gpu = {"unavailable": f"{type(e).__name__}: {e}"[:400]}
        del mid_eager
        torch.cuda.synchronize(dev)
    del g_s1
    # the timed step's results, for the parity check against the oracle
    tqb.stage1(w["q_rot"], w["kv"], w["bt"], w["seq_lens"], w["cents"], mid, layout=args.layout)
    tqb.stage2(mid, w["seq_lens"], out, lse)
    torch.cuda.synchronize(dev)

    # -- end to end through the production entry point, host buffers ------
    e2e = None
    if args.e2e_steps > 0:
        e2e = measure_e2e(args, w, dev, world, B, Hq, S)

    if rank != 0:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    peak, peak_kind = measured_peak_hbm()
    alg = algorithmic_bytes(w)
    achieved = alg / (s1_avg_ms * 1e-3) / 1e9
    traffic = ncu_traffic(args.config, args.layout)
    line = {
        "metric": "decode_tokens_per_s",
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": LAYOUT_DTYPE[args.layout[3:] or "_k4"],
        "data": "synthetic (seeded N(0,1) K/V written by the sm_100a store, seeded rotation)",
        "config": c1_config(cfg, args.layout, B, w["L"], S, world, w["kv"].numel() / 1e6),
        "stage1_us": s1_avg_ms * 1e3,
        "stage2_us": s2_ms * 1e3,
        "timing": ("value: exactly `steps` CUDA-graph replays of the decode step (Stage1 + Stage2) after "
                   "`warmup`, CUDA events; stage1_us: `steps` Stage1-only replays (the roofline's duration); "
                   "stage2_us: the step minus Stage1 on each rank, max over ranks; "
                   "stage1_us_reference_protocol: the reference's protocol (benchmarks/stage1.py, 20 warm-up + "
                   "100 timed, 5 rotated rounds, median) in reference_gpu"),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6.65 TB/s",
                     "algorithmic_bytes_per_launch": alg,
                     "kernel": STAGE1_KERNEL[args.layout]},
        "gpu_launches": 2 * K,
        "clocks": clocks.summary(),
        "e2e": e2e,
    }
    if ref_gpu is not None:
        line["reference_gpu"] = ref_gpu
        med = ref_gpu.get("median_us", {})
        if "tqb (graph replay)" in med:
            line["stage1_us_reference_protocol"] = med["tqb (graph replay)"]
            line["speedup_vs_v2_fixed"] = ref_gpu["speedup_vs_v2_fixed"]["tqb (graph replay)"]
    if args.layout == "soa":
        line["store"] = measure_store(w, dev, peak)
    if not args.no_cpu_baseline and world == 1 and args.layout in ("soa", "aos"):
        # the C restatement covers the 4-bit keys only
        line["cpu_baseline"], oracle_res = cpu_baseline(w)
        line["parity"] = parity_vs_oracle(mid, out, lse, oracle_res)
        del oracle_res
    if single_c1 and args.layout == "soa" and not args.no_interpreter:
        line["reference_interpreter"] = interpreter_sample(w)
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
