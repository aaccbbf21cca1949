"""Generate the golden vectors that pin the CPU oracle and the CUDA path.

This script runs the reference's own Triton kernels on the host CPU under
``TRITON_INTERPRET=1`` and saves their inputs and outputs as small ``.npz``
fixtures next to this file.  It needs a reference checkout, named by the
``TQ_REFERENCE_DIR`` environment variable (required), and is only run where
that checkout exists; the fixtures it writes are what travels and what the tests
read.  Nothing here is imported by the product.

Reference kernels exercised (paths relative to the reference checkout):

* SoA store      ``reference/soa_store.py:223-373`` (``_tq_fused_store_mse``),
  launcher ``:381-524`` (``triton_turboquant_store``)
* AoS store      ``reference/aos_store.py:221-340``, launcher ``:350-447``
* SoA V1 Stage1  ``reference/soa_decode_v1.py:43-314`` (the correctness oracle)
* AoS V1 Stage1  ``reference/aos_decode.py:43-313``
* V2-fixed       ``baseline/triton_v2.py:58-561`` (fp16 tensor-core baseline)
* Stage2 merge   ``baseline/stage2.py:8-55``
* Codebook       ``reference/centroids.py:31-86``
* Other presets  FP8 keys (``_tq_fused_store_fp8``, ``reference/soa_store.py:
  125-221``; SoA Stage1 with ``KEY_FP8=1``), 3-bit keys with 4-bit or 3-bit
  values (the MSE store with ``MSE_BITS=3`` / ``VQB=3``, ``:223-373``, and
  the SoA Stage1 with those constexprs), attention sinks (SoA Stage1 with
  ``USE_SINKS=1``, ``reference/soa_decode_v1.py:134-145``), and the AoS
  forms of the three presets (``reference/aos_store.py:145-340``,
  ``reference/aos_decode.py:43-313``)

Note on FP8: the interpreter's float -> e4m3 cast rounds ties up, flushes
subnormals and wraps on overflow, unlike the hardware cast the compiled
reference uses on sm_90+, so the FP8 fixture's key bytes pin nothing; its
value bytes, meta and Stage1 output (decoding is exact) are used.

The kernels are launched through the raw ``kernel[grid](...)`` form with each
fixture's constexprs, because the harness launchers assert the fixed
B64x4K shapes (``baseline/triton_v2.py:594-607``).

Usage::

    python tests/golden/make_golden.py            # all fixtures
    python tests/golden/make_golden.py c0 store   # a subset
"""

from __future__ import annotations

import importlib.util
import math
import os
import sys
import time
import types
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402

HERE = Path(__file__).resolve().parent
if not os.environ.get("TQ_REFERENCE_DIR"):
    raise SystemExit("set TQ_REFERENCE_DIR to a zben777/turboquant-cuda-decode checkout")
REF = Path(os.environ["TQ_REFERENCE_DIR"])

HEAD_DIM = 128
BLOCK_SIZE = 16
MSE_BITS = 4
VALUE_BITS = 4
MSE_BYTES = HEAD_DIM * MSE_BITS // 8  # 64
VAL_BYTES = HEAD_DIM * VALUE_BITS // 8  # 64
SLOT = MSE_BYTES + VAL_BYTES + 6  # 134
AOS_KPS = MSE_BYTES + 2  # key_packed_size for the AoS slot


# ---------------------------------------------------------------------------
# Loading the reference modules with the minimal vLLM import surface they use
# ---------------------------------------------------------------------------


def _stub_modules() -> None:
    names = (
        "vllm",
        "vllm.platforms",
        "vllm.triton_utils",
        "vllm.v1",
        "vllm.v1.attention",
        "vllm.v1.attention.ops",
        "vllm.v1.attention.ops.triton_decode_attention",
        "vllm.v1.attention.ops.triton_turboquant_decode",
    )
    for name in names:
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["vllm.platforms"].current_platform = types.SimpleNamespace(
        is_cuda_alike=lambda: False
    )
    sys.modules["vllm.triton_utils"].tl = triton.language
    sys.modules["vllm.triton_utils"].triton = triton
    sys.modules["vllm.v1.attention.ops.triton_decode_attention"]._fwd_kernel_stage2 = None
    sys.modules["vllm.v1.attention.ops.triton_turboquant_decode"]._use_fp8_e4b15 = (
        lambda device=0: 0
    )
    # soa_store.py uses a package-relative import of the decode module.
    pkg = "_tqref"
    if pkg not in sys.modules:
        mod = types.ModuleType(pkg)
        mod.__path__ = []
        sys.modules[pkg] = mod
        dec = types.ModuleType(pkg + ".triton_turboquant_decode")
        dec._use_fp8_e4b15 = lambda device=0: 0
        sys.modules[pkg + ".triton_turboquant_decode"] = dec


def _load(relpath: str, modname: str):
    _stub_modules()
    spec = importlib.util.spec_from_file_location(modname, REF / relpath)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[modname] = mod
    spec.loader.exec_module(mod)
    return mod


class Ref:
    """Lazily loaded reference kernels."""

    def __init__(self) -> None:
        self.centroids_mod = _load("reference/centroids.py", "_tqref_centroids")
        self.soa_dec = _load("reference/soa_decode_v1.py", "_tqref.soa_decode_v1")
        self.aos_dec = _load("reference/aos_decode.py", "_tqref.aos_decode")
        self.soa_store = _load("reference/soa_store.py", "_tqref.triton_turboquant_store")
        self.aos_store = _load("reference/aos_store.py", "_tqref.aos_store")
        # baseline/triton_v2.py and stage2.py import `.common`, which imports
        # the centroid module by bare name; give them a tiny package.
        sys.path.insert(0, str(REF / "reference"))
        base = types.ModuleType("_tqbase")
        base.__path__ = [str(REF / "baseline")]
        sys.modules["_tqbase"] = base
        self.common = _load("baseline/common.py", "_tqbase.common")
        self.v2 = _load("baseline/triton_v2.py", "_tqbase.triton_v2")
        self.stage2 = _load("baseline/stage2.py", "_tqbase.stage2")


# ---------------------------------------------------------------------------
# Launch helpers (raw grids, fixture-specific constexprs)
# ---------------------------------------------------------------------------


def soa_meta_offset(hk: int) -> int:
    return BLOCK_SIZE * hk * (MSE_BYTES + VAL_BYTES)


def run_soa_v1(ref: Ref, q_rot, kv, bt, seq_lens, cents, num_splits, sinks=None):
    B, Hq, D = q_rot.shape
    Hk = kv.shape[2]
    mid = torch.full((B, Hq, num_splits, D + 1), float("nan"), dtype=torch.float32)
    ref.soa_dec._tq_decode_stage1[(B, Hq, num_splits)](
        q_rot, kv, kv.view(torch.uint16), bt, seq_lens, cents, mid, sinks,
        q_rot.stride(0), q_rot.stride(1), kv.stride(0), bt.stride(0),
        mid.stride(0), mid.stride(1), mid.stride(2),
        NUM_KV_HEADS=Hk, HEAD_DIM=D, BLOCK_SIZE=BLOCK_SIZE,
        NUM_KV_SPLITS=num_splits, KV_GROUP_SIZE=Hq // Hk,
        MSE_BITS=MSE_BITS, MSE_BYTES=MSE_BYTES, VQB=VALUE_BITS,
        VAL_DATA_BYTES=VAL_BYTES, KEY_DATA_BYTES=MSE_BYTES,
        META_REGION_OFFSET=soa_meta_offset(Hk), NUM_SOA_FIELDS=3,
        SOA_K_NORM=0, SOA_V_SCALE=1, SOA_V_ZERO=2,
        ATTN_SCALE=1.0 / math.sqrt(D), BLOCK_D=triton.next_power_of_2(D),
        BLOCK_KV=4, KEY_FP8=0, NORM_CORRECTION=1, FP8_E4B15=0,
        USE_SINKS=0 if sinks is None else 1,
        num_warps=1, num_stages=1,
    )
    return mid


def run_soa_k8(ref: Ref, query, kv, bt, seq_lens, cents, num_splits):
    """SoA V1 Stage1 with FP8 (e4m3) keys: the query goes in unrotated."""
    B, Hq, D = query.shape
    Hk = kv.shape[2]
    mid = torch.full((B, Hq, num_splits, D + 1), float("nan"), dtype=torch.float32)
    ref.soa_dec._tq_decode_stage1[(B, Hq, num_splits)](
        query, kv, kv.view(torch.uint16), bt, seq_lens, cents, mid, None,
        query.stride(0), query.stride(1), kv.stride(0), bt.stride(0),
        mid.stride(0), mid.stride(1), mid.stride(2),
        NUM_KV_HEADS=Hk, HEAD_DIM=D, BLOCK_SIZE=BLOCK_SIZE,
        NUM_KV_SPLITS=num_splits, KV_GROUP_SIZE=Hq // Hk,
        MSE_BITS=MSE_BITS, MSE_BYTES=MSE_BYTES, VQB=VALUE_BITS,
        VAL_DATA_BYTES=VAL_BYTES, KEY_DATA_BYTES=HEAD_DIM,
        META_REGION_OFFSET=BLOCK_SIZE * Hk * (HEAD_DIM + VAL_BYTES), NUM_SOA_FIELDS=2,
        SOA_K_NORM=0, SOA_V_SCALE=0, SOA_V_ZERO=1,
        ATTN_SCALE=1.0 / math.sqrt(D), BLOCK_D=triton.next_power_of_2(D),
        BLOCK_KV=4, KEY_FP8=1, NORM_CORRECTION=0, FP8_E4B15=0, USE_SINKS=0,
        num_warps=1, num_stages=1,
    )
    return mid


def build_k8_case(ref: Ref, name, *, seed, seq_lens, hq, hk, num_splits, pool_blocks):
    """turboquant_k8v4: fp16 keys cast to e4m3 by the reference FP8 store
    (``reference/soa_store.py:125-221``), 4-bit values, then the reference
    SoA Stage1 with ``KEY_FP8=1`` on the fp16 query (no rotation) and
    Stage2."""
    t0 = time.time()
    B = len(seq_lens)
    g = torch.Generator().manual_seed(seed)
    pages = [max(1, math.ceil(L / BLOCK_SIZE)) for L in seq_lens]
    perm = torch.randperm(pool_blocks, generator=g)
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]].to(torch.int32)
        k += pages[b]
    slot = HEAD_DIM + VAL_BYTES + 4  # 196: fp8 key, 4-bit value, v-scale, v-zero
    kv = torch.randint(0, 256, (pool_blocks, BLOCK_SIZE, hk, slot), generator=g, dtype=torch.uint8)
    ntok = sum(seq_lens)
    # keys spread over the e4m3 range (a few beyond 448 saturate), fp16 inputs
    key = (torch.randn(ntok, hk, HEAD_DIM, generator=g) * 3.0).to(torch.float16)
    key[0, 0, :8] = torch.tensor([500.0, -600.0, 448.0, 0.001, -0.0001, 17.0, 19.0, 0.0])
    val = torch.randn(ntok, hk, HEAD_DIM, generator=g).to(torch.float16)
    slots = []
    for b in range(B):
        for t in range(seq_lens[b]):
            slots.append(int(bt[b, t // BLOCK_SIZE]) * BLOCK_SIZE + t % BLOCK_SIZE)
    slot_mapping = torch.tensor(slots, dtype=torch.int32)
    before = kv.clone()
    cents = ref.centroids_mod.get_centroids(HEAD_DIM, MSE_BITS).to(torch.float32)
    mids = ((cents[:-1] + cents[1:]) * 0.5).contiguous()
    ref.soa_store.triton_turboquant_store(
        key, val, kv, slot_mapping, torch.eye(HEAD_DIM), mids, MSE_BITS, HEAD_DIM, VALUE_BITS,
        key_fp8=True)
    query = (torch.randn(B, hq, HEAD_DIM, generator=g) * 0.5).to(torch.float16)
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    print(f"[{name}] store done {time.time() - t0:.1f}s", flush=True)
    mid = run_soa_k8(ref, query, kv, bt, sl, cents, num_splits)
    print(f"[{name}] SoA K8 Stage1 done {time.time() - t0:.1f}s", flush=True)
    o2, l2 = run_stage2(ref, mid, sl)
    save(name, dict(key=key.float(), value=val.float(), slot_mapping=slot_mapping, cache_before=before,
                    kv_cache=kv, block_table=bt, seq_lens=sl, query=query.float(),
                    num_splits=np.int32(num_splits), mid_o=mid, out_stage2=o2, lse_stage2=l2))


def build_k3_case(ref: Ref, name, *, seed, seq_lens, hq, hk, num_splits, pool_blocks, vbits=VALUE_BITS):
    """turboquant_k3v4_nc: 3-bit Lloyd-Max keys (48 bytes, dim d at bit 3d),
    4-bit values, norm correction; the reference SoA store with mse_bits=3
    (``reference/soa_store.py:305-345``) and the reference SoA Stage1 with
    MSE_BITS=3.  Also saves the store kernel's inputs as the reference
    launcher computes them (``reference/soa_store.py:482-487``).  ``vbits=3``
    is ``turboquant_3bit_nc``: 3-bit values too (48 bytes, same packing)."""
    t0 = time.time()
    bits, mse_bytes = 3, HEAD_DIM * 3 // 8
    vbytes = HEAD_DIM * vbits // 8
    B = len(seq_lens)
    g = torch.Generator().manual_seed(seed)
    pages = [max(1, math.ceil(L / BLOCK_SIZE)) for L in seq_lens]
    perm = torch.randperm(pool_blocks, generator=g)
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]].to(torch.int32)
        k += pages[b]
    R = orthogonal(seed + 1)
    cents = ref.centroids_mod.get_centroids(HEAD_DIM, bits).to(torch.float32)
    mids = ((cents[:-1] + cents[1:]) * 0.5).contiguous()
    slot = mse_bytes + vbytes + 6  # 118 (4-bit values) or 102 (3-bit)
    kv = torch.randint(0, 256, (pool_blocks, BLOCK_SIZE, hk, slot), generator=g, dtype=torch.uint8)
    ntok = sum(seq_lens)
    key = torch.randn(ntok, hk, HEAD_DIM, generator=g, dtype=torch.float32)
    val = torch.randn(ntok, hk, HEAD_DIM, generator=g, dtype=torch.float32)
    slots = []
    for b in range(B):
        for t in range(seq_lens[b]):
            slots.append(int(bt[b, t // BLOCK_SIZE]) * BLOCK_SIZE + t % BLOCK_SIZE)
    slot_mapping = torch.tensor(slots, dtype=torch.int32)
    before = kv.clone()
    ref.soa_store.triton_turboquant_store(
        key, val, kv, slot_mapping, R, mids, bits, mse_bytes + 2, vbits,
        key_fp8=False, centroids=cents, norm_correction=True)
    k_flat = key.float().reshape(ntok * hk, HEAD_DIM)
    norms = k_flat.norm(dim=1, keepdim=True)
    y = (k_flat / (norms + 1e-8)) @ R
    q = torch.randn(B, hq, HEAD_DIM, generator=g, dtype=torch.float32)
    q_rot = (q @ R).contiguous()
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    print(f"[{name}] store done {time.time() - t0:.1f}s", flush=True)
    mid = torch.full((B, hq, num_splits, HEAD_DIM + 1), float("nan"), dtype=torch.float32)
    ref.soa_dec._tq_decode_stage1[(B, hq, num_splits)](
        q_rot, kv, kv.view(torch.uint16), bt, sl, cents, mid, None,
        q_rot.stride(0), q_rot.stride(1), kv.stride(0), bt.stride(0),
        mid.stride(0), mid.stride(1), mid.stride(2),
        NUM_KV_HEADS=hk, HEAD_DIM=HEAD_DIM, BLOCK_SIZE=BLOCK_SIZE,
        NUM_KV_SPLITS=num_splits, KV_GROUP_SIZE=hq // hk,
        MSE_BITS=bits, MSE_BYTES=mse_bytes, VQB=vbits,
        VAL_DATA_BYTES=vbytes, KEY_DATA_BYTES=mse_bytes,
        META_REGION_OFFSET=BLOCK_SIZE * hk * (mse_bytes + vbytes), NUM_SOA_FIELDS=3,
        SOA_K_NORM=0, SOA_V_SCALE=1, SOA_V_ZERO=2,
        ATTN_SCALE=1.0 / math.sqrt(HEAD_DIM), BLOCK_D=triton.next_power_of_2(HEAD_DIM),
        BLOCK_KV=4, KEY_FP8=0, NORM_CORRECTION=1, FP8_E4B15=0, USE_SINKS=0,
        num_warps=1, num_stages=1,
    )
    print(f"[{name}] SoA K3 Stage1 done {time.time() - t0:.1f}s", flush=True)
    o2, l2 = run_stage2(ref, mid, sl)
    save(name, dict(y=y, norms=norms.squeeze(1), value=val.reshape(ntok * hk, HEAD_DIM), rotation=R,
                    slot_mapping=slot_mapping, cache_before=before, kv_cache=kv, centroids=cents,
                    midpoints=mids, block_table=bt, seq_lens=sl, q_rot=q_rot,
                    num_splits=np.int32(num_splits), mid_o=mid, out_stage2=o2, lse_stage2=l2))


def build_aos_preset_case(ref: Ref, name, *, preset, seed, seq_lens, hq, hk, num_splits, pool_blocks):
    """AoS forms of the FP8-key and 3-bit presets: the reference AoS store
    (``reference/aos_store.py:145-219`` FP8, ``:221-340`` MSE with
    MSE_BITS=3, values ``:26-116``; slot = [key codes | raw fp16 norm (MSE
    keys) | value codes | vscale | vzero]) and the reference AoS V1 Stage1
    (``reference/aos_decode.py:43-313``) with KEY_FP8=1 (``preset="k8"``, the
    fp16 query unrotated) or MSE_BITS=3 and VQB=4 / 3 (``"k3"`` / ``"k3v3"``,
    NORM_CORRECTION=1), then Stage2.  The 3-bit cases also save the store
    kernel's inputs as the reference launcher computes them
    (``reference/aos_store.py:425-429``)."""
    t0 = time.time()
    fp8 = preset == "k8"
    bits = 4 if fp8 else 3
    vbits = 3 if preset == "k3v3" else 4
    kbytes = HEAD_DIM if fp8 else HEAD_DIM * 3 // 8
    kps = kbytes if fp8 else kbytes + 2
    vbytes = HEAD_DIM * vbits // 8
    slot = kps + vbytes + 4  # 196, 118 or 102
    B = len(seq_lens)
    g = torch.Generator().manual_seed(seed)
    pages = [max(1, math.ceil(L / BLOCK_SIZE)) for L in seq_lens]
    perm = torch.randperm(pool_blocks, generator=g)
    bt = torch.zeros(B, max(pages), dtype=torch.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]].to(torch.int32)
        k += pages[b]
    kv = torch.randint(0, 256, (pool_blocks, BLOCK_SIZE, hk, slot), generator=g, dtype=torch.uint8)
    ntok = sum(seq_lens)
    slots = []
    for b in range(B):
        for t in range(seq_lens[b]):
            slots.append(int(bt[b, t // BLOCK_SIZE]) * BLOCK_SIZE + t % BLOCK_SIZE)
    slot_mapping = torch.tensor(slots, dtype=torch.int32)
    before = kv.clone()
    cents = ref.centroids_mod.get_centroids(HEAD_DIM, bits).to(torch.float32)
    mids = ((cents[:-1] + cents[1:]) * 0.5).contiguous()
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    extra = {}
    if fp8:
        key = (torch.randn(ntok, hk, HEAD_DIM, generator=g) * 3.0).to(torch.float16)
        val = torch.randn(ntok, hk, HEAD_DIM, generator=g).to(torch.float16)
        ref.aos_store.triton_turboquant_store(key, val, kv, slot_mapping, torch.eye(HEAD_DIM), mids, bits, kps,
                                              vbits, key_fp8=True)
        q = (torch.randn(B, hq, HEAD_DIM, generator=g) * 0.5).to(torch.float16).float()
        extra.update(key=key.float(), value=val.float(), query=q)
    else:
        R = orthogonal(seed + 1)
        key = torch.randn(ntok, hk, HEAD_DIM, generator=g, dtype=torch.float32)
        val = torch.randn(ntok, hk, HEAD_DIM, generator=g, dtype=torch.float32)
        ref.aos_store.triton_turboquant_store(key, val, kv, slot_mapping, R, mids, bits, kps, vbits)
        k_flat = key.reshape(ntok * hk, HEAD_DIM)
        norms = k_flat.norm(dim=1, keepdim=True)
        y = (k_flat / (norms + 1e-8)) @ R
        q = (torch.randn(B, hq, HEAD_DIM, generator=g, dtype=torch.float32) @ R).contiguous()
        extra.update(y=y, norms=norms.squeeze(1), value=val.reshape(ntok * hk, HEAD_DIM), rotation=R, q_rot=q)
    print(f"[{name}] AoS store done {time.time() - t0:.1f}s", flush=True)
    mid = torch.full((B, hq, num_splits, HEAD_DIM + 1), float("nan"), dtype=torch.float32)
    ref.aos_dec._tq_decode_stage1[(B, hq, num_splits)](
        q, kv, bt, sl, cents, mid,
        q.stride(0), q.stride(1), kv.stride(0), kv.stride(1), kv.stride(2),
        bt.stride(0), mid.stride(0), mid.stride(1), mid.stride(2),
        NUM_KV_HEADS=hk, HEAD_DIM=HEAD_DIM, BLOCK_SIZE=BLOCK_SIZE,
        NUM_KV_SPLITS=num_splits, KV_GROUP_SIZE=hq // hk,
        MSE_BITS=bits, MSE_BYTES=HEAD_DIM * bits // 8, KPS=kps, VQB=vbits,
        VAL_DATA_BYTES=vbytes, ATTN_SCALE=1.0 / math.sqrt(HEAD_DIM),
        BLOCK_D=triton.next_power_of_2(HEAD_DIM), BLOCK_KV=4, KEY_FP8=1 if fp8 else 0,
        NORM_CORRECTION=0 if fp8 else 1, FP8_E4B15=0, num_warps=1, num_stages=1,
    )
    print(f"[{name}] AoS V1 Stage1 done {time.time() - t0:.1f}s", flush=True)
    o2, l2 = run_stage2(ref, mid, sl)
    save(name, dict(slot_mapping=slot_mapping, cache_before=before, kv_cache=kv, centroids=cents,
                    midpoints=mids, block_table=bt, seq_lens=sl, num_splits=np.int32(num_splits),
                    mid_o=mid, out_stage2=o2, lse_stage2=l2, **extra))


def run_aos_v1(ref: Ref, q_rot, kv, bt, seq_lens, cents, num_splits):
    B, Hq, D = q_rot.shape
    Hk = kv.shape[2]
    mid = torch.full((B, Hq, num_splits, D + 1), float("nan"), dtype=torch.float32)
    ref.aos_dec._tq_decode_stage1[(B, Hq, num_splits)](
        q_rot, kv, bt, seq_lens, cents, mid,
        q_rot.stride(0), q_rot.stride(1), kv.stride(0), kv.stride(1), kv.stride(2),
        bt.stride(0), mid.stride(0), mid.stride(1), mid.stride(2),
        NUM_KV_HEADS=Hk, HEAD_DIM=D, BLOCK_SIZE=BLOCK_SIZE,
        NUM_KV_SPLITS=num_splits, KV_GROUP_SIZE=Hq // Hk,
        MSE_BITS=MSE_BITS, MSE_BYTES=MSE_BYTES, KPS=AOS_KPS, VQB=VALUE_BITS,
        VAL_DATA_BYTES=VAL_BYTES, ATTN_SCALE=1.0 / math.sqrt(D),
        BLOCK_D=triton.next_power_of_2(D), BLOCK_KV=4, KEY_FP8=0,
        NORM_CORRECTION=1, FP8_E4B15=0, num_warps=1, num_stages=1,
    )
    return mid


def run_v2(ref: Ref, q_rot, kv, bt, seq_lens, cents, num_splits):
    B, Hq, D = q_rot.shape
    Hk = kv.shape[2]
    G = Hq // Hk
    pair_lut = ref.common.build_pair_lut(cents)
    mid = torch.full((B, Hq, num_splits, D + 1), float("nan"), dtype=torch.float32)
    ref.v2.tq4_decode_stage1_v2[(B, Hk, num_splits)](
        q_rot, kv, kv.view(torch.uint16), bt, seq_lens, cents, pair_lut, mid,
        q_rot.stride(0), q_rot.stride(1), kv.stride(0), bt.stride(0),
        mid.stride(0), mid.stride(1), mid.stride(2),
        NUM_Q_HEADS=Hq, NUM_KV_HEADS=Hk, HEAD_DIM=D, BLOCK_SIZE=BLOCK_SIZE,
        PADDED_SLOT=kv.shape[3], MAX_NUM_BLOCKS=bt.shape[1],
        NUM_KV_SPLITS=num_splits, KV_GROUP_SIZE=G,
        MSE_BITS=MSE_BITS, MSE_BYTES=MSE_BYTES, VQB=VALUE_BITS,
        VAL_DATA_BYTES=VAL_BYTES, KEY_DATA_BYTES=MSE_BYTES,
        META_REGION_OFFSET=soa_meta_offset(Hk), NUM_SOA_FIELDS=3,
        SOA_K_NORM=0, SOA_V_SCALE=1, SOA_V_ZERO=2, N_CENTROIDS=16,
        ATTN_SCALE=1.0 / math.sqrt(D), BLOCK_D=triton.next_power_of_2(D),
        TILE_SIZE=16, BLOCK_M=max(16, triton.next_power_of_2(G)),
        KEY_FP8=0, NORM_CORRECTION=1, FP8_E4B15=0, USE_PAIR_LUT=1,
        USE_BF16_DOT=0, num_warps=4, num_stages=2,
    )
    return mid, pair_lut


def run_stage2(ref: Ref, mid, seq_lens):
    B, Hq, S, D1 = mid.shape
    out = torch.full((B, Hq, D1 - 1), float("nan"), dtype=torch.float32)
    lse = torch.full((B, Hq), float("nan"), dtype=torch.float32)
    ref.stage2.tq4_stage2_kernel[(B, Hq)](
        mid, out, lse, seq_lens,
        mid.stride(0), mid.stride(1), mid.stride(2),
        out.stride(0), out.stride(1), lse.stride(0),
        NUM_SPLITS=S, BLOCK_D=triton.next_power_of_2(D1 - 1), D=D1 - 1,
        num_warps=4, num_stages=2,
    )
    return out, lse


# ---------------------------------------------------------------------------
# Seeded inputs
# ---------------------------------------------------------------------------


def orthogonal(seed: int, d: int = HEAD_DIM) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(d, d, generator=g, dtype=torch.float64)
    q, r = torch.linalg.qr(a)
    q = q * torch.sign(torch.diagonal(r))[None, :]
    return q.to(torch.float32).contiguous()


def build_case(ref: Ref, name, *, seed, seq_lens, hq, hk, num_splits,
               pool_blocks, aos=True, v2=True, sinks=False):
    """Store seeded K/V with the reference SoA (and AoS) store, then run the
    reference Stage1 kernels and Stage2 on the result.  ``sinks=True`` adds a
    run of the SoA Stage1 with per-head sink logits (``USE_SINKS=1``,
    ``reference/soa_decode_v1.py:134-145``) and its Stage2."""
    t0 = time.time()
    B = len(seq_lens)
    g = torch.Generator().manual_seed(seed)
    pages = [max(1, math.ceil(L / BLOCK_SIZE)) for L in seq_lens]
    max_pages = max(pages)
    assert sum(pages) <= pool_blocks
    perm = torch.randperm(pool_blocks, generator=g)
    bt = torch.zeros(B, max_pages, dtype=torch.int32)
    k = 0
    for b in range(B):
        bt[b, : pages[b]] = perm[k : k + pages[b]].to(torch.int32)
        k += pages[b]
    # Unused table entries point at a block that exists; the kernels never
    # read them for in-range tokens.
    R = orthogonal(seed + 1)
    cents = ref.centroids_mod.get_centroids(HEAD_DIM, MSE_BITS).to(torch.float32)
    mids = ((cents[:-1] + cents[1:]) * 0.5).contiguous()

    # Cache starts as seeded garbage: tokens past seq_len keep random bytes
    # (random fp16 metadata included), which the decoders must mask.
    kv_soa = torch.randint(0, 256, (pool_blocks, BLOCK_SIZE, hk, SLOT),
                           generator=g, dtype=torch.uint8)
    kv_aos = kv_soa.clone()
    ntok = sum(seq_lens)
    key = torch.randn(ntok, hk, HEAD_DIM, generator=g, dtype=torch.float32)
    val = torch.randn(ntok, hk, HEAD_DIM, generator=g, dtype=torch.float32)
    slots = []
    for b in range(B):
        for t in range(seq_lens[b]):
            slots.append(int(bt[b, t // BLOCK_SIZE]) * BLOCK_SIZE + t % BLOCK_SIZE)
    slot_mapping = torch.tensor(slots, dtype=torch.int32)
    ref.soa_store.triton_turboquant_store(
        key, val, kv_soa, slot_mapping, R, mids, MSE_BITS, AOS_KPS, VALUE_BITS,
        key_fp8=False, centroids=cents, norm_correction=True)
    if aos:
        ref.aos_store.triton_turboquant_store(
            key, val, kv_aos, slot_mapping, R, mids, MSE_BITS, AOS_KPS, VALUE_BITS,
            key_fp8=False)
    q = torch.randn(B, hq, HEAD_DIM, generator=g, dtype=torch.float32)
    q_rot = (q @ R).contiguous()
    sl = torch.tensor(seq_lens, dtype=torch.int32)
    print(f"[{name}] store done {time.time() - t0:.1f}s", flush=True)

    out = dict(q_rot=q_rot, rotation=R, kv_cache=kv_soa, block_table=bt,
               seq_lens=sl, centroids=cents, midpoints=mids,
               num_splits=np.int32(num_splits))
    mid_v1 = run_soa_v1(ref, q_rot, kv_soa, bt, sl, cents, num_splits)
    out["mid_o_soa_v1"] = mid_v1
    print(f"[{name}] SoA V1 done {time.time() - t0:.1f}s", flush=True)
    o2, l2 = run_stage2(ref, mid_v1, sl)
    out["out_stage2"], out["lse_stage2"] = o2, l2
    if sinks:
        # one head without a sink (-inf), one whose sink dominates its scores
        sk = torch.randn(hq, generator=g, dtype=torch.float32) * 2.0
        sk[0] = float("-inf")
        sk[1] = 12.0
        mid_s = run_soa_v1(ref, q_rot, kv_soa, bt, sl, cents, num_splits, sinks=sk)
        out["sinks"], out["mid_o_soa_v1_sinks"] = sk, mid_s
        out["out_stage2_sinks"], out["lse_stage2_sinks"] = run_stage2(ref, mid_s, sl)
        print(f"[{name}] SoA V1 with sinks done {time.time() - t0:.1f}s", flush=True)
    if aos:
        out["kv_cache_aos"] = kv_aos
        out["mid_o_aos_v1"] = run_aos_v1(ref, q_rot, kv_aos, bt, sl, cents, num_splits)
        print(f"[{name}] AoS V1 done {time.time() - t0:.1f}s", flush=True)
    if v2:
        mid_v2, lut = run_v2(ref, q_rot, kv_soa, bt, sl, cents, num_splits)
        out["mid_o_v2"], out["pair_lut"] = mid_v2, lut
        print(f"[{name}] V2 done {time.time() - t0:.1f}s", flush=True)
    save(name, out)


def build_store_case(ref: Ref, name, *, seed, ntok, hk, pool_blocks):
    """Bit-exactness fixture for the store: the kernel inputs the reference
    store computes on the host (rotated unit keys ``y``, key norms, values)
    and the bytes its kernel writes, for both layouts."""
    g = torch.Generator().manual_seed(seed)
    R = orthogonal(seed + 1)
    cents = ref.centroids_mod.get_centroids(HEAD_DIM, MSE_BITS).to(torch.float32)
    mids = ((cents[:-1] + cents[1:]) * 0.5).contiguous()
    key = torch.randn(ntok, hk, HEAD_DIM, generator=g, dtype=torch.float32)
    val = torch.randn(ntok, hk, HEAD_DIM, generator=g, dtype=torch.float32)
    # A few rows that hit the edge cases of the value quantiser: constant
    # rows (scale clamps to 1e-8) and rows with large dynamic range.
    val[0, 0, :] = 0.25
    val[1, 0, :] = -3.0
    val[2, 0, ::2] *= 1000.0
    key[3, 0, :] = 0.0  # zero key: norm 0, every code from y == 0
    slots = torch.randperm(pool_blocks * BLOCK_SIZE, generator=g)[:ntok].to(torch.int32)
    slots[-1] = -1  # padding token: skipped by the store
    kv_soa = torch.randint(0, 256, (pool_blocks, BLOCK_SIZE, hk, SLOT),
                           generator=g, dtype=torch.uint8)
    kv_aos = kv_soa.clone()
    before = kv_soa.clone()
    ref.soa_store.triton_turboquant_store(
        key, val, kv_soa, slots, R, mids, MSE_BITS, AOS_KPS, VALUE_BITS,
        key_fp8=False, centroids=cents, norm_correction=True)
    ref.aos_store.triton_turboquant_store(
        key, val, kv_aos, slots, R, mids, MSE_BITS, AOS_KPS, VALUE_BITS,
        key_fp8=False)
    # Host-side part of the reference launcher, kept verbatim in meaning
    # (reference/soa_store.py:482-487) so the fixture pins the kernel inputs.
    k_flat = key.float().reshape(ntok * hk, HEAD_DIM)
    norms = k_flat.norm(dim=1, keepdim=True)
    y = (k_flat / (norms + 1e-8)) @ R
    save(name, dict(key=key, value=val, rotation=R, y=y, norms=norms.squeeze(1),
                    slot_mapping=slots,
                    centroids=cents, midpoints=mids, cache_before=before,
                    kv_cache_soa=kv_soa, kv_cache_aos=kv_aos))


def save(name, d):
    arrs = {}
    for k, v in d.items():
        arrs[k] = v.numpy() if isinstance(v, torch.Tensor) else np.asarray(v)
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, **arrs)
    print(f"wrote {path} ({path.stat().st_size} bytes)", flush=True)


CASES = {
    # B2 x 256, 32/8 heads, 4 splits, shuffled pool.
    "c0": dict(seed=20261201, seq_lens=[256, 256], hq=32, hk=8, num_splits=4,
               pool_blocks=32),
    # Ragged: an empty-split sequence, a 45-token sequence with splits that
    # start mid-page, a 130-token sequence ending one token into a page.
    "ragged_gqa4": dict(seed=7, seq_lens=[1, 45, 130], hq=32, hk=8, num_splits=4,
                        pool_blocks=16),
    # GQA-8 with one KV head per GPU (the TP-by-head shard of config 3).
    "ragged_gqa8_hk1": dict(seed=11, seq_lens=[77, 300], hq=8, hk=1, num_splits=5,
                            pool_blocks=32),
    # GQA-8 with two KV heads and uneven splits.
    "ragged_gqa8_hk2": dict(seed=13, seq_lens=[160, 33], hq=16, hk=2, num_splits=3,
                            pool_blocks=16, aos=False),
    # Attention sinks (per-head logits folded into split 0), ragged lengths.
    "sinks_gqa4": dict(seed=17, seq_lens=[1, 45, 130], hq=16, hk=4, num_splits=4,
                       pool_blocks=16, aos=False, v2=False, sinks=True),
}


def main(argv):
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = Ref()
    aos_presets = {"aos_k8v4_ragged": ("k8", 41), "aos_k3v4_ragged": ("k3", 43), "aos_k3v3_ragged": ("k3v3", 47)}
    wanted = argv or list(CASES) + ["store", "k8v4_ragged", "k3v4_ragged", "k3v3_ragged"] + list(aos_presets)
    for name in wanted:
        if name in aos_presets:
            # AoS forms of the presets: ragged lengths (an empty-split
            # sequence, splits starting mid-page), GQA-4
            build_aos_preset_case(ref, name, preset=aos_presets[name][0], seed=aos_presets[name][1],
                                  seq_lens=[1, 45, 130], hq=16, hk=4, num_splits=4, pool_blocks=16)
        elif name == "store":
            build_store_case(ref, "store_small", seed=99, ntok=48, hk=4, pool_blocks=5)
        elif name == "k3v4_ragged":
            # 3-bit keys, 4-bit values: ragged lengths, GQA-4
            build_k3_case(ref, name, seed=29, seq_lens=[1, 45, 130], hq=16, hk=4, num_splits=4,
                          pool_blocks=16)
        elif name == "k3v3_ragged":
            # 3-bit keys and 3-bit values (turboquant_3bit_nc), GQA-4
            build_k3_case(ref, name, seed=37, seq_lens=[1, 45, 130], hq=16, hk=4, num_splits=4,
                          pool_blocks=16, vbits=3)
        elif name == "k8v4_ragged":
            # FP8-key preset: ragged lengths (an empty-split sequence, splits
            # starting mid-page), GQA-4
            build_k8_case(ref, name, seed=23, seq_lens=[1, 45, 130], hq=16, hk=4, num_splits=4,
                          pool_blocks=16)
        else:
            build_case(ref, name, **CASES[name])


if __name__ == "__main__":
    main(sys.argv[1:])
