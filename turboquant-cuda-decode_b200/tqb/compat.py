"""Drop-in entry points with the reference's names and argument meaning.

Each function here replaces a launcher of zben777/turboquant-cuda-decode and
routes to the sm_100a kernels of ``libtqb.so`` (via ``tqb.ops``):

=============================================  =========================================
this module                                    reference
=============================================  =========================================
``launch_soa_v1_stage1``                       baseline/triton_v1.py:145-203
``launch_aos_v1_stage1``                       baseline/triton_v1.py:90-142
``launch_tq4_v2_stage1``                       baseline/triton_v2.py:569-706
``launch_stage2``                              baseline/stage2.py:58-81
``tq4_cuda_stage1`` / ``_stage2`` / ``_full``  cuda/tq4_cuda_v7_bind.cpp:14-21 (pybind)
``triton_turboquant_decode_attention``         reference/soa_decode_v1.py:485-643
``triton_turboquant_store``                    reference/soa_store.py:381-524 (SoA),
                                               reference/aos_store.py:350-447 (AoS)
``convert_soa_to_aos_kv_cache``                baseline/common.py:554-672
=============================================  =========================================

Differences, all widenings: the reference harness launchers assert the fixed
Qwen3-4B shapes (B64, Hq32/Hk8, 32 splits) while these accept any batch, any
GQA group up to 8 and any split count (taken from ``mid_o.shape[2]``), plus
optional per-sequence split counts.  Shape errors raise ``TqbError``
(a ``RuntimeError``) instead of ``AssertionError``.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

from . import ops
from .codebook import build_pair_lut, get_centroids  # noqa: F401  (re-exported)
from .layout import (
    BLOCK_SIZE,
    DATA_BYTES_PER_SLOT,
    HEAD_DIM,
    MSE_BYTES,
    NUM_SOA_FIELDS,
    SOA_K_NORM,
    SOA_V_SCALE,
    SOA_V_ZERO,
    VAL_DATA_BYTES,
    meta_region_offset,
)

NUM_KV_SPLITS = 32  # default split count of the reference harness (baseline/common.py:53)


def launch_soa_v1_stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o) -> None:
    """Stage1 on the SoA cache; split count = ``mid_o.shape[2]``."""
    ops.stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o, layout="soa")


def launch_aos_v1_stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o) -> None:
    """Stage1 on the AoS cache (norm correction applied while decoding)."""
    ops.stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o, layout="aos")


def launch_tq4_v2_stage1(q_rot, kv_cache, block_table, seq_lens, centroids, pair_lut,
                         mid_o: Optional[torch.Tensor] = None,
                         num_splits: int = NUM_KV_SPLITS) -> torch.Tensor:
    """V2-style launcher: same inputs (``pair_lut`` accepted and checked but
    not needed), allocates ``mid_o [B, Hq, num_splits, D+1]`` when omitted,
    returns it."""
    if pair_lut is not None and tuple(pair_lut.shape) != (256, 2):
        raise ops.TqbError(ops._lib.TQB_ERR_INVALID_ARG, "pair_lut must be [256, 2]")
    if mid_o is None:
        B, Hq, D = q_rot.shape
        mid_o = torch.empty(B, Hq, num_splits, D + 1, dtype=torch.float32, device=q_rot.device)
    ops.stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o, layout="soa",
               pair_lut=pair_lut)
    return mid_o


def launch_stage2(mid_o, seq_lens, output, lse) -> None:
    ops.stage2(mid_o, seq_lens, output, lse)


def tq4_cuda_stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o) -> torch.Tensor:
    """pybind-style Stage1 entry (returns ``mid_o``)."""
    ops.stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o, layout="soa")
    return mid_o


def tq4_cuda_stage2(mid_o, output, lse, seq_lens: Optional[torch.Tensor] = None) -> torch.Tensor:
    """pybind-style Stage2.  The reference CUDA Stage2 merges all splits
    without a seq_lens argument (cuda/tq4_cuda_v7.cu:11-52), which is only
    correct when no split is empty; pass ``seq_lens`` to skip empty splits
    as baseline/stage2.py does.  Without it every split counts as non-empty
    (seq_len taken as a multiple of the split count)."""
    if seq_lens is None:
        B, Hq, S, _ = mid_o.shape
        seq_lens = torch.full((B,), S, dtype=torch.int32, device=mid_o.device)
    ops.stage2(mid_o, seq_lens, output, lse)
    return output


def tq4_cuda_full(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o, output, lse) -> torch.Tensor:
    """Stage1 + Stage2 on the same stream."""
    ops.stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o, layout="soa")
    ops.stage2(mid_o, seq_lens, output, lse)
    return output


def triton_turboquant_decode_attention(
    query: torch.Tensor,
    kv_cache: torch.Tensor,
    block_table: torch.Tensor,
    seq_lens: torch.Tensor,
    Pi: torch.Tensor,
    centroids: torch.Tensor,
    scale: float,
    mse_bits: int,
    key_packed_size: int,
    value_quant_bits: int,
    key_fp8: bool = False,
    norm_correction: bool = False,
    PiT: Optional[torch.Tensor] = None,
    mid_o_buf: Optional[torch.Tensor] = None,
    output_buf: Optional[torch.Tensor] = None,
    lse_buf: Optional[torch.Tensor] = None,
    buf_holder: Any = None,
    max_num_kv_splits: int = 32,
    sinks: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Production decode (q rotation, Stage1, Stage2) for the
    ``turboquant_4bit_nc`` preset; returns ``[B, Hq, D]`` in query's dtype.
    ``sinks`` ([Hq] per-head sink logits, cast to float32) enters split 0 of
    every sequence as the reference's ``USE_SINKS`` does
    (reference/soa_decode_v1.py:134-145, 565-605).  FP8 keys and 3-bit codes
    are other presets of the reference and raise ``NotImplementedError``.
    ``key_fp8=True`` is the ``turboquant_k8v4`` preset: e4m3 keys, 4-bit
    values, the query used unrotated (reference/soa_decode_v1.py:532-533);
    ``mse_bits=3`` the ``turboquant_k3v4_nc`` preset (3-bit keys, 8
    centroids), with ``value_quant_bits=3`` too ``turboquant_3bit_nc``."""
    layout = _preset_layout(key_fp8, mse_bits, value_quant_bits)
    return decode_attention(query, kv_cache, block_table, seq_lens, Pi, centroids, scale, layout, PiT=PiT,
                            mid_o_buf=mid_o_buf, output_buf=output_buf, lse_buf=lse_buf, buf_holder=buf_holder,
                            max_num_kv_splits=max_num_kv_splits, sinks=sinks)


def _preset_layout(key_fp8: bool, mse_bits: int, value_quant_bits: int, family: str = "soa") -> str:
    """Cache layout of a TurboQuant preset (reference/config.py:20-41) in the
    SoA or AoS ``family``."""
    if key_fp8 and value_quant_bits == 4:
        suffix = "_k8"         # turboquant_k8v4
    elif not key_fp8 and mse_bits == 4 and value_quant_bits == 4:
        suffix = ""            # turboquant_4bit_nc
    elif not key_fp8 and mse_bits == 3 and value_quant_bits == 4:
        suffix = "_k3"         # turboquant_k3v4_nc
    elif not key_fp8 and mse_bits == 3 and value_quant_bits == 3:
        suffix = "_k3v3"       # turboquant_3bit_nc
    else:
        raise NotImplementedError(f"no TurboQuant preset with key_fp8={key_fp8}, mse_bits={mse_bits}, "
                                  f"value_quant_bits={value_quant_bits}")
    return family + suffix


def decode_attention(query, kv_cache, block_table, seq_lens, Pi, centroids, scale, layout, *, PiT=None,
                     mid_o_buf=None, output_buf=None, lse_buf=None, buf_holder=None,
                     max_num_kv_splits: int = 32, sinks=None) -> torch.Tensor:
    """Query rotation, Stage1 on the ``layout`` ("soa"/"aos"/"soa_k8") cache (with the
    optional attention ``sinks`` folded into split 0), Stage2; the body of
    both reference launchers (reference/soa_decode_v1.py:486-643,
    reference/aos_decode.py:486-...) with the buffer reuse they offer."""
    B, Hq, D = query.shape
    fused = None  # (query, rotation) rotated inside the Stage1 launch
    if layout in ("soa_k8", "k8v4", "aos_k8"):
        # FP8 keys score against the query itself, read as fp32
        # (reference/soa_decode_v1.py:532-533)
        q_rot = query.float().contiguous()
    else:
        if PiT is None:
            PiT = Pi.T.contiguous()
        if query.dtype in (torch.float32, torch.float16, torch.bfloat16):
            # q_rot = query.float() @ PiT (reference/soa_decode_v1.py:535-538)
            # computed by Stage1 itself (tqb_stage1_rotated: one kernel on the
            # page ring, else the fused cast + rotation kernel first)
            q_rot = torch.empty(B, Hq, D, dtype=torch.float32, device=query.device)
            fused = (query if query.stride(2) == 1 else query.contiguous(), PiT.float().contiguous())
        else:
            q_rot = (query.float() @ PiT).contiguous()
    S = max_num_kv_splits
    if mid_o_buf is not None and mid_o_buf.shape[0] >= B and mid_o_buf.shape[2] >= S:
        mid_o = mid_o_buf[:B, :Hq, :S, :]
    else:
        mid_o = torch.empty(B, Hq, S, D + 1, dtype=torch.float32, device=query.device)
        if buf_holder is not None:
            buf_holder._tq_mid_o_buf = mid_o
    if sinks is not None:
        sinks = sinks.to(device=query.device, dtype=torch.float32).contiguous()
    ops.stage1(q_rot, kv_cache, block_table, seq_lens, centroids, mid_o, layout=layout,
               attn_scale=scale, sinks=sinks, query=None if fused is None else fused[0],
               rotation=None if fused is None else fused[1])
    if output_buf is not None and output_buf.shape[0] >= B:
        # the caller's workspace, in its own dtype (vLLM hands it out in the
        # query's dtype, reference/turboquant_attn.py:1133-1141); Stage2
        # writes float32, float16 or bfloat16 directly
        output = output_buf[:B, :Hq, :D]
    elif query.dtype in (torch.float16, torch.bfloat16):
        # Stage2 writes the query's dtype directly (the reference merges into
        # fp32 and then casts: reference/soa_decode_v1.py:643; same rounding)
        output = torch.empty(B, Hq, D, dtype=query.dtype, device=query.device)
    else:
        output = torch.empty(B, Hq, D, dtype=torch.float32, device=query.device)
        if buf_holder is not None:
            buf_holder._tq_output_buf = output
    if lse_buf is not None and lse_buf.shape[0] >= B:
        lse = lse_buf[:B, :Hq]
    else:
        lse = torch.empty(B, Hq, dtype=torch.float32, device=query.device)
        if buf_holder is not None:
            buf_holder._tq_lse_buf = lse
    ops.stage2(mid_o, seq_lens, output, lse)
    return output if output.dtype == query.dtype else output.to(query.dtype)


def triton_turboquant_store(
    key: torch.Tensor,
    value: torch.Tensor,
    kv_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    PiT: torch.Tensor,
    midpoints: torch.Tensor,
    mse_bits: int,
    key_packed_size: int,
    value_quant_bits: int,
    key_fp8: bool = False,
    centroids: Optional[torch.Tensor] = None,
    norm_correction: bool = False,
    layout: str = "soa",
) -> None:
    """Store raw ``key``/``value`` ``[N, H, D]`` into the cache.  The host
    part (norm, normalise, rotation GEMM) is the reference launcher's
    (reference/soa_store.py:482-487); the quantise/pack kernel is sm_100a.
    ``key_fp8=True`` (``turboquant_k8v4``) casts the raw key to e4m3 in the
    kernel, 196 bytes per token-head (reference/soa_store.py:446-479,
    reference/aos_store.py:386-412).  ``layout="aos"`` writes the AoS slot
    form of the preset (reference/aos_store.py:350-447), storing the raw key
    norm."""
    family = "aos" if str(layout).lower().startswith("aos") else "soa"
    layout = _preset_layout(key_fp8, mse_bits, value_quant_bits, family)
    N, H, D = key.shape
    if key_fp8:
        ops.store(key.float().reshape(N * H, D).contiguous(), None, value.float().reshape(N * H, D).contiguous(),
                  kv_cache, slot_mapping, None, None, layout=layout, norm_correction=False)
        return
    k_flat = key.float().reshape(N * H, D)
    norms = k_flat.norm(dim=1, keepdim=True)
    x_hat = k_flat / (norms + 1e-8)
    y = (x_hat @ PiT).contiguous()
    v_flat = value.float().reshape(N * H, D).contiguous()
    ops.store(y, norms.reshape(-1).contiguous(), v_flat, kv_cache, slot_mapping, midpoints,
              centroids, layout=layout, norm_correction=norm_correction)


def convert_soa_to_aos_kv_cache(soa_cache: torch.Tensor, centroids: torch.Tensor) -> torch.Tensor:
    """Re-lay a SoA cache as the equivalent AoS cache: same codes, V scale
    and zero; the raw K norm is rebuilt as fp16(folded_norm * |c|) because
    AoS decoders apply the norm correction themselves."""
    nb, bs, hk, slot = soa_cache.shape
    blocks = soa_cache.reshape(nb, bs * hk * slot)
    data = blocks[:, : meta_region_offset(hk, bs)].reshape(nb, bs, hk, DATA_BYTES_PER_SLOT)
    meta = blocks[:, meta_region_offset(hk, bs):].contiguous().view(torch.float16)
    meta = meta[:, : hk * NUM_SOA_FIELDS * bs].reshape(nb, hk, NUM_SOA_FIELDS, bs)
    aos = torch.zeros_like(soa_cache)
    aos[..., :MSE_BYTES] = data[..., :MSE_BYTES]
    aos[..., MSE_BYTES + 2 : MSE_BYTES + 2 + VAL_DATA_BYTES] = data[..., MSE_BYTES:]
    half = aos.view(torch.float16)  # [nb, bs, hk, 67]
    half[..., (MSE_BYTES + 2 + VAL_DATA_BYTES) // 2] = meta[:, :, SOA_V_SCALE, :].permute(0, 2, 1)
    half[..., (MSE_BYTES + 4 + VAL_DATA_BYTES) // 2] = meta[:, :, SOA_V_ZERO, :].permute(0, 2, 1)
    c = centroids.float()
    for s in range(0, nb, 128):
        e = min(s + 128, nb)
        packed = data[s:e, ..., :MSE_BYTES]
        idx = torch.stack([packed & 0xF, packed >> 4], -1).reshape(e - s, bs, hk, HEAD_DIM).long()
        cnorm = torch.linalg.vector_norm(c[idx], dim=-1)
        folded = meta[s:e, :, SOA_K_NORM, :].permute(0, 2, 1).float()
        half[s:e, ..., MSE_BYTES // 2] = (folded * cnorm).to(torch.float16)
    return aos
