"""Torch-facing entry points over the C ABI (``include/tqb.h``).

Each function takes CUDA tensors, reads their pointers/strides, and calls the
matching ``libtqb.so`` entry point on the tensors' device and its current
torch stream.  Launches are asynchronous; nothing is allocated here unless a
function says so.  Errors raise ``TqbError`` (a ``RuntimeError``), mirroring
the ``TORCH_CHECK`` behaviour of the reference's native entry points
(cuda/tq4_cuda_v9.cu:279-297).
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib
from ._lib import MergeArgs, RotateArgs, SinkArgs, Stage1Args, Stage2Args, StoreArgs, TqbError
from .layout import (BLOCK_SIZE, FP8_KEY_LAYOUTS, HEAD_DIM, KEY3_LAYOUTS, LAYOUT_AOS, LAYOUT_SOA, LAYOUT_SOA_K3,
                     LAYOUT_SOA_K3V3, LAYOUT_SOA_K8, layout_id)

_SOA_FAMILY = (LAYOUT_SOA, LAYOUT_SOA_K8, LAYOUT_SOA_K3, LAYOUT_SOA_K3V3)  # block-as-raw-bytes layouts


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise TqbError(_lib.TQB_ERR_INVALID_ARG, msg)


def _cuda(t: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    _require(isinstance(t, torch.Tensor), f"{name} must be a torch.Tensor")
    _require(t.is_cuda, f"{name} must be a CUDA tensor")
    _require(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")


_DTYPE_ID = {torch.float32: _lib.TQB_DTYPE_F32, torch.float16: _lib.TQB_DTYPE_F16,
             torch.bfloat16: _lib.TQB_DTYPE_BF16}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _block_dense(kv_cache: torch.Tensor) -> bool:
    """True when the inner dims ``[16, Hk, slot]`` cover one block's bytes
    densely with the slot bytes innermost, in either order of the token and
    head dims: the cache as allocated, or vLLM's ``(blocks, H, N, C)`` storage
    seen through ``kv_cache.transpose(1, 2)`` (reference/turboquant_attn.py:
    565).  An SoA block is raw bytes from its base (the reference kernels use
    only ``kv_cache.stride(0)``, reference/soa_decode_v1.py:579), so either
    view reads the same block."""
    if kv_cache.stride(3) != 1:
        return False
    dims = sorted((kv_cache.stride(i), kv_cache.shape[i]) for i in (1, 2, 3) if kv_cache.shape[i] > 1)
    expect = 1
    for st, n in dims:
        if st != expect:
            return False
        expect *= n
    return True


def stage1(q_rot: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor,
           seq_lens: torch.Tensor, centroids: torch.Tensor, mid_o: torch.Tensor, *,
           layout="soa", num_splits_per_seq: Optional[torch.Tensor] = None,
           pair_lut: Optional[torch.Tensor] = None, attn_scale: Optional[float] = None,
           sinks: Optional[torch.Tensor] = None, query: Optional[torch.Tensor] = None,
           rotation: Optional[torch.Tensor] = None, stream: Optional[int] = None) -> torch.Tensor:
    """Decode Stage1 into ``mid_o [B, Hq, S, D+1]`` (S = ``mid_o.shape[2]``).

    With ``query`` and ``rotation`` given, ``q_rot`` is an output: Stage1
    first computes ``q_rot = float(query) @ rotation`` (:func:`rotate_query`)
    and decodes with it; ``tqb_stage1_rotated`` does both in one kernel where
    the page ring serves the cache and the GQA group is at most 4.

    ``kv_cache`` is the ``[num_blocks, 16, Hk, 134]`` uint8 cache (a view
    with a non-unit block stride is accepted; SoA needs the inner three dims
    contiguous).  ``num_splits_per_seq`` (int32 ``[B]``, each <= S) switches
    from the uniform split count S to per-sequence counts.  ``sinks``
    (float32 ``[Hq]`` logits) adds the reference's attention sinks
    (``USE_SINKS``, reference/soa_decode_v1.py:134-145) to split 0, through
    :func:`fold_sinks` on the same stream.
    """
    lay = layout_id(layout)
    _cuda(q_rot, "q_rot", torch.float32)
    _cuda(kv_cache, "kv_cache", torch.uint8)
    _cuda(block_table, "block_table", torch.int32)
    _cuda(seq_lens, "seq_lens", torch.int32)
    if centroids is not None or lay not in FP8_KEY_LAYOUTS:  # FP8 keys use no centroids
        _cuda(centroids, "centroids", torch.float32)
    _cuda(mid_o, "mid_o", torch.float32)
    _require(q_rot.dim() == 3 and q_rot.stride(2) == 1, "q_rot must be [B, Hq, D] with unit inner stride")
    _require(kv_cache.dim() == 4, "kv_cache must be [num_blocks, block_size, Hk, slot]")
    _require(block_table.dim() == 2 and block_table.stride(1) == 1, "block_table must be [B, max_blocks] row-major")
    _require(seq_lens.dim() == 1 and seq_lens.is_contiguous(), "seq_lens must be a contiguous [B] tensor")
    _require(centroids is None or centroids.is_contiguous(), "centroids must be contiguous")
    _require(mid_o.dim() == 4 and mid_o.stride(3) == 1, "mid_o must be [B, Hq, S, D+1] with unit inner stride")
    B, Hq, D = q_rot.shape
    nb, bs, Hk, slot = kv_cache.shape
    _require(tuple(mid_o.shape[:2]) == (B, Hq) and mid_o.shape[3] == D + 1,
             f"mid_o shape {tuple(mid_o.shape)} does not match q_rot {tuple(q_rot.shape)}")
    _require(block_table.shape[0] == B and seq_lens.shape[0] == B, "batch mismatch")
    if lay in _SOA_FAMILY:
        _require(_block_dense(kv_cache), "SoA cache needs each block's bytes contiguous")
    devs = {t.device for t in (q_rot, kv_cache, block_table, seq_lens, centroids, mid_o) if t is not None}
    _require(len(devs) == 1, f"all tensors must be on one device, got {devs}")
    nsp = None
    if num_splits_per_seq is not None:
        _cuda(num_splits_per_seq, "num_splits_per_seq", torch.int32)
        _require(num_splits_per_seq.shape == (B,) and num_splits_per_seq.is_contiguous(),
                 "num_splits_per_seq must be a contiguous [B] tensor")
        nsp = num_splits_per_seq
    if sinks is not None:
        _cuda(sinks, "sinks", torch.float32)
        _require(sinks.shape == (Hq,) and sinks.is_contiguous() and sinks.device == mid_o.device,
                 "sinks must be a contiguous [Hq] float32 tensor on mid_o's device")
    r = None
    if query is not None or rotation is not None:
        _require(query is not None and rotation is not None, "query and rotation go together")
        r = _rotate_args(query, rotation, q_rot)
    a = Stage1Args()
    a.q_rot = q_rot.data_ptr()
    a.q_stride_b, a.q_stride_h = q_rot.stride(0), q_rot.stride(1)
    a.kv_cache = kv_cache.data_ptr()
    a.layout = lay
    a.cache_stride_block, a.cache_stride_pos, a.cache_stride_head = (
        kv_cache.stride(0), kv_cache.stride(1), kv_cache.stride(2))
    a.num_blocks = nb
    a.block_table = block_table.data_ptr()
    a.block_table_stride = block_table.stride(0)
    a.max_blocks_per_seq = block_table.shape[1]
    a.seq_lens = seq_lens.data_ptr()
    a.centroids = centroids.data_ptr() if centroids is not None else None
    a.n_centroids = centroids.numel() if centroids is not None else 0
    a.pair_lut = pair_lut.data_ptr() if pair_lut is not None else None
    a.num_splits_per_seq = nsp.data_ptr() if nsp is not None else None
    a.mid_o = mid_o.data_ptr()
    a.mid_stride_b, a.mid_stride_h, a.mid_stride_s = mid_o.stride(0), mid_o.stride(1), mid_o.stride(2)
    a.batch, a.num_q_heads, a.num_kv_heads, a.head_dim = B, Hq, Hk, D
    a.block_size, a.num_splits = bs, mid_o.shape[2]
    a.attn_scale = float(attn_scale) if attn_scale is not None else 1.0 / math.sqrt(D)
    with torch.cuda.device(mid_o.device):
        st = stream if stream is not None else _stream(mid_o.device)
        if r is None:
            _lib.check(_lib.load().tqb_stage1(a, st))
        else:
            _lib.check(_lib.load().tqb_stage1_rotated(r, a, st))
    if sinks is not None:
        fold_sinks(mid_o, seq_lens, sinks, stream=stream)
    return mid_o


def fold_sinks(mid_o: torch.Tensor, seq_lens: torch.Tensor, sinks: torch.Tensor, *,
               stream: Optional[int] = None) -> torch.Tensor:
    """Fold per-head sink logits ``sinks [Hq]`` (float32) into split 0 of
    ``mid_o [B, Hq, S, D+1]`` in place, for every sequence with seq_len > 0:
    one extra token of logit ``sinks[h]`` and value 0, as the reference
    Stage1 with ``USE_SINKS`` (reference/soa_decode_v1.py:134-145)."""
    _cuda(mid_o, "mid_o", torch.float32)
    _cuda(seq_lens, "seq_lens", torch.int32)
    _cuda(sinks, "sinks", torch.float32)
    _require(mid_o.dim() == 4 and mid_o.stride(3) == 1, "mid_o must be [B, Hq, S, D+1] with unit inner stride")
    B, Hq, _, D1 = mid_o.shape
    _require(seq_lens.shape == (B,) and seq_lens.is_contiguous(), "seq_lens must be a contiguous [B] tensor")
    _require(sinks.shape == (Hq,) and sinks.is_contiguous(), "sinks must be a contiguous [Hq] tensor")
    devs = {t.device for t in (mid_o, seq_lens, sinks)}
    _require(len(devs) == 1, f"all tensors must be on one device, got {devs}")
    a = SinkArgs()
    a.mid_o = mid_o.data_ptr()
    a.mid_stride_b, a.mid_stride_h = mid_o.stride(0), mid_o.stride(1)
    a.seq_lens = seq_lens.data_ptr()
    a.sinks = sinks.data_ptr()
    a.batch, a.num_q_heads, a.head_dim = B, Hq, D1 - 1
    with torch.cuda.device(mid_o.device):
        _lib.check(_lib.load().tqb_fold_sinks(a, stream if stream is not None else _stream(mid_o.device)))
    return mid_o


def stage2(mid_o: torch.Tensor, seq_lens: torch.Tensor, output: torch.Tensor, lse: torch.Tensor, *,
           num_splits_per_seq: Optional[torch.Tensor] = None, stream: Optional[int] = None):
    """Merge the non-empty splits of ``mid_o`` into ``output [B, Hq, D]`` and
    ``lse [B, Hq]``.  ``output`` may be float32, float16 or bfloat16: a
    16-bit output receives the fp32 result rounded to nearest even (the
    launcher's ``output.to(query.dtype)``, reference/soa_decode_v1.py:643,
    without the extra pass)."""
    _cuda(mid_o, "mid_o", torch.float32)
    _cuda(seq_lens, "seq_lens", torch.int32)
    _require(isinstance(output, torch.Tensor) and output.is_cuda and output.dtype in _DTYPE_ID,
             "output must be a float32/float16/bfloat16 CUDA tensor")
    _cuda(lse, "lse", torch.float32)
    _require(mid_o.dim() == 4 and mid_o.stride(3) == 1, "mid_o must be [B, Hq, S, D+1]")
    B, Hq, S, D1 = mid_o.shape
    _require(tuple(output.shape) == (B, Hq, D1 - 1) and output.stride(2) == 1, "output must be [B, Hq, D]")
    _require(tuple(lse.shape) == (B, Hq) and lse.stride(1) == 1, "lse must be [B, Hq]")
    _require(seq_lens.shape == (B,) and seq_lens.is_contiguous(), "seq_lens must be a contiguous [B] tensor")
    a = Stage2Args()
    a.mid_o = mid_o.data_ptr()
    a.mid_stride_b, a.mid_stride_h, a.mid_stride_s = mid_o.stride(0), mid_o.stride(1), mid_o.stride(2)
    a.seq_lens = seq_lens.data_ptr()
    if num_splits_per_seq is not None:
        _cuda(num_splits_per_seq, "num_splits_per_seq", torch.int32)
        a.num_splits_per_seq = num_splits_per_seq.data_ptr()
    a.output = output.data_ptr()
    a.out_stride_b, a.out_stride_h = output.stride(0), output.stride(1)
    a.lse = lse.data_ptr()
    a.lse_stride_b = lse.stride(0)
    a.batch, a.num_q_heads, a.head_dim, a.num_splits = B, Hq, D1 - 1, S
    with torch.cuda.device(mid_o.device):
        st = stream if stream is not None else _stream(mid_o.device)
        if output.dtype == torch.float32:
            _lib.check(_lib.load().tqb_stage2(a, st))
        else:
            _lib.check(_lib.load().tqb_stage2_typed(a, _DTYPE_ID[output.dtype], output.data_ptr(), st))
    return output, lse


def _rotate_args(query: torch.Tensor, rotation: torch.Tensor, out: torch.Tensor) -> RotateArgs:
    _require(isinstance(query, torch.Tensor) and query.is_cuda and query.dtype in _DTYPE_ID,
             "query must be a float32/float16/bfloat16 CUDA tensor")
    _cuda(rotation, "rotation", torch.float32)
    _require(query.dim() == 3 and query.shape[2] == HEAD_DIM and query.stride(2) == 1,
             "query must be [B, Hq, 128] with unit stride over the last dim")
    _require(tuple(rotation.shape) == (HEAD_DIM, HEAD_DIM) and rotation.is_contiguous(),
             "rotation must be a contiguous [128, 128] matrix")
    B, Hq, D = query.shape
    _cuda(out, "out", torch.float32)
    _require(tuple(out.shape) == (B, Hq, D) and out.stride(2) == 1, "out must be [B, Hq, 128]")
    a = RotateArgs()
    a.query, a.query_dtype = query.data_ptr(), _DTYPE_ID[query.dtype]
    a.q_stride_b, a.q_stride_h = query.stride(0), query.stride(1)
    a.rotation, a.q_rot = rotation.data_ptr(), out.data_ptr()
    a.out_stride_b, a.out_stride_h = out.stride(0), out.stride(1)
    a.batch, a.num_q_heads, a.head_dim = B, Hq, D
    return a


def rotate_query(query: torch.Tensor, rotation: torch.Tensor, out: Optional[torch.Tensor] = None, *,
                 stream: Optional[int] = None) -> torch.Tensor:
    """``float(query) @ rotation`` for ``query [B, Hq, D]`` (float32, float16
    or bfloat16, unit stride over D) and ``rotation = Pi^T [D, D]`` float32:
    the launcher's cast + GEMM + copy (reference/soa_decode_v1.py:535-538) in
    one kernel, fp32 accumulation.  Writes ``out`` (float32 [B, Hq, D],
    allocated when None) and returns it."""
    _require(isinstance(query, torch.Tensor) and query.is_cuda and query.dim() == 3,
             "query must be a [B, Hq, 128] CUDA tensor")
    if out is None:
        out = torch.empty(query.shape, dtype=torch.float32, device=query.device)
    a = _rotate_args(query, rotation, out)
    with torch.cuda.device(query.device):
        _lib.check(_lib.load().tqb_rotate_query(a, stream if stream is not None else _stream(query.device)))
    return out


def merge_partials(partials: torch.Tensor, output: torch.Tensor, lse: Optional[torch.Tensor] = None, *,
                   stream: Optional[int] = None):
    """LSE-merge ``partials [G, B, Hq, D+1]`` (one (O, LSE) per KV range) into
    ``output [B, Hq, D]`` and optionally ``lse [B, Hq]``."""
    _cuda(partials, "partials", torch.float32)
    _cuda(output, "output", torch.float32)
    _require(partials.dim() == 4 and partials.is_contiguous(), "partials must be a contiguous [G, B, Hq, D+1]")
    G, B, Hq, D1 = partials.shape
    _require(tuple(output.shape) == (B, Hq, D1 - 1) and output.is_contiguous(), "output must be contiguous [B, Hq, D]")
    a = MergeArgs()
    a.partials = partials.data_ptr()
    a.num_parts, a.batch, a.num_q_heads, a.head_dim = G, B, Hq, D1 - 1
    a.output = output.data_ptr()
    if lse is not None:
        _cuda(lse, "lse", torch.float32)
        _require(tuple(lse.shape) == (B, Hq) and lse.is_contiguous(), "lse must be contiguous [B, Hq]")
        a.lse = lse.data_ptr()
    with torch.cuda.device(output.device):
        _lib.check(_lib.load().tqb_merge_partials(a, stream if stream is not None else _stream(output.device)))
    return output, lse


def store(y: torch.Tensor, norms: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor,
          slot_mapping: torch.Tensor, midpoints: torch.Tensor, centroids: Optional[torch.Tensor] = None, *,
          layout="soa", norm_correction: bool = True, stream: Optional[int] = None) -> None:
    """Quantise ``N*H`` token-heads into the cache (kernel stage of the
    reference store; ``y``/``norms``/``value`` are its inputs).  With
    ``layout="soa_k8"`` or ``"aos_k8"`` (FP8 keys) ``y`` is the raw key, cast
    to e4m3, and ``norms``/``midpoints``/``centroids`` are unused (may be
    None).  AoS layouts store the raw norm (their decoders apply the norm
    correction), so ``norm_correction`` only affects the SoA layouts."""
    lay = layout_id(layout)
    k8 = lay in FP8_KEY_LAYOUTS
    _cuda(y, "y", torch.float32)
    _cuda(value, "value", torch.float32)
    _cuda(kv_cache, "kv_cache", torch.uint8)
    _cuda(slot_mapping, "slot_mapping", torch.int32)
    if not k8:
        _cuda(norms, "norms", torch.float32)
        _cuda(midpoints, "midpoints", torch.float32)
    nb, bs, H, slot = kv_cache.shape
    N = slot_mapping.shape[0]
    _require(y.is_contiguous() and value.is_contiguous() and (k8 or norms.is_contiguous()),
             "inputs must be contiguous")
    _require(y.numel() == N * H * HEAD_DIM and value.numel() == N * H * HEAD_DIM and (k8 or norms.numel() == N * H),
             "y/value must be [N*H, 128] and norms [N*H]")
    if k8:
        _require(not norm_correction, "FP8 keys have no norm correction")
    if lay in _SOA_FAMILY:
        _require(_block_dense(kv_cache), "SoA cache needs each block's bytes contiguous")
    if norm_correction:
        _require(centroids is not None, "norm_correction=True requires centroids")
    if centroids is not None:
        _cuda(centroids, "centroids", torch.float32)
    a = StoreArgs()
    a.y, a.value = y.data_ptr(), value.data_ptr()
    a.norms = norms.data_ptr() if norms is not None else None
    a.midpoints = midpoints.data_ptr() if midpoints is not None else None
    a.centroids = centroids.data_ptr() if centroids is not None else None
    a.slot_mapping = slot_mapping.data_ptr()
    a.kv_cache = kv_cache.data_ptr()
    a.layout = lay
    a.cache_stride_block, a.cache_stride_pos, a.cache_stride_head = (
        kv_cache.stride(0), kv_cache.stride(1), kv_cache.stride(2))
    a.num_blocks = nb
    a.num_tokens, a.num_kv_heads, a.head_dim, a.block_size = N, H, HEAD_DIM, bs
    a.n_centroids = 8 if lay in KEY3_LAYOUTS else 16
    a.norm_correction = int(bool(norm_correction)) if lay in (LAYOUT_SOA, LAYOUT_SOA_K3, LAYOUT_SOA_K3V3) else 0
    with torch.cuda.device(kv_cache.device):
        _lib.check(_lib.load().tqb_store(a, stream if stream is not None else _stream(kv_cache.device)))
