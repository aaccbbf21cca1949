"""tqb_decode_static (the allocation-free decode entry point), through the C
ABI: two calls in a row, each compared with the caller-buffer path
(tqb_stage1 into a caller mid_o, then tqb_stage2) and with the CPU oracle
(Stage1 + Stage2 of the reference algorithm, within the decode parity bar).
Further cases: a call exactly at the static buffer's row limit, per-sequence
split counts, and an AoS cache.  Collected last so it also runs after every
other test in the same process; it passes alone too."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import assert_close, random_case
from oracle import oracle as O
from tqb import _lib

pytestmark = pytest.mark.gpu

D = 128


def _stage1_args(q, kv, bt, sl, cents, S, layout=_lib.TQB_LAYOUT_SOA, nsp=None):
    a = _lib.Stage1Args()
    a.q_rot, a.q_stride_b, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    a.kv_cache, a.layout = kv.data_ptr(), layout
    a.num_splits_per_seq = None if nsp is None else nsp.data_ptr()
    a.cache_stride_block, a.cache_stride_pos, a.cache_stride_head = kv.stride(0), kv.stride(1), kv.stride(2)
    a.num_blocks = kv.shape[0]
    a.block_table, a.block_table_stride, a.max_blocks_per_seq = bt.data_ptr(), bt.stride(0), bt.shape[1]
    a.seq_lens, a.centroids, a.n_centroids = sl.data_ptr(), cents.data_ptr(), cents.numel()
    a.batch, a.num_q_heads, a.num_kv_heads = q.shape[0], q.shape[1], kv.shape[2]
    a.head_dim, a.block_size, a.num_splits = D, 16, S
    return a


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _via_caller_buffer(lib, dev, t, S):
    B, Hq = t["q"].shape[:2]
    mid = torch.empty(B, Hq, S, D + 1, device=dev)
    a = _stage1_args(t["q"], t["kv"], t["bt"], t["sl"], t["cents"], S, t["layout"], t["nsp"])
    a.mid_o, a.mid_stride_b, a.mid_stride_h, a.mid_stride_s = mid.data_ptr(), mid.stride(0), mid.stride(1), mid.stride(2)
    _lib.check(lib.tqb_stage1(ctypes.byref(a), _stream(dev)))
    out = torch.empty(B, Hq, D, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    s2 = _lib.Stage2Args()
    s2.mid_o, s2.mid_stride_b, s2.mid_stride_h, s2.mid_stride_s = mid.data_ptr(), mid.stride(0), mid.stride(1), mid.stride(2)
    s2.seq_lens = t["sl"].data_ptr()
    s2.num_splits_per_seq = None if t["nsp"] is None else t["nsp"].data_ptr()
    s2.output, s2.out_stride_b, s2.out_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    s2.lse, s2.lse_stride_b = lse.data_ptr(), lse.stride(0)
    s2.batch, s2.num_q_heads, s2.head_dim, s2.num_splits = B, Hq, D, S
    _lib.check(lib.tqb_stage2(ctypes.byref(s2), _stream(dev)))
    return out, lse


def _via_static(lib, dev, t, S):
    B, Hq = t["q"].shape[:2]
    out = torch.full((B, Hq, D), -7.0, device=dev)
    lse = torch.full((B, Hq), -7.0, device=dev)
    a = _lib.DecodeStaticArgs()
    a.stage1 = _stage1_args(t["q"], t["kv"], t["bt"], t["sl"], t["cents"], S, t["layout"], t["nsp"])
    a.output, a.out_stride_b, a.out_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    a.lse, a.lse_stride_b = lse.data_ptr(), lse.stride(0)
    _lib.check(lib.tqb_decode_static(ctypes.byref(a), _stream(dev)))
    return out, lse


def _tensors(c, dev, layout=_lib.TQB_LAYOUT_SOA, nsp=None):
    return dict(q=torch.from_numpy(c["q_rot"]).to(dev), kv=torch.from_numpy(c["kv_cache"]).to(dev),
                bt=torch.from_numpy(c["block_table"]).to(dev), sl=torch.from_numpy(c["seq_lens"]).to(dev),
                cents=torch.from_numpy(c["centroids"]).to(dev), layout=layout,
                nsp=None if nsp is None else torch.tensor(nsp, dtype=torch.int32, device=dev), case=c,
                nsp_np=None if nsp is None else np.asarray(nsp, np.int32))


def _oracle(t, S):
    c = t["case"]
    lay = O.LAYOUT_SOA if t["layout"] == _lib.TQB_LAYOUT_SOA else O.LAYOUT_AOS
    mid = O.stage1(c["q_rot"], c["kv_cache"], c["block_table"], c["seq_lens"], c["centroids"], S, layout=lay,
                   num_splits_per_seq=t["nsp_np"])
    return O.stage2(mid, c["seq_lens"], num_splits_per_seq=t["nsp_np"])


def _identical(a, b):
    """Bit-identical, NaN matching NaN (a sequence without tokens merges to NaN)."""
    return bool(((a == b) | (torch.isnan(a) & torch.isnan(b))).all())


def _check(lib, dev, t, S, what):
    got_o, got_l = _via_static(lib, dev, t, S)
    ref_o, ref_l = _via_caller_buffer(lib, dev, t, S)
    torch.cuda.synchronize(dev)
    # same kernels, same order of operations: identical results
    assert _identical(got_o, ref_o), f"{what}: output differs from the caller-buffer path"
    assert _identical(got_l, ref_l), f"{what}: lse differs from the caller-buffer path"
    # and the reference algorithm on the CPU, within the decode parity bar
    o_ref, l_ref = _oracle(t, S)
    live = t["case"]["seq_lens"] > 0
    assert_close(got_o.cpu().numpy()[live], o_ref[live], what=f"{what}: output vs oracle")
    assert_close(got_l.cpu().numpy()[live], l_ref[live], what=f"{what}: lse vs oracle")


def test_decode_static_matches_caller_buffer_two_calls(cuda_device):
    lib = _lib.load()
    dev = cuda_device
    cases = [(_tensors(random_case(901, 3, 32, 8, [300, 17, 1024]), dev), 8),
             (_tensors(random_case(902, 4, 64, 8, [2000, 1, 640, 129]), dev), 16)]
    for i, (t, S) in enumerate(cases):  # two calls in a row, different shapes
        _check(lib, dev, t, S, f"call {i}")


def test_decode_static_at_the_row_limit(cuda_device):
    """batch * num_q_heads * num_splits == 8192, the largest call the static
    buffer takes: every row of it is written and merged."""
    lib = _lib.load()
    t = _tensors(random_case(904, 8, 32, 8, [4096, 77, 1500, 2048, 16, 3000, 640, 4095]), cuda_device)
    _check(lib, cuda_device, t, 32, "8 x 32 x 32 rows")


def test_decode_static_per_sequence_splits_and_aos(cuda_device):
    """Per-sequence split counts (num_splits_per_seq), then an AoS cache,
    through the static buffer."""
    lib = _lib.load()
    lens = [900, 33, 2500, 0, 128]
    t = _tensors(random_case(905, 5, 32, 8, lens), cuda_device, nsp=[2, 1, 5, 1, 4])
    _check(lib, cuda_device, t, 8, "per-sequence splits")
    t = _tensors(random_case(906, 3, 32, 8, [700, 5, 1800], layout="aos"), cuda_device, layout=_lib.TQB_LAYOUT_AOS)
    _check(lib, cuda_device, t, 8, "AoS cache")


def test_decode_static_rejects_oversize(cuda_device):
    lib = _lib.load()
    t = _tensors(random_case(903, 2, 32, 8, [64, 64]), cuda_device)
    a = _lib.DecodeStaticArgs()
    a.stage1 = _stage1_args(t["q"], t["kv"], t["bt"], t["sl"], t["cents"], 129)  # 2*32*129 > 8192 rows
    out = torch.empty(2, 32, D, device=cuda_device)
    a.output, a.lse = out.data_ptr(), out.data_ptr()
    rc = lib.tqb_decode_static(ctypes.byref(a), _stream(cuda_device))
    assert rc == _lib.TQB_ERR_UNSUPPORTED
    assert b"exceeds the static partial buffer" in lib.tqb_last_error_detail()
