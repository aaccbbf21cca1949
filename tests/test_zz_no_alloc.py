"""tqb_decode_static (the allocation-free decode entry point), through the C
ABI: two calls in a row, each compared with the caller-buffer path
(tqb_stage1 into a caller mid_o, then tqb_stage2).  Collected last so it
also runs after every other test in the same process; it passes alone too."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import random_case
from tqb import _lib

pytestmark = pytest.mark.gpu

D = 128


def _stage1_args(q, kv, bt, sl, cents, S):
    a = _lib.Stage1Args()
    a.q_rot, a.q_stride_b, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    a.kv_cache, a.layout = kv.data_ptr(), _lib.TQB_LAYOUT_SOA
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
    a = _stage1_args(t["q"], t["kv"], t["bt"], t["sl"], t["cents"], S)
    a.mid_o, a.mid_stride_b, a.mid_stride_h, a.mid_stride_s = mid.data_ptr(), mid.stride(0), mid.stride(1), mid.stride(2)
    _lib.check(lib.tqb_stage1(ctypes.byref(a), _stream(dev)))
    out = torch.empty(B, Hq, D, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    s2 = _lib.Stage2Args()
    s2.mid_o, s2.mid_stride_b, s2.mid_stride_h, s2.mid_stride_s = mid.data_ptr(), mid.stride(0), mid.stride(1), mid.stride(2)
    s2.seq_lens = t["sl"].data_ptr()
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
    a.stage1 = _stage1_args(t["q"], t["kv"], t["bt"], t["sl"], t["cents"], S)
    a.output, a.out_stride_b, a.out_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    a.lse, a.lse_stride_b = lse.data_ptr(), lse.stride(0)
    _lib.check(lib.tqb_decode_static(ctypes.byref(a), _stream(dev)))
    return out, lse


def _tensors(c, dev):
    return dict(q=torch.from_numpy(c["q_rot"]).to(dev), kv=torch.from_numpy(c["kv_cache"]).to(dev),
                bt=torch.from_numpy(c["block_table"]).to(dev), sl=torch.from_numpy(c["seq_lens"]).to(dev),
                cents=torch.from_numpy(c["centroids"]).to(dev))


def test_decode_static_matches_caller_buffer_two_calls(cuda_device):
    lib = _lib.load()
    dev = cuda_device
    cases = [(_tensors(random_case(901, 3, 32, 8, [300, 17, 1024]), dev), 8),
             (_tensors(random_case(902, 4, 64, 8, [2000, 1, 640, 129]), dev), 16)]
    for i, (t, S) in enumerate(cases):  # two calls in a row, different shapes
        got_o, got_l = _via_static(lib, dev, t, S)
        ref_o, ref_l = _via_caller_buffer(lib, dev, t, S)
        torch.cuda.synchronize(dev)
        # same kernels, same order of operations: identical results
        assert torch.equal(got_o, ref_o), f"call {i}: output differs"
        assert torch.equal(got_l, ref_l), f"call {i}: lse differs"


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
