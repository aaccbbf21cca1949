"""The C ABI library (CPU only: no kernel is launched here).

Checks that libtqb.so is built for sm_100a, loads, exports every function
declared in include/tqb.h, and that the ctypes argument structs have the
exact layout of the C structs (compiled with gcc against the header).
"""

from __future__ import annotations

import ctypes
import os
import re
import subprocess
import tempfile
from pathlib import Path

import pytest

from conftest import PKG, ROOT
from tqb import _build, _lib

HEADER = ROOT / "include" / "tqb.h"


@pytest.fixture(scope="module")
def lib():
    _build.build()
    return _lib.load()


def header_functions() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(tqb_\w+)\s*\(", text, re.M)))


def test_header_declares_the_bound_symbols():
    assert header_functions() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_header_symbol(lib):
    for name in header_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (tqb_\w+)", out))
    assert set(header_functions()) <= exported


def test_library_holds_sm100a_code():
    out = subprocess.run(["cuobjdump", "--list-elf", str(_lib.LIB_PATH)], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr
    assert "sm_100a" in out.stdout


def test_host_only_entry_points(lib):
    assert lib.tqb_version() == 1000
    assert _lib.version() == 1000
    assert lib.tqb_strerror(0) == b"ok"
    assert lib.tqb_strerror(_lib.TQB_ERR_UNSUPPORTED) == b"unsupported shape or configuration"
    assert lib.tqb_strerror(-99) == b"unknown tqb status"


def test_argument_validation_without_launch(lib):
    """Rejections happen on the host before any device call."""
    a = _lib.Stage1Args()
    a.batch, a.num_q_heads, a.num_kv_heads, a.num_splits = 1, 32, 8, 4
    a.head_dim, a.block_size, a.n_centroids = 64, 16, 16
    assert lib.tqb_stage1(ctypes.byref(a), None) == _lib.TQB_ERR_UNSUPPORTED
    assert b"head_dim" in lib.tqb_last_error_detail()
    a.head_dim = 128
    a.num_q_heads = 30  # not a multiple of Hk
    assert lib.tqb_stage1(ctypes.byref(a), None) == _lib.TQB_ERR_INVALID_ARG
    a.num_q_heads, a.num_kv_heads = 64, 4  # GQA 16
    assert lib.tqb_stage1(ctypes.byref(a), None) == _lib.TQB_ERR_UNSUPPORTED
    a.num_kv_heads = 8
    assert lib.tqb_stage1(ctypes.byref(a), None) == _lib.TQB_ERR_INVALID_ARG  # NULL pointers
    assert lib.tqb_stage1(None, None) == _lib.TQB_ERR_INVALID_ARG
    r = _lib.RotateArgs()
    r.batch, r.num_q_heads, r.head_dim, r.query_dtype = 1, 32, 128, 7  # no such dtype
    assert lib.tqb_rotate_query(ctypes.byref(r), None) == _lib.TQB_ERR_INVALID_ARG
    r.query_dtype, r.head_dim = _lib.TQB_DTYPE_BF16, 64
    assert lib.tqb_rotate_query(ctypes.byref(r), None) == _lib.TQB_ERR_UNSUPPORTED
    r.head_dim = 128
    assert lib.tqb_rotate_query(ctypes.byref(r), None) == _lib.TQB_ERR_INVALID_ARG  # NULL pointers
    t = _lib.Stage2Args()
    t.batch, t.num_q_heads, t.head_dim, t.num_splits = 1, 32, 128, 4
    assert lib.tqb_stage2_typed(ctypes.byref(t), 5, None, None) == _lib.TQB_ERR_INVALID_ARG
    assert b"out_dtype" in lib.tqb_last_error_detail()
    k = _lib.SinkArgs()
    k.batch, k.num_q_heads, k.head_dim = 1, 32, 64
    assert lib.tqb_fold_sinks(ctypes.byref(k), None) == _lib.TQB_ERR_UNSUPPORTED
    k.head_dim = 128
    assert lib.tqb_fold_sinks(ctypes.byref(k), None) == _lib.TQB_ERR_INVALID_ARG  # NULL pointers
    assert lib.tqb_fold_sinks(None, None) == _lib.TQB_ERR_INVALID_ARG
    k.batch = 0
    assert lib.tqb_fold_sinks(ctypes.byref(k), None) == _lib.TQB_OK  # empty batch: no-op
    s = _lib.StoreArgs()
    s.num_tokens, s.num_kv_heads, s.head_dim, s.block_size, s.n_centroids = 1, 8, 128, 16, 8
    assert lib.tqb_store(ctypes.byref(s), None) == _lib.TQB_ERR_UNSUPPORTED
    # The preset layouts: 3-bit keys need 8 centroids; FP8 keys none; an
    # unknown layout is rejected; the FP8-key store has no norm correction.
    a = _lib.Stage1Args()
    a.batch, a.num_q_heads, a.num_kv_heads, a.num_splits = 1, 32, 8, 4
    a.head_dim, a.block_size, a.n_centroids = 128, 16, 16
    for lay in (_lib.TQB_LAYOUT_SOA_K3, _lib.TQB_LAYOUT_SOA_K3V3):
        a.layout = lay
        assert lib.tqb_stage1(ctypes.byref(a), None) == _lib.TQB_ERR_UNSUPPORTED
        assert b"n_centroids" in lib.tqb_last_error_detail()
    a.layout, a.n_centroids = _lib.TQB_LAYOUT_SOA_K8, 0
    assert lib.tqb_stage1(ctypes.byref(a), None) == _lib.TQB_ERR_INVALID_ARG  # NULL pointers, not centroids
    assert b"NULL" in lib.tqb_last_error_detail()
    a.layout, a.n_centroids = 9, 16
    assert lib.tqb_stage1(ctypes.byref(a), None) == _lib.TQB_ERR_INVALID_ARG
    s = _lib.StoreArgs()
    s.num_tokens, s.num_kv_heads, s.head_dim, s.block_size, s.n_centroids = 1, 8, 128, 16, 16
    s.layout, s.norm_correction = _lib.TQB_LAYOUT_SOA_K8, 1
    assert lib.tqb_store(ctypes.byref(s), None) == _lib.TQB_ERR_INVALID_ARG
    assert b"norm correction" in lib.tqb_last_error_detail()
    # Empty batches are valid no-ops.
    a = _lib.Stage1Args()
    a.batch, a.num_q_heads, a.num_kv_heads, a.num_splits = 0, 32, 8, 32
    a.head_dim, a.block_size, a.n_centroids = 128, 16, 16
    assert lib.tqb_stage1(ctypes.byref(a), None) == _lib.TQB_OK


C_LAYOUT_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "tqb.h"
#define F(T, f) printf("%s.%s %zu\n", #T, #f, offsetof(T, f));
int main(void) {
  printf("tqb_stage1_args %zu\n", sizeof(tqb_stage1_args));
  printf("tqb_stage2_args %zu\n", sizeof(tqb_stage2_args));
  printf("tqb_merge_args %zu\n", sizeof(tqb_merge_args));
  printf("tqb_store_args %zu\n", sizeof(tqb_store_args));
  printf("tqb_decode_static_args %zu\n", sizeof(tqb_decode_static_args));
  printf("tqb_rotate_args %zu\n", sizeof(tqb_rotate_args));
  printf("tqb_sink_args %zu\n", sizeof(tqb_sink_args));
  printf("tqb_sp_exchange_args %zu\n", sizeof(tqb_sp_exchange_args));
  printf("tqb_sp_merge_args %zu\n", sizeof(tqb_sp_merge_args));
  %FIELDS%
  return 0;
}
"""


def test_p2p_entry_points_reject_on_the_host(lib):
    """The SP exchange validates rank, world and capacity before any device
    call, and sizes its buffer as rows of tagged elements (value + epoch, 8
    bytes each) + CTA counter + step counter."""
    row = 129 * 4
    assert lib.tqb_p2p_buffer_bytes(2, 128) == 2 * 2 * 128 * 2 * row + 8 + 8
    assert lib.tqb_p2p_buffer_bytes(0, 128) == -1
    assert lib.tqb_p2p_buffer_bytes(_lib.TQB_P2P_MAX_RANKS + 1, 128) == -1
    a = _lib.SpExchangeArgs()
    a.stage2.batch, a.stage2.num_q_heads, a.stage2.head_dim, a.stage2.num_splits = 2, 32, 128, 4
    a.rank, a.world, a.cap_rows, a.epoch = 0, 2, 64, 1
    a.rank = 2  # not below world
    assert lib.tqb_sp_exchange(ctypes.byref(a), None) == _lib.TQB_ERR_INVALID_ARG
    a.rank, a.epoch, a.cap_rows = 0, 0, 63  # device epochs; batch * heads = 64 rows do not fit
    assert lib.tqb_sp_exchange(ctypes.byref(a), None) == _lib.TQB_ERR_INVALID_ARG
    assert b"cap_rows" in lib.tqb_last_error_detail()
    a.cap_rows = 64  # rows fit, but no mid_o / buffers given
    assert lib.tqb_sp_exchange(ctypes.byref(a), None) == _lib.TQB_ERR_INVALID_ARG
    m = _lib.SpMergeArgs()
    m.world, m.batch, m.num_q_heads, m.head_dim, m.cap_rows, m.epoch = 2, 2, 32, 128, 64, 1
    assert lib.tqb_sp_merge(ctypes.byref(m), None) == _lib.TQB_ERR_INVALID_ARG  # no buffer / output
    m.world = 0
    assert lib.tqb_sp_merge(ctypes.byref(m), None) == _lib.TQB_ERR_INVALID_ARG
    assert lib.tqb_p2p_free(None) == _lib.TQB_OK and lib.tqb_ipc_close(None) == _lib.TQB_OK


def test_ctypes_structs_match_c_layout(tmp_path: Path):
    structs = {"tqb_stage1_args": _lib.Stage1Args, "tqb_stage2_args": _lib.Stage2Args,
               "tqb_merge_args": _lib.MergeArgs, "tqb_store_args": _lib.StoreArgs,
               "tqb_decode_static_args": _lib.DecodeStaticArgs, "tqb_rotate_args": _lib.RotateArgs,
               "tqb_sink_args": _lib.SinkArgs, "tqb_sp_exchange_args": _lib.SpExchangeArgs, "tqb_sp_merge_args": _lib.SpMergeArgs}
    fields = "\n".join(f"F({c}, {f})" for c, py in structs.items() for f, _ in py._fields_)
    src = tmp_path / "probe.c"
    src.write_text(C_LAYOUT_PROBE.replace("%FIELDS%", fields))
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include",
                    str(src), "-o", str(exe)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run(
        [str(exe)], capture_output=True, text=True, check=True).stdout.splitlines())
    for cname, py in structs.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(py, f).offset, f"{cname}.{f}"


def test_missing_library_raises_promptly(tmp_path: Path):
    """A library path that does not exist gives TqbError at once (the error
    text must not need the library it reports as missing)."""
    import subprocess
    import sys

    code = ("import sys; sys.path.insert(0, %r)\n"
            "from tqb import _lib\n"
            "try:\n    _lib.load()\nexcept _lib.TqbError as e:\n    print('raised', e.status, e)\n") % str(PKG)
    env = dict(os.environ, TQB_LIBRARY=str(tmp_path / "absent.so"))
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert "raised -5" in out.stdout and "absent.so" in out.stdout


def test_status_text_matches_library(lib):
    for status, text in _lib.STATUS_TEXT.items():
        assert lib.tqb_strerror(status).decode() == text


def test_stage1_rotated_rejects_on_the_host(lib):
    """tqb_stage1_rotated checks, before any device call, that the rotation
    writes Stage1's own query buffer and that the query dtype is known."""
    r = _lib.RotateArgs()
    a = _lib.Stage1Args()
    r.q_rot, a.q_rot = 0x1000, 0x2000  # different buffers
    r.batch = a.batch = 2
    r.num_q_heads = a.num_q_heads = 32
    r.head_dim = a.head_dim = 128
    assert lib.tqb_stage1_rotated(ctypes.byref(r), ctypes.byref(a), None) == _lib.TQB_ERR_INVALID_ARG
    assert b"rotation's output" in lib.tqb_last_error_detail()
    r.q_rot = a.q_rot
    r.query_dtype = 7
    assert lib.tqb_stage1_rotated(ctypes.byref(r), ctypes.byref(a), None) == _lib.TQB_ERR_INVALID_ARG
    assert b"query_dtype" in lib.tqb_last_error_detail()
