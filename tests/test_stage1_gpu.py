"""Stage1 parity of the sm_100a kernel (GPU).

Bar: |got - ref| <= 1e-4 + 2e-3 |ref| on every written O and LSE element
(conftest.ATOL/RTOL), against (a) the reference's own SoA/AoS V1 outputs
stored in the golden fixtures and (b) the CPU oracle on fresh seeded inputs.
Empty splits must stay unwritten, exactly as in the reference.

Every test runs twice: with the SoA cache served by the TMA page-ring kernel
(the default) and by the register-ring kernel (TQB_STAGE1_KERNEL=regs); the
AoS cache always uses the register-ring kernel.  After each run the device's
count of bounded waits that gave up must be zero.
"""

from __future__ import annotations

import functools
import math
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN_CASES, RTOL, assert_close, random_case
from oracle import oracle as O
import tqb
from tqb import layout as L

pytestmark = pytest.mark.gpu

SENTINEL = -12345.0


@pytest.fixture(autouse=True, params=["ring", "regs"])
def stage1_kernel(request, cuda_device):
    old = os.environ.get("TQB_STAGE1_KERNEL")
    os.environ["TQB_STAGE1_KERNEL"] = request.param
    tqb.wait_timeouts(reset=True)
    yield request.param
    torch.cuda.synchronize()
    assert tqb.wait_timeouts(reset=True) == 0, "a bounded device wait gave up"
    if old is None:
        os.environ.pop("TQB_STAGE1_KERNEL", None)
    else:
        os.environ["TQB_STAGE1_KERNEL"] = old


def _to(dev, z, key, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(z[key]))
    return t.to(dev) if dtype is None else t.to(dev, dtype)


def _run(dev, z, cache_key="kv_cache", layout="soa", nsp=None, S=None, sinks=None):
    S = int(z["num_splits"]) if S is None else S
    q = _to(dev, z, "q_rot")
    mid = torch.full((q.shape[0], q.shape[1], S, q.shape[2] + 1), SENTINEL, device=dev)
    tqb.stage1(q, _to(dev, z, cache_key), _to(dev, z, "block_table"), _to(dev, z, "seq_lens"),
               _to(dev, z, "centroids"), mid, layout=layout,
               num_splits_per_seq=None if nsp is None else torch.tensor(nsp, dtype=torch.int32, device=dev),
               sinks=None if sinks is None else _to(dev, z, sinks))
    torch.cuda.synchronize()
    return mid.cpu().numpy()


def _check(got, ref, what):
    written = ~np.isnan(ref[..., 0])
    # unwritten in the reference -> untouched here
    assert np.all(got[~written] == SENTINEL), f"{what}: wrote into an empty split"
    assert_close(got[written], ref[written], what=what)


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_soa_vs_reference_golden(cuda_device, golden, name):
    z = golden[name]
    _check(_run(cuda_device, z), z["mid_o_soa_v1"], f"{name} SoA")


def test_soa_sinks_vs_reference_golden(cuda_device, golden_sinks):
    """Attention sinks against the reference Stage1 run with USE_SINKS=1
    (reference/soa_decode_v1.py:134-145): a -inf sink, a sink that dominates
    its head's scores, ragged lengths with empty splits; then Stage2."""
    z = golden_sinks
    got = _run(cuda_device, z, sinks="sinks")
    _check(got, z["mid_o_soa_v1_sinks"], "SoA with sinks")
    # without sinks the same case matches the plain reference run
    _check(_run(cuda_device, z), z["mid_o_soa_v1"], "SoA without sinks")
    dev = cuda_device
    mid = torch.from_numpy(np.where(np.isnan(z["mid_o_soa_v1_sinks"]), 0.0, got).astype(np.float32)).to(dev)
    B, Hq = mid.shape[:2]
    out = torch.empty(B, Hq, 128, device=dev)
    lse = torch.empty(B, Hq, device=dev)
    tqb.stage2(mid, _to(dev, z, "seq_lens"), out, lse)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), z["out_stage2_sinks"], what="Stage2 with sinks out")
    assert_close(lse.cpu().numpy(), z["lse_stage2_sinks"], what="Stage2 with sinks lse")


@pytest.mark.parametrize("name", [n for n in GOLDEN_CASES if n != "ragged_gqa8_hk2"])
def test_aos_vs_reference_golden(cuda_device, golden, name):
    z = golden[name]
    _check(_run(cuda_device, z, "kv_cache_aos", "aos"), z["mid_o_aos_v1"], f"{name} AoS")


def test_compat_launchers(cuda_device, golden):
    z = golden["c0"]
    dev = cuda_device
    q, kv, bt, sl, c = (_to(dev, z, k) for k in ("q_rot", "kv_cache", "block_table", "seq_lens", "centroids"))
    mid = torch.full((2, 32, 4, 129), SENTINEL, device=dev)
    tqb.launch_soa_v1_stage1(q, kv, bt, sl, c, mid)
    lut = tqb.build_pair_lut(c)
    mid2 = tqb.launch_tq4_v2_stage1(q, kv, bt, sl, c, lut, num_splits=4)
    out = torch.empty(2, 32, 128, device=dev)
    lse = torch.empty(2, 32, device=dev)
    tqb.launch_stage2(mid, sl, out, lse)
    torch.cuda.synchronize()
    _check(mid.cpu().numpy(), z["mid_o_soa_v1"], "launch_soa_v1_stage1")
    assert_close(mid2.cpu().numpy(), z["mid_o_soa_v1"], what="launch_tq4_v2_stage1")
    assert_close(out.cpu().numpy(), z["out_stage2"], what="launch_stage2 out")
    assert_close(lse.cpu().numpy(), z["lse_stage2"], what="launch_stage2 lse")


@pytest.mark.parametrize("hq,hk", [(32, 8), (64, 8), (8, 1), (16, 2), (24, 8), (6, 2), (4, 4),
                                   (48, 16), (12, 3), (40, 8), (10, 5), (28, 4)])
def test_gqa_shapes_vs_oracle(cuda_device, hq, hk):
    z = random_case(hq * 100 + hk, 3, hq, hk, [300, 17, 1024])
    S = 5
    ref = O.stage1(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], S)
    _check(_run(cuda_device, z, S=S), ref, f"GQA {hq}/{hk}")


@pytest.mark.parametrize("hq,hk", [(32, 8), (64, 8), (8, 1), (16, 2), (16, 4), (32, 4), (8, 8), (48, 16), (12, 3)])
def test_aos_gqa_shapes_vs_oracle(cuda_device, hq, hk):
    """AoS cache: KV head counts dividing 8 run on the TMA page ring (whole
    blocks per run), the others on the register kernel."""
    z = random_case(hq * 100 + hk + 7, 3, hq, hk, [300, 17, 1024], layout="aos")
    S = 5
    ref = O.stage1(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], S,
                   layout=O.LAYOUT_AOS)
    _check(_run(cuda_device, z, layout="aos", S=S), ref, f"AoS GQA {hq}/{hk}")


def test_ragged_per_sequence_splits(cuda_device):
    lens = [512, 1, 16, 17, 4000, 777, 33, 1500]
    z = random_case(5, len(lens), 32, 8, lens)
    nsp = L.splits_per_sequence(lens, 512, 32)
    nsp[3] = 4  # 17 tokens in 4 splits of 5: the last split holds 2 tokens
    S = 32
    ref = O.stage1(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], S,
                   num_splits_per_seq=np.asarray(nsp, np.int32))
    _check(_run(cuda_device, z, nsp=nsp, S=S), ref, "per-seq splits")


@functools.lru_cache(maxsize=1)
def _ragged_batch():
    rng = np.random.default_rng(77)
    lens = rng.integers(0, 1500, size=160)
    lens[::23] = 0
    lens = lens.tolist()
    return lens, random_case(31, len(lens), 32, 8, lens)


@pytest.mark.parametrize("per_seq", [False, True])
def test_ragged_batch_weight_cuts(cuda_device, per_seq):
    """A large ragged batch (empty sequences included) takes the weight-cut
    tile walk: every group gets a contiguous tile range that can start and
    end inside a sequence, and every non-empty split is written once."""
    lens, z = _ragged_batch()
    S = 16
    nsp = L.splits_per_sequence(lens, 96, S) if per_seq else None
    ref = O.stage1(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], S,
                   num_splits_per_seq=None if nsp is None else np.asarray(nsp, np.int32))
    _check(_run(cuda_device, z, nsp=nsp, S=S), ref, "ragged batch")


def test_long_split_reloads_block_ids(cuda_device):
    """A split spanning > 32 pages exercises the block-id window refill."""
    lens = [16 * 70 + 5, 16 * 33]
    z = random_case(9, 2, 32, 8, lens)
    ref = O.stage1(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], 1)
    _check(_run(cuda_device, z, S=1), ref, "long split")


def test_strided_views(cuda_device):
    """Non-contiguous q/mid_o views and a block stride larger than the block
    (a cache carved out of a bigger allocation)."""
    z = random_case(3, 2, 32, 8, [200, 70])
    dev = cuda_device
    nb = z["kv_cache"].shape[0]
    big = torch.zeros(nb, 17152 + 256, dtype=torch.uint8, device=dev)
    big[:, :17152] = torch.from_numpy(z["kv_cache"].reshape(nb, -1)).to(dev)
    kv = torch.as_strided(big, (nb, 16, 8, 134), (17152 + 256, 8 * 134, 134, 1))
    qbig = torch.zeros(2, 40, 128, device=dev)
    qbig[:, :32] = torch.from_numpy(z["q_rot"]).to(dev)
    q = qbig[:, :32]
    midbig = torch.full((2, 32, 6, 140), SENTINEL, device=dev)
    mid = midbig[:, :, :4, :129]
    tqb.stage1(q, kv, torch.from_numpy(z["block_table"]).to(dev), torch.from_numpy(z["seq_lens"]).to(dev),
               torch.from_numpy(z["centroids"]).to(dev), mid)
    torch.cuda.synchronize()
    ref = O.stage1(z["q_rot"], z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], 4)
    _check(mid.cpu().numpy(), ref, "strided")
    assert torch.all(midbig[:, :, 4:] == SENTINEL) and torch.all(midbig[..., 129:] == SENTINEL)


@pytest.mark.parametrize("name", ["c0", "ragged_gqa4"])
@pytest.mark.parametrize("layout", ["soa", "aos"])
def test_vllm_transposed_cache_view(cuda_device, golden, name, layout):
    """The cache as vLLM hands it over: ``(blocks, H, N, C)`` storage seen
    through ``kv_cache.transpose(1, 2)`` (reference/turboquant_attn.py:565),
    through the reference-named launcher.  An SoA block is raw bytes from its
    base (the reference reads only ``kv_cache.stride(0)``), so the reference
    bytes under the transposed view give the reference output; AoS reads
    slot (t, h) through the view's strides (head-major here), so the
    head-major copy of the reference AoS cache gives the reference AoS
    output."""
    z = golden[name]
    dev = cuda_device
    if layout == "soa":
        kv = z["kv_cache"]
        nb, bs, hk, slot = kv.shape
        storage = torch.from_numpy(kv.reshape(nb, hk, bs, slot).copy()).to(dev)
        ref = z["mid_o_soa_v1"]
    else:
        kv = z["kv_cache_aos"]
        storage = torch.from_numpy(kv.transpose(0, 2, 1, 3).copy()).to(dev)
        ref = z["mid_o_aos_v1"]
    view = storage.transpose(1, 2)
    assert not view.is_contiguous() and tuple(view.shape) == kv.shape
    S = int(z["num_splits"])
    q = _to(dev, z, "q_rot")
    mid = torch.full((q.shape[0], q.shape[1], S, q.shape[2] + 1), SENTINEL, device=dev)
    tqb.stage1(q, view, _to(dev, z, "block_table"), _to(dev, z, "seq_lens"), _to(dev, z, "centroids"), mid,
               layout=layout)
    torch.cuda.synchronize()
    _check(mid.cpu().numpy(), ref, f"{name} {layout} vLLM view")


def test_large_magnitudes(cuda_device):
    """Query magnitudes far from 1 (power-of-two scaling keeps the fp16
    operand split exact) and large V scales."""
    z = random_case(21, 2, 32, 8, [256, 100])
    S = 4
    for scale in (1e-3, 30.0):
        z2 = dict(z, q_rot=(z["q_rot"] * scale).astype(np.float32))
        ref = O.stage1(z2["q_rot"], z2["kv_cache"], z2["block_table"], z2["seq_lens"], z2["centroids"], S)
        _check(_run(cuda_device, z2, S=S), ref, f"q scale {scale}")


def test_errors_raise(cuda_device, golden):
    z = golden["c0"]
    dev = cuda_device
    q = _to(dev, z, "q_rot")
    kv = _to(dev, z, "kv_cache")
    bt, sl, c = _to(dev, z, "block_table"), _to(dev, z, "seq_lens"), _to(dev, z, "centroids")
    mid = torch.empty(2, 32, 4, 129, device=dev)
    with pytest.raises(tqb.TqbError):
        tqb.stage1(q.double(), kv, bt, sl, c, mid)
    with pytest.raises(tqb.TqbError):
        tqb.stage1(q, kv, bt, sl, c, torch.empty(2, 32, 4, 128, device=dev))
    with pytest.raises(tqb.TqbError):
        tqb.stage1(q[:, :30], kv, bt, sl, c, torch.empty(2, 30, 4, 129, device=dev))


@pytest.mark.parametrize("layout,qdtype", [("soa", torch.float32), ("soa", torch.bfloat16),
                                            ("aos", torch.float32), ("aos", torch.float16)])
def test_decode_launcher_vs_oracle(cuda_device, layout, qdtype):
    """The production launchers (reference/soa_decode_v1.py and
    reference/aos_decode.py ``triton_turboquant_decode_attention``): fused
    query cast + rotation, Stage1, Stage2 into the query's dtype, against the
    oracle's Stage1 + Stage2 on ``query.float() @ PiT``."""
    from tqb import compat, compat_aos
    dev = cuda_device
    lens = [300, 17, 1024, 0, 555]
    z = random_case(41 + (layout == "aos"), len(lens), 32, 8, lens, layout=layout)
    rng = np.random.default_rng(3)
    Pi = np.linalg.qr(rng.standard_normal((128, 128)))[0].astype(np.float32)
    query = torch.from_numpy(rng.standard_normal((len(lens), 32, 128)).astype(np.float32)).to(qdtype)
    q_rot = (query.float() @ torch.from_numpy(Pi).T).numpy()
    S = 8
    mid = O.stage1(q_rot, z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], S,
                   layout=O.LAYOUT_SOA if layout == "soa" else O.LAYOUT_AOS)
    ref_out, ref_lse = O.stage2(mid, z["seq_lens"])
    fn = compat.triton_turboquant_decode_attention if layout == "soa" else \
        compat_aos.triton_turboquant_decode_attention
    lse = torch.empty(len(lens), 32, device=dev)
    out = fn(query.to(dev), _to(dev, z, "kv_cache"), _to(dev, z, "block_table"), _to(dev, z, "seq_lens"),
             torch.from_numpy(Pi).to(dev), _to(dev, z, "centroids"), 1.0 / math.sqrt(128), 4, 66, 4,
             norm_correction=True, max_num_kv_splits=S, lse_buf=lse)
    torch.cuda.synchronize()
    assert out.dtype == qdtype and tuple(out.shape) == (len(lens), 32, 128)
    live = np.asarray(lens) > 0
    got = out.float().cpu().numpy()
    ref = ref_out.astype(np.float32)
    if qdtype == torch.float32:
        assert_close(got[live], ref[live], what=f"{layout} decode out")
    else:  # the fp32 result rounded to 16 bits: one unit in the last place more
        ulp = 2.0 ** -7 if qdtype == torch.bfloat16 else 2.0 ** -10
        assert_close(got[live], torch.from_numpy(ref[live]).to(qdtype).float().numpy(),
                     rtol=RTOL + ulp, what=f"{layout} decode out")
    assert_close(lse.cpu().numpy()[live], ref_lse[live], what=f"{layout} decode lse")
    assert np.all(np.isnan(got[~live])), "a sequence without tokens gets NaN, as in the reference"


@pytest.mark.parametrize("layout", ["soa", "aos"])
def test_decode_launcher_sinks_vs_oracle(cuda_device, layout):
    """``triton_turboquant_decode_attention(..., sinks=...)`` with bf16 sink
    logits (cast to float32 as the reference does) against the float64
    oracle with the sinks in split 0, then Stage2; an empty sequence stays
    NaN (no split is written, so no sink either)."""
    from tqb import compat
    dev = cuda_device
    lens = [300, 17, 0, 555]
    z = random_case(43 + (layout == "aos"), len(lens), 32, 8, lens, layout=layout)
    rng = np.random.default_rng(5)
    Pi = np.linalg.qr(rng.standard_normal((128, 128)))[0].astype(np.float32)
    query = torch.from_numpy(rng.standard_normal((len(lens), 32, 128)).astype(np.float32))
    sinks = torch.from_numpy((rng.standard_normal(32) * 3.0).astype(np.float32)).to(torch.bfloat16)
    sinks[5] = float("-inf")
    q_rot = (query @ torch.from_numpy(Pi).T).numpy()
    S = 6
    mid = O.stage1_np(q_rot, z["kv_cache"], z["block_table"], z["seq_lens"], z["centroids"], S,
                      layout=O.LAYOUT_SOA if layout == "soa" else O.LAYOUT_AOS, sinks=sinks.float().numpy())
    ref_out, ref_lse = O.stage2_np(mid, z["seq_lens"])
    lse = torch.empty(len(lens), 32, device=dev)
    out = compat.decode_attention(query.to(dev), _to(dev, z, "kv_cache"), _to(dev, z, "block_table"),
                                  _to(dev, z, "seq_lens"), torch.from_numpy(Pi).to(dev), _to(dev, z, "centroids"),
                                  1.0 / math.sqrt(128), layout, max_num_kv_splits=S, lse_buf=lse,
                                  sinks=sinks.to(dev))
    torch.cuda.synchronize()
    live = np.asarray(lens) > 0
    assert_close(out.cpu().numpy()[live], ref_out[live], what=f"{layout} decode with sinks out")
    assert_close(lse.cpu().numpy()[live], ref_lse[live], what=f"{layout} decode with sinks lse")
    assert np.all(np.isnan(out.cpu().numpy()[~live]))


def test_decode_launcher_cuda_graph_workspace(cuda_device):
    """vLLM's decode use of ``triton_turboquant_decode_attention``
    (reference/turboquant_attn.py:1125-1141, 368-373): workspace buffers for
    mid_o, the output (in the query's dtype) and the LSE, a fixed split
    count, the call captured once in a CUDA graph and replayed with new
    queries and sequence lengths written into the captured input tensors.
    The result lands in the caller's output buffer, and every replay matches
    the oracle for that replay's inputs."""
    from tqb import compat
    dev = cuda_device
    lens = [300, 17, 1024, 555]
    B, Hq, S = len(lens), 32, 8
    z = random_case(47, B, Hq, 8, lens)
    rng = np.random.default_rng(9)
    Pi = np.linalg.qr(rng.standard_normal((128, 128)))[0].astype(np.float32)
    PiT = torch.from_numpy(Pi).T.contiguous()
    kv, bt, cents = _to(dev, z, "kv_cache"), _to(dev, z, "block_table"), _to(dev, z, "centroids")
    Pi_d, PiT_d = torch.from_numpy(Pi).to(dev), PiT.to(dev)
    q_in = torch.zeros(B, Hq, 128, dtype=torch.bfloat16, device=dev)
    sl_in = _to(dev, z, "seq_lens")
    mid_ws = torch.empty(B, Hq, S, 129, device=dev)
    out_ws = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=dev)
    lse_ws = torch.empty(B, Hq, device=dev)

    def call():
        return compat.triton_turboquant_decode_attention(
            q_in, kv, bt, sl_in, Pi_d, cents, 1.0 / math.sqrt(128), 4, 66, 4,
            norm_correction=True, PiT=PiT_d, mid_o_buf=mid_ws, output_buf=out_ws, lse_buf=lse_ws,
            max_num_kv_splits=S)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        call()  # eager warm-up (one-time kernel attribute set-up)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = call()
    assert out.data_ptr() == out_ws.data_ptr(), "the result must land in the workspace buffer"
    # each replay's lengths stay within the tokens stored for that sequence
    # (slots past them hold random bytes, NaN norms included)
    for trial, new_lens in enumerate(([300, 17, 1024, 555], [129, 1, 700, 0], [16, 9, 1023, 300])):
        query = torch.from_numpy(rng.standard_normal((B, Hq, 128)).astype(np.float32)).to(torch.bfloat16)
        q_in.copy_(query.to(dev))
        sl_in.copy_(torch.tensor(new_lens, dtype=torch.int32))
        graph.replay()
        torch.cuda.synchronize(dev)
        q_rot = (query.float() @ PiT).numpy()
        mid = O.stage1(q_rot, z["kv_cache"], z["block_table"], np.asarray(new_lens, np.int32), z["centroids"], S)
        ref_out, ref_lse = O.stage2(mid, np.asarray(new_lens, np.int32))
        live = np.asarray(new_lens) > 0
        got = out_ws.float().cpu().numpy()
        ref = torch.from_numpy(ref_out[live].astype(np.float32)).to(torch.bfloat16).float().numpy()
        assert_close(got[live], ref, rtol=RTOL + 2.0 ** -7, what=f"graph replay {trial} out")
        assert_close(lse_ws.cpu().numpy()[live], ref_lse[live], what=f"graph replay {trial} lse")
    del graph
