"""AoS-cache decode launcher under the reference's name and signature.

``reference/aos_decode.py`` defines its own ``triton_turboquant_decode_attention``
for the AoS cache (the SoA one lives in ``reference/soa_decode_v1.py``); a call
site that imports the AoS one switches to::

    from tqb.compat_aos import triton_turboquant_decode_attention

Every preset of ``reference/config.py:20-41`` is served on its AoS slot
layout: ``turboquant_4bit_nc`` (the default), FP8 keys (``key_fp8=True``,
``turboquant_k8v4``), 3-bit keys with 4-bit or 3-bit values (``mse_bits=3``,
``turboquant_k3v4_nc`` / ``turboquant_3bit_nc``).  The Lloyd-Max presets
are decoded with the in-kernel norm correction (the reference's
``NORM_CORRECTION=1``, as ``baseline/triton_v1.py`` launches it), so
``norm_correction=False`` raises ``NotImplementedError``.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

from .compat import _preset_layout, decode_attention


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
) -> torch.Tensor:
    """Decode over an AoS cache ``[num_blocks, 16, Hk, slot]`` (slot 134,
    196, 118 or 102 bytes by preset); returns ``[B, Hq, D]`` in the query's
    dtype."""
    layout = _preset_layout(key_fp8, mse_bits, value_quant_bits, "aos")
    if not key_fp8 and not norm_correction:
        raise NotImplementedError("the AoS kernels implement the norm-corrected decode (norm_correction=True) "
                                  "of the Lloyd-Max presets")
    return decode_attention(query, kv_cache, block_table, seq_lens, Pi, centroids, scale, layout, PiT=PiT,
                            mid_o_buf=mid_o_buf, output_buf=output_buf, lse_buf=lse_buf, buf_holder=buf_holder,
                            max_num_kv_splits=max_num_kv_splits)
