"""AoS-cache decode launcher under the reference's name and signature.

``reference/aos_decode.py`` defines its own ``triton_turboquant_decode_attention``
for the AoS cache (the SoA one lives in ``reference/soa_decode_v1.py``); a call
site that imports the AoS one switches to::

    from tqb.compat_aos import triton_turboquant_decode_attention

The AoS Stage1 kernels implement the norm-corrected decode of the
``turboquant_4bit_nc`` preset (the reference's ``NORM_CORRECTION=1``, as
``baseline/triton_v1.py`` launches it); other presets raise
``NotImplementedError``.
"""

from __future__ import annotations

from typing import Any, Optional

import torch

from .compat import decode_attention


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
    """Decode over an AoS cache ``[num_blocks, 16, Hk, 134]``; returns
    ``[B, Hq, D]`` in the query's dtype."""
    if key_fp8 or mse_bits != 4 or value_quant_bits != 4:
        raise NotImplementedError("the AoS cache serves the turboquant_4bit_nc preset; the FP8-key and 3-bit "
                                  "presets use the SoA cache (tqb.compat.triton_turboquant_decode_attention)")
    if not norm_correction:
        raise NotImplementedError("the AoS kernels implement the norm-corrected decode (norm_correction=True) "
                                  "of the turboquant_4bit_nc preset")
    return decode_attention(query, kv_cache, block_table, seq_lens, Pi, centroids, scale, "aos", PiT=PiT,
                            mid_o_buf=mid_o_buf, output_buf=output_buf, lse_buf=lse_buf, buf_holder=buf_holder,
                            max_num_kv_splits=max_num_kv_splits)
