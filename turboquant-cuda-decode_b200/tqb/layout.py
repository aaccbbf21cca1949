"""TurboQuant ``turboquant_4bit_nc`` paged-cache layout.

Physical cache tensor: ``uint8[num_blocks, block_size=16, Hk, 134]``
(reference: baseline/common.py:56-224, reference/config.py:127-174).

SoA block (reference/soa_store.py:286-300, reference/soa_decode_v1.py:168-188)::

    byte 0                     data region  [16 tokens][Hk][K 64 B | V 64 B]
    byte 16*Hk*128             meta region  [Hk][3 fields][16 tokens] fp16
                               field 0 = K norm with 1/|c| folded in
                               field 1 = V scale, field 2 = V zero

AoS slot (reference/aos_decode.py:148-152,213-299)::

    [K 64 B | raw K norm fp16 | V 64 B | V scale fp16 | V zero fp16]

Packed 4-bit codes: byte j holds dim 2j in the low nibble and dim 2j+1 in
the high nibble (reference/soa_store.py:319-325).
"""

from __future__ import annotations

HEAD_DIM = 128
BLOCK_SIZE = 16
MSE_BITS = 4
VALUE_BITS = 4
N_CENTROIDS = 1 << MSE_BITS
MSE_BYTES = HEAD_DIM * MSE_BITS // 8          # 64
VAL_DATA_BYTES = HEAD_DIM * VALUE_BITS // 8   # 64
KEY_DATA_BYTES = MSE_BYTES
DATA_BYTES_PER_SLOT = KEY_DATA_BYTES + VAL_DATA_BYTES  # 128
NUM_SOA_FIELDS = 3
SOA_K_NORM, SOA_V_SCALE, SOA_V_ZERO = 0, 1, 2
SLOT_SIZE = DATA_BYTES_PER_SLOT + 2 * NUM_SOA_FIELDS   # 134
SLOT_SIZE_ALIGNED = SLOT_SIZE + SLOT_SIZE % 2          # 134
AOS_KEY_PACKED_SIZE = MSE_BYTES + 2                    # 66

LAYOUT_SOA = 0
LAYOUT_AOS = 1
# turboquant_k8v4: e4m3 keys (128 B) + 4-bit values (64 B) per token-head,
# meta region [Hk][2][16] fp16 (vscale, vzero): 196 bytes per token-head
LAYOUT_SOA_K8 = 2
K8_KEY_BYTES = HEAD_DIM
K8_SLOT_SIZE = HEAD_DIM + VAL_DATA_BYTES + 4  # 196
# turboquant_k3v4_nc: 3-bit keys (48 B, dim d at bit 3d) + 4-bit values,
# meta region [Hk][3][16] fp16 (knorm, vscale, vzero): 118 bytes per token-head
LAYOUT_SOA_K3 = 3
K3_KEY_BYTES = HEAD_DIM * 3 // 8
K3_SLOT_SIZE = K3_KEY_BYTES + VAL_DATA_BYTES + 6  # 118
# turboquant_3bit_nc: 3-bit keys and 3-bit values (48 + 48 B), same meta
LAYOUT_SOA_K3V3 = 4
K3V3_SLOT_SIZE = K3_KEY_BYTES + HEAD_DIM * 3 // 8 + 6  # 102
# AoS forms of the three presets (reference/aos_store.py:26-340): one slot per
# (token, KV head), [key codes | raw fp16 norm (Lloyd-Max keys) | value codes
# | fp16 vscale | fp16 vzero], the same byte counts as their SoA forms
LAYOUT_AOS_K8 = 5    # 128 e4m3 key bytes, no norm, 64 value bytes: 196
LAYOUT_AOS_K3 = 6    # 48 key bytes, norm, 64 value bytes: 118
LAYOUT_AOS_K3V3 = 7  # 48 key bytes, norm, 48 value bytes: 102
AOS_FAMILY = (LAYOUT_AOS, LAYOUT_AOS_K8, LAYOUT_AOS_K3, LAYOUT_AOS_K3V3)
FP8_KEY_LAYOUTS = (LAYOUT_SOA_K8, LAYOUT_AOS_K8)
KEY3_LAYOUTS = (LAYOUT_SOA_K3, LAYOUT_SOA_K3V3, LAYOUT_AOS_K3, LAYOUT_AOS_K3V3)
SLOT_BYTES = {LAYOUT_SOA: SLOT_SIZE, LAYOUT_AOS: SLOT_SIZE, LAYOUT_SOA_K8: K8_SLOT_SIZE,
              LAYOUT_SOA_K3: K3_SLOT_SIZE, LAYOUT_SOA_K3V3: K3V3_SLOT_SIZE, LAYOUT_AOS_K8: K8_SLOT_SIZE,
              LAYOUT_AOS_K3: K3_SLOT_SIZE, LAYOUT_AOS_K3V3: K3V3_SLOT_SIZE}


def layout_id(layout) -> int:
    if layout in (LAYOUT_SOA, "soa", "SoA", "SOA"):
        return LAYOUT_SOA
    if layout in (LAYOUT_AOS, "aos", "AoS", "AOS"):
        return LAYOUT_AOS
    if layout in (LAYOUT_SOA_K8, "soa_k8", "k8v4"):
        return LAYOUT_SOA_K8
    if layout in (LAYOUT_SOA_K3, "soa_k3", "k3v4"):
        return LAYOUT_SOA_K3
    if layout in (LAYOUT_SOA_K3V3, "soa_k3v3", "3bit"):
        return LAYOUT_SOA_K3V3
    if layout in (LAYOUT_AOS_K8, "aos_k8"):
        return LAYOUT_AOS_K8
    if layout in (LAYOUT_AOS_K3, "aos_k3"):
        return LAYOUT_AOS_K3
    if layout in (LAYOUT_AOS_K3V3, "aos_k3v3"):
        return LAYOUT_AOS_K3V3
    raise ValueError(f"unknown cache layout {layout!r} (expected 'soa', 'aos', 'soa_k8', 'soa_k3', 'soa_k3v3', "
                     "'aos_k8', 'aos_k3' or 'aos_k3v3')")


def block_bytes(num_kv_heads: int, block_size: int = BLOCK_SIZE) -> int:
    """Bytes of one physical block: block_size * Hk * 134."""
    return block_size * num_kv_heads * SLOT_SIZE_ALIGNED


def data_region_bytes(num_kv_heads: int, block_size: int = BLOCK_SIZE) -> int:
    return block_size * num_kv_heads * DATA_BYTES_PER_SLOT


def meta_region_offset(num_kv_heads: int, block_size: int = BLOCK_SIZE) -> int:
    """Byte offset of the SoA metadata region inside a block."""
    return data_region_bytes(num_kv_heads, block_size)


def meta_region_bytes(num_kv_heads: int, block_size: int = BLOCK_SIZE) -> int:
    return num_kv_heads * NUM_SOA_FIELDS * block_size * 2


def split_range(seq_len: int, num_splits: int, split: int) -> tuple[int, int]:
    """Token range of a KV split (reference/soa_decode_v1.py:104-107)."""
    split_len = -(-seq_len // num_splits) if num_splits > 0 else 0
    start = split_len * split
    return start, min(start + split_len, seq_len)


def splits_per_sequence(seq_lens, tokens_per_split: int = 512, max_splits: int = 32):
    """Per-sequence split counts ceil(len / tokens_per_split) capped at
    ``max_splits`` (the ragged-batch policy; at least one split each)."""
    return [max(1, min(max_splits, -(-int(n) // tokens_per_split))) for n in seq_lens]
