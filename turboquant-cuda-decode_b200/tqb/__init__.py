"""tqb — B200-native TurboQuant ``turboquant_4bit_nc`` decode attention.

Hot path: decode Stage1 (split-KV partial attention over the 4-bit paged
K/V cache), its Stage2 LSE merge, the cross-GPU merge, and the cache store,
all as hand-written sm_100a kernels in ``libtqb.so`` behind a C ABI
(``include/tqb.h``).  This package is the host side: ctypes bindings
(``tqb._lib``), torch-facing calls (``tqb.ops``), the reference-named
drop-in launchers (``tqb.compat``), the cache layout (``tqb.layout``), the
codebook (``tqb.codebook``) and multi-GPU sharding (``tqb.sharding``).
"""

from ._lib import TqbError, version, wait_timeouts  # noqa: F401
from .codebook import build_pair_lut, get_centroids, get_midpoints  # noqa: F401
from .compat import (  # noqa: F401
    convert_soa_to_aos_kv_cache,
    launch_aos_v1_stage1,
    launch_soa_v1_stage1,
    launch_stage2,
    launch_tq4_v2_stage1,
    tq4_cuda_full,
    tq4_cuda_stage1,
    tq4_cuda_stage2,
    triton_turboquant_decode_attention,
    triton_turboquant_store,
)
from .ops import fold_sinks, merge_partials, rotate_query, stage1, stage2, store  # noqa: F401
from . import compat_aos  # noqa: F401
