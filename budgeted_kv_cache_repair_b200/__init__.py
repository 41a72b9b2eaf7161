"""B200-native packed refresh executor for budgeted KV-cache repair.

Drop-in for the packed path of yh0903/budgeted-kv-cache-repair: the same
``repair_after_deletion`` / ``select_support`` / ``packed_interval_repair`` /
``IndexedPlan`` surface and ``DynamicCache`` results, computed by hand-written
sm_100a kernels behind the C ABI in ``include/kvr_b200.h`` (libkvr_b200.so)
with cuBLAS projections. CUDA only; no CPU or eager fallback.
"""

from .alignment import token_alignment
from .api import RepairResult, Selection, positions_to_intervals, repair_after_deletion, select_support
from .cache import OperatorShim, build_halo_cache, clone_cache, merge_intervals, rotate_half, shifted_suffix_keys
from .indexed import indexed_causal_attention, indexed_kv_scatter_
from .packed import packed_interval_repair
from .plan import BLOCK_M, BLOCK_N, DeviceIndexedPlan, IndexedPlan

__all__ = [
    "BLOCK_M", "BLOCK_N", "DeviceIndexedPlan", "IndexedPlan", "OperatorShim", "RepairResult", "Selection",
    "build_halo_cache", "clone_cache", "indexed_causal_attention", "indexed_kv_scatter_", "merge_intervals",
    "packed_interval_repair", "positions_to_intervals", "repair_after_deletion", "rotate_half",
    "select_support", "shifted_suffix_keys", "token_alignment",
]
