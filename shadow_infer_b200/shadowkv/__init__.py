"""ShadowKV packed-KV data plane on B200 (drop-in for ``shadowinfer.shadowkv``'s data plane)."""

from .kv_cache_manager import (
    EvictionPolicy,
    ImportanceAgeEvictionPolicy,
    KVCacheEntry,
    KVCacheManager,
    LeastImportantEvictionPolicy,
    TokenHeadScore,
)
from .importance_model import compute_irap_importance
from .packed_attention import packed_attention, packed_block_forward
from .packed_kv_cache import PackedKVCache
from .paged_kv_store import PagedKVStore
from .precision_plan import (
    CODE_PRECISIONS,
    EVICTED,
    PRECISION_CODES,
    PRECISION_ORDER,
    PrecisionPlan,
    codes_to_map,
    map_to_codes,
)
from .rd_allocator import admit_budget, admit_codes, entry_bytes, kv_sensitivity, predict_codes_bytes

__all__ = [
    "PackedKVCache", "PrecisionPlan", "map_to_codes", "codes_to_map", "PRECISION_ORDER", "PRECISION_CODES",
    "CODE_PRECISIONS", "EVICTED", "admit_codes", "admit_budget", "entry_bytes", "kv_sensitivity",
    "predict_codes_bytes", "packed_attention", "packed_block_forward", "KVCacheManager", "KVCacheEntry", "TokenHeadScore",
    "EvictionPolicy", "LeastImportantEvictionPolicy", "ImportanceAgeEvictionPolicy", "PagedKVStore",
    "compute_irap_importance",
]
