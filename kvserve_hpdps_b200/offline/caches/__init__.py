"""Offline KV caches for Hugging Face models: KVServe's hybrid-precision
cache and the KIVI, CacheGen and DuoAttention baselines, used to measure
accuracy and compression ratio of a configuration before it enters a
profile library."""

from kvserve_hpdps_b200.offline.caches.baselines import (CacheGenCache, CacheGenCacheConfig,
                                                         DuoAttentionCache, DuoAttentionCacheConfig,
                                                         KIVICache, KIVICacheConfig,
                                                         cachegen_bins, enable_query_capture,
                                                         search_hyperplane)
from kvserve_hpdps_b200.offline.caches.custom import CustomCache, CustomCacheConfig
from kvserve_hpdps_b200.offline.caches.transforms import (AffineTransform, HeadHadamard,
                                                          NoneTransform, make_transform)

__all__ = ["CustomCache", "CustomCacheConfig", "KIVICache", "KIVICacheConfig", "CacheGenCache",
           "CacheGenCacheConfig", "DuoAttentionCache", "DuoAttentionCacheConfig",
           "enable_query_capture", "search_hyperplane", "cachegen_bins", "AffineTransform",
           "HeadHadamard", "NoneTransform", "make_transform"]
