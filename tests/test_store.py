"""The per-token cache store: the oracle against the reference's torch store path (golden), on CPU."""

import numpy as np

from oracle.kv_oracle import store_kvcache, store_latents


def test_the_oracle_store_matches_the_reference_on_nhd_and_hnd_caches(golden):
    meta, arrays = golden
    slots = arrays["store_slots"]
    key, value = arrays["store_key"], arrays["store_value"]
    for layout in ("NHD", "HND"):
        cache = arrays[f"store_{layout}_before"].copy()
        view = cache if layout == "NHD" else cache.swapaxes(2, 3)  # (2, blocks, block, heads, dim) either way
        store_kvcache(key, value, view[0], view[1], slots)
        assert np.array_equal(cache, arrays[f"store_{layout}_after"]), layout


def test_the_oracle_latent_store_matches_the_reference(golden):
    _, arrays = golden
    cache = arrays["store_latent_before"].copy()
    store_latents(arrays["store_latent"], cache[0], arrays["store_slots"])
    assert np.array_equal(cache, arrays["store_latent_after"])


def test_padding_slots_leave_the_cache_alone(golden):
    _, arrays = golden
    cache = arrays["store_NHD_before"].copy()
    store_kvcache(arrays["store_key"], arrays["store_value"], cache[0], cache[1], np.full(10, -1))
    assert np.array_equal(cache, arrays["store_NHD_before"])
