"""LRU paging of adapters over the pool's slots (CPU): residency, eviction
order, slot contents after a reload, zeroing of modules the new adapter
lacks, PEFT directories as sources, and the errors."""

import pytest
import torch

from peft_fixture import GEOM as MISTRAL, write_adapter
from persona.adapter_pool import AdapterCache, AdapterPool, MODULE_POOLS

GEOM = (128, 64, 256)  # hidden, k/v out, MLP intermediate
R, LAYERS = 4, 2
DIMS = {"q_proj": (128, 128), "k_proj": (128, 64), "v_proj": (128, 64), "o_proj": (128, 128),
        "gate_proj": (128, 256), "up_proj": (128, 256), "down_proj": (256, 128)}


def _adapter(seed, modules=tuple(DIMS)):
    g = torch.Generator().manual_seed(seed)
    return {li: {m: (torch.randn(R, DIMS[m][0], generator=g).half(), torch.randn(DIMS[m][1], R, generator=g).half())
                 for m in modules} for li in range(LAYERS)}


def _pool(slots=3):
    return AdapterPool(max_slots=slots, r=R, device=torch.device("cpu"), num_layers=LAYERS, geometry=GEOM)


def _check_slot(pool, slot, layers):
    for li in range(LAYERS):
        for m in DIMS:
            a = pool.a_pool(li, m)[slot]
            b = pool.b_pool(li, m)[slot]
            if m in layers[li]:
                assert torch.equal(a, layers[li][m][0]) and torch.equal(b, layers[li][m][1])
            else:
                assert torch.all(a == 0) and torch.all(b == 0)


def test_lru_eviction_reload_and_stats():
    pool = _pool(3)
    cache = AdapterCache(pool)
    ads = {f"p{i}": _adapter(i, tuple(DIMS) if i != 3 else ("q_proj", "down_proj")) for i in range(5)}
    for n, layers in ads.items():
        cache.register(n, layers=layers)
    s = cache.acquire(["p0", "p1", "p2"])
    assert len(set(s)) == 3 and cache.resident == ["p0", "p1", "p2"]
    cache.acquire(["p0"])                      # p0 becomes the most recent
    s3 = cache.acquire(["p3", "p0"])           # evicts p1, the least recently used
    assert "p1" not in cache.resident and cache.resident[-2:] == ["p3", "p0"]
    assert s3[1] == s[0] and s3[0] == s[1]     # p3 took p1's slot
    _check_slot(pool, s3[0], ads["p3"])        # p1's other modules were cleared
    s4 = cache.acquire(["p4", "p1", "p1"])     # repeats map to one slot
    assert s4[1] == s4[2]
    for n in ("p4", "p1", "p0", "p3", "p2"):
        if n in cache.resident:
            _check_slot(pool, pool.name_to_slot[n], ads[n])
    assert cache.misses == 6 and cache.hits == 2 and cache.evictions == 3
    assert len(cache.resident) == 3 and set(pool.name_to_slot) == set(cache.resident)


def test_batch_larger_than_pool_and_unknown_names():
    pool = _pool(2)
    cache = AdapterCache(pool)
    for i in range(3):
        cache.register(f"p{i}", layers=_adapter(i))
    with pytest.raises(RuntimeError, match="does not fit"):
        cache.acquire(["p0", "p1", "p2"])
    with pytest.raises(KeyError):
        cache.acquire(["nope"])
    with pytest.raises(ValueError):
        cache.register("x")
    # a slot held by an adapter loaded into the pool directly is never evicted
    pool2 = _pool(1)
    pool2.load_random_adapter("fixed", generator=torch.Generator().manual_seed(0))
    c2 = AdapterCache(pool2)
    c2.register("p0", layers=_adapter(0))
    with pytest.raises(RuntimeError, match="no slot can be freed"):
        c2.acquire(["p0"])


def test_peft_directory_source_matches_pool_loader(tmp_path):
    """An adapter registered from a PEFT directory lands in its slot, after
    an eviction, with the bytes AdapterPool.load_adapter writes."""
    d, _ = write_adapter(tmp_path / "a", r=R, alpha=8, modules=("q_proj", "v_proj", "down_proj"), layers=(0, 1),
                         seed=3)
    direct = AdapterPool(max_slots=1, r=R, device=torch.device("cpu"), num_layers=LAYERS)
    direct.load_adapter("a", d)
    pool = AdapterPool(max_slots=1, r=R, device=torch.device("cpu"), num_layers=LAYERS)
    cache = AdapterCache(pool)
    cache.register("a", adapter_dir=d)
    g = torch.Generator().manual_seed(9)
    k_in, n_out = MISTRAL["o_proj"]
    cache.register("b", layers={li: {"o_proj": (torch.randn(R, k_in, generator=g).half(),
                                                torch.randn(n_out, R, generator=g).half())} for li in range(LAYERS)})
    cache.acquire(["b"])
    slot = cache.acquire(["a"])[0]  # evicts b; its o_proj must not survive
    assert cache.evictions == 1
    for li in range(LAYERS):
        for m in MISTRAL:
            assert torch.equal(pool.a_pool(li, m)[slot], direct.a_pool(li, m)[0])
            assert torch.equal(pool.b_pool(li, m)[slot], direct.b_pool(li, m)[0])
    assert MODULE_POOLS["q_proj"][0] == "A_qkv"
