"""CPU tests of the quantized prefix store: the reference's restore-plan,
reusable-prefix and hash rules (golden vectors written by the reference's
own OnDiskPrefixKVStore, tests/golden/make_prefix_golden.py), and a
bit-exact save / lookup / load round trip of quantized pages."""
import json
from pathlib import Path

import pytest
import torch

from aether_kernels.paged import TurboQuantPagedCache
from aether_kernels.prefix_store import (HybridCacheLayout, LayerPages, QuantizedPrefixStore, RestorePlan,
                                         SWACacheMode)

GOLDEN = Path(__file__).resolve().parent / "golden" / "prefix_store_plans.json"


def test_policy_matches_reference_golden(tmp_path):
    cases = json.loads(GOLDEN.read_text())
    assert len(cases) > 200
    stores = {}
    for c in cases:
        key = (tuple(c["layout"]), c["mode"], c["stride"])
        if key not in stores:
            stores[key] = QuantizedPrefixStore(str(tmp_path / str(len(stores))), HybridCacheLayout(*c["layout"]),
                                               swa_mode=SWACacheMode(c["mode"]), checkpoint_stride=c["stride"])
        st = stores[key]
        n = c["tokens"]
        assert st.layout.block_tokens == c["block_tokens"]
        assert st.layout.full_block_prefix(n) == c["reusable"]
        tokens = [(37 * i + 11) % 50000 for i in range(n)]
        if c["reusable"] > 0:
            assert st.prefix_hash(tokens[: c["reusable"]]) == c["hash"]
        assert st.make_restore_plan(n) == RestorePlan(**c["plan"]), c


def _cache(num_pages, bits, seed):
    c = TurboQuantPagedCache(num_pages, bits, "cpu")
    g = torch.Generator().manual_seed(seed)
    c.kv_pages.copy_(torch.randint(0, 256, c.kv_pages.shape, generator=g, dtype=torch.uint8))
    c.idx_pages.copy_(torch.randint(0, 256, c.idx_pages.shape, generator=g, dtype=torch.uint8))
    return c


@pytest.mark.parametrize("mode", list(SWACacheMode))
def test_round_trip_pages_bit_exact(tmp_path, mode):
    layout = HybridCacheLayout(4, 128, 128, 2)
    store = QuantizedPrefixStore(str(tmp_path), layout, swa_mode=mode, checkpoint_stride=256)
    g = torch.Generator().manual_seed(3)
    src = {"l0": _cache(40, 4, 1), "l1": _cache(40, 8, 2)}
    tokens = list(range(1000, 1000 + 900))  # 896 reusable tokens -> 224 CSA blocks
    layers = {}
    for name, c in src.items():
        nb = layout.full_block_prefix(len(tokens)) // 4
        ids = torch.randperm(40, generator=g)[: (nb + 63) // 64].tolist()
        layers[name] = LayerPages(c, ids, nb)
    swa = {"window": torch.randn(2, 128, 16, generator=g)}
    md = store.save_prefix(tokens, layers, swa_state=swa)
    assert md.reusable_token_count == 896 and md.prefix_token_count == 900
    # a longer request with the same reusable prefix finds it
    found = store.lookup_prefix(tokens + [5, 6, 7])
    assert found is not None and found.prefix_hash == md.prefix_hash
    assert store.lookup_prefix(tokens[:896] + [1] * 4) is not None  # same 896-token prefix, other tail
    assert store.lookup_prefix([9] * 900) is None
    dst = {"l0": TurboQuantPagedCache(50, 4, "cpu"), "l1": TurboQuantPagedCache(50, 8, "cpu")}
    rows = store.load_pages(found, dst, generator=torch.Generator().manual_seed(9))
    for name, lp in layers.items():
        table, nb = rows[name]
        assert nb == lp.nblocks
        for stream in ("kv_pages", "idx_pages"):
            a = getattr(src[name], stream)[torch.tensor(lp.page_ids)]
            b = getattr(dst[name], stream)[table.long()]
            assert torch.equal(a, b), (name, stream)
    state = store.load_swa_state(found)
    if mode == SWACacheMode.ZERO:
        assert state is None
    else:
        assert torch.equal(state["window"], swa["window"])
    if mode == SWACacheMode.PERIODIC:
        assert any("swa_ckpt_768" in f for f in found.files.values())


def test_layout_and_format_checks(tmp_path):
    store = QuantizedPrefixStore(str(tmp_path), HybridCacheLayout(4, 128, 128, 2))
    c = _cache(8, 4, 5)
    with pytest.raises(ValueError, match="does not contain a full compression block"):
        store.save_prefix(list(range(100)), {"l": LayerPages(c, [0], 25)})
    md = store.save_prefix(list(range(128)), {"l": LayerPages(c, [3], 32)})
    other = QuantizedPrefixStore(str(tmp_path), HybridCacheLayout(4, 128, 64, 2))
    with pytest.raises(ValueError, match="SWA window size"):
        other.lookup_prefix(list(range(128)))
    with pytest.raises(ValueError, match="8-bit"):
        store.load_pages(md, {"l": TurboQuantPagedCache(8, 8, "cpu")})
