"""Writes tests/golden/prefix_store_plans.json from the reference's own
prefix-store policy (aether_pipeline/serving.py:17-68 HybridCacheLayout /
SWACacheMode / RestorePlan, :174-338 OnDiskPrefixKVStore): for a grid of
layouts, SWA modes, checkpoint strides and prefix lengths it records
full_block_prefix, make_restore_plan and the prefix hash that save_prefix /
lookup_prefix key on.  Run where the reference checkout is available (path
as the first argument or AETHER_REFERENCE); the JSON it writes is committed,
so the tests never need the reference."""
import json
import os
import sys
import tempfile
from dataclasses import asdict
from pathlib import Path

_ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AETHER_REFERENCE")
if not _ref:
    sys.exit("usage: make_prefix_golden.py <reference checkout>  (or set AETHER_REFERENCE)")
sys.path.insert(0, str(Path(_ref)))

from aether_pipeline.serving import HybridCacheLayout, OnDiskPrefixKVStore, SWACacheMode  # noqa: E402

cases = []
with tempfile.TemporaryDirectory() as tmp:
    for layout in [(4, 128, 128, 24), (4, 16, 8, 2), (3, 5, 7, 3)]:
        lay = HybridCacheLayout(*layout)
        for mode in SWACacheMode:
            for stride in (8, 1000, 4096):
                store = OnDiskPrefixKVStore(os.path.join(tmp, f"{len(cases)}"), lay, swa_mode=mode,
                                            checkpoint_stride=stride)
                for n in (0, 1, 7, 16, 17, 128, 129, 999, 4096, 5000, 70001):
                    tokens = [(37 * i + 11) % 50000 for i in range(n)]
                    reusable = lay.full_block_prefix(n)
                    h = store._hash_tokens(tokens[:reusable]) if reusable > 0 else None
                    cases.append({"layout": list(layout), "mode": mode.value, "stride": stride, "tokens": n,
                                  "block_tokens": lay.block_tokens, "reusable": reusable, "hash": h,
                                  "plan": asdict(store.make_restore_plan(n))})
out = Path(__file__).resolve().parent / "prefix_store_plans.json"
out.write_text(json.dumps(cases, indent=0, sort_keys=True))
print(f"wrote {len(cases)} cases to {out}")
