"""Writes tests/golden/engine_decode_round.npz from the reference's own
serving engine (aether_2b/serving.py): a tiny-config Aether2BForCausalLM
decoding three sequences token by token through Aether2BServingEngine with a
4-bit TurboQuant compressed cache.  For every step and every attention layer
it records what the fused decode round needs and what the reference produced:

  CSA (serving.py:597-654): position, q (after q_norm), index query, raw
      index weights, the step's window entry, the compression inputs
      kv_a/z_a/kv_b/z_b and index_kv_a/index_z_a/index_kv_b/index_z_b, the
      reference's selected blocks (its torch.topk), and the attention output
      with the inverse RoPE applied (_post_attention before the output
      projection), and every visible block's index score (nan padded)
  HCA (serving.py:507-538): position, q, window entry, kv_proj(x),
      z_proj(x) (the slot bias is added by the consumer), output as above
  per layer: sink, kv_norm weight, emit biases

The index head weights go through softplus, as in the model's canonical
indexer (aether_2b/modeling.py:609-611); serving.py's decode path omits it,
which is the one documented difference.  Biases, sinks and norm weights are
drawn at random (the model initialises them to constants).

The engine memoises dequantized cache reads keyed by the cache tensor's
data_ptr and shape (serving.py:346-376).  When a freed cache tensor's
address is reused by another sequence's tensor of the same shape, the memo
returns the earlier sequence's values: recording three sequences with the
memo live gave attention outputs built from another sequence's cache.  The
fixture therefore empties the memo before every read.

Run where the reference checkout is available (path as the first argument
or AETHER_REFERENCE); the fixture is committed, so the tests never need the
reference."""
import os
import sys
from pathlib import Path

import numpy as np
import torch

_ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AETHER_REFERENCE")
if not _ref:
    sys.exit("usage: make_engine_golden.py <reference checkout>  (or set AETHER_REFERENCE)")
sys.path.insert(0, str(Path(_ref)))

import torch.nn.functional as F  # noqa: E402

from aether_2b.configuration import Aether2BConfig  # noqa: E402
from aether_2b.modeling import Aether2BForCausalLM, apply_rope  # noqa: E402
from aether_2b.serving import Aether2BServingEngine  # noqa: E402
from aether_pipeline.serving import PytorchAttentionBackend  # noqa: E402

torch.manual_seed(1234)
cfg = Aether2BConfig(vocab_size=128, hidden_size=128, num_hidden_layers=3, num_attention_heads=4,
                     attention_head_dim=128, query_compression_dim=64, indexer_num_heads=4, indexer_head_dim=64,
                     csa_compression=4, hca_compression=8, csa_top_k=8, sliding_window=16, rope_dim=64,
                     output_groups=2, group_output_dim=64, num_routed_experts=4, num_shared_experts=1,
                     num_experts_per_tok=2, moe_intermediate_size=32, hash_routed_layers=1, mhc_expansion=2,
                     mtp_depth=1)
model = Aether2BForCausalLM(cfg).eval()
engine = Aether2BServingEngine(model, backend=PytorchAttentionBackend(), device="cpu", turbo_quant_bits=4)
kinds = [cfg.attention_type(i) for i in range(cfg.num_hidden_layers)]


class Softplus(torch.nn.Module):
    def __init__(self, inner):
        super().__init__()
        self.inner = inner

    def forward(self, x):
        return F.softplus(self.inner(x))


params = {}
with torch.no_grad():
    for li, block in enumerate(model.model.layers):
        attn = block.attn.sublayer
        attn.sink.normal_(0.0, 1.0)
        attn.kv_norm.weight.uniform_(0.5, 1.5)
        params[f"L{li}_sink"] = attn.sink.clone()
        params[f"L{li}_norm_w"] = attn.kv_norm.weight.clone()
        params[f"L{li}_norm_eps"] = torch.tensor(attn.kv_norm.eps)
        if kinds[li] == "csa":
            for nm in ("bias_a", "bias_b", "index_bias_a", "index_bias_b"):
                getattr(attn, nm).normal_(0.0, 0.5)
                params[f"L{li}_{nm}"] = getattr(attn, nm).clone()
            attn.index_weight = Softplus(attn.index_weight)
        else:
            attn.bias.normal_(0.0, 0.5)
            params[f"L{li}_bias"] = attn.bias.clone()

rec = {}
current = {}
orig_post = engine._post_attention


def post(attn, out, position):
    neg = torch.full((out.size(0), out.size(1)), -position, dtype=torch.long)
    current["out"] = apply_rope(out, neg, cfg.rope_dim, cfg.rope_theta, config=cfg)[0].clone()
    return orig_post(attn, out, position)


engine._post_attention = post
orig_csa, orig_hca = engine._attention_step_csa, engine._attention_step_hca


def cap_csa(attn, model_state, state, li, x):
    pos = state.token_count
    q, latent = engine._query(attn, x, pos)
    r = {"pos": pos, "q": q[0, 0], "window_entry": engine._window_entry(attn, x, pos)[0, 0],
         "index_q": attn.index_q_up(latent).view(cfg.indexer_num_heads, cfg.indexer_head_dim),
         "index_w": attn.index_weight.inner(x)[0]}
    for nm in ("kv_a", "z_a", "kv_b", "z_b", "index_kv_a", "index_z_a", "index_kv_b", "index_z_b"):
        r[nm] = getattr(attn, nm)(x)[0]
    visible = engine._visible_csa_blocks(model_state, state, li)
    sel = torch.full((cfg.csa_top_k,), -1, dtype=torch.long)
    scores = torch.full((STEPS // cfg.csa_compression,), float("nan"))
    if visible:
        keys = engine._read_compressed(state.index_compressed, state.index_compressed_scale)[0, :visible]
        score = (F.relu(r["index_q"] @ keys.T) * F.softplus(r["index_w"]).unsqueeze(-1)).sum(0)
        k = min(cfg.csa_top_k, visible)
        sel[:k] = torch.sort(torch.topk(score, k).indices).values
        scores[:visible] = score
    r["sel"] = sel
    r["score"] = scores
    y = orig_csa(attn, model_state, state, li, x)
    r["out"] = current["out"]
    rec.setdefault(li, []).append(r)
    return y


def cap_hca(attn, model_state, state, li, x):
    pos = state.token_count
    q, _ = engine._query(attn, x, pos)
    r = {"pos": pos, "q": q[0, 0], "window_entry": engine._window_entry(attn, x, pos)[0, 0],
         "kv": attn.kv_proj(x)[0], "z": attn.z_proj(x)[0]}
    y = orig_hca(attn, model_state, state, li, x)
    r["out"] = current["out"]
    rec.setdefault(li, []).append(r)
    return y


engine._attention_step_csa, engine._attention_step_hca = cap_csa, cap_hca
orig_read = engine._read_compressed


def read_uncached(data, scale):
    # The engine memoises dequantized reads by (data_ptr, shape); a freed
    # cache tensor whose address is reused by another sequence's (or
    # layer's) tensor of the same shape then returns stale values.  The
    # fixture records the engine with that memo emptied before every read.
    engine._dequant_cache.clear()
    return orig_read(data, scale)


engine._read_compressed = read_uncached
SEQS, STEPS = 3, 60
g = torch.Generator().manual_seed(7)
with torch.no_grad():
    for s in range(SEQS):
        state = None
        for t in torch.randint(2, cfg.vocab_size, (STEPS,), generator=g).tolist():
            _, state = engine.step_token(t, state)

out = {"kinds": np.array(kinds), "seqs": np.array(SEQS), "steps": np.array(STEPS),
       "config": np.array([cfg.csa_compression, cfg.hca_compression, cfg.csa_top_k, cfg.sliding_window,
                           cfg.rope_dim, cfg.num_attention_heads]),
       "rope_theta": np.array(cfg.rope_theta), "bits": np.array(4)}
for k, v in params.items():
    out[k] = v.float().numpy()
for li, rows in rec.items():
    assert len(rows) == SEQS * STEPS
    for key in rows[0]:
        vals = [r[key] for r in rows]
        arr = np.array(vals) if key == "pos" else torch.stack(vals).float().numpy() if key != "sel" else torch.stack(vals).numpy()
        out[f"L{li}_{key}"] = arr.reshape(SEQS, STEPS, *arr.shape[1:])
path = Path(__file__).resolve().parent / "engine_decode_round.npz"
np.savez_compressed(path, **out)
print("wrote", path, path.stat().st_size, "bytes;", {k: v.shape for k, v in out.items() if k.startswith("L2")})
