"""Writes tests/golden/reference_vectors.npz from the reference implementation.

Run where the reference checkout is available: its path is the first
argument, or the AETHER_REFERENCE environment variable.  The fixtures it
writes are committed, so the tests never need the reference at run time.  Every array below is
produced by the reference's own code:

  aether_2b/turbo_quant.py         PolarQuant.encode / decode, _wht, _diag
  aether_pipeline/serving.py       PytorchAttentionBackend.sparse_attention
  aether_2b/modeling.py            get_rope_freqs, rope_attention_scale, apply_rope
  aether_2b/modeling.py:609-615    indexer formula, evaluated with the
                                   reference's decoded keys (torch ops only)
  aether_2b/serving.py:495-505     Aether2BServingEngine._hca_emit and
                     :540-590      _emit_csa_block, called unbound on a
                                   stand-in engine (config + _quant_append)
"""
import sys
from pathlib import Path

import numpy as np
import torch

import os  # noqa: E402

_ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AETHER_REFERENCE")
if not _ref:
    sys.exit("usage: make_golden.py <reference checkout>  (or set AETHER_REFERENCE)")
REF = Path(_ref)
sys.path.insert(0, str(REF))

from aether_2b.configuration import Aether2BConfig  # noqa: E402
from aether_2b.modeling import apply_rope, get_rope_freqs, rope_attention_scale  # noqa: E402
from aether_2b.turbo_quant import PolarQuant, _wht  # noqa: E402
from aether_pipeline.serving import PytorchAttentionBackend  # noqa: E402

out = {}
g = torch.Generator().manual_seed(20260101)

# --- TurboQuant encode / decode (bf16 and fp32 inputs, special vectors)
for bits in (8, 4):
    pq = PolarQuant(bits)
    for d in (128, 64):
        x = torch.randn(3, 40, d, generator=g) * 2.5
        x[0, 0] = 0.0
        x[0, 1] = torch.linspace(-1, 1, d)
        x[0, 2, 0] = 1e4
        for dt in ("bf16", "f32"):
            xi = x.to(torch.bfloat16) if dt == "bf16" else x
            c, s = pq.encode(xi)
            key = f"tq{bits}_d{d}_{dt}"
            out[key + "_x"] = xi.float().numpy()
            out[key + "_codes"] = c.numpy()
            out[key + "_scale"] = s.numpy()
            out[key + "_dec_f32"] = pq.decode(c, s, out_dtype=torch.float32).numpy()
            out[key + "_dec_bf16"] = pq.decode(c, s).view(torch.int16).numpy()
        out[f"diag_d{d}_seed42"] = pq._diag(d, torch.device("cpu")).numpy()
out["diag_d128_seed7"] = PolarQuant(8, seed=7)._diag(128, torch.device("cpu")).numpy()
w = torch.randn(5, 128, generator=g)
out["wht_x"] = w.numpy()
out["wht_y"] = _wht(w).numpy()

# --- sparse sink attention (shapes of tests/test_cuda_runtime.py:19-47)
q = torch.randn(2, 5, 4, 16, generator=g)
kv = torch.randn(2, 23, 2, 16, generator=g)
idx = torch.randint(0, 23, (2, 5, 7), generator=g)
sink = torch.randn(4, generator=g)
be = PytorchAttentionBackend()
out["sa_q"], out["sa_kv"], out["sa_idx"], out["sa_sink"] = q.numpy(), kv.numpy(), idx.numpy(), sink.numpy()
out["sa_out"] = be.sparse_attention(q, kv, idx, sink, 0.125).numpy()
out["sa_out_scalar_sink"] = be.sparse_attention(q, kv, idx, sink[:1].reshape(()), 0.125).numpy()

# --- RoPE / YaRN
for name, kw in (("plain", {}), ("yarn4", dict(rope_scaling_type="yarn", rope_scaling_factor=4.0)),
                 ("yarn8", dict(rope_scaling_type="yarn", rope_scaling_factor=8.0))):
    cfg = Aether2BConfig(**kw)
    out[f"rope_freqs_{name}"] = get_rope_freqs(1, cfg).numpy()
    out[f"rope_scale_{name}"] = np.array(rope_attention_scale(cfg))
    xr = torch.randn(6, 128, generator=g)
    pos = torch.arange(6) * 4 + 3
    out[f"rope_x_{name}"] = xr.numpy()
    out[f"rope_y_{name}"] = apply_rope(xr, pos, cfg.rope_dim, cfg.rope_theta, config=cfg).numpy()

# --- CSA decode step composed from reference pieces (small shapes)
for bits in (8, 4):
    pq = PolarQuant(bits)
    nb, H = 300, 12
    kraw = torch.randn(nb, 128, generator=g)
    iraw = torch.randn(nb, 64, generator=g)
    kc, ks = pq.encode(kraw)
    ic, iscale = pq.encode(iraw)
    keys = pq.decode(ic, iscale, out_dtype=torch.float32)
    main = pq.decode(kc, ks, out_dtype=torch.float32)
    iq = torch.randn(4, 64, generator=g)
    iw = torch.randn(4, generator=g)
    score = (torch.relu(torch.einsum("hc,sc->hs", iq, keys)) * torch.nn.functional.softplus(iw).unsqueeze(-1)).sum(0)
    sel = torch.sort(torch.topk(score, k=256).indices).values
    win = torch.randn(128, 128, generator=g)
    qq = torch.randn(1, 1, H, 128, generator=g)
    snk = torch.randn(H, generator=g)
    src = torch.cat([main[sel], win], 0)
    kvp = torch.stack([src, src], dim=1).unsqueeze(0)
    full = torch.arange(src.shape[0]).view(1, 1, -1)
    o = be.sparse_attention(qq, kvp, full, snk, 128 ** -0.5)
    p = f"csa{bits}_"
    for k_, v_ in dict(kc=kc, ks=ks, ic=ic, iscale=iscale, iq=iq, iw=iw, win=win, q=qq, sink=snk, score=score,
                       sel=sel, out=o).items():
        out[p + k_] = v_.numpy()

# --- compress-on-emit: the reference's own emit methods, unbound, fp32
from types import SimpleNamespace  # noqa: E402

from aether_2b.modeling import RMSNorm  # noqa: E402
from aether_2b.serving import Aether2BServingEngine as _Eng  # noqa: E402

torch.set_grad_enabled(False)

for bits in (8, 4):
    cfg = Aether2BConfig(rope_scaling_type="yarn", rope_scaling_factor=4.0)
    eng = SimpleNamespace(config=cfg, _polar_quant=PolarQuant(bits))
    eng._quant_append = _Eng._quant_append.__get__(eng)
    norm = RMSNorm(128, cfg.rms_norm_eps)
    with torch.no_grad():
        norm.weight.copy_(1.0 + 0.2 * torch.randn(128, generator=g))
    p = f"emit{bits}_"
    out[p + "norm_w"] = norm.weight.detach().numpy()
    # HCA: 128 rows, bias already inside buffer_z (serving.py:527-530)
    cs, zs, outs_c, outs_s = [], [], [], []
    for b in range(3):
        c = torch.randn(1, 128, 128, generator=g)
        z = torch.randn(1, 128, 128, generator=g) * 2.0
        st = SimpleNamespace(buffer_c=c.clone(), buffer_z=z.clone(), compressed=None, compressed_scale=None)
        _Eng._hca_emit(eng, SimpleNamespace(kv_norm=norm), st, 128 * (b + 5) - 1)
        cs.append(c[0]), zs.append(z[0]), outs_c.append(st.compressed[0, 0]), outs_s.append(st.compressed_scale[0, 0])
    out[p + "hca_c"], out[p + "hca_z"] = torch.stack(cs).numpy(), torch.stack(zs).numpy()
    out[p + "hca_pos"] = np.array([128 * (b + 5) - 1 for b in range(3)], dtype=np.int32)
    out[p + "hca_codes"], out[p + "hca_scale"] = torch.stack(outs_c).numpy(), torch.stack(outs_s).numpy()
    # CSA: 4 rows of this block's a half + the previous block's b half
    m = cfg.csa_compression
    attn = SimpleNamespace(kv_norm=norm, bias_a=torch.randn(m, 128, generator=g) * 0.5,
                           bias_b=torch.randn(m, 128, generator=g) * 0.5,
                           index_bias_a=torch.randn(m, 64, generator=g) * 0.5,
                           index_bias_b=torch.randn(m, 64, generator=g) * 0.5)
    for k_ in ("bias_a", "bias_b", "index_bias_a", "index_bias_b"):
        out[p + "csa_" + k_] = getattr(attn, k_).numpy()
    rec = {k_: [] for k_ in ("a_c", "a_z", "b_c", "b_z", "ia_c", "ia_z", "ib_c", "ib_z", "has_prev", "pos",
                             "codes", "scale", "icodes", "iscale")}
    for b in range(4):
        t = lambda d_: torch.randn(1, m, d_, generator=g)
        a_c, a_z, b_c, b_z = t(128), t(128) * 2, t(128), t(128) * 2
        ia_c, ia_z, ib_c, ib_z = t(64), t(64) * 2, t(64), t(64) * 2
        has_prev = b % 2 == 1
        tok = m * (b + 3) - 1
        st = SimpleNamespace(curr_a_c=a_c, curr_a_z=a_z, curr_b_c=None, curr_b_z=None,
                             curr_index_a_c=ia_c, curr_index_a_z=ia_z, curr_index_b_c=None, curr_index_b_z=None,
                             prev_b_c=b_c if has_prev else None, prev_b_z=b_z if has_prev else None,
                             prev_index_b_c=ib_c if has_prev else None, prev_index_b_z=ib_z if has_prev else None,
                             compressed=None, compressed_scale=None, index_compressed=None,
                             index_compressed_scale=None)
        _Eng._emit_csa_block(eng, attn, st, tok)
        for k_, v_ in (("a_c", a_c), ("a_z", a_z), ("b_c", b_c), ("b_z", b_z), ("ia_c", ia_c), ("ia_z", ia_z),
                       ("ib_c", ib_c), ("ib_z", ib_z)):
            rec[k_].append(v_[0])
        rec["has_prev"].append(torch.tensor(int(has_prev)))
        rec["pos"].append(torch.tensor(tok - (m - 1)))
        rec["codes"].append(st.compressed[0, 0]), rec["scale"].append(st.compressed_scale[0, 0])
        rec["icodes"].append(st.index_compressed[0, 0]), rec["iscale"].append(st.index_compressed_scale[0, 0])
    for k_, v_ in rec.items():
        out[p + "csa_" + k_] = torch.stack(v_).numpy()
    out[p + "inv_freq"] = get_rope_freqs(1, cfg)[: cfg.rope_dim // 2].numpy()

dst = Path(__file__).resolve().parent / "reference_vectors.npz"
np.savez_compressed(dst, **out)
print(dst, sum(v.nbytes for v in out.values()), "bytes raw")
