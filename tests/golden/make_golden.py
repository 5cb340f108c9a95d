"""Writes tests/golden/reference_vectors.npz from the reference implementation.

Run in a container that has the reference checkout (the path is the first
argument, default /root/reference); the fixtures it writes are committed so
that the tests never need the reference at run time.  Every array below is
produced by the reference's own code:

  aether_2b/turbo_quant.py         PolarQuant.encode / decode, _wht, _diag
  aether_pipeline/serving.py       PytorchAttentionBackend.sparse_attention
  aether_2b/modeling.py            get_rope_freqs, rope_attention_scale, apply_rope
  aether_2b/modeling.py:609-615    indexer formula, evaluated with the
                                   reference's decoded keys (torch ops only)
"""
import sys
from pathlib import Path

import numpy as np
import torch

REF = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
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

dst = Path(__file__).resolve().parent / "reference_vectors.npz"
np.savez_compressed(dst, **out)
print(dst, sum(v.nbytes for v in out.values()), "bytes raw")
