"""The CPU oracle and the host-side helpers against golden vectors written
by the reference implementation itself (tests/golden/make_golden.py)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import decode as odec
from oracle import turboquant as otq

G = np.load(Path(__file__).resolve().parent / "golden" / "reference_vectors.npz")


def T(name):
    return torch.from_numpy(G[name])


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("d", [128, 64])
@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_oracle_encode_decode_bit_exact(bits, d, dt):
    key = f"tq{bits}_d{d}_{dt}"
    x = T(key + "_x")
    if dt == "bf16":
        x = x.to(torch.bfloat16)
    codes, scale = otq.encode(x, bits)
    assert torch.equal(codes, T(key + "_codes"))
    assert torch.equal(scale, T(key + "_scale"))
    assert torch.equal(otq.decode(codes, scale, bits), T(key + "_dec_f32"))
    assert torch.equal(otq.decode(codes, scale, bits, out_dtype=torch.bfloat16).view(torch.int16),
                       T(key + "_dec_bf16"))


def test_oracle_diag_and_wht():
    assert torch.equal(otq.rademacher(128, 42), T("diag_d128_seed42"))
    assert torch.equal(otq.rademacher(64, 42), T("diag_d64_seed42"))
    assert torch.equal(otq.rademacher(128, 7), T("diag_d128_seed7"))
    assert torch.equal(otq.wht(T("wht_x")), T("wht_y"))


def test_oracle_wht_errors():
    with pytest.raises(ValueError, match="power of 2"):
        otq.wht(torch.randn(3, 12))
    with pytest.raises(ValueError, match="bits must be 4 or 8"):
        otq.encode(torch.randn(2, 64), 3)


def test_package_diag_matches_reference():
    from aether_kernels.ops import rademacher_diag

    assert torch.equal(rademacher_diag(128, 42, torch.device("cpu")), T("diag_d128_seed42"))
    assert torch.equal(rademacher_diag(64, 42, torch.device("cpu")), T("diag_d64_seed42"))


def test_oracle_sparse_attention():
    args = (T("sa_q"), T("sa_kv"), T("sa_idx"), T("sa_sink"), 0.125)
    torch.testing.assert_close(oatt.sparse_attention(*args), T("sa_out"), atol=1e-6, rtol=1e-5)
    args = (T("sa_q"), T("sa_kv"), T("sa_idx"), T("sa_sink")[:1].reshape(()), 0.125)
    torch.testing.assert_close(oatt.sparse_attention(*args), T("sa_out_scalar_sink"), atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("name,factor", [("plain", 1.0), ("yarn4", 4.0), ("yarn8", 8.0)])
def test_rope_helpers_match_reference(name, factor):
    from aether_kernels.rope import RopeConfig, apply_rope, get_rope_freqs, rope_attention_scale

    cfg = RopeConfig() if factor == 1.0 else RopeConfig.yarn(factor)
    torch.testing.assert_close(get_rope_freqs(cfg), T(f"rope_freqs_{name}"), atol=0, rtol=0)
    assert rope_attention_scale(cfg) == pytest.approx(float(G[f"rope_scale_{name}"]), abs=0)
    pos = torch.arange(6) * 4 + 3
    torch.testing.assert_close(apply_rope(T(f"rope_x_{name}"), pos, cfg), T(f"rope_y_{name}"), atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("bits", [8, 4])
def test_oracle_csa_step_matches_reference(bits):
    p = f"csa{bits}_"
    nb = G[p + "kc"].shape[0]
    npg = (nb + 63) // 64
    pad = npg * 64 - nb

    def pool(x):
        x = torch.cat([T(p + x)] if not pad else [T(p + x), torch.zeros(pad, *G[p + x].shape[1:],
                                                                        dtype=T(p + x).dtype)])
        return x.view(npg, 64, *x.shape[1:])

    kc, ic = pool("kc"), pool("ic")
    ks, isc = pool("ks").squeeze(-1), pool("iscale").squeeze(-1)
    if bits == 8:
        kc, ic = kc.view(torch.uint8), ic.view(torch.uint8)
    table = torch.arange(npg, dtype=torch.int32).view(1, -1)
    res = odec.decode_step("csa", T(p + "q")[0], T(p + "iq")[None], T(p + "iw")[None], T(p + "sink"),
                           T(p + "win")[None].to(torch.bfloat16).float(), torch.tensor([128]), ic, isc, kc, ks,
                           table, torch.tensor([nb]), bits, 256, 128 ** -0.5)
    assert torch.equal(res.selected[0], T(p + "sel"))
    # the golden window was fp32: compare with the oracle run on the same fp32 window
    res32 = odec.decode_step("csa", T(p + "q")[0], T(p + "iq")[None], T(p + "iw")[None], T(p + "sink"),
                             T(p + "win")[None], torch.tensor([128]), ic, isc, kc, ks, table, torch.tensor([nb]),
                             bits, 256, 128 ** -0.5)
    torch.testing.assert_close(res32.out[0], T(p + "out")[0, 0], atol=1e-5, rtol=1e-5)


def _emit_inputs(bits, kind):
    p = f"emit{bits}_"
    if kind == "hca":
        return dict(c0=T(p + "hca_c"), z0=T(p + "hca_z"), positions=T(p + "hca_pos"), inv_freq=T(p + "inv_freq"),
                    norm_weight=T(p + "norm_w")), (T(p + "hca_codes"), T(p + "hca_scale"))
    q = p + "csa_"
    main = dict(c0=T(q + "a_c"), z0=T(q + "a_z"), bias0=T(q + "bias_a"), c1=T(q + "b_c"), z1=T(q + "b_z"),
                bias1=T(q + "bias_b"), has1=T(q + "has_prev"), positions=T(q + "pos"), inv_freq=T(p + "inv_freq"),
                norm_weight=T(p + "norm_w"))
    index = dict(c0=T(q + "ia_c"), z0=T(q + "ia_z"), bias0=T(q + "index_bias_a"), c1=T(q + "ib_c"),
                 z1=T(q + "ib_z"), bias1=T(q + "index_bias_b"), has1=T(q + "has_prev"))
    return (main, (T(q + "codes"), T(q + "scale"))), (index, (T(q + "icodes"), T(q + "iscale")))


@pytest.mark.parametrize("bits", [8, 4])
def test_oracle_emit_matches_reference_emit(bits):
    """oracle.compress.emit reproduces Aether2BServingEngine._hca_emit and
    _emit_csa_block (serving.py:495-505, 540-575) code for code."""
    from oracle import compress as ocmp

    cases = [_emit_inputs(bits, "hca")] + list(_emit_inputs(bits, "csa"))
    for kw, (codes, scale) in cases:
        _, c, s = ocmp.emit(**kw, bits=bits)
        assert torch.equal(c, codes)
        assert torch.equal(s, scale)
