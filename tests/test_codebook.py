"""Lloyd-Max level format (the alternative TurboQuant codebook): the
codebook against Max's published N(0, 1) table and the oracle's own
restatement of Lloyd's algorithm, and the oracle's encode/decode properties."""
import torch

from oracle import turboquant as otq

# J. Max (1960), optimum 16-level quantizer for N(0, 1): positive output levels
MAX_16 = [0.1284, 0.3881, 0.6568, 0.9424, 1.2562, 1.6181, 2.0690, 2.7326]


def test_codebook_matches_published_16_levels():
    from aether_kernels.codebook import codebook

    lv, th = codebook(4)
    assert lv.shape == (16,) and th.shape == (15,)
    torch.testing.assert_close(lv[8:].double(), torch.tensor(MAX_16, dtype=torch.float64), atol=2e-4, rtol=0)
    assert torch.equal(lv, -lv.flip(0))
    assert bool((lv[1:] > lv[:-1]).all()) and bool((th > lv[:-1]).all()) and bool((th < lv[1:]).all())


def test_codebook_matches_oracle_restatement():
    from aether_kernels.codebook import lloyd_max_levels

    for levels in (16, 256):
        pkg = torch.tensor(lloyd_max_levels(levels), dtype=torch.float64)
        torch.testing.assert_close(pkg, otq.lloyd_max_levels(levels), atol=1e-6, rtol=0)


def test_oracle_lut_round_trip_and_ties():
    from aether_kernels.codebook import codebook

    g = torch.Generator().manual_seed(0)
    x = torch.randn(200, 128, generator=g)
    lv4, _ = codebook(4)
    c, s = otq.encode_lut(x, 4, lv4)
    xr = otq.decode_lut(c, s, 4, lv4)
    cu, su = otq.encode(x, 4)
    # for Gaussian-like rotated vectors the 16 Lloyd-Max levels beat 15 uniform ones
    assert ((xr - x) ** 2).mean() < ((otq.decode(cu, su, 4) - x) ** 2).mean()
    # a value exactly on a midpoint takes the lower level
    lv8, _ = codebook(8)
    thr = (lv8[:-1] + lv8[1:]) * 0.5
    u = thr[100:101].view(1, 1)
    assert int(torch.searchsorted(thr, u, right=False)) == 100
