"""The Lloyd-Max level format through the fused paged decode kernels: a
cache whose codes index the N(0, 1) Lloyd-Max table decodes against the
oracle restatement (oracle.turboquant.decode_lut): exact top-256 outside the
near-tie band, attention within 2e-2 max-abs / 1e-3 mean-abs."""
import pytest
import torch

from oracle import decode as odec

pytestmark = pytest.mark.gpu


def _batch(kind, bits, B, lo, hi, compression, seed, rope=None):
    from aether_kernels.paged import TurboQuantPagedCache
    from aether_kernels.synthetic import make_decode_batch

    pages = B * ((hi // compression + 63) // 64) + 4
    cache = TurboQuantPagedCache(pages, bits, "cuda", with_index=(kind == "csa"), codebook="lloyd-max")
    kw = {} if rope is None else {"rope": rope}
    return make_decode_batch(kind, B, lo, hi, bits, compression, seed=seed, device="cuda", cache=cache, **kw)


def _oracle(b, bits, use_selection=None):
    from aether_kernels.codebook import codebook

    c = b.cache
    return odec.decode_step(b.kind, b.q.cpu(), None if b.index_q is None else b.index_q.cpu(),
                            None if b.index_weight is None else b.index_weight.cpu(), b.sink.cpu(), b.window.cpu(),
                            b.window_len.cpu(), None if c.idx_codes is None else c.idx_codes.cpu(),
                            None if c.idx_scale is None else c.idx_scale.cpu(), c.kv_codes.cpu(), c.kv_scale.cpu(),
                            b.page_table.cpu(), b.nblocks.cpu(), bits, b.top_k, b.softmax_scale,
                            use_selection=use_selection, levels=codebook(bits)[0])


@pytest.mark.parametrize("bits", [4, 8])
def test_csa_decode_lloyd_max(cuda_device, bits):
    from aether_kernels.paged import csa_decode_paged

    b = _batch("csa", bits, 6, 3000, 32768, 4, seed=900 + bits)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, sel = csa_decode_paged(b.q, b.index_q, b.index_weight, b.sink, b.window, b.window_len, b.cache,
                                b.page_table, b.nblocks, b.softmax_scale, top_k=b.top_k, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = _oracle(b, bits)
    kern_sel, ties = [], 0
    for i in range(6):
        k = min(b.top_k, int(b.nblocks[i]))
        got = sel[i].cpu()
        assert (got[k:] == -1).all()
        got = got[:k].long()
        kern_sel.append(got)
        if not torch.equal(got, ref.selected[i]):
            assert ref.near_tie[i], f"row {i}: top-k differs outside the near-tie band"
            ties += 1
    if ties:
        ref = _oracle(b, bits, use_selection=kern_sel)
    d = (out.float().cpu() - ref.out).abs()
    assert d.max() < 2e-2 and d.mean() < 1e-3, (float(d.max()), float(d.mean()))


@pytest.mark.parametrize("bits", [4, 8])
def test_hca_decode_lloyd_max(cuda_device, bits):
    from aether_kernels.paged import hca_decode_paged
    from aether_kernels.rope import RopeConfig

    b = _batch("hca", bits, 5, 20000, 131072, 128, seed=950 + bits, rope=RopeConfig.yarn(4.0))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = hca_decode_paged(b.q, b.sink, b.window, b.window_len, b.cache, b.page_table, b.nblocks, b.softmax_scale,
                           err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = _oracle(b, bits)
    d = (out.float().cpu() - ref.out).abs()
    assert d.max() < 2e-2 and d.mean() < 1e-3, (float(d.max()), float(d.mean()))


def test_lloyd_max_cache_matches_dense_encode(cuda_device):
    """The cache write of the level format stores exactly the codes and
    scales of the dense PolarQuant(codebook="lloyd-max") encode."""
    from aether_kernels.turbo_quant import PolarQuant

    b = _batch("csa", 4, 2, 5000, 9000, 4, seed=3)
    assert b.raw_kv is None
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(1, 100, 128, generator=g, device="cuda")
    pt = b.page_table[:1]
    start = torch.zeros(1, dtype=torch.int32, device="cuda")
    b.cache.write(pt, start, x)
    codes, scale = PolarQuant(4, codebook="lloyd-max").encode(x[0])
    pages = pt[0, :2].long()
    got_c = b.cache.kv_codes[pages].reshape(128, -1)[:100]
    got_s = b.cache.kv_scale[pages].reshape(128)[:100]
    assert torch.equal(got_c, codes) and torch.equal(got_s, scale.squeeze(-1))
