"""GPU parity of the fused compress-on-emit kernel (pool -> RoPE -> RMSNorm
-> TurboQuant encode -> page write) against the oracle and against the
reference's own emit methods (golden vectors from serving.py:495-505,
540-575)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import compress as ocmp
from oracle import turboquant as otq

pytestmark = pytest.mark.gpu

G = np.load(Path(__file__).resolve().parent / "golden" / "reference_vectors.npz")

# fp32 pooling / RoPE / RMSNorm in another summation order than torch's CPU
# kernels: entries agree to a few ulp; a code may then move by one level
# where the rotated value sits on a rounding boundary.
ENTRY_RTOL = 2e-5
MAX_CODE_FLIPS = 0.01


def T(name, dev=None):
    t = torch.from_numpy(G[name])
    return t if dev is None else t.to(dev)


@pytest.fixture(scope="module")
def ops(cuda_device):
    from aether_kernels import _lib, ops

    _lib.load()
    return ops


def _pool(B, d, bits, dev, gen):
    rb = d * bits // 8
    npages = B + 3
    pool = torch.zeros(npages, 64 * rb + 256, dtype=torch.uint8, device=dev)
    perm = torch.randperm(npages, generator=gen)[:B]
    slot = torch.randint(0, 64 * 3, (B,), generator=gen, dtype=torch.int32)
    table = torch.zeros(B, 3, dtype=torch.int32)
    table[torch.arange(B), (slot // 64).long()] = perm.to(torch.int32)
    return pool, table.to(dev), slot.to(dev), rb


def _read(pool, table, slot, rb):
    t, s = table.cpu(), slot.cpu()
    codes, scales = [], []
    p = pool.cpu()
    for b in range(t.shape[0]):
        pg = int(t[b, int(s[b]) // 64])
        sl = int(s[b]) % 64
        codes.append(p[pg, sl * rb: (sl + 1) * rb])
        scales.append(p[pg, 64 * rb + 4 * sl: 64 * rb + 4 * sl + 4].view(torch.float32))
    return torch.stack(codes), torch.stack(scales)


def _check_codes(codes, scale, ref_codes, ref_scale, bits):
    a = otq.unpack_codes(codes, bits)
    r = otq.unpack_codes(ref_codes.view(torch.uint8) if bits == 8 else ref_codes, bits)
    diff = (a - r).abs()
    assert diff.max().item() <= 1
    assert (diff > 0).float().mean().item() <= MAX_CODE_FLIPS
    torch.testing.assert_close(scale.view(-1), ref_scale.view(-1).float(), rtol=ENTRY_RTOL, atol=0)


def _emit_cases(bits, dev):
    p = f"emit{bits}_"
    q = p + "csa_"
    hca = dict(c0=T(p + "hca_c", dev), z0=T(p + "hca_z", dev), positions=T(p + "hca_pos", dev),
               inv_freq=T(p + "inv_freq", dev), norm_weight=T(p + "norm_w", dev))
    has = T(q + "has_prev", dev).to(torch.int32)
    main = dict(c0=T(q + "a_c", dev), z0=T(q + "a_z", dev), bias0=T(q + "bias_a", dev), c1=T(q + "b_c", dev),
                z1=T(q + "b_z", dev), bias1=T(q + "bias_b", dev), has_seg1=has,
                positions=T(q + "pos", dev).to(torch.int32), inv_freq=T(p + "inv_freq", dev),
                norm_weight=T(p + "norm_w", dev))
    index = dict(c0=T(q + "ia_c", dev), z0=T(q + "ia_z", dev), bias0=T(q + "index_bias_a", dev),
                 c1=T(q + "ib_c", dev), z1=T(q + "ib_z", dev), bias1=T(q + "index_bias_b", dev), has_seg1=has)
    return [(hca, T(p + "hca_codes"), T(p + "hca_scale")), (main, T(q + "codes"), T(q + "scale")),
            (index, T(q + "icodes"), T(q + "iscale"))]


@pytest.mark.parametrize("bits", [8, 4])
def test_emit_matches_reference_emit_vectors(ops, cuda_device, bits):
    gen = torch.Generator().manual_seed(3)
    for kw, ref_codes, ref_scale in _emit_cases(bits, cuda_device):
        B, _, d = kw["c0"].shape
        pool, table, slot, rb = _pool(B, d, bits, cuda_device, gen)
        out = ops.compress_emit(**kw, bits=bits, page_table=table, slot_pos=slot, page_pool=pool)
        torch.cuda.synchronize()
        codes, scale = _read(pool, table, slot, rb)
        _check_codes(codes, scale, ref_codes, ref_scale, bits)
        # the fused entry against the oracle's fp32 entry
        okw = {k if k != "has_seg1" else "has1": (v.cpu() if torch.is_tensor(v) else v) for k, v in kw.items()}
        x, _, _ = ocmp.emit(**okw)
        torch.testing.assert_close(out.cpu(), x, rtol=ENTRY_RTOL, atol=ENTRY_RTOL)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("kind", ["hca", "csa_main", "csa_index"])
def test_emit_random_batch(ops, cuda_device, bits, dtype, kind):
    """64 sequences emitting at once, pages in random order; the fused write
    equals the stand-alone encoder applied to the fused entry, bit for bit."""
    from aether_kernels.rope import RopeConfig, get_rope_freqs

    gen = torch.Generator().manual_seed(bits * 10 + (dtype == torch.bfloat16))
    B = 64
    d = 64 if kind == "csa_index" else 128
    m0, m1 = (128, 0) if kind == "hca" else (4, 4)
    rnd = lambda *s: torch.randn(*s, generator=gen)
    kw = dict(c0=rnd(B, m0, d).to(dtype), z0=(rnd(B, m0, d) * 2).to(dtype))
    if m1:
        kw.update(bias0=rnd(m0, d) * 0.5, c1=rnd(B, m1, d).to(dtype), z1=(rnd(B, m1, d) * 2).to(dtype),
                  bias1=rnd(m1, d) * 0.5, has_seg1=(torch.rand(B, generator=gen) > 0.2).to(torch.int32))
    if kind != "csa_index":
        kw.update(positions=torch.randint(0, 1 << 20, (B,), generator=gen, dtype=torch.int32),
                  inv_freq=get_rope_freqs(RopeConfig.yarn(4.0))[:32].float(),
                  norm_weight=1.0 + 0.2 * rnd(d))
    dkw = {k: v.to(cuda_device) for k, v in kw.items()}
    pool, table, slot, rb = _pool(B, d, bits, cuda_device, gen)
    out = ops.compress_emit(**dkw, bits=bits, page_table=table, slot_pos=slot, page_pool=pool)
    torch.cuda.synchronize()
    codes, scale = _read(pool, table, slot, rb)
    c2, s2 = ops.tq_encode(out, bits)
    assert torch.equal(codes, c2.cpu().view(torch.uint8))
    assert torch.equal(scale.view(-1), s2.cpu().view(-1))
    okw = {k if k != "has_seg1" else "has1": v for k, v in kw.items()}
    x, oc, osc = ocmp.emit(**okw, bits=bits)
    # large positions: the angle's own fp32 rounding dominates (same in both)
    torch.testing.assert_close(out.cpu(), x, rtol=1e-4, atol=1e-4)
    _check_codes(codes, scale, oc, osc, bits)


def test_emit_errors(ops, cuda_device):
    from aether_kernels._lib import AetherKernelError

    c = torch.zeros(2, 4, 96, device=cuda_device)
    with pytest.raises((AetherKernelError, RuntimeError), match="dim must be 64 or 128"):
        ops.compress_emit(c, c)
    c = torch.zeros(2, 4, 128, device=cuda_device)
    with pytest.raises((AetherKernelError, RuntimeError), match="RoPE needs positions"):
        ops.compress_emit(c, c, inv_freq=torch.ones(32, device=cuda_device))


@pytest.mark.parametrize("bits", [8, 4])
def test_emitted_cache_feeds_decode(ops, cuda_device, bits):
    """Build a CSA cache only through the fused emit path (every block of 4
    sequences in one launch per stream), check every stored entry against
    the oracle's emit, then run the paged decode over it."""
    from aether_kernels.paged import TurboQuantPagedCache
    from aether_kernels.rope import RopeConfig, get_rope_freqs
    from aether_kernels.synthetic import make_decode_batch
    from test_gpu_kernels import _check_decode, _run_decode

    batch = make_decode_batch("csa", 4, 1200, 3000, bits, 4, seed=5, device="cuda")
    cache: TurboQuantPagedCache = batch.cache
    cache.kv_pages.zero_()
    cache.idx_pages.zero_()
    gen = torch.Generator().manual_seed(17)
    nbs = batch.nblocks.cpu().tolist()
    rows = [(b, i) for b, n in enumerate(nbs) for i in range(n)]
    R = len(rows)
    rnd = lambda *s: torch.randn(*s, generator=gen)
    main = [rnd(R, 4, 128), rnd(R, 4, 128) * 2, rnd(4, 128) * 0.5, rnd(R, 4, 128), rnd(R, 4, 128) * 2,
            rnd(4, 128) * 0.5]
    index = [rnd(R, 4, 64), rnd(R, 4, 64) * 2, rnd(4, 64) * 0.5, rnd(R, 4, 64), rnd(R, 4, 64) * 2, rnd(4, 64) * 0.5]
    has_prev = torch.tensor([int(i > 0) for _, i in rows], dtype=torch.int32)
    pos = torch.tensor([4 * i + 3 for _, i in rows], dtype=torch.int32)
    slot = torch.tensor([i for _, i in rows], dtype=torch.int32)
    table = batch.page_table.cpu()[torch.tensor([b for b, _ in rows])].contiguous()
    inv_freq = get_rope_freqs(RopeConfig())[:32].float()
    norm_w = 1.0 + 0.1 * rnd(128)
    dev = lambda ts: [t.to(cuda_device) for t in ts]
    cache.emit_csa(table.to(cuda_device), slot.to(cuda_device), dev(main), dev(index), has_prev.to(cuda_device),
                   pos.to(cuda_device), inv_freq.to(cuda_device), norm_w.to(cuda_device))
    torch.cuda.synchronize()

    _, oc, osc = ocmp.emit(*main, has1=has_prev, positions=pos, inv_freq=inv_freq, norm_weight=norm_w, bits=bits)
    _, ic, isc = ocmp.emit(*index, has1=has_prev, bits=bits)
    kc, ks = _read(cache.kv_pages, table, slot, 128 * bits // 8)
    _check_codes(kc, ks, oc, osc, bits)
    ikc, iks = _read(cache.idx_pages, table, slot, 64 * bits // 8)
    _check_codes(ikc, iks, ic, isc, bits)

    out, sel = _run_decode(None, batch)
    _check_decode(batch, out, sel)
