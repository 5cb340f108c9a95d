"""GPU parity of the sm_100a kernels against the CPU oracle (bit-exact codes,
exact top-k indices, attention within the bf16 tolerance)."""
import pytest
import torch

from oracle import attention as oatt
from oracle import decode as odec
from oracle import turboquant as otq

pytestmark = pytest.mark.gpu

# attention tolerance of the decode path: bf16 output vs the fp32 oracle
MAX_ABS = 2e-2
MEAN_ABS = 1e-3


@pytest.fixture(scope="module")
def ak(cuda_device):
    import aether_kernels
    from aether_kernels import _lib

    _lib.load()
    return aether_kernels


# ------------------------------------------------------------- TurboQuant
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("d", [128, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_tq_encode_bit_exact(ak, bits, d, dtype):
    from aether_kernels.turbo_quant import PolarQuant

    g = torch.Generator().manual_seed(bits * 1000 + d)
    x = (torch.randn(7, 333, d, generator=g) * 3).to(dtype)
    x[0, 0] = 0  # all-zero vector: absmax clamps to 1e-8
    x[0, 1] = torch.linspace(-1, 1, d).to(dtype)
    codes, scale = PolarQuant(bits).encode(x.cuda())
    rc, rs = otq.encode(x, bits)
    assert codes.dtype == rc.dtype and codes.shape == rc.shape
    assert torch.equal(codes.cpu(), rc)
    assert torch.equal(scale.cpu(), rs)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("d", [128, 64])
def test_tq_decode_matches(ak, bits, d):
    from aether_kernels.turbo_quant import PolarQuant, _wht

    g = torch.Generator().manual_seed(5 + bits + d)
    x = torch.randn(4, 100, d, generator=g)
    rc, rs = otq.encode(x, bits)
    pq = PolarQuant(bits)
    got = pq.decode(rc.cuda(), rs.cuda(), out_dtype=torch.float32).cpu()
    ref = otq.decode(rc, rs, bits)
    assert torch.equal(got, ref)
    got_bf = pq.decode(rc.cuda(), rs.cuda()).cpu()
    assert torch.equal(got_bf, ref.to(torch.bfloat16))
    assert torch.equal(_wht(x.cuda()).cpu(), otq.wht(x))


# ------------------------------------------------ reference extension ops
@pytest.mark.parametrize("dtype,index_dtype", [(torch.float32, torch.int64), (torch.float16, torch.int32),
                                               (torch.bfloat16, torch.int64)])
def test_sparse_sink_attention_reference_case(ak, dtype, index_dtype):
    """The reference's own kernel test (tests/test_cuda_runtime.py:19-47)."""
    ext = ak.load_aether_cuda_kernels()
    torch.manual_seed(0)
    q = torch.randn(2, 5, 4, 16, device="cuda", dtype=dtype)
    kv = torch.randn(2, 23, 2, 16, device="cuda", dtype=dtype)
    topk = torch.randint(0, 23, (2, 5, 7), device="cuda", dtype=index_dtype)
    sink = torch.randn(4, device="cuda", dtype=dtype)
    got = ext.sparse_sink_attention(q, kv, topk, sink, 0.125)
    exp = oatt.sparse_attention(q.cpu(), kv.cpu(), topk.cpu(), sink.cpu(), 0.125).to(dtype)
    tol = 5e-3 if dtype != torch.float32 else 1e-4
    torch.testing.assert_close(got.float().cpu(), exp.float(), atol=tol, rtol=tol)


def test_sparse_sink_attention_serving_shape(ak):
    """Serving decode call: T=1, K=S full indices, D=128, bf16, scalar sink."""
    torch.manual_seed(1)
    B, S, H, D = 3, 300, 12, 128
    q = torch.randn(B, 1, H, D, device="cuda", dtype=torch.bfloat16)
    vals = torch.randn(B, S, D, device="cuda", dtype=torch.bfloat16)
    kv = torch.stack([vals, vals], dim=2)
    idx = torch.arange(S, device="cuda").view(1, 1, S).expand(B, 1, S).contiguous()
    idx[0, 0, :5] = -1  # skipped
    sink = torch.randn(1, device="cuda", dtype=torch.bfloat16)
    got = ak.sparse_sink_attention(q, kv, idx, sink, D ** -0.5)
    exp = oatt.sparse_attention(q.cpu(), kv.cpu(), idx.cpu(), sink.cpu(), D ** -0.5)
    assert (got.float().cpu() - exp).abs().max() < MAX_ABS


def test_tiled_prefill_attention(ak):
    from aether_kernels.sparse_attention import tiled_prefill_attention

    torch.manual_seed(2)
    q = torch.randn(2, 9, 4, 64, device="cuda")
    kv = torch.randn(2, 40, 2, 64, device="cuda")
    sink = torch.randn(4, device="cuda")
    got = tiled_prefill_attention(q, kv, sink, 0.125, tile_size=16)
    idx = torch.arange(40).view(1, 1, 40).expand(2, 9, 40)
    exp = oatt.sparse_attention(q.cpu(), kv.cpu(), idx, sink.cpu(), 0.125)
    torch.testing.assert_close(got.cpu(), exp, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("S,k", [(23, 7), (1000, 256), (5000, 256), (300, 300)])
def test_csa_indexer_topk(ak, S, k):
    from aether_kernels.sparse_attention import csa_indexer_topk

    g = torch.Generator().manual_seed(S)
    iq = torch.randn(3, 4, 64, generator=g)
    ikv = torch.randn(3, S, 64, generator=g)
    iw = torch.randn(3, 4, generator=g)
    got = csa_indexer_topk(iq.cuda(), ikv.cuda(), iw.cuda(), k).cpu()
    exp, _ = oatt.dense_index_topk(iq, ikv, iw, k)
    s64, mag = oatt.dense_index_scores64(iq, ikv, iw)
    assert got.dtype == torch.int64 and got.shape == (3, k)
    for b in range(3):
        band = 1e-5 * float(mag[b])  # fp32 rounding of the score sums, scaled to the row
        srt = torch.sort(s64[b], descending=True).values
        # the selected set is exact unless ranks k and k+1 are a near tie
        if not torch.equal(torch.sort(got[b]).values, torch.sort(exp[b]).values):
            assert k < S and float(srt[k - 1] - srt[k]) <= band, f"row {b}: set differs outside the near-tie band"
        # the order is score descending up to the same band, lower index first on equal scores
        sg = s64[b][got[b]]
        assert bool((sg[:-1] >= sg[1:] - band).all()), f"row {b}: order"


def test_csa_indexer_topk_ties_lowest_index(ak):
    from aether_kernels.sparse_attention import csa_indexer_topk

    iq = torch.ones(1, 4, 64)
    ikv = torch.zeros(1, 50, 64)
    ikv[0, ::2] = 1.0  # 25 equal positive scores, 25 zeros
    iw = torch.zeros(1, 4)
    got = csa_indexer_topk(iq.cuda(), ikv.cuda(), iw.cuda(), 30).cpu()[0]
    assert got[:25].tolist() == list(range(0, 50, 2))
    assert got[25:].tolist() == [1, 3, 5, 7, 9]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_hca_compress(ak, dtype):
    from aether_kernels.sparse_attention import hca_compress

    torch.manual_seed(3)
    c = torch.randn(4, 128, 128, device="cuda", dtype=dtype)
    z = torch.randn(4, 128, 128, device="cuda", dtype=dtype)
    got = hca_compress(c, z).float().cpu()
    exp = oatt.hca_compress(c.cpu(), z.cpu())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    torch.testing.assert_close(got, exp, atol=tol, rtol=tol)


# ------------------------------------------------ fused paged decode path
def _run_decode(ak, batch, check_rows=None):
    from aether_kernels.paged import csa_decode_paged, hca_decode_paged

    c = batch.cache
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    if batch.kind == "csa":
        out, sel = csa_decode_paged(batch.q, batch.index_q, batch.index_weight, batch.sink, batch.window,
                                    batch.window_len, c, batch.page_table, batch.nblocks, batch.softmax_scale,
                                    top_k=batch.top_k, err=err)
    else:
        out = hca_decode_paged(batch.q, batch.sink, batch.window, batch.window_len, c, batch.page_table,
                               batch.nblocks, batch.softmax_scale, err=err)
        sel = None
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out, sel


def _oracle(batch, rows=None, use_selection=None):
    c = batch.cache
    rows = list(range(batch.q.shape[0])) if rows is None else rows
    r = torch.tensor(rows)
    return odec.decode_step(
        batch.kind, batch.q.cpu()[r], None if batch.index_q is None else batch.index_q.cpu()[r],
        None if batch.index_weight is None else batch.index_weight.cpu()[r], batch.sink.cpu(),
        batch.window.cpu()[r], batch.window_len.cpu()[r], None if c.idx_codes is None else c.idx_codes.cpu(),
        None if c.idx_scale is None else c.idx_scale.cpu(), c.kv_codes.cpu(), c.kv_scale.cpu(),
        batch.page_table.cpu()[r], batch.nblocks.cpu()[r], batch.bits, batch.top_k, batch.softmax_scale,
        use_selection=use_selection)


def _check_decode(batch, out, sel, rows=None):
    rows = list(range(batch.q.shape[0])) if rows is None else rows
    ref = _oracle(batch, rows)
    ties = 0
    kern_sel = []
    for i, b in enumerate(rows):
        if sel is not None:
            k = min(batch.top_k, int(batch.nblocks[b]))
            got = sel[b].cpu()
            assert (got[k:] == -1).all()
            got = got[:k].long()
            assert torch.equal(got, torch.sort(got).values), "indices must be ascending"
            kern_sel.append(got)
            if not torch.equal(got, ref.selected[i]):
                assert ref.near_tie[i], f"row {b}: top-k differs outside the near-tie band"
                ties += 1
    if ties:
        ref = _oracle(batch, rows, use_selection=kern_sel)
    diff = (out.float().cpu()[torch.tensor(rows)] - ref.out).abs()
    assert diff.max() < MAX_ABS, f"max abs {diff.max():.3e}"
    assert diff.mean() < MEAN_ABS, f"mean abs {diff.mean():.3e}"
    return ties


@pytest.mark.parametrize("bits", [8, 4])
def test_csa_decode_small_ragged(ak, bits):
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 6, 40, 6000, bits, 4, seed=11 + bits, device="cuda")
    out, sel = _run_decode(ak, batch)
    _check_decode(batch, out, sel)


def test_csa_decode_config0(ak):
    """batch 4, 8192 tokens -> 2048 blocks, 8-bit."""
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 4, 8192, 8192, 8, 4, seed=0, device="cuda")
    out, sel = _run_decode(ak, batch)
    _check_decode(batch, out, sel)


def test_csa_decode_config1(ak):
    """BASELINE config 1 (4-bit, 16K-32K tokens, batch 64): every row's
    selection and output against the oracle."""
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 64, 16384, 32768, 4, 4, seed=1, device="cuda")
    out, sel = _run_decode(ak, batch)
    _check_decode(batch, out, sel)


def test_csa_decode_workspace_reuse(ak):
    """Consecutive steps of different batches through one workspace (the
    persistent path leaves its key rows and queue state clean) equal the same
    steps each with a fresh workspace."""
    from aether_kernels.paged import csa_decode_paged, csa_workspace_bytes
    from aether_kernels.synthetic import make_decode_batch

    batches = [make_decode_batch("csa", 9, lo, hi, bits, 4, seed=200 + i, device="cuda")
               for i, (lo, hi, bits) in enumerate([(16000, 32000, 4), (100, 900, 4), (8000, 20000, 4),
                                                   (30000, 32768, 4)])]
    need = max(csa_workspace_bytes(9, 8192) for _ in batches)
    shared = torch.zeros(need, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for b in batches:
        pt = torch.zeros(9, 128, dtype=torch.int32, device="cuda")
        pt[:, : b.page_table.shape[1]] = b.page_table
        args = (b.q, b.index_q, b.index_weight, b.sink, b.window, b.window_len, b.cache, pt, b.nblocks,
                b.softmax_scale)
        o1, s1 = csa_decode_paged(*args, top_k=b.top_k, workspace=shared, err=err)
        o2, s2 = csa_decode_paged(*args, top_k=b.top_k)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(s1, s2) and torch.equal(o1, o2)


def test_csa_decode_short_and_empty(ak):
    """nb = 0, nb < top_k, nb == top_k, partial windows."""
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 5, 0, 1100, 4, 4, seed=3, device="cuda")
    toks = [0, 3, 50, 1024, 1100]
    # rebuild with explicit lengths
    batches = [make_decode_batch("csa", 1, t, t, 4, 4, seed=20 + i, device="cuda") for i, t in enumerate(toks)]
    for bt in batches:
        out, sel = _run_decode(ak, bt)
        _check_decode(bt, out, sel)
    del batch


def test_csa_decode_exact_ties(ak):
    """Identical index entries give bit-identical scores in the kernel and the
    oracle; the kernel must take the lowest block indices among them."""
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 2, 4000, 4000, 8, 4, seed=4, device="cuda")
    c = batch.cache
    # every block of row 0 gets the same index entry -> all scores equal
    for p in batch.page_table[0, : (1000 + 63) // 64].tolist():
        c.idx_codes[p] = c.idx_codes[batch.page_table[0, 0]][0]
        c.idx_scale[p] = c.idx_scale[batch.page_table[0, 0]][0]
    out, sel = _run_decode(ak, batch)
    assert sel[0, :256].cpu().tolist() == list(range(256))
    _check_decode(batch, out, sel)


def test_csa_decode_key_range_extremes(ak):
    """The selection rescales each sequence's keys onto the full bin range
    before its histogram.  Row 0: every score is zero (index query zero), so
    all keys are equal across ~8000 blocks and the lowest block ids win.
    Row 1: one block's index scale is raised 1000x, so (unless its score is
    zero) one key sits far above the band holding the other winners and
    dominates the rescale range.  Row 2 is left as generated."""
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 3, 32000, 32768, 4, 4, seed=77, device="cuda")
    batch.index_q[0].zero_()
    c = batch.cache
    p1 = int(batch.page_table[1, 3])
    c.idx_scale[p1, 5] *= 1000.0
    out, sel = _run_decode(ak, batch)
    assert sel[0, :256].cpu().tolist() == list(range(256))
    _check_decode(batch, out, sel)


@pytest.mark.parametrize("bits", [4, 8])
def test_hca_decode(ak, bits):
    """BASELINE config 2 shapes (HCA, 131072 tokens -> 1024 blocks, YaRN 4) at
    batch 6."""
    from aether_kernels.rope import RopeConfig
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("hca", 6, 60000, 131072, bits, 128, seed=5, device="cuda",
                              rope=RopeConfig.yarn(4.0))
    out, _ = _run_decode(ak, batch)
    _check_decode(batch, out, None)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("window", [128, 20])
def test_hca_decode_ragged(ak, bits, window):
    """Ragged contexts from empty to the 1024-block maximum, a block count
    that is not a page multiple, short and empty windows."""
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("hca", 9, 0, 131072, bits, 128, window=window, seed=21 + bits + window,
                              device="cuda")
    batch.nblocks[2] = 0
    batch.nblocks[3] = 1024 if batch.page_table.shape[1] * 64 >= 1024 else batch.nblocks[3]
    batch.nblocks[4] = min(int(batch.nblocks[4]), 1000)
    batch.window_len[5] = 0
    batch.window_len[6] = 1
    out, _ = _run_decode(ak, batch)
    _check_decode(batch, out, None)


def test_hca_decode_overlap_prefetch(ak):
    """Back-to-back HCA launches with programmatic dependent launch give the
    same bits as plain launches."""
    from aether_kernels.paged import hca_decode_paged
    from aether_kernels.synthetic import make_decode_batch

    bs = [make_decode_batch("hca", 8, 20000, 131072, 4, 128, seed=60 + i, device="cuda") for i in range(3)]
    plain = [_run_decode(ak, b)[0] for b in bs]
    outs = [hca_decode_paged(b.q, b.sink, b.window, b.window_len, b.cache, b.page_table, b.nblocks,
                             b.softmax_scale, overlap_prefetch=True) for b in bs for _ in range(2)]
    torch.cuda.synchronize()
    for i, o in enumerate(outs):
        assert torch.equal(o, plain[i // 2])


def test_csa_decode_overlap_prefetch(ak):
    """Back-to-back launches with programmatic dependent launch give the
    same results as plain launches."""
    from aether_kernels.paged import csa_decode_paged
    from aether_kernels.synthetic import make_decode_batch

    bs = [make_decode_batch("csa", 8, 9000, 30000, 4, 4, seed=40 + i, device="cuda") for i in range(3)]
    plain = [_run_decode(ak, b) for b in bs]
    outs = []
    for b in bs:
        outs.append(csa_decode_paged(b.q, b.index_q, b.index_weight, b.sink, b.window, b.window_len, b.cache,
                                     b.page_table, b.nblocks, b.softmax_scale, top_k=b.top_k, overlap_prefetch=True))
    torch.cuda.synchronize()
    for (o, s), (po, ps) in zip(outs, plain):
        assert torch.equal(s, ps)
        assert torch.equal(o, po)


def test_kernels_against_reference_golden_vectors(ak):
    """Kernel outputs against vectors written by the reference itself."""
    from pathlib import Path

    import numpy as np
    from aether_kernels.turbo_quant import PolarQuant

    G = np.load(Path(__file__).resolve().parent / "golden" / "reference_vectors.npz")
    for bits in (8, 4):
        for d in (128, 64):
            for dt in ("bf16", "f32"):
                key = f"tq{bits}_d{d}_{dt}"
                x = torch.from_numpy(G[key + "_x"])
                x = x.to(torch.bfloat16) if dt == "bf16" else x
                codes, scale = PolarQuant(bits).encode(x.cuda())
                assert torch.equal(codes.cpu(), torch.from_numpy(G[key + "_codes"]))
                assert torch.equal(scale.cpu(), torch.from_numpy(G[key + "_scale"]))
                dec = PolarQuant(bits).decode(codes, scale).cpu().view(torch.int16)
                assert torch.equal(dec, torch.from_numpy(G[key + "_dec_bf16"]))
    ext = ak.load_aether_cuda_kernels()
    got = ext.sparse_sink_attention(*(torch.from_numpy(G[k]).cuda() for k in ("sa_q", "sa_kv", "sa_idx", "sa_sink")),
                                    0.125)
    torch.testing.assert_close(got.cpu(), torch.from_numpy(G["sa_out"]), atol=1e-5, rtol=1e-5)


def test_csa_decode_dirty_workspace(ak):
    """Results never depend on the workspace's previous contents."""
    from aether_kernels.paged import csa_decode_paged, csa_workspace_bytes
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 8, 4000, 30000, 4, 4, seed=23, device="cuda")
    args = (batch.q, batch.index_q, batch.index_weight, batch.sink, batch.window, batch.window_len, batch.cache,
            batch.page_table, batch.nblocks, batch.softmax_scale)
    need = csa_workspace_bytes(8, batch.page_table.shape[1] * 64)
    ref_out, ref_sel = csa_decode_paged(*args, workspace=torch.zeros(need, dtype=torch.uint8, device="cuda"))
    for fill in (7, 255):
        ws = torch.full((need,), fill, dtype=torch.uint8, device="cuda")
        out, sel = csa_decode_paged(*args, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(sel, ref_sel)
        assert torch.equal(out, ref_out)
    _check_decode(batch, ref_out, ref_sel)


@pytest.mark.parametrize("distinct", [2, 40, 300])
def test_csa_decode_repeated_entries(ak, distinct):
    """Index entries drawn from a few distinct vectors: scores repeat many
    times, so the boundary of the top-k falls inside a run of equal keys
    (lowest block indices must win) and the boundary bin holds from tens to
    thousands of keys."""
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 3, 20000, 32000, 4, 4, seed=31 + distinct, device="cuda")
    c = batch.cache
    g = torch.Generator().manual_seed(distinct)
    for row in range(3):
        nbr = int(batch.nblocks[row])
        pages = batch.page_table[row, : (nbr + 63) // 64].long()
        codes = c.idx_codes[pages].reshape(-1, c.idx_codes.shape[-1])[:nbr]
        scales = c.idx_scale[pages].reshape(-1)[:nbr]
        pick = torch.randint(0, distinct, (nbr,), generator=g).to(codes.device)
        new_codes, new_scales = codes[:distinct][pick], scales[:distinct][pick]
        flat_c = c.idx_codes[pages].reshape(-1, c.idx_codes.shape[-1])
        flat_s = c.idx_scale[pages].reshape(-1)
        flat_c[:nbr] = new_codes
        flat_s[:nbr] = new_scales
        c.idx_codes[pages] = flat_c.view(len(pages), 64, -1)
        c.idx_scale[pages] = flat_s.view(len(pages), 64)
    out, sel = _run_decode(ak, batch)
    _check_decode(batch, out, sel)


def test_csa_decode_host_buffers_match_device_path(ak):
    """aether_csa_decode_paged_host (one call: host->device copy, decode,
    device->host copy) returns exactly the device-resident path's result."""
    from aether_kernels.paged import HostDecodeBuffers, csa_decode_paged, csa_decode_paged_host, csa_workspace_bytes
    from aether_kernels.synthetic import make_decode_batch

    b = make_decode_batch("csa", 8, 3000, 20000, 4, 4, seed=77, device="cuda")
    ref_o, ref_s = csa_decode_paged(b.q, b.index_q, b.index_weight, b.sink, b.window, b.window_len, b.cache,
                                    b.page_table, b.nblocks, b.softmax_scale)
    bufs = HostDecodeBuffers(8, 12, 256, "cuda")
    hin = bufs.pack_inputs(b.q, b.index_q, b.index_weight, b.window_len, b.nblocks)
    hout = bufs.new_host_output()
    ws = torch.zeros(csa_workspace_bytes(8, b.page_table.shape[1] * 64), dtype=torch.uint8, device="cuda")
    csa_decode_paged_host(bufs, hin, hout, b.sink, b.window, b.cache, b.page_table, b.softmax_scale, ws)
    torch.cuda.synchronize()
    o, s = bufs.unpack_outputs(hout)
    assert torch.equal(s, ref_s.cpu())
    assert torch.equal(o, ref_o.cpu())


def test_csa_decode_host_buffers_copy_streams(ak):
    """Host-buffer steps on copy streams, two staging slots, kernels ordered
    by the slots' copy-completion words: every step's host result equals the
    device-resident path's, and no bounded wait runs out."""
    from aether_kernels.paged import (CopyStreams, HostDecodeBuffers, csa_decode_paged, csa_decode_paged_host,
                                      csa_workspace_bytes)
    from aether_kernels.synthetic import make_decode_batch

    batches = [make_decode_batch("csa", 8, 3000, 20000, 4, 4, seed=300 + k, device="cuda") for k in range(3)]
    refs = [csa_decode_paged(b.q, b.index_q, b.index_weight, b.sink, b.window, b.window_len, b.cache, b.page_table,
                             b.nblocks, b.softmax_scale) for b in batches]
    bufs = [HostDecodeBuffers(8, 12, 256, "cuda") for _ in range(2)]
    hins = [bufs[0].pack_inputs(b.q, b.index_q, b.index_weight, b.window_len, b.nblocks) for b in batches]
    copies = CopyStreams(torch.device("cuda"))
    ws = torch.zeros(max(csa_workspace_bytes(8, b.page_table.shape[1] * 64) for b in batches), dtype=torch.uint8,
                     device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    steps = 12
    houts = [bufs[0].new_host_output() for _ in range(steps)]
    for i in range(steps):
        b = batches[i % 3]
        csa_decode_paged_host(bufs[i & 1], hins[i % 3], houts[i], b.sink, b.window, b.cache, b.page_table,
                              b.softmax_scale, ws, err, copies=copies, slot=i & 1, overlap_prefetch=True)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert bufs[0].seq == steps // 2 and bufs[1].seq == steps // 2
    for i in range(steps):
        o, s = bufs[0].unpack_outputs(houts[i])
        assert torch.equal(s, refs[i % 3][1].cpu()), i
        assert torch.equal(o, refs[i % 3][0].cpu()), i


def test_csa_decode_host_plan(ak):
    """The prepared host-buffer plan (one short C call per step, alternating
    staging slots): every step's host result equals the device-resident
    path's; fences order the copies; no bounded wait runs out."""
    from aether_kernels.paged import CsaDecodeHostPlan, csa_decode_paged
    from aether_kernels.synthetic import make_decode_batch

    batches = [make_decode_batch("csa", 8, 3000, 20000, 4, 4, seed=400 + k, device="cuda") for k in range(3)]
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for overlap in (False, True):
        for b in batches:
            ref = csa_decode_paged(b.q, b.index_q, b.index_weight, b.sink, b.window, b.window_len, b.cache,
                                   b.page_table, b.nblocks, b.softmax_scale)
            plan = CsaDecodeHostPlan(b.cache, 8, b.page_table.shape[1], window=b.window.shape[1], err=err,
                                     overlap_prefetch=overlap)
            hin = plan.pack_inputs(b.q, b.index_q, b.index_weight, b.window_len, b.nblocks)
            houts = [plan.new_host_output() for _ in range(5)]
            plan.fence(wait_for_copies=False)
            for i in range(5):
                plan.step(hin, houts[i], b.page_table, b.sink, b.window, b.softmax_scale)
            plan.fence(wait_for_copies=True)
            torch.cuda.synchronize()
            for i in range(5):
                o, s = plan.unpack_outputs(houts[i])
                assert torch.equal(s, ref[1].cpu()), (overlap, i)
                assert torch.equal(o, ref[0].cpu()), (overlap, i)
            plan.close()
    assert int(err.item()) == 0
    with pytest.raises(RuntimeError):
        plan.step(hin, houts[0], batches[0].page_table, batches[0].sink, batches[0].window, 1.0)


def test_csa_decode_host_slot_wait_runs_out(ak):
    """A copy-completion word that never reaches its target: the attend
    kernel's bounded poll gives up (after 0.2 s of GPU time), sets the wait-timeout bit and
    the step still completes; the context stays usable."""
    from aether_kernels.paged import CopyStreams, HostDecodeBuffers, csa_decode_paged_host, csa_workspace_bytes
    from aether_kernels.synthetic import make_decode_batch

    b = make_decode_batch("csa", 2, 3000, 20000, 4, 4, seed=91, device="cuda")
    bufs = HostDecodeBuffers(2, 12, 256, "cuda")
    hin = bufs.pack_inputs(b.q, b.index_q, b.index_weight, b.window_len, b.nblocks)
    hout = bufs.new_host_output()
    ws = torch.zeros(csa_workspace_bytes(2, b.page_table.shape[1] * 64), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    bufs.seq = 1000  # the output word holds 0, the step waits for 1000
    csa_decode_paged_host(bufs, hin, hout, b.sink, b.window, b.cache, b.page_table, b.softmax_scale, ws, err,
                          copies=CopyStreams(torch.device("cuda")), slot=0)
    torch.cuda.synchronize()
    assert int(err.item()) & 1
    assert bufs.slot_flags.tolist() == [1001, 1001]
    torch.ones(4, device="cuda").sum().item()  # the context still works


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("d", [128, 64])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tq_lloyd_max_bit_exact(ak, bits, d, dtype):
    """The Lloyd-Max level format: kernel codes, scales and decodes equal the
    oracle's bit for bit (same fp32 level table)."""
    from aether_kernels.codebook import codebook
    from aether_kernels.turbo_quant import PolarQuant

    g = torch.Generator().manual_seed(bits * 1000 + d)
    x = (torch.randn(300, d, generator=g) * 3).to(dtype)
    pq = PolarQuant(bits, codebook="lloyd-max")
    c, s = pq.encode(x.cuda())
    lv, _ = codebook(bits)
    oc, osc = otq.encode_lut(x.float() if dtype == torch.float32 else x, bits, lv)
    assert torch.equal(c.cpu(), oc)
    assert torch.equal(s.cpu(), osc)
    dec = pq.decode(c, s, out_dtype=torch.float32)
    assert torch.equal(dec.cpu(), otq.decode_lut(oc, osc, bits, lv))


def test_csa_decode_fused_output_rope(ak):
    """The fused inverse output RoPE equals the oracle's attention output
    rotated by -position (aether_2b/serving.py:469-472)."""
    from aether_kernels.paged import csa_decode_paged
    from aether_kernels.rope import RopeConfig, get_rope_freqs
    from aether_kernels.synthetic import make_decode_batch
    from oracle import compress as ocmp

    b = make_decode_batch("csa", 6, 3000, 20000, 4, 4, seed=88, device="cuda")
    inv = get_rope_freqs(RopeConfig.yarn(4.0))[:32].float()
    pos = torch.tensor(b.tokens, dtype=torch.int32)
    out, sel = csa_decode_paged(b.q, b.index_q, b.index_weight, b.sink, b.window, b.window_len, b.cache,
                                b.page_table, b.nblocks, b.softmax_scale, rope_positions=pos.cuda(),
                                rope_inv_freq=inv.cuda())
    torch.cuda.synchronize()
    ref = _oracle(b)
    for i in range(6):
        k = min(256, int(b.nblocks[i]))
        assert torch.equal(sel[i, :k].cpu().long(), ref.selected[i]) or ref.near_tie[i]
    rot = torch.stack([ocmp.rope(ref.out[i], (-pos[i:i + 1]).expand(12), inv) for i in range(6)])
    diff = (out.float().cpu() - rot).abs()
    assert diff.max() < MAX_ABS and diff.mean() < MEAN_ABS, (float(diff.max()), float(diff.mean()))
