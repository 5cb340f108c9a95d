"""GPU parity of the tcgen05 chunked-prefill indexer: exact top-k block sets
per query token against the CPU oracle (aether_2b/modeling.py:591-615 with
the causal block mask), near-tie rows reported, not failed."""
import pytest
import torch

from oracle import prefill as opf

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(cuda_device):
    from aether_kernels import _lib

    _lib.load()


def _requests(batch, nq_list):
    from aether_kernels.prefill import PrefillRequest

    reqs, row = [], 0
    for b, nq in enumerate(nq_list):
        toks = batch.tokens[b]
        nblk = int(batch.nblocks[b])
        pos0 = max(0, toks - nq)
        reqs.append(PrefillRequest(row, nq, pos0, nblk))
        row += nq
    return reqs, row


def _run(batch, nq_list, top_k=256, seed=0):
    from aether_kernels.prefill import csa_prefill_topk

    reqs, Q = _requests(batch, nq_list)
    g = torch.Generator().manual_seed(seed)
    iq = torch.randn(Q, 4, 64, generator=g)
    iw = torch.randn(Q, 4, generator=g)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    keys, ids = csa_prefill_topk(iq.cuda(), iw.cuda(), batch.cache, batch.page_table, reqs, top_k=top_k, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    c = batch.cache
    sels, ties = opf.prefill_topk(iq, iw, c.idx_codes.cpu(), c.idx_scale.cpu(), batch.page_table.cpu(),
                                  [(r.first_row, r.num_queries, r.position, r.nblocks) for r in reqs], batch.bits,
                                  top_k)
    ids = ids.cpu()
    keys = keys.cpu()
    mism = 0
    for row, (ref, tie) in enumerate(zip(sels, ties)):
        k = ref.numel()
        got = ids[row]
        assert (got[k:] == -1).all() and (keys[row, k:] == 0).all(), f"row {row}: padding"
        got = got[:k].long()
        assert torch.equal(got, torch.sort(got).values), f"row {row}: ids not ascending"
        if not torch.equal(got, ref):
            assert tie, f"row {row}: selection differs outside the near-tie band"
            mism += 1
    return mism, len(sels)


@pytest.mark.parametrize("bits", [4, 8])
def test_prefill_topk_matches_oracle(lib, bits):
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 3, 2400, 14000, bits, 4, seed=50 + bits, device="cuda")
    mism, n = _run(batch, [70, 33, 130], seed=bits)
    assert mism <= max(1, n // 100)


def test_prefill_topk_short_context_and_small_k(lib):
    """Queries that see fewer blocks than top_k take them all; top_k < 256."""
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 2, 500, 1100, 4, 4, seed=7, device="cuda")
    mism, _ = _run(batch, [64, 40], top_k=256, seed=3)
    assert mism == 0
    mism, _ = _run(batch, [64, 40], top_k=40, seed=4)
    assert mism <= 1


def test_prefill_topk_repeated_entries(lib):
    """Identical index entries: equal scores; the lower block index wins."""
    from aether_kernels.synthetic import make_decode_batch

    batch = make_decode_batch("csa", 2, 6000, 8000, 8, 4, seed=9, device="cuda")
    c = batch.cache
    g = torch.Generator().manual_seed(1)
    for row in range(2):
        nbr = int(batch.nblocks[row])
        pages = batch.page_table[row, : (nbr + 63) // 64].long()
        flat_c = c.idx_codes[pages].reshape(-1, c.idx_codes.shape[-1])
        flat_s = c.idx_scale[pages].reshape(-1)
        pick = torch.randint(0, 5, (nbr,), generator=g).to(flat_c.device)
        flat_c[:nbr] = flat_c[:5][pick].clone()
        flat_s[:nbr] = flat_s[:5][pick].clone()
        c.idx_codes[pages] = flat_c.view(len(pages), 64, -1)
        c.idx_scale[pages] = flat_s.view(len(pages), 64)
    mism, _ = _run(batch, [40, 50], seed=5)
    assert mism == 0


@pytest.mark.parametrize("bits", [4, 8])
def test_prefill_chunk_attention_matches_oracle(lib, bits):
    """Indexer + attention for every query token of the chunks: the output
    matches the fp32 oracle's sink attention over the selected blocks and the
    causal window within the decode tolerance (2e-2 max, 1e-3 mean abs)."""
    from aether_kernels.prefill import csa_prefill_chunk
    from aether_kernels.synthetic import make_decode_batch
    from oracle import decode as odec
    from oracle import turboquant as otq

    batch = make_decode_batch("csa", 3, 2400, 14000, bits, 4, seed=60 + bits, device="cuda")
    nq = [70, 33, 130]
    reqs, Q = _requests(batch, nq)
    g = torch.Generator().manual_seed(bits)
    H = 12
    iq = torch.randn(Q, 4, 64, generator=g)
    iw = torch.randn(Q, 4, generator=g)
    q = torch.randn(Q, H, 128, generator=g).to(torch.bfloat16)
    sink = torch.randn(H, generator=g)
    first, rows = [], 0
    for r in reqs:
        first.append(rows)
        rows += 127 + r.num_queries
    window = torch.randn(rows, 128, generator=g).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, ids = csa_prefill_chunk(q.cuda(), iq.cuda(), iw.cuda(), sink.cuda(), window.cuda(), first, batch.cache,
                                 batch.page_table, reqs, batch.softmax_scale, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    c = batch.cache
    sels, ties = opf.prefill_topk(iq, iw, c.idx_codes.cpu(), c.idx_scale.cpu(), batch.page_table.cpu(),
                                  [(r.first_row, r.num_queries, r.position, r.nblocks) for r in reqs], bits, 256)
    ids, out = ids.cpu(), out.float().cpu()
    kvc, kvs, pt = c.kv_codes.cpu(), c.kv_scale.cpu(), batch.page_table.cpu()
    worst, total, n = 0.0, 0.0, 0
    for ri, r in enumerate(reqs):
        main = otq.decode(odec.gather_pages(kvc, pt[ri], r.nblocks), odec.gather_pages(kvs, pt[ri], r.nblocks).unsqueeze(-1),
                          bits)
        for i in range(r.num_queries):
            row = r.first_row + i
            t = r.position + i
            k = sels[row].numel()
            got = ids[row, :k].long()
            assert ties[row] or torch.equal(got, sels[row]), f"row {row}: selection"
            assert (ids[row, k:] == -1).all(), f"row {row}: unused index slots hold -1"
            wl = min(128, t + 1)
            w0 = first[ri] + i + (128 - wl)
            src = torch.cat([main[got], window[w0: w0 + wl].float()], dim=0)
            ref = odec.sink_attention(q[row].float(), src, sink, batch.softmax_scale)
            d = (out[row] - ref).abs()
            worst = max(worst, float(d.max()))
            total += float(d.sum())
            n += d.numel()
    assert worst < 2e-2, worst
    assert total / n < 1e-3, total / n


def test_prefill_config4_shape(lib):
    """BASELINE config 4 at its own shape: 8 requests, each a 4096-token
    chunk at positions 65536..69631 against 16384 + 1024 cached 4-bit blocks
    (every query's streaming top-k prunes its candidate buffer many times).
    A strided subsample of 256 query rows per request is checked against the
    oracle: exact top-256 sets outside the near-tie band, attention within
    2e-2 max-abs / 1e-3 mean-abs."""
    from aether_kernels.prefill import PrefillRequest, csa_prefill_chunk
    from aether_kernels.synthetic import make_decode_batch
    from oracle import decode as odec
    from oracle import turboquant as otq

    R, NQ, POS0, bits, H = 8, 4096, 65536, 4, 12
    nblk = (POS0 + NQ) // 4
    batch = make_decode_batch("csa", R, POS0 + NQ, POS0 + NQ, bits, 4, seed=404, device="cuda",
                              gen_device="cuda")
    assert int(batch.nblocks.min()) == nblk
    reqs = [PrefillRequest(r * NQ, NQ, POS0, nblk) for r in range(R)]
    Q = R * NQ
    g = torch.Generator(device="cuda").manual_seed(44)
    iq = torch.randn(Q, 4, 64, generator=g, device="cuda")
    iw = torch.randn(Q, 4, generator=g, device="cuda")
    q = torch.randn(Q, H, 128, generator=g, device="cuda").to(torch.bfloat16)
    sink = torch.randn(H, generator=g, device="cuda")
    first = [r * (127 + NQ) for r in range(R)]
    window = torch.randn(R * (127 + NQ), 128, generator=g, device="cuda").to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, ids = csa_prefill_chunk(q, iq, iw, sink, window, first, batch.cache, batch.page_table, reqs,
                                 batch.softmax_scale, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    rows = [r * NQ + i for r in range(R) for i in range(0, NQ, NQ // 256)]
    c = batch.cache
    pt = batch.page_table.cpu()
    sels, ties = opf.prefill_topk(iq.cpu(), iw.cpu(), c.idx_codes.cpu(), c.idx_scale.cpu(), pt,
                                  [(r.first_row, r.num_queries, r.position, r.nblocks) for r in reqs], bits, 256,
                                  rows=rows)
    ids, out, q, window, sink = ids.cpu(), out.float().cpu(), q.cpu(), window.cpu(), sink.cpu()
    kvc, kvs = c.kv_codes.cpu(), c.kv_scale.cpu()
    worst, total, n, mism = 0.0, 0.0, 0, 0
    for ri in range(R):
        main = otq.decode(odec.gather_pages(kvc, pt[ri], nblk), odec.gather_pages(kvs, pt[ri], nblk).unsqueeze(-1),
                          bits)
        for j, row in enumerate(rows):
            if not ri * NQ <= row < (ri + 1) * NQ:
                continue
            i = row - ri * NQ
            ref_sel, tie = sels[j], ties[j]
            got = ids[row, :256].long()
            assert torch.equal(got, torch.sort(got).values), f"row {row}: ids not ascending"
            if not torch.equal(got, ref_sel):
                assert tie, f"row {row}: selection differs outside the near-tie band"
                mism += 1
            w0 = first[ri] + i  # window rows [first + i, first + i + 128): 127 earlier tokens and this one
            src = torch.cat([main[got], window[w0: w0 + 128].float()], dim=0)
            ref = odec.sink_attention(q[row].float(), src, sink, batch.softmax_scale)
            d = (out[row] - ref).abs()
            worst = max(worst, float(d.max()))
            total += float(d.sum())
            n += d.numel()
    assert mism <= len(rows) // 100
    assert worst < 2e-2, worst
    assert total / n < 1e-3, total / n


@pytest.mark.parametrize("bits,H,top_k", [(4, 5, 256), (8, 16, 64)])
def test_prefill_attention_sequence_start(lib, bits, H, top_k):
    """Query tokens from position 0: the first tokens see no compressed
    block (an empty candidate list) and windows shorter than 128 rows; later
    ones see fewer than top_k blocks.  Odd head counts and a short top-k."""
    from aether_kernels.prefill import PrefillRequest, csa_prefill_chunk
    from aether_kernels.synthetic import make_decode_batch
    from oracle import decode as odec
    from oracle import turboquant as otq

    batch = make_decode_batch("csa", 2, 1200, 1600, bits, 4, seed=90 + bits, device="cuda")
    nq = [300, 157]
    reqs, Q = [], 0
    for b, n in enumerate(nq):
        reqs.append(PrefillRequest(Q, n, 0, int(batch.nblocks[b])))
        Q += n
    g = torch.Generator().manual_seed(7 + bits)
    iq = torch.randn(Q, 4, 64, generator=g)
    iw = torch.randn(Q, 4, generator=g)
    q = torch.randn(Q, H, 128, generator=g).to(torch.bfloat16)
    sink = torch.randn(H, generator=g)
    first, rows = [], 0
    for r in reqs:
        first.append(rows)
        rows += 127 + r.num_queries
    window = torch.randn(rows, 128, generator=g).to(torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out, ids = csa_prefill_chunk(q.cuda(), iq.cuda(), iw.cuda(), sink.cuda(), window.cuda(), first, batch.cache,
                                 batch.page_table, reqs, batch.softmax_scale, top_k=top_k, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    c = batch.cache
    sels, ties = opf.prefill_topk(iq, iw, c.idx_codes.cpu(), c.idx_scale.cpu(), batch.page_table.cpu(),
                                  [(r.first_row, r.num_queries, r.position, r.nblocks) for r in reqs], bits, top_k)
    ids, out = ids.cpu(), out.float().cpu()
    kvc, kvs, pt = c.kv_codes.cpu(), c.kv_scale.cpu(), batch.page_table.cpu()
    worst, total, n = 0.0, 0.0, 0
    for ri, r in enumerate(reqs):
        main = otq.decode(odec.gather_pages(kvc, pt[ri], r.nblocks), odec.gather_pages(kvs, pt[ri], r.nblocks).unsqueeze(-1),
                          bits)
        for i in range(r.num_queries):
            row = r.first_row + i
            k = sels[row].numel()
            assert k == min(top_k, i // 4)
            got = ids[row, :k].long()
            assert ties[row] or torch.equal(got, sels[row]), f"row {row}: selection"
            assert (ids[row, k:] == -1).all(), f"row {row}: unused index slots hold -1"
            wl = min(128, i + 1)
            w0 = first[ri] + i + (128 - wl)
            src = torch.cat([main[got], window[w0: w0 + wl].float()], dim=0)
            ref = odec.sink_attention(q[row].float(), src, sink, batch.softmax_scale)
            d = (out[row] - ref).abs()
            worst = max(worst, float(d.max()))
            total += float(d.sum())
            n += d.numel()
    assert worst < 2e-2, worst
    assert total / n < 1e-3, total / n
