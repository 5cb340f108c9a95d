"""The optional e4m3 prefill indexer (the paper's low-precision CSA indexer,
Aether.txt:765-769, 1087-1093).  Its scores are approximate, so its parity is
a recall: the share of the exact top-k blocks (the CPU oracle,
aether_2b/modeling.py:609-615) that it also selects.  The attention over the
blocks it selects is checked against the oracle as usual."""
import pytest
import torch

from oracle import prefill as opf

pytestmark = pytest.mark.gpu

# measured on B200 for these seeded inputs, with margin: 4-bit codes are exact
# in e4m3, only the query is rounded; 8-bit codes are rounded as well
MIN_RECALL = {4: 0.97, 8: 0.95}
MIN_ROW_RECALL = {4: 0.80, 8: 0.75}


@pytest.mark.parametrize("bits", [4, 8])
def test_prefill_fp8_indexer_recall_and_attention(cuda_device, bits):
    from aether_kernels.prefill import PrefillRequest, csa_prefill_chunk
    from aether_kernels.synthetic import make_decode_batch
    from oracle import decode as odec
    from oracle import turboquant as otq

    batch = make_decode_batch("csa", 3, 2400, 14000, bits, 4, seed=160 + bits, device="cuda")
    nq = [70, 33, 130]
    reqs, Q = [], 0
    for b, n in enumerate(nq):
        reqs.append(PrefillRequest(Q, n, max(0, batch.tokens[b] - n), int(batch.nblocks[b])))
        Q += n
    g = torch.Generator().manual_seed(9 + bits)
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
                                 batch.page_table, reqs, batch.softmax_scale, err=err, indexer="fp8")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    c = batch.cache
    sels, _ = opf.prefill_topk(iq, iw, c.idx_codes.cpu(), c.idx_scale.cpu(), batch.page_table.cpu(),
                               [(r.first_row, r.num_queries, r.position, r.nblocks) for r in reqs], bits, 256)
    ids, out = ids.cpu(), out.float().cpu()
    kvc, kvs, pt = c.kv_codes.cpu(), c.kv_scale.cpu(), batch.page_table.cpu()
    hit = tot = 0
    worst_row = 1.0
    worst, total, n = 0.0, 0.0, 0
    for ri, r in enumerate(reqs):
        main = otq.decode(odec.gather_pages(kvc, pt[ri], r.nblocks),
                          odec.gather_pages(kvs, pt[ri], r.nblocks).unsqueeze(-1), bits)
        for i in range(r.num_queries):
            row = r.first_row + i
            k = sels[row].numel()
            got = ids[row, :k].long()
            assert (ids[row, k:] == -1).all(), f"row {row}: as many blocks as the exact indexer"
            assert torch.equal(got, torch.sort(got).values) and bool((got >= 0).all()), f"row {row}: ids"
            common = len(set(got.tolist()) & set(sels[row].tolist()))
            hit += common
            tot += k
            worst_row = min(worst_row, common / k)
            t = r.position + i
            wl = min(128, t + 1)
            w0 = first[ri] + i + (128 - wl)
            src = torch.cat([main[got], window[w0: w0 + wl].float()], dim=0)
            ref = odec.sink_attention(q[row].float(), src, sink, batch.softmax_scale)
            d = (out[row] - ref).abs()
            worst = max(worst, float(d.max()))
            total += float(d.sum())
            n += d.numel()
    recall = hit / tot
    print(f"fp8 indexer {bits}-bit: recall {recall:.4f}, worst row {worst_row:.3f}")
    assert recall >= MIN_RECALL[bits] and worst_row >= MIN_ROW_RECALL[bits], (recall, worst_row)
    assert worst < 2e-2 and total / n < 1e-3, (worst, total / n)
