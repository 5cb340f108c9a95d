"""CPU checks of the host-side bookkeeping around the kernels: the per-query
rows of chunked prefill (causal visibility, aether_2b/modeling.py:612-614,
and the causal 128-token window), the prefill tile plan, and the packed
staging layout of the host-buffer decode.  No kernel runs."""
import torch

from aether_kernels.paged import HostDecodeBuffers
from aether_kernels.prefill import QUERIES_PER_CTA, PrefillRequest, _plan, query_rows


def test_query_rows_visibility_and_window():
    reqs = [PrefillRequest(0, 5, 0, 3), PrefillRequest(5, 70, 1000, 267)]
    first = [0, 200]
    q_row, vis, wrow, wlen = query_rows(reqs, 4, 128, first, "cpu")
    assert q_row.tolist() == [0] * 5 + [1] * 70
    # a query at position t sees blocks s < t // 4, capped by the cache
    assert vis[:5].tolist() == [min(3, t // 4) for t in range(5)]
    assert vis[5:].tolist() == [min(267, t // 4) for t in range(1000, 1070)]
    # the window ends at the query's own token: min(128, t + 1) rows
    assert wlen[:5].tolist() == [t + 1 for t in range(5)]
    assert (wlen[5:] == 128).all()
    # rows of the flat buffer: request r's row of position p is
    # first[r] + (p - (position - 127)); the window's first row is p = t - wlen + 1
    for i in range(5):
        t = i
        assert int(wrow[i]) == first[0] + (t - int(wlen[i]) + 1) - (0 - 127)
    for i in range(70):
        t = 1000 + i
        assert int(wrow[5 + i]) == first[1] + (t - 127) - (1000 - 127)
    assert wrow.dtype == torch.int64 and vis.dtype == torch.int32


def test_plan_tiles_cover_every_query_once():
    reqs = [PrefillRequest(0, 70, 0, 10), PrefillRequest(70, 32, 500, 125), PrefillRequest(102, 1, 9, 2)]
    info, tiles, n = _plan(reqs, "cpu")
    assert info.tolist() == [[0, 70, 0, 10], [70, 32, 500, 125], [102, 1, 9, 2]]
    assert n == tiles.shape[0] == 3 + 1 + 1
    covered = []
    for r, q0 in tiles.tolist():
        covered += [(r, q) for q in range(q0, min(q0 + QUERIES_PER_CTA, reqs[r].num_queries))]
    assert sorted(covered) == [(r, q) for r, req in enumerate(reqs) for q in range(req.num_queries)]


def test_host_decode_staging_layout():
    """Packed fields are 256-byte aligned, in the order the C entry expects,
    and the views alias the staging buffers."""
    bufs = HostDecodeBuffers(64, 12, 256, "cpu")
    assert bufs.in_offsets[0] == 0 and bufs.out_offsets[0] == 0
    for offs, total in ((bufs.in_offsets, bufs.in_bytes), (bufs.out_offsets, bufs.out_bytes)):
        assert all(o % 256 == 0 for o in offs) and total % 256 == 0
        assert list(offs) == sorted(offs) and offs[-1] < total
    q, iq, iw, wl, nb = bufs.inputs
    assert q.shape == (64, 12, 128) and q.dtype == torch.bfloat16
    assert iq.shape == (64, 4, 64) and iw.shape == (64, 4) and wl.shape == (64,) and nb.shape == (64,)
    assert bufs.out.shape == (64, 12, 128) and bufs.indices.shape == (64, 256)
    # 64*12*128*2 + 64*4*64*4 + 64*4*4 + 2 * 256 (two small int32 fields, 256-byte aligned)
    assert bufs.in_bytes == 196608 + 65536 + 1024 + 256 + 256
    assert bufs.out_bytes == 196608 + 65536
    nb.fill_(7)
    assert bufs.dev_in[bufs.in_offsets[4]: bufs.in_offsets[4] + 4].view(torch.int32).item() == 7
    # a host result buffer unpacks into the same views
    host = torch.zeros(bufs.out_bytes, dtype=torch.uint8)
    o, s = bufs.unpack_outputs(host)
    s[3, 5] = 42
    assert host[bufs.out_offsets[1]:].view(torch.int32)[3 * 256 + 5].item() == 42
