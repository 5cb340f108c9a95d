"""A prefix saved from a device page pool and restored into another pool
decodes bit-identically (the pages travel as raw quantized bytes)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_restored_prefix_decodes_identically(cuda_device, tmp_path):
    from aether_kernels.paged import TurboQuantPagedCache, csa_decode_paged
    from aether_kernels.prefix_store import HybridCacheLayout, LayerPages, QuantizedPrefixStore, SWACacheMode
    from aether_kernels.synthetic import make_decode_batch

    b = make_decode_batch("csa", 3, 8192, 8192, 4, 4, seed=31, device="cuda")
    store = QuantizedPrefixStore(str(tmp_path), HybridCacheLayout(4, 128, 128, 1), swa_mode=SWACacheMode.ZERO)
    tokens_by_seq = [[(7 * i + s) % 1000 for i in range(8192)] for s in range(3)]
    dst = TurboQuantPagedCache(b.cache.num_pages + 7, 4, "cuda")
    rows = []
    for s in range(3):
        nb = int(b.nblocks[s])
        ids = b.page_table[s, : (nb + 63) // 64].tolist()
        md = store.save_prefix(tokens_by_seq[s], {"csa0": LayerPages(b.cache, ids, nb)})
        got = store.load_pages(store.lookup_prefix(tokens_by_seq[s]), {"csa0": dst},
                               generator=torch.Generator().manual_seed(s))
        table, nb2 = got["csa0"]
        assert nb2 == nb and md.reusable_token_count == 8192
        rows.append(table)
    pt2 = torch.stack(rows).cuda()
    args = (b.q, b.index_q, b.index_weight, b.sink, b.window, b.window_len)
    o1, s1 = csa_decode_paged(*args, b.cache, b.page_table, b.nblocks, b.softmax_scale)
    o2, s2 = csa_decode_paged(*args, dst, pt2, b.nblocks, b.softmax_scale)
    torch.cuda.synchronize()
    assert torch.equal(s1, s2) and torch.equal(o1, o2)
