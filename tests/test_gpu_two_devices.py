"""One process driving two GPUs: the kernels' shared-memory attributes are set
per device, so a launch on cuda:1 after cuda:0 has run must succeed and give
the same result for the same inputs (the reference's layer-sharded serving
moves layers between devices inside one process, aether_2b/serving.py
_run_backend).  Skipped with fewer than two GPUs."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_decode_on_two_devices_in_one_process():
    from aether_kernels.paged import csa_decode_paged, hca_decode_paged
    from aether_kernels.synthetic import make_decode_batch

    results = []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            b = make_decode_batch("csa", 4, 4096, 32768, 4, 4, seed=5, device=dev)
            err = torch.zeros(1, dtype=torch.int32, device=dev)
            out, sel = csa_decode_paged(b.q, b.index_q, b.index_weight, b.sink, b.window, b.window_len, b.cache,
                                        b.page_table, b.nblocks, b.softmax_scale, top_k=b.top_k, err=err)
            h = make_decode_batch("hca", 4, 8192, 131072, 4, 128, seed=6, device=dev)
            hout = hca_decode_paged(h.q, h.sink, h.window, h.window_len, h.cache, h.page_table, h.nblocks,
                                    h.softmax_scale, err=err)
            torch.cuda.synchronize(dev)
            assert int(err.item()) == 0
            results.append((out.cpu(), sel.cpu(), hout.cpu()))
    for a, b in zip(*results):
        assert torch.equal(a, b)
