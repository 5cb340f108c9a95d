"""PagedKVAllocator: the reference's API and LRU / spill behaviour
(aether_kernels/paged_kv_allocator.py:46-252, tests/test_paged_kv_allocator.py),
on CPU; the quantized pools feeding the paged decode kernels on the GPU."""
from pathlib import Path

import pytest
import torch

from aether_kernels.paged_kv_allocator import PagedKVAllocator, quantized_page_shape


def _disk(tmp_path):
    d = tmp_path / "spill"
    d.mkdir()

    def path(key):
        return d / (key.replace(":", "_") + ".pt")

    def write(key, tensors):
        torch.save({n: t.cpu() for n, t in tensors.items()}, path(key))

    def read(key):
        return torch.load(path(key), map_location="cpu", weights_only=True)

    return write, read


def test_spill_to_disk_and_back_keeps_handles_consistent(tmp_path):
    write, read = _disk(tmp_path)
    a = PagedKVAllocator(1, 1, {"hca": (1, 4)}, dtype=torch.float32, device="cpu",
                         write_to_disk=write, read_from_disk=read)
    h = a.allocate("seq")
    for v in (1.0, 2.0, 3.0):
        a.append_page(h, {"hca": torch.full((1, 4), v)})
    # oldest page on disk, middle one on the host, newest on the device
    assert h.page_slots[0] == (None, None)
    assert h.page_slots[1][0] is None and h.page_slots[1][1] is not None
    assert h.page_slots[2][0] is not None and h.page_slots[2][1] is None
    assert (a.device_pages_used(), a.host_pages_used()) == (1, 1)
    pages = a.load_pages(h, (0, 3))
    assert [p["hca"][0, 0].item() for p in pages] == [1.0, 2.0, 3.0]
    assert [p["hca"][0, 3].item() for p in a.load_pages(h)] == [1.0, 2.0, 3.0]
    a.free(h)
    assert (a.device_pages_used(), a.host_pages_used()) == (0, 0)
    assert h.page_slots == []


def test_lru_order_and_touch_on_load():
    a = PagedKVAllocator(2, 4, {"x": (3,)}, dtype=torch.float32, device="cpu")
    h = a.allocate("s")
    for v in range(3):
        a.append_page(h, {"x": torch.full((3,), float(v))})
    assert h.page_slots[0][0] is None          # page 0 was the LRU victim
    a.load_pages(h, (1, 2))                    # touch page 1: page 2 is now LRU
    a.load_pages(h, (0, 1))                    # page 0 back in, page 2 out
    assert h.page_slots[0][0] is not None and h.page_slots[1][0] is not None
    assert h.page_slots[2][0] is None
    assert [p["x"][0].item() for p in a.load_pages(h)] == [0.0, 1.0, 2.0]


def test_error_messages():
    a = PagedKVAllocator(1, 1, {"x": (2,)}, dtype=torch.float32, device="cpu")
    h = a.allocate("s")
    a.append_page(h, {"x": torch.zeros(2)})
    a.append_page(h, {"x": torch.zeros(2)})
    with pytest.raises(MemoryError, match="no write_to_disk handler"):
        a.append_page(h, {"x": torch.zeros(2)})
    b = PagedKVAllocator(1, 0, {"x": (2,)}, dtype=torch.float32, device="cpu")
    hb = b.allocate("t")
    b.append_page(hb, {"x": torch.zeros(2)})
    with pytest.raises(MemoryError, match="no host page can be evicted"):
        b.append_page(hb, {"x": torch.zeros(2)})


def test_page_table_pages_in_a_batch():
    a = PagedKVAllocator(4, 8, {"x": (2,)}, dtype=torch.int32, device="cpu")
    hs = [a.allocate(f"s{i}") for i in range(3)]
    for i, h in enumerate(hs):
        for p in range(2):
            a.append_page(h, {"x": torch.tensor([i, p], dtype=torch.int32)})
    t = a.page_table(hs[:2], max_pages=3)
    assert t.dtype == torch.int32 and tuple(t.shape) == (2, 3)
    pool = a.pool("x")
    for b in range(2):
        for p in range(2):
            assert pool[t[b, p]].tolist() == [b, p]
    with pytest.raises(MemoryError):
        a.page_table(hs)                       # 6 pages > 4 device slots


def test_quantized_page_shape():
    s4, s8 = quantized_page_shape(4), quantized_page_shape(8)
    assert s4 == {"kv": (64 * 64 + 256,), "idx": (64 * 32 + 256,)}
    assert s8 == {"kv": (64 * 128 + 256,), "idx": (64 * 64 + 256,)}
    with pytest.raises(ValueError):
        quantized_page_shape(3)


@pytest.mark.gpu
def test_quantized_pools_feed_paged_decode(cuda_device, tmp_path):
    """Pages that went device -> host -> disk -> device decode exactly as the
    pages they were copied from."""
    from aether_kernels.paged import csa_decode_paged
    from aether_kernels.synthetic import make_decode_batch

    write, read = _disk(tmp_path)
    bits = 4
    batch = make_decode_batch("csa", 6, 2048, 6000, bits, 4, seed=11)
    a = PagedKVAllocator(64, 4, quantized_page_shape(bits), dtype=torch.uint8, device="cuda",
                         write_to_disk=write, read_from_disk=read)
    src = batch.cache
    handles = []
    pt = batch.page_table.cpu()
    for b in range(6):
        h = a.allocate(f"req{b}")
        npg = (int(batch.nblocks[b]) + 63) // 64
        for p in range(npg):
            pid = int(pt[b, p])
            a.append_page(h, {"kv": src.kv_pages[pid], "idx": src.idx_pages[pid]})
        handles.append(h)
    assert any(s[0] is None for h in handles for s in h.page_slots)   # something was spilled
    ref_out, ref_sel = csa_decode_paged(batch.q, batch.index_q, batch.index_weight, batch.sink, batch.window,
                                        batch.window_len, src, batch.page_table, batch.nblocks,
                                        batch.softmax_scale)
    cache = a.as_cache(bits)
    for rows in ([0, 1], [4, 5], [2, 3]):
        table = a.page_table([handles[r] for r in rows], max_pages=batch.page_table.shape[1])
        r = torch.tensor(rows, device=batch.q.device)
        out, sel = csa_decode_paged(batch.q[r], batch.index_q[r], batch.index_weight[r], batch.sink,
                                    batch.window[r], batch.window_len[r], cache, table, batch.nblocks[r],
                                    batch.softmax_scale)
        torch.cuda.synchronize()
        assert torch.equal(sel, ref_sel[r])
        assert torch.equal(out, ref_out[r])
