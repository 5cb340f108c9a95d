"""The allocation-free indexer entry point, checked against the regular one.

aether_csa_indexer_topk_noalloc exists for callers that cannot allocate
device memory when they need the indexer (host callbacks, allocator hooks,
code that runs while a stream is being captured, plugins that only receive
their input and output buffers).  It keeps its scores in a fixed array inside
the library.  This file is collected last so that a run stopping at the first
failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(lib, name, iq, ikv, iw, k, out, scratch=None):
    B, IH, IC = iq.shape
    S = ikv.shape[1]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = [ctypes.c_void_p(iq.data_ptr()), ctypes.c_void_p(ikv.data_ptr()), ctypes.c_void_p(iw.data_ptr()),
            B, IH, IC, S, k]
    if scratch is not None:
        args.append(ctypes.c_void_p(scratch.data_ptr()))
    args += [ctypes.c_void_p(out.data_ptr()), stream]
    return getattr(lib, name)(*args)


def test_noalloc_indexer_matches_regular_entry_point(cuda_device):
    from aether_kernels import _lib

    lib = _lib.load()
    for call, (B, S, k) in enumerate([(4, 5000, 256), (3, 1200, 100)]):  # two calls in a row
        g = torch.Generator().manual_seed(100 + call)
        iq = torch.randn(B, 4, 64, generator=g).cuda()
        ikv = torch.randn(B, S, 64, generator=g).cuda()
        iw = torch.randn(B, 4, generator=g).cuda()
        ref = torch.empty(B, k, dtype=torch.int64, device="cuda")
        got = torch.full((B, k), -7, dtype=torch.int64, device="cuda")
        scratch = torch.empty(B * S, dtype=torch.float32, device="cuda")
        assert _call(lib, "aether_csa_indexer_topk", iq, ikv, iw, k, ref, scratch) == 0, _lib.last_error()
        assert _call(lib, "aether_csa_indexer_topk_noalloc", iq, ikv, iw, k, got) == 0, _lib.last_error()
        torch.cuda.synchronize()
        # same kernels on the same inputs: identical (score desc, index asc) lists
        assert torch.equal(got, ref)


def test_noalloc_indexer_rejects_oversize(cuda_device):
    from aether_kernels import _lib

    lib = _lib.load()
    cap = lib.aether_csa_indexer_topk_noalloc_max_scores()
    B, S = 32, 60000  # 1.92 M scores > 1 Mi
    assert B * S > cap
    iq = torch.zeros(B, 4, 64, device="cuda")
    ikv = torch.zeros(1, 1, 64, device="cuda").expand(B, S, 64)  # never read: the call is rejected first
    iw = torch.zeros(B, 4, device="cuda")
    out = torch.empty(B, 8, dtype=torch.int64, device="cuda")
    rc = _call(lib, "aether_csa_indexer_topk_noalloc", iq, ikv, iw, 8, out)
    assert rc == 1
    assert "exceeds the built-in scratch" in _lib.last_error()
