"""Host-side logic on the CPU: the loader contract the reference's tests pin
(tests/test_cuda_loader.py:12-29), error messages of the PolarQuant API
(aether_2b/turbo_quant.py:59, 99), the page allocator and the seeded input
generator."""
import pytest
import torch


def test_cuda_build_environment_keys():
    from aether_kernels.loader import cuda_build_environment

    assert set(cuda_build_environment()) == {
        "torch_cuda_built", "torch_cuda_available", "cuda_home", "nvcc", "conda_target_include",
        "conda_target_lib", "cuda_runtime_lib",
    }


def test_unavailable_reason_consistent_without_device():
    from aether_kernels.loader import cuda_extension_unavailable_reason

    if torch.cuda.is_available():
        pytest.skip("host without a GPU only")
    assert cuda_extension_unavailable_reason(require_device=True) == \
        "No CUDA device is available for executing the custom kernels."


def test_polarquant_api_errors():
    from aether_kernels.turbo_quant import PolarQuant, _wht

    with pytest.raises(ValueError, match="bits must be 4 or 8"):
        PolarQuant(bits=3)
    with pytest.raises(ValueError, match="power of 2"):
        _wht(torch.randn(3, 12))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        PolarQuant(8).encode(torch.randn(2, 128))


def test_page_pool_allocation_cpu():
    from aether_kernels.paged import TurboQuantPagedCache

    c = TurboQuantPagedCache(10, 4, "cpu")
    assert c.kv_pages.shape == (10, 64 * 64 + 256) and c.idx_pages.shape == (10, 64 * 32 + 256)
    assert c.kv_codes.shape == (10, 64, 64) and c.kv_scale.shape == (10, 64)
    c.kv_scale[3, 5] = 2.5  # views write through to the page
    assert c.kv_pages[3, 64 * 64 + 20: 64 * 64 + 24].view(torch.float32).item() == 2.5
    g = torch.Generator().manual_seed(1)
    a = c.alloc_pages(4, generator=g)
    b = c.alloc_pages(6)
    assert len(set(a) | set(b)) == 10 and c.free_pages == 0
    with pytest.raises(MemoryError):
        c.alloc_pages(1)
    c.release_pages(a)
    assert c.free_pages == 4
    with pytest.raises(ValueError):
        TurboQuantPagedCache(2, 5, "cpu")


def test_sink_attention_handles_empty_sources():
    from oracle import decode as odec

    q = torch.randn(12, 128)
    out = odec.sink_attention(q, torch.empty(0, 128), torch.zeros(12), 0.1)
    assert torch.equal(out, torch.zeros_like(q))
