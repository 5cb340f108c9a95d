"""The drop-in ops of aether_kernels.sparse_attention against the reference's
own CUDA extension (its aether_kernels/csrc, built for sm_100a by
oracle/build_ref.py into oracle/_ref/), called with identical arguments.
Skipped when that build is absent.  csa_indexer_topk is not compared: the
reference kernel computes sum_h relu(w_h) * (q_h . k), the model's indexer
(and this package) sum_h softplus(w_h) * relu(q_h . k)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_ext():
    from oracle.build_ref import load_built

    mod = load_built()
    if mod is None:
        pytest.skip("reference extension not built (oracle/build_ref.py)")
    return mod


@pytest.mark.parametrize("T,dtype", [(1, torch.bfloat16), (4, torch.bfloat16), (1, torch.float32)])
def test_sparse_sink_attention_matches_reference_kernel(cuda_device, ref_ext, T, dtype):
    from aether_kernels.sparse_attention import sparse_sink_attention

    g = torch.Generator(device="cuda").manual_seed(11 + T)
    B, H, D, S, K = 6, 12, 128, 700, 384
    q = torch.randn(B, T, H, D, generator=g, device="cuda").to(dtype)
    kv = torch.randn(B, S, 2, D, generator=g, device="cuda").to(dtype)
    idx = torch.randint(0, S, (B, T, K), generator=g, device="cuda", dtype=torch.int64)
    idx[:, :, -5:] = S + 3  # out of range: skipped by both
    sink = torch.randn(H, generator=g, device="cuda").to(dtype)
    ours = sparse_sink_attention(q, kv, idx, sink, D ** -0.5)
    ref = ref_ext.sparse_sink_attention(q, kv, idx, sink, D ** -0.5)
    torch.cuda.synchronize()
    d = (ours.float() - ref.float()).abs()
    assert ours.shape == ref.shape and ours.dtype == ref.dtype
    assert float(d.max()) < 2e-2 and float(d.mean()) < 1e-3, (float(d.max()), float(d.mean()))


def test_hca_compress_matches_reference_kernel(cuda_device, ref_ext):
    from aether_kernels.sparse_attention import hca_compress

    g = torch.Generator(device="cuda").manual_seed(5)
    c = torch.randn(8, 128, 128, generator=g, device="cuda")
    z = torch.randn(8, 128, 128, generator=g, device="cuda") * 3
    ours, ref = hca_compress(c, z), ref_ext.hca_compress(c, z)
    torch.cuda.synchronize()
    assert torch.allclose(ours, ref, rtol=1e-4, atol=1e-5), float((ours - ref).abs().max())


def test_sparse_sink_attention_speed_against_reference_kernel(cuda_device, ref_ext):
    """Config-1 decode shape through the literal drop-in op: 64 sequences, 12
    heads, 256 selected blocks + 128 window rows gathered from 8320 sources.
    Reports both times; ours must not be slower."""
    from aether_kernels.sparse_attention import sparse_sink_attention

    g = torch.Generator(device="cuda").manual_seed(3)
    B, H, D, S, K = 64, 12, 128, 8320, 384
    q = torch.randn(B, 1, H, D, generator=g, device="cuda").to(torch.bfloat16)
    kv = torch.randn(B, S, 2, D, generator=g, device="cuda").to(torch.bfloat16)
    idx = torch.randint(0, S, (B, 1, K), generator=g, device="cuda", dtype=torch.int32)
    sink = torch.randn(H, generator=g, device="cuda").to(torch.bfloat16)

    def time(fn, n=50):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n * 1e3

    t_ours = time(lambda: sparse_sink_attention(q, kv, idx, sink, D ** -0.5))
    t_ref = time(lambda: ref_ext.sparse_sink_attention(q, kv, idx, sink, D ** -0.5))
    print(f"sparse_sink_attention B64 H12 K384: ours {t_ours:.1f} us, reference kernel {t_ref:.1f} us")
    assert t_ours <= t_ref * 1.05, (t_ours, t_ref)
