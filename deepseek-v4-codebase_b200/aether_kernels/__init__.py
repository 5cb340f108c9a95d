"""B200-native (sm_100a) kernels for Aether-2B's CSA/HCA decode path over a
paged TurboQuant KV cache, behind the reference's ``aether_kernels`` API."""
from .loader import cuda_build_environment, cuda_extension_unavailable_reason, load_aether_cuda_kernels
from .sparse_attention import sparse_sink_attention
from .paged import TurboQuantPagedCache, csa_decode_paged, hca_decode_paged
from .prefix_store import QuantizedPrefixStore
from .engine import AttentionLayerSpec, DecodeRound

__all__ = [
    "cuda_build_environment",
    "cuda_extension_unavailable_reason",
    "load_aether_cuda_kernels",
    "sparse_sink_attention",
    "TurboQuantPagedCache",
    "csa_decode_paged",
    "hca_decode_paged",
    "QuantizedPrefixStore",
    "AttentionLayerSpec",
    "DecodeRound",
]
