"""ctypes binding of the C-ABI library ``libaether_b200.so`` (sm_100a kernels).

The shared library is built in-tree by ``aether_kernels._build.build()`` (or
``__graft_entry__.build()``); there is no fallback of any kind: if the
library is missing or was not built for this device, every op raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path
from typing import Optional

LIB_NAME = "libaether_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

_c_int = ctypes.c_int
_c_ll = ctypes.c_longlong
_c_f = ctypes.c_float
_p = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/aether_b200.h
SIGNATURES = {
    "aether_last_error": (ctypes.c_char_p, []),
    "aether_abi_version": (_c_int, []),
    "aether_compiled_arch": (_c_int, []),
    "aether_tq_encode": (_c_int, [_p, _c_int, _c_ll, _c_int, _c_int, _p, _p, _p, _p, _p]),
    "aether_tq_encode_into_pages": (
        _c_int,
        [_p, _c_int, _c_int, _c_int, _c_int, _c_int, _p, _p, _c_int, _p, _c_int, _p, _p, _p],
    ),
    "aether_compress_emit": (
        _c_int,
        [_p, _p, _p, _c_int, _p, _p, _p, _c_int, _p, _c_int, _c_int, _c_int,   # segments, has_seg1, dtype, B, d
         _p, _p, _c_int, _p, _c_f, _c_int, _p,                              # positions .. bits, diag
         _p, _c_int, _p, _c_int, _p, _p, _p, _p],                           # page_table .. err, stream
    ),
    "aether_tq_encode_lut": (_c_int, [_p, _c_int, _c_ll, _c_int, _c_int, _p, _p, _c_f, _p, _p, _p]),
    "aether_tq_decode_lut": (_c_int, [_p, _p, _c_ll, _c_int, _c_int, _p, _p, _p, _c_int, _p]),
    "aether_tq_decode": (_c_int, [_p, _p, _c_ll, _c_int, _c_int, _p, _p, _c_int, _p]),
    "aether_wht": (_c_int, [_p, _p, _c_ll, _c_int, _p]),
    "aether_sparse_sink_attention": (
        _c_int,
        [_p, _p, _p, _c_int, _p, _c_int, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_f, _p],
    ),
    "aether_tiled_prefill_attention": (
        _c_int,
        [_p, _p, _p, _c_int, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_f, _c_int, _p],
    ),
    "aether_csa_indexer_topk_scratch_bytes": (ctypes.c_size_t, [_c_int, _c_int]),
    "aether_csa_indexer_topk": (
        _c_int,
        [_p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _p, _p, _p],
    ),
    "aether_csa_indexer_topk_noalloc_max_scores": (_c_ll, []),
    "aether_csa_indexer_topk_noalloc": (
        _c_int,
        [_p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _p, _p],
    ),
    "aether_hca_compress": (_c_int, [_p, _p, _p, _c_int, _c_int, _c_int, _c_int, _p]),
    "aether_csa_decode_paged": (
        _c_int,
        [
            _p, _p, _p, _p, _p, _p,            # q, index_q, index_w, sink, window, window_len
            _p, _p,                            # idx_pages, kv_pages
            _p, _c_int, _c_int, _p, _c_int,    # page_table, stride, num_pages, nblocks, max_nblocks
            _p, _p,                            # diag_idx, diag_kv
            _c_int, _c_int, _c_int, _c_int, _c_int, _c_f,  # B, H, W, bits, top_k, scale
            _p, _p, _p, _p, _c_int, _c_int, _p,  # out, sel_out, workspace, err, cluster, pdl, stream
        ],
    ),
    "aether_csa_decode_paged_scores": (
        _c_int,
        [
            _p, _p, _p, _p, _p, _p,
            _p, _p,
            _p, _c_int, _c_int, _p, _c_int,
            _p, _p,
            _c_int, _c_int, _c_int, _c_int, _c_int, _c_f,
            _p, _p, _p, _c_int, _p, _p, _c_int, _c_int, _p,  # out, sel, score_out, stride, ws, err, cluster, pdl, stream
        ],
    ),
    "aether_csa_decode_paged_levels": (
        _c_int,
        [
            _p, _p, _p, _p, _p, _p,            # q, index_q, index_w, sink, window, window_len
            _p, _p,                            # idx_pages, kv_pages
            _p, _c_int, _c_int, _p, _c_int,    # page_table, stride, num_pages, nblocks, max_nblocks
            _p, _p,                            # diag_idx, diag_kv
            _c_int, _c_int, _c_int, _c_int, _c_int, _c_f,  # B, H, W, bits, top_k, scale
            _p, _p, _p, _p, _p, _c_int, _p,    # levels, out, sel_out, workspace, err, pdl, stream
        ],
    ),
    "aether_hca_decode_paged_levels": (
        _c_int,
        [_p, _p, _p, _p, _p, _p, _c_int, _c_int, _p, _c_int, _p,  # q .. diag_kv
         _c_int, _c_int, _c_int, _c_int, _c_f, _p, _p, _p, _c_int, _p],  # B, H, W, bits, scale, levels, out, err, pdl, stream
    ),
    "aether_csa_decode_smem_bytes": (_c_int, [_c_int]),
    "aether_csa_decode_workspace_bytes": (ctypes.c_size_t, [_c_int, _c_int]),
    "aether_csa_decode_set_debug_timer": (None, [_p]),
    "aether_csa_local_candidates": (
        _c_int,
        [_p, _p, _p, _p, _c_int, _c_int, _p, _c_int, _p, _c_int, _c_int, _c_int, _c_int, _p, _p, _p, _p, _p],
    ),
    "aether_csa_attend_candidates": (
        _c_int,
        [_p, _p, _p, _p, _p, _p, _c_int, _c_int, _p, _c_int, _p, _p, _p, _c_int, _c_int, _c_int,
         _c_int, _c_int, _c_int, _c_int, _c_int, _c_f, _p, _p, _p, _p, _p, _p],
    ),
    "aether_lse_merge": (_c_int, [_p, _p, _p, _c_int, _c_int, _c_int, _p, _p]),
    "aether_cp_control_bytes": (_c_ll, []),
    "aether_cp_buffer_create": (_c_int, [_c_ll, ctypes.POINTER(_p), _p]),
    "aether_cp_buffer_open": (_c_int, [_p, ctypes.POINTER(_p)]),
    "aether_cp_buffer_close": (_c_int, [_p]),
    "aether_cp_buffer_destroy": (_c_int, [_p]),
    "aether_peer_push": (
        _c_int,
        [_p, _c_ll, _c_ll, _c_ll,            # src, rows, row_bytes, src_stride
         _p, _c_int, _c_int,                 # bases[G], G, rank
         _c_ll, _c_ll, _c_ll, _c_int, _c_int, _p],  # dst_offset, dst_stride, dst_col, kind, bump, stream
    ),
    "aether_peer_wait": (_c_int, [_p, _c_int, _c_int, _p, _p]),
    "aether_lse_merge_strided": (_c_int, [_p, _p, _c_ll, _c_ll, _p, _c_int, _c_int, _c_int, _p, _p]),
    "aether_csa_prefill_attend": (
        _c_int,
        [_p, _p, _p, _p, _p, _p,             # q, sink, window, win_row, window_len, kv_pages
         _p, _c_int, _c_int, _p, _p, _c_int,  # page_table, stride, num_pages, q_row, nblocks, max_nblocks
         _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_f,  # diag, keys, ids, stride, B, H, bits, top_k, scale
         _p, _p, _p, _p],                    # out, sel_out, err, stream
    ),
    "aether_csa_prefill_topk": (
        _c_int,
        [_p, _p, _p, _p, _c_int, _c_int,     # index_q, index_w, idx_pages, page_table, stride, num_pages
         _p, _p, _c_int, _c_int, _p, _c_int, _c_int,  # req_info, tiles, ntiles, compression, diag, bits, top_k
         _p, _p, _p, _p],                    # cand_keys, cand_ids, err, stream
    ),
    "aether_csa_prefill_topk_fp8": (
        _c_int,
        [_p, _p, _p, _p, _c_int, _c_int,
         _p, _p, _c_int, _c_int, _p, _c_int, _c_int,
         _p, _p, _p, _p],
    ),
    "aether_csa_decode_paged_rope": (
        _c_int,
        [_p, _p, _p, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _p, _c_int, _p, _p,
         _c_int, _c_int, _c_int, _c_int, _c_int, _c_f, _p, _p, _p, _p, _c_int, _p, _p, _c_int, _p],
    ),
    "aether_csa_decode_paged_host": (
        _c_int,
        [_p, _p, ctypes.c_size_t, _p, _p, ctypes.c_size_t,  # host_in, dev_in, in_bytes, host_out, dev_out, out_bytes
         _p, _p, _p, _p, _p, _p,                              # q, index_q, index_w, sink, window, window_len
         _p, _p, _p, _c_int, _c_int, _p, _c_int,             # idx_pages, kv_pages, page_table, stride, num_pages, nblocks, max_nb
         _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int, _c_f,  # diag_idx, diag_kv, B, H, W, bits, top_k, scale
         _p, _p, _p, _p, _c_int, _p,                          # out, sel_out, workspace, err, pdl, stream
         _p, _p, _p, _p, _p,                                  # h2d_stream, d2h_stream, ev_h2d, ev_comp, ev_d2h
         _p, ctypes.c_uint32],                                # slot_flags, seq
    ),
    "aether_csa_decode_host_plan_create": (
        _c_int,
        [_p, _p, ctypes.c_size_t, _p, _p, _p, ctypes.c_size_t, _p,  # dev_in0/1, in_bytes, in_offsets, dev_out0/1, ...
         _p, _p, _p, _c_int, _c_int, _c_int, _p, _p,              # slot_flags, idx/kv pages, stride, num_pages, max_nb, diags
         _c_int, _c_int, _c_int, _c_int, _c_int, _p, _p, _c_int, _p],  # B, H, W, bits, top_k, workspace, err, pdl, plan_out
    ),
    "aether_csa_decode_host_plan_step": (_c_int, [_p, _p, _p, _p, _c_int, _p, _p, _c_f, _p]),
    "aether_csa_decode_host_plan_fence": (_c_int, [_p, _p, _c_int]),
    "aether_csa_decode_host_plan_destroy": (None, [_p]),
    "aether_hca_decode_paged": (
        _c_int,
        [
            _p, _p, _p, _p,                    # q, sink, window, window_len
            _p,                                # kv_pages
            _p, _c_int, _c_int, _p, _c_int,    # page_table, stride, num_pages, nblocks, max_nblocks
            _p,                                # diag_kv
            _c_int, _c_int, _c_int, _c_int, _c_f,  # B, H, W, bits, scale
            _p, _p, _c_int, _c_int, _p,        # out, err, cluster, pdl, stream
        ],
    ),
}

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None


class AetherKernelError(RuntimeError):
    pass


def library_path() -> Path:
    return LIB_PATH


def load() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise AetherKernelError(
                    f"Aether CUDA kernels are unavailable: {LIB_PATH} is not built "
                    "(run aether_kernels._build.build() or __graft_entry__.build())."
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().aether_last_error()
    return msg.decode() if msg else ""


def call(name: str, *args) -> None:
    """Invoke a C entry point; translate a non-zero status into RuntimeError."""
    rc = getattr(load(), name)(*args)
    if rc != 0:
        raise AetherKernelError(f"{name} failed ({rc}): {last_error()}")
