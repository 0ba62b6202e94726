"""ctypes binding of libfastembedr_b200.so (the C ABI in include/fastembedr_b200.h).

The shared library is built in-tree by ``fastembedr_b200.build_lib``.  There is
no fallback: if the library is missing or no B200 is visible, calls raise.
"""
from __future__ import annotations

import ctypes
import os
import re
from typing import List

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libfastembedr_b200.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "fastembedr_b200.h")

c_int_p = ctypes.POINTER(ctypes.c_int)
c_float_p = ctypes.POINTER(ctypes.c_float)
c_double_p = ctypes.POINTER(ctypes.c_double)
c_ll_p = ctypes.POINTER(ctypes.c_longlong)
c_void_p = ctypes.c_void_p
I, F, D, U, LL = ctypes.c_int, ctypes.c_float, ctypes.c_double, ctypes.c_uint, ctypes.c_longlong

_TSNE_KNN_ARGS = [c_void_p, c_void_p, c_float_p, I, I, I, I, F, I, I, F, F, F, I, F, F, F, F, U, I, c_float_p]

_SIGNATURES = {
    "fastembedr_cuda_available": (ctypes.c_bool, []),
    "fastembedr_cuda_embedding_last_error": (ctypes.c_char_p, []),
    "fe_b200_version": (ctypes.c_char_p, []),
    "fe_b200_release_memory": (I, []),
    "fastembedr_cuda_opentsne_fft_from_knn": (I, _TSNE_KNN_ARGS),
    "fastembedr_cuda_opentsne_fft_from_knn_float": (I, _TSNE_KNN_ARGS),
    "fastembedr_cuda_opentsne_fft_from_device_knn_float": (I, _TSNE_KNN_ARGS),
    "fastembedr_cuda_landmark_tsne_from_device_knn": (I, [c_void_p, c_void_p, I, c_float_p, c_float_p, c_float_p,
                                                          I, I, I, I, F, I, I, F, F, F, F, F, F, F, I, I, U, I,
                                                          F, F, c_float_p]),
    "fastembedr_cuda_umap_optimize_coo": (I, [c_int_p, c_int_p, c_float_p, c_float_p, c_float_p, I, I, I, I,
                                              F, F, F, F, U, I, c_float_p]),
    "fastembedr_cuda_umap_from_knn_spectral": (I, [c_void_p, c_void_p, I, I, I, I, F, F, F, F, I, U, I, I,
                                                   c_float_p]),
    "fastembedr_cuda_umap_from_knn_spectral_float": (I, [c_void_p, c_void_p, I, I, I, I, F, F, F, F, I, U, I, I,
                                                         c_float_p]),
    "fastembedr_cuda_umap_from_device_knn_spectral_float": (I, [c_void_p, c_void_p, I, I, I, I, F, F, F, F, I, U,
                                                                I, I, I, c_float_p]),
    "fastembedr_cuda_umap_graph_dump_from_knn": (I, [c_void_p, c_void_p, I, I, I, c_int_p, c_int_p, c_float_p,
                                                     c_float_p, c_int_p, c_int_p]),
    "fe_b200_umap_epochs": (I, [c_int_p, c_int_p, c_float_p, LL, c_float_p, I, I, I, I, I, F, F, F, F, U, I, I,
                                c_ll_p]),
    "fe_b200_umap_epochs_noalloc": (I, [c_void_p, c_void_p, c_void_p, LL, c_void_p, I, I, I, I, I, F, F, F, F,
                                        U, I, c_void_p]),
    "fe_b200_tsne_create": (I, [c_void_p, c_void_p, I, I, I, F, c_float_p, U, I, I, ctypes.POINTER(c_void_p)]),
    "fe_b200_tsne_create_csr": (I, [c_int_p, c_int_p, c_float_p, I, c_float_p, I, ctypes.POINTER(c_void_p)]),
    "fe_b200_tsne_iterate": (I, [c_void_p, I, F, F, F, F, F]),
    "fe_b200_tsne_prepare": (I, [c_void_p, F, F, F, F, F]),
    "fe_b200_tsne_gradient": (I, [c_void_p, F, c_float_p, c_double_p]),
    "fe_b200_tsne_get_layout": (I, [c_void_p, c_void_p, I]),
    "fe_b200_tsne_set_layout": (I, [c_void_p, c_void_p, I, I]),
    "fe_b200_tsne_get_state": (I, [c_void_p, c_float_p, c_float_p]),
    "fe_b200_tsne_set_state": (I, [c_void_p, c_float_p, c_float_p]),
    "fe_b200_tsne_info": (I, [c_void_p, c_int_p, c_int_p, c_ll_p, c_ll_p]),
    "fe_b200_tsne_staged_blocks": (I, [c_void_p, c_int_p, c_int_p]),
    "fe_b200_pca_start": (I, [c_void_p, I, I, I, c_float_p]),
    "fe_b200_tsne_set_interpolation": (I, [c_void_p, I]),
    "fe_b200_knn_exact": (I, [c_void_p, I, I, I, I, I, I, c_void_p, c_void_p]),
    "fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_double": (I, [c_void_p, c_void_p, c_void_p, I, I, I,
                                                                         I, F, I, I, F, F, F, I, F, F, F, F, U, I,
                                                                         c_float_p]),
    "fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_float": (I, [c_void_p, c_void_p, c_void_p, I, I, I,
                                                                        I, F, I, I, F, F, F, I, F, F, F, F, U, I,
                                                                        c_float_p]),
    "fe_b200_tsne_get_p": (I, [c_void_p, c_int_p, c_int_p, c_float_p]),
    "fe_b200_tsne_stream": (c_void_p, [c_void_p]),
    "fe_b200_tsne_profile": (I, [c_void_p, I]),
    "fe_b200_tsne_kernel_times": (I, [c_void_p, c_double_p, c_ll_p, I]),
    "fe_b200_tsne_kernel_name": (ctypes.c_char_p, [I]),
    "fe_b200_tsne_destroy": (None, [c_void_p]),
    "fe_b200_nccl_unique_id": (I, [c_void_p, I]),
    "fe_b200_umap_create": (I, [c_void_p, c_void_p, I, I, I, I, I, I, U, ctypes.POINTER(c_void_p)]),
    "fe_b200_umap_run": (I, [c_void_p, I, I, I, I, F, F, F, F, U, I]),
    "fe_b200_umap_count_samples": (I, [c_void_p, I, I, I, c_ll_p, c_ll_p]),
    "fe_b200_umap_get_layout": (I, [c_void_p, c_void_p, I]),
    "fe_b200_umap_set_layout": (I, [c_void_p, c_void_p, I]),
    "fe_b200_umap_info": (I, [c_void_p, c_int_p, c_ll_p]),
    "fe_b200_umap_get_graph": (I, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "fe_b200_umap_stream": (c_void_p, [c_void_p]),
    "fe_b200_umap_destroy": (None, [c_void_p]),
    "fe_b200_umap_shard": (I, [c_void_p, c_void_p, I, I, I]),
    "fe_b200_umap_shard_comm": (I, [c_void_p, c_void_p]),
    "fe_b200_comm_create": (I, [c_void_p, I, I, I, ctypes.POINTER(c_void_p)]),
    "fe_b200_comm_destroy": (None, [c_void_p]),
    "fe_b200_tsne_shard_comm": (I, [c_void_p, c_void_p]),
    "fe_b200_tsne_shard": (I, [c_void_p, c_void_p, I, I, I]),
}

_lib = None


class CudaBackendError(RuntimeError):
    """A C-ABI call returned status 1."""


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing; build it with `python -m fastembedr_b200.build_lib`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return load().fastembedr_cuda_embedding_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise CudaBackendError(f"{what} failed: {last_error()}")


def header_functions() -> List[str]:
    """Every function the public header declares (for export checks)."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(", text)
    keep = [n for n in names if n.startswith(("fastembedr_cuda_", "fe_b200_"))]
    return sorted(set(keep))
