"""ctypes binding of the flashcart_b200 C ABI (``include/flashcart_b200.h``).

The product path loads ``_lib/libflashcart_b200.so`` (sm_100a kernels) and fails
loudly when it is missing or when CUDA is unavailable: there is no CPU fallback.
``bind(path)`` binds any library exporting the same ABI (the CPU tests bind the
host-emulation build with it).
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib")
CUDA_LIB_PATH = os.path.join(LIB_DIR, "libflashcart_b200.so")

FC_OK = 0
FC_ERR_INVALID = -1
FC_ERR_UNSUPPORTED = -2
FC_ERR_LAUNCH = -3
FC_ERR_CAPACITY = -4
FC_NOALLOC_MAX_NODES = 1 << 18
FC_DEV_BAD_INDEX = 1
FC_DEV_UNSORTED = 2
FC_DEV_TIMEOUT = 4
FC_F32 = 0
FC_F64 = 1
FC_BF16 = 2
FC_ACT_NONE = 0
FC_ACT_SILU = 1
FC_PREC_IEEE = 0
FC_PREC_TF32 = 1
FC_MAX_L = 3

EXPORTED_SYMBOLS = (
    "fc_version", "fc_last_error", "fc_build_rowptr", "fc_tp_num_paths", "fc_tp_out_dim",
    "fc_tp_fwd", "fc_tp_bwd", "fc_tp_dbwd", "fc_irreps_fwd", "fc_irreps_bwd", "fc_irreps_dbwd",
    "fc_linear_fwd", "fc_linear_bwd", "fc_tp_conv_fwd_noalloc", "fc_newton_schulz",
    "fc_rms_norm_fwd", "fc_rms_norm_bwd", "fc_gate_fwd", "fc_gate_bwd",
    "fc_neighbor_workspace_bytes", "fc_neighbor_count", "fc_neighbor_fill",
    "fc_edge_expand_fwd", "fc_edge_expand_bwd",
    "fc_linear_presplit", "fc_linear_fwd_presplit", "fc_linear_bwd_presplit",
    "fc_linear_fwd_residual", "fc_linear_bwd_residual", "fc_tp_bwd_residual",
    "fc_linear_dbwd", "fc_halo_pack", "fc_halo_unpack", "fc_edge_geometry_fwd", "fc_edge_geometry_bwd",
    "fc_edge_geometry_vec_fwd", "fc_edge_geometry_vec_bwd",
)


class TpDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "in1_l_max", "in2_l_max", "out_l_max", "in1_features", "in2_features",
        "symmetric_product", "shared_weights", "reduce_paths", "dtype")]


class EdgeGeometryDesc(ctypes.Structure):
    _fields_ = [("l_max", ctypes.c_int32), ("n_radial", ctypes.c_int32), ("cosine", ctypes.c_int32),
                ("poly_order", ctypes.c_int32), ("use_shifts", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("r_min", ctypes.c_double), ("r_max", ctypes.c_double), ("r_cut", ctypes.c_double)]


class LinearDesc(ctypes.Structure):
    _fields_ = [
        ("n_active", ctypes.c_int32), ("dtype", ctypes.c_int32),
        ("precision", ctypes.c_int32), ("act", ctypes.c_int32),
        ("in_dim", ctypes.c_int64), ("out_dim", ctypes.c_int64),
        ("in_offsets", ctypes.c_int64 * (FC_MAX_L + 1)),
        ("out_offsets", ctypes.c_int64 * (FC_MAX_L + 1)),
        ("m_values", ctypes.c_int32 * (FC_MAX_L + 1)),
        ("f_in_values", ctypes.c_int32 * (FC_MAX_L + 1)),
        ("f_out_values", ctypes.c_int32 * (FC_MAX_L + 1)),
    ]


class NlDesc(ctypes.Structure):
    _fields_ = [("lengths", ctypes.c_double * 3), ("inv_lengths", ctypes.c_double * 3),
                ("bin_widths", ctypes.c_double * 3), ("r_max_sq", ctypes.c_double),
                ("bins", ctypes.c_int32 * 3), ("reserved", ctypes.c_int32)]


class NativeError(RuntimeError):
    pass


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32


def bind(path: str) -> ctypes.CDLL:
    """Load a library exporting the flashcart_b200 ABI and declare its signatures."""
    lib = ctypes.CDLL(path)
    lib.fc_version.restype = ctypes.c_char_p
    lib.fc_version.argtypes = []
    lib.fc_last_error.restype = ctypes.c_char_p
    lib.fc_last_error.argtypes = []
    lib.fc_build_rowptr.restype = ctypes.c_int
    lib.fc_build_rowptr.argtypes = [_P, _I64, _I64, _P, _P, _P]
    lib.fc_tp_num_paths.restype = ctypes.c_int
    lib.fc_tp_num_paths.argtypes = [ctypes.POINTER(TpDesc)]
    lib.fc_tp_out_dim.restype = ctypes.c_int64
    lib.fc_tp_out_dim.argtypes = [ctypes.POINTER(TpDesc)]
    lib.fc_tp_fwd.restype = ctypes.c_int
    lib.fc_tp_fwd.argtypes = [ctypes.POINTER(TpDesc), _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P]
    lib.fc_tp_bwd.restype = ctypes.c_int
    lib.fc_tp_bwd.argtypes = [ctypes.POINTER(TpDesc), _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P]
    lib.fc_tp_dbwd.restype = ctypes.c_int
    lib.fc_tp_dbwd.argtypes = [ctypes.POINTER(TpDesc), _P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64,
                               _P, _P, _P, _P, _P, _P]
    lib.fc_irreps_fwd.restype = ctypes.c_int
    lib.fc_irreps_fwd.argtypes = [_P, _I64, _I32, _I32, _P, _P]
    lib.fc_irreps_bwd.restype = ctypes.c_int
    lib.fc_irreps_bwd.argtypes = [_P, _P, _I64, _I32, _I32, _P, _P]
    lib.fc_irreps_dbwd.restype = ctypes.c_int
    lib.fc_irreps_dbwd.argtypes = [_P, _P, _P, _I64, _I32, _I32, _P, _P, _P]
    lib.fc_linear_fwd.restype = ctypes.c_int
    lib.fc_linear_fwd.argtypes = [ctypes.POINTER(LinearDesc), _P, _P, _P, _I64, _P, _P, _P]
    lib.fc_tp_conv_fwd_noalloc.restype = ctypes.c_int
    lib.fc_tp_conv_fwd_noalloc.argtypes = [ctypes.POINTER(TpDesc), _P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _P,
                                            _P]
    lib.fc_linear_bwd.restype = ctypes.c_int
    lib.fc_linear_bwd.argtypes = [ctypes.POINTER(LinearDesc), _P, _P, _P, _P, _I64, _P, _P, _P, _P]
    lib.fc_linear_dbwd.restype = ctypes.c_int
    lib.fc_linear_dbwd.argtypes = [ctypes.POINTER(LinearDesc), _P, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _P, _P]
    lib.fc_halo_pack.restype = ctypes.c_int
    lib.fc_halo_pack.argtypes = [_P, _I64, _I64, _I32, _P, _I64, _P, _P, _P]
    lib.fc_halo_unpack.restype = ctypes.c_int
    lib.fc_halo_unpack.argtypes = [_P, _I64, _I64, _I32, _P, _P, _I64, _I32, _P, _P]
    lib.fc_newton_schulz.restype = ctypes.c_int
    lib.fc_newton_schulz.argtypes = [_P, _I32, _I64, _I32, _I32, _P, _I32, _P, _I32, ctypes.c_float, _P, _P, _P]
    lib.fc_rms_norm_fwd.restype = ctypes.c_int
    lib.fc_rms_norm_fwd.argtypes = [_I32, _I32, _I32, _P, _P, _P, ctypes.c_double, _I64, _P, _P, _P]
    lib.fc_rms_norm_bwd.restype = ctypes.c_int
    lib.fc_rms_norm_bwd.argtypes = [_I32, _I32, _I32, _P, _P, _P, _P, _P, _I64, _P, _P]
    lib.fc_neighbor_workspace_bytes.restype = ctypes.c_int64
    lib.fc_neighbor_workspace_bytes.argtypes = [ctypes.POINTER(NlDesc), _I64]
    lib.fc_neighbor_count.restype = ctypes.c_int
    lib.fc_neighbor_count.argtypes = [ctypes.POINTER(NlDesc), _P, _I64, _P, _P, _P, _P]
    lib.fc_neighbor_fill.restype = ctypes.c_int
    lib.fc_neighbor_fill.argtypes = [ctypes.POINTER(NlDesc), _I64, _P, _P, _I64, _P, _P, _P, _P]
    lib.fc_linear_presplit.restype = ctypes.c_int
    lib.fc_linear_presplit.argtypes = [ctypes.POINTER(LinearDesc), _P, _I32, _P, _P]
    lib.fc_linear_fwd_presplit.restype = ctypes.c_int
    lib.fc_linear_fwd_presplit.argtypes = [ctypes.POINTER(LinearDesc), _P, _P, _P, _P, _I64, _P, _P, _P]
    lib.fc_linear_bwd_presplit.restype = ctypes.c_int
    lib.fc_linear_bwd_presplit.argtypes = [ctypes.POINTER(LinearDesc), _P, _P, _P, _P, _P, _I64, _P, _P, _P, _P]
    lib.fc_tp_bwd_residual.restype = ctypes.c_int
    lib.fc_tp_bwd_residual.argtypes = [ctypes.POINTER(TpDesc), _P, _P, _P, _P, _I64, _P, _I64, ctypes.c_int32, _P,
                                       _P, _P, _P, _P]
    for name in ("fc_linear_fwd_residual", "fc_linear_bwd_residual"):
        getattr(lib, name).restype = ctypes.c_int
        getattr(lib, name).argtypes = [ctypes.POINTER(LinearDesc), _P, _P, _P, _P, _I64, _P, _P, _P, _P]
    lib.fc_edge_expand_fwd.restype = ctypes.c_int
    lib.fc_edge_expand_fwd.argtypes = [_I32, _I32, _I32, _I32, _P, _P, _I64, _P, _P]
    lib.fc_edge_expand_bwd.restype = ctypes.c_int
    lib.fc_edge_expand_bwd.argtypes = [_I32, _I32, _I32, _I32, _P, _P, _P, _I64, _P, _P, _P]
    lib.fc_edge_geometry_fwd.restype = ctypes.c_int
    lib.fc_edge_geometry_fwd.argtypes = [ctypes.POINTER(EdgeGeometryDesc), _P, _I64, _P, _I64, _P, _P, _P, _I64, _P,
                                         _P, _P, _P]
    lib.fc_edge_geometry_bwd.restype = ctypes.c_int
    lib.fc_edge_geometry_bwd.argtypes = [ctypes.POINTER(EdgeGeometryDesc), _P, _I64, _P, _I64, _P, _P, _P, _I64, _P,
                                         _P, _P, _P, _P, _P]
    lib.fc_edge_geometry_vec_fwd.restype = ctypes.c_int
    lib.fc_edge_geometry_vec_fwd.argtypes = [ctypes.POINTER(EdgeGeometryDesc), _P, _I64, _P, _P, _P, _P]
    lib.fc_edge_geometry_vec_bwd.restype = ctypes.c_int
    lib.fc_edge_geometry_vec_bwd.argtypes = [ctypes.POINTER(EdgeGeometryDesc), _P, _I64, _P, _P, _P, _P, _P]
    lib.fc_gate_fwd.restype = ctypes.c_int
    lib.fc_gate_fwd.argtypes = [_I32, _I32, _I32, _P, _P, _I64, _P, _P]
    lib.fc_gate_bwd.restype = ctypes.c_int
    lib.fc_gate_bwd.argtypes = [_I32, _I32, _I32, _P, _P, _P, _I64, _P, _P, _P]
    return lib


def check(lib: ctypes.CDLL, rc: int, what: str) -> None:
    """Map a C status to the reference's exception types."""
    if rc == FC_OK:
        return
    msg = lib.fc_last_error().decode(errors="replace") or f"{what} failed ({rc})"
    if rc == FC_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if rc == FC_ERR_INVALID:
        raise ValueError(msg)
    raise NativeError(msg)


_LIB: Optional[ctypes.CDLL] = None
_LOCK = threading.Lock()


def lib() -> ctypes.CDLL:
    """The sm_100a library; raises if it was not built or CUDA is unavailable."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not os.path.exists(CUDA_LIB_PATH):
                raise NativeError(
                    f"flashcart_b200 CUDA library not found at {CUDA_LIB_PATH}; run "
                    "`python -m flashcart_b200.build_ext` (there is no CPU fallback)")
            _LIB = bind(CUDA_LIB_PATH)
    return _LIB
