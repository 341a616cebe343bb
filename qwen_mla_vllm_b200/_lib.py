"""ctypes binding of libqmla.so (the C ABI declared in include/qmla.h).

The shared library is built in-tree (``qwen_mla_vllm_b200/libqmla.so``, see
``build.py``).  Loading fails loudly: there is no CPU or Python fallback for
any entry point.
"""
from __future__ import annotations

import ctypes
import os
import pathlib

_HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = _HERE / "libqmla.so"

# element types / rms modes (include/qmla.h)
DT_BF16, DT_F16, DT_F32, DT_FP8E4M3 = 0, 1, 2, 3
RMS_NONE, RMS_NATIVE, RMS_BF16, RMS_LOG8 = 0, 1, 2, 3

OK = 0
ERRORS = {
    -1: "invalid argument",
    -2: "unsupported shape or dtype",
    -3: "pointer or stride not 16-byte aligned",
    -4: "workspace too small",
    -5: "CUDA call failed",
    -6: "device wait timed out",
}


class QmlaError(RuntimeError):
    """A libqmla entry point returned a negative status."""

    def __init__(self, fn: str, code: int):
        super().__init__(f"{fn} failed: {ERRORS.get(code, 'unknown error')} ({code})")
        self.code = code


class DecodeParams(ctypes.Structure):
    """Mirror of ``qmla_decode_params`` (field order and types must match qmla.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("q_stride_row", ctypes.c_int64),
        ("q_stride_head", ctypes.c_int64),
        ("q_pe", ctypes.c_void_p),
        ("qpe_stride_row", ctypes.c_int64),
        ("qpe_stride_head", ctypes.c_int64),
        ("q_dtype", ctypes.c_int32),
        ("kv_cache", ctypes.c_void_p),
        ("kv_stride_page", ctypes.c_int64),
        ("kv_stride_token", ctypes.c_int64),
        ("kv_num_pages", ctypes.c_int64),
        ("kv_row_width", ctypes.c_int32),
        ("kv_dtype", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("block_table", ctypes.c_void_p),
        ("block_table_stride", ctypes.c_int64),
        ("seq_lens", ctypes.c_void_p),
        ("num_rows", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("qk_dim", ctypes.c_int32),
        ("rms_offset", ctypes.c_int32),
        ("rms_mode", ctypes.c_int32),
        ("sm_scale", ctypes.c_float),
        ("logit_cap", ctypes.c_float),
        ("k_scale", ctypes.c_void_p),
        ("qrows", ctypes.c_int32),
        ("o", ctypes.c_void_p),
        ("o_stride_row", ctypes.c_int64),
        ("o_stride_head", ctypes.c_int64),
        ("o_dtype", ctypes.c_int32),
        ("lse", ctypes.c_void_p),
        ("lse_stride_row", ctypes.c_int64),
        ("lse_dtype", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
        ("plan_tile_prefix", ctypes.c_void_p),
        ("num_ctas", ctypes.c_int32),
        ("device", ctypes.c_int32),
    ]


DCP_MAX_WORLD = 8
DCP_ALL_HEADS, DCP_HEAD_SCATTER = 0, 1
IPC_HANDLE_BYTES = 64


class DcpP2PParams(ctypes.Structure):
    """Mirror of ``qmla_dcp_p2p_params`` (field order and types must match qmla.h)."""

    _fields_ = [
        ("bufs", ctypes.c_void_p * DCP_MAX_WORLD),
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("num_rows", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("mode", ctypes.c_int32),
        ("epoch", ctypes.c_uint32),
        ("out", ctypes.c_void_p),
        ("out_stride_row", ctypes.c_int64),
        ("out_stride_head", ctypes.c_int64),
        ("out_dtype", ctypes.c_int32),
        ("lse_out", ctypes.c_void_p),
        ("timeout_ns", ctypes.c_int64),
        ("device", ctypes.c_int32),
    ]


class GatherParams(ctypes.Structure):
    """Mirror of ``qmla_gather_params`` (field order and types must match qmla.h)."""

    _fields_ = [
        ("src_cache", ctypes.c_void_p),
        ("src_stride_page", ctypes.c_int64),
        ("src_stride_token", ctypes.c_int64),
        ("page_size", ctypes.c_int32),
        ("num_pages", ctypes.c_int32),
        ("src_dtype", ctypes.c_int32),
        ("row_elems", ctypes.c_int32),
        ("rms_offset", ctypes.c_int32),
        ("rms_heads", ctypes.c_int32),
        ("rms_mode", ctypes.c_int32),
        ("scale", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("block_table_stride", ctypes.c_int64),
        ("block_table_cols", ctypes.c_int32),
        ("cu_seq_lens", ctypes.c_void_p),
        ("token_to_seq", ctypes.c_void_p),
        ("seq_starts", ctypes.c_void_p),
        ("num_seqs", ctypes.c_int32),
        ("num_tokens", ctypes.c_int32),
        ("dst", ctypes.c_void_p),
        ("dst_stride_row", ctypes.c_int64),
        ("dst_dtype", ctypes.c_int32),
        ("status", ctypes.c_void_p),
        ("device", ctypes.c_int32),
    ]


# device status bits (qmla_read_status / the gather's status word)
DEV_ERR_TIMEOUT, DEV_ERR_INDEX = 1, 2

# exported symbols and their ctypes prototypes: (restype, argtypes)
_VP, _I32, _I64, _F32P = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p
PROTOTYPES = {
    "qmla_abi_version": (ctypes.c_int, []),
    "qmla_error_string": (ctypes.c_char_p, [ctypes.c_int]),
    "qmla_decode_workspace_bytes": (ctypes.c_int, [ctypes.POINTER(DecodeParams), ctypes.POINTER(_I64)]),
    "qmla_mla_decode": (ctypes.c_int, [ctypes.POINTER(DecodeParams), _VP]),
    "qmla_mla_decode_static": (ctypes.c_int, [ctypes.POINTER(DecodeParams), _VP]),
    "qmla_read_status": (ctypes.c_int, [_VP, _VP, ctypes.POINTER(_I32)]),
    "qmla_static_read_status": (ctypes.c_int, [_I32, _VP, ctypes.POINTER(_I32)]),
    "qmla_plan": (ctypes.c_int, [_VP, _I32, _I32, _VP, _VP, _VP, ctypes.POINTER(_I64), ctypes.POINTER(_I64)]),
    "qmla_dcp_correct": (ctypes.c_int, [_VP, _I32, _I64, _I64, _VP, _I64, _I64, _VP, _I32, _I32, _I32,
                                        _I32, _I32, _I32, _VP]),
    "qmla_dcp_merge": (ctypes.c_int, [_VP, _I32, _VP, _VP, _I32, _VP, _I32, _I32, _I32, _I32, _VP]),
    "qmla_fp8_cache_write": (ctypes.c_int, [_VP, _I64, _VP, _I64, _VP, _I32, _I32, _I32, _I32, _I32, _VP,
                                            _VP, _I64, _VP]),
    "qmla_dcp_buffer_layout": (ctypes.c_int, [_I32, _I32, _I32] + [ctypes.POINTER(_I64)] * 5),
    "qmla_dcp_buffer_alloc": (ctypes.c_int, [_I32, _I64, ctypes.POINTER(_VP), _VP]),
    "qmla_dcp_buffer_open": (ctypes.c_int, [_I32, _VP, ctypes.POINTER(_VP)]),
    "qmla_dcp_buffer_close": (ctypes.c_int, [_VP]),
    "qmla_dcp_buffer_free": (ctypes.c_int, [_VP]),
    "qmla_dcp_p2p_merge": (ctypes.c_int, [ctypes.POINTER(DcpP2PParams), _VP]),
    "qmla_dcp_read_status": (ctypes.c_int, [_VP, _VP, ctypes.POINTER(_I32)]),
    "qmla_gather_cache": (ctypes.c_int, [ctypes.POINTER(GatherParams), _VP]),
}

_lib = None


def load(path: os.PathLike | str | None = None) -> ctypes.CDLL:
    """Load libqmla.so once and attach prototypes.  Raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    if path is None and os.environ.get("QMLA_LIB_PATH"):
        path = os.environ["QMLA_LIB_PATH"]  # an alternate build of the same ABI
        if _lib is not None:
            return _lib
    p = pathlib.Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise ImportError(f"libqmla.so not found at {p}: build it with "
                          f"`python -c 'import __graft_entry__ as g; g.build()'` or "
                          f"`python -m qwen_mla_vllm_b200.build`")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None or os.environ.get("QMLA_LIB_PATH") == str(path):
        _lib = lib
    return lib


def check(fn: str, code: int) -> None:
    if code != OK:
        raise QmlaError(fn, code)
