"""ctypes binding of ``libdcckv.so`` (the C ABI declared in include/dcc_kv.h).

The shared library is built in-tree (``dcc_kv_b200/libdcckv.so``) by
``dcc_kv_b200/build.py``.  Loading it never touches a GPU, so the symbol
table can be checked on a CPU-only machine; every compute entry point needs
CUDA tensors and fails loudly when given anything else.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libdcckv.so")

DCC_OK = 0
DCC_ERR_INVALID_ARGUMENT = 1
DCC_ERR_SHAPE = 2
DCC_ERR_DTYPE = 3
DCC_ERR_WORKSPACE = 4
DCC_ERR_CUDA = 5
DCC_ERR_UNSUPPORTED = 6
DCC_ERR_TIMEOUT = 7

DCC_F32 = 0
DCC_BF16 = 1
DCC_F64 = 2

MAX_SEGMENTS = 16

_DTYPES = {torch.float32: DCC_F32, torch.bfloat16: DCC_BF16, torch.float64: DCC_F64}


class DccError(RuntimeError):
    """A CUDA-side failure reported by the library (status code in ``.status``)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class dcc_query_set(C.Structure):
    _fields_ = [("queries", C.c_void_p), ("seg_rows", C.c_int64), ("seg_stride", C.c_int64),
                ("row_stride", C.c_int64), ("n_seg", C.c_int32), ("reserved", C.c_int32),
                ("out_repr", C.c_void_p), ("out_idx", C.c_void_p)]


class dcc_build_problem(C.Structure):
    _fields_ = [("keys", C.c_void_p), ("values", C.c_void_p), ("repr", C.c_void_p),
                ("L_s", C.c_int64), ("ld_k", C.c_int64), ("ld_v", C.c_int64),
                ("budget", C.c_int32), ("num_repr", C.c_int32),
                ("out_keys", C.c_void_p), ("out_values", C.c_void_p), ("out_bias", C.c_void_p),
                ("out_idx", C.c_void_p), ("out_mass", C.c_void_p)]


class dcc_kv_segment(C.Structure):
    _fields_ = [("k", C.c_void_p), ("v", C.c_void_p), ("bias", C.c_void_p),
                ("k_head_stride", C.c_int64), ("v_head_stride", C.c_int64),
                ("row_stride", C.c_int64), ("bias_head_stride", C.c_int64), ("len", C.c_int64)]


class dcc_attn_problem(C.Structure):
    _fields_ = [("q", C.c_void_p), ("q_head_stride", C.c_int64), ("q_row_stride", C.c_int64),
                ("o", C.c_void_p), ("o_head_stride", C.c_int64), ("o_row_stride", C.c_int64),
                ("lse", C.c_void_p), ("lse_head_stride", C.c_int64), ("Lq", C.c_int64),
                ("n_seg", C.c_int32), ("causal", C.c_int32), ("causal_offset", C.c_int64),
                ("seg", dcc_kv_segment * MAX_SEGMENTS),
                ("o_init", C.c_void_p), ("lse_init", C.c_void_p), ("lse_init_head_stride", C.c_int64)]


_P = C.c_void_p
_I = C.c_int
_I64 = C.c_int64
_D = C.c_double
_SZ = C.c_size_t

# name -> (restype, argtypes); every name here is declared in include/dcc_kv.h
SIGNATURES = {
    "dcc_status_string": (C.c_char_p, [_I]),
    "dcc_last_error": (C.c_char_p, []),
    "dcc_version": (_I, []),
    "dcc_struct_size": (_SZ, [C.c_char_p]),
    "dcc_rademacher_projection": (_I, [_I, _I, C.c_uint64, _P]),
    "dcc_fps_start_index": (_I64, [_I64, C.c_uint64]),
    "dcc_select_representative_queries_workspace_bytes": (_SZ, [_P, _I, _I, _I]),
    "dcc_select_representative_queries": (_I, [_P, _I, _I, _I, _I, C.c_uint64, _I, _P, _SZ, _P]),
    "dcc_build_compact_kv_workspace_bytes": (_SZ, [_P, _I, _I, _I, _I]),
    "dcc_build_compact_kv_batched": (_I, [_P, _I, _I, _I, _D, _D, _I, _P, _SZ, _P]),
    "dcc_build_compact_kv_workspace": (_SZ, [_I64, _I64, _I, _I, _I, _I, _I, _I]),
    "dcc_build_compact_kv": (_I, [_P, _P, _P, _I64, _I64, _I, _I, _I, _I, _I, _D, _D, C.c_uint64, _I,
                                  _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "dcc_build_compact_kv_noalloc": (_I, [_P, _P, _P, _I64, _I64, _I, _I, _I, _I, _I, _D, _D, C.c_uint64, _I,
                                          _P, _P, _P, _P, _P, _P]),
    "dcc_stage_workspace_bytes": (_SZ, [_I64, _I, _I, _I, _I, _I]),
    "dcc_select_topk_keys": (_I, [_P, _P, _I64, _I, _I, _I, _I, _P, _P, _P, _SZ, _P]),
    "dcc_fit_logit_bias": (_I, [_P, _P, _P, _I, _I, _I, _D, _I, _P, _P, _SZ, _P]),
    "dcc_fit_compact_value": (_I, [_P, _P, _P, _P, _P, _I64, _I, _I, _I, _I, _D, _I, _P, _P, _SZ, _P]),
    "dcc_farthest_point_sampling_workspace_bytes": (_SZ, [_I64, _I]),
    "dcc_farthest_point_sampling": (_I, [_P, _I64, _I, _I, C.c_uint64, _I, _P, _P, _SZ, _P]),
    "dcc_rms_per_token_score": (_I, [_P, _I64, _I64, _I, _P, _P]),
    "dcc_nnls_workspace_bytes": (_SZ, [_I64, _I64]),
    "dcc_nonneg_least_squares": (_I, [_P, _P, _I64, _I64, _D, _I, _I, _P, _P, _SZ, _P]),
    "dcc_ridge_workspace_bytes": (_SZ, [_I64, _I64, _I64]),
    "dcc_ridge_regression_value": (_I, [_P, _P, _I64, _I64, _I64, _D, _I, _P, _P, _SZ, _P]),
    "dcc_attention_fwd": (_I, [_P, _I, _I, _I, _I, _D, _I, _P]),
    "dcc_device_error_status": (_I, [_I]),
    "dcc_build_error_status": (_I, [_I]),
    "dcc_device_error_flags_async": (_I, [_P, _P]),
    "dcc_debug_expire_wait": (_I, [C.c_uint64, _P]),
    "dcc_online_softmax_from_attention": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I, _P, _P, _P, _P]),
    "dcc_merge_softmax_states": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I, _P, _P, _P, _P]),
    "dcc_merge_lse": (_I, [_P, _P, _I, _I64, _I64, _I, _P, _P, _P]),
}

_lib: Optional[C.CDLL] = None


def lib() -> C.CDLL:
    """Load the library once; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m dcc_kv_b200.build` "
                              "(nvcc, sm_100a) before using the CUDA path")
        handle = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    """Map a status code to the exception type the reference raises."""
    if status == DCC_OK:
        return
    msg = f"{what}: {lib().dcc_last_error().decode(errors='replace')}"
    if status in (DCC_ERR_INVALID_ARGUMENT, DCC_ERR_UNSUPPORTED, DCC_ERR_DTYPE, DCC_ERR_WORKSPACE):
        raise ValueError(msg)
    if status == DCC_ERR_SHAPE:
        raise AssertionError(msg)
    raise DccError(status, msg)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; use float32, float64 or bfloat16") from None


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("dcc_kv_b200 runs on CUDA tensors only (no CPU fallback); "
                             f"got a tensor on {t.device}")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """A caller-owned scratch buffer (the library itself never allocates)."""
    return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)


class DeviceErrorWatch:
    """Bounded device-side waits that gave up, seen from the host without a
    synchronisation.  The tcgen05 kernels never hang: a wait that passes its
    limit records a flag and the kernel unwinds, leaving its outputs
    unusable.  ``record`` enqueues one tiny kernel that writes the library's
    two flags (attention, scoring) into a pinned host pair at the end of a
    forward; ``poll`` raises ``DccError(DCC_ERR_TIMEOUT)`` when the pair, as
    last written, shows a flag, so a forward whose kernel gave up is reported
    by the next call.  ``check`` synchronises the device first.  The flags
    belong to the device: a wait that gave up in any of the library's
    kernels on it is reported, whichever layer launched it."""

    def __init__(self):
        self.host: Optional[torch.Tensor] = None

    def record(self, stream: torch.cuda.Stream) -> None:
        if self.host is None:
            self.host = torch.zeros(2, dtype=torch.int32).pin_memory()
        check(lib().dcc_device_error_flags_async(self.host.data_ptr(), stream.cuda_stream),
              "device_error_flags_async")

    def poll(self) -> None:
        if self.host is None:
            return
        a, s = (int(x) for x in self.host.tolist())
        if a or s:
            self.host.zero_()
            # clears the device words (this synchronises; only on the error path)
            lib().dcc_device_error_status(1)
            lib().dcc_build_error_status(1)
            raise DccError(DCC_ERR_TIMEOUT,
                           f"a bounded device wait expired in an earlier forward (attention flags {a}, "
                           f"scoring flags {s}); its output is not valid")

    def check(self, device: torch.device) -> None:
        torch.cuda.synchronize(device)
        self.poll()
        check(lib().dcc_device_error_status(1), "attention")
        check(lib().dcc_build_error_status(1), "compact-KV build")
