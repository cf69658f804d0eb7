"""ctypes binding of libcab_b200.so (the C ABI declared in include/cab_capi.h).

Every op of this package calls through here. There is no other implementation: if the
library is missing or the tensors are not on an sm_100 CUDA device, the call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB_NAME = "libcab_b200.so"
_lock = threading.Lock()
_lib = None
_supported: dict = {}

CAB_OK = 0
CAB_ERR_TIMEOUT = 4
DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
NORMALIZATIONS = {"abs": 0, "minmax": 1, "raw": 2}
FORMULAS = {"additive": 0, "multiplicative": 1}
REDUNDANCY_SCALES = {"none": 0, "inv_m": 1}

_c_i64 = ctypes.c_int64
_c_ptr = ctypes.c_void_p
_c_int = ctypes.c_int
_c_float = ctypes.c_float
_c_size = ctypes.c_size_t
_i64_3 = ctypes.c_int64 * 3

# name -> (argtypes) ; every entry point returns int except cab_last_error_string
SIGNATURES = {
    "cab_get_version": [],
    "cab_last_error_string": [],
    "cab_device_supported": [_c_int],
    "cab_device_status": [_c_ptr, ctypes.POINTER(_c_int)],
    "cab_selftest_wait_timeout": [_c_i64, _c_ptr, _c_ptr],
    "cab_coarsen_maxl2": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                          _c_i64, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_int, _c_ptr],
    "cab_frc_workspace_size": [_c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_int,
                               ctypes.POINTER(_c_size)],
    "cab_frc": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                _c_int, _c_float, _c_float, _c_int, _c_int, _c_int, _c_ptr, _c_size, _c_ptr],
    "cab_topk_blocks": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_int, _c_int,
                        _c_int, _c_ptr],
    "cab_topk_blocks_hybrid": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                               ctypes.c_double, _c_int, _c_int, _c_int, _c_ptr],
    "cab_block_maxpool": [_c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_int, _c_ptr],
    "cab_sparse_attn_workspace_size": [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_int,
                                       ctypes.POINTER(_c_size)],
    "cab_sparse_attn_fwd": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64,
                            _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_ptr, _c_ptr,
                            _c_ptr, _c_ptr, _c_float, _c_int, _c_int, _c_ptr, _c_size, _c_ptr],
    "cab_sparse_attn_fwd_noalloc": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64,
                                    _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_ptr,
                                    _c_ptr, _c_ptr, _c_ptr, _c_float, _c_int, _c_int, _c_ptr],
    "cab_flash_attn_workspace_size": [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_int, _c_int,
                                      ctypes.POINTER(_c_size)],
    "cab_flash_attn_fwd": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                           _c_i64, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_float, _c_int,
                           _c_int, _c_ptr, _c_size, _c_ptr],
    "cab_node_frc": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_int, _c_ptr],
    "cab_evict_workspace_size": [_c_i64, _c_i64, _c_int, ctypes.POINTER(_c_size)],
    "cab_evict_select": [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_i64, _c_i64, ctypes.c_double,
                         ctypes.c_double, _c_ptr, _c_ptr, _c_ptr, _c_size, _c_ptr],
    "cab_prefill_host_workspace_size": [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64,
                                        _c_int, _c_int, ctypes.POINTER(_c_size)],
    "cab_prefill_host": [_c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64,
                         _c_i64, _c_i64, _c_i64, _c_i64, _c_float, _c_float, _c_int, _c_int,
                         _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _c_ptr, _c_size,
                         _c_ptr],
}


def library_path() -> Path:
    override = os.environ.get("CAB_B200_LIBRARY")
    return Path(override) if override else Path(__file__).resolve().parent / _LIB_NAME


def lib():
    """Loads libcab_b200.so once; raises ImportError if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not path.exists():
                raise ImportError(f"{path} is missing: build it with "
                                  "`python <package>/cab_build.py` (nvcc, sm_100a)")
            handle = ctypes.CDLL(str(path))
            for name, argtypes in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = argtypes
                fn.restype = ctypes.c_char_p if name == "cab_last_error_string" else ctypes.c_int
            _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != CAB_OK:
        msg = lib().cab_last_error_string().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def strides3(t: torch.Tensor):
    """{b, h, n} element strides of a [B,H,N,D] tensor whose last dimension is dense."""
    if t.stride(3) != 1:
        raise ValueError("innermost dimension must be contiguous")
    return _i64_3(t.stride(0), t.stride(1), t.stride(2))


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("CAB kernels run on an sm_100 CUDA device only (tensor on "
                               f"{t.device}); there is no CPU implementation")
    dev = next(t for t in tensors if t is not None).device
    index = dev.index if dev.index is not None else torch.cuda.current_device()
    ok = _supported.get(index)
    if ok is None:
        ok = _supported[index] = bool(lib().cab_device_supported(index))
    if not ok:
        raise RuntimeError("CAB kernels are built for sm_100 (B200); device "
                           f"{torch.cuda.get_device_name(dev)} is not supported")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return DTYPE_CODES[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; use bfloat16, float16 or float32")


def workspace(nbytes: int, device) -> torch.Tensor | None:
    if nbytes == 0:
        return None
    return torch.empty(int(nbytes), dtype=torch.uint8, device=device)


def device_status(device=None) -> int:
    """Synchronises the current stream and returns (and clears) the kernels' status word."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    out = ctypes.c_int(0)
    check(lib().cab_device_status(torch.cuda.current_stream(dev).cuda_stream, ctypes.byref(out)),
          "cab_device_status")
    return out.value
