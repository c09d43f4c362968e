"""ctypes binding of libtjb200.so, the sm_100a kernel library.

The library sits next to this file.  Importing this module does not load it;
``lib()`` does, and raises ``RuntimeError`` when it is missing, so a product
call without the compiled kernels fails loudly instead of falling back.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

# The in-tree build (tiktok-techjam-2026_b200/build.py writes it here).
LIB_PATH = Path(__file__).resolve().with_name("libtjb200.so")

TJB_F32, TJB_F16, TJB_BF16 = 0, 1, 2

_c_int, _c_i64, _c_f32, _p = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/tjb200.h.
SIGNATURES = {
    "tjb_version": (_c_int, []),
    "tjb_status_string": (ctypes.c_char_p, [_c_int]),
    "tjb_last_cuda_error": (ctypes.c_char_p, []),
    "tjb_add_layernorm": (_c_int, [_p, _p, _p, _p, _p, _p, _c_i64, _c_int, _c_f32,
                                   _c_int, _c_int, _p, _p]),
    "tjb_add_layernorm_tiles": (_c_int, [_p, _p, _p, _p, _p, _p, _c_i64, _c_int, _c_f32,
                                         _c_int, _c_int, _p, _p, _p]),
    "tjb_gemm_bias": (_c_int, [_p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int,
                               _c_int, _c_int, _c_int, _c_int, _p]),
    "tjb_gemm_bias_tiles": (_c_int, [_p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int,
                                     _c_int, _c_int, _c_int, _c_int, _p, _p]),
    "tjb_flash_fwd": (_c_int, [_p, _p, _c_int, _c_int, _c_int, _c_int, _c_f32, _c_int,
                               _p, _p, _p, _c_int, _p]),
    "tjb_flash_fwd_sched": (_c_int, [_p, _p, _c_int, _c_int, _c_int, _c_int, _c_f32, _c_int,
                                     _p, _p, _p, _c_int, _p, _c_int, _p]),
    "tjb_ffn": (_c_int, [_p, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int,
                         _c_int, _p]),
    "tjb_ffn_tiles": (_c_int, [_p, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int,
                               _c_int, _p, _p]),
    "tjb_gemm_workspace_bytes": (ctypes.c_size_t, []),
    "tjb_gemm_bias_tiles_ws": (_c_int, [_p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int,
                                        _c_int, _c_int, _c_int, _c_int, _p, _p, ctypes.c_size_t,
                                        _p]),
    "tjb_ffn_tiles_ws": (_c_int, [_p, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int,
                                  _c_int, _p, _p, ctypes.c_size_t, _p]),
    "tjb_gemm_add_layernorm": (_c_int, [_p, _p, _p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int,
                                        ctypes.c_float, _c_int, _c_int, _p, _p, _p,
                                        ctypes.c_size_t, _p]),
    "tjb_gemm_add_layernorm_workspace_bytes": (ctypes.c_size_t, [_c_int, _c_int]),
    "tjb_ffn_fused": (_c_int, [_p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int, _c_int,
                               _p, _p]),
    "tjb_row_tiles": (_c_int, [_p, _p, _c_int, _c_int, _p, _p]),
    "tjb_ffn_noalloc": (_c_int, [_p, _p, _p, _p, _p, _p, _c_int, _c_int, _c_int, _c_int,
                                 _c_int, _p]),
    "tjb_mask_lengths": (_c_int, [_p, _c_int, _c_int, _p, _p, _p]),
    "tjb_mask_lengths_tiles": (_c_int, [_p, _c_int, _c_int, _p, _p, _p, _p]),
    "tjb_device_status": (_c_int, [_c_int]),
    "tjb_device_status_async": (_c_int, [_p, _p]),
    "tjb_selftest_wait": (_c_int, [_p, _c_i64, _p]),
    "tjb_forward_small_workspace_bytes": (ctypes.c_size_t, [_c_int, _c_int, _c_int, _c_int]),
    "tjb_forward_small": (_c_int, [_p, _c_int, _p, _p, _c_f32, _p, _p, _p, _c_int, _c_int,
                                   _c_int, _c_int, _c_int, _c_int, _c_int, _p, ctypes.c_size_t,
                                   _p]),
}


class SmallLayer(ctypes.Structure):
    """tjb_small_layer: one block's device pointers for tjb_forward_small."""

    _fields_ = [("wqkv", _p), ("wo", _p), ("w1", _p), ("w2", _p), ("bqkv", _p), ("bo", _p),
                ("b1", _p), ("b2", _p), ("ln1_w", _p), ("ln1_b", _p), ("ln2_w", _p),
                ("ln2_b", _p), ("ln1_eps", _c_f32), ("ln2_eps", _c_f32)]

_lock = threading.Lock()
_lib = None


class KernelError(RuntimeError):
    """A libtjb200 entry point returned a non-zero status."""

    def __init__(self, what: str, status: int, message: str) -> None:
        super().__init__(f"{what}: {message} (status {status})")
        self.status = status


def load(path: Path = LIB_PATH) -> ctypes.CDLL:
    """Load the library and declare every entry point's signature."""
    if not path.exists():
        raise RuntimeError(
            f"libtjb200.so not found at {path}; build it with "
            "`python tiktok-techjam-2026_b200/build.py` (needs nvcc)")
    handle = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    return handle


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                _lib = load()
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().tjb_status_string(status).decode()
        if status == 5:  # TJB_ERR_LAUNCH: add the CUDA error behind it
            msg += ": " + lib().tjb_last_cuda_error().decode()
        raise KernelError(what, status, msg)
