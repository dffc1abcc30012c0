"""ctypes binding of ``libcdlb200.so`` (the C ABI in ``include/cdlb200.h``).

The library is loaded from the package directory.  There is no fallback: if
the shared library is missing or the tensors are not on a CUDA device, calls
raise instead of computing anything on the CPU.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcdlb200.so")

OK = 0
ERR_INVALID_ARG = -1
ERR_ALIGNMENT = -2
ERR_UNSUPPORTED = -3
ERR_LAUNCH = -4
ERR_TIMEOUT = -5
ERR_WORKSPACE = -6
ERR_CUDA = -7
AMAX_WORDS = 32  # CDLB200_AMAX_WORDS

SCALE_LINEAR = 0
SCALE_SWIZZLED = 1
DTYPE_F32, DTYPE_F16 = 1, 2
DUAL_ROW_LINEAR, DUAL_COL_LINEAR = 1, 2

_lib = None
_lock = threading.Lock()

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_SZ = ctypes.c_size_t
_F = ctypes.c_float
_D = ctypes.c_double

# name -> (restype, argtypes); every symbol declared in include/*.h
SIGNATURES: dict[str, tuple] = {
    "cdlb200_status_string": (ctypes.c_char_p, [_I]),
    "cdlb200_version": (_I, []),
    "cdlb200_set_wait_limit": (ctypes.c_uint32, [ctypes.c_uint32]),
    "cdlb200_set_persistent_sm_limit": (_I, [_I]),
    "cdlb200_nvfp4_quant_workspace_bytes": (_SZ, [_I64, _I64]),
    "cdlb200_nvfp4_quant": (_I, [_P, _I64, _I64, _I64, _I, _P, _P, _I, _P, _P, _P, _SZ, _P]),
    "cdlb200_nvfp4_quant_noalloc": (_I, [_P, _I64, _I64, _I64, _I, _P, _P, _I, _P, _P, _P]),
    "cdlb200_nvfp4_amax": (_I, [_P, _I64, _I64, _I64, _P, _P, _P, _SZ, _P]),
    "cdlb200_mxfp4_quant": (_I, [_P, _I64, _I64, _I64, _I, _P, _P, _I, _P]),
    "cdlb200_mxfp8_quant": (_I, [_P, _I64, _I64, _I64, _I, _P, _P, _I, _P]),
    "cdlb200_quant_wide": (_I, [_P, _I, _I, _I64, _I64, _I64, _I, _P, _P, _I, _P, _P, _SZ, _P]),
    "cdlb200_fp4_dequant": (_I, [_P, _P, _P, _I64, _I64, _I, _I, _P, _P]),
    "cdlb200_fp4_dequant_swizzled": (_I, [_P, _P, _P, _I64, _I64, _I, _I, _P, _P]),
    "cdlb200_mxfp8_dequant": (_I, [_P, _P, _P, _I64, _I64, _P, _P]),
    "cdlb200_swizzle_scales": (_I, [_P, _I64, _I64, _P, _P]),
    "cdlb200_mm_fp4": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _P, _I64, _P, _P]),
    "cdlb200_mm_mxfp8": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _P, _I64, _P, _P]),
    "cdlb200_mm_fp4_alpha2": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _P, _I64, _P, _P]),
    "cdlb200_mm_fp4_alpha2_acc": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I, _I, _P, _I64, _P, _P]),
    # include/cdlb200_step.h
    "cdlb200_rmsnorm_fwd": (_I, [_P, _P, _I64, _I64, ctypes.c_float, _P, _P, _P, _P]),
    "cdlb200_rmsnorm_bwd_workspace_bytes": (_I64, [_I64, _I64]),
    "cdlb200_rmsnorm_bwd": (_I, [_P, _P, _P, _P, _I64, _I64, _P, _P, _P, _I64, _P]),
    "cdlb200_add_rmsnorm_fwd": (_I, [_P, _P, _P, _I64, _I64, ctypes.c_float, _P, _P, _P, _P, _P]),
    "cdlb200_rmsnorm_bwd_add": (_I, [_P, _P, _P, _P, _P, _I64, _I64, _P, _P, _P, _P, _I64, _P]),
    "cdlb200_rope": (_I, [_P, _P, _P, _I64, _I64, _I64, _I64, _I, _P, _P, _P]),
    "cdlb200_swiglu_fwd": (_I, [_P, _P, _I64, _P, _P, _P]),
    "cdlb200_swiglu_bwd": (_I, [_P, _P, _P, _I64, _P, _P, _P, _P, _P]),
    "cdlb200_cross_entropy": (_I, [_P, _P, _I64, _I64, _F, _P, _P]),
    "cdlb200_scale_bf16": (_I, [_P, _I64, _P, _P]),
    "cdlb200_ecdl_fwd": (_I, [_P, _I, _I64, _I64, _I, _I, _P, _P, _I, _P, _P, _P, _P, _P]),
    "cdlb200_ecdl_bwd_workspace_bytes": (_I64, [_I64, _I64, _I]),
    "cdlb200_ecdl_bwd": (_I, [_P, _P, _I, _I64, _I64, _I, _P, _P, _P, _I, _P, _P, _P, _I64, _P]),
    "cdlb200_ccdl_fwd": (_I, [_P, _I, _I64, _I64, _I, _P, _I64, _P, _P, _P, _P, _I, _I, _P, _P, _P]),
    "cdlb200_ccdl_round": (_I, [_P, _I, _I64, _I64, _I, _P, _I64, _P, _I, _P, _P, _P]),
    "cdlb200_ccdl_bwd_workspace_bytes": (_I64, [_I64, _I64, _I]),
    "cdlb200_ccdl_bwd": (_I, [_P, _P, _I, _I64, _I64, _I, _P, _I64, _P, _I64, _P, _P, _P, _I, _I, _P, _P, _P, _P,
                              _I64, _P]),
    "cdlb200_clip_adamw_workspace_bytes": (_I64, [_P, _I]),
    "cdlb200_clip_adamw": (_I, [_P, _I, _D, _D, _D, _D, _D, _D, _P, _I64, _P, _P]),
    "cdlb200_nvfp4_encode_multi": (_I, [_P, _I, _P]),
    "cdlb200_nvfp4_dual_multi": (_I, [_P, _I, _P]),
}


class AdamwTensor(ctypes.Structure):
    """``cdlb200_adamw_tensor`` (include/cdlb200_step.h)."""

    _fields_ = [("param", _P), ("grad", _P), ("exp_avg", _P), ("exp_avg_sq", _P), ("numel", _I64), ("amax", _P)]


class Nvfp4EncodeTensor(ctypes.Structure):
    """``cdlb200_nvfp4_encode_tensor`` (include/cdlb200_step.h)."""

    _fields_ = [("x", _P), ("rows", _I64), ("k", _I64), ("amax", _P), ("amax_words", ctypes.c_int32),
                ("pad", ctypes.c_int32), ("packed", _P), ("scale", _P), ("alpha", _P), ("deq", _P)]


class Nvfp4DualTensor(ctypes.Structure):
    """``cdlb200_nvfp4_dual_tensor`` (include/cdlb200_step.h)."""

    _fields_ = [("x", _P), ("rows", _I64), ("cols", _I64), ("amax", _P), ("gmax", _P),
                ("amax_words", ctypes.c_int32), ("flags", ctypes.c_int32), ("alpha", _P), ("row_packed", _P),
                ("row_scale", _P), ("col_packed", _P), ("col_scale", _P)]


class CdlB200Error(RuntimeError):
    """A libcdlb200 call returned a non-zero status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed: {msg} (status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load (once) and return the shared library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is not built; run `python -m cdl_b200.build` "
                    "(there is no CPU fallback for the cdl_b200 kernels)"
                )
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


# kernels one call of an entry point launches (default 1); `launches` counts
# them over the process, so a benchmark can report how many ran
KERNELS_PER_CALL = {"cdlb200_rmsnorm_bwd": 2, "cdlb200_rmsnorm_bwd_add": 2, "cdlb200_clip_adamw": 3, "cdlb200_ecdl_fwd": 2, "cdlb200_ecdl_bwd": 2,
                    "cdlb200_ccdl_bwd": 2}
launches = 0


def call(name: str, *args) -> None:
    global launches
    launches += KERNELS_PER_CALL.get(name, 1)
    status = getattr(lib(), name)(*args)
    if status != OK:
        msg = lib().cdlb200_status_string(status).decode()
        if status in (ERR_INVALID_ARG, ERR_ALIGNMENT, ERR_WORKSPACE):
            raise ValueError(f"{name}: {msg} (status {status})")
        raise CdlB200Error(name, status, msg)


def set_persistent_sm_limit(sms: int) -> None:
    """Cap the SMs the persistent kernels fill (0: all); a host-side setting,
    no kernel launch (``cdlb200_set_persistent_sm_limit``)."""
    status = lib().cdlb200_set_persistent_sm_limit(int(sms))
    if status != OK:
        raise ValueError(f"cdlb200_set_persistent_sm_limit({sms}): {lib().cdlb200_status_string(status).decode()}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                "cdl_b200 kernels run on CUDA tensors only (no CPU fallback); got a tensor on "
                f"{t.device}"
            )
        dev = t.device if dev is None else dev
    return dev


_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}
_STATUS: dict[int, torch.Tensor] = {}
WS_STATUS_OFFSET = 8  # status word of an NVFP4 quantize workspace (include/cdlb200.h)


def _dev_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device uint32 status word (as int32) that every block-scaled GEMM
    call of this package passes to the kernel: a timed-out bounded wait sets
    it non-zero.  Allocated (zeroed) on first use; ``check_status`` reads and
    clears it."""
    idx = _dev_index(device)
    st = _STATUS.get(idx)
    if st is None:
        st = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = st
    return st


def check_status(device: torch.device | None = None) -> None:
    """Raise ``CdlB200Error`` (``ERR_TIMEOUT``) if a kernel of this package on
    ``device`` (default: every device used) recorded a timed-out bounded wait
    since the last check: the GEMM status word, or the status word of an NVFP4
    quantize workspace.  The words are cleared.  This reads device memory
    (a synchronizing copy): call it between steps, not inside a timed region
    or a graph capture."""
    idx = None if device is None else _dev_index(device)
    words = [(f"GEMM status (cuda:{d})", t[0:1]) for d, t in _STATUS.items() if idx is None or d == idx]
    words += [(f"NVFP4 quantize workspace (cuda:{d})", ws[WS_STATUS_OFFSET:WS_STATUS_OFFSET + 4].view(torch.int32))
              for (d, _s), ws in _WORKSPACES.items() if idx is None or d == idx]
    bad = [name for name, w in words if int(w.item()) != 0]
    for _name, w in words:
        w.zero_()
    if bad:
        raise CdlB200Error("check_status", ERR_TIMEOUT,
                           f"{lib().cdlb200_status_string(ERR_TIMEOUT).decode()} in: {', '.join(bad)}")


def nvfp4_workspace(device: torch.device) -> torch.Tensor:
    """Per-(device, stream) scratch of the NVFP4 global amax (zeroed once).

    The kernels leave it re-armed, so one buffer serves every stream-ordered
    call.  Calls on different streams get different buffers.
    """
    key = (_dev_index(device), stream(device))
    ws = _WORKSPACES.get(key)
    if ws is None:
        nbytes = lib().cdlb200_nvfp4_quant_workspace_bytes(0, 0)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws
