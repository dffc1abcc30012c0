"""CPU oracle for cdl's block-scaled quantize path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use this package, and only as the checker.  The product (``cdl_b200``)
never imports it.

The heavy lifting is ``cdl_oracle.c`` (a plain-C restatement of the
reference's torch "nearest round" path, see the citations at the top of that
file), loaded through ctypes.  This module adds numpy glue and the GEMM oracle
``deq(A) @ deq(B)^T`` in fp32, which is how the reference's FP4/FP8 GEMM
(``cdl/model/wrapper/flashinfer.py:5-62``, a third-party FlashInfer call) is
specified: the GEMM itself lives in flashinfer-python 0.7.1 (absent here), so
GEMM parity is anchored on this dequantize-then-matmul definition.

Formats: ``NVFP4`` (block 16, e4m3 scales, per-tensor alpha), ``MXFP4`` (block
32, e8m0), ``MXFP8`` (block 32, e8m0, e4m3 elements).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

NVFP4, MXFP4, MXFP8 = 0, 1, 2
BLOCK = {NVFP4: 16, MXFP4: 32, MXFP8: 32}

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libcdl_oracle.so")
_lib = None


def build() -> None:
    """Compile ``libcdl_oracle.so`` with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _load():
    global _lib
    if _lib is not None:
        return _lib
    src = os.path.join(_HERE, "cdl_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    P, I64, I, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
    lib.oracle_quant.argtypes = [P, I64, I64, I64, I, F, P, P]
    lib.oracle_dequant.argtypes = [P, P, I64, I64, I, F, I, P]
    lib.oracle_swizzle.argtypes = [P, I64, I64, P]
    lib.oracle_nvfp4_global.argtypes = [P, I64, P, P]
    lib.oracle_f32_to_e4m3.argtypes = [F]
    lib.oracle_f32_to_e4m3.restype = ctypes.c_uint8
    lib.oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
    lib.oracle_e4m3_to_f32.restype = F
    lib.oracle_f32_to_bf16.argtypes = [F]
    lib.oracle_f32_to_bf16.restype = ctypes.c_uint16
    _lib = lib
    return lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def nvfp4_global(x: np.ndarray) -> tuple[float, float]:
    """(gmax, alpha) of a bf16-bits array, as quant.py:96-101."""
    lib = _load()
    x = np.ascontiguousarray(x, dtype=np.uint16)
    g = np.zeros(1, np.float32)
    a = np.zeros(1, np.float32)
    lib.oracle_nvfp4_global(_ptr(x), x.size, _ptr(g), _ptr(a))
    return float(g[0]), float(a[0])


def quant(x: np.ndarray, fmt: int, gmax: float | None = None):
    """Row-wise block quantize of bf16 bits ``x[rows, k]``.

    Returns ``(packed, scale, alpha)`` exactly as the reference's
    ``nvfp4_quant`` / ``mxfp4_quant`` / ``mxfp8_quant`` (quant.py:126-146):
    packed uint8 ``[rows, nb*B/2]`` (FP4) or ``[rows, nb*B]`` (FP8 bytes),
    scale uint8 ``[rows, nb]``, alpha float32 ``[1]`` (NVFP4: gmax/2688 as the device forms it, gmax * RN(1/2688),
    MXFP4: 1.0) or ``None`` (MXFP8).
    """
    lib = _load()
    x = np.ascontiguousarray(x, dtype=np.uint16)
    if x.ndim != 2:
        raise ValueError(f"expected a 2D tensor [rows, k], got shape {x.shape}")
    rows, k = x.shape
    B = BLOCK[fmt]
    nb = (k + B - 1) // B
    pstride = nb * B if fmt == MXFP8 else nb * B // 2
    packed = np.zeros((rows, pstride), np.uint8)
    scale = np.zeros((rows, nb), np.uint8)
    alpha = None
    if fmt == NVFP4:
        g, a = nvfp4_global(x)
        if gmax is None:
            gmax = g
        alpha = np.array([a], np.float32)
    elif fmt == MXFP4:
        alpha = np.ones(1, np.float32)
    if rows and k:
        lib.oracle_quant(_ptr(x), rows, k, k, fmt, float(gmax or 0.0), _ptr(packed), _ptr(scale))
    return packed, scale, alpha


def dequant(packed: np.ndarray, scale: np.ndarray, fmt: int, alpha=None) -> np.ndarray:
    """bf16 bits of ``(value * scale) * alpha`` (dequant.py:25-72)."""
    lib = _load()
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scale = np.ascontiguousarray(scale, dtype=np.uint8)
    rows = packed.shape[0]
    k = packed.shape[1] * (1 if fmt == MXFP8 else 2)
    out = np.zeros((rows, k), np.uint16)
    has_alpha = alpha is not None
    a = float(np.asarray(alpha, np.float32).reshape(-1)[0]) if has_alpha else 1.0
    if rows and k:
        lib.oracle_dequant(_ptr(packed), _ptr(scale), rows, k, fmt, a, int(has_alpha), _ptr(out))
    return out


def swizzle(sf: np.ndarray) -> np.ndarray:
    """``swizzle_scale_factors`` (swizzle.py:5-14) on a uint8 ``[m, b]`` array."""
    lib = _load()
    sf = np.ascontiguousarray(sf, dtype=np.uint8)
    m, b = sf.shape
    out = np.zeros(((m + 127) // 128 * 128, (b + 3) // 4 * 4), np.uint8)
    if m and b:
        lib.oracle_swizzle(_ptr(sf), m, b, _ptr(out))
    return out


_E2M1 = np.array([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6], np.float32)


def e4m3_values(b: np.ndarray) -> np.ndarray:
    lib = _load()
    table = np.array([lib.oracle_e4m3_to_f32(i) for i in range(256)], np.float32)
    return table[np.asarray(b, np.uint8)]


def e8m0_values(b: np.ndarray) -> np.ndarray:
    b = np.asarray(b, np.uint8).astype(np.uint32)
    return np.where(b == 0, np.uint32(0x00400000), b << 23).astype(np.uint32).view(np.float32)


def dequant_f32(packed: np.ndarray, scale: np.ndarray, fmt: int) -> np.ndarray:
    """Exact fp32 ``value * block_scale`` (no alpha, no bf16 rounding)."""
    B = BLOCK[fmt]
    if fmt == MXFP8:
        vals = e4m3_values(packed)
    else:
        lo = packed & 15
        hi = packed >> 4
        nib = np.stack([lo, hi], axis=-1).reshape(packed.shape[0], -1)
        vals = _E2M1[nib]
    sv = e4m3_values(scale) if fmt == NVFP4 else e8m0_values(scale)
    return vals * np.repeat(sv, B, axis=1)[:, : vals.shape[1]]


def mm(a_packed, a_scale, b_packed, b_scale, fmt: int, alpha: float = 1.0) -> np.ndarray:
    """GEMM oracle: ``alpha * deq(A) @ deq(B)^T`` in fp32, A ``[M, K]``, B ``[N, K]``."""
    A = dequant_f32(a_packed, a_scale, fmt)
    Bm = dequant_f32(b_packed, b_scale, fmt)
    return (A @ Bm.T) * np.float32(alpha)
