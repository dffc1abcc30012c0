"""CPU oracle of the block-scaled quantize of fp32 / fp16 input -- TEST
INFRASTRUCTURE ONLY (imported by ``tests/`` alone).

cdl's ``_quant`` accepts any floating tensor (``cdl/core/kernel/quant.py:71-123``):
the NVFP4 global amax is ``x.abs().amax().float().clamp_min(tiny)`` and alpha
``gmax / (448 * 6)`` (quant.py:96-101), which torch computes on the device as
``gmax * RN(1 / 2688)``; the Triton ``_quant_kernel``
(quant.py:13-68) loads each block, casts it to fp32 and performs, in fp32:

* E8M0 scale (quant.py:39-46): ``byte = clamp(floor(log2(max(bamax, tiny))) -
  emax + 127, 0, 254)``, ``s = 2^(byte - 127)`` (byte 0 = the subnormal 2^-127);
* UE4M3 scale (quant.py:47-51): ``q = div_rn(bamax * 448, gmax)``,
  ``byte = ue4m3 ordinal(q) + 1`` (RNE to e4m3 after clamping to [2^-9, 448],
  ``formats/ordinals.py:23-29``), ``s = e4m3(byte) * alpha``;
* ``v = div_rn(x, s)``; FP4 code = the number of e2m1 midpoints
  {.25, .75, 1.25, 1.75, 2.5, 3.5, 5} that ``min(|v|, 6)`` exceeds, with the
  sign bit of v (``ordinals.py:7-20``, quant.py:55-65); FP8 = RNE e4m3 of
  ``clamp(v, -448, 448)`` (quant.py:66-68).

This numpy restatement keeps every operation in float32 (numpy rounds each
float32 operation to nearest even).  One deliberate difference from the
Triton formula: an infinite block amax gives E8M0 byte 254, as the
reference's torch path (``core/ecdl.py:59-73``) and the golden vectors made
from it; the Triton formula would give 253 (MXFP4) / 247 (MXFP8).  Pinned by
``tests/test_oracle.py``: on bf16-valued inputs it equals the C oracle, which
the reference's golden vectors pin.
"""

from __future__ import annotations

import numpy as np

from oracle import BLOCK, MXFP4, MXFP8, NVFP4
from oracle.ecdl import e4m3_rne, e4m3_value

_MIDS = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
_TINY = np.float32(np.finfo(np.float32).tiny)
_EMAX = {NVFP4: 2, MXFP4: 2, MXFP8: 8}


def _e8m0(bamax: np.ndarray, emax: int) -> np.ndarray:
    bits = np.maximum(bamax, _TINY).astype(np.float32).view(np.uint32).astype(np.int64)
    b = np.clip((bits >> 23) - 127 - emax + 127, 0, 254)
    b = np.where(np.isinf(bamax), 254, b)
    return np.where(np.isnan(bamax), 0, b).astype(np.int64)


def _e8m0_value(byte: np.ndarray) -> np.ndarray:
    bits = np.where(byte == 0, 0x00400000, byte.astype(np.int64) << 23).astype(np.uint32)
    return bits.view(np.float32)


def quant_wide(x: np.ndarray, fmt: int):
    """``(packed uint8, scale uint8 [rows, nb], alpha float32 [1] or None)`` of
    a float32 (or float16, widened exactly) matrix ``x[rows, k]``, row-wise
    blocks, K zero-padded to the block (quant.py:34)."""
    x = np.asarray(x)
    if x.ndim != 2:
        raise ValueError(f"expected a 2D tensor [rows, k], got shape {x.shape}")
    x = x.astype(np.float32)
    rows, k = x.shape
    B = BLOCK[fmt]
    nb = (k + B - 1) // B
    xp = np.zeros((rows, nb * B), np.float32)
    xp[:, :k] = x
    blk = xp.reshape(rows, nb, B)
    bamax = np.abs(blk).max(axis=-1) if nb else np.zeros((rows, 0), np.float32)
    alpha = None
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        if fmt == NVFP4:
            g = np.float32(np.abs(x).max()) if x.size else np.float32(0)
            gmax = g if (np.isnan(g) or g >= _TINY) else _TINY
            # formed on the device: gmax * RN(1 / 2688) (cdl_oracle.c, nvfp4_alpha)
            alpha = np.array([gmax * (np.float32(1.0) / np.float32(2688.0))], np.float32)
            q = (bamax * np.float32(448.0)).astype(np.float32) / gmax
            q = np.where(np.isnan(q), np.float32(448.0), np.clip(q, np.float32(2.0 ** -9), np.float32(448.0)))
            byte = e4m3_rne(q.astype(np.float32))
            s = (e4m3_value(byte).astype(np.float32) * alpha[0]).astype(np.float32)
        else:
            byte = _e8m0(bamax, _EMAX[fmt])
            s = _e8m0_value(byte)
        v = (blk / s[..., None]).astype(np.float32)
        if fmt == MXFP8:
            codes = e4m3_rne(np.clip(v, np.float32(-448.0), np.float32(448.0))).astype(np.uint8)
            packed = codes.reshape(rows, nb * B)
        else:
            av = np.minimum(np.abs(v), np.float32(6.0))
            mag = (av[..., None] > _MIDS).sum(axis=-1)
            code = (mag | (np.signbit(v).astype(np.int64) << 3)).astype(np.uint8).reshape(rows, nb * B)
            packed = (code[:, 0::2] | (code[:, 1::2] << 4)).astype(np.uint8)
    return packed, byte.astype(np.uint8), alpha
