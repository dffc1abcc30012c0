"""Straight-through-estimator quantizer, mirroring
``cdl.model.components.quant.ste`` (cdl/model/components/quant/ste.py:13-89).

``SteTensor`` quantizes its ``theta`` (flattened to 2-D) with the B200
kernels under ``no_grad``; ``proxy()`` is ``theta`` itself, so gradients pass
straight through (identity, no clipping mask); ``dequantize()`` serves the
``native`` backend.
"""

from __future__ import annotations

import ctypes
import weakref
from dataclasses import dataclass
from typing import Literal

import torch

from cdl_b200 import _lib

from cdl_b200.api.quant import QTensor, Quant
from cdl_b200.core.kernel.dequant import mxfp4_dequant, mxfp8_dequant, nvfp4_dequant
from cdl_b200.core.kernel.quant import mxfp4_quant, mxfp8_quant, nvfp4_dual_quant, nvfp4_quant

Simulation = Literal["nvfp4", "mxfp4", "mxfp8"]

# recent activation encodings, most recent first: (weakref to the storage
# owner, (format, view, version), (codes, scales, alpha))
_ENCODED: list = []
_ENCODED_MAX = 4
# attribute the optimizer's weight encoder sets on a weight (train/optim.py)
_ENCODED_ATTR = "_cdlb200_nvfp4"
# attribute of an activation whose producing kernel formed its amax
# (model/components/fused.py)
_AMAX_ATTR = "_cdlb200_amax"


def _lookup(owner: torch.Tensor, key):
    for ref, k, res in _ENCODED:
        if k == key and ref() is owner:
            return res
    return None


def _encode_with_amax(theta: torch.Tensor, amax: torch.Tensor):
    """NVFP4 (codes, GEMM-layout scales, alpha) and the dequantized copy of a
    contiguous [rows, k] bf16 tensor whose amax word is given."""
    rows, k = theta.shape
    dev = theta.device
    packed = torch.empty(rows, k // 2, dtype=torch.uint8, device=dev)
    scale = torch.empty(rows, k // 16, dtype=torch.uint8, device=dev)
    alpha = torch.empty(1, dtype=torch.float32, device=dev)
    deq = torch.empty(rows, k, dtype=torch.bfloat16, device=dev)
    t = _lib.Nvfp4EncodeTensor(theta.data_ptr(), rows, k, amax.data_ptr(), amax.numel(), 0, packed.data_ptr(),
                               scale.data_ptr(), alpha.data_ptr(), deq.data_ptr())
    _lib.call("cdlb200_nvfp4_encode_multi", ctypes.addressof(t), 1, _lib.stream(dev))
    return (packed, scale, alpha), deq


@dataclass
class SteTensor(QTensor):
    theta: torch.Tensor
    simulation: Simulation | None

    @property
    def leading_shape(self) -> torch.Size:
        return self.theta.shape[:-1]

    @property
    def k(self) -> int:
        return self.theta.shape[-1]

    def _encode(self, fn):
        with torch.no_grad():
            packed, scale, alpha = fn(self.theta.reshape(-1, self.k))
            packed = packed.reshape(*self.leading_shape, packed.shape[-1])
            scale = scale.reshape(*self.leading_shape, scale.shape[-1])
            return packed, scale, alpha

    def nvfp4(self):
        return self._encode(nvfp4_quant)

    def mxfp4(self):
        return self._encode(mxfp4_quant)

    def mxfp8(self):
        return self._encode(mxfp8_quant)

    def encode_swizzled(self, fmt: Simulation):
        """``(codes, scales, alpha)`` of ``theta`` flattened to 2-D, with the
        scales already in the 128x4 layout of the block-scaled GEMM (one
        quantize launch, no separate swizzle).  Same codes and scale bytes as
        ``nvfp4()`` / ``mxfp4()`` / ``mxfp8()``.

        An activation read by several linears (q/k/v, gate/up) is encoded
        once: the result is kept for the tensor it came from while that tensor
        is alive and unmodified (same storage owner, view and version)."""
        fn = {"nvfp4": nvfp4_quant, "mxfp4": mxfp4_quant, "mxfp8": mxfp8_quant}[fmt]
        enc = self._weight_encoding(fmt)
        if enc is not None:  # written by the optimizer step that produced this weight
            return enc[1], enc[2], enc[3]
        theta = self.theta.reshape(-1, self.k)
        owner = theta._base if theta._base is not None else theta
        # parameters are excluded: optimizers may update them without a version bump
        cacheable = not (owner.is_leaf and owner.requires_grad)
        if cacheable:
            key = (fmt, theta.data_ptr(), tuple(theta.shape), theta.stride(), theta.dtype, theta._version)
            hit = _lookup(owner, key)
            if hit is not None:
                return hit[:3]
        deq = None
        with torch.no_grad():
            amax = getattr(owner, _AMAX_ATTR, None)
            if (fmt == "nvfp4" and amax is not None and amax[1] == owner._version and theta.is_contiguous()
                    and theta.data_ptr() == owner.data_ptr() and theta.numel() == owner.numel()
                    and theta.shape[0] % 128 == 0 and self.k % 64 == 0):
                # the producing kernel formed the amax: encode in one pass, with
                # the dequantized copy the wgrad GEMM reads
                res, deq = _encode_with_amax(theta, amax[0])
            else:
                res = fn(theta, swizzled=True)
        if cacheable:
            _ENCODED.insert(0, (weakref.ref(owner), key, (*res, deq)))
            del _ENCODED[_ENCODED_MAX:]
        return res

    def encode_dual(self):
        """NVFP4 encodings ``(row, col)`` of ``theta`` flattened to 2-D
        ``[R, C]`` (R and C multiples of 64): ``row`` = ``encode_swizzled
        ("nvfp4")`` and ``col`` the encoding of its transpose (blocks of 16
        along dim 0), each ``(codes, GEMM-layout scales, alpha)``, from one
        read of ``theta`` -- the forward GEMM's operand and the quantized
        backward's.  A weight uses the optimizer's dual encoding while it is
        current; an activation is kept, as in ``encode_swizzled``, for the
        linears that share it, and uses its producer's amax words when they
        exist."""
        enc = self._weight_encoding("nvfp4")
        if enc is not None and len(enc) > 5:
            return (enc[1], enc[2], enc[3]), (enc[5], enc[6], enc[3])
        theta = self.theta.reshape(-1, self.k)
        owner = theta._base if theta._base is not None else theta
        cacheable = not (owner.is_leaf and owner.requires_grad)
        key = ("nvfp4_dual", theta.data_ptr(), tuple(theta.shape), theta.stride(), theta.dtype, theta._version)
        if cacheable:
            hit = _lookup(owner, key)
            if hit is not None:
                return hit
        with torch.no_grad():
            amax = getattr(owner, _AMAX_ATTR, None)
            words = None
            if (amax is not None and amax[1] == owner._version and theta.is_contiguous()
                    and theta.data_ptr() == owner.data_ptr() and theta.numel() == owner.numel()):
                words = amax[0]
            res = nvfp4_dual_quant(theta, amax=words)
        if cacheable:
            _ENCODED.insert(0, (weakref.ref(owner), key, res))
            del _ENCODED[_ENCODED_MAX:]
        return res

    def _weight_encoding(self, fmt: Simulation):
        """The optimizer's NVFP4 encoding of this (weight) tensor, if it is
        current: (version, codes, scales, alpha, dequantized)."""
        enc = getattr(self.theta, _ENCODED_ATTR, None)
        if fmt != "nvfp4" or enc is None or enc[0] != self.theta._version or self.theta.dim() != 2:
            return None
        return enc

    def cached_dequant(self, fmt: Simulation) -> torch.Tensor | None:
        """bf16 ``deq(Q(theta))`` if one was formed with the encoding (the
        optimizer's weight encoding, or an activation encoded with its
        producer's amax), else None.  Call after ``encode_swizzled``."""
        enc = self._weight_encoding(fmt)
        if enc is not None:
            return enc[4]
        theta = self.theta.reshape(-1, self.k)
        owner = theta._base if theta._base is not None else theta
        key = (fmt, theta.data_ptr(), tuple(theta.shape), theta.stride(), theta.dtype, theta._version)
        hit = _lookup(owner, key)
        return None if hit is None else hit[3]

    def dequantize(self) -> torch.Tensor:
        if self.simulation is None:
            return self.theta
        if self.simulation == "nvfp4":
            packed, scale, alpha = self.nvfp4()
            fn = nvfp4_dequant
        elif self.simulation == "mxfp4":
            packed, scale, alpha = self.mxfp4()
            fn = mxfp4_dequant
        elif self.simulation == "mxfp8":
            packed, scale, alpha = self.mxfp8()
            fn = mxfp8_dequant
        else:
            raise ValueError(f"{self.simulation} is not supported")
        out = fn(packed.reshape(-1, packed.shape[-1]), scale.reshape(-1, scale.shape[-1]), alpha)
        return out.reshape(*self.leading_shape, out.shape[-1])[..., : self.k].to(self.theta.dtype)

    def proxy(self) -> torch.Tensor | None:
        return self.theta


class SteQuant(Quant):
    def __init__(self, simulation: Simulation | None):
        super().__init__()
        self.simulation = simulation

    def forward(self, x: torch.Tensor) -> QTensor:
        return SteTensor(theta=x, simulation=self.simulation)
