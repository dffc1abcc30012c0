"""cdl_b200 -- B200-native (sm_100a) low-precision hot path of cdl.

Block-scaled NVFP4/MXFP4/MXFP8 quantize/dequantize kernels, tcgen05
block-scaled GEMMs and the SmolLM2 QAT step, behind cdl's own Python
quantizer / linear-layer API.  The CUDA code lives in ``cdl_b200/csrc`` and
is loaded from the in-tree ``libcdlb200.so`` through a plain C ABI
(``include/cdlb200.h``).
"""

__version__ = "0.1.0"
