"""``mxfp8`` backend: the drop-in for ``cdl.core.mm.mxfp8`` (cdl/core/mm/mxfp8.py:9)."""

from cdl_b200.core.mm.blockscaled import make_matmul

matmul = make_matmul("mxfp8")
# dgrad and wgrad in mxfp8 as well (see blockscaled.py)
matmul_qbwd = make_matmul("mxfp8", quantized_backward=True)
