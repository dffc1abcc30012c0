"""``mxfp4`` backend: the drop-in for ``cdl.core.mm.mxfp4`` (cdl/core/mm/mxfp4.py:9)."""

from cdl_b200.core.mm.blockscaled import make_matmul

matmul = make_matmul("mxfp4")
# dgrad and wgrad in mxfp4 as well (see blockscaled.py)
matmul_qbwd = make_matmul("mxfp4", quantized_backward=True)
