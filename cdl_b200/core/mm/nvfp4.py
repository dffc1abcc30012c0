"""``nvfp4`` backend: the drop-in for ``cdl.core.mm.nvfp4`` (cdl/core/mm/nvfp4.py:9)."""

from cdl_b200.core.mm.blockscaled import make_matmul

matmul = make_matmul("nvfp4")
# dgrad and wgrad in nvfp4 as well (see blockscaled.py)
matmul_qbwd = make_matmul("nvfp4", quantized_backward=True)
