"""B200-native (sm_100a) CDQ-LRR decode path.

Packed 5-bit (26-state) / 4-bit (16-state) lattice weights with float8 tile
scales and sparse bf16 residuals, served by a fused dequant-GEMV that never
writes the dequantised weight to HBM, plus a bit-exact GPU tile quantizer
and drop-in mirrors of the reference's Python entry points:

* ``cdq_lrr_b200.quant``     - code/cdq_lrr_qwen05.py (quantize_cdq_lrr,
  dequantize, CDQLinear)
* ``cdq_lrr_b200.loader``    - code/cdq_loader.py (load_cdq, loader CDQLinear)
* ``cdq_lrr_b200.pack_file`` - code/cdq_pack.py (.cdq codec, packer CLI)
* ``cdq_lrr_b200.ops``       - device packs and the raw kernel calls
* ``include/cdq.h``          - the C ABI (libcdq_b200.so)
"""
from ._lib import CdqError, lib  # noqa: F401

__all__ = ["CdqError", "lib"]
