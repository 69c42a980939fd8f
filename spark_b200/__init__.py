"""spark_b200 -- SPARK's online-dequant linear path, native on B200 (sm_100a).

The packed weight formats, the quantize/pack path, the STE fake-quant and the
dequant linear of DJAzzs/SPARK, computed by hand-written CUDA kernels behind a
C ABI (include/spark_b200.h).  The reference's layer/loader API is mirrored in
``quant_linear``, ``fp3_linear``, ``spark_loader`` and ``inference_v3``.
"""
from . import ops  # noqa: F401
from . import torch_ops  # noqa: F401  (registers torch.ops.spark.*)
from ._lib import SparkError  # noqa: F401

__version__ = "0.1.0"
