"""openquant_b200: OpenQuant's quantize-and-multiply path on NVIDIA B200.

Hand-written sm_100a CUDA kernels (openquant_b200/csrc, C ABI in
include/openquant_b200.h) behind the reference package's Python API:

  openquant_b200.quantization   QuantizedWeights, quantize, dequantize
  openquant_b200.groupwise      Groupwise4, quantize_int4_groupwise,
                                dequantize_int4_groupwise
  openquant_b200.gpu_benchmark  decode_gpu
  openquant_b200.group_benchmark restore_groupwise_torch
  openquant_b200.triton_int4    int4_linear
  openquant_b200.cli            main (`openquant gpu|tune|cpu|report`)

The top-level `openquant` package re-exports these under the reference's
module paths.
"""

__version__ = "0.1.0"
