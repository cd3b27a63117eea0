"""prismaquant_b200 — B200 (sm_100a) kernels for prismaquant's per-(Linear, format)
quantization-cost path, behind the reference's Python API.

Modules mirror the reference modules they stand in for:
  format_registry           FormatSpec / REGISTRY / get_format (CUDA quantize_dequantize)
  measure_quant_cost        fused multi-format MSE_W sweep, measure_batched_gpu & co.
  export_native_compressed  NVFP4 / MXFP8 / FP8 packing into compressed-tensors layouts
  sensitivity_probe         Fisher-trace hooks (FisherAccumulator, _GradNormCapture)
  distributed               unit sharding across ranks + the NCCL cost-table exchange
"""
__version__ = "0.1.0"
