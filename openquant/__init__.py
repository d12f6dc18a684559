"""Reference-compatible module paths for openquant_b200.

`openquant.<module>` re-exports `openquant_b200.<module>`, so code written
against the reference package (openquant 0.5.0) imports this build without
changes: openquant.quantization, openquant.groupwise, openquant.triton_int4,
openquant.gpu_benchmark, openquant.group_benchmark, openquant.autotune,
openquant.fused_benchmark, openquant.benchmark, openquant.report and
openquant.cli.
"""
