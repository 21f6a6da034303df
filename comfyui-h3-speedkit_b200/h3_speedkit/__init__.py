"""H3 SpeedKit quantized DiT-block linear path, rebuilt for NVIDIA B200 (sm_100a).

The package mirrors the reference plugin's ``h3_speedkit`` layout for the
accelerated path: ``ops.norm_quant`` (fused prologue), ``ops.convrot``
(ConvRot256 INT8 quantiser), ``ops.gemm`` (tcgen05 INT8 GEMMs with fused
epilogues), ``runtime`` (Backend / patch_model), ``stack`` (the token-sharded
block stack) and ``nodes`` (the "Optimize DiT" node).  All compute runs in
``_native/libh3sk_b200.so``; there is no CPU fallback.
"""

__version__ = "0.1.0"
