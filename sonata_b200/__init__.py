"""sonata_b200: B200-native (sm_100a) hot paths of Zonos-hybrid streaming inference.

Hand-written CUDA kernels behind the C ABI in ``include/sonata_b200.h``
(``libsonata_b200.so``), with Python wrappers that keep the reference's
``kernels.gemv`` / ``kernels.bmm`` / ``kernels.fused_snake_conv`` /
``kernels.patch`` signatures under ``sonata_b200.kernels``.
"""
__version__ = "0.1.0"
