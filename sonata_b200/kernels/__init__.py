"""B200 drop-ins for the reference's ``kernels`` package.

``sonata_b200.kernels.gemv``, ``.bmm``, ``.fused_snake_conv`` and ``.patch``
keep the call signatures of the reference modules of the same names.
"""
