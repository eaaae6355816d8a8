"""B200-native (sm_100a) complex-valued Conv2d for PyTorch.

Drop-in for the ``complex_conv2d`` package of cutlass-complex-conv
(``complex_conv2d/__init__.py:3-5``): the public object is ``ComplexConv2d``.
"""

from .modules import ComplexConv2d

__all__ = ["ComplexConv2d"]
