"""B200 (sm_100a) implementation of the ParaConv2d paraboloid convolution.

Drop-in for GeoND-tech/ParaConv2d: ``torch.ops.ptparaconv2d.forward/backward``
(same schema, registered from C++ by ``libptparaconv2d.so``) and the
``ptparaconv2d`` module mirror (``ParaConv2d``, ``ParaConv2dFunction``,
``spotlightinit``, ``pnnconvert``).  The kernels live in ``libpc2d_sm100.so``
behind the C ABI of ``include/paraconv2d.h``.

Importing this package loads the op library; a missing library raises.
"""
from ._lib import (  # noqa: F401
    PC2D_ALGO_AUTO,
    PC2D_ALGO_SIMT,
    PC2D_ALGO_TC,
    cabi,
    load_op_library,
    set_algo,
)
from . import ptparaconv2d  # noqa: F401
from .ptparaconv2d import ParaConv2d, ParaConv2dFunction, pnnconvert, spotlightinit  # noqa: F401

__all__ = ["ParaConv2d", "ParaConv2dFunction", "spotlightinit", "pnnconvert", "ptparaconv2d", "cabi", "set_algo",
           "load_op_library", "PC2D_ALGO_AUTO", "PC2D_ALGO_SIMT", "PC2D_ALGO_TC"]
