"""ORACLE -- test infrastructure only.

CPU checkers for the ParaConv2d paraboloid convolution:

* ``pc2d_oracle.c``: a plain-C restatement of the reference CPU path
  (GeoND-tech/ParaConv2d ``paraconv2d.cc:70-239``), built on demand into
  ``oracle/_build/libpc2d_oracle.so`` and called through ctypes;
* ``_ref/libptparaconv2d_ref.so``: the reference op itself, compiled from its
  own sources by ``oracle/build_ref.sh`` (only where those sources exist), and
  registered as ``torch.ops.ptparaconv2d_ref``.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this package.  The product path never does.
"""
from .pc2d_oracle import (  # noqa: F401
    build_oracle,
    forward,
    backward,
    out_size,
    load_reference,
    reference_available,
    ref_forward,
    ref_backward,
)
