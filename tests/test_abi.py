"""The C ABI library and the torch op library load and expose what the
header declares (no GPU needed: nothing here launches a kernel)."""
import ctypes
import os
import re

import pytest
import torch

from paraconv2d_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "paraconv2d.h")

REF_FORWARD_SCHEMA = ("ptparaconv2d::forward(Tensor input, Tensor parameters, float doublefactor, "
                      "Tensor kernel_size_tensor, Tensor strides_tensor, Tensor dilation_rate_tensor) -> Tensor[]")
REF_BACKWARD_SCHEMA = ("ptparaconv2d::backward(Tensor grad, Tensor input, Tensor parameters, Tensor hsum, "
                       "float doublefactor, Tensor kernel_size_tensor, Tensor strides_tensor, "
                       "Tensor dilation_rate_tensor, bool skip_input_grad) -> Tensor[]")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(pc2d_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("pc2d_forward", "pc2d_backward", "pc2d_forward_workspace_size", "pc2d_backward_workspace_size"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.KERNEL_LIB)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_host_only_entry_points():
    lib = _lib.cabi()
    assert lib.pc2d_abi_version() == 1
    assert lib.pc2d_out_size(34, 3, 1, 1) == 32
    assert lib.pc2d_out_size(230, 7, 2, 1) == 112
    assert lib.pc2d_infer_m(73856, 64, 3, 3) == 64
    assert lib.pc2d_infer_m(73857, 64, 3, 3) == -1
    assert lib.pc2d_status_string(0) == b"PC2D_OK"
    prev = lib.pc2d_set_algo(_lib.PC2D_ALGO_SIMT)
    assert lib.pc2d_get_algo() == _lib.PC2D_ALGO_SIMT
    lib.pc2d_set_algo(prev)
    assert lib.pc2d_set_algo(7) == -1


@pytest.mark.parametrize("args,code", [
    # dtype 5 is not a pc2d_dtype
    (dict(dtype=5), _lib.PC2D_ERR_INVALID_ARGUMENT),
    # even kernel sizes read outside the window in the reference
    (dict(k0=2, k1=2), _lib.PC2D_ERR_UNSUPPORTED),
    # input smaller than the kernel
    (dict(H=2, W=2), _lib.PC2D_ERR_INVALID_ARGUMENT),
    (dict(s0=0), _lib.PC2D_ERR_INVALID_ARGUMENT),
])
def test_invalid_arguments_rejected_before_any_launch(args, code):
    lib = _lib.cabi()
    a = dict(dtype=0, k0=3, k1=3, s0=1, s1=1, d0=1, d1=1, n=1, C=3, H=8, W=8, m=2)
    a.update(args)
    st = lib.pc2d_forward(a["dtype"], None, None, 1.0, a["k0"], a["k1"], a["s0"], a["s1"], a["d0"], a["d1"], a["n"],
                          a["C"], a["H"], a["W"], a["m"], None, None, None, 0, None)
    assert st == code
    assert lib.pc2d_last_error() != b""


def test_torch_op_schema_identical_to_reference():
    _lib.load_op_library()
    assert str(torch.ops.ptparaconv2d.forward.default._schema) == REF_FORWARD_SCHEMA
    assert str(torch.ops.ptparaconv2d.backward.default._schema) == REF_BACKWARD_SCHEMA


def test_op_has_no_cpu_fallback():
    _lib.load_op_library()
    x = torch.zeros(1, 3, 5, 5)
    pars = torch.zeros(2 * (27 + 1))
    it = torch.tensor([3, 3], dtype=torch.int)
    one = torch.tensor([1, 1], dtype=torch.int)
    with pytest.raises(NotImplementedError):
        torch.ops.ptparaconv2d.forward(x, pars, 1.0, it, one, one)


def test_module_ops_registered_beside_the_reference_schema():
    """The module mirror's two fused steps live in their own namespace; the
    reference's namespace keeps exactly its two ops."""
    _lib.load_op_library()
    assert str(torch.ops.paraconv2d_b200.pad_scale.default._schema).startswith(
        "paraconv2d_b200::pad_scale(Tensor input, int[] padding, float scale) -> Tensor")
    assert "need_input_grad" in str(torch.ops.paraconv2d_b200.backward_interior.default._schema)
    assert str(torch.ops.ptparaconv2d.forward.default._schema) == REF_FORWARD_SCHEMA
