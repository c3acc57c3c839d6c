"""The C ABI library: it builds for sm_100a, loads without a GPU, and exports every entry point of
include/npu_b200.h (no compute calls here: those need a B200 and live in the -m gpu tests)."""
import ctypes
import os
import re

from npu_ai_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"^\s*(?:int|const char\*|void)\s+\**(npub200_\w+)\s*\(", src, re.M))
    return names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    declared = _declared()
    assert len(declared) >= 12, declared
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, f"declared in include/*.h but not exported: {missing}"


def test_binding_covers_header():
    assert _declared() == set(_lib.exported_symbols())
    assert set(_lib.exported_symbols()) <= _declared()


def test_version_and_error_without_gpu():
    lib = _lib.load()
    assert lib.npub200_version() >= 100
    assert isinstance(_lib.last_error(), str)


def test_error_mapping():
    import pytest
    with pytest.raises(ValueError):
        _lib.check(_lib.EINVAL, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ECUDA, "x")
    _lib.check(_lib.OK, "x")


def test_torch_operators_register_over_the_c_abi():
    """libnpub200_torch.so registers npub200::gemm and npub200::attention with the torch dispatcher (a CUDA kernel
    only: CPU tensors are refused, there is no CPU path)."""
    import pytest
    import torch
    ops = _lib.torch_ops()
    assert ops is not None, "libnpub200_torch.so is not built"
    g = str(ops.gemm.default._schema)
    a = str(ops.attention.default._schema)
    assert g.startswith("npub200::gemm(Tensor x, Tensor w, Tensor? bias=None, Tensor? out=None, int variant=0")
    assert a.startswith("npub200::attention(Tensor q, Tensor k, Tensor v, Tensor? out, int B, int H, int Sq, int Skv, "
                        "int d, int q_row_stride, int kv_row_stride, int o_row_stride, bool head_major_in, "
                        "bool head_major_out, float scale, int variant")
    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        ops.gemm(x, torch.zeros(16, 8, dtype=torch.bfloat16))
