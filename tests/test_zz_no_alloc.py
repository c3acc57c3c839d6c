"""The GEMM entry point that allocates nothing (npub200_gemm_noalloc), through the C ABI.

It exists for callers that cannot allocate device memory — a host whose device memory belongs to its own pool
manager and must not grow during a request, an FFI binding that only holds the pointers it was given, code that must
not call cudaMalloc because it synchronises the device. Its scratch is one fixed device array per GPU shared by every
call, so this checks two calls in a row (the second finds the first one's leftovers) against the regular entry
point's output with the GEMM tolerance used throughout (max-abs <= 2e-2, relative L2 <= 5e-3), on shapes that use
the scratch for split-K partials and for repacked operands, and that an oversize request is refused.
This file is collected last so that a failure here never hides the other tests.
"""
import ctypes

import pytest
import torch

from oracle import rel_l2_err

pytestmark = pytest.mark.gpu


def _noalloc(x, w, b, out):
    from npu_ai_b200 import _lib
    lib = _lib.load()
    rc = lib.npub200_gemm_noalloc(
        ctypes.c_void_p(x.data_ptr()), x.stride(0), x.shape[0], x.shape[1], ctypes.c_void_p(w.data_ptr()),
        w.stride(0), w.shape[0], ctypes.c_void_p(b.data_ptr()), _lib.DTYPE_BF16, ctypes.c_void_p(out.data_ptr()),
        out.stride(0), _lib.DTYPE_F32, 0, ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    _lib.check(rc, "npub200_gemm_noalloc")
    return out


@pytest.mark.parametrize("MKN", [(77, 5120, 1280), (154, 2560, 640), (100, 100, 100), (4096, 320, 320)],
                         ids=["split_k", "split_k_2", "repacked", "no_scratch"])
def test_noalloc_matches_regular_entry_point_twice(cuda_device, MKN):
    from npu_ai_b200 import kernels
    M, K, N = MKN
    g = torch.Generator().manual_seed(K + N)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(cuda_device)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16).to(cuda_device)
    ref = kernels.gemm(x, w, b, out_dtype=torch.float32)
    kernels.check_status(cuda_device)
    ref = ref.float().cpu()
    for _ in range(2):
        out = torch.full((M, N), float("nan"), device=cuda_device)
        _noalloc(x, w, b, out)
        kernels.check_status(cuda_device)
        y = out.cpu()
        assert torch.isfinite(y).all()
        assert float((y - ref).abs().max()) <= 2e-2
        assert rel_l2_err(y, ref) <= 5e-3


def test_noalloc_rejects_oversize_scratch(cuda_device):
    """An unaligned K forces repacking; at this size the repacked operands exceed the fixed array."""
    M, K, N = 4096, 1001, 64
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=cuda_device)
    w = torch.zeros(N, K, dtype=torch.bfloat16, device=cuda_device)
    b = torch.zeros(N, dtype=torch.bfloat16, device=cuda_device)
    out = torch.empty(M, N, device=cuda_device)
    with pytest.raises(ValueError, match="scratch"):
        _noalloc(x, w, b, out)
