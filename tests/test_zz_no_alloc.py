"""The GEMM entry point that allocates nothing (npub200_gemm_noalloc), through the C ABI.

It exists for callers that cannot allocate device memory — a host whose device memory belongs to its own pool
manager and must not grow during a request, an FFI binding that only holds the pointers it was given, code that must
not call cudaMalloc because it synchronises the device. The only scratch a GEMM needs is a repacked copy of an operand
TMA cannot address; here that copy goes to one fixed device array per GPU shared by every call. So each case runs
two calls in a row with a call of another shape in between (each call finds the previous one's leftovers in the
array) and checks both against the regular entry point and against the CPU oracle, with the GEMM tolerance used
throughout (max-abs <= 2e-2, relative L2 <= 5e-3). The cases use the array for a repacked x (K % 8 != 0; a row stride
off the 8-element grid), a repacked W only, and neither; an oversize request is refused.
This file is collected last so that a failure here never hides the other tests.
"""
import ctypes

import pytest
import torch

from oracle import linear_ref, rel_l2_err

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


def _scratch_need(x, w):
    from npu_ai_b200 import _lib
    nbytes = ctypes.c_size_t(0)
    _lib.call("npub200_gemm_workspace_size", ctypes.c_void_p(x.data_ptr()), x.stride(0), x.shape[0], x.shape[1],
              ctypes.c_void_p(w.data_ptr()), w.stride(0), w.shape[0], 0, ctypes.byref(nbytes))
    return nbytes.value


def _operands(M, K, N, device, x_pad=0, w_pad=0, seed=0):
    """bf16 x [M, K] and W [N, K], as views of wider buffers when a pad is given (row strides K + pad)."""
    g = torch.Generator().manual_seed(seed + K + N)
    xf = torch.randn(M, K + x_pad, generator=g).to(torch.bfloat16).to(device)
    wf = (torch.randn(N, K + w_pad, generator=g) * 0.02).to(torch.bfloat16).to(device)
    b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16).to(device)
    return xf[:, :K], wf[:, :K], b


CASES = {
    "k_unaligned": dict(MKN=(100, 100, 100)),           # K % 8 != 0: x and W repacked with K padded to 104
    "k_unaligned_sd15": dict(MKN=(77, 770, 320)),       # same, small M and a longer K
    "x_strided": dict(MKN=(300, 320, 640), x_pad=3),    # ldx = 323: only x repacked
    "w_strided": dict(MKN=(256, 640, 640), w_pad=5),    # ldw = 645: only W repacked
    "no_scratch": dict(MKN=(4096, 320, 320)),           # TMA-addressable: the array is not touched
}


def _check(y, ref_gpu, ref_cpu):
    assert torch.isfinite(y).all()
    for ref in (ref_gpu, ref_cpu):
        assert float((y - ref).abs().max()) <= 2e-2
        assert rel_l2_err(y, ref) <= 5e-3


@pytest.mark.parametrize("case", list(CASES), ids=list(CASES))
def test_noalloc_matches_regular_entry_point_and_oracle(cuda_device, case):
    from npu_ai_b200 import kernels
    c = CASES[case]
    M, K, N = c["MKN"]
    x, w, b = _operands(M, K, N, cuda_device, c.get("x_pad", 0), c.get("w_pad", 0))
    if case != "no_scratch":
        assert _scratch_need(x, w) > 0, "this case must use the scratch array"
    ref_gpu = kernels.gemm(x, w, b, out_dtype=torch.float32)
    kernels.check_status(cuda_device)
    ref_gpu = ref_gpu.float().cpu()
    ref_cpu = linear_ref(x.cpu(), w.cpu(), b.cpu())
    # a call of another shape between the two, which leaves its own repacked operands in the array
    ox, ow, ob = _operands(64, 136 + 1, 200, cuda_device, seed=7)
    for i in range(2):
        out = torch.full((M, N), float("nan"), device=cuda_device)
        _noalloc(x, w, b, out)
        kernels.check_status(cuda_device)
        _check(out.cpu(), ref_gpu, ref_cpu)
        if i == 0:
            other = torch.full((64, 200), float("nan"), device=cuda_device)
            _noalloc(ox, ow, ob, other)
            kernels.check_status(cuda_device)
            _check(other.cpu(), kernels.gemm(ox, ow, ob, out_dtype=torch.float32).float().cpu(),
                   linear_ref(ox.cpu(), ow.cpu(), ob.cpu()))


def test_noalloc_rejects_oversize_scratch(cuda_device):
    """An unaligned K forces repacking; at this size the repacked x alone (33 MB) exceeds the fixed array."""
    M, K, N = 16384, 1001, 64
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=cuda_device)
    w = torch.zeros(N, K, dtype=torch.bfloat16, device=cuda_device)
    b = torch.zeros(N, dtype=torch.bfloat16, device=cuda_device)
    out = torch.empty(M, N, device=cuda_device)
    assert _scratch_need(x, w) > 3 * 8 * 1024 * 1024  # far above NPUB200_NOALLOC_SCRATCH_BYTES (8 MiB)
    with pytest.raises(ValueError, match="scratch"):
        _noalloc(x, w, b, out)
