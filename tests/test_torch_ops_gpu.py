"""The torch operators torch.ops.npub200.gemm / .attention (libnpub200_torch.so, TORCH_LIBRARY over the C ABI) on
the B200 against the CPU oracle: they run on torch's current stream, take torch tensors and raise ValueError for
requests the kernels refuse (the reference's NpuProgram.submit_gemm / submit_attn boundary,
npu/xdna1_program.py:441-473). Tolerances as elsewhere: GEMM max-abs <= 2e-2 and relative L2 <= 5e-3 on the f32
output, attention max-abs <= 2e-2."""
import pytest
import torch

from oracle import attention_ref, linear_ref, rel_l2_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from npu_ai_b200 import _lib
    o = _lib.torch_ops()
    assert o is not None, "libnpub200_torch.so is not built"
    return o


@pytest.mark.parametrize("MKN", [(4096, 320, 320), (77, 768, 1280), (100, 100, 100), (8192, 1280, 10240)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_op(cuda_device, ops, MKN, out_dtype):
    M, K, N = MKN
    g = torch.Generator().manual_seed(M + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    ref = linear_ref(x, w, b)
    side = torch.cuda.Stream(cuda_device)
    with torch.cuda.stream(side):   # the op launches on the current stream
        y = ops.gemm(x.to(cuda_device), w.to(cuda_device), b.to(cuda_device), out_dtype=out_dtype)
    side.synchronize()
    assert y.dtype == out_dtype and y.shape == (M, N)
    y = y.float().cpu()
    if out_dtype == torch.float32:
        assert float((y - ref).abs().max()) <= 2e-2 and rel_l2_err(y, ref) <= 5e-3
    else:  # one bf16 ulp of the rounded oracle (plus a small absolute floor)
        ulp = torch.finfo(torch.bfloat16).eps * ref.abs().clamp_min(1e-30)
        assert bool(((y - ref).abs() <= 2 * ulp + 1e-4).all())


def test_gemm_op_out_and_residual(cuda_device, ops):
    M, K, N = 512, 640, 640
    g = torch.Generator().manual_seed(3)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).to(cuda_device)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    r = torch.randn(M, N, generator=g).to(torch.bfloat16).to(cuda_device)
    out = torch.empty(M, N, device=cuda_device)
    y = ops.gemm(x, w, None, out, 0, None, 0, r)
    torch.cuda.synchronize()
    assert y.data_ptr() == out.data_ptr()
    ref = linear_ref(x.cpu(), w.cpu()) + r.cpu().float()
    assert float((out.cpu() - ref).abs().max()) <= 2e-2


def test_gemm_op_errors(cuda_device, ops):
    x = torch.zeros(4, 8, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError, match="K mismatch"):
        ops.gemm(x, torch.zeros(16, 16, dtype=torch.bfloat16, device=cuda_device))
    with pytest.raises(ValueError, match="bf16"):
        ops.gemm(x.float(), torch.zeros(16, 8, dtype=torch.bfloat16, device=cuda_device))


@pytest.mark.parametrize("shape,head_major", [((2, 8, 4096, 4096, 40), False), ((2, 8, 4096, 77, 40), False),
                                              ((2, 8, 1024, 1024, 80), True), ((2, 8, 256, 256, 160), False)])
def test_attention_op(cuda_device, ops, shape, head_major):
    B, H, Sq, Skv, D = shape
    g = torch.Generator().manual_seed(D)
    q = torch.randn(B, Sq, H * D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Skv, H * D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Skv, H * D, generator=g).to(torch.bfloat16)
    ref = attention_ref(q, k, v, H)
    if head_major:
        q, k, v = (t.view(B, t.shape[1], H, D).transpose(1, 2).contiguous() for t in (q, k, v))
        ref = ref.view(B, Sq, H, D).transpose(1, 2)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    rs = (D, D, D) if head_major else (H * D, H * D, H * D)
    o = ops.attention(qd, kd, vd, None, B, H, Sq, Skv, D, *rs, head_major, head_major, D ** -0.5, 0)
    torch.cuda.synchronize()
    assert o.dtype == torch.float32
    assert float((o.cpu() - ref).abs().max()) <= 2e-2


def test_attention_op_checks_declared_strides(cuda_device, ops):
    q = torch.zeros(1, 64, 80, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError, match="row stride"):
        ops.attention(q, q, q, None, 1, 2, 64, 64, 40, 96, 0, 0, False, False, 0.0, 0)
