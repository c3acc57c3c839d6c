"""GEGLU projection kernel on the B200 (npub200_gemm_geglu through the C ABI) against the CPU oracle.

The oracle is the projection on bf16-rounded operands in f32 followed by value * gelu(gate) with the exact GELU,
what SD1.5's feed-forward block computes on the host around the reference's Linear offload. Tolerances are the
GEMM's (max-abs <= 2e-2, relative L2 <= 5e-3 on f32 output; bf16 output within one bf16 ulp of the oracle).
"""
import pytest
import torch

from oracle import geglu_ref
from test_gemm_gpu import _check_bf16, _check_f32

pytestmark = pytest.mark.gpu

# (M, K, n): the SD1.5 GEGLU projections (K = block width, 2n = 8 K) at batch-2 token counts, small-M, ragged.
SHAPES = [(8192, 320, 1280), (2048, 640, 2560), (512, 1280, 5120), (128, 1280, 5120), (154, 320, 1280),
          (77, 640, 2560), (130, 72, 100), (1, 64, 32), (300, 96, 200)]


def _inputs(M, K, n, seed=0, bias=True, bias_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * n, K, generator=g) * 0.05).to(torch.bfloat16)
    b = (torch.randn(2 * n, generator=g) * 0.1).to(bias_dtype) if bias else None
    return x, w, b


def _run(x, w, b, out_dtype=torch.float32, variant=0):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    y = kernels.gemm_geglu(x.to(dev), w.to(dev), b.to(dev) if b is not None else None, out_dtype=out_dtype,
                           variant=variant)
    kernels.check_status(dev)
    return y


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_geglu_shapes(cuda_device, shape):
    M, K, n = shape
    x, w, b = _inputs(M, K, n, seed=M + K + n)
    ref = geglu_ref(x, w, b)
    _check_f32(_run(x, w, b), ref)
    _check_bf16(_run(x, w, b, torch.bfloat16), ref)


@pytest.mark.parametrize("variant", [64, 128, 192, 256, 1128, 1192, 1256])
def test_geglu_every_tile(cuda_device, variant):
    """Each accumulator tile (half value, half gate columns), including 192 whose 96 output columns end in a
    remainder chunk, on a shape with ragged M and n."""
    x, w, b = _inputs(1000, 320, 1000, seed=variant)
    ref = geglu_ref(x, w, b)
    _check_f32(_run(x, w, b, variant=variant), ref)
    _check_bf16(_run(x, w, b, torch.bfloat16, variant=variant), ref)


@pytest.mark.parametrize("bias", ["none", "bf16", "f32"])
def test_geglu_bias_forms(cuda_device, bias):
    x, w, b = _inputs(256, 640, 2560, seed=3, bias=bias != "none",
                      bias_dtype=torch.float32 if bias == "f32" else torch.bfloat16)
    _check_f32(_run(x, w, b), geglu_ref(x, w, b))


def test_geglu_strided_and_unaligned_operands(cuda_device):
    """x as a padded-row view (TMA-addressable), then K = 70 (not a multiple of 8: both operands repacked in the
    workspace with the 2n-row weight)."""
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, w, b = _inputs(500, 320, 640, seed=5)
    buf = torch.zeros(500, 384, dtype=torch.bfloat16)
    buf[:, :320] = x
    y = kernels.gemm_geglu(buf.to(dev)[:, :320], w.to(dev), b.to(dev))
    kernels.check_status(dev)
    _check_f32(y, geglu_ref(x, w, b))
    x, w, b = _inputs(33, 70, 96, seed=6)
    _check_f32(_run(x, w, b), geglu_ref(x, w, b))


def test_geglu_argument_errors(cuda_device):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x = torch.zeros(8, 64, dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError, match="even number of rows"):
        kernels.gemm_geglu(x, torch.zeros(63, 64, dtype=torch.bfloat16, device=dev))
    with pytest.raises(AssertionError, match="K mismatch"):
        kernels.gemm_geglu(x, torch.zeros(64, 32, dtype=torch.bfloat16, device=dev))
    with pytest.raises(RuntimeError, match="GEGLU"):
        kernels.gemm_geglu(x, torch.zeros(64, 64, dtype=torch.bfloat16, device=dev), variant=96)


def test_geglu_matches_projection_then_gating(cuda_device):
    """The fused kernel against this library's own two-step path (GEMM to 2n columns, then torch gating on the
    GPU): same arithmetic, so they agree to f32 rounding of the gating."""
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, w, b = _inputs(4096, 320, 1280, seed=9)
    xd, wd, bd = x.to(dev), w.to(dev), b.to(dev)
    y2 = kernels.gemm(xd, wd, bd)
    a, gate = y2.chunk(2, dim=-1)
    two_step = a * torch.nn.functional.gelu(gate)
    fused = kernels.gemm_geglu(xd, wd, bd)
    kernels.check_status(dev)
    assert float((fused - two_step).abs().max()) < 1e-4
