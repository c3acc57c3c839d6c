"""LayerNorm over the last dimension (npub200_layer_norm through the C ABI) against the CPU oracle (F.layer_norm
in f32 on bf16-rounded input): bf16 output within one bf16 ulp of the oracle."""
import pytest
import torch

from oracle import layer_norm_ref
from test_gemm_gpu import _check_bf16

pytestmark = pytest.mark.gpu

# (rows, C): the SD1.5 transformer widths at batch 2 (64x64, 32x32, 16x16, 8x8 latents) and batch 16, a width that
# leaves lanes without a chunk (C / 8 not a multiple of 32), the largest supported width, and single rows.
SHAPES = [(8192, 320), (2048, 640), (512, 1280), (128, 1280), (65536, 320), (3, 8), (7, 200), (100, 2048), (1, 768)]


def _inputs(rows, c, seed=0, param_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(rows, c, generator=g) * 3.0 + 1.0).to(torch.bfloat16)
    gamma = (1.0 + 0.1 * torch.randn(c, generator=g)).to(param_dtype)
    beta = (0.1 * torch.randn(c, generator=g)).to(param_dtype)
    return x, gamma, beta


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("param_dtype", [torch.bfloat16, torch.float32], ids=["bf16", "f32"])
def test_layer_norm(cuda_device, shape, param_dtype):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, gamma, beta = _inputs(*shape, seed=sum(shape), param_dtype=param_dtype)
    y = kernels.layer_norm(x.to(dev), gamma.to(dev), beta.to(dev), eps=1e-5)
    kernels.check_status(dev)
    _check_bf16(y, layer_norm_ref(x, gamma, beta, eps=1e-5))


def test_layer_norm_3d_strided_rows_and_determinism(cuda_device):
    """A [B, S, C] activation, a 2-D view with a padded row stride, and bitwise-equal repeats."""
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, gamma, beta = _inputs(2 * 1024, 640, seed=5)
    x3 = x.reshape(2, 1024, 640).to(dev)
    y1 = kernels.layer_norm(x3, gamma.to(dev), beta.to(dev), eps=1e-6)
    y2 = kernels.layer_norm(x3, gamma.to(dev), beta.to(dev), eps=1e-6)
    kernels.check_status(dev)
    assert y1.shape == (2, 1024, 640) and torch.equal(y1, y2)
    _check_bf16(y1.reshape(-1, 640), layer_norm_ref(x, gamma, beta, eps=1e-6))
    wide = torch.zeros(300, 648, dtype=torch.bfloat16, device=dev)
    wide[:, :640] = x[:300].to(dev)
    y = kernels.layer_norm(wide[:, :640], gamma.to(dev), beta.to(dev))
    _check_bf16(y, layer_norm_ref(x[:300], gamma, beta))


def test_layer_norm_unsupported_widths_are_refused(cuda_device):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, gamma, beta = _inputs(4, 4100)
    with pytest.raises(RuntimeError, match="at most 2048"):
        kernels.layer_norm(x.to(dev)[:, :4096].contiguous(), gamma[:4096].to(dev), beta[:4096].to(dev))
    x, gamma, beta = _inputs(4, 12)
    with pytest.raises(RuntimeError, match="multiples of 8"):
        kernels.layer_norm(x.to(dev), gamma.to(dev), beta.to(dev))
