"""GroupNorm (+ SiLU) over NHWC activations (npub200_group_norm through the C ABI) against the CPU oracle
(F.group_norm in f32 on bf16-rounded input): bf16 output within one bf16 ulp of the oracle."""
import pytest
import torch

from oracle import group_norm_ref
from test_gemm_gpu import _check_bf16

pytestmark = pytest.mark.gpu

# (n, h, w, c): the SD1.5 ResBlock widths (group sizes 10, 20, 30, 40, 60, 80 channels) at batch 2 (below 4M values:
# two launches) and 16 (the one-launch cooperative form), 4608 channels (past the cooperative form's 4096), and a
# six-pixel image.
SHAPES = [(2, 64, 64, 320), (2, 32, 32, 640), (2, 8, 8, 1280), (2, 16, 16, 1920), (1, 8, 8, 960), (16, 32, 32, 640),
          (2, 16, 16, 2560), (16, 64, 64, 320), (1, 8, 8, 4608), (1, 2, 3, 320)]
# Debug bits forcing each form on every shape (the cooperative one where it takes the shape).
FORMS = {"auto": 0, "two_launch": 2, "cooperative": 4}


def _inputs(n, h, w, c, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(n, h, w, c, generator=g) * 2.0 + 0.5).to(torch.bfloat16)
    gamma = 1.0 + 0.1 * torch.randn(c, generator=g)
    beta = 0.1 * torch.randn(c, generator=g)
    return x, gamma, beta


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("silu", [False, True])
@pytest.mark.parametrize("form", list(FORMS))
def test_group_norm(cuda_device, shape, silu, form):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, gamma, beta = _inputs(*shape, seed=sum(shape))
    kernels.set_debug_flags(FORMS[form])
    try:
        y = kernels.group_norm(x.to(dev), 32, gamma, beta, eps=1e-5, silu=silu)
    finally:
        kernels.set_debug_flags(0)
    kernels.check_status(dev)
    _check_bf16(y, group_norm_ref(x, 32, gamma, beta, eps=1e-5, silu=silu))


@pytest.mark.parametrize("groups,c", [(6, 48), (3, 24), (1, 8), (16, 1280)])
@pytest.mark.parametrize("form", list(FORMS))
def test_group_norm_other_group_counts(cuda_device, groups, c, form):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, gamma, beta = _inputs(2, 5, 7, c, seed=c + groups)
    kernels.set_debug_flags(FORMS[form])
    try:
        y = kernels.group_norm(x.to(dev), groups, gamma, beta, eps=1e-5, silu=True)
    finally:
        kernels.set_debug_flags(0)
    kernels.check_status(dev)
    _check_bf16(y, group_norm_ref(x, groups, gamma, beta, eps=1e-5, silu=True))


@pytest.mark.parametrize("shape", [(2, 32, 32, 640), (16, 64, 64, 320)], ids=lambda s: "x".join(map(str, s)))
def test_group_norm_in_place_and_eps(cuda_device, shape):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, gamma, beta = _inputs(*shape, seed=4)
    xd = x.to(dev)
    kernels.group_norm(xd, 32, gamma, beta, eps=1e-6, silu=True, out=xd)
    kernels.check_status(dev)
    _check_bf16(xd, group_norm_ref(x, 32, gamma, beta, eps=1e-6, silu=True))


@pytest.mark.parametrize("shape", [(2, 64, 64, 320), (16, 64, 64, 320)], ids=lambda s: "x".join(map(str, s)))
def test_group_norm_is_deterministic(cuda_device, shape):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, gamma, beta = _inputs(*shape, seed=5)
    xd = x.to(dev)
    a = kernels.group_norm(xd, 32, gamma, beta, silu=True)
    b = kernels.group_norm(xd, 32, gamma, beta, silu=True)
    assert torch.equal(a, b)
