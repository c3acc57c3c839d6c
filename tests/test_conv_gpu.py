"""3x3 convolution (implicit GEMM, npub200_conv3x3 through the C ABI) against the CPU oracle.

The oracle is F.conv2d in f32 on bf16-rounded operands (plus the bias, per-image bias and residual the ResBlock
fusion adds). Tolerances are the GEMM's: max-abs <= 2e-2 and relative L2 <= 5e-3 on f32 output, bf16 output within
one bf16 ulp of the oracle.
"""
import pytest
import torch

from oracle import conv3x3_ref
from test_gemm_gpu import _check_bf16, _check_f32

pytestmark = pytest.mark.gpu

# (n, h, w, cin, cout): the SD1.5 UNet's 3x3 convolutions at batch 2 (64x64 latent), the 128x128 level, channel
# changes, and shapes whose last tile is ragged (odd image counts with two images per tile, cout not a tile multiple).
SHAPES = [(2, 64, 64, 320, 320), (2, 32, 32, 640, 640), (2, 16, 16, 1280, 1280), (2, 8, 8, 1280, 1280),
          (2, 32, 32, 320, 640), (2, 16, 16, 1920, 1280), (1, 128, 128, 320, 320), (3, 8, 8, 64, 96),
          (1, 16, 16, 128, 100), (5, 32, 32, 64, 64)]


def _inputs(n, h, w, cin, cout, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, h, w, cin, generator=g).to(torch.bfloat16)
    wt = (torch.randn(cout, cin, 3, 3, generator=g) / (9 * cin) ** 0.5).to(torch.bfloat16)
    b = (torch.randn(cout, generator=g) * 0.1).to(torch.float32)
    return x, wt, b


def _run(x, wt, b=None, residual=None, out_dtype=torch.float32, variant=0):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    y = kernels.conv3x3(x.to(dev), kernels.pack_conv3x3_weight(wt.to(dev)), b.to(dev) if b is not None else None,
                        residual.to(dev) if residual is not None else None, out_dtype=out_dtype, variant=variant)
    kernels.check_status(dev)
    return y


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_conv3x3_shapes(cuda_device, shape):
    n, h, w, cin, cout = shape
    x, wt, b = _inputs(n, h, w, cin, cout, seed=sum(shape))
    ref = conv3x3_ref(x, wt, b)
    _check_f32(_run(x, wt, b), ref)
    _check_bf16(_run(x, wt, b, out_dtype=torch.bfloat16), ref)


@pytest.mark.parametrize("variant", [64, 96, 128, 160, 192, 256, 1128, 1192, 1256])
def test_conv3x3_every_tile(cuda_device, variant):
    x, wt, b = _inputs(2, 16, 16, 320, 640, seed=variant)
    _check_f32(_run(x, wt, b, variant=variant), conv3x3_ref(x, wt, b))


@pytest.mark.parametrize("variant", [1128, 1256])
def test_conv3x3_pair_tiles_ragged(cuda_device, variant):
    """256-pixel tiles on a two-CTA cluster where the last tile's second CTA starts past the last image (3 images
    of 8x8 = 192 pixels) and a per-image bias row plus a residual in the epilogue."""
    x, wt, b = _inputs(3, 8, 8, 64, 96, seed=variant)
    g = torch.Generator().manual_seed(variant)
    b2 = b[None, :] + torch.randn(3, 96, generator=g)
    res = torch.randn(3, 8, 8, 96, generator=g).to(torch.bfloat16)
    _check_f32(_run(x, wt, b2, res, variant=variant), conv3x3_ref(x, wt, b2, res))
    _check_f32(_run(x, wt, b, variant=variant), conv3x3_ref(x, wt, b))


@pytest.mark.parametrize("shape", [(2, 32, 32, 640, 640), (2, 8, 8, 1280, 1280)], ids=["32x32", "8x8_splitK"])
def test_conv3x3_resblock_epilogue(cuda_device, shape):
    """The ResBlock fusions: a bias row per image (conv bias + time embedding) and a residual added after it, also
    on a small image where K is split across CTAs and the reducing split applies them."""
    n, h, w, cin, cout = shape
    x, wt, b = _inputs(n, h, w, cin, cout, seed=7)
    g = torch.Generator().manual_seed(8)
    b2 = b[None, :] + torch.randn(n, cout, generator=g)
    res = torch.randn(n, h, w, cout, generator=g).to(torch.bfloat16)
    ref = conv3x3_ref(x, wt, b2, res)
    _check_f32(_run(x, wt, b2, res), ref)
    _check_bf16(_run(x, wt, b2, res, out_dtype=torch.bfloat16), ref)
    # bf16 per-image bias and no bias at all
    _check_f32(_run(x, wt, b2.to(torch.bfloat16)), conv3x3_ref(x, wt, b2.to(torch.bfloat16)))
    _check_f32(_run(x, wt, None, res), conv3x3_ref(x, wt, None, res))


def test_conv3x3_channels_last_view_in_and_out(cuda_device):
    """An NCHW channels_last activation goes in as its NHWC view, the output is a strided NHWC view of a
    channels_last tensor: no copies on either side."""
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, wt, b = _inputs(2, 16, 16, 320, 320, seed=3)
    x_cl = x.permute(0, 3, 1, 2).contiguous(memory_format=torch.channels_last).to(dev)
    out_cl = torch.empty(2, 320, 16, 16, device=dev, dtype=torch.bfloat16, memory_format=torch.channels_last)
    kernels.conv3x3(x_cl.permute(0, 2, 3, 1), kernels.pack_conv3x3_weight(wt.to(dev)), b.to(dev),
                    out=out_cl.permute(0, 2, 3, 1))
    kernels.check_status(dev)
    _check_bf16(out_cl.permute(0, 2, 3, 1), conv3x3_ref(x, wt, b))


def test_conv3x3_unsupported_shapes_are_refused(cuda_device):
    with pytest.raises(RuntimeError, match="multiples of 64"):
        _run(*_inputs(1, 8, 8, 4, 64)[:2])
    with pytest.raises(RuntimeError, match="width dividing 128"):
        _run(*_inputs(1, 12, 12, 64, 64)[:2])
