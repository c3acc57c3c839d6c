"""NHWC nearest 2x upsampling and channel concatenation (npub200_upsample_nearest2x / npub200_concat_channels through
the C ABI) against the CPU oracle (F.interpolate / torch.cat on the host). Both are copies, so parity is bit-exact,
in bf16 and f16, for the SD1.5 decoder's shapes at batch 2 and 16, ragged and single-pixel edge cases."""
import ctypes

import pytest
import torch

from oracle import concat_channels_ref, upsample_nearest2x_ref

pytestmark = pytest.mark.gpu

# (n, c, h, w): the decoder's three Upsample inputs at batch 2 and 16 (64x64 latent), a 128x128-latent one, odd
# sizes and a single pixel with the narrowest legal channel count.
UPSAMPLE = [(2, 1280, 8, 8), (2, 1280, 16, 16), (2, 640, 32, 32), (16, 640, 32, 32), (2, 640, 64, 64),
            (3, 24, 5, 7), (1, 8, 1, 1)]
# (n, ca, cb, h, w): the decoder's skip concatenations at batch 2 and 16, and ragged cases.
CONCAT = [(2, 1280, 1280, 8, 8), (2, 1280, 640, 16, 16), (2, 640, 320, 64, 64), (16, 320, 320, 64, 64),
          (16, 1280, 640, 32, 32), (3, 8, 24, 5, 7), (1, 16, 8, 1, 1)]


def _nhwc(shape, dtype, seed, dev):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g).to(dtype)
    return x, x.to(dev).contiguous(memory_format=torch.channels_last)


@pytest.mark.parametrize("shape", UPSAMPLE, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_upsample_nearest2x_exact(cuda_device, shape, dtype):
    from npu_ai_b200 import kernels
    x, xd = _nhwc(shape, dtype, sum(shape), cuda_device)
    y = kernels.upsample_nearest2x(xd)
    kernels.check_status(cuda_device)
    assert y.is_contiguous(memory_format=torch.channels_last)
    assert torch.equal(y.cpu(), upsample_nearest2x_ref(x))


@pytest.mark.parametrize("shape", CONCAT, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_concat_channels_exact(cuda_device, shape, dtype):
    from npu_ai_b200 import kernels
    n, ca, cb, h, w = shape
    a, ad = _nhwc((n, ca, h, w), dtype, 1 + sum(shape), cuda_device)
    b, bd = _nhwc((n, cb, h, w), dtype, 2 + sum(shape), cuda_device)
    y = kernels.concat_channels(ad, bd)
    kernels.check_status(cuda_device)
    assert y.is_contiguous(memory_format=torch.channels_last)
    assert torch.equal(y.cpu(), concat_channels_ref(a, b))


def test_concat_channels_strided_rows_through_the_c_abi(cuda_device):
    """Row strides wider than the channel counts (pixels of larger buffers) leave the gaps untouched."""
    from npu_ai_b200 import _lib
    P, ca, cb = 1000, 40, 24
    g = torch.Generator().manual_seed(3)
    a = torch.randn(P, 64, generator=g).to(torch.bfloat16).to(cuda_device)
    b = torch.randn(P, 32, generator=g).to(torch.bfloat16).to(cuda_device)
    out = torch.full((P, 80), 7.0, dtype=torch.bfloat16, device=cuda_device)
    _lib.call("npub200_concat_channels", ctypes.c_void_p(a.data_ptr()), 64, ca, ctypes.c_void_p(b.data_ptr()), 32,
              cb, P, ctypes.c_void_p(out.data_ptr()), 80, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ref = torch.cat([a[:, :ca], b[:, :cb], torch.full((P, 80 - ca - cb), 7.0, dtype=torch.bfloat16,
                                                      device=cuda_device)], dim=1)
    assert torch.equal(out, ref)


def test_nhwc_copy_rejections(cuda_device):
    """Requests the kernels do not take fail before any launch: channel counts off the 8-element grid, NCHW
    inputs, an output overlapping its source."""
    from npu_ai_b200 import _lib, kernels
    x = torch.zeros(1, 12, 4, 4, dtype=torch.bfloat16, device=cuda_device).contiguous(
        memory_format=torch.channels_last)
    with pytest.raises(RuntimeError):
        kernels.upsample_nearest2x(x)
    with pytest.raises(ValueError):
        kernels.upsample_nearest2x(torch.zeros(1, 16, 4, 4, dtype=torch.bfloat16, device=cuda_device))
    with pytest.raises(ValueError):
        kernels.concat_channels(torch.zeros(1, 16, 4, 4, dtype=torch.float32, device=cuda_device),
                                torch.zeros(1, 16, 4, 4, dtype=torch.float32, device=cuda_device))
    buf = torch.zeros(64, 32, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError):
        _lib.call("npub200_concat_channels", ctypes.c_void_p(buf.data_ptr()), 32, 16,
                  ctypes.c_void_p(buf[:, 16:].data_ptr()), 32, 16, 64, ctypes.c_void_p(buf.data_ptr()), 32,
                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    kernels.check_status(cuda_device)
