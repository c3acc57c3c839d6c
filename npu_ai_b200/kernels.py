"""Tensor-level calls into libnpub200: torch CUDA tensors in, pointers/strides through the C ABI, torch out.

torch provides device memory and the current stream; the arithmetic runs in the sm_100a kernels of the
library. The GEMM and the attention go through the library's torch operators (torch.ops.npub200.gemm /
.attention, libnpub200_torch.so) when that layer is built, else straight through ctypes; both reach the same C ABI
and kernels. Nothing here computes on the CPU, and there is no fallback when a kernel refuses a request.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_DT = {torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (got {t.device})")


def device_sms(device: torch.device | int | None = None) -> int:
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        n = ctypes.c_int(0)
        _lib.call("npub200_device_sms", ctypes.byref(n))
        return n.value


def register_weight(w_nk: torch.Tensor) -> int:
    """Register a resident [N, K] bf16 device weight; returns the library handle (TMA descriptors cached)."""
    _require_cuda(w_nk, "weight")
    if w_nk.dtype != torch.bfloat16 or w_nk.dim() != 2 or w_nk.stride(1) != 1:
        raise ValueError("resident weights are [N, K] bf16 with contiguous rows")
    h = ctypes.c_int64(0)
    with torch.cuda.device(w_nk.device):
        _lib.call("npub200_weight_register", ctypes.c_void_p(w_nk.data_ptr()), w_nk.shape[0], w_nk.shape[1],
                  w_nk.stride(0), ctypes.byref(h))
    return h.value


def gemm_plan(M: int, N: int, K: int, variant: int = 0, device: torch.device | int | None = None) -> tuple[int, int]:
    """(tile variant, split-K factor) the library picks for an M x K x N GEMM on the device. The variant is the N
    tile (64 ... 256), or 1000 + the N tile for 256-row tiles shared by a two-CTA cluster."""
    bn, sp = ctypes.c_int(0), ctypes.c_int(0)
    with torch.cuda.device(device if device is not None else torch.cuda.current_device()):
        _lib.call("npub200_gemm_plan", int(M), int(N), int(K), int(variant), ctypes.byref(bn), ctypes.byref(sp))
    return bn.value, sp.value


def release_weight(handle: int) -> None:
    _lib.call("npub200_weight_release", handle)


# One persistent workspace per (device, stream) for operands TMA cannot read as given (repacked copies): allocated
# zeroed once and only ever grown, never handed back to the caching allocator while this process may still launch
# on that stream. Split K needs none: it reduces inside a cluster's shared memory.
_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def _gemm_workspace(x: torch.Tensor, w: torch.Tensor | None, M: int, K: int, N: int, variant: int):
    nbytes = ctypes.c_size_t(0)
    _lib.call("npub200_gemm_workspace_size", ctypes.c_void_p(x.data_ptr()), x.stride(0), M, K,
              ctypes.c_void_p(w.data_ptr()) if w is not None else None, w.stride(0) if w is not None else 0, N,
              int(variant), ctypes.byref(nbytes))
    return _workspace(x.device, nbytes.value)


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor | None:
    """The zeroed per-(device, stream) workspace shared by the GEMM and convolution calls on that stream (grown to
    a power of two, at least 4 MiB)."""
    if nbytes == 0:
        return None
    key = (device.index or 0, torch.cuda.current_stream(device).cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        size = max(nbytes, 1 << 22)
        size = 1 << (size - 1).bit_length()
        ws = torch.zeros(size, dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def reset_workspaces() -> None:
    """Re-zero the cached workspaces (after a kernel aborted)."""
    for ws in _WORKSPACES.values():
        ws.zero_()


def gemm(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
         out_dtype: torch.dtype = torch.float32, variant: int = 0, handle: int | None = None,
         residual: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] = x[M, K] @ w[N, K]^T (+ bias) (+ residual) with bf16 operands and f32 accumulation.

    x and w are bf16 CUDA matrices with a unit inner stride (any row stride); bias is bf16 or f32 [N]; residual a
    bf16 [M, N] matrix with unit inner stride (may be `out`). With `handle` (from register_weight for this very `w`)
    the cached weight descriptor is used.
    """
    _require_cuda(x, "x")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("gemm operands must be bf16")
    if x.dim() != 2 or w.dim() != 2 or x.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("gemm operands must be 2-D with contiguous rows")
    M, K = x.shape
    N, K2 = w.shape
    if K != K2:
        raise AssertionError(f"K mismatch: x has {K}, weight has {K2}")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=x.device)
    if out.dtype not in _DT or out.stride(1) != 1 or tuple(out.shape) != (M, N):
        raise ValueError("out must be an [M, N] bf16/f32 matrix with contiguous rows")
    if bias is not None:
        if bias.dtype not in _DT or bias.numel() != N or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous [N] bf16/f32 vector")
    if residual is not None:
        if residual.dtype != torch.bfloat16 or residual.dim() != 2 or tuple(residual.shape) != (M, N) or \
                residual.stride(1) != 1:
            raise ValueError("residual must be a bf16 [M, N] matrix with contiguous rows")
        handle = None  # the residual entry point takes the weight itself
    ops = _lib.torch_ops()
    if ops is not None:
        return ops.gemm(x, w, bias, out, int(variant), None, int(handle or 0), residual)
    ws = _gemm_workspace(x, None if handle is not None else w, M, K, N, variant)
    args_tail = (ctypes.c_void_p(bias.data_ptr()) if bias is not None else None,
                 _DT[bias.dtype] if bias is not None else _lib.DTYPE_BF16,
                 ctypes.c_void_p(out.data_ptr()), out.stride(0), _DT[out.dtype],
                 ctypes.c_void_p(ws.data_ptr()) if ws is not None else None, ws.numel() if ws is not None else 0,
                 int(variant), ctypes.c_void_p(_stream_ptr(x.device)))
    with torch.cuda.device(x.device):
        if residual is not None:
            _lib.call("npub200_gemm_residual", ctypes.c_void_p(x.data_ptr()), x.stride(0), M, K,
                      ctypes.c_void_p(w.data_ptr()), w.stride(0), N, args_tail[0], args_tail[1],
                      ctypes.c_void_p(residual.data_ptr()), residual.stride(0), *args_tail[2:])
        elif handle is not None:
            _lib.call("npub200_gemm_w", ctypes.c_void_p(x.data_ptr()), x.stride(0), M, K, int(handle), *args_tail)
        else:
            _lib.call("npub200_gemm", ctypes.c_void_p(x.data_ptr()), x.stride(0), M, K, ctypes.c_void_p(w.data_ptr()),
                      w.stride(0), N, *args_tail)
    return out


def gemm_geglu(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, out: torch.Tensor | None = None,
               out_dtype: torch.dtype = torch.float32, variant: int = 0) -> torch.Tensor:
    """GEGLU projection in one kernel: with y = x @ w^T (+ bias), out[M, n] = y[:, :n] * gelu(y[:, n:]).

    w is the [2n, K] bf16 weight of the GEGLU `proj` Linear (value rows, then gate rows), bias bf16/f32 [2n];
    f32 accumulation and gating, exact (erf) GELU. The 2n-wide projection is never written to memory.
    """
    _require_cuda(x, "x")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("gemm_geglu operands must be bf16")
    if x.dim() != 2 or w.dim() != 2 or x.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("gemm_geglu operands must be 2-D with contiguous rows")
    M, K = x.shape
    N2, K2 = w.shape
    if K != K2:
        raise AssertionError(f"K mismatch: x has {K}, weight has {K2}")
    if N2 % 2:
        raise ValueError(f"GEGLU weight needs an even number of rows (value and gate halves), got {N2}")
    n = N2 // 2
    if out is None:
        out = torch.empty((M, n), dtype=out_dtype, device=x.device)
    if out.dtype not in _DT or out.stride(1) != 1 or tuple(out.shape) != (M, n):
        raise ValueError("out must be an [M, n] bf16/f32 matrix with contiguous rows")
    if bias is not None:
        if bias.dtype not in _DT or bias.numel() != N2 or not bias.is_contiguous():
            raise ValueError("bias must be a contiguous [2n] bf16/f32 vector")
    ws = _gemm_workspace(x, w, M, K, N2, variant)  # sized for the 2n-row weight: covers every repack
    with torch.cuda.device(x.device):
        _lib.call("npub200_gemm_geglu", ctypes.c_void_p(x.data_ptr()), x.stride(0), M, K,
                  ctypes.c_void_p(w.data_ptr()), w.stride(0), n,
                  ctypes.c_void_p(bias.data_ptr()) if bias is not None else None,
                  _DT[bias.dtype] if bias is not None else _lib.DTYPE_BF16,
                  ctypes.c_void_p(out.data_ptr()), out.stride(0), _DT[out.dtype],
                  ctypes.c_void_p(ws.data_ptr()) if ws is not None else None, ws.numel() if ws is not None else 0,
                  int(variant), ctypes.c_void_p(_stream_ptr(x.device)))
    return out


def pack_conv3x3_weight(w: torch.Tensor) -> torch.Tensor:
    """PyTorch conv weight [cout, cin, 3, 3] -> the kernel's [cout, 3, 3, cin] bf16 layout (once per weight)."""
    if w.dim() != 4 or tuple(w.shape[2:]) != (3, 3):
        raise ValueError("expected a [cout, cin, 3, 3] convolution weight")
    return w.detach().permute(0, 2, 3, 1).to(torch.bfloat16).contiguous()


def conv3x3(x: torch.Tensor, w_packed: torch.Tensor, bias: torch.Tensor | None = None,
            residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
            out_dtype: torch.dtype = torch.bfloat16, variant: int = 0) -> torch.Tensor:
    """3x3 convolution (stride 1, zero padding 1) as an implicit GEMM, NHWC in and out.

    x: bf16 [n, h, w, cin] contiguous (an NCHW channels_last tensor's `.permute(0, 2, 3, 1)` is such a view);
    w_packed: from pack_conv3x3_weight; bias: [cout] or [n, cout] (one row per image, rows may be strided), f32 or
    bf16; residual: bf16 [n, h, w, cout] added after the bias. Returns [n, h, w, cout].
    """
    _require_cuda(x, "x")
    if x.dtype != torch.bfloat16 or w_packed.dtype != torch.bfloat16:
        raise ValueError("conv3x3 operands must be bf16")
    if x.dim() != 4 or not x.is_contiguous():
        raise ValueError("conv3x3 input must be a contiguous [n, h, w, cin] (NHWC) tensor")
    n, h, wd, cin = x.shape
    if w_packed.dim() != 4 or tuple(w_packed.shape[1:]) != (3, 3, cin) or not w_packed.is_contiguous():
        raise ValueError(f"conv3x3 weight must be a contiguous [cout, 3, 3, {cin}] tensor (pack_conv3x3_weight)")
    cout = w_packed.shape[0]
    if out is None:
        out = torch.empty((n, h, wd, cout), dtype=out_dtype, device=x.device)
    if out.dtype not in _DT or tuple(out.shape) != (n, h, wd, cout) or out.stride(-1) != 1 or \
            out.stride(2) != out.stride(-2) or out.stride(1) != wd * out.stride(2) or out.stride(0) != h * out.stride(1):
        raise ValueError("out must be [n, h, w, cout] with uniformly strided pixel rows")
    img_stride = 0
    if bias is not None:
        if bias.dtype not in _DT or tuple(bias.shape) not in ((cout,), (n, cout)) or bias.stride(-1) != 1 or \
                (bias.dim() == 2 and bias.stride(0) < cout):
            raise ValueError("bias must be a [cout] or [n, cout] f32/bf16 tensor with unit column stride")
        img_stride = bias.stride(0) if bias.dim() == 2 else 0
    ldr = 0
    if residual is not None:
        if residual.dtype != torch.bfloat16 or tuple(residual.shape) != (n, h, wd, cout) or residual.stride(-1) != 1 \
                or residual.stride(0) != h * residual.stride(1) or residual.stride(1) != wd * residual.stride(2):
            raise ValueError("residual must be a bf16 [n, h, w, cout] tensor with uniformly strided pixel rows")
        ldr = residual.stride(2)
    with torch.cuda.device(x.device):
        nbytes = ctypes.c_size_t(0)
        _lib.call("npub200_conv3x3_workspace_size", n, h, wd, cin, cout, int(variant), ctypes.byref(nbytes))
        ws = _workspace(x.device, nbytes.value)
        _lib.call("npub200_conv3x3", ctypes.c_void_p(x.data_ptr()), n, h, wd, cin, ctypes.c_void_p(w_packed.data_ptr()),
                  cout, ctypes.c_void_p(bias.data_ptr()) if bias is not None else None,
                  _DT[bias.dtype] if bias is not None else _lib.DTYPE_BF16, img_stride,
                  ctypes.c_void_p(residual.data_ptr()) if residual is not None else None, ldr,
                  ctypes.c_void_p(out.data_ptr()), out.stride(2), _DT[out.dtype],
                  ctypes.c_void_p(ws.data_ptr()) if ws is not None else None, ws.numel() if ws is not None else 0,
                  int(variant), ctypes.c_void_p(_stream_ptr(x.device)))
    return out


_GN_STATS: dict[tuple[int, int], torch.Tensor] = {}


def group_norm(x: torch.Tensor, groups: int, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
               silu: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """GroupNorm (optionally + SiLU) over a contiguous NHWC bf16 tensor [n, h, w, c] (a channels_last activation's
    `.permute(0, 2, 3, 1)`); gamma, beta: [c]. Returns [n, h, w, c] bf16 (`out` may be `x`)."""
    _require_cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() != 4 or not x.is_contiguous():
        raise ValueError("group_norm takes a contiguous bf16 [n, h, w, c] tensor")
    n, h, w, c = x.shape
    if c % groups:
        raise ValueError(f"{c} channels do not split into {groups} groups")
    g32 = gamma.detach().to(x.device, torch.float32).contiguous()
    b32 = beta.detach().to(x.device, torch.float32).contiguous()
    if out is None:
        out = torch.empty_like(x)
    if out.shape != x.shape or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 tensor shaped like x")
    nbytes = ctypes.c_size_t(0)
    _lib.call("npub200_group_norm_scratch_size", n, int(groups), ctypes.byref(nbytes))
    key = (x.device.index or 0, torch.cuda.current_stream(x.device).cuda_stream)
    st = _GN_STATS.get(key)
    if st is None or st.numel() * 4 < nbytes.value:
        # zeroed once: the scratch ends in ticket counters the kernels leave zero
        st = torch.zeros(max(nbytes.value // 4 + 1, 1 << 16), dtype=torch.float32, device=x.device)
        _GN_STATS[key] = st
    with torch.cuda.device(x.device):
        _lib.call("npub200_group_norm", ctypes.c_void_p(x.data_ptr()), n, h * w, c, int(groups),
                  ctypes.c_void_p(g32.data_ptr()), ctypes.c_void_p(b32.data_ptr()), ctypes.c_float(eps), int(silu),
                  ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(st.data_ptr()),
                  ctypes.c_void_p(_stream_ptr(x.device)))
    return out


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """LayerNorm over the last dimension of a bf16 tensor whose rows are evenly strided (contiguous, or a 2-D view
    with unit column stride); weight, bias: [C] bf16 or f32 on the device. Returns bf16 shaped like x."""
    _require_cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() < 1:
        raise ValueError("layer_norm takes a bf16 tensor")
    C = x.shape[-1]
    if x.is_contiguous():
        x2 = x.reshape(-1, C)
    elif x.dim() == 2 and x.stride(1) == 1:
        x2 = x
    else:
        raise ValueError("layer_norm needs rows with a unit column stride and one row stride")
    if weight.shape != (C,) or bias.shape != (C,) or weight.dtype != bias.dtype or \
            weight.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("weight and bias must be [C] tensors of one dtype, bf16 or f32")
    weight = weight.detach().to(x.device).contiguous()
    bias = bias.detach().to(x.device).contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    if out.shape != x.shape or out.dtype != torch.bfloat16 or not out.is_contiguous():
        raise ValueError("out must be a contiguous bf16 tensor shaped like x")
    rows = x2.shape[0]
    if rows == 0:
        return out
    with torch.cuda.device(x.device):
        _lib.call("npub200_layer_norm", ctypes.c_void_p(x2.data_ptr()), rows, C, x2.stride(0),
                  ctypes.c_void_p(weight.data_ptr()), ctypes.c_void_p(bias.data_ptr()),
                  _lib.DTYPE_F32 if weight.dtype == torch.float32 else _lib.DTYPE_BF16, ctypes.c_float(eps),
                  ctypes.c_void_p(out.data_ptr()), C, ctypes.c_void_p(_stream_ptr(x.device)))
    return out


def _nhwc_2byte(t: torch.Tensor, name: str) -> None:
    _require_cuda(t, name)
    if t.dtype not in (torch.bfloat16, torch.float16) or t.dim() != 4:
        raise ValueError(f"{name} must be a 4-D bf16 or f16 tensor")


def upsample_nearest2x(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Nearest-neighbour 2x upsampling of a channels-last [n, c, h, w] tensor (torch's
    F.interpolate(x, scale_factor=2, mode="nearest")): returns channels-last [n, c, 2h, 2w]."""
    _nhwc_2byte(x, "x")
    if not x.is_contiguous(memory_format=torch.channels_last):
        raise ValueError("upsample_nearest2x takes a channels-last tensor")
    n, c, h, w = x.shape
    if out is None:
        out = torch.empty((n, c, 2 * h, 2 * w), dtype=x.dtype, device=x.device, memory_format=torch.channels_last)
    if out.shape != (n, c, 2 * h, 2 * w) or out.dtype != x.dtype or \
            not out.is_contiguous(memory_format=torch.channels_last):
        raise ValueError("out must be a channels-last tensor of x's dtype shaped [n, c, 2h, 2w]")
    with torch.cuda.device(x.device):
        _lib.call("npub200_upsample_nearest2x", ctypes.c_void_p(x.data_ptr()), n, h, w, c,
                  ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(_stream_ptr(x.device)))
    return out


def concat_channels(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """torch.cat([a, b], dim=1) of two channels-last [n, c, h, w] tensors: returns the channels-last
    [n, ca + cb, h, w] concatenation."""
    _nhwc_2byte(a, "a")
    _nhwc_2byte(b, "b")
    if a.dtype != b.dtype or a.device != b.device or a.shape[0] != b.shape[0] or a.shape[2:] != b.shape[2:]:
        raise ValueError("a and b must share dtype, device, batch and spatial size")
    if not (a.is_contiguous(memory_format=torch.channels_last) and b.is_contiguous(memory_format=torch.channels_last)):
        raise ValueError("concat_channels takes channels-last tensors")
    n, ca, h, w = a.shape
    cb = b.shape[1]
    if out is None:
        out = torch.empty((n, ca + cb, h, w), dtype=a.dtype, device=a.device, memory_format=torch.channels_last)
    if out.shape != (n, ca + cb, h, w) or out.dtype != a.dtype or \
            not out.is_contiguous(memory_format=torch.channels_last):
        raise ValueError("out must be a channels-last tensor shaped [n, ca + cb, h, w]")
    with torch.cuda.device(a.device):
        _lib.call("npub200_concat_channels", ctypes.c_void_p(a.data_ptr()), ca, ca, ctypes.c_void_p(b.data_ptr()),
                  cb, cb, n * h * w, ctypes.c_void_p(out.data_ptr()), ca + cb,
                  ctypes.c_void_p(_stream_ptr(a.device)))
    return out


def _bshd_strides(t: torch.Tensor, head_major: bool) -> tuple[int, int, int]:
    """(batch, seq, head) element strides of a (B, S, H, D) view given as (B, S, H*D) or (B, H, S, D)."""
    if head_major:
        return t.stride(0), t.stride(2), t.stride(1)
    return t.stride(0), t.stride(1), -1


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, scale: float | None = None,
              head_major_in: bool = False, head_major_out: bool = False, out_dtype: torch.dtype = torch.float32,
              out: torch.Tensor | None = None, variant: int = 0) -> torch.Tensor:
    """softmax(q k^T * scale) v for every (batch, head) pair in one launch.

    q/k/v: bf16 CUDA tensors, (B, S, H*D) or (B, H, S, D) when head_major_in; the output (B, Sq, H*D) or
    (B, H, Sq, D) when head_major_out. Strides may be padded (views), the last dimension must be contiguous.
    variant: key tile (0 = automatic, 64, 96, 128) + 1000 x query tiles of 128 rows per CTA (0 = automatic, 1, 2,
    or 4 with 64-key tiles for head dims up to 64); e.g. 2128 = two query tiles with 128-key tiles.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(t, name)
        if t.dtype != torch.bfloat16:
            raise ValueError(f"attention {name} must be bf16")
        if t.dim() != (4 if head_major_in else 3) or t.stride(-1) != 1:
            raise ValueError(f"attention {name} must be {'(B, H, S, D)' if head_major_in else '(B, S, H*D)'} with a "
                             "contiguous last dimension")
    if head_major_in:
        B, H, Sq, D = q.shape
        Skv = k.shape[2]
        if k.shape != (B, H, Skv, D) or v.shape != (B, H, Skv, D):
            raise ValueError("k/v shapes do not match q")
        qs, ks, vs = (_bshd_strides(t, True) for t in (q, k, v))
    else:
        B, Sq, inner = q.shape
        H = int(heads)
        if H <= 0 or inner % H:
            raise ValueError(f"q's last dimension {inner} is not a multiple of heads={heads}")
        D = inner // H
        Skv = k.shape[1]
        if k.shape != (B, Skv, inner) or v.shape != (B, Skv, inner):
            raise ValueError("k/v shapes do not match q")
        qs, ks, vs = ((t.stride(0), t.stride(1), D) for t in (q, k, v))
    scale = D ** -0.5 if scale is None else float(scale)
    if out is None:
        shape = (B, H, Sq, D) if head_major_out else (B, Sq, H * D)
        out = torch.empty(shape, dtype=out_dtype, device=q.device)
    if out.dtype not in _DT or out.stride(-1) != 1:
        raise ValueError("attention output must be bf16/f32 with a contiguous last dimension")
    ops = _lib.torch_ops()
    if ops is not None:
        return ops.attention(q, k, v, out, B, H, Sq, Skv, D, 0, 0, 0, bool(head_major_in), bool(head_major_out),
                             float(scale), int(variant), None)
    os_ = (out.stride(0), out.stride(2), out.stride(1)) if head_major_out else (out.stride(0), out.stride(1), D)
    with torch.cuda.device(q.device):
        _lib.call("npub200_attention",
                  ctypes.c_void_p(q.data_ptr()), *qs, ctypes.c_void_p(k.data_ptr()), *ks,
                  ctypes.c_void_p(v.data_ptr()), *vs, ctypes.c_void_p(out.data_ptr()), *os_, _DT[out.dtype],
                  B, H, Sq, Skv, D, ctypes.c_float(scale), int(variant), ctypes.c_void_p(_stream_ptr(q.device)))
    return out


def status(device: torch.device | int | None = None, clear: bool = True) -> int:
    """Synchronise the current stream and return the device status bits kernels reported (0 = healthy)."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    bits = ctypes.c_uint32(0)
    with torch.cuda.device(dev):
        _lib.call("npub200_status_read", ctypes.c_void_p(_stream_ptr(dev)), ctypes.byref(bits), 1 if clear else 0)
    return bits.value


def check_status(device: torch.device | int | None = None) -> None:
    """Raise RuntimeError if a kernel reported a failure (the reference's NpuProgram.wait, xdna1_program.py:475-479)."""
    bits = status(device)
    if bits:
        reset_workspaces()
        raise RuntimeError(f"GPU kernel reported failure status 0x{bits:x} (a bounded wait expired)")


def set_wait_timeout_ns(ns: int) -> None:
    _lib.call("npub200_set_wait_timeout_ns", ctypes.c_uint64(int(ns)))


def set_debug_flags(flags: int) -> None:
    _lib.call("npub200_set_debug_flags", ctypes.c_uint32(int(flags)))
