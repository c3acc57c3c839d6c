"""torch-CPU restatement of the reference's CPU semantics (TEST INFRASTRUCTURE ONLY, see oracle/__init__.py)."""
from __future__ import annotations

import torch
import torch.nn.functional as F


def bf16_round(t: torch.Tensor) -> torch.Tensor:
    """Round to bf16 (RNE, torch's `.to(bfloat16)` as the reference's to_bf16, npu/xdna1_gemm.py:71-76) and back
    to f32."""
    return t.detach().to("cpu").to(torch.bfloat16).float()


def linear_ref(x: torch.Tensor, w_nk: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """f32 y = bf16(x) @ bf16(W)^T (+ bias in f32).

    x: (..., K); w_nk: (N, K) in nn.Linear's layout. Follows scripts/05-gemm-test.py:30
    (`x.to(bf16).float() @ W.to(bf16).float()`, W there given as (K, N)) and the bias add of
    npu/xdna1_gemm.py:417-418 (f32 bias, after the accumulation). The bias keeps the precision it is given in.
    """
    xb = bf16_round(x)
    wb = bf16_round(w_nk)
    y = xb.reshape(-1, xb.shape[-1]) @ wb.t()
    if bias is not None:
        y = y + bias.detach().to("cpu").float()
    return y.reshape(*x.shape[:-1], w_nk.shape[0])


def geglu_ref(x: torch.Tensor, w_2n_k: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """f32 GEGLU: y = linear_ref(x, W, bias) over the 2n rows of W (value rows, then gate rows), then
    y[..., :n] * gelu(y[..., n:]) with the exact (erf) GELU, the host-side rest of SD1.5's feed-forward block after
    the reference offloads its Linear (docs/02-results.md:411-413)."""
    y = linear_ref(x, w_2n_k, bias)
    a, gate = y.chunk(2, dim=-1)
    return a * F.gelu(gate)


def conv3x3_ref(x_nhwc: torch.Tensor, w_oihw: torch.Tensor, bias: torch.Tensor | None = None,
                residual: torch.Tensor | None = None) -> torch.Tensor:
    """f32 3x3 convolution (stride 1, zero padding 1) on bf16-rounded operands, NHWC in and out: the CPU
    convolution a SD1.5 UNet runs around the reference's offloaded layers (docs/02-results.md:411-413), restated with
    `F.conv2d`. bias: [cout] or [n, cout] (one row per image); residual: [n, h, w, cout], added after the bias."""
    x = bf16_round(x_nhwc).permute(0, 3, 1, 2)
    y = F.conv2d(x, bf16_round(w_oihw), padding=1).permute(0, 2, 3, 1)
    if bias is not None:
        b = bias.detach().to("cpu").float()
        y = y + (b[:, None, None, :] if b.dim() == 2 else b)
    if residual is not None:
        y = y + bf16_round(residual)
    return y


def group_norm_ref(x_nhwc: torch.Tensor, groups: int, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
                   silu: bool = False) -> torch.Tensor:
    """f32 `F.group_norm` (+ SiLU) on a bf16-rounded NHWC tensor, NHWC out: the host-side normalisation of a UNet
    ResBlock around the reference's offloaded layers (docs/02-results.md:411-413)."""
    x = bf16_round(x_nhwc).permute(0, 3, 1, 2)
    y = F.group_norm(x, groups, gamma.detach().to("cpu").float(), beta.detach().to("cpu").float(), eps)
    if silu:
        y = F.silu(y)
    return y.permute(0, 2, 3, 1)


def layer_norm_ref(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """f32 `F.layer_norm` over the last dimension of a bf16-rounded tensor: the host-side norm1/norm2/norm3 of a
    transformer block around the reference's offloaded projections (docs/02-results.md:411-413)."""
    x = bf16_round(x)
    return F.layer_norm(x, (x.shape[-1],), gamma.detach().to("cpu").float(), beta.detach().to("cpu").float(), eps)


def upsample_nearest2x_ref(x_nchw: torch.Tensor) -> torch.Tensor:
    """Nearest-neighbour 2x upsampling of an [n, c, h, w] tensor, as the UNet's Upsample block computes it on the
    host (F.interpolate(scale_factor=2, mode="nearest")): a pure copy, so any layout and dtype is exact."""
    return F.interpolate(x_nchw, scale_factor=2.0, mode="nearest")


def concat_channels_ref(a_nchw: torch.Tensor, b_nchw: torch.Tensor) -> torch.Tensor:
    """The decoder's skip concatenation of two [n, c, h, w] tensors along channels (torch.cat on the host)."""
    return torch.cat([a_nchw, b_nchw], dim=1)


def attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, scale: float | None = None,
                  head_major: bool = False) -> torch.Tensor:
    """f32 softmax(bf16(q) bf16(k)^T * scale) bf16(v) for every (batch, head) pair.

    q/k/v: (B, S, H*D) (the model's layout) or (B, H, S, D) with head_major. Returns the same layout as the
    input. Follows scripts/11-attn-fused-test.py:115-119 (SDPA in f32 on bf16-rounded inputs, the reference's
    "bf16 floor") with the reference runner's default scale d^-0.5 (npu/xdna1_gemm.py:528).
    """
    if head_major:
        B, H, Sq, D = q.shape
        qh, kh, vh = (bf16_round(t) for t in (q, k, v))
    else:
        B, Sq, inner = q.shape
        H = heads
        D = inner // H
        qh, kh, vh = (bf16_round(t).view(B, t.shape[1], H, D).transpose(1, 2) for t in (q, k, v))
    s = D ** -0.5 if scale is None else float(scale)
    o = F.scaled_dot_product_attention(qh, kh, vh, scale=s)
    if head_major:
        return o
    return o.transpose(1, 2).reshape(B, Sq, H * D)


def rel_max_err(a: torch.Tensor, ref: torch.Tensor) -> float:
    """max |a - ref| / max |ref|: the reference's accuracy metric (scripts/05-gemm-test.py:37,
    scripts/11-attn-fused-test.py:49-50, comfyui node :229)."""
    a = a.detach().float().cpu()
    ref = ref.detach().float().cpu()
    return float((a - ref).abs().max() / (ref.abs().max() + 1e-12))


def cosine(a: torch.Tensor, ref: torch.Tensor) -> float:
    """Cosine similarity of the flattened tensors (scripts/05-gemm-test.py:38)."""
    a = a.detach().double().cpu().reshape(-1)
    ref = ref.detach().double().cpu().reshape(-1)
    return float(a @ ref / (a.norm() * ref.norm() + 1e-12))


def rel_l2_err(a: torch.Tensor, ref: torch.Tensor) -> float:
    a = a.detach().double().cpu()
    ref = ref.detach().double().cpu()
    return float((a - ref).norm() / (ref.norm() + 1e-30))
