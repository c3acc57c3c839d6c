"""CPU oracle for the npu-ai offload hot path. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline/reference legs may import this package, and
only as the checker (or the timed CPU baseline), never as the thing measured or shipped. The product path
(npu_ai_b200) never imports it and has no CPU fallback.

What it restates: the reference's own CPU semantics for the path, i.e. what Tobynau/npu-ai falls back to and
checks its NPU results against.
  * GEMM: bf16-rounded x and W multiplied in f32 (scripts/05-gemm-test.py:30, the ComfyUI node's CPU fallback
    `F.linear`, comfyui/custom_nodes/comfyui_xdna1_npu/__init__.py:151), bias added in f32 after the product
    (npu/xdna1_gemm.py:417-418).
  * Attention: scaled dot-product attention in f32 on bf16-rounded q/k/v (scripts/11-attn-fused-test.py:115-119).
  * 3x3 convolution: `F.conv2d` in f32 on bf16-rounded operands, bias then residual added in f32 (the host-side
    convolutions of the UNet around the offloaded layers, docs/02-results.md:411-413).
  * GroupNorm (+ SiLU): `F.group_norm` in f32 on bf16-rounded activations (the same host-side work).
  * Nearest 2x upsampling and the skip concatenation of the UNet decoder: `F.interpolate` and `torch.cat`, pure
    copies (the same host-side work).
  * GEGLU feed-forward projection: the projection as above, then value * gelu(gate) in f32 with the exact (erf)
    GELU, as the host side of a transformer block computes it after the reference's Linear offload
    (docs/02-results.md:411-413 lists GEGLU among the host work; ComfyUI's GEGLU module is
    `x, gate = proj(x).chunk(2, dim=-1); return x * F.gelu(gate)`).
Pinning: tests/golden/ holds fixtures produced by running the reference's CPU fallback code itself
(tests/golden/make_golden.py imports the reference's ComfyUI node module) and the reference's published
accuracy figures (docs/02-results.md:709) that the attention oracle reproduces on the reference's own seeded
inputs; see tests/test_oracle.py.
"""
from .reference_ops import (attention_ref, bf16_round, concat_channels_ref, conv3x3_ref, cosine,  # noqa: F401
                            geglu_ref, group_norm_ref, layer_norm_ref, linear_ref, rel_l2_err, rel_max_err,
                            upsample_nearest2x_ref)
