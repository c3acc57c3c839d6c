"""Which modules the ComfyUI runtime routes to the fused B200 forwards, decided on the host without a GPU.

The runtime replaces a module's forward only when every part it fuses was itself taken over (a ResBlock whose
GroupNorms and 3x3 convolutions are on the kernels, a transformer block whose three output Linears are, a spatial
transformer whose GroupNorm and 1x1 projections are); anything else keeps its own forward. These checks run the
plan functions on SD1.5-architecture modules with a stand-in runtime that records what was taken over."""
import types

import torch

from npu_ai_b200 import comfy_nodes as cn
from npu_ai_b200.sd15_unet import BasicTransformerBlock, ResBlock, SpatialTransformer


def _rt(**tables):
    base = {"convs": {}, "norms": {}, "weights": {}}
    base.update(tables)
    return types.SimpleNamespace(**base)


def _resblock_rt(rb, skip_kind="1x1"):
    rt = _rt()
    rt.convs[id(rb.in_layers[2])] = ("3x3", None, None)
    rt.convs[id(rb.out_layers[-1])] = ("3x3", None, None)
    rt.norms[id(rb.in_layers[0])] = (None, None)
    rt.norms[id(rb.out_layers[0])] = (None, None)
    if not isinstance(rb.skip_connection, torch.nn.Identity) and skip_kind:
        rt.convs[id(rb.skip_connection)] = (skip_kind, None, None)
    return rt


def test_resblock_plan_needs_every_part_taken_over():
    rb = ResBlock(64, 128, 256)  # channel change: 1x1 skip convolution
    rt = _resblock_rt(rb)
    plan = cn._resblock_plan(rb, rt)
    assert plan == (rb.in_layers[0], rb.in_layers[2], rb.out_layers[0], rb.out_layers[-1], rb.skip_connection)
    del rt.norms[id(rb.out_layers[0])]
    assert cn._resblock_plan(rb, rt) is None
    assert cn._resblock_plan(rb, _resblock_rt(rb, skip_kind=None)) is None  # skip conv not on the GEMM
    same = ResBlock(64, 64, 256)  # identity skip
    assert cn._resblock_plan(same, _resblock_rt(same))[-1] is same.skip_connection


def test_resblock_plan_skips_up_down_and_scale_shift_variants():
    rb = ResBlock(64, 64, 256)
    rt = _resblock_rt(rb)
    rb.use_scale_shift_norm = True
    assert cn._resblock_plan(rb, rt) is None
    rb.use_scale_shift_norm = False
    rb.updown = True
    assert cn._resblock_plan(rb, rt) is None


def test_transformer_block_plan_uses_the_three_output_linears():
    blk = BasicTransformerBlock(64, 4, 96)
    outs = (blk.attn1.to_out, blk.attn2.to_out, blk.ff.net[-1])  # plain Linears here (ComfyUI: Linear + Dropout)
    assert all(cn._out_linear(m) is m for m in outs)
    rt = _rt()
    for lin in outs:
        rt.weights[id(lin)] = (None, None, "")
    assert cn._tblock_plan(blk, rt) == outs
    del rt.weights[id(outs[2])]
    assert cn._tblock_plan(blk, rt) is None


def test_spatial_transformer_plan():
    st = SpatialTransformer(64, 4, 96)
    rt = _rt()
    rt.norms[id(st.norm)] = (None, None)
    rt.convs[id(st.proj_in)] = ("1x1", None, None)
    rt.convs[id(st.proj_out)] = ("1x1", None, None)
    assert cn._stransformer_plan(st, rt) == (st.norm, st.proj_in, st.proj_out)
    st.use_linear = True  # linear-projection variants keep their own forward
    assert cn._stransformer_plan(st, rt) is None
    st.use_linear = False
    rt.convs[id(st.proj_out)] = ("3x3", None, None)
    assert cn._stransformer_plan(st, rt) is None
    assert cn._stransformer_plan(ResBlock(64, 64, 256), rt) is None


def test_convolution_tile_shapes():
    # 128-pixel tiles of whole rows: widths dividing 128 and heights that are multiples of the rows per tile
    for h, w in ((64, 64), (32, 32), (16, 16), (8, 8), (4, 4), (128, 128), (1, 128), (2, 4)):
        assert cn._conv_tiles(h, w), (h, w)
    for h, w in ((64, 96), (3, 64), (8, 256), (5, 5), (6, 4)):
        assert not cn._conv_tiles(h, w), (h, w)


def test_channels_last_bf16_predicate():
    x = torch.zeros(2, 16, 4, 4, dtype=torch.bfloat16).contiguous(memory_format=torch.channels_last)
    assert not cn._cl_bf16(x)  # a CPU tensor never takes the kernel path
    assert not cn._cl_bf16(torch.zeros(2, 16, 4, 4))


def test_output_linear_of_comfyui_style_to_out():
    lin = torch.nn.Linear(8, 8)
    assert cn._out_linear(torch.nn.Sequential(lin, torch.nn.Dropout(0.0))) is lin
    assert cn._out_linear(torch.nn.Sequential(lin, torch.nn.ReLU())) is None
    assert cn._out_linear(torch.nn.Identity()) is None
