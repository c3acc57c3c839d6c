"""Host-side logic of the ComfyUI nodes and the hot path's Python surface, without a GPU.

Covers what the reference's node file defines (comfyui/custom_nodes/comfyui_xdna1_npu/__init__.py): the node
classes under the reference's names (:400-409), their ComfyUI interface (INPUT_TYPES / RETURN_TYPES / FUNCTION,
:260-291, :362-391), the attention gate's static routing rules (:39-99: masked and GQA calls, small shapes, mode
off -> the model's own attention), and that the runner and every kernel wrapper refuse host tensors or a host
without a CUDA device instead of falling back to the CPU (the reference never falls back silently either,
node :5-7)."""
import pytest
import torch

from npu_ai_b200 import comfy_nodes as cn


def test_reference_node_names_resolve_to_the_b200_nodes():
    for ref_name, ours in (("XDNA1NpuLinearOffload", cn.B200LinearOffload), ("XDNA1NpuStatus", cn.B200Status),
                           ("XDNA1NpuRelease", cn.B200Release)):
        assert cn.NODE_CLASS_MAPPINGS[ref_name] is ours
    assert set(cn.NODE_CLASS_MAPPINGS) == set(cn.NODE_DISPLAY_NAME_MAPPINGS)


@pytest.mark.parametrize("name", ["B200LinearOffload", "B200Status", "B200Release"])
def test_node_interface(name):
    cls = cn.NODE_CLASS_MAPPINGS[name]
    spec = cls.INPUT_TYPES()
    assert "required" in spec and isinstance(spec["required"], dict)
    assert isinstance(cls.RETURN_TYPES, tuple) and cls.RETURN_TYPES
    assert callable(getattr(cls, cls.FUNCTION))


def test_offload_node_keeps_the_reference_inputs_and_defaults():
    spec = cn.B200LinearOffload.INPUT_TYPES()
    req, opt = spec["required"], spec.get("optional", {})
    both = {**req, **opt}
    # the reference node's inputs (node :264-281) under the same names and defaults
    assert req["model"][0] == "MODEL"
    assert both["enabled"][1]["default"] is True
    assert both["min_tokens"][1]["default"] == 64
    assert both["min_features"][1]["default"] == 320
    assert both["skip_names"][1]["default"] == "time_embed,label_emb,emb_layers"
    assert both["attention"][1]["default"] == "auto"
    assert both["attn_min_tokens"][1]["default"] == 1  # every SD1.5 attention shape on the kernel
    assert cn.B200LinearOffload.RETURN_TYPES == ("MODEL",)


def test_attention_variants_cover_the_sd15_head_dims():
    for d in (40, 80, 160):
        v = cn.attn_variants(d)
        assert v and 0 in v and len(set(v)) == len(v)


@pytest.mark.parametrize("mode,mask,gqa,fits,tq,min_tokens,expect", [
    ("auto", False, False, True, 4096, 1, None),
    ("gpu", False, False, True, 256, 1, None),
    ("auto", False, False, True, 64, 1, None),        # the SD1.5 middle block stays on the fused kernel
    ("off", False, False, True, 4096, 1, "attention mode = off"),
    ("auto", True, False, True, 4096, 1, "masked attention"),
    ("auto", False, True, True, 4096, 1, "grouped-query attention"),
    ("auto", False, False, False, 4096, 1, "outside the fused kernel's range"),
    ("auto", False, False, True, 77, 256, "fewer than 256 query tokens"),
])
def test_attention_gate_static_routing(mode, mask, gqa, fits, tq, min_tokens, expect):
    gate = cn.AttentionGate(mode=mode, min_tokens=min_tokens)
    key = (2, tq, tq, 8, 40)
    assert gate.model_route_reason(key, mask, gqa, fits) == expect
    if expect is not None:
        assert gate.shapes[key].model_reason == expect
        assert str(key) in gate.table() and expect in gate.table()  # the reason shows in the Status node's table
        gate.model_route_reason(key, mask, gqa, fits)
        assert gate.shapes[key].model_reason == expect      # logged and recorded once
    else:
        assert key not in gate.shapes


def test_default_gate_keeps_every_sd15_attention_on_the_kernel():
    gate = cn.AttentionGate()
    assert gate.mode == "auto" and gate.min_tokens == 1
    for key in ((2, 4096, 4096, 8, 40), (2, 4096, 77, 8, 40), (2, 1024, 1024, 8, 80), (2, 256, 256, 8, 160),
                (2, 64, 64, 8, 160), (2, 64, 77, 8, 160)):
        assert gate.model_route_reason(key, False, False, True) is None


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour on a host without a CUDA device")
def test_runner_refuses_to_run_without_a_cuda_device():
    from npu_ai_b200.runner import NpuGemm
    with pytest.raises(RuntimeError, match="no CPU path"):
        NpuGemm()
    with pytest.raises(ValueError, match="no CPU path"):
        NpuGemm(device="cpu")


def test_unet_skip_concatenation_on_the_cpu_is_torch_cat():
    from npu_ai_b200.sd15_unet import cat_channels
    a, b = torch.randn(2, 16, 3, 5), torch.randn(2, 8, 3, 5)
    assert torch.equal(cat_channels(a, b), torch.cat([a, b], dim=1))


def test_bench_kernel_kinds():
    import bench
    assert bench._kernel_kind("void npub200::gemm_bf16_tcgen05_kernel<160, 5, 2, false>(CUtensorMap)") == \
        "3x3 convolution"
    assert bench._kernel_kind("void npub200::gemm_bf16_tcgen05_kernel<256, 4, 1, false>(CUtensorMap)") == \
        "GEGLU GEMM"
    assert bench._kernel_kind("void npub200::gemm_bf16_tcgen05_kernel<256, 6, 0, true>(CUtensorMap)") == "GEMM"
    assert bench._kernel_kind("void npub200::attention_fwd_qt2_tcgen05_kernel<48, 96, 2>(x)") == "attention"
    assert bench._kernel_kind("npub200::(anonymous namespace)::concat_channels_kernel(uint4 const*)") == "NHWC copy"
    assert bench._kernel_kind("cutlass3x_sm100_tensorop_s256x128x16implicit_gemm_fprop_bf16") == \
        "torch convolution (cuDNN)"


def _cpu_bf16(*shape):
    return torch.zeros(*shape, dtype=torch.bfloat16)


@pytest.mark.parametrize("call", [
    lambda k: k.gemm(_cpu_bf16(4, 8), _cpu_bf16(16, 8)),
    lambda k: k.gemm_geglu(_cpu_bf16(4, 8), _cpu_bf16(16, 8)),
    lambda k: k.conv3x3(_cpu_bf16(1, 4, 4, 64), _cpu_bf16(8, 3, 3, 64)),
    lambda k: k.group_norm(_cpu_bf16(1, 4, 4, 64), 32, torch.ones(64), torch.zeros(64)),
    lambda k: k.layer_norm(_cpu_bf16(4, 64), torch.ones(64), torch.zeros(64)),
    lambda k: k.upsample_nearest2x(_cpu_bf16(1, 8, 2, 2).contiguous(memory_format=torch.channels_last)),
    lambda k: k.concat_channels(_cpu_bf16(1, 8, 2, 2), _cpu_bf16(1, 8, 2, 2)),
    lambda k: k.attention(_cpu_bf16(1, 16, 80), _cpu_bf16(1, 16, 80), _cpu_bf16(1, 16, 80), 2),
    lambda k: k.register_weight(_cpu_bf16(16, 8)),
], ids=["gemm", "gemm_geglu", "conv3x3", "group_norm", "layer_norm", "upsample", "concat", "attention",
        "register_weight"])
def test_every_kernel_refuses_host_tensors(call):
    """No op computes on the CPU: host tensors are refused before anything launches (the product path has no
    fallback; callers copy to the device, as NpuGemm does for the reference's CPU inputs)."""
    from npu_ai_b200 import kernels
    with pytest.raises(ValueError, match="CUDA tensor"):
        call(kernels)
