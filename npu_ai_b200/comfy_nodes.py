"""ComfyUI custom nodes for B200: run the diffusion model's Linear layers and attention on the sm_100a kernels.

Drop-in for the reference's node module (comfyui/custom_nodes/comfyui_xdna1_npu/__init__.py): the same three
nodes, inputs, Linear takeover, attention override hook and per-call log line, with the device side replaced.
The nodes are registered under the reference's class names too, so saved workflows load unchanged.

  B200: Offload Linear layers  (MODEL -> MODEL)   also installs the attention override   (node :260-360)
  B200: Status                 (-> STRING)                                                (node :363-381)
  B200: Release                (MODEL -> MODEL)                                           (node :384-397)

What changes: the model runs on the GPU, so calls route by device `cuda` (the reference routes CPU tensors to the
NPU, node :150, :174). The attention gate no longer chooses between the accelerator and the CPU: it chooses
between kernel variants of the fused attention (query tiles per CTA x key tile) by timing each once per shape, and still
checks the first result of every shape against the model's own attention (max relative error <= 0.1, else
RuntimeError, node :225-232). Shapes with a mask or GQA (which the fused kernel does not implement) and
attention mode "off" (the reference's "cpu") run the model's own attention function, logged once per shape.
"""
from __future__ import annotations

import threading
import time
import types
import weakref
from dataclasses import dataclass, field

import numpy as np
import torch

_RUNTIME = None
_RUNTIME_LOCK = threading.RLock()
ATTENTION_MODES = ["auto", "gpu", "off", "npu", "cpu"]   # "npu" / "cpu": the reference's names for gpu / off


def attn_variants(head_dim: int) -> tuple[int, ...]:
    """Fused-attention variants the gate times for a head dim: 0 (the kernel's own measured choice) first, then
    every distinct (query tiles per CTA, key tile) pair the head dim allows, encoded as 1000 * tiles + keys."""
    dp = (head_dim + 15) // 16 * 16
    keys = (64, 96, 128) if dp <= 64 else ((64, 128) if dp <= 128 else (64,))
    qts = (1, 2) if dp <= 192 else (1,)
    four = (4064,) if dp <= 64 else ()  # four Q tiles per CTA: 64-key tiles, head dims up to 64
    return (0,) + tuple(1000 * qt + bn for qt in qts for bn in keys) + four


def _log(msg: str) -> None:
    print(f"[npu-b200] {msg}", flush=True)


def _mode(m: str) -> str:
    return {"npu": "gpu", "cpu": "off"}.get(m, m if m in ATTENTION_MODES else "auto")


@dataclass
class ShapeRecord:
    """The gate's knowledge of one attention shape, keyed (batch, query tokens, key tokens, heads, head dim)."""
    variant_ms: dict[int, float] = field(default_factory=dict)  # timed once per variant on the first call
    model_ms: float | None = None        # the model's own attention, timed after one warm-up call
    variant: int | None = None           # the fused-kernel variant this shape runs
    model_reason: str | None = None      # set when the shape must run the model's own attention
    max_rel_err: float | None = None     # first-call check against the model's own attention

    def describe(self) -> str:
        parts = [f"variant {v} {t:.3f} ms" for v, t in sorted(self.variant_ms.items())]
        if self.model_ms is not None:
            parts.append(f"model {self.model_ms:.3f} ms")
        if self.max_rel_err is not None:
            parts.append(f"max rel err {self.max_rel_err:.1e}")
        outcome = self.model_reason if self.model_reason is not None else \
            ("pending" if self.variant is None else f"variant {self.variant}")
        return ", ".join(parts) + f" -> {outcome}"


class AttentionGate:
    """Which fused-attention variant each attention shape runs (the role of the reference's AttentionGate,
    node :39-99; there the choice is NPU or CPU, here it is among kernel variants only).

    Mode ``auto`` times every variant the head dim allows once, on the shape's first call, and keeps the fastest;
    ``gpu`` keeps the kernel's own automatic variant; ``off`` (the reference's ``cpu``) hands every call to the
    model's own attention. In every mode the first fused result of a shape is compared with the model's own
    attention (max relative error <= 0.1, else RuntimeError). The model's attention also serves the calls the
    kernel does not implement: an attention mask or grouped-query heads. ``min_tokens`` (default 1, so every SD1.5
    self- and cross-attention, the 64-token middle block included, stays on the kernel) sends shorter query
    sequences there too; each such shape is logged once with its reason.
    """

    def __init__(self, mode: str = "auto", min_tokens: int = 1):
        self.mode = mode
        self.min_tokens = min_tokens
        self.shapes: dict[tuple, ShapeRecord] = {}
        self.fused_calls = 0
        self.model_calls = 0
        self.fused_seconds = 0.0     # host time of the calls (kernel launches are asynchronous)
        self.model_seconds = 0.0
        self.fused_flops = 0.0

    def record(self, key: tuple) -> ShapeRecord:
        rec = self.shapes.get(key)
        if rec is None:
            rec = self.shapes[key] = ShapeRecord()
        return rec

    def model_route_reason(self, key: tuple, masked: bool, gqa: bool, fits: bool) -> str | None:
        """Why this call must run the model's own attention, or None when the fused kernel takes it."""
        rules = ((self.mode == "off", "attention mode = off"),
                 (masked, "masked attention"),
                 (gqa, "grouped-query attention"),
                 (not fits, "outside the fused kernel's range"),
                 (key[1] < self.min_tokens, f"fewer than {self.min_tokens} query tokens"))
        why = next((text for hit, text in rules if hit), None)
        if why is not None:
            rec = self.record(key)
            if rec.model_reason is None:
                rec.model_reason = why
                _log(f"attention {key} runs the model's own attention: {why}")
        return why

    def reset(self) -> None:
        self.shapes.clear()

    def table(self) -> str:
        return "; ".join(f"{key}: {rec.describe()}" for key, rec in sorted(self.shapes.items()))

    def summary(self) -> str:
        return (f"attention: {self.fused_calls} calls on the fused kernel ({self.fused_seconds:.2f}s), "
                f"{self.model_calls} on the model's own attention ({self.model_seconds:.2f}s); "
                f"gate: {self.table()}")


def _time_gpu(fn, device) -> tuple[object, float]:
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(torch.cuda.current_stream(device))
    y = fn()
    e.record(torch.cuda.current_stream(device))
    e.synchronize()
    return y, s.elapsed_time(e)


class B200Runtime:
    """The process-wide GPU side of the nodes: the runner, the gate, and every module whose forward it replaced
    (the role of the reference's XDNA1Runtime, node :102-143, with a resident [N, K] weight per Linear instead of a
    transposed NPU upload)."""

    def __init__(self, device=None):
        from .runner import NpuGemm  # loads libnpub200.so; fails loudly without it
        self.gemm = NpuGemm(device=device, verbose=False)
        self.attn = AttentionGate()
        # Switches the node's UNet wrapper flips around each call: `enabled` routes patched modules to the kernels;
        # `record_only` (the shape-discovery pass) runs them on torch and collects each GEMM's (tokens, K, N).
        self.enabled = False
        self.record_only = False
        self.recorded: set[tuple[int, int, int]] = set()
        self.min_tokens = 64          # Linear calls with fewer rows keep torch's F.linear
        self.calls = 0
        self.last_summary = ""
        # Every patched module: patched[id] = (module, the forward it had before), restored by release().
        self.patched: dict[int, tuple] = {}
        # Linears on the GEMM kernel: weights[id] = (resident NpuWeight, f32 bias on the device or None, name).
        self.weights: dict[int, tuple] = {}
        self.geglu_modules: set[int] = set()     # GEGLU modules routed to the fused projection + gating kernel
        # Sibling projections fed the same input (self-attention q/k/v, cross-attention k/v) run as ONE GEMM over
        # the concatenated weight: leader id -> (fused NpuWeight, fused bias | None, [(member id, column slice)]),
        # member id -> leader id; `pending` holds the member outputs of the last leader call until consumed.
        self.fused_groups: dict[int, tuple] = {}
        self.fused_member: dict[int, int] = {}
        self.pending: dict[int, tuple] = {}
        # Convolution-side takeover (channels-last activations): id(conv) -> (kind "3x3" | "1x1", packed weight or
        # NpuWeight, f32 bias | None); id(GroupNorm) -> (f32 gamma, f32 beta); id(ResBlock) -> its fused plan.
        self.convs: dict[int, tuple] = {}
        self.norms: dict[int, tuple] = {}
        self.resblocks: dict[int, tuple] = {}
        # Time-embedding projections of the fused ResBlocks, grouped: every ResBlock of a UNet call reads the same
        # `emb`, so their SiLU + Linear (with the first convolution's bias folded in) run as ONE GEMM per input
        # width. emb_groups[i] = (fused NpuWeight, f32 bias); emb_slices[id(ResBlock)] = (i, column offset, cout);
        # emb_cache[i] = (weakref to the emb it was computed for, its version, [n, columns] f32 result).
        self.emb_groups: list[tuple] = []
        self.emb_slices: dict[int, tuple] = {}
        self.emb_cache: dict[int, tuple] = {}
        self.conv_calls = 0  # convolution-side calls that ran on the B200 kernels (ResBlocks count once)
        # Transformer blocks whose residual adds go into the output Linears' GEMM epilogues: id(block) ->
        # (attn1 out Linear, attn2 out Linear, feed-forward out Linear); pending_res: id(Linear) -> residual.
        self.tblocks: dict[int, tuple] = {}
        self.pending_res: dict[int, torch.Tensor] = {}
        # LayerNorms of those blocks (norm1/norm2/norm3) on the row-wise LayerNorm kernel: id -> (f32 gamma, beta).
        self.lnorms: dict[int, tuple] = {}
        # Upsample blocks whose nearest 2x step runs on the NHWC upsampling kernel, and spatial transformers whose
        # closing residual add goes into proj_out's GEMM epilogue: id(module) -> (GroupNorm, proj_in, proj_out).
        self.upsamples: set[int] = set()
        self.stransformers: dict[int, tuple] = {}
        # GroupNorm -> SiLU -> convolution sequences (the UNet's output head, ResBlock layer stacks) with the SiLU
        # in the GroupNorm kernel: id(Sequential) -> (GroupNorm, convolution).
        self.norm_silu: dict[int, tuple] = {}
        # A second stream per device for work off a ResBlock's critical path (its 1x1 skip convolution).
        self.side_streams: dict[int, torch.cuda.Stream] = {}

    def _patch(self, mod: torch.nn.Module, forward) -> None:
        """Swap `mod.forward` for `forward` bound to it, keeping the old one for release()."""
        self.patched[id(mod)] = (mod, mod.forward)
        mod.forward = types.MethodType(forward, mod)

    @staticmethod
    def _linear_eligible(name: str, mod: torch.nn.Module, min_features: int, skip: tuple[str, ...]) -> bool:
        """A Linear the node takes over: both feature counts reach `min_features` and no `skip` substring occurs
        in its module name (the reference's filter, node :119-136)."""
        if not isinstance(mod, torch.nn.Linear):
            return False
        if min(mod.in_features, mod.out_features) < min_features:
            return False
        return not any(s and s in name for s in skip)

    def take_over(self, diffusion_model: torch.nn.Module, min_features: int, skip: tuple[str, ...],
                  convolutions: bool = True) -> int:
        """Patch the model's eligible modules onto the kernels; returns how many Linears were newly taken."""
        todo = [(name, mod) for name, mod in diffusion_model.named_modules()
                if id(mod) not in self.patched and self._linear_eligible(name, mod, min_features, skip)]
        dev = self.gemm.device
        for name, lin in todo:
            bias = None if lin.bias is None else lin.bias.detach().to(dev, torch.float32).contiguous()
            # nn.Linear's own [N, K] weight is the kernel's B operand: no transpose
            self.weights[id(lin)] = (self.gemm.upload_weight(lin.weight.detach(), layout="nk"), bias, name)
            self._patch(lin, _gpu_linear_forward)
        n_new = len(todo)
        self._fuse_projections(diffusion_model)
        for mod in diffusion_model.modules():
            plan = _tblock_plan(mod, self)
            if plan is not None and id(mod) not in self.patched:
                self.tblocks[id(mod)] = plan
                self._patch(mod, _gpu_tblock_forward)
        for mod in diffusion_model.modules():
            if id(mod) not in self.tblocks:
                continue
            for nm in ("norm1", "norm2", "norm3"):
                ln = getattr(mod, nm, None)
                if (isinstance(ln, torch.nn.LayerNorm) and ln.elementwise_affine and ln.bias is not None
                        and len(ln.normalized_shape) == 1 and ln.normalized_shape[0] % 8 == 0
                        and ln.normalized_shape[0] <= 2048 and id(ln) not in self.patched):
                    self.lnorms[id(ln)] = (ln.weight.detach().to(self.gemm.device, torch.float32).contiguous(),
                                           ln.bias.detach().to(self.gemm.device, torch.float32).contiguous())
                    self._patch(ln, _gpu_layer_norm_forward)
        if convolutions:
            self._take_over_convs(diffusion_model)
        # GEGLU feed-forward blocks whose projection was taken over: projection + gating in one kernel.
        for name, mod in diffusion_model.named_modules():
            proj = getattr(mod, "proj", None)
            if (type(mod).__name__ == "GEGLU" and isinstance(proj, torch.nn.Linear) and id(proj) in self.weights
                    and id(mod) not in self.patched and proj.out_features % 2 == 0):
                self.geglu_modules.add(id(mod))
                self._patch(mod, _gpu_geglu_forward)
        return n_new

    def _fuse_projections(self, diffusion_model: torch.nn.Module) -> None:
        """q/k/v of an attention module with one input width become one GEMM (to_q leads). k/v projections of
        cross-attention modules read the text context, which every block of a UNet call shares: all of them with
        one input width become ONE grouped GEMM over the concatenated weights (the first block's to_k leads), so a
        UNet call projects the context once instead of once per block."""
        cross: dict[int, list] = {}
        for mod in diffusion_model.modules():
            lins = [getattr(mod, n, None) for n in ("to_q", "to_k", "to_v")]
            if not all(isinstance(m, torch.nn.Linear) and id(m) in self.weights for m in lins):
                continue
            if any(id(m) in self.fused_member or id(m) in self.fused_groups for m in lins):
                continue
            q, k, v = lins
            if q.in_features == k.in_features == v.in_features:
                self._add_group([q, k, v])
            elif k.in_features == v.in_features:
                cross.setdefault(k.in_features, []).extend([k, v])
        for group in cross.values():
            self._add_group(group)

    def _take_over_convs(self, dm: torch.nn.Module) -> None:
        """3x3 convolutions (stride 1, padding 1, input channels in multiples of 64) onto the implicit-GEMM kernel,
        1x1 convolutions onto the GEMM over the channels-last view, GroupNorms onto the NHWC GroupNorm kernel, and
        ResBlocks built from those onto a fused forward (conv bias + time embedding as a per-image bias row of the
        first convolution, the skip path as the residual of the second). Every patched forward falls back to the
        module's own forward for inputs it does not take (not channels-last bf16 on the GPU, other shapes)."""
        from . import kernels
        dev = self.gemm.device
        for mod in dm.modules():
            if id(mod) in self.patched:
                continue
            if isinstance(mod, torch.nn.Conv2d) and mod.groups == 1 and mod.dilation == (1, 1) \
                    and mod.padding_mode == "zeros":
                bias = mod.bias.detach().to(dev, torch.float32).contiguous() if mod.bias is not None else None
                if mod.kernel_size == (3, 3) and mod.stride == (1, 1) and mod.padding == (1, 1) \
                        and mod.in_channels % 64 == 0:
                    entry = ("3x3", kernels.pack_conv3x3_weight(mod.weight.to(dev)), bias)
                elif mod.kernel_size == (1, 1) and mod.stride == (1, 1) and mod.padding == (0, 0) \
                        and mod.in_channels % 8 == 0:
                    w = mod.weight.detach().reshape(mod.out_channels, mod.in_channels)
                    entry = ("1x1", self.gemm.upload_weight(w, layout="nk"), bias)
                else:
                    continue
                self.convs[id(mod)] = entry
                self._patch(mod, _gpu_conv_forward)
            elif isinstance(mod, torch.nn.GroupNorm) and mod.affine and mod.num_channels % 8 == 0:
                self.norms[id(mod)] = (mod.weight.detach().to(dev, torch.float32).contiguous(),
                                       mod.bias.detach().to(dev, torch.float32).contiguous())
                self._patch(mod, _gpu_group_norm_forward)
        for mod in dm.modules():
            plan = _resblock_plan(mod, self)
            if plan is not None and id(mod) not in self.patched:
                self.resblocks[id(mod)] = plan
                self._patch(mod, _gpu_resblock_forward)
        for mod in dm.modules():
            if id(mod) in self.patched:
                continue
            if (type(mod).__name__ == "Upsample" and getattr(mod, "dims", 2) == 2 and getattr(mod, "use_conv", True)
                    and self.convs.get(id(getattr(mod, "conv", None)), ("",))[0] == "3x3"):
                self.upsamples.add(id(mod))
                self._patch(mod, _gpu_upsample_forward)
                continue
            plan = _stransformer_plan(mod, self)
            if plan is not None:
                self.stransformers[id(mod)] = plan
                self._patch(mod, _gpu_spatial_transformer_forward)
                continue
            if (type(mod) is torch.nn.Sequential and len(mod) == 3 and isinstance(mod[0], torch.nn.GroupNorm)
                    and id(mod[0]) in self.norms and isinstance(mod[1], torch.nn.SiLU)
                    and isinstance(mod[2], torch.nn.Conv2d)):
                self.norm_silu[id(mod)] = (mod[0], mod[2])
                self._patch(mod, _gpu_norm_silu_conv_forward)
        by_width: dict[int, list] = {}
        for mod in dm.modules():
            if id(mod) in self.resblocks and id(mod) not in self.emb_slices:
                by_width.setdefault(mod.emb_layers[1].in_features, []).append(mod)
        for blocks in by_width.values():
            lins = [b.emb_layers[1] for b in blocks]
            w = torch.cat([lin.weight.detach() for lin in lins])
            parts = []
            for b, lin in zip(blocks, lins):
                cb = self.convs[id(self.resblocks[id(b)][1])][2]
                e = lin.bias.detach().to(dev, torch.float32) if lin.bias is not None else \
                    torch.zeros(lin.out_features, device=dev)
                parts.append(e + cb if cb is not None else e)
            gi = len(self.emb_groups)
            self.emb_groups.append((self.gemm.upload_weight(w, layout="nk"), torch.cat(parts).contiguous()))
            off = 0
            for b, lin in zip(blocks, lins):
                self.emb_slices[id(b)] = (gi, off, lin.out_features)
                off += lin.out_features

    def _add_group(self, group: list) -> None:
        w = torch.cat([m.weight.detach() for m in group])
        nw = self.gemm.upload_weight(w, layout="nk")
        bias = None
        if any(m.bias is not None for m in group):
            bias = torch.cat([m.bias.detach().float() if m.bias is not None else
                              torch.zeros(m.out_features, device=m.weight.device) for m in group])
            bias = bias.to(self.gemm.device, torch.float32).contiguous()
        members, col = [], group[0].out_features
        for m in group[1:]:
            members.append((id(m), col, col + m.out_features))
            self.fused_member[id(m)] = id(group[0])
            col += m.out_features
        self.fused_groups[id(group[0])] = (nw, bias, members, group[0].out_features)

    def side_stream(self, device: torch.device) -> torch.cuda.Stream:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        st = self.side_streams.get(idx)
        if st is None:
            st = torch.cuda.Stream(device=torch.device("cuda", idx))
            self.side_streams[idx] = st
        return st

    def release(self) -> None:
        for mod, orig in self.patched.values():
            mod.forward = orig
        for w, _, _ in self.weights.values():
            w.release()
        for nw, _, _, _ in self.fused_groups.values():
            nw.release()
        for kind, wt, _ in self.convs.values():
            if kind == "1x1":
                wt.release()
        for nw, _ in self.emb_groups:
            nw.release()
        self.emb_groups.clear()
        self.emb_slices.clear()
        self.emb_cache.clear()
        self.convs.clear()
        self.norms.clear()
        self.lnorms.clear()
        self.resblocks.clear()
        self.upsamples.clear()
        self.stransformers.clear()
        self.norm_silu.clear()
        self.tblocks.clear()
        self.pending_res.clear()
        self.fused_groups.clear()
        self.fused_member.clear()
        self.pending.clear()
        self.patched.clear()
        self.weights.clear()
        self.geglu_modules.clear()
        self.enabled = False


def _gpu_linear_forward(self: torch.nn.Linear, x: torch.Tensor) -> torch.Tensor:
    rt = _RUNTIME
    entry = rt.weights.get(id(self)) if rt is not None else None
    tokens = x.numel() // x.shape[-1] if x.numel() else 0
    if entry is None or tokens < rt.min_tokens or x.device.type != "cuda":
        return torch.nn.functional.linear(x, self.weight, self.bias)
    w, bias, _name = entry
    if rt.record_only or not rt.enabled:
        if rt.record_only:
            rt.recorded.add((tokens, w.K, w.N))
        return torch.nn.functional.linear(x, self.weight, self.bias)
    out_dtype = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.float32
    res = rt.pending_res.get(id(self))
    if res is not None and out_dtype == torch.bfloat16 and res.dtype == torch.bfloat16 and \
            tuple(res.shape) == (*x.shape[:-1], w.N) and res.is_contiguous():
        del rt.pending_res[id(self)]  # consumed: the residual add happens in this GEMM's epilogue
        return rt.gemm.linear(x, w, bias, out_dtype=out_dtype, residual=res)
    key = (x.data_ptr(), tuple(x.shape), tuple(x.stride()), x._version, out_dtype)
    if id(self) in rt.fused_member:
        hit = rt.pending.pop(id(self), None)
        if hit is not None and hit[0] == key and hit[2]() is x:
            return hit[1]  # computed by the group's leading projection on this very input tensor
    group = rt.fused_groups.get(id(self))
    if group is not None:
        nw, fbias, members, n_own = group
        y = rt.gemm.linear(x, nw, fbias, out_dtype=out_dtype)
        if y.dtype != x.dtype:
            y = y.to(dtype=x.dtype)
        ref = weakref.ref(x)  # a later tensor at the same address can never match a freed input
        for mid, c0, c1 in members:
            rt.pending[mid] = (key, y[..., c0:c1], ref)
        return y[..., :n_own]
    y = rt.gemm.linear(x, w, bias, out_dtype=out_dtype)
    return y if y.dtype == x.dtype else y.to(dtype=x.dtype)


def _gpu_geglu_forward(self, x: torch.Tensor) -> torch.Tensor:
    """GEGLU.forward (`a, gate = proj(x).chunk(2, -1); a * gelu(gate)`) as one GEMM whose epilogue gates: the
    2n-wide projection never reaches memory. Falls back to the module's own forward exactly where its Linear
    would (runtime off, discovery pass, too few tokens, CPU tensors)."""
    rt = _RUNTIME
    proj = self.proj
    entry = rt.weights.get(id(proj)) if rt is not None else None
    tokens = x.numel() // x.shape[-1] if x.numel() else 0
    if (entry is None or not rt.enabled or rt.record_only or tokens < rt.min_tokens or x.device.type != "cuda"
            or id(self) not in rt.patched):
        if rt is not None and id(self) in rt.patched:
            return rt.patched[id(self)][1](x)
        a, gate = proj(x).chunk(2, dim=-1)
        return a * torch.nn.functional.gelu(gate)
    w, bias, _name = entry
    out_dtype = x.dtype if x.dtype in (torch.bfloat16, torch.float32) else torch.float32
    y = rt.gemm.linear_geglu(x, w, bias, out_dtype=out_dtype)
    return y if y.dtype == x.dtype else y.to(dtype=x.dtype)


def _out_linear(m):
    """The Linear at the end of an attention's to_out (a Linear, or Linear + Dropout) or a feed-forward's net."""
    if isinstance(m, torch.nn.Linear):
        return m
    if isinstance(m, torch.nn.Sequential) and len(m) and isinstance(m[0], torch.nn.Linear) and \
            all(isinstance(t, (torch.nn.Dropout, torch.nn.Identity)) for t in list(m)[1:]):
        return m[0]
    return None


def _tblock_plan(mod, rt):
    """(attn1 out Linear, attn2 out Linear, feed-forward out Linear) of an SD-style BasicTransformerBlock whose
    three were taken over, or None."""
    if type(mod).__name__ != "BasicTransformerBlock":
        return None
    try:
        a1, a2, ff = mod.attn1, mod.attn2, mod.ff
        mod.norm1, mod.norm2, mod.norm3
        net = ff.net
    except AttributeError:
        return None
    o1, o2 = _out_linear(getattr(a1, "to_out", None)), _out_linear(getattr(a2, "to_out", None))
    o3 = net[-1] if isinstance(net, torch.nn.Sequential) and isinstance(net[-1], torch.nn.Linear) else None
    if any(o is None or id(o) not in rt.weights for o in (o1, o2, o3)):
        return None
    return (o1, o2, o3)


def _with_residual(rt, lin, res, fn):
    """fn() with `res` offered to Linear `lin` as its epilogue residual; added here if the Linear did not take it
    (its own forward ran, or shapes differed), so the result is x + f(x) either way."""
    rt.pending_res[id(lin)] = res
    try:
        y = fn()
    finally:
        left = rt.pending_res.pop(id(lin), None)
    return y + res if left is not None else y


def _gpu_tblock_forward(self, x, context=None, transformer_options=None, **kwargs):
    """BasicTransformerBlock.forward with its three residual adds in the output GEMMs' epilogues:
    x = x + attn1(norm1 x); x = x + attn2(norm2 x, context); x = x + ff(norm3 x). Blocks with ComfyUI patches,
    disabled self-attention or extra arguments keep their own forward."""
    rt = _RUNTIME
    to = transformer_options if transformer_options is not None else {}
    plan = rt.tblocks.get(id(self)) if rt is not None else None
    if (plan is None or not _runtime_on(rt) or kwargs or self.training or not x.is_cuda or x.dtype != torch.bfloat16
            or not x.is_contiguous() or to.get("patches") or to.get("patches_replace")
            or getattr(self, "disable_self_attn", False)):
        return rt.patched[id(self)][1](x, context, transformer_options, **kwargs)
    o1, o2, o3 = plan
    x = _with_residual(rt, o1, x, lambda: self.attn1(self.norm1(x), context=None, transformer_options=to))
    x = _with_residual(rt, o2, x, lambda: self.attn2(self.norm2(x), context=context, transformer_options=to))
    x = _with_residual(rt, o3, x, lambda: self.ff(self.norm3(x)))
    return x


def _cl_bf16(x) -> bool:
    """A channels-last bf16 CUDA activation (its NHWC view is contiguous)."""
    return (isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 4
            and x.is_contiguous(memory_format=torch.channels_last))


def _conv_tiles(h: int, w: int) -> bool:
    """Image shapes the implicit-GEMM convolution tiles: 128-pixel tiles of whole rows (or whole images)."""
    if w > 128 or 128 % w:
        return False
    th = min(h, 128 // w)
    return h % th == 0 and 128 % (th * w) == 0


def _runtime_on(rt) -> bool:
    return rt is not None and rt.enabled and not rt.record_only


def _gpu_conv_forward(self, x: torch.Tensor) -> torch.Tensor:
    """Conv2d.forward on the B200 kernels for channels-last bf16 activations: 3x3 on the implicit-GEMM
    convolution, 1x1 on the GEMM; the result is channels-last."""
    rt = _RUNTIME
    entry = rt.convs.get(id(self)) if rt is not None else None
    n, c, h, w = x.shape if x.dim() == 4 else (0, 0, 0, 0)
    if entry is None or not _runtime_on(rt) or not _cl_bf16(x) or (entry[0] == "3x3" and not _conv_tiles(h, w)):
        return rt.patched[id(self)][1](x) if rt is not None and id(self) in rt.patched else \
            torch.nn.Conv2d.forward(self, x)
    from . import kernels
    rt.conv_calls += 1
    kind, wt, bias = entry
    if kind == "3x3":
        out = torch.empty((n, self.out_channels, h, w), dtype=torch.bfloat16, device=x.device,
                          memory_format=torch.channels_last)
        kernels.conv3x3(x.permute(0, 2, 3, 1), wt, bias, out=out.permute(0, 2, 3, 1))
        return out
    res = rt.pending_res.get(id(self))
    if res is not None and _cl_bf16(res) and tuple(res.shape) == (n, self.out_channels, h, w):
        del rt.pending_res[id(self)]  # consumed: the residual add happens in this GEMM's epilogue
        y = rt.gemm.linear(x.permute(0, 2, 3, 1), wt, bias, out_dtype=torch.bfloat16,
                           residual=res.permute(0, 2, 3, 1))
    else:
        y = rt.gemm.linear(x.permute(0, 2, 3, 1), wt, bias, out_dtype=torch.bfloat16)  # [n, h, w, cout]
    return y.permute(0, 3, 1, 2)


def _own_forward(rt, mod):
    """The forward a module had before the takeover (its class's forward once the runtime is gone)."""
    if rt is not None and id(mod) in rt.patched:
        return rt.patched[id(mod)][1]
    return types.MethodType(type(mod).forward, mod)


def _gpu_upsample_forward(self, x, *args, **kwargs):
    """Upsample.forward (nearest-neighbour 2x, then the 3x3 convolution) with the 2x step on the NHWC upsampling
    kernel for channels-last bf16 activations. A target size other than exactly 2x (the `output_shape` a UNet passes
    for odd encoder sizes) and every other input keep the module's own forward."""
    rt = _RUNTIME
    orig = _own_forward(rt, self)
    output_shape = kwargs.get("output_shape", args[0] if args else None)
    if (rt is None or id(self) not in rt.upsamples or not _runtime_on(rt) or not _cl_bf16(x) or x.shape[1] % 8
            or len(args) > 1 or any(k != "output_shape" for k in kwargs)
            or (output_shape is not None and tuple(output_shape[2:4]) != (2 * x.shape[2], 2 * x.shape[3]))):
        return orig(x, *args, **kwargs)
    from . import kernels
    return self.conv(kernels.upsample_nearest2x(x))


def _gpu_norm_silu_conv_forward(self, x):
    """Sequential(GroupNorm, SiLU, convolution).forward with the SiLU applied inside the NHWC GroupNorm kernel for
    channels-last bf16 activations (one launch and one activation round trip fewer); the convolution is the
    module's own (the B200 kernel where it was taken over)."""
    rt = _RUNTIME
    plan = rt.norm_silu.get(id(self)) if rt is not None else None
    if plan is None or not _runtime_on(rt) or not _cl_bf16(x) or x.shape[1] % 8:
        return _own_forward(rt, self)(x)
    from . import kernels
    gn, conv = plan
    gamma, beta = rt.norms[id(gn)]
    t = torch.empty_like(x, memory_format=torch.channels_last)
    kernels.group_norm(x.permute(0, 2, 3, 1), gn.num_groups, gamma, beta, eps=gn.eps, silu=True,
                       out=t.permute(0, 2, 3, 1))
    return conv(t)


def _stransformer_plan(mod, rt):
    """(GroupNorm, proj_in, proj_out) of an SD1.5-style SpatialTransformer (GroupNorm, 1x1 convolution in and out
    around its transformer blocks, + x) whose three were taken over, or None. Linear-projection variants keep
    their own forward."""
    if type(mod).__name__ != "SpatialTransformer" or getattr(mod, "use_linear", False):
        return None
    norm, pin, pout = (getattr(mod, nm, None) for nm in ("norm", "proj_in", "proj_out"))
    if not isinstance(getattr(mod, "transformer_blocks", None), torch.nn.ModuleList) or id(norm) not in rt.norms:
        return None
    if rt.convs.get(id(pin), ("",))[0] != "1x1" or rt.convs.get(id(pout), ("",))[0] != "1x1":
        return None
    return (norm, pin, pout)


def _gpu_spatial_transformer_forward(self, x, *args, **kwargs):
    """SpatialTransformer.forward: x + proj_out(blocks(proj_in(norm(x)))) over the (b, h*w, c) tokens of a
    channels-last activation (views, no copies), with the closing residual add in proj_out's GEMM epilogue. The
    context may be one tensor or one per block, and transformer_options gets the block index before each block,
    as in the UNet's own forward. Inputs with ComfyUI patches or anything else keep the module's own forward."""
    rt = _RUNTIME
    orig = _own_forward(rt, self)
    names = ("context", "transformer_options")
    plan = rt.stransformers.get(id(self)) if rt is not None else None
    bound = dict(zip(names, args))
    bound.update(kwargs)
    to = bound.get("transformer_options")
    if (plan is None or not _runtime_on(rt) or len(args) > 2 or any(k not in names for k in kwargs)
            or self.training or not _cl_bf16(x) or (to is not None and not isinstance(to, dict))
            or (to or {}).get("patches") or (to or {}).get("patches_replace")):
        return orig(x, *args, **kwargs)
    norm, proj_in, proj_out = plan
    blocks = self.transformer_blocks
    context = bound.get("context")
    if not isinstance(context, list):
        context = [context] * len(blocks)
    b, c, h, w = x.shape
    if to is not None:
        to["activations_shape"] = list(x.shape)
    t = proj_in(norm(x))
    t = t.permute(0, 2, 3, 1).reshape(b, h * w, t.shape[1])
    for i, blk in enumerate(blocks):
        if to is not None:
            to["block_index"] = i
        t = blk(t, context=context[i], transformer_options=to if to is not None else {})
    t = t.reshape(b, h, w, t.shape[-1]).permute(0, 3, 1, 2)
    return _with_residual(rt, proj_out, x, lambda: proj_out(t))


def _gpu_group_norm_forward(self, x: torch.Tensor) -> torch.Tensor:
    """GroupNorm.forward on the NHWC GroupNorm kernel for channels-last bf16 activations (torch's own kernel would
    reorder them to NCHW and back)."""
    rt = _RUNTIME
    entry = rt.norms.get(id(self)) if rt is not None else None
    if entry is None or not _runtime_on(rt) or not _cl_bf16(x):
        return rt.patched[id(self)][1](x) if rt is not None and id(self) in rt.patched else \
            torch.nn.GroupNorm.forward(self, x)
    from . import kernels
    out = torch.empty_like(x, memory_format=torch.channels_last)
    kernels.group_norm(x.permute(0, 2, 3, 1), self.num_groups, entry[0], entry[1], eps=self.eps,
                       out=out.permute(0, 2, 3, 1))
    return out


def _gpu_layer_norm_forward(self, x: torch.Tensor) -> torch.Tensor:
    """LayerNorm.forward (norm1/norm2/norm3 of a taken-over transformer block) on the row-wise LayerNorm kernel for
    contiguous bf16 CUDA activations; anything else takes the module's own forward."""
    rt = _RUNTIME
    entry = rt.lnorms.get(id(self)) if rt is not None else None
    if (entry is None or not _runtime_on(rt) or not isinstance(x, torch.Tensor) or not x.is_cuda
            or x.dtype != torch.bfloat16 or not x.is_contiguous() or x.shape[-1] != entry[0].shape[0]):
        return rt.patched[id(self)][1](x) if rt is not None and id(self) in rt.patched else \
            torch.nn.LayerNorm.forward(self, x)
    from . import kernels
    return kernels.layer_norm(x, entry[0], entry[1], eps=self.eps)


def _resblock_plan(mod, rt):
    """The fused plan of an SD-style ResBlock (in_layers = GroupNorm, SiLU, 3x3 conv; emb_layers = SiLU, Linear;
    out_layers = GroupNorm, SiLU, [Dropout], 3x3 conv; skip = identity or 1x1 conv) whose parts were taken over,
    or None. Blocks with up/down-sampling or scale-shift conditioning keep their own forward."""
    if type(mod).__name__ != "ResBlock":
        return None
    if getattr(mod, "updown", False) or getattr(mod, "use_scale_shift_norm", False) or \
            getattr(mod, "skip_t_emb", False) or getattr(mod, "exchange_temb_dims", False):
        return None
    try:
        il, ol, el, skip = mod.in_layers, mod.out_layers, mod.emb_layers, mod.skip_connection
    except AttributeError:
        return None
    if not (len(il) == 3 and isinstance(il[0], torch.nn.GroupNorm) and isinstance(il[1], torch.nn.SiLU)
            and isinstance(il[2], torch.nn.Conv2d) and isinstance(ol[0], torch.nn.GroupNorm)
            and isinstance(ol[1], torch.nn.SiLU) and isinstance(ol[-1], torch.nn.Conv2d)
            and all(isinstance(m, torch.nn.Dropout) for m in list(ol)[2:-1])):
        return None
    if not (len(el) == 2 and isinstance(el[0], torch.nn.SiLU) and isinstance(el[1], torch.nn.Linear)):
        return None
    conv1, conv2 = il[2], ol[-1]
    if rt.convs.get(id(conv1), ("",))[0] != "3x3" or rt.convs.get(id(conv2), ("",))[0] != "3x3":
        return None
    if id(il[0]) not in rt.norms or id(ol[0]) not in rt.norms:
        return None
    if not isinstance(skip, torch.nn.Identity) and rt.convs.get(id(skip), ("",))[0] != "1x1":
        return None
    return (il[0], conv1, ol[0], conv2, skip)


def _resblock_emb_rows(rt, block, emb, conv1) -> torch.Tensor:
    """conv1's per-image bias rows, emb_layers(emb) + conv1.bias in f32: a column slice of the grouped projection of
    all ResBlocks, computed by the first ResBlock that sees this `emb` tensor (identity and version checked)."""
    ent = rt.emb_slices.get(id(block))
    if ent is None or not isinstance(emb, torch.Tensor) or not emb.is_cuda:
        e = block.emb_layers(emb).float()
        b1 = rt.convs[id(conv1)][2]
        return (e + b1 if b1 is not None else e).contiguous()
    gi, off, cout = ent
    cached = rt.emb_cache.get(gi)
    if cached is None or cached[0]() is not emb or cached[1] != emb._version:
        nw, bias = rt.emb_groups[gi]
        e_all = rt.gemm.linear(torch.nn.functional.silu(emb), nw, bias, out_dtype=torch.float32)
        cached = (weakref.ref(emb), emb._version, e_all)
        rt.emb_cache[gi] = cached
    return cached[2][:, off:off + cout]


# Largest ResBlock activation (pixels over the batch) whose skip convolution runs on the side stream: 8192 pixels are
# 64 convolution row tiles, well under one wave of tiles on 148 SMs (batch 2 at the 64x64 latent's top level).
_SIDE_STREAM_MAX_PIXELS = 8192


def _gpu_resblock_forward(self, x, emb, *args, **kwargs):
    """ResBlock.forward in four launches plus the small time-embedding Linear: GroupNorm+SiLU, conv1 with the
    bias row of each image = conv bias + emb_layers(emb), GroupNorm+SiLU, conv2 with the skip path (x or its 1x1
    convolution) added in the epilogue. For small activations (at most 8192 pixels, where the convolutions' grids
    do not fill the GPU) a 1x1 skip convolution runs on a second stream, forked before the first GroupNorm and
    joined before conv2, so it overlaps the latency-bound main chain (a parallel branch in a captured graph);
    larger ones keep it in line, where it would only contend with a main chain that already fills the GPU."""
    rt = _RUNTIME
    plan = rt.resblocks.get(id(self)) if rt is not None else None
    if plan is None or not _runtime_on(rt) or not _cl_bf16(x) or self.training or args or \
            any(k != "transformer_options" for k in kwargs) or not _conv_tiles(x.shape[2], x.shape[3]):
        return rt.patched[id(self)][1](x, emb, *args, **kwargs)
    from . import kernels
    rt.conv_calls += 1
    gn1, conv1, gn2, conv2, skip = plan
    n, c, h, w = x.shape
    xh = x.permute(0, 2, 3, 1)
    main = side = None
    if not isinstance(skip, torch.nn.Identity):
        _kind, ws, bs = rt.convs[id(skip)]
        if n * h * w <= _SIDE_STREAM_MAX_PIXELS:
            main = torch.cuda.current_stream(x.device)
            side = rt.side_stream(x.device)
            side.wait_stream(main)
            with torch.cuda.stream(side):
                res = rt.gemm.linear(xh, ws, bs, out_dtype=torch.bfloat16)
        else:
            res = rt.gemm.linear(xh, ws, bs, out_dtype=torch.bfloat16)
    t1 = torch.empty_like(xh)
    g1 = rt.norms[id(gn1)]
    kernels.group_norm(xh, gn1.num_groups, g1[0], g1[1], eps=gn1.eps, silu=True, out=t1)
    rows = _resblock_emb_rows(rt, self, emb, conv1)  # [n, cout] f32: conv bias + time embedding per image
    cout = conv1.out_channels
    h1 = torch.empty((n, h, w, cout), dtype=torch.bfloat16, device=x.device)
    kernels.conv3x3(t1, rt.convs[id(conv1)][1], rows, out=h1)
    g2 = rt.norms[id(gn2)]
    kernels.group_norm(h1, gn2.num_groups, g2[0], g2[1], eps=gn2.eps, silu=True, out=h1)
    if isinstance(skip, torch.nn.Identity):
        res = xh
    elif side is not None:
        main.wait_stream(side)
        res.record_stream(main)  # allocated on the side stream, read and released on this one
    out = torch.empty((n, conv2.out_channels, h, w), dtype=torch.bfloat16, device=x.device,
                      memory_format=torch.channels_last)
    kernels.conv3x3(h1, rt.convs[id(conv2)][1], rt.convs[id(conv2)][2], residual=res, out=out.permute(0, 2, 3, 1))
    return out


def _gpu_attention_override(func, q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                            skip_output_reshape=False, **kwargs):
    """transformer_options["optimized_attention_override"] (the reference's _npu_attention_override,
    node :161-247): route the block to the fused kernel variant the gate picked."""
    rt = _RUNTIME

    def model_attn():
        return func(q, k, v, heads, mask=mask, attn_precision=attn_precision, skip_reshape=skip_reshape,
                    skip_output_reshape=skip_output_reshape, **kwargs)

    if rt is None or not (rt.enabled or rt.record_only) or q.device.type != "cuda":
        return model_attn()
    gate = rt.attn
    if skip_reshape:
        b, h, tq, d = q.shape
        tk = k.shape[2]
    else:
        b, tq, inner = q.shape
        h, d = heads, inner // heads
        tk = k.shape[1]
    key = (b, tq, tk, h, d)
    fits = rt.gemm.attention_fits(tq, tk, d, b * h)
    why = gate.model_route_reason(key, mask is not None, bool(kwargs.get("enable_gqa", False)), fits)
    if why is not None or rt.record_only:
        t0 = time.perf_counter()
        out = model_attn()
        gate.model_seconds += time.perf_counter() - t0
        gate.model_calls += 1
        return out
    scale = kwargs.get("scale", None)
    out_dtype = q.dtype if q.dtype in (torch.bfloat16, torch.float32) else torch.float32

    def fused(variant):
        from . import kernels
        qd, kd, vd = (rt.gemm._attn_operand(t) for t in (q, k, v))
        return kernels.attention(qd, kd, vd, h, scale=scale, head_major_in=skip_reshape,
                                 head_major_out=skip_output_reshape, out_dtype=out_dtype, variant=variant)

    rec = gate.record(key)
    if rec.variant is None:
        # First call of this shape: time the variants (each after one warm-up launch), then check the first
        # result against the model's own attention, also timed after a warm-up call.
        y = None
        for var in (attn_variants(d) if gate.mode == "auto" else (0,)):
            fused(var)
            y_v, rec.variant_ms[var] = _time_gpu(lambda: fused(var), rt.gemm.device)
            y = y_v if y is None else y
        model_attn()
        ref, rec.model_ms = _time_gpu(model_attn, rt.gemm.device)
        err = float((y.float() - ref.float()).abs().max() / (ref.float().abs().max() + 1e-12))
        rec.max_rel_err = err
        if not np.isfinite(err) or err > 0.1:
            raise RuntimeError(f"fused attention result for {key} does not match the model's attention "
                               f"(max rel err {err:.3g})")
        rec.variant = min(rec.variant_ms, key=rec.variant_ms.get)
        _log(f"attention gate {key}: {rec.describe()}")
    t0 = time.perf_counter()
    y = fused(rec.variant)
    gate.fused_seconds += time.perf_counter() - t0
    gate.fused_calls += 1
    gate.fused_flops += 4.0 * b * h * tq * tk * d
    return y


def _get_runtime(device=None) -> B200Runtime:
    global _RUNTIME
    with _RUNTIME_LOCK:
        if _RUNTIME is None:
            t0 = time.perf_counter()
            _RUNTIME = B200Runtime(device)
            _log(f"GPU runtime ready in {time.perf_counter() - t0:.1f}s")
        return _RUNTIME


class B200LinearOffload:
    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "model": ("MODEL",),
                "enabled": ("BOOLEAN", {"default": True}),
                "min_tokens": ("INT", {"default": 64, "min": 1, "max": 65536,
                                       "tooltip": "Linear calls with fewer rows than this use torch's own linear"}),
                "min_features": ("INT", {"default": 320, "min": 1, "max": 65536,
                                         "tooltip": "Linear layers narrower than this are not taken over"}),
                "skip_names": ("STRING", {"default": "time_embed,label_emb,emb_layers",
                                          "tooltip": "comma-separated substrings of module names to leave alone"}),
            },
            "optional": {
                "attention": (ATTENTION_MODES, {"default": "auto",
                                                "tooltip": "auto = time the fused kernel's variants per shape once "
                                                           "and keep the fastest, gpu = default variant, off = the "
                                                           "model's own attention"}),
                "attn_min_tokens": ("INT", {"default": 1, "min": 1, "max": 65536,
                                            "tooltip": "attention calls with fewer query tokens use the model's "
                                                       "own attention (1: every unmasked call runs the fused "
                                                       "kernel)"}),
                "convolutions": ("BOOLEAN", {"default": True,
                                             "tooltip": "also run 3x3/1x1 convolutions, GroupNorms and ResBlocks "
                                                        "of channels-last bf16 models on the B200 kernels"}),
            },
        }

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "apply"
    CATEGORY = "GPU/B200"
    DESCRIPTION = "Runs the model's Linear layers and attention on hand-written B200 (sm_100a) kernels."

    def apply(self, model, enabled, min_tokens, min_features, skip_names, attention="auto", attn_min_tokens=1,
              convolutions=True):
        if not enabled:
            return (model,)
        rt = _get_runtime()
        rt.min_tokens = int(min_tokens)
        mode = _mode(attention)
        if mode != rt.attn.mode or int(attn_min_tokens) != rt.attn.min_tokens:
            rt.attn.reset()
            _log(f"attention mode {rt.attn.mode} -> {mode} (min tokens {attn_min_tokens}); gate decisions reset")
        rt.attn.mode = mode
        rt.attn.min_tokens = int(attn_min_tokens)
        skip = tuple(s.strip() for s in skip_names.split(",") if s.strip())
        state = {"prepared": False}

        def snapshot():
            rt.gemm.flush_timing()
            g, a = rt.gemm.stats, rt.attn
            return dict(g, attn_gpu=a.fused_calls, attn_model=a.model_calls, attn_gpu_s=a.fused_seconds,
                        attn_model_s=a.model_seconds, attn_flops=a.fused_flops)

        def wrapper(apply_model, args):
            x, t, c = args["input"], args["timestep"], args["c"]
            dm = model.model.diffusion_model
            with _RUNTIME_LOCK:
                if not state["prepared"]:
                    # Weights are taken after the ModelPatcher applied its patches (LoRA etc.), i.e. now.
                    t0 = time.perf_counter()
                    n = rt.take_over(dm, int(min_features), skip, bool(convolutions))
                    _log(f"took over {n} new Linear layers ({len(rt.weights)} total) in {time.perf_counter() - t0:.1f}s")
                    # One pass with the model's own ops records every (tokens, K, N) so the kernels are warmed up
                    # for each shape before the first accelerated run.
                    rt.record_only, rt.enabled = True, False
                    t0 = time.perf_counter()
                    apply_model(x, t, **c)
                    rt.record_only = False
                    shapes = sorted(rt.recorded)
                    rt.gemm.prepare(shapes)
                    _log(f"shape-discovery pass {time.perf_counter() - t0:.1f}s; warmed {len(shapes)} GEMM shapes")
                    state["prepared"] = True
                rt.enabled = True
                s0 = snapshot()
                t0 = time.perf_counter()
                try:
                    out = apply_model(x, t, **c)
                finally:
                    rt.enabled = False
                torch.cuda.synchronize(rt.gemm.device)
                wall = time.perf_counter() - t0
                s1 = snapshot()
                gpu_s = s1["npu_seconds"] - s0["npu_seconds"]
                gemm_wall = s1["total_seconds"] - s0["total_seconds"]
                calls = s1["calls"] - s0["calls"]
                fl = s1["flops"] - s0["flops"]
                an, am = s1["attn_gpu"] - s0["attn_gpu"], s1["attn_model"] - s0["attn_model"]
                an_s, am_s = s1["attn_gpu_s"] - s0["attn_gpu_s"], s1["attn_model_s"] - s0["attn_model_s"]
                afl = s1["attn_flops"] - s0["attn_flops"]
                rt.calls += 1
                rt.last_summary = (
                    f"UNet call {rt.calls}: {wall:.3f}s wall | {calls} Linear GEMMs on GPU: {fl / 1e9:.0f} GFLOP, "
                    f"GPU {gpu_s:.3f}s timed ({fl / max(gpu_s, 1e-9) / 1e9:.0f} GFLOPS), GEMM host {gemm_wall:.3f}s "
                    f"| attention: {an} calls on the fused kernel ({an_s:.3f}s host, {afl / 1e9:.0f} GFLOP), "
                    f"{am} on the model's own ({am_s:.3f}s)")
                _log(rt.last_summary)
            return out

        m = model.clone()
        m.set_model_unet_function_wrapper(wrapper)
        to = m.model_options.setdefault("transformer_options", {})
        to["optimized_attention_override"] = _gpu_attention_override
        return (m,)


class B200Status:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"trigger": ("IMAGE",)}}

    RETURN_TYPES = ("STRING",)
    FUNCTION = "status"
    CATEGORY = "GPU/B200"
    OUTPUT_NODE = True

    def status(self, trigger):
        rt = _RUNTIME
        if rt is None:
            s = "B200 runtime not started"
        else:
            s = (rt.gemm.summary() + " | layers on GPU kernels: %d (GEGLU blocks fused: %d, q/k/v groups in one GEMM: "
                 "%d) | %s | last: %s" % (len(rt.weights), len(rt.geglu_modules), len(rt.fused_groups),
                                          rt.attn.summary(), rt.last_summary))
        _log(s)
        return {"ui": {"text": [s]}, "result": (s,)}


class B200Release:
    @classmethod
    def INPUT_TYPES(cls):
        return {"required": {"model": ("MODEL",)}}

    RETURN_TYPES = ("MODEL",)
    FUNCTION = "release"
    CATEGORY = "GPU/B200"

    def release(self, model):
        if _RUNTIME is not None:
            _RUNTIME.release()
            _log("released all Linear layers back to torch")
        return (model,)


NODE_CLASS_MAPPINGS = {
    "B200LinearOffload": B200LinearOffload,
    "B200Status": B200Status,
    "B200Release": B200Release,
    # the reference's class names (node :400-404), so workflows saved against it load unchanged
    "XDNA1NpuLinearOffload": B200LinearOffload,
    "XDNA1NpuStatus": B200Status,
    "XDNA1NpuRelease": B200Release,
}
NODE_DISPLAY_NAME_MAPPINGS = {
    "B200LinearOffload": "B200: Offload Linear layers",
    "B200Status": "B200: Status",
    "B200Release": "B200: Release",
    "XDNA1NpuLinearOffload": "B200: Offload Linear layers (XDNA1 workflow name)",
    "XDNA1NpuStatus": "B200: Status (XDNA1 workflow name)",
    "XDNA1NpuRelease": "B200: Release (XDNA1 workflow name)",
}
