"""An SD1.5-architecture UNet (random init, seeded) and an Euler sampler: the end-to-end harness for the hot path.

The reference runs SD1.5 inside ComfyUI, whose UNet code and checkpoints are not part of it (or of this
environment). This module is an independent implementation of the same architecture from its published
description, so the integration can be exercised and timed: in_channels 4; channels 320 / 640 / 1280 / 1280;
2 ResBlocks per level; one transformer block (self-attention, cross-attention to a 768-wide text context, GEGLU
feed-forward x4) per attention level; 8 heads (head dims 40 / 80 / 160). That gives the reference's Linear
inventory: 10 nn.Linear per transformer block x 16 blocks = 160 GEMMs per UNet call (docs/02-results.md:279),
plus the time-embedding Linears the reference keeps off the NPU by name (skip_names, comfyui node :271).

Hooks that mirror ComfyUI's, so the reference's node logic applies unchanged:
  * every Linear is a plain torch.nn.Linear (the node swaps its `forward`, comfyui node :119-136);
  * attention calls `transformer_options["optimized_attention_override"](func, q, k, v, heads, ...)` when set
    (installed by the node, comfyui node :358-359), with `func` the model's own attention (torch SDPA).
The one place the model itself calls this package is the decoder's skip concatenation, which lives in the UNet's
forward rather than in a module the node can take over: channels-last bf16/f16 CUDA activations are concatenated
by the NHWC concatenation kernel, everything else (CPU runs, f32) by torch.cat.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


def sdpa_attention(q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False, skip_output_reshape=False,
                   **kwargs):
    """The model's own attention (ComfyUI's `optimized_attention` signature): torch SDPA."""
    if skip_reshape:
        b, h, tq, d = q.shape
        qh, kh, vh = q, k, v
    else:
        b, tq, inner = q.shape
        h, d = heads, inner // heads
        qh, kh, vh = (t.view(b, -1, h, d).transpose(1, 2) for t in (q, k, v))
    o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, scale=kwargs.get("scale"))
    if skip_output_reshape:
        return o
    return o.transpose(1, 2).reshape(b, tq, h * d)


class CrossAttention(nn.Module):
    def __init__(self, dim: int, context_dim: int | None, heads: int):
        super().__init__()
        self.heads = heads
        cd = context_dim or dim
        self.to_q = nn.Linear(dim, dim, bias=False)
        self.to_k = nn.Linear(cd, dim, bias=False)
        self.to_v = nn.Linear(cd, dim, bias=False)
        self.to_out = nn.Linear(dim, dim)

    def forward(self, x, context=None, transformer_options=None):
        ctx = x if context is None else context
        q, k, v = self.to_q(x), self.to_k(ctx), self.to_v(ctx)
        override = (transformer_options or {}).get("optimized_attention_override")
        if override is not None:
            o = override(sdpa_attention, q, k, v, self.heads, mask=None, attn_precision=None, skip_reshape=False,
                         skip_output_reshape=False, _inside_attn_wrapper=True)
        else:
            o = sdpa_attention(q, k, v, self.heads)
        return self.to_out(o.to(x.dtype))


class GEGLU(nn.Module):
    def __init__(self, dim: int, inner: int):
        super().__init__()
        self.proj = nn.Linear(dim, inner * 2)

    def forward(self, x):
        a, gate = self.proj(x).chunk(2, dim=-1)
        return a * F.gelu(gate)


class FeedForward(nn.Module):
    def __init__(self, dim: int, mult: int = 4):
        super().__init__()
        self.net = nn.Sequential(GEGLU(dim, dim * mult), nn.Identity(), nn.Linear(dim * mult, dim))

    def forward(self, x):
        return self.net(x)


class BasicTransformerBlock(nn.Module):
    def __init__(self, dim: int, heads: int, context_dim: int):
        super().__init__()
        self.attn1 = CrossAttention(dim, None, heads)
        self.ff = FeedForward(dim)
        self.attn2 = CrossAttention(dim, context_dim, heads)
        self.norm1, self.norm2, self.norm3 = nn.LayerNorm(dim), nn.LayerNorm(dim), nn.LayerNorm(dim)

    def forward(self, x, context, transformer_options=None):
        x = x + self.attn1(self.norm1(x), None, transformer_options)
        x = x + self.attn2(self.norm2(x), context, transformer_options)
        return x + self.ff(self.norm3(x))


class SpatialTransformer(nn.Module):
    def __init__(self, channels: int, heads: int, context_dim: int):
        super().__init__()
        self.norm = nn.GroupNorm(32, channels, eps=1e-6)
        self.proj_in = nn.Conv2d(channels, channels, 1)
        self.transformer_blocks = nn.ModuleList([BasicTransformerBlock(channels, heads, context_dim)])
        self.proj_out = nn.Conv2d(channels, channels, 1)

    def forward(self, x, context, transformer_options=None):
        b, c, h, w = x.shape
        res = x
        x = self.proj_in(self.norm(x))
        x = x.permute(0, 2, 3, 1).reshape(b, h * w, c)
        for blk in self.transformer_blocks:
            x = blk(x, context, transformer_options)
        x = x.reshape(b, h, w, c).permute(0, 3, 1, 2)
        return self.proj_out(x) + res


class ResBlock(nn.Module):
    def __init__(self, cin: int, cout: int, emb_dim: int):
        super().__init__()
        self.in_layers = nn.Sequential(nn.GroupNorm(32, cin), nn.SiLU(), nn.Conv2d(cin, cout, 3, padding=1))
        self.emb_layers = nn.Sequential(nn.SiLU(), nn.Linear(emb_dim, cout))
        self.out_layers = nn.Sequential(nn.GroupNorm(32, cout), nn.SiLU(), nn.Conv2d(cout, cout, 3, padding=1))
        self.skip_connection = nn.Identity() if cin == cout else nn.Conv2d(cin, cout, 1)

    def forward(self, x, emb):
        h = self.in_layers(x)
        h = h + self.emb_layers(emb)[:, :, None, None].to(h.dtype)
        return self.skip_connection(x) + self.out_layers(h)


class Downsample(nn.Module):
    def __init__(self, ch: int):
        super().__init__()
        self.op = nn.Conv2d(ch, ch, 3, stride=2, padding=1)

    def forward(self, x):
        return self.op(x)


class Upsample(nn.Module):
    def __init__(self, ch: int):
        super().__init__()
        self.conv = nn.Conv2d(ch, ch, 3, padding=1)

    def forward(self, x):
        return self.conv(F.interpolate(x, scale_factor=2.0, mode="nearest"))


def cat_channels(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """torch.cat([a, b], dim=1) of the decoder activation and its skip tensor."""
    if (a.is_cuda and a.dim() == 4 and a.dtype in (torch.bfloat16, torch.float16) and b.dtype == a.dtype
            and a.shape[1] % 8 == 0 and b.shape[1] % 8 == 0 and a.is_contiguous(memory_format=torch.channels_last)
            and b.is_contiguous(memory_format=torch.channels_last)):
        from . import kernels
        return kernels.concat_channels(a, b)
    return torch.cat([a, b], dim=1)


def timestep_embedding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    args = t.float()[:, None] * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


class SD15UNet(nn.Module):
    """UNet of the SD1.5 architecture. forward(x [B,4,H,W], timesteps [B], context [B,77,768]) -> eps [B,4,H,W]."""

    def __init__(self, in_channels: int = 4, model_channels: int = 320, channel_mult=(1, 2, 4, 4),
                 num_res_blocks: int = 2, attention_levels=(0, 1, 2), heads: int = 8, context_dim: int = 768):
        super().__init__()
        self.model_channels = model_channels
        emb_dim = model_channels * 4
        self.time_embed = nn.Sequential(nn.Linear(model_channels, emb_dim), nn.SiLU(), nn.Linear(emb_dim, emb_dim))
        self.input_blocks = nn.ModuleList([nn.ModuleList([nn.Conv2d(in_channels, model_channels, 3, padding=1)])])
        chans = [model_channels]
        ch = model_channels
        for level, mult in enumerate(channel_mult):
            for _ in range(num_res_blocks):
                layers = [ResBlock(ch, mult * model_channels, emb_dim)]
                ch = mult * model_channels
                if level in attention_levels:
                    layers.append(SpatialTransformer(ch, heads, context_dim))
                self.input_blocks.append(nn.ModuleList(layers))
                chans.append(ch)
            if level != len(channel_mult) - 1:
                self.input_blocks.append(nn.ModuleList([Downsample(ch)]))
                chans.append(ch)
        self.middle_block = nn.ModuleList([ResBlock(ch, ch, emb_dim), SpatialTransformer(ch, heads, context_dim),
                                           ResBlock(ch, ch, emb_dim)])
        self.output_blocks = nn.ModuleList()
        for level, mult in list(enumerate(channel_mult))[::-1]:
            for i in range(num_res_blocks + 1):
                skip = chans.pop()
                layers = [ResBlock(ch + skip, mult * model_channels, emb_dim)]
                ch = mult * model_channels
                if level in attention_levels:
                    layers.append(SpatialTransformer(ch, heads, context_dim))
                if level and i == num_res_blocks:
                    layers.append(Upsample(ch))
                self.output_blocks.append(nn.ModuleList(layers))
        self.out = nn.Sequential(nn.GroupNorm(32, ch), nn.SiLU(), nn.Conv2d(ch, in_channels, 3, padding=1))

    def _run(self, layers, h, emb, context, transformer_options):
        for layer in layers:
            if isinstance(layer, ResBlock):
                h = layer(h, emb)
            elif isinstance(layer, SpatialTransformer):
                h = layer(h, context, transformer_options)
            else:
                h = layer(h)
        return h

    def forward(self, x, timesteps, context, transformer_options=None):
        emb = self.time_embed(timestep_embedding(timesteps, self.model_channels).to(x.dtype))
        hs = []
        h = x
        for blk in self.input_blocks:
            h = self._run(blk, h, emb, context, transformer_options)
            hs.append(h)
        h = self._run(self.middle_block, h, emb, context, transformer_options)
        for blk in self.output_blocks:
            h = cat_channels(h, hs.pop())
            h = self._run(blk, h, emb, context, transformer_options)
        return self.out(h)


def build_unet(seed: int = 0, device="cpu", dtype=torch.float32) -> SD15UNet:
    """Random-init SD1.5-architecture UNet, deterministic for a seed (no checkpoint exists in this environment)."""
    with torch.random.fork_rng(devices=[]):
        torch.manual_seed(seed)
        m = SD15UNet()
    return m.to(device=device, dtype=dtype).eval()


def karras_sigmas(n: int, sigma_min: float = 0.0292, sigma_max: float = 14.6146, rho: float = 7.0) -> torch.Tensor:
    ramp = torch.linspace(0, 1, n)
    inv_min, inv_max = sigma_min ** (1 / rho), sigma_max ** (1 / rho)
    s = (inv_max + ramp * (inv_min - inv_max)) ** rho
    return torch.cat([s, torch.zeros(1)])


def sigma_to_t(sigma: torch.Tensor) -> torch.Tensor:
    """Map a sigma to a DDPM-style timestep in [0, 999] (log-linear; the exact schedule does not matter for a
    random-init model, only that it is deterministic)."""
    return (torch.log(sigma.clamp_min(1e-4)) - math.log(0.0292)) / (math.log(14.6146) - math.log(0.0292)) * 999.0


def euler_cfg_sample(model, latent, context, uncond, steps: int = 4, cfg: float = 7.5, transformer_options=None,
                     step_callback=None):
    """Euler sampling with classifier-free guidance; the CFG pair (uncond, cond) of every prompt runs in one
    batch. latent [P, 4, h, w]; context / uncond [P, 77, 768]. Returns the final latent."""
    sigmas = karras_sigmas(steps).to(latent.device)
    x = latent * sigmas[0]
    ctx = torch.cat([uncond, context], dim=0)
    for i in range(steps):
        s = sigmas[i]
        x_in = torch.cat([x, x], dim=0) / torch.sqrt(s * s + 1.0)
        t = sigma_to_t(s).expand(x_in.shape[0]).to(latent.device)
        eps = model(x_in, t, ctx, transformer_options)
        eu, ec = eps.chunk(2, dim=0)
        e = eu + cfg * (ec - eu)
        x = x + (sigmas[i + 1] - s) * e.to(x.dtype)
        if step_callback is not None:
            step_callback(i, x)
    return x


def prompt_shard(n_prompts: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous prompt range [lo, hi) of `rank`: prompts split as evenly as possible, each prompt's CFG pair
    (uncond, cond) stays on one rank so the guidance combine and the Euler update need no communication."""
    base, extra = divmod(n_prompts, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def seeded_prompts(n_prompts: int, latent_hw: int, seed: int = 0, device="cpu", dtype=torch.float32,
                   context_len: int = 77, context_dim: int = 768):
    """Per-prompt seeded latents [P,4,h,w] ~ N(0,1), text contexts and unconditional contexts [P,77,768] ~ N(0,1).
    Each prompt draws from its own generator, so a prompt's inputs do not depend on how prompts are sharded."""
    lat, ctx, unc = [], [], []
    for p in range(n_prompts):
        g = torch.Generator().manual_seed(seed * 100003 + p)
        lat.append(torch.randn(1, 4, latent_hw, latent_hw, generator=g))
        ctx.append(torch.randn(1, context_len, context_dim, generator=g))
        unc.append(torch.randn(1, context_len, context_dim, generator=g))
    cat = lambda xs: torch.cat(xs).to(device=device, dtype=dtype)  # noqa: E731
    return cat(lat), cat(ctx), cat(unc)


def sample_sharded(model, latents, context, uncond, steps: int = 4, cfg: float = 7.5, transformer_options=None,
                   group=None):
    """Euler CFG sampling of all prompts with the batch sharded over the ranks of `group` (torch.distributed):
    each rank denoises its own prompts (both CFG halves) and the final latents are all-gathered. `latents`,
    `context`, `uncond` hold ALL prompts; every rank returns the full result. Without a process group it is plain
    single-device sampling."""
    import torch.distributed as dist
    world = dist.get_world_size(group) if (group is not None or (dist.is_available() and dist.is_initialized())) else 1
    rank = dist.get_rank(group) if world > 1 else 0
    P = latents.shape[0]
    lo, hi = prompt_shard(P, world, rank)
    mine = euler_cfg_sample(model, latents[lo:hi], context[lo:hi], uncond[lo:hi], steps=steps, cfg=cfg,
                            transformer_options=transformer_options)
    if world == 1:
        return mine
    # Uneven shards are padded to the largest one for a single all-gather, then trimmed.
    width = -(-P // world)
    padded = torch.zeros((width, *latents.shape[1:]), dtype=mine.dtype, device=mine.device)
    padded[: hi - lo] = mine
    gathered = torch.empty((world * width, *latents.shape[1:]), dtype=mine.dtype, device=mine.device)
    dist.all_gather_into_tensor(gathered, padded, group=group)
    return torch.cat([gathered[r * width: r * width + (prompt_shard(P, world, r)[1] - prompt_shard(P, world, r)[0])]
                      for r in range(world)])
