"""Fused attention parity on the B200: the tcgen05 flash kernel through the C ABI against the CPU oracle.

Semantics follow the reference's attention test (scripts/11-attn-fused-test.py: seeded q, k ~ 1.5 N(0,1) and
v ~ N(0,1), SDPA in f32 as the reference, max|err|/max|ref|, padded-stride views) and the benchmarked attention
blocks (q/k/v ~ N(0,1), scale 1/sqrt(d)), with the stated tolerance: max-abs <= 2e-2 against SDPA in f32 on
bf16-rounded inputs.
"""
import functools

import pytest
import torch

from oracle import attention_ref, rel_max_err

pytestmark = pytest.mark.gpu

TOL_ABS = 2e-2


def _qkv(B, H, Sq, Skv, D, seed=0, qk_scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, Sq, H * D, generator=g) * qk_scale).to(torch.bfloat16)
    k = (torch.randn(B, Skv, H * D, generator=g) * qk_scale).to(torch.bfloat16)
    v = torch.randn(B, Skv, H * D, generator=g).to(torch.bfloat16)
    return q, k, v


@functools.lru_cache(maxsize=8)
def _block(B, H, Sq, Skv, D, seed):
    q, k, v = _qkv(B, H, Sq, Skv, D, seed=seed)
    return q, k, v, attention_ref(q, k, v, H)


def _run(q, k, v, H, out_dtype=torch.float32, **kw):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    o = kernels.attention(q.to(dev), k.to(dev), v.to(dev), H, out_dtype=out_dtype, **kw)
    kernels.check_status(dev)
    return o


def _check(o, ref, tol=TOL_ABS):
    o = o.float().cpu()
    err = float((o - ref).abs().max())
    assert torch.isfinite(o).all(), "non-finite output"
    assert err <= tol, f"max-abs {err} (rel {rel_max_err(o, ref):.2e})"


@pytest.mark.parametrize("shape", [(2, 8, 4096, 4096, 40), (2, 8, 1024, 1024, 80), (2, 8, 256, 256, 160),
                                   (2, 8, 4096, 77, 40)],
                         ids=["self64x64_d40", "self32x32_d80", "self16x16_d160", "cross4096x77_d40"])
@pytest.mark.parametrize("variant", [0, 64, 96, 128, 1064, 1096, 1128, 2064, 2096, 2128])
def test_baseline_blocks(cuda_device, shape, variant):
    """The SD1.5 self-/cross-attention blocks, all (b, h) pairs in one launch, for the automatic choice and every
    kernel variant: 64-, 96- or 128-key tiles with one query tile per CTA (two CTAs per SM where they fit) or two
    (two S buffers per query tile where TMEM holds them)."""
    B, H, Sq, Skv, D = shape
    q, k, v, ref = _block(B, H, Sq, Skv, D, D)
    _check(_run(q, k, v, H, variant=variant), ref)
    _check(_run(q, k, v, H, out_dtype=torch.bfloat16, variant=variant), ref)


@pytest.mark.parametrize("shape", [(2, 8, 4096, 4096, 40), (2, 8, 4096, 77, 40), (1, 1, 1, 1, 40), (1, 2, 100, 300, 40),
                                   (1, 2, 1000, 129, 64), (3, 5, 600, 257, 16), (1, 3, 513, 1000, 32)])
def test_four_query_tiles_per_cta(cuda_device, shape):
    """The four-Q-tile kernel (variant 4064: 512 query rows per CTA, 64-key tiles, d <= 64), full and ragged
    shapes whose trailing Q tiles lie partly or wholly past Sq."""
    B, H, Sq, Skv, D = shape
    q, k, v, ref = _block(B, H, Sq, Skv, D, 3)
    _check(_run(q, k, v, H, variant=4064), ref)
    _check(_run(q, k, v, H, out_dtype=torch.bfloat16, variant=4064), ref)


def test_unet_batch16_self_attention_block(cuda_device):
    """The batch-16 UNet's top-level self-attention (16, 8, 4096, 4096, 40) on the automatic variant, the
    two-query-tile kernel the UNet step runs, in both output types."""
    B, H, Sq, Skv, D = 16, 8, 4096, 4096, 40
    q, k, v, ref = _block(B, H, Sq, Skv, D, 16)
    _check(_run(q, k, v, H), ref)
    _check(_run(q, k, v, H, out_dtype=torch.bfloat16), ref)


@pytest.mark.parametrize("world", [2, 3, 8])
@pytest.mark.parametrize("shape,head_major", [((2, 8, 1024, 1024, 80), False), ((3, 5, 300, 77, 40), False),
                                              ((2, 8, 256, 256, 160), True)])
def test_pair_sharded_attention_ranks(cuda_device, world, shape, head_major):
    """Every rank's part of a (batch, head)-pair-sharded block (npu_ai_b200.sharding: contiguous pair ranges, at
    most three strided in-place views per rank), emulated for all ranks in one process and assembled as the
    all-gather does, against the oracle on the whole block."""
    from npu_ai_b200 import kernels
    from npu_ai_b200.sharding import attention_shard, pair_width
    B, H, Sq, Skv, D = shape
    q, k, v, ref = _block(B, H, Sq, Skv, D, 5)
    if head_major:
        q, k, v = (t.view(B, t.shape[1], H, D).transpose(1, 2).contiguous() for t in (q, k, v))
        ref = ref.view(B, Sq, H, D).transpose(1, 2)
    qd, kd, vd = (t.to(cuda_device) for t in (q, k, v))
    parts = [attention_shard(qd, kd, vd, H, r, world, head_major_in=head_major, out_dtype=torch.float32)
             for r in range(world)]
    kernels.check_status(cuda_device)
    assert all(p.shape[0] == pair_width(B * H, world) for p in parts)
    hm = torch.cat(parts)[:B * H].view(B, H, Sq, D)
    got = hm if head_major else hm.permute(0, 2, 1, 3).reshape(B, Sq, H * D)
    _check(got, ref)


@pytest.mark.parametrize("shape", ["1x4x256x256x40", "1x4x512x256x80", "2x8x1024x1024x80"])
def test_reference_script_shapes(cuda_device, shape):
    """The reference's default shapes with its input distribution (q, k ~ 1.5 N(0,1))."""
    B, H, Sq, Skv, D = (int(t) for t in shape.split("x"))
    q, k, v = _qkv(B, H, Sq, Skv, D, seed=0, qk_scale=1.5)
    ref = attention_ref(q, k, v, H)
    o = _run(q, k, v, H)
    _check(o, ref)
    assert rel_max_err(o, ref) < 0.1  # the reference's own mismatch threshold


@pytest.mark.parametrize("shape", [(1, 1, 1, 1, 40), (1, 2, 100, 300, 40), (3, 5, 129, 257, 80), (1, 3, 77, 77, 160),
                                   (2, 1, 300, 1, 80), (1, 2, 1000, 129, 64), (2, 2, 200, 500, 128),
                                   (1, 1, 130, 70, 24)])
@pytest.mark.parametrize("variant", [0, 1096, 2064, 2096, 2128])
def test_ragged_shapes(cuda_device, shape, variant):
    """Any Sq / Skv (query and key tails handled in the kernel), odd head counts, d beyond the SD1.5 set; also
    forced onto the two-query-tile kernel, whose second tile is then partly or wholly past Sq."""
    B, H, Sq, Skv, D = shape
    q, k, v = _qkv(B, H, Sq, Skv, D, seed=Sq + Skv)
    _check(_run(q, k, v, H, variant=variant), attention_ref(q, k, v, H))


@pytest.mark.parametrize("shape", [(1, 2, 16384, 16384, 40), (2, 8, 16384, 77, 40)], ids=["self128x128", "cross128x128"])
def test_long_sequences_128x128_latent(cuda_device, shape):
    """The 128x128-latent blocks of the batched UNet config (self-attention over 16384 tokens, cross-attention to
    77), which the reference's fused path cannot hold (its buffer caps send them to the CPU)."""
    B, H, Sq, Skv, D = shape
    q, k, v = _qkv(B, H, Sq, Skv, D, seed=16)
    _check(_run(q, k, v, H), attention_ref(q, k, v, H))


def test_head_dim_above_192_runs_one_query_tile(cuda_device):
    """d = 256 takes the one-query-tile kernel; asking for two query tiles per CTA is refused, not faked."""
    B, H, Sq, Skv, D = 1, 2, 300, 200, 256
    q, k, v = _qkv(B, H, Sq, Skv, D, seed=3)
    _check(_run(q, k, v, H), attention_ref(q, k, v, H))
    with pytest.raises(RuntimeError, match="two Q tiles"):
        _run(q, k, v, H, variant=2064)


def test_head_major_and_strided(cuda_device):
    """skip_reshape / skip_output_reshape layouts, and inputs as padded-row views (the reference's --strided)."""
    B, H, Sq, Skv, D = 2, 4, 300, 200, 40
    q, k, v = _qkv(B, H, Sq, Skv, D, seed=4)
    ref = attention_ref(q, k, v, H)
    dev = torch.device("cuda", 0)
    from npu_ai_b200 import kernels
    # head-major in and out
    qh, kh, vh = (t.view(B, t.shape[1], H, D).transpose(1, 2).contiguous() for t in (q, k, v))
    oh = kernels.attention(qh.to(dev), kh.to(dev), vh.to(dev), H, head_major_in=True, head_major_out=True)
    kernels.check_status(dev)
    _check(oh.transpose(1, 2).reshape(B, Sq, H * D), ref)
    # padded row stride: (B, S, 256) buffers viewed as (B, S, 160)
    def padded(t):
        buf = torch.zeros(B, t.shape[1], 256, dtype=t.dtype)
        buf[:, :, :H * D] = t
        return buf.to(dev)[:, :, :H * D]
    out_buf = torch.full((B, Sq, 200), 5.0, device=dev)
    kernels.attention(padded(q), padded(k), padded(v), H, out=out_buf[:, :, :H * D])
    kernels.check_status(dev)
    _check(out_buf[:, :, :H * D], ref)
    assert bool((out_buf[:, :, H * D:] == 5.0).all()), "kernel wrote outside the output view"


@pytest.mark.parametrize("variant", [0, 1064, 1096, 2064, 2096, 2128, 4064])
def test_running_max_moves(cuda_device, variant):
    """Later key tiles with much larger scores force the lazy running max to move (the O/l correction path)."""
    B, H, Sq, Skv, D = 1, 2, 256, 1024, 40
    g = torch.Generator().manual_seed(7)
    q = torch.randn(B, Sq, H * D, generator=g)
    k = torch.randn(B, Skv, H * D, generator=g)
    ramp = torch.linspace(0.2, 4.0, Skv).view(1, Skv, 1)
    k = (k * ramp).to(torch.bfloat16)
    q = (q * 2.0).to(torch.bfloat16)
    v = torch.randn(B, Skv, H * D, generator=g).to(torch.bfloat16)
    _check(_run(q, k, v, H, variant=variant), attention_ref(q, k, v, H))


def test_custom_scale(cuda_device):
    B, H, Sq, Skv, D = 1, 2, 200, 300, 80
    q, k, v = _qkv(B, H, Sq, Skv, D, seed=12)
    _check(_run(q, k, v, H, scale=0.05), attention_ref(q, k, v, H, scale=0.05))


@pytest.mark.parametrize("variant", [1064, 2064, 2128, 4064])
def test_forced_timeout_reports_status_and_recovers(cuda_device, variant):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    B, H, Sq, Skv, D = 1, 2, 256, 512, 40
    q, k, v = _qkv(B, H, Sq, Skv, D, seed=2)
    kernels.status(dev)
    kernels.set_wait_timeout_ns(2_000_000)
    kernels.set_debug_flags(1)
    try:
        kernels.attention(q.to(dev), k.to(dev), v.to(dev), H, variant=variant)
        with pytest.raises(RuntimeError, match="failure status"):
            kernels.check_status(dev)
    finally:
        kernels.set_debug_flags(0)
        kernels.set_wait_timeout_ns(0)
    _check(_run(q, k, v, H, variant=variant), attention_ref(q, k, v, H))
