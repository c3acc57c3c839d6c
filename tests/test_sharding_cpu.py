"""UNet batch sharding across ranks, on CPU with gloo (world size 2): the host-side logic of the multi-GPU path.

The sharded path splits prompts across ranks with each prompt's CFG pair kept local and all-gathers the final
latents; the result must equal single-process sampling (prompts are independent and seeded per prompt). Uses a
small UNet of the same architecture with the oracle's torch ops (no GPU).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from npu_ai_b200.sd15_unet import SD15UNet, prompt_shard, sample_sharded, seeded_prompts


def _tiny_unet(seed=0):
    torch.manual_seed(seed)
    return SD15UNet(model_channels=32, channel_mult=(1, 2), num_res_blocks=1, attention_levels=(1,), heads=2,
                    context_dim=16).eval()


def _inputs(P):
    lat, ctx, unc = seeded_prompts(P, 8, seed=3, context_len=5, context_dim=16)
    return lat, ctx, unc


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, P, out_path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        model = _tiny_unet()
        lat, ctx, unc = _inputs(P)
        with torch.no_grad():
            out = sample_sharded(model, lat, ctx, unc, steps=2)
        if rank == 0:
            torch.save(out, out_path)
    finally:
        dist.destroy_process_group()


def test_prompt_shard_covers_all():
    for P in (1, 7, 8, 16):
        for W in (1, 2, 3, 8):
            ranges = [prompt_shard(P, W, r) for r in range(W)]
            assert ranges[0][0] == 0 and ranges[-1][1] == P
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            assert max(h - l for l, h in ranges) - min(h - l for l, h in ranges) <= 1


def test_seeded_prompts_independent_of_count():
    a = seeded_prompts(3, 4, seed=1, context_len=2, context_dim=4)
    b = seeded_prompts(5, 4, seed=1, context_len=2, context_dim=4)
    for x, y in zip(a, b):
        assert torch.equal(x, y[:3])


@pytest.mark.parametrize("P", [4, 3])
def test_sharded_sampling_matches_single_process(tmp_path, P):
    out_path = str(tmp_path / "out.pt")
    mp.start_processes(_worker, args=(2, _free_port(), P, out_path), nprocs=2, join=True, start_method="spawn")
    sharded = torch.load(out_path)
    torch.set_num_threads(2)
    model = _tiny_unet()
    lat, ctx, unc = _inputs(P)
    with torch.no_grad():
        single = sample_sharded(model, lat, ctx, unc, steps=2)
    # equal up to float reassociation: CPU matmuls block differently for different batch sizes (~1e-6 relative)
    scale = float(single.abs().max())
    assert torch.allclose(sharded, single, rtol=1e-4, atol=1e-5 * scale), float((sharded - single).abs().max())


def _failing_worker(rank, world, port, P, out_dir, mode):
    """A rank of a sharded run in which rank 1 fails on the host: it raises before the latent gather ("raises")
    or never joins the process group ("never_joins"). Every rank records how its run ended."""
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    path = os.path.join(out_dir, f"rank{rank}.txt")
    if mode == "never_joins" and rank == 1:
        with open(path, "w") as f:
            f.write("left")
        return
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    except Exception as e:  # noqa: BLE001 - the outcome is what the test checks
        with open(path, "w") as f:
            f.write(f"init failed: {type(e).__name__}")
        return
    try:
        torch.set_num_threads(1)
        model = _tiny_unet()
        lat, ctx, unc = _inputs(P)
        if mode == "raises" and rank == 1:
            raise RuntimeError("injected host-side failure before the gather")
        with torch.no_grad():
            sample_sharded(model, lat, ctx, unc, steps=1)
        outcome = "ok"
    except Exception as e:  # noqa: BLE001
        outcome = f"failed: {type(e).__name__}"
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass
    with open(path, "w") as f:
        f.write(outcome)


@pytest.mark.parametrize("mode", ["raises", "never_joins"])
def test_rank_failure_surfaces_as_error_on_the_other_rank(tmp_path, mode):
    """Failure detection for the sharded path without any GPU: when one rank fails on the host, the surviving
    rank's collective (or rendezvous) ends with an exception within the process group's timeout instead of
    waiting for good."""
    import time
    t0 = time.time()
    mp.start_processes(_failing_worker, args=(2, _free_port(), 2, str(tmp_path), mode), nprocs=2, join=True,
                       start_method="spawn")
    assert time.time() - t0 < 120
    survivor = (tmp_path / "rank0.txt").read_text()
    assert survivor.startswith(("failed", "init failed")), survivor


# ---- attention over (batch, head) pairs split across ranks -------------------------------------------------------
def test_pair_segments_tile_every_range():
    from npu_ai_b200.sharding import pair_range, pair_segments, pair_width
    for B, H in ((2, 8), (3, 5), (1, 7), (16, 8)):
        pairs = B * H
        for W in (1, 2, 3, 4, 5, 8):
            covered = []
            for r in range(W):
                lo, hi = pair_range(pairs, W, r)
                assert hi - lo <= pair_width(pairs, W)
                segs = pair_segments(lo, hi, H)
                assert len(segs) <= 3
                for b0, b1, h0, h1 in segs:
                    assert 0 <= b0 < b1 <= B and 0 <= h0 < h1 <= H and (b1 - b0 == 1 or (h0, h1) == (0, H))
                    covered += [b * H + h for b in range(b0, b1) for h in range(h0, h1)]
            assert covered == list(range(pairs)), (B, H, W)


def _cpu_compute(q, k, v, heads, out, head_major_in, scale, variant):
    """CPU stand-in for the kernel launch (the oracle's attention), writing the head-major output view."""
    from oracle import attention_ref
    o = attention_ref(q, k, v, heads, scale=scale, head_major=head_major_in)
    if not head_major_in:
        o = o.view(q.shape[0], q.shape[1], heads, -1).transpose(1, 2)
    out.copy_(o.to(out.dtype))


def _block(B, H, Sq, Skv, D, head_major):
    g = torch.Generator().manual_seed(11)
    shp = (lambda S: (B, H, S, D)) if head_major else (lambda S: (B, S, H * D))
    return (torch.randn(*shp(Sq), generator=g).bfloat16(), torch.randn(*shp(Skv), generator=g).bfloat16(),
            torch.randn(*shp(Skv), generator=g).bfloat16())


def _attn_worker(rank, world, port, dims, head_major, out_path):
    import torch.distributed as dist
    from npu_ai_b200.sharding import attention_sharded
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.set_num_threads(1)
        q, k, v = _block(*dims, head_major)
        out = attention_sharded(q, k, v, dims[1], head_major_in=head_major, head_major_out=head_major,
                                out_dtype=torch.float32, compute=_cpu_compute)
        torch.save(out, out_path.format(rank))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,dims,head_major", [
    (2, (2, 4, 24, 16, 8), False),
    (3, (2, 4, 24, 16, 8), False),     # 8 pairs over 3 ranks: ranges cut through a batch's heads, uneven chunks
    (3, (3, 5, 16, 9, 16), True),      # head-major in and out, odd head count
])
def test_attention_pairs_sharded_over_ranks_match_the_oracle(tmp_path, world, dims, head_major):
    """Every rank computes its contiguous (batch, head) pair range and the all-gather assembles the block: each
    rank's result equals the oracle on the whole block (host logic with a CPU stand-in for the kernel launch)."""
    from oracle import attention_ref
    out_path = str(tmp_path / "out{}.pt")
    mp.start_processes(_attn_worker, args=(world, _free_port(), dims, head_major, out_path), nprocs=world,
                       join=True, start_method="spawn")
    q, k, v = _block(*dims, head_major)
    ref = attention_ref(q, k, v, dims[1], head_major=head_major)
    for r in range(world):
        got = torch.load(out_path.format(r))
        assert got.shape == ref.shape
        assert torch.allclose(got, ref, atol=1e-6, rtol=1e-5), (r, float((got - ref).abs().max()))
