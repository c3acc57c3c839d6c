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
