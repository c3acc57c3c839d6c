"""GEMM parity on the B200: the tcgen05 kernel through the C ABI against the CPU oracle.

Semantics follow the reference's GEMM test (scripts/05-gemm-test.py: seeded inputs, torch CPU reference on
bf16-rounded inputs in f32, max|err|/max|ref| and cosine, an unaligned 100x100x100 case) with the offload path's
stated tolerance: max-abs <= 2e-2 and relative L2 <= 5e-3 on the f32 output. bf16 outputs are compared with the
oracle rounded to bf16: at most 1 bf16 ulp apart (accumulation order can flip a rounding), never more.
"""
import pytest
import torch

from oracle import cosine, linear_ref, rel_l2_err, rel_max_err

pytestmark = pytest.mark.gpu

SD15_KN = [(320, 320), (320, 2560), (1280, 320), (768, 320), (640, 640), (640, 5120), (2560, 640), (1280, 1280),
           (1280, 10240), (5120, 1280), (768, 1280)]
SD15_M = [77, 154, 256, 1024, 4096, 8192]


def _inputs(M, K, N, seed=0, bias=True, bias_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.01).to(bias_dtype) if bias else None
    return x, w, b


def _check_f32(y, ref):
    y = y.float().cpu()
    err_abs = float((y - ref).abs().max())
    assert err_abs <= 2e-2, f"max-abs {err_abs}"
    assert rel_l2_err(y, ref) <= 5e-3, f"rel-L2 {rel_l2_err(y, ref)}"
    assert rel_max_err(y, ref) < 1e-3
    assert cosine(y, ref) > 0.999


def _check_bf16(y, ref):
    y = y.float().cpu()
    rb = ref.to(torch.bfloat16).float()
    diff = (y - rb).abs()
    # One bf16 ulp at the reference's magnitude (2^(e-7)) plus an absolute floor for the f32 accumulation-order
    # difference (~1e-6 here), which exceeds an ulp only for outputs near zero where bf16 spacing is tiny.
    ulp = torch.pow(2.0, torch.floor(torch.log2(rb.abs().clamp_min(1e-30))) - 7)
    bad = int((diff > ulp * 1.0001 + 1e-4).sum())
    assert bad == 0, f"{bad} outputs more than 1 bf16 ulp from the oracle (max diff {float(diff.max())})"


def _run(x, w, b, out_dtype=torch.float32, variant=0):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    y = kernels.gemm(x.to(dev), w.to(dev), b.to(dev) if b is not None else None, out_dtype=out_dtype,
                     variant=variant)
    kernels.check_status(dev)
    return y


def test_config1_linear_to_q(cuda_device):
    """SD1.5 to_q at the 64x64 latent: x [4096x320] ~N(0,1), W [320x320] ~N(0,0.02^2), b ~N(0,0.01^2), f32
    accumulate, bf16 out."""
    x, w, b = _inputs(4096, 320, 320)
    ref = linear_ref(x, w, b)
    _check_f32(_run(x, w, b, torch.float32), ref)
    _check_bf16(_run(x, w, b, torch.bfloat16), ref)


@pytest.mark.parametrize("M", SD15_M)
@pytest.mark.parametrize("KN", SD15_KN, ids=lambda kn: f"K{kn[0]}N{kn[1]}")
def test_sd15_sweep_f32(cuda_device, M, KN):
    K, N = KN
    x, w, b = _inputs(M, K, N, seed=M * 7 + K + N)
    _check_f32(_run(x, w, b), linear_ref(x, w, b))


@pytest.mark.parametrize("MKN", [(77, 768, 320), (154, 768, 1280), (4096, 1280, 320), (8192, 320, 2560)])
def test_sd15_bf16_out(cuda_device, MKN):
    M, K, N = MKN
    x, w, b = _inputs(M, K, N, seed=3)
    _check_bf16(_run(x, w, b, torch.bfloat16), linear_ref(x, w, b))


@pytest.mark.parametrize("variant", [64, 96, 128, 160, 192, 256, 1128, 1192, 1256])
def test_forced_variants(cuda_device, variant):
    """Every tile variant, 1000 + N tile being 256-row tiles on a two-CTA cluster; M = 1100 leaves the last
    256-row tile's second CTA with 76 rows, M = 1000 a ragged last row block."""
    for M in (1000, 1100):
        x, w, b = _inputs(M, 704, 1000, seed=variant + M)
        _check_f32(_run(x, w, b, variant=variant), linear_ref(x, w, b))
        _check_bf16(_run(x, w, b, torch.bfloat16, variant=variant), linear_ref(x, w, b))


@pytest.mark.parametrize("MKN", [(1, 8, 8), (1, 320, 320), (3, 16, 17), (129, 72, 200), (255, 1024, 33),
                                 (100, 100, 100), (77, 77, 77), (5, 3, 2)])
def test_ragged_and_unaligned(cuda_device, MKN):
    """Any M/N/K: tails in-kernel; K % 8 != 0 goes through the workspace repack (the reference's 100x100x100)."""
    M, K, N = MKN
    x, w, b = _inputs(M, K, N, seed=M + K + N)
    _check_f32(_run(x, w, b), linear_ref(x, w, b))


def test_no_bias_and_f32_bias(cuda_device):
    x, w, _ = _inputs(300, 320, 640, bias=False)
    _check_f32(_run(x, w, None), linear_ref(x, w, None))
    x, w, b = _inputs(300, 320, 640, bias_dtype=torch.float32)
    _check_f32(_run(x, w, b), linear_ref(x, w, b))


def test_strided_views(cuda_device):
    """x as a padded-row view (as the reference's zero-copy outputs are) and an output written into a wider buffer."""
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, w, b = _inputs(500, 320, 320, seed=11)
    big = torch.zeros(500, 384, dtype=torch.bfloat16)
    big[:, :320] = x
    xv = big.to(dev)[:, :320]
    outbuf = torch.full((500, 400), -7.0, device=dev)
    out = outbuf[:, :320]
    kernels.gemm(xv, w.to(dev), b.to(dev), out=out)
    kernels.check_status(dev)
    _check_f32(out, linear_ref(x, w, b))
    assert bool((outbuf[:, 320:] == -7.0).all()), "kernel wrote outside the output view"


def test_registered_weight_handle(cuda_device):
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, w, b = _inputs(2048, 640, 5120, seed=5)
    wd = w.to(dev)
    h = kernels.register_weight(wd)
    try:
        for _ in range(2):
            y = kernels.gemm(x.to(dev), wd, b.to(dev), handle=h)
        kernels.check_status(dev)
        _check_f32(y, linear_ref(x, w, b))
    finally:
        kernels.release_weight(h)


def test_guard_band(cuda_device):
    """Output canaries: nothing beyond [M, N] is written (contiguous output followed by a guard region)."""
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    M, K, N = 130, 256, 136
    x, w, b = _inputs(M, K, N, seed=9)
    buf = torch.full((M * N + 4096,), 123.0, device=dev)
    out = buf[: M * N].view(M, N)
    kernels.gemm(x.to(dev), w.to(dev), b.to(dev), out=out)
    kernels.check_status(dev)
    assert bool((buf[M * N:] == 123.0).all())
    _check_f32(out, linear_ref(x, w, b))


def test_forced_timeout_reports_status_and_recovers(cuda_device):
    """Failure detection without a GPU fault: the MMA role waits on a barrier nothing signals under a 2 ms
    deadline; the kernel must record the timeout in the status word, exit cleanly, and the next call must work."""
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    x, w, b = _inputs(512, 320, 320, seed=1)
    kernels.status(dev)  # clear
    kernels.set_wait_timeout_ns(2_000_000)
    kernels.set_debug_flags(1)
    try:
        kernels.gemm(x.to(dev), w.to(dev), b.to(dev))
        with pytest.raises(RuntimeError, match="failure status"):
            kernels.check_status(dev)
    finally:
        kernels.set_debug_flags(0)
        kernels.set_wait_timeout_ns(0)
    y = _run(x, w, b)
    _check_f32(y, linear_ref(x, w, b))


@pytest.mark.parametrize("MKN", [(77, 5120, 1280), (154, 2560, 640), (256, 1280, 320), (8, 8192, 256)])
def test_split_k_deterministic_and_reused_workspace(cuda_device, MKN):
    """Few output tiles with a long K split K across CTAs: f32 partials summed in a fixed order (bitwise
    repeatable), counters left zero so the cached workspace serves the next problem of any size."""
    M, K, N = MKN
    x, w, b = _inputs(M, K, N, seed=K)
    y1 = _run(x, w, b)
    _check_f32(y1, linear_ref(x, w, b))
    # a different problem in between reuses the same workspace
    x2, w2, b2 = _inputs(33, 4096, 4000, seed=1)
    _check_f32(_run(x2, w2, b2), linear_ref(x2, w2, b2))
    y2 = _run(x, w, b)
    assert torch.equal(y1, y2), "split-K result changed between identical calls"


def test_repack_then_split_k_share_workspace(cuda_device):
    """A call that only repacks (K % 8 != 0) followed by split-K calls on the same cached workspace: the repack must
    not land on the split-K counters."""
    for MKN in [(100, 100, 100), (154, 768, 320), (99, 1001, 77), (512, 1280, 1280), (77, 5120, 1280)]:
        x, w, b = _inputs(*MKN, seed=sum(MKN))
        _check_f32(_run(x, w, b), linear_ref(x, w, b))


@pytest.mark.parametrize("shape", [(4096, 320, 320), (77, 5120, 1280), (300, 640, 200)],
                         ids=["to_out", "splitK", "ragged"])
def test_gemm_residual_epilogue(cuda_device, shape):
    """out = x W^T + b + residual in one kernel (a transformer block's residual connection), also in place (the
    residual buffer receives the result) and on a split-K shape, where the reducing split adds it."""
    from npu_ai_b200 import kernels
    dev = torch.device("cuda", 0)
    M, K, N = shape
    x, w, b = _inputs(M, K, N, seed=M + K + 11)
    r = torch.randn(M, N, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    ref = linear_ref(x, w, b) + r.float()
    xd, wd, bd = x.to(dev), w.to(dev), b.to(dev)
    y = kernels.gemm(xd, wd, bd, out_dtype=torch.float32, residual=r.to(dev))
    kernels.check_status(dev)
    _check_f32(y, ref)
    rd = r.to(dev).clone()
    kernels.gemm(xd, wd, bd, out=rd, residual=rd)
    kernels.check_status(dev)
    _check_bf16(rd, ref)
