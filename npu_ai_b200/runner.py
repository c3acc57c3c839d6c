"""`NpuGemm` on B200: the reference runner's Python API (npu/xdna1_gemm.py:184-773) over the sm_100a kernels.

Same class, method names, signatures, stats keys and exception types as the reference, so callers written for
the NPU runner (its ComfyUI node, its test scripts) run unchanged:

  upload_weight(w_kn) -> NpuWeight          xdna1_gemm.py:311-321  (also takes nn.Linear's [N, K] via layout="nk")
  matmul_t(x, w, bias=None) -> tensor       xdna1_gemm.py:349-422
  matmul(x, w) -> numpy                     xdna1_gemm.py:424-426
  linear(x, w, bias=None)                   xdna1_gemm.py:428-448
  prepare(shapes), dispatch_shapes(M,K,N)   xdna1_gemm.py:295-308
  attention(q, k, v, heads, scale=None, skip_reshape=False, skip_output_reshape=False)   xdna1_gemm.py:499-600
  attention_fits / attention_warmup / attention_fused_fits                              xdna1_gemm.py:451-497
  summary(), stats, pool                    xdna1_gemm.py:201-209, :755-773

What changes on B200 (and why):
  * Device: one CUDA device instead of an NPU; tensors live in HBM. Inputs may be CPU (copied over) or CUDA
    tensors; results are CUDA tensors (f32 by default, the reference's output type; `out_dtype=torch.bfloat16`
    gives bf16 output, the benchmarked configuration's).
  * No padding and no chunking: the kernels take any M, N, K (ragged tails in-kernel) and any sequence length, so
    the NPU alignment (M % 256, K % 64, N % 320) and chunk limits (xdna1_gemm.py:220-229, :274-293) disappear. The
    NPU-only constructor arguments are accepted and recorded but do not change the computation.
  * Weights stay resident in HBM in nn.Linear's [N, K] layout with their TMA descriptors cached.
  * No CPU path: every call runs on the GPU kernels or raises (the reference never falls back silently either,
    comfyui node :5-7).
"""
from __future__ import annotations

import threading
import time
import weakref
from dataclasses import dataclass, field

import numpy as np
import torch

from . import kernels


def _as_tensor(x) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x.detach()
    return torch.from_numpy(np.ascontiguousarray(np.asarray(x, dtype=np.float32)))


@dataclass
class NpuWeight:
    """A weight resident in HBM (the reference's NpuWeight, npu/xdna1_gemm.py:89-99).

    `tensor` is the bf16 [N, Kp] device matrix (Kp = K rounded up to 8 when K is not a multiple of 8, zero
    columns); `handle` is the library's registration (TMA descriptors cached) or None for padded weights.
    """
    K: int
    N: int
    Kp: int
    tensor: torch.Tensor
    handle: int | None = None
    chunks: list = field(default_factory=list)  # kept for API compatibility: one chunk, the whole weight

    @property
    def nbytes(self) -> int:
        return self.tensor.numel() * self.tensor.element_size()

    def release(self) -> None:
        if self.handle is not None:
            kernels.release_weight(self.handle)
            self.handle = None


class _DeviceBuf:
    """A leased device buffer with a 2-D view (the reference's _Buf, npu/xdna1_gemm.py:102-132)."""
    __slots__ = ("key", "t2d", "in_use", "pool", "nbytes", "base")

    def __init__(self, key, t2d: torch.Tensor, pool):
        self.key, self.t2d, self.pool = key, t2d, pool
        self.nbytes = t2d.numel() * t2d.element_size()
        self.base = t2d.data_ptr()
        self.in_use = True

    def release(self) -> None:
        self.pool.release(self)


class _DevicePool:
    """Zero-initialised device buffers keyed by (kind, logical shape) (the reference's _BufPool,
    npu/xdna1_gemm.py:135-181). The runner itself allocates through torch's caching allocator; the pool is kept
    for callers that lease buffers directly (the reference's attention test does)."""

    def __init__(self, stats: dict, device: torch.device):
        self._free: dict[tuple, list[_DeviceBuf]] = {}
        self._all: list[_DeviceBuf] = []
        self._lock = threading.Lock()
        self.stats = stats
        self.device = device

    def find(self, ptr: int):
        for b in self._all:
            off = ptr - b.base
            if 0 <= off < b.nbytes:
                return b, off
        return None

    def lease(self, key: tuple, rows: int, cols: int, torch_dtype) -> _DeviceBuf:
        with self._lock:
            lst = self._free.get(key)
            if lst:
                b = lst.pop()
                b.in_use = True
                return b
        t0 = time.perf_counter()
        b = _DeviceBuf(key, torch.zeros((rows, cols), dtype=torch_dtype, device=self.device), self)
        with self._lock:
            self._all.append(b)
        self.stats["buffers"] += 1
        self.stats["buffer_bytes"] += b.nbytes
        self.stats["alloc_seconds"] += time.perf_counter() - t0
        return b

    def release(self, b: _DeviceBuf) -> None:
        with self._lock:
            if b.in_use:
                b.in_use = False
                self._free.setdefault(b.key, []).append(b)


class NpuGemm:
    """Shape-agnostic bf16 GEMM and fused attention runner on one B200 (API of npu/xdna1_gemm.py:184)."""

    def __init__(self, n_cols: int = 4, max_n_chunk: int = 4096, max_m_chunk: int = 4096, max_k_chunk: int = 8192,
                 verbose: bool = True, attn_head_dims: tuple[int, ...] = (40, 80), attn_lazy_compile: bool = False,
                 gemm_head_dim: int = 80, *, device: torch.device | int | str | None = None,
                 out_dtype: torch.dtype = torch.float32, timing: bool = False):
        """`n_cols`, the chunk limits, `attn_head_dims`, `attn_lazy_compile` and `gemm_head_dim` describe the NPU
        program layout; they are recorded for compatibility. The B200 kernels need no per-head-dim program and
        no chunking: every head dim that is a multiple of 8 up to 256 is served. `timing=True` records CUDA events
        around each call so `stats["npu_seconds"]` holds GPU time (resolved lazily, no per-call sync)."""
        t0 = time.perf_counter()
        if device is None:
            if not torch.cuda.is_available():
                raise RuntimeError("NpuGemm needs a CUDA device and none is available; there is no CPU path")
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        if self.device.type != "cuda":
            raise ValueError("NpuGemm runs on a CUDA device; there is no CPU path")
        self.verbose = verbose
        self.out_dtype = out_dtype
        self.timing = timing
        self.n_cols, self.max_n_chunk, self.max_m_chunk, self.max_k_chunk = n_cols, max_n_chunk, max_m_chunk, max_k_chunk
        self.attn_head_dims = tuple(attn_head_dims)
        self.attn_lazy_compile = attn_lazy_compile
        self.gemm_head_dim = gemm_head_dim
        self.stats = {"calls": 0, "dispatches": 0, "npu_seconds": 0.0, "total_seconds": 0.0, "flops": 0.0,
                      "compile_seconds": 0.0, "buffers": 0, "buffer_bytes": 0, "alloc_seconds": 0.0,
                      "program_switches": 0,
                      "attn_calls": 0, "attn_pairs": 0, "attn_seconds": 0.0, "attn_flops": 0.0,
                      "attn_fused_calls": 0, "attn_fused_npu_seconds": 0.0, "attn_fused_seconds": 0.0,
                      "attn_fused_q_inplace": 0, "attn_t_convert": 0.0, "attn_t_submit": 0.0, "attn_t_wait": 0.0,
                      "attn_t_sync_out": 0.0, "attn_by_shape": {}, "attn_fused_flops": 0.0,
                      "attn_compile_seconds": 0.0}
        self.pool = _DevicePool(self.stats, self.device)
        self._lock = threading.RLock()
        self._pending: list[tuple[str, torch.cuda.Event, torch.cuda.Event, tuple | None]] = []
        self._attn_warm: set[tuple[int, int, int, int]] = set()
        self.attn_parts = 1         # one launch covers every pair; kept for API compatibility
        self.attn_first_pairs = 0
        self.align_m = self.align_k = self.align_n = 1
        self.sms = kernels.device_sms(self.device)   # loads the library, fails loudly without it
        self.stats["compile_seconds"] = time.perf_counter() - t0
        if verbose:
            print(f"[npu_b200] runner ready on {torch.cuda.get_device_name(self.device)} ({self.sms} SMs) in "
                  f"{self.stats['compile_seconds']:.2f}s; GEMM and attention kernels take any shape", flush=True)

    # -- timing ---------------------------------------------------------------------------------
    def _events(self):
        if not self.timing:
            return None, None
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(torch.cuda.current_stream(self.device))
        return s, e

    def _close(self, kind: str, ev, key=None) -> None:
        s, e = ev
        if s is None:
            return
        e.record(torch.cuda.current_stream(self.device))
        self._pending.append((kind, s, e, key))
        if len(self._pending) > 4096:
            self.flush_timing()

    def flush_timing(self) -> None:
        """Wait for the recorded calls and add their GPU time to stats (npu_seconds / attn_fused_npu_seconds)."""
        with self._lock:
            pend, self._pending = self._pending, []
        for kind, s, e, key in pend:
            e.synchronize()
            dt = s.elapsed_time(e) / 1e3
            if kind == "gemm":
                self.stats["npu_seconds"] += dt
            else:
                self.stats["attn_fused_npu_seconds"] += dt
                if key is not None:
                    self.stats["attn_by_shape"][key][3] += dt

    # -- shapes ---------------------------------------------------------------------------------
    def dispatch_shapes(self, M: int, K: int, N: int) -> list[tuple[int, int, int]]:
        """One launch per GEMM whatever its size (the reference splits into padded chunks, xdna1_gemm.py:295-297)."""
        return [(int(M), int(K), int(N))]

    def prepare(self, shapes) -> None:
        """Warm the kernels up for these logical (M, K, N) shapes (one launch each on zeros), so the first real
        call pays no one-off setup (the reference pre-generates instruction streams, xdna1_gemm.py:299-308)."""
        for M, K, N in shapes:
            x = torch.zeros((M, K), dtype=torch.bfloat16, device=self.device)
            w = torch.zeros((N, K), dtype=torch.bfloat16, device=self.device)
            kernels.gemm(x, w, out_dtype=self.out_dtype)

    # -- weights --------------------------------------------------------------------------------
    def upload_weight(self, w, layout: str = "kn") -> NpuWeight:
        """w: (K, N) array (numpy or torch, any float dtype; the reference's convention) -> resident bf16 weight.
        With layout="nk" w is nn.Linear's own (N, K) weight and is used without a transpose."""
        wt = _as_tensor(w)
        if wt.dim() != 2:
            raise ValueError("weights are 2-D")
        if layout == "kn":
            wt = wt.t()
        elif layout != "nk":
            raise ValueError(f"unknown weight layout {layout!r}")
        N, K = wt.shape
        Kp = (K + 7) // 8 * 8
        with self._lock:
            dev = torch.zeros((N, Kp), dtype=torch.bfloat16, device=self.device)
            dev[:, :K].copy_(wt.to(self.device, torch.bfloat16))
            handle = kernels.register_weight(dev) if Kp == K else None
            nw = NpuWeight(K=K, N=N, Kp=Kp, tensor=dev, handle=handle)
            nw.chunks = [(dev, 0, K, Kp, 0, N, N)]
            weakref.finalize(nw, _release_handle, handle)
        return nw

    # -- GEMM -----------------------------------------------------------------------------------
    def _x_device(self, x) -> torch.Tensor:
        xt = _as_tensor(x)
        if xt.device != self.device:
            xt = xt.to(self.device, non_blocking=xt.is_pinned())
        if xt.dtype != torch.bfloat16:
            xt = xt.to(torch.bfloat16)
        if xt.stride(-1) != 1:
            xt = xt.contiguous()
        return xt

    def _bias_device(self, bias) -> torch.Tensor | None:
        if bias is None:
            return None
        b = _as_tensor(bias)
        if b.device != self.device:
            b = b.to(self.device, non_blocking=b.is_pinned())  # stream-ordered: no host sync for pinned biases
        if b.dtype not in (torch.float32, torch.bfloat16):
            b = b.float()
        return b.contiguous()

    def matmul_t(self, x, w: NpuWeight, bias=None, out: torch.Tensor | None = None,
                 out_dtype: torch.dtype | None = None, residual: torch.Tensor | None = None) -> torch.Tensor:
        """x: (M, K) numpy/torch float -> (M, N) CUDA tensor = x @ W (+ bias); bf16 operands, f32 accumulation,
        bias in f32 (npu/xdna1_gemm.py:349-422). f32 output unless `out_dtype`/`out` say otherwise."""
        t_start = time.perf_counter()
        x2 = self._x_device(x)
        if x2.dim() != 2:
            raise ValueError("matmul_t takes a 2-D x; use linear() for n-D inputs")
        M, K = x2.shape
        assert K == w.K, f"K mismatch: x has {K}, weight has {w.K}"
        ev = self._events()
        y = kernels.gemm(x2, w.tensor[:, :K] if w.handle is None else w.tensor, self._bias_device(bias), out=out,
                         out_dtype=out_dtype or self.out_dtype, handle=w.handle, residual=residual)
        self._close("gemm", ev)
        with self._lock:
            self.stats["calls"] += 1
            self.stats["dispatches"] += 1
            self.stats["flops"] += 2.0 * M * K * w.N
            self.stats["total_seconds"] += time.perf_counter() - t_start
        return y

    def matmul(self, x, w: NpuWeight) -> np.ndarray:
        """x: (M, K) -> (M, N) float32 numpy array (copied back to the host)."""
        return self.matmul_t(x, w, out_dtype=torch.float32).cpu().numpy()

    def linear(self, x, w: NpuWeight, bias=None, out_dtype: torch.dtype | None = None,
               residual: torch.Tensor | None = None):
        """x: (..., K) -> (..., N) = x @ W (+ bias) (+ residual, a bf16 (..., N) CUDA tensor added in the GEMM's
        epilogue). torch in -> torch (CUDA) out, numpy in -> numpy out (npu/xdna1_gemm.py:428-448)."""
        is_torch = isinstance(x, torch.Tensor)
        xt = _as_tensor(x)
        shp = tuple(xt.shape)
        x2 = xt.reshape(-1, shp[-1])
        r2 = residual.reshape(-1, w.N) if residual is not None else None
        y = self.matmul_t(x2, w, bias, out_dtype=out_dtype, residual=r2).view(*shp[:-1], w.N)
        return y if is_torch else y.cpu().numpy()

    def linear_geglu(self, x, w: NpuWeight, bias=None, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """GEGLU feed-forward projection in one kernel: x (..., K) with w the resident [2n, K] weight of a GEGLU
        `proj` Linear -> (..., n) = y[..., :n] * gelu(y[..., n:]), y = x @ W^T (+ bias). The reference offloads the
        projection through linear() (npu/xdna1_gemm.py:428-448) and gates on the host."""
        t_start = time.perf_counter()
        xt = _as_tensor(x)
        shp = tuple(xt.shape)
        x2 = self._x_device(xt.reshape(-1, shp[-1]))
        M, K = x2.shape
        assert K == w.K, f"K mismatch: x has {K}, weight has {w.K}"
        ev = self._events()
        y = kernels.gemm_geglu(x2, w.tensor[:, :K] if w.tensor.shape[1] != K else w.tensor, self._bias_device(bias),
                               out_dtype=out_dtype or self.out_dtype)
        self._close("gemm", ev)
        with self._lock:
            self.stats["calls"] += 1
            self.stats["dispatches"] += 1
            self.stats["flops"] += 2.0 * M * K * w.N
            self.stats["total_seconds"] += time.perf_counter() - t_start
        return y.view(*shp[:-1], w.N // 2)

    # -- attention ------------------------------------------------------------------------------
    def attention_fused_fits(self, tq: int, tk: int, d: int, bh: int) -> bool:
        return d % 8 == 0 and 8 <= d <= 256 and tq >= 1 and tk >= 1 and 1 <= bh <= 65535

    def attention_fits(self, tq: int, tk: int, d: int, bh: int | None = None) -> bool:
        """Whether attention() takes this shape; with `bh` the first query for a shape also warms it up
        (npu/xdna1_gemm.py:451-464)."""
        ok = self.attention_fused_fits(tq, tk, d, bh if bh is not None else 1)
        if ok and bh is not None:
            self.attention_warmup(tq, tk, d, bh)
        return ok

    def attention_warmup(self, tq: int, tk: int, d: int, bh: int) -> None:
        """Run the fused kernel once for a shape on zeros (npu/xdna1_gemm.py:466-493)."""
        key = (tq, tk, d, bh)
        if key in self._attn_warm or not self.attention_fused_fits(tq, tk, d, bh):
            return
        self._attn_warm.add(key)
        b = 2 if bh % 2 == 0 else 1
        h = bh // b
        z = torch.zeros((b, tq, h * d), dtype=torch.bfloat16, device=self.device)
        zk = torch.zeros((b, tk, h * d), dtype=torch.bfloat16, device=self.device)
        kernels.attention(z, zk, zk, h, out_dtype=self.out_dtype)

    def _attn_operand(self, t) -> torch.Tensor:
        t = self._x_device(t)
        # TMA addressing: 16-byte aligned base and strides in multiples of 8 elements, else one compact copy.
        if t.data_ptr() % 16 or any(s % 8 for s in t.stride()[:-1]):
            t = t.contiguous()
        return t

    def attention(self, q, k, v, heads: int, scale: float | None = None, skip_reshape: bool = False,
                  skip_output_reshape: bool = False, out_dtype: torch.dtype | None = None, *,
                  group=None) -> torch.Tensor:
        """softmax(Q K^T * scale) V for all (batch, head) pairs in ONE launch (bf16 in, f32 accumulate).

        q/k/v: (b, t, heads*d), or (b, heads, t, d) when skip_reshape. Returns (b, tq, heads*d) (or
        (b, heads, tq, d) when skip_output_reshape), f32 unless `out_dtype` (npu/xdna1_gemm.py:499-533).
        `group` (a torch.distributed process group, every rank holding the whole block on its GPU) splits the pairs
        over the group's ranks in contiguous ranges and all-gathers the result (npu_ai_b200.sharding).
        """
        t_start = time.perf_counter()
        qd, kd, vd = (self._attn_operand(t) for t in (q, k, v))
        # Q read in place: the caller's device tensor itself reached the kernel (no host copy, cast or compaction)
        q_inplace = isinstance(q, torch.Tensor) and q.is_cuda and q.data_ptr() == qd.data_ptr() and q.dtype == qd.dtype
        if skip_reshape:
            b, h, tq, d = qd.shape
            tk = kd.shape[2]
        else:
            b, tq, inner = qd.shape
            h = int(heads)
            d = inner // h
            tk = kd.shape[1]
        if not self.attention_fused_fits(tq, tk, d, b * h):
            raise ValueError(f"attention shape tq={tq} tk={tk} d={d} b*h={b * h} is outside the kernel's range")
        key = (b, tq, tk, h, d)
        ev = self._events()
        if group is not None:
            from .sharding import attention_sharded
            y = attention_sharded(qd, kd, vd, h, group=group, scale=scale, head_major_in=skip_reshape,
                                  head_major_out=skip_output_reshape, out_dtype=out_dtype or self.out_dtype)
        else:
            y = kernels.attention(qd, kd, vd, h, scale=scale, head_major_in=skip_reshape,
                                  head_major_out=skip_output_reshape, out_dtype=out_dtype or self.out_dtype)
        with self._lock:
            sh = self.stats["attn_by_shape"].setdefault(key, [0, 0.0, 0.0, 0.0, 0.0, 0, 0.0])
            self._close("attn", ev, key)
            wall = time.perf_counter() - t_start
            sh[0] += 1
            sh[2] += wall
            sh[5] += int(q_inplace)
            sh[6] += wall
            self.stats["attn_fused_calls"] += 1
            self.stats["attn_fused_q_inplace"] += int(q_inplace)
            self.stats["attn_fused_flops"] += 4.0 * b * h * tq * tk * d
            self.stats["attn_fused_seconds"] += wall
        return y

    # -- reporting ------------------------------------------------------------------------------
    def summary(self) -> str:
        """Same shape of text as the reference (npu/xdna1_gemm.py:755-773), with GPU time in place of NPU time."""
        self.flush_timing()
        s = self.stats
        gf = s["flops"] / s["npu_seconds"] / 1e9 if s["npu_seconds"] else 0.0
        msg = (f"NpuGemm[B200]: {s['calls']} calls, {s['dispatches']} dispatches, GPU {s['npu_seconds']:.3f}s, "
               f"wall {s['total_seconds']:.3f}s, {gf:.0f} GFLOPS (GPU time), {s['program_switches']} program switches, "
               f"setup {s['compile_seconds']:.2f}s, {s['buffers']} pooled buffers "
               f"({s['buffer_bytes'] / 2**20:.0f} MiB, {s['alloc_seconds']:.2f}s to allocate)")
        if s["attn_fused_calls"]:
            ns = max(s["attn_fused_npu_seconds"], 1e-9)
            msg += (f"; fused attention: {s['attn_fused_calls']} blocks, GPU {s['attn_fused_npu_seconds']:.3f}s, "
                    f"wall {s['attn_fused_seconds']:.3f}s, "
                    f"{s['attn_fused_flops'] / max(s['attn_fused_seconds'], 1e-9) / 1e9:.0f} GFLOPS end-to-end "
                    f"({s['attn_fused_flops'] / ns / 1e9:.0f} GPU)")
            for key, (n, conv, sub, gpu, sync, inpl, wall) in sorted(s["attn_by_shape"].items()):
                msg += (f"; {key}: {n} blocks, per block wall {wall / n * 1e3:.2f} ms = launch {sub / n * 1e3:.3f} "
                        f"+ GPU {gpu / n * 1e3:.3f} (timed calls), operands in place {inpl}/{n}")
        return msg


def _release_handle(handle) -> None:
    if handle is not None:
        try:
            kernels.release_weight(handle)
        except Exception:  # the library may already be unloaded at interpreter exit
            pass
