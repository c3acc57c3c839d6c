// torch_ops.cpp - the GEMM and the fused attention as torch operators (torch.ops.npub200.gemm / .attention).
//
// The reference hands each request to its NPU as one XRT command: NpuProgram.submit_gemm / submit_attn
// (npu/xdna1_program.py:441-473) with three buffer objects and 13 int32 parameters. Here the same two requests are
// operators registered with the torch dispatcher (TORCH_LIBRARY), so torch code, CUDA-graph capture and
// torch.compile-free callers see them as ordinary ops on CUDA tensors. Each one checks its tensors, then calls
// the library's C ABI (include/npu_b200.h) on at::cuda::getCurrentCUDAStream() of the tensors' device; nothing is
// computed here and there is no CPU kernel (CPU tensors are refused by the dispatcher). Errors raise like the
// reference's runner: an invalid request is a ValueError, anything else a RuntimeError.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <cmath>
#include <optional>

#include "npu_b200.h"

namespace {

void check_rc(int rc, const char* what) {
  if (rc == NPUB200_OK) return;
  const char* msg = npub200_last_error();
  // EINVAL: the request itself (the reference's ValueError for shapes its programs cannot take,
  // npu/xdna1_gemm.py:227-229); anything else, a legal request without a variant or a device failure, is a
  // RuntimeError (a failed NPU command, npu/xdna1_program.py:475-479), as in the ctypes binding.
  TORCH_CHECK_VALUE(rc != NPUB200_EINVAL, what, ": ", msg);
  TORCH_CHECK(false, what, ": ", msg, " (code ", rc, ")");
}

int dtype_code(const at::Tensor& t, const char* name) {
  if (t.scalar_type() == at::kBFloat16) return NPUB200_DTYPE_BF16;
  if (t.scalar_type() == at::kFloat) return NPUB200_DTYPE_F32;
  TORCH_CHECK_VALUE(false, name, " must be bf16 or f32, got ", t.scalar_type());
  return -1;
}

void check_operand(const at::Tensor& t, const at::Tensor& ref, const char* name) {
  TORCH_CHECK_VALUE(t.is_cuda() && t.device() == ref.device(), name, " must be a CUDA tensor on ", ref.device());
  TORCH_CHECK_VALUE(t.scalar_type() == at::kBFloat16, name, " must be bf16, got ", t.scalar_type());
  TORCH_CHECK_VALUE(t.dim() >= 1 && t.stride(-1) == 1, name, " must have a contiguous last dimension");
}

void* stream_of(const at::Tensor& t) { return at::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

// out[M, N] = x[M, K] . w[N, K]^T (+ bias) (+ residual); bf16 operands, f32 accumulation, bias in f32.
// Replaces NpuGemm.matmul_t (npu/xdna1_gemm.py:349-422) / NpuProgram.submit_gemm (npu/xdna1_program.py:451-454).
at::Tensor gemm(const at::Tensor& x, const at::Tensor& w, const std::optional<at::Tensor>& bias,
                const std::optional<at::Tensor>& out, int64_t variant, std::optional<at::ScalarType> out_dtype,
                int64_t weight_handle, const std::optional<at::Tensor>& residual) {
  check_operand(x, x, "x");
  check_operand(w, x, "w");
  TORCH_CHECK_VALUE(x.dim() == 2 && w.dim() == 2, "gemm takes 2-D x [M, K] and w [N, K]");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK_VALUE(w.size(1) == K, "K mismatch: x has ", K, ", w has ", w.size(1));
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor y;
  if (out.has_value()) {
    y = *out;
    TORCH_CHECK_VALUE(y.is_cuda() && y.device() == x.device() && y.dim() == 2 && y.size(0) == M && y.size(1) == N &&
                          y.stride(1) == 1,
                      "out must be an [M, N] CUDA matrix with contiguous rows on x's device");
  } else {
    y = at::empty({M, N}, x.options().dtype(out_dtype.value_or(at::kFloat)));
  }
  const int out_code = dtype_code(y, "out");
  const void* b_ptr = nullptr;
  int b_code = NPUB200_DTYPE_BF16;
  if (bias.has_value()) {
    const at::Tensor& b = *bias;
    TORCH_CHECK_VALUE(b.is_cuda() && b.device() == x.device() && b.numel() == N && b.is_contiguous(),
                      "bias must be a contiguous [N] CUDA vector on x's device");
    b_code = dtype_code(b, "bias");
    b_ptr = b.data_ptr();
  }
  void* st = stream_of(x);
  if (residual.has_value()) {
    const at::Tensor& r = *residual;
    check_operand(r, x, "residual");
    TORCH_CHECK_VALUE(r.dim() == 2 && r.size(0) == M && r.size(1) == N, "residual must be [M, N]");
    size_t ws_bytes = 0;
    check_rc(npub200_gemm_workspace_size(x.data_ptr(), x.stride(0), M, K, w.data_ptr(), w.stride(0), N,
                                         int(variant), &ws_bytes),
             "npub200::gemm");
    at::Tensor ws = at::empty({int64_t(ws_bytes)}, x.options().dtype(at::kByte));
    check_rc(npub200_gemm_residual(x.data_ptr(), x.stride(0), M, K, w.data_ptr(), w.stride(0), N, b_ptr, b_code,
                                   r.data_ptr(), r.stride(0), y.data_ptr(), y.stride(0), out_code,
                                   ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, int(variant), st),
             "npub200::gemm");
    return y;
  }
  size_t ws_bytes = 0;
  check_rc(npub200_gemm_workspace_size(x.data_ptr(), x.stride(0), M, K, weight_handle ? nullptr : w.data_ptr(),
                                       w.stride(0), N, int(variant), &ws_bytes),
           "npub200::gemm");
  at::Tensor ws = at::empty({int64_t(ws_bytes)}, x.options().dtype(at::kByte));
  void* ws_ptr = ws_bytes ? ws.data_ptr() : nullptr;
  if (weight_handle != 0) {
    check_rc(npub200_gemm_w(x.data_ptr(), x.stride(0), M, K, weight_handle, b_ptr, b_code, y.data_ptr(), y.stride(0),
                            out_code, ws_ptr, ws_bytes, int(variant), st),
             "npub200::gemm");
  } else {
    check_rc(npub200_gemm(x.data_ptr(), x.stride(0), M, K, w.data_ptr(), w.stride(0), N, b_ptr, b_code, y.data_ptr(),
                          y.stride(0), out_code, ws_ptr, ws_bytes, int(variant), st),
             "npub200::gemm");
  }
  return y;
}

// (batch, seq, head) element strides of a (B, S, H*d) tensor or, head-major, a (B, H, S, d) tensor.
void bsh_strides(const at::Tensor& t, bool head_major, int64_t d, int64_t* sb, int64_t* ss, int64_t* sh) {
  *sb = t.stride(0);
  if (head_major) {
    *sh = t.stride(1);
    *ss = t.stride(2);
  } else {
    *ss = t.stride(1);
    *sh = d;
  }
}

void check_layout(const at::Tensor& t, bool head_major, int64_t B, int64_t H, int64_t S, int64_t d,
                  int64_t row_stride, const char* name) {
  if (head_major) {
    TORCH_CHECK_VALUE(t.dim() == 4 && t.size(0) == B && t.size(1) == H && t.size(2) == S && t.size(3) == d, name,
                      " must be (B, H, S, d) = (", B, ", ", H, ", ", S, ", ", d, "), got ", t.sizes());
  } else {
    TORCH_CHECK_VALUE(t.dim() == 3 && t.size(0) == B && t.size(1) == S && t.size(2) == H * d, name,
                      " must be (B, S, H*d) = (", B, ", ", S, ", ", H * d, "), got ", t.sizes());
  }
  const int64_t rs = head_major ? t.stride(2) : t.stride(1);
  TORCH_CHECK_VALUE(row_stride <= 0 || row_stride == rs, name, " row stride ", rs, " differs from the declared ",
                    row_stride);
}

// softmax(q k^T * scale) v for every (batch, head) pair in one launch. Replaces NpuGemm.attention /
// _attention_fused (npu/xdna1_gemm.py:499-752) and NpuProgram.submit_attn (npu/xdna1_program.py:461-473). The
// declared row strides are checked against the tensors (0: take the tensor's); scale <= 0 means d^-0.5.
at::Tensor attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const std::optional<at::Tensor>& out,
                     int64_t B, int64_t H, int64_t Sq, int64_t Skv, int64_t d, int64_t q_row_stride,
                     int64_t kv_row_stride, int64_t o_row_stride, bool head_major_in, bool head_major_out,
                     double scale, int64_t variant, std::optional<at::ScalarType> out_dtype) {
  check_operand(q, q, "q");
  check_operand(k, q, "k");
  check_operand(v, q, "v");
  check_layout(q, head_major_in, B, H, Sq, d, q_row_stride, "q");
  check_layout(k, head_major_in, B, H, Skv, d, kv_row_stride, "k");
  check_layout(v, head_major_in, B, H, Skv, d, kv_row_stride, "v");
  const c10::cuda::CUDAGuard guard(q.device());
  at::Tensor o;
  if (out.has_value()) {
    o = *out;
    TORCH_CHECK_VALUE(o.is_cuda() && o.device() == q.device() && o.stride(-1) == 1,
                      "out must be a CUDA tensor on q's device with a contiguous last dimension");
  } else {
    o = head_major_out ? at::empty({B, H, Sq, d}, q.options().dtype(out_dtype.value_or(at::kFloat)))
                       : at::empty({B, Sq, H * d}, q.options().dtype(out_dtype.value_or(at::kFloat)));
  }
  check_layout(o, head_major_out, B, H, Sq, d, o_row_stride, "out");
  int64_t qs[3], ks[3], vs[3], os[3];
  bsh_strides(q, head_major_in, d, &qs[0], &qs[1], &qs[2]);
  bsh_strides(k, head_major_in, d, &ks[0], &ks[1], &ks[2]);
  bsh_strides(v, head_major_in, d, &vs[0], &vs[1], &vs[2]);
  bsh_strides(o, head_major_out, d, &os[0], &os[1], &os[2]);
  const float s = scale > 0 ? float(scale) : float(1.0 / std::sqrt(double(d)));
  check_rc(npub200_attention(q.data_ptr(), qs[0], qs[1], qs[2], k.data_ptr(), ks[0], ks[1], ks[2], v.data_ptr(),
                             vs[0], vs[1], vs[2], o.data_ptr(), os[0], os[1], os[2], dtype_code(o, "out"), B, H, Sq,
                             Skv, d, s, int(variant), stream_of(q)),
           "npub200::attention");
  return o;
}

}  // namespace

TORCH_LIBRARY(npub200, m) {
  m.def("gemm(Tensor x, Tensor w, Tensor? bias=None, Tensor? out=None, int variant=0, ScalarType? out_dtype=None, "
        "int weight_handle=0, Tensor? residual=None) -> Tensor");
  m.def("attention(Tensor q, Tensor k, Tensor v, Tensor? out, int B, int H, int Sq, int Skv, int d, "
        "int q_row_stride, int kv_row_stride, int o_row_stride, bool head_major_in, bool head_major_out, "
        "float scale, int variant, ScalarType? out_dtype=None) -> Tensor");
}

TORCH_LIBRARY_IMPL(npub200, CUDA, m) {
  m.impl("gemm", &gemm);
  m.impl("attention", &attention);
}
