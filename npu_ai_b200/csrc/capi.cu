// capi.cu - the extern "C" entry points of libnpub200 (declared in include/npu_b200.h) and the host plumbing
// behind them: argument checks, per-device state (SM count, status word), TMA descriptor encoding, and the
// resident-weight registry.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "npu_b200.h"
#include "internal.h"

namespace npub200 {

// One status word per device; kernels OR StatusBits into it. Read and cleared by npub200_status_read.
__device__ uint32_t g_status_word;

namespace {

thread_local char g_last_error[1024] = {0};
std::mutex g_dev_mutex;
DeviceInfo g_devices[64];
std::atomic<uint64_t> g_timeout_ns{0};
std::atomic<uint32_t> g_debug_flags{0};
constexpr uint64_t kDefaultTimeoutNs = 4000000000ull;  // 4 s per wait: far above any legitimate stall

struct WeightEntry {
  const void* w;
  int64_t n, k, ldw;
  int device;
  std::unordered_map<int, CUtensorMap> maps;  // per N tile
};
std::mutex g_w_mutex;
std::unordered_map<int64_t, WeightEntry> g_weights;
int64_t g_next_handle = 1;

}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return kOk;
  return fail(kErrCuda, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

uint64_t wait_timeout_ns() {
  const uint64_t t = g_timeout_ns.load();
  return t ? t : kDefaultTimeoutNs;
}

int current_device_info(const DeviceInfo** out) {
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= 64) return fail(kErrInvalid, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  DeviceInfo& d = g_devices[dev];
  if (d.device < 0) {
    cudaDeviceProp prop;
    if (int rc = check_cuda(cudaGetDeviceProperties(&prop, dev), "cudaGetDeviceProperties")) return rc;
    if (prop.major != 10)
      return fail(kErrUnsupported, "device %d (%s, sm_%d%d) is not a B200-class sm_100 GPU", dev, prop.name,
                  prop.major, prop.minor);
    void* p = nullptr;
    if (int rc = check_cuda(cudaGetSymbolAddress(&p, g_status_word), "cudaGetSymbolAddress(status)")) return rc;
    d.sms = prop.multiProcessorCount;
    d.smem_optin = int(prop.sharedMemPerBlockOptin);
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    d.status = static_cast<uint32_t*>(p);
    d.device = dev;
  }
  *out = &d;
  return kOk;
}

int encode_tiled_fn(EncodeTiledFn* out) {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  static int rc_once = kOk;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
      rc_once = kErrCuda;
    } else {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  if (fn == nullptr) return fail(kErrCuda, "cuTensorMapEncodeTiled is unavailable from the CUDA driver");
  *out = fn;
  return rc_once;
}

}  // namespace npub200

using namespace npub200;

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// TMA needs a 16-byte aligned base, a row stride that is a multiple of 16 bytes and >= the row length.
bool tma_rows_ok(const void* p, int64_t ld, int64_t cols) { return aligned16(p) && ld % 8 == 0 && ld >= cols; }

int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// Workspace layout: [4 KiB reserved][split bytes the plan reports][repacked x][repacked W]. Split K reduces inside a
// cluster's shared memory, so plans report no split bytes and the workspace holds only operands that TMA cannot
// read as given, repacked; the leading region stays reserved so the layout does not depend on the plan.
constexpr size_t kCounterRegion = 4096;
struct WsLayout {
  size_t split_bytes = 0;
  size_t x_off = 0, x_bytes = 0;
  size_t w_off = 0, w_bytes = 0;
  size_t total = 0;
};

WsLayout gemm_ws_layout(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                        int variant, int sms, int geglu = 0) {
  WsLayout L;
  const int64_t kp = round_up(k, 8);
  const bool pad_k = (k % 8) != 0;
  const int64_t w_rows = geglu ? 2 * n : n;
  L.split_bytes = (sms > 0 && !geglu) ? gemm_plan(m, n, kp, sms, variant).split_ws_bytes : 0;  // counters + partials
  size_t off = L.split_bytes > 0 ? L.split_bytes : kCounterRegion;
  if (pad_k || !tma_rows_ok(x, ldx, k)) {
    L.x_off = off;
    L.x_bytes = size_t(round_up(m * kp * 2, 256));
    off += L.x_bytes;
  }
  if (w != nullptr && (pad_k || !tma_rows_ok(w, ldw, k))) {
    L.w_off = off;
    L.w_bytes = size_t(round_up(w_rows * kp * 2, 256));
    off += L.w_bytes;
  }
  L.total = (L.split_bytes > 0 || L.x_bytes > 0 || L.w_bytes > 0) ? off : 0;
  return L;
}

int check_gemm_common(int64_t m, int64_t k, int64_t n, int bias_dtype, const void* out, int64_t ldo,
                      int out_dtype) {
  if (m <= 0 || k <= 0 || n <= 0)
    return fail(kErrInvalid, "GEMM sizes must be positive (M=%lld K=%lld N=%lld)", (long long)m, (long long)k,
                (long long)n);
  if (out == nullptr) return fail(kErrInvalid, "GEMM output pointer is null");
  if (ldo < n) return fail(kErrInvalid, "output row stride %lld < N=%lld", (long long)ldo, (long long)n);
  if (out_dtype != NPUB200_DTYPE_BF16 && out_dtype != NPUB200_DTYPE_F32)
    return fail(kErrInvalid, "unknown output dtype code %d", out_dtype);
  if (bias_dtype != NPUB200_DTYPE_BF16 && bias_dtype != NPUB200_DTYPE_F32)
    return fail(kErrInvalid, "unknown bias dtype code %d", bias_dtype);
  return kOk;
}

}  // namespace

namespace npub200 {

size_t gemm_workspace_bytes(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                            int variant, int sms, int geglu) {
  return gemm_ws_layout(x, ldx, m, k, w, ldw, n, variant, sms, geglu).total;
}

int gemm_with_workspace(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                        const CUtensorMap* w_map, const void* bias, int bias_dtype, void* out, int64_t ldo,
                        int out_dtype, void* workspace, size_t workspace_bytes, int variant, void* stream,
                        int geglu, const void* residual, int64_t ldr) {
  if (int rc = check_gemm_common(m, k, n, bias_dtype, out, ldo, out_dtype)) return rc;
  if (x == nullptr || w == nullptr) return fail(kErrInvalid, "GEMM operand pointer is null");
  if (ldx < k) return fail(kErrInvalid, "x row stride %lld < K=%lld", (long long)ldx, (long long)k);
  if (ldw < k) return fail(kErrInvalid, "W row stride %lld < K=%lld", (long long)ldw, (long long)k);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GemmProblem p;
  memset(&p, 0, sizeof(p));
  p.x = x;
  p.ldx = ldx;
  p.w = w;
  p.ldw = ldw;
  p.bias = bias;
  p.bias_f32 = bias_dtype == NPUB200_DTYPE_F32;
  p.out = out;
  p.ldo = ldo;
  p.out_f32 = out_dtype == NPUB200_DTYPE_F32;
  p.M = m;
  p.N = n;
  p.K = k;
  p.variant = variant;
  p.w_map_cache = w_map;
  p.debug = g_debug_flags.load();
  p.geglu = geglu;
  if (residual != nullptr && ldr < n) return fail(kErrInvalid, "residual row stride %lld < N=%lld", (long long)ldr,
                                                  (long long)n);
  p.residual = residual;
  p.ldr = ldr;

  const DeviceInfo* dev = nullptr;
  if (int rc = current_device_info(&dev)) return rc;
  const bool pad_k = (k % 8) != 0;
  const bool x_ok = !pad_k && tma_rows_ok(x, ldx, k);
  const bool w_ok = !pad_k && tma_rows_ok(w, ldw, k);
  const WsLayout L = gemm_ws_layout(x, ldx, m, k, w_map ? nullptr : w, ldw, n, variant, dev->sms, geglu);
  if (workspace != nullptr && !aligned16(workspace)) return fail(kErrInvalid, "workspace must be 16-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int64_t kp = round_up(k, 8);
  if (!x_ok || !w_ok) {
    // Repack path: dense copies with K padded to a multiple of 8 (zero columns add nothing to the dot products).
    if (ws == nullptr || workspace_bytes < L.total)
      return fail(kErrInvalid, "this GEMM needs a %zu-byte workspace (operands are not TMA-addressable), got %zu",
                  L.total, workspace_bytes);
    if (!x_ok) {
      if (int rc = repack_rows_bf16(x, ldx, m, k, ws + L.x_off, kp, st)) return rc;
      p.x = ws + L.x_off;
      p.ldx = kp;
    }
    if (!w_ok) {
      if (int rc = repack_rows_bf16(w, ldw, geglu ? 2 * n : n, k, ws + L.w_off, kp, st)) return rc;
      p.w = ws + L.w_off;
      p.ldw = kp;
      p.w_map_cache = nullptr;
    }
    if (pad_k) p.K = kp;
  }
  // Split-K bytes the plan asked for (none: split K reduces inside a cluster).
  if (ws != nullptr && L.split_bytes > 0 && workspace_bytes >= L.split_bytes) {
    p.ws_split = ws;
    p.ws_split_bytes = L.split_bytes;
  }
  return gemm_launch(p, st);
}

}  // namespace npub200

namespace {

int gemm_common(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                const CUtensorMap* w_map, const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype,
                void* workspace, size_t workspace_bytes, int variant, void* stream) {
  return gemm_with_workspace(x, ldx, m, k, w, ldw, n, w_map, bias, bias_dtype, out, ldo, out_dtype, workspace,
                             workspace_bytes, variant, stream);
}

}  // namespace

extern "C" {

int npub200_version(void) { return 100; }

const char* npub200_last_error(void) { return g_last_error; }

int npub200_device_sms(int* sms_out) {
  const DeviceInfo* d = nullptr;
  if (int rc = current_device_info(&d)) return rc;
  if (sms_out) *sms_out = d->sms;
  return kOk;
}

int npub200_weight_register(const void* w, int64_t n, int64_t k, int64_t ldw, int64_t* handle_out) {
  if (w == nullptr || handle_out == nullptr) return fail(kErrInvalid, "null weight or handle pointer");
  if (n <= 0 || k <= 0) return fail(kErrInvalid, "weight sizes must be positive (N=%lld K=%lld)", (long long)n,
                                    (long long)k);
  if (k % 8 != 0 || !tma_rows_ok(w, ldw, k))
    return fail(kErrInvalid,
                "resident weights need K %% 8 == 0, ldw %% 8 == 0 and a 16-byte aligned base (got K=%lld ldw=%lld)",
                (long long)k, (long long)ldw);
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  std::lock_guard<std::mutex> lock(g_w_mutex);
  const int64_t h = g_next_handle++;
  WeightEntry e;
  e.w = w;
  e.n = n;
  e.k = k;
  e.ldw = ldw;
  e.device = dev;
  g_weights.emplace(h, std::move(e));
  *handle_out = h;
  return kOk;
}

int npub200_weight_release(int64_t handle) {
  std::lock_guard<std::mutex> lock(g_w_mutex);
  if (g_weights.erase(handle) == 0) return fail(kErrInvalid, "unknown weight handle %lld", (long long)handle);
  return kOk;
}

int npub200_gemm_workspace_size(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw,
                                int64_t n, int variant, size_t* bytes_out) {
  if (bytes_out == nullptr) return fail(kErrInvalid, "null output pointer");
  if (m <= 0 || k <= 0 || n <= 0) return fail(kErrInvalid, "GEMM sizes must be positive");
  const DeviceInfo* d = nullptr;
  if (int rc = current_device_info(&d)) return rc;
  *bytes_out = gemm_ws_layout(x, ldx, m, k, w, ldw, n, variant, d->sms).total;
  return kOk;
}

int npub200_gemm_plan(int64_t m, int64_t n, int64_t k, int variant, int* tile_n_out, int* splits_out) {
  if (m <= 0 || n <= 0 || k <= 0) return fail(kErrInvalid, "GEMM sizes must be positive");
  const DeviceInfo* d = nullptr;
  if (int rc = current_device_info(&d)) return rc;
  const GemmPlan plan = gemm_plan(m, n, round_up(k, 8), d->sms, variant);
  if (tile_n_out) *tile_n_out = gemm_plan_variant(plan);
  if (splits_out) *splits_out = plan.splits;
  return kOk;
}

int npub200_gemm(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                 const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype, void* workspace,
                 size_t workspace_bytes, int variant, void* stream) {
  if (int rc = check_gemm_common(m, k, n, bias_dtype, out, ldo, out_dtype)) return rc;
  return gemm_common(x, ldx, m, k, w, ldw, n, nullptr, bias, bias_dtype, out, ldo, out_dtype, workspace,
                     workspace_bytes, variant, stream);
}

int npub200_gemm_residual(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                          const void* bias, int bias_dtype, const void* residual, int64_t ldr, void* out, int64_t ldo,
                          int out_dtype, void* workspace, size_t workspace_bytes, int variant, void* stream) {
  if (int rc = check_gemm_common(m, k, n, bias_dtype, out, ldo, out_dtype)) return rc;
  if (residual == nullptr) return fail(kErrInvalid, "npub200_gemm_residual needs a residual");
  return gemm_with_workspace(x, ldx, m, k, w, ldw, n, nullptr, bias, bias_dtype, out, ldo, out_dtype, workspace,
                             workspace_bytes, variant, stream, 0, residual, ldr);
}

int npub200_gemm_geglu(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                       const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype, void* workspace,
                       size_t workspace_bytes, int variant, void* stream) {
  if (int rc = check_gemm_common(m, k, n, bias_dtype, out, ldo, out_dtype)) return rc;
  if (n > INT32_MAX / 4) return fail(kErrInvalid, "GEGLU width %lld too large", (long long)n);
  return gemm_with_workspace(x, ldx, m, k, w, ldw, n, nullptr, bias, bias_dtype, out, ldo, out_dtype, workspace,
                             workspace_bytes, variant, stream, 1);
}

int npub200_conv3x3(const void* x, int64_t n, int64_t h, int64_t w, int64_t cin, const void* weight, int64_t cout,
                    const void* bias, int bias_dtype, int64_t bias_img_stride, const void* residual, int64_t ldr,
                    void* out, int64_t ldo, int out_dtype, void* workspace, size_t workspace_bytes, int variant,
                    void* stream) {
  if (out_dtype != NPUB200_DTYPE_BF16 && out_dtype != NPUB200_DTYPE_F32)
    return fail(kErrInvalid, "unknown output dtype code %d", out_dtype);
  if (bias_dtype != NPUB200_DTYPE_BF16 && bias_dtype != NPUB200_DTYPE_F32)
    return fail(kErrInvalid, "unknown bias dtype code %d", bias_dtype);
  if (bias_img_stride < 0) return fail(kErrInvalid, "negative bias row stride");
  ConvProblem p;
  memset(&p, 0, sizeof(p));
  p.x = x;
  p.n = n;
  p.h = h;
  p.w = w;
  p.cin = cin;
  p.wt = weight;
  p.cout = cout;
  p.bias = bias;
  p.bias_f32 = bias_dtype == NPUB200_DTYPE_F32;
  p.bias_img_stride = bias_img_stride;
  p.residual = residual;
  p.ldr = ldr;
  p.out = out;
  p.ldo = ldo;
  p.out_f32 = out_dtype == NPUB200_DTYPE_F32;
  p.variant = variant;
  p.debug = g_debug_flags.load();
  p.ws_split = workspace;
  p.ws_split_bytes = workspace_bytes;
  return conv3x3_launch(p, static_cast<cudaStream_t>(stream));
}

int npub200_group_norm(const void* x, int64_t n, int64_t hw, int64_t c, int64_t groups, const float* gamma,
                       const float* beta, float eps, int apply_silu, void* out, float* stats, void* stream) {
  return group_norm_launch(x, n, hw, c, groups, gamma, beta, eps, apply_silu, out, stats,
                           static_cast<cudaStream_t>(stream), g_debug_flags.load());
}

int npub200_layer_norm(const void* x, int64_t rows, int64_t cols, int64_t ldx, const void* gamma, const void* beta,
                       int param_dtype, float eps, void* out, int64_t ldo, void* stream) {
  if (param_dtype != NPUB200_DTYPE_F32 && param_dtype != NPUB200_DTYPE_BF16)
    return fail(kErrInvalid, "layer_norm: gamma/beta dtype must be f32 or bf16 (got %d)", param_dtype);
  return layer_norm_launch(x, rows, cols, ldx, gamma, beta, param_dtype == NPUB200_DTYPE_F32 ? 1 : 0, eps, out, ldo,
                           static_cast<cudaStream_t>(stream));
}

int npub200_upsample_nearest2x(const void* x, int64_t n, int64_t h, int64_t w, int64_t c, void* out, void* stream) {
  return upsample_nearest2x_launch(x, n, h, w, c, out, static_cast<cudaStream_t>(stream));
}

int npub200_concat_channels(const void* a, int64_t lda, int64_t ca, const void* b, int64_t ldb, int64_t cb,
                            int64_t pixels, void* out, int64_t ldo, void* stream) {
  return concat_channels_launch(a, lda, ca, b, ldb, cb, pixels, out, ldo, static_cast<cudaStream_t>(stream));
}

int npub200_group_norm_scratch_size(int64_t n, int64_t groups, size_t* bytes_out) {
  if (bytes_out == nullptr) return fail(kErrInvalid, "null output pointer");
  if (n <= 0 || groups <= 0) return fail(kErrInvalid, "group_norm sizes must be positive");
  *bytes_out = group_norm_scratch_bytes(n, groups);
  return kOk;
}

int npub200_conv3x3_workspace_size(int64_t n, int64_t h, int64_t w, int64_t cin, int64_t cout, int variant,
                                   size_t* bytes_out) {
  if (bytes_out == nullptr) return fail(kErrInvalid, "null output pointer");
  const DeviceInfo* d = nullptr;
  if (int rc = current_device_info(&d)) return rc;
  *bytes_out = conv3x3_workspace_bytes(n, h, w, cin, cout, variant, d->sms);
  return kOk;
}

int npub200_gemm_w(const void* x, int64_t ldx, int64_t m, int64_t k, int64_t weight, const void* bias,
                   int bias_dtype, void* out, int64_t ldo, int out_dtype, void* workspace, size_t workspace_bytes,
                   int variant, void* stream) {
  const void* w = nullptr;
  int64_t n = 0, ldw = 0;
  CUtensorMap map;
  const CUtensorMap* map_ptr = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_w_mutex);
    auto it = g_weights.find(weight);
    if (it == g_weights.end()) return fail(kErrInvalid, "unknown weight handle %lld", (long long)weight);
    WeightEntry& e = it->second;
    if (e.k != k) return fail(kErrInvalid, "K mismatch: x has %lld, weight has %lld", (long long)k, (long long)e.k);
    w = e.w;
    n = e.n;
    ldw = e.ldw;
    if (int rc = check_gemm_common(m, k, n, bias_dtype, out, ldo, out_dtype)) return rc;
    const DeviceInfo* d = nullptr;
    if (int rc = current_device_info(&d)) return rc;
    if (d->device != e.device) return fail(kErrInvalid, "weight was registered on device %d, current is %d",
                                           e.device, d->device);
    const GemmPlan plan = gemm_plan(m, n, k, d->sms, variant);
    const int box_rows = gemm_plan_box_rows(plan, false);
    auto mit = e.maps.find(box_rows);
    if (mit == e.maps.end()) {
      CUtensorMap fresh;
      if (int rc = gemm_encode_b_map(e.w, e.ldw, e.n, e.k, box_rows, &fresh)) return rc;
      mit = e.maps.emplace(box_rows, fresh).first;
    }
    map = mit->second;
    map_ptr = &map;
    variant = gemm_plan_variant(plan);  // the launch takes the same plan the map was encoded for
  }
  return gemm_common(x, ldx, m, k, w, ldw, n, map_ptr, bias, bias_dtype, out, ldo, out_dtype, workspace,
                     workspace_bytes, variant, stream);
}

int npub200_attention(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, const void* k, int64_t k_sb,
                      int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                      void* out, int64_t o_sb, int64_t o_ss, int64_t o_sh, int out_dtype, int64_t batch,
                      int64_t heads, int64_t sq, int64_t skv, int64_t head_dim, float scale, int variant,
                      void* stream) {
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(kErrInvalid, "attention tensor pointer is null");
  if (batch <= 0 || heads <= 0 || sq <= 0 || skv <= 0 || head_dim <= 0)
    return fail(kErrInvalid, "attention sizes must be positive (B=%lld H=%lld Sq=%lld Skv=%lld D=%lld)",
                (long long)batch, (long long)heads, (long long)sq, (long long)skv, (long long)head_dim);
  if (out_dtype != NPUB200_DTYPE_BF16 && out_dtype != NPUB200_DTYPE_F32)
    return fail(kErrInvalid, "unknown output dtype code %d", out_dtype);
  AttnProblem p;
  memset(&p, 0, sizeof(p));
  p.q = q;
  p.k = k;
  p.v = v;
  p.o = out;
  p.q_sb = q_sb;
  p.q_ss = q_ss;
  p.q_sh = q_sh;
  p.k_sb = k_sb;
  p.k_ss = k_ss;
  p.k_sh = k_sh;
  p.v_sb = v_sb;
  p.v_ss = v_ss;
  p.v_sh = v_sh;
  p.o_sb = o_sb;
  p.o_ss = o_ss;
  p.o_sh = o_sh;
  p.B = batch;
  p.H = heads;
  p.Sq = sq;
  p.Skv = skv;
  p.D = head_dim;
  p.scale = scale;
  p.out_f32 = out_dtype == NPUB200_DTYPE_F32;
  p.variant = variant;
  p.debug = g_debug_flags.load();
  return attention_launch(p, static_cast<cudaStream_t>(stream));
}

int npub200_status_read(void* stream, uint32_t* bits_out, int clear) {
  const DeviceInfo* d = nullptr;
  if (int rc = current_device_info(&d)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_cuda(cudaStreamSynchronize(st), "cudaStreamSynchronize")) return rc;
  uint32_t bits = 0;
  if (int rc = check_cuda(cudaMemcpyFromSymbol(&bits, g_status_word, sizeof(bits)), "read status word")) return rc;
  if (clear && bits) {
    const uint32_t zero = 0;
    if (int rc = check_cuda(cudaMemcpyToSymbol(g_status_word, &zero, sizeof(zero)), "clear status word")) return rc;
  }
  if (bits_out) *bits_out = bits;
  return kOk;
}

int npub200_set_wait_timeout_ns(uint64_t ns) {
  g_timeout_ns.store(ns);
  return kOk;
}

int npub200_set_debug_flags(uint32_t flags) {
  g_debug_flags.store(flags);
  return kOk;
}

}  // extern "C"
