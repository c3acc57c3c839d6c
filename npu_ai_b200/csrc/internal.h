// internal.h - host-side plumbing shared by the translation units of libnpub200 (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "sm100_ptx.cuh"

namespace npub200 {

// Launch with programmatic dependent launch allowed: the kernel may start while the previous kernel on the stream
// finishes, so it must wait (pdl_wait) before touching memory that kernel writes; it lets the next one start early
// with pdl_launch_dependents.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Error codes returned by the C entry points (mirrored in include/npu_b200.h).
constexpr int kOk = 0;
constexpr int kErrInvalid = -1;      // bad shape / stride / alignment / dtype: the caller's mistake
constexpr int kErrCuda = -2;         // a CUDA runtime or driver call failed
constexpr int kErrUnsupported = -3;  // a legal request this build has no kernel variant for
constexpr int kErrDevice = -4;       // a kernel reported a failure through its status word

// Records the message of the last failing call on this thread and returns `code`.
int fail(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);

struct DeviceInfo {
  int device = -1;
  int sms = 0;
  int smem_optin = 0;
  int cc_major = 0, cc_minor = 0;
  uint32_t* status = nullptr;  // device address of this device's status word
};
// Cached properties of the current device (initialised on first use per device).
int current_device_info(const DeviceInfo** out);

// Per-wait deadline handed to kernels (nanoseconds); tests shorten it through the C ABI.
uint64_t wait_timeout_ns();

// cuTensorMapEncodeTiled, resolved through the runtime's driver entry point (no link-time libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
int encode_tiled_fn(EncodeTiledFn* out);

// ---- GEMM --------------------------------------------------------------------------------------------------------
struct GemmProblem {
  const void* x;  // [M, K] bf16, row stride ldx elements
  int64_t ldx;
  const void* w;  // [N, K] bf16 (nn.Linear layout), row stride ldw elements
  int64_t ldw;
  const void* bias;  // [N] or null
  int bias_f32;      // 1: bias is f32, 0: bf16
  void* out;         // [M, N], row stride ldo elements
  int64_t ldo;
  int out_f32;       // 1: f32 output, 0: bf16
  int64_t M, N, K;
  int variant;       // 0 = automatic, else a forced N tile (64, 96, 128, 160, 192, 256)
  const CUtensorMap* w_map_cache;  // optional cached B tensor map (matching the chosen tile), may be null
  void* ws_split;                  // caller workspace (split K needs none: it reduces inside a cluster)
  size_t ws_split_bytes;
  uint32_t debug;
  int geglu;  // 1: W has 2N rows [a; gate] and out[:, j] = (x.W[j] + b[j]) * gelu(x.W[N+j] + b[N+j]); bias has 2N
  const void* residual;  // bf16 [M, N] added after the bias (row stride ldr), or null
  int64_t ldr;
};
// Launch plan for a problem: the N tile and the split-K factor (what `variant == 0` resolves to).
struct GemmPlan {
  int bn;
  int splits;
  int kb_per_split;
  size_t split_ws_bytes;  // bytes of split-K workspace the plan needs (0: split K reduces inside a cluster)
  bool pair;              // 256-row tiles on a two-CTA cluster (tcgen05 cta_group::2)
};
// Tile variants: BN (64 ... 256) for one CTA per tile, kGemmPairVariant + BN (128, 192, 256) for a CTA pair.
constexpr int kGemmPairVariant = 1000;
// Split K runs the splits of a tile as one cluster (the portable cluster size bounds it).
constexpr int kGemmMaxSplits = 8;
// Clusters of `size` one-CTA-per-SM GEMM CTAs that can be resident at once on the current device (0: unknown).
int gemm_cluster_slots(int size);
bool gemm_variant_known(int variant, bool geglu);
// auto_pair: whether the automatic choice (variant 0) may pick a pair tile.
GemmPlan gemm_plan(int64_t M, int64_t N, int64_t K, int sms, int variant, bool geglu = false, bool auto_pair = true);
inline int gemm_plan_variant(const GemmPlan& p) { return p.pair ? kGemmPairVariant + p.bn : p.bn; }
// Weight rows per TMA box: BN, or BN/2 for the GEGLU form (a and gate halves) and for one CTA of a pair.
inline int gemm_plan_box_rows(const GemmPlan& p, bool geglu) { return (p.pair || geglu) ? p.bn / 2 : p.bn; }
int gemm_encode_b_map(const void* w, int64_t ldw, int64_t N, int64_t K, int box_rows, CUtensorMap* out);
// Bytes of workspace the GEMM entry points use for a problem (split-K counters + partials, repack buffers).
size_t gemm_workspace_bytes(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                            int variant, int sms, int geglu = 0);
// The GEMM entry point's body with a caller-given workspace (argument checks, repacking, split-K, launch).
int gemm_with_workspace(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                        const CUtensorMap* w_map, const void* bias, int bias_dtype, void* out, int64_t ldo,
                        int out_dtype, void* workspace, size_t workspace_bytes, int variant, void* stream,
                        int geglu = 0, const void* residual = nullptr, int64_t ldr = 0);
int gemm_launch(const GemmProblem& p, cudaStream_t stream);

// 3x3 convolution, stride 1, zero padding 1, as an implicit GEMM on the GEMM kernel (its convolution form).
struct ConvProblem {
  const void* x;  // NHWC bf16 [n][h][w][cin], dense
  int64_t n, h, w, cin;
  const void* wt;  // [cout][3][3][cin] bf16, dense
  int64_t cout;
  const void* bias;           // [cout], or one row per image when bias_img_stride > 0; may be null
  int bias_f32;
  int64_t bias_img_stride;    // elements between the bias rows of consecutive images (0: one row for all)
  const void* residual;       // bf16 [n*h*w, cout] added to the result (row stride ldr), or null
  int64_t ldr;
  void* out;                  // [n*h*w, cout] (NHWC), row stride ldo
  int64_t ldo;
  int out_f32;
  int variant;                // 0 or a forced output-channel tile
  uint32_t debug;
  void* ws_split;             // caller workspace (split K needs none: it reduces inside a cluster)
  size_t ws_split_bytes;
};
int conv3x3_launch(const ConvProblem& p, cudaStream_t stream);
// GroupNorm (+ SiLU) over NHWC bf16: x, out [n][hw][c]; gamma, beta f32 [c]; stats: group_norm_scratch_bytes()
// of scratch whose counters (the last n*groups words) are zero on first use and left zero.
size_t group_norm_scratch_bytes(int64_t n, int64_t groups);
// Debug bits 1 and 2 force the two-launch or the cooperative GroupNorm form (the latter where it applies), so tests
// run both forms on the same shapes.
constexpr uint32_t kDebugGnTwoLaunch = 2u, kDebugGnCooperative = 4u;
int group_norm_launch(const void* x, int64_t n, int64_t hw, int64_t c, int64_t groups, const float* gamma,
                      const float* beta, float eps, int apply_silu, void* out, float* stats, cudaStream_t stream,
                      uint32_t debug);
// LayerNorm over the last dimension of bf16 rows: x [rows][ldx], out [rows][ldo] (cols valid); gamma, beta [cols]
// in f32 (param_f32) or bf16.
int layer_norm_launch(const void* x, int64_t rows, int64_t cols, int64_t ldx, const void* gamma, const void* beta,
                      int param_f32, float eps, void* out, int64_t ldo, cudaStream_t stream);
// NHWC data movement (two-byte elements): nearest 2x upsampling of a dense [n][h][w][c] tensor into
// [n][2h][2w][c], and the channel concatenation out[p] = a[p] ++ b[p] over row-strided pixels.
int upsample_nearest2x_launch(const void* x, int64_t n, int64_t h, int64_t w, int64_t c, void* out,
                              cudaStream_t stream);
int concat_channels_launch(const void* a, int64_t lda, int64_t ca, const void* b, int64_t ldb, int64_t cb,
                           int64_t pixels, void* out, int64_t ldo, cudaStream_t stream);
// Split-K workspace bytes the convolution's fastest plan uses (0: none).
size_t conv3x3_workspace_bytes(int64_t n, int64_t h, int64_t w, int64_t cin, int64_t cout, int variant, int sms);
// bf16 copy of a row-strided matrix into a dense [rows, cols_pad] buffer, zero-filling the pad columns.
int repack_rows_bf16(const void* src, int64_t ld_src, int64_t rows, int64_t cols, void* dst, int64_t cols_pad,
                     cudaStream_t stream);

// ---- attention ---------------------------------------------------------------------------------------------------
struct AttnProblem {
  const void* q;  // bf16, element (b, s, h, e) at b*sb + s*ss + h*sh + e
  const void* k;
  const void* v;
  void* o;
  int64_t q_sb, q_ss, q_sh;
  int64_t k_sb, k_ss, k_sh;
  int64_t v_sb, v_ss, v_sh;
  int64_t o_sb, o_ss, o_sh;
  int64_t B, H, Sq, Skv, D;
  float scale;
  int out_f32;
  int variant;
  uint32_t debug;
};
int attention_launch(const AttnProblem& p, cudaStream_t stream);

}  // namespace npub200
