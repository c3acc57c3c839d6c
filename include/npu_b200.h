/*
 * npu_b200.h - C ABI of libnpub200, the B200 (sm_100a) backend of the npu-ai offload hot path.
 *
 * The reference (Tobynau/npu-ai) drives an AMD XDNA1 NPU from Python: `NpuGemm` in npu/xdna1_gemm.py builds
 * buffers and calls `NpuProgram.submit_gemm` / `submit_attn` (npu/xdna1_program.py:451-473), which hand three
 * buffer objects and 13 int32 parameters to one XRT kernel command (xdna1_program.py:441-446). This header is
 * the B200 equivalent of that dispatch boundary: plain device pointers, sizes and element strides, a CUDA stream
 * passed as `void*` (a cudaStream_t; NULL = the legacy default stream), no torch types. Everything launches
 * asynchronously on the given stream; nothing here synchronises except npub200_status_read.
 *
 * Conventions
 *   - bf16 tensors are `uint16_t` bit patterns (__nv_bfloat16 / torch.bfloat16); dtype codes below.
 *   - Strides are in elements. The innermost dimension is always contiguous.
 *   - Return value: 0 on success, a negative NPUB200_E* code on failure; npub200_last_error() then holds a
 *     message for the calling thread. There is no CPU fallback: a request no kernel variant takes fails.
 *   - Kernels never trap. A bounded wait that expires inside a kernel sets bits in the device's status word;
 *     npub200_status_read() reports them (the reference's `NpuProgram.wait` raising RuntimeError,
 *     xdna1_program.py:475-479).
 */
#ifndef NPU_B200_H_
#define NPU_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NPUB200_OK 0
#define NPUB200_EINVAL (-1)      /* invalid shape, stride, alignment or dtype */
#define NPUB200_ECUDA (-2)       /* a CUDA runtime/driver call failed */
#define NPUB200_EUNSUPPORTED (-3) /* legal request without a kernel variant in this build */
#define NPUB200_EDEVICE (-4)     /* a kernel reported a failure (see npub200_status_read) */

#define NPUB200_DTYPE_BF16 0
#define NPUB200_DTYPE_F32 1

/* Library version (major * 10000 + minor * 100 + patch). */
int npub200_version(void);

/* Message of the last failing call made by this thread ("" if none). */
const char* npub200_last_error(void);

/* Number of SMs of the current device (initialises the library's per-device state). */
int npub200_device_sms(int* sms_out);

/* ----------------------------------------------------------------------------------------------------------
 * Resident weights. Replaces NpuGemm.upload_weight / NpuWeight (npu/xdna1_gemm.py:311-321, :89-99): the weight
 * stays in HBM in nn.Linear's own [N, K] layout (no transpose, no padding copy) and the handle caches the TMA
 * descriptors built for it. `w` must stay allocated until npub200_weight_release. K % 8 == 0 and ldw % 8 == 0
 * with a 16-byte aligned base (TMA addressing); callers pad other weights once at upload.
 * ---------------------------------------------------------------------------------------------------------- */
int npub200_weight_register(const void* w, int64_t n, int64_t k, int64_t ldw, int64_t* handle_out);
int npub200_weight_release(int64_t handle);

/* ----------------------------------------------------------------------------------------------------------
 * GEMM: out[M, N] = x[M, K] . W[N, K]^T (+ bias[N]); bf16 operands, f32 accumulation, bias added in f32,
 * out f32 or bf16. Replaces NpuGemm.matmul_t (npu/xdna1_gemm.py:349-422) and the GEMM mode of the unified NPU
 * program (npu/xdna1_program.py:451-454, npu/kernels/xdna1_attn.cc:480-574). Any M, N, K >= 1: ragged tails are
 * handled in the kernel. x rows need a 16-byte aligned base and ldx % 8 == 0 (TMA); otherwise x is first
 * repacked into `workspace`. Shapes with few output tiles and a long K split K across the CTAs of a cluster,
 * which reduce their partials in shared memory: no workspace. npub200_gemm_workspace_size() gives the bytes a call
 * needs (repacked operands, else 0); a workspace reused on one stream is fine, concurrent calls must not share one,
 * and NULL is accepted when the operands need no repacking. `variant` 0 picks the tile automatically, or forces an
 * N tile in {64, 96, 128, 160, 192, 256}, or 1000 + {128, 192, 256} for 256-row tiles on a two-CTA cluster.
 * ---------------------------------------------------------------------------------------------------------- */
int npub200_gemm_workspace_size(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw,
                                int64_t n, int variant, size_t* bytes_out);
int npub200_gemm(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                 const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype, void* workspace,
                 size_t workspace_bytes, int variant, void* stream);
/* The launch plan the library picks for a GEMM shape on the current device: tile variant (N tile, or 1000 + N tile
 * for 256-row tiles on a two-CTA cluster) and split-K factor (the B200 counterpart of NpuGemm.dispatch_shapes,
 * npu/xdna1_gemm.py:295-297, which lists the padded chunks). */
int npub200_gemm_plan(int64_t m, int64_t n, int64_t k, int variant, int* tile_n_out, int* splits_out);
/* Same with a registered weight (the resident-weight path the runner uses). */
int npub200_gemm_w(const void* x, int64_t ldx, int64_t m, int64_t k, int64_t weight, const void* bias,
                   int bias_dtype, void* out, int64_t ldo, int out_dtype, void* workspace, size_t workspace_bytes,
                   int variant, void* stream);
/* GEMM with a residual added in the epilogue: out = x . W^T + bias + residual, residual bf16 [M, N] with row
 * stride ldr (may be `out` itself). The residual connections of a transformer block (x + to_out(attn),
 * x + ff(..)), which the reference's host code adds after its offloaded Linear (npu/xdna1_gemm.py:428-448 returns
 * the projection alone), land in the same kernel. Otherwise as npub200_gemm. */
int npub200_gemm_residual(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                          const void* bias, int bias_dtype, const void* residual, int64_t ldr, void* out, int64_t ldo,
                          int out_dtype, void* workspace, size_t workspace_bytes, int variant, void* stream);
/* GEGLU feed-forward projection in one kernel: W is [2n, K] (nn.Linear layout of SD1.5's GEGLU `proj`: the n
 * value rows, then the n gate rows), bias [2n] or NULL, and out[M, n] = (x.W[j] + b[j]) * gelu(x.W[n+j] + b[n+j])
 * with the exact (erf) GELU, f32 accumulation and gating, out f32 or bf16. The reference computes the projection
 * with NpuGemm.linear (npu/xdna1_gemm.py:428-448) and gates on the CPU in ComfyUI's GEGLU module (the "rest" of a
 * transformer block, docs/02-results.md:411-413); here the 2n-column projection never reaches memory. `variant`:
 * 0 or an accumulator tile in {64, 128, 192, 256} (half value, half gate columns). The workspace is used only for
 * operands TMA cannot address; npub200_gemm_workspace_size() with 2n columns gives a sufficient size. */
int npub200_gemm_geglu(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                       const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype, void* workspace,
                       size_t workspace_bytes, int variant, void* stream);

/* ----------------------------------------------------------------------------------------------------------
 * 3x3 convolution, stride 1, zero padding 1, as an implicit GEMM on the tensor cores: out[n, y, x, co] =
 * bias[co] + sum over (dy, dx, ci) of in[n, y+dy-1, x+dx-1, ci] * weight[co, dy, dx, ci] (+ residual). The
 * reference names im2col + GEMM convolutions (K = 2880-11520) as its next experiment (docs/03-next-steps.md:112-114)
 * and runs its convolutions on the CPU; here the im2col is a shifted TMA box per tap, never materialised.
 * x: NHWC bf16 [n][h][w][cin], dense; weight: [cout][3][3][cin] bf16, dense (a PyTorch [cout][cin][3][3] weight
 * permuted once); out: [n*h*w][cout] rows (NHWC) with row stride ldo, bf16 or f32. bias: [cout], or with
 * bias_img_stride > 0 one row per image (e.g. conv bias + a ResBlock's time embedding), f32 or bf16, or NULL.
 * residual: bf16 [n*h*w][cout] rows with stride ldr, added after the bias, or NULL. Needs cin % 64 == 0, a width
 * dividing 128, and a height that is a multiple of the rows a 128-pixel tile takes (128 / width, capped at the
 * height); other shapes are NPUB200_EUNSUPPORTED. `variant`: 0 or an output-channel tile in
 * {64, 96, 128, 160, 192, 256}. Allocates nothing.
 * ---------------------------------------------------------------------------------------------------------- */
int npub200_conv3x3(const void* x, int64_t n, int64_t h, int64_t w, int64_t cin, const void* weight, int64_t cout,
                    const void* bias, int bias_dtype, int64_t bias_img_stride, const void* residual, int64_t ldr,
                    void* out, int64_t ldo, int out_dtype, void* workspace, size_t workspace_bytes, int variant,
                    void* stream);
/* Workspace bytes npub200_conv3x3 needs: 0 (split K, for small images with many channels, reduces inside a
 * cluster's shared memory); NULL is accepted. Kept so callers size a workspace the same way as for the GEMM. */
int npub200_conv3x3_workspace_size(int64_t n, int64_t h, int64_t w, int64_t cin, int64_t cout, int variant,
                                   size_t* bytes_out);

/* GroupNorm over NHWC bf16 activations, optionally followed by SiLU (the normalisation in front of each
 * convolution of an SD1.5 ResBlock, which the reference leaves on the host, docs/02-results.md:411-413):
 * out[n][p][ch] = act((x - mean_g) * rstd_g * gamma[ch] + beta[ch]) with the mean and variance of group g over all
 * pixels and its c/groups channels, in f32. x, out: [n][hw][c] bf16 (NHWC, may alias), c % 8 == 0, 16-byte
 * aligned; gamma, beta: f32 [c]; stats: caller scratch of npub200_group_norm_scratch_size() bytes, ZERO before its
 * first use (it ends in ticket counters the kernels leave zero; one scratch per stream). Deterministic: the
 * statistics pass splits each (image, group) over pixel slices and combines them in slice order. Allocates
 * nothing. */
int npub200_group_norm(const void* x, int64_t n, int64_t hw, int64_t c, int64_t groups, const float* gamma,
                       const float* beta, float eps, int apply_silu, void* out, float* stats, void* stream);
int npub200_group_norm_scratch_size(int64_t n, int64_t groups, size_t* bytes_out);

/* LayerNorm over the last dimension of bf16 rows (norm1/norm2/norm3 of every SD1.5 transformer block, which the
 * reference leaves on the host, docs/02-results.md:411-413): out[r][j] = (x[r][j] - mean_r) * rstd_r * gamma[j] +
 * beta[j], mean and variance of row r over its cols values in f32, bf16 out. x: [rows][ldx], out: [rows][ldo];
 * cols, ldx, ldo multiples of 8, cols <= 2048, tensors 16-byte aligned; gamma, beta: [cols] of param_dtype (f32 or
 * bf16). Deterministic (fixed-order reductions); allocates nothing. */
int npub200_layer_norm(const void* x, int64_t rows, int64_t cols, int64_t ldx, const void* gamma, const void* beta,
                       int param_dtype, float eps, void* out, int64_t ldo, void* stream);

/* The two data-movement steps of an SD1.5 UNet decoder on NHWC (channels-last) activations, which the reference
 * leaves to the host with the rest of the UNet (docs/02-results.md:411-413). Elements are any two-byte type (bf16,
 * f16); channel counts and row strides are multiples of 8 elements, tensors 16-byte aligned (else
 * NPUB200_EUNSUPPORTED); out must not overlap a source (NPUB200_EINVAL). Allocate nothing.
 * npub200_upsample_nearest2x: nearest-neighbour 2x upsampling (torch's F.interpolate(scale_factor=2,
 *   mode="nearest") of an Upsample block): x dense [n][h][w][c] -> out dense [n][2h][2w][c],
 *   out[i][y][x] = x[i][y/2][x/2].
 * npub200_concat_channels: the skip concatenation in front of each output ResBlock (torch.cat along channels):
 *   out[p][0:ca] = a[p][:], out[p][ca:ca+cb] = b[p][:] for pixels p, rows of a/b/out lda/ldb/ldo elements apart. */
int npub200_upsample_nearest2x(const void* x, int64_t n, int64_t h, int64_t w, int64_t c, void* out, void* stream);
int npub200_concat_channels(const void* a, int64_t lda, int64_t ca, const void* b, int64_t ldb, int64_t cb,
                            int64_t pixels, void* out, int64_t ldo, void* stream);

/* ----------------------------------------------------------------------------------------------------------
 * GEMM without a workspace, for callers that cannot allocate device memory (a host whose device memory is owned
 * by its own pool manager and may not grow during a request, an FFI binding holding only the pointers it was
 * given, code that must not call cudaMalloc because it synchronises the device). No counterpart in the reference:
 * its NPU runner allocates its own pinned buffers. Same arguments and result as npub200_gemm minus the
 * workspace. The only scratch such a GEMM needs is a repacked copy of an operand TMA cannot address (K % 8 != 0,
 * a row stride that is not a multiple of 8 elements, an unaligned base); here it goes to one fixed device array of
 * NPUB200_NOALLOC_SCRATCH_BYTES per GPU, held from library load to process exit, and this call allocates nothing.
 * A shape whose repacked operands (plus a reserved 4 KiB) exceed the array is rejected with NPUB200_EINVAL;
 * npub200_gemm_workspace_size gives that need. The first call on a device resolves the array's address (make it
 * before any stream capture). All calls share the array and it keeps the last call's contents: calls that overlap
 * on the GPU (several streams, several host threads) race and must be serialised by the caller, e.g. on one stream.
 * ---------------------------------------------------------------------------------------------------------- */
#define NPUB200_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)
int npub200_gemm_noalloc(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw, int64_t n,
                         const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype, int variant,
                         void* stream);

/* ----------------------------------------------------------------------------------------------------------
 * Fused attention: out = softmax(Q K^T * scale) V for every (batch, head) pair in ONE launch; bf16 q/k/v,
 * f32 softmax statistics and accumulation, out bf16 or f32. Replaces NpuGemm.attention / _attention_fused
 * (npu/xdna1_gemm.py:499-752), NpuProgram.submit_attn (npu/xdna1_program.py:461-473) and the AIE flash kernel
 * (npu/kernels/xdna1_attn.cc:342-445). Element (b, s, h, e) of a tensor lives at b*sb + s*ss + h*sh + e, so both
 * the model's (B, S, H*D) layout and the head-major (B, H, S, D) layout (`skip_reshape`) are strided views.
 * Strides must be multiples of 8 elements and bases 16-byte aligned (TMA). Head dims 40, 80, 160 (any multiple
 * of 8 up to 256 is accepted); any Sq, Skv >= 1 (key tails are masked in the kernel, no padding).
 * ---------------------------------------------------------------------------------------------------------- */
int npub200_attention(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, const void* k, int64_t k_sb,
                      int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                      void* out, int64_t o_sb, int64_t o_ss, int64_t o_sh, int out_dtype, int64_t batch,
                      int64_t heads, int64_t sq, int64_t skv, int64_t head_dim, float scale, int variant,
                      void* stream);

/* ----------------------------------------------------------------------------------------------------------
 * Device status word (failure detection; the reference's RuntimeError from NpuProgram.wait,
 * npu/xdna1_program.py:475-479). Synchronises `stream`, returns the OR of the status bits kernels on the current
 * device reported since the last clear (0 = healthy), and clears them when `clear` is non-zero.
 * ---------------------------------------------------------------------------------------------------------- */
int npub200_status_read(void* stream, uint32_t* bits_out, int clear);

/* Test hooks (failure detection without a GPU fault): per-wait deadline in ns (0 restores the default), and
 * debug flags applied to the next launches (bit 0: the MMA role waits on a barrier nothing signals, so the
 * bounded wait expires and the kernel takes its abort path; bits 1, 2: npub200_group_norm uses its two-launch or
 * its one-launch cooperative form, the latter where it takes the shape, so tests cover both forms on the same
 * inputs). */
int npub200_set_wait_timeout_ns(uint64_t ns);
int npub200_set_debug_flags(uint32_t flags);

#ifdef __cplusplus
}
#endif

#endif /* NPU_B200_H_ */
