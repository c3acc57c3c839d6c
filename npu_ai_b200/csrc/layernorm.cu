// layernorm.cu - LayerNorm over the last dimension of bf16 activations: the norm1/norm2/norm3 in front of the
// attention and feed-forward projections of every SD1.5 transformer block. The reference leaves LayerNorm to the
// host (docs/02-results.md:411-413, "convolutions, GroupNorm/LayerNorm, ..."); on B200 torch's kernel for these
// shapes runs far from the HBM roofline (tokens x 320..1280 channels, one read and one write of the tensor).
//
// A power-of-two group of lanes per row (several rows per warp for narrow rows), the row held in registers as
// 16-byte chunks (8 bf16), so the tensor is read once: mean and variance (two passes over the registers, exact) by
// fixed-order shuffles within the group, then y = (x - mean) * rstd * gamma + beta in f32, rounded to bf16.
// Deterministic.
#include <algorithm>

#include "internal.h"

namespace npub200 {

namespace {

constexpr int kLnThreads = 256;  // 8 rows per block


__device__ __forceinline__ void unpack8(const uint4& raw, float (&f)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[2 * e] = __uint_as_float(w[e] << 16);
    f[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
  }
}

// Affine parameters of 8 consecutive columns from chunk c (bf16 or f32 storage).
__device__ __forceinline__ void load_param8(const void* p, int param_f32, int c, float (&f)[8]) {
  if (param_f32) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p) + 2 * c);
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 2 * c + 1);
    f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
  } else {
    unpack8(__ldg(reinterpret_cast<const uint4*>(p) + c), f);
  }
}

// G lanes per row (a power of two, rows of a warp side by side), CPL 16-byte chunks per lane: a 320-channel row is
// 40 chunks on 8 lanes (4 rows per warp), 1280 channels 160 chunks on 32 lanes, so no lane idles in the chunk loop
// and the per-row reductions are log2(G) shuffle steps.
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int G, int CPL>
__global__ void __launch_bounds__(kLnThreads)
    layer_norm_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, __nv_bfloat16* __restrict__ y,
                      long long ldy, long long rows, int cols, const void* __restrict__ gamma,
                      const void* __restrict__ beta, int param_f32, float eps) {
  pdl_wait();  // x is the previous kernel's output
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int q = lane % G;
  const long long row = ((long long)blockIdx.x * (kLnThreads / 32) + (threadIdx.x >> 5)) * (32 / G) + lane / G;
  const bool valid = row < rows;  // every lane stays for the shuffles
  const int chunks = cols / 8;
  const uint4* src = reinterpret_cast<const uint4*>(x + (valid ? row : 0) * ldx);
  uint4 raw[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = q + G * i;
    raw[i] = (valid && c < chunks) ? src[c] : make_uint4(0u, 0u, 0u, 0u);
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    float f[8];
    unpack8(raw[i], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) s += f[e];  // chunks past the row are zeros
  }
  const float mean = group_sum<G>(s) / float(cols);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    if (q + G * i < chunks) {
      float f[8];
      unpack8(raw[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = f[e] - mean;
        ss = fmaf(d, d, ss);
      }
    }
  }
  const float rstd = rsqrtf(group_sum<G>(ss) / float(cols) + eps);
  if (!valid) return;
  uint4* dst = reinterpret_cast<uint4*>(y + row * ldy);
#pragma unroll
  for (int i = 0; i < CPL; ++i) {
    const int c = q + G * i;
    if (c < chunks) {
      float f[8], g[8], b[8];
      unpack8(raw[i], f);
      load_param8(gamma, param_f32, c, g);
      load_param8(beta, param_f32, c, b);
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o[e] = pack_bf16x2(fmaf((f[2 * e] - mean) * rstd, g[2 * e], b[2 * e]),
                           fmaf((f[2 * e + 1] - mean) * rstd, g[2 * e + 1], b[2 * e + 1]));
      dst[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

}  // namespace

int layer_norm_launch(const void* x, int64_t rows, int64_t cols, int64_t ldx, const void* gamma, const void* beta,
                      int param_f32, float eps, void* out, int64_t ldo, cudaStream_t stream) {
  if (x == nullptr || out == nullptr || gamma == nullptr || beta == nullptr)
    return fail(kErrInvalid, "layer_norm: null pointer");
  if (rows <= 0 || cols <= 0 || ldx < cols || ldo < cols)
    return fail(kErrInvalid, "layer_norm: bad sizes (rows=%lld cols=%lld ldx=%lld ldo=%lld)", (long long)rows,
                (long long)cols, (long long)ldx, (long long)ldo);
  const uintptr_t align = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                          reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta);
  if (cols % 8 != 0 || ldx % 8 != 0 || ldo % 8 != 0 || (align & 15) != 0)
    return fail(kErrUnsupported, "layer_norm needs cols and row strides in multiples of 8 and 16-byte aligned tensors");
  if (cols > 2048) return fail(kErrUnsupported, "layer_norm: at most 2048 columns (got %lld)", (long long)cols);
  // Lanes per row: the smallest power of two (4 ... 32) that leaves at most 8 chunks per lane.
  const int64_t chunks = cols / 8;
  int g = 4;
  while (g < 32 && (chunks + g - 1) / g > 8) g *= 2;
  const int cpl = int((chunks + g - 1) / g);
  const int64_t rows_per_block = (kLnThreads / 32) * (32 / g);
  const int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  if (blocks > INT32_MAX) return fail(kErrInvalid, "layer_norm: too many rows");
  auto run = [&](auto kern) {
    return check_cuda(launch_pdl(kern, dim3(unsigned(blocks)), dim3(kLnThreads), 0, stream,
                                 static_cast<const __nv_bfloat16*>(x), (long long)ldx,
                                 static_cast<__nv_bfloat16*>(out), (long long)ldo, (long long)rows, int(cols), gamma,
                                 beta, param_f32, eps),
                      "layer_norm launch");
  };
#define NPUB200_LN_CASES(G)                          \
  case 1: return run(layer_norm_kernel<G, 1>);       \
  case 2: return run(layer_norm_kernel<G, 2>);       \
  case 3: return run(layer_norm_kernel<G, 3>);       \
  case 4: return run(layer_norm_kernel<G, 4>);       \
  case 5: return run(layer_norm_kernel<G, 5>);       \
  case 6: return run(layer_norm_kernel<G, 6>);       \
  case 7: return run(layer_norm_kernel<G, 7>);       \
  default: return run(layer_norm_kernel<G, 8>);
  switch (g) {
    case 4:
      switch (cpl) { NPUB200_LN_CASES(4) }
    case 8:
      switch (cpl) { NPUB200_LN_CASES(8) }
    case 16:
      switch (cpl) { NPUB200_LN_CASES(16) }
    default:
      switch (cpl) { NPUB200_LN_CASES(32) }
  }
#undef NPUB200_LN_CASES
}

}  // namespace npub200
