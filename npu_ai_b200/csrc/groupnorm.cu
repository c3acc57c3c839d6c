// groupnorm.cu - GroupNorm (+ SiLU) over NHWC bf16 activations, the normalisation in front of every convolution of
// an SD1.5 UNet ResBlock. The reference leaves GroupNorm to the host (docs/02-results.md:411-413, "convolutions,
// GroupNorm/LayerNorm, ..."); on B200 it matters because the convolutions run channels-last: torch's GroupNorm
// converts such tensors to NCHW and back, which costs more than the normalisation itself.
//
// Two HBM-bound passes, deterministic (fixed-order reductions):
//   gn_stats_kernel  blocks over (group, image, pixel slice): partial sums and sums of squares of the group's values
//                    in f32; the last slice block of each (image, group) combines them in slice order into
//                    (mean, rstd).
//   gn_apply_kernel  8 channels (16 bytes) per thread: y = (x - mean) * rstd * gamma + beta, optionally SiLU,
//                    bf16 out (same NHWC layout).
#include <algorithm>
#include <cstdio>

#include "internal.h"

namespace npub200 {

constexpr int kGnMaxSlices = 32;       // pixel slices per (image, group) in the statistics pass
constexpr int64_t kGnCounters = 65536;  // ticket counters at the start of the scratch: images x groups <= this

namespace {

constexpr int kStatsThreads = 256;

// Statistics of group g of image img over pixel slice blockIdx.z: partial (sum, sum of squares) in f32. The last
// slice block of the (image, group) to finish (ticket from `counters`, which it resets to zero) adds the partials in
// slice order and writes (mean, rstd), so the result does not depend on which block finishes last.
__global__ void __launch_bounds__(kStatsThreads)
    gn_stats_kernel(const __nv_bfloat16* __restrict__ x, int hw, int c, int cg, float eps, float2* __restrict__ stats,
                    float2* __restrict__ partials, unsigned int* __restrict__ counters) {
  const int img = blockIdx.y;
  const int g = blockIdx.x;
  const int slices = gridDim.z;
  const int slice = blockIdx.z;
  const int p_begin = int((long long)hw * slice / slices);
  const int p_end = int((long long)hw * (slice + 1) / slices);
  const __nv_bfloat16* base = x + (long long)img * hw * c + (long long)g * cg;
  float s = 0.f, ss = 0.f;
  if ((cg & 1) == 0 && cg / 2 <= kStatsThreads) {
    // Each thread keeps one channel pair of the group and strides over pixels (no per-element index division);
    // the threads of a pixel row read its contiguous cg-channel segment.
    const int pairs = cg / 2;
    const int rows = kStatsThreads / pairs;  // pixel rows per pass
    const int k = threadIdx.x % pairs;
    const int r = threadIdx.x / pairs;
    if (r < rows) {
      const __nv_bfloat162* col = reinterpret_cast<const __nv_bfloat162*>(base) + k;
      const long long step = (long long)rows * c / 2;  // bf16 pairs between passes
      const __nv_bfloat162* ptr = col + (long long)(p_begin + r) * c / 2;
#pragma unroll 4
      for (int p = p_begin + r; p < p_end; p += rows, ptr += step) {  // unrolled: several loads in flight
        const float2 v = __bfloat1622float2(*ptr);
        s += v.x + v.y;
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, ss));
      }
    }
  } else {
    for (int i = p_begin * cg + threadIdx.x; i < p_end * cg; i += kStatsThreads) {
      const int p = i / cg;
      const float v = __bfloat162float(base[(long long)p * c + (i - p * cg)]);
      s += v;
      ss = fmaf(v, v, ss);
    }
  }
  // Fixed-order reduction: warp shuffles, then the warp totals in order.
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  __shared__ float ws[kStatsThreads / 32][2];
  __shared__ int last;
  if ((threadIdx.x & 31) == 0) {
    ws[threadIdx.x >> 5][0] = s;
    ws[threadIdx.x >> 5][1] = ss;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float ts = 0.f, tss = 0.f;
    for (int w = 0; w < kStatsThreads / 32; ++w) {
      ts += ws[w][0];
      tss += ws[w][1];
    }
    const int slot = img * gridDim.x + g;
    __stcg(&partials[(long long)slot * slices + slice], make_float2(ts, tss));
    __threadfence();
    const unsigned int ticket = atomicAdd(&counters[slot], 1u);
    last = ticket == unsigned(slices - 1);
    if (last) {
      __threadfence();
      float as = 0.f, ass = 0.f;
      for (int i = 0; i < slices; ++i) {
        const float2 pv = __ldcg(&partials[(long long)slot * slices + i]);
        as += pv.x;
        ass += pv.y;
      }
      const float cnt = float(hw) * float(cg);
      const float mean = as / cnt;
      const float var = fmaxf(ass / cnt - mean * mean, 0.f);
      stats[slot] = make_float2(mean, rsqrtf(var + eps));
      counters[slot] = 0u;  // left zero for the next call
    }
  }
}


constexpr int kApplyThreads = 256;

// y = act(x * A[ch] + B[ch]) with A = rstd * gamma, B = beta - mean * A for this image: the block builds the table
// for its image's channels in shared memory, then streams its pixels 8 channels (16 bytes) per thread.
// x and y may be the same tensor (each element is read and written by one thread), so neither is __restrict__.
__global__ void __launch_bounds__(kApplyThreads)
    gn_apply_kernel(const __nv_bfloat16* x, __nv_bfloat16* y, int hw, int c, int cg, int groups, int block_pixels,
                    const float2* __restrict__ stats, const float* __restrict__ gamma,
                    const float* __restrict__ beta, int apply_silu) {
  extern __shared__ float2 ab[];  // [c]: (A, B)
  const int img = blockIdx.y;
  for (int ch = threadIdx.x; ch < c; ch += kApplyThreads) {
    const float2 st = stats[img * groups + ch / cg];
    const float a = st.y * gamma[ch];
    ab[ch] = make_float2(a, beta[ch] - st.x * a);
  }
  __syncthreads();
  const int chunks = c / 8;
  const int p0 = blockIdx.x * block_pixels;
  const int np = min(block_pixels, hw - p0);
  const long long base = ((long long)img * hw + p0) * c;
  for (int i = threadIdx.x; i < np * chunks; i += kApplyThreads) {
    const int p = i / chunks;  // one division per 8 values
    const int c0 = (i - p * chunks) * 8;
    const long long off = base + (long long)p * c + c0;
    const uint4 raw = *reinterpret_cast<const uint4*>(x + off);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 ab0 = ab[c0 + 2 * e], ab1 = ab[c0 + 2 * e + 1];
      float v0 = fmaf(__uint_as_float(w[e] << 16), ab0.x, ab0.y);
      float v1 = fmaf(__uint_as_float(w[e] & 0xFFFF0000u), ab1.x, ab1.y);
      if (apply_silu) {
        v0 = __fdividef(v0, 1.0f + __expf(-v0));
        v1 = __fdividef(v1, 1.0f + __expf(-v1));
      }
      o[e] = pack_bf16x2(v0, v1);
    }
    *reinterpret_cast<uint4*>(y + off) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace

size_t group_norm_scratch_bytes(int64_t n, int64_t groups) {
  // Fixed region of zero-initialised ticket counters first (the same place whatever the sizes, so a scratch reused
  // across shapes always finds them zero), then (mean, rstd) per (image, group), then the slice partials.
  return size_t(kGnCounters) * 4 + size_t(n * groups) * (8 + 8 * kGnMaxSlices);
}

int group_norm_launch(const void* x, int64_t n, int64_t hw, int64_t c, int64_t groups, const float* gamma,
                      const float* beta, float eps, int apply_silu, void* out, float* stats, cudaStream_t stream) {
  const DeviceInfo* dev = nullptr;
  if (int rc = current_device_info(&dev)) return rc;
  if (x == nullptr || out == nullptr || gamma == nullptr || beta == nullptr || stats == nullptr)
    return fail(kErrInvalid, "group_norm: null pointer");
  if (n <= 0 || hw <= 0 || c <= 0 || groups <= 0 || c % groups != 0)
    return fail(kErrInvalid, "group_norm: bad sizes (n=%lld hw=%lld c=%lld groups=%lld)", (long long)n,
                (long long)hw, (long long)c, (long long)groups);
  if (c % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return fail(kErrUnsupported, "group_norm needs c %% 8 == 0 and 16-byte aligned tensors");
  if (n > 65535 || groups > 65535 || n * groups > kGnCounters || hw > INT32_MAX / 64 ||
      hw * (c / groups) > INT32_MAX)
    return fail(kErrInvalid, "group_norm: too large (images x groups <= %lld)", (long long)kGnCounters);
  // Pixel slices per (image, group): enough blocks to fill the GPU, each with at least a few thousand values.
  const int64_t cg = c / groups;
  int64_t slices = std::max<int64_t>(1, (int64_t(dev->sms) * 4 + n * groups - 1) / (n * groups));
  slices = std::min<int64_t>({slices, int64_t(kGnMaxSlices), std::max<int64_t>(1, hw * cg / 4096)});
  unsigned int* counters = reinterpret_cast<unsigned int*>(stats);         // [kGnCounters]
  float* st = stats + kGnCounters;                                         // [n * groups] float2
  float* partials = st + 2 * n * groups;                                   // [n * groups * slices] float2
  gn_stats_kernel<<<dim3(unsigned(groups), unsigned(n), unsigned(slices)), kStatsThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), int(hw), int(c), int(cg), eps, reinterpret_cast<float2*>(st),
      reinterpret_cast<float2*>(partials), counters);
  if (int rc = check_cuda(cudaGetLastError(), "group_norm stats launch")) return rc;
  if (c > 6144) return fail(kErrUnsupported, "group_norm: at most 6144 channels");  // 48 KB scale/shift table
  // Pixels per apply block (within one image): about four blocks per SM over the whole tensor, at least one pixel.
  const int64_t vecs = n * hw * (c / 8);
  const int64_t per_block = (vecs + int64_t(dev->sms) * 4 - 1) / (int64_t(dev->sms) * 4);
  const int64_t block_pixels = std::max<int64_t>(1, std::min<int64_t>(hw, (per_block + c / 8 - 1) / (c / 8)));
  const dim3 agrid(unsigned((hw + block_pixels - 1) / block_pixels), unsigned(n));
  gn_apply_kernel<<<agrid, kApplyThreads, size_t(c) * sizeof(float2), stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), int(hw), int(c), int(c / groups),
      int(groups), int(block_pixels), reinterpret_cast<const float2*>(st), gamma, beta, apply_silu);
  return check_cuda(cudaGetLastError(), "group_norm apply launch");
}

}  // namespace npub200
