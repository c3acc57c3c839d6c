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
  if ((cg & 1) == 0) {
    // channel pairs (c and cg even, so the group's first channel is even)
    const int pairs = cg / 2;
    for (int i = p_begin * pairs + threadIdx.x; i < p_end * pairs; i += kStatsThreads) {
      const int p = i / pairs;
      const int k = i - p * pairs;
      const float2 v = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(base + (long long)p * c)[k]);
      s += v.x + v.y;
      ss = fmaf(v.x, v.x, fmaf(v.y, v.y, ss));
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

__device__ __forceinline__ float silu(float v) { return v / (1.0f + __expf(-v)); }

// x and y may be the same tensor (each element is read and written by one thread), so neither is __restrict__.
__global__ void gn_apply_kernel(const __nv_bfloat16* x, __nv_bfloat16* y, long long pixels,
                                int hw, int c, int cg, int groups, const float2* __restrict__ stats,
                                const float* __restrict__ gamma, const float* __restrict__ beta, int apply_silu) {
  const int chunks = c / 8;
  const long long total = pixels * chunks;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long p = i / chunks;
    const int c0 = int(i - p * chunks) * 8;
    const int img = int(p / hw);
    const uint4 raw = *reinterpret_cast<const uint4*>(x + p * c + c0);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float v[2] = {__uint_as_float(w[e] << 16), __uint_as_float(w[e] & 0xFFFF0000u)};
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int ch = c0 + 2 * e + t;
        const float2 st = stats[img * groups + ch / cg];
        float r = (v[t] - st.x) * st.y * gamma[ch] + beta[ch];
        if (apply_silu) r = silu(r);
        v[t] = r;
      }
      o[e] = pack_bf16x2(v[0], v[1]);
    }
    *reinterpret_cast<uint4*>(y + p * c + c0) = make_uint4(o[0], o[1], o[2], o[3]);
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
  const long long total = n * hw * (c / 8);
  const int threads = 256;
  const int grid = int(std::min<long long>((total + threads - 1) / threads, (long long)dev->sms * 16));
  gn_apply_kernel<<<grid, threads, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out),
                                                n * hw, int(hw), int(c), int(c / groups), int(groups),
                                                reinterpret_cast<const float2*>(st), gamma, beta, apply_silu);
  return check_cuda(cudaGetLastError(), "group_norm apply launch");
}

}  // namespace npub200
