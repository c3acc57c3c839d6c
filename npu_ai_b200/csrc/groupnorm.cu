// groupnorm.cu - GroupNorm (+ SiLU) over NHWC bf16 activations, the normalisation in front of every convolution of
// an SD1.5 UNet ResBlock. The reference leaves GroupNorm to the host (docs/02-results.md:411-413, "convolutions,
// GroupNorm/LayerNorm, ..."); on B200 it matters because the convolutions run channels-last: torch's GroupNorm
// converts such tensors to NCHW and back, which costs more than the normalisation itself.
//
// One launch normally (gn_fused_kernel, a cooperative grid: every block resident), two for small tensors and as a
// fallback; both HBM-bound and deterministic (fixed-order reductions):
//   gn_fused_kernel  blocks over (pixel slice, image) read their pixels as whole 16-byte channel chunks, sum per
//                    channel in f32, fold channels into groups and publish per-slice partials; a grid barrier;
//                    then each block combines its image's partials in slice order into (mean, rstd) and
//                    normalises its slice again (from L2).
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
constexpr int kGnFusedMaxSlices = 64;  // pixel slices per image in the one-launch form
constexpr int64_t kGnCounters = 65536;  // ticket counters at the start of the scratch: images x groups <= this
constexpr int64_t kGnBarrier = kGnCounters - 2;  // the one-launch form's grid barrier: two counters at the end

namespace {

constexpr int kStatsThreads = 256;

// Statistics of group g of image img over pixel slice blockIdx.z: partial (sum, sum of squares) in f32. The last
// slice block of the (image, group) to finish (ticket from `counters`, which it resets to zero) adds the partials in
// slice order and writes (mean, rstd), so the result does not depend on which block finishes last.
__global__ void __launch_bounds__(kStatsThreads)
    gn_stats_kernel(const __nv_bfloat16* __restrict__ x, int hw, int c, int cg, float eps, float2* __restrict__ stats,
                    float2* __restrict__ partials, unsigned int* __restrict__ counters) {
  pdl_wait();  // x is the previous kernel's output
  pdl_launch_dependents();
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
  pdl_wait();  // the statistics kernel's results
  pdl_launch_dependents();
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

constexpr int kFusedThreads = 512;

__device__ __forceinline__ void unpack_bf16x8(const uint4& raw, float (&f)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    f[2 * e] = __uint_as_float(w[e] << 16);
    f[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
  }
}

// The one-launch GroupNorm (+ SiLU). Launched cooperatively (all blocks resident), grid (slices, images). Each
// thread owns one 16-byte channel chunk of a pixel row and strides over the slice's pixels; per-channel sums go
// through shared memory in fixed order, then per group. After the grid barrier (a bounded spin on two counters:
// arrivals, then departures; the last block to depart resets both), each block sums its image's slice partials in
// slice order. x and y may be the same tensor: phase 2 reads and writes each element in one thread, and no block
// writes before every block has finished reading in phase 1.
__global__ void __launch_bounds__(kFusedThreads)
    gn_fused_kernel(const __nv_bfloat16* x, __nv_bfloat16* y, int hw, int c, int cg, int groups, float eps,
                    const float* __restrict__ gamma, const float* __restrict__ beta, int apply_silu,
                    float2* partials, unsigned int* bar, unsigned int nblocks, uint32_t* status,
                    unsigned long long timeout_ns) {
  extern __shared__ float fs[];
  __shared__ int barrier_ok;
  const int img = blockIdx.y;
  const int slice = blockIdx.x;
  const int slices = gridDim.x;
  const int chunks = c / 8;
  const int rows = kFusedThreads / chunks;  // pixel rows per pass (c <= 4096)
  const int k = threadIdx.x % chunks;
  const int r = threadIdx.x / chunks;
  const int p0 = int((long long)hw * slice / slices);
  const int p1 = int((long long)hw * (slice + 1) / slices);
  const __nv_bfloat16* xi = x + (long long)img * hw * c + 8 * k;
  float* red_s = fs;                   // [rows][c]
  float* red_ss = fs + rows * c;       // [rows][c]
  float* ch_s = red_ss + rows * c;     // [c]
  float* ch_ss = ch_s + c;             // [c]
  float2* gst = reinterpret_cast<float2*>(ch_ss + c);  // [groups] (mean, rstd)
  if (r < rows) {
    float s[8], ss[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) s[e] = ss[e] = 0.f;
#pragma unroll 4
    for (int p = p0 + r; p < p1; p += rows) {
      float f[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(xi + (long long)p * c), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s[e] += f[e];
        ss[e] = fmaf(f[e], f[e], ss[e]);
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      red_s[r * c + 8 * k + e] = s[e];
      red_ss[r * c + 8 * k + e] = ss[e];
    }
  }
  __syncthreads();
  for (int ch = threadIdx.x; ch < c; ch += kFusedThreads) {
    float a = 0.f, b = 0.f;
    for (int rr = 0; rr < rows; ++rr) {
      a += red_s[rr * c + ch];
      b += red_ss[rr * c + ch];
    }
    ch_s[ch] = a;
    ch_ss[ch] = b;
  }
  __syncthreads();
  for (int g = threadIdx.x; g < groups; g += kFusedThreads) {
    float a = 0.f, b = 0.f;
    for (int j = 0; j < cg; ++j) {
      a += ch_s[g * cg + j];
      b += ch_ss[g * cg + j];
    }
    __stcg(&partials[((long long)img * slices + slice) * groups + g], make_float2(a, b));
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    atomicAdd(&bar[0], 1u);
    const unsigned long long t0 = globaltimer_ns();
    while (atomicAdd(&bar[0], 0u) < nblocks) {
      __nanosleep(128);
      if (globaltimer_ns() - t0 > timeout_ns) {
        atomicOr(status, kStatusTimeoutEpilogue);
        ok = 0;
        break;
      }
    }
    __threadfence();
    if (atomicAdd(&bar[1], 1u) == nblocks - 1) {  // every block has left the spin: reset for the next launch
      atomicExch(&bar[0], 0u);
      atomicExch(&bar[1], 0u);
    }
    barrier_ok = ok;
  }
  __syncthreads();
  if (!barrier_ok) return;
  // Group statistics of this image: 16 lanes per group, lane q summing slices q, q + 16, ... (their loads in
  // flight together), then a fixed 16-lane shuffle tree: one L2 round trip per 16 slices instead of per slice.
  const float cnt = float(hw) * float(cg);
  for (int g0 = 0; g0 < groups; g0 += kFusedThreads / 16) {
    const int g = g0 + int(threadIdx.x) / 16;
    const int q = int(threadIdx.x) % 16;
    float a = 0.f, b = 0.f;
    if (g < groups) {
      for (int sl = q; sl < slices; sl += 16) {
        const float2 pv = __ldcg(&partials[((long long)img * slices + sl) * groups + g]);
        a += pv.x;
        b += pv.y;
      }
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      a += __shfl_xor_sync(0xffffffffu, a, o);
      b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    if (g < groups && q == 0) {
      const float mean = a / cnt;
      const float var = fmaxf(b / cnt - mean * mean, 0.f);
      gst[g] = make_float2(mean, rsqrtf(var + eps));
    }
  }
  __syncthreads();
  float2* ab = reinterpret_cast<float2*>(fs);  // [c] (scale, shift), over the spent per-row sums
  for (int ch = threadIdx.x; ch < c; ch += kFusedThreads) {
    const float2 st = gst[ch / cg];
    const float a = st.y * gamma[ch];
    ab[ch] = make_float2(a, beta[ch] - st.x * a);
  }
  __syncthreads();
  if (r < rows) {
    __nv_bfloat16* yi = y + (long long)img * hw * c + 8 * k;
    float2 t[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) t[e] = ab[8 * k + e];
#pragma unroll 4
    for (int p = p0 + r; p < p1; p += rows) {
      float f[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(xi + (long long)p * c), f);
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v0 = fmaf(f[2 * e], t[2 * e].x, t[2 * e].y);
        float v1 = fmaf(f[2 * e + 1], t[2 * e + 1].x, t[2 * e + 1].y);
        if (apply_silu) {
          v0 = __fdividef(v0, 1.0f + __expf(-v0));
          v1 = __fdividef(v1, 1.0f + __expf(-v1));
        }
        o[e] = pack_bf16x2(v0, v1);
      }
      *reinterpret_cast<uint4*>(yi + (long long)p * c) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

size_t fused_smem_bytes(int64_t c, int64_t groups) {
  const int64_t rows = kFusedThreads / (c / 8);
  return size_t(2 * rows * c + 2 * c + 2 * groups) * sizeof(float);
}

}  // namespace

size_t group_norm_scratch_bytes(int64_t n, int64_t groups) {
  // Fixed region of zero-initialised ticket counters first (the same place whatever the sizes, so a scratch reused
  // across shapes always finds them zero), then (mean, rstd) per (image, group), then the slice partials.
  return size_t(kGnCounters) * 4 + size_t(n * groups) * (8 + 8 * std::max(kGnMaxSlices, kGnFusedMaxSlices));
}

int group_norm_launch(const void* x, int64_t n, int64_t hw, int64_t c, int64_t groups, const float* gamma,
                      const float* beta, float eps, int apply_silu, void* out, float* stats, cudaStream_t stream,
                      uint32_t debug) {
  const DeviceInfo* dev = nullptr;
  if (int rc = current_device_info(&dev)) return rc;
  if (x == nullptr || out == nullptr || gamma == nullptr || beta == nullptr || stats == nullptr)
    return fail(kErrInvalid, "group_norm: null pointer");
  if (n <= 0 || hw <= 0 || c <= 0 || groups <= 0 || c % groups != 0)
    return fail(kErrInvalid, "group_norm: bad sizes (n=%lld hw=%lld c=%lld groups=%lld)", (long long)n,
                (long long)hw, (long long)c, (long long)groups);
  if (c % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return fail(kErrUnsupported, "group_norm needs c %% 8 == 0 and 16-byte aligned tensors");
  if (n > 65535 || groups > 65535 || n * groups > kGnBarrier || hw > INT32_MAX / 64 ||
      hw * (c / groups) > INT32_MAX)
    return fail(kErrInvalid, "group_norm: too large (images x groups <= %lld)", (long long)kGnBarrier);
  if (c > 6144) return fail(kErrUnsupported, "group_norm: at most 6144 channels");  // 48 KB scale/shift table
  unsigned int* counters = reinterpret_cast<unsigned int*>(stats);         // [kGnCounters]
  float* st = stats + kGnCounters;                                         // [n * groups] float2
  float* partials = st + 2 * n * groups;                                   // slice partials, float2
  // One launch for large tensors when every block of a grid with at least one slice per image can be resident at
  // once. Below ~4M values the grid barrier costs more than the second launch it saves (measured on the SD1.5
  // ResBlocks: batch 2 slower by ~3.6 us per call, batch 16 at 64x64 faster, 32 vs 47 us).
  const uint32_t forced = debug & (kDebugGnTwoLaunch | kDebugGnCooperative);
  if (c <= 4096 && (forced ? forced == kDebugGnCooperative : n * hw * c >= (int64_t(1) << 22))) {
    static int per_sm[64] = {0};
    const size_t smem = fused_smem_bytes(c, groups);
    if (dev->device < 0 || dev->device >= 64) return fail(kErrInvalid, "device ordinal out of range");
    if (per_sm[dev->device] == 0) {
      cudaError_t e = cudaFuncSetAttribute(gn_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
      if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(group_norm)");
      int nb = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, gn_fused_kernel, kFusedThreads, 96 * 1024);
      if (e != cudaSuccess) return check_cuda(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor(group_norm)");
      per_sm[dev->device] = std::max(nb, 1);  // at 96 KB of shared memory: a floor for any smaller table
    }
    const int64_t capacity = int64_t(per_sm[dev->device]) * dev->sms;
    if (smem <= 96 * 1024 && n <= capacity) {
      const int64_t rows = kFusedThreads / (c / 8);
      int64_t slices = std::min<int64_t>({int64_t(kGnFusedMaxSlices), capacity / n,
                                          std::max<int64_t>(1, (hw + rows - 1) / rows)});
      slices = std::max<int64_t>(slices, 1);
      cudaLaunchConfig_t cfg;
      memset(&cfg, 0, sizeof(cfg));
      cfg.gridDim = dim3(unsigned(slices), unsigned(n));
      cfg.blockDim = dim3(kFusedThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      return check_cuda(
          cudaLaunchKernelEx(&cfg, gn_fused_kernel, static_cast<const __nv_bfloat16*>(x),
                             static_cast<__nv_bfloat16*>(out), int(hw), int(c), int(c / groups), int(groups), eps,
                             gamma, beta, apply_silu, reinterpret_cast<float2*>(partials), counters + kGnBarrier,
                             unsigned(slices * n), dev->status, (unsigned long long)wait_timeout_ns()),
          "group_norm launch");
    }
  }
  const int64_t cg = c / groups;
  // Pixel slices per (image, group): enough blocks to fill the GPU, each with at least a few thousand values.
  int64_t slices = std::max<int64_t>(1, (int64_t(dev->sms) * 4 + n * groups - 1) / (n * groups));
  slices = std::min<int64_t>({slices, int64_t(kGnMaxSlices), std::max<int64_t>(1, hw * cg / 4096)});
  if (int rc = check_cuda(launch_pdl(gn_stats_kernel, dim3(unsigned(groups), unsigned(n), unsigned(slices)),
                                     dim3(kStatsThreads), 0, stream, static_cast<const __nv_bfloat16*>(x), int(hw),
                                     int(c), int(cg), eps, reinterpret_cast<float2*>(st),
                                     reinterpret_cast<float2*>(partials), counters),
                          "group_norm stats launch"))
    return rc;
  // Pixels per apply block (within one image): about four blocks per SM over the whole tensor, at least one pixel.
  const int64_t vecs = n * hw * (c / 8);
  const int64_t per_block = (vecs + int64_t(dev->sms) * 4 - 1) / (int64_t(dev->sms) * 4);
  const int64_t block_pixels = std::max<int64_t>(1, std::min<int64_t>(hw, (per_block + c / 8 - 1) / (c / 8)));
  const dim3 agrid(unsigned((hw + block_pixels - 1) / block_pixels), unsigned(n));
  return check_cuda(launch_pdl(gn_apply_kernel, agrid, dim3(kApplyThreads), size_t(c) * sizeof(float2), stream,
                               static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), int(hw),
                               int(c), int(c / groups), int(groups), int(block_pixels),
                               reinterpret_cast<const float2*>(st), gamma, beta, apply_silu),
                    "group_norm apply launch");
}

}  // namespace npub200
