// nhwc_copy.cu - the two pure data-movement steps of an SD1.5 UNet's decoder on NHWC (channels-last) activations:
// nearest-neighbour 2x upsampling in front of each Upsample block's 3x3 convolution, and the channel concatenation
// of the decoder's activations with the encoder's skip tensors in front of each output ResBlock. The reference
// leaves both to the host with the rest of the UNet (docs/02-results.md:411-413); torch's NHWC kernels for them run
// at 0.4-2 TB/s on B200, far from the HBM roofline.
//
// Both move 16-byte chunks (8 two-byte elements): one chunk per work unit, four units per thread with the loads of
// all four issued before the stores. Upsampling reads each input chunk once and writes it to its 2x2 output pixels;
// concatenation writes each output chunk once from whichever source owns its channels. Algorithmic bytes = reads +
// writes, each exactly once. The element type only has to be two bytes wide (bf16 or f16).
#include <algorithm>

#include "internal.h"

namespace npub200 {

namespace {

constexpr int kCopyThreads = 256;
constexpr int kUnitsPerThread = 4;

// out[img][2y+a][2x+b][:] = in[img][y][x][:] for a, b in {0, 1}. Unit i = chunk j of input pixel q = (row r, x),
// r = img * h + y; output row 2r is the top row of that pixel's 2x2 block.
__global__ void __launch_bounds__(kCopyThreads)
    upsample_nearest2x_kernel(const uint4* __restrict__ in, uint4* __restrict__ out, uint32_t units, uint32_t cc,
                              uint32_t w) {
  pdl_wait();  // the input is the previous kernel's output
  pdl_launch_dependents();
  const uint32_t stride = gridDim.x * kCopyThreads;
  const uint32_t first = blockIdx.x * kCopyThreads + threadIdx.x;
  uint4 v[kUnitsPerThread];
#pragma unroll
  for (int u = 0; u < kUnitsPerThread; ++u) {
    const uint32_t i = first + u * stride;
    if (i < units) v[u] = __ldg(in + i);
  }
  const size_t row_chunks = size_t(2) * w * cc;  // chunks in one output row
#pragma unroll
  for (int u = 0; u < kUnitsPerThread; ++u) {
    const uint32_t i = first + u * stride;
    if (i >= units) break;
    const uint32_t q = i / cc;
    const uint32_t j = i - q * cc;
    const uint32_t r = q / w;
    const uint32_t x = q - r * w;
    uint4* o = out + (size_t(2) * r) * row_chunks + size_t(2) * x * cc + j;
    o[0] = v[u];
    o[cc] = v[u];
    o[row_chunks] = v[u];
    o[row_chunks + cc] = v[u];
  }
}

// out[p][0:ca] = a[p][:], out[p][ca:ca+cb] = b[p][:] for every pixel p; strides in chunks. Unit i = output chunk k
// of pixel p.
__global__ void __launch_bounds__(kCopyThreads)
    concat_channels_kernel(const uint4* __restrict__ a, uint32_t lda, uint32_t ca, const uint4* __restrict__ b,
                           uint32_t ldb, uint4* __restrict__ out, uint32_t ldo, uint32_t co, uint32_t units) {
  pdl_wait();  // either source may be the previous kernel's output
  pdl_launch_dependents();
  const uint32_t stride = gridDim.x * kCopyThreads;
  const uint32_t first = blockIdx.x * kCopyThreads + threadIdx.x;
  uint4 v[kUnitsPerThread];
#pragma unroll
  for (int u = 0; u < kUnitsPerThread; ++u) {
    const uint32_t i = first + u * stride;
    if (i < units) {
      const uint32_t p = i / co;
      const uint32_t k = i - p * co;
      v[u] = k < ca ? __ldg(a + size_t(p) * lda + k) : __ldg(b + size_t(p) * ldb + (k - ca));
    }
  }
#pragma unroll
  for (int u = 0; u < kUnitsPerThread; ++u) {
    const uint32_t i = first + u * stride;
    if (i >= units) break;
    const uint32_t p = i / co;
    out[size_t(p) * ldo + (i - p * co)] = v[u];
  }
}

unsigned copy_blocks(uint64_t units) {
  return unsigned((units + uint64_t(kCopyThreads) * kUnitsPerThread - 1) / (uint64_t(kCopyThreads) * kUnitsPerThread));
}

bool overlaps(const void* p, size_t pb, const void* q, size_t qb) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p), b = reinterpret_cast<uintptr_t>(q);
  return a < b + qb && b < a + pb;
}

}  // namespace

int upsample_nearest2x_launch(const void* x, int64_t n, int64_t h, int64_t w, int64_t c, void* out,
                              cudaStream_t stream) {
  if (x == nullptr || out == nullptr || n < 0 || h < 0 || w < 0 || c < 0)
    return fail(kErrInvalid, "upsample_nearest2x: bad arguments (n=%lld h=%lld w=%lld c=%lld)", (long long)n,
                (long long)h, (long long)w, (long long)c);
  if (c % 8 != 0 || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) != 0)
    return fail(kErrUnsupported, "upsample_nearest2x needs channels in multiples of 8 and 16-byte aligned tensors");
  const uint64_t units = uint64_t(n) * uint64_t(h) * uint64_t(w) * uint64_t(c / 8);
  if (units == 0) return kOk;
  // Output chunk offsets reach 4 * units; keep every index of the kernel in 32 bits (and its products in size_t).
  if (4 * units >= (uint64_t(1) << 32) || uint64_t(copy_blocks(units)) * kCopyThreads * kUnitsPerThread >= (uint64_t(1) << 32))
    return fail(kErrUnsupported, "upsample_nearest2x: tensor too large (%llu chunks)", (unsigned long long)units);
  if (overlaps(x, units * 16, out, 4 * units * 16))
    return fail(kErrInvalid, "upsample_nearest2x: out overlaps the input");
  return check_cuda(launch_pdl(upsample_nearest2x_kernel, dim3(copy_blocks(units)), dim3(kCopyThreads), 0, stream,
                               static_cast<const uint4*>(x), static_cast<uint4*>(out), uint32_t(units),
                               uint32_t(c / 8), uint32_t(w)),
                    "upsample_nearest2x launch");
}

int concat_channels_launch(const void* a, int64_t lda, int64_t ca, const void* b, int64_t ldb, int64_t cb,
                           int64_t pixels, void* out, int64_t ldo, cudaStream_t stream) {
  if (a == nullptr || b == nullptr || out == nullptr || pixels < 0 || ca <= 0 || cb <= 0 || lda < ca || ldb < cb ||
      ldo < ca + cb)
    return fail(kErrInvalid, "concat_channels: bad arguments (pixels=%lld ca=%lld lda=%lld cb=%lld ldb=%lld ldo=%lld)",
                (long long)pixels, (long long)ca, (long long)lda, (long long)cb, (long long)ldb, (long long)ldo);
  const uintptr_t align = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                          reinterpret_cast<uintptr_t>(out);
  if (ca % 8 != 0 || cb % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0 || ldo % 8 != 0 || (align & 15) != 0)
    return fail(kErrUnsupported, "concat_channels needs channel counts and row strides in multiples of 8 and "
                                 "16-byte aligned tensors");
  if (pixels == 0) return kOk;
  const uint64_t co = uint64_t(ca + cb) / 8;
  const uint64_t units = uint64_t(pixels) * co;
  const uint64_t span_out = (uint64_t(pixels - 1) * uint64_t(ldo) + uint64_t(ca + cb)) * 2;
  if (units >= (uint64_t(1) << 32) || uint64_t(copy_blocks(units)) * kCopyThreads * kUnitsPerThread >= (uint64_t(1) << 32) ||
      uint64_t(ldo) / 8 >= (uint64_t(1) << 32) || uint64_t(lda) / 8 >= (uint64_t(1) << 32) ||
      uint64_t(ldb) / 8 >= (uint64_t(1) << 32))
    return fail(kErrUnsupported, "concat_channels: tensor too large (%llu chunks)", (unsigned long long)units);
  if (overlaps(a, (uint64_t(pixels - 1) * lda + ca) * 2, out, span_out) ||
      overlaps(b, (uint64_t(pixels - 1) * ldb + cb) * 2, out, span_out))
    return fail(kErrInvalid, "concat_channels: out overlaps a source");
  return check_cuda(launch_pdl(concat_channels_kernel, dim3(copy_blocks(units)), dim3(kCopyThreads), 0, stream,
                               static_cast<const uint4*>(a), uint32_t(lda / 8), uint32_t(ca / 8),
                               static_cast<const uint4*>(b), uint32_t(ldb / 8), static_cast<uint4*>(out),
                               uint32_t(ldo / 8), uint32_t(co), uint32_t(units)),
                    "concat_channels launch");
}

}  // namespace npub200
