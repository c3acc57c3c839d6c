// gemm_noalloc.cu - the GEMM entry point for callers that cannot allocate device memory.
//
// npub200_gemm needs a caller-provided workspace when an operand is not TMA-addressable (K % 8 != 0, a row stride
// that is not a multiple of 8 elements, an unaligned base): the kernel reads a repacked dense copy of it. Some
// callers have no way to provide one: a host application whose device memory belongs to its own pool manager and
// that forbids allocations while it serves a request, an FFI binding that holds only the pointers it was handed (no
// allocator of its own), or code that must not call cudaMalloc because that call synchronises the whole device
// mid-stream. npub200_gemm_noalloc serves them: the repacked operands go to one file-scope device array of a fixed
// size that every GPU loading this library keeps until process exit; the entry point itself calls no cudaMalloc,
// cudaFree or allocating library routine.
//
// What the array holds: after a 4 KiB leading region that the workspace layout reserves (nothing reads or writes
// it), the repacked x and/or W of the latest call that needed them. Split K needs no scratch (its partials are
// reduced in a cluster's distributed shared memory). Every repack writes all the bytes the kernel then reads, pad
// columns included, so nothing has to start at zero and nothing is cleared.
//
// Sharing rules: every call on a device uses the same array, and the array keeps the last call's contents. The
// first call on each device resolves the array's device address (cudaGetSymbolAddress, which may load the module's
// device code), so make that first call before any stream capture. Calls whose work overlaps on the GPU (different
// streams, or host threads racing on one device) race on the array: callers must serialise them, e.g. by issuing
// every call on one stream.
#include <cstring>
#include <mutex>

#include "npu_b200.h"
#include "internal.h"

namespace npub200 {

// The shared scratch (repacked operands, after the reserved leading region). Host code sees only a stand-in for this
// symbol; its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NPUB200_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Once per device, with that device current: resolve the array's device address (no allocation, no device sync).
int noalloc_setup(int device, void** out) {
  if (device < 0 || device >= kMaxDevices)
    return fail(kErrInvalid, "npub200_gemm_noalloc: device ordinal %d outside [0, %d)", device, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[device] == nullptr) {
    void* p = nullptr;
    if (int rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(no-alloc scratch)"))
      return rc;
    g_scratch_ptr[device] = p;
  }
  *out = g_scratch_ptr[device];
  return kOk;
}

}  // namespace

}  // namespace npub200

using namespace npub200;

extern "C" int npub200_gemm_noalloc(const void* x, int64_t ldx, int64_t m, int64_t k, const void* w, int64_t ldw,
                                    int64_t n, const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype,
                                    int variant, void* stream) {
  if (m <= 0 || k <= 0 || n <= 0)
    return fail(kErrInvalid, "GEMM sizes must be positive (M=%lld K=%lld N=%lld)", (long long)m, (long long)k,
                (long long)n);
  const DeviceInfo* dev = nullptr;
  if (int rc = current_device_info(&dev)) return rc;
  const size_t need = gemm_workspace_bytes(x, ldx, m, k, w, ldw, n, variant, dev->sms);
  if (need > size_t(NPUB200_NOALLOC_SCRATCH_BYTES))
    return fail(kErrInvalid,
                "npub200_gemm_noalloc: this GEMM (M=%lld K=%lld N=%lld) needs %zu bytes of scratch, above the "
                "library's fixed %d-byte array; use npub200_gemm with a workspace",
                (long long)m, (long long)k, (long long)n, need, int(NPUB200_NOALLOC_SCRATCH_BYTES));
  void* scratch = nullptr;
  if (int rc = noalloc_setup(dev->device, &scratch)) return rc;
  return gemm_with_workspace(x, ldx, m, k, w, ldw, n, nullptr, bias, bias_dtype, out, ldo, out_dtype, scratch,
                             size_t(NPUB200_NOALLOC_SCRATCH_BYTES), variant, stream);
}
