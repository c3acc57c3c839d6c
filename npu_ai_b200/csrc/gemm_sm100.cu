// gemm_sm100.cu - shape-agnostic bf16 GEMM for nn.Linear on B200: y[M,N] = x[M,K] . W[N,K]^T (+ bias).
//
// Replaces the NPU GEMM of the reference runner (npu/xdna1_gemm.py:349-422 `NpuGemm.matmul_t`, dispatched
// through npu/xdna1_program.py:451-454 `submit_gemm`, computed by npu/kernels/xdna1_attn.cc:480-574
// `gemm_step`/`gemm_zero`/`gemm_store`). Same arithmetic contract: bf16 operands, f32 accumulation, bias added
// in f32 after the accumulation (xdna1_gemm.py:417-418); the output is f32 (the reference's) or bf16.
//
// Design (one persistent CTA per SM, 192 threads):
//   warp 0      TMA producer: 128x64 tiles of x and BNx64 tiles of W (128-byte swizzle) into a STAGES-deep ring
//   warp 1      TMEM owner + MMA issuer: tcgen05.mma kind::f16, M=128, N=BN, K=16 steps, f32 accumulators in
//               TMEM, double-buffered so the epilogue of tile i overlaps the main loop of tile i+1
//   warps 2-5   epilogue: tcgen05.ld of the accumulator rows, bias add, cast, predicated stores
// Ragged M/N/K need no padding: TMA zero-fills out-of-bounds rows and columns, the epilogue stores only rows < M
// and columns < N. The only layout requirement is TMA's: 16-byte aligned base and row strides (K % 8 == 0 for a
// dense matrix); anything else is repacked by the host into a caller-provided workspace first.
#include <algorithm>
#include <cstdio>

#include "internal.h"

namespace npub200 {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // one 128-byte swizzle atom of bf16 along K
constexpr int kGemmThreads = 192;

struct GemmArgs {
  int M, N, K;
  int num_m_blk, num_tiles, num_kb;
  const void* bias;
  int bias_f32;
  void* out;
  long long ldo;
  int out_f32;
  KernelCtl ctl;
};

template <int BN, int STAGES>
struct GemmLayout {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kNumBars = 2 * STAGES + 5;  // full[S], empty[S], acc_full[2], acc_empty[2], drain
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOffset + 16 + 1024;  // + slack to align the base to 1 KB
  static_assert(kBBytes % 1024 == 0, "B stage must keep 1 KB alignment for the 128-byte swizzle");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128 is a multiple of 16 in [16, 256]");
};

__device__ __forceinline__ float bias_at(const GemmArgs& a, int col) {
  return a.bias_f32 ? __ldg(static_cast<const float*>(a.bias) + col)
                    : __bfloat162float(static_cast<const __nv_bfloat16*>(a.bias)[col]);
}

// Store 16 consecutive accumulator columns of one output row (columns gcol .. gcol+15, rows/cols predicated).
__device__ __forceinline__ void store_row16(const GemmArgs& a, int grow, int gcol, const uint32_t (&r)[16]) {
  if (grow >= a.M) return;
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
  const int ncols = min(16, a.N - gcol);
  if (ncols <= 0) return;
  if (a.bias != nullptr) {
    if (ncols == 16) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] += bias_at(a, gcol + j);
    } else {
      for (int j = 0; j < ncols; ++j) v[j] += bias_at(a, gcol + j);
    }
  }
  if (a.out_f32) {
    float* o = static_cast<float*>(a.out) + (long long)grow * a.ldo + gcol;
    if (ncols == 16 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
      for (int j = 0; j < 4; ++j) o4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
      for (int j = 0; j < ncols; ++j) o[j] = v[j];
    }
  } else {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out) + (long long)grow * a.ldo + gcol;
    if (ncols == 16 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
      uint4 p0, p1;
      p0.x = pack_bf16x2(v[0], v[1]);
      p0.y = pack_bf16x2(v[2], v[3]);
      p0.z = pack_bf16x2(v[4], v[5]);
      p0.w = pack_bf16x2(v[6], v[7]);
      p1.x = pack_bf16x2(v[8], v[9]);
      p1.y = pack_bf16x2(v[10], v[11]);
      p1.z = pack_bf16x2(v[12], v[13]);
      p1.w = pack_bf16x2(v[14], v[15]);
      uint4* o4 = reinterpret_cast<uint4*>(o);
      o4[0] = p0;
      o4[1] = p1;
    } else {
      for (int j = 0; j < ncols; ++j) o[j] = __float2bfloat16_rn(v[j]);
    }
  }
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                             const GemmArgs args) {
  using L = GemmLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOffset);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = args.num_tiles;
  const int num_m = args.num_m_blk;
  const int num_kb = args.num_kb;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        const int m0 = (tile % num_m) * kGemmBM;
        const int n0 = (tile / num_m) * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, args.ctl, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          tma_load_2d(&tm_x, &full[stage], sA + stage * L::kABytes, kb * kGemmBK, m0);
          tma_load_2d(&tm_w, &full[stage], sB + stage * L::kBBytes, kb * kGemmBK, n0);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Abort: let the (at most STAGES) loads still in flight land before the CTA's shared memory goes away.
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < min(issued, STAGES); ++i) {
          if (s == 0) {
            s = STAGES - 1;
            ph ^= 1u;
          } else {
            --s;
          }
          mbar_wait_drain(&full[s], ph, args.ctl);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_bf16_f32(kGemmBM, BN, false);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      if (args.ctl.debug & 1u) {
        // Test hook: wait on a barrier nothing arrives on, so the bounded wait expires and the abort path runs.
        if (!mbar_wait_bounded(drain, 0, abort_flag, args.ctl, kStatusForced)) ok = false;
      }
      int local = 0;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1u, abort_flag, args.ctl, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, args.ctl, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_desc = smem_desc_kmajor_sw128(smem_u32(sA + stage * L::kABytes));
          const uint64_t b_desc = smem_desc_kmajor_sw128(smem_u32(sB + stage * L::kBBytes));
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            // +32 bytes per K step of 16 bf16 inside the swizzle atom (descriptor address field is >> 4).
            umma_f16_ss(d_tmem, a_desc + 2u * k, b_desc + 2u * k, kIdesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);  // frees the smem stage once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);  // accumulator complete
      }
      if (!ok) {
        // Abort: wait until every MMA this thread issued has finished before TMEM is released.
        umma_commit(drain);
        mbar_wait_drain(drain, 0u, args.ctl);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;  // TMEM lanes this warp may access: [32*quarter, 32*quarter + 32)
    const int row = quarter * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&acc_full[acc], acc_phase, abort_flag, args.ctl, kStatusTimeoutEpilogue)) break;
      tc_fence_after();
      const int m0 = (tile % num_m) * kGemmBM;
      const int n0 = (tile / num_m) * BN;
      const uint32_t t_row = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld16(t_row + uint32_t(c), r);
        tmem_wait_ld();
        store_row16(args, m0 + row, n0 + c, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------------------------
namespace {

template <int BN, int STAGES>
int launch_variant(const CUtensorMap& mx, const CUtensorMap& mw, const GemmArgs& args, int grid, cudaStream_t st,
                   int device) {
  using L = GemmLayout<BN, STAGES>;
  static bool configured[64] = {false};
  auto kern = gemm_bf16_tcgen05_kernel<BN, STAGES>;
  if (device < 0 || device >= 64) return fail(kErrInvalid, "device ordinal %d out of range", device);
  if (!configured[device]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(gemm smem)");
    configured[device] = true;
  }
  kern<<<grid, kGemmThreads, L::kSmemBytes, st>>>(mx, mw, args);
  return check_cuda(cudaGetLastError(), "gemm kernel launch");
}

int encode_kmajor_map(const void* base, int64_t rows, int64_t k, int64_t ld, int box_rows, CUtensorMap* out) {
  EncodeTiledFn enc = nullptr;
  if (int rc = encode_tiled_fn(&enc)) return rc;
  cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  cuuint32_t box[2] = {cuuint32_t(kGemmBK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(kErrInvalid, "cuTensorMapEncodeTiled failed (%d) for a %lld x %lld bf16 operand, ld %lld", int(r),
                (long long)rows, (long long)k, (long long)ld);
  return kOk;
}

constexpr int kTileChoices[] = {64, 80, 128, 160, 256};

}  // namespace

int gemm_pick_bn(int64_t M, int64_t N, int64_t K, int sms) {
  // Cost model: waves of persistent tiles x per-tile time, where a tile's main loop is bounded by the larger of
  // the tensor-core time (2*BN clocks per 64-deep K block at 8192 FLOP/clk/SM) and the time to stream its
  // operands into shared memory (~64 B/clk/SM), plus a fixed epilogue/turnaround cost per tile.
  const int64_t kb = (K + kGemmBK - 1) / kGemmBK;
  const int64_t mblk = (M + kGemmBM - 1) / kGemmBM;
  double best = 1e300;
  int best_bn = 128;
  for (int bn : kTileChoices) {
    const int64_t tiles = mblk * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + sms - 1) / sms;
    const double mma = 2.0 * bn;
    const double load = (kGemmBM + bn) * 128.0 / 64.0;
    const double t_tile = double(kb) * std::max(mma, load) + 150.0 + 4.0 * bn;
    const double cost = double(waves) * t_tile;
    if (cost < best * 0.999 || (cost <= best * 1.001 && bn > best_bn)) {
      best = cost;
      best_bn = bn;
    }
  }
  return best_bn;
}

int gemm_encode_b_map(const void* w, int64_t ldw, int64_t N, int64_t K, int bn, CUtensorMap* out) {
  return encode_kmajor_map(w, N, K, ldw, bn, out);
}

int gemm_launch(const GemmProblem& p, cudaStream_t stream) {
  const DeviceInfo* dev = nullptr;
  if (int rc = current_device_info(&dev)) return rc;
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return fail(kErrInvalid, "GEMM sizes must be positive (M=%lld N=%lld K=%lld)",
                                                    (long long)p.M, (long long)p.N, (long long)p.K);
  if (p.M > INT32_MAX / 2 || p.N > INT32_MAX / 2 || p.K > INT32_MAX / 2)
    return fail(kErrInvalid, "GEMM dimension too large");
  int bn = p.variant ? p.variant : gemm_pick_bn(p.M, p.N, p.K, dev->sms);
  bool known = false;
  for (int c : kTileChoices) known |= (c == bn);
  if (!known) return fail(kErrUnsupported, "no GEMM variant with an N tile of %d", bn);

  CUtensorMap mx, mw;
  if (int rc = encode_kmajor_map(p.x, p.M, p.K, p.ldx, kGemmBM, &mx)) return rc;
  if (p.w_map_cache != nullptr) {
    mw = *p.w_map_cache;
  } else if (int rc = encode_kmajor_map(p.w, p.N, p.K, p.ldw, bn, &mw)) {
    return rc;
  }

  GemmArgs a;
  a.M = int(p.M);
  a.N = int(p.N);
  a.K = int(p.K);
  a.num_m_blk = int((p.M + kGemmBM - 1) / kGemmBM);
  const int num_n = int((p.N + bn - 1) / bn);
  const int64_t tiles = int64_t(a.num_m_blk) * num_n;
  if (tiles > INT32_MAX) return fail(kErrInvalid, "GEMM has too many tiles");
  a.num_tiles = int(tiles);
  a.num_kb = int((p.K + kGemmBK - 1) / kGemmBK);
  a.bias = p.bias;
  a.bias_f32 = p.bias_f32;
  a.out = p.out;
  a.ldo = p.ldo;
  a.out_f32 = p.out_f32;
  a.ctl.status = dev->status;
  a.ctl.timeout_ns = wait_timeout_ns();
  a.ctl.debug = p.debug;
  const int grid = int(std::min<int64_t>(tiles, dev->sms));

  switch (bn) {
    case 64: return launch_variant<64, 8>(mx, mw, a, grid, stream, dev->device);
    case 80: return launch_variant<80, 8>(mx, mw, a, grid, stream, dev->device);
    case 128: return launch_variant<128, 6>(mx, mw, a, grid, stream, dev->device);
    case 160: return launch_variant<160, 5>(mx, mw, a, grid, stream, dev->device);
    case 256: return launch_variant<256, 4>(mx, mw, a, grid, stream, dev->device);
  }
  return fail(kErrUnsupported, "no GEMM variant with an N tile of %d", bn);
}

// ---------------------------------------------------------------------------------------------------------------
// Repack (the workspace path for operands whose rows TMA cannot address: K % 8 != 0 or unaligned strides)
// ---------------------------------------------------------------------------------------------------------------
__global__ void repack_rows_bf16_kernel(const __nv_bfloat16* __restrict__ src, long long ld_src, long long rows,
                                        long long cols, __nv_bfloat16* __restrict__ dst, long long cols_pad) {
  const long long total = rows * cols_pad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols_pad;
    const long long c = i - r * cols_pad;
    dst[i] = c < cols ? src[r * ld_src + c] : __float2bfloat16_rn(0.0f);
  }
}

int repack_rows_bf16(const void* src, int64_t ld_src, int64_t rows, int64_t cols, void* dst, int64_t cols_pad,
                     cudaStream_t stream) {
  const DeviceInfo* dev = nullptr;
  if (int rc = current_device_info(&dev)) return rc;
  const long long total = rows * cols_pad;
  const int threads = 256;
  const long long want = (total + threads - 1) / threads;
  const int grid = int(std::max<long long>(1, std::min<long long>(want, int64_t(dev->sms) * 8)));
  repack_rows_bf16_kernel<<<grid, threads, 0, stream>>>(static_cast<const __nv_bfloat16*>(src), ld_src, rows, cols,
                                                         static_cast<__nv_bfloat16*>(dst), cols_pad);
  return check_cuda(cudaGetLastError(), "repack kernel launch");
}

}  // namespace npub200
