// gemm_sm100.cu - shape-agnostic bf16 GEMM for nn.Linear on B200: y[M,N] = x[M,K] . W[N,K]^T (+ bias).
//
// Replaces the NPU GEMM of the reference runner (npu/xdna1_gemm.py:349-422 `NpuGemm.matmul_t`, dispatched
// through npu/xdna1_program.py:451-454 `submit_gemm`, computed by npu/kernels/xdna1_attn.cc:480-574
// `gemm_step`/`gemm_zero`/`gemm_store`). Same arithmetic contract: bf16 operands, f32 accumulation, bias added
// in f32 after the accumulation (xdna1_gemm.py:417-418); the output is f32 (the reference's) or bf16.
//
// Design (one persistent CTA per SM, 320 threads = kGemmThreads):
//   warp 0      TMA producer: 128x64 tiles of x and BNx64 tiles of W (128-byte swizzle) into a STAGES-deep ring
//   warp 1      TMEM owner + MMA issuer: tcgen05.mma kind::f16, M=128, N=BN, K=16 steps, f32 accumulators in
//               TMEM, double-buffered so the epilogue of tile i overlaps the main loop of tile i+1
//   warps 2-9   epilogue, two warps per TMEM lane quarter on alternate 64-column chunks: tcgen05.ld of the
//               accumulator rows, bias add, cast, swizzled staging + TMA store (or predicated direct stores)
// Ragged M/N/K need no padding: TMA zero-fills out-of-bounds rows and columns, the epilogue stores only rows < M
// and columns < N.
// GEGLU form (template flag): W holds 2N rows ([a; gate], the GEGLU projection of SD1.5's feed-forward block) and
// out[:, j] = (x.W[j] + b[j]) * gelu(x.W[N+j] + b[N+j]), the exact (erf) GELU. A tile's BN accumulator columns are
// BN/2 a-rows and the BN/2 matching gate rows (two TMA boxes per stage), so the epilogue gates in registers and
// the 2N-column projection is never written to memory.
// 3x3 convolution form (template mode): implicit GEMM over an NHWC input, M = images x H x W pixels, N = output
// channels, K = 9 taps x input channels. The A tile of K block (tap, 64-channel block) is one 4-D TMA box of 64
// channels x a 128-pixel patch of whole image rows, shifted by the tap; the out-of-range rows and columns of the
// shift are TMA zeros, which is the convolution's zero padding. The weights are [Cout, 3, 3, Cin] (K-major) and the
// output tile is 128 consecutive NHWC pixels, so the epilogue is the GEMM's. The epilogue can also add a per-image
// bias row (conv bias + time embedding) and a residual tensor. The only layout requirement is TMA's: 16-byte aligned base and row strides (K % 8 == 0 for a
// dense matrix); anything else is repacked by the host into a caller-provided workspace first.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "internal.h"

namespace npub200 {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // one 128-byte swizzle atom of bf16 along K
// Warp roles: 0 = TMA producer, 1 = MMA issuer, 2..9 = epilogue. Two epilogue warps share each TMEM lane quarter
// (32 accumulator rows) and take alternate output chunks, so one warp's TMEM-load and store latencies overlap the
// other's arithmetic.
constexpr int kGemmEpiWarps = 8;
constexpr int kGemmEpiThreads = kGemmEpiWarps * 32;
constexpr int kGemmThreads = 64 + kGemmEpiThreads;

struct GemmArgs {
  int M, N, K;
  int num_m_blk, num_n_blk, num_tiles, num_kb;
  int n_fastest;  // tile raster: 1 = N tiles innermost (x stays in L2 across them), 0 = M tiles innermost
  const void* bias;
  int bias_f32;
  int bias_n;     // bias entries (N, or 2N in the GEGLU form)
  long long bias_img_stride;  // > 0: bias row per image (rows of bias_img_pixels output rows), else one bias row
  int bias_img_pixels, bias_imgs;
  const void* residual;       // bf16 [M, N] added in the epilogue (row stride ldr), or null
  long long ldr;
  int cv_w, cv_hw, cv_cblocks;  // 3x3 convolution form: image width, pixels per image, 64-channel blocks of Cin
  void* out;
  long long ldo;
  int out_f32;
  int tma_store;  // 1: the output goes out through TMA stores (aligned output), 0: direct predicated stores
  // Split-K: `splits` CTAs, one cluster, share an output tile, each over `kb_per_split` K blocks. Each parks its
  // f32 partial in its own shared memory; after all have, each sums a slice of the tile over every CTA's partial
  // in split order (distributed shared memory), so the result does not depend on timing.
  int splits, kb_per_split;
  KernelCtl ctl;
};

// BROWS: rows of the B tile this CTA holds per stage (BN, or BN/2 for one CTA of a pair).
template <int BN, int STAGES, int BROWS = BN>
struct GemmLayout {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr int kBBytes = BROWS * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  // Epilogue staging: per epilogue warp one 32-row x 128-byte tile (128-byte swizzle) for the TMA stores.
  static constexpr int kStagingOffset = STAGES * kStageBytes;
  static constexpr int kStagingBytes = kGemmEpiWarps * 32 * 128;
  static constexpr int kBarOffset = kStagingOffset + kStagingBytes;
  // full[S], empty[S], acc_full[2], acc_empty[2], drain, bias_full, bias_free, parts_ready
  static constexpr int kNumBars = 2 * STAGES + 8;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  // The tile's bias in f32 (BN entries: the output columns', then in the GEGLU form the gate columns').
  static constexpr int kBiasOffset = (kMiscOffset + 16 + 15) / 16 * 16;
  static constexpr int kSmemBytes = kBiasOffset + BN * 4 + 1024;  // + slack to align the base to 1 KB
  static_assert(kBBytes % 1024 == 0, "B stage must keep 1 KB alignment for the 128-byte swizzle");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "N tile: a multiple of 32 (UMMA N for M=128 <= 256)");
  static_assert(kSmemBytes <= 232448, "shared memory budget of one CTA");
};

// Bias for 32 consecutive output columns starting at gcol (0 beyond N). Compile-time indices only, so the values
// stay in registers; the loads are broadcasts (every thread of the warp reads the same addresses).
__device__ __forceinline__ void load_bias32(const GemmArgs& a, int gcol, float (&b)[32], long long row_off = 0) {
  if (a.bias == nullptr) {
#pragma unroll
    for (int j = 0; j < 32; ++j) b[j] = 0.0f;
    return;
  }
  if (a.bias_f32) {
    const float* p = static_cast<const float*>(a.bias) + row_off + gcol;
    if (gcol + 32 <= a.bias_n && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(p) + j);
        b[4 * j] = t.x;
        b[4 * j + 1] = t.y;
        b[4 * j + 2] = t.z;
        b[4 * j + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) b[j] = (gcol + j < a.bias_n) ? __ldg(p + j) : 0.0f;
    }
  } else {
    const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(a.bias) + row_off + gcol;
    if (gcol + 32 <= a.bias_n && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 t = __ldg(reinterpret_cast<const uint4*>(p) + j);
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          b[8 * j + 2 * e] = __uint_as_float(w[e] << 16);
          b[8 * j + 2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) b[j] = (gcol + j < a.bias_n) ? __bfloat162float(p[j]) : 0.0f;
    }
  }
}

// Bias of column gcol + j for one row (row_off: that row's bias row), 0 beyond bias_n or without a bias.
__device__ __forceinline__ float load_bias_own(const GemmArgs& a, int gcol, int j, long long row_off) {
  if (a.bias == nullptr || gcol + j >= a.bias_n) return 0.0f;
  return a.bias_f32 ? __ldg(static_cast<const float*>(a.bias) + row_off + gcol + j)
                    : __bfloat162float(static_cast<const __nv_bfloat16*>(a.bias)[row_off + gcol + j]);
}

// Direct-store epilogue for outputs TMA cannot address: 32 columns of one row, rows/columns predicated with
// compile-time indices (no dynamically indexed arrays, so nothing spills to local memory).
__device__ __forceinline__ void store_row32_direct(const GemmArgs& a, int grow, int gcol, const float (&v)[32]) {
  if (grow >= a.M || gcol >= a.N) return;
  const bool full = gcol + 32 <= a.N;
  if (a.out_f32) {
    float* o = static_cast<float*>(a.out) + (long long)grow * a.ldo + gcol;
    if (full && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        reinterpret_cast<float4*>(o)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (gcol + j < a.N) o[j] = v[j];
    }
  } else {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out) + (long long)grow * a.ldo + gcol;
    if (full && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 t;
        t.x = pack_bf16x2(v[8 * j], v[8 * j + 1]);
        t.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
        t.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
        t.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
        reinterpret_cast<uint4*>(o)[j] = t;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (gcol + j < a.N) o[j] = __float2bfloat16_rn(v[j]);
    }
  }
}

// v += residual[grow, gcol .. gcol+31] (bf16), predicated on the output bounds.
__device__ __forceinline__ void add_residual32(const GemmArgs& a, int grow, int gcol, float (&v)[32]) {
  if (grow >= a.M) return;
  const __nv_bfloat16* p = static_cast<const __nv_bfloat16*>(a.residual) + (long long)grow * a.ldr + gcol;
  if (gcol + 32 <= a.N && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 t = *(reinterpret_cast<const uint4*>(p) + j);
      const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[8 * j + 2 * e] += __uint_as_float(w[e] << 16);
        v[8 * j + 2 * e + 1] += __uint_as_float(w[e] & 0xFFFF0000u);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (gcol + j < a.N) v[j] += __bfloat162float(p[j]);
  }
}

constexpr int kModePlain = 0;
constexpr int kModeGeglu = 1;
constexpr int kModeConv3x3 = 2;

// GELU with the error function (torch's default `F.gelu`, approximate='none'): y * Phi(y) = y/2 * (1 + erf(y/sqrt2)).
// erf by Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.26 (Hastings' rational approximation,
// |error| <= 1.5e-7): for z >= 0, erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2), t = 1 / (1 + p z).
// One reciprocal and one exp2 on the MUFU and a handful of FMAs, so the gating keeps up with the main loop. For
// y < 0 the factor 1 + erf = t (...) exp(-z^2) is taken directly, without cancelling against 1.
__device__ __forceinline__ float gelu_erf(float y) {
  const float z = fabsf(y) * 0.70710678118654752f;
  const float t = __fdividef(1.0f, fmaf(0.3275911f, z, 1.0f));
  float q = fmaf(1.061405429f, t, -1.453152027f);
  q = fmaf(q, t, 1.421413741f);
  q = fmaf(q, t, -0.284496736f);
  q = fmaf(q, t, 0.254829592f);
  const float tail = q * t * fast_exp2(-z * z * 1.4426950408889634f);  // 1 - erf(z)
  return 0.5f * y * (y >= 0.0f ? 2.0f - tail : tail);
}

__device__ __forceinline__ void tile_coords(const GemmArgs& a, int tile, int& m_blk, int& n_blk) {
  if (a.n_fastest) {
    m_blk = tile / a.num_n_blk;
    n_blk = tile - m_blk * a.num_n_blk;
  } else {
    n_blk = tile / a.num_m_blk;
    m_blk = tile - n_blk * a.num_m_blk;
  }
}

// PAIR: the CTA is one of a cluster of two that share a 256 x BN tile on both SMs' tensor cores (tcgen05
// cta_group::2). Each CTA loads its own 128 rows of x and its half of the BN weight rows; the leader (rank 0) issues
// the MMAs, whose commits arrive on both CTAs' barriers; each CTA's epilogue drains its own 128 accumulator rows.
// Per SM that is 16 KB + BN/2 x 128 B of operands per K block instead of 16 KB + BN x 128 B.
template <int BN, int STAGES, int MODE, bool PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                             const __grid_constant__ CUtensorMap tm_out, const GemmArgs args) {
  using L = GemmLayout<BN, STAGES, PAIR ? BN / 2 : BN>;
  constexpr bool GEGLU = MODE == kModeGeglu;
  static_assert(!PAIR || (BN % 32 == 0 && BN >= 64), "a pair splits the weight rows of a tile in two 16-row multiples");
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // CTA rank in the pair (0 = leader)
  constexpr int kTileM = PAIR ? 2 * kGemmBM : kGemmBM;  // output rows per tile
  // Stage `stage`'s full barrier as the TMA completion target: the leader's, for both CTAs of a pair.
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* full = bars;
  auto tma2 = [&](const CUtensorMap* map, int stage, uint8_t* dst, int x, int y) {
    if constexpr (PAIR)
      tma_load_2d_pair(map, cluster_smem_addr(&full[stage], 0), dst, x, y);
    else
      tma_load_2d(map, &full[stage], dst, x, y);
  };
  // A tile of K block kb for the output rows from m0: a 2-D box of x, or in the convolution form the input patch
  // of tap kb / cblocks (kh, kw) and channel block kb % cblocks, shifted by (kh - 1, kw - 1).
  auto load_x = [&](int stage, uint8_t* dst, int kb, int m0) {
    if constexpr (MODE == kModeConv3x3) {
      const int tap = kb / args.cv_cblocks;
      const int cb = kb - tap * args.cv_cblocks;
      const int kh = tap / 3;
      const int kw = tap - 3 * kh;
      const int img = m0 / args.cv_hw;
      const int h0 = (m0 - img * args.cv_hw) / args.cv_w;
      if constexpr (PAIR)
        tma_load_4d_pair(&tm_x, cluster_smem_addr(&full[stage], 0), dst, cb * kGemmBK, kw - 1, h0 + kh - 1, img);
      else
        tma_load_4d(&tm_x, &full[stage], dst, cb * kGemmBK, kw - 1, h0 + kh - 1, img);
    } else {
      tma2(&tm_x, stage, dst, kb * kGemmBK, m0);
    }
  };
  // Output columns per tile: BN, or BN/2 gated columns in the GEGLU form (a then gate rows of W in the B tile).
  constexpr int kOutCols = GEGLU ? BN / 2 : BN;
  static_assert(!GEGLU || (BN % 64 == 0), "GEGLU tiles hold two halves of a multiple of 32 columns");
  // W tile of stage i for the output-column block nb: one box of BN rows, or BN/2 a-rows then BN/2 gate-rows. In a
  // pair each CTA holds one half: rows [nb*BN + rank*BN/2, +BN/2), or in the GEGLU form the a-rows (leader) or the
  // gate rows (second CTA).
  auto load_w = [&](int stage, uint8_t* dst, int kb, int nb) {
    if constexpr (PAIR) {
      const int row0 = GEGLU ? (rank == 0 ? nb * kOutCols : args.N + nb * kOutCols) : nb * BN + int(rank) * (BN / 2);
      tma2(&tm_w, stage, dst, kb * kGemmBK, row0);
    } else if constexpr (GEGLU) {
      tma2(&tm_w, stage, dst, kb * kGemmBK, nb * kOutCols);
      tma2(&tm_w, stage, dst + kOutCols * 128, kb * kGemmBK, args.N + nb * kOutCols);
    } else {
      tma2(&tm_w, stage, dst, kb * kGemmBK, nb * BN);
    }
  };
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * L::kABytes;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* bias_full = drain + 1;  // the epilogue warps have written this tile's bias table
  uint64_t* bias_free = drain + 2;  // the epilogue warps are done reading the previous tile's table
  uint64_t* parts_ready = drain + 3;  // split K: every CTA of the cluster has parked its partial tile
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
      mbar_init(&acc_empty[a], PAIR ? 2 * kGemmEpiWarps : kGemmEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    mbar_init(bias_full, kGemmEpiThreads);  // one arrival per epilogue thread
    mbar_init(bias_free, kGemmEpiThreads);
    mbar_init(parts_ready, uint32_t(args.splits));  // one arrival from each CTA of a split-K cluster
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, L::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, L::kTmemCols);
      tmem_relinquish();
    }
    tc_fence_before();
  }
  // A pair's (or split-K cluster's) barriers must be initialised in every CTA before another CTA's copies, commits
  // or arrivals reach them.
  const bool clustered = PAIR || (!GEGLU && args.splits > 1);  // the GEGLU form never splits K
  if (clustered)
    cluster_sync();
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Let the next kernel on the stream start its prologue on idle SMs; it waits for this grid before reading.
  pdl_launch_dependents();

  const int num_units = args.num_tiles * args.splits;
  // Work units go round the persistent grid; a pair (two consecutive CTAs of a cluster) takes each unit together.
  const int unit0 = PAIR ? int(blockIdx.x) / 2 : int(blockIdx.x);
  const int unit_stride = PAIR ? int(gridDim.x) / 2 : int(gridDim.x);
  // Bytes a stage's full barrier (the leader's, in a pair) expects: both CTAs' tiles in a pair.
  constexpr uint32_t kFullBytes = PAIR ? 2u * L::kStageBytes : uint32_t(L::kStageBytes);
  const int num_kb = args.num_kb;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      // The weight never depends on the previous kernel on the stream: the first stages' W tiles are requested
      // before waiting on it (programmatic dependent launch), so their fetch overlaps that kernel's tail.
      int pre = 0;
      if (unit0 < num_units) {
        int mb, nb;
        tile_coords(args, unit0 / args.splits, mb, nb);
        const int kb0 = (unit0 % args.splits) * args.kb_per_split;
        pre = min(STAGES, min(num_kb, kb0 + args.kb_per_split) - kb0);
        for (int i = 0; i < pre; ++i) {
          if (rank == 0) mbar_arrive_expect_tx(&full[i], kFullBytes);
          load_w(i, sB + i * L::kBBytes, kb0 + i, nb);
        }
      }
      pdl_wait();  // x may be the previous kernel's output
      for (int unit = unit0; ok && unit < num_units; unit += unit_stride) {
        const int tile = unit / args.splits;
        int mb, nb;
        tile_coords(args, tile, mb, nb);
        const int m0 = mb * kTileM + int(rank) * kGemmBM;
        const int kb_begin = (unit % args.splits) * args.kb_per_split;
        const int kb_end = min(num_kb, kb_begin + args.kb_per_split);
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (pre > 0) {
            // stage already armed and its W tile in flight (first stages of the first unit)
            load_x(stage, sA + stage * L::kABytes, kb, m0);
            --pre;
          } else {
            if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, args.ctl, kStatusTimeoutProducer)) {
              ok = false;
              break;
            }
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], kFullBytes);
            load_x(stage, sA + stage * L::kABytes, kb, m0);
            load_w(stage, sB + stage * L::kBBytes, kb, nb);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (PAIR && ok) {
        // Wait until the leader's MMAs have released every stage: their commits arrive on this CTA's barriers, which
        // must outlive them.
        for (int i = 0; i < STAGES; ++i) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, args.ctl, kStatusTimeoutProducer)) break;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && rank == 0) {
        // Abort: let the (at most STAGES) loads still in flight land before the CTA's shared memory goes away (in a
        // pair the leader's full barriers count both CTAs' loads).
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
    // The whole warp runs the loop (operands stay warp-uniform, which keeps tcgen05.mma issue at the tensor core's
    // pace); one elected lane issues the MMAs and their commits. In a pair only the leader issues: its MMAs read
    // both CTAs' stages and write both CTAs' accumulators, and its commits arrive on both CTAs' barriers.
    constexpr uint32_t kIdesc = idesc_bf16_f32(kTileM, BN, false);
    constexpr uint16_t kBoth = 3;  // commit multicast mask: both CTAs of the pair
    auto mma = [&](uint32_t d, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate) {
      if constexpr (PAIR)
        umma_f16_ss_pair(d, a_desc, b_desc, kIdesc, accumulate);
      else
        umma_f16_ss(d, a_desc, b_desc, kIdesc, accumulate);
    };
    auto commit = [&](uint64_t* bar, uint16_t mask) {
      if constexpr (PAIR)
        umma_commit_pair(bar, mask);
      else
        umma_commit(bar);
    };
    if (!PAIR || rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      if (args.ctl.debug & 1u) {
        // Test hook: wait on a barrier nothing arrives on, so the bounded wait expires and the abort path runs.
        if (!mbar_wait_bounded_warp(drain, 0, abort_flag, args.ctl, kStatusForced)) ok = false;
      }
      int local = 0;
      for (int unit = unit0; ok && unit < num_units; unit += unit_stride, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded_warp(&acc_empty[acc], acc_phase ^ 1u, abort_flag, args.ctl, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        const int kb_begin = (unit % args.splits) * args.kb_per_split;
        const int kb_end = min(num_kb, kb_begin + args.kb_per_split);
        for (int kb = kb_begin; kb < kb_end; ++kb) {
          if (!mbar_wait_bounded_warp(&full[stage], phase, abort_flag, args.ctl, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a_desc = smem_desc_kmajor_sw128(smem_u32(sA + stage * L::kABytes));
          const uint64_t b_desc = smem_desc_kmajor_sw128(smem_u32(sB + stage * L::kBBytes));
          if (elect_one()) {
#pragma unroll
            for (int k = 0; k < kGemmBK / 16; ++k) {
              // +32 bytes per K step of 16 bf16 inside the swizzle atom (descriptor address field is >> 4).
              mma(d_tmem, a_desc + 2u * k, b_desc + 2u * k, (kb > kb_begin || k > 0) ? 1u : 0u);
            }
            commit(&empty[stage], kBoth);  // frees the smem stage (in both CTAs) once these MMAs have read it
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elect_one()) commit(&acc_full[acc], kBoth);  // accumulator complete
        __syncwarp();
      }
      if (PAIR && ok) {
        // Wait until both CTAs' epilogues have released the last two accumulators: the second CTA's releases are
        // arrivals on this CTA's barriers, which must outlive them.
        for (int i = 0; i < 2; ++i, ++local) {
          if (!mbar_wait_bounded_warp(&acc_empty[local & 1], ((local >> 1) & 1) ^ 1u, abort_flag, args.ctl,
                                      kStatusTimeoutMma))
            break;
        }
      }
      if (!ok) {
        // Abort: wait until every MMA this warp issued has finished before TMEM is released.
        if (elect_one()) commit(drain, 1);
        __syncwarp();
        mbar_wait_drain(drain, 0u, args.ctl);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..9)
    const int quarter = warp & 3;  // TMEM lanes this warp may access: [32*quarter, 32*quarter + 32)
    const int half = (warp - 2) >> 2;  // which of the quarter's two warps: output chunks half, half + 2, ...
    const int row = quarter * 32 + lane;
    // Output goes out in chunks of 128-byte rows (64 bf16 or 32 f32 columns) through a staging tile per warp,
    // laid out with the 128-byte swizzle so the row-per-thread writes hit distinct banks; the quarter's two warps
    // alternate chunks. A chunk that would reach past the tile (BN not a multiple of the chunk) is written with
    // direct stores instead.
    uint8_t* sb = smem + L::kStagingOffset + (warp - 2) * (32 * 128);
    const int cw = args.out_f32 ? 32 : 64;
    const int splits = args.splits;
    int local = 0;
    // One bias row for the whole output: read from a per-tile table in shared memory. A bias row per image is read
    // by each thread for its own row.
    const bool table_bias = args.bias != nullptr && args.bias_img_stride == 0;
    float* bias_tab = reinterpret_cast<float*>(smem + L::kBiasOffset);
    pdl_wait();  // the previous kernel may still read (or write) the output / bias
    for (int unit = unit0; unit < num_units; unit += unit_stride, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (args.bias != nullptr && warp == 2) {
        // Pull this tile's bias into L2 while the main loop runs (one 128-byte line per lane).
        int pmb, pnb;
        tile_coords(args, unit / splits, pmb, pnb);
        const int esz = args.bias_f32 ? 4 : 2;
        const int bytes = min(kOutCols, args.N - pnb * kOutCols) * esz;
        if (lane * 128 < bytes)
          prefetch_l2(static_cast<const uint8_t*>(args.bias) + size_t(pnb) * kOutCols * esz + lane * 128);
        if (GEGLU && lane * 128 < bytes)
          prefetch_l2(static_cast<const uint8_t*>(args.bias) + (size_t(args.N) + size_t(pnb) * kOutCols) * esz +
                      lane * 128);
      }
      const int tile = unit / splits;
      const int split = unit % splits;
      int mb, nb;
      tile_coords(args, tile, mb, nb);
      const int m0 = mb * kTileM + int(rank) * kGemmBM;  // this CTA's 128 rows of the tile
      const int n0 = nb * kOutCols;
      if (table_bias) {
        // This tile's bias table: each epilogue thread fetches up to two entries (requested before any wait),
        // stores them once every warp is done with the previous tile's table, then all wait for the full table.
        static_assert(BN <= kGemmEpiThreads, "one bias table entry per epilogue thread");
        const int i = int(threadIdx.x) - 64;
        const int col = i < kOutCols ? n0 + i : args.N + n0 + (i - kOutCols);
        const float e = (i < BN && col < args.bias_n)
                            ? (args.bias_f32 ? __ldg(static_cast<const float*>(args.bias) + col)
                                             : __bfloat162float(static_cast<const __nv_bfloat16*>(args.bias)[col]))
                            : 0.0f;
        if (local > 0 &&
            !mbar_wait_bounded(bias_free, uint32_t(local - 1) & 1u, abort_flag, args.ctl, kStatusTimeoutEpilogue))
          break;
        if (i < BN) bias_tab[i] = e;
        mbar_arrive(bias_full);
        if (!mbar_wait_bounded(bias_full, uint32_t(local) & 1u, abort_flag, args.ctl, kStatusTimeoutEpilogue)) break;
      }
      if (!mbar_wait_bounded(&acc_full[acc], acc_phase, abort_flag, args.ctl, kStatusTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (uint32_t(quarter * 32) << 16) + uint32_t(acc * BN);
      if (!GEGLU && splits > 1) {
        // Split K over the CTAs of this cluster (one per split, launched together): park this split's partial tile
        // in shared memory ([row][BN + 4] f32; the operand ring is idle once the accumulator is complete, and a
        // split-K CTA has no further unit), tell every CTA of the cluster, wait for all of them, then sum this CTA's
        // slice of rows over every CTA's partial in split order through distributed shared memory and store it.
        constexpr int kPS = BN + 4;
        float* part = reinterpret_cast<float*>(smem);
#pragma unroll 1
        for (int c = half * 32; c < BN; c += 64) {
          uint32_t r[32];
          tmem_ld32(t_row + uint32_t(c), r);
          tmem_wait_ld();
          float4* dst = reinterpret_cast<float4*>(part + row * kPS + c);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                 __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
        }
        named_barrier_sync(1, kGemmEpiThreads);
        if (threadIdx.x == 64) {
          fence_acq_rel_cluster();
          for (int s2 = 0; s2 < splits; ++s2) mbar_arrive_cluster(cluster_smem_addr(parts_ready, uint32_t(s2)));
        }
        if (!mbar_wait_cluster_bounded(parts_ready, 0u, abort_flag, args.ctl, kStatusTimeoutEpilogue)) break;
        const int r0 = (kGemmBM * split) / splits;
        const int r1 = (kGemmBM * (split + 1)) / splits;
        const int items = (r1 - r0) * (BN / 4);
#pragma unroll 1
        for (int it = int(threadIdx.x) - 64; it < items; it += kGemmEpiThreads) {
          const int rr = r0 + it / (BN / 4);
          const int cc = (it % (BN / 4)) * 4;
          const float* mine = part + rr * kPS + cc;
          float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
          for (int s2 = 0; s2 < splits; ++s2) {
            const float4 p4 = ld_cluster_f32x4(cluster_smem_addr(mine, uint32_t(s2)));
            v[0] += p4.x;
            v[1] += p4.y;
            v[2] += p4.z;
            v[3] += p4.w;
          }
          const int grow = m0 + rr;
          const int gcol = n0 + cc;
          if (grow >= args.M || gcol >= args.N) continue;
          const long long own =
              args.bias_img_stride > 0
                  ? (long long)min(grow / args.bias_img_pixels, args.bias_imgs - 1) * args.bias_img_stride
                  : 0;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float b = 0.f;
            if (table_bias)
              b = bias_tab[cc + j];
            else
              b = load_bias_own(args, gcol, j, own);
            v[j] += b;
            if (args.residual != nullptr && gcol + j < args.N)
              v[j] += __bfloat162float(static_cast<const __nv_bfloat16*>(args.residual)[(long long)grow * args.ldr +
                                                                                          gcol + j]);
          }
          if (args.out_f32) {
            float* o = static_cast<float*>(args.out) + (long long)grow * args.ldo + gcol;
            if (gcol + 4 <= args.N && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
              *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (gcol + j < args.N) o[j] = v[j];
            }
          } else {
            __nv_bfloat16* o = static_cast<__nv_bfloat16*>(args.out) + (long long)grow * args.ldo + gcol;
            if (gcol + 4 <= args.N && (reinterpret_cast<uintptr_t>(o) & 7) == 0) {
              *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (gcol + j < args.N) o[j] = __float2bfloat16_rn(v[j]);
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c0 = half * cw; c0 < kOutCols; c0 += 2 * cw) {
          const bool chunk_tma = args.tma_store && c0 + cw <= kOutCols;
          // This warp's previous TMA store must have read the staging tile before the first staging write of this
          // chunk; waiting only there lets that read overlap this chunk's TMEM loads and arithmetic.
          bool staged = false;
          auto stage_wait = [&]() {
            if (!staged) {
              if (lane == 0) bulk_wait_read<0>();
              __syncwarp();
              staged = true;
            }
          };
          // The chunk's 32-column groups: both TMEM loads of a 64-column chunk are issued before one wait.
          uint32_t racc[2][32];
          if constexpr (!GEGLU) {
            tmem_ld32(t_row + uint32_t(c0), racc[0]);
            if (c0 + 32 < min(c0 + cw, kOutCols)) tmem_ld32(t_row + uint32_t(c0 + 32), racc[1]);
            tmem_wait_ld();
          }
#pragma unroll
          for (int sub = 0; sub < 2; ++sub) {
            const int c = c0 + 32 * sub;
            if (c >= min(c0 + cw, kOutCols)) break;
            // Bias of the 32 columns from column offset `off` of the tile (the table) or of the output (own row).
            auto fetch_bias = [&](float (&bb)[32], int off, int gcol) {
              if (table_bias) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const float4 t4 = reinterpret_cast<const float4*>(bias_tab + off)[j];
                  bb[4 * j] = t4.x;
                  bb[4 * j + 1] = t4.y;
                  bb[4 * j + 2] = t4.z;
                  bb[4 * j + 3] = t4.w;
                }
              } else {
                long long bias_row = 0;
                if (args.bias_img_stride > 0)
                  bias_row =
                      (long long)min((m0 + row) / args.bias_img_pixels, args.bias_imgs - 1) * args.bias_img_stride;
                load_bias32(args, gcol, bb, bias_row);
              }
            };
            float v[32];
            if constexpr (GEGLU) {
              // The GEGLU form has one bias row (or none): its table holds the a-columns' then the gate columns'.
              uint32_t r[32], rg[32];
              tmem_ld32(t_row + uint32_t(c), r);
              tmem_ld32(t_row + uint32_t(kOutCols + c), rg);
              tmem_wait_ld();
#pragma unroll
              for (int j4 = 0; j4 < 8; ++j4) {
                const float4 b4 = table_bias ? reinterpret_cast<const float4*>(bias_tab + c)[j4]
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
                const float4 g4 = table_bias ? reinterpret_cast<const float4*>(bias_tab + kOutCols + c)[j4]
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
                const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
                const float gg[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int j = 4 * j4 + e;
                  v[j] = (__uint_as_float(r[j]) + bb[e]) * gelu_erf(__uint_as_float(rg[j]) + gg[e]);
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(racc[sub][j]);
              float b[32];
              fetch_bias(b, c, n0 + c);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += b[j];
              if (args.residual != nullptr) add_residual32(args, m0 + row, n0 + c, v);
            }
            if (chunk_tma) {
              stage_wait();
              uint8_t* rowp = sb + lane * 128;
              if (args.out_f32) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const int phys = j ^ (lane & 7);
                  *reinterpret_cast<float4*>(rowp + phys * 16) =
                      make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                }
              } else {
                const int chunk0 = ((c - c0) * 2) / 16;  // 16-byte chunk index of this column group in the row
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  uint4 t;
                  t.x = pack_bf16x2(v[8 * j], v[8 * j + 1]);
                  t.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
                  t.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
                  t.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
                  const int phys = (chunk0 + j) ^ (lane & 7);
                  *reinterpret_cast<uint4*>(rowp + phys * 16) = t;
                }
              }
            } else {
              store_row32_direct(args, m0 + row, n0 + c, v);
            }
          }
          if (chunk_tma) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && n0 + c0 < args.N && m0 + quarter * 32 < args.M) {
              tma_store_2d(&tm_out, sb, n0 + c0, m0 + quarter * 32);
              bulk_commit();
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          mbar_arrive_cluster(cluster_smem_addr(&acc_empty[acc], 0));  // the leader's MMA waits on it
        else
          mbar_arrive(&acc_empty[acc]);
      }
      if (table_bias) mbar_arrive(bias_free);
    }
    if (args.tma_store && lane == 0) bulk_wait_read<0>();  // staging must not be released while being read
  }

  // Nothing of a CTA of a pair or split-K cluster (its barriers, its parked partial) may go while another CTA of the
  // cluster can still reach it.
  if (clustered)
    cluster_sync();
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, L::kTmemCols);
    else
      tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------------------------
namespace {

// Launch one instantiation over `units` work units: a persistent grid of one CTA per SM; for a pair variant one
// two-CTA cluster per SM pair (as many as can be resident at once, from the occupancy query); for split K one
// cluster of `splits` CTAs per output tile, one unit per CTA.
template <int BN, int STAGES, int MODE = kModePlain, bool PAIR = false>
int launch_variant(const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& mo, const GemmArgs& args,
                   int64_t units, int sms, cudaStream_t st, int device) {
  using L = GemmLayout<BN, STAGES, PAIR ? BN / 2 : BN>;
  static bool configured[64] = {false};
  static int resident_clusters[64][kGemmMaxSplits + 1] = {};
  auto kern = gemm_bf16_tcgen05_kernel<BN, STAGES, MODE, PAIR>;
  if (device < 0 || device >= 64) return fail(kErrInvalid, "device ordinal %d out of range", device);
  const int cluster = PAIR ? 2 : args.splits;
  if (cluster < 1 || cluster > kGemmMaxSplits) return fail(kErrInvalid, "GEMM cluster of %d CTAs", cluster);
  if (PAIR && args.splits != 1) return fail(kErrInvalid, "paired GEMM tiles do not split K");
  if (!configured[device]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(gemm smem)");
    configured[device] = true;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = unsigned(cluster);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster > 1 ? 2 : 1;
  int64_t grid = std::min<int64_t>(units, sms);
  if (cluster > 1) {
    int& resident = resident_clusters[device][cluster];
    if (resident == 0) {
      cfg.gridDim = dim3(unsigned(cluster * (sms / cluster)));
      int n = 0;
      cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess) return check_cuda(e, "cudaOccupancyMaxActiveClusters(gemm)");
      if (n < 1) return fail(kErrUnsupported, "no %d-CTA cluster of the GEMM fits on this device", cluster);
      resident = n;
    }
    // Pairs: persistent over units. Split K: every unit gets its own CTA (the clusters beyond the resident ones
    // start as others finish).
    grid = PAIR ? 2 * std::min<int64_t>(units, resident) : units;
  }
  if (grid > INT32_MAX) return fail(kErrInvalid, "GEMM grid too large");
  cfg.gridDim = dim3(unsigned(grid));
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, mx, mw, mo, args), "gemm kernel launch");
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

// Output map for the TMA-store epilogue: boxes of 32 rows x 128 bytes (64 bf16 or 32 f32), 128-byte swizzle.
int encode_out_map(void* out, int64_t M, int64_t N, int64_t ldo, bool f32, CUtensorMap* map) {
  EncodeTiledFn enc = nullptr;
  if (int rc = encode_tiled_fn(&enc)) return rc;
  const int esz = f32 ? 4 : 2;
  cuuint64_t dims[2] = {cuuint64_t(N), cuuint64_t(M)};
  cuuint64_t strides[1] = {cuuint64_t(ldo) * esz};
  cuuint32_t box[2] = {cuuint32_t(128 / esz), 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrInvalid;
}

constexpr int kTileChoices[] = {64, 96, 128, 160, 192, 256};

}  // namespace

namespace {

// Modelled time (SM clocks) of a plan: waves of persistent work units x per-unit time. A unit's main loop is
// bounded by the larger of the tensor-core time (2*BN clocks per 64-deep K block at 8192 FLOP/clk/SM) and the
// time to stream its operands into shared memory (~64 B/clk/SM); each unit pays a fixed pipeline fill. A split
// tile pays for parking its f32 partial in shared memory, the cluster hand-off, and its slice of the reduction
// over the cluster's partials (distributed shared memory).
double plan_cost(int64_t M, int64_t N, int64_t kb, int bn, int splits, int sms) {
  const int64_t tiles = ((M + kGemmBM - 1) / kGemmBM) * ((N + bn - 1) / bn);
  const int64_t units = tiles * splits;
  const int64_t waves = (units + sms - 1) / sms;
  const int64_t kb_unit = (kb + splits - 1) / splits;
  const double mma = 2.0 * bn;
  const double load = (kGemmBM + bn) * 128.0 / 64.0;
  double t = double(kb_unit) * std::max(mma, load) + 1500.0 + 8.0 * bn;
  if (splits > 1) t += 4000.0 + 12.0 * bn + 150.0 * splits;
  return double(waves) * t;
}
}  // namespace

namespace {
// Modelled time of a paired plan: tiles of 256 x BN rows x columns, one per two-CTA cluster (about sms / 2
// resident). Per SM the tensor core does the same work per K block as for a one-CTA BN tile while only half of B
// arrives in its shared memory; measured on B200 that makes the main loop about 8% faster for BN = 256 (less for
// narrower tiles, which never won), against about 1 us more per launch (cluster launch, the pair's hand-offs and
// teardown), so pairs pay only for long-running wide tiles.
double plan_cost_pair(int64_t M, int64_t N, int64_t kb, int bn, int sms) {
  const int64_t tiles = ((M + 2 * kGemmBM - 1) / (2 * kGemmBM)) * ((N + bn - 1) / bn);
  const int64_t clusters = std::max(1, sms / 2);
  const int64_t waves = (tiles + clusters - 1) / clusters;
  const double mma = 2.0 * bn;
  const double load = (kGemmBM + bn) * 128.0 / 64.0;
  return double(waves) * (0.92 * double(kb) * std::max(mma, load) + 1500.0 + 8.0 * bn) + 2000.0;
}

bool pair_tile(int bn) { return bn == 128 || bn == 192 || bn == 256; }

}  // namespace

bool gemm_variant_known(int variant, bool geglu) {
  const bool pair = variant >= kGemmPairVariant;
  const int bn = pair ? variant - kGemmPairVariant : variant;
  bool known = false;
  for (int c : kTileChoices) known |= (c == bn);
  return known && (!pair || pair_tile(bn)) && (!geglu || bn % 64 == 0);
}

int gemm_cluster_slots(int size) {
  // Filled once per (device, cluster size) under a lock: planning runs on any host thread.
  static std::mutex fill_mutex;
  static int slots[64][kGemmMaxSplits + 1] = {};
  if (size < 2 || size > kGemmMaxSplits) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(fill_mutex);
  if (slots[dev][size] == 0) {
    // Every GEMM instantiation holds one CTA per SM (more than half of the shared memory), so one stands for all.
    using L = GemmLayout<64, 8>;
    auto kern = gemm_bf16_tcgen05_kernel<64, 8, kModePlain, false>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes) != cudaSuccess)
      return 0;
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = L::kSmemBytes;
    cfg.gridDim = dim3(unsigned(size * 16));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(size);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      (void)cudaGetLastError();
      return 0;
    }
    slots[dev][size] = n > 0 ? n : -1;
  }
  return std::max(slots[dev][size], 0);
}

GemmPlan gemm_plan(int64_t M, int64_t N, int64_t K, int sms, int variant, bool geglu, bool auto_pair) {
  // N counts accumulator columns: for the GEGLU form the 2 x inner projection columns, and only tiles with an even
  // split into a and gate halves of 32-column multiples are candidates. `variant` (when not 0) forces one tile:
  // BN, or kGemmPairVariant + BN for the paired form.
  const int64_t kb = (K + kGemmBK - 1) / kGemmBK;
  GemmPlan best{128, 1, int(kb), 0, false};
  double best_cost = 1e300;
  for (int bn : kTileChoices) {
    if (variant && bn != variant) continue;
    if (geglu && bn % 64 != 0) continue;
    const int64_t tiles = ((M + kGemmBM - 1) / kGemmBM) * ((N + bn - 1) / bn);
    // Split K only when the tiles leave most SMs idle and each split keeps >= 4 K blocks (never for GEGLU, whose
    // gating needs the finished sums).
    int max_split = 1;
    if (!geglu && tiles * 2 <= sms && kb >= 8)
      max_split = int(std::min<int64_t>(std::min<int64_t>(sms / tiles, kb / 4), kGemmMaxSplits));
    for (int sp = 1; sp <= max_split; ++sp) {
      const int kps = int((kb + sp - 1) / sp);
      const int eff = int((kb + kps - 1) / kps);  // splits actually needed with kps blocks each
      if (eff != sp) continue;
      // A split plan runs as tiles clusters of sp CTAs; clusters are placed within a GPC, so only as many as
      // gemm_cluster_slots(sp) run at once. Plans needing a second wave of clusters are not taken.
      if (sp > 1 && tiles > gemm_cluster_slots(sp)) continue;
      const double cost = plan_cost(M, N, kb, bn, sp, sms);
      if (cost < best_cost * 0.999 || (cost <= best_cost * 1.001 && bn > best.bn && sp <= best.splits)) {
        best_cost = cost;
        best.bn = bn;
        best.splits = sp;
        best.kb_per_split = kps;
        best.split_ws_bytes = 0;  // split K reduces through distributed shared memory: no workspace
      }
    }
  }
  // Paired tiles (never with split K): automatically only 192- and 256-column tiles over at least 12 K blocks
  // outside the GEGLU form (shorter tiles are bound by their epilogue, which the pair does not speed up), when the
  // output has at least two 128-row blocks, and only where the cost model prefers them; any pair tile when forced.
  // (192-column pairs from 12 K blocks: the SD1.5 sweep's M = 1024 group 124.9 -> 122.9 us, UNet steps level.)
  for (int bn : kTileChoices) {
    if (!pair_tile(bn) || (geglu && bn % 64 != 0) || M <= kGemmBM) continue;
    if (variant ? variant != kGemmPairVariant + bn : (!auto_pair || bn < 192 || geglu || kb < 12)) continue;
    const double cost = plan_cost_pair(M, N, kb, bn, sms);
    if (variant || cost < best_cost * 0.999) {
      best_cost = cost;
      best = GemmPlan{bn, 1, int(kb), 0, true};
    }
  }
  return best;
}

int gemm_encode_b_map(const void* w, int64_t ldw, int64_t N, int64_t K, int box_rows, CUtensorMap* out) {
  return encode_kmajor_map(w, N, K, ldw, box_rows, out);
}

int gemm_launch(const GemmProblem& p, cudaStream_t stream) {
  const DeviceInfo* dev = nullptr;
  if (int rc = current_device_info(&dev)) return rc;
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return fail(kErrInvalid, "GEMM sizes must be positive (M=%lld N=%lld K=%lld)",
                                                    (long long)p.M, (long long)p.N, (long long)p.K);
  if (p.M > INT32_MAX / 2 || p.N > INT32_MAX / 2 || p.K > INT32_MAX / 2)
    return fail(kErrInvalid, "GEMM dimension too large");
  const bool geglu = p.geglu != 0;
  if (p.variant && !gemm_variant_known(p.variant, geglu))
    return fail(kErrUnsupported, "no GEMM%s variant %d", geglu ? " (GEGLU)" : "", p.variant);
  if (geglu && p.w_map_cache != nullptr) return fail(kErrInvalid, "the GEGLU form encodes its own weight map");
  GemmPlan plan = gemm_plan(p.M, geglu ? 2 * p.N : p.N, p.K, dev->sms, p.variant, geglu);
  const int bn = plan.bn;
  const int out_cols = geglu ? bn / 2 : bn;  // output columns per tile

  CUtensorMap mx, mw;
  if (int rc = encode_kmajor_map(p.x, p.M, p.K, p.ldx, kGemmBM, &mx)) return rc;
  if (p.w_map_cache != nullptr) {
    mw = *p.w_map_cache;  // encoded with gemm_plan_box_rows(plan) rows per box
  } else if (int rc = encode_kmajor_map(p.w, geglu ? 2 * p.N : p.N, p.K, p.ldw, gemm_plan_box_rows(plan, geglu),
                                        &mw)) {
    return rc;
  }

  // TMA-store epilogue when the output rows are 16-byte aligned; otherwise direct predicated stores.
  CUtensorMap mo;
  memset(&mo, 0, sizeof(mo));
  const int esz = p.out_f32 ? 4 : 2;
  bool tma_store = (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 && (p.ldo * esz) % 16 == 0;
  if (tma_store && encode_out_map(p.out, p.M, p.N, p.ldo, p.out_f32 != 0, &mo) != kOk) tma_store = false;

  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.tma_store = tma_store ? 1 : 0;
  a.M = int(p.M);
  a.N = int(p.N);
  a.K = int(p.K);
  const int tile_m = plan.pair ? 2 * kGemmBM : kGemmBM;
  a.num_m_blk = int((p.M + tile_m - 1) / tile_m);
  const int num_n = int((p.N + out_cols - 1) / out_cols);
  a.num_n_blk = num_n;
  // Raster: keep the larger operand's tiles in L2 while the smaller one streams past them.
  a.n_fastest = (p.M >= p.N) ? 1 : 0;
  const int64_t tiles = int64_t(a.num_m_blk) * num_n;
  if (tiles > INT32_MAX) return fail(kErrInvalid, "GEMM has too many tiles");
  a.num_tiles = int(tiles);
  a.num_kb = int((p.K + kGemmBK - 1) / kGemmBK);
  a.bias = p.bias;
  a.bias_f32 = p.bias_f32;
  a.bias_n = int(geglu ? 2 * p.N : p.N);
  a.residual = geglu ? nullptr : p.residual;
  a.ldr = p.ldr;
  a.out = p.out;
  a.ldo = p.ldo;
  a.out_f32 = p.out_f32;
  a.splits = plan.splits;
  a.kb_per_split = plan.kb_per_split;
  a.ctl.status = dev->status;
  a.ctl.timeout_ns = wait_timeout_ns();
  a.ctl.debug = p.debug;
  const int64_t units = tiles * plan.splits;
  const int sms = dev->sms;
  const int d = dev->device;

  if (plan.pair) {
    if (geglu) {
      switch (bn) {
        case 128: return launch_variant<128, 8, kModeGeglu, true>(mx, mw, mo, a, units, sms, stream, d);
        case 192: return launch_variant<192, 6, kModeGeglu, true>(mx, mw, mo, a, units, sms, stream, d);
        case 256: return launch_variant<256, 6, kModeGeglu, true>(mx, mw, mo, a, units, sms, stream, d);
      }
    } else {
      switch (bn) {
        case 128: return launch_variant<128, 8, kModePlain, true>(mx, mw, mo, a, units, sms, stream, d);
        case 192: return launch_variant<192, 6, kModePlain, true>(mx, mw, mo, a, units, sms, stream, d);
        case 256: return launch_variant<256, 6, kModePlain, true>(mx, mw, mo, a, units, sms, stream, d);
      }
    }
    return fail(kErrUnsupported, "no paired GEMM variant with an N tile of %d", bn);
  }
  if (geglu) {
    switch (bn) {
      case 64: return launch_variant<64, 8, kModeGeglu>(mx, mw, mo, a, units, sms, stream, d);
      case 128: return launch_variant<128, 6, kModeGeglu>(mx, mw, mo, a, units, sms, stream, d);
      case 192: return launch_variant<192, 4, kModeGeglu>(mx, mw, mo, a, units, sms, stream, d);
      case 256: return launch_variant<256, 4, kModeGeglu>(mx, mw, mo, a, units, sms, stream, d);
    }
    return fail(kErrUnsupported, "no GEGLU GEMM variant with an N tile of %d", bn);
  }
  switch (bn) {
    case 64: return launch_variant<64, 8>(mx, mw, mo, a, units, sms, stream, d);
    case 96: return launch_variant<96, 6>(mx, mw, mo, a, units, sms, stream, d);
    case 128: return launch_variant<128, 6>(mx, mw, mo, a, units, sms, stream, d);
    case 160: return launch_variant<160, 5>(mx, mw, mo, a, units, sms, stream, d);
    case 192: return launch_variant<192, 4>(mx, mw, mo, a, units, sms, stream, d);
    case 256: return launch_variant<256, 4>(mx, mw, mo, a, units, sms, stream, d);
  }
  return fail(kErrUnsupported, "no GEMM variant with an N tile of %d", bn);
}

// ---------------------------------------------------------------------------------------------------------------
// 3x3 convolution (implicit GEMM, the kernel's convolution form)
// ---------------------------------------------------------------------------------------------------------------
int conv3x3_launch(const ConvProblem& p, cudaStream_t stream) {
  const DeviceInfo* dev = nullptr;
  if (int rc = current_device_info(&dev)) return rc;
  if (p.x == nullptr || p.wt == nullptr || p.out == nullptr) return fail(kErrInvalid, "conv3x3: null pointer");
  if (p.n <= 0 || p.h <= 0 || p.w <= 0 || p.cin <= 0 || p.cout <= 0)
    return fail(kErrInvalid, "conv3x3 sizes must be positive");
  if (p.cin % kGemmBK != 0)
    return fail(kErrUnsupported, "conv3x3 needs input channels in multiples of 64 (got %lld)", (long long)p.cin);
  // A tile is 128 output pixels made of whole image rows (and whole images when an image has fewer than 128).
  if (p.w > 128 || 128 % p.w != 0)
    return fail(kErrUnsupported, "conv3x3 needs an image width dividing 128 (got %lld)", (long long)p.w);
  const int64_t th = std::min<int64_t>(p.h, 128 / p.w);
  if (p.h % th != 0)
    return fail(kErrUnsupported, "conv3x3: image height %lld is not a multiple of %lld rows", (long long)p.h,
                (long long)th);
  const int64_t imgs = 128 / (th * p.w);
  if (th * p.w * imgs != 128)
    return fail(kErrUnsupported, "conv3x3: %lld x %lld images do not tile 128 pixels", (long long)p.h, (long long)p.w);
  const int64_t M = p.n * p.h * p.w, K = 9 * p.cin;
  if (M > INT32_MAX / 2 || K > INT32_MAX / 2 || p.cout > INT32_MAX / 4) return fail(kErrInvalid, "conv3x3 too large");
  if (reinterpret_cast<uintptr_t>(p.x) & 15 || reinterpret_cast<uintptr_t>(p.wt) & 15)
    return fail(kErrInvalid, "conv3x3 input and weight must be 16-byte aligned");
  if (p.ldo < p.cout) return fail(kErrInvalid, "conv3x3 output row stride below the channel count");
  if (p.residual != nullptr && p.ldr < p.cout) return fail(kErrInvalid, "conv3x3 residual row stride too small");
  if (p.variant && !gemm_variant_known(p.variant, false))
    return fail(kErrUnsupported, "no conv3x3 variant %d", p.variant);
  // Pairs only when forced: on the SD1.5 convolutions they measured level with or slower than one-CTA tiles.
  GemmPlan plan = gemm_plan(M, p.cout, K, dev->sms, p.variant, false, false);
  const int bn = plan.bn;
  const int tile_m = plan.pair ? 2 * kGemmBM : kGemmBM;

  EncodeTiledFn enc = nullptr;
  if (int rc = encode_tiled_fn(&enc)) return rc;
  CUtensorMap mx, mw, mo;
  {
    cuuint64_t dims[4] = {cuuint64_t(p.cin), cuuint64_t(p.w), cuuint64_t(p.h), cuuint64_t(p.n)};
    cuuint64_t strides[3] = {cuuint64_t(p.cin) * 2, cuuint64_t(p.w * p.cin) * 2, cuuint64_t(p.h * p.w * p.cin) * 2};
    cuuint32_t box[4] = {cuuint32_t(kGemmBK), cuuint32_t(p.w), cuuint32_t(th), cuuint32_t(imgs)};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(p.x), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(kErrInvalid, "cuTensorMapEncodeTiled failed (%d) for the conv input", int(r));
  }
  if (int rc = encode_kmajor_map(p.wt, p.cout, K, K, plan.pair ? bn / 2 : bn, &mw)) return rc;
  memset(&mo, 0, sizeof(mo));
  const int esz = p.out_f32 ? 4 : 2;
  bool tma_store = (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 && (p.ldo * esz) % 16 == 0;
  if (tma_store && encode_out_map(p.out, M, p.cout, p.ldo, p.out_f32 != 0, &mo) != kOk) tma_store = false;

  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.tma_store = tma_store ? 1 : 0;
  a.M = int(M);
  a.N = int(p.cout);
  a.K = int(K);
  a.num_m_blk = int((M + tile_m - 1) / tile_m);
  a.num_n_blk = int((p.cout + bn - 1) / bn);
  a.n_fastest = 1;  // the input patch stays in L2 while the output-channel tiles of a pixel tile go by
  a.num_tiles = a.num_m_blk * a.num_n_blk;
  a.num_kb = int(K / kGemmBK);
  a.bias = p.bias;
  a.bias_f32 = p.bias_f32;
  a.bias_n = int(p.cout);
  a.bias_img_stride = p.bias != nullptr ? p.bias_img_stride : 0;
  a.bias_img_pixels = int(p.h * p.w);
  a.bias_imgs = int(p.n);
  a.residual = p.residual;
  a.ldr = p.ldr;
  a.out = p.out;
  a.ldo = p.ldo;
  a.out_f32 = p.out_f32;
  a.splits = plan.splits;
  a.kb_per_split = plan.kb_per_split;
  a.cv_w = int(p.w);
  a.cv_hw = int(p.h * p.w);
  a.cv_cblocks = int(p.cin / kGemmBK);
  a.ctl.status = dev->status;
  a.ctl.timeout_ns = wait_timeout_ns();
  a.ctl.debug = p.debug;
  const int64_t units = int64_t(a.num_tiles) * plan.splits;
  const int sms = dev->sms;
  const int d = dev->device;
  if (plan.pair) {
    switch (bn) {
      case 128: return launch_variant<128, 8, kModeConv3x3, true>(mx, mw, mo, a, units, sms, stream, d);
      case 192: return launch_variant<192, 6, kModeConv3x3, true>(mx, mw, mo, a, units, sms, stream, d);
      case 256: return launch_variant<256, 6, kModeConv3x3, true>(mx, mw, mo, a, units, sms, stream, d);
    }
    return fail(kErrUnsupported, "no paired conv3x3 variant with an output-channel tile of %d", bn);
  }
  switch (bn) {
    case 64: return launch_variant<64, 8, kModeConv3x3>(mx, mw, mo, a, units, sms, stream, d);
    case 96: return launch_variant<96, 6, kModeConv3x3>(mx, mw, mo, a, units, sms, stream, d);
    case 128: return launch_variant<128, 6, kModeConv3x3>(mx, mw, mo, a, units, sms, stream, d);
    case 160: return launch_variant<160, 5, kModeConv3x3>(mx, mw, mo, a, units, sms, stream, d);
    case 192: return launch_variant<192, 4, kModeConv3x3>(mx, mw, mo, a, units, sms, stream, d);
    case 256: return launch_variant<256, 4, kModeConv3x3>(mx, mw, mo, a, units, sms, stream, d);
  }
  return fail(kErrUnsupported, "no conv3x3 variant with an output-channel tile of %d", bn);
}

size_t conv3x3_workspace_bytes(int64_t n, int64_t h, int64_t w, int64_t cin, int64_t cout, int variant, int sms) {
  if (n <= 0 || h <= 0 || w <= 0 || cin <= 0 || cout <= 0 || sms <= 0) return 0;
  return gemm_plan(n * h * w, cout, 9 * cin, sms, variant, false, false).split_ws_bytes;
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
