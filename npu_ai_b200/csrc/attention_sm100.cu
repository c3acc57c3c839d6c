// attention_sm100.cu - fused flash attention on B200: out = softmax(Q K^T * scale) V for every (batch, head)
// pair of a block in ONE launch (bf16 q/k/v, f32 statistics and accumulation, bf16 or f32 out).
//
// Replaces the reference's fused NPU attention: NpuGemm.attention / _attention_fused (npu/xdna1_gemm.py:499-752),
// NpuProgram.submit_attn (npu/xdna1_program.py:461-473) and the AIE kernel npu/kernels/xdna1_attn.cc:342-445
// (attn_round_init / attn_block_main / attn_block_last / attn_round_finish). Kept from the reference: the online
// softmax in base 2 with the scale folded in as scale*log2(e) (xdna1_attn.cc:24-32, :344-358) and the lazy
// rescale that moves a row's running max only when it grows by more than 8 (log2 units, RESCALE_THRESHOLD,
// xdna1_attn.cc:80-82, :276-289), so the O/l correction is rare. Not kept: the NPU's layout marshalling
// (K/V interleaving, Q slabs, parts), its tiling limits (tq % 4bq, tk % bk, bh % 4; xdna1_program.py:422-426) and
// the per-head fallback: any Sq/Skv works here, the key tail (e.g. Skv = 77) is masked in the kernel.
//
// One CTA per (128-query tile, (b, h) pair); 192 threads:
//   warps 0-3   softmax: thread t owns query row t of the tile = TMEM lane t. Reads its S row from TMEM,
//               masks the key tail, keeps the running max m and sum l in registers, writes P (bf16) to shared
//               memory, rescales its O row in TMEM when m moves, and normalises + stores O at the end.
//   warp 4      TMA producer: Q once, then K and V tiles into a STAGES-deep ring.
//   warp 5      TMEM owner + MMA issuer: S[j%2] = Q K_j^T (tcgen05, M=128, N=BN), then O += P_{j-1} V_{j-1}, so the
//               tensor core computes the next scores while the softmax works on the current ones.
// Data layout: every operand lives in shared memory as 128-byte-swizzled atoms of 64 head-dim (or key) columns,
// loaded by TMA with 128-byte rows from a 4-D (dim, head, seq, batch) tensor map over the caller's strided
// tensor. The map's innermost extent is the true head dim, so the columns past it (40 -> 64, 80 -> 128,
// 160 -> 192) come in as TMA's out-of-bounds zeros: no host padding, no copies of the model's tensors, and the
// tensor core reads K-major Q/K/P and MN-major V straight from those atoms.
#include <algorithm>
#include <cstdio>
#include <cstring>

#include "internal.h"

namespace npub200 {

constexpr int kAttnBM = 128;
constexpr int kAttnThreads = 192;
constexpr int kSoftmaxWarps = 4;
constexpr int kAtomBytesPerRow = 128;  // one 128-byte swizzle atom row: 64 bf16

struct MapPos {
  int s, h, b;  // position (1..3) of the seq / head / batch dimension in the tensor map
};

struct AttnArgs {
  int Sq, Skv, H, nkv;
  float scale_log2;     // scale * log2(e)
  float rescale_thr;    // lazy-rescale threshold in log2 units
  void* out;
  long long o_sb, o_ss, o_sh;
  int out_f32;
  int D;                // true head dim (output columns)
  MapPos pq, pk, pv;
  KernelCtl ctl;
};

template <int DP, int BN, int STAGES>
struct AttnLayout {
  static constexpr int kNA = (DP + 63) / 64;             // 64-column atoms along the head dim
  static constexpr int kQAtom = kAttnBM * kAtomBytesPerRow;  // 16 KB
  static constexpr int kKVAtom = BN * kAtomBytesPerRow;
  static constexpr int kQBytes = kNA * kQAtom;
  static constexpr int kKVBytes = kNA * kKVAtom;         // one K (or V) tile
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + STAGES * kKVBytes;
  static constexpr int kBarOff = kVOff + STAGES * kKVBytes;
  // q_full, k_full[S], v_full[S], kv_empty[S], s_full[2], s_empty[2], p_full[2], pv_done[2], drain
  static constexpr int kNumBars = 1 + 3 * STAGES + 8 + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 16 + 1024;  // + slack to align the base to 1 KB
  static constexpr int kSCol = 0;            // S[0] at column 0, S[1] at column BN
  static constexpr int kOCol = 2 * BN;       // O accumulator (DP columns)
  // P[0], P[1]: bf16 pairs, BN/2 columns each (the A operand of P V), 32-column aligned.
  static constexpr int kPCol = (2 * BN + DP + 31) / 32 * 32;
  static constexpr int kTmemUsed = kPCol + BN;
  static constexpr int kTmemCols = (kTmemUsed <= 128) ? 128 : (kTmemUsed <= 256) ? 256 : 512;
  static_assert(DP % 16 == 0 && DP >= 16 && DP <= 256, "padded head dim must be a multiple of 16 in [16, 256]");
  static_assert(BN % 64 == 0 && BN <= 256, "key tile must be a multiple of 64");
  static_assert(kTmemUsed <= 512, "S double buffer + O + P double buffer must fit in 512 TMEM columns");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

// Coordinates (dim, then the three outer dims in the map's order) of 64-column atom `atom` of row s of (b, h).
__device__ __forceinline__ void map_coords(const MapPos& p, int atom, int s, int h, int b, int& c0, int& c1, int& c2,
                                           int& c3) {
  c0 = atom * 64;
  c1 = p.s == 1 ? s : (p.h == 1 ? h : b);
  c2 = p.s == 2 ? s : (p.h == 2 ? h : b);
  c3 = p.s == 3 ? s : (p.h == 3 ? h : b);
}

template <int DP, int BN, int STAGES>
__global__ void __launch_bounds__(kAttnThreads, (AttnLayout<DP, BN, STAGES>::kSmemBytes <= 113 * 1024 &&
                                                  AttnLayout<DP, BN, STAGES>::kTmemCols <= 256) ? 2 : 1)
    attention_fwd_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                                 const __grid_constant__ CUtensorMap tm_v, const AttnArgs args) {
  using L = AttnLayout<DP, BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* kv_empty = v_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* pv_done = p_full + 2;
  uint64_t* drain = pv_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * kAttnBM;
  const int pair = blockIdx.y;
  const int hh = pair % args.H;
  const int bb = pair / args.H;
  const int nkv = args.nkv;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kSoftmaxWarps);
      mbar_init(&p_full[i], kSoftmaxWarps);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 4) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      pdl_wait();  // q/k/v may be the previous kernel's outputs
      int c0, c1, c2, c3;
      mbar_arrive_expect_tx(q_full, L::kQBytes);
      for (int a = 0; a < L::kNA; ++a) {
        map_coords(args.pq, a, q0, hh, bb, c0, c1, c2, c3);
        tma_load_4d(&tm_q, q_full, sQ + a * L::kQAtom, c0, c1, c2, c3);
      }
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        if (!mbar_wait_bounded(&kv_empty[stage], phase ^ 1u, abort_flag, args.ctl, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        const int kv0 = j * BN;
        mbar_arrive_expect_tx(&k_full[stage], L::kKVBytes);
        for (int a = 0; a < L::kNA; ++a) {
          map_coords(args.pk, a, kv0, hh, bb, c0, c1, c2, c3);
          tma_load_4d(&tm_k, &k_full[stage], sK + stage * L::kKVBytes + a * L::kKVAtom, c0, c1, c2, c3);
        }
        mbar_arrive_expect_tx(&v_full[stage], L::kKVBytes);
        for (int a = 0; a < L::kNA; ++a) {
          map_coords(args.pv, a, kv0, hh, bb, c0, c1, c2, c3);
          tma_load_4d(&tm_v, &v_full[stage], sV + stage * L::kKVBytes + a * L::kKVAtom, c0, c1, c2, c3);
        }
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // Drain: Q and the loads of the last min(issued, STAGES) tiles must land before shared memory is released.
      mbar_wait_drain(q_full, 0, args.ctl);
      if (!ok) {
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < min(issued, STAGES); ++i) {
          if (s == 0) {
            s = STAGES - 1;
            ph ^= 1u;
          } else {
            --s;
          }
          mbar_wait_drain(&k_full[s], ph, args.ctl);
          mbar_wait_drain(&v_full[s], ph, args.ctl);
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescS = idesc_bf16_f32(kAttnBM, BN, false);  // S = Q K^T: both K-major
      constexpr uint32_t kIdescO = idesc_bf16_f32(kAttnBM, DP, true);   // O += P V: V is MN-major
      bool ok = true;
      if (args.ctl.debug & 1u) {
        if (!mbar_wait_bounded(drain, 0, abort_flag, args.ctl, kStatusForced)) ok = false;
      }
      if (ok && !mbar_wait_bounded(q_full, 0, abort_flag, args.ctl, kStatusTimeoutMma)) ok = false;
      tc_fence_after();
      // Descriptors are built once; every operand of every step is the base plus a byte offset (whose >> 4 lands in
      // the descriptor's address field), so the issue loop is one 64-bit add per operand per MMA.
      const uint64_t q_desc = smem_desc_kmajor_sw128(smem_u32(sQ));
      const uint64_t k_desc = smem_desc_kmajor_sw128(smem_u32(sK));
      const uint64_t v_desc = smem_desc_mnmajor_sw128(smem_u32(sV), L::kKVAtom);
      auto issue_pv = [&](int i) -> bool {
        const int st = i % STAGES;
        const uint32_t ph = uint32_t(i / STAGES) & 1u;
        const int buf = i & 1;
        if (!mbar_wait_bounded(&v_full[st], ph, abort_flag, args.ctl, kStatusTimeoutMma)) return false;
        if (!mbar_wait_bounded(&p_full[buf], uint32_t(i >> 1) & 1u, abort_flag, args.ctl, kStatusTimeoutMma))
          return false;
        tc_fence_after();
        const uint32_t pa = tmem_base + uint32_t(L::kPCol + buf * (BN / 2));
        const uint64_t va = v_desc + uint64_t((st * L::kKVBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // P from TMEM: 16 keys = 8 columns per K step. V: MN-major (head dim contiguous), 16 keys = 16 rows of
          // 128 B further per K step.
          umma_f16_ts(tmem_base + L::kOCol, pa + uint32_t(kk * 8), va + uint64_t((kk * 16 * kAtomBytesPerRow) >> 4),
                      kIdescO, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&pv_done[buf]);
        umma_commit(&kv_empty[st]);
        return true;
      };
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j % STAGES;
        const uint32_t ph = uint32_t(j / STAGES) & 1u;
        const int buf = j & 1;
        if (!mbar_wait_bounded(&k_full[st], ph, abort_flag, args.ctl, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        if (!mbar_wait_bounded(&s_empty[buf], (uint32_t(j >> 1) & 1u) ^ 1u, abort_flag, args.ctl,
                               kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ka = k_desc + uint64_t((st * L::kKVBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk) {
          // Q and K: K-major over the head dim, atoms of 64 columns, +32 B per 16 columns inside an atom.
          umma_f16_ss(tmem_base + L::kSCol + buf * BN, q_desc + uint64_t(((kk >> 2) * L::kQAtom + (kk & 3) * 32) >> 4),
                      ka + uint64_t(((kk >> 2) * L::kKVAtom + (kk & 3) * 32) >> 4), kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[buf]);
        if (j >= 1 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && nkv >= 1 && !issue_pv(nkv - 1)) ok = false;
      if (!ok) {
        umma_commit(drain);
        mbar_wait_drain(drain, 0u, args.ctl);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / correction / epilogue (warps 0-3)
    const int row = warp * 32 + lane;  // query row in the tile == TMEM lane
    const uint32_t lane_base = tmem_base + (uint32_t(warp * 32) << 16);
    const float c = args.scale_log2;
    float m = -INFINITY;  // running max in log2 units (scores * scale * log2 e)
    float l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int buf = j & 1;
      if (!mbar_wait_bounded(&s_full[buf], uint32_t(j >> 1) & 1u, abort_flag, args.ctl, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[BN];  // raw scores of this row (the scale is folded into the exponent below)
#pragma unroll
      for (int cc = 0; cc < BN; cc += 32) {
        uint32_t r[32];
        tmem_ld32(lane_base + uint32_t(L::kSCol + buf * BN + cc), r);
#pragma unroll
        for (int t = 0; t < 32; ++t) s[cc + t] = __uint_as_float(r[t]);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[buf]);

      const int kv0 = j * BN;
      if (kv0 + BN > args.Skv) {
#pragma unroll
        for (int t = 0; t < BN; ++t)
          if (kv0 + t >= args.Skv) s[t] = -INFINITY;
      }
      // Row max as 8 independent chains, then a 3-level tree (short dependency chains keep the pipes busy).
      float mx8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx8[e] = s[e];
#pragma unroll
      for (int t = 8; t < BN; t += 8)
#pragma unroll
        for (int e = 0; e < 8; ++e) mx8[e] = fmaxf(mx8[e], s[t + e]);
#pragma unroll
      for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
        for (int e = 0; e < w; ++e) mx8[e] = fmaxf(mx8[e], mx8[e + w]);
      const float mx = mx8[0] * c;  // log2 units (c = scale * log2 e > 0)
      // Lazy running max: move only when this tile's max beats it by more than the threshold.
      const bool move = mx > m + args.rescale_thr;
      const float m_new = move ? mx : m;
      const float alpha = fast_exp2(m - m_new);  // 1 when unchanged, 0 on the first tile
      const float neg_m = -m_new;
      float rs8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      // P buffer `buf` is free once PV of tile j-2 has completed.
      if (j >= 2 &&
          !mbar_wait_bounded(&pv_done[buf], (uint32_t((j - 2) >> 1) & 1u), abort_flag, args.ctl,
                             kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      // P row into TMEM (this thread's lane): bf16 pairs, 32 keys = 16 columns per store.
      const uint32_t p_cols = lane_base + uint32_t(L::kPCol + buf * (BN / 2));
#pragma unroll
      for (int c32 = 0; c32 < BN / 32; ++c32) {
        uint32_t pk[16];
#pragma unroll
        for (int e2 = 0; e2 < 16; ++e2) {
          const float p0 = fast_exp2(fmaf(s[c32 * 32 + 2 * e2], c, neg_m));
          const float p1 = fast_exp2(fmaf(s[c32 * 32 + 2 * e2 + 1], c, neg_m));
          rs8[(2 * e2) & 7] += p0;
          rs8[(2 * e2 + 1) & 7] += p1;
          pk[e2] = pack_bf16x2(p0, p1);
        }
        tmem_st16(p_cols + uint32_t(c32 * 16), pk);
      }
#pragma unroll
      for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
        for (int e = 0; e < w; ++e) rs8[e] += rs8[e + w];
      l = l * alpha + rs8[0];
      m = m_new;
      // O correction (rare with the lazy max): O_row *= alpha once PV of tile j-1 has landed. Warp-uniform because
      // tcgen05.ld/st are warp-wide; lanes whose max did not move scale by 1.
      if (j > 0 && __any_sync(0xffffffffu, move)) {
        if (!mbar_wait_bounded(&pv_done[(j - 1) & 1], uint32_t((j - 1) >> 1) & 1u, abort_flag, args.ctl,
                               kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < DP; cc += 16) {
          uint32_t r[16];
          tmem_ld16(lane_base + uint32_t(L::kOCol + cc), r);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 16; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
          tmem_st16(lane_base + uint32_t(L::kOCol + cc), r);
        }
        tmem_wait_st();
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[buf]);
    }
    if (ok && nkv >= 1) {
      const int last = nkv - 1;
      pdl_wait();  // the previous kernel may still read the output buffer
      if (mbar_wait_bounded(&pv_done[last & 1], uint32_t(last >> 1) & 1u, abort_flag, args.ctl,
                            kStatusTimeoutEpilogue)) {
        tc_fence_after();
        const float inv_l = 1.0f / l;
        const int grow = q0 + row;
        const bool store = grow < args.Sq;
        const long long obase = (long long)bb * args.o_sb + (long long)grow * args.o_ss + (long long)hh * args.o_sh;
#pragma unroll
        for (int cc = 0; cc < DP; cc += 16) {
          uint32_t r[16];
          tmem_ld16(lane_base + uint32_t(L::kOCol + cc), r);
          tmem_wait_ld();
          if (store) {
            float o[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) o[t] = __uint_as_float(r[t]) * inv_l;
            const int ncols = min(16, args.D - cc);
            if (args.out_f32) {
              float* dst = static_cast<float*>(args.out) + obase + cc;
              if (ncols == 16 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
                for (int t = 0; t < 4; ++t)
                  reinterpret_cast<float4*>(dst)[t] = make_float4(o[4 * t], o[4 * t + 1], o[4 * t + 2], o[4 * t + 3]);
              } else {
#pragma unroll
                for (int t = 0; t < 16; ++t)
                  if (t < ncols) dst[t] = o[t];
              }
            } else {
              __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(args.out) + obase + cc;
              if (ncols >= 8 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                uint4 v0;
                v0.x = pack_bf16x2(o[0], o[1]);
                v0.y = pack_bf16x2(o[2], o[3]);
                v0.z = pack_bf16x2(o[4], o[5]);
                v0.w = pack_bf16x2(o[6], o[7]);
                reinterpret_cast<uint4*>(dst)[0] = v0;
                if (ncols == 16) {
                  uint4 v1;
                  v1.x = pack_bf16x2(o[8], o[9]);
                  v1.y = pack_bf16x2(o[10], o[11]);
                  v1.z = pack_bf16x2(o[12], o[13]);
                  v1.w = pack_bf16x2(o[14], o[15]);
                  reinterpret_cast<uint4*>(dst)[1] = v1;
                } else {
#pragma unroll
                  for (int t = 8; t < 16; ++t)
                    if (t < ncols) dst[t] = __float2bfloat16_rn(o[t]);
                }
              } else {
#pragma unroll
                for (int t = 0; t < 16; ++t)
                  if (t < ncols) dst[t] = __float2bfloat16_rn(o[t]);
              }
            }
          }
        }
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------------------------
namespace {

struct DimStride {
  int64_t extent;
  int64_t stride;  // elements
  int which;       // 0 = seq, 1 = head, 2 = batch
};

// 4-D map (dim, then seq/head/batch sorted by stride) with a box of 64 dim-elements (one 128-byte swizzle atom) x
// `rows` sequence rows. The dim extent is the true head dim: the columns of the atom past it read as zeros.
int encode_bshd_map(const void* base, int64_t D, int64_t S, int64_t H, int64_t B, int64_t ss, int64_t sh, int64_t sb,
                    int rows, CUtensorMap* out, MapPos* pos) {
  EncodeTiledFn enc = nullptr;
  if (int rc = encode_tiled_fn(&enc)) return rc;
  DimStride d[3] = {{S, ss, 0}, {H, sh, 1}, {B, sb, 2}};
  int64_t maxs = D;
  for (auto& x : d)
    if (x.extent > 1) maxs = std::max(maxs, x.stride);
  for (auto& x : d) {
    if (x.extent == 1) x.stride = (maxs + 7) / 8 * 8;  // coordinate is always 0: any legal stride will do
    if (x.stride <= 0 || x.stride % 8 != 0)
      return fail(kErrInvalid, "attention strides must be positive multiples of 8 elements (got %lld)",
                  (long long)x.stride);
  }
  std::sort(d, d + 3, [](const DimStride& a, const DimStride& b) { return a.stride < b.stride; });
  cuuint64_t dims[4] = {cuuint64_t(D), cuuint64_t(d[0].extent), cuuint64_t(d[1].extent), cuuint64_t(d[2].extent)};
  cuuint64_t strides[3] = {cuuint64_t(d[0].stride) * 2, cuuint64_t(d[1].stride) * 2, cuuint64_t(d[2].stride) * 2};
  cuuint32_t box[4] = {64, 1, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  for (int i = 0; i < 3; ++i) {
    if (d[i].which == 0) {
      box[i + 1] = cuuint32_t(rows);
      pos->s = i + 1;
    } else if (d[i].which == 1) {
      pos->h = i + 1;
    } else {
      pos->b = i + 1;
    }
  }
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(kErrInvalid, "cuTensorMapEncodeTiled failed (%d) for an attention operand (D=%lld S=%lld H=%lld B=%lld)",
                int(r), (long long)D, (long long)S, (long long)H, (long long)B);
  return kOk;
}

template <int DP, int BN, int STAGES>
int launch_attn(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnArgs& a, dim3 grid,
                cudaStream_t st, int device) {
  using L = AttnLayout<DP, BN, STAGES>;
  static bool configured[64] = {false};
  auto kern = attention_fwd_tcgen05_kernel<DP, BN, STAGES>;
  if (!configured[device]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(attention smem)");
    configured[device] = true;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = L::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, a), "attention kernel launch");
}

// Kernel variant for a padded head dim and key tile (64 or 128 keys per tile).
int launch_for(int64_t DP, int BN, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
               const AttnArgs& a, dim3 grid, cudaStream_t st, int dev) {
#define NPUB200_ATTN_CASE(dp, bn, stages) \
  if (DP == dp && BN == bn) return launch_attn<dp, bn, stages>(mq, mk, mv, a, grid, st, dev);
  // one 64-column atom of head dim (d <= 64)
  NPUB200_ATTN_CASE(16, 64, 3)
  NPUB200_ATTN_CASE(32, 64, 3)
  NPUB200_ATTN_CASE(48, 64, 3)
  NPUB200_ATTN_CASE(64, 64, 3)
  NPUB200_ATTN_CASE(16, 128, 3)
  NPUB200_ATTN_CASE(32, 128, 3)
  NPUB200_ATTN_CASE(48, 128, 3)
  NPUB200_ATTN_CASE(64, 128, 3)
  // two atoms (64 < d <= 128)
  NPUB200_ATTN_CASE(80, 64, 3)
  NPUB200_ATTN_CASE(96, 64, 3)
  NPUB200_ATTN_CASE(112, 64, 3)
  NPUB200_ATTN_CASE(128, 64, 3)
  NPUB200_ATTN_CASE(80, 128, 2)
  NPUB200_ATTN_CASE(96, 128, 2)
  NPUB200_ATTN_CASE(112, 128, 2)
  NPUB200_ATTN_CASE(128, 128, 2)
  // three or four atoms (128 < d <= 256): 64-key tiles only (TMEM: 2 x 64 S columns + d O columns)
  NPUB200_ATTN_CASE(144, 64, 2)
  NPUB200_ATTN_CASE(160, 64, 2)
  NPUB200_ATTN_CASE(176, 64, 2)
  NPUB200_ATTN_CASE(192, 64, 2)
  NPUB200_ATTN_CASE(208, 64, 2)
  NPUB200_ATTN_CASE(224, 64, 2)
  NPUB200_ATTN_CASE(240, 64, 2)
  NPUB200_ATTN_CASE(256, 64, 2)
#undef NPUB200_ATTN_CASE
  return fail(kErrUnsupported, "no attention variant for padded head dim %lld with %d-key tiles", (long long)DP, BN);
}

}  // namespace

int attention_launch(const AttnProblem& p, cudaStream_t stream) {
  const DeviceInfo* dev = nullptr;
  if (int rc = current_device_info(&dev)) return rc;
  if (p.D % 8 != 0 || p.D > 256)
    return fail(kErrUnsupported, "head dim %lld is not a multiple of 8 in [8, 256]", (long long)p.D);
  if (!(p.scale > 0.0f)) return fail(kErrInvalid, "attention scale must be positive (got %g)", double(p.scale));
  const int64_t pairs = p.B * p.H;
  if (pairs > 65535) return fail(kErrUnsupported, "batch*heads = %lld exceeds 65535", (long long)pairs);
  if (p.Sq > INT32_MAX / 2 || p.Skv > INT32_MAX / 2) return fail(kErrInvalid, "sequence too long");
  for (const void* ptr : {p.q, p.k, p.v})
    if (reinterpret_cast<uintptr_t>(ptr) & 15u) return fail(kErrInvalid, "q/k/v base addresses must be 16-byte aligned");
  const int64_t DP = (p.D + 15) / 16 * 16;
  // Key tile (variant): for head dims up to 64 the default is 64 keys, which halves the per-CTA footprint so two
  // CTAs share an SM (their softmax warps hide each other's latencies); 128 keys otherwise. 64 is the only tile for
  // head dims above 128.
  int BN = p.variant ? p.variant : (DP <= 64 ? 64 : 128);
  if (BN != 64 && BN != 128) return fail(kErrUnsupported, "attention key tile %d (variants: 64, 128)", BN);
  if (DP > 128) BN = 64;

  CUtensorMap mq, mk, mv;
  AttnArgs a;
  memset(&a, 0, sizeof(a));
  if (int rc = encode_bshd_map(p.q, p.D, p.Sq, p.H, p.B, p.q_ss, p.q_sh, p.q_sb, kAttnBM, &mq, &a.pq)) return rc;
  if (int rc = encode_bshd_map(p.k, p.D, p.Skv, p.H, p.B, p.k_ss, p.k_sh, p.k_sb, BN, &mk, &a.pk)) return rc;
  if (int rc = encode_bshd_map(p.v, p.D, p.Skv, p.H, p.B, p.v_ss, p.v_sh, p.v_sb, BN, &mv, &a.pv)) return rc;
  a.Sq = int(p.Sq);
  a.Skv = int(p.Skv);
  a.H = int(p.H);
  a.nkv = int((p.Skv + BN - 1) / BN);
  a.scale_log2 = p.scale * 1.4426950408889634f;
  a.rescale_thr = 8.0f;
  a.out = p.o;
  a.o_sb = p.o_sb;
  a.o_ss = p.o_ss;
  a.o_sh = p.o_sh;
  a.out_f32 = p.out_f32;
  a.D = int(p.D);
  a.ctl.status = dev->status;
  a.ctl.timeout_ns = wait_timeout_ns();
  a.ctl.debug = p.debug;
  const dim3 grid(unsigned((p.Sq + kAttnBM - 1) / kAttnBM), unsigned(pairs));
  if (grid.x > 0x7fffffffu) return fail(kErrInvalid, "too many query tiles");
  return launch_for(DP, BN, mq, mk, mv, a, grid, stream, dev->device);
}

}  // namespace npub200
