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
// Two kernels share one structure (softmax warps, a TMA producer warp, MMA-issuing warps) and differ in how many
// 128-row query tiles a CTA owns:
//   attention_fwd_mq_tcgen05_kernel  QT = 2 or 4 Q tiles (256 or 512 query rows) per CTA, one CTA per SM, 96 + 128 QT
//       threads. All tiles share every K/V tile. One warp issues every S = Q K^T into a ring of S buffers shared by
//       the tiles (ahead of need, as buffers free up), another every O += P V, so a tile's next S no longer waits
//       behind its own P V and the other tiles' MMAs.
//   attention_fwd_tcgen05_kernel      one Q tile per CTA with S double-buffered (S_j, S_{j+1}), 192 threads, up to
//       two CTAs per SM: for grids too small to fill the GPU with 256-row CTAs, and head dims above 192.
// Roles:
//   softmax warps  thread t of a warpgroup owns query row t of its Q tile = TMEM lane t. Reads its S row from TMEM,
//                  masks the key tail, keeps the running max m and sum l in registers, writes P (bf16 pairs) back
//                  into the TMEM columns its S tile came from (the A operand of P V), rescales its O row in TMEM
//                  when m moves, and normalises + stores O at the end.
//   producer warp  TMA: Q once, then K and V tiles into STAGES-deep rings, K one tile ahead of V. A K slot is
//                  released as soon as its S MMAs complete, a V slot when its P V MMAs complete.
//   MMA warp(s)    TMEM owner + tcgen05 issue: S = Q K_j^T (M=128, N=BN, both K-major in shared memory) and
//                  O += P V_j (P from TMEM, V MN-major in shared memory). tcgen05.mma ops of one thread execute in
//                  issue order and a tcgen05.commit covers every MMA its thread issued before it; between the two
//                  issuers of kernel 2 the order comes from mbarriers (a buffer is refilled only after its P V).
// Data layout: every operand lives in shared memory as 128-byte-swizzled atoms of 64 head-dim (or key) columns,
// loaded by TMA with 128-byte rows from a 4-D (dim, head, seq, batch) tensor map over the caller's strided
// tensor. The map's innermost extent is the true head dim, so the columns past it (40 -> 64, 80 -> 128,
// 160 -> 192) come in as TMA's out-of-bounds zeros: no host padding, no copies of the model's tensors.
#include <algorithm>
#include <cstdio>
#include <cstring>

#include "internal.h"

namespace npub200 {

constexpr int kAttnBM = 128;           // query rows per Q tile (one softmax warpgroup, one TMEM lane per row)
constexpr int kSoftmaxWarps = 4;       // per Q tile
constexpr int kAtomBytesPerRow = 128;  // one 128-byte swizzle atom row: 64 bf16
// Of every 8 (key, key+1) pairs of a softmax row, this many take their exponentials from the FMA-pipe polynomial
// (exp2_poly3_x2) instead of the MUFU. Measured: head dims up to 64 (the least MMA work per exponential) gain from
// moving 2 of 8 to the FP32 pipe with one or two Q tiles per CTA; with four Q tiles per CTA the issue slots the
// polynomial takes cost more than the MUFU time it saves; larger head dims run best with none.
template <int DP, int QT>
constexpr int exp_poly_pairs_per8() {
  return (DP <= 64 && QT <= 2) ? 2 : 0;
}

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

// Coordinates (dim, then the three outer dims in the map's order) of 64-column atom `atom` of row s of (b, h).
__device__ __forceinline__ void map_coords(const MapPos& p, int atom, int s, int h, int b, int& c0, int& c1, int& c2,
                                           int& c3) {
  c0 = atom * 64;
  c1 = p.s == 1 ? s : (p.h == 1 ? h : b);
  c2 = p.s == 2 ? s : (p.h == 2 ? h : b);
  c3 = p.s == 3 ? s : (p.h == 3 ? h : b);
}

// ---------------------------------------------------------------------------------------------------------------
// Producer: K and V tiles of one (b, h) pair into STAGES-deep rings, K one tile ahead of V (K_j is needed a whole
// softmax step before V_j). On an abort it waits for the loads it issued before returning, so shared memory is
// not released under an in-flight copy.
// ---------------------------------------------------------------------------------------------------------------
template <int NA, int BN, int STAGES>
__device__ __forceinline__ void kv_producer(const CUtensorMap* tm_k, const CUtensorMap* tm_v, const AttnArgs& args,
                                            uint8_t* sK, uint8_t* sV, uint64_t* k_full, uint64_t* v_full,
                                            uint64_t* k_empty, uint64_t* v_empty, volatile int* abort_flag, int hh,
                                            int bb) {
  constexpr int kAtom = BN * kAtomBytesPerRow;
  constexpr int kTile = NA * kAtom;
  const int nkv = args.nkv;
  int issued_k = 0, issued_v = 0;
  bool ok = true;
  int c0, c1, c2, c3;
  for (int j = 0; j <= nkv; ++j) {
    if (j < nkv) {
      const int st = j % STAGES;
      if (!mbar_wait_bounded(&k_empty[st], (uint32_t(j / STAGES) & 1u) ^ 1u, abort_flag, args.ctl,
                             kStatusTimeoutProducer)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&k_full[st], kTile);
      for (int a = 0; a < NA; ++a) {
        map_coords(args.pk, a, j * BN, hh, bb, c0, c1, c2, c3);
        tma_load_4d(tm_k, &k_full[st], sK + st * kTile + a * kAtom, c0, c1, c2, c3);
      }
      ++issued_k;
    }
    if (j >= 1) {
      const int i = j - 1;
      const int st = i % STAGES;
      if (!mbar_wait_bounded(&v_empty[st], (uint32_t(i / STAGES) & 1u) ^ 1u, abort_flag, args.ctl,
                             kStatusTimeoutProducer)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&v_full[st], kTile);
      for (int a = 0; a < NA; ++a) {
        map_coords(args.pv, a, i * BN, hh, bb, c0, c1, c2, c3);
        tma_load_4d(tm_v, &v_full[st], sV + st * kTile + a * kAtom, c0, c1, c2, c3);
      }
      ++issued_v;
    }
  }
  if (!ok) {
    for (int i = max(0, issued_k - STAGES); i < issued_k; ++i)
      mbar_wait_drain(&k_full[i % STAGES], uint32_t(i / STAGES) & 1u, args.ctl);
    for (int i = max(0, issued_v - STAGES); i < issued_v; ++i)
      mbar_wait_drain(&v_full[i % STAGES], uint32_t(i / STAGES) & 1u, args.ctl);
  }
}

// S = Q K_j^T for one Q tile: K-major over the head dim, atoms of 64 columns, +32 B per 16 columns in an atom.
template <int DP, int BN>
__device__ __forceinline__ void issue_s(uint32_t d_tmem, uint64_t q_desc, uint64_t k_desc, int q_atom_bytes,
                                        int kv_atom_bytes) {
  constexpr uint32_t kIdescS = idesc_bf16_f32(kAttnBM, BN, false);
#pragma unroll
  for (int kk = 0; kk < DP / 16; ++kk)
    umma_f16_ss(d_tmem, q_desc + uint64_t(((kk >> 2) * q_atom_bytes + (kk & 3) * 32) >> 4),
                k_desc + uint64_t(((kk >> 2) * kv_atom_bytes + (kk & 3) * 32) >> 4), kIdescS, kk > 0 ? 1u : 0u);
}

// O += P V_j: P from TMEM (16 keys = 8 columns of bf16 pairs per K step), V MN-major (head dim contiguous), 16 keys
// = 16 rows of 128 B further per K step.
template <int DP, int BN>
__device__ __forceinline__ void issue_pv(uint32_t o_tmem, uint32_t p_tmem, uint64_t v_desc, bool accumulate) {
  constexpr uint32_t kIdescO = idesc_bf16_f32(kAttnBM, DP, true);
#pragma unroll
  for (int kk = 0; kk < BN / 16; ++kk)
    umma_f16_ts(o_tmem, p_tmem + uint32_t(kk * 8), v_desc + uint64_t((kk * 16 * kAtomBytesPerRow) >> 4), kIdescO,
                (accumulate || kk > 0) ? 1u : 0u);
}

// ---------------------------------------------------------------------------------------------------------------
// Softmax-warp pieces shared by both kernels. A softmax thread owns one query row = one TMEM lane.
// ---------------------------------------------------------------------------------------------------------------

// One online-softmax step over a key tile for this thread's row: reads the BN scores (TMEM columns from s_addr),
// masks keys >= Skv, moves the running max m lazily (only when the tile's max beats it by more than thr, log2
// units), writes P = exp2(s*c - m) as bf16 pairs over the first BN/2 of those columns and updates the running
// sum l. Returns the factor O must be scaled by (1 when m did not move); `move` tells whether it moved. The caller
// signals P once its stores are complete (tmem_wait_st).
template <int BN, int POLY>
__device__ __forceinline__ float softmax_step(uint32_t s_addr, int kv0, int Skv, float c, float thr, float& m,
                                              float& l, bool& move) {
  float s[BN];  // raw scores of this row (the scale is folded into the exponent below)
#pragma unroll
  for (int cc = 0; cc < BN; cc += 32) {
    uint32_t r[32];
    tmem_ld32(s_addr + uint32_t(cc), r);
#pragma unroll
    for (int t = 0; t < 32; ++t) s[cc + t] = __uint_as_float(r[t]);
  }
  tmem_wait_ld();
  if (kv0 + BN > Skv) {
#pragma unroll
    for (int t = 0; t < BN; ++t)
      if (kv0 + t >= Skv) s[t] = -INFINITY;
  }
  // Row max as 8 independent chains of three-input maxima, then a two-level tree.
  float mx8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) mx8[e] = s[e];
#pragma unroll
  for (int t = 8; t + 16 <= BN; t += 16)
#pragma unroll
    for (int e = 0; e < 8; ++e) mx8[e] = fmax3(mx8[e], s[t + e], s[t + 8 + e]);
  if constexpr ((BN - 8) % 16 != 0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) mx8[e] = fmaxf(mx8[e], s[BN - 8 + e]);
  }
  const float mx = fmax3(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])) *
                   c;  // log2 units (c = scale * log2 e > 0)
  move = mx > m + thr;
  const float m_new = move ? mx : m;
  const float alpha = fast_exp2(m - m_new);  // 1 when unchanged, 0 on the first tile
  const float neg_m = -m_new;
  // x = s * c - m and the row sums two keys per instruction (f32x2 FMA / add); P row into TMEM over this lane's S
  // (already in registers): bf16 pairs, 32 keys = 16 columns per store.
  const uint64_t c2 = f2_pack(c, c);
  const uint64_t nm2 = f2_pack(neg_m, neg_m);
  uint64_t rs2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
  for (int c32 = 0; c32 < BN / 32; ++c32) {
    uint32_t pk[16];
#pragma unroll
    for (int e2 = 0; e2 < 16; ++e2) {
      float x0, x1, p0, p1;
      f2_unpack(f2_fma(f2_pack(s[c32 * 32 + 2 * e2], s[c32 * 32 + 2 * e2 + 1]), c2, nm2), x0, x1);
      if ((e2 & 7) >= 8 - POLY) {
        exp2_poly3_x2(x0, x1, p0, p1);
      } else {
        p0 = fast_exp2(x0);
        p1 = fast_exp2(x1);
      }
      rs2[e2 & 3] = f2_add(rs2[e2 & 3], f2_pack(p0, p1));
      pk[e2] = pack_bf16x2(p0, p1);
    }
    tmem_st16(s_addr + uint32_t(c32 * 16), pk);
  }
  rs2[0] = f2_add(rs2[0], rs2[2]);
  rs2[1] = f2_add(rs2[1], rs2[3]);
  float r0, r1;
  f2_unpack(f2_add(rs2[0], rs2[1]), r0, r1);
  l = l * alpha + (r0 + r1);
  m = m_new;
  return alpha;
}

// O row *= alpha (TMEM columns from o_addr). Warp-wide: lanes whose max did not move pass alpha = 1.
template <int DP>
__device__ __forceinline__ void rescale_o_row(uint32_t o_addr, float alpha) {
#pragma unroll
  for (int cc = 0; cc < DP; cc += 16) {
    uint32_t r[16];
    tmem_ld16(o_addr + uint32_t(cc), r);
    tmem_wait_ld();
#pragma unroll
    for (int t = 0; t < 16; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
    tmem_st16(o_addr + uint32_t(cc), r);
  }
  tmem_wait_st();
}

// Normalised O row (TMEM columns from o_addr) to the output: the first D columns of row `grow` of pair (bb, hh),
// bf16 or f32, 16-byte vector stores where aligned. Rows past Sq only drain TMEM (tcgen05.ld is warp-wide).
template <int DP>
__device__ __forceinline__ void store_o_row(uint32_t o_addr, const AttnArgs& args, int grow, int bb, int hh,
                                            float inv_l) {
  const bool store = grow < args.Sq;
  const long long obase = (long long)bb * args.o_sb + (long long)grow * args.o_ss + (long long)hh * args.o_sh;
#pragma unroll
  for (int cc = 0; cc < DP; cc += 16) {
    uint32_t r[16];
    tmem_ld16(o_addr + uint32_t(cc), r);
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

// ---------------------------------------------------------------------------------------------------------------
// Kernel 1: one Q tile per CTA, S double-buffered. Warps 0-3 softmax, warp 4 producer, warp 5 MMA.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kAttn1Threads = 192;

template <int DP, int BN, int STAGES>
struct Attn1Layout {
  static constexpr int kNA = (DP + 63) / 64;                 // 64-column atoms along the head dim
  static constexpr int kQAtom = kAttnBM * kAtomBytesPerRow;  // 16 KB
  static constexpr int kKVAtom = BN * kAtomBytesPerRow;
  static constexpr int kQBytes = kNA * kQAtom;
  static constexpr int kKVBytes = kNA * kKVAtom;  // one K (or V) tile
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;
  static constexpr int kVOff = kKOff + STAGES * kKVBytes;
  static constexpr int kBarOff = kVOff + STAGES * kKVBytes;
  // q_full, k_full[S], v_full[S], k_empty[S], v_empty[S], s_full[2], p_full[2], pv_done[2], drain
  static constexpr int kNumBars = 1 + 4 * STAGES + 6 + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 16 + 1024;  // + slack to align the base to 1 KB
  // S[0] at column 0, S[1] at column BN; P_j overwrites the first half of its own S buffer; O after them.
  static constexpr int kSCol = 0;
  static constexpr int kOCol = 2 * BN;
  static constexpr int kTmemUsed = kOCol + DP;
  static constexpr int kTmemCols = (kTmemUsed <= 128) ? 128 : (kTmemUsed <= 256) ? 256 : 512;
  static constexpr bool kTwoPerSm = kSmemBytes <= 113 * 1024 && kTmemCols <= 256;
  static_assert(DP % 16 == 0 && DP >= 16 && DP <= 256, "padded head dim must be a multiple of 16 in [16, 256]");
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "key tile must be a multiple of 32 in [64, 256]");
  static_assert(kTmemUsed <= 512, "S double buffer + O must fit in 512 TMEM columns");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

template <int DP, int BN, int STAGES>
__global__ void __launch_bounds__(kAttn1Threads, Attn1Layout<DP, BN, STAGES>::kTwoPerSm ? 2 : 1)
    attention_fwd_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                                 const __grid_constant__ CUtensorMap tm_v, const AttnArgs args) {
  using L = Attn1Layout<DP, BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* k_empty = v_full + STAGES;
  uint64_t* v_empty = k_empty + STAGES;
  uint64_t* s_full = v_empty + STAGES;
  uint64_t* p_full = s_full + 2;
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
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
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
      kv_producer<L::kNA, BN, STAGES>(&tm_k, &tm_v, args, sK, sV, k_full, v_full, k_empty, v_empty, abort_flag, hh,
                                      bb);
      mbar_wait_drain(q_full, 0, args.ctl);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop (operands stay warp-uniform); one elected lane issues the MMAs and their commits.
    bool ok = true;
    if (args.ctl.debug & 1u) {
      if (!mbar_wait_bounded_warp(drain, 0, abort_flag, args.ctl, kStatusForced)) ok = false;
    }
    if (ok && !mbar_wait_bounded_warp(q_full, 0, abort_flag, args.ctl, kStatusTimeoutMma)) ok = false;
    tc_fence_after();
    // Descriptors are built once; every operand of every step is the base plus a byte offset (whose >> 4 lands in
    // the descriptor's address field).
    const uint64_t q_desc = smem_desc_kmajor_sw128(smem_u32(sQ));
    const uint64_t k_desc = smem_desc_kmajor_sw128(smem_u32(sK));
    const uint64_t v_desc = smem_desc_mnmajor_sw128(smem_u32(sV), L::kKVAtom);
    auto pv_step = [&](int i) -> bool {
      const int st = i % STAGES;
      const int buf = i & 1;
      if (!mbar_wait_bounded_warp(&v_full[st], uint32_t(i / STAGES) & 1u, abort_flag, args.ctl, kStatusTimeoutMma))
        return false;
      if (!mbar_wait_bounded_warp(&p_full[buf], uint32_t(i >> 1) & 1u, abort_flag, args.ctl, kStatusTimeoutMma))
        return false;
      tc_fence_after();
      if (elect_one()) {
        issue_pv<DP, BN>(tmem_base + L::kOCol, tmem_base + uint32_t(L::kSCol + buf * BN),
                         v_desc + uint64_t((st * L::kKVBytes) >> 4), i > 0);
        umma_commit(&pv_done[buf]);
        umma_commit(&v_empty[st]);
      }
      __syncwarp();
      return true;
    };
    for (int j = 0; ok && j < nkv; ++j) {
      const int st = j % STAGES;
      const int buf = j & 1;
      if (!mbar_wait_bounded_warp(&k_full[st], uint32_t(j / STAGES) & 1u, abort_flag, args.ctl, kStatusTimeoutMma)) {
        ok = false;
        break;
      }
      // S[buf] is free: the softmax read S_{j-2} before it wrote P_{j-2} there (p_full), and P_{j-2} V_{j-2} was
      // issued before this MMA.
      tc_fence_after();
      if (elect_one()) {
        issue_s<DP, BN>(tmem_base + uint32_t(L::kSCol + buf * BN), q_desc, k_desc + uint64_t((st * L::kKVBytes) >> 4),
                        L::kQAtom, L::kKVAtom);
        umma_commit(&s_full[buf]);
        umma_commit(&k_empty[st]);
      }
      __syncwarp();
      if (j >= 1 && !pv_step(j - 1)) {
        ok = false;
        break;
      }
    }
    if (ok && nkv >= 1 && !pv_step(nkv - 1)) ok = false;
    if (!ok) {
      if (elect_one()) umma_commit(drain);
      __syncwarp();
      mbar_wait_drain(drain, 0u, args.ctl);
    }
  } else {
    // ------------------------------------------------------------------ softmax / correction / epilogue (warps 0-3)
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
      // P_j overwrites S_j; P_{j-2} V_{j-2}, the last reader of these columns, completed before s_full of tile j.
      bool move;
      const float alpha = softmax_step<BN, exp_poly_pairs_per8<DP, 1>()>(
          lane_base + uint32_t(L::kSCol + buf * BN), j * BN, args.Skv, c, args.rescale_thr, m, l, move);
      // O correction (rare with the lazy max): O_row *= alpha once P_{j-1} V_{j-1} has landed.
      if (j > 0 && __any_sync(0xffffffffu, move)) {
        if (!mbar_wait_bounded(&pv_done[(j - 1) & 1], uint32_t((j - 1) >> 1) & 1u, abort_flag, args.ctl,
                               kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        rescale_o_row<DP>(lane_base + uint32_t(L::kOCol), alpha);
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
        store_o_row<DP>(lane_base + uint32_t(L::kOCol), args, q0 + warp * 32 + lane, bb, hh, 1.0f / l);
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
// Kernel 2: QT Q tiles (QT x 128 query rows, QT = 2 or 4) per CTA sharing every K/V tile. Softmax warps 4w..4w+3
// serve Q tile w (warp v reaches TMEM lanes 32*(v%4)..+31, so each scheduler holds one warp of every Q tile); warp
// 4 QT is the TMA producer, warp 4 QT + 1 issues every S = Q K^T and warp 4 QT + 2 every O += P V. More Q tiles
// per SM mean more softmax warps in flight per scheduler: the softmax of d <= 64 heads is latency-bound.
// With one MMA warp serving the tiles in order (P_w(t-1) V then S_w(t), tile after tile), each tile's next S waited
// for that warp's whole round: per tile two barrier waits, 7 tcgen05.mma at d <= 64 (S: K = 48 in 3; P V: 64 keys
// in 4) and their commits took ~600 cycles of latency (clock64 timeline on B200), and a d = 40 softmax warpgroup
// idled most of each key step. So S is issued ahead of need by its own warp, and P V by another:
//   * TMEM holds NB S buffers shared by the Q tiles as a ring, then the QT O accumulators. S number k = t QT + w
//     (key tile t, Q tile w) goes into buffer k % NB as soon as the P V of S number k - NB has completed: with
//     NB > QT the next S of a tile is computed while its softmax still works on the current one.
//   * P_w(t) is written as bf16 pairs over the first BN/2 columns of the buffer S_w(t) came from. The P V issuer
//     takes the P's in the same order and frees each buffer with a commit after its P V (buf_free).
//   * The softmax rescales O_w only after P_w(t-1) V has completed (pv_done[w]). NB <= 2 QT keeps that wait's
//     parity unambiguous: S_w(t) went out after the P V of S number tQT + w - NB, so the issuer's in-order
//     completion had already finished P_w(t-2) V.
// ---------------------------------------------------------------------------------------------------------------
template <int QT>
constexpr int attn_mq_threads() {
  return QT * kSoftmaxWarps * 32 + 3 * 32;  // softmax warpgroups, TMA producer, S issuer, P V issuer
}

template <int DP, int BN, int STAGES, int QT>
struct AttnMqLayout {
  static constexpr int kNA = (DP + 63) / 64;
  static constexpr int kQAtom = kAttnBM * kAtomBytesPerRow;  // 16 KB
  static constexpr int kKVAtom = BN * kAtomBytesPerRow;
  static constexpr int kQBytes = kNA * kQAtom;    // one Q tile
  static constexpr int kKVBytes = kNA * kKVAtom;  // one K (or V) tile
  static constexpr int kQOff = 0;                 // Q tiles 0..QT-1
  static constexpr int kKOff = kQOff + QT * kQBytes;
  static constexpr int kVOff = kKOff + STAGES * kKVBytes;
  static constexpr int kBarOff = kVOff + STAGES * kKVBytes;
  // TMEM (all 512 columns): S buffers 0..NB-1 at b * BN, then O_w at kOCol + w * DP.
  static constexpr int kTmemCols = 512;
  static constexpr int kOCol = kTmemCols - QT * DP;
  static constexpr int NB = (kOCol / BN < 2 * QT) ? kOCol / BN : 2 * QT;
  // q_full, k_full[S], v_full[S], k_empty[S], v_empty[S], s_full[NB], p_full[NB], buf_free[NB], pv_done[QT],
  // o_full[QT], drain[2] (one per issuing warp).
  static constexpr int kNumBars = 1 + 4 * STAGES + 3 * NB + 2 * QT + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kSmemBytes = kMiscOff + 16 + 1024;
  static_assert(QT == 2 || QT == 4, "two or four Q tiles per CTA");
  static_assert(DP % 16 == 0 && DP >= 16 && DP <= 192, "padded head dim must be a multiple of 16 in [16, 192]");
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 128, "key tile must be 64, 96 or 128");
  static_assert(NB >= QT, "every Q tile needs an S buffer next to the O tiles in 512 TMEM columns");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

template <int DP, int BN, int STAGES, int QT>
__global__ void __launch_bounds__(attn_mq_threads<QT>(), 1)
    attention_fwd_mq_tcgen05_kernel(const __grid_constant__ CUtensorMap tm_q,
                                    const __grid_constant__ CUtensorMap tm_k,
                                    const __grid_constant__ CUtensorMap tm_v, const AttnArgs args) {
  using L = AttnMqLayout<DP, BN, STAGES, QT>;
  constexpr int NB = L::NB;
  constexpr int kProducerWarp = QT * kSoftmaxWarps;
  constexpr int kSWarp = kProducerWarp + 1;   // S issuer; owns the TMEM allocation
  constexpr int kPvWarp = kProducerWarp + 2;  // P V issuer
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* k_empty = v_full + STAGES;
  uint64_t* v_empty = k_empty + STAGES;
  uint64_t* s_full = v_empty + STAGES;  // [buffer]
  uint64_t* p_full = s_full + NB;       // [buffer]
  uint64_t* buf_free = p_full + NB;     // [buffer]
  uint64_t* pv_done = buf_free + NB;    // [Q tile]
  uint64_t* o_full = pv_done + QT;      // [Q tile]
  uint64_t* drain = o_full + QT;        // [issuer]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOff + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * (QT * kAttnBM);
  const int pair = blockIdx.y;
  const int hh = pair % args.H;
  const int bb = pair / args.H;
  const int nkv = args.nkv;
  const int total = nkv * QT;  // S (and P V) products of the CTA, numbered k = t QT + w

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int b = 0; b < NB; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], kSoftmaxWarps);
      mbar_init(&buf_free[b], 1);
    }
    for (int i = 0; i < QT; ++i) {
      mbar_init(&pv_done[i], 1);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kSWarp) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      pdl_wait();  // q/k/v may be the previous kernel's outputs
      int c0, c1, c2, c3;
      mbar_arrive_expect_tx(q_full, QT * L::kQBytes);
      for (int w = 0; w < QT; ++w)
        for (int a = 0; a < L::kNA; ++a) {
          map_coords(args.pq, a, q0 + w * kAttnBM, hh, bb, c0, c1, c2, c3);
          tma_load_4d(&tm_q, q_full, sQ + w * L::kQBytes + a * L::kQAtom, c0, c1, c2, c3);
        }
      kv_producer<L::kNA, BN, STAGES>(&tm_k, &tm_v, args, sK, sV, k_full, v_full, k_empty, v_empty, abort_flag, hh,
                                      bb);
      mbar_wait_drain(q_full, 0, args.ctl);
    }
  } else if (warp == kSWarp || warp == kPvWarp) {
    // ------------------------------------------------------------------ MMA issuers
    // The whole warp runs the loop (operands stay warp-uniform); one elected lane issues the MMAs and commits.
    const bool s_role = warp == kSWarp;
    uint64_t* my_drain = &drain[s_role ? 0 : 1];
    bool ok = true;
    if (args.ctl.debug & 1u) {
      if (!mbar_wait_bounded_warp(my_drain, 0, abort_flag, args.ctl, kStatusForced)) ok = false;
    }
    if (s_role) {
      // S_w(t) = Q_w K_t^T into buffer k % NB, once the P V that last read that buffer has completed.
      if (ok && !mbar_wait_bounded_warp(q_full, 0, abort_flag, args.ctl, kStatusTimeoutMma)) ok = false;
      tc_fence_after();
      const uint64_t q_desc = smem_desc_kmajor_sw128(smem_u32(sQ));
      const uint64_t k_desc = smem_desc_kmajor_sw128(smem_u32(sK));
      for (int k = 0; ok && k < total; ++k) {
        const int t = k / QT, w = k % QT, b = k % NB, n = k / NB;
        const int st = t % STAGES;
        if (n > 0 && !mbar_wait_bounded_warp(&buf_free[b], uint32_t(n - 1) & 1u, abort_flag, args.ctl,
                                             kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        if (w == 0 && !mbar_wait_bounded_warp(&k_full[st], uint32_t(t / STAGES) & 1u, abort_flag, args.ctl,
                                              kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (elect_one()) {
          issue_s<DP, BN>(tmem_base + uint32_t(b * BN), q_desc + uint64_t((w * L::kQBytes) >> 4),
                          k_desc + uint64_t((st * L::kKVBytes) >> 4), L::kQAtom, L::kKVAtom);
          umma_commit(&s_full[b]);
          if (w == QT - 1) umma_commit(&k_empty[st]);
        }
        __syncwarp();
      }
    } else {
      // O_w += P_w(t) V_t from buffer k % NB, in the order the S products went out; each commit frees the buffer.
      const uint64_t v_desc = smem_desc_mnmajor_sw128(smem_u32(sV), L::kKVAtom);
      for (int k = 0; ok && k < total; ++k) {
        const int t = k / QT, w = k % QT, b = k % NB, n = k / NB;
        const int st = t % STAGES;
        if (w == 0 && !mbar_wait_bounded_warp(&v_full[st], uint32_t(t / STAGES) & 1u, abort_flag, args.ctl,
                                              kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        if (!mbar_wait_bounded_warp(&p_full[b], uint32_t(n) & 1u, abort_flag, args.ctl, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (elect_one()) {
          issue_pv<DP, BN>(tmem_base + uint32_t(L::kOCol + w * DP), tmem_base + uint32_t(b * BN),
                           v_desc + uint64_t((st * L::kKVBytes) >> 4), t > 0);
          umma_commit(&buf_free[b]);
          umma_commit(&pv_done[w]);
          if (w == QT - 1) umma_commit(&v_empty[st]);
          if (t == nkv - 1) umma_commit(&o_full[w]);
        }
        __syncwarp();
      }
    }
    if (!ok) {
      if (elect_one()) umma_commit(my_drain);
      __syncwarp();
      mbar_wait_drain(my_drain, 0u, args.ctl);
    }
  } else {
    // ------------------------------------------------------------------ softmax / correction / epilogue
    const int w = warp >> 2;  // Q tile
    const int wq = warp & 3;  // TMEM lane quarter
    const uint32_t lane_base = tmem_base + (uint32_t(wq * 32) << 16);
    const uint32_t o_addr = lane_base + uint32_t(L::kOCol + w * DP);
    const float c = args.scale_log2;
    float m = -INFINITY;  // running max in log2 units (scores * scale * log2 e)
    float l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int k = j * QT + w;
      const int b = k % NB;
      if (!mbar_wait_bounded(&s_full[b], uint32_t(k / NB) & 1u, abort_flag, args.ctl, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      bool move;
      const float alpha = softmax_step<BN, exp_poly_pairs_per8<DP, QT>()>(lane_base + uint32_t(b * BN), j * BN,
                                                                           args.Skv, c, args.rescale_thr, m, l, move);
      // O correction (rare with the lazy max), once P_w(j-1) V_{j-1} has completed.
      if (j > 0 && __any_sync(0xffffffffu, move)) {
        if (!mbar_wait_bounded(&pv_done[w], uint32_t(j - 1) & 1u, abort_flag, args.ctl, kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        rescale_o_row<DP>(o_addr, alpha);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }
    if (ok && nkv >= 1) {
      pdl_wait();  // the previous kernel may still read the output buffer
      if (mbar_wait_bounded(&o_full[w], 0u, abort_flag, args.ctl, kStatusTimeoutEpilogue)) {
        tc_fence_after();
        store_o_row<DP>(o_addr, args, q0 + w * kAttnBM + wq * 32 + lane, bb, hh, 1.0f / l);
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == kSWarp) {
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

template <typename Kern>
int launch_kernel(Kern kern, int smem_bytes, int threads, bool* configured, const CUtensorMap& mq,
                  const CUtensorMap& mk, const CUtensorMap& mv, const AttnArgs& a, dim3 grid, cudaStream_t st) {
  if (!*configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(attention smem)");
    *configured = true;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, a), "attention kernel launch");
}

template <int DP, int BN, int STAGES>
int launch_qt1(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnArgs& a, dim3 grid,
               cudaStream_t st, int device) {
  static bool configured[64] = {false};
  return launch_kernel(attention_fwd_tcgen05_kernel<DP, BN, STAGES>, Attn1Layout<DP, BN, STAGES>::kSmemBytes,
                       kAttn1Threads, &configured[device], mq, mk, mv, a, grid, st);
}

template <int DP, int BN, int STAGES, int QT>
int launch_mq(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const AttnArgs& a, dim3 grid,
              cudaStream_t st, int device) {
  static bool configured[64] = {false};
  return launch_kernel(attention_fwd_mq_tcgen05_kernel<DP, BN, STAGES, QT>,
                       AttnMqLayout<DP, BN, STAGES, QT>::kSmemBytes, attn_mq_threads<QT>(), &configured[device], mq,
                       mk, mv, a, grid, st);
}

// Kernel variant for a padded head dim, key tile and Q tiles per CTA.
int launch_for(int64_t DP, int BN, int QT, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
               const AttnArgs& a, dim3 grid, cudaStream_t st, int dev) {
#define NPUB200_ATTN_QT1(dp, bn, stages) \
  if (QT == 1 && DP == dp && BN == bn) return launch_qt1<dp, bn, stages>(mq, mk, mv, a, grid, st, dev);
#define NPUB200_ATTN_QT2(dp, bn, stages) \
  if (QT == 2 && DP == dp && BN == bn) return launch_mq<dp, bn, stages, 2>(mq, mk, mv, a, grid, st, dev);
#define NPUB200_ATTN_QT4(dp, bn, stages) \
  if (QT == 4 && DP == dp && BN == bn) return launch_mq<dp, bn, stages, 4>(mq, mk, mv, a, grid, st, dev);
  // One Q tile per CTA. d <= 64 with 64-key tiles: two CTAs per SM.
  NPUB200_ATTN_QT1(16, 64, 5)
  NPUB200_ATTN_QT1(32, 64, 5)
  NPUB200_ATTN_QT1(48, 64, 5)
  NPUB200_ATTN_QT1(64, 64, 5)
  NPUB200_ATTN_QT1(16, 96, 3)
  NPUB200_ATTN_QT1(32, 96, 3)
  NPUB200_ATTN_QT1(48, 96, 3)
  NPUB200_ATTN_QT1(64, 96, 3)
  NPUB200_ATTN_QT1(16, 128, 4)
  NPUB200_ATTN_QT1(32, 128, 4)
  NPUB200_ATTN_QT1(48, 128, 4)
  NPUB200_ATTN_QT1(64, 128, 4)
  NPUB200_ATTN_QT1(80, 64, 2)
  NPUB200_ATTN_QT1(96, 64, 2)
  NPUB200_ATTN_QT1(112, 64, 2)
  NPUB200_ATTN_QT1(128, 64, 2)
  NPUB200_ATTN_QT1(80, 128, 2)
  NPUB200_ATTN_QT1(96, 128, 2)
  NPUB200_ATTN_QT1(112, 128, 2)
  NPUB200_ATTN_QT1(128, 128, 2)
  NPUB200_ATTN_QT1(144, 64, 2)
  NPUB200_ATTN_QT1(160, 64, 2)
  NPUB200_ATTN_QT1(176, 64, 2)
  NPUB200_ATTN_QT1(192, 64, 2)
  NPUB200_ATTN_QT1(208, 64, 2)
  NPUB200_ATTN_QT1(224, 64, 2)
  NPUB200_ATTN_QT1(240, 64, 2)
  NPUB200_ATTN_QT1(256, 64, 2)
  // Two Q tiles per CTA (one CTA per SM).
  NPUB200_ATTN_QT2(16, 64, 6)
  NPUB200_ATTN_QT2(32, 64, 6)
  NPUB200_ATTN_QT2(48, 64, 6)
  NPUB200_ATTN_QT2(64, 64, 6)
  NPUB200_ATTN_QT2(16, 96, 4)
  NPUB200_ATTN_QT2(32, 96, 4)
  NPUB200_ATTN_QT2(48, 96, 4)
  NPUB200_ATTN_QT2(64, 96, 4)
  NPUB200_ATTN_QT2(16, 128, 4)
  NPUB200_ATTN_QT2(32, 128, 4)
  NPUB200_ATTN_QT2(48, 128, 4)
  NPUB200_ATTN_QT2(64, 128, 4)
  NPUB200_ATTN_QT2(80, 64, 4)
  NPUB200_ATTN_QT2(96, 64, 4)
  NPUB200_ATTN_QT2(112, 64, 4)
  NPUB200_ATTN_QT2(128, 64, 4)
  NPUB200_ATTN_QT2(80, 128, 2)
  NPUB200_ATTN_QT2(96, 128, 2)
  NPUB200_ATTN_QT2(112, 128, 2)
  NPUB200_ATTN_QT2(128, 128, 2)
  NPUB200_ATTN_QT2(144, 64, 2)
  NPUB200_ATTN_QT2(160, 64, 2)
  NPUB200_ATTN_QT2(176, 64, 2)
  NPUB200_ATTN_QT2(192, 64, 2)
  // Four Q tiles per CTA (one CTA per SM, 16 softmax warps), 64-key tiles, one S buffer per Q tile: d <= 64.
  NPUB200_ATTN_QT4(16, 64, 6)
  NPUB200_ATTN_QT4(32, 64, 6)
  NPUB200_ATTN_QT4(48, 64, 6)
  NPUB200_ATTN_QT4(64, 64, 6)
#undef NPUB200_ATTN_QT1
#undef NPUB200_ATTN_QT2
#undef NPUB200_ATTN_QT4
  return fail(kErrUnsupported, "no attention variant for padded head dim %lld with %d-key tiles and %d Q tiles per CTA",
              (long long)DP, BN, QT);
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
  // variant = key tile (0 = automatic, 64, 96, 128) + 1000 * Q tiles per CTA (0 = automatic, 1, 2, 4).
  const int QT_req = p.variant / 1000;
  int BN = p.variant % 1000;
  if (p.variant < 0 || QT_req == 3 || QT_req > 4 || (BN != 0 && BN != 64 && BN != 96 && BN != 128))
    return fail(kErrUnsupported, "attention variant %d (key tile 0/64/96/128 plus 1000 x Q tiles per CTA 0/1/2/4)",
                p.variant);
  if (QT_req == 4 && (DP > 64 || (BN != 0 && BN != 64)))
    return fail(kErrUnsupported, "four Q tiles per CTA need head dim <= 64 and 64-key tiles (variant %d)", p.variant);
  // Automatic choice (measured on the SD1.5 blocks at batch 2 and 16):
  //   d <= 64       two Q tiles per CTA with 128-key tiles (three S buffers in the ring) once their grid reaches
  //                 2/3 of the SMs, or 1/3 with at least 2048 keys; else one Q tile with 96-key tiles. Measured at
  //                 d = 40: (2, 8, 4096, 4096) 88 us against 111 with one Q tile, 94 with two of 96-key tiles and 96
  //                 with four; 8 pairs of 4096 (128 two-tile CTAs) 44 against 66 us; 1 pair of 16384 (64) 157
  //                 against 171; 4 pairs of 4096 (64) 43 against 47; 16 pairs of 1024 (64, short keys) 14.2
  //                 against 12.8 with one Q tile; 2 pairs of 4096 (32) 42 against 36.
  //                 Up to 256 keys (one to four 64-key steps, so no S runs ahead and fill and drain dominate): four Q
  //                 tiles per CTA when their grid reaches half the SMs, else one. The cross-attention (2, 8, 4096, 77)
  //                 9.4 us against 12.5 with two Q tiles and 10.7 with one; batch 16 60.5 against 82.9 and 61.7.
  //   64 < d <= 128 one Q tile; 64-key tiles (two CTAs per SM) when the grid fills two per SM, else 128.
  //   d > 128       64-key tiles; two Q tiles per CTA when one-tile CTAs would take more than one wave.
  const int64_t ctas_qt1 = (p.Sq + kAttnBM - 1) / kAttnBM * pairs;
  const int64_t sms = dev->sms;
  int QT = QT_req;
  if (DP <= 64) {
    if (QT == 0) {
      if (p.Skv <= 256) {
        const int64_t ctas_qt4 = (p.Sq + 4 * kAttnBM - 1) / (4 * kAttnBM) * pairs;
        QT = 2 * ctas_qt4 >= sms ? 4 : 1;
      } else {
        const int64_t ctas_qt2 = (p.Sq + 2 * kAttnBM - 1) / (2 * kAttnBM) * pairs;
        QT = (3 * ctas_qt2 >= 2 * sms || (3 * ctas_qt2 >= sms && p.Skv >= 2048)) ? 2 : 1;
      }
    }
    if (BN == 0) BN = QT == 2 ? 128 : 96;
  } else if (DP <= 128) {
    if (QT == 0) QT = 1;
    if (BN == 0) BN = (QT == 1 && ctas_qt1 >= 2 * sms) ? 64 : 128;
  } else {
    if (QT == 0) QT = (DP <= 192 && ctas_qt1 > sms) ? 2 : 1;
    BN = 64;
  }
  if (QT == 2 && DP > 192) return fail(kErrUnsupported, "two Q tiles per CTA need head dim <= 192");
  if (BN == 96 && DP > 64) BN = 64;
  if (QT == 4) BN = 64;

  const int q_rows = QT * kAttnBM;
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
  const int64_t gx = (p.Sq + q_rows - 1) / q_rows;
  if (gx > 0x7fffffff) return fail(kErrInvalid, "too many query tiles");
  const dim3 grid{unsigned(gx), unsigned(pairs), 1u};
  return launch_for(DP, BN, QT, mq, mk, mv, a, grid, stream, dev->device);
}

}  // namespace npub200
