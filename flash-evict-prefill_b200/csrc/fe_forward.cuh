// Attention forward (traversal 1) for sm_100a.
//
// Restates the first KV traversal of `_prefill` (flash_evict/prefill.py:23-60):
// online softmax in the log2 domain (logits * scale * log2e), P cast to the
// input dtype before the PV product, FP32 row max m and row sum l; plus the
// store of O = acc / l (prefill.py:59-60).  In addition it writes the final
// (m, l) of every row so the replay kernel can normalise without a second
// online pass.
//
// CTA work unit: one query block = two 128-row query tiles (Q0, Q1) of one
// query head.  KV tiles are 128 keys.  Roles (384 threads, 3 warpgroups):
//   warps 0-3  softmax for Q0 (thread = TMEM lane = query row)
//   warps 4-7  softmax for Q1
//   warp  8    TMA producer (Q once, K/V through a STAGES-deep ring)
//   warp  9    tcgen05 issuer (one thread) and TMEM owner
//   warps 10-11 idle
// Registers: launched at 168/thread; the producer warpgroup drops to
// FWD_REGS_LOW and the softmax warpgroups rise to FWD_REGS_HIGH
// (2*128*216 + 128*64 = 63488 <= 384*168 = 64512).
// TMEM (512 columns): S0 [0,128), S1 [128,256), O0 [256,256+DV), O1 after.
// P (16-bit) overwrites the first 64 columns of its S tile and feeds the PV
// MMA straight from TMEM (A operand in TMEM, V as an MN-major B operand).
//
// Issue order on the tensor pipe per KV tile j:
//   PV0(j), S0(j+1), PV1(j), S1(j+1)
// so that when softmax t observes S_t(j+1) complete, PV_t(j) has completed
// too and O_t may be rescaled in place.  The O rescale is lazy: the max used
// for exponentiation only moves when the true max exceeds it by more than
// 2^8, which keeps P <= 256 and makes rescales rare.
//
// The softmax is written for the FP32x2 pipe (packed FMA for the exponent
// arguments, packed adds for the row sums) with MUFU ex2 for the
// exponentials.  Measured alternatives that were slower and are not used:
// turn-taking between the two softmax warpgroups, a share of the
// exponentials on the FMA pipe (FWD_POLY, FWD_POLY_PAIRS), scalar FP32
// arithmetic, and double-buffered 64-key S tiles.
#pragma once

#include <type_traits>

#include "fe_ptx.cuh"

namespace fe {

struct FwdParams {
  void* out;          // [B, Hq, N, D] contiguous, input dtype
  float* row_stats;   // [B, Hq, N, 2] {m, l}
  const int32_t* blocks;  // optional list of query blocks (256 rows), heaviest first
  int num_blocks;     // length of `blocks`, or number of blocks when blocks == nullptr
  int B, Hq, Hkv, N, D, G;
  float sc;           // scale * log2(e)
  int causal;
  int vcol0;          // first V / output channel of this launch (0, or 128 for the second half of D > 128)
  uint64_t timeout_ns;
};

// DQK: channels of the QK^T contraction (64, 128 or 256, zero padded); DV:
// channels of V (and O) this launch computes (64 or 128).  Heads with more
// than 128 channels run two launches, one per 128-channel half of V, because
// two 256-column O accumulators do not fit in TMEM next to the S tiles.
template <int DQK, int DV>
struct FwdCfg {
  static constexpr int TILE = 128 * DQK * 2;       // bytes of one 128-row Q or K tile
  static constexpr int VTILE = 128 * DV * 2;       // bytes of one 128-row V tile
  static constexpr int STAGES = (DQK <= 64) ? 4 : (DQK <= 128 ? 2 : 1);
  static constexpr int NCH = DQK / 64;             // 64-column swizzle chunks of Q and K
  static constexpr int NCHV = DV / 64;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = 2 * TILE;
  static constexpr int OFF_V = OFF_K + STAGES * TILE;
  static constexpr int OFF_BAR = OFF_V + STAGES * VTILE;
  // barriers: q_full, k_full[S], v_full[S], k_empty[S], v_empty[S], s_full[2], p_full[2], o_full[2], drain
  static constexpr int NBAR = 1 + 4 * STAGES + 7;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + tmem holder/abort + alignment slack
  static constexpr int THREADS = 384;
};

// Exponentials per 16 computed by exp2_poly instead of MUFU ex2.
constexpr int FWD_POLY = 0;
// Exponential pairs per 8 (16 exponentials) computed by exp2_poly_x2 (packed
// FP32x2 on the FMA pipe) instead of MUFU ex2.  Measured at 2/3/4 pairs: the
// attention kernel got 3 %/7 %/13 % slower (c3), so MUFU throughput is not
// what bounds this softmax; kept at 0.
#ifndef FE_FWD_POLY_PAIRS
#define FE_FWD_POLY_PAIRS 0
#endif
constexpr int FWD_POLY_PAIRS = FE_FWD_POLY_PAIRS;
// Lazy rescale threshold (log2 units): the max used for the exponentials only
// moves when the row's true max exceeds it by more than this, so P <= 2^this.
constexpr float FWD_RESCALE_LOG2 = 8.0f;

constexpr uint32_t FWD_REGS_HIGH = 216;
constexpr uint32_t FWD_REGS_LOW = 64;
// Registers per thread the launch must provide for the split above.
constexpr int FWD_REGS_NEEDED = (2 * 128 * FWD_REGS_HIGH + 128 * FWD_REGS_LOW + 383) / 384;

// One softmax exponential pass over a 128-column row: p = 2^(x*sce - m) with
// packed FP32x2 FMAs for the arguments, MUFU ex2 for the exponentials (POLY of
// every 16 on the FMA pipe instead), packed adds into four pair accumulators,
// and optionally the largest argument.  Returns the row sum; P is packed into pk.
template <bool BF16, int POLY, bool TRACK_MAX, int POLYP = 0>
__device__ __forceinline__ float softmax_exp_pass(const float (&x)[128], float sce, float m, uint32_t (&pk)[64],
                                                  float& amax) {
  const uint64_t sc2 = f2_pack(sce, sce);
  const uint64_t nm2 = f2_pack(-m, -m);
  uint64_t acc2[4];
  float am[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    acc2[c] = 0ull;
    am[c] = -INFINITY;
  }
#pragma unroll
  for (int c = 0; c < 128; c += 2) {
    const uint64_t a2 = f2_fma(f2_pack(x[c], x[c + 1]), sc2, nm2);
    float a0, a1;
    f2_unpack(a2, a0, a1);
    if (TRACK_MAX) am[(c >> 1) & 3] = fmax3(am[(c >> 1) & 3], a0, a1);
    float p0, p1;
    uint64_t p2;
    if (((c >> 1) & 7) < POLYP) {
      p2 = exp2_poly_x2(a2);
      f2_unpack(p2, p0, p1);
    } else {
      p0 = ((c & 15) >= 16 - POLY) ? exp2_poly(a0) : ex2_approx(a0);
      p1 = (((c + 1) & 15) >= 16 - POLY) ? exp2_poly(a1) : ex2_approx(a1);
      p2 = f2_pack(p0, p1);
    }
    acc2[(c >> 1) & 3] = f2_add(acc2[(c >> 1) & 3], p2);
    pk[c >> 1] = pack2<BF16>(p0, p1);
  }
  amax = fmaxf(fmaxf(am[0], am[1]), fmaxf(am[2], am[3]));
  float sacc[8];
#pragma unroll
  for (int c = 0; c < 4; ++c) f2_unpack(acc2[c], sacc[2 * c], sacc[2 * c + 1]);
  return ((sacc[0] + sacc[1]) + (sacc[2] + sacc[3])) + ((sacc[4] + sacc[5]) + (sacc[6] + sacc[7]));
}

// Row maximum of the scaled logits (x * sce), eight independent 3-input-max chains.
__device__ __forceinline__ float row_max_scaled(const float (&x)[128], float sce) {
  float mm[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) mm[c] = x[c];
#pragma unroll
  for (int c = 8; c < 128; c += 2) mm[(c >> 1) & 7] = fmax3(mm[(c >> 1) & 7], x[c], x[c + 1]);
  return fmax3(fmax3(mm[0], mm[1], mm[2]), fmax3(mm[3], mm[4], mm[5]), fmaxf(mm[6], mm[7])) * sce;
}

// One KV tile of a query row's softmax, with S already in registers: scale
// and mask (GENERAL only: columns past `lim` get -inf), row max, lazy O
// rescale, exponentials, row sum and the P store over the first 64 columns of
// the S tile.
template <bool BF16, int DV, bool GENERAL>
__device__ __forceinline__ void fwd_softmax_tile(float (&x)[128], int j, int lim, float sc, float sce, bool sc_pos,
                                                 float& m_used, float& l, uint32_t tS, uint32_t tO) {
  if constexpr (GENERAL) {
    if (!sc_pos) {
#pragma unroll
      for (int c = 0; c < 128; ++c) x[c] *= sc;
    }
#pragma unroll
    for (int c = 0; c < 128; ++c) x[c] = (c <= lim) ? x[c] : -INFINITY;
  }
  // Row max first.  The max used for the exponentials only moves when the
  // true max exceeds it by more than 2^8 (lazy rescale); tracking the max
  // inside the exponential pass instead was measured slower (extreme logits
  // force frequent redo passes).
  const float m_new = fmaxf(m_used, row_max_scaled(x, sce));
  if (j == 0) {
    m_used = m_new;
  } else if (__any_sync(0xffffffffu, m_new > m_used + FWD_RESCALE_LOG2)) {
    // Rescale this warp's O rows; PV_t(j-1) is complete (see the header).
    const float f = ex2_approx(m_used - m_new);
    l *= f;
    m_used = m_new;
#pragma unroll 1
    for (int c0 = 0; c0 < DV; c0 += 32) {
      uint32_t o[32];
      tmem_ld32_sync(tO + c0, o);
#pragma unroll
      for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * f);
      tmem_st32(tO + c0, o);
    }
    tmem_wait_st();
  }
  uint32_t pk[64];
  float amax;
  l += softmax_exp_pass<BF16, FWD_POLY, false, FWD_POLY_PAIRS>(x, sce, m_used, pk, amax);
  tmem_st32(tS, pk);
  tmem_st32(tS + 32, pk + 32);
  tmem_wait_st();
}

template <bool BF16, int DQK, int DV>
__global__ void __launch_bounds__(384, 1)
    fe_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const FwdParams p) {
  using C = FwdCfg<DQK, DV>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + C::STAGES;
  uint64_t* k_empty = v_full + C::STAGES;
  uint64_t* v_empty = k_empty + C::STAGES;
  uint64_t* s_full = v_empty + C::STAGES;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* drain = o_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + C::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;

  // ---- work item: (query block, b, hkv, g) ----
  // Causal: heaviest query blocks first (longest-processing-time order), the G
  // heads of a group adjacent so they share K/V in L2.  Non-causal: every
  // block costs the same, so the blocks of one head are adjacent instead and
  // share that head's K/V.
  int item = blockIdx.x;
  int g, hkv, b, rank;
  if (p.causal) {
    g = item % p.G;
    item /= p.G;
    hkv = item % p.Hkv;
    item /= p.Hkv;
    b = item % p.B;
    rank = item / p.B;
  } else {
    rank = item % p.num_blocks;
    item /= p.num_blocks;
    g = item % p.G;
    item /= p.G;
    hkv = item % p.Hkv;
    b = item / p.Hkv;
  }
  int blk;
  if (p.blocks != nullptr) {
    blk = p.blocks[rank];
  } else {
    blk = p.causal ? (p.num_blocks - 1 - rank) : rank;
  }
  const int hq = hkv * p.G + g;
  const int nkv = (p.N + 127) / 128;
  const int row0 = blk * 256;
  const int row1 = row0 + 128;
  const int n0 = (row0 < p.N) ? (p.causal ? min(nkv, row0 / 128 + 1) : nkv) : 0;
  const int n1 = (row1 < p.N) ? (p.causal ? min(nkv, row1 / 128 + 1) : nkv) : 0;
  const int nmax = max(n0, n1);

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(q_full, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_full[t], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    __syncwarp();
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint64_t TO = p.timeout_ns;

  if (warp >= 8) {
  setmaxnreg_dec<FWD_REGS_LOW>();
  if (warp == 8) {
    // ------------------------------------------------------------ producer --
    if (lane == 0 && nmax > 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      tma_prefetch_desc(&tv);
      uint32_t loads[C::STAGES];
      for (int s = 0; s < C::STAGES; ++s) loads[s] = 0;
      // Q is read once; K/V are re-read by every query block of the head
      // group: keep them in L2 ahead of the streaming Q reads and O writes.
      const uint64_t pol_q = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();
      mbar_expect_tx(q_full, ((n0 > 0) + (n1 > 0)) * C::TILE);
      for (int c = 0; c < C::NCH; ++c) {
        if (n0 > 0) tma_load_4d_hint(smem + C::OFF_Q + c * 16384, &tq, q_full, c * 64, row0, hq, b, pol_q);
        if (n1 > 0) tma_load_4d_hint(smem + C::OFF_Q + C::TILE + c * 16384, &tq, q_full, c * 64, row1, hq, b, pol_q);
      }
      bool ok = true;
      for (int j = 0; j < nmax && ok; ++j) {
        const int s = j % C::STAGES;
        const uint32_t use = j / C::STAGES;
        if (use > 0) ok = mbar_wait(&k_empty[s], (use - 1) & 1, TO, abort_flag);
        if (!ok) break;
        mbar_expect_tx(&k_full[s], C::TILE);
        for (int c = 0; c < C::NCH; ++c)
          tma_load_4d_hint(smem + C::OFF_K + s * C::TILE + c * 16384, &tk, &k_full[s], c * 64, j * 128, hkv, b,
                           pol_kv);
        if (use > 0) ok = mbar_wait(&v_empty[s], (use - 1) & 1, TO, abort_flag);
        if (!ok) {
          loads[s] = use * 2 + 1;  // K of this use in flight, V not issued
          break;
        }
        mbar_expect_tx(&v_full[s], C::VTILE);
        for (int c = 0; c < C::NCHV; ++c)
          tma_load_4d_hint(smem + C::OFF_V + s * C::VTILE + c * 16384, &tv, &v_full[s], p.vcol0 + c * 64, j * 128,
                           hkv, b, pol_kv);
        loads[s] = use * 2 + 2;
      }
      // Never leave the CTA with a TMA write in flight: wait for the last load
      // issued into each stage (already complete on the normal path).
      mbar_wait_inflight(q_full, 0, TO);
      for (int s = 0; s < C::STAGES; ++s) {
        if (loads[s] == 0) continue;
        const uint32_t use = (loads[s] - 1) / 2;
        mbar_wait_inflight(&k_full[s], use & 1, TO);
        if (loads[s] % 2 == 0) mbar_wait_inflight(&v_full[s], use & 1, TO);
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0 && nmax > 0) {
      constexpr uint32_t ID_S = idesc_f16(128, 128, BF16, false);
      constexpr uint32_t ID_PV = idesc_f16(128, DV, BF16, true);
      const uint32_t q_addr = smem_u32(smem + C::OFF_Q);
      const uint32_t k_addr = smem_u32(smem + C::OFF_K);
      const uint32_t v_addr = smem_u32(smem + C::OFF_V);
      // Descriptors are computed once; a k-step or a stage only moves the
      // start-address field (address >> 4 in the low 14 bits), so it is a
      // plain 32-bit add on the descriptor's low word.
      const uint64_t dq = smem_desc_sw128(q_addr, 16, 1024);
      const uint64_t dk = smem_desc_sw128(k_addr, 16, 1024);
      const uint64_t dv = smem_desc_sw128(v_addr, 16384, 1024);
      constexpr uint64_t TILE16 = C::TILE >> 4;
      constexpr uint64_t VTILE16 = C::VTILE >> 4;
      const uint32_t dq_hi = static_cast<uint32_t>(dq >> 32), dk_hi = static_cast<uint32_t>(dk >> 32);
      const uint32_t dv_hi = static_cast<uint32_t>(dv >> 32);
      auto issue_s = [&](int t, int s) {
        const uint32_t a = static_cast<uint32_t>(dq) + t * static_cast<uint32_t>(TILE16);
        const uint32_t bb = static_cast<uint32_t>(dk) + s * static_cast<uint32_t>(TILE16);
        const uint32_t d = tmem + t * 128;
#pragma unroll 8
        for (int kk = 0; kk < DQK / 16; ++kk) {
          const uint32_t off = static_cast<uint32_t>(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
          umma_ss_lohi(d, a + off, dq_hi, bb + off, dk_hi, ID_S, kk > 0);
        }
      };
      auto issue_pv = [&](int t, int s, int j) {
        const uint32_t bb = static_cast<uint32_t>(dv) + s * static_cast<uint32_t>(VTILE16);
        const uint32_t d = tmem + 256 + t * DV;
        const uint32_t pa = tmem + t * 128;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          umma_ts_lohi(d, pa + kk * 8, bb + static_cast<uint32_t>(kk * (2048 >> 4)), dv_hi, ID_PV,
                       (j > 0 || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, TO, abort_flag);
      if (ok) ok = mbar_wait(&k_full[0], 0, TO, abort_flag);
      if (ok) {
        tc_fence_after();
        if (n0 > 0) {
          issue_s(0, 0);
          umma_commit(&s_full[0]);
        }
        if (n1 > 0) {
          issue_s(1, 0);
          umma_commit(&s_full[1]);
        }
        if (C::STAGES < nmax) umma_commit(&k_empty[0]);
      }
      for (int j = 0; j < nmax && ok; ++j) {
        const int s = j % C::STAGES;
        const int s2 = (j + 1) % C::STAGES;
        const bool next = (j + 1 < nmax);
        bool k_next_ready = false;
        ok = mbar_wait(&v_full[s], (j / C::STAGES) & 1, TO, abort_flag);
        if (!ok) break;
        for (int t = 0; t < 2 && ok; ++t) {
          const int nt = t == 0 ? n0 : n1;
          if (j >= nt) continue;
          ok = mbar_wait(&p_full[t], j & 1, TO, abort_flag);
          if (!ok) break;
          tc_fence_after();
          issue_pv(t, s, j);
          if (j + 1 < nt) {
            if (!k_next_ready) {
              ok = mbar_wait(&k_full[s2], ((j + 1) / C::STAGES) & 1, TO, abort_flag);
              if (!ok) break;
              tc_fence_after();
              k_next_ready = true;
            }
            issue_s(t, s2);
            umma_commit(&s_full[t]);
          } else {
            umma_commit(&o_full[t]);
          }
        }
        if (!ok) break;
        // Release the stages only when the producer will refill them.
        if (j + C::STAGES < nmax) umma_commit(&v_empty[s]);
        if (next && (j + 1 + C::STAGES < nmax)) umma_commit(&k_empty[s2]);
      }
      // Drain: every MMA issued above has completed once this returns.
      umma_commit(drain);
      mbar_wait_inflight(drain, 0, TO);
    }
  }
  } else {
    setmaxnreg_inc<FWD_REGS_HIGH>();
    // ------------------------------------------------------------- softmax --
    const int t = warp >> 2;
    const int nt = t == 0 ? n0 : n1;
    const int rbase = t == 0 ? row0 : row1;
    const int r = ((warp & 3) << 5) + static_cast<int>(lane);
    const int row = rbase + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + 256 + t * DV;
    const float sc = p.sc;
    // Positive scale: max on raw logits, scale folded into one FFMA per
    // element.  Otherwise scale first and use an effective scale of 1.
    const bool sc_pos = sc > 0.f;
    const float sce = sc_pos ? sc : 1.0f;
    float m_used = -INFINITY;
    float l = 0.f;
    bool ok = true;
    // KV tiles that need per-element work (the diagonal tiles of a causal
    // block, the ragged end of N; every tile for a non-positive scale) come
    // last and run in a loop of their own, so the loop over all other tiles
    // carries no masking code.
    int n_plain = p.causal ? min(nt, rbase / 128) : nt;
    if ((p.N % 128) != 0 && n_plain == nkv) n_plain = nkv - 1;
    if (!sc_pos) n_plain = 0;
    auto tile_step = [&](int j, auto general) -> bool {
      if (!warp_all(mbar_wait(&s_full[t], j & 1, TO, abort_flag))) return false;
      tc_fence_after();
      float x[128];
      {
        uint32_t* xr = reinterpret_cast<uint32_t*>(x);
        tmem_ld64_sync(tS, xr);
        tmem_ld64_sync(tS + 64, xr + 64);
      }
      const int lim = (p.causal ? min(p.N - 1, row) : (p.N - 1)) - j * 128;
      fwd_softmax_tile<BF16, DV, decltype(general)::value>(x, j, lim, sc, sce, sc_pos, m_used, l, tS, tO);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
      return true;
    };
    for (int j = 0; j < n_plain && ok; ++j) ok = tile_step(j, std::false_type{});
    for (int j = n_plain; j < nt && ok; ++j) ok = tile_step(j, std::true_type{});
    if (nt > 0 && ok) ok = warp_all(mbar_wait(&o_full[t], 0, TO, abort_flag));
    if (nt > 0 && !ok && row < p.N) {
      // Aborted (watchdog): mark this row's statistics and output channels
      // as NaN so that nothing downstream (the replay, a caller reading the
      // output) mistakes stale memory for a result.
      if (p.vcol0 == 0) {
        float2* st = reinterpret_cast<float2*>(p.row_stats) + (static_cast<size_t>(b) * p.Hq + hq) * p.N + row;
        *st = make_float2(__int_as_float(0x7fffffff), __int_as_float(0x7fffffff));
      }
      using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
      T* orow = reinterpret_cast<T*>(p.out) + ((static_cast<size_t>(b) * p.Hq + hq) * p.N + row) * p.D + p.vcol0;
      const uint16_t nan16 = BF16 ? 0x7fc0 : 0x7e00;
      for (int c = 0; c < DV && c < p.D - p.vcol0; ++c) reinterpret_cast<uint16_t*>(orow)[c] = nan16;
    }
    if (nt > 0 && ok) {
      {
        tc_fence_after();
        const bool live = row < p.N;
        if (live && p.vcol0 == 0) {
          float2* st = reinterpret_cast<float2*>(p.row_stats) + (static_cast<size_t>(b) * p.Hq + hq) * p.N + row;
          *st = make_float2(m_used, l);
        }
        const float inv = 1.0f / l;
        using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
        T* orow = reinterpret_cast<T*>(p.out) + ((static_cast<size_t>(b) * p.Hq + hq) * p.N + row) * p.D + p.vcol0;
        const int dlim = p.D - p.vcol0;  // channels of this launch's half that exist
        const bool vec = (p.D % 8) == 0;
#pragma unroll 1
        for (int c0 = 0; c0 < DV; c0 += 32) {
          uint32_t o[32];
          tmem_ld32_sync(tO + c0, o);
          if (live && c0 < dlim) {
            uint32_t w[16];
#pragma unroll
            for (int c = 0; c < 16; ++c)
              w[c] = pack2<BF16>(__uint_as_float(o[2 * c]) * inv, __uint_as_float(o[2 * c + 1]) * inv);
            if (vec) {
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4) {
                if (c0 + q4 * 8 < dlim)
                  __stcs(reinterpret_cast<uint4*>(orow + c0 + q4 * 8),
                         make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]));  // streaming (evict first)
              }
            } else {
              const uint16_t* h = reinterpret_cast<const uint16_t*>(w);
              for (int c = 0; c < 32 && c0 + c < dlim; ++c) reinterpret_cast<uint16_t*>(orow)[c0 + c] = h[c];
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fe
