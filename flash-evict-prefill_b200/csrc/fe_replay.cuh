// Exact per-KV-token importance by replay (traversal 2) for sm_100a.
//
// Restates the replay loop of `_prefill` (flash_evict/prefill.py:61-83) and
// the zero-initialised score buffer it accumulates into (prefill.py:129):
//   I[b,hkv,k] = ||v_k||_1 * sum_{g,q} w_q * exp2(s_qk*scale*log2e - m_q) / l_q
//   w_q = exp(decay * (q - (N-1))) * [q >= N - W]
// but key-stationary instead of query-stationary: one CTA owns 128 keys of
// one (b, hkv) and walks every scored (query tile, group head) pair, computing
// S^T = K Q^T on the tensor cores with keys on the TMEM lanes.  Each thread
// owns one key, so the reduction over queries is a register sum with no
// shuffles and no atomics, and every importance element is stored exactly
// once (deterministic, no zero-fill launch).
//
// The per-query normaliser and weight fold into one exponent bias:
//   w_q / l_q * exp2(x - m_q) = exp2(x - bias_q),
//   bias_q = m_q + log2(l_q) - decay*log2(e)*(q - (N-1))
// with bias_q = +inf for rows outside the window or past N.  The reduction
// needs more exponentials than MUFU delivers per S^T MMA, so a share of them
// (REPLAY_POLY_PAIRS column pairs of every 8) runs on the FMA pipe as a packed
// FP32x2 polynomial (exp2_poly_x2, relative error < 3e-6), and the exponent
// arithmetic uses packed FP32x2 too.  Query tiles whose every weight is below
// 2^-127 (decay * distance beyond ~88) are skipped.
//
// Roles: REPLAY_WGS reduce warpgroups (thread = key) -- warpgroup w takes
// items w, w+WGS, w+2*WGS, ...; item i's S^T lives in TMEM buffer i % NBUF
// (columns [128*(i % NBUF), +128)), NBUF = WGS * REPLAY_SBUF -- then the TMA
// producer warp (K once, Q through an NBUF-deep ring) and the tcgen05 issuer /
// TMEM owner warp.  4 warpgroups with one CTA per SM, or 2 with two CTAs per SM: either
// way every SM sub-partition has four reduce warps to keep its MUFU busy.
// The warpgroups' FP64 sums of a key are added in a fixed order at the end
// (deterministic).
#pragma once

#include <type_traits>

#include "fe_ptx.cuh"

namespace fe {

struct ReplayParams {
  const float* row_stats;   // [B, Hq, N, 2]
  float* importance;        // [B, Hkv, N]
  const uint8_t* v;         // V base pointer (bytes)
  int64_t v_sb, v_sh, v_sn; // V strides in elements
  const int32_t* blocks;    // optional query-block list (256-row blocks)
  int num_blocks;
  int B, Hq, Hkv, N, D, G;
  float sc;                 // scale * log2(e)
  float decay_log2;         // recency_decay * log2(e)
  int s_lo;                 // first scored row (window and underflow cut)
  int causal, weighted;
  int kt0, nkt;             // key tiles [kt0, kt0 + nkt) of this launch
  uint64_t timeout_ns;
};

// Column pairs per 8 (off the diagonal tile) exponentiated by exp2_poly_x2
// on the FMA pipe instead of MUFU ex2: the reduction needs 16384
// exponentials per 512-cycle S^T MMA, more than MUFU delivers in that time.
#ifndef FE_REPLAY_POLY_PAIRS
#define FE_REPLAY_POLY_PAIRS 2
#endif
constexpr int REPLAY_POLY_PAIRS = FE_REPLAY_POLY_PAIRS;
// Reduce warpgroups per CTA and S^T buffers per warpgroup; TMEM holds
// 4 buffers per SM, so CTAs per SM = 4 / (WGS * SBUF).  Double-buffered S^T
// (SBUF 2: WGS 2 with one CTA per SM, or WGS 1 with two) measured 10-25 %
// slower than 2 x 1 with two CTAs per SM: four reduce warps per SM
// sub-partition matter more than hiding the S^T MMA behind the reduction.
constexpr int REPLAY_WGS = 2;
constexpr int REPLAY_SBUF = 1;

template <int DP>
struct ReplayCfg {
  static constexpr int WGS = REPLAY_WGS;            // reduce warpgroups
  static constexpr int NBUF = WGS * REPLAY_SBUF;    // S^T buffers; item i uses buffer i % NBUF
  static constexpr int CTAS_PER_SM = 4 / NBUF;      // TMEM: NBUF*128 columns per CTA
  static constexpr int TILE = 128 * DP * 2;
  static constexpr int QST = (DP <= 128) ? NBUF : 2;  // Q tile ring depth (shared memory)
  static constexpr int NCH = DP / 64;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_Q = TILE;
  static constexpr int OFF_BIAS = OFF_Q + QST * TILE;           // float[16 warps][2][128]
  static constexpr int OFF_RED = OFF_BIAS + WGS * 4 * 256 * 4;  // double[WGS][128]
  static constexpr int OFF_MAP = OFF_RED + WGS * 128 * 8;       // uint32 bitmap of listed query blocks
  static constexpr int MAP_WORDS = 256;                         // up to 8192 blocks
  static constexpr int OFF_BAR = OFF_MAP + MAP_WORDS * 4;
  // k_full, q_full[QST], q_empty[QST], s_full[NBUF], s_free[NBUF], drain
  static constexpr int NBAR = 1 + 2 * QST + 2 * NBUF + 1;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static constexpr int PRODUCER = WGS * 4;          // warp indices
  static constexpr int ISSUER = WGS * 4 + 1;
  static constexpr int THREADS = (WGS * 4 + 2) * 32;
};

// Iterates the CTA's (query tile, head-in-group) items in a fixed order.
struct ReplayItems {
  int qt, qt_end, g, G;
  const uint32_t* map;  // nullptr: every query tile
  __device__ __forceinline__ bool listed(int tile) const {
    if (map == nullptr) return true;
    const int blk = tile >> 1;
    return (map[blk >> 5] >> (blk & 31)) & 1u;
  }
  __device__ __forceinline__ void init(int lo, int hi, int groups, const uint32_t* m) {
    qt = lo;
    qt_end = hi;
    g = 0;
    G = groups;
    map = m;
    while (qt < qt_end && !listed(qt)) ++qt;
  }
  __device__ __forceinline__ bool valid() const { return qt < qt_end; }
  __device__ __forceinline__ void advance(int n) {
    for (int i = 0; i < n && valid(); ++i) next();
  }
  __device__ __forceinline__ void next() {
    if (++g == G) {
      g = 0;
      ++qt;
      while (qt < qt_end && !listed(qt)) ++qt;
    }
  }
};

template <bool BF16, int DP>
__global__ void __launch_bounds__(ReplayCfg<DP>::THREADS, ReplayCfg<DP>::CTAS_PER_SM)
    fe_replay_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const ReplayParams p) {
  using C = ReplayCfg<DP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sbias = reinterpret_cast<float*>(smem + C::OFF_BIAS);
  double* sred = reinterpret_cast<double*>(smem + C::OFF_RED);
  uint32_t* smap = reinterpret_cast<uint32_t*>(smem + C::OFF_MAP);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* k_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = q_full + C::QST;
  uint64_t* s_full = q_empty + C::QST;
  uint64_t* s_free = s_full + C::NBUF;
  uint64_t* drain = s_free + C::NBUF;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + C::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;

  // ---- work item: (key tile, b, hkv) ----
  // Non-causal: every key tile has the same work; the key tiles of one
  // (b, hkv) are adjacent so the CTAs that stream the same Q rows run together
  // and share them in L2.  Causal: key tile kt has work proportional to the
  // query tiles at or after it, so the key tiles are issued in ascending order
  // across all (b, hkv) (heaviest first, longest-processing-time order).
  const int nqt = (p.N + 127) / 128;
  int kt, hkv, b;
  if (p.causal) {
    const int nbh = p.B * p.Hkv;
    kt = blockIdx.x / nbh;
    const int bh = blockIdx.x - kt * nbh;
    hkv = bh % p.Hkv;
    b = bh / p.Hkv;
  } else {
    int item = blockIdx.x;
    kt = item % p.nkt;
    item /= p.nkt;
    hkv = item % p.Hkv;
    b = item / p.Hkv;
  }
  kt += p.kt0;
  const int qt_lo = max(p.s_lo / 128, p.causal ? kt : 0);
  const uint32_t* map = nullptr;

  if (p.blocks != nullptr) {
    for (int i = threadIdx.x; i < C::MAP_WORDS; i += blockDim.x) smap[i] = 0;
  }
  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(k_full, 1);
    for (int s = 0; s < C::QST; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    for (int s = 0; s < C::NBUF; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == C::ISSUER) {
    __syncwarp();
    tmem_alloc(tmem_holder, C::NBUF * 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (p.blocks != nullptr) {
    for (int i = threadIdx.x; i < p.num_blocks; i += blockDim.x) {
      const int blk = p.blocks[i];
      atomicOr(&smap[blk >> 5], 1u << (blk & 31));
    }
    __syncthreads();
    map = smap;
  }
  const uint32_t tmem = *tmem_holder;
  const uint64_t TO = p.timeout_ns;

  if (warp == C::PRODUCER) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      ReplayItems it;
      it.init(qt_lo, nqt, p.G, map);
      uint32_t issued = 0;
      if (it.valid()) {
        mbar_expect_tx(k_full, C::TILE);
        for (int c = 0; c < C::NCH; ++c)
          tma_load_4d(smem + C::OFF_K + c * 16384, &tk, k_full, c * 64, kt * 128, hkv, b);
        bool ok = true;
        for (; it.valid(); it.next(), ++issued) {
          const int s = issued % C::QST;
          const uint32_t use = issued / C::QST;
          if (use > 0) ok = mbar_wait(&q_empty[s], (use - 1) & 1, TO, abort_flag);
          if (!ok) break;
          mbar_expect_tx(&q_full[s], C::TILE);
          const int hq = hkv * p.G + it.g;
          for (int c = 0; c < C::NCH; ++c)
            tma_load_4d(smem + C::OFF_Q + s * C::TILE + c * 16384, &tq, &q_full[s], c * 64, it.qt * 128, hq, b);
        }
        // Every load must have landed before the CTA exits.
        mbar_wait_inflight(k_full, 0, TO);
        for (uint32_t i = (issued > C::QST ? issued - C::QST : 0); i < issued; ++i)
          mbar_wait_inflight(&q_full[i % C::QST], (i / C::QST) & 1, TO);
      }
    }
  } else if (warp == C::ISSUER) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t ID_S = idesc_f16(128, 128, BF16, false);
      const uint64_t dk = smem_desc_sw128(smem_u32(smem + C::OFF_K), 16, 1024);
      const uint64_t dq = smem_desc_sw128(smem_u32(smem + C::OFF_Q), 16, 1024);
      const uint32_t dk_lo = static_cast<uint32_t>(dk), dk_hi = static_cast<uint32_t>(dk >> 32);
      const uint32_t dq_lo = static_cast<uint32_t>(dq), dq_hi = static_cast<uint32_t>(dq >> 32);
      ReplayItems it;
      it.init(qt_lo, nqt, p.G, map);
      if (it.valid()) {
        bool ok = mbar_wait(k_full, 0, TO, abort_flag);
        uint32_t i = 0;
        for (; it.valid() && ok; it.next(), ++i) {
          const int s = i % C::QST;
          const int sb = i % C::NBUF;
          ok = mbar_wait(&q_full[s], (i / C::QST) & 1, TO, abort_flag);
          if (!ok) break;
          if (i >= C::NBUF) ok = mbar_wait(&s_free[sb], ((i / C::NBUF) - 1) & 1, TO, abort_flag);
          if (!ok) break;
          tc_fence_after();
          // Descriptor low words step by (address offset >> 4); no carry leaves
          // the 14-bit start-address field (shared memory is below 256 KB).
          const uint32_t qa = dq_lo + static_cast<uint32_t>(s * (C::TILE >> 4));
#pragma unroll
          for (int kk = 0; kk < DP / 16; ++kk) {
            const uint32_t off = static_cast<uint32_t>(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
            umma_ss_lohi(tmem + sb * 128, dk_lo + off, dk_hi, qa + off, dq_hi, ID_S, kk > 0);
          }
          umma_commit(&s_full[sb]);
          umma_commit(&q_empty[s]);
        }
        umma_commit(drain);
        mbar_wait_inflight(drain, 0, TO);
      }
    }
  } else {
    // ------------------------------------------------ reduce (thread = key) --
    const int wg = warp >> 2;                              // this warpgroup's items: wg, wg+4, ...
    const int kr = ((warp & 3) << 5) + static_cast<int>(lane);  // key row in tile
    const int key = kt * 128 + kr;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const uint32_t tS0 = tmem + lane_off;
    const float sc = p.sc;
    double acc = 0.0;
    ReplayItems it;
    it.init(qt_lo, nqt, p.G, map);
    it.advance(wg);
    // Row statistics {m, l} of an item's 128 query rows (4 per lane).
    auto load_stats = [&](const ReplayItems& x, float2* dst) {
      const float2* st =
          reinterpret_cast<const float2*>(p.row_stats) + (static_cast<size_t>(b) * p.Hq + hkv * p.G + x.g) * p.N;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int q = x.qt * 128 + static_cast<int>(lane) + 32 * u;
        dst[u] = (q < p.N && q >= p.s_lo) ? ld_global_f2_pinned(st + q) : make_float2(0.f, 1.f);
      }
    };
    // Exponent bias of an item's 128 query columns, stored negated (the
    // exponent is x*sc + bias) into one of this warp's two bias buffers;
    // lane l fills columns l, l+32, l+64, l+96, so no cross-warp barrier.
    auto write_bias = [&](int qt, const float2* ml, float* dst) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = static_cast<int>(lane) + 32 * u;
        const int q = qt * 128 + c;
        float bias = INFINITY;
        // l >= 1 for every attended row; a row without statistics (l == 0,
        // the zeros a query-sharded rank holds for rows it did not compute)
        // is treated as unscored rather than producing inf.  NaN statistics
        // (an aborted attention launch) give a NaN bias, which poisons every
        // key the row reaches.
        if (q < p.N && q >= p.s_lo && !(ml[u].y <= 0.f))
          bias = fmaf(-p.decay_log2, static_cast<float>(q - (p.N - 1)), ml[u].x + lg2_approx(ml[u].y));
        dst[c] = -bias;
      }
    };
    // The bias of this warpgroup's next item is computed while the current one
    // is reduced; the statistics of the one after are prefetched then.
    float2 ml_next[4];
    if (it.valid()) {
      float2 ml0[4];
      load_stats(it, ml0);
      write_bias(it.qt, ml0, sbias + warp * 256);
      ReplayItems nx = it;
      nx.advance(C::WGS);
      if (nx.valid()) load_stats(nx, ml_next);
    }
    uint32_t li = 0;  // this warpgroup's item count
    bool ok = true;
    const uint64_t sc2 = f2_pack(sc, sc);
    // One item: wait for its S^T, reduce it into `acc`, release the buffer.
    // The diagonal tile (causal, query tile == key tile) is its own
    // instantiation: columns q < key are masked to -inf and every
    // exponential runs on MUFU, so masked entries are exactly 0.  Elsewhere
    // REPLAY_POLY_PAIRS column pairs of every 8 are exponentiated on the FMA
    // pipe (exp2_poly_x2, packed) and the rest on MUFU.  The diagonal items
    // come first in a CTA's item order, so the two instantiations run as two
    // loops one after the other, each with straight-line code per item
    // (branching per 32-column quarter instead measured 7-8 % slower).
    auto process_item = [&](auto diag_tag) -> bool {
      constexpr bool DIAG = decltype(diag_tag)::value;
      const int bb = li & 1;
      const float* wbias = sbias + warp * 256 + bb * 128;
      // global item index wg + li*WGS -> S^T buffer and its use count
      const uint32_t gi = static_cast<uint32_t>(wg) + li * C::WGS;
      const int sb = static_cast<int>(gi % C::NBUF);
      const uint32_t tS = tS0 + sb * 128;
      __syncwarp();  // this item's bias is written; the other buffer is free
      if (!warp_all(mbar_wait(&s_full[sb], (gi / C::NBUF) & 1, TO, abort_flag))) return false;
      tc_fence_after();
      uint64_t acc2[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) acc2[c] = 0ull;
      // exp2(x*sc - bias_q) over the 128 query columns in eight 16-column
      // chunks, the next chunk's TMEM load in flight while this one is
      // reduced: packed FP32x2 FMA for the exponents, packed adds into four
      // pair accumulators (the same order as one pass over the columns).
      float xa[16], xb[16];
      tmem_ld16_nowait(tS, reinterpret_cast<uint32_t*>(xa));
      tmem_wait_ld16(reinterpret_cast<uint32_t*>(xa));
      auto chunk = [&](const int h, float (&x)[16], float (&xn)[16]) {
        if (h < 7) tmem_ld16_nowait(tS + (h + 1) * 16, reinterpret_cast<uint32_t*>(xn));
        const float4* nb4 = reinterpret_cast<const float4*>(wbias + h * 16);
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const float4 nb = nb4[c4];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int c = c4 * 4 + hh * 2;
            const int col = h * 16 + c;
            const uint64_t a2 =
                f2_fma(f2_pack(x[c], x[c + 1]), sc2, hh == 0 ? f2_pack(nb.x, nb.y) : f2_pack(nb.z, nb.w));
            uint64_t p2;
            if constexpr (DIAG) {
              float a0, a1;
              f2_unpack(a2, a0, a1);
              a0 = (col >= kr) ? a0 : -INFINITY;
              a1 = (col + 1 >= kr) ? a1 : -INFINITY;
              p2 = f2_pack(ex2_approx(a0), ex2_approx(a1));
            } else if (((col & 15) >> 1) >= 8 - REPLAY_POLY_PAIRS) {
              p2 = exp2_poly_x2(a2);
            } else {
              float a0, a1;
              f2_unpack(a2, a0, a1);
              p2 = f2_pack(ex2_approx(a0), ex2_approx(a1));
            }
            acc2[(col >> 1) & 3] = f2_add(acc2[(col >> 1) & 3], p2);
          }
        }
        if (h < 7) tmem_wait_ld16(reinterpret_cast<uint32_t*>(xn));
        if (h == 6) {
          // every load of this S^T buffer has completed: release it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[sb]);
        }
        if (h == 3) {
          ReplayItems nx = it;
          nx.advance(C::WGS);
          if (nx.valid()) {
            write_bias(nx.qt, ml_next, sbias + warp * 256 + (bb ^ 1) * 128);
            nx.advance(C::WGS);
            if (nx.valid()) load_stats(nx, ml_next);
          }
        }
      };
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        if (h & 1) chunk(h, xb, xa);
        else chunk(h, xa, xb);
      }
      float a0, a1, a2, a3, a4, a5, a6, a7;
      f2_unpack(acc2[0], a0, a1);
      f2_unpack(acc2[1], a2, a3);
      f2_unpack(acc2[2], a4, a5);
      f2_unpack(acc2[3], a6, a7);
      acc += static_cast<double>(((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7)));
      return true;
    };
    for (; it.valid() && p.causal && it.qt == kt && ok; it.advance(C::WGS), ++li) ok = process_item(std::true_type{});
    for (; it.valid() && ok; it.advance(C::WGS), ++li) ok = process_item(std::false_type{});
    // Combine the four warpgroups' sums of each key in a fixed order.
    sred[wg * 128 + kr] = acc;
    named_bar_sync(1, C::WGS * 128);
    if (wg == 0 && key < p.N && *abort_flag) {
      // Aborted (watchdog): the sums are incomplete; store NaN, never a
      // plausible-looking partial value.
      p.importance[(static_cast<size_t>(b) * p.Hkv + hkv) * p.N + key] = __int_as_float(0x7fffffff);
    } else if (wg == 0 && key < p.N) {
      double total = sred[kr];
#pragma unroll
      for (int w = 1; w < C::WGS; ++w) total += sred[w * 128 + kr];
      float vn = 1.0f;
      if (p.weighted) {
        using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
        const T* vrow = reinterpret_cast<const T*>(p.v) + b * p.v_sb + hkv * p.v_sh + static_cast<int64_t>(key) * p.v_sn;
        // ||v_key||_1 in channel order.  The row is read with 16-byte loads
        // issued back to back (a scalar loop of dependent 2-byte loads ran
        // at memory latency per channel and dominated short replays); the
        // adds keep the sequential channel order.
        auto to_f = [](T h) -> float {
          if constexpr (BF16) return __bfloat162float(h);
          else return __half2float(h);
        };
        float s = 0.f;
        int d = 0;
        if ((reinterpret_cast<uintptr_t>(vrow) & 15u) == 0) {
          constexpr int NV = DP / 8;  // 16-byte chunks; four in flight at a time
#pragma unroll
          for (int i0 = 0; i0 < NV; i0 += 4) {
            uint4 u[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if ((i0 + i) * 8 + 8 <= p.D) u[i] = __ldg(reinterpret_cast<const uint4*>(vrow) + i0 + i);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              if ((i0 + i) * 8 + 8 <= p.D) {
                const T* h = reinterpret_cast<const T*>(&u[i]);
#pragma unroll
                for (int e = 0; e < 8; ++e) s += fabsf(to_f(h[e]));
              }
            }
          }
          d = p.D & ~7;
        }
        for (; d < p.D; ++d) s += fabsf(to_f(vrow[d]));
        vn = s;
      }
      p.importance[(static_cast<size_t>(b) * p.Hkv + hkv) * p.N + key] = static_cast<float>(total) * vn;
    }
    (void)ok;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == C::ISSUER) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::NBUF * 128);
  }
}

}  // namespace fe
