// Attention forward (traversal 1) on CTA pairs, for heads of 65-128 channels.
//
// Same arithmetic as fe_fwd_kernel (flash_evict/prefill.py:23-60: online
// softmax in the log2 domain, P cast to the input dtype before PV, FP32 m and
// l, O = acc / l, {m, l} written per row) and the same per-CTA roles, TMEM
// map and softmax code; what changes is how the two SMs of a cluster pair
// share the tensor-core work.
//
// A cluster of two CTAs owns one 512-row query block of one query head.  Its
// "pair tile" t (t = 0, 1) is rows [512*blk + 256*t, +256): CTA c holds rows
// +128*c of it in shared memory (Q) and in TMEM (S, P, O).  One thread of CTA
// 0 issues every MMA with cta_group::2 and M = 256:
//   S_t = Q_t K^T  (N = 128 keys: each CTA holds 64 of the K tile's keys)
//   O_t += P_t V   (N = 128 channels: each CTA holds 64 of V's channels)
// so per 128-key step each SM reads 32 KB of Q and 16 KB of K from shared
// memory for its S (instead of 32 + 32 KB), and TMA brings 32 KB of K/V per
// SM (instead of 64 KB): the S MMAs are no longer bound by shared-memory
// bandwidth, and K/V traffic from L2 halves.
//
// Synchronisation: both CTAs' TMA loads complete on CTA 0's barriers (CTA 0
// posts the expected byte counts); the issuing thread commits every MMA group
// to the barrier of each CTA that waits for it (s_full, o_full, K/V stage
// release, drain); the softmax warps of both CTAs arrive on CTA 0's p_full
// (8 warps).  A fully masked KV tile (the pair tile's extent is the extent of
// its last rows, one tile more than CTA 0's rows need on the causal
// diagonal) gives P = 0 and leaves m and l unchanged.
#pragma once

#include "fe_forward.cuh"

namespace fe {

struct FwdPairCfg {
  static constexpr int QTILE = 128 * 128 * 2;  // one 128-row Q tile: two 64-channel chunks of 16 KB
  static constexpr int KHALF = 64 * 128 * 2;   // 64 keys x 128 channels: two chunks of 8 KB
  static constexpr int VHALF = 128 * 64 * 2;   // 128 keys x 64 channels: one chunk
  static constexpr int STAGES = 4;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = 2 * QTILE;
  static constexpr int OFF_V = OFF_K + STAGES * KHALF;
  static constexpr int OFF_BAR = OFF_V + STAGES * VHALF;
  // q_full, k_full[S], v_full[S], k_empty[S], v_empty[S], s_full[2], p_full[2], o_full[2], drain
  static constexpr int NBAR = 1 + 4 * STAGES + 7;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static constexpr int THREADS = 384;
  static constexpr int BLOCK_ROWS = 512;  // query rows per cluster
};

template <bool BF16>
__global__ void __launch_bounds__(384, 1)
    fe_fwd_pair_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tkh,
                       const __grid_constant__ CUtensorMap tv, const FwdParams p) {
  using C = FwdPairCfg;
  constexpr int DV = 128;
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
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;

  // ---- work item of the pair: (512-row query block, b, hkv, g), in the
  // order of fe_fwd_kernel (causal: heaviest blocks first, the G heads of a
  // group adjacent; non-causal: the blocks of one head adjacent).
  int item = blockIdx.x >> 1;
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
  const int blk = p.causal ? (p.num_blocks - 1 - rank) : rank;
  const int hq = hkv * p.G + g;
  const int nkv = (p.N + 127) / 128;
  // KV tiles of pair tile t: those its last valid row reaches.
  int ntl[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int start = blk * C::BLOCK_ROWS + t * 256;
    const int last = min(p.N - 1, start + 255);
    ntl[t] = (start < p.N) ? (p.causal ? min(nkv, last / 128 + 1) : nkv) : 0;
  }
  const int n0 = ntl[0], n1 = ntl[1];
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
      mbar_init(&p_full[t], 8);  // four softmax warps in each CTA
      mbar_init(&o_full[t], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    __syncwarp();
    tmem_alloc_pair(tmem_holder, 512);
    tmem_relinquish_pair();
  }
  // Barriers of both CTAs are initialised before any TMA or arrive of the
  // peer can reach them.
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint64_t TO = p.timeout_ns;

  if (warp >= 8) {
    setmaxnreg_dec<FWD_REGS_LOW>();
    if (warp == 8) {
      // ---------------------------------------------------------- producer --
      // Both CTAs load their own Q rows and their half of every K/V tile;
      // the bytes are counted on CTA 0's barriers, whose expected counts
      // CTA 0 posts.
      if (lane == 0) {
        tma_prefetch_desc(&tq);
        tma_prefetch_desc(&tkh);
        tma_prefetch_desc(&tv);
        const uint64_t pol_q = l2_policy_evict_first();
        const uint64_t pol_kv = l2_policy_evict_last();
        uint32_t loads[C::STAGES];
        for (int s = 0; s < C::STAGES; ++s) loads[s] = 0;
        if (leader) mbar_expect_tx(q_full, 4 * C::QTILE);
        const uint32_t q_full_l = mapa_shared(smem_u32(q_full), 0);
        for (int t = 0; t < 2; ++t)
          for (int c = 0; c < 2; ++c)
            tma_load_4d_pair(smem + C::OFF_Q + t * C::QTILE + c * 16384, &tq, q_full_l, c * 64,
                             blk * C::BLOCK_ROWS + t * 256 + static_cast<int>(crank) * 128, hq, b, pol_q);
        bool ok = true;
        for (int j = 0; j < nmax && ok; ++j) {
          const int s = j % C::STAGES;
          const uint32_t use = j / C::STAGES;
          if (use > 0) ok = mbar_wait(&k_empty[s], (use - 1) & 1, TO, abort_flag);
          if (!ok) break;
          if (leader) mbar_expect_tx(&k_full[s], 2 * C::KHALF);
          const uint32_t kf = mapa_shared(smem_u32(&k_full[s]), 0);
          for (int c = 0; c < 2; ++c)
            tma_load_4d_pair(smem + C::OFF_K + s * C::KHALF + c * 8192, &tkh, kf, c * 64,
                             j * 128 + static_cast<int>(crank) * 64, hkv, b, pol_kv);
          if (use > 0) ok = mbar_wait(&v_empty[s], (use - 1) & 1, TO, abort_flag);
          if (!ok) {
            loads[s] = use * 2 + 1;
            break;
          }
          if (leader) mbar_expect_tx(&v_full[s], 2 * C::VHALF);
          tma_load_4d_pair(smem + C::OFF_V + s * C::VHALF, &tv, mapa_shared(smem_u32(&v_full[s]), 0),
                           p.vcol0 + static_cast<int>(crank) * 64, j * 128, hkv, b, pol_kv);
          loads[s] = use * 2 + 2;
        }
        // CTA 0 holds the barriers of both CTAs' loads: it waits (bounded)
        // for the last load of each stage before the pair leaves (the
        // closing cluster barrier keeps CTA 1 alive until then).  On the
        // normal path the MMA thread has already waited for all of them.
        if (leader) {
          mbar_wait_inflight(q_full, 0, TO);
          for (int s = 0; s < C::STAGES; ++s) {
            if (loads[s] == 0) continue;
            const uint32_t use = (loads[s] - 1) / 2;
            mbar_wait_inflight(&k_full[s], use & 1, TO);
            if (loads[s] % 2 == 0) mbar_wait_inflight(&v_full[s], use & 1, TO);
          }
        }
      }
    } else if (warp == 9 && lane == 0) {
      if (leader) {
        // ------------------------------------------------------ MMA issuer --
        constexpr uint32_t ID_S = idesc_f16(256, 128, BF16, false);
        constexpr uint32_t ID_PV = idesc_f16(256, DV, BF16, true);
        const uint64_t dq = smem_desc_sw128(smem_u32(smem + C::OFF_Q), 16, 1024);
        const uint64_t dk = smem_desc_sw128(smem_u32(smem + C::OFF_K), 16, 1024);
        const uint64_t dv = smem_desc_sw128(smem_u32(smem + C::OFF_V), 16384, 1024);
        const uint32_t dq_lo = static_cast<uint32_t>(dq), dq_hi = static_cast<uint32_t>(dq >> 32);
        const uint32_t dk_lo = static_cast<uint32_t>(dk), dk_hi = static_cast<uint32_t>(dk >> 32);
        const uint32_t dv_lo = static_cast<uint32_t>(dv), dv_hi = static_cast<uint32_t>(dv >> 32);
        auto commit_both = [&](uint64_t* bar) {
          const uint32_t a = smem_u32(bar);
          umma_commit_pair(a);
          umma_commit_pair(mapa_shared(a, 1));
        };
        auto issue_s = [&](int t, int s) {
          const uint32_t a = dq_lo + static_cast<uint32_t>(t * (C::QTILE >> 4));
          const uint32_t bb = dk_lo + static_cast<uint32_t>(s * (C::KHALF >> 4));
          const uint32_t d = tmem + t * 128;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t offa = static_cast<uint32_t>(((kk >> 2) * 16384 + (kk & 3) * 32) >> 4);
            const uint32_t offb = static_cast<uint32_t>(((kk >> 2) * 8192 + (kk & 3) * 32) >> 4);
            umma_pair_ss_lohi(d, a + offa, dq_hi, bb + offb, dk_hi, ID_S, kk > 0);
          }
        };
        auto issue_pv = [&](int t, int s, int j) {
          const uint32_t bb = dv_lo + static_cast<uint32_t>(s * (C::VHALF >> 4));
          const uint32_t d = tmem + 256 + t * DV;
          const uint32_t pa = tmem + t * 128;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_pair_ts_lohi(d, pa + kk * 8, bb + static_cast<uint32_t>(kk * (2048 >> 4)), dv_hi, ID_PV,
                              (j > 0 || kk > 0) ? 1u : 0u);
        };
        bool ok = mbar_wait(q_full, 0, TO, abort_flag);
        if (ok) ok = mbar_wait(&k_full[0], 0, TO, abort_flag);
        if (ok) {
          tc_fence_after();
          if (n0 > 0) {
            issue_s(0, 0);
            commit_both(&s_full[0]);
          }
          if (n1 > 0) {
            issue_s(1, 0);
            commit_both(&s_full[1]);
          }
          if (C::STAGES < nmax) commit_both(&k_empty[0]);
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
            ok = mbar_wait_cluster(&p_full[t], j & 1, TO, abort_flag);
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
              commit_both(&s_full[t]);
            } else {
              commit_both(&o_full[t]);
            }
          }
          if (!ok) break;
          if (j + C::STAGES < nmax) commit_both(&v_empty[s]);
          if (next && (j + 1 + C::STAGES < nmax)) commit_both(&k_empty[s2]);
        }
        // Drain: every pair MMA has completed once both CTAs see this.
        commit_both(drain);
        mbar_wait_inflight(drain, 0, TO);
      } else {
        // CTA 1's TMEM and shared memory are read by the pair MMAs: keep
        // them until the last one has completed.
        mbar_wait_inflight(drain, 0, TO);
      }
    }
  } else {
    setmaxnreg_inc<FWD_REGS_HIGH>();
    // ------------------------------------------------------------- softmax --
    const int t = warp >> 2;
    const int nt = t == 0 ? n0 : n1;
    const int rbase = blk * C::BLOCK_ROWS + t * 256 + static_cast<int>(crank) * 128;
    const int r = ((warp & 3) << 5) + static_cast<int>(lane);
    const int row = rbase + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) << 5) << 16;
    const uint32_t tS = tmem + lane_off + t * 128;
    const uint32_t tO = tmem + lane_off + 256 + t * DV;
    const uint32_t p_full_l = mapa_shared(smem_u32(&p_full[t]), 0);
    const float sc = p.sc;
    const bool sc_pos = sc > 0.f;
    const float sce = sc_pos ? sc : 1.0f;
    float m_used = -INFINITY;
    float l = 0.f;
    bool ok = true;
    // Tiles that need per-element masking for this CTA's rows (diagonal,
    // ragged end of N, the fully masked extra tile of CTA 0) run last.
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
      if (lane == 0) mbar_arrive_cluster(p_full_l);
      return true;
    };
    for (int j = 0; j < n_plain && ok; ++j) ok = tile_step(j, std::false_type{});
    for (int j = n_plain; j < nt && ok; ++j) ok = tile_step(j, std::true_type{});
    if (nt > 0 && ok) ok = warp_all(mbar_wait(&o_full[t], 0, TO, abort_flag));
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    if (nt > 0 && !ok && row < p.N) {
      // Aborted (watchdog): NaN statistics and output channels for this row.
      if (p.vcol0 == 0) {
        float2* st = reinterpret_cast<float2*>(p.row_stats) + (static_cast<size_t>(b) * p.Hq + hq) * p.N + row;
        *st = make_float2(__int_as_float(0x7fffffff), __int_as_float(0x7fffffff));
      }
      T* orow = reinterpret_cast<T*>(p.out) + ((static_cast<size_t>(b) * p.Hq + hq) * p.N + row) * p.D + p.vcol0;
      const uint16_t nan16 = BF16 ? 0x7fc0 : 0x7e00;
      for (int c = 0; c < DV && c < p.D - p.vcol0; ++c) reinterpret_cast<uint16_t*>(orow)[c] = nan16;
    }
    if (nt > 0 && ok) {
      tc_fence_after();
      const bool live = row < p.N;
      if (live && p.vcol0 == 0) {
        float2* st = reinterpret_cast<float2*>(p.row_stats) + (static_cast<size_t>(b) * p.Hq + hq) * p.N + row;
        *st = make_float2(m_used, l);
      }
      const float inv = 1.0f / l;
      T* orow = reinterpret_cast<T*>(p.out) + ((static_cast<size_t>(b) * p.Hq + hq) * p.N + row) * p.D + p.vcol0;
      const int dlim = p.D - p.vcol0;
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
                       make_uint4(w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2], w[4 * q4 + 3]));
            }
          } else {
            const uint16_t* h = reinterpret_cast<const uint16_t*>(w);
            for (int c = 0; c < 32 && c0 + c < dlim; ++c) reinterpret_cast<uint16_t*>(orow)[c0 + c] = h[c];
          }
        }
      }
    }
  }

  // Both CTAs are done with TMEM, their shared memory and each other's
  // barriers before the pair's TMEM is released; the second barrier keeps
  // both CTAs resident until both have released it.
  tc_fence_before();
  cluster_sync_all();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
  cluster_sync_all();
}

}  // namespace fe
