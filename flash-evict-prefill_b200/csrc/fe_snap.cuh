// SnapKV observation-window scores for sm_100a.
//
// Restates `snap_scores` (flash_evict/baselines.py:12-26):
//   logits = Q[:, :, N-w:] K^T computed in the input dtype (the FP32 dot
//            products rounded to fp16/bf16), then cast to FP32 and scaled
//   logits[key > query position] = -inf
//   p      = softmax(logits) over the keys (FP32)
//   score  = sum of p over the w window rows, then the mean over the G query
//            heads of each KV head.
// without materialising the G*w x N probability matrix, in two launches:
//
//  fe_snap_stats_kernel  -- one CTA per (b, hkv, row group, key chunk):
//    S = Q_w K^T on the tensor cores (window rows on the TMEM lanes), each
//    thread keeps its row's running max and exponential sum over the chunk's
//    keys in the log2 domain and writes one partial {m, l} per row.
//  fe_snap_score_kernel  -- one CTA per (b, hkv, 128-key tile):
//    merges the partials of every window row into one exponent bias
//    (m + log2 l), computes S^T = K Q_w^T with the keys on the TMEM lanes and
//    sums exp2(round(x) * scale * log2e - bias) over the rows in registers:
//    one thread per key, one store per key, no atomics.
//
// Row groups: the w window rows of each of the G heads are padded to w8 (a
// multiple of 8 rows, so every head starts on a 1024-byte swizzle atom) and
// packed floor(256 / w8) heads to a group of at most 256 rows (two 128-row
// M tiles); windows longer than 256 rows are cut into 256-row pieces, one
// group each.  Q rows past the window (the padding) are loaded past the end of
// the sequence, where TMA fills zeros, and rows no load covers are zeroed in
// shared memory, so every padded row is finite and is then excluded by its
// bias (+inf).
#pragma once

#include "fe_ptx.cuh"

namespace fe {

struct SnapParams {
  float2* partial;  // [B*Hkv, groups, nchunk, 256] {m, l} per row group row
  float* scores;    // [B, Hkv, N]
  int B, Hq, Hkv, N, D, G;
  int w;            // window rows, 1..N
  int w8;           // w rounded up to a multiple of 8
  int hpg;          // heads per group when w8 <= 256, else 0
  int ppg;          // 256-row pieces per head when w8 > 256, else 0
  int groups;       // row groups per KV head
  int nchunk;       // key chunks of the statistics pass
  int chunk_tiles;  // 128-key tiles per chunk
  float sc;         // scale * log2(e)
  uint64_t timeout_ns;
};

struct SnapGroup {
  int h0;    // first head (index within the KV head's group of G)
  int nh;    // heads loaded
  int r0;    // first window row (pieces of long windows)
  int rows;  // shared-memory rows written by the loads
  __device__ __forceinline__ void init(const SnapParams& p, int j) {
    if (p.hpg > 0) {
      h0 = j * p.hpg;
      nh = min(p.hpg, p.G - h0);
      r0 = 0;
      rows = nh * p.w8;
    } else {
      h0 = j / p.ppg;
      nh = 1;
      r0 = (j % p.ppg) * 256;
      rows = 256;
    }
  }
  __device__ __forceinline__ int mtiles() const { return rows > 128 ? 2 : 1; }
  // Window row (0..w-1) held in shared-memory row i, or -1 for padding.
  __device__ __forceinline__ int window_row(const SnapParams& p, int i) const {
    if (i >= rows) return -1;
    const int r = p.hpg > 0 ? i % p.w8 : r0 + i;
    return r < p.w ? r : -1;
  }
  __device__ __forceinline__ int box_rows(const SnapParams& p) const { return p.hpg > 0 ? p.w8 : 256; }
};

template <int DP>
struct SnapCfg {
  static constexpr int NCH = DP / 64;
  static constexpr int QHALF = 256 * 128;  // one 64-channel half of a 256-row group
  static constexpr int QBYTES = NCH * QHALF;
  static constexpr int KTILE = 128 * DP * 2;
  static constexpr int KST = DP <= 128 ? 3 : 1;  // K ring depth of the statistics pass (shared memory)
  static constexpr int THREADS = 192;
  // statistics pass: q_full, k_full[KST], k_empty[KST], s_full[2], s_free[2], drain
  static constexpr int A_OFF_Q = 0;
  static constexpr int A_OFF_K = QBYTES;
  static constexpr int A_OFF_BAR = A_OFF_K + KST * KTILE;
  static constexpr int A_NBAR = 1 + 2 * KST + 5;
  static constexpr int A_SMEM = A_OFF_BAR + A_NBAR * 8 + 16 + 1024;
  // scoring pass: k_full, q_full, q_empty, s_full[2], s_free[2], drain
  static constexpr int B_OFF_K = 0;
  static constexpr int B_OFF_Q = KTILE;
  static constexpr int B_OFF_BIAS = B_OFF_Q + QBYTES;  // float[256], negated
  static constexpr int B_OFF_QPOS = B_OFF_BIAS + 256 * 4;
  static constexpr int B_OFF_BAR = B_OFF_QPOS + 256 * 4;
  static constexpr int B_NBAR = 3 + 5;
  static constexpr int B_SMEM = B_OFF_BAR + B_NBAR * 8 + 16 + 1024;
};

// Zero the shared-memory Q rows [from, to) of every channel half (rows that no
// load of the current group writes), then make the stores visible to the
// tensor-core proxy.  Called by `nthr` threads with index `t`.
template <int DP>
__device__ __forceinline__ void snap_zero_rows(uint8_t* q, int from, int to, int t, int nthr) {
  using C = SnapCfg<DP>;
  const int per_half = (to - from) * 8;  // 16-byte chunks
  for (int i = t; i < per_half * C::NCH; i += nthr) {
    const int c = i / per_half;
    const int r = i - c * per_half;
    *reinterpret_cast<uint4*>(q + c * C::QHALF + from * 128 + r * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  fence_proxy_async_smem();
}

// Issue the TMA loads of one row group's Q rows (one box per head, or the
// 256-row piece) onto `bar`.
template <int DP>
__device__ __forceinline__ void snap_load_q(const CUtensorMap* tq, uint8_t* q, uint64_t* bar, const SnapParams& p,
                                            const SnapGroup& gr, int hkv, int b) {
  using C = SnapCfg<DP>;
  const int box = gr.box_rows(p);
  mbar_expect_tx(bar, static_cast<uint32_t>(gr.nh * box * 128 * C::NCH));
  for (int hh = 0; hh < gr.nh; ++hh)
    for (int c = 0; c < C::NCH; ++c)
      tma_load_4d(q + c * C::QHALF + hh * box * 128, tq, bar, c * 64, p.N - p.w + gr.r0, hkv * p.G + gr.h0 + hh, b);
}

template <bool BF16, int DP>
__global__ void __launch_bounds__(192, 1)
    fe_snap_stats_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const SnapParams p) {
  using C = SnapCfg<DP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::A_OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = k_full + C::KST;
  uint64_t* s_full = k_empty + C::KST;
  uint64_t* s_free = s_full + 2;
  uint64_t* drain = s_free + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + C::A_NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;

  int item = blockIdx.x;
  const int chunk = item % p.nchunk;
  item /= p.nchunk;
  const int grp = item % p.groups;
  const int bh = item / p.groups;
  const int b = bh / p.Hkv;
  const int hkv = bh - b * p.Hkv;
  const int ntiles = (p.N + 127) / 128;
  const int t0 = chunk * p.chunk_tiles;
  const int nt = min(ntiles, t0 + p.chunk_tiles) - t0;
  SnapGroup gr;
  gr.init(p, grp);
  const int MT = gr.mtiles();

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(q_full, 1);
    for (int s = 0; s < C::KST; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    __syncwarp();
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  if (gr.rows < MT * 128) snap_zero_rows<DP>(smem + C::A_OFF_Q, gr.rows, MT * 128, threadIdx.x, C::THREADS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint64_t TO = p.timeout_ns;

  if (warp == 4) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      snap_load_q<DP>(&tq, smem + C::A_OFF_Q, q_full, p, gr, hkv, b);
      int issued = 0;
      bool ok = true;
      for (; issued < nt; ++issued) {
        const int s = issued % C::KST;
        const uint32_t use = issued / C::KST;
        if (use > 0) ok = mbar_wait(&k_empty[s], (use - 1) & 1, TO, abort_flag);
        if (!ok) break;
        mbar_expect_tx(&k_full[s], C::KTILE);
        for (int c = 0; c < C::NCH; ++c)
          tma_load_4d(smem + C::A_OFF_K + s * C::KTILE + c * 16384, &tk, &k_full[s], c * 64, (t0 + issued) * 128,
                      hkv, b);
      }
      // Every load must have landed before the CTA exits.
      mbar_wait_inflight(q_full, 0, TO);
      for (int i = (issued > C::KST ? issued - C::KST : 0); i < issued; ++i)
        mbar_wait_inflight(&k_full[i % C::KST], (i / C::KST) & 1, TO);
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t ID = idesc_f16(128, 128, BF16, false);
      const uint32_t q_addr = smem_u32(smem + C::A_OFF_Q);
      const uint32_t k_addr = smem_u32(smem + C::A_OFF_K);
      bool ok = mbar_wait(q_full, 0, TO, abort_flag);
      for (int i = 0; i < nt && ok; ++i) {
        const int s = i % C::KST;
        const int sb = i & 1;
        ok = mbar_wait(&k_full[s], (i / C::KST) & 1, TO, abort_flag);
        if (!ok) break;
        if (i >= 2) ok = mbar_wait(&s_free[sb], ((i >> 1) - 1) & 1, TO, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t ka = k_addr + s * C::KTILE;
        for (int m = 0; m < MT; ++m) {
#pragma unroll
          for (int kk = 0; kk < DP / 16; ++kk) {
            const uint32_t qoff = (kk >> 2) * C::QHALF + m * 16384 + (kk & 3) * 32;
            const uint32_t koff = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_ss(tmem + (sb * 2 + m) * 128, smem_desc_sw128(q_addr + qoff, 16, 1024),
                    smem_desc_sw128(ka + koff, 16, 1024), ID, kk > 0);
          }
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[s]);
      }
      umma_commit(drain);
      mbar_wait_inflight(drain, 0, TO);
    }
  } else {
    // ------------------------------------------- row statistics (thread = row)
    const int row = (warp << 5) + static_cast<int>(lane);
    const uint32_t lane_off = static_cast<uint32_t>(warp << 5) << 16;
    const float sc = p.sc;
    float mrun[2] = {-INFINITY, -INFINITY};
    float lrun[2] = {0.f, 0.f};
    int qpos[2];
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const int wr = gr.window_row(p, m * 128 + row);
      qpos[m] = wr >= 0 ? p.N - p.w + wr : p.N - 1;
    }
    const int qmin = p.N - p.w + gr.r0;
    bool ok = true;
    for (int i = 0; i < nt; ++i) {
      const int sb = i & 1;
      ok = warp_all(mbar_wait(&s_full[sb], (i >> 1) & 1, TO, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int key0 = (t0 + i) * 128;
      const bool edge = key0 + 127 > qmin;  // a key of this tile lies past some row's position (or past N)
      for (int m = 0; m < MT; ++m) {
        float x[128];
        tmem_ld64_sync(tmem + lane_off + (sb * 2 + m) * 128, reinterpret_cast<uint32_t*>(x));
        tmem_ld64_sync(tmem + lane_off + (sb * 2 + m) * 128 + 64, reinterpret_cast<uint32_t*>(x + 64));
        if (m == MT - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[sb]);
        }
        // logits rounded to the input dtype (the reference's matmul output),
        // then scaled into the log2 domain
#pragma unroll
        for (int c = 0; c < 128; c += 2) {
          round_pair<BF16>(x[c], x[c + 1]);
          x[c] *= sc;
          x[c + 1] *= sc;
        }
        if (edge) {
          const int lim = qpos[m] - key0;  // keys key0+c with c > lim are masked (qpos <= N-1)
#pragma unroll
          for (int c = 0; c < 128; ++c) x[c] = c > lim ? -INFINITY : x[c];
        }
        float t = fmax3(x[0], x[1], x[2]);
#pragma unroll
        for (int c = 3; c < 127; c += 2) t = fmax3(t, x[c], x[c + 1]);
        t = fmaxf(t, x[127]);
        if (t > -INFINITY) {
          const float mn = fmaxf(mrun[m], t);
          float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
          for (int c = 0; c < 128; c += 4) {
            s0 += ex2_approx(x[c] - mn);
            s1 += ex2_approx(x[c + 1] - mn);
            s2 += ex2_approx(x[c + 2] - mn);
            s3 += ex2_approx(x[c + 3] - mn);
          }
          lrun[m] = fmaf(lrun[m], ex2_approx(mrun[m] - mn), (s0 + s1) + (s2 + s3));
          mrun[m] = mn;
        }
      }
    }
    {
      // On an abort (watchdog) the partial sums are NaN, which the scoring
      // pass turns into NaN scores instead of using stale workspace.
      const float nan = __int_as_float(0x7fffffff);
      float2* dst = p.partial + ((static_cast<size_t>(bh) * p.groups + grp) * p.nchunk + chunk) * 256;
      for (int m = 0; m < MT; ++m) dst[m * 128 + row] = ok ? make_float2(mrun[m], lrun[m]) : make_float2(nan, nan);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool BF16, int DP>
__global__ void __launch_bounds__(192, 2)
    fe_snap_score_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                         const SnapParams p) {
  using C = SnapCfg<DP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sbias = reinterpret_cast<float*>(smem + C::B_OFF_BIAS);
  int* sqpos = reinterpret_cast<int*>(smem + C::B_OFF_QPOS);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::B_OFF_BAR);
  uint64_t* k_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* s_free = s_full + 2;
  uint64_t* drain = s_free + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + C::B_NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31;
  const int ntiles = (p.N + 127) / 128;
  const int kt = blockIdx.x % ntiles;
  const int bh = blockIdx.x / ntiles;
  const int b = bh / p.Hkv;
  const int hkv = bh - b * p.Hkv;

  if (threadIdx.x == 0) {
    *abort_flag = 0;
    mbar_init(k_full, 1);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    __syncwarp();
    tmem_alloc(tmem_holder, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint64_t TO = p.timeout_ns;

  if (warp == 4) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      tma_prefetch_desc(&tq);
      tma_prefetch_desc(&tk);
      mbar_expect_tx(k_full, C::KTILE);
      for (int c = 0; c < C::NCH; ++c)
        tma_load_4d(smem + C::B_OFF_K + c * 16384, &tk, k_full, c * 64, kt * 128, hkv, b);
    }
    bool ok = true;
    int issued = 0;
    for (; issued < p.groups; ++issued) {
      if (issued > 0) ok = warp_all(mbar_wait(q_empty, (issued - 1) & 1, TO, abort_flag));
      if (!ok) break;
      SnapGroup gr;
      gr.init(p, issued);
      const int MT = gr.mtiles();
      if (gr.rows < MT * 128) snap_zero_rows<DP>(smem + C::B_OFF_Q, gr.rows, MT * 128, lane, 32);
      __syncwarp();
      if (lane == 0) snap_load_q<DP>(&tq, smem + C::B_OFF_Q, q_full, p, gr, hkv, b);
    }
    if (lane == 0) {
      mbar_wait_inflight(k_full, 0, TO);
      if (issued > 0) mbar_wait_inflight(q_full, (issued - 1) & 1, TO);
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t ID = idesc_f16(128, 128, BF16, false);
      const uint32_t k_addr = smem_u32(smem + C::B_OFF_K);
      const uint32_t q_addr = smem_u32(smem + C::B_OFF_Q);
      bool ok = mbar_wait(k_full, 0, TO, abort_flag);
      int it = 0;
      for (int grp = 0; grp < p.groups && ok; ++grp) {
        ok = mbar_wait(q_full, grp & 1, TO, abort_flag);
        if (!ok) break;
        SnapGroup gr;
        gr.init(p, grp);
        const int MT = gr.mtiles();
        for (int m = 0; m < MT && ok; ++m, ++it) {
          const int sb = it & 1;
          if (it >= 2) ok = mbar_wait(&s_free[sb], ((it >> 1) - 1) & 1, TO, abort_flag);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < DP / 16; ++kk) {
            const uint32_t koff = (kk >> 2) * 16384 + (kk & 3) * 32;
            const uint32_t qoff = (kk >> 2) * C::QHALF + m * 16384 + (kk & 3) * 32;
            umma_ss(tmem + sb * 128, smem_desc_sw128(k_addr + koff, 16, 1024),
                    smem_desc_sw128(q_addr + qoff, 16, 1024), ID, kk > 0);
          }
          umma_commit(&s_full[sb]);
        }
        umma_commit(q_empty);
      }
      umma_commit(drain);
      mbar_wait_inflight(drain, 0, TO);
    }
  } else {
    // ------------------------------------------------ reduce (thread = key) --
    const int kr = (warp << 5) + static_cast<int>(lane);
    const int key = kt * 128 + kr;
    const uint32_t lane_off = static_cast<uint32_t>(warp << 5) << 16;
    const float sc = p.sc;
    const uint64_t sc2 = f2_pack(sc, sc);
    double acc = 0.0;
    bool ok = true;
    int it = 0;
    for (int grp = 0; grp < p.groups; ++grp) {
      SnapGroup gr;
      gr.init(p, grp);
      const int MT = gr.mtiles();
      // Merge the statistics pass's partials into one bias per row.  The two
      // barriers run on every path (also after a failed wait), so the four
      // reduce warps always meet.
      named_bar_sync(1, 128);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = kr + 128 * u;
        const int wr = gr.window_row(p, i);
        float nb = -INFINITY;
        int qp = 0x7fffffff;
        if (wr >= 0) {
          const float2* part = p.partial + (static_cast<size_t>(bh) * p.groups + grp) * p.nchunk * 256 + i;
          float m = -INFINITY;
          for (int c = 0; c < p.nchunk; ++c) m = fmaxf(m, part[c * 256].x);
          float l = 0.f;
          for (int c = 0; c < p.nchunk; ++c) {
            const float2 ml = part[c * 256];
            l = fmaf(ml.y, ex2_approx(ml.x - m), l);
          }
          nb = -(m + lg2_approx(l));
          qp = p.N - p.w + wr;
        }
        sbias[i] = nb;
        sqpos[i] = qp;
      }
      named_bar_sync(1, 128);
      const bool mask = kt * 128 + 127 > p.N - p.w + gr.r0;  // some key past some row's position
      for (int m = 0; m < MT; ++m, ++it) {
        if (!ok) continue;
        const int sb = it & 1;
        ok = warp_all(mbar_wait(&s_full[sb], (it >> 1) & 1, TO, abort_flag));
        if (!ok) continue;
        tc_fence_after();
        uint64_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float x[64];
          tmem_ld64_sync(tmem + lane_off + sb * 128 + h * 64, reinterpret_cast<uint32_t*>(x));
          if (h == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_free[sb]);
          }
          const float* nb = sbias + m * 128 + h * 64;
          const int* qp = sqpos + m * 128 + h * 64;
#pragma unroll
          for (int c = 0; c < 64; c += 2) {
            round_pair<BF16>(x[c], x[c + 1]);
            float a0, a1;
            f2_unpack(f2_fma(f2_pack(x[c], x[c + 1]), sc2, f2_pack(nb[c], nb[c + 1])), a0, a1);
            if (mask) {
              a0 = key > qp[c] ? -INFINITY : a0;
              a1 = key > qp[c + 1] ? -INFINITY : a1;
            }
            acc2[(c >> 1) & 3] = f2_add(acc2[(c >> 1) & 3], f2_pack(ex2_approx(a0), ex2_approx(a1)));
          }
        }
        float a0, a1, a2, a3, a4, a5, a6, a7;
        f2_unpack(acc2[0], a0, a1);
        f2_unpack(acc2[1], a2, a3);
        f2_unpack(acc2[2], a4, a5);
        f2_unpack(acc2[3], a6, a7);
        acc += static_cast<double>(((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7)));
      }
    }
    // mean over the G heads of the KV head, as the reference's mean(2)
    if (key < p.N)
      p.scores[static_cast<size_t>(bh) * p.N + key] =
          ok ? __fdiv_rn(static_cast<float>(acc), static_cast<float>(p.G)) : __int_as_float(0x7fffffff);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace fe
