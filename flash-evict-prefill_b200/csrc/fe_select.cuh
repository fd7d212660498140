// Token selection: SnapKV-style pooling, exact top-k by radix select, and the
// keep/evict mask, in one launch.
//
// Restates `select_tokens` (flash_evict/prefill.py:140-170):
//   past   = importance[:, :N-recent]
//   pooled = avg_pool1d(past, pool_kernel, stride 1, pad pool_kernel//2)
//            (zero padding counted in the divisor), only if pool_kernel > 1 and
//            budget > recent (prefill.py:161-163)
//   keep the budget-recent largest pooled values plus the suffix [N-recent, N)
//   indices ascending (prefill.py:164-168), mask by scatter (prefill.py:169).
// The reference's tie order is torch.topk's (unspecified).  This kernel fixes
// it: larger value first, among equal values the lower index; NaN is the
// largest value and -0.0 equals +0.0.
//
// One thread-block cluster of C CTAs per row (C grows with the row length so
// that short batches still spread over several SMs); CTA r holds a
// contiguous slice of the past region as order-preserving uint32 keys in
// shared memory.  The
// (budget-recent)-th largest key is found MSB-first with four 8-bit radix
// passes whose histograms are merged through distributed shared memory.
// Compaction walks each slice in index order (ballot/popc scans), so indices
// come out already sorted; each CTA takes its output offset from the pass
// histograms of the CTAs before it (read through distributed shared memory).
// Optionally the same launch compacts K and V into dense [rows, budget,
// channels] buffers: once every CTA of the cluster has written its indices
// (a cluster barrier orders them), CTA r copies the rows of output positions
// [r*budget/C, (r+1)*budget/C), so the copy is balanced however unevenly the
// kept tokens fall across the slices.
#pragma once

#include <cooperative_groups.h>

#include "fe_gather.cuh"
#include "fe_ptx.cuh"

namespace fe {

namespace cg = cooperative_groups;

struct SelectParams {
  const float* importance;  // [rows, N]
  int64_t N, budget, recent;
  int pool;
  int64_t* indices;  // [rows, budget]
  uint8_t* mask;     // [rows, N]
  int mask_evict;
  int64_t chunk;     // slice length per CTA
  int gather;        // nonzero: also copy the kept K/V rows (spec g)
  GatherSpec g;
};

constexpr int SEL_THREADS = 1024;
constexpr int SEL_WARPS = SEL_THREADS / 32;

// One launch selects for up to SEL_MAX_POLICIES policies (budget, reserved
// suffix, pooling, score tensor, outputs) over the same rows x N shape, as the
// paired multi-policy controller does for one prompt
// (flash_evict/quality_adapter.py:95-111 choose_indices per method).  All
// policies share the launch's cluster size; each has its own slice length.
constexpr int SEL_MAX_POLICIES = 8;
// Keys per CTA held in shared memory (192 KiB); longer slices use the
// global-key variant of the kernel.
constexpr int64_t SEL_SMEM_KEYS = 49152;
struct SelectLaunch {
  int64_t rows;  // rows per policy
  int npol;
  SelectParams pol[SEL_MAX_POLICIES];
};

// Order-preserving map float -> uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t order_key(float x) {
  if (x != x) return 0xFFFFFFFFu;  // NaN sorts above +inf
  if (x == 0.0f) x = 0.0f;         // -0.0 ties with +0.0
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide exclusive scan of one 0/1 flag per thread in index order.
// Returns this thread's exclusive prefix; *total receives the block sum.
__device__ __forceinline__ int block_flag_scan(bool flag, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const uint32_t bal = __ballot_sync(0xffffffffu, flag);
  const int in_warp = __popc(bal & ((1u << lane) - 1u));
  if (lane == 0) warp_sums[warp] = __popc(bal);
  __syncthreads();
  if (warp == 0) {
    int v = (lane < SEL_WARPS) ? warp_sums[lane] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane < SEL_WARPS) warp_sums[32 + lane] = incl - v;
    if (lane == 31) warp_sums[64] = incl;
  }
  __syncthreads();
  const int res = warp_sums[32 + warp] + in_warp;
  *total = warp_sums[64];
  __syncthreads();
  return res;
}

// Block-wide exclusive scan of one small count per thread in thread order.
// Returns this thread's exclusive prefix; *total receives the block sum.
__device__ __forceinline__ int block_count_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = (lane < SEL_WARPS) ? warp_sums[lane] : 0;
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += n;
    }
    if (lane < SEL_WARPS) warp_sums[32 + lane] = wi - w;
    if (lane == 31) warp_sums[64] = wi;
  }
  __syncthreads();
  const int res = warp_sums[32 + warp] + incl - v;
  *total = warp_sums[64];
  __syncthreads();
  return res;
}

// Split cluster barrier: arrive after this CTA's last read of another CTA's
// shared memory, wait before leaving, so no CTA exits while a peer still
// reads its histograms.
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}

// After the row's indices are complete (every CTA of the cluster calls this
// once, after its last index store), copy the K/V rows of this CTA's share of
// the output positions.  The cluster barrier (release/acquire at cluster
// scope) makes the other CTAs' index stores visible; the gather reads the
// indices through L2.
__device__ __forceinline__ void gather_share(const SelectParams& p, cg::cluster_group& cluster, int64_t row,
                                             const int64_t* out_idx, int C, int crank) {
  cluster.sync();
  const int64_t per = (p.budget + C - 1) / C;
  const int64_t a = min(p.budget, static_cast<int64_t>(crank) * per);
  const int64_t e = min(p.budget, a + per);
  // two loads in flight per thread (1024 threads): the selection kernel runs
  // at its 64-register limit
  gather_rows<2>(p.g, row, out_idx, a, e - a, threadIdx.x, SEL_THREADS);
}

// SMEM_KEYS: the slice's keys are computed once into shared memory (slices of
// up to SEL_SMEM_KEYS keys).  Otherwise (longer rows) every pass recomputes a
// key from the scores in global memory (L2/HBM reads instead of shared
// memory; same arithmetic, same result).
template <bool SMEM_KEYS>
__global__ void __launch_bounds__(SEL_THREADS, 1) fe_select_kernel(const __grid_constant__ SelectLaunch L) {
  cg::cluster_group cluster = cg::this_cluster();
  const int C = static_cast<int>(cluster.num_blocks());
  const int crank = static_cast<int>(cluster.block_rank());
  const int64_t cl_index = blockIdx.x / C;  // cluster index: (policy, row)
  const int pi = static_cast<int>(cl_index / L.rows);
  const int64_t row = cl_index - static_cast<int64_t>(pi) * L.rows;
  const SelectParams& p = L.pol[pi];

  extern __shared__ __align__(16) uint32_t keys[];
  __shared__ uint32_t hist[2][256];
  __shared__ uint32_t tot[256];
  __shared__ int warp_sums[72];
  __shared__ uint32_t sel_digit, sel_krem, sel_done;

  const int64_t N = p.N;
  const int64_t P = N - p.recent;
  const int64_t kk = p.budget - p.recent;
  const float* imp = p.importance + row * N;
  int64_t* out_idx = p.indices + row * p.budget;
  uint8_t* out_mask = p.mask + row * N;
  const uint8_t keep_v = p.mask_evict ? 0 : 1;
  const uint8_t evict_v = p.mask_evict ? 1 : 0;

  const int64_t lo = min(P, static_cast<int64_t>(crank) * p.chunk);
  const int64_t hi = min(P, lo + p.chunk);
  const int len = static_cast<int>(hi - lo);

  // Reserved suffix: always kept, placed after the budget-recent past picks.
  if (crank == 0) {
    for (int64_t j = threadIdx.x; j < p.recent; j += SEL_THREADS) {
      out_idx[kk + j] = P + j;
      out_mask[P + j] = keep_v;
    }
  }
  if (kk == 0) {
    for (int i = threadIdx.x; i < len; i += SEL_THREADS) out_mask[lo + i] = evict_v;
  } else {
    // ---- keys of this slice (pooled if requested) ----
    const bool pooled = p.pool > 1;
    const int r = p.pool / 2;
    auto key_from_scores = [&](int i) -> uint32_t {
      const int64_t gi = lo + i;
      float x;
      if (pooled) {
        // Same accumulation as avg_pool1d: taps left to right inside the row,
        // padding contributes nothing, divisor = kernel size.
        float s = 0.f;
        const int64_t a = gi - r > 0 ? gi - r : 0;
        const int64_t e = gi + r + 1 < P ? gi + r + 1 : P;
        for (int64_t t = a; t < e; ++t) s = __fadd_rn(s, imp[t]);
        x = __fdiv_rn(s, static_cast<float>(p.pool));
      } else {
        x = imp[gi];
      }
      return order_key(x);
    };
    auto key_at = [&](int i) -> uint32_t {
      if constexpr (SMEM_KEYS) return keys[i];
      else return key_from_scores(i);
    };
    if constexpr (SMEM_KEYS) {
      if (!pooled) {
        // Four loads in flight per thread (the key pass is latency-bound).
#pragma unroll 4
        for (int i = threadIdx.x; i < len; i += SEL_THREADS) keys[i] = order_key(imp[lo + i]);
      } else {
        for (int i = threadIdx.x; i < len; i += SEL_THREADS) keys[i] = key_from_scores(i);
      }
    }
    for (int i = threadIdx.x; i < 512; i += SEL_THREADS) (&hist[0][0])[i] = 0;
    __syncthreads();

    // ---- radix select of the kk-th largest key over the whole cluster ----
    uint32_t prefix = 0, pmask = 0;
    uint32_t krem = static_cast<uint32_t>(kk);
    // Keys of the CTAs before this one (cluster rank < crank) that are above
    // the threshold, counted per digit from the same histograms the pass
    // totals are made of: at every pass, the keys whose digit exceeds the
    // selected one (thread d < 256 keeps digit d's share).  The keys of the
    // final bucket (equal to the threshold, or the whole kept bucket when the
    // passes stop early) are counted separately: earlier CTAs, whole cluster.
    uint32_t gt_bef_d = 0;
    __shared__ uint32_t fin_bef, fin_tot;
    if (threadIdx.x == 0) sel_done = 0u;
    for (int pass = 0; pass < 4; ++pass) {
      const int buf = pass & 1;
      const int shift = 24 - 8 * pass;
      if (pass >= 2) {
        // hist[buf] was last read by the cluster before the previous pass's
        // cluster.sync(); clear it for reuse.
        for (int i = threadIdx.x; i < 256; i += SEL_THREADS) hist[buf][i] = 0;
        __syncthreads();
      }
      // Warp-aggregated counting: the lanes holding the same digit elect one
      // of them to add the group's count (scores are often concentrated in a
      // few digits, which would otherwise serialise the shared-memory atomics).
      for (int base = 0; base < len; base += SEL_THREADS) {
        const int i = base + threadIdx.x;
        const uint32_t k = i < len ? key_at(i) : 0u;
        const bool match = (i < len) && ((k & pmask) == prefix);
        const uint32_t digit = match ? ((k >> shift) & 255u) : 0x100u;
        const uint32_t peers = __match_any_sync(0xffffffffu, digit);
        if (match && (threadIdx.x & 31) == static_cast<uint32_t>(__ffs(peers) - 1))
          atomicAdd(&hist[buf][digit], static_cast<uint32_t>(__popc(peers)));
      }
      cluster.sync();
      uint32_t bef_d = 0;
      if (threadIdx.x < 256) {
        uint32_t s = 0;
        for (int rr = 0; rr < C; ++rr) {
          const uint32_t h = cluster.map_shared_rank(&hist[buf][0], rr)[threadIdx.x];
          s += h;
          if (rr < crank) bef_d += h;
        }
        tot[threadIdx.x] = s;
      }
      __syncthreads();
      if (threadIdx.x < 32) {
        // lane l owns digits [248-8l, 255-8l], scanned from the top.
        const int lane = threadIdx.x;
        uint32_t lsum = 0;
  #pragma unroll
        for (int d = 0; d < 8; ++d) lsum += tot[255 - 8 * lane - d];
        uint32_t incl = lsum;
  #pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += n;
        }
        uint32_t cum = incl - lsum;  // keys with a larger digit than this lane's range
        if (cum < krem && krem <= incl) {
  #pragma unroll 1
          for (int d = 0; d < 8; ++d) {
            const int digit = 255 - 8 * lane - d;
            const uint32_t c = tot[digit];
            if (cum + c >= krem) {
              sel_digit = static_cast<uint32_t>(digit);
              sel_krem = krem - cum;
              // Every key of this bucket is kept: the threshold can stop here.
              sel_done = (cum + c == krem) ? 1u : 0u;
              break;
            }
            cum += c;
          }
        }
      }
      __syncthreads();
      prefix |= sel_digit << shift;
      pmask |= 255u << shift;
      krem = sel_krem;
      const bool done = sel_done != 0u;
      if (threadIdx.x < 256) {
        if (threadIdx.x > sel_digit) gt_bef_d += bef_d;
        if (threadIdx.x == sel_digit) {
          fin_bef = bef_d;
          fin_tot = tot[threadIdx.x];
        }
      }
      __syncthreads();
      if (done) {
        // The bucket holding the kk-th largest key is kept whole: every key
        // at or above its smallest possible value (prefix, low bits zero).
        krem = 0xFFFFFFFFu;
        break;
      }
    }
    const uint32_t T = prefix;    // the kk-th largest key, or the kept bucket's floor
    const uint32_t need_eq = krem; // how many keys equal to T are kept (lowest indices)

    // Every read of another CTA's histograms is behind us.
    cluster_arrive_release();

    // ---- offsets of this CTA's kept keys (from the pass histograms) ----
    long long gt_before, eq_before, eq_total;
    {
      uint32_t v = threadIdx.x < 256 ? gt_bef_d : 0u;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if ((threadIdx.x & 31) == 0 && threadIdx.x < 256) warp_sums[threadIdx.x >> 5] = static_cast<int>(v);
      __syncthreads();
      long long g = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) g += static_cast<uint32_t>(warp_sums[w]);
      gt_before = g;
      eq_before = fin_bef;
      eq_total = fin_tot;
      __syncthreads();
    }

    // ---- ordered compaction ----
    if (eq_total <= static_cast<long long>(need_eq)) {
      // Every key equal to T is kept (the usual case: no tie is cut at the
      // threshold), so kept == (k >= T) and one scan per tile places it.
      // Four consecutive keys per thread, one block scan per 4096 keys.
      long long run = gt_before + eq_before;
      for (int base = 0; base < len; base += 4 * SEL_THREADS) {
        const int i0 = base + 4 * static_cast<int>(threadIdx.x);
        uint32_t k4[4];
        if constexpr (SMEM_KEYS) {
          if (i0 + 3 < len) {
            const uint4 q = *reinterpret_cast<const uint4*>(&keys[i0]);
            k4[0] = q.x;
            k4[1] = q.y;
            k4[2] = q.z;
            k4[3] = q.w;
          } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) k4[u] = (i0 + u < len) ? keys[i0 + u] : 0u;
          }
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u) k4[u] = (i0 + u < len) ? key_at(i0 + u) : 0u;
        }
        bool kept[4];
        int cnt = 0;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          kept[u] = (i0 + u < len) && k4[u] >= T;
          cnt += kept[u] ? 1 : 0;
        }
        int tot_kept;
        const int pos = block_count_scan(cnt, warp_sums, &tot_kept);
        int w = 0;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = i0 + u;
          if (i < len) {
            if (kept[u]) out_idx[run + pos + w++] = lo + i;
            out_mask[lo + i] = kept[u] ? keep_v : evict_v;
          }
        }
        run += tot_kept;
      }
    } else {
    long long run_gt = gt_before, run_eq = eq_before;
    for (int base = 0; base < len; base += SEL_THREADS) {
      const int i = base + threadIdx.x;
      const bool in = i < len;
      const uint32_t k = in ? key_at(i) : 0u;
      const bool is_eq = in && (k == T);
      int tot_eq;
      const int eq_rank = block_flag_scan(is_eq, warp_sums, &tot_eq);
      const bool kept_eq = is_eq && (run_eq + eq_rank < static_cast<long long>(need_eq));
      const bool kept = (in && k > T) || kept_eq;
      int tot_kept;
      const int pos = block_flag_scan(kept, warp_sums, &tot_kept);
      // kept elements before this one over the whole row:
      //   gt before the tile + kept-equal before the tile + in-tile prefix
      const long long kept_eq_before = min(run_eq, static_cast<long long>(need_eq));
      if (in) {
        if (kept) out_idx[run_gt + kept_eq_before + pos] = lo + i;
        out_mask[lo + i] = kept ? keep_v : evict_v;
      }
      const long long kept_eq_after = min(run_eq + tot_eq, static_cast<long long>(need_eq));
      run_gt += tot_kept - (kept_eq_after - kept_eq_before);
      run_eq += tot_eq;
    }
    }
    cluster_wait_acquire();
  }

  // ---- K/V compaction, an equal share of the output per CTA ----
  if (p.gather) gather_share(p, cluster, row, out_idx, C, crank);
}

}  // namespace fe
