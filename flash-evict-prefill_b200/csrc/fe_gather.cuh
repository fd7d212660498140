// KV compaction: copy the kept token rows of K and V into dense
// [rows, budget, channels] buffers.
//
// Restates the gather the reference's adapters apply to the selected indices
// (`gather_tokens(state['k'], indices)` at flash_evict/kv_distill_adapter.py:38-39,
// flash_evict/streaming_adapter.py:86, flash_evict/quality_adapter.py:109-110;
// semantics given in README.md:31 as
// `k.gather(2, indices[..., None].expand(-1, -1, -1, k.shape[-1]))`):
//   dst[b, h, j, :] = src[b, h, indices[b, h, j], :].
//
// Pure data movement, so the result is bitwise the source rows.  The copy is
// split into 16/8/4/2/1-byte chunks (the widest the row size, strides and
// base addresses allow); consecutive threads take consecutive chunks of one
// row, K row then V row of the same position, so each warp reads and writes
// whole 128-byte lines, and every thread keeps four loads in flight before it
// stores.  Used two ways: by fe_gather_kernel (caller-supplied indices,
// range-checked) and by the selection kernel's output pass (indices it has
// just produced, an equal share of the output per CTA of the row's cluster).
#pragma once

#include "fe_ptx.cuh"

namespace fe {

struct GatherSpec {
  const uint8_t* k_src;      // [B, H, N, D] with byte strides below (channel stride = element size)
  const uint8_t* v_src;      // may be null (gather K only)
  int64_t k_sb, k_sh, k_sn;  // byte strides
  int64_t v_sb, v_sh, v_sn;
  uint8_t* k_dst;  // [B*H, budget, D] contiguous
  uint8_t* v_dst;
  int64_t heads, tokens, budget;
  int row_bytes;  // channels * element size
  int vec;        // chunk bytes: 16, 8, 4, 2 or 1
};

// FE_STATUS_BAD_INDEX: a gather index outside [0, tokens); the destination
// row is written with zeros instead of faulting.
constexpr int STATUS_BAD_INDEX = 5;

template <typename T, int U>
__device__ __forceinline__ void gather_rows_vec(const GatherSpec& g, int64_t row, const int64_t* idx_row,
                                                int64_t pos0, int64_t cnt, int tid, int nth) {
  const int cpr = g.row_bytes / static_cast<int>(sizeof(T));
  const bool two = g.v_src != nullptr;
  const int64_t per_pos = two ? 2 * cpr : cpr;
  const int64_t total = cnt * per_pos;
  const int64_t b = row / g.heads, h = row - b * g.heads;
  const uint8_t* kb = g.k_src + b * g.k_sb + h * g.k_sh;
  const uint8_t* vb = two ? g.v_src + b * g.v_sb + h * g.v_sh : nullptr;
  uint8_t* kd = g.k_dst + row * g.budget * g.row_bytes;
  uint8_t* vd = two ? g.v_dst + row * g.budget * g.row_bytes : nullptr;
  for (int64_t base = tid; base < total; base += static_cast<int64_t>(U) * nth) {
    T val[U];
    T* dst[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = base + static_cast<int64_t>(u) * nth;
      dst[u] = nullptr;
      if (i < total) {
        const int64_t p = i / per_pos;
        const int r = static_cast<int>(i - p * per_pos);
        const bool is_v = r >= cpr;
        const int c = is_v ? r - cpr : r;
        const int64_t pos = pos0 + p;
        const int64_t tok = __ldcg(idx_row + pos);  // through L2: may have been written by another CTA
        const int64_t off = pos * g.row_bytes + static_cast<int64_t>(c) * sizeof(T);
        dst[u] = reinterpret_cast<T*>((is_v ? vd : kd) + off);
        if (tok >= 0 && tok < g.tokens) {
          const uint8_t* s = is_v ? vb + tok * g.v_sn : kb + tok * g.k_sn;
          val[u] = __ldg(reinterpret_cast<const T*>(s + static_cast<int64_t>(c) * sizeof(T)));
        } else {
          val[u] = T{};
          raise_status(STATUS_BAD_INDEX);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (dst[u]) *dst[u] = val[u];
  }
}

// Copy positions [pos0, pos0+cnt) of one row; idx_row[pos] names the token.
// U = loads each thread keeps in flight before storing.
template <int U = 4>
__device__ __forceinline__ void gather_rows(const GatherSpec& g, int64_t row, const int64_t* idx_row, int64_t pos0,
                                            int64_t cnt, int tid, int nth) {
  if (cnt <= 0) return;
  switch (g.vec) {
    case 16: gather_rows_vec<uint4, U>(g, row, idx_row, pos0, cnt, tid, nth); break;
    case 8: gather_rows_vec<uint2, U>(g, row, idx_row, pos0, cnt, tid, nth); break;
    case 4: gather_rows_vec<uint32_t, U>(g, row, idx_row, pos0, cnt, tid, nth); break;
    case 2: gather_rows_vec<uint16_t, U>(g, row, idx_row, pos0, cnt, tid, nth); break;
    default: gather_rows_vec<uint8_t, U>(g, row, idx_row, pos0, cnt, tid, nth); break;
  }
}

constexpr int GATHER_THREADS = 256;
constexpr int GATHER_POSITIONS = 32;  // output positions per CTA

// Standalone gather: CTA (row, block of GATHER_POSITIONS positions).
__global__ void __launch_bounds__(GATHER_THREADS) fe_gather_kernel(const GatherSpec g, const int64_t* indices,
                                                                   int64_t blocks_per_row) {
  const int64_t row = blockIdx.x / blocks_per_row;
  const int64_t blk = blockIdx.x - row * blocks_per_row;
  const int64_t pos0 = blk * GATHER_POSITIONS;
  const int64_t cnt = min(static_cast<int64_t>(GATHER_POSITIONS), g.budget - pos0);
  gather_rows(g, row, indices + row * g.budget, pos0, cnt, threadIdx.x, GATHER_THREADS);
}

}  // namespace fe
