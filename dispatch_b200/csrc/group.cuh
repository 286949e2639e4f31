// Stable counting sort of the T*k flat (token, slot) pairs by expert id.
//
// Pass 1 (group_hist_kernel, one CTA per 256-pair chunk): the chunk's expert
// histogram into the workspace.
// Pass 2 (group_scatter_kernel, same chunks): each CTA reads all chunk
// histograms (nchunks x E int32, L2-resident), forms per-expert totals, the
// exclusive prefix sum `offsets` and its own chunk base rows; a pair's grouped
// row = chunk base + rows of the same expert in earlier warps of the chunk +
// its rank among equal ids in its own warp (match.any + popc). That is exactly
// a stable argsort. The pass also writes the inverse permutation, the sorted
// token ids / weights, and gathers the activation rows (16-byte vectors,
// converted to the tensor-core type) into expert-contiguous order.
// No atomics across CTAs, no ticket, nothing to re-arm: the workspace needs no
// initialisation.
#pragma once
#include "ptx.cuh"

namespace moe {
namespace group {

constexpr int kThreads = 256;
constexpr int kChunk = kThreads;
constexpr int kMaxE = 256;
constexpr int kHistTile = 8192;  // int32 histogram entries staged per block (32 KiB)
static_assert(kMaxE <= kThreads, "one thread per expert in the scatter's base sums");

struct Params {
  const void* idx;
  int idx64;
  const float* w;
  int64_t n;  // T * k
  int k;
  int E;
  int nchunks;
  int32_t* counts;
  int32_t* offsets;
  int32_t* pos;
  int64_t* sorted_token_idx;
  float* sorted_weight;
  const void* x;
  int x_dtype;
  int64_t H;
  void* xs;
  int xs_f16;
  int32_t* hist;  // [nchunks][E]
  int32_t* status;
};

__device__ __forceinline__ int load_id(const Params& p, int64_t f) {
  return p.idx64 ? static_cast<int>(reinterpret_cast<const int64_t*>(p.idx)[f])
                 : reinterpret_cast<const int32_t*>(p.idx)[f];
}

__global__ void __launch_bounds__(kThreads) group_hist_kernel(const Params p) {
  pdl_trigger();
  pdl_wait();  // before the first global memory access
  __shared__ int hist[kMaxE];
  const int tid = threadIdx.x;
  for (int e = tid; e < p.E; e += kThreads) hist[e] = 0;
  __syncthreads();
  const int64_t f = static_cast<int64_t>(blockIdx.x) * kChunk + tid;
  if (f < p.n) {
    const int e = load_id(p, f);
    if (e < 0 || e >= p.E) {
      if (p.status) atomicCAS(p.status, 0, MOE_ERR_BAD_EXPERT);
    } else {
      atomicAdd(&hist[e], 1);
    }
  }
  __syncthreads();
  for (int e = tid; e < p.E; e += kThreads) p.hist[static_cast<int64_t>(blockIdx.x) * p.E + e] = hist[e];
}

__device__ __forceinline__ void copy_row(const Params& p, int64_t dst_row, int64_t src_row, int lane) {
  const int64_t H = p.H;
  if (p.x_dtype == MOE_DT_F32) {
    const float* src = reinterpret_cast<const float*>(p.x) + src_row * H;
    for (int64_t h = lane * 8; h < H; h += 256) {
      const float4 a = *reinterpret_cast<const float4*>(src + h);
      const float4 b = *reinterpret_cast<const float4*>(src + h + 4);
      uint4 o;
      if (p.xs_f16) {
        __half2 q0 = __floats2half2_rn(a.x, a.y), q1 = __floats2half2_rn(a.z, a.w);
        __half2 q2 = __floats2half2_rn(b.x, b.y), q3 = __floats2half2_rn(b.z, b.w);
        o = make_uint4(*reinterpret_cast<uint32_t*>(&q0), *reinterpret_cast<uint32_t*>(&q1),
                       *reinterpret_cast<uint32_t*>(&q2), *reinterpret_cast<uint32_t*>(&q3));
      } else {
        __nv_bfloat162 q0 = __floats2bfloat162_rn(a.x, a.y), q1 = __floats2bfloat162_rn(a.z, a.w);
        __nv_bfloat162 q2 = __floats2bfloat162_rn(b.x, b.y), q3 = __floats2bfloat162_rn(b.z, b.w);
        o = make_uint4(*reinterpret_cast<uint32_t*>(&q0), *reinterpret_cast<uint32_t*>(&q1),
                       *reinterpret_cast<uint32_t*>(&q2), *reinterpret_cast<uint32_t*>(&q3));
      }
      *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.xs) + dst_row * H + h) = o;
    }
  } else {
    // same 16-bit type (checked on the host)
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.x) + src_row * H);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.xs) + dst_row * H);
    for (int64_t v = lane; v < H / 8; v += 32) dst[v] = __ldg(src + v);
  }
}

__global__ void __launch_bounds__(kThreads) group_scatter_kernel(const Params p) {
  pdl_trigger();
  pdl_wait();  // before the first global memory access
  __shared__ int base[kMaxE];
  __shared__ int total[kMaxE];
  __shared__ int wcnt[kThreads / 32][kMaxE];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x;
  // per expert: rows in earlier chunks and rows overall. The (nchunks, E)
  // histograms are staged through shared memory a block of chunks at a time
  // (every thread's loads of a block are independent and in flight together);
  // a per-thread serial walk over global memory was a long chain of L2
  // round trips at prefill sizes.
  __shared__ int tile[kHistTile];
  const int rows_per_tile = kHistTile / p.E;
  int before = 0, all = 0;  // for expert tid (tid < E; E <= kThreads)
  for (int cc0 = 0; cc0 < p.nchunks; cc0 += rows_per_tile) {
    const int rows = min(rows_per_tile, p.nchunks - cc0);
    const int n_items = rows * p.E;
    const int* src = p.hist + static_cast<int64_t>(cc0) * p.E;
    for (int i = tid; i < n_items; i += kThreads) tile[i] = src[i];
    __syncthreads();
    if (tid < p.E) {
      for (int j = 0; j < rows; ++j) {
        const int v = tile[j * p.E + tid];
        before += cc0 + j < c ? v : 0;
        all += v;
      }
    }
    __syncthreads();
  }
  if (tid < p.E) {
    base[tid] = before;
    total[tid] = all;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) wcnt[w][tid] = 0;
  }
  __syncthreads();
  // exclusive prefix sum over experts (one warp), added to the chunk bases
  if (warp == 0) {
    int running = 0;
    for (int e0 = 0; e0 < p.E; e0 += 32) {
      const int e = e0 + lane;
      const int cnt = e < p.E ? total[e] : 0;
      int v = cnt;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += o;
      }
      if (e < p.E) {
        const int off = running + v - cnt;
        base[e] += off;
        if (c == 0 && blockIdx.y == 0) {
          p.counts[e] = cnt;
          p.offsets[e] = off;
        }
      }
      running += __shfl_sync(0xffffffffu, v, 31);
    }
    if (c == 0 && lane == 0 && blockIdx.y == 0) p.offsets[p.E] = running;
  }
  __syncthreads();
  const int64_t f = static_cast<int64_t>(c) * kChunk + tid;
  int e = -1;
  if (f < p.n) {
    e = load_id(p, f);
    if (e < 0 || e >= p.E) e = -1;
  }
  const uint32_t peers = __match_any_sync(0xffffffffu, e);
  const uint32_t lt = (1u << lane) - 1u;
  const int rank = __popc(peers & lt);
  if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(peers);
  __syncthreads();
  int row = -1;
  const bool writer = blockIdx.y == 0;  // copy slices > 0 only gather rows
  if (e >= 0) {
    row = base[e] + rank;
    for (int w = 0; w < warp; ++w) row += wcnt[w][e];
    if (writer) {
      p.pos[f] = row;
      const int64_t tok = f / p.k;
      if (p.sorted_token_idx) p.sorted_token_idx[row] = tok;
      if (p.sorted_weight) p.sorted_weight[row] = p.w[f];
    }
  } else if (f < p.n && writer) {
    p.pos[f] = -1;  // invalid id: the histogram pass already raised the status
  }
  if (!p.xs) return;
  if (p.x_dtype == MOE_DT_F32) {
    for (int i = 0; i < 32; ++i) {
      const int r = __shfl_sync(0xffffffffu, row, i);
      if (r < 0) continue;
      const int64_t fi = static_cast<int64_t>(c) * kChunk + warp * 32 + i;
      copy_row(p, r, fi / p.k, lane);
    }
    return;
  }
  // 16-bit rows: this CTA copies column slice blockIdx.y of its 32 x 8 rows,
  // eight independent 16-byte loads in flight per lane.
  __shared__ int s_dst[kThreads / 32][32];
  __shared__ int s_src[kThreads / 32][32];
  s_dst[warp][lane] = row;
  s_src[warp][lane] = row >= 0 ? static_cast<int>(f / p.k) : -1;
  __syncwarp();
  const int per_row = static_cast<int>(p.H / 8);
  const int cols = per_row / static_cast<int>(gridDim.y);
  const int c0 = static_cast<int>(blockIdx.y) * cols;
  const int n_items = 32 * cols;
  const uint4* src = reinterpret_cast<const uint4*>(p.x);
  uint4* dst = reinterpret_cast<uint4*>(p.xs);
  for (int b0 = 0; b0 < n_items; b0 += 32 * 8) {
    uint4 v[8];
    int64_t to[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = b0 + u * 32 + lane;
      to[u] = -1;
      if (i < n_items) {
        const int r = i / cols, cc = c0 + i % cols;
        const int s = s_src[warp][r];
        if (s >= 0) {
          v[u] = __ldg(src + static_cast<int64_t>(s) * per_row + cc);
          to[u] = static_cast<int64_t>(s_dst[warp][r]) * per_row + cc;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (to[u] >= 0) dst[to[u]] = v[u];
  }
}

}  // namespace group
}  // namespace moe
