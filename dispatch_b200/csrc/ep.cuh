// Expert-parallel dispatch over NVLink peer memory.
//
// One CTA per 256 flat (token, slot) pairs, like the grouping kernels. Every
// CTA derives the receive layout from the (world, E) count matrix: for expert
// e owned by rank d = e / E_loc (local index j),
//   first row of this rank's block = sum over experts j' < j of d of all
//   sources' rows + rows of expert e from sources below this rank,
// then a slot's remote row is that base plus its rank among this rank's rows
// of e (its grouped row minus offsets[e]; the grouping is a stable sort, so
// this is the slot's stable order). Rows are copied with 16-byte vectors,
// eight loads in flight per lane, over column slices (grid.y) so small
// batches still spread over the GPU; stores go straight to the owner's
// receive buffer through its IPC mapping. No atomics, no flags: ordering
// against the owner's reads is the caller's barrier after this kernel.
#pragma once
#include "ptx.cuh"

namespace moe {
namespace ep {

constexpr int kThreads = 256;
constexpr int kChunk = kThreads;
constexpr int kMaxE = 256;
constexpr int kMaxRanks = 16;

struct DispatchParams {
  const void* x;  // (T, H) 16-bit rows
  int64_t H;
  const void* idx;
  int idx64;
  int64_t n;  // T * k
  int k;
  const int32_t* pos;         // (n) grouped row of each slot on this rank
  const int32_t* offsets;     // (E + 1) this rank's group offsets
  const int32_t* counts_all;  // (world, E)
  int rank;
  int world;
  int E;
  int e_loc;
  void* const* peer_recv;     // (world) receive rows, (recv_cap, H) each
  int32_t* const* peer_ret;   // (world) return codes, (recv_cap) each
  int64_t recv_cap;
  int32_t* recv_offsets;  // (e_loc + 1) on this rank
  int32_t* status;
};

__device__ __forceinline__ int load_id(const DispatchParams& p, int64_t f) {
  return p.idx64 ? static_cast<int>(reinterpret_cast<const int64_t*>(p.idx)[f])
                 : reinterpret_cast<const int32_t*>(p.idx)[f];
}

__global__ void __launch_bounds__(kThreads) dispatch_kernel(const DispatchParams p) {
  pdl_trigger();
  pdl_wait();  // before the first global memory access
  __shared__ int s_scan[kMaxE + 1];  // exclusive prefix over experts of all sources' rows
  __shared__ int s_pre[kMaxE];       // rows of expert e from sources below this rank
  __shared__ uint4* s_recv[kMaxRanks];
  __shared__ int32_t* s_ret[kMaxRanks];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid < p.world) {
    s_recv[tid] = reinterpret_cast<uint4*>(p.peer_recv[tid]);
    s_ret[tid] = p.peer_ret[tid];
  }
  for (int e = tid; e < p.E; e += kThreads) {
    int tot = 0, pre = 0;
    for (int s = 0; s < p.world; ++s) {
      const int v = p.counts_all[s * p.E + e];
      tot += v;
      pre += s < p.rank ? v : 0;
    }
    s_scan[e] = tot;
    s_pre[e] = pre;
  }
  __syncthreads();
  if (warp == 0) {
    int running = 0;
    for (int e0 = 0; e0 < p.E; e0 += 32) {
      const int e = e0 + lane;
      const int cnt = e < p.E ? s_scan[e] : 0;
      int v = cnt;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += o;
      }
      if (e < p.E) s_scan[e] = running + v - cnt;
      running += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) s_scan[p.E] = running;
  }
  __syncthreads();
  if (blockIdx.x == 0 && blockIdx.y == 0) {
    const int first = p.rank * p.e_loc;
    for (int j = tid; j <= p.e_loc; j += kThreads) p.recv_offsets[j] = s_scan[first + j] - s_scan[first];
  }
  const int64_t f = static_cast<int64_t>(blockIdx.x) * kChunk + tid;
  int dst = -1;  // owner rank
  int64_t q = -1;  // row on the owner
  int src = -1;    // token
  if (f < p.n) {
    const int e = load_id(p, f);
    if (e >= 0 && e < p.E) {
      const int row = p.pos[f];
      const int lo = p.offsets[e], hi = p.offsets[e + 1];
      const int d = e / p.e_loc;
      const int64_t qq = static_cast<int64_t>(s_scan[e] - s_scan[d * p.e_loc] + s_pre[e]) + (row - lo);
      if (row < lo || row >= hi || qq >= p.recv_cap) {
        if (p.status) atomicCAS(p.status, 0, MOE_ERR_BAD_OFFSETS);
      } else {
        dst = d;
        q = qq;
        src = static_cast<int>(f / p.k);
        if (blockIdx.y == 0) s_ret[d][q] = (row << 4) | p.rank;
      }
    } else if (p.status) {
      atomicCAS(p.status, 0, MOE_ERR_BAD_EXPERT);
    }
  }
  // this warp's 32 rows, column slice blockIdx.y of each
  __shared__ uint4* s_dst[kThreads / 32][32];
  __shared__ int s_src[kThreads / 32][32];
  const int per_row = static_cast<int>(p.H / 8);
  s_dst[warp][lane] = dst >= 0 ? s_recv[dst] + q * per_row : nullptr;
  s_src[warp][lane] = src;
  __syncwarp();
  const int cols = per_row / static_cast<int>(gridDim.y);
  const int c0 = static_cast<int>(blockIdx.y) * cols;
  const int n_items = 32 * cols;
  const uint4* xv = reinterpret_cast<const uint4*>(p.x);
  for (int b0 = 0; b0 < n_items; b0 += 32 * 8) {
    uint4 v[8];
    uint4* to[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = b0 + u * 32 + lane;
      to[u] = nullptr;
      if (i < n_items) {
        const int r = i / cols, cc = c0 + i % cols;
        const int s = s_src[warp][r];
        if (s >= 0) {
          v[u] = __ldg(xv + static_cast<int64_t>(s) * per_row + cc);
          to[u] = s_dst[warp][r] + cc;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (to[u]) *to[u] = v[u];
  }
  // make this thread's peer stores visible system-wide before the kernel ends
  __threadfence_system();
}

// ---------------------------------------------------------------------------
// Exchange / barrier over the ranks' signal buffers (one CTA). Signal buffer
// layout: int32 flags[kFlagSlots][kMaxRanks] in the first kSignalHeader bytes,
// then an int32 payload area of (world, n).
constexpr int kFlagSlots = 4;
constexpr int kSignalHeader = 256;
static_assert(kFlagSlots * kMaxRanks * 4 <= kSignalHeader, "flag rows fit the header");

struct ExchangeParams {
  const int32_t* payload;  // n int32 of this rank (may be null when n == 0)
  int64_t n;
  void* const* peer_signal;  // (world) signal buffers as mapped here (own entry = local)
  int32_t* local_signal;
  int slot, rank, world;
  int32_t epoch;
  int32_t* status;
};

__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) exchange_kernel(const ExchangeParams p) {
  pdl_trigger();
  pdl_wait();  // the previous kernel's stores (payload, peer rows) are complete
  const int tid = threadIdx.x;
  for (int d = 0; d < p.world; ++d) {
    int32_t* dst = reinterpret_cast<int32_t*>(static_cast<char*>(p.peer_signal[d]) + kSignalHeader) + p.rank * p.n;
    for (int64_t i = tid; i < p.n; i += blockDim.x) dst[i] = p.payload[i];
  }
  __threadfence_system();
  __syncthreads();
  if (tid < p.world) {
    st_release_sys(static_cast<int32_t*>(p.peer_signal[tid]) + p.slot * kMaxRanks + p.rank, p.epoch);
    const int32_t* f = p.local_signal + p.slot * kMaxRanks + tid;
    const uint64_t t0 = globaltimer_ns();
    // wrap-safe "flag < epoch" on the int32 epoch sequence
    while (static_cast<int32_t>(static_cast<uint32_t>(ld_acquire_sys(f)) - static_cast<uint32_t>(p.epoch)) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        if (p.status) atomicCAS(p.status, 0, MOE_ERR_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
}

}  // namespace ep
}  // namespace moe
