// The tiled grouped GEMM on CTA pairs (tcgen05 cta_group::2) for prefill-sized
// groups.
//
// A tile is 256 token rows x 256 weight columns computed by a cluster of two
// CTAs on two SMs: one MMA of M=256 (each CTA holds 128 of the rows, its half
// of A) and N=256 (each CTA holds 128 of the weight rows, its half of B; for
// SwiGLU the even CTA the gate rows, the odd CTA the matching up rows). Each
// SM then stages 32 KB of operands per 64-wide k-block for 128 x 256 x 64 of
// its own MMA work, against 48 KB on the one-SM kernel: shared-memory traffic
// (TMA writes plus MMA operand reads), which bounds the one-SM kernel at about
// half the tensor rate, drops by a third, and six stages fit instead of four.
// Every element is the same K-ordered sum as in the one-SM kernel, so the
// bits do not change.
//
// Protocol (the even CTA of the pair leads):
//  - both CTAs load their halves with TMA (cta_group::2 form, no multicast),
//    and the transfers complete on the LEADER's `full` barrier, which the
//    leader arms for both halves' bytes;
//  - the leader's MMA thread issues cta_group::2 MMAs into both CTAs' TMEM
//    (a pair allocation) and commits to `empty` / `tfull` of both CTAs
//    (tcgen05.commit with a two-CTA mask);
//  - each CTA's epilogue drains its own TMEM rows and releases the accumulator
//    on the leader's `tempty` barrier (one arrival per warp, across the pair).
// Waits are bounded as everywhere; both CTAs meet at a cluster barrier before
// the pair frees its TMEM.
#pragma once
#include "gemm.cuh"

namespace moe {
namespace gemm {

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared-memory address of the same object in the pair's leading CTA: the
// cta_group::2 TMA forms take the barrier address with the peer bit cleared.
constexpr uint32_t kPeerBitMask = 0xFEFFFFFFu;

__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* map, uint64_t* bar, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar) & kPeerBitMask), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const void* map, uint64_t* bar, int32_t c0, int32_t c1,
                                                 int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar) & kPeerBitMask), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void mma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the barrier at this shared-memory offset in both CTAs of
// the pair when every MMA this thread issued has completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// Arrive on the barrier at this offset in CTA `cta` of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t cta) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\t"
      "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
      "r"(cta)
      : "memory");
}

constexpr int kPairStages = 6;
constexpr uint32_t kPairBHalf = 128 * BK * 2;  // 16 KiB: this CTA's 128 weight rows of a k-block
constexpr uint32_t kPairStageBytes = A_BYTES + kPairBHalf;
constexpr int kPairThreads = 192;  // warps: TMA, MMA (leader) / idle, 4 epilogue

struct PairCtrl {
  uint64_t full[kPairStages];
  uint64_t empty[kPairStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int seg_tiles[kMaxSegs];
  int off[kMaxSegs][kMaxGroups + 1];
  int mt[kMaxSegs][kMaxGroups + 1];
};
constexpr uint32_t kPairCtrlBytes = (sizeof(PairCtrl) + 15) & ~uint32_t(15);

constexpr size_t pair_smem_bytes() { return 1024 + kPairStages * kPairStageBytes + kPairCtrlBytes + kEpiStageBytes; }

// Each segment: mma_n = 256 (SwiGLU: 128 gate + 128 up columns; plain: 256
// weight rows, 128 per CTA), one K range, 16-bit bf16/f16 weights.
__global__ void __launch_bounds__(kPairThreads, 1) grouped_gemm_pair_kernel(const __grid_constant__ Params p) {
  constexpr int S = kPairStages;
  constexpr int RT = 2 * BM;  // token rows per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = sA + S * A_BYTES;
  PairCtrl& c = *reinterpret_cast<PairCtrl*>(sB + S * kPairBHalf);
  volatile int* abort_flag = &c.abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pid = static_cast<int>(cluster_id_x());
  const int npairs = static_cast<int>(nclusters_x());

  pdl_trigger();
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&c.tfull[i], 1);
      mbar_init(&c.tempty[i], 8);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(&c.drain, 1);
    c.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&c.tmem_base, 2 * BN);
    tmem_relinquish_pair();
  }
  if (tid == 0) {
    for (int s = 0; s < p.num_segs; ++s) {
      tma_prefetch_desc(&p.seg[s].map_a);
      tma_prefetch_desc(&p.seg[s].map_b0);
      if (p.seg[s].swiglu) tma_prefetch_desc(&p.seg[s].map_b1);
    }
  }
  pdl_wait();
  for (int s = 0; s < p.num_segs; ++s) {
    const Segment& Sg = p.seg[s];
    for (int g = tid; g <= Sg.groups; g += kPairThreads)
      c.off[s][g] = Sg.offsets ? Sg.offsets[g] : (g == 0 ? 0 : Sg.dense_rows);
  }
  __syncthreads();
  if (warp < p.num_segs) {
    const int s = warp;
    const Segment& Sg = p.seg[s];
    int running = 0;
    bool bad = lane == 0 && (c.off[s][0] < 0 || c.off[s][Sg.groups] > Sg.dense_rows);
    if (lane == 0) c.mt[s][0] = 0;
    for (int g0 = 0; g0 < Sg.groups; g0 += 32) {
      const int g = g0 + lane;
      int v = 0;
      if (g < Sg.groups) {
        const int rows = c.off[s][g + 1] - c.off[s][g];
        bad |= rows < 0;
        v = rows > 0 ? (rows + RT - 1) / RT : 0;
      }
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += o;
      }
      if (g < Sg.groups) c.mt[s][g + 1] = running + v;
      running += __shfl_sync(0xffffffffu, v, 31);
    }
    bad = __any_sync(0xffffffffu, bad);
    if (lane == 0) {
      const int oc = out_cols_per_tile(Sg);
      c.seg_tiles[s] = bad ? 0 : running * ((Sg.n + oc - 1) / oc);
      if (bad && p.status && leader) atomicCAS(p.status, 0, MOE_ERR_BAD_OFFSETS);
    }
  }
  tc_fence_before();
  __syncthreads();
  // both CTAs' barriers are initialised and the pair's TMEM allocated before
  // either CTA signals the other
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = c.tmem_base;
  int total = 0;
  for (int s = 0; s < p.num_segs; ++s) total += c.seg_tiles[s];

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      bool ok = true, any = false;
      for (int t = pid; ok && t < total; t += npairs) {
        Tile tl;
        decode_tile(c, p, t, tl, RT);
        const Segment& Sg = p.seg[tl.seg];
        const int n0 = tl.n_tile * out_cols_per_tile(Sg);
        for (int kb = tl.kb0; kb < tl.kb1; ++kb) {
          if (!wait_parity_bounded(&c.empty[stage], phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&c.full[stage], 2 * kPairStageBytes);
          tma_load_2d_pair(sA + stage * A_BYTES, &Sg.map_a, &c.full[stage], kb * BK, tl.row0 + static_cast<int>(rank) * BM);
          if (Sg.swiglu)
            tma_load_3d_pair(sB + stage * kPairBHalf, leader ? &Sg.map_b0 : &Sg.map_b1, &c.full[stage], kb * BK, n0,
                             tl.widx);
          else
            tma_load_3d_pair(sB + stage * kPairBHalf, &Sg.map_b0, &c.full[stage], kb * BK,
                             n0 + static_cast<int>(rank) * BM, tl.widx);
          any = true;
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok && any) {
        // transfers still in flight complete on the leader's barriers: give
        // them time to land in this CTA's shared memory before it exits
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 10000000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader && lane == 0) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      bool ok = true, issued = false;
      for (int t = pid; ok && t < total; t += npairs) {
        Tile tl;
        decode_tile(c, p, t, tl, RT);
        const Segment& Sg = p.seg[tl.seg];
        const uint32_t idesc = idesc_f16(2 * BM, Sg.mma_n, p.in_f16 != 0);
        // the epilogue warps of both CTAs release the accumulator (release.cluster)
        if (!wait_parity_bounded<true>(&c.tempty[acc], acc_phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = tl.kb0; kb < tl.kb1; ++kb) {
          if (!wait_parity_bounded(&c.full[stage], phase, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * kPairBHalf);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            mma_f16_ss_pair(d, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), idesc,
                            (kb != tl.kb0 || kk != 0) ? 1u : 0u);
          }
          issued = true;
          mma_commit_pair(&c.empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit_pair(&c.tfull[acc]);
        acc ^= 1u;
        if (acc == 0) acc_phase ^= 1u;
      }
      if (!ok && issued) {
        mma_commit_pair(&c.drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&c.drain, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int r = static_cast<int>(rank) * BM + q * 32 + lane;  // this thread's row of the 256-row tile
    uint4* estage = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(&c) + kPairCtrlBytes) + q * 128;
    uint32_t acc = 0, acc_phase = 0;
    for (int t = pid; t < total; t += npairs) {
      Tile tl;
      decode_tile(c, p, t, tl, RT);
      const Segment& Sg = p.seg[tl.seg];
      if (!wait_parity_bounded(&c.tfull[acc], acc_phase, abort_flag, p.status)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      epilogue_rows<false>(p, Sg, tl, tb, r, lane, estage);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(&c.tempty[acc], 0);
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (p.remote_out) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

}  // namespace gemm
}  // namespace moe
