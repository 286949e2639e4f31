// The tiled grouped GEMM on CTA pairs (tcgen05 cta_group::2) for prefill-sized
// groups.
//
// A tile is 256 weight rows x up to 256 token rows of one group, computed by a
// cluster of two CTAs on two SMs as MMAs of M=256 and N=token columns: the
// weights sit on the MMA's M side (each CTA holds 128 weight rows, its half of
// A; for SwiGLU 64 gate rows and the same 64 channels' up rows) and the
// group's tokens on the N side (each CTA holds half of the token rows, its
// half of B). N is the group's remaining rows rounded up to 32, so a group's
// last tile computes at most 31 rows that are not stored, where a 256-row
// token tile would compute up to 255. Each SM stages 32 KB of operands per
// 64-wide k-block for 128 x 256 x 64 of its own MMA work, against 48 KB on the
// one-SM kernel, whose shared-memory traffic (TMA writes plus MMA operand
// reads, 128 bytes per cycle measured) bounds it; six stages fit instead of
// four. Every element is the same K-ordered sum as in the one-SM kernel with
// the operands on either side, so the bits do not change.
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
constexpr uint32_t kPairWBytes = BM * BK * 2;  // 16 KiB: this CTA's 128 weight rows of a k-block
constexpr uint32_t kPairXBytes = BM * BK * 2;  // 16 KiB: this CTA's token rows (up to 128) of a k-block
constexpr uint32_t kPairStageBytes = kPairWBytes + kPairXBytes;
constexpr int kPairEpiWarps = 8;  // two per TMEM lane quarter, on alternate 32-token chunks
constexpr int kPairThreads = 32 * (2 + kPairEpiWarps);  // warps: TMA, MMA (leader) / idle, epilogue
constexpr int kPairTokQuant = 32;  // the MMA's token columns are a multiple of this (16 per CTA)
constexpr uint32_t kPairEpiBytes = kPairEpiWarps * 2048;  // per epilogue warp: exchange / transpose buffer

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

constexpr size_t pair_smem_bytes() { return 1024 + kPairStages * kPairStageBytes + kPairCtrlBytes + kPairEpiBytes; }

// MMA N (token columns) for a tile of `rows` token rows.
__device__ __forceinline__ int pair_tok_cols(int rows) {
  const int n = (rows + kPairTokQuant - 1) / kPairTokQuant * kPairTokQuant;
  return n < kPairTokQuant ? kPairTokQuant : n;
}

// Drains this warp's 32 accumulator lanes (weight rows) over the tile's token
// columns, every other chunk of 32 from chunk ch0 (the warp's twin on the same
// lane quarter takes the others). SwiGLU: TMEM lanes 0-63 hold gate rows and 64-127
// the matching up rows of the CTA's 64 channels, so warp q (lanes 32q..) and
// warp q^2 hold gate and up of the same 32 channels; each hands the other the
// half of the 32 tokens that the other finishes, so both compute silu(g) * u
// for 16 tokens. The values are then transposed through the warp's buffer
// into token rows (32 channels = 64 bytes per row) and stored 16 bytes a lane.
__device__ __forceinline__ void pair_epilogue(const Params& p, const Segment& Sg, const Tile& tl, uint32_t tb,
                                              int q, int lane, int rank, int ch0, int bar, float* xmine,
                                              const float* xpeer, uint16_t* tbuf) {
  const int oc = out_cols_per_tile(Sg);
  const int n0 = tl.n_tile * oc;
  const int nchunks = (tl.rows + 31) >> 5;
  const bool swiglu = Sg.swiglu != 0;
  const bool up = swiglu && q >= 2;
  // output channel of lane 0 of this warp
  const int cbase = swiglu ? n0 + rank * (BM / 2) + 32 * (q & 1) : n0 + rank * BM + 32 * q;
  const int cnt = swiglu ? 16 : 32;  // token rows this warp stores per chunk
#pragma unroll 1
  for (int ch = ch0; ch < nchunks; ch += 2) {
    uint32_t v[32];
    tmem_ld_32x32b_x32(tb + ch * 32, v);
    tmem_ld_wait();
    float h[32];
    int t0 = ch * 32;
    if (swiglu) {
      // gate warps keep tokens 0-15 of the chunk, up warps tokens 16-31
#pragma unroll
      for (int j = 0; j < 16; ++j) xmine[j * 32 + lane] = __uint_as_float(up ? v[j] : v[16 + j]);
      named_bar_sync(bar, 64);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float o = xpeer[j * 32 + lane];
        const float m = __uint_as_float(up ? v[16 + j] : v[j]);
        const float g = up ? o : m;
        const float u = up ? m : o;
        h[j] = g / (1.0f + __expf(-g)) * u;
      }
      named_bar_sync(bar, 64);
      if (up) t0 += 16;
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) h[j] = __uint_as_float(v[j]);
    }
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < cnt) tbuf[j * 32 + lane] = static_cast<uint16_t>(pack2(h[j], 0.f, p.in_f16) & 0xFFFFu);
    __syncwarp();
    for (int i = lane; i < cnt * 4; i += 32) {
      const int j = i >> 2, vq = i & 3;
      const int tok = t0 + j;
      if (tok >= tl.rows) continue;
      int64_t orow = tl.row0 + tok;
      uint16_t* obase = reinterpret_cast<uint16_t*>(Sg.out);
      if (Sg.out_rows) {
        const int code = Sg.out_rows[orow];
        const int dst = code & 15;
        orow = code >> 4;
        if (code < 0 || dst >= Sg.out_table_n || orow >= Sg.out_table_rows) {
          if (p.status) atomicCAS(p.status, 0, MOE_ERR_BAD_OFFSETS);
          continue;
        }
        obase = reinterpret_cast<uint16_t*>(Sg.out_table[dst]);
      }
      const int col = cbase + vq * 8;
      uint16_t* d = obase + orow * Sg.ldo + col;
      const uint16_t* s = tbuf + j * 32 + vq * 8;
      if (col + 8 <= Sg.n && (reinterpret_cast<uintptr_t>(d) & 15) == 0) {
        *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(s);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (col + e < Sg.n) d[e] = s[e];
      }
    }
    __syncwarp();
  }
}

// Each segment: 16-bit weights, one K range, 16-bit outputs; SwiGLU: 128
// channels per tile (64 per CTA), plain: 256 output channels (128 per CTA).
__global__ void __launch_bounds__(kPairThreads, 1) grouped_gemm_pair_kernel(const __grid_constant__ Params p) {
  constexpr int S = kPairStages;
  constexpr int RT = 2 * BM;  // token rows per tile (most)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = base;                     // S weight slots (1024-aligned)
  uint8_t* sX = sW + S * kPairWBytes;     // S token slots (1024-aligned)
  PairCtrl& c = *reinterpret_cast<PairCtrl*>(sX + S * kPairXBytes);
  uint8_t* epi = reinterpret_cast<uint8_t*>(&c) + kPairCtrlBytes;
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
      mbar_init(&c.tempty[i], 2 * kPairEpiWarps);  // one arrival per epilogue warp of both CTAs
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
        // the even CTA holds the tile's first half of token columns, the odd CTA the second
        const int half = pair_tok_cols(tl.rows) / 2;
        const int tok0 = tl.row0 + static_cast<int>(rank) * half;
        const uint32_t cta_bytes = kPairStageBytes;
        for (int kb = tl.kb0; kb < tl.kb1; ++kb) {
          if (!wait_parity_bounded(&c.empty[stage], phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&c.full[stage], 2 * cta_bytes);
          uint8_t* w_dst = sW + stage * kPairWBytes;
          if (Sg.swiglu) {
            // 64 gate rows, then the same 64 channels' up rows
            const int ch0 = n0 + static_cast<int>(rank) * (BM / 2);
            tma_load_3d_pair(w_dst, &Sg.map_b0, &c.full[stage], kb * BK, ch0, tl.widx);
            tma_load_3d_pair(w_dst + kPairWBytes / 2, &Sg.map_b1, &c.full[stage], kb * BK, ch0, tl.widx);
          } else {
            tma_load_3d_pair(w_dst, &Sg.map_b0, &c.full[stage], kb * BK, n0 + static_cast<int>(rank) * BM,
                             tl.widx);
          }
          tma_load_2d_pair(sX + stage * kPairXBytes, &Sg.map_a, &c.full[stage], kb * BK, tok0);
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
        // M = the pair's 256 weight rows, N = the tile's token columns
        const uint32_t idesc = idesc_f16(2 * BM, pair_tok_cols(tl.rows), p.in_f16 != 0);
        // the epilogue warps of both CTAs release the accumulator (release.cluster)
        if (!wait_parity_bounded<true>(&c.tempty[acc], acc_phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = tl.kb0; kb < tl.kb1; ++kb) {
          if (!wait_parity_bounded(&c.full[stage], phase, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sW + stage * kPairWBytes);
          const uint32_t b0 = smem_u32(sX + stage * kPairXBytes);
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
    const int q = warp & 3;          // TMEM lane quarter of this warp
    const int h = (warp - 2) >> 2;   // which of the quarter's two warps: even or odd chunks
    const int bar = 1 + (q & 1) + 2 * h;  // named barrier shared with the SwiGLU partner (quarter q ^ 2)
    float* xmine = reinterpret_cast<float*>(epi + (4 * h + q) * 2048);
    const float* xpeer = reinterpret_cast<const float*>(epi + (4 * h + (q ^ 2)) * 2048);
    uint16_t* tbuf = reinterpret_cast<uint16_t*>(epi + (4 * h + q) * 2048);
    uint32_t acc = 0, acc_phase = 0;
    for (int t = pid; t < total; t += npairs) {
      Tile tl;
      decode_tile(c, p, t, tl, RT);
      const Segment& Sg = p.seg[tl.seg];
      bool got = wait_parity_bounded(&c.tfull[acc], acc_phase, abort_flag, p.status);
      // the two warps that exchange SwiGLU halves leave together or not at all
      got = named_bar_and(bar, 64, got);
      if (!got) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      pair_epilogue(p, Sg, tl, tb, q, lane, static_cast<int>(rank), h, bar, xmine, xpeer, tbuf);
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
