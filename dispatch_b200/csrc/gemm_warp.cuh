// Warp-MMA weight streaming for decode-sized groups (a few token rows per
// expert).
//
// With one or two token rows per expert the tcgen05 kernels, which issue every
// MMA of a CTA from one thread, read their weights well below HBM speed (C2
// T=16: both FFN launches at ~4.75 TB/s, against 6.9 TB/s for the same TMA
// boxes streamed with no math). Here eight (or four) warps per CTA each run
// their own short chain of warp-level MMAs (mma.sync m16n8k16: 16 weight rows
// x 8 token rows x 16 K) on operands that TMA stages in shared memory, so a
// CTA keeps that many chains in flight and an SM two CTAs; the same launches
// read at 5.7-5.9 TB/s.
//
// Bits: an m16n8k16 MMA chain walked over K in order, 16 at a time, with f32
// accumulation gives the same f32 values as the tcgen05 MMAs of the other
// kernels (checked on B200 bit for bit against the tcgen05 router logits, and
// the layer outputs of all kernels are compared in the tests), so the kernel
// choice changes speed only.
//
// Unit of work (a "tile"): (segment, group, channel block, token block): 16 x
// kWarps weight rows (128 or 64) -- SwiGLU: half gate rows + the matching up
// rows, plain: output channels -- against a token tile of nt rows (8, 16 or
// 32, per launch) of one group, over all of K. Warp 0 lane 0 issues the TMA
// loads of each 64-wide k-block (the weight rows and the token rows, both
// 128-byte swizzled) into a ring of four (128-row tiles) or eight (64-row
// tiles) stages; MMA warp w (1..kWarps) owns weight rows 16(w-1) ..
// 16(w-1)+15, reads its operands with ldmatrix and keeps up to four 16x8
// accumulators (32 token rows). SwiGLU: the up warp of each pair hands its
// accumulators to the matching gate warp through shared memory. Every wait is
// bounded; the two warps of a pair agree on every wait's outcome before they
// meet, so a timeout in one cannot leave the other waiting.
#pragma once
#include "gemm.cuh"

namespace moe {
namespace gemm {

constexpr int kWTok = 32;  // most token rows per tile (four n8 MMA tiles)
constexpr uint32_t kWXBytes = kWTok * BK * 2;  // token-row slot of a stage: 4 KiB

// kWarps MMA warps own 16 weight rows each: 8 warps (128-row tiles, four
// stages, two CTAs per SM) when a launch has many tiles, 4 warps (64-row
// tiles, eight stages, two CTAs per SM) when it has few, so that a decode
// step's few tiles still keep enough weight bytes in flight per SM.
template <int kWarps>
struct WarpConfig {
  static constexpr int kRows = 16 * kWarps;
  static constexpr int kStages = kWarps == 8 ? 4 : 8;
  static constexpr uint32_t kWBytes = kRows * BK * 2;
  static constexpr int kThreads = 32 * (1 + kWarps);
  static constexpr int kPairs = kWarps / 2;  // SwiGLU: gate warp w with up warp w + kPairs
};

struct WarpCtrl {
  uint64_t full[8];
  uint64_t empty[8];
  int abort;
  int seg_tiles[kMaxSegs];
  int off[kMaxSegs][kMaxGroups + 1];
  int mt[kMaxSegs][kMaxGroups + 1];
};
constexpr uint32_t kWCtrlBytes = (sizeof(WarpCtrl) + 15) & ~uint32_t(15);
// the up warps' accumulators for the gate warps: up to 4 pairs x 32 lanes x 16 floats
constexpr uint32_t kWXchgBytes = 4 * 32 * 16 * 4;

template <int kWarps>
constexpr size_t warp_smem_bytes() {
  return 1024 + WarpConfig<kWarps>::kStages * (WarpConfig<kWarps>::kWBytes + kWXBytes) + kWCtrlBytes + kWXchgBytes;
}

// One launch: the segments and the token-row tile (8, 16 or 32) of every tile.
struct WarpParams {
  Params p;
  int nt;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D (16x8, f32) += A (16x16, row) * B (16x8, col) on bf16 or f16 operands.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                          int f16) {
  if (f16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// Shared-memory address of 16-byte chunk `chunk` (0..7) of row `row` in a
// 128-byte-swizzled tile of 128-byte rows (the layout TMA writes).
__device__ __forceinline__ uint32_t sw128_addr(uint32_t base, int row, int chunk) {
  return base + static_cast<uint32_t>(row) * 128u + (static_cast<uint32_t>(chunk ^ (row & 7)) << 4);
}

// Stores one output value (16-bit) of row r (of the segment's logical rows)
// and channel ch, through the scattered-output table when the segment has one.
__device__ __forceinline__ void warp_store(const Params& p, const Segment& Sg, int64_t r, int ch, float v) {
  uint16_t* obase = reinterpret_cast<uint16_t*>(Sg.out);
  int64_t orow = r;
  if (Sg.out_rows) {
    const int code = Sg.out_rows[r];
    const int dst = code & 15;
    orow = code >> 4;
    if (code < 0 || dst >= Sg.out_table_n || orow >= Sg.out_table_rows) {
      if (p.status) atomicCAS(p.status, 0, MOE_ERR_BAD_OFFSETS);
      return;
    }
    obase = reinterpret_cast<uint16_t*>(Sg.out_table[dst]);
  }
  obase[orow * Sg.ldo + ch] = static_cast<uint16_t>(pack2(v, 0.f, p.in_f16) & 0xFFFFu);
}

// Exact int8 -> bf16/f16 of two packed bytes (the low byte in the low half).
__device__ __forceinline__ uint32_t cvt_i8x2(uint32_t v, int f16) {
  const uint32_t w = (v ^ 0x8080u) & 0xFFFFu;
  return pack_exact2(sub_magic_f32x2(__byte_perm(w, 0x4B000000u, 0x7540u), __byte_perm(w, 0x4B000000u, 0x7541u)),
                     f16);
}

// Segments: mma_n = 16 x kWarps (SwiGLU: half of it output channels per
// tile), 16-bit weights -- or, in the int8 build, int8 weights with
// per-channel scales applied in the epilogue as in the tiled kernel -- one K
// range, 16-bit outputs, no gathered rows. An int8 stage holds the weight rows
// as 64-byte unswizzled rows; each MMA warp converts its own 16 rows straight
// into the MMA's operand registers (exact), so no converted copy is written.
template <int kWarps, bool kInt8>
__global__ void __launch_bounds__(WarpConfig<kWarps>::kThreads)
    grouped_gemm_warp_kernel(const __grid_constant__ WarpParams wp) {
  using Cfg = WarpConfig<kWarps>;
  constexpr int S = Cfg::kStages;
  constexpr uint32_t kWWBytes = Cfg::kWBytes;
  constexpr int kWThreads = Cfg::kThreads;
  const Params& p = wp.p;
  const int nt_tile = wp.nt;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = base;                   // S weight slots (1024-aligned)
  uint8_t* sX = sW + S * kWWBytes;      // S token-row slots of 4 KiB (1024-aligned)
  WarpCtrl& c = *reinterpret_cast<WarpCtrl*>(sX + S * kWXBytes);
  float* xchg = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(&c) + kWCtrlBytes);
  volatile int* abort_flag = &c.abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  pdl_trigger();
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.empty[i], kWarps);
    }
    c.abort = 0;
    fence_mbar_init();
    for (int s = 0; s < p.num_segs; ++s) {
      tma_prefetch_desc(&p.seg[s].map_a);
      tma_prefetch_desc(&p.seg[s].map_b0);
      if (p.seg[s].swiglu) tma_prefetch_desc(&p.seg[s].map_b1);
    }
  }
  pdl_wait();
  for (int s = 0; s < p.num_segs; ++s) {
    const Segment& Sg = p.seg[s];
    for (int g = tid; g <= Sg.groups; g += kWThreads)
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
        v = rows > 0 ? (rows + nt_tile - 1) / nt_tile : 0;
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
      if (bad && p.status) atomicCAS(p.status, 0, MOE_ERR_BAD_OFFSETS);
    }
  }
  __syncthreads();
  int total = 0;
  for (int s = 0; s < p.num_segs; ++s) total += c.seg_tiles[s];

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        Tile tl;
        decode_tile(c, p, t, tl, nt_tile);
        const Segment& Sg = p.seg[tl.seg];
        const int n0 = tl.n_tile * out_cols_per_tile(Sg);
        const bool q8 = kInt8 && Sg.b_int8;
        // int8 rows are half as wide: a stage then carries two k-blocks (the
        // second fully beyond K is zero-filled and not computed)
        const int kpb = (q8 && 2 * nt_tile * BK * 2 <= static_cast<int>(kWXBytes)) ? 2 : 1;
        for (int kb = tl.kb0; kb < tl.kb1; kb += kpb) {
          if (!wait_parity_bounded(&c.empty[stage], phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
          const uint32_t w_bytes = q8 ? kWWBytes / 2 : kWWBytes;  // per k-block; int8: 64-byte rows
          const uint32_t x_bytes = static_cast<uint32_t>(nt_tile) * BK * 2;
          mbar_arrive_expect_tx(&c.full[stage], static_cast<uint32_t>(kpb) * (w_bytes + x_bytes));
          for (int j = 0; j < kpb; ++j) {
            uint8_t* w_dst = sW + stage * kWWBytes + j * w_bytes;
            tma_load_2d(sX + stage * kWXBytes + j * x_bytes, &Sg.map_a, &c.full[stage], (kb + j) * BK, tl.row0);
            tma_load_3d(w_dst, &Sg.map_b0, &c.full[stage], (kb + j) * BK, n0, tl.widx);
            if (Sg.swiglu)
              tma_load_3d(w_dst + w_bytes / 2, &Sg.map_b1, &c.full[stage], (kb + j) * BK, n0, tl.widx);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        // let every copy in flight land before the CTA exits
        for (int i = 0; i < S; ++i) {
          if (!(issued_mask & (1u << i))) continue;
          const uint32_t par = (issued_parity >> i) & 1u;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&c.full[i], par) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ MMA warps + epilogue
    const int w = warp - 1;                  // owns weight rows 16w .. 16w+15 of each stage
    const int pair = w % Cfg::kPairs;        // SwiGLU: gate warp w (< kPairs) with up warp w + kPairs
    const bool up_warp = w >= Cfg::kPairs;
    const int g = lane >> 2, tq = lane & 3;
    // ldmatrix row addresses: A (weights) x4 = rows 0-7 / 8-15 x k 0-7 / 8-15;
    // B (tokens) x4 = tokens 0-7 x k 0-7, k 8-15, tokens 8-15 x k 0-7, k 8-15
    const int a_row = 16 * w + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int a_khalf = lane >> 4;
    const int b_row = (lane & 7) + ((lane >> 4) & 1) * 8;
    const int b_khalf = (lane >> 3) & 1;
    uint32_t stage = 0, phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      Tile tl;
      decode_tile(c, p, t, tl, nt_tile);
      const Segment& Sg = p.seg[tl.seg];
      const bool q8 = kInt8 && Sg.b_int8;
      const int nt = (tl.rows + 7) >> 3;  // n8 token tiles in use (1 .. nt_tile / 8)
      float acc[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;
      const int kpb = (q8 && 2 * nt_tile * BK * 2 <= static_cast<int>(kWXBytes)) ? 2 : 1;
      for (int kb = tl.kb0; ok && kb < tl.kb1; kb += kpb) {
        // every lane waits (its own acquire of the TMA bytes); the warp then
        // agrees on the outcome so that it leaves the loop together
        const bool got = wait_parity_bounded(&c.full[stage], phase, abort_flag, p.status);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        const uint32_t wbase = smem_u32(sW + stage * kWWBytes);
        for (int j = 0; j < kpb && kb + j < tl.kb1; ++j) {
        const uint32_t xbase = smem_u32(sX + stage * kWXBytes) + static_cast<uint32_t>(j * nt_tile * BK * 2);
        // int8: this thread's bytes (rows g and g + 8, k = 2tq.. and 8 + 2tq..)
        const uint8_t* q0 = sW + stage * kWWBytes + j * (kWWBytes / 2) + (16 * w + g) * BK + 2 * tq;
#pragma unroll
        for (int s = 0; s < BK / 16; ++s) {
          uint32_t a[4];
          if (q8) {
            const uint8_t* qs = q0 + 16 * s;
            a[0] = cvt_i8x2(*reinterpret_cast<const uint16_t*>(qs), p.in_f16);
            a[1] = cvt_i8x2(*reinterpret_cast<const uint16_t*>(qs + 8 * BK), p.in_f16);
            a[2] = cvt_i8x2(*reinterpret_cast<const uint16_t*>(qs + 8), p.in_f16);
            a[3] = cvt_i8x2(*reinterpret_cast<const uint16_t*>(qs + 8 * BK + 8), p.in_f16);
          } else {
            ldsm_x4(sw128_addr(wbase, a_row, 2 * s + a_khalf), a[0], a[1], a[2], a[3]);
          }
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            if (2 * jj < nt) {
              uint32_t b[4];
              ldsm_x4(sw128_addr(xbase, 16 * jj + b_row, 2 * s + b_khalf), b[0], b[1], b[2], b[3]);
              mma_16816(acc[2 * jj], a, b[0], b[1], p.in_f16);
              if (2 * jj + 1 < nt) mma_16816(acc[2 * jj + 1], a, b[2], b[3], p.in_f16);
            }
          }
        }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&c.empty[stage]);
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      const int oc = out_cols_per_tile(Sg);
      const int n0 = tl.n_tile * oc;
      const int64_t sc_base = static_cast<int64_t>(tl.widx) * Sg.n;
      if (Sg.swiglu) {
        // both warps of a pair leave together or not at all
        ok = named_bar_and(1 + pair, 64, ok);
        if (!ok) break;
        float* xb = xchg + (pair * 32 + lane) * 16;
        if (up_warp) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) xb[4 * j + e] = acc[j][e];
        }
        named_bar_sync(1 + pair, 64);  // the up values are in shared memory
        if (!up_warp) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int tok = 8 * j + 2 * tq + (e & 1);
              const int ch = n0 + 16 * w + g + ((e >> 1) << 3);
              if (j < nt && tok < tl.rows && ch < Sg.n) {
                float gv = acc[j][e];
                float uv = xb[4 * j + e];
                if (q8) {
                  gv *= ld_scale(Sg.scale0, Sg.scale_bf16, sc_base + ch);
                  uv *= ld_scale(Sg.scale1, Sg.scale_bf16, sc_base + ch);
                }
                warp_store(p, Sg, tl.row0 + tok, ch, gv / (1.0f + __expf(-gv)) * uv);
              }
            }
          }
        }
        named_bar_sync(1 + pair, 64);  // the gate warp has read the exchange slot
      } else {
        if (!ok) break;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int tok = 8 * j + 2 * tq + (e & 1);
            const int ch = n0 + 16 * w + g + ((e >> 1) << 3);
            if (j < nt && tok < tl.rows && ch < Sg.n) {
              float o = acc[j][e];
              if (q8) o *= ld_scale(Sg.scale0, Sg.scale_bf16, sc_base + ch);
              warp_store(p, Sg, tl.row0 + tok, ch, o);
            }
          }
        }
      }
    }
    if (p.remote_out) __threadfence_system();
  }
}

}  // namespace gemm
}  // namespace moe
