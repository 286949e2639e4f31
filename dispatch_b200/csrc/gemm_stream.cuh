// Weight-streaming grouped GEMM for small row counts (decode batches and the
// small per-expert groups of expert-parallel ranks).
//
// The prefill kernel (gemm.cuh) puts 128 token rows on the MMA's M side and
// the weight rows on N; with one or a few rows per expert most of its A tile
// is rows of other experts and its CTAs hold three 48 KB stages, so a decode
// step streams weights from few tiles with few bytes in flight. This kernel
// swaps the operands: the MMA's M side is 128 WEIGHT rows (output channels)
// and its N side is a tile of nt token rows (nt = 32 ... 256), so with a
// narrow row tile a stage is 16 KB of weights + nt x 128 bytes of rows and up
// to 12 stages (about 200 KB of weights) are in flight per SM. A tile's MMA
// width is its row count rounded up to 16 (at most nt), so the last row tile
// of a group computes no more than 15 rows it does not keep.
//
// D[ch, r] = sum_k W[ch, k] X[r, k] is the transpose of the prefill kernel's
// D[r, ch]: the same products summed over the same 64-wide k-blocks in the
// same order (four K=16 MMAs each), and the tensor cores give the same bits
// in either orientation (checked on B200: f32 and bf16 outputs of both
// orientations are equal bit for bit), so a row's result does not depend on
// which of the two kernels computed it. That keeps the expert-parallel output
// byte-identical to the 1-GPU output whichever kernel each launch picks.
//
// Tile = (segment, group, channel block, row block). A SwiGLU segment's
// channel block is 64 gate rows + the matching 64 up rows of the weight
// (accumulator lanes 0-63 gate, 64-127 up; the epilogue pairs lane l with
// lane l + 64 through shared memory); a plain segment's is 128 weight rows.
// Row blocks of one channel block are adjacent in the tile order, so a group
// with more than nt rows re-reads that weight block from L2, not HBM.
//
// Warp roles as in the prefill kernel: warp 0 TMA producer, warp 1 TMEM owner
// and MMA issuer, then the int8 dequantisers (int8 build), then four epilogue
// warps (TMEM lane quarter = warp % 4). Every wait is bounded; the epilogue
// warps that exchange gate/up values agree on every wait's outcome (a barrier
// with an AND reduction) before they meet at the exchange barriers, so a
// timeout in one of them cannot leave the other waiting.
#pragma once
#include "gemm.cuh"

namespace moe {
namespace gemm {

constexpr int SM_ROWS = 128;        // weight rows per chain block (MMA M)
constexpr int kStreamMaxStages = 12;
constexpr int kStreamMaxRowTile = 256;  // token rows per tile (MMA N) at most
constexpr int kStreamMaxChains = 2;
constexpr uint32_t SA_BYTES = SM_ROWS * BK * 2;  // 16 KiB of weights (16-bit) per chain block and stage
constexpr uint32_t SQ_BYTES = SM_ROWS * BK;      // 8 KiB int8 staging per chain block and stage

template <bool kInt8>
struct StreamConfig {
  static constexpr int kConvWarps = kInt8 ? 10 : 0;
  static constexpr int kConvThreads = 32 * kConvWarps;
  static constexpr int kConvItems =
      kInt8 ? (kStreamMaxChains * SM_ROWS * (BK / 16) + kConvThreads - 1) / kConvThreads : 0;
  static constexpr int kEpiWarp0 = 2 + kConvWarps;
  static constexpr int kThreads = 32 * (kEpiWarp0 + 4);
  static constexpr int kMaxRegs = (16384 / (32 * ((kThreads / 32 + 3) / 4))) & ~7;
};

struct StreamCtrl {
  uint64_t full[kStreamMaxStages];
  uint64_t conv[kStreamMaxStages];
  uint64_t empty[kStreamMaxStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int seg_tiles[kMaxSegs];
  int off[kMaxSegs][kMaxGroups + 1];
  int mt[kMaxSegs][kMaxGroups + 1];
};

// Shared memory: control block, epilogue exchange (8 KiB), then 1 KiB-aligned
// stage rings: weights (chains x SA_BYTES each), rows (nt_max x 128 B each)
// and, for int8, the raw weight staging (chains x SQ_BYTES each).
constexpr uint32_t kStreamCtrlBytes = (sizeof(StreamCtrl) + 15) & ~uint32_t(15);
constexpr uint32_t kStreamXchgBytes = 2 * 32 * 32 * 4;

__host__ __device__ constexpr uint32_t stream_fixed_bytes() {
  return ((kStreamCtrlBytes + kStreamXchgBytes + 1023) & ~uint32_t(1023)) + 1024;  // + base alignment slack
}
__host__ __device__ constexpr uint32_t stream_stage_bytes(bool int8, int nt_max, int chains) {
  return static_cast<uint32_t>(chains) * (SA_BYTES + (int8 ? SQ_BYTES : 0u)) + static_cast<uint32_t>(nt_max) * 128u;
}

// One launch: the segments (Segment::mma_n = 128 weight rows per chain block,
// one K range, 16-bit outputs, no gathered rows), each segment's row tile, and
// the chain count: a tile holds `chains` weight blocks that share the tile's
// rows and accumulate into separate TMEM accumulators, their MMAs issued
// interleaved. One accumulator's MMAs depend on each other and the tensor
// core runs such a chain at roughly a third of its rate (measured on B200,
// M=128 K=16: ~330 cycles per dependent MMA whatever N, against ~210 per MMA
// for two interleaved chains), so two chains keep the tensor pipe busier.
struct StreamParams {
  Params p;
  int row_tile[kMaxSegs];  // nt of each segment (multiple of 32, <= kStreamMaxRowTile)
  int nt_max;              // largest row tile: the row stage and the accumulator width
  int stages;              // stage ring depth (<= kStreamMaxStages)
  int chains;              // weight blocks per tile (1 or 2)
  int acc_slots;           // accumulator buffers (1 or 2): chains x nt_max x acc_slots <= 512 columns
};

struct StreamTile {
  int seg, group, widx, cpair, nch, row0, rows;
};

__device__ __forceinline__ void decode_stream_tile(const StreamCtrl& c, const StreamParams& sp, int t, StreamTile& tl) {
  const Params& p = sp.p;
  int s = 0;
  while (s + 1 < p.num_segs && t >= c.seg_tiles[s]) {
    t -= c.seg_tiles[s];
    ++s;
  }
  const Segment& S = p.seg[s];
  const int nt = sp.row_tile[s];
  const int oc = out_cols_per_tile(S);
  const int ct = (S.n + oc - 1) / oc;                // channel blocks
  const int cpt = (ct + sp.chains - 1) / sp.chains;  // tiles (chain groups) per row block
  int lo = 0, hi = S.groups;  // largest g with mt[g] * cpt <= t
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (c.mt[s][mid] * cpt <= t) lo = mid; else hi = mid;
  }
  const int local = t - c.mt[s][lo] * cpt;
  const int rtg = c.mt[s][lo + 1] - c.mt[s][lo];
  const int r_tile = local % rtg;  // row blocks of one channel group are adjacent
  tl.seg = s;
  tl.group = lo;
  tl.widx = lo % S.weight_mod;
  tl.cpair = local / rtg;
  tl.nch = min(sp.chains, ct - tl.cpair * sp.chains);
  tl.row0 = c.off[s][lo] + r_tile * nt;
  tl.rows = min(nt, c.off[s][lo + 1] - tl.row0);
}

__device__ __forceinline__ uint16_t to16(float v, int f16) {
  return static_cast<uint16_t>(pack2(v, 0.f, f16) & 0xFFFFu);
}

template <bool kInt8>
__global__ void __launch_bounds__(StreamConfig<kInt8>::kThreads)
    __maxnreg__(StreamConfig<kInt8>::kMaxRegs < 168 ? StreamConfig<kInt8>::kMaxRegs : 168)
        grouped_gemm_stream_kernel(const __grid_constant__ StreamParams sp) {
  using Cfg = StreamConfig<kInt8>;
  const Params& p = sp.p;
  const int S = sp.stages;
  const int nt_max = sp.nt_max;
  const int chains = sp.chains;
  const int slots = sp.acc_slots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  StreamCtrl& c = *reinterpret_cast<StreamCtrl*>(base);
  float* xchg = reinterpret_cast<float*>(base + kStreamCtrlBytes);
  uint8_t* sA = base + ((kStreamCtrlBytes + kStreamXchgBytes + 1023) & ~uint32_t(1023));
  const uint32_t a_stage = static_cast<uint32_t>(chains) * SA_BYTES;
  const uint32_t b_stage = static_cast<uint32_t>(nt_max) * 128u;
  const uint32_t q_stage = static_cast<uint32_t>(chains) * SQ_BYTES;
  uint8_t* sB = sA + S * a_stage;
  uint8_t* sQ = sB + S * b_stage;
  volatile int* abort_flag = &c.abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // accumulators: slot a, chain ch at column (a * chains + ch) * nt_max; the
  // allocation is a power of two >= 32 columns
  const uint32_t acc_cols = static_cast<uint32_t>(slots * chains * nt_max);
  uint32_t tmem_cols = 32;
  while (tmem_cols < acc_cols) tmem_cols <<= 1;

  pdl_trigger();
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.conv[i], kInt8 ? Cfg::kConvThreads : 1);
      mbar_init(&c.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&c.tfull[i], 1);
      mbar_init(&c.tempty[i], 4 * 32);
    }
    mbar_init(&c.drain, 1);
    c.abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&c.tmem_base, tmem_cols);
    tmem_relinquish();
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
    for (int g = tid; g <= Sg.groups; g += Cfg::kThreads)
      c.off[s][g] = Sg.offsets ? Sg.offsets[g] : (g == 0 ? 0 : Sg.dense_rows);
  }
  __syncthreads();
  if (warp < p.num_segs) {
    const int s = warp;
    const Segment& Sg = p.seg[s];
    const int nt = sp.row_tile[s];
    int running = 0;
    bool bad = lane == 0 && (c.off[s][0] < 0 || c.off[s][Sg.groups] > Sg.dense_rows);
    if (lane == 0) c.mt[s][0] = 0;
    for (int g0 = 0; g0 < Sg.groups; g0 += 32) {
      const int g = g0 + lane;
      int v = 0;
      if (g < Sg.groups) {
        const int rows = c.off[s][g + 1] - c.off[s][g];
        bad |= rows < 0;
        v = rows > 0 ? (rows + nt - 1) / nt : 0;
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
      const int ct = (Sg.n + oc - 1) / oc;
      c.seg_tiles[s] = bad ? 0 : running * ((ct + chains - 1) / chains);
      if (bad && p.status) atomicCAS(p.status, 0, MOE_ERR_BAD_OFFSETS);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = c.tmem_base;
  int total = 0;
  for (int s = 0; s < p.num_segs; ++s) total += c.seg_tiles[s];

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        StreamTile tl;
        decode_stream_tile(c, sp, t, tl);
        const Segment& Sg = p.seg[tl.seg];
        const int oc = out_cols_per_tile(Sg);
        const bool q8 = kInt8 && Sg.b_int8;
        const uint32_t row_bytes = q8 ? BK : BK * 2;  // bytes of one weight row in a stage
        const uint32_t part = SM_ROWS * row_bytes;     // one chain block of weights
        const uint32_t rows_bytes = static_cast<uint32_t>(sp.row_tile[tl.seg]) * 128u;
        const int nkb = (Sg.k + BK - 1) / BK;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!wait_parity_bounded(&c.empty[stage], phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
          uint8_t* w_dst = q8 ? sQ + stage * q_stage : sA + stage * a_stage;
          mbar_arrive_expect_tx(&c.full[stage], tl.nch * part + rows_bytes);
          for (int ch = 0; ch < tl.nch; ++ch) {
            const int n0 = (tl.cpair * chains + ch) * oc;
            uint8_t* dst = w_dst + ch * part;
            if (Sg.swiglu) {
              tma_load_3d(dst, &Sg.map_b0, &c.full[stage], kb * BK, n0, tl.widx);
              tma_load_3d(dst + (SM_ROWS / 2) * row_bytes, &Sg.map_b1, &c.full[stage], kb * BK, n0, tl.widx);
            } else {
              tma_load_3d(dst, &Sg.map_b0, &c.full[stage], kb * BK, n0, tl.widx);
            }
          }
          tma_load_2d(sB + stage * b_stage, &Sg.map_a, &c.full[stage], kb * BK, tl.row0);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == static_cast<uint32_t>(S)) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        for (int i = 0; i < S; ++i) {
          if (!(issued_mask & (1u << i))) continue;
          const uint32_t par = (issued_parity >> i) & 1u;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&c.full[i], par) && globaltimer_ns() - t0 < 100000000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
      uint32_t conv_par = 0;
      bool ok = true, issued = false;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        StreamTile tl;
        decode_stream_tile(c, sp, t, tl);
        const Segment& Sg = p.seg[tl.seg];
        // MMA width: the tile's rows rounded up to 16 (N of an M=128 MMA is a multiple of 16)
        const int n_mma = min(sp.row_tile[tl.seg], (tl.rows + 15) & ~15);
        const uint32_t idesc = idesc_f16(SM_ROWS, n_mma, p.in_f16 != 0);
        if (!wait_parity_bounded(&c.tempty[acc], acc_phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d0 = tmem_base + acc * static_cast<uint32_t>(chains * nt_max);
        const int nkb = (Sg.k + BK - 1) / BK;
        for (int kb = 0; kb < nkb; ++kb) {
          if (kInt8 && Sg.b_int8) {
            if (!wait_parity_bounded(&c.conv[stage], (conv_par >> stage) & 1u, abort_flag, p.status)) {
              ok = false;
              break;
            }
            conv_par ^= 1u << stage;
          } else if (!wait_parity_bounded(&c.full[stage], phase, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * a_stage);
          const uint32_t b0 = smem_u32(sB + stage * b_stage);
          // the chains' MMAs interleaved: one chain's next MMA waits on its
          // previous one, the other chain's MMA fills that gap
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            for (int ch = 0; ch < tl.nch; ++ch)
              mma_f16_ss(d0 + ch * nt_max, sw128_kmajor_desc(a0 + ch * SA_BYTES + kk * 32),
                         sw128_kmajor_desc(b0 + kk * 32), idesc, (kb != 0 || kk != 0) ? 1u : 0u);
          }
          issued = true;
          mma_commit(&c.empty[stage]);
          if (++stage == static_cast<uint32_t>(S)) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit(&c.tfull[acc]);
        if (++acc == static_cast<uint32_t>(slots)) { acc = 0; acc_phase ^= 1u; }
      }
      if (!ok && issued) {
        mma_commit(&c.drain);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&c.drain, 0) && globaltimer_ns() - t0 < 100000000ull) {
        }
      }
    }
    __syncwarp();
  } else if (warp < Cfg::kEpiWarp0) {
    // ------------------------------------------------------------ int8 -> bf16/f16 (weight stage)
    if constexpr (kInt8) {
      const int ct = tid - 64;
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        StreamTile tl;
        decode_stream_tile(c, sp, t, tl);
        const Segment& Sg = p.seg[tl.seg];
        const int items = tl.nch * SM_ROWS * 4;  // 16-byte int8 chunks in one stage
        const int nkb = (Sg.k + BK - 1) / BK;
        for (int kb = 0; kb < nkb; ++kb) {
          if (Sg.b_int8) {
            if (!wait_parity_bounded(&c.full[stage], phase, abort_flag, p.status)) { ok = false; break; }
            const uint8_t* q = sQ + stage * q_stage;
            uint8_t* a = sA + stage * a_stage;
            constexpr int NI = Cfg::kConvItems;
            uint4 v[NI];
#pragma unroll
            for (int j = 0; j < NI; ++j) {
              const int item = ct + j * Cfg::kConvThreads;
              if (item < items) v[j] = *reinterpret_cast<const uint4*>(q + (item >> 2) * 64 + (item & 3) * 16);
            }
#pragma unroll
            for (int j = 0; j < NI; ++j) {
              const int item = ct + j * Cfg::kConvThreads;
              if (item < items) {
                const int r = item >> 2, cc = item & 3;  // r: row over the chain blocks (128 per block)
                uint4 lo, hi;
                dequant16(v[j], p.in_f16, lo, hi);
                uint8_t* row = a + (r >> 7) * SA_BYTES + (r & 127) * 128;
                *reinterpret_cast<uint4*>(row + (((2 * cc) ^ (r & 7)) << 4)) = lo;
                *reinterpret_cast<uint4*>(row + (((2 * cc + 1) ^ (r & 7)) << 4)) = hi;
              }
            }
            fence_proxy_async_smem();
            mbar_arrive(&c.conv[stage]);
          }
          if (++stage == static_cast<uint32_t>(S)) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Lane quarter q holds weight rows 32q..32q+31 of each chain block;
    // accumulator column j is token row row0 + j. SwiGLU: quarters 0/1 are
    // gate channels, 2/3 the matching up channels; up warp q+2 hands its
    // values to gate warp q through xchg (named barrier 1 + q, 64 threads).
    const int q = warp & 3;
    const int pair = q & 1;
    const bool gate_warp = q < 2;
    float* xb = xchg + pair * (32 * 32);
    uint32_t acc = 0, acc_phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      StreamTile tl;
      decode_stream_tile(c, sp, t, tl);
      const Segment& Sg = p.seg[tl.seg];
      bool ok = wait_parity_bounded(&c.tfull[acc], acc_phase, abort_flag, p.status);
      // both warps of a gate/up pair leave together or not at all
      ok = named_bar_and(1 + pair, 64, ok);
      if (!ok) break;
      tc_fence_after();
      const int oc = out_cols_per_tile(Sg);
      const int64_t sc_base = static_cast<int64_t>(tl.widx) * Sg.n;
#pragma unroll 1
      for (int chn = 0; chn < tl.nch; ++chn) {
        const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                            (acc * chains + chn) * static_cast<uint32_t>(nt_max);
        const int n0 = (tl.cpair * chains + chn) * oc;
        if (Sg.swiglu) {
          const int ch = n0 + pair * 32 + lane;  // this thread's output channel
          float gs = 1.f, us = 1.f;
          if (kInt8 && Sg.b_int8 && gate_warp && ch < Sg.n) {
            gs = ld_scale(Sg.scale0, Sg.scale_bf16, sc_base + ch);
            us = ld_scale(Sg.scale1, Sg.scale_bf16, sc_base + ch);
          }
#pragma unroll 1
          for (int c0 = 0; c0 < tl.rows; c0 += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tb + c0, v);
            tmem_ld_wait();
            named_bar_sync(1 + pair, 64);  // the gate warp has read the previous chunk
            if (!gate_warp) {
#pragma unroll
              for (int j = 0; j < 32; ++j) xb[j * 32 + lane] = __uint_as_float(v[j]);
            }
            named_bar_sync(1 + pair, 64);  // this chunk's up values are in xb
            if (gate_warp && ch < Sg.n) {
              uint16_t* out = reinterpret_cast<uint16_t*>(Sg.out);
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (c0 + j < tl.rows) {
                  const float g = __uint_as_float(v[j]) * gs;
                  const float u = xb[j * 32 + lane] * us;
                  out[static_cast<int64_t>(tl.row0 + c0 + j) * Sg.ldo + ch] =
                      to16(g / (1.0f + __expf(-g)) * u, p.in_f16);
                }
              }
            }
          }
        } else {
          const int ch = n0 + q * 32 + lane;
          float ss = 1.f;
          if (kInt8 && Sg.b_int8 && ch < Sg.n) ss = ld_scale(Sg.scale0, Sg.scale_bf16, sc_base + ch);
#pragma unroll 1
          for (int c0 = 0; c0 < tl.rows; c0 += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tb + c0, v);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (c0 + j >= tl.rows) continue;
              const int64_t r = tl.row0 + c0 + j;
              uint16_t* obase = reinterpret_cast<uint16_t*>(Sg.out);
              int64_t orow = r;
              if (Sg.out_rows) {
                const int code = Sg.out_rows[r];
                const int dst = code & 15;
                orow = code >> 4;
                if (code < 0 || dst >= Sg.out_table_n || orow >= Sg.out_table_rows) {
                  if (p.status && lane == 0) atomicCAS(p.status, 0, MOE_ERR_BAD_OFFSETS);
                  continue;
                }
                obase = reinterpret_cast<uint16_t*>(Sg.out_table[dst]);
              }
              if (ch < Sg.n) obase[orow * Sg.ldo + ch] = to16(__uint_as_float(v[j]) * ss, p.in_f16);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&c.tempty[acc]);
      if (++acc == static_cast<uint32_t>(slots)) { acc = 0; acc_phase ^= 1u; }
    }
    if (p.remote_out) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

}  // namespace gemm
}  // namespace moe
