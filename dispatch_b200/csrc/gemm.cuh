// Persistent, warp-specialised grouped GEMM on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA) for the routed expert FFN and the router logits.
//
// One launch walks a flat tile space made of up to two "segments" (e.g. the
// routed experts and the shared expert). A segment is a list of row groups
// (one per expert) over one A matrix, sharing N, K and a stacked (G, N, K)
// weight. Row offsets of the groups live on the device (written by the
// grouping kernel), so the tile list is derived in-kernel and the host never
// synchronises.
//
// Tile = 128 rows x mma_n MMA columns (mma_n <= 256, per segment), K in blocks
// of 64 (one 128-byte swizzle atom of bf16). In a SwiGLU segment the mma_n
// columns are mma_n/2 gate rows and the matching mma_n/2 up rows of the
// weight, and the epilogue writes h = silu(gate) * up; in a plain segment all
// mma_n columns are outputs (bf16/f16, or f32 for the router logits).
//
// Warp roles: warp 0 issues TMA loads, warp 1 owns TMEM and issues
// tcgen05.mma from one thread, then (int8 build only) ten warps dequantise the
// int8 weight rows of each stage to bf16/f16 in shared memory, and the last
// four warps drain the double-buffered TMEM accumulator (lane quarter =
// warp % 4) and store.
// Every mbarrier wait is bounded (ptx.cuh); on expiry the CTA drains its
// in-flight copies and MMAs, frees TMEM and returns with MOE_ERR_TIMEOUT in the
// status word. Group offsets are validated before use (MOE_ERR_BAD_OFFSETS).
#pragma once
#include "ptx.cuh"

namespace moe {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int BN = 256;  // largest MMA N; TMEM columns per accumulator buffer
constexpr int kMaxGroups = 256;
constexpr int kMaxSegs = 2;
constexpr uint32_t A_BYTES = BM * BK * 2;  // 16 KiB
constexpr uint32_t B_BYTES = BN * BK * 2;  // 32 KiB (largest B stage)
constexpr uint32_t Q_BYTES = BN * BK;      // 16 KiB int8 staging
constexpr uint32_t kTmemCols = 2 * BN;     // two accumulators of 256 f32 columns

template <bool kInt8>
struct Config {
  static constexpr int kStages = kInt8 ? 3 : 4;
  static constexpr uint32_t kStageBytes = A_BYTES + B_BYTES + (kInt8 ? Q_BYTES : 0);
  // int8 build: ten dequantiser warps (2-11; 16 warps in all, four per SM
  // sub-partition, the most that 128 registers a thread allow); the epilogue
  // is always the last four warps (one per TMEM lane quarter). Same box, C3
  // T=4096: 6 warps 1.18 ms, 8 warps 0.908 ms, 10 warps 0.896 ms.
  static constexpr int kConvWarps = kInt8 ? 10 : 0;
  static constexpr int kConvThreads = 32 * kConvWarps;
  // 16-byte int8 chunks per dequantiser thread and stage (a 256-row tile)
  static constexpr int kConvItems = kInt8 ? (BN * (BK / 16) + kConvThreads - 1) / kConvThreads : 0;
  static constexpr int kEpiWarp0 = 2 + kConvWarps;
  static constexpr int kThreads = 32 * (kEpiWarp0 + 4);
  // Each SM sub-partition holds a quarter of the 64K registers and the
  // CTA's warps are spread over the four: the busiest one holds
  // ceil(warps / 4) warps.
  static constexpr int kMaxRegs = (16384 / (32 * ((kThreads / 32 + 3) / 4))) & ~7;
};

struct Segment {
  CUtensorMap map_a;   // 2D {K, rows}, box {64, 128}, 128B swizzle
  CUtensorMap map_b0;  // 3D {K, N, G}: plain weight, or gate for SwiGLU
  CUtensorMap map_b1;  // 3D up weight (SwiGLU only)
  const int32_t* offsets;  // G+1 row offsets on the device; nullptr = dense
  const int64_t* gather_rows;  // if set, logical row r of A is row gather_rows[r] of map_a (4-row gathers)
  const void* scale0;      // (G, N) per-channel scales of b0 (int8 only)
  const void* scale1;      // of b1
  void* out;               // (rows, ldo)
  int64_t ldo;
  int groups;
  int dense_rows;  // rows of A (and of out)
  int n;           // output columns
  int k;
  int mma_n;       // MMA N of this segment: multiple of 32 (64 for SwiGLU), <= 256
  int swiglu;
  int b_int8;
  int scale_bf16;
  int out_f32;
  int weight_mod;  // group g multiplies weight g % weight_mod (expert-parallel: (rank, expert) groups)
  int k_splits;    // > 1: K is split into k_splits ranges, each writing an f32 partial slab
  int64_t split_stride;  // elements between the partial slabs of consecutive K ranges
  // Scattered output (expert-parallel return): if out_rows is set, logical row
  // r is stored at row out_rows[r] >> 4 of out_table[out_rows[r] & 15] (a
  // table of out_table_n bases of out_table_rows rows each, possibly peer
  // memory) instead of row r of out.
  const int32_t* out_rows;
  void* const* out_table;
  int out_table_n;
  int64_t out_table_rows;
};

struct Params {
  Segment seg[kMaxSegs];
  int num_segs;
  int in_f16;  // A/B element type: 0 bf16, 1 f16 (also the 16-bit output type)
  int remote_out;  // some segment stores through out_table: fence at system scope before exit
  int32_t* status;
};

struct Ctrl {
  uint64_t full[4];
  uint64_t conv[4];
  uint64_t empty[4];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int seg_tiles[kMaxSegs];
  int off[kMaxSegs][kMaxGroups + 1];
  int mt[kMaxSegs][kMaxGroups + 1];
};

// the control block rounded to 16 bytes, then the epilogue's staging (2 KiB per epilogue warp)
constexpr uint32_t kCtrlBytes = (sizeof(Ctrl) + 15) & ~uint32_t(15);
constexpr uint32_t kEpiStageBytes = 4 * 32 * 64;

__host__ __device__ __forceinline__ int out_cols_per_tile(const Segment& s) {
  return s.swiglu ? s.mma_n / 2 : s.mma_n;
}

struct Tile {
  int seg, group, widx, row0, rows, n_tile, split, kb0, kb1;
};

// Tile t of the launch -> (segment, group, weight slot, rows, n-tile, K
// range); rt = token rows per tile. C is the kernel's control block (its
// seg_tiles, off and mt tables).
template <class C>
__device__ __forceinline__ void decode_tile(const C& c, const Params& p, int t, Tile& tl, int rt = BM) {
  int s = 0;
  while (s + 1 < p.num_segs && t >= c.seg_tiles[s]) {
    t -= c.seg_tiles[s];
    ++s;
  }
  const Segment& S = p.seg[s];
  const int oc = out_cols_per_tile(S);
  const int nt = (S.n + oc - 1) / oc;
  // split-K: the segment's tile list repeats once per K range
  const int per_split = c.mt[s][S.groups] * nt;
  const int split = t / per_split;
  t -= split * per_split;
  const int nkb = (S.k + BK - 1) / BK;
  tl.split = split;
  tl.kb0 = split * nkb / S.k_splits;
  tl.kb1 = (split + 1) * nkb / S.k_splits;
  int lo = 0, hi = S.groups;  // largest g in [0, G) with mt[g] * nt <= t
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (c.mt[s][mid] * nt <= t) lo = mid; else hi = mid;
  }
  const int local = t - c.mt[s][lo] * nt;
  const int mtg = c.mt[s][lo + 1] - c.mt[s][lo];
  const int m_tile = local % mtg;
  tl.seg = s;
  tl.group = lo;
  tl.widx = lo % S.weight_mod;
  tl.n_tile = local / mtg;
  tl.row0 = c.off[s][lo] + m_tile * rt;
  tl.rows = min(rt, c.off[s][lo + 1] - tl.row0);
}

__device__ __forceinline__ float ld_scale(const void* p, int bf16, int64_t i) {
  return bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}

// Eight consecutive per-channel scales from index i (n valid, the rest 1):
// one or two 16-byte loads when aligned, else scalar loads.
__device__ __forceinline__ void ld_scales8(const void* p, int bf16, int64_t i, int n, float (&s)[8]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p) + static_cast<uintptr_t>(i) * (bf16 ? 2u : 4u);
  if (n >= 8 && (a & 15u) == 0) {
    if (bf16) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(a));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[2 * j] = __uint_as_float(w[j] << 16);
        s[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      }
    } else {
      const float4 x = __ldg(reinterpret_cast<const float4*>(a));
      const float4 y = __ldg(reinterpret_cast<const float4*>(a) + 1);
      s[0] = x.x; s[1] = x.y; s[2] = x.z; s[3] = x.w; s[4] = y.x; s[5] = y.y; s[6] = y.z; s[7] = y.w;
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j] = j < n ? ld_scale(p, bf16, i + j) : 1.f;
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int f16) {
  if (f16) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Stores 32 consecutive f32 values of one output row as bf16/f16/f32; only
// the first ncols are written.
__device__ __forceinline__ void store_row32(void* out, int64_t elem_off, const float (&v)[32], int ncols, int f16,
                                            int f32, bool vec_ok) {
  if (f32) {
    float* o = reinterpret_cast<float*>(out) + elem_off;
    if (ncols == 32 && vec_ok) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(o)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncols) o[j] = v[j];
    }
    return;
  }
  uint16_t* o = reinterpret_cast<uint16_t*>(out) + elem_off;
  if (ncols == 32 && vec_ok) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      reinterpret_cast<uint4*>(o)[q] =
          make_uint4(pack2(v[q * 8 + 0], v[q * 8 + 1], f16), pack2(v[q * 8 + 2], v[q * 8 + 3], f16),
                     pack2(v[q * 8 + 4], v[q * 8 + 5], f16), pack2(v[q * 8 + 6], v[q * 8 + 7], f16));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < ncols) {
        const uint32_t b = pack2(v[j], 0.f, f16);
        o[j] = static_cast<uint16_t>(b & 0xFFFFu);
      }
    }
  }
}

// Staged 16-bit store of a warp's 32 x 32 block: lane i holds 32 values of
// row i; the block goes through 2 KiB of shared memory (16-byte slots XOR-
// swizzled so both passes are bank-conflict free) and leaves as 8 rows x 64
// contiguous bytes per store instruction instead of 32 rows x 16 bytes -- a
// quarter of the write requests, which matters most when the rows live in a
// peer GPU's memory. rowp[s] is the destination row (element col0) of row
// s * 8 + lane / 4, or null to skip it.
__device__ __forceinline__ void store_block32_staged(uint4* stage, const float (&v)[32], int f16, int lane,
                                                     uint16_t* const (&rowp)[4], int col0) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 pk = make_uint4(pack2(v[q * 8 + 0], v[q * 8 + 1], f16), pack2(v[q * 8 + 2], v[q * 8 + 3], f16),
                                pack2(v[q * 8 + 4], v[q * 8 + 5], f16), pack2(v[q * 8 + 6], v[q * 8 + 7], f16));
    stage[lane * 4 + (q ^ ((lane >> 1) & 3))] = pk;
  }
  __syncwarp();
  const int c = lane & 3;
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const int rr = s * 8 + (lane >> 2);
    const uint4 val = stage[rr * 4 + (c ^ ((rr >> 1) & 3))];
    if (rowp[s]) *reinterpret_cast<uint4*>(rowp[s] + col0 + c * 8) = val;
  }
  __syncwarp();
}

// Exact int8 -> 16-bit float for 16 packed bytes. Each signed byte b becomes
// the f32 2^23 + (b + 128) by byte placement, minus 2^23 + 128 -- two values
// per packed f32x2 subtraction (sm_100). The results are integers in
// [-128, 127], exact in bf16 and f16: bf16 keeps the f32's high half (a byte
// permute), f16 converts.
__device__ __forceinline__ uint64_t sub_magic_f32x2(uint32_t a, uint32_t b) {
  const uint64_t x = (static_cast<uint64_t>(b) << 32) | a;
  constexpr uint64_t kMagic = 0x4B0000804B000080ull;  // two f32 2^23 + 128
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(x), "l"(kMagic));
  return d;
}

__device__ __forceinline__ uint32_t pack_exact2(uint64_t ab, int f16) {
  const uint32_t a = static_cast<uint32_t>(ab), b = static_cast<uint32_t>(ab >> 32);
  if (f16) return pack2(__uint_as_float(a), __uint_as_float(b), 1);
  return __byte_perm(a, b, 0x7632);
}

__device__ __forceinline__ void dequant16(uint4 q, int f16, uint4& lo, uint4& hi) {
  const uint32_t w[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
  uint32_t out[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t bits[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) bits[b] = __byte_perm(w[i], 0x4B000000u, 0x7540u | static_cast<uint32_t>(b));
    out[2 * i] = pack_exact2(sub_magic_f32x2(bits[0], bits[1]), f16);
    out[2 * i + 1] = pack_exact2(sub_magic_f32x2(bits[2], bits[3]), f16);
  }
  lo = make_uint4(out[0], out[1], out[2], out[3]);
  hi = make_uint4(out[4], out[5], out[6], out[7]);
}

// Drains one 128-row accumulator into the segment's output: lane i of the
// calling warp holds tile row r (a row of the tile is valid if r < tl.rows),
// tb its TMEM address (lane quarter and accumulator columns included); 16-bit
// rows go out through the warp's 2 KiB staging buffer. Shared by the tiled
// kernels.
template <bool kInt8>
__device__ __forceinline__ void epilogue_rows(const Params& p, const Segment& Sg, const Tile& tl, uint32_t tb,
                                              int r, int lane, uint4* estage) {
  bool valid = r < tl.rows;
  void* obase = Sg.out;
  int64_t orow = tl.row0 + r;
  if (Sg.out_rows && valid) {
    const int code = Sg.out_rows[orow];
    const int dst = code & 15;
    orow = code >> 4;
    if (code < 0 || dst >= Sg.out_table_n || orow >= Sg.out_table_rows) {
      if (p.status) atomicCAS(p.status, 0, MOE_ERR_BAD_OFFSETS);
      valid = false;
    } else {
      obase = Sg.out_table[dst];
    }
  }
  const int64_t row_off = orow * Sg.ldo + tl.split * Sg.split_stride;
  const bool vec_ok = (Sg.ldo % 8) == 0;
  const int64_t sc_base = static_cast<int64_t>(tl.widx) * Sg.n;
  const int oc = out_cols_per_tile(Sg);
  const int n0 = tl.n_tile * oc;
  // whole 32-column chunks of 16-bit rows go through the staged store
  const bool staged = !Sg.out_f32 && vec_ok && (Sg.n % 32) == 0;
  uint16_t* rowp[4];
  {
    uint16_t* mine = valid ? reinterpret_cast<uint16_t*>(obase) + row_off : nullptr;
#pragma unroll
    for (int s2 = 0; s2 < 4; ++s2)
      rowp[s2] = reinterpret_cast<uint16_t*>(
          __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(mine), s2 * 8 + (lane >> 2)));
  }
  if (Sg.swiglu) {
#pragma unroll 1
    for (int ch = 0; ch < oc / 32; ++ch) {
      uint32_t gv[32], uv[32];
      tmem_ld_32x32b_x32(tb + ch * 32, gv);
      tmem_ld_32x32b_x32(tb + oc + ch * 32, uv);
      tmem_ld_wait();
      const int col0 = n0 + ch * 32;
      if (staged ? col0 < Sg.n : (valid && col0 < Sg.n)) {
        const int nc = min(32, Sg.n - col0);
        float h[32];
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float gs[8], us[8];
          if (kInt8 && Sg.b_int8) {
            ld_scales8(Sg.scale0, Sg.scale_bf16, sc_base + col0 + 8 * q8, nc - 8 * q8, gs);
            ld_scales8(Sg.scale1, Sg.scale_bf16, sc_base + col0 + 8 * q8, nc - 8 * q8, us);
          }
#pragma unroll
          for (int j8 = 0; j8 < 8; ++j8) {
            const int j = 8 * q8 + j8;
            float g = __uint_as_float(gv[j]);
            float u = __uint_as_float(uv[j]);
            if (kInt8 && Sg.b_int8 && j < nc) {
              g *= gs[j8];
              u *= us[j8];
            }
            h[j] = g / (1.0f + __expf(-g)) * u;
          }
        }
        if (staged)
          store_block32_staged(estage, h, p.in_f16, lane, rowp, col0);
        else
          store_row32(obase, row_off + col0, h, nc, p.in_f16, 0, vec_ok);
      }
    }
  } else {
#pragma unroll 1
    for (int ch = 0; ch < oc / 32; ++ch) {
      uint32_t v[32];
      tmem_ld_32x32b_x32(tb + ch * 32, v);
      tmem_ld_wait();
      const int col0 = n0 + ch * 32;
      if (staged ? col0 < Sg.n : (valid && col0 < Sg.n)) {
        const int nc = min(32, Sg.n - col0);
        float o[32];
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float ss[8];
          if (kInt8 && Sg.b_int8) ld_scales8(Sg.scale0, Sg.scale_bf16, sc_base + col0 + 8 * q8, nc - 8 * q8, ss);
#pragma unroll
          for (int j8 = 0; j8 < 8; ++j8) {
            const int j = 8 * q8 + j8;
            o[j] = __uint_as_float(v[j]);
            if (kInt8 && Sg.b_int8 && j < nc) o[j] *= ss[j8];
          }
        }
        if (staged)
          store_block32_staged(estage, o, p.in_f16, lane, rowp, col0);
        else
          store_row32(obase, row_off + col0, o, nc, p.in_f16, Sg.out_f32, Sg.out_f32 ? (Sg.ldo % 4) == 0 : vec_ok);
      }
    }
  }
}

template <bool kInt8>
__global__ void __launch_bounds__(Config<kInt8>::kThreads)
    __maxnreg__(Config<kInt8>::kMaxRegs < 168 ? Config<kInt8>::kMaxRegs : 168) grouped_gemm_kernel(const __grid_constant__ Params p) {
  using Cfg = Config<kInt8>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;
  uint8_t* sB = sA + S * A_BYTES;
  uint8_t* sQ = sB + S * B_BYTES;
  Ctrl& c = *reinterpret_cast<Ctrl*>(sB + S * B_BYTES + (kInt8 ? S * Q_BYTES : 0));
  volatile int* abort_flag = &c.abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  // ---- setup: barriers, TMEM and descriptor prefetch (no global memory),
  // then -- once the previous kernel in the stream is complete -- group
  // offsets and the per-group m-tile prefix in shared memory
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
    tmem_alloc(&c.tmem_base, kTmemCols);
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
    int running = 0;
    // Offsets come from another kernel: refuse (and report) a segment whose
    // offsets are not monotone inside [0, rows] instead of storing out of range.
    bool bad = lane == 0 && (c.off[s][0] < 0 || c.off[s][Sg.groups] > Sg.dense_rows);
    if (lane == 0) c.mt[s][0] = 0;
    for (int g0 = 0; g0 < Sg.groups; g0 += 32) {
      const int g = g0 + lane;
      int v = 0;
      if (g < Sg.groups) {
        const int rows = c.off[s][g + 1] - c.off[s][g];
        bad |= rows < 0;
        v = rows > 0 ? (rows + BM - 1) / BM : 0;
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
      c.seg_tiles[s] = bad ? 0 : running * ((Sg.n + oc - 1) / oc) * Sg.k_splits;
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
    // Lane 0 waits, arms the stage barrier and loads B (and a tiled A); in a
    // gather segment every lane also loads 4 of the tile's 128 A rows.
    {
      uint32_t stage = 0, phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        Tile tl;
        decode_tile(c, p, t, tl);
        const Segment& Sg = p.seg[tl.seg];
        const int n0 = tl.n_tile * out_cols_per_tile(Sg);
        const bool q8 = kInt8 && Sg.b_int8;
        const uint32_t row_bytes = q8 ? BK : BK * 2;  // bytes of one weight row in a stage
        const uint32_t b_bytes = static_cast<uint32_t>(Sg.mma_n) * row_bytes;
        const uint32_t half = static_cast<uint32_t>(Sg.mma_n / 2) * row_bytes;
        const bool gather = Sg.gather_rows != nullptr;
        int32_t gr[4] = {0, 0, 0, 0};
        if (gather) {
          // rows past the group's end read source row 0; their results are not stored
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int r = 4 * lane + j;
            gr[j] = r < tl.rows ? static_cast<int32_t>(Sg.gather_rows[tl.row0 + r]) : 0;
          }
        }
        for (int kb = tl.kb0; kb < tl.kb1; ++kb) {
          int waited = 1;
          if (lane == 0) waited = wait_parity_bounded(&c.empty[stage], phase ^ 1u, abort_flag, p.status) ? 1 : 0;
          if (!__shfl_sync(0xffffffffu, waited, 0)) { ok = false; break; }
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = q8 ? sQ + stage * Q_BYTES : sB + stage * B_BYTES;
          if (lane == 0) {
            mbar_arrive_expect_tx(&c.full[stage], A_BYTES + b_bytes);
            if (!gather) tma_load_2d(a_dst, &Sg.map_a, &c.full[stage], kb * BK, tl.row0);
            tma_load_3d(b_dst, &Sg.map_b0, &c.full[stage], kb * BK, n0, tl.widx);
            if (Sg.swiglu) tma_load_3d(b_dst + half, &Sg.map_b1, &c.full[stage], kb * BK, n0, tl.widx);
          }
          if (gather) {
            __syncwarp();
            tma_gather4(a_dst + lane * 4 * (BK * 2), &Sg.map_a, &c.full[stage], kb * BK, gr[0], gr[1], gr[2], gr[3]);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok && lane == 0) {
        // Let every copy this thread started land before the CTA exits.
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
      // conv[s] completes a phase only when an int8 tile uses stage s, so its
      // parity is tracked per stage, apart from the full/empty phase.
      uint32_t conv_par = 0;
      bool ok = true, issued = false;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        Tile tl;
        decode_tile(c, p, t, tl);
        const Segment& Sg = p.seg[tl.seg];
        const uint32_t idesc = idesc_f16(BM, Sg.mma_n, p.in_f16 != 0);
        if (!wait_parity_bounded(&c.tempty[acc], acc_phase ^ 1u, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem_base + acc * BN;
        for (int kb = tl.kb0; kb < tl.kb1; ++kb) {
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
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            mma_f16_ss(d, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), idesc,
                       (kb != tl.kb0 || kk != 0) ? 1u : 0u);
          }
          issued = true;
          mma_commit(&c.empty[stage]);
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        mma_commit(&c.tfull[acc]);
        acc ^= 1u;
        if (acc == 0) acc_phase ^= 1u;
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
    // ------------------------------------------------------------ int8 -> bf16/f16
    if constexpr (kInt8) {
      const int ct = tid - 64;
      uint32_t stage = 0, phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
        Tile tl;
        decode_tile(c, p, t, tl);
        const Segment& Sg = p.seg[tl.seg];
        const int items = Sg.mma_n * 4;  // 16-byte int8 chunks in one stage
        for (int kb = tl.kb0; kb < tl.kb1; ++kb) {
          if (Sg.b_int8) {
            if (!wait_parity_bounded(&c.full[stage], phase, abort_flag, p.status)) { ok = false; break; }
            const uint8_t* q = sQ + stage * Q_BYTES;
            uint8_t* b = sB + stage * B_BYTES;
            // all of this thread's chunk loads first, then dequantise and store
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
                const int r = item >> 2, cc = item & 3;
                uint4 lo, hi;
                dequant16(v[j], p.in_f16, lo, hi);
                uint8_t* row = b + r * 128;
                *reinterpret_cast<uint4*>(row + (((2 * cc) ^ (r & 7)) << 4)) = lo;
                *reinterpret_cast<uint4*>(row + (((2 * cc + 1) ^ (r & 7)) << 4)) = hi;
              }
            }
            fence_proxy_async_smem();
            mbar_arrive(&c.conv[stage]);
          }
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int r = q * 32 + lane;
    uint4* estage = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(&c) + kCtrlBytes) + q * 128;
    uint32_t acc = 0, acc_phase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      Tile tl;
      decode_tile(c, p, t, tl);
      const Segment& Sg = p.seg[tl.seg];
      if (!wait_parity_bounded(&c.tfull[acc], acc_phase, abort_flag, p.status)) break;
      tc_fence_after();
      const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      epilogue_rows<kInt8>(p, Sg, tl, tb, r, lane, estage);
      tc_fence_before();
      mbar_arrive(&c.tempty[acc]);
      acc ^= 1u;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (p.remote_out) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <bool kInt8>
constexpr size_t smem_bytes() {
  return 1024 + Config<kInt8>::kStages * Config<kInt8>::kStageBytes + kCtrlBytes + kEpiStageBytes;
}

}  // namespace gemm
}  // namespace moe
