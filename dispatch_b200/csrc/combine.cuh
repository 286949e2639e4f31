// Weighted combine (unpermute): one warp per token sums its k expert rows in
// slot order in f32, adds the shared expert's row, rounds once. 16-byte loads.
// Also the per-channel int8 quantiser (one warp per weight row).
#pragma once
#include "ptx.cuh"

namespace moe {
namespace combine {

constexpr int kThreads = 256;
constexpr int kMaxK = 32;

struct Params {
  const void* y;
  const void* y_shared;
  const int32_t* pos;
  const float* w;
  void* out;
  int32_t* status;
  int64_t T, H;
  int k, y_dtype, out_dtype;
};

__device__ __forceinline__ void load8(const void* base, int dt, int64_t off, float (&v)[8]) {
  if (dt == MOE_DT_F32) {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + off);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + off + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + off);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (dt == MOE_DT_BF16) {
        const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
        v[2 * i] = __low2float(h);
        v[2 * i + 1] = __high2float(h);
      } else {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        v[2 * i] = __low2float(h);
        v[2 * i + 1] = __high2float(h);
      }
    }
  }
}

__device__ __forceinline__ void store8(void* base, int dt, int64_t off, const float (&v)[8]) {
  if (dt == MOE_DT_F32) {
    float* o = reinterpret_cast<float*>(base) + off;
    *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(o + 4) = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (dt == MOE_DT_BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(base) + off) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// 8 consecutive values of a 16-bit row, raw (16 bytes).
__device__ __forceinline__ uint4 load_raw16(const void* base, int64_t off) {
  return *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(base) + off);
}

__device__ __forceinline__ void unpack8(uint4 u, int dt, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (dt == MOE_DT_BF16) {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      v[2 * i] = __low2float(h);
      v[2 * i + 1] = __high2float(h);
    } else {
      const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      v[2 * i] = __low2float(h);
      v[2 * i + 1] = __high2float(h);
    }
  }
}

// One warp per (token, run of spw 256-column slices): lane l owns 8 columns of
// a slice, loads the token's k expert rows (and the shared row) for them
// kBatch at a time, then sums in slot order. Few tokens: one slice per warp,
// so a single token is spread over H/256 warps; many tokens: a warp walks
// several slices of its token.
constexpr int kBatch = 4;

__global__ void __launch_bounds__(kThreads, 4) combine_kernel(const Params p, int spw) {
  pdl_trigger();
  pdl_wait();  // before the first global memory access
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t slices = (p.H + 255) / 256;
  const int64_t runs = (slices + spw - 1) / spw;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + warp;
  if (unit >= p.T * runs) return;
  const int64_t t = unit / runs;
  const int64_t rows = p.T * p.k;
  int my_r = 0;
  float my_w = 0.f;
  if (lane < p.k) {
    my_r = p.pos[t * p.k + lane];
    my_w = p.w[t * p.k + lane];
    if (my_r < 0 || my_r >= rows) {
      // a slot the grouping rejected (or a corrupted position): contributes 0
      if (p.status && my_r >= rows) atomicCAS(p.status, 0, MOE_ERR_BAD_OFFSETS);
      my_r = 0;
      my_w = 0.f;
    }
  }
  const bool y16 = p.y_dtype != MOE_DT_F32;
  const int64_t slice0 = (unit % runs) * spw;
  for (int64_t sl = slice0; sl < slice0 + spw && sl < slices; ++sl) {
    const int64_t h = sl * 256 + lane * 8;
    const bool active = h < p.H;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < p.k; s0 += kBatch) {
      int r[kBatch];
      float ws[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        r[j] = __shfl_sync(0xffffffffu, my_r, (s0 + j) & 31);
        ws[j] = __shfl_sync(0xffffffffu, my_w, (s0 + j) & 31);
      }
      if (!active) continue;
      if (y16) {
        uint4 raw[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j)
          if (s0 + j < p.k) raw[j] = load_raw16(p.y, static_cast<int64_t>(r[j]) * p.H + h);
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
          if (s0 + j < p.k) {
            float v[8];
            unpack8(raw[j], p.y_dtype, v);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = fmaf(ws[j], v[i], acc[i]);
          }
        }
      } else {
        for (int j = 0; j < kBatch && s0 + j < p.k; ++j) {
          float v[8];
          load8(p.y, p.y_dtype, static_cast<int64_t>(r[j]) * p.H + h, v);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = fmaf(ws[j], v[i], acc[i]);
        }
      }
    }
    if (!active) continue;
    if (p.y_shared) {
      float v[8];
      load8(p.y_shared, p.y_dtype, t * p.H + h, v);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += v[i];
    }
    store8(p.out, p.out_dtype, t * p.H + h, acc);
  }
}

struct QuantParams {
  const void* w;
  int8_t* q;
  void* scale;
  int64_t rows, K;
  int w_dtype, scale_bf16;
};

__device__ __forceinline__ float ldf(const void* p, int dt, int64_t i) {
  if (dt == MOE_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == MOE_DT_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__global__ void __launch_bounds__(kThreads) quantize_kernel(const QuantParams p) {
  pdl_trigger();
  pdl_wait();  // before the first global memory access
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + warp;
  if (r >= p.rows) return;
  const int64_t off = r * p.K;
  float amax = 0.f;
  for (int64_t i = lane; i < p.K; i += 32) amax = fmaxf(amax, fabsf(ldf(p.w, p.w_dtype, off + i)));
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, d));
  const float scale = amax == 0.f ? 1.0f : amax / 127.0f;
  for (int64_t i = lane; i < p.K; i += 32) {
    float qv = rintf(ldf(p.w, p.w_dtype, off + i) / scale);
    qv = fminf(127.f, fmaxf(-127.f, qv));
    p.q[off + i] = static_cast<int8_t>(qv);
  }
  if (lane == 0) {
    if (p.scale_bf16) reinterpret_cast<__nv_bfloat16*>(p.scale)[r] = __float2bfloat16_rn(scale);
    else reinterpret_cast<float*>(p.scale)[r] = scale;
  }
}

}  // namespace combine
}  // namespace moe
