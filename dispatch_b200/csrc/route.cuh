// Router: logits (x @ router_w^T, f32 accumulate) and expert selection in one
// kernel. A CTA stages TB token rows of x in shared memory as f32 and each warp
// walks a strided set of experts, streaming that expert's router row once for
// all TB tokens; then one warp per token runs the selection:
//   softmax mode: max, sum of exp, k rounds of warp arg-max (lower id wins a
//   tie), weight = exp(l - max) / sum, optional renormalisation;
//   sigmoid-group mode (DeepSeek-V3): s = sigmoid(l), c = s + bias, group
//   score = top1 + top2 of c in each group, keep topk_group groups, k rounds
//   of arg-max of c inside them, weight = s (normalised, scaled).
#pragma once
#include "ptx.cuh"

namespace moe {
namespace route {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxE = 256;
constexpr int kMaxK = 16;
constexpr int kMaxTB = 16;
constexpr int kMaxSplits = 16;  // most f32 partial-logit slabs

struct Params {
  const void* x;
  const void* w;
  const float* logits_in;
  const float* bias;
  int32_t* topk_idx;
  float* topk_w;
  float* logits_out;
  int32_t* status;
  int64_t T, H;
  int E, k, mode, renorm, n_group, topk_group, x_dtype, w_dtype, tb;
  int n_splits;  // logits_in holds n_splits f32 slabs of (T, E) partial sums, added in order
  float scaling;
};

__device__ __forceinline__ float to_f32(const void* p, int dt, int64_t i) {
  if (dt == MOE_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == MOE_DT_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// 8 consecutive elements as f32 (16-byte aligned): one 16-byte load for 16-bit
// types, two for f32.
__device__ __forceinline__ void load8f(const void* p, int dt, int64_t i, float (&v)[8]) {
  if (dt == MOE_DT_F32) {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    return;
  }
  const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + i);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (dt == MOE_DT_BF16) {
      const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[j]);
      v[2 * j] = __low2float(h);
      v[2 * j + 1] = __high2float(h);
    } else {
      const __half2 h = *reinterpret_cast<const __half2*>(&w[j]);
      v[2 * j] = __low2float(h);
      v[2 * j + 1] = __high2float(h);
    }
  }
}

// Warp arg-max: larger value wins, equal values go to the lower index.
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, d);
    const int oi = __shfl_xor_sync(0xffffffffu, i, d);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}

// J: experts per lane in the selection (32 * J >= E): the launch picks 2, 4 or
// 8, so that a 64-expert router walks 2 slots per lane in each of its k
// rounds instead of 8 (slots past E hold -inf and are never chosen, so J
// changes the work, not the result).
template <int J>
__global__ void __launch_bounds__(kThreads, 4) route_kernel(const Params p) {
  pdl_trigger();
  pdl_wait();  // before the first global memory access
  extern __shared__ float smem_f[];
  const int tb = p.tb;
  const int E = p.E;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * tb;
  const int ntok = static_cast<int>((p.T - t0) < tb ? (p.T - t0) : tb);
  // [tb][H] x rows (compute mode; 16-byte aligned since H % 8 == 0), then [tb][E] logits
  float* xs = smem_f;
  float* lg = smem_f + (p.logits_in ? 0 : static_cast<int64_t>(tb) * p.H);
  __shared__ float cbuf[kWarps][kMaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (p.logits_in) {
    // all slab loads in flight first, then the sum in slab order
    const int64_t slab = p.T * E;
    for (int i = threadIdx.x; i < ntok * E; i += kThreads) {
      float part[kMaxSplits];
#pragma unroll
      for (int s = 0; s < kMaxSplits; ++s) part[s] = s < p.n_splits ? p.logits_in[s * slab + t0 * E + i] : 0.f;
      float v = part[0];
#pragma unroll
      for (int s = 1; s < kMaxSplits; ++s)
        if (s < p.n_splits) v += part[s];
      lg[i] = v;
    }
  } else {
    const int64_t H = p.H;
    for (int64_t i = threadIdx.x; i < static_cast<int64_t>(ntok) * H; i += kThreads)
      xs[i] = to_f32(p.x, p.x_dtype, t0 * H + i);
    __syncthreads();
    for (int e = warp; e < E; e += kWarps) {
      float acc[kMaxTB];
#pragma unroll
      for (int t = 0; t < kMaxTB; ++t) acc[t] = 0.f;
      // 8 consecutive weights per lane per step (H % 8 == 0, checked on the host)
#pragma unroll 2
      for (int64_t h = lane * 8; h < H; h += 256) {
        float wv[8];
        load8f(p.w, p.w_dtype, static_cast<int64_t>(e) * H + h, wv);
#pragma unroll
        for (int t = 0; t < kMaxTB; ++t) {
          if (t < ntok) {
            const float4 a = *reinterpret_cast<const float4*>(xs + t * H + h);
            const float4 b = *reinterpret_cast<const float4*>(xs + t * H + h + 4);
            float s = acc[t];
            s = fmaf(a.x, wv[0], s); s = fmaf(a.y, wv[1], s); s = fmaf(a.z, wv[2], s); s = fmaf(a.w, wv[3], s);
            s = fmaf(b.x, wv[4], s); s = fmaf(b.y, wv[5], s); s = fmaf(b.z, wv[6], s); s = fmaf(b.w, wv[7], s);
            acc[t] = s;
          }
        }
      }
#pragma unroll
      for (int t = 0; t < kMaxTB; ++t) {
        if (t < ntok) {
          const float s = warp_sum(acc[t]);
          if (lane == 0) lg[t * E + e] = s;
        }
      }
    }
  }
  __syncthreads();
  // logits_out holds the raw gate output, before any bias
  if (p.logits_out)
    for (int i = threadIdx.x; i < ntok * E; i += kThreads) p.logits_out[t0 * E + i] = lg[i];
  if (p.mode == MOE_ROUTER_SOFTMAX && p.bias) {
    // softmax mode: the bias is part of the logits (a gate Linear with bias)
    __syncthreads();
    for (int i = threadIdx.x; i < ntok * E; i += kThreads) lg[i] += p.bias[i % E];
    __syncthreads();
  }

  for (int t = warp; t < ntok; t += kWarps) {
    const float* l = lg + t * E;
    float v[J];
    // slot q's expert and weight are kept by lane q
    int my_sel = 0;
    float my_w = 0.f;
    if (p.mode == MOE_ROUTER_SOFTMAX) {
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int e = lane + 32 * j;
        v[j] = e < E ? l[e] : -INFINITY;
      }
      float m = -INFINITY;
#pragma unroll
      for (int j = 0; j < J; ++j) m = fmaxf(m, v[j]);
      m = warp_max(m);
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < J; ++j)
        if (lane + 32 * j < E) s += expf(v[j] - m);
      s = warp_sum(s);
      for (int q = 0; q < p.k; ++q) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < J; ++j) {
          const int e = lane + 32 * j;
          if (e < E && (v[j] > bv || (v[j] == bv && e < bi))) {
            bv = v[j];
            bi = e;
          }
        }
        warp_argmax(bv, bi);
        if (lane == q) {
          my_sel = bi;
          my_w = expf(bv - m) / s;
        }
        if ((bi & 31) == lane) {
#pragma unroll
          for (int j = 0; j < J; ++j)
            if (lane + 32 * j == bi) v[j] = -INFINITY;
        }
      }
      if (p.renorm) my_w = my_w / warp_sum(lane < p.k ? my_w : 0.f);
    } else {
      // sigmoid, group-limited
      float* cb = cbuf[warp];
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int e = lane + 32 * j;
        if (e < E) {
          const float sg = 1.0f / (1.0f + expf(-l[e]));
          cb[e] = sg + (p.bias ? p.bias[e] : 0.f);
        }
      }
      __syncwarp();
      const int G = p.n_group, per = E / G;
      float gs = -INFINITY;
      if (lane < G) {
        float b1 = -INFINITY, b2 = -INFINITY;
        for (int i = 0; i < per; ++i) {
          const float c = cb[lane * per + i];
          if (c > b1) {
            b2 = b1;
            b1 = c;
          } else if (c > b2) {
            b2 = c;
          }
        }
        gs = per >= 2 ? b1 + b2 : b1;
      }
      uint32_t gmask = 0;
      for (int q = 0; q < p.topk_group; ++q) {
        float bv = (lane < G && !((gmask >> lane) & 1u)) ? gs : -INFINITY;
        int bi = lane < G && !((gmask >> lane) & 1u) ? lane : 0x7fffffff;
        warp_argmax(bv, bi);
        if (bi < 32) gmask |= 1u << bi;
      }
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int e = lane + 32 * j;
        v[j] = (e < E && ((gmask >> (e / per)) & 1u)) ? cb[e] : -INFINITY;
      }
      for (int q = 0; q < p.k; ++q) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < J; ++j) {
          const int e = lane + 32 * j;
          if (e < E && v[j] != -INFINITY && (v[j] > bv || (v[j] == bv && e < bi))) {
            bv = v[j];
            bi = e;
          }
        }
        warp_argmax(bv, bi);
        if (lane == q) {
          my_sel = bi;
          my_w = 1.0f / (1.0f + expf(-l[bi]));
        }
        if ((bi & 31) == lane) {
#pragma unroll
          for (int j = 0; j < J; ++j)
            if (lane + 32 * j == bi) v[j] = -INFINITY;
        }
      }
      if (p.renorm) my_w = my_w / warp_sum(lane < p.k ? my_w : 0.f);
      my_w *= p.scaling;
      __syncwarp();
    }
    if (lane < p.k) {
      int si = my_sel;
      const float sw = my_w;
      if (si < 0 || si >= E) {
        if (p.status) atomicCAS(p.status, 0, MOE_ERR_BAD_EXPERT);
        si = 0;
      }
      p.topk_idx[(t0 + t) * p.k + lane] = si;
      p.topk_w[(t0 + t) * p.k + lane] = sw;
    }
  }
}

}  // namespace route
}  // namespace moe
