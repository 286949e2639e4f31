// Host side of the C ABIs declared in include/moe_b200.h and
// include/moe_ep_b200.h: argument checks, TMA tensor-map encoding and kernel
// launches. Nothing allocates except the moe_peer_* set-up calls.
#include <cuda.h>
#include <cuda_runtime.h>

#include <array>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/moe_b200.h"
#include "../../include/moe_ep_b200.h"
#include "combine.cuh"
#include "ep.cuh"
#include "gemm.cuh"
#include "gemm2sm.cuh"
#include "gemm_stream.cuh"
#include "gemm_warp.cuh"
#include "group.cuh"
#include "route.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define CUDA_TRY(expr, what)                 \
  do {                                       \
    cudaError_t _e = (expr);                 \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

// Launches a kernel with programmatic stream serialisation: it may begin its
// set-up while the previous kernel in the stream drains, and waits for that
// kernel (griddepcontrol.wait) before touching global memory. Works under
// stream capture (the graph keeps a programmatic edge).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

#define CHECK_ARG(cond, ...)                                   \
  do {                                                         \
    if (!(cond)) return fail(MOE_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  std::once_flag once;
  int sms = 0;
  int major = 0;
};
std::array<DeviceInfo, kMaxDevices> g_dev;

int device_info(int* sms) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(MOE_ERR_NO_DEVICE, "no CUDA device is current");
  DeviceInfo& d = g_dev[dev];
  std::call_once(d.once, [&] {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
  });
  if (d.major != 10) return fail(MOE_ERR_NO_DEVICE, "device %d is sm_%d0, this library is built for sm_100a", dev, d.major);
  *sms = d.sms;
  return MOE_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool is16(int dt) { return dt == MOE_DT_BF16 || dt == MOE_DT_F16; }
size_t dt_size(int dt) {
  switch (dt) {
    case MOE_DT_BF16: case MOE_DT_F16: return 2;
    case MOE_DT_F32: case MOE_DT_I32: return 4;
    case MOE_DT_I8: return 1;
    case MOE_DT_I64: return 8;
    default: return 0;
  }
}
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A operand: 2D {K, rows} with row stride lda elements, box {64, 128}.
int make_map_a(CUtensorMap* m, const void* a, int dt, int64_t rows, int64_t K, int64_t lda, int box_rows = 128) {
  EncodeTiledFn enc = encoder();
  if (!enc) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(lda * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, dt == MOE_DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(a), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MOE_ERR_INVALID_ARG, "tensor map (A) encode failed (%d)", static_cast<int>(r));
  return MOE_OK;
}

// B operand: 3D {K, N, G}, box {64, box_rows, 1}; 16-bit types use the
// 128-byte swizzle, int8 is staged unswizzled for the in-smem dequantiser.
int make_map_b(CUtensorMap* m, const void* w, int dt, int64_t G, int64_t N, int64_t K, int box_rows) {
  EncodeTiledFn enc = encoder();
  if (!enc) return fail(MOE_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const size_t es_b = dt_size(dt);
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(G)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(K * es_b), static_cast<cuuint64_t>(N * K * es_b)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUtensorMapDataType t = dt == MOE_DT_I8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                          : dt == MOE_DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = enc(m, t, 3, const_cast<void*>(w), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   dt == MOE_DT_I8 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MOE_ERR_INVALID_ARG, "tensor map (B) encode failed (%d)", static_cast<int>(r));
  return MOE_OK;
}

// Description of one GEMM segment before encoding.
struct SegSpec {
  const void* a;
  int64_t a_rows;
  int64_t lda;
  const void* b0;
  const void* b1;
  int b_dtype;  // activation type or MOE_DT_I8
  const void* scale0;
  const void* scale1;
  int scale_dtype;
  int64_t G, N, K;         // G row groups (offsets has G+1 entries)
  int64_t Gw = 0;          // weight experts; group g uses weight g % Gw (0 => Gw = G)
  const int32_t* offsets;  // nullptr => dense over a_rows
  void* out;
  int64_t ldo;
  bool swiglu;
  int mma_n = moe::gemm::BN;  // multiple of 32 (64 for SwiGLU), <= 256
  bool out_f32 = false;
  // Gathered A: logical row r reads row gather_rows[r] of `a`, which has
  // gather_src_rows rows (a_rows stays the logical row count).
  const int64_t* gather_rows = nullptr;
  int64_t gather_src_rows = 0;
  // split-K into f32 partial slabs out + s * split_stride (plain f32 segments)
  int k_splits = 1;
  int64_t split_stride = 0;
  // scattered output rows (Segment::out_rows); out is then unused
  const int32_t* out_rows = nullptr;
  void* const* out_table = nullptr;
  int out_table_n = 0;
  int64_t out_table_rows = 0;
  // rows of the A (activation) TMA box: 128 for the tiled kernel, the row
  // tile for the streaming kernel
  int a_box_rows = moe::gemm::BM;
  // rows of the weight TMA boxes; 0: mma_n (mma_n / 2 for SwiGLU). The CTA-pair
  // kernel loads 128 weight rows per CTA.
  int b_box_rows = 0;
};

int fill_segment(moe::gemm::Segment* s, const SegSpec& sp, int act_dtype) {
  std::memset(s, 0, sizeof(*s));
  // a gathered A is fetched one row per box, four boxes per tile::gather4
  int rc = sp.gather_rows ? make_map_a(&s->map_a, sp.a, act_dtype, sp.gather_src_rows, sp.K, sp.lda, 1)
                          : make_map_a(&s->map_a, sp.a, act_dtype, sp.a_rows, sp.K, sp.lda, sp.a_box_rows);
  if (rc) return rc;
  const int box_rows = sp.b_box_rows > 0 ? sp.b_box_rows : (sp.swiglu ? sp.mma_n / 2 : sp.mma_n);
  const int64_t gw = sp.Gw > 0 ? sp.Gw : sp.G;
  rc = make_map_b(&s->map_b0, sp.b0, sp.b_dtype, gw, sp.N, sp.K, box_rows);
  if (rc) return rc;
  if (sp.swiglu) {
    rc = make_map_b(&s->map_b1, sp.b1, sp.b_dtype, gw, sp.N, sp.K, box_rows);
    if (rc) return rc;
  }
  s->offsets = sp.offsets;
  s->gather_rows = sp.gather_rows;
  s->scale0 = sp.scale0;
  s->scale1 = sp.scale1;
  s->out = sp.out;
  s->ldo = sp.ldo;
  s->groups = static_cast<int>(sp.offsets ? sp.G : 1);
  s->weight_mod = static_cast<int>(sp.offsets ? gw : 1);
  s->dense_rows = static_cast<int>(sp.a_rows);
  s->n = static_cast<int>(sp.N);
  s->k = static_cast<int>(sp.K);
  s->swiglu = sp.swiglu ? 1 : 0;
  s->b_int8 = sp.b_dtype == MOE_DT_I8 ? 1 : 0;
  s->scale_bf16 = sp.scale_dtype == MOE_DT_BF16 ? 1 : 0;
  s->mma_n = sp.mma_n;
  s->out_f32 = sp.out_f32 ? 1 : 0;
  s->k_splits = sp.k_splits;
  s->split_stride = sp.split_stride;
  s->out_rows = sp.out_rows;
  s->out_table = sp.out_table;
  s->out_table_n = sp.out_table_n;
  s->out_table_rows = sp.out_table_rows;
  return MOE_OK;
}

int check_seg(const SegSpec& sp, int act_dtype) {
  CHECK_ARG(sp.a && sp.b0 && (sp.out || sp.out_rows), "null operand pointer");
  CHECK_ARG(!sp.out_rows || (sp.out_table && sp.out_table_n >= 1 && sp.out_table_n <= MOE_EP_MAX_RANKS &&
                             sp.out_table_rows >= 1 && sp.k_splits == 1 && !sp.out_f32 && sp.ldo % 8 == 0),
            "scattered output needs a table of 1..%d bases, one K range, 16-bit rows", MOE_EP_MAX_RANKS);
  CHECK_ARG(!sp.swiglu || sp.b1, "null up-projection pointer");
  CHECK_ARG(sp.a_rows > 0 && sp.a_rows < (1ll << 31), "row count %lld out of range", (long long)sp.a_rows);
  CHECK_ARG(sp.G >= 1 && sp.G <= moe::gemm::kMaxGroups, "expert count %lld not in [1, %d]", (long long)sp.G,
            moe::gemm::kMaxGroups);
  CHECK_ARG(sp.N >= 1 && sp.N < (1ll << 31) && sp.K >= 1 && sp.K < (1ll << 31), "bad N/K");
  CHECK_ARG(is16(act_dtype), "activation dtype must be bf16 or f16");
  CHECK_ARG(sp.b_dtype == act_dtype || sp.b_dtype == MOE_DT_I8, "dtype mismatch: weight %d vs activation %d",
            sp.b_dtype, act_dtype);
  const int kmul = sp.b_dtype == MOE_DT_I8 ? 16 : 8;
  CHECK_ARG(sp.K % kmul == 0, "K mismatch: K=%lld must be a multiple of %d", (long long)sp.K, kmul);
  CHECK_ARG(sp.mma_n >= 32 && sp.mma_n <= moe::gemm::BN && sp.mma_n % (sp.swiglu ? 64 : 32) == 0,
            "MMA width %d must be a multiple of %d in [32, 256]", sp.mma_n, sp.swiglu ? 64 : 32);
  CHECK_ARG(!sp.out_f32 || !sp.swiglu, "f32 output is for plain segments");
  CHECK_ARG(sp.k_splits >= 1 && sp.k_splits <= (sp.K + 63) / 64 && (sp.k_splits == 1 || sp.out_f32),
            "split-K needs 1 <= splits <= K/64 and an f32 output");
  CHECK_ARG(sp.lda % 8 == 0 && aligned16(sp.a) && aligned16(sp.b0) && (!sp.b1 || aligned16(sp.b1)),
            "operands must be 16-byte aligned with row strides a multiple of 16 bytes");
  if (sp.b_dtype == MOE_DT_I8) {
    CHECK_ARG(sp.scale0 && (!sp.swiglu || sp.scale1), "int8 weights need scales");
    CHECK_ARG(sp.scale_dtype == MOE_DT_F32 || sp.scale_dtype == MOE_DT_BF16, "scale dtype must be f32 or bf16");
  }
  return MOE_OK;
}

template <bool kInt8>
int launch_gemm(const moe::gemm::Params& p, int sms, cudaStream_t stream) {
  constexpr size_t smem = moe::gemm::smem_bytes<kInt8>();
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(moe::gemm::grouped_gemm_kernel<kInt8>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute(gemm)");
  CUDA_TRY(launch_pdl(moe::gemm::grouped_gemm_kernel<kInt8>, dim3(sms), dim3(moe::gemm::Config<kInt8>::kThreads),
                      smem, stream, p),
           "grouped_gemm_kernel launch");
  return MOE_OK;
}

// Upper bound of a segment's tiles: a non-empty group of c rows has
// ceil(c/128) <= c/128 + 1 tiles, so a segment has at most R/128 + min(G, R).
int64_t tile_bound(const SegSpec& sp, int mma_n) {
  const int oc = sp.swiglu ? mma_n / 2 : mma_n;
  const int64_t mt = sp.offsets ? sp.a_rows / moe::gemm::BM + (sp.G < sp.a_rows ? sp.G : sp.a_rows)
                                : (sp.a_rows + moe::gemm::BM - 1) / moe::gemm::BM;
  return mt * ((sp.N + oc - 1) / oc) * sp.k_splits;
}

int run_gemm(const SegSpec* specs_in, int nseg, int act_dtype, int32_t* status, cudaStream_t stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  SegSpec specs[moe::gemm::kMaxSegs];
  for (int i = 0; i < nseg; ++i) specs[i] = specs_in[i];
  // Narrowing the tiles of small launches (a row's result does not depend on
  // the tile width) was measured slower on B200: the zero-filled 128-row A
  // boxes then dominate the TMA traffic. Kept off; the loop below only runs
  // when kNarrowSmallLaunches is set.
  constexpr bool kNarrowSmallLaunches = false;
  for (; kNarrowSmallLaunches;) {
    int64_t total = 0;
    bool can_halve = true;
    for (int i = 0; i < nseg; ++i) {
      total += tile_bound(specs[i], specs[i].mma_n);
      can_halve &= !specs[i].out_f32 && specs[i].mma_n >= (specs[i].swiglu ? 128 : 64) &&
                   specs[i].mma_n % (specs[i].swiglu ? 128 : 64) == 0;
    }
    if (total >= sms || !can_halve) break;
    for (int i = 0; i < nseg; ++i) specs[i].mma_n /= 2;
  }
  moe::gemm::Params p;
  std::memset(&p, 0, sizeof(p));
  bool any_i8 = false;
  int64_t tiles_bound = 0;
  for (int i = 0; i < nseg; ++i) {
    rc = check_seg(specs[i], act_dtype);
    if (rc) return rc;
    rc = fill_segment(&p.seg[i], specs[i], act_dtype);
    if (rc) return rc;
    any_i8 |= specs[i].b_dtype == MOE_DT_I8;
    tiles_bound += tile_bound(specs[i], specs[i].mma_n);
    p.remote_out |= specs[i].out_rows ? 1 : 0;
  }
  p.num_segs = nseg;
  p.in_f16 = act_dtype == MOE_DT_F16 ? 1 : 0;
  p.status = status;
  const int grid = static_cast<int>(tiles_bound < sms ? tiles_bound : sms);
  if (grid <= 0) return MOE_OK;
  return any_i8 ? launch_gemm<true>(p, grid, stream) : launch_gemm<false>(p, grid, stream);
}

// ---------------------------------------------------------------- CTA-pair kernel
// Cluster launch of two CTAs per tile (programmatic dependent launch too).
int launch_pair(const moe::gemm::Params& p, int grid, cudaStream_t stream) {
  constexpr size_t smem = moe::gemm::pair_smem_bytes();
  static_assert(smem <= 232448, "shared memory of the CTA-pair kernel");
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(moe::gemm::grouped_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem));
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute(pair gemm)");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(moe::gemm::kPairThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  CUDA_TRY(cudaLaunchKernelEx(&cfg, moe::gemm::grouped_gemm_pair_kernel, p), "grouped_gemm_pair_kernel launch");
  return MOE_OK;
}

// The CTA-pair kernel over up to two FFN segments (16-bit weights, one K
// range, no gathered rows, 16-bit outputs): tiles of 256 weight rows x up to
// 256 token rows.
int run_gemm_pair(const SegSpec* specs_in, int nseg, int act_dtype, int32_t* status, cudaStream_t stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  moe::gemm::Params p;
  std::memset(&p, 0, sizeof(p));
  int64_t tiles = 0;
  for (int i = 0; i < nseg; ++i) {
    SegSpec spec = specs_in[i];
    CHECK_ARG(!spec.out_f32 && spec.k_splits == 1 && !spec.gather_rows && spec.b_dtype != MOE_DT_I8,
              "the CTA-pair kernel takes 16-bit weights, one K range, 16-bit outputs");
    spec.mma_n = 2 * moe::gemm::BM;
    // each CTA loads 128 weight rows (64 gate + 64 up rows, or 128 plain rows)
    // and its half of the tile's token rows in one 128-row box (smaller boxes,
    // several per k-block, measured slower)
    spec.b_box_rows = spec.swiglu ? moe::gemm::BM / 2 : moe::gemm::BM;
    rc = check_seg(spec, act_dtype);
    if (rc) return rc;
    rc = fill_segment(&p.seg[i], spec, act_dtype);
    if (rc) return rc;
    const int oc = spec.swiglu ? moe::gemm::BM : 2 * moe::gemm::BM;
    const int64_t rt = 2 * moe::gemm::BM;
    const int64_t mt = spec.offsets ? spec.a_rows / rt + (spec.G < spec.a_rows ? spec.G : spec.a_rows)
                                    : (spec.a_rows + rt - 1) / rt;
    tiles += mt * ((spec.N + oc - 1) / oc);
    p.remote_out |= spec.out_rows ? 1 : 0;
  }
  p.num_segs = nseg;
  p.in_f16 = act_dtype == MOE_DT_F16 ? 1 : 0;
  p.status = status;
  const int64_t pairs = tiles < sms / 2 ? tiles : sms / 2;
  if (pairs <= 0) return MOE_OK;
  return launch_pair(p, static_cast<int>(2 * pairs), stream);
}

// ---------------------------------------------------------------- warp-MMA kernel
template <int kWarps, bool kInt8>
int launch_warp(const moe::gemm::WarpParams& wp, int grid, cudaStream_t stream) {
  constexpr size_t smem = moe::gemm::warp_smem_bytes<kWarps>();
  static_assert(2 * (smem + 1024) <= 233472, "two warp-MMA CTAs per SM");
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(moe::gemm::grouped_gemm_warp_kernel<kWarps, kInt8>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute(warp gemm)");
  CUDA_TRY(launch_pdl(moe::gemm::grouped_gemm_warp_kernel<kWarps, kInt8>, dim3(grid),
                      dim3(moe::gemm::WarpConfig<kWarps>::kThreads), smem, stream, wp),
           "grouped_gemm_warp_kernel launch");
  return MOE_OK;
}

// The warp-MMA kernel over up to two FFN segments (16-bit or int8 weights,
// one K range, no gathered rows, 16-bit outputs), two CTAs per SM. Tiles of 64
// weight rows (four MMA warps, eight stages) when even twice as many tiles as
// 128-row ones leave CTA slots free -- a decode step's few tiles then use
// twice the SMs with the same weight bytes in flight per tile (C2 T=1 layer
// graph 73.3 -> 71.2 us) -- else of 128 rows (eight warps, four stages: with
// 64-row tiles beyond the slots, T=2 was 80 -> 99 us); the token-row tile is
// the smallest of 8 / 16 / 32 that holds the average group.
int run_gemm_warp(const SegSpec* specs_in, int nseg, const int64_t* avg_rows, int act_dtype, int32_t* status,
                  cudaStream_t stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  int64_t most = 1;
  for (int i = 0; i < nseg; ++i) most = avg_rows[i] > most ? avg_rows[i] : most;
  const int nt = most <= 8 ? 8 : most <= 16 ? 16 : moe::gemm::kWTok;
  const int64_t slots = 2 * static_cast<int64_t>(sms);
  // tiles with 128-row weight blocks
  int64_t tiles128 = 0;
  for (int i = 0; i < nseg; ++i) {
    const SegSpec& spec = specs_in[i];
    const int oc = spec.swiglu ? 64 : 128;
    const int64_t mt = spec.offsets ? spec.a_rows / nt + (spec.G < spec.a_rows ? spec.G : spec.a_rows)
                                    : (spec.a_rows + nt - 1) / nt;
    tiles128 += mt * ((spec.N + oc - 1) / oc);
  }
  const int warps = 2 * tiles128 <= slots ? 4 : 8;
  moe::gemm::WarpParams wp;
  std::memset(&wp, 0, sizeof(wp));
  wp.nt = nt;
  int64_t tiles = 0;
  bool any_i8 = false;
  for (int i = 0; i < nseg; ++i) {
    SegSpec spec = specs_in[i];
    CHECK_ARG(!spec.out_f32 && spec.k_splits == 1 && !spec.gather_rows,
              "the warp-MMA kernel takes one K range, no gathered rows, 16-bit outputs");
    any_i8 |= spec.b_dtype == MOE_DT_I8;
    spec.mma_n = 16 * warps;
    spec.a_box_rows = nt;
    spec.b_box_rows = 0;  // half gate, half up rows, or all rows
    rc = check_seg(spec, act_dtype);
    if (rc) return rc;
    rc = fill_segment(&wp.p.seg[i], spec, act_dtype);
    if (rc) return rc;
    const int oc = spec.swiglu ? 8 * warps : 16 * warps;
    const int64_t mt = spec.offsets ? spec.a_rows / nt + (spec.G < spec.a_rows ? spec.G : spec.a_rows)
                                    : (spec.a_rows + nt - 1) / nt;
    tiles += mt * ((spec.N + oc - 1) / oc);
    wp.p.remote_out |= spec.out_rows ? 1 : 0;
  }
  wp.p.num_segs = nseg;
  wp.p.in_f16 = act_dtype == MOE_DT_F16 ? 1 : 0;
  wp.p.status = status;
  const int64_t grid = tiles < slots ? tiles : slots;
  if (grid <= 0) return MOE_OK;
  if (any_i8)
    return warps == 8 ? launch_warp<8, true>(wp, static_cast<int>(grid), stream)
                      : launch_warp<4, true>(wp, static_cast<int>(grid), stream);
  return warps == 8 ? launch_warp<8, false>(wp, static_cast<int>(grid), stream)
                    : launch_warp<4, false>(wp, static_cast<int>(grid), stream);
}

// ---------------------------------------------------------------- streaming kernel
std::atomic<int> g_ffn_kernel{MOE_FFN_KERNEL_AUTO};

// Largest dynamic shared memory of one CTA on sm_100 (227 KiB).
constexpr size_t kMaxDynSmem = 232448;

template <bool kInt8>
int launch_stream(const moe::gemm::StreamParams& sp, int grid, size_t smem, cudaStream_t stream) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err = cudaFuncSetAttribute(moe::gemm::grouped_gemm_stream_kernel<kInt8>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kMaxDynSmem));
  });
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute(stream gemm)");
  CUDA_TRY(launch_pdl(moe::gemm::grouped_gemm_stream_kernel<kInt8>, dim3(grid),
                      dim3(moe::gemm::StreamConfig<kInt8>::kThreads), smem, stream, sp),
           "grouped_gemm_stream_kernel launch");
  return MOE_OK;
}

// The streaming kernel over up to two segments; row_tiles[i] (a multiple of
// 32, at most 256) is segment i's token rows per tile. Segments must be plain
// 16-bit-output GEMMs with one K range and no gathered rows.
//
// Chains per tile (1 or 2 weight blocks sharing the tile's rows, their MMAs
// interleaved): a single accumulator's dependent MMAs run at ~330 cycles each
// on B200 whatever the MMA width, two interleaved chains at ~420 cycles per
// pair, so two chains nearly double the tensor rate of a tile -- but halve
// the tile count. Two chains are used unless that leaves the launch with
// fewer tiles than SMs where one chain would have had several per SM
// (estimated from the tile-count bound: waves x chain cost).
int run_gemm_stream(const SegSpec* specs_in, const int* row_tiles, int nseg, int act_dtype, int32_t* status,
                    cudaStream_t stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  moe::gemm::StreamParams sp;
  std::memset(&sp, 0, sizeof(sp));
  bool any_i8 = false;
  int64_t tiles1 = 0, tiles2 = 0;  // tile-count bounds with one and with two chains
  int nt_max = 0;
  for (int i = 0; i < nseg; ++i) {
    SegSpec spec = specs_in[i];
    const int nt = row_tiles[i];
    CHECK_ARG(nt % 32 == 0 && nt >= 32 && nt <= moe::gemm::kStreamMaxRowTile,
              "row tile %d must be a multiple of 32 in [32, %d]", nt, moe::gemm::kStreamMaxRowTile);
    CHECK_ARG(!spec.out_f32 && spec.k_splits == 1 && !spec.gather_rows,
              "the streaming kernel takes plain 16-bit-output segments");
    spec.mma_n = moe::gemm::SM_ROWS;
    spec.a_box_rows = nt;
    rc = check_seg(spec, act_dtype);
    if (rc) return rc;
    rc = fill_segment(&sp.p.seg[i], spec, act_dtype);
    if (rc) return rc;
    sp.row_tile[i] = nt;
    nt_max = nt > nt_max ? nt : nt_max;
    any_i8 |= spec.b_dtype == MOE_DT_I8;
    const int oc = spec.swiglu ? moe::gemm::SM_ROWS / 2 : moe::gemm::SM_ROWS;
    const int64_t rt = spec.offsets ? spec.a_rows / nt + (spec.G < spec.a_rows ? spec.G : spec.a_rows)
                                    : (spec.a_rows + nt - 1) / nt;
    const int64_t ct = (spec.N + oc - 1) / oc;
    tiles1 += rt * ct;
    tiles2 += rt * ((ct + 1) / 2);
    sp.p.remote_out |= spec.out_rows ? 1 : 0;
  }
  const int64_t waves1 = (tiles1 + sms - 1) / sms, waves2 = (tiles2 + sms - 1) / sms;
  const int chains = (waves2 * 420 <= waves1 * 330) ? 2 : 1;
  sp.p.num_segs = nseg;
  sp.p.in_f16 = act_dtype == MOE_DT_F16 ? 1 : 0;
  sp.p.status = status;
  sp.nt_max = nt_max;
  sp.chains = chains;
  sp.acc_slots = chains * nt_max * 2 <= 512 ? 2 : 1;
  const size_t stage = moe::gemm::stream_stage_bytes(any_i8, nt_max, chains);
  size_t stages = (kMaxDynSmem - moe::gemm::stream_fixed_bytes()) / stage;
  if (stages > static_cast<size_t>(moe::gemm::kStreamMaxStages)) stages = moe::gemm::kStreamMaxStages;
  CHECK_ARG(stages >= 2, "streaming kernel: stages do not fit shared memory");
  sp.stages = static_cast<int>(stages);
  const size_t smem = moe::gemm::stream_fixed_bytes() + stages * stage;
  const int64_t tiles = chains == 2 ? tiles2 : tiles1;
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  if (grid <= 0) return MOE_OK;
  return any_i8 ? launch_stream<true>(sp, grid, smem, stream) : launch_stream<false>(sp, grid, smem, stream);
}

// Most K ranges the router's logit GEMM is split into (f32 slabs in the
// router workspace).
constexpr int kRouteMaxSplits = moe::route::kMaxSplits;

int route_tb(int64_t H, int E, bool computing) {
  if (!computing) return moe::route::kWarps;  // one warp per token for the selection
  int tb = 16;
  while (tb > 1 && static_cast<int64_t>(tb) * (H + E) * 4 > 120 * 1024) tb >>= 1;
  return tb;
}

// The grouping's two launches (histogram, then scatter + gather). Copies of
// 16-bit rows are split by column slices (at least 128 bytes of a row per CTA)
// over more CTAs so the gather uses the whole GPU (about four CTAs per SM:
// 0.651 -> 0.647 ms for the C2 T=4096 step against two) even for a decode
// step's few rows.
int launch_grouping(const moe::group::Params& p, int sms, cudaStream_t s) {
  unsigned split = 1;
  if (p.xs && p.x_dtype != MOE_DT_F32) {
    const int64_t per_row = p.H / 8;
    while (split < 32 && static_cast<int64_t>(p.nchunks) * split < 4 * sms && per_row % (2 * split) == 0 &&
           per_row / (2 * split) >= 8)
      split *= 2;
  }
  CUDA_TRY(launch_pdl(moe::group::group_hist_kernel, dim3(p.nchunks), dim3(moe::group::kThreads), 0, s, p),
           "group_hist_kernel launch");
  CUDA_TRY(launch_pdl(moe::group::group_scatter_kernel, dim3(p.nchunks, split), dim3(moe::group::kThreads), 0, s, p),
           "group_scatter_kernel launch");
  return MOE_OK;
}

}  // namespace

extern "C" {

int moe_abi_version(void) { return MOE_B200_ABI_VERSION; }

int moe_set_ffn_kernel(int choice) {
  if (choice != MOE_FFN_KERNEL_AUTO && choice != MOE_FFN_KERNEL_TILED && choice != MOE_FFN_KERNEL_STREAM &&
      choice != MOE_FFN_KERNEL_PAIR && choice != MOE_FFN_KERNEL_WARP)
    return -1;
  return g_ffn_kernel.exchange(choice);
}

static int ffn_auto_kernel(int64_t R, int64_t G, int64_t T_shared, int64_t H, int64_t I, int w_dtype,
                           bool gather);

int moe_ffn_kernel_auto(int64_t R, int64_t G, int64_t T_shared, int64_t H, int64_t I, int w_dtype) {
  if (R < 0 || G < 1 || T_shared < 0 || H < 0 || I < 0) return -1;
  return ffn_auto_kernel(R, G, T_shared, H, I, w_dtype, false);
}

const char* moe_status_string(int code) {
  switch (code) {
    case MOE_OK: return "ok";
    case MOE_ERR_INVALID_ARG: return "invalid argument";
    case MOE_ERR_UNSUPPORTED: return "unsupported";
    case MOE_ERR_CUDA: return "CUDA error";
    case MOE_ERR_NO_DEVICE: return "no sm_100 device";
    case MOE_ERR_TIMEOUT: return "device wait timed out";
    case MOE_ERR_BAD_EXPERT: return "expert id out of range";
    case MOE_ERR_BAD_OFFSETS: return "group offsets or row positions out of range";
    default: return "unknown status";
  }
}

const char* moe_last_error(void) { return g_last_error.c_str(); }

int moe_device_sm_count(void) {
  int sms = 0;
  return device_info(&sms) == MOE_OK ? sms : 0;
}

size_t moe_route_workspace_bytes(int64_t T, int64_t E) {
  return static_cast<size_t>(kRouteMaxSplits) * static_cast<size_t>(T > 0 ? T : 1) * static_cast<size_t>(E) *
         sizeof(float);
}

int moe_route(const void* x, int x_dtype, const void* router_w, int w_dtype, const float* logits_in, int64_t T,
              int64_t H, int64_t E, int k, int mode, int renorm, const float* e_score_bias, int n_group,
              int topk_group, float routed_scaling, int32_t* topk_idx, float* topk_w, float* logits_out,
              void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  CHECK_ARG(T >= 0 && E >= 1 && E <= moe::route::kMaxE, "E=%lld must be in [1, %d]", (long long)E, moe::route::kMaxE);
  CHECK_ARG(k >= 1 && k <= moe::route::kMaxK && k <= E, "top_k=%d must be in [1, min(E, %d)]", k, moe::route::kMaxK);
  if (T == 0) return MOE_OK;  // nothing to route (empty tensors may come with null pointers)
  CHECK_ARG(topk_idx && topk_w, "null output pointer");
  CHECK_ARG(logits_in || (x && router_w && H >= 1), "need logits_in or x and router_w");
  if (!logits_in) {
    CHECK_ARG(x_dtype == MOE_DT_BF16 || x_dtype == MOE_DT_F16 || x_dtype == MOE_DT_F32, "bad x dtype");
    CHECK_ARG(w_dtype == MOE_DT_BF16 || w_dtype == MOE_DT_F16 || w_dtype == MOE_DT_F32, "bad router dtype");
    CHECK_ARG(H % 8 == 0 && aligned16(x) && aligned16(router_w), "H must be a multiple of 8, x/router_w aligned");
  }
  CHECK_ARG(mode == MOE_ROUTER_SOFTMAX || mode == MOE_ROUTER_SIGMOID_GROUP, "unknown router mode %d", mode);
  if (mode == MOE_ROUTER_SIGMOID_GROUP) {
    CHECK_ARG(n_group >= 1 && n_group <= 32 && E % n_group == 0, "n_group=%d must divide E and be <= 32", n_group);
    CHECK_ARG(topk_group >= 1 && topk_group <= n_group, "topk_group=%d not in [1, n_group]", topk_group);
    CHECK_ARG(static_cast<int64_t>(topk_group) * (E / n_group) >= k, "kept groups hold fewer than top_k experts");
  }
  if (T == 0) return MOE_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // bf16/f16 x and router weight: the logits are a dense tcgen05 GEMM with an
  // f32 epilogue (into logits_out), then the selection kernel reads them.
  const bool tensor_logits = !logits_in && is16(x_dtype) && w_dtype == x_dtype && H % 8 == 0 && aligned16(x) &&
                             aligned16(router_w);
  int n_splits = 1;
  if (tensor_logits) {
    CHECK_ARG(workspace && workspace_bytes >= moe_route_workspace_bytes(T, E), "router workspace too small");
    // Split K into up to 16 ranges of at least 2 k-blocks so that many CTAs
    // work on the few 128-row tiles of a small batch (a decode step's logits
    // are one tile); each range writes an f32 slab and the selection kernel
    // sums the slabs in order. The split depends on H only, never on T, so a
    // token's logits (and therefore its ids and weights) are the same bits
    // whatever the batch it is routed in -- which keeps the expert-parallel
    // output byte-identical to the 1-GPU output.
    const int64_t nkb = (H + moe::gemm::BK - 1) / moe::gemm::BK;
    int64_t splits = nkb / 2;
    if (splits > kRouteMaxSplits) splits = kRouteMaxSplits;
    n_splits = static_cast<int>(splits < 1 ? 1 : splits);
    SegSpec sp{};
    sp.a = x;
    sp.a_rows = T;
    sp.lda = H;
    sp.b0 = router_w;
    sp.b_dtype = w_dtype;
    sp.G = 1;
    sp.N = E;
    sp.K = H;
    sp.offsets = nullptr;
    sp.out = workspace;
    sp.ldo = E;
    sp.swiglu = false;
    sp.mma_n = static_cast<int>((E + 31) / 32 * 32);
    sp.out_f32 = true;
    sp.k_splits = n_splits;
    sp.split_stride = T * E;
    rc = run_gemm(&sp, 1, x_dtype, status, s);
    if (rc) return rc;
    logits_in = static_cast<const float*>(workspace);
  }
  moe::route::Params p;
  p.n_splits = n_splits;
  p.x = x;
  p.w = router_w;
  p.logits_in = logits_in;
  p.bias = e_score_bias;
  p.topk_idx = topk_idx;
  p.topk_w = topk_w;
  p.logits_out = logits_out;
  p.status = status;
  p.T = T;
  p.H = H;
  p.E = static_cast<int>(E);
  p.k = k;
  p.mode = mode;
  p.renorm = renorm;
  p.n_group = n_group;
  p.topk_group = topk_group;
  p.x_dtype = x_dtype;
  p.w_dtype = w_dtype;
  p.scaling = routed_scaling;
  p.tb = route_tb(H, p.E, logits_in == nullptr);
  const size_t smem = static_cast<size_t>(p.tb) * (p.E + (logits_in ? 0 : H)) * sizeof(float);
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(moe::route::route_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    cudaFuncSetAttribute(moe::route::route_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    cudaFuncSetAttribute(moe::route::route_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
  });
  const int64_t grid = (T + p.tb - 1) / p.tb;
  // experts per lane in the selection: the fewest that cover E
  auto kernel = p.E <= 64 ? moe::route::route_kernel<2> : p.E <= 128 ? moe::route::route_kernel<4>
                                                                        : moe::route::route_kernel<8>;
  CUDA_TRY(launch_pdl(kernel, dim3(static_cast<unsigned>(grid)), dim3(moe::route::kThreads), smem, s, p),
           "route_kernel launch");
  return MOE_OK;
}

size_t moe_group_workspace_bytes(int64_t T, int k, int64_t E) {
  const int64_t n = T * k;
  const int64_t chunks = (n + moe::group::kChunk - 1) / moe::group::kChunk;
  return static_cast<size_t>((chunks > 0 ? chunks : 1) * E) * sizeof(int32_t);
}

int moe_group_tokens(const void* topk_idx, int idx_dtype, const float* topk_w, int64_t T, int k, int64_t E,
                     int32_t* counts, int32_t* offsets, int32_t* pos, int64_t* sorted_token_idx,
                     float* sorted_weight, const void* x, int x_dtype, int64_t H, void* xs, int xs_dtype,
                     void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  CHECK_ARG(E >= 1 && E <= moe::group::kMaxE, "E=%lld must be in [1, %d]", (long long)E, moe::group::kMaxE);
  CHECK_ARG(k >= 1 && T >= 0, "bad T/k");
  CHECK_ARG(idx_dtype == MOE_DT_I32 || idx_dtype == MOE_DT_I64, "topk_idx must be int32 or int64");
  CHECK_ARG(counts && offsets && (pos || T == 0), "null output pointer");
  CHECK_ARG(!sorted_weight || topk_w, "sorted_weight needs topk_w");
  CHECK_ARG(workspace && workspace_bytes >= moe_group_workspace_bytes(T, k, E), "workspace too small");
  if (xs) {
    CHECK_ARG(x && H >= 8 && H % 8 == 0, "gather needs x and H a multiple of 8");
    CHECK_ARG(is16(xs_dtype), "xs dtype must be bf16 or f16");
    CHECK_ARG(x_dtype == MOE_DT_F32 || x_dtype == xs_dtype, "x dtype must be f32 or match xs");
    CHECK_ARG(aligned16(x) && aligned16(xs), "x/xs must be 16-byte aligned");
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n = T * k;
  if (n == 0) {
    CUDA_TRY(cudaMemsetAsync(counts, 0, E * sizeof(int32_t), s), "memset counts");
    CUDA_TRY(cudaMemsetAsync(offsets, 0, (E + 1) * sizeof(int32_t), s), "memset offsets");
    return MOE_OK;
  }
  moe::group::Params p;
  p.idx = topk_idx;
  p.idx64 = idx_dtype == MOE_DT_I64;
  p.w = topk_w;
  p.n = n;
  p.k = k;
  p.E = static_cast<int>(E);
  p.nchunks = static_cast<int>((n + moe::group::kChunk - 1) / moe::group::kChunk);
  p.counts = counts;
  p.offsets = offsets;
  p.pos = pos;
  p.sorted_token_idx = sorted_token_idx;
  p.sorted_weight = sorted_weight;
  p.x = x;
  p.x_dtype = x_dtype;
  p.H = H;
  p.xs = xs;
  p.xs_f16 = xs_dtype == MOE_DT_F16;
  p.hist = static_cast<int32_t*>(workspace);
  p.status = status;
  return launch_grouping(p, sms, s);
}

}  // extern "C"

// ---------------------------------------------------------------- no-allocation grouping
// Scratch of moe_group_tokens_noalloc: the per-chunk expert histograms live in
// this fixed array of the library's device image instead of a caller buffer.
// Every device that loads the library holds these 1 MiB until the process exits.
static __device__ __align__(256) int32_t g_group_scratch[MOE_GROUP_NOALLOC_SCRATCH_INTS];

namespace {
std::mutex g_scratch_mu;
std::array<int32_t*, kMaxDevices> g_scratch{};

// Device address of g_group_scratch on the current device. On the host the
// symbol name is only a stand-in, so the address is looked up per device,
// with that device current, and kept once a lookup has succeeded; a failed
// lookup (say, one attempted during a stream capture) is reported and tried
// again on the next call.
int group_scratch(int32_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(MOE_ERR_NO_DEVICE, "no CUDA device is current");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_group_scratch);
    if (e != cudaSuccess || p == nullptr) return cuda_fail(e, "cudaGetSymbolAddress(group scratch)");
    g_scratch[dev] = static_cast<int32_t*>(p);
  }
  *out = g_scratch[dev];
  return MOE_OK;
}
}  // namespace

extern "C" {

int moe_group_tokens_noalloc(const void* topk_idx, int idx_dtype, const float* topk_w, int64_t T, int k, int64_t E,
                             int32_t* counts, int32_t* offsets, int32_t* pos, int64_t* sorted_token_idx,
                             float* sorted_weight, const void* x, int x_dtype, int64_t H, void* xs, int xs_dtype,
                             int32_t* status, void* stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  CHECK_ARG(E >= 1 && E <= moe::group::kMaxE, "E=%lld must be in [1, %d]", (long long)E, moe::group::kMaxE);
  CHECK_ARG(k >= 1 && T >= 0, "bad T/k");
  const int64_t n = T * k;
  const int64_t chunks = (n + moe::group::kChunk - 1) / moe::group::kChunk;
  CHECK_ARG(chunks * E <= MOE_GROUP_NOALLOC_SCRATCH_INTS,
            "moe_group_tokens_noalloc: ceil(T*k/256)*E = %lld exceeds the built-in scratch of %d int32 "
            "(T*k=%lld, E=%lld); use moe_group_tokens with a caller workspace",
            (long long)(chunks * E), MOE_GROUP_NOALLOC_SCRATCH_INTS, (long long)n, (long long)E);
  CHECK_ARG(idx_dtype == MOE_DT_I32 || idx_dtype == MOE_DT_I64, "topk_idx must be int32 or int64");
  CHECK_ARG(counts && offsets && (pos || T == 0), "null output pointer");
  CHECK_ARG(!sorted_weight || topk_w, "sorted_weight needs topk_w");
  if (xs) {
    CHECK_ARG(x && H >= 8 && H % 8 == 0, "gather needs x and H a multiple of 8");
    CHECK_ARG(is16(xs_dtype), "xs dtype must be bf16 or f16");
    CHECK_ARG(x_dtype == MOE_DT_F32 || x_dtype == xs_dtype, "x dtype must be f32 or match xs");
    CHECK_ARG(aligned16(x) && aligned16(xs), "x/xs must be 16-byte aligned");
  }
  int32_t* scratch = nullptr;
  rc = group_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n == 0) {
    CUDA_TRY(cudaMemsetAsync(counts, 0, E * sizeof(int32_t), s), "memset counts");
    CUDA_TRY(cudaMemsetAsync(offsets, 0, (E + 1) * sizeof(int32_t), s), "memset offsets");
    return MOE_OK;
  }
  moe::group::Params p;
  p.idx = topk_idx;
  p.idx64 = idx_dtype == MOE_DT_I64;
  p.w = topk_w;
  p.n = n;
  p.k = k;
  p.E = static_cast<int>(E);
  p.nchunks = static_cast<int>(chunks);
  p.counts = counts;
  p.offsets = offsets;
  p.pos = pos;
  p.sorted_token_idx = sorted_token_idx;
  p.sorted_weight = sorted_weight;
  p.x = x;
  p.x_dtype = x_dtype;
  p.H = H;
  p.xs = xs;
  p.xs_f16 = xs_dtype == MOE_DT_F16;
  // The histogram kernel writes every scratch entry the scatter kernel reads,
  // so the scratch needs no clearing between calls.
  p.hist = scratch;
  p.status = status;
  return launch_grouping(p, sms, s);
}

int moe_grouped_gemm(const void* a, int a_dtype, int64_t M, int64_t K, const void* w, int w_dtype,
                     const void* scale, int scale_dtype, int64_t E, int64_t N, const int32_t* offsets, void* out,
                     int64_t ldo, int32_t* status, void* stream) {
  CHECK_ARG(offsets, "null group offsets");
  if (M == 0) return MOE_OK;
  CHECK_ARG(ldo >= N, "ldo < N");
  SegSpec sp{};
  sp.a = a;
  sp.a_rows = M;
  sp.lda = K;
  sp.b0 = w;
  sp.b_dtype = w_dtype;
  sp.scale0 = scale;
  sp.scale_dtype = scale_dtype;
  sp.G = E;
  sp.N = N;
  sp.K = K;
  sp.offsets = offsets;
  sp.out = out;
  sp.ldo = ldo;
  sp.swiglu = false;
  return run_gemm(&sp, 1, a_dtype, status, static_cast<cudaStream_t>(stream));
}

size_t moe_ffn_workspace_bytes(int64_t R, int64_t I, int64_t T_shared, int64_t I_shared) {
  auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
  return up(static_cast<size_t>(R) * I * 2) + up(static_cast<size_t>(T_shared) * I_shared * 2);
}

int moe_expert_ffn_part(int part, const void* xs, int act_dtype, int64_t R, int64_t H, const int32_t* offsets,
                        int64_t E, int64_t I, const void* gate, const void* up, const void* down, int w_dtype,
                        const void* gate_scale, const void* up_scale, const void* down_scale, int scale_dtype,
                        const void* x_shared, int64_t T_shared, int64_t I_shared, const void* shared_gate,
                        const void* shared_up, const void* shared_down, void* y, void* y_shared, void* workspace,
                        size_t workspace_bytes, int32_t* status, void* stream) {
  return moe_expert_ffn_grouped(part, xs, act_dtype, R, H, offsets, E, E, nullptr, 0, I, gate, up, down, w_dtype,
                                gate_scale, up_scale, down_scale, scale_dtype, x_shared, T_shared, I_shared,
                                shared_gate, shared_up, shared_down, y, y_shared, workspace, workspace_bytes, status,
                                stream);
}

// Automatic FFN kernel choice: the streaming kernel for the gate/up
// projection when the routed groups average at most this many rows and the
// shared expert has at most this many. Measured on B200, C2 gate/up launch
// (tiled -> streaming with two chains): T=1 54.4 -> 35.8 us, T=16 128.1 ->
// 123.5 us, T=128 141.8 -> 175.8 us.
constexpr int64_t kStreamMaxAvgRows = 2;
constexpr int64_t kStreamMaxSharedRows = 32;
// AUTO takes the warp-MMA kernel for int8 weights with H or I beyond this
// only for launches of at most kWarpI8WideMaxRows routed rows.
constexpr int64_t kWarpI8MaxK = 4096;
constexpr int64_t kWarpI8WideMaxRows = 8;

// Where the routed down projection stores its rows: y, or scattered through
// a table of (possibly peer) return buffers.
struct RoutedOut {
  const int32_t* rows = nullptr;
  void* const* table = nullptr;
  int table_n = 0;
  int64_t table_rows = 0;
};

// The kernel MOE_FFN_KERNEL_AUTO runs for one expert-FFN call (both
// projections): R routed rows in G groups, a shared expert over T_shared rows
// (0: none), hidden size H, intermediate size I, weight dtype w_dtype.
//  - Decode-sized batches (routed groups averaging at most kStreamMaxAvgRows
//    rows, a shared expert of at most kStreamMaxSharedRows): the warp-MMA
//    kernel (C2 layer as a CUDA graph on B200, against the streaming gate/up
//    + tiled down: T=1 81 -> 71 us, T=4 137 -> 117 us, T=16 209 -> 190 us;
//    slower from T=64 on). int8: an int8 stage holds half the weight bytes of
//    a 16-bit one. C3 (H 2048, I 1408) layer graphs, warp-MMA / tiled /
//    streaming, us: T=1 81 / 117 / 105, T=16 254 / 268 / 298, T=32 329 / 313
//    / 366; C5 (H 7168, I 2048): T=1 283 / 295 / 344, T=2 408 / 385 / 462,
//    T=8 1244 / 1051 / 1387. So with K beyond kWarpI8MaxK the warp-MMA kernel
//    only for about one token's rows; the streaming kernel, slower than one
//    of the others at every point measured, never.
//  - The CTA-pair kernel (16-bit weights) for groups of prefill size whose
//    last 256-row tile is not nearly empty, judged from the average group.
//    Both tcgen05 kernels are bound by shared-memory traffic per k-block,
//    which a tile pays whatever its row count (B200, C2 T=4096, per-CTA cycle
//    counters): 771 cycles per k-block on one SM for a 128-row tile, 661 per
//    SM of a CTA pair for up to 256 token rows; so the pair kernel gains
//    where its tiles are full and loses where a group's last tile holds a few
//    rows. C2 layer graphs, tiled / pair, us (average group r): T=1024 (96)
//    287 / 309, T=2048 (192) 426 / 405, T=3072 (288) 593 / 620, T=4096 (384)
//    715-736 / 677-717, T=6144 (576) 1016 / 1026, T=8192 (768) 1290 / 1239.
//  - Else the tiled kernel. Gathered rows (TMA tile::gather4) only run there.
static int ffn_auto_kernel(int64_t R, int64_t G, int64_t T_shared, int64_t H, int64_t I, int w_dtype, bool gather) {
  if (gather) return MOE_FFN_KERNEL_TILED;
  const bool has_shared = T_shared > 0;
  const bool small = (R == 0 || R <= kStreamMaxAvgRows * G) && (!has_shared || T_shared <= kStreamMaxSharedRows);
  const bool wide_i8 = w_dtype == MOE_DT_I8 && (H > kWarpI8MaxK || I > kWarpI8MaxK);
  if (small && (!wide_i8 || R <= kWarpI8WideMaxRows)) return MOE_FFN_KERNEL_WARP;
  const int64_t avg_group = R > 0 ? (R + G - 1) / G : T_shared;
  const int64_t tail = avg_group % 256;
  if (w_dtype != MOE_DT_I8 && avg_group >= 160 && (tail == 0 || tail >= 96)) return MOE_FFN_KERNEL_PAIR;
  return MOE_FFN_KERNEL_TILED;
}

static int ffn_impl(int part, const void* xs, int act_dtype, int64_t R, int64_t H, const int32_t* offsets, int64_t G,
                    int64_t E, const int64_t* gather_rows, int64_t gather_src_rows, int64_t I, const void* gate,
                    const void* up, const void* down, int w_dtype, const void* gate_scale, const void* up_scale,
                    const void* down_scale, int scale_dtype, const void* x_shared, int64_t T_shared,
                    int64_t I_shared, const void* shared_gate, const void* shared_up, const void* shared_down,
                    void* y, void* y_shared, void* workspace, size_t workspace_bytes, int32_t* status,
                    void* stream, const RoutedOut& ro) {
  CHECK_ARG(part >= 1 && part <= 3, "part must be 1 (gate/up), 2 (down) or 3 (both)");
  CHECK_ARG(E >= 1 && G >= E && G % E == 0, "groups G=%lld must be a positive multiple of the experts E=%lld",
            (long long)G, (long long)E);
  CHECK_ARG(!gather_rows || gather_src_rows >= 1, "gathered rows need the source row count");
  const bool has_shared = T_shared > 0 && x_shared;
  CHECK_ARG(workspace && workspace_bytes >= moe_ffn_workspace_bytes(R, I, has_shared ? T_shared : 0, I_shared),
            "workspace too small");
  CHECK_ARG(R == 0 || offsets, "null group offsets");
  if (has_shared) CHECK_ARG(shared_gate && shared_up && shared_down && y_shared && I_shared > 0, "shared expert args");
  auto up256 = [](size_t b) { return (b + 255) & ~size_t(255); };
  void* h = workspace;
  void* hs = static_cast<char*>(workspace) + up256(static_cast<size_t>(R) * I * 2);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  SegSpec g1[2];
  SegSpec g2[2];
  int n = 0;
  if (R > 0) {
    SegSpec a{};
    a.a = xs; a.a_rows = R; a.lda = H; a.b0 = gate; a.b1 = up; a.b_dtype = w_dtype; a.scale0 = gate_scale;
    a.scale1 = up_scale; a.scale_dtype = scale_dtype; a.G = G; a.Gw = E; a.N = I; a.K = H; a.offsets = offsets;
    a.out = h; a.ldo = I; a.swiglu = true;
    a.gather_rows = gather_rows;
    a.gather_src_rows = gather_src_rows;
    SegSpec b{};
    b.a = h; b.a_rows = R; b.lda = I; b.b0 = down; b.b_dtype = w_dtype; b.scale0 = down_scale;
    b.scale_dtype = scale_dtype; b.G = G; b.Gw = E; b.N = H; b.K = I; b.offsets = offsets; b.out = y; b.ldo = H;
    b.swiglu = false;
    b.out_rows = ro.rows; b.out_table = ro.table; b.out_table_n = ro.table_n; b.out_table_rows = ro.table_rows;
    g1[n] = a;
    g2[n] = b;
    ++n;
  }
  if (has_shared) {
    SegSpec a{};
    a.a = x_shared; a.a_rows = T_shared; a.lda = H; a.b0 = shared_gate; a.b1 = shared_up; a.b_dtype = act_dtype;
    a.G = 1; a.N = I_shared; a.K = H; a.offsets = nullptr; a.out = hs; a.ldo = I_shared; a.swiglu = true;
    SegSpec b{};
    b.a = hs; b.a_rows = T_shared; b.lda = I_shared; b.b0 = shared_down; b.b_dtype = act_dtype; b.G = 1;
    b.N = H; b.K = I_shared; b.offsets = nullptr; b.out = y_shared; b.ldo = H; b.swiglu = false;
    g1[n] = a;
    g2[n] = b;
    ++n;
  }
  if (n == 0) return MOE_OK;
  // Kernel choice (every choice gives the same bits): the forced one, or
  // ffn_auto_kernel's; STREAM runs the streaming kernel for both projections.
  const int choice = g_ffn_kernel.load();
  const bool streamable = !gather_rows;
  CHECK_ARG(choice != MOE_FFN_KERNEL_STREAM || streamable, "the streaming kernel does not take gathered rows");
  CHECK_ARG(choice != MOE_FFN_KERNEL_WARP || streamable, "the warp-MMA kernel takes no gathered rows");
  CHECK_ARG(choice != MOE_FFN_KERNEL_PAIR || (streamable && w_dtype != MOE_DT_I8),
            "the CTA-pair kernel takes 16-bit weights and no gathered rows");
  const int pick = choice == MOE_FFN_KERNEL_AUTO
                       ? ffn_auto_kernel(R, G, has_shared ? T_shared : 0, H, I, w_dtype, gather_rows != nullptr)
                       : choice;
  const bool warp_mma = pick == MOE_FFN_KERNEL_WARP;
  const bool stream1 = pick == MOE_FFN_KERNEL_STREAM;
  const bool stream2 = pick == MOE_FFN_KERNEL_STREAM;
  const bool pair = pick == MOE_FFN_KERNEL_PAIR;
  // row tile per segment for the streaming kernel: about the rows a group
  // holds (routed: the average per group; shared: all of its rows), in [32, 256]
  auto row_tile = [](int64_t rows) { return rows <= 32 ? 32 : rows <= 64 ? 64 : rows <= 128 ? 128 : 256; };
  int nts[2];
  {
    int i = 0;
    if (R > 0) nts[i++] = row_tile((R + G - 1) / G);
    if (has_shared) nts[i++] = row_tile(T_shared);
  }
  int64_t avg_rows[2] = {1, 1};  // rows of the average group per segment (warp-MMA token tile)
  {
    int i = 0;
    if (R > 0) avg_rows[i++] = (R + G - 1) / G;
    if (has_shared) avg_rows[i++] = T_shared;
  }
  auto launch = [&](const SegSpec* g, bool stream_it) {
    if (warp_mma) return run_gemm_warp(g, n, avg_rows, act_dtype, status, s);
    if (stream_it) return run_gemm_stream(g, nts, n, act_dtype, status, s);
    if (pair) return run_gemm_pair(g, n, act_dtype, status, s);
    return run_gemm(g, n, act_dtype, status, s);
  };
  if (part & 1) {
    int rc = launch(g1, stream1);
    if (rc) return rc;
  }
  if (part & 2) return launch(g2, stream2);
  return MOE_OK;
}

int moe_expert_ffn_grouped(int part, const void* xs, int act_dtype, int64_t R, int64_t H, const int32_t* offsets,
                           int64_t G, int64_t E, const int64_t* gather_rows, int64_t gather_src_rows, int64_t I,
                           const void* gate, const void* up, const void* down, int w_dtype, const void* gate_scale,
                           const void* up_scale, const void* down_scale, int scale_dtype, const void* x_shared,
                           int64_t T_shared, int64_t I_shared, const void* shared_gate, const void* shared_up,
                           const void* shared_down, void* y, void* y_shared, void* workspace, size_t workspace_bytes,
                           int32_t* status, void* stream) {
  return ffn_impl(part, xs, act_dtype, R, H, offsets, G, E, gather_rows, gather_src_rows, I, gate, up, down, w_dtype,
                  gate_scale, up_scale, down_scale, scale_dtype, x_shared, T_shared, I_shared, shared_gate, shared_up,
                  shared_down, y, y_shared, workspace, workspace_bytes, status, stream, RoutedOut{});
}

int moe_expert_ffn(const void* xs, int act_dtype, int64_t R, int64_t H, const int32_t* offsets, int64_t E,
                   int64_t I, const void* gate, const void* up, const void* down, int w_dtype,
                   const void* gate_scale, const void* up_scale, const void* down_scale, int scale_dtype,
                   const void* x_shared, int64_t T_shared, int64_t I_shared, const void* shared_gate,
                   const void* shared_up, const void* shared_down, void* y, void* y_shared, void* workspace,
                   size_t workspace_bytes, int32_t* status, void* stream) {
  return moe_expert_ffn_part(3, xs, act_dtype, R, H, offsets, E, I, gate, up, down, w_dtype, gate_scale, up_scale,
                             down_scale, scale_dtype, x_shared, T_shared, I_shared, shared_gate, shared_up,
                             shared_down, y, y_shared, workspace, workspace_bytes, status, stream);
}

int moe_combine(const void* y, int y_dtype, const int32_t* pos, const float* topk_w, int64_t T, int k,
                int64_t H, const void* y_shared, void* out, int out_dtype, int32_t* status, void* stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  CHECK_ARG(k >= 1 && k <= moe::combine::kMaxK, "top_k=%d must be in [1, %d]", k, moe::combine::kMaxK);
  CHECK_ARG(H % 8 == 0, "H=%lld must be a multiple of 8", (long long)H);
  CHECK_ARG(y_dtype == MOE_DT_BF16 || y_dtype == MOE_DT_F16 || y_dtype == MOE_DT_F32, "bad y dtype");
  CHECK_ARG(out_dtype == MOE_DT_BF16 || out_dtype == MOE_DT_F16 || out_dtype == MOE_DT_F32, "bad out dtype");
  if (T == 0) return MOE_OK;  // nothing to combine (empty tensors may come with null pointers)
  CHECK_ARG(out && y && pos && topk_w, "null pointer");
  CHECK_ARG(aligned16(y) && aligned16(out) && aligned16(y_shared), "y/out must be 16-byte aligned");
  moe::combine::Params p;
  p.y = y;
  p.y_shared = y_shared;
  p.pos = pos;
  p.w = topk_w;
  p.out = out;
  p.T = T;
  p.H = H;
  p.k = k;
  p.y_dtype = y_dtype;
  p.out_dtype = out_dtype;
  p.status = status;
  const int64_t per = moe::combine::kThreads / 32;
  // Slices of 256 columns per warp: enough warps to cover the GPU (~32 per SM),
  // but no more, so large batches keep one warp per token.
  const int64_t slices = (H + 255) / 256;
  int64_t spw = (T * slices) / (static_cast<int64_t>(sms) * 64);
  spw = spw < 1 ? 1 : (spw > slices ? slices : spw);
  const int64_t units = T * ((slices + spw - 1) / spw);
  CUDA_TRY(launch_pdl(moe::combine::combine_kernel, dim3(static_cast<unsigned>((units + per - 1) / per)),
                      dim3(moe::combine::kThreads), 0, static_cast<cudaStream_t>(stream), p, static_cast<int>(spw)),
           "combine_kernel launch");
  return MOE_OK;
}

int moe_quantize_int8(const void* w, int w_dtype, int64_t rows, int64_t K, int8_t* q, void* scale,
                      int scale_dtype, void* stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  CHECK_ARG(w && q && scale, "null pointer");
  CHECK_ARG(w_dtype == MOE_DT_BF16 || w_dtype == MOE_DT_F16 || w_dtype == MOE_DT_F32, "bad weight dtype");
  CHECK_ARG(scale_dtype == MOE_DT_F32 || scale_dtype == MOE_DT_BF16, "bad scale dtype");
  if (rows == 0 || K == 0) return MOE_OK;
  moe::combine::QuantParams p;
  p.w = w;
  p.q = q;
  p.scale = scale;
  p.rows = rows;
  p.K = K;
  p.w_dtype = w_dtype;
  p.scale_bf16 = scale_dtype == MOE_DT_BF16;
  const int64_t per = moe::combine::kThreads / 32;
  CUDA_TRY(launch_pdl(moe::combine::quantize_kernel, dim3(static_cast<unsigned>((rows + per - 1) / per)),
                      dim3(moe::combine::kThreads), 0, static_cast<cudaStream_t>(stream), p),
           "quantize_kernel launch");
  return MOE_OK;
}

// ------------------------------------------------------------------ layer
namespace {
struct LayerWs {
  size_t idx, w, logits, counts, offsets, pos, xs, y, ys, group, ffn, total;
};
LayerWs layer_ws(const MoeLayerDesc* d) {
  auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
  LayerWs l{};
  const size_t T = static_cast<size_t>(d->T), R = T * d->k;
  const bool shared = d->I_shared > 0;
  size_t o = 0;
  l.idx = o; o += up(R * 4);
  l.logits = o; o += up(moe_route_workspace_bytes(d->T, d->E));
  l.w = o; o += up(R * 4);
  l.counts = o; o += up(static_cast<size_t>(d->E) * 4);
  l.offsets = o; o += up(static_cast<size_t>(d->E + 1) * 4);
  l.pos = o; o += up(R * 4);
  l.xs = o; o += up(R * d->H * 2);
  l.y = o; o += up(R * d->H * 2);
  l.ys = o; o += shared ? up(T * d->H * 2) : 0;
  l.group = o; o += up(moe_group_workspace_bytes(d->T, d->k, d->E));
  l.ffn = o; o += up(moe_ffn_workspace_bytes(static_cast<int64_t>(R), d->I, shared ? d->T : 0, d->I_shared));
  l.total = o;
  return l;
}
}  // namespace

size_t moe_layer_workspace_bytes(const MoeLayerDesc* d) { return d ? layer_ws(d).total : 0; }

}  // extern "C"

// ---------------------------------------------------------------- decode fork of the shared expert
namespace {
// The shared expert of a one-token layer call runs on a second stream,
// beside the router, the grouping and the routed FFN that it does not depend
// on, instead of inside the routed FFN's launches after them: each
// projection is then a long K-ordered chain of small MMAs on few SMs, and the
// two chains overlap instead of adding up. Same kernels, same bits. C2 layer
// as a CUDA graph on B200 (forked vs in the routed launches): T=1 84.8 vs
// 94.8 us; T=4 147 vs 141, T=16 222 vs 214, T=32 266 vs 245 us -- with more
// tokens the two launches' tiles no longer fit beside each other.
constexpr int64_t kSharedForkMaxT = 1;

struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
std::mutex g_side_mu;  // held while a call records and waits on the events
std::array<SideStream, kMaxDevices> g_side{};

// The current device's side stream and events, created on first use (call
// the layer once before capturing it in a CUDA graph). Caller holds g_side_mu.
int side_stream(SideStream** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(MOE_ERR_NO_DEVICE, "no CUDA device is current");
  SideStream& ss = g_side[dev];
  if (ss.s == nullptr) {
    SideStream n;
    cudaError_t e = cudaStreamCreateWithFlags(&n.s, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&n.fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&n.join, cudaEventDisableTiming);
    if (e != cudaSuccess) {
      if (n.join) cudaEventDestroy(n.join);
      if (n.fork) cudaEventDestroy(n.fork);
      if (n.s) cudaStreamDestroy(n.s);
      return cuda_fail(e, "side stream for the shared expert");
    }
    ss = n;
  }
  *out = &ss;
  return MOE_OK;
}
}  // namespace

extern "C" {

int moe_layer_forward(const MoeLayerDesc* d, const void* x, const void* router_w, const float* e_score_bias,
                      const int32_t* topk_idx_in, const float* topk_w_in, const void* gate, const void* up,
                      const void* down, const void* gate_scale, const void* up_scale, const void* down_scale,
                      const void* shared_gate, const void* shared_up, const void* shared_down, void* out,
                      int32_t* topk_idx, float* topk_w, int32_t* counts, int32_t* offsets, void* workspace,
                      size_t workspace_bytes, int32_t* status, void* stream) {
  CHECK_ARG(d && x && out, "null pointer");
  CHECK_ARG(is16(d->act_dtype), "act dtype must be bf16 or f16");
  CHECK_ARG(d->x_dtype == d->act_dtype || d->x_dtype == MOE_DT_F32, "x dtype must be f32 or the act dtype");
  const LayerWs l = layer_ws(d);
  CHECK_ARG(workspace && workspace_bytes >= l.total, "workspace too small (%zu < %zu)", workspace_bytes, l.total);
  if (d->T == 0) return MOE_OK;
  char* ws = static_cast<char*>(workspace);
  const bool shared = d->I_shared > 0;
  CHECK_ARG(!shared || d->x_dtype == d->act_dtype, "the shared expert needs x in the activation dtype");
  void* ys = shared ? ws + l.ys : nullptr;
  // Decode: the shared expert forks onto the side stream first (it reads
  // only x); the combine waits for it.
  const size_t routed_ffn_bytes = moe_ffn_workspace_bytes(d->T * d->k, d->I, 0, 0);
  std::unique_lock<std::mutex> side_lock;
  SideStream* side = nullptr;
  if (shared && d->T <= kSharedForkMaxT) {
    side_lock = std::unique_lock<std::mutex>(g_side_mu);
    int rc = side_stream(&side);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    CUDA_TRY(cudaEventRecord(side->fork, s), "cudaEventRecord(fork)");
    CUDA_TRY(cudaStreamWaitEvent(side->s, side->fork, 0), "cudaStreamWaitEvent(side)");
    rc = moe_expert_ffn_grouped(3, nullptr, d->act_dtype, 0, d->H, nullptr, 1, 1, nullptr, 0, d->I, gate, up, down,
                                d->w_dtype, nullptr, nullptr, nullptr, d->scale_dtype, x, d->T, d->I_shared,
                                shared_gate, shared_up, shared_down, nullptr, ys, ws + l.ffn + routed_ffn_bytes,
                                moe_ffn_workspace_bytes(0, d->I, d->T, d->I_shared), status, side->s);
    if (rc) return rc;
    CUDA_TRY(cudaEventRecord(side->join, side->s), "cudaEventRecord(join)");
  }
  int32_t* idx = topk_idx ? topk_idx : reinterpret_cast<int32_t*>(ws + l.idx);
  float* wts = topk_w ? topk_w : reinterpret_cast<float*>(ws + l.w);
  int32_t* cnt = counts ? counts : reinterpret_cast<int32_t*>(ws + l.counts);
  int32_t* off = offsets ? offsets : reinterpret_cast<int32_t*>(ws + l.offsets);
  int32_t* pos = reinterpret_cast<int32_t*>(ws + l.pos);
  void* xs = ws + l.xs;
  void* y = ws + l.y;
  int rc;
  if (topk_idx_in) {
    CHECK_ARG(topk_w_in, "topk_w_in missing");
    idx = const_cast<int32_t*>(topk_idx_in);
    wts = const_cast<float*>(topk_w_in);
  } else {
    rc = moe_route(x, d->x_dtype, router_w, d->router_w_dtype, nullptr, d->T, d->H, d->E, d->k, d->router_mode,
                   d->renorm, e_score_bias, d->n_group, d->topk_group, d->routed_scaling, idx, wts, nullptr,
                   ws + l.logits, moe_route_workspace_bytes(d->T, d->E), status, stream);
    if (rc) return rc;
  }
  // The grouping kernel writes the gathered rows xs (16-byte copies, f32 x
  // converted on the way). Gathering inside the GEMM with TMA tile::gather4
  // is supported (moe_expert_ffn_grouped with gather_rows) and bit-identical,
  // but 128 one-row TMA requests per k-block made the gate/up GEMM 2.5x
  // slower on B200, so the layer keeps the copy.
  const bool gather = false;
  int64_t* sti = gather ? reinterpret_cast<int64_t*>(xs) : nullptr;
  rc = moe_group_tokens(idx, MOE_DT_I32, wts, d->T, d->k, d->E, cnt, off, pos, sti, nullptr, gather ? nullptr : x,
                        d->x_dtype, d->H, gather ? nullptr : xs, d->act_dtype, ws + l.group,
                        moe_group_workspace_bytes(d->T, d->k, d->E), status, stream);
  if (rc) return rc;
  // The shared expert (unless forked above) runs in the routed FFN's launches;
  // it reads x directly, so it needs x in the activation type.
  const bool fused_shared = shared && side == nullptr;
  rc = moe_expert_ffn_grouped(3, gather ? x : xs, d->act_dtype, d->T * d->k, d->H, off, d->E, d->E, sti,
                              gather ? d->T : 0, d->I, gate, up, down, d->w_dtype, gate_scale, up_scale, down_scale,
                              d->scale_dtype, fused_shared ? x : nullptr, fused_shared ? d->T : 0, d->I_shared,
                              shared_gate, shared_up, shared_down, y, fused_shared ? ys : nullptr, ws + l.ffn,
                              moe_ffn_workspace_bytes(d->T * d->k, d->I, fused_shared ? d->T : 0, d->I_shared),
                              status, stream);
  if (rc) return rc;
  if (side) CUDA_TRY(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), side->join, 0), "cudaStreamWaitEvent(join)");
  return moe_combine(y, d->act_dtype, pos, wts, d->T, d->k, d->H, ys, out, d->out_dtype, status, stream);
}


// ----------------------------------------------------------------------------
// Expert-parallel peer exchange (include/moe_ep_b200.h)

static_assert(sizeof(cudaIpcMemHandle_t) == MOE_PEER_HANDLE_BYTES, "IPC handle size");

int moe_peer_alloc(size_t bytes, void** ptr) {
  CHECK_ARG(ptr && bytes > 0, "null pointer or zero size");
  *ptr = nullptr;
  void* p = nullptr;
  CUDA_TRY(cudaMalloc(&p, bytes), "cudaMalloc(peer buffer)");
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "cudaMemset(peer buffer)");
  }
  *ptr = p;
  return MOE_OK;
}

int moe_peer_free(void* ptr) {
  if (!ptr) return MOE_OK;
  CUDA_TRY(cudaFree(ptr), "cudaFree(peer buffer)");
  return MOE_OK;
}

int moe_peer_export(const void* ptr, void* handle) {
  CHECK_ARG(ptr && handle, "null pointer");
  cudaIpcMemHandle_t h;
  CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  return MOE_OK;
}

int moe_peer_import(const void* handle, void** ptr) {
  CHECK_ARG(handle && ptr, "null pointer");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return MOE_OK;
}

int moe_peer_release(void* ptr) {
  if (!ptr) return MOE_OK;
  CUDA_TRY(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
  return MOE_OK;
}

int moe_peer_can_access(int peer) {
  int dev = 0, ok = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (peer == dev) return 1;
  if (cudaDeviceCanAccessPeer(&ok, dev, peer) != cudaSuccess) return 0;
  return ok ? 1 : 0;
}

int moe_ep_dispatch(const void* x, int x_dtype, int64_t T, int64_t H, const void* topk_idx, int idx_dtype, int k,
                    const int32_t* pos, const int32_t* offsets, const int32_t* counts_all, int rank, int world,
                    int64_t E, void* const* peer_recv, int32_t* const* peer_ret, int64_t recv_cap,
                    int32_t* recv_offsets, int32_t* status, void* stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  CHECK_ARG(world >= 1 && world <= MOE_EP_MAX_RANKS && rank >= 0 && rank < world, "rank %d / world %d out of range",
            rank, world);
  CHECK_ARG(E >= world && E <= moe::ep::kMaxE && E % world == 0,
            "E=%lld must be a multiple of world=%d and at most %d", (long long)E, world, moe::ep::kMaxE);
  CHECK_ARG(is16(x_dtype), "x must be bf16 or f16");
  CHECK_ARG(idx_dtype == MOE_DT_I32 || idx_dtype == MOE_DT_I64, "topk_idx must be int32 or int64");
  CHECK_ARG(k >= 1 && T >= 0 && H % 8 == 0 && H > 0, "bad T/H/k");
  CHECK_ARG(T * k < (int64_t(1) << 27), "T*k=%lld exceeds the return code's 2^27 rows", (long long)(T * k));
  CHECK_ARG(recv_cap >= 0 && recv_cap < (int64_t(1) << 31), "recv_cap out of range");
  CHECK_ARG(counts_all && peer_recv && peer_ret && recv_offsets, "null pointer");
  CHECK_ARG(T == 0 || (x && topk_idx && pos && offsets), "null pointer");
  CHECK_ARG(aligned16(x), "x must be 16-byte aligned");
  moe::ep::DispatchParams p;
  p.x = x;
  p.H = H;
  p.idx = topk_idx;
  p.idx64 = idx_dtype == MOE_DT_I64;
  p.n = T * k;
  p.k = k;
  p.pos = pos;
  p.offsets = offsets;
  p.counts_all = counts_all;
  p.rank = rank;
  p.world = world;
  p.E = static_cast<int>(E);
  p.e_loc = static_cast<int>(E / world);
  p.peer_recv = peer_recv;
  p.peer_ret = peer_ret;
  p.recv_cap = recv_cap;
  p.recv_offsets = recv_offsets;
  p.status = status;
  // at least one CTA so this rank's receive offsets are written even with no tokens
  const int64_t chunks = p.n > 0 ? (p.n + moe::ep::kChunk - 1) / moe::ep::kChunk : 1;
  unsigned split = 1;
  const int64_t per_row = H / 8;
  while (split < 32 && chunks * split < 2 * sms && per_row % (2 * split) == 0 && per_row / (2 * split) >= 8)
    split *= 2;
  CUDA_TRY(launch_pdl(moe::ep::dispatch_kernel, dim3(static_cast<unsigned>(chunks), split), dim3(moe::ep::kThreads),
                      0, static_cast<cudaStream_t>(stream), p),
           "dispatch_kernel launch");
  return MOE_OK;
}

int moe_ep_expert_ffn(const void* recv, int act_dtype, int64_t recv_cap, int64_t H, const int32_t* recv_offsets,
                      int64_t E_loc, const int32_t* recv_ret, void* const* peer_back, int world, int64_t back_rows,
                      int64_t I, const void* gate, const void* up, const void* down, int w_dtype,
                      const void* gate_scale, const void* up_scale, const void* down_scale, int scale_dtype,
                      const void* x_shared, int64_t T_shared, int64_t I_shared, const void* shared_gate,
                      const void* shared_up, const void* shared_down, void* y_shared, void* workspace,
                      size_t workspace_bytes, int32_t* status, void* stream) {
  CHECK_ARG(world >= 1 && world <= MOE_EP_MAX_RANKS, "world %d out of range", world);
  CHECK_ARG(recv_cap == 0 || (recv && recv_ret && peer_back && back_rows > 0), "null receive/return buffers");
  RoutedOut ro;
  ro.rows = recv_ret;
  ro.table = peer_back;
  ro.table_n = world;
  ro.table_rows = back_rows;
  return ffn_impl(3, recv, act_dtype, recv_cap, H, recv_offsets, E_loc, E_loc, nullptr, 0, I, gate, up, down,
                  w_dtype, gate_scale, up_scale, down_scale, scale_dtype, x_shared, T_shared, I_shared, shared_gate,
                  shared_up, shared_down, nullptr, y_shared, workspace, workspace_bytes, status, stream, ro);
}


static_assert(MOE_EP_SIGNAL_HEADER_BYTES == moe::ep::kSignalHeader && MOE_EP_FLAG_SLOTS == moe::ep::kFlagSlots,
              "signal buffer layout");

size_t moe_ep_signal_bytes(int world, int64_t n) {
  if (world < 1 || n < 0) return 0;
  return MOE_EP_SIGNAL_HEADER_BYTES + static_cast<size_t>(world) * static_cast<size_t>(n) * sizeof(int32_t);
}

int moe_ep_exchange(const int32_t* payload, int64_t n, void* const* peer_signal, int32_t* local_signal,
                    size_t signal_bytes, int slot, int rank, int world, int32_t epoch, int32_t* status,
                    void* stream) {
  int sms = 0;
  int rc = device_info(&sms);
  if (rc) return rc;
  CHECK_ARG(world >= 1 && world <= MOE_EP_MAX_RANKS && rank >= 0 && rank < world, "rank %d / world %d out of range",
            rank, world);
  CHECK_ARG(slot >= 0 && slot < MOE_EP_FLAG_SLOTS, "flag slot %d not in [0, %d)", slot, MOE_EP_FLAG_SLOTS);
  CHECK_ARG(n >= 0 && (n == 0 || payload), "payload of %lld int32 needs a pointer", (long long)n);
  CHECK_ARG(peer_signal && local_signal, "null signal buffer");
  CHECK_ARG(moe_ep_signal_bytes(world, n) <= signal_bytes,
            "signal buffers of %zu bytes cannot hold the header and a (%d, %lld) int32 payload (%zu bytes)",
            signal_bytes, world, (long long)n, moe_ep_signal_bytes(world, n));
  moe::ep::ExchangeParams p;
  p.payload = payload;
  p.n = n;
  p.peer_signal = peer_signal;
  p.local_signal = local_signal;
  p.slot = slot;
  p.rank = rank;
  p.world = world;
  p.epoch = epoch;
  p.status = status;
  CUDA_TRY(launch_pdl(moe::ep::exchange_kernel, dim3(1), dim3(256), 0, static_cast<cudaStream_t>(stream), p),
           "exchange_kernel launch");
  return MOE_OK;
}

}  // extern "C"
