/*
 * moe_b200.h -- C ABI of the B200 (sm_100a) MoE-layer hot path.
 *
 * Every entry point takes raw device pointers, element counts and a CUDA
 * stream (as void*), enqueues its kernels on that stream and returns
 * MOE_OK or a MOE_ERR_* code. Nothing throws across the ABI and nothing
 * allocates: the caller owns every buffer, including workspaces sized by the
 * *_workspace_bytes() helpers. Errors found on the device (an expert id out
 * of range, a bounded wait that expired) are written to a caller-provided
 * int32 status word in device memory (first error wins; 0 = OK); the caller
 * reads it after synchronising. Calls are stream-ordered and thread-compatible:
 * one stream per call, no global mutable state apart from a per-device cache
 * of the SM count and the driver's tensor-map encoder, a per-device side
 * stream of moe_layer_forward (one-token calls), and the process-wide FFN
 * kernel choice of moe_set_ffn_kernel.
 *
 * Layouts (row-major, contiguous unless a leading dimension is passed):
 *   x            (T, H)        activations, bf16 / f16 / f32
 *   router_w     (E, H)        bf16 / f32
 *   gate, up     (E, I, H)     bf16 / f16, or int8 + per-channel scale (E, I)
 *   down         (E, H, I)     bf16 / f16, or int8 + scale (E, H)
 *   topk_idx     (T, k) int32, topk_w (T, k) f32
 *   group offsets (E + 1) int32 exclusive prefix sum of per-expert counts
 *   pos          (T * k) int32: grouped row of flat slot t*k+s
 *
 * Each entry point names the reference function it replaces
 * (bsreecharanreddy/dispatch, path relative to the project root).
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_B200_ABI_VERSION 1

/* status codes */
#define MOE_OK 0
#define MOE_ERR_INVALID_ARG 1   /* shapes, dtypes, alignment, null pointers */
#define MOE_ERR_UNSUPPORTED 2   /* a valid request this build does not implement */
#define MOE_ERR_CUDA 3          /* a CUDA runtime / driver call failed */
#define MOE_ERR_NO_DEVICE 4     /* no sm_100 device current */
#define MOE_ERR_TIMEOUT 5       /* device: a bounded wait expired (status word) */
#define MOE_ERR_BAD_EXPERT 6    /* device: an expert id outside [0, E) (status word) */
#define MOE_ERR_BAD_OFFSETS 7   /* device: group offsets / row positions out of range (status word) */

/* element types */
#define MOE_DT_BF16 0
#define MOE_DT_F16 1
#define MOE_DT_F32 2
#define MOE_DT_I8 3
#define MOE_DT_I32 4
#define MOE_DT_I64 5

/*
 * Which grouped-GEMM kernel the expert-FFN entry points (moe_expert_ffn,
 * moe_expert_ffn_part, moe_expert_ffn_grouped, moe_ep_expert_ffn,
 * moe_layer_forward) launch:
 *   MOE_FFN_KERNEL_TILED   128 token rows x 256 weight columns per tile
 *                          (prefill-sized groups);
 *   MOE_FFN_KERNEL_PAIR    256 weight rows x up to 256 token rows (a
 *                          multiple of 32) per tile on a pair of SMs (tcgen05
 *                          cta_group::2, each SM stages 128 weight rows and
 *                          half of the token rows); 16-bit weights only;
 *   MOE_FFN_KERNEL_STREAM  one or two blocks of 128 weight rows x a tile of
 *                          32 to 256 token rows, up to 12 stages of weights
 *                          in flight per SM (decode-sized groups);
 *   MOE_FFN_KERNEL_WARP    64 or 128 weight rows x 8 to 32 token rows per
 *                          tile, each warp of the CTA running its own chain
 *                          of warp-level MMAs (mma.sync) on TMA-staged
 *                          operands, two CTAs per SM (decode-sized groups);
 *                          int8 weights are converted in registers;
 *   MOE_FFN_KERNEL_AUTO    (default) when the routed groups average at most
 *                          2 rows and the shared expert has at most 32: WARP
 *                          for both projections (int8 weights with H or I
 *                          above 4096: only for at most 8 routed rows);
 *                          otherwise PAIR (16-bit weights) when the average
 *                          group has at least 160 rows and its last 256-row
 *                          tile is empty or holds at least 96 rows, else
 *                          TILED. STREAM only when forced.
 * Every kernel gives every row the same bits (same k-block order; the tensor
 * cores' result depends neither on operand orientation nor on the tile or
 * CTA-group shape), so the choice changes speed only. Process-wide; returns the previous choice, or -1 for an
 * unknown one (nothing changes). No reference counterpart: the reference's
 * tile size is the caller's block_m (src/dispatch/kernels/tile_schedule.py).
 */
#define MOE_FFN_KERNEL_AUTO 0
#define MOE_FFN_KERNEL_TILED 1
#define MOE_FFN_KERNEL_STREAM 2
#define MOE_FFN_KERNEL_PAIR 3
#define MOE_FFN_KERNEL_WARP 4
int moe_set_ffn_kernel(int choice);

/*
 * The kernel (MOE_FFN_KERNEL_WARP, _PAIR or _TILED) that AUTO runs for an
 * expert-FFN call with R routed rows in G groups (experts, or (rank, expert)
 * groups), a shared expert over T_shared rows (0: none), hidden size H,
 * intermediate size I and weight dtype w_dtype (MOE_DT_BF16 / _F16 / _I8),
 * without gathered rows. Host-only (no device, no allocation); for logs and
 * benchmarks that name the kernel they time. -1 for a negative size or G < 1.
 * No reference counterpart.
 */
int moe_ffn_kernel_auto(int64_t R, int64_t G, int64_t T_shared, int64_t H, int64_t I, int w_dtype);

/* router modes */
#define MOE_ROUTER_SOFTMAX 0        /* softmax top-k (optionally renormalised) */
#define MOE_ROUTER_SIGMOID_GROUP 1  /* DeepSeek-V3 group-limited sigmoid top-k */

int moe_abi_version(void);
const char* moe_status_string(int code);
/* Message of the last failing call on this host thread ("" if none). */
const char* moe_last_error(void);
/* Number of SMs of the current device (0 if none). */
int moe_device_sm_count(void);

/*
 * Router. Replaces ReferenceMoE.route (src/dispatch/kernels/reference_moe.py:56-61):
 * logits = x @ router_w^T (fp32 accumulate), then for MOE_ROUTER_SOFTMAX the
 * fp32 softmax and its top-k (ties to the lower expert id, slots in
 * descending order), renormalised to sum 1 when renorm != 0 (e_score_bias,
 * if non-NULL, is added to the logits first: a gate with bias); for
 * MOE_ROUTER_SIGMOID_GROUP the group-limited sigmoid selection with
 * e_score_bias (E floats, may be NULL), n_group / topk_group, renorm and
 * routed_scaling. When logits_in is non-NULL it is used instead of x/router_w
 * (x and router_w may then be NULL). With bf16/f16 x and a router weight of the
 * same type the logits are a dense tcgen05 GEMM, split along K into f32 partial
 * slabs in the workspace (moe_route_workspace_bytes; the selection sums the
 * slabs in a fixed order); otherwise (f32 inputs) a CUDA-core kernel computes
 * them and the workspace may be NULL. logits_out (T, E) f32, may be NULL,
 * receives the raw gate logits. H must be a multiple of 8.
 */
size_t moe_route_workspace_bytes(int64_t T, int64_t E);
int moe_route(const void* x, int x_dtype, const void* router_w, int w_dtype, const float* logits_in, int64_t T,
              int64_t H, int64_t E, int k, int mode, int renorm, const float* e_score_bias, int n_group,
              int topk_group, float routed_scaling, int32_t* topk_idx, float* topk_w, float* logits_out,
              void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Token grouping. Replaces group_tokens_by_expert
 * (src/dispatch/kernels/grouping.py:25-41) and the host-side prefix sum of
 * build_tile_schedule (src/dispatch/kernels/tile_schedule.py:28-50): a stable
 * counting sort of the T*k flat (token, slot) pairs by expert, entirely on the
 * device (no host sync). Outputs: counts (E) int32, offsets (E+1) int32,
 * pos (T*k) int32; optional (NULL to skip): sorted_token_idx (T*k) int64,
 * sorted_weight (T*k) f32 (needs topk_w), and the row gather
 * xs[pos[f]] = x[f / k] (xs (T*k, H) in xs_dtype, bf16 or f16; x in x_dtype).
 * topk_idx is int32 or int64 (idx_dtype). workspace: moe_group_workspace_bytes
 * (per-chunk histograms; needs no initialisation). A slot whose id is out of
 * range gets pos = -1 and MOE_ERR_BAD_EXPERT in the status word.
 */
size_t moe_group_workspace_bytes(int64_t T, int k, int64_t E);
int moe_group_tokens(const void* topk_idx, int idx_dtype, const float* topk_w, int64_t T, int k, int64_t E,
                     int32_t* counts, int32_t* offsets, int32_t* pos, int64_t* sorted_token_idx,
                     float* sorted_weight, const void* x, int x_dtype, int64_t H, void* xs, int xs_dtype,
                     void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Token grouping without a workspace argument. It has no counterpart in the
 * reference: it exists for callers that cannot allocate device memory, such
 * as a host runtime that binds this library over FFI and can only hand over
 * buffers it already owns, or code running where a cudaMalloc would stall the
 * device or is forbidden by a fixed memory plan. Same arguments, outputs and
 * kernels as moe_group_tokens; the per-chunk histograms go to a fixed array
 * compiled into the library (MOE_GROUP_NOALLOC_SCRATCH_INTS int32 = 1 MiB,
 * resident on every device that loads the library until the process exits).
 * Limit: ceil(T*k/256) * E <= MOE_GROUP_NOALLOC_SCRATCH_INTS (e.g. T*k up to
 * 262144 pairs with E = 256), else MOE_ERR_INVALID_ARG and nothing runs.
 * The first call on each device looks up the array's device address with that
 * device current; make that first call before any stream capture. All calls
 * on a device share the one array (nothing in it needs to start at zero), so
 * calls that overlap on the GPU -- concurrent streams, or host threads sharing
 * a device -- race and must be serialised by the caller.
 */
#define MOE_GROUP_NOALLOC_SCRATCH_INTS (256 * 1024)
int moe_group_tokens_noalloc(const void* topk_idx, int idx_dtype, const float* topk_w, int64_t T, int k, int64_t E,
                             int32_t* counts, int32_t* offsets, int32_t* pos, int64_t* sorted_token_idx,
                             float* sorted_weight, const void* x, int x_dtype, int64_t H, void* xs, int xs_dtype,
                             int32_t* status, void* stream);

/*
 * Grouped GEMM, the GroupedMatmul contract (src/dispatch/kernels/moe_forward.py:21,
 * grouped_matmul at src/dispatch/kernels/grouped_gemm.py:177-207):
 * out[rows of e] = a[rows of e] @ w[e]^T, rows of e = [offsets[e], offsets[e+1]).
 * a (M, K) bf16/f16, w (E, N, K) same type, out (M, ldo) same type, f32
 * accumulate on tcgen05 tensor cores. With w_dtype == MOE_DT_I8 this is
 * grouped_matmul_int8 (src/dispatch/kernels/grouped_gemm_int8.py:141-176): w is
 * int8, dequantised exactly to the activation type before the MMA, and
 * scale (E, N) (scale_dtype f32 or bf16) multiplies the accumulator after the
 * K loop. K must be a multiple of 8 (16 for int8); offsets live on the device.
 */
int moe_grouped_gemm(const void* a, int a_dtype, int64_t M, int64_t K, const void* w, int w_dtype,
                     const void* scale, int scale_dtype, int64_t E, int64_t N, const int32_t* offsets, void* out,
                     int64_t ldo, int32_t* status, void* stream);

/*
 * Expert FFN over grouped rows, the three GEMMs plus SwiGLU of
 * grouped_moe_routed (src/dispatch/kernels/moe_forward.py:65-68) fused into
 * two tcgen05 launches: h = silu(xs @ gate^T) * (xs @ up^T) with gate and up in
 * one N=2x128 tile and the activation in the epilogue, then y = h @ down^T.
 * Routed rows: xs (R, H), offsets (E+1), y (R, H). The optional shared expert
 * (src/dispatch/kernels/reference_moe.py:50-54,74-78) runs in the same
 * launches as one more group over all T rows of x_shared: shared_gate/up
 * (I_s, H), shared_down (H, I_s), y_shared (T, H). Pass NULL shared pointers
 * and T_shared = 0 to skip it. w_dtype is the routed weights' type (bf16, f16
 * or int8 with scales); the shared expert is always in the activation type.
 * workspace: moe_ffn_workspace_bytes (holds h).
 */
size_t moe_ffn_workspace_bytes(int64_t R, int64_t I, int64_t T_shared, int64_t I_shared);
int moe_expert_ffn(const void* xs, int act_dtype, int64_t R, int64_t H, const int32_t* offsets, int64_t E,
                   int64_t I, const void* gate, const void* up, const void* down, int w_dtype,
                   const void* gate_scale, const void* up_scale, const void* down_scale, int scale_dtype,
                   const void* x_shared, int64_t T_shared, int64_t I_shared, const void* shared_gate,
                   const void* shared_up, const void* shared_down, void* y, void* y_shared, void* workspace,
                   size_t workspace_bytes, int32_t* status, void* stream);
/* The same, one half at a time: part 1 = gate/up GEMM + SwiGLU (writes h into
 * the workspace), part 2 = down GEMM (reads h), part 3 = both. Lets a caller
 * time or overlap the two launches separately. */
int moe_expert_ffn_part(int part, const void* xs, int act_dtype, int64_t R, int64_t H, const int32_t* offsets,
                        int64_t E, int64_t I, const void* gate, const void* up, const void* down, int w_dtype,
                        const void* gate_scale, const void* up_scale, const void* down_scale, int scale_dtype,
                        const void* x_shared, int64_t T_shared, int64_t I_shared, const void* shared_gate,
                        const void* shared_up, const void* shared_down, void* y, void* y_shared, void* workspace,
                        size_t workspace_bytes, int32_t* status, void* stream);

/*
 * The expert FFN over G = R * E row groups for expert parallelism: group g
 * (offsets has G+1 entries) is multiplied by weight g % E, so rows received
 * from R source ranks in (source rank, local expert) order are processed where
 * they landed, with no regrouping copy. Replaces the local compute of
 * make_ep_moe_infer (src/dispatch/kernels/expert_parallel.py:170-178).
 * gather_rows (R int64, may be NULL): routed row r is read from row
 * gather_rows[r] of xs, which then has gather_src_rows rows -- the
 * x[sorted_token_idx] gather of moe_forward.py:72 done by the GEMM's TMA
 * (tile::gather4) instead of a copy. Other arguments as moe_expert_ffn_part;
 * with G == E and no gather it is moe_expert_ffn_part.
 */
int moe_expert_ffn_grouped(int part, const void* xs, int act_dtype, int64_t R, int64_t H, const int32_t* offsets,
                           int64_t G, int64_t E, const int64_t* gather_rows, int64_t gather_src_rows, int64_t I,
                           const void* gate, const void* up, const void* down, int w_dtype, const void* gate_scale,
                           const void* up_scale, const void* down_scale, int scale_dtype, const void* x_shared,
                           int64_t T_shared, int64_t I_shared, const void* shared_gate, const void* shared_up,
                           const void* shared_down, void* y, void* y_shared, void* workspace, size_t workspace_bytes,
                           int32_t* status, void* stream);

/*
 * Weighted combine / unpermute. Replaces ungroup_and_combine
 * (src/dispatch/kernels/grouping.py:44-61): out[t] = sum_s topk_w[t,s] *
 * y[pos[t*k+s]] (+ y_shared[t]), summed in slot order in f32 and rounded once
 * to out_dtype -- deterministic, unlike the reference's index_add_.
 * y, y_shared in y_dtype (bf16/f16/f32); y_shared may be NULL.
 */
int moe_combine(const void* y, int y_dtype, const int32_t* pos, const float* topk_w, int64_t T, int k,
                int64_t H, const void* y_shared, void* out, int out_dtype, int32_t* status, void* stream);

/*
 * Per-output-channel int8 quantisation. Replaces quantize_per_channel_int8
 * (src/dispatch/kernels/quantization.py:31-50): scale = absmax/127 in f32 (1 for
 * an all-zero channel), q = clamp(round_half_even(w / scale), -127, 127).
 * w (rows, K) in w_dtype (bf16/f16/f32), q (rows, K) int8, scale (rows) stored
 * as scale_dtype (f32, or bf16 rounded from the f32 value).
 */
int moe_quantize_int8(const void* w, int w_dtype, int64_t rows, int64_t K, int8_t* q, void* scale,
                      int scale_dtype, void* stream);

/*
 * Whole layer: route -> group + gather -> expert FFN -> combine, five
 * launches and no host synchronisation. Replaces ReferenceMoE.forward
 * (src/dispatch/kernels/reference_moe.py:74-78) and, with topk_in given, the
 * moe_infer closure of src/dispatch/kernels/integration.py:158-175.
 * If topk_idx_in/topk_w_in (int32 / f32, (T,k)) are non-NULL the router is
 * skipped. Outputs: out (T, H) in out_dtype; topk_idx/topk_w (T,k) (written by
 * the router, or copies of the inputs are not made: pass the same buffers),
 * counts (E), offsets (E+1) (all may be NULL except out).
 * With a shared expert and T = 1 the shared expert runs on a second stream
 * of the library's (one per device, made by the first such call: make it
 * before capturing the call in a CUDA graph), forked from `stream` with an
 * event and joined before the combine; host threads that call this on one
 * device at once take turns for that part of the enqueue.
 */
typedef struct MoeLayerDesc {
  int64_t T, H, E, I, I_shared;
  int k;
  int act_dtype;      /* bf16 or f16: the tensor-core input type */
  int x_dtype;        /* bf16, f16 or f32 */
  int out_dtype;      /* bf16, f16 or f32 */
  int w_dtype;        /* routed weights: act type or MOE_DT_I8 */
  int scale_dtype;    /* f32 or bf16 (int8 only) */
  int router_mode;    /* MOE_ROUTER_* */
  int renorm;
  int n_group, topk_group;
  float routed_scaling;
  int router_w_dtype; /* bf16 or f32 */
} MoeLayerDesc;

size_t moe_layer_workspace_bytes(const MoeLayerDesc* d);
int moe_layer_forward(const MoeLayerDesc* d, const void* x, const void* router_w, const float* e_score_bias,
                      const int32_t* topk_idx_in, const float* topk_w_in, const void* gate, const void* up,
                      const void* down, const void* gate_scale, const void* up_scale, const void* down_scale,
                      const void* shared_gate, const void* shared_up, const void* shared_down, void* out,
                      int32_t* topk_idx, float* topk_w, int32_t* counts, int32_t* offsets, void* workspace,
                      size_t workspace_bytes, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* MOE_B200_H_ */
