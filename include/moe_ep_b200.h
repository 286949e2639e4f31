/*
 * moe_ep_b200.h -- C ABI of the expert-parallel peer exchange (one process
 * per GPU, GPUs of one NVSwitch box).
 *
 * Replaces the DeepEP V1 Buffer round trip that the reference wires into its
 * grouped-GEMM path -- buffer.get_dispatch_layout / buffer.dispatch /
 * buffer.combine in make_ep_moe_infer (src/dispatch/kernels/expert_parallel.py:
 * 119-190) -- with direct NVLink stores between the ranks' device buffers:
 *
 *   dispatch  every (token, slot) row is written by the source GPU straight
 *             into the receive buffer of the rank that owns its expert
 *             (moe_ep_dispatch), at the row the full count matrix assigns it;
 *   FFN       the owner runs the grouped SwiGLU FFN over its receive buffer,
 *             and the down projection's epilogue stores each output row
 *             straight back into the source rank's return buffer
 *             (moe_ep_expert_ffn);
 *   combine   the source rank sums its k returned rows per token in slot
 *             order (moe_combine of moe_b200.h).
 *
 * No row is staged through a send buffer and nothing is synchronised with the
 * host: the only collectives are an all-gather of the (E,) per-expert counts
 * and two stream-ordered barriers, each one moe_ep_exchange launch over the
 * ranks' signal buffers (an NCCL all-gather and all-reduce serve as well).
 * Peer memory is plain CUDA IPC (cudaIpcGetMemHandle / cudaIpcOpenMemHandle):
 * no multicast object, no TMA multicast load.
 *
 * Receive layout on the rank that owns experts [rank*E_loc, (rank+1)*E_loc):
 * local expert j's rows are contiguous, j-major; inside a block the rows come
 * in source-rank order, and in a source's stable (token, slot) order. Each
 * received row q carries a return code ret[q] = (p << 4) | source_rank, p its
 * row in the source's expert-sorted order (the `pos` of moe_group_tokens).
 *
 * Unlike moe_b200.h, the moe_peer_* calls allocate and map device memory;
 * they are set-up calls, made once per buffer, outside any stream capture.
 */
#ifndef MOE_EP_B200_H_
#define MOE_EP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_PEER_HANDLE_BYTES 64 /* size of an exported handle (cudaIpcMemHandle_t) */
#define MOE_EP_MAX_RANKS 16      /* the return code keeps the source rank in 4 bits */

/*
 * Peer-shareable device memory. moe_peer_alloc: `bytes` on the current device
 * (cudaMalloc; zero-filled). moe_peer_export writes the handle of a pointer
 * returned by moe_peer_alloc; moe_peer_import maps another process's handle
 * into this one (peer access enabled on first use) and moe_peer_release unmaps
 * it; moe_peer_free frees an allocation. No reference counterpart (DeepEP
 * allocates its NVL buffers inside Buffer.__init__, deep_ep/buffer.py, a
 * third-party dependency of the reference).
 */
int moe_peer_alloc(size_t bytes, void** ptr);
int moe_peer_free(void* ptr);
int moe_peer_export(const void* ptr, void* handle);
int moe_peer_import(const void* handle, void** ptr);
int moe_peer_release(void* ptr);
/* 1 if the current device can map device `peer`'s memory, else 0. */
int moe_peer_can_access(int peer);

/*
 * Dispatch. Replaces buffer.get_dispatch_layout + buffer.dispatch
 * (src/dispatch/kernels/expert_parallel.py:159-168).
 *
 * x (T, H) 16-bit activations of this rank; topk_idx (T, k) int32/int64 global
 * expert ids; pos (T*k) and offsets (E+1) from moe_group_tokens of the same
 * ids on this rank; counts_all (world, E) int32 = every rank's per-expert
 * counts (the all-gather of moe_group_tokens' counts), identical on all ranks.
 * peer_recv / peer_ret: device arrays of `world` pointers, entry d = rank d's
 * receive rows (recv_cap, H) and return codes (recv_cap) int32, as mapped in
 * this process (this rank's own entry is its local buffer). Writes this rank's
 * rows and return codes into the owners' buffers and, on this rank,
 * recv_offsets (E/world + 1) int32 = group offsets of the rows this rank will
 * receive. A row index at or past recv_cap raises MOE_ERR_BAD_OFFSETS in the
 * status word and is not written. Every thread fences its peer stores at
 * system scope before the kernel ends; the caller then issues a barrier over
 * the ranks before any rank reads its receive buffer.
 */
int moe_ep_dispatch(const void* x, int x_dtype, int64_t T, int64_t H, const void* topk_idx, int idx_dtype, int k,
                    const int32_t* pos, const int32_t* offsets, const int32_t* counts_all, int rank, int world,
                    int64_t E, void* const* peer_recv, int32_t* const* peer_ret, int64_t recv_cap,
                    int32_t* recv_offsets, int32_t* status, void* stream);

/*
 * Expert FFN on the received rows with the return stores fused into the down
 * projection. Replaces local_expert_contribution + buffer.combine's transfer
 * (src/dispatch/kernels/expert_parallel.py:44-86, 170-187).
 *
 * recv (recv_cap, H) and recv_ret (recv_cap) are this rank's receive buffers,
 * recv_offsets (E_loc + 1) the offsets moe_ep_dispatch wrote; gate/up/down
 * hold the E_loc local experts (layouts, int8 scales and the shared expert as
 * moe_expert_ffn; the shared expert runs on x_shared (T_shared, H) in the same
 * launches and writes y_shared locally). Output row q (unweighted) is stored
 * at row ret[q] >> 4 of peer_back[ret[q] & 15], a device array of `world`
 * pointers to the ranks' return buffers (back_rows, H) of the activation type;
 * a code outside [0, world) x [0, back_rows) raises MOE_ERR_BAD_OFFSETS and is
 * skipped. Workspace: moe_ffn_workspace_bytes(recv_cap, I, T_shared, I_shared).
 * As for the dispatch, the peer stores are fenced at system scope and the
 * caller issues a barrier before the sources combine.
 */
int moe_ep_expert_ffn(const void* recv, int act_dtype, int64_t recv_cap, int64_t H, const int32_t* recv_offsets,
                      int64_t E_loc, const int32_t* recv_ret, void* const* peer_back, int world, int64_t back_rows,
                      int64_t I, const void* gate, const void* up, const void* down, int w_dtype,
                      const void* gate_scale, const void* up_scale, const void* down_scale, int scale_dtype,
                      const void* x_shared, int64_t T_shared, int64_t I_shared, const void* shared_gate,
                      const void* shared_up, const void* shared_down, void* y_shared, void* workspace,
                      size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Stream-ordered exchange and barrier over the ranks' signal buffers, in
 * place of the NCCL all-gather and barriers around the dispatch and the FFN
 * (the synchronisation DeepEP's Buffer does inside dispatch/combine,
 * src/dispatch/kernels/expert_parallel.py:160-187).
 *
 * A signal buffer (moe_ep_signal_bytes, from moe_peer_alloc, zero at
 * allocation) holds MOE_EP_FLAG_SLOTS rows of MOE_EP_MAX_RANKS int32 flags
 * in its first MOE_EP_SIGNAL_HEADER_BYTES, then a (world, n) int32 payload
 * area. `signal_bytes` is the size of every rank's signal buffer (all ranks
 * allocate the same size); a payload that does not fit, i.e.
 * moe_ep_signal_bytes(world, n) > signal_bytes, is refused with
 * MOE_ERR_INVALID_ARG before anything is stored into peer memory.
 * One launch (a single CTA) on this rank: copies `payload` (n int32, may
 * be 0) into row `rank` of every rank's payload area, fences at system scope,
 * stores `epoch` into flag [slot][rank] of every rank (release), then waits
 * until flags [slot][0..world) of its own buffer are >= epoch (acquire).
 * Kernels enqueued after it see every rank's stores made before that rank's
 * exchange. Every rank makes the same calls with the same epoch, which grows
 * by one per layer call. The wait is bounded (2 s): on expiry it sets
 * MOE_ERR_TIMEOUT in the status word and returns.
 */
#define MOE_EP_SIGNAL_HEADER_BYTES 256
#define MOE_EP_FLAG_SLOTS 4
size_t moe_ep_signal_bytes(int world, int64_t n);
int moe_ep_exchange(const int32_t* payload, int64_t n, void* const* peer_signal, int32_t* local_signal,
                    size_t signal_bytes, int slot, int rank, int world, int32_t epoch, int32_t* status,
                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_EP_B200_H_ */
