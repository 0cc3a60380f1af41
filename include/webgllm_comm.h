/*
 * webgllm_comm.h: tensor-parallel exchange for libwebgllm_b200.so — a
 * one-shot push all-reduce over NVLink peer memory, fused into the
 * row-parallel matmul that produces the partial sums.
 *
 * No reference counterpart: webgllm runs a model on one device. This is the
 * exchange of the 8B-shape config split across the GPUs of one node
 * (o and down projections are row parallel: each rank holds a K slice and
 * produces a partial [M][N] that must be summed across ranks). NCCL's
 * all-reduce does the same in a separate launch; here the matmul's own
 * epilogue stores its partial into every rank's exchange buffer (P2P
 * stores of 64-bit words, each carrying its value and the exchange's
 * sequence number, so no flag or fence orders them); wg_comm_reduce polls
 * its local buffer until every word carries the expected sequence number
 * (at most 2 s by default, wg_comm_set_wait, then WG_TIMEOUT from wg_sync)
 * and sums the partials.
 *
 * Setup, per rank (one process per GPU): wg_ipc_alloc a buffer, exchange
 * the 64-byte handles (e.g. an all-gather over torch.distributed),
 * wg_ipc_open every peer's handle, then wg_comm_init with the world's
 * buffers in rank order (this rank's own at index rank). Every rank must
 * issue the same sequence of wg_q4_matmul_push / wg_comm_reduce pairs.
 */
#ifndef WEBGLLM_COMM_H
#define WEBGLLM_COMM_H

#include <stddef.h>

#include "webgllm_q4.h"

#ifdef __cplusplus
extern "C" {
#endif

#define WG_IPC_HANDLE_BYTES 64

typedef struct wg_comm wg_comm;

/* A zeroed device buffer of `bytes` that peers can map; handle receives its
 * WG_IPC_HANDLE_BYTES-byte CUDA IPC handle. */
int wg_ipc_alloc(wg_ctx *ctx, size_t bytes, void **dptr, void *handle);
int wg_ipc_free(wg_ctx *ctx, void *dptr);
/* Maps a peer's buffer into this context's device. */
int wg_ipc_open(wg_ctx *ctx, const void *handle, void **dptr);
int wg_ipc_close(wg_ctx *ctx, void *dptr);

/* An exchange over `world` (<= 8) ranks' buffers of `bytes` each
 * (buffers[rank] is this rank's own). The caller keeps owning the buffers
 * and mappings. */
int wg_comm_init(wg_ctx *ctx, int world, int rank, void *const *buffers, size_t bytes, wg_comm **out);
int wg_comm_destroy(wg_ctx *ctx, wg_comm *comm);
/* How long a consumer (wg_comm_reduce, wg_comm_reduce_norm) waits for a
 * peer's partial before it gives up: wait_ns nanoseconds (default 2 s, the
 * value wg_comm_init sets). A wait that runs out makes the next wg_sync
 * return WG_TIMEOUT; the launch ends after about one wait (the words still
 * missing read as 0) and the context stays usable. The limit applies to
 * launches enqueued after the call (a CUDA graph keeps the value it was
 * captured with). Replaces the reference's context-loss detection
 * (GpuError, src/gpu/gl.ts:502; classified in src/worker-errors.ts:14-24). */
int wg_comm_set_wait(wg_comm *comm, unsigned long long wait_ns);

/* Floats one rank's partial may hold (M * N of a pushing matmul). */
int wg_comm_slot(const wg_comm *comm, size_t *floats);

/* y_partial = x . W^T (x as wg_q4_matmul, or made by `pro` as
 * wg_q4_matmul_fused when pro is not NULL), pushed into every rank's
 * exchange buffer instead of being stored. M <= 32 (the decode GEMV). */
int wg_q4_matmul_push(wg_ctx *ctx, const wg_q4mat *m, const wg_prologue *pro, const void *x, int x_dtype, int M,
                      wg_comm *comm);

/* out fp32 [M][N] = the sum over ranks of the next exchange's partials
 * (waits for every rank's push). */
int wg_comm_reduce(wg_ctx *ctx, wg_comm *comm, int M, int N, float *out);

/* The exchange fused with what consumes it in a decoder layer: v = resid +
 * (the sum over ranks of the next exchange's partials, M x K), resid_out =
 * v (if not NULL; must not alias resid), x_out fp16 = rmsnorm(v) * weight —
 * the all-reduce, the residual add and the next RMS norm in one launch
 * (addNormed, src/engine.ts:5695), one thread-block cluster per row. */
int wg_comm_reduce_norm(wg_ctx *ctx, wg_comm *comm, int M, int K, const float *resid, const float *weight, float eps,
                        float *resid_out, void *x_out);

/* ------------------------------------------------------------------------
 * The tensor-parallel group: NCCL behind the C ABI, so that a host without
 * PyTorch (the reference's TypeScript host through a Node-API addon) can
 * join a group, all-reduce and set up the push exchange. The reference runs
 * one worker per model (src/client.ts:64); here one process per GPU joins a
 * group of `nranks` with wg_tp_init(ctx, nranks, rank, id), the 128-byte
 * NCCL unique id made by one rank. NCCL is loaded on first use (dlopen of libnccl.so.2,
 * or the path in WG_NCCL_LIBRARY): a process that already loaded it shares
 * that copy, and the library still loads where NCCL is absent (these calls
 * then return WG_UNSUPPORTED).
 *
 * Bootstrap: one rank calls wg_tp_unique_id, the caller sends those
 * WG_TP_ID_BYTES bytes to every rank by any transport (a worker message, a
 * file, a store), and every rank calls wg_tp_init with its rank. Every rank
 * must then issue the same collectives in the same order. */
#define WG_TP_ID_BYTES 128

/* all-reduce element types and operations */
enum { WG_TP_F32 = 0, WG_TP_F16 = 1, WG_TP_BF16 = 2, WG_TP_I64 = 3 };
enum { WG_TP_SUM = 0, WG_TP_MAX = 1 };

typedef struct wg_tp wg_tp;

/* A new group id (ncclGetUniqueId) into id[WG_TP_ID_BYTES]. */
int wg_tp_unique_id(void *id);
/* Joins the group `id` as `rank` of `nranks` on ctx's device (blocks until
 * every rank has joined). */
int wg_tp_init(wg_ctx *ctx, int nranks, int rank, const void *id, wg_tp **out);
/* Leaves the group (after the ctx's stream has drained). */
int wg_tp_destroy(wg_ctx *ctx, wg_tp *tp);
int wg_tp_info(const wg_tp *tp, int *nranks, int *rank);
/* In-place all-reduce of `count` elements on ctx's stream (WG_TP_SUM of
 * f32 / f16 / bf16, WG_TP_MAX of i64): the row-parallel sums of prompt
 * rows and the vocabulary-parallel greedy pick. Can be captured in a CUDA
 * graph with the rest of a step. */
int wg_tp_allreduce(wg_ctx *ctx, wg_tp *tp, void *buf, size_t count, int dtype, int op);
/* Every rank reaches this point: a one-word all-reduce, waited for on the
 * host for at most timeout_ms (0: 60 s). If a rank never arrives, the group
 * is aborted (ncclCommAbort) and WG_TIMEOUT returned; the group is then
 * unusable (wg_tp_destroy it) while the context stays usable. */
int wg_tp_barrier(wg_ctx *ctx, wg_tp *tp, int timeout_ms);
/* The push exchange (wg_q4_matmul_push / wg_comm_reduce) over this group:
 * allocates this rank's buffer of `bytes`, all-gathers the IPC handles
 * through NCCL, maps every peer's buffer and returns the communicator.
 * wg_comm_destroy of such a communicator also unmaps the peers' buffers
 * and frees this rank's (with a barrier of the group before each, so it
 * is a collective call). */
int wg_tp_comm(wg_ctx *ctx, wg_tp *tp, size_t bytes, wg_comm **out);

#ifdef __cplusplus
}
#endif

#endif
