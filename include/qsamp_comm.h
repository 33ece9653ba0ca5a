/* qsamp_comm.h -- the candidate exchange of vocab-sharded selection over
 * NCCL, with failure detection (libqsamp_comm.so; separate from
 * libqsamp.so so that the selection library does not depend on NCCL).
 *
 * No counterpart in the reference: its sampler sees whole rows
 * (src/sampling/sampling.cpp:158-163) and its server has only a request
 * timeout and a cancel flag (inference_server.h:170,319-334). A
 * tensor-parallel output head splits the vocabulary over GPUs; each rank runs
 * qsamp_shard_topk, the ranks exchange their [B][k] candidate blocks with
 * qsamp_comm_allgather_candidates, and every rank runs qsamp_merge_topk
 * (include/qsamp.h).
 *
 * Failure detection. The communicator is non-blocking
 * (ncclCommInitRankConfig with blocking = 0). Every wait -- for the
 * communicator to initialise, for a collective to be enqueued, and
 * qsamp_comm_wait for the stream's work to complete -- polls the
 * communicator's asynchronous error (ncclCommGetAsyncError) against the
 * communicator's deadline. An asynchronous error or a deadline that passes
 * (a rank that never joins, a peer that died) aborts the communicator
 * (ncclCommAbort, which also ends its collectives in flight on the GPU) and
 * the call returns QSAMP_ERR_COMM or QSAMP_ERR_TIMEOUT; every later call on
 * that communicator returns QSAMP_ERR_COMM, and the caller destroys it and
 * builds a new one. No call waits without a bound.
 *
 * Threading: a communicator is used from one host thread at a time.
 */
#ifndef QSAMP_COMM_H
#define QSAMP_COMM_H

#include <stddef.h>
#include <stdint.h>

#include "qsamp.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct qsamp_comm qsamp_comm;

#define QSAMP_COMM_ID_BYTES 128

/* A new unique id (ncclGetUniqueId); rank 0 makes it and every rank passes
 * the same bytes to qsamp_comm_create (the transport between the processes
 * is the caller's). */
qsamp_status qsamp_comm_unique_id(unsigned char id[QSAMP_COMM_ID_BYTES]);

/* Joins rank `rank` of `nranks` on CUDA device `device`; every later wait of
 * this communicator gives up after timeout_ms (> 0). err, when non-NULL,
 * receives a message of at most err_len bytes on failure. */
qsamp_status qsamp_comm_create(int32_t nranks, int32_t rank, const unsigned char id[QSAMP_COMM_ID_BYTES],
                               int32_t device, int64_t timeout_ms, qsamp_comm** out, char* err, size_t err_len);

/* Enqueues, on `stream` (a cudaStream_t), the all-gather of every rank's
 * candidate block: vals [per_rank] float and ids [per_rank] int32 (this
 * rank's [B][k]) into all_vals / all_ids [nranks][per_rank], rank-major --
 * the layout qsamp_merge_topk reads. Returns once the collectives are
 * enqueued (or the deadline passed); the caller continues on the stream and
 * calls qsamp_comm_wait before reading results on the host. */
qsamp_status qsamp_comm_allgather_candidates(qsamp_comm* comm, const float* vals, const int32_t* ids,
                                             int64_t per_rank, float* all_vals, int32_t* all_ids, void* stream);

/* Waits until the work enqueued on `stream` has completed, polling the
 * communicator's asynchronous error; on an error or when the deadline
 * passes, aborts the communicator (QSAMP_ERR_COMM / QSAMP_ERR_TIMEOUT). */
qsamp_status qsamp_comm_wait(qsamp_comm* comm, void* stream);

/* QSAMP_OK, or QSAMP_ERR_COMM once the communicator was aborted. */
qsamp_status qsamp_comm_status(const qsamp_comm* comm);
const char* qsamp_comm_last_error(const qsamp_comm* comm);
void qsamp_comm_destroy(qsamp_comm* comm);

/* The deadline logic run against a fake collective, with no GPU and no NCCL
 * call (a test of the failure path that hangs nothing): scenario 0 -- never
 * completes (expect QSAMP_ERR_TIMEOUT), 1 -- reports an asynchronous error
 * on its third poll (QSAMP_ERR_COMM), 2 -- completes on its third poll
 * (QSAMP_OK). *aborted tells whether the abort path ran. */
qsamp_status qsamp_comm_selftest(int32_t scenario, int64_t timeout_ms, int32_t* aborted);

#ifdef __cplusplus
}
#endif

#endif
