// comm.h -- the library's NCCL communicator (one process per GPU), opened at run time so that
// libacb needs NCCL only when a caller shards a job. Every wait on peers is bounded: NCCL runs in
// non-blocking mode, the host polls the communicator's state and the stream against a deadline,
// and on a timeout aborts the communicator and returns ACB_ERR_TIMEOUT.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#include "../../include/acb_models.h"

struct acb_comm;

namespace acb {

// out[world * bytes] = every rank's in[bytes] in rank order (ncclAllGather); enqueued on stream
acb_status comm_all_gather(acb_comm * c, const void * in, void * out, size_t bytes, cudaStream_t stream);
// send `bytes` to peer and receive as many from it (one grouped ncclSend / ncclRecv)
acb_status comm_exchange(acb_comm * c, int peer, const void * send, void * recv, size_t bytes, cudaStream_t stream);
// wait for everything enqueued on stream (bounded by the communicator's timeout)
acb_status comm_wait(acb_comm * c, cudaStream_t stream);
int        comm_rank(const acb_comm * c);
int        comm_world(const acb_comm * c);

}  // namespace acb
