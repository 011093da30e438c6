// Tensor parallelism: weight shards and the NCCL entry points.
//
// NCCL is not linked at build time. A communicator only works with the NCCL
// library instance that created it, and a process may hold one already
// (PyTorch ships its own), so the entry points are resolved at run time from
// the libnccl.so.2 already loaded in the process, or loaded by soname when
// there is none.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

#include <cuda_runtime.h>
#include <nccl.h>

#include "status.h"

namespace ifx {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId *);
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t);
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                            cudaStream_t);
  const char *(*GetErrorString)(ncclResult_t);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
  ncclResult_t (*CommAbort)(ncclComm_t);
};

// Resolves the entry points once per process.
ifx_status nccl_api(const NcclApi **out);
ifx_status nccl_fail(const NcclApi *api, ncclResult_t r, const char *what);

// Waits for `st` (work that includes collectives on `comm`) at most
// timeout_ms; on an asynchronous NCCL error or at the deadline aborts `comm`
// (its outstanding kernels end; the communicator is unusable afterwards)
// and returns IFX_ERR_NCCL / IFX_ERR_TIMEOUT.
ifx_status tp_wait(cudaStream_t st, ncclComm_t comm, const NcclApi *api, double timeout_ms);

// Whether tp_wait aborted `comm` (ncclCommAbort frees it, so it must not be
// destroyed again); take_aborted() also forgets it.
bool tp_take_aborted(void *comm);

#define IFX_NCCL(api, call)                                           \
  do {                                                                \
    const ncclResult_t r_ = (call);                                   \
    if (r_ != ncclSuccess) return ::ifx::nccl_fail((api), r_, #call); \
  } while (0)

// The shard of a GGUF-layout matrix [rows, cols] (rows stored contiguously,
// each row cols / block_elems blocks) held by `rank` of `tp`:
//  split_k = 0: rows [rank * rows / tp, (rank + 1) * rows / tp)   (column parallel)
//  split_k = 1: every row's columns [rank * cols / tp, ...)        (row parallel)
// The split must fall on whole rows / whole quantisation blocks.
ifx_status tp_shard(int type, const uint8_t *bytes, size_t nbytes, uint64_t rows, uint64_t cols,
                    int split_k, int tp, int rank, std::vector<uint8_t> *out);

}  // namespace ifx
