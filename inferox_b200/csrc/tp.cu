// Tensor parallelism: NCCL entry points resolved at run time, weight shards.
#include <dlfcn.h>

#include <cstring>
#include <mutex>
#include <string>

#include <chrono>
#include <thread>
#include <unordered_set>

#include "quant.cuh"
#include "tp.h"
#include "watchdog.h"

namespace ifx {

namespace {
std::mutex g_aborted_mu;
std::unordered_set<void *> g_aborted;  // communicators tp_wait aborted
std::once_flag g_nccl_once;
NcclApi g_nccl{};
std::string g_nccl_err;

template <typename F>
bool sym(void *h, const char *name, F *out) {
  *out = reinterpret_cast<F>(dlsym(h, name));
  return *out != nullptr;
}

void resolve() {
  // a libnccl.so.2 already in the process (the one whose communicators the
  // caller holds) comes first; otherwise load it by soname
  void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    g_nccl_err = std::string("libnccl.so.2 not found: ") + dlerror();
    return;
  }
  NcclApi a{};
  if (!(sym(h, "ncclGetUniqueId", &a.GetUniqueId) && sym(h, "ncclCommInitRank", &a.CommInitRank) &&
        sym(h, "ncclCommDestroy", &a.CommDestroy) && sym(h, "ncclAllReduce", &a.AllReduce) &&
        sym(h, "ncclAllGather", &a.AllGather) && sym(h, "ncclGetErrorString", &a.GetErrorString) &&
        sym(h, "ncclCommGetAsyncError", &a.CommGetAsyncError) && sym(h, "ncclCommAbort", &a.CommAbort))) {
    g_nccl_err = "libnccl.so.2 lacks an entry point the tensor-parallel path needs";
    return;
  }
  g_nccl = a;
}
}  // namespace

ifx_status nccl_api(const NcclApi **out) {
  std::call_once(g_nccl_once, resolve);
  if (!g_nccl.AllReduce) return fail(IFX_ERR_NCCL, g_nccl_err);
  *out = &g_nccl;
  return IFX_OK;
}

ifx_status nccl_fail(const NcclApi *api, ncclResult_t r, const char *what) {
  return fail(IFX_ERR_NCCL, std::string(what) + ": " + (api ? api->GetErrorString(r) : "error"));
}

bool tp_take_aborted(void *comm) {
  std::lock_guard<std::mutex> lk(g_aborted_mu);
  return g_aborted.erase(comm) > 0;
}

ifx_status tp_wait(cudaStream_t st, ncclComm_t comm, const NcclApi *api, double timeout_ms) {
  using clk = std::chrono::steady_clock;
  cudaError_t dev_err = cudaSuccess;
  ncclResult_t comm_err = ncclSuccess;
  auto query = [&]() {
    const cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return 0;
    if (e == cudaErrorNotReady) return 1;
    dev_err = e;
    return -1;
  };
  auto comm_error = [&]() {
    ncclResult_t r = ncclSuccess;
    if (api->CommGetAsyncError(comm, &r) != ncclSuccess) return false;
    if (r == ncclSuccess || r == ncclInProgress) return false;
    comm_err = r;
    return true;
  };
  auto abort = [&]() {
    {
      std::lock_guard<std::mutex> lk(g_aborted_mu);
      g_aborted.insert((void *)comm);
    }
    api->CommAbort(comm);
  };
  auto now_ms = []() {
    return std::chrono::duration<double, std::milli>(clk::now().time_since_epoch()).count();
  };
  // spin (yielding) through the first 50 ms, the length of any normal step,
  // then poll every 200 us
  const double t_spin = now_ms() + 50.0;
  auto pause = [&]() {
    if (now_ms() < t_spin) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(200));
  };
  const WaitEnd end = bounded_wait(query, comm_error, abort, now_ms, pause, timeout_ms);
  switch (end) {
    case WaitEnd::Done: return IFX_OK;
    case WaitEnd::DeviceError:
      return fail(IFX_ERR_CUDA, std::string("tensor-parallel step: ") + cudaGetErrorString(dev_err));
    case WaitEnd::CommError:
      return fail(IFX_ERR_NCCL, std::string("tensor-parallel step: a collective failed (") +
                                    api->GetErrorString(comm_err) +
                                    "); the communicator was aborted");
    case WaitEnd::TimedOut:
      break;
  }
  return fail(IFX_ERR_TIMEOUT, "tensor-parallel step: collectives did not finish within " +
                                   std::to_string((long long)timeout_ms) +
                                   " ms (a peer rank stopped?); the communicator was aborted");
}

ifx_status tp_shard(int type, const uint8_t *bytes, size_t nbytes, uint64_t rows, uint64_t cols,
                    int split_k, int tp, int rank, std::vector<uint8_t> *out) {
  const BlockInfo b = block_info(type);
  if (!b.elems) return fail(IFX_ERR_UNSUPPORTED, "tp_shard: unsupported tensor type");
  if (tp < 1 || rank < 0 || rank >= tp) return fail(IFX_ERR_INVALID_ARGUMENT, "tp_shard: bad rank");
  if (cols % b.elems) return fail(IFX_ERR_SHAPE, "tp_shard: row length is not whole blocks");
  const uint64_t row_bytes = cols / b.elems * b.bytes;
  if (rows * row_bytes > nbytes) return fail(IFX_ERR_UNEXPECTED_EOF, "tp_shard: tensor bytes short");
  if (!split_k) {
    if (rows % tp) return fail(IFX_ERR_SHAPE, "tp_shard: rows do not split evenly");
    const uint64_t r0 = rows / tp * rank, nr = rows / tp;
    out->assign(bytes + r0 * row_bytes, bytes + (r0 + nr) * row_bytes);
    return IFX_OK;
  }
  if (cols % ((uint64_t)tp * b.elems))
    return fail(IFX_ERR_SHAPE, "tp_shard: the input dimension does not split into whole blocks");
  const uint64_t part = row_bytes / tp;  // bytes of one row's slice
  out->resize(rows * part);
  for (uint64_t r = 0; r < rows; ++r)
    std::memcpy(out->data() + r * part, bytes + r * row_bytes + part * rank, part);
  return IFX_OK;
}

}  // namespace ifx
