// group.cu — one process driving several GPUs of a node (osc_group_*): a
// context per GPU and an NCCL communicator clique among them, for batch-level
// inference sharded by image / row / sequence with the shards' outputs
// all-gathered over NVLink.
//
// The reference runs one Net per process on the CPU and has no multi-device
// path; its single-Net contract is that Forward() returns the whole batch's
// output (src/OnnxSharp/Core/Net.cs:258-262). A C# host keeps that contract
// over N GPUs by splitting the batch, replaying each GPU's captured plan on its
// shard and all-gathering the shards (osc_group_run_sharded), so every GPU —
// in particular the one the host reads from — holds the whole output.
//
// NCCL is opened at run time (dlopen of libnccl.so.2, the one the process has
// already loaded if any), so the library loads and every single-GPU entry
// works on a machine without NCCL; the group entries then return OSC_ENCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <vector>

#include "runtime.h"

namespace osc {
namespace {

struct NcclApi {
  decltype(&ncclCommInitAll) comm_init_all = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  std::string load_error;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) {
      const char* e = dlerror();
      api.load_error = e ? e : "libnccl.so.2 not found";
      return;
    }
    api.comm_init_all = reinterpret_cast<decltype(api.comm_init_all)>(dlsym(h, "ncclCommInitAll"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.group_start = reinterpret_cast<decltype(api.group_start)>(dlsym(h, "ncclGroupStart"));
    api.group_end = reinterpret_cast<decltype(api.group_end)>(dlsym(h, "ncclGroupEnd"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!api.comm_init_all || !api.comm_destroy || !api.all_gather || !api.all_reduce || !api.group_start ||
        !api.group_end || !api.error_string) {
      api.load_error = "libnccl.so.2 lacks a required symbol";
      api.comm_init_all = nullptr;
    }
  });
  return api;
}

int nccl_fail(ncclResult_t r, const char* what) {
  return fail(OSC_ENCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

#define OSC_NCCL(expr, what)                                   \
  do {                                                         \
    ncclResult_t _r = (expr);                                  \
    if (_r != ncclSuccess) return ::osc::nccl_fail(_r, what);  \
  } while (0)

}  // namespace
}  // namespace osc

struct osc_group {
  std::vector<osc_ctx*> ctx;
  std::vector<ncclComm_t> comms;
};

using namespace osc;

namespace {

int check_group(osc_group* g, const char* what) {
  if (g == nullptr || g->ctx.empty()) return fail(OSC_EINVAL, "%s: null group", what);
  if (nccl().comm_init_all == nullptr) return fail(OSC_ENCCL, "%s: NCCL unavailable (%s)", what, nccl().load_error.c_str());
  return OSC_OK;
}

}  // namespace

extern "C" {

OSC_API int osc_group_destroy(osc_group* g) {
  if (g == nullptr) return OSC_OK;
  for (osc_ctx* c : g->ctx)
    if (c != nullptr) {
      cudaSetDevice(c->device);
      cudaStreamSynchronize(c->stream);
    }
  if (nccl().comm_destroy != nullptr)
    for (ncclComm_t comm : g->comms)
      if (comm != nullptr) nccl().comm_destroy(comm);
  for (osc_ctx* c : g->ctx) osc_destroy(c);
  delete g;
  return OSC_OK;
}

OSC_API int osc_group_create(int ndev, const int* devices, osc_group** out) {
  if (out == nullptr) return fail(OSC_EINVAL, "osc_group_create: out is null");
  *out = nullptr;
  if (ndev < 1 || devices == nullptr) return fail(OSC_EINVAL, "osc_group_create: %d devices", ndev);
  if (fault_injected("create")) return fail(OSC_EFAULT_INJECTED, "injected failure (create)");
  for (int i = 0; i < ndev; ++i)
    for (int j = 0; j < i; ++j)
      if (devices[i] == devices[j]) return fail(OSC_EINVAL, "osc_group_create: device %d listed twice", devices[i]);
  if (nccl().comm_init_all == nullptr)
    return fail(OSC_ENCCL, "osc_group_create: NCCL unavailable (%s)", nccl().load_error.c_str());
  auto* g = new osc_group();
  for (int i = 0; i < ndev; ++i) {
    osc_ctx* c = nullptr;
    const int st = osc_create(devices[i], &c);
    if (st != OSC_OK) {
      osc_group_destroy(g);
      return st;
    }
    g->ctx.push_back(c);
  }
  g->comms.assign(ndev, nullptr);
  const ncclResult_t r = nccl().comm_init_all(g->comms.data(), ndev, devices);
  if (r != ncclSuccess) {
    g->comms.assign(ndev, nullptr);
    const int st = nccl_fail(r, "ncclCommInitAll");
    osc_group_destroy(g);
    return st;
  }
  *out = g;
  return OSC_OK;
}

OSC_API int osc_group_size(osc_group* g, int* n) {
  if (g == nullptr || n == nullptr) return fail(OSC_EINVAL, "osc_group_size: null argument");
  *n = static_cast<int>(g->ctx.size());
  return OSC_OK;
}

OSC_API int osc_group_ctx(osc_group* g, int rank, osc_ctx** out) {
  if (out == nullptr) return fail(OSC_EINVAL, "osc_group_ctx: out is null");
  *out = nullptr;
  if (g == nullptr || rank < 0 || rank >= static_cast<int>(g->ctx.size()))
    return fail(OSC_EINVAL, "osc_group_ctx: rank %d out of range", rank);
  *out = g->ctx[rank];
  return OSC_OK;
}

OSC_API int osc_group_allgather(osc_group* g, const void* const* send, void* const* recv, size_t bytes) {
  OSC_TRY(check_group(g, "osc_group_allgather"));
  if (send == nullptr || recv == nullptr) return fail(OSC_EINVAL, "osc_group_allgather: null pointer array");
  const int n = static_cast<int>(g->ctx.size());
  for (int r = 0; r < n; ++r)
    if (send[r] == nullptr || recv[r] == nullptr) return fail(OSC_EINVAL, "osc_group_allgather: null buffer (rank %d)", r);
  if (bytes == 0) return OSC_OK;
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  OSC_NCCL(nccl().group_start(), "ncclGroupStart");
  for (int r = 0; r < n; ++r) {
    const ncclResult_t e = nccl().all_gather(send[r], recv[r], bytes, ncclUint8, g->comms[r], g->ctx[r]->stream);
    if (e != ncclSuccess) {
      nccl().group_end();
      return nccl_fail(e, "ncclAllGather");
    }
  }
  OSC_NCCL(nccl().group_end(), "ncclGroupEnd (all-gather)");
  return OSC_OK;
}

OSC_API int osc_group_allreduce_minmax(osc_group* g, float* const* minmax) {
  OSC_TRY(check_group(g, "osc_group_allreduce_minmax"));
  if (minmax == nullptr) return fail(OSC_EINVAL, "osc_group_allreduce_minmax: null pointer array");
  const int n = static_cast<int>(g->ctx.size());
  for (int r = 0; r < n; ++r)
    if (minmax[r] == nullptr) return fail(OSC_EINVAL, "osc_group_allreduce_minmax: null buffer (rank %d)", r);
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  OSC_NCCL(nccl().group_start(), "ncclGroupStart");
  for (int r = 0; r < n; ++r) {
    ncclResult_t e = nccl().all_reduce(minmax[r], minmax[r], 1, ncclFloat, ncclMin, g->comms[r], g->ctx[r]->stream);
    if (e == ncclSuccess)
      e = nccl().all_reduce(minmax[r] + 1, minmax[r] + 1, 1, ncclFloat, ncclMax, g->comms[r], g->ctx[r]->stream);
    if (e != ncclSuccess) {
      nccl().group_end();
      return nccl_fail(e, "ncclAllReduce (min / max)");
    }
  }
  OSC_NCCL(nccl().group_end(), "ncclGroupEnd (all-reduce)");
  return OSC_OK;
}

OSC_API int osc_group_run_sharded(osc_group* g, const osc_graph* const* graphs, const void* const* shard_out,
                                  void* const* gathered_out, size_t shard_bytes) {
  OSC_TRY(check_group(g, "osc_group_run_sharded"));
  if (graphs == nullptr) return fail(OSC_EINVAL, "osc_group_run_sharded: null graph array");
  const int n = static_cast<int>(g->ctx.size());
  for (int r = 0; r < n; ++r) OSC_TRY(osc_graph_launch(g->ctx[r], graphs[r]));
  return osc_group_allgather(g, shard_out, gathered_out, shard_bytes);
}

OSC_API int osc_group_synchronize(osc_group* g, int timeout_ms) {
  if (g == nullptr) return fail(OSC_EINVAL, "osc_group_synchronize: null group");
  for (osc_ctx* c : g->ctx) OSC_TRY(osc_synchronize(c, timeout_ms));
  return OSC_OK;
}

}  // extern "C"
