// runtime.cu — context lifetime, errors, scratch arena, bounded synchronisation,
// device memory helpers and the TMA descriptor encoder.
//
// The context replaces the reference's per-Net runtime state (NetImpl,
// src/OnnxSharp/Core/NetImpl.cs:10) on one GPU: one stream, one device error
// word that kernels write when a bounded internal wait runs out, and a
// grow-only scratch arena for per-call temporaries (the reference rents such
// buffers from ArrayPool, e.g. Ops/AttentionOps.cs:307).
#include <cudaTypedefs.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <thread>
#include <utility>

#include "runtime.h"
#include "sm100.cuh"

namespace osc {

namespace {
thread_local std::string g_last_error;
}

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(OSC_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

bool fault_injected(const char* site) {
  const char* env = std::getenv("OSC_FAULT");
  if (env == nullptr || *env == '\0') return false;
  std::string list = std::string(",") + env + ",";
  if (list.find(",all,") != std::string::npos) return true;
  return list.find(std::string(",") + site + ",") != std::string::npos;
}

int enter(osc_ctx* ctx) {
  if (ctx == nullptr) return fail(OSC_EINVAL, "null context");
  OSC_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
  return OSC_OK;
}

bool capturing(osc_ctx* ctx) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(ctx->stream, &st) != cudaSuccess) return false;
  return st != cudaStreamCaptureStatusNone;
}

int scratch(osc_ctx* ctx, size_t bytes, void** out) {
  bytes = round_up(bytes < 256 ? 256 : bytes, 256);
  if (bytes > ctx->scratch_bytes) {
    if (capturing(ctx))
      return fail(OSC_EINVAL, "scratch arena must grow to %zu bytes during stream capture; call osc_reserve_scratch first",
                  bytes);
    if (fault_injected("alloc")) return fail(OSC_EFAULT_INJECTED, "injected allocation failure (scratch)");
    if (ctx->scratch != nullptr) {
      // The old arena may still be read by queued kernels.
      OSC_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize (scratch grow)");
      OSC_CUDA(cudaFree(ctx->scratch), "cudaFree (scratch)");
      ctx->scratch = nullptr;
      ctx->scratch_bytes = 0;
    }
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(OSC_ENOMEM, "scratch arena of %zu bytes: %s", bytes, cudaGetErrorString(e));
    }
    ctx->scratch = p;
    ctx->scratch_bytes = bytes;
  }
  *out = ctx->scratch;
  return OSC_OK;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  static cudaError_t lookup_err = cudaSuccess;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    lookup_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (lookup_err == cudaSuccess && q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (fn == nullptr) return fail(OSC_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(OSC_EINVAL, "TMA base address %p is not 16-byte aligned", base);
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) {
      s[i] = strides_bytes[i];
      if (strides_bytes[i] % 16 != 0)
        return fail(OSC_EINVAL, "TMA stride %llu bytes (dim %d) is not a multiple of 16",
                    static_cast<unsigned long long>(strides_bytes[i]), i + 1);
    }
  }
  CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(OSC_ECUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return OSC_OK;
}

static cudaEvent_t pool_event(osc_ctx* ctx) {
  if (!ctx->prof_pool.empty()) {
    cudaEvent_t ev = ctx->prof_pool.back();
    ctx->prof_pool.pop_back();
    return ev;
  }
  cudaEvent_t ev = nullptr;
  if (cudaEventCreate(&ev) != cudaSuccess) return nullptr;
  return ev;
}

void prof_begin(osc_ctx* ctx) {
  if (!ctx->prof_on || capturing(ctx)) return;
  cudaEvent_t ev = pool_event(ctx);
  if (ev != nullptr && cudaEventRecord(ev, ctx->stream) == cudaSuccess) ctx->prof_pending = ev;
}

int check_launch(osc_ctx* ctx, const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  ctx->launches += 1;
  if (ctx->prof_pending != nullptr) {
    cudaEvent_t stop = pool_event(ctx);
    if (stop != nullptr && cudaEventRecord(stop, ctx->stream) == cudaSuccess)
      ctx->prof_recs.push_back({what, ctx->prof_pending, stop});
    ctx->prof_pending = nullptr;
  }
  static const bool sync_check = [] {
    const char* v = std::getenv("OSC_SYNC_CHECK");
    return v != nullptr && v[0] == '1';
  }();
  if (sync_check && !capturing(ctx)) {
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, what);
  }
  return OSC_OK;
}

int set_smem_attr(osc_ctx* ctx, const void* func, int bytes) {
  // The attribute is raised whenever a launch needs more than was set before
  // (kernels whose shared memory depends on the shape).
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> set_bytes;
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(ctx->device, func);
  const auto it = set_bytes.find(key);
  if (it != set_bytes.end() && it->second >= bytes) return OSC_OK;
  OSC_CUDA(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
           "cudaFuncSetAttribute (dynamic shared memory)");
  set_bytes[key] = bytes;
  return OSC_OK;
}

}  // namespace osc

using namespace osc;

extern "C" {

OSC_API int osc_version(void) { return 100; }

OSC_API const char* osc_last_error(void) { return g_last_error.c_str(); }

OSC_API int osc_create(int device, osc_ctx** out) {
  if (out == nullptr) return fail(OSC_EINVAL, "osc_create: out is null");
  *out = nullptr;
  if (fault_injected("create")) return fail(OSC_EFAULT_INJECTED, "injected failure (create)");
  int count = 0;
  OSC_CUDA(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
  if (device < 0 || device >= count) return fail(OSC_EINVAL, "device %d out of range (%d devices)", device, count);
  OSC_CUDA(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop;
  OSC_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(OSC_EUNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device,
                prop.major, prop.minor);
  auto* ctx = new osc_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  cudaError_t e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete ctx;
    return cuda_fail(e, "cudaStreamCreateWithFlags");
  }
  ctx->stream = ctx->own_stream;
  e = cudaMalloc(&ctx->d_err, 64);
  if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, 64);
  if (e != cudaSuccess) {
    cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return cuda_fail(e, "cudaMalloc (error word)");
  }
  *out = ctx;
  return OSC_OK;
}

OSC_API int osc_profile_enable(osc_ctx* ctx, int on) {
  if (ctx == nullptr) return fail(OSC_EINVAL, "null context");
  ctx->prof_on = on != 0;
  return OSC_OK;
}

OSC_API int osc_profile_read(osc_ctx* ctx, const char* prefix, double* total_ms, int* launches) {
  OSC_TRY(enter(ctx));
  double ms = 0.0;
  int count = 0;
  const size_t plen = prefix ? std::strlen(prefix) : 0;
  for (const auto& r : ctx->prof_recs) {
    if (plen && r.name.compare(0, plen, prefix) != 0) continue;
    OSC_CUDA(cudaEventSynchronize(r.stop), "cudaEventSynchronize (profile)");
    float t = 0.0f;
    OSC_CUDA(cudaEventElapsedTime(&t, r.start, r.stop), "cudaEventElapsedTime (profile)");
    ms += t;
    count += 1;
  }
  if (total_ms) *total_ms = ms;
  if (launches) *launches = count;
  return OSC_OK;
}

OSC_API int osc_profile_reset(osc_ctx* ctx) {
  OSC_TRY(enter(ctx));
  for (auto& r : ctx->prof_recs) {
    ctx->prof_pool.push_back(r.start);
    ctx->prof_pool.push_back(r.stop);
  }
  ctx->prof_recs.clear();
  return OSC_OK;
}

OSC_API unsigned long long osc_launch_count(osc_ctx* ctx) { return ctx ? ctx->launches : 0ull; }

// ---- static-plan capture: the executor's "one CUDA graph per input
// signature" (the reference caches a plan per input signature, LayerPlan.cs:32-94).
struct osc_graph {
  int device;
  cudaGraph_t graph;
  cudaGraphExec_t exec;
};

OSC_API int osc_graph_begin(osc_ctx* ctx) {
  OSC_TRY(enter(ctx));
  if (ctx->stream == nullptr) return fail(OSC_EINVAL, "osc_graph_begin: cannot capture the legacy default stream");
  if (capturing(ctx)) return fail(OSC_EINVAL, "osc_graph_begin: already capturing");
  ctx->prof_on = false;  // event records are not captured
  OSC_CUDA(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  return OSC_OK;
}

OSC_API int osc_graph_end(osc_ctx* ctx, osc_graph** out) {
  if (out == nullptr) return fail(OSC_EINVAL, "osc_graph_end: out is null");
  *out = nullptr;
  OSC_TRY(enter(ctx));
  cudaGraph_t g = nullptr;
  OSC_CUDA(cudaStreamEndCapture(ctx->stream, &g), "cudaStreamEndCapture");
  cudaGraphExec_t ex = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    return cuda_fail(e, "cudaGraphInstantiate");
  }
  *out = new osc_graph{ctx->device, g, ex};
  return OSC_OK;
}

OSC_API int osc_graph_launch(osc_ctx* ctx, const osc_graph* graph) {
  OSC_TRY(enter(ctx));
  if (graph == nullptr || graph->device != ctx->device) return fail(OSC_EINVAL, "osc_graph_launch: bad graph");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  OSC_CUDA(cudaGraphLaunch(graph->exec, ctx->stream), "cudaGraphLaunch");
  return OSC_OK;
}

OSC_API int osc_graph_free(osc_graph* graph) {
  if (graph == nullptr) return OSC_OK;
  cudaSetDevice(graph->device);
  cudaGraphExecDestroy(graph->exec);
  cudaGraphDestroy(graph->graph);
  delete graph;
  return OSC_OK;
}

OSC_API int osc_destroy(osc_ctx* ctx) {
  if (ctx == nullptr) return OSC_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  for (auto& r : ctx->prof_recs) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  for (auto ev : ctx->prof_pool) cudaEventDestroy(ev);
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return OSC_OK;
}

OSC_API int osc_set_stream(osc_ctx* ctx, void* stream) {
  if (ctx == nullptr) return fail(OSC_EINVAL, "null context");
  ctx->stream = static_cast<cudaStream_t>(stream);
  return OSC_OK;
}

OSC_API void* osc_get_stream(osc_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

OSC_API void* osc_own_stream(osc_ctx* ctx) { return ctx ? static_cast<void*>(ctx->own_stream) : nullptr; }

OSC_API int osc_synchronize(osc_ctx* ctx, int timeout_ms) {
  OSC_TRY(enter(ctx));
  if (fault_injected("sync")) return fail(OSC_EFAULT_INJECTED, "injected failure (sync)");
  const auto limit = std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 60000);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery(ctx->stream);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return cuda_fail(e, "stream execution");
    if (std::chrono::steady_clock::now() - t0 > limit)
      return fail(OSC_ETIMEDOUT, "osc_synchronize: stream still busy after %d ms", timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  int word = 0;
  OSC_CUDA(cudaMemcpy(&word, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost), "read device error word");
  if (word != DEV_OK) {
    // also clears the grid-barrier counters that share the allocation (a kernel
    // that gave up may have left them mid-count)
    OSC_CUDA(cudaMemset(ctx->d_err, 0, 64), "reset device error word");
    if (word == DEV_ERR_TIMEOUT)
      return fail(OSC_ETIMEDOUT, "a kernel's bounded internal wait ran out (device error word %d)", word);
    return fail(OSC_EINVAL, "a kernel rejected its arguments (device error word %d)", word);
  }
  return OSC_OK;
}

OSC_API int osc_reserve_scratch(osc_ctx* ctx, size_t bytes) {
  OSC_TRY(enter(ctx));
  void* p = nullptr;
  return scratch(ctx, bytes, &p);
}

OSC_API int osc_malloc(osc_ctx* ctx, size_t bytes, void** out) {
  if (out == nullptr) return fail(OSC_EINVAL, "osc_malloc: out is null");
  *out = nullptr;
  OSC_TRY(enter(ctx));
  if (fault_injected("alloc")) return fail(OSC_EFAULT_INJECTED, "injected allocation failure");
  cudaError_t e = cudaMalloc(out, bytes ? bytes : 1);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(OSC_ENOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  }
  return OSC_OK;
}

OSC_API int osc_free(osc_ctx* ctx, void* ptr) {
  OSC_TRY(enter(ctx));
  if (ptr == nullptr) return OSC_OK;
  OSC_CUDA(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize (free)");
  OSC_CUDA(cudaFree(ptr), "cudaFree");
  return OSC_OK;
}

OSC_API int osc_memcpy_htod(osc_ctx* ctx, void* dst, const void* src, size_t bytes) {
  OSC_TRY(enter(ctx));
  if (bytes == 0) return OSC_OK;
  if (dst == nullptr || src == nullptr) return fail(OSC_EINVAL, "osc_memcpy_htod: null pointer");
  OSC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream), "cudaMemcpyAsync H2D");
  return OSC_OK;
}

OSC_API int osc_memcpy_dtoh(osc_ctx* ctx, void* dst, const void* src, size_t bytes) {
  OSC_TRY(enter(ctx));
  if (bytes == 0) return OSC_OK;
  if (dst == nullptr || src == nullptr) return fail(OSC_EINVAL, "osc_memcpy_dtoh: null pointer");
  OSC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "cudaMemcpyAsync D2H");
  return OSC_OK;
}

}  // extern "C"
