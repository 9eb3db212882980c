// runtime.h — internal state behind the C ABI: the per-GPU context (stream,
// device error word, scratch arena), error reporting, host-side fault
// injection and the TMA descriptor encoder.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "onnxsharp_cuda.h"

struct osc_prof_rec {
  std::string name;
  cudaEvent_t start, stop;
};

struct osc_ctx {
  int device = 0;
  int num_sms = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;  // where work is enqueued (own or caller's)
  int* d_err = nullptr;           // device error word, written by kernels on failure;
                                  // words 4..5 of the same 64-byte zeroed allocation are the
                                  // arrival/departure counters of in-kernel grid barriers
  void* scratch = nullptr;        // grow-only per-call temporaries
  size_t scratch_bytes = 0;
  // Launch accounting and per-kernel event timing (osc_profile_*).
  unsigned long long launches = 0;
  bool prof_on = false;
  cudaEvent_t prof_pending = nullptr;  // start event of the launch being made
  std::vector<osc_prof_rec> prof_recs;
  std::vector<cudaEvent_t> prof_pool;
};

namespace osc {

// Records a formatted message for osc_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Maps a CUDA error to OSC_ECUDA with a message naming the call site.
int cuda_fail(cudaError_t e, const char* what);

// Host-side fault injection: OSC_FAULT=<site>[,<site>...] makes the named
// sites ("alloc", "launch", "sync", "prepack", "all") fail with
// OSC_EFAULT_INJECTED before touching the device.
bool fault_injected(const char* site);

// Makes `ctx->device` current; returns OSC_OK or an error code.
int enter(osc_ctx* ctx);

// YOLO11 PSA attention on the tensor cores (gemm_tf32x3.cu).
int psa_composed(osc_ctx* ctx, const float* qkv, long long qkv_nstride, int B, int heads, int kd, int hd, int T,
                 float scale, float* out, long long out_nstride);
int psa_fused(osc_ctx* ctx, const float* qkv, long long qkv_nstride, int B, int heads, int kd, int hd, int T,
                 float scale, float* out, long long out_nstride);

// FusedAttention for T > 128 or head sizes other than 32 / 64, composed of
// tensor-core batched products and a row softmax (gemm_tf32x3.cu).
int attention_composed(osc_ctx* ctx, const float* q, const float* k, const float* v, const float* mask,
                       int mask_rows, int B, int T, int H, int D, float scale, int out_head_space, float* out);

// Scratch arena of at least `bytes`, 256-byte aligned. Fails during stream
// capture if it would have to grow.
int scratch(osc_ctx* ctx, size_t bytes, void** out);

// True while ctx->stream is being captured into a CUDA graph.
bool capturing(osc_ctx* ctx);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes /* rank-1 */, const uint32_t* box,
                 CUtensorMapSwizzle swizzle);

// Call right before every kernel launch: when profiling is on (and the
// stream is not being captured) it records the launch's start event.
void prof_begin(osc_ctx* ctx);

// Checks a kernel launch, counts it, records its stop event when profiling,
// and (when OSC_SYNC_CHECK=1) synchronises to surface faults at the call that
// caused them. `what` is the kernel name used by osc_profile_read.
int check_launch(osc_ctx* ctx, const char* what);

// Raises a kernel's dynamic shared memory limit once per (device, kernel).
int set_smem_attr(osc_ctx* ctx, const void* func, int bytes);

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// A kernel launched with programmatic stream serialization (launch_pdl) may
// start while the previous kernel on its stream is still draining: its CTAs
// set up (barriers, TMEM, tensor-map prefetch) and then griddep_wait() until
// that kernel has completed and its memory is visible -- before reading what
// it wrote or writing what it may still read. griddep_launch() lets the next
// kernel be scheduled once every CTA of this one has started. Both are no-ops
// for a kernel launched without the attribute.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch on the context's stream with programmatic stream serialization: the
// kernel may begin while the previous kernel on the stream drains, so its
// set-up overlaps that kernel's tail (in a captured graph this becomes a
// programmatic edge). Only for kernels that call griddep_wait() before any
// access to memory the previous kernel writes or reads. Records profiling
// events and checks the launch like check_launch.
template <typename... KArgs, typename... Args>
int launch_pdl(osc_ctx* ctx, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, const char* what,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  prof_begin(ctx);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return cuda_fail(e, what);
  return check_launch(ctx, what);
}

}  // namespace osc

#define OSC_TRY(expr)          \
  do {                         \
    int _st = (expr);          \
    if (_st != OSC_OK) return _st; \
  } while (0)

#define OSC_CUDA(expr, what)                                  \
  do {                                                        \
    cudaError_t _e = (expr);                                  \
    if (_e != cudaSuccess) return ::osc::cuda_fail(_e, what); \
  } while (0)
