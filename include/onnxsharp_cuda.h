/*
 * onnxsharp_cuda.h — C ABI of libonnxsharp_cuda, the B200 (sm_100a) kernels
 * behind OnnxSharp's matrix-multiply operators.
 *
 * Boundary. OnnxSharp (pure C#) reaches its operators through
 * LayerRegistry.Register(type, factory) (src/OnnxSharp/Core/LayerRegistry.cs:14)
 * and calls the Layer virtuals GetMemoryShapes -> PrepackWeights/Finalize ->
 * Forward (src/OnnxSharp/Core/LayerInfo.cs:75-218, Core/Interpreter.cs:87-146).
 * A CUDA-backed layer keeps that contract and forwards to this library through
 * P/Invoke: PrepackWeights maps to the osc_*_prepack calls (once per constant
 * weight, as the reference caches packed panels by tensor identity,
 * Ops/DnnOps.cs:2823-2832), Forward maps to the kernel entry points.
 *
 * Conventions.
 *  - Every call returns an int status (OSC_OK == 0). The message of the last
 *    failure on the calling thread is returned by osc_last_error(). No call
 *    throws, aborts or resets the device.
 *  - Tensor pointers passed to kernel entry points are DEVICE pointers
 *    (from osc_malloc, cudaMalloc or a framework allocator) in the context's
 *    device. FP32 tensors are dense row-major (NCHW for images) unless a
 *    stride argument says otherwise. Host pointers are accepted only by
 *    osc_memcpy_htod / osc_memcpy_dtoh / osc_*_prepack_host.
 *  - Work is enqueued on the context's stream and is asynchronous;
 *    osc_synchronize() waits (with a bound) and reports device-side errors
 *    (a kernel whose internal wait ran out reports OSC_ETIMEDOUT).
 *  - One context per GPU. Calls on one context must be serialised by the
 *    caller (the reference interpreter is single-threaded, Interpreter.cs:30);
 *    different contexts may be driven from different host threads.
 */
#ifndef ONNXSHARP_CUDA_H
#define ONNXSHARP_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define OSC_API __declspec(dllexport)
#else
#define OSC_API __attribute__((visibility("default")))
#endif

/* ------------------------------------------------------------ status codes */
enum osc_status {
  OSC_OK = 0,
  OSC_EINVAL = 1,            /* bad argument (shape, null pointer, unsupported attribute) */
  OSC_ENOMEM = 2,            /* device allocation failed */
  OSC_ECUDA = 3,             /* a CUDA runtime/driver call failed */
  OSC_ENCCL = 4,             /* reserved for collective failures */
  OSC_ETIMEDOUT = 5,         /* a bounded wait (host or device) ran out */
  OSC_EFAULT_INJECTED = 6,   /* host-side fault injection (env OSC_FAULT) */
  OSC_EUNSUPPORTED = 7       /* valid ONNX, not implemented by this backend */
};

/* Fused activation codes (Conv.FusedActivation, Ops/DnnOps.cs:104, :493-499).
 * OSC_ACT_FAST may be OR-ed into the code given to osc_conv2d_direct_f32:
 * Sigmoid / SiLU then come from the hardware ex2 / rcp instructions (within
 * 2e-6 of the exact form in |d| / max(1, |ref|), see osc_selfcheck_fast_act)
 * instead of the reference's VectorMath restated bit for bit. The tensor-core
 * conv entries always compute the fast form (their sums are not bit-identical
 * to the reference's anyway); the other entries accept the plain codes. */
enum osc_act { OSC_ACT_NONE = 0, OSC_ACT_SILU = 1, OSC_ACT_RELU = 2, OSC_ACT_SIGMOID = 3, OSC_ACT_FAST = 16 };

typedef struct osc_ctx osc_ctx;
typedef struct osc_gemm_weights osc_gemm_weights;

/* ------------------------------------------------------------ context */

/* Version of this ABI (major*10000 + minor*100 + patch). */
OSC_API int osc_version(void);

/* Message of the last failed call on this thread ("" if none). */
OSC_API const char* osc_last_error(void);

/* Create a context on `device` with its own non-blocking stream.
 * Replaces the per-Net state of NetImpl (src/OnnxSharp/Core/NetImpl.cs:10). */
OSC_API int osc_create(int device, osc_ctx** out);
OSC_API int osc_destroy(osc_ctx* ctx);

/* Make the context enqueue on a caller-owned stream (cudaStream_t), e.g. a
 * framework's current stream. The handle is taken literally: NULL is the
 * CUDA legacy default stream. osc_own_stream() returns the context's own
 * stream, to switch back. */
OSC_API int osc_set_stream(osc_ctx* ctx, void* stream);
OSC_API void* osc_get_stream(osc_ctx* ctx);
OSC_API void* osc_own_stream(osc_ctx* ctx);

/* Wait (bounded by timeout_ms; <= 0 means 60 s) for all work on the context's
 * stream and report device-side error words. */
OSC_API int osc_synchronize(osc_ctx* ctx, int timeout_ms);

/* Grow the context's scratch arena to at least `bytes` (per-call
 * temporaries such as the TF32 hi/lo split of activations). Call before
 * stream capture: a call that would need to grow it while capturing fails. */
OSC_API int osc_reserve_scratch(osc_ctx* ctx, size_t bytes);

/* Per-kernel timing (the CUDA counterpart of Net.ProfileAll,
 * src/OnnxSharp/Core/Net.cs:282-332): while enabled, every kernel launch made
 * through this context outside stream capture is bracketed by CUDA events on
 * the context's stream. osc_profile_read sums the durations (ms) and counts
 * the launches whose kernel name starts with `prefix` (NULL or "" = all);
 * osc_profile_reset drops the records. osc_launch_count counts every kernel
 * launch the context has made (profiling on or off). */
OSC_API int osc_profile_enable(osc_ctx* ctx, int on);
OSC_API int osc_profile_read(osc_ctx* ctx, const char* prefix, double* total_ms, int* launches);
OSC_API int osc_profile_reset(osc_ctx* ctx);
OSC_API unsigned long long osc_launch_count(osc_ctx* ctx);

/* Static-plan capture: the executor runs a shape-specialised plan once to
 * size the scratch arena, then records it between osc_graph_begin and
 * osc_graph_end (stream capture of the context's stream) and replays it with
 * osc_graph_launch — one CUDA graph per input signature, the device
 * counterpart of the reference's per-signature plan cache
 * (Core/LayerPlan.cs:32-94, Core/Interpreter.cs:87-146). */
typedef struct osc_graph osc_graph;
OSC_API int osc_graph_begin(osc_ctx* ctx);
OSC_API int osc_graph_end(osc_ctx* ctx, osc_graph** out);
OSC_API int osc_graph_launch(osc_ctx* ctx, const osc_graph* graph);
OSC_API int osc_graph_free(osc_graph* graph);

/* Static plan of fused nodes (the executor of NetImpl.PrepareForGraph /
 * BufferAllocator.Assign / Interpreter.Run, src/OnnxSharp/Engine/NetImpl.cs:151-192,
 * Engine/BufferAllocator.cs:41-138, Core/Interpreter.cs:30-186) for a host
 * that hands the library its whole fused graph at once. Buffers are NCHW,
 * described per image (C, H, W; the batch is the plan's); nodes read and write
 * channel slices of them (osc_plan_ref), so Concat is producers writing into
 * slices of one buffer and Split is slices of one buffer. osc_plan_build
 * colours the buffers' live ranges into slots with the reference's rule (by
 * first write; a slot is reused only when its last reader is strictly before
 * the new first write; the largest buffer sizes the slot) and allocates one
 * device arena. The buffer `input_buf` is not in the arena: osc_plan_run binds
 * it to the caller's pointer. The first run with an (input, output) pointer
 * pair runs the nodes once and captures them into a CUDA graph (the
 * reference's per-signature plan cache, Core/LayerPlan.cs:32-94); later runs
 * with that pair replay it (up to 8 pairs are kept). Weights: an
 * osc_conv_weights* (OSC_OP_CONV), the raw [M, C/group, k, k] device tensor
 * (OSC_OP_CONV_DIRECT), an osc_gemm_weights* (OSC_OP_MATMUL_BIAS); they must
 * outlive the plan.
 *
 * Node attributes (iattr / fattr):
 *   CONV, CONV_DIRECT  in = {x, residual?}; iattr = {stride, pad, dilation, act, k, group}
 *                      (y = residual + act(conv(x) + bias); CONV is group 1, k from the weights)
 *   MAXPOOL            iattr = {k, stride, pad}
 *   RESIZE_NEAREST     iattr = {scale}
 *   PSA                in = {qkv}; iattr = {heads, kd, hd}; fattr = {scale}
 *   YOLO_DECODE        in = {box0, box1, box2, cls0, cls1, cls2}, no out (writes the plan
 *                      output [B, 4 + nc, A]); iattr = {nc}; fattr = {stride0, stride1, stride2}
 *   MATMUL_BIAS        whole buffers; rows = B*C*H, k = W; out W = n; iattr[3] = act
 *   SOFTMAX            whole buffers; over W
 *   UNARY              whole buffers; iattr[3] = act
 *   ATTENTION          in = {q, k, v} whole buffers [B, T = C, 1, heads * D = W]; iattr = {heads};
 *                      fattr = {scale}; out [B, T, 1, heads * D] */
enum osc_plan_op {
  OSC_OP_CONV = 1, OSC_OP_CONV_DIRECT = 2, OSC_OP_MAXPOOL = 3, OSC_OP_RESIZE_NEAREST = 4, OSC_OP_PSA = 5,
  OSC_OP_YOLO_DECODE = 6, OSC_OP_MATMUL_BIAS = 7, OSC_OP_SOFTMAX = 8, OSC_OP_UNARY = 9, OSC_OP_ATTENTION = 10
};
#define OSC_PLAN_MAX_IN 6
typedef struct osc_plan_ref { int buf, c0, c; } osc_plan_ref; /* channels [c0, c0 + c) of buffer buf */
typedef struct osc_plan_node {
  int op, n_in, n_out;
  osc_plan_ref in[OSC_PLAN_MAX_IN];
  osc_plan_ref out[1];
  int iattr[8];
  float fattr[4];
  const void* weights;
  const float* bias;
} osc_plan_node;
typedef struct osc_plan_desc {
  int batch;
  int n_buffers;
  const int* buf_chw; /* [n_buffers][3] */
  int input_buf;
  int n_nodes;
  const osc_plan_node* nodes;
} osc_plan_desc;
typedef struct osc_plan osc_plan;
OSC_API int osc_plan_build(osc_ctx* ctx, const osc_plan_desc* desc, osc_plan** out);
OSC_API int osc_plan_run(osc_plan* plan, const float* input, float* output);
OSC_API int osc_plan_arena_bytes(const osc_plan* plan, size_t* bytes);
/* Device address (and image stride in elements) of a buffer for a given input
 * pointer: the arena slot of an activation, or `input` for the input buffer. */
OSC_API int osc_plan_buffer(const osc_plan* plan, int buffer, const float* input, float** ptr, long long* nstride);
OSC_API int osc_plan_free(osc_plan* plan);

/* The colouring osc_plan_build uses, on the host (no device): byte offset per
 * buffer (-1 if first_write < 0) and the arena size. */
OSC_API int osc_arena_assign(int n, const int* first_write, const int* last_read, const size_t* bytes,
                             long long* offsets, size_t* total);

/* Device memory and copies, for callers without a framework allocator (the
 * reference's Tensor buffers are pinned host arrays, Tensors/Tensor.cs:65-155). */
OSC_API int osc_malloc(osc_ctx* ctx, size_t bytes, void** out);
OSC_API int osc_free(osc_ctx* ctx, void* ptr);
OSC_API int osc_memcpy_htod(osc_ctx* ctx, void* dst, const void* src, size_t bytes);
OSC_API int osc_memcpy_dtoh(osc_ctx* ctx, void* dst, const void* src, size_t bytes);

/* ------------------------------------------------------------ several GPUs of one node
 * Batch-level inference sharded by image / row / sequence over the GPUs of a
 * node, driven from ONE host process (a C# host keeps one Net): a context per
 * GPU (osc_group_ctx; use it like any context, it is owned by the group) and
 * an NCCL communicator clique among them. The reference has no multi-device
 * path; its contract that one Forward() returns the whole batch's output
 * (src/OnnxSharp/Core/Net.cs:258-262) is kept by all-gathering the shards.
 * NCCL is loaded at run time (libnccl.so.2); without it these entries return
 * OSC_ENCCL and everything else still works. Work is enqueued on each
 * context's stream; osc_group_synchronize waits for all of them. */
typedef struct osc_group osc_group;
OSC_API int osc_group_create(int ndev, const int* devices, osc_group** out);
OSC_API int osc_group_destroy(osc_group* g);
OSC_API int osc_group_size(osc_group* g, int* n);
OSC_API int osc_group_ctx(osc_group* g, int rank, osc_ctx** out);
OSC_API int osc_group_synchronize(osc_group* g, int timeout_ms);

/* All-gather: `bytes` from send[r] (a device buffer of rank r's GPU) land at
 * recv[i] + r * bytes on every rank i (recv[i] holds ndev * bytes). */
OSC_API int osc_group_allgather(osc_group* g, const void* const* send, void* const* recv, size_t bytes);

/* DynamicQuantizeMatMul over row shards: minmax[r] (2 device floats on rank
 * r, from osc_minmax_f32 on that rank's rows) becomes the global {min, max}
 * on every rank, so each shard's osc_dqmm_f32(..., minmax_override = minmax[r])
 * quantises exactly as the whole tensor would (QuantizedMatMulOps.cs:146-156). */
OSC_API int osc_group_allreduce_minmax(osc_group* g, float* const* minmax);

/* One sharded step: on every rank r, replay graphs[r] (the plan over that
 * GPU's shard, captured on osc_group_ctx(g, r)), then all-gather the shard
 * outputs shard_out[r] (shard_bytes each) into gathered_out[r]. */
OSC_API int osc_group_run_sharded(osc_group* g, const osc_graph* const* graphs, const void* const* shard_out,
                                  void* const* gathered_out, size_t shard_bytes);

/* ------------------------------------------------------------ MatMul (+FusedBias)
 * Replaces MatMulLayer.Forward with FusedBias (src/OnnxSharp/Ops/DnnOps.cs:2789-3102)
 * over GemmKernel.Pack / MultiplyPacked (src/OnnxSharp/Tensors/GemmKernel.cs:503, :675-852).
 *
 * osc_gemm_prepack_f32: pack constant B once. b_layout 0: B is [k, n] row-major
 * (ONNX MatMul); 1: B is [n, k] row-major (ONNX Gemm transB=1). The packed
 * form is the 3xTF32 hi/lo split in the tensor-core operand layout.
 * `b` is a device pointer (osc_gemm_prepack_f32) or host pointer (_host). */
OSC_API int osc_gemm_prepack_f32(osc_ctx* ctx, const float* b, int k, int n, int b_layout,
                                 osc_gemm_weights** out);
OSC_API int osc_gemm_prepack_f32_host(osc_ctx* ctx, const float* b, int k, int n, int b_layout,
                                      osc_gemm_weights** out);
OSC_API int osc_gemm_weights_free(osc_gemm_weights* w);

/* C[m, n] = A[m, k] * B + col_bias[n] (col_bias may be NULL), then `act`.
 * lda / ldc are row strides in elements (0 = dense). FP32 in and out,
 * computed with 3xTF32 on the tensor cores (tcgen05 kind::tf32). */
OSC_API int osc_gemm_bias_f32(osc_ctx* ctx, const float* a, int m, int k, int lda,
                              const osc_gemm_weights* w, const float* col_bias, int act, float* c,
                              int ldc);

/* osc_gemm_bias_f32 in two steps, for an activation that feeds several
 * MatMuls (the Q, K and V projections of one input, each its own MatMul node
 * with FusedBias in the reference: Ops/DnnOps.cs:2902-3102): split A once,
 * then multiply the split by each packed weight. Same kernels and results as
 * osc_gemm_bias_f32. osc_gemm_split_a_f32 writes the K-major TF32 operands
 * a_hi, a_lo [m][kp] (kp = k rounded up to a multiple of 4, the packed
 * weights' kp; both 16-byte aligned, caller-allocated, m * kp floats each).
 * osc_gemm_bias_presplit_f32 then computes C = A @ B + bias (then act) from
 * them; its kp must match the weights'. */
OSC_API int osc_gemm_split_a_f32(osc_ctx* ctx, const float* a, int m, int k, int lda, int kp,
                                 float* a_hi, float* a_lo);
OSC_API int osc_gemm_bias_presplit_f32(osc_ctx* ctx, const float* a_hi, const float* a_lo, int m,
                                       int kp, const osc_gemm_weights* w, const float* col_bias,
                                       int act, float* c, int ldc);

/* Same as osc_gemm_bias_f32, but allocates no device memory: for callers that
 * must not call cudaMalloc while serving (a host that fixes its GPU memory
 * budget at start-up, or one sharing the GPU with other work, where an
 * allocation can synchronise the whole device at an arbitrary moment). This
 * entry point has no counterpart in the reference (which has no device).
 * Its temporaries live in a fixed 8 MiB array compiled into the library (held
 * by every GPU that loads it, until the process exits): a call needs
 * m * round_up(k, 4) <= 1048576 (e.g. 2048 x 512) and is rejected with
 * OSC_EINVAL beyond that. The first call on a device looks up that array's
 * device address (cudaGetSymbolAddress) and should come before any stream
 * capture. All calls share the array: calls whose kernels may overlap on the
 * GPU (other streams or contexts on the same device) race and must be
 * serialised by the caller. */
OSC_API int osc_gemm_bias_f32_noalloc(osc_ctx* ctx, const float* a, int m, int k, int lda,
                                      const osc_gemm_weights* w, const float* col_bias, int act, float* c,
                                      int ldc);

/* ------------------------------------------------------------ Conv (+FusedActivation)
 * Replaces ConvLayer.Forward (src/OnnxSharp/Ops/DnnOps.cs:411-500) and its
 * kernel chain (Kernels/ConvKernels.cs Im2Col/Pointwise, NchwcConv,
 * Winograd, PackedConv, FirstConv) plus the in-place fused activation
 * (DnnOps.cs:493-499), for group == 1.
 *
 * osc_conv_prepack_f32: pack constant W [M, C, kh, kw] once (host != 0: `w` is
 * a host pointer). kh*kw <= 49. */
typedef struct osc_conv_weights osc_conv_weights;
OSC_API int osc_conv_prepack_f32(osc_ctx* ctx, const float* w, int M, int C, int kh, int kw, int host,
                                 osc_conv_weights** out);
OSC_API int osc_conv_weights_free(osc_conv_weights* w);

/* y[N, M, OH, OW] = act(conv(x[N, C, H, W], W) + bias[M]) with ONNX Conv
 * semantics (strides, pads top/left/bottom/right, dilations; group must be 1;
 * equal strides). OH/OW must equal the ONNX output size (floor mode,
 * DnnOps.cs:53-66). bias may be NULL. NCHW FP32 in and out; computed as an
 * implicit GEMM with 3xTF32 on the tensor cores. */
OSC_API int osc_conv2d_bias_act_f32(osc_ctx* ctx, const float* x, int N, int C, int H, int W,
                                    const osc_conv_weights* w, int stride_h, int stride_w, int pad_t, int pad_l,
                                    int pad_b, int pad_r, int dil_h, int dil_w, int group, const float* bias, int act,
                                    float* y, int OH, int OW);

/* ------------------------------------------------------------ DynamicQuantizeMatMul (int8)
 * Replaces DynamicQuantizeMatMulLayer (src/OnnxSharp/Ops/QuantizedMatMulOps.cs:28-376)
 * with Quantizer.MinMax (Tensors/Quantization.cs:109-181): per-tensor dynamic
 * uint8 quantisation of A, int8/uint8 weights with per-column zero points,
 * exact int32 accumulation on the tensor cores (tcgen05 kind::i8), then
 * y = acc * (a_scale * w_scale[j]) + bias[j] with the reference's rounding
 * (one FMA on full 16-column panels of 12/6/4-row groups, mul then add on
 * tail columns / leftover rows), so y is bit-identical to the reference's
 * single-threaded (row-block = all rows) result.
 *
 * osc_dqmm_prepack: W [k, n] row-major bytes (is_signed: int8, else uint8),
 * n_zp zero points (0: none, 1: per tensor, n: per column; host array).
 * host != 0: `w` is a host pointer. */
typedef struct osc_dqmm_weights osc_dqmm_weights;
OSC_API int osc_dqmm_prepack(osc_ctx* ctx, const void* w, int k, int n, int is_signed, const int32_t* w_zp,
                             int n_zp, int host, osc_dqmm_weights** out);
OSC_API int osc_dqmm_weights_free(osc_dqmm_weights* w);

/* y[m, n] = DynamicQuantizeMatMul(A[m, k]); all pointers are device pointers.
 * w_scale has n_scale entries (1 or n); bias may be NULL.
 * minmax_override (NULL or 2 floats {min, max}) replaces the range of A: a
 * row-sharded multi-GPU caller all-reduces the shards' ranges (see
 * osc_minmax_f32) so every shard quantises exactly as the whole tensor would.
 * Optional outputs (NULL to skip): q_out [m, k] uint8 quantised A, acc_out
 * [m, n] int32 accumulators sum (q - zp)(w - wzp), params_out {scale, zp}. */
OSC_API int osc_dqmm_f32(osc_ctx* ctx, const float* a, int m, int k, int lda, const osc_dqmm_weights* w,
                         const float* w_scale, int n_scale, const float* bias, float* y, const float* minmax_override,
                         uint8_t* q_out, int32_t* acc_out, float* params_out);

/* osc_dqmm_f32 for a row shard: A holds rows [row0, row0 + m) of a tensor of
 * rows_total rows, quantised with that tensor's range minmax_global (device,
 * {min, max}, e.g. all-reduced over the shards). The reference rounds a row's
 * epilogue with one FMA when the row lies in the 12/6/4-row micro-kernel
 * groups of the whole matrix and with mul+add otherwise
 * (GemmKernel.cs:746-790, 1594-1608); this entry classifies the shard's rows
 * by their index in the whole tensor, so the shards' q, accumulators AND y
 * are bit-identical to the unsharded call's. */
OSC_API int osc_dqmm_shard_f32(osc_ctx* ctx, const float* a, int m, int k, int lda, const osc_dqmm_weights* w,
                               const float* w_scale, int n_scale, const float* bias, float* y,
                               const float* minmax_global, int row0, int rows_total, uint8_t* q_out,
                               int32_t* acc_out, float* params_out);

/* minmax_out[0..1] (device) = {min(x, 0), max(x, 0)} over `count` floats, NaN
 * skipped (Quantizer.MinMax). */
OSC_API int osc_minmax_f32(osc_ctx* ctx, const float* x, long count, float* minmax_out);

/* ------------------------------------------------------------ FusedAttention
 * Replaces AttentionLayer.Forward (src/OnnxSharp/Ops/AttentionOps.cs:249-351),
 * heads form: q, k, v are [B, T, H*D] (the fused node's inputs
 * [Q, K, V, mask?] with attributes scale / heads / output_head_space,
 * GraphFusion.cs:1139-1162). out = softmax(scale*Q K^T + mask) V as
 * [B, T, H*D] (out_head_space = 0) or [B, H, T, D] (1). mask may be NULL or
 * [B, 1, mask_rows, T] with mask_rows 1 or T. T <= 128 with D in {32, 64}: one
 * head per SM, QK^T / softmax / .V on chip; otherwise (any T, any D) a composed
 * path: batched QK^T, the reference's lazy softmax, e.V scaled by 1/sum. Both
 * on the 3xTF32 tensor cores. */
OSC_API int osc_attention_f32(osc_ctx* ctx, const float* q, const float* k, const float* v, const float* mask,
                              int mask_rows, int B, int T, int H, int D, float scale, int out_head_space,
                              float* out);

/* ------------------------------------------------------------ graph glue (YOLO11n-shaped graph)
 * NCHW tensors may be channel slices of larger buffers: *_nstride is the
 * element distance between consecutive images (0 = dense), so a Split output
 * is a pointer offset and a Concat input can be produced in place. */

/* Conv with image strides and an optional residual added after the
 * activation: y = residual + act(conv(x) + bias) (the C3k2 / PSA bottleneck
 * Add of the exported graph fused into the conv). group must be 1. */
OSC_API int osc_conv2d_ex_f32(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W,
                              const osc_conv_weights* w, int stride_h, int stride_w, int pad_t, int pad_l, int pad_b,
                              int pad_r, int dil_h, int dil_w, const float* bias, int act, const float* residual,
                              long long res_nstride, float* y, long long y_nstride, int OH, int OW);

/* Direct (CUDA-core) conv for grouped / depthwise convs and first layers with
 * few input channels (Kernels/DepthwiseConv.cs:25-93, Kernels/FirstConv.cs:54-121).
 * w is the raw [M, C/group, kh, kw] device tensor. */
OSC_API int osc_conv2d_direct_f32(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W,
                                  const float* w, int M, int kh, int kw, int stride_h, int stride_w, int pad_t,
                                  int pad_l, int pad_b, int pad_r, int dil_h, int dil_w, int group, const float* bias,
                                  int act, const float* residual, long long res_nstride, float* y, long long y_nstride,
                                  int OH, int OW);

/* MaxPool (Ops/DnnOps.cs:1335), floor mode, padding ignored in the max. */
OSC_API int osc_maxpool2d_f32(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W, int kh,
                              int kw, int stride_h, int stride_w, int pad_t, int pad_l, int pad_b, int pad_r, float* y,
                              long long y_nstride, int OH, int OW);

/* Resize, nearest, integer up-scale factors (Ops/DnnOps.cs:2215). */
OSC_API int osc_resize_nearest_f32(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W,
                                   int scale_h, int scale_w, float* y, long long y_nstride);

/* y = a (op) b with numpy broadcasting, rank <= 4, dense tensors;
 * op: 0 Add, 1 Sub, 2 Mul, 3 Div (Ops/BroadcastOps.cs). Shapes are host arrays. */
OSC_API int osc_binary_f32(osc_ctx* ctx, int op, const float* a, const long long* a_shape, int a_rank, const float* b,
                           const long long* b_shape, int b_rank, float* y);

/* y[i] = act(x[i]) with the reference's VectorMath formulas (SiLU / Sigmoid / ReLU). */
OSC_API int osc_unary_f32(osc_ctx* ctx, const float* x, float* y, long long n, int act);

/* Softmax over the last axis of a [rows, len] tensor (Ops/DnnOps.cs:2547 ->
 * VectorMath.SoftmaxRow, VectorMath.cs:282). */
OSC_API int osc_softmax_f32(osc_ctx* ctx, const float* x, float* y, long long rows, int len);

/* DflSoftmax (Ops/DflOps.cs:90-250): x [B, sides*bins, pixels] ->
 * out [B, sides, pixels] = sum_b b * softmax_b. bins <= 32. */
OSC_API int osc_dfl_f32(osc_ctx* ctx, const float* x, int B, int sides, int bins, int pixels, float* out);

/* The YOLO Detect tail fused: per scale i (3 scales) the box logits box[i]
 * [B, 64, hs[i], ws[i]] and class logits cls[i] [B, nc, hs[i], ws[i]] (views)
 * -> out [B, 4 + nc, A] (A = sum hs*ws): DFL (reg_max 16), dist2bbox with
 * anchor points (x + 0.5, y + 0.5) in the exported graph's op order, times
 * strides[i]; sigmoid of the class logits. Pointer arrays are host arrays. */
OSC_API int osc_yolo_decode_f32(osc_ctx* ctx, int B, int nc, const float* const* box, const long long* box_nstride,
                                const float* const* cls, const long long* cls_nstride, const int* hs, const int* ws,
                                const float* strides, float* out);

/* LayerNormalization over the trailing `inner` elements (Ops/AttnOps.cs:199-358).
 * gamma / beta may be NULL. */
OSC_API int osc_layernorm_f32(osc_ctx* ctx, const float* x, int outer, int inner, const float* gamma,
                              const float* beta, float eps, float* y);

/* Attention of YOLO11's PSA block (sequence T = H*W, not limited to 128):
 * qkv [B, heads*(2*kd + hd), T] -> out [B, heads*hd, T] with
 * out = v softmax(scale * q^T k)^T per head (the exported MatMul / Mul /
 * Softmax / MatMul sequence). */
OSC_API int osc_psa_attention_f32(osc_ctx* ctx, const float* qkv, long long qkv_nstride, int B, int heads, int kd,
                                  int hd, int T, float scale, float* out, long long out_nstride);

/* Batched / transposed-view MatMul with a non-constant B (Ops/DnnOps.cs:2945-3094,
 * the gemm_view strides folded in by Core/GraphFusion.cs:1424): for batch
 * z = o * inner + i (o < outer, i < inner), y[z] [m, n] (dense) =
 * A[z] [m, k] x B[z] [k, n] (+ col_bias [n]), element (r, c) of A[z] at
 * a + o*a_outer + i*a_inner + r*a_row + c*a_col, element (t, j) of B[z] at
 * b + o*b_outer + i*b_inner + t*b_row + j*b_col (strides in elements; 0
 * broadcasts). 3xTF32. outer*inner <= 65535. */
OSC_API int osc_matmul_batched_f32(osc_ctx* ctx, int outer, int inner, int m, int k, int n, const float* a,
                                   long long a_outer, long long a_inner, long long a_row, long long a_col,
                                   const float* b, long long b_outer, long long b_inner, long long b_row,
                                   long long b_col, const float* col_bias, float* y);

/* ONNX Gemm (Ops/AttnOps.cs:31-128): y [m, n] = alpha * A' B' + beta * C with
 * A' = A [m, k] or A^T (trans_a, A stored [k, m]); B' from prepacked weights
 * w (transB resolved by osc_gemm_prepack_f32's b_layout) or, with w = NULL,
 * from a device B [k, n] (or [n, k] with trans_b). C (c_len elements, may be
 * 0) broadcasts as the reference does: c_len >= m*n full, 1 scalar, else
 * c[j % c_len]. The epilogue rounds alpha*acc, beta*c and their sum separately. */
OSC_API int osc_gemm_onnx_f32(osc_ctx* ctx, const float* a, int trans_a, int m, int k, const osc_gemm_weights* w,
                              const float* b, int trans_b, int n, float alpha, float beta, const float* c,
                              long long c_len, float* y);

/* DynamicQuantizeLinear as a standalone op (Ops/QuantOps.cs:155-231):
 * x [count] f32 -> y [count] u8, *y_scale (f32) and *y_zero_point (u8), all
 * device pointers (the scalars may be NULL). Same range, scale, zero point
 * and rounding as osc_dqmm_f32's quantisation; NaN inputs give 0. */
OSC_API int osc_dynamic_quantize_linear_f32(osc_ctx* ctx, const float* x, long long count, uint8_t* y,
                                            float* y_scale, uint8_t* y_zero_point);

/* MatMulInteger (Ops/QuantOps.cs:234-345, Kernels/Int8Gemm.cs:185-238):
 * y [m, n] s32 = sum_t (a[i,t] - a_zero_point) * (W[t,j] - w_zp[j]) with A
 * u8 (a_signed = 0) or s8 (a_signed = 1), row pitch lda bytes (0 = k), a
 * scalar a_zero_point, and W prepacked by osc_dqmm_prepack (s8 or u8, per
 * column or per tensor zero points). Exact integer arithmetic on the int8
 * tensor cores. */
OSC_API int osc_matmul_integer_i8(osc_ctx* ctx, const void* a, int a_signed, int m, int k, int lda, int a_zero_point,
                                  const osc_dqmm_weights* w, int32_t* y);

/* ImagePreprocessor.Letterbox (Vision/ImagePreprocessor.cs:57-100) on the device:
 * u8 pixels [height][row_stride] (bytes_per_pixel 3 or 4; bgr = 1 for BGR(A)
 * order) -> dst [3, target_h, target_w] f32 (a slice of the batch input):
 * aspect-preserving bilinear resize (ImageGeometry.Contain, AxisMap.Bilinear),
 * centred, pad 114/255, /255 normalisation; bit-identical to the reference.
 * placement (host, may be NULL) gets {resized_w, resized_h, offset_x, offset_y}. */
OSC_API int osc_letterbox_u8(osc_ctx* ctx, const uint8_t* pixels, int width, int height, int row_stride,
                             int bytes_per_pixel, int bgr, int target_w, int target_h, float* dst, int* placement);

/* osc_letterbox_u8 over a batch of B frames of one size (a camera batch), one
 * launch: frame z at pixels + z * image_stride bytes (0 = row_stride * height)
 * -> dst + z * dst_nstride floats (0 = 3 * target_h * target_w), each
 * bit-identical to osc_letterbox_u8 on that frame. placement as there (the
 * same for every frame). */
OSC_API int osc_letterbox_batch_u8(osc_ctx* ctx, const uint8_t* pixels, int B, long long image_stride, int width,
                                   int height, int row_stride, int bytes_per_pixel, int bgr, int target_w,
                                   int target_h, float* dst, long long dst_nstride, int* placement);

/* The YOLO detect tail (YoloDecoder.Decode + DetectionNms.SuppressSorted,
 * Vision/YoloDecoder.cs:68-188, Vision/Detection.cs:62-107) on the device, one
 * image per CTA: output [B, fields, anchors] channels-first (fields = 4 +
 * classes) -> dets [B, max_det, 6] (class, score, x, y, w, h) and counts [B].
 * Candidates: first class maximum >= conf, finite, positive size; sorted by
 * score (ties by anchor index); greedy NMS per class (or class_agnostic) with
 * IoU > iou suppressing; at most max_candidates considered and max_det kept.
 * transforms [B][6] (device, may be NULL) = {resized_w, resized_h, offset_x,
 * offset_y, source_w, source_h} maps boxes back to source pixels (clamped,
 * zero-area boxes dropped). anchors <= 16384, max_det <= 1024. */
OSC_API int osc_yolo_detect_f32(osc_ctx* ctx, const float* output, int B, int fields, int anchors, float conf,
                                float iou, int max_det, int max_candidates, int class_agnostic,
                                const float* transforms, float* dets, int* counts);

/* Diagnostics (no counterpart in the reference): the maximum error, over
 * every finite float x, of the hardware-instruction Sigmoid and SiLU used in
 * the tensor-core conv epilogues against the exact VectorMath restatement, in
 * the parity metric |fast - exact| / max(1, |exact|). */
OSC_API int osc_selfcheck_fast_act(osc_ctx* ctx, float* max_sigmoid_err, float* max_silu_err);

/* Diagnostics (no counterpart in the reference): checks on the device that the
 * branch-free reciprocal inside the exact Sigmoid/SiLU (the CUDA-core
 * epilogues and the activation ops) returns the
 * same bits as the IEEE division 1/d for every float d in [1, 2^126) (the
 * range of 1 + exp(-x) after the reference's clamp). *mismatches gets the
 * count, *first_bad the first differing d's bits (0 if none); both are host
 * pointers and the call synchronises the context's stream. */
OSC_API int osc_selfcheck_recip(osc_ctx* ctx, unsigned long long* mismatches, unsigned int* first_bad);

/* Failure detection (no counterpart in the reference, which has no device
 * waits): every wait inside this library's kernels gives up after a bounded
 * time (about 1.5 s at full clock), sets the context's device error word and
 * lets the kernel return, so a wait that can never complete reports an error
 * instead of hanging the GPU. This call enqueues a kernel whose wait cannot
 * complete, without faulting anything: which = 0 is the grid barrier of the
 * DynamicQuantizeLinear kernel told to expect one CTA more than it launched;
 * which = 1 an mbarrier no thread arrives on. The next osc_synchronize then
 * returns OSC_ETIMEDOUT and clears the error word and the barrier counters, and
 * the context stays usable. */
OSC_API int osc_selfcheck_timeout(osc_ctx* ctx, int which);

#ifdef __cplusplus
}
#endif

#endif /* ONNXSHARP_CUDA_H */
