// plan.cu — the static-plan executor behind osc_plan_*: the device
// counterpart of the reference's NetImpl.PrepareForGraph / BufferAllocator /
// Interpreter.Run (src/OnnxSharp/Engine/NetImpl.cs:151-192,
// Engine/BufferAllocator.cs:41-138, Core/Interpreter.cs:30-186).
//
// A plan is a list of NCHW buffers (per-image C, H, W; the batch is the
// plan's) and a list of fused nodes that read and write CHANNEL SLICES of
// them, so a Concat is producers writing into slices of one buffer and a
// Split is slices of one buffer: no copies. At build time every buffer gets
// its live range (first write, last read) and the buffers are coloured into
// slots exactly as the reference's allocator does — ordered by first write
// (ties by index), each takes the slot whose previous occupant's last read is
// the LATEST one strictly before this buffer's first write, else a new slot —
// and the slots are laid out back to back (256-byte aligned) in ONE device
// arena. The graph input (the buffer marked as input) is not in the arena: it
// is the caller's pointer, as the reference references caller-owned input
// tensors without a copy (NetImpl.SetInput, NetImpl.cs:256-273).
//
// Run: the reference caches one plan per input signature
// (Core/LayerPlan.cs:32-94). Shapes here are fixed at build time, so the
// signature is the (input, output) pointer pair: the first run with a pair
// executes the nodes eagerly once (scratch sizes, kernel attributes), then
// captures them into a CUDA graph on the context's stream; later runs with
// that pair replay the graph (one launch per inference).
#include <algorithm>
#include <cstring>
#include <vector>

#include "runtime.h"

using namespace osc;

namespace {

struct PlanBuf {
  int c, h, w;
  long long off;  // byte offset in the arena (-1: the plan input, or never written)
};

struct CacheEntry {
  const float* in;
  float* out;
  osc_graph* graph;
};

constexpr size_t kArenaAlign = 256;
constexpr int kMaxCache = 8;

}  // namespace

struct osc_plan {
  osc_ctx* ctx = nullptr;
  int batch = 0;
  int input_buf = -1;
  std::vector<PlanBuf> bufs;
  std::vector<osc_plan_node> nodes;
  void* arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<CacheEntry> cache;
  // The plan runs and is captured on its own stream, ordered after the
  // caller's stream (ev_in) and before later work on it (ev_out), so a caller
  // on the legacy default stream can run it too.
  cudaStream_t stream = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
};

namespace {

// The reference's lifetime colouring (BufferAllocator.Assign, strict '<').
int assign_offsets(int n, const int* first, const int* last, const size_t* bytes, long long* offsets, size_t* total) {
  std::vector<int> order;
  for (int i = 0; i < n; ++i)
    if (first[i] >= 0) order.push_back(i);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return first[a] < first[b]; });
  std::vector<int> slot_of(n, -1);
  std::vector<int> free_at;       // last read of each slot's current occupant
  std::vector<size_t> slot_size;  // largest buffer of each slot
  for (int i : order) {
    const int start = first[i], end = std::max(last[i], start);
    int chosen = -1, best = 0;
    for (int s = 0; s < static_cast<int>(free_at.size()); ++s)
      if (free_at[s] < start && (chosen < 0 || free_at[s] > best)) {
        best = free_at[s];
        chosen = s;
      }
    if (chosen < 0) {
      chosen = static_cast<int>(free_at.size());
      free_at.push_back(end);
      slot_size.push_back(0);
    } else {
      free_at[chosen] = end;
    }
    slot_of[i] = chosen;
    slot_size[chosen] = std::max(slot_size[chosen], bytes[i]);
  }
  std::vector<size_t> base(slot_size.size());
  size_t off = 0;
  for (size_t s = 0; s < slot_size.size(); ++s) {
    base[s] = off;
    off += round_up(slot_size[s], kArenaAlign);
  }
  for (int i = 0; i < n; ++i) offsets[i] = slot_of[i] >= 0 ? static_cast<long long>(base[slot_of[i]]) : -1;
  *total = off;
  return OSC_OK;
}

int node_arity(int op, int* n_in_min, int* n_in_max, int* n_out) {
  *n_out = 1;
  switch (op) {
    case OSC_OP_CONV:
    case OSC_OP_CONV_DIRECT: *n_in_min = 1; *n_in_max = 2; return OSC_OK;  // x, optional residual
    case OSC_OP_MAXPOOL:
    case OSC_OP_RESIZE_NEAREST:
    case OSC_OP_PSA:
    case OSC_OP_MATMUL_BIAS:
    case OSC_OP_SOFTMAX:
    case OSC_OP_UNARY: *n_in_min = *n_in_max = 1; return OSC_OK;
    case OSC_OP_ATTENTION: *n_in_min = *n_in_max = 3; return OSC_OK;
    case OSC_OP_YOLO_DECODE: *n_in_min = *n_in_max = 6; *n_out = 0; return OSC_OK;  // writes the plan output
    default: return fail(OSC_EUNSUPPORTED, "osc_plan_build: op %d", op);
  }
}

struct View {
  float* p;
  long long nstride;  // elements between images
  int c, h, w;
};

View view_of(const osc_plan* pl, const osc_plan_ref& r, const float* input) {
  const PlanBuf& b = pl->bufs[r.buf];
  float* base = r.buf == pl->input_buf ? const_cast<float*>(input)
                                       : reinterpret_cast<float*>(static_cast<uint8_t*>(pl->arena) + b.off);
  const long long plane = static_cast<long long>(b.h) * b.w;
  return View{base + static_cast<long long>(r.c0) * plane, static_cast<long long>(b.c) * plane, r.c, b.h, b.w};
}

int run_nodes(osc_plan* pl, const float* input, float* output) {
  osc_ctx* ctx = pl->ctx;
  const int B = pl->batch;
  for (size_t ni = 0; ni < pl->nodes.size(); ++ni) {
    const osc_plan_node& n = pl->nodes[ni];
    const int* ia = n.iattr;
    int st = OSC_OK;
    switch (n.op) {
      case OSC_OP_CONV:
      case OSC_OP_CONV_DIRECT: {
        const View x = view_of(pl, n.in[0], input), y = view_of(pl, n.out[0], input);
        const View r = n.n_in > 1 ? view_of(pl, n.in[1], input) : View{nullptr, 0, 0, 0, 0};
        const int s = ia[0], p = ia[1], d = ia[2], act = ia[3];
        if (n.op == OSC_OP_CONV)
          st = osc_conv2d_ex_f32(ctx, x.p, x.nstride, B, x.c, x.h, x.w, static_cast<const osc_conv_weights*>(n.weights),
                                 s, s, p, p, p, p, d, d, n.bias, act, r.p, r.nstride, y.p, y.nstride, y.h, y.w);
        else
          st = osc_conv2d_direct_f32(ctx, x.p, x.nstride, B, x.c, x.h, x.w, static_cast<const float*>(n.weights), y.c,
                                     ia[4], ia[4], s, s, p, p, p, p, d, d, ia[5], n.bias, act, r.p, r.nstride, y.p,
                                     y.nstride, y.h, y.w);
        break;
      }
      case OSC_OP_MAXPOOL: {
        const View x = view_of(pl, n.in[0], input), y = view_of(pl, n.out[0], input);
        st = osc_maxpool2d_f32(ctx, x.p, x.nstride, B, x.c, x.h, x.w, ia[0], ia[0], ia[1], ia[1], ia[2], ia[2], ia[2],
                               ia[2], y.p, y.nstride, y.h, y.w);
        break;
      }
      case OSC_OP_RESIZE_NEAREST: {
        const View x = view_of(pl, n.in[0], input), y = view_of(pl, n.out[0], input);
        st = osc_resize_nearest_f32(ctx, x.p, x.nstride, B, x.c, x.h, x.w, ia[0], ia[0], y.p, y.nstride);
        break;
      }
      case OSC_OP_PSA: {
        const View x = view_of(pl, n.in[0], input), y = view_of(pl, n.out[0], input);
        st = osc_psa_attention_f32(ctx, x.p, x.nstride, B, ia[0], ia[1], ia[2], x.h * x.w, n.fattr[0], y.p, y.nstride);
        break;
      }
      case OSC_OP_YOLO_DECODE: {
        const float* box[3];
        const float* cls[3];
        long long bs[3], cs[3];
        int hs[3], ws[3];
        for (int i = 0; i < 3; ++i) {
          const View b = view_of(pl, n.in[i], input), c = view_of(pl, n.in[3 + i], input);
          box[i] = b.p;
          bs[i] = b.nstride;
          cls[i] = c.p;
          cs[i] = c.nstride;
          hs[i] = b.h;
          ws[i] = b.w;
        }
        st = osc_yolo_decode_f32(ctx, B, ia[0], box, bs, cls, cs, hs, ws, n.fattr, output);
        break;
      }
      case OSC_OP_MATMUL_BIAS: {  // rows = B*C*H of a dense buffer, k = W; out rows x n
        const View x = view_of(pl, n.in[0], input), y = view_of(pl, n.out[0], input);
        st = osc_gemm_bias_f32(ctx, x.p, B * x.c * x.h, x.w, x.w, static_cast<const osc_gemm_weights*>(n.weights),
                               n.bias, ia[3], y.p, y.w);
        break;
      }
      case OSC_OP_SOFTMAX: {
        const View x = view_of(pl, n.in[0], input), y = view_of(pl, n.out[0], input);
        st = osc_softmax_f32(ctx, x.p, y.p, static_cast<long long>(B) * x.c * x.h, x.w);
        break;
      }
      case OSC_OP_UNARY: {
        const View x = view_of(pl, n.in[0], input), y = view_of(pl, n.out[0], input);
        st = osc_unary_f32(ctx, x.p, y.p, static_cast<long long>(B) * x.c * x.h * x.w, ia[3]);
        break;
      }
      case OSC_OP_ATTENTION: {  // q, k, v [B, T = C, 1, heads * D = W]
        const View q = view_of(pl, n.in[0], input), k = view_of(pl, n.in[1], input);
        const View v = view_of(pl, n.in[2], input), y = view_of(pl, n.out[0], input);
        st = osc_attention_f32(ctx, q.p, k.p, v.p, nullptr, 0, B, q.c, ia[0], q.w / ia[0], n.fattr[0], 0, y.p);
        break;
      }
      default:
        st = fail(OSC_EUNSUPPORTED, "osc_plan_run: op %d", n.op);
    }
    if (st != OSC_OK) {
      const std::string msg = osc_last_error();
      return fail(st, "osc_plan node %zu (op %d): %s", ni, n.op, msg.c_str());
    }
  }
  return OSC_OK;
}

int validate(const osc_plan_desc* d) {
  if (d->batch < 1 || d->n_buffers < 1 || d->buf_chw == nullptr || d->n_nodes < 1 || d->nodes == nullptr)
    return fail(OSC_EINVAL, "osc_plan_build: empty plan");
  if (d->input_buf < 0 || d->input_buf >= d->n_buffers) return fail(OSC_EINVAL, "osc_plan_build: input buffer");
  for (int b = 0; b < d->n_buffers; ++b)
    if (d->buf_chw[3 * b] < 1 || d->buf_chw[3 * b + 1] < 1 || d->buf_chw[3 * b + 2] < 1)
      return fail(OSC_EINVAL, "osc_plan_build: buffer %d shape", b);
  for (int i = 0; i < d->n_nodes; ++i) {
    const osc_plan_node& n = d->nodes[i];
    int lo, hi, no;
    OSC_TRY(node_arity(n.op, &lo, &hi, &no));
    if (n.n_in < lo || n.n_in > hi || n.n_in > OSC_PLAN_MAX_IN || n.n_out != no)
      return fail(OSC_EINVAL, "osc_plan_build: node %d (op %d) has %d inputs / %d outputs", i, n.op, n.n_in, n.n_out);
    for (int j = 0; j < n.n_in + n.n_out; ++j) {
      const osc_plan_ref& r = j < n.n_in ? n.in[j] : n.out[j - n.n_in];
      if (r.buf < 0 || r.buf >= d->n_buffers || r.c0 < 0 || r.c < 1 || r.c0 + r.c > d->buf_chw[3 * r.buf])
        return fail(OSC_EINVAL, "osc_plan_build: node %d ref %d out of its buffer", i, j);
    }
    for (int j = 0; j < n.n_out; ++j)
      if (n.out[j].buf == d->input_buf) return fail(OSC_EINVAL, "osc_plan_build: node %d writes the plan input", i);
    const bool needs_w = n.op == OSC_OP_CONV || n.op == OSC_OP_CONV_DIRECT || n.op == OSC_OP_MATMUL_BIAS;
    if (needs_w && n.weights == nullptr) return fail(OSC_EINVAL, "osc_plan_build: node %d has no weights", i);
    if ((n.op == OSC_OP_MATMUL_BIAS || n.op == OSC_OP_SOFTMAX || n.op == OSC_OP_UNARY || n.op == OSC_OP_ATTENTION)) {
      for (int j = 0; j < n.n_in; ++j)
        if (n.in[j].c0 != 0 || n.in[j].c != d->buf_chw[3 * n.in[j].buf])
          return fail(OSC_EINVAL, "osc_plan_build: node %d (op %d) needs whole buffers", i, n.op);
      if (n.out[0].c0 != 0 || n.out[0].c != d->buf_chw[3 * n.out[0].buf])
        return fail(OSC_EINVAL, "osc_plan_build: node %d (op %d) needs a whole output buffer", i, n.op);
    }
    if (n.op == OSC_OP_ATTENTION && (n.iattr[0] < 1 || d->buf_chw[3 * n.in[0].buf + 2] % n.iattr[0] != 0))
      return fail(OSC_EINVAL, "osc_plan_build: node %d heads", i);
  }
  return OSC_OK;
}

// On the plan's stream (ctx->stream points at it): replay the graph cached for
// (input, output), or run the nodes once eagerly (sizes the scratch arena),
// capture them and cache the graph.
int plan_launch(osc_plan* plan, const float* input, float* output) {
  osc_ctx* ctx = plan->ctx;
  for (const CacheEntry& e : plan->cache)
    if (e.in == input && e.out == output) return osc_graph_launch(ctx, e.graph);
  OSC_TRY(run_nodes(plan, input, output));
  OSC_TRY(osc_synchronize(ctx, 0));
  OSC_TRY(osc_graph_begin(ctx));
  const int st = run_nodes(plan, input, output);
  osc_graph* g = nullptr;
  const int st2 = osc_graph_end(ctx, &g);
  if (st != OSC_OK) {
    osc_graph_free(g);
    return st;
  }
  if (st2 != OSC_OK) return st2;
  if (static_cast<int>(plan->cache.size()) >= kMaxCache) {
    osc_graph_free(plan->cache.front().graph);
    plan->cache.erase(plan->cache.begin());
  }
  plan->cache.push_back(CacheEntry{input, output, g});
  return osc_graph_launch(ctx, g);
}

}  // namespace

extern "C" {

OSC_API int osc_arena_assign(int n, const int* first_write, const int* last_read, const size_t* bytes,
                             long long* offsets, size_t* total) {
  if (n < 0 || (n > 0 && (first_write == nullptr || last_read == nullptr || bytes == nullptr || offsets == nullptr)) ||
      total == nullptr)
    return fail(OSC_EINVAL, "osc_arena_assign: bad arguments");
  return assign_offsets(n, first_write, last_read, bytes, offsets, total);
}

OSC_API int osc_plan_build(osc_ctx* ctx, const osc_plan_desc* desc, osc_plan** out) {
  if (out == nullptr || desc == nullptr) return fail(OSC_EINVAL, "osc_plan_build: null argument");
  *out = nullptr;
  OSC_TRY(enter(ctx));
  OSC_TRY(validate(desc));
  auto* pl = new osc_plan();
  pl->ctx = ctx;
  pl->batch = desc->batch;
  pl->input_buf = desc->input_buf;
  pl->nodes.assign(desc->nodes, desc->nodes + desc->n_nodes);
  const int nb = desc->n_buffers;
  // live ranges: node index of the first write and of the last read
  std::vector<int> first(nb, -1), last(nb, 0);
  for (int i = 0; i < desc->n_nodes; ++i) {
    const osc_plan_node& n = desc->nodes[i];
    for (int j = 0; j < n.n_out; ++j)
      if (first[n.out[j].buf] < 0) first[n.out[j].buf] = i;
    for (int j = 0; j < n.n_in; ++j) last[n.in[j].buf] = std::max(last[n.in[j].buf], i);
  }
  first[desc->input_buf] = -1;  // the caller's buffer, not the arena's
  std::vector<size_t> bytes(nb);
  for (int b = 0; b < nb; ++b)
    bytes[b] = static_cast<size_t>(desc->batch) * desc->buf_chw[3 * b] * desc->buf_chw[3 * b + 1] *
               desc->buf_chw[3 * b + 2] * sizeof(float);
  std::vector<long long> off(nb);
  size_t total = 0;
  assign_offsets(nb, first.data(), last.data(), bytes.data(), off.data(), &total);
  for (int b = 0; b < nb; ++b)
    pl->bufs.push_back(PlanBuf{desc->buf_chw[3 * b], desc->buf_chw[3 * b + 1], desc->buf_chw[3 * b + 2], off[b]});
  for (int i = 0; i < desc->n_nodes; ++i) {  // every buffer read must be written earlier (or be the input)
    const osc_plan_node& n = desc->nodes[i];
    for (int j = 0; j < n.n_in; ++j) {
      const int b = n.in[j].buf;
      if (b != desc->input_buf && (first[b] < 0 || first[b] >= i)) {
        delete pl;
        return fail(OSC_EINVAL, "osc_plan_build: node %d reads buffer %d before any node writes it", i, b);
      }
    }
  }
  if (fault_injected("alloc")) {
    delete pl;
    return fail(OSC_EFAULT_INJECTED, "injected allocation failure (plan arena)");
  }
  if (total > 0) {
    const cudaError_t e = cudaMalloc(&pl->arena, total);
    if (e != cudaSuccess) {
      cudaGetLastError();
      delete pl;
      return fail(OSC_ENOMEM, "osc_plan_build: arena of %zu bytes: %s", total, cudaGetErrorString(e));
    }
  }
  pl->arena_bytes = total;
  cudaError_t e = cudaStreamCreateWithFlags(&pl->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&pl->ev_in, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&pl->ev_out, cudaEventDisableTiming);
  if (e != cudaSuccess) {
    osc_plan_free(pl);
    return cuda_fail(e, "osc_plan_build: stream / events");
  }
  *out = pl;
  return OSC_OK;
}

OSC_API int osc_plan_arena_bytes(const osc_plan* plan, size_t* bytes) {
  if (plan == nullptr || bytes == nullptr) return fail(OSC_EINVAL, "osc_plan_arena_bytes: null argument");
  *bytes = plan->arena_bytes;
  return OSC_OK;
}

OSC_API int osc_plan_buffer(const osc_plan* plan, int buffer, const float* input, float** ptr, long long* nstride) {
  if (plan == nullptr || ptr == nullptr || buffer < 0 || buffer >= static_cast<int>(plan->bufs.size()))
    return fail(OSC_EINVAL, "osc_plan_buffer: bad arguments");
  const PlanBuf& b = plan->bufs[buffer];
  if (buffer != plan->input_buf && b.off < 0) return fail(OSC_EINVAL, "osc_plan_buffer: buffer %d is never written", buffer);
  const View v = view_of(plan, osc_plan_ref{buffer, 0, b.c}, input);
  *ptr = v.p;
  if (nstride) *nstride = v.nstride;
  return OSC_OK;
}

OSC_API int osc_plan_run(osc_plan* plan, const float* input, float* output) {
  if (plan == nullptr) return fail(OSC_EINVAL, "osc_plan_run: null plan");
  osc_ctx* ctx = plan->ctx;
  OSC_TRY(enter(ctx));
  if (input == nullptr) return fail(OSC_EINVAL, "osc_plan_run: null input");
  if (output == nullptr)
    for (const osc_plan_node& n : plan->nodes)
      if (n.op == OSC_OP_YOLO_DECODE) return fail(OSC_EINVAL, "osc_plan_run: the plan writes an output; got null");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  if (capturing(ctx)) return run_nodes(plan, input, output);  // the caller captures the whole plan itself
  cudaStream_t caller = ctx->stream;
  OSC_CUDA(cudaEventRecord(plan->ev_in, caller), "osc_plan_run: record");
  OSC_CUDA(cudaStreamWaitEvent(plan->stream, plan->ev_in, 0), "osc_plan_run: wait");
  ctx->stream = plan->stream;
  const int st = plan_launch(plan, input, output);
  ctx->stream = caller;
  if (st != OSC_OK) return st;
  OSC_CUDA(cudaEventRecord(plan->ev_out, plan->stream), "osc_plan_run: record");
  OSC_CUDA(cudaStreamWaitEvent(caller, plan->ev_out, 0), "osc_plan_run: wait");
  return OSC_OK;
}

OSC_API int osc_plan_free(osc_plan* plan) {
  if (plan == nullptr) return OSC_OK;
  cudaSetDevice(plan->ctx->device);
  if (plan->stream) cudaStreamSynchronize(plan->stream);
  for (CacheEntry& e : plan->cache) osc_graph_free(e.graph);
  if (plan->arena) cudaFree(plan->arena);
  if (plan->ev_in) cudaEventDestroy(plan->ev_in);
  if (plan->ev_out) cudaEventDestroy(plan->ev_out);
  if (plan->stream) cudaStreamDestroy(plan->stream);
  delete plan;
  return OSC_OK;
}

}  // extern "C"
