// detect.cu — the steps either side of the YOLO forward pass, on the device:
// letterbox pre-processing of u8 frames into the [B, 3, H, W] input, and the
// detect tail (argmax, confidence filter, score sort, greedy NMS, mapping
// back to source pixels), so a batch crosses PCIe as frames in and
// detections out instead of two FP32 tensors.
//
// Letterbox: ImagePreprocessor.Letterbox (src/OnnxSharp/Vision/
// ImagePreprocessor.cs:57-100) = ImageGeometry.Contain (Imaging/AxisMap.cs:
// 97-112) + AxisMap.Bilinear (:22-40) + ImageTensor.ToChw (Imaging/
// ImageTensor.cs:13-170) with Divide255 normalisation and pad 114/255. Every
// float operation is the reference's, in its order, with explicit rounding,
// so the tensor is bit-identical.
//
// Detect: YoloDecoder.Decode (Vision/YoloDecoder.cs:68-188) +
// DetectionNms.SuppressSorted (Vision/Detection.cs:62-107) on the
// channels-first [4 + nc, A] output. Candidates are ordered by score
// (descending), ties by anchor index (the reference's List.Sort is
// unstable, so ties have no single reference order; this is the stable one).
#include <algorithm>
#include <cmath>

#include "runtime.h"

namespace osc {
namespace {

// ---------------------------------------------------------------- letterbox
struct LetterboxArgs {
  int width, height, row_stride, bpp, bgr;
  int tw, th, rw, rh, ox, oy;
  float pad, gain, bias;
};

// One image per blockIdx.y: image z reads px + z * px_stride bytes and writes
// dst + z * dst_stride floats.
__global__ void k_letterbox(const uint8_t* __restrict__ px, const __grid_constant__ LetterboxArgs a,
                            float* __restrict__ dst, long long px_stride, long long dst_stride) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  const long plane = static_cast<long>(a.th) * a.tw;
  px += blockIdx.y * px_stride;
  dst += blockIdx.y * dst_stride;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < plane;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int y = static_cast<int>(i / a.tw), x = static_cast<int>(i - static_cast<long>(y) * a.tw);
    const int dx = x - a.ox, dy = y - a.oy;
    if (dx < 0 || dx >= a.rw || dy < 0 || dy >= a.rh) {
      dst[i] = a.pad;
      dst[plane + i] = a.pad;
      dst[2 * plane + i] = a.pad;
      continue;
    }
    // AxisMap.Bilinear: sample = clamp((i + 0.5) * src / dst - 0.5, 0, src - 1)
    float sy = __fsub_rn(__fdiv_rn(__fmul_rn(__fadd_rn(static_cast<float>(dy), 0.5f), static_cast<float>(a.height)),
                                   static_cast<float>(a.rh)),
                         0.5f);
    sy = fminf(fmaxf(sy, 0.0f), static_cast<float>(a.height - 1));
    float sx = __fsub_rn(__fdiv_rn(__fmul_rn(__fadd_rn(static_cast<float>(dx), 0.5f), static_cast<float>(a.width)),
                                   static_cast<float>(a.rw)),
                         0.5f);
    sx = fminf(fmaxf(sx, 0.0f), static_cast<float>(a.width - 1));
    const int y0 = static_cast<int>(sy), y1 = min(y0 + 1, a.height - 1);
    const int x0 = static_cast<int>(sx), x1 = min(x0 + 1, a.width - 1);
    const float fy = __fsub_rn(sy, static_cast<float>(y0)), omfy = __fsub_rn(1.0f, fy);
    const float fx = __fsub_rn(sx, static_cast<float>(x0)), omfx = __fsub_rn(1.0f, fx);
    const uint8_t* top = px + static_cast<size_t>(y0) * a.row_stride;
    const uint8_t* bot = px + static_cast<size_t>(y1) * a.row_stride;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const int co = a.bgr ? 2 - c : c;
      const float t = __fadd_rn(__fmul_rn(static_cast<float>(top[x0 * a.bpp + co]), omfx),
                                __fmul_rn(static_cast<float>(top[x1 * a.bpp + co]), fx));
      const float b = __fadd_rn(__fmul_rn(static_cast<float>(bot[x0 * a.bpp + co]), omfx),
                                __fmul_rn(static_cast<float>(bot[x1 * a.bpp + co]), fx));
      const float v = __fadd_rn(__fmul_rn(t, omfy), __fmul_rn(b, fy));
      dst[c * plane + i] = __fadd_rn(__fmul_rn(v, a.gain), a.bias);
    }
  }
}

// ---------------------------------------------------------------- detect
constexpr int kDetThreads = 1024;
constexpr int kMaxAnchors = 16384;  // sort capacity (YOLO11 at 640: 8400)
constexpr int kMaxKeep = 1024;

struct DetectArgs {
  int fields, anchors;  // channels-first [fields][anchors] per image, fields = 4 + classes
  float conf, iou;
  int max_det, max_candidates, class_agnostic;
  const float* transforms;  // [B][6]: resized_w, resized_h, offset_x, offset_y, source_w, source_h (or null)
};

// Order-preserving float -> u32 (larger float, larger key).
__device__ __forceinline__ uint32_t orderable(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct Box {
  float x, y, w, h, score;
  int cls;
};

// Detection.IoU (Detection.cs:31-50) with its rounding: a = kept box, b = candidate.
__device__ __forceinline__ float iou_ref(const Box& a, const Box& b) {
  const float x1 = fmaxf(a.x, b.x), y1 = fmaxf(a.y, b.y);
  const float x2 = fminf(__fadd_rn(a.x, a.w), __fadd_rn(b.x, b.w));
  const float y2 = fminf(__fadd_rn(a.y, a.h), __fadd_rn(b.y, b.h));
  const float iw = __fsub_rn(x2, x1), ih = __fsub_rn(y2, y1);
  if (iw <= 0.0f || ih <= 0.0f) return 0.0f;
  const float inter = __fmul_rn(iw, ih);
  const float uni = __fsub_rn(__fadd_rn(__fmul_rn(a.w, a.h), __fmul_rn(b.w, b.h)), inter);
  return uni <= 0.0f ? 0.0f : __fdiv_rn(inter, uni);
}

__device__ __forceinline__ Box cand_box(const float* __restrict__ out, int anchors, int a, int cls, float score) {
  const float cx = out[a], cy = out[anchors + a], w = out[2 * anchors + a], h = out[3 * anchors + a];
  Box b;
  b.score = score;
  b.x = __fsub_rn(cx, __fmul_rn(w, 0.5f));
  b.y = __fsub_rn(cy, __fmul_rn(h, 0.5f));
  b.w = w;
  b.h = h;
  b.cls = cls;
  return b;
}

// Candidate key of an anchor (YoloDecoder.Decode's filter): the first
// maximum over the class fields, then the confidence and box checks. Keys sort
// ascending in (descending score, ascending anchor) order.
__device__ __forceinline__ bool anchor_key(const float* __restrict__ out, const DetectArgs& d, int a,
                                           unsigned long long* key) {
  float score = -INFINITY;
  int cls = 0;
  for (int c = 4; c < d.fields; ++c) {
    const float v = out[static_cast<size_t>(c) * d.anchors + a];
    if (v > score) {
      score = v;
      cls = c - 4;
    }
  }
  if (!isfinite(score) || score < d.conf) return false;
  const float x = out[a], y = out[d.anchors + a], w = out[2 * d.anchors + a], h = out[3 * d.anchors + a];
  if (!isfinite(x) || !isfinite(y) || !isfinite(w) || !isfinite(h) || w <= 0.0f || h <= 0.0f) return false;
  *key = (static_cast<unsigned long long>(~orderable(score)) << 32) | (static_cast<unsigned long long>(a) << 16) |
         static_cast<unsigned long long>(cls);
  return true;
}

// 1. Candidates of every image at once: blockIdx.x = image, blockIdx.y = a
// block of 256 anchors (the class scan reads the whole [fields][anchors]
// output, so it is spread over the SMs rather than one CTA per image). Keys are
// appended to the image's list with one atomic per warp; their order there is
// arbitrary, the sort makes it unique (keys are distinct).
__global__ void __launch_bounds__(256) k_det_candidates(const float* __restrict__ outputs,
                                                        const __grid_constant__ DetectArgs d,
                                                        unsigned long long* __restrict__ keys,
                                                        int* __restrict__ n_cand) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  const int img = blockIdx.x, lane = threadIdx.x & 31;
  const int a = blockIdx.y * 256 + threadIdx.x;
  const float* out = outputs + static_cast<size_t>(img) * d.fields * d.anchors;
  unsigned long long key = 0;
  const bool ok = a < d.anchors && anchor_key(out, d, a, &key);
  const unsigned m = __ballot_sync(0xffffffffu, ok);
  int base = 0;
  if (lane == 0 && m != 0u) base = atomicAdd(n_cand + img, __popc(m));
  base = __shfl_sync(0xffffffffu, base, 0);
  if (ok) keys[static_cast<size_t>(img) * d.anchors + base + __popc(m & ((1u << lane) - 1u))] = key;
}

// Bitonic sort (ascending) of n = E * kDetThreads keys, thread t holding keys
// t*E .. t*E+E-1 in registers: compare-exchange partners inside a thread are
// register pairs, partners up to 32*E apart are lanes of the same warp
// (shuffles), and only the strides of 32*E and more go through shared memory
// (one store, one load and two barriers per stride, XOR-swizzled so a warp's
// 64-bit accesses take the minimum two wavefronts). The network is the same
// as the plain shared-memory one, so is the result.
template <int E>
__device__ void sort_keys_regs(unsigned long long* keys, const unsigned long long* __restrict__ src, int nsrc) {
  const int t = threadIdx.x;
  const int sw = ((t * E) >> 4) & (E - 1);  // swizzle of this thread's slots
  unsigned long long r[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = t * E + e;
    r[e] = i < nsrc ? src[i] : ~0ull;
  }
  const int n = E * kDetThreads;
  for (int k = 2; k <= n; k <<= 1) {
    const bool up = ((t * E) & k) == 0;  // k >= 2E here whenever it is used below (k > j >= E)
    int j = k >> 1;
    for (; j >= 32 * E; j >>= 1) {
      __syncthreads();  // the previous stride's loads are done
#pragma unroll
      for (int e = 0; e < E; ++e) keys[t * E + (e ^ sw)] = r[e];
      __syncthreads();
      const int tp = t ^ (j / E);  // partner thread: same slot e, same swizzle (j / E >= 32)
      const bool lower = (t & (j / E)) == 0;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const unsigned long long o = keys[tp * E + (e ^ sw)];
        r[e] = (lower == up) ? (r[e] < o ? r[e] : o) : (r[e] > o ? r[e] : o);
      }
    }
    for (; j >= E; j >>= 1) {
      const int lm = j / E;  // lane distance (< 32)
      const bool lower = (t & lm) == 0;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, r[e], lm);
        r[e] = (lower == up) ? (r[e] < o ? r[e] : o) : (r[e] > o ? r[e] : o);
      }
    }
#pragma unroll
    for (int jj = E / 2; jj >= 1; jj >>= 1) {
      if (jj > (k >> 1)) continue;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if ((e & jj) != 0) continue;
        const int f = e | jj;
        const bool u = ((t * E + e) & k) == 0;
        if ((r[e] > r[f]) == u) {
          const unsigned long long x = r[e];
          r[e] = r[f];
          r[f] = x;
        }
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < E; ++e) keys[t * E + e] = r[e];
  __syncthreads();
}

// Plain shared-memory bitonic sort for short lists (n < kDetThreads).
__device__ void sort_keys_smem(unsigned long long* keys, const unsigned long long* __restrict__ src, int nsrc,
                               int n) {
  const int tid = threadIdx.x;
  for (int i = tid; i < n; i += kDetThreads) keys[i] = i < nsrc ? src[i] : ~0ull;
  __syncthreads();
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < n; i += kDetThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = keys[i], b = keys[ixj];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            keys[i] = b;
            keys[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

constexpr int kChunk = 256;              // candidates resolved per NMS round
constexpr int kChunkWords = kChunk / 32;

// 2-4. One CTA per image: sort its candidate keys, greedy NMS, output.
__global__ void __launch_bounds__(kDetThreads, 1)
    k_yolo_detect(const float* __restrict__ outputs, const __grid_constant__ DetectArgs d,
                  const unsigned long long* __restrict__ cand_keys, const int* __restrict__ n_cand,
                  float* __restrict__ dets, int* __restrict__ counts) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  extern __shared__ __align__(16) uint8_t smem_det[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_det);  // [kMaxAnchors]
  Box* kept = reinterpret_cast<Box*>(keys + kMaxAnchors);                     // [kMaxKeep]
  Box* cbox = kept + kMaxKeep;                                                // [kChunk]
  uint32_t* mat = reinterpret_cast<uint32_t*>(cbox + kChunk);                 // [kChunk][kChunkWords]
  uint32_t* removed0 = mat + kChunk * kChunkWords;                            // [kChunkWords]
  __shared__ int n_kept;
  const int img = blockIdx.x, tid = threadIdx.x;
  const float* out = outputs + static_cast<size_t>(img) * d.fields * d.anchors;
  const int nc = min(n_cand[img], d.anchors);
  const unsigned long long* src = cand_keys + static_cast<size_t>(img) * d.anchors;
  // 2. sort the keys (a power-of-two network, padded with ~0)
  int np2 = 1;
  while (np2 < nc) np2 <<= 1;
  switch (np2 / kDetThreads) {
    case 0: sort_keys_smem(keys, src, nc, np2); break;
    case 1: sort_keys_regs<1>(keys, src, nc); break;
    case 2: sort_keys_regs<2>(keys, src, nc); break;
    case 4: sort_keys_regs<4>(keys, src, nc); break;
    case 8: sort_keys_regs<8>(keys, src, nc); break;
    default: sort_keys_regs<16>(keys, src, nc); break;
  }
  // 3. greedy NMS in score order (DetectionNms.SuppressSorted), kChunk
  // candidates per round. A candidate is suppressed when its IoU with a kept
  // box of its class (any class if class_agnostic) exceeds the threshold.
  //  a. each candidate is tested against the boxes kept in earlier rounds
  //     (4 threads per candidate, every 4th kept box each);
  //  b. the round's suppression matrix: bit j of row i is set when candidate
  //     i, kept, would suppress the later candidate j (iou_ref(i, j), the
  //     kept box first, as in the one-at-a-time loop);
  //  c. one warp walks the round in order: the first candidate not yet
  //     removed is kept and its row is ORed into the removed set.
  // Each candidate thus meets exactly the boxes kept before it, in order, and
  // the loop stops at max_det kept: the one-at-a-time greedy loop's decisions.
  const int ncand = min(nc, d.max_candidates);
  const int keep_cap = min(d.max_det, kMaxKeep);
  const int lane = tid & 31, warp = tid >> 5;
  int nk = 0;  // uniform across the CTA
  for (int base = 0; base < ncand && nk < keep_cap; base += kChunk) {
    const int cnt = min(kChunk, ncand - base);
    if (tid < kChunkWords) removed0[tid] = 0u;
    __syncthreads();
    {
      const int c = tid >> 2, q = tid & 3;  // candidate base + c (c < kChunk), quarter q
      bool sup = false;
      Box cb{};
      if (c < cnt) {
        const unsigned long long key = keys[base + c];
        const int a = static_cast<int>((key >> 16) & 0xFFFFull);
        const int cls = static_cast<int>(key & 0xFFFFull);
        cb = cand_box(out, d.anchors, a, cls, out[static_cast<size_t>(4 + cls) * d.anchors + a]);
        for (int j = q; j < nk && !sup; j += 4) {
          const Box kb = kept[j];
          if ((d.class_agnostic || kb.cls == cls) && iou_ref(kb, cb) > d.iou) sup = true;
        }
      }
      sup = __shfl_xor_sync(0xffffffffu, sup, 1) || sup;
      sup = __shfl_xor_sync(0xffffffffu, sup, 2) || sup;
      if (q == 0) {
        cbox[c] = cb;
        if (c >= cnt || sup) atomicOr(removed0 + (c >> 5), 1u << (c & 31));
      }
    }
    __syncthreads();
    {
      const int i = tid >> 2, w0 = (tid & 3) * 2;  // row i, words w0 and w0 + 1
      const bool row_live = i < cnt && ((removed0[i >> 5] >> (i & 31)) & 1u) == 0u;
      const Box ci = cbox[i];
#pragma unroll
      for (int ww = 0; ww < 2; ++ww) {
        const int w = w0 + ww;
        uint32_t bits = 0u;
        if (row_live && w * 32 + 31 > i) {
          for (int b = 0; b < 32; ++b) {
            const int j = w * 32 + b;
            if (j <= i || j >= cnt) continue;
            const Box bj = cbox[j];
            if ((d.class_agnostic || ci.cls == bj.cls) && iou_ref(ci, bj) > d.iou) bits |= 1u << b;
          }
        }
        mat[i * kChunkWords + w] = bits;
      }
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t rem = lane < kChunkWords ? removed0[lane] : 0xffffffffu;
      int n = nk;
      for (int w = 0; w < kChunkWords && n < keep_cap; ++w) {
        uint32_t avail = ~__shfl_sync(0xffffffffu, rem, w);
        while (avail != 0u && n < keep_cap) {
          const int b = __ffs(avail) - 1;
          const int i = w * 32 + b;
          if (lane == 0) kept[n] = cbox[i];
          ++n;
          if (lane < kChunkWords) rem |= mat[i * kChunkWords + lane];
          avail = ~__shfl_sync(0xffffffffu, rem, w) & ~((2u << b) - 1u);  // later bits of this word
        }
      }
      if (lane == 0) n_kept = n;
    }
    __syncthreads();
    nk = n_kept;
  }
  if (tid == 0) n_kept = nk;
  __syncthreads();
  // 4. back to source pixels (Letterbox.ToSourceX/Y), clamped; zero-area boxes dropped (keeps order)
  if (tid == 0) {
    const int nk = n_kept;
    float* o = dets + static_cast<size_t>(img) * d.max_det * 6;
    int w = 0;
    const float* tf = d.transforms ? d.transforms + img * 6 : nullptr;
    for (int j = 0; j < nk; ++j) {
      const Box b = kept[j];
      float x1 = b.x, y1 = b.y, x2 = __fadd_rn(b.x, b.w), y2 = __fadd_rn(b.y, b.h);
      if (tf) {
        const float sx = __fdiv_rn(tf[0], tf[4]), sy = __fdiv_rn(tf[1], tf[5]);
        x1 = fminf(fmaxf(__fdiv_rn(__fsub_rn(x1, tf[2]), sx), 0.0f), tf[4]);
        y1 = fminf(fmaxf(__fdiv_rn(__fsub_rn(y1, tf[3]), sy), 0.0f), tf[5]);
        x2 = fminf(fmaxf(__fdiv_rn(__fsub_rn(x2, tf[2]), sx), 0.0f), tf[4]);
        y2 = fminf(fmaxf(__fdiv_rn(__fsub_rn(y2, tf[3]), sy), 0.0f), tf[5]);
        if (x2 <= x1 || y2 <= y1) continue;
        o[w * 6 + 2] = x1;
        o[w * 6 + 3] = y1;
        o[w * 6 + 4] = __fsub_rn(x2, x1);
        o[w * 6 + 5] = __fsub_rn(y2, y1);
      } else {
        o[w * 6 + 2] = b.x;
        o[w * 6 + 3] = b.y;
        o[w * 6 + 4] = b.w;
        o[w * 6 + 5] = b.h;
      }
      o[w * 6 + 0] = static_cast<float>(b.cls);
      o[w * 6 + 1] = b.score;
      ++w;
    }
    counts[img] = w;
  }
}

}  // namespace
}  // namespace osc

using namespace osc;

namespace {

// ImageGeometry.Contain (Imaging/AxisMap.cs:97-112) in the reference's float
// arithmetic, plus the Divide255 normalisation and the 114 grey pad.
int letterbox_args(int width, int height, int row_stride, int bytes_per_pixel, int bgr, int target_w, int target_h,
                   LetterboxArgs* a) {
  if (width <= 0 || height <= 0 || target_w <= 0 || target_h <= 0 || (bytes_per_pixel != 3 && bytes_per_pixel != 4))
    return fail(OSC_EINVAL, "letterbox: bad geometry");
  if (row_stride < width * bytes_per_pixel) return fail(OSC_EINVAL, "letterbox: row_stride %d", row_stride);
  const float gx = static_cast<float>(target_w) / static_cast<float>(width);
  const float gy = static_cast<float>(target_h) / static_cast<float>(height);
  const float gain = std::min(gx, gy);
  const int rw = std::clamp(static_cast<int>(std::nearbyint(static_cast<float>(width) * gain)), 1, target_w);
  const int rh = std::clamp(static_cast<int>(std::nearbyint(static_cast<float>(height) * gain)), 1, target_h);
  *a = LetterboxArgs{};
  a->width = width;
  a->height = height;
  a->row_stride = row_stride;
  a->bpp = bytes_per_pixel;
  a->bgr = bgr ? 1 : 0;
  a->tw = target_w;
  a->th = target_h;
  a->rw = rw;
  a->rh = rh;
  a->ox = (target_w - rw) / 2;
  a->oy = (target_h - rh) / 2;
  a->pad = 114.0f / 255.0f;
  a->gain = 1.0f / (255.0f * 1.0f);  // Divide255: 1 / (255 * std)
  a->bias = -0.0f / 1.0f;            // -mean / std
  return OSC_OK;
}

int letterbox_launch(osc_ctx* ctx, const uint8_t* pixels, int B, long long image_stride, const LetterboxArgs& a,
                     float* dst, long long dst_stride, int* placement) {
  if (placement != nullptr) {
    placement[0] = a.rw;
    placement[1] = a.rh;
    placement[2] = a.ox;
    placement[3] = a.oy;
  }
  const long plane = static_cast<long>(a.th) * a.tw;
  long blocks = std::min<long>((plane + 255) / 256, static_cast<long>(ctx->num_sms) * 16);
  blocks = std::max<long>(1, std::min<long>(blocks, (static_cast<long>(ctx->num_sms) * 16 + B - 1) / B));
  return launch_pdl(ctx, k_letterbox, dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(B)), dim3(256), 0,
                    "k_letterbox", pixels, a, dst, image_stride, dst_stride);
}

}  // namespace

extern "C" {

OSC_API int osc_letterbox_u8(osc_ctx* ctx, const uint8_t* pixels, int width, int height, int row_stride,
                             int bytes_per_pixel, int bgr, int target_w, int target_h, float* dst, int* placement) {
  OSC_TRY(enter(ctx));
  if (row_stride == 0) row_stride = width * bytes_per_pixel;
  LetterboxArgs a;
  OSC_TRY(letterbox_args(width, height, row_stride, bytes_per_pixel, bgr, target_w, target_h, &a));
  if (pixels == nullptr || dst == nullptr) return fail(OSC_EINVAL, "osc_letterbox_u8: null pointer");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  return letterbox_launch(ctx, pixels, 1, 0, a, dst, 0, placement);
}

OSC_API int osc_letterbox_batch_u8(osc_ctx* ctx, const uint8_t* pixels, int B, long long image_stride, int width,
                                   int height, int row_stride, int bytes_per_pixel, int bgr, int target_w,
                                   int target_h, float* dst, long long dst_nstride, int* placement) {
  OSC_TRY(enter(ctx));
  if (B < 0 || B > 65535) return fail(OSC_EINVAL, "osc_letterbox_batch_u8: B=%d", B);
  if (row_stride == 0) row_stride = width * bytes_per_pixel;
  LetterboxArgs a;
  OSC_TRY(letterbox_args(width, height, row_stride, bytes_per_pixel, bgr, target_w, target_h, &a));
  if (image_stride == 0) image_stride = static_cast<long long>(row_stride) * height;
  if (dst_nstride == 0) dst_nstride = 3ll * target_w * target_h;
  if (image_stride < static_cast<long long>(row_stride) * height || dst_nstride < 3ll * target_w * target_h)
    return fail(OSC_EINVAL, "osc_letterbox_batch_u8: image_stride %lld / dst_nstride %lld too small", image_stride,
                dst_nstride);
  if (B == 0) return OSC_OK;
  if (pixels == nullptr || dst == nullptr) return fail(OSC_EINVAL, "osc_letterbox_batch_u8: null pointer");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  return letterbox_launch(ctx, pixels, B, image_stride, a, dst, dst_nstride, placement);
}

OSC_API int osc_yolo_detect_f32(osc_ctx* ctx, const float* output, int B, int fields, int anchors, float conf,
                                float iou, int max_det, int max_candidates, int class_agnostic,
                                const float* transforms, float* dets, int* counts) {
  OSC_TRY(enter(ctx));
  if (B < 0 || fields < 5 || anchors <= 0 || max_det <= 0 || max_candidates <= 0)
    return fail(OSC_EINVAL, "osc_yolo_detect_f32: bad arguments");
  if (anchors > kMaxAnchors) return fail(OSC_EUNSUPPORTED, "osc_yolo_detect_f32: %d anchors > %d", anchors, kMaxAnchors);
  if (max_det > kMaxKeep) return fail(OSC_EUNSUPPORTED, "osc_yolo_detect_f32: max_det %d > %d", max_det, kMaxKeep);
  if (fields - 4 > 65535) return fail(OSC_EUNSUPPORTED, "osc_yolo_detect_f32: %d classes > 65535", fields - 4);
  if (B == 0) return OSC_OK;
  if (output == nullptr || dets == nullptr || counts == nullptr)
    return fail(OSC_EINVAL, "osc_yolo_detect_f32: null pointer");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  DetectArgs d{fields, anchors, conf, iou, max_det, max_candidates, class_agnostic ? 1 : 0, transforms};
  // candidate keys [B][anchors] and their counts [B] in the scratch arena
  const size_t key_bytes = round_up(static_cast<size_t>(B) * anchors * 8, 256);
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, key_bytes + static_cast<size_t>(B) * sizeof(int), &buf));
  auto* cand_keys = static_cast<unsigned long long*>(buf);
  int* n_cand = reinterpret_cast<int*>(static_cast<uint8_t*>(buf) + key_bytes);
  OSC_CUDA(cudaMemsetAsync(n_cand, 0, static_cast<size_t>(B) * sizeof(int), ctx->stream), "cudaMemsetAsync (detect)");
  OSC_TRY(launch_pdl(ctx, k_det_candidates, dim3(static_cast<unsigned>(B), static_cast<unsigned>((anchors + 255) / 256)),
                     dim3(256), 0, "k_det_candidates", output, d, cand_keys, n_cand));
  const int smem = kMaxAnchors * 8 + (kMaxKeep + kChunk) * static_cast<int>(sizeof(Box)) +
                   (kChunk + 1) * kChunkWords * static_cast<int>(sizeof(uint32_t));
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_yolo_detect), smem));
  return launch_pdl(ctx, k_yolo_detect, dim3(static_cast<unsigned>(B)), dim3(kDetThreads), smem, "k_yolo_detect",
                    output, d, cand_keys, n_cand, dets, counts);
}

}  // extern "C"
