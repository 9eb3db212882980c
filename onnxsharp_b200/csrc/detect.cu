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

// One CTA per image.
__global__ void __launch_bounds__(kDetThreads, 1)
    k_yolo_detect(const float* __restrict__ outputs, const __grid_constant__ DetectArgs d, float* __restrict__ dets,
                  int* __restrict__ counts) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  extern __shared__ __align__(16) uint8_t smem_det[];
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_det);  // [kMaxAnchors]
  Box* kept = reinterpret_cast<Box*>(keys + kMaxAnchors);                     // [kMaxKeep]
  __shared__ int n_cand, n_kept;
  const int img = blockIdx.x, tid = threadIdx.x;
  const float* out = outputs + static_cast<size_t>(img) * d.fields * d.anchors;
  if (tid == 0) n_cand = 0;
  __syncthreads();
  // 1. per anchor: first maximum over the class fields, confidence and box checks
  for (int a = tid; a < d.anchors; a += kDetThreads) {
    float score = -INFINITY;
    int cls = 0;
    for (int c = 4; c < d.fields; ++c) {
      const float v = out[static_cast<size_t>(c) * d.anchors + a];
      if (v > score) {
        score = v;
        cls = c - 4;
      }
    }
    if (!isfinite(score) || score < d.conf) continue;
    const float x = out[a], y = out[d.anchors + a], w = out[2 * d.anchors + a], h = out[3 * d.anchors + a];
    if (!isfinite(x) || !isfinite(y) || !isfinite(w) || !isfinite(h) || w <= 0.0f || h <= 0.0f) continue;
    const int slot = atomicAdd(&n_cand, 1);
    // descending score, then ascending anchor: sort ascending on (~score key, anchor, class)
    keys[slot] = (static_cast<unsigned long long>(~orderable(score)) << 32) |
                 (static_cast<unsigned long long>(a) << 16) | static_cast<unsigned long long>(cls);
  }
  __syncthreads();
  const int nc = n_cand;
  int np2 = 1;
  while (np2 < nc) np2 <<= 1;
  for (int i = nc + tid; i < np2; i += kDetThreads) keys[i] = ~0ull;
  __syncthreads();
  // 2. bitonic sort of keys[0, np2)
  for (int k = 2; k <= np2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np2; i += kDetThreads) {
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
  // 3. greedy NMS in score order, a chunk of kDetThreads candidates at a time
  // (one per thread). A candidate is suppressed when its IoU with a kept box of
  // its class (any class if class_agnostic) exceeds the threshold. Each thread
  // first tests its candidate against the boxes kept from earlier chunks; then
  // the chunk is resolved in order: the lowest-index surviving candidate is
  // kept and every later candidate of the chunk is tested against it, until no
  // candidate survives. The decisions are those of the one-at-a-time greedy
  // loop (DetectionNms.SuppressSorted): each candidate meets exactly the boxes
  // kept before it, in the same order, and the loop stops at max_det kept.
  const int ncand = min(nc, d.max_candidates);
  const int keep_cap = min(d.max_det, kMaxKeep);
  __shared__ unsigned alive_mask[kDetThreads / 32];
  const int lane = tid & 31, warp = tid >> 5;
  int nk = 0;  // uniform across the CTA
  for (int base = 0; base < ncand && nk < keep_cap; base += kDetThreads) {
    const int i = base + tid;
    bool alive = i < ncand;
    Box cb{};
    if (alive) {
      const unsigned long long key = keys[i];
      const int a = static_cast<int>((key >> 16) & 0xFFFFull);
      const int cls = static_cast<int>(key & 0xFFFFull);
      cb = cand_box(out, d.anchors, a, cls, out[static_cast<size_t>(4 + cls) * d.anchors + a]);
      for (int j = 0; j < nk && alive; ++j) {
        const Box kb = kept[j];
        if ((d.class_agnostic || kb.cls == cls) && iou_ref(kb, cb) > d.iou) alive = false;
      }
    }
    for (;;) {
      const unsigned m = __ballot_sync(0xffffffffu, alive);
      if (lane == 0) alive_mask[warp] = m;
      __syncthreads();
      int first = -1;
      for (int w = 0; w < kDetThreads / 32; ++w) {
        const unsigned mw = alive_mask[w];
        if (mw != 0u) {
          first = w * 32 + __ffs(mw) - 1;
          break;
        }
      }
      __syncthreads();  // every thread has read the masks before they are rewritten
      if (first < 0) break;
      if (tid == first) {
        kept[nk] = cb;
        alive = false;
      }
      __syncthreads();
      const Box kb = kept[nk];
      ++nk;
      if (nk >= keep_cap) break;
      if (alive && tid > first && (d.class_agnostic || kb.cls == cb.cls) && iou_ref(kb, cb) > d.iou) alive = false;
    }
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
  const int smem = kMaxAnchors * 8 + kMaxKeep * static_cast<int>(sizeof(Box));
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_yolo_detect), smem));
  return launch_pdl(ctx, k_yolo_detect, dim3(B), dim3(kDetThreads), smem, "k_yolo_detect", output, d, dets, counts);
}

}  // extern "C"
