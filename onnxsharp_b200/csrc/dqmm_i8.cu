// dqmm_i8.cu — DynamicQuantizeMatMul on the sm_100a integer tensor cores.
//
// Replaces DynamicQuantizeMatMulLayer.Forward (src/OnnxSharp/Ops/
// QuantizedMatMulOps.cs:115-201), which fuses DynamicQuantizeLinear ->
// MatMulInteger -> Cast -> Mul -> Add:
//   1. (min, max) of A including 0, NaN skipped (Tensors/Quantization.cs:109-181)
//   2. scale = (max-min)/255 (1 if !(scale > 0)); zp = clamp(rne(-min/scale), 0, 255)
//      (QuantizedMatMulOps.cs:146-156)
//   3. q = clamp(rne(x * (1/scale)) + zp, 0, 255)        (QuantizeAndWiden :280-335)
//   4. acc = sum_t (q - zp)(w - wzp[j])  — exact integers (the reference
//      accumulates them in F32, exact while |partial sums| < 2^24)
//   5. y = acc * (scale * wscale[j]) + bias[j], as one FMA on the 16-column
//      panels of 12/6/4-row groups and as mul-then-add on tail columns and
//      leftover rows (GemmKernel.cs:1210-1241 vs ScaleColumns :1594-1608),
//      reproduced here element by element so y is bit-identical.
// Kernels: k_minmax_partial -> k_dql_params (1 thread) -> k_quantize_rows
// (u8 q, per-row sum of q, NaN-row flag) -> k_dqmm_i8 (TMA -> smem ->
// tcgen05.mma kind::i8, u8 x s8|u8 -> s32 in TMEM, then the corrections
// acc = sum(q*w) - wzp[j]*rowsum[i] - zp*colsum[j] + k*zp*wzp[j] and the
// epilogue above, coalesced stores through shared memory).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <vector>

#include "runtime.h"
#include "sm100.cuh"

struct osc_dqmm_weights {
  int device = 0;
  int k = 0, n = 0, kp = 0;  // kp: K padded to a multiple of 128 (one SW128 row of int8)
  int is_signed = 1;
  int8_t* wt = nullptr;       // [n][kp] raw weight bytes, transposed
  int32_t* colsum = nullptr;  // [n] sum_t w[t][j] (as signed/unsigned integers)
  int32_t* zp = nullptr;      // [n] weight zero point per column
  int has_zp = 0;             // any column has a non-zero weight zero point
};

namespace osc {
namespace {

constexpr int kQBM = 128, kQBN = 256, kQBK = 128, kQStages = 4;
constexpr int kQThreads = 64 + 8 * 32;  // producer, MMA, 8 epilogue warps
constexpr int kQA = kQBM * kQBK;        // 16 KB
constexpr int kQB = kQBN * kQBK;        // 32 KB
constexpr int kQStage = kQA + kQB;
constexpr int kQTiles = kQStages * kQStage;
constexpr int kQSmem = kQTiles + 1024 + 256;
static_assert(kQBM * (kQBN + 4) * 4 + 4 * kQBN * 4 + 2 * kQBM * 4 <= kQTiles, "staging + tile constants fit");

// Device-side quantisation parameters, written by k_dql_params.
struct QParams {
  float scale, inverse;
  int zp, pad;
};

__device__ __forceinline__ float maxps(float a, float b) { return a > b ? a : b; }
__device__ __forceinline__ float minps(float a, float b) { return a < b ? a : b; }

__global__ void k_minmax_partial(const float* __restrict__ a, long n, float2* __restrict__ part) {
  float mn = 0.0f, mx = 0.0f;  // 0 is always inside the range
  const long i4 = n / 4;
  const bool vec = (reinterpret_cast<uintptr_t>(a) & 15u) == 0;
  if (vec) {
    for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < i4;
         i += static_cast<long>(gridDim.x) * blockDim.x) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(a) + i);
      const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 4; ++t)
        if (e[t] == e[t]) {
          mn = fminf(mn, e[t]);
          mx = fmaxf(mx, e[t]);
        }
    }
  }
  for (long i = (vec ? i4 * 4 : 0) + blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float e = a[i];
    if (e == e) {
      mn = fminf(mn, e);
      mx = fmaxf(mx, e);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  __shared__ float smn[32], smx[32];
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    smn[w] = mn;
    smx[w] = mx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (blockDim.x >> 5); ++i) {
      mn = fminf(mn, smn[i]);
      mx = fmaxf(mx, smx[i]);
    }
    part[blockIdx.x] = make_float2(mn, mx);
  }
}

__global__ void k_minmax_final(const float2* __restrict__ part, int nparts, float* __restrict__ out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float mn = 0.0f, mx = 0.0f;
  for (int i = 0; i < nparts; ++i) {
    mn = fminf(mn, part[i].x);
    mx = fmaxf(mx, part[i].y);
  }
  out[0] = mn;
  out[1] = mx;
}

// Reduces the partials (or takes a caller-supplied global range) and derives
// scale / zero point exactly as the reference does.
__global__ void k_dql_params(const float2* __restrict__ part, int nparts, const float* __restrict__ override_mm,
                             QParams* __restrict__ out, float* __restrict__ params_out) {
  // One warp: strided partial reduction, then a shuffle tree (min/max are
  // order-independent, so the result equals a serial scan).
  float mn = 0.0f, mx = 0.0f;
  if (override_mm != nullptr) {
    mn = fminf(0.0f, override_mm[0]);
    mx = fmaxf(0.0f, override_mm[1]);
  } else {
    for (int i = threadIdx.x; i < nparts; i += 32) {
      const float2 p = part[i];
      mn = fminf(mn, p.x);
      mx = fmaxf(mx, p.y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
  }
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  float scale = __fdiv_rn(__fsub_rn(mx, mn), 255.0f);
  if (!(scale > 0.0f)) scale = 1.0f;
  const float z = rintf(__fdiv_rn(-mn, scale));
  int zp = (z != z) ? 0 : (z >= 2147483520.0f ? 2147483647 : (z <= -2147483648.0f ? (-2147483647 - 1) : static_cast<int>(z)));
  zp = zp < 0 ? 0 : (zp > 255 ? 255 : zp);
  QParams p;
  p.scale = scale;
  p.inverse = __fdiv_rn(1.0f, scale);
  p.zp = zp;
  p.pad = 0;
  *out = p;
  if (params_out != nullptr) {
    params_out[0] = scale;
    params_out[1] = static_cast<float>(zp);
  }
}

// One warp per row: q = clamp(rne(x*inv) + zp, 0, 255) as u8 into [m][kp]
// (zero padding), rowsum[i] = sum q, nanrow[i] = 1 if any x*inv is NaN.
__global__ void k_quantize_rows(const float* __restrict__ a, int m, int k, int lda, int kp,
                                const QParams* __restrict__ qp, uint8_t* __restrict__ q, int32_t* __restrict__ rowsum,
                                int32_t* __restrict__ nanrow) {
  const int warps = (blockDim.x >> 5) * gridDim.x;
  const int lane = threadIdx.x & 31;
  const float inv = qp->inverse;
  const float zpf = static_cast<float>(qp->zp);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const float* ar = a + static_cast<size_t>(r) * lda;
    uint8_t* qr = q + static_cast<size_t>(r) * kp;
    int sum = 0, nan = 0;
    const bool vec = ((lda & 3) == 0) && ((reinterpret_cast<uintptr_t>(a) & 15u) == 0);
    for (int c0 = lane * 4; c0 < kp; c0 += 128) {
      uint32_t packed = 0;
      float xv[4];
      if (vec && c0 + 4 <= k) {
        const float4 t4 = __ldg(reinterpret_cast<const float4*>(ar + c0));
        xv[0] = t4.x; xv[1] = t4.y; xv[2] = t4.z; xv[3] = t4.w;
      } else {
#pragma unroll
        for (int t = 0; t < 4; ++t) xv[t] = (c0 + t < k) ? ar[c0 + t] : 0.0f;
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int c = c0 + t;
        uint32_t v = 0;
        if (c < k) {
          const float s = __fmul_rn(xv[t], inv);
          if (s != s) {
            nan = 1;
          } else {
            const float f = minps(255.0f, maxps(0.0f, __fadd_rn(rintf(s), zpf)));
            v = static_cast<uint32_t>(f);
          }
        }
        sum += static_cast<int>(v);
        packed |= v << (8 * t);
      }
      *reinterpret_cast<uint32_t*>(qr + c0) = packed;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sum += __shfl_xor_sync(0xffffffffu, sum, o);
      nan |= __shfl_xor_sync(0xffffffffu, nan, o);
    }
    if (lane == 0) {
      rowsum[r] = sum;
      nanrow[r] = nan;
    }
  }
}

// The whole DynamicQuantizeLinear as ONE cooperative kernel when A's rows fit
// in the CTAs' shared memory: each CTA loads its contiguous rows of A once
// (HBM -> smem, min/max on the fly), publishes a partial range, meets the other
// CTAs at a grid barrier (bounded spin on a device counter), reduces the
// partials to scale/zero point (same arithmetic as k_dql_params) and quantizes
// its rows from shared memory (same arithmetic as k_quantize_rows). A is read
// from HBM once and the range and quantisation need no extra launches.
// Counters: sync[0] arrivals, sync[1] departures; the last CTA to leave
// resets both, so every launch starts from zero.
constexpr int kDqlThreads = 512;

__device__ __forceinline__ QParams dql_params_from(float mn, float mx) {
  float scale = __fdiv_rn(__fsub_rn(mx, mn), 255.0f);
  if (!(scale > 0.0f)) scale = 1.0f;
  const float z = rintf(__fdiv_rn(-mn, scale));
  int zp = (z != z) ? 0 : (z >= 2147483520.0f ? 2147483647 : (z <= -2147483648.0f ? (-2147483647 - 1) : static_cast<int>(z)));
  zp = zp < 0 ? 0 : (zp > 255 ? 255 : zp);
  QParams p;
  p.scale = scale;
  p.inverse = __fdiv_rn(1.0f, scale);
  p.zp = zp;
  p.pad = 0;
  return p;
}

__global__ void __launch_bounds__(kDqlThreads, 1)
    k_dql_fused(const float* __restrict__ a, int m, int k, int lda, int kp, int rows_per_cta, int extra_arrivals,
                const float* __restrict__ override_mm, float2* __restrict__ part, unsigned* __restrict__ sync,
                QParams* __restrict__ qp_out, float* __restrict__ params_out, uint8_t* __restrict__ q,
                int32_t* __restrict__ rowsum, int32_t* __restrict__ nanrow, int* __restrict__ err) {
  extern __shared__ float rows_s[];  // [rows_per_cta][k], then row sums and NaN flags
  int* s_sum = reinterpret_cast<int*>(rows_s + static_cast<size_t>(rows_per_cta) * k);
  int* s_nan = s_sum + rows_per_cta;
  __shared__ float red_mn[kDqlThreads / 32], red_mx[kDqlThreads / 32];
  __shared__ QParams sp;
  __shared__ int s_ok;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int r0 = blockIdx.x * rows_per_cta;
  const int nrows = max(0, min(m, r0 + rows_per_cta) - r0);
  const int count = nrows * k;
  for (int r = tid; r < nrows; r += kDqlThreads) {
    s_sum[r] = 0;
    s_nan[r] = 0;
  }
  float mn = 0.0f, mx = 0.0f;  // 0 is always inside the range
  auto take = [&](float e) {
    if (e == e) {
      mn = fminf(mn, e);
      mx = fmaxf(mx, e);
    }
  };
  if (lda == k && (k & 3) == 0 && (reinterpret_cast<uintptr_t>(a) & 15u) == 0) {
    // the CTA's rows are one contiguous block: 8 independent 16-byte loads in flight per thread
    const float4* src = reinterpret_cast<const float4*>(a + static_cast<size_t>(r0) * k);
    float4* dst = reinterpret_cast<float4*>(rows_s);
    const int n4 = count >> 2;
    for (int base = 0; base < n4; base += 8 * kDqlThreads) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * kDqlThreads + tid;
        if (i < n4) v[u] = __ldg(src + i);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = base + u * kDqlThreads + tid;
        if (i < n4) {
          dst[i] = v[u];
          take(v[u].x);
          take(v[u].y);
          take(v[u].z);
          take(v[u].w);
        }
      }
    }
  } else {
    for (int i = tid; i < count; i += kDqlThreads) {
      const int row = i / k, c = i - row * k;
      const float e = a[static_cast<size_t>(r0 + row) * lda + c];
      rows_s[i] = e;
      take(e);
    }
  }
  const int G = gridDim.x;
  if (override_mm == nullptr) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) {
      red_mn[wid] = mn;
      red_mx[wid] = mx;
    }
    __syncthreads();
    if (wid == 0) {
      mn = lane < kDqlThreads / 32 ? red_mn[lane] : 0.0f;
      mx = lane < kDqlThreads / 32 ? red_mx[lane] : 0.0f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      }
      if (lane == 0) {
        part[blockIdx.x] = make_float2(mn, mx);
        __threadfence();
        atomicAdd(&sync[0], 1u);
        // grid barrier: bounded spin until every CTA has published its range
        const long long c0 = clock64();
        int ok = 1;
        const unsigned want = static_cast<unsigned>(G + extra_arrivals);
        while (*reinterpret_cast<volatile unsigned*>(&sync[0]) < want) {
          if (clock64() - c0 > kWaitLimitCycles) {
            ok = 0;
            atomicExch(err, DEV_ERR_TIMEOUT);
            break;
          }
        }
        __threadfence();
        s_ok = ok;
      }
      __syncwarp();
      // every CTA reduces all partials (order-independent, equals a serial scan);
      // each lane's loads are independent so they are in flight together
      float2 pp[5];
#pragma unroll
      for (int u = 0; u < 5; ++u) {
        const int i = lane + 32 * u;
        pp[u] = i < G ? __ldcg(part + i) : make_float2(0.0f, 0.0f);
      }
      mn = 0.0f;
      mx = 0.0f;
#pragma unroll
      for (int u = 0; u < 5; ++u) {
        mn = fminf(mn, pp[u].x);
        mx = fmaxf(mx, pp[u].y);
      }
      for (int i = lane + 160; i < G; i += 32) {
        const float2 t = __ldcg(part + i);
        mn = fminf(mn, t.x);
        mx = fmaxf(mx, t.y);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      }
      if (lane == 0) sp = dql_params_from(mn, mx);
    }
  } else if (tid == 0) {
    s_ok = 1;
    sp = dql_params_from(fminf(0.0f, override_mm[0]), fmaxf(0.0f, override_mm[1]));
  }
  __syncthreads();
  // the GEMM that follows (launched with launch_pdl) may be scheduled once
  // every CTA of this grid has passed here, i.e. all of them are running, so
  // its CTAs never hold an SM this grid still needs; it waits for this
  // grid's completion before it reads q
  griddep_launch();
  if (!s_ok) {
    // gave up at the barrier (error word set): still count the departure so
    // the last CTA out leaves the counters at zero for the next launch
    if (override_mm == nullptr && tid == 0 && atomicAdd(&sync[1], 1u) == static_cast<unsigned>(G) - 1u) {
      sync[0] = 0u;
      sync[1] = 0u;
      __threadfence();
    }
    return;
  }
  const QParams p = sp;
  if (blockIdx.x == 0 && tid == 0) {
    *qp_out = p;
    if (params_out != nullptr) {
      params_out[0] = p.scale;
      params_out[1] = static_cast<float>(p.zp);
    }
  }
  // quantize the CTA's rows from shared memory: one warp per row, 4-element
  // groups, four groups per lane in flight; the row's sum stays in registers
  // and is reduced once per row (integer sums: any order gives the same value)
  const float inv = p.inverse, zpf = static_cast<float>(p.zp);
  const int gpr = kp >> 2;  // a multiple of 32
  const bool vk = (k & 3) == 0;
  for (int row = wid; row < nrows; row += kDqlThreads / 32) {
    const float* xr = rows_s + static_cast<size_t>(row) * k;
    uint8_t* qr = q + static_cast<size_t>(r0 + row) * kp;
    int sum = 0, nan = 0;
    for (int g0 = 0; g0 < gpr; g0 += 4 * 32) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int g = g0 + u * 32 + lane;
        if (g < gpr) {
          const int c0 = g * 4;
          float xv[4];
          if (vk && c0 + 4 <= k) {
            const float4 t4 = *reinterpret_cast<const float4*>(xr + c0);
            xv[0] = t4.x;
            xv[1] = t4.y;
            xv[2] = t4.z;
            xv[3] = t4.w;
          } else {
#pragma unroll
            for (int t = 0; t < 4; ++t) xv[t] = c0 + t < k ? xr[c0 + t] : 0.0f;
          }
          uint32_t packed = 0;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint32_t v = 0;
            if (c0 + t < k) {
              const float sv = __fmul_rn(xv[t], inv);
              if (sv != sv) {
                nan = 1;
              } else {
                v = static_cast<uint32_t>(minps(255.0f, maxps(0.0f, __fadd_rn(rintf(sv), zpf))));
              }
            }
            sum += static_cast<int>(v);
            packed |= v << (8 * t);
          }
          *reinterpret_cast<uint32_t*>(qr + c0) = packed;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sum += __shfl_xor_sync(0xffffffffu, sum, o);
      nan |= __shfl_xor_sync(0xffffffffu, nan, o);
    }
    if (lane == 0) {
      s_sum[row] = sum;
      s_nan[row] = nan;
    }
  }
  __syncthreads();
  for (int r = tid; r < nrows; r += kDqlThreads) {
    rowsum[r0 + r] = s_sum[r];
    nanrow[r0 + r] = s_nan[r];
  }
  if (override_mm == nullptr && tid == 0 && atomicAdd(&sync[1], 1u) == static_cast<unsigned>(G) - 1u) {
    sync[0] = 0u;  // every CTA has passed the barrier: reset for the next launch
    sync[1] = 0u;
    __threadfence();
  }
}

// ---------------------------------------------------------------- unfused ops
// DynamicQuantizeLinear over a flat tensor (QuantOps.cs:155-231 via
// Quantization.cs:68-103): q = clamp(rne(x * (1/scale)) + zp, 0, 255); NaN
// inputs give 0 (the reference's saturating byte conversion of NaN). Block 0
// also writes the scalar outputs y_scale (f32) and y_zero_point (u8).
__global__ void k_quantize_flat(const float* __restrict__ x, long n, const QParams* __restrict__ qp,
                                uint8_t* __restrict__ y, float* __restrict__ y_scale, uint8_t* __restrict__ y_zp) {
  const float inv = qp->inverse;
  const float zpf = static_cast<float>(qp->zp);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (y_scale) *y_scale = qp->scale;
    if (y_zp) *y_zp = static_cast<uint8_t>(qp->zp);
  }
  auto quant = [&](float v) -> uint32_t {
    const float sv = __fmul_rn(v, inv);
    if (sv != sv) return 0u;
    return static_cast<uint32_t>(minps(255.0f, maxps(0.0f, __fadd_rn(rintf(sv), zpf))));
  };
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(y) & 3u) == 0;
  const long n4 = vec ? n / 4 : 0;
  for (long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
    reinterpret_cast<uint32_t*>(y)[i] = quant(v.x) | (quant(v.y) << 8) | (quant(v.z) << 16) | (quant(v.w) << 24);
  }
  for (long i = n4 * 4 + blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long>(gridDim.x) * blockDim.x)
    y[i] = static_cast<uint8_t>(quant(x[i]));
}

// MatMulInteger's activation side: the zero point goes into the same
// QParams the int8 GEMM reads; per-row sums of A for the weight zero-point
// correction (signed or unsigned bytes); no NaN rows.
__global__ void k_set_qparams(QParams* __restrict__ qp, int zp) {
  QParams p;
  p.scale = 1.0f;
  p.inverse = 1.0f;
  p.zp = zp;
  p.pad = 0;
  *qp = p;
}

__global__ void k_rowsum_i8(const uint8_t* __restrict__ a, int m, int k, long long lda, int a_signed,
                            int32_t* __restrict__ rowsum, int32_t* __restrict__ nanrow) {
  const int warps = (blockDim.x >> 5) * gridDim.x;
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const uint8_t* ar = a + static_cast<size_t>(r) * lda;
    int sum = 0;
    for (int c = lane; c < k; c += 32) sum += a_signed ? static_cast<int>(static_cast<int8_t>(ar[c])) : ar[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) {
      rowsum[r] = sum;
      nanrow[r] = 0;
    }
  }
}

// Rows [0, grouped) went through the reference's 12/6/4-row micro-kernels
// (fused FMA epilogue); see GemmKernel.cs:746-790.
__host__ __device__ inline int grouped_rows(int m) {
  int row = 0;
  while (row + 12 <= m) row += 12;
  while (row + 6 <= m) row += 6;
  while (row + 4 <= m) row += 4;
  return row;
}

struct DqmmArgs {
  int M, N, K, num_kb;
  int fused_rows, full_cols;
  const QParams* qp;
  const int32_t* rowsum;
  const int32_t* nanrow;
  const int32_t* colsum;
  const int32_t* wzp;
  const float* wscale;
  int n_scale;
  const float* bias;
  float* y;
  int32_t* acc_out;
  int has_wzp;
  int int_out;  // MatMulInteger: y receives the s32 accumulators (bit patterns) instead of the FP32 epilogue
  int cpm;      // q-resident schedule: CTAs per 128-row block
};

__global__ void __launch_bounds__(kQThreads, 1)
    k_dqmm_i8(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mW,
              const __grid_constant__ DqmmArgs args, uint32_t idesc, int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(tiles + kQTiles);
  uint64_t* empty = full + kQStages;
  uint64_t* done = empty + kQStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kQBM, n0 = blockIdx.x * kQBN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&mQ);
    tma_prefetch(&mW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kQBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int num_kb = args.num_kb;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % kQStages;
        const uint32_t ph = (kb / kQStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, err)) break;
        uint8_t* st = tiles + s * kQStage;
        mbar_arrive_expect_tx(&full[s], kQStage);
        tma_load_2d(st, &mQ, &full[s], kb * kQBK, m0);
        tma_load_2d(st + kQA, &mW, &full[s], kb * kQBK, n0);
        issued = kb + 1;
      }
      if (*abort_flag) {
        const int first = issued > kQStages ? issued - kQStages : 0;
        for (int kb = first; kb < issued; ++kb) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[kb % kQStages], (kb / kQStages) & 1u) &&
                 globaltimer_ns() - t0 < 50ull * 1000ull * 1000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % kQStages;
        const uint32_t ph = (kb / kQStages) & 1u;
        if (!mbar_wait(&full[s], ph, abort_flag, err)) break;
        tc_fence_after();
        const uint32_t base = smem_addr(tiles + s * kQStage);
        const uint64_t dA = sdesc_kmajor_sw128(base);
        const uint64_t dB = sdesc_kmajor_sw128(base + kQA);
#pragma unroll
        for (int kk = 0; kk < kQBK / 32; ++kk) {
          const uint64_t off = static_cast<uint64_t>(kk * 2);  // +32 bytes per 32-wide K step
          mma_i8(tmem, dA + off, dB + off, idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        mma_commit(&empty[s]);
      }
      mma_commit(done);
    }
  } else {
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    bool ok = mbar_wait(done, 0, abort_flag, err);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    constexpr int kPitch = kQBN + 4;
    uint32_t* stage = reinterpret_cast<uint32_t*>(tiles);
    if (ok) {
      const int row = q * 32 + lane;
      const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(half * 128);
#pragma unroll
      for (int g = 0; g < 8; g += 2) {
        uint32_t r0[16], r1[16];
        tmem_ld16(base + g * 16, r0);
        tmem_ld16(base + (g + 1) * 16, r1);
        tmem_wait_ld();
        uint32_t* dst = stage + row * kPitch + half * 128 + g * 16;
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
          *reinterpret_cast<uint4*>(dst + j) = make_uint4(r0[j], r0[j + 1], r0[j + 2], r0[j + 3]);
          *reinterpret_cast<uint4*>(dst + 16 + j) = make_uint4(r1[j], r1[j + 1], r1[j + 2], r1[j + 3]);
        }
      }
    }
    // Per-column constants of this tile, one epilogue thread per column:
    // comb = a_scale * w_scale[j], bias, corr = -zp*colsum[j] + K*zp*wzp[j], wzp.
    float* c_comb = reinterpret_cast<float*>(stage + kQBM * kPitch);
    float* c_bias = c_comb + kQBN;
    int32_t* c_corr = reinterpret_cast<int32_t*>(c_bias + kQBN);
    int32_t* c_wzp = c_corr + kQBN;
    int32_t* r_sum = c_wzp + kQBN;  // per-row sum of q and NaN flag of this tile
    int32_t* r_nan = r_sum + kQBM;
    const QParams p = *args.qp;
    {
      const int jj = threadIdx.x - 64;  // 0..255
      const int j = n0 + jj;
      if (j < args.N) {
        const int wz = __ldg(args.wzp + j);
        c_comb[jj] = __fmul_rn(p.scale, __ldg(args.wscale + (args.n_scale > 1 ? j : 0)));
        c_bias[jj] = args.bias ? __ldg(args.bias + j) : 0.0f;
        c_corr[jj] = -p.zp * __ldg(args.colsum + j) + args.K * p.zp * wz;
        c_wzp[jj] = wz;
      }
      if (jj < kQBM && m0 + jj < args.M) {
        r_sum[jj] = __ldg(args.rowsum + m0 + jj);
        r_nan[jj] = __ldg(args.nanrow + m0 + jj);
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(8 * 32) : "memory");
    if (ok) {
      const int e = warp - 2;
      for (int r = e; r < kQBM; r += 8) {
        const int i = m0 + r;
        if (i >= args.M) break;
        const int rs = r_sum[r];
        const bool nanr = r_nan[r] != 0;
        const bool fused_row = i < args.fused_rows;
        float* yr = args.y + static_cast<size_t>(i) * args.N;
        for (int h = 0; h < kQBN; h += 128) {
          const int jl = h + lane * 4;
          const int j0 = n0 + jl;
          if (j0 >= args.N) continue;
          const uint4 raw = *reinterpret_cast<const uint4*>(stage + r * kPitch + jl);
          const int32_t s4[4] = {static_cast<int32_t>(raw.x), static_cast<int32_t>(raw.y),
                                 static_cast<int32_t>(raw.z), static_cast<int32_t>(raw.w)};
          float out[4];
          int32_t accs[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int j = j0 + t;
            if (j >= args.N) {
              out[t] = 0.0f;
              accs[t] = 0;
              continue;
            }
            const int32_t acc = s4[t] - c_wzp[jl + t] * rs + c_corr[jl + t];
            accs[t] = acc;
            const float comb = c_comb[jl + t];
            const float b = c_bias[jl + t];
            const float af = static_cast<float>(acc);
            float v;
            if (fused_row && j < args.full_cols) {
              v = __fmaf_rn(af, comb, b);
            } else {
              v = __fmul_rn(af, comb);
              if (args.bias) v = __fadd_rn(v, b);
            }
            out[t] = args.int_out ? __int_as_float(acc) : (nanr ? __int_as_float(0x7fc00000) : v);
          }
          if (j0 + 4 <= args.N && (args.N & 3) == 0) {
            *reinterpret_cast<float4*>(yr + j0) = make_float4(out[0], out[1], out[2], out[3]);
            if (args.acc_out)
              *reinterpret_cast<int4*>(args.acc_out + static_cast<size_t>(i) * args.N + j0) =
                  make_int4(accs[0], accs[1], accs[2], accs[3]);
          } else {
            for (int t = 0; t < 4; ++t)
              if (j0 + t < args.N) {
                yr[j0 + t] = out[t];
                if (args.acc_out) args.acc_out[static_cast<size_t>(i) * args.N + j0 + t] = accs[t];
              }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kQBN);
  }
}

// ---------------------------------------------------------------- persistent form
// One CTA per SM walks 128 x 128 output tiles (tile t, t + grid, ...). The
// TMEM holds two 128-column accumulators, so the MMA warp fills tile i+1
// while the epilogue warps drain tile i; the epilogue writes each warp's
// 32 x 64 result block into 128-byte-swizzled shared memory and one lane
// stores it with two TMA tensor stores (async; the staging is reused once
// the store engine has read it). Same arithmetic per element as k_dqmm_i8.
constexpr int kPBN = 128, kPStages = 4;
constexpr int kPA = kQBM * kQBK, kPB = kPBN * kQBK, kPStage = kPA + kPB;  // 16 + 16 KB
constexpr int kPRing = kPStages * kPStage;                                  // 128 KB
constexpr int kPEpiWarps = 8;
constexpr int kPBox = 32 * 32 * 4;                                          // one 32x32 f32 store box
constexpr int kPOut = kPEpiWarps * 2 * kPBox;                               // 64 KB
constexpr int kPThreads = 64 + kPEpiWarps * 32;
constexpr int kPSmem = 1024 + kPRing + kPOut + 256;
static_assert(kPSmem <= 227 * 1024, "persistent DQMM smem");
// q-resident schedule (K <= 512): the CTA's 128 quantised rows stay in shared
// memory (4 k-blocks, 64 KB) and only weight k-blocks stream through a
// 6-stage ring (1.5 tiles ahead).
constexpr int kRStages = 6, kRMaxKb = 4;
constexpr int kRRes = kRMaxKb * kPB;                  // 64 KB
constexpr int kRRing = kRStages * kPA;                // 96 KB
constexpr int kRSmem = 1024 + kRRes + kRRing + kPOut + 256;
static_assert(kRSmem <= 232448, "q-resident DQMM smem");

// Barrier over the epilogue warps that also ANDs a predicate across them, so a
// wait that gave up in one warp stops every epilogue warp at the same tile.
__device__ __forceinline__ bool epi_all_dqmm(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(kPEpiWarps * 32)
      : "memory");
  return r != 0;
}

// Raw per-column inputs of the epilogue constants (loaded one tile ahead).
struct ColRaw {
  int wz, cs;
  float ws, b;
};
__device__ __forceinline__ ColRaw dqmm_col_load(const DqmmArgs& args, int j) {
  ColRaw c{0, 0, 0.0f, 0.0f};
  if (j < args.N) {
    c.wz = __ldg(args.wzp + j);
    c.cs = __ldg(args.colsum + j);
    c.ws = __ldg(args.wscale + (args.n_scale > 1 ? j : 0));
    c.b = args.bias ? __ldg(args.bias + j) : 0.0f;
  }
  return c;
}

// Transposed tiles: the MMA computes D = Wt[n0:n0+128] . q[m0:m0+128]^T, so a
// TMEM lane is an output COLUMN j and a TMEM column an output row i. Each
// epilogue thread therefore owns one column: its constants
// (a_scale*w_scale[j], bias[j], the zero-point correction) sit in registers
// for the whole tile and every element costs an integer add, a conversion,
// one FMA and a 4-byte shared store. One CTA per SM walks the tiles (t,
// t + grid, ...); two 128-column TMEM accumulators let the MMA warp fill
// tile i+1 while the epilogue drains tile i. Each epilogue warp writes its
// 64 rows x 32 columns into 128-byte-swizzled boxes that one lane stores
// with TMA tensor stores. Same arithmetic per element as k_dqmm_i8.
template <bool QRES>
__global__ void __launch_bounds__(kPThreads, 1)
    k_dqmm_i8_persistent(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mW,
                         const __grid_constant__ CUtensorMap mY, const __grid_constant__ DqmmArgs args,
                         uint32_t idesc, int* __restrict__ err) {
  constexpr int STAGES = QRES ? kRStages : kPStages;
  constexpr int STAGE = QRES ? kPA : kPStage;  // q-resident: weight k-blocks only
  extern __shared__ uint8_t smem_raw[];
  uint8_t* qres = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = qres + (QRES ? kRRes : 0);
  uint8_t* ostage = ring + STAGES * STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(ostage + kPOut);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* qfull = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (args.M + kPBN - 1) / kPBN;  // row tiles (the MMA's N side)
  const int nt = (args.N + kQBM - 1) / kQBM;  // weight-column tiles
  const int tiles = mt * nt;
  const int num_kb = args.num_kb;
  // The CTA's tile lt: grid-strided over all tiles, or (q-resident) its own
  // row block and every cpm-th column block.
  auto tile_at = [&](int lt, int& m0, int& n0) -> bool {
    if (QRES) {
      const int mb = blockIdx.x / args.cpm, nb = static_cast<int>(blockIdx.x % args.cpm) + lt * args.cpm;
      m0 = mb * kPBN;
      n0 = nb * kQBM;
      return mb < mt && nb < nt;
    }
    const int t = static_cast<int>(blockIdx.x) + lt * static_cast<int>(gridDim.x);
    m0 = (t % mt) * kPBN;
    n0 = (t / mt) * kQBM;
    return t < tiles;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kPEpiWarps);
    }
    mbar_init(qfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&mQ);
    tma_prefetch(&mW);
    tma_prefetch(&mY);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kPBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();  // launched with launch_pdl: q, its row sums and the parameters are complete past here
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      int g = 0, issued = 0;
      bool q_issued = false;
      int m0, n0;
      for (int lt = 0; tile_at(lt, m0, n0) && !*abort_flag; ++lt) {
        if (QRES && !q_issued) {  // the CTA's quantised rows, once
          mbar_arrive_expect_tx(qfull, num_kb * kPB);
          for (int kb = 0; kb < num_kb; ++kb) tma_load_2d(qres + kb * kPB, &mQ, qfull, kb * kQBK, m0);
          q_issued = true;
        }
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % STAGES;
          if (!mbar_wait(&empty[s], ((g / STAGES) & 1u) ^ 1u, abort_flag, err)) break;
          uint8_t* st = ring + s * STAGE;
          mbar_arrive_expect_tx(&full[s], STAGE);
          tma_load_2d(st, &mW, &full[s], kb * kQBK, n0);           // A: 128 weight columns
          if (!QRES) tma_load_2d(st + kPA, &mQ, &full[s], kb * kQBK, m0);  // B: 128 quantised rows
          issued = g + 1;
        }
      }
      if (*abort_flag) {  // let in-flight loads land before the CTA's shared memory goes away
        for (int x = issued > STAGES ? issued - STAGES : 0; x < issued; ++x) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[x % STAGES], (x / STAGES) & 1u) &&
                 globaltimer_ns() - t0 < 50ull * 1000ull * 1000ull) {
          }
        }
        if (q_issued) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(qfull, 0) && globaltimer_ns() - t0 < 50ull * 1000ull * 1000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int g = 0, m0, n0;
      bool q_ready = !QRES;
      for (int lt = 0; tile_at(lt, m0, n0); ++lt) {
        const int tb = lt & 1;
        if (!q_ready) {
          if (!mbar_wait(qfull, 0, abort_flag, err)) break;
          q_ready = true;
        }
        if (!mbar_wait(&tempty[tb], ((lt >> 1) & 1u) ^ 1u, abort_flag, err)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(tb * kPBN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % STAGES;
          if (!mbar_wait(&full[s], (g / STAGES) & 1u, abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_addr(ring + s * STAGE);
          const uint64_t dA = sdesc_kmajor_sw128(base);
          const uint64_t dB = sdesc_kmajor_sw128(QRES ? smem_addr(qres + kb * kPB) : base + kPA);
#pragma unroll
          for (int kk = 0; kk < kQBK / 32; ++kk) {
            const uint64_t off = static_cast<uint64_t>(kk * 2);
            mma_i8(d, dA + off, dB + off, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&tfull[tb]);
      }
    }
  } else {
    const int ew = warp - 2;
    const int q = warp & 3;   // TMEM lane quadrant: output columns 32q .. 32q+31 of the tile
    const int h = ew >> 2;    // output rows 64h .. 64h+63 of the tile
    uint8_t* my_out = ostage + ew * 2 * kPBox;
    const QParams p = *args.qp;
    ColRaw raw{0, 0, 0.0f, 0.0f};
    int rs_a = 0, rs_b = 0, nan_a = 0, nan_b = 0;  // rows 64h + lane and 64h + 32 + lane
    auto load_tile_inputs = [&](int mm, int nn) {
      mm += h * 64;
      raw = dqmm_col_load(args, nn + q * 32 + lane);
      const int ia = mm + lane, ib = mm + 32 + lane;
      nan_a = ia < args.M ? __ldg(args.nanrow + ia) : 0;
      nan_b = ib < args.M ? __ldg(args.nanrow + ib) : 0;
      if (args.has_wzp) {
        rs_a = ia < args.M ? __ldg(args.rowsum + ia) : 0;
        rs_b = ib < args.M ? __ldg(args.rowsum + ib) : 0;
      }
    };
    int m0, n0;
    if (tile_at(0, m0, n0)) load_tile_inputs(m0, n0);
    for (int lt = 0; tile_at(lt, m0, n0); ++lt) {
      const int tb = lt & 1;
      const int j = n0 + q * 32 + lane;  // this thread's output column
      const int i0 = m0 + h * 64;        // first of this warp's 64 output rows
      const float comb = __fmul_rn(p.scale, raw.ws);
      const float bias = raw.b;
      const int corr = -p.zp * raw.cs + args.K * p.zp * raw.wz;
      const int wz = raw.wz;
      const bool full_col = j < args.full_cols;
      const int my_rs_a = rs_a, my_rs_b = rs_b;
      const bool any_nan = __any_sync(0xffffffffu, (nan_a | nan_b) != 0);
      const int my_nan_a = nan_a, my_nan_b = nan_b;
      {
        int mn, nn;
        if (tile_at(lt + 1, mn, nn)) load_tile_inputs(mn, nn);  // in flight meanwhile
      }
      if (!epi_all_dqmm(mbar_wait(&tfull[tb], (lt >> 1) & 1u, abort_flag, err))) break;
      tc_fence_after();
      if (lane == 0) bulk_wait_read_all();  // the previous tile's stores have read the staging
      __syncwarp();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(tb * kPBN + h * 64);
      const int nf = min(max(args.fused_rows - i0, 0), 64);  // rows of this block on the fused-FMA path
      const bool fast = !args.has_wzp && __all_sync(0xffffffffu, full_col) && nf == 64;
      const float bias_u = args.bias ? bias : -0.0f;  // x + (-0) == x for every x, -0 included
      // element (row i0 + 32*half + e, column j) -> box `half`, row e, 16-byte chunk (lane/4) ^ (e%8)
      float* ocol = reinterpret_cast<float*>(my_out + (lane & 3) * 4);
      const int swz = lane >> 2;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        uint32_t r[32];
        tmem_ld32(tbase + half * 32, r);
        tmem_wait_ld();
        if (half == 1) {  // the accumulator buffer is free for the tile after next
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[tb]);
        }
        float* obox = ocol + half * (kPBox / 4);
        if (args.int_out) {  // MatMulInteger: the corrected s32 accumulators themselves
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            int32_t acc = static_cast<int32_t>(r[e]) + corr;
            acc -= args.has_wzp ? wz * __shfl_sync(0xffffffffu, half == 0 ? my_rs_a : my_rs_b, e) : 0;
            r[e] = static_cast<uint32_t>(acc);
            obox[e * 32 + ((swz ^ (e & 7)) << 2)] = __int_as_float(acc);
          }
        } else if (fast) {  // common case: every element is fma(acc, a_scale*w_scale[j], bias[j])
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int32_t acc = static_cast<int32_t>(r[e]) + corr;
            r[e] = static_cast<uint32_t>(acc);
            obox[e * 32 + ((swz ^ (e & 7)) << 2)] = __fmaf_rn(static_cast<float>(acc), comb, bias);
          }
        } else {  // tails (unfused mul-then-add), weight zero points: selects, no branches per element
          const int rs_h = half == 0 ? my_rs_a : my_rs_b;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            int32_t acc = static_cast<int32_t>(r[e]) + corr;
            acc -= args.has_wzp ? wz * __shfl_sync(0xffffffffu, rs_h, e) : 0;
            r[e] = static_cast<uint32_t>(acc);
            const float af = static_cast<float>(acc);
            const float vf = __fmaf_rn(af, comb, bias);
            const float vu = __fadd_rn(__fmul_rn(af, comb), bias_u);
            obox[e * 32 + ((swz ^ (e & 7)) << 2)] = (half * 32 + e < nf && full_col) ? vf : vu;
          }
        }
        if (any_nan && !args.int_out) {  // rows whose input held a NaN are NaN throughout (rare)
          const int nan_h = half == 0 ? my_nan_a : my_nan_b;
#pragma unroll 1
          for (int e = 0; e < 32; ++e)
            if (__shfl_sync(0xffffffffu, nan_h, e) != 0) obox[e * 32 + ((swz ^ (e & 7)) << 2)] = __int_as_float(0x7fc00000);
        }
        if (args.acc_out != nullptr && j < args.N) {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int i = i0 + half * 32 + e;
            if (i < args.M) args.acc_out[static_cast<size_t>(i) * args.N + j] = static_cast<int32_t>(r[e]);
          }
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int col0 = n0 + q * 32;
        if (col0 < args.N) {
          if (i0 < args.M) tma_store_2d(&mY, my_out, col0, i0);
          if (i0 + 32 < args.M) tma_store_2d(&mY, my_out + kPBox, col0, i0 + 32);
        }
        bulk_commit();
      }
    }
    if (lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kPBN);
  }
}

// W [k][n] (s8 or u8) -> Wt [n][kp] + column sums; one thread per output column strip.
__global__ void k_pack_dqmm_w(const int8_t* __restrict__ w, int k, int n, int kp, int is_signed,
                              int8_t* __restrict__ wt, int32_t* __restrict__ colsum) {
  __shared__ int8_t tile[32][33];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int yy = ty; yy < 32; yy += 8) {
    const int kk = k0 + yy, nn = n0 + tx;
    tile[yy][tx] = (kk < k && nn < n) ? w[static_cast<size_t>(kk) * n + nn] : 0;
  }
  __syncthreads();
  for (int yy = ty; yy < 32; yy += 8) {
    const int nn = n0 + yy, kk = k0 + tx;
    if (nn < n && kk < kp) {
      const int8_t v = tile[tx][yy];
      wt[static_cast<size_t>(nn) * kp + kk] = v;
      int iv = is_signed ? static_cast<int>(v) : static_cast<int>(static_cast<uint8_t>(v));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) iv += __shfl_xor_sync(0xffffffffu, iv, o);
      if (tx == 0) atomicAdd(colsum + nn, iv);
    }
  }
}

}  // namespace

static int minmax_params(osc_ctx* ctx, const float* a, long count, const float* override_mm, void* work,
                         QParams* qp, float* params_out) {
  float2* part = static_cast<float2*>(work);
  int blocks = 0;
  if (override_mm == nullptr) {
    blocks = static_cast<int>(std::min<long>(std::max<long>((count / 4 + 255) / 256, 1), ctx->num_sms * 4L));
    prof_begin(ctx);
    k_minmax_partial<<<blocks, 256, 0, ctx->stream>>>(a, count, part);
    OSC_TRY(check_launch(ctx, "k_minmax_partial"));
  }
  prof_begin(ctx);
  k_dql_params<<<1, 32, 0, ctx->stream>>>(part, blocks, override_mm, qp, params_out);
  return check_launch(ctx, "k_dql_params");
}

// The int8 GEMM of DynamicQuantizeMatMul and MatMulInteger: q [m][k] bytes
// (row pitch q_pitch, the tensor map spans q_cols columns and zero-fills the
// rest of the last 128-byte K block), prepacked weights, and the epilogue
// described by `args` (FP32 with the reference's rounding, or s32 with
// args.int_out). Persistent transposed tiles when y allows TMA stores.
static int int8_gemm(osc_ctx* ctx, const uint8_t* q, size_t q_pitch, int q_cols, int q_signed, int m,
                     const osc_dqmm_weights* w, DqmmArgs& args) {
  float* y = args.y;
  const uint32_t q_fmt = q_signed ? 1u : 0u;
  CUtensorMap mQ, mW;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(q_cols), static_cast<uint64_t>(m)};
    const uint64_t pitch[1] = {static_cast<uint64_t>(q_pitch)};
    const uint32_t box[2] = {kQBK, kQBM};
    OSC_TRY(encode_tiled(&mQ, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(w->kp), static_cast<uint64_t>(w->n)};
    const uint64_t pitch[1] = {static_cast<uint64_t>(w->kp)};
    const uint32_t box[2] = {kQBK, kQBN};
    OSC_TRY(encode_tiled(&mW, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->wt, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  const uint32_t b_fmt = w->is_signed ? 1u : 0u;
  if (w->n % 4 == 0 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0) {
    // persistent transposed tiles with TMA stores (row pitch N*4 bytes is a multiple of 16)
    CUtensorMap mQp, mY;
    {
      const uint64_t dims[2] = {static_cast<uint64_t>(q_cols), static_cast<uint64_t>(m)};
      const uint64_t pitch[1] = {static_cast<uint64_t>(q_pitch)};
      const uint32_t box[2] = {kQBK, kPBN};
      OSC_TRY(encode_tiled(&mQp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, q, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
    }
    CUtensorMap mWp;
    {
      const uint64_t dims[2] = {static_cast<uint64_t>(w->kp), static_cast<uint64_t>(w->n)};
      const uint64_t pitch[1] = {static_cast<uint64_t>(w->kp)};
      const uint32_t box[2] = {kQBK, kQBM};
      OSC_TRY(encode_tiled(&mWp, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->wt, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
    }
    {
      const uint64_t dims[2] = {static_cast<uint64_t>(w->n), static_cast<uint64_t>(m)};
      const uint64_t pitch[1] = {static_cast<uint64_t>(w->n) * 4};
      const uint32_t box[2] = {32, 32};
      OSC_TRY(encode_tiled(&mY, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, y, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
    }
    // A = weights (s8 or u8), B = activations (u8 or s8); M = 128 columns, N = 128 rows
    const uint32_t idesc_p = (2u << 4) | (b_fmt << 7) | (q_fmt << 10) | (static_cast<uint32_t>(kPBN >> 3) << 17) |
                             (static_cast<uint32_t>(kQBM >> 4) << 24);
    const int mt = (m + kPBN - 1) / kPBN, nt = (w->n + kQBM - 1) / kQBM;
    if (args.num_kb <= kRMaxKb) {
      // q-resident: cpm CTAs share each 128-row block, each walking every cpm-th column block
      args.cpm = std::max(1, std::min(nt, ctx->num_sms / std::max(1, mt)));
      OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_dqmm_i8_persistent<true>), kRSmem));
      return launch_pdl(ctx, k_dqmm_i8_persistent<true>, dim3(mt * args.cpm), dim3(kPThreads), kRSmem, "k_dqmm_i8",
                        mQp, mWp, mY, args, idesc_p, ctx->d_err);
    }
    OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_dqmm_i8_persistent<false>), kPSmem));
    return launch_pdl(ctx, k_dqmm_i8_persistent<false>, dim3(std::min(mt * nt, ctx->num_sms)), dim3(kPThreads),
                      kPSmem, "k_dqmm_i8", mQp, mWp, mY, args, idesc_p, ctx->d_err);
  }
  const uint32_t idesc = (2u << 4) | (q_fmt << 7) | (b_fmt << 10) |
                         (static_cast<uint32_t>(kQBN >> 3) << 17) | (static_cast<uint32_t>(kQBM >> 4) << 24);
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_dqmm_i8), kQSmem));
  dim3 grid((w->n + kQBN - 1) / kQBN, (m + kQBM - 1) / kQBM);
  prof_begin(ctx);
  k_dqmm_i8<<<grid, kQThreads, kQSmem, ctx->stream>>>(mQ, mW, args, idesc, ctx->d_err);
  return check_launch(ctx, "k_dqmm_i8");
}

}  // namespace osc

using namespace osc;

extern "C" {

OSC_API int osc_dqmm_prepack(osc_ctx* ctx, const void* w, int k, int n, int is_signed, const int32_t* w_zp,
                             int n_zp, int host, osc_dqmm_weights** out) {
  if (out == nullptr) return fail(OSC_EINVAL, "osc_dqmm_prepack: out is null");
  *out = nullptr;
  OSC_TRY(enter(ctx));
  if (w == nullptr || k <= 0 || n <= 0) return fail(OSC_EINVAL, "osc_dqmm_prepack: bad W [%d, %d]", k, n);
  if (n_zp != 0 && n_zp != 1 && n_zp != n) return fail(OSC_EINVAL, "osc_dqmm_prepack: %d zero points for %d columns", n_zp, n);
  if (n_zp > 0 && w_zp == nullptr) return fail(OSC_EINVAL, "osc_dqmm_prepack: null zero points");
  if (fault_injected("prepack")) return fail(OSC_EFAULT_INJECTED, "injected failure (prepack)");
  auto* d = new osc_dqmm_weights();
  d->device = ctx->device;
  d->k = k;
  d->n = n;
  d->kp = static_cast<int>(round_up(static_cast<size_t>(k), kQBK));
  d->is_signed = is_signed ? 1 : 0;
  std::vector<int32_t> zp(static_cast<size_t>(n), 0);
  for (int j = 0; j < n; ++j) {
    zp[j] = n_zp == 0 ? 0 : (n_zp == 1 ? w_zp[0] : w_zp[j]);
    if (zp[j] != 0) d->has_zp = 1;
  }
  const size_t wbytes = static_cast<size_t>(k) * n;
  int8_t* staged = nullptr;
  cudaError_t e = cudaMalloc(&d->wt, static_cast<size_t>(n) * d->kp);
  if (e == cudaSuccess) e = cudaMalloc(&d->colsum, sizeof(int32_t) * n);
  if (e == cudaSuccess) e = cudaMalloc(&d->zp, sizeof(int32_t) * n);
  if (e == cudaSuccess) e = cudaMemsetAsync(d->colsum, 0, sizeof(int32_t) * n, ctx->stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(d->zp, zp.data(), sizeof(int32_t) * n, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess && host) {
    e = cudaMalloc(&staged, wbytes);
    if (e == cudaSuccess) e = cudaMemcpyAsync(staged, w, wbytes, cudaMemcpyHostToDevice, ctx->stream);
    w = staged;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    cudaFree(d->wt);
    cudaFree(d->colsum);
    cudaFree(d->zp);
    cudaFree(staged);
    delete d;
    return fail(OSC_ENOMEM, "osc_dqmm_prepack: %s", cudaGetErrorString(e));
  }
  dim3 grid((n + 31) / 32, (d->kp + 31) / 32);
  prof_begin(ctx);
  k_pack_dqmm_w<<<grid, 256, 0, ctx->stream>>>(static_cast<const int8_t*>(w), k, n, d->kp, d->is_signed, d->wt,
                                               d->colsum);
  int st = check_launch(ctx, "k_pack_dqmm_w");
  cudaStreamSynchronize(ctx->stream);  // the host zero-point vector above must outlive its copy
  if (staged) cudaFree(staged);
  if (st != OSC_OK) {
    osc_dqmm_weights_free(d);
    return st;
  }
  *out = d;
  return OSC_OK;
}

OSC_API int osc_dqmm_weights_free(osc_dqmm_weights* w) {
  if (w == nullptr) return OSC_OK;
  cudaSetDevice(w->device);
  cudaDeviceSynchronize();
  cudaFree(w->wt);
  cudaFree(w->colsum);
  cudaFree(w->zp);
  delete w;
  return OSC_OK;
}

OSC_API int osc_minmax_f32(osc_ctx* ctx, const float* x, long count, float* minmax_out) {
  OSC_TRY(enter(ctx));
  if (x == nullptr || minmax_out == nullptr || count < 0) return fail(OSC_EINVAL, "osc_minmax_f32: bad arguments");
  void* buf = nullptr;
  const int blocks = static_cast<int>(std::min<long>(std::max<long>((count / 4 + 255) / 256, 1), ctx->num_sms * 4L));
  OSC_TRY(scratch(ctx, sizeof(float2) * blocks + 256, &buf));
  prof_begin(ctx);
  k_minmax_partial<<<blocks, 256, 0, ctx->stream>>>(x, count, static_cast<float2*>(buf));
  OSC_TRY(check_launch(ctx, "k_minmax_partial"));
  prof_begin(ctx);
  k_minmax_final<<<1, 32, 0, ctx->stream>>>(static_cast<const float2*>(buf), blocks, minmax_out);
  return check_launch(ctx, "k_minmax_final");
}

}  // extern "C"

// The DynamicQuantizeMatMul of rows [row0, row0 + m) of an A with rows_total
// rows. The reference's epilogue rounds a row with one FMA when the row falls
// in the 12/6/4-row micro-kernel groups of the WHOLE matrix and with mul+add
// otherwise (GemmKernel.cs:746-790, 1594-1608); the grouped rows are a prefix
// of the matrix, so a shard's grouped rows are a prefix of the shard.
static int dqmm_rows(osc_ctx* ctx, const float* a, int m, int k, int lda, const osc_dqmm_weights* w,
                     const float* w_scale, int n_scale, const float* bias, float* y, const float* minmax_override,
                     int row0, int rows_total, uint8_t* q_out, int32_t* acc_out, float* params_out) {
  OSC_TRY(enter(ctx));
  if (w == nullptr) return fail(OSC_EINVAL, "osc_dqmm_f32: null weights");
  if (w->device != ctx->device) return fail(OSC_EINVAL, "osc_dqmm_f32: weights live on another device");
  if (k != w->k) return fail(OSC_EINVAL, "osc_dqmm_f32: A has k=%d, W has k=%d", k, w->k);
  if (n_scale != 1 && n_scale != w->n) return fail(OSC_EINVAL, "osc_dqmm_f32: %d scales for %d columns", n_scale, w->n);
  if (m < 0 || w_scale == nullptr) return fail(OSC_EINVAL, "osc_dqmm_f32: bad arguments");
  if (lda == 0) lda = k;
  if (lda < k) return fail(OSC_EINVAL, "osc_dqmm_f32: lda=%d < k=%d", lda, k);
  if (m == 0) return OSC_OK;
  if (a == nullptr || y == nullptr) return fail(OSC_EINVAL, "osc_dqmm_f32: null pointer");
  if (lda != k && minmax_override == nullptr)
    return fail(OSC_EUNSUPPORTED, "osc_dqmm_f32: strided A needs minmax_override (the range is per tensor)");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  const int kp = w->kp;
  // scratch: partials | params | q [m][kp] | rowsum [m] | nanrow [m]
  const size_t off_params = 8192, off_q = 8192 + 256;
  const size_t q_bytes = round_up(static_cast<size_t>(m) * kp, 256);
  const size_t off_rs = off_q + q_bytes, off_nan = off_rs + round_up(sizeof(int32_t) * m, 256);
  const size_t total = off_nan + round_up(sizeof(int32_t) * m, 256);
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, total, &buf));
  uint8_t* base = static_cast<uint8_t*>(buf);
  QParams* qp = reinterpret_cast<QParams*>(base + off_params);
  uint8_t* q = base + off_q;
  int32_t* rowsum = reinterpret_cast<int32_t*>(base + off_rs);
  int32_t* nanrow = reinterpret_cast<int32_t*>(base + off_nan);
  const int dql_ctas = std::min(m, ctx->num_sms);
  const int rows_per_cta = (m + dql_ctas - 1) / dql_ctas;
  const size_t dql_smem = static_cast<size_t>(rows_per_cta) * (static_cast<size_t>(k) * sizeof(float) + 8);
  if (dql_smem <= 200 * 1024) {
    // one cooperative launch: range, grid barrier, quantisation
    OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_dql_fused), static_cast<int>(dql_smem)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(dql_ctas));
    cfg.blockDim = dim3(kDqlThreads);
    cfg.dynamicSmemBytes = dql_smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    unsigned* sync = reinterpret_cast<unsigned*>(ctx->d_err) + 4;
    prof_begin(ctx);
    const cudaError_t le = cudaLaunchKernelEx(&cfg, k_dql_fused, a, m, k, lda, kp, rows_per_cta, 0, minmax_override,
                                              reinterpret_cast<float2*>(base), sync, qp, params_out, q, rowsum,
                                              nanrow, ctx->d_err);
    if (le != cudaSuccess) return cuda_fail(le, "k_dql_fused launch");
    OSC_TRY(check_launch(ctx, "k_dql_fused"));
  } else {
    OSC_TRY(minmax_params(ctx, a, static_cast<long>(m) * k, minmax_override, base, qp, params_out));
    const int blocks = std::min((m + 7) / 8, ctx->num_sms * 8);
    prof_begin(ctx);
    k_quantize_rows<<<blocks, 256, 0, ctx->stream>>>(a, m, k, lda, kp, qp, q, rowsum, nanrow);
    OSC_TRY(check_launch(ctx, "k_quantize_rows"));
  }
  if (q_out != nullptr)
    OSC_CUDA(cudaMemcpy2DAsync(q_out, k, q, kp, k, m, cudaMemcpyDeviceToDevice, ctx->stream), "copy q_out");
  DqmmArgs args{};
  args.M = m;
  args.N = w->n;
  args.K = k;
  args.num_kb = kp / kQBK;
  args.fused_rows = std::max(0, std::min(m, grouped_rows(rows_total) - row0));
  args.full_cols = (w->n / 16) * 16;
  args.qp = qp;
  args.rowsum = rowsum;
  args.nanrow = nanrow;
  args.colsum = w->colsum;
  args.wzp = w->zp;
  args.wscale = w_scale;
  args.n_scale = n_scale;
  args.bias = bias;
  args.y = y;
  args.acc_out = acc_out;
  args.has_wzp = w->has_zp;
  args.int_out = 0;
  return int8_gemm(ctx, q, kp, kp, 0, m, w, args);
}

extern "C" {

OSC_API int osc_dqmm_f32(osc_ctx* ctx, const float* a, int m, int k, int lda, const osc_dqmm_weights* w,
                         const float* w_scale, int n_scale, const float* bias, float* y, const float* minmax_override,
                         uint8_t* q_out, int32_t* acc_out, float* params_out) {
  return dqmm_rows(ctx, a, m, k, lda, w, w_scale, n_scale, bias, y, minmax_override, 0, m, q_out, acc_out,
                   params_out);
}

OSC_API int osc_dqmm_shard_f32(osc_ctx* ctx, const float* a, int m, int k, int lda, const osc_dqmm_weights* w,
                               const float* w_scale, int n_scale, const float* bias, float* y,
                               const float* minmax_global, int row0, int rows_total, uint8_t* q_out, int32_t* acc_out,
                               float* params_out) {
  if (minmax_global == nullptr) return fail(OSC_EINVAL, "osc_dqmm_shard_f32: the global range is required");
  if (row0 < 0 || m < 0 || rows_total < row0 + m)
    return fail(OSC_EINVAL, "osc_dqmm_shard_f32: rows [%d, %d) outside a tensor of %d rows", row0, row0 + m,
                rows_total);
  return dqmm_rows(ctx, a, m, k, lda, w, w_scale, n_scale, bias, y, minmax_global, row0, rows_total, q_out, acc_out,
                   params_out);
}

OSC_API int osc_dynamic_quantize_linear_f32(osc_ctx* ctx, const float* x, long long count, uint8_t* y,
                                            float* y_scale, uint8_t* y_zero_point) {
  OSC_TRY(enter(ctx));
  if (count < 0) return fail(OSC_EINVAL, "osc_dynamic_quantize_linear_f32: count=%lld", count);
  if (count > 0 && (x == nullptr || y == nullptr))
    return fail(OSC_EINVAL, "osc_dynamic_quantize_linear_f32: null pointer");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, 8192 + 256, &buf));
  uint8_t* base = static_cast<uint8_t*>(buf);
  QParams* qp = reinterpret_cast<QParams*>(base + 8192);
  // an empty tensor still has a range: {0, 0} -> scale 1, zero point 0
  OSC_TRY(minmax_params(ctx, x, static_cast<long>(count), nullptr, base, qp, nullptr));
  const int blocks = static_cast<int>(std::min<long long>(std::max<long long>((count / 4 + 255) / 256, 1),
                                                          static_cast<long long>(ctx->num_sms) * 8));
  prof_begin(ctx);
  k_quantize_flat<<<blocks, 256, 0, ctx->stream>>>(x, static_cast<long>(count), qp, y, y_scale, y_zero_point);
  return check_launch(ctx, "k_quantize_flat");
}

OSC_API int osc_matmul_integer_i8(osc_ctx* ctx, const void* a, int a_signed, int m, int k, int lda, int a_zero_point,
                                  const osc_dqmm_weights* w, int32_t* y) {
  OSC_TRY(enter(ctx));
  if (w == nullptr) return fail(OSC_EINVAL, "osc_matmul_integer_i8: null weights");
  if (w->device != ctx->device) return fail(OSC_EINVAL, "osc_matmul_integer_i8: weights live on another device");
  if (k != w->k) return fail(OSC_EINVAL, "osc_matmul_integer_i8: A has k=%d, B has k=%d", k, w->k);
  if (m < 0) return fail(OSC_EINVAL, "osc_matmul_integer_i8: m=%d", m);
  if (lda == 0) lda = k;
  if (lda < k) return fail(OSC_EINVAL, "osc_matmul_integer_i8: lda=%d < k=%d", lda, k);
  if (a_signed ? (a_zero_point < -128 || a_zero_point > 127) : (a_zero_point < 0 || a_zero_point > 255))
    return fail(OSC_EINVAL, "osc_matmul_integer_i8: a_zero_point %d out of range", a_zero_point);
  if (m == 0) return OSC_OK;
  if (a == nullptr || y == nullptr) return fail(OSC_EINVAL, "osc_matmul_integer_i8: null pointer");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  const int kp = w->kp;
  // TMA reads A in place when its rows are 16-byte aligned; otherwise a pitched copy
  const bool direct = (lda % 16) == 0 && (reinterpret_cast<uintptr_t>(a) & 15u) == 0;
  const size_t off_params = 0, off_rs = 256;
  const size_t off_nan = off_rs + round_up(sizeof(int32_t) * m, 256);
  const size_t off_q = off_nan + round_up(sizeof(int32_t) * m, 256);
  const size_t total = off_q + (direct ? 0 : round_up(static_cast<size_t>(m) * kp, 256));
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, total, &buf));
  uint8_t* base = static_cast<uint8_t*>(buf);
  QParams* qp = reinterpret_cast<QParams*>(base + off_params);
  int32_t* rowsum = reinterpret_cast<int32_t*>(base + off_rs);
  int32_t* nanrow = reinterpret_cast<int32_t*>(base + off_nan);
  const uint8_t* q = static_cast<const uint8_t*>(a);
  size_t q_pitch = static_cast<size_t>(lda);
  if (!direct) {
    uint8_t* qc = base + off_q;
    OSC_CUDA(cudaMemcpy2DAsync(qc, kp, a, lda, k, m, cudaMemcpyDeviceToDevice, ctx->stream), "copy A");
    q = qc;
    q_pitch = static_cast<size_t>(kp);
  }
  prof_begin(ctx);
  k_set_qparams<<<1, 1, 0, ctx->stream>>>(qp, a_zero_point);
  OSC_TRY(check_launch(ctx, "k_set_qparams"));
  prof_begin(ctx);
  k_rowsum_i8<<<std::min((m + 7) / 8, ctx->num_sms * 8), 256, 0, ctx->stream>>>(q, m, k, static_cast<long long>(q_pitch),
                                                                              a_signed, rowsum, nanrow);
  OSC_TRY(check_launch(ctx, "k_rowsum_i8"));
  DqmmArgs args{};
  args.M = m;
  args.N = w->n;
  args.K = k;
  args.num_kb = kp / kQBK;
  args.fused_rows = 0;
  args.full_cols = 0;
  args.qp = qp;
  args.rowsum = rowsum;
  args.nanrow = nanrow;
  args.colsum = w->colsum;
  args.wzp = w->zp;
  args.wscale = &qp->scale;  // unused by the s32 epilogue, but a valid address (the kernels load it)
  args.n_scale = 1;
  args.bias = nullptr;
  args.y = reinterpret_cast<float*>(y);
  args.acc_out = nullptr;
  args.has_wzp = w->has_zp;
  args.int_out = 1;
  return int8_gemm(ctx, q, q_pitch, k, a_signed, m, w, args);
}


// ---- failure detection: bounded device waits that run out.
// A kernel stuck behind a wait that can never complete (a CTA that never
// arrives, a copy that never lands) must end with an error the host can read
// instead of hanging the GPU. These probes make a wait run out on purpose,
// without faulting anything: the host then sees OSC_ETIMEDOUT from
// osc_synchronize, which also clears the error word and barrier counters.
__global__ void k_mbar_starved(int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);  // one arrival expected; none is ever made
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, err);
}

OSC_API int osc_selfcheck_timeout(osc_ctx* ctx, int which) {
  OSC_TRY(enter(ctx));
  if (which == 1) {
    prof_begin(ctx);
    k_mbar_starved<<<1, 32, 0, ctx->stream>>>(ctx->d_err);
    return check_launch(ctx, "k_mbar_starved");
  }
  if (which != 0) return fail(OSC_EINVAL, "osc_selfcheck_timeout: which=%d (0: grid barrier, 1: mbarrier)", which);
  // The DynamicQuantizeLinear kernel's grid barrier told to expect one CTA
  // more than the grid has: every CTA gives up after the wait limit.
  const int m = ctx->num_sms, k = 128, kp = 128;
  const size_t a_bytes = round_up(static_cast<size_t>(m) * k * sizeof(float), 256);
  const size_t off_part = a_bytes, off_params = off_part + 8192, off_q = off_params + 256;
  const size_t off_rs = off_q + round_up(static_cast<size_t>(m) * kp, 256);
  const size_t off_nan = off_rs + round_up(sizeof(int32_t) * m, 256);
  const size_t total = off_nan + round_up(sizeof(int32_t) * m, 256);
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, total, &buf));
  uint8_t* base = static_cast<uint8_t*>(buf);
  OSC_CUDA(cudaMemsetAsync(base, 0, a_bytes, ctx->stream), "zero probe input");
  const size_t smem = static_cast<size_t>(k) * sizeof(float) + 8;
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_dql_fused), static_cast<int>(smem)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(m));
  cfg.blockDim = dim3(kDqlThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  unsigned* sync = reinterpret_cast<unsigned*>(ctx->d_err) + 4;
  prof_begin(ctx);
  const cudaError_t le = cudaLaunchKernelEx(
      &cfg, k_dql_fused, reinterpret_cast<const float*>(base), m, k, k, kp, 1, 1, static_cast<const float*>(nullptr),
      reinterpret_cast<float2*>(base + off_part), sync, reinterpret_cast<QParams*>(base + off_params),
      static_cast<float*>(nullptr), base + off_q, reinterpret_cast<int32_t*>(base + off_rs),
      reinterpret_cast<int32_t*>(base + off_nan), ctx->d_err);
  if (le != cudaSuccess) return cuda_fail(le, "k_dql_fused launch (timeout probe)");
  return check_launch(ctx, "k_dql_fused");
}

}  // extern "C"
