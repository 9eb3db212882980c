// glue.cu — the memory-bound operators around the tensor-core kernels on the
// YOLO11n-shaped graph and the attention block: direct conv (first layer /
// depthwise), MaxPool, nearest Resize, broadcasting binary ops, unary
// activations, Softmax, DflSoftmax, the fused YOLO head decode and LayerNorm
// (CUDA cores, 128-bit accesses where the layout allows, warp-shuffle
// reductions), and the entry of the C2PSA attention, whose products run on the
// tensor cores (gemm_tf32x3.cu). Reference file:line per kernel.
//
// NCHW tensors may be channel slices of larger buffers: `*_nstride` is the
// element distance between consecutive images (0 = dense), so Split outputs
// are pointer offsets and Concat inputs are written in place.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "runtime.h"
#include "sm100.cuh"
#include "vmath.cuh"

namespace osc {
namespace {

inline int blocks_for(osc_ctx* ctx, long long work, int threads = 256, int per_sm = 16) {
  long long b = (work + threads - 1) / threads;
  const long long cap = static_cast<long long>(ctx->num_sms) * per_sm;
  if (b > cap) b = cap;
  return static_cast<int>(b < 1 ? 1 : b);
}

__device__ __forceinline__ float maxps(float a, float b) { return a > b ? a : b; }

// ---------------------------------------------------------------- direct conv
// Ops/DnnOps.cs:411-500 via Kernels/DepthwiseConv.cs:25-93 (groups == C == M)
// and Kernels/FirstConv.cs:54-121 (few input channels). One thread per output
// pixel and group, OCB output channels at a time; acc = bias, then FMA over
// (ic, ky, kx) ascending with padded taps contributing fmaf(w, 0, acc) (the
// im2col order of ConvKernels.cs:525-654).
template <int OCB>
__global__ void k_conv_direct(const float* __restrict__ x, long long x_nstride, int N, int C, int H, int W,
                              const float* __restrict__ w, int M, int kh, int kw, int sh, int sw, int pt, int pl,
                              int dh, int dw, int group, const float* __restrict__ bias, int act,
                              const float* __restrict__ res, long long res_nstride, float* __restrict__ y,
                              long long y_nstride, int OH, int OW) {
  const int cpg = C / group, mpg = M / group;
  const int ocb_per_group = (mpg + OCB - 1) / OCB;
  const long long total = static_cast<long long>(N) * group * ocb_per_group * OH * OW;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    long long t = i;
    const int ox = static_cast<int>(t % OW);
    t /= OW;
    const int oy = static_cast<int>(t % OH);
    t /= OH;
    const int ob = static_cast<int>(t % ocb_per_group);
    t /= ocb_per_group;
    const int g = static_cast<int>(t % group);
    const int n = static_cast<int>(t / group);
    const int oc0 = g * mpg + ob * OCB;
    const int noc = min(OCB, mpg - ob * OCB);
    float acc[OCB];
#pragma unroll
    for (int o = 0; o < OCB; ++o) acc[o] = (o < noc && bias) ? __ldg(bias + oc0 + o) : 0.0f;
    const float* xn = x + static_cast<size_t>(n) * x_nstride;
    for (int ic = 0; ic < cpg; ++ic) {
      const float* xc = xn + static_cast<size_t>(g * cpg + ic) * H * W;
      for (int ky = 0; ky < kh; ++ky) {
        const int iy = oy * sh - pt + ky * dh;
        for (int kx = 0; kx < kw; ++kx) {
          const int ix = ox * sw - pl + kx * dw;
          const float xv = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? __ldg(xc + static_cast<size_t>(iy) * W + ix) : 0.0f;
#pragma unroll
          for (int o = 0; o < OCB; ++o)
            if (o < noc)
              acc[o] = __fmaf_rn(__ldg(w + ((static_cast<size_t>(oc0 + o) * cpg + ic) * kh + ky) * kw + kx), xv, acc[o]);
        }
      }
    }
#pragma unroll
    for (int o = 0; o < OCB; ++o) {
      if (o >= noc) continue;
      const size_t off = (static_cast<size_t>(oc0 + o) * OH + oy) * OW + ox;
      float v = apply_act(acc[o], act);
      if (res) v = __fadd_rn(__ldg(res + static_cast<size_t>(n) * res_nstride + off), v);
      y[static_cast<size_t>(n) * y_nstride + off] = v;
    }
  }
}

// Direct conv with the whole weight tensor staged in shared memory (first
// layers: few input channels, M*C*kh*kw small). One thread per output pixel
// computes OCB output channels; same summation order as k_conv_direct.
template <int OCB>
__global__ void __launch_bounds__(256) k_conv_direct_smw(const float* __restrict__ x, long long x_nstride, int N,
                                                         int C, int H, int W, const float* __restrict__ w, int M,
                                                         int kh, int kw, int sh, int sw, int pt, int pl,
                                                         const float* __restrict__ bias, int act,
                                                         float* __restrict__ y, long long y_nstride, int OH, int OW) {
  extern __shared__ float sw_[];
  const int wn = M * C * kh * kw;
  for (int i = threadIdx.x; i < wn; i += blockDim.x) sw_[i] = __ldg(w + i);
  __syncthreads();
  const int ocbs = (M + OCB - 1) / OCB;
  const int plane = OH * OW;
  const long long total = static_cast<long long>(N) * ocbs * plane;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(i % plane);
    const long long t = i / plane;
    const int ob = static_cast<int>(t % ocbs);
    const int n = static_cast<int>(t / ocbs);
    const int oy = p / OW, ox = p - oy * OW;
    const int oc0 = ob * OCB;
    float acc[OCB];
#pragma unroll
    for (int o = 0; o < OCB; ++o) acc[o] = (oc0 + o < M && bias) ? __ldg(bias + oc0 + o) : 0.0f;
    const float* xn = x + static_cast<size_t>(n) * x_nstride;
    for (int ic = 0; ic < C; ++ic) {
      const float* xc = xn + static_cast<size_t>(ic) * H * W;
      for (int ky = 0; ky < kh; ++ky) {
        const int iy = oy * sh - pt + ky;
        for (int kx = 0; kx < kw; ++kx) {
          const int ix = ox * sw - pl + kx;
          const float xv = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? __ldg(xc + iy * W + ix) : 0.0f;
          const float* wp = sw_ + ((oc0 * C + ic) * kh + ky) * kw + kx;
#pragma unroll
          for (int o = 0; o < OCB; ++o)
            if (oc0 + o < M) acc[o] = __fmaf_rn(wp[o * C * kh * kw], xv, acc[o]);
        }
      }
    }
    float* yn = y + static_cast<size_t>(n) * y_nstride + p;
#pragma unroll
    for (int o = 0; o < OCB; ++o)
      if (oc0 + o < M) yn[static_cast<size_t>(oc0 + o) * plane] = apply_act(acc[o], act);
  }
}

// Depthwise conv (group == C == M), the head's and PSA's 3x3: one block per
// (image, channel, band of TH output rows); the input band plus halo is
// staged in shared memory, the k*k weights live in registers. Order per
// output: acc = bias, FMA over (ky, kx) with zero taps outside the image.
constexpr int kDwTH = 16;

template <int KS>
__global__ void __launch_bounds__(256) k_conv_depthwise(const float* __restrict__ x, long long x_nstride, int N, int C,
                                                        int H, int W, const float* __restrict__ w, int sh, int sw,
                                                        int pt, int pl, const float* __restrict__ bias, int act,
                                                        const float* __restrict__ res, long long res_nstride,
                                                        float* __restrict__ y, long long y_nstride, int OH, int OW) {
  extern __shared__ float tile[];
  const int nc = blockIdx.x;  // n * C + c
  const int n = nc / C, c = nc - n * C;
  const int oy0 = blockIdx.y * kDwTH;
  const int rows = min(kDwTH, OH - oy0);
  const int iy0 = oy0 * sh - pt;
  const int in_rows = (rows - 1) * sh + KS;
  const int in_cols = (OW - 1) * sw + KS;
  const float* xc = x + static_cast<size_t>(n) * x_nstride + static_cast<size_t>(c) * H * W;
  for (int i = threadIdx.x; i < in_rows * in_cols; i += blockDim.x) {
    const int r = i / in_cols, q = i - r * in_cols;
    const int iy = iy0 + r, ix = q - pl;
    tile[i] = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? __ldg(xc + iy * W + ix) : 0.0f;
  }
  float wr[KS * KS];
  const float* wc = w + static_cast<size_t>(c) * KS * KS;
#pragma unroll
  for (int t = 0; t < KS * KS; ++t) wr[t] = __ldg(wc + t);
  const float b = bias ? __ldg(bias + c) : 0.0f;
  __syncthreads();
  const size_t plane = static_cast<size_t>(OH) * OW;
  float* yc = y + static_cast<size_t>(n) * y_nstride + static_cast<size_t>(c) * plane;
  const float* rc = res ? res + static_cast<size_t>(n) * res_nstride + static_cast<size_t>(c) * plane : nullptr;
  for (int i = threadIdx.x; i < rows * OW; i += blockDim.x) {
    const int r = i / OW, ox = i - r * OW;
    float acc = b;
#pragma unroll
    for (int ky = 0; ky < KS; ++ky) {
      const float* trow = tile + (r * sh + ky) * in_cols + ox * sw;
#pragma unroll
      for (int kx = 0; kx < KS; ++kx) acc = __fmaf_rn(wr[ky * KS + kx], trow[kx], acc);
    }
    float v = apply_act(acc, act);
    const size_t off = static_cast<size_t>(oy0 + r) * OW + ox;
    if (rc) v = __fadd_rn(rc[off], v);
    yc[off] = v;
  }
}

// Depthwise 3x3, stride 1, pad 1: one thread per (plane, strip of kDw3Rows
// output rows, column). The (kDw3Rows + 2) x 3 input window goes into
// registers first (all its loads independent, so each thread keeps many in
// flight; the neighbouring columns are L1 hits), then each output takes
// acc = bias and the nine FMAs in (ky, kx) order with zero taps outside the
// image: the same arithmetic as k_conv_depthwise.
constexpr int kDw3Rows = 8;
constexpr int kDw3Threads = 256;

template <int ACT>
__global__ void __launch_bounds__(kDw3Threads) k_dw3s1(const float* __restrict__ x, long long x_nstride, int C, int H,
                                                       int W, const float* __restrict__ w,
                                                       const float* __restrict__ bias, const float* __restrict__ res,
                                                       long long res_nstride, float* __restrict__ y,
                                                       long long y_nstride, unsigned strips, unsigned total) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  const unsigned t = blockIdx.x * kDw3Threads + threadIdx.x;
  if (t >= total) return;
  const unsigned ps = t / static_cast<unsigned>(W);
  const int ox = static_cast<int>(t - ps * static_cast<unsigned>(W));
  const unsigned plane = ps / strips;
  const int oy0 = static_cast<int>(ps - plane * strips) * kDw3Rows;
  const unsigned n = plane / static_cast<unsigned>(C);
  const int c = static_cast<int>(plane - n * static_cast<unsigned>(C));
  const long long plane_off = static_cast<long long>(c) * H * W;
  const float* xc = x + static_cast<long long>(n) * x_nstride + plane_off;
  float in[kDw3Rows + 2][3];
#pragma unroll
  for (int r = 0; r < kDw3Rows + 2; ++r) {
    const int iy = oy0 - 1 + r;
    const bool row_ok = iy >= 0 && iy < H;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const int ix = ox - 1 + k;
      in[r][k] = (row_ok && ix >= 0 && ix < W) ? __ldg(xc + static_cast<long long>(iy) * W + ix) : 0.0f;
    }
  }
  float wr[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) wr[i] = __ldg(w + c * 9 + i);
  const float b = bias ? __ldg(bias + c) : 0.0f;
  float* yc = y + static_cast<long long>(n) * y_nstride + plane_off;
  const float* rc = res ? res + static_cast<long long>(n) * res_nstride + plane_off : nullptr;
#pragma unroll
  for (int r = 0; r < kDw3Rows; ++r) {
    const int oy = oy0 + r;
    if (oy < H) {
      float acc = b;
#pragma unroll
      for (int ky = 0; ky < 3; ++ky)
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) acc = __fmaf_rn(wr[ky * 3 + kx], in[r + ky][kx], acc);
      float v = act_t<ACT>(acc);
      const long long off = static_cast<long long>(oy) * W + ox;
      if (rc) v = __fadd_rn(__ldg(rc + off), v);
      yc[off] = v;
    }
  }
}

// The same with four adjacent columns per thread (W % 4 == 0, 16-byte
// aligned planes): per input row one float4 load plus the two halo columns,
// per output row one float4 store.
template <int ACT>
__global__ void __launch_bounds__(kDw3Threads) k_dw3s1_v4(const float* __restrict__ x, long long x_nstride, int C,
                                                          int H, int W, const float* __restrict__ w,
                                                          const float* __restrict__ bias,
                                                          const float* __restrict__ res, long long res_nstride,
                                                          float* __restrict__ y, long long y_nstride, unsigned strips,
                                                          unsigned total) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  const unsigned t = blockIdx.x * kDw3Threads + threadIdx.x;
  if (t >= total) return;
  const unsigned W4 = static_cast<unsigned>(W) >> 2;
  const unsigned ps = t / W4;
  const int ox = static_cast<int>(t - ps * W4) * 4;
  const unsigned plane = ps / strips;
  const int oy0 = static_cast<int>(ps - plane * strips) * kDw3Rows;
  const unsigned n = plane / static_cast<unsigned>(C);
  const int c = static_cast<int>(plane - n * static_cast<unsigned>(C));
  const long long plane_off = static_cast<long long>(c) * H * W;
  const float* xc = x + static_cast<long long>(n) * x_nstride + plane_off;
  float in[kDw3Rows + 2][6];  // columns ox-1 .. ox+4
#pragma unroll
  for (int r = 0; r < kDw3Rows + 2; ++r) {
    const int iy = oy0 - 1 + r;
    if (iy >= 0 && iy < H) {
      const float* xr = xc + static_cast<long long>(iy) * W + ox;
      const float4 v = __ldg(reinterpret_cast<const float4*>(xr));
      in[r][0] = ox > 0 ? __ldg(xr - 1) : 0.0f;
      in[r][1] = v.x;
      in[r][2] = v.y;
      in[r][3] = v.z;
      in[r][4] = v.w;
      in[r][5] = ox + 4 < W ? __ldg(xr + 4) : 0.0f;
    } else {
#pragma unroll
      for (int k = 0; k < 6; ++k) in[r][k] = 0.0f;
    }
  }
  float wr[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) wr[i] = __ldg(w + c * 9 + i);
  const float b = bias ? __ldg(bias + c) : 0.0f;
  float* yc = y + static_cast<long long>(n) * y_nstride + plane_off;
  const float* rc = res ? res + static_cast<long long>(n) * res_nstride + plane_off : nullptr;
#pragma unroll
  for (int r = 0; r < kDw3Rows; ++r) {
    const int oy = oy0 + r;
    if (oy < H) {
      float o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float acc = b;
#pragma unroll
        for (int ky = 0; ky < 3; ++ky)
#pragma unroll
          for (int kx = 0; kx < 3; ++kx) acc = __fmaf_rn(wr[ky * 3 + kx], in[r + ky][j + kx], acc);
        o[j] = act_t<ACT>(acc);
      }
      const long long off = static_cast<long long>(oy) * W + ox;
      if (rc) {
        const float4 rv = __ldg(reinterpret_cast<const float4*>(rc + off));
        o[0] = __fadd_rn(rv.x, o[0]);
        o[1] = __fadd_rn(rv.y, o[1]);
        o[2] = __fadd_rn(rv.z, o[2]);
        o[3] = __fadd_rn(rv.w, o[3]);
      }
      *reinterpret_cast<float4*>(yc + off) = make_float4(o[0], o[1], o[2], o[3]);
    }
  }
}

// Register-blocked tiled conv on CUDA cores for group-1 K x K (K = 1, 3)
// convs with few channels (the YOLO stem and the 8/16/32-channel layers, where
// a 128-row tensor-core tile and 32-channel K padding would waste most of the
// MMA and the hi/lo transform would dominate). Output tile per CTA: 8*G
// channels x (4*P rows x 32 columns); each thread owns 8 channels x 4
// adjacent pixels (32 accumulators). Input channels are staged CC at a time
// (tile + halo) together with the matching weights in [c][ky][kx][oc]
// order, double buffered: the halo tile by one TMA copy when the NCHW rows
// are 16-byte aligned (out-of-image rows, columns and channels arrive as
// zeros), else by 4-byte cp.async with src-size 0 for the padding. Per output
// the chain is acc = bias, then fmaf over (ic, ky, kx) ascending, the im2col
// order of ConvKernels.cs:525-654, so the result equals the reference's
// im2col path (padded taps give fmaf(w, 0, acc)).

// Packed FP32 (two lanes of a 64-bit register): fma.rn.f32x2 rounds each
// lane exactly as fmaf, so a pair of accumulators takes one instruction.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

template <int K, int S, int G, int P, bool TMA>
struct TileConv {
  static constexpr int OCB = 8 * G, TH = 4 * P, TW = 32;
  static constexpr int IH = (TH - 1) * S + K, IW = (TW - 1) * S + K;
  // TMA staging reads the halo row from the 16-byte aligned column below its
  // first column (pad_left = K/2 is required), so the halo starts D floats
  // into the shared row.
  static constexpr int D = TMA ? (4 - (K / 2) % 4) % 4 : 0;
  static constexpr int IP = (IW + D + 3) / 4 * 4;
  static constexpr int CC = S == 1 ? 8 : 4;
  static constexpr int NX = 3 * S + K;             // input columns one thread reads per row
  static constexpr int NXL = (D + NX + 3) / 4 * 4;  // floats loaded per row (16-byte loads)
  static constexpr int THREADS = 32 * G * P;
  static constexpr int XS = CC * IH * IP, WS = CC * K * K * OCB;
  static constexpr int STAGE = (XS + WS + 31) / 32 * 32;  // 128-byte aligned stages
  static constexpr int SMEM = 2 * STAGE * static_cast<int>(sizeof(float)) + (TMA ? 32 : 0);
  static_assert(IP <= 256, "TMA box width");
};

template <int K, int S, int G, int P, bool TMA>
__global__ void __launch_bounds__(32 * G * P) k_conv_tile(
    const __grid_constant__ CUtensorMap xmap, const float* __restrict__ x, long long x_nstride, int C, int H, int W,
    const float* __restrict__ w, int M, int pt, int pl, const float* __restrict__ bias, int act,
    const float* __restrict__ res, long long res_nstride, float* __restrict__ y, long long y_nstride, int OH, int OW,
    int tiles_x, bool vec4, int* __restrict__ err) {
  using T = TileConv<K, S, G, P, TMA>;
  extern __shared__ __align__(128) float smem_tile[];
  const int tid = threadIdx.x;
  const int n = blockIdx.z;
  const int oc0 = blockIdx.y * T::OCB;
  const int ty0 = (blockIdx.x / tiles_x) * T::TH, tx0 = (blockIdx.x % tiles_x) * T::TW;
  const int gy0 = ty0 * S - pt, gx0 = tx0 * S - pl;
  const float* xn = x + static_cast<size_t>(n) * x_nstride;
  const int chunks = (C + T::CC - 1) / T::CC;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_tile + 2 * T::STAGE);  // TMA: one barrier per stage
  int* abort_flag = reinterpret_cast<int*>(full + 2);
  if constexpr (TMA) {
    if (tid == 0) {
      mbar_init(&full[0], 1);
      mbar_init(&full[1], 1);
      *abort_flag = 0;
      fence_mbar_init();
      tma_prefetch(&xmap);
    }
    __syncthreads();
  }
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();

  auto issue = [&](int chunk) {
    float* xs = smem_tile + (chunk & 1) * T::STAGE;
    float* ws = xs + T::XS;
    const int c0 = chunk * T::CC;
    const int nc = min(T::CC, C - c0);
    if constexpr (TMA) {
      // the whole [CC][IH][IP] halo tile in one copy; out-of-image rows,
      // columns and channels read as zeros
      if (tid == 0) {
        mbar_arrive_expect_tx(&full[chunk & 1], T::XS * 4);
        tma_load_4d(xs, &xmap, &full[chunk & 1], gx0 - T::D, gy0, c0, n);
      }
    } else {
      for (int i = tid; i < nc * T::IH * T::IW; i += T::THREADS) {
        const int c = i / (T::IH * T::IW);
        const int rem = i - c * (T::IH * T::IW);
        const int iy = rem / T::IW, ix = rem - iy * T::IW;
        const int gy = gy0 + iy, gx = gx0 + ix;
        const bool ok = gy >= 0 && gy < H && gx >= 0 && gx < W;
        const float* src = ok ? xn + (static_cast<size_t>(c0 + c) * H + gy) * W + gx : xn;
        cp_async4(xs + (c * T::IH + iy) * T::IP + ix, src, ok);
      }
    }
    for (int i = tid; i < nc * K * K * T::OCB; i += T::THREADS) {
      const int o = i % T::OCB;
      const int ct = i / T::OCB;  // c * K*K + tap
      const int c = ct / (K * K), tap = ct - c * (K * K);
      const bool ok = oc0 + o < M;
      const float* src = ok ? w + (static_cast<size_t>(oc0 + o) * C + c0 + c) * (K * K) + tap : w;
      cp_async4(ws + i, src, ok);
    }
    cp_async_commit();
  };

  const int lane = tid & 31, wid = tid >> 5;
  const int og = wid % G, pg = wid / G;
  const int r = lane >> 3, cg = lane & 7;
  // accp[ip][j]: output channels 2ip (low lane) and 2ip+1 (high lane) at pixel j
  unsigned long long accp[4][4];
#pragma unroll
  for (int ip = 0; ip < 4; ++ip) {
    const int oc = oc0 + og * 8 + 2 * ip;
    const float b0 = (bias && oc < M) ? __ldg(bias + oc) : 0.0f;
    const float b1 = (bias && oc + 1 < M) ? __ldg(bias + oc + 1) : 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) accp[ip][j] = f2_pack(b0, b1);
  }

  issue(0);
  for (int chunk = 0; chunk < chunks; ++chunk) {
    if (chunk + 1 < chunks) {
      issue(chunk + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    if constexpr (TMA) mbar_wait(&full[chunk & 1], (chunk >> 1) & 1u, abort_flag, err);
    __syncthreads();
    const float* xs = smem_tile + (chunk & 1) * T::STAGE;
    const float* ws = xs + T::XS + og * 8;
    const int nc = min(T::CC, C - chunk * T::CC);
    // this thread's input columns start at cg*4*S + D; read 16-byte aligned
    const float* xrow0 = xs + ((pg * 4 + r) * S) * T::IP + cg * 4 * S;
    for (int c = 0; c < nc; ++c) {
#pragma unroll
      for (int ky = 0; ky < K; ++ky) {
        const float* xp = xrow0 + (c * T::IH + ky) * T::IP;
        float xl[T::NXL];
#pragma unroll
        for (int q = 0; q < T::NXL; q += 4) {
          const float4 v = *reinterpret_cast<const float4*>(xp + q);
          xl[q] = v.x;
          xl[q + 1] = v.y;
          xl[q + 2] = v.z;
          xl[q + 3] = v.w;
        }
        unsigned long long xd[T::NX];  // (x, x): each input column in both lanes
#pragma unroll
        for (int q = 0; q < T::NX; ++q) xd[q] = f2_pack(xl[T::D + q], xl[T::D + q]);
#pragma unroll
        for (int kx = 0; kx < K; ++kx) {
          const ulonglong2* wp = reinterpret_cast<const ulonglong2*>(ws + ((c * K + ky) * K + kx) * T::OCB);
          const ulonglong2 wa = wp[0], wb = wp[1];  // channel pairs (0,1) (2,3) | (4,5) (6,7)
          const unsigned long long wv[4] = {wa.x, wa.y, wb.x, wb.y};
#pragma unroll
          for (int ip = 0; ip < 4; ++ip)
#pragma unroll
            for (int j = 0; j < 4; ++j) accp[ip][j] = f2_fma(wv[ip], xd[j * S + kx], accp[ip][j]);
        }
      }
    }
    __syncthreads();
  }
  if constexpr (TMA) {
    // error path: a copy still in flight must land before the CTA exits
    // (each buffer's phases complete in order, so the last two chunks cover all)
    if (tid == 0 && *abort_flag) {
      for (int c = max(0, chunks - 2); c < chunks; ++c) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&full[c & 1], (c >> 1) & 1u) && globaltimer_ns() - t0 < 50ull * 1000ull * 1000ull) {
        }
      }
    }
  }

  float acc[8][4];
#pragma unroll
  for (int ip = 0; ip < 4; ++ip)
#pragma unroll
    for (int j = 0; j < 4; ++j) f2_unpack(accp[ip][j], acc[2 * ip][j], acc[2 * ip + 1][j]);
  const int oy = ty0 + pg * 4 + r, ox = tx0 + cg * 4;
  if (oy >= OH || ox >= OW) return;
  const size_t plane = static_cast<size_t>(OH) * OW;
  float* yn = y + static_cast<size_t>(n) * y_nstride + static_cast<size_t>(oy) * OW + ox;
  const float* rn = res ? res + static_cast<size_t>(n) * res_nstride + static_cast<size_t>(oy) * OW + ox : nullptr;
  with_act(act, [&](auto tag) {
    constexpr int ACT = decltype(tag)::value;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int oc = oc0 + og * 8 + i;
      if (oc >= M) break;
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = act_t<ACT>(acc[i][j]);
      const size_t off = static_cast<size_t>(oc) * plane;
      if (vec4 && ox + 4 <= OW) {
        if (rn) {
          const float4 rv = *reinterpret_cast<const float4*>(rn + off);
          v[0] = __fadd_rn(rv.x, v[0]);
          v[1] = __fadd_rn(rv.y, v[1]);
          v[2] = __fadd_rn(rv.z, v[2]);
          v[3] = __fadd_rn(rv.w, v[3]);
        }
        *reinterpret_cast<float4*>(yn + off) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (ox + j >= OW) break;
          yn[off + j] = rn ? __fadd_rn(rn[off + j], v[j]) : v[j];
        }
      }
    }
  });
}

template <int K, int S, int G, int P>
int launch_conv_tile(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W, const float* w,
                     int M, int pt, int pl, const float* bias, int act, const float* res, long long res_nstride,
                     float* y, long long y_nstride, int OH, int OW) {
  const int tiles_x = (OW + 31) / 32, tiles_y = (OH + 4 * P - 1) / (4 * P);
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec4 = OW % 4 == 0 && y_nstride % 4 == 0 && al16(y) &&
                    (res == nullptr || (res_nstride % 4 == 0 && al16(res)));
  dim3 grid(static_cast<unsigned>(tiles_x) * tiles_y, (M + 8 * G - 1) / (8 * G), N);
  // TMA-staged input tile when the NCHW rows are 16-byte aligned and the left
  // padding is K/2 (the halo column the tile's shared rows are aligned to)
  const bool tma = W % 4 == 0 && x_nstride % 4 == 0 && al16(x) && pl == K / 2 &&
                   static_cast<long long>(H) * W * 4 < (1ll << 40);
  CUtensorMap xmap{};
  if (tma) {
    using T = TileConv<K, S, G, P, true>;
    const uint64_t dims[4] = {static_cast<uint64_t>(W), static_cast<uint64_t>(H), static_cast<uint64_t>(C),
                              static_cast<uint64_t>(N)};
    const uint64_t pitch[3] = {static_cast<uint64_t>(W) * 4, static_cast<uint64_t>(H) * W * 4,
                               static_cast<uint64_t>(x_nstride) * 4};
    const uint32_t box[4] = {static_cast<uint32_t>(T::IP), static_cast<uint32_t>(T::IH), static_cast<uint32_t>(T::CC),
                             1};
    OSC_TRY(encode_tiled(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_NONE));
    OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_conv_tile<K, S, G, P, true>), T::SMEM));
    return launch_pdl(ctx, k_conv_tile<K, S, G, P, true>, grid, dim3(T::THREADS), T::SMEM, "k_conv_tile", xmap, x,
                      x_nstride, C, H, W, w, M, pt, pl, bias, act, res, res_nstride, y, y_nstride, OH, OW, tiles_x,
                      vec4, ctx->d_err);
  }
  using T = TileConv<K, S, G, P, false>;
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_conv_tile<K, S, G, P, false>), T::SMEM));
  return launch_pdl(ctx, k_conv_tile<K, S, G, P, false>, grid, dim3(T::THREADS), T::SMEM, "k_conv_tile", xmap, x,
                    x_nstride, C, H, W, w, M, pt, pl, bias, act, res, res_nstride, y, y_nstride, OH, OW, tiles_x, vec4,
                    ctx->d_err);
}

template <int K, int S>
int conv_tile_by_m(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W, const float* w, int M,
                   int pt, int pl, const float* bias, int act, const float* res, long long res_nstride, float* y,
                   long long y_nstride, int OH, int OW) {
  if (M <= 8)
    return launch_conv_tile<K, S, 1, 4>(ctx, x, x_nstride, N, C, H, W, w, M, pt, pl, bias, act, res, res_nstride, y,
                                        y_nstride, OH, OW);
  if (M <= 16)
    return launch_conv_tile<K, S, 2, 4>(ctx, x, x_nstride, N, C, H, W, w, M, pt, pl, bias, act, res, res_nstride, y,
                                        y_nstride, OH, OW);
  return launch_conv_tile<K, S, 4, 2>(ctx, x, x_nstride, N, C, H, W, w, M, pt, pl, bias, act, res, res_nstride, y,
                                      y_nstride, OH, OW);
}

// ---------------------------------------------------------------- MaxPool
// Ops/DnnOps.cs:1335 (MaxPoolLayer): max over the window's in-bounds elements,
// taken row by row, column by column (the reference's order, which decides
// which operand survives when a NaN is met). One CTA row per plane (n, c),
// 4 outputs per thread; the window re-reads hit L1.
constexpr int kPoolThreads = 128, kPoolPerThread = 4;

__global__ void __launch_bounds__(kPoolThreads) k_maxpool(const float* __restrict__ x, long long x_nstride, int C,
                                                          int H, int W, int kh, int kw, int sh, int sw, int pt, int pl,
                                                          float* __restrict__ y, long long y_nstride, int OH, int OW) {
  const int plane = blockIdx.x;
  const int n = plane / C, c = plane - n * C;
  const float* xc = x + static_cast<size_t>(n) * x_nstride + static_cast<size_t>(c) * H * W;
  float* yc = y + static_cast<size_t>(n) * y_nstride + static_cast<size_t>(c) * OH * OW;
  const int total = OH * OW;
  const int base = blockIdx.y * (kPoolThreads * kPoolPerThread) + threadIdx.x;
#pragma unroll
  for (int j = 0; j < kPoolPerThread; ++j) {
    const int o = base + j * kPoolThreads;
    if (o >= total) break;
    const int oy = o / OW, ox = o - oy * OW;
    float m = -INFINITY;
    for (int ky = 0; ky < kh; ++ky) {
      const int iy = oy * sh - pt + ky;
      if (iy < 0 || iy >= H) continue;
      const float* row = xc + static_cast<size_t>(iy) * W;
      for (int kx = 0; kx < kw; ++kx) {
        const int ix = ox * sw - pl + kx;
        if (ix < 0 || ix >= W) continue;
        m = maxps(__ldg(row + ix), m);
      }
    }
    yc[o] = m;
  }
}

// Planes up to 256 columns wide (the SPPF pools: 20x20): several planes per
// CTA, staged in shared memory inside a -inf border of the padding width, so
// no window tap needs a bounds check (maxps(-inf, m) keeps m, exactly as
// skipping the tap). One thread per (plane, column) stages its input column
// (loads in independent batches of kPoolBatch) and then slides down its output
// column: the row maxima of the last K rows sit in a register ring, and each
// output takes their maximum. With maxps(x, m) a NaN x never replaces m and m
// starts at -inf, so NaNs are skipped; among equal maxima the first in (ky, kx)
// order is kept both by the reference's row-major scan and by this separable
// form (the first row that attains the maximum, its first column), so signed
// zeros come out the same too.
constexpr int kPoolColThreads = 256;
constexpr int kPoolBatch = 8;

template <int K>
__global__ void __launch_bounds__(kPoolColThreads) k_maxpool_cols(
    const float* __restrict__ x, long long x_nstride, int C, int H, int W, int sh, int sw, int pt, int pl,
    float* __restrict__ y, long long y_nstride, int OH, int OW, long long planes, int ppc, int PH, int PW) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  extern __shared__ float pool_sm[];  // [ppc][PH][PW]
  const int PHW = PH * PW;
  const long long plane0 = static_cast<long long>(blockIdx.x) * ppc;
  const int np = static_cast<int>(min(static_cast<long long>(ppc), planes - plane0));
  for (int i = threadIdx.x; i < np * PHW; i += kPoolColThreads) pool_sm[i] = -INFINITY;
  __syncthreads();
  {
    const int p = threadIdx.x / W, col = threadIdx.x - p * W;
    if (p < np) {
      const long long g = plane0 + p, n = g / C, c = g - n * C;
      const float* src = x + n * x_nstride + c * H * W + col;
      float* dst = pool_sm + p * PHW + pt * PW + pl + col;
      for (int h0 = 0; h0 < H; h0 += kPoolBatch) {
        float v[kPoolBatch];
#pragma unroll
        for (int j = 0; j < kPoolBatch; ++j)
          v[j] = h0 + j < H ? __ldg(src + static_cast<long long>(h0 + j) * W) : 0.0f;
#pragma unroll
        for (int j = 0; j < kPoolBatch; ++j)
          if (h0 + j < H) dst[(h0 + j) * PW] = v[j];
      }
    }
  }
  __syncthreads();
  const int p = threadIdx.x / OW, ox = threadIdx.x - p * OW;
  if (p >= np) return;
  const long long g = plane0 + p, n = g / C, c = g - n * C;
  float* dst = y + n * y_nstride + c * OH * OW + ox;
  const float* colp = pool_sm + p * PHW + ox * sw;
  auto row_max = [&](int h) {
    const float* r = colp + h * PW;
    float m = -INFINITY;
#pragma unroll
    for (int kx = 0; kx < K; ++kx) m = maxps(r[kx], m);
    return m;
  };
  float ring[K];  // ring[0] = oldest row of the window
#pragma unroll
  for (int k = 0; k + 1 < K; ++k) ring[k + 1] = row_max(k);
  for (int oy = 0, h = K - 1; oy < OH; ++h) {
#pragma unroll
    for (int k = 0; k + 1 < K; ++k) ring[k] = ring[k + 1];
    ring[K - 1] = row_max(h);
    if (h - (K - 1) == oy * sh) {
      float m = -INFINITY;
#pragma unroll
      for (int k = 0; k < K; ++k) m = maxps(ring[k], m);
      dst[static_cast<long long>(oy) * OW] = m;
      ++oy;
    }
  }
}

// ---------------------------------------------------------------- Resize (nearest, integer up-scale)
// Ops/DnnOps.cs:2215 (ResizeLayer), nearest mode with integer scales:
// out[y][x] = in[y / sy][x / sx]. Grid: (planes, tiles of a plane).
__global__ void __launch_bounds__(256) k_resize_nearest(const float* __restrict__ x, long long x_nstride, int C, int H,
                                                        int W, int sy, int sx, float* __restrict__ y,
                                                        long long y_nstride) {
  const int plane = blockIdx.x;
  const int n = plane / C, c = plane - n * C;
  const int OH = H * sy, OW = W * sx;
  const float* xc = x + static_cast<size_t>(n) * x_nstride + static_cast<size_t>(c) * H * W;
  float* yc = y + static_cast<size_t>(n) * y_nstride + static_cast<size_t>(c) * OH * OW;
  const int o = blockIdx.y * 256 + threadIdx.x;
  if (o >= OH * OW) return;
  const int oy = o / OW, ox = o - oy * OW;
  yc[o] = __ldg(xc + (oy / sy) * W + ox / sx);
}

// 2x nearest up-scale: each thread reads 2 adjacent inputs (8 bytes) and writes
// the 2x4 output block as two 16-byte stores. Needs an even W and 16-byte
// aligned output rows (checked by the launcher).
__global__ void __launch_bounds__(256) k_resize_nearest2x(const float* __restrict__ x, long long x_nstride, int C,
                                                          int H, int W, float* __restrict__ y, long long y_nstride) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  const int plane = blockIdx.x;
  const int n = plane / C, c = plane - n * C;
  const int hw2 = (H * W) >> 1;
  const int i = blockIdx.y * 256 + threadIdx.x;
  if (i >= hw2) return;
  const float2 v = __ldg(reinterpret_cast<const float2*>(x + static_cast<size_t>(n) * x_nstride +
                                                         static_cast<size_t>(c) * H * W) + i);
  const int e = 2 * i, h = e / W, w = e - h * W;
  float* yc = y + static_cast<size_t>(n) * y_nstride + static_cast<size_t>(c) * 4 * H * W;
  const float4 q = make_float4(v.x, v.x, v.y, v.y);
  float4* r0 = reinterpret_cast<float4*>(yc + static_cast<size_t>(2 * h) * (2 * W) + 2 * w);
  r0[0] = q;
  r0[W >> 1] = q;  // the next output row starts 2W floats later
}

// ---------------------------------------------------------------- binary (numpy broadcasting, rank <= 4)
// Ops/BroadcastOps.cs / Tensors/TensorOps.cs: elementwise Add/Sub/Mul/Div.
struct Bcast {
  int rank;
  long long out_dims[4];
  long long a_strides[4], b_strides[4];  // 0 on broadcast dimensions
};

__global__ void k_binary(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y, Bcast bc,
                         long long total, int op) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    long long t = i, ia = 0, ib = 0;
    for (int d = bc.rank - 1; d >= 0; --d) {
      const long long c = t % bc.out_dims[d];
      t /= bc.out_dims[d];
      ia += c * bc.a_strides[d];
      ib += c * bc.b_strides[d];
    }
    const float x = __ldg(a + ia), z = __ldg(b + ib);
    float v;
    switch (op) {
      case 0: v = __fadd_rn(x, z); break;
      case 1: v = __fsub_rn(x, z); break;
      case 2: v = __fmul_rn(x, z); break;
      default: v = __fdiv_rn(x, z); break;
    }
    y[i] = v;
  }
}

// ---------------------------------------------------------------- unary (VectorMath bulk path)
__global__ void k_unary(const float* __restrict__ x, float* __restrict__ y, long long n, int act) {
  const long long n4 = n / 4;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15u) == 0;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long start = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
  if (vec) {
    for (long long i = start; i < n4; i += stride) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
      reinterpret_cast<float4*>(y)[i] =
          make_float4(apply_act(v.x, act), apply_act(v.y, act), apply_act(v.z, act), apply_act(v.w, act));
    }
  }
  for (long long i = (vec ? n4 * 4 : 0) + start; i < n; i += stride) y[i] = apply_act(x[i], act);
}

// ---------------------------------------------------------------- softmax over the last axis
// Ops/DnnOps.cs:2547 (SoftmaxLayer, inner == 1) -> VectorMath.SoftmaxRow
// (VectorMath.cs:282): max, exp (polynomial on 8-lane groups, MathF.Exp on the
// tail) summed in 8 lane partials then in order, then x * (1/sum).
// One warp per row; lane l holds the running partial of elements j with
// j % 8 == l % 8 for the vector part, combined in the reference's order.
__global__ void k_softmax_rows(const float* __restrict__ x, float* __restrict__ y, long long rows, int len) {
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const float* xr = x + r * len;
    float* yr = y + r * len;
    float mx = -INFINITY;
    for (int j = lane; j < len; j += 32) mx = fmaxf(mx, xr[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int vend = len & ~7;
    // lane l (< 8) accumulates elements l, l+8, l+16, ... of the vector part in order.
    float part = 0.0f;
    if (lane < 8)
      for (int j = lane; j < vend; j += 8) {
        const float e = ref_exp(__fsub_rn(xr[j], mx));
        yr[j] = e;
        part = __fadd_rn(part, e);
      }
    float total = 0.0f;
    for (int l = 0; l < 8; ++l) total = __fadd_rn(total, __shfl_sync(0xffffffffu, part, l));
    for (int j = vend; j < len; ++j) {  // scalar tail (uniform across the warp)
      const float e = expf(__fsub_rn(xr[j], mx));
      if (lane == 0) yr[j] = e;
      total = __fadd_rn(total, e);
    }
    __syncwarp();
    const float inv = __fdiv_rn(1.0f, total);
    for (int j = lane; j < len; j += 32) yr[j] = __fmul_rn(yr[j], inv);
  }
}

// ---------------------------------------------------------------- DflSoftmax
// Ops/DflOps.cs:167-250 (ApplyBlock): per column, max over bins, e_b = exp(x - max)
// (polynomial for the 8-aligned columns of each 64-column block, MathF.Exp on
// the tail), total = sum_b e_b in order, inv = 1/total, out = sum_b fma(e_b*inv, b, .)
// (tail columns: out += (e_b*inv)*b, unfused).
__device__ __forceinline__ float dfl_column(const float* src, long long stride, int bins, bool vector_col) {
  float mx = -INFINITY;
  for (int b = 0; b < bins; ++b) {
    const float v = __ldg(src + b * stride);
    mx = vector_col ? maxps(mx, v) : fmaxf(mx, v);
  }
  float e[32];
  float total = 0.0f;
#pragma unroll
  for (int b = 0; b < 32; ++b) {
    if (b >= bins) break;
    const float sh = __fsub_rn(__ldg(src + b * stride), mx);
    e[b] = vector_col ? ref_exp(sh) : expf(sh);
    total = __fadd_rn(total, e[b]);
  }
  const float inv = __fdiv_rn(1.0f, total);
  float acc = 0.0f;
#pragma unroll
  for (int b = 0; b < 32; ++b) {
    if (b >= bins) break;
    const float p = __fmul_rn(e[b], inv);
    acc = vector_col ? __fmaf_rn(p, static_cast<float>(b), acc) : __fadd_rn(acc, __fmul_rn(p, static_cast<float>(b)));
  }
  return acc;
}

__device__ __forceinline__ bool dfl_vector_col(int j, int pixels) {
  const int column = (j / 64) * 64;
  const int width = min(64, pixels - column);
  return (j - column) < (width & ~7);
}

__global__ void k_dfl(const float* __restrict__ x, int B, int sides, int bins, int pixels, float* __restrict__ out) {
  const long long total = static_cast<long long>(B) * sides * pixels;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(i % pixels);
    const long long gs = i / pixels;  // batch * sides + side
    out[i] = dfl_column(x + gs * bins * pixels + j, pixels, bins, dfl_vector_col(j, pixels));
  }
}

// ---------------------------------------------------------------- fused YOLO head decode
// The Detect head tail of the YOLO11n-shaped graph (model.23, nodes 302-319):
// per scale the box branch (64 = 4*16 DFL logits) and class branch (nc
// logits) are read in place from the head convs' outputs; DFL as above;
// dist2bbox exactly as the exported graph: x1y1 = anchor - lt, x2y2 =
// anchor + rb, c = (x1y1 + x2y2) / 2, wh = x2y2 - x1y1, both * stride; classes
// through Sigmoid (VectorMath.cs:70-74). Output [B, 4 + nc, A].
struct YoloScales {
  const float* box[3];   // [B, 64, h, w] views
  const float* cls[3];   // [B, nc, h, w] views
  long long box_nstride[3], cls_nstride[3];
  int h[3], w[3];
  float stride[3];
  int nc, total_anchors;
};

// Grid: x over anchors, y over images (strided when B exceeds the grid), so
// no per-element division splits a flat index.
__global__ void k_yolo_decode(const __grid_constant__ YoloScales s, int B, float* __restrict__ out) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  const int A = s.total_anchors;
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  if (a >= A) return;
  for (int n = blockIdx.y; n < B; n += gridDim.y) {
    int sc = 0, base = 0;
    while (sc < 2 && a >= base + s.h[sc] * s.w[sc]) {
      base += s.h[sc] * s.w[sc];
      ++sc;
    }
    const int p = a - base;
    const int hw = s.h[sc] * s.w[sc];
    const float ax = static_cast<float>(p % s.w[sc]) + 0.5f, ay = static_cast<float>(p / s.w[sc]) + 0.5f;
    const float* bx = s.box[sc] + static_cast<size_t>(n) * s.box_nstride[sc] + p;
    // The exported graph concatenates the three scales to [B, 144, A] before
    // DflSoftmax, so the 64-column block structure runs over A, not per scale.
    const bool vcol = dfl_vector_col(a, A);
    float d[4];
#pragma unroll
    for (int side = 0; side < 4; ++side) d[side] = dfl_column(bx + static_cast<size_t>(side) * 16 * hw, hw, 16, vcol);
    const float x1 = __fsub_rn(ax, d[0]), y1 = __fsub_rn(ay, d[1]);
    const float x2 = __fadd_rn(ax, d[2]), y2 = __fadd_rn(ay, d[3]);
    const float cx = __fdiv_rn(__fadd_rn(x1, x2), 2.0f), cy = __fdiv_rn(__fadd_rn(y1, y2), 2.0f);
    const float bw = __fsub_rn(x2, x1), bh = __fsub_rn(y2, y1);
    float* o = out + static_cast<size_t>(n) * (4 + s.nc) * A + a;
    const float st = s.stride[sc];
    o[0] = __fmul_rn(cx, st);
    o[static_cast<size_t>(A)] = __fmul_rn(cy, st);
    o[2 * static_cast<size_t>(A)] = __fmul_rn(bw, st);
    o[3 * static_cast<size_t>(A)] = __fmul_rn(bh, st);
    const float* cl = s.cls[sc] + static_cast<size_t>(n) * s.cls_nstride[sc] + p;
#pragma unroll 4
    for (int c = 0; c < s.nc; ++c)
      o[static_cast<size_t>(4 + c) * A] = ref_sigmoid(__ldg(cl + static_cast<size_t>(c) * hw));
  }
}

// ---------------------------------------------------------------- LayerNorm
// Ops/AttnOps.cs:199-358: sums of x and x^2 in 16 float lanes (AVX-512 path),
// lanes combined in double in order, tail in double; mean/var in double;
// y = ((x - mean) * inv_std) * gamma + beta. One warp per row; lanes 0..15
// own the 16 float lanes.
__global__ void k_layernorm(const float* __restrict__ x, int outer, int inner, const float* __restrict__ gamma,
                            const float* __restrict__ beta, float eps, float* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < outer; r += warps) {
    const float* xr = x + static_cast<size_t>(r) * inner;
    float* yr = y + static_cast<size_t>(r) * inner;
    const int vend = inner >= 16 ? (inner / 16) * 16 : 0;
    float s = 0.0f, q = 0.0f;
    if (lane < 16)
      for (int i = lane; i < vend; i += 16) {
        const float v = xr[i];
        s = __fadd_rn(s, v);
        q = __fadd_rn(q, __fmul_rn(v, v));
      }
    double sum = 0.0, sumsq = 0.0;
    for (int l = 0; l < 16; ++l) {
      sum += static_cast<double>(__shfl_sync(0xffffffffu, s, l));
      sumsq += static_cast<double>(__shfl_sync(0xffffffffu, q, l));
    }
    for (int i = vend; i < inner; ++i) {
      const float v = xr[i];
      sum += v;
      sumsq += static_cast<double>(v) * v;
    }
    const double mean_d = sum / inner;
    double var_d = sumsq / inner - mean_d * mean_d;
    if (var_d < 0) var_d = 0;
    const float mean = static_cast<float>(mean_d);
    const float inv_std = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(static_cast<float>(var_d), eps)));
    for (int j = lane; j < inner; j += 32) {
      float v = __fmul_rn(__fsub_rn(xr[j], mean), inv_std);
      if (gamma) v = __fmul_rn(v, __ldg(gamma + j));
      if (beta) v = __fadd_rn(v, __ldg(beta + j));
      yr[j] = v;
    }
  }
}

// Exhaustive check of recip_1up against the IEEE division over [1, 2^126).
__global__ void k_selfcheck_recip(unsigned long long* mismatches, unsigned int* first_bad) {
  const unsigned int lo = 0x3F800000u, hi = 0x7E800000u;  // bits of 1.0f and 2^126
  unsigned long long bad = 0;
  for (unsigned int i = lo + blockIdx.x * blockDim.x + threadIdx.x; i < hi; i += gridDim.x * blockDim.x) {
    const float d = __uint_as_float(i);
    if (__float_as_uint(recip_1up(d)) != __float_as_uint(__fdiv_rn(1.0f, d))) {
      ++bad;
      atomicMin(first_bad, i);
    }
  }
  for (int o = 16; o > 0; o >>= 1) bad += __shfl_xor_sync(0xffffffffu, bad, o);
  if ((threadIdx.x & 31) == 0 && bad) atomicAdd(mismatches, bad);
}

// The hardware-instruction sigmoid / SiLU of the tensor-core epilogues
// against the exact restatement, over every finite float x, in the parity
// metric |fast - exact| / max(1, |exact|). The maxima are non-negative floats,
// so their bit patterns order like the values (atomicMax on the bits).
__global__ void k_selfcheck_fast_act(unsigned int* max_sigmoid, unsigned int* max_silu) {
  float ms = 0.0f, mu = 0.0f;
  for (unsigned long long i = blockIdx.x * static_cast<unsigned long long>(blockDim.x) + threadIdx.x;
       i < 0x100000000ull; i += static_cast<unsigned long long>(gridDim.x) * blockDim.x) {
    const float x = __uint_as_float(static_cast<unsigned int>(i));
    if (!isfinite(x)) continue;
    const float s0 = ref_sigmoid(x), s1 = act_fast<ACT_SIGMOID>(x);
    const float u0 = ref_silu(x), u1 = act_fast<ACT_SILU>(x);
    ms = fmaxf(ms, fabsf(s1 - s0) / fmaxf(1.0f, fabsf(s0)));
    mu = fmaxf(mu, fabsf(u1 - u0) / fmaxf(1.0f, fabsf(u0)));
  }
  for (int o = 16; o > 0; o >>= 1) {
    ms = fmaxf(ms, __shfl_xor_sync(0xffffffffu, ms, o));
    mu = fmaxf(mu, __shfl_xor_sync(0xffffffffu, mu, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMax(max_sigmoid, __float_as_uint(ms));
    atomicMax(max_silu, __float_as_uint(mu));
  }
}

}  // namespace
}  // namespace osc

using namespace osc;

extern "C" {

OSC_API int osc_selfcheck_fast_act(osc_ctx* ctx, float* max_sigmoid_err, float* max_silu_err) {
  OSC_TRY(enter(ctx));
  if (max_sigmoid_err == nullptr || max_silu_err == nullptr)
    return fail(OSC_EINVAL, "osc_selfcheck_fast_act: null output");
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, 256, &buf));
  auto* d = static_cast<unsigned int*>(buf);
  OSC_CUDA(cudaMemsetAsync(d, 0, 2 * sizeof(unsigned int), ctx->stream), "selfcheck reset");
  prof_begin(ctx);
  k_selfcheck_fast_act<<<ctx->num_sms * 8, 256, 0, ctx->stream>>>(d, d + 1);
  OSC_TRY(check_launch(ctx, "k_selfcheck_fast_act"));
  unsigned int h[2] = {0, 0};
  OSC_CUDA(cudaMemcpyAsync(h, d, sizeof(h), cudaMemcpyDeviceToHost, ctx->stream), "selfcheck read");
  OSC_CUDA(cudaStreamSynchronize(ctx->stream), "selfcheck sync");
  std::memcpy(max_sigmoid_err, &h[0], sizeof(float));
  std::memcpy(max_silu_err, &h[1], sizeof(float));
  return OSC_OK;
}

OSC_API int osc_selfcheck_recip(osc_ctx* ctx, unsigned long long* mismatches, unsigned int* first_bad) {
  OSC_TRY(enter(ctx));
  if (mismatches == nullptr || first_bad == nullptr) return fail(OSC_EINVAL, "osc_selfcheck_recip: null output");
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, 256, &buf));
  auto* d_count = static_cast<unsigned long long*>(buf);
  auto* d_first = reinterpret_cast<unsigned int*>(d_count + 1);
  OSC_CUDA(cudaMemsetAsync(d_count, 0, sizeof(unsigned long long), ctx->stream), "selfcheck reset");
  OSC_CUDA(cudaMemsetAsync(d_first, 0xFF, sizeof(unsigned int), ctx->stream), "selfcheck reset");
  prof_begin(ctx);
  k_selfcheck_recip<<<ctx->num_sms * 8, 256, 0, ctx->stream>>>(d_count, d_first);
  OSC_TRY(check_launch(ctx, "k_selfcheck_recip"));
  OSC_CUDA(cudaMemcpyAsync(mismatches, d_count, sizeof(unsigned long long), cudaMemcpyDeviceToHost, ctx->stream),
           "selfcheck read");
  OSC_CUDA(cudaMemcpyAsync(first_bad, d_first, sizeof(unsigned int), cudaMemcpyDeviceToHost, ctx->stream),
           "selfcheck read");
  OSC_CUDA(cudaStreamSynchronize(ctx->stream), "selfcheck sync");
  if (*first_bad == 0xFFFFFFFFu) *first_bad = 0;
  return OSC_OK;
}

OSC_API int osc_conv2d_direct_f32(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W,
                                  const float* w, int M, int kh, int kw, int stride_h, int stride_w, int pad_t,
                                  int pad_l, int pad_b, int pad_r, int dil_h, int dil_w, int group, const float* bias,
                                  int act, const float* residual, long long res_nstride, float* y, long long y_nstride,
                                  int OH, int OW) {
  OSC_TRY(enter(ctx));
  if (group <= 0 || C % group || M % group) return fail(OSC_EINVAL, "osc_conv2d_direct_f32: group=%d", group);
  if (N < 0 || C <= 0 || H <= 0 || W <= 0 || M <= 0 || kh <= 0 || kw <= 0 || stride_h <= 0 || stride_w <= 0 ||
      dil_h <= 0 || dil_w <= 0 || pad_t < 0 || pad_l < 0 || pad_b < 0 || pad_r < 0)
    return fail(OSC_EINVAL, "osc_conv2d_direct_f32: bad geometry");
  const int oh = (H + pad_t + pad_b - ((kh - 1) * dil_h + 1)) / stride_h + 1;
  const int ow = (W + pad_l + pad_r - ((kw - 1) * dil_w + 1)) / stride_w + 1;
  if (oh != OH || ow != OW || oh <= 0 || ow <= 0)
    return fail(OSC_EINVAL, "osc_conv2d_direct_f32: output must be %dx%d, got %dx%d", oh, ow, OH, OW);
  const int act_code = act & ~OSC_ACT_FAST;
  if (act_code < OSC_ACT_NONE || act_code > OSC_ACT_SIGMOID)
    return fail(OSC_EINVAL, "osc_conv2d_direct_f32: act=%d", act);
  if (x_nstride == 0) x_nstride = static_cast<long long>(C) * H * W;
  if (y_nstride == 0) y_nstride = static_cast<long long>(M) * OH * OW;
  if (res_nstride == 0) res_nstride = static_cast<long long>(M) * OH * OW;
  if (N == 0) return OSC_OK;
  if (x == nullptr || w == nullptr || y == nullptr) return fail(OSC_EINVAL, "osc_conv2d_direct_f32: null pointer");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  const int mpg = M / group;
  const bool unit_dil = dil_h == 1 && dil_w == 1;
  // Depthwise 3x3, stride 1, "same" padding (the head's DWConv, PSA's
  // position encoding): register-window kernel.
  if (group == C && group == M && kh == 3 && kw == 3 && stride_h == 1 && stride_w == 1 && pad_t == 1 &&
      pad_l == 1 && OH == H && OW == W && unit_dil) {
    const long long strips = (H + kDw3Rows - 1) / kDw3Rows;
    const long long total = static_cast<long long>(N) * C * strips * W;
    const bool vec4 = W % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 && x_nstride % 4 == 0 &&
                      reinterpret_cast<uintptr_t>(y) % 16 == 0 && y_nstride % 4 == 0 &&
                      (residual == nullptr || (reinterpret_cast<uintptr_t>(residual) % 16 == 0 && res_nstride % 4 == 0));
    if (vec4 && total <= 0x7fffffffLL) {
      const long long total4 = total / 4;
      const unsigned blocks = static_cast<unsigned>((total4 + kDw3Threads - 1) / kDw3Threads);
      int st = OSC_OK;
      with_act(act, [&](auto tag) {
        st = launch_pdl(ctx, k_dw3s1_v4<decltype(tag)::value>, dim3(blocks), dim3(kDw3Threads), 0, "k_dw3s1_v4", x,
                        x_nstride, C, H, W, w, bias, residual, res_nstride, y, y_nstride,
                        static_cast<unsigned>(strips), static_cast<unsigned>(total4));
      });
      return st;
    }
    if (total <= 0x7fffffffLL) {
      const unsigned blocks = static_cast<unsigned>((total + kDw3Threads - 1) / kDw3Threads);
      int st = OSC_OK;
      with_act(act, [&](auto tag) {
        st = launch_pdl(ctx, k_dw3s1<decltype(tag)::value>, dim3(blocks), dim3(kDw3Threads), 0, "k_dw3s1", x,
                        x_nstride, C, H, W, w, bias, residual, res_nstride, y, y_nstride,
                        static_cast<unsigned>(strips), static_cast<unsigned>(total));
      });
      return st;
    }
  }
  // Depthwise (group == C == M), square 3/5/7 kernels: band-tiled kernel.
  if (group == C && group == M && kh == kw && (kh == 3 || kh == 5 || kh == 7) && unit_dil) {
    const int in_cols = (OW - 1) * stride_w + kw;
    const int in_rows = (kDwTH - 1) * stride_h + kh;
    const size_t smem = static_cast<size_t>(in_rows) * in_cols * sizeof(float);
    if (smem <= 48 * 1024) {
      dim3 grid(static_cast<unsigned>(N) * C, (OH + kDwTH - 1) / kDwTH);
      if (grid.x <= 2147483647u && grid.y <= 65535u) {
        prof_begin(ctx);
        if (kh == 3)
          k_conv_depthwise<3><<<grid, 256, smem, ctx->stream>>>(x, x_nstride, N, C, H, W, w, stride_h, stride_w, pad_t,
                                                                pad_l, bias, act, residual, res_nstride, y, y_nstride,
                                                                OH, OW);
        else if (kh == 5)
          k_conv_depthwise<5><<<grid, 256, smem, ctx->stream>>>(x, x_nstride, N, C, H, W, w, stride_h, stride_w, pad_t,
                                                                pad_l, bias, act, residual, res_nstride, y, y_nstride,
                                                                OH, OW);
        else
          k_conv_depthwise<7><<<grid, 256, smem, ctx->stream>>>(x, x_nstride, N, C, H, W, w, stride_h, stride_w, pad_t,
                                                                pad_l, bias, act, residual, res_nstride, y, y_nstride,
                                                                OH, OW);
        return check_launch(ctx, "k_conv_depthwise");
      }
    }
  }
  // Group-1 1x1 / 3x3 convs of stride 1 or 2: register-blocked tiles.
  if (group == 1 && unit_dil && kh == kw && (kh == 1 || kh == 3) && stride_h == stride_w &&
      (stride_h == 1 || stride_h == 2) && N <= 65535) {
    if (kh == 1 && stride_h == 1)
      return conv_tile_by_m<1, 1>(ctx, x, x_nstride, N, C, H, W, w, M, pad_t, pad_l, bias, act, residual, res_nstride,
                                  y, y_nstride, OH, OW);
    if (kh == 1)
      return conv_tile_by_m<1, 2>(ctx, x, x_nstride, N, C, H, W, w, M, pad_t, pad_l, bias, act, residual, res_nstride,
                                  y, y_nstride, OH, OW);
    if (stride_h == 1)
      return conv_tile_by_m<3, 1>(ctx, x, x_nstride, N, C, H, W, w, M, pad_t, pad_l, bias, act, residual, res_nstride,
                                  y, y_nstride, OH, OW);
    return conv_tile_by_m<3, 2>(ctx, x, x_nstride, N, C, H, W, w, M, pad_t, pad_l, bias, act, residual, res_nstride, y,
                                y_nstride, OH, OW);
  }
  // First layers (group 1, small weight tensor): weights staged in shared memory.
  const size_t wbytes = static_cast<size_t>(M) * C * kh * kw * sizeof(float);
  if (group == 1 && unit_dil && residual == nullptr && wbytes <= 48 * 1024) {
    const long long work = static_cast<long long>(N) * ((M + 15) / 16) * OH * OW;
    prof_begin(ctx);
    k_conv_direct_smw<16><<<blocks_for(ctx, work, 256, 32), 256, wbytes, ctx->stream>>>(
        x, x_nstride, N, C, H, W, w, M, kh, kw, stride_h, stride_w, pad_t, pad_l, bias, act, y, y_nstride, OH, OW);
    return check_launch(ctx, "k_conv_direct_smw");
  }
  prof_begin(ctx);
  if (mpg >= 8) {
    const long long work = static_cast<long long>(N) * group * ((mpg + 15) / 16) * OH * OW;
    k_conv_direct<16><<<blocks_for(ctx, work), 256, 0, ctx->stream>>>(x, x_nstride, N, C, H, W, w, M, kh, kw, stride_h,
                                                                       stride_w, pad_t, pad_l, dil_h, dil_w, group, bias,
                                                                       act, residual, res_nstride, y, y_nstride, OH, OW);
  } else {
    const long long work = static_cast<long long>(N) * group * mpg * OH * OW;
    k_conv_direct<1><<<blocks_for(ctx, work), 256, 0, ctx->stream>>>(x, x_nstride, N, C, H, W, w, M, kh, kw, stride_h,
                                                                      stride_w, pad_t, pad_l, dil_h, dil_w, group, bias,
                                                                      act, residual, res_nstride, y, y_nstride, OH, OW);
  }
  return check_launch(ctx, "k_conv_direct");
}

OSC_API int osc_maxpool2d_f32(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W, int kh,
                              int kw, int stride_h, int stride_w, int pad_t, int pad_l, int pad_b, int pad_r, float* y,
                              long long y_nstride, int OH, int OW) {
  OSC_TRY(enter(ctx));
  const int oh = (H + pad_t + pad_b - kh) / stride_h + 1, ow = (W + pad_l + pad_r - kw) / stride_w + 1;
  if (kh <= 0 || kw <= 0 || stride_h <= 0 || stride_w <= 0 || oh != OH || ow != OW || oh <= 0 || ow <= 0)
    return fail(OSC_EINVAL, "osc_maxpool2d_f32: bad geometry (expected %dx%d)", oh, ow);
  if (x_nstride == 0) x_nstride = static_cast<long long>(C) * H * W;
  if (y_nstride == 0) y_nstride = static_cast<long long>(C) * OH * OW;
  if (N == 0) return OSC_OK;
  const long long planes = static_cast<long long>(N) * C;
  const long long tiles = (static_cast<long long>(OH) * OW + kPoolThreads * kPoolPerThread - 1) /
                          (kPoolThreads * kPoolPerThread);
  if (planes > 0x7fffffffLL || tiles > 65535 || static_cast<long long>(H) * W > 0x7fffffffLL)
    return fail(OSC_EINVAL, "osc_maxpool2d_f32: %lld planes of %dx%d exceed the launch limits", planes, OH, OW);
  // square 2/3/5/7 windows on planes up to 256 columns wide whose bordered
  // copy fits 48 KB: column-sliding kernel, several planes per CTA
  const int PH = std::max(H + pad_t + pad_b, (OH - 1) * stride_h + kh);
  const int PW = std::max(W + pad_l + pad_r, (OW - 1) * stride_w + kw);
  const long long plane_bytes = static_cast<long long>(PH) * PW * 4;
  if (kh == kw && (kh == 2 || kh == 3 || kh == 5 || kh == 7) && pad_t >= 0 && pad_l >= 0 && pad_b >= 0 &&
      pad_r >= 0 && std::max(W, OW) <= kPoolColThreads && plane_bytes <= 48 * 1024) {
    const int ppc = static_cast<int>(
        std::min<long long>(kPoolColThreads / std::max(W, OW), (48 * 1024) / plane_bytes));
    const long long ctas = (planes + ppc - 1) / ppc;
    const size_t smem = static_cast<size_t>(ppc * plane_bytes);
    if (ctas <= 0x7fffffffLL) {
      const dim3 grid(static_cast<unsigned>(ctas));
#define OSC_POOL_LAUNCH(KS)                                                                                        \
  launch_pdl(ctx, k_maxpool_cols<KS>, grid, dim3(kPoolColThreads), smem, "k_maxpool_cols", x, x_nstride, C, H, W, \
             stride_h, stride_w, pad_t, pad_l, y, y_nstride, OH, OW, planes, ppc, PH, PW)
      if (kh == 2) return OSC_POOL_LAUNCH(2);
      if (kh == 3) return OSC_POOL_LAUNCH(3);
      if (kh == 5) return OSC_POOL_LAUNCH(5);
      return OSC_POOL_LAUNCH(7);
#undef OSC_POOL_LAUNCH
    }
  }
  prof_begin(ctx);
  k_maxpool<<<dim3(static_cast<unsigned>(planes), static_cast<unsigned>(tiles)), kPoolThreads, 0, ctx->stream>>>(
      x, x_nstride, C, H, W, kh, kw, stride_h, stride_w, pad_t, pad_l, y, y_nstride, OH, OW);
  return check_launch(ctx, "k_maxpool");
}

OSC_API int osc_resize_nearest_f32(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W,
                                   int scale_h, int scale_w, float* y, long long y_nstride) {
  OSC_TRY(enter(ctx));
  if (scale_h <= 0 || scale_w <= 0 || N < 0 || C <= 0 || H <= 0 || W <= 0)
    return fail(OSC_EINVAL, "osc_resize_nearest_f32: bad arguments");
  if (x_nstride == 0) x_nstride = static_cast<long long>(C) * H * W;
  if (y_nstride == 0) y_nstride = static_cast<long long>(C) * H * scale_h * W * scale_w;
  if (N == 0) return OSC_OK;
  const long long planes = static_cast<long long>(N) * C;
  const long long outs = static_cast<long long>(H) * scale_h * W * scale_w;
  if (planes > 0x7fffffffLL || (outs + 255) / 256 > 65535)
    return fail(OSC_EINVAL, "osc_resize_nearest_f32: %lld planes of %lld outputs exceed the launch limits", planes,
                outs);
  const bool vec2x = scale_h == 2 && scale_w == 2 && W % 2 == 0 && reinterpret_cast<uintptr_t>(x) % 8 == 0 &&
                     x_nstride % 2 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0 && y_nstride % 4 == 0;
  if (vec2x) {
    const long long pairs = static_cast<long long>(H) * W / 2;
    return launch_pdl(ctx, k_resize_nearest2x,
                      dim3(static_cast<unsigned>(planes), static_cast<unsigned>((pairs + 255) / 256)), dim3(256), 0,
                      "k_resize_nearest2x", x, x_nstride, C, H, W, y, y_nstride);
  }
  prof_begin(ctx);
  k_resize_nearest<<<dim3(static_cast<unsigned>(planes), static_cast<unsigned>((outs + 255) / 256)), 256, 0,
                     ctx->stream>>>(x, x_nstride, C, H, W, scale_h, scale_w, y, y_nstride);
  return check_launch(ctx, "k_resize_nearest");
}

OSC_API int osc_binary_f32(osc_ctx* ctx, int op, const float* a, const long long* a_shape, int a_rank, const float* b,
                           const long long* b_shape, int b_rank, float* y) {
  OSC_TRY(enter(ctx));
  if (op < 0 || op > 3 || a_rank < 0 || b_rank < 0 || a_rank > 4 || b_rank > 4)
    return fail(OSC_EINVAL, "osc_binary_f32: op %d, ranks %d/%d (rank <= 4)", op, a_rank, b_rank);
  Bcast bc{};
  bc.rank = std::max(a_rank, b_rank);
  if (bc.rank == 0) bc.rank = 1;
  long long as[4], bs[4];
  for (int d = 0; d < bc.rank; ++d) {
    const int da = d - (bc.rank - a_rank), db = d - (bc.rank - b_rank);
    as[d] = da >= 0 ? a_shape[da] : 1;
    bs[d] = db >= 0 ? b_shape[db] : 1;
    if (as[d] != bs[d] && as[d] != 1 && bs[d] != 1)
      return fail(OSC_EINVAL, "osc_binary_f32: shapes do not broadcast at axis %d (%lld vs %lld)", d, as[d], bs[d]);
    bc.out_dims[d] = std::max(as[d], bs[d]);
  }
  long long sa = 1, sb = 1, total = 1;
  for (int d = bc.rank - 1; d >= 0; --d) {
    bc.a_strides[d] = as[d] == 1 ? 0 : sa;
    bc.b_strides[d] = bs[d] == 1 ? 0 : sb;
    sa *= as[d];
    sb *= bs[d];
    total *= bc.out_dims[d];
  }
  if (total == 0) return OSC_OK;
  if (a == nullptr || b == nullptr || y == nullptr) return fail(OSC_EINVAL, "osc_binary_f32: null pointer");
  prof_begin(ctx);
  k_binary<<<blocks_for(ctx, total), 256, 0, ctx->stream>>>(a, b, y, bc, total, op);
  return check_launch(ctx, "k_binary");
}

OSC_API int osc_unary_f32(osc_ctx* ctx, const float* x, float* y, long long n, int act) {
  OSC_TRY(enter(ctx));
  if (act < OSC_ACT_NONE || act > OSC_ACT_SIGMOID || n < 0) return fail(OSC_EINVAL, "osc_unary_f32: bad arguments");
  if (n == 0) return OSC_OK;
  prof_begin(ctx);
  k_unary<<<blocks_for(ctx, n / 4 + 1), 256, 0, ctx->stream>>>(x, y, n, act);
  return check_launch(ctx, "k_unary");
}

OSC_API int osc_softmax_f32(osc_ctx* ctx, const float* x, float* y, long long rows, int len) {
  OSC_TRY(enter(ctx));
  if (rows < 0 || len <= 0) return fail(OSC_EINVAL, "osc_softmax_f32: bad shape");
  if (rows == 0) return OSC_OK;
  prof_begin(ctx);
  k_softmax_rows<<<blocks_for(ctx, rows * 32), 256, 0, ctx->stream>>>(x, y, rows, len);
  return check_launch(ctx, "k_softmax_rows");
}

OSC_API int osc_dfl_f32(osc_ctx* ctx, const float* x, int B, int sides, int bins, int pixels, float* out) {
  OSC_TRY(enter(ctx));
  if (B < 0 || sides <= 0 || bins <= 0 || bins > 32 || pixels <= 0)
    return fail(OSC_EINVAL, "osc_dfl_f32: bad shape (bins <= 32)");
  if (B == 0) return OSC_OK;
  prof_begin(ctx);
  k_dfl<<<blocks_for(ctx, static_cast<long long>(B) * sides * pixels), 256, 0, ctx->stream>>>(x, B, sides, bins,
                                                                                               pixels, out);
  return check_launch(ctx, "k_dfl");
}

OSC_API int osc_yolo_decode_f32(osc_ctx* ctx, int B, int nc, const float* const* box, const long long* box_nstride,
                                const float* const* cls, const long long* cls_nstride, const int* hs, const int* ws,
                                const float* strides, float* out) {
  OSC_TRY(enter(ctx));
  if (B < 0 || nc <= 0 || box == nullptr || cls == nullptr || hs == nullptr || ws == nullptr || strides == nullptr)
    return fail(OSC_EINVAL, "osc_yolo_decode_f32: bad arguments");
  YoloScales s{};
  s.nc = nc;
  s.total_anchors = 0;
  for (int i = 0; i < 3; ++i) {
    s.box[i] = box[i];
    s.cls[i] = cls[i];
    s.h[i] = hs[i];
    s.w[i] = ws[i];
    s.stride[i] = strides[i];
    s.box_nstride[i] = box_nstride[i] ? box_nstride[i] : 64LL * hs[i] * ws[i];
    s.cls_nstride[i] = cls_nstride[i] ? cls_nstride[i] : static_cast<long long>(nc) * hs[i] * ws[i];
    s.total_anchors += hs[i] * ws[i];
  }
  if (s.total_anchors <= 0 || hs[0] <= 0 || hs[1] <= 0 || hs[2] <= 0 || ws[0] <= 0 || ws[1] <= 0 || ws[2] <= 0)
    return fail(OSC_EINVAL, "osc_yolo_decode_f32: empty scale");
  if (B == 0) return OSC_OK;
  const dim3 grid(static_cast<unsigned>((s.total_anchors + 255) / 256), static_cast<unsigned>(std::min(B, 65535)));
  return launch_pdl(ctx, k_yolo_decode, grid, dim3(256), 0, "k_yolo_decode", s, B, out);
}

OSC_API int osc_layernorm_f32(osc_ctx* ctx, const float* x, int outer, int inner, const float* gamma,
                              const float* beta, float eps, float* y) {
  OSC_TRY(enter(ctx));
  if (outer < 0 || inner <= 0) return fail(OSC_EINVAL, "osc_layernorm_f32: bad shape");
  if (outer == 0) return OSC_OK;
  prof_begin(ctx);
  k_layernorm<<<blocks_for(ctx, static_cast<long long>(outer) * 32), 256, 0, ctx->stream>>>(x, outer, inner, gamma,
                                                                                             beta, eps, y);
  return check_launch(ctx, "k_layernorm");
}

// The attention of YOLO11's PSA block (model.10.m.0.attn, exported as
// Reshape/Split/Transpose/MatMul/Mul/Softmax/MatMul, shapes in the reference's
// tests/data/yolo11n.shapes.tsv nodes 123-134): from qkv [B, heads*(2*kd+hd), T]
// per head q [kd][T], k [kd][T], v [hd][T];
//   S[i][j] = (sum_c q[c][i] * k[c][j]) * scale   (MatMul, then Mul)
//   P = SoftmaxRow(S)                            (VectorMath.SoftmaxRow)
//   out[d][i] = sum_j v[d][j] * P[i][j]           (MatMul over j)
// YOLO11's head shape (kd 32, hd 64, T <= 512) runs as one fused kernel
// (psa_fused); other shapes take both products on the tensor cores
// (psa_composed).
OSC_API int osc_psa_attention_f32(osc_ctx* ctx, const float* qkv, long long qkv_nstride, int B, int heads, int kd,
                                  int hd, int T, float scale, float* out, long long out_nstride) {
  OSC_TRY(enter(ctx));
  if (B < 0 || heads <= 0 || kd <= 0 || hd <= 0 || T <= 0) return fail(OSC_EINVAL, "osc_psa_attention_f32: bad shape");
  if (qkv_nstride == 0) qkv_nstride = static_cast<long long>(heads) * (2 * kd + hd) * T;
  if (out_nstride == 0) out_nstride = static_cast<long long>(heads) * hd * T;
  if (B == 0) return OSC_OK;
  if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0 || out_nstride % 4 != 0)
    return fail(OSC_EINVAL, "osc_psa_attention_f32: out must be 16-byte aligned with a 4-element image stride");
  const int st = psa_fused(ctx, qkv, qkv_nstride, B, heads, kd, hd, T, scale, out, out_nstride);
  if (st != OSC_EUNSUPPORTED) return st;
  return psa_composed(ctx, qkv, qkv_nstride, B, heads, kd, hd, T, scale, out, out_nstride);
}

}  // extern "C"
