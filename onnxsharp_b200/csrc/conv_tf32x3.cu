// conv_tf32x3.cu — Conv(+bias, +fused activation) as an implicit GEMM on the
// sm_100a tensor cores (3xTF32), replacing the reference's CPU conv chain
// (ConvLayer.Forward, src/OnnxSharp/Ops/DnnOps.cs:411-500: depthwise /
// first-layer / NCHWc / Winograd / packed / im2col kernels, then an in-place
// SiLU pass, :493-499) for group == 1 convolutions.
//
// Mapping: D[oc][px] = W[oc][K] * X[px][K]^T with K ordered (ky, kx, c).
//  - A operand (M = 128 output channels): weights prepacked once into the
//    3xTF32 hi/lo split, [Mp][taps*Cp] K-major (osc_conv_prepack_f32).
//  - B operand (N = 256 output pixels, a BW x BH box of one image): the input
//    is transformed once per call from NCHW into "phase images" in NHWC with
//    the hi/lo split and channels padded to Cp = roundup(C, 32):
//    P[phase][n][h'][w'][c] = X[n][c][h'*s + py][w'*s + px], phase = py*s+px.
//    Tap (ky, kx) of a stride-s conv then reads a stride-1 box from one phase
//    image at offset (floor((ky*d-pt)/s), floor((kx*d-pl)/s)); pixels outside
//    the image are zeros written by the transform or TMA's out-of-bounds
//    fill (negative box coordinates are legal for loads; the channel
//    coordinate, innermost, is always a multiple of 32).
//  - Epilogue: bias[oc] + activation (Sigmoid/SiLU from the hardware ex2 /
//    rcp instructions, act_fast) and coalesced NCHW stores through a
//    shared-memory staging tile.
// The reference's im2col path accumulates acc = b[oc], then FMA over
// (ic, ky, kx) (Kernels/ConvKernels.cs:262-462); the tensor cores sum in a
// different order, so parity is |d| / max(1, |ref|) <= 1e-4.
#include <algorithm>
#include <cstdlib>

#include "runtime.h"
#include "sm100.cuh"
#include "tf32x3_core.cuh"
#include "vmath.cuh"

struct osc_conv_weights {
  int device = 0;
  int M = 0, C = 0, kh = 0, kw = 0;
  int Cp = 0, Kp = 0;    // channels padded to 32; Kp = kh*kw*Cp
  float* hi = nullptr;   // [M][Kp]
  float* lo = nullptr;
};

namespace osc {
namespace {

using ConvCfg = Tf32x3Cfg<256, 2, 2>;
constexpr int kMaxTaps = 49;

struct ConvTaps {
  int n_taps;
  int cp_blocks;                  // Cp / 32
  short phase[kMaxTaps];          // phase image index (py * s + px)
  short dy[kMaxTaps], dx[kMaxTaps];  // offsets inside the phase image
};

struct ConvGeom {
  int N, M, OH, OW;   // output
  int BW, BH;         // pixel box (BW * BH == 256, BW a power of two)
  int bw_log2;
  int tiles_w, tiles_h;
  int act;
  long long y_nstride;      // elements between images of y (>= M*OH*OW: y may be a channel slice)
  const float* res;         // optional residual added after the activation (same geometry as y)
  long long res_nstride;
  int vec4;                 // y (and res) rows allow 16-byte stores: OW, strides and bases multiples of 4 floats
};

// STACKED for layers of at most 64 output channels: 64-row weight boxes, the
// lo box landing right below the hi box, so [W hi; W lo] is one 128-row A
// operand; 2 MMAs per K step instead of 3 (see mma_loop), 80 KB stages
// instead of 96 KB; the epilogue adds D rows r and r + 64.
template <bool STACKED>
__global__ void __launch_bounds__(ConvCfg::THREADS, 1)
    k_conv_tf32x3(const __grid_constant__ CUtensorMap mWh, const __grid_constant__ CUtensorMap mWl,
                  const __grid_constant__ CUtensorMap mXh, const __grid_constant__ CUtensorMap mXl,
                  const __grid_constant__ ConvTaps taps, const __grid_constant__ ConvGeom g,
                  const float* __restrict__ bias, float* __restrict__ y, int* __restrict__ err) {
  using Cfg = ConvCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = tiles_base<Cfg>(smem_raw);
  PipeBarriers* pb = barriers<Cfg>(tiles);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int t = blockIdx.x;
  const int tx = t % g.tiles_w;
  t /= g.tiles_w;
  const int ty = t % g.tiles_h;
  const int n = t / g.tiles_h;
  const int ox0 = tx * g.BW, oy0 = ty * g.BH;
  const int m0 = blockIdx.y * kBM;
  const int num_kb = taps.n_taps * taps.cp_blocks;

  if (threadIdx.x == 0) {
    tma_prefetch(&mWh);
    tma_prefetch(&mWl);
    tma_prefetch(&mXh);
    tma_prefetch(&mXl);
  }
  const uint32_t tmem = pipe_setup<Cfg>(pb);
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();

  if (warp == 0) {
    if (lane == 0)
      producer_loop<Cfg>(tiles, pb, num_kb, err, [&](int kb, uint8_t* st, uint64_t* bar) {
        const int tap = kb / taps.cp_blocks;
        const int c0 = (kb - tap * taps.cp_blocks) * 32;
        const int kcol = kb * 32;  // == tap * Cp + c0
        tma_load_2d(st, &mWh, bar, kcol, m0);
        tma_load_2d(st + (STACKED ? Cfg::A_BYTES / 2 : Cfg::A_BYTES), &mWl, bar, kcol, m0);
        const int x = ox0 + taps.dx[tap], yy = oy0 + taps.dy[tap];
        const int nn = taps.phase[tap] * g.N + n;
        tma_load_4d(st + 2 * Cfg::A_BYTES, &mXh, bar, c0, x, yy, nn);
        tma_load_4d(st + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &mXl, bar, c0, x, yy, nn);
      }, static_cast<uint32_t>(STACKED ? Cfg::STAGE_BYTES - Cfg::A_BYTES : Cfg::STAGE_BYTES));
  } else if (warp == 1) {
    if (lane == 0) mma_loop<Cfg, STACKED>(tiles, pb, tmem, num_kb, err);
  } else {
    float acc[128];
    if (drain_loop<Cfg>(pb, tmem, num_kb, acc, err)) stage_tile<Cfg>(tiles, acc);
    const int jj = threadIdx.x - 64;  // bias of this tile's 128 channels
    if (jj < kBM)
      reinterpret_cast<float*>(tiles)[kBM * (Cfg::BN + 4) + jj] =
          (bias != nullptr && m0 + jj < g.M) ? __ldg(bias + m0 + jj) : 0.0f;
  }
  // All 10 warps (the producer and MMA warps are idle by now) write the staged
  // tile out: bias + activation (+ residual) and 16-byte coalesced stores.
  asm volatile("bar.sync 1, %0;" ::"r"(Cfg::THREADS) : "memory");
  if (!pb->abort_flag) {
    constexpr int kPitch = Cfg::BN + 4;
    const float* stage = reinterpret_cast<const float*>(tiles);
    const float* sbias = stage + kBM * kPitch;
    constexpr int kWarps = Cfg::THREADS / 32;
    with_act(g.act, [&](auto tag) {
      constexpr int ACT = decltype(tag)::value;
      // 4 channel rows per warp in flight (their residual loads overlap)
      for (int r0 = warp; r0 < kBM; r0 += 4 * kWarps) {
#pragma unroll
       for (int u = 0; u < 4; ++u) {
        const int r = r0 + u * kWarps;
        const int oc = m0 + r;
        if (r >= kBM || oc >= g.M) continue;
        const float b = sbias[r];
        const size_t plane_off = static_cast<size_t>(oc) * g.OH * g.OW;
        float* yplane = y + static_cast<size_t>(n) * g.y_nstride + plane_off;
        const float* rplane = g.res ? g.res + static_cast<size_t>(n) * g.res_nstride + plane_off : nullptr;
#pragma unroll
        for (int h = 0; h < Cfg::BN; h += 128) {
          const int p = h + lane * 4;  // 4 consecutive pixels of one box row (BW >= 8)
          const int oy = oy0 + (p >> g.bw_log2), ox = ox0 + (p & (g.BW - 1));
          if (oy >= g.OH) continue;
          float4 sv = *reinterpret_cast<const float4*>(stage + r * kPitch + p);
          if (STACKED) {  // W lo * X from D row r + 64
            const float4 lv = *reinterpret_cast<const float4*>(stage + (r + 64) * kPitch + p);
            sv = make_float4(__fadd_rn(sv.x, lv.x), __fadd_rn(sv.y, lv.y), __fadd_rn(sv.z, lv.z), __fadd_rn(sv.w, lv.w));
          }
          const float v[4] = {sv.x, sv.y, sv.z, sv.w};
          float* dst = yplane + static_cast<size_t>(oy) * g.OW + ox;
          const float* rsrc = rplane ? rplane + static_cast<size_t>(oy) * g.OW + ox : nullptr;
          float o[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) o[q] = act_fast<ACT>(__fadd_rn(v[q], b));
          if (g.vec4 && ox + 4 <= g.OW) {  // one 16-byte store: whole 32-byte sectors per warp
            if (rsrc) {
              const float4 rv = __ldg(reinterpret_cast<const float4*>(rsrc));
              o[0] = __fadd_rn(rv.x, o[0]);  // residual Add(x, act(conv)) as in the graph
              o[1] = __fadd_rn(rv.y, o[1]);
              o[2] = __fadd_rn(rv.z, o[2]);
              o[3] = __fadd_rn(rv.w, o[3]);
            }
            *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (ox + q < g.OW) dst[q] = rsrc ? __fadd_rn(rsrc[q], o[q]) : o[q];
          }
        }
       }
      }
    });
  }
  pipe_teardown<Cfg>(pb, tmem);
}

// ------------------------------------------------------------ pointwise (1x1)
// A 1x1, stride-1, unpadded conv is a GEMM per image, D[px][oc] =
// X[px][c] * W[oc][c]^T, whose A operand is the NCHW input itself: for a fixed
// channel the pixels are contiguous, i.e. A is MN-major. So the input is read
// straight from NCHW by TMA (no transform pass, 4 bytes per element instead of
// the transform's 4 + 8 and the conv's 8); two converter warps write its lo
// part (x - trunc_tf32(x)) beside it in shared memory, the landed fp32 tile
// being the hi part (a tf32 operand is read as its top 19 bits), and both
// feed tcgen05 through the A-MN-major descriptor.
//  - tile: 128 pixels (TMEM lanes) x up to 128 output channels (columns; the
//    MMA's N is the tile's channel count rounded to 16), or a 64-channel
//    tile with a deeper ring for layers of at most 64 output channels;
//  - stage: A as 4 TMA boxes of 32 pixels x 32 channels (4 KB each; the
//    128-byte swizzle with 32-byte atoms that MN-major TF32 operands need:
//    4-channel groups 512 bytes apart, 32-pixel groups 4 KB apart), its lo
//    part, and the prepacked weight hi/lo boxes (K-major);
//  - persistent CTAs walk the tiles; TMEM holds 4 accumulators (all 512
//    columns: 128 per accumulator on either tile width, the 64-channel tile
//    stacking its hi / lo weight products side by side), so the epilogue of
//    one tile overlaps the main loop of the next and the MMA runs several
//    TMEM chunks ahead of the drain;
//  - epilogue (16 warps, four per TMEM lane quadrant): lane = pixel, so each
//    warp store writes 32 consecutive pixels of one output channel (128
//    bytes): NCHW without a staging tile. Biases come from a shared-memory
//    table filled once per CTA.
namespace pw {
constexpr int kA = kBM * kBK * 4;         // 16 KB: 128 px x 32 ch
constexpr int kConvWarps = 2;
constexpr int kEpiWarps = 16;             // kEpiGroups per TMEM lane quadrant
constexpr int kEpiGroups = kEpiWarps / 4;
constexpr int kEpiBase = 2 + kConvWarps;  // first epilogue warp (a multiple of 4: warp % 4 = lane quadrant)
constexpr int kThreads = 32 * (kEpiBase + kEpiWarps);  // producer, MMA, converters, epilogue
constexpr int kKC = 2;                    // k-blocks per TMEM chunk
constexpr int kMaxStages = 4;
constexpr int kMaxBias = 4096;            // output channels whose biases fit the shared-memory table
constexpr int kMaxAcc = 8;                // TMEM accumulator buffers (all 512 columns on 64-channel tiles)
constexpr int kBarsBytes = 512;           // the barrier block (the bias table follows it)
struct Bars {
  uint64_t full[kMaxStages], conv[kMaxStages], empty[kMaxStages];
  uint64_t acc_full[kMaxAcc], acc_empty[kMaxAcc];
  uint64_t mma_done;
  uint32_t tmem_slot;
  int abort_flag;
};
// Per tile width: 128 output channels (3 stages of 64 KB) or 64 (4 stages of
// 48 KB): a stage is released only when its MMAs complete, so on layers with
// at most 64 output channels the narrower weight tile buys a deeper ring,
// i.e. more k-blocks in flight.
template <int BN>
struct Cfg {
  static constexpr int kBN = BN;                          // output channels per tile
  static constexpr int kStages = BN == 64 ? 4 : 3;
  static constexpr int kB = BN * kBK * 4;                 // one weight part: BN oc x 32 ch
  static constexpr int kStage = 2 * kA + 2 * kB;          // A (hi after the split) | A lo | W hi | W lo
  static constexpr int kTx = kA + 2 * kB;                 // bytes TMA lands per stage
  // 64-channel tiles stack [W hi; W lo] along N: per K step one MMA of
  // A hi against both weight parts (N = 64 + the tile's channels) and one of
  // A lo against W hi, instead of three N = 64 MMAs (an MMA costs at least
  // ~50 cycles, measured on B200: 51 at N = 64, 67 at N = 128). The
  // accumulator then spans 2 * BN columns: A*W hi in the first BN, A hi*W lo
  // in the next, added by the drain.
  static constexpr bool kStackN = BN == 64;
  static constexpr int kAccCols = kStackN ? 2 * BN : BN;
  // Every TMEM column: 512 / kAccCols accumulators, so the MMA runs up to that
  // many TMEM chunks ahead of the epilogue warps, which drain a chunk every
  // kKC k-blocks and also store the previous tile's outputs.
  static constexpr int kAccBufs = 512 / kAccCols;
  static constexpr int kTmemCols = 512;
  static constexpr int kColsMax = BN / kEpiGroups;        // output channels per epilogue warp on a full tile
  static constexpr int kSmemBase = kStages * kStage + 1024 + kBarsBytes;  // + the bias table (M floats, rounded to 16 bytes)
  static_assert(kStages <= kMaxStages, "stages");
  static_assert(kAccBufs <= kMaxAcc, "accumulator barriers");
  static_assert(kStage % 1024 == 0 && kA % 1024 == 0 && kB % 1024 == 0, "1024-byte aligned operand boxes");
  static_assert(kColsMax % 16 == 0, "TMEM drain granularity");
  static_assert(kSmemBase + kMaxBias * 4 <= 232448, "shared memory budget");
};
static_assert(kEpiBase % 4 == 0, "epilogue warps must start on a lane-quadrant boundary");
static_assert(sizeof(Bars) <= kBarsBytes, "barrier block");
}  // namespace pw

struct PwGeom {
  int C, HW, M;            // input channels, output pixels per image (OH*OW), output channels
  int ptiles, otiles;      // pixel tiles per image, channel tiles
  long long tiles;
  int num_kb;
  int act;
  long long y_nstride, res_nstride;
  const float* res;
  // TAPS form only: output geometry, the pixel box (BW x BH <= 128 pixels),
  // 32-channel blocks per tap, bytes of one A box
  int OW, OH, BW, BH, tiles_w, cp_blocks, a_bytes;
  int N;                   // images
  // split-K (few output tiles, long K): tile t is output tile t % base_tiles,
  // K slice t / base_tiles = TMEM chunks [slice * cps, slice * cps + cps);
  // each slice writes its raw sums to ws [ksplit][N][M][HW] and
  // k_conv_splitk_reduce adds them in slice order and applies the epilogue
  long long base_tiles;
  int ksplit, cps;
  float* ws;
};

// The tile's output tile and TMEM chunk / k-block range.
struct PwTile {
  int ot, pt, n, ks, c_begin, c_end, kb_begin, kb_end;
};
__device__ __forceinline__ PwTile pw_tile(const PwGeom& g, long long t, int nchunks, int kkc) {
  PwTile r;
  const long long tb = t % g.base_tiles;
  r.ks = static_cast<int>(t / g.base_tiles);
  r.ot = static_cast<int>(tb % g.otiles);
  const long long q = tb / g.otiles;
  r.pt = static_cast<int>(q % g.ptiles);
  r.n = static_cast<int>(q / g.ptiles);
  r.c_begin = r.ks * g.cps;
  r.c_end = min(nchunks, r.c_begin + g.cps);
  r.kb_begin = r.c_begin * kkc;
  r.kb_end = min(g.num_kb, r.c_end * kkc);
  return r;
}

// TAPS = false: the pointwise form above. TAPS = true: any K x K / stride
// conv on the same pixel-major tiles, its A operand read from the phase
// images of the NHWC hi/lo transform (K-major, one box of BW x BH pixels x 32
// channels per tap and channel block, hi and lo), no converter warps. Pixels
// as M spare the MMA the empty rows a channel-major tile has when the layer
// has only 32 or 64 output channels.
template <bool TAPS, int BN>
__global__ void __launch_bounds__(pw::kThreads, 1)
    k_conv_px_tf32x3(const __grid_constant__ CUtensorMap mX, const __grid_constant__ CUtensorMap mXl,
                     const __grid_constant__ CUtensorMap mWh, const __grid_constant__ CUtensorMap mWl,
                     const __grid_constant__ PwGeom g, const __grid_constant__ ConvTaps taps,
                     const float* __restrict__ bias, float* __restrict__ y, int* __restrict__ err) {
  using namespace pw;
  using CF = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* pb = reinterpret_cast<Bars*>(tiles + CF::kStages * CF::kStage);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < CF::kStages; ++s) {
      mbar_init(&pb->full[s], 1);
      mbar_init(&pb->conv[s], kConvWarps);
      mbar_init(&pb->empty[s], 1);
    }
    for (int b = 0; b < CF::kAccBufs; ++b) {
      mbar_init(&pb->acc_full[b], 1);
      mbar_init(&pb->acc_empty[b], kEpiWarps);
    }
    mbar_init(&pb->mma_done, 1);
    pb->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&mX);
    if (TAPS) tma_prefetch(&mXl);
    tma_prefetch(&mWh);
    tma_prefetch(&mWl);
  }
  if (warp == 1) {
    tmem_alloc(&pb->tmem_slot, CF::kTmemCols);
    tmem_relinquish();
  }
  // every output channel's bias, read once per CTA (the epilogue reads it from
  // shared memory instead of a global load in each store's dependency chain)
  float* s_bias = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(pb) + kBarsBytes);
  for (int j = threadIdx.x; j < g.M; j += kThreads) s_bias[j] = bias != nullptr ? __ldg(bias + j) : 0.0f;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = pb->tmem_slot;
  const int nchunks = (g.num_kb + kKC - 1) / kKC;
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      int i = 0;
      bool ok = true;
      const uint32_t tx_bytes = TAPS ? static_cast<uint32_t>(2 * g.a_bytes + 2 * CF::kB) : static_cast<uint32_t>(CF::kTx);
      for (long long t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
        const PwTile tl = pw_tile(g, t, nchunks, kKC);
        const int pt = tl.pt, n = tl.n;
        const int p0 = pt * kBM, oc0 = tl.ot * CF::kBN;
        const int ox0 = TAPS ? (pt % g.tiles_w) * g.BW : 0, oy0 = TAPS ? (pt / g.tiles_w) * g.BH : 0;
        for (int kb = tl.kb_begin; kb < tl.kb_end; ++kb) {
          const int s = i % CF::kStages;
          const uint32_t ph = (i / CF::kStages) & 1u;
          if (!mbar_wait(&pb->empty[s], ph ^ 1u, &pb->abort_flag, err)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&pb->full[s], tx_bytes);
          uint8_t* st = tiles + s * CF::kStage;
          if constexpr (TAPS) {
            const int tap = kb / g.cp_blocks;
            const int c0 = (kb - tap * g.cp_blocks) * kBK;
            const int xx = ox0 + taps.dx[tap], yy = oy0 + taps.dy[tap], nn = taps.phase[tap] * g.N + n;
            tma_load_4d(st, &mX, &pb->full[s], c0, xx, yy, nn);
            tma_load_4d(st + kA, &mXl, &pb->full[s], c0, xx, yy, nn);
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) tma_load_3d(st + q * 4096, &mX, &pb->full[s], p0 + 32 * q, kb * kBK, n);
          }
          tma_load_2d(st + 2 * kA, &mWh, &pb->full[s], kb * kBK, oc0);
          tma_load_2d(st + 2 * kA + CF::kB, &mWl, &pb->full[s], kb * kBK, oc0);
          ++i;
        }
      }
      if (!ok) {  // error path: let the copies in flight land before the CTA exits
        for (int j = i > CF::kStages ? i - CF::kStages : 0; j < i; ++j) {
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&pb->full[j % CF::kStages], (j / CF::kStages) & 1u) &&
                 globaltimer_ns() - t0 < 50ull * 1000ull * 1000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int i = 0, gc = 0;
      bool ok = true;
      for (long long t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
        const PwTile tl = pw_tile(g, t, nchunks, kKC);
        const int oc0 = tl.ot * CF::kBN;
        const int nn = min(CF::kBN, ((g.M - oc0) + 15) & ~15);
        const uint32_t idesc = TAPS ? idesc_tf32(kBM, nn) : idesc_tf32_amn(kBM, nn);
        const uint32_t idesc_st = TAPS ? idesc_tf32(kBM, CF::kBN + nn) : idesc_tf32_amn(kBM, CF::kBN + nn);
        int kb = tl.kb_begin;
        for (int c = tl.c_begin; c < tl.c_end && ok; ++c, ++gc) {
          const int buf = gc % CF::kAccBufs;
          if (!mbar_wait(&pb->acc_empty[buf], ((gc / CF::kAccBufs) & 1u) ^ 1u, &pb->abort_flag, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + static_cast<uint32_t>(buf * CF::kAccCols);
          const int kb_end = min(g.num_kb, kb + kKC);
          uint32_t acc = 0u;
          for (; kb < kb_end; ++kb, ++i) {
            const int s = i % CF::kStages;
            const uint32_t ph = (i / CF::kStages) & 1u;
            // pointwise: conv[s] follows full[s] (the converters waited on it);
            // the second wait returns at once and orders the weight boxes too
            if ((!TAPS && !mbar_wait(&pb->conv[s], ph, &pb->abort_flag, err)) ||
                !mbar_wait(&pb->full[s], ph, &pb->abort_flag, err)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t base = smem_addr(tiles + s * CF::kStage);
            const uint64_t dAh = TAPS ? sdesc_kmajor_sw128(base) : sdesc_mnmajor_sw128_32b(base, 4096, 512);
            const uint64_t dAl = TAPS ? sdesc_kmajor_sw128(base + kA) : sdesc_mnmajor_sw128_32b(base + kA, 4096, 512);
            const uint64_t dBh = sdesc_kmajor_sw128(base + 2 * kA);
            const uint64_t dBl = sdesc_kmajor_sw128(base + 2 * kA + CF::kB);
#pragma unroll
            for (int kk = 0; kk < kBK / 8; ++kk) {
              // +1024 bytes: the next 8 channel rows (MN-major); +32 bytes inside the K-major row
              const uint64_t ao = static_cast<uint64_t>(TAPS ? kk * 2 : kk * 64);
              const uint64_t bo = static_cast<uint64_t>(kk * 2);   // +32 bytes inside the K-major row
              if constexpr (CF::kStackN) {
                mma_tf32(d, dAh + ao, dBh + bo, idesc_st, acc);  // A hi * [W hi; W lo]
                acc = 1u;
                mma_tf32(d, dAl + ao, dBh + bo, idesc, 1u);      // A lo * W hi
              } else {
                mma_tf32(d, dAh + ao, dBh + bo, idesc, acc);
                acc = 1u;
                mma_tf32(d, dAh + ao, dBl + bo, idesc, 1u);
                mma_tf32(d, dAl + ao, dBh + bo, idesc, 1u);
              }
            }
            mma_commit(&pb->empty[s]);
          }
          if (ok) mma_commit(&pb->acc_full[buf]);
        }
      }
      // Every MMA issued so far completes before TMEM is released.
      mma_commit(&pb->mma_done);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&pb->mma_done, 0u) && globaltimer_ns() - t0 < 50ull * 1000ull * 1000ull) {
      }
    }
  } else if (warp < kEpiBase) {
    // converters (pointwise form only): the landed fp32 A stays in place as the
    // hi operand (a tf32 operand is read as its top 19 bits, i.e. trunc(x)),
    // and lo = x - trunc(x) (exact) is written beside it: one 16 KB write per
    // k-block instead of two, on a path bound by shared-memory bandwidth
    const int ct = threadIdx.x - 64;
    int i = 0;
    bool ok = !TAPS;
    for (long long t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
      const PwTile tl = pw_tile(g, t, nchunks, kKC);
      for (int kb = tl.kb_begin; kb < tl.kb_end; ++kb, ++i) {
        const int s = i % CF::kStages;
        const uint32_t ph = (i / CF::kStages) & 1u;
        bool got = mbar_wait(&pb->full[s], ph, &pb->abort_flag, err);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
          ok = false;
          break;
        }
        float4* a = reinterpret_cast<float4*>(tiles + s * CF::kStage);
        float4* al = reinterpret_cast<float4*>(tiles + s * CF::kStage + kA);
#pragma unroll 4
        for (int j = ct; j < kA / 16; j += 32 * kConvWarps) {
          const float4 v = a[j];
          constexpr uint32_t kTf32Mask = 0xffffe000u;  // sign, exponent, top 10 mantissa bits
          float4 l;
          l.x = __fsub_rn(v.x, __uint_as_float(__float_as_uint(v.x) & kTf32Mask));
          l.y = __fsub_rn(v.y, __uint_as_float(__float_as_uint(v.y) & kTf32Mask));
          l.z = __fsub_rn(v.z, __uint_as_float(__float_as_uint(v.z) & kTf32Mask));
          l.w = __fsub_rn(v.w, __uint_as_float(__float_as_uint(v.w) & kTf32Mask));
          al[j] = l;
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pb->conv[s]);
      }
    }
  } else {
    // epilogue: warp kEpiBase + 4h + q drains TMEM lanes 32q.. (pixels p0 + 32q + lane),
    // columns cpw*h .. (output channels oc0 + cpw*h ..): cpw = CF::kColsMax, or half
    // of it when the tile has at most 64 channels, so that every warp group
    // shares the drain, the activations and the stores of narrow tiles
    const int q = warp & 3;
    const int h = (warp - kEpiBase) >> 2;
    int gc = 0;
    bool ok = true;
    for (long long t = blockIdx.x; t < g.tiles && ok; t += gridDim.x) {
      const PwTile tl = pw_tile(g, t, nchunks, kKC);
      const int ot = tl.ot, pt = tl.pt, n = tl.n;
      const int cpw = CF::kColsMax >= 32 && g.M - ot * CF::kBN <= CF::kBN / 2 ? CF::kColsMax / 2 : CF::kColsMax;  // channels per warp
      const int oc0 = ot * CF::kBN + h * cpw;
      const int nvalid = min(cpw, g.M - oc0);  // may be <= 0 for the upper groups of a narrow tile
      float acc[CF::kColsMax];
      for (int c = tl.c_begin; c < tl.c_end; ++c, ++gc) {
        const int buf = gc % CF::kAccBufs;
        bool got = mbar_wait(&pb->acc_full[buf], (gc / CF::kAccBufs) & 1u, &pb->abort_flag, err);
        got = __all_sync(0xffffffffu, got);
        if (!got) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base =
            tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * CF::kAccCols + h * cpw);
        if constexpr (CF::kStackN) {  // 16 channels per warp: A * W hi plus A hi * W lo
          static_assert(CF::kColsMax == 16, "stacked drain");
          uint32_t r0[16], r1[16];
          tmem_ld16(base, r0);
          tmem_ld16(base + CF::kBN, r1);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float v = __fadd_rn(__uint_as_float(r0[j]), __uint_as_float(r1[j]));
            acc[j] = c == tl.c_begin ? v : __fadd_rn(acc[j], v);
          }
        } else {
#pragma unroll
        for (int gg = 0; gg < CF::kColsMax / 16; gg += CF::kColsMax > 32 ? 2 : 1) {
          if (gg * 16 >= cpw) break;
          const bool two = CF::kColsMax > 32 && (gg + 1) * 16 < cpw;  // 16-column groups in pairs on wide warps
          uint32_t r0[16], r1[16];
          tmem_ld16(base + gg * 16, r0);
          if (two) tmem_ld16(base + (gg + 1) * 16, r1);
          tmem_wait_ld();
          if (c == tl.c_begin) {
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[gg * 16 + j] = __uint_as_float(r0[j]);
            if (two) {
#pragma unroll
              for (int j = 0; j < 16; ++j) acc[(gg + 1) * 16 + j] = __uint_as_float(r1[j]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[gg * 16 + j] = __fadd_rn(acc[gg * 16 + j], __uint_as_float(r0[j]));
            if (two) {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                acc[(gg + 1) * 16 + j] = __fadd_rn(acc[(gg + 1) * 16 + j], __uint_as_float(r1[j]));
            }
          }
        }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pb->acc_empty[buf]);
      }
      if (!ok) break;
      // this lane's output pixel: linear in the plane (pointwise) or inside the BW x BH box (taps)
      int p;
      bool pvalid;
      if constexpr (TAPS) {
        const int pb_ = q * 32 + lane;
        const int iy = pb_ / g.BW, ix = pb_ - iy * g.BW;
        const int oy = (pt / g.tiles_w) * g.BH + iy, ox = (pt % g.tiles_w) * g.BW + ix;
        pvalid = iy < g.BH && oy < g.OH && ox < g.OW;
        p = oy * g.OW + ox;
      } else {
        p = pt * kBM + q * 32 + lane;
        pvalid = p < g.HW;
      }
      if (pvalid && nvalid > 0 && g.ksplit > 1) {  // this K slice's raw sums
        float* wp = g.ws + (static_cast<size_t>(tl.ks) * g.N + n) * g.M * static_cast<size_t>(g.HW) +
                    static_cast<size_t>(oc0) * g.HW + p;
#pragma unroll
        for (int j = 0; j < CF::kColsMax; ++j) {
          if (j >= cpw) break;
          if (j < nvalid) wp[static_cast<size_t>(j) * g.HW] = acc[j];
        }
      } else if (pvalid && nvalid > 0) {
        float* yp = y + static_cast<size_t>(n) * g.y_nstride + static_cast<size_t>(oc0) * g.HW + p;
        const float* rp =
            g.res ? g.res + static_cast<size_t>(n) * g.res_nstride + static_cast<size_t>(oc0) * g.HW + p : nullptr;
        const float* sb = s_bias + oc0;
        with_act(g.act, [&](auto tag) {
          constexpr int ACT = decltype(tag)::value;
#pragma unroll
          for (int j0 = 0; j0 < CF::kColsMax; j0 += 8) {
            if (j0 >= cpw) break;
            // residuals of 8 channels in flight at once (clamped rows, no branch between the loads)
            float rv[8];
            if (rp) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                rv[j] = __ldg(rp + static_cast<size_t>(min(j0 + j, nvalid - 1)) * g.HW);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int jj = min(j0 + j, nvalid - 1);
              float o = act_fast<ACT>(__fadd_rn(acc[j0 + j], sb[jj]));
              if (rp) o = __fadd_rn(rv[j], o);  // residual Add(x, act(conv)) as in the graph
              if (j0 + j < nvalid) yp[static_cast<size_t>(j0 + j) * g.HW] = o;
            }
          }
        });
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, CF::kTmemCols);
  }
}

// NCHW x -> phase-split NHWC hi/lo: out[(phase*N + n)][h'][w'][c], Cp channels,
// phase = py*s + px for input pixel (h'*s + py, w'*s + px). One block per
// (input row h < Hp*s, strip of 32*s input pixels, 32-channel strip; rows past
// the image give the zeros of the last phase rows): the row strip is
// read once with 16-byte loads (contiguous, all s phases at a time) and each
// of the s phase rows it feeds is written channel-innermost with 16-byte hi/lo
// stores.
constexpr int kPhaseMaxS = 4;
__global__ void __launch_bounds__(256) k_nchw_to_phase_nhwc(const float* __restrict__ x, long long x_nstride, int N,
                                                            int C, int H, int W, int s, int Hp, int Wp, int Cp,
                                                            int z_base, float* __restrict__ hi,
                                                            float* __restrict__ lo) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  __shared__ float tile[32][32 * kPhaseMaxS + 1];
  const int span = 32 * s;               // input pixels of this strip
  const int w0 = blockIdx.x * span;      // first input pixel
  const int c0 = blockIdx.y * 32;
  const int z = z_base + blockIdx.z;     // n * Hp*s + ih: rows ih >= H are the zero rows of the last phase row
  const int ih = z % (Hp * s), n = z / (Hp * s);
  const int tid = threadIdx.x;
  // read: thread -> channel tid/8, pixels (tid%8)*4 + 32*k for k < s
  {
    const int c = c0 + (tid >> 3);
    const float* src = x + static_cast<size_t>(n) * x_nstride + (static_cast<size_t>(c) * H + ih) * W;
    for (int k = 0; k < s; ++k) {
      const int wl = (tid & 7) * 4 + 32 * k, w = w0 + wl;
      float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (c < C && ih < H) {
        if (w + 4 <= W && (reinterpret_cast<uintptr_t>(src + w) & 15u) == 0) {
          const float4 t = __ldg(reinterpret_cast<const float4*>(src + w));
          v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (w + q < W) v[q] = __ldg(src + w + q);
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) tile[tid >> 3][wl + q] = v[q];
    }
  }
  __syncthreads();
  // write: for each column phase px, thread -> w' = tid/8 of the strip, channels (tid%8)*4..+3
  const int py = ih % s, hq = ih / s;
  const int wq = blockIdx.x * 32 + (tid >> 3);
  const int cq = (tid & 7) * 4;
  if (hq >= Hp || wq >= Wp || c0 + cq >= Cp) return;
  for (int px = 0; px < s; ++px) {
    const int wl = (tid >> 3) * s + px;  // input pixel of w' in this strip
    float h4[4], l4[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float v = tile[cq + q][wl];
      h4[q] = to_tf32(v);
      l4[q] = __fsub_rn(v, h4[q]);
    }
    const int phase = py * s + px;
    const size_t o = (((static_cast<size_t>(phase) * N + n) * Hp + hq) * Wp + wq) * Cp + c0 + cq;
    *reinterpret_cast<float4*>(hi + o) = make_float4(h4[0], h4[1], h4[2], h4[3]);
    *reinterpret_cast<float4*>(lo + o) = make_float4(l4[0], l4[1], l4[2], l4[3]);
  }
}

// Stride-1 fast path of the transform (a single phase image): NHWC of a
// stride-1 conv is [n][h*W + w][c], so per image it is a plain transpose of
// [C][HW] -> [HW][Cp] over the flattened plane (no per-row tiles, whose
// short rows at 20x20 or 40x40 would leave a third of each tile empty). One
// block moves 32 channels x 64 pixels: two 16-byte loads and two 16-byte hi
// and lo stores per thread.
__global__ void __launch_bounds__(256) k_nchw_to_nhwc_split(const float* __restrict__ x, long long x_nstride, int N,
                                                            int C, int HW, int Cp, int z_base,
                                                            float* __restrict__ hi, float* __restrict__ lo) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  __shared__ float tile[32][65];
  const int p0 = blockIdx.x * 64;
  const int c0 = blockIdx.y * 32;
  const int n = z_base + blockIdx.z;
  const int tid = threadIdx.x;
  {
    const int c = c0 + (tid >> 3), pl = (tid & 7) * 8, pp = p0 + pl;
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = 0.0f;
    if (c < C) {
      const float* src = x + static_cast<size_t>(n) * x_nstride + static_cast<size_t>(c) * HW + pp;
      if (pp + 8 <= HW && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        const float4 t0 = __ldg(reinterpret_cast<const float4*>(src));
        const float4 t1 = __ldg(reinterpret_cast<const float4*>(src) + 1);
        v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w;
        v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (pp + q < HW) v[q] = __ldg(src + q);
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) tile[tid >> 3][pl + q] = v[q];
  }
  __syncthreads();
  {
    const int pl = tid >> 2, cq = (tid & 3) * 8, pp = p0 + pl;
    if (pp < HW) {
      float h8[8], l8[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float v = tile[cq + q][pl];
        h8[q] = to_tf32(v);
        l8[q] = __fsub_rn(v, h8[q]);
      }
      const size_t o = (static_cast<size_t>(n) * HW + pp) * Cp + c0 + cq;
      *reinterpret_cast<float4*>(hi + o) = make_float4(h8[0], h8[1], h8[2], h8[3]);
      *reinterpret_cast<float4*>(hi + o + 4) = make_float4(h8[4], h8[5], h8[6], h8[7]);
      *reinterpret_cast<float4*>(lo + o) = make_float4(l8[0], l8[1], l8[2], l8[3]);
      *reinterpret_cast<float4*>(lo + o + 4) = make_float4(l8[4], l8[5], l8[6], l8[7]);
    }
  }
}

// Split-K epilogue of the pixel-major conv: y = act(sum_s ws[s] + bias) (+
// residual), the K slices added in slice order, then the same bias /
// activation / residual arithmetic as the kernel's own epilogue.
__global__ void __launch_bounds__(256) k_conv_splitk_reduce(const float* __restrict__ ws, int ksplit, int N, int M,
                                                            int HW, const float* __restrict__ bias, int act,
                                                            const float* __restrict__ res, long long res_nstride,
                                                            float* __restrict__ y, long long y_nstride) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  const long long total = static_cast<long long>(N) * M * HW;
  with_act(act, [&](auto tag) {
    constexpr int ACT = decltype(tag)::value;
    for (long long i = blockIdx.x * 256ll + threadIdx.x; i < total; i += static_cast<long long>(gridDim.x) * 256) {
      const int p = static_cast<int>(i % HW);
      const long long r = i / HW;
      const int oc = static_cast<int>(r % M), n = static_cast<int>(r / M);
      float v = ws[i];
      for (int k = 1; k < ksplit; ++k) v = __fadd_rn(v, ws[k * total + i]);
      float o = act_fast<ACT>(__fadd_rn(v, bias != nullptr ? __ldg(bias + oc) : 0.0f));
      if (res != nullptr) o = __fadd_rn(__ldg(res + n * res_nstride + static_cast<long long>(oc) * HW + p), o);
      y[n * y_nstride + static_cast<long long>(oc) * HW + p] = o;
    }
  });
}

// W[M][C][kh][kw] -> hi/lo [M][(ky*kw + kx)*Cp + c], zero for c >= C.
__global__ void k_pack_conv_w(const float* __restrict__ w, int M, int C, int kh, int kw, int Cp, float* __restrict__ hi,
                              float* __restrict__ lo) {
  const size_t total = static_cast<size_t>(M) * kh * kw * Cp;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % Cp);
    const size_t r = i / Cp;
    const int tap = static_cast<int>(r % (kh * kw));
    const int m = static_cast<int>(r / (kh * kw));
    const int ky = tap / kw, kx = tap % kw;
    const float v = c < C ? w[((static_cast<size_t>(m) * C + c) * kh + ky) * kw + kx] : 0.0f;
    const float h = to_tf32(v);
    hi[i] = h;
    lo[i] = __fsub_rn(v, h);
  }
}

int floor_div(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }

// Split-K for the pixel-major conv when its output tiles would leave most SMs
// idle (small batches, deep layers: e.g. 256 -> 64 3x3 at 20x20 and B=1 is 4
// tiles of 72 k-blocks): K is cut into slices of at least two TMEM chunks so
// that tiles x slices fills the SMs once. Sets base_tiles / ksplit / cps /
// tiles; returns the workspace bytes (0 without a split).
static size_t choose_ksplit(const osc_ctx* ctx, PwGeom& g) {
  const int nchunks = (g.num_kb + pw::kKC - 1) / pw::kKC;
  g.base_tiles = g.tiles;
  g.ksplit = 1;
  g.cps = nchunks;
  g.ws = nullptr;
  if (g.tiles >= ctx->num_sms || nchunks < 4) return 0;
  const int s = static_cast<int>(std::min<long long>(ctx->num_sms / g.tiles, nchunks / 2));
  if (s < 2) return 0;
  g.cps = (nchunks + s - 1) / s;
  g.ksplit = (nchunks + g.cps - 1) / g.cps;
  g.tiles = g.base_tiles * g.ksplit;
  return round_up(static_cast<size_t>(g.ksplit) * g.N * g.M * static_cast<size_t>(g.HW) * sizeof(float), 256);
}

static int splitk_reduce(osc_ctx* ctx, const PwGeom& g, const float* bias, int act, float* y) {
  const long long total = static_cast<long long>(g.N) * g.M * g.HW;
  const long long blocks = std::min<long long>((total + 255) / 256, static_cast<long long>(ctx->num_sms) * 8);
  return launch_pdl(ctx, k_conv_splitk_reduce, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                    "k_conv_splitk_reduce", g.ws, g.ksplit, g.N, g.M, g.HW, bias, act, g.res, g.res_nstride, y,
                    g.y_nstride);
}

}  // namespace

// Chooses the pixel box (BW x BH = 256) that wastes the least MMA work.
static void choose_box(int OH, int OW, int* BW, int* BH) {
  const int cands[5] = {32, 16, 64, 8, 128};
  long best = -1;
  for (int bw : cands) {
    const int bh = 256 / bw;
    const long cost = static_cast<long>((OW + bw - 1) / bw) * bw * (static_cast<long>((OH + bh - 1) / bh) * bh);
    if (best < 0 || cost < best) {
      best = cost;
      *BW = bw;
      *BH = bh;
    }
  }
}

// 1x1 / stride 1 / no padding, NCHW input with 4-aligned pixel planes: the
// transform-free pointwise kernel.
static bool pointwise_ok(const osc_conv_weights* w, const float* x, long long x_nstride, int H, int W, int sh,
                         int sw, int pt, int pl, int OH, int OW) {
  return w->kh == 1 && w->kw == 1 && w->M <= pw::kMaxBias && sh == 1 && sw == 1 && pt == 0 && pl == 0 &&
         OH == H && OW == W &&
         (static_cast<long long>(H) * W) % 4 == 0 && x_nstride % 4 == 0 &&
         (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
}

template <int BN>
static int conv1x1_launch(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int HW,
                          const osc_conv_weights* w, const float* bias, int act, const float* res,
                          long long res_nstride, float* y, long long y_nstride) {
  PwGeom g{};
  g.C = C;
  g.HW = HW;
  g.M = w->M;
  g.ptiles = (HW + kBM - 1) / kBM;
  g.otiles = (w->M + pw::Cfg<BN>::kBN - 1) / pw::Cfg<BN>::kBN;
  g.tiles = static_cast<long long>(N) * g.ptiles * g.otiles;
  g.num_kb = w->Cp / kBK;
  g.N = N;
  g.act = act;
  g.y_nstride = y_nstride;
  g.res_nstride = res_nstride;
  g.res = res;
  if (const size_t ws_bytes = choose_ksplit(ctx, g)) {
    void* ws = nullptr;
    OSC_TRY(scratch(ctx, ws_bytes, &ws));
    g.ws = static_cast<float*>(ws);
  }
  CUtensorMap mX, mWh, mWl;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(HW), static_cast<uint64_t>(C), static_cast<uint64_t>(N)};
    const uint64_t pitch[2] = {static_cast<uint64_t>(HW) * 4, static_cast<uint64_t>(x_nstride) * 4};
    const uint32_t box[3] = {32, kBK, 1};
    OSC_TRY(encode_tiled(&mX, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, x, dims, pitch, box,
                         CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(w->Kp), static_cast<uint64_t>(w->M)};
    const uint64_t pitch[1] = {static_cast<uint64_t>(w->Kp) * 4};
    const uint32_t box[2] = {kBK, pw::Cfg<BN>::kBN};
    OSC_TRY(encode_tiled(&mWh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w->hi, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
    OSC_TRY(encode_tiled(&mWl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w->lo, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  const int smem = pw::Cfg<BN>::kSmemBase + static_cast<int>(round_up(static_cast<size_t>(w->M) * 4, 16));
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_conv_px_tf32x3<false, BN>), smem));
  const long long grid = std::min<long long>(g.tiles, ctx->num_sms);
  const ConvTaps no_taps{};
  OSC_TRY(launch_pdl(ctx, k_conv_px_tf32x3<false, BN>, dim3(static_cast<unsigned>(grid)), dim3(pw::kThreads), smem,
                     "k_conv_px_tf32x3", mX, mX, mWh, mWl, g, no_taps, bias, y, ctx->d_err));
  return g.ksplit > 1 ? splitk_reduce(ctx, g, bias, act, y) : OSC_OK;
}

// Layers with at most 64 output channels take the 64-channel tile (4-stage
// ring), wider ones the 128-channel tile.
static int conv1x1_tf32x3(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int HW,
                          const osc_conv_weights* w, const float* bias, int act, const float* res,
                          long long res_nstride, float* y, long long y_nstride) {
  if (w->M <= 64)
    return conv1x1_launch<64>(ctx, x, x_nstride, N, C, HW, w, bias, act, res, res_nstride, y, y_nstride);
  return conv1x1_launch<128>(ctx, x, x_nstride, N, C, HW, w, bias, act, res, res_nstride, y, y_nstride);
}

// Pixel-major tiles for K x K convs with few output channels on small images
// (measured on B200, YOLO shapes at B=64: 256->64 and 64->64 3x3 at 20x20
// 19-24 % faster; at 40x40 and above the channel-major kernel's 256-pixel
// tiles move fewer operand bytes per output and win) -- and at any image size
// when the channel-major kernel would not fill two waves of the SMs (small
// batches: its 128-channel tiles leave half the MMA rows empty at <= 64
// output channels, and the persistent pixel-major kernel has twice the tiles).
// Wider layers take pixel tiles when the channel-major grid fills at most
// half the SMs (measured at B=8: 128->128 3x3 s2 at 40x40 16 % faster, at
// 20x20 10 %; 64->128 at 160x160 and B=1, 100 channel-major tiles, stays),
// and up to 128 channels on images of at most 24x24 (128->128 3x3 s2 at
// 20x20 and B=64: 19 % faster).
static bool px_taps_ok(const osc_ctx* ctx, int M, int N, int OH, int OW) {
  if (M > pw::kMaxBias) return false;
  int BW = 0, BH = 0;
  choose_box(OH, OW, &BW, &BH);
  const long tiles = static_cast<long>(N) * ((OW + BW - 1) / BW) * ((OH + BH - 1) / BH);
  // wider layers: when the channel-major grid fills at most half the SMs,
  // the pixel tiles (split along K where they are still few) fill them; up to
  // 128 channels also on small images
  if (M > 64)
    return 2 * tiles * ((M + kBM - 1) / kBM) <= ctx->num_sms || (M <= 128 && static_cast<long>(OH) * OW <= 576);
  if (static_cast<long>(OH) * OW <= 576) return true;
  return tiles < 2L * ctx->num_sms;
}

// The pixel box of the pixel-major conv: BW x BH <= 128 pixels, the shape
// with the fewest tiles (then the widest rows).
static void choose_px_box(int OH, int OW, int* BW, int* BH) {
  long best = -1;
  const int cands[6] = {OW, 128, 64, 32, 16, 8};
  for (int bw : cands) {
    if (bw < 1 || bw > 128) continue;
    const int bh = 128 / bw;
    const long tiles = static_cast<long>((OW + bw - 1) / bw) * ((OH + bh - 1) / bh);
    if (best < 0 || tiles < best || (tiles == best && bw > *BW)) {
      best = tiles;
      *BW = bw;
      *BH = bh;
    }
  }
}

// Output channels per pixel-major K x K tile: layers of at most 64 output
// channels take the 64-channel tile, whose weight boxes carry no zero rows and
// whose 48 KB stages give a 4-deep ring.
static int px_taps_bn(int M) { return M <= 64 ? 64 : 128; }

// Geometry of the pixel-major K x K conv (split-K included); returns the
// split workspace bytes (0 without a split).
static size_t px_taps_geom(const osc_ctx* ctx, const osc_conv_weights* w, int N, int OH, int OW, int act,
                           const float* res, long long res_nstride, long long y_nstride, PwGeom& g) {
  g = PwGeom{};
  g.C = w->C;
  g.HW = OH * OW;
  g.M = w->M;
  g.OW = OW;
  g.OH = OH;
  choose_px_box(OH, OW, &g.BW, &g.BH);
  g.tiles_w = (OW + g.BW - 1) / g.BW;
  g.ptiles = g.tiles_w * ((OH + g.BH - 1) / g.BH);
  g.otiles = (w->M + px_taps_bn(w->M) - 1) / px_taps_bn(w->M);
  g.tiles = static_cast<long long>(N) * g.ptiles * g.otiles;
  g.cp_blocks = w->Cp / kBK;
  g.num_kb = w->kh * w->kw * g.cp_blocks;
  g.N = N;
  g.a_bytes = g.BW * g.BH * kBK * 4;
  g.act = act;
  g.y_nstride = y_nstride;
  g.res_nstride = res_nstride;
  g.res = res;
  return choose_ksplit(ctx, g);
}

// g from px_taps_geom, with g.ws set when it asked for a workspace.
template <int BN>
static int conv_px_taps(osc_ctx* ctx, const float* xh, const float* xl, int N, int Hp, int Wp, int s,
                        const osc_conv_weights* w, const ConvTaps& taps, const PwGeom& g, const float* bias,
                        float* y) {
  CUtensorMap mXh, mXl, mWh, mWl;
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(w->Cp), static_cast<uint64_t>(Wp), static_cast<uint64_t>(Hp),
                              static_cast<uint64_t>(s) * s * N};
    const uint64_t pitch[3] = {static_cast<uint64_t>(w->Cp) * 4, static_cast<uint64_t>(w->Cp) * 4 * Wp,
                               static_cast<uint64_t>(w->Cp) * 4 * Wp * Hp};
    const uint32_t box[4] = {kBK, static_cast<uint32_t>(g.BW), static_cast<uint32_t>(g.BH), 1};
    OSC_TRY(encode_tiled(&mXh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xh, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
    OSC_TRY(encode_tiled(&mXl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xl, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(w->Kp), static_cast<uint64_t>(w->M)};
    const uint64_t pitch[1] = {static_cast<uint64_t>(w->Kp) * 4};
    const uint32_t box[2] = {kBK, pw::Cfg<BN>::kBN};
    OSC_TRY(encode_tiled(&mWh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w->hi, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
    OSC_TRY(encode_tiled(&mWl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w->lo, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  const int smem = pw::Cfg<BN>::kSmemBase + static_cast<int>(round_up(static_cast<size_t>(w->M) * 4, 16));
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_conv_px_tf32x3<true, BN>), smem));
  const long long grid = std::min<long long>(g.tiles, ctx->num_sms);
  OSC_TRY(launch_pdl(ctx, k_conv_px_tf32x3<true, BN>, dim3(static_cast<unsigned>(grid)), dim3(pw::kThreads), smem,
                     "k_conv_px_tf32x3", mXh, mXl, mWh, mWl, g, taps, bias, y, ctx->d_err));
  return g.ksplit > 1 ? splitk_reduce(ctx, g, bias, g.act, y) : OSC_OK;
}

int conv_tf32x3(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W, const osc_conv_weights* w,
                int sh, int sw, int pt, int pl, int dh, int dw, const float* bias, int act, const float* res,
                long long res_nstride, float* y, long long y_nstride, int OH, int OW) {
  if (pointwise_ok(w, x, x_nstride, H, W, sh, sw, pt, pl, OH, OW))
    return conv1x1_tf32x3(ctx, x, x_nstride, N, C, H * W, w, bias, act, res, res_nstride, y, y_nstride);
  if (sh != sw) return fail(OSC_EUNSUPPORTED, "conv: unequal strides %d x %d", sh, sw);
  const int s = sh;
  const int Hp = (H + s - 1) / s, Wp = (W + s - 1) / s;
  const int Cp = w->Cp;
  const bool px = px_taps_ok(ctx, w->M, N, OH, OW);
  PwGeom pg{};
  const size_t ws_bytes = px ? px_taps_geom(ctx, w, N, OH, OW, act, res, res_nstride, y_nstride, pg) : 0;
  // 1. input transform into the scratch arena (then the split-K workspace)
  const size_t plane = static_cast<size_t>(s) * s * N * Hp * Wp * Cp;
  const size_t half = round_up(plane * sizeof(float), 256);
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, 2 * half + ws_bytes, &buf));
  float* xh = static_cast<float*>(buf);
  float* xl = reinterpret_cast<float*>(static_cast<uint8_t*>(buf) + half);
  if (ws_bytes != 0) pg.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(buf) + 2 * half);
  {
    if (s > kPhaseMaxS) return fail(OSC_EUNSUPPORTED, "conv: stride %d (at most %d)", s, kPhaseMaxS);
    // s == 1: one z per image (flattened planes); s > 1: one z per input row (all phases of it), Hp*s rows per image
    const long zt = s == 1 ? static_cast<long>(N) : static_cast<long>(N) * Hp * s;
    const long zmax = 65535;  // gridDim.z limit: split into several launches
    for (long z0 = 0; z0 < zt; z0 += zmax) {
      const unsigned gx = s == 1 ? static_cast<unsigned>((static_cast<long>(H) * W + 63) / 64)
                                 : static_cast<unsigned>((Wp + 31) / 32);
      dim3 grid(gx, Cp / 32, static_cast<unsigned>(std::min(zmax, zt - z0)));
      if (s == 1)
        OSC_TRY(launch_pdl(ctx, k_nchw_to_nhwc_split, grid, dim3(256), 0, "k_nchw_to_nhwc_split", x, x_nstride, N, C,
                           H * W, Cp, static_cast<int>(z0), xh, xl));
      else
        OSC_TRY(launch_pdl(ctx, k_nchw_to_phase_nhwc, grid, dim3(256), 0, "k_nchw_to_phase_nhwc", x, x_nstride, N, C,
                           H, W, s, Hp, Wp, Cp, static_cast<int>(z0), xh, xl));
    }
  }
  // 2. tap table
  ConvTaps taps{};
  taps.n_taps = w->kh * w->kw;
  taps.cp_blocks = Cp / 32;
  for (int ky = 0; ky < w->kh; ++ky)
    for (int kx = 0; kx < w->kw; ++kx) {
      const int t = ky * w->kw + kx;
      const int oy = ky * dh - pt, ox = kx * dw - pl;
      const int py = ((oy % s) + s) % s, px = ((ox % s) + s) % s;
      taps.phase[t] = static_cast<short>(py * s + px);
      taps.dy[t] = static_cast<short>(floor_div(oy - py, s));
      taps.dx[t] = static_cast<short>(floor_div(ox - px, s));
    }
  if (px)
    return px_taps_bn(w->M) == 64 ? conv_px_taps<64>(ctx, xh, xl, N, Hp, Wp, s, w, taps, pg, bias, y)
                                  : conv_px_taps<128>(ctx, xh, xl, N, Hp, Wp, s, w, taps, pg, bias, y);
  ConvGeom g{};
  g.N = N;
  g.M = w->M;
  g.OH = OH;
  g.OW = OW;
  g.act = act;
  g.y_nstride = y_nstride;
  g.res = res;
  g.res_nstride = res_nstride;
  choose_box(OH, OW, &g.BW, &g.BH);
  g.bw_log2 = 0;
  while ((1 << g.bw_log2) < g.BW) ++g.bw_log2;
  {
    auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    g.vec4 = (OW % 4 == 0) && (y_nstride % 4 == 0) && al16(y) &&
             (res == nullptr || (res_nstride % 4 == 0 && al16(res)));
  }
  g.tiles_w = (OW + g.BW - 1) / g.BW;
  g.tiles_h = (OH + g.BH - 1) / g.BH;
  // 3. tensor maps
  CUtensorMap mWh, mWl, mXh, mXl;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(w->Kp), static_cast<uint64_t>(w->M)};
    const uint64_t pitch[1] = {static_cast<uint64_t>(w->Kp) * 4};
    const uint32_t box[2] = {kBK, w->M <= 64 ? 64u : static_cast<uint32_t>(kBM)};
    OSC_TRY(encode_tiled(&mWh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w->hi, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
    OSC_TRY(encode_tiled(&mWl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w->lo, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(Cp), static_cast<uint64_t>(Wp), static_cast<uint64_t>(Hp),
                              static_cast<uint64_t>(s) * s * N};
    const uint64_t pitch[3] = {static_cast<uint64_t>(Cp) * 4, static_cast<uint64_t>(Cp) * 4 * Wp,
                               static_cast<uint64_t>(Cp) * 4 * Wp * Hp};
    const uint32_t box[4] = {32, static_cast<uint32_t>(g.BW), static_cast<uint32_t>(g.BH), 1};
    OSC_TRY(encode_tiled(&mXh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xh, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
    OSC_TRY(encode_tiled(&mXl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, xl, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  const long tiles = static_cast<long>(g.tiles_w) * g.tiles_h * N;
  if (tiles > 2147483647L) return fail(OSC_EINVAL, "conv: too many tiles");
  dim3 grid(static_cast<unsigned>(tiles), (w->M + kBM - 1) / kBM);
  if (w->M <= 64) {
    OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_conv_tf32x3<true>), ConvCfg::SMEM_BYTES));
    return launch_pdl(ctx, k_conv_tf32x3<true>, grid, dim3(ConvCfg::THREADS), ConvCfg::SMEM_BYTES, "k_conv_tf32x3", mWh,
                      mWl, mXh, mXl, taps, g, bias, y, ctx->d_err);
  }
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_conv_tf32x3<false>), ConvCfg::SMEM_BYTES));
  return launch_pdl(ctx, k_conv_tf32x3<false>, grid, dim3(ConvCfg::THREADS), ConvCfg::SMEM_BYTES, "k_conv_tf32x3", mWh,
                    mWl, mXh, mXl, taps, g, bias, y, ctx->d_err);
}

}  // namespace osc

using namespace osc;

extern "C" {

OSC_API int osc_conv_prepack_f32(osc_ctx* ctx, const float* w, int M, int C, int kh, int kw, int host,
                                 osc_conv_weights** out) {
  if (out == nullptr) return fail(OSC_EINVAL, "osc_conv_prepack_f32: out is null");
  *out = nullptr;
  OSC_TRY(enter(ctx));
  if (w == nullptr || M <= 0 || C <= 0 || kh <= 0 || kw <= 0 || kh * kw > kMaxTaps)
    return fail(OSC_EINVAL, "osc_conv_prepack_f32: bad weight shape [%d,%d,%d,%d]", M, C, kh, kw);
  if (fault_injected("prepack")) return fail(OSC_EFAULT_INJECTED, "injected failure (prepack)");
  auto* cw = new osc_conv_weights();
  cw->device = ctx->device;
  cw->M = M;
  cw->C = C;
  cw->kh = kh;
  cw->kw = kw;
  cw->Cp = static_cast<int>(round_up(static_cast<size_t>(C), 32));
  cw->Kp = kh * kw * cw->Cp;
  const size_t n = static_cast<size_t>(M) * cw->Kp;
  const size_t src_bytes = static_cast<size_t>(M) * C * kh * kw * sizeof(float);
  float* staged = nullptr;
  cudaError_t e = cudaMalloc(&cw->hi, n * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&cw->lo, n * sizeof(float));
  if (e == cudaSuccess && host) {
    e = cudaMalloc(&staged, src_bytes);
    if (e == cudaSuccess) e = cudaMemcpyAsync(staged, w, src_bytes, cudaMemcpyHostToDevice, ctx->stream);
    w = staged;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    cudaFree(cw->hi);
    cudaFree(cw->lo);
    cudaFree(staged);
    delete cw;
    return fail(OSC_ENOMEM, "osc_conv_prepack_f32: %s", cudaGetErrorString(e));
  }
  const int blocks = static_cast<int>(std::min<size_t>((n + 255) / 256, static_cast<size_t>(ctx->num_sms) * 8));
  prof_begin(ctx);
  k_pack_conv_w<<<blocks, 256, 0, ctx->stream>>>(w, M, C, kh, kw, cw->Cp, cw->hi, cw->lo);
  int st = check_launch(ctx, "k_pack_conv_w");
  if (staged) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(staged);
  }
  if (st != OSC_OK) {
    cudaFree(cw->hi);
    cudaFree(cw->lo);
    delete cw;
    return st;
  }
  *out = cw;
  return OSC_OK;
}

OSC_API int osc_conv_weights_free(osc_conv_weights* w) {
  if (w == nullptr) return OSC_OK;
  cudaSetDevice(w->device);
  cudaDeviceSynchronize();
  cudaFree(w->hi);
  cudaFree(w->lo);
  delete w;
  return OSC_OK;
}

static int conv_entry(osc_ctx* ctx, const char* fn, const float* x, long long x_nstride, int N, int C, int H, int W,
                      const osc_conv_weights* w, int stride_h, int stride_w, int pad_t, int pad_l, int pad_b,
                      int pad_r, int dil_h, int dil_w, int group, const float* bias, int act, const float* res,
                      long long res_nstride, float* y, long long y_nstride, int OH, int OW) {
  OSC_TRY(enter(ctx));
  if (w == nullptr) return fail(OSC_EINVAL, "%s: null weights", fn);
  if (w->device != ctx->device) return fail(OSC_EINVAL, "%s: weights live on another device", fn);
  if (group != 1) return fail(OSC_EUNSUPPORTED, "%s: group=%d (use osc_conv2d_direct_f32)", fn, group);
  if (C != w->C) return fail(OSC_EINVAL, "%s: input has %d channels, weights %d", fn, C, w->C);
  if (N < 0 || H <= 0 || W <= 0 || stride_h <= 0 || stride_w <= 0 || dil_h <= 0 || dil_w <= 0 || pad_t < 0 ||
      pad_l < 0 || pad_b < 0 || pad_r < 0)
    return fail(OSC_EINVAL, "%s: bad geometry", fn);
  if (act < OSC_ACT_NONE || act > OSC_ACT_SIGMOID) return fail(OSC_EINVAL, "%s: act=%d", fn, act);
  // Output size as Ops/DnnOps.cs:53-66 (floor mode).
  const int eh = (w->kh - 1) * dil_h + 1, ew = (w->kw - 1) * dil_w + 1;
  const int oh = (H + pad_t + pad_b - eh) / stride_h + 1;
  const int ow = (W + pad_l + pad_r - ew) / stride_w + 1;
  if (oh != OH || ow != OW || oh <= 0 || ow <= 0)
    return fail(OSC_EINVAL, "%s: output must be %dx%d, got %dx%d", fn, oh, ow, OH, OW);
  const long long dense_x = static_cast<long long>(C) * H * W, dense_y = static_cast<long long>(w->M) * OH * OW;
  if (x_nstride == 0) x_nstride = dense_x;
  if (y_nstride == 0) y_nstride = dense_y;
  if (res_nstride == 0) res_nstride = dense_y;
  if (x_nstride < dense_x || y_nstride < dense_y || (res != nullptr && res_nstride < dense_y))
    return fail(OSC_EINVAL, "%s: image stride smaller than one image", fn);
  if (N == 0) return OSC_OK;
  if (x == nullptr || y == nullptr) return fail(OSC_EINVAL, "%s: null pointer", fn);
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  return conv_tf32x3(ctx, x, x_nstride, N, C, H, W, w, stride_h, stride_w, pad_t, pad_l, dil_h, dil_w, bias, act, res,
                     res_nstride, y, y_nstride, OH, OW);
}

OSC_API int osc_conv2d_bias_act_f32(osc_ctx* ctx, const float* x, int N, int C, int H, int W,
                                    const osc_conv_weights* w, int stride_h, int stride_w, int pad_t, int pad_l,
                                    int pad_b, int pad_r, int dil_h, int dil_w, int group, const float* bias, int act,
                                    float* y, int OH, int OW) {
  return conv_entry(ctx, "osc_conv2d_bias_act_f32", x, 0, N, C, H, W, w, stride_h, stride_w, pad_t, pad_l, pad_b,
                    pad_r, dil_h, dil_w, group, bias, act, nullptr, 0, y, 0, OH, OW);
}

OSC_API int osc_conv2d_ex_f32(osc_ctx* ctx, const float* x, long long x_nstride, int N, int C, int H, int W,
                              const osc_conv_weights* w, int stride_h, int stride_w, int pad_t, int pad_l, int pad_b,
                              int pad_r, int dil_h, int dil_w, const float* bias, int act, const float* residual,
                              long long res_nstride, float* y, long long y_nstride, int OH, int OW) {
  return conv_entry(ctx, "osc_conv2d_ex_f32", x, x_nstride, N, C, H, W, w, stride_h, stride_w, pad_t, pad_l, pad_b,
                    pad_r, dil_h, dil_w, 1, bias, act, residual, res_nstride, y, y_nstride, OH, OW);
}

}  // extern "C"
