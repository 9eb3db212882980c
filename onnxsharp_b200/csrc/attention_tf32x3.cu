// attention_tf32x3.cu — FusedAttention for sequence length <= 128 with the
// whole head resident on one SM: QK^T, softmax and .V never leave the chip.
//
// Replaces AttentionLayer.Forward (src/OnnxSharp/Ops/AttentionOps.cs:249-351)
// and its GEMM-blocked kernel ComputeBlocks (:464-690), heads form
// (Q/K/V [B, T, H*D], output [B, T, H*D] or [B, H, T, D]), optional additive
// mask [B, 1, 1|T, T].
//
// Persistent CTAs (one per SM) walk the (b, h) heads; the stages of
// consecutive heads overlap:
//   producer warp   TMA loads of Q, K (into buffers freed when the previous
//                   head's S = Q K^T has completed) and V (freed when its
//                   P V has completed); rows >= T are zero-filled.
//   converter warps the 3xTF32 low parts beside the landed tiles: the landed
//                   fp32 tile is its own high part (a tf32 operand is read as
//                   its top 19 bits, i.e. trunc(x)), lo = x - trunc(x) is
//                   exact. Q is first multiplied by `scale` with one
//                   rounding, as the reference does (q' = q * scale,
//                   AttentionOps.cs:531-537).
//   MMA warp        S = Q' K^T (kind::tf32, three products per 8-wide K
//                   step) into TMEM; O = P V with P read from TMEM (the
//                   A-from-tensor-memory form) and V read MN-major straight
//                   from its landed [keys][d] tile (no transpose), into one
//                   of two TMEM accumulators.
//   softmax warps   16 warps, 4 per TMEM lane quadrant x 4 blocks of 32 keys:
//                   each thread owns a query row's 32 keys: mask add, max,
//                   e = exp(s - max) with the reference's polynomial
//                   (VectorMath.Exp) and its 8-lane partial-sum order
//                   (VectorMath.SumExp, :355-384), 1/sum; the unnormalised e
//                   (split hi/lo) goes to TMEM as the A operand of P V (the
//                   reference's lazy softmax, :590-604); then the previous
//                   head's O is read from TMEM, scaled by its 1/sum
//                   (:636-643) and stored, while this head's P V runs.
// The reference sums S and O as FMA chains; the tensor cores sum in another
// order, so parity is a tolerance (the reference's attention golden uses
// max |d| < 1e-5, AttentionTests.cs:20-58).
#include <algorithm>

#include "runtime.h"
#include "sm100.cuh"
#include "vmath.cuh"

namespace osc {
namespace {

constexpr int kAT = 128;                       // padded sequence length (TMEM lanes)
constexpr int kNConv = 6;                      // converter warps: 4 for Q / K, 2 for V
constexpr int kNConvQK = 4;
constexpr int kNSoft = 16;                     // softmax warps: 4 per TMEM lane quadrant x 4 key blocks
constexpr int kAWarps = 2 + kNConv + kNSoft;   // + producer, MMA
constexpr int kAThreads = kAWarps * 32;
constexpr int kBox = kAT * 32 * 4;             // one [128 rows][32 fp32] box = 16 KB
constexpr int kPart = 2 * kBox;                // one operand part (raw or lo) at D = 64
constexpr int kXmax = 2 * 4 * kAT;             // [2 heads][4 key blocks][128 rows] partial maxima
constexpr int kXlanes = kAT * 8;               // [128 rows][8] running lane sums
constexpr int kXtail = kAT * 8;                // [128 rows][< 8] e of the keys past the last 8-key group
constexpr int kXpinv = 2 * kAT;                // [2 heads][128 rows] 1 / sum
constexpr int kXBytes = (kXmax + kXlanes + kXtail + kXpinv) * 4;
constexpr int kASmem = 1024 + 6 * kPart + kXBytes + 256;
static_assert(kASmem <= 232448, "attention shared memory budget");
// TMEM columns: S, P hi, P lo, two O accumulators
constexpr uint32_t kColS = 0, kColPh = 128, kColPl = 256, kColO = 384;

struct AttnBars {
  uint64_t qk_full, v_full, qk_ready, v_ready, s_full, s_free, p_ready, o_full, o_free[2], mma_done;
  uint32_t tmem_slot;
  int abort_flag;
};

struct AttnArgs {
  int B, T, H, D;
  float scale;
  const float* mask;  // [B, 1, mask_rows, T] or null
  int mask_rows;
  int out_head_space;
  float* out;
};

__device__ __forceinline__ float trunc_tf32(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }
// The low 3xTF32 parts x - trunc(x) (exact) of four values.
__device__ __forceinline__ float4 lo4(float4 x) {
  return make_float4(__fsub_rn(x.x, trunc_tf32(x.x)), __fsub_rn(x.y, trunc_tf32(x.y)), __fsub_rn(x.z, trunc_tf32(x.z)),
                     __fsub_rn(x.w, trunc_tf32(x.w)));
}

// Named barrier over the softmax warps that also ORs a predicate across them,
// so every softmax warp stops after the same head.
__device__ __forceinline__ bool soft_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 5, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(kNSoft * 32)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// Bounded wait that ignores the CTA's abort flag: used to let copies already
// in flight land (or MMAs retire) before the CTA exits.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* err) {
  int never = 0;
  mbar_wait(bar, parity, &never, err);
}

__global__ void __launch_bounds__(kAThreads, 1)
    k_attention_tf32x3(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mK,
                       const __grid_constant__ CUtensorMap mV, const __grid_constant__ AttnArgs args,
                       int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;                // Q' (scaled; its own hi part), then Q lo
  uint8_t* sql = smem + kPart;
  uint8_t* sk = smem + 2 * kPart;    // K, K lo
  uint8_t* skl = smem + 3 * kPart;
  uint8_t* sv = smem + 4 * kPart;    // V [keys][d] MN-major (128-byte rows, 32-byte swizzle atoms), V lo
  uint8_t* svl = smem + 5 * kPart;
  float* xmax = reinterpret_cast<float*>(smem + 6 * kPart);
  float* xlanes = xmax + kXmax;
  float* xtail = xlanes + kXlanes;
  float* xpinv = xtail + kXtail;
  AttnBars* bar = reinterpret_cast<AttnBars*>(xpinv + kXpinv);
  volatile int* abort_flag = &bar->abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = args.D, T = args.T, H = args.H;
  const int half = (D / 32) * kBox;  // bytes of one operand part
  const int nheads = args.B * H;

  if (threadIdx.x == 0) {
    mbar_init(&bar->qk_full, 1);
    mbar_init(&bar->v_full, 1);
    mbar_init(&bar->qk_ready, kNConvQK);
    mbar_init(&bar->v_ready, kNConv - kNConvQK);
    mbar_init(&bar->s_full, 1);
    mbar_init(&bar->s_free, kNSoft);
    mbar_init(&bar->p_ready, kNSoft);
    mbar_init(&bar->o_full, 1);
    mbar_init(&bar->o_free[0], kNSoft);
    mbar_init(&bar->o_free[1], kNSoft);
    mbar_init(&bar->mma_done, 1);
    bar->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&mQ);
    tma_prefetch(&mK);
    tma_prefetch(&mV);
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_slot;

  // Every barrier completes once per head: head `it` of this CTA waits on parity it & 1.
  if (warp == 0) {
    if (lane == 0) {
      // Two independent load streams: Q, K of head i once S of head i-1 has
      // completed (its buffers are free), V of head i once P V of head i-1
      // has. Neither waits behind the other.
      const int nh = (nheads - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                     static_cast<int>(gridDim.x);
      int nq = 0, nv = 0;
      long long idle_since = clock64();
      while (nq < nh || nv < nh) {
        bool progress = false;
        if (nq < nh && (nq == 0 || mbar_test_wait(&bar->s_full, (nq - 1) & 1))) {
          const int bh = blockIdx.x + nq * gridDim.x, b = bh / H, h = bh % H;
          mbar_arrive_expect_tx(&bar->qk_full, 2 * half);
          for (int i = 0; i < D / 32; ++i) {
            tma_load_3d(sq + i * kBox, &mQ, &bar->qk_full, h * D + 32 * i, 0, b);
            tma_load_3d(sk + i * kBox, &mK, &bar->qk_full, h * D + 32 * i, 0, b);
          }
          ++nq;
          progress = true;
        }
        if (nv < nh && (nv == 0 || mbar_test_wait(&bar->o_full, (nv - 1) & 1))) {
          const int bh = blockIdx.x + nv * gridDim.x, b = bh / H, h = bh % H;
          mbar_arrive_expect_tx(&bar->v_full, half);
          for (int i = 0; i < D / 32; ++i) tma_load_3d(sv + i * kBox, &mV, &bar->v_full, h * D + 32 * i, 0, b);
          ++nv;
          progress = true;
        }
        if (progress) {
          idle_since = clock64();
        } else if (*abort_flag) {
          break;
        } else if (clock64() - idle_since > kWaitLimitCycles) {  // bounded like every other wait
          *abort_flag = 1;
          atomicExch(err, DEV_ERR_TIMEOUT);
          break;
        }
      }
      // no copy may land after the CTA has exited
      if (nq > 0) drain_wait(&bar->qk_full, (nq - 1) & 1, err);
      if (nv > 0) drain_wait(&bar->v_full, (nv - 1) & 1, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_tf32(kAT, kAT);
      const uint32_t idO = idesc_tf32_bmn(kAT, D);
      const uint32_t q0 = smem_addr(sq), ql0 = smem_addr(sql), k0 = smem_addr(sk), kl0 = smem_addr(skl);
      const uint32_t v0 = smem_addr(sv), vl0 = smem_addr(svl);
      // Two issue streams, each in head order: S of head i once Q, K are split
      // and S of head i-1 has been read out of TMEM; P V of head i once P and
      // V are ready and its O accumulator is drained. Whichever is ready is
      // issued first, so the next head's Q K^T runs while this head's softmax
      // is computed.
      const int nh = (nheads - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                     static_cast<int>(gridDim.x);
      int ns = 0, np = 0;
      long long idle_since = clock64();
      while (np < nh) {
        bool progress = false;
        if (ns < nh && mbar_test_wait(&bar->qk_ready, ns & 1) &&
            (ns == 0 || mbar_test_wait(&bar->s_free, (ns - 1) & 1))) {
          // S = Q' K^T : M = 128 queries, N = 128 keys, K = D
          tc_fence_after();
          for (int ks = 0; ks < D / 8; ++ks) {
            const uint32_t off = (ks / 4) * kBox + (ks % 4) * 32;
            const uint64_t qh = sdesc_kmajor_sw128(q0 + off), ql = sdesc_kmajor_sw128(ql0 + off);
            const uint64_t kh = sdesc_kmajor_sw128(k0 + off), kl = sdesc_kmajor_sw128(kl0 + off);
            mma_tf32(tmem + kColS, qh, kh, idS, ks > 0 ? 1u : 0u);
            mma_tf32(tmem + kColS, qh, kl, idS, 1u);
            mma_tf32(tmem + kColS, ql, kh, idS, 1u);
          }
          mma_commit(&bar->s_full);
          ++ns;
          progress = true;
        }
        if (np < ns && mbar_test_wait(&bar->p_ready, np & 1) && mbar_test_wait(&bar->v_ready, np & 1) &&
            (np < 2 || mbar_test_wait(&bar->o_free[np & 1], ((np >> 1) - 1) & 1))) {
          // O = P V : M = 128 queries, N = D, K = 128 keys; P from TMEM, V MN-major
          tc_fence_after();
          const uint32_t tO = tmem + kColO + 64u * static_cast<uint32_t>(np & 1);
          for (int ks = 0; ks < kAT / 8; ++ks) {
            const uint64_t vh = sdesc_mnmajor_sw128_32b(v0 + ks * 1024, kBox, 512);
            const uint64_t vl = sdesc_mnmajor_sw128_32b(vl0 + ks * 1024, kBox, 512);
            const uint32_t ph = tmem + kColPh + 8u * ks, pl = tmem + kColPl + 8u * ks;
            mma_tf32_ts(tO, ph, vh, idO, ks > 0 ? 1u : 0u);
            mma_tf32_ts(tO, ph, vl, idO, 1u);
            mma_tf32_ts(tO, pl, vh, idO, 1u);
          }
          mma_commit(&bar->o_full);
          ++np;
          progress = true;
        }
        if (progress) {
          idle_since = clock64();
        } else if (*abort_flag) {
          break;
        } else if (clock64() - idle_since > kWaitLimitCycles) {  // bounded like every other wait
          *abort_flag = 1;
          atomicExch(err, DEV_ERR_TIMEOUT);
          break;
        }
      }
      // every MMA issued has retired before TMEM is released
      mma_commit(&bar->mma_done);
      drain_wait(&bar->mma_done, 0, err);
    }
  } else if (warp < 2 + kNConvQK) {
    // Q, K low parts (Q scaled first)
    const int ctid = threadIdx.x - 64;
    const int n4 = half / 16;
    int it = 0;
    for (int bh = blockIdx.x; bh < nheads; bh += gridDim.x, ++it) {
      const bool ok = mbar_wait(&bar->qk_full, it & 1, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) break;
      // four float4 of Q and four of K in flight per thread
      for (int i0 = ctid; i0 < n4; i0 += 4 * kNConvQK * 32) {
        float4 q[4], k[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = i0 + u * kNConvQK * 32;
          if (i < n4) {
            q[u] = reinterpret_cast<const float4*>(sq)[i];
            k[u] = reinterpret_cast<const float4*>(sk)[i];
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = i0 + u * kNConvQK * 32;
          if (i < n4) {
            const float4 x = make_float4(__fmul_rn(q[u].x, args.scale), __fmul_rn(q[u].y, args.scale),
                                         __fmul_rn(q[u].z, args.scale), __fmul_rn(q[u].w, args.scale));
            reinterpret_cast<float4*>(sq)[i] = x;
            reinterpret_cast<float4*>(sql)[i] = lo4(x);
            reinterpret_cast<float4*>(skl)[i] = lo4(k[u]);
          }
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->qk_ready);
    }
  } else if (warp < 2 + kNConv) {
    // V low part
    const int ctid = threadIdx.x - 64 - kNConvQK * 32;
    const int n4 = half / 16;
    int it = 0;
    for (int bh = blockIdx.x; bh < nheads; bh += gridDim.x, ++it) {
      const bool ok = mbar_wait(&bar->v_full, it & 1, abort_flag, err);
      if (!__all_sync(0xffffffffu, ok)) break;
      constexpr int kVT = (kNConv - kNConvQK) * 32;
      for (int i0 = ctid; i0 < n4; i0 += 8 * kVT) {  // eight float4 in flight per thread
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (i0 + u * kVT < n4) v[u] = reinterpret_cast<const float4*>(sv)[i0 + u * kVT];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (i0 + u * kVT < n4) reinterpret_cast<float4*>(svl)[i0 + u * kVT] = lo4(v[u]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->v_ready);
    }
  } else {
    const int sid = warp - 2 - kNConv;  // 0..15
    const int q4 = warp & 3;            // TMEM lane quadrant this warp may access
    const int part = sid >> 2;          // key block [32*part, 32*part + 32) of the row
    const int row = q4 * 32 + lane;     // query row == TMEM lane
    const uint32_t lanebase = static_cast<uint32_t>(q4 * 32) << 16;
    const int j0 = part * 32;
    const int tv = T & ~7;              // vector part of VectorMath.SumExp
    const int dq = D / 4;               // output columns of this thread's row
    auto csync = [] { asm volatile("bar.sync 1, %0;" ::"n"(kNSoft * 32) : "memory"); };
    // The previous head's O: read from TMEM, times 1/sum, stored.
    auto epilogue = [&](int it_done, int pbh) {
      tc_fence_after();
      const int ob = it_done & 1;
      const float pinv = xpinv[ob * kAT + row];
      const uint32_t base = tmem + kColO + 64u * ob + lanebase + static_cast<uint32_t>(part * dq);
      const int b = pbh / H, h = pbh % H;
      float* dst = args.out_head_space ? args.out + ((static_cast<size_t>(pbh) * T + row) * D + part * dq)
                                       : args.out + ((static_cast<size_t>(b) * T + row) * (H * D) + h * D + part * dq);
      for (int g = 0; g < dq; g += 8) {
        uint32_t r[8];
        tmem_ld8(base + g, r);
        tmem_wait_ld();
        if (row < T) {
          reinterpret_cast<float4*>(dst + g)[0] =
              make_float4(__fmul_rn(__uint_as_float(r[0]), pinv), __fmul_rn(__uint_as_float(r[1]), pinv),
                          __fmul_rn(__uint_as_float(r[2]), pinv), __fmul_rn(__uint_as_float(r[3]), pinv));
          reinterpret_cast<float4*>(dst + g)[1] =
              make_float4(__fmul_rn(__uint_as_float(r[4]), pinv), __fmul_rn(__uint_as_float(r[5]), pinv),
                          __fmul_rn(__uint_as_float(r[6]), pinv), __fmul_rn(__uint_as_float(r[7]), pinv));
        }
      }
      tc_fence_before();
      __syncwarp();
    };
    bool ok = true;
    int it = 0, prev = -1;
    for (int bh = blockIdx.x; bh < nheads; bh += gridDim.x, ++it) {
      const int b = bh / H;
      float s[32];
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar->s_full, it & 1, abort_flag, err));
      if (ok) {
        tc_fence_after();
        uint32_t r[32];
        tmem_ld32(tmem + kColS + lanebase + static_cast<uint32_t>(j0), r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) s[j] = __uint_as_float(r[j]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->s_free);  // S may be overwritten by the next head's Q K^T
        if (args.mask != nullptr && row < T) {
          const float* mr =
              args.mask + (static_cast<size_t>(b) * args.mask_rows + (args.mask_rows == 1 ? 0 : row)) * T;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j0 + j < T) s[j] = __fadd_rn(s[j], __ldg(mr + j0 + j));
        }
        float mx = -INFINITY;
        if (j0 + 32 <= T) {
#pragma unroll
          for (int j = 0; j < 32; ++j) mx = fmaxf(mx, s[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j0 + j < T) mx = fmaxf(mx, s[j]);
        }
        xmax[(it & 1) * 4 * kAT + part * kAT + row] = mx;
      }
      csync();
      if (ok) {
        const float* xm = xmax + (it & 1) * 4 * kAT;
        const float mx = fmaxf(fmaxf(xm[row], xm[kAT + row]), fmaxf(xm[2 * kAT + row], xm[3 * kAT + row]));
        if (j0 + 32 <= tv) {  // the whole key block in the vector part: no per-key branches
#pragma unroll
          for (int j = 0; j < 32; ++j) s[j] = ref_exp(__fsub_rn(s[j], mx));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int jj = j0 + j;
            if (jj < tv) s[j] = ref_exp(__fsub_rn(s[j], mx));
            else if (jj < T) s[j] = expf(__fsub_rn(s[j], mx));  // scalar tail: MathF.Exp
            else s[j] = 0.0f;
            if (jj >= tv && jj < T) xtail[row * 8 + (jj - tv)] = s[j];
          }
        }
      }
      // The row sum in the reference's order: 8 lane sums running over the keys
      // in sequence (key block 0, then 1, 2, 3), then the lanes in order, then the
      // scalar tail. The running sums pass from block to block through shared
      // memory (named barriers 2..4 pair consecutive blocks).
      {
        float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (part > 0) {
          asm volatile("bar.sync %0, %1;" ::"r"(1 + part), "n"(2 * 4 * 32) : "memory");
#pragma unroll
          for (int l = 0; l < 8; ++l) lanes[l] = xlanes[row * 8 + l];
        }
        if (ok && j0 + 32 <= tv) {
#pragma unroll
          for (int j = 0; j < 32; ++j) lanes[j & 7] = __fadd_rn(lanes[j & 7], s[j]);
        } else if (ok) {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j0 + j < tv) lanes[j & 7] = __fadd_rn(lanes[j & 7], s[j]);
        }
        if (part < 3) {
#pragma unroll
          for (int l = 0; l < 8; ++l) xlanes[row * 8 + l] = lanes[l];
          asm volatile("bar.arrive %0, %1;" ::"r"(2 + part), "n"(2 * 4 * 32) : "memory");
        } else {
          float total = 0.0f;
#pragma unroll
          for (int l = 0; l < 8; ++l) total = __fadd_rn(total, lanes[l]);
          for (int j = tv; j < T; ++j) total = __fadd_rn(total, xtail[row * 8 + (j - tv)]);
          xpinv[(it & 1) * kAT + row] = __fdiv_rn(1.0f, total);
        }
      }
      // P (this head) may replace P (previous head) once that head's P V is done
      if (ok && it > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bar->o_full, (it - 1) & 1, abort_flag, err));
      if (ok) {
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          hi[j] = __float_as_uint(s[j]);
          lo[j] = __float_as_uint(__fsub_rn(s[j], trunc_tf32(s[j])));
        }
        tmem_st32(tmem + kColPh + lanebase + static_cast<uint32_t>(j0), hi);
        tmem_st32(tmem + kColPl + lanebase + static_cast<uint32_t>(j0), lo);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->p_ready);
      }
      if (ok && it > 0) {
        epilogue(it - 1, prev);
        if (lane == 0) mbar_arrive(&bar->o_free[(it - 1) & 1]);
      }
      prev = bh;
      if (soft_any(!ok || *abort_flag)) {
        ok = false;
        break;
      }
    }
    if (ok && it > 0) {
      if (__all_sync(0xffffffffu, mbar_wait(&bar->o_full, (it - 1) & 1, abort_flag, err))) epilogue(it - 1, prev);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace
}  // namespace osc

using namespace osc;

extern "C" {

OSC_API int osc_attention_f32(osc_ctx* ctx, const float* q, const float* k, const float* v, const float* mask,
                              int mask_rows, int B, int T, int H, int D, float scale, int out_head_space,
                              float* out) {
  OSC_TRY(enter(ctx));
  if (B < 0 || T <= 0 || H <= 0 || D <= 0) return fail(OSC_EINVAL, "osc_attention_f32: bad shape");
  if (mask != nullptr && mask_rows != 1 && mask_rows != T)
    return fail(OSC_EINVAL, "osc_attention_f32: mask rows %d (1 or T)", mask_rows);
  if (B == 0) return OSC_OK;
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(OSC_EINVAL, "osc_attention_f32: null pointer");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  // one head resident per SM for T <= 128 and D in {32, 64}; otherwise the composed path
  if (T > kAT || (D != 32 && D != 64) || (reinterpret_cast<uintptr_t>(out) & 15u) != 0)
    return attention_composed(ctx, q, k, v, mask, mask_rows, B, T, H, D, scale, out_head_space, out);
  const int width = H * D;
  CUtensorMap mQ, mK, mV;
  const uint64_t dims[3] = {static_cast<uint64_t>(width), static_cast<uint64_t>(T), static_cast<uint64_t>(B)};
  const uint64_t pitch[2] = {static_cast<uint64_t>(width) * 4, static_cast<uint64_t>(width) * 4 * T};
  const uint32_t box[3] = {32, static_cast<uint32_t>(kAT), 1};
  OSC_TRY(encode_tiled(&mQ, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, q, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mK, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, k, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  // V lands MN-major for P V: [keys][32 d] rows of 128 bytes, 32-byte swizzle atoms
  OSC_TRY(encode_tiled(&mV, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, v, dims, pitch, box,
                       CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
  AttnArgs a{};
  a.B = B;
  a.T = T;
  a.H = H;
  a.D = D;
  a.scale = scale;
  a.mask = mask;
  a.mask_rows = mask_rows;
  a.out_head_space = out_head_space;
  a.out = out;
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_attention_tf32x3), kASmem));
  prof_begin(ctx);
  const int grid = std::min(B * H, ctx->num_sms);  // persistent: each CTA walks heads blockIdx.x + i * grid
  k_attention_tf32x3<<<grid, kAThreads, kASmem, ctx->stream>>>(mQ, mK, mV, a, ctx->d_err);
  return check_launch(ctx, "k_attention_tf32x3");
}

}  // extern "C"
