// attention_tf32x3.cu — FusedAttention for sequence length <= 128 with the
// whole head resident on one SM: QK^T, softmax and .V never leave the chip.
//
// Replaces AttentionLayer.Forward (src/OnnxSharp/Ops/AttentionOps.cs:249-351)
// and its GEMM-blocked kernel ComputeBlocks (:464-690), heads form
// (Q/K/V [B, T, H*D], output [B, T, H*D] or [B, H, T, D]), optional additive
// mask [B, 1, 1|T, T].
//
// Per CTA (one (b, h)):
//   1. TMA loads the raw Q, K, V tiles ([128 rows][32 fp32] SW128 boxes; rows
//      >= T are zero-filled).
//   2. Four compute warps split them in place into 3xTF32 hi/lo parts; Q is
//      first multiplied by `scale` with one rounding, as the reference does
//      (q' = q * scale, AttentionOps.cs:531-537).
//   3. S = Q' K^T on tcgen05 (kind::tf32, 3 products per 8-wide K step) into TMEM.
//   4. Each compute thread owns one query row: mask add, max, e = exp(s - max)
//      with the reference's polynomial (VectorMath.Exp) and its 8-lane
//      partial-sum order (VectorMath.SumExp, :355-384), pinv = 1/sum; the
//      unnormalised e goes back to shared memory (split hi/lo) as the A
//      operand of the second GEMM (the reference's lazy softmax, :590-604).
//   5. O = e V on tcgen05 (V transposed to a K-major [D][keys] hi/lo tile by
//      the compute warps during its split), O *= pinv (:636-643), then
//      coalesced stores through a shared-memory staging tile.
// The reference sums S and O as FMA chains; the tensor cores sum in another
// order, so parity is a tolerance (the reference's attention golden uses
// max |d| < 1e-5, AttentionTests.cs:20-58).
#include <algorithm>

#include "runtime.h"
#include "sm100.cuh"
#include "vmath.cuh"

namespace osc {
namespace {

constexpr int kAT = 128;                   // padded sequence length (TMEM lanes)
constexpr int kACW = 16;                   // compute warps: 4 per TMEM lane quadrant, 32 keys each
constexpr int kAThreads = (2 + kACW) * 32; // warp 0 TMA, warp 1 MMA/TMEM, warps 2-17 compute
constexpr int kBox = kAT * 32 * 4;         // one [128][32] fp32 SW128 box = 16 KB
constexpr int kRegion = 4 * kBox;          // hi (2 boxes) + lo (2 boxes) for D = 64
constexpr int kVRaw = 2 * kBox;            // raw V as loaded: [128 keys][64 d] in two boxes
constexpr int kVt = 2 * 4 * 64 * 128;      // V^T hi | lo: 4 key-blocks of [64 d][32 keys]
// Softmax exchange (row maxima of the 4 key blocks, running lane sums, 1/sum):
// kept in the tail of the raw-V region, free once V^T is split and dead
// before the output staging reuses it.
constexpr int kAXchg = 4 * kAT * 4 + kAT * 8 * 4 + kAT * 4;
constexpr int kASmem = 2 * kRegion + kVRaw + kVt + 1024 + 256;
static_assert(kASmem <= 232448, "attention shared memory budget");

struct AttnBarriers {
  uint64_t full_qk, full_v, qk_split, v_split, s_full, p_ready, o_full;
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

// Splits `n4` float4s at p in place into hi (at p) and lo (at p + lo_off floats),
// optionally scaling first.
__device__ __forceinline__ void split_inplace(float* p, int lo_off, int n4, float scale, bool do_scale, int tid,
                                              int nthreads) {
  for (int i = tid; i < n4; i += nthreads) {
    float4 v = reinterpret_cast<float4*>(p)[i];
    float e[4] = {v.x, v.y, v.z, v.w};
    float h[4], l[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float x = do_scale ? __fmul_rn(e[q], scale) : e[q];
      h[q] = to_tf32(x);
      l[q] = __fsub_rn(x, h[q]);
    }
    reinterpret_cast<float4*>(p)[i] = make_float4(h[0], h[1], h[2], h[3]);
    reinterpret_cast<float4*>(p + lo_off)[i] = make_float4(l[0], l[1], l[2], l[3]);
  }
}

__global__ void __launch_bounds__(kAThreads, 1)
    k_attention_tf32x3(const __grid_constant__ CUtensorMap mQ, const __grid_constant__ CUtensorMap mK,
                       const __grid_constant__ CUtensorMap mV, const __grid_constant__ AttnArgs args,
                       int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* rq = smem;                 // Q hi | Q lo   (later P hi)
  uint8_t* rk = smem + kRegion;       // K hi | K lo   (later P lo)
  uint8_t* rv = smem + 2 * kRegion;   // raw V [keys][d] (later the output staging tile)
  uint8_t* rvt = rv + kVRaw;          // V^T hi | lo, K-major over keys
  float* xmax = reinterpret_cast<float*>(rv + kVRaw - kAXchg);  // [4 key blocks][128 rows] partial maxima
  float* xlanes = xmax + 4 * kAT;                                // [128 rows][8] running lane sums
  float* xpinv = xlanes + kAT * 8;                               // [128 rows] 1 / sum
  AttnBarriers* bar = reinterpret_cast<AttnBarriers*>(rvt + kVt);
  volatile int* abort_flag = &bar->abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int b = bh / args.H, h = bh % args.H;
  const int D = args.D, T = args.T;
  const int dboxes = D / 32;
  const int half_bytes = dboxes * kBox;  // bytes of one hi (or lo) operand part

  if (threadIdx.x == 0) {
    mbar_init(&bar->full_qk, 1);
    mbar_init(&bar->full_v, 1);
    mbar_init(&bar->qk_split, kACW);
    mbar_init(&bar->v_split, kACW);
    mbar_init(&bar->s_full, 1);
    mbar_init(&bar->p_ready, kACW);
    mbar_init(&bar->o_full, 1);
    bar->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch(&mQ);
    tma_prefetch(&mK);
    tma_prefetch(&mV);
  }
  if (warp == 1) {
    tmem_alloc(&bar->tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&bar->full_qk, 2 * half_bytes);
      for (int i = 0; i < dboxes; ++i) {
        tma_load_3d(rq + i * kBox, &mQ, &bar->full_qk, h * D + 32 * i, 0, b);
        tma_load_3d(rk + i * kBox, &mK, &bar->full_qk, h * D + 32 * i, 0, b);
      }
      mbar_arrive_expect_tx(&bar->full_v, half_bytes);
      for (int i = 0; i < dboxes; ++i) tma_load_3d(rv + i * kBox, &mV, &bar->full_v, h * D + 32 * i, 0, b);
      // The compute warps consume both loads before the CTA can finish; on
      // an abort, wait (bounded) for the copies to land before exiting.
      mbar_wait(&bar->full_qk, 0, abort_flag, err);
      mbar_wait(&bar->full_v, 0, abort_flag, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // S = Q' K^T : M = 128 queries, N = 128 keys, K = D.
      bool ok = mbar_wait(&bar->qk_split, 0, abort_flag, err);
      if (ok) {
        tc_fence_after();
        constexpr uint32_t idS = idesc_tf32(128, 128);
        const uint32_t q0 = smem_addr(rq), k0 = smem_addr(rk);
        for (int ks = 0; ks < D / 8; ++ks) {
          const uint32_t off = (ks / 4) * kBox + (ks % 4) * 32;
          const uint64_t qh = sdesc_kmajor_sw128(q0 + off), ql = sdesc_kmajor_sw128(q0 + half_bytes + off);
          const uint64_t kh = sdesc_kmajor_sw128(k0 + off), kl = sdesc_kmajor_sw128(k0 + half_bytes + off);
          mma_tf32(tS, qh, kh, idS, ks > 0 ? 1u : 0u);
          mma_tf32(tS, qh, kl, idS, 1u);
          mma_tf32(tS, ql, kh, idS, 1u);
        }
        mma_commit(&bar->s_full);
        // O = P V : M = 128 queries, N = D, K = 128 keys; V is MN-major.
        ok = mbar_wait(&bar->v_split, 0, abort_flag, err) && mbar_wait(&bar->p_ready, 0, abort_flag, err);
        if (ok) {
          tc_fence_after();
          const uint32_t idO = idesc_tf32(128, D);
          const uint32_t p0 = smem_addr(rq), v0 = smem_addr(rvt);
          constexpr int kPHalf = 4 * kBox;  // P hi / lo: 4 boxes of 32 keys
          const int vblk = D * 128;         // one [D rows][32 keys] block of V^T
          for (int ks = 0; ks < kAT / 8; ++ks) {
            const uint32_t offp = (ks / 4) * kBox + (ks % 4) * 32;
            const uint64_t ph = sdesc_kmajor_sw128(p0 + offp), pl = sdesc_kmajor_sw128(p0 + kPHalf + offp);
            const uint32_t offv = (ks / 4) * vblk + (ks % 4) * 32;
            const uint64_t vh = sdesc_kmajor_sw128(v0 + offv), vl = sdesc_kmajor_sw128(v0 + 4 * vblk + offv);
            mma_tf32(tO, ph, vh, idO, ks > 0 ? 1u : 0u);
            mma_tf32(tO, ph, vl, idO, 1u);
            mma_tf32(tO, pl, vh, idO, 1u);
          }
        }
      }
      mma_commit(&bar->o_full);
    }
  } else {
    const int ctid = threadIdx.x - 64;  // 0..511
    const int q4 = warp & 3;            // TMEM lane quadrant this warp may read
    const int part = (warp - 2) >> 2;   // key block [32*part, 32*part + 32) of the row
    const int row = q4 * 32 + lane;     // query row == TMEM lane
    constexpr int kCT = kACW * 32;
    // named barrier 1: all compute warps
    auto csync = [] { asm volatile("bar.sync 1, %0;" ::"n"(kACW * 32) : "memory"); };
    // 2. split Q (scaled) and K, then V.
    bool ok = mbar_wait(&bar->full_qk, 0, abort_flag, err);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      split_inplace(reinterpret_cast<float*>(rq), half_bytes / 4, half_bytes / 16, args.scale, true, ctid, kCT);
      split_inplace(reinterpret_cast<float*>(rk), half_bytes / 4, half_bytes / 16, 1.0f, false, ctid, kCT);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->qk_split);
      ok = mbar_wait(&bar->full_v, 0, abort_flag, err);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      // V^T split: thread (key, quarter) reads D/4 values of its key from the
      // swizzled raw rows and scatters hi/lo into the K-major V^T blocks (a
      // warp's 32 keys fill one 128-byte row of a block: no bank conflicts).
      const int key = ctid & 127, dq = ctid >> 7;
      const int kb = key >> 5, kc = key & 31;
      const int vblk = D * 128;
      const float* raw = reinterpret_cast<const float*>(rv);
      float* vth = reinterpret_cast<float*>(rvt + kb * vblk);
      float* vtl = reinterpret_cast<float*>(rvt + 4 * vblk + kb * vblk);
      for (int d = dq * (D / 4); d < (dq + 1) * (D / 4); ++d) {
        const int box = d >> 5, dc = d & 31;
        const float x = raw[(box * kBox + key * 128 + (((dc >> 2) ^ (key & 7)) << 4)) / 4 + (dc & 3)];
        const float hh = to_tf32(x);
        const int o = (d * 128 + ((((kc >> 2) ^ (d & 7)) << 4))) / 4 + (kc & 3);
        vth[o] = hh;
        vtl[o] = __fsub_rn(x, hh);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->v_split);
    }
    // every compute warp takes the same barriers below, whatever `ok` says
    csync();  // raw V is no longer read: its tail holds the softmax exchange
    if (ok) {
      ok = mbar_wait(&bar->s_full, 0, abort_flag, err);
      ok = __all_sync(0xffffffffu, ok);
    }
    float s[32];
    const int j0 = part * 32;
    if (ok) {
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(tS + (static_cast<uint32_t>(q4 * 32) << 16) + static_cast<uint32_t>(j0), r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) s[j] = __uint_as_float(r[j]);
      // 4. softmax of this row (keys >= T do not exist)
      if (args.mask != nullptr && row < T) {
        const float* mr = args.mask + (static_cast<size_t>(b) * args.mask_rows + (args.mask_rows == 1 ? 0 : row)) * T;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j0 + j < T) s[j] = __fadd_rn(s[j], __ldg(mr + j0 + j));
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j0 + j < T) mx = fmaxf(mx, s[j]);
      xmax[part * kAT + row] = mx;
    }
    csync();
    const int tv = T & ~7;  // vector part of VectorMath.SumExp
    if (ok) {
      const float mx = fmaxf(fmaxf(xmax[row], xmax[kAT + row]), fmaxf(xmax[2 * kAT + row], xmax[3 * kAT + row]));
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int jj = j0 + j;
        if (jj < tv) s[j] = ref_exp(__fsub_rn(s[j], mx));
        else if (jj < T) s[j] = expf(__fsub_rn(s[j], mx));  // scalar tail: MathF.Exp
        else s[j] = 0.0f;
      }
      // e (unnormalised) -> P hi (over Q) / lo (over K): box `part` of 32 keys
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float hh[4], ll[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          hh[q] = to_tf32(s[c * 4 + q]);
          ll[q] = __fsub_rn(s[c * 4 + q], hh[q]);
        }
        const int off = part * kBox + row * 128 + ((c ^ (row & 7)) << 4);
        *reinterpret_cast<float4*>(rq + off) = make_float4(hh[0], hh[1], hh[2], hh[3]);
        *reinterpret_cast<float4*>(rk + off) = make_float4(ll[0], ll[1], ll[2], ll[3]);
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar->p_ready);
    }
    // The row sum in the reference's order: 8 lane sums running over the
    // keys in sequence (key block 0, then 1, 2, 3), then the lanes in order,
    // then the scalar tail. The running sums pass from block to block through
    // shared memory (named barriers 2..4 pair consecutive blocks).
    {
      float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (part > 0) {
        asm volatile("bar.sync %0, %1;" ::"r"(1 + part), "n"(2 * 4 * 32) : "memory");
#pragma unroll
        for (int l = 0; l < 8; ++l) lanes[l] = xlanes[row * 8 + l];
      }
      if (ok) {
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
        for (int j = tv; j < T; ++j) {  // the scalar tail, in key order (its e values live in other blocks)
          const int pb = j >> 5, c = (j & 31) >> 2, qq = j & 3;
          const int off = pb * kBox + row * 128 + ((c ^ (row & 7)) << 4) + qq * 4;
          total = __fadd_rn(total, __fadd_rn(*reinterpret_cast<const float*>(rq + off),
                                             *reinterpret_cast<const float*>(rk + off)));
        }
        xpinv[row] = __fdiv_rn(1.0f, total);
      }
    }
    if (ok) {
      ok = mbar_wait(&bar->o_full, 0, abort_flag, err);
      ok = __all_sync(0xffffffffu, ok);
    }
    csync();  // 1/sum of every row is in shared memory; O is complete
    const float pinv = xpinv[row];
    const bool all_ok = !*abort_flag;
    csync();  // the exchange area is dead: the staging below overwrites it
    // 5. O row -> * (1/sum) -> staging (over raw V and V^T; the O MMA is complete) -> global
    float* stage = reinterpret_cast<float*>(rv);
    const int pitch = D + 4;
    if (ok && all_ok) {
      tc_fence_after();
      const int dq = D / 4;  // this warp's output columns [part*dq, part*dq + dq)
      const uint32_t base = tO + (static_cast<uint32_t>(q4 * 32) << 16) + static_cast<uint32_t>(part * dq);
      for (int g = 0; g < dq; g += 8) {
        uint32_t r[8];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
            : "r"(base + g));
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; j += 4)
          *reinterpret_cast<float4*>(stage + row * pitch + part * dq + g + j) =
              make_float4(__fmul_rn(__uint_as_float(r[j]), pinv), __fmul_rn(__uint_as_float(r[j + 1]), pinv),
                          __fmul_rn(__uint_as_float(r[j + 2]), pinv), __fmul_rn(__uint_as_float(r[j + 3]), pinv));
      }
    }
    csync();
    if (ok && all_ok) {
      // rows of D floats = D/4 float4 (16 lanes for D = 64): 2 rows per warp instruction
      const int per_row = D / 4;
      const int rows_per_iter = 32 / per_row;
      for (int r0 = (warp - 2) * rows_per_iter; r0 < T; r0 += kACW * rows_per_iter) {
        const int r = r0 + lane / per_row;
        const int c = (lane % per_row) * 4;
        if (r < T) {
          float* dst = args.out_head_space
                           ? args.out + ((static_cast<size_t>(bh) * T + r) * D + c)
                           : args.out + ((static_cast<size_t>(b) * T + r) * (args.H * D) + h * D + c);
          *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(stage + r * pitch + c);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
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
  if (T > kAT || (D != 32 && D != 64))
    return attention_composed(ctx, q, k, v, mask, mask_rows, B, T, H, D, scale, out_head_space, out);
  const int width = H * D;
  CUtensorMap mQ, mK, mV;
  const uint64_t dims[3] = {static_cast<uint64_t>(width), static_cast<uint64_t>(T), static_cast<uint64_t>(B)};
  const uint64_t pitch[2] = {static_cast<uint64_t>(width) * 4, static_cast<uint64_t>(width) * 4 * T};
  const uint32_t box[3] = {32, static_cast<uint32_t>(kAT), 1};
  OSC_TRY(encode_tiled(&mQ, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, q, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mK, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, k, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mV, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, v, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B));
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
  k_attention_tf32x3<<<B * H, kAThreads, kASmem, ctx->stream>>>(mQ, mK, mV, a, ctx->d_err);
  return check_launch(ctx, "k_attention_tf32x3");
}

}  // extern "C"
