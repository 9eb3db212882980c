// gemm_tf32x3.cu — FP32 MatMul(+FusedBias, +activation) on the sm_100a tensor
// cores with the 3xTF32 split.
//
// Replaces GemmKernel.MultiplyPacked (src/OnnxSharp/Tensors/GemmKernel.cs:675-852)
// behind MatMulLayer with FusedBias (src/OnnxSharp/Ops/DnnOps.cs:2789-3102).
// The reference accumulates each C element as one FMA chain from bias[j]
// (GemmKernel.cs:1156-1208); on the tensor cores the summation order differs,
// so parity is the reference's own tolerance |d|/max(1,|ref|) <= 1e-4
// (tests/OnnxSharp.Tests/GemmKernelTests.cs:116-120).
//
// Numerics: every FP32 operand x is split into hi = tf32(x) and lo = x - hi
// (exact in FP32); C += Ahi*Bhi + Ahi*Blo + Alo*Bhi with FP32 accumulation in
// TMEM. The dropped Alo*Blo term is ~2^-22 relative.
//
// Kernel shape: one 128 x BN output tile per CTA, BK = 32 (one 128-byte
// swizzle row per operand row). Warp 0 issues TMA loads of the four operand
// tiles (A hi/lo, B hi/lo) into a STAGES-deep shared-memory ring; warp 1
// allocates TMEM and issues tcgen05.mma (3 per 8-wide K step) from one
// thread, releasing each stage with tcgen05.commit; warps 2-5 read the
// accumulator back from TMEM and apply bias + activation.
#include <cstdlib>
#include <mutex>

#include "runtime.h"
#include "sm100.cuh"
#include "tf32x3_core.cuh"
#include "vmath.cuh"
#include <algorithm>

struct osc_gemm_weights {
  int device = 0;
  int k = 0, n = 0, kp = 0;  // kp: K padded to a multiple of 4 (16-byte TMA row pitch)
  float* hi = nullptr;       // [n][kp] tf32(B^T)
  float* lo = nullptr;       // [n][kp] B^T - hi
};

namespace osc {
namespace {

// Staging of one 128-row CTA tile for the batched kernel's epilogue (epilogue
// warps): the drained accumulator goes to the (free) operand ring at a pitch
// of BN+4 floats and the tile's column bias next to it.
template <class Cfg>
__device__ __forceinline__ void gemm_stage(uint8_t* tiles, const float (&acc)[128], bool ok, int n0, int N,
                                           const float* __restrict__ col_bias) {
  if (ok) stage_tile<Cfg>(tiles, acc);
  constexpr int kPitch = Cfg::BN + 4;
  float* sbias = reinterpret_cast<float*>(tiles) + kBM * kPitch;
  const int jj = threadIdx.x - 64;
  sbias[jj] = (col_bias != nullptr && n0 + jj < N) ? __ldg(col_bias + n0 + jj) : 0.0f;
}

// TMA-store epilogue (C 16-byte aligned with a 16-byte row pitch),
// gemm_stage_store_boxes (epilogue warps, right after the drain): bias +
// activation of the thread's row of 128 columns into 32-column boxes in the
// free operand ring (128 rows x 128 bytes each, 128-byte swizzle: 16-byte
// chunk c of row r at chunk c ^ (r % 8), so a warp's 32 rows hit every bank
// once), each box stored with TMA (rows and columns outside C are clipped) as
// soon as its 128 rows are staged.
// The tile's column biases in the shared words past the barriers, written by
// the epilogue warps before their drain (named barrier 2 among them).
template <class Cfg>
__device__ __forceinline__ float* tile_bias(uint8_t* tiles) {
  return reinterpret_cast<float*>(tiles + Cfg::RING_BYTES + 256);
}

template <class Cfg>
__device__ __forceinline__ void load_tile_bias(uint8_t* tiles, int n0, int N, const float* __restrict__ col_bias) {
  const int jj = threadIdx.x - 64;  // epilogue thread index: BN of them
  tile_bias<Cfg>(tiles)[jj] = (col_bias != nullptr && n0 + jj < N) ? __ldg(col_bias + n0 + jj) : 0.0f;
  asm volatile("bar.sync 2, %0;" ::"r"(Cfg::EPI_WARPS * 32) : "memory");
}

// Epilogue warps: bias + activation of this thread's row into the 32-column
// boxes, box by box; as soon as the four warps of a column half have staged a
// box (named barrier 3 + half), one thread of the half issues its TMA store,
// so the stores of the first boxes overlap the staging of the later ones. The
// issuing threads wait for their copies' shared-memory reads before the CTA
// may end. On a failed drain the boxes are not written and nothing is stored.
template <class Cfg, int ACT>
__device__ __forceinline__ void gemm_stage_store_boxes(uint8_t* tiles, const float (&acc)[128], bool ok,
                                                       bool has_bias, const CUtensorMap* mC, int m0, int n0) {
  const int warp = threadIdx.x >> 5;
  const int row = (warp & 3) * 32 + (threadIdx.x & 31);
  const int half = (warp - 2) >> 2;
  const bool issuer = (threadIdx.x - 64) % 128 == 0;
  const float* sb = tile_bias<Cfg>(tiles) + half * 128;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    uint8_t* box = tiles + (half * 4 + b) * (kBM * 128) + row * 128;
    if (ok) {
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float4 bv = *reinterpret_cast<const float4*>(sb + b * 32 + c * 4);  // broadcast
        const float bb[4] = {bv.x, bv.y, bv.z, bv.w};
        float v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int j = b * 32 + c * 4 + t;
          v[t] = act_t<ACT>(has_bias ? __fadd_rn(acc[j], bb[t]) : acc[j]);
        }
        *reinterpret_cast<float4*>(box + ((c ^ (row & 7)) << 4)) = make_float4(v[0], v[1], v[2], v[3]);
      }
      fence_async_smem();
    }
    asm volatile("bar.sync %0, 128;" ::"r"(3 + half) : "memory");
    if (issuer && ok) tma_store_2d(mC, tiles + (half * 4 + b) * (kBM * 128), n0 + 32 * (half * 4 + b), m0);
  }
  if (issuer && ok) {
    bulk_commit();
    bulk_wait_read_all();  // the shared-memory boxes must outlive the copies' reads
  }
}

static_assert(kBM * 128 * 8 <= Tf32x3Cfg<256, 2, 2>::TILE_BYTES, "TMA-store boxes fit the operand ring");

// ACT: the fused activation as a compile-time constant (no per-element switch).
template <class Cfg, int ACT>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    k_gemm_tf32x3(const __grid_constant__ CUtensorMap mAh, const __grid_constant__ CUtensorMap mAl,
                  const __grid_constant__ CUtensorMap mBh, const __grid_constant__ CUtensorMap mBl, int M, int N,
                  int Kp, const float* __restrict__ col_bias, const __grid_constant__ CUtensorMap mC,
                  int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = tiles_base<Cfg>(smem_raw);
  PipeBarriers* pb = barriers<Cfg>(tiles);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM;
  const int n0 = blockIdx.x * Cfg::BN;
  const int num_kb = (Kp + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    tma_prefetch(&mAh);
    tma_prefetch(&mAl);
    tma_prefetch(&mBh);
    tma_prefetch(&mBl);
  }
  const uint32_t tmem = pipe_setup<Cfg>(pb);
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();

  if (warp == 0) {
    if (lane == 0)
      producer_loop<Cfg>(tiles, pb, num_kb, err, [&](int kb, uint8_t* st, uint64_t* bar) {
        const int kc = kb * kBK;
        tma_load_2d(st, &mAh, bar, kc, m0);
        tma_load_2d(st + Cfg::A_BYTES, &mAl, bar, kc, m0);
        tma_load_2d(st + 2 * Cfg::A_BYTES, &mBh, bar, kc, n0);
        tma_load_2d(st + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &mBl, bar, kc, n0);
      });
  } else if (warp == 1) {
    if (lane == 0) mma_loop<Cfg>(tiles, pb, tmem, num_kb, err);
  } else {
    load_tile_bias<Cfg>(tiles, n0, N, col_bias);
    float acc[128];
    const bool ok = drain_loop<Cfg>(pb, tmem, num_kb, acc, err);
    gemm_stage_store_boxes<Cfg, ACT>(tiles, acc, ok, col_bias != nullptr, &mC, m0, n0);
  }
  pipe_teardown<Cfg>(pb, tmem);
}

// CTA-pair form (cluster of 2, tcgen05 cta_group::2): the pair computes a
// 256 x BN tile; CTA r of the pair owns rows m0 + 128r and loads columns
// n0 + r*BN/2 .. of B, so each CTA streams 2/3 of the single-CTA operand bytes
// for the same MMA work. Grid: x = 2 * column tiles (clusters of 2 along x),
// y = 256-row tiles.
template <class Cfg, int ACT>
__global__ void __launch_bounds__(Cfg::THREADS, 1)
    k_gemm_tf32x3_pair(const __grid_constant__ CUtensorMap mAh, const __grid_constant__ CUtensorMap mAl,
                       const __grid_constant__ CUtensorMap mBh, const __grid_constant__ CUtensorMap mBl, int M, int N,
                       int Kp, const float* __restrict__ col_bias, const __grid_constant__ CUtensorMap mC,
                       int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = tiles_base<Cfg>(smem_raw);
  PairBarriers* pb = pair_barriers<Cfg>(tiles);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int m0 = blockIdx.y * (2 * kBM) + static_cast<int>(rank) * kBM;
  const int n0 = (blockIdx.x >> 1) * Cfg::BN;
  const int nb = n0 + static_cast<int>(rank) * (Cfg::BN / 2);
  const int num_kb = (Kp + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    tma_prefetch(&mAh);
    tma_prefetch(&mAl);
    tma_prefetch(&mBh);
    tma_prefetch(&mBl);
  }
  const uint32_t tmem = pipe_setup_pair<Cfg>(pb);
  griddep_wait();  // launched with programmatic stream serialization: the previous kernel has completed
  griddep_launch();

  if (warp == 0) {
    if (lane == 0)
      producer_loop_pair<Cfg>(tiles, pb, num_kb, rank, err, [&](int kb, uint8_t* st, uint32_t bar) {
        const int kc = kb * kBK;
        tma_load_2d_pair(st, &mAh, bar, kc, m0);
        tma_load_2d_pair(st + Cfg::A_BYTES, &mAl, bar, kc, m0);
        tma_load_2d_pair(st + 2 * Cfg::A_BYTES, &mBh, bar, kc, nb);
        tma_load_2d_pair(st + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &mBl, bar, kc, nb);
      });
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) mma_loop_pair<Cfg>(tiles, pb, tmem, num_kb, err);
  } else {
    load_tile_bias<Cfg>(tiles, n0, N, col_bias);
    float acc[128];
    const bool ok = drain_loop_pair<Cfg>(pb, tmem, num_kb, acc, err);
    gemm_stage_store_boxes<Cfg, ACT>(tiles, acc, ok, col_bias != nullptr, &mC, m0, n0);
  }
  pipe_teardown_pair<Cfg>(pb, tmem, rank, err);
}

// ------------------------------------------------------------ general / batched
// Operands of a MatMul whose B is not a prepacked constant, of a batched
// (or transposed-view) MatMul and of ONNX Gemm: any strided [batch][rows][K]
// view is gathered into the K-major hi/lo layout the MMA reads, then a
// batched kernel (3-D tensor maps over the batch) runs the same main loop.
struct EpiAffine {
  float alpha, beta;       // ONNX Gemm: y = alpha * acc + beta * C (as two rounded products and a rounded add)
  const float* c;          // C broadcast as Gemm does: [M*N] full, 1 scalar, else c[j % c_len]
  long long c_len;
  long long y_outer, y_inner;  // y of batch z = o * inner + i starts at o * y_outer + i * y_inner
  int inner;
  long long y_ld;          // row pitch of y
  int b_batched;           // B differs per batch (else batch 0 for all)
  const float* row_scale;  // optional [batches][M]: y *= row_scale (FusedAttention's lazy 1/sum)
};

// src element (z, r, c) at src + (z / inner) * so + (z % inner) * si + r * sr + c * sc
// -> hi/lo [z][r][kp] with c contiguous, zero for c >= cols. 32 x 32 tiles
// through shared memory so both the read (along whichever source stride is 1)
// and the write are coalesced.
__global__ void k_gather_split(const float* __restrict__ src, int inner, long long so, long long si, long long sr,
                               long long sc, int rows, int cols, int kp, float* __restrict__ hi,
                               float* __restrict__ lo) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  __shared__ float tile[32][33];
  const int z = blockIdx.z;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const float* base = src + static_cast<long long>(z / inner) * so + static_cast<long long>(z % inner) * si;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  const bool rows_contig = sr == 1 && sc != 1;
  for (int yy = ty; yy < 32; yy += 8) {
    // read: consecutive threads along the contiguous source dimension
    const int r = rows_contig ? r0 + tx : r0 + yy;
    const int c = rows_contig ? c0 + yy : c0 + tx;
    const float v = (r < rows && c < cols) ? __ldg(base + r * sr + c * sc) : 0.0f;
    if (rows_contig) tile[yy][tx] = v;  // tile[c][r]
    else tile[tx][yy] = v;              // tile[c][r]
  }
  __syncthreads();
  for (int yy = ty; yy < 32; yy += 8) {
    const int r = r0 + yy, c = c0 + tx;
    if (r < rows && c < kp) {
      const float v = tile[tx][yy];
      const float h = to_tf32(v);
      const size_t o = (static_cast<size_t>(z) * rows + r) * kp + c;
      hi[o] = h;
      lo[o] = __fsub_rn(v, h);
    }
  }
}

template <class Cfg>
__global__ void __launch_bounds__(Cfg::THREADS, Cfg::STAGES == 1 ? 2 : 1)
    k_gemm_tf32x3_batched(const __grid_constant__ CUtensorMap mAh, const __grid_constant__ CUtensorMap mAl,
                          const __grid_constant__ CUtensorMap mBh, const __grid_constant__ CUtensorMap mBl, int M,
                          int N, int Kp, const float* __restrict__ col_bias, int act,
                          const __grid_constant__ EpiAffine ep, float* __restrict__ Y, int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* tiles = tiles_base<Cfg>(smem_raw);
  PipeBarriers* pb = barriers<Cfg>(tiles);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM;
  const int n0 = blockIdx.x * Cfg::BN;
  const int z = blockIdx.z, zb = ep.b_batched ? z : 0;
  const int num_kb = (Kp + kBK - 1) / kBK;
  if (Cfg::TMEM_COLS < 2 * Cfg::BN && num_kb > Cfg::KC) {  // one accumulator buffer: one chunk at most
    if (threadIdx.x == 0) atomicCAS(err, 0, OSC_EINVAL);
    return;
  }
  if (threadIdx.x == 0) {
    tma_prefetch(&mAh);
    tma_prefetch(&mAl);
    tma_prefetch(&mBh);
    tma_prefetch(&mBl);
  }
  const uint32_t tmem = pipe_setup<Cfg>(pb);
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  if (warp == 0) {
    if (lane == 0)
      producer_loop<Cfg>(tiles, pb, num_kb, err, [&](int kb, uint8_t* st, uint64_t* bar) {
        const int kc = kb * kBK;
        tma_load_3d(st, &mAh, bar, kc, m0, z);
        tma_load_3d(st + Cfg::A_BYTES, &mAl, bar, kc, m0, z);
        tma_load_3d(st + 2 * Cfg::A_BYTES, &mBh, bar, kc, n0, zb);
        tma_load_3d(st + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &mBl, bar, kc, n0, zb);
      });
  } else if (warp == 1) {
    if (lane == 0) mma_loop<Cfg>(tiles, pb, tmem, num_kb, err);
  } else {
    float acc[128];
    const bool ok = drain_loop<Cfg>(pb, tmem, num_kb, acc, err);
    gemm_stage<Cfg>(tiles, acc, ok, n0, N, col_bias);
  }
  asm volatile("bar.sync 1, %0;" ::"r"(Cfg::THREADS) : "memory");
  if (!pb->abort_flag) {
    // Every warp copies rows out: 4 rows per warp in flight, 16-byte shared
    // loads, the per-element steps (bias, alpha, beta * C, row scale,
    // activation) decided once per tile. Per element the order is unchanged.
    constexpr int kPitch = Cfg::BN + 4;
    constexpr int kWarps = Cfg::THREADS / 32;
    const float* stage = reinterpret_cast<const float*>(tiles);
    const float* sbias = stage + kBM * kPitch;
    float* Yz = Y + static_cast<long long>(z / ep.inner) * ep.y_outer + static_cast<long long>(z % ep.inner) * ep.y_inner;
    const bool has_bias = col_bias != nullptr;
    const bool scale_a = ep.alpha != 1.0f;
    const bool add_c = ep.beta != 0.0f && ep.c != nullptr && ep.c_len > 0;
    const bool full_c = ep.c_len >= static_cast<long long>(M) * N;
    const bool has_rs = ep.row_scale != nullptr;
    with_act(act, [&](auto tag) {
      constexpr int ACT = decltype(tag)::value;
      for (int r0 = warp; r0 < kBM; r0 += 4 * kWarps) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int r = r0 + u * kWarps;
          const int row = m0 + r;
          if (r < kBM && row < M) {
            float* yrow = Yz + static_cast<size_t>(row) * ep.y_ld;
            const float rs = has_rs ? ep.row_scale[static_cast<size_t>(z) * M + row] : 1.0f;
            const bool vec_row = (reinterpret_cast<uintptr_t>(yrow) & 15u) == 0;
#pragma unroll
            for (int h = 0; h < Cfg::BN; h += 128) {
              const int c0 = h + lane * 4;
              const int j0 = n0 + c0;
              const float4 sv = *reinterpret_cast<const float4*>(stage + r * kPitch + c0);
              float v[4] = {sv.x, sv.y, sv.z, sv.w};
              if (has_bias) {
                const float4 bv = *reinterpret_cast<const float4*>(sbias + c0);
                v[0] = __fadd_rn(v[0], bv.x);
                v[1] = __fadd_rn(v[1], bv.y);
                v[2] = __fadd_rn(v[2], bv.z);
                v[3] = __fadd_rn(v[3], bv.w);
              }
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const int j = j0 + t;
                if (scale_a) v[t] = __fmul_rn(ep.alpha, v[t]);  // Gemm (AttnOps.cs:100-128): alpha * d, then + beta * c
                if (add_c && j < N) {
                  const float cv = full_c ? ep.c[static_cast<size_t>(row) * N + j]
                                          : (ep.c_len == 1 ? ep.c[0] : ep.c[j % ep.c_len]);
                  v[t] = __fadd_rn(v[t], __fmul_rn(ep.beta, cv));
                }
                if (has_rs) v[t] = __fmul_rn(v[t], rs);
                v[t] = act_t<ACT>(v[t]);
              }
              if (vec_row && j0 + 4 <= N) {  // 16-byte stores: whole 32-byte sectors per lane pair
                *reinterpret_cast<float4*>(yrow + j0) = make_float4(v[0], v[1], v[2], v[3]);
              } else {
#pragma unroll
                for (int t = 0; t < 4; ++t)
                  if (j0 + t < N) yrow[j0 + t] = v[t];
              }
            }
          }
        }
      }
    });
  }
  pipe_teardown<Cfg>(pb, tmem);
}

// [rows][k] (row pitch ld) -> hi/lo [rows][kp], zero-padded for k <= c < kp.
__global__ void k_split_rows(const float* __restrict__ src, int rows, int k, int ld, int kp, float* __restrict__ hi,
                             float* __restrict__ lo) {
  const size_t total4 = static_cast<size_t>(rows) * (kp >> 2);
  const bool vec = ((ld & 3) == 0) && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total4;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / (kp >> 2);
    const int c = static_cast<int>(i - r * (kp >> 2)) * 4;
    const float* s = src + r * static_cast<size_t>(ld);
    float v[4];
    if (vec && c + 4 <= k) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(s + c));
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = (c + j < k) ? s[c + j] : 0.0f;
    }
    float h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = to_tf32(v[j]);
      l[j] = __fsub_rn(v[j], h[j]);
    }
    const size_t o = r * static_cast<size_t>(kp) + c;
    *reinterpret_cast<float4*>(hi + o) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4*>(lo + o) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

// B[k][n] (row-major, MatMul layout) -> hi/lo [n][kp] (transposed, split, zero-padded).
__global__ void k_pack_b_kn(const float* __restrict__ b, int k, int n, int kp, float* __restrict__ hi,
                            float* __restrict__ lo) {
  __shared__ float tile[32][33];
  const int n0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (int yy = ty; yy < 32; yy += 8) {
    const int kk = k0 + yy, nn = n0 + tx;
    tile[yy][tx] = (kk < k && nn < n) ? b[static_cast<size_t>(kk) * n + nn] : 0.0f;
  }
  __syncthreads();
  for (int yy = ty; yy < 32; yy += 8) {
    const int nn = n0 + yy, kk = k0 + tx;
    if (nn < n && kk < kp) {
      const float v = tile[tx][yy];
      const float h = to_tf32(v);
      hi[static_cast<size_t>(nn) * kp + kk] = h;
      lo[static_cast<size_t>(nn) * kp + kk] = __fsub_rn(v, h);
    }
  }
}

// The kernel instantiation for a runtime activation code.
template <class Cfg>
auto gemm_kernel(int act) {
  switch (act) {
    case ACT_SILU: return k_gemm_tf32x3<Cfg, ACT_SILU>;
    case ACT_RELU: return k_gemm_tf32x3<Cfg, ACT_RELU>;
    case ACT_SIGMOID: return k_gemm_tf32x3<Cfg, ACT_SIGMOID>;
    default: return k_gemm_tf32x3<Cfg, ACT_NONE>;
  }
}
template <class Cfg>
auto gemm_pair_kernel(int act) {
  switch (act) {
    case ACT_SILU: return k_gemm_tf32x3_pair<Cfg, ACT_SILU>;
    case ACT_RELU: return k_gemm_tf32x3_pair<Cfg, ACT_RELU>;
    case ACT_SIGMOID: return k_gemm_tf32x3_pair<Cfg, ACT_SIGMOID>;
    default: return k_gemm_tf32x3_pair<Cfg, ACT_NONE>;
  }
}

// Tensor map of C for the TMA-store epilogue (32 x 128 boxes, 128-byte
// swizzle). C's base and row pitch must be 16-byte aligned (c_tma_ok).
static bool c_tma_ok(const float* C, int N, int ldc) {
  return (reinterpret_cast<uintptr_t>(C) & 15u) == 0 && ldc % 4 == 0 && ldc >= N;
}

static int store_map(CUtensorMap* map, float* C, int M, int N, int ldc) {
  const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
  const uint64_t pitch[1] = {static_cast<uint64_t>(ldc) * 4};
  const uint32_t box[2] = {32, kBM};
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, C, dims, pitch, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <class Cfg>
int launch_gemm(osc_ctx* ctx, const float* ahi, const float* alo, int M, int Kp, const osc_gemm_weights* w,
                const float* bias, int act, float* C, int ldc) {
  CUtensorMap mAh, mAl, mBh, mBl;
  const uint64_t dimsA[2] = {static_cast<uint64_t>(Kp), static_cast<uint64_t>(M)};
  const uint64_t dimsB[2] = {static_cast<uint64_t>(Kp), static_cast<uint64_t>(w->n)};
  const uint64_t pitch[1] = {static_cast<uint64_t>(Kp) * 4};
  const uint32_t boxA[2] = {kBK, kBM};
  const uint32_t boxB[2] = {kBK, static_cast<uint32_t>(Cfg::BN)};
  OSC_TRY(encode_tiled(&mAh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ahi, dimsA, pitch, boxA, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mAl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, alo, dimsA, pitch, boxA, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mBh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w->hi, dimsB, pitch, boxB, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mBl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w->lo, dimsB, pitch, boxB, CU_TENSOR_MAP_SWIZZLE_128B));
  CUtensorMap mC{};
  OSC_TRY(store_map(&mC, C, M, w->n, ldc));
  auto kern = gemm_kernel<Cfg>(act);
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(kern), Cfg::SMEM_BYTES));
  dim3 grid((w->n + Cfg::BN - 1) / Cfg::BN, (M + kBM - 1) / kBM);
  return launch_pdl(ctx, kern, grid, dim3(Cfg::THREADS), Cfg::SMEM_BYTES, "k_gemm_tf32x3", mAh, mAl, mBh, mBl, M, w->n,
                    Kp, bias, mC, ctx->d_err);
}

template <class Cfg>
int launch_gemm_pair(osc_ctx* ctx, const float* ahi, const float* alo, int M, int Kp, const osc_gemm_weights* w,
                     const float* bias, int act, float* C, int ldc) {
  CUtensorMap mAh, mAl, mBh, mBl;
  const uint64_t dimsA[2] = {static_cast<uint64_t>(Kp), static_cast<uint64_t>(M)};
  const uint64_t dimsB[2] = {static_cast<uint64_t>(Kp), static_cast<uint64_t>(w->n)};
  const uint64_t pitch[1] = {static_cast<uint64_t>(Kp) * 4};
  const uint32_t boxA[2] = {kBK, kBM};
  const uint32_t boxB[2] = {kBK, static_cast<uint32_t>(Cfg::BN / 2)};
  OSC_TRY(encode_tiled(&mAh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ahi, dimsA, pitch, boxA, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mAl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, alo, dimsA, pitch, boxA, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mBh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w->hi, dimsB, pitch, boxB, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mBl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, w->lo, dimsB, pitch, boxB, CU_TENSOR_MAP_SWIZZLE_128B));
  auto kern = gemm_pair_kernel<Cfg>(act);
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(kern), Cfg::SMEM_BYTES));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * ((w->n + Cfg::BN - 1) / Cfg::BN), (M + 2 * kBM - 1) / (2 * kBM));
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // set-up overlaps the previous kernel's tail
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  prof_begin(ctx);
  CUtensorMap mC{};
  OSC_TRY(store_map(&mC, C, M, w->n, ldc));
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mAh, mAl, mBh, mBl, M, w->n, Kp, bias, mC, ctx->d_err);
  if (e != cudaSuccess) return cuda_fail(e, "k_gemm_tf32x3_pair launch");
  return check_launch(ctx, "k_gemm_tf32x3");
}

int grid_for(osc_ctx* ctx, size_t work, int per_thread) {
  size_t blocks = (work + static_cast<size_t>(256) * per_thread - 1) / (static_cast<size_t>(256) * per_thread);
  const size_t cap = static_cast<size_t>(ctx->num_sms) * 8;
  if (blocks > cap) blocks = cap;
  return static_cast<int>(blocks < 1 ? 1 : blocks);
}

}  // namespace

// Shared with the other kernels that consume split activations.
int split_tf32(osc_ctx* ctx, const float* src, int rows, int k, int ld, int kp, float* hi, float* lo) {
  const size_t work = static_cast<size_t>(rows) * (kp / 4);
  prof_begin(ctx);
  k_split_rows<<<grid_for(ctx, work, 1), 256, 0, ctx->stream>>>(src, rows, k, ld, kp, hi, lo);
  return check_launch(ctx, "k_split_rows");
}

static int gemm_batched(osc_ctx* ctx, const float* ahi, const float* alo, int batches, int M, int Kp,
                        const float* bhi, const float* blo, int b_batches, int N, const float* col_bias, int act,
                        const EpiAffine& ep, float* y);

// Routes an A already split into K-major hi/lo parts [m][kp] to the GEMM
// kernel for its shape. Allocates nothing.
int gemm_presplit(osc_ctx* ctx, const float* ahi, const float* alo, int m, int kp, const osc_gemm_weights* w,
                  const float* col_bias, int act, float* c, int ldc) {
  if (!c_tma_ok(c, w->n, ldc)) {  // C not 16-byte aligned: the batched kernel's plain-store epilogue
    const EpiAffine ep{1.0f, 0.0f, nullptr, 0, 0, 0, 1, ldc, 0, nullptr};
    return gemm_batched(ctx, ahi, alo, 1, m, kp, w->hi, w->lo, 1, w->n, col_bias, act, ep, c);
  }
  // Prefer the wider tile (less operand traffic per FLOP) unless it leaves
  // most SMs idle; wide tiles of more than one row block run on CTA pairs.
  const long tiles256 = static_cast<long>((w->n + 255) / 256) * ((m + kBM - 1) / kBM);
  const bool wide = w->n > 128 && tiles256 >= ctx->num_sms * 3 / 4;
  if (wide && m > kBM)
    return launch_gemm_pair<Tf32x3PairCfg<256, 3, 2>>(ctx, ahi, alo, m, kp, w, col_bias, act, c, ldc);
  if (wide) return launch_gemm<Tf32x3Cfg<256, 2, 2>>(ctx, ahi, alo, m, kp, w, col_bias, act, c, ldc);
  return launch_gemm<Tf32x3Cfg<128, 3, 2>>(ctx, ahi, alo, m, kp, w, col_bias, act, c, ldc);
}

int gemm_tf32x3(osc_ctx* ctx, const float* a, int m, int k, int lda, const osc_gemm_weights* w,
                const float* col_bias, int act, float* c, int ldc) {
  const int kp = w->kp;
  void* buf = nullptr;
  const size_t half = round_up(static_cast<size_t>(m) * kp * sizeof(float), 256);
  OSC_TRY(scratch(ctx, 2 * half, &buf));
  float* ahi = static_cast<float*>(buf);
  float* alo = reinterpret_cast<float*>(static_cast<uint8_t*>(buf) + half);
  OSC_TRY(split_tf32(ctx, a, m, k, lda, kp, ahi, alo));
  return gemm_presplit(ctx, ahi, alo, m, kp, w, col_bias, act, c, ldc);
}

// A strided view [batches][rows][cols] -> hi/lo [batches][rows][kp] in `dst_hi/lo`.
static int gather_split(osc_ctx* ctx, const float* src, int batches, int inner, long long so, long long si,
                        long long sr, long long sc, int rows, int cols, int kp, float* hi, float* lo) {
  if (batches > 65535) return fail(OSC_EUNSUPPORTED, "matmul: %d batches (65535 at most)", batches);
  dim3 grid((kp + 31) / 32, (rows + 31) / 32, batches);
  return launch_pdl(ctx, k_gather_split, grid, dim3(256), 0, "k_gather_split", src, inner, so, si, sr, sc, rows, cols,
                    kp, hi, lo);
}

// C[z] = A[z] (M x K) * B[zb] (K x N) on split operands Ahi/lo [batches][M][Kp],
// Bhi/lo [b_batches][N][Kp].
template <class Cfg>
static int gemm_batched_cfg(osc_ctx* ctx, const float* ahi, const float* alo, int batches, int M, int Kp,
                            const float* bhi, const float* blo, int b_batches, int N, const float* col_bias, int act,
                            const EpiAffine& ep, float* y) {
  CUtensorMap mAh, mAl, mBh, mBl;
  const uint64_t dimsA[3] = {static_cast<uint64_t>(Kp), static_cast<uint64_t>(M), static_cast<uint64_t>(batches)};
  const uint64_t dimsB[3] = {static_cast<uint64_t>(Kp), static_cast<uint64_t>(N), static_cast<uint64_t>(b_batches)};
  const uint64_t pitchA[2] = {static_cast<uint64_t>(Kp) * 4, static_cast<uint64_t>(Kp) * 4 * M};
  const uint64_t pitchB[2] = {static_cast<uint64_t>(Kp) * 4, static_cast<uint64_t>(Kp) * 4 * N};
  const uint32_t boxA[3] = {kBK, kBM, 1};
  const uint32_t boxB[3] = {kBK, static_cast<uint32_t>(Cfg::BN), 1};
  OSC_TRY(encode_tiled(&mAh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ahi, dimsA, pitchA, boxA, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mAl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, alo, dimsA, pitchA, boxA, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mBh, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, bhi, dimsB, pitchB, boxB, CU_TENSOR_MAP_SWIZZLE_128B));
  OSC_TRY(encode_tiled(&mBl, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, blo, dimsB, pitchB, boxB, CU_TENSOR_MAP_SWIZZLE_128B));
  auto kern = k_gemm_tf32x3_batched<Cfg>;
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(kern), Cfg::SMEM_BYTES));
  if (batches > 65535) return fail(OSC_EUNSUPPORTED, "matmul: %d batches (65535 at most)", batches);
  dim3 grid((N + Cfg::BN - 1) / Cfg::BN, (M + kBM - 1) / kBM, batches);
  return launch_pdl(ctx, kern, grid, dim3(Cfg::THREADS), Cfg::SMEM_BYTES, "k_gemm_tf32x3", mAh, mAl, mBh, mBl, M, N,
                    Kp, col_bias, act, ep, y, ctx->d_err);
}

// Products of at most two k-blocks (K <= 64: PSA's q.k^T with 32 channels)
// take the one-stage configuration: ~70 KB of shared memory and one
// 128-column accumulator, so three CTAs share an SM and one CTA's loads and
// MMAs run under another's epilogue (with the three-stage ring a CTA holds
// the SM alone and every tile's setup, load, MMA and stores run in series).
static int gemm_batched(osc_ctx* ctx, const float* ahi, const float* alo, int batches, int M, int Kp,
                        const float* bhi, const float* blo, int b_batches, int N, const float* col_bias, int act,
                        const EpiAffine& ep, float* y) {
  if ((Kp + kBK - 1) / kBK <= 2)
    return gemm_batched_cfg<Tf32x3Cfg<128, 1, 2>>(ctx, ahi, alo, batches, M, Kp, bhi, blo, b_batches, N, col_bias,
                                                  act, ep, y);
  return gemm_batched_cfg<Tf32x3Cfg<128, 3, 2>>(ctx, ahi, alo, batches, M, Kp, bhi, blo, b_batches, N, col_bias, act,
                                                ep, y);
}

// Bytes of work space batched_strided needs for its split operands.
static size_t batched_work_bytes(long long batches, int m, int k, int n) {
  const size_t kp = round_up(static_cast<size_t>(k), 4);
  return 2 * round_up(static_cast<size_t>(batches) * m * kp * sizeof(float), 256) +
         2 * round_up(static_cast<size_t>(batches) * n * kp * sizeof(float), 256);
}

// Strided batched product into `y` with epilogue `ep` (its y strides), using
// caller-provided `work` (batched_work_bytes) for the split operands.
static int batched_strided(osc_ctx* ctx, int outer, int inner, int m, int k, int n, const float* a, long long a_outer,
                           long long a_inner, long long a_row, long long a_col, const float* b, long long b_outer,
                           long long b_inner, long long b_row, long long b_col, const float* col_bias,
                           const EpiAffine& ep, float* y, void* work) {
  const long long batches = static_cast<long long>(outer) * inner;
  const int kp = static_cast<int>(round_up(static_cast<size_t>(k), 4));
  const size_t abytes = round_up(static_cast<size_t>(batches) * m * kp * sizeof(float), 256);
  const size_t bbytes = round_up(static_cast<size_t>(batches) * n * kp * sizeof(float), 256);
  uint8_t* p = static_cast<uint8_t*>(work);
  float* ahi = reinterpret_cast<float*>(p);
  float* alo = reinterpret_cast<float*>(p + abytes);
  float* bhi = reinterpret_cast<float*>(p + 2 * abytes);
  float* blo = reinterpret_cast<float*>(p + 2 * abytes + bbytes);
  const int nb = static_cast<int>(batches);
  OSC_TRY(gather_split(ctx, a, nb, inner, a_outer, a_inner, a_row, a_col, m, k, kp, ahi, alo));
  OSC_TRY(gather_split(ctx, b, nb, inner, b_outer, b_inner, b_col, b_row, n, k, kp, bhi, blo));
  return gemm_batched(ctx, ahi, alo, nb, m, kp, bhi, blo, nb, n, col_bias, OSC_ACT_NONE, ep, y);
}

// y = x * s, each product rounded once (AttentionOps.cs:531-537: q' = q * scale).
__global__ void k_scale_copy(const float* __restrict__ x, long long n, float s, float* __restrict__ y) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = __fmul_rn(__ldg(x + i), s);
}

// The lazy softmax of AttentionOps.cs:590-604 on rows of S [B*H][T][T] in
// place: optional additive mask, row max, e = exp(s - max) (the reference's
// polynomial on the 8-aligned part, MathF.Exp on the tail) left unnormalised,
// 1/sum per row (8 lane sums in key order, then the lanes, then the tail).
__global__ void k_attn_rows(float* __restrict__ S, long long rows, int T, int H, const float* __restrict__ mask,
                            int mask_rows, float* __restrict__ pinv) {
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += warps) {
    float* sr = S + r * T;
    const long long z = r / T;
    const int t = static_cast<int>(r - z * T);
    const int b = static_cast<int>(z / H);
    if (mask != nullptr) {
      const float* mr = mask + (static_cast<long long>(b) * mask_rows + (mask_rows == 1 ? 0 : t)) * T;
      for (int j = lane; j < T; j += 32) sr[j] = __fadd_rn(sr[j], __ldg(mr + j));
      __syncwarp();
    }
    float mx = -INFINITY;
    for (int j = lane; j < T; j += 32) mx = fmaxf(mx, sr[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int vend = T & ~7;
    float part = 0.0f;
    if (lane < 8)
      for (int j = lane; j < vend; j += 8) {
        const float e = ref_exp(__fsub_rn(sr[j], mx));
        sr[j] = e;
        part = __fadd_rn(part, e);
      }
    float total = 0.0f;
    for (int l = 0; l < 8; ++l) total = __fadd_rn(total, __shfl_sync(0xffffffffu, part, l));
    for (int j = vend; j < T; ++j) {  // scalar tail (uniform across the warp)
      const float e = expf(__fsub_rn(sr[j], mx));
      __syncwarp();
      if (lane == 0) sr[j] = e;
      total = __fadd_rn(total, e);
    }
    if (lane == 0) pinv[r] = __fdiv_rn(1.0f, total);
  }
}

// FusedAttention for any T and head size: S = (q*scale) K^T per head on the
// tensor cores, the lazy softmax above, O = e V with the 1/sum row scaling in
// the product's epilogue (AttentionOps.cs:636-643), written straight into the
// requested output layout.
int attention_composed(osc_ctx* ctx, const float* q, const float* k, const float* v, const float* mask,
                       int mask_rows, int B, int T, int H, int D, float scale, int out_head_space, float* out) {
  const long long W = static_cast<long long>(H) * D;
  const long long qn = static_cast<long long>(B) * T * W;
  const long long sn = static_cast<long long>(B) * H * T * T;
  const size_t q_bytes = round_up(static_cast<size_t>(qn) * 4, 256);
  const size_t s_bytes = round_up(static_cast<size_t>(sn) * 4, 256);
  const size_t p_bytes = round_up(static_cast<size_t>(B) * H * T * 4, 256);
  const size_t w_bytes = std::max(batched_work_bytes(static_cast<long long>(B) * H, T, D, T),
                                  batched_work_bytes(static_cast<long long>(B) * H, T, T, D));
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, q_bytes + s_bytes + p_bytes + w_bytes, &buf));
  uint8_t* base = static_cast<uint8_t*>(buf);
  float* qs = reinterpret_cast<float*>(base);
  float* S = reinterpret_cast<float*>(base + q_bytes);
  float* pinv = reinterpret_cast<float*>(base + q_bytes + s_bytes);
  void* work = base + q_bytes + s_bytes + p_bytes;
  {
    const int blocks = static_cast<int>(std::min<long long>((qn + 255) / 256, static_cast<long long>(ctx->num_sms) * 8));
    prof_begin(ctx);
    k_scale_copy<<<blocks, 256, 0, ctx->stream>>>(q, qn, scale, qs);
    OSC_TRY(check_launch(ctx, "k_scale_copy"));
  }
  // S[b,h] = q'[b,:,h,:] K[b,:,h,:]^T : dense [B*H][T][T]
  {
    EpiAffine ep{1.0f, 0.0f, nullptr, 0, static_cast<long long>(H) * T * T, static_cast<long long>(T) * T, H, T, 1,
                 nullptr};
    OSC_TRY(batched_strided(ctx, B, H, T, D, T, qs, T * W, D, W, 1, k, T * W, D, 1, W, nullptr, ep, S, work));
  }
  {
    const long long rows = static_cast<long long>(B) * H * T;
    const int blocks = static_cast<int>(std::min<long long>((rows + 7) / 8, static_cast<long long>(ctx->num_sms) * 16));
    prof_begin(ctx);
    k_attn_rows<<<blocks, 256, 0, ctx->stream>>>(S, rows, T, H, mask, mask_rows, pinv);
    OSC_TRY(check_launch(ctx, "k_attn_rows"));
  }
  // O[b,h] = e[b,h] V[b,:,h,:], times 1/sum per row, into [B,H,T,D] or [B,T,H*D]
  EpiAffine ep{1.0f, 0.0f, nullptr, 0, 0, 0, H, 0, 1, pinv};
  if (out_head_space) {
    ep.y_outer = static_cast<long long>(H) * T * D;
    ep.y_inner = static_cast<long long>(T) * D;
    ep.y_ld = D;
  } else {
    ep.y_outer = T * W;
    ep.y_inner = D;
    ep.y_ld = W;
  }
  return batched_strided(ctx, B, H, T, T, D, S, static_cast<long long>(H) * T * T, static_cast<long long>(T) * T, T, 1,
                         v, T * W, D, W, 1, nullptr, ep, out, work);
}

// The reference's Softmax op (DnnOps.cs:2547; the order of k_softmax_rows:
// row max, e = exp(s - max) summed in 8 lanes over the 8-aligned part, the
// scalar tail, p = e * (1/sum)) on rows of S [rows][len], written as the
// hi/lo split MMA operand [rows][kp] (zero for len <= j < kp). One warp per
// row; e is parked in `hi` between the passes.
__global__ void k_softmax_split(const float* __restrict__ S, long long rows, int len, int kp, float* __restrict__ hi,
                                float* __restrict__ lo) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += warps) {
    const float* sr = S + r * len;
    float* hr = hi + r * kp;
    float* lr = lo + r * kp;
    float mx = -INFINITY;
    for (int j = lane; j < len; j += 32) mx = fmaxf(mx, __ldg(sr + j));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int vend = len & ~7;
    float part = 0.0f;
    if (lane < 8)
      for (int j = lane; j < vend; j += 8) {
        const float e = ref_exp(__fsub_rn(__ldg(sr + j), mx));
        hr[j] = e;
        part = __fadd_rn(part, e);
      }
    float total = 0.0f;
    for (int l = 0; l < 8; ++l) total = __fadd_rn(total, __shfl_sync(0xffffffffu, part, l));
    for (int j = vend; j < len; ++j) {  // scalar tail (uniform across the warp)
      const float e = expf(__fsub_rn(__ldg(sr + j), mx));
      if (lane == 0) hr[j] = e;
      total = __fadd_rn(total, e);
    }
    __syncwarp();
    const float inv = __fdiv_rn(1.0f, total);
    for (int j = lane; j < kp; j += 32) {
      const float p = j < len ? __fmul_rn(hr[j], inv) : 0.0f;
      const float h = to_tf32(p);
      hr[j] = h;
      lr[j] = __fsub_rn(p, h);
    }
  }
}

// The same for rows of at most kSoftRegs * 32 split columns (PSA: 400): the
// row lives in registers (element j in lane j % 32, slot j / 32), so S is
// read once and nothing is parked in global memory. All 32 lanes compute the
// exponentials; the reference's 8 partial sums keep their order: chain l
// (lanes 0..7) adds e[l], e[l+8], e[l+16], e[l+24], e[l+32], ... fetched by
// shuffles, then the chains are summed 0..7 and the scalar tail follows.
constexpr int kSoftRegs = 16;

__global__ void k_softmax_split_reg(const float* __restrict__ S, long long rows, int len, int kp,
                                    float* __restrict__ hi, float* __restrict__ lo) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const int vend = len & ~7;
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += warps) {
    const float* sr = S + r * len;
    float v[kSoftRegs];
#pragma unroll
    for (int k = 0; k < kSoftRegs; ++k) {
      const int j = lane + 32 * k;
      v[k] = j < len ? __ldg(sr + j) : -INFINITY;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kSoftRegs; ++k) mx = fmaxf(mx, v[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float e[kSoftRegs];
#pragma unroll
    for (int k = 0; k < kSoftRegs; ++k) {
      const int j = lane + 32 * k;
      e[k] = j < vend ? ref_exp(__fsub_rn(v[k], mx)) : (j < len ? expf(__fsub_rn(v[k], mx)) : 0.0f);
    }
    float part = 0.0f;  // chain (lane & 7), meaningful in lanes 0..7
#pragma unroll
    for (int k = 0; k < kSoftRegs; ++k) {
      if (32 * k >= vend) break;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float t = __shfl_sync(0xffffffffu, e[k], (lane & 7) + 8 * q);
        if (32 * k + 8 * q + (lane & 7) < vend) part = __fadd_rn(part, t);
      }
    }
    float total = 0.0f;
    for (int l = 0; l < 8; ++l) total = __fadd_rn(total, __shfl_sync(0xffffffffu, part, l));
    for (int j = vend; j < len; ++j) {  // scalar tail in order (uniform across the warp)
      const int kk = j >> 5;
      float mine = 0.0f;
#pragma unroll
      for (int k = 0; k < kSoftRegs; ++k)
        if (k == kk) mine = e[k];
      total = __fadd_rn(total, __shfl_sync(0xffffffffu, mine, j & 31));
    }
    const float inv = __fdiv_rn(1.0f, total);
    float* hr = hi + r * kp;
    float* lr = lo + r * kp;
#pragma unroll
    for (int k = 0; k < kSoftRegs; ++k) {
      const int j = lane + 32 * k;
      if (j < kp) {
        const float p = j < len ? __fmul_rn(e[k], inv) : 0.0f;
        const float h = to_tf32(p);
        hr[j] = h;
        lr[j] = __fsub_rn(p, h);
      }
    }
  }
}

// YOLO11's PSA attention fused in one kernel for its own head shape (key
// dim 32, head dim 64, up to kPsaMaxT tokens): one CTA per (block of QB
// query tokens, head, image), everything in shared memory, FP32 FMA on the
// CUDA cores -- the products are small (32 x T and T x 64 per query), so the
// composed path's S / P round trips through HBM and its six launches cost
// more than the arithmetic.
//   1. K^T [T][32] into shared memory; each thread keeps its query's 32 q
//      values in registers: S[n][m] = fl(q_n . k_m) * scale (FMA over c);
//   2. each warp takes rows of S through the reference's softmax (max, the
//      8 partial-sum chains of ref_exp, the expf tail, one reciprocal: the
//      same steps as k_softmax_split_reg), P in place, FP32;
//   3. V^T [T][64] over K^T's space (copied while the softmax runs);
//      out[d][n] = sum_m v[d][m] P[n][m] (FMA over m in order), written
//      channel-major like the composed path.
constexpr int kPsaKd = 32, kPsaHd = 64, kPsaMaxT = kSoftRegs * 32;
constexpr int kPsaKPitch = kPsaKd + 4, kPsaVPitch = kPsaHd + 4;  // 16-byte rows, fewer bank conflicts

template <int QB, int NT>
__global__ void __launch_bounds__(NT, 1)
    k_psa_fused(const float* __restrict__ qkv, long long qkv_nstride, int heads, int T, float scale,
                float* __restrict__ out, long long out_nstride) {
  griddep_wait();  // launched with launch_pdl: the previous kernel has completed past here
  griddep_launch();
  constexpr int G = NT / QB;            // thread groups (key groups in phase 1, channel groups in phase 3)
  constexpr int DPT = kPsaHd / G;       // output channels per thread in phase 3
  constexpr int NW = NT / 32;
  static_assert(NT % QB == 0 && kPsaHd % G == 0 && DPT % 4 == 0, "PSA tile shape");
  extern __shared__ __align__(16) float psa_smem[];
  const int Tp = (T + 3) & ~3;
  const int ppitch = Tp + 4;            // P rows: 16-byte aligned
  float* kv = psa_smem;                 // K^T [Tp][36], later V^T [Tp][68]
  float* P = psa_smem + static_cast<size_t>(Tp) * kPsaVPitch;  // [QB][ppitch]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int h = blockIdx.y, b = blockIdx.z;
  const int n0 = blockIdx.x * QB;
  const float* base = qkv + static_cast<long long>(b) * qkv_nstride +
                      static_cast<long long>(h) * (2 * kPsaKd + kPsaHd) * T;
  const float* qg = base;
  const float* kg = base + static_cast<long long>(kPsaKd) * T;
  const float* vg = base + static_cast<long long>(2 * kPsaKd) * T;
  // 1. K^T (asynchronous 4-byte copies, all in flight at once) and S (four
  //    keys per step: independent FMA chains)
  for (int c = warp; c < kPsaKd; c += NW)
    for (int m = lane; m < T; m += 32) cp_async4(kv + m * kPsaKPitch + c, kg + static_cast<long long>(c) * T + m, true);
  cp_async_commit();
  const int n = tid % QB, g = tid / QB;
  const bool nvalid = n0 + n < T;
  float q[kPsaKd];
#pragma unroll
  for (int c = 0; c < kPsaKd; ++c) q[c] = nvalid ? __ldg(qg + static_cast<long long>(c) * T + n0 + n) : 0.0f;
  cp_async_wait<0>();
  __syncthreads();
  for (int m0 = g; m0 < T; m0 += 4 * G) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float4* kr[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) kr[u] = reinterpret_cast<const float4*>(kv + min(m0 + u * G, T - 1) * kPsaKPitch);
#pragma unroll
    for (int c4 = 0; c4 < kPsaKd / 4; ++c4) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 k4 = kr[u][c4];
        acc[u] = __fmaf_rn(q[4 * c4 + 0], k4.x, acc[u]);
        acc[u] = __fmaf_rn(q[4 * c4 + 1], k4.y, acc[u]);
        acc[u] = __fmaf_rn(q[4 * c4 + 2], k4.z, acc[u]);
        acc[u] = __fmaf_rn(q[4 * c4 + 3], k4.w, acc[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (m0 + u * G < T) P[n * ppitch + m0 + u * G] = __fmul_rn(acc[u], scale);
  }
  __syncthreads();
  // V^T over K^T (zero rows up to Tp), landing while the softmax runs
  for (int d = warp; d < kPsaHd; d += NW)
    for (int m = lane; m < Tp; m += 32)
      cp_async4(kv + m * kPsaVPitch + d, vg + static_cast<long long>(d) * T + min(m, T - 1), m < T);
  cp_async_commit();
  // 2. softmax per row (rows past T are never stored)
  const int vend = T & ~7;
  for (int r = warp; r < QB; r += NW) {
    if (n0 + r >= T) break;
    float* pr = P + r * ppitch;
    float v[kSoftRegs];
#pragma unroll
    for (int k = 0; k < kSoftRegs; ++k) {
      const int j = lane + 32 * k;
      v[k] = j < T ? pr[j] : -INFINITY;
    }
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kSoftRegs; ++k) mx = fmaxf(mx, v[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float e[kSoftRegs];
#pragma unroll
    for (int k = 0; k < kSoftRegs; ++k) {
      const int j = lane + 32 * k;
      e[k] = j < vend ? ref_exp(__fsub_rn(v[k], mx)) : (j < T ? expf(__fsub_rn(v[k], mx)) : 0.0f);
    }
    float part = 0.0f;  // chain (lane & 7), meaningful in lanes 0..7
#pragma unroll
    for (int k = 0; k < kSoftRegs; ++k) {
      if (32 * k >= vend) break;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) {
        const float t = __shfl_sync(0xffffffffu, e[k], (lane & 7) + 8 * qq);
        if (32 * k + 8 * qq + (lane & 7) < vend) part = __fadd_rn(part, t);
      }
    }
    float total = 0.0f;
    for (int l = 0; l < 8; ++l) total = __fadd_rn(total, __shfl_sync(0xffffffffu, part, l));
    for (int j = vend; j < T; ++j) {  // scalar tail in order (uniform across the warp)
      const int kk = j >> 5;
      float mine = 0.0f;
#pragma unroll
      for (int k = 0; k < kSoftRegs; ++k)
        if (k == kk) mine = e[k];
      total = __fadd_rn(total, __shfl_sync(0xffffffffu, mine, j & 31));
    }
    const float inv = __fdiv_rn(1.0f, total);
#pragma unroll
    for (int k = 0; k < kSoftRegs; ++k) {
      const int j = lane + 32 * k;
      if (j < Tp) pr[j] = j < T ? __fmul_rn(e[k], inv) : 0.0f;
    }
  }
  // 3. out = V P^T
  cp_async_wait<0>();
  __syncthreads();
  if (!nvalid) return;
  const int d0 = g * DPT;
  float acc[DPT];
#pragma unroll
  for (int j = 0; j < DPT; ++j) acc[j] = 0.0f;
  const float* pr = P + n * ppitch;
  for (int m = 0; m < Tp; m += 4) {
    const float4 p4 = *reinterpret_cast<const float4*>(pr + m);
    const float pm[4] = {p4.x, p4.y, p4.z, p4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float4* vr = reinterpret_cast<const float4*>(kv + (m + u) * kPsaVPitch + d0);
#pragma unroll
      for (int j4 = 0; j4 < DPT / 4; ++j4) {
        const float4 v4 = vr[j4];
        acc[4 * j4 + 0] = __fmaf_rn(v4.x, pm[u], acc[4 * j4 + 0]);
        acc[4 * j4 + 1] = __fmaf_rn(v4.y, pm[u], acc[4 * j4 + 1]);
        acc[4 * j4 + 2] = __fmaf_rn(v4.z, pm[u], acc[4 * j4 + 2]);
        acc[4 * j4 + 3] = __fmaf_rn(v4.w, pm[u], acc[4 * j4 + 3]);
      }
    }
  }
  float* og = out + static_cast<long long>(b) * out_nstride + static_cast<long long>(h) * kPsaHd * T + n0 + n;
#pragma unroll
  for (int j = 0; j < DPT; ++j) og[static_cast<long long>(d0 + j) * T] = acc[j];
}

static size_t psa_fused_smem(int T, int QB) {
  const size_t Tp = (static_cast<size_t>(T) + 3) & ~size_t(3);
  return (Tp * kPsaVPitch + static_cast<size_t>(QB) * (Tp + 4)) * sizeof(float);
}

// The fused kernel when the head shape is YOLO11's and the tiles fit; returns
// OSC_EUNSUPPORTED (nothing launched) otherwise. Small batches take 16-query
// blocks (more CTAs), larger ones 64 (fewer K / V reloads).
int psa_fused(osc_ctx* ctx, const float* qkv, long long qkv_nstride, int B, int heads, int kd, int hd, int T,
              float scale, float* out, long long out_nstride) {
  if (kd != kPsaKd || hd != kPsaHd || T > kPsaMaxT || heads > 65535 || B > 65535) return OSC_EUNSUPPORTED;
  const long long blocks64 = static_cast<long long>(B) * heads * ((T + 63) / 64);
  const bool small = blocks64 < 2LL * ctx->num_sms;
  const int QB = small ? 16 : 64;
  const size_t smem = psa_fused_smem(T, QB);
  if (smem > 227 * 1024) return OSC_EUNSUPPORTED;
  const dim3 grid(static_cast<unsigned>((T + QB - 1) / QB), static_cast<unsigned>(heads), static_cast<unsigned>(B));
  if (small) {
    OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_psa_fused<16, 256>), static_cast<int>(smem)));
    return launch_pdl(ctx, k_psa_fused<16, 256>, grid, dim3(256), smem, "k_psa_fused", qkv, qkv_nstride, heads, T,
                      scale, out, out_nstride);
  }
  OSC_TRY(set_smem_attr(ctx, reinterpret_cast<const void*>(k_psa_fused<64, 512>), static_cast<int>(smem)));
  return launch_pdl(ctx, k_psa_fused<64, 512>, grid, dim3(512), smem, "k_psa_fused", qkv, qkv_nstride, heads, T,
                    scale, out, out_nstride);
}

// YOLO11's PSA attention (the exported MatMul -> Mul -> Softmax -> MatMul
// chain) on the tensor cores, per image b and head h of qkv [B][heads*(2kd+hd)][T]:
//   S = (q^T k) * scale        [T][T]   (batched 3xTF32 product, scale in the epilogue)
//   P = softmax_rows(S)                  (straight into the split operand)
//   out[b][h*hd + d][n] = sum_m v[d][m] P[n][m]
int psa_composed(osc_ctx* ctx, const float* qkv, long long qkv_nstride, int B, int heads, int kd, int hd, int T,
                 float scale, float* out, long long out_nstride) {
  const long long Z = static_cast<long long>(B) * heads;
  if (Z > 65535) return fail(OSC_EUNSUPPORTED, "psa attention: %lld image-heads (65535 at most)", Z);
  const int kq = static_cast<int>(round_up(static_cast<size_t>(kd), 4));
  const int kt = static_cast<int>(round_up(static_cast<size_t>(T), 4));
  const size_t q_bytes = round_up(static_cast<size_t>(Z) * T * kq * 4, 256);
  const size_t s_bytes = round_up(static_cast<size_t>(Z) * T * T * 4, 256);
  const size_t p_bytes = round_up(static_cast<size_t>(Z) * T * kt * 4, 256);
  const size_t v_bytes = round_up(static_cast<size_t>(Z) * hd * kt * 4, 256);
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, 4 * q_bytes + s_bytes + 2 * p_bytes + 2 * v_bytes, &buf));
  uint8_t* p = static_cast<uint8_t*>(buf);
  float* qhi = reinterpret_cast<float*>(p);
  float* qlo = reinterpret_cast<float*>(p + q_bytes);
  float* khi = reinterpret_cast<float*>(p + 2 * q_bytes);
  float* klo = reinterpret_cast<float*>(p + 3 * q_bytes);
  float* S = reinterpret_cast<float*>(p + 4 * q_bytes);
  float* phi = reinterpret_cast<float*>(p + 4 * q_bytes + s_bytes);
  float* plo = reinterpret_cast<float*>(p + 4 * q_bytes + s_bytes + p_bytes);
  float* vhi = reinterpret_cast<float*>(p + 4 * q_bytes + s_bytes + 2 * p_bytes);
  float* vlo = reinterpret_cast<float*>(p + 4 * q_bytes + s_bytes + 2 * p_bytes + v_bytes);
  const long long per = static_cast<long long>(2 * kd + hd) * T;  // one head's q, k, v channels
  const int nz = static_cast<int>(Z);
  // q^T and k^T as [z][token][channel]: the source is channel-major (tokens contiguous)
  OSC_TRY(gather_split(ctx, qkv, nz, heads, qkv_nstride, per, 1, T, T, kd, kq, qhi, qlo));
  OSC_TRY(gather_split(ctx, qkv + static_cast<long long>(kd) * T, nz, heads, qkv_nstride, per, 1, T, T, kd, kq, khi,
                       klo));
  {
    EpiAffine ep{scale, 0.0f, nullptr, 0, static_cast<long long>(heads) * T * T, static_cast<long long>(T) * T, heads,
                 T, 1, nullptr};
    OSC_TRY(gemm_batched(ctx, qhi, qlo, nz, T, kq, khi, klo, nz, T, nullptr, OSC_ACT_NONE, ep, S));
  }
  {
    const long long rows = Z * T;
    const int blocks = static_cast<int>(std::min<long long>((rows + 7) / 8, static_cast<long long>(ctx->num_sms) * 16));
    if (kt <= kSoftRegs * 32)
      OSC_TRY(launch_pdl(ctx, k_softmax_split_reg, dim3(blocks), dim3(256), 0, "k_softmax_split_reg", S, rows, T, kt,
                         phi, plo));
    else
      OSC_TRY(launch_pdl(ctx, k_softmax_split, dim3(blocks), dim3(256), 0, "k_softmax_split", S, rows, T, kt, phi,
                         plo));
  }
  // v as [z][channel][token] (already K-major)
  OSC_TRY(gather_split(ctx, qkv + 2LL * kd * T, nz, heads, qkv_nstride, per, T, 1, hd, T, kt, vhi, vlo));
  EpiAffine ep{1.0f, 0.0f, nullptr, 0, out_nstride, static_cast<long long>(hd) * T, heads, T, 1, nullptr};
  return gemm_batched(ctx, vhi, vlo, nz, hd, kt, phi, plo, nz, T, nullptr, OSC_ACT_NONE, ep, out);
}

}  // namespace osc

using namespace osc;

static int gemm_prepack(osc_ctx* ctx, const float* b, int k, int n, int b_layout, bool host, osc_gemm_weights** out) {
  if (out == nullptr) return fail(OSC_EINVAL, "osc_gemm_prepack_f32: out is null");
  *out = nullptr;
  OSC_TRY(enter(ctx));
  if (b == nullptr || k <= 0 || n <= 0) return fail(OSC_EINVAL, "osc_gemm_prepack_f32: bad B [%d, %d]", k, n);
  if (b_layout != 0 && b_layout != 1) return fail(OSC_EINVAL, "osc_gemm_prepack_f32: b_layout must be 0 or 1");
  if (fault_injected("prepack")) return fail(OSC_EFAULT_INJECTED, "injected failure (prepack)");
  auto* w = new osc_gemm_weights();
  w->device = ctx->device;
  w->k = k;
  w->n = n;
  w->kp = static_cast<int>(round_up(static_cast<size_t>(k), 4));
  const size_t bytes = static_cast<size_t>(n) * w->kp * sizeof(float);
  float* staged = nullptr;
  cudaError_t e = cudaMalloc(&w->hi, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&w->lo, bytes);
  if (e == cudaSuccess && host) {
    e = cudaMalloc(&staged, static_cast<size_t>(k) * n * sizeof(float));
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(staged, b, static_cast<size_t>(k) * n * sizeof(float), cudaMemcpyHostToDevice, ctx->stream);
    b = staged;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    cudaFree(w->hi);
    cudaFree(w->lo);
    cudaFree(staged);
    delete w;
    return fail(OSC_ENOMEM, "osc_gemm_prepack_f32: %s", cudaGetErrorString(e));
  }
  int st;
  if (b_layout == 0) {
    dim3 grid((n + 31) / 32, (w->kp + 31) / 32);
    prof_begin(ctx);
    k_pack_b_kn<<<grid, 256, 0, ctx->stream>>>(b, k, n, w->kp, w->hi, w->lo);
    st = check_launch(ctx, "k_pack_b_kn");
  } else {
    st = split_tf32(ctx, b, n, k, k, w->kp, w->hi, w->lo);
  }
  if (staged) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(staged);
  }
  if (st != OSC_OK) {
    osc_gemm_weights_free(w);
    return st;
  }
  *out = w;
  return OSC_OK;
}

extern "C" {

OSC_API int osc_gemm_prepack_f32(osc_ctx* ctx, const float* b, int k, int n, int b_layout, osc_gemm_weights** out) {
  return gemm_prepack(ctx, b, k, n, b_layout, false, out);
}

OSC_API int osc_gemm_prepack_f32_host(osc_ctx* ctx, const float* b, int k, int n, int b_layout,
                                      osc_gemm_weights** out) {
  return gemm_prepack(ctx, b, k, n, b_layout, true, out);
}

OSC_API int osc_gemm_weights_free(osc_gemm_weights* w) {
  if (w == nullptr) return OSC_OK;
  cudaSetDevice(w->device);
  cudaDeviceSynchronize();
  cudaFree(w->hi);
  cudaFree(w->lo);
  delete w;
  return OSC_OK;
}

OSC_API int osc_gemm_bias_f32(osc_ctx* ctx, const float* a, int m, int k, int lda, const osc_gemm_weights* w,
                              const float* col_bias, int act, float* c, int ldc) {
  OSC_TRY(enter(ctx));
  if (w == nullptr) return fail(OSC_EINVAL, "osc_gemm_bias_f32: null weights");
  if (m == 0 && k == w->k) return OSC_OK;  // empty batch: nothing to read or write
  if (a == nullptr || c == nullptr) return fail(OSC_EINVAL, "osc_gemm_bias_f32: null pointer");
  if (w->device != ctx->device) return fail(OSC_EINVAL, "osc_gemm_bias_f32: weights live on another device");
  if (k != w->k) return fail(OSC_EINVAL, "osc_gemm_bias_f32: A has k=%d, packed B has k=%d", k, w->k);
  if (m < 0) return fail(OSC_EINVAL, "osc_gemm_bias_f32: m=%d", m);
  if (act < OSC_ACT_NONE || act > OSC_ACT_SIGMOID) return fail(OSC_EINVAL, "osc_gemm_bias_f32: act=%d", act);
  if (lda == 0) lda = k;
  if (ldc == 0) ldc = w->n;
  if (lda < k || ldc < w->n) return fail(OSC_EINVAL, "osc_gemm_bias_f32: lda=%d ldc=%d too small", lda, ldc);
  if (m == 0) return OSC_OK;
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  return gemm_tf32x3(ctx, a, m, k, lda, w, col_bias, act, c, ldc);
}

// MatMul in two steps for activations that feed several MatMuls (the Q, K and
// V projections of one input): split A once into its K-major TF32 hi/lo
// operands, then multiply that split by each packed weight. Same kernels and
// results as osc_gemm_bias_f32, without re-splitting A per weight.
OSC_API int osc_gemm_split_a_f32(osc_ctx* ctx, const float* a, int m, int k, int lda, int kp, float* a_hi,
                                 float* a_lo) {
  OSC_TRY(enter(ctx));
  if (m < 0 || k <= 0) return fail(OSC_EINVAL, "osc_gemm_split_a_f32: m=%d k=%d", m, k);
  if (lda == 0) lda = k;
  if (lda < k) return fail(OSC_EINVAL, "osc_gemm_split_a_f32: lda=%d < k=%d", lda, k);
  if (kp != static_cast<int>(round_up(static_cast<size_t>(k), 4)))
    return fail(OSC_EINVAL, "osc_gemm_split_a_f32: kp=%d, expected k rounded up to 4 (%d)", kp,
                static_cast<int>(round_up(static_cast<size_t>(k), 4)));
  if (m == 0) return OSC_OK;
  if (a == nullptr || a_hi == nullptr || a_lo == nullptr) return fail(OSC_EINVAL, "osc_gemm_split_a_f32: null pointer");
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(a_hi) || !al16(a_lo)) return fail(OSC_EINVAL, "osc_gemm_split_a_f32: a_hi / a_lo not 16-byte aligned");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  return split_tf32(ctx, a, m, k, lda, kp, a_hi, a_lo);
}

OSC_API int osc_gemm_bias_presplit_f32(osc_ctx* ctx, const float* a_hi, const float* a_lo, int m, int kp,
                                       const osc_gemm_weights* w, const float* col_bias, int act, float* c, int ldc) {
  OSC_TRY(enter(ctx));
  if (w == nullptr) return fail(OSC_EINVAL, "osc_gemm_bias_presplit_f32: null weights");
  if (w->device != ctx->device)
    return fail(OSC_EINVAL, "osc_gemm_bias_presplit_f32: weights live on another device");
  if (kp != w->kp) return fail(OSC_EINVAL, "osc_gemm_bias_presplit_f32: A split with kp=%d, packed B has kp=%d", kp, w->kp);
  if (m < 0) return fail(OSC_EINVAL, "osc_gemm_bias_presplit_f32: m=%d", m);
  if (act < OSC_ACT_NONE || act > OSC_ACT_SIGMOID) return fail(OSC_EINVAL, "osc_gemm_bias_presplit_f32: act=%d", act);
  if (ldc == 0) ldc = w->n;
  if (ldc < w->n) return fail(OSC_EINVAL, "osc_gemm_bias_presplit_f32: ldc=%d too small", ldc);
  if (m == 0) return OSC_OK;
  if (a_hi == nullptr || a_lo == nullptr || c == nullptr)
    return fail(OSC_EINVAL, "osc_gemm_bias_presplit_f32: null pointer");
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(a_hi) || !al16(a_lo)) return fail(OSC_EINVAL, "osc_gemm_bias_presplit_f32: a_hi / a_lo not 16-byte aligned");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  return gemm_presplit(ctx, a_hi, a_lo, m, kp, w, col_bias, act, c, ldc);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// MatMul + bias without any device allocation (osc_gemm_bias_f32_noalloc).
//
// Some callers cannot allocate device memory while they run inference: a host
// that sizes all of its GPU memory once at start-up and must not grow it per
// request, or one serving several models from the same GPU, where a
// cudaMalloc / cudaFree can synchronise the whole device and stall every
// other stream at an unpredictable point. osc_gemm_bias_f32 takes its
// per-call temporaries (the TF32 hi/lo split of A) from the context's
// scratch arena, which grows with cudaMalloc; this variant takes them from a
// fixed array compiled into the library instead, so a call never allocates.
//
// The array below is in every GPU that loads the library, for the life of the
// process: 2 x kNoAllocMaxElems floats = 8 MiB. A call needs
// m * round_up(k, 4) <= kNoAllocMaxElems (e.g. 2048 x 512); larger calls are
// rejected with OSC_EINVAL. All calls on a device share the array and it keeps
// the previous call's contents: every element a call reads is first written by
// that call's split kernel (including the zero padding of K), so nothing needs
// clearing, but two calls whose kernels overlap on the GPU (different streams,
// or different contexts on the same device) race on it and must be serialised
// by the caller.
namespace osc {
namespace {

constexpr size_t kNoAllocMaxElems = size_t(1) << 20;  // per hi / lo part

__device__ __align__(256) float g_noalloc_scratch[2 * kNoAllocMaxElems];

// In host code g_noalloc_scratch names a host-side stand-in, not device
// memory; the device address is looked up once per device with that device
// current and cached here.
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64] = {};

int noalloc_scratch(int device, float** out) {
  if (device < 0 || device >= 64) return fail(OSC_EINVAL, "osc_gemm_bias_f32_noalloc: device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress (no-alloc scratch)");
    g_noalloc_ptr[device] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[device];
  return OSC_OK;
}

}  // namespace
}  // namespace osc

extern "C" {

OSC_API int osc_gemm_bias_f32_noalloc(osc_ctx* ctx, const float* a, int m, int k, int lda, const osc_gemm_weights* w,
                                      const float* col_bias, int act, float* c, int ldc) {
  OSC_TRY(enter(ctx));
  if (w == nullptr) return fail(OSC_EINVAL, "osc_gemm_bias_f32_noalloc: null weights");
  if (w->device != ctx->device) return fail(OSC_EINVAL, "osc_gemm_bias_f32_noalloc: weights live on another device");
  if (k != w->k) return fail(OSC_EINVAL, "osc_gemm_bias_f32_noalloc: A has k=%d, packed B has k=%d", k, w->k);
  if (m < 0) return fail(OSC_EINVAL, "osc_gemm_bias_f32_noalloc: m=%d", m);
  if (act < OSC_ACT_NONE || act > OSC_ACT_SIGMOID) return fail(OSC_EINVAL, "osc_gemm_bias_f32_noalloc: act=%d", act);
  if (lda == 0) lda = k;
  if (ldc == 0) ldc = w->n;
  if (lda < k || ldc < w->n) return fail(OSC_EINVAL, "osc_gemm_bias_f32_noalloc: lda=%d ldc=%d too small", lda, ldc);
  const size_t elems = static_cast<size_t>(m) * static_cast<size_t>(w->kp);
  if (elems > kNoAllocMaxElems)
    return fail(OSC_EINVAL,
                "osc_gemm_bias_f32_noalloc: m * round_up(k, 4) = %zu exceeds the fixed scratch limit of %zu "
                "elements (%d rows at k=%d); use osc_gemm_bias_f32 or split the rows",
                elems, kNoAllocMaxElems, static_cast<int>(kNoAllocMaxElems / static_cast<size_t>(w->kp)), k);
  if (m == 0) return OSC_OK;
  if (a == nullptr || c == nullptr) return fail(OSC_EINVAL, "osc_gemm_bias_f32_noalloc: null pointer");
  float* base = nullptr;
  OSC_TRY(noalloc_scratch(ctx->device, &base));
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  float* ahi = base;
  float* alo = base + kNoAllocMaxElems;
  // the same split kernel and GEMM routing as osc_gemm_bias_f32, with A's
  // hi/lo parts in the fixed array instead of the scratch arena
  OSC_TRY(split_tf32(ctx, a, m, k, lda, w->kp, ahi, alo));
  return gemm_presplit(ctx, ahi, alo, m, w->kp, w, col_bias, act, c, ldc);
}

OSC_API int osc_matmul_batched_f32(osc_ctx* ctx, int outer, int inner, int m, int k, int n, const float* a,
                                   long long a_outer, long long a_inner, long long a_row, long long a_col,
                                   const float* b, long long b_outer, long long b_inner, long long b_row,
                                   long long b_col, const float* col_bias, float* y) {
  OSC_TRY(enter(ctx));
  if (outer < 0 || inner <= 0 || m < 0 || k <= 0 || n <= 0)
    return fail(OSC_EINVAL, "osc_matmul_batched_f32: bad shape outer=%d inner=%d [%d,%d]x[%d,%d]", outer, inner, m,
                k, k, n);
  const long long batches = static_cast<long long>(outer) * inner;
  if (batches == 0 || m == 0) return OSC_OK;
  if (a == nullptr || b == nullptr || y == nullptr) return fail(OSC_EINVAL, "osc_matmul_batched_f32: null pointer");
  if (batches > 65535) return fail(OSC_EUNSUPPORTED, "osc_matmul_batched_f32: %lld batches", batches);
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, batched_work_bytes(batches, m, k, n), &buf));
  EpiAffine ep{1.0f, 0.0f, nullptr, 0, static_cast<long long>(inner) * m * n, static_cast<long long>(m) * n, inner, n,
               1, nullptr};
  return batched_strided(ctx, outer, inner, m, k, n, a, a_outer, a_inner, a_row, a_col, b, b_outer, b_inner, b_row,
                         b_col, col_bias, ep, y, buf);
}

OSC_API int osc_gemm_onnx_f32(osc_ctx* ctx, const float* a, int trans_a, int m, int k, const osc_gemm_weights* w,
                              const float* b, int trans_b, int n, float alpha, float beta, const float* c,
                              long long c_len, float* y) {
  OSC_TRY(enter(ctx));
  if (m < 0 || k <= 0) return fail(OSC_EINVAL, "osc_gemm_onnx_f32: bad shape m=%d k=%d", m, k);
  if (w != nullptr) {
    if (w->k != k) return fail(OSC_EINVAL, "osc_gemm_onnx_f32: A has k=%d, packed B has k=%d", k, w->k);
    if (w->device != ctx->device) return fail(OSC_EINVAL, "osc_gemm_onnx_f32: weights live on another device");
    n = w->n;
  } else if (b == nullptr || n <= 0) {
    return fail(OSC_EINVAL, "osc_gemm_onnx_f32: neither packed weights nor B");
  }
  if (c_len < 0) return fail(OSC_EINVAL, "osc_gemm_onnx_f32: c_len=%lld", c_len);
  if (m == 0) return OSC_OK;
  if (a == nullptr || y == nullptr || (c_len > 0 && c == nullptr))
    return fail(OSC_EINVAL, "osc_gemm_onnx_f32: null pointer");
  if (fault_injected("launch")) return fail(OSC_EFAULT_INJECTED, "injected failure (launch)");
  const int kp = w != nullptr ? w->kp : static_cast<int>(round_up(static_cast<size_t>(k), 4));
  const size_t abytes = round_up(static_cast<size_t>(m) * kp * sizeof(float), 256);
  const size_t bbytes = w != nullptr ? 0 : round_up(static_cast<size_t>(n) * kp * sizeof(float), 256);
  void* buf = nullptr;
  OSC_TRY(scratch(ctx, 2 * abytes + 2 * bbytes, &buf));
  uint8_t* p = static_cast<uint8_t*>(buf);
  float* ahi = reinterpret_cast<float*>(p);
  float* alo = reinterpret_cast<float*>(p + abytes);
  // A stored [m][k] (or [k][m] with trans_a)
  OSC_TRY(gather_split(ctx, a, 1, 1, 0, 0, trans_a ? 1 : k, trans_a ? m : 1, m, k, kp, ahi, alo));
  const float* bhi = w != nullptr ? w->hi : reinterpret_cast<float*>(p + 2 * abytes);
  const float* blo = w != nullptr ? w->lo : reinterpret_cast<float*>(p + 2 * abytes + bbytes);
  if (w == nullptr)  // B stored [k][n] (or [n][k] with trans_b) -> K-major [n][kp]
    OSC_TRY(gather_split(ctx, b, 1, 1, 0, 0, trans_b ? k : 1, trans_b ? 1 : n, n, k, kp, const_cast<float*>(bhi),
                         const_cast<float*>(blo)));
  EpiAffine ep{alpha, beta, c, c_len, 0, 0, 1, n, 0, nullptr};
  return gemm_batched(ctx, ahi, alo, 1, m, kp, bhi, blo, 1, n, nullptr, OSC_ACT_NONE, ep, y);
}

}  // extern "C"
