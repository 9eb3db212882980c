// tf32x3_core.cuh — the shared main loop of the FP32-accurate tensor-core
// kernels (GEMM and implicit-GEMM convolution): a TMA -> shared memory ring,
// 3xTF32 tcgen05 MMAs into a double-buffered TMEM accumulator, and epilogue
// warps that drain the accumulator into FP32 registers every KC k-blocks.
//
// Why chunked draining: the tensor core adds each MMA's products into the
// TMEM accumulator with truncation, so the error of one long accumulation
// grows linearly with K (measured on B200: 7e-5 relative at K=512 with one
// accumulator). Restarting the TMEM accumulator every KC*32 of K and summing
// the chunk results with round-to-nearest FP32 adds in registers keeps the
// error at the level of one short chunk.
//
// Roles (one elected thread per role warp):
//   warp 0           producer: issues the kernel-specific TMA loads per k-block
//   warp 1           TMEM owner and MMA issuer (3 MMAs per 8-wide K step)
//   warps 2..        epilogue: EPI_WARPS warps, warp w drains TMEM lanes
//                    32*(w%4).. (tile rows), columns 128*((w-2)/4)..+128
#pragma once

#include "sm100.cuh"

namespace osc {

constexpr int kBM = 128;  // tile rows (TMEM lanes)
constexpr int kBK = 32;   // K per stage: one 128-byte swizzle row of FP32

template <int BN_, int STAGES_, int KC_>
struct Tf32x3Cfg {
  static constexpr int BN = BN_;
  static constexpr int STAGES = STAGES_;
  static constexpr int KC = KC_;                 // k-blocks per TMEM chunk
  static constexpr int EPI_WARPS = 4 * (BN / 128);
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int A_BYTES = kBM * kBK * 4;  // one operand part (hi or lo)
  static constexpr int B_BYTES = BN * kBK * 4;
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  // The epilogue's row staging (gemm_stage: kBM x (BN + 4) floats + BN
  // biases) reuses the ring; a one-stage ring is smaller than that, so the
  // region is the larger of the two.
  static constexpr int STAGING_BYTES = kBM * (BN + 4) * 4 + BN * 4;
  static constexpr int RING_BYTES =
      TILE_BYTES >= STAGING_BYTES ? TILE_BYTES : (STAGING_BYTES + 1023) / 1024 * 1024;
  // Two accumulator buffers; a one-stage configuration serves only GEMMs of
  // at most KC k-blocks (one chunk), so it holds one.
  static constexpr int TMEM_COLS = (STAGES == 1 ? 1 : 2) * BN;
  // ring | barriers (256 bytes) | column biases of the tile (BN floats)
  static constexpr int SMEM_BYTES = RING_BYTES + 1024 + 256 + BN * 4;
  static_assert(BN == 128 || BN == 256, "BN");
  static_assert(STAGES <= 8, "stages");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

struct PipeBarriers {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_slot;
  int abort_flag;
};

template <class Cfg>
__device__ __forceinline__ uint8_t* tiles_base(uint8_t* smem_raw) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
}

template <class Cfg>
__device__ __forceinline__ PipeBarriers* barriers(uint8_t* tiles) {
  return reinterpret_cast<PipeBarriers*>(tiles + Cfg::RING_BYTES);
}

// Barrier init + TMEM allocation; every thread of the CTA calls it.
template <class Cfg>
__device__ __forceinline__ uint32_t pipe_setup(PipeBarriers* pb) {
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&pb->full[s], 1);
      mbar_init(&pb->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pb->acc_full[b], 1);
      mbar_init(&pb->acc_empty[b], Cfg::EPI_WARPS);
    }
    pb->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&pb->tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return pb->tmem_slot;
}

template <class Cfg>
__device__ __forceinline__ void pipe_teardown(PipeBarriers* pb, uint32_t tmem) {
  tc_fence_before();
  __syncthreads();
  if ((threadIdx.x >> 5) == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// Producer skeleton: `issue(kb, stage_ptr, bar)` enqueues the TMA loads of
// k-block kb (`tx` bytes in total, STAGE_BYTES unless the A boxes are shorter
// than kBM rows) on `bar`. Run by one thread.
template <class Cfg, class Issue>
__device__ __forceinline__ void producer_loop(uint8_t* tiles, PipeBarriers* pb, int num_kb, int* err, Issue issue,
                                              uint32_t tx = Cfg::STAGE_BYTES) {
  int issued = 0;
  for (int kb = 0; kb < num_kb; ++kb) {
    const int s = kb % Cfg::STAGES;
    const uint32_t ph = (kb / Cfg::STAGES) & 1u;
    if (!mbar_wait(&pb->empty[s], ph ^ 1u, &pb->abort_flag, err)) break;
    mbar_arrive_expect_tx(&pb->full[s], tx);
    issue(kb, tiles + s * Cfg::STAGE_BYTES, &pb->full[s]);
    issued = kb + 1;
  }
  if (pb->abort_flag) {
    // Error path: let copies already in flight land before the CTA exits.
    const int first = issued > Cfg::STAGES ? issued - Cfg::STAGES : 0;
    for (int kb = first; kb < issued; ++kb) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&pb->full[kb % Cfg::STAGES], (kb / Cfg::STAGES) & 1u) &&
             globaltimer_ns() - t0 < 50ull * 1000ull * 1000ull) {
      }
    }
  }
}

// MMA issuer: for each chunk of KC k-blocks, wait for the accumulator buffer
// to be drained, then 3 MMAs per 8-wide K step (hi*hi, hi*lo, lo*hi); each
// stage is released by tcgen05.commit, each finished chunk is signalled on
// acc_full. Stage layout: A hi | A lo | B hi | B lo.
// STACKED (A of at most 64 rows): the A hi region holds [A hi; A lo] as one
// 128-row operand, and 2 MMAs per K step (stack * B hi, stack * B lo) leave
// A hi * B in D rows 0-63 and A lo * B in rows 64-127 (the lo * lo product
// included), which the epilogue adds: 8 MMAs per k-block instead of 12, an
// MMA of 64 rows costing about as much as one of 128. Run by one thread.
template <class Cfg, bool STACKED = false>
__device__ __forceinline__ void mma_loop(uint8_t* tiles, PipeBarriers* pb, uint32_t tmem, int num_kb, int* err) {
  constexpr uint32_t idesc = idesc_tf32(kBM, Cfg::BN);
  const int nchunks = (num_kb + Cfg::KC - 1) / Cfg::KC;
  int kb = 0;
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    if (!mbar_wait(&pb->acc_empty[buf], ((c >> 1) & 1u) ^ 1u, &pb->abort_flag, err)) return;
    tc_fence_after();
    const uint32_t d = tmem + static_cast<uint32_t>(buf * Cfg::BN);
    const int kb_end = min(num_kb, kb + Cfg::KC);
    uint32_t acc = 0u;
    for (; kb < kb_end; ++kb) {
      const int s = kb % Cfg::STAGES;
      const uint32_t ph = (kb / Cfg::STAGES) & 1u;
      if (!mbar_wait(&pb->full[s], ph, &pb->abort_flag, err)) return;
      tc_fence_after();
      const uint32_t base = smem_addr(tiles + s * Cfg::STAGE_BYTES);
      const uint64_t dAh = sdesc_kmajor_sw128(base);
      const uint64_t dAl = sdesc_kmajor_sw128(base + Cfg::A_BYTES);
      const uint64_t dBh = sdesc_kmajor_sw128(base + 2 * Cfg::A_BYTES);
      const uint64_t dBl = sdesc_kmajor_sw128(base + 2 * Cfg::A_BYTES + Cfg::B_BYTES);
#pragma unroll
      for (int kk = 0; kk < kBK / 8; ++kk) {
        const uint64_t off = static_cast<uint64_t>(kk * 2);  // +32 bytes per 8-wide K step
        mma_tf32(d, dAh + off, dBh + off, idesc, acc);
        acc = 1u;
        mma_tf32(d, dAh + off, dBl + off, idesc, 1u);
        if (!STACKED) mma_tf32(d, dAl + off, dBh + off, idesc, 1u);
      }
      mma_commit(&pb->empty[s]);
    }
    mma_commit(&pb->acc_full[buf]);
  }
}

// Epilogue drain: accumulates this thread's 128 columns of its tile row over
// all chunks into acc[] (round-to-nearest FP32 adds). Returns false if a wait
// gave up. All lanes of the warp call it.
template <class Cfg>
__device__ __forceinline__ bool drain_loop(PipeBarriers* pb, uint32_t tmem, int num_kb, float (&acc)[128],
                                           int* err) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q = warp & 3;
  const int half = (warp - 2) >> 2;
  const int nchunks = (num_kb + Cfg::KC - 1) / Cfg::KC;
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    bool ok = mbar_wait(&pb->acc_full[buf], (c >> 1) & 1u, &pb->abort_flag, err);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) return false;
    tc_fence_after();
    const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) +
                          static_cast<uint32_t>(buf * Cfg::BN + half * 128);
#pragma unroll
    for (int g = 0; g < 8; g += 2) {
      uint32_t r0[16], r1[16];
      tmem_ld16(base + g * 16, r0);
      tmem_ld16(base + (g + 1) * 16, r1);
      tmem_wait_ld();
      if (c == 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc[g * 16 + j] = __uint_as_float(r0[j]);
          acc[(g + 1) * 16 + j] = __uint_as_float(r1[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc[g * 16 + j] = __fadd_rn(acc[g * 16 + j], __uint_as_float(r0[j]));
          acc[(g + 1) * 16 + j] = __fadd_rn(acc[(g + 1) * 16 + j], __uint_as_float(r1[j]));
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&pb->acc_empty[buf]);
  }
  return true;
}

// Output staging: after the last chunk every MMA has completed, so the
// operand ring is free and holds the 128 x BN tile at a pitch of BN+4 floats
// (the +4 keeps a quarter-warp's float4 stores to 8 different rows on 8
// different bank groups). Each epilogue thread writes its row's 128 columns;
// after epi_sync() the warps copy whole rows out with coalesced stores.
template <class Cfg>
__device__ __forceinline__ float* stage_tile(uint8_t* tiles, const float (&acc)[128]) {
  constexpr int kPitch = Cfg::BN + 4;
  float* stage = reinterpret_cast<float*>(tiles);
  const int warp = threadIdx.x >> 5;
  const int row = (warp & 3) * 32 + (threadIdx.x & 31);
  float* dst = stage + row * kPitch + ((warp - 2) >> 2) * 128;
#pragma unroll
  for (int j = 0; j < 128; j += 4)
    *reinterpret_cast<float4*>(dst + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
  return stage;
}

// Barrier among the epilogue warps only (named barrier 1).
template <class Cfg>
__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(Cfg::EPI_WARPS * 32) : "memory");
}

static_assert(kBM * (256 + 4) * 4 <= Tf32x3Cfg<256, 2, 2>::TILE_BYTES, "staging fits the operand ring");

// ------------------------------------------------------------------ CTA pairs
// The same main loop on a cluster of two CTAs with tcgen05 cta_group::2: the
// pair computes a 256 x BN tile, each CTA loads its own 128 rows of A and
// half of B's BN columns (per k-block 2*16 KB of A + 2*(BN/2)*128 B of B
// instead of the single-CTA 2*16 KB + 2*BN*128 B), and the even CTA issues
// M = 256 MMAs that read both CTAs' shared memory and write both CTAs' TMEM.
// Barriers: both CTAs' TMA loads count their bytes on the even CTA's `full`
// barrier; the even CTA's MMA thread commits to `empty` and `acc_full` of both
// CTAs (two commits, no multicast); both CTAs' epilogue warps release a
// drained accumulator on the even CTA's `acc_empty`.
template <int BN_, int STAGES_, int KC_>
struct Tf32x3PairCfg {
  static constexpr int BN = BN_;                 // output columns of the pair tile (both CTAs)
  static constexpr int STAGES = STAGES_;
  static constexpr int KC = KC_;
  static constexpr int EPI_WARPS = 4 * (BN / 128);
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int A_BYTES = kBM * kBK * 4;
  static constexpr int B_BYTES = (BN / 2) * kBK * 4;  // this CTA's half of B
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int TILE_BYTES = STAGES * STAGE_BYTES;
  static constexpr int RING_BYTES = TILE_BYTES;  // the staging fits the ring (asserted below)
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = TILE_BYTES + 1024 + 256 + BN * 4;  // + the tile's column biases
  static_assert(BN == 128 || BN == 256, "BN");
  static_assert(STAGES <= 8, "stages");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(kBM * (BN + 4) * 4 + BN * 4 <= TILE_BYTES, "staging + bias fit the operand ring");
};

struct PairBarriers {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t exit_bar;
  uint32_t tmem_slot;
  int abort_flag;
  int no_abort;  // always 0: lets the exit handshake wait its full bound
};

template <class Cfg>
__device__ __forceinline__ PairBarriers* pair_barriers(uint8_t* tiles) {
  return reinterpret_cast<PairBarriers*>(tiles + Cfg::TILE_BYTES);
}

// Barrier init + paired TMEM allocation + a cluster-wide sync (so no remote
// arrival or complete_tx can reach a barrier before it is initialised).
template <class Cfg>
__device__ __forceinline__ uint32_t pipe_setup_pair(PairBarriers* pb) {
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(&pb->full[s], 1);
      mbar_init(&pb->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pb->acc_full[b], 1);
      mbar_init(&pb->acc_empty[b], 2 * Cfg::EPI_WARPS);
    }
    mbar_init(&pb->exit_bar, 1);
    pb->abort_flag = 0;
    pb->no_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&pb->tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  return pb->tmem_slot;
}

// Exit handshake: a CTA leaves only after its peer has finished every access
// to it (the peer's MMAs read this CTA's shared memory and write its TMEM,
// its commits arrive on this CTA's barriers). Bounded; after a timeout both
// CTAs first let any copy still in flight land.
template <class Cfg>
__device__ __forceinline__ void pipe_teardown_pair(PairBarriers* pb, uint32_t tmem, uint32_t rank, int* err) {
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (pb->abort_flag) {
      const uint64_t t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 50ull * 1000ull * 1000ull) {
      }
    }
    mbar_arrive_cluster(mapa_shared(&pb->exit_bar, rank ^ 1u));
    mbar_wait(&pb->exit_bar, 0, &pb->no_abort, err);
  }
  __syncthreads();
  if ((threadIdx.x >> 5) == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
  }
}

// Producer (both CTAs): `issue(kb, stage_ptr, leader_full_bar)` enqueues this
// CTA's TMA loads of k-block kb (STAGE_BYTES) counted on the even CTA's barrier.
template <class Cfg, class Issue>
__device__ __forceinline__ void producer_loop_pair(uint8_t* tiles, PairBarriers* pb, int num_kb, uint32_t rank,
                                                   int* err, Issue issue) {
  const uint32_t full0 = mapa_shared(&pb->full[0], 0);
  for (int kb = 0; kb < num_kb; ++kb) {
    const int s = kb % Cfg::STAGES;
    const uint32_t ph = (kb / Cfg::STAGES) & 1u;
    if (!mbar_wait(&pb->empty[s], ph ^ 1u, &pb->abort_flag, err)) break;
    if (rank == 0) mbar_arrive_expect_tx(&pb->full[s], 2 * Cfg::STAGE_BYTES);
    issue(kb, tiles + s * Cfg::STAGE_BYTES, full0 + static_cast<uint32_t>(s * 8));
  }
}

// MMA issuer of the even CTA: M = 256 (both CTAs' A rows), N = BN (both CTAs'
// B halves); each stage and each finished chunk is signalled to both CTAs.
template <class Cfg>
__device__ __forceinline__ void mma_loop_pair(uint8_t* tiles, PairBarriers* pb, uint32_t tmem, int num_kb, int* err) {
  constexpr uint32_t idesc = idesc_tf32(2 * kBM, Cfg::BN);
  const uint32_t empty_own = mapa_shared(&pb->empty[0], 0), empty_peer = mapa_shared(&pb->empty[0], 1);
  const uint32_t accf_own = mapa_shared(&pb->acc_full[0], 0), accf_peer = mapa_shared(&pb->acc_full[0], 1);
  const int nchunks = (num_kb + Cfg::KC - 1) / Cfg::KC;
  int kb = 0;
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    if (!mbar_wait(&pb->acc_empty[buf], ((c >> 1) & 1u) ^ 1u, &pb->abort_flag, err)) return;
    tc_fence_after();
    const uint32_t d = tmem + static_cast<uint32_t>(buf * Cfg::BN);
    const int kb_end = min(num_kb, kb + Cfg::KC);
    uint32_t acc = 0u;
    for (; kb < kb_end; ++kb) {
      const int s = kb % Cfg::STAGES;
      const uint32_t ph = (kb / Cfg::STAGES) & 1u;
      if (!mbar_wait(&pb->full[s], ph, &pb->abort_flag, err)) return;
      tc_fence_after();
      const uint32_t base = smem_addr(tiles + s * Cfg::STAGE_BYTES);
      const uint64_t dAh = sdesc_kmajor_sw128(base);
      const uint64_t dAl = sdesc_kmajor_sw128(base + Cfg::A_BYTES);
      const uint64_t dBh = sdesc_kmajor_sw128(base + 2 * Cfg::A_BYTES);
      const uint64_t dBl = sdesc_kmajor_sw128(base + 2 * Cfg::A_BYTES + Cfg::B_BYTES);
#pragma unroll
      for (int kk = 0; kk < kBK / 8; ++kk) {
        const uint64_t off = static_cast<uint64_t>(kk * 2);
        mma_tf32_pair(d, dAh + off, dBh + off, idesc, acc);
        acc = 1u;
        mma_tf32_pair(d, dAh + off, dBl + off, idesc, 1u);
        mma_tf32_pair(d, dAl + off, dBh + off, idesc, 1u);
      }
      mma_commit_pair(empty_own + static_cast<uint32_t>(s * 8));
      mma_commit_pair(empty_peer + static_cast<uint32_t>(s * 8));
    }
    mma_commit_pair(accf_own + static_cast<uint32_t>(buf * 8));
    mma_commit_pair(accf_peer + static_cast<uint32_t>(buf * 8));
  }
}

// Epilogue drain of a pair CTA: as drain_loop, releasing on the even CTA's acc_empty.
template <class Cfg>
__device__ __forceinline__ bool drain_loop_pair(PairBarriers* pb, uint32_t tmem, int num_kb, float (&acc)[128],
                                                int* err) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q = warp & 3;
  const int half = (warp - 2) >> 2;
  const int nchunks = (num_kb + Cfg::KC - 1) / Cfg::KC;
  const uint32_t acce0 = mapa_shared(&pb->acc_empty[0], 0);
  for (int c = 0; c < nchunks; ++c) {
    const int buf = c & 1;
    bool ok = mbar_wait(&pb->acc_full[buf], (c >> 1) & 1u, &pb->abort_flag, err);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) return false;
    tc_fence_after();
    const uint32_t base = tmem + (static_cast<uint32_t>(q * 32) << 16) +
                          static_cast<uint32_t>(buf * Cfg::BN + half * 128);
#pragma unroll
    for (int g = 0; g < 8; g += 2) {
      uint32_t r0[16], r1[16];
      tmem_ld16(base + g * 16, r0);
      tmem_ld16(base + (g + 1) * 16, r1);
      tmem_wait_ld();
      if (c == 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc[g * 16 + j] = __uint_as_float(r0[j]);
          acc[(g + 1) * 16 + j] = __uint_as_float(r1[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          acc[g * 16 + j] = __fadd_rn(acc[g * 16 + j], __uint_as_float(r0[j]));
          acc[(g + 1) * 16 + j] = __fadd_rn(acc[(g + 1) * 16 + j], __uint_as_float(r1[j]));
        }
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(acce0 + static_cast<uint32_t>(buf * 8));
  }
  return true;
}

}  // namespace osc
