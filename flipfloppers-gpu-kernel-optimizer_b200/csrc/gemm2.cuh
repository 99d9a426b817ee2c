// CTA-pair (2-SM) tcgen05 projection GEMM: the same contract and epilogues as
// k_gemm_tn, for large projections whose speed is bounded by how fast one SM
// can pull operand tiles from L2.
//
// A cluster of two CTAs computes one 256x256 output tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16 per instruction): each CTA
// stages its own 128 rows of A and 128 rows (half the N range) of W per 64-wide
// K slice, and the instruction issued by the leader CTA (cluster rank 0) reads
// both CTAs' shared memory and writes each CTA's 128 output rows into that
// CTA's tensor memory.  Per SM and K slice that is 32 KB of operands for the
// same tensor work the one-SM 128x256 tile needs 48 KB for.
//
//   warp 0, both CTAs   TMA producer for the CTA's half of each stage; the loads
//                       use .cta_group::2 and complete on the leader's `full`
//                       barrier (the leader announces both halves' bytes); a
//                       stage is refilled when the leader's MMAs that read it
//                       have completed (multicast commit to both CTAs' `empty`).
//   warp 1, leader      TMEM double buffer (2 x 256 columns, allocated as a
//                       pair) and the MMA issuer; accumulator-full is committed
//                       to both CTAs.
//   warps 2.., both     epilogue of the CTA's 128 rows (gemm_epilogue_cols;
//                       8 or 16 warps); each warp arrives on the leader's
//                       accumulator-empty barrier.
// No TMA load uses multicast: every CTA loads only its own operand halves.
// Every wait is bounded (ptx.cuh); the CTAs meet at a cluster barrier before
// the pair frees its tensor memory and exits, so no remote arrival or copy
// targets a CTA that has left.
#pragma once

#include "gemm.cuh"

namespace b200 {

// tiled load into this CTA's shared memory, completing on an mbarrier of either
// CTA of the pair (shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// arrive (once) on the barrier at this shared::cta offset in every CTA of
// `cta_mask` when the leader's prior tcgen05 ops are complete
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               ::"r"(smem_u32(bar)), "h"(cta_mask)
               : "memory");
}
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}\n"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

template <int STAGES, int EW>
struct Gemm2Smem {
  static constexpr int A_BYTES = 128 * 64 * 2;  // this CTA's 128 rows of A
  static constexpr int B_BYTES = 128 * 64 * 2;  // this CTA's 128 rows (N half) of W
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STG_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = STG_OFF + EW * 4096;  // two 2 KB staging slots per epilogue warp
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;
};

// EW epilogue warps per CTA: 8 (two per SMSP) with a 6-stage operand ring, or
// 16 (four per SMSP, each taking 64 of the tile's columns) with 4 stages for
// short K, where the mainloop is a few K slices and the epilogue alone sets the
// speed (its warps are latency-bound one by one).
__host__ __device__ constexpr int gemm2_stages(int ew) { return ew == 16 ? 4 : 6; }
__host__ __device__ constexpr int gemm2_threads(int ew) { return 64 + 32 * ew; }

template <int EPI, int EW>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gemm2_threads(EW), 1)
    k_gemm2_tn(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
               const __grid_constant__ CUtensorMap tmO, const GemmParams p) {
  static_assert(EW == 8 || EW == 16, "8 or 16 epilogue warps");
  constexpr int STAGES = gemm2_stages(EW);
  using L = Gemm2Smem<STAGES, EW>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2] (used in the leader)
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cid = static_cast<int>(blockIdx.x) >> 1, ncl = static_cast<int>(gridDim.x) >> 1;
  const int mt = (p.M + 255) / 256, ntl = (p.N + 255) / 256;
  const int ntiles = mt * ntl;
  const int my_tiles = (ntiles - cid + ncl - 1) / ncl;
  const int nk = (p.K + 63) / 64;
  constexpr uint32_t TMEM_COLS = 512;  // two 256-column accumulators

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // the leader's expect_tx arrival (+ both halves' bytes)
      mbar_init(&empty[s], 1);  // the leader's multicast commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * EW);  // EW epilogue warps in each of the two CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();  // thread 0 rejoins warp 0: barrier.cluster is warp-aligned
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_sync();  // the previous kernel's outputs are complete from here on

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmW);
      int it = 0;
      bool ok = true;
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int t = cid + i * ncl;
        const int m0 = (t / ntl) * 256, n0 = (t % ntl) * 256;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, abort_flag, DERR_WAIT_SLOT)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * L::STAGE_BYTES;
          if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * L::STAGE_BYTES);
          const uint32_t fbar = mapa_shared(smem_u32(&full[s]), 0);
          tma_load_2d_pair(st, &tmA, fbar, kb * 64, p.a_row0 + m0 + 128 * static_cast<int>(rank));
          tma_load_2d_pair(st + L::A_BYTES, &tmW, fbar, kb * 64, n0 + 128 * static_cast<int>(rank));
        }
      }
      if (*abort_flag && rank == 0)
        for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j) mbar_wait_drain(&full[j % STAGES], (j / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_f16(256, 256, false);
      int it = 0;
      bool ok = true;
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int b = i & 1;
        // both CTAs' epilogues must have drained this accumulator buffer (tile i-2)
        if (i >= 2 && !mbar_wait(&acc_empty[b], ((i >> 1) - 1) & 1, abort_flag, DERR_WAIT_MMA)) break;
        tc_fence_after();
        const uint32_t dcol = tmem + b * 256;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1, abort_flag, DERR_WAIT_TMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * L::STAGE_BYTES);
          const uint32_t b_addr = a_addr + L::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_ss_pair(dcol, make_sdesc(a_addr + kk * 32, 16, 1024, UMMA_SW128),
                             make_sdesc(b_addr + kk * 32, 16, 1024, UMMA_SW128), idesc, (kb | kk) != 0 ? 1u : 0u);
          tc_commit_pair(&empty[s], 0x3);
        }
        if (!ok) break;
        tc_commit_pair(&acc_full[b], 0x3);
      }
      if (*abort_flag) {
        tc_commit_pair(drain, 0x1);
        mbar_wait_drain(drain, 0);
      }
    }
  } else {
    // epilogue warps 2..EW+1: this CTA's 128 rows of each 256x256 tile; the EW/4 warps
    // of TMEM lane quadrant q split its 256 columns
    constexpr int CWE = 256 / (EW / 4);
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;
    uint8_t* stg = smem + L::STG_OFF + (warp - 2) * 4096;
    const uint32_t empty_leader0 = mapa_shared(smem_u32(&acc_empty[0]), 0);
    if (lane == 0) tma_prefetch_desc(&tmO);
    int gc = 0;
    for (int i = 0; i < my_tiles; ++i) {
      const int b = i & 1;
      const int t = cid + i * ncl;
      const int m0 = (t / ntl) * 256 + 128 * static_cast<int>(rank), n0 = (t % ntl) * 256;
      const bool ok = mbar_wait_warp(&acc_full[b], (i >> 1) & 1, abort_flag, DERR_WAIT_MMA);
      if (!ok || *abort_flag) break;
      tc_fence_after();
      gemm_epilogue_cols<EPI>(&tmO, p, tmem + (static_cast<uint32_t>(q * 32) << 16) + b * 256, part * CWE,
                              (part + 1) * CWE, n0, m0 + q * 32, stg, gc, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(empty_leader0 + b * 8);
    }
    if (lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncwarp();  // lane-0 roles rejoin their warp: bar.sync is warp-aligned
  __syncthreads();
  cluster_sync_all();  // no remote arrival or copy is still headed for either CTA
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

}  // namespace b200
