// tcgen05 projection GEMM with fused epilogues:
//   out[M,N] = epi( A[M,K] . W[N,K]^T + bias[N] (+ resid[M,N]) )
// A, W fp16 row-major (K contiguous, "K-major" for UMMA); fp32 accumulation in
// TMEM; fp32 bias.  Epilogues:
//   EPI_BIAS_F16       fp16 out            (QKV projection, reference TTB:1303)
//   EPI_BIAS_GELU_F16  fp16 gelu_as(.)    (ffn_in + exact GELU, TTB:1350-1354)
//   EPI_BIAS_RESID_F32 fp32 out = resid+.  (out_proj / ffn_out + residual,
//                                           TTB:1333-1339, 1368-1369)
//   EPI_BIAS_F32       fp32 out            (row-parallel partial sums before
//                                           the tensor-parallel all-reduce)
// It replaces the reference's mma.sync GEMM `ws_gemm_kernel`
// (csrc/g4_4_warpspec_gemm.cu:273-795) with a Blackwell design:
//   warp 0     TMA producer: 64-wide K slices of A and W, SWIZZLE_128B, into a
//              STAGES-deep shared-memory ring (full/empty mbarriers);
//   warp 1     allocates TMEM and issues tcgen05.mma (one elected lane),
//              committing each stage back to the producer;
//   warps 2-5  epilogue: tcgen05.ld of the 128xBN fp32 tile (one row per
//              thread), bias/GELU/residual, vector stores.
// One 128xBN output tile per CTA.
#pragma once

#include "ptx.cuh"

namespace b200 {

enum GemmEpilogue : int { EPI_BIAS_F16 = 0, EPI_BIAS_GELU_F16 = 1, EPI_BIAS_RESID_F32 = 2, EPI_BIAS_F32 = 3 };

struct GemmParams {
  int M, N, K;
  int a_row0;            // first row of A addressed by the tensor map (row offset of this call)
  const float* bias;     // [N] fp32, may be null
  const float* resid;    // [M, ld_resid] fp32 (EPI_BIAS_RESID_F32)
  int64_t ld_resid;
  void* out;             // [M, ld_out], fp16 or fp32
  int64_t ld_out;
};

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int A_BYTES = 128 * 64 * 2;
  static constexpr int B_BYTES = BN * 64 * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_OFF = STAGES * STAGE_BYTES;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;  // barriers + 1 KB alignment slack
};

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(192, 1)
    k_gemm_tn(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, const GemmParams p) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * 128, n0 = blockIdx.x * BN;
  const int nk = (p.K + 63) / 64;
  constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmW);
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        if (kb >= STAGES && !mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1, abort_flag, DERR_WAIT_SLOT)) break;
        uint8_t* st = smem + s * L::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
        tma_load_2d(st, &tmA, &full[s], kb * 64, p.a_row0 + m0);
        tma_load_2d(st + L::A_BYTES, &tmW, &full[s], kb * 64, n0);
        issued = kb + 1;
      }
      if (*abort_flag) {
        // drain: every issued stage must land before the CTA's smem is released
        for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb)
          mbar_wait_drain(&full[kb % STAGES], (kb / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(128, BN, false);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        if (!mbar_wait(&full[s], (kb / STAGES) & 1, abort_flag, DERR_WAIT_TMA)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * L::STAGE_BYTES);
        const uint32_t b_addr = a_addr + L::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = make_sdesc(a_addr + kk * 32, 16, 1024, UMMA_SW128);
          const uint64_t bd = make_sdesc(b_addr + kk * 32, 16, 1024, UMMA_SW128);
          umma_f16_ss(tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(accf);  // also issued on abort: teardown waits on it before freeing TMEM
      if (*abort_flag) mbar_wait_drain(accf, 0);
    }
  } else {
    // epilogue warps 2..5: warp%4 selects the TMEM lane quadrant it may access
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    const bool ok = mbar_wait_warp(accf, 0, abort_flag, DERR_WAIT_MMA);
    if (ok && !*abort_flag) {
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c, v);
        const int col = n0 + c;
        if (row < p.M && col < p.N) {
          if (p.bias != nullptr) {
            const float4* b4 = reinterpret_cast<const float4*>(p.bias + col);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 b = __ldg(b4 + i);
              v[4 * i + 0] += b.x;
              v[4 * i + 1] += b.y;
              v[4 * i + 2] += b.z;
              v[4 * i + 3] += b.w;
            }
          }
          if constexpr (EPI == EPI_BIAS_RESID_F32) {
            const float4* r4 = reinterpret_cast<const float4*>(p.resid + static_cast<int64_t>(row) * p.ld_resid + col);
            float4* o4 = reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<int64_t>(row) * p.ld_out + col);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 r = r4[i];
              o4[i] = make_float4(v[4 * i] + r.x, v[4 * i + 1] + r.y, v[4 * i + 2] + r.z, v[4 * i + 3] + r.w);
            }
          } else if constexpr (EPI == EPI_BIAS_F32) {
            float4* o4 = reinterpret_cast<float4*>(static_cast<float*>(p.out) + static_cast<int64_t>(row) * p.ld_out + col);
#pragma unroll
            for (int i = 0; i < 8; ++i) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
            if constexpr (EPI == EPI_BIAS_GELU_F16) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = gelu_as(v[i]);
            }
            uint4* o4 = reinterpret_cast<uint4*>(static_cast<__half*>(p.out) + static_cast<int64_t>(row) * p.ld_out + col);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              o4[i] = make_uint4(pack_half2(v[8 * i + 0], v[8 * i + 1]), pack_half2(v[8 * i + 2], v[8 * i + 3]),
                                 pack_half2(v[8 * i + 4], v[8 * i + 5]), pack_half2(v[8 * i + 6], v[8 * i + 7]));
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
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace b200
