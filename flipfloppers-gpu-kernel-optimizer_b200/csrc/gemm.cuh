// tcgen05 projection GEMM with fused epilogues:
//   out[M,N] = epi( A[M,K] . W[N,K]^T + bias[N] (+ resid[M,N]) )
// A, W fp16 row-major (K contiguous, "K-major" for UMMA); fp32 accumulation in
// TMEM; fp32 bias.  Epilogues:
//   EPI_BIAS_F16       fp16 out            (QKV projection, reference TTB:1303)
//   EPI_BIAS_GELU_F16  fp16 gelu(.)        (ffn_in + exact GELU, TTB:1350-1354)
//   EPI_BIAS_RESID_F32 fp32 out += .       (out_proj / ffn_out + residual,
//                                           TTB:1333-1339, 1368-1369; `out`
//                                           holds the residual on entry)
//   EPI_BIAS_F32       fp32 out            (row-parallel partial sums before
//                                           the tensor-parallel all-reduce)
// It replaces the reference's mma.sync GEMM `ws_gemm_kernel`
// (csrc/g4_4_warpspec_gemm.cu:273-795) with a persistent Blackwell design:
//   grid = min(tiles, SMs); CTA c takes output tiles c, c+grid, ... (tiles
//   ordered N-fastest: the CTAs running at one time cover a band of A rows
//   across every N tile, so each A tile is read from HBM once and then from
//   L2, and W -- a few MB -- stays L2-resident; M-fastest order would stream
//   all of A once per N column when A is larger than L2);
//   warp 0     TMA producer: 64-wide K slices of A and W, SWIZZLE_128B, into a
//              STAGES-deep shared-memory ring that runs across tiles;
//   warp 1     TMEM owner and tcgen05.mma issuer (one lane), accumulating tile
//              i into TMEM buffer i%2 while the epilogue drains buffer (i-1)%2;
//   warps 2-9  epilogue: warp w reads TMEM lane quadrant w%4 (one output row
//              per thread) and half (w-2)/4 of the tile's columns, in chunks of
//              64 bytes per row (32 fp16 or 16 fp32 columns).  Each chunk is
//              staged as a 32-row SWIZZLE_64B box in one of the warp's two
//              2 KB shared-memory slots and written by a TMA store -- or, for
//              the residual epilogue, a TMA add-reduce into `out`, which then
//              already holds the residual.  Per-thread stores of a row would
//              touch 32 rows per warp instruction.
#pragma once

#include "ptx.cuh"

namespace b200 {

enum GemmEpilogue : int {
  EPI_BIAS_F16 = 0,
  EPI_BIAS_GELU_F16 = 1,
  EPI_BIAS_RESID_F32 = 2,
  EPI_BIAS_F32 = 3,
  // x1 = out + acc + bias (out holds the residual; x1 written back to out) and
  // ln_out = LayerNorm(x1)*gamma + beta in fp16 -- out_proj + residual + LN2
  EPI_BIAS_RESID_LN16 = 4,
  // ln_out = LayerNorm(out + acc + bias)*gamma + beta in fp32, out untouched --
  // ffn_out + residual + final norm
  EPI_BIAS_RESID_LN32 = 5,
};
__host__ __device__ constexpr bool epi_is_ln(int e) { return e == EPI_BIAS_RESID_LN16 || e == EPI_BIAS_RESID_LN32; }

struct GemmParams {
  int M, N, K;
  int a_row0;            // first row of A addressed by the tensor map (row offset of this call)
  const float* bias;     // [N] fp32, may be null
  const float* gamma;    // LayerNorm epilogues: [N] fp32
  const float* beta;
  float eps;
};

template <int BN, int STAGES, int EPI = EPI_BIAS_F16>
struct GemmSmem {
  static constexpr int A_BYTES = 128 * 64 * 2;
  static constexpr int B_BYTES = BN * 64 * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // epilogue staging per warp: two 2 KB slots, or for the LayerNorm epilogues the
  // warp's 32 rows x 64 columns of the residual (fp32, two SW128 boxes) + the
  // fp16 LayerNorm output box
  static constexpr int STG_WARP = epi_is_ln(EPI) ? 12288 : 4096;
  static constexpr int STG_OFF = STAGES * STAGE_BYTES;
  static constexpr int STATS_OFF = STG_OFF + 8 * STG_WARP;             // LN row statistics [2][2][128] fp32
  static constexpr int BAR_OFF = STATS_OFF + (epi_is_ln(EPI) ? 2048 : 0);
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;  // barriers + 1 KB alignment slack
};

constexpr int GEMM_THREADS = 320;  // producer, MMA, 8 epilogue warps

// Epilogue of one accumulator tile for one epilogue warp: TMEM lane quadrant q
// (rows row0 .. row0+31 of the output), columns [c_begin, c_end) of the tile
// at TMEM column tcol (column col0 of the output).  Chunks of 64 bytes per row
// alternate between the warp's two 2 KB staging slots `stg`; `gc` counts the
// chunks this warp has staged (it selects the slot).
template <int EPI>
__device__ __forceinline__ void gemm_epilogue_cols(const CUtensorMap* tmO, const GemmParams& p, uint32_t taddr0,
                                                   int c_begin, int c_end, int col0, int row0, uint8_t* stg, int& gc,
                                                   int lane) {
  constexpr bool F32 = EPI == EPI_BIAS_RESID_F32 || EPI == EPI_BIAS_F32;
  constexpr int CC = F32 ? 16 : 32;                            // columns per 64-byte chunk row
  const uint32_t sw = static_cast<uint32_t>((lane >> 1) & 3);  // SWIZZLE_64B phase of row `lane`
#pragma unroll 1
  for (int c = c_begin; c < c_end; c += CC, ++gc) {
    const uint32_t taddr = taddr0 + c;
    const int col = col0 + c;
    uint8_t* slot = stg + (gc & 1) * 2048;
    uint32_t w[16];  // the chunk's 64 bytes of this row
    // the chunk's bias is loaded before the TMEM load (whose wait orders every
    // memory access after it), so the two latencies overlap
    const bool has_bias = p.bias != nullptr && col < p.N;
    float4 bb[CC / 4];
#pragma unroll
    for (int j = 0; j < CC / 4; ++j)
      bb[j] = has_bias ? __ldg(reinterpret_cast<const float4*>(p.bias + col) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (F32) {
      float v[16];
      tmem_ld16(taddr, v);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[4 * j] += bb[j].x; v[4 * j + 1] += bb[j].y; v[4 * j + 2] += bb[j].z; v[4 * j + 3] += bb[j].w;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) w[j] = __float_as_uint(v[j]);
    } else {
      float v[32];
      tmem_ld32(taddr, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        f2upk(f2add(f2pk(v[4 * j], v[4 * j + 1]), f2pk(bb[j].x, bb[j].y)), v[4 * j], v[4 * j + 1]);
        f2upk(f2add(f2pk(v[4 * j + 2], v[4 * j + 3]), f2pk(bb[j].z, bb[j].w)), v[4 * j + 2], v[4 * j + 3]);
      }
      if constexpr (EPI == EPI_BIAS_GELU_F16) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) gelu_as2(v[j], v[j + 1]);
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) w[j] = pack_half2(v[2 * j], v[2 * j + 1]);
    }
    // the slot's previous chunk (two chunks ago) must have been read by its store
    if (lane == 0) bulk_wait_read_1();
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<uint4*>(slot + lane * 64 + ((j ^ sw) << 4)) =
          make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if constexpr (EPI == EPI_BIAS_RESID_F32)
        tma_reduce_add_2d(tmO, slot, col, row0);
      else
        tma_store_2d(tmO, slot, col, row0);
      bulk_commit();
    }
  }
}

// LayerNorm epilogue of one 128-column tile (the whole row: N == 128) for one
// epilogue warp: rows row0 .. row0+31 (TMEM lane quadrant q), columns
// 64*half .. +64, accumulator already in v.  The warp's residual box pair has
// been TMA-loaded into stg; v = residual + acc + bias, row mean/variance
// combined with the other half-warp of the quadrant through `stats` behind
// named barrier 1+q, then x1 (LN16) and the normalised row leave by TMA store
// (skipped when !ok; the barriers are always executed, so the partner warp is
// never left waiting).
template <int EPI>
__device__ __forceinline__ void gemm_epilogue_ln(const CUtensorMap* tmX, const CUtensorMap* tmN, const GemmParams& p,
                                                 float (&v)[64], int row0, int q, int half, uint8_t* stg,
                                                 float* stats, int lane, bool ok) {
  const int c0 = 64 * half;
  const uint32_t sw = static_cast<uint32_t>(lane & 7);
  // v += residual (two SW128 fp32 boxes of 32 columns) + bias
#pragma unroll
  for (int bx = 0; bx < 2; ++bx) {
    const uint8_t* box = stg + bx * 4096 + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 r = *reinterpret_cast<const float4*>(box + ((j ^ sw) << 4));
      const float4 bb = p.bias ? __ldg(reinterpret_cast<const float4*>(p.bias + c0 + 32 * bx + 4 * j))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
      float* w = v + 32 * bx + 4 * j;
      w[0] += r.x + bb.x; w[1] += r.y + bb.y; w[2] += r.z + bb.z; w[3] += r.w + bb.w;
    }
  }
  // row statistics over the 128 columns (two-pass), shared with the other half
  const int r = q * 32 + lane;
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < 64; i += 2) { s0 += v[i]; s1 += v[i + 1]; }
  stats[half * 128 + r] = s0 + s1;
  nbar_sync(1 + q, 64);
  const float mean = (stats[r] + stats[128 + r]) * (1.f / 128.f);
  float q0 = 0.f, q1 = 0.f;
#pragma unroll
  for (int i = 0; i < 64; i += 2) {
    const float a = v[i] - mean, b = v[i + 1] - mean;
    q0 += a * a; q1 += b * b;
  }
  stats[256 + half * 128 + r] = q0 + q1;
  nbar_sync(1 + q, 64);
  const float rstd = rsqrtf((stats[256 + r] + stats[384 + r]) * (1.f / 128.f) + p.eps);
  if constexpr (EPI == EPI_BIAS_RESID_LN16) {
    // x1 back into the residual boxes (stored in place), LayerNorm output to the fp16 box
#pragma unroll
    for (int bx = 0; bx < 2; ++bx) {
      uint8_t* box = stg + bx * 4096 + lane * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float* w = v + 32 * bx + 4 * j;
        *reinterpret_cast<float4*>(box + ((j ^ sw) << 4)) = make_float4(w[0], w[1], w[2], w[3]);
      }
    }
    uint8_t* nbox = stg + 8192 + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int c = 8 * j + e;
        y[e] = (v[c] - mean) * rstd * __ldg(p.gamma + c0 + c) + __ldg(p.beta + c0 + c);
      }
      *reinterpret_cast<uint4*>(nbox + ((j ^ sw) << 4)) =
          make_uint4(pack_half2(y[0], y[1]), pack_half2(y[2], y[3]), pack_half2(y[4], y[5]), pack_half2(y[6], y[7]));
    }
  } else {
    // the normalised row, fp32, into the residual boxes
#pragma unroll
    for (int bx = 0; bx < 2; ++bx) {
      uint8_t* box = stg + bx * 4096 + lane * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = 32 * bx + 4 * j;
        const float4 g = __ldg(reinterpret_cast<const float4*>(p.gamma + c0 + c));
        const float4 b = __ldg(reinterpret_cast<const float4*>(p.beta + c0 + c));
        *reinterpret_cast<float4*>(box + ((j ^ sw) << 4)) =
            make_float4((v[c] - mean) * rstd * g.x + b.x, (v[c + 1] - mean) * rstd * g.y + b.y,
                        (v[c + 2] - mean) * rstd * g.z + b.z, (v[c + 3] - mean) * rstd * g.w + b.w);
      }
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0 && ok) {
    if constexpr (EPI == EPI_BIAS_RESID_LN16) {
      tma_store_2d(tmX, stg, c0, row0);
      tma_store_2d(tmX, stg + 4096, c0 + 32, row0);
      tma_store_2d(tmN, stg + 8192, c0, row0);
    } else {
      tma_store_2d(tmN, stg, c0, row0);
      tma_store_2d(tmN, stg + 4096, c0 + 32, row0);
    }
    bulk_commit();
  }
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    k_gemm_tn(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
              const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmN,
              const GemmParams p) {
  using L = GemmSmem<BN, STAGES, EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* drain = acc_empty + 2;
  uint64_t* rbar = drain + 1;            // [8] LayerNorm epilogues: residual box loads, one per epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (p.M + 127) / 128, ntl = (p.N + BN - 1) / BN;
  const int ntiles = mt * ntl;
  const int my_tiles = (ntiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                       static_cast<int>(gridDim.x);
  const int nk = (p.K + 63) / 64;
  constexpr uint32_t TMEM_COLS = 2 * BN;  // double-buffered accumulator

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 256);  // every epilogue thread arrives once per tile
    }
    mbar_init(drain, 1);
    for (int w = 0; w < 8; ++w) mbar_init(&rbar[w], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncwarp();  // lane-0 roles rejoin their warp: bar.sync is warp-aligned
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_sync();  // the previous kernel's outputs are complete from here on

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmW);
      int it = 0;  // global k-slice counter across tiles
      bool ok = true;
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int t = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
        const int m0 = (t / ntl) * 128, n0 = (t % ntl) * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(&empty[s], ((it / STAGES) - 1) & 1, abort_flag, DERR_WAIT_SLOT)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * L::STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
          tma_load_2d(st, &tmA, &full[s], kb * 64, p.a_row0 + m0);
          tma_load_2d(st + L::A_BYTES, &tmW, &full[s], kb * 64, n0);
        }
      }
      if (*abort_flag)
        for (int j = (it > STAGES ? it - STAGES : 0); j < it; ++j) mbar_wait_drain(&full[j % STAGES], (j / STAGES) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(128, BN, false);
      int it = 0;
      bool ok = true;
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int b = i & 1;
        // the epilogue must have drained this accumulator buffer (tile i-2)
        if (i >= 2 && !mbar_wait(&acc_empty[b], ((i >> 1) - 1) & 1, abort_flag, DERR_WAIT_MMA)) break;
        tc_fence_after();
        const uint32_t dcol = tmem + b * BN;
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
            umma_f16_ss(dcol, make_sdesc(a_addr + kk * 32, 16, 1024, UMMA_SW128),
                        make_sdesc(b_addr + kk * 32, 16, 1024, UMMA_SW128), idesc, (kb | kk) != 0 ? 1u : 0u);
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(&acc_full[b]);
      }
      if (*abort_flag) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0);
      }
    }
  } else if constexpr (epi_is_ln(EPI)) {
    // LayerNorm epilogue warps 2..9 (N == BN == 128: every tile holds whole rows).
    // No early exit: the quadrant's two warps meet at named barriers each tile,
    // so after a failed wait a warp keeps stepping through the tiles with its
    // loads, waits and stores switched off.
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* stg = smem + L::STG_OFF + (warp - 2) * L::STG_WARP;
    float* stats = reinterpret_cast<float*>(smem + L::STATS_OFF);
    uint64_t* my_rbar = rbar + (warp - 2);
    if (lane == 0) {
      tma_prefetch_desc(&tmO);
      tma_prefetch_desc(&tmN);
    }
    bool ok = true;
    int loads = 0;         // residual loads issued (one phase of my_rbar each)
    bool pending = false;  // a load not yet waited for
    for (int i = 0; i < my_tiles; ++i) {
      const int b = i & 1;
      const int t = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
      const int row0 = (t / ntl) * 128 + q * 32;
      if (ok) {  // the residual rows of this tile, while its MMAs run
        if (lane == 0) {
          bulk_wait_read_all();  // the previous tile's stores have read these boxes
          mbar_arrive_expect_tx(my_rbar, 8192);
          tma_load_2d(stg, &tmO, my_rbar, 64 * half, row0);
          tma_load_2d(stg + 4096, &tmO, my_rbar, 64 * half + 32, row0);
        }
        ++loads;
        pending = true;
      }
      __syncwarp();
      if (ok) ok = mbar_wait_warp(&acc_full[b], (i >> 1) & 1, abort_flag, DERR_WAIT_MMA);
      if (ok) tc_fence_after();
      float v[64];
      tmem_ld64(tmem + (static_cast<uint32_t>(q * 32) << 16) + b * BN + 64 * half, v);
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);  // the accumulator is in registers: the MMA may reuse the buffer
      if (ok && pending) {
        ok = mbar_wait_warp(my_rbar, static_cast<uint32_t>((loads - 1) & 1), abort_flag, DERR_WAIT_TMA);
        if (ok) pending = false;
      }
      gemm_epilogue_ln<EPI>(&tmO, &tmN, p, v, row0, q, half, stg, stats, lane, ok);
    }
    if (pending) mbar_wait_drain(my_rbar, static_cast<uint32_t>((loads - 1) & 1));
    if (lane == 0) bulk_wait_all();
  } else {
    // epilogue warps 2..9
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int CW = BN / 2;                             // columns per warp per tile
    uint8_t* stg = smem + L::STG_OFF + (warp - 2) * 4096;  // two 2 KB slots
    if (lane == 0) tma_prefetch_desc(&tmO);
    int gc = 0;
    for (int i = 0; i < my_tiles; ++i) {
      const int b = i & 1;
      const int t = static_cast<int>(blockIdx.x) + i * static_cast<int>(gridDim.x);
      const int m0 = (t / ntl) * 128, n0 = (t % ntl) * BN;
      const bool ok = mbar_wait_warp(&acc_full[b], (i >> 1) & 1, abort_flag, DERR_WAIT_MMA);
      if (!ok || *abort_flag) break;
      tc_fence_after();
      gemm_epilogue_cols<EPI>(&tmO, p, tmem + (static_cast<uint32_t>(q * 32) << 16) + b * BN, half * CW,
                              (half + 1) * CW, n0, m0 + q * 32, stg, gc, lane);
      // every tcgen05.ld of buffer b has completed (each waits for its data)
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
    if (lane == 0) bulk_wait_all();  // the last stores are complete before the CTA exits
  }
  tc_fence_before();
  __syncwarp();  // lane-0 roles rejoin their warp: bar.sync is warp-aligned
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace b200
