// Fused causal block for small models: d_model = 128, 4 heads of 32,
// ffn_dim in {128, 256, 384, 512}, seq_len <= 128, any number of layers.
//
// This is the B200 counterpart of the reference's unwired megakernel
// (csrc/g5_mega_causal.cu:160-290, one CTA per sequence, residual on chip,
// hard-specialised to d=128) and of its causal forward (TTB:1282-1373): one
// persistent CTA per SM walks sequences; for each sequence and layer the whole
// pre-LN block runs on chip -- LN1, QKV projection, 4-head causal attention,
// out_proj + residual, LN2, ffn_in + erf-GELU, ffn_out + residual, and the
// final LayerNorm after the last layer.  Only x is read and y written in HBM,
// both by TMA (x as four 128-row x 32-column fp32 boxes, prefetched for the
// next sequence while the current one is in its FFN; y as one 32x32 box per
// worker warp); weights (384 KB per layer at ffn=512) are streamed from L2 by
// TMA.  Every global access is a bulk copy: a thread owns a row, so plain
// per-thread loads and stores would touch 32 rows per warp instruction.
//
// Roles (18 warps):
//   warp 0      TMA producer: x of each sequence, and 128x64 fp16 weight boxes
//               (SWIZZLE_128B) through a 3-stage ring, in exactly the order
//               the MMA warp consumes them;
//   warp 1      TMEM owner (512 columns) and tcgen05.mma issuer;
//   warps 2-17  workers: warp w owns TMEM lane quadrant q = w%4 (rows
//               32q..32q+31, one row per lane) and column group g = (w-2)/4
//               (32 of the 128 columns; in attention g is also the head).
//               Row statistics (LayerNorm mean/variance, softmax max/sum) are
//               combined across the 4 groups of a row in shared memory behind
//               one named barrier per quadrant.
//
// TMEM columns:  [384,512) is the residual stream: x is stored there before
//   LN1, out_proj accumulates onto it (x + ctx.Wo^T), the bias is added in
//   place (x1), and ffn_out accumulates onto x1.  [0,384) QKV accumulator |
//   then [0,128),[128,256) S of two heads in flight, [256,384) O of the 4
//   heads | then [0,128),[128,256) ffn_in chunk accumulators (ping-pong).
// Shared memory (1 CTA/SM): XA 32 KB (LN1 out -> context -> LN2 out, fp16,
//   SW128 K-major), Q/K/V 3 x 4 heads x 8 KB (SW64; V read MN-major), P 32 KB,
//   weight ring 48 KB, GELU chunk ping-pong aliasing the Q and K areas, the
//   layer's biases and LayerNorm parameters (7.5 KB, staged once per layer).
//   The layer input XIN (fp32, four SW128 boxes of 128 rows x 128 bytes)
//   aliases V and P: it is filled by TMA (layer 0, after the previous
//   sequence's attention) or by each thread's own W7 stores (later layers).
//   The y staging boxes (16 x 4 KB, one per worker warp) alias Q and K.
//
// Every wait is bounded (ptx.cuh); a worker that gives up still executes every
// named barrier (control flow never depends on data), so the CTA always
// reaches its teardown.
#pragma once

#include "ptx.cuh"

namespace b200 {

struct SmallParams {
  int num_seq;        // sequences
  int seq_len;        // rows per sequence (<= 128)
  int layers;
  int ffn;            // multiple of 128, <= 512
  int heads;          // 1, 2 or 4 (head_dim 128, 64 or 32)
  const float* x;     // [num_seq*seq_len, 128]
  float* y;           // [num_seq*seq_len, 128]
  const float* ln1_w; const float* ln1_b;   // [layers, 128]
  const float* b_qkv;                       // [layers, 384]
  const float* b_o;                         // [layers, 128]
  const float* ln2_w; const float* ln2_b;   // [layers, 128]
  const float* b_in;                        // [layers, ffn]
  const float* b_out;                       // [layers, 128]
  const float* lnf_w; const float* lnf_b;   // [128]
  float eps;
  float scale_log2;   // head_dim^-0.5 * log2(e)
  const unsigned char* row_valid;  // [num_seq*seq_len] key-padding mask (0 = padded row), may be null
  int non_causal;                  // 1: every query sees every valid key
};

struct SmallCfg {
  static constexpr int D = 128;
  static constexpr int NW = 16;                 // worker warps
  static constexpr int THREADS = 32 * (2 + NW);
  static constexpr int WST = 3;                 // weight ring stages
  static constexpr int BOX = 128 * 64 * 2;      // one 128x64 fp16 weight box
  static constexpr int OFF_XA = 0;              // 32 KB
  static constexpr int OFF_Q = 32768;           // 4 x 8 KB
  static constexpr int OFF_K = 65536;
  static constexpr int OFF_V = 98304;
  static constexpr int OFF_P = 131072;          // 32 KB
  static constexpr int OFF_W = 163840;          // WST x 16 KB
  static constexpr int OFF_XIN = OFF_V;         // 64 KB layer input, aliases V and P
  static constexpr int OFF_YST = OFF_Q;         // 64 KB y staging, aliases Q and K
  static constexpr int OFF_STATS = OFF_W + WST * BOX;   // float [4][4][128]
  static constexpr int OFF_VEC = OFF_STATS + 4 * 4 * 128 * 4;  // per-layer vectors, fp32
  // float offsets inside the vector block
  static constexpr int V_LN1W = 0, V_LN1B = 128, V_BQKV = 256, V_BO = 640, V_LN2W = 768, V_LN2B = 896,
                       V_BIN = 1024, V_BOUT = 1536, V_LNFW = 1664, V_LNFB = 1792, V_TOTAL = 1920;
  static constexpr int OFF_BAR = OFF_VEC + V_TOTAL * 4;
  static constexpr int TOTAL = OFF_BAR + 512 + 1024;
};

// Barrier slots
enum SmallBar : int {
  SB_WFULL = 0,        // [WST]
  SB_WEMPTY = 3,       // [WST]
  SB_N1 = 6,           // workers: LN1 output in XA
  SB_QKV_DONE = 7,     // MMA: QKV accumulator complete
  SB_QKV_SMEM = 8,     // workers: Q/K/V in shared memory, QKV TMEM read
  SB_S_FULL = 9,       // [2] MMA: S of a head complete
  SB_P_FULL = 11,      // workers: P of a head in shared memory
  SB_PV_DONE = 12,     // MMA: O += P.V of a head complete
  SB_CTX = 13,         // workers: context in XA
  SB_OP_DONE = 14,     // MMA: out_proj accumulator complete
  SB_N2 = 15,          // workers: LN2 output in XA, x1 in TMEM
  SB_FIN = 16,         // [2] MMA: ffn_in chunk accumulator complete
  SB_H = 18,           // [2] workers: GELU chunk in shared memory
  SB_HFREE = 20,       // [2] MMA: ffn_out consumed a GELU chunk buffer
  SB_FOUT = 22,        // MMA: ffn_out accumulator complete
  SB_DRAIN = 23,
  SB_XFULL = 24,       // TMA: x of the CTA's current sequence in XIN
  SB_VFULL = 25,       // bulk copies: the layer's vectors in shared memory
  // row-split mode only: extra weight slots in areas idle at the time
  SB_QKF = 26,         // [3] QKV boxes 3-5 in the Q/K area (free until the QKV results are written)
  SB_VPF = 29,         // [4] ffn_out boxes in the V/P area (free once attention is done): loaded
  SB_VPE = 33,         // [4] ... and consumed
  SB_COUNT = 37
};

__device__ __forceinline__ void named_bar(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// completion parity of the idx-th completion (within one sequence-layer step)
// of a barrier that completes `per` times per step, at step `step`
__device__ __forceinline__ uint32_t par(int step, int per, int idx) {
  return static_cast<uint32_t>((step * per + idx) & 1);
}

// The kernel body.  ROWS = false: one CTA per sequence (persistent over
// sequences and layers).  ROWS = true: two CTAs per sequence, one layer (the
// row-split mode, see k_block_rows); the producer and MMA roles are the same
// in both modes, only the workers' phases differ.  NH: heads (1, 2 or 4; a
// compile-time constant so the per-head loops unroll as for a fixed shape).
template <bool ROWS, int NH>
__device__ __forceinline__ void block_small_body(const CUtensorMap* tm_qkv, const CUtensorMap* tm_o,
                                                 const CUtensorMap* tm_in, const CUtensorMap* tm_out,
                                                 const CUtensorMap* tm_x, const CUtensorMap* tm_y,
                                                 const SmallParams& p) {
  using C = SmallCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + SB_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* stats = reinterpret_cast<float*>(smem + C::OFF_STATS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = p.ffn / 128;                              // ffn chunks of 128
  // sequences this CTA handles: seq_first, seq_first + gridDim.x, ... (ROWS: its pair's one sequence)
  const int seq_first = ROWS ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int nseq_cta = ROWS ? (seq_first < p.num_seq ? 1 : 0)
                            : (p.num_seq - seq_first + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x);
  const int nsteps = nseq_cta * p.layers;
  // completions per step of the ping-pong barriers (buffer b serves chunks b, b+2, ...)
  const int per_b0 = (nch + 1) / 2, per_b1 = nch / 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::WST; ++s) {
      mbar_init(&bar[SB_WFULL + s], 1);
      mbar_init(&bar[SB_WEMPTY + s], 1);
    }
    mbar_init(&bar[SB_N1], 32 * C::NW);
    mbar_init(&bar[SB_QKV_DONE], 1);
    mbar_init(&bar[SB_QKV_SMEM], 32 * C::NW);
    mbar_init(&bar[SB_S_FULL + 0], 1);
    mbar_init(&bar[SB_S_FULL + 1], 1);
    mbar_init(&bar[SB_P_FULL], 32 * C::NW);
    mbar_init(&bar[SB_PV_DONE], 1);
    mbar_init(&bar[SB_CTX], 32 * C::NW);
    mbar_init(&bar[SB_OP_DONE], 1);
    mbar_init(&bar[SB_N2], 32 * C::NW);
    mbar_init(&bar[SB_FIN + 0], 1);
    mbar_init(&bar[SB_FIN + 1], 1);
    mbar_init(&bar[SB_H + 0], 32 * C::NW);
    mbar_init(&bar[SB_H + 1], 32 * C::NW);
    mbar_init(&bar[SB_HFREE + 0], 1);
    mbar_init(&bar[SB_HFREE + 1], 1);
    mbar_init(&bar[SB_FOUT], 1);
    mbar_init(&bar[SB_DRAIN], 1);
    mbar_init(&bar[SB_XFULL], 1);
    mbar_init(&bar[SB_VFULL], 1);
    for (int i = 0; i < 3; ++i) mbar_init(&bar[SB_QKF + i], 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bar[SB_VPF + i], 1);
      mbar_init(&bar[SB_VPE + i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncwarp();  // lane-0 roles rejoin their warp: bar.sync is warp-aligned
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_sync();  // the previous kernel's outputs are complete from here on

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(tm_qkv);
      tma_prefetch_desc(tm_o);
      tma_prefetch_desc(tm_in);
      tma_prefetch_desc(tm_out);
      tma_prefetch_desc(tm_x);
      int box = 0;
      bool ok = true;
      // x of sequence `seq` (rows past seq_len are zero-filled) -> XIN
      int xloads = 0;
      auto load_x = [&](int seq) {
        ++xloads;
        mbar_arrive_expect_tx(&bar[SB_XFULL], 4 * 128 * 128);
        for (int g = 0; g < 4; ++g)
          tma_load_3d(smem + C::OFF_XIN + g * 16384, tm_x, &bar[SB_XFULL], 32 * g, 0, seq);
      };
      if (nsteps > 0) load_x(seq_first);
      auto load = [&](const CUtensorMap* m, int col, int row) {
        const int s = box % C::WST;
        if (box >= C::WST && !mbar_wait(&bar[SB_WEMPTY + s], ((box / C::WST) - 1) & 1, abort_flag, DERR_WAIT_SLOT)) {
          ok = false;
          return;
        }
        mbar_arrive_expect_tx(&bar[SB_WFULL + s], C::BOX);
        tma_load_2d(smem + C::OFF_W + s * C::BOX, m, &bar[SB_WFULL + s], col, row);
        ++box;
      };
      // row-split mode: QKV boxes 3-5 into the Q/K area, ffn_out boxes through a 4-slot ring in V/P
      int qk = 0, vp = 0;
      auto load_qk = [&](const CUtensorMap* m, int col, int row) {
        mbar_arrive_expect_tx(&bar[SB_QKF + qk], C::BOX);
        tma_load_2d(smem + C::OFF_Q + qk * C::BOX, m, &bar[SB_QKF + qk], col, row);
        ++qk;
      };
      auto load_vp = [&](const CUtensorMap* m, int col, int row) {
        const int s = vp & 3;
        if (vp >= 4 && !mbar_wait(&bar[SB_VPE + s], ((vp >> 2) - 1) & 1, abort_flag, DERR_WAIT_SLOT)) {
          ok = false;
          return;
        }
        mbar_arrive_expect_tx(&bar[SB_VPF + s], C::BOX);
        tma_load_2d(smem + C::OFF_V + s * C::BOX, m, &bar[SB_VPF + s], col, row);
        ++vp;
      };
      if constexpr (ROWS) {
        // one step; boxes in the MMA's order within each buffer set
        load(tm_qkv, 0, 0);
        if (ok) load(tm_qkv, 64, 0);
        if (ok) load(tm_qkv, 0, 128);
        load_qk(tm_qkv, 64, 128);
        load_qk(tm_qkv, 0, 256);
        load_qk(tm_qkv, 64, 256);
        for (int kh = 0; ok && kh < 2; ++kh) load(tm_o, kh * 64, 0);
        // V and P are free once the context is published
        if (ok && nsteps > 0 && !mbar_wait(&bar[SB_CTX], 0, abort_flag, DERR_WAIT_SOFTMAX)) ok = false;
        for (int c = 0; ok && c < nch && c < 2; ++c)
          for (int kh = 0; ok && kh < 2; ++kh) load_vp(tm_out, c * 128 + kh * 64, 0);
        // ffn_in chunk c waits only for ring slots that earlier ffn_in MMAs free;
        // ffn_out chunk c (c >= 2) for the V/P slot of chunk c-2's ffn_out
        for (int c = 0; ok && c < nch; ++c) {
          for (int kh = 0; ok && kh < 2; ++kh) load(tm_in, kh * 64, c * 128);
          if (c >= 2)
            for (int kh = 0; ok && kh < 2; ++kh) load_vp(tm_out, c * 128 + kh * 64, 0);
        }
      }
      for (int step = 0; !ROWS && ok && step < nsteps; ++step) {
        const int l = step % p.layers;
        for (int nt = 0; ok && nt < 3; ++nt)
          for (int kh = 0; ok && kh < 2; ++kh) load(tm_qkv, kh * 64, l * 384 + nt * 128);
        for (int kh = 0; ok && kh < 2; ++kh) load(tm_o, kh * 64, l * 128);
        for (int kh = 0; ok && kh < 2; ++kh) load(tm_in, kh * 64, l * p.ffn);
        // after the last layer's attention (V and P consumed, CTX published) the
        // next sequence's x can overwrite XIN while this one runs its FFN
        const int next_seq = ROWS ? p.num_seq : seq_first + (step / p.layers + 1) * static_cast<int>(gridDim.x);
        if (ok && l == p.layers - 1 && next_seq < p.num_seq) {
          if (!mbar_wait(&bar[SB_CTX], par(step, 1, 0), abort_flag, DERR_WAIT_SOFTMAX)) {
            ok = false;
            break;
          }
          load_x(next_seq);
        }
        for (int c = 0; ok && c < nch; ++c) {
          if (c + 1 < nch)
            for (int kh = 0; ok && kh < 2; ++kh) load(tm_in, kh * 64, l * p.ffn + (c + 1) * 128);
          for (int kh = 0; ok && kh < 2; ++kh) load(tm_out, c * 128 + kh * 64, l * 128);
        }
      }
      if (*abort_flag) {
        for (int b = (box > C::WST ? box - C::WST : 0); b < box; ++b)
          mbar_wait_drain(&bar[SB_WFULL + b % C::WST], (b / C::WST) & 1);
        if (xloads > 0) mbar_wait_drain(&bar[SB_XFULL], (xloads - 1) & 1);
        for (int i = 0; i < qk; ++i) mbar_wait_drain(&bar[SB_QKF + i], 0);
        for (int b = (vp > 4 ? vp - 4 : 0); b < vp; ++b) mbar_wait_drain(&bar[SB_VPF + (b & 3)], (b >> 2) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t ID_N128 = make_idesc_f16(128, 128, false);
      constexpr uint32_t ID_PV = make_idesc_f16(128, 32, true);
      const uint32_t xa = smem_u32(smem + C::OFF_XA);
      const uint32_t qs = smem_u32(smem + C::OFF_Q), ks = smem_u32(smem + C::OFF_K), vs = smem_u32(smem + C::OFF_V);
      const uint32_t ps = smem_u32(smem + C::OFF_P);
      const uint32_t ws = smem_u32(smem + C::OFF_W);
      int box = 0, qk = 0, vp = 0;
      bool ok = true;
      // where a weight box comes from: the ring, or (row-split mode) a Q/K or V/P slot
      enum { FROM_RING = 0, FROM_QK = 1, FROM_VP = 2 };
      auto acquire = [&](int src) -> uint32_t {
        uint64_t* full;
        uint32_t parity, w;
        if (src == FROM_RING) {
          full = &bar[SB_WFULL + box % C::WST], parity = (box / C::WST) & 1, w = ws + (box % C::WST) * C::BOX;
        } else if (src == FROM_QK) {
          full = &bar[SB_QKF + qk], parity = 0, w = qs + qk * C::BOX;
        } else {
          full = &bar[SB_VPF + (vp & 3)], parity = (vp >> 2) & 1, w = vs + (vp & 3) * C::BOX;
        }
        if (!mbar_wait(full, parity, abort_flag, DERR_WAIT_TMA)) {
          ok = false;
          return 0;
        }
        tc_fence_after();
        return w;
      };
      auto release = [&](int src) {  // after the MMAs reading the box are issued
        if (src == FROM_RING) {
          tc_commit(&bar[SB_WEMPTY + box % C::WST]);
          ++box;
        } else if (src == FROM_QK) {
          ++qk;  // read once, never refilled
        } else {
          tc_commit(&bar[SB_VPE + (vp & 3)]);
          ++vp;
        }
      };
      // D[tmem_col] (+)= A(128x128, SW128 K-major at a) . W-box^T over two 64-wide K halves
      auto gemm_k128 = [&](uint32_t a, uint32_t dcol, bool acc_in, int src0 = FROM_RING, int src1 = FROM_RING) {
        for (int kh = 0; kh < 2 && ok; ++kh) {
          const int src = kh ? src1 : src0;
          const uint32_t w = acquire(src);
          if (!ok) return;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_ss(tmem + dcol, make_sdesc(a + kh * 16384 + kk * 32, 16, 1024, UMMA_SW128),
                        make_sdesc(w + kk * 32, 16, 1024, UMMA_SW128), ID_N128, (acc_in || kh || kk) ? 1u : 0u);
          release(src);
        }
      };
      // head h spans the 32-column Q / K / V tiles gpb*h .. gpb*h + gpb - 1 (SW64, one
      // per column group): S = Q.K^T takes two K=16 steps per tile
      constexpr int H = NH, gpb = 4 / NH;
      auto issue_s = [&](int h) {
#pragma unroll
        for (int kk = 0; kk < 2 * gpb; ++kk) {
          const uint32_t off = static_cast<uint32_t>((gpb * h + (kk >> 1)) * 8192 + (kk & 1) * 32);
          umma_f16_ss(tmem + (h & 1) * 128, make_sdesc(qs + off, 16, 512, UMMA_SW64),
                      make_sdesc(ks + off, 16, 512, UMMA_SW64), ID_N128, kk ? 1u : 0u);
        }
        tc_commit(&bar[SB_S_FULL + (h & 1)]);
      };
      for (int step = 0; ok && step < nsteps; ++step) {
        // QKV projection
        if (!mbar_wait(&bar[SB_N1], par(step, 1, 0), abort_flag, DERR_WAIT_SOFTMAX)) break;
        tc_fence_after();
        if constexpr (ROWS) {
          gemm_k128(xa, 0, false);
          if (ok) gemm_k128(xa, 128, false, FROM_RING, FROM_QK);
          if (ok) gemm_k128(xa, 256, false, FROM_QK, FROM_QK);
        } else {
          for (int nt = 0; nt < 3 && ok; ++nt) gemm_k128(xa, nt * 128, false);
        }
        if (!ok) break;
        tc_commit(&bar[SB_QKV_DONE]);
        // attention: S of heads 0 and 1, then per head PV and the S two heads ahead
        if (!mbar_wait(&bar[SB_QKV_SMEM], par(step, 1, 0), abort_flag, DERR_WAIT_SOFTMAX)) break;
        tc_fence_after();
        issue_s(0);
        if (H > 1) issue_s(1);
        for (int h = 0; h < H && ok; ++h) {
          if (!mbar_wait(&bar[SB_P_FULL], par(step, H, h), abort_flag, DERR_WAIT_SOFTMAX)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int tt = 0; tt < gpb; ++tt) {  // O columns 32t.. from V tile t
            const int t = gpb * h + tt;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_f16_ss(tmem + 256 + 32 * t,
                          make_sdesc(ps + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024, UMMA_SW128),
                          make_sdesc(vs + t * 8192 + kk * 16 * 64, 128 * 64, 512, UMMA_SW64), ID_PV, kk ? 1u : 0u);
          }
          tc_commit(&bar[SB_PV_DONE]);
          if (h + 2 < H) issue_s(h + 2);
        }
        if (!ok) break;
        // out_proj
        if (!mbar_wait(&bar[SB_CTX], par(step, 1, 0), abort_flag, DERR_WAIT_SOFTMAX)) break;
        tc_fence_after();
        gemm_k128(xa, 384, true);  // onto the residual x stored by the workers
        if (!ok) break;
        tc_commit(&bar[SB_OP_DONE]);
        // FFN: fin_0, then per chunk c: fin_{c+1}, fout_c
        if (!mbar_wait(&bar[SB_N2], par(step, 1, 0), abort_flag, DERR_WAIT_SOFTMAX)) break;
        tc_fence_after();
        gemm_k128(xa, 0, false);
        if (!ok) break;
        tc_commit(&bar[SB_FIN + 0]);
        for (int c = 0; c < nch && ok; ++c) {
          if (c + 1 < nch) {
            gemm_k128(xa, ((c + 1) & 1) * 128, false);
            if (!ok) break;
            tc_commit(&bar[SB_FIN + ((c + 1) & 1)]);
          }
          const int b = c & 1;
          if (!mbar_wait(&bar[SB_H + b], par(step, b ? per_b1 : per_b0, c >> 1), abort_flag, DERR_WAIT_SOFTMAX)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // onto the residual; row-split mode reads these boxes from the V/P ring
          gemm_k128(smem_u32(smem + (b ? C::OFF_K : C::OFF_Q)), 384, true, ROWS ? FROM_VP : FROM_RING,
                    ROWS ? FROM_VP : FROM_RING);
          if (!ok) break;
          tc_commit(&bar[SB_HFREE + b]);
        }
        if (!ok) break;
        tc_commit(&bar[SB_FOUT]);
      }
      if (*abort_flag) {
        tc_commit(&bar[SB_DRAIN]);
        mbar_wait_drain(&bar[SB_DRAIN], 0);
      }
    }
  } else {
    // ------------------------------------------------------------ workers
    const int q = warp & 3;
    const int g = (warp - 2) >> 2;       // column group (32 columns; head g in attention)
    const int r = q * 32 + lane;         // row of the tile (TMEM lane)
    const int c0 = 32 * g;               // first column of this thread
    const int bar_id = 1 + q;            // named barrier of the quadrant (4 warps)
    const uint32_t trow = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float* st0 = stats;                  // [4][128]
    float* st1 = stats + 512;
    float* st2 = stats + 1024;           // second halves of the merged (max, sum) reductions
    float* st3 = stats + 1536;
    // heads: H of head_dim 128 / H; column group g (32 columns) belongs to head hg.
    // The last head's row sum goes to st_f, the buffer its max did not use, and the
    // LayerNorms after it take (st_o, st_f), so consecutive reductions still alternate.
    constexpr int H = NH;
    const int hg = g / (4 / NH);
    float* st_f = ((H - 1) & 1) ? st0 : st1;
    float* st_o = ((H - 1) & 1) ? st1 : st0;
    float* vec = reinterpret_cast<float*>(smem + C::OFF_VEC);
    const int wtid = threadIdx.x - 64;   // 0..511 among the workers
    uint8_t* xa = smem + C::OFF_XA;
    bool ok = true;
    float v[32];

    auto wait_w = [&](int slot, uint32_t parity) {
      if (ok) ok = mbar_wait_warp(&bar[slot], parity, abort_flag, DERR_WAIT_MMA);
      if (ok) tc_fence_after();
    };
    // sum of one per-thread partial over the 4 column groups of the row
    auto row_sum = [&](float part, float* buf) {
      buf[g * 128 + r] = part;
      named_bar(bar_id, 128);
      return buf[r] + buf[128 + r] + buf[256 + r] + buf[384 + r];
    };
    // a head's row max and the previous head's row sum behind one barrier
    auto row_max_sum = [&](float pmax, float psum, float* bm, float* bs, float& m, float& l) {
      bm[g * 128 + r] = pmax;
      bs[g * 128 + r] = psum;
      named_bar(bar_id, 128);
      m = fmaxf(fmaxf(bm[r], bm[128 + r]), fmaxf(bm[256 + r], bm[384 + r]));
      l = bs[r] + bs[128 + r] + bs[256 + r] + bs[384 + r];
    };
    // LayerNorm of v (32 columns of this row) in place, two-pass statistics
    // (f32x2 pairs throughout: the statistics use 2 pair accumulators each);
    // vec_parity >= 0: wait for that phase of the vector copies (SB_VFULL)
    // only before gamma and beta are read; bm / bv: the statistics buffers of the
    // mean and the variance (default st0 / st1)
    auto layer_norm = [&](const float* gamma, const float* beta, int vec_parity = -1, float* bm = nullptr,
                          float* bv = nullptr) {  // gamma/beta: shared memory
      uint64_t a0 = f2pk(0.f, 0.f), a1 = a0;
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        a0 = f2add(a0, f2pk(v[i], v[i + 1]));
        a1 = f2add(a1, f2pk(v[i + 2], v[i + 3]));
      }
      float t0, t1, t2, t3;
      f2upk(a0, t0, t1);
      f2upk(a1, t2, t3);
      const float mean = row_sum((t0 + t2) + (t1 + t3), bm ? bm : st0) * (1.f / 128.f);
      const uint64_t nm = f2pk(-mean, -mean);
      a0 = f2pk(0.f, 0.f);
      a1 = a0;
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const uint64_t d0 = f2add(f2pk(v[i], v[i + 1]), nm), d1 = f2add(f2pk(v[i + 2], v[i + 3]), nm);
        a0 = f2fma(d0, d0, a0);
        a1 = f2fma(d1, d1, a1);
        f2upk(d0, v[i], v[i + 1]);
        f2upk(d1, v[i + 2], v[i + 3]);
      }
      f2upk(a0, t0, t1);
      f2upk(a1, t2, t3);
      const float rstd = rsqrtf(row_sum((t0 + t2) + (t1 + t3), bv ? bv : st1) * (1.f / 128.f) + p.eps);
      const uint64_t rs = f2pk(rstd, rstd);
      if (vec_parity >= 0) wait_w(SB_VFULL, static_cast<uint32_t>(vec_parity));
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const float4 gg = *reinterpret_cast<const float4*>(gamma + c0 + i);
        const float4 bb = *reinterpret_cast<const float4*>(beta + c0 + i);
        f2upk(f2fma(f2mul(f2pk(v[i], v[i + 1]), rs), f2pk(gg.x, gg.y), f2pk(bb.x, bb.y)), v[i], v[i + 1]);
        f2upk(f2fma(f2mul(f2pk(v[i + 2], v[i + 3]), rs), f2pk(gg.z, gg.w), f2pk(bb.z, bb.w)), v[i + 2], v[i + 3]);
      }
    };
    // 32 fp16 values of this row at column c0 of a 128-wide SW128 K-major tile (2 atoms of 64)
    auto store_sw128 = [&](uint8_t* base) {
      uint8_t* atom = base + (c0 >> 6) * 16384;
      const int ch0 = (c0 & 63) >> 3;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(atom + sw128_off(r, ch0 + j)) =
            make_uint4(pack_half2(v[8 * j], v[8 * j + 1]), pack_half2(v[8 * j + 2], v[8 * j + 3]),
                       pack_half2(v[8 * j + 4], v[8 * j + 5]), pack_half2(v[8 * j + 6], v[8 * j + 7]));
    };
    // 32 fp16 values of this row into a 128x32 SW64 tile (64-byte rows)
    auto store_sw64 = [&](uint8_t* base) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(base + r * 64 + ((j ^ ((r >> 1) & 3)) << 4)) =
            make_uint4(pack_half2(v[8 * j], v[8 * j + 1]), pack_half2(v[8 * j + 2], v[8 * j + 3]),
                       pack_half2(v[8 * j + 4], v[8 * j + 5]), pack_half2(v[8 * j + 6], v[8 * j + 7]));
    };
    auto publish = [&](int slot) {
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bar[slot]);
    };

    // a layer's biases and LayerNorm parameters -> shared memory: ten bulk copies
    // issued by one worker, completing on SB_VFULL (one HBM/L2 round trip that
    // overlaps the x load, instead of dependent per-thread loads)
    int nstaged = 0;  // stagings issued (by worker 0)
    auto stage_vectors = [&](int l) {
      if (wtid != 0) return;
      ++nstaged;
      fence_proxy_async_smem();  // the previous layer's reads of these buffers come first
      const uint32_t fb = 4u * static_cast<uint32_t>(p.ffn);
      mbar_arrive_expect_tx(&bar[SB_VFULL], 8u * 512u + 1536u + fb);
      bulk_load(vec + C::V_LN1W, p.ln1_w + l * 128, 512, &bar[SB_VFULL]);
      bulk_load(vec + C::V_LN1B, p.ln1_b + l * 128, 512, &bar[SB_VFULL]);
      bulk_load(vec + C::V_BQKV, p.b_qkv + l * 384, 1536, &bar[SB_VFULL]);
      bulk_load(vec + C::V_BO, p.b_o + l * 128, 512, &bar[SB_VFULL]);
      bulk_load(vec + C::V_LN2W, p.ln2_w + l * 128, 512, &bar[SB_VFULL]);
      bulk_load(vec + C::V_LN2B, p.ln2_b + l * 128, 512, &bar[SB_VFULL]);
      bulk_load(vec + C::V_BIN, p.b_in + static_cast<int64_t>(l) * p.ffn, fb, &bar[SB_VFULL]);
      bulk_load(vec + C::V_BOUT, p.b_out + l * 128, 512, &bar[SB_VFULL]);
      bulk_load(vec + C::V_LNFW, p.lnf_w, 512, &bar[SB_VFULL]);
      bulk_load(vec + C::V_LNFB, p.lnf_b, 512, &bar[SB_VFULL]);
    };

    if constexpr (!ROWS) {
      for (int step = 0; step < nsteps; ++step) {
        const int l = step % p.layers;
        const int seq = seq_first + (step / p.layers) * static_cast<int>(gridDim.x);
        const bool row_ok = r < p.seq_len;
        const int64_t grow = static_cast<int64_t>(seq) * p.seq_len + r;
        // this thread's 32 columns of row r in XIN (box g, SW128)
        uint8_t* xin_row = smem + C::OFF_XIN + g * 16384;
        // ---- W1: x -> residual in TMEM [384,512); LN1 -> XA
        const bool restage = step == 0 || p.layers > 1;
        if (restage) {
          if (step > 0) named_bar(5, 32 * C::NW);  // every worker is done with the previous layer's vectors
          stage_vectors(l);
        }
        // layer 0: x arrives by TMA; later layers: this thread wrote its own slice in W7
        if (l == 0) wait_w(SB_XFULL, static_cast<uint32_t>((step / p.layers) & 1));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 t = *reinterpret_cast<const float4*>(xin_row + sw128_off(r, j));
          v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
        }
        if (ok) tmem_st32(trow + 384 + c0, v);
        layer_norm(vec + C::V_LN1W, vec + C::V_LN1B, restage ? ((p.layers > 1 ? step : 0) & 1) : -1);
        store_sw128(xa);
        // the previous step's y store must have read its staging box before Q/K
        // (which it aliases) are rewritten, and they are rewritten only after N1
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
        publish(SB_N1);
        // ---- W2: QKV accumulator -> Q/K/V tiles (head g = column group g)
        wait_w(SB_QKV_DONE, par(step, 1, 0));
#pragma unroll 1
        for (int nt = 0; nt < 3; ++nt) {
          if (ok) tmem_ld32(trow + nt * 128 + c0, v);
          f2_add_bias32(v, vec + C::V_BQKV + nt * 128 + c0);
          store_sw64(smem + (nt == 0 ? C::OFF_Q : nt == 1 ? C::OFF_K : C::OFF_V) + g * 8192);
        }
        publish(SB_QKV_SMEM);
        // ---- W3: softmax per head (this thread: row r, keys c0..c0+31)
        // bit i: key c0+i exists and is not padding (the causal bound is applied per row below);
        // lane i of the warp tests key c0+i (one coalesced byte load) and the ballot gathers them
        uint32_t kvalid;
        {
          const int k = c0 + lane;
          bool v_ok = k < p.seq_len;
          if (v_ok && p.row_valid != nullptr) v_ok = p.row_valid[static_cast<int64_t>(seq) * p.seq_len + k] != 0;
          kvalid = __ballot_sync(0xffffffffu, v_ok);
        }
        if (!p.non_causal) kvalid &= (r >= c0 + 31) ? 0xffffffffu : (r < c0 ? 0u : (0xffffffffu >> (31 - (r - c0))));
        float my_l = 1.f;  // softmax denominator of head hg (this thread's head in the context step)
        float prev_sum = 0.f;  // this thread's partial row sum of the previous head
#pragma unroll 1
        for (int h = 0; h < H; ++h) {
          wait_w(SB_S_FULL + (h & 1), par(step, (h & 1) ? H / 2 : (H + 1) / 2, h >> 1));
          if (ok) tmem_ld32(trow + (h & 1) * 128 + c0, v);
          if (kvalid != 0xffffffffu) {  // raw scores; the positive scale is applied in the exponent
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (!((kvalid >> i) & 1u)) v[i] = -INFINITY;
          }
          float mx = -INFINITY;
#pragma unroll
          for (int i = 0; i < 32; i += 2) mx = fmax3(mx, v[i], v[i + 1]);
          // head h's max with head h-1's sum; the pairs alternate (st0, st2) / (st1, st3)
          float m, lprev;
          row_max_sum(mx, prev_sum, (h & 1) ? st1 : st0, (h & 1) ? st3 : st2, m, lprev);
          if (h > 0 && h - 1 == hg) my_l = lprev;
          // a row that sees no key (its mask excludes every visible key) keeps P = 0 and a zero
          // context, as the reference's masked-out rows end up after their block (TTB:163-164)
          m = (m == -INFINITY) ? 0.f : m * p.scale_log2;
          const uint64_t sc = f2pk(p.scale_log2, p.scale_log2), nm = f2pk(-m, -m);
          uint64_t a0 = f2pk(0.f, 0.f), a1 = a0;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float e0, e1, e2, e3;
            f2upk(f2fma(f2pk(v[i], v[i + 1]), sc, nm), e0, e1);
            f2upk(f2fma(f2pk(v[i + 2], v[i + 3]), sc, nm), e2, e3);
            v[i] = fast_exp2(e0); v[i + 1] = fast_exp2(e1); v[i + 2] = fast_exp2(e2); v[i + 3] = fast_exp2(e3);
            a0 = f2add(a0, f2pk(v[i], v[i + 1]));
            a1 = f2add(a1, f2pk(v[i + 2], v[i + 3]));
          }
          float t0, t1, t2, t3;
          f2upk(a0, t0, t1);
          f2upk(a1, t2, t3);
          prev_sum = (t0 + t2) + (t1 + t3);
          // P of the previous head must have been consumed before P is overwritten
          if (h > 0) wait_w(SB_PV_DONE, par(step, H, h - 1));
          store_sw128(smem + C::OFF_P);
          publish(SB_P_FULL);
        }
        {
          const float lf = row_sum(prev_sum, st_f);  // the last head's sum
          if (hg == H - 1) my_l = lf;
        }
        // ---- W4: context = O / l of head hg -> XA (this thread's 32 columns)
        wait_w(SB_PV_DONE, par(step, H, H - 1));
        if (ok) tmem_ld32(trow + 256 + c0, v);
        {
          const float inv = my_l > 0.f ? 1.f / my_l : 0.f;
          const uint64_t iv = f2pk(inv, inv);
#pragma unroll
          for (int i = 0; i < 32; i += 2) f2upk(f2mul(f2pk(v[i], v[i + 1]), iv), v[i], v[i + 1]);
        }
        store_sw128(xa);
        publish(SB_CTX);
        // ---- W5: x1 = (x + ctx.Wo^T, accumulated in TMEM) + bo, back into TMEM ; LN2 -> XA
        wait_w(SB_OP_DONE, par(step, 1, 0));
        if (ok) tmem_ld32(trow + 384 + c0, v);
        f2_add_bias32(v, vec + C::V_BO + c0);
        if (ok) tmem_st32(trow + 384 + c0, v);
        layer_norm(vec + C::V_LN2W, vec + C::V_LN2B, -1, st_o, st_f);  // after st_f (the last head's sum)
        store_sw128(xa);
        publish(SB_N2);
        // ---- W6: GELU chunks -> H ping-pong
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          const int b = c & 1;
          wait_w(SB_FIN + b, par(step, b ? per_b1 : per_b0, c >> 1));
          if (ok) tmem_ld32(trow + b * 128 + c0, v);
          f2_add_bias32(v, vec + C::V_BIN + c * 128 + c0);
#pragma unroll
          for (int i = 0; i < 32; i += 2) gelu_as2(v[i], v[i + 1]);
          // the buffer's previous chunk (c-2) must have been consumed by ffn_out
          if (c >= 2) wait_w(SB_HFREE + b, par(step, b ? per_b1 : per_b0, (c >> 1) - 1));
          store_sw128(smem + (b ? C::OFF_K : C::OFF_Q));
          publish(SB_H + b);
        }
        // ---- W7: x2 = (x1 + h.W2^T, accumulated in TMEM) + b2 ; final LayerNorm (last layer) -> y
        wait_w(SB_FOUT, par(step, 1, 0));
        if (ok) tmem_ld32(trow + 384 + c0, v);
        f2_add_bias32(v, vec + C::V_BOUT + c0);
        if (l == p.layers - 1) {
          layer_norm(vec + C::V_LNFW, vec + C::V_LNFB, -1, st_o, st_f);  // after st_f (LN2's variance)
          // padded rows of the model output are zero (with causal attention and prefix-valid
          // padding the valid rows never see a padded key, so only the output needs masking)
          const bool zero = row_ok && p.row_valid != nullptr && p.row_valid[grow] == 0;
          // this warp's 32x32 box of y (rows 32q.., columns c0..), staged SW128 and stored
          // by TMA; rows past seq_len fall outside the tensor map and are not written
          uint8_t* ybox = smem + C::OFF_YST + (q * 4 + g) * 4096;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(ybox + sw128_off(lane, j)) =
                zero ? make_float4(0.f, 0.f, 0.f, 0.f) : make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && ok) {
            tma_store_3d(tm_y, ybox, c0, 32 * q, seq);
            bulk_commit();
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(xin_row + sw128_off(r, j)) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
        // the next step's LN1 (which reuses the statistics buffers) must not race
        // this step's final row reduction
        named_bar(bar_id, 128);
      }
    } else if (nsteps > 0) {
      // ---- row-split mode (one layer): this CTA owns 64 query rows of its
      // sequence -- half 0 rows 0-31 and 96-127, half 1 rows 32-95, equal
      // causal work.  Own row k (0..63) sits in TMEM lanes 32(k/16) + k%16 and
      // the lane 16 above it: the tiles the MMAs read for Q, P, the context,
      // LN2 and the GELU chunks hold every own row twice, so lanes j and j+16
      // of a warp share a row and split its 32 columns, 16 each.  LN1, K and V
      // cover all 128 rows (every own row attends to keys of the other half).
      const int half = static_cast<int>(blockIdx.x & 1);
      const int hh = lane >> 4;                    // which 16 of the warp's 32 columns
      const int k = q * 16 + (lane & 15);          // own row held by this TMEM lane
      const int srow = half ? k + 32 : (k < 32 ? k : k + 64);  // its sequence row
      const int cc = c0 + 16 * hh;                 // this thread's 16 columns
      // own index of natural row r (natural-layout accumulators: LN1, QKV), -1 if not own
      const int kn = half ? ((r >= 32 && r < 96) ? r - 32 : -1) : (r < 32 ? r : (r >= 96 ? r - 64 : -1));
      const int seq = seq_first;
      const int64_t srow_g = static_cast<int64_t>(seq) * p.seq_len + srow;
      uint8_t* xin_box = smem + C::OFF_XIN + g * 16384;
      float u[16];
      auto take_half = [&]() {
#pragma unroll
        for (int i = 0; i < 16; ++i) u[i] = hh ? v[16 + i] : v[i];
      };
      auto add16 = [&](const float* b) {  // u += b[0..15] (shared memory)
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const float4 bb = *reinterpret_cast<const float4*>(b + i);
          f2upk(f2add(f2pk(u[i], u[i + 1]), f2pk(bb.x, bb.y)), u[i], u[i + 1]);
          f2upk(f2add(f2pk(u[i + 2], u[i + 3]), f2pk(bb.z, bb.w)), u[i + 2], u[i + 3]);
        }
      };
      // row statistics over the 8 threads of an own row: the lane pair, then the 4
      // column groups (slot: the pair's lower TMEM lane, inside this quadrant's
      // 32 slots like every other reduction of the quadrant)
      const int ks = r & ~16;
      auto own_sum = [&](float part, float* buf) {
        part += __shfl_xor_sync(0xffffffffu, part, 16);
        buf[g * 128 + ks] = part;
        named_bar(bar_id, 128);
        return buf[ks] + buf[128 + ks] + buf[256 + ks] + buf[384 + ks];
      };
      // the head's max (lane j's slot) and the previous head's row sum (lane j+16's
      // otherwise unused slot) in one reduction
      auto own_max_sum = [&](float pmax, float psum, float* buf, float& m, float& l) {
        pmax = fmaxf(pmax, __shfl_xor_sync(0xffffffffu, pmax, 16));
        psum += __shfl_xor_sync(0xffffffffu, psum, 16);
        buf[g * 128 + r] = hh ? psum : pmax;
        named_bar(bar_id, 128);
        m = fmaxf(fmaxf(buf[ks], buf[128 + ks]), fmaxf(buf[256 + ks], buf[384 + ks]));
        l = buf[ks + 16] + buf[144 + ks] + buf[272 + ks] + buf[400 + ks];
      };
      // LayerNorm of u (columns cc.. of an own row) in place, two-pass statistics (the mean
      // reduced in bm, the variance in bv: consecutive reductions use different buffers)
      auto layer_norm16 = [&](const float* gamma, const float* beta, float* bm, float* bv) {
        uint64_t a0 = f2pk(0.f, 0.f), a1 = a0;
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          a0 = f2add(a0, f2pk(u[i], u[i + 1]));
          a1 = f2add(a1, f2pk(u[i + 2], u[i + 3]));
        }
        float t0, t1, t2, t3;
        f2upk(a0, t0, t1);
        f2upk(a1, t2, t3);
        const float mean = own_sum((t0 + t2) + (t1 + t3), bm) * (1.f / 128.f);
        const uint64_t nm = f2pk(-mean, -mean);
        a0 = f2pk(0.f, 0.f);
        a1 = a0;
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const uint64_t d0 = f2add(f2pk(u[i], u[i + 1]), nm), d1 = f2add(f2pk(u[i + 2], u[i + 3]), nm);
          a0 = f2fma(d0, d0, a0);
          a1 = f2fma(d1, d1, a1);
          f2upk(d0, u[i], u[i + 1]);
          f2upk(d1, u[i + 2], u[i + 3]);
        }
        f2upk(a0, t0, t1);
        f2upk(a1, t2, t3);
        const float rstd = rsqrtf(own_sum((t0 + t2) + (t1 + t3), bv) * (1.f / 128.f) + p.eps);
        const uint64_t rs = f2pk(rstd, rstd);
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const float4 gg = *reinterpret_cast<const float4*>(gamma + cc + i);
          const float4 bb = *reinterpret_cast<const float4*>(beta + cc + i);
          f2upk(f2fma(f2mul(f2pk(u[i], u[i + 1]), rs), f2pk(gg.x, gg.y), f2pk(bb.x, bb.y)), u[i], u[i + 1]);
          f2upk(f2fma(f2mul(f2pk(u[i + 2], u[i + 3]), rs), f2pk(gg.z, gg.w), f2pk(bb.z, bb.w)), u[i + 2], u[i + 3]);
        }
      };
      // u as 16 fp16 values at columns cc of a 128-wide SW128 tile, into both lanes of the own row
      auto store16_sw128 = [&](uint8_t* base) {
        uint8_t* atom = base + (cc >> 6) * 16384;
        const int ch = (cc & 63) >> 3;
        const uint4 a = make_uint4(pack_half2(u[0], u[1]), pack_half2(u[2], u[3]), pack_half2(u[4], u[5]),
                                   pack_half2(u[6], u[7]));
        const uint4 b = make_uint4(pack_half2(u[8], u[9]), pack_half2(u[10], u[11]), pack_half2(u[12], u[13]),
                                   pack_half2(u[14], u[15]));
        *reinterpret_cast<uint4*>(atom + sw128_off(r, ch)) = a;
        *reinterpret_cast<uint4*>(atom + sw128_off(r, ch + 1)) = b;
        *reinterpret_cast<uint4*>(atom + sw128_off(r ^ 16, ch)) = a;
        *reinterpret_cast<uint4*>(atom + sw128_off(r ^ 16, ch + 1)) = b;
      };
      // v (32 values) as fp16 row `row` of a 128x32 SW64 tile
      auto store_sw64_row = [&](uint8_t* base, int row) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(base + row * 64 + ((j ^ ((row >> 1) & 3)) << 4)) =
              make_uint4(pack_half2(v[8 * j], v[8 * j + 1]), pack_half2(v[8 * j + 2], v[8 * j + 3]),
                         pack_half2(v[8 * j + 4], v[8 * j + 5]), pack_half2(v[8 * j + 6], v[8 * j + 7]));
      };
      auto load_x_row = [&](int row) {  // 32 fp32 columns c0.. of sequence row `row` from XIN
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 t = *reinterpret_cast<const float4*>(xin_box + sw128_off(row, j));
          v[4 * j] = t.x; v[4 * j + 1] = t.y; v[4 * j + 2] = t.z; v[4 * j + 3] = t.w;
        }
      };

      // ---- W1: the own row's x -> residual in TMEM [384,512); LN1 of natural row r -> XA
      stage_vectors(0);
      wait_w(SB_XFULL, 0);
      load_x_row(srow);
      if (ok) tmem_st32(trow + 384 + c0, v);
      load_x_row(r);
      layer_norm(vec + C::V_LN1W, vec + C::V_LN1B, 0);
      store_sw128(xa);
      publish(SB_N1);
      // ---- W2: QKV (natural rows) -> K, V tiles; Q of own rows into both of their tile rows
      wait_w(SB_QKV_DONE, 0);
#pragma unroll 1
      for (int nt = 0; nt < 3; ++nt) {
        if (ok) tmem_ld32(trow + nt * 128 + c0, v);
        f2_add_bias32(v, vec + C::V_BQKV + nt * 128 + c0);
        uint8_t* tile = smem + (nt == 0 ? C::OFF_Q : nt == 1 ? C::OFF_K : C::OFF_V) + g * 8192;
        if (nt > 0) {
          store_sw64_row(tile, r);
        } else if (kn >= 0) {
          const int i1 = (kn >> 4) * 32 + (kn & 15);
          store_sw64_row(tile, i1);
          store_sw64_row(tile, i1 + 16);
        }
      }
      publish(SB_QKV_SMEM);
      // ---- W3: softmax per head (own row srow, keys cc..cc+15)
      uint32_t kvalid;
      {
        const int key = c0 + lane;
        bool v_ok = key < p.seq_len;
        if (v_ok && p.row_valid != nullptr) v_ok = p.row_valid[static_cast<int64_t>(seq) * p.seq_len + key] != 0;
        kvalid = (__ballot_sync(0xffffffffu, v_ok) >> (16 * hh)) & 0xffffu;
      }
      if (!p.non_causal) kvalid &= (srow >= cc + 15) ? 0xffffu : (srow < cc ? 0u : (0xffffu >> (15 - (srow - cc))));
      float my_l = 1.f;  // softmax denominator of head hg
      float prev_sum = 0.f;  // the previous head's partial row sum, reduced with this head's max
#pragma unroll 1
      for (int h = 0; h < H; ++h) {
        wait_w(SB_S_FULL + (h & 1), par(0, (h & 1) ? H / 2 : (H + 1) / 2, h >> 1));
        if (ok) tmem_ld32(trow + (h & 1) * 128 + c0, v);
        take_half();
        if (kvalid != 0xffffu) {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (!((kvalid >> i) & 1u)) u[i] = -INFINITY;
        }
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < 16; i += 2) mx = fmax3(mx, u[i], u[i + 1]);
        float m, lprev;
        own_max_sum(mx, prev_sum, (h & 1) ? st1 : st0, m, lprev);  // reductions alternate st0/st1 strictly
        if (h > 0 && h - 1 == hg) my_l = lprev;
        // a row that sees no key (its mask excludes every visible key) keeps P = 0 and a zero
        // context, as the reference's masked-out rows end up after their block (TTB:163-164)
        m = (m == -INFINITY) ? 0.f : m * p.scale_log2;
        const uint64_t sc = f2pk(p.scale_log2, p.scale_log2), nm = f2pk(-m, -m);
        uint64_t a0 = f2pk(0.f, 0.f), a1 = a0;
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          float e0, e1, e2, e3;
          f2upk(f2fma(f2pk(u[i], u[i + 1]), sc, nm), e0, e1);
          f2upk(f2fma(f2pk(u[i + 2], u[i + 3]), sc, nm), e2, e3);
          u[i] = fast_exp2(e0); u[i + 1] = fast_exp2(e1); u[i + 2] = fast_exp2(e2); u[i + 3] = fast_exp2(e3);
          a0 = f2add(a0, f2pk(u[i], u[i + 1]));
          a1 = f2add(a1, f2pk(u[i + 2], u[i + 3]));
        }
        float t0, t1, t2, t3;
        f2upk(a0, t0, t1);
        f2upk(a1, t2, t3);
        const float sum = (t0 + t2) + (t1 + t3);
        if (h > 0) wait_w(SB_PV_DONE, par(0, H, h - 1));  // P of the previous head consumed
        store16_sw128(smem + C::OFF_P);
        publish(SB_P_FULL);
        prev_sum = sum;
      }
      {
        const float lf = own_sum(prev_sum, st_f);  // the last head's sum
        if (hg == H - 1) my_l = lf;
      }
      // ---- W4: context (16 columns of head hg) = O / l -> XA
      wait_w(SB_PV_DONE, par(0, H, H - 1));
      if (ok) tmem_ld32(trow + 256 + c0, v);
      take_half();
      {
        const float inv = my_l > 0.f ? 1.f / my_l : 0.f;
        const uint64_t iv = f2pk(inv, inv);
#pragma unroll
        for (int i = 0; i < 16; i += 2) f2upk(f2mul(f2pk(u[i], u[i + 1]), iv), u[i], u[i + 1]);
      }
      store16_sw128(xa);
      publish(SB_CTX);
      // ---- W5: x1 = (x + ctx.Wo^T, in TMEM) + bo, kept in TMEM without bo (ffn_out
      // accumulates onto it; W7 adds bo and b2) ; LN2 -> XA
      wait_w(SB_OP_DONE, 0);
      if (ok) tmem_ld32(trow + 384 + c0, v);
      take_half();
      add16(vec + C::V_BO + cc);
      layer_norm16(vec + C::V_LN2W, vec + C::V_LN2B, st_o, st_f);  // after st_f (the last softmax sum)
      store16_sw128(xa);
      publish(SB_N2);
      // ---- W6: GELU chunks -> H ping-pong
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        const int b = c & 1;
        wait_w(SB_FIN + b, par(0, b ? per_b1 : per_b0, c >> 1));
        if (ok) tmem_ld32(trow + b * 128 + c0, v);
        take_half();
        add16(vec + C::V_BIN + c * 128 + cc);
#pragma unroll
        for (int i = 0; i < 16; i += 2) gelu_as2(u[i], u[i + 1]);
        if (c >= 2) wait_w(SB_HFREE + b, par(0, b ? per_b1 : per_b0, (c >> 1) - 1));
        store16_sw128(smem + (b ? C::OFF_K : C::OFF_Q));
        publish(SB_H + b);
      }
      // ---- W7: x2 = (x + attn + ffn, in TMEM) + bo + b2 ; final LayerNorm -> y (16 rows x 32 columns per warp)
      wait_w(SB_FOUT, 0);
      if (ok) tmem_ld32(trow + 384 + c0, v);
      take_half();
      add16(vec + C::V_BO + cc);
      add16(vec + C::V_BOUT + cc);
      layer_norm16(vec + C::V_LNFW, vec + C::V_LNFB, st_o, st_f);
      {
        const bool zero = srow < p.seq_len && p.row_valid != nullptr && p.row_valid[srow_g] == 0;
        // the warp's own rows are 16 consecutive sequence rows: one 16x32 box, staged SW128
        uint8_t* ybox = smem + C::OFF_YST + (q * 4 + g) * 2048;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<float4*>(ybox + sw128_off(lane & 15, 4 * hh + j)) =
              zero ? make_float4(0.f, 0.f, 0.f, 0.f) : make_float4(u[4 * j], u[4 * j + 1], u[4 * j + 2], u[4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && ok) {
          tma_store_3d(tm_y, ybox, c0, half ? 32 + 16 * q : (q < 2 ? 16 * q : 64 + 16 * q), seq);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait_all();  // the last y stores are complete before the CTA exits
    // after an abort, the last vector copies land before shared memory is released
    if (wtid == 0 && *abort_flag && nstaged > 0) mbar_wait_drain(&bar[SB_VFULL], static_cast<uint32_t>((nstaged - 1) & 1));
  }
  tc_fence_before();
  __syncwarp();  // lane-0 roles rejoin their warp: bar.sync is warp-aligned
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int NH>
__global__ void __launch_bounds__(SmallCfg::THREADS, 1)
    k_block_small(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_o,
                  const __grid_constant__ CUtensorMap tm_in, const __grid_constant__ CUtensorMap tm_out,
                  const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_y,
                  const SmallParams p) {
  block_small_body<false, NH>(&tm_qkv, &tm_o, &tm_in, &tm_out, &tm_x, &tm_y, p);
}

// Row-split mode for one layer and at most one sequence per two SMs: CTAs 2s
// and 2s+1 both run sequence s, each finishing 64 of its query rows (tm_y has
// 16-row boxes).  No data moves between the two CTAs: each computes LN1, K and
// V for all 128 rows itself, which costs less than exchanging them.
template <int NH>
__global__ void __launch_bounds__(SmallCfg::THREADS, 1)
    k_block_rows(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_o,
                 const __grid_constant__ CUtensorMap tm_in, const __grid_constant__ CUtensorMap tm_out,
                 const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_y,
                 const SmallParams p) {
  block_small_body<true, NH>(&tm_qkv, &tm_o, &tm_in, &tm_out, &tm_x, &tm_y, p);
}

}  // namespace b200
