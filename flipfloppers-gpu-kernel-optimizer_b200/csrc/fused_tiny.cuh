// Fused block for tiny models: d_model = 32 (head_dim 8, 16 or 32), ffn_dim a
// multiple of 32 up to 128, seq_len <= 128, any number of layers.
//
// The reference's official matrix has such a shape (d=32 H=4 ffn=32, 4
// layers; run_eval.sh:44-58).  At d = 32 a 128-row tcgen05 tile would be
// mostly padding in attention (head_dim 8) and every stage of the per-layer
// kernel chain is a few microseconds of launch and prologue around almost no
// arithmetic, so the whole model runs in one kernel on the CUDA cores.
//
// What bounds it is shared memory, not arithmetic: a 128-bit shared load
// costs four wavefronts even when every lane of a quarter-warp reads the
// same address, so the design goal is few loaded bytes per multiply-add.
// One CTA per sequence (512 threads), or, when the sequences leave SMs idle,
// a cluster of two CTAs per sequence (512 threads each, 64 causally balanced
// rows each, K/V rows exchanged through distributed shared memory; see the
// kernel).  A group of G adjacent lanes (an octet, G = 8, with one CTA per
// sequence; G = 16 in the cluster) owns the row pair (2i, 2i+1) and thread u
// of the group owns columns C*u .. C*u + C-1 of both rows (C = 32 / G; the
// residual stream lives in registers).  Every projection is a register-blocked
// product over the pair: each weight loaded from shared memory feeds both rows,
// each activation load feeds 2 to 12 outputs (QKV: 3*C outputs x 2 rows per
// thread).  LayerNorm statistics combine over the group with shuffles.
// Attention at head_dim 8 gives each thread a (head, key residue) of the pair,
// so one K / V load serves two query rows; at head_dim 16 / 32 a thread takes
// one row and a share of its keys.  Partial softmaxes merge with shuffles.
// Weights are staged as fp32 in shared memory (the next layer's fp16 copies
// arrive by bulk copy during this one) with 4 floats of padding after every C
// rows, so the 8 rows a quarter-warp reads in one instruction fall on distinct
// bank groups.
//
// Matrix products accumulate in fp32 from the fp16 weight copies the other
// paths use, as f32x2 pairs (even / odd k) in independent chains.
#pragma once

#include "ptx.cuh"

namespace b200 {

struct TinyParams {
  int num_seq, seq_len, layers, heads, ffn;
  const float* x;  // [num_seq*seq_len, 32]
  float* y;
  const float* ln1_w; const float* ln1_b;   // [layers, 32]
  const __half* w_qkv;                      // [layers, 96, 32]
  const float* b_qkv;                       // [layers, 96]
  const __half* w_o;                        // [layers, 32, 32]
  const float* b_o;                         // [layers, 32]
  const float* ln2_w; const float* ln2_b;   // [layers, 32]
  const __half* w_in;                       // [layers, ffn, 32]
  const float* b_in;                        // [layers, ffn]
  const __half* w_out;                      // [layers, 32, ffn]
  const float* b_out;                       // [layers, 32]
  const float* lnf_w; const float* lnf_b;   // [32]
  float eps;
  float scale_log2;                         // head_dim^-0.5 * log2(e)
  const unsigned char* row_valid;           // [num_seq*seq_len], may be null
  int non_causal;
};

// floats of a [rows][ld] weight staged with 4 floats of padding after every P rows
constexpr int tiny_padded(int rows, int ld, int P) { return rows * ld + (rows / P) * 4; }

// SPLIT = false: one CTA per sequence, 512 threads, an octet (G = 8 lanes) per row
// pair, 4 columns per thread.  SPLIT = true: a cluster of two CTAs per sequence,
// each owning 64 rows with 512 threads, a group of G = 16 lanes per row pair, 2
// columns per thread (the K / V rows the other CTA needs cross over distributed
// shared memory).  Weights are padded with 4 floats after every C rows (C =
// columns per thread): the C-row stripes the 8 lanes of a quarter-warp read in one
// instruction then fall on 8 distinct bank groups.
template <bool SPLIT>
struct TinyCfgT {
  static constexpr int D = 32;
  static constexpr int S = 128;                 // rows per sequence
  static constexpr int RL = SPLIT ? 64 : 128;   // rows owned by a CTA
  static constexpr int G = SPLIT ? 16 : 8;      // lanes per row pair
  static constexpr int C = D / G;               // columns per thread (4 or 2)
  static constexpr int THREADS = RL * G / 2;    // 512
  static constexpr int KVB = SPLIT ? 2 : 1;     // K / V buffers (by layer parity when split)
  static constexpr int FMAX = 128;
  static constexpr int LD = D + 4;       // row stride (floats) of the K / V / row buffers
  static constexpr int HL = FMAX + 4;    // row stride of the hidden-unit buffer
  // shared memory (floats)
  static constexpr int W_QKV = 0;                                  // [96][32]
  static constexpr int W_O = W_QKV + tiny_padded(3 * D, D, C);     // [32][32]
  static constexpr int W_IN = W_O + tiny_padded(D, D, C);          // [FMAX][32]
  static constexpr int W_OUT = W_IN + tiny_padded(FMAX, D, C);     // [32][ffn]
  static constexpr int VEC = W_OUT + tiny_padded(D, FMAX, C);      // ln1 w,b | b_qkv | b_o | ln2 w,b | b_in | b_out
  static constexpr int V_LN1W = 0, V_LN1B = 32, V_BQKV = 64, V_BO = 160, V_LN2W = 192, V_LN2B = 224, V_BIN = 256,
                       V_BOUT = 256 + FMAX, V_TOTAL = 288 + FMAX;
  static constexpr int KS = VEC + V_TOTAL;              // [KVB][S][LD] keys
  static constexpr int VS = KS + KVB * S * LD;          // [KVB][S][LD] values
  static constexpr int NB = VS + KVB * S * LD;          // [RL][LD] a row's LN output, then Q, then the context
  static constexpr int HB = NB + RL * LD;               // [RL][HL] GELU(hidden units)
  // the next layer's fp16 weights and fp32 vectors as they arrive by bulk copy
  // (row-major, unpadded; the vectors in the VEC layout), converted into the
  // regions above at the layer boundary
  static constexpr int STG_QKV = HB + RL * HL;          // [96][32] fp16
  static constexpr int STG_O = STG_QKV + 3 * D * D / 2; // [32][32] fp16
  static constexpr int STG_IN = STG_O + D * D / 2;      // [ffn][32] fp16
  static constexpr int STG_OUT = STG_IN + FMAX * D / 2; // [32][ffn] fp16
  static constexpr int STG_VEC = STG_OUT + D * FMAX / 2;
  static constexpr int BAR = STG_VEC + V_TOTAL;         // weight mbarrier, abort flag, 2 exchange mbarriers
  static constexpr int TOTAL_FLOATS = BAR + 8;
  static constexpr int TOTAL = TOTAL_FLOATS * 4;
  static_assert(TOTAL <= 232448, "shared memory");
  static_assert(W_O % 4 == 0 && W_IN % 4 == 0 && W_OUT % 4 == 0 && VEC % 4 == 0 && KS % 4 == 0 && NB % 4 == 0 &&
                    HB % 4 == 0 && STG_QKV % 4 == 0 && STG_VEC % 4 == 0 && BAR % 2 == 0,
                "16-byte aligned regions");
};
using TinyCfg = TinyCfgT<false>;

// offset (floats) of row `row` of a weight staged with row stride ld, padded every C rows
template <int C>
__device__ __forceinline__ int tiny_row(int row, int ld) {
  return row * ld + (row / C) * 4;
}

// sum over the G lanes of a row pair's group (adjacent lanes)
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = 1; o < G; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// C consecutive floats at p (aligned to 4*C bytes) -> v / v -> p
template <int C>
__device__ __forceinline__ void ldc(const float* p, float (&v)[C]) {
  if constexpr (C == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  } else {
    const float2 a = *reinterpret_cast<const float2*>(p);
    v[0] = a.x; v[1] = a.y;
  }
}
template <int C>
__device__ __forceinline__ void stc(float* p, const float (&v)[C]) {
  if constexpr (C == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  }
}

// LayerNorm of a 32-wide row held as C columns per thread of its G-lane group
// (two-pass statistics); gamma / beta: this thread's C parameters
template <int G, int C>
__device__ __forceinline__ void tiny_layer_norm(float (&v)[C], const float* gamma, const float* beta, float eps) {
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < C; ++i) t += v[i];
  const float mean = group_sum<G>(t) * (1.f / 32.f);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < C; ++i) {
    v[i] -= mean;
    sq = fmaf(v[i], v[i], sq);
  }
  const float rstd = rsqrtf(group_sum<G>(sq) * (1.f / 32.f) + eps);
  float g[C], b[C];
  ldc<C>(gamma, g);
  ldc<C>(beta, b);
#pragma unroll
  for (int i = 0; i < C; ++i) v[i] = fmaf(v[i] * rstd, g[i], b[i]);
}

// acc[r][C*g + i] += sum_k a_r[k] * W[32g + C*u + i][k0 + k] for k in [0, 32), rows
// r = 0, 1 (a0 / a1: the two rows' 32 activations in shared memory, W: row-major
// weight with row stride ld, padded every C rows).  Per 4-k step: two activation
// loads and C*NG weight loads feed 4*C*NG multiply-adds.  Accumulators are f32x2
// pairs of the even / odd k partial sums.
template <int NG, int C>
__device__ __forceinline__ void tiny_mm32(const float* a0, const float* a1, const float* W, int ld, int u, int k0,
                                          uint64_t (&acc)[2][C * NG]) {
  const float* wb = W + tiny_row<C>(C * u, ld) + k0;
#pragma unroll
  for (int k = 0; k < 32; k += 4) {
    const float4 x0 = *reinterpret_cast<const float4*>(a0 + k);
    const float4 x1 = *reinterpret_cast<const float4*>(a1 + k);
    const uint64_t x0a = f2pk(x0.x, x0.y), x0b = f2pk(x0.z, x0.w);
    const uint64_t x1a = f2pk(x1.x, x1.y), x1b = f2pk(x1.z, x1.w);
#pragma unroll
    for (int g = 0; g < NG; ++g) {
#pragma unroll
      for (int i = 0; i < C; ++i) {
        // row 32g + C*u + i: (32g + C*u + i) * ld + (32g / C + u) * 4
        const float4 w = *reinterpret_cast<const float4*>(wb + g * (32 * ld + 128 / C) + i * ld + k);
        const uint64_t wa = f2pk(w.x, w.y), wc = f2pk(w.z, w.w);
        acc[0][C * g + i] = f2fma(x0b, wc, f2fma(x0a, wa, acc[0][C * g + i]));
        acc[1][C * g + i] = f2fma(x1b, wc, f2fma(x1a, wa, acc[1][C * g + i]));
      }
    }
  }
}

template <int N>
__device__ __forceinline__ void tiny_zero(uint64_t (&acc)[2][N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) acc[0][i] = acc[1][i] = 0ull;
}

// the C outputs Cg .. Cg+C-1 of row r of an accumulator, plus the bias at b
template <int C, int N>
__device__ __forceinline__ void tiny_out(const uint64_t (&acc)[2][N], int r, int g, const float* b, float (&o)[C]) {
  float bb[C];
  ldc<C>(b, bb);
#pragma unroll
  for (int i = 0; i < C; ++i) {
    float e, d;
    f2upk(acc[r][C * g + i], e, d);
    o[i] = bb[i] + (e + d);
  }
}

// fp16 weight [rows][ld] (shared memory, as staged) -> fp32 shared memory padded every
// C rows (ld a multiple of 8), all threads of the CTA
template <int C>
__device__ __forceinline__ void tiny_stage_f16(float* dst, const __half* src, int rows, int ld) {
  for (int i = static_cast<int>(threadIdx.x) * 8; i < rows * ld; i += static_cast<int>(blockDim.x) * 8) {
    const uint4 t = *reinterpret_cast<const uint4*>(src + i);
    const __half2* h2 = reinterpret_cast<const __half2*>(&t);
    const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]), f2 = __half22float2(h2[2]),
                 f3 = __half22float2(h2[3]);
    float* d = dst + tiny_row<C>(i / ld, ld) + i % ld;
    *reinterpret_cast<float4*>(d) = make_float4(f0.x, f0.y, f1.x, f1.y);
    *reinterpret_cast<float4*>(d + 4) = make_float4(f2.x, f2.y, f3.x, f3.y);
  }
}

// Attention of a row pair's G-lane group for head_dim HD; thread u of the group whose
// row pair starts at r0 (nbp: the pair's two rows of NB; ks / vs: the key and value
// rows of the sequence).  Q of the rows is in NB (its columns head*HD..); the
// context of each (row, head) goes back to the same place.  Head_dim 8: a thread
// takes both rows of the pair, one head and every T-th key (one K / V load serves
// two rows); head_dim 16 / 32: one row, one head and every T-th key (T = the
// group's threads per (rows, head): 2 or 4 for octets, 4 or 8 for 16-lane
// groups).  Online softmax in the log2 domain per row; the T threads of a (rows,
// head) merge their partial (max, sum, context) with shuffles.  Keys are walked in
// blocks of 32 (kw: key validity words, bit i of word w = key 32w + i exists and is
// not padding); masked keys are skipped, never weighted by zero.
template <int HD, int G>
__device__ __forceinline__ void tiny_attention(const float* ks, const float* vs, float* nbp, int u, int r0,
                                               const uint32_t (&kw)[4],
                                               const TinyParams& p) {
  using C = TinyCfg;
  constexpr int H = C::D / HD;
  constexpr int R = HD == 8 ? 2 : 1;       // query rows per thread
  constexpr int TPR = R == 2 ? G : G / 2;  // threads sharing a row set
  constexpr int T = TPR / H;               // threads per (row set, head)
  constexpr int KB = 32 / T;               // keys per thread per 32-key block
  constexpr int VPT = R * HD / T;          // context values each thread writes (8 or 4)
  const int idx = R == 2 ? u : (u % TPR);
  const int rbase = R == 2 ? r0 : r0 + u / TPR;
  // heads on the low lane bits: the 8 lanes of a quarter-warp then read K / V rows of
  // different heads and key residues whose 16-byte chunks fall on distinct banks
  const int head = idx % H, sub = idx / H;
  const int kend = p.non_causal ? p.seq_len : min(rbase + R, p.seq_len);  // keys 0..kend-1 may be visible

  uint64_t q2[R][HD / 2], o[R][HD / 2];
  float m[R], l[R];
#pragma unroll
  for (int rr = 0; rr < R; ++rr) {
    const float* qr = nbp + (rbase - r0 + rr) * C::LD + head * HD;
#pragma unroll
    for (int e = 0; e < HD; e += 4) {
      const float4 a = *reinterpret_cast<const float4*>(qr + e);
      q2[rr][e / 2] = f2pk(a.x * p.scale_log2, a.y * p.scale_log2);  // scores come out in log2 units
      q2[rr][e / 2 + 1] = f2pk(a.z * p.scale_log2, a.w * p.scale_log2);
      o[rr][e / 2] = o[rr][e / 2 + 1] = 0ull;
    }
    m[rr] = -INFINITY;
    l[rr] = 0.f;
  }
  for (int kb = 0; kb < kend; kb += 32) {
    const uint32_t word = (kb < 32 ? kw[0] : kb < 64 ? kw[1] : kb < 96 ? kw[2] : kw[3]) >> sub;
    float s[R][KB];
    float mb[R];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) mb[rr] = -INFINITY;
#pragma unroll
    for (int jj = 0; jj < KB; ++jj) {
      const int j = kb + sub + jj * T;
      float acc[R];
#pragma unroll
      for (int rr = 0; rr < R; ++rr) acc[rr] = -INFINITY;
      if (j < kend && ((word >> (jj * T)) & 1u)) {
        const float* kr = ks + j * C::LD + head * HD;
        uint64_t a2[R];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) a2[rr] = 0ull;
#pragma unroll
        for (int e = 0; e < HD; e += 4) {
          const float4 kk = *reinterpret_cast<const float4*>(kr + e);
          const uint64_t ka = f2pk(kk.x, kk.y), kc = f2pk(kk.z, kk.w);
#pragma unroll
          for (int rr = 0; rr < R; ++rr) a2[rr] = f2fma(q2[rr][e / 2 + 1], kc, f2fma(q2[rr][e / 2], ka, a2[rr]));
        }
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          if (p.non_causal || j <= rbase + rr) {
            float lo, hi;
            f2upk(a2[rr], lo, hi);
            acc[rr] = lo + hi;
          }
        }
      }
#pragma unroll
      for (int rr = 0; rr < R; ++rr) {
        s[rr][jj] = acc[rr];
        mb[rr] = fmaxf(mb[rr], acc[rr]);
      }
    }
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      if (mb[rr] != -INFINITY) {  // rows with no visible key in this block keep their state
        const float mn = fmaxf(m[rr], mb[rr]);
        const float corr = fast_exp2(m[rr] - mn);  // 0 on the row's first visible block
        l[rr] *= corr;
        const uint64_t c2 = f2pk(corr, corr);
#pragma unroll
        for (int e = 0; e < HD / 2; ++e) o[rr][e] = f2mul(o[rr][e], c2);
        m[rr] = mn;
      }
    }
#pragma unroll
    for (int jj = 0; jj < KB; ++jj) {
      bool any = false;
#pragma unroll
      for (int rr = 0; rr < R; ++rr) any |= s[rr][jj] != -INFINITY;
      if (any) {
        const float* vr = vs + (kb + sub + jj * T) * C::LD + head * HD;
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          // a masked score gives 0 here (exp2(-inf)) without touching l or o below
          const float pj = s[rr][jj] != -INFINITY ? fast_exp2(s[rr][jj] - m[rr]) : 0.f;
          s[rr][jj] = pj;
          l[rr] += pj;
        }
#pragma unroll
        for (int e = 0; e < HD; e += 4) {
          const float4 vv = *reinterpret_cast<const float4*>(vr + e);
          const uint64_t va = f2pk(vv.x, vv.y), vc = f2pk(vv.z, vv.w);
#pragma unroll
          for (int rr = 0; rr < R; ++rr) {
            if (R == 1 || s[rr][jj] != 0.f) {
              const uint64_t p2 = f2pk(s[rr][jj], s[rr][jj]);
              o[rr][e / 2] = f2fma(p2, va, o[rr][e / 2]);
              o[rr][e / 2 + 1] = f2fma(p2, vc, o[rr][e / 2 + 1]);
            }
          }
        }
      }
    }
  }
  // merge the partial softmaxes of the T threads of a (rows, head) (lanes H apart)
#pragma unroll
  for (int off = H; off < H * T; off <<= 1) {
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m[rr], off), l2 = __shfl_xor_sync(0xffffffffu, l[rr], off);
      const float mm = fmaxf(m[rr], m2);
      const float a = (m[rr] == -INFINITY) ? 0.f : fast_exp2(m[rr] - mm);
      const float b2 = (m2 == -INFINITY) ? 0.f : fast_exp2(m2 - mm);
      l[rr] = l[rr] * a + l2 * b2;
      const uint64_t a_2 = f2pk(a, a), b_2 = f2pk(b2, b2);
#pragma unroll
      for (int e = 0; e < HD / 2; ++e) {
        const uint64_t other = __shfl_xor_sync(0xffffffffu, o[rr][e], off);
        o[rr][e] = f2fma(o[rr][e], a_2, f2mul(other, b_2));
      }
      m[rr] = mm;
    }
  }
  // each of the T threads writes 8 of the R*HD results: row sub % R, dims 8*(sub / R)..
  // each of the T threads writes VPT of the R*HD results: row sub % R, dims VPT*(sub / R)..
  const int rw = sub % R, dc = sub / R;
  uint64_t w[VPT / 2];
  float inv = 0.f;
#pragma unroll
  for (int rr = 0; rr < R; ++rr) {
    if (rr == rw) {
      inv = l[rr] > 0.f ? 1.f / l[rr] : 0.f;  // a row with no visible key (padding) gets 0
#pragma unroll
      for (int c = 0; c < HD / VPT; ++c)
        if (c == dc) {
#pragma unroll
          for (int e = 0; e < VPT / 2; ++e) w[e] = o[rr][(VPT / 2) * c + e];
        }
    }
  }
  __syncwarp();  // every thread of the group has read its Q
  const uint64_t inv2 = f2pk(inv, inv);
  float* dst = nbp + (rbase - r0 + rw) * C::LD + head * HD + VPT * dc;
  float v[VPT];
#pragma unroll
  for (int e = 0; e < VPT / 2; ++e) f2upk(f2mul(w[e], inv2), v[2 * e], v[2 * e + 1]);
#pragma unroll
  for (int e = 0; e < VPT; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
}

// SPLIT = false: one CTA per sequence (grid = sequences).  SPLIT = true: a cluster
// of two CTAs per sequence (grid = 2 x sequences, cluster dims 2): half 0 owns
// rows 0-31 and 96-127, half 1 rows 32-95 (equal causal work).  Each half
// computes K and V of its own rows and also stores the ones the other half
// attends to (half 1 needs keys 0-31, or all when non-causal; half 0 keys 32-95) into that CTA's
// shared memory, then arrives on the other CTA's exchange mbarrier (release at
// cluster scope) and waits, bounded, on its own.  The K / V buffers alternate by
// layer parity, so a half can write layer l+1's rows while the other still
// reads layer l's: it gets there only after the other half's layer-l arrival,
// which follows that half's layer-(l-1) attention.
template <int HD, bool SPLIT>
__global__ void __launch_bounds__(TinyCfgT<SPLIT>::THREADS, 1) k_block_tiny(const TinyParams p) {
  using C = TinyCfgT<SPLIT>;
  static_assert(HD == 8 || HD == 16 || HD == 32, "head_dim 8, 16 or 32");
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);

  griddep_sync();
  constexpr int G = C::G, CC = C::C;  // lanes per row pair, columns per thread
  constexpr int RW = 64 / G;          // rows per warp (a block): 8 or 4
  const int u = static_cast<int>(threadIdx.x) % G;   // columns CC*u .. CC*u + CC-1 of the group's rows
  const int gi = static_cast<int>(threadIdx.x) / G;  // the group (row pair) within the CTA
  // warp w holds the RW-row block b(w), its groups the row pairs b(w)*RW + 2k, + 1.
  // Warps w, w+4, w+8, w+12 share a scheduler; one CTA per sequence gives them
  // 8-row blocks s, 7-s, 8+s, 15-s (s = w % 4), which balances the causal
  // attention work across the four schedulers; split, 4-row blocks s, 7-s, 24+s,
  // 31-s (half 0: rows 0-31 and 96-127) or 8+s, 15-s, 16+s, 23-s (half 1: rows 32-95)
  const int wid = static_cast<int>(threadIdx.x >> 5), ws = wid & 3, wt = wid >> 2;
  uint32_t half = 0;
  int rblk;
  if constexpr (SPLIT) {
    half = cluster_ctarank();
    rblk = half == 0 ? (wt == 0 ? ws : wt == 1 ? 7 - ws : wt == 2 ? 24 + ws : 31 - ws)
                     : (wt == 0 ? 8 + ws : wt == 1 ? 15 - ws : wt == 2 ? 16 + ws : 23 - ws);
  } else {
    rblk = wt == 0 ? ws : wt == 1 ? 7 - ws : wt == 2 ? 8 + ws : 15 - ws;
  }
  const int r0 = rblk * RW + (gi % (32 / G)) * 2;  // the group's row pair r0, r0 + 1
  const int lr0 = gi * 2;                          // its rows in NB / HB (private to the group)
  const int seq = SPLIT ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int F = p.ffn;
  const bool ok0 = r0 < p.seq_len, ok1 = r0 + 1 < p.seq_len;
  const int64_t g0 = static_cast<int64_t>(seq) * p.seq_len + r0;  // global row of r0
  float* vec = sm + C::VEC;
  float* nb0 = sm + C::NB + lr0 * C::LD;
  float* nb1 = nb0 + C::LD;
  float* hb0 = sm + C::HB + lr0 * C::HL;
  float* hb1 = hb0 + C::HL;
  uint64_t* wbar = reinterpret_cast<uint64_t*>(sm + C::BAR);  // a layer's staged weights and vectors
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + C::BAR + 2);
  uint64_t* xbar = reinterpret_cast<uint64_t*>(sm + C::BAR + 4);  // [2] the other half's K / V rows, by layer parity
  // one thread copies layer l's weights and vectors into the staging area (twelve bulk
  // copies, one mbarrier phase): issued a layer ahead, so the HBM / L2 round trip
  // overlaps the previous layer's arithmetic instead of stalling every boundary
  auto fetch = [&](int l) {
    const uint32_t fb = 4u * static_cast<uint32_t>(F);  // bytes of b_in; w_in and w_out are 16 * fb each
    fence_proxy_async_smem();  // the previous layer's reads of the staging area come first
    mbar_arrive_expect_tx(wbar, 8192u + 1152u + 33u * fb);
    bulk_load(sm + C::STG_QKV, p.w_qkv + static_cast<int64_t>(l) * 96 * 32, 6144, wbar);
    bulk_load(sm + C::STG_O, p.w_o + static_cast<int64_t>(l) * 32 * 32, 2048, wbar);
    bulk_load(sm + C::STG_IN, p.w_in + static_cast<int64_t>(l) * F * 32, 16u * fb, wbar);
    bulk_load(sm + C::STG_OUT, p.w_out + static_cast<int64_t>(l) * 32 * F, 16u * fb, wbar);
    float* sv = sm + C::STG_VEC;
    bulk_load(sv + C::V_LN1W, p.ln1_w + l * 32, 128, wbar);
    bulk_load(sv + C::V_LN1B, p.ln1_b + l * 32, 128, wbar);
    bulk_load(sv + C::V_BQKV, p.b_qkv + l * 96, 384, wbar);
    bulk_load(sv + C::V_BO, p.b_o + l * 32, 128, wbar);
    bulk_load(sv + C::V_LN2W, p.ln2_w + l * 32, 128, wbar);
    bulk_load(sv + C::V_LN2B, p.ln2_b + l * 32, 128, wbar);
    bulk_load(sv + C::V_BIN, p.b_in + static_cast<int64_t>(l) * F, fb, wbar);
    bulk_load(sv + C::V_BOUT, p.b_out + l * 32, 128, wbar);
  };
  if (threadIdx.x == 0) {
    mbar_init(wbar, 1);
    if (SPLIT) {
      mbar_init(&xbar[0], C::THREADS);  // every thread of the other half arrives once per layer
      mbar_init(&xbar[1], C::THREADS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) fetch(0);
  // layer whose weight copy is in flight and not yet waited for (-1: none); the same
  // value in every thread (the fetch schedule does not depend on data)
  int pending = 0;
  bool aborted = false;
  // shared::cluster addresses of the other half's K / V buffers and exchange barriers
  uint32_t peer_ks = 0, peer_vs = 0, peer_xbar = 0;
  if constexpr (SPLIT) {
    cluster_sync_all();  // both halves' barriers are initialised before any remote arrival
    peer_ks = mapa_shared(smem_u32(sm + C::KS), half ^ 1u);
    peer_vs = mapa_shared(smem_u32(sm + C::VS), half ^ 1u);
    peer_xbar = mapa_shared(smem_u32(xbar), half ^ 1u);
  }
  // key validity as four 32-bit words in registers (lane i tests key 32w + i)
  uint32_t kw[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int j = 32 * w + (threadIdx.x & 31);
    kw[w] = __ballot_sync(0xffffffffu, j < p.seq_len && (p.row_valid == nullptr ||
                                                          p.row_valid[static_cast<int64_t>(seq) * p.seq_len + j] != 0));
  }

  float x0[CC], x1[CC];  // the residual stream
#pragma unroll
  for (int i = 0; i < CC; ++i) x0[i] = x1[i] = 0.f;
  if (ok0) ldc<CC>(p.x + g0 * 32 + CC * u, x0);
  if (ok1) ldc<CC>(p.x + (g0 + 1) * 32 + CC * u, x1);

  for (int l = 0; l < p.layers; ++l) {
    __syncthreads();  // the previous layer's weights, K / V and row buffers are no longer read
    // layer l's staged copies -> fp32 weights (padded layout) and vectors
    const bool got = mbar_wait(wbar, static_cast<uint32_t>(l & 1), abort_flag, DERR_WAIT_TMA);
    if (got) {
      tiny_stage_f16<CC>(sm + C::W_QKV, reinterpret_cast<const __half*>(sm + C::STG_QKV), 96, 32);
      tiny_stage_f16<CC>(sm + C::W_O, reinterpret_cast<const __half*>(sm + C::STG_O), 32, 32);
      tiny_stage_f16<CC>(sm + C::W_IN, reinterpret_cast<const __half*>(sm + C::STG_IN), F, 32);
      tiny_stage_f16<CC>(sm + C::W_OUT, reinterpret_cast<const __half*>(sm + C::STG_OUT), 32, F);
      if (threadIdx.x < C::V_TOTAL / 4)
        reinterpret_cast<float4*>(vec)[threadIdx.x] = reinterpret_cast<const float4*>(sm + C::STG_VEC)[threadIdx.x];
    }
    // a copy that never landed (bounded wait, error recorded) ends the layer loop here
    if (__syncthreads_or(!got)) {
      aborted = true;
      break;
    }
    pending = -1;
    if (l + 1 < p.layers) {
      if (threadIdx.x == 0) fetch(l + 1);
      pending = l + 1;
    }

    // ---- LN1 -> NB
    {
      float t0[CC], t1[CC];
#pragma unroll
      for (int i = 0; i < CC; ++i) t0[i] = x0[i], t1[i] = x1[i];
      tiny_layer_norm<G, CC>(t0, vec + C::V_LN1W + CC * u, vec + C::V_LN1B + CC * u, p.eps);
      tiny_layer_norm<G, CC>(t1, vec + C::V_LN1W + CC * u, vec + C::V_LN1B + CC * u, p.eps);
      stc<CC>(nb0 + CC * u, t0);
      stc<CC>(nb1 + CC * u, t1);
    }
    __syncwarp();
    // ---- QKV: columns CC*u.. of Q, K and V for both rows; Q -> NB, K / V -> KS / VS
    const int kvo = SPLIT ? (l & 1) * C::S * C::LD : 0;  // this layer's K / V buffer
    float* ksl = sm + C::KS + kvo;
    float* vsl = sm + C::VS + kvo;
    {
      uint64_t acc[2][3 * CC];
      tiny_zero(acc);
      tiny_mm32<3, CC>(nb0, nb1, sm + C::W_QKV, 32, u, 0, acc);
      float o[CC];
      __syncwarp();  // the group has read its LN rows (Q overwrites them)
      tiny_out<CC>(acc, 0, 0, vec + C::V_BQKV + CC * u, o);
      stc<CC>(nb0 + CC * u, o);
      tiny_out<CC>(acc, 1, 0, vec + C::V_BQKV + CC * u, o);
      stc<CC>(nb1 + CC * u, o);
      // the other half attends to these rows: half 1 needs keys 0-31 (all keys when
      // non-causal), half 0 keys 32-95
      const bool send = SPLIT && (half == 1 || r0 < 32 || p.non_causal);
#pragma unroll
      for (int t = 0; t < 4; ++t) {  // K row r0, K row r0+1, V row r0, V row r0+1
        tiny_out<CC>(acc, t & 1, 1 + (t >> 1), vec + C::V_BQKV + 32 * (1 + (t >> 1)) + CC * u, o);
        const int off = kvo + (r0 + (t & 1)) * C::LD + CC * u;
        stc<CC>(sm + ((t >> 1) ? C::VS : C::KS) + off, o);
        if (send) {
          const uint32_t dst = ((t >> 1) ? peer_vs : peer_ks) + 4u * static_cast<uint32_t>(off);
          if constexpr (CC == 4) st_cluster_f4(dst, make_float4(o[0], o[1], o[2], o[3]));
          else st_cluster_f2(dst, make_float2(o[0], o[1]));
        }
      }
    }
    bool have_kv = true;
    if constexpr (SPLIT) {
      mbar_arrive_cluster(peer_xbar + 8u * static_cast<uint32_t>(l & 1));
      have_kv = mbar_wait_cluster(&xbar[l & 1], static_cast<uint32_t>((l >> 1) & 1), abort_flag, DERR_WAIT_GRID);
    }
    // every row's K and V are in place (a bounded exchange wait that gave up ends the loop)
    if (__syncthreads_or(!have_kv)) {
      aborted = true;
      break;
    }
    // ---- attention -> the context in NB
    tiny_attention<HD, G>(ksl, vsl, nb0, u, r0, kw, p);
    __syncwarp();
    // ---- out_proj + residual; LN2 -> NB
    {
      uint64_t acc[2][CC];
      tiny_zero(acc);
      tiny_mm32<1, CC>(nb0, nb1, sm + C::W_O, 32, u, 0, acc);
      float o[CC];
      tiny_out<CC>(acc, 0, 0, vec + C::V_BO + CC * u, o);
#pragma unroll
      for (int i = 0; i < CC; ++i) x0[i] += o[i];
      tiny_out<CC>(acc, 1, 0, vec + C::V_BO + CC * u, o);
#pragma unroll
      for (int i = 0; i < CC; ++i) x1[i] += o[i];
      float t0[CC], t1[CC];
#pragma unroll
      for (int i = 0; i < CC; ++i) t0[i] = x0[i], t1[i] = x1[i];
      tiny_layer_norm<G, CC>(t0, vec + C::V_LN2W + CC * u, vec + C::V_LN2B + CC * u, p.eps);
      tiny_layer_norm<G, CC>(t1, vec + C::V_LN2W + CC * u, vec + C::V_LN2B + CC * u, p.eps);
      __syncwarp();  // the group has read the context
      stc<CC>(nb0 + CC * u, t0);
      stc<CC>(nb1 + CC * u, t1);
    }
    __syncwarp();
    // ---- FFN in: hidden units 32m + CC*u .. of both rows, GELU -> HB
#pragma unroll 1
    for (int m = 0; m < F / 32; ++m) {
      uint64_t acc[2][CC];
      tiny_zero(acc);
      tiny_mm32<1, CC>(nb0, nb1, sm + C::W_IN + tiny_row<CC>(32 * m, 32), 32, u, 0, acc);
      float o[CC];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        tiny_out<CC>(acc, r, 0, vec + C::V_BIN + 32 * m + CC * u, o);
#pragma unroll
        for (int i = 0; i < CC; i += 2) gelu_as2(o[i], o[i + 1]);
        stc<CC>((r ? hb1 : hb0) + 32 * m + CC * u, o);
      }
    }
    __syncwarp();
    // ---- FFN out + residual: columns CC*u.. over all hidden units
    {
      uint64_t acc[2][CC];
      tiny_zero(acc);
#pragma unroll 1
      for (int k0 = 0; k0 < F; k0 += 32) tiny_mm32<1, CC>(hb0 + k0, hb1 + k0, sm + C::W_OUT, F, u, k0, acc);
      float o[CC];
      tiny_out<CC>(acc, 0, 0, vec + C::V_BOUT + CC * u, o);
#pragma unroll
      for (int i = 0; i < CC; ++i) x0[i] += o[i];
      tiny_out<CC>(acc, 1, 0, vec + C::V_BOUT + CC * u, o);
#pragma unroll
      for (int i = 0; i < CC; ++i) x1[i] += o[i];
    }
  }

  if (aborted) {
    // shared memory is released at exit: let the weight copy still in flight land first
    // (bounded; a copy that never lands records DERR_WAIT_DRAIN)
    if (threadIdx.x == 0 && pending >= 0) mbar_wait_drain(wbar, static_cast<uint32_t>(pending & 1));
  } else {
    // final LayerNorm -> y (padded rows are zero)
    tiny_layer_norm<G, CC>(x0, p.lnf_w + CC * u, p.lnf_b + CC * u, p.eps);
    tiny_layer_norm<G, CC>(x1, p.lnf_w + CC * u, p.lnf_b + CC * u, p.eps);
    if (ok0) {
      if (p.row_valid != nullptr && p.row_valid[g0] == 0) {
#pragma unroll
        for (int i = 0; i < CC; ++i) x0[i] = 0.f;
      }
      stc<CC>(p.y + g0 * 32 + CC * u, x0);
    }
    if (ok1) {
      if (p.row_valid != nullptr && p.row_valid[g0 + 1] == 0) {
#pragma unroll
        for (int i = 0; i < CC; ++i) x1[i] = 0.f;
      }
      stc<CC>(p.y + (g0 + 1) * 32 + CC * u, x1);
    }
  }
  if constexpr (SPLIT) {
    // Neither half exits while the other may still store K / V rows or arrive on a
    // barrier in its shared memory.  Every wait above is bounded and no path returns
    // early, so both halves reach this cluster barrier: a half that gave up waits here
    // while the other runs into its own (bounded) exchange wait, gives up too and joins.
    __syncwarp();
    cluster_sync_all();
  }
}

}  // namespace b200
