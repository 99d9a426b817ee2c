// Fused block for tiny models: d_model = 32 (head_dim 8, 16 or 32), ffn_dim a
// multiple of 32 up to 128, seq_len <= 128, any number of layers.
//
// The reference's official matrix has such a shape (d=32 H=4 ffn=32, 4
// layers; run_eval.sh:44-58).  At d = 32 a 128-row tcgen05 tile would be
// mostly padding and every stage of the per-layer kernel chain is a few
// microseconds of launch and prologue around almost no arithmetic, so the
// whole model runs in one kernel on the CUDA cores:
//
//   one CTA per sequence, four threads per row (512 threads): thread (r, c)
//   owns columns 8c..8c+7 of row r (x, the LN outputs, the context); the
//   LayerNorm statistics combine over the quad with two shuffles; a product
//   that needs a whole row (the projections, the FFN hidden units) reads it
//   from a per-row shared-memory buffer the quad fills (the quad is one
//   warp's lanes, so __syncwarp orders it); each thread computes 8 of the
//   outputs.  The layer's weights are staged in shared memory as fp32 (read
//   at one address by many lanes: broadcasts); K and V of every row go to
//   shared memory.  Attention runs per (row, head): with 4 heads one thread
//   per head walks the visible keys with an online softmax (log2 domain);
//   with fewer heads the threads of a head take alternate keys and merge
//   their (max, sum, context) with shuffles.
//
// Matrix products accumulate in fp32 from the fp16 weight copies the other
// paths use, in chains of 4 independent outputs so the FMA latency overlaps.
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

// floats of a [rows][ld] weight staged with 4 floats of padding after every 8 rows
constexpr int tiny_padded(int rows, int ld) { return rows * ld + (rows / 8) * 4; }

struct TinyCfg {
  static constexpr int D = 32;
  static constexpr int S = 128;          // rows per CTA
  static constexpr int THREADS = 4 * S;  // a quad per row
  static constexpr int FMAX = 128;
  static constexpr int LD = D + 4;       // padded row stride (floats) of the K / V rows
  static constexpr int RL = FMAX + 4;    // row stride of the exchange buffer
  // Weights are row-major with 4 floats of padding after every 8 rows
  // (tiny_row): the quad's threads read rows 8 apart in the same instruction,
  // which without the padding would fall on the same banks.
  // shared memory (floats)
  static constexpr int W_QKV = 0;                                   // [96][32]
  static constexpr int W_O = W_QKV + tiny_padded(3 * D, D);              // [32][32]
  static constexpr int W_IN = W_O + tiny_padded(D, D);                   // [FMAX][32]
  static constexpr int W_OUT = W_IN + tiny_padded(FMAX, D);              // [32][ffn]
  static constexpr int VEC = W_OUT + tiny_padded(D, FMAX);               // ln1 w,b | b_qkv | b_o | ln2 w,b | b_in | b_out
  static constexpr int V_LN1W = 0, V_LN1B = 32, V_BQKV = 64, V_BO = 160, V_LN2W = 192, V_LN2B = 224, V_BIN = 256,
                       V_BOUT = 256 + FMAX, V_TOTAL = 288 + FMAX;
  static constexpr int KS = VEC + V_TOTAL;              // [S][LD]
  static constexpr int VS = KS + S * LD;                // [S][LD]
  static constexpr int ROWS = VS + S * LD;              // [S][RL] exchange buffer (a row's n, context or hidden units)
  static constexpr int KOK = ROWS + S * RL;             // [S] 1: key exists and is not padding
  // the next layer's fp16 weights and fp32 vectors as they arrive by bulk copy
  // (row-major, unpadded; the vectors in the VEC layout), converted into the
  // regions above at the layer boundary
  static constexpr int STG_QKV = KOK + S;               // [96][32] fp16
  static constexpr int STG_O = STG_QKV + 3 * D * D / 2; // [32][32] fp16
  static constexpr int STG_IN = STG_O + D * D / 2;      // [ffn][32] fp16
  static constexpr int STG_OUT = STG_IN + FMAX * D / 2; // [32][ffn] fp16
  static constexpr int STG_VEC = STG_OUT + D * FMAX / 2;
  static constexpr int BAR = STG_VEC + V_TOTAL;         // mbarrier (8 bytes) + abort flag
  static constexpr int TOTAL_FLOATS = BAR + 4;
  static constexpr int TOTAL = TOTAL_FLOATS * 4;
};

// sum over the quad (the 4 threads of a row: adjacent lanes)
__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

// LayerNorm of a 32-wide row held as 8 columns per quad thread (two-pass statistics)
__device__ __forceinline__ void tiny_layer_norm8(float (&v)[8], const float* gamma8, const float* beta8, float eps) {
  const float mean = quad_sum(((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]))) * (1.f / 32.f);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] -= mean;
    sq = fmaf(v[i], v[i], sq);
  }
  const float rstd = rsqrtf(quad_sum(sq) * (1.f / 32.f) + eps);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = fmaf(v[i] * rstd, gamma8[i], beta8[i]);
}

// offset (floats) of row `row` of a weight staged with row stride ld (TinyCfg::padded layout)
__device__ __forceinline__ int tiny_row(int row, int ld) { return row * ld + (row >> 3) * 4; }

// out[c] = bias[c] + a . W[row0 + c] for c in [0, N): W row-major [.][32] fp32 in shared
// memory (padded layout), a as 16 packed pairs.  Four outputs at a time, each
// accumulating its even and odd products as one f32x2 pair (independent chains).
template <int N>
__device__ __forceinline__ void tiny_matvec32(const uint64_t (&a)[16], const float* W, int row0, const float* bias,
                                              float (&out)[N]) {
#pragma unroll
  for (int c = 0; c < N; c += 4) {
    uint64_t acc0 = 0, acc1 = 0, acc2 = 0, acc3 = 0;  // (0.f, 0.f)
    const float* W0 = W + tiny_row(row0 + c, 32);
    const float* W1 = W + tiny_row(row0 + c + 1, 32);
    const float* W2 = W + tiny_row(row0 + c + 2, 32);
    const float* W3 = W + tiny_row(row0 + c + 3, 32);
#pragma unroll
    for (int k = 0; k < 32; k += 4) {
      const float4 w0 = *reinterpret_cast<const float4*>(W0 + k);
      const float4 w1 = *reinterpret_cast<const float4*>(W1 + k);
      const float4 w2 = *reinterpret_cast<const float4*>(W2 + k);
      const float4 w3 = *reinterpret_cast<const float4*>(W3 + k);
      acc0 = f2fma(a[k / 2 + 1], f2pk(w0.z, w0.w), f2fma(a[k / 2], f2pk(w0.x, w0.y), acc0));
      acc1 = f2fma(a[k / 2 + 1], f2pk(w1.z, w1.w), f2fma(a[k / 2], f2pk(w1.x, w1.y), acc1));
      acc2 = f2fma(a[k / 2 + 1], f2pk(w2.z, w2.w), f2fma(a[k / 2], f2pk(w2.x, w2.y), acc2));
      acc3 = f2fma(a[k / 2 + 1], f2pk(w3.z, w3.w), f2fma(a[k / 2], f2pk(w3.x, w3.y), acc3));
    }
    float e, o;
    f2upk(acc0, e, o);
    out[c] = bias[c] + (e + o);
    f2upk(acc1, e, o);
    out[c + 1] = bias[c + 1] + (e + o);
    f2upk(acc2, e, o);
    out[c + 2] = bias[c + 2] + (e + o);
    f2upk(acc3, e, o);
    out[c + 3] = bias[c + 3] + (e + o);
  }
}

// acc[o] += sum_k h[k] * W[row0 + o][col0 + k] for o in [0, N): a 32-column slice of a
// row-major weight with row stride ld (padded layout), h as 16 packed pairs
template <int N>
__device__ __forceinline__ void tiny_matvec32_acc(const uint64_t (&h)[16], const float* W, int row0, int ld, int col0,
                                                  float (&acc)[N]) {
#pragma unroll
  for (int o = 0; o < N; o += 4) {
    uint64_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    const float* W0 = W + tiny_row(row0 + o, ld) + col0;
    const float* W1 = W + tiny_row(row0 + o + 1, ld) + col0;
    const float* W2 = W + tiny_row(row0 + o + 2, ld) + col0;
    const float* W3 = W + tiny_row(row0 + o + 3, ld) + col0;
#pragma unroll
    for (int k = 0; k < 32; k += 4) {
      const float4 w0 = *reinterpret_cast<const float4*>(W0 + k);
      const float4 w1 = *reinterpret_cast<const float4*>(W1 + k);
      const float4 w2 = *reinterpret_cast<const float4*>(W2 + k);
      const float4 w3 = *reinterpret_cast<const float4*>(W3 + k);
      a0 = f2fma(h[k / 2 + 1], f2pk(w0.z, w0.w), f2fma(h[k / 2], f2pk(w0.x, w0.y), a0));
      a1 = f2fma(h[k / 2 + 1], f2pk(w1.z, w1.w), f2fma(h[k / 2], f2pk(w1.x, w1.y), a1));
      a2 = f2fma(h[k / 2 + 1], f2pk(w2.z, w2.w), f2fma(h[k / 2], f2pk(w2.x, w2.y), a2));
      a3 = f2fma(h[k / 2 + 1], f2pk(w3.z, w3.w), f2fma(h[k / 2], f2pk(w3.x, w3.y), a3));
    }
    float e, od;
    f2upk(a0, e, od);
    acc[o] += e + od;
    f2upk(a1, e, od);
    acc[o + 1] += e + od;
    f2upk(a2, e, od);
    acc[o + 2] += e + od;
    f2upk(a3, e, od);
    acc[o + 3] += e + od;
  }
}

// fp16 weight [rows][ld] (shared memory, as staged) -> fp32 shared memory in the
// padded layout (ld a multiple of 8), all threads of the CTA
__device__ __forceinline__ void tiny_stage_f16(float* dst, const __half* src, int rows, int ld) {
  for (int i = static_cast<int>(threadIdx.x) * 8; i < rows * ld; i += TinyCfg::THREADS * 8) {
    const uint4 t = *reinterpret_cast<const uint4*>(src + i);
    const __half2* h2 = reinterpret_cast<const __half2*>(&t);
    const float2 f0 = __half22float2(h2[0]), f1 = __half22float2(h2[1]), f2 = __half22float2(h2[2]),
                 f3 = __half22float2(h2[3]);
    float* d = dst + tiny_row(i / ld, ld) + i % ld;
    *reinterpret_cast<float4*>(d) = make_float4(f0.x, f0.y, f1.x, f1.y);
    *reinterpret_cast<float4*>(d + 4) = make_float4(f2.x, f2.y, f3.x, f3.y);
  }
}

// 8 consecutive floats at p (16-byte aligned) -> v / v -> p
__device__ __forceinline__ void ld8(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void st8(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
// 32 consecutive floats at p (16-byte aligned) as 16 packed pairs
__device__ __forceinline__ void ld32x2(const float* p, uint64_t (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 a = *reinterpret_cast<const float4*>(p + 4 * j);
    v[2 * j] = f2pk(a.x, a.y);
    v[2 * j + 1] = f2pk(a.z, a.w);
  }
}

template <int HD>
__global__ void __launch_bounds__(TinyCfg::THREADS, 1) k_block_tiny(const TinyParams p) {
  using C = TinyCfg;
  static_assert(HD == 8 || HD == 16 || HD == 32, "head_dim 8, 16 or 32");
  constexpr int H = C::D / HD;  // heads
  constexpr int T = 4 / H;      // threads of a quad per head; they take alternate keys
  constexpr int KB = HD == 32 ? 16 : 32;  // keys per softmax block (fewer live scores at head_dim 32)
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);

  griddep_sync();
  const int r = threadIdx.x >> 2;  // row
  const int c = threadIdx.x & 3;   // column quarter: columns 8c..8c+7
  const int head = c / T, sub = c % T;
  const int seq = blockIdx.x;
  const int F = p.ffn;
  const bool row_ok = r < p.seq_len;
  const int64_t grow = static_cast<int64_t>(seq) * p.seq_len + r;
  float* vec = sm + C::VEC;
  float* rowbuf = sm + C::ROWS + r * C::RL;
  const float* key_ok = sm + C::KOK;
  uint64_t* wbar = reinterpret_cast<uint64_t*>(sm + C::BAR);  // a layer's staged weights and vectors
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + C::BAR + 2);
  // one thread copies layer l's weights and vectors into the staging area (ten bulk
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
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) fetch(0);
  if (c == 0) sm[C::KOK + r] = (row_ok && (p.row_valid == nullptr || p.row_valid[grow] != 0)) ? 1.f : 0.f;
  const int kend = p.non_causal ? p.seq_len : min(r + 1, p.seq_len);  // keys 0..kend-1 may be visible
  // key validity as four 32-bit words in registers (lane i tests key 32w + i)
  uint32_t kw[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int j = 32 * w + (threadIdx.x & 31);
    kw[w] = __ballot_sync(0xffffffffu, j < p.seq_len && (p.row_valid == nullptr ||
                                                          p.row_valid[static_cast<int64_t>(seq) * p.seq_len + j] != 0));
  }

  float x[8];
  if (row_ok) {
    ld8(p.x + grow * 32 + 8 * c, x);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = 0.f;
  }

  for (int l = 0; l < p.layers; ++l) {
    __syncthreads();  // the previous layer's weights and K / V are no longer read
    // layer l's staged copies -> fp32 weights (padded layout) and vectors
    const bool got = mbar_wait(wbar, static_cast<uint32_t>(l & 1), abort_flag, DERR_WAIT_TMA);
    if (got) {
      tiny_stage_f16(sm + C::W_QKV, reinterpret_cast<const __half*>(sm + C::STG_QKV), 96, 32);
      tiny_stage_f16(sm + C::W_O, reinterpret_cast<const __half*>(sm + C::STG_O), 32, 32);
      tiny_stage_f16(sm + C::W_IN, reinterpret_cast<const __half*>(sm + C::STG_IN), F, 32);
      tiny_stage_f16(sm + C::W_OUT, reinterpret_cast<const __half*>(sm + C::STG_OUT), 32, F);
      if (threadIdx.x < C::V_TOTAL / 4)
        reinterpret_cast<float4*>(vec)[threadIdx.x] = reinterpret_cast<const float4*>(sm + C::STG_VEC)[threadIdx.x];
    }
    // a copy that never landed (bounded wait, error recorded) ends the whole CTA here
    if (__syncthreads_or(!got)) return;
    if (threadIdx.x == 0 && l + 1 < p.layers) fetch(l + 1);

    // LN1 -> the row buffer -> the whole row n; this quarter's K and V columns -> shared memory
    uint64_t n[16];  // the row's LN output as packed pairs
    {
      float t8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) t8[i] = x[i];
      tiny_layer_norm8(t8, vec + C::V_LN1W + 8 * c, vec + C::V_LN1B + 8 * c, p.eps);
      st8(rowbuf + 8 * c, t8);
      __syncwarp();
      ld32x2(rowbuf, n);
      float kv[8];
      tiny_matvec32<8>(n, sm + C::W_QKV, 32 + 8 * c, vec + C::V_BQKV + 32 + 8 * c, kv);
      st8(sm + C::KS + r * C::LD + 8 * c, kv);
      tiny_matvec32<8>(n, sm + C::W_QKV, 64 + 8 * c, vec + C::V_BQKV + 64 + 8 * c, kv);
      st8(sm + C::VS + r * C::LD + 8 * c, kv);
    }
    __syncthreads();  // every row's K and V are in place

    // attention for (row r, head): this thread's keys are sub, sub + T, ...
    // (query and context accumulator as packed pairs: dot products and the P.V update
    // run as f32x2 FMAs)
    uint64_t o[HD / 2];
    float m = -INFINITY, lsum = 0.f;
    {
      uint64_t q2[HD / 2];
      {
        float q[HD];
        tiny_matvec32<HD>(n, sm + C::W_QKV, head * HD, vec + C::V_BQKV + head * HD, q);
#pragma unroll
        for (int e = 0; e < HD; e += 2) {
          q2[e / 2] = f2pk(q[e] * p.scale_log2, q[e + 1] * p.scale_log2);  // scores in log2 units
          o[e / 2] = 0;
        }
      }
      for (int j0 = sub; j0 < kend; j0 += KB * T) {
        float s[KB];
        float mb = -INFINITY;
        // one head per thread (T == 1): the block's keys j0.. share one validity word
        const uint32_t kv_word = T == 1 ? (j0 < 32 ? kw[0] : j0 < 64 ? kw[1] : j0 < 96 ? kw[2] : kw[3]) >> (j0 & 31)
                                        : 0u;
#pragma unroll
        for (int jj = 0; jj < KB; ++jj) {
          const int j = j0 + jj * T;
          float acc = -INFINITY;
          const bool valid = T == 1 ? ((kv_word >> jj) & 1u) != 0u : key_ok[j] != 0.f;
          if (j < kend && valid) {
            const float* kr = sm + C::KS + j * C::LD + head * HD;
            uint64_t a2 = 0;
#pragma unroll
            for (int e = 0; e < HD; e += 4) {
              const float4 kk = *reinterpret_cast<const float4*>(kr + e);
              a2 = f2fma(q2[e / 2 + 1], f2pk(kk.z, kk.w), f2fma(q2[e / 2], f2pk(kk.x, kk.y), a2));
            }
            float lo, hi;
            f2upk(a2, lo, hi);
            acc = lo + hi;
          }
          s[jj] = acc;
          mb = fmaxf(mb, acc);
        }
        if (mb == -INFINITY) continue;  // no visible key in this block
        const float mn = fmaxf(m, mb);
        const float corr = fast_exp2(m - mn);  // 0 on the first visible block
        lsum *= corr;
        const uint64_t corr2 = f2pk(corr, corr);
#pragma unroll
        for (int e = 0; e < HD / 2; ++e) o[e] = f2mul(o[e], corr2);
        m = mn;
#pragma unroll
        for (int jj = 0; jj < KB; ++jj) {
          if (s[jj] != -INFINITY) {  // masked keys are skipped, never weighted by zero
            const float pj = fast_exp2(s[jj] - m);
            lsum += pj;
            const uint64_t p2 = f2pk(pj, pj);
            const float* vr = sm + C::VS + (j0 + jj * T) * C::LD + head * HD;
#pragma unroll
            for (int e = 0; e < HD; e += 4) {
              const float4 vv = *reinterpret_cast<const float4*>(vr + e);
              o[e / 2] = f2fma(p2, f2pk(vv.x, vv.y), o[e / 2]);
              o[e / 2 + 1] = f2fma(p2, f2pk(vv.z, vv.w), o[e / 2 + 1]);
            }
          }
        }
      }
    }
    // merge the partial softmaxes of a head's T threads (alternate keys)
#pragma unroll
    for (int off = 1; off < T; off <<= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, off), l2 = __shfl_xor_sync(0xffffffffu, lsum, off);
      const float mm = fmaxf(m, m2);
      const float a = (m == -INFINITY) ? 0.f : fast_exp2(m - mm);
      const float b2 = (m2 == -INFINITY) ? 0.f : fast_exp2(m2 - mm);
      lsum = lsum * a + l2 * b2;
      const uint64_t a_2 = f2pk(a, a), b_2 = f2pk(b2, b2);
#pragma unroll
      for (int e = 0; e < HD / 2; ++e) {
        const uint64_t other = __shfl_xor_sync(0xffffffffu, o[e], off);
        o[e] = f2fma(o[e], a_2, f2mul(other, b_2));
      }
      m = mm;
    }
    {
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;  // a row with no visible key (padding) gets 0
      __syncwarp();  // the quad has read n from the row buffer
      if (sub == 0) {
        const uint64_t inv2 = f2pk(inv, inv);
#pragma unroll
        for (int e = 0; e < HD; e += 2) {
          float lo, hi;
          f2upk(f2mul(o[e / 2], inv2), lo, hi);
          *reinterpret_cast<float2*>(rowbuf + head * HD + e) = make_float2(lo, hi);
        }
      }
      __syncwarp();
    }
    // out_proj + residual (this quarter's 8 columns); LN2 -> the row buffer -> n
    {
      uint64_t cx[16];
      ld32x2(rowbuf, cx);
      float t8[8];
      tiny_matvec32<8>(cx, sm + C::W_O, 8 * c, vec + C::V_BO + 8 * c, t8);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        x[i] += t8[i];
        t8[i] = x[i];
      }
      tiny_layer_norm8(t8, vec + C::V_LN2W + 8 * c, vec + C::V_LN2B + 8 * c, p.eps);
      __syncwarp();  // the quad has read the context
      st8(rowbuf + 8 * c, t8);
      __syncwarp();
      ld32x2(rowbuf, n);
    }
    // FFN: this quarter's hidden units -> the row buffer; then its 8 output columns over all units
    __syncwarp();  // the quad has read n
    for (int u0 = c * (F / 4); u0 < (c + 1) * (F / 4); u0 += 8) {
      float h8[8];
      tiny_matvec32<8>(n, sm + C::W_IN, u0, vec + C::V_BIN + u0, h8);
#pragma unroll
      for (int i = 0; i < 8; ++i) h8[i] = gelu_as(h8[i]);
      st8(rowbuf + u0, h8);
    }
    __syncwarp();
    {
      float acc[8];
      ld8(vec + C::V_BOUT + 8 * c, acc);
#pragma unroll 1
      for (int k0 = 0; k0 < F; k0 += 32) {
        uint64_t h32[16];
        ld32x2(rowbuf + k0, h32);
        tiny_matvec32_acc<8>(h32, sm + C::W_OUT, 8 * c, F, k0, acc);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] += acc[i];
    }
    __syncwarp();  // the row buffer is free for the next layer
  }

  // final LayerNorm -> y (padded rows are zero)
  tiny_layer_norm8(x, p.lnf_w + 8 * c, p.lnf_b + 8 * c, p.eps);
  if (!row_ok) return;
  if (p.row_valid != nullptr && p.row_valid[grow] == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = 0.f;
  }
  st8(p.y + grow * 32 + 8 * c, x);
}

}  // namespace b200
