// Causal / prefix-causal / non-causal attention for head_dim 8 and 16.
//
// At these head dims a score costs 2*HD multiply-adds against one
// exponential, so the work is bound by the exponential and the FMA pipe, not
// by the tensor cores (a tcgen05 MMA needs K >= 16 and would compute mostly
// padding).  The reference's official matrix has two such shapes
// (d=32 H=4 and d=128 H=16, head_dim 8; run_eval.sh:44-58).
//
// One CTA per (128-row query tile, head, sequence), one thread per query row:
// K and V of the tile's visible keys are staged in shared memory 128 keys at
// a time (every thread reads the same key: broadcast), scores go through an
// online softmax in the log2 domain, 32 keys per max update, with fp32
// accumulation; the context row is written as fp16.  Same arguments and
// semantics as k_flash_causal (AttnParams: prefix chunks via q_offset,
// per-sequence key lengths, non-causal).
#pragma once

#include "attn.cuh"

namespace b200 {

constexpr int ATTN_SMALL_ROWS = 128;   // query rows (threads) per CTA
constexpr int ATTN_SMALL_KEYS = 128;   // keys staged per block

template <int HD>
__global__ void __launch_bounds__(ATTN_SMALL_ROWS)
    k_attn_small(const __half* __restrict__ q, int64_t ld_q, const __half* __restrict__ k, int64_t ld_k,
                 const __half* __restrict__ v, int64_t ld_v, const AttnParams p) {
  static_assert(HD == 8 || HD == 16, "head_dim 8 or 16");
  constexpr int CH = HD / 8;  // 16-byte chunks per head row
  __shared__ uint4 ks[ATTN_SMALL_KEYS][CH];
  __shared__ uint4 vs[ATTN_SMALL_KEYS][CH];

  griddep_sync();
  const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int i = tile * ATTN_SMALL_ROWS + threadIdx.x;  // query row within this call
  const bool active = i < p.q_len;
  const int kv_eff = attn_kv_eff(p, b);
  const int qpos = p.q_offset + i;
  const int klim = p.non_causal ? kv_eff - 1 : min(qpos, kv_eff - 1);  // last visible key of this row
  // keys any row of the tile sees
  const int last_row = min(p.q_len, (tile + 1) * ATTN_SMALL_ROWS) - 1;
  const int kend = p.non_causal ? kv_eff : min(p.q_offset + last_row, kv_eff - 1) + 1;

  float qf[HD];
  if (active) {
    const uint4* qr = reinterpret_cast<const uint4*>(
        q + (static_cast<int64_t>(p.q_row0) + static_cast<int64_t>(b) * p.q_seq_rows + i) * ld_q + p.q_col0 + h * HD);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const uint4 t = qr[c];
      const __half2* hp = reinterpret_cast<const __half2*>(&t);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(hp[e]);
        qf[8 * c + 2 * e] = f.x * p.scale_log2;  // scores come out in log2 units
        qf[8 * c + 2 * e + 1] = f.y * p.scale_log2;
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < HD; ++e) qf[e] = 0.f;
  }
  float o[HD];
#pragma unroll
  for (int e = 0; e < HD; ++e) o[e] = 0.f;
  float m = -INFINITY, l = 0.f;

  const int64_t kv_base = static_cast<int64_t>(p.kv_row0) + static_cast<int64_t>(b) * p.kv_seq_rows;
  for (int k0 = 0; k0 < kend; k0 += ATTN_SMALL_KEYS) {
    const int nk = min(ATTN_SMALL_KEYS, kend - k0);
    __syncthreads();  // the previous block's keys are no longer read
    if (static_cast<int>(threadIdx.x) < nk) {
      const int64_t row = kv_base + k0 + threadIdx.x;
      const uint4* kr = reinterpret_cast<const uint4*>(k + row * ld_k + p.k_col0 + h * HD);
      const uint4* vr = reinterpret_cast<const uint4*>(v + row * ld_v + p.v_col0 + h * HD);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        ks[threadIdx.x][c] = kr[c];
        vs[threadIdx.x][c] = vr[c];
      }
    }
    __syncthreads();
    if (!active) continue;
    const int jmax = min(nk, klim - k0 + 1);  // keys of this block this row sees
    for (int j0 = 0; j0 < jmax; j0 += 32) {
      const int jn = min(32, jmax - j0);
      float s[32];
      float mb = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        float acc = -INFINITY;
        if (jj < jn) {
          acc = 0.f;
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const uint4 t = ks[j0 + jj][c];
            const __half2* hp = reinterpret_cast<const __half2*>(&t);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(hp[e]);
              acc = fmaf(qf[8 * c + 2 * e], f.x, acc);
              acc = fmaf(qf[8 * c + 2 * e + 1], f.y, acc);
            }
          }
        }
        s[jj] = acc;
        mb = fmaxf(mb, acc);
      }
      const float mn = fmaxf(m, mb);
      const float corr = fast_exp2(m - mn);  // 0 on the first block (m = -inf)
      l *= corr;
#pragma unroll
      for (int e = 0; e < HD; ++e) o[e] *= corr;
      m = mn;
#pragma unroll
      for (int jj = 0; jj < 32; ++jj) {
        if (jj < jn) {
          const float pj = fast_exp2(s[jj] - m);
          l += pj;
#pragma unroll
          for (int c = 0; c < CH; ++c) {
            const uint4 t = vs[j0 + jj][c];
            const __half2* hp = reinterpret_cast<const __half2*>(&t);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(hp[e]);
              o[8 * c + 2 * e] = fmaf(pj, f.x, o[8 * c + 2 * e]);
              o[8 * c + 2 * e + 1] = fmaf(pj, f.y, o[8 * c + 2 * e + 1]);
            }
          }
        }
      }
    }
  }
  if (!active) return;
  const float inv_l = 1.f / l;  // every row sees key 0, so l >= 1
  uint4* orow = reinterpret_cast<uint4*>(p.out + (static_cast<int64_t>(b) * p.out_seq_rows + i) * p.ld_out + h * HD);
#pragma unroll
  for (int c = 0; c < CH; ++c)
    orow[c] = make_uint4(pack_half2(o[8 * c] * inv_l, o[8 * c + 1] * inv_l), pack_half2(o[8 * c + 2] * inv_l, o[8 * c + 3] * inv_l),
                         pack_half2(o[8 * c + 4] * inv_l, o[8 * c + 5] * inv_l), pack_half2(o[8 * c + 6] * inv_l, o[8 * c + 7] * inv_l));
}

}  // namespace b200
