// Causal / prefix-causal / non-causal attention for head_dim 8 and 16.
//
// At these head dims a score costs 2*HD multiply-adds against one
// exponential, so the work is bound by the exponential, the FMA pipe and the
// shared-memory loads, not by the tensor cores (a tcgen05 MMA needs K >= 16
// and would compute mostly padding).  The reference's official matrix has two
// such shapes (d=32 H=4 and d=128 H=16, head_dim 8; run_eval.sh:44-58).
//
// One CTA per (128-row query tile, head, sequence), 128 threads: the two
// threads of a pair take the query rows 2i and 2i+1 together and split the keys
// by parity, so every K / V row loaded from shared memory serves two query rows.
// K and V of the tile's visible keys are staged in shared memory as fp32, 128
// keys at a time (converted once, not per query row); scores go through an
// online softmax in the log2 domain, 16 keys per max update, with f32x2
// multiply-adds and fp32 accumulation; the pair merges its two partial
// softmaxes with shuffles and each thread writes one row's context as fp16.
// Same arguments and semantics as k_flash_causal (AttnParams: prefix chunks via
// q_offset, per-sequence key lengths, non-causal).
#pragma once

#include "attn.cuh"

namespace b200 {

constexpr int ATTN_SMALL_ROWS = 128;   // query rows per CTA (and threads)
constexpr int ATTN_SMALL_KEYS = 128;   // keys staged per block

template <int HD>
__global__ void __launch_bounds__(ATTN_SMALL_ROWS)
    k_attn_small(const __half* __restrict__ q, int64_t ld_q, const __half* __restrict__ k, int64_t ld_k,
                 const __half* __restrict__ v, int64_t ld_v, const AttnParams p) {
  static_assert(HD == 8 || HD == 16, "head_dim 8 or 16");
  constexpr int CH = HD / 8;  // 16-byte fp16 chunks per head row
  constexpr int KB = 16;      // keys per thread between max updates
  __shared__ float4 ks[ATTN_SMALL_KEYS][HD / 4];
  __shared__ float4 vs[ATTN_SMALL_KEYS][HD / 4];

  griddep_sync();
  const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int par = threadIdx.x & 1;                                          // key parity of this thread
  const int i0 = tile * ATTN_SMALL_ROWS + 2 * static_cast<int>(threadIdx.x >> 1);  // rows i0, i0 + 1
  const int kv_eff = attn_kv_eff(p, b);
  const bool holes = attn_has_holes(p, b);
  const uint32_t* kbits = holes ? p.key_bits + static_cast<int64_t>(b) * p.key_words : nullptr;
  int klim[2];  // last visible key of each row (-1: row not in this call)
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int i = i0 + rr;
    klim[rr] = i < p.q_len ? (p.non_causal ? kv_eff - 1 : min(p.q_offset + i, kv_eff - 1)) : -1;
  }
  // keys any row of the tile sees
  const int last_row = min(p.q_len, (tile + 1) * ATTN_SMALL_ROWS) - 1;
  const int kend = p.non_causal ? kv_eff : min(p.q_offset + last_row, kv_eff - 1) + 1;

  uint64_t q2[2][HD / 2], o[2][HD / 2];
  float m[2], l[2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    if (klim[rr] >= 0) {
      const uint4* qr = reinterpret_cast<const uint4*>(
          q + (static_cast<int64_t>(p.q_row0) + static_cast<int64_t>(b) * p.q_seq_rows + i0 + rr) * ld_q + p.q_col0 +
          h * HD);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const uint4 t = qr[c];
        const __half2* hp = reinterpret_cast<const __half2*>(&t);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(hp[e]);
          q2[rr][4 * c + e] = f2pk(f.x * p.scale_log2, f.y * p.scale_log2);  // scores come out in log2 units
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < HD / 2; ++e) q2[rr][e] = 0ull;
    }
#pragma unroll
    for (int e = 0; e < HD / 2; ++e) o[rr][e] = 0ull;
    m[rr] = -INFINITY;
    l[rr] = 0.f;
  }
  const int jlast = max(klim[0], klim[1]);  // the later row sees the most keys

  const int64_t kv_base = static_cast<int64_t>(p.kv_row0) + static_cast<int64_t>(b) * p.kv_seq_rows;
  for (int k0 = 0; k0 < kend; k0 += ATTN_SMALL_KEYS) {
    const int nk = min(ATTN_SMALL_KEYS, kend - k0);
    __syncthreads();  // the previous block's keys are no longer read
    if (static_cast<int>(threadIdx.x) < nk) {  // key k0 + t, fp16 -> fp32
      const int64_t row = kv_base + k0 + threadIdx.x;
      const uint4* kr = reinterpret_cast<const uint4*>(k + row * ld_k + p.k_col0 + h * HD);
      const uint4* vr = reinterpret_cast<const uint4*>(v + row * ld_v + p.v_col0 + h * HD);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        const uint4 kt = kr[c], vt = vr[c];
        const __half2* kh = reinterpret_cast<const __half2*>(&kt);
        const __half2* vh = reinterpret_cast<const __half2*>(&vt);
        const float2 k01 = __half22float2(kh[0]), k23 = __half22float2(kh[1]), k45 = __half22float2(kh[2]),
                     k67 = __half22float2(kh[3]);
        const float2 v01 = __half22float2(vh[0]), v23 = __half22float2(vh[1]), v45 = __half22float2(vh[2]),
                     v67 = __half22float2(vh[3]);
        ks[threadIdx.x][2 * c] = make_float4(k01.x, k01.y, k23.x, k23.y);
        ks[threadIdx.x][2 * c + 1] = make_float4(k45.x, k45.y, k67.x, k67.y);
        vs[threadIdx.x][2 * c] = make_float4(v01.x, v01.y, v23.x, v23.y);
        vs[threadIdx.x][2 * c + 1] = make_float4(v45.x, v45.y, v67.x, v67.y);
      }
    }
    __syncthreads();
    const int jmax = min(nk - 1, jlast - k0);  // last key of this block the pair sees
    for (int j0 = par; j0 <= jmax; j0 += 2 * KB) {
      float s[2][KB];
      float mb[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int jj = 0; jj < KB; ++jj) {
        const int j = j0 + 2 * jj;  // this thread's keys: one parity
        float a[2] = {-INFINITY, -INFINITY};
        if (j <= jmax) {
          uint64_t d2[2] = {0ull, 0ull};
#pragma unroll
          for (int e = 0; e < HD / 4; ++e) {
            const float4 kk = ks[j][e];
            const uint64_t ka = f2pk(kk.x, kk.y), kc = f2pk(kk.z, kk.w);
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) d2[rr] = f2fma(q2[rr][2 * e + 1], kc, f2fma(q2[rr][2 * e], ka, d2[rr]));
          }
          // a key the sequence's mask excludes scores -inf for both rows
          const bool kvalid = !holes || ((__ldg(kbits + ((k0 + j) >> 5)) >> ((k0 + j) & 31)) & 1u);
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            if (kvalid && k0 + j <= klim[rr]) {
              float lo, hi;
              f2upk(d2[rr], lo, hi);
              a[rr] = lo + hi;
            }
          }
        }
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          s[rr][jj] = a[rr];
          mb[rr] = fmaxf(mb[rr], a[rr]);
        }
      }
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        if (mb[rr] != -INFINITY) {
          const float mn = fmaxf(m[rr], mb[rr]);
          const float corr = fast_exp2(m[rr] - mn);  // 0 on the row's first visible block (m = -inf)
          l[rr] *= corr;
          const uint64_t c2 = f2pk(corr, corr);
#pragma unroll
          for (int e = 0; e < HD / 2; ++e) o[rr][e] = f2mul(o[rr][e], c2);
          m[rr] = mn;
        }
      }
#pragma unroll
      for (int jj = 0; jj < KB; ++jj) {
        const int j = j0 + 2 * jj;
        if (j <= jmax) {
          float pj[2];
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            pj[rr] = s[rr][jj] != -INFINITY ? fast_exp2(s[rr][jj] - m[rr]) : 0.f;  // a masked key adds nothing
            l[rr] += pj[rr];
          }
          const uint64_t p0 = f2pk(pj[0], pj[0]), p1 = f2pk(pj[1], pj[1]);
#pragma unroll
          for (int e = 0; e < HD / 4; ++e) {
            const float4 vv = vs[j][e];
            const uint64_t va = f2pk(vv.x, vv.y), vc = f2pk(vv.z, vv.w);
            o[0][2 * e] = f2fma(p0, va, o[0][2 * e]);
            o[0][2 * e + 1] = f2fma(p0, vc, o[0][2 * e + 1]);
            o[1][2 * e] = f2fma(p1, va, o[1][2 * e]);
            o[1][2 * e + 1] = f2fma(p1, vc, o[1][2 * e + 1]);
          }
        }
      }
    }
  }
  // merge the pair's two partial softmaxes (even / odd keys)
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m[rr], 1), l2 = __shfl_xor_sync(0xffffffffu, l[rr], 1);
    const float mm = fmaxf(m[rr], m2);
    const float a = (m[rr] == -INFINITY) ? 0.f : fast_exp2(m[rr] - mm);
    const float b2 = (m2 == -INFINITY) ? 0.f : fast_exp2(m2 - mm);
    l[rr] = l[rr] * a + l2 * b2;
    const uint64_t a_2 = f2pk(a, a), b_2 = f2pk(b2, b2);
#pragma unroll
    for (int e = 0; e < HD / 2; ++e) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, o[rr][e], 1);
      o[rr][e] = f2fma(o[rr][e], a_2, f2mul(other, b_2));
    }
  }
  // thread `par` of the pair writes row i0 + par
  const int i = i0 + par;
  if (i >= p.q_len) return;
  uint64_t w[HD / 2];
  float lw = l[0];
#pragma unroll
  for (int e = 0; e < HD / 2; ++e) w[e] = par ? o[1][e] : o[0][e];
  if (par) lw = l[1];
  const float inv_l = lw > 0.f ? 1.f / lw : 0.f;  // a row whose visible keys are all masked: context 0
  const uint64_t iv = f2pk(inv_l, inv_l);
  uint4* orow = reinterpret_cast<uint4*>(p.out + (static_cast<int64_t>(b) * p.out_seq_rows + i) * p.ld_out + h * HD);
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    float f[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) f2upk(f2mul(w[4 * c + e], iv), f[2 * e], f[2 * e + 1]);
    orow[c] = make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]), pack_half2(f[6], f[7]));
  }
}

}  // namespace b200
