// Causal flash attention on tcgen05: persistent CTAs, each walking a share of
// the (128-row query tile, head, sequence) work items.
//
// Semantics follow the reference module's attention (TTB:117-132 of
// torch_transformer_benchmark.py): scores = q.k^T * head_dim^-0.5, keys after
// the query masked, fp32 softmax, probs.v.  Query row i of this call sits at
// absolute position q_offset+i and sees keys 0..q_offset+i -- with q_offset=0
// that is the reference's triu(1) mask, with q_offset>0 it is the prefix-causal
// (bottom-right aligned) attention of the reference's chunked forward
// (TTB:1491-1500) over an incrementally filled K/V cache.
//
// Per CTA (192 threads):
//   warp 0     TMA producer: each item's 128-row Q tile (two buffers where they
//              fit), then its K_j/V_j tiles into a 2-deep ring (kv_full /
//              kv_empty mbarriers), running ahead into the next item;
//   warp 1     TMEM owner + MMA issuer: S_j = Q.K_j^T into TMEM columns
//              [0,BN); O += P_j.V_j into columns [BN, BN+HD) with V read
//              MN-major (head_dim contiguous) straight from the TMA tile.
//              The next S (of this item or of the next) is issued as soon as
//              the softmax has read S_j into registers (s_free), so it
//              overlaps the softmax of tile j;
//   warps 2-5  softmax: one query row per thread (TMEM lane = row), running
//              max / sum in the log2 domain, P_j (fp16) written to TMEM or to
//              shared memory in the 128B-swizzled K-major layout UMMA reads, O
//              rescaled in TMEM when the running max moves; final O/l -> fp16
//              context, then straight on to the next item's first S.
// Key tiles past the diagonal are never loaded (causal tile skipping); only
// tiles that straddle the diagonal apply the mask.
#pragma once

#include "ptx.cuh"

namespace b200 {

// ---- row softmax pieces shared by the attention kernels (one row per thread)

// this thread's TMEM row, N fp32 columns, one load instruction and one wait
template <int N>
__device__ __forceinline__ void tmem_ld_row(uint32_t taddr, float (&s)[N]) {
  if constexpr (N == 128) {
    tmem_ld128(taddr, s);
  } else {
    static_assert(N == 64, "rows of 64 or 128 columns");
    tmem_ld64(taddr, s);
  }
}
// max of N values: eight independent chains of three-input maxima (short
// dependency chains; two warps per SMSP cannot hide a 64-deep chain)
template <int N>
__device__ __forceinline__ float row_max(const float (&s)[N]) {
  static_assert(N % 16 == 0, "N multiple of 16");
  float m[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) m[k] = fmaxf(s[2 * k], s[2 * k + 1]);
#pragma unroll
  for (int c = 16; c < N; c += 16)
#pragma unroll
    for (int k = 0; k < 8; ++k) m[k] = fmax3(m[k], s[c + 2 * k], s[c + 2 * k + 1]);
  return fmaxf(fmax3(m[0], m[1], m[2]), fmaxf(fmax3(m[3], m[4], m[5]), fmaxf(m[6], m[7])));
}
// s[c] = 2^(s[c]*scale - m) in place; returns the sum (f32x2 pairs: the
// scale/subtract and the four running sums take half the issue slots).
// (Computing part of the exponentials with a polynomial on the FMA pipe was
// measured here and did not pay: these softmax loops are latency-bound, not
// bound by the SFU.)
template <int N>
__device__ __forceinline__ float row_exp2_sum(float (&s)[N], float scale, float m) {
  const uint64_t sc = f2pk(scale, scale), nm = f2pk(-m, -m);
  uint64_t acc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) acc[k] = f2pk(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < N; c += 2) {
    float a, b;
    f2upk(f2fma(f2pk(s[c], s[c + 1]), sc, nm), a, b);
    s[c] = fast_exp2(a);
    s[c + 1] = fast_exp2(b);
    acc[(c >> 1) & 3] = f2add(acc[(c >> 1) & 3], f2pk(s[c], s[c + 1]));
  }
  float t[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) f2upk(acc[k], t[2 * k], t[2 * k + 1]);
  return ((t[0] + t[1]) + (t[2] + t[3])) + ((t[4] + t[5]) + (t[6] + t[7]));
}

struct AttnParams {
  int H;
  int batch;             // sequences
  int q_len;             // query rows per sequence handled by this call
  int q_offset;          // absolute position of query row 0 inside its sequence
  int kv_len;            // keys available per sequence (>= q_offset + q_len)
  int q_seq_rows;        // rows between consecutive sequences in the Q tensor
  int kv_seq_rows;       // rows between consecutive sequences in the K/V tensors
  int q_row0, kv_row0;   // row of sequence 0 / position 0 in the Q and K/V tensors
  int q_col0, k_col0, v_col0;  // column of head 0 in the Q / K / V tensors
  __half* out;           // context [rows, ld_out]; head h at column h*HD
  int64_t ld_out;
  int out_seq_rows;      // rows between consecutive sequences in out
  float scale_log2;      // head_dim^-0.5 * log2(e)
  int non_causal;        // 1: every query sees every valid key (the reference without --causal)
  const int* kv_lens;    // per-sequence key count (one past the last valid key; key-padding mask), may be null
  // key-padding masks that are not prefix-valid: key_holes[b] != 0 marks such a sequence, whose
  // key validity is read from key_bits[b * key_words + w] (bit i: key 32w + i) -- one 16-byte
  // group per 128 keys.  Null: every key below the count is valid.
  const uint32_t* key_bits;
  int key_words;
  const int* key_holes;
};

// Whether sequence b's keys must be tested one by one (its mask has holes).
__device__ __forceinline__ bool attn_has_holes(const AttnParams& p, int b) {
  return p.key_holes != nullptr && p.key_holes[b] != 0;
}

// s[c] = -inf for the keys k0 + c (c < N) that sequence b's mask excludes (N = 64 or 128,
// k0 a multiple of N)
template <int N>
__device__ __forceinline__ void attn_mask_keys(const AttnParams& p, int b, int k0, float (&s)[N]) {
  const uint32_t* kb = p.key_bits + static_cast<int64_t>(b) * p.key_words + (k0 >> 5);
  uint32_t w[N / 32];
  if constexpr (N == 128) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(kb));
    w[0] = q.x; w[1] = q.y; w[2] = q.z; w[3] = q.w;
  } else {
    const uint2 q = __ldg(reinterpret_cast<const uint2*>(kb));
    w[0] = q.x; w[1] = q.y;
  }
#pragma unroll
  for (int c = 0; c < N; ++c)
    if (!((w[c >> 5] >> (c & 31)) & 1u)) s[c] = -INFINITY;
}

// Keys [0, kv_eff) of sequence b are valid (at least one, so a row is never empty).
__device__ __forceinline__ int attn_kv_eff(const AttnParams& p, int b) {
  const int l = p.kv_lens ? min(p.kv_len, p.kv_lens[b]) : p.kv_len;
  return l > 0 ? l : 1;
}

template <int HD, int BN>
struct AttnCfg {
  static constexpr int ATOM_E = HD >= 64 ? 64 : HD;   // elements per swizzle row
  static constexpr int ROWB = ATOM_E * 2;             // bytes per swizzle row (128 or 64)
  static constexpr uint32_t SWZ = ATOM_E == 64 ? UMMA_SW128 : UMMA_SW64;
  static constexpr int NBOX = HD / ATOM_E;
  static constexpr int Q_BYTES = 128 * HD * 2;
  static constexpr int KV_BYTES = BN * HD * 2;
  static constexpr int P_BYTES = 128 * BN * 2;
  // P (fp16 pairs, BN/2 columns) in TMEM at column TM_P when it fits beside S
  // and O in the 256 columns each of the two resident CTAs owns; else in smem
  static constexpr bool P_TMEM = BN == 128 && HD <= 64;
  static constexpr uint32_t TM_P = 192;
  static constexpr int ST = 2;  // K/V ring stages
  // two Q buffers (the next work item's Q lands while this one's S MMAs still
  // read the other) wherever they fit
  static constexpr int QS = (2 * Q_BYTES + ST * 2 * KV_BYTES + (P_TMEM ? 0 : P_BYTES) + 256 + 1024) <= 227 * 1024 ? 2 : 1;
  static constexpr int OFF_Q = 0;                   // Q slot q at OFF_Q + q * Q_BYTES
  static constexpr int OFF_KV = QS * Q_BYTES;       // stage s: K at OFF_KV + s * 2 * KV_BYTES, V after it
  static constexpr int OFF_P = OFF_KV + ST * 2 * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + (P_TMEM ? 0 : P_BYTES);
  static constexpr int TOTAL = OFF_BAR + 256 + 1024;
  static constexpr uint32_t TMEM_COLS = (BN + HD) <= 256 ? 256 : 512;
  static_assert(HD % ATOM_E == 0, "head_dim must tile the swizzle atom");
  static_assert(BN % 64 == 0, "key tile must be a multiple of 64");
  static_assert(TOTAL <= 227 * 1024, "shared memory");
};

// One work item of the persistent kernel: a 128-row query tile of one head of one sequence.
struct AttnItem {
  int qt, h, b;
  int q_first, q_last;  // absolute positions of the tile's first and last query rows
  int kv_eff;           // valid keys of the sequence
  int nkt;              // key tiles the tile visits
  bool holes;
};

// Items are numbered longest first: t = r * (H * batch) + b * H + h with query tile
// nqt - 1 - r.  CTA c of G takes t = k * G + c in even rounds k and k * G + (G - 1 - c)
// in odd ones, so that every CTA's sum of key tiles comes out nearly equal.
__device__ __forceinline__ long long attn_item_index(long long k, int G, int c) {
  return k * G + ((k & 1) ? G - 1 - c : c);
}

template <int BN>
__device__ __forceinline__ AttnItem attn_item(const AttnParams& p, long long t, int nqt) {
  AttnItem it;
  // 32-bit arithmetic: the launcher admits fewer than 2^31 items
  const int hb = p.H * p.batch;
  const int ti = static_cast<int>(t);
  const int r = ti / hb;
  const int rem = ti - r * hb;
  it.qt = nqt - 1 - r;
  it.h = rem % p.H;
  it.b = rem / p.H;
  it.q_first = p.q_offset + it.qt * 128;
  it.q_last = p.q_offset + min(p.q_len, (it.qt + 1) * 128) - 1;
  it.kv_eff = attn_kv_eff(p, it.b);
  it.holes = attn_has_holes(p, it.b);
  it.nkt = p.non_causal ? (it.kv_eff + BN - 1) / BN : min(it.q_last / BN + 1, (it.kv_eff + BN - 1) / BN);
  return it;
}

// Persistent: gridDim.x CTAs (two per SM where shared memory allows) walk the
// work items in the order of attn_item_index.  The roles run ahead across item
// boundaries: the producer loads the next item's Q (second buffer) and K/V tiles
// through the same ring, and the MMA warp issues the next item's first S = Q.K^T
// as soon as the softmax has read the last S of this one, so the next item's
// softmax starts while this item's context is normalised and stored.  One
// running tile count g orders every barrier phase across items.
template <int HD, int BN>
__global__ void __launch_bounds__(192, 2)  // two CTAs per SM (registers <= 170)
    k_flash_causal(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using C = AttnCfg<HD, BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars + 0;    // [QS]
  uint64_t* q_empty = bars + 2;   // [QS]: the item's last S MMA has read Q
  uint64_t* kv_full = bars + 4;   // [ST]
  uint64_t* kv_empty = bars + 6;  // [ST]
  uint64_t* s_full = bars + 8;
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint64_t* drain = bars + 11;
  uint64_t* s_free = bars + 12;  // softmax has read S into registers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = (p.q_len + 127) / 128;
  const long long items = static_cast<long long>(nqt) * p.H * p.batch;
  const int G = gridDim.x, cta = blockIdx.x;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < C::QS; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
#pragma unroll
    for (int i = 0; i < C::ST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    mbar_init(s_free, 128);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncwarp();  // lane-0 roles rejoin their warp: bar.sync is warp-aligned
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_sync();  // the previous kernel's outputs (and the mask's key counts) are complete from here on

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      long long g = 0;        // K/V tiles issued
      int nq0 = 0, nq1 = 0;   // Q loads issued into buffer 0 / 1 (for the abort drain)
      bool ok = true;
      for (long long k = 0; ok; ++k) {
        const long long t = attn_item_index(k, G, cta);
        if (t >= items) break;
        const AttnItem it = attn_item<BN>(p, t, nqt);
        const int qs = static_cast<int>(k % C::QS);
        if (k >= C::QS &&
            !mbar_wait(&q_empty[qs], static_cast<uint32_t>((k / C::QS - 1) & 1), abort_flag, DERR_WAIT_SLOT))
          break;
        const int qrow = p.q_row0 + it.b * p.q_seq_rows + it.qt * 128;
        mbar_arrive_expect_tx(&q_full[qs], C::Q_BYTES);
#pragma unroll
        for (int bx = 0; bx < C::NBOX; ++bx)
          tma_load_2d(smem + C::OFF_Q + qs * C::Q_BYTES + bx * 128 * C::ROWB, &tmQ, &q_full[qs],
                      p.q_col0 + it.h * HD + bx * C::ATOM_E, qrow);
        if (qs) ++nq1; else ++nq0;
        for (int j = 0; j < it.nkt; ++j, ++g) {
          const int s = static_cast<int>(g % C::ST);
          if (g >= C::ST &&
              !mbar_wait(&kv_empty[s], static_cast<uint32_t>((g / C::ST - 1) & 1), abort_flag, DERR_WAIT_SLOT)) {
            ok = false;
            break;
          }
          const int krow = p.kv_row0 + it.b * p.kv_seq_rows + j * BN;
          uint8_t* ks = smem + C::OFF_KV + s * 2 * C::KV_BYTES;
          uint8_t* vs = ks + C::KV_BYTES;
          mbar_arrive_expect_tx(&kv_full[s], 2 * C::KV_BYTES);
#pragma unroll
          for (int bx = 0; bx < C::NBOX; ++bx)
            tma_load_2d(ks + bx * BN * C::ROWB, &tmK, &kv_full[s], p.k_col0 + it.h * HD + bx * C::ATOM_E, krow);
#pragma unroll
          for (int bx = 0; bx < C::NBOX; ++bx)
            tma_load_2d(vs + bx * BN * C::ROWB, &tmV, &kv_full[s], p.v_col0 + it.h * HD + bx * C::ATOM_E, krow);
        }
      }
      if (*abort_flag) {  // let the copies in flight land before the CTA's shared memory goes away
        if (nq0 > 0) mbar_wait_drain(&q_full[0], static_cast<uint32_t>((nq0 - 1) & 1));
        if (nq1 > 0) mbar_wait_drain(&q_full[1], static_cast<uint32_t>((nq1 - 1) & 1));
        for (long long u = (g > C::ST ? g - C::ST : 0); u < g; ++u)
          mbar_wait_drain(&kv_full[u % C::ST], static_cast<uint32_t>((u / C::ST) & 1));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_f16(128, BN, false);
      constexpr uint32_t idesc_o = make_idesc_f16(128, HD, true);
      const uint32_t p_addr = smem_u32(smem + C::OFF_P);
      // S = Q(buffer qs) . K(stage s)^T into TMEM columns [0, BN)
      auto issue_s = [&](int qs, int s) {
        const uint32_t q_addr = smem_u32(smem + C::OFF_Q + qs * C::Q_BYTES);
        const uint32_t k_addr = smem_u32(smem + C::OFF_KV + s * 2 * C::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const int box = (kk * 16) / C::ATOM_E;
          const uint32_t within = ((kk * 16) % C::ATOM_E) * 2;
          const uint64_t ad = make_sdesc(q_addr + box * 128 * C::ROWB + within, 16, 8 * C::ROWB, C::SWZ);
          const uint64_t bd = make_sdesc(k_addr + box * BN * C::ROWB + within, 16, 8 * C::ROWB, C::SWZ);
          umma_f16_ss(tmem, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
      };
      long long t = attn_item_index(0, G, cta);
      if (t < items) {
        AttnItem cur = attn_item<BN>(p, t, nqt);
        long long k = 0;  // item of the CTA
        int j = 0;        // key tile of the item
        long long g = 0;  // key tiles so far
        bool ok = mbar_wait(&q_full[0], 0, abort_flag, DERR_WAIT_TMA) &&
                  mbar_wait(&kv_full[0], 0, abort_flag, DERR_WAIT_TMA);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          if (cur.nkt == 1) tc_commit(&q_empty[0]);
        }
        while (ok) {
          // the tile after g: the next key tile of this item, or the next item's first
          AttnItem nxt = cur;
          long long nk = k;
          int nj = j + 1;
          bool more = true;
          if (nj == cur.nkt) {
            t = attn_item_index(k + 1, G, cta);
            more = t < items;
            if (more) {
              nxt = attn_item<BN>(p, t, nqt);
              nk = k + 1;
              nj = 0;
            }
          }
          // its S as soon as the softmax has read S of tile g (runs during that softmax)
          if (more) {
            const int nqs = static_cast<int>(nk % C::QS);
            if (!mbar_wait(s_free, static_cast<uint32_t>(g & 1), abort_flag, DERR_WAIT_SOFTMAX)) break;
            if (nj == 0 &&
                !mbar_wait(&q_full[nqs], static_cast<uint32_t>((nk / C::QS) & 1), abort_flag, DERR_WAIT_TMA))
              break;
            if (!mbar_wait(&kv_full[(g + 1) % C::ST], static_cast<uint32_t>(((g + 1) / C::ST) & 1), abort_flag,
                           DERR_WAIT_TMA))
              break;
            tc_fence_after();
            issue_s(nqs, static_cast<int>((g + 1) % C::ST));
            if (nj == nxt.nkt - 1) tc_commit(&q_empty[nqs]);  // the item's last read of its Q buffer
          }
          // O += P_g . V_g
          if (!mbar_wait(p_full, static_cast<uint32_t>(g & 1), abort_flag, DERR_WAIT_SOFTMAX)) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + C::OFF_KV + static_cast<int>(g % C::ST) * 2 * C::KV_BYTES + C::KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t bd = make_sdesc(v_addr + kk * 16 * C::ROWB, BN * C::ROWB, 8 * C::ROWB, C::SWZ);
            if constexpr (C::P_TMEM) {
              umma_f16_ts(tmem + BN, tmem + C::TM_P + 8 * kk, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint64_t ad = make_sdesc(p_addr + (kk >> 2) * (128 * 128) + (kk & 3) * 32, 16, 1024, UMMA_SW128);
              umma_f16_ss(tmem + BN, ad, bd, idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
            }
          }
          tc_commit(pv_done);
          tc_commit(&kv_empty[g % C::ST]);
          ++g;
          if (!more) break;
          cur = nxt;
          k = nk;
          j = nj;
        }
      }
      if (*abort_flag) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0);
      }
    }
  } else {
    // softmax / epilogue warps: one query row per thread
    const int qd = warp & 3;
    const int rl = qd * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    uint8_t* ps = smem + C::OFF_P;
    long long g = 0;
    bool ok = true;
    for (long long k = 0; ok; ++k) {
      const long long t = attn_item_index(k, G, cta);
      if (t >= items) break;
      const AttnItem it = attn_item<BN>(p, t, nqt);
      const int qpos = it.q_first + rl;
      // last visible key of this row, and the last one every row of the tile sees
      const int klim = p.non_causal ? it.kv_eff - 1 : min(qpos, it.kv_eff - 1);
      const int kall = p.non_causal ? it.kv_eff - 1 : min(it.q_first, it.kv_eff - 1);
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < it.nkt; ++j, ++g) {
        ok = mbar_wait_warp(s_full, static_cast<uint32_t>(g & 1), abort_flag, DERR_WAIT_MMA);
        if (!ok) break;
        tc_fence_after();
        float s[BN];
        tmem_ld_row<BN>(trow, s);
        tc_fence_before();
        mbar_arrive(s_free);  // the MMA warp may now overwrite S with the next key tile
        const int k0 = j * BN;
        if (k0 + BN - 1 > kall) {  // raw scores; the positive scale is applied in the exponent
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (k0 + c > klim) s[c] = -INFINITY;
        }
        if (it.holes) attn_mask_keys<BN>(p, it.b, k0, s);
        const float m_new = fmaxf(m, row_max<BN>(s) * p.scale_log2);
        // rows with nothing visible yet keep p = 0 (cannot happen for real rows: key 0 is always visible)
        const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
        const float alpha = fast_exp2(m - m_use);  // m = -inf on the first tile -> 0
        const float sum = row_exp2_sum<BN>(s, p.scale_log2, m_use);
        l = l * alpha + sum;
        m = m_new;
        if (j > 0) {  // (tile 0: the previous item's epilogue already waited for its last PV)
          ok = mbar_wait_warp(pv_done, static_cast<uint32_t>((g - 1) & 1), abort_flag, DERR_WAIT_MMA);
          if (!ok) break;
          tc_fence_after();
        }
        if constexpr (C::P_TMEM) {
          // P_j -> TMEM, keys 2i, 2i+1 in column TM_P + i (the PV MMA's A operand)
          uint32_t pk[BN / 2];
#pragma unroll
          for (int i = 0; i < BN / 2; ++i) pk[i] = pack_half2(s[2 * i], s[2 * i + 1]);
          tmem_st64(trow + C::TM_P, pk);
        } else {
          // P_j -> shared memory, 128B-swizzled K-major (keys contiguous), 64 keys per swizzle atom
#pragma unroll
          for (int ch = 0; ch < BN / 8; ++ch) {
            const uint4 v = make_uint4(pack_half2(s[8 * ch + 0], s[8 * ch + 1]), pack_half2(s[8 * ch + 2], s[8 * ch + 3]),
                                       pack_half2(s[8 * ch + 4], s[8 * ch + 5]), pack_half2(s[8 * ch + 6], s[8 * ch + 7]));
            *reinterpret_cast<uint4*>(ps + (ch >> 3) * (128 * 128) + sw128_off(rl, ch & 7)) = v;
          }
        }
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            float o[32];
            tmem_ld32(trow + BN + c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(trow + BN + c, o);
          }
        }
        if constexpr (!C::P_TMEM) fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(p_full);
      }
      if (!ok) break;
      ok = mbar_wait_warp(pv_done, static_cast<uint32_t>((g - 1) & 1), abort_flag, DERR_WAIT_MMA);
      if (!ok || __any_sync(0xffffffffu, *abort_flag != 0)) break;
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;  // a row whose visible keys are all masked: context 0
      const int row_in_seq = it.qt * 128 + rl;
      __half* orow = p.out + (static_cast<int64_t>(it.b) * p.out_seq_rows + row_in_seq) * p.ld_out + it.h * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float o[32];
        tmem_ld32(trow + BN + c, o);
        if (row_in_seq < p.q_len) {
          uint4* o4 = reinterpret_cast<uint4*>(orow + c);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o4[i] = make_uint4(pack_half2(o[8 * i + 0] * inv_l, o[8 * i + 1] * inv_l),
                               pack_half2(o[8 * i + 2] * inv_l, o[8 * i + 3] * inv_l),
                               pack_half2(o[8 * i + 4] * inv_l, o[8 * i + 5] * inv_l),
                               pack_half2(o[8 * i + 6] * inv_l, o[8 * i + 7] * inv_l));
        }
      }
      tc_fence_before();  // the context is read out of TMEM before the next item's PV overwrites it
    }
  }
  tc_fence_before();
  __syncwarp();  // lane-0 roles rejoin their warp: bar.sync is warp-aligned
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace b200
