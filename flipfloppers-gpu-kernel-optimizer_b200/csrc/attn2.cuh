// Causal flash attention, two query tiles per CTA (head_dim 32 or 64).
//
// Same semantics and argument block as k_flash_causal (attn.cuh): the
// reference's causal attention (TTB:117-132) with the prefix offset of its
// chunked forward (TTB:1491-1500).  Structure:
//   warp 0      TMA producer: Q tiles t=0,1 (rows qp*256 + t*128 ...), then K_j / V_j
//               into a 3-deep ring shared by both query tiles;
//   warp 1      TMEM owner and MMA issuer, ping-ponging the two tiles:
//               S_t,j = Q_t.K_j^T into TMEM columns [128t, 128t+128) and
//               O_t += P_t,j.V_j into [256 + t*HD, ...).  S_t,j+1 is issued as
//               soon as the softmax has read S_t,j into registers (s_free), so
//               the next tile's QK^T runs during this tile's softmax and the
//               softmax never waits for an MMA round trip;
//   warps 2-5   softmax of query tile 0, warps 6-9 of tile 1: one row per
//               thread, log2-domain running max with lazy rescaling (the max
//               used for the exponentials moves only when a new tile raises it
//               by more than 8, i.e. P <= 2^8; only then is O rescaled in TMEM),
//               P in fp16 into TMEM columns [384 + 64t, 448 + 64t) (two keys
//               per 32-bit column), which the PV MMA reads as its A operand.
// TMEM: S_0 [0,128) | S_1 [128,256) | O_0, O_1 [256, 256+2*HD) | P_0, P_1 [384,512).
// Key tiles past a query tile's diagonal are skipped; query tile 1 may need
// one more key tile than tile 0.
#pragma once

#include "attn.cuh"

namespace b200 {

template <int HD>
struct Attn2Cfg {
  static constexpr int BN = 128;
  static constexpr int ATOM_E = HD;                     // 32 -> SW64, 64 -> SW128 (one box per tile)
  static constexpr int ROWB = HD * 2;
  static constexpr uint32_t SWZ = HD == 64 ? UMMA_SW128 : UMMA_SW64;
  static constexpr int ST = 3;                          // K/V ring depth
  static constexpr int Q_BYTES = 128 * HD * 2;
  static constexpr int KV_BYTES = BN * HD * 2;
  static constexpr int OFF_Q = 0;                       // [2]
  static constexpr int OFF_K = 2 * Q_BYTES;             // [ST] K, then [ST] V
  static constexpr int OFF_V = OFF_K + ST * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + ST * KV_BYTES;
  static constexpr uint32_t TM_P = 384;                 // P_t at TM_P + 64 t
  static constexpr int TOTAL = OFF_BAR + 256 + 1024;
  static constexpr float RESCALE_THRESHOLD = 8.0f;      // log2 units
  static_assert(HD == 32 || HD == 64, "two-tile kernel covers head_dim 32 and 64");
};

template <int HD>
__global__ void __launch_bounds__(320, 1)
    k_flash_causal2(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnParams p) {
  using C = Attn2Cfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;            // [ST]
  uint64_t* kv_empty = kv_full + C::ST;    // [ST]
  uint64_t* s_full = kv_empty + C::ST;     // [2]
  uint64_t* p_full = s_full + 2;           // [2]
  uint64_t* pv_done = p_full + 2;          // [2]
  uint64_t* s_free = pv_done + 2;          // [2] softmax has read S_t into registers
  uint64_t* drain = s_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npair = (p.q_len + 255) / 256;
  const int qp = npair - 1 - static_cast<int>(blockIdx.x);  // latest query rows first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kv_eff = attn_kv_eff(p, b);
  const bool holes = attn_has_holes(p, b);
  const int kv_tiles = (kv_eff + C::BN - 1) / C::BN;
  // key tiles each query tile needs (0 if the tile holds no query row)
  int ntile[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int r0 = qp * 256 + t * 128;
    if (r0 >= p.q_len) {
      ntile[t] = 0;
    } else {
      const int q_last = p.q_offset + min(p.q_len, r0 + 128) - 1;
      ntile[t] = p.non_causal ? kv_tiles : min(q_last / C::BN + 1, kv_tiles);
    }
  }
  const int n_all = max(ntile[0], ntile[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::ST; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 128);
      mbar_init(&pv_done[t], 1);
      mbar_init(&s_free[t], 128);
    }
    mbar_init(drain, 1);
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
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const int qrow = p.q_row0 + b * p.q_seq_rows + qp * 256;
      mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
      tma_load_2d(smem + C::OFF_Q, &tmQ, q_full, p.q_col0 + h * HD, qrow);
      tma_load_2d(smem + C::OFF_Q + C::Q_BYTES, &tmQ, q_full, p.q_col0 + h * HD, qrow + 128);
      int issued = 0;
      for (int j = 0; j < n_all; ++j) {
        const int s = j % C::ST;
        if (j >= C::ST && !mbar_wait(&kv_empty[s], ((j / C::ST) - 1) & 1, abort_flag, DERR_WAIT_SLOT)) break;
        const int krow = p.kv_row0 + b * p.kv_seq_rows + j * C::BN;
        mbar_arrive_expect_tx(&kv_full[s], 2 * C::KV_BYTES);
        tma_load_2d(smem + C::OFF_K + s * C::KV_BYTES, &tmK, &kv_full[s], p.k_col0 + h * HD, krow);
        tma_load_2d(smem + C::OFF_V + s * C::KV_BYTES, &tmV, &kv_full[s], p.v_col0 + h * HD, krow);
        issued = j + 1;
      }
      if (*abort_flag) {
        mbar_wait_drain(q_full, 0);
        for (int j = (issued > C::ST ? issued - C::ST : 0); j < issued; ++j)
          mbar_wait_drain(&kv_full[j % C::ST], (j / C::ST) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_f16(128, C::BN, false);
      constexpr uint32_t idesc_o = make_idesc_f16(128, HD, true);
      const uint32_t q_addr = smem_u32(smem + C::OFF_Q);
      const uint32_t k_addr = smem_u32(smem + C::OFF_K);
      const uint32_t v_addr = smem_u32(smem + C::OFF_V);
      int kv_seen = 0;  // key tiles whose TMA load has been waited for
      bool ok = mbar_wait(q_full, 0, abort_flag, DERR_WAIT_TMA);
      auto need_kv = [&](int j) {
        while (ok && kv_seen <= j) {
          if (!mbar_wait(&kv_full[kv_seen % C::ST], (kv_seen / C::ST) & 1, abort_flag, DERR_WAIT_TMA)) ok = false;
          ++kv_seen;
        }
        if (ok) tc_fence_after();
        return ok;
      };
      auto issue_s = [&](int t, int j) {
        const uint32_t kk_base = k_addr + (j % C::ST) * C::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          umma_f16_ss(tmem + t * 128, make_sdesc(q_addr + t * C::Q_BYTES + kk * 32, 16, 8 * C::ROWB, C::SWZ),
                      make_sdesc(kk_base + kk * 32, 16, 8 * C::ROWB, C::SWZ), idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[t]);
      };
      if (ok && n_all > 0 && need_kv(0)) {
        if (ntile[0] > 0) issue_s(0, 0);
        if (ntile[1] > 0) issue_s(1, 0);
      }
      auto issue_pv = [&](int t, int j) {
        tc_fence_after();
        const uint32_t vb = v_addr + (j % C::ST) * C::KV_BYTES;
        const uint32_t pt = tmem + C::TM_P + 64 * t;  // P_t: 16 keys per 8 columns
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk)
          umma_f16_ts(tmem + 256 + t * HD, pt + 8 * kk,
                      make_sdesc(vb + kk * 16 * C::ROWB, C::BN * C::ROWB, 8 * C::ROWB, C::SWZ), idesc_o,
                      (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&pv_done[t]);
      };
      // Issue order = the order the softmax events arrive (the two tiles' exp phases
      // alternate, so tile 0 frees S of key tile j before tile 1 hands over P of tile j-1,
      // and so on): S_0,j+1 | P_1,j-1.V (then key tile j-1's K/V slot is released) |
      // S_1,j+1 | P_0,j.V.  Waiting for the four in a fixed per-tile order instead held
      // tile 0's next QK^T behind tile 1's PV by most of an exp phase.
      for (int j = 0; ok && j <= n_all; ++j) {
        if (j + 1 < ntile[0]) {
          if (!mbar_wait(&s_free[0], j & 1, abort_flag, DERR_WAIT_SOFTMAX) || !need_kv(j + 1)) {
            ok = false;
            break;
          }
          issue_s(0, j + 1);
        }
        if (j >= 1) {
          if (j - 1 < ntile[1]) {
            if (!mbar_wait(&p_full[1], (j - 1) & 1, abort_flag, DERR_WAIT_SOFTMAX)) {
              ok = false;
              break;
            }
            issue_pv(1, j - 1);
          }
          tc_commit(&kv_empty[(j - 1) % C::ST]);  // both query tiles are done with key tile j-1
        }
        if (j == n_all) break;
        if (j + 1 < ntile[1]) {
          if (!mbar_wait(&s_free[1], j & 1, abort_flag, DERR_WAIT_SOFTMAX) || !need_kv(j + 1)) {
            ok = false;
            break;
          }
          issue_s(1, j + 1);
        }
        if (j < ntile[0]) {
          if (!mbar_wait(&p_full[0], j & 1, abort_flag, DERR_WAIT_SOFTMAX)) {
            ok = false;
            break;
          }
          issue_pv(0, j);
        }
      }
      if (*abort_flag) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0);
      }
    }
  } else {
    // softmax warpgroup t = 0 (warps 2-5) or 1 (warps 6-9)
    const int t = (warp - 2) >> 2;
    const int qd = warp & 3;
    const int rl = qd * 32 + lane;
    const int row_in_seq = qp * 256 + t * 128 + rl;
    const int qpos = p.q_offset + row_in_seq;
    const int q_first = p.q_offset + qp * 256 + t * 128;
    const uint32_t trow = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    const int nt = ntile[t];
    // The two softmax warps that share an SMSP (quadrant qd of tile 0 and of
    // tile 1) take turns on the exponentials: tile 0 waits for token A, tile 1
    // for token B, each passes the other's token on when its exp loop is done.
    // Alternating keeps the SFU busy while the other warp loads S, reduces the
    // max and writes P.  Token k of each kind is passed only when its receiver
    // has a k-th exp phase (tile 1 may have one key tile more, or none), and
    // the sequence never depends on data or errors, so no wait is left
    // unmatched.
    const int n0 = ntile[0], n1 = ntile[1];
    const int bar_a = 1 + qd, bar_b = 5 + qd;
    if (t == 1 && n0 > 0) nbar_arrive(bar_a, 64);
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      if (ok) ok = mbar_wait_warp(&s_full[t], j & 1, abort_flag, DERR_WAIT_MMA);
      float s[C::BN];
      float alpha = 1.f, m_use = 0.f;
      if (ok) {
        tc_fence_after();
        tmem_ld_row<C::BN>(trow + t * 128, s);
        tc_fence_before();
        mbar_arrive(&s_free[t]);  // the MMA warp may now overwrite S_t with the next key tile
        const int k0 = j * C::BN;
        const int klim = p.non_causal ? kv_eff - 1 : min(qpos, kv_eff - 1);  // last visible key of this row
        const bool need_mask = (k0 + C::BN - 1) > (p.non_causal ? kv_eff - 1 : min(q_first, kv_eff - 1));
        if (need_mask) {  // raw scores; the positive scale is applied in the exponent
#pragma unroll
          for (int c = 0; c < C::BN; ++c)
            if (k0 + c > klim) s[c] = -INFINITY;
        }
        if (holes) attn_mask_keys<C::BN>(p, b, k0, s);
        const float mx = row_max<C::BN>(s) * p.scale_log2;
        // lazy rescale: move the reference max only when this tile raises it by more than the threshold
        const bool grow = mx > m_used + C::RESCALE_THRESHOLD;
        const float m_new = grow ? mx : m_used;
        alpha = grow ? fast_exp2(m_used - m_new) : 1.f;  // 0 on the first tile
        m_use = (m_new == -INFINITY) ? 0.f : m_new;
        m_used = m_new;
      } else {
#pragma unroll
        for (int c = 0; c < C::BN; ++c) s[c] = 0.f;  // keeps the exp phase unconditional
      }
      if (t == 0) {
        if (j == 0 || j - 1 < n1) nbar_sync(bar_a, 64);
      } else {
        if (j < n0) nbar_sync(bar_b, 64);
      }
      l = l * alpha + row_exp2_sum<C::BN>(s, p.scale_log2, m_use);
      if (t == 0) {
        if (j < n1) nbar_arrive(bar_b, 64);
      } else {
        if (j + 1 < n0) nbar_arrive(bar_a, 64);
      }
      if (ok && j > 0) {
        ok = mbar_wait_warp(&pv_done[t], (j - 1) & 1, abort_flag, DERR_WAIT_MMA);
        if (ok) tc_fence_after();
      }
      if (ok) {
        uint32_t pk[C::BN / 2];  // keys 2i, 2i+1 -> column i (low, high half)
#pragma unroll
        for (int i = 0; i < C::BN / 2; ++i) pk[i] = pack_half2(s[2 * i], s[2 * i + 1]);
        tmem_st64(trow + C::TM_P + 64 * t, pk);
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < HD; c += 32) {
            float o[32];
            tmem_ld32(trow + 256 + t * HD + c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(trow + 256 + t * HD + c, o);
          }
        }
        tc_fence_before();
        mbar_arrive(&p_full[t]);
      }
    }
    if (ok && nt > 0) ok = mbar_wait_warp(&pv_done[t], (nt - 1) & 1, abort_flag, DERR_WAIT_MMA);
    if (ok && nt > 0 && !*abort_flag) {
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;  // a row whose visible keys are all masked: context 0
      __half* orow = p.out + (static_cast<int64_t>(b) * p.out_seq_rows + row_in_seq) * p.ld_out + h * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float o[32];
        tmem_ld32(trow + 256 + t * HD + c, o);
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
    }
  }
  tc_fence_before();
  __syncwarp();  // lane-0 roles rejoin their warp: bar.sync is warp-aligned
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace b200
