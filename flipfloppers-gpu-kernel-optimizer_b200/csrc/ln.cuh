// Row LayerNorm, nn.LayerNorm semantics (biased variance, eps inside the
// square root, affine gamma/beta): the reference's norm1 / norm2 / final_norm
// (TTB:146-150, 160-161, 178-189 of torch_transformer_benchmark.py).
// One warp per row; the row is held in registers, mean and variance are two
// warp-shuffle reductions (two-pass, no E[x^2]-E[x]^2 cancellation).
// fp32 in; fp16 out (feeds a GEMM's A operand) or fp32 out (model output).
// Optionally the input row is also copied to `copy_out` (fp32): the block's
// residual stream, onto which the next projection GEMM accumulates in place.
#pragma once

#include "ptx.cuh"

namespace b200 {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// VEC4: d % 128 == 0, each lane handles VPL float4 at columns 4*lane + 128*i.
// Otherwise each lane handles VPL floats at columns lane + 32*i (d % 32 == 0).
template <int VPL, bool VEC4, bool OUT_F16>
__global__ void __launch_bounds__(256)
    k_layernorm(const float* __restrict__ x, int64_t ld_x, const float* __restrict__ gamma,
                const float* __restrict__ beta, void* __restrict__ out, int64_t ld_out, int rows, int d, float eps,
                float* __restrict__ copy_out, int64_t ld_copy) {
  griddep_sync();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (row >= rows) return;
  const float* xr = x + row * ld_x;
  constexpr int NV = VEC4 ? 4 * VPL : VPL;
  float v[NV];
  float s = 0.f;
  if constexpr (VEC4) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const float4 t = *reinterpret_cast<const float4*>(xr + 4 * lane + 128 * i);
      v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
      if (copy_out) *reinterpret_cast<float4*>(copy_out + row * ld_copy + 4 * lane + 128 * i) = t;
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      v[i] = xr[lane + 32 * i];
      if (copy_out) copy_out[row * ld_copy + lane + 32 * i] = v[i];
    }
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) s += v[i];
  const float mean = warp_sum(s) / static_cast<float>(d);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] -= mean;
    q += v[i] * v[i];
  }
  const float var = warp_sum(q) / static_cast<float>(d);
  const float rstd = rsqrtf(var + eps);
  if constexpr (VEC4) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = 4 * lane + 128 * i;
      const float4 g = *reinterpret_cast<const float4*>(gamma + c);
      const float4 bb = *reinterpret_cast<const float4*>(beta + c);
      const float y0 = v[4 * i] * rstd * g.x + bb.x, y1 = v[4 * i + 1] * rstd * g.y + bb.y;
      const float y2 = v[4 * i + 2] * rstd * g.z + bb.z, y3 = v[4 * i + 3] * rstd * g.w + bb.w;
      if constexpr (OUT_F16) {
        *reinterpret_cast<uint2*>(static_cast<__half*>(out) + row * ld_out + c) =
            make_uint2(pack_half2(y0, y1), pack_half2(y2, y3));
      } else {
        *reinterpret_cast<float4*>(static_cast<float*>(out) + row * ld_out + c) = make_float4(y0, y1, y2, y3);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = lane + 32 * i;
      const float y = v[i] * rstd * gamma[c] + beta[c];
      if constexpr (OUT_F16) {
        static_cast<__half*>(out)[row * ld_out + c] = __float2half_rn(y);
      } else {
        static_cast<float*>(out)[row * ld_out + c] = y;
      }
    }
  }
}

// sum = a + b (+ bias per column), written out in fp32, then LayerNorm(sum) ->
// out (fp16 or fp32): the residual add after a tensor-parallel all-reduce fused
// with the LayerNorm that follows it.  d % 128 == 0.  sum_out may alias a
// (each element is read and written by the same thread).
template <int VPL, bool OUT_F16>
__global__ void __launch_bounds__(256)
    k_add_layernorm(const float* a, const float* __restrict__ b, const float* __restrict__ bias,
                    float* sum_out, const float* __restrict__ gamma, const float* __restrict__ beta,
                    void* __restrict__ out, int rows, int d, float eps) {
  griddep_sync();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (row >= rows) return;
  float v[4 * VPL];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = 4 * lane + 128 * i;
    const float4 ta = *reinterpret_cast<const float4*>(a + row * d + c);
    const float4 tb = *reinterpret_cast<const float4*>(b + row * d + c);
    float4 tc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (bias) tc = *reinterpret_cast<const float4*>(bias + c);
    v[4 * i] = ta.x + tb.x + tc.x;
    v[4 * i + 1] = ta.y + tb.y + tc.y;
    v[4 * i + 2] = ta.z + tb.z + tc.z;
    v[4 * i + 3] = ta.w + tb.w + tc.w;
    *reinterpret_cast<float4*>(sum_out + row * d + c) = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    s += v[4 * i] + v[4 * i + 1] + v[4 * i + 2] + v[4 * i + 3];
  }
  const float mean = warp_sum(s) / static_cast<float>(d);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 4 * VPL; ++i) {
    v[i] -= mean;
    q += v[i] * v[i];
  }
  const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(d) + eps);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = 4 * lane + 128 * i;
    const float4 g = *reinterpret_cast<const float4*>(gamma + c);
    const float4 bb = *reinterpret_cast<const float4*>(beta + c);
    const float y0 = v[4 * i] * rstd * g.x + bb.x, y1 = v[4 * i + 1] * rstd * g.y + bb.y;
    const float y2 = v[4 * i + 2] * rstd * g.z + bb.z, y3 = v[4 * i + 3] * rstd * g.w + bb.w;
    if constexpr (OUT_F16) {
      *reinterpret_cast<uint2*>(static_cast<__half*>(out) + row * d + c) = make_uint2(pack_half2(y0, y1), pack_half2(y2, y3));
    } else {
      *reinterpret_cast<float4*>(static_cast<float*>(out) + row * d + c) = make_float4(y0, y1, y2, y3);
    }
  }
}

// ------------------------------------------------------------------ key-padding mask, read on the device
// The reference's valid_token_mask [B, S] (TTB:125-128, 140-141, 163-164,
// 190-191): padded keys are excluded from attention and padded rows of every
// block output are zero.  The mask is read on the device on every call --
// nothing about its contents is cached on the host, where an in-place edit or
// a new mask at a reused address would go unseen.  k_mask_prepare turns it
// into what the attention kernels take: per sequence the key count to scan
// (one past the last valid key), a flag for masks that are not prefix-valid
// (a valid token after a padded one), and the mask packed as bits, 128 keys
// per 16-byte group.  A prefix-valid sequence (every mask the reference
// harness generates, TTB:1793-1803) needs only the key count; the attention
// kernels read the bits only for flagged sequences.

// One CTA per sequence: the number of valid tokens, one past the last valid one, and
// whether a valid token follows a padded one (not prefix-valid).  Called by every thread.
__device__ __forceinline__ void mask_scan(const unsigned char* __restrict__ m, int S, int& count, int& end,
                                          bool& holes) {
  int c = 0, e = 0;
  bool h = false;
  int i0 = 0;  // first byte left to the scalar loop
  if ((reinterpret_cast<uintptr_t>(m) & 15u) == 0) {
    // 16 bytes per thread and step; byte k of a chunk is valid if nonzero, and a hole is a
    // valid byte after a padded one (the byte before the chunk comes from a scalar load)
    const int nv = S >> 4;
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
      const uint4 q = reinterpret_cast<const uint4*>(m)[v];
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
      bool prev = v > 0 ? m[16 * v - 1] != 0 : true;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const bool cur = ((w[k >> 2] >> (8 * (k & 3))) & 0xffu) != 0;
        c += cur;
        if (cur) e = max(e, 16 * v + k + 1);
        h |= cur && !prev;
        prev = cur;
      }
    }
    i0 = nv << 4;
  }
  for (int i = i0 + threadIdx.x; i < S; i += blockDim.x) {
    const bool v = m[i] != 0;
    c += v;
    if (v) e = max(e, i + 1);
    if (v && i > 0 && m[i - 1] == 0) h = true;
  }
  // block reductions: sum and max (per-warp shuffles, then shared memory) and an OR
  __shared__ int part[2][32];
  for (int o = 16; o > 0; o >>= 1) {
    c += __shfl_xor_sync(0xffffffffu, c, o);
    e = max(e, __shfl_xor_sync(0xffffffffu, e, o));
  }
  if ((threadIdx.x & 31) == 0) {
    part[0][threadIdx.x >> 5] = c;
    part[1][threadIdx.x >> 5] = e;
  }
  holes = __syncthreads_or(h) != 0;
  int t = 0, te = 0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
    t += part[0][w];
    te = max(te, part[1][w]);
  }
  count = t;
  end = te;
}

// Per sequence b (grid = batch, block = 256): kv_lens[b] = one past the last valid key
// (keys past it are never scanned), holes[b] = mask not prefix-valid, and
// key_bits[b * words + w] bit i = key 32w + i valid (words = 4 * ceil(S / 128); bits past
// S are 0).  holes / key_bits may be null (prefix-valid masks only need kv_lens).
__global__ void __launch_bounds__(256)
    k_mask_prepare(const unsigned char* __restrict__ mask, int S, int* __restrict__ kv_lens, int* __restrict__ holes,
                   uint32_t* __restrict__ key_bits, int words) {
  griddep_sync();
  const unsigned char* m = mask + static_cast<int64_t>(blockIdx.x) * S;
  int count, end;
  bool h;
  mask_scan(m, S, count, end, h);
  if (threadIdx.x == 0) {
    kv_lens[blockIdx.x] = end;
    if (holes) holes[blockIdx.x] = h ? 1 : 0;
  }
  if (key_bits != nullptr && h) {  // the attention kernels read the bits of flagged sequences only
    uint32_t* kb = key_bits + static_cast<int64_t>(blockIdx.x) * words;
    for (int w = threadIdx.x; w < words; w += blockDim.x) {
      uint32_t bits = 0;
      for (int i = 0; i < 32; ++i) {
        const int k = 32 * w + i;
        if (k < S && m[k] != 0) bits |= 1u << i;
      }
      kb[w] = bits;
    }
  }
}

// After the forward: every row whose mask byte is 0 is set to 0 (the reference zeroes
// padded rows of the output, TTB:190-191).  A warp takes 32 consecutive rows: one
// coalesced byte load per lane, a ballot, then the whole warp zeroes each padded row of
// the 32 (a mask without padding costs one pass over its bytes).  y fp32 [rows, d].
__global__ void __launch_bounds__(256)
    k_mask_finish(float* __restrict__ y, const unsigned char* __restrict__ mask, long long rows, int d, int vec4) {
  griddep_sync();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long r0 = (static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + warp) * 32;
  if (r0 >= rows) return;
  const long long r = r0 + lane;
  uint32_t pad = __ballot_sync(0xffffffffu, r < rows && mask[r] == 0);
  while (pad) {
    const int k = __ffs(pad) - 1;
    pad &= pad - 1;
    float* yr = y + (r0 + k) * d;
    if (vec4) {  // d % 4 == 0 and y 16-byte aligned (checked by the launcher)
      for (int c = lane; c < d / 4; c += 32) reinterpret_cast<float4*>(yr)[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    } else {
      for (int c = lane; c < d; c += 32) yr[c] = 0.f;
    }
  }
}

}  // namespace b200
