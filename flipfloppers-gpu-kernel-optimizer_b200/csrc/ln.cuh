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

// y[r, :] = 0 for every row whose valid flag is 0 (the reference zeroes padded
// query rows of the model output, TTB:190-191).  One warp per row.
__global__ void __launch_bounds__(256)
    k_zero_masked_rows(float* __restrict__ y, const unsigned char* __restrict__ valid, long long rows, int d) {
  griddep_sync();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (row >= rows || valid[row]) return;
  float* yr = y + row * d;
  for (int c = lane; c < d; c += 32) yr[c] = 0.f;
}

// ------------------------------------------------------------------ key-padding mask, checked on the device
// The reference's valid_token_mask [B, S] (TTB:125-128, 140-141, 163-164,
// 190-191): padded keys are excluded from attention and padded rows of every
// block output are zero.  The kernel chain handles prefix-valid masks (valid
// tokens first, padding last, what the harness's generate_random_case makes,
// TTB:1793-1803) through per-sequence key counts, so the mask is read on the
// device on every call -- nothing about its contents is cached on the host,
// where an in-place edit or a new mask at a reused address would go unseen.

// One CTA per sequence: the number of valid tokens and whether a valid token
// follows a padded one (a hole: not prefix-valid).  Called by every thread.
__device__ __forceinline__ void mask_scan(const unsigned char* __restrict__ m, int S, int& count, bool& holes) {
  int c = 0;
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
        h |= cur && !prev;
        prev = cur;
      }
    }
    i0 = nv << 4;
  }
  for (int i = i0 + threadIdx.x; i < S; i += blockDim.x) {
    const bool v = m[i] != 0;
    c += v;
    if (v && i > 0 && m[i - 1] == 0) h = true;
  }
  // block reductions: a sum (per-warp shuffles, then shared memory) and an OR
  __shared__ int part[32];
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
  holes = __syncthreads_or(h) != 0;
  int t = 0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += part[w];
  count = t;
}

// kv_lens[b] = valid tokens of sequence b (the key count attention uses);
// a mask with a hole records DERR_MASK_HOLES.  grid = batch, block = 256.
__global__ void __launch_bounds__(256)
    k_mask_prepare(const unsigned char* __restrict__ mask, int S, int* __restrict__ kv_lens) {
  griddep_sync();
  int count;
  bool holes;
  mask_scan(mask + static_cast<int64_t>(blockIdx.x) * S, S, count, holes);
  if (threadIdx.x == 0) {
    kv_lens[blockIdx.x] = count;
    if (holes) record_error(DERR_MASK_HOLES);
  }
}

// After the chain: the padded rows [count, S) of sequence b are set to 0.  A
// sequence whose mask has a hole was computed with the wrong key set, so all of
// its rows are set to NaN and DERR_MASK_HOLES is recorded: a wrong result never
// passes as a plausible one.  grid = batch, block = 256; y fp32 [B*S, d].
__global__ void __launch_bounds__(256)
    k_mask_finish(float* __restrict__ y, const unsigned char* __restrict__ mask, int S, int d, int vec4) {
  griddep_sync();
  int count;
  bool holes;
  mask_scan(mask + static_cast<int64_t>(blockIdx.x) * S, S, count, holes);
  if (holes && threadIdx.x == 0) record_error(DERR_MASK_HOLES);
  const int r0 = holes ? 0 : count;
  const float fill = holes ? __int_as_float(0x7fc00000) : 0.f;
  float* ys = y + (static_cast<int64_t>(blockIdx.x) * S + r0) * d;
  const int64_t n = static_cast<int64_t>(S - r0) * d;
  if (vec4) {  // d % 4 == 0 and y 16-byte aligned (checked by the launcher)
    float4* y4 = reinterpret_cast<float4*>(ys);
    for (int64_t i = threadIdx.x; i < n / 4; i += blockDim.x) y4[i] = make_float4(fill, fill, fill, fill);
  } else {
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) ys[i] = fill;
  }
}

}  // namespace b200
