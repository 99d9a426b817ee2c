/*
 * b200_block.h -- C ABI of the B200 (sm_100a) causal transformer-block library
 * (libb200block.so).
 *
 * Plain pointers, sizes and an opaque CUDA stream; no framework types.  All
 * device pointers are CUDA device addresses on the calling thread's current
 * device.  Every launcher returns an int status (B200_OK or a negative code,
 * see b200_status_str) and never synchronises; none falls back to another
 * implementation when a shape is unsupported -- it returns the error.
 *
 * It replaces the native boundary of yeoshuyi/Flipfloppers-GPU-Kernel-Optimizer:
 *   - ws_gemm_launch(cfg, In, W, bias, Out, M, N, K, stream, &smem)
 *       (csrc/g4_4_warpspec_gemm.cu:997-1005) and its ffn_gelu_linear variant
 *       (torch_transformer_benchmark.py:518-586)  -> b200_gemm_launch
 *   - the attention call of the causal forward, SDPA is_causal=True
 *       (torch_transformer_benchmark.py:1309-1312) and the prefix-causal flash
 *       call of the chunked forward (torch_transformer_benchmark.py:1491-1500)
 *                                                  -> b200_flash_causal_launch
 *   - F.layer_norm of norm1 / norm2 / final_norm
 *       (torch_transformer_benchmark.py:1293, 1348, 1373) -> b200_layernorm_launch
 *       (norm1 together with the residual copy: b200_layernorm_residual_launch;
 *        out_proj / ffn_out + residual + norm2 / final_norm in one kernel:
 *        b200_gemm_residual_layernorm_launch)
 *   - the per-layer body of _optimized_forward_causal
 *       (torch_transformer_benchmark.py:1282-1373)  -> b200_block_forward
 *   - the unwired causal megakernel mega_causal_forward
 *       (csrc/g5_mega_causal.cpp:7-18)              -> b200_block_fused_small_launch
 *   - ws_gemm_num_cfg / ws_gemm_cfg_desc (csrc/g4_4_warpspec_gemm.cu:1022-1069)
 *       -> b200_abi_version / b200_status_str (no config table: tiles are
 *          chosen inside the library from the shape)
 */
#ifndef B200_BLOCK_H
#define B200_BLOCK_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t passed as an opaque pointer; 0 is the legacy default stream. */
typedef void* b200_stream_t;

#define B200_ABI_VERSION 2  /* 2: key-padding masks of any shape (key_bits / key_holes) */

/* Status codes.  -1..-4 keep the meaning of the reference's ws_launch return
 * codes (csrc/g4_4_warpspec_gemm.cu:958-975); the rest are new. */
enum {
  B200_OK = 0,
  B200_ERR_CONFIG = -1,    /* unknown epilogue / unsupported configuration          */
  B200_ERR_TILE = -2,      /* a dimension is not a multiple of the required granule  */
  B200_ERR_SPLIT = -3,     /* (reserved: the reference's K % SPLIT check)            */
  B200_ERR_SMEM = -4,      /* dynamic shared-memory opt-in refused                   */
  B200_ERR_ALIGN = -5,     /* pointer or leading dimension not 16-byte aligned       */
  B200_ERR_HEAD_DIM = -6,  /* head_dim not in {8, 16, 32, 64, 128, 256}             */
  B200_ERR_DEVICE = -7,    /* a device-side wait timed out (see b200_device_error)   */
  B200_ERR_LAUNCH = -8,    /* the CUDA launch itself failed                          */
  B200_ERR_ARG = -9,       /* null pointer, negative size or inconsistent arguments  */
  B200_ERR_TMAP = -10,     /* TMA tensor-map encoding failed                         */
  B200_ERR_ARCH = -11,     /* current device is not compute capability 10.0 (B200)  */
  B200_ERR_WORKSPACE = -12, /* workspace missing or smaller than required            */
  B200_ERR_NOALLOC_LIMIT = -13, /* problem needs more scratch than B200_NOALLOC_SCRATCH_BYTES */
  B200_ERR_SCRATCH_SETUP = -14  /* the static scratch buffer's device address could not be resolved */
};

/* Epilogues of b200_gemm_launch. */
enum {
  B200_EPI_BIAS_F16 = 0,       /* out(f16) = A.W^T + bias                     */
  B200_EPI_BIAS_GELU_F16 = 1,  /* out(f16) = gelu_erf(A.W^T + bias)           */
  B200_EPI_BIAS_RESID_F32 = 2, /* out(f32) = resid + A.W^T + bias (in place ok) */
  B200_EPI_BIAS_F32 = 3        /* out(f32) = A.W^T + bias (bias may be null)   */
};

int b200_abi_version(void);
const char* b200_status_str(int status);

/* Human-readable detail of the calling thread's last failed CUDA call inside
 * the library (e.g. the CUDA error string of a failed launch); "" if none. */
const char* b200_last_error_detail(void);

/* Device error word of the current device: first device-side failure code
 * since the last clear (0 = none).  Synchronises the device.  clear != 0
 * resets it to 0. */
int b200_device_error(int clear);

/* out[r, :] = LayerNorm(x[r, :]) * gamma + beta over d columns (biased
 * variance, eps inside the sqrt).  out_f16 selects fp16 or fp32 output.
 * d % 32 == 0, d <= 4096. */
int b200_layernorm_launch(const float* x, long long ld_x, const float* gamma, const float* beta, void* out,
                          long long ld_out, int out_f16, int rows, int d, float eps, b200_stream_t stream);

/* b200_layernorm_launch that also copies x's rows (fp32) into residual_out
 * [rows, ld_residual]: norm1 together with the residual stream the block's
 * output projection then accumulates onto in place (torch_transformer_benchmark.py
 * 1293 and 1333-1339, `residual = x`).  residual_out must not overlap x or out. */
int b200_layernorm_residual_launch(const float* x, long long ld_x, const float* gamma, const float* beta, void* out,
                                   long long ld_out, int out_f16, float* residual_out, long long ld_residual,
                                   int rows, int d, float eps, b200_stream_t stream);

/* sum_out = a + b (+ bias[col]) in fp32, then out = LayerNorm(sum_out) *
 * gamma + beta (fp16 or fp32): the residual add after a tensor-parallel
 * all-reduce fused with the LayerNorm that follows (norm2 / final_norm of the
 * reference, TTB:160-161, 189).  Row-major [rows, d], d % 128 == 0. */
int b200_add_layernorm_launch(const float* a, const float* b, const float* bias, float* sum_out, const float* gamma,
                              const float* beta, void* out, int out_f16, int rows, int d, float eps,
                              b200_stream_t stream);

/* y[r, :] = 0 for every row r with row_valid[r] == 0: the reference zeroes
 * padded query rows of the model output (torch_transformer_benchmark.py:190-191).
 * y fp32 [rows, d], row_valid uint8 [rows] (nonzero = valid). */
int b200_zero_masked_rows(float* y, const unsigned char* row_valid, long long rows, int d, b200_stream_t stream);

/* The key-padding mask of the kernel chain (b200_block_forward and the chunked
 * forward), read on the device on every call so that nothing about a mask's
 * contents has to be cached on the host.  Replaces the reference's
 * `_mask_is_all_ones` property cache (torch_transformer_benchmark.py:1011-1025);
 * the semantics are the reference's masking of padded keys and rows (TTB:125-128,
 * 140-141, 163-164, 190-191) for any mask.  mask: [batch, seq_len] bytes,
 * nonzero = valid token (a torch bool tensor as is).
 *
 * b200_mask_prepare writes, per sequence b: kv_lens[b] = one past the last valid
 * token (attention scans no key past it); key_holes[b] = 1 if a valid token
 * follows a padded one (the mask is not prefix-valid), else 0; and for such a
 * sequence the mask as bits, key_bits[b * b200_mask_key_words(seq_len) + w] bit i
 * = token 32w + i valid.  Pass the three to B200BlockArgs / B200AttnArgs
 * (key_words = b200_mask_key_words(seq_len)).  key_holes / key_bits may be NULL
 * when only prefix-valid masks occur (what the reference harness generates,
 * TTB:1793-1803); kv_lens is then all attention needs under causal attention.
 * After the forward, b200_zero_masked_rows(y, mask, batch*seq_len, d) zeroes the
 * padded rows.  (The single-kernel path, b200_block_fused_small_launch, reads the
 * mask bytes itself.) */
int b200_mask_key_words(int seq_len);
int b200_mask_prepare(const unsigned char* mask, int batch, int seq_len, int* kv_lens, int* key_holes,
                      unsigned int* key_bits, b200_stream_t stream);

/* out[M,N] = epilogue(A[M,K] . W[N,K]^T + bias[N]).  A, W fp16 row-major with
 * leading dimensions lda, ldw (elements); bias fp32 (may be null); resid fp32
 * [M, ld_resid] for B200_EPI_BIAS_RESID_F32.  The residual epilogue adds onto
 * out in place (out == resid, same leading dimension: no extra traffic);
 * a different resid is first copied into out, so it must not overlap out.
 * Requires N % 32 == 0, K % 8 == 0, lda/ldw % 8 == 0, 16-byte aligned
 * pointers.  fp32 accumulation on the tcgen05 tensor cores. */
/* The residual projection with the LayerNorm that follows it in the epilogue:
 * out_proj + residual + norm2 (torch_transformer_benchmark.py:1328-1348) or
 * ffn_out + residual + final_norm (1368-1373).  res [M, ld_res] fp32 holds the
 * residual on entry; v = res + A.W^T + bias (fp32 accumulation);
 * ln_out_f16 != 0: res = v (in place) and ln_out = LayerNorm(v)*gamma + beta
 * in fp16 (the next GEMM's operand); ln_out_f16 == 0: ln_out = LayerNorm(v)*
 * gamma + beta in fp32 and res is left unchanged.  One 128-column tile holds a
 * whole row: requires N == 128, K % 8 == 0, 16-byte aligned pointers and leading
 * dimensions.  ln_out must not overlap res. */
int b200_gemm_residual_layernorm_launch(const void* A, long long lda, const void* W, long long ldw, const float* bias,
                                        float* res, long long ld_res, const float* gamma, const float* beta, float eps,
                                        void* ln_out, long long ld_ln, int ln_out_f16, int M, int N, int K,
                                        b200_stream_t stream);

int b200_gemm_launch(int epilogue, const void* A, long long lda, const void* W, long long ldw, const float* bias,
                     const float* resid, long long ld_resid, void* out, long long ld_out, int M, int N, int K,
                     b200_stream_t stream);

/* Causal (or, with non_causal = 1, full) attention.  Q, K, V fp16 2-D tensors [rows, ld] holding head h of
 * sequence b at rows (row0 + b*seq_rows + position) and columns
 * (col0 + h*head_dim ...).  Query i of a sequence sits at absolute position
 * q_offset + i and attends keys 0..q_offset+i (prefix-causal).  Writes the
 * fp16 context [out_row0 + b*out_seq_rows + i, h*head_dim ...].
 * Keys are read in tiles: rows of the last tile past a sequence's kv_len but
 * below kv_rows are read too (with probability 0) and must hold finite values;
 * rows at or past kv_rows read as zeros. */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  long long ld_q, ld_k, ld_v;      /* row strides in elements (multiples of 8) */
  long long q_rows, kv_rows;       /* rows addressable through q and through k / v */
  int batch, heads, head_dim;
  int q_len, q_offset, kv_len;     /* q_offset + q_len <= kv_len */
  int q_seq_rows, kv_seq_rows;     /* rows between consecutive sequences */
  int q_row0, kv_row0;             /* row of (sequence 0, position 0) */
  int q_col0, k_col0, v_col0;      /* column of head 0 */
  void* out;
  long long ld_out;
  int out_seq_rows;
  int out_row0;
  int non_causal;        /* 0: causal (query i sees keys <= q_offset+i); 1: every valid key */
  const int* kv_lens;    /* device [batch]: keys to scan per sequence (one past the last valid key); NULL = kv_len */
  /* Key-padding masks that are not prefix-valid (see b200_mask_prepare): for a sequence b with
   * key_holes[b] != 0, key k is valid iff bit (k % 32) of key_bits[b * key_words + k / 32] is set.
   * key_words: a multiple of 4 (one 16-byte group per 128 keys), >= 4 * ceil(kv_len / 128);
   * key_bits 16-byte aligned.  NULL key_holes: every key below kv_lens / kv_len is valid. */
  const unsigned int* key_bits;
  int key_words;
  const int* key_holes;
} B200AttnArgs;

/* heads and batch at most 65535 each, and fewer than 2^31 query tiles of 128 rows in all
 * (ceil(q_len / 128) * heads * batch); larger launches return B200_ERR_TILE. */
int b200_flash_causal_launch(const B200AttnArgs* args, b200_stream_t stream);

/* One pre-LN causal block, the reference's per-layer body
 * (torch_transformer_benchmark.py:160-161), optionally followed by the final
 * LayerNorm (TTB:189): y = LN_f(x1 + W2.gelu(W1.LN2(x1)+b1)+b2),
 * x1 = x + Wo.attn(LN1(x)) + bo.  Weights fp16 (nn.Linear layout [out, in]),
 * biases and LayerNorm affine fp32.  lnf_w == NULL skips the final LayerNorm
 * (y is then the block output, for stacking layers). */
typedef struct {
  int batch, seq_len, d_model, num_heads, ffn_dim;
  const float* x;          /* [batch*seq_len, d_model] fp32 */
  float* y;                /* [batch*seq_len, d_model] fp32, may not alias x */
  const float* ln1_w;
  const float* ln1_b;
  const void* w_qkv;       /* [3*d_model, d_model] fp16: q rows, then k, then v */
  const float* b_qkv;      /* [3*d_model] */
  const void* w_o;         /* [d_model, d_model] fp16 */
  const float* b_o;
  const float* ln2_w;
  const float* ln2_b;
  const void* w_in;        /* [ffn_dim, d_model] fp16 */
  const float* b_in;
  const void* w_out;       /* [d_model, ffn_dim] fp16 */
  const float* b_out;
  const float* lnf_w;      /* final LayerNorm; NULL = none */
  const float* lnf_b;
  float eps;
  void* workspace;         /* >= b200_block_workspace_bytes(batch*seq_len, d_model, ffn_dim) */
  size_t workspace_bytes;
  int non_causal;          /* 0: causal block; 1: full attention (the reference without --causal) */
  const int* kv_lens;      /* device [batch] keys to scan per sequence (b200_mask_prepare), NULL = all */
  const unsigned int* key_bits;  /* key-padding masks with holes (b200_mask_prepare), NULL = none */
  int key_words;
  const int* key_holes;
} B200BlockArgs;

size_t b200_block_workspace_bytes(long long tokens, int d_model, int ffn_dim);
int b200_block_forward(const B200BlockArgs* args, b200_stream_t stream);

/* The same block, sequence-chunked for problems whose full activations do
 * not fit (the reference's _chunked_forward_causal,
 * torch_transformer_benchmark.py:1378-1609): per sequence, query chunks of
 * chunk_rows rows in order; each chunk appends its K/V rows to an fp16 cache
 * [batch*seq_len, 2*d_model] and attends keys [0, chunk end) prefix-causally.
 * workspace >= b200_block_chunked_workspace_bytes(batch*seq_len, chunk_rows,
 * d_model, ffn_dim) = the K/V cache plus one chunk's activations. */
size_t b200_block_chunked_workspace_bytes(long long tokens, int chunk_rows, int d_model, int ffn_dim);
int b200_block_forward_chunked(const B200BlockArgs* args, int chunk_rows, b200_stream_t stream);

/* Whole causal model (num_layers pre-LN blocks + final LayerNorm) in ONE
 * kernel, for small models: d_model == 128, num_heads 1, 2 or 4, ffn_dim a
 * multiple of 128 up to 512, seq_len <= 128 (tensor-core kernels: one
 * persistent CTA per sequence, or two CTAs per sequence for one layer and few
 * sequences), or d_model == 32, num_heads 1, 2 or 4, ffn_dim a multiple of 32
 * up to 128, seq_len <= 128 (a CUDA-core kernel, one CTA per sequence).  Every
 * intermediate stays on chip (TMEM / shared memory); per layer the weights are stacked
 * along rows: w_qkv [L*3d, d], w_o [L*d, d], w_in [L*ffn, d], w_out [L*d, ffn]
 * (fp16), biases / LayerNorm parameters [L, n] (fp32).  Every pointer must be
 * 16-byte aligned (the weights and vectors arrive by bulk copy), else
 * B200_ERR_ALIGN.  y must not alias x (y carries the residual between
 * layers).  Other shapes return B200_ERR_CONFIG. */
typedef struct {
  int batch, seq_len, d_model, num_heads, ffn_dim, num_layers;
  const float* x;
  float* y;
  const float* ln1_w;
  const float* ln1_b;
  const void* w_qkv;
  const float* b_qkv;
  const void* w_o;
  const float* b_o;
  const float* ln2_w;
  const float* ln2_b;
  const void* w_in;
  const float* b_in;
  const void* w_out;
  const float* b_out;
  const float* lnf_w;
  const float* lnf_b;
  float eps;
  const void* row_valid;   /* [batch*seq_len] uint8 key-padding mask (0 = padded row; prefix-valid per
                              sequence); padded keys are masked and padded rows of y written as 0.
                              NULL = no padding. */
  int non_causal;          /* 0: causal; 1: full attention */
} B200FusedSmallArgs;

int b200_block_fused_small_launch(const B200FusedSmallArgs* args, b200_stream_t stream);

/* Same computation as b200_block_forward, for callers that cannot allocate
 * device memory: a plugin host whose memory belongs to someone else's pool
 * and that hands out no workspace, a foreign-language caller with no CUDA
 * allocator of its own, or a latency-critical loop that cannot afford the
 * implicit device synchronisation of cudaMalloc/cudaFree.  It allocates
 * nothing: the intermediates live in one static device buffer of
 * B200_NOALLOC_SCRATCH_BYTES that the library defines, which every GPU that
 * loads the library holds until the process exits.  The caller still passes
 * x, y and the weights; args->workspace and args->workspace_bytes are ignored.
 *
 * Limit: b200_block_workspace_bytes(batch*seq_len, d_model, ffn_dim) must not
 * exceed B200_NOALLOC_SCRATCH_BYTES (e.g. up to 11915 tokens at d_model=128,
 * ffn_dim=512); larger problems return B200_ERR_NOALLOC_LIMIT before anything
 * is launched.
 * Set-up: the first call on a device (with that device current) looks up the
 * buffer's device address; make that first call before any stream capture.
 * The address is kept per device and CUDA context: after cudaDeviceReset (or
 * from another context on the same device) the next call looks it up again,
 * and that call, too, must come before any stream capture.
 * Sharing: every call on a device uses the same buffer, which keeps the last
 * call's contents (nothing in it needs to start at zero: every region is
 * written before it is read).  Calls whose work overlaps on the GPU (other
 * streams, other host threads) race on the buffer; serialise them.
 * No counterpart in the reference: its extensions allocate through PyTorch. */
#define B200_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)
int b200_block_forward_noalloc(const B200BlockArgs* args, b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_BLOCK_H */
