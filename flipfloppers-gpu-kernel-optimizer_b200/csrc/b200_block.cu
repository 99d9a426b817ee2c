// Host side of libb200block.so: argument checks, TMA tensor maps, tile
// selection, launches, and the per-layer chain b200_block_forward.
// The whole library is this one translation unit (kernel headers included
// below), built for sm_100a only.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "b200_block.h"
#include "ptx.cuh"
#include "ln.cuh"
#include "gemm.cuh"
#include "gemm2.cuh"
#include "attn.cuh"
#include "attn2.cuh"
#include "attn_small.cuh"
#include "fused_small.cuh"
#include "fused_tiny.cuh"

using namespace b200;

namespace {

// ------------------------------------------------------------------ runtime state
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
std::mutex g_mu;
std::set<std::pair<const void*, int>> g_attr_done;  // (kernel, device) with smem opt-in set
int g_arch_state[128] = {0};                          // per device: 0 unknown, 1 ok, -1 not sm_100

thread_local char g_detail[256] = "";

void set_detail(const char* what, cudaError_t e) {
  snprintf(g_detail, sizeof(g_detail), "%s: %s (%d)", what, cudaGetErrorString(e), static_cast<int>(e));
}

int ensure_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    else
      cudaGetLastError();
  });
  return g_encode ? B200_OK : B200_ERR_TMAP;
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int check_arch() {
  const int dev = current_device();
  if (dev < 0 || dev >= 128) return B200_ERR_ARCH;
  int st;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    st = g_arch_state[dev];
  }
  if (st == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    st = (major == 10 && minor == 0) ? 1 : -1;
    std::lock_guard<std::mutex> lk(g_mu);
    g_arch_state[dev] = st;
  }
  return st == 1 ? B200_OK : B200_ERR_ARCH;
}

int set_smem(const void* fn, int bytes) {
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_attr_done.count({fn, dev})) return B200_OK;
  const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_detail("cudaFuncSetAttribute(MaxDynamicSharedMemorySize)", e);
    return B200_ERR_SMEM;
  }
  g_attr_done.insert({fn, dev});
  return B200_OK;
}

int num_sms() {
  int dev = current_device(), n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return B200_OK;
  set_detail("kernel launch", e);
  return B200_ERR_LAUNCH;
}

// Programmatic dependent launch: a kernel may start its prologue while the
// previous kernel of the stream finishes (each kernel waits for it in
// griddep_sync before touching global data).  B200_PDL=0 launches with plain
// stream order instead.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("B200_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

// (errors are left for the caller's launch_status(), like a <<<>>> launch);
// cluster_x > 1: thread-block clusters of cluster_x CTAs along x
template <typename... Params, typename... Args>
void launch_kernel_cluster(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                           unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
template <typename... Params, typename... Args>
void launch_kernel(void (*kern)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  launch_kernel_cluster(kern, grid, block, smem, st, 1u, std::forward<Args>(args)...);
}

// Refuse a launch the kernel's compiled resources cannot satisfy, with the reason recorded.
int check_block_fits(const void* fn, int threads) {
  cudaFuncAttributes fa{};
  const cudaError_t e = cudaFuncGetAttributes(&fa, fn);
  if (e != cudaSuccess) {
    set_detail("cudaFuncGetAttributes", e);
    return B200_ERR_LAUNCH;
  }
  if (fa.maxThreadsPerBlock < threads) {
    snprintf(g_detail, sizeof(g_detail), "kernel allows %d threads per block (%d registers/thread), %d requested",
             fa.maxThreadsPerBlock, fa.numRegs, threads);
    return B200_ERR_CONFIG;
  }
  return B200_OK;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 2-D fp16 tensor [rows, cols] with row stride ld (elements); box box_rows x box_cols.
int make_map_f16(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle sw) {
  if (ensure_encode() != B200_OK) return B200_ERR_TMAP;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_TMAP;
}

// [rows, cols] row-major matrix (leading dimension ld elements) as a 2-D map
// with boxes of box_cols x box_rows.
int make_map_2d(CUtensorMap* m, CUtensorMapDataType dt, uint32_t esize, const void* base, uint64_t rows,
                uint64_t cols, uint64_t ld, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle sw) {
  if (ensure_encode() != B200_OK) return B200_ERR_TMAP;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * esize};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_TMAP;
}

// [num_seq, seq_len, cols] fp32 activations as a 3-D map with SWIZZLE_128B
// boxes of 32 columns x box_rows rows x 1 sequence: rows past seq_len are
// zero-filled on load and not written on store, so a box never reaches into
// the next sequence.
int make_map_f32_seq(CUtensorMap* m, const void* base, uint64_t num_seq, uint64_t seq_len, uint64_t cols,
                     uint32_t box_rows) {
  if (ensure_encode() != B200_OK) return B200_ERR_TMAP;
  cuuint64_t dims[3] = {cols, seq_len, num_seq};
  cuuint64_t strides[2] = {cols * 4, seq_len * cols * 4};
  cuuint32_t box[3] = {32, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_TMAP;
}

// ------------------------------------------------------------------ GEMM
template <int BN, int STAGES, int EPI>
int launch_gemm_t(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const GemmParams& p,
                  cudaStream_t st, const CUtensorMap* tn = nullptr) {
  auto kern = k_gemm_tn<BN, STAGES, EPI>;
  const int smem = GemmSmem<BN, STAGES, EPI>::TOTAL;
  if (int rc = set_smem(reinterpret_cast<const void*>(kern), smem)) return rc;
  const long long tiles = static_cast<long long>((p.M + 127) / 128) * ((p.N + BN - 1) / BN);
  const int grid = static_cast<int>(tiles < num_sms() ? tiles : num_sms());
  launch_kernel(kern, dim3(grid), dim3(GEMM_THREADS), smem, st, ta, tw, to, tn ? *tn : to, p);
  return launch_status();
}

template <int BN, int STAGES>
int launch_gemm_bn(int epi, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const GemmParams& p,
                   cudaStream_t st) {
  switch (epi) {
    case EPI_BIAS_F16: return launch_gemm_t<BN, STAGES, EPI_BIAS_F16>(ta, tw, to, p, st);
    case EPI_BIAS_GELU_F16: return launch_gemm_t<BN, STAGES, EPI_BIAS_GELU_F16>(ta, tw, to, p, st);
    case EPI_BIAS_RESID_F32: return launch_gemm_t<BN, STAGES, EPI_BIAS_RESID_F32>(ta, tw, to, p, st);
    case EPI_BIAS_F32: return launch_gemm_t<BN, STAGES, EPI_BIAS_F32>(ta, tw, to, p, st);
    default: return B200_ERR_CONFIG;
  }
}

// 128x256 tiles keep 192 KB of operands in flight (4 stages), enough to cover
// the L2 round trip at full MMA rate; 128x128 tiles (6 x 32 KB) are not, so
// they are used only when N is not a multiple of 256.
int pick_bn(long long M, int N) {
  (void)M;
  return N % 256 == 0 ? 256 : 128;
}

// CTA-pair kernel: clusters that can be resident at once (queried once per device
// and epilogue-warp count)
int g_pair_clusters[2][128] = {{0}};

template <int EPI, int EW>
int launch_gemm2_t(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const GemmParams& p,
                   cudaStream_t st) {
  auto kern = k_gemm2_tn<EPI, EW>;
  const int smem = Gemm2Smem<gemm2_stages(EW), EW>::TOTAL;
  const int threads = gemm2_threads(EW);
  if (int rc = set_smem(reinterpret_cast<const void*>(kern), smem)) return rc;
  const int dev = current_device();
  int* cache = g_pair_clusters[EW == 16 ? 1 : 0];
  int maxcl = (dev >= 0 && dev < 128) ? cache[dev] : 0;
  if (maxcl <= 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(num_sms()));
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(kern), &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    maxcl = n;
    if (dev >= 0 && dev < 128) cache[dev] = n;
  }
  const long long tiles = static_cast<long long>((p.M + 255) / 256) * ((p.N + 255) / 256);
  const int clusters = static_cast<int>(tiles < maxcl ? tiles : maxcl);
  launch_kernel(kern, dim3(2 * clusters), dim3(threads), smem, st, ta, tw, to, p);
  return launch_status();
}

// Epilogue warps of the pair kernel: 16 when K is short (<= 256: at most four
// 64-wide K slices per tile, so the epilogue sets the speed), else 8.
template <int EPI>
int launch_gemm2_k(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const GemmParams& p,
                   cudaStream_t st) {
  if (p.K <= 256) return launch_gemm2_t<EPI, 16>(ta, tw, to, p, st);
  return launch_gemm2_t<EPI, 8>(ta, tw, to, p, st);
}

// 0: one-SM kernel, 1: CTA-pair kernel, -1 (default): by shape
int gemm_pair_mode() {
  static const int mode = [] {
    const char* e = std::getenv("B200_GEMM_PAIR");
    return e ? std::atoi(e) : -1;
  }();
  return mode;
}

// Measured on B200 (N-fastest tile order, L2 flushed): the pair kernel is
// ahead wherever whole 256-column tiles exist and both CTAs get rows, e.g.
// 100000x3072x1024 434 vs 480 us, 16384x4096x4096 338 vs 365 us, 8192x1024x4096
// (+residual) 60 vs 67 us; the one-SM kernel keeps N not a multiple of 256
// (QKV at d=128: N=384) and short M.
bool use_pair_gemm(long long M, int N, int K) {
  (void)K;
  const int mode = gemm_pair_mode();
  if (mode >= 0) return mode == 1 && M >= 256 && N >= 256;
  return N % 256 == 0 && M >= 512;
}

int gemm_impl(int epi, const void* A, long long lda, const void* W, long long ldw, const float* bias,
              const float* resid, long long ld_resid, void* out, long long ld_out, int M, int N, int K,
              cudaStream_t st) {
  if (!A || !W || !out || M < 0 || N <= 0 || K <= 0) return B200_ERR_ARG;
  if (epi < 0 || epi > 3) return B200_ERR_CONFIG;
  if (epi == EPI_BIAS_RESID_F32 && !resid) return B200_ERR_ARG;
  if (M == 0) return B200_OK;
  if (N % 32 || K % 8 || lda % 8 || ldw % 8 || lda < K || ldw < K) return B200_ERR_TILE;
  const bool f32_out = epi == EPI_BIAS_RESID_F32 || epi == EPI_BIAS_F32;
  if (ld_out < N || ld_out % (f32_out ? 4 : 8)) return B200_ERR_ALIGN;
  if (!al16(A) || !al16(W) || !al16(out) || (bias && !al16(bias))) return B200_ERR_ALIGN;
  if (epi == EPI_BIAS_RESID_F32 && (!al16(resid) || ld_resid % 4 || ld_resid < N)) return B200_ERR_ALIGN;
  if (int rc = check_arch()) return rc;
  const int BN = pick_bn(M, N);
  CUtensorMap ta, tw;
  if (int rc = make_map_f16(&ta, A, M, K, lda, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  if (int rc = make_map_f16(&tw, W, N, K, ldw, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  // the epilogue writes 64-byte rows of 32-row boxes (SWIZZLE_64B): 32 fp16 or 16 fp32 columns
  CUtensorMap to;
  if (f32_out) {
    if (int rc = make_map_2d(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, out, M, N, ld_out, 16, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return rc;
  } else {
    if (int rc = make_map_2d(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, out, M, N, ld_out, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
      return rc;
  }
  // the residual epilogue adds onto `out` in place (TMA add-reduce); a distinct
  // residual is copied into `out` first
  if (epi == EPI_BIAS_RESID_F32 && (resid != out || ld_resid != ld_out)) {
    const cudaError_t e = cudaMemcpy2DAsync(out, static_cast<size_t>(ld_out) * 4, resid, static_cast<size_t>(ld_resid) * 4,
                                            static_cast<size_t>(N) * 4, static_cast<size_t>(M), cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return B200_ERR_LAUNCH;
    }
  }
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_row0 = 0;
  p.bias = bias;
  if (use_pair_gemm(M, N, K)) {
    CUtensorMap tw2;  // each CTA of the pair loads 128 rows (half the tile's N range) of W
    if (int rc = make_map_f16(&tw2, W, N, K, ldw, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    switch (epi) {
      case EPI_BIAS_F16: return launch_gemm2_k<EPI_BIAS_F16>(ta, tw2, to, p, st);
      case EPI_BIAS_GELU_F16: return launch_gemm2_k<EPI_BIAS_GELU_F16>(ta, tw2, to, p, st);
      case EPI_BIAS_RESID_F32: return launch_gemm2_k<EPI_BIAS_RESID_F32>(ta, tw2, to, p, st);
      default: return launch_gemm2_k<EPI_BIAS_F32>(ta, tw2, to, p, st);
    }
  }
  if (BN == 256) return launch_gemm_bn<256, 4>(epi, ta, tw, to, p, st);
  return launch_gemm_bn<128, 6>(epi, ta, tw, to, p, st);
}

// The chain fuses the residual projections with the following LayerNorm when a
// 128-column tile holds the whole row (d == 128); B200_GEMM_LN=0 keeps the
// separate LayerNorm kernel (A/B comparisons).
bool fuse_ln(int d) {
  static const bool on = [] {
    const char* e = std::getenv("B200_GEMM_LN");
    return e == nullptr || e[0] != '0';
  }();
  return on && d == 128;
}

// out_proj / ffn_out with the residual add and the following LayerNorm in the
// epilogue (one 128-column tile holds a whole row, so N must be 128):
//   res[M,N] holds the residual on entry;  v = res + A.W^T + bias;
//   ln_f16:  res = v (x1, in place) and ln_out = LN(v)*gamma + beta in fp16;
//   !ln_f16: ln_out = LN(v)*gamma + beta in fp32 (res is left unchanged).
int gemm_ln_impl(const void* A, long long lda, const void* W, long long ldw, const float* bias, float* res,
                 long long ld_res, const float* gamma, const float* beta, float eps, void* ln_out, long long ld_ln,
                 int ln_f16, int M, int N, int K, cudaStream_t st) {
  if (!A || !W || !res || !gamma || !beta || !ln_out || M < 0 || K <= 0) return B200_ERR_ARG;
  if (M == 0) return B200_OK;
  if (N != 128) return B200_ERR_CONFIG;
  if (K % 8 || lda % 8 || ldw % 8 || lda < K || ldw < K) return B200_ERR_TILE;
  if (ld_res < N || ld_res % 4 || ld_ln < N || ld_ln % (ln_f16 ? 8 : 4)) return B200_ERR_ALIGN;
  if (!al16(A) || !al16(W) || !al16(res) || !al16(ln_out) || !al16(gamma) || !al16(beta) || (bias && !al16(bias)))
    return B200_ERR_ALIGN;
  if (int rc = check_arch()) return rc;
  CUtensorMap ta, tw, tx, tn;
  if (int rc = make_map_f16(&ta, A, M, K, lda, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  if (int rc = make_map_f16(&tw, W, N, K, ldw, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  if (int rc = make_map_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, res, M, N, ld_res, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (ln_f16) {
    if (int rc = make_map_2d(&tn, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ln_out, M, N, ld_ln, 64, 32,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  } else {
    if (int rc = make_map_2d(&tn, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ln_out, M, N, ld_ln, 32, 32,
                             CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  }
  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.a_row0 = 0;
  p.bias = bias;
  p.gamma = gamma;
  p.beta = beta;
  p.eps = eps;
  if (ln_f16) return launch_gemm_t<128, 3, EPI_BIAS_RESID_LN16>(ta, tw, tx, p, st, &tn);
  return launch_gemm_t<128, 3, EPI_BIAS_RESID_LN32>(ta, tw, tx, p, st, &tn);
}

// ------------------------------------------------------------------ LayerNorm
template <int VPL, bool VEC4>
int launch_ln_t(const float* x, long long ldx, const float* g, const float* b, void* out, long long ldo, bool f16,
                int rows, int d, float eps, float* copy, long long ldc, cudaStream_t st) {
  const int warps = 8;
  dim3 grid((rows + warps - 1) / warps);
  if (f16)
    launch_kernel(k_layernorm<VPL, VEC4, true>, dim3(grid), dim3(32 * warps), 0, st, x, ldx, g, b, out, ldo, rows, d,
                  eps, copy, ldc);
  else
    launch_kernel(k_layernorm<VPL, VEC4, false>, dim3(grid), dim3(32 * warps), 0, st, x, ldx, g, b, out, ldo, rows, d,
                  eps, copy, ldc);
  return launch_status();
}

// copy (may be null): fp32 copy of x's rows, leading dimension ldc
int ln_impl(const float* x, long long ldx, const float* g, const float* b, void* out, long long ldo, int f16,
            int rows, int d, float eps, cudaStream_t st, float* copy = nullptr, long long ldc = 0) {
  if (!x || !g || !b || !out || rows < 0 || d <= 0) return B200_ERR_ARG;
  if (rows == 0) return B200_OK;
  if (d % 32 || d > 4096 || ldx < d || ldo < d || (copy && ldc < d)) return B200_ERR_TILE;
  if (int rc = check_arch()) return rc;
  if (d % 128 == 0 && ldx % 4 == 0 && ldo % 4 == 0 && al16(x) && al16(out) && al16(g) && al16(b) &&
      (!copy || (ldc % 4 == 0 && al16(copy)))) {
    switch (d / 128) {
      case 1: return launch_ln_t<1, true>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
      case 2: return launch_ln_t<2, true>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
      case 4: return launch_ln_t<4, true>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
      case 8: return launch_ln_t<8, true>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
      case 16: return launch_ln_t<16, true>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
      case 32: return launch_ln_t<32, true>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
      default: break;
    }
  }
  switch (d / 32) {
    case 1: return launch_ln_t<1, false>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
    case 2: return launch_ln_t<2, false>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
    case 3: return launch_ln_t<3, false>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
    case 4: return launch_ln_t<4, false>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
    case 6: return launch_ln_t<6, false>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
    case 8: return launch_ln_t<8, false>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
    case 12: return launch_ln_t<12, false>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
    case 16: return launch_ln_t<16, false>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
    case 24: return launch_ln_t<24, false>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
    case 32: return launch_ln_t<32, false>(x, ldx, g, b, out, ldo, f16, rows, d, eps, copy, ldc, st);
    default: return B200_ERR_TILE;
  }
}

template <int VPL>
int launch_add_ln_t(const float* a, const float* b, const float* bias, float* sum_out, const float* g,
                    const float* be, void* out, bool f16, int rows, int d, float eps, cudaStream_t st) {
  dim3 grid((rows + 7) / 8);
  if (f16)
    launch_kernel(k_add_layernorm<VPL, true>, dim3(grid), dim3(256), 0, st, a, b, bias, sum_out, g, be, out, rows, d,
                  eps);
  else
    launch_kernel(k_add_layernorm<VPL, false>, dim3(grid), dim3(256), 0, st, a, b, bias, sum_out, g, be, out, rows, d,
                  eps);
  return launch_status();
}

int add_ln_impl(const float* a, const float* b, const float* bias, float* sum_out, const float* g, const float* be,
                void* out, int f16, int rows, int d, float eps, cudaStream_t st) {
  if (!a || !b || !sum_out || !g || !be || !out || rows < 0 || d <= 0) return B200_ERR_ARG;
  if (rows == 0) return B200_OK;
  if (d % 128 || d > 4096) return B200_ERR_TILE;
  if (!al16(a) || !al16(b) || !al16(sum_out) || !al16(g) || !al16(be) || !al16(out) || (bias && !al16(bias)))
    return B200_ERR_ALIGN;
  if (int rc = check_arch()) return rc;
  switch (d / 128) {
    case 1: return launch_add_ln_t<1>(a, b, bias, sum_out, g, be, out, f16, rows, d, eps, st);
    case 2: return launch_add_ln_t<2>(a, b, bias, sum_out, g, be, out, f16, rows, d, eps, st);
    case 4: return launch_add_ln_t<4>(a, b, bias, sum_out, g, be, out, f16, rows, d, eps, st);
    case 8: return launch_add_ln_t<8>(a, b, bias, sum_out, g, be, out, f16, rows, d, eps, st);
    case 16: return launch_add_ln_t<16>(a, b, bias, sum_out, g, be, out, f16, rows, d, eps, st);
    case 32: return launch_add_ln_t<32>(a, b, bias, sum_out, g, be, out, f16, rows, d, eps, st);
    default: return B200_ERR_TILE;
  }
}

// ------------------------------------------------------------------ attention
// Kernel parameters of one launch (every attention kernel takes the same ones)
template <int HD>
AttnParams attn_params(const B200AttnArgs& a) {
  AttnParams p{};
  p.H = a.heads;
  p.batch = a.batch;
  p.q_len = a.q_len;
  p.q_offset = a.q_offset;
  p.kv_len = a.kv_len;
  p.q_seq_rows = a.q_seq_rows;
  p.kv_seq_rows = a.kv_seq_rows;
  p.q_row0 = a.q_row0;
  p.kv_row0 = a.kv_row0;
  p.q_col0 = a.q_col0;
  p.k_col0 = a.k_col0;
  p.v_col0 = a.v_col0;
  p.out = static_cast<__half*>(a.out) + static_cast<int64_t>(a.out_row0) * a.ld_out;
  p.ld_out = a.ld_out;
  p.out_seq_rows = a.out_seq_rows;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / __builtin_sqrt(static_cast<double>(HD)));
  p.non_causal = a.non_causal;
  p.kv_lens = a.kv_lens;
  p.key_bits = reinterpret_cast<const uint32_t*>(a.key_bits);
  p.key_words = a.key_words;
  p.key_holes = a.key_holes;
  return p;
}

template <int HD, int BN>
int launch_attn_t(const B200AttnArgs& a, cudaStream_t st) {
  using C = AttnCfg<HD, BN>;
  constexpr CUtensorMapSwizzle SW = C::ATOM_E == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUtensorMap tq, tk, tv;
  if (int rc = make_map_f16(&tq, a.q, a.q_rows, a.ld_q, a.ld_q, C::ATOM_E, 128, SW)) return rc;
  if (int rc = make_map_f16(&tk, a.k, a.kv_rows, a.ld_k, a.ld_k, C::ATOM_E, BN, SW)) return rc;
  if (int rc = make_map_f16(&tv, a.v, a.kv_rows, a.ld_v, a.ld_v, C::ATOM_E, BN, SW)) return rc;
  const AttnParams p = attn_params<HD>(a);
  // TMEM: at most two 256-column CTAs per SM, so request enough shared memory
  // that a third cannot be co-resident and block in tcgen05.alloc.
  int smem = C::TOTAL;
  if (C::TMEM_COLS == 256 && smem < 80 * 1024) smem = 80 * 1024;
  auto kern = k_flash_causal<HD, BN>;
  if (int rc = set_smem(reinterpret_cast<const void*>(kern), smem)) return rc;
  // persistent: as many CTAs as can be resident (two per SM when two fit in
  // shared memory), each walking its share of the (query tile, head, sequence) items
  const long long items = static_cast<long long>((a.q_len + 127) / 128) * a.heads * a.batch;
  if (items > 0x7fffffffLL) return B200_ERR_TILE;  // the kernel numbers its items in 32 bits
  const long long per_sm = 2LL * smem + 2048 <= 228LL * 1024 ? 2 : 1;
  const long long ctas = std::min(items, per_sm * num_sms());
  launch_kernel(kern, dim3(static_cast<unsigned>(ctas)), dim3(192), smem, st, tq, tk, tv, p);
  return launch_status();
}

// head_dim 8 / 16: CUDA-core kernel (attn_small.cuh), no tensor maps
template <int HD>
int launch_attn_small_t(const B200AttnArgs& a, cudaStream_t st) {
  const AttnParams p = attn_params<HD>(a);
  dim3 grid((a.q_len + ATTN_SMALL_ROWS - 1) / ATTN_SMALL_ROWS, a.heads, a.batch);
  launch_kernel(k_attn_small<HD>, dim3(grid), dim3(ATTN_SMALL_ROWS), 0, st, static_cast<const __half*>(a.q), a.ld_q,
                static_cast<const __half*>(a.k), a.ld_k, static_cast<const __half*>(a.v), a.ld_v, p);
  return launch_status();
}

template <int HD>
int launch_attn2_t(const B200AttnArgs& a, cudaStream_t st) {
  using C = Attn2Cfg<HD>;
  constexpr CUtensorMapSwizzle SW = HD == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUtensorMap tq, tk, tv;
  if (int rc = make_map_f16(&tq, a.q, a.q_rows, a.ld_q, a.ld_q, HD, 128, SW)) return rc;
  if (int rc = make_map_f16(&tk, a.k, a.kv_rows, a.ld_k, a.ld_k, HD, C::BN, SW)) return rc;
  if (int rc = make_map_f16(&tv, a.v, a.kv_rows, a.ld_v, a.ld_v, HD, C::BN, SW)) return rc;
  const AttnParams p = attn_params<HD>(a);
  auto kern = k_flash_causal2<HD>;
  const int smem = C::TOTAL;
  if (int rc = set_smem(reinterpret_cast<const void*>(kern), smem)) return rc;
  dim3 grid((a.q_len + 255) / 256, a.heads, a.batch);
  launch_kernel(kern, dim3(grid), dim3(320), smem, st, tq, tk, tv, p);
  return launch_status();
}

// B200_ATTN_TILES=1 / =2 forces the one- / two-query-tile kernel (head_dim 32
// and 64) for every shape (A/B comparisons); unset: by shape (attn_impl).
constexpr int ATTN_TWO_TILE_MIN_Q_HD64 = 2048;
constexpr int ATTN_TWO_TILE_MIN_WAVES = 16;

int attn_tiles_forced() {
  static const int forced = [] {
    const char* e = getenv("B200_ATTN_TILES");
    return (e != nullptr && (e[0] == '1' || e[0] == '2')) ? e[0] - '0' : 0;
  }();
  return forced;
}

int attn_impl(const B200AttnArgs* a, cudaStream_t st) {
  if (!a || !a->q || !a->k || !a->v || !a->out) return B200_ERR_ARG;
  if (a->batch <= 0 || a->heads <= 0 || a->q_len < 0 || a->q_offset < 0 || a->kv_len <= 0) return B200_ERR_ARG;
  if (a->q_len == 0) return B200_OK;
  if (a->q_offset + a->q_len > a->kv_len) return B200_ERR_ARG;
  const int hd = a->head_dim;
  if (hd != 8 && hd != 16 && hd != 32 && hd != 64 && hd != 128 && hd != 256) return B200_ERR_HEAD_DIM;
  if (a->ld_q % 8 || a->ld_k % 8 || a->ld_v % 8 || a->ld_out % 8) return B200_ERR_ALIGN;
  if (!al16(a->q) || !al16(a->k) || !al16(a->v) || !al16(a->out)) return B200_ERR_ALIGN;
  if (a->q_col0 % 8 || a->k_col0 % 8 || a->v_col0 % 8) return B200_ERR_ALIGN;
  const long long span = static_cast<long long>(a->heads) * hd;
  if (a->q_col0 + span > a->ld_q || a->k_col0 + span > a->ld_k || a->v_col0 + span > a->ld_v || span > a->ld_out)
    return B200_ERR_ARG;
  if (static_cast<long long>(a->q_row0) + static_cast<long long>(a->batch - 1) * a->q_seq_rows + a->q_len > a->q_rows)
    return B200_ERR_ARG;
  if (static_cast<long long>(a->kv_row0) + static_cast<long long>(a->batch - 1) * a->kv_seq_rows + a->kv_len >
      a->kv_rows)
    return B200_ERR_ARG;
  if (a->heads > 65535 || a->batch > 65535) return B200_ERR_TILE;
  if ((a->key_holes == nullptr) != (a->key_bits == nullptr)) return B200_ERR_ARG;
  if (a->key_bits != nullptr) {
    if (a->key_words % 4 || a->key_words < 4 * ((a->kv_len + 127) / 128)) return B200_ERR_ARG;
    if (!al16(a->key_bits)) return B200_ERR_ALIGN;
  }
  if (int rc = check_arch()) return rc;
  // Two query tiles per CTA (k_flash_causal2: shared K/V loads, one tile's MMA
  // under the other's softmax, alternating exp phases; one CTA per pair of
  // tiles) against the persistent one-tile kernel (two CTAs per SM walking all
  // items), measured (L2 flushed, B*S = 64K or 128K tokens):
  //   head_dim 32, H=4: one tile at every length, S=512..16384 (S=1024 79.7 vs
  //     100.5 us, S=16384 737 vs 830 us);
  //   head_dim 64, H=16: one tile to S=1024 (330 vs 365 us), two from S=2048
  //     (S=2048 543 vs 560, S=16384 3069 vs 3437 us: 27.7 waves of pairs);
  //   head_dim 64, H=2: one tile at every length (S=2048 141 vs 158, S=16384 776
  //     vs 855 us: 6.9 waves of pairs, whose tail the persistent kernel avoids).
  // So two tiles for head_dim 64 from S=2048 when the pairs fill >= 16 waves.
  if (hd == 8) return launch_attn_small_t<8>(*a, st);
  if (hd == 16) return launch_attn_small_t<16>(*a, st);
  const int forced = attn_tiles_forced();
  if (forced == 2 && hd == 32) return launch_attn2_t<32>(*a, st);
  if (hd == 64) {
    const long long pairs = static_cast<long long>((a->q_len + 255) / 256) * a->heads * a->batch;
    const bool two = forced == 2 || (forced == 0 && a->q_len >= ATTN_TWO_TILE_MIN_Q_HD64 &&
                                      pairs >= static_cast<long long>(ATTN_TWO_TILE_MIN_WAVES) * num_sms());
    if (two) return launch_attn2_t<64>(*a, st);
  }
  switch (hd) {
    case 32: return launch_attn_t<32, 128>(*a, st);
    case 64: return launch_attn_t<64, 128>(*a, st);
    case 128: return launch_attn_t<128, 128>(*a, st);
    case 256: return launch_attn_t<256, 64>(*a, st);
    default: return B200_ERR_HEAD_DIM;
  }
}

// ------------------------------------------------------------------ fused small-model kernel
// 0: one CTA per sequence, 1: the row-split kernel whenever it applies (one
// layer), -1 (default): row split when every sequence's two CTAs fit on the
// device at once
int small_rows_mode() {
  static const int mode = [] {
    const char* e = std::getenv("B200_SMALL_ROWS");
    return e ? std::atoi(e) : -1;
  }();
  return mode;
}

// B200_TINY_SPLIT=0|1 forces one CTA per sequence / a two-CTA cluster per sequence
// for d_model = 32 (default: the cluster when the sequences leave SMs idle)
int tiny_split_mode() {
  static const int mode = [] {
    const char* e = std::getenv("B200_TINY_SPLIT");
    return e ? std::atoi(e) : -1;
  }();
  return mode;
}

// d_model = 32: the CUDA-core kernel of fused_tiny.cuh (head_dim 8 / 16 / 32)
int fused_tiny_impl(const B200FusedSmallArgs* a, cudaStream_t st) {
  const int H = a->num_heads;
  if (H != 1 && H != 2 && H != 4) return B200_ERR_CONFIG;
  if (a->ffn_dim <= 0 || a->ffn_dim % 32 || a->ffn_dim > TinyCfg::FMAX || a->seq_len > TinyCfg::S)
    return B200_ERR_CONFIG;
  if (a->batch > 0x7fffffff / TinyCfg::S) return B200_ERR_TILE;
  TinyParams p{};
  p.num_seq = a->batch;
  p.seq_len = a->seq_len;
  p.layers = a->num_layers;
  p.heads = H;
  p.ffn = a->ffn_dim;
  p.x = a->x;
  p.y = a->y;
  p.ln1_w = a->ln1_w;
  p.ln1_b = a->ln1_b;
  p.w_qkv = static_cast<const __half*>(a->w_qkv);
  p.b_qkv = a->b_qkv;
  p.w_o = static_cast<const __half*>(a->w_o);
  p.b_o = a->b_o;
  p.ln2_w = a->ln2_w;
  p.ln2_b = a->ln2_b;
  p.w_in = static_cast<const __half*>(a->w_in);
  p.b_in = a->b_in;
  p.w_out = static_cast<const __half*>(a->w_out);
  p.b_out = a->b_out;
  p.lnf_w = a->lnf_w;
  p.lnf_b = a->lnf_b;
  p.eps = a->eps;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / __builtin_sqrt(static_cast<double>(32 / H)));
  p.row_valid = static_cast<const unsigned char*>(a->row_valid);
  p.non_causal = a->non_causal;
  const int split_mode = tiny_split_mode();
  const bool split = split_mode != 0 && (split_mode == 1 || 2LL * a->batch <= num_sms()) && a->batch <= 0x3fffffff;
  auto launch = [&](auto kern, auto cfg) {
    using Cfg = decltype(cfg);
    if (int rc = set_smem(reinterpret_cast<const void*>(kern), Cfg::TOTAL)) return rc;
    if (int rc = check_block_fits(reinterpret_cast<const void*>(kern), Cfg::THREADS)) return rc;
    const unsigned cl = Cfg::RL < Cfg::S ? 2u : 1u;
    launch_kernel_cluster(kern, dim3(a->batch * cl), dim3(Cfg::THREADS), Cfg::TOTAL, st, cl, p);
    return launch_status();
  };
  if (split) {
    if (H == 4) return launch(k_block_tiny<8, true>, TinyCfgT<true>{});
    if (H == 2) return launch(k_block_tiny<16, true>, TinyCfgT<true>{});
    return launch(k_block_tiny<32, true>, TinyCfgT<true>{});
  }
  if (H == 4) return launch(k_block_tiny<8, false>, TinyCfg{});
  if (H == 2) return launch(k_block_tiny<16, false>, TinyCfg{});
  return launch(k_block_tiny<32, false>, TinyCfg{});
}

int fused_small_impl(const B200FusedSmallArgs* a, cudaStream_t st) {
  if (!a || !a->x || !a->y || !a->w_qkv || !a->w_o || !a->w_in || !a->w_out) return B200_ERR_ARG;
  if (!a->ln1_w || !a->ln1_b || !a->ln2_w || !a->ln2_b || !a->lnf_w || !a->lnf_b || !a->b_qkv || !a->b_o ||
      !a->b_in || !a->b_out)
    return B200_ERR_ARG;
  if (a->batch <= 0 || a->seq_len <= 0 || a->num_layers <= 0) return B200_ERR_ARG;
  // every per-layer vector arrives by bulk copy (16-byte aligned source)
  const float* vecs[] = {a->ln1_w, a->ln1_b, a->ln2_w, a->ln2_b, a->lnf_w, a->lnf_b, a->b_qkv, a->b_o, a->b_in, a->b_out};
  if (a->d_model == 32) {
    if (a->x == a->y) return B200_ERR_ARG;
    if (!al16(a->x) || !al16(a->y) || !al16(a->w_qkv) || !al16(a->w_o) || !al16(a->w_in) || !al16(a->w_out))
      return B200_ERR_ALIGN;
    for (const float* v : vecs)
      if (!al16(v)) return B200_ERR_ALIGN;
    if (int rc = check_arch()) return rc;
    return fused_tiny_impl(a, st);
  }
  if (a->d_model != 128 || (a->num_heads != 1 && a->num_heads != 2 && a->num_heads != 4) || a->ffn_dim <= 0 ||
      a->ffn_dim % 128 || a->ffn_dim > 512 || a->seq_len > 128)
    return B200_ERR_CONFIG;
  if (a->x == a->y) return B200_ERR_ARG;
  if (!al16(a->x) || !al16(a->y) || !al16(a->w_qkv) || !al16(a->w_o) || !al16(a->w_in) || !al16(a->w_out))
    return B200_ERR_ALIGN;
  for (const float* v : vecs)
    if (!al16(v)) return B200_ERR_ALIGN;
  if (static_cast<long long>(a->batch) * a->seq_len > 0x7fffffffLL) return B200_ERR_TILE;
  if (int rc = check_arch()) return rc;
  const int L = a->num_layers, F = a->ffn_dim;
  CUtensorMap tq, to, ti, tout;
  if (int rc = make_map_f16(&tq, a->w_qkv, static_cast<uint64_t>(L) * 384, 128, 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  if (int rc = make_map_f16(&to, a->w_o, static_cast<uint64_t>(L) * 128, 128, 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  if (int rc = make_map_f16(&ti, a->w_in, static_cast<uint64_t>(L) * F, 128, 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  if (int rc = make_map_f16(&tout, a->w_out, static_cast<uint64_t>(L) * 128, F, F, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
  CUtensorMap tx, ty;
  if (int rc = make_map_f32_seq(&tx, a->x, a->batch, a->seq_len, 128, 128)) return rc;
  if (int rc = make_map_f32_seq(&ty, a->y, a->batch, a->seq_len, 128, 32)) return rc;
  SmallParams p{};
  p.num_seq = a->batch;
  p.seq_len = a->seq_len;
  p.layers = L;
  p.ffn = F;
  p.x = a->x;
  p.y = a->y;
  p.ln1_w = a->ln1_w;
  p.ln1_b = a->ln1_b;
  p.b_qkv = a->b_qkv;
  p.b_o = a->b_o;
  p.ln2_w = a->ln2_w;
  p.ln2_b = a->ln2_b;
  p.b_in = a->b_in;
  p.b_out = a->b_out;
  p.lnf_w = a->lnf_w;
  p.lnf_b = a->lnf_b;
  p.eps = a->eps;
  p.heads = a->num_heads;
  p.scale_log2 = static_cast<float>(1.4426950408889634 / __builtin_sqrt(128.0 / a->num_heads));
  p.row_valid = static_cast<const unsigned char*>(a->row_valid);
  p.non_causal = a->non_causal;
  const int smem = SmallCfg::TOTAL;
  // Two CTAs per sequence (each finishing half of the query rows) halve the
  // latency-bound per-row phases while the batch leaves SMs idle (measured
  // at C2: see DESIGN); one layer only, as each CTA rebuilds K/V from x.
  const int rows_mode = small_rows_mode();
  const bool rows = L == 1 && rows_mode != 0 && (rows_mode == 1 || 2LL * a->batch <= num_sms()) &&
                    a->batch <= 0x3fffffff;
  CUtensorMap ty16;  // row-split mode: 16-row y boxes (a worker warp's own rows)
  if (rows) {
    if (int rc = make_map_f32_seq(&ty16, a->y, a->batch, a->seq_len, 128, 16)) return rc;
  }
  auto launch = [&](auto k_small, auto k_rows) {
    if (rows) {
      if (int rc = set_smem(reinterpret_cast<const void*>(k_rows), smem)) return rc;
      if (int rc = check_block_fits(reinterpret_cast<const void*>(k_rows), SmallCfg::THREADS)) return rc;
      launch_kernel(k_rows, dim3(2 * a->batch), dim3(SmallCfg::THREADS), smem, st, tq, to, ti, tout, tx, ty16, p);
      return launch_status();
    }
    if (int rc = set_smem(reinterpret_cast<const void*>(k_small), smem)) return rc;
    if (int rc = check_block_fits(reinterpret_cast<const void*>(k_small), SmallCfg::THREADS)) return rc;
    const int grid = a->batch < num_sms() ? a->batch : num_sms();
    launch_kernel(k_small, dim3(grid), dim3(SmallCfg::THREADS), smem, st, tq, to, ti, tout, tx, ty, p);
    return launch_status();
  };
  if (a->num_heads == 4) return launch(k_block_small<4>, k_block_rows<4>);
  if (a->num_heads == 2) return launch(k_block_small<2>, k_block_rows<2>);
  return launch(k_block_small<1>, k_block_rows<1>);
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct BlockWs {
  __half* n;     // [M, d] fp16 LayerNorm output (LN1, then LN2)
  __half* qkv;   // [M, 3d] fp16
  __half* ctx;   // [M, d] fp16
  float* x1;     // [M, d] fp32 residual stream after attention (then after FFN)
  __half* h;     // [M, ffn] fp16 GELU activations
  size_t bytes;
};

BlockWs carve(void* base, long long M, int d, int ffn) {
  BlockWs w{};
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* r = p ? p + off : nullptr;
    off += align256(n);
    return r;
  };
  w.n = reinterpret_cast<__half*>(take(static_cast<size_t>(M) * d * 2));
  w.qkv = reinterpret_cast<__half*>(take(static_cast<size_t>(M) * 3 * d * 2));
  w.ctx = reinterpret_cast<__half*>(take(static_cast<size_t>(M) * d * 2));
  w.x1 = reinterpret_cast<float*>(take(static_cast<size_t>(M) * d * 4));
  w.h = reinterpret_cast<__half*>(take(static_cast<size_t>(M) * ffn * 2));
  w.bytes = off;
  return w;
}

int block_impl(const B200BlockArgs* a, cudaStream_t st) {
  if (!a || !a->x || !a->y || !a->w_qkv || !a->w_o || !a->w_in || !a->w_out) return B200_ERR_ARG;
  if (!a->ln1_w || !a->ln1_b || !a->ln2_w || !a->ln2_b || !a->b_qkv || !a->b_o || !a->b_in || !a->b_out)
    return B200_ERR_ARG;
  if ((a->lnf_w == nullptr) != (a->lnf_b == nullptr)) return B200_ERR_ARG;
  if (a->batch <= 0 || a->seq_len <= 0 || a->d_model <= 0 || a->num_heads <= 0 || a->ffn_dim <= 0) return B200_ERR_ARG;
  if (a->d_model % a->num_heads) return B200_ERR_ARG;
  if (a->x == a->y) return B200_ERR_ARG;
  const long long M = static_cast<long long>(a->batch) * a->seq_len;
  const int d = a->d_model, F = a->ffn_dim, H = a->num_heads, hd = d / H;
  if (hd != 8 && hd != 16 && hd != 32 && hd != 64 && hd != 128 && hd != 256) return B200_ERR_HEAD_DIM;
  if (M > 0x7fffffffLL) return B200_ERR_TILE;
  BlockWs w = carve(a->workspace, M, d, F);
  if (!a->workspace || a->workspace_bytes < w.bytes) return B200_ERR_WORKSPACE;
  if (!al16(a->workspace)) return B200_ERR_ALIGN;
  int rc;
  // residual stream: x1 (final norm follows) or y itself; the projection GEMMs
  // add onto it in place
  float* res = a->lnf_w ? w.x1 : a->y;
  // 1. n = LN1(x) (fp16), res = x
  if ((rc = ln_impl(a->x, d, a->ln1_w, a->ln1_b, w.n, d, 1, static_cast<int>(M), d, a->eps, st, res, d))) return rc;
  // 2. qkv = n . Wqkv^T + bqkv
  if ((rc = gemm_impl(EPI_BIAS_F16, w.n, d, a->w_qkv, d, a->b_qkv, nullptr, 0, w.qkv, 3 * d, static_cast<int>(M),
                      3 * d, d, st)))
    return rc;
  // 3. ctx = causal_attention(q, k, v)
  B200AttnArgs at{};
  at.q = at.k = at.v = w.qkv;
  at.ld_q = at.ld_k = at.ld_v = 3 * d;
  at.q_rows = at.kv_rows = M;
  at.batch = a->batch;
  at.heads = H;
  at.head_dim = hd;
  at.q_len = at.kv_len = a->seq_len;
  at.q_offset = 0;
  at.q_seq_rows = at.kv_seq_rows = a->seq_len;
  at.q_row0 = at.kv_row0 = 0;
  at.q_col0 = 0;
  at.k_col0 = d;
  at.v_col0 = 2 * d;
  at.out = w.ctx;
  at.ld_out = d;
  at.out_seq_rows = a->seq_len;
  at.out_row0 = 0;
  at.non_causal = a->non_causal;
  at.kv_lens = a->kv_lens;
  at.key_bits = a->key_bits;
  at.key_words = a->key_words;
  at.key_holes = a->key_holes;
  if ((rc = attn_impl(&at, st))) return rc;
  // 4. x1 = x + ctx . Wo^T + bo  (res += ...);  5. n = LN2(x1) -- one kernel when d == 128
  if (fuse_ln(d)) {
    if ((rc = gemm_ln_impl(w.ctx, d, a->w_o, d, a->b_o, res, d, a->ln2_w, a->ln2_b, a->eps, w.n, d, 1,
                           static_cast<int>(M), d, d, st)))
      return rc;
  } else {
    if ((rc = gemm_impl(EPI_BIAS_RESID_F32, w.ctx, d, a->w_o, d, a->b_o, res, d, res, d, static_cast<int>(M), d, d,
                        st)))
      return rc;
    if ((rc = ln_impl(res, d, a->ln2_w, a->ln2_b, w.n, d, 1, static_cast<int>(M), d, a->eps, st))) return rc;
  }
  // 6. h = gelu(n . W1^T + b1)
  if ((rc = gemm_impl(EPI_BIAS_GELU_F16, w.n, d, a->w_in, d, a->b_in, nullptr, 0, w.h, F, static_cast<int>(M), F, d,
                      st)))
    return rc;
  // 7. x2 = x1 + h . W2^T + b2  (res += ...; without a final norm res is y);
  //    8. y = LN_f(x2) in the same kernel when d == 128
  if (a->lnf_w && fuse_ln(d)) {
    return gemm_ln_impl(w.h, F, a->w_out, F, a->b_out, res, d, a->lnf_w, a->lnf_b, a->eps, a->y, d, 0,
                        static_cast<int>(M), d, F, st);
  }
  if ((rc = gemm_impl(EPI_BIAS_RESID_F32, w.h, F, a->w_out, F, a->b_out, res, d, res, d, static_cast<int>(M), d, F,
                      st)))
    return rc;
  // 8. y = LN_f(x2)
  if (a->lnf_w) {
    if ((rc = ln_impl(w.x1, d, a->lnf_w, a->lnf_b, a->y, d, 0, static_cast<int>(M), d, a->eps, st))) return rc;
  }
  return B200_OK;
}

// ------------------------------------------------------------------ sequence-chunked forward
// The reference's _chunked_forward_causal (TTB:1378-1609): for each sequence,
// query chunks [c0, c1) in order; the chunk's K/V rows are appended to an fp16
// cache [tokens, 2d] and its queries attend keys [0, c1) through the
// prefix-causal attention (q_offset = c0, TTB:1491-1500); the position-wise
// rest of the block runs on the chunk only.  Peak memory: the K/V cache plus
// one chunk's activations.
struct ChunkWs {
  __half* kv;    // [M, 2d]
  __half* q;     // [R, d]
  __half* n;     // [R, d]
  __half* ctx;   // [R, d]
  float* x1;     // [R, d]
  __half* h;     // [R, F]
  size_t bytes;
};

ChunkWs carve_chunked(void* base, long long M, long long R, int d, int F) {
  ChunkWs w{};
  uint8_t* p = static_cast<uint8_t*>(base);
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* r = p ? p + off : nullptr;
    off += align256(n);
    return r;
  };
  w.kv = reinterpret_cast<__half*>(take(static_cast<size_t>(M) * 2 * d * 2));
  w.q = reinterpret_cast<__half*>(take(static_cast<size_t>(R) * d * 2));
  w.n = reinterpret_cast<__half*>(take(static_cast<size_t>(R) * d * 2));
  w.ctx = reinterpret_cast<__half*>(take(static_cast<size_t>(R) * d * 2));
  w.x1 = reinterpret_cast<float*>(take(static_cast<size_t>(R) * d * 4));
  w.h = reinterpret_cast<__half*>(take(static_cast<size_t>(R) * F * 2));
  w.bytes = off;
  return w;
}

int block_chunked_impl(const B200BlockArgs* a, int chunk_rows, cudaStream_t st) {
  if (!a || !a->x || !a->y || !a->w_qkv || !a->w_o || !a->w_in || !a->w_out) return B200_ERR_ARG;
  if (!a->ln1_w || !a->ln1_b || !a->ln2_w || !a->ln2_b || !a->b_qkv || !a->b_o || !a->b_in || !a->b_out)
    return B200_ERR_ARG;
  if ((a->lnf_w == nullptr) != (a->lnf_b == nullptr)) return B200_ERR_ARG;
  if (a->batch <= 0 || a->seq_len <= 0 || a->d_model <= 0 || a->num_heads <= 0 || a->ffn_dim <= 0 || chunk_rows <= 0)
    return B200_ERR_ARG;
  if (a->d_model % a->num_heads || a->x == a->y) return B200_ERR_ARG;
  if (a->non_causal) return B200_ERR_CONFIG;  // prefix chunking is a causal construction
  const long long M = static_cast<long long>(a->batch) * a->seq_len;
  const int d = a->d_model, F = a->ffn_dim, H = a->num_heads, hd = d / H, S = a->seq_len;
  if (hd != 8 && hd != 16 && hd != 32 && hd != 64 && hd != 128 && hd != 256) return B200_ERR_HEAD_DIM;
  if (M > 0x7fffffffLL) return B200_ERR_TILE;
  const int R = chunk_rows < S ? chunk_rows : S;
  ChunkWs w = carve_chunked(a->workspace, M, R, d, F);
  if (!a->workspace || a->workspace_bytes < w.bytes) return B200_ERR_WORKSPACE;
  if (!al16(a->workspace)) return B200_ERR_ALIGN;
  const __half* wq = static_cast<const __half*>(a->w_qkv);
  int rc;
  for (int b = 0; b < a->batch; ++b) {
    for (int c0 = 0; c0 < S; c0 += R) {
      const int Rc = (S - c0) < R ? (S - c0) : R;
      const long long row0 = static_cast<long long>(b) * S + c0;
      const float* xr = a->x + row0 * d;
      float* yr = a->y + row0 * d;
      float* res = a->lnf_w ? w.x1 : yr;  // the chunk's residual stream
      if ((rc = ln_impl(xr, d, a->ln1_w, a->ln1_b, w.n, d, 1, Rc, d, a->eps, st, res, d))) return rc;
      // q rows of the fused QKV weight -> chunk buffer; k|v rows -> the cache at this chunk's rows
      if ((rc = gemm_impl(EPI_BIAS_F16, w.n, d, wq, d, a->b_qkv, nullptr, 0, w.q, d, Rc, d, d, st))) return rc;
      if ((rc = gemm_impl(EPI_BIAS_F16, w.n, d, wq + static_cast<size_t>(d) * d, d, a->b_qkv + d, nullptr, 0,
                          w.kv + row0 * 2 * d, 2 * d, Rc, 2 * d, d, st)))
        return rc;
      B200AttnArgs at{};
      at.q = w.q;
      at.k = at.v = w.kv;
      at.ld_q = d;
      at.ld_k = at.ld_v = 2 * d;
      at.q_rows = Rc;
      // the cache rows after this chunk are not written yet: end the tensor at the
      // last valid key so the key tile that straddles it is zero-filled by TMA
      at.kv_rows = static_cast<long long>(b) * S + c0 + Rc;
      at.batch = 1;
      at.heads = H;
      at.head_dim = hd;
      at.q_len = Rc;
      at.q_offset = c0;
      at.kv_len = c0 + Rc;
      at.q_seq_rows = Rc;
      at.kv_seq_rows = S;
      at.q_row0 = 0;
      at.kv_row0 = static_cast<int>(static_cast<long long>(b) * S);
      at.q_col0 = 0;
      at.k_col0 = 0;
      at.v_col0 = d;
      at.out = w.ctx;
      at.ld_out = d;
      at.out_seq_rows = Rc;
      at.out_row0 = 0;
      if (a->key_holes != nullptr) {  // this sequence's key-padding mask (a one-sequence call)
        at.key_bits = a->key_bits + static_cast<size_t>(b) * a->key_words;
        at.key_words = a->key_words;
        at.key_holes = a->key_holes + b;
      }
      if ((rc = attn_impl(&at, st))) return rc;
      if (fuse_ln(d)) {
        if ((rc = gemm_ln_impl(w.ctx, d, a->w_o, d, a->b_o, res, d, a->ln2_w, a->ln2_b, a->eps, w.n, d, 1, Rc, d, d,
                               st)))
          return rc;
      } else {
        if ((rc = gemm_impl(EPI_BIAS_RESID_F32, w.ctx, d, a->w_o, d, a->b_o, res, d, res, d, Rc, d, d, st))) return rc;
        if ((rc = ln_impl(res, d, a->ln2_w, a->ln2_b, w.n, d, 1, Rc, d, a->eps, st))) return rc;
      }
      if ((rc = gemm_impl(EPI_BIAS_GELU_F16, w.n, d, a->w_in, d, a->b_in, nullptr, 0, w.h, F, Rc, F, d, st))) return rc;
      if (a->lnf_w && fuse_ln(d)) {
        if ((rc = gemm_ln_impl(w.h, F, a->w_out, F, a->b_out, res, d, a->lnf_w, a->lnf_b, a->eps, yr, d, 0, Rc, d, F,
                               st)))
          return rc;
        continue;
      }
      if ((rc = gemm_impl(EPI_BIAS_RESID_F32, w.h, F, a->w_out, F, a->b_out, res, d, res, d, Rc, d, F, st))) return rc;
      if (a->lnf_w && (rc = ln_impl(w.x1, d, a->lnf_w, a->lnf_b, yr, d, 0, Rc, d, a->eps, st))) return rc;
    }
  }
  return B200_OK;
}

}  // namespace

// ====================================================================== C ABI
extern "C" {

int b200_abi_version(void) { return B200_ABI_VERSION; }

const char* b200_last_error_detail(void) { return g_detail; }

const char* b200_status_str(int s) {
  switch (s) {
    case B200_OK: return "ok";
    case B200_ERR_CONFIG: return "unsupported configuration or epilogue";
    case B200_ERR_TILE: return "dimension is not a multiple of the required granule";
    case B200_ERR_SPLIT: return "K is not a multiple of the split size";
    case B200_ERR_SMEM: return "dynamic shared memory opt-in refused";
    case B200_ERR_ALIGN: return "pointer or leading dimension not 16-byte aligned";
    case B200_ERR_HEAD_DIM: return "head_dim must be 32, 64, 128 or 256";
    case B200_ERR_DEVICE: return "device-side wait timed out";
    case B200_ERR_LAUNCH: return "CUDA kernel launch failed";
    case B200_ERR_ARG: return "invalid argument";
    case B200_ERR_TMAP: return "TMA tensor map encoding failed";
    case B200_ERR_ARCH: return "current device is not compute capability 10.0 (B200, sm_100a)";
    case B200_ERR_WORKSPACE: return "workspace missing or too small";
    case B200_ERR_NOALLOC_LIMIT:
      return "problem needs more scratch than the no-allocation entry point's static buffer "
             "(B200_NOALLOC_SCRATCH_BYTES = 32 MiB); use b200_block_forward with a workspace";
    case B200_ERR_SCRATCH_SETUP: return "could not resolve the static scratch buffer's device address";
    default: return "unknown status";
  }
}

int b200_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_b200_err, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_LAUNCH;
  }
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_b200_err, &zero, sizeof(int));
  }
  return v;
}

int b200_layernorm_launch(const float* x, long long ld_x, const float* gamma, const float* beta, void* out,
                          long long ld_out, int out_f16, int rows, int d, float eps, b200_stream_t stream) {
  return ln_impl(x, ld_x, gamma, beta, out, ld_out, out_f16, rows, d, eps, static_cast<cudaStream_t>(stream));
}

int b200_gemm_residual_layernorm_launch(const void* A, long long lda, const void* W, long long ldw, const float* bias,
                                        float* res, long long ld_res, const float* gamma, const float* beta, float eps,
                                        void* ln_out, long long ld_ln, int ln_out_f16, int M, int N, int K,
                                        b200_stream_t stream) {
  return gemm_ln_impl(A, lda, W, ldw, bias, res, ld_res, gamma, beta, eps, ln_out, ld_ln, ln_out_f16, M, N, K,
                      static_cast<cudaStream_t>(stream));
}

int b200_layernorm_residual_launch(const float* x, long long ld_x, const float* gamma, const float* beta, void* out,
                                   long long ld_out, int out_f16, float* residual_out, long long ld_residual,
                                   int rows, int d, float eps, b200_stream_t stream) {
  if (!residual_out) return B200_ERR_ARG;
  return ln_impl(x, ld_x, gamma, beta, out, ld_out, out_f16, rows, d, eps, static_cast<cudaStream_t>(stream),
                 residual_out, ld_residual);
}

int b200_add_layernorm_launch(const float* a, const float* b, const float* bias, float* sum_out, const float* gamma,
                              const float* beta, void* out, int out_f16, int rows, int d, float eps,
                              b200_stream_t stream) {
  return add_ln_impl(a, b, bias, sum_out, gamma, beta, out, out_f16, rows, d, eps, static_cast<cudaStream_t>(stream));
}

int b200_zero_masked_rows(float* y, const unsigned char* row_valid, long long rows, int d, b200_stream_t stream) {
  if (!y || !row_valid || rows < 0 || d <= 0) return B200_ERR_ARG;
  if (rows == 0) return B200_OK;
  if (int rc = check_arch()) return rc;
  const int vec4 = (d % 4 == 0 && al16(y)) ? 1 : 0;
  launch_kernel(k_mask_finish, dim3(static_cast<unsigned>((rows + 255) / 256)), dim3(256), 0,
                static_cast<cudaStream_t>(stream), y, row_valid, rows, d, vec4);
  return launch_status();
}

int b200_mask_key_words(int seq_len) { return seq_len > 0 ? 4 * ((seq_len + 127) / 128) : 0; }

int b200_mask_prepare(const unsigned char* mask, int batch, int seq_len, int* kv_lens, int* key_holes,
                      unsigned int* key_bits, b200_stream_t stream) {
  if (!mask || !kv_lens || batch <= 0 || seq_len <= 0) return B200_ERR_ARG;
  if ((key_holes == nullptr) != (key_bits == nullptr)) return B200_ERR_ARG;
  if (key_bits != nullptr && !al16(key_bits)) return B200_ERR_ALIGN;
  if (int rc = check_arch()) return rc;
  launch_kernel(k_mask_prepare, dim3(static_cast<unsigned>(batch)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                mask, seq_len, kv_lens, key_holes, reinterpret_cast<uint32_t*>(key_bits),
                b200_mask_key_words(seq_len));
  return launch_status();
}

int b200_gemm_launch(int epilogue, const void* A, long long lda, const void* W, long long ldw, const float* bias,
                     const float* resid, long long ld_resid, void* out, long long ld_out, int M, int N, int K,
                     b200_stream_t stream) {
  return gemm_impl(epilogue, A, lda, W, ldw, bias, resid, ld_resid, out, ld_out, M, N, K,
                   static_cast<cudaStream_t>(stream));
}

int b200_flash_causal_launch(const B200AttnArgs* args, b200_stream_t stream) {
  return attn_impl(args, static_cast<cudaStream_t>(stream));
}

size_t b200_block_workspace_bytes(long long tokens, int d_model, int ffn_dim) {
  if (tokens <= 0 || d_model <= 0 || ffn_dim <= 0) return 0;
  return carve(nullptr, tokens, d_model, ffn_dim).bytes;
}

int b200_block_forward(const B200BlockArgs* args, b200_stream_t stream) {
  return block_impl(args, static_cast<cudaStream_t>(stream));
}

size_t b200_block_chunked_workspace_bytes(long long tokens, int chunk_rows, int d_model, int ffn_dim) {
  if (tokens <= 0 || chunk_rows <= 0 || d_model <= 0 || ffn_dim <= 0) return 0;
  return carve_chunked(nullptr, tokens, chunk_rows, d_model, ffn_dim).bytes;
}

int b200_block_forward_chunked(const B200BlockArgs* args, int chunk_rows, b200_stream_t stream) {
  return block_chunked_impl(args, chunk_rows, static_cast<cudaStream_t>(stream));
}

int b200_block_fused_small_launch(const B200FusedSmallArgs* args, b200_stream_t stream) {
  return fused_small_impl(args, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ====================================================================== no-allocation entry point
// Scratch for b200_block_forward_noalloc: one static device buffer per GPU
// that loads the library, held until exit.  In host code `g_noalloc_scratch`
// names a host-side stand-in, not a device address; its device address is
// looked up with cudaGetSymbolAddress once per device (with that device
// current) and that address is what the kernels are given.
static __device__ __align__(256) unsigned char g_noalloc_scratch[B200_NOALLOC_SCRATCH_BYTES];

namespace {
// Per device: the context the address was resolved in, and the address.  A call
// from another context on the same device (a new primary context after
// cudaDeviceReset, or a context the caller created) resolves it again.
CUcontext g_noalloc_ctx[128] = {nullptr};
void* g_noalloc_addr[128] = {nullptr};
PFN_cuCtxGetCurrent_v4000 g_ctx_get = nullptr;
std::once_flag g_ctx_once;

CUcontext current_context() {
  std::call_once(g_ctx_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_get = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    else
      cudaGetLastError();
  });
  CUcontext c = nullptr;
  if (g_ctx_get == nullptr || g_ctx_get(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

int noalloc_scratch_addr(void** out) {
  const int dev = current_device();
  if (dev < 0 || dev >= 128) return B200_ERR_SCRATCH_SETUP;
  const CUcontext ctx = current_context();
  if (ctx == nullptr) return B200_ERR_SCRATCH_SETUP;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_noalloc_addr[dev] == nullptr || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      set_detail("cudaGetSymbolAddress(g_noalloc_scratch)", e);
      return B200_ERR_SCRATCH_SETUP;
    }
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_addr[dev];
  return B200_OK;
}
}  // namespace

extern "C" int b200_block_forward_noalloc(const B200BlockArgs* args, b200_stream_t stream) {
  if (!args || args->batch <= 0 || args->seq_len <= 0 || args->d_model <= 0 || args->ffn_dim <= 0)
    return B200_ERR_ARG;
  const long long tokens = static_cast<long long>(args->batch) * args->seq_len;
  if (carve(nullptr, tokens, args->d_model, args->ffn_dim).bytes > B200_NOALLOC_SCRATCH_BYTES)
    return B200_ERR_NOALLOC_LIMIT;
  if (int rc = check_arch()) return rc;
  void* scratch = nullptr;
  if (int rc = noalloc_scratch_addr(&scratch)) return rc;
  B200BlockArgs a = *args;
  a.workspace = scratch;
  a.workspace_bytes = B200_NOALLOC_SCRATCH_BYTES;
  return block_impl(&a, static_cast<cudaStream_t>(stream));
}
