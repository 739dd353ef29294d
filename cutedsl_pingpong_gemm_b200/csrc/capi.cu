// Host side of the C ABI declared in include/cpgemm.h: configuration checks (the reference's
// constructor asserts), problem checks, kernel selection, tensor-map encoding and launch.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "cpgemm.h"
#include "gemm_decode.cuh"
#include "gemm_fp8_block.cuh"
#include "gemm_kernel.cuh"
#include "peer_kernels.cuh"
#include "quant_kernels.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(CPG_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) return;
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) return;
    ok = true;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

// 3-D tiled tensor map (columns, rows, batches) with a box of box_rows x box_cols x 1, 128-byte
// swizzled unless told otherwise.  An unbatched operand has one batch; its batch stride is then
// any legal value.
int encode_tiled(CUtensorMap* m, CUtensorMapDataType dt, int elem_bytes, const void* ptr,
                 int64_t rows, int64_t cols, int64_t ld, int box_rows, int box_cols,
                 int64_t batches = 1, int64_t batch_stride = 0,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(CPG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (batches < 1) batches = 1;
  if (batches == 1) {
    const int64_t span = (rows > 1 ? rows : 1) * ld;
    batch_stride = batch_stride > span ? batch_stride : span;
    batch_stride = (batch_stride * elem_bytes + 15) / 16 * 16 / elem_bytes;
  }
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batches)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * elem_bytes),
                           static_cast<cuuint64_t>(batch_stride * elem_bytes)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(CPG_ERR_CUDA,
                "cuTensorMapEncodeTiled failed (%d) rows=%lld cols=%lld ld=%lld batches=%lld "
                "batch_stride=%lld",
                static_cast<int>(r), static_cast<long long>(rows), static_cast<long long>(cols),
                static_cast<long long>(ld), static_cast<long long>(batches),
                static_cast<long long>(batch_stride));
  }
  return CPG_OK;
}

using KernelFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                          const CUtensorMap, const cpg::GemmParams);

struct Variant {
  int bn;
  int cta_group;
  int dtype_ab;
  int dtype_d;
  int scale_mode;  // CPG_SCALE_TENSOR (plain kernel) or CPG_SCALE_BLOCK
  const void* fn;
  int (*smem_bytes)(int, int, int);
  int threads;
  int epi_warps;  // epilogue warps per CTA (each owns 32 rows and a share of the columns)
};

template <int BN, int CG>
int smem_bytes_of(int stages, int epi_stages, int reuse_ab) {
  return cpg::GemmSmem<BN, CG>::bytes(stages, epi_stages, reuse_ab);
}

template <typename T>
constexpr int dtype_code();
template <>
constexpr int dtype_code<__nv_bfloat16>() { return CPG_DTYPE_BF16; }
template <>
constexpr int dtype_code<cpg::e4m3_t>() { return CPG_DTYPE_E4M3; }
template <>
constexpr int dtype_code<float>() { return CPG_DTYPE_F32; }

template <int BN, int CG, typename AB, typename OutT>
Variant make_variant() {
  KernelFn fn = &cpg::gemm_sm100_kernel<BN, CG, AB, OutT>;
  return Variant{BN, CG, dtype_code<AB>(), dtype_code<OutT>(), CPG_SCALE_TENSOR,
                 reinterpret_cast<const void*>(fn), &smem_bytes_of<BN, CG>,
                 cpg::EpiShape<BN>::kThreads, cpg::EpiShape<BN>::kWarps};
}

template <int BN, int CG>
int block_smem_bytes_of(int stages, int epi_stages, int reuse_ab) {
  return cpg::BlockSmem<BN, CG>::bytes(stages, epi_stages, reuse_ab);
}

template <int BN, int CG>
Variant make_block_variant() {
  using BlockFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                           const cpg::GemmParams, const cpg::BlockScales);
  BlockFn fn = &cpg::gemm_fp8_block_kernel<BN, CG>;
  return Variant{BN, CG, CPG_DTYPE_E4M3, CPG_DTYPE_BF16, CPG_SCALE_BLOCK,
                 reinterpret_cast<const void*>(fn), &block_smem_bytes_of<BN, CG>,
                 cpg::BlockShape<BN>::kThreads, cpg::kBlockEpiWarps};
}

template <typename AB, typename OutT>
void add_variants(Variant* t, int& n) {
  t[n++] = make_variant<512, 1, AB, OutT>();
  t[n++] = make_variant<512, 2, AB, OutT>();
  t[n++] = make_variant<256, 1, AB, OutT>();
  t[n++] = make_variant<128, 1, AB, OutT>();
  t[n++] = make_variant<64, 1, AB, OutT>();
  t[n++] = make_variant<256, 2, AB, OutT>();
  t[n++] = make_variant<128, 2, AB, OutT>();
  t[n++] = make_variant<64, 2, AB, OutT>();
}

bool find_variant(int bn, int cta_group, int dtype_ab, int dtype_d, int scale_mode,
                  Variant* out) {
  static Variant table[36];
  static int count = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    add_variants<__nv_bfloat16, __nv_bfloat16>(table, count);
    add_variants<__nv_bfloat16, float>(table, count);
    add_variants<cpg::e4m3_t, __nv_bfloat16>(table, count);
    add_variants<cpg::e4m3_t, float>(table, count);
    table[count++] = make_block_variant<128, 1>();
    table[count++] = make_block_variant<128, 2>();
    table[count++] = make_block_variant<256, 1>();
    table[count++] = make_block_variant<256, 2>();
  });
  if (scale_mode != CPG_SCALE_BLOCK) scale_mode = CPG_SCALE_TENSOR;
  for (int i = 0; i < count; ++i) {
    const Variant& v = table[i];
    if (v.bn == bn && v.cta_group == cta_group && v.dtype_ab == dtype_ab && v.dtype_d == dtype_d &&
        v.scale_mode == scale_mode) {
      *out = v;
      return true;
    }
  }
  return false;
}

int elem_bytes(int dtype) { return dtype == CPG_DTYPE_E4M3 ? 1 : (dtype == CPG_DTYPE_F32 ? 4 : 2); }

// Raster group size of a plan whose K ranges hold k_iters k-blocks.  The dynamic schedule starts
// clusters in id order, so the clusters running at any time hold about consecutive ids: a
// group's re-read operand panel (raster AlongN: the B rows of its cluster columns over one K
// range; AlongM: the A rows of its cluster rows) should stay in L2 while the group's tiles pass.
// The group size is lowered until that panel is at most 32 MiB.  Measured on B200 with 256 x 512
// pair tiles against the reference's 8: the LLM shape (BF16, K = 8192: 8 MiB per column, so 4)
// +1.7 %, the fused SwiGLU +1.9 %, 8192^3 equal; FP8 at K = 8192 (4 MiB per column, stays 8)
// ran 2 % slower with 4.  The static schedule keeps the configured size.
int32_t plan_group_size(const cpg_gemm_config* cfg, int64_t k_iters) {
  const int64_t group_size = cfg->group_size;
  if (!cfg->dynamic_scheduler) return cfg->group_size;
  const int64_t panel_rows = cfg->raster_order == CPG_RASTER_ALONG_N
                                 ? int64_t(cfg->tile_n) * cfg->cluster_n
                                 : int64_t(128) * cfg->cluster_m;
  const int64_t panel = panel_rows * k_iters * cpg::kRowBytes;
  const int64_t fit = panel > 0 ? (int64_t(32) << 20) / panel : group_size;
  return static_cast<int32_t>(std::max<int64_t>(1, std::min<int64_t>(group_size, fit)));
}

CUtensorMapDataType tma_dtype(int dtype) {
  switch (dtype) {
    case CPG_DTYPE_E4M3: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
    case CPG_DTYPE_F32: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    default: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  }
}

template <typename OutT>
__global__ void fill_rows_kernel(OutT* d, int64_t m, int64_t n, int64_t ldd,
                                 const __nv_bfloat16* bias) {
  int64_t total = m * n;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t r = i / n, c = i % n;
    float v = bias != nullptr ? __bfloat162float(bias[c]) : 0.f;
    d[r * ldd + c] = static_cast<OutT>(v);
  }
}

// Status word value of a grouped launch whose offsets broke the rule (groups made empty).
constexpr int32_t kStatusBadGroups = 0x200;
constexpr int kPrefixThreads = 1024;

// Cluster-tile prefix of a grouped GEMM: prefix[g] = sum over h < g of
// ceil(M_h / rows_per_cluster) * n_clusters with M_h = offsets[h + 1] - offsets[h].  One block:
// thread t sums its contiguous run of groups, a block-wide scan gives each run's start.
__global__ void __launch_bounds__(kPrefixThreads)
    group_tile_prefix_kernel(const int32_t* offsets, int32_t groups, int64_t rows,
                             int32_t rows_per_cluster, int32_t n_clusters, int32_t* prefix,
                             int32_t* status) {
  __shared__ int64_t sums[kPrefixThreads];
  const int t = threadIdx.x;
  const int per = (groups + kPrefixThreads - 1) / kPrefixThreads;
  const int g0 = min(t * per, groups), g1 = min(g0 + per, groups);
  bool bad = false;
  auto tiles = [&](int g) -> int64_t {
    const int32_t s = offsets[g], e = offsets[g + 1];
    if (s < 0 || e < s || e > rows) {
      bad = true;
      return 0;
    }
    return static_cast<int64_t>((e - s + rows_per_cluster - 1) / rows_per_cluster) * n_clusters;
  };
  int64_t local = 0;
  for (int g = g0; g < g1; ++g) local += tiles(g);
  sums[t] = local;
  __syncthreads();
  for (int o = 1; o < kPrefixThreads; o <<= 1) {
    const int64_t v = t >= o ? sums[t - o] : 0;
    __syncthreads();
    sums[t] += v;
    __syncthreads();
  }
  int64_t run = t > 0 ? sums[t - 1] : 0;
  for (int g = g0; g < g1; ++g) {
    prefix[g] = static_cast<int32_t>(run);
    run += tiles(g);
  }
  if (t == kPrefixThreads - 1) prefix[groups] = static_cast<int32_t>(sums[t]);
  if (bad && status != nullptr) atomicCAS(status, 0, kStatusBadGroups);
}

// Grid of cast_f32_bf16_kernel: x covers a row's columns in quads of 4 (256 threads per block),
// y covers rows (grid-stride beyond 65535), about 32 k blocks in total.
dim3 cast_grid(int64_t rows, int64_t cols) {
  const int64_t bx = (cols + 1023) / 1024;
  int64_t by = (32768 + bx - 1) / bx;
  if (by > rows) by = rows;
  if (by > 65535) by = 65535;
  if (by < 1) by = 1;
  return dim3(static_cast<unsigned>(bx), static_cast<unsigned>(by), 1);
}

// Raise (never lower) a kernel's dynamic shared-memory limit on the current device.  Plans of
// different shapes share a kernel function: a plan created later with a smaller need must not
// make an earlier plan's launch fail.
cudaError_t raise_smem_limit(const void* fn, int smem) {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, fn);
  if (e != cudaSuccess) return e;
  if (fa.maxDynamicSharedSizeBytes >= smem) return cudaSuccess;
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}

int query_max_active_clusters(const Variant& v, int smem, int cm, int cn, int* out) {
  cudaError_t e = raise_smem_limit(v.fn, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(max dynamic smem)");
  int dev = 0;
  cudaGetDevice(&dev);
  if (cm * cn == 1) {
    int per_sm = 0, sms = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, v.fn, v.threads, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    *out = per_sm * sms;
    return CPG_OK;
  }
  cudaLaunchConfig_t lc = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cm;
  attr[0].val.clusterDim.y = cn;
  attr[0].val.clusterDim.z = 1;
  lc.gridDim = dim3(cm, cn, 1);
  lc.blockDim = dim3(v.threads, 1, 1);
  lc.dynamicSmemBytes = smem;
  lc.attrs = attr;
  lc.numAttrs = 1;
  int n = 0;
  e = cudaOccupancyMaxActiveClusters(&n, v.fn, &lc);
  if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
  *out = n;
  return CPG_OK;
}

}  // namespace

struct cpg_gemm {
  cpg_gemm_config cfg;
  cpg_gemm_problem prob;
  int device;
  Variant v;
  int smem_bytes;
  int grid[3];
  int cluster[3];
  int max_active_clusters;
  cpg::SchedParams sched;
  int32_t* status_dev;
  int32_t* trace;
  int32_t trace_stride;
  uint64_t timeout_ns;
  int32_t fault_inject;
  int32_t l2_policy_a, l2_policy_b, l2_policy_d;
  int32_t k_iters;
  int32_t k_iters_per_split;
  int32_t splits;
  int32_t stream_k;
  // Stream-K with in-kernel fixup (BF16 Stream-K, and the data-parallel + Stream-K hybrid):
  // leading whole tiles, FP32 workspace tiles and k-block counts of the Stream-K tail.
  int32_t fixup;
  int32_t dp_tiles;
  float* ws_dev;
  int32_t* cnt_dev;
  int64_t ws_bytes, cnt_bytes;
  CUtensorMap tm_ws;
  int64_t batches;
  int64_t groups;            // grouped GEMM: number of groups (0: not grouped)
  int32_t group_n_clusters;  // cluster columns of every group
  int32_t* tile_prefix_dev;  // [groups + 1], written by group_tile_prefix_kernel per launch
  bool maps_valid;
  const void* map_a_ptr;
  const void* map_b_ptr;
  const void* map_d_ptr;
  CUtensorMap tm_a, tm_b, tm_d;
  // Small-M plan (CPG_SPLIT_K_DECODE): gemm_decode_kernel with these launch constants.
  int32_t decode;
  int32_t dec_mma_n, dec_tmem_cols, dec_kps, dec_splits, dec_stages, dec_cg, dec_spin, dec_rotate;
  int32_t dec_pdl;  // launched as a programmatic dependent of the stream's previous kernel
  int32_t dec_st_async;  // partial sums by per-thread st.async (else staged bulk copies)
};

extern "C" {

int cpg_abi_version(void) { return 14; }

const char* cpg_strerror(int code) {
  switch (code) {
    case CPG_OK: return "ok";
    case CPG_ERR_INVALID_CONFIG: return "invalid GEMM configuration";
    case CPG_ERR_INVALID_SHAPE: return "invalid problem shape or stride";
    case CPG_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case CPG_ERR_DTYPE: return "unsupported element type";
    case CPG_ERR_UNSUPPORTED: return "configuration not implemented on sm_100a";
    case CPG_ERR_NO_DEVICE: return "no usable sm_100 device";
    case CPG_ERR_CUDA: return "CUDA call failed";
    case CPG_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    case CPG_ERR_SMEM: return "configuration exceeds shared memory";
    case CPG_ERR_NULL: return "null pointer argument";
    default: return "unknown error";
  }
}

const char* cpg_last_error_message(void) { return g_last_error.c_str(); }

int cpg_config_validate(const cpg_gemm_config* c) {
  if (c == nullptr) return fail(CPG_ERR_NULL, "config is NULL");
  // gemm_base.py:72
  if (!(c->atom_m >= 1 && c->atom_m <= 3) || !(c->atom_n >= 1 && c->atom_n <= 2))
    return fail(CPG_ERR_INVALID_CONFIG, "atom_layout_mn must be in {1,2,3} x {1,2}, got (%d, %d)",
                c->atom_m, c->atom_n);
  // gemm_base.py:73-74
  if (!(c->atom_m == 1 || c->tile_m % (c->atom_m * 64) == 0))
    return fail(CPG_ERR_INVALID_CONFIG, "tile_m %d must be a multiple of atom_m * 64", c->tile_m);
  if (!(c->atom_n == 1 || c->tile_n % (c->atom_n * 32) == 0))
    return fail(CPG_ERR_INVALID_CONFIG, "tile_n %d must be a multiple of atom_n * 32", c->tile_n);
  // gemm_base.py:86-87
  int wg = c->atom_m * c->atom_n;
  if (wg < 1 || wg > 3)
    return fail(CPG_ERR_INVALID_CONFIG, "atom_m * atom_n must be 1, 2 or 3, got %d", wg);
  // gemm_base.py:113
  if (c->atom_n > 1 && c->epi_tile_n != c->tile_n)
    return fail(CPG_ERR_INVALID_CONFIG, "when atom layout n > 1, epi tile n must equal tile n");
  // gemm_base.py:122
  if (c->reuse_ab && c->is_persistent)
    return fail(CPG_ERR_INVALID_CONFIG, "persistent kernel can't reuse AB for epilogue");
  // tile_scheduler.py:51
  if (c->cluster_k != 1) return fail(CPG_ERR_INVALID_CONFIG, "cluster_shape_mnk[2] must be 1");
  if (c->tile_m <= 0 || c->tile_n <= 0 || c->epi_tile_m <= 0 || c->epi_tile_n <= 0 ||
      c->cluster_m <= 0 || c->cluster_n <= 0 || c->ab_stage <= 0 || c->epi_stage <= 0 ||
      c->group_size <= 0 || c->gemm_n_prologue < 0)
    return fail(CPG_ERR_INVALID_CONFIG, "tile, cluster, stage and group sizes must be positive");
  if (c->raster_order != CPG_RASTER_ALONG_M && c->raster_order != CPG_RASTER_ALONG_N)
    return fail(CPG_ERR_INVALID_CONFIG, "raster_order must be 0 (AlongM) or 1 (AlongN)");
  if (c->dynamic_scheduler != 0 && c->dynamic_scheduler != 1)
    return fail(CPG_ERR_INVALID_CONFIG, "dynamic_scheduler must be 0 or 1");
  if (c->dynamic_scheduler && c->reuse_ab)
    return fail(CPG_ERR_INVALID_CONFIG,
                "the dynamic scheduler runs several tiles per CTA and can't reuse AB for the "
                "epilogue");
  return CPG_OK;
}

// One FP32 workspace tile (128 rows x the tile's output columns) and one k-block count per
// epilogue warp per CTA of `tiles` cluster tiles, zero between launches: the tiles whose
// k-blocks are shared by several segments (Stream-K, or split-K into peer memory) sum there.
static int alloc_fixup_workspace(cpg_gemm* g, int64_t tiles) {
  const int64_t ctas = int64_t(g->cfg.cluster_m) * g->cfg.cluster_n;
  const int64_t ws_rows = tiles * ctas * 128;
  const int64_t ws_cols = g->cfg.tile_n;
  g->ws_bytes = ws_rows * ws_cols * 4;
  g->cnt_bytes = tiles * ctas * g->v.epi_warps * 4;
  cudaError_t e = cudaMalloc(&g->ws_dev, g->ws_bytes);
  if (e == cudaSuccess) e = cudaMalloc(&g->cnt_dev, g->cnt_bytes);
  if (e == cudaSuccess) e = cudaMemset(g->ws_dev, 0, g->ws_bytes);
  if (e == cudaSuccess) e = cudaMemset(g->cnt_dev, 0, g->cnt_bytes);
  const int rc = e == cudaSuccess
                     ? encode_tiled(&g->tm_ws, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, g->ws_dev,
                                    ws_rows, ws_cols, ws_cols, 32, cpg::kRowBytes / 4)
                     : cuda_fail(e, "fixup workspace");
  if (rc != CPG_OK) {
    if (g->ws_dev) cudaFree(g->ws_dev);
    if (g->cnt_dev) cudaFree(g->cnt_dev);
    g->ws_dev = nullptr;
    g->cnt_dev = nullptr;
    g->ws_bytes = g->cnt_bytes = 0;
  }
  return rc;
}

using DecodeFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap,
                          const cpg::DecodeParams);

static const void* decode_kernel(int dtype_ab, int dtype_d, int cta_group) {
  const bool fp8 = dtype_ab == CPG_DTYPE_E4M3, f32 = dtype_d == CPG_DTYPE_F32;
  DecodeFn fn;
  if (cta_group == 2) {
    fn = fp8 ? (f32 ? &cpg::gemm_decode_kernel<cpg::e4m3_t, float, 2>
                    : &cpg::gemm_decode_kernel<cpg::e4m3_t, __nv_bfloat16, 2>)
             : (f32 ? &cpg::gemm_decode_kernel<__nv_bfloat16, float, 2>
                    : &cpg::gemm_decode_kernel<__nv_bfloat16, __nv_bfloat16, 2>);
  } else {
    fn = fp8 ? (f32 ? &cpg::gemm_decode_kernel<cpg::e4m3_t, float, 1>
                    : &cpg::gemm_decode_kernel<cpg::e4m3_t, __nv_bfloat16, 1>)
             : (f32 ? &cpg::gemm_decode_kernel<__nv_bfloat16, float, 1>
                    : &cpg::gemm_decode_kernel<__nv_bfloat16, __nv_bfloat16, 1>);
  }
  return reinterpret_cast<const void*>(fn);
}

// Plan of the small-M kernel (CPG_SPLIT_K_DECODE).  Tiles: 128 rows of B per CTA.  The K range of
// a tile is split over a cluster of S CTAs, S the largest of 4, 2, 1 that keeps every CTA of the
// grid resident at once (tiles * S <= SMs) and gives every CTA a k-block.  Stages: the deepest
// ring that fits (at most the CTA's k-blocks), and at least enough to hold the reduction's
// receive buffer.  Measured on N = K = 8192 against the CTA-pair form (CPG_DECODE_PAIR=1: 256-row
// tiles, one cta_group::2 MMA per k-step for both CTAs): M = 16 / 64 / 128 28.7 / 32.8 / 36.6 us
// single against 30.7 / 34.8 / 38.2 us paired, on one box in one call.
static int create_decode_plan(const cpg_gemm_config* cfg, const cpg_gemm_problem* prob, int device,
                              const cudaDeviceProp& prop, cpg_gemm** out) {
  if (prob->m < 1 || prob->m > cpg::kDecodeMaxM)
    return fail(CPG_ERR_INVALID_SHAPE, "the small-M kernel takes 1 <= M <= %d, got %lld",
                cpg::kDecodeMaxM, static_cast<long long>(prob->m));
  if (prob->scale_mode != CPG_SCALE_TENSOR || prob->gated || prob->grouped || prob->l > 1)
    return fail(CPG_ERR_UNSUPPORTED,
                "the small-M kernel has no block scales, gating, batches or groups");
  const int64_t bk = cpg::kRowBytes / elem_bytes(prob->dtype_ab);
  const int64_t k_iters = (prob->k + bk - 1) / bk;
  const int64_t sms = prop.multiProcessorCount;
  const int mma_n = static_cast<int>((prob->m + 15) / 16 * 16);
  // Tuning overrides (measurement only): CPG_DECODE_PAIR (1: CTA pairs), CPG_DECODE_SPLITS
  // (1, 2, 4), CPG_DECODE_STAGES (>= 2), CPG_DECODE_SPIN (0: sleeping waits),
  // CPG_DECODE_ROTATE (0: every tile walks its K range from the start).
  const char* env_pair = std::getenv("CPG_DECODE_PAIR");
  const char* env_s = std::getenv("CPG_DECODE_SPLITS");
  const char* env_st = std::getenv("CPG_DECODE_STAGES");
  const int cg = (env_pair != nullptr && std::atoi(env_pair) == 1) ? 2 : 1;
  const int64_t tile_rows = int64_t(cg) * cpg::kDecodeTileN;
  const int64_t tiles = (prob->n + tile_rows - 1) / tile_rows;
  if (tiles > 65535)
    return fail(CPG_ERR_INVALID_SHAPE, "the small-M kernel takes N <= %lld",
                static_cast<long long>(65535 * tile_rows));
  int splits = 1;
  for (int s = cpg::kDecodeMaxSplits; s > 1; s /= 2) {
    if (tiles * cg * s <= sms && k_iters >= s) {
      splits = s;
      break;
    }
  }
  if (env_s != nullptr) {
    const int v = std::atoi(env_s);
    if ((v == 1 || v == 2 || v == 4) && v <= k_iters) splits = v;
  }
  int tmem_cols = 32;
  while (tmem_cols < mma_n) tmem_cols *= 2;
  const int64_t kps = k_iters > 0 ? (k_iters + splits - 1) / splits : 0;
  int stages = 0;
  for (int st = cpg::kDecodeMaxStages; st >= 2; --st) {
    if (static_cast<int64_t>(cpg::decode_layout(st, mma_n, splits, cg).bytes) <=
        static_cast<int64_t>(prop.sharedMemPerBlockOptin)) {
      stages = st;
      break;
    }
  }
  if (stages == 0) return fail(CPG_ERR_SMEM, "the small-M kernel does not fit in shared memory");
  if (kps >= 2 && stages > kps) stages = static_cast<int>(kps);
  if (env_st != nullptr && std::atoi(env_st) >= 2 && std::atoi(env_st) < stages)
    stages = std::atoi(env_st);
  if (stages < 2) stages = 2;
  // The send blocks and the D boxes of the epilogue live in the stages.
  const int out_bytes = elem_bytes(prob->dtype_d);
  while (static_cast<int64_t>(stages) * cpg::decode_layout(stages, mma_n, splits, cg).stage_bytes <
         cpg::decode_layout(stages, mma_n, splits, cg).epi_bytes(out_bytes))
    ++stages;
  const int smem = static_cast<int>(cpg::decode_layout(stages, mma_n, splits, cg).bytes);
  if (smem > static_cast<int>(prop.sharedMemPerBlockOptin))
    return fail(CPG_ERR_SMEM, "the small-M kernel does not fit in shared memory");
  const void* fn = decode_kernel(prob->dtype_ab, prob->dtype_d, cg);
  cudaError_t e = raise_smem_limit(fn, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(small-M kernel smem)");
  int mac = 0;
  {
    cudaLaunchConfig_t lc = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cg * splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.gridDim = dim3(cg * splits, 1, 1);
    lc.blockDim = dim3(cpg::kDecodeThreads, 1, 1);
    lc.dynamicSmemBytes = smem;
    lc.attrs = attr;
    lc.numAttrs = 1;
    e = cudaOccupancyMaxActiveClusters(&mac, fn, &lc);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters(small-M kernel)");
    if (mac <= 0) return fail(CPG_ERR_NO_DEVICE, "the small-M kernel cannot be resident");
  }

  cpg_gemm* g = new cpg_gemm();
  std::memset(static_cast<void*>(g), 0, sizeof(*g));
  g->cfg = *cfg;
  g->prob = *prob;
  g->device = device;
  g->v = Variant{cpg::kDecodeTileN * cg, cg, prob->dtype_ab, prob->dtype_d, CPG_SCALE_TENSOR, fn,
                 nullptr, cpg::kDecodeThreads, cpg::kDecodeEpiWarps};
  g->smem_bytes = smem;
  g->max_active_clusters = mac;
  g->timeout_ns = 10ull * 1000ull * 1000ull * 1000ull;
  const char* env = std::getenv("CPG_WAIT_TIMEOUT_MS");
  if (env != nullptr && std::atoi(env) > 0) g->timeout_ns = uint64_t(std::atoi(env)) * 1000000ull;
  // B streams through once; every cluster re-reads A (a few rows): keep A in L2.
  g->l2_policy_a = 2;
  g->l2_policy_b = 1;
  g->k_iters = static_cast<int32_t>(k_iters);
  g->k_iters_per_split = static_cast<int32_t>(kps);
  g->splits = 1;  // no split-K ranges in the scheduler's sense: the cluster reduces in place
  g->batches = 1;
  g->sched = cpg::sched_params_create(1, static_cast<int32_t>(tiles > 0 ? tiles : 1), 1,
                                      CPG_RASTER_ALONG_N, 1, 1, 1, 0);
  g->grid[0] = cg * splits;
  g->grid[1] = static_cast<int32_t>(tiles > 0 ? tiles : 1);
  g->grid[2] = 1;
  g->cluster[0] = cg * splits;
  g->cluster[1] = 1;
  g->cluster[2] = 1;
  g->decode = 1;
  g->dec_mma_n = mma_n;
  g->dec_tmem_cols = tmem_cols;
  g->dec_kps = static_cast<int32_t>(kps);
  g->dec_splits = splits;
  g->dec_stages = stages;
  g->dec_cg = cg;
  const char* env_spin = std::getenv("CPG_DECODE_SPIN");
  g->dec_spin = env_spin != nullptr ? (std::atoi(env_spin) != 0) : 1;
  const char* env_rot = std::getenv("CPG_DECODE_ROTATE");
  g->dec_rotate = env_rot != nullptr ? (std::atoi(env_rot) != 0) : 1;
  const char* env_pdl = std::getenv("CPG_DECODE_PDL");
  g->dec_pdl = env_pdl != nullptr ? (std::atoi(env_pdl) != 0) : 1;
  const char* env_sta = std::getenv("CPG_DECODE_STASYNC");
  g->dec_st_async = env_sta != nullptr ? (std::atoi(env_sta) != 0) : 0;
  e = cudaMalloc(&g->status_dev, sizeof(int32_t) * 4);
  if (e == cudaSuccess) e = cudaMemset(g->status_dev, 0, sizeof(int32_t) * 4);
  if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
  if (e != cudaSuccess) {
    cpg_gemm_destroy(g);
    return cuda_fail(e, "small-M plan status word");
  }
  *out = g;
  return CPG_OK;
}

static int run_decode(cpg_gemm* g, const void* a, const void* b, void* d, const cpg_epilogue* epi,
                      cudaStream_t st) {
  const cpg_gemm_problem& pr = g->prob;
  if (epi != nullptr && (epi->activation != CPG_ACT_NONE || epi->source != nullptr))
    return fail(CPG_ERR_UNSUPPORTED, "the small-M kernel has no activation and no C source");
  const int eab = elem_bytes(pr.dtype_ab);
  const int bk = cpg::kRowBytes / eab;
  const int ed = elem_bytes(pr.dtype_d);
  if (!g->maps_valid || g->map_a_ptr != a || g->map_b_ptr != b || g->map_d_ptr != d) {
    // Each CTA loads its 128 rows of B and (pairs) half of the token rows of A.
    int rc = encode_tiled(&g->tm_a, tma_dtype(pr.dtype_ab), eab, a, pr.m, pr.k, pr.lda,
                          g->dec_mma_n / g->dec_cg, bk);
    if (rc != CPG_OK) return rc;
    rc = encode_tiled(&g->tm_b, tma_dtype(pr.dtype_ab), eab, b, pr.n, pr.k, pr.ldb,
                      cpg::kDecodeTileN, bk);
    if (rc != CPG_OK) return rc;
    // D is written in boxes of 16 token rows x 32 columns (rows of D^T of one TMEM lane
    // quadrant), staged unswizzled in shared memory; rows past M and columns past N are clipped.
    rc = encode_tiled(&g->tm_d, tma_dtype(pr.dtype_d), ed, d, pr.m, pr.n, pr.ldd, 16, 32, 1, 0,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc != CPG_OK) return rc;
    g->map_a_ptr = a;
    g->map_b_ptr = b;
    g->map_d_ptr = d;
    g->maps_valid = true;
  }
  cpg::DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  p.m = static_cast<int32_t>(pr.m);
  p.n = static_cast<int32_t>(pr.n);
  p.k = static_cast<int32_t>(pr.k);
  p.mma_n = g->dec_mma_n;
  p.tmem_cols = g->dec_tmem_cols;
  p.k_iters = g->k_iters;
  p.kps = g->dec_kps;
  p.splits = g->dec_splits;
  p.spin = g->dec_spin;
  p.rotate = g->dec_rotate;
  p.pdl = g->dec_pdl;
  p.st_async = g->dec_st_async;
  p.stages = g->dec_stages;
  p.alpha = epi != nullptr ? epi->alpha : 1.0f;
  p.scale_a = epi != nullptr ? epi->scale_a : nullptr;
  p.scale_b = epi != nullptr ? epi->scale_b : nullptr;
  p.bias = epi != nullptr ? static_cast<const __nv_bfloat16*>(epi->bias) : nullptr;
  p.d = d;
  p.ldd = pr.ldd;
  p.status = g->status_dev;
  p.timeout_ns = g->timeout_ns;
  p.l2_policy_a = g->l2_policy_a;
  p.l2_policy_b = g->l2_policy_b;
  cudaLaunchConfig_t lc = {};
  cudaLaunchAttribute attr[2];
  lc.gridDim = dim3(g->grid[0], g->grid[1], 1);
  lc.blockDim = dim3(cpg::kDecodeThreads, 1, 1);
  lc.dynamicSmemBytes = g->smem_bytes;
  lc.stream = st;
  lc.attrs = attr;
  lc.numAttrs = 0;
  if (g->dec_splits * g->dec_cg > 1) {
    attr[lc.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[lc.numAttrs].val.clusterDim.x = g->dec_splits * g->dec_cg;
    attr[lc.numAttrs].val.clusterDim.y = 1;
    attr[lc.numAttrs].val.clusterDim.z = 1;
    ++lc.numAttrs;
  }
  if (g->dec_pdl) {
    // The kernel may start while the stream's previous kernel finishes: it sets up (barriers,
    // TMEM, an L2 prefetch of its first tiles of B) and then waits for that kernel to complete
    // before it touches any other global memory.
    attr[lc.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[lc.numAttrs].val.programmaticStreamSerializationAllowed = 1;
    ++lc.numAttrs;
  }
  void* args[] = {&g->tm_a, &g->tm_b, &g->tm_d, &p};
  cudaError_t e = cudaLaunchKernelExC(&lc, g->v.fn, args);
  return e == cudaSuccess ? CPG_OK : cuda_fail(e, "small-M kernel launch");
}

int cpg_gemm_create(const cpg_gemm_config* cfg, const cpg_gemm_problem* prob, int device,
                    cpg_gemm** out) {
  if (cfg == nullptr || prob == nullptr || out == nullptr)
    return fail(CPG_ERR_NULL, "cfg, prob and out must be non-NULL");
  *out = nullptr;
  int rc = cpg_config_validate(cfg);
  if (rc != CPG_OK) return rc;

  // What this sm_100a build implements.
  if (cfg->tile_m != 128)
    return fail(CPG_ERR_UNSUPPORTED, "tile_m must be 128 (one TMEM lane per row), got %d",
                cfg->tile_m);
  if (cfg->tile_n != 64 && cfg->tile_n != 128 && cfg->tile_n != 256 && cfg->tile_n != 512)
    return fail(CPG_ERR_UNSUPPORTED, "tile_n must be 64, 128, 256 or 512, got %d", cfg->tile_n);
  if (cfg->cluster_m > 2 || cfg->cluster_n > 2)
    return fail(CPG_ERR_UNSUPPORTED, "cluster_shape_mnk must be within (2, 2, 1)");
  if (cfg->tile_m % cfg->epi_tile_m != 0 || cfg->tile_n % cfg->epi_tile_n != 0)
    return fail(CPG_ERR_UNSUPPORTED, "epi_tile_mn must divide tile_shape_mn");
  if (cfg->ab_stage > cpg::kMaxStages)
    return fail(CPG_ERR_SMEM, "ab_stage %d exceeds %d", cfg->ab_stage, cpg::kMaxStages);
  if (cfg->epi_stage > cpg::kMaxEpiStages)
    return fail(CPG_ERR_UNSUPPORTED, "epi_stage %d exceeds %d", cfg->epi_stage,
                cpg::kMaxEpiStages);
  if (cfg->gemm_n_prologue >= cfg->ab_stage)
    return fail(CPG_ERR_INVALID_CONFIG, "gemm_n_prologue must be below ab_stage");

  // Problem checks.
  if (prob->dtype_ab != CPG_DTYPE_BF16 && prob->dtype_ab != CPG_DTYPE_E4M3)
    return fail(CPG_ERR_DTYPE, "A and B must be BF16 or FP8 E4M3");
  if (prob->dtype_d != CPG_DTYPE_BF16 && prob->dtype_d != CPG_DTYPE_F32)
    return fail(CPG_ERR_DTYPE, "D must be BF16 or FP32");
  const int64_t lim = (int64_t(1) << 31) - 1;
  if (prob->m < 0 || prob->n < 0 || prob->k < 0 || prob->m > lim || prob->n > lim || prob->k > lim)
    return fail(CPG_ERR_INVALID_SHAPE, "M, N, K must be in [0, 2^31)");
  if (prob->lda < prob->k || prob->ldb < prob->k || prob->ldd < prob->n)
    return fail(CPG_ERR_INVALID_SHAPE, "row strides must be at least the row length");
  {
    const int eab = elem_bytes(prob->dtype_ab), ed = elem_bytes(prob->dtype_d);
    if ((prob->lda * eab) % 16 != 0 || (prob->ldb * eab) % 16 != 0 || (prob->ldd * ed) % 16 != 0)
      return fail(CPG_ERR_ALIGNMENT, "row strides must be multiples of 16 bytes");
  }

  DeviceGuard guard(device);
  if (!guard.ok) return fail(CPG_ERR_NO_DEVICE, "cannot select device %d", device);
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(CPG_ERR_NO_DEVICE, "device %d is sm_%d%d; this build targets sm_100a", device,
                prop.major, prop.minor);
  if (prob->split_k == CPG_SPLIT_K_DECODE) return create_decode_plan(cfg, prob, device, prop, out);

  Variant v;
  const int cta_group = cfg->cluster_m == 2 ? 2 : 1;
  if (prob->scale_mode != CPG_SCALE_TENSOR && prob->scale_mode != CPG_SCALE_BLOCK)
    return fail(CPG_ERR_INVALID_CONFIG, "scale_mode must be 0 (none / per tensor) or 1 (block)");
  if (prob->scale_mode == CPG_SCALE_BLOCK &&
      (prob->dtype_ab != CPG_DTYPE_E4M3 || prob->dtype_d != CPG_DTYPE_BF16 ||
       (cfg->tile_n != 128 && cfg->tile_n != 256)))
    return fail(CPG_ERR_UNSUPPORTED,
                "block scales need E4M3 operands, BF16 output and tile_n 128 or 256");
  if (!find_variant(cfg->tile_n, cta_group, prob->dtype_ab, prob->dtype_d, prob->scale_mode, &v))
    return fail(CPG_ERR_UNSUPPORTED, "no kernel for tile_n %d, cta_group %d, dtypes %d/%d",
                cfg->tile_n, cta_group, prob->dtype_ab, prob->dtype_d);
  if (v.scale_mode == CPG_SCALE_BLOCK && cfg->reuse_ab)
    return fail(CPG_ERR_UNSUPPORTED, "reuse_ab is not implemented for block-scaled FP8");
  if (prob->split_k < CPG_SPLIT_K_HYBRID)
    return fail(CPG_ERR_INVALID_SHAPE,
                "split_k must be >= 0, CPG_SPLIT_K_STREAM, CPG_SPLIT_K_HYBRID or "
                "CPG_SPLIT_K_DECODE");
  const bool sk_any = prob->split_k == CPG_SPLIT_K_STREAM || prob->split_k == CPG_SPLIT_K_HYBRID;
  if (prob->split_k > 1 &&
      (prob->dtype_d != CPG_DTYPE_F32 || v.scale_mode != CPG_SCALE_TENSOR))
    return fail(CPG_ERR_UNSUPPORTED, "split-K ranges accumulate into an FP32 D (no block scales)");
  if (sk_any && v.scale_mode != CPG_SCALE_TENSOR)
    return fail(CPG_ERR_UNSUPPORTED, "Stream-K is not available with block scales");
  if (cfg->dynamic_scheduler && sk_any)
    return fail(CPG_ERR_UNSUPPORTED, "the dynamic scheduler is not available with Stream-K");
  if (sk_any && !cfg->is_persistent)
    return fail(CPG_ERR_UNSUPPORTED, "Stream-K needs a persistent kernel");
  if (prob->gated != 0 && prob->gated != 1)
    return fail(CPG_ERR_INVALID_CONFIG, "gated must be 0 or 1, got %d", prob->gated);
  if (prob->gated && (cfg->tile_n != 512 || v.scale_mode != CPG_SCALE_TENSOR ||
                      prob->split_k > 1 || sk_any))
    return fail(CPG_ERR_UNSUPPORTED,
                "gated GEMM needs tile_n 512 (256 gate + 256 up columns), no block scales and "
                "no split-K");
  if (prob->gated && prob->n > (int64_t(1) << 30))
    return fail(CPG_ERR_INVALID_SHAPE, "gated GEMM: 2 N must fit in 31 bits");
  if (prob->l < 0) return fail(CPG_ERR_INVALID_SHAPE, "l (batches) must be >= 0");
  if (prob->grouped != 0 && prob->grouped != 1)
    return fail(CPG_ERR_INVALID_CONFIG, "grouped must be 0 or 1, got %d", prob->grouped);
  const int64_t groups = prob->grouped ? prob->l : 0;
  if (prob->grouped) {
    if (groups < 1 || groups > (int64_t(1) << 20))
      return fail(CPG_ERR_INVALID_SHAPE, "a grouped GEMM needs 1 <= l (groups) <= 2^20");
    if (!cfg->is_persistent)
      return fail(CPG_ERR_UNSUPPORTED, "a grouped GEMM needs a persistent kernel");
    if (prob->split_k > 1 || sk_any || v.scale_mode != CPG_SCALE_TENSOR)
      return fail(CPG_ERR_UNSUPPORTED, "grouped GEMM: no split-K and no block scales");
    if (prob->k == 0) return fail(CPG_ERR_UNSUPPORTED, "grouped GEMM: K must be > 0");
    if ((prob->batch_stride_b * elem_bytes(prob->dtype_ab)) % 16 != 0 || prob->batch_stride_b < 0)
      return fail(CPG_ERR_ALIGNMENT, "batch_stride_b must be a multiple of 16 bytes");
  }
  const int64_t batches = (!prob->grouped && prob->l > 1) ? prob->l : 1;
  if (batches > 1) {
    if (v.scale_mode == CPG_SCALE_BLOCK)
      return fail(CPG_ERR_UNSUPPORTED, "batched block-scaled FP8 is not implemented");
    const int eab = elem_bytes(prob->dtype_ab), ed = elem_bytes(prob->dtype_d);
    if (batches > 65535) return fail(CPG_ERR_INVALID_SHAPE, "at most 65535 batches");
    if ((prob->batch_stride_a * eab) % 16 != 0 || (prob->batch_stride_b * eab) % 16 != 0 ||
        (prob->batch_stride_d * ed) % 16 != 0 || prob->batch_stride_a < 0 ||
        prob->batch_stride_b < 0)
      return fail(CPG_ERR_ALIGNMENT, "batch strides must be multiples of 16 bytes");
    if (prob->batch_stride_d < prob->m * prob->ldd)
      return fail(CPG_ERR_INVALID_SHAPE, "batches of D overlap: batch_stride_d %lld < m * ldd",
                  static_cast<long long>(prob->batch_stride_d));
  }
  const int smem = v.smem_bytes(cfg->ab_stage, cfg->epi_stage, cfg->reuse_ab);
  if (smem > static_cast<int>(prop.sharedMemPerBlockOptin))
    return fail(CPG_ERR_SMEM, "%d stages need %d bytes of shared memory, device allows %d",
                cfg->ab_stage, smem, static_cast<int>(prop.sharedMemPerBlockOptin));
  int mac = 0;
  rc = query_max_active_clusters(v, smem, cfg->cluster_m, cfg->cluster_n, &mac);
  if (rc != CPG_OK) return rc;
  if (mac <= 0) return fail(CPG_ERR_NO_DEVICE, "kernel cannot be resident (occupancy 0)");

  cpg_gemm* g = new cpg_gemm();
  std::memset(static_cast<void*>(g), 0, sizeof(*g));
  g->cfg = *cfg;
  g->prob = *prob;
  g->device = device;
  g->v = v;
  g->smem_bytes = smem;
  g->max_active_clusters = mac;
  g->timeout_ns = 10ull * 1000ull * 1000ull * 1000ull;
  const char* env = std::getenv("CPG_WAIT_TIMEOUT_MS");
  if (env != nullptr && std::atoi(env) > 0) g->timeout_ns = uint64_t(std::atoi(env)) * 1000000ull;
  // L2 eviction priority of the A / B tile loads (0 normal, 1 evict-first, 2 evict-last).  The
  // grouped raster walks the slow dimension inside a group of `group_size` cluster columns
  // (AlongN) or rows (AlongM): the operand of the group's columns / rows is re-read by every
  // tile of the group and is kept (evict-last), the other one streams (evict-first).  Measured
  // on 8192^3 BF16: +2-3% over the default priority.  CPG_L2_POLICY_A / _B override.
  g->l2_policy_a = cfg->raster_order == CPG_RASTER_ALONG_N ? 1 : 2;
  g->l2_policy_b = cfg->raster_order == CPG_RASTER_ALONG_N ? 2 : 1;
  {
    // Shapes with one or two row (column) tiles re-read A (B) for every tile along the other
    // dimension while the other operand streams once: keep that one.  Decode-like M = 128,
    // N = K = 8192: 44.1 -> 37.2 us per step.
    const int64_t row_tiles = (prob->m + 128 * cfg->cluster_m - 1) / (128 * cfg->cluster_m);
    const int64_t tile_out = prob->gated ? cfg->tile_n / 2 : cfg->tile_n;
    const int64_t col_tiles = (prob->n + tile_out - 1) / tile_out;
    if (row_tiles <= 2 && col_tiles > 2) {
      g->l2_policy_a = 2;
      g->l2_policy_b = 1;
    } else if (col_tiles <= 2 && row_tiles > 2) {
      g->l2_policy_a = 1;
      g->l2_policy_b = 2;
    }
  }
  // D tiles are written once and never read back by the kernel.
  g->l2_policy_d = 1;
  const char* pa = std::getenv("CPG_L2_POLICY_A");
  const char* pb = std::getenv("CPG_L2_POLICY_B");
  const char* pd = std::getenv("CPG_L2_POLICY_D");
  if (pa != nullptr) g->l2_policy_a = std::atoi(pa);
  if (pb != nullptr) g->l2_policy_b = std::atoi(pb);
  if (pd != nullptr) g->l2_policy_d = std::atoi(pd);

  const int64_t ntm = prob->m > 0 ? (prob->m + 127) / 128 : 1;
  // A gated tile stores 256 output columns (its 512 accumulator columns are gate and up).
  const int64_t tile_out_n = prob->gated ? cfg->tile_n / 2 : cfg->tile_n;
  const int64_t ntn = prob->n > 0 ? (prob->n + tile_out_n - 1) / tile_out_n : 1;
  // Split-K: the L index of the scheduler selects a K range of k_iters_per_split k-blocks;
  // every split is non-empty.
  const int64_t bk = cpg::kRowBytes / elem_bytes(prob->dtype_ab);
  g->k_iters = static_cast<int32_t>((prob->k + bk - 1) / bk);
  g->stream_k = sk_any ? 1 : 0;
  // FP32 Stream-K adds straight into D (after a memset); BF16 Stream-K and the hybrid finish
  // their split tiles in the kernel from an FP32 workspace.
  g->fixup = (prob->split_k == CPG_SPLIT_K_HYBRID ||
              (prob->split_k == CPG_SPLIT_K_STREAM && prob->dtype_d != CPG_DTYPE_F32)) ? 1 : 0;
  int32_t splits = prob->split_k > 1 ? prob->split_k : 1;
  if (splits > g->k_iters && g->k_iters > 0) splits = g->k_iters;
  g->k_iters_per_split = g->k_iters > 0 ? (g->k_iters + splits - 1) / splits : 0;
  g->splits = g->k_iters_per_split > 0
                  ? (g->k_iters + g->k_iters_per_split - 1) / g->k_iters_per_split : 1;
  g->batches = batches;
  g->groups = groups;
  // The scheduler's L index runs over batches x split-K ranges (batch-major).
  const int64_t ntl = int64_t(g->splits) * batches;
  if (ntm * ntn * ntl > (int64_t(1) << 31) - 1) {
    delete g;
    return fail(CPG_ERR_INVALID_SHAPE, "more than 2^31 - 1 tiles");
  }
  g->sched = cpg::sched_params_create(static_cast<int32_t>(ntm), static_cast<int32_t>(ntn),
                                      static_cast<int32_t>(ntl), cfg->raster_order,
                                      plan_group_size(cfg, g->k_iters_per_split),
                                      cfg->cluster_m, cfg->cluster_n, cfg->is_persistent);
  int32_t grid[3];
  cpg::sched_grid_shape(g->sched, mac, grid);
  if (g->stream_k) {
    // Every resident cluster takes an equal share of the k-blocks, even with fewer tiles.
    const int64_t units = int64_t(cpg::sched_total_clusters(g->sched)) * g->k_iters;
    grid[2] = static_cast<int32_t>(units < mac ? (units > 0 ? units : 1) : mac);
  }
  if (groups > 0) {
    // Grouped: at most ceil(m / rows per cluster) + groups cluster rows (each group adds at
    // most one partial row of tiles) times the cluster columns.
    const int64_t rows_per_cluster = 128 * cfg->cluster_m;
    const int64_t ncol = (ntn + cfg->cluster_n - 1) / cfg->cluster_n;
    const int64_t bound = ((prob->m + rows_per_cluster - 1) / rows_per_cluster + groups) * ncol;
    if (bound > (int64_t(1) << 31) - 1) {
      delete g;
      return fail(CPG_ERR_INVALID_SHAPE, "grouped GEMM: more than 2^31 - 1 tiles");
    }
    g->group_n_clusters = static_cast<int32_t>(ncol);
    grid[2] = static_cast<int32_t>(bound < mac ? (bound > 0 ? bound : 1) : mac);
  }
  if (cfg->dynamic_scheduler) {
    // One cluster per cluster tile (the grouped GEMM's bound), along x.
    const int64_t tiles = groups > 0 ? (((prob->m + 128 * cfg->cluster_m - 1) /
                                         (128 * cfg->cluster_m)) + groups) * g->group_n_clusters
                                     : int64_t(cpg::sched_total_clusters(g->sched));
    if (tiles * cfg->cluster_m > (int64_t(1) << 31) - 1) {
      delete g;
      return fail(CPG_ERR_INVALID_SHAPE, "dynamic scheduler: more than 2^31 - 1 CTAs along x");
    }
    grid[0] = static_cast<int32_t>((tiles > 0 ? tiles : 1) * cfg->cluster_m);
    grid[1] = cfg->cluster_n;
    grid[2] = 1;
  }
  for (int i = 0; i < 3; ++i) g->grid[i] = grid[i];
  g->cluster[0] = cfg->cluster_m;
  g->cluster[1] = cfg->cluster_n;
  g->cluster[2] = 1;
  int64_t sk_tiles = 0;
  if (g->fixup) {
    // Hybrid: all full waves but the last are computed whole; the last full wave and the
    // partial one go to Stream-K, so every cluster finishes with about the same work and each
    // split tile has at most two or three contributors.
    const int64_t total = cpg::sched_total_clusters(g->sched);
    const int64_t waves_g = grid[2];
    int64_t dp = 0;
    if (prob->split_k == CPG_SPLIT_K_HYBRID) {
      if (total % waves_g == 0) dp = total;
      else if (total >= 2 * waves_g) dp = (total / waves_g - 1) * waves_g;
    }
    g->dp_tiles = static_cast<int32_t>(dp);
    sk_tiles = total - dp;
  }

  e = cudaMalloc(&g->status_dev, sizeof(int32_t) * 4);
  if (e != cudaSuccess) {
    delete g;
    return cuda_fail(e, "cudaMalloc(status word)");
  }
  e = cudaMemset(g->status_dev, 0, sizeof(int32_t) * 4);
  if (e != cudaSuccess) {
    cudaFree(g->status_dev);
    delete g;
    return cuda_fail(e, "cudaMemset(status word)");
  }
  if (sk_tiles > 0) {
    const int rc2 = alloc_fixup_workspace(g, sk_tiles);
    if (rc2 != CPG_OK) {
      cudaFree(g->status_dev);
      delete g;
      return rc2;
    }
  }
  if (groups > 0) {
    e = cudaMalloc(&g->tile_prefix_dev, sizeof(int32_t) * (groups + 1));
    if (e != cudaSuccess) {
      cudaFree(g->status_dev);
      delete g;
      return cuda_fail(e, "cudaMalloc(group tile prefix)");
    }
  }
  // The zeroing above ran on the legacy default stream, which does not order launches on
  // non-blocking streams: let it finish before the plan is used (once per plan).
  e = cudaStreamSynchronize(nullptr);
  if (e != cudaSuccess) {
    cpg_gemm_destroy(g);
    return cuda_fail(e, "cudaStreamSynchronize(plan setup)");
  }
  *out = g;
  return CPG_OK;
}

int cpg_gemm_destroy(cpg_gemm* g) {
  if (g == nullptr) return CPG_OK;
  if (g->status_dev != nullptr || g->tile_prefix_dev != nullptr || g->ws_dev != nullptr ||
      g->cnt_dev != nullptr) {
    DeviceGuard guard(g->device);
    if (g->status_dev != nullptr) cudaFree(g->status_dev);
    if (g->tile_prefix_dev != nullptr) cudaFree(g->tile_prefix_dev);
    if (g->ws_dev != nullptr) cudaFree(g->ws_dev);
    if (g->cnt_dev != nullptr) cudaFree(g->cnt_dev);
  }
  delete g;
  return CPG_OK;
}

int cpg_gemm_launch_info(const cpg_gemm* g, int32_t grid[3], int32_t cluster[3], int32_t* threads,
                         int32_t* smem_bytes, int32_t* max_active_clusters) {
  if (g == nullptr) return fail(CPG_ERR_NULL, "plan is NULL");
  for (int i = 0; i < 3; ++i) {
    if (grid) grid[i] = g->grid[i];
    if (cluster) cluster[i] = g->cluster[i];
  }
  if (threads) *threads = g->v.threads;
  if (smem_bytes) *smem_bytes = g->smem_bytes;
  if (max_active_clusters) *max_active_clusters = g->max_active_clusters;
  return CPG_OK;
}

int cpg_gemm_sched_params(const cpg_gemm* g, cpg_sched_params* out) {
  if (g == nullptr || out == nullptr) return fail(CPG_ERR_NULL, "plan and out must be non-NULL");
  static_assert(sizeof(cpg_sched_params) == sizeof(cpg::SchedParams), "layout mismatch");
  std::memcpy(out, &g->sched, sizeof(*out));
  return CPG_OK;
}

int cpg_gemm_set_trace(cpg_gemm* g, int32_t* device_buf, int32_t tiles_per_cta) {
  if (g == nullptr) return fail(CPG_ERR_NULL, "plan is NULL");
  if (device_buf != nullptr && tiles_per_cta <= 0)
    return fail(CPG_ERR_INVALID_SHAPE, "tiles_per_cta must be positive");
  g->trace = device_buf;
  g->trace_stride = device_buf != nullptr ? tiles_per_cta : 0;
  return CPG_OK;
}

int cpg_gemm_set_timeout_ms(cpg_gemm* g, int32_t timeout_ms) {
  if (g == nullptr) return fail(CPG_ERR_NULL, "plan is NULL");
  if (timeout_ms <= 0) return fail(CPG_ERR_INVALID_SHAPE, "timeout must be positive");
  g->timeout_ns = uint64_t(timeout_ms) * 1000000ull;
  return CPG_OK;
}

int cpg_gemm_set_fault_injection(cpg_gemm* g, int32_t flags) {
  if (g == nullptr) return fail(CPG_ERR_NULL, "plan is NULL");
  if ((flags & ~CPG_INJECT_SKIP_LOADS) != 0)
    return fail(CPG_ERR_INVALID_CONFIG, "unknown fault-injection flags %d", flags);
  g->fault_inject = flags;
  return CPG_OK;
}

int cpg_gemm_status(cpg_gemm* g, int32_t* status) {
  if (g == nullptr || status == nullptr) return fail(CPG_ERR_NULL, "plan and status non-NULL");
  DeviceGuard guard(g->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int32_t s = 0;
  e = cudaMemcpy(&s, g->status_dev, sizeof(s), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status)");
  *status = s;
  if (s != 0) {
    cudaMemset(g->status_dev, 0, sizeof(int32_t));
    // A launch that stopped early may have left Stream-K workspace tiles and counts behind.
    if (g->ws_dev != nullptr) cudaMemset(g->ws_dev, 0, g->ws_bytes);
    if (g->cnt_dev != nullptr) cudaMemset(g->cnt_dev, 0, g->cnt_bytes);
    cudaDeviceSynchronize();  // the clears land before any later launch, on any stream
    if (s == kStatusBadGroups)
      return fail(CPG_ERR_INVALID_SHAPE, "group offsets not non-decreasing within [0, m]");
    return fail(CPG_ERR_DEVICE_TIMEOUT, "kernel wait timed out at site %d", s & 0xFF);
  }
  return CPG_OK;
}

static int run_impl(cpg_gemm* g, const void* a, const void* b, void* d, const cpg_epilogue* epi,
                    void* stream, const int32_t* group_offsets,
                    const cpg_reduce_scatter* rs = nullptr);

int cpg_gemm_run(cpg_gemm* g, const void* a, const void* b, void* d, const cpg_epilogue* epi,
                 void* stream) {
  if (g == nullptr) return fail(CPG_ERR_NULL, "plan is NULL");
  if (g->groups > 0)
    return fail(CPG_ERR_INVALID_CONFIG, "grouped plan: launch it with cpg_gemm_run_grouped");
  return run_impl(g, a, b, d, epi, stream, nullptr);
}

int cpg_gemm_run_grouped(cpg_gemm* g, const void* a, const void* b, void* d,
                         const int32_t* group_offsets, const cpg_epilogue* epi, void* stream) {
  if (g == nullptr) return fail(CPG_ERR_NULL, "plan is NULL");
  if (g->groups == 0)
    return fail(CPG_ERR_INVALID_CONFIG, "plan is not grouped (create it with prob->grouped = 1)");
  if (group_offsets == nullptr) return fail(CPG_ERR_NULL, "group_offsets is NULL");
  if ((reinterpret_cast<uintptr_t>(group_offsets) & 3u) != 0)
    return fail(CPG_ERR_ALIGNMENT, "group_offsets must be 4-byte aligned");
  return run_impl(g, a, b, d, epi, stream, group_offsets);
}

static int run_impl(cpg_gemm* g, const void* a, const void* b, void* d, const cpg_epilogue* epi,
                    void* stream, const int32_t* group_offsets, const cpg_reduce_scatter* rs) {
  const cpg_gemm_problem& pr = g->prob;
  if (pr.m == 0 || pr.n == 0) return CPG_OK;
  if (d == nullptr) return fail(CPG_ERR_NULL, "D is NULL");
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != g->device)
    return fail(CPG_ERR_NO_DEVICE, "current device %d differs from the plan's device %d", cur,
                g->device);
  const void* bias = epi != nullptr ? epi->bias : nullptr;
  const float alpha = epi != nullptr ? epi->alpha : 1.0f;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if ((reinterpret_cast<uintptr_t>(d) & 15u) != 0)
    return fail(CPG_ERR_ALIGNMENT, "D must be 16-byte aligned");
  if (bias != nullptr && (reinterpret_cast<uintptr_t>(bias) & 1u) != 0)
    return fail(CPG_ERR_ALIGNMENT, "bias must be 2-byte aligned");
  const int32_t act = epi != nullptr ? epi->activation : CPG_ACT_NONE;
  const void* src = epi != nullptr ? epi->source : nullptr;
  if (act < CPG_ACT_NONE || act > CPG_ACT_GELU_TANH)
    return fail(CPG_ERR_INVALID_CONFIG, "activation %d is not one of CPG_ACT_*", act);
  if ((act != CPG_ACT_NONE || src != nullptr) && (g->splits > 1 || g->stream_k))
    return fail(CPG_ERR_UNSUPPORTED,
                "activations and a C source need the whole K in one pass (no split-K)");
  if (g->v.scale_mode == CPG_SCALE_BLOCK && (act != CPG_ACT_NONE || src != nullptr))
    return fail(CPG_ERR_UNSUPPORTED, "the block-scaled FP8 kernel has no activation or C source");
  if (pr.gated && (bias != nullptr || src != nullptr))
    return fail(CPG_ERR_UNSUPPORTED, "gated GEMM takes no bias and no C source");
  if (src != nullptr) {
    const int es = elem_bytes(pr.dtype_d);
    if (epi->ld_source < pr.n || (epi->ld_source * es) % 16 != 0)
      return fail(CPG_ERR_ALIGNMENT, "C row stride %lld must be >= N and a multiple of 16 bytes",
                  static_cast<long long>(epi->ld_source));
    if (g->batches > 1 && (epi->batch_stride_source * es) % 16 != 0)
      return fail(CPG_ERR_ALIGNMENT, "C batch stride must be a multiple of 16 bytes");
    if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0)
      return fail(CPG_ERR_ALIGNMENT, "C must be 16-byte aligned");
  }

  if (pr.k == 0) {
    if (act != CPG_ACT_NONE || src != nullptr)
      return fail(CPG_ERR_UNSUPPORTED, "K = 0 with an activation or a C source");
    // D = bias (or 0): nothing to contract.
    int blocks = static_cast<int>((pr.m * pr.n + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    const int ed0 = elem_bytes(pr.dtype_d);
    for (int64_t bt = 0; bt < g->batches; ++bt) {
      void* db = static_cast<char*>(d) + bt * pr.batch_stride_d * ed0;
      if (pr.dtype_d == CPG_DTYPE_F32) {
        fill_rows_kernel<float><<<blocks, 256, 0, st>>>(static_cast<float*>(db), pr.m, pr.n,
                                                        pr.ldd,
                                                        static_cast<const __nv_bfloat16*>(bias));
      } else {
        fill_rows_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
            static_cast<__nv_bfloat16*>(db), pr.m, pr.n, pr.ldd,
            static_cast<const __nv_bfloat16*>(bias));
      }
    }
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CPG_OK : cuda_fail(e, "fill kernel launch");
  }
  if (a == nullptr || b == nullptr) return fail(CPG_ERR_NULL, "A and B must be non-NULL");
  if ((reinterpret_cast<uintptr_t>(a) & 15u) != 0 || (reinterpret_cast<uintptr_t>(b) & 15u) != 0)
    return fail(CPG_ERR_ALIGNMENT, "A and B must be 16-byte aligned");
  if (g->decode) {
    if (rs != nullptr) return fail(CPG_ERR_UNSUPPORTED, "a small-M plan has no peer exchange");
    return run_decode(g, a, b, d, epi, st);
  }

  const int eab = elem_bytes(pr.dtype_ab), ed = elem_bytes(pr.dtype_d);
  const int bk = cpg::kRowBytes / eab;         // k-block: one 128-byte row of A / B
  const int store_cols = cpg::kRowBytes / ed;  // epilogue box: one 128-byte row of D
  if (!g->maps_valid || g->map_a_ptr != a || g->map_b_ptr != b || g->map_d_ptr != d) {
    int rc = encode_tiled(&g->tm_a, tma_dtype(pr.dtype_ab), eab, a, pr.m, pr.k, pr.lda, cpg::kBM,
                          bk, g->batches, pr.batch_stride_a);
    if (rc != CPG_OK) return rc;
    // One B box per MMA: min(tile_n, 256) / cta_group rows; a gated B holds 2 N rows; a
    // grouped B has one batch per group.
    rc = encode_tiled(&g->tm_b, tma_dtype(pr.dtype_ab), eab, b, pr.gated ? 2 * pr.n : pr.n, pr.k,
                      pr.ldb, (g->v.bn > 256 ? 256 : g->v.bn) / g->v.cta_group, bk,
                      g->groups > 0 ? g->groups : g->batches, pr.batch_stride_b);
    if (rc != CPG_OK) return rc;
    rc = encode_tiled(&g->tm_d, tma_dtype(pr.dtype_d), ed, d, pr.m, pr.n, pr.ldd, 32, store_cols,
                      g->batches, pr.batch_stride_d);
    if (rc != CPG_OK) return rc;
    g->map_a_ptr = a;
    g->map_b_ptr = b;
    g->map_d_ptr = d;
    g->maps_valid = true;
  }

  cpg::GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.sched = g->sched;
  p.m = static_cast<int32_t>(pr.m);
  p.n = static_cast<int32_t>(pr.n);
  p.k = static_cast<int32_t>(pr.k);
  p.k_iters = g->k_iters;
  p.k_iters_per_split = g->k_iters_per_split;
  p.reduce_add = (g->splits > 1 || (g->stream_k && !g->fixup)) ? 1 : 0;
  p.stream_k = g->stream_k;
  p.fixup = g->fixup;
  p.dp_tiles = g->dp_tiles;
  p.fixup_count = g->cnt_dev;
  p.fixup_ws = g->ws_dev;
  p.ws_cols = g->cfg.tile_n;
  p.ab_stages = g->cfg.ab_stage;
  p.epi_stages = g->cfg.epi_stage;
  p.reuse_ab = g->cfg.reuse_ab;
  p.dynamic = g->cfg.dynamic_scheduler;
  p.alpha = alpha;
  const bool block = g->v.scale_mode == CPG_SCALE_BLOCK;
  cpg::BlockScales bs{nullptr, nullptr};
  if (block) {
    if (epi == nullptr || epi->scale_a == nullptr || epi->scale_b == nullptr)
      return fail(CPG_ERR_NULL, "block-scaled FP8 needs scale_a and scale_b");
    bs.sa = epi->scale_a;
    bs.sb = epi->scale_b;
  } else {
    p.scale_a = epi != nullptr ? epi->scale_a : nullptr;
    p.scale_b = epi != nullptr ? epi->scale_b : nullptr;
  }
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.tile_trace = g->trace;
  p.trace_stride = g->trace_stride;
  p.status = g->status_dev;
  p.timeout_ns = g->timeout_ns;
  p.fault_inject = g->fault_inject;
  p.l2_policy_a = g->l2_policy_a;
  p.l2_policy_b = g->l2_policy_b;
  p.l2_policy_d = g->l2_policy_d;
  p.act = act;
  p.beta = epi != nullptr ? epi->beta : 0.f;
  p.src = src;
  p.ld_src = src != nullptr ? epi->ld_source : 0;
  p.src_batch_stride = (src != nullptr && g->batches > 1) ? epi->batch_stride_source : 0;
  p.gated = pr.gated;
  p.num_splits = g->splits;
  p.d = d;
  p.ldd = pr.ldd;
  if (rs != nullptr) {
    // Peer reduce-scatter: the epilogue adds into the owners' buffers (checked by the caller);
    // D is not written, so nothing is cleared here.
    p.reduce_add = 0;
    // K ranges of a tile sum in the plan's workspace first; the last one sends the tile.
    p.fixup = g->splits > 1 ? 1 : 0;
    p.dp_tiles = 0;
    p.rs_ranks = rs->ranks;
    for (int q = 0; q <= rs->ranks; ++q) p.rs_row_start[q] = static_cast<int32_t>(rs->row_start[q]);
    p.rs_ld = rs->ld;
    for (int q = 0; q < rs->ranks; ++q) {
      p.rs_dst[q] = rs->dst[q];
      p.rs_count[q] = rs->count[q];
    }
  }
  if (g->groups > 0) {
    p.num_groups = static_cast<int32_t>(g->groups);
    p.group_offsets = group_offsets;
    p.tile_prefix = g->tile_prefix_dev;
    p.group_n_clusters = g->group_n_clusters;
    group_tile_prefix_kernel<<<1, kPrefixThreads, 0, st>>>(
        group_offsets, p.num_groups, pr.m, 128 * g->cfg.cluster_m, g->group_n_clusters,
        g->tile_prefix_dev, g->status_dev);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "group tile prefix launch");
  }

  if ((g->splits > 1 || (g->stream_k && !g->fixup)) && rs == nullptr) {
    // The splits / Stream-K segments add their partial sums into D.
    for (int64_t bt = 0; bt < g->batches; ++bt) {
      cudaError_t e = cudaMemset2DAsync(static_cast<char*>(d) + bt * pr.batch_stride_d * ed,
                                        pr.ldd * ed, 0, pr.n * ed, pr.m, st);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemset2DAsync(D)");
    }
  }
  cudaLaunchConfig_t lc = {};
  cudaLaunchAttribute attr[1];
  lc.gridDim = dim3(g->grid[0], g->grid[1], g->grid[2]);
  lc.blockDim = dim3(g->v.threads, 1, 1);
  lc.dynamicSmemBytes = g->smem_bytes;
  lc.stream = st;
  lc.numAttrs = 0;
  lc.attrs = attr;
  if (g->cluster[0] * g->cluster[1] > 1) {
    attr[lc.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[lc.numAttrs].val.clusterDim.x = g->cluster[0];
    attr[lc.numAttrs].val.clusterDim.y = g->cluster[1];
    attr[lc.numAttrs].val.clusterDim.z = 1;
    ++lc.numAttrs;
  }

  void* args[] = {&g->tm_a, &g->tm_b, &g->tm_d, &g->tm_ws, &p};
  void* block_args[] = {&g->tm_a, &g->tm_b, &g->tm_d, &p, &bs};
  cudaError_t e = cudaLaunchKernelExC(&lc, g->v.fn, block ? block_args : args);
  if (e != cudaSuccess) return cuda_fail(e, "GEMM kernel launch");
  return CPG_OK;
}

int cpg_fast_divmod_create(int32_t divisor, cpg_fast_divmod* out) {
  if (out == nullptr) return fail(CPG_ERR_NULL, "out is NULL");
  if (divisor < 1) return fail(CPG_ERR_INVALID_SHAPE, "divisor must be >= 1, got %d", divisor);
  cpg::FastDivmod f = cpg::fast_divmod_create(divisor);
  out->divisor = f.divisor;
  out->multiplier = f.multiplier;
  out->shift_right = f.shift_right;
  return CPG_OK;
}

int cpg_fast_divmod_divmod(const cpg_fast_divmod* f, int32_t x, int32_t* q, int32_t* r) {
  if (f == nullptr || q == nullptr || r == nullptr) return fail(CPG_ERR_NULL, "NULL argument");
  cpg::FastDivmod ff{f->divisor, f->multiplier, f->shift_right};
  cpg::fast_divmod(ff, x, *q, *r);
  return CPG_OK;
}

int cpg_fast_divmod_device(const cpg_fast_divmod* f, const int32_t* x, int32_t* q, int32_t* r,
                           int64_t n, void* stream) {
  if (f == nullptr || (n > 0 && (x == nullptr || q == nullptr || r == nullptr)))
    return fail(CPG_ERR_NULL, "NULL argument");
  if (n <= 0) return CPG_OK;
  cpg::FastDivmod ff{f->divisor, f->multiplier, f->shift_right};
  const int threads = 256;
  const int64_t blocks = (n + threads - 1) / threads;
  cpg::fast_divmod_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                            reinterpret_cast<cudaStream_t>(stream)>>>(ff, x, q, r, n);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CPG_OK : cuda_fail(e, "fast_divmod_kernel launch");
}

int cpg_sched_params_create(int32_t ntiles_m, int32_t ntiles_n, int32_t ntiles_l,
                            int32_t raster_order, int32_t group_size, int32_t cluster_m,
                            int32_t cluster_n, int32_t cluster_k, int32_t is_persistent,
                            cpg_sched_params* out) {
  if (out == nullptr) return fail(CPG_ERR_NULL, "out is NULL");
  if (cluster_k != 1) return fail(CPG_ERR_INVALID_CONFIG, "cluster_shape_mnk[2] must be 1");
  if (ntiles_m < 1 || ntiles_n < 1 || ntiles_l < 1 || group_size < 1 || cluster_m < 1 ||
      cluster_n < 1)
    return fail(CPG_ERR_INVALID_SHAPE, "tile counts, group size and cluster dims must be >= 1");
  if (raster_order != CPG_RASTER_ALONG_M && raster_order != CPG_RASTER_ALONG_N)
    return fail(CPG_ERR_INVALID_CONFIG, "raster_order must be 0 or 1");
  cpg::SchedParams p = cpg::sched_params_create(ntiles_m, ntiles_n, ntiles_l, raster_order,
                                                group_size, cluster_m, cluster_n, is_persistent);
  std::memcpy(out, &p, sizeof(*out));
  return CPG_OK;
}

int cpg_sched_plan_group_size(const cpg_gemm_config* cfg, int64_t k, int32_t dtype_ab,
                              int32_t* out) {
  if (cfg == nullptr || out == nullptr) return fail(CPG_ERR_NULL, "NULL argument");
  const int rc = cpg_config_validate(cfg);
  if (rc != CPG_OK) return rc;
  if (dtype_ab != CPG_DTYPE_BF16 && dtype_ab != CPG_DTYPE_E4M3)
    return fail(CPG_ERR_DTYPE, "dtype_ab must be BF16 or E4M3, got %d", dtype_ab);
  if (k < 0) return fail(CPG_ERR_INVALID_SHAPE, "k must be >= 0, got %lld", (long long)k);
  const int64_t bk = cpg::kRowBytes / elem_bytes(dtype_ab);
  *out = plan_group_size(cfg, (k + bk - 1) / bk);
  return CPG_OK;
}

int cpg_sched_grid_shape(const cpg_sched_params* p, int32_t max_active_clusters, int32_t grid[3]) {
  if (p == nullptr || grid == nullptr) return fail(CPG_ERR_NULL, "NULL argument");
  cpg::SchedParams sp;
  std::memcpy(&sp, p, sizeof(sp));
  cpg::sched_grid_shape(sp, max_active_clusters, grid);
  return CPG_OK;
}

int cpg_sched_cluster_map(const cpg_sched_params* p, int32_t* out, int64_t n) {
  if (p == nullptr || (n > 0 && out == nullptr)) return fail(CPG_ERR_NULL, "NULL argument");
  cpg::SchedParams sp;
  std::memcpy(&sp, p, sizeof(sp));
  for (int64_t i = 0; i < n; ++i) {
    int32_t cm, cn;
    cpg::sched_map_cluster(sp, static_cast<int32_t>(i), cm, cn);
    out[2 * i] = cm;
    out[2 * i + 1] = cn;
  }
  return CPG_OK;
}

int cpg_sched_cluster_map_device(const cpg_sched_params* p, int32_t* device_out, int64_t n,
                                 void* stream) {
  if (p == nullptr || (n > 0 && device_out == nullptr)) return fail(CPG_ERR_NULL, "NULL argument");
  if (n <= 0) return CPG_OK;
  cpg::SchedParams sp;
  std::memcpy(&sp, p, sizeof(sp));
  const int threads = 256;
  const int64_t blocks = (n + threads - 1) / threads;
  cpg::sched_cluster_map_kernel<<<static_cast<unsigned>(blocks), threads, 0,
                                  reinterpret_cast<cudaStream_t>(stream)>>>(sp, device_out, n);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CPG_OK : cuda_fail(e, "sched_cluster_map_kernel launch");
}

int cpg_max_active_clusters(int32_t cluster_size, int32_t* out) {
  if (out == nullptr) return fail(CPG_ERR_NULL, "out is NULL");
  if (cluster_size < 1 || cluster_size > 4)
    return fail(CPG_ERR_UNSUPPORTED, "cluster size must be 1..4, got %d", cluster_size);
  Variant v;
  const int cg = (cluster_size % 2 == 0) ? 2 : 1;
  find_variant(256, cg, CPG_DTYPE_BF16, CPG_DTYPE_BF16, CPG_SCALE_TENSOR, &v);
  const int smem = v.smem_bytes(4, 2, 0);
  int cm = cluster_size >= 2 ? 2 : 1;
  int cn = cluster_size == 4 ? 2 : (cluster_size == 3 ? 3 : 1);
  if (cluster_size == 3) cm = 1;
  int n = 0;
  int rc = query_max_active_clusters(v, smem, cm, cn, &n);
  if (rc != CPG_OK) return rc;
  *out = n;
  return CPG_OK;
}

int cpg_quantize_e4m3(const void* x, int32_t dtype_x, int64_t rows, int64_t cols, int64_t ldx,
                      void* q, int64_t ldq, float* scales, int32_t block_rows, int32_t block_cols,
                      void* stream) {
  if (rows < 0 || cols < 0 || ldx < cols || ldq < cols)
    return fail(CPG_ERR_INVALID_SHAPE, "bad quantisation extents");
  if (dtype_x != CPG_DTYPE_BF16 && dtype_x != CPG_DTYPE_F32)
    return fail(CPG_ERR_DTYPE, "x must be BF16 or FP32");
  if (scales == nullptr) return fail(CPG_ERR_NULL, "scales is NULL");
  const bool per_tensor = block_rows == 0 && block_cols == 0;
  const bool row_block = block_rows == 1 && block_cols == 128;
  const bool tile_block = block_rows == 128 && block_cols == 128;
  if (!per_tensor && !row_block && !tile_block)
    return fail(CPG_ERR_UNSUPPORTED, "blocks must be (0,0) per tensor, (1,128) or (128,128)");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (per_tensor) {
    cudaError_t e = cudaMemsetAsync(scales, 0, sizeof(float), st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(scale)");
  }
  if (rows == 0 || cols == 0) {
    if (per_tensor) cpg::finalize_scale_kernel<<<1, 1, 0, st>>>(reinterpret_cast<unsigned*>(scales));
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CPG_OK : cuda_fail(e, "quantize launch");
  }
  if (x == nullptr || q == nullptr) return fail(CPG_ERR_NULL, "x and q must be non-NULL");
  uint8_t* qq = static_cast<uint8_t*>(q);
  const int threads = 256;
  const unsigned row_blocks = static_cast<unsigned>(rows < 65535 ? rows : 65535);
  auto launch = [&](auto tag) {
    using T = decltype(tag);
    const T* xx = static_cast<const T*>(x);
    if (per_tensor) {
      unsigned* amax = reinterpret_cast<unsigned*>(scales);
      // Whole 16-byte vectors per row (x rows 16-byte aligned, q rows aligned to a vector's
      // E4M3 bytes): the vectorised kernels; otherwise the element kernels.
      constexpr int V = cpg::Vec16<T>::kElems;
      const bool vec = cols % V == 0 && ldx % V == 0 && ldq % V == 0 &&
                       (reinterpret_cast<uintptr_t>(xx) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(qq) & static_cast<uintptr_t>(V - 1)) == 0;
      if (vec) {
        cpg::amax_vec_kernel<T><<<row_blocks, threads, 0, st>>>(xx, rows, cols, ldx, amax);
        cpg::quant_per_tensor_vec_kernel<T><<<row_blocks, threads, 0, st>>>(xx, rows, cols, ldx,
                                                                             qq, ldq, amax);
      } else {
        cpg::amax_kernel<T><<<row_blocks, threads, 0, st>>>(xx, rows, cols, ldx, amax);
        cpg::quant_per_tensor_kernel<T><<<row_blocks, threads, 0, st>>>(xx, rows, cols, ldx, qq,
                                                                         ldq, amax);
      }
      cpg::finalize_scale_kernel<<<1, 1, 0, st>>>(amax);
    } else if (row_block) {
      const int64_t warps = rows * ((cols + 127) / 128);
      const int64_t blocks = (warps * 32 + threads - 1) / threads;
      // 16-byte loads of x and V-byte stores of q: row starts aligned to V elements of both.
      constexpr int V = cpg::Vec16<T>::kElems;
      const bool vec = ldx % V == 0 && ldq % V == 0 &&
                       (reinterpret_cast<uintptr_t>(xx) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(qq) & static_cast<uintptr_t>(V - 1)) == 0;
      if (vec) {
        constexpr int kPerWarp = cpg::row_blocks_per_warp<T>();
        const int64_t groups = (((cols + 127) / 128) + kPerWarp - 1) / kPerWarp;
        const int64_t vblocks = (rows * groups * 32 + threads - 1) / threads;
        cpg::quant_row_block_vec_kernel<T><<<static_cast<unsigned>(vblocks), threads, 0, st>>>(
            xx, rows, cols, ldx, qq, ldq, scales);
      } else {
        cpg::quant_row_block_kernel<T><<<static_cast<unsigned>(blocks), threads, 0, st>>>(
            xx, rows, cols, ldx, qq, ldq, scales);
      }
    } else {
      const int64_t blocks = ((rows + 127) / 128) * ((cols + 127) / 128);
      constexpr int V = cpg::Vec16<T>::kElems;
      const bool vec = ldx % V == 0 && ldq % V == 0 &&
                       (reinterpret_cast<uintptr_t>(xx) & 15u) == 0 &&
                       (reinterpret_cast<uintptr_t>(qq) & static_cast<uintptr_t>(V - 1)) == 0;
      if (vec) {
        cpg::quant_tile_block_vec_kernel<T>
            <<<static_cast<unsigned>(blocks), cpg::kTileBlockThreads, 0, st>>>(
            xx, rows, cols, ldx, qq, ldq, scales);
      } else {
        cpg::quant_tile_block_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
            xx, rows, cols, ldx, qq, ldq, scales);
      }
    }
  };
  if (dtype_x == CPG_DTYPE_BF16) {
    launch(__nv_bfloat16{});
  } else {
    launch(float{});
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CPG_OK : cuda_fail(e, "quantize launch");
}

// ------------------------------------------------------------ reduce-scatter over peer memory
static_assert(sizeof(cpg_ipc_handle) == sizeof(cudaIpcMemHandle_t), "IPC handle size");
static_assert(CPG_MAX_PEERS == cpg::kMaxPeers, "peer count");

int cpg_peer_alloc(int64_t bytes, void** dev_ptr, cpg_ipc_handle* handle) {
  if (dev_ptr == nullptr || handle == nullptr) return fail(CPG_ERR_NULL, "NULL argument");
  *dev_ptr = nullptr;
  if (bytes <= 0) return fail(CPG_ERR_INVALID_SHAPE, "bytes must be positive");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(peer buffer)");
  e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  // cudaMemset of device memory may return before the zeros land; other processes write into
  // this buffer as soon as they hold its handle, so the zeros must be in place first.
  if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "peer buffer setup");
  }
  std::memcpy(handle->bytes, &h, sizeof(h));
  *dev_ptr = p;
  return CPG_OK;
}

int cpg_peer_open(const cpg_ipc_handle* handle, void** dev_ptr) {
  if (handle == nullptr || dev_ptr == nullptr) return fail(CPG_ERR_NULL, "NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *dev_ptr = p;
  return CPG_OK;
}

int cpg_peer_close(void* dev_ptr) {
  if (dev_ptr == nullptr) return CPG_OK;
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? CPG_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int cpg_peer_free(void* dev_ptr) {
  if (dev_ptr == nullptr) return CPG_OK;
  cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? CPG_OK : cuda_fail(e, "cudaFree(peer buffer)");
}

static int check_reduce_scatter(const cpg_gemm* g, const cpg_reduce_scatter* rs) {
  if (g == nullptr || rs == nullptr) return fail(CPG_ERR_NULL, "plan and rs must be non-NULL");
  const cpg_gemm_problem& pr = g->prob;
  if (pr.dtype_d != CPG_DTYPE_F32 || g->stream_k || g->groups > 0 || g->batches > 1 ||
      pr.gated || g->v.scale_mode != CPG_SCALE_TENSOR || g->decode)
    return fail(CPG_ERR_UNSUPPORTED,
                "the peer reduce-scatter needs an FP32-output plan without Stream-K, batches, "
                "groups, gating or block scales");
  if (rs->ranks < 1 || rs->ranks > CPG_MAX_PEERS || rs->rank < 0 || rs->rank >= rs->ranks)
    return fail(CPG_ERR_INVALID_CONFIG, "rank %d of %d ranks (at most %d)", rs->rank, rs->ranks,
                CPG_MAX_PEERS);
  if (rs->row_start[0] != 0 || rs->row_start[rs->ranks] != pr.m)
    return fail(CPG_ERR_INVALID_SHAPE, "row_start must run from 0 to M = %lld",
                static_cast<long long>(pr.m));
  for (int q = 0; q < rs->ranks; ++q) {
    if (rs->row_start[q + 1] < rs->row_start[q])
      return fail(CPG_ERR_INVALID_SHAPE, "row_start must not decrease");
    if (q > 0 && rs->row_start[q] != pr.m && rs->row_start[q] % cpg::kBM != 0)
      return fail(CPG_ERR_ALIGNMENT, "row blocks must start on 128-row tiles (or at M)");
    if (rs->dst[q] == nullptr || rs->count[q] == nullptr)
      return fail(CPG_ERR_NULL, "dst[%d] and count[%d] must be non-NULL", q, q);
    if ((reinterpret_cast<uintptr_t>(rs->dst[q]) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(rs->count[q]) & 3u) != 0)
      return fail(CPG_ERR_ALIGNMENT, "dst 16-byte and count 4-byte aligned");
  }
  if (pr.n % 4 != 0 || rs->ld < pr.n || rs->ld % 4 != 0)
    return fail(CPG_ERR_ALIGNMENT, "N and ld must be multiples of 4 (16-byte atomics), ld >= N");
  return CPG_OK;
}

// One arrival of a reduce-scatter call on every rank's counter, after the call's GEMM (and so
// after this rank's previous cpg_peer_finish, in stream order).  A rank that owns no rows gets no
// tile arrivals: without this its finish would return at once and its next-but-one call could add
// into an owner's buffer before the owner had read and cleared it.  With it, every finish waits
// until every rank has completed its previous finish.
struct EpochCounters {
  uint32_t* count[CPG_MAX_PEERS];
  int32_t ranks;
};
__global__ void rs_epoch_kernel(const EpochCounters c) {
  if (static_cast<int32_t>(threadIdx.x) < c.ranks) {
    cpg::ptx::fence_sc_sys();
    cpg::ptx::red_release_sys_add_u32(c.count[threadIdx.x], 1u);
  }
}

static int rs_epoch(const cpg_reduce_scatter* rs, cudaStream_t st) {
  EpochCounters c;
  std::memset(&c, 0, sizeof(c));
  c.ranks = rs->ranks;
  for (int q = 0; q < rs->ranks; ++q) c.count[q] = static_cast<uint32_t*>(rs->count[q]);
  rs_epoch_kernel<<<1, 32, 0, st>>>(c);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CPG_OK : cuda_fail(e, "reduce-scatter epoch kernel launch");
}

int cpg_gemm_run_reduce_scatter(cpg_gemm* g, const void* a, const void* b,
                                const cpg_reduce_scatter* rs, const cpg_epilogue* epi,
                                void* stream) {
  int rc = check_reduce_scatter(g, rs);
  if (rc != CPG_OK) return rc;
  const cpg_gemm_problem& pr = g->prob;
  if (epi != nullptr &&
      (epi->bias != nullptr || epi->activation != CPG_ACT_NONE || epi->source != nullptr))
    return fail(CPG_ERR_UNSUPPORTED, "bias, activations and C belong to cpg_peer_finish");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pr.m == 0 || pr.n == 0 || pr.k == 0) return rs_epoch(rs, st);  // no tile arrivals
  if (g->splits > 1 && g->ws_dev == nullptr) {
    // The K ranges of a tile are summed in this GPU's L2 first (the Stream-K fixup workspace,
    // one tile per cluster tile of the problem), so each tile crosses to its owner once.
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != g->device)
      return fail(CPG_ERR_NO_DEVICE, "current device %d differs from the plan's device %d", cur,
                  g->device);
    const int rc2 = alloc_fixup_workspace(
        g, int64_t(g->sched.ncluster_m) * g->sched.ncluster_n);
    if (rc2 != CPG_OK) return rc2;
  }
  // The output tensor map is built on this rank's buffer and never used for stores.
  rc = run_impl(g, a, b, rs->dst[rs->rank], epi, stream, nullptr, rs);
  if (rc != CPG_OK) return rc;
  return rs_epoch(rs, st);
}

// Every CTA tile of the schedule (row tiles of all clusters, including a pair's tile past M)
// sends its sum once (with K ranges, the last range to finish sends it); each of its epilogue
// warps (4, or 8 for 512-wide tiles) then arrives once on the counter of the rank owning its
// rows (rows past M: the last).
static void rs_arrivals(const cpg::SchedParams& sp, int epi_warps, const cpg_reduce_scatter* rs,
                        uint32_t* per_rank) {
  for (int q = 0; q < rs->ranks; ++q) per_rank[q] = 0;
  const int64_t cta_rows = int64_t(sp.ncluster_m) * sp.cluster_m;
  const int64_t cta_cols = int64_t(sp.ncluster_n) * sp.cluster_n;
  const int64_t per_tile = int64_t(epi_warps) * cta_cols;
  for (int64_t i = 0; i < cta_rows; ++i) {
    const int64_t row = i * cpg::kBM;
    int owner = rs->ranks - 1;
    for (int q = 0; q < rs->ranks; ++q) {
      if (row < rs->row_start[q + 1]) {
        owner = q;
        break;
      }
    }
    per_rank[owner] += static_cast<uint32_t>(per_tile);
  }
}

int cpg_sched_rs_arrivals(const cpg_sched_params* sp, int32_t tile_n,
                          const cpg_reduce_scatter* rs, uint32_t* per_rank) {
  if (sp == nullptr || rs == nullptr || per_rank == nullptr)
    return fail(CPG_ERR_NULL, "NULL argument");
  if (tile_n != 64 && tile_n != 128 && tile_n != 256 && tile_n != 512)
    return fail(CPG_ERR_UNSUPPORTED, "tile_n must be 64, 128, 256 or 512");
  if (rs->ranks < 1 || rs->ranks > CPG_MAX_PEERS)
    return fail(CPG_ERR_INVALID_CONFIG, "1 to %d ranks", CPG_MAX_PEERS);
  cpg::SchedParams p;
  static_assert(sizeof(cpg_sched_params) == sizeof(cpg::SchedParams), "layout mismatch");
  std::memcpy(&p, sp, sizeof(p));
  rs_arrivals(p, tile_n == 512 ? cpg::EpiShape<512>::kWarps : cpg::kEpiWarps, rs, per_rank);
  return CPG_OK;
}

int cpg_gemm_rs_arrivals(const cpg_gemm* g, const cpg_reduce_scatter* rs, uint32_t* per_rank) {
  int rc = check_reduce_scatter(g, rs);
  if (rc != CPG_OK) return rc;
  if (per_rank == nullptr) return fail(CPG_ERR_NULL, "per_rank is NULL");
  for (int q = 0; q < rs->ranks; ++q) per_rank[q] = 0;
  const cpg_gemm_problem& pr = g->prob;
  if (pr.m != 0 && pr.n != 0 && pr.k != 0) rs_arrivals(g->sched, g->v.epi_warps, rs, per_rank);
  for (int q = 0; q < rs->ranks; ++q) ++per_rank[q];  // the call's epoch arrival (rs_epoch)
  return CPG_OK;
}

int cpg_peer_finish(float* w, int64_t ldw, const uint32_t* count, uint32_t target, int64_t rows,
                    int64_t cols, void* d, int64_t ldd, const void* bias, int32_t* status,
                    int32_t timeout_ms, void* stream) {
  if (rows < 0 || cols < 0 || ldw < cols || ldd < cols)
    return fail(CPG_ERR_INVALID_SHAPE, "bad extents");
  if (cols % 4 != 0 || ldw % 4 != 0 || ldd % 4 != 0)
    return fail(CPG_ERR_ALIGNMENT, "cols, ldw and ldd must be multiples of 4");
  if (count == nullptr || status == nullptr) return fail(CPG_ERR_NULL, "count and status");
  if (timeout_ms <= 0) return fail(CPG_ERR_INVALID_SHAPE, "timeout must be positive");
  if (rows > 0 && cols > 0 && (w == nullptr || d == nullptr))
    return fail(CPG_ERR_NULL, "w and d must be non-NULL");
  if ((reinterpret_cast<uintptr_t>(w) & 15u) != 0 || (reinterpret_cast<uintptr_t>(d) & 7u) != 0)
    return fail(CPG_ERR_ALIGNMENT, "w 16-byte and d 8-byte aligned");
  // At least one CTA waits even without rows, so a finish always observes its call's arrivals.
  const int64_t blocks = rows < 1 ? 1 : (rows < 1024 ? rows : 1024);
  cpg::peer_finish_kernel<<<static_cast<unsigned>(blocks), 256, 0,
                            reinterpret_cast<cudaStream_t>(stream)>>>(
      w, ldw, count, target, rows, cols, static_cast<__nv_bfloat16*>(d), ldd,
      static_cast<const __nv_bfloat16*>(bias), status, uint64_t(timeout_ms) * 1000000ull);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CPG_OK : cuda_fail(e, "peer finish launch");
}

int cpg_cast_f32_bf16(const float* x, int64_t rows, int64_t cols, int64_t ldx, void* y,
                      int64_t ldy, const void* bias, void* stream) {
  if (rows < 0 || cols < 0 || ldx < cols || ldy < cols)
    return fail(CPG_ERR_INVALID_SHAPE, "bad cast extents");
  if (rows == 0 || cols == 0) return CPG_OK;
  if (x == nullptr || y == nullptr) return fail(CPG_ERR_NULL, "x and y must be non-NULL");
  const dim3 grid = cast_grid(rows, cols);
  cpg::cast_f32_bf16_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, rows, cols, ldx, static_cast<__nv_bfloat16*>(y), ldy,
      static_cast<const __nv_bfloat16*>(bias));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CPG_OK : cuda_fail(e, "cast launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Split-K GEMM with BF16 output that allocates no device memory (cpg_gemm_splitk_static).
//
// The split-K path needs an FP32 buffer of M x N partial sums between the GEMM (whose K ranges
// add into it with TMA reduce-add) and the cast to BF16.  Callers that cannot allocate device
// memory (for example an embedding runtime whose device memory is carved up in advance, or
// code that must not call cudaMalloc while other work is being captured into a CUDA graph)
// get that buffer from this file-scope array instead.  Every GPU that loads the library holds
// the array until the process exits.
namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;  // 16 MiB: M * N <= 4,194,304 fp32
constexpr int kStaticMaxDevices = 64;

static __device__ __align__(256) float g_splitk_scratch[kStaticScratchBytes / sizeof(float)];

std::mutex g_static_mu;
void* g_static_scratch_addr[kStaticMaxDevices];  // device address of the array, per device

// Device address of g_splitk_scratch on the current device.  The array's name in host code is
// only a stand-in; the address must come from cudaGetSymbolAddress with the device current,
// once per device (the first call on a device also loads the module there).
int static_scratch_address(int dev, float** out) {
  if (dev < 0 || dev >= kStaticMaxDevices) return fail(CPG_ERR_NO_DEVICE, "device %d", dev);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (g_static_scratch_addr[dev] == nullptr) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_splitk_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static split-K scratch)");
    g_static_scratch_addr[dev] = ptr;
  }
  *out = static_cast<float*>(g_static_scratch_addr[dev]);
  return CPG_OK;
}

}  // namespace

extern "C" int cpg_gemm_splitk_static(const cpg_gemm_config* cfg, const cpg_gemm_problem* prob,
                                      const void* a, const void* b, void* d,
                                      const cpg_epilogue* epi, void* stream) {
  if (cfg == nullptr || prob == nullptr) return fail(CPG_ERR_NULL, "cfg and prob must be non-NULL");
  int rc = cpg_config_validate(cfg);
  if (rc != CPG_OK) return rc;
  if (cfg->dynamic_scheduler)
    return fail(CPG_ERR_UNSUPPORTED, "the dynamic scheduler is not available on this entry point");
  if (cfg->tile_m != 128 ||
      (cfg->tile_n != 64 && cfg->tile_n != 128 && cfg->tile_n != 256 && cfg->tile_n != 512) ||
      cfg->cluster_m > 2 || cfg->cluster_n > 2 || cfg->ab_stage > cpg::kMaxStages ||
      cfg->epi_stage > cpg::kMaxEpiStages || cfg->gemm_n_prologue >= cfg->ab_stage)
    return fail(CPG_ERR_UNSUPPORTED, "tile (128, 64/128/256/512), cluster within (2, 2, 1) only");
  if (prob->dtype_ab != CPG_DTYPE_BF16 && prob->dtype_ab != CPG_DTYPE_E4M3)
    return fail(CPG_ERR_DTYPE, "A and B must be BF16 or FP8 E4M3");
  if (prob->dtype_d != CPG_DTYPE_BF16) return fail(CPG_ERR_DTYPE, "D must be BF16");
  if (prob->scale_mode != CPG_SCALE_TENSOR)
    return fail(CPG_ERR_UNSUPPORTED, "block-scaled FP8 is not available on this entry point");
  if (prob->gated != 0 || prob->l > 1 ||
      (epi != nullptr && (epi->activation != CPG_ACT_NONE || epi->source != nullptr)))
    return fail(CPG_ERR_UNSUPPORTED,
                "gated GEMM, batches, activations and C are not available here");
  const int64_t lim = (int64_t(1) << 31) - 1;
  if (prob->m < 0 || prob->n < 0 || prob->k < 0 || prob->m > lim || prob->n > lim ||
      prob->k > lim || prob->lda < prob->k || prob->ldb < prob->k || prob->ldd < prob->n ||
      prob->split_k < 0)
    return fail(CPG_ERR_INVALID_SHAPE, "bad extents or strides");
  const int eab = elem_bytes(prob->dtype_ab);
  if ((prob->lda * eab) % 16 != 0 || (prob->ldb * eab) % 16 != 0 || (prob->ldd * 2) % 16 != 0)
    return fail(CPG_ERR_ALIGNMENT, "row strides must be multiples of 16 bytes");
  const int64_t ldw = (prob->n + 3) / 4 * 4;  // FP32 [M, N] rows padded to 16 bytes
  // Compare by division first: M and N may each be up to 2^31 - 1, so M * ldw * 4 could pass
  // 2^63 and wrap before a multiplied comparison saw it.
  const int64_t cap_floats = static_cast<int64_t>(kStaticScratchBytes / sizeof(float));
  if (prob->m > 0 && ldw > cap_floats / prob->m)
    return fail(CPG_ERR_INVALID_SHAPE,
                "M x N = %lld x %lld needs %.0f bytes of FP32 scratch; the static scratch holds "
                "%lld bytes (M * round_up(N, 4) <= %lld)",
                static_cast<long long>(prob->m), static_cast<long long>(prob->n),
                static_cast<double>(prob->m) * static_cast<double>(ldw) * sizeof(float),
                static_cast<long long>(kStaticScratchBytes), static_cast<long long>(cap_floats));
  const int64_t need = prob->m * ldw * static_cast<int64_t>(sizeof(float));  // <= 16 MiB now
  if (prob->m == 0 || prob->n == 0) return CPG_OK;
  if (d == nullptr) return fail(CPG_ERR_NULL, "D is NULL");
  if ((reinterpret_cast<uintptr_t>(d) & 15u) != 0) return fail(CPG_ERR_ALIGNMENT, "D alignment");
  const void* bias = epi != nullptr ? epi->bias : nullptr;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const unsigned cast_blocks = static_cast<unsigned>(prob->m < 65535 ? prob->m : 65535);

  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  int major = 0;
  e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  if (major != 10) return fail(CPG_ERR_NO_DEVICE, "device %d is not sm_100", dev);
  float* ws = nullptr;
  rc = static_scratch_address(dev, &ws);
  if (rc != CPG_OK) return rc;

  if (prob->k == 0) {  // D = bias (or 0): nothing to contract
    fill_rows_kernel<__nv_bfloat16><<<cast_blocks, 256, 0, st>>>(
        static_cast<__nv_bfloat16*>(d), prob->m, prob->n, prob->ldd,
        static_cast<const __nv_bfloat16*>(bias));
    e = cudaGetLastError();
    return e == cudaSuccess ? CPG_OK : cuda_fail(e, "fill kernel launch");
  }
  if (a == nullptr || b == nullptr) return fail(CPG_ERR_NULL, "A and B must be non-NULL");
  if ((reinterpret_cast<uintptr_t>(a) & 15u) != 0 || (reinterpret_cast<uintptr_t>(b) & 15u) != 0)
    return fail(CPG_ERR_ALIGNMENT, "A and B must be 16-byte aligned");

  // Kernel, shared memory and grid (the same choices cpg_gemm_create makes, kept on the stack).
  Variant v;
  const int cta_group = cfg->cluster_m == 2 ? 2 : 1;
  if (!find_variant(cfg->tile_n, cta_group, prob->dtype_ab, CPG_DTYPE_F32, CPG_SCALE_TENSOR, &v))
    return fail(CPG_ERR_UNSUPPORTED, "no kernel for this configuration");
  const int smem = v.smem_bytes(cfg->ab_stage, cfg->epi_stage, cfg->reuse_ab);
  int optin = 0;
  e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(smem)");
  if (smem > optin) return fail(CPG_ERR_SMEM, "%d stages need %d bytes", cfg->ab_stage, smem);
  int mac = 0;
  rc = query_max_active_clusters(v, smem, cfg->cluster_m, cfg->cluster_n, &mac);
  if (rc != CPG_OK) return rc;
  if (mac <= 0) return fail(CPG_ERR_NO_DEVICE, "kernel cannot be resident");
  const int bk = cpg::kRowBytes / eab;
  const int32_t k_iters = static_cast<int32_t>((prob->k + bk - 1) / bk);
  int32_t splits = prob->split_k > 1 ? prob->split_k : 1;
  if (splits > k_iters) splits = k_iters;
  const int32_t kps = (k_iters + splits - 1) / splits;
  splits = (k_iters + kps - 1) / kps;
  const int32_t ntm = static_cast<int32_t>((prob->m + 127) / 128);
  const int32_t ntn = static_cast<int32_t>((prob->n + cfg->tile_n - 1) / cfg->tile_n);

  cpg::GemmParams p;
  std::memset(&p, 0, sizeof(p));
  p.sched = cpg::sched_params_create(ntm, ntn, splits, cfg->raster_order, cfg->group_size,
                                     cfg->cluster_m, cfg->cluster_n, cfg->is_persistent);
  int32_t grid[3];
  cpg::sched_grid_shape(p.sched, mac, grid);
  p.m = static_cast<int32_t>(prob->m);
  p.n = static_cast<int32_t>(prob->n);
  p.k = static_cast<int32_t>(prob->k);
  p.k_iters = k_iters;
  p.k_iters_per_split = kps;
  p.num_splits = splits;
  p.reduce_add = splits > 1 ? 1 : 0;
  p.ab_stages = cfg->ab_stage;
  p.epi_stages = cfg->epi_stage;
  p.reuse_ab = cfg->reuse_ab;
  p.alpha = epi != nullptr ? epi->alpha : 1.0f;
  p.scale_a = epi != nullptr ? epi->scale_a : nullptr;
  p.scale_b = epi != nullptr ? epi->scale_b : nullptr;
  p.bias = nullptr;      // added once, by the cast
  p.status = nullptr;    // no status word: a wait past its deadline just stops the kernel
  p.timeout_ns = 10ull * 1000ull * 1000ull * 1000ull;

  CUtensorMap tm_a, tm_b, tm_w;
  rc = encode_tiled(&tm_a, tma_dtype(prob->dtype_ab), eab, a, prob->m, prob->k, prob->lda,
                    cpg::kBM, bk);
  if (rc != CPG_OK) return rc;
  rc = encode_tiled(&tm_b, tma_dtype(prob->dtype_ab), eab, b, prob->n, prob->k, prob->ldb,
                    (v.bn > 256 ? 256 : v.bn) / v.cta_group, bk);
  if (rc != CPG_OK) return rc;
  rc = encode_tiled(&tm_w, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ws, prob->m, prob->n, ldw, 32,
                    cpg::kRowBytes / 4);
  if (rc != CPG_OK) return rc;

  // The array keeps the previous call's sums: clear the region the K ranges add into.
  if (splits > 1) {
    e = cudaMemsetAsync(ws, 0, static_cast<size_t>(need), st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(static scratch)");
  }
  cudaLaunchConfig_t lc = {};
  cudaLaunchAttribute attr[1];
  lc.gridDim = dim3(grid[0], grid[1], grid[2]);
  lc.blockDim = dim3(v.threads, 1, 1);
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  if (cfg->cluster_m * cfg->cluster_n > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cfg->cluster_m;
    attr[0].val.clusterDim.y = cfg->cluster_n;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
  }
  CUtensorMap tm_unused;  // the Stream-K workspace map: no Stream-K here
  std::memset(&tm_unused, 0, sizeof(tm_unused));
  void* args[] = {&tm_a, &tm_b, &tm_w, &tm_unused, &p};
  e = cudaLaunchKernelExC(&lc, v.fn, args);
  if (e != cudaSuccess) return cuda_fail(e, "split-K GEMM launch");
  cpg::cast_f32_bf16_kernel<<<cast_grid(prob->m, prob->n), 256, 0, st>>>(
      ws, prob->m, prob->n, ldw, static_cast<__nv_bfloat16*>(d), prob->ldd,
      static_cast<const __nv_bfloat16*>(bias));
  e = cudaGetLastError();
  return e == cudaSuccess ? CPG_OK : cuda_fail(e, "cast kernel launch");
}
