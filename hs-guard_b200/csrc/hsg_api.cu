// HS-Guard B200 streaming engine: state pools, the per-tick kernel sequence, CUDA-graph capture per (rows, tokens)
// bucket, and the C ABI declared in include/hsg.h.
#include <cudaTypedefs.h>

#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/hsg.h"
#include "attn.cuh"
#include "common.cuh"
#include "gdn.cuh"
#include "gdn_tc.cuh"
#include "gdn_chunk.cuh"
#include "gdn_cols.cuh"
#include "gdn_wy.cuh"
#include "ring_decode_split.cuh"
#include "gemm.cuh"
#include "gemm_persist.cuh"
#include "norm.cuh"
#include "ring_decode.cuh"
#include "ring_prefill.cuh"
#include "ring_prefill_tc.cuh"

using namespace hsg;

// ---- error plumbing ---------------------------------------------------------------------------------------------
static thread_local std::string g_last_error;

static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define CU(call)                                                                                   \
  do {                                                                                             \
    cudaError_t e_ = (call);                                                                       \
    if (e_ != cudaSuccess) return fail(HSG_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                                       __FILE__, __LINE__);                                        \
  } while (0)

static const char* device_error_text(int code) {
  switch (code) {
    case ERR_TIMEOUT_TMA: return "a bounded wait for a TMA copy timed out";
    case ERR_TIMEOUT_MMA: return "a bounded wait for tensor-core completion timed out";
    case ERR_BAD_SLOT: return "a slot index was outside [0, max_slots]";
    case ERR_BAD_TOKEN: return "a token id was outside the vocabulary";
    case ERR_BAD_LEN: return "a row length was outside [0, lb]";
    default: return "unknown device error";
  }
}

// ---- TMA descriptors --------------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_encoder() {
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && fn)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode ? HSG_OK : fail(HSG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
}

// 2-D row-major tensor map: `rows` x `cols` elements of `dtype`, rows `row_bytes` apart, box `box_cols` x `box_rows`.
static int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                       uint64_t cols, uint64_t row_bytes, int box_cols, int box_rows, CUtensorMapSwizzle swizzle) {
  if (get_encoder() != HSG_OK) return HSG_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15) || ((uint64_t)box_cols * elem_bytes) % 16 ||
      box_rows < 1 || box_rows > 256 || box_cols > 256 || rows < 1)
    return fail(HSG_ERR_INVALID, "bad tensor map (base %p, row bytes %llu, box %d x %d)", base,
                (unsigned long long)row_bytes, box_cols, box_rows);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HSG_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return HSG_OK;
}

// 3-D tensor map, no swizzle: extents d0 (contiguous) x d1 x d2 with byte strides s1, s2; box b0 x b1 x b2.
static int make_map_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes, uint64_t d0,
                       uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2, int b0, int b1, int b2) {
  if (get_encoder() != HSG_OK) return HSG_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (s1 & 15) || (s2 & 15) || ((uint64_t)b0 * elem_bytes) % 16 ||
      b0 < 1 || b1 < 1 || b2 < 1 || b0 > 256 || b1 > 256 || b2 > 256 || d2 < 1)
    return fail(HSG_ERR_INVALID, "bad 3-D tensor map (base %p, strides %llu %llu, box %d x %d x %d)", base,
                (unsigned long long)s1, (unsigned long long)s2, b0, b1, b2);
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  cuuint64_t strides[2] = {(cuuint64_t)s1, (cuuint64_t)s2};
  cuuint32_t box[3] = {(cuuint32_t)b0, (cuuint32_t)b1, (cuuint32_t)b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HSG_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", (int)r);
  return HSG_OK;
}

// GEMM operand: bf16 [rows][k], box [64 k][box_rows], 128-byte swizzle (the tcgen05 K-major SW128 layout).
static int make_map(CUtensorMap* map, const void* base, int rows, int k, int box_rows) {
  if (k % 64 || box_rows < 16) return fail(HSG_ERR_INVALID, "bad operand map (k %d, box %d)", k, box_rows);
  return make_map_2d(map, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, k, (uint64_t)k * 2, 64, box_rows,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

// ---- GEMM planning ----------------------------------------------------------------------------------------------
struct GemmPlan {
  int tb, tn, splits, kps, stages, smem;
  int persist;  // 1: gemm_pc_kernel (persistent, double-buffered accumulator), one CTA per SM
  int halves;   // gemm_pc_kernel: 128-row weight halves per tile
};

static constexpr int SM_COUNT = 148;
static constexpr int SMEM_MAX = 227 * 1024;

static int gemm_smem(int tn, int use_lo, int stages) {
  return stages * gemm_stage_bytes(tn, use_lo) + (2 * stages + 1) * 8 + 16 + 1024;
}

// Choose token blocking (tb blocks of tn tokens), K splits (atomic mode only) and pipeline depth. Modelled CTA time
// in SM cycles: a fixed cost (barrier/TMEM set-up, first TMA latency) + per 64-wide K block the weight-tile load and
// the MMAs over tn tokens (x2 with the lo operand) + the epilogue; the grid runs in ceil(CTAs / 148) waves.
static long gemm_cost(int tiles, int KB, int tb, int tn, int splits, int kps, int mode, int use_lo) {
  const long ctas = (long)tiles * tb * splits;
  const long waves = (ctas + SM_COUNT - 1) / SM_COUNT;
  const long per_kb = 256 + 2L * tn * (1 + use_lo);
  const long epi = (long)tn * (mode == GEMM_ATOMIC ? 8 : 4);
  return waves * (3000 + kps * per_kb + epi);
}

static GemmPlan plan_gemm(int n_w, int K, int M, int mode, int use_lo) {
  const int tiles = n_w / 128, KB = K / 64;
  GemmPlan best{0, 0, 0, 0, 0, 0, 0, 1};
  long best_cost = -1;
  const int max_tb = (M + 15) / 16;
  for (int tb = 1; tb <= max_tb; ++tb) {
    const int tn = ((M + tb - 1) / tb + 15) / 16 * 16;
    if (tn > 256) continue;
    const int max_splits = mode == GEMM_ATOMIC ? std::max(1, KB / 2) : 1;
    for (int sp = 1; sp <= max_splits; ++sp) {
      const int kps = (KB + sp - 1) / sp;
      const int splits = (KB + kps - 1) / kps;
      if (splits != sp) continue;
      const long cost = gemm_cost(tiles, KB, tb, tn, splits, kps, mode, use_lo);
      if (best_cost < 0 || cost < best_cost) {
        best_cost = cost;
        best = {tb, tn, splits, kps, 0, 0, 0, 1};
      }
    }
  }
  int stages = 4;
  while (stages > 2 && gemm_smem(best.tn, use_lo, stages) > SMEM_MAX) --stages;
  best.stages = std::min(stages, std::max(2, best.kps));
  const int tb_full = (M + 255) / 256;
  const long full_tiles = (long)tiles * tb_full;
  // GEMM_CONV always takes the persistent kernel (its epilogue carries the conv along a tile's 32-token chunks)
  if (mode == GEMM_CONV || full_tiles >= 4L * SM_COUNT || (mode != GEMM_ATOMIC && full_tiles >= 2L * SM_COUNT)) {
    // A long-running grid: the persistent kernel, one CTA per SM looping over 256-token tiles with the accumulator
    // double-buffered in TMEM (all 512 columns; each tile's epilogue overlaps the next tile's MMAs) and two load
    // stages beside the two epilogue chunk buffers. Measured (algorithmic TFLOP/s, in_proj / gate-up / out_proj /
    // down): 22,528 tokens 621 / 638 / 529 / 563 against 381 / 342 / 392 / 415 for the per-tile kernel and 529 / 531
    // / 486 / 519 with 128-token tiles; at 2,048 tokens in_proj 520 against 443. Split-K reduce-add GEMMs keep the
    // per-tile kernel below 4 waves of full tiles, where its K splits fill the machine better.
    best.persist = 1;
    best.halves = mode == GEMM_ATOMIC ? 2 : 1;  // 256 x 128 tiles for the reduce-add shapes, else 128 x 256
    best.tn = 256 / best.halves;
    best.tb = (M + best.tn - 1) / best.tn;
    best.splits = 1;
    best.kps = KB;
    int st = 6;
    while (st > 2 && gpc_smem(best.tn, use_lo, st, mode, best.halves) > SMEM_MAX) --st;
    best.stages = st;
    best.smem = gpc_smem(best.tn, use_lo, st, mode, best.halves);
    return best;
  }
  best.smem = gemm_smem(best.tn, use_lo, best.stages);
  return best;
}

// The chunked delta rule of 32/64-token ticks runs on tcgen05 (gdn_wy_kernel); HSG_GDN_WY=0 selects the warp-MMA
// kernel (gdn_chunk_kernel) instead, kept as the comparison.
static bool use_wy_chunk() {
  const char* s = getenv("HSG_GDN_WY");
  return !(s && strcmp(s, "0") == 0);
}
// With the tcgen05 chunked kernel the causal conv + SiLU of q | k | v runs in the input projection's epilogue
// (GEMM_CONV); HSG_GDN_CONV_GEMM=0 leaves it in the GDN kernel instead.
static bool use_conv_in_gemm() {
  const char* s = getenv("HSG_GDN_CONV_GEMM");
  return !(s && strcmp(s, "0") == 0);
}

// Kernel launch with the programmatic-stream-serialization attribute (programmatic dependent launch): the kernel may
// begin while its predecessor drains; every kernel calls pdl_wait() before touching memory its predecessor uses.
template <typename... KArgs, typename... Args>
static cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// The same with the thread-block-cluster dimension attribute (clusters of cluster_x CTAs along x).
template <typename... KArgs, typename... Args>
static cudaError_t launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, int cluster_x, size_t smem,
                                  cudaStream_t st, bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Single-token ring decode: with fewer (row, kv head) items than SMs each item is split over a cluster of
// RDS_SPLIT CTAs (ring_decode_split_kernel), else whole items go to one persistent CTA per SM.
static bool ring_decode_splits(int nb) { return nb * ATT_HKV < SM_COUNT; }

struct hsg_engine;
static void prof_mark(hsg_engine* e, int cls);

static int launch_gemm(cudaStream_t st, const void* w, int n_w, int K, const void* xhi, const void* xlo, int m_alloc,
                       int M, int mode, float* y, int ldy, __nv_bfloat16* ahi, __nv_bfloat16* alo, int ld_act,
                       int* err, int force_splits = 0, hsg_engine* prof = nullptr, int prof_cls = -1,
                       bool pdl = false, const GemmConv* conv = nullptr) {
  if (mode == GEMM_CONV && (!conv || conv->lb % GPC_CHUNK != 0 || 256 % conv->lb != 0))
    return fail(HSG_ERR_INVALID, "GEMM_CONV needs requests of 32 or 64 tokens");
  const int use_lo = xlo != nullptr;
  GemmPlan p = plan_gemm(n_w, K, M, mode, use_lo);
  if (force_splits > 0 && mode == GEMM_ATOMIC && !p.persist) {
    const int KB = K / 64;
    p.kps = (KB + force_splits - 1) / force_splits;
    p.splits = (KB + p.kps - 1) / p.kps;
  }
  CUtensorMap tw, th, tl, t0, t1;
  int rc;
  if ((rc = make_map(&tw, w, n_w, K, 128 * p.halves)) != HSG_OK) return rc;
  if ((rc = make_map(&th, xhi, m_alloc, K, p.tn)) != HSG_OK) return rc;
  if ((rc = make_map(&tl, use_lo ? xlo : xhi, m_alloc, K, p.tn)) != HSG_OK) return rc;
  const int out_rows = p.persist ? GPC_CHUNK : p.tn;  // the persistent kernel stores 32-token chunks
  if (mode == GEMM_SILU_MUL) {
    if ((rc = make_map_2d(&t0, ahi, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, n_w / 2, (uint64_t)ld_act * 2, 64,
                          out_rows, CU_TENSOR_MAP_SWIZZLE_NONE)) != HSG_OK)
      return rc;
    if ((rc = make_map_2d(&t1, alo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, n_w / 2, (uint64_t)ld_act * 2, 64,
                          out_rows, CU_TENSOR_MAP_SWIZZLE_NONE)) != HSG_OK)
      return rc;
  } else {
    if ((rc = make_map_2d(&t0, y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, M, n_w, (uint64_t)ldy * 4, 128, out_rows,
                          CU_TENSOR_MAP_SWIZZLE_NONE)) != HSG_OK)
      return rc;
    t1 = t0;
  }
  if (p.persist) {
    GemmPcArgs a;
    a.halves = p.halves;
    a.n_w = n_w;
    a.tiles_w = (n_w / 128 + p.halves - 1) / p.halves;
    a.tb = p.tb;
    a.splits = 1;
    a.kps = K / 64;
    a.k_blocks_total = K / 64;
    a.tn = p.tn;
    a.m = M;
    a.use_lo = use_lo;
    a.stages = p.stages;
    a.mode = mode;
    a.err = err;
    a.conv = conv ? *conv : GemmConv{};
    const int total = a.tiles_w * a.tb;
    if (prof) prof_mark(prof, prof_cls);
    CU(launch_k(gemm_pc_kernel, dim3(std::min(total, SM_COUNT)), dim3(GPC_THREADS), p.smem, st, pdl, tw, th, tl, t0,
                t1, a));
    if (prof) prof_mark(prof, -1);
    return HSG_OK;
  }
  GemmArgs a;
  a.k_blocks_per_split = p.kps;
  a.k_blocks_total = K / 64;
  a.tn = p.tn;
  a.use_lo = use_lo;
  a.stages = p.stages;
  a.mode = mode;
  a.err = err;
  dim3 grid(p.tb, n_w / 128, p.splits);
  if (prof) prof_mark(prof, prof_cls);
  CU(launch_k(gemm_tc_kernel, grid, dim3(GEMM_THREADS), p.smem, st, pdl, tw, th, tl, t0, t1, a));
  if (prof) prof_mark(prof, -1);
  return HSG_OK;
}

// Tensor map of an fp16 recurrent-state pool [(slots+1)*16 tiles][128 k][128 v] viewed as [rows][128], read and
// written in [128 k x 64 v] halves with 128-byte swizzle (gdn_tc_kernel).
static int make_state_map(CUtensorMap* map, const void* base, int64_t slots_plus_one) {
  return make_map_2d(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)slots_plus_one * GDN_H * GDN_D, GDN_D,
                     GDN_D * 2, 64, GDN_D, CU_TENSOR_MAP_SWIZZLE_128B);
}

// Tensor maps of the single-token decode kernel: a [rows][256] fp16 tensor read in [64 dims x 32 rows] boxes.
static int make_decode_map(CUtensorMap* map, const void* base, uint64_t rows) {
  return make_map_2d(map, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, rows, ATT_D, ATT_D * 2, 64, RD_TILE,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

static int set_kernel_attributes() {
  CU(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX));
  CU(cudaFuncSetAttribute(gemm_pc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX));
  CU(cudaFuncSetAttribute(gdn_step_kernel<true, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_SMEM_LIMIT));
  CU(cudaFuncSetAttribute(gdn_step_kernel<false, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_SMEM_LIMIT));
  CU(cudaFuncSetAttribute(gdn_step_kernel<true, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_SMEM_LIMIT));
  CU(cudaFuncSetAttribute(gdn_step_kernel<false, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          GDN_SMEM_LIMIT));
  CU(cudaFuncSetAttribute(gdn_tc_kernel<true, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_SMEM_LIMIT));
  CU(cudaFuncSetAttribute(gdn_tc_kernel<true, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_SMEM_LIMIT));
  CU(cudaFuncSetAttribute(gdn_tc_kernel<false, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_SMEM_LIMIT));
  CU(cudaFuncSetAttribute(gdn_tc_kernel<false, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_SMEM_LIMIT));
  CU(cudaFuncSetAttribute(gdn_chunk_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_SMEM_LIMIT));
  CU(cudaFuncSetAttribute(gdn_chunk_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDN_SMEM_LIMIT));
  CU(cudaFuncSetAttribute(gdn_wy_kernel<64, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDNW_SMEM));
  CU(cudaFuncSetAttribute(gdn_wy_kernel<32, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDNW_SMEM));
  CU(cudaFuncSetAttribute(gdn_wy_kernel<64, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDNW_SMEM));
  CU(cudaFuncSetAttribute(gdn_wy_kernel<32, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, GDNW_SMEM));
  CU(cudaFuncSetAttribute(ring_attn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem_bytes(4)));
  CU(cudaFuncSetAttribute(ring_attn_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem_bytes(8)));
  CU(cudaFuncSetAttribute(ring_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, rd_smem_bytes()));
  CU(cudaFuncSetAttribute(ring_decode_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, rds_smem_bytes()));
  CU(cudaFuncSetAttribute(ring_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pf_smem_bytes()));
  CU(cudaFuncSetAttribute(ring_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, pt_smem_bytes()));
  return HSG_OK;
}

// ---- engine -----------------------------------------------------------------------------------------------------
struct Bucket {
  cudaGraphExec_t exec = nullptr;
  int launches = 0;
};

struct hsg_engine {
  hsg_config cfg;
  hsg_weights w;
  int S = 0, device = 0, flags = 0;
  int n_gdn = 0, n_attn = 0;
  int max_tokens = 0, m_alloc = 0;
  cudaStream_t stream = nullptr;
  // pools
  char* rec = nullptr;  // recurrent state, rec_elem bytes per element (fp16 by default, fp32 with HSG_FLAG_STATE_F32)
  int rec_elem = 2;
  float* conv = nullptr;
  __half* ring_k = nullptr;
  __half* ring_v = nullptr;
  int64_t* ring_pos = nullptr;
  // per-tick buffers
  int64_t* packed = nullptr;
  float* hidden = nullptr;
  __nv_bfloat16 *xhi = nullptr, *xlo = nullptr, *ohi = nullptr, *olo = nullptr, *ahi = nullptr, *alo = nullptr;
  float* proj = nullptr;
  float* qbuf = nullptr;
  __half *knew = nullptr, *vnew = nullptr;
  float* hbuf = nullptr;
  float* probs = nullptr;
  int* err = nullptr;
  int* err_host = nullptr;
  std::map<std::pair<int, int>, Bucket> graphs;
  CUtensorMap ring_maps[6][2];  // per attention layer: ring K, ring V as 2-D [rows][256] fp16, [64 x 32] SW128 boxes
  CUtensorMap new_maps[2];      // the tick's new K, V ([rows = row*2 + head][256], 1-token ticks)
  CUtensorMap state_maps[18];   // per GDN layer: the fp16 state pool (gdn_tc_kernel)
  CUtensorMap conv_maps[18];    // per GDN layer: the conv history as [(S+1)*3][3][2048], [3][3][128] boxes
  std::vector<void*> allocations;
  // profiling
  std::vector<cudaEvent_t> events;
  std::vector<int> event_class;
  bool profiling = false;
  bool pdl = true;
  int launch_count = 0;

  size_t rec_slot() const { return (size_t)GDN_H * GDN_D * GDN_D; }  // elements per slot and layer
  size_t conv_slot() const { return (size_t)CONV_KEEP * CONV_DIM; }
  size_t ring_slot() const { return (size_t)ATT_HKV * RING_COLS * ATT_D; }
};

template <class T>
static int dalloc(hsg_engine* e, T** p, size_t count) {
  void* q = nullptr;
  CU(cudaMalloc(&q, count * sizeof(T)));
  e->allocations.push_back(q);
  *p = static_cast<T*>(q);
  return HSG_OK;
}

static int check_config(const hsg_config* c) {
  if (!c) return fail(HSG_ERR_INVALID, "config is NULL");
  if (c->hidden != HIDDEN || c->intermediate != INTER || c->n_layers != HSG_N_LAYERS || c->full_attn_interval != 4 ||
      c->gdn_heads != GDN_H || c->gdn_head_dim != GDN_D || c->conv_kernel != CONV_K || c->attn_heads != ATT_HQ ||
      c->kv_heads != ATT_HKV || c->attn_head_dim != ATT_D || c->rotary_dim != ROT || c->window != WIN ||
      c->head_hidden != HEAD_E || c->n_classes != N_CLS || c->n_roles != N_ROLES || c->vocab <= 0)
    return fail(HSG_ERR_UNSUPPORTED, "unsupported architecture: the kernels are built for the HS-Guard backbone");
  return HSG_OK;
}

static bool is_attn_layer(int i) { return (i + 1) % 4 == 0; }

// Profiling: a timing event right before (class >= 0) and right after (class -1) each kernel launch.
static void prof_mark(hsg_engine* e, int cls) {
  if (cls >= 0) e->launch_count++;
  if (!e->profiling) return;
  cudaEvent_t ev;
  cudaEventCreate(&ev);
  cudaEventRecord(ev, e->stream);
  e->events.push_back(ev);
  e->event_class.push_back(cls);
}

struct ProfScope {
  hsg_engine* e;
  ProfScope(hsg_engine* e_, int c) : e(e_) { prof_mark(e, c); }
  ~ProfScope() { prof_mark(e, -1); }
};

// The whole tick as a sequence of kernels on e->stream (captured into a graph, or run eagerly when profiling).
static int enqueue_step(hsg_engine* e, int nb, int lb) {
  const int M = nb * lb;
  cudaStream_t st = e->stream;
  const int64_t* ids = e->packed;
  const int64_t* lens = ids + M;
  const int64_t* slots = lens + nb;
  const int64_t* starts = slots + nb;
  const int use_lo = !(e->flags & HSG_FLAG_BF16_ACT);
  const float eps = e->cfg.rms_eps;
  int rc;
  auto lo = [&](__nv_bfloat16* p) { return use_lo ? p : nullptr; };
  GdntMaps tc_maps;  // the tensor-core GDN kernel's projection maps for this tick shape
  if (e->rec_elem == 2 && lb <= GDNT_MAX_LB) {
    if ((rc = make_map_3d(&tc_maps.in1, e->proj, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, KEY_DIM, 4, M, KEY_DIM * 4,
                          GDN_IN * 4, GDN_D, 4, lb)) != HSG_OK)
      return rc;
    if ((rc = make_map_2d(&tc_maps.in2, e->proj + GDN_B_OFF, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, M, GDNT_AB,
                          GDN_IN * 4, GDNT_AB, lb, CU_TENSOR_MAP_SWIZZLE_NONE)) != HSG_OK)
      return rc;
  }
  // the chunked kernel (fp16 state, ticks of 32 or 64 tokens): the projection's q|k|v columns, [lb][3][128] boxes
  const bool chunked = e->rec_elem == 2 && lb > GDNT_MAX_LB && lb % GDNC_SUB == 0 && lb <= GDNC_MAX_LB;
  // 32/64-token ticks on the tcgen05 chunked kernel take their conv from the input projection's epilogue
  const bool pre_conv = chunked && use_wy_chunk() && (lb == 32 || lb == 64) && use_conv_in_gemm();
  GdntMaps ch_maps;
  if (chunked &&
      (rc = make_map_3d(&ch_maps.in1, e->proj, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, KEY_DIM, 3, M, KEY_DIM * 4,
                        GDN_IN * 4, GDN_D, 3, lb)) != HSG_OK)
    return rc;
  {
    ProfScope ps(e, HSG_PROF_EMBED);
    embed_norm_kernel<<<M, NORM_THREADS, 0, st>>>(ids, static_cast<const __nv_bfloat16*>(e->w.embed), e->cfg.vocab,
                                                  e->w.layers[0].norm_in, eps, e->hidden, e->xhi, e->xlo, M, e->err);
    CU(cudaGetLastError());
  }
  int gi = 0, ai = 0;
  for (int i = 0; i < HSG_N_LAYERS; ++i) {
    const hsg_layer_weights& L = e->w.layers[i];
    if (!is_attn_layer(i)) {
      {
        GemmConv cv{lens, slots, e->conv + (size_t)gi * (e->S + 1) * e->conv_slot(), L.conv_w, lb, e->S};
        if ((rc = launch_gemm(st, L.w_in, GDN_IN, HIDDEN, e->xhi, lo(e->xlo), e->m_alloc, M,
                              pre_conv ? GEMM_CONV : GEMM_STORE, e->proj, GDN_IN, nullptr, nullptr, 0, e->err, 0, e,
                              HSG_PROF_GEMM_IN, e->pdl, pre_conv ? &cv : nullptr)) != HSG_OK)
          return rc;
      }
      GdnArgs g{};
      g.slots = slots; g.lens = lens; g.nb = nb; g.lb = lb; g.max_slots = e->S;
      g.proj = e->proj;
      g.conv_pool = e->conv + (size_t)gi * (e->S + 1) * e->conv_slot();
      g.conv_w = L.conv_w; g.gnorm_w = L.gnorm_w; g.eps = eps;
      g.out_hi = e->ohi; g.out_lo = e->olo;
      g.A_log = L.A_log; g.dt_bias = L.dt_bias;
      g.state = e->rec + (size_t)gi * (e->S + 1) * e->rec_slot() * e->rec_elem;
      g.err = e->err;
      {
        ProfScope ps(e, HSG_PROF_GDN);
        const dim3 grid(GDN_H, std::min(nb, GDN_CTAS_PER_HEAD));
        if (e->rec_elem == 2 && lb <= GDNT_MAX_LB) {
          g.stages = gdnt_stages(lb, true);
          tc_maps.state = e->state_maps[gi];
          tc_maps.in0 = e->conv_maps[gi];
          if (lb == 1)
            CU(launch_k(gdn_tc_kernel<true, 4>, grid, dim3(GDNT_THREADS), gdnt_smem_bytes(lb, true), st, e->pdl,
                        tc_maps, g));
          else
            CU(launch_k(gdn_tc_kernel<true, 3>, grid, dim3(GDNT_THREADS), gdnt_smem_bytes(lb, true), st, e->pdl,
                        tc_maps, g));
        } else if (chunked && use_wy_chunk()) {
          GdntMaps wy;
          wy.state = e->state_maps[gi];
          wy.in0 = e->conv_maps[gi];
          if ((rc = make_map_2d(&wy.in1, e->proj, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, M, GDN_IN, GDN_IN * 4, GDN_D,
                                lb, CU_TENSOR_MAP_SWIZZLE_NONE)) != HSG_OK)
            return rc;
          wy.in2 = wy.in1;
          auto kfn = lb == 64 ? (pre_conv ? gdn_wy_kernel<64, true> : gdn_wy_kernel<64, false>)
                              : (pre_conv ? gdn_wy_kernel<32, true> : gdn_wy_kernel<32, false>);
          CU(launch_k(kfn, grid, dim3(GDNW_THREADS), GDNW_SMEM, st, e->pdl, wy, g));
        } else if (chunked) {
          g.stages = gdnc_stages(lb, true);
          ch_maps.state = e->state_maps[gi];
          ch_maps.in0 = e->conv_maps[gi];
          ch_maps.in2 = ch_maps.in1;
          CU(launch_k(gdn_chunk_kernel<true>, grid, dim3(GDNT_THREADS), gdnc_smem_bytes(lb, true), st, e->pdl,
                      ch_maps, g));
        } else if (e->rec_elem == 2) {
          const int tile = GDN_D * GDN_D * 2;
          g.stages = gdn_stages(lb, tile);
          CU(launch_k(gdn_step_kernel<true, __half>, grid, dim3(GDN_THREADS), gdn_smem_bytes(lb, tile), st, e->pdl,
                      g));
        } else {
          const int tile = GDN_D * GDN_D * 4;
          g.stages = gdn_stages(lb, tile);
          CU(launch_k(gdn_step_kernel<true, float>, grid, dim3(GDN_THREADS), gdn_smem_bytes(lb, tile), st, e->pdl,
                      g));
        }
      }
      ++gi;
    } else {
      {
        if ((rc = launch_gemm(st, L.w_in, ATT_IN, HIDDEN, e->xhi, lo(e->xlo), e->m_alloc, M, GEMM_STORE, e->proj,
                              ATT_IN, nullptr, nullptr, 0, e->err, 0, e, HSG_PROF_GEMM_IN, e->pdl)) != HSG_OK)
          return rc;
      }
      AttnArgs a{};
      a.slots = slots; a.lens = lens; a.starts = starts; a.nb = nb; a.lb = lb; a.max_slots = e->S;
      a.proj = e->proj; a.q_norm = L.q_norm; a.k_norm = L.k_norm; a.inv_freq = e->w.inv_freq; a.eps = eps;
      a.qbuf = e->qbuf; a.knew = e->knew; a.vnew = e->vnew;
      a.ring_k = e->ring_k + (size_t)ai * (e->S + 1) * e->ring_slot();
      a.ring_v = e->ring_v + (size_t)ai * (e->S + 1) * e->ring_slot();
      a.ring_pos = e->ring_pos;
      a.out_hi = e->ohi; a.out_lo = e->olo; a.out_raw = nullptr;
      a.write_ring = lb == 1;
      a.scale = 1.0f / 16.0f;  // 256^-1/2
      a.err = e->err;
      {
        ProfScope ps(e, HSG_PROF_ATTN_PREP);
        CU(launch_k(attn_prep_kernel, dim3(M), dim3(256), 0, st, e->pdl, a));
      }
      {
        ProfScope ps(e, HSG_PROF_RING_ATTN);
        if (lb == 1 && ring_decode_splits(nb))
          CU(launch_cluster(ring_decode_split_kernel, dim3(RDS_SPLIT, nb * ATT_HKV), dim3(RD_THREADS), RDS_SPLIT,
                            rds_smem_bytes(), st, e->pdl, e->ring_maps[ai][0], e->ring_maps[ai][1], e->new_maps[0],
                            e->new_maps[1], a));
        else if (lb == 1)
          CU(launch_k(ring_decode_kernel, dim3(std::min(SM_COUNT, nb * ATT_HKV)), dim3(RD_THREADS), rd_smem_bytes(),
                      st, e->pdl, e->ring_maps[ai][0], e->ring_maps[ai][1], e->new_maps[0], e->new_maps[1], a));
        else if (lb >= 32)
          CU(launch_k(ring_prefill_tc_kernel, dim3(nb, ATT_HKV, ATT_G * lb / PT_ROWS), dim3(PT_THREADS),
                      pt_smem_bytes(), st, e->pdl, e->ring_maps[ai][0], e->ring_maps[ai][1], e->new_maps[0],
                      e->new_maps[1], a));
        else if (lb >= 16)
          CU(launch_k(ring_prefill_kernel, dim3(nb, ATT_HKV, (ATT_G * lb + PF_ROWS - 1) / PF_ROWS), dim3(PF_THREADS),
                      pf_smem_bytes(), st, e->pdl, e->ring_maps[ai][0], e->ring_maps[ai][1], e->new_maps[0],
                      e->new_maps[1], a));
        else
          CU(launch_k(ring_attn_kernel<8>, dim3(nb, ATT_HKV, (ATT_G * lb + 7) / 8), dim3(ATT_THREADS),
                      attn_smem_bytes(8), st, e->pdl, a));
      }
      if (lb > 1) {
        ProfScope ps(e, HSG_PROF_RING_APPEND);
        CU(launch_k(ring_append_kernel, dim3(nb, ATT_HKV), dim3(ATT_D), 0, st, e->pdl, a));
      }
      ++ai;
    }
    {
      if ((rc = launch_gemm(st, L.w_out, HIDDEN, KEY_DIM, e->ohi, lo(e->olo), e->m_alloc, M, GEMM_ATOMIC, e->hidden,
                            HIDDEN, nullptr, nullptr, 0, e->err, 0, e, HSG_PROF_GEMM_OUT, e->pdl)) != HSG_OK)
        return rc;
    }
    {
      ProfScope ps(e, HSG_PROF_NORM);
      CU(launch_k(resid_norm_kernel, dim3(M), dim3(NORM_THREADS), 0, st, e->pdl, (const float*)e->hidden,
                  L.norm_post, eps, e->xhi, e->xlo, M));
    }
    {
      if ((rc = launch_gemm(st, L.w_gu, 2 * INTER, HIDDEN, e->xhi, lo(e->xlo), e->m_alloc, M, GEMM_SILU_MUL, nullptr,
                            0, e->ahi, e->alo, INTER, e->err, 0, e, HSG_PROF_GEMM_GU, e->pdl)) != HSG_OK)
        return rc;
    }
    {
      if ((rc = launch_gemm(st, L.w_down, HIDDEN, INTER, e->ahi, lo(e->alo), e->m_alloc, M, GEMM_ATOMIC, e->hidden,
                            HIDDEN, nullptr, nullptr, 0, e->err, 0, e, HSG_PROF_GEMM_DOWN, e->pdl)) != HSG_OK)
        return rc;
    }
    {
      ProfScope ps(e, HSG_PROF_NORM);
      const float* nxt = i + 1 < HSG_N_LAYERS ? e->w.layers[i + 1].norm_in : e->w.final_norm;
      CU(launch_k(resid_norm_kernel, dim3(M), dim3(NORM_THREADS), 0, st, e->pdl, (const float*)e->hidden, nxt, eps,
                  e->xhi, e->xlo, M));
    }
  }
  {
    if ((rc = launch_gemm(st, e->w.head_w1, N_ROLES * HEAD_E, HIDDEN, e->xhi, lo(e->xlo), e->m_alloc, M, GEMM_STORE,
                          e->hbuf, N_ROLES * HEAD_E, nullptr, nullptr, 0, e->err, 0, e, HSG_PROF_HEAD_GEMM, e->pdl)) != HSG_OK)
      return rc;
  }
  {
    ProfScope ps(e, HSG_PROF_HEAD);
    CU(launch_k(head_finish_kernel, dim3(M), dim3(256), 0, st, e->pdl, (const float*)e->hbuf, e->w.head_b1,
                e->w.head_ln_w, e->w.head_ln_b, e->w.head_w2, e->w.head_b2, e->cfg.head_ln_eps, e->probs, M));
  }
  {
    ProfScope ps(e, HSG_PROF_COMMIT);
    CU(launch_k(ring_commit_kernel, dim3((M + 255) / 256), dim3(256), 0, st, e->pdl, slots, lens, starts, nb, lb, e->S,
                e->ring_pos));
  }
  return HSG_OK;
}

static int check_shape(const hsg_engine* e, int nb, int lb) {
  if (!e) return fail(HSG_ERR_INVALID, "engine is NULL");
  if (lb < 1 || lb > MAX_LB) return fail(HSG_ERR_INVALID, "lb must be in [1, %d], got %d", MAX_LB, lb);
  if (nb < 1 || nb > e->S || nb * lb > e->max_tokens)
    return fail(HSG_ERR_INVALID, "nb must be in [1, max_slots=%d], got %d", e->S, nb);
  return HSG_OK;
}

// Host-side validation of a packed tick (the kernels also bound-check and report through the error flag).
static int validate_packed(const hsg_engine* e, const int64_t* packed, int nb, int lb) {
  if (!packed) return fail(HSG_ERR_INVALID, "packed is NULL");
  const int64_t* lens = packed + (size_t)nb * lb;
  const int64_t* slots = lens + nb;
  const int64_t* starts = slots + nb;
  std::vector<char> seen(e->S + 1, 0);
  for (int n = 0; n < nb; ++n) {
    if (lens[n] < 0 || lens[n] > lb) return fail(HSG_ERR_INVALID, "row %d: length %lld outside [0, %d]", n,
                                                 (long long)lens[n], lb);
    if (slots[n] < 0 || slots[n] > e->S) return fail(HSG_ERR_INVALID, "row %d: slot %lld outside [0, %d]", n,
                                                     (long long)slots[n], e->S);
    if (lens[n] > 0) {
      if (slots[n] == e->S) return fail(HSG_ERR_INVALID, "row %d: the scratch slot cannot carry tokens", n);
      if (seen[slots[n]]) return fail(HSG_ERR_INVALID, "slot %lld appears twice in one tick", (long long)slots[n]);
      seen[slots[n]] = 1;
      if (starts[n] < 0) return fail(HSG_ERR_INVALID, "row %d: negative start", n);
    }
    for (int t = 0; t < lens[n]; ++t) {
      const int64_t id = packed[(size_t)n * lb + t];
      if (id < 0 || id >= e->cfg.vocab) return fail(HSG_ERR_INVALID, "token id %lld outside [0, %d)",
                                                    (long long)id, e->cfg.vocab);
    }
  }
  return HSG_OK;
}

static int get_graph(hsg_engine* e, int nb, int lb, Bucket** out) {
  auto key = std::make_pair(nb, lb);
  auto it = e->graphs.find(key);
  if (it != e->graphs.end()) {
    *out = &it->second;
    return HSG_OK;
  }
  Bucket b;
  cudaGraph_t g = nullptr;
  e->launch_count = 0;
  CU(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_step(e, nb, lb);
  cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
  if (rc != HSG_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (ce != cudaSuccess) return fail(HSG_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(ce));
  ce = cudaGraphInstantiate(&b.exec, g, 0);
  cudaGraphDestroy(g);
  if (ce != cudaSuccess) return fail(HSG_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(ce));
  b.launches = e->launch_count;
  e->graphs[key] = b;
  *out = &e->graphs[key];
  return HSG_OK;
}

// One thread waits, with the bounded wait of every kernel here, on an mbarrier that nothing arrives on.
__global__ void bounded_wait_probe_kernel(int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_wait(&bar, 0, err, ERR_TIMEOUT_TMA);
  }
}

extern "C" {

int hsg_check_bounded_wait(int device, double* seconds) {
  CU(cudaSetDevice(device));
  cudaStream_t st = nullptr;
  int* err = nullptr;
  CU(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  cudaError_t ce = cudaMalloc(&err, sizeof(int));
  int code = -1;
  double s = 0.0;
  if (ce == cudaSuccess) ce = cudaMemsetAsync(err, 0, sizeof(int), st);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
  if (ce == cudaSuccess) {
    const auto t0 = std::chrono::steady_clock::now();
    bounded_wait_probe_kernel<<<1, 32, 0, st>>>(err);
    ce = cudaGetLastError();
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(&code, err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
    s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  }
  if (err) cudaFree(err);
  cudaStreamDestroy(st);
  if (ce != cudaSuccess) return fail(HSG_ERR_CUDA, "bounded-wait probe: %s", cudaGetErrorString(ce));
  if (seconds) *seconds = s;
  if (code != ERR_TIMEOUT_TMA)
    return fail(HSG_ERR_DEVICE, "bounded-wait probe ended without recording its timeout (code %d)", code);
  return HSG_OK;
}

const char* hsg_last_error(void) { return g_last_error.c_str(); }
const char* hsg_version(void) { return "hsg-b200 0.1 (sm_100a)"; }

int hsg_create(const hsg_config* cfg, const hsg_weights* w, int max_slots, int device, int flags, hsg_engine** out) {
  int rc;
  if (!out || !w) return fail(HSG_ERR_INVALID, "NULL argument");
  *out = nullptr;
  if ((rc = check_config(cfg)) != HSG_OK) return rc;
  if (max_slots < 1 || max_slots > 4096) return fail(HSG_ERR_INVALID, "max_slots must be in [1, 4096]");
  CU(cudaSetDevice(device));
  cudaDeviceProp prop;
  CU(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return fail(HSG_ERR_UNSUPPORTED, "device %d is sm_%d%d; the kernels are built for sm_100a",
                                    device, prop.major, prop.minor);
  if ((rc = set_kernel_attributes()) != HSG_OK) return rc;
  if ((rc = get_encoder()) != HSG_OK) return rc;
  hsg_engine* e = new hsg_engine();
  e->cfg = *cfg;
  e->w = *w;
  e->S = max_slots;
  e->device = device;
  e->flags = flags;
  e->n_gdn = 18;
  e->n_attn = 6;
  e->max_tokens = max_slots * MAX_LB;
  e->m_alloc = e->max_tokens + 256;
  const size_t S1 = (size_t)max_slots + 1, M = e->m_alloc;
#define TRY(x)                 \
  if ((rc = (x)) != HSG_OK) {  \
    hsg_destroy(e);            \
    return rc;                 \
  }
  e->rec_elem = (flags & HSG_FLAG_STATE_F32) ? 4 : 2;
  TRY(dalloc(e, &e->rec, (size_t)e->n_gdn * S1 * e->rec_slot() * e->rec_elem));
  TRY(dalloc(e, &e->conv, (size_t)e->n_gdn * S1 * e->conv_slot()));
  TRY(dalloc(e, &e->ring_k, (size_t)e->n_attn * S1 * e->ring_slot()));
  TRY(dalloc(e, &e->ring_v, (size_t)e->n_attn * S1 * e->ring_slot()));
  TRY(dalloc(e, &e->ring_pos, S1 * RING_COLS));
  TRY(dalloc(e, &e->packed, M + 3 * S1));
  TRY(dalloc(e, &e->hidden, M * HIDDEN));
  TRY(dalloc(e, &e->xhi, M * HIDDEN));
  TRY(dalloc(e, &e->xlo, M * HIDDEN));
  TRY(dalloc(e, &e->proj, M * GDN_IN));
  TRY(dalloc(e, &e->ohi, M * KEY_DIM));
  TRY(dalloc(e, &e->olo, M * KEY_DIM));
  TRY(dalloc(e, &e->ahi, M * INTER));
  TRY(dalloc(e, &e->alo, M * INTER));
  TRY(dalloc(e, &e->qbuf, M * ATT_HQ * ATT_D));
  TRY(dalloc(e, &e->knew, M * ATT_HKV * ATT_D));
  TRY(dalloc(e, &e->vnew, M * ATT_HKV * ATT_D));
  TRY(dalloc(e, &e->hbuf, M * N_ROLES * HEAD_E));
  TRY(dalloc(e, &e->probs, (size_t)N_ROLES * M * N_CLS));
  TRY(dalloc(e, &e->err, 1));
  for (int a = 0; a < e->n_attn; ++a) {
    const uint64_t rows = S1 * ATT_HKV * RING_COLS;
    TRY(make_decode_map(&e->ring_maps[a][0], e->ring_k + (size_t)a * S1 * e->ring_slot(), rows));
    TRY(make_decode_map(&e->ring_maps[a][1], e->ring_v + (size_t)a * S1 * e->ring_slot(), rows));
  }
  if (e->rec_elem == 2)
    for (int gi = 0; gi < e->n_gdn; ++gi) {
      TRY(make_state_map(&e->state_maps[gi], e->rec + (size_t)gi * S1 * e->rec_slot() * 2, (int64_t)S1));
      TRY(make_map_3d(&e->conv_maps[gi], e->conv + (size_t)gi * S1 * e->conv_slot(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                      4, KEY_DIM, 3, S1 * CONV_KEEP, KEY_DIM * 4, CONV_DIM * 4, GDN_D, 3, CONV_KEEP));
    }
  TRY(make_decode_map(&e->new_maps[0], e->knew, M * ATT_HKV));
  TRY(make_decode_map(&e->new_maps[1], e->vnew, M * ATT_HKV));
#undef TRY
  if (cudaMallocHost(&e->err_host, sizeof(int)) != cudaSuccess) {
    hsg_destroy(e);
    return fail(HSG_ERR_CUDA, "cudaMallocHost failed");
  }
  if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) {
    hsg_destroy(e);
    return fail(HSG_ERR_CUDA, "cudaStreamCreate failed");
  }
  // activation buffers start clean so padded GEMM rows never read uninitialised memory
  cudaMemsetAsync(e->xhi, 0, M * HIDDEN * 2, e->stream);
  cudaMemsetAsync(e->xlo, 0, M * HIDDEN * 2, e->stream);
  cudaMemsetAsync(e->ohi, 0, M * KEY_DIM * 2, e->stream);
  cudaMemsetAsync(e->olo, 0, M * KEY_DIM * 2, e->stream);
  cudaMemsetAsync(e->ahi, 0, M * INTER * 2, e->stream);
  cudaMemsetAsync(e->alo, 0, M * INTER * 2, e->stream);
  cudaMemsetAsync(e->err, 0, sizeof(int), e->stream);
  *out = e;
  rc = hsg_reset_all(e);
  if (rc != HSG_OK) {
    hsg_destroy(e);
    *out = nullptr;
  }
  return rc;
}

int hsg_destroy(hsg_engine* e) {
  if (!e) return HSG_OK;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (auto& kv : e->graphs)
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
  for (void* p : e->allocations) cudaFree(p);
  if (e->err_host) cudaFreeHost(e->err_host);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
  return HSG_OK;
}

void* hsg_stream(hsg_engine* e) { return e ? (void*)e->stream : nullptr; }

int hsg_synchronize(hsg_engine* e) {
  if (!e) return fail(HSG_ERR_INVALID, "engine is NULL");
  CU(cudaStreamSynchronize(e->stream));
  return HSG_OK;
}

int hsg_stage(hsg_engine* e, const int64_t* packed, int nb, int lb) {
  int rc;
  if ((rc = check_shape(e, nb, lb)) != HSG_OK) return rc;
  if ((rc = validate_packed(e, packed, nb, lb)) != HSG_OK) return rc;
  CU(cudaSetDevice(e->device));
  CU(cudaMemcpyAsync(e->packed, packed, ((size_t)nb * lb + 3 * nb) * sizeof(int64_t), cudaMemcpyHostToDevice,
                     e->stream));
  return HSG_OK;
}

int hsg_launch(hsg_engine* e, const int64_t* packed_dev, int nb, int lb) {
  int rc;
  if ((rc = check_shape(e, nb, lb)) != HSG_OK) return rc;
  CU(cudaSetDevice(e->device));
  if (packed_dev)
    CU(cudaMemcpyAsync(e->packed, packed_dev, ((size_t)nb * lb + 3 * nb) * sizeof(int64_t),
                       cudaMemcpyDeviceToDevice, e->stream));
  Bucket* b = nullptr;
  if ((rc = get_graph(e, nb, lb, &b)) != HSG_OK) return rc;
  CU(cudaGraphLaunch(b->exec, e->stream));
  return HSG_OK;
}

int hsg_fetch(hsg_engine* e, int nb, int lb, float* out_probs) {
  int rc;
  if ((rc = check_shape(e, nb, lb)) != HSG_OK) return rc;
  CU(cudaSetDevice(e->device));
  if (out_probs)
    CU(cudaMemcpyAsync(out_probs, e->probs, (size_t)N_ROLES * nb * lb * N_CLS * sizeof(float),
                       cudaMemcpyDeviceToHost, e->stream));
  CU(cudaMemcpyAsync(e->err_host, e->err, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
  CU(cudaStreamSynchronize(e->stream));
  if (*e->err_host) {
    const int code = *e->err_host;
    CU(cudaMemsetAsync(e->err, 0, sizeof(int), e->stream));
    CU(cudaStreamSynchronize(e->stream));
    return fail(HSG_ERR_DEVICE, "device error %d: %s", code, device_error_text(code));
  }
  return HSG_OK;
}

int hsg_step(hsg_engine* e, const int64_t* packed, int nb, int lb, float* out_probs) {
  int rc;
  if ((rc = hsg_stage(e, packed, nb, lb)) != HSG_OK) return rc;
  if ((rc = hsg_launch(e, nullptr, nb, lb)) != HSG_OK) return rc;
  return hsg_fetch(e, nb, lb, out_probs);
}

int hsg_launches_per_step(const hsg_engine* e, int nb, int lb) {
  if (check_shape(e, nb, lb) != HSG_OK) return -1;
  auto it = e->graphs.find(std::make_pair(nb, lb));
  return it == e->graphs.end() ? -1 : it->second.launches;
}

int hsg_profile_step(hsg_engine* e, const int64_t* packed, int nb, int lb, float* out_probs, float* kernel_ms,
                     int* launches) {
  int rc;
  if ((rc = hsg_stage(e, packed, nb, lb)) != HSG_OK) return rc;
  e->profiling = true;
  e->events.clear();
  e->event_class.clear();
  e->launch_count = 0;
  rc = enqueue_step(e, nb, lb);
  e->profiling = false;
  if (rc != HSG_OK) return rc;
  if ((rc = hsg_fetch(e, nb, lb, out_probs)) != HSG_OK) return rc;
  for (size_t i = 0; i + 1 < e->events.size(); i += 2) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e->events[i], e->events[i + 1]);
    const int c = e->event_class[i];
    if (c >= 0 && c < HSG_PROF_N) {
      if (kernel_ms) kernel_ms[c] += ms;
      if (launches) launches[c] += 1;
    }
  }
  for (cudaEvent_t ev : e->events) cudaEventDestroy(ev);
  e->events.clear();
  e->event_class.clear();
  return HSG_OK;
}

int hsg_reset_all(hsg_engine* e) {
  if (!e) return fail(HSG_ERR_INVALID, "engine is NULL");
  CU(cudaSetDevice(e->device));
  const size_t S1 = (size_t)e->S + 1;
  CU(cudaMemsetAsync(e->rec, 0, (size_t)e->n_gdn * S1 * e->rec_slot() * e->rec_elem, e->stream));
  CU(cudaMemsetAsync(e->conv, 0, (size_t)e->n_gdn * S1 * e->conv_slot() * sizeof(float), e->stream));
  CU(cudaMemsetAsync(e->ring_k, 0, (size_t)e->n_attn * S1 * e->ring_slot() * sizeof(__half), e->stream));
  CU(cudaMemsetAsync(e->ring_v, 0, (size_t)e->n_attn * S1 * e->ring_slot() * sizeof(__half), e->stream));
  CU(cudaMemsetAsync(e->ring_pos, 0xFF, S1 * RING_COLS * sizeof(int64_t), e->stream));  // -1
  CU(cudaStreamSynchronize(e->stream));
  return HSG_OK;
}

// (pool base, bytes per slot, layers) of the four per-layer pools and ring_pos (one "layer").
struct PoolView {
  char* base;
  size_t slot_bytes;
  int layers;
};

static void pool_views(const hsg_engine* e, PoolView v[5]) {
  v[0] = {e->rec, e->rec_slot() * e->rec_elem, e->n_gdn};
  v[1] = {(char*)e->conv, e->conv_slot() * sizeof(float), e->n_gdn};
  v[2] = {(char*)e->ring_k, e->ring_slot() * sizeof(__half), e->n_attn};
  v[3] = {(char*)e->ring_v, e->ring_slot() * sizeof(__half), e->n_attn};
  v[4] = {(char*)e->ring_pos, RING_COLS * sizeof(int64_t), 1};
}

size_t hsg_slot_state_bytes(const hsg_engine* e) {
  if (!e) return 0;
  PoolView v[5];
  pool_views(e, v);
  size_t total = 0;
  for (auto& p : v) total += p.slot_bytes * p.layers;
  return total;
}

int hsg_reset_slot(hsg_engine* e, int slot) {
  if (!e) return fail(HSG_ERR_INVALID, "engine is NULL");
  if (slot < 0 || slot >= e->S) return fail(HSG_ERR_INVALID, "slot %d outside [0, %d)", slot, e->S);
  CU(cudaSetDevice(e->device));
  PoolView v[5];
  pool_views(e, v);
  const size_t S1 = (size_t)e->S + 1;
  for (int i = 0; i < 5; ++i) {
    const size_t pitch = v[i].slot_bytes * S1;
    CU(cudaMemset2DAsync(v[i].base + slot * v[i].slot_bytes, pitch, i == 4 ? 0xFF : 0, v[i].slot_bytes,
                         v[i].layers, e->stream));
  }
  CU(cudaStreamSynchronize(e->stream));
  return HSG_OK;
}

static int copy_slot(hsg_engine* e, int slot, char* buf, bool to_buf) {
  if (!e || !buf) return fail(HSG_ERR_INVALID, "NULL argument");
  if (slot < 0 || slot >= e->S) return fail(HSG_ERR_INVALID, "slot %d outside [0, %d)", slot, e->S);
  CU(cudaSetDevice(e->device));
  PoolView v[5];
  pool_views(e, v);
  const size_t S1 = (size_t)e->S + 1;
  size_t off = 0;
  for (int i = 0; i < 5; ++i) {
    const size_t pitch = v[i].slot_bytes * S1, w = v[i].slot_bytes;
    char* pool = v[i].base + slot * w;
    if (to_buf) CU(cudaMemcpy2DAsync(buf + off, w, pool, pitch, w, v[i].layers, cudaMemcpyDeviceToDevice, e->stream));
    else CU(cudaMemcpy2DAsync(pool, pitch, buf + off, w, w, v[i].layers, cudaMemcpyDeviceToDevice, e->stream));
    off += w * v[i].layers;
  }
  CU(cudaStreamSynchronize(e->stream));
  return HSG_OK;
}

int hsg_snapshot_slot(hsg_engine* e, int slot, void* dst) { return copy_slot(e, slot, (char*)dst, true); }
int hsg_restore_slot(hsg_engine* e, int slot, const void* src) { return copy_slot(e, slot, (char*)src, false); }

int hsg_get_pools(const hsg_engine* e, hsg_pools* out) {
  if (!e || !out) return fail(HSG_ERR_INVALID, "NULL argument");
  out->rec = e->rec;
  out->rec_dtype = e->rec_elem == 2 ? HSG_STATE_F16 : HSG_STATE_F32;
  out->conv = e->conv;
  out->ring_k = e->ring_k;
  out->ring_v = e->ring_v;
  out->ring_pos = e->ring_pos;
  out->max_slots = e->S;
  out->n_gdn = e->n_gdn;
  out->n_attn = e->n_attn;
  return HSG_OK;
}

// ---- isolated kernels ---------------------------------------------------------------------------------------------
int hsg_gdn_step(const void* packed, const float* a, const float* b, const float* A_log, const float* dt_bias,
                 void* state, int state_dtype, const int64_t* slots, const int64_t* lens, int n, int lb,
                 int max_slots, float* o, int* err, void* stream) {
  if (!packed || !a || !b || !A_log || !dt_bias || !state || !slots || !lens || !o)
    return fail(HSG_ERR_INVALID, "NULL argument");
  if (n < 1 || lb < 1 || lb > MAX_LB || max_slots < 1) return fail(HSG_ERR_INVALID, "bad shape n=%d lb=%d", n, lb);
  if (reinterpret_cast<uintptr_t>(state) & 15) return fail(HSG_ERR_INVALID, "state must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(packed) | reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15)
    return fail(HSG_ERR_INVALID, "packed, a and b must be 16-byte aligned");
  if (state_dtype != HSG_STATE_F32 && state_dtype != HSG_STATE_F16)
    return fail(HSG_ERR_INVALID, "state_dtype must be HSG_STATE_F32 or HSG_STATE_F16");
  int rc;
  if ((rc = set_kernel_attributes()) != HSG_OK) return rc;
  GdnArgs g{};
  g.slots = slots; g.lens = lens; g.nb = n; g.lb = lb; g.max_slots = max_slots;
  g.packed = static_cast<const __nv_bfloat16*>(packed);
  g.a_raw = a; g.b_raw = b; g.o_raw = o;
  g.A_log = A_log; g.dt_bias = dt_bias; g.state = state; g.err = err;
  const dim3 grid(GDN_H, std::min(n, GDN_CTAS_PER_HEAD));
  if (state_dtype == HSG_STATE_F32 && n <= GDNS_MAX_ROWS) {
    // a small fp32 batch: one CTA per 32-column slice of each (row, head) state, one wave
    gdn_cols_kernel<float><<<dim3(GDNS_SLICES, GDN_H, n), GDNS_THREADS, 0, (cudaStream_t)stream>>>(g);
  } else if (state_dtype == HSG_STATE_F16 && lb <= GDNT_MAX_LB) {
    GdntMaps maps;
    if ((rc = make_state_map(&maps.state, state, (int64_t)max_slots + 1)) != HSG_OK) return rc;
    if ((rc = make_map_3d(&maps.in0, packed, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, KEY_DIM, 3, (uint64_t)n * lb,
                          KEY_DIM * 2, CONV_DIM * 2, GDN_D, 3, lb)) != HSG_OK)
      return rc;
    maps.in1 = maps.in2 = maps.in0;
    g.stages = gdnt_stages(lb, false);
    if (lb == 1)
      gdn_tc_kernel<false, 4><<<grid, GDNT_THREADS, gdnt_smem_bytes(lb, false), (cudaStream_t)stream>>>(maps, g);
    else
      gdn_tc_kernel<false, 3><<<grid, GDNT_THREADS, gdnt_smem_bytes(lb, false), (cudaStream_t)stream>>>(maps, g);
  } else if (state_dtype == HSG_STATE_F16 && lb % GDNC_SUB == 0) {  // 32 or 64 tokens: the chunked kernel
    GdntMaps maps;
    if ((rc = make_state_map(&maps.state, state, (int64_t)max_slots + 1)) != HSG_OK) return rc;
    if ((rc = make_map_3d(&maps.in0, packed, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, KEY_DIM, 3, (uint64_t)n * lb,
                          KEY_DIM * 2, CONV_DIM * 2, GDN_D, 3, lb)) != HSG_OK)
      return rc;
    maps.in1 = maps.in2 = maps.in0;
    g.stages = gdnc_stages(lb, false);
    gdn_chunk_kernel<false><<<grid, GDNT_THREADS, gdnc_smem_bytes(lb, false), (cudaStream_t)stream>>>(maps, g);
  } else if (state_dtype == HSG_STATE_F16) {
    const int tile = GDN_D * GDN_D * 2;
    g.stages = gdn_stages(lb, tile);
    gdn_step_kernel<false, __half><<<grid, GDN_THREADS, gdn_smem_bytes(lb, tile), (cudaStream_t)stream>>>(g);
  } else {
    const int tile = GDN_D * GDN_D * 4;
    g.stages = gdn_stages(lb, tile);
    gdn_step_kernel<false, float><<<grid, GDN_THREADS, gdn_smem_bytes(lb, tile), (cudaStream_t)stream>>>(g);
  }
  CU(cudaGetLastError());
  return HSG_OK;
}

int hsg_ring_attention(const float* q, void* ring_k, void* ring_v, const void* new_k, const void* new_v,
                       const int64_t* ring_pos, const int64_t* slots, const int64_t* starts, const int64_t* lens,
                       int n, int lb, int max_slots, float scale, float* out, int write_ring, int* err, void* stream) {
  if (!q || !ring_k || !ring_v || !new_k || !new_v || !ring_pos || !slots || !starts || !lens || !out)
    return fail(HSG_ERR_INVALID, "NULL argument");
  if (n < 1 || lb < 1 || lb > MAX_LB || max_slots < 1) return fail(HSG_ERR_INVALID, "bad shape n=%d lb=%d", n, lb);
  if (write_ring && lb != 1) return fail(HSG_ERR_INVALID, "write_ring needs lb == 1");
  for (const void* p : {(const void*)ring_k, (const void*)ring_v, new_k, new_v})
    if (reinterpret_cast<uintptr_t>(p) & 15) return fail(HSG_ERR_INVALID, "K/V pointers must be 16-byte aligned");
  int rc;
  if ((rc = set_kernel_attributes()) != HSG_OK) return rc;
  AttnArgs a{};
  a.slots = slots; a.lens = lens; a.starts = starts; a.nb = n; a.lb = lb; a.max_slots = max_slots;
  a.qbuf = const_cast<float*>(q);
  a.knew = static_cast<__half*>(const_cast<void*>(new_k));
  a.vnew = static_cast<__half*>(const_cast<void*>(new_v));
  a.ring_k = static_cast<__half*>(ring_k);
  a.ring_v = static_cast<__half*>(ring_v);
  a.ring_pos = const_cast<int64_t*>(ring_pos);
  a.out_raw = out;
  a.write_ring = write_ring;
  a.scale = scale;
  a.err = err;
  cudaStream_t st = (cudaStream_t)stream;
  if (lb == 1) {
    CUtensorMap rk, rv, nk, nv;
    const uint64_t ring_rows = ((uint64_t)max_slots + 1) * ATT_HKV * RING_COLS;
    if ((rc = make_decode_map(&rk, ring_k, ring_rows)) != HSG_OK || (rc = make_decode_map(&rv, ring_v, ring_rows)) ||
        (rc = make_decode_map(&nk, new_k, (uint64_t)n * ATT_HKV)) ||
        (rc = make_decode_map(&nv, new_v, (uint64_t)n * ATT_HKV)))
      return rc;
    if (ring_decode_splits(n))
      CU(launch_cluster(ring_decode_split_kernel, dim3(RDS_SPLIT, n * ATT_HKV), dim3(RD_THREADS), RDS_SPLIT,
                        rds_smem_bytes(), st, false, rk, rv, nk, nv, a));
    else
      ring_decode_kernel<<<dim3(std::min(SM_COUNT, n * ATT_HKV)), RD_THREADS, rd_smem_bytes(), st>>>(rk, rv, nk, nv,
                                                                                                   a);
  } else if (lb >= 16) {
    CUtensorMap rk, rv, nk, nv;
    const uint64_t ring_rows = ((uint64_t)max_slots + 1) * ATT_HKV * RING_COLS;
    if ((rc = make_decode_map(&rk, ring_k, ring_rows)) != HSG_OK || (rc = make_decode_map(&rv, ring_v, ring_rows)) ||
        (rc = make_decode_map(&nk, new_k, (uint64_t)n * ATT_HKV * lb)) ||
        (rc = make_decode_map(&nv, new_v, (uint64_t)n * ATT_HKV * lb)))
      return rc;
    if (lb >= 32)
      ring_prefill_tc_kernel<<<dim3(n, ATT_HKV, ATT_G * lb / PT_ROWS), PT_THREADS, pt_smem_bytes(), st>>>(rk, rv, nk,
                                                                                                        nv, a);
    else
      ring_prefill_kernel<<<dim3(n, ATT_HKV, (ATT_G * lb + PF_ROWS - 1) / PF_ROWS), PF_THREADS, pf_smem_bytes(),
                            st>>>(rk, rv, nk, nv, a);
  }
  else ring_attn_kernel<8><<<dim3(n, ATT_HKV, (ATT_G * lb + 7) / 8), ATT_THREADS, attn_smem_bytes(8), st>>>(a);
  CU(cudaGetLastError());
  return HSG_OK;
}

int hsg_gemm(const void* w, int n, int k, const void* x_hi, const void* x_lo, int m, int m_alloc, float* y,
             void* act_hi, void* act_lo, int mode, int splits, int* err, void* stream) {
  if (!w || !x_hi) return fail(HSG_ERR_INVALID, "NULL argument");
  if (n <= 0 || n % 128 || k <= 0 || k % 64 || m < 1 || m_alloc < m) return fail(HSG_ERR_INVALID, "bad GEMM shape");
  if (mode < 0 || mode > 2) return fail(HSG_ERR_INVALID, "bad mode %d", mode);
  if (mode != GEMM_SILU_MUL && !y) return fail(HSG_ERR_INVALID, "y is NULL");
  if (mode == GEMM_SILU_MUL && (!act_hi || !act_lo)) return fail(HSG_ERR_INVALID, "act_hi/act_lo are NULL");
  int rc;
  if ((rc = set_kernel_attributes()) != HSG_OK) return rc;
  return launch_gemm((cudaStream_t)stream, w, n, k, x_hi, x_lo, m_alloc, m, mode, y, n,
                     static_cast<__nv_bfloat16*>(act_hi), static_cast<__nv_bfloat16*>(act_lo), n / 2, err, splits);
}

}  // extern "C"

// ---- GEMM without allocation --------------------------------------------------------------------------------------
// Some callers cannot allocate device memory on their call path. A host whose caching allocator (PyTorch's, for one)
// already holds the GPU's free memory can see cudaMalloc fail although that allocator has room, and cudaFree waits
// for the whole device, which would stall every other stream of a serving loop that must answer within milliseconds.
// hsg_gemm_f32_noalloc therefore takes fp32 activations and splits them into the bf16 (hi, lo) operand pair inside a
// scratch area that is part of the library image, so the call allocates nothing. No element of the area needs to
// start at zero: the split kernel writes every element the GEMM then reads, in stream order, in the same call.
static __device__ __align__(256) __nv_bfloat16 g_noalloc_operands[2 * (size_t)HSG_NOALLOC_MAX_ELEMS];

namespace {
constexpr int kNoallocMaxDevices = 64;

// Per device: the CUDA context in which the scratch address was looked up and the GEMM kernels' shared-memory
// attributes were set, and that address. A call compares the device's current context with the recorded one and
// repeats the set-up when they differ (a cudaDeviceReset or a rebuilt primary context loads the module again, which
// may move the scratch area and drops the attributes), so the address a kernel is given always belongs to the live
// context. The fast path reads two atomics and takes no lock; the mutex only serialises the set-up itself.
struct NoallocDevice {
  std::atomic<void*> ctx{nullptr};
  std::atomic<__nv_bfloat16*> base{nullptr};
};
NoallocDevice g_noalloc[kNoallocMaxDevices];
std::mutex g_noalloc_mu;
PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;

int current_context(void** out) {
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && fn)
      g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
  });
  if (!g_ctx_current) return fail(HSG_ERR_CUDA, "cuCtxGetCurrent is unavailable");
  CUcontext c = nullptr;
  if (g_ctx_current(&c) != CUDA_SUCCESS || !c) return fail(HSG_ERR_CUDA, "no current CUDA context");
  *out = c;
  return HSG_OK;
}

// The current device's copy of the scratch area. The first call in a context sets the two GEMM kernels' dynamic
// shared-memory limit and resolves the area's address with cudaGetSymbolAddress; that call may also be where the
// CUDA runtime loads the library's device code (lazy module loading) and so places the area: the one call of this
// entry point that can allocate.
int noalloc_scratch(__nv_bfloat16** out) {
  int dev = 0;
  CU(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoallocMaxDevices)
    return fail(HSG_ERR_UNSUPPORTED, "device ordinal %d is beyond the %d the scratch table covers", dev,
                kNoallocMaxDevices);
  int rc;
  void* ctx = nullptr;
  if ((rc = current_context(&ctx)) != HSG_OK) return rc;
  NoallocDevice& d = g_noalloc[dev];
  if (d.ctx.load(std::memory_order_acquire) == ctx) {
    *out = d.base.load(std::memory_order_relaxed);
    return HSG_OK;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (d.ctx.load(std::memory_order_acquire) != ctx) {
    CU(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX));
    CU(cudaFuncSetAttribute(gemm_pc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX));
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_operands);
    if (e != cudaSuccess || !p)
      return fail(HSG_ERR_CUDA, "cudaGetSymbolAddress of the GEMM scratch area failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    d.base.store(static_cast<__nv_bfloat16*>(p), std::memory_order_relaxed);
    d.ctx.store(ctx, std::memory_order_release);
  }
  *out = d.base.load(std::memory_order_relaxed);
  return HSG_OK;
}

// x [count] fp32 -> hi = bf16(x), lo = bf16(x - hi); count is a multiple of 4 and x is 16-byte aligned.
__global__ void __launch_bounds__(256) split_operand_kernel(const float4* __restrict__ x, __nv_bfloat162* hi,
                                                            __nv_bfloat162* lo, int64_t count4) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = x[i];
    __nv_bfloat16 h0, h1, h2, h3, l0, l1, l2, l3;
    split_bf16(v.x, h0, l0);
    split_bf16(v.y, h1, l1);
    split_bf16(v.z, h2, l2);
    split_bf16(v.w, h3, l3);
    hi[2 * i] = __halves2bfloat162(h0, h1);
    hi[2 * i + 1] = __halves2bfloat162(h2, h3);
    lo[2 * i] = __halves2bfloat162(l0, l1);
    lo[2 * i + 1] = __halves2bfloat162(l2, l3);
  }
}
}  // namespace

extern "C" int hsg_gemm_f32_noalloc(const void* w, int n, int k, const float* x, int m, float* y, void* act_hi,
                                    void* act_lo, int mode, int splits, int* err, void* stream) {
  if (!w || !x) return fail(HSG_ERR_INVALID, "NULL argument");
  if (n <= 0 || n % 128 || k <= 0 || k % 64 || m < 1) return fail(HSG_ERR_INVALID, "bad GEMM shape");
  if ((int64_t)m * k > HSG_NOALLOC_MAX_ELEMS)
    return fail(HSG_ERR_INVALID, "m * k = %lld exceeds the scratch limit HSG_NOALLOC_MAX_ELEMS = %d elements",
                (long long)m * k, HSG_NOALLOC_MAX_ELEMS);
  if (reinterpret_cast<uintptr_t>(x) & 15) return fail(HSG_ERR_INVALID, "x must be 16-byte aligned");
  if (mode < 0 || mode > 2) return fail(HSG_ERR_INVALID, "bad mode %d", mode);
  if (mode != GEMM_SILU_MUL && !y) return fail(HSG_ERR_INVALID, "y is NULL");
  if (mode == GEMM_SILU_MUL && (!act_hi || !act_lo)) return fail(HSG_ERR_INVALID, "act_hi/act_lo are NULL");
  int rc;
  __nv_bfloat16* hi = nullptr;
  if ((rc = noalloc_scratch(&hi)) != HSG_OK) return rc;
  __nv_bfloat16* lo = hi + HSG_NOALLOC_MAX_ELEMS;
  const int64_t count4 = (int64_t)m * k / 4;
  const int64_t want = (count4 + 255) / 256;
  const int blocks = want < 8 * SM_COUNT ? (int)want : 8 * SM_COUNT;
  cudaStream_t st = (cudaStream_t)stream;
  split_operand_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const float4*>(x),
                                               reinterpret_cast<__nv_bfloat162*>(hi),
                                               reinterpret_cast<__nv_bfloat162*>(lo), count4);
  CU(cudaGetLastError());
  return launch_gemm(st, w, n, k, hi, lo, m, m, mode, y, n, static_cast<__nv_bfloat16*>(act_hi),
                     static_cast<__nv_bfloat16*>(act_lo), n / 2, err, splits);
}
