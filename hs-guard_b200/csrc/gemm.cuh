// Weight-streaming GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
//   Y[t, n] (+)= sum_k X[t, k] * W[n, k]        X: activations [tokens, K], W: weights [N, K], both bf16 K-major
//
// "Swap-AB" orientation: the 128 weight rows of a tile sit on the MMA's M side and the tokens on its N side, so a
// tile streams a 128-row slab of W once from HBM while the (small, L2-resident) activation block is re-read. The
// activation operand is given as two bf16 matrices (hi, lo) with hi + lo ~= the fp32 activation; both are
// accumulated into the same TMEM accumulator, which makes the product accurate to near fp32 against bf16 weights.
//
// Roles in a 128-thread CTA: thread 0 issues the TMA loads (a STAGES-deep ring of shared-memory buffers), thread 32
// issues tcgen05.mma and commits each stage back to the producer, then all four warps drain TMEM in the epilogue
// (warp w owns accumulator lanes 32w..32w+31 = weight rows). Every wait is bounded and reports through `err`.
#pragma once
#include "common.cuh"

namespace hsg {

enum GemmMode : int {
  GEMM_STORE = 0,     // Y[t, n] = acc                      (fp32)
  GEMM_ATOMIC = 1,    // Y[t, n] += acc  (split-K partial sums and residual accumulation, fp32 red.add)
  GEMM_SILU_MUL = 2,  // W rows interleaved [64 gate | 64 up] per tile: act[t, f] = silu(g) * u as a bf16 hi/lo pair
};

struct GemmArgs {
  int k_blocks_per_split;  // 64-wide K blocks handled by one CTA
  int k_blocks_total;
  int tn;                  // tokens per CTA (multiple of 16, <= 256)
  int use_lo;              // accumulate the lo half of the activation split
  int m_store;             // token rows written by the epilogue (rows >= m_store are skipped)
  int stages;
  int mode;
  float* y;                // GEMM_STORE / GEMM_ATOMIC output, row stride ldy
  int ldy;
  __nv_bfloat16* act_hi;   // GEMM_SILU_MUL output pair, row stride ld_act
  __nv_bfloat16* act_lo;
  int ld_act;
  int* err;
};

constexpr int GEMM_THREADS = 128;
constexpr int GEMM_BK = 64;                       // K elements per stage (128 bytes: one swizzle row)
constexpr int GEMM_A_BYTES = 128 * GEMM_BK * 2;   // 16 KB weight tile

__host__ __device__ inline int gemm_stage_bytes(int tn, int use_lo) {
  return GEMM_A_BYTES + (use_lo ? 2 : 1) * tn * GEMM_BK * 2;
}

// grid: x = token block, y = weight tile (128 rows), z = K split.
__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_xhi,
               const __grid_constant__ CUtensorMap tm_xlo, const GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t gemm_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = args.stages;
  const int stage_bytes = gemm_stage_bytes(args.tn, args.use_lo);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* done = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* progress = reinterpret_cast<int*>(tmem_slot + 1);   // [0] loads issued, [1] stages consumed by the MMA
  float* xchg = reinterpret_cast<float*>(tmem_slot + 4);  // 64 x 16 fp32 exchange buffer (SILU_MUL epilogue)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tok0 = blockIdx.x * args.tn;
  const int wrow0 = blockIdx.y * 128;
  const int kb0 = blockIdx.z * args.k_blocks_per_split;
  const int kb1 = min(kb0 + args.k_blocks_per_split, args.k_blocks_total);
  const int nk = kb1 - kb0;
  uint32_t ncols = 32;
  while (ncols < (uint32_t)args.tn) ncols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    progress[0] = progress[1] = 0;
    fence_barrier_init();
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_xhi);
    if (args.use_lo) prefetch_tmap(&tm_xlo);
  }
  if (warp == 0) tmem_alloc(tmem_slot, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (threadIdx.x == 0) {
    // ---- TMA producer ----
    const uint32_t bytes = stage_bytes;
    for (int i = 0; i < nk && ok; ++i) {
      const int s = i % S, r = i / S;
      if (r > 0) ok = mbar_wait(&empty[s], (r - 1) & 1, args.err, ERR_TIMEOUT_MMA);
      if (!ok) break;
      uint8_t* a = smem + s * stage_bytes;
      uint8_t* bh = a + GEMM_A_BYTES;
      uint8_t* bl = bh + args.tn * GEMM_BK * 2;
      const int kx = (kb0 + i) * GEMM_BK;
      mbar_arrive_expect_tx(&full[s], bytes);
      tma_load_2d(a, &tm_w, kx, wrow0, &full[s]);
      tma_load_2d(bh, &tm_xhi, kx, tok0, &full[s]);
      if (args.use_lo) tma_load_2d(bl, &tm_xlo, kx, tok0, &full[s]);
      progress[0] = i + 1;
    }
  } else if (threadIdx.x == 32) {
    // ---- MMA issuer ----
    const uint32_t idesc = idesc_bf16(128, args.tn);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S, r = i / S;
      if (!mbar_wait(&full[s], r & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
      tc_fence_after();
      const uint32_t a = smem_u32(smem + s * stage_bytes);
      const uint32_t bh = a + GEMM_A_BYTES;
      const uint32_t bl = bh + args.tn * GEMM_BK * 2;
#pragma unroll
      for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
        const uint64_t da = sw128_desc(a + kk * 32);
        mma_bf16(tmem, da, sw128_desc(bh + kk * 32), idesc, (i > 0 || kk > 0) ? 1u : 0u);
        if (args.use_lo) mma_bf16(tmem, da, sw128_desc(bl + kk * 32), idesc, 1u);
      }
      mma_commit(&empty[s]);
      progress[1] = i + 1;
    }
    mma_commit(done);
  }
  __syncwarp();
  // ---- epilogue: every warp waits for the accumulator ----
  const bool have = __syncthreads_and(mbar_wait(done, 0, args.err, ERR_TIMEOUT_MMA));
  tc_fence_after();
  if (have && nk > 0) {
    const int row = warp * 32 + lane;  // accumulator lane == weight row within the tile
    const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
    for (int c = 0; c < args.tn; c += 16) {
      float v[16];
      tmem_ld16(lane_base + c, v);
      if (args.mode == GEMM_SILU_MUL) {
        // rows 0..63 hold gate features, rows 64..127 the matching up features
        __syncthreads();
        if (warp >= 2) {
#pragma unroll
          for (int j = 0; j < 16; ++j) xchg[(row - 64) * 16 + j] = v[j];
        }
        __syncthreads();
        if (warp < 2) {
          const int f = blockIdx.y * 64 + row;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int t = tok0 + c + j;
            if (t < args.m_store) {
              const float a = silu(v[j]) * xchg[row * 16 + j];
              __nv_bfloat16 hi, lo;
              split_bf16(a, hi, lo);
              args.act_hi[(size_t)t * args.ld_act + f] = hi;
              args.act_lo[(size_t)t * args.ld_act + f] = lo;
            }
          }
        }
      } else {
        const int n = wrow0 + row;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int t = tok0 + c + j;
          if (t < args.m_store) {
            float* p = args.y + (size_t)t * args.ldy + n;
            if (args.mode == GEMM_ATOMIC) atomicAdd(p, v[j]);
            else *p = v[j];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    // Error path only: loads the MMA never consumed may still be in flight; wait for them (bounded) before exit.
    for (int i = progress[1]; i < progress[0]; ++i) mbar_wait(&full[i % S], (i / S) & 1, args.err, ERR_TIMEOUT_TMA);
  }
  __syncwarp();
  if (warp == 0) tmem_dealloc(tmem, ncols);
}

}  // namespace hsg
