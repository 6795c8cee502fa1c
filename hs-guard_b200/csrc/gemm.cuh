// Weight-streaming GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA.
//
//   Y[t, n] (+)= sum_k X[t, k] * W[n, k]        X: activations [tokens, K], W: weights [N, K], both bf16 K-major
//
// "Swap-AB" orientation: the 128 weight rows of a tile sit on the MMA's M side and the tokens on its N side, so a
// tile streams a 128-row slab of W once from HBM while the (small, L2-resident) activation block is re-read. The
// activation operand is given as two bf16 matrices (hi, lo) with hi + lo ~= the fp32 activation; both are
// accumulated into the same TMEM accumulator, which makes the product accurate to near fp32 against bf16 weights.
//
// Roles in a 256-thread CTA: thread 0 issues the TMA loads (a STAGES-deep ring of shared-memory buffers), thread 32
// issues tcgen05.mma and commits each stage back to the producer, then all eight warps drain TMEM into a
// shared-memory tile that one TMA bulk store (or bulk reduce-add, for split-K partial sums accumulated into the fp32
// residual stream) writes out: warps w and w + 4 share accumulator lanes 32 (w % 4) .. + 31 (= weight rows) and
// take one half of the token columns each, so every scheduler has two warps to overlap the epilogue's latencies. Before the dependency
// wait of programmatic dependent launch the CTA sets up its barriers and TMEM, requests its first weight tiles and
// asks L2 to prefetch the rest of its weight slab. Every wait is bounded and reports through `err`.
#pragma once
#include "common.cuh"

namespace hsg {

enum GemmMode : int {
  GEMM_STORE = 0,     // Y[t, n] = acc                      (fp32)
  GEMM_ATOMIC = 1,    // Y[t, n] += acc  (TMA bulk reduce-add in L2; split-K partial sums, residual accumulation)
  GEMM_SILU_MUL = 2,  // W rows in (gate, up) pairs: act[t, f] = silu(gate_f) * up_f as a bf16 hi/lo pair
  GEMM_CONV = 3,      // the fused GDN input projection (persistent kernel only): as GEMM_STORE, with the causal conv
                      // + SiLU of the q | k | v rows applied along each request's tokens and the conv history kept
};
// Per-launch inputs of GEMM_CONV: request r covers tokens r * lb .. r * lb + lb - 1 (lb a multiple of 32), holds
// lens[r] valid tokens and belongs to slots[r]; pool = the layer's conv history [slots + 1][3][6144] fp32 (raw
// inputs 3, 2, 1 tokens before a request's first), w = the conv taps [6144] float4 (x: 3 tokens back .. w: the token).
struct GemmConv {
  const int64_t* lens;
  const int64_t* slots;
  float* pool;
  const float* w;
  int lb, max_slots;
};

struct GemmArgs {
  int k_blocks_per_split;  // 64-wide K blocks handled by one CTA
  int k_blocks_total;
  int tn;                  // tokens per CTA (multiple of 16, <= 256)
  int use_lo;              // accumulate the lo half of the activation split
  int stages;
  int mode;
  int* err;
};

constexpr int GEMM_THREADS = 256;
constexpr int GEMM_BK = 64;                       // K elements per stage (128 bytes: one swizzle row)
constexpr int GEMM_A_BYTES = 128 * GEMM_BK * 2;   // 16 KB weight tile

__host__ __device__ inline int gemm_stage_bytes(int tn, int use_lo) {
  return GEMM_A_BYTES + (use_lo ? 2 : 1) * tn * GEMM_BK * 2;
}

// grid: x = token block, y = weight tile (128 rows), z = K split.
// Output maps: STORE / ATOMIC: tm_o0 = fp32 Y [tokens][N] with a [128 x tn] box; SILU_MUL: tm_o0 / tm_o1 = bf16
// act_hi / act_lo [tokens][N/2] with [64 x tn] boxes. The maps' row extent is the number of valid tokens, so rows
// past it are never written.
__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_xhi,
               const __grid_constant__ CUtensorMap tm_xlo, const __grid_constant__ CUtensorMap tm_o0,
               const __grid_constant__ CUtensorMap tm_o1, const GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t gemm_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = args.stages;
  const int stage_bytes = gemm_stage_bytes(args.tn, args.use_lo);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * stage_bytes);
  uint64_t* empty = full + S;
  uint64_t* done = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  int* progress = reinterpret_cast<int*>(tmem_slot + 1);   // [0] loads issued, [1] stages consumed by the MMA

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tn = args.tn;
  const int tok0 = blockIdx.x * tn;
  const int wrow0 = blockIdx.y * 128;
  const int kb0 = blockIdx.z * args.k_blocks_per_split;
  const int kb1 = min(kb0 + args.k_blocks_per_split, args.k_blocks_total);
  const int nk = kb1 - kb0;
  uint32_t ncols = 32;
  while (ncols < (uint32_t)tn) ncols <<= 1;

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
    prefetch_tmap(&tm_o0);
    if (args.mode == GEMM_SILU_MUL) prefetch_tmap(&tm_o1);
  }
  if (warp == 0) tmem_alloc(tmem_slot, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (threadIdx.x == 0) {
    // ---- TMA producer ----
    // Weights do not depend on the previous kernel: the first stages' weight tiles are requested and the rest of the
    // slab is prefetched into L2 before the dependency wait, overlapping the previous kernel's tail.
    const uint32_t bytes = stage_bytes;
    const int pre = nk < S ? nk : S;
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], bytes);
      tma_load_2d(smem + i * stage_bytes, &tm_w, (kb0 + i) * GEMM_BK, wrow0, &full[i]);
    }
    for (int i = pre; i < nk; ++i) tma_prefetch_l2_2d(&tm_w, (kb0 + i) * GEMM_BK, wrow0);
    pdl_wait();
    for (int i = 0; i < nk && ok; ++i) {
      const int s = i % S, r = i / S;
      if (r > 0) ok = mbar_wait(&empty[s], (r - 1) & 1, args.err, ERR_TIMEOUT_MMA);
      if (!ok) break;
      uint8_t* a = smem + s * stage_bytes;
      uint8_t* bh = a + GEMM_A_BYTES;
      uint8_t* bl = bh + tn * GEMM_BK * 2;
      const int kx = (kb0 + i) * GEMM_BK;
      if (i >= pre) {
        mbar_arrive_expect_tx(&full[s], bytes);
        tma_load_2d(a, &tm_w, kx, wrow0, &full[s]);
      }
      tma_load_2d(bh, &tm_xhi, kx, tok0, &full[s]);
      if (args.use_lo) tma_load_2d(bl, &tm_xlo, kx, tok0, &full[s]);
      progress[0] = i + 1;
    }
  } else if (threadIdx.x == 32) {
    // ---- MMA issuer ----
    const uint32_t idesc = idesc_bf16(128, tn);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S, r = i / S;
      if (!mbar_wait(&full[s], r & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
      tc_fence_after();
      const uint32_t a = smem_u32(smem + s * stage_bytes);
      const uint32_t bh = a + GEMM_A_BYTES;
      const uint32_t bl = bh + tn * GEMM_BK * 2;
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
  pdl_wait();     // the epilogue writes memory the previous kernel may still read
  pdl_trigger();  // the next kernel may start its own set-up now
  // ---- epilogue: TMEM -> shared-memory tile (the drained stage buffers) -> one TMA bulk store ----
  const bool have = __syncthreads_and(mbar_wait(done, 0, args.err, ERR_TIMEOUT_MMA));
  tc_fence_after();
  if (have && nk > 0) {
    const int quad = warp & 3;          // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane;   // accumulator lane == weight row within the tile
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const int nch = (tn + 31) / 32, half_ch = (nch + 1) / 2;  // 32-column chunks: warps 0-3 the first half
    const int c_begin = (warp >> 2) ? half_ch * 32 : 0, c_end = (warp >> 2) ? nch * 32 : half_ch * 32;
    if (args.mode == GEMM_SILU_MUL) {
      // rows (2f, 2f+1) hold (gate, up) of feature f: the pair sits in adjacent lanes
      __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(smem);  // [tn][64]
      __nv_bfloat16* sl = sh + tn * 64;                              // [tn][64]
      // after the exchange the even lane holds (gate, up) of even tokens, the odd lane of odd tokens
      const int f = row >> 1, odd = lane & 1;
      for (int c = c_begin; c < c_end; c += 32) {
        float v[32];
        tmem_ld32(lane_base + c, v);
#pragma unroll
        for (int j0 = 0; j0 < 32; j0 += 4) {  // two tokens of this lane per paired hi/lo conversion
          float y[2];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int j = j0 + 2 * q;
            // even lane sends v[j+1] (gate of token j+1), odd lane sends v[j] (up of token j)
            const float other = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
            const float gate = odd ? other : v[j];
            const float up = odd ? v[j + 1] : other;
            y[q] = silu_fast(gate) * up;
          }
          __nv_bfloat162 h2, l2;
          split_bf16x2(y[0], y[1], h2, l2);
          const int tok = c + j0 + odd;  // tn is a multiple of 16, so tok < tn implies tok + 2 < tn
          if (tok < tn) {
            sh[tok * 64 + f] = h2.x;
            sl[tok * 64 + f] = l2.x;
            sh[(tok + 2) * 64 + f] = h2.y;
            sl[(tok + 2) * 64 + f] = l2.y;
          }
        }
      }
    } else {
      float* tile = reinterpret_cast<float*>(smem);  // [tn][128]
      for (int c = c_begin; c < c_end; c += 32) {
        float v[32];
        tmem_ld32(lane_base + c, v);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c + j < tn) tile[(c + j) * 128 + row] = v[j];
      }
    }
    fence_proxy_async();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
  if (threadIdx.x == 0) {
    if (have && nk > 0) {
      if (args.mode == GEMM_SILU_MUL) {
        const __nv_bfloat16* sh = reinterpret_cast<const __nv_bfloat16*>(smem);
        tma_store_2d(&tm_o0, sh, blockIdx.y * 64, tok0);
        tma_store_2d(&tm_o1, sh + tn * 64, blockIdx.y * 64, tok0);
      } else if (args.mode == GEMM_STORE) {
        tma_store_2d(&tm_o0, smem, wrow0, tok0);
      } else {
        tma_reduce_add_2d(&tm_o0, smem, wrow0, tok0);
      }
      bulk_commit();
      // only the shared-memory source must outlive the CTA; the writes complete with the grid, which is what the
      // next kernel's dependency wait observes
      bulk_wait_read_all();
    }
    // Error path only: loads the MMA never consumed may still be in flight; wait for them (bounded) before exit.
    for (int i = progress[1]; i < progress[0]; ++i) mbar_wait(&full[i % S], (i / S) & 1, args.err, ERR_TIMEOUT_TMA);
  }
}

}  // namespace hsg
