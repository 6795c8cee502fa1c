// Persistent weight-streaming GEMM for long-running grids (many 128 x tn tiles, e.g. 64-token ticks of 352 rows):
// the contract, operand layout and epilogue modes of gemm_tc_kernel, but one CTA per SM loops over tiles with the
// accumulator double-buffered in TMEM, so that draining tile i (TMEM -> registers -> shared -> TMA store, in
// 32-token chunks) overlaps the loads and MMAs of tile i + 1, and the load ring runs on across tiles.
//
// A tile is `halves` x 128 weight rows by tn tokens. With two halves (256 weight rows x 128 tokens, two N = 128
// accumulators side by side in TMEM) one 64-wide K block moves 64 KB for the same MMA work that 80 KB feeds in a
// 128 x 256 tile (the activation operand is a hi/lo pair, so it dominates the stage), in three stages instead of two.
// Measured at 22,528 tokens: ~10 % faster for the split-K reduce-add shapes (out_proj, down: N = 1024), 6-11 %
// slower for the store and SiLU-mul shapes (in_proj, gate/up), so the planner takes it for the former only. A weight
// tile whose upper half lies beyond the matrix skips that half.
//
// Roles in a 192-thread CTA: warp 0 lane 0 issues the TMA loads (a STAGES-deep ring of [A | B_hi | B_lo] stages
// shared by all of the CTA's tiles); warp 1 owns TMEM and its lane 0 issues tcgen05.mma, committing each stage back to
// the producer and each finished accumulator to the epilogue; warps 2-5 are the epilogue, warp w reading accumulator
// lanes 32 (w % 4) .. + 31 (= weight rows), and hand each accumulator back once drained. Tiles are numbered weight
// tile fastest, then token block, then K split, so the CTAs that run at the same time share activation blocks in L2.
// Every wait is bounded and reports through `err`.
#pragma once
#include "gemm.cuh"

namespace hsg {

constexpr int GPC_THREADS = 192;
constexpr int GPC_CHUNK = 32;  // tokens per epilogue chunk (one TMA store)

struct GemmPcArgs {
  int tiles_w, tb, splits, kps, k_blocks_total;
  int tn;       // tokens per tile: 128 or 256
  int halves;   // 128-row weight halves per tile: 1 or 2 (halves * tn <= 256: two accumulators fit TMEM)
  int n_w;      // weight rows
  int m;        // valid tokens (chunks wholly beyond are not stored)
  int use_lo, stages, mode;
  int* err;
  GemmConv conv;  // GEMM_CONV only
};

__host__ __device__ inline int gpc_chunk_bytes(int mode) {
  return mode == GEMM_SILU_MUL ? 2 * GPC_CHUNK * 64 * 2 : GPC_CHUNK * 128 * 4;
}
__host__ __device__ inline int gpc_stage_bytes(int tn, int use_lo, int halves) {
  return gemm_stage_bytes(tn, use_lo) + (halves - 1) * GEMM_A_BYTES;
}
__host__ __device__ inline int gpc_smem(int tn, int use_lo, int stages, int mode, int halves) {
  return stages * gpc_stage_bytes(tn, use_lo, halves) + 2 * gpc_chunk_bytes(mode) + (2 * stages + 5) * 8 + 16 + 1024;
}

__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

// tm_w: a [64 x 128 * halves] box. Output maps: STORE / ATOMIC: tm_o0 = fp32 Y [tokens][N] with a [128 x 32] box;
// SILU_MUL: tm_o0 / tm_o1 = bf16 act_hi / act_lo [tokens][N/2] with [64 x 32] boxes.
__global__ void __launch_bounds__(GPC_THREADS, 1)
gemm_pc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_xhi,
               const __grid_constant__ CUtensorMap tm_xlo, const __grid_constant__ CUtensorMap tm_o0,
               const __grid_constant__ CUtensorMap tm_o1, const GemmPcArgs args) {
  extern __shared__ __align__(1024) uint8_t gpc_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gpc_smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = args.stages, tn = args.tn, halves = args.halves;
  const int a_bytes = halves * GEMM_A_BYTES;
  const int stage_bytes = gpc_stage_bytes(tn, args.use_lo, halves);
  const int chunk_bytes = gpc_chunk_bytes(args.mode);
  uint8_t* outbuf = smem + S * stage_bytes;                                   // [2] epilogue chunks
  uint64_t* full = reinterpret_cast<uint64_t*>(outbuf + 2 * chunk_bytes);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;   // [2] MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;  // [2] epilogue -> MMA
  uint64_t* mma_done = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  int* progress = reinterpret_cast<int*>(tmem_slot + 1);  // [0] loads issued, [1] stages consumed by the MMA

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = args.tiles_w * args.tb * args.splits;
  const int acc_cols = halves * tn;  // one accumulator buffer: the halves side by side
  uint32_t ncols = 32;
  while (ncols < (uint32_t)(2 * acc_cols)) ncols <<= 1;
  auto decode = [&](int j, int& wrow0, int& tok0, int& kb0, int& nk) {
    const int wt = j % args.tiles_w, r = j / args.tiles_w;
    wrow0 = wt * 128 * halves;
    tok0 = (r % args.tb) * tn;
    kb0 = (r / args.tb) * args.kps;
    nk = min(args.kps, args.k_blocks_total - kb0);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(mma_done, 1);
    progress[0] = progress[1] = 0;
    fence_barrier_init();
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_xhi);
    if (args.use_lo) prefetch_tmap(&tm_xlo);
    prefetch_tmap(&tm_o0);
    if (args.mode == GEMM_SILU_MUL) prefetch_tmap(&tm_o1);
  }
  if (warp == 1) tmem_alloc(tmem_slot, ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // activations come from the previous kernel; the outputs may still be read by it
  if (threadIdx.x == 0) pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer: one ring of stages across all of this CTA's tiles ----
      int cnt = 0;
      bool ok = true;
      for (int j = blockIdx.x; j < total && ok; j += gridDim.x) {
        int wrow0, tok0, kb0, nk;
        decode(j, wrow0, tok0, kb0, nk);
        for (int i = 0; i < nk; ++i, ++cnt) {
          const int s = cnt % S, r = cnt / S;
          if (r > 0 && !mbar_wait(&empty[s], (r - 1) & 1, args.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
          uint8_t* a = smem + s * stage_bytes;
          uint8_t* bh = a + a_bytes;
          uint8_t* bl = bh + tn * GEMM_BK * 2;
          const int kx = (kb0 + i) * GEMM_BK;
          mbar_arrive_expect_tx(&full[s], stage_bytes);
          tma_load_2d(a, &tm_w, kx, wrow0, &full[s]);
          tma_load_2d(bh, &tm_xhi, kx, tok0, &full[s]);
          if (args.use_lo) tma_load_2d(bl, &tm_xlo, kx, tok0, &full[s]);
          progress[0] = cnt + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      const uint32_t idesc = idesc_bf16(128, tn);
      int cnt = 0, lt = 0;
      bool ok = true;
      for (int j = blockIdx.x; j < total && ok; j += gridDim.x, ++lt) {
        int wrow0, tok0, kb0, nk;
        decode(j, wrow0, tok0, kb0, nk);
        const int buf = lt & 1;
        const int nh = (halves > 1 && wrow0 + 128 < args.n_w) ? 2 : 1;  // weight halves inside the matrix
        if (lt >= 2 && !mbar_wait(&acc_empty[buf], ((lt >> 1) - 1) & 1, args.err, ERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        for (int i = 0; i < nk; ++i, ++cnt) {
          const int s = cnt % S, r = cnt / S;
          if (!mbar_wait(&full[s], r & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * stage_bytes);
          const uint32_t bh = a0 + a_bytes;
          const uint32_t bl = bh + tn * GEMM_BK * 2;
          for (int hf = 0; hf < nh; ++hf) {
            const uint32_t d = tmem + (uint32_t)(buf * acc_cols + hf * tn);
            const uint32_t a = a0 + hf * GEMM_A_BYTES;  // weight rows 128 hf .. of the box
#pragma unroll
            for (int kk = 0; kk < GEMM_BK / 16; ++kk) {
              const uint64_t da = sw128_desc(a + kk * 32);
              mma_bf16(d, da, sw128_desc(bh + kk * 32), idesc, (i > 0 || kk > 0) ? 1u : 0u);
              if (args.use_lo) mma_bf16(d, da, sw128_desc(bl + kk * 32), idesc, 1u);
            }
          }
          mma_commit(&empty[s]);
          progress[1] = cnt + 1;
        }
        if (ok) mma_commit(&acc_full[buf]);
      }
      mma_commit(mma_done);  // arrives once every MMA issued above has completed
    }
  } else {
    // ---- epilogue: per tile, 32-token chunks TMEM -> shared -> one TMA store each, two chunk buffers ----
    const int quad = warp & 3;
    const int row = quad * 32 + lane;  // accumulator lane == weight row within the tile
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const bool issuer = warp == 2 && lane == 0;
    int lt = 0, seq = 0;
    for (int j = blockIdx.x; j < total; j += gridDim.x, ++lt) {
      int wrow0, tok0, kb0, nk;
      decode(j, wrow0, tok0, kb0, nk);
      const int buf = lt & 1;
      const int nh = (halves > 1 && wrow0 + 128 < args.n_w) ? 2 : 1;
      if (!named_sync_and_id<3, 128>(mbar_wait(&acc_full[buf], (lt >> 1) & 1, args.err, ERR_TIMEOUT_MMA))) break;
      tc_fence_after();
      // GEMM_CONV: this row's conv taps (q | k | v rows only) and the raw inputs carried from chunk to chunk
      float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);
      float ch_h0 = 0.f, ch_h1 = 0.f, ch_h2 = 0.f;
      if (args.mode == GEMM_CONV && wrow0 < CONV_DIM) cw = reinterpret_cast<const float4*>(args.conv.w)[wrow0 + row];
      for (int q = 0; q < nh * tn; q += GPC_CHUNK, ++seq) {
        const int hf = q / tn, c = q % tn, wr = wrow0 + 128 * hf;  // weight half, token chunk, first weight row
        uint8_t* cb = outbuf + (seq & 1) * chunk_bytes;
        if (issuer) bulk_wait_read_1();  // the store issued from this buffer two chunks ago has read it
        named_sync_id<3, 128>();
        float v[32];
        tmem_ld32(lane_base + (uint32_t)(buf * acc_cols + q), v);
        if (args.mode == GEMM_CONV && wr < CONV_DIM) {
          // q | k | v channel ch = this thread's weight row: causal conv (4 taps) + SiLU along the chunk's 32 tokens,
          // which lie in one request (chunks and requests both start at multiples of 32). The raw inputs of the 3
          // tokens before the chunk come from the conv history at a request's first chunk, else from the previous
          // chunk (the same thread drains a tile's chunks in order). Padded tokens (position >= len) give 0; the
          // request's last three raw inputs go back to the history.
          const GemmConv& cv = args.conv;
          const int ch = wr + row, gt = tok0 + c, r = gt / cv.lb, p0 = gt % cv.lb;
          int len = 0;
          int64_t slot = 0;
          if (gt < args.m) {
            len = (int)cv.lens[r];
            slot = cv.slots[r];
            if (len < 0 || len > cv.lb || slot < 0 || slot > cv.max_slots) len = 0;  // reported by the GDN kernel
          }
          float* hp = cv.pool + (size_t)slot * CONV_KEEP * CONV_DIM + ch;
          if (p0 == 0) {
            ch_h0 = len > 0 ? hp[0] : 0.f;
            ch_h1 = len > 0 ? hp[CONV_DIM] : 0.f;
            ch_h2 = len > 0 ? hp[2 * CONV_DIM] : 0.f;
          }
          if (len >= p0 + 32) {
            // every token of the chunk is valid (the common case): no masks; the history is the chunk's last three
            // raw inputs if the request ends here
#pragma unroll
            for (int t = 0; t < 32; ++t) {
              const float x = v[t];
              v[t] = silu_fast(fmaf(cw.w, x, fmaf(cw.z, ch_h2, fmaf(cw.y, ch_h1, cw.x * ch_h0))));
              ch_h0 = ch_h1;
              ch_h1 = ch_h2;
              ch_h2 = x;
            }
            if (len == p0 + 32) {
              hp[0] = ch_h0;
              hp[CONV_DIM] = ch_h1;
              hp[2 * CONV_DIM] = ch_h2;
            }
          } else {
            float n0 = 0.f, n1 = 0.f, n2 = 0.f;
#pragma unroll
            for (int t = 0; t < 32; ++t) {
              const float x = v[t];
              const float y = silu_fast(fmaf(cw.w, x, fmaf(cw.z, ch_h2, fmaf(cw.y, ch_h1, cw.x * ch_h0))));
              if (p0 + t == len - 1) {
                n0 = ch_h1;
                n1 = ch_h2;
                n2 = x;
              }
              v[t] = p0 + t < len ? y : 0.f;
              ch_h0 = ch_h1;
              ch_h1 = ch_h2;
              ch_h2 = x;
            }
            if (len > 0 && p0 <= len - 1) {
              hp[0] = n0;
              hp[CONV_DIM] = n1;
              hp[2 * CONV_DIM] = n2;
            }
          }
        }
        if (args.mode == GEMM_SILU_MUL) {
          // rows (2f, 2f+1) hold (gate, up) of feature f: the even lane keeps even tokens, the odd lane odd ones
          __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(cb);  // [32][64]
          __nv_bfloat16* sl = sh + GPC_CHUNK * 64;
          const int f = row >> 1, odd = lane & 1;
#pragma unroll
          for (int t = 0; t < 32; t += 4) {  // two tokens of this lane per paired hi/lo conversion
            float y[2];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const int j = t + 2 * q;
              const float other = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
              const float gate = odd ? other : v[j];
              const float up = odd ? v[j + 1] : other;
              y[q] = silu_fast(gate) * up;
            }
            __nv_bfloat162 h2, l2;
            split_bf16x2(y[0], y[1], h2, l2);
            const int tok = t + odd;
            sh[tok * 64 + f] = h2.x;
            sl[tok * 64 + f] = l2.x;
            sh[(tok + 2) * 64 + f] = h2.y;
            sl[(tok + 2) * 64 + f] = l2.y;
          }
        } else {
          float* tile = reinterpret_cast<float*>(cb);  // [32][128]
#pragma unroll
          for (int t = 0; t < 32; ++t) tile[t * 128 + row] = v[t];
        }
        fence_proxy_async();
        named_sync_id<3, 128>();
        if (issuer) {
          if (tok0 + c < args.m) {
            if (args.mode == GEMM_SILU_MUL) {
              tma_store_2d(&tm_o0, cb, wr / 2, tok0 + c);
              tma_store_2d(&tm_o1, cb + GPC_CHUNK * 64 * 2, wr / 2, tok0 + c);
            } else if (args.mode == GEMM_STORE || args.mode == GEMM_CONV) {
              tma_store_2d(&tm_o0, cb, wr, tok0 + c);
            } else {
              tma_reduce_add_2d(&tm_o0, cb, wr, tok0 + c);
            }
          }
          bulk_commit();
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);  // this accumulator may be overwritten by the tile after next
    }
    if (issuer) bulk_wait_read_all();  // the shared-memory sources of the last stores have been read
  }

  // ---- teardown: every MMA done, every issued load landed (error paths), then release TMEM ----
  if (threadIdx.x == 32) mbar_wait(mma_done, 0, args.err, ERR_TIMEOUT_MMA);
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0)
    for (int i = progress[1]; i < progress[0]; ++i) mbar_wait(&full[i % S], (i / S) & 1, args.err, ERR_TIMEOUT_TMA);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

}  // namespace hsg
