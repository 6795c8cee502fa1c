// Chunked gated delta rule for multi-token ticks (32 or 64 tokens; prefill and 64-token scheduling ticks), fp16
// recurrent state, every product on the tensor cores (warp-level mma.sync, fp16 operands split into hi/lo pairs
// where exactness matters, fp32 accumulation).
//
// The tick's tokens are processed as 16-token sub-chunks. For a sub-chunk with state S (dk x dv) at its start,
// normalised keys/queries k^_t = rk_t k_t, q^_t = rq_t q_t, gates beta_t, log decays g_t, cumulative decay
// gam_t = sum_{s<=t} g_s, Gam_t = e^gam_t, Gam_C = Gam_15 (the WY form of the delta rule, as in the published chunked
// algorithm the reference's complete-message path uses through FLA, fla/ops/gated_delta_rule/chunk.py):
//   A[t][s]   = beta_t (Gam_t / Gam_s) k^_t . k^_s   (s < t),   T = (I + A)^-1
//   X[v][t]   = beta_t (v_t[v] - Gam_t (S^T k^_t)[v])
//   U^T       = X T^T                                          (delta-corrected values)
//   o_t       = Gam_t S^T q^_t + sum_{s<=t} (Gam_t / Gam_s)(q^_t . k^_s) u_s
//   S        <- Gam_C S + sum_s (Gam_C / Gam_s) k^_s u_s^T
// which equals the token-by-token recurrence of gdn.cuh / gdn_tc.cuh exactly in exact arithmetic.
//
// Warp roles (same grid and pipeline skeleton as gdn_tc.cuh):
//  * producer (warp 9): per (row, head) item, TMA loads of the fp16 state tile (two swizzled halves), the row's
//    q|k|v projection slices for all lb tokens (FUSED) or bf16 q|k|v (RAW), the conv history. The inputs and the
//    state have their own barriers: the next item's inputs are requested as soon as the consumers and the prologue
//    have read this item's for the last time (during the last sub-chunk), its state once this item's state has been
//    stored; the item metadata (slot, length) is double-buffered;
//  * prologue (warps 10, 11), per sub-chunk, into a double-buffered scratch area: conv + SiLU (or widening) of q, k
//    (warp 10: channels 0-95, warp 11: 96-127), v (warp 11) and the gates; the k/q MMA operand columns (fp16 hi/lo),
//    per-token norm factors and cumulative decays; then warp 10 the decay-masked q.k table and K~ = (Gam_C/Gam_s) k^_s
//    (hi/lo), warp 11 the k.k table, A and T = (I + A)^-1 by forward substitution (fp32), T as hi/lo;
//  * consumers (warps 0-7): warp w owns state columns v in [16 w, 16 w + 16) for all 128 k as fp32 registers in
//    m16n8k16 fragment layout. Per sub-chunk: S^T K^T and S^T Q^T (fp16 state x hi/lo k, q), X, U^T = X T^T,
//    O^T = Gam R + U^T Mqk^T, the gated RMSNorm of o (partial sums of squares across the 8 warps through shared
//    memory) written as the out_proj operand, and S^T <- Gam_C S^T + U^T K~ with the state registers as the
//    accumulator (the m16n8k16 D layout of two 8-column tiles is the A layout of one 16 x 16 fragment);
//  * epilogue (warp 8): zero rows for padding, the new state back to the pool with two TMA stores.
// Padded tokens (t >= len) carry k = q = v = 0, beta = 0, g = 0: they change nothing and their outputs are zero.
#pragma once
#include "gdn_tc.cuh"

namespace hsg {

constexpr int GDNC_SUB = 16;      // tokens per sub-chunk
constexpr int GDNC_MAX_LB = 64;
// sub-chunk scratch (two buffers, by global sub-chunk parity); byte offsets. Padded rows keep fragment loads free of
// bank conflicts: a token's operand row is 1040 bytes, K~ / T / Mqk rows 48 bytes.
constexpr int GDNC_BOP_ROW = 4 * GDN_D * 2 + 16;               // k_hi | k_lo | q_hi | q_lo, fp16, + pad
constexpr int GDNC_KT_ROW = 48;                                // K~^T[k][s] 16 fp16 + pad
constexpr int GDNC_T_ROW = 48;                                 // T[t][s], Mqk[t][s] 16 fp16 + pad
constexpr int GDNC_OFF_BOP = 0;
constexpr int GDNC_OFF_KT = GDNC_OFF_BOP + GDNC_SUB * GDNC_BOP_ROW;       // [2][128] rows
constexpr int GDNC_OFF_TM = GDNC_OFF_KT + 2 * GDN_D * GDNC_KT_ROW;        // [2][16] rows (A fp32 [16][16] overlays)
constexpr int GDNC_OFF_MQ = GDNC_OFF_TM + 2 * GDNC_SUB * GDNC_T_ROW;      // [2][16] rows
constexpr int GDNC_OFF_PART = GDNC_OFF_MQ + 2 * GDNC_SUB * GDNC_T_ROW;    // [16][2 warps][4] f32
constexpr int GDNC_OFF_VEC = GDNC_OFF_PART + GDNC_SUB * 2 * 4 * 4;        // [6][16] f32: gam, beta, Gam, rk, rq, GC
constexpr int GDNC_OFF_SQ = GDNC_OFF_VEC + 6 * GDNC_SUB * 4;              // [8 warps][16] f32 output sums of squares
constexpr int GDNC_SCRATCH = (GDNC_OFF_SQ + 8 * GDNC_SUB * 4 + 127) & ~127;
// per-item area (one buffer): per-token partial sums of q.q, k.k from the four q/k consumer warps [64][4][2] f32,
// log decays [64], betas [64]
constexpr int GDNC_ITEM = GDNC_MAX_LB * 4 * 2 * 4 + 2 * GDNC_MAX_LB * 4;

// Stage: state halves | x [lb][XS][128] fp32 (FUSED: q, k, v; RAW: v) | FUSED: conv history [3][3][128] fp32,
// RAW: bf16 q|k|v [lb][3][128]; rounded up to 1 KB.
__host__ __device__ inline int gdnc_stage_bytes(int lb, bool fused) {
  return (GDNT_TILE + lb * (fused ? 3 : 1) * GDN_D * 4 + (fused ? 9 * GDN_D * 4 : lb * 3 * GDN_D * 2) + 1023) & ~1023;
}
__host__ __device__ inline int gdnc_fixed_bytes() {
  return 2 * GDNC_SCRATCH + GDNC_ITEM + GDN_MAX_STAGES * (16 + 3 * 8) + 2 * 2 * 8 + 8 + 1024;
}
// One stage: the per-item arrays (partial sums, gates) and the team conv keep exactly one item in flight (a 64-token
// item's stage is 133 KB, so a second would not fit beside the scratch anyway).
__host__ __device__ inline int gdnc_stages(int, bool) { return 1; }
__host__ __device__ inline int gdnc_smem_bytes(int lb, bool fused) {
  return gdnc_stages(lb, fused) * gdnc_stage_bytes(lb, fused) + gdnc_fixed_bytes();
}

__device__ __forceinline__ uint32_t ld_u32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Causal depthwise conv (kernel 4: c.x oldest .. c.w current) + SiLU of one channel over tokens tb..tb+15, in place
// (xc[t * stride]). w holds the three inputs before the block and afterwards the block's last three; outputs of
// tokens >= len are 0 and hist receives the three inputs ending at token len - 1 when that token is in the block;
// sq gets the squared outputs. All loads are issued before the arithmetic so the 16 tokens overlap.
__device__ __forceinline__ void conv_block16(float* xc, int stride, float4 c, float (&w)[3], int tb, int len,
                                             float (&hist)[3], float (&sq)[16]) {
  float in[19];
  in[0] = w[0];
  in[1] = w[1];
  in[2] = w[2];
#pragma unroll
  for (int u = 0; u < 16; ++u) in[3 + u] = xc[(tb + u) * stride];
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const float y = silu_fast(fmaf(c.w, in[u + 3], fmaf(c.z, in[u + 2], fmaf(c.y, in[u + 1], c.x * in[u]))));
    const float o = tb + u < len ? y : 0.f;
    xc[(tb + u) * stride] = o;
    sq[u] = o * o;
    if (tb + u == len - 1) {
      hist[0] = in[u + 1];
      hist[1] = in[u + 2];
      hist[2] = in[u + 3];
    }
  }
  w[0] = in[16];
  w[1] = in[17];
  w[2] = in[18];
}

// Sum of v[i] over the 32 lanes for 16 values at once (a transposing butterfly: 8 + 4 + 2 + 1 + 1 shuffles instead
// of 16 x 5). Lane l ends with the total of value ((l >> 4) & 1) * 8 + ((l >> 3) & 1) * 4 + ((l >> 2) & 1) * 2
// + ((l >> 1) & 1); lanes l and l ^ 1 hold the same total.
__device__ __forceinline__ int reduce16_index(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}
__device__ __forceinline__ float reduce16(float (&v)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool up = lane & 16;
    const float send = up ? v[i] : v[i + 8];
    const float keep = up ? v[i + 8] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 8;
    const float send = up ? v[i] : v[i + 4];
    const float keep = up ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 4;
    const float send = up ? v[i] : v[i + 2];
    const float keep = up ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const bool up = lane & 2;
    const float send = up ? v[0] : v[1];
    const float keep = up ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// maps: state = the fp16 pool; in0 = conv history (FUSED) or bf16 q|k|v [rows][3][2048] box [lb][3][128] (RAW);
// in1 = the projection's q|k|v columns [rows][3][2048] box [lb][3][128] (FUSED).
template <bool FUSED>
__global__ void __launch_bounds__(GDNT_THREADS, 1)
gdn_chunk_kernel(const __grid_constant__ GdntMaps maps, const GdnArgs args) {
  constexpr int XS = FUSED ? 3 : 1;        // fp32 slots per token in x
  constexpr int SV = FUSED ? 2 : 0;        // the v slot
  const CUtensorMap* tm_state = &maps.state;
  extern __shared__ __align__(1024) uint8_t gdnc_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gdnc_smem_raw) + 1023) & ~uintptr_t(1023));
  const int lb = args.lb, S = args.stages, nsub = lb / GDNC_SUB;
  const int sbytes = gdnc_stage_bytes(lb, FUSED);
  uint8_t* scr0 = smem + S * sbytes;
  float* ipart = reinterpret_cast<float*>(scr0 + 2 * GDNC_SCRATCH);  // [64][4][2]
  float* igl = ipart + GDNC_MAX_LB * 8;                               // [64] log decays
  float* ibe = igl + GDNC_MAX_LB;                                     // [64] betas
  GdnMeta* meta = reinterpret_cast<GdnMeta*>(ibe + GDNC_MAX_LB);
  // One stage (the host passes stages = 1): full[0] the item's inputs landed, full[1] its state tile landed;
  // empty[0] the state region is free (epilogue's store has read it), empty[1] the input region is free.
  uint64_t* full = reinterpret_cast<uint64_t*>(meta + GDN_MAX_STAGES);  // producer -> prologue, consumers
  uint64_t* done = full + GDN_MAX_STAGES;                               // consumers -> epilogue
  uint64_t* empty = done + GDN_MAX_STAGES;                              // epilogue, readers -> producer
  uint64_t* sfull = empty + GDN_MAX_STAGES;                             // [2] prologue -> consumers (sub-chunk)
  uint64_t* sdone = sfull + 2;                                          // [2] consumers -> prologue (buffer free)
  uint64_t* cdone = sdone + 2;                                          // consumers' conv -> prologue (per item)

  const int h = blockIdx.x, p = blockIdx.y, P = gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_items = args.nb > p ? (args.nb - p + P - 1) / P : 0;
  auto row_of = [&](int i) { return p + i * P; };
  auto stage_ptr = [&](int s) { return smem + s * sbytes; };
  auto x_of = [&](int s) { return reinterpret_cast<float*>(stage_ptr(s) + GDNT_TILE); };
  auto tail_of = [&](int s) { return x_of(s) + lb * XS * GDN_D; };  // FUSED conv history / RAW bf16 inputs
  auto tile_row = [&](int64_t slot) { return (int)((slot * GDN_H + h) * GDN_D); };
  auto scr = [&](int j) { return scr0 + (j & 1) * GDNC_SCRATCH; };

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(&done[0], GDNT_CONS);
    mbar_init(&empty[0], 1);
    // every consumer, prologue and epilogue thread, once per item: the epilogue warp counts too, so that the inputs
    // barrier cannot complete twice before it has waited for it (runs of padding items release their inputs at once)
    mbar_init(&empty[1], GDNT_CONS + 64 + 32);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sfull[b], 64);
      mbar_init(&sdone[b], GDNT_CONS);
    }
    mbar_init(cdone, FUSED ? GDNT_THREADS : GDNT_CONS);
    fence_barrier_init();
    prefetch_tmap(&maps.state);
    prefetch_tmap(&maps.in0);
    if (FUSED) prefetch_tmap(&maps.in1);
  }
  __syncthreads();

  // FUSED: the causal conv of an item is shared by all twelve warps, one channel a thread: thread t owns channel
  // t & 127 of part t >> 7 (q, k, v) and runs conv + SiLU over the item's tokens in place, writes the per-token
  // partial sums of the squared q / k outputs (one per warp) and the new conv history; v threads with channel c < lb
  // also compute token c's gates. Every thread then arrives on cdone. Callers have passed pdl_wait (gates read proj).
  const int cpart = tid >> 7, cch = tid & (GDN_D - 1);
  float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);
  if (FUSED) cw = (reinterpret_cast<const float4*>(args.conv_w) + h * GDN_D)[cpart * KEY_DIM + cch];
  const float negA = -expf(args.A_log[h]), dtb = args.dt_bias[h];
  auto team_conv = [&](int s, int n, int len, int64_t slot) {
    // the gate inputs first: issued after the conv-history stores below, these global loads could not be moved
    // above them (possible aliasing) and would add a full round trip to every item's conv
    const bool gate_thread = cpart == 2 && cch < lb;
    float xa = 0.f, xb = 0.f;
    if (gate_thread && cch < len) {
      const size_t rt = (size_t)n * lb + cch;
      xa = args.proj[rt * GDN_IN + GDN_A_OFF + h];
      xb = args.proj[rt * GDN_IN + GDN_B_OFF + h];
    }
    float* x = x_of(s);
    const float* hist = tail_of(s);
    float w[3] = {hist[(0 * 3 + cpart) * GDN_D + cch], hist[(1 * 3 + cpart) * GDN_D + cch],
                  hist[(2 * 3 + cpart) * GDN_D + cch]};
    float hh[3] = {0.f, 0.f, 0.f};
    for (int tb = 0; tb < lb; tb += GDNC_SUB) {
      float sq[GDNC_SUB];
      conv_block16(x + cpart * GDN_D + cch, XS * GDN_D, cw, w, tb, len, hh, sq);
      if (cpart < 2) {  // warp-uniform
        const float tot = reduce16(sq, lane);
        if (!(lane & 1)) ipart[((tb + reduce16_index(lane)) * 4 + (warp & 3)) * 2 + cpart] = tot;
      }
    }
    float* gp = args.conv_pool + (size_t)slot * CONV_KEEP * CONV_DIM + cpart * KEY_DIM + h * GDN_D + cch;
    gp[0] = hh[0];
    gp[CONV_DIM] = hh[1];
    gp[2 * CONV_DIM] = hh[2];
    if (gate_thread) {  // gates of token cch: log decay -exp(A_log) softplus(a + dt_bias), beta
      float gl = 0.f, be = 0.f;
      if (cch < len) {
        const float xg = xa + dtb;
        gl = negA * (xg > 20.f ? xg : log1pf(expf(xg)));
        be = sigmoidf_(xb);
      }
      igl[cch] = gl;
      ibe[cch] = be;
    }
  };
  // FUSED roles other than the consumers: wait for item i's stage, take part in its conv
  auto join_conv = [&](int i) {
    if (!mbar_wait(&full[0], i & 1, args.err, ERR_TIMEOUT_TMA)) return false;
    const int len = meta[i & 1].len;
    if (len > 0) {
      team_conv(0, row_of(i), len, meta[i & 1].slot);
      mbar_arrive(cdone);
    }
    return true;
  };

  if (warp == GDNT_PROD_WARP) {
    // ===================================== producer =====================================
    int held_len[2] = {};
    int64_t held_slot[2] = {};
    auto take = [&](int i, int64_t len64, int64_t slot) {  // item i's checked length and slot (metadata i & 1)
      int len = (int)len64;
      if (len64 < 0 || len64 > lb) {
        if (lane == 0) set_error(args.err, ERR_BAD_LEN);
        len = 0;
      }
      if (len > 0 && (slot < 0 || slot > args.max_slots)) {
        if (lane == 0) set_error(args.err, ERR_BAD_SLOT);
        len = 0;
      }
      held_len[i & 1] = len;
      held_slot[i & 1] = slot;
    };
    auto issue_state = [&](int i) {
      const int len = held_len[i & 1];
      if (lane == 0) {
        if (len > 0)
          mbar_arrive_expect_tx(&full[1], GDNT_TILE);
        else
          mbar_arrive(&full[1]);
      }
      __syncwarp();
      if (len == 0 || lane != 0) return;
      uint8_t* st = stage_ptr(0);
      tma_load_2d(st, tm_state, 0, tile_row(held_slot[i & 1]), &full[1]);
      tma_load_2d(st + GDNT_HALF, tm_state, 64, tile_row(held_slot[i & 1]), &full[1]);
    };
    auto issue_inputs = [&](int i) {  // metadata, then the inputs (whole boxes: padded tokens' rows too, in bounds)
      const int len = held_len[i & 1], n = row_of(i);
      if (lane == 0) {
        meta[i & 1].slot = held_slot[i & 1];
        meta[i & 1].len = len;
        if (len > 0)
          mbar_arrive_expect_tx(&full[0], FUSED ? lb * 3 * GDN_D * 4 + 9 * GDN_D * 4 : lb * 3 * GDN_D * 2);
        else
          mbar_arrive(&full[0]);
      }
      __syncwarp();
      if (len == 0 || lane != 0) return;
      if (FUSED) {
        tma_load_3d(tail_of(0), &maps.in0, h * GDN_D, 0, (int)held_slot[i & 1] * CONV_KEEP, &full[0]);
        tma_load_3d(x_of(0), &maps.in1, h * GDN_D, 0, n * lb, &full[0]);
      } else {
        tma_load_3d(tail_of(0), &maps.in0, h * GDN_D, 0, n * lb, &full[0]);
      }
    };
    if (n_items > 0) {
      take(0, args.lens[row_of(0)], args.slots[row_of(0)]);
      issue_state(0);  // the state pool is this kernel's own: requested before the dependency wait
    }
    pdl_wait();
    if (n_items > 0) issue_inputs(0);
    for (int i = 0; i < n_items; ++i) {
      if (i > 0) {
        if (!mbar_wait(&empty[0], (i - 1) & 1, args.err, ERR_TIMEOUT_TMA)) break;  // item i - 1 stored
        issue_state(i);
      }
      if (FUSED && !join_conv(i)) break;
      if (i + 1 < n_items) {
        take(i + 1, args.lens[row_of(i + 1)], args.slots[row_of(i + 1)]);
        if (!mbar_wait(&empty[1], i & 1, args.err, ERR_TIMEOUT_TMA)) break;  // item i's inputs read for the last time
        issue_inputs(i + 1);
      }
    }
    return;
  }

  if (warp == GDNT_EPI_WARP) {
    // ===================================== epilogue =====================================
    pdl_wait();  // the outputs may still be read by an earlier kernel
    for (int i = 0; i < n_items; ++i) {
      const int s = 0, n = row_of(i);
      if (FUSED ? !join_conv(i) : !mbar_wait(&full[0], i & 1, args.err, ERR_TIMEOUT_TMA)) break;
      mbar_arrive(&empty[1]);  // seen this item's inputs (it reads them only in the conv)
      if (!mbar_wait(&done[0], i & 1, args.err, ERR_TIMEOUT_TMA)) break;
      const int len = meta[i & 1].len;
      if (len == 0) {  // a padding row: zero outputs (the consumers write the outputs of real rows)
        for (int t = 0; t < lb; ++t) {
          const size_t row = (size_t)n * lb + t;
          if (FUSED) {
            *reinterpret_cast<uint2*>(args.out_hi + row * KEY_DIM + h * GDN_D + lane * 4) = make_uint2(0u, 0u);
            *reinterpret_cast<uint2*>(args.out_lo + row * KEY_DIM + h * GDN_D + lane * 4) = make_uint2(0u, 0u);
          } else {
            reinterpret_cast<float4*>(args.o_raw + (row * GDN_H + h) * GDN_D)[lane] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
      if (lane == 0) {
        if (len > 0) {  // the new state back to the pool
          const int row = tile_row(meta[i & 1].slot);
          tma_store_2d(tm_state, stage_ptr(s), 0, row);
          tma_store_2d(tm_state, stage_ptr(s) + GDNT_HALF, 64, row);
          bulk_commit();
          bulk_wait_read_all();  // the stores have read the stage
        }
        mbar_arrive(&empty[0]);
      }
      __syncwarp();
    }
    if (lane == 0) bulk_wait_all();
    return;
  }

  if (warp == GDNT_QK_WARP || warp == GDNT_V_WARP) {
    // ===================================== prologue =====================================
    // Per sub-chunk, from the consumers' conv outputs: norm factors and cumulative decay; the k/q operand columns
    // (hi/lo); warp 10: the q.k table Mqk and K~; warp 11: the k.k table, A and T. The two warps synchronise on
    // barrier 2.
    const bool w10 = warp == GDNT_QK_WARP;
    const float scale = 0.08838834764831845f;  // 128^-1/2, correctly rounded
    if (FUSED) pdl_wait();  // the conv history written below may still be read by an earlier kernel
    int jsub = 0, item_seq = 0;
    for (int i = 0; i < n_items; ++i) {
      const int s = 0;
      bool ok = FUSED ? join_conv(i) : mbar_wait(&full[0], i & 1, args.err, ERR_TIMEOUT_TMA);
      const int len = ok ? meta[i & 1].len : 1;
      if (ok && len > 0) ok = mbar_wait(cdone, item_seq & 1, args.err, ERR_TIMEOUT_TMA);
      if (!named_sync_and_id<2, 64>(ok)) return;
      if (len == 0) {
        mbar_arrive(&empty[1]);
        continue;
      }
      ++item_seq;
      const float* x = x_of(s);
      const __nv_bfloat16* raw = reinterpret_cast<const __nv_bfloat16*>(tail_of(s));
      for (int sc = 0; sc < nsub; ++sc, ++jsub) {
        // this scratch buffer was last used by sub-chunk jsub - 2
        const bool okb = jsub < 2 || mbar_wait(&sdone[jsub & 1], ((jsub >> 1) - 1) & 1, args.err, ERR_TIMEOUT_TMA);
        if (!named_sync_and_id<2, 64>(okb)) return;
        uint8_t* sb = scr(jsub);
        uint8_t* bb = sb + GDNC_OFF_BOP;
        float* vec = reinterpret_cast<float*>(sb + GDNC_OFF_VEC);
        const int t0 = sc * GDNC_SUB;
        // ---- (1) factors (warp 11, lanes 0-15) and operand columns (warp 10: tokens 0-7, warp 11: 8-15) ----
        if (!w10) {
          const int t = t0 + (lane & (GDNC_SUB - 1));
          float gam = lane < GDNC_SUB ? igl[t] : 0.f;
#pragma unroll
          for (int off = 1; off < GDNC_SUB; off <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, gam, off, GDNC_SUB);
            if ((lane & (GDNC_SUB - 1)) >= off) gam += y;
          }
          const float gC = __shfl_sync(0xffffffffu, gam, GDNC_SUB - 1);
          if (lane < GDNC_SUB) {
            float sq = 0.f, sk = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < 4; ++w2) {
              sq += ipart[(t * 4 + w2) * 2 + 0];
              sk += ipart[(t * 4 + w2) * 2 + 1];
            }
            vec[0 * GDNC_SUB + lane] = gam;
            vec[1 * GDNC_SUB + lane] = ibe[t];
            vec[2 * GDNC_SUB + lane] = expf(gam);
            vec[3 * GDNC_SUB + lane] = rsqrtf(sk + 1e-6f);
            vec[4 * GDNC_SUB + lane] = scale * rsqrtf(sq + 1e-6f);
            if (lane == 0) vec[5 * GDNC_SUB] = expf(gC);
          }
        }
        {
          // lane owns channels 4 lane .. 4 lane + 3 of 8 tokens: k_hi | k_lo | q_hi | q_lo as half2 pairs
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int tt = (w10 ? 0 : 8) + u, t = t0 + tt;
            float4 q4, k4;
            if (FUSED) {
              q4 = reinterpret_cast<const float4*>(x + (t * XS + 0) * GDN_D)[lane];
              k4 = reinterpret_cast<const float4*>(x + (t * XS + 1) * GDN_D)[lane];
            } else if (t < len) {
              const __nv_bfloat162* rq2 = reinterpret_cast<const __nv_bfloat162*>(raw + (t * 3 + 0) * GDN_D) + 2 * lane;
              const __nv_bfloat162* rk2 = reinterpret_cast<const __nv_bfloat162*>(raw + (t * 3 + 1) * GDN_D) + 2 * lane;
              const float2 qa = __bfloat1622float2(rq2[0]), qb = __bfloat1622float2(rq2[1]);
              const float2 ka = __bfloat1622float2(rk2[0]), kb = __bfloat1622float2(rk2[1]);
              q4 = make_float4(qa.x, qa.y, qb.x, qb.y);
              k4 = make_float4(ka.x, ka.y, kb.x, kb.y);
            } else {
              q4 = k4 = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            uint32_t kh0, kl0, kh1, kl1, qh0, ql0, qh1, ql1;
            split_half2x(k4.x, k4.y, kh0, kl0);
            split_half2x(k4.z, k4.w, kh1, kl1);
            split_half2x(q4.x, q4.y, qh0, ql0);
            split_half2x(q4.z, q4.w, qh1, ql1);
            uint8_t* row = bb + tt * GDNC_BOP_ROW + lane * 8;
            *reinterpret_cast<uint2*>(row + 0 * GDN_D * 2) = make_uint2(kh0, kh1);
            *reinterpret_cast<uint2*>(row + 1 * GDN_D * 2) = make_uint2(kl0, kl1);
            *reinterpret_cast<uint2*>(row + 2 * GDN_D * 2) = make_uint2(qh0, qh1);
            *reinterpret_cast<uint2*>(row + 3 * GDN_D * 2) = make_uint2(ql0, ql1);
          }
        }
        named_sync_id<2, 64>();  // operand columns and factors of the 16 tokens are in shared memory
        // ---- (2) 16 x 16 token tables with the tensor cores: warp 10 q.k, warp 11 k.k ----
        {
          const int g = lane >> 2, t4 = lane & 3;
          const int va = w10 ? 2 : 0;  // A operand rows: q (warp 10) or k (warp 11)
          // three independent accumulator chains per 8-token tile (hi.hi, hi.lo, lo.hi), summed at the end
          float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
          float dx[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
          float dy[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
          for (int kt = 0; kt < 8; ++kt) {
            const int ko = (16 * kt + 2 * t4) * 2;
            uint32_t a[2][4];
#pragma unroll
            for (int hl = 0; hl < 2; ++hl) {
              const int vo = (va + hl) * GDN_D * 2;
              a[hl][0] = ld_u32(bb + g * GDNC_BOP_ROW + vo + ko);
              a[hl][1] = ld_u32(bb + (g + 8) * GDNC_BOP_ROW + vo + ko);
              a[hl][2] = ld_u32(bb + g * GDNC_BOP_ROW + vo + ko + 16);
              a[hl][3] = ld_u32(bb + (g + 8) * GDNC_BOP_ROW + vo + ko + 16);
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              const uint8_t* br = bb + (8 * nt + g) * GDNC_BOP_ROW + ko;
              const uint32_t bh0 = ld_u32(br), bh1 = ld_u32(br + 16);
              const uint32_t bl0 = ld_u32(br + GDN_D * 2), bl1 = ld_u32(br + GDN_D * 2 + 16);
              mma_f16_16816(d[nt], a[0][0], a[0][1], a[0][2], a[0][3], bh0, bh1);
              mma_f16_16816(dx[nt], a[0][0], a[0][1], a[0][2], a[0][3], bl0, bl1);
              mma_f16_16816(dy[nt], a[1][0], a[1][1], a[1][2], a[1][3], bh0, bh1);
            }
          }
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) d[nt][e] += dx[nt][e] + dy[nt][e];
          // D: rows t = g, g + 8; cols s = 8 nt + 2 t4 + e
          const float* gamv = vec;
          const float* bev = vec + 1 * GDNC_SUB;
          const float* rkv = vec + 3 * GDNC_SUB;
          const float* rqv = vec + 4 * GDNC_SUB;
          // K~^T[k][s] = e^(gam_C - gam_s) rk_s k_s[k] as hi/lo for the tokens s of one half (warp 10: 0-7, warp 11:
          // 8-15); the exponent is <= 0, so strong decay underflows to 0, never 0/0. Lane owns k = 4 lane .. 4 lane + 3.
          // The 4-byte column (s pair) of row k is stored XOR-ed with (k >> 3) & 7, which spreads a warp's stores over
          // 16 banks (rows are 48 bytes apart) and keeps the consumers' fragment loads conflict-free.
          auto kt_half = [&](int half) {
            const float gC = gamv[GDNC_SUB - 1];
            uint8_t* ktb = sb + GDNC_OFF_KT;
            const int f = (lane >> 1) & 7;
#pragma unroll
            for (int s2 = 0; s2 < GDNC_SUB / 2; s2 += 2) {
              const int s = 8 * half + s2;
              const float f0 = expf(gC - gamv[s]) * rkv[s], f1 = expf(gC - gamv[s + 1]) * rkv[s + 1];
              float4 ka, kb;
              if (FUSED) {
                ka = reinterpret_cast<const float4*>(x + ((t0 + s) * XS + 1) * GDN_D)[lane];
                kb = reinterpret_cast<const float4*>(x + ((t0 + s + 1) * XS + 1) * GDN_D)[lane];
              } else {
                auto rawk = [&](int t) {
                  if (t >= len) return make_float4(0.f, 0.f, 0.f, 0.f);
                  const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(raw + (t * 3 + 1) * GDN_D) + 2 * lane;
                  const float2 u0 = __bfloat1622float2(r2[0]), u1 = __bfloat1622float2(r2[1]);
                  return make_float4(u0.x, u0.y, u1.x, u1.y);
                };
                ka = rawk(t0 + s);
                kb = rawk(t0 + s + 1);
              }
              const float kav[4] = {ka.x, ka.y, ka.z, ka.w}, kbv[4] = {kb.x, kb.y, kb.z, kb.w};
              const int col = ((s >> 1) ^ f) * 4;
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                uint32_t hi, lo;
                split_half2x(kav[c] * f0, kbv[c] * f1, hi, lo);
                const int k = 4 * lane + c;
                *reinterpret_cast<uint32_t*>(ktb + k * GDNC_KT_ROW + col) = hi;
                *reinterpret_cast<uint32_t*>(ktb + (GDN_D + k) * GDNC_KT_ROW + col) = lo;
              }
            }
          };
          if (w10) {  // Mqk[t][s] = rq_t rk_s e^(gam_t - gam_s) q.k for s <= t, as hi/lo
            uint8_t* mq = sb + GDNC_OFF_MQ;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int hr = 0; hr < 2; ++hr) {
                const int t = g + 8 * hr;
                float val[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const int sidx = 8 * nt + 2 * t4 + e;
                  val[e] = sidx <= t ? d[nt][2 * hr + e] * rqv[t] * rkv[sidx] * expf(gamv[t] - gamv[sidx]) : 0.f;
                }
                uint32_t hi, lo;
                split_half2x(val[0], val[1], hi, lo);
                const int off = t * GDNC_T_ROW + (8 * nt + 2 * t4) * 2;
                *reinterpret_cast<uint32_t*>(mq + off) = hi;
                *reinterpret_cast<uint32_t*>(mq + GDNC_SUB * GDNC_T_ROW + off) = lo;
              }
            kt_half(0);
          } else {  // A[t][s] = beta_t rk_t rk_s e^(gam_t - gam_s) k.k for s < t; T = (I + A)^-1
            float* am = reinterpret_cast<float*>(sb + GDNC_OFF_TM);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int hr = 0; hr < 2; ++hr) {
                const int t = g + 8 * hr;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const int sidx = 8 * nt + 2 * t4 + e;
                  am[t * GDNC_SUB + sidx] = sidx < t ? d[nt][2 * hr + e] * bev[t] * rkv[t] * rkv[sidx] *
                                                           expf(gamv[t] - gamv[sidx])
                                                     : 0.f;
                }
              }
            __syncwarp();
            // forward substitution: lane j (< 16) builds column j of T; T[t][j] = [t == j] - sum_{s<t} A[t][s] T[s][j]
            float tc[GDNC_SUB];
#pragma unroll
            for (int t = 0; t < GDNC_SUB; ++t) {
              float v = (t == lane) ? 1.f : 0.f;
#pragma unroll
              for (int s2 = 0; s2 < t; ++s2) v = fmaf(-am[t * GDNC_SUB + s2], tc[s2], v);
              tc[t] = v;
            }
            __syncwarp();  // every lane has read A; T overwrites it
            if (lane < GDNC_SUB) {
              __half* tm = reinterpret_cast<__half*>(sb + GDNC_OFF_TM);
#pragma unroll
              for (int t = 0; t < GDNC_SUB; ++t) {
                const __half hi = __float2half_rn(tc[t]);
                tm[(t * GDNC_T_ROW) / 2 + lane] = hi;
                tm[(GDNC_SUB * GDNC_T_ROW + t * GDNC_T_ROW) / 2 + lane] = __float2half_rn(tc[t] - __half2float(hi));
              }
            }
            kt_half(1);
          }
        }
        mbar_arrive(&sfull[jsub & 1]);
      }
      mbar_arrive(&empty[1]);  // this item's inputs are not read by the prologue again
    }
    return;
  }

  // ===================================== consumers =====================================
  const int g = lane >> 2, t4 = lane & 3;
  const int frag_k = (lane & 7) + ((lane >> 4) & 1) * 8;
  const int frag_c = 2 * (warp & 3) + ((lane >> 3) & 1);
  const int v0 = 16 * warp + g;  // this lane's state columns: v0 (fragment rows g) and v0 + 8
  const float gw0 = FUSED ? args.gnorm_w[v0] : 0.f, gw1 = FUSED ? args.gnorm_w[v0 + 8] : 0.f;
  // the isolated kernel's widening: thread c < 128 owns q and k channel c, thread 128 + c owns v channel c and
  // (c < lb) token c's gates
  const bool qk_thread = tid < GDN_D;
  const int cc = tid & (GDN_D - 1);
  pdl_wait();  // z comes from the preceding GEMM's output; the outputs may still be read by an earlier kernel
  if (tid == 0) pdl_trigger();
  int jsub = 0;
  bool alive = true;
  for (int i = 0; i < n_items && alive; ++i) {
    const int s = 0, n = row_of(i);
    if (!mbar_wait(&full[0], i & 1, args.err, ERR_TIMEOUT_TMA)) break;
    const int len = meta[i & 1].len;
    if (len == 0) {
      mbar_arrive(&empty[1]);
      // a padding item's state barrier completes with a plain arrive, issued after the producer has seen the
      // previous item stored; waiting for it keeps this item's done (and so its stored signal) behind that
      if (!mbar_wait(&full[1], i & 1, args.err, ERR_TIMEOUT_TMA)) break;
    }
    if (len > 0) {
      float* x = x_of(s);
      const float* hist = tail_of(s);
      const __nv_bfloat16* raw = reinterpret_cast<const __nv_bfloat16*>(tail_of(s));
      // ---- conv + SiLU (FUSED, shared with the other warps) or widening of all tokens; partial sums; gates ----
      if (FUSED) {
        team_conv(s, n, len, meta[i & 1].slot);
      } else if (qk_thread) {  // the isolated kernel's q, k: widened from bf16
        for (int tb = 0; tb < lb; tb += GDNC_SUB) {
          float psq[GDNC_SUB], psk[GDNC_SUB];
#pragma unroll
          for (int u = 0; u < GDNC_SUB; ++u) {
            const int t = tb + u;
            const float qv = t < len ? __bfloat162float(raw[(t * 3 + 0) * GDN_D + cc]) : 0.f;
            const float kv = t < len ? __bfloat162float(raw[(t * 3 + 1) * GDN_D + cc]) : 0.f;
            psq[u] = qv * qv;
            psk[u] = kv * kv;
          }
          const float tq = reduce16(psq, lane), tk = reduce16(psk, lane);
          if (!(lane & 1))
            *reinterpret_cast<float2*>(ipart + ((tb + reduce16_index(lane)) * 4 + warp) * 2) = make_float2(tq, tk);
        }
      } else {
        if (cc < lb) {  // gates of token cc: log decay g = -exp(A_log) softplus(a + dt_bias) (threshold 20), beta
          float gl = 0.f, be = 0.f;
          if (cc < len) {
            const size_t rt = (size_t)n * lb + cc;
            const float xg = args.a_raw[rt * GDN_H + h] + dtb;
            gl = negA * (xg > 20.f ? xg : log1pf(expf(xg)));
            be = sigmoidf_(args.b_raw[rt * GDN_H + h]);
          }
          igl[cc] = gl;
          ibe[cc] = be;
        }
        for (int t = 0; t < lb; ++t)  // the isolated kernel's v: widened from bf16
          x[(t * XS + SV) * GDN_D + cc] = t < len ? __bfloat162float(raw[(t * 3 + 2) * GDN_D + cc]) : 0.f;
      }
      mbar_arrive(cdone);  // the prologue may build this item's tables
      if (!mbar_wait(&full[1], i & 1, args.err, ERR_TIMEOUT_TMA)) break;  // the state tile landed
      const uint32_t half_base = smem_u32(stage_ptr(s)) + (warp >> 2) * GDNT_HALF;
      float sv[8][8];
#pragma unroll
      for (int kt = 0; kt < 8; ++kt) {
        uint32_t r[4];
        ldmatrix_x4_trans(half_base + sw128_off(16 * kt + frag_k, frag_c), r[0], r[1], r[2], r[3]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_half2(r[j]);
          sv[kt][2 * j] = f.x;
          sv[kt][2 * j + 1] = f.y;
        }
      }
      for (int sc = 0; sc < nsub; ++sc, ++jsub) {
        const int t0 = sc * GDNC_SUB;
        // z of this lane's outputs (tokens 8 nt + 2 t4 + e, columns v0, v0 + 8), requested early
        float zz[2][2][2] = {};
        if (FUSED) {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int t = t0 + 8 * nt + 2 * t4 + e;
              if (t < len) {
                const float* zr = args.proj + ((size_t)n * lb + t) * GDN_IN + GDN_Z_OFF + h * GDN_D + v0;
                zz[nt][e][0] = zr[0];
                zz[nt][e][1] = zr[8];
              }
            }
        }
        const bool ok = mbar_wait(&sfull[jsub & 1], (jsub >> 1) & 1, args.err, ERR_TIMEOUT_TMA);
        if (!named_sync_and<GDNT_CONS>(ok)) { alive = false; break; }
        const uint8_t* sb = scr(jsub);
        const uint8_t* bb = sb + GDNC_OFF_BOP;
        const float* vec = reinterpret_cast<const float*>(sb + GDNC_OFF_VEC);
        // ---- P = S^T K^T, R = S^T Q^T (16 v x 16 t each, two 8-token tiles) ----
        float pk[2][4] = {}, pq[2][4] = {};
#pragma unroll
        for (int kt = 0; kt < 8; ++kt) {
          const uint32_t a0 = pack_half2(sv[kt][0], sv[kt][1]), a1 = pack_half2(sv[kt][2], sv[kt][3]);
          const uint32_t a2 = pack_half2(sv[kt][4], sv[kt][5]), a3 = pack_half2(sv[kt][6], sv[kt][7]);
          const int ko = (16 * kt + 2 * t4) * 2;
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            const uint8_t* br = bb + (8 * nt + g) * GDNC_BOP_ROW + ko;
            mma_f16_16816(pk[nt], a0, a1, a2, a3, ld_u32(br), ld_u32(br + 16));
            mma_f16_16816(pk[nt], a0, a1, a2, a3, ld_u32(br + 256), ld_u32(br + 256 + 16));
            mma_f16_16816(pq[nt], a0, a1, a2, a3, ld_u32(br + 512), ld_u32(br + 512 + 16));
            mma_f16_16816(pq[nt], a0, a1, a2, a3, ld_u32(br + 768), ld_u32(br + 768 + 16));
          }
        }
        // ---- X[v][t] = beta_t (v_t[v] - Gam_t rk_t P) ----
        float xv[2][4], gq[2][2];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int tl = 8 * nt + 2 * t4 + e, t = t0 + tl;
            const float be = vec[1 * GDNC_SUB + tl], Gm = vec[2 * GDNC_SUB + tl];
            const float rk = vec[3 * GDNC_SUB + tl], rq = vec[4 * GDNC_SUB + tl];
            const float* vr = x + (t * XS + SV) * GDN_D + v0;
            xv[nt][e] = be * (vr[0] - Gm * rk * pk[nt][e]);
            xv[nt][2 + e] = be * (vr[8] - Gm * rk * pk[nt][2 + e]);
            gq[nt][e] = Gm * rq;  // o = Gam_t rq_t (S^T q_t) + ...
          }
        if (sc == nsub - 1) mbar_arrive(&empty[1]);  // this item's inputs are not read by the consumers again
        // ---- U^T = X T^T ----
        uint32_t xh[4], xl[4];
        split_half2x(xv[0][0], xv[0][1], xh[0], xl[0]);
        split_half2x(xv[0][2], xv[0][3], xh[1], xl[1]);
        split_half2x(xv[1][0], xv[1][1], xh[2], xl[2]);
        split_half2x(xv[1][2], xv[1][3], xh[3], xl[3]);
        const uint8_t* tmb = sb + GDNC_OFF_TM;
        const uint8_t* mqb = sb + GDNC_OFF_MQ;
        float u[2][4] = {};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const uint8_t* th = tmb + (8 * nt + g) * GDNC_T_ROW + 4 * t4;
          const uint8_t* tl = th + GDNC_SUB * GDNC_T_ROW;
          const uint32_t bh0 = ld_u32(th), bh1 = ld_u32(th + 16), bl0 = ld_u32(tl), bl1 = ld_u32(tl + 16);
          mma_f16_16816(u[nt], xh[0], xh[1], xh[2], xh[3], bh0, bh1);
          mma_f16_16816(u[nt], xh[0], xh[1], xh[2], xh[3], bl0, bl1);
          mma_f16_16816(u[nt], xl[0], xl[1], xl[2], xl[3], bh0, bh1);
        }
        uint32_t uh[4], ul[4];
        split_half2x(u[0][0], u[0][1], uh[0], ul[0]);
        split_half2x(u[0][2], u[0][3], uh[1], ul[1]);
        split_half2x(u[1][0], u[1][1], uh[2], ul[2]);
        split_half2x(u[1][2], u[1][3], uh[3], ul[3]);
        // ---- O^T = Gam rq (S^T Q^T) + U^T Mqk^T ----
        float o[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            o[nt][e] = gq[nt][e] * pq[nt][e];
            o[nt][2 + e] = gq[nt][e] * pq[nt][2 + e];
          }
          const uint8_t* mh = mqb + (8 * nt + g) * GDNC_T_ROW + 4 * t4;
          const uint8_t* ml = mh + GDNC_SUB * GDNC_T_ROW;
          const uint32_t bh0 = ld_u32(mh), bh1 = ld_u32(mh + 16), bl0 = ld_u32(ml), bl1 = ld_u32(ml + 16);
          mma_f16_16816(o[nt], uh[0], uh[1], uh[2], uh[3], bh0, bh1);
          mma_f16_16816(o[nt], uh[0], uh[1], uh[2], uh[3], bl0, bl1);
          mma_f16_16816(o[nt], ul[0], ul[1], ul[2], ul[3], bh0, bh1);
        }
        // ---- S^T <- Gam_C S^T + U^T K~ (the state registers are the accumulator) ----
        {
          const float GC = vec[5 * GDNC_SUB];
          const float2 gc2 = make_float2(GC, GC);
#pragma unroll
          for (int kt = 0; kt < 8; ++kt)
#pragma unroll
            for (int q4 = 0; q4 < 8; q4 += 2) {
              const float2 r = __fmul2_rn(make_float2(sv[kt][q4], sv[kt][q4 + 1]), gc2);
              sv[kt][q4] = r.x;
              sv[kt][q4 + 1] = r.y;
            }
          const uint8_t* ktb = sb + GDNC_OFF_KT;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            // row 8 j + g, s pairs t4 and t4 + 4, columns XOR-ed with (row >> 3) & 7 = j & 7
            const uint8_t* kh = ktb + (8 * j + g) * GDNC_KT_ROW;
            const uint8_t* kl = kh + GDN_D * GDNC_KT_ROW;
            const int c0 = (t4 ^ (j & 7)) * 4, c1 = ((t4 + 4) ^ (j & 7)) * 4;
            const uint32_t bh0 = ld_u32(kh + c0), bh1 = ld_u32(kh + c1), bl0 = ld_u32(kl + c0), bl1 = ld_u32(kl + c1);
            float* dd = &sv[j >> 1][4 * (j & 1)];
            mma_f16_16816_r(dd[0], dd[1], dd[2], dd[3], uh[0], uh[1], uh[2], uh[3], bh0, bh1);
            mma_f16_16816_r(dd[0], dd[1], dd[2], dd[3], uh[0], uh[1], uh[2], uh[3], bl0, bl1);
            mma_f16_16816_r(dd[0], dd[1], dd[2], dd[3], ul[0], ul[1], ul[2], ul[3], bh0, bh1);
          }
        }
        // ---- outputs ----
        if (FUSED) {
          // gated RMSNorm over the 128 v of each token: sums of squares across the 8 consumer warps
          float* sq = reinterpret_cast<float*>(scr(jsub) + GDNC_OFF_SQ);
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              float ss = o[nt][e] * o[nt][e] + o[nt][2 + e] * o[nt][2 + e];
              ss += __shfl_xor_sync(0xffffffffu, ss, 4);
              ss += __shfl_xor_sync(0xffffffffu, ss, 8);
              ss += __shfl_xor_sync(0xffffffffu, ss, 16);
              if (g == 0) sq[warp * GDNC_SUB + 8 * nt + 2 * t4 + e] = ss;
            }
          named_sync<GDNT_CONS>();
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int tl = 8 * nt + 2 * t4 + e, t = t0 + tl;
              if (t >= lb) continue;
              float var = 0.f;
#pragma unroll
              for (int w2 = 0; w2 < GDNT_CWARPS; ++w2) var += sq[w2 * GDNC_SUB + tl];
              const float r = rsqrtf(var * (1.0f / GDN_D) + args.eps);
              const size_t row = (size_t)n * lb + t;
              __nv_bfloat16 h0, l0, h1, l1;
              if (t < len) {
                split_bf16(gw0 * (o[nt][e] * r) * silu_fast(zz[nt][e][0]), h0, l0);
                split_bf16(gw1 * (o[nt][2 + e] * r) * silu_fast(zz[nt][e][1]), h1, l1);
              } else {
                h0 = l0 = h1 = l1 = __float2bfloat16_rn(0.f);
              }
              args.out_hi[row * KEY_DIM + h * GDN_D + v0] = h0;
              args.out_lo[row * KEY_DIM + h * GDN_D + v0] = l0;
              args.out_hi[row * KEY_DIM + h * GDN_D + v0 + 8] = h1;
              args.out_lo[row * KEY_DIM + h * GDN_D + v0 + 8] = l1;
            }
        } else {
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int t = t0 + 8 * nt + 2 * t4 + e;
              const size_t row = (size_t)n * lb + t;
              float* orow = args.o_raw + (row * GDN_H + h) * GDN_D;
              orow[v0] = t < len ? o[nt][e] : 0.f;
              orow[v0 + 8] = t < len ? o[nt][2 + e] : 0.f;
            }
        }
        mbar_arrive(&sdone[jsub & 1]);
      }
      if (!alive) break;
      // the new state, rounded to fp16 once, back into the stage
#pragma unroll
      for (int kt = 0; kt < 8; ++kt)
        stmatrix_x4_trans(half_base + sw128_off(16 * kt + frag_k, frag_c), pack_half2(sv[kt][0], sv[kt][1]),
                          pack_half2(sv[kt][2], sv[kt][3]), pack_half2(sv[kt][4], sv[kt][5]),
                          pack_half2(sv[kt][6], sv[kt][7]));
    }
    fence_proxy_async();   // this thread's writes to the stage are visible to the TMA store
    mbar_arrive(&done[0]);
  }
}

}  // namespace hsg
