// Gated delta rule ("GDN") slot step as a persistent, head-stationary, warp-specialised TMA pipeline (sm_100a).
//
// Work item = (session row n, head h). The grid is (16 heads, P) with P = 9 CTAs per head (144 CTAs, one per SM);
// CTA (h, p) serves rows p, p + P, p + 2P, ... of head h, so its conv and gated-norm weights, A_log and dt_bias stay
// in registers for the whole launch.
//
// The recurrent state is kept in HBM as fp16 (the reference StreamingGuard's state_dtype, runtime.py:157) or fp32
// (template parameter ST); in shared memory it keeps that type and in registers it is fp32.
//
// Producer warp (warp 16): for each item, waits until its shared-memory stage is free, writes the previous occupant's
// updated state tile (32 KB fp16 / 64 KB fp32) back to HBM with one TMA bulk store, then loads the item's inputs with
// TMA bulk copies -- the state tile (contiguous in the pool [S+1][16][128][128]), the head's q/k/v/z projection slices
// and the slot's 3-row conv history -- completing on the stage's `full` barrier. It runs up to STAGES items ahead.
// Consumer warps (16 warps; thread t owns state column t % 128, rows 32*(t/128)..+31, in registers), per item:
//   conv: silu(causal depthwise conv, kernel 4) over [history | new tokens] in place, history rolled to global;
//   q, k L2-normalised (eps 1e-6), q scaled by 128^-1/2; g = -exp(A_log) softplus(a + dt_bias) (threshold 20),
//   beta = sigmoid(b)  (reference engine/fused_kernels.py:140-194, transformers torch_recurrent_gated_delta_rule);
//   per token: S <- e^g S; delta = beta (v - S^T k); S <- S + k delta^T; o = S^T q, computed as
//   o = e^g S_old^T q + (k.q) delta from one pass over the registers, the four row-group partial sums combined in
//   shared memory; the new state goes back into the stage; output = gated RMSNorm w * (o * rsqrt(mean(o^2)+eps)) *
//   silu(z) as the out_proj operand (bf16 hi/lo pair); then every consumer arrives on the stage's `empty` barrier.
// RAW variant (isolated kernel, contract of the reference's gdn_slot_v8, fused_kernels.py:197-211): q/k/v arrive
// post-conv as bf16 [n][lb][6144], a/b as fp32 [n][lb][16], the output o is fp32 [n][lb][16][128].
#pragma once
#include "common.cuh"

namespace hsg {

struct GdnArgs {
  const int64_t* slots;  // [nb]
  const int64_t* lens;   // [nb]
  int nb, lb, max_slots;
  int stages;            // shared-memory stages (host: gdn_stages(lb))
  // FUSED inputs
  const float* proj;     // [nb*lb, GDN_IN] fp32 output of the fused input projection
  float* conv_pool;      // [max_slots+1, 3, CONV_DIM] fp32 history (this layer)
  const float* conv_w;   // [CONV_DIM, 4]
  const float* gnorm_w;  // [128]
  float eps;
  __nv_bfloat16* out_hi; // [nb*lb, KEY_DIM] out_proj operand
  __nv_bfloat16* out_lo;
  // RAW inputs
  const __nv_bfloat16* packed;  // [nb, lb, CONV_DIM] q | k | v after conv+silu
  const float* a_raw;           // [nb, lb, 16]
  const float* b_raw;           // [nb, lb, 16]
  float* o_raw;                 // [nb, lb, 16, 128]
  // both
  const float* A_log;   // [16]
  const float* dt_bias; // [16]
  void* state;          // [max_slots+1, 16, 128, 128] ST (fp16 or fp32), updated in place
  int* err;
};

constexpr int GDN_CONSUMERS = 512;
constexpr int GDN_THREADS = GDN_CONSUMERS + 32;  // + one producer warp
constexpr int GDN_CWARPS = GDN_CONSUMERS / 32;
constexpr int GDN_RG = GDN_CONSUMERS / GDN_D;    // 4 row groups of 32 rows
constexpr int GDN_CTAS_PER_HEAD = 9;             // 16 x 9 = 144 persistent CTAs on the 148 SMs
constexpr int GDN_SMEM_LIMIT = 227 * 1024;
constexpr int GDN_MAX_STAGES = 6;
template <typename ST>
__host__ __device__ constexpr int gdn_tile_bytes() { return GDN_D * GDN_D * (int)sizeof(ST); }

struct GdnMeta {  // per stage, written by the producer before it arrives on `full`
  int64_t slot;
  int len, pad;
};

// Stage layout: state tile (tile_bytes) | x [lb][4][128] fp32 (q, k, v, z slices; RAW: q, k, v bf16 in the first
// half) | hist [3][3][128] fp32 (q, k, v channel blocks).
__host__ __device__ inline int gdn_stage_bytes(int lb, int tile_bytes) {
  return tile_bytes + lb * 4 * GDN_D * 4 + 9 * GDN_D * 4;
}
__host__ __device__ inline int gdn_fixed_bytes() {
  // partial sums [2][4][128] float2 | g, beta, q.k [64] | meta, full, empty barriers [GDN_MAX_STAGES] | alignment
  return 2 * GDN_RG * GDN_D * 8 + 3 * MAX_LB * 4 + GDN_MAX_STAGES * (16 + 2 * 8) + 128;
}
__host__ __device__ inline int gdn_stages(int lb, int tile_bytes) {
  int s = (GDN_SMEM_LIMIT - gdn_fixed_bytes()) / gdn_stage_bytes(lb, tile_bytes);
  return s > GDN_MAX_STAGES ? GDN_MAX_STAGES : (s < 1 ? 1 : s);
}
__host__ __device__ inline int gdn_smem_bytes(int lb, int tile_bytes) {
  return gdn_stages(lb, tile_bytes) * gdn_stage_bytes(lb, tile_bytes) + gdn_fixed_bytes();
}

template <bool FUSED, typename ST>
__global__ void __launch_bounds__(GDN_THREADS, 1) gdn_step_kernel(const GdnArgs args) {
  constexpr int TILE = gdn_tile_bytes<ST>();
  ST* const state_pool = static_cast<ST*>(args.state);
  extern __shared__ __align__(128) uint8_t gdn_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gdn_smem_raw) + 127) & ~uintptr_t(127));
  const int lb = args.lb, S = args.stages;
  const int sbytes = gdn_stage_bytes(lb, TILE);
  uint8_t* fixed = smem + S * sbytes;
  float2* red = reinterpret_cast<float2*>(fixed);                  // [2][4][128]
  float* gv = reinterpret_cast<float*>(red + 2 * GDN_RG * GDN_D);  // decay factors e^g per token
  float* bv = gv + MAX_LB;                                         // beta per token
  float* qk = bv + MAX_LB;                                         // q.k per token
  GdnMeta* meta = reinterpret_cast<GdnMeta*>(qk + MAX_LB);         // [GDN_MAX_STAGES]
  uint64_t* full = reinterpret_cast<uint64_t*>(meta + GDN_MAX_STAGES);
  uint64_t* empty = full + GDN_MAX_STAGES;

  const int h = blockIdx.x, p = blockIdx.y, P = gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_items = args.nb > p ? (args.nb - p + P - 1) / P : 0;
  auto row_of = [&](int i) { return p + i * P; };
  auto stage_ptr = [&](int s) { return smem + s * sbytes; };

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GDN_CONSUMERS);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == GDN_CWARPS) {
    // ===================================== producer =====================================
    int64_t held_slot[GDN_MAX_STAGES] = {};
    int held_len[GDN_MAX_STAGES] = {};
    // Part 1 of an item's loads: metadata, expected bytes, the state tile and the conv history. These belong to this
    // layer alone (no earlier kernel of the tick touches them), so for the first stages they are issued before the
    // dependency wait. Part 2: the projection slices written by the preceding GEMM.
    auto issue_state = [&](int i) {
      const int s = i % S, n = row_of(i);
      int len = (int)args.lens[n];
      const int64_t slot = args.slots[n];
      if (len < 0 || len > lb) {
        if (lane == 0) set_error(args.err, ERR_BAD_LEN);
        len = 0;
      }
      if (len > 0 && (slot < 0 || slot > args.max_slots)) {
        if (lane == 0) set_error(args.err, ERR_BAD_SLOT);
        len = 0;
      }
      held_slot[s] = slot;
      held_len[s] = len;
      uint8_t* st = stage_ptr(s);
      float* hist = reinterpret_cast<float*>(st + TILE) + lb * 4 * GDN_D;
      if (lane == 0) {
        meta[s].slot = slot;
        meta[s].len = len;
        if (len > 0)
          mbar_arrive_expect_tx(&full[s], TILE +
                                              (FUSED ? len * 4 * GDN_D * 4 + 9 * GDN_D * 4 : len * 3 * GDN_D * 2));
        else
          mbar_arrive(&full[s]);
      }
      __syncwarp();
      if (len == 0) return;
      if (lane == 0) bulk_g2s(st, state_pool + ((size_t)slot * GDN_H + h) * (GDN_D * GDN_D), TILE, &full[s]);
      if (FUSED && lane < 9) {  // conv history: 3 rows x (q, k, v) channel blocks
        const int rr = lane / 3, part = lane % 3;
        const float* src = args.conv_pool + ((size_t)slot * CONV_KEEP + rr) * CONV_DIM + part * KEY_DIM + h * GDN_D;
        bulk_g2s(hist + (rr * 3 + part) * GDN_D, src, GDN_D * 4, &full[s]);
      }
    };
    auto issue_inputs = [&](int i) {
      const int s = i % S, n = row_of(i), len = held_len[s];
      if (len == 0) return;
      float* x = reinterpret_cast<float*>(stage_ptr(s) + TILE);
      if (FUSED) {
        for (int j = lane; j < len * 4; j += 32) {  // q, k, v, z slices of each token: 4 x 512 B
          const int t = j >> 2, part = j & 3;
          const float* src = args.proj + ((size_t)n * lb + t) * GDN_IN + part * KEY_DIM + h * GDN_D;
          bulk_g2s(x + (t * 4 + part) * GDN_D, src, GDN_D * 4, &full[s]);
        }
      } else {
        __nv_bfloat16* xb = reinterpret_cast<__nv_bfloat16*>(x);
        for (int j = lane; j < len * 3; j += 32) {
          const int t = j / 3, part = j % 3;
          const __nv_bfloat16* src = args.packed + ((size_t)n * lb + t) * CONV_DIM + part * KEY_DIM + h * GDN_D;
          bulk_g2s(xb + (t * 3 + part) * GDN_D, src, GDN_D * 2, &full[s]);
        }
      }
    };
    const int pre = n_items < S ? n_items : S;
    for (int i = 0; i < pre; ++i) issue_state(i);
    pdl_wait();
    for (int i = 0; i < pre; ++i) issue_inputs(i);
    for (int i = S; i < n_items + S; ++i) {
      const int s = i % S, r = i / S;
      if (i - S < n_items) {
        // the consumers are done with item i - S in stage s: write its state back
        if (!mbar_wait(&empty[s], (r - 1) & 1, args.err, ERR_TIMEOUT_TMA)) break;
        if (lane == 0 && held_len[s] > 0) {
          bulk_s2g(state_pool + ((size_t)held_slot[s] * GDN_H + h) * (GDN_D * GDN_D), stage_ptr(s), TILE);
          bulk_commit();
        }
      }
      if (i >= n_items) continue;
      if (lane == 0) bulk_wait_read_all();  // the store has read the stage
      __syncwarp();
      issue_state(i);
      issue_inputs(i);
    }
    if (lane == 0) bulk_wait_all();
    return;
  }

  // ===================================== consumers =====================================
  const int col = tid & (GDN_D - 1), rg = tid >> 7;
  float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);  // thread t < 384 owns conv channel t % 128 of block t / 128
  if (FUSED && tid < 3 * GDN_D)
    cw = *reinterpret_cast<const float4*>(args.conv_w + (size_t)((tid >> 7) * KEY_DIM + h * GDN_D + col) * CONV_K);
  const float4 gw = FUSED ? reinterpret_cast<const float4*>(args.gnorm_w)[lane] : make_float4(0.f, 0.f, 0.f, 0.f);
  const float negA = -expf(args.A_log[h]), dtb = args.dt_bias[h];

  // a, b of an item (thread t < lb holds token t), loaded one item ahead so the latency hides behind compute
  auto load_ab = [&](int i, float& a, float& b) {
    a = 0.f;
    b = 0.f;
    if (i >= n_items || tid >= lb) return;
    const int n = row_of(i);  // padded tokens' values are loaded too (in bounds) and never used
    if (FUSED) {
      const float* row = args.proj + ((size_t)n * lb + tid) * GDN_IN;
      a = row[GDN_A_OFF + h];
      b = row[GDN_B_OFF + h];
    } else {
      a = args.a_raw[((size_t)n * lb + tid) * GDN_H + h];
      b = args.b_raw[((size_t)n * lb + tid) * GDN_H + h];
    }
  };
  pdl_wait();
  if (tid == 0) pdl_trigger();
  float cur_a, cur_b;
  load_ab(0, cur_a, cur_b);
  bool broken = false;

  for (int i = 0; i < n_items && !broken; ++i) {
    float nxt_a, nxt_b;
    load_ab(i + 1, nxt_a, nxt_b);
    const int s = i % S, n = row_of(i);
    uint8_t* st = stage_ptr(s);
    ST* stile = reinterpret_cast<ST*>(st);
    float* x = reinterpret_cast<float*>(st + TILE);
    float* hist = x + lb * 4 * GDN_D;
    if (!named_sync_and<GDN_CONSUMERS>(mbar_wait(&full[s], (i / S) & 1, args.err, ERR_TIMEOUT_TMA))) {
      broken = true;
      break;
    }
    const int len = meta[s].len;
    const int64_t slot = meta[s].slot;
    if (len == 0) {
      for (int e = tid; e < lb * GDN_D; e += GDN_CONSUMERS) {
        const size_t row = (size_t)n * lb + e / GDN_D;
        if (FUSED) {
          args.out_hi[row * KEY_DIM + h * GDN_D + (e & 127)] = __float2bfloat16_rn(0.f);
          args.out_lo[row * KEY_DIM + h * GDN_D + (e & 127)] = __float2bfloat16_rn(0.f);
        } else {
          args.o_raw[(row * GDN_H + h) * GDN_D + (e & 127)] = 0.f;
        }
      }
    } else {
      // ---- prologue: q, k, v of the tokens, in place at x[t][0..2] ----
      if (FUSED) {
        if (tid < 3 * GDN_D) {
          const int c3 = tid >> 7;
          float e0 = hist[(0 * 3 + c3) * GDN_D + col], e1 = hist[(1 * 3 + c3) * GDN_D + col],
                e2 = hist[(2 * 3 + c3) * GDN_D + col];
          for (int t = 0; t < len; ++t) {
            float* xp = x + (t * 4 + c3) * GDN_D + col;
            const float xv = *xp;
            float acc = cw.x * e0;
            acc = fmaf(cw.y, e1, acc);
            acc = fmaf(cw.z, e2, acc);
            acc = fmaf(cw.w, xv, acc);
            *xp = silu(acc);
            e0 = e1; e1 = e2; e2 = xv;
          }
          float* g = args.conv_pool + (size_t)slot * CONV_KEEP * CONV_DIM + c3 * KEY_DIM + h * GDN_D + col;
          g[0] = e0;
          g[CONV_DIM] = e1;
          g[2 * CONV_DIM] = e2;
        }
      } else {
        // bf16 q, k, v occupy the first half of the x area: widen from the last token down
        const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(x);
        for (int t = len - 1; t >= 0; --t) {
          float v = 0.f;
          if (tid < 3 * GDN_D) v = __bfloat162float(xb[(t * 3 + (tid >> 7)) * GDN_D + col]);
          named_sync<GDN_CONSUMERS>();
          if (tid < 3 * GDN_D) x[(t * 4 + (tid >> 7)) * GDN_D + col] = v;
          named_sync<GDN_CONSUMERS>();
        }
      }
      if (tid < len) {
        const float xg = cur_a + dtb;
        const float sp = xg > 20.f ? xg : log1pf(expf(xg));
        gv[tid] = expf(negA * sp);
        bv[tid] = sigmoidf_(cur_b);
      }
      named_sync<GDN_CONSUMERS>();  // conv outputs, decay and beta of every token are in shared memory
      // ---- recurrence ----
      float sv[32];
#pragma unroll
      for (int r = 0; r < 32; ++r) sv[r] = to_f32(stile[(rg * 32 + r) * GDN_D + col]);
      const float scale = 0.08838834764831845f;  // 128^-1/2, correctly rounded
      for (int t = 0; t < len; ++t) {
        // L2 norms (eps 1e-6) and q.k of token t, computed by every warp from the raw conv outputs (no barrier);
        // the normalisation is folded into the dot products and the update below
        float rq, rk, dqk;
        {
          const float4 qa = reinterpret_cast<const float4*>(x + (t * 4 + 0) * GDN_D)[lane];
          const float4 ka = reinterpret_cast<const float4*>(x + (t * 4 + 1) * GDN_D)[lane];
          const float sq = warp_sum(qa.x * qa.x + qa.y * qa.y + qa.z * qa.z + qa.w * qa.w);
          const float sk = warp_sum(ka.x * ka.x + ka.y * ka.y + ka.z * ka.z + ka.w * ka.w);
          const float sqk = warp_sum(qa.x * ka.x + qa.y * ka.y + qa.z * ka.z + qa.w * ka.w);
          rq = scale / sqrtf(sq + 1e-6f);
          rk = 1.0f / sqrtf(sk + 1e-6f);
          dqk = sqk * rq * rk;
        }
        const float4* q4 = reinterpret_cast<const float4*>(x + (t * 4 + 0) * GDN_D + rg * 32);
        const float4* k4 = reinterpret_cast<const float4*>(x + (t * 4 + 1) * GDN_D + rg * 32);
        float pk0 = 0.f, pk1 = 0.f, pq0 = 0.f, pq1 = 0.f;
#pragma unroll
        for (int r4 = 0; r4 < 8; ++r4) {
          const float4 kk = k4[r4], qq = q4[r4];
          pk0 = fmaf(sv[4 * r4 + 0], kk.x, pk0); pk1 = fmaf(sv[4 * r4 + 1], kk.y, pk1);
          pk0 = fmaf(sv[4 * r4 + 2], kk.z, pk0); pk1 = fmaf(sv[4 * r4 + 3], kk.w, pk1);
          pq0 = fmaf(sv[4 * r4 + 0], qq.x, pq0); pq1 = fmaf(sv[4 * r4 + 1], qq.y, pq1);
          pq0 = fmaf(sv[4 * r4 + 2], qq.z, pq0); pq1 = fmaf(sv[4 * r4 + 3], qq.w, pq1);
        }
        float2* rb = red + (t & 1) * GDN_RG * GDN_D;
        rb[rg * GDN_D + col] = make_float2((pk0 + pk1) * rk, (pq0 + pq1) * rq);
        named_sync<GDN_CONSUMERS>();
        float kvs = 0.f, qss = 0.f;
#pragma unroll
        for (int r = 0; r < GDN_RG; ++r) {
          const float2 a = rb[r * GDN_D + col];
          kvs += a.x;
          qss += a.y;
        }
        const float eg = gv[t];
        const float dl = bv[t] * (x[(t * 4 + 2) * GDN_D + col] - eg * kvs);
        // q[t] was consumed before the barrier above: its slot now holds o[t]
        if (rg == 0) x[(t * 4 + 0) * GDN_D + col] = fmaf(eg, qss, dqk * dl);
        const float kdl = rk * dl;
#pragma unroll
        for (int r4 = 0; r4 < 8; ++r4) {
          const float4 kk = k4[r4];
          sv[4 * r4 + 0] = fmaf(eg, sv[4 * r4 + 0], kk.x * kdl);
          sv[4 * r4 + 1] = fmaf(eg, sv[4 * r4 + 1], kk.y * kdl);
          sv[4 * r4 + 2] = fmaf(eg, sv[4 * r4 + 2], kk.z * kdl);
          sv[4 * r4 + 3] = fmaf(eg, sv[4 * r4 + 3], kk.w * kdl);
        }
      }
#pragma unroll
      for (int r = 0; r < 32; ++r) stile[(rg * 32 + r) * GDN_D + col] = from_f32<ST>(sv[r]);
      named_sync<GDN_CONSUMERS>();  // o[t] complete for the epilogue
      // ---- epilogue ----
      if (FUSED) {
        for (int t = warp; t < lb; t += GDN_CWARPS) {
          const size_t row = (size_t)n * lb + t;
          __nv_bfloat16* oh = args.out_hi + row * KEY_DIM + h * GDN_D + lane * 4;
          __nv_bfloat16* ol = args.out_lo + row * KEY_DIM + h * GDN_D + lane * 4;
          __nv_bfloat16 hv[4], lv[4];
          if (t >= len) {
#pragma unroll
            for (int j = 0; j < 4; ++j) hv[j] = lv[j] = __float2bfloat16_rn(0.f);
          } else {
            const float4 o4 = reinterpret_cast<const float4*>(x + (t * 4 + 0) * GDN_D)[lane];
            const float4 z4 = reinterpret_cast<const float4*>(x + (t * 4 + 3) * GDN_D)[lane];
            const float var = warp_sum(o4.x * o4.x + o4.y * o4.y + o4.z * o4.z + o4.w * o4.w) * (1.0f / GDN_D);
            const float r = 1.0f / sqrtf(var + args.eps);
            const float y[4] = {gw.x * (o4.x * r) * silu(z4.x), gw.y * (o4.y * r) * silu(z4.y),
                                gw.z * (o4.z * r) * silu(z4.z), gw.w * (o4.w * r) * silu(z4.w)};
#pragma unroll
            for (int j = 0; j < 4; ++j) split_bf16(y[j], hv[j], lv[j]);
          }
          *reinterpret_cast<uint2*>(oh) = *reinterpret_cast<uint2*>(hv);
          *reinterpret_cast<uint2*>(ol) = *reinterpret_cast<uint2*>(lv);
        }
      } else {
        for (int e = tid; e < lb * GDN_D; e += GDN_CONSUMERS) {
          const int t = e >> 7;
          const size_t row = (size_t)n * lb + t;
          args.o_raw[(row * GDN_H + h) * GDN_D + (e & 127)] = t < len ? x[(t * 4 + 0) * GDN_D + (e & 127)] : 0.f;
        }
      }
    }
    fence_proxy_async();   // this thread's writes to the stage are visible to the bulk store
    mbar_arrive(&empty[s]);
    cur_a = nxt_a;
    cur_b = nxt_b;
  }
}

}  // namespace hsg
