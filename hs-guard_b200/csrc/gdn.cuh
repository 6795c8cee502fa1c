// Gated delta rule ("GDN") slot step: one CTA per (session row, head), 128 threads.
//
// The per-(slot, head) state S is a 128 x 128 fp32 tile (64 KB, contiguous in the pool [S+1][16][128][128]). It is
// staged into shared memory with one TMA bulk copy issued before anything else, so the HBM read overlaps the
// prologue. Each thread then owns a 32-row x 4-column block of S in registers (thread t: columns 4*(t%32)..+3, rows
// 32*(t/32)..+31) and, per token,
//     S <- e^g S;  delta = beta (v - S^T k);  S <- S + k delta^T;  o = S^T q
// using  S^T k  and  S^T q  from one pass over the registers (o = e^g S_old^T q + (k.q) delta), with the four
// row-group partial sums combined through shared memory (double-buffered, one barrier per token). The final state
// is written back with coalesced 16-byte stores.
//
// FUSED variant (engine): the prologue is the causal depthwise conv (kernel 4) + SiLU over the head's 384 q/k/v
// channels of the fused input projection, rolling the slot's fp32 conv history; the epilogue is the gated RMSNorm
// over dv = 128 with z (Qwen3_5RMSNormGated) and writes the out_proj operand as a bf16 hi/lo pair.
// RAW variant (isolated kernel, reference engine/fused_kernels.py:140-211 contract): q/k/v come post-conv as bf16,
// the output o is fp32.
//
// Reference math: q, k L2-normalised with eps 1e-6 and q scaled by dk^-1/2; g = -exp(A_log) softplus(a + dt_bias)
// (softplus threshold 20); beta = sigmoid(b) (fused_kernels.py:166-188; transformers torch_recurrent_gated_delta_rule).
#pragma once
#include "common.cuh"

namespace hsg {

struct GdnArgs {
  // session rows
  const int64_t* slots;  // [nb]
  const int64_t* lens;   // [nb]
  int nb, lb, max_slots;
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
  float* state;         // [max_slots+1, 16, 128, 128] fp32, updated in place
  int* err;
};

constexpr int GDN_THREADS = 128;
constexpr int GDN_TILE_BYTES = GDN_D * GDN_D * 4;

__host__ __device__ inline int gdn_smem_bytes(int lb) {
  // state tile | q,k,v,o [lb][128] | partial sums [2][4][128] float2 | g, beta, qk [lb] | mbarrier
  return GDN_TILE_BYTES + 4 * lb * GDN_D * 4 + 2 * 4 * GDN_D * 8 + 3 * MAX_LB * 4 + 64 + 128;
}

template <bool FUSED>
__global__ void __launch_bounds__(GDN_THREADS, 3) gdn_step_kernel(const GdnArgs args) {
  extern __shared__ __align__(128) uint8_t gdn_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gdn_smem_raw) + 127) & ~uintptr_t(127));
  const int lb = args.lb;
  float* st = reinterpret_cast<float*>(smem);
  float* qs = st + GDN_D * GDN_D;
  float* ks = qs + lb * GDN_D;
  float* vs = ks + lb * GDN_D;
  float* os = vs + lb * GDN_D;
  float2* red = reinterpret_cast<float2*>(os + lb * GDN_D);  // [2][4][128]
  float* gv = reinterpret_cast<float*>(red + 2 * 4 * GDN_D);
  float* bv = gv + MAX_LB;
  float* qk = bv + MAX_LB;
  uint64_t* bar = reinterpret_cast<uint64_t*>(qk + MAX_LB);

  const int h = blockIdx.x, n = blockIdx.y, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  int len = (int)args.lens[n];
  int64_t slot = args.slots[n];
  if (len < 0 || len > lb) {
    if (tid == 0) set_error(args.err, ERR_BAD_LEN);
    len = 0;
  }
  if (len > 0 && (slot < 0 || slot > args.max_slots)) {
    if (tid == 0) set_error(args.err, ERR_BAD_SLOT);
    len = 0;
  }
  float* gstate = args.state + ((size_t)slot * GDN_H + h) * (GDN_D * GDN_D);

  if (len == 0) {  // padding row: zero output, no state or history update
    for (int t = 0; t < lb; ++t) {
      const size_t row = (size_t)n * lb + t;
      if (FUSED) {
        args.out_hi[row * KEY_DIM + h * GDN_D + tid] = __float2bfloat16_rn(0.f);
        args.out_lo[row * KEY_DIM + h * GDN_D + tid] = __float2bfloat16_rn(0.f);
      } else {
        args.o_raw[(row * GDN_H + h) * GDN_D + tid] = 0.f;
      }
    }
    return;
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(bar, GDN_TILE_BYTES);
    bulk_g2s(st, gstate, GDN_TILE_BYTES, bar);
  }

  // ---- prologue: q, k, v for the head into shared memory ----
  if (FUSED) {
    const int chan[3] = {h * GDN_D + tid, KEY_DIM + h * GDN_D + tid, 2 * KEY_DIM + h * GDN_D + tid};
    float* dst[3] = {qs, ks, vs};
    float* hist = args.conv_pool + (size_t)slot * CONV_KEEP * CONV_DIM;
#pragma unroll
    for (int c3 = 0; c3 < 3; ++c3) {
      const int c = chan[c3];
      const float4 w = *reinterpret_cast<const float4*>(args.conv_w + (size_t)c * CONV_K);
      float e0 = hist[c], e1 = hist[CONV_DIM + c], e2 = hist[2 * CONV_DIM + c];
      for (int t = 0; t < len; ++t) {
        const float x = args.proj[((size_t)n * lb + t) * GDN_IN + c];
        float acc = w.x * e0;
        acc = fmaf(w.y, e1, acc);
        acc = fmaf(w.z, e2, acc);
        acc = fmaf(w.w, x, acc);
        dst[c3][t * GDN_D + tid] = silu(acc);
        e0 = e1; e1 = e2; e2 = x;
      }
      hist[c] = e0;
      hist[CONV_DIM + c] = e1;
      hist[2 * CONV_DIM + c] = e2;
    }
  } else {
    for (int t = 0; t < len; ++t) {
      const __nv_bfloat16* src = args.packed + ((size_t)n * lb + t) * CONV_DIM + h * GDN_D + tid;
      qs[t * GDN_D + tid] = __bfloat162float(src[0]);
      ks[t * GDN_D + tid] = __bfloat162float(src[KEY_DIM]);
      vs[t * GDN_D + tid] = __bfloat162float(src[2 * KEY_DIM]);
    }
  }
  if (tid < len) {
    float a, b;
    if (FUSED) {
      const float* row = args.proj + ((size_t)n * lb + tid) * GDN_IN;
      a = row[GDN_A_OFF + h];
      b = row[GDN_B_OFF + h];
    } else {
      a = args.a_raw[((size_t)n * lb + tid) * GDN_H + h];
      b = args.b_raw[((size_t)n * lb + tid) * GDN_H + h];
    }
    const float x = a + args.dt_bias[h];
    const float sp = x > 20.f ? x : log1pf(expf(x));
    gv[tid] = expf(-expf(args.A_log[h]) * sp);   // decay factor e^g
    bv[tid] = sigmoidf_(b);
  }
  __syncthreads();
  // L2 norms (eps 1e-6) and q.k per token; warp w takes tokens w, w+4, ...
  const float scale = 0.08838834764831845f;  // 128^-1/2, correctly rounded
  for (int t = warp; t < len; t += 4) {
    float4 q4 = reinterpret_cast<float4*>(qs + t * GDN_D)[lane];
    float4 k4 = reinterpret_cast<float4*>(ks + t * GDN_D)[lane];
    float sq = warp_sum(q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w);
    float sk = warp_sum(k4.x * k4.x + k4.y * k4.y + k4.z * k4.z + k4.w * k4.w);
    const float rq = scale / sqrtf(sq + 1e-6f), rk = 1.0f / sqrtf(sk + 1e-6f);
    q4.x *= rq; q4.y *= rq; q4.z *= rq; q4.w *= rq;
    k4.x *= rk; k4.y *= rk; k4.z *= rk; k4.w *= rk;
    reinterpret_cast<float4*>(qs + t * GDN_D)[lane] = q4;
    reinterpret_cast<float4*>(ks + t * GDN_D)[lane] = k4;
    const float d = warp_sum(q4.x * k4.x + q4.y * k4.y + q4.z * k4.z + q4.w * k4.w);
    if (lane == 0) qk[t] = d;
  }
  // ---- recurrence ----
  const bool have = __syncthreads_and(mbar_wait(bar, 0, args.err, ERR_TIMEOUT_TMA));
  if (!have) {  // the bulk copy never landed: error recorded, state left untouched; one more bounded wait, then leave
    mbar_wait(bar, 0, nullptr, 0);
    return;
  }
  const int c4 = lane, rg = warp;      // columns 4*c4..4*c4+3, rows 32*rg..32*rg+31
  float4 s[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) s[i] = reinterpret_cast<const float4*>(st + (rg * 32 + i) * GDN_D)[c4];
  for (int t = 0; t < len; ++t) {
    const float* kt = ks + t * GDN_D + rg * 32;
    const float* qt = qs + t * GDN_D + rg * 32;
    float4 pk = make_float4(0.f, 0.f, 0.f, 0.f), pq = pk;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float kv = kt[i], qv = qt[i];
      pk.x = fmaf(s[i].x, kv, pk.x); pk.y = fmaf(s[i].y, kv, pk.y);
      pk.z = fmaf(s[i].z, kv, pk.z); pk.w = fmaf(s[i].w, kv, pk.w);
      pq.x = fmaf(s[i].x, qv, pq.x); pq.y = fmaf(s[i].y, qv, pq.y);
      pq.z = fmaf(s[i].z, qv, pq.z); pq.w = fmaf(s[i].w, qv, pq.w);
    }
    float2* rb = red + (t & 1) * 4 * GDN_D;
    float4* rbv = reinterpret_cast<float4*>(rb + rg * GDN_D + c4 * 4);
    rbv[0] = make_float4(pk.x, pq.x, pk.y, pq.y);
    rbv[1] = make_float4(pk.z, pq.z, pk.w, pq.w);
    __syncthreads();
    float kvs[4] = {0.f, 0.f, 0.f, 0.f}, qss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float4* p = reinterpret_cast<const float4*>(rb + r * GDN_D + c4 * 4);
      const float4 a0 = p[0], a1 = p[1];
      kvs[0] += a0.x; qss[0] += a0.y; kvs[1] += a0.z; qss[1] += a0.w;
      kvs[2] += a1.x; qss[2] += a1.y; kvs[3] += a1.z; qss[3] += a1.w;
    }
    const float eg = gv[t], beta = bv[t], dqk = qk[t];
    const float4 v4 = reinterpret_cast<const float4*>(vs + t * GDN_D)[c4];
    const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
    float dl[4], ov[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dl[j] = beta * (vv[j] - eg * kvs[j]);
      ov[j] = fmaf(eg, qss[j], dqk * dl[j]);
    }
    if (rg == 0) reinterpret_cast<float4*>(os + t * GDN_D)[c4] = make_float4(ov[0], ov[1], ov[2], ov[3]);
    const float* kr = ks + t * GDN_D + rg * 32;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float kv = kr[i];
      s[i].x = fmaf(eg, s[i].x, kv * dl[0]);
      s[i].y = fmaf(eg, s[i].y, kv * dl[1]);
      s[i].z = fmaf(eg, s[i].z, kv * dl[2]);
      s[i].w = fmaf(eg, s[i].w, kv * dl[3]);
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) reinterpret_cast<float4*>(gstate + (rg * 32 + i) * GDN_D)[c4] = s[i];
  __syncthreads();

  // ---- epilogue ----
  if (FUSED) {
    // gated RMSNorm over dv: w * (o * rsqrt(mean(o^2) + eps)) * silu(z); warp w takes tokens w, w+4, ...
    const float4 gw = reinterpret_cast<const float4*>(args.gnorm_w)[lane];
    for (int t = warp; t < lb; t += 4) {
      const size_t row = (size_t)n * lb + t;
      __nv_bfloat16* oh = args.out_hi + row * KEY_DIM + h * GDN_D + lane * 4;
      __nv_bfloat16* ol = args.out_lo + row * KEY_DIM + h * GDN_D + lane * 4;
      if (t >= len) {
        for (int j = 0; j < 4; ++j) { oh[j] = __float2bfloat16_rn(0.f); ol[j] = __float2bfloat16_rn(0.f); }
        continue;
      }
      const float4 o4 = reinterpret_cast<const float4*>(os + t * GDN_D)[lane];
      const float var = warp_sum(o4.x * o4.x + o4.y * o4.y + o4.z * o4.z + o4.w * o4.w) * (1.0f / GDN_D);
      const float r = 1.0f / sqrtf(var + args.eps);
      const float4 z4 = *reinterpret_cast<const float4*>(args.proj + row * GDN_IN + GDN_Z_OFF + h * GDN_D + lane * 4);
      const float y[4] = {gw.x * (o4.x * r) * silu(z4.x), gw.y * (o4.y * r) * silu(z4.y),
                          gw.z * (o4.z * r) * silu(z4.z), gw.w * (o4.w * r) * silu(z4.w)};
#pragma unroll
      for (int j = 0; j < 4; ++j) split_bf16(y[j], oh[j], ol[j]);
    }
  } else {
    for (int t = 0; t < lb; ++t) {
      const size_t row = (size_t)n * lb + t;
      args.o_raw[(row * GDN_H + h) * GDN_D + tid] = t < len ? os[t * GDN_D + tid] : 0.f;
    }
  }
}

}  // namespace hsg
