// Gated softmax attention over a 512-token ring window, per session slot (reference engine/fused_kernels.py:252-376,
// engine/slot_engine_v8.py:241-256, window_attention.py:34-53).
//
// Ring layout (per attention layer): K and V [max_slots+1][2 kv heads][513][256] fp16; column c of a slot holds the
// token at position p with p % 512 == c, ring_pos[slot][c] = p (-1 when empty); column 512 and slot max_slots are
// scratch. A query at position p sees key position kp iff 0 <= kp <= p and kp > p - 512.
//
// attn_prep_kernel   one CTA per token: per-head RMSNorm (1 + w) of q (8 heads) and k (2 heads), RoPE on the first
//                    64 dims (rotate-half, fp32 sincos of pos * inv_freq), q -> fp32 grouped layout
//                    [nb][kv head][4*lb rows][256] (row = group * lb + token), k, v -> fp16 [nb][kv head][lb][256].
// ring_attn_kernel   one CTA per (row, kv head, block of RB query rows): streams the slot's ring (32-column tiles of
//                    K and V, 16 KB each, one TMA bulk copy per tile, double-buffered, empty tiles skipped) and then
//                    this tick's new keys, with an online softmax in fp32; epilogue multiplies by sigmoid(gate) and
//                    writes the o_proj operand as a bf16 hi/lo pair. For 1-token ticks it also writes the new K/V into
//                    the ring (the overwritten column holds position p - 512, which this query cannot see).
// ring_append_kernel multi-token ticks: writes the tick's K/V into the ring after attention (earlier queries of the
//                    tick may still need the positions the new columns overwrite).
// ring_commit_kernel after all layers: ring_pos[slot][p % 512] = p for valid tokens; padded tokens write -1 to the
//                    scratch column (reference slot_engine_v8.py:224).
#pragma once
#include "common.cuh"

namespace hsg {

struct AttnArgs {
  const int64_t* slots;
  const int64_t* lens;
  const int64_t* starts;
  int nb, lb, max_slots;
  const float* proj;        // [nb*lb, ATT_IN] fused input projection (q|gate per head, k, v)
  const float* q_norm;      // [256] 1 + w
  const float* k_norm;      // [256] 1 + w
  const float* inv_freq;    // [32]
  float eps;
  float* qbuf;              // [nb][2][4*lb][256]
  __half* knew;             // [nb][2][lb][256]
  __half* vnew;
  __half* ring_k;           // [max_slots+1][2][513][256] (this layer)
  __half* ring_v;
  int64_t* ring_pos;        // [max_slots+1][513]
  __nv_bfloat16* out_hi;    // [nb*lb, 2048]
  __nv_bfloat16* out_lo;
  float* out_raw;           // isolated kernel: ungated fp32 output [nb][2][4*lb][256] instead of out_hi/out_lo
  int write_ring;           // 1-token ticks: store the new key/value at column start % 512 after attending
  float scale;
  int* err;
};

constexpr int RING_COLS = WIN + 1;

// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) attn_prep_kernel(const AttnArgs args) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  const int n = m / args.lb, t = m % args.lb;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t pos = args.starts[n] + t;
  const float* row = args.proj + (size_t)m * ATT_IN;
  // rotary angles for this lane's 8 dims (only lanes 0..7 cover the 64 rotary dims)
  float cs[8], sn[8];
  if (lane < 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float ang = (float)pos * args.inv_freq[(lane * 8 + j) & 31];
      sincosf(ang, &sn[j], &cs[j]);
    }
  }
  // this warp's jobs (heads): warp and warp + 8. Every input and norm weight is requested before the first output
  // store: a load issued after a global store cannot be moved above it (possible aliasing), which would cost warps
  // with two jobs a second round trip.
  constexpr int NJOB = ATT_HQ + 2 * ATT_HKV;
  float x[2][8], wn[2][8];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int job = warp + 8 * r;
    if (job >= NJOB) break;
    const float* src;
    const float* w = nullptr;
    if (job < ATT_HQ) { src = row + job * 2 * ATT_D; w = args.q_norm; }
    else if (job < ATT_HQ + ATT_HKV) { src = row + ATT_K_OFF + (job - ATT_HQ) * ATT_D; w = args.k_norm; }
    else src = row + ATT_V_OFF + (job - ATT_HQ - ATT_HKV) * ATT_D;
    const float4 a = reinterpret_cast<const float4*>(src)[lane * 2];
    const float4 b = reinterpret_cast<const float4*>(src)[lane * 2 + 1];
    x[r][0] = a.x; x[r][1] = a.y; x[r][2] = a.z; x[r][3] = a.w; x[r][4] = b.x; x[r][5] = b.y; x[r][6] = b.z; x[r][7] = b.w;
    if (w) {
      const float4 c = reinterpret_cast<const float4*>(w)[lane * 2];
      const float4 d = reinterpret_cast<const float4*>(w)[lane * 2 + 1];
      wn[r][0] = c.x; wn[r][1] = c.y; wn[r][2] = c.z; wn[r][3] = c.w; wn[r][4] = d.x; wn[r][5] = d.y; wn[r][6] = d.z; wn[r][7] = d.w;
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int job = warp + 8 * r;
    if (job >= NJOB) break;
    float* xr = x[r];
    if (job < ATT_HQ + ATT_HKV) {  // q and k heads: RMSNorm (1 + w) and RoPE
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += xr[j] * xr[j];
      const float rs = 1.0f / sqrtf(warp_sum(ss) * (1.0f / ATT_D) + args.eps);
#pragma unroll
      for (int j = 0; j < 8; ++j) xr[j] = xr[j] * rs * wn[r][j];
      // rotate-half over dims 0..63: partner of dim d < 32 is d + 32 (lane + 4)
      float partner[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) partner[j] = __shfl_xor_sync(0xffffffffu, xr[j], 4);
      if (lane < 8) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float rot = lane < 4 ? -partner[j] : partner[j];
          xr[j] = xr[j] * cs[j] + rot * sn[j];
        }
      }
    }
    if (job < ATT_HQ) {
      const int kvh = job / ATT_G, g = job % ATT_G;
      float* dst = args.qbuf + (((size_t)n * ATT_HKV + kvh) * (ATT_G * args.lb) + g * args.lb + t) * ATT_D + lane * 8;
      reinterpret_cast<float4*>(dst)[0] = make_float4(xr[0], xr[1], xr[2], xr[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(xr[4], xr[5], xr[6], xr[7]);
    } else {
      const bool is_k = job < ATT_HQ + ATT_HKV;
      const int kvh = is_k ? job - ATT_HQ : job - ATT_HQ - ATT_HKV;
      __half* dst = (is_k ? args.knew : args.vnew) + (((size_t)n * ATT_HKV + kvh) * args.lb + t) * ATT_D + lane * 8;
      __half2 h4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) h4[j] = __floats2half2_rn(xr[2 * j], xr[2 * j + 1]);
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(h4);
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
constexpr int ATT_TILE = 32;                       // keys per tile
constexpr int ATT_TILE_BYTES = ATT_TILE * ATT_D * 2;  // 16 KB (fp16)
constexpr int ATT_THREADS = 256;

constexpr int ATT_RPOS_BYTES = 2096;  // 513 int32 ring positions + tile count, rounded up to 16 bytes

__host__ __device__ inline int attn_smem_bytes(int rb) {
  // K,V double buffer | ring_pos (int32) + tile count | scores/probs [32][rb] | acc exchange [4][256] | row stats |
  // barriers
  return 4 * ATT_TILE_BYTES + ATT_RPOS_BYTES + ATT_TILE * rb * 4 + 4 * ATT_D * 4 + 3 * 8 * 4 + 2 * 8 + 128;
}

// Reduce-scatter of N (16 or 32) per-lane values over a warp: afterwards lane L holds the warp-wide sum of value
// index L (N = 32) or L >> 1 (N = 16).
template <int N>
__device__ __forceinline__ float reduce_scatter(float (&v)[N], int lane) {
#pragma unroll
  for (int off = 16, n = N; n > 1; off >>= 1, n >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  if (N == 16) v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
  return v[0];
}

// RB query rows per CTA (4 or 8). Thread layout in the P.V step: thread t owns dims 2*(t%128), +1; with RB = 8 the
// two 128-thread groups split the rows (4 each), with RB = 4 they split the keys (even / odd) and are summed at the end.
template <int RB>
__global__ void __launch_bounds__(ATT_THREADS, 2) ring_attn_kernel(const AttnArgs args) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t attn_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(attn_smem_raw) + 127) & ~uintptr_t(127));
  __half* kbuf = reinterpret_cast<__half*>(smem);                 // [2][32][256]
  __half* vbuf = kbuf + 2 * ATT_TILE * ATT_D;                     // [2][32][256]
  int* rpos = reinterpret_cast<int*>(vbuf + 2 * ATT_TILE * ATT_D);  // [513]
  int* ntiles_sh = rpos + RING_COLS;
  float* sc = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(rpos) + ATT_RPOS_BYTES);  // [32 keys][RB rows]
  float* xacc = sc + ATT_TILE * RB;                               // [4][256]
  float* m_i = xacc + 4 * ATT_D;
  float* l_i = m_i + 8;
  float* alpha = l_i + 8;
  uint64_t* full = reinterpret_cast<uint64_t*>(alpha + 8);        // [2]

  const int n = blockIdx.x, kvh = blockIdx.y, rb0 = blockIdx.z * RB;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lb = args.lb, M = ATT_G * lb;
  int len = (int)args.lens[n];
  const int64_t slot = args.slots[n], start = args.starts[n];
  if (len > 0 && (slot < 0 || slot > args.max_slots)) {
    if (tid == 0) set_error(args.err, ERR_BAD_SLOT);
    len = 0;
  }
  const size_t head = (size_t)n * ATT_HKV + kvh;

  // per-row query position (rows beyond M or padded tokens never see a key)
  int64_t qpos[RB];
  bool qval[RB];
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    const int row = rb0 + r;
    const int t = row % lb;
    qpos[r] = start + t;
    qval[r] = row < M && t < len;
  }

  if (len == 0) {
    for (int r = 0; r < RB; ++r) {
      const int row = rb0 + r;
      if (row >= M) break;
      if (args.out_raw) {
        args.out_raw[(head * M + row) * ATT_D + tid] = 0.f;
        continue;
      }
      const int g = row / lb, t = row % lb;
      const size_t o = ((size_t)n * lb + t) * (ATT_HQ * ATT_D) + (kvh * ATT_G + g) * ATT_D + tid;
      args.out_hi[o] = __float2bfloat16_rn(0.f);
      args.out_lo[o] = __float2bfloat16_rn(0.f);
    }
    return;
  }
  const __half* rk = args.ring_k + ((size_t)slot * ATT_HKV + kvh) * RING_COLS * ATT_D;
  const __half* rv = args.ring_v + ((size_t)slot * ATT_HKV + kvh) * RING_COLS * ATT_D;
  const __half* nk = args.knew + head * lb * ATT_D;
  const __half* nv = args.vnew + head * lb * ATT_D;

  // ring positions -> shared (int32); tiles with no filled column are skipped
  for (int c = tid; c < RING_COLS; c += ATT_THREADS) {
    const int64_t p = args.ring_pos[(size_t)slot * RING_COLS + c];
    rpos[c] = p < 0 ? -1 : (p > 0x7fffffff ? 0x7fffffff : (int)p);
  }
  if (tid < 8) { m_i[tid] = -INFINITY; l_i[tid] = 0.f; }
  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_barrier_init();
  }
  __syncthreads();
  // tile list: ring tiles 0..15 with any filled column, then ceil(lb / 32) tiles of this tick's keys
  __shared__ uint8_t tiles[WIN / ATT_TILE + 2];
  if (tid == 0) {
    int nt = 0;
    for (int i = 0; i < WIN / ATT_TILE; ++i) {
      bool any = false;
      for (int c = 0; c < ATT_TILE; ++c) any |= rpos[i * ATT_TILE + c] >= 0;
      if (any) tiles[nt++] = (uint8_t)i;
    }
    for (int j = 0; j * ATT_TILE < lb; ++j) tiles[nt++] = (uint8_t)(WIN / ATT_TILE + j);
    *ntiles_sh = nt;
  }
  __syncthreads();
  const int nt = *ntiles_sh;

  auto issue = [&](int i) {
    const int tile = tiles[i], b = i & 1;
    const __half *ks, *vs;
    uint32_t rows;
    if (tile < WIN / ATT_TILE) {
      ks = rk + (size_t)tile * ATT_TILE * ATT_D;
      vs = rv + (size_t)tile * ATT_TILE * ATT_D;
      rows = ATT_TILE;
    } else {
      const int t0 = (tile - WIN / ATT_TILE) * ATT_TILE;
      ks = nk + (size_t)t0 * ATT_D;
      vs = nv + (size_t)t0 * ATT_D;
      rows = min(ATT_TILE, lb - t0);
    }
    fence_proxy_async();
    mbar_arrive_expect_tx(&full[b], 2 * rows * ATT_D * 2);
    bulk_g2s(kbuf + b * ATT_TILE * ATT_D, ks, rows * ATT_D * 2, &full[b]);
    bulk_g2s(vbuf + b * ATT_TILE * ATT_D, vs, rows * ATT_D * 2, &full[b]);
  };
  if (tid == 0 && nt > 0) issue(0);

  // queries for this lane's 8 dims, all RB rows, in registers
  float q[RB][8];
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    const int row = min(rb0 + r, M - 1);
    const float* src = args.qbuf + (head * M + row) * ATT_D + lane * 8;
    const float4 a = reinterpret_cast<const float4*>(src)[0], b = reinterpret_cast<const float4*>(src)[1];
    q[r][0] = a.x; q[r][1] = a.y; q[r][2] = a.z; q[r][3] = a.w;
    q[r][4] = b.x; q[r][5] = b.y; q[r][6] = b.z; q[r][7] = b.w;
  }
  // P.V accumulators: 2 dims x 4 rows per thread
  const int grp = tid >> 7, dp = tid & 127;
  float acc[4][2];
#pragma unroll
  for (int r = 0; r < 4; ++r) acc[r][0] = acc[r][1] = 0.f;
  const int row_off = RB == 8 ? grp * 4 : 0;
  bool ok = true;

  for (int i = 0; i < nt && ok; ++i) {
    const int b = i & 1, tile = tiles[i];
    if (tid == 0 && i + 1 < nt) issue(i + 1);
    ok = __syncthreads_and(mbar_wait(&full[b], (i >> 1) & 1, args.err, ERR_TIMEOUT_TMA));
    if (!ok) break;
    const bool ring_tile = tile < WIN / ATT_TILE;
    const int ncols = ring_tile ? ATT_TILE : min(ATT_TILE, lb - (tile - WIN / ATT_TILE) * ATT_TILE);
    const __half* kt = kbuf + b * ATT_TILE * ATT_D;
    const __half* vt = vbuf + b * ATT_TILE * ATT_D;
    // ---- scores: warp w handles keys 4w..4w+3 ----
    {
      float part[4 * RB];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int c = warp * 4 + kk;
        float kf[8];
        if (c < ncols) {
          const uint4 raw = *reinterpret_cast<const uint4*>(kt + c * ATT_D + lane * 8);
          const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(h2[j]);
            kf[2 * j] = f.x; kf[2 * j + 1] = f.y;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) kf[j] = 0.f;
        }
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          float d = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) d = fmaf(q[r][j], kf[j], d);
          part[kk * RB + r] = d;
        }
      }
      const float s = reduce_scatter<4 * RB>(part, lane);
      const int idx = RB == 8 ? lane : (lane >> 1);
      const int kk = idx / RB, r = idx % RB;
      const int c = warp * 4 + kk;
      int64_t kp;
      if (ring_tile) kp = rpos[tile * ATT_TILE + c];
      else {
        const int t2 = (tile - WIN / ATT_TILE) * ATT_TILE + c;
        kp = (c < ncols && t2 < len) ? start + t2 : -1;
      }
      const bool vis = qval[r] && kp >= 0 && kp <= qpos[r] && kp > qpos[r] - WIN;
      if (RB == 8 || (lane & 1) == 0) sc[c * RB + r] = vis ? s * args.scale : -INFINITY;
    }
    __syncthreads();
    // ---- online softmax: warp r updates row r ----
    if (warp < RB) {
      const int r = warp;
      const float s = sc[lane * RB + r];
      const float mt = warp_max(s);
      const float mold = m_i[r];
      const float mnew = fmaxf(mold, mt);
      const float msafe = mnew == -INFINITY ? 0.f : mnew;
      const float p = expf(s - msafe);
      const float ps = warp_sum(p);
      sc[lane * RB + r] = p;
      if (lane == 0) {
        const float al = expf(mold - msafe);
        alpha[r] = al;
        l_i[r] = l_i[r] * al + ps;
        m_i[r] = mnew;
      }
    }
    __syncthreads();
    // ---- P.V ----
    {
      float al[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) al[r] = r + row_off < RB ? alpha[r + row_off] : 1.f;
#pragma unroll
      for (int r = 0; r < 4; ++r) { acc[r][0] *= al[r]; acc[r][1] *= al[r]; }
      const int cstart = RB == 4 ? grp : 0, cstep = RB == 4 ? 2 : 1;
      for (int c = cstart; c < ncols; c += cstep) {
        const float2 vf = __half22float2(reinterpret_cast<const __half2*>(vt + c * ATT_D)[dp]);
        const float4 p = *reinterpret_cast<const float4*>(sc + c * RB + row_off);
        acc[0][0] = fmaf(p.x, vf.x, acc[0][0]); acc[0][1] = fmaf(p.x, vf.y, acc[0][1]);
        acc[1][0] = fmaf(p.y, vf.x, acc[1][0]); acc[1][1] = fmaf(p.y, vf.y, acc[1][1]);
        acc[2][0] = fmaf(p.z, vf.x, acc[2][0]); acc[2][1] = fmaf(p.z, vf.y, acc[2][1]);
        acc[3][0] = fmaf(p.w, vf.x, acc[3][0]); acc[3][1] = fmaf(p.w, vf.y, acc[3][1]);
      }
    }
    __syncthreads();  // buffer b may be refilled by the next issue
  }
  if (!ok) {
    // error path: wait (bounded) for any copy still in flight before leaving
    for (int b = 0; b < 2; ++b) mbar_wait(&full[b], 0, nullptr, 0);
    return;
  }
  if (RB == 4) {  // sum the even-key and odd-key halves
    if (grp == 1) {
#pragma unroll
      for (int r = 0; r < 4; ++r) { xacc[r * ATT_D + 2 * dp] = acc[r][0]; xacc[r * ATT_D + 2 * dp + 1] = acc[r][1]; }
    }
    __syncthreads();
    if (grp == 0) {
#pragma unroll
      for (int r = 0; r < 4; ++r) { acc[r][0] += xacc[r * ATT_D + 2 * dp]; acc[r][1] += xacc[r * ATT_D + 2 * dp + 1]; }
    }
  }
  if (RB == 8 || grp == 0) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int rr = r + row_off, row = rb0 + rr;
      if (row >= M) continue;
      const int g = row / lb, t = row % lb, j = kvh * ATT_G + g;
      if (args.out_raw) {
        const float inv = (qval[rr] && l_i[rr] > 0.f) ? 1.0f / l_i[rr] : 0.f;
        *reinterpret_cast<float2*>(args.out_raw + (head * M + row) * ATT_D + 2 * dp) =
            make_float2(acc[r][0] * inv, acc[r][1] * inv);
        continue;
      }
      const size_t o = ((size_t)n * lb + t) * (ATT_HQ * ATT_D) + j * ATT_D + 2 * dp;
      float y0 = 0.f, y1 = 0.f;
      if (qval[rr] && l_i[rr] > 0.f) {
        const float* gate = args.proj + ((size_t)n * lb + t) * ATT_IN + j * 2 * ATT_D + ATT_D + 2 * dp;
        const float inv = 1.0f / l_i[rr];
        y0 = acc[r][0] * inv * sigmoidf_(gate[0]);
        y1 = acc[r][1] * inv * sigmoidf_(gate[1]);
      }
      split_bf16(y0, args.out_hi[o], args.out_lo[o]);
      split_bf16(y1, args.out_hi[o + 1], args.out_lo[o + 1]);
    }
  }
  if (args.write_ring && lb == 1 && blockIdx.z == 0) {
    // single-token tick: the new key/value go straight into the ring (column start % 512)
    __syncthreads();
    const size_t col = (size_t)(start % WIN);
    __half* dk = args.ring_k + (((size_t)slot * ATT_HKV + kvh) * RING_COLS + col) * ATT_D;
    __half* dv = args.ring_v + (((size_t)slot * ATT_HKV + kvh) * RING_COLS + col) * ATT_D;
    if (tid < ATT_D) { dk[tid] = nk[tid]; dv[tid] = nv[tid]; }
  }
}

// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) ring_append_kernel(const AttnArgs args) {
  pdl_wait();
  pdl_trigger();
  const int n = blockIdx.x, kvh = blockIdx.y;
  const int len = (int)args.lens[n];
  const int64_t slot = args.slots[n], start = args.starts[n];
  if (len <= 0 || slot < 0 || slot > args.max_slots) return;
  const size_t head = (size_t)n * ATT_HKV + kvh;
  // thread = (16-byte chunk c of a 256-dim row, token t0 + 8 i): every load is issued before any store (a store
  // could alias a later load as far as the compiler knows, which would serialise one round trip per token)
  static_assert(MAX_LB <= 64 && ATT_D * 2 / 16 == 32, "eight tokens of 32 chunks per pass, at most 64 tokens");
  const int c = threadIdx.x & 31, t0 = threadIdx.x >> 5;
  const uint4* nk = reinterpret_cast<const uint4*>(args.knew) + head * args.lb * 32;
  const uint4* nv = reinterpret_cast<const uint4*>(args.vnew) + head * args.lb * 32;
  uint4 kr[8], vr[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int t = t0 + 8 * i;
    if (t < len) {
      kr[i] = nk[t * 32 + c];
      vr[i] = nv[t * 32 + c];
    }
  }
  uint4* rk = reinterpret_cast<uint4*>(args.ring_k) + ((size_t)slot * ATT_HKV + kvh) * RING_COLS * 32;
  uint4* rv = reinterpret_cast<uint4*>(args.ring_v) + ((size_t)slot * ATT_HKV + kvh) * RING_COLS * 32;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int t = t0 + 8 * i;
    if (t < len) {
      const size_t col = (size_t)((start + t) % WIN);
      rk[col * 32 + c] = kr[i];
      rv[col * 32 + c] = vr[i];
    }
  }
}

__global__ void ring_commit_kernel(const int64_t* slots, const int64_t* lens, const int64_t* starts, int nb, int lb,
                                   int max_slots, int64_t* ring_pos) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nb * lb) return;
  const int n = i / lb, t = i % lb;
  const int64_t slot = slots[n];
  if (slot < 0 || slot > max_slots) return;
  const bool valid = t < lens[n];
  const int64_t pos = starts[n] + t;
  const int64_t col = valid ? pos % WIN : WIN;
  ring_pos[slot * RING_COLS + col] = valid ? pos : -1;
}

}  // namespace hsg
