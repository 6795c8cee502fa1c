// Gated delta rule slot step for small batches (the isolated kernel contract, RAW inputs): the state of one (row,
// head) split into four 32-column slices, one CTA each.
//
// The update is independent per value column v of the state S (dk x dv): with k^ = k / |k|, q^ = q 128^-1/2 / |q|,
//   kv_v = e^g sum_k S[k][v] k^_k,  delta_v = beta (v_v - kv_v),  S[k][v] <- e^g S[k][v] + k^_k delta_v,
//   o_v = e^g sum_k S_old[k][v] q^_k + (k^ . q^) delta_v
// (reference engine/fused_kernels.py:166-194, which tiles the same way with BV = 32). A slice is 128 x 32 values:
// 16 KB of fp32 state (8 KB fp16). With n rows the grid is (4 slices, 16 heads, n) -- 1,024 CTAs at 16 rows -- so a
// small batch is one wave of CTAs that each read their slice once and write it once, where the persistent kernels
// (144 CTAs, one (row, head) tile of 64 KB after another) leave most of the machine waiting on a few long chains.
//
// CTA of 256 threads: warp w owns state rows 16 w .. 16 w + 15 and lane l the slice's column l, 16 fp32 registers a
// thread. Per token the raw q, k (bf16, 128 each) and the slice's 32 v go to shared memory (three buffers, by token
// index mod 3), every warp forms |q|, |k| and q . k itself, the eight warps' partial column sums meet in shared memory
// (two buffers), then every thread finishes its column and updates its registers; one barrier a token. Slots outside
// [0, max_slots] and lengths outside [0, lb] are recorded in `err` and the row is skipped; padded tokens (t >= len)
// give o = 0. Measured at 16 rows (1,024 CTAs): 7.1 us a step inside a 1,000-step graph, 14.4 us for a single step
// after an L2 flush; 128-thread CTAs (32 rows a warp, one wave at eight a SM) took 12.3 / 23.5 us, 256 threads held
// to 40 registers (six a SM) 8.0 / 16.4 us.
#pragma once
#include "gdn.cuh"

namespace hsg {

constexpr int GDNS_SLICE = 32;                   // value columns per CTA
constexpr int GDNS_SLICES = GDN_D / GDNS_SLICE;  // 4
constexpr int GDNS_THREADS = 256;
constexpr int GDNS_ROWS = GDN_D / (GDNS_THREADS / 32);  // 16 state rows per warp
constexpr int GDNS_MAX_ROWS = 32;                // batches up to this many rows use this kernel

template <typename ST>
__global__ void __launch_bounds__(GDNS_THREADS) gdn_cols_kernel(const GdnArgs args) {
  // Token t's inputs go to buffer t % 3: the load of token t + 1 (before token t's barrier) must not meet a warp still
  // reading token t - 1's k and v (its update runs after token t - 1's barrier). The partial sums are written and read
  // on either side of one barrier, so two buffers suffice for them.
  __shared__ __align__(16) float qk[3][2 * GDN_D];          // raw q | k of the token
  __shared__ float vs[3][GDNS_SLICE];                       // the slice's raw v
  __shared__ float2 part[2][GDNS_THREADS / 32][GDNS_SLICE];  // per warp: (S^T k, S^T q) partial sums of a column
  const int slice = blockIdx.x, h = blockIdx.y, n = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lb = args.lb;
  const int col = slice * GDNS_SLICE + lane;
  int len = (int)args.lens[n];
  const int64_t slot = args.slots[n];
  if (len < 0 || len > lb) {
    if (tid == 0) set_error(args.err, ERR_BAD_LEN);
    len = 0;
  }
  if (len > 0 && (slot < 0 || slot > args.max_slots)) {
    if (tid == 0) set_error(args.err, ERR_BAD_SLOT);
    len = 0;
  }
  float* o_row = args.o_raw + ((size_t)n * lb * GDN_H + h) * GDN_D + col;  // o[n][t][h][col] = o_row[t * 16 * 128]
  if (warp == 0)
    for (int t = len; t < lb; ++t) o_row[(size_t)t * GDN_H * GDN_D] = 0.f;
  if (len == 0) return;

  ST* tile = static_cast<ST*>(args.state) + ((size_t)slot * GDN_H + h) * (GDN_D * GDN_D);
  float sv[GDNS_ROWS];
#pragma unroll
  for (int r = 0; r < GDNS_ROWS; ++r) sv[r] = to_f32(tile[(warp * GDNS_ROWS + r) * GDN_D + col]);
  const float negA = -expf(args.A_log[h]), dtb = args.dt_bias[h];
  const float scale = 0.08838834764831845f;  // 128^-1/2, correctly rounded

  auto load_token = [&](int t) {
    const size_t row = (size_t)n * lb + t;
    const __nv_bfloat16* src = args.packed + row * CONV_DIM + h * GDN_D;
    for (int i = tid; i < 2 * GDN_D; i += GDNS_THREADS)  // q (i < 128), then k
      qk[t % 3][i] = __bfloat162float(src[(i >> 7) * KEY_DIM + (i & 127)]);
    if (tid < GDNS_SLICE) vs[t % 3][tid] = __bfloat162float(src[2 * KEY_DIM + slice * GDNS_SLICE + tid]);
  };
  load_token(0);
  __syncthreads();
  for (int t = 0; t < len; ++t) {
    const float* q = qk[t % 3];
    const float* k = q + GDN_D;
    // |q|, |k| and q . k of the token by every warp (no barrier); the normalisation is folded in below
    float rq, rk, dqk;
    {
      const float4 qa = reinterpret_cast<const float4*>(q)[lane];
      const float4 ka = reinterpret_cast<const float4*>(k)[lane];
      const float sq = warp_sum(qa.x * qa.x + qa.y * qa.y + qa.z * qa.z + qa.w * qa.w);
      const float sk = warp_sum(ka.x * ka.x + ka.y * ka.y + ka.z * ka.z + ka.w * ka.w);
      const float sqk = warp_sum(qa.x * ka.x + qa.y * ka.y + qa.z * ka.z + qa.w * ka.w);
      rq = scale / sqrtf(sq + 1e-6f);
      rk = 1.0f / sqrtf(sk + 1e-6f);
      dqk = sqk * rq * rk;
    }
    const size_t row = (size_t)n * lb + t;
    const float xg = args.a_raw[row * GDN_H + h] + dtb;
    const float sp = xg > 20.f ? xg : log1pf(expf(xg));
    const float eg = expf(negA * sp);
    const float beta = sigmoidf_(args.b_raw[row * GDN_H + h]);
    float pk0 = 0.f, pk1 = 0.f, pq0 = 0.f, pq1 = 0.f;
    const float* kr = k + warp * GDNS_ROWS;
    const float* qr = q + warp * GDNS_ROWS;
#pragma unroll
    for (int r = 0; r < GDNS_ROWS; r += 2) {
      pk0 = fmaf(sv[r], kr[r], pk0);
      pk1 = fmaf(sv[r + 1], kr[r + 1], pk1);
      pq0 = fmaf(sv[r], qr[r], pq0);
      pq1 = fmaf(sv[r + 1], qr[r + 1], pq1);
    }
    part[t & 1][warp][lane] = make_float2((pk0 + pk1) * rk, (pq0 + pq1) * rq);
    if (t + 1 < len) load_token(t + 1);
    __syncthreads();
    float kvs = 0.f, qss = 0.f;
#pragma unroll
    for (int w = 0; w < GDNS_THREADS / 32; ++w) {
      const float2 p = part[t & 1][w][lane];
      kvs += p.x;
      qss += p.y;
    }
    const float dl = beta * (vs[t % 3][lane] - eg * kvs);
    if (warp == 0) o_row[(size_t)t * GDN_H * GDN_D] = fmaf(eg, qss, dqk * dl);
    const float kdl = rk * dl;
#pragma unroll
    for (int r = 0; r < GDNS_ROWS; ++r) sv[r] = fmaf(eg, sv[r], kr[r] * kdl);
  }
#pragma unroll
  for (int r = 0; r < GDNS_ROWS; ++r) tile[(warp * GDNS_ROWS + r) * GDN_D + col] = from_f32<ST>(sv[r]);
}

}  // namespace hsg
