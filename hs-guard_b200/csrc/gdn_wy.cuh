// Chunked gated delta rule on the 5th-generation tensor cores (tcgen05, accumulators in TMEM) for 32- and 64-token
// ticks with fp16 recurrent state (the engine's FUSED inputs): the whole tick is one chunk of C = lb tokens.
//
// Per (row, head) item, with the state S (dk x dv, fp16 at the tick's start), k^_t = rk_t k_t, q^_t = rq_t q_t,
// cumulative log decay gam_t = sum_{s<=t} g_s, Gam_t = e^gam_t, beta_t (the chunked WY form of the reference's
// complete-message path, FLA chunk.py; the same algebra as gdn_chunk.cuh with one chunk instead of four):
//   KK = K^ K^T, QK = Q^ K^T, P = S^T K^T, R = S^T Q^T                       (tensor cores, fp16 hi/lo operands)
//   A[t][s] = beta_t e^(gam_t - gam_s) KK[t][s] (s < t),  T = (I + A)^-1    (CUDA cores, fp32 forward substitution)
//   Mqk[t][s] = e^(gam_t - gam_s) QK[t][s] (s <= t)
//   X[v][t] = beta_t (v_t[v] - Gam_t P[v][t])
//   U^T = X T^T                                                               (tensor cores)
//   O^T = U^T Mqk^T,  dS^T = U^T K~  with K~[s][k] = e^(gam_C - gam_s) k^_s[k]   (tensor cores)
//   o_t = Gam_t R[., t] + O^T[., t],   S <- Gam_C S + dS
// Every exponent is <= 0. Padded tokens (t >= len) carry q = k = v = 0, g = 0, beta = 0: they change nothing.
//
// Every tensor-core operand is K-major with 128-byte swizzle in 64-element K blocks (rows of 128 bytes, 8-row atoms),
// the layout the GEMM kernels use: K^, Q^ (rows = tokens), the state transposed to S^T (rows = v, built from the
// TMA-loaded [k][v] tile with ldmatrix.trans / stmatrix), T and Mqk (rows = t, K = s), X and U^T (rows = v, K = t),
// K~^T (rows = k, K = s). K^ and Q^ are stacked in one operand (rows 0 .. C - 1 and 64 .. 64 + C - 1 of each 128-row
// K block), so KK and QK are one M = 128 product with K^ and P, R one N = 128 product with S^T. All MMAs are M = 128.
// TMEM (fp32 columns): KK|QK (C) | P|R (128) | U^T | O^T (C each) | dS^T (128): 448 columns at C = 64.
//
// Warps: 0-7 compute (warp w reads TMEM lane quadrant w % 4), 8 the TMA producer, 9 the MMA issuer (owns TMEM).
// Shared memory regions are reused as the item proceeds: the fp32 q and k inputs become the K^ / Q^ operands in
// place, then after the first MMAs hold T / Mqk (q region) and U^T (k region); the S^T copy becomes X. The next item's
// inputs are loaded as soon as the last MMAs of this one have completed; its state once this item's state is stored.
// Every wait is bounded and reports through `err`.
#pragma once
#include "gdn_chunk.cuh"

namespace hsg {

constexpr int GDNW_COMPUTE = 256;
constexpr int GDNW_PROD_WARP = 8;
constexpr int GDNW_MMA_WARP = 9;
constexpr int GDNW_THREADS = GDNW_COMPUTE + 64;
constexpr int GDNW_MAXC = 64;
// region byte offsets (sized for C = 64; a 32-token tick uses the same layout)
constexpr int GDNW_R_STATE = 0;                               // fp16 state tile, two [128 k][64 v] SW128 halves
constexpr int GDNW_R_Q = GDNW_R_STATE + GDNT_TILE;            // q fp32 [C][128] -> [K^; Q^] hi -> T hi|lo, Mqk hi|lo
constexpr int GDNW_R_K = GDNW_R_Q + GDNW_MAXC * GDN_D * 4;    // k fp32 [C][128] -> [K^; Q^] lo -> U^T hi|lo
constexpr int GDNW_R_V = GDNW_R_K + GDNW_MAXC * GDN_D * 4;    // v fp32 [C][128]
constexpr int GDNW_R_ST = GDNW_R_V + GDNW_MAXC * GDN_D * 4;   // S^T fp16 (two K blocks of [128 v][64 k]) -> X hi|lo
constexpr int GDNW_R_KT = GDNW_R_ST + GDN_D * GDN_D * 2;      // K~^T hi | lo, [128 k][64 s] each
constexpr int GDNW_R_HIST = GDNW_R_KT + 2 * GDN_D * 128;      // conv history [3][3][128] fp32
constexpr int GDNW_A_STRIDE = GDNW_MAXC + 1;
constexpr int GDNW_R_A = GDNW_R_HIST + 9 * GDN_D * 4;         // A [64][65] fp32 for the triangular solve
constexpr int GDNW_R_VEC = GDNW_R_A + GDNW_MAXC * GDNW_A_STRIDE * 4;  // gam, Gam, beta, rk, rq, g [64] f32 + gC
constexpr int GDNW_R_PART = GDNW_R_VEC + 7 * GDNW_MAXC * 4;   // per-token q.q, k.k partial sums [64][4][2] f32
constexpr int GDNW_R_ONORM = GDNW_R_PART + GDNW_MAXC * 8 * 4; // output sum of squares [4 quadrants][64] f32
constexpr int GDNW_R_META = GDNW_R_ONORM + 4 * GDNW_MAXC * 4; // item metadata (slot, len) x 2, by item parity
constexpr int GDNW_R_BAR = GDNW_R_META + 32;                  // mbarriers
constexpr int GDNW_NBAR = 12;
constexpr int GDNW_SMEM = GDNW_R_BAR + GDNW_NBAR * 8 + 16 + 1024;
// TMEM column offsets for a chunk of C tokens. KK and QK share columns [0, C): KK in lanes 0 .. C - 1, QK in lanes
// 64 .. 64 + C - 1 (one product of the stacked [K^; Q^] operand with K^). P and R share the 128 columns of one
// N = 128 product S^T [K^; Q^]^T: P in the first C, R in the C from column 64.
__host__ __device__ constexpr int gdnw_col_kq(int) { return 0; }
__host__ __device__ constexpr int gdnw_col_p(int c) { return c; }
__host__ __device__ constexpr int gdnw_col_r(int c) { return c + 64; }
__host__ __device__ constexpr int gdnw_col_u(int c) { return c + 128; }
__host__ __device__ constexpr int gdnw_col_o(int c) { return 2 * c + 128; }
__host__ __device__ constexpr int gdnw_col_ds(int c) { return 3 * c + 128; }

// Byte offset of element (row r, K index k) in a K-major SW128 operand whose K blocks of 64 are `kblock` bytes apart.
__device__ __forceinline__ uint32_t kmaj_off(int r, int k, int kblock) {
  return (k >> 6) * kblock + r * 128 + ((((k & 63) >> 3) ^ (r & 7)) << 4) + (k & 7) * 2;
}
// Byte offset of state element (k, v) in the TMA-loaded tile (two [128 k][64 v] halves with 128-byte swizzle).
__device__ __forceinline__ uint32_t state_off(int k, int v) {
  return (v >> 6) * GDNT_HALF + k * 128 + ((((v & 63) >> 3) ^ (k & 7)) << 4) + (v & 7) * 2;
}
__device__ __forceinline__ void stmatrix_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(r0), "r"(r1), "r"(r2),
               "r"(r3)
               : "memory");
}
// 8 fp32 values as fp16 (hi, lo) pairs packed into two 16-byte chunks
__device__ __forceinline__ void split8(const float (&x)[8], uint4& hi, uint4& lo) {
  split_half2x(x[0], x[1], hi.x, lo.x);
  split_half2x(x[2], x[3], hi.y, lo.y);
  split_half2x(x[4], x[5], hi.z, lo.z);
  split_half2x(x[6], x[7], hi.w, lo.w);
}
__device__ __forceinline__ void st_shared_u16(uint8_t* base, uint32_t off, __half v) {
  *reinterpret_cast<__half*>(base + off) = v;
}

// maps.state = the fp16 state pool; maps.in0 = the conv history [(S+1)*3][3][2048] fp32, box [3][3][128];
// maps.in1 = the projection [rows][8320] fp32, box [128 columns][C rows] (one box per q / k / v slice).
template <int C>
__global__ void __launch_bounds__(GDNW_THREADS, 1)
gdn_wy_kernel(const __grid_constant__ GdntMaps maps, const GdnArgs args) {
  extern __shared__ __align__(1024) uint8_t gdnw_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gdnw_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* r_state = smem + GDNW_R_STATE;
  float* xq = reinterpret_cast<float*>(smem + GDNW_R_Q);
  float* xk = reinterpret_cast<float*>(smem + GDNW_R_K);
  float* xv = reinterpret_cast<float*>(smem + GDNW_R_V);
  float* hist = reinterpret_cast<float*>(smem + GDNW_R_HIST);
  float* amat = reinterpret_cast<float*>(smem + GDNW_R_A);
  float* vgam = reinterpret_cast<float*>(smem + GDNW_R_VEC);
  float* vGam = vgam + GDNW_MAXC;
  float* vbeta = vGam + GDNW_MAXC;
  float* vrk = vbeta + GDNW_MAXC;
  float* vrq = vrk + GDNW_MAXC;
  float* vg = vrq + GDNW_MAXC;
  float* vgc = vg + GDNW_MAXC;  // [0] = e^gam_C, [1] = gam_C
  float* part = reinterpret_cast<float*>(smem + GDNW_R_PART);
  float* onorm = reinterpret_cast<float*>(smem + GDNW_R_ONORM);
  GdnMeta* meta = reinterpret_cast<GdnMeta*>(smem + GDNW_R_META);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + GDNW_R_BAR);
  uint64_t* in_full = bar + 0;   // producer -> all: the item's q, k, v and conv history landed (or a padding item)
  uint64_t* st_full = bar + 1;   // producer -> compute: the state tile landed (or a padding item)
  uint64_t* ops3 = bar + 2;      // compute -> MMA: K^, Q^, S^T ready
  uint64_t* mma3 = bar + 3;      // MMA -> compute: KK, QK, P, R in TMEM
  uint64_t* ops6 = bar + 4;      // compute -> MMA: X, T ready
  uint64_t* mma6 = bar + 5;      // MMA -> compute: U^T in TMEM
  uint64_t* ops8 = bar + 6;      // compute -> MMA: U^T operand, Mqk ready
  uint64_t* mma8 = bar + 7;      // MMA -> compute: O^T, dS^T in TMEM
  uint64_t* x_free = bar + 8;    // -> producer: the input regions may be refilled
  uint64_t* st_free = bar + 9;   // -> producer: the state tile has been stored
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + GDNW_NBAR);

  const int h = blockIdx.x, p = blockIdx.y, P = gridDim.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lb = args.lb;  // == C
  const int n_items = args.nb > p ? (args.nb - p + P - 1) / P : 0;
  auto row_of = [&](int i) { return p + i * P; };
  const float scale = 0.08838834764831845f;  // 128^-1/2, correctly rounded

  if (tid == 0) {
    mbar_init(in_full, 1);
    mbar_init(st_full, 1);
    mbar_init(ops3, GDNW_COMPUTE);
    mbar_init(mma3, 1);
    mbar_init(ops6, GDNW_COMPUTE);
    mbar_init(mma6, 1);
    mbar_init(ops8, GDNW_COMPUTE);
    mbar_init(mma8, 1);
    mbar_init(x_free, 1);
    mbar_init(st_free, 1);
    fence_barrier_init();
    prefetch_tmap(&maps.state);
    prefetch_tmap(&maps.in0);
    prefetch_tmap(&maps.in1);
  }
  if (warp == GDNW_MMA_WARP) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == GDNW_PROD_WARP) {
    // ===================================== producer =====================================
    int issued = -1;  // the last item whose loads went out
    bool ok = true;
    for (int i = 0; i < n_items && ok; ++i) {
      const int n = row_of(i);
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
      if (i == 0) pdl_wait();  // the projection comes from the preceding GEMM
      if (i > 0 && lane == 0) ok = mbar_wait(x_free, (i - 1) & 1, args.err, ERR_TIMEOUT_TMA);
      ok = __shfl_sync(0xffffffffu, (int)ok, 0);
      if (!ok) break;
      if (lane == 0) {
        // metadata by item parity: a reader of item i - 1's (the MMA warp) may still be behind
        meta[i & 1].slot = slot;
        meta[i & 1].len = len;
        if (len > 0) {
          mbar_arrive_expect_tx(in_full, 3 * C * GDN_D * 4 + 9 * GDN_D * 4);
          tma_load_3d(hist, &maps.in0, h * GDN_D, 0, (int)slot * CONV_KEEP, in_full);
          tma_load_2d(xq, &maps.in1, 0 * KEY_DIM + h * GDN_D, n * lb, in_full);
          tma_load_2d(xk, &maps.in1, 1 * KEY_DIM + h * GDN_D, n * lb, in_full);
          tma_load_2d(xv, &maps.in1, 2 * KEY_DIM + h * GDN_D, n * lb, in_full);
        } else {
          mbar_arrive(in_full);
        }
        if (i > 0) ok = mbar_wait(st_free, (i - 1) & 1, args.err, ERR_TIMEOUT_TMA);
        if (ok) {
          if (len > 0) {
            mbar_arrive_expect_tx(st_full, GDNT_TILE);
            const int row = (int)((slot * GDN_H + h) * GDN_D);
            tma_load_2d(r_state, &maps.state, 0, row, st_full);
            tma_load_2d(r_state + GDNT_HALF, &maps.state, 64, row, st_full);
          } else {
            mbar_arrive(st_full);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, (int)ok, 0);
      issued = i;
    }
    // error paths: loads still in flight must land before the CTA exits (bounded)
    if (lane == 0 && issued >= 0) {
      mbar_wait(in_full, issued & 1, args.err, ERR_TIMEOUT_TMA);
      mbar_wait(st_full, issued & 1, args.err, ERR_TIMEOUT_TMA);
    }
  } else if (warp == GDNW_MMA_WARP) {
    // ===================================== MMA issuer =====================================
    if (lane == 0) {
      const uint32_t id_c = idesc_f16(128, C), id_128 = idesc_f16(128, 128);
      const uint32_t sm = smem_u32(smem);
      const uint32_t kq = sm + GDNW_R_K, qq = sm + GDNW_R_Q, st = sm + GDNW_R_ST;
      const uint32_t kq_hi = qq, kq_lo = kq;             // [K^; Q^]: K blocks of 128 rows, 16 KB apart
      const uint32_t t_hi = qq, t_lo = qq + C * 128, m_hi = qq + 2 * C * 128, m_lo = qq + 3 * C * 128;
      const uint32_t x_hi = st, x_lo = st + 128 * 128, u_hi = kq, u_lo = kq + 128 * 128;
      const uint32_t kt_hi = sm + GDNW_R_KT, kt_lo = kt_hi + 128 * 128;
      auto mma = [&](int col, uint32_t a, uint32_t b, int kstride_a, int kstride_b, int ksteps, uint32_t idesc,
                     bool first) {
        for (int s = 0; s < ksteps; ++s) {
          const uint32_t ao = a + (s >> 2) * kstride_a + (s & 3) * 32, bo = b + (s >> 2) * kstride_b + (s & 3) * 32;
          mma_bf16(tmem + (uint32_t)col, sw128_desc(ao), sw128_desc(bo), idesc, (first && s == 0) ? 0u : 1u);
        }
      };
      int seq = 0;
      bool ok = true;
      for (int i = 0; i < n_items && ok; ++i) {
        if (!mbar_wait(in_full, i & 1, args.err, ERR_TIMEOUT_TMA)) break;
        if (meta[i & 1].len == 0) continue;  // a padding row: the compute warps release its buffers
        const uint32_t ph = seq & 1;
        // step 3: KK = K^ K^T, QK = Q^ K^T (hi.hi + hi.lo + lo.hi), P = S^T K^T, R = S^T Q^T (S fp16 exact)
        if (!mbar_wait(ops3, ph, args.err, ERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        constexpr int KB = 128 * 128;
        mma(gdnw_col_kq(C), kq_hi, kq_hi, KB, KB, 8, id_c, true);     // [K^; Q^] K^T: KK | QK
        mma(gdnw_col_kq(C), kq_hi, kq_lo, KB, KB, 8, id_c, false);
        mma(gdnw_col_kq(C), kq_lo, kq_hi, KB, KB, 8, id_c, false);
        mma(gdnw_col_p(C), st, kq_hi, KB, KB, 8, id_128, true);       // S^T [K^; Q^]^T: P | R
        mma(gdnw_col_p(C), st, kq_lo, KB, KB, 8, id_128, false);
        mma_commit(mma3);
        // step 6: U^T = X T^T
        if (!mbar_wait(ops6, ph, args.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
        mma(gdnw_col_u(C), x_hi, t_hi, 0, 0, C / 16, id_c, true);
        mma(gdnw_col_u(C), x_hi, t_lo, 0, 0, C / 16, id_c, false);
        mma(gdnw_col_u(C), x_lo, t_hi, 0, 0, C / 16, id_c, false);
        mma_commit(mma6);
        // step 8: O^T = U^T Mqk^T, dS^T = U^T K~
        if (!mbar_wait(ops8, ph, args.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
        mma(gdnw_col_o(C), u_hi, m_hi, 0, 0, C / 16, id_c, true);
        mma(gdnw_col_o(C), u_hi, m_lo, 0, 0, C / 16, id_c, false);
        mma(gdnw_col_o(C), u_lo, m_hi, 0, 0, C / 16, id_c, false);
        mma(gdnw_col_ds(C), u_hi, kt_hi, 0, 0, C / 16, id_128, true);
        mma(gdnw_col_ds(C), u_hi, kt_lo, 0, 0, C / 16, id_128, false);
        mma(gdnw_col_ds(C), u_lo, kt_hi, 0, 0, C / 16, id_128, false);
        mma_commit(mma8);
        mma_commit(x_free);  // this item's operand regions have been read: the producer may refill them
        ++seq;
      }
    }
  } else {
    // ===================================== compute (warps 0-7) =====================================
    const int quad = warp & 3, half = warp >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    // head-stationary weights: conv taps of this thread's channels, gated-norm weight of its v lane
    const int c_part = tid >> 7, c_ch = tid & 127;  // first channel (q or k); v channel tid for tid < 128
    const float4 cw0 = (reinterpret_cast<const float4*>(args.conv_w) + h * GDN_D)[c_part * KEY_DIM + c_ch];
    const float4 cw1 = (reinterpret_cast<const float4*>(args.conv_w) + h * GDN_D)[2 * KEY_DIM + (tid & 127)];
    const float negA = -expf(args.A_log[h]), dtb = args.dt_bias[h];
    const int vrow = quad * 32 + lane;  // this thread's v (TMEM lane)
    const float gw = args.gnorm_w[vrow];
    int seq = 0;
    bool ok = true;
    if (n_items > 0) pdl_wait();  // z and the gates come from the preceding GEMM; outputs may still be read
    for (int i = 0; i < n_items && ok; ++i) {
      const int n = row_of(i);
      ok = named_sync_and_id<1, GDNW_COMPUTE>(mbar_wait(in_full, i & 1, args.err, ERR_TIMEOUT_TMA));
      if (!ok) break;
      const int len = meta[i & 1].len;
      const int64_t slot = meta[i & 1].slot;
      if (len == 0) {  // a padding row: zero outputs; nothing to load or store
        for (int e = tid; e < lb * GDN_D; e += GDNW_COMPUTE) {
          const size_t row = (size_t)n * lb + e / GDN_D;
          args.out_hi[row * KEY_DIM + h * GDN_D + (e & 127)] = __float2bfloat16_rn(0.f);
          args.out_lo[row * KEY_DIM + h * GDN_D + (e & 127)] = __float2bfloat16_rn(0.f);
        }
        ok = mbar_wait(st_full, i & 1, args.err, ERR_TIMEOUT_TMA);
        named_sync_id<1, GDNW_COMPUTE>();
        if (tid == 0) {
          mbar_arrive(x_free);
          mbar_arrive(st_free);
        }
        continue;
      }
      const uint32_t ph = seq & 1;
      // ---- A: causal conv + SiLU (q, k by all 256 threads, then v by 128), squared norms, gates ----
      {
        float xa = 0.f, xb = 0.f;
        if (tid < C && tid < len) {
          const size_t rt = (size_t)n * lb + tid;
          xa = args.proj[rt * GDN_IN + GDN_A_OFF + h];
          xb = args.proj[rt * GDN_IN + GDN_B_OFF + h];
        }
        float* xs = c_part == 0 ? xq : xk;
        float w[3] = {hist[(0 * 3 + c_part) * GDN_D + c_ch], hist[(1 * 3 + c_part) * GDN_D + c_ch],
                      hist[(2 * 3 + c_part) * GDN_D + c_ch]};
        float hh[3] = {0.f, 0.f, 0.f};
        for (int tb = 0; tb < C; tb += GDNC_SUB) {
          float sq[GDNC_SUB];
          conv_block16(xs + c_ch, GDN_D, cw0, w, tb, len, hh, sq);
          const float tot = reduce16(sq, lane);
          if (!(lane & 1)) part[((tb + reduce16_index(lane)) * 4 + (warp & 3)) * 2 + c_part] = tot;
        }
        float* gp = args.conv_pool + (size_t)slot * CONV_KEEP * CONV_DIM + c_part * KEY_DIM + h * GDN_D + c_ch;
        gp[0] = hh[0];
        gp[CONV_DIM] = hh[1];
        gp[2 * CONV_DIM] = hh[2];
        if (tid < 128) {
          float wv[3] = {hist[(0 * 3 + 2) * GDN_D + tid], hist[(1 * 3 + 2) * GDN_D + tid],
                         hist[(2 * 3 + 2) * GDN_D + tid]};
          float hv[3] = {0.f, 0.f, 0.f};
          for (int tb = 0; tb < C; tb += GDNC_SUB) {
            float sq[GDNC_SUB];
            conv_block16(xv + tid, GDN_D, cw1, wv, tb, len, hv, sq);
          }
          float* gv = args.conv_pool + (size_t)slot * CONV_KEEP * CONV_DIM + 2 * KEY_DIM + h * GDN_D + tid;
          gv[0] = hv[0];
          gv[CONV_DIM] = hv[1];
          gv[2 * CONV_DIM] = hv[2];
        }
        if (tid < C) {
          float g = 0.f, be = 0.f;
          if (tid < len) {
            const float x = xa + dtb;
            g = negA * (x > 20.f ? x : log1pf(expf(x)));
            be = sigmoidf_(xb);
          }
          vg[tid] = g;
          vbeta[tid] = be;
        }
      }
      named_sync_id<1, GDNW_COMPUTE>();
      // ---- factors: norms and cumulative decay (warp 0) ----
      if (warp == 0) {
        constexpr int PER = C / 32;  // tokens per lane
        float gl[PER], acc = 0.f;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
          gl[j] = vg[lane * PER + j];
          acc += gl[j];
        }
        float incl = acc;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += y;
        }
        float run = incl - acc;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
          const int t = lane * PER + j;
          run += gl[j];
          vgam[t] = run;
          vGam[t] = expf(run);
          float sq = 0.f, sk = 0.f;
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            sq += part[(t * 4 + w4) * 2 + 0];
            sk += part[(t * 4 + w4) * 2 + 1];
          }
          vrq[t] = scale * rsqrtf(sq + 1e-6f);
          vrk[t] = rsqrtf(sk + 1e-6f);
        }
        const float gC = __shfl_sync(0xffffffffu, run, 31);
        if (lane == 0) {
          vgc[0] = expf(gC);
          vgc[1] = gC;
        }
      }
      named_sync_id<1, GDNW_COMPUTE>();
      // ---- B: operands. K^, Q^ (hi, lo) over their fp32 sources in place; K~^T; the transposed state ----
      {
        constexpr int CH = C * 16 / GDNW_COMPUTE;   // 16-byte chunks of K^ / Q^ (8 channels of one token) per thread
        constexpr int KT = GDN_D * (C / 8) / GDNW_COMPUTE;  // 16-byte chunks of K~^T (8 tokens of one channel)
        // K~^T[k][s] = e^(gam_C - gam_s) rk_s k_s[k] into its own region (no barrier needed): thread takes channel
        // k = id & 127, tokens 8 (id >> 7) .. + 7, one 16-byte chunk of each half
        {
          uint8_t* ktop = smem + GDNW_R_KT;
          const float egc = vgam[C - 1];
#pragma unroll
          for (int r = 0; r < KT; ++r) {
            const int id = tid + GDNW_COMPUTE * r, k = id & 127, s0 = (id >> 7) * 8;
            float ktv[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int sx = s0 + e;
              ktv[e] = xk[sx * GDN_D + k] * (vrk[sx] * expf(egc - vgam[sx]));
            }
            const uint32_t off = kmaj_off(k, s0, 128 * 128);
            uint4 hi, lo;
            split8(ktv, hi, lo);
            *reinterpret_cast<uint4*>(ktop + off) = hi;
            *reinterpret_cast<uint4*>(ktop + 128 * 128 + off) = lo;
          }
        }
        float kv[CH][8], qv[CH][8];
        int ct[CH], cj[CH];
#pragma unroll
        for (int r = 0; r < CH; ++r) {
          const int cidx = tid + GDNW_COMPUTE * r;
          ct[r] = cidx >> 4;
          cj[r] = cidx & 15;
          const float4* ks = reinterpret_cast<const float4*>(xk + ct[r] * GDN_D + cj[r] * 8);
          const float4* qs = reinterpret_cast<const float4*>(xq + ct[r] * GDN_D + cj[r] * 8);
          const float4 k0 = ks[0], k1 = ks[1], q0 = qs[0], q1 = qs[1];
          const float rk = vrk[ct[r]], rq = vrq[ct[r]];
          kv[r][0] = k0.x * rk; kv[r][1] = k0.y * rk; kv[r][2] = k0.z * rk; kv[r][3] = k0.w * rk;
          kv[r][4] = k1.x * rk; kv[r][5] = k1.y * rk; kv[r][6] = k1.z * rk; kv[r][7] = k1.w * rk;
          qv[r][0] = q0.x * rq; qv[r][1] = q0.y * rq; qv[r][2] = q0.z * rq; qv[r][3] = q0.w * rq;
          qv[r][4] = q1.x * rq; qv[r][5] = q1.y * rq; qv[r][6] = q1.z * rq; qv[r][7] = q1.w * rq;
        }
        named_sync_id<1, GDNW_COMPUTE>();  // every fp32 q, k read: their regions become the operands
        // [K^; Q^]: hi in the q region, lo in the k region, each two K blocks of 128 rows (K^ row t, Q^ row 64 + t)
        uint8_t* kqh = smem + GDNW_R_Q;
        uint8_t* kql = smem + GDNW_R_K;
#pragma unroll
        for (int r = 0; r < CH; ++r) {
          const uint32_t ok_ = kmaj_off(ct[r], cj[r] * 8, 128 * 128), oq = kmaj_off(64 + ct[r], cj[r] * 8, 128 * 128);
          uint4 hi, lo;
          split8(kv[r], hi, lo);
          *reinterpret_cast<uint4*>(kqh + ok_) = hi;
          *reinterpret_cast<uint4*>(kql + ok_) = lo;
          split8(qv[r], hi, lo);
          *reinterpret_cast<uint4*>(kqh + oq) = hi;
          *reinterpret_cast<uint4*>(kql + oq) = lo;
        }
      }
      ok = mbar_wait(st_full, i & 1, args.err, ERR_TIMEOUT_TMA);
      {
        // S^T (rows v, K = k) from the [k][v] tile: per warp eight rounds of four 8 x 8 blocks (8 k x 32 v)
        const uint32_t src = smem_u32(r_state), dst = smem_u32(smem + GDNW_R_ST);
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int b = warp * 8 + it;
          const int k0 = (b >> 2) * 8, v0 = (b & 3) * 32;
          const int mi = lane >> 3, rr = lane & 7;
          uint32_t r0, r1, r2, r3;
          ldmatrix_x4_trans(src + state_off(k0 + rr, v0 + 8 * mi), r0, r1, r2, r3);
          stmatrix_x4(dst + kmaj_off(v0 + 8 * mi + rr, k0, 128 * 128), r0, r1, r2, r3);
        }
      }
      fence_proxy_async();
      tc_fence_before();
      if (!named_sync_and_id<1, GDNW_COMPUTE>(ok)) break;
      mbar_arrive(ops3);
      // ---- C: A and Mqk from KK / QK (lanes 0 .. C - 1), X from P (all lanes); then T = (I + A)^-1 ----
      ok = named_sync_and_id<1, GDNW_COMPUTE>(mbar_wait(mma3, ph, args.err, ERR_TIMEOUT_MMA));
      if (!ok) break;
      tc_fence_after();
      {
        const int cb = half * (C / 2);  // this warp's half of the C columns
        const bool kk_rows = quad < C / 32, qk_rows = quad >= 2 && quad - 2 < C / 32;
        if (kk_rows || qk_rows) {
          // token row t of KK (lanes 0 ..) or QK (lanes 64 ..): A[t][s] = beta_t e^(gam_t - gam_s) KK[t][s] (s < t),
          // Mqk[t][s] = e^(gam_t - gam_s) QK[t][s] (s <= t)
          const int t = (kk_rows ? quad : quad - 2) * 32 + lane;
          const float gt = vgam[t], bt = vbeta[t];
          uint8_t* mop = smem + GDNW_R_Q + 2 * C * 128;  // Mqk hi | lo (rows t, K = s), after T hi | lo
          for (int c0 = cb; c0 < cb + C / 2; c0 += 16) {
            float d16[16];
            tmem_ld16(lane_base + (uint32_t)(gdnw_col_kq(C) + c0), d16);
            if (kk_rows) {
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const int sx = c0 + e;
                amat[t * GDNW_A_STRIDE + sx] = sx < t ? bt * expf(gt - vgam[sx]) * d16[e] : 0.f;
              }
            } else {
#pragma unroll
              for (int e8 = 0; e8 < 16; e8 += 8) {
                float mv[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  const int sx = c0 + e8 + e;
                  mv[e] = sx <= t ? expf(gt - vgam[sx]) * d16[e8 + e] : 0.f;
                }
                uint4 hi, lo;
                split8(mv, hi, lo);
                const uint32_t off = kmaj_off(t, c0 + e8, 0);
                *reinterpret_cast<uint4*>(mop + off) = hi;
                *reinterpret_cast<uint4*>(mop + C * 128 + off) = lo;
              }
            }
          }
        }
        // X[v][t] = beta_t (v_t[v] - Gam_t P[v][t]) as hi|lo, rows v, K = t
        uint8_t* xop = smem + GDNW_R_ST;
        for (int c0 = cb; c0 < cb + C / 2; c0 += 16) {
          float pv[16];
          tmem_ld16(lane_base + (uint32_t)(gdnw_col_p(C) + c0), pv);
#pragma unroll
          for (int e8 = 0; e8 < 16; e8 += 8) {
            float xv8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int t = c0 + e8 + e;
              xv8[e] = vbeta[t] * (xv[t * GDN_D + vrow] - vGam[t] * pv[e8 + e]);
            }
            uint4 hi, lo;
            split8(xv8, hi, lo);
            const uint32_t off = kmaj_off(vrow, c0 + e8, 0);
            *reinterpret_cast<uint4*>(xop + off) = hi;
            *reinterpret_cast<uint4*>(xop + 128 * 128 + off) = lo;
          }
        }
      }
      named_sync_id<1, GDNW_COMPUTE>();  // A complete; v read for the last time (its region holds T below)
      {
        // Blocked inverse of the unit lower triangular I + A in 16 x 16 blocks (fp32, into tf = the v region):
        // diagonal blocks by forward substitution (thread = one column of one block), then block rows below the
        // diagonal level by level: W_ij = sum_{j <= m < i} A_im T_mj, T_ij = -T_ii W_ij.
        constexpr int NB = C / 16;
        float* tf = xv;                            // [64][65]
        float* wbuf = tf + GDNW_MAXC * GDNW_A_STRIDE;  // [NB - 1 blocks][16][17]
        if (tid < C) {
          const int b = tid >> 4, j = tid & 15, base = b * 16;
          float col[16];
#pragma unroll
          for (int tt = 0; tt < 16; ++tt) {
            float acc = tt == j ? 1.f : 0.f;
#pragma unroll
            for (int sx = 0; sx < tt; ++sx) acc = fmaf(-amat[(base + tt) * GDNW_A_STRIDE + base + sx], col[sx], acc);
            col[tt] = acc;
          }
#pragma unroll
          for (int tt = 0; tt < 16; ++tt) tf[(base + tt) * GDNW_A_STRIDE + base + j] = col[tt];
        } else {
          // zero the blocks above the diagonal (T is lower triangular)
          for (int e = tid - C; e < C * C; e += GDNW_COMPUTE - C) {
            const int tt = e / C, sx = e % C;
            if ((sx >> 4) > (tt >> 4)) tf[tt * GDNW_A_STRIDE + sx] = 0.f;
          }
        }
        named_sync_id<1, GDNW_COMPUTE>();
        for (int d = 1; d < NB; ++d) {
          const int nblk = NB - d;  // blocks (i, j = i - d)
          for (int e = tid; e < nblk * 256; e += GDNW_COMPUTE) {
            const int q = e >> 8, r = (e >> 4) & 15, c = e & 15, bi = q + d, bj = q;
            float acc = 0.f;
            for (int m = bj; m < bi; ++m) {
#pragma unroll
              for (int x = 0; x < 16; ++x)
                acc = fmaf(amat[(bi * 16 + r) * GDNW_A_STRIDE + m * 16 + x], tf[(m * 16 + x) * GDNW_A_STRIDE + bj * 16 + c],
                           acc);
            }
            wbuf[(q * 16 + r) * 17 + c] = acc;
          }
          named_sync_id<1, GDNW_COMPUTE>();
          for (int e = tid; e < nblk * 256; e += GDNW_COMPUTE) {
            const int q = e >> 8, r = (e >> 4) & 15, c = e & 15, bi = q + d, bj = q;
            float acc = 0.f;
#pragma unroll
            for (int x = 0; x < 16; ++x)
              acc = fmaf(tf[(bi * 16 + r) * GDNW_A_STRIDE + bi * 16 + x], wbuf[(q * 16 + x) * 17 + c], acc);
            tf[(bi * 16 + r) * GDNW_A_STRIDE + bj * 16 + c] = -acc;
          }
          named_sync_id<1, GDNW_COMPUTE>();
        }
        // T as hi|lo operand: rows t, K = s, 16-byte chunks of 8 s
        uint8_t* top = smem + GDNW_R_Q;
        for (int e = tid; e < C * (C / 8); e += GDNW_COMPUTE) {
          const int tt = e / (C / 8), s0 = (e % (C / 8)) * 8;
          float tv[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) tv[x] = tf[tt * GDNW_A_STRIDE + s0 + x];
          uint4 hi, lo;
          split8(tv, hi, lo);
          const uint32_t off = kmaj_off(tt, s0, 0);
          *reinterpret_cast<uint4*>(top + off) = hi;
          *reinterpret_cast<uint4*>(top + C * 128 + off) = lo;
        }
      }
      fence_proxy_async();
      tc_fence_before();
      named_sync_id<1, GDNW_COMPUTE>();
      mbar_arrive(ops6);
      // ---- E: U^T as hi|lo operand, rows v, K = t ----
      ok = named_sync_and_id<1, GDNW_COMPUTE>(mbar_wait(mma6, ph, args.err, ERR_TIMEOUT_MMA));
      if (!ok) break;
      tc_fence_after();
      {
        uint8_t* uop = smem + GDNW_R_K;
        const int cb = half * (C / 2);
        for (int c0 = cb; c0 < cb + C / 2; c0 += 16) {
          float uv[16];
          tmem_ld16(lane_base + (uint32_t)(gdnw_col_u(C) + c0), uv);
#pragma unroll
          for (int e8 = 0; e8 < 16; e8 += 8) {
            float u8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) u8[e] = uv[e8 + e];
            uint4 hi, lo;
            split8(u8, hi, lo);
            const uint32_t off = kmaj_off(vrow, c0 + e8, 0);
            *reinterpret_cast<uint4*>(uop + off) = hi;
            *reinterpret_cast<uint4*>(uop + 128 * 128 + off) = lo;
          }
        }
      }
      fence_proxy_async();
      tc_fence_before();
      named_sync_id<1, GDNW_COMPUTE>();
      mbar_arrive(ops8);
      // ---- F: outputs (gated RMSNorm of o_t over v) and the new state ----
      ok = named_sync_and_id<1, GDNW_COMPUTE>(mbar_wait(mma8, ph, args.err, ERR_TIMEOUT_MMA));
      if (!ok) break;
      tc_fence_after();
      {
        // o_t = Gam_t R[v][t] + O^T[v][t] for this warp's half of the tokens, 16 at a time: first the per-token sums
        // of squares over v (TMEM lanes), then after the barrier the outputs from a second read of O^T and R
        const int cb = half * (C / 2);
#pragma unroll
        for (int c0 = 0; c0 < C / 2; c0 += 16) {
          float ov[16], rv[16], sq[16];
          tmem_ld16(lane_base + (uint32_t)(gdnw_col_o(C) + cb + c0), ov);
          tmem_ld16(lane_base + (uint32_t)(gdnw_col_r(C) + cb + c0), rv);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float o = fmaf(vGam[cb + c0 + e], rv[e], ov[e]);
            sq[e] = o * o;
          }
          const float tot = reduce16(sq, lane);
          if (!(lane & 1)) onorm[quad * GDNW_MAXC + cb + c0 + reduce16_index(lane)] = tot;
        }
        named_sync_id<1, GDNW_COMPUTE>();
#pragma unroll
        for (int c0 = 0; c0 < C / 2; c0 += 16) {
          float ov[16], rv[16], z[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int t = cb + c0 + e;
            z[e] = t < len ? args.proj[((size_t)n * lb + t) * GDN_IN + GDN_Z_OFF + h * GDN_D + vrow] : 0.f;
          }
          tmem_ld16(lane_base + (uint32_t)(gdnw_col_o(C) + cb + c0), ov);
          tmem_ld16(lane_base + (uint32_t)(gdnw_col_r(C) + cb + c0), rv);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int t = cb + c0 + e;
            const size_t row = (size_t)n * lb + t;
            __nv_bfloat16 hv = __float2bfloat16_rn(0.f), lv = hv;
            if (t < len) {
              const float o = fmaf(vGam[t], rv[e], ov[e]);
              const float ss = onorm[t] + onorm[GDNW_MAXC + t] + onorm[2 * GDNW_MAXC + t] + onorm[3 * GDNW_MAXC + t];
              const float r = 1.0f / sqrtf(ss * (1.0f / GDN_D) + args.eps);
              split_bf16(gw * (o * r) * silu(z[e]), hv, lv);
            }
            args.out_hi[row * KEY_DIM + h * GDN_D + vrow] = hv;
            args.out_lo[row * KEY_DIM + h * GDN_D + vrow] = lv;
          }
        }
        // S <- Gam_C S + dS: this thread's v, k in [64 half, 64 half + 64)
        const float egC = vgc[0];
        for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 32) {
          float dv[32];
          tmem_ld32(lane_base + (uint32_t)(gdnw_col_ds(C) + c0), dv);
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const uint32_t off = state_off(c0 + e, vrow);
            __half* sp = reinterpret_cast<__half*>(r_state + off);
            *sp = __float2half_rn(fmaf(egC, __half2float(*sp), dv[e]));
          }
        }
      }
      fence_proxy_async();
      tc_fence_before();
      named_sync_id<1, GDNW_COMPUTE>();
      if (tid == 0) {
        const int row = (int)((slot * GDN_H + h) * GDN_D);
        tma_store_2d(&maps.state, r_state, 0, row);
        tma_store_2d(&maps.state, r_state + GDNT_HALF, 64, row);
        bulk_commit();
        bulk_wait_read_all();
        mbar_arrive(st_free);
      }
      ++seq;
    }
    if (tid == 0) bulk_wait_all();
  }

  // ---- teardown ----
  tc_fence_before();
  __syncthreads();
  if (warp == GDNW_MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace hsg
