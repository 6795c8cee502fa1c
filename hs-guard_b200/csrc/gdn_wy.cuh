// Chunked gated delta rule on the 5th-generation tensor cores (tcgen05, accumulators in TMEM) for 32- and 64-token
// ticks with fp16 recurrent state (the engine's FUSED inputs): the whole tick is one chunk of C = lb tokens.
//
// Per (row, head) item, with the state S (dk x dv, fp16 at the tick's start), k^_t = rk_t k_t, q^_t = rq_t q_t,
// cumulative log decay gam_t = sum_{s<=t} g_s, Gam_t = e^gam_t, beta_t (the chunked WY form of the reference's
// complete-message path, FLA chunk.py; the same algebra as gdn_chunk.cuh with one chunk instead of four):
//   KK = K^ K^T, QK = Q^ K^T, P = S^T K^T, R' = Q^ S                          (tensor cores, fp16 hi/lo operands)
//   A[t][s] = beta_t e^(gam_t - gam_s) KK[t][s] (s < t),  T = (I + A)^-1    (CUDA cores, fp32 blocked substitution)
//   Mqk[t][s] = e^(gam_t - gam_s) QK[t][s] (s <= t)
//   X[v][t] = beta_t (v_t[v] - Gam_t P[v][t])
//   U^T = X T^T                                                               (tensor cores)
//   O = Mqk U,  dS = K~^T U  with K~[s][k] = e^(gam_C - gam_s) k^_s[k]       (tensor cores)
//   o_t = Gam_t R'[t] + O[t],   S <- Gam_C S + dS
// Every exponent is <= 0. Padded tokens (t >= len) carry q = k = v = 0, g = 0, beta = 0: they change nothing.
//
// Every tensor-core operand is K-major with 128-byte swizzle in 64-element K blocks (rows of 128 bytes, 8-row atoms),
// the layout the GEMM kernels use: K^ and Q^ stacked in one operand (rows 0 .. C - 1 and 64 .. 64 + C - 1 of each
// 128-row K block), the state transposed to S^T (rows v, built from the TMA-loaded [k][v] tile with ldmatrix.trans /
// stmatrix), T and Mqk (rows t, K = s), X and U^T (rows v, K = t), K~^T (rows k, K = s). All MMAs are M = 128. The
// products whose results leave the kernel are laid out for their consumers: O and R' with TMEM lanes = tokens (rows
// 64 + t of the stacked operand, and of an Mqk operand addressed 64 rows early) so the gated RMSNorm of a token is a
// per-thread sum and its output row is written with 16-byte stores; dS with lanes = k so the new state is read,
// updated and written back in 16-byte chunks of the swizzled tile.
// TMEM (fp32 columns): KK|QK [0, C) | P [64, 64 + C) | U^T [128, 128 + C) | dS [0, 128) after those are read |
// O [256, 384) | R' [384, 512).
//
// Warps: 0-15 compute (warp w reads TMEM lane quadrant w % 4 and takes column group w / 4), 16 the TMA producer
// (inputs, state loads and the new state's store), 17 the MMA issuer (owns TMEM). Shared memory regions are reused as
// the item proceeds: the fp32 q and k inputs become the [K^; Q^] operand (hi, lo) in place, then after the first MMAs
// hold T / Mqk (q region) and U^T (k region); the S^T copy becomes X. The next item's inputs are loaded as soon as the
// last MMAs of this one have completed; its state once this item's state has been stored. Every wait is bounded and
// reports through `err`.
#pragma once
#include "gdn_chunk.cuh"

namespace hsg {

constexpr int GDNW_CWARPS = 16;
constexpr int GDNW_COMPUTE = GDNW_CWARPS * 32;
constexpr int GDNW_PROD_WARP = GDNW_CWARPS;
constexpr int GDNW_MMA_WARP = GDNW_CWARPS + 1;
constexpr int GDNW_THREADS = GDNW_COMPUTE + 64;
constexpr int GDNW_MAXC = 64;
// region byte offsets (sized for C = 64; a 32-token tick uses the same layout)
constexpr int GDNW_R_STATE = 0;                               // fp16 state tile, two [128 k][64 v] SW128 halves
constexpr int GDNW_R_Q = GDNW_R_STATE + GDNT_TILE;            // q fp32 [C][128] -> [K^; Q^] hi -> T hi|lo, Mqk hi|lo
constexpr int GDNW_R_K = GDNW_R_Q + GDNW_MAXC * GDN_D * 4;    // k fp32 [C][128] -> [K^; Q^] lo -> U^T hi|lo
constexpr int GDNW_R_V = GDNW_R_K + GDNW_MAXC * GDN_D * 4;    // v fp32 [C][128] -> the fp32 inverse T
constexpr int GDNW_R_ST = GDNW_R_V + GDNW_MAXC * GDN_D * 4;   // S^T fp16 (two K blocks of [128 v][64 k]) -> X hi|lo
constexpr int GDNW_R_KT = GDNW_R_ST + GDN_D * GDN_D * 2;      // K~^T hi | lo, [128 k][64 s] each
constexpr int GDNW_R_HIST = GDNW_R_KT + 2 * GDN_D * 128;      // conv history [3][3][128] fp32
constexpr int GDNW_A_STRIDE = GDNW_MAXC + 1;
constexpr int GDNW_T_STRIDE = GDNW_MAXC + 4;  // rows of the fp32 inverse T (16-byte aligned)
constexpr int GDNW_R_A = GDNW_R_HIST + 9 * GDN_D * 4;         // A [64][65] fp32 for the triangular solve
// gam, Gam, beta, rk, rq, g, (Gam_C, gam_C), K~ scale [64] f32 each, the gated-norm weight [128]
constexpr int GDNW_R_VEC = GDNW_R_A + GDNW_MAXC * GDNW_A_STRIDE * 4;
constexpr int GDNW_R_PART = GDNW_R_VEC + (8 * GDNW_MAXC + GDN_D) * 4;  // per-token q.q, k.k partials [64][4][2] f32
constexpr int GDNW_R_ONORM = GDNW_R_PART;                     // later: output sums of squares [8 column groups][64]
constexpr int GDNW_R_META = GDNW_R_PART + GDNW_MAXC * 8 * 4;  // item metadata (slot, len) x 2, by item parity
constexpr int GDNW_R_CW = GDNW_R_META + 32;                   // this head's conv taps [3 parts][128] float4
constexpr int GDNW_R_BAR = GDNW_R_CW + 3 * GDN_D * 16;        // mbarriers
constexpr int GDNW_NBAR = 14;
constexpr int GDNW_SMEM = GDNW_R_BAR + GDNW_NBAR * 8 + 16 + 1024;
// TMEM column offsets
constexpr int GDNW_COL_KQ = 0;    // KK in lanes 0 .. C - 1, QK in lanes 64 .. 64 + C - 1 (the stacked operand x K^)
constexpr int GDNW_COL_P = 64;    // P = S^T K^T, lanes v
constexpr int GDNW_COL_U = 128;   // U^T, lanes v
constexpr int GDNW_COL_R2 = 192;  // R' = Q^ S for v < 64 in lanes t (the stacked operand read from row 64)
constexpr int GDNW_COL_DS = 0;    // dS, lanes k, 128 columns v (written after KK, QK, P, U^T have been read)
constexpr int GDNW_COL_O = 256;   // O for v < 64 in lanes t, then O for v >= 64 in lanes 64 + t (64 columns each)
constexpr int GDNW_COL_R = 384;   // [K^; Q^] S for v >= 64: R' = Q^ S in lanes 64 + t, 64 columns
// Mqk hi | lo (rows t, K = s) inside the q region after T hi | lo. The O product for v >= 64 addresses it 64 rows
// early so that its rows land in TMEM lanes 64 + t, beside R'.
constexpr int GDNW_MQK = 16384;

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
// Two 32-lane x 16-column TMEM loads with one wait (tmem_ld16 waits after each).
__device__ __forceinline__ void tmem_ld16x2(uint32_t ta, float (&a)[16], uint32_t tb, float (&b)[16]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(ta), "r"(tb));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    a[i] = __uint_as_float(r[i]);
    b[i] = __uint_as_float(r[16 + i]);
  }
}
// 8 fp32 values as bf16 (hi, lo) pairs packed into two 16-byte chunks
__device__ __forceinline__ void split8_bf16(const float (&x)[8], uint4& hi, uint4& lo) {
  uint32_t* h = reinterpret_cast<uint32_t*>(&hi);
  uint32_t* l = reinterpret_cast<uint32_t*>(&lo);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 a, b;
    split_bf16x2(x[2 * j], x[2 * j + 1], a, b);
    h[j] = *reinterpret_cast<uint32_t*>(&a);
    l[j] = *reinterpret_cast<uint32_t*>(&b);
  }
}

// Causal conv (4 taps) + SiLU of 16 consecutive tokens of one channel, in place (rows GDN_D floats apart); w = the
// three raw inputs before the first token; sq = the squared outputs. FULL: all 16 tokens are valid (no masking).
template <bool FULL>
__device__ __forceinline__ void wy_conv16(float* xc, float4 c, const float (&w)[3], int tb, int len, float (&sq)[16]) {
  float in[19];
  in[0] = w[0];
  in[1] = w[1];
  in[2] = w[2];
#pragma unroll
  for (int u = 0; u < 16; ++u) in[3 + u] = xc[(tb + u) * GDN_D];
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    const float y = silu_fast(fmaf(c.w, in[u + 3], fmaf(c.z, in[u + 2], fmaf(c.y, in[u + 1], c.x * in[u]))));
    const float o = FULL || tb + u < len ? y : 0.f;
    xc[(tb + u) * GDN_D] = o;
    sq[u] = o * o;
  }
}

// maps.state = the fp16 state pool; maps.in0 = the conv history [(S+1)*3][3][2048] fp32, box [3][3][128];
// maps.in1 = the projection [rows][8320] fp32, box [128 columns][C rows] (one box per q / k / v slice).
// PRE: the projection's q | k | v columns already hold conv + SiLU (the input projection's GEMM_CONV epilogue, which
// also keeps the conv history): this kernel then reads no conv history and forms only the norms in phase A.
template <int C, bool PRE>
__global__ void __launch_bounds__(GDNW_THREADS, 1)
gdn_wy_kernel(const __grid_constant__ GdntMaps maps, const GdnArgs args) {
  static_assert(C == 32 || C == 64, "32- or 64-token chunks");
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
  float* vgc = vg + GDNW_MAXC;    // [0] = e^gam_C, [1] = gam_C
  float* vkt = vgc + GDNW_MAXC;   // K~ row scale e^(gam_C - gam_s) rk_s
  float* gwv = vkt + GDNW_MAXC;   // gated-norm weight [128]
  float* part = reinterpret_cast<float*>(smem + GDNW_R_PART);
  float* onorm = reinterpret_cast<float*>(smem + GDNW_R_ONORM);
  float4* cws = reinterpret_cast<float4*>(smem + GDNW_R_CW);
  GdnMeta* meta = reinterpret_cast<GdnMeta*>(smem + GDNW_R_META);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + GDNW_R_BAR);
  uint64_t* in_full = bar + 0;   // producer -> all: the item's q, k, v and conv history landed (or a padding item)
  uint64_t* st_full = bar + 1;   // producer -> compute: the state tile landed (or a padding item)
  uint64_t* ops3 = bar + 2;      // compute -> MMA: [K^; Q^] ready
  uint64_t* mma3 = bar + 3;      // MMA -> compute: KK, QK in TMEM
  uint64_t* ops6 = bar + 4;      // compute -> MMA: X, T ready
  uint64_t* mma6 = bar + 5;      // MMA -> compute: U^T in TMEM
  uint64_t* ops8 = bar + 6;      // compute -> MMA: U^T operand, Mqk ready
  uint64_t* mma8 = bar + 7;      // MMA -> compute: O, dS in TMEM
  uint64_t* x_free = bar + 8;    // -> producer: the input regions may be refilled
  uint64_t* st_done = bar + 9;   // compute -> producer: the new state is in the tile (or a padding item)
  uint64_t* ops3s = bar + 10;    // compute -> MMA: S^T ready
  uint64_t* mma3s = bar + 11;    // MMA -> compute: P, R' in TMEM
  uint64_t* mma8s = bar + 12;    // MMA -> compute: dS in TMEM (mma8: O)
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
    mbar_init(st_done, 1);
    mbar_init(ops3s, GDNW_COMPUTE);
    mbar_init(mma3s, 1);
    mbar_init(mma8s, 1);
    fence_barrier_init();
    prefetch_tmap(&maps.state);
    prefetch_tmap(&maps.in0);
    prefetch_tmap(&maps.in1);
  }
  if (tid < GDN_D) gwv[tid] = args.gnorm_w[tid];
  for (int e = tid; e < 3 * GDN_D; e += GDNW_THREADS)
    cws[e] = reinterpret_cast<const float4*>(args.conv_w)[(e >> 7) * KEY_DIM + h * GDN_D + (e & 127)];
  if (warp == GDNW_MMA_WARP) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == GDNW_PROD_WARP) {
    // ===================================== producer =====================================
    int in_issued = -1, st_issued = -1;  // the last item whose input / state loads went out
    int prev_len = 0;
    int64_t prev_slot = 0;
    bool ok = true;
    auto store_state = [&](int64_t slot) {  // lane 0: the new state of `slot` from the tile to the pool
      const int row = (int)((slot * GDN_H + h) * GDN_D);
      tma_store_2d(&maps.state, r_state, 0, row);
      tma_store_2d(&maps.state, r_state + GDNT_HALF, 64, row);
      bulk_commit();
    };
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
      if (lane == 0) {
        if (i > 0) ok = mbar_wait(x_free, (i - 1) & 1, args.err, ERR_TIMEOUT_TMA);
        if (ok) {
          // metadata by item parity: a reader of item i - 1's (the MMA warp) may still be behind
          meta[i & 1].slot = slot;
          meta[i & 1].len = len;
          if (len > 0) {
            mbar_arrive_expect_tx(in_full, 3 * C * GDN_D * 4 + (PRE ? 0 : 9 * GDN_D * 4));
            if (!PRE) tma_load_3d(hist, &maps.in0, h * GDN_D, 0, (int)slot * CONV_KEEP, in_full);
            tma_load_2d(xq, &maps.in1, 0 * KEY_DIM + h * GDN_D, n * lb, in_full);
            tma_load_2d(xk, &maps.in1, 1 * KEY_DIM + h * GDN_D, n * lb, in_full);
            tma_load_2d(xv, &maps.in1, 2 * KEY_DIM + h * GDN_D, n * lb, in_full);
            tma_prefetch_l2_2d(&maps.in1, GDN_Z_OFF + h * GDN_D, n * lb);  // z, read by the output rows at the end
          } else {
            mbar_arrive(in_full);
          }
          in_issued = i;
          if (i > 0) {
            // the previous item's new state out of the tile before this item's comes in
            ok = mbar_wait(st_done, (i - 1) & 1, args.err, ERR_TIMEOUT_TMA);
            if (ok && prev_len > 0) {
              store_state(prev_slot);
              bulk_wait_read_all();
            }
          }
          if (ok) {
            if (len > 0) {
              mbar_arrive_expect_tx(st_full, GDNT_TILE);
              const int row = (int)((slot * GDN_H + h) * GDN_D);
              tma_load_2d(r_state, &maps.state, 0, row, st_full);
              tma_load_2d(r_state + GDNT_HALF, &maps.state, 64, row, st_full);
            } else {
              mbar_arrive(st_full);
            }
            st_issued = i;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, (int)ok, 0);
      prev_len = len;
      prev_slot = slot;
    }
    if (lane == 0) {
      if (ok && n_items > 0 && mbar_wait(st_done, (n_items - 1) & 1, args.err, ERR_TIMEOUT_TMA) && prev_len > 0)
        store_state(prev_slot);
      // error paths: loads still in flight must land before the CTA exits (bounded)
      if (!ok) {
        if (in_issued >= 0) mbar_wait(in_full, in_issued & 1, args.err, ERR_TIMEOUT_TMA);
        if (st_issued >= 0) mbar_wait(st_full, st_issued & 1, args.err, ERR_TIMEOUT_TMA);
      }
      bulk_wait_all();
    }
  } else if (warp == GDNW_MMA_WARP) {
    // ===================================== MMA issuer =====================================
    if (lane == 0) {
      const uint32_t id_c = idesc_f16(128, C), id_128 = idesc_f16(128, 128), id_c64 = idesc_f16(128, 64);
      const uint32_t sm = smem_u32(smem);
      const uint32_t kq_hi = sm + GDNW_R_Q, kq_lo = sm + GDNW_R_K, st = sm + GDNW_R_ST;  // K blocks 16 KB apart
      const uint32_t t_hi = sm + GDNW_R_Q, t_lo = t_hi + C * 128;
      const uint32_t m_hi = sm + GDNW_R_Q + GDNW_MQK, m_lo = m_hi + 64 * 128;
      const uint32_t x_hi = st, x_lo = st + 128 * 128, u_hi = kq_lo, u_lo = kq_lo + 128 * 128;
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
        // step 3: KK | QK = [K^; Q^] K^T (hi.hi + hi.lo + lo.hi) as soon as the operand is ready, then, once the
        // transposed state is, P = S^T K^T and [K^; Q^] S (S fp16 exact) while the compute warps form A and Mqk
        if (!mbar_wait(ops3, ph, args.err, ERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        constexpr int KB = 128 * 128;
        mma(GDNW_COL_KQ, kq_hi, kq_hi, KB, KB, 8, id_c, true);
        mma(GDNW_COL_KQ, kq_hi, kq_lo, KB, KB, 8, id_c, false);
        mma(GDNW_COL_KQ, kq_lo, kq_hi, KB, KB, 8, id_c, false);
        mma_commit(mma3);
        if (!mbar_wait(ops3s, ph, args.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
        mma(GDNW_COL_P, st, kq_hi, KB, KB, 8, id_c, true);
        mma(GDNW_COL_P, st, kq_lo, KB, KB, 8, id_c, false);
        mma(GDNW_COL_R, kq_hi, st + 64 * 128, KB, KB, 8, id_c64, true);  // B = S^T rows v >= 64
        mma(GDNW_COL_R, kq_lo, st + 64 * 128, KB, KB, 8, id_c64, false);
        // Q^ S again for v < 64 with the A rows read from row 64 (Q^ into lanes 0 .. 63; lanes 64 .. see the rows
        // after it, unused): the outputs of v < 64 are formed by the warps of lane quadrants 0 and 1
        mma(GDNW_COL_R2, kq_hi + 64 * 128, st, KB, KB, 8, id_c64, true);
        mma(GDNW_COL_R2, kq_lo + 64 * 128, st, KB, KB, 8, id_c64, false);
        mma_commit(mma3s);
        // step 6: U^T = X T^T
        if (!mbar_wait(ops6, ph, args.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
        mma(GDNW_COL_U, x_hi, t_hi, 0, 0, C / 16, id_c, true);
        mma(GDNW_COL_U, x_hi, t_lo, 0, 0, C / 16, id_c, false);
        mma(GDNW_COL_U, x_lo, t_hi, 0, 0, C / 16, id_c, false);
        mma_commit(mma6);
        // step 8: O = Mqk U (lanes 64 + t), dS = K~^T U (lanes k); B = the U^T operand (rows v, K = s)
        if (!mbar_wait(ops8, ph, args.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
        // O for v < 64 (Mqk from row 0: lanes t) and for v >= 64 (Mqk addressed 64 rows early: lanes 64 + t)
        mma(GDNW_COL_O, m_hi, u_hi, 0, 0, C / 16, id_c64, true);
        mma(GDNW_COL_O, m_hi, u_lo, 0, 0, C / 16, id_c64, false);
        mma(GDNW_COL_O, m_lo, u_hi, 0, 0, C / 16, id_c64, false);
        mma(GDNW_COL_O + 64, m_hi - 64 * 128, u_hi + 64 * 128, 0, 0, C / 16, id_c64, true);
        mma(GDNW_COL_O + 64, m_hi - 64 * 128, u_lo + 64 * 128, 0, 0, C / 16, id_c64, false);
        mma(GDNW_COL_O + 64, m_lo - 64 * 128, u_hi + 64 * 128, 0, 0, C / 16, id_c64, false);
        mma_commit(mma8);  // the outputs can start while dS is computed
        mma(GDNW_COL_DS, kt_hi, u_hi, 0, 0, C / 16, id_128, true);
        mma(GDNW_COL_DS, kt_hi, u_lo, 0, 0, C / 16, id_128, false);
        mma(GDNW_COL_DS, kt_lo, u_hi, 0, 0, C / 16, id_128, false);
        mma_commit(mma8s);
        mma_commit(x_free);  // this item's operand regions have been read: the producer may refill them
        ++seq;
      }
    }
  } else {
    // ===================================== compute (warps 0-15) =====================================
    const int quad = warp & 3, cg = warp >> 2;  // TMEM lane quadrant; column group
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    // conv: this thread's channel cc of each of q, k, v over the tokens [16 quad, 16 quad + 16)
    const int cc = cg * 32 + lane, tq = quad;
    const float negA = -expf(args.A_log[h]), dtb = args.dt_bias[h];
    const int vrow = quad * 32 + lane;  // this thread's TMEM lane: v (P, U^T), k (dS), 64 + t (O, R')
    // outputs: token ot = 32 (quad & 1) + lane in lanes ot (quadrants 0, 1: v < 64) and 64 + ot (quadrants 2, 3:
    // v >= 64); warp (quad, cg) forms the 16 columns ov0 .. ov0 + 15. NOUT threads take part.
    constexpr int NOUT = 8 * C;
    const bool out_warp = (quad & 1) < C / 32;
    const int ot = (quad & 1) * 32 + lane, ov0 = (quad >> 1) * 64 + cg * 16;
    const int col_o = GDNW_COL_O + ov0;                                      // this warp's O columns
    const int col_rr = quad < 2 ? GDNW_COL_R2 + cg * 16 : GDNW_COL_R + cg * 16;  // and R' columns
    int seq = 0;
    bool ok = true;
    if (n_items > 0) pdl_wait();  // z and the gates come from the preceding GEMM; outputs may still be read
    for (int i = 0; i < n_items && ok; ++i) {
      const int n = row_of(i);
      float xa = 0.f, xb = 0.f;  // this thread's token's gate inputs (tid < C), read before the inputs land
      if (tid < C) {
        const size_t rt = (size_t)n * lb + tid;
        xa = args.proj[rt * GDN_IN + GDN_A_OFF + h];
        xb = args.proj[rt * GDN_IN + GDN_B_OFF + h];
      }
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
          mbar_arrive(st_done);
        }
        continue;
      }
      const uint32_t ph = seq & 1;
      // ---- A: causal conv + SiLU in place, squared norms of q, k, gates ----
      if (PRE && 16 * tq < C) {
        // the squared norms of q and k over this warp's 32 channels for its 16 tokens (the inputs are conv'd and
        // zero past len already)
#pragma unroll
        for (int c3 = 0; c3 < 2; ++c3) {
          const float* xc = (c3 == 0 ? xq : xk) + cc;
          float sq[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            const float x = xc[(16 * tq + u) * GDN_D];
            sq[u] = x * x;
          }
          const float tot = reduce16(sq, lane);
          if (!(lane & 1)) part[((16 * tq + reduce16_index(lane)) * 4 + cg) * 2 + c3] = tot;
        }
      } else if (!PRE && 16 * tq < C) {
        // the q, k, v regions are consecutive: channel part c3's inputs start at xq + c3 * (64 x 128)
        constexpr int XPART = GDNW_MAXC * GDN_D;
        auto raw = [&](int c3, int t) {  // raw input t of this channel (t < 0: the conv history)
          return t >= 0 ? xq[c3 * XPART + t * GDN_D + cc] : hist[((t + 3) * 3 + c3) * GDN_D + cc];
        };
        float w3[3][3];
#pragma unroll
        for (int c3 = 0; c3 < 3; ++c3)
#pragma unroll
          for (int j = 0; j < 3; ++j) w3[c3][j] = raw(c3, 16 * tq - 3 + j);
        if (((len - 1) >> 4) == tq) {
          // this quarter holds the last token: the new history (the last three raw inputs) goes to the pool
#pragma unroll
          for (int c3 = 0; c3 < 3; ++c3) {
            float* gp = args.conv_pool + (size_t)slot * CONV_KEEP * CONV_DIM + c3 * KEY_DIM + h * GDN_D + cc;
#pragma unroll
            for (int j = 0; j < 3; ++j) gp[j * CONV_DIM] = raw(c3, len - 3 + j);
          }
        }
        named_sync_id<2, 4 * C * 2>();  // every raw value read before the in-place conv overwrites it
        const bool full = len >= 16 * tq + 16;
#pragma unroll 1
        for (int c3 = 0; c3 < 3; ++c3) {
          // selects, not indexing: a register array indexed by the (not unrolled) loop would go to local memory
          const float4 cw = cws[c3 * GDN_D + cc];
          float wv[3], sq[16];
#pragma unroll
          for (int j = 0; j < 3; ++j) wv[j] = c3 == 0 ? w3[0][j] : (c3 == 1 ? w3[1][j] : w3[2][j]);
          if (full)
            wy_conv16<true>(xq + c3 * XPART + cc, cw, wv, 16 * tq, len, sq);
          else
            wy_conv16<false>(xq + c3 * XPART + cc, cw, wv, 16 * tq, len, sq);
          if (c3 < 2) {
            const float tot = reduce16(sq, lane);
            if (!(lane & 1)) part[((16 * tq + reduce16_index(lane)) * 4 + cg) * 2 + c3] = tot;
          }
        }
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
      named_sync_id<1, GDNW_COMPUTE>();
      // ---- factors: norms, cumulative decay, K~ scale (warp 0) ----
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
        float run = incl - acc, gm[PER], rkv[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) {
          const int t = lane * PER + j;
          run += gl[j];
          gm[j] = run;
          vgam[t] = run;
          vGam[t] = expf(run);
          float sq = 0.f, sk = 0.f;
#pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            sq += part[(t * 4 + w4) * 2 + 0];
            sk += part[(t * 4 + w4) * 2 + 1];
          }
          vrq[t] = scale * rsqrtf(sq + 1e-6f);
          rkv[j] = rsqrtf(sk + 1e-6f);
          vrk[t] = rkv[j];
        }
        const float gC = __shfl_sync(0xffffffffu, run, 31);
#pragma unroll
        for (int j = 0; j < PER; ++j) vkt[lane * PER + j] = rkv[j] * expf(gC - gm[j]);
        if (lane == 0) {
          vgc[0] = expf(gC);
          vgc[1] = gC;
        }
      }
      named_sync_id<1, GDNW_COMPUTE>();
      // ---- B: operands. [K^; Q^] (hi, lo) over their fp32 sources in place; K~^T; the transposed state ----
      {
        constexpr int CH = C * 16 / GDNW_COMPUTE;           // 16-byte chunks of K^ / Q^ (8 channels of a token)
        constexpr int KT = GDN_D * (C / 8) / GDNW_COMPUTE;  // 16-byte chunks of K~^T (8 tokens of a channel)
        // K~^T[k][s] = e^(gam_C - gam_s) rk_s k_s[k] into its own region: channel k = id & 127, tokens 8 (id >> 7) ..
        {
          uint8_t* ktop = smem + GDNW_R_KT;
#pragma unroll
          for (int r = 0; r < KT; ++r) {
            const int id = tid + GDNW_COMPUTE * r, k = id & 127, s0 = (id >> 7) * 8;
            float ktv[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) ktv[e] = xk[(s0 + e) * GDN_D + k] * vkt[s0 + e];
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
        named_sync_id<1, GDNW_COMPUTE>();  // every fp32 q, k read: their regions become the operand
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
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(ops3);  // KK | QK can start while the state is transposed
      ok = mbar_wait(st_full, i & 1, args.err, ERR_TIMEOUT_TMA);
      {
        // S^T (rows v, K = k) from the [k][v] tile: per warp four rounds of four 8 x 8 blocks (8 k x 32 v)
        const uint32_t src = smem_u32(r_state), dst = smem_u32(smem + GDNW_R_ST);
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          const int b = warp * 4 + it;
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
      mbar_arrive(ops3s);
      // ---- C: A (KK lanes), Mqk (QK lanes), then X from P (all lanes); column group cg takes 16 of the C columns ----
      ok = named_sync_and_id<1, GDNW_COMPUTE>(mbar_wait(mma3, ph, args.err, ERR_TIMEOUT_MMA));
      if (!ok) break;
      tc_fence_after();
      {
        // Warp (quad, cg) takes the 16 columns [16 cg, 16 cg + 16) of the C (none when 16 cg >= C). Token row t of KK
        // (lanes 0 ..): A[t][s] = beta_t e^(gam_t - gam_s) KK[t][s] (s < t) to amat while P and R' are computed; of
        // QK (lanes 64 ..): Mqk[t][s] = e^(gam_t - gam_s) QK[t][s] (s <= t) meanwhile into registers, stored once
        // those MMAs (which read its place in the q region) are done.
        const bool kk_rows = quad < C / 32, qk_rows = quad >= 2 && quad - 2 < C / 32;
        const int c0 = cg * 16;
        const int t = (kk_rows ? quad : quad - 2) * 32 + lane;
        uint4 mhi[2], mlo[2];
        if ((kk_rows || qk_rows) && c0 < C) {
          const float gt = vgam[t];
          float d16[16];
          tmem_ld16(lane_base + (uint32_t)(GDNW_COL_KQ + c0), d16);
          if (kk_rows) {
            const float bt = vbeta[t];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int sx = c0 + e;
              amat[t * GDNW_A_STRIDE + sx] = sx < t ? bt * __expf(gt - vgam[sx]) * d16[e] : 0.f;
            }
          } else {
#pragma unroll
            for (int e8 = 0; e8 < 2; ++e8) {
              float mv[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int sx = c0 + 8 * e8 + e;
                mv[e] = sx <= t ? __expf(gt - vgam[sx]) * d16[8 * e8 + e] : 0.f;
              }
              split8(mv, mhi[e8], mlo[e8]);
            }
          }
        }
        ok = named_sync_and_id<1, GDNW_COMPUTE>(mbar_wait(mma3s, ph, args.err, ERR_TIMEOUT_MMA));
        if (!ok) break;
        tc_fence_after();
        if (qk_rows && c0 < C) {
          uint8_t* mop = smem + GDNW_R_Q + GDNW_MQK;  // Mqk hi | lo (rows t, K = s)
#pragma unroll
          for (int e8 = 0; e8 < 2; ++e8) {
            const uint32_t off = kmaj_off(t, c0 + 8 * e8, 0);
            *reinterpret_cast<uint4*>(mop + off) = mhi[e8];
            *reinterpret_cast<uint4*>(mop + 64 * 128 + off) = mlo[e8];
          }
        }
        // X[v][t] = beta_t (v_t[v] - Gam_t P[v][t]) as hi|lo, rows v, K = t (into the S^T region: its MMAs are done)
        uint8_t* xop = smem + GDNW_R_ST;
        if (c0 < C) {
          float pv[16];
          tmem_ld16(lane_base + (uint32_t)(GDNW_COL_P + c0), pv);
#pragma unroll
          for (int e8 = 0; e8 < 16; e8 += 8) {
            float xv8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int tt = c0 + e8 + e;
              xv8[e] = vbeta[tt] * (xv[tt * GDN_D + vrow] - vGam[tt] * pv[e8 + e]);
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
        // Blocked inverse of the unit lower triangular I + A in 16 x 16 blocks (fp32, into tf = the v region, rows
        // 68 floats apart so a thread reads four consecutive columns with one 16-byte load): the diagonal blocks
        // T_ii by forward substitution (thread = one column of one block; the entries above the diagonal come out 0),
        // then A~_im = T_ii A_im for every block below the diagonal at once, then the block rows level by level,
        // T_ij = -sum_{j <= m < i} A~_im T_mj (each thread four columns of one row). The blocks above the diagonal
        // are never formed (masked below).
        constexpr int NB = C / 16, TS = GDNW_T_STRIDE, AS = 17;
        constexpr int NOFF = NB * (NB - 1) / 2;  // blocks below the diagonal: (i, m) -> i (i - 1) / 2 + m
        float* tf = xv;                     // [64][68]
        float* at = tf + GDNW_MAXC * TS;    // A~ [NOFF][16][17]
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
          for (int tt = 0; tt < 16; ++tt) tf[(base + tt) * TS + base + j] = col[tt];
        }
        named_sync_id<1, GDNW_COMPUTE>();
        if (tid < NOFF * 64) {
          // A~_im[r][c4 ..] = sum_{x <= r} T_ii[r][x] A_im[x][c4 ..]
          const int blk = tid >> 6, r = (tid >> 2) & 15, c4 = (tid & 3) * 4;
          const int bi = blk == 0 ? 1 : (blk < 3 ? 2 : 3), m = blk - bi * (bi - 1) / 2;
          float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
          for (int x = 0; x < 16; ++x) {
            const float tv = tf[(bi * 16 + r) * TS + bi * 16 + x];
            const float* ar = amat + (bi * 16 + x) * GDNW_A_STRIDE + m * 16 + c4;
            a0 = fmaf(tv, ar[0], a0);
            a1 = fmaf(tv, ar[1], a1);
            a2 = fmaf(tv, ar[2], a2);
            a3 = fmaf(tv, ar[3], a3);
          }
          float* o = at + (blk * 16 + r) * AS + c4;
          o[0] = a0;
          o[1] = a1;
          o[2] = a2;
          o[3] = a3;
        }
        named_sync_id<1, GDNW_COMPUTE>();
#pragma unroll 1
        for (int d = 1; d < NB; ++d) {
          const int nblk = NB - d;  // blocks (i, j = i - d); task: block tid >> 6, row (tid >> 2) & 15, columns 4 (tid & 3)
          if (tid < nblk * 64) {
            const int q = tid >> 6, r = (tid >> 2) & 15, c4 = (tid & 3) * 4, bi = q + d, bj = q;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
            for (int m = bj; m < bi; ++m) {
              const float* ar = at + ((bi * (bi - 1) / 2 + m) * 16 + r) * AS;
#pragma unroll
              for (int x = 0; x < 16; ++x) {
                const float a = ar[x];
                const float4 t4 = *reinterpret_cast<const float4*>(tf + (m * 16 + x) * TS + bj * 16 + c4);
                acc.x = fmaf(a, t4.x, acc.x);
                acc.y = fmaf(a, t4.y, acc.y);
                acc.z = fmaf(a, t4.z, acc.z);
                acc.w = fmaf(a, t4.w, acc.w);
              }
            }
            *reinterpret_cast<float4*>(tf + (bi * 16 + r) * TS + bj * 16 + c4) =
                make_float4(-acc.x, -acc.y, -acc.z, -acc.w);
          }
          named_sync_id<1, GDNW_COMPUTE>();
        }
        // T as hi|lo operand: rows t, K = s, 16-byte chunks of 8 s (zero above the diagonal blocks)
        uint8_t* top = smem + GDNW_R_Q;
        for (int e = tid; e < C * (C / 8); e += GDNW_COMPUTE) {
          const int tt = e / (C / 8), s0 = (e % (C / 8)) * 8;
          float tv[8];
          if ((s0 >> 4) > (tt >> 4)) {
#pragma unroll
            for (int x = 0; x < 8; ++x) tv[x] = 0.f;
          } else {
            const float4 a = *reinterpret_cast<const float4*>(tf + tt * TS + s0);
            const float4 b = *reinterpret_cast<const float4*>(tf + tt * TS + s0 + 4);
            tv[0] = a.x; tv[1] = a.y; tv[2] = a.z; tv[3] = a.w;
            tv[4] = b.x; tv[5] = b.y; tv[6] = b.z; tv[7] = b.w;
          }
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
        for (int c0 = cg * 16; c0 < C; c0 += 64) {
          float uv[16];
          tmem_ld16(lane_base + (uint32_t)(GDNW_COL_U + c0), uv);
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
      // the output rows' z (prefetched to L2 with the inputs) while the last MMAs run
      float4 z4[4];
      if (out_warp) {
        const float4* zr = reinterpret_cast<const float4*>(args.proj + ((size_t)n * lb + ot) * GDN_IN + GDN_Z_OFF +
                                                           h * GDN_D + ov0);
#pragma unroll
        for (int j = 0; j < 4; ++j) z4[j] = ot < len ? zr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      // ---- F: outputs (gated RMSNorm of o_t over v) and the new state ----
      ok = named_sync_and_id<1, GDNW_COMPUTE>(mbar_wait(mma8, ph, args.err, ERR_TIMEOUT_MMA));
      if (!ok) break;
      tc_fence_after();
      if (out_warp) {
        // token ot, v in [ov0, ov0 + 16): o = Gam_t R' + O; the eight column groups' sums of squares meet in onorm
        float ov[16], rv[16];
        tmem_ld16x2(lane_base + (uint32_t)col_o, ov, lane_base + (uint32_t)col_rr, rv);
        const float gt = vGam[ot];
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          ov[e] = fmaf(gt, rv[e], ov[e]);
          ss = fmaf(ov[e], ov[e], ss);
        }
        onorm[((quad >> 1) * 4 + cg) * GDNW_MAXC + ot] = ss;
        named_sync_id<3, NOUT>();
        float tot = 0.f;
#pragma unroll
        for (int g = 0; g < 8; ++g) tot += onorm[g * GDNW_MAXC + ot];
        const float r = ot < len ? rsqrtf(tot * (1.0f / GDN_D) + args.eps) : 0.f;
        const size_t obase = ((size_t)n * lb + ot) * KEY_DIM + h * GDN_D + ov0;
        const float4* gw4 = reinterpret_cast<const float4*>(gwv + ov0);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float4 ga = gw4[2 * j], gb = gw4[2 * j + 1];
          const float4 z0 = z4[2 * j], z1 = z4[2 * j + 1];
          const float g8[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
          const float zz[8] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = g8[e] * (ov[8 * j + e] * r) * silu_fast(zz[e]);
          uint4 hi, lo;
          split8_bf16(y, hi, lo);
          *reinterpret_cast<uint4*>(args.out_hi + obase + 8 * j) = hi;
          *reinterpret_cast<uint4*>(args.out_lo + obase + 8 * j) = lo;
        }
      }
      ok = named_sync_and_id<1, GDNW_COMPUTE>(mbar_wait(mma8s, ph, args.err, ERR_TIMEOUT_MMA));
      if (!ok) break;
      tc_fence_after();
      {
        // S <- Gam_C S + dS: row k = this thread's lane, v in [32 cg, 32 cg + 32), four 16-byte chunks of the tile
        float dv[32];
        tmem_ld32(lane_base + (uint32_t)(GDNW_COL_DS + cg * 32), dv);
        const float egC = vgc[0];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4* sp = reinterpret_cast<uint4*>(r_state + state_off(vrow, cg * 32 + 8 * c));
          uint4 s = *sp;
          uint32_t* w = reinterpret_cast<uint32_t*>(&s);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = unpack_half2(w[j]);
            w[j] = pack_half2(fmaf(egC, f.x, dv[8 * c + 2 * j]), fmaf(egC, f.y, dv[8 * c + 2 * j + 1]));
          }
          *sp = s;
        }
      }
      fence_proxy_async();
      tc_fence_before();
      named_sync_id<1, GDNW_COMPUTE>();
      if (tid == 0) mbar_arrive(st_done);
      ++seq;
    }
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
