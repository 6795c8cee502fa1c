// Multi-token ring-window attention for ticks of 32 or 64 tokens on the 5th-generation tensor cores (tcgen05, TMEM).
//
// CTA = (session row n, kv head h, block of 128 query rows: row r = group * lb + token), 256 threads; thread r < 128
// owns query row r, which is TMEM lane r of both accumulators: S (32 columns, the scores of one 32-key tile) and O
// (256 columns, the output); threads 128-255 transpose each V tile while the row threads run the softmax. Thread 0
// also issues the TMA loads and the MMAs. Per listed 32-key tile (the slot's filled ring tiles, then this tick's own
// keys; K and V in a 4-stage shared-memory ring filled by TMA, 128-byte swizzle):
//   S = Q K^T        tcgen05.mma kind::f16, M = 128, N = 32, K = 256 (A = Q staged once as fp16, B = the K tile)
//   softmax          each thread loads its row of S, masks it (key position kp visible to query position qp iff
//                    0 <= kp <= qp and kp > qp - 512), and forms P = 2^(s log2e / 16 - m) against a running maximum m
//                    that is raised only when a tile's maximum exceeds it by more than 8 (log2 units): then the
//                    row's O and sum are rescaled once (tcgen05.ld / st), otherwise P stays below 2^8 and fp16 holds
//                    it; P goes to shared memory as fp16 (64-byte swizzle, K-major); meanwhile the other four
//                    warps transpose the V tile into V^T [256 dims][32 keys] the same way;
//   O += P V         tcgen05.mma, M = 128, N = 256, K = 32 (A = P, B = V^T), accumulating in TMEM.
// A tcgen05.commit after each tile's S MMA also covers the previous tile's PV MMA, so one wait per tile orders the
// reuse of S, P and V^T. Epilogue: O / l times sigmoid(gate) as the o_proj operand (bf16 hi/lo) or the ungated fp32
// output; rows of padded tokens write zeros. Same contract as ring_prefill_kernel (reference
// engine/fused_kernels.py:288-376), which remains the path for 16-token ticks.
#pragma once
#include "ring_prefill.cuh"

namespace hsg {

constexpr int PT_THREADS = 256;  // warps 0-3: one query row a thread (TMEM lanes); warps 4-7: the V^T transpose
constexpr int PT_ROWS = 128;
constexpr int PT_QBOX = PT_ROWS * 128;         // one [128 rows x 64 dims] fp16 box of Q (16 KB)
constexpr int PT_Q = 4 * PT_QBOX;              // 64 KB
constexpr int PT_KVSTAGE = 2 * PF_KV_BYTES;    // K then V of one 32-key tile (32 KB)
constexpr int PT_STAGES = 4;
constexpr int PT_P = PT_ROWS * 64;             // P [128 rows][32 keys] fp16 (8 KB)
constexpr int PT_VT = ATT_D * 64;              // V^T [256 dims][32 keys] fp16 (16 KB)
constexpr uint32_t PT_TMEM_COLS = 512;         // S double-buffered at columns 0..31 and 32..63, O at 256..511
constexpr uint32_t PT_O_COL = 256;

__host__ __device__ inline int pt_smem_bytes() {
  return PT_Q + PT_STAGES * PT_KVSTAGE + PT_P + PT_VT + (int)sizeof(PfMeta) + (PT_STAGES + 4) * 8 + 16 + 1024;
}

// 2^x by the PTX fast approximation (a few ulp of fp32: far below the fp16 rounding the softmax weights then get).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(PT_THREADS, 1)
ring_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_rk, const __grid_constant__ CUtensorMap tm_rv,
                       const __grid_constant__ CUtensorMap tm_nk, const __grid_constant__ CUtensorMap tm_nv,
                       const AttnArgs args) {
  extern __shared__ __align__(1024) uint8_t pt_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pt_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qsm = smem;                                  // Q, 4 boxes of [128 rows x 128 B], SW128
  uint8_t* kvs = qsm + PT_Q;                            // [STAGES] K | V, each 4 boxes of [32 keys x 128 B], SW128
  uint8_t* psm = kvs + PT_STAGES * PT_KVSTAGE;          // P [128 rows x 64 B], SW64
  uint8_t* vts = psm + PT_P;                            // V^T [256 rows x 64 B], SW64
  PfMeta* meta = reinterpret_cast<PfMeta*>(vts + PT_VT);
  uint64_t* full = reinterpret_cast<uint64_t*>(meta + 1);  // [STAGES]
  uint64_t* sbar = full + PT_STAGES;                       // [2] S buffer b holds S_t (t % 2 == b): one phase per t
  uint64_t* pvbar = sbar + 2;                              // PV_t complete: one phase per tile
  uint64_t* mdone = pvbar + 1;                             // every MMA of the CTA complete (teardown)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = blockIdx.x, h = blockIdx.y, rb0 = blockIdx.z * PT_ROWS;
  const int lb = args.lb, M = ATT_G * lb;
  if (tid == 0) {
    for (int s = 0; s < PT_STAGES; ++s) mbar_init(&full[s], 1);
    mbar_init(&sbar[0], 1);
    mbar_init(&sbar[1], 1);
    mbar_init(pvbar, 1);
    mbar_init(mdone, 1);
    fence_barrier_init();
    prefetch_tmap(&tm_rk);
    prefetch_tmap(&tm_rv);
    prefetch_tmap(&tm_nk);
    prefetch_tmap(&tm_nv);
  }
  if (warp == 0) tmem_alloc(tmem_slot, PT_TMEM_COLS);
  pdl_wait();  // qbuf, the new keys and the ring come from earlier kernels of the tick
  if (tid == 0) pdl_trigger();
  int len = (int)args.lens[n];
  const int64_t slot = args.slots[n], start = args.starts[n];
  if (len > 0 && (slot < 0 || slot > args.max_slots)) {
    if (tid == 0) set_error(args.err, ERR_BAD_SLOT);
    len = 0;
  }
  const size_t head = (size_t)n * ATT_HKV + h;

  if (warp == 0) {
    // ---- metadata: listed tiles and key positions (as ring_prefill_kernel) ----
    int nt = 0;
    if (len > 0) {
      const int64_t* rp = args.ring_pos + (size_t)slot * RING_COLS;
      int kp[16];
      bool any = false;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int64_t p = rp[lane * 16 + i];
        kp[i] = p < 0 ? -1 : (p > 0x7fffffff ? 0x7fffffff : (int)p);
        any |= kp[i] >= 0;
      }
      const unsigned anym = __ballot_sync(0xffffffffu, any);
      const bool tile_on = ((anym >> (lane & ~1)) & 3u) != 0;
      const unsigned pairs = anym | (anym >> 1);
      unsigned even_on = 0;
      for (int t = 0; t < 16; ++t) even_on |= ((pairs >> (2 * t)) & 1u) << t;
      const int pos = __popc(even_on & ((1u << (lane >> 1)) - 1u));
      if (tile_on) {
#pragma unroll
        for (int i = 0; i < 16; ++i) meta->kpos[pos * PF_TILE + (lane & 1) * 16 + i] = kp[i];
        if (!(lane & 1)) meta->tile[pos] = lane >> 1;
      }
      nt = __popc(even_on);
      for (int j = 0; j * PF_TILE < lb; ++j, ++nt) {
        const int c = j * PF_TILE + lane;
        meta->kpos[nt * PF_TILE + lane] = c < len ? (int)(start + c) : -1;
        if (lane == 0) meta->tile[nt] = WIN / PF_TILE + j;
      }
    }
    if (lane == 0) meta->ntile = nt;
  }
  // ---- Q -> fp16, SW128 boxes; warp w stages rows 16 w .. 16 w + 15, lane = 8-dim chunk ----
  for (int r0 = 0; r0 < 16; r0 += 4) {
    float4 a[4], b[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int row = rb0 + 16 * warp + r0 + u;
      a[u] = b[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row < M) {
        const float4* src = reinterpret_cast<const float4*>(args.qbuf + (head * M + row) * ATT_D + lane * 8);
        a[u] = src[0];
        b[u] = src[1];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = 16 * warp + r0 + u;
      *reinterpret_cast<uint4*>(qsm + (lane >> 3) * PT_QBOX + sw128_off(r, lane & 7)) =
          make_uint4(pack_half2(a[u].x, a[u].y), pack_half2(a[u].z, a[u].w), pack_half2(b[u].x, b[u].y),
                     pack_half2(b[u].z, b[u].w));
    }
  }
  // this thread's query row (threads 0-127), and its output gates into L2 (read in the epilogue)
  const bool rowt = tid < PT_ROWS;
  const int row = rb0 + (tid & (PT_ROWS - 1));
  const int tok = row % lb, grp = row / lb;
  const bool valid = rowt && row < M && tok < len;
  const int64_t qp = start + tok;
  const float* gate = args.proj + ((size_t)n * lb + tok) * ATT_IN + (h * ATT_G + grp) * 2 * ATT_D + ATT_D;
  if (!args.out_raw && rowt && row < M) {
#pragma unroll
    for (int c = 0; c < 8; ++c) asm volatile("prefetch.global.L2 [%0];" ::"l"(gate + 32 * c));
  }
  fence_proxy_async();  // Q (generic writes) is read by the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  const int nt = meta->ntile;

  const int ring_row = (int)((slot * ATT_HKV + h) * RING_COLS);
  const int new_row = (int)head * lb;
  auto issue = [&](int t) {  // thread 0: K and V of listed tile t into stage t % PT_STAGES
    const int s = t % PT_STAGES;
    const int tile = meta->tile[t];
    const bool ring = tile < WIN / PF_TILE;
    const int y = ring ? ring_row + tile * PF_TILE : new_row + (tile - WIN / PF_TILE) * PF_TILE;
    uint8_t* dst = kvs + s * PT_KVSTAGE;
    mbar_arrive_expect_tx(&full[s], PT_KVSTAGE);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      tma_load_2d(dst + q * PF_BOX, ring ? &tm_rk : &tm_nk, q * 64, y, &full[s]);
      tma_load_2d(dst + PF_KV_BYTES + q * PF_BOX, ring ? &tm_rv : &tm_nv, q * 64, y, &full[s]);
    }
  };
  const uint32_t idesc_s = idesc_f16(PT_ROWS, PF_TILE), idesc_o = idesc_f16(PT_ROWS, ATT_D);
  auto issue_s = [&](int t) {  // thread 0: S_t = Q K_t^T into S buffer t % 2, committed to sbar[t % 2]
    const uint32_t kb = smem_u32(kvs + (t % PT_STAGES) * PT_KVSTAGE), qb = smem_u32(qsm);
    const uint32_t d = tmem + (uint32_t)((t & 1) * PF_TILE);
#pragma unroll
    for (int box = 0; box < 4; ++box)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_bf16(d, sw128_desc(qb + box * PT_QBOX + kk * 32), sw128_desc(kb + box * PF_BOX + kk * 32), idesc_s,
                 (box > 0 || kk > 0) ? 1u : 0u);
    mma_commit(&sbar[t & 1]);
  };
  int issued = 0;
  bool ok = true;
  if (tid == 0 && nt > 0) {
    for (; issued < min(nt, PT_STAGES); ++issued) issue(issued);
    for (int t = 0; t < min(nt, 2) && ok; ++t) {  // S_0 and S_1 ahead of the loop
      ok = mbar_wait(&full[t % PT_STAGES], (t / PT_STAGES) & 1, args.err, ERR_TIMEOUT_TMA);
      if (ok) {
        tc_fence_after();
        issue_s(t);
      }
    }
  }
  // Pipeline: S_{t+2} is issued at the end of iteration t (its buffer's S_t has been read), so the scores of the next
  // tile are ready while this one's softmax runs; PV_t is committed to its own barrier and waited for only where
  // iteration t + 1 touches what it reads or writes (P, V^T, a rescale of O).
  const float sl2 = args.scale * 1.4426950408889634f;  // scores in log2 units
  float m = -INFINITY, l = 0.f;
  for (int t = 0; t < nt; ++t) {
    const int s = t % PT_STAGES;
    if (!rowt) {
      // ---- V_t -> V^T [256 dims][32 keys], 64-byte swizzle: thread 128 + i owns dims 2 i, 2 i + 1 ----
      if (ok) ok = mbar_wait(&full[s], (t / PT_STAGES) & 1, args.err, ERR_TIMEOUT_TMA);
      const int tw = warp - 4;
      const uint8_t* vb = kvs + s * PT_KVSTAGE + PF_KV_BYTES + tw * PF_BOX;  // the box of dims 64 tw .. 64 tw + 63
      const int ch = lane >> 2, sub = (lane & 3) * 4;                         // 16-byte chunk, byte within it
      uint32_t lo[16], hi[16];
#pragma unroll
      for (int k = 0; k < 32; k += 2) {
        const uint32_t a = *reinterpret_cast<const uint32_t*>(vb + sw128_off(k, ch) + sub);
        const uint32_t b = *reinterpret_cast<const uint32_t*>(vb + sw128_off(k + 1, ch) + sub);
        lo[k >> 1] = __byte_perm(a, b, 0x5410);  // (dim d, key k) | (dim d, key k + 1)
        hi[k >> 1] = __byte_perm(a, b, 0x7632);  // (dim d + 1, key k) | (dim d + 1, key k + 1)
      }
      if (ok && t > 0) ok = mbar_wait(pvbar, (t - 1) & 1, args.err, ERR_TIMEOUT_MMA);  // PV_{t-1} read V^T
      const int d = 2 * (tid - PT_ROWS);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        *reinterpret_cast<uint4*>(vts + sw64_off(d, c)) = make_uint4(lo[4 * c], lo[4 * c + 1], lo[4 * c + 2], lo[4 * c + 3]);
        *reinterpret_cast<uint4*>(vts + sw64_off(d + 1, c)) =
            make_uint4(hi[4 * c], hi[4 * c + 1], hi[4 * c + 2], hi[4 * c + 3]);
      }
    } else {
    // ---- this row's scores, mask, running maximum (lazily raised), P ----
    float sc[32];
    if (ok) ok = mbar_wait(&sbar[t & 1], (t >> 1) & 1, args.err, ERR_TIMEOUT_MMA);
    tc_fence_after();
    tmem_ld32(lane_base + (uint32_t)((t & 1) * PF_TILE), sc);
    const int* kpos = meta->kpos + t * PF_TILE;
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int kp = kpos[j];
      const bool vis = valid && kp >= 0 && kp <= qp && kp > qp - WIN;
      sc[j] = vis ? sc[j] * sl2 : -INFINITY;
      mt = fmaxf(mt, sc[j]);
    }
    const bool raise = mt > m + 8.f || (m == -INFINITY && mt > -INFINITY);
    const float alpha = raise ? (m == -INFINITY ? 0.f : ex2_approx(m - mt)) : 1.f;
    if (raise) {
      m = mt;
      l *= alpha;
    }
    // PV_{t-1} read P and accumulates into O: done before P is rewritten or O rescaled
    if (ok && t > 0) ok = mbar_wait(pvbar, (t - 1) & 1, args.err, ERR_TIMEOUT_MMA);
    if (t > 0 && __any_sync(0xffffffffu, raise)) {  // the warp's rows whose maximum rose: rescale their O
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < ATT_D; c += 32) {
        float ov[32];
        tmem_ld32(lane_base + PT_O_COL + c, ov);
#pragma unroll
        for (int j = 0; j < 32; ++j) ov[j] *= alpha;
        tmem_st32(lane_base + PT_O_COL + c, ov);
      }
    }
    uint32_t pp[16];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const float p0 = sc[j] == -INFINITY ? 0.f : ex2_approx(sc[j] - m);
      const float p1 = sc[j + 1] == -INFINITY ? 0.f : ex2_approx(sc[j + 1] - m);
      l += p0 + p1;
      pp[j >> 1] = pack_half2(p0, p1);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<uint4*>(psm + sw64_off(tid, c)) = make_uint4(pp[4 * c], pp[4 * c + 1], pp[4 * c + 2], pp[4 * c + 3]);
    }
    fence_proxy_async();  // P and V^T (generic writes) are read by the tensor cores
    tc_fence_before();
    if (!__syncthreads_and(ok)) { ok = false; break; }
    if (tid == 0) {
      tc_fence_after();
      // O += P V^T
      const uint32_t pb = smem_u32(psm), vtb = smem_u32(vts);
#pragma unroll
      for (int kk = 0; kk < 2; ++kk)
        mma_bf16(tmem + PT_O_COL, sw64_desc(pb + kk * 32), sw64_desc(vtb + kk * 32), idesc_o,
                 (t > 0 || kk > 0) ? 1u : 0u);
      mma_commit(pvbar);
      // the stage of tile t is free (S_t done, V_t transposed): fetch tile t + STAGES; S_{t+2} into S_t's buffer
      if (issued < nt) issue(issued++);
      if (t + 2 < nt) {
        if (mbar_wait(&full[(t + 2) % PT_STAGES], ((t + 2) / PT_STAGES) & 1, args.err, ERR_TIMEOUT_TMA)) {
          tc_fence_after();
          issue_s(t + 2);
        } else {
          ok = false;  // the rows' wait for S_{t+2} then runs out and reports
        }
      }
    }
  }
  // ---- epilogue: O / l times sigmoid(gate) ----
  if (ok && nt > 0) ok = __syncthreads_and(mbar_wait(pvbar, (nt - 1) & 1, args.err, ERR_TIMEOUT_MMA));
  tc_fence_after();
  const float inv = (ok && valid && l > 0.f) ? 1.0f / l : 0.f;
  if (rowt && row < M) {
#pragma unroll 1
    for (int c = 0; c < ATT_D; c += 32) {
      float ov[32];
      if (nt > 0) {
        tmem_ld32(lane_base + PT_O_COL + c, ov);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) ov[j] = 0.f;
      }
      if (args.out_raw) {
        float* dst = args.out_raw + (head * M + row) * ATT_D + c;
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4*>(dst + j) = make_float4(ov[j] * inv, ov[j + 1] * inv, ov[j + 2] * inv, ov[j + 3] * inv);
        continue;
      }
      float4 gt[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) gt[j] = inv != 0.f ? reinterpret_cast<const float4*>(gate + c)[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      uint32_t hh[16], ll[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float2 g2 = j & 2 ? make_float2(gt[j >> 2].z, gt[j >> 2].w) : make_float2(gt[j >> 2].x, gt[j >> 2].y);
        const float y0 = ov[j] * inv * __fdividef(1.0f, 1.0f + __expf(-g2.x));
        const float y1 = ov[j + 1] * inv * __fdividef(1.0f, 1.0f + __expf(-g2.y));
        __nv_bfloat162 h2, l2;
        split_bf16x2(y0, y1, h2, l2);
        hh[j >> 1] = *reinterpret_cast<uint32_t*>(&h2);
        ll[j >> 1] = *reinterpret_cast<uint32_t*>(&l2);
      }
      const size_t ob = ((size_t)n * lb + tok) * (ATT_HQ * ATT_D) + (h * ATT_G + grp) * ATT_D + c;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        reinterpret_cast<uint4*>(args.out_hi + ob)[j] = make_uint4(hh[4 * j], hh[4 * j + 1], hh[4 * j + 2], hh[4 * j + 3]);
        reinterpret_cast<uint4*>(args.out_lo + ob)[j] = make_uint4(ll[4 * j], ll[4 * j + 1], ll[4 * j + 2], ll[4 * j + 3]);
      }
    }
  }
  // ---- teardown: every MMA done and the last copies landed (both only pending on error paths), TMEM released ----
  if (tid == 0) {
    mma_commit(mdone);
    mbar_wait(mdone, 0, args.err, ERR_TIMEOUT_MMA);
    for (int t = max(0, issued - PT_STAGES); t < issued; ++t)
      mbar_wait(&full[t % PT_STAGES], (t / PT_STAGES) & 1, nullptr, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, PT_TMEM_COLS);
  }
}

}  // namespace hsg
