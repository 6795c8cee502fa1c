// Multi-token ring-window attention (ticks of 16..64 tokens) on the tensor cores: an online-softmax ("flash") kernel
// with warp-level MMA (mma.sync m16n8k16, fp16 operands, fp32 accumulate) fed by TMA.
//
// CTA = (session row n, kv head h, block of 128 query rows); query row r = group * lb + token (the qbuf layout), so a
// block holds up to 128 of the 4 * lb rows that share the kv head's keys. Eight warps, each owning 16 query rows (the
// 16 x 256 fp32 accumulator needs ~190 registers a thread, so the CTA stays at two warps per SM sub-partition: no
// separate producer warp).
// Warp 0 first lists the slot's ring tiles (32 columns) holding any filled column, then ceil(lb / 32) tiles of this
// tick's own keys, and publishes every listed key's position; its lane 0 streams each tile's K and V (32 keys x 256
// dims fp16, four [32 x 64] boxes each, 128-byte swizzle) by TMA through a 4-stage ring, refilling a stage once all
// warps have released it. Every warp stages its queries in shared memory as fp16 (same swizzled layout) and per tile
// computes
//   S[16 x 32] = Q K^T          A = Q by ldmatrix, B = K by ldmatrix from the [key][dim] tile (16 k-steps of 16 dims),
//   mask                        key position kp visible to query position qp iff 0 <= kp <= qp and kp > qp - 512,
//   online softmax (fp32)       running row max m and sum l; the accumulator is rescaled by e^(m_old - m_new),
//   O[16 x 256] += P V          A = P (the score fragments as fp16), B = V by ldmatrix.trans,
// and releases the stage. Epilogue: O / l times sigmoid(gate) as the o_proj operand (bf16 hi/lo), or the ungated fp32
// output for the isolated kernel. Rows of padded tokens (token >= lens[n]) write zeros.
// Same contract as ring_attn_kernel (reference engine/fused_kernels.py:288-376; window_attention.py:34-53 for the
// complete-message form), which remains the path for 2..8-token ticks.
#pragma once
#include "attn.cuh"

namespace hsg {

constexpr int PF_THREADS = 256;                   // 8 warps
constexpr int PF_ROWS = 128;                      // query rows per CTA
constexpr int PF_TILE = 32;                       // keys per tile
constexpr int PF_BOX = PF_TILE * 64 * 2;          // one [32 keys x 64 dims] box (4 KB)
constexpr int PF_KV_BYTES = 4 * PF_BOX;           // K or V of one tile (16 KB)
constexpr int PF_STAGE = 2 * PF_KV_BYTES;         // K then V
constexpr int PF_STAGES = 4;
constexpr int PF_QBOX = 16 * 64 * 2;              // one warp's [16 rows x 64 dims] query box (2 KB)
constexpr int PF_QWARP = 4 * PF_QBOX;             // one warp's queries (8 KB)
constexpr int PF_MAXT = WIN / PF_TILE + MAX_LB / PF_TILE;  // 16 ring tiles + 2 tiles of new keys

struct alignas(16) PfMeta {
  int ntile;
  int tile[PF_MAXT];             // ring tile index 0..15, or 16 + j for new-key tile j
  int kpos[PF_MAXT * PF_TILE];   // key position per listed column (-1: never visible)
};

__host__ __device__ inline int pf_smem_bytes() {
  return PF_STAGES * PF_STAGE + 8 * PF_QWARP + (int)sizeof(PfMeta) + 2 * PF_STAGES * 8 + 1024;
}

// tm_rk / tm_rv: this layer's ring K / V as 2-D [rows = (slot*2 + head)*513 + column][256] fp16;
// tm_nk / tm_nv: the tick's new keys / values as [rows = (row*2 + head)*lb + token][256] fp16. [64 x 32] boxes, SW128.
__global__ void __launch_bounds__(PF_THREADS, 1)
ring_prefill_kernel(const __grid_constant__ CUtensorMap tm_rk, const __grid_constant__ CUtensorMap tm_rv,
                    const __grid_constant__ CUtensorMap tm_nk, const __grid_constant__ CUtensorMap tm_nv,
                    const AttnArgs args) {
  extern __shared__ __align__(1024) uint8_t pf_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pf_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qsm = smem + PF_STAGES * PF_STAGE;
  PfMeta* meta = reinterpret_cast<PfMeta*>(qsm + 8 * PF_QWARP);
  uint64_t* full = reinterpret_cast<uint64_t*>(meta + 1);
  uint64_t* empty = full + PF_STAGES;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n = blockIdx.x, h = blockIdx.y, rb0 = blockIdx.z * PF_ROWS;
  const int lb = args.lb, M = ATT_G * lb;
  const int nact = min(8, (M - rb0 + 15) / 16);  // consumer warps with at least one row
  if (tid == 0) {
    for (int s = 0; s < PF_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], nact);
    }
    fence_barrier_init();
    prefetch_tmap(&tm_rk);
    prefetch_tmap(&tm_rv);
    prefetch_tmap(&tm_nk);
    prefetch_tmap(&tm_nv);
  }
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
    // ---- metadata: listed tiles and key positions ----
    int nt = 0;
    if (len > 0) {
      const int64_t* rp = args.ring_pos + (size_t)slot * RING_COLS;
      int kp[16];
      bool any = false;
#pragma unroll
      for (int i = 0; i < 16; ++i) {  // lane L covers ring columns 16L..16L+15 (a tile is a lane pair)
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
  if (warp < nact) {
    // ---- this warp's 16 query rows -> fp16, swizzled like the K tiles (rows beyond M are zero) ----
    uint8_t* qw = qsm + warp * PF_QWARP;
    const int ch = lane;  // this lane's 8-dim chunk of each row
    for (int r0 = 0; r0 < 16; r0 += 4) {  // four rows' loads in flight before any conversion
      float4 a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int row = rb0 + 16 * warp + r0 + u;
        a[u] = b[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row < M) {
          const float4* src = reinterpret_cast<const float4*>(args.qbuf + (head * M + row) * ATT_D + ch * 8);
          a[u] = src[0];
          b[u] = src[1];
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(qw + (ch >> 3) * PF_QBOX + sw128_off(r0 + u, ch & 7)) =
            make_uint4(pack_half2(a[u].x, a[u].y), pack_half2(a[u].z, a[u].w), pack_half2(b[u].x, b[u].y),
                       pack_half2(b[u].z, b[u].w));
    }
    if (!args.out_raw) {
      // the output gates of these rows into L2 now (read in the epilogue): 16 rows x 1 KB, four lines a lane
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int e = lane * 4 + u, r = e >> 3, row = rb0 + 16 * warp + r;
        if (row < M) {
          const int grp = row / lb, tok = row % lb;
          const float* gp = args.proj + ((size_t)n * lb + tok) * ATT_IN + (h * ATT_G + grp) * 2 * ATT_D + ATT_D +
                            (e & 7) * 32;
          asm volatile("prefetch.global.L2 [%0];" ::"l"(gp));
        }
      }
    }
  }
  __syncthreads();
  const int nt = meta->ntile;
  if (warp >= nact) return;

  // the K and V of listed tile t into stage t % PF_STAGES (thread 0)
  const int ring_row = (int)((slot * ATT_HKV + h) * RING_COLS);
  const int new_row = (int)head * lb;
  auto issue = [&](int t) {
    const int s = t % PF_STAGES;
    const int tile = meta->tile[t];
    const bool ring = tile < WIN / PF_TILE;
    const int y = ring ? ring_row + tile * PF_TILE : new_row + (tile - WIN / PF_TILE) * PF_TILE;
    uint8_t* dst = smem + (size_t)s * PF_STAGE;
    mbar_arrive_expect_tx(&full[s], PF_STAGE);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      tma_load_2d(dst + q * PF_BOX, ring ? &tm_rk : &tm_nk, q * 64, y, &full[s]);
      tma_load_2d(dst + PF_KV_BYTES + q * PF_BOX, ring ? &tm_rv : &tm_nv, q * 64, y, &full[s]);
    }
  };
  int issued = 0;
  if (tid == 0) {
    fence_proxy_async();
    for (; issued < min(nt, PF_STAGES); ++issued) issue(issued);
  }

  // ===================================== consumers =====================================
  const int g = lane >> 2, c4 = lane & 3;
  const int r0 = rb0 + 16 * warp + g, r1 = r0 + 8;  // this thread's two query rows
  const int t0 = r0 % lb, t1 = r1 % lb;
  const bool v0 = r0 < M && t0 < len, v1 = r1 < M && t1 < len;
  const int64_t qp0 = start + t0, qp1 = start + t1;
  const float sl = args.scale;
  const uint32_t qbase = smem_u32(qsm + warp * PF_QWARP);
  float o[32][4];
#pragma unroll
  for (int d = 0; d < 32; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  bool ok = true;
  for (int t = 0; t < nt; ++t) {
    const int s = t % PF_STAGES;
    if (tid == 0 && issued < nt && t >= 1) {
      // refill the stage released by tile t - 1 once every warp has passed it
      const int sp = (t - 1) % PF_STAGES;
      if (!mbar_wait(&empty[sp], ((t - 1) / PF_STAGES) & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
      issue(issued++);
    }
    __syncwarp();
    if (!mbar_wait(&full[s], (t / PF_STAGES) & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
    const uint32_t kb = smem_u32(smem + (size_t)s * PF_STAGE), vb = kb + PF_KV_BYTES;
    // ---- S = Q K^T: 4 key n-tiles of 8 ----
    float sc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 16; ++ks) {
      const int box = ks >> 2, ch0 = 2 * (ks & 3);
      uint32_t a0, a1, a2, a3;
      ldmatrix_x4(qbase + box * PF_QBOX + sw128_off((lane & 7) + ((lane >> 3) & 1) * 8, ch0 + (lane >> 4)), a0, a1,
                  a2, a3);
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kb + box * PF_BOX + sw128_off(16 * kp + ((lane >> 4) & 1) * 8 + (lane & 7), ch0 + ((lane >> 3) & 1)),
                    b0, b1, b2, b3);
        mma_f16_16816(sc[2 * kp], a0, a1, a2, a3, b0, b1);
        mma_f16_16816(sc[2 * kp + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // ---- mask + online softmax (rows g: elements 0, 1; g + 8: elements 2, 3) ----
    const int* kpos = meta->kpos + t * PF_TILE;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kp = kpos[8 * j + 2 * c4 + e];
        const bool vis0 = v0 && kp >= 0 && kp <= qp0 && kp > qp0 - WIN;
        const bool vis1 = v1 && kp >= 0 && kp <= qp1 && kp > qp1 - WIN;
        sc[j][e] = vis0 ? sc[j][e] * sl : -INFINITY;
        sc[j][2 + e] = vis1 ? sc[j][2 + e] * sl : -INFINITY;
        mx0 = fmaxf(mx0, sc[j][e]);
        mx1 = fmaxf(mx1, sc[j][2 + e]);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float ms0 = mn0 == -INFINITY ? 0.f : mn0, ms1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = __expf(m0 - ms0), al1 = __expf(m1 - ms1);
    m0 = mn0;
    m1 = mn1;
    uint32_t pa[2][4];
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float p0 = __expf(sc[j][0] - ms0), p1 = __expf(sc[j][1] - ms0);
      const float p2 = __expf(sc[j][2] - ms1), p3 = __expf(sc[j][3] - ms1);
      ps0 += p0 + p1;
      ps1 += p2 + p3;
      pa[j >> 1][(j & 1) * 2 + 0] = pack_half2(p0, p1);  // a0 / a2: row g, keys 16kk + 8(j&1) + 2c4
      pa[j >> 1][(j & 1) * 2 + 1] = pack_half2(p2, p3);  // a1 / a3: row g + 8
    }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
    if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        o[d][0] *= al0; o[d][1] *= al0;
        o[d][2] *= al1; o[d][3] *= al1;
      }
    }
    // ---- O += P V: 16-dim pairs of n-tiles, two 16-key k-steps ----
#pragma unroll
    for (int dp = 0; dp < 16; ++dp) {
      const int box = dp >> 2, ch0 = 2 * (dp & 3);
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vb + box * PF_BOX + sw128_off(16 * kk + ((lane >> 3) & 1) * 8 + (lane & 7), ch0 + (lane >> 4)),
                          b0, b1, b2, b3);
        mma_f16_16816(o[2 * dp], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
        mma_f16_16816(o[2 * dp + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (tid == 0) {
    // leave only after every issued copy has landed (bounded; in the normal path they all have)
    for (int t = max(0, issued - PF_STAGES); t < issued; ++t)
      mbar_wait(&full[t % PF_STAGES], (t / PF_STAGES) & 1, nullptr, 0);
  }
  if (!ok) return;
  // ---- epilogue: row sums over the quad, normalise, gate ----
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = (v0 && l0 > 0.f) ? 1.0f / l0 : 0.f, inv1 = (v1 && l1 > 0.f) ? 1.0f / l1 : 0.f;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = hr ? r1 : r0;
    if (row >= M) continue;
    const float inv = hr ? inv1 : inv0;
    const int grp = row / lb, tok = row % lb, jq = h * ATT_G + grp;
    if (args.out_raw) {
      float* dst = args.out_raw + (head * M + row) * ATT_D + 2 * c4;
#pragma unroll
      for (int d = 0; d < 32; ++d)
        *reinterpret_cast<float2*>(dst + 8 * d) = make_float2(o[d][2 * hr] * inv, o[d][2 * hr + 1] * inv);
      continue;
    }
    const size_t ob = ((size_t)n * lb + tok) * (ATT_HQ * ATT_D) + jq * ATT_D + 2 * c4;
    const float* gate = args.proj + ((size_t)n * lb + tok) * ATT_IN + jq * 2 * ATT_D + ATT_D + 2 * c4;
    const bool live = inv != 0.f;
#pragma unroll
    for (int d0 = 0; d0 < 32; d0 += 8) {
      // eight gate pairs loaded before this batch's stores (a store may alias a later load as far as the compiler
      // knows, which would otherwise serialise one memory round trip per pair)
      float2 gt[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        gt[u] = live ? *reinterpret_cast<const float2*>(gate + 8 * (d0 + u)) : make_float2(0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int d = d0 + u;
        float y0 = 0.f, y1 = 0.f;
        if (live) {
          y0 = o[d][2 * hr] * inv * __fdividef(1.0f, 1.0f + __expf(-gt[u].x));
          y1 = o[d][2 * hr + 1] * inv * __fdividef(1.0f, 1.0f + __expf(-gt[u].y));
        }
        __nv_bfloat16 h0, h1, lo0, lo1;
        split_bf16(y0, h0, lo0);
        split_bf16(y1, h1, lo1);
        *reinterpret_cast<__nv_bfloat162*>(args.out_hi + ob + 8 * d) = __halves2bfloat162(h0, h1);
        *reinterpret_cast<__nv_bfloat162*>(args.out_lo + ob + 8 * d) = __halves2bfloat162(lo0, lo1);
      }
    }
  }
}

}  // namespace hsg
