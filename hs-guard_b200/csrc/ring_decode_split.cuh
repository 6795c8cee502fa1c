// Single-token ring-window attention decode for small batches: each (session row, kv head) item is split over a
// cluster of RDS_SPLIT CTAs (split-KV, flash-decoding style) so that a few dozen slots still fill the machine.
//
// ring_decode_kernel (ring_decode.cuh) deals whole items to one persistent CTA per SM; with fewer items than SMs a
// call lasts as long as the fullest ring takes to stream through one SM (up to 512 keys of K and V, 512 KB). Here CTA
// `split` of an item's cluster takes the item's listed 32-key tiles split, split + RDS_SPLIT, ... (the list and the
// per-key positions are built as in ring_decode_kernel, by every CTA of the cluster), runs the same two passes on
// them (S = K Q^T and P V on warp-level MMA, fp16 in, fp32 accumulate), and keeps the unnormalised partial output
// O_s, the maximum m_s and the sum l_s of each query row in its shared memory. After a cluster barrier CTA 0 combines
// them through distributed shared memory,
//   M = max_s m_s,  L = sum_s l_s e^(m_s - M),  o = sum_s O_s e^(m_s - M) / L,
// writes the output (ungated fp32 for the isolated kernel, else out * sigmoid(gate) as the o_proj operand) and the
// new key/value into ring column start % 512; a second cluster barrier keeps the other CTAs' shared memory alive
// until it has been read. Every CTA reaches both barriers on every path (errors included): the waits before them are
// bounded and report through `err`.
// Same contract as ring_decode_kernel (reference engine/fused_kernels.py:288-376 for Lb = 1).
#pragma once
#include <cooperative_groups.h>
#include "ring_decode.cuh"

namespace hsg {

constexpr int RDS_SPLIT = 2;                                        // CTAs per item (cluster size)
constexpr int RDS_STAGES = 5;                                       // 80 KB of tiles in flight: two CTAs a SM
constexpr int RDS_MAXT = (RD_MAXT + RDS_SPLIT - 1) / RDS_SPLIT;     // listed tiles per CTA (5)
constexpr int RDS_MAXK = RDS_MAXT * RD_TILE;
constexpr int RDS_PSTRIDE = RDS_MAXK + 8;

__host__ __device__ inline int rds_smem_bytes() {
  // stages | meta | partial scores [4][MAXK][4] f32 | probabilities [4][PSTRIDE] f16 | row max, sum [4] each |
  // partial output [4][256] f32 | barriers
  return RDS_STAGES * RD_TILE_BYTES + (int)sizeof(RdMeta) + 4 * RDS_MAXK * 4 * 4 + 4 * RDS_PSTRIDE * 2 + 32 +
         ATT_G * ATT_D * 4 + 64 + (2 * RDS_STAGES + 1) * 8 + 1024;
}

// grid (RDS_SPLIT, nb * 2) in clusters of (RDS_SPLIT, 1, 1); maps as ring_decode_kernel's.
__global__ void __launch_bounds__(RD_THREADS, 2)
ring_decode_split_kernel(const __grid_constant__ CUtensorMap tm_rk, const __grid_constant__ CUtensorMap tm_rv,
                         const __grid_constant__ CUtensorMap tm_nk, const __grid_constant__ CUtensorMap tm_nv,
                         const AttnArgs args) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(1024) uint8_t rds_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rds_smem_raw) + 1023) & ~uintptr_t(1023));
  RdMeta* meta = reinterpret_cast<RdMeta*>(smem + RDS_STAGES * RD_TILE_BYTES);
  float* scp = reinterpret_cast<float*>(meta + 1);                 // [4 dim ranges][MAXK][4 rows] partial scores
  __half* pr = reinterpret_cast<__half*>(scp + 4 * RDS_MAXK * 4);  // [4 rows][PSTRIDE] probabilities
  float* lmax = reinterpret_cast<float*>(pr + 4 * RDS_PSTRIDE);    // [4] row maxima over this CTA's keys
  float* lsum = lmax + 4;                                           // [4] row sums of e^(s - max)
  float* opart = lsum + 4;                                          // [4 rows][256] unnormalised partial output
  float* hmax = opart + ATT_G * ATT_D;                              // [2 key halves][4 rows] maxima
  float* hsum = hmax + 8;                                           // [2 key halves][4 rows] sums
  uint64_t* full = reinterpret_cast<uint64_t*>(hsum + 8);           // [RDS_STAGES]
  uint64_t* empty = full + RDS_STAGES;                                  // [RDS_STAGES]
  uint64_t* meta_full = empty + RDS_STAGES;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, item = blockIdx.y;
  const int n = item / ATT_HKV, h = item % ATT_HKV;
  if (tid == 0) {
    for (int s = 0; s < RDS_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], RD_CONS);
    }
    mbar_init(meta_full, 1);
    fence_barrier_init();
    prefetch_tmap(&tm_rk);
    prefetch_tmap(&tm_rv);
    prefetch_tmap(&tm_nk);
    prefetch_tmap(&tm_nv);
  }
  __syncthreads();
  pdl_wait();
  if (tid == 0) pdl_trigger();
  RdMeta& m = *meta;
  bool ok = true;

  if (warp == RD_CONS / 32) {
    // ===================================== producer =====================================
    int len = (int)args.lens[n];
    const int64_t slot = args.slots[n], start = args.starts[n];
    if (len > 0 && (slot < 0 || slot > args.max_slots)) {
      if (lane == 0 && split == 0) set_error(args.err, ERR_BAD_SLOT);
      len = 0;
    }
    int nt = 0;
    if (len > 0) {
      const int64_t* rp = args.ring_pos + (size_t)slot * RING_COLS;
      // lane L covers ring columns 16L..16L+15 (tiles are lane pairs)
      int kp[16];
      bool any = false;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int64_t p = rp[lane * 16 + i];
        kp[i] = p < 0 ? -1 : (p > 0x7fffffff ? 0x7fffffff : (int)p);
        any |= kp[i] >= 0;
      }
      const unsigned anym = __ballot_sync(0xffffffffu, any);
      // tile t is listed when lane 2t or 2t+1 saw a filled column; its list position = listed tiles before it
      const bool tile_on = ((anym >> (lane & ~1)) & 3u) != 0;
      const unsigned pairs = anym | (anym >> 1);
      unsigned even_on = 0;
      for (int t = 0; t < 16; ++t) even_on |= ((pairs >> (2 * t)) & 1u) << t;
      const int pos = __popc(even_on & ((1u << (lane >> 1)) - 1u));
      if (tile_on) {
#pragma unroll
        for (int i = 0; i < 16; ++i) m.kpos[pos * RD_TILE + (lane & 1) * 16 + i] = kp[i];
        if (!(lane & 1)) m.tile[pos] = lane >> 1;
      }
      nt = __popc(even_on);
      // the tick's own key: the new-key tile (its other 31 columns are never visible)
      m.kpos[nt * RD_TILE + lane] = lane < len ? (int)(start + lane) : -1;
      if (lane == 0) m.tile[nt] = -1;
      ++nt;
    }
    __syncwarp();  // every lane's metadata writes are ordered before lane 0's releasing arrive
    if (lane == 0) {
      m.qpos = start;
      m.slot = slot;
      m.len = len;
      m.ntile = nt;
      mbar_arrive(meta_full);
    }
    __syncwarp();
    const int ntl = nt > split ? (nt - split + RDS_SPLIT - 1) / RDS_SPLIT : 0;  // this CTA's tiles
    const int ring_row = (int)((slot * ATT_HKV + h) * RING_COLS);
    const int new_row = n * ATT_HKV + h;
    int cnt = 0;
    for (int pass = 0; pass < 2 && ok; ++pass) {
      const CUtensorMap* ring = pass == 0 ? &tm_rk : &tm_rv;
      const CUtensorMap* fresh = pass == 0 ? &tm_nk : &tm_nv;
      for (int lt = 0; lt < ntl; ++lt, ++cnt) {
        const int s = cnt % RDS_STAGES;
        if (cnt >= RDS_STAGES && !mbar_wait(&empty[s], ((cnt / RDS_STAGES) - 1) & 1, args.err, ERR_TIMEOUT_TMA)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const int tile = m.tile[split + lt * RDS_SPLIT];
          const CUtensorMap* map = tile >= 0 ? ring : fresh;
          const int y = tile >= 0 ? ring_row + tile * RD_TILE : new_row;
          uint8_t* dst = smem + (size_t)s * RD_TILE_BYTES;
          mbar_arrive_expect_tx(&full[s], RD_TILE_BYTES);
#pragma unroll
          for (int q = 0; q < 4; ++q) tma_load_2d(dst + q * RD_SUB_BYTES, map, q * 64, y, &full[s]);
        }
        __syncwarp();
      }
    }
    // loads still in flight land before the CTA leaves (bounded; on the normal path the consumers waited for all)
    if (lane == 0 && cnt > 0) mbar_wait(&full[(cnt - 1) % RDS_STAGES], ((cnt - 1) / RDS_STAGES) & 1, args.err,
                                        ERR_TIMEOUT_TMA);
  } else {
    // ===================================== consumers =====================================
    const int g = lane >> 2, c4 = lane & 3;   // mma fragment coordinates
    const int kh = warp & 1, kr = warp >> 1;  // pass 1: key half of the tile, dim range
    ok = named_sync_and<RD_CONS>(mbar_wait(meta_full, 0, args.err, ERR_TIMEOUT_TMA));
    const int nt = ok ? m.ntile : 0;
    const int len = ok ? m.len : 0;
    const int64_t qpos = m.qpos;
    const int ntl = nt > split ? (nt - split + RDS_SPLIT - 1) / RDS_SPLIT : 0;
    float o[2][4];
#pragma unroll
    for (int mb = 0; mb < 2; ++mb) o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.f;
    if (ntl > 0) {
      // pass-1 B fragments: Q^T for this warp's 64 dims (4 k-steps); query row = fragment column g (rows >= 4 zero)
      uint32_t qb[4][2];
      {
        const float* qrow = args.qbuf + (((size_t)n * ATT_HKV + h) * ATT_G + (g & 3)) * ATT_D + kr * 64;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const float2 lo2 = *reinterpret_cast<const float2*>(qrow + ks * 16 + 2 * c4);
          const float2 hi2 = *reinterpret_cast<const float2*>(qrow + ks * 16 + 8 + 2 * c4);
          qb[ks][0] = g < ATT_G ? pack_half2(lo2.x, lo2.y) : 0u;
          qb[ks][1] = g < ATT_G ? pack_half2(hi2.x, hi2.y) : 0u;
        }
      }
      float* sp = scp + (size_t)kr * RDS_MAXK * 4;
      int cnt = 0;
      // ---- pass 1: partial scores over this warp's dim range, this CTA's tiles ----
      for (int lt = 0; lt < ntl && ok; ++lt, ++cnt) {
        const int s = cnt % RDS_STAGES;
        if (!mbar_wait(&full[s], (cnt / RDS_STAGES) & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
        const uint32_t sub = smem_u32(smem + (size_t)s * RD_TILE_BYTES + kr * RD_SUB_BYTES);
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          // A = K[keys 16kh..+15][dims 16ks..+15]: matrix mi = lane/8 -> key +8*(mi&1), chunk +(mi>>1)
          const int mi = lane >> 3, r = 16 * kh + (mi & 1) * 8 + (lane & 7), ch = 2 * ks + (mi >> 1);
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(sub + sw128_off(r, ch), a0, a1, a2, a3);
          mma_f16_16816(d, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
        }
        mbar_arrive(&empty[s]);  // this warp has read the K tile
        if (c4 < 2) {             // fragment columns 2*c4, +1 are query rows 0..3
          const int key = lt * RD_TILE + 16 * kh + g;
          *reinterpret_cast<float2*>(sp + key * 4 + 2 * c4) = make_float2(d[0], d[1]);
          *reinterpret_cast<float2*>(sp + (key + 8) * 4 + 2 * c4) = make_float2(d[2], d[3]);
        }
      }
      ok = named_sync_and<RD_CONS>(ok);
      // ---- softmax per query row r over this CTA's keys: warps r and r + 4 take alternate 32-key tiles (sum the
      // four dim ranges, mask); the two halves' maxima and sums meet in shared memory ----
      if (ok) {
        const int r = warp & 3, hf = warp >> 2, nk = ntl * RD_TILE;
        float mx = -INFINITY;
#pragma unroll 4
        for (int c = hf * RD_TILE + lane; c < nk; c += 2 * RD_TILE) {
          const int kp = m.kpos[(split + (c / RD_TILE) * RDS_SPLIT) * RD_TILE + (c % RD_TILE)];
          float sc = -INFINITY;
          if (kp >= 0 && kp <= qpos && kp > qpos - WIN)
            sc = (scp[c * 4 + r] + scp[(RDS_MAXK + c) * 4 + r] + scp[(2 * RDS_MAXK + c) * 4 + r] +
                  scp[(3 * RDS_MAXK + c) * 4 + r]) * args.scale;
          scp[c * 4 + r] = sc;
          mx = fmaxf(mx, sc);
        }
        mx = warp_max(mx);
        if (lane == 0) hmax[hf * 4 + r] = mx;
        named_sync<RD_CONS>();
        mx = fmaxf(hmax[r], hmax[4 + r]);
        const float msafe = mx == -INFINITY ? 0.f : mx;
        float sum = 0.f;
#pragma unroll 4
        for (int c = hf * RD_TILE + lane; c < nk; c += 2 * RD_TILE) {
          const float p = __expf(scp[c * 4 + r] - msafe);  // rounded to fp16 below
          pr[r * RDS_PSTRIDE + c] = __float2half_rn(p);
          sum += p;
        }
        sum = warp_sum(sum);
        if (lane == 0) hsum[hf * 4 + r] = sum;
      }
      named_sync<RD_CONS>();
      if (tid < ATT_G) {
        lmax[tid] = ok ? fmaxf(hmax[tid], hmax[4 + tid]) : -INFINITY;
        lsum[tid] = ok ? hsum[tid] + hsum[4 + tid] : 0.f;
      }
      // ---- pass 2: O^T[dims 32w..32w+31] += V^T P^T ----
      const int dsub = warp >> 1;        // the 64-dim box holding dims 32w..32w+31
      const int cbase = (warp & 1) * 4;  // first 16-byte chunk of those dims inside the box
      for (int lt = 0; lt < ntl && ok; ++lt, ++cnt) {
        const int s = cnt % RDS_STAGES;
        if (!mbar_wait(&full[s], (cnt / RDS_STAGES) & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
        const uint32_t sub = smem_u32(smem + (size_t)s * RD_TILE_BYTES + dsub * RD_SUB_BYTES);
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {  // 16 keys per k-step
          const int kc = lt * RD_TILE + 16 * ks + 2 * c4;
          const uint32_t b0 = g < ATT_G ? *reinterpret_cast<const uint32_t*>(pr + (g & 3) * RDS_PSTRIDE + kc) : 0u;
          const uint32_t b1 =
              g < ATT_G ? *reinterpret_cast<const uint32_t*>(pr + (g & 3) * RDS_PSTRIDE + kc + 8) : 0u;
#pragma unroll
          for (int mb = 0; mb < 2; ++mb) {
            const int mi = lane >> 3, r = 16 * ks + (mi >> 1) * 8 + (lane & 7), ch = cbase + 2 * mb + (mi & 1);
            uint32_t a0, a1, a2, a3;
            ldmatrix_x4_trans(sub + sw128_off(r, ch), a0, a1, a2, a3);
            mma_f16_16816(o[mb], a0, a1, a2, a3, b0, b1);
          }
        }
        mbar_arrive(&empty[s]);
      }
    } else if (tid < ATT_G) {
      lmax[tid] = -INFINITY;  // no keys here
      lsum[tid] = 0.f;
    }
    // ---- this CTA's unnormalised partial output (lanes with c4 < 2: rows 2*c4, +1; dims 32w + 16mb + g (+8)) ----
    if (c4 < 2) {
#pragma unroll
      for (int mb = 0; mb < 2; ++mb)
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
            opart[(2 * c4 + cc) * ATT_D + 32 * warp + 16 * mb + g + 8 * half] = ok ? o[mb][2 * half + cc] : 0.f;
    }
    (void)len;
  }
  cluster.sync();  // every CTA's partial output, maxima and sums are in its shared memory
  if (split == 0 && tid < RD_CONS) {
    const int len = m.len;
    const int64_t qpos = m.qpos;
    __nv_bfloat16* ohi = args.out_hi + (size_t)n * (ATT_HQ * ATT_D) + h * ATT_G * ATT_D;
    __nv_bfloat16* olo = args.out_lo + (size_t)n * (ATT_HQ * ATT_D) + h * ATT_G * ATT_D;
    // thread: query row r = tid / 64, dims 4 (tid % 64) .. + 3
    const int r = tid >> 6, d0 = (tid & 63) * 4;
    float mxs[RDS_SPLIT], ls[RDS_SPLIT];
    float M = -INFINITY;
#pragma unroll
    for (int s = 0; s < RDS_SPLIT; ++s) {
      const float* rl = cluster.map_shared_rank(lmax, s);
      mxs[s] = rl[r];
      ls[s] = rl[4 + r];  // lsum follows lmax
      M = fmaxf(M, mxs[s]);
    }
    float L = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < RDS_SPLIT; ++s) {
      const float w = mxs[s] == -INFINITY ? 0.f : __expf(mxs[s] - M);
      L = fmaf(w, ls[s], L);
      const float4 v = *reinterpret_cast<const float4*>(cluster.map_shared_rank(opart, s) + r * ATT_D + d0);
      acc[0] = fmaf(w, v.x, acc[0]);
      acc[1] = fmaf(w, v.y, acc[1]);
      acc[2] = fmaf(w, v.z, acc[2]);
      acc[3] = fmaf(w, v.w, acc[3]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float val = len > 0 && L > 0.f ? acc[e] / L : 0.f;
      const int dim = d0 + e;
      if (args.out_raw) {
        args.out_raw[(((size_t)n * ATT_HKV + h) * ATT_G + r) * ATT_D + dim] = val;
      } else {
        const float gt = len > 0 ? args.proj[(size_t)n * ATT_IN + (h * ATT_G + r) * 2 * ATT_D + ATT_D + dim] : 0.f;
        split_bf16(val * __fdividef(1.0f, 1.0f + __expf(-gt)), ohi[r * ATT_D + dim], olo[r * ATT_D + dim]);
      }
    }
    if (args.write_ring && len > 0 && tid < ATT_D / 2) {
      // the new key/value go into ring column start % 512 (every CTA of the cluster has read its tiles)
      const size_t src = ((size_t)n * ATT_HKV + h) * ATT_D + 2 * tid;
      const size_t col = (size_t)(qpos % WIN);
      const size_t dst = (((size_t)m.slot * ATT_HKV + h) * RING_COLS + col) * ATT_D + 2 * tid;
      *reinterpret_cast<__half2*>(args.ring_k + dst) = *reinterpret_cast<const __half2*>(args.knew + src);
      *reinterpret_cast<__half2*>(args.ring_v + dst) = *reinterpret_cast<const __half2*>(args.vnew + src);
    }
  }
  cluster.sync();  // the other CTAs' shared memory stays alive until CTA 0 has read it
}

}  // namespace hsg
