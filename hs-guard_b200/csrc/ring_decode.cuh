// Single-token ring-window attention decode (1-token ticks), a persistent warp-specialised TMA pipeline (sm_100a).
//
// Work item = (session row n, kv head h): the 4 query heads of group h attend over the slot's ring (up to 512 keys)
// plus the tick's own key. Grid = one CTA per SM; items are dealt round-robin.
//
// Producer warp: per item it reads the slot's ring positions, lists the 32-column tiles holding any filled column
// plus the new-key tile, publishes the list (with every key's position) in a double-buffered metadata block, then
// streams the K tiles and after them the V tiles (16 KB fp16 each, one TMA bulk copy) through an 8-stage ring.
// Consumer warps (8): pass 1 scores every listed key (warp w takes keys 4w..4w+3 of a tile; lanes split the 256 dims,
// a warp reduce-scatter finishes the 16 dot products), masked by the window rule 0 <= kpos <= qpos, kpos > qpos - 512;
// one softmax per query row over all scores (fp32); pass 2 accumulates P.V (thread t: dims 2*(t%128), +1, keys of
// parity t/128). Stages are released by mbarrier arrivals, so no block-wide barrier sits inside the tile loops.
// Output: out * sigmoid(gate) as the o_proj operand (bf16 hi/lo). Then the new key/value are written into ring
// column start % 512 (the position there, start - 512, is outside this query's window).
// Same contract and results as ring_attn_kernel<4> (reference engine/fused_kernels.py:288-376 for Lb = 1).
#pragma once
#include "attn.cuh"

namespace hsg {

constexpr int RD_CONS = 256;                     // consumer threads
constexpr int RD_THREADS = RD_CONS + 32;         // + producer warp
constexpr int RD_TILE = 32;                      // keys per tile
constexpr int RD_TILE_BYTES = RD_TILE * ATT_D * 2;
constexpr int RD_STAGES = 8;
constexpr int RD_MAXT = WIN / RD_TILE + 1;       // 16 ring tiles + the new-key tile
constexpr int RD_MAXK = RD_MAXT * RD_TILE;

struct alignas(16) RdMeta {  // 16-byte multiple: the score array after the two copies stays float4-aligned
  int64_t qpos;
  int len, ntile;
  int tile[RD_MAXT];      // ring tile index, or -1 for the new-key tile
  int kpos[RD_MAXK];      // key position per listed tile column (-1: not visible)
};

__host__ __device__ inline int rd_smem_bytes() {
  // stages | meta x2 | scores [MAXK][4] | partial acc [4][256] | row sums [4] | barriers (8 full, 8 empty, 2+2 meta)
  return RD_STAGES * RD_TILE_BYTES + 2 * (int)sizeof(RdMeta) + RD_MAXK * 4 * 4 + 4 * ATT_D * 4 + 16 +
         (2 * RD_STAGES + 4) * 8 + 128;
}

__global__ void __launch_bounds__(RD_THREADS, 1) ring_decode_kernel(const AttnArgs args) {
  extern __shared__ __align__(128) uint8_t rd_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rd_smem_raw) + 127) & ~uintptr_t(127));
  __half* stages = reinterpret_cast<__half*>(smem);
  RdMeta* meta = reinterpret_cast<RdMeta*>(smem + RD_STAGES * RD_TILE_BYTES);
  float* sc = reinterpret_cast<float*>(meta + 2);            // [MAXK][4]
  float* xacc = sc + RD_MAXK * 4;                            // [4][256]
  float* lsum = xacc + 4 * ATT_D;                            // [4]
  uint64_t* full = reinterpret_cast<uint64_t*>(lsum + 4);    // [8]
  uint64_t* empty = full + RD_STAGES;                        // [8]
  uint64_t* meta_full = empty + RD_STAGES;                   // [2]
  uint64_t* meta_free = meta_full + 2;                       // [2]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_items = args.nb * ATT_HKV;
  if (tid == 0) {
    for (int s = 0; s < RD_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], RD_CONS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&meta_full[b], 1);
      mbar_init(&meta_free[b], RD_CONS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  if (tid == 0) pdl_trigger();

  if (warp == RD_CONS / 32) {
    // ===================================== producer =====================================
    int cnt = 0, k = 0;
    for (int j = blockIdx.x; j < n_items; j += gridDim.x, ++k) {
      const int b = k & 1, n = j / ATT_HKV, h = j % ATT_HKV;
      if (k >= 2 && !mbar_wait(&meta_free[b], ((k >> 1) - 1) & 1, args.err, ERR_TIMEOUT_TMA)) return;
      int len = (int)args.lens[n];
      const int64_t slot = args.slots[n], start = args.starts[n];
      if (len > 0 && (slot < 0 || slot > args.max_slots)) {
        if (lane == 0) set_error(args.err, ERR_BAD_SLOT);
        len = 0;
      }
      RdMeta& m = meta[b];
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
        // the tick's own key(s): the new-key tile
        if (lane < RD_TILE) m.kpos[nt * RD_TILE + lane] = lane < len ? (int)(start + lane) : -1;
        if (lane == 0) m.tile[nt] = -1;
        ++nt;
      }
      __syncwarp();  // every lane's metadata writes are ordered before lane 0's releasing arrive
      if (lane == 0) {
        m.qpos = start;
        m.len = len;
        m.ntile = nt;
        mbar_arrive(&meta_full[b]);
      }
      __syncwarp();
      if (len == 0) continue;
      const size_t head = ((size_t)slot * ATT_HKV + h) * RING_COLS * ATT_D;
      const size_t nhead = ((size_t)n * ATT_HKV + h) * ATT_D;  // lb == 1: one new row per (row, head)
      for (int pass = 0; pass < 2; ++pass) {
        const __half* ring = pass == 0 ? args.ring_k : args.ring_v;
        const __half* fresh = pass == 0 ? args.knew : args.vnew;
        for (int t = 0; t < nt; ++t, ++cnt) {
          const int s = cnt % RD_STAGES;
          if (cnt >= RD_STAGES && !mbar_wait(&empty[s], ((cnt / RD_STAGES) - 1) & 1, args.err, ERR_TIMEOUT_TMA))
            return;
          if (lane == 0) {
            const int tile = m.tile[t];
            const uint32_t bytes = tile >= 0 ? RD_TILE_BYTES : ATT_D * 2;
            const __half* src = tile >= 0 ? ring + head + (size_t)tile * RD_TILE * ATT_D : fresh + nhead;
            mbar_arrive_expect_tx(&full[s], bytes);
            bulk_g2s(stages + (size_t)s * RD_TILE * ATT_D, src, bytes, &full[s]);
          }
          __syncwarp();
        }
      }
    }
    return;
  }

  // ===================================== consumers =====================================
  const int dp = tid & 127, par = tid >> 7;
  int cnt = 0, k = 0;
  bool ok = true;
  for (int j = blockIdx.x; j < n_items && ok; j += gridDim.x, ++k) {
    const int b = k & 1, n = j / ATT_HKV, h = j % ATT_HKV;
    if (!named_sync_and<RD_CONS>(mbar_wait(&meta_full[b], (k >> 1) & 1, args.err, ERR_TIMEOUT_TMA))) break;
    const RdMeta& m = meta[b];
    const int len = m.len, nt = m.ntile;
    const int64_t qpos = m.qpos;
    __nv_bfloat16* ohi = args.out_hi + (size_t)n * (ATT_HQ * ATT_D) + h * ATT_G * ATT_D;
    __nv_bfloat16* olo = args.out_lo + (size_t)n * (ATT_HQ * ATT_D) + h * ATT_G * ATT_D;
    if (len == 0) {
      for (int e = tid; e < ATT_G * ATT_D; e += RD_CONS) {
        if (args.out_raw) {
          args.out_raw[((size_t)n * ATT_HKV + h) * ATT_G * ATT_D + e] = 0.f;
        } else {
          ohi[e] = __float2bfloat16_rn(0.f);
          olo[e] = __float2bfloat16_rn(0.f);
        }
      }
      mbar_arrive(&meta_free[b]);
      continue;
    }
    // queries: lane holds dims 8*lane..+7 of the 4 rows of group h
    float q[ATT_G][8];
#pragma unroll
    for (int r = 0; r < ATT_G; ++r) {
      const float* src = args.qbuf + (((size_t)n * ATT_HKV + h) * ATT_G + r) * ATT_D + lane * 8;
      const float4 a = reinterpret_cast<const float4*>(src)[0], c = reinterpret_cast<const float4*>(src)[1];
      q[r][0] = a.x; q[r][1] = a.y; q[r][2] = a.z; q[r][3] = a.w;
      q[r][4] = c.x; q[r][5] = c.y; q[r][6] = c.z; q[r][7] = c.w;
    }
    // ---- pass 1: scores ----
    for (int t = 0; t < nt && ok; ++t, ++cnt) {
      const int s = cnt % RD_STAGES;
      if (!mbar_wait(&full[s], (cnt / RD_STAGES) & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
      const __half* kt = stages + (size_t)s * RD_TILE * ATT_D;
      const int ncols = m.tile[t] >= 0 ? RD_TILE : 1;
      float part[4 * ATT_G];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int c = warp * 4 + kk;
        float kf[8];
        if (c < ncols) {
          const uint4 raw = *reinterpret_cast<const uint4*>(kt + c * ATT_D + lane * 8);
          const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(h2[i]);
            kf[2 * i] = f.x; kf[2 * i + 1] = f.y;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) kf[i] = 0.f;
        }
#pragma unroll
        for (int r = 0; r < ATT_G; ++r) {
          float d = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) d = fmaf(q[r][i], kf[i], d);
          part[kk * ATT_G + r] = d;
        }
      }
      mbar_arrive(&empty[s]);  // the K tile has been read
      const float sres = reduce_scatter<4 * ATT_G>(part, lane);
      const int idx = lane >> 1, kk = idx / ATT_G, r = idx % ATT_G;
      const int c = warp * 4 + kk;
      const int kp = m.kpos[t * RD_TILE + c];
      const bool vis = c < ncols && kp >= 0 && kp <= qpos && kp > qpos - WIN;
      if (!(lane & 1)) sc[(t * RD_TILE + c) * 4 + r] = vis ? sres * args.scale : -INFINITY;
    }
    if (!named_sync_and<RD_CONS>(ok)) break;
    // ---- softmax per query row (warp r) ----
    if (warp < ATT_G) {
      const int r = warp, nk = nt * RD_TILE;
      float mx = -INFINITY;
      for (int c = lane; c < nk; c += 32) mx = fmaxf(mx, sc[c * 4 + r]);
      mx = warp_max(mx);
      const float msafe = mx == -INFINITY ? 0.f : mx;
      float sum = 0.f;
      for (int c = lane; c < nk; c += 32) {
        const float p = expf(sc[c * 4 + r] - msafe);
        sc[c * 4 + r] = p;
        sum += p;
      }
      sum = warp_sum(sum);
      if (lane == 0) lsum[r] = sum;
    }
    named_sync<RD_CONS>();
    // ---- pass 2: P.V ----
    float acc[ATT_G][2];
#pragma unroll
    for (int r = 0; r < ATT_G; ++r) acc[r][0] = acc[r][1] = 0.f;
    for (int t = 0; t < nt && ok; ++t, ++cnt) {
      const int s = cnt % RD_STAGES;
      if (!mbar_wait(&full[s], (cnt / RD_STAGES) & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
      const __half* vt = stages + (size_t)s * RD_TILE * ATT_D;
      const int ncols = m.tile[t] >= 0 ? RD_TILE : 1;
      for (int c = par; c < ncols; c += 2) {
        const float2 vf = __half22float2(reinterpret_cast<const __half2*>(vt + c * ATT_D)[dp]);
        const float4 p = *reinterpret_cast<const float4*>(sc + (t * RD_TILE + c) * 4);
        acc[0][0] = fmaf(p.x, vf.x, acc[0][0]); acc[0][1] = fmaf(p.x, vf.y, acc[0][1]);
        acc[1][0] = fmaf(p.y, vf.x, acc[1][0]); acc[1][1] = fmaf(p.y, vf.y, acc[1][1]);
        acc[2][0] = fmaf(p.z, vf.x, acc[2][0]); acc[2][1] = fmaf(p.z, vf.y, acc[2][1]);
        acc[3][0] = fmaf(p.w, vf.x, acc[3][0]); acc[3][1] = fmaf(p.w, vf.y, acc[3][1]);
      }
      mbar_arrive(&empty[s]);
    }
    if (par == 1) {
#pragma unroll
      for (int r = 0; r < ATT_G; ++r) {
        xacc[r * ATT_D + 2 * dp] = acc[r][0];
        xacc[r * ATT_D + 2 * dp + 1] = acc[r][1];
      }
    }
    if (!named_sync_and<RD_CONS>(ok)) break;
    if (par == 0 && args.out_raw) {
      // isolated kernel: ungated fp32 output [n][2][4][256]
#pragma unroll
      for (int r = 0; r < ATT_G; ++r) {
        const float l = lsum[r];
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        float* o = args.out_raw + (((size_t)n * ATT_HKV + h) * ATT_G + r) * ATT_D + 2 * dp;
        o[0] = (acc[r][0] + xacc[r * ATT_D + 2 * dp]) * inv;
        o[1] = (acc[r][1] + xacc[r * ATT_D + 2 * dp + 1]) * inv;
      }
    } else if (par == 0) {
      const float* gate_row = args.proj + (size_t)n * ATT_IN;
#pragma unroll
      for (int r = 0; r < ATT_G; ++r) {
        const int jq = h * ATT_G + r;
        const float l = lsum[r];
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        const float a0 = (acc[r][0] + xacc[r * ATT_D + 2 * dp]) * inv;
        const float a1 = (acc[r][1] + xacc[r * ATT_D + 2 * dp + 1]) * inv;
        const float* g = gate_row + jq * 2 * ATT_D + ATT_D + 2 * dp;
        const float y0 = a0 * sigmoidf_(g[0]), y1 = a1 * sigmoidf_(g[1]);
        __nv_bfloat16 hv[2], lv[2];
        split_bf16(y0, hv[0], lv[0]);
        split_bf16(y1, hv[1], lv[1]);
        *reinterpret_cast<__nv_bfloat162*>(ohi + r * ATT_D + 2 * dp) = *reinterpret_cast<__nv_bfloat162*>(hv);
        *reinterpret_cast<__nv_bfloat162*>(olo + r * ATT_D + 2 * dp) = *reinterpret_cast<__nv_bfloat162*>(lv);
      }
    } else if (args.write_ring) {
      // par 1 threads: the new key/value go into ring column start % 512 (every copy of this item has landed)
      const int64_t slot = args.slots[n];
      const size_t col = (size_t)(qpos % WIN);
      const size_t dst = (((size_t)slot * ATT_HKV + h) * RING_COLS + col) * ATT_D + 2 * dp;
      const size_t src = ((size_t)n * ATT_HKV + h) * ATT_D + 2 * dp;
      *reinterpret_cast<__half2*>(args.ring_k + dst) = *reinterpret_cast<const __half2*>(args.knew + src);
      *reinterpret_cast<__half2*>(args.ring_v + dst) = *reinterpret_cast<const __half2*>(args.vnew + src);
    }
    mbar_arrive(&meta_free[b]);
    named_sync<RD_CONS>();  // scores and partial sums are reused by the next item
  }
}

}  // namespace hsg
