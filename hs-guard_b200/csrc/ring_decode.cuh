// Single-token ring-window attention decode (1-token ticks): a persistent, warp-specialised TMA pipeline whose score
// and P.V products run on the tensor cores (sm_100a).
//
// Work item = (session row n, kv head h): the 4 query heads of group h attend over the slot's ring (up to 512 keys)
// plus the tick's own key. Grid = one CTA per SM; items are dealt round-robin.
//
// Producer warp: per item it reads the slot's ring positions, lists the 32-column tiles holding any filled column
// plus the new-key tile, publishes the list (with every key's position) in a double-buffered metadata block, then
// streams the K tiles and after them the V tiles through an 11-stage ring. A tile is 32 keys x 256 dims fp16 (16 KB),
// loaded as four [32 x 64] boxes by 2-D TMA with 128-byte swizzle, so the tensor-core fragment loads below are free
// of shared-memory bank conflicts.
// Consumer warps (8) -- warp-level MMA (mma.sync m16n8k16, fp16 in, fp32 accumulate); the 4 query rows sit in an
// 8-row operand whose other rows are zero:
//   pass 1: S^T[keys x rows] = K_tile[keys x dims] Q^T; warp w takes key half w & 1 and dims 64(w>>1)..+63, and adds
//           its partial dot products into its own slice of a score buffer (no barrier per tile);
//   softmax: per query row over all listed keys, masked by 0 <= kpos <= qpos, kpos > qpos - 512 (fp32);
//   pass 2: O^T[dims x rows] += V_tile^T[dims x keys] P^T; warp w owns dims 32w..32w+31.
// Stages are released by mbarrier arrivals. Output: out * sigmoid(gate) as the o_proj operand (bf16 hi/lo), or the
// ungated fp32 output for the isolated kernel; then the new key/value are written into ring column start % 512 (the
// position held there, start - 512, is outside this query's window).
// Same contract as ring_attn_kernel (reference engine/fused_kernels.py:288-376 for Lb = 1).
#pragma once
#include "attn.cuh"

namespace hsg {

constexpr int RD_CONS = 256;                     // consumer threads
constexpr int RD_THREADS = RD_CONS + 32;         // + producer warp
constexpr int RD_TILE = 32;                      // keys per tile
constexpr int RD_TILE_BYTES = RD_TILE * ATT_D * 2;
constexpr int RD_SUB_BYTES = RD_TILE * 64 * 2;   // one [32 keys x 64 dims] swizzled box
constexpr int RD_STAGES = 11;                   // 176 KB in flight per SM (the most that fits)
constexpr int RD_MAXT = WIN / RD_TILE + 1;       // 16 ring tiles + the new-key tile
constexpr int RD_MAXK = RD_MAXT * RD_TILE;
constexpr int RD_PSTRIDE = RD_MAXK + 8;          // fp16 probabilities row stride (bank-spread)

struct alignas(16) RdMeta {
  int64_t qpos;
  int64_t slot;
  int len, ntile;
  int tile[RD_MAXT];      // ring tile index, or -1 for the new-key tile
  int kpos[RD_MAXK];      // key position per listed tile column (-1: not visible)
};

__host__ __device__ inline int rd_smem_bytes() {
  // stages | meta x2 | partial scores [4][MAXK][4] f32 | probabilities [4][PSTRIDE] f16 | row sums and maxima
  // [2][4] each | barriers
  return RD_STAGES * RD_TILE_BYTES + 2 * (int)sizeof(RdMeta) + 4 * RD_MAXK * 4 * 4 + 4 * RD_PSTRIDE * 2 + 64 +
         (2 * RD_STAGES + 4) * 8 + 1024;
}

// tm_rk / tm_rv: this layer's ring K / V as 2-D [rows = (slot*2 + head)*513 + column][256] fp16;
// tm_nk / tm_nv: the tick's new keys / values as [rows = row*2 + head][256] fp16. All with [64 x 32] boxes, SW128.
__global__ void __launch_bounds__(RD_THREADS, 1)
ring_decode_kernel(const __grid_constant__ CUtensorMap tm_rk, const __grid_constant__ CUtensorMap tm_rv,
                   const __grid_constant__ CUtensorMap tm_nk, const __grid_constant__ CUtensorMap tm_nv,
                   const AttnArgs args) {
  extern __shared__ __align__(1024) uint8_t rd_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rd_smem_raw) + 1023) & ~uintptr_t(1023));
  RdMeta* meta = reinterpret_cast<RdMeta*>(smem + RD_STAGES * RD_TILE_BYTES);
  float* scp = reinterpret_cast<float*>(meta + 2);             // [4 dim ranges][MAXK][4 rows] partial scores
  __half* pr = reinterpret_cast<__half*>(scp + 4 * RD_MAXK * 4);  // [4 rows][PSTRIDE] probabilities
  float* lsum = reinterpret_cast<float*>(pr + 4 * RD_PSTRIDE);    // [2 key halves][4 rows] sums
  float* smax = lsum + 8;                                         // [2 key halves][4 rows] maxima
  uint64_t* full = reinterpret_cast<uint64_t*>(smax + 8);       // [RD_STAGES]
  uint64_t* empty = full + RD_STAGES;                           // [RD_STAGES]
  uint64_t* meta_full = empty + RD_STAGES;                      // [2]
  uint64_t* meta_free = meta_full + 2;                          // [2]

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
    prefetch_tmap(&tm_rk);
    prefetch_tmap(&tm_rv);
    prefetch_tmap(&tm_nk);
    prefetch_tmap(&tm_nv);
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
        mbar_arrive(&meta_full[b]);
      }
      __syncwarp();
      if (len == 0) continue;
      const int ring_row = (int)((slot * ATT_HKV + h) * RING_COLS);
      const int new_row = n * ATT_HKV + h;
      for (int pass = 0; pass < 2; ++pass) {
        const CUtensorMap* ring = pass == 0 ? &tm_rk : &tm_rv;
        const CUtensorMap* fresh = pass == 0 ? &tm_nk : &tm_nv;
        for (int t = 0; t < nt; ++t, ++cnt) {
          const int s = cnt % RD_STAGES;
          if (cnt >= RD_STAGES && !mbar_wait(&empty[s], ((cnt / RD_STAGES) - 1) & 1, args.err, ERR_TIMEOUT_TMA))
            return;
          if (lane == 0) {
            const int tile = m.tile[t];
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
    }
    return;
  }

  // ===================================== consumers =====================================
  const int g = lane >> 2, c4 = lane & 3;     // mma fragment coordinates
  const int kh = warp & 1, kr = warp >> 1;    // pass 1: key half of the tile, dim range
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
    // the output gates of this lane's (row, dim) outputs, loaded now so the latency hides behind both passes
    // this item's new key / value pair for the ring write at its end, loaded now (a load issued after the output
    // stores could not be moved ahead of them and would add a memory round trip to every item)
    __half2 nk2 = __floats2half2_rn(0.f, 0.f), nv2 = nk2;
    if (args.write_ring && tid < ATT_D / 2) {
      const size_t src = ((size_t)n * ATT_HKV + h) * ATT_D + 2 * tid;
      nk2 = *reinterpret_cast<const __half2*>(args.knew + src);
      nv2 = *reinterpret_cast<const __half2*>(args.vnew + src);
    }
    float gate[2][2][2] = {};
    if (!args.out_raw && c4 < 2) {
#pragma unroll
      for (int mb = 0; mb < 2; ++mb)
#pragma unroll
        for (int half = 0; half < 2; ++half)
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int dim = 32 * warp + 16 * mb + g + 8 * half, jq = h * ATT_G + 2 * c4 + cc;
            gate[mb][half][cc] = args.proj[(size_t)n * ATT_IN + jq * 2 * ATT_D + ATT_D + dim];
          }
    }
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
    float* sp = scp + (size_t)kr * RD_MAXK * 4;
    // ---- pass 1: partial scores over this warp's dim range ----
    for (int t = 0; t < nt && ok; ++t, ++cnt) {
      const int s = cnt % RD_STAGES;
      if (!mbar_wait(&full[s], (cnt / RD_STAGES) & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
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
        const int key = t * RD_TILE + 16 * kh + g;
        *reinterpret_cast<float2*>(sp + key * 4 + 2 * c4) = make_float2(d[0], d[1]);
        *reinterpret_cast<float2*>(sp + (key + 8) * 4 + 2 * c4) = make_float2(d[2], d[3]);
      }
    }
    if (!named_sync_and<RD_CONS>(ok)) break;
    // ---- softmax per query row r: warps r and r + 4 take alternate 32-key tiles (sum the four dim ranges, mask);
    // the two halves' maxima and sums meet in shared memory ----
    {
      const int r = warp & 3, hf = warp >> 2, nk = nt * RD_TILE;
      float mx = -INFINITY;
#pragma unroll 4
      for (int c = hf * RD_TILE + lane; c < nk; c += 2 * RD_TILE) {
        const int kp = m.kpos[c];
        float sc = -INFINITY;
        if (kp >= 0 && kp <= qpos && kp > qpos - WIN)
          sc = (scp[c * 4 + r] + scp[(RD_MAXK + c) * 4 + r] + scp[(2 * RD_MAXK + c) * 4 + r] +
                scp[(3 * RD_MAXK + c) * 4 + r]) * args.scale;
        scp[c * 4 + r] = sc;
        mx = fmaxf(mx, sc);
      }
      mx = warp_max(mx);
      if (lane == 0) smax[hf * 4 + r] = mx;
      named_sync<RD_CONS>();
      mx = fmaxf(smax[r], smax[4 + r]);
      const float msafe = mx == -INFINITY ? 0.f : mx;
      float sum = 0.f;
#pragma unroll 4
      for (int c = hf * RD_TILE + lane; c < nk; c += 2 * RD_TILE) {
        const float p = __expf(scp[c * 4 + r] - msafe);  // rounded to fp16 below
        pr[r * RD_PSTRIDE + c] = __float2half_rn(p);
        sum += p;
      }
      sum = warp_sum(sum);
      if (lane == 0) lsum[hf * 4 + r] = sum;
    }
    named_sync<RD_CONS>();
    // ---- pass 2: O^T[dims 32w..32w+31] += V^T P^T ----
    float o[2][4];
#pragma unroll
    for (int mb = 0; mb < 2; ++mb) o[mb][0] = o[mb][1] = o[mb][2] = o[mb][3] = 0.f;
    const int dsub = warp >> 1;              // the 64-dim box holding dims 32w..32w+31
    const int cbase = (warp & 1) * 4;        // first 16-byte chunk of those dims inside the box
    for (int t = 0; t < nt && ok; ++t, ++cnt) {
      const int s = cnt % RD_STAGES;
      if (!mbar_wait(&full[s], (cnt / RD_STAGES) & 1, args.err, ERR_TIMEOUT_TMA)) { ok = false; break; }
      const uint32_t sub = smem_u32(smem + (size_t)s * RD_TILE_BYTES + dsub * RD_SUB_BYTES);
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {   // 16 keys per k-step
        // B = P^T[keys][rows]: fragment column g = query row (rows >= 4 zero)
        const int kc = t * RD_TILE + 16 * ks + 2 * c4;
        const uint32_t b0 = g < ATT_G ? *reinterpret_cast<const uint32_t*>(pr + (g & 3) * RD_PSTRIDE + kc) : 0u;
        const uint32_t b1 = g < ATT_G ? *reinterpret_cast<const uint32_t*>(pr + (g & 3) * RD_PSTRIDE + kc + 8) : 0u;
#pragma unroll
        for (int mb = 0; mb < 2; ++mb) {
          // A = V^T[dims 16mb..+15][keys 16ks..+15] via transposed loads of the stored [key][dim] blocks:
          // matrix mi: keys +8*(mi>>1), dim chunk +(mi&1)
          const int mi = lane >> 3, r = 16 * ks + (mi >> 1) * 8 + (lane & 7), ch = cbase + 2 * mb + (mi & 1);
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4_trans(sub + sw128_off(r, ch), a0, a1, a2, a3);
          mma_f16_16816(o[mb], a0, a1, a2, a3, b0, b1);
        }
      }
      mbar_arrive(&empty[s]);
    }
    if (!named_sync_and<RD_CONS>(ok)) break;
    // ---- output: lanes with c4 < 2 hold query rows 2*c4, 2*c4+1 for dims 32w + 16mb + g (+8) ----
    if (c4 < 2) {
#pragma unroll
      for (int mb = 0; mb < 2; ++mb) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int dim = 32 * warp + 16 * mb + g + 8 * half;
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const int r = 2 * c4 + cc;
            const float l = lsum[r] + lsum[4 + r];
            const float val = l > 0.f ? o[mb][2 * half + cc] / l : 0.f;
            if (args.out_raw) {
              args.out_raw[(((size_t)n * ATT_HKV + h) * ATT_G + r) * ATT_D + dim] = val;
            } else {
              const float gt = gate[mb][half][cc];
              split_bf16(val * __fdividef(1.0f, 1.0f + __expf(-gt)), ohi[r * ATT_D + dim], olo[r * ATT_D + dim]);
            }
          }
        }
      }
    }
    if (args.write_ring && tid < ATT_D / 2) {
      // the new key/value go into ring column start % 512 (every copy of this item has landed)
      const size_t col = (size_t)(qpos % WIN);
      const size_t dst = (((size_t)m.slot * ATT_HKV + h) * RING_COLS + col) * ATT_D + 2 * tid;
      *reinterpret_cast<__half2*>(args.ring_k + dst) = nk2;
      *reinterpret_cast<__half2*>(args.ring_v + dst) = nv2;
    }
    mbar_arrive(&meta_free[b]);
    named_sync<RD_CONS>();  // scores and probabilities are reused by the next item
  }
}

}  // namespace hsg
