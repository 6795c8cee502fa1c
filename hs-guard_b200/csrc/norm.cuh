// Row-wise kernels around the GEMMs: embedding gather + RMSNorm, residual RMSNorm, and the classifier heads.
//
// The residual stream is kept in fp32 ([tokens, 1024]); the out_proj / o_proj / down_proj GEMMs accumulate straight
// into it. Every RMSNorm (Qwen3_5RMSNorm: x * rsqrt(mean(x^2) + eps) * (1 + w), reference
// transformers modeling_qwen3_5.py Qwen3_5RMSNorm, engine/fused_kernels.py:56-72) writes the next GEMM's activation
// operand as a bf16 hi/lo pair. Rows in [m, m_pad) are zero-filled so the padded GEMM tiles read clean data.
#pragma once
#include "common.cuh"

namespace hsg {

constexpr int NORM_THREADS = 256;  // 4 elements of the 1024-wide row per thread

// hidden[m] = float(embed[ids[m]]) (row m < m_valid), then RMSNorm -> (x_hi, x_lo).
__global__ void __launch_bounds__(NORM_THREADS) embed_norm_kernel(const int64_t* ids, const __nv_bfloat16* embed,
                                                                  int vocab, const float* w1, float eps,
                                                                  float* hidden, __nv_bfloat16* x_hi,
                                                                  __nv_bfloat16* x_lo, int m_valid, int* err) {
  pdl_wait();
  pdl_trigger();
  __shared__ float scratch[NORM_THREADS / 32];
  const int m = blockIdx.x, d = threadIdx.x * 4;
  float x[4] = {0.f, 0.f, 0.f, 0.f};
  if (m < m_valid) {
    int64_t id = ids[m];
    if (id < 0 || id >= vocab) {
      if (threadIdx.x == 0) set_error(err, ERR_BAD_TOKEN);
      id = 0;
    }
    const uint2 raw = *reinterpret_cast<const uint2*>(embed + (size_t)id * HIDDEN + d);
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 a = __bfloat1622float2(p[0]), b = __bfloat1622float2(p[1]);
    x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
  }
  *reinterpret_cast<float4*>(hidden + (size_t)m * HIDDEN + d) = make_float4(x[0], x[1], x[2], x[3]);
  const float ss = block_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3], scratch, NORM_THREADS);
  const float r = 1.0f / sqrtf(ss * (1.0f / HIDDEN) + eps);
  const float4 w = *reinterpret_cast<const float4*>(w1 + d);
  const float y[4] = {x[0] * r * w.x, x[1] * r * w.y, x[2] * r * w.z, x[3] * r * w.w};
  __nv_bfloat16 hi[4], lo[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) split_bf16(m < m_valid ? y[j] : 0.f, hi[j], lo[j]);
  *reinterpret_cast<uint2*>(x_hi + (size_t)m * HIDDEN + d) = *reinterpret_cast<uint2*>(hi);
  *reinterpret_cast<uint2*>(x_lo + (size_t)m * HIDDEN + d) = *reinterpret_cast<uint2*>(lo);
}

// (x_hi, x_lo)[m] = RMSNorm(hidden[m]) * w1 for m < m_valid; zeros for padded rows.
__global__ void __launch_bounds__(NORM_THREADS) resid_norm_kernel(const float* hidden, const float* w1, float eps,
                                                                  __nv_bfloat16* x_hi, __nv_bfloat16* x_lo,
                                                                  int m_valid) {
  pdl_wait();
  pdl_trigger();
  __shared__ float scratch[NORM_THREADS / 32];
  const int m = blockIdx.x, d = threadIdx.x * 4;
  float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
  if (m < m_valid) x = *reinterpret_cast<const float4*>(hidden + (size_t)m * HIDDEN + d);
  const float4 w = *reinterpret_cast<const float4*>(w1 + d);  // requested before the reduction's barriers
  const float ss = block_sum(x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w, scratch, NORM_THREADS);
  const float r = m < m_valid ? 1.0f / sqrtf(ss * (1.0f / HIDDEN) + eps) : 0.f;
  __nv_bfloat162 hi[2], lo[2];
  split_bf16x2(x.x * r * w.x, x.y * r * w.y, hi[0], lo[0]);
  split_bf16x2(x.z * r * w.z, x.w * r * w.w, hi[1], lo[1]);
  *reinterpret_cast<uint2*>(x_hi + (size_t)m * HIDDEN + d) = *reinterpret_cast<uint2*>(hi);
  *reinterpret_cast<uint2*>(x_lo + (size_t)m * HIDDEN + d) = *reinterpret_cast<uint2*>(lo);
}

// Role heads after the first Linear (done on the tensor cores into hbuf [tokens, 2*512]):
//   x = hbuf + b1 -> LayerNorm(512, eps) (w, b) -> SiLU -> logits = W2 x + b2 (3 classes) -> softmax
// (reference runtime.py:54-75 readout; engine/slot_engine_v7.py:58-61). probs layout [role][token][3].
// One CTA per token, 128 threads per role.
__global__ void __launch_bounds__(256) head_finish_kernel(const float* hbuf, const float* b1, const float* ln_w,
                                                          const float* ln_b, const float* w2, const float* b2,
                                                          float eps, float* probs, int m_valid) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8][4];
  const int m = blockIdx.x, role = threadIdx.x >> 7, t = threadIdx.x & 127;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wr = warp & 3;
  const int e0 = role * HEAD_E + t * 4;
  float4 x = *reinterpret_cast<const float4*>(hbuf + (size_t)m * (N_ROLES * HEAD_E) + e0);
  const float4 bb = *reinterpret_cast<const float4*>(b1 + e0);
  // the LayerNorm and classifier weights too, ahead of the reductions' barriers
  const float4 lw = *reinterpret_cast<const float4*>(ln_w + e0), lb = *reinterpret_cast<const float4*>(ln_b + e0);
  float4 w2r[N_CLS];
#pragma unroll
  for (int c = 0; c < N_CLS; ++c) w2r[c] = *reinterpret_cast<const float4*>(w2 + ((size_t)role * N_CLS + c) * HEAD_E + t * 4);
  x.x += bb.x; x.y += bb.y; x.z += bb.z; x.w += bb.w;
  // mean
  float s = warp_sum(x.x + x.y + x.z + x.w);
  if (lane == 0) red[warp][0] = s;
  __syncthreads();
  const float mean = (red[role * 4][0] + red[role * 4 + 1][0] + red[role * 4 + 2][0] + red[role * 4 + 3][0]) *
                     (1.0f / HEAD_E);
  const float d0 = x.x - mean, d1 = x.y - mean, d2 = x.z - mean, d3 = x.w - mean;
  s = warp_sum(d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3);
  if (lane == 0) red[warp][1] = s;
  __syncthreads();
  const float var = (red[role * 4][1] + red[role * 4 + 1][1] + red[role * 4 + 2][1] + red[role * 4 + 3][1]) *
                    (1.0f / HEAD_E);
  const float r = 1.0f / sqrtf(var + eps);
  const float y[4] = {silu(d0 * r * lw.x + lb.x), silu(d1 * r * lw.y + lb.y), silu(d2 * r * lw.z + lb.z),
                      silu(d3 * r * lw.w + lb.w)};
  float logit[N_CLS];
#pragma unroll
  for (int c = 0; c < N_CLS; ++c) {
    const float4 w = w2r[c];
    logit[c] = warp_sum(y[0] * w.x + y[1] * w.y + y[2] * w.z + y[3] * w.w);
  }
  if (lane == 0) { red[warp][2] = logit[0]; red[warp][3] = logit[1]; }
  __syncthreads();
  float l0 = red[role * 4][2] + red[role * 4 + 1][2] + red[role * 4 + 2][2] + red[role * 4 + 3][2];
  float l1 = red[role * 4][3] + red[role * 4 + 1][3] + red[role * 4 + 2][3] + red[role * 4 + 3][3];
  __syncthreads();
  if (lane == 0) red[warp][0] = logit[2];
  __syncthreads();
  float l2 = red[role * 4][0] + red[role * 4 + 1][0] + red[role * 4 + 2][0] + red[role * 4 + 3][0];
  if (t == 0 && m < m_valid) {
    l0 += b2[role * N_CLS]; l1 += b2[role * N_CLS + 1]; l2 += b2[role * N_CLS + 2];
    const float mx = fmaxf(l0, fmaxf(l1, l2));
    const float e0_ = expf(l0 - mx), e1_ = expf(l1 - mx), e2_ = expf(l2 - mx);
    const float inv = 1.0f / (e0_ + e1_ + e2_);
    float* p = probs + ((size_t)role * m_valid + m) * N_CLS;
    p[0] = e0_ * inv; p[1] = e1_ * inv; p[2] = e2_ * inv;
  }
  (void)wr;
}

}  // namespace hsg
