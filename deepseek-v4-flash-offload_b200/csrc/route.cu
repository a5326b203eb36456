// Router: OffloadDeepseekV4MoE._route (deepseek_v4.py:118-148).
//   phase 1: fp32 logits = float(x) @ gate_w^T, tiled through shared memory,
//            split along H into fixed chunks (deterministic partial sums);
//   phase 2: one warp per token: sum the chunks in order, score function,
//            biased top-k (or hash table), unbiased weights, renormalise,
//            scale.
#include "capi_internal.h"
#include "common.cuh"

namespace dsv4 {

constexpr int RT_T = 16;    // tokens per tile
constexpr int RT_E = 32;    // experts per tile
constexpr int RT_H = 128;   // hidden chunk
constexpr int RT_PAD = RT_H + 1;
constexpr int RT_MAX_E = 256;

__global__ __launch_bounds__(256) void route_logits_kernel(const uint16_t* __restrict__ x,
                                                           const float* __restrict__ w, float* __restrict__ part,
                                                           int64_t T, int H, int E) {
  __shared__ float xs[RT_T][RT_PAD];
  __shared__ float ws[RT_E][RT_PAD];
  const int e0 = blockIdx.x * RT_E;
  const int64_t t0 = (int64_t)blockIdx.y * RT_T;
  const int h0 = blockIdx.z * RT_H;
  const int tid = threadIdx.x;
  // x tile: 16 x 256 bf16 -> f32
  for (int i = tid; i < RT_T * RT_H / 2; i += 256) {
    const int r = i / (RT_H / 2), c = (i % (RT_H / 2)) * 2;
    float a = 0.f, b = 0.f;
    if (t0 + r < T) {
      const uint32_t v = *reinterpret_cast<const uint32_t*>(x + (t0 + r) * H + h0 + c);
      a = bf16_from_bits(v & 0xffffu);
      b = bf16_from_bits(v >> 16);
    }
    xs[r][c] = a;
    xs[r][c + 1] = b;
  }
  // gate tile: 32 x 256 f32
  for (int i = tid; i < RT_E * RT_H / 4; i += 256) {
    const int r = i / (RT_H / 4), c = (i % (RT_H / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e0 + r < E) v = *reinterpret_cast<const float4*>(w + (int64_t)(e0 + r) * H + h0 + c);
    ws[r][c] = v.x;
    ws[r][c + 1] = v.y;
    ws[r][c + 2] = v.z;
    ws[r][c + 3] = v.w;
  }
  __syncthreads();
  const int el = tid >> 3, tp = (tid & 7) * 2;
  float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
  for (int h = 0; h < RT_H; ++h) {
    const float wv = ws[el][h];
    a0 = fmaf(xs[tp][h], wv, a0);
    a1 = fmaf(xs[tp + 1][h], wv, a1);
  }
  const int e = e0 + el;
  if (e < E) {
    float* dst = part + ((int64_t)blockIdx.z * T) * E;
    if (t0 + tp < T) dst[(t0 + tp) * E + e] = a0;
    if (t0 + tp + 1 < T) dst[(t0 + tp + 1) * E + e] = a1;
  }
}

__device__ __forceinline__ float softplus_f(float v) { return v > 20.f ? v : log1pf(expf(v)); }

__global__ __launch_bounds__(256) void route_topk_kernel(const float* __restrict__ part, int nchunks, int64_t T,
                                                         int E, int K, int score_func, int renorm, float scale,
                                                         const float* __restrict__ bias,
                                                         const int32_t* __restrict__ tid2eid,
                                                         const int64_t* __restrict__ ids, float* __restrict__ w_out,
                                                         int32_t* __restrict__ i_out) {
  constexpr int PER = RT_MAX_E / 32;
  const int lane = threadIdx.x & 31;
  const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  float sc[PER], ch[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    float l = 0.f;
    if (e < E)
      for (int c = 0; c < nchunks; ++c) l += part[((int64_t)c * T + t) * E + e];
    sc[j] = (e < E) ? l : -INFINITY;
  }
  if (score_func == DSV4_SCORE_SOFTMAX) {
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < PER; ++j) m = fmaxf(m, sc[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      sc[j] = (lane + 32 * j < E) ? expf(sc[j] - m) : 0.f;
      s += sc[j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
    for (int j = 0; j < PER; ++j) sc[j] = sc[j] / s;
  } else if (score_func == DSV4_SCORE_SIGMOID) {
#pragma unroll
    for (int j = 0; j < PER; ++j) sc[j] = 1.f / (1.f + expf(-sc[j]));
  } else {
#pragma unroll
    for (int j = 0; j < PER; ++j) sc[j] = sqrtf(softplus_f(sc[j]));
  }
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    ch[j] = (e < E) ? (bias ? sc[j] + bias[e] : sc[j]) : -INFINITY;
  }
  float wsel[16];
  int isel[16];
  for (int r = 0; r < K; ++r) {
    int pick;
    if (tid2eid) {
      pick = tid2eid[ids[t] * K + r];
    } else {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int e = lane + 32 * j;
        if (e < E && (ch[j] > bv || (ch[j] == bv && e < bi))) {
          bv = ch[j];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      pick = bi;
      if ((pick & 31) == lane) {
#pragma unroll
        for (int j = 0; j < PER; ++j)
          if (j == (pick >> 5)) ch[j] = -INFINITY;
      }
    }
    // unbiased score of the pick lives in lane pick%32, slot pick/32
    float v = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (j == (pick >> 5)) v = sc[j];
    v = __shfl_sync(0xffffffffu, v, pick & 31);
    wsel[r] = v;
    isel[r] = pick;
  }
  if (lane == 0) {
    float s = 0.f;
    for (int r = 0; r < K; ++r) s += wsel[r];
    for (int r = 0; r < K; ++r) {
      float v = renorm ? wsel[r] / s : wsel[r];
      w_out[t * K + r] = v * scale;
      i_out[t * K + r] = isel[r];
    }
  }
}

}  // namespace dsv4

using namespace dsv4;

extern "C" int64_t dsv4_route_workspace_bytes(int64_t n_tokens, int32_t hidden, int32_t n_experts) {
  if (n_tokens < 0 || hidden <= 0 || n_experts <= 0) return DSV4_EINVAL;
  return (int64_t)(hidden / RT_H) * n_tokens * n_experts * (int64_t)sizeof(float);
}

extern "C" int dsv4_route_topk(const void* x_bf16, const float* gate_w, const float* bias, const int32_t* tid2eid,
                               const int64_t* input_ids, int64_t n_tokens, int32_t hidden, int32_t n_experts,
                               int32_t topk, int32_t score_func, int32_t renormalize, float route_scale,
                               float* weights_out, int32_t* indices_out, void* workspace, int64_t workspace_bytes,
                               void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16 && gate_w && weights_out && indices_out && workspace, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && hidden % RT_H == 0, "hidden must be a positive multiple of 128");
  DSV4_CHECK_ARG(n_experts > 0 && n_experts <= RT_MAX_E, "n_experts must be in [1, 256]");
  DSV4_CHECK_ARG(topk > 0 && topk <= 16 && topk <= n_experts, "topk must be in [1, min(16, n_experts)]");
  DSV4_CHECK_ARG(score_func >= 0 && score_func <= 2, "unknown score function");
  DSV4_CHECK_ARG(!tid2eid || input_ids, "hash routing needs input_ids");
  DSV4_CHECK_ARG(workspace_bytes >= dsv4_route_workspace_bytes(n_tokens, hidden, n_experts),
                 "workspace too small");
  if (n_tokens == 0) return DSV4_OK;
  if (int rc = bind_device_of(x_bf16, nullptr)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const int nchunks = hidden / RT_H;
  dim3 g1((n_experts + RT_E - 1) / RT_E, (unsigned)((n_tokens + RT_T - 1) / RT_T), nchunks);
  route_logits_kernel<<<g1, 256, 0, st>>>((const uint16_t*)x_bf16, gate_w, (float*)workspace, n_tokens, hidden,
                                          n_experts);
  const int64_t threads = n_tokens * 32;
  route_topk_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      (const float*)workspace, nchunks, n_tokens, n_experts, topk, score_func, renormalize, route_scale, bias,
      tid2eid, input_ids, weights_out, indices_out);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}
