// Router: OffloadDeepseekV4MoE._route (deepseek_v4.py:118-148).
//   phase 1: fp32 logits = float(x) @ gate_w^T, gate rows staged in shared
//            memory, one warp per dot product (deterministic);
//   phase 2: one warp per token: score function,
//            biased top-k (or hash table), unbiased weights, renormalise,
//            scale.
#include <mutex>
#include <string>

#include "capi_internal.h"
#include "common.cuh"

namespace dsv4 {

constexpr int RT_MAX_E = 256;
constexpr int RT_TOK = 256;   // tokens per CTA (grid y)

// logits[t, e] = sum_h float(x[t, h]) * w[e, h].  A CTA keeps EPB gate rows in
// shared memory; each warp takes whole (token, expert-group) dot products,
// lanes stride H in 4-element steps, then a fixed butterfly reduction: one
// writer per logit, so the result is deterministic.
template <int EPB>
__global__ __launch_bounds__(256) void route_logits_kernel(const uint16_t* __restrict__ x,
                                                           const float* __restrict__ w, float* __restrict__ logits,
                                                           int64_t T, int H, int E) {
  extern __shared__ float ws[];  // [EPB][H]
  const int e0 = blockIdx.x * EPB;
  for (int i = threadIdx.x * 4; i < EPB * H; i += blockDim.x * 4) {
    const int r = i / H, c = i - r * H;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e0 + r < E) v = *reinterpret_cast<const float4*>(w + (int64_t)(e0 + r) * H + c);
    *reinterpret_cast<float4*>(ws + i) = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t_end = min(T, (int64_t)(blockIdx.y + 1) * RT_TOK);
  for (int64_t t = (int64_t)blockIdx.y * RT_TOK + warp; t < t_end; t += blockDim.x >> 5) {
    float acc[EPB];
#pragma unroll
    for (int j = 0; j < EPB; ++j) acc[j] = 0.f;
    const uint16_t* xr = x + t * H;
    for (int h = lane * 4; h < H; h += 128) {
      const uint2 raw = *reinterpret_cast<const uint2*>(xr + h);
      const float a0 = bf16_from_bits(raw.x & 0xffffu), a1 = bf16_from_bits(raw.x >> 16);
      const float a2 = bf16_from_bits(raw.y & 0xffffu), a3 = bf16_from_bits(raw.y >> 16);
#pragma unroll
      for (int j = 0; j < EPB; ++j) {
        const float4 g = *reinterpret_cast<const float4*>(ws + j * H + h);
        acc[j] = fmaf(a0, g.x, acc[j]);
        acc[j] = fmaf(a1, g.y, acc[j]);
        acc[j] = fmaf(a2, g.z, acc[j]);
        acc[j] = fmaf(a3, g.w, acc[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < EPB; ++j) {
      float v = acc[j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && e0 + j < E) logits[t * E + e0 + j] = v;
    }
  }
}

__device__ __forceinline__ float softplus_f(float v) { return v > 20.f ? v : log1pf(expf(v)); }

__global__ __launch_bounds__(256) void route_topk_kernel(const float* __restrict__ logits, int64_t T,
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
    sc[j] = (e < E) ? logits[t * E + e] : -INFINITY;
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
  return n_tokens * n_experts * (int64_t)sizeof(float);
}

extern "C" int dsv4_route_topk(const void* x_bf16, const float* gate_w, const float* bias, const int32_t* tid2eid,
                               const int64_t* input_ids, int64_t n_tokens, int32_t hidden, int32_t n_experts,
                               int32_t topk, int32_t score_func, int32_t renormalize, float route_scale,
                               float* weights_out, int32_t* indices_out, void* workspace, int64_t workspace_bytes,
                               void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16 && gate_w && weights_out && indices_out && workspace, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && hidden % 128 == 0 && hidden <= 6144, "hidden must be a multiple of 128, <= 6144");
  DSV4_CHECK_ARG(n_experts > 0 && n_experts <= RT_MAX_E, "n_experts must be in [1, 256]");
  DSV4_CHECK_ARG(topk > 0 && topk <= 16 && topk <= n_experts, "topk must be in [1, min(16, n_experts)]");
  DSV4_CHECK_ARG(score_func >= 0 && score_func <= 2, "unknown score function");
  DSV4_CHECK_ARG(!tid2eid || input_ids, "hash routing needs input_ids");
  DSV4_CHECK_ARG(workspace_bytes >= dsv4_route_workspace_bytes(n_tokens, hidden, n_experts),
                 "workspace too small");
  if (n_tokens == 0) return DSV4_OK;
  if (int rc = bind_device_of(x_bf16, nullptr)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned gy = (unsigned)((n_tokens + RT_TOK - 1) / RT_TOK);
  if (n_tokens <= 512) {  // decode: 2 gate rows per CTA, E/2 CTAs
    const size_t smem = (size_t)2 * hidden * sizeof(float);
    DSV4_CUDA_CHECK(cudaFuncSetAttribute(route_logits_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    route_logits_kernel<2><<<dim3((n_experts + 1) / 2, gy), 256, smem, st>>>(
        (const uint16_t*)x_bf16, gate_w, (float*)workspace, n_tokens, hidden, n_experts);
  } else {  // prefill: 8 gate rows per CTA so x is re-read E/8 times
    const size_t smem = (size_t)8 * hidden * sizeof(float);
    DSV4_CUDA_CHECK(cudaFuncSetAttribute(route_logits_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    route_logits_kernel<8><<<dim3((n_experts + 7) / 8, gy), 256, smem, st>>>(
        (const uint16_t*)x_bf16, gate_w, (float*)workspace, n_tokens, hidden, n_experts);
  }
  const int64_t threads = n_tokens * 32;
  route_topk_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      (const float*)workspace, n_tokens, n_experts, topk, score_func, renormalize, route_scale, bias, tid2eid,
      input_ids, weights_out, indices_out);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

// ---------------------------------------------------------------------------
// Router variant that allocates nothing.
//
// Some callers cannot allocate device memory when they route a batch: a
// serving engine that has handed nearly all free HBM to its pre-sized cache
// pool has no room left for a new cudaMalloc in the middle of a step, and a
// plain C caller bound through an FFI may have no device allocator at all.
// For them the logits scratch of the router lives in this fixed file-scope
// device array instead of a caller workspace.  Limits and rules:
//   * at most DSV4_ROUTE_NOALLOC_MAX_LOGITS (n_tokens * n_experts) logits,
//     256 KiB of device memory that every GPU loading the library keeps
//     until the process exits; larger calls are rejected with DSV4_EINVAL;
//   * the first call on a device looks up the array's device address on
//     that device (cudaGetSymbolAddress); make that first call before any
//     stream capture;
//   * all calls share the one array and it keeps the last call's logits;
//     the logits kernel writes every element the top-k kernel then reads, so
//     nothing needs clearing, but calls that overlap on the GPU (on different
//     streams, or from several threads) race on it.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_route_noalloc_scratch[DSV4_ROUTE_NOALLOC_MAX_LOGITS];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {};
}  // namespace

extern "C" int dsv4_route_topk_noalloc(const void* x_bf16, const float* gate_w, const float* bias,
                                       const int32_t* tid2eid, const int64_t* input_ids, int64_t n_tokens,
                                       int32_t hidden, int32_t n_experts, int32_t topk, int32_t score_func,
                                       int32_t renormalize, float route_scale, float* weights_out,
                                       int32_t* indices_out, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16 && gate_w && weights_out && indices_out, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && hidden % 128 == 0 && hidden <= 6144, "hidden must be a multiple of 128, <= 6144");
  DSV4_CHECK_ARG(n_experts > 0 && n_experts <= RT_MAX_E, "n_experts must be in [1, 256]");
  DSV4_CHECK_ARG(topk > 0 && topk <= 16 && topk <= n_experts, "topk must be in [1, min(16, n_experts)]");
  DSV4_CHECK_ARG(score_func >= 0 && score_func <= 2, "unknown score function");
  DSV4_CHECK_ARG(!tid2eid || input_ids, "hash routing needs input_ids");
  DSV4_CHECK_ARG(n_tokens >= 0 && n_tokens * (int64_t)n_experts <= DSV4_ROUTE_NOALLOC_MAX_LOGITS,
                 "n_tokens * n_experts exceeds the fixed scratch of " +
                     std::to_string(DSV4_ROUTE_NOALLOC_MAX_LOGITS) +
                     " logits; use dsv4_route_topk with a caller workspace");
  if (n_tokens == 0) return DSV4_OK;
  int dev = 0;
  if (int rc = bind_device_of(x_bf16, &dev)) return rc;
  DSV4_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "device ordinal out of range");
  float* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      // set-up, once per device, with that device current (bind_device_of)
      void* p = nullptr;
      DSV4_CUDA_CHECK(cudaGetSymbolAddress(&p, g_route_noalloc_scratch));
      g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    scratch = g_noalloc_ptr[dev];
  }
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned gy = (unsigned)((n_tokens + RT_TOK - 1) / RT_TOK);
  if (n_tokens <= 512) {
    const size_t smem = (size_t)2 * hidden * sizeof(float);
    DSV4_CUDA_CHECK(cudaFuncSetAttribute(route_logits_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    route_logits_kernel<2><<<dim3((n_experts + 1) / 2, gy), 256, smem, st>>>(
        (const uint16_t*)x_bf16, gate_w, scratch, n_tokens, hidden, n_experts);
  } else {
    const size_t smem = (size_t)8 * hidden * sizeof(float);
    DSV4_CUDA_CHECK(cudaFuncSetAttribute(route_logits_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    route_logits_kernel<8><<<dim3((n_experts + 7) / 8, gy), 256, smem, st>>>(
        (const uint16_t*)x_bf16, gate_w, scratch, n_tokens, hidden, n_experts);
  }
  const int64_t threads = n_tokens * 32;
  route_topk_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      scratch, n_tokens, n_experts, topk, score_func, renormalize, route_scale, bias, tid2eid, input_ids,
      weights_out, indices_out);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}
