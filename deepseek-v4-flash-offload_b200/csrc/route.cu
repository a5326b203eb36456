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
constexpr int RT_EPB = 8;      // experts per CTA (one warp each)
constexpr int RT_TT = 64;      // tokens per CTA (two per lane)
constexpr int RT_KC = 64;      // K elements per shared-memory tile
constexpr int RT_SPLIT = 16;   // split of H on the workspace path; partials summed in order by the top-k kernel
constexpr int RT_SPLIT_NOALLOC = 4;  // split on the fixed-scratch path

// partial[c, t, e] = sum over H-chunk c of float(x[t, h]) * w[e, h].  Tiles of
// 64 tokens x 64 h (bf16 -> f32, padded rows) and 8 gate rows x 64 h are
// staged in shared memory; warp w owns expert e0 + w, lane owns tokens lane
// and lane + 32.  One writer per partial: deterministic.
__global__ __launch_bounds__(256) void route_logits_kernel(const uint16_t* __restrict__ x,
                                                           const float* __restrict__ w, float* __restrict__ part,
                                                           int64_t T, int H, int E, int split) {
  __shared__ float xs[RT_TT][RT_KC + 1];
  __shared__ float ws[RT_EPB][RT_KC];
  griddep_wait();
  griddep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.x * RT_EPB;
  const int chunk = blockIdx.y;
  const int64_t t0 = (int64_t)blockIdx.z * RT_TT;
  const int kc = H / split;
  const int kbeg = chunk * kc;
  float a0 = 0.f, a1 = 0.f;
  for (int k0 = kbeg; k0 < kbeg + kc; k0 += RT_KC) {
    for (int i = threadIdx.x; i < RT_TT * RT_KC / 2; i += 256) {
      const int r = i / (RT_KC / 2), c = (i % (RT_KC / 2)) * 2;
      float lo = 0.f, hi = 0.f;
      if (t0 + r < T) {
        const uint32_t v = *reinterpret_cast<const uint32_t*>(x + (t0 + r) * H + k0 + c);
        lo = bf16_from_bits(v & 0xffffu);
        hi = bf16_from_bits(v >> 16);
      }
      xs[r][c] = lo;
      xs[r][c + 1] = hi;
    }
    for (int i = threadIdx.x; i < RT_EPB * RT_KC; i += 256) {
      const int r = i / RT_KC, c = i % RT_KC;
      ws[r][c] = (e0 + r < E) ? w[(int64_t)(e0 + r) * H + k0 + c] : 0.f;
    }
    __syncthreads();
#pragma unroll 16
    for (int k = 0; k < RT_KC; ++k) {
      const float g = ws[warp][k];
      a0 = fmaf(xs[lane][k], g, a0);
      a1 = fmaf(xs[lane + 32][k], g, a1);
    }
    __syncthreads();
  }
  const int e = e0 + warp;
  if (e < E) {
    float* dst = part + (int64_t)chunk * T * E;
    if (t0 + lane < T) dst[(t0 + lane) * E + e] = a0;
    if (t0 + lane + 32 < T) dst[(t0 + lane + 32) * E + e] = a1;
  }
}

__device__ __forceinline__ float softplus_f(float v) { return v > 20.f ? v : log1pf(expf(v)); }

__global__ __launch_bounds__(256) void route_topk_kernel(const float* __restrict__ logits, int split, int64_t T,
                                                         int E, int K, int score_func, int renorm, float scale,
                                                         const float* __restrict__ bias,
                                                         const int32_t* __restrict__ tid2eid,
                                                         const int64_t* __restrict__ ids, float* __restrict__ w_out,
                                                         int32_t* __restrict__ i_out) {
  constexpr int PER = RT_MAX_E / 32;
  griddep_wait();
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  float sc[PER], ch[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    float l = 0.f;
    if (e < E) {
      // partial sums of the H chunks, loaded together, added in chunk order
      float v[RT_SPLIT];
#pragma unroll
      for (int c = 0; c < RT_SPLIT; ++c) v[c] = c < split ? logits[((int64_t)c * T + t) * E + e] : 0.f;
#pragma unroll
      for (int c = 0; c < RT_SPLIT; ++c)
        if (c < split) l += v[c];
    }
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
  return RT_SPLIT * n_tokens * n_experts * (int64_t)sizeof(float);
}

extern "C" int dsv4_route_topk(const void* x_bf16, const float* gate_w, const float* bias, const int32_t* tid2eid,
                               const int64_t* input_ids, int64_t n_tokens, int32_t hidden, int32_t n_experts,
                               int32_t topk, int32_t score_func, int32_t renormalize, float route_scale,
                               float* weights_out, int32_t* indices_out, void* workspace, int64_t workspace_bytes,
                               void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16 && gate_w && weights_out && indices_out && workspace, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && hidden % (RT_SPLIT * RT_KC) == 0, "hidden must be a positive multiple of 1024");
  DSV4_CHECK_ARG(n_experts > 0 && n_experts <= RT_MAX_E, "n_experts must be in [1, 256]");
  DSV4_CHECK_ARG(topk > 0 && topk <= 16 && topk <= n_experts, "topk must be in [1, min(16, n_experts)]");
  DSV4_CHECK_ARG(score_func >= 0 && score_func <= 2, "unknown score function");
  DSV4_CHECK_ARG(!tid2eid || input_ids, "hash routing needs input_ids");
  DSV4_CHECK_ARG(workspace_bytes >= dsv4_route_workspace_bytes(n_tokens, hidden, n_experts),
                 "workspace too small");
  if (n_tokens == 0) return DSV4_OK;
  if (int rc = bind_device_of(x_bf16, nullptr)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((n_experts + RT_EPB - 1) / RT_EPB, RT_SPLIT, (unsigned)((n_tokens + RT_TT - 1) / RT_TT));
  const bool pdl = pdl_enabled();
  DSV4_CUDA_CHECK(launch_k(route_logits_kernel, grid, dim3(256), 0, st, pdl, (const uint16_t*)x_bf16, gate_w,
                           (float*)workspace, n_tokens, hidden, n_experts, RT_SPLIT));
  const int64_t threads = n_tokens * 32;
  DSV4_CUDA_CHECK(launch_k(route_topk_kernel, dim3((unsigned)((threads + 255) / 256)), dim3(256), 0, st, pdl,
                           (const float*)workspace, RT_SPLIT, n_tokens, n_experts, topk, score_func, renormalize,
                           route_scale, bias, tid2eid, input_ids, weights_out, indices_out));
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
//   * at most DSV4_ROUTE_NOALLOC_MAX_LOGITS (n_tokens * n_experts) logits;
//     the array holds the router's fixed split of partial sums for that many
//     logits (1 MiB of device memory that every GPU loading the library keeps
//     until the process exits); larger calls are rejected with DSV4_EINVAL;
//   * the first call on a device looks up the array's device address on
//     that device (cudaGetSymbolAddress); make that first call before any
//     stream capture;
//   * all calls share the one array and it keeps the last call's logits;
//     the logits kernel writes every element the top-k kernel then reads, so
//     nothing needs clearing, but calls that overlap on the GPU (on different
//     streams, or from several threads) race on it.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_route_noalloc_scratch[RT_SPLIT_NOALLOC * DSV4_ROUTE_NOALLOC_MAX_LOGITS];

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
  DSV4_CHECK_ARG(hidden > 0 && hidden % (RT_SPLIT * RT_KC) == 0, "hidden must be a positive multiple of 1024");
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
  const dim3 grid((n_experts + RT_EPB - 1) / RT_EPB, RT_SPLIT_NOALLOC, (unsigned)((n_tokens + RT_TT - 1) / RT_TT));
  route_logits_kernel<<<grid, 256, 0, st>>>((const uint16_t*)x_bf16, gate_w, scratch, n_tokens, hidden, n_experts,
                                            RT_SPLIT_NOALLOC);
  const int64_t threads = n_tokens * 32;
  route_topk_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(
      scratch, RT_SPLIT_NOALLOC, n_tokens, n_experts, topk, score_func, renormalize, route_scale, bias, tid2eid, input_ids,
      weights_out, indices_out);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}
