// Router: OffloadDeepseekV4MoE._route (deepseek_v4.py:118-148).
//   phase 1: fp32 partial logits, split over slices of H (128 wide for
//            decode batches, H/8 wide from 256 tokens on):
//            part[s, t, e] = sum over slice s of float(x[t, k]) * w[e, k];
//   phase 2: one CTA per token: add the slices in order (deterministic),
//            then one warp applies the score function, the biased top-k (or
//            the hash table), the unbiased weights, renormalisation, scale.
#include <mutex>
#include <string>

#include "capi_internal.h"
#include "common.cuh"

namespace dsv4 {

constexpr int RT_MAX_E = 256;
constexpr int RL_TOK = 64;    // tokens per CTA
constexpr int RL_EXP = 64;    // experts per CTA
constexpr int RL_KC = 64;     // K elements per shared-memory chunk
constexpr int RL_SLICE = 128; // K elements per CTA on the workspace path (one partial per 128 of H)
constexpr int RT_SPLIT_NOALLOC = 4;  // slices of H on the fixed-scratch path

// One CTA: 64 tokens x 64 experts over kslice elements of H (a multiple of
// 64).  Each 64-wide chunk is staged transposed in shared memory (xs[k][t],
// ws[k][e], conflict-free stores); thread (tq, eq) accumulates tokens
// 4tq..4tq+3 against experts 4eq..4eq+3, two 16-byte loads per 16 FMAs.  The
// next chunk's global loads are issued before the current chunk is computed.
// One writer per partial: deterministic.
__global__ __launch_bounds__(256) void route_logits_kernel(const uint16_t* __restrict__ x,
                                                           const float* __restrict__ w, float* __restrict__ part,
                                                           int64_t T, int H, int E, int kslice) {
  __shared__ __align__(16) float xs[RL_KC][RL_TOK];
  __shared__ __align__(16) float ws[RL_KC][RL_EXP];
  griddep_wait();
  griddep_launch();
  const int tid = threadIdx.x;
  const int e0 = blockIdx.x * RL_EXP;
  const int slice = blockIdx.y;
  const int64_t t0 = (int64_t)blockIdx.z * RL_TOK;
  const int kbeg = slice * kslice;
  // chunk staging in registers, row index fastest across lanes so the
  // transposed shared-memory stores of a warp hit consecutive banks
  uint4 xr[2];
  float4 wr[4];
  auto load = [&](int kc) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = tid + 256 * j, t = i & (RL_TOK - 1), c = (i >> 6) * 8;
      xr[j] = t0 + t < T ? *reinterpret_cast<const uint4*>(x + (t0 + t) * H + kc + c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = tid + 256 * j, e = i & (RL_EXP - 1), c = (i >> 6) * 4;
      wr[j] = e0 + e < E ? *reinterpret_cast<const float4*>(w + (int64_t)(e0 + e) * H + kc + c)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  load(kbeg);
  const int tq = tid & 15, eq = tid >> 4;
  float acc[4][4] = {};
  for (int kc = kbeg; kc < kbeg + kslice; kc += RL_KC) {
    __syncthreads();   // the previous chunk has been consumed
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = tid + 256 * j, t = i & (RL_TOK - 1), c = (i >> 6) * 8;
      const uint32_t v[4] = {xr[j].x, xr[j].y, xr[j].z, xr[j].w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        xs[c + 2 * m][t] = bf16_from_bits(v[m] & 0xffffu);
        xs[c + 2 * m + 1][t] = bf16_from_bits(v[m] >> 16);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = tid + 256 * j, e = i & (RL_EXP - 1), c = (i >> 6) * 4;
      ws[c][e] = wr[j].x;
      ws[c + 1][e] = wr[j].y;
      ws[c + 2][e] = wr[j].z;
      ws[c + 3][e] = wr[j].w;
    }
    __syncthreads();
    if (kc + RL_KC < kbeg + kslice) load(kc + RL_KC);
#pragma unroll 8
    for (int k = 0; k < RL_KC; ++k) {
      const float4 xv = *reinterpret_cast<const float4*>(&xs[k][4 * tq]);
      const float4 wv = *reinterpret_cast<const float4*>(&ws[k][4 * eq]);
      const float xa[4] = {xv.x, xv.y, xv.z, xv.w}, wa[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(xa[a], wa[b], acc[a][b]);
    }
  }
  float* dst = part + (int64_t)slice * T * E;
  const int e = e0 + 4 * eq;
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t t = t0 + 4 * tq + a;
    if (t >= T) break;
    if (e + 3 < E && (E & 3) == 0) {   // 16-byte aligned quads
      *reinterpret_cast<float4*>(dst + t * E + e) = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
    } else {
#pragma unroll
      for (int b = 0; b < 4; ++b)
        if (e + b < E) dst[t * E + e + b] = acc[a][b];
    }
  }
}

// Prefill-sized batches: one CTA computes 128 tokens x 128 experts over
// kslice elements of H (a multiple of 32), thread (ty, tx) accumulating
// tokens 8ty..8ty+7 against experts 8tx..8tx+7: four 16-byte shared loads
// per 64 FMAs, so the FMA pipe rather than shared memory sets the pace.
// Chunks of 32 of K are staged transposed as in route_logits_kernel.
constexpr int RW_TOK = 128, RW_EXP = 128, RW_KC = 32;
__global__ __launch_bounds__(256, 1) void route_logits_wide_kernel(const uint16_t* __restrict__ x,
                                                                   const float* __restrict__ w,
                                                                   float* __restrict__ part, int64_t T, int H,
                                                                   int E, int kslice) {
  __shared__ __align__(16) float xs[RW_KC][RW_TOK];
  __shared__ __align__(16) float ws[RW_KC][RW_EXP];
  griddep_wait();
  griddep_launch();
  const int tid = threadIdx.x;
  const int e0 = blockIdx.x * RW_EXP;
  const int slice = blockIdx.y;
  const int64_t t0 = (int64_t)blockIdx.z * RW_TOK;
  const int kbeg = slice * kslice;
  uint4 xr[2];
  float4 wr[4];
  auto load = [&](int kc) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = tid + 256 * j, t = i & (RW_TOK - 1), c = (i >> 7) * 8;
      xr[j] = t0 + t < T ? *reinterpret_cast<const uint4*>(x + (t0 + t) * H + kc + c) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = tid + 256 * j, e = i & (RW_EXP - 1), c = (i >> 7) * 4;
      wr[j] = e0 + e < E ? *reinterpret_cast<const float4*>(w + (int64_t)(e0 + e) * H + kc + c)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  load(kbeg);
  const int tx = tid & 15, ty = tid >> 4;
  float acc[8][8] = {};
  for (int kc = kbeg; kc < kbeg + kslice; kc += RW_KC) {
    __syncthreads();   // the previous chunk has been consumed
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = tid + 256 * j, t = i & (RW_TOK - 1), c = (i >> 7) * 8;
      const uint32_t v[4] = {xr[j].x, xr[j].y, xr[j].z, xr[j].w};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        xs[c + 2 * m][t] = bf16_from_bits(v[m] & 0xffffu);
        xs[c + 2 * m + 1][t] = bf16_from_bits(v[m] >> 16);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = tid + 256 * j, e = i & (RW_EXP - 1), c = (i >> 7) * 4;
      ws[c][e] = wr[j].x;
      ws[c + 1][e] = wr[j].y;
      ws[c + 2][e] = wr[j].z;
      ws[c + 3][e] = wr[j].w;
    }
    __syncthreads();
    if (kc + RW_KC < kbeg + kslice) load(kc + RW_KC);
#pragma unroll 4
    for (int k = 0; k < RW_KC; ++k) {
      const float4 x0 = *reinterpret_cast<const float4*>(&xs[k][8 * ty]);
      const float4 x1 = *reinterpret_cast<const float4*>(&xs[k][8 * ty + 4]);
      const float4 w0 = *reinterpret_cast<const float4*>(&ws[k][8 * tx]);
      const float4 w1 = *reinterpret_cast<const float4*>(&ws[k][8 * tx + 4]);
      const float xa[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      const float wa[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) acc[a][b] = fmaf(xa[a], wa[b], acc[a][b]);
    }
  }
  float* dst = part + (int64_t)slice * T * E;
  const int e = e0 + 8 * tx;
#pragma unroll
  for (int a = 0; a < 8; ++a) {
    const int64_t t = t0 + 8 * ty + a;
    if (t >= T) break;
    if (e + 7 < E && (E & 3) == 0) {   // 16-byte aligned quads
      *reinterpret_cast<float4*>(dst + t * E + e) = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
      *reinterpret_cast<float4*>(dst + t * E + e + 4) = make_float4(acc[a][4], acc[a][5], acc[a][6], acc[a][7]);
    } else {
#pragma unroll
      for (int b = 0; b < 8; ++b)
        if (e + b < E) dst[t * E + e + b] = acc[a][b];
    }
  }
}

__device__ __forceinline__ float softplus_f(float v) { return v > 20.f ? v : log1pf(expf(v)); }

// One CTA (256 threads) per token.  Thread e adds the slices of logit
// (t, e) in slice order and applies the score function; warp 0 then takes
// the biased top-k (ties to the lower expert id, as torch.topk on the
// reference's CPU path), or reads the hash table, and writes the unbiased
// weights, renormalised and scaled.
__global__ __launch_bounds__(256) void route_topk_kernel(const float* __restrict__ logits, int split, int64_t T,
                                                         int E, int K, int score_func, int renorm, float scale,
                                                         const float* __restrict__ bias,
                                                         const int32_t* __restrict__ tid2eid,
                                                         const int64_t* __restrict__ ids, float* __restrict__ w_out,
                                                         int32_t* __restrict__ i_out) {
  constexpr int PER = RT_MAX_E / 32;
  __shared__ float sc_s[RT_MAX_E], ch_s[RT_MAX_E];
  __shared__ float red[2][8];
  griddep_wait();
  griddep_launch();
  const int64_t t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int e = tid;
  float l = -INFINITY;
  if (e < E) {
    const float* src = logits + t * E + e;
    const int64_t stride = T * E;
    l = 0.f;
    for (int s0 = 0; s0 < split; s0 += 32) {
      float v[32];
#pragma unroll
      for (int u = 0; u < 32; ++u) v[u] = s0 + u < split ? src[(s0 + u) * stride] : 0.f;
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (s0 + u < split) l += v[u];
    }
  }
  float sc;
  if (score_func == DSV4_SCORE_SOFTMAX) {
    float m = l;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[0][warp] = m;
    __syncthreads();
    m = red[0][0];
    for (int i = 1; i < 8; ++i) m = fmaxf(m, red[0][i]);
    const float ex = e < E ? expf(l - m) : 0.f;
    float sum = ex;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[1][warp] = sum;
    __syncthreads();
    sum = 0.f;
    for (int i = 0; i < 8; ++i) sum += red[1][i];
    sc = ex / sum;
  } else if (score_func == DSV4_SCORE_SIGMOID) {
    sc = 1.f / (1.f + expf(-l));
  } else {
    sc = sqrtf(softplus_f(l));
  }
  sc_s[e] = sc;
  ch_s[e] = e < E ? (bias ? sc + bias[e] : sc) : -INFINITY;
  __syncthreads();
  if (warp != 0) return;
  float ch[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) ch[j] = ch_s[lane + 32 * j];
  float wsel = 0.f;   // lane r keeps pick r
  int isel = 0;
  for (int r = 0; r < K; ++r) {
    int pick;
    if (tid2eid) {
      pick = tid2eid[ids[t] * K + r];
    } else {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int ej = lane + 32 * j;
        if (ej < E && (ch[j] > bv || (ch[j] == bv && ej < bi))) {
          bv = ch[j];
          bi = ej;
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
    if (lane == r) {
      wsel = (pick >= 0 && pick < E) ? sc_s[pick] : 0.f;   // unbiased score of the pick
      isel = pick;
    }
  }
  // renormalise over the K picks in pick order (lane 0 adds them up)
  float ssum = 0.f;
  for (int r = 0; r < K; ++r) ssum += __shfl_sync(0xffffffffu, wsel, r);
  if (lane < K) {
    const float v = renorm ? wsel / ssum : wsel;
    w_out[t * K + lane] = v * scale;
    i_out[t * K + lane] = isel;
  }
}

}  // namespace dsv4

using namespace dsv4;

extern "C" int64_t dsv4_route_workspace_bytes(int64_t n_tokens, int32_t hidden, int32_t n_experts) {
  if (n_tokens < 0 || hidden <= 0 || n_experts <= 0) return DSV4_EINVAL;
  return (int64_t)(hidden / RL_SLICE) * n_tokens * n_experts * (int64_t)sizeof(float);
}

extern "C" int dsv4_route_topk(const void* x_bf16, const float* gate_w, const float* bias, const int32_t* tid2eid,
                               const int64_t* input_ids, int64_t n_tokens, int32_t hidden, int32_t n_experts,
                               int32_t topk, int32_t score_func, int32_t renormalize, float route_scale,
                               float* weights_out, int32_t* indices_out, void* workspace, int64_t workspace_bytes,
                               void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16 && gate_w && weights_out && indices_out && workspace, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && hidden % 1024 == 0, "hidden must be a positive multiple of 1024");
  DSV4_CHECK_ARG(n_experts > 0 && n_experts <= RT_MAX_E, "n_experts must be in [1, 256]");
  DSV4_CHECK_ARG(topk > 0 && topk <= 16 && topk <= n_experts, "topk must be in [1, min(16, n_experts)]");
  DSV4_CHECK_ARG(score_func >= 0 && score_func <= 2, "unknown score function");
  DSV4_CHECK_ARG(!tid2eid || input_ids, "hash routing needs input_ids");
  DSV4_CHECK_ARG(workspace_bytes >= dsv4_route_workspace_bytes(n_tokens, hidden, n_experts),
                 "workspace too small");
  if (n_tokens == 0) return DSV4_OK;
  if (int rc = bind_device_of(x_bf16, nullptr)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = pdl_enabled();
  int split;
  if (n_tokens >= 2 * RW_TOK) {
    // prefill: 128 x 128 tiles, H split into 8 slices (512 of H each at
    // H = 4096): 256 CTAs at T = 2048, E = 256, and 8 partials per logit
    split = 8;
    const dim3 grid((n_experts + RW_EXP - 1) / RW_EXP, split, (unsigned)((n_tokens + RW_TOK - 1) / RW_TOK));
    DSV4_CUDA_CHECK(launch_k(route_logits_wide_kernel, grid, dim3(256), 0, st, pdl, (const uint16_t*)x_bf16,
                             gate_w, (float*)workspace, n_tokens, hidden, n_experts, hidden / split));
  } else {
    // decode: 64 x 64 tiles, one slice per 128 of H, so that a handful of
    // tokens still spreads over 128+ CTAs
    split = hidden / RL_SLICE;
    const dim3 grid((n_experts + RL_EXP - 1) / RL_EXP, split, (unsigned)((n_tokens + RL_TOK - 1) / RL_TOK));
    DSV4_CUDA_CHECK(launch_k(route_logits_kernel, grid, dim3(256), 0, st, pdl, (const uint16_t*)x_bf16, gate_w,
                             (float*)workspace, n_tokens, hidden, n_experts, (int)RL_SLICE));
  }
  DSV4_CUDA_CHECK(launch_k(route_topk_kernel, dim3((unsigned)n_tokens), dim3(256), 0, st, pdl,
                           (const float*)workspace, split, n_tokens, n_experts, topk, score_func, renormalize,
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
  DSV4_CHECK_ARG(hidden > 0 && hidden % 1024 == 0, "hidden must be a positive multiple of 1024");
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
  const dim3 grid((n_experts + RL_EXP - 1) / RL_EXP, RT_SPLIT_NOALLOC, (unsigned)((n_tokens + RL_TOK - 1) / RL_TOK));
  route_logits_kernel<<<grid, 256, 0, st>>>((const uint16_t*)x_bf16, gate_w, scratch, n_tokens, hidden, n_experts,
                                            hidden / RT_SPLIT_NOALLOC);
  route_topk_kernel<<<(unsigned)n_tokens, 256, 0, st>>>(
      scratch, RT_SPLIT_NOALLOC, n_tokens, n_experts, topk, score_func, renormalize, route_scale, bias, tid2eid, input_ids,
      weights_out, indices_out);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}
