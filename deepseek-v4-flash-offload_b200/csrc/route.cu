// Router: OffloadDeepseekV4MoE._route (deepseek_v4.py:118-148).
//   phase 1: fp32 partial logits, split over slices of H:
//            part[s, t, e] = sum over slice s of float(x[t, k]) * w[e, k];
//            decode batches (< 256 tokens) on the FP32 pipes, 128-wide
//            slices; larger batches on the tensor cores (route_logits_tc_kernel),
//            four slices;
//   phase 2: one CTA per token: add the slices in order (deterministic),
//            then one warp applies the score function, the biased top-k (or
//            the hash table), the unbiased weights, renormalisation, scale.
#include <stdlib.h>

#include <algorithm>
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
__device__ __forceinline__ void logits_tile(const uint16_t* __restrict__ x, const float* __restrict__ w,
                                            float* __restrict__ part, int64_t T, int H, int E, int kslice,
                                            float (*xs)[RL_TOK], float (*ws)[RL_EXP]) {
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

__global__ __launch_bounds__(256) void route_logits_kernel(const uint16_t* __restrict__ x,
                                                           const float* __restrict__ w, float* __restrict__ part,
                                                           int64_t T, int H, int E, int kslice) {
  __shared__ __align__(16) float xs[RL_KC][RL_TOK];
  __shared__ __align__(16) float ws[RL_KC][RL_EXP];
  griddep_wait();
  griddep_launch();
  logits_tile(x, w, part, T, H, E, kslice, xs, ws);
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

// ---------------------------------------------------------------------------
// Prefill router on the tensor cores.
//
// The fp32 gate w is split, per call, into three bf16 matrices whose sum is
// w exactly: hi = bf16(w), mid = bf16(w - hi), lo = bf16(w - hi - mid).  Each
// residual is exact in fp32 and the last one fits bf16's 8 significant bits
// (for |w| below bf16's largest finite value, 3.39e38).
// x is bf16, so every product x*hi, x*mid, x*lo is exact in fp32, and the
// tensor cores accumulate them in fp32: the logits keep fp32 accuracy, in a
// different summation order than the FP32-pipe kernels (as any two fp32 GEMMs
// differ).  One CTA computes 128 experts (MMA M) x 128 tokens (MMA N) over
// H/RTC_SPLIT, one tcgen05.mma.kind::f16 per (16 of K, gate term), into 128
// TMEM columns.  Warp 0: TMA producer; warp 1: TMEM owner and MMA issuer;
// warps 2-5: epilogue (TMEM lane quarter warp % 4).
// ---------------------------------------------------------------------------
constexpr int RTC_M = 128, RTC_N = 128, RTC_KC = 64, RTC_STAGES = 3, RTC_TERMS = 3, RTC_SPLIT = 4;
constexpr int RTC_TERM_BYTES = RTC_M * RTC_KC * 2;                 // 16 KB: 128 rows x 128 B
constexpr int RTC_A_BYTES = RTC_TERMS * RTC_TERM_BYTES;            // 48 KB
constexpr int RTC_B_BYTES = RTC_N * RTC_KC * 2;                    // 16 KB
constexpr int RTC_STAGE_BYTES = RTC_A_BYTES + RTC_B_BYTES;         // 64 KB
constexpr int RTC_SMEM = RTC_STAGES * RTC_STAGE_BYTES + 256 + 1024;
constexpr int RTC_THREADS = 192;
constexpr uint32_t RTC_TMEM_COLS = 128;

// hi / mid / lo terms of the gate, [3][E*H] bf16; also clears the call's
// error word (read by route_topk_kernel after the logits kernel).
__global__ void gate_split_kernel(const float4* __restrict__ w, int64_t n4, uint2* __restrict__ out,
                                  int* __restrict__ err) {
  griddep_wait();
  griddep_launch();
  if (blockIdx.x == 0 && threadIdx.x == 0) *err = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v4 = w[i];
    const float v[4] = {v4.x, v4.y, v4.z, v4.w};
    uint32_t h[4], m[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = bf16_bits(v[j]);
      const float r1 = v[j] - bf16_from_bits(h[j]);
      m[j] = bf16_bits(r1);
      const float r2 = r1 - bf16_from_bits(m[j]);
      l[j] = bf16_bits(r2);
    }
    out[i] = make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
    out[n4 + i] = make_uint2(m[0] | (m[1] << 16), m[2] | (m[3] << 16));
    out[2 * n4 + i] = make_uint2(l[0] | (l[1] << 16), l[2] | (l[3] << 16));
  }
}

__global__ void __launch_bounds__(RTC_THREADS, 1)
    route_logits_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                           float* __restrict__ part, int64_t T, int E, int kslice, int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + RTC_STAGES * RTC_STAGE_BYTES);
  uint64_t* empty = full + RTC_STAGES;
  uint64_t* accfull = empty + RTC_STAGES;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(accfull + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.x * RTC_M;
  const int64_t t0 = (int64_t)blockIdx.y * RTC_N;
  const int slice = blockIdx.z;
  const int kbeg = slice * kslice;
  const int nch = kslice / RTC_KC;
  if (threadIdx.x == 0) {
    for (int s = 0; s < RTC_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accfull, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmW);
    prefetch_tensormap(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, RTC_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  griddep_wait();   // the gate terms come from the split kernel just before
  griddep_launch();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_last();   // x and the gate terms are read by several CTAs
      int issued = 0;
      for (int c = 0; c < nch; ++c) {
        const int s = c % RTC_STAGES;
        const uint32_t ph = (uint32_t)(c / RTC_STAGES) & 1u;
        if (c >= RTC_STAGES && !mbar_wait(&empty[s], ph ^ 1u, err)) break;
        uint8_t* st = smem + s * RTC_STAGE_BYTES;
        mbar_expect_tx(&full[s], RTC_STAGE_BYTES);
        tma_load_3d(st, &tmW, &full[s], kbeg + c * RTC_KC, e0, 0, pol);
        tma_load_2d(st + RTC_A_BYTES, &tmX, &full[s], kbeg + c * RTC_KC, (int)t0, pol);
        mbar_arrive(&full[s]);   // the barrier's one arrival; the copies complete its transaction bytes
        ++issued;
      }
      // the last stages' copies have landed before the CTA can exit
      for (int c = issued - RTC_STAGES < 0 ? 0 : issued - RTC_STAGES; c < issued; ++c) {
        const uint64_t tw = globaltimer_ns();
        while (!mbar_try_wait(&full[c % RTC_STAGES], (uint32_t)(c / RTC_STAGES) & 1u) &&
               globaltimer_ns() - tw < DSV4_WAIT_NS) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(RTC_M, RTC_N);
      for (int c = 0; c < nch; ++c) {
        const int s = c % RTC_STAGES;
        const uint32_t ph = (uint32_t)(c / RTC_STAGES) & 1u;
        if (!mbar_wait(&full[s], ph, err)) break;
        tc_fence_after();
        const uint32_t a = smem_u32(smem + s * RTC_STAGE_BYTES);
        const uint64_t db = desc_sw128(a + RTC_A_BYTES);
#pragma unroll
        for (int term = 0; term < RTC_TERMS; ++term) {
          const uint64_t da = desc_sw128(a + term * RTC_TERM_BYTES);
#pragma unroll
          for (int j = 0; j < RTC_KC / 16; ++j)   // +32 bytes (16 bf16) of K per step in the swizzle row
            tc_mma_bf16(tmem, da + 2u * j, db + 2u * j, idesc, (c | term | j) != 0 ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      // every MMA issued above has completed once this arrives
      tc_commit(accfull);
      const uint64_t tw = globaltimer_ns();
      while (!mbar_try_wait(accfull, 0) && globaltimer_ns() - tw < DSV4_WAIT_NS) {
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3;   // TMEM lanes 32q..32q+31 = experts e0+32q..
    // warp-uniform decision: tcgen05.ld below needs all 32 lanes
    const bool ok = __all_sync(0xffffffffu, mbar_wait(accfull, 0, err) && read_status(err) == 0);
    tc_fence_after();
    if (ok) {
      const int e = e0 + q * 32 + lane;
      float* dst = part + (int64_t)slice * T * E + e;
#pragma unroll 1
      for (int c0 = 0; c0 < RTC_N; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
        tc_wait_ld();
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          const int64_t t = t0 + c0 + n;
          if (t < T && e < E) dst[t * E] = v[n];
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, RTC_TMEM_COLS);
  }
}

__device__ __forceinline__ float softplus_f(float v) { return v > 20.f ? v : log1pf(expf(v)); }

// One CTA (256 threads) per token.  Thread e adds the slices of logit
// (t, e) in slice order and applies the score function; warp 0 then takes
// the biased top-k (ties to the lower expert id, as torch.topk on the
// reference's CPU path), or reads the hash table, and writes the unbiased
// weights, renormalised and scaled.  A hash-table token id outside
// [0, vocab) reads nothing: its picks are written as expert id E (out of
// range), which the layer's align rejects with DSV4_EINVAL.
struct TopkSmem {
  float sc[RT_MAX_E], ch[RT_MAX_E];
  float red[2][8];
};

// Token t's picks by one CTA of 256 threads (see route_topk_kernel).
__device__ __forceinline__ void topk_token(int64_t t, const float* __restrict__ logits, int split, int64_t T, int E,
                                           int K, int score_func, int renorm, float scale,
                                           const float* __restrict__ bias, const int32_t* __restrict__ tid2eid,
                                           const int64_t* __restrict__ ids, int64_t vocab, float* __restrict__ w_out,
                                           int32_t* __restrict__ i_out, TopkSmem& sm) {
  constexpr int PER = RT_MAX_E / 32;
  float* sc_s = sm.sc;
  float* ch_s = sm.ch;
  float (*red)[8] = sm.red;
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
  if (warp != 0) return;   // the caller synchronises the CTA before reusing sm
  float ch[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) ch[j] = ch_s[lane + 32 * j];
  float wsel = 0.f;   // lane r keeps pick r
  int isel = 0;
  for (int r = 0; r < K; ++r) {
    int pick;
    if (tid2eid) {
      const int64_t id = ids[t];
      pick = (id >= 0 && id < vocab) ? tid2eid[id * K + r] : E;
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
    // a rejected hash row (picks E) gets weight 0, not 0 / 0
    const float v = (isel >= E) ? 0.f : (renorm ? wsel / ssum : wsel);
    w_out[t * K + lane] = v * scale;
    i_out[t * K + lane] = isel;
  }
}

// Token t's picks by one warp: lane L holds experts L + 32 j (j < 8).  The
// same arithmetic in the same order as topk_token (the slices added in
// order; the softmax sum as the per-32-expert shuffle trees added in expert
// order), so the results are bit-identical; no block barrier, so a CTA of
// 8 warps takes 8 tokens (prefill batches: a few slices per logit).
__device__ __forceinline__ void topk_token_warp(int64_t t, const float* __restrict__ logits, int split, int64_t T,
                                                int E, int K, int score_func, int renorm, float scale,
                                                const float* __restrict__ bias, const int32_t* __restrict__ tid2eid,
                                                const int64_t* __restrict__ ids, int64_t vocab,
                                                float* __restrict__ w_out, int32_t* __restrict__ i_out) {
  constexpr int PER = RT_MAX_E / 32;
  const int lane = threadIdx.x & 31;
  float l[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) l[j] = lane + 32 * j < E ? 0.f : -INFINITY;
  {
    const float* src = logits + t * E + lane;
    const int64_t stride = T * E;
    for (int s0 = 0; s0 < split; s0 += 4) {
      float v[4][PER];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int j = 0; j < PER; ++j)
          v[u][j] = (s0 + u < split && lane + 32 * j < E) ? src[(s0 + u) * stride + 32 * j] : 0.f;
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int j = 0; j < PER; ++j)
          if (s0 + u < split && lane + 32 * j < E) l[j] += v[u][j];
    }
  }
  float sc[PER];
  if (score_func == DSV4_SCORE_SOFTMAX) {
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < PER; ++j) m = fmaxf(m, l[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float ex[PER];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      ex[j] = lane + 32 * j < E ? expf(l[j] - m) : 0.f;
      float s = ex[j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      sum += s;
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) sc[j] = ex[j] / sum;
  } else if (score_func == DSV4_SCORE_SIGMOID) {
#pragma unroll
    for (int j = 0; j < PER; ++j) sc[j] = 1.f / (1.f + expf(-l[j]));
  } else {
#pragma unroll
    for (int j = 0; j < PER; ++j) sc[j] = sqrtf(softplus_f(l[j]));
  }
  float ch[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int ej = lane + 32 * j;
    ch[j] = ej < E ? (bias ? sc[j] + bias[ej] : sc[j]) : -INFINITY;
  }
  float wsel = 0.f;   // lane r keeps pick r
  int isel = 0;
  for (int r = 0; r < K; ++r) {
    int pick;
    if (tid2eid) {
      const int64_t id = ids[t];
      pick = (id >= 0 && id < vocab) ? tid2eid[id * K + r] : E;
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
    // the unbiased score of the pick, from the lane that holds it
    const bool ok = pick >= 0 && pick < E;
    float mine = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (ok && j == (pick >> 5)) mine = sc[j];
    const float sp = __shfl_sync(0xffffffffu, mine, ok ? (pick & 31) : 0);
    if (lane == r) {
      wsel = ok ? sp : 0.f;
      isel = pick;
    }
  }
  float ssum = 0.f;
  for (int r = 0; r < K; ++r) ssum += __shfl_sync(0xffffffffu, wsel, r);
  if (lane < K) {
    const float v = (isel >= E) ? 0.f : (renorm ? wsel / ssum : wsel);
    w_out[t * K + lane] = v * scale;
    i_out[t * K + lane] = isel;
  }
}

__global__ __launch_bounds__(256) void route_topk_warp_kernel(const float* __restrict__ logits, int split, int64_t T,
                                                              int E, int K, int score_func, int renorm, float scale,
                                                              const float* __restrict__ bias,
                                                              const int32_t* __restrict__ tid2eid,
                                                              const int64_t* __restrict__ ids, int64_t vocab,
                                                              float* __restrict__ w_out, int32_t* __restrict__ i_out,
                                                              const int* __restrict__ err) {
  griddep_wait();
  griddep_launch();
  const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  if (err && *reinterpret_cast<const volatile int*>(err) != 0) {
    if ((int)(threadIdx.x & 31) < K) {   // the logits kernel gave up on a wait: picks out of range
      w_out[t * K + (threadIdx.x & 31)] = 0.f;
      i_out[t * K + (threadIdx.x & 31)] = E;
    }
    return;
  }
  topk_token_warp(t, logits, split, T, E, K, score_func, renorm, scale, bias, tid2eid, ids, vocab, w_out, i_out);
}

// picks of a token whose logits are not available (a wait gave up):
// expert id E is out of range, so the layer's align rejects them and its
// status reports it
__device__ __forceinline__ void topk_token_failed(int64_t t, int E, int K, float* __restrict__ w_out,
                                                  int32_t* __restrict__ i_out) {
  if ((int)threadIdx.x < K) {
    w_out[t * K + threadIdx.x] = 0.f;
    i_out[t * K + threadIdx.x] = E;
  }
}

__global__ __launch_bounds__(256) void route_topk_kernel(const float* __restrict__ logits, int split, int64_t T,
                                                         int E, int K, int score_func, int renorm, float scale,
                                                         const float* __restrict__ bias,
                                                         const int32_t* __restrict__ tid2eid,
                                                         const int64_t* __restrict__ ids, int64_t vocab,
                                                         float* __restrict__ w_out,
                                                         int32_t* __restrict__ i_out, const int* __restrict__ err) {
  __shared__ TopkSmem sm;
  griddep_wait();
  griddep_launch();
  const int64_t t = blockIdx.x;
  if (err && *reinterpret_cast<const volatile int*>(err) != 0) {
    topk_token_failed(t, E, K, w_out, i_out);   // the logits kernel gave up on a wait
    return;
  }
  topk_token(t, logits, split, T, E, K, score_func, renorm, scale, bias, tid2eid, ids, vocab, w_out, i_out, sm);
}

// Decode router in one launch (batches of fewer than 256 tokens): every CTA
// computes its 64 x 64 x 128 tile of partial logits (logits_tile), the grid
// meets at a barrier, then CTA b takes the top-k of tokens b, b + G, ... .
// The barrier is a counter in zeroed memory that the last CTA to finish sets
// back to zero (bar[0]: arrivals, bar[1]: CTAs past the top-k), so a launch
// finds it at zero; the host launches this only when the whole grid fits on
// the GPU at once, and the wait is bounded (DSV4_ETIMEOUT into `status`,
// the affected tokens' picks marked invalid).  A CTA that arrives late still
// completes its share and the count, so the counter is back at zero after
// every launch.
__global__ __launch_bounds__(256) void route_fused_kernel(const uint16_t* __restrict__ x,
                                                          const float* __restrict__ w, float* __restrict__ part,
                                                          int64_t T, int H, int E, int kslice, int* bar, int K,
                                                          int score_func, int renorm, float scale,
                                                          const float* __restrict__ bias,
                                                          const int32_t* __restrict__ tid2eid,
                                                          const int64_t* __restrict__ ids, int64_t vocab,
                                                          float* __restrict__ w_out, int32_t* __restrict__ i_out,
                                                          int* status) {
  __shared__ __align__(16) float xs[RL_KC][RL_TOK];
  __shared__ __align__(16) float ws[RL_KC][RL_EXP];
  __shared__ TopkSmem sm;
  __shared__ int ok_s;
  griddep_wait();
  griddep_launch();
  const int G = (int)(gridDim.x * gridDim.y * gridDim.z);
  const int b = (int)(blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z));
  logits_tile(x, w, part, T, H, E, kslice, xs, ws);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    red_release_add(bar, 1);
    ok_s = wait_count_geq(bar, G, status) ? 1 : 0;
  }
  __syncthreads();
  const int split = H / kslice;
  for (int64_t t = b; t < T; t += G) {
    if (ok_s)
      topk_token(t, part, split, T, E, K, score_func, renorm, scale, bias, tid2eid, ids, vocab, w_out, i_out, sm);
    else
      topk_token_failed(t, E, K, w_out, i_out);
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (atomicAdd(bar + 1, 1) == G - 1) {   // every CTA is past the barrier
      atomicExch(bar, 0);
      atomicExch(bar + 1, 0);
    }
  }
}

}  // namespace dsv4

using namespace dsv4;

namespace {
// Batches from this many tokens take the tensor-core logits kernel.
constexpr int64_t RTC_MIN_TOKENS = 256;
int64_t al256(int64_t v) { return (v + 255) / 256 * 256; }
// Tensor-core path workspace: [error word | gate terms bf16 [3][E][H] | partials [RTC_SPLIT][T][E] fp32]
int64_t tc_terms_off() { return 256; }
int64_t tc_part_off(int32_t hidden, int32_t n_experts) {
  return 256 + al256((int64_t)RTC_TERMS * n_experts * hidden * 2);
}
// DSV4_ROUTE_TC=0 keeps prefill batches on the FP32-pipe kernel (the
// tensor-core path is the default).
const bool g_route_no_tc = [] {
  const char* e = getenv("DSV4_ROUTE_TC");
  return e && e[0] == '0';
}();
std::mutex g_tc_mu;
bool g_tc_ready[64] = {};
// The tensor-core kernel's shared-memory opt-in, once per device.
int prepare_route_tc() {
  int dev = 0;
  DSV4_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(g_tc_mu);
  if (dev >= 0 && dev < 64 && g_tc_ready[dev]) return DSV4_OK;
  DSV4_CUDA_CHECK(cudaFuncSetAttribute(route_logits_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RTC_SMEM));
  if (dev >= 0 && dev < 64) g_tc_ready[dev] = true;
  return DSV4_OK;
}
std::mutex g_fused_mu;
int g_fused_cap[64] = {};   // CTAs of route_fused_kernel resident at once, per device (0: not known yet)
}  // namespace

namespace dsv4 {
int route_fused_launch(const void* x_bf16, const float* gate_w, const float* bias, const int32_t* tid2eid,
                       const int64_t* input_ids, int64_t vocab, int64_t n_tokens, int hidden, int n_experts,
                       int topk, int score_func, int renormalize, float route_scale, float* weights_out,
                       int32_t* indices_out, float* part, int* bar, int* status, cudaStream_t st, bool* launched) {
  *launched = false;
  if (n_tokens <= 0 || n_tokens >= RTC_MIN_TOKENS || n_experts > RT_MAX_E || hidden % RL_SLICE != 0) return DSV4_OK;
  int dev = 0;
  DSV4_CUDA_CHECK(cudaGetDevice(&dev));
  int cap = 0;
  {
    std::lock_guard<std::mutex> lock(g_fused_mu);
    if (dev >= 0 && dev < 64 && g_fused_cap[dev] > 0) {
      cap = g_fused_cap[dev];
    } else {
      int per_sm = 0, sms = 0;
      DSV4_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, route_fused_kernel, 256, 0));
      DSV4_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
      cap = per_sm * sms;
      if (dev >= 0 && dev < 64) g_fused_cap[dev] = cap;
    }
  }
  const dim3 grid((n_experts + RL_EXP - 1) / RL_EXP, hidden / RL_SLICE, (unsigned)((n_tokens + RL_TOK - 1) / RL_TOK));
  // the barrier needs every CTA resident at once; half the capacity leaves
  // room for the kernels it may still share the GPU with under PDL
  if ((int64_t)grid.x * grid.y * grid.z > cap / 2) return DSV4_OK;
  DSV4_CUDA_CHECK(launch_k(route_fused_kernel, grid, dim3(256), 0, st, pdl_enabled(), (const uint16_t*)x_bf16, gate_w,
                           part, n_tokens, hidden, n_experts, (int)RL_SLICE, bar, topk, score_func, renormalize,
                           route_scale, bias, tid2eid, input_ids, vocab, weights_out, indices_out, status));
  *launched = true;
  return DSV4_OK;
}
}  // namespace dsv4

extern "C" int64_t dsv4_route_workspace_bytes(int64_t n_tokens, int32_t hidden, int32_t n_experts) {
  if (n_tokens < 0 || hidden <= 0 || n_experts <= 0) return DSV4_EINVAL;
  const int64_t simt = (int64_t)(hidden / RL_SLICE) * n_tokens * n_experts * (int64_t)sizeof(float);
  if (n_tokens < RTC_MIN_TOKENS || n_experts < RTC_M) return simt;
  const int64_t tc = tc_part_off(hidden, n_experts) + (int64_t)RTC_SPLIT * n_tokens * n_experts * 4;
  return std::max(simt, tc);
}

extern "C" int dsv4_route_topk(const void* x_bf16, const float* gate_w, const float* bias, const int32_t* tid2eid,
                               const int64_t* input_ids, int64_t vocab_size, int64_t n_tokens, int32_t hidden,
                               int32_t n_experts, int32_t topk, int32_t score_func, int32_t renormalize,
                               float route_scale, float* weights_out, int32_t* indices_out, void* workspace,
                               int64_t workspace_bytes, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16 && gate_w && weights_out && indices_out && workspace, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && hidden % 1024 == 0, "hidden must be a positive multiple of 1024");
  DSV4_CHECK_ARG(n_experts > 0 && n_experts <= RT_MAX_E, "n_experts must be in [1, 256]");
  DSV4_CHECK_ARG(topk > 0 && topk <= 16 && topk <= n_experts, "topk must be in [1, min(16, n_experts)]");
  DSV4_CHECK_ARG(score_func >= 0 && score_func <= 2, "unknown score function");
  DSV4_CHECK_ARG(!tid2eid || (input_ids && vocab_size > 0), "hash routing needs input_ids and vocab_size");
  DSV4_CHECK_ARG(n_tokens >= 0, "n_tokens must not be negative");
  DSV4_CHECK_ARG(workspace_bytes >= dsv4_route_workspace_bytes(n_tokens, hidden, n_experts),
                 "workspace too small");
  if (n_tokens == 0) return DSV4_OK;
  if (int rc = bind_device_of(x_bf16, nullptr)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = pdl_enabled();
  int split;
  const float* logits = (const float*)workspace;
  const int* err = nullptr;
  const bool tc = n_tokens >= RTC_MIN_TOKENS && n_experts >= RTC_M && ((uintptr_t)x_bf16 % 16) == 0 &&
                  ((uintptr_t)workspace % 16) == 0 && ((uintptr_t)gate_w % 16) == 0 && !g_route_no_tc;
  if (tc) {
    // prefill: gate split into three bf16 terms, then the tensor-core logits
    uint8_t* ws = (uint8_t*)workspace;
    int* err_w = (int*)ws;
    uint16_t* terms = (uint16_t*)(ws + tc_terms_off());
    float* part = (float*)(ws + tc_part_off(hidden, n_experts));
    const int64_t n4 = (int64_t)n_experts * hidden / 4;
    DSV4_CUDA_CHECK(launch_k(gate_split_kernel, dim3(296), dim3(256), 0, st, pdl, (const float4*)gate_w, n4,
                             (uint2*)terms, err_w));
    CUtensorMap tmW, tmX;
    {
      const uint64_t dims[3] = {(uint64_t)hidden, (uint64_t)n_experts, (uint64_t)RTC_TERMS};
      const uint64_t str[2] = {(uint64_t)hidden * 2, (uint64_t)hidden * n_experts * 2};
      const uint32_t box[3] = {RTC_KC, RTC_M, RTC_TERMS};
      if (int rc = make_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, terms, dims, str, box, "gate terms")) return rc;
    }
    {
      const uint64_t dims[2] = {(uint64_t)hidden, (uint64_t)n_tokens};
      const uint64_t str[1] = {(uint64_t)hidden * 2};
      const uint32_t box[2] = {RTC_KC, RTC_N};
      if (int rc = make_map(&tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (void*)x_bf16, dims, str, box, "x")) return rc;
    }
    if (int rc = prepare_route_tc()) return rc;
    split = RTC_SPLIT;
    const dim3 grid((n_experts + RTC_M - 1) / RTC_M, (unsigned)((n_tokens + RTC_N - 1) / RTC_N), RTC_SPLIT);
    DSV4_CUDA_CHECK(launch_k(route_logits_tc_kernel, grid, dim3(RTC_THREADS), RTC_SMEM, st, pdl, tmW, tmX, part,
                             n_tokens, n_experts, hidden / RTC_SPLIT, err_w));
    logits = part;
    err = err_w;
  } else if (n_tokens >= 2 * RW_TOK) {
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
  if (n_tokens >= RTC_MIN_TOKENS)   // a few slices per logit: a warp per token, 8 tokens per CTA
    DSV4_CUDA_CHECK(launch_k(route_topk_warp_kernel, dim3((unsigned)((n_tokens + 7) / 8)), dim3(256), 0, st, pdl,
                             logits, split, n_tokens, n_experts, topk, score_func, renormalize, route_scale, bias,
                             tid2eid, input_ids, vocab_size, weights_out, indices_out, err));
  else   // 32 slices per logit: a CTA per token, a thread per expert
    DSV4_CUDA_CHECK(launch_k(route_topk_kernel, dim3((unsigned)n_tokens), dim3(256), 0, st, pdl, logits, split,
                             n_tokens, n_experts, topk, score_func, renormalize, route_scale, bias, tid2eid,
                             input_ids, vocab_size, weights_out, indices_out, err));
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
                                       const int32_t* tid2eid, const int64_t* input_ids, int64_t vocab_size,
                                       int64_t n_tokens, int32_t hidden, int32_t n_experts, int32_t topk,
                                       int32_t score_func,
                                       int32_t renormalize, float route_scale, float* weights_out,
                                       int32_t* indices_out, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16 && gate_w && weights_out && indices_out, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && hidden % 1024 == 0, "hidden must be a positive multiple of 1024");
  DSV4_CHECK_ARG(n_experts > 0 && n_experts <= RT_MAX_E, "n_experts must be in [1, 256]");
  DSV4_CHECK_ARG(topk > 0 && topk <= 16 && topk <= n_experts, "topk must be in [1, min(16, n_experts)]");
  DSV4_CHECK_ARG(score_func >= 0 && score_func <= 2, "unknown score function");
  DSV4_CHECK_ARG(!tid2eid || (input_ids && vocab_size > 0), "hash routing needs input_ids and vocab_size");
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
      vocab_size, weights_out, indices_out, nullptr);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}
