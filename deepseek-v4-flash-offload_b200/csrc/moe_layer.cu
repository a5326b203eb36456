// Routed-expert layer: moe_align, activation quant + gather, the two grouped
// GEMMs (moe_gemm.cuh) and the deterministic combine, bound together by a
// plan that owns the TMA descriptors.  Mirrors _routed / _routed_mxfp4
// (deepseek_v4.py:150-245) of the reference.
#include <stdlib.h>

#include <algorithm>
#include <memory>
#include <string>

#include "capi_internal.h"
#include "common.cuh"
#include "moe_gemm.cuh"

namespace dsv4 {

// ---------------------------------------------------------------------------
// moe_align (deepseek_v4.py:154-164): one CTA of 1024 threads, a stable
// counting sort.  The rank of an assignment among equal experts of its warp
// comes from ballots over the expert id's bits; the rank across warps from a
// per-warp, per-expert count table and its prefix over the warps.  Up to 1024
// assignments take one pass (one per thread); larger batches give each warp
// a contiguous segment that it walks twice (count, then place).  Also emits
// the active-expert list and the GEMM work chunks.  With pad > 1 every expert's group starts at a multiple of
// pad rows (the GEMM tile height); padding positions get sorted_flat = -1
// and each chunk is one pad-row block of one expert.
// ---------------------------------------------------------------------------
constexpr int AL_THREADS = 1024;
constexpr int GEMM_BN_MAX = 128;   // bound on the GEMM tile (64 or 112 tokens per expert chunk)

// Lanes of the warp holding the same value v (v = -1 or 0 <= v < 2^nbits),
// from nbits + 1 ballots: the same set as __match_any_sync, at a fraction of
// its latency.
__device__ __forceinline__ unsigned match_small(int v, int nbits) {
  const bool valid = v >= 0;
  const unsigned bv = __ballot_sync(0xffffffffu, valid);
  unsigned same = valid ? bv : ~bv;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = valid && ((v >> b) & 1);
    const unsigned bal = __ballot_sync(0xffffffffu, bit);
    same &= bit ? bal : ~bal;
  }
  return same;
}

__device__ __forceinline__ int block_exclusive_scan(int v, int* scratch, int* total) {
  // scratch: 32 ints.  All 1024 threads participate.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = scratch[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    scratch[lane] = w;
  }
  __syncthreads();
  const int excl = x - v + (warp > 0 ? scratch[warp - 1] : 0);
  if (total) *total = scratch[31];
  __syncthreads();
  return excl;
}

// Exclusive scan of three values over the block (all AL_THREADS threads
// call it); scratch: 96 ints.  Two barriers; the caller separates the next
// use of scratch by another barrier.
__device__ __forceinline__ int3 block_scan3(int a, int b, int c, int* scratch, int3* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int xa = a, xb = b, xc = c;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ya = __shfl_up_sync(0xffffffffu, xa, o);
    const int yb = __shfl_up_sync(0xffffffffu, xb, o);
    const int yc = __shfl_up_sync(0xffffffffu, xc, o);
    if (lane >= o) {
      xa += ya;
      xb += yb;
      xc += yc;
    }
  }
  if (lane == 31) {
    scratch[warp] = xa;
    scratch[32 + warp] = xb;
    scratch[64 + warp] = xc;
  }
  __syncthreads();
  if (warp < 3) {
    int v = scratch[32 * warp + lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    scratch[32 * warp + lane] = v;
  }
  __syncthreads();
  *total = make_int3(scratch[31], scratch[63], scratch[95]);
  return make_int3(xa - a + (warp > 0 ? scratch[warp - 1] : 0), xb - b + (warp > 0 ? scratch[31 + warp] : 0),
                   xc - c + (warp > 0 ? scratch[63 + warp] : 0));
}

// Assignment a = t * topk + j of the layer: the router's pick j of token t
// for j < k_in; with a shared expert (shared_e >= 0, topk = k_in + 1) the
// last assignment of every token is the shared expert with weight 1.
__device__ __forceinline__ int assign_expert(const int32_t* __restrict__ idx, int a, int topk, int k_in,
                                             int shared_e) {
  if (shared_e < 0) return idx[a];
  const int t = a / topk, j = a - t * topk;
  return j < k_in ? idx[t * k_in + j] : shared_e;
}
__device__ __forceinline__ float assign_weight(const float* __restrict__ w, int a, int topk, int k_in, int shared_e) {
  if (shared_e < 0) return w[a];
  const int t = a / topk, j = a - t * topk;
  return j < k_in ? w[t * k_in + j] : 1.0f;
}

__global__ void __launch_bounds__(AL_THREADS, 1)
    moe_align_kernel(const int32_t* __restrict__ idx, int P, int topk, int E, const float* __restrict__ w_flat,
                     int32_t* __restrict__ counts, int32_t* __restrict__ offsets, int32_t* __restrict__ sorted_flat,
                     int32_t* __restrict__ inv, int32_t* __restrict__ active, int32_t* __restrict__ n_active,
                     float* __restrict__ sorted_w, int4* __restrict__ chunks, int32_t* __restrict__ n_chunks,
                     int pad, int* status, const int32_t* __restrict__ n_tokens_dev, int k_in, int shared_e,
                     int* __restrict__ chunk_done, int max_chunks) {
  extern __shared__ int sm[];
  int* cnt = sm;                 // E
  int* run = cnt + E;            // E
  int* scratch = run + E;        // 32
  int* sidx = scratch + 32;      // AL_THREADS ints: scan scratch of the one-pass path
  uint16_t* wc = reinterpret_cast<uint16_t*>(sidx + AL_THREADS);  // [32][E] u16 (one pass) or u32 (two passes)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ebits = 32 - __clz(max(E - 1, 1));   // bits of the largest expert id
  griddep_wait();
  griddep_launch();
  for (int j = tid; j < max_chunks; j += AL_THREADS) chunk_done[j] = 0;
  // a token count known only on the device (rows received by expert
  // parallelism): the first n tokens of the buffers
  if (n_tokens_dev) P = min(P, max(0, *n_tokens_dev) * topk);
  const bool small = P <= AL_THREADS;

  if (small) {
    // Decode-sized batch, one assignment per thread, five barriers: the
    // stable rank of assignment p in its expert is its rank among equal
    // experts of its warp (match) plus the count of that expert in the
    // warps before it (exclusive prefix over the per-warp count table).
    uint32_t* wc32 = reinterpret_cast<uint32_t*>(wc);
    for (int j = tid; j < 16 * E; j += AL_THREADS) wc32[j] = 0u;
    int e = -1;
    float wv = 0.f;
    if (tid < P) {
      // both loads issued together (the weight does not depend on the id)
      e = assign_expert(idx, tid, topk, k_in, shared_e);
      if (sorted_w) wv = assign_weight(w_flat, tid, topk, k_in, shared_e);
      if (e == -1) {   // an empty assignment (padding of the expert-parallel exchange)
        inv[tid] = -1;
      } else if (e < 0 || e >= E) {
        set_status(status, DSV4_EINVAL);
        inv[tid] = -1;
        e = -1;
      }
    }
    __syncthreads();
    const unsigned same = match_small(e, ebits);
    const int rank = __popc(same & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wc[warp * E + e] = (uint16_t)__popc(same);
    __syncthreads();
    int c = 0;
    if (tid < E) {
      uint16_t v[32];
#pragma unroll
      for (int w = 0; w < 32; ++w) v[w] = wc[w * E + tid];
#pragma unroll
      for (int w = 0; w < 32; ++w) {
        wc[w * E + tid] = (uint16_t)c;
        c += v[w];
      }
    }
    const int cpad = (c + pad - 1) / pad * pad;
    const int nch = cpad / pad;
    int3 tot3;
    const int3 ex = block_scan3(cpad, c > 0 ? 1 : 0, nch, sidx, &tot3);
    if (tid < E) {
      run[tid] = ex.x;   // start row of the group
      cnt[tid] = c;
      counts[tid] = c;
      offsets[tid] = ex.x;
      if (c > 0) active[ex.y] = tid;
      if (chunks)
        for (int j = 0; j < nch; ++j)
          chunks[ex.z + j] = make_int4(tid, ex.x + j * pad, min(pad, c - j * pad), nch > 1);
    }
    if (tid == 0) {
      offsets[E] = tot3.x;
      *n_active = tot3.y;
      if (chunks) *n_chunks = tot3.z;
    }
    __syncthreads();
    if (e >= 0) {
      const int pos = run[e] + wc[warp * E + e] + rank;
      sorted_flat[pos] = tid;
      inv[tid] = pos;
      if (sorted_w) sorted_w[pos] = wv;
    }
    // padding rows of each group (fewer than `pad`), one warp per group so
    // the stores of a warp are contiguous
    for (int g = warp; g < E; g += AL_THREADS / 32) {
      const int r0 = run[g] + cnt[g], r1 = run[g] + (cnt[g] + pad - 1) / pad * pad;
      for (int r = r0 + lane; r < r1; r += 32) {
        sorted_flat[r] = -1;
        if (sorted_w) sorted_w[r] = 0.f;
      }
    }
    return;
  }

  // Larger batches: warp w owns the contiguous segment [w*seg, (w+1)*seg)
  // of assignments and walks it 32 at a time, in order, twice.  Pass 1
  // counts each expert per warp ([32][E] table); a column prefix over the
  // warps then gives every warp the start of its rows inside each group,
  // and pass 2 hands out the positions.  The order is the stable counting
  // sort's; there is no block barrier inside the passes.
  uint32_t* wcn = reinterpret_cast<uint32_t*>(wc);   // [32][E]
  for (int j = tid; j < 32 * E; j += AL_THREADS) wcn[j] = 0u;
  __syncthreads();
  const int seg = (P + 31) / 32;
  const int s0 = min(P, warp * seg), s1 = min(P, s0 + seg);
  constexpr int R = 8;   // rounds whose indices are loaded together
  for (int b0 = s0; b0 < s1; b0 += 32 * R) {
    int ev[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int p = b0 + r * 32 + lane;
      ev[r] = p < s1 ? assign_expert(idx, p, topk, k_in, shared_e) : -1;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int p = b0 + r * 32 + lane;
      int e = ev[r];
      if (p < s1 && e != -1 && (e < 0 || e >= E)) {
        set_status(status, DSV4_EINVAL);
        e = -1;
      }
      if (p < s1 && e < 0) inv[p] = -1;   // empty (-1) or rejected assignment
      const unsigned same = match_small(e, ebits);
      if (e >= 0 && (same & ((1u << lane) - 1u)) == 0u) wcn[warp * E + e] += (uint32_t)__popc(same);
      __syncwarp();
    }
  }
  __syncthreads();
  // per expert: exclusive prefix over the warps, in place, and the total
  for (int x = tid; x < E; x += AL_THREADS) {
    uint32_t sum = 0;
    for (int w = 0; w < 32; ++w) {
      const uint32_t v = wcn[w * E + x];
      wcn[w * E + x] = sum;
      sum += v;
    }
    cnt[x] = (int)sum;
  }
  __syncthreads();
  // exclusive scan of the (padded) group sizes (E <= 1024: one expert per thread)
  int total = 0;
  const int c = tid < E ? cnt[tid] : 0;
  const int cpad = (c + pad - 1) / pad * pad;
  const int off = block_exclusive_scan(cpad, scratch, &total);
  if (tid < E) {
    run[tid] = off;
    counts[tid] = c;
    offsets[tid] = off;
  }
  if (tid == 0) offsets[E] = total;
  __syncthreads();
  // padding rows of each group (fewer than `pad`), one warp per group so the
  // stores of a warp are contiguous
  for (int e = warp; e < E; e += AL_THREADS / 32) {
    const int r0 = run[e] + cnt[e], r1 = run[e] + (cnt[e] + pad - 1) / pad * pad;
    for (int r = r0 + lane; r < r1; r += 32) {
      sorted_flat[r] = -1;
      if (sorted_w) sorted_w[r] = 0.f;
    }
  }
  // pass 2: positions, in assignment order
  for (int b0 = s0; b0 < s1; b0 += 32 * R) {
    int ev[R];
    float wv[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int p = b0 + r * 32 + lane;
      ev[r] = p < s1 ? assign_expert(idx, p, topk, k_in, shared_e) : -1;
      wv[r] = (p < s1 && sorted_w) ? assign_weight(w_flat, p, topk, k_in, shared_e) : 0.f;
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int p = b0 + r * 32 + lane;
      int e = ev[r];
      if (e < 0 || e >= E) e = -1;
      const unsigned same = match_small(e, ebits);
      const int rank = __popc(same & ((1u << lane) - 1u));
      if (e >= 0) {
        const int pos = run[e] + (int)wcn[warp * E + e] + rank;
        sorted_flat[pos] = p;
        inv[p] = pos;
        if (sorted_w) sorted_w[pos] = wv[r];
      }
      __syncwarp();
      if (e >= 0 && rank == 0) wcn[warp * E + e] += (uint32_t)__popc(same);
      __syncwarp();
    }
  }

  // active experts, ascending
  int nact = 0;
  const int flag = (tid < E && cnt[tid] > 0) ? 1 : 0;
  const int apos = block_exclusive_scan(flag, scratch, &nact);
  if (flag) active[apos] = tid;
  if (tid == 0) *n_active = nact;
  // work chunks: one pad-row block of one expert each
  if (chunks) {
    const int nch = cpad / pad;
    int nchunk_total = 0;
    const int cpos = block_exclusive_scan(nch, scratch, &nchunk_total);
    for (int j = 0; j < nch; ++j) {
      const int r0 = off + j * pad;
      chunks[cpos + j] = make_int4(tid, r0, min(pad, c - j * pad), nch > 1);
    }
    if (tid == 0) *n_chunks = nchunk_total;
  }
}

// ---------------------------------------------------------------------------
// moe_align for large batches on many CTAs (the same stable counting sort):
//   count  CTA b takes assignments [1024 b, 1024 b + 1024), one per thread,
//          and writes its per-expert counts cnt_blk[b][E];
//   scan   one CTA: per expert, the exclusive prefix over the blocks and the
//          total; the padded group offsets, active list and GEMM chunks as
//          the one-CTA kernel; cnt_blk becomes each block's start row inside
//          each group; padding rows;
//   place  CTA b again: an assignment's row is its block's start in its
//          expert's group plus its rank among the block's earlier equal
//          experts (warp ballots + per-warp counts), so the order stays
//          token-major within an expert.
// The token count may be known only on the device (n_tokens_dev); CTAs past
// it do nothing.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int align_count_p(int P, int topk, const int32_t* __restrict__ n_tokens_dev) {
  return n_tokens_dev ? min(P, max(0, *n_tokens_dev) * topk) : P;
}

// ranks of this CTA's assignments among equal experts of the CTA: returns
// the rank, leaves per-expert counts of the CTA in cnt[E] (smem)
__device__ __forceinline__ int block_rank(int e, int E, int ebits, uint16_t* wc, int* cnt) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t* wc32 = reinterpret_cast<uint32_t*>(wc);
  for (int j = tid; j < 16 * E; j += AL_THREADS) wc32[j] = 0u;
  __syncthreads();
  const unsigned same = match_small(e, ebits);
  const int rank = __popc(same & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) wc[warp * E + e] = (uint16_t)__popc(same);
  __syncthreads();
  for (int x = tid; x < E; x += AL_THREADS) {
    int c = 0;
    for (int w = 0; w < 32; ++w) {
      const int v = wc[w * E + x];
      wc[w * E + x] = (uint16_t)c;
      c += v;
    }
    cnt[x] = c;
  }
  __syncthreads();
  return e >= 0 ? (int)wc[warp * E + e] + rank : -1;
}

__device__ __forceinline__ int align_read(const int32_t* __restrict__ idx, int a, int P, int topk, int E, int k_in,
                                          int shared_e, int* status, int32_t* __restrict__ inv, bool write_inv) {
  if (a >= P) return -1;
  int e = assign_expert(idx, a, topk, k_in, shared_e);
  if (e == -1) {
    if (write_inv) inv[a] = -1;
  } else if (e < 0 || e >= E) {
    if (write_inv) {
      set_status(status, DSV4_EINVAL);
      inv[a] = -1;
    }
    e = -1;
  }
  return e;
}

__global__ void __launch_bounds__(AL_THREADS, 1)
    align_count_kernel(const int32_t* __restrict__ idx, int P, int topk, int E, int k_in, int shared_e,
                       const int32_t* __restrict__ n_tokens_dev, int32_t* __restrict__ cnt_blk, int* status) {
  extern __shared__ int sm[];
  int* cnt = sm;                                              // E
  uint16_t* wc = reinterpret_cast<uint16_t*>(cnt + E);       // [32][E]
  griddep_wait();
  griddep_launch();
  P = align_count_p(P, topk, n_tokens_dev);
  if ((int64_t)blockIdx.x * AL_THREADS >= P) return;
  const int ebits = 32 - __clz(max(E - 1, 1));
  const int a = blockIdx.x * AL_THREADS + threadIdx.x;
  const int e = align_read(idx, a, P, topk, E, k_in, shared_e, status, nullptr, false);
  block_rank(e, E, ebits, wc, cnt);
  for (int x = threadIdx.x; x < E; x += AL_THREADS) cnt_blk[(int64_t)blockIdx.x * E + x] = cnt[x];
}

__global__ void __launch_bounds__(AL_THREADS, 1)
    align_scan_kernel(int P, int topk, int E, const int32_t* __restrict__ n_tokens_dev, int32_t* __restrict__ cnt_blk,
                      int32_t* __restrict__ counts, int32_t* __restrict__ offsets, int32_t* __restrict__ sorted_flat,
                      int32_t* __restrict__ active, int32_t* __restrict__ n_active, float* __restrict__ sorted_w,
                      int4* __restrict__ chunks, int32_t* __restrict__ n_chunks, int pad,
                      int* __restrict__ chunk_done, int max_chunks) {
  __shared__ int scratch[96];
  __shared__ int run_s[1024], cnt_s[1024];
  griddep_wait();
  griddep_launch();
  P = align_count_p(P, topk, n_tokens_dev);
  const int nblk = (P + AL_THREADS - 1) / AL_THREADS;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int j = tid; j < max_chunks; j += AL_THREADS) chunk_done[j] = 0;
  int c = 0;
  if (tid < E) {
    for (int b = 0; b < nblk; ++b) {
      const int v = cnt_blk[(int64_t)b * E + tid];
      cnt_blk[(int64_t)b * E + tid] = c;
      c += v;
    }
  }
  const int cpad = (c + pad - 1) / pad * pad;
  const int nch = cpad / pad;
  int3 tot3;
  const int3 ex = block_scan3(cpad, c > 0 ? 1 : 0, nch, scratch, &tot3);
  if (tid < E) {
    run_s[tid] = ex.x;
    cnt_s[tid] = c;
    counts[tid] = c;
    offsets[tid] = ex.x;
    if (c > 0) active[ex.y] = tid;
    if (chunks)
      for (int j = 0; j < nch; ++j)
        chunks[ex.z + j] = make_int4(tid, ex.x + j * pad, min(pad, c - j * pad), nch > 1);
    for (int b = 0; b < nblk; ++b) cnt_blk[(int64_t)b * E + tid] += ex.x;   // absolute start rows
  }
  if (tid == 0) {
    offsets[E] = tot3.x;
    *n_active = tot3.y;
    if (chunks) *n_chunks = tot3.z;
  }
  __syncthreads();
  for (int g = warp; g < E; g += AL_THREADS / 32) {
    const int r0 = run_s[g] + cnt_s[g], r1 = run_s[g] + (cnt_s[g] + pad - 1) / pad * pad;
    for (int r = r0 + lane; r < r1; r += 32) {
      sorted_flat[r] = -1;
      if (sorted_w) sorted_w[r] = 0.f;
    }
  }
}

__global__ void __launch_bounds__(AL_THREADS, 1)
    align_place_kernel(const int32_t* __restrict__ idx, int P, int topk, int E, int k_in, int shared_e,
                       const float* __restrict__ w_flat, const int32_t* __restrict__ n_tokens_dev,
                       const int32_t* __restrict__ start_blk, int32_t* __restrict__ sorted_flat,
                       int32_t* __restrict__ inv, float* __restrict__ sorted_w, int* status) {
  extern __shared__ int sm[];
  int* cnt = sm;
  uint16_t* wc = reinterpret_cast<uint16_t*>(cnt + E);
  griddep_wait();
  griddep_launch();
  P = align_count_p(P, topk, n_tokens_dev);
  if ((int64_t)blockIdx.x * AL_THREADS >= P) return;
  const int ebits = 32 - __clz(max(E - 1, 1));
  const int a = blockIdx.x * AL_THREADS + threadIdx.x;
  const int e = align_read(idx, a, P, topk, E, k_in, shared_e, status, inv, true);
  const int r = block_rank(e, E, ebits, wc, cnt);
  if (e >= 0) {
    const int pos = start_blk[(int64_t)blockIdx.x * E + e] + r;
    sorted_flat[pos] = a;
    inv[a] = pos;
    if (sorted_w) sorted_w[pos] = assign_weight(w_flat, a, topk, k_in, shared_e);
  }
}

// ---------------------------------------------------------------------------
// activation quant + gather into the GEMM B operand.  Assignment a = t*topk+j
// writes token t's row to its sorted row inv[a] (padding rows are never
// touched; invalid assignments, inv < 0, are skipped).  Scales
// go to 512-byte atoms, one per (128-column k-tile kt, 64-row block rb) at
// (kt * rb_cap + rb) * 512 for BN-row blocks (BN = 64 or 112, the GEMM
// tile), row n of the block (n = row % BN) at (n%32)*16 + (n/32)*4, one
// byte per 32-block (FP8: the per-128 exponent replicated four times): the
// order the tensor cores read after a 32x128b.warpx4 copy.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int64_t act_sf_offset(int64_t row, int kt, int64_t rb_cap, int bn) {
  const int n = (int)(row % bn);   // row inside its tile (tiles of 112 rows do not start on a 32-row boundary)
  return ((int64_t)kt * rb_cap + row / bn) * 512 + (n % 32) * 16 + (n / 32) * 4;
}

// One warp per (token, 128-column block): the token's row is read and
// quantised once, then written to the sorted rows of its topk assignments
// (inv[t*topk + j]), 4 bytes per lane per row; lanes 0..topk-1 store the
// rows' scale words.
// IN = DSV4_ROWS_BF16: x is [n_tokens][K] bf16, quantised here (FP8 per
// 128: one E4M3 byte per column and the block exponent fp8_scale_exp(amax);
// MXFP4 (a4w4) per 32: an E8M0 scale floor(log2(amax/6)) + 127 and E2M1
// codes, round to nearest even, saturating; lanes 8g..8g+7 own block g).
// IN = DSV4_ROWS_FP8 / DSV4_ROWS_MXFP4: x holds rows of row_bytes already
// quantised the same way at the token's source (the expert-parallel
// dispatch), codes then block scales; they are only gathered.
template <bool FP4, int IN>
__global__ void quant_gather_kernel(const uint8_t* __restrict__ x, int64_t row_bytes, const int32_t* __restrict__ inv,
                                    int64_t n_tokens, int topk, int K, int64_t rb_cap, int bn,
                                    uint8_t* __restrict__ q, uint8_t* __restrict__ sf,
                                    const int32_t* __restrict__ n_tokens_dev) {
  griddep_wait();
  griddep_launch();
  if (n_tokens_dev) n_tokens = min(n_tokens, (int64_t)max(0, *n_tokens_dev));
  const int lane = threadIdx.x & 31;
  const int kblk = K / 128;
  const int64_t ntask = n_tokens * kblk;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = warp0; b < ntask; b += nwarps) {
    const int64_t tok = b / kblk;
    const int kb = (int)(b - tok * kblk);
    const int my_row = lane < topk ? inv[tok * topk + lane] : -1;
    if (__ballot_sync(0xffffffffu, my_row >= 0) == 0u) continue;   // no assignment to write
    const uint8_t* xr = x + tok * row_bytes;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (IN == DSV4_ROWS_BF16) {
      const uint2 raw = *reinterpret_cast<const uint2*>(xr + (int64_t)(kb * 128 + lane * 4) * 2);
      v[0] = bf16_from_bits(raw.x & 0xffffu);
      v[1] = bf16_from_bits(raw.x >> 16);
      v[2] = bf16_from_bits(raw.y & 0xffffu);
      v[3] = bf16_from_bits(raw.y >> 16);
    }
    if constexpr (!FP4) {
      uint32_t o;
      int e;
      if constexpr (IN == DSV4_ROWS_BF16) {
        o = fp8_block_quant(v, &e);
      } else {
        o = *reinterpret_cast<const uint32_t*>(xr + kb * 128 + lane * 4);
        e = (int)xr[K + kb] - 127;
      }
      for (int j = 0; j < topk; ++j) {
        const int64_t row = __shfl_sync(0xffffffffu, my_row, j);
        if (row >= 0) *reinterpret_cast<uint32_t*>(q + row * K + kb * 128 + lane * 4) = o;
      }
      if (my_row >= 0)
        *reinterpret_cast<uint32_t*>(sf + act_sf_offset(my_row, kb, rb_cap, bn)) = (uint32_t)(e + 127) * 0x01010101u;
    } else {
      uint32_t packed, sword;
      if constexpr (IN == DSV4_ROWS_BF16) {
        int e;
        packed = mxfp4_block_quant(v, &e);
        // the four block scales of this 128-column block as one word
        sword = (uint32_t)(__shfl_sync(0xffffffffu, e, 0) + 127) |
                ((uint32_t)(__shfl_sync(0xffffffffu, e, 8) + 127) << 8) |
                ((uint32_t)(__shfl_sync(0xffffffffu, e, 16) + 127) << 16) |
                ((uint32_t)(__shfl_sync(0xffffffffu, e, 24) + 127) << 24);
      } else {
        packed = *reinterpret_cast<const uint16_t*>(xr + kb * 64 + lane * 2);
        sword = *reinterpret_cast<const uint32_t*>(xr + K / 2 + kb * 4);
      }
      for (int j = 0; j < topk; ++j) {
        const int64_t row = __shfl_sync(0xffffffffu, my_row, j);
        if (row >= 0) *reinterpret_cast<uint16_t*>(q + row * (K / 2) + kb * 64 + lane * 2) = (uint16_t)packed;
      }
      if (my_row >= 0) *reinterpret_cast<uint32_t*>(sf + act_sf_offset(my_row, kb, rb_cap, bn)) = sword;
    }
  }
}

// ---------------------------------------------------------------------------
// combine (deepseek_v4.py:195-197): y[t] = bf16(sum over the token's k rows,
// in ascending sorted position = ascending expert id, fp32 from zero).
// One block per token, eight columns per thread.
// ---------------------------------------------------------------------------
// grid (T, H / (8 * blockDim.x)): each CTA covers 8 * blockDim.x columns.
// `extra` (bf16 [T, H] or null): a row added after the k expert rows (the
// shared expert's output when it ran as a separate pass, model_npu.py:532).
__global__ void combine_kernel(const uint16_t* __restrict__ out, const int32_t* __restrict__ inv, int topk, int H,
                               uint16_t* __restrict__ y, int64_t T, const int32_t* __restrict__ n_tokens_dev,
                               const uint16_t* __restrict__ extra) {
  griddep_wait();
  griddep_launch();
  const int64_t t = blockIdx.x;
  if (t >= T || (n_tokens_dev && t >= *n_tokens_dev)) return;
  int pos[16];
  int k = 0;
  for (int j = 0; j < topk; ++j) {
    const int v = inv[t * topk + j];
    if (v < 0) continue;
    int i = k++;
    while (i > 0 && pos[i - 1] > v) {
      pos[i] = pos[i - 1];
      --i;
    }
    pos[i] = v;
  }
  // a token without any assignment (every id -1: padding of the expert-
  // parallel exchange) has no output row to write
  if (k == 0 && !extra) return;
  for (int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8; c < H; c += gridDim.y * blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // the rows' loads are issued together (up to 8 in flight), then added
    // in ascending position
    for (int j0 = 0; j0 < k; j0 += 8) {
      uint4 r[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (j0 + u < k) r[u] = *reinterpret_cast<const uint4*>(out + (int64_t)pos[j0 + u] * H + c);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (j0 + u < k) {
          const uint32_t w[4] = {r[u].x, r[u].y, r[u].z, r[u].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            acc[2 * q] += bf16_from_bits(w[q] & 0xffffu);
            acc[2 * q + 1] += bf16_from_bits(w[q] >> 16);
          }
        }
      }
    }
    if (extra) {
      const uint4 r = *reinterpret_cast<const uint4*>(extra + t * H + c);
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += bf16_from_bits(w[q] & 0xffffu);
        acc[2 * q + 1] += bf16_from_bits(w[q] >> 16);
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) o[q] = (uint32_t)bf16_bits(acc[2 * q]) | ((uint32_t)bf16_bits(acc[2 * q + 1]) << 16);
    *reinterpret_cast<uint4*>(y + t * H + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Same sum, rows taken in the caller's order (no sorting).
__global__ void combine_ordered_kernel(const uint16_t* __restrict__ rows, const int32_t* __restrict__ order,
                                       int topk, int H, uint16_t* __restrict__ y, int64_t T) {
  griddep_wait();
  griddep_launch();
  const int64_t t = blockIdx.x;
  if (t >= T) return;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < topk; ++j) {
      const int pos = order[t * topk + j];
      if (pos < 0) continue;
      const uint4 r = *reinterpret_cast<const uint4*>(rows + (int64_t)pos * H + c);
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += bf16_from_bits(w[q] & 0xffffu);
        acc[2 * q + 1] += bf16_from_bits(w[q] >> 16);
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) o[q] = (uint32_t)bf16_bits(acc[2 * q]) | ((uint32_t)bf16_bits(acc[2 * q + 1]) << 16);
    *reinterpret_cast<uint4*>(y + t * H + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------------------
// plan
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encoder() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int make_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, void* base, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box, const char* what, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = get_encoder();
  if (!enc) return fail(DSV4_ECUDA, "cuTensorMapEncodeTiled is not available");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i < rank - 1) s[i] = strides_bytes[i];
  }
  CUresult r = enc(m, dt, (cuuint32_t)rank, base, d, s, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DSV4_ECUDA, std::string("tensor map encode failed for ") + what +
                                                     " (CUresult " + std::to_string((int)r) + ")");
  return DSV4_OK;
}

// Gate/up and down GEMMs in one launch: 1 always, 0 never, -1 (default)
// with the 64-token decode tile only.  Measured on config 1 / 2 (graph
// replay): equal to the two PDL-chained launches at T = 1-64, 2.5 % slower
// at the 112-token prefill tile, whose SwiGLU epilogue is the longest role.
// DSV4_FUSED_FFN=0|1 overrides the default.
static int fused_ffn_default() {
  const char* e = getenv("DSV4_FUSED_FFN");
  if (e && e[0] == '0') return 0;
  if (e && e[0] == '1') return 1;
  return -1;
}

struct WsLayout {
  int64_t status, counts, offsets, active, n_active, n_chunks, sorted_flat, inv, sorted_w, chunks;
  int64_t xq, xsf, hq, hsf, out, ys, blk, done, rbar, rpart, bytes;
  int64_t p_max, p_cap, max_chunks;
};

static int64_t al256(int64_t v) { return (v + 255) / 256 * 256; }

// E and topk count the shared expert when the plan has one; `shared`
// adds the [max_tokens, H] bf16 output of its separate pass (a4w4 profile).
static WsLayout ws_layout(int64_t H, int64_t I, int64_t E, int64_t topk, int64_t max_tokens, bool shared = false) {
  WsLayout w;
  w.p_max = max_tokens * topk;
  // every expert group is padded to a multiple of the GEMM tile (64 or 112
  // rows): room for padding up to 128 rows, and a tile of slack at the end
  w.p_cap = (w.p_max + (GEMM_BN_MAX - 1) * std::min<int64_t>(E, w.p_max) + GEMM_BN_MAX - 1) / GEMM_BN_MAX *
                GEMM_BN_MAX + GEMM_BN_MAX;
  w.max_chunks = w.p_cap / G_BN + 1;
  int64_t o = 0;
  auto take = [&](int64_t bytes) {
    const int64_t at = o;
    o = al256(o + bytes);
    return at;
  };
  w.status = take(16);
  w.counts = take(4 * E);
  w.offsets = take(4 * (E + 1));
  w.active = take(4 * E);
  w.n_active = take(4);
  w.n_chunks = take(4);
  w.sorted_flat = take(4 * w.p_cap);  // indexed by padded row position
  w.inv = take(4 * std::max<int64_t>(w.p_max, 1));
  w.sorted_w = take(4 * w.p_cap);
  w.chunks = take(16 * w.max_chunks);
  w.xq = take(w.p_cap * H);
  w.xsf = take((H / 128) * (w.p_cap / G_BN) * 512);
  w.hq = take(w.p_cap * I);
  w.hsf = take((I / 128) * (w.p_cap / G_BN) * 512);
  w.out = take(2 * w.p_cap * H);
  w.ys = shared ? take(2 * max_tokens * H) : 0;
  w.blk = take(4 * E * ((w.p_max + AL_THREADS - 1) / AL_THREADS + 1));   // per-block counts of the large align
  w.done = take(4 * w.max_chunks);   // finished gate/up tiles per chunk (fused launch)
  // decode router (dsv4_moe_route): its grid barrier, zero between launches,
  // and its partial logits for up to 255 tokens
  w.rbar = take(256);
  w.rpart = take(route_fused_part_bytes(std::min<int64_t>(max_tokens, 255), (int)H, (int)(E - (shared ? 1 : 0))));
  w.bytes = o;
  return w;
}

}  // namespace dsv4

struct dsv4_moe_plan {
  int device = 0;
  int num_sms = 148;
  int H = 0, I = 0, E = 0, topk = 0;   // E and topk include the shared expert when the plan has one
  bool shared = false;                  // expert E - 1 is the shared expert, every token's last assignment
  int64_t max_tokens = 0;
  float swiglu_limit = 0.f;
  uint8_t* arena = nullptr;
  int64_t n_slots = 0;
  dsv4::SlotLayout slot;
  uint8_t* ws = nullptr;
  dsv4::WsLayout wl;
  CUtensorMap tmA13, tmA2;      // weights expanded to one byte per element (bf16 profile)
  CUtensorMap tmA13p, tmA2p;    // weights packed, two per byte (a4w4)
  CUtensorMap tmB1_fp8[4], tmB1_fp4[4], tmB2_fp8[4], tmB2_fp4[4];  // 16, 32, 64, 112 activation rows per box
  bool timing = false;
  int gemm_tile = 0;   // tokens per GEMM tile; 0 = default
  int fused_ffn = -1;   // gate/up and down GEMMs in one launch: 1, 0, -1 = with the 64-token tile
  cudaEvent_t ev[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  ~dsv4_moe_plan() {
    for (auto& e : ev)
      if (e) cudaEventDestroy(e);
  }
};

using namespace dsv4;

template <typename T>
static T* wsp(dsv4_moe_plan* p, int64_t off) {
  return reinterpret_cast<T*>(p->ws + off);
}

extern "C" int64_t dsv4_moe_workspace_bytes_ex(int32_t hidden, int32_t inter, int32_t n_experts, int32_t topk,
                                               int64_t max_tokens, int32_t with_shared) {
  if (hidden <= 0 || inter <= 0 || n_experts <= 0 || topk <= 0 || max_tokens < 0) return DSV4_EINVAL;
  const int sh = with_shared ? 1 : 0;
  return ws_layout(hidden, inter, n_experts + sh, topk + sh, max_tokens, sh).bytes;
}

extern "C" int64_t dsv4_moe_workspace_bytes(int32_t hidden, int32_t inter, int32_t n_experts, int32_t topk,
                                            int64_t max_tokens) {
  return dsv4_moe_workspace_bytes_ex(hidden, inter, n_experts, topk, max_tokens, 0);
}

// The shared-memory opt-in is a per-device function attribute: set it for
// the current device every time a plan is created.
template <int NUM_A, bool B_FP4, int EPI>
static int prepare_gemm() {
  DSV4_CUDA_CHECK(cudaFuncSetAttribute(moe_gemm_kernel<NUM_A, B_FP4, EPI, 64, false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       GemmCfg<NUM_A, 64, B_FP4>::SMEM_BYTES));
  DSV4_CUDA_CHECK(cudaFuncSetAttribute(moe_gemm_kernel<NUM_A, B_FP4, EPI, 112, false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       GemmCfg<NUM_A, 112, B_FP4>::SMEM_BYTES));
  if constexpr (EPI != EPI_STORE_BF16) {
    DSV4_CUDA_CHECK(cudaFuncSetAttribute(moe_gemm_kernel<NUM_A, B_FP4, EPI, 64, true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GemmCfg<NUM_A, 64, B_FP4>::SMEM_BYTES));
    DSV4_CUDA_CHECK(cudaFuncSetAttribute(moe_gemm_kernel<NUM_A, B_FP4, EPI, 112, true>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GemmCfg<NUM_A, 112, B_FP4>::SMEM_BYTES));
  }
  return DSV4_OK;
}

// The GEMM tile: the plan's setting, else the environment's
// (DSV4_GEMM_BN=64|112), else by batch size.  A 112-token tile issues 1.75x
// fewer MMA instructions per token than a 64-token one, at the cost of more
// padding rows per expert group (and, with FP8 activations, a 4-stage ring
// instead of 5).  Decode batches (a few rows per expert) take 64.  a4w4
// (packed operands, an 8-stage ring at both widths) takes the wide tile from
// 16 assignments per expert on average (T = 512 at top-8 of 256): measured
// 1.08x faster on the layer at T = 512, 1.17x at 2048.  The bf16 profile,
// which gives up a ring stage for it, from 32 per expert.
static int gemm_bn(int plan_bn, int64_t assignments, int n_experts, bool packed) {
  static const int env_bn = [] {
    const char* e = getenv("DSV4_GEMM_BN");
    return e ? atoi(e) : 0;
  }();
  if (plan_bn == 64 || plan_bn == 112) return plan_bn;
  if (env_bn == 64 || env_bn == 112) return env_bn;
  return assignments >= (packed ? 16 : 32) * (int64_t)n_experts ? 112 : 64;
}

static GemmMaps gemm_maps(int bn, const CUtensorMap& tmA, const CUtensorMap* tmB, const CUtensorMap& tmAsh) {
  GemmMaps m;
  m.A = tmA;
  m.B16 = tmB[0];
  m.B32 = tmB[1];
  m.B64 = tmB[2];
  m.Bwide = bn == 112 ? tmB[3] : tmB[2];
  m.Ash = tmAsh;
  return m;
}

// One GEMM (m0, g0; m1 and g1 unused copies), or with FUSED the gate/up
// GEMM (m0, g0) and the down GEMM (m1, g1) in one launch.
template <bool B_FP4, int EPI, bool FUSED>
static cudaError_t launch_gemm(int bn, cudaStream_t st, bool pdl, int num_sms, const GemmMaps& m0,
                               const GemmParams& g0, const GemmMaps& m1, const GemmParams& g1) {
  const dim3 grid(num_sms), block(G_THREADS);
  if (bn == 112)
    return launch_k(moe_gemm_kernel<2, B_FP4, EPI, 112, FUSED>, grid, block, GemmCfg<2, 112, B_FP4>::SMEM_BYTES, st,
                    pdl, m0, g0, m1, g1);
  return launch_k(moe_gemm_kernel<2, B_FP4, EPI, 64, FUSED>, grid, block, GemmCfg<2, 64, B_FP4>::SMEM_BYTES, st, pdl,
                  m0, g0, m1, g1);
}

// Tensor maps of the shared expert's FP8 slot (w13 and w2 blocks, UINT8,
// 128-byte swizzle): the same boxes as the packed weights expanded by TMA.
static int shared_maps(const dsv4_moe_plan* p, const uint8_t* slot, CUtensorMap* m13, CUtensorMap* m2) {
  const SlotLayout L = shared_slot_layout(p->H, p->I);
  const uint64_t H = p->H, I = p->I, SB = (uint64_t)L.bytes;
  const uint32_t box[5] = {G_BK, 2 * G_BM, 1, 1, 1};
  const CUtensorMapDataType U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  {
    const uint64_t kt = H / 128, np = I / 128;
    const uint64_t dims[5] = {128, 256, kt, np, 1}, str[4] = {128, 32768, kt * 32768, SB};
    if (int rc = make_map(m13, U8, 5, (void*)(slot + L.w13p), dims, str, box, "shared w13")) return rc;
  }
  {
    const uint64_t kt = I / 128, np = H / 256;
    const uint64_t dims[5] = {128, 256, kt, np, 1}, str[4] = {128, 32768, kt * 32768, SB};
    if (int rc = make_map(m2, U8, 5, (void*)(slot + L.w2p), dims, str, box, "shared w2")) return rc;
  }
  return DSV4_OK;
}

extern "C" int dsv4_moe_plan_create_ex(dsv4_moe_plan** out, int32_t hidden, int32_t inter, int32_t n_experts,
                                       int32_t topk, int64_t max_tokens, float swiglu_limit, uint8_t* slot_arena,
                                       int64_t n_slots, void* workspace, int64_t workspace_bytes,
                                       int32_t with_shared) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(out && slot_arena && workspace, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && inter > 0 && hidden % 256 == 0 && inter % 128 == 0,
                 "hidden must be a positive multiple of 256 and inter of 128");
  const int sh = with_shared ? 1 : 0;
  DSV4_CHECK_ARG(n_experts > 0 && n_experts + sh <= 1024, "n_experts must be in [1, 1024]");
  DSV4_CHECK_ARG(topk > 0 && topk + sh <= 16, "topk must be in [1, 16]");
  DSV4_CHECK_ARG(max_tokens > 0 && n_slots > 0, "max_tokens and n_slots must be positive");
  DSV4_CHECK_ARG(((uintptr_t)slot_arena % 256) == 0 && ((uintptr_t)workspace % 256) == 0,
                 "slot arena and workspace must be 256-byte aligned");
  n_experts += sh;
  topk += sh;
  const WsLayout wl = ws_layout(hidden, inter, n_experts, topk, max_tokens, sh);
  DSV4_CHECK_ARG(workspace_bytes >= wl.bytes, "workspace too small");
  std::unique_ptr<dsv4_moe_plan> p(new dsv4_moe_plan());
  int rc0 = bind_device_of(slot_arena, &p->device);
  if (rc0 != 0) return rc0;
  DSV4_CUDA_CHECK(cudaDeviceGetAttribute(&p->num_sms, cudaDevAttrMultiProcessorCount, p->device));
  p->H = hidden;
  p->I = inter;
  p->E = n_experts;
  p->topk = topk;
  p->shared = sh != 0;
  p->max_tokens = max_tokens;
  p->swiglu_limit = swiglu_limit;
  p->fused_ffn = fused_ffn_default();
  p->arena = slot_arena;
  p->n_slots = n_slots;
  p->slot = slot_layout(hidden, inter);
  p->ws = (uint8_t*)workspace;
  p->wl = wl;
  DSV4_CUDA_CHECK(cudaMemset(workspace, 0, (size_t)wl.bytes));
  const uint64_t H = hidden, I = inter, SB = (uint64_t)p->slot.bytes, PC = (uint64_t)wl.p_cap;
  const CUtensorMapDataType U4 = CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  int rc;
  // weights are stored as contiguous 16 KiB blocks of a 256-row pair x 128 E2M1
  // elements (slot_layout.h): dims (element, row in pair, k tile, pair, slot)
  {  // w13: I/128 pairs (w1 tile, w3 tile), K = H
    const uint64_t kt = H / 128, np = I / 128;
    const uint64_t dims[5] = {128, 256, kt, np, (uint64_t)n_slots}, str[4] = {64, 16384, kt * 16384, SB};
    const uint32_t box[5] = {G_BK, 2 * G_BM, 1, 1, 1};
    if ((rc = make_map(&p->tmA13, U4, 5, slot_arena + p->slot.w13p, dims, str, box, "w13")) != 0) return rc;
    const uint64_t dimsp[5] = {64, 256, kt, np, (uint64_t)n_slots};   // packed: 64 bytes per row
    const uint32_t boxp[5] = {64, 2 * G_BM, 1, 1, 1};
    if ((rc = make_map(&p->tmA13p, U8, 5, slot_arena + p->slot.w13p, dimsp, str, boxp, "w13 packed",
                       CU_TENSOR_MAP_SWIZZLE_64B)) != 0)
      return rc;
  }
  {  // w2: H/256 pairs of 128-row tiles, K = I
    const uint64_t kt = I / 128, np = H / 256;
    const uint64_t dims[5] = {128, 256, kt, np, (uint64_t)n_slots}, str[4] = {64, 16384, kt * 16384, SB};
    const uint32_t box[5] = {G_BK, 2 * G_BM, 1, 1, 1};
    if ((rc = make_map(&p->tmA2, U4, 5, slot_arena + p->slot.w2p, dims, str, box, "w2")) != 0) return rc;
    const uint64_t dimsp[5] = {64, 256, kt, np, (uint64_t)n_slots};
    const uint32_t boxp[5] = {64, 2 * G_BM, 1, 1, 1};
    if ((rc = make_map(&p->tmA2p, U8, 5, slot_arena + p->slot.w2p, dimsp, str, boxp, "w2 packed",
                       CU_TENSOR_MAP_SWIZZLE_64B)) != 0)
      return rc;
  }
  const uint32_t brows[4] = {16, 32, 64, 112};
  // activations: FP8 one byte per element (128-byte swizzle), E2M1 packed
  // two per byte (64-byte swizzle, 64 bytes per row of a k-tile)
  for (int j = 0; j < 4; ++j) {
    const uint32_t bbox[2] = {G_BK, brows[j]}, bboxp[2] = {G_BK / 2, brows[j]};
    const CUtensorMapSwizzle SW64 = CU_TENSOR_MAP_SWIZZLE_64B;
    {
      const uint64_t dims[2] = {H, PC}, dimsp[2] = {H / 2, PC}, s8[1] = {H}, s4[1] = {H / 2};
      if ((rc = make_map(&p->tmB1_fp8[j], U8, 2, p->ws + wl.xq, dims, s8, bbox, "x fp8")) != 0) return rc;
      if ((rc = make_map(&p->tmB1_fp4[j], U8, 2, p->ws + wl.xq, dimsp, s4, bboxp, "x fp4", SW64)) != 0) return rc;
    }
    {
      const uint64_t dims[2] = {I, PC}, dimsp[2] = {I / 2, PC}, s8[1] = {I}, s4[1] = {I / 2};
      if ((rc = make_map(&p->tmB2_fp8[j], U8, 2, p->ws + wl.hq, dims, s8, bbox, "h fp8")) != 0) return rc;
      if ((rc = make_map(&p->tmB2_fp4[j], U8, 2, p->ws + wl.hq, dimsp, s4, bboxp, "h fp4", SW64)) != 0) return rc;
    }
  }
  if ((rc = prepare_gemm<2, false, EPI_SWIGLU_FP8>()) != 0) return rc;
  if ((rc = prepare_gemm<2, true, EPI_SWIGLU_MXFP4>()) != 0) return rc;
  if ((rc = prepare_gemm<2, false, EPI_STORE_BF16>()) != 0) return rc;
  if ((rc = prepare_gemm<2, true, EPI_STORE_BF16>()) != 0) return rc;
  const size_t al_smem = (size_t)(2 * n_experts + 32 + AL_THREADS) * 4 + (size_t)32 * n_experts * 4;
  DSV4_CUDA_CHECK(
      cudaFuncSetAttribute(moe_align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)al_smem));
  const size_t blk_smem = (size_t)n_experts * 4 + (size_t)32 * n_experts * 2;
  DSV4_CUDA_CHECK(
      cudaFuncSetAttribute(align_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)blk_smem));
  DSV4_CUDA_CHECK(
      cudaFuncSetAttribute(align_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)blk_smem));
  *out = p.release();
  DSV4_API_END
}

extern "C" int dsv4_moe_plan_create(dsv4_moe_plan** out, int32_t hidden, int32_t inter, int32_t n_experts,
                                    int32_t topk, int64_t max_tokens, float swiglu_limit, uint8_t* slot_arena,
                                    int64_t n_slots, void* workspace, int64_t workspace_bytes) {
  return dsv4_moe_plan_create_ex(out, hidden, inter, n_experts, topk, max_tokens, swiglu_limit, slot_arena, n_slots,
                                 workspace, workspace_bytes, 0);
}

extern "C" int dsv4_moe_plan_destroy(dsv4_moe_plan* plan) {
  delete plan;
  return DSV4_OK;
}

// One pass of the layer over `n_tokens` tokens with `topk` assignments each
// (the router's k_in picks, plus the shared expert `shared_e` as the last one
// when shared_e >= 0): align, activation quant + gather, the two GEMMs and
// the combine into y (skipped when y is null), `extra` added last.
struct PassArgs {
  bool fp4;
  int topk, k_in, shared_e;
  const CUtensorMap* sh13;   // shared expert maps (with shared_e >= 0)
  const CUtensorMap* sh2;
  const uint8_t* shared_slot;
  const uint16_t* extra;
  bool timed;                // records the stage events
  uint16_t* const* assign_dst = nullptr;   // down GEMM scatter targets (expert parallelism)
  int x_format = DSV4_ROWS_BF16;           // rows of x: bf16, or quantised at their source
  int64_t x_row_bytes = 0;                 // bytes per row of a quantised x
};

static int moe_pass(dsv4_moe_plan* p, const PassArgs& a, const void* x_bf16, int64_t n_tokens,
                    const int32_t* n_tokens_dev, const float* route_weights, const int32_t* route_indices,
                    const int32_t* slot_of_expert, void* y_bf16, cudaStream_t st) {
  const WsLayout& w = p->wl;
  const int P = (int)(n_tokens * a.topk);
  const int bn = gemm_bn(p->gemm_tile, P, p->E, a.fp4);   // GEMM tile = group padding
  int* status = wsp<int>(p, w.status);
  int32_t* sorted_flat = wsp<int32_t>(p, w.sorted_flat);
  int32_t* inv = wsp<int32_t>(p, w.inv);
  int32_t* n_active = wsp<int32_t>(p, w.n_active);
  int* n_chunks = wsp<int>(p, w.n_chunks);
  const size_t al_smem = (size_t)(2 * p->E + 32 + AL_THREADS) * 4 + (size_t)32 * p->E * 4;
  auto mark = [&](int i) {
    if (p->timing && a.timed) cudaEventRecord(p->ev[i], st);
  };
  // events between stages break the programmatic overlap: no PDL while timing
  const bool pdl = pdl_enabled() && !p->timing;
  mark(0);
  if (P <= AL_THREADS) {
    DSV4_CUDA_CHECK(launch_k(moe_align_kernel, dim3(1), dim3(AL_THREADS), al_smem, st, pdl, route_indices, P,
                             a.topk, p->E, route_weights, wsp<int32_t>(p, w.counts), wsp<int32_t>(p, w.offsets),
                             sorted_flat, inv, wsp<int32_t>(p, w.active), n_active, wsp<float>(p, w.sorted_w),
                             wsp<int4>(p, w.chunks), n_chunks, bn, status, n_tokens_dev, a.k_in, a.shared_e,
                             wsp<int>(p, w.done), (int)w.max_chunks));
  } else {
    // large batches: count per block, scan on one CTA, place per block
    const unsigned nblk = (unsigned)((P + AL_THREADS - 1) / AL_THREADS);
    const size_t blk_smem = (size_t)p->E * 4 + (size_t)32 * p->E * 2;
    int32_t* cnt_blk = wsp<int32_t>(p, w.blk);
    DSV4_CUDA_CHECK(launch_k(align_count_kernel, dim3(nblk), dim3(AL_THREADS), blk_smem, st, pdl, route_indices, P,
                             a.topk, p->E, a.k_in, a.shared_e, n_tokens_dev, cnt_blk, status));
    DSV4_CUDA_CHECK(launch_k(align_scan_kernel, dim3(1), dim3(AL_THREADS), 0, st, pdl, P, a.topk, p->E,
                             n_tokens_dev, cnt_blk, wsp<int32_t>(p, w.counts), wsp<int32_t>(p, w.offsets),
                             sorted_flat, wsp<int32_t>(p, w.active), n_active, wsp<float>(p, w.sorted_w),
                             wsp<int4>(p, w.chunks), n_chunks, bn, wsp<int>(p, w.done), (int)w.max_chunks));
    DSV4_CUDA_CHECK(launch_k(align_place_kernel, dim3(nblk), dim3(AL_THREADS), blk_smem, st, pdl, route_indices, P,
                             a.topk, p->E, a.k_in, a.shared_e, route_weights, n_tokens_dev,
                             (const int32_t*)cnt_blk, sorted_flat, inv, wsp<float>(p, w.sorted_w), status));
  }
  mark(1);
  const int64_t rb_cap = (w.p_cap + bn - 1) / bn;   // BN-row scale blocks per k-tile
  {
    const int64_t warps = n_tokens * (p->H / 128);
    int64_t blocks = (warps * 32 + 255) / 256;
    blocks = std::min<int64_t>(blocks, (int64_t)p->num_sms * 16);
    auto qk = a.x_format == DSV4_ROWS_FP8     ? quant_gather_kernel<false, DSV4_ROWS_FP8>
              : a.x_format == DSV4_ROWS_MXFP4 ? quant_gather_kernel<true, DSV4_ROWS_MXFP4>
              : a.fp4                         ? quant_gather_kernel<true, DSV4_ROWS_BF16>
                                              : quant_gather_kernel<false, DSV4_ROWS_BF16>;
    const int64_t row_bytes = a.x_format == DSV4_ROWS_BF16 ? 2 * (int64_t)p->H : a.x_row_bytes;
    DSV4_CUDA_CHECK(launch_k(qk, dim3((unsigned)blocks), dim3(256), 0, st, pdl, (const uint8_t*)x_bf16, row_bytes,
                             (const int32_t*)inv, n_tokens, a.topk, p->H, rb_cap, bn, p->ws + w.xq, p->ws + w.xsf,
                             n_tokens_dev));
  }
  mark(2);
  GemmParams g1{};
  g1.arena = p->arena;
  g1.slot_bytes = p->slot.bytes;
  g1.sfa_off = p->slot.sf13;
  g1.k_tiles = p->H / 128;
  g1.a_row_tiles = p->I / 128;   // one (w1, w3) tile pair per work tile
  g1.out_tile_cols = 128;
  g1.b_sf = p->ws + w.xsf;
  g1.rb_cap = rb_cap;
  g1.chunks = wsp<int4>(p, w.chunks);
  g1.n_chunks = n_chunks;
  g1.slot_of = slot_of_expert;
  g1.n_slots = (int)p->n_slots;
  g1.sorted_w = wsp<float>(p, w.sorted_w);
  g1.out_q = p->ws + w.hq;
  g1.out_sf = p->ws + w.hsf;
  g1.out_ld = p->I;
  g1.swiglu_limit = p->swiglu_limit;
  g1.status = status;
  g1.chunk_done = wsp<int>(p, w.done);
  g1.shared_expert = a.shared_e;
  g1.shared_slot = a.shared_slot;
  const SlotLayout sl = shared_slot_layout(p->H, p->I);
  g1.shared_sfa_off = sl.sf13;
  GemmParams g2 = g1;
  g2.sfa_off = p->slot.sf2;
  g2.shared_sfa_off = sl.sf2;
  g2.k_tiles = p->I / 128;
  g2.a_row_tiles = p->H / 256;   // two 128-row tiles of w2 per work tile
  g2.out_tile_cols = 256;
  g2.b_sf = p->ws + w.hsf;
  g2.out_q = nullptr;
  g2.out_sf = nullptr;
  g2.out_bf16 = wsp<uint16_t>(p, w.out);
  g2.out_ld = p->H;
  g2.sorted_flat = sorted_flat;
  g2.assign_dst = a.assign_dst;
  // without a shared expert the kernels never read the shared maps; any
  // valid map fills the parameter
  const CUtensorMap& sh13 = a.sh13 ? *a.sh13 : p->tmA13;
  const CUtensorMap& sh2 = a.sh2 ? *a.sh2 : p->tmA2;
  const GemmMaps m1 = a.fp4 ? gemm_maps(bn, p->tmA13p, p->tmB1_fp4, sh13) : gemm_maps(bn, p->tmA13, p->tmB1_fp8, sh13);
  const GemmMaps m2 = a.fp4 ? gemm_maps(bn, p->tmA2p, p->tmB2_fp4, sh2) : gemm_maps(bn, p->tmA2, p->tmB2_fp8, sh2);
  if (p->fused_ffn == 1 || (p->fused_ffn < 0 && bn == 64)) {
    // gate/up, SwiGLU, requant and down in one persistent launch; the
    // stage events put its whole time under the gate/up stage
    if (a.fp4)
      DSV4_CUDA_CHECK((launch_gemm<true, EPI_SWIGLU_MXFP4, true>(bn, st, pdl, p->num_sms, m1, g1, m2, g2)));
    else
      DSV4_CUDA_CHECK((launch_gemm<false, EPI_SWIGLU_FP8, true>(bn, st, pdl, p->num_sms, m1, g1, m2, g2)));
    mark(3);
  } else {
    if (a.fp4)
      DSV4_CUDA_CHECK((launch_gemm<true, EPI_SWIGLU_MXFP4, false>(bn, st, pdl, p->num_sms, m1, g1, m1, g1)));
    else
      DSV4_CUDA_CHECK((launch_gemm<false, EPI_SWIGLU_FP8, false>(bn, st, pdl, p->num_sms, m1, g1, m1, g1)));
    mark(3);
    if (a.fp4)
      DSV4_CUDA_CHECK((launch_gemm<true, EPI_STORE_BF16, false>(bn, st, pdl, p->num_sms, m2, g2, m2, g2)));
    else
      DSV4_CUDA_CHECK((launch_gemm<false, EPI_STORE_BF16, false>(bn, st, pdl, p->num_sms, m2, g2, m2, g2)));
  }
  mark(4);
  if (y_bf16) {
    const int threads = std::min(128, p->H / 8);
    const unsigned gy = (unsigned)std::max(1, p->H / (8 * threads));
    DSV4_CUDA_CHECK(launch_k(combine_kernel, dim3((unsigned)n_tokens, gy), dim3(threads), 0, st, pdl,
                             (const uint16_t*)wsp<uint16_t>(p, w.out), (const int32_t*)inv, a.topk, p->H,
                             (uint16_t*)y_bf16, (int64_t)n_tokens, n_tokens_dev, a.extra));
  }
  mark(5);
  return DSV4_OK;
}

static int moe_forward_impl(dsv4_moe_plan* p, int32_t profile, const void* x_bf16, int64_t n_tokens,
                            const int32_t* n_tokens_dev, const float* route_weights, const int32_t* route_indices,
                            const int32_t* slot_of_expert, const uint8_t* shared_slot, void* y_bf16, void* stream,
                            uint16_t* const* assign_dst = nullptr, int x_format = DSV4_ROWS_BF16) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(p && x_bf16 && route_weights && route_indices && slot_of_expert, "null pointer");
  DSV4_CHECK_ARG(profile == DSV4_PROFILE_BF16 || profile == DSV4_PROFILE_A4W4, "unknown profile");
  DSV4_CHECK_ARG(n_tokens >= 0 && n_tokens <= p->max_tokens, "n_tokens exceeds the plan's max_tokens");
  DSV4_CHECK_ARG(((uintptr_t)x_bf16 % 16) == 0 && ((uintptr_t)y_bf16 % 16) == 0, "x and y must be 16-byte aligned");
  DSV4_CHECK_ARG(p->shared == (shared_slot != nullptr),
                 "a plan created with a shared expert needs its FP8 slot, and only such a plan takes one");
  DSV4_CHECK_ARG(((uintptr_t)shared_slot % 256) == 0, "the shared expert's slot must be 256-byte aligned");
  if (n_tokens == 0) return DSV4_OK;
  DSV4_CUDA_CHECK(cudaSetDevice(p->device));
  cudaStream_t st = (cudaStream_t)stream;
  const bool fp4 = profile == DSV4_PROFILE_A4W4;
  DSV4_CHECK_ARG(!assign_dst || (!y_bf16 && !p->shared), "scatter mode writes no y and runs no shared expert");
  DSV4_CHECK_ARG(x_format == DSV4_ROWS_BF16 || (!p->shared && x_format == (fp4 ? DSV4_ROWS_MXFP4 : DSV4_ROWS_FP8)),
                 "quantised rows must be in the profile's format (FP8 for bf16, MXFP4 for a4w4), without a shared "
                 "expert");
  if (!p->shared) {
    PassArgs a{fp4, p->topk, p->topk, -1, nullptr, nullptr, nullptr, nullptr, true, assign_dst};
    a.x_format = x_format;
    a.x_row_bytes = x_format == DSV4_ROWS_BF16 ? 0 : dsv4_ep_row_bytes(x_format, p->H);
    if (int rc = moe_pass(p, a, x_bf16, n_tokens, n_tokens_dev, route_weights, route_indices, slot_of_expert,
                          y_bf16, st))
      return rc;
  } else {
    CUtensorMap m13, m2;
    if (int rc = shared_maps(p, shared_slot, &m13, &m2)) return rc;
    const int k = p->topk - 1, shared_e = p->E - 1;
    if (!fp4) {
      // bf16 profile: the shared expert is one more assignment of every token
      // in the same launches (FP8 weights, FP8 activations)
      const PassArgs a{false, p->topk, k, shared_e, &m13, &m2, shared_slot, nullptr, true};
      if (int rc = moe_pass(p, a, x_bf16, n_tokens, n_tokens_dev, route_weights, route_indices, slot_of_expert,
                            y_bf16, st))
        return rc;
    } else {
      // a4w4: the routed GEMMs read packed E2M1 activations, the shared
      // expert FP8 ones, so it runs first as its own pass into ys, which the
      // routed pass's combine adds after the routed rows
      DSV4_CHECK_ARG(y_bf16, "the a4w4 profile with a shared expert needs y");
      uint16_t* ys = wsp<uint16_t>(p, p->wl.ys);
      const PassArgs s1{false, 1, 0, shared_e, &m13, &m2, shared_slot, nullptr, false};
      if (int rc = moe_pass(p, s1, x_bf16, n_tokens, n_tokens_dev, route_weights, route_indices, slot_of_expert, ys,
                            st))
        return rc;
      const PassArgs s2{true, k, k, -1, nullptr, nullptr, nullptr, ys, true};
      if (int rc = moe_pass(p, s2, x_bf16, n_tokens, n_tokens_dev, route_weights, route_indices, slot_of_expert,
                            y_bf16, st))
        return rc;
    }
  }
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

extern "C" int dsv4_moe_forward(dsv4_moe_plan* p, int32_t profile, const void* x_bf16, int64_t n_tokens,
                                const float* route_weights, const int32_t* route_indices,
                                const int32_t* slot_of_expert, void* y_bf16, void* stream) {
  if (!y_bf16) return fail(DSV4_EINVAL, "dsv4_moe_forward: null pointer");
  return moe_forward_impl(p, profile, x_bf16, n_tokens, nullptr, route_weights, route_indices, slot_of_expert,
                          nullptr, y_bf16, stream);
}

extern "C" int dsv4_moe_forward_shared(dsv4_moe_plan* p, int32_t profile, const void* x_bf16, int64_t n_tokens,
                                       const float* route_weights, const int32_t* route_indices,
                                       const int32_t* slot_of_expert, const uint8_t* shared_slot, void* y_bf16,
                                       void* stream) {
  if (!y_bf16 || !shared_slot) return fail(DSV4_EINVAL, "dsv4_moe_forward_shared: null pointer");
  return moe_forward_impl(p, profile, x_bf16, n_tokens, nullptr, route_weights, route_indices, slot_of_expert,
                          shared_slot, y_bf16, stream);
}

extern "C" int dsv4_moe_forward_rows(dsv4_moe_plan* p, int32_t profile, const void* x_bf16, int64_t max_tokens,
                                     const int32_t* n_tokens_dev, const float* route_weights,
                                     const int32_t* route_indices, const int32_t* slot_of_expert, void* y_bf16,
                                     void* stream) {
  return moe_forward_impl(p, profile, x_bf16, max_tokens, n_tokens_dev, route_weights, route_indices,
                          slot_of_expert, nullptr, y_bf16, stream);
}

extern "C" int dsv4_moe_forward_scatter(dsv4_moe_plan* p, int32_t profile, const void* x_bf16, int64_t max_tokens,
                                        const int32_t* n_tokens_dev, const float* route_weights,
                                        const int32_t* route_indices, const int32_t* slot_of_expert,
                                        void* const* assign_dst, void* stream) {
  if (!assign_dst) return fail(DSV4_EINVAL, "dsv4_moe_forward_scatter: null assign_dst");
  return moe_forward_impl(p, profile, x_bf16, max_tokens, n_tokens_dev, route_weights, route_indices,
                          slot_of_expert, nullptr, nullptr, stream, reinterpret_cast<uint16_t* const*>(assign_dst));
}

extern "C" int dsv4_moe_forward_scatter_q(dsv4_moe_plan* p, int32_t profile, const void* x_rows, int32_t x_format,
                                          int64_t max_tokens, const int32_t* n_tokens_dev,
                                          const float* route_weights, const int32_t* route_indices,
                                          const int32_t* slot_of_expert, void* const* assign_dst, void* stream) {
  if (!assign_dst) return fail(DSV4_EINVAL, "dsv4_moe_forward_scatter_q: null assign_dst");
  return moe_forward_impl(p, profile, x_rows, max_tokens, n_tokens_dev, route_weights, route_indices, slot_of_expert,
                          nullptr, nullptr, stream, reinterpret_cast<uint16_t* const*>(assign_dst), x_format);
}

extern "C" int dsv4_moe_output_rows(dsv4_moe_plan* p, void** rows_bf16, int32_t** inv) {
  if (!p || !rows_bf16 || !inv) return fail(DSV4_EINVAL, "dsv4_moe_output_rows: null pointer");
  *rows_bf16 = p->ws + p->wl.out;
  *inv = wsp<int32_t>(p, p->wl.inv);
  return DSV4_OK;
}

extern "C" int dsv4_moe_enable_timing(dsv4_moe_plan* p, int32_t enable) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(p, "null plan");
  DSV4_CUDA_CHECK(cudaSetDevice(p->device));
  if (enable)
    for (auto& e : p->ev)
      if (!e) DSV4_CUDA_CHECK(cudaEventCreate(&e));
  p->timing = enable != 0;
  DSV4_API_END
}

extern "C" int dsv4_moe_set_gemm_tile(dsv4_moe_plan* p, int32_t tokens_per_tile) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(p, "null plan");
  DSV4_CHECK_ARG(tokens_per_tile == 0 || tokens_per_tile == 64 || tokens_per_tile == 112,
                 "tokens per GEMM tile must be 0 (default), 64 or 112");
  p->gemm_tile = tokens_per_tile;
  DSV4_API_END
}

// The router of the plan's layer for a decode batch, in the plan's
// workspace: one launch (partial logits, grid barrier, top-k) when the batch
// has fewer than 256 tokens and the grid fits on the GPU at once, else the
// two kernels of dsv4_route_topk's decode path.
extern "C" int dsv4_moe_route(dsv4_moe_plan* p, const void* x_bf16, const float* gate_w, const float* bias,
                              const int32_t* tid2eid, const int64_t* input_ids, int64_t vocab_size, int64_t n_tokens,
                              int32_t topk, int32_t score_func, int32_t renormalize, float route_scale,
                              float* weights_out, int32_t* indices_out, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(p, "null plan");
  const int E = p->E - (p->shared ? 1 : 0);
  DSV4_CHECK_ARG(n_tokens >= 0 && n_tokens < 256 && n_tokens <= p->max_tokens,
                 "n_tokens must be below 256 and within the plan's max_tokens");
  DSV4_CHECK_ARG(x_bf16 && gate_w && weights_out && indices_out, "null pointer");
  DSV4_CHECK_ARG(E <= 256, "n_experts must be in [1, 256]");
  DSV4_CHECK_ARG(topk > 0 && topk <= 16 && topk <= E, "topk must be in [1, min(16, n_experts)]");
  DSV4_CHECK_ARG(score_func >= 0 && score_func <= 2, "unknown score function");
  DSV4_CHECK_ARG(!tid2eid || (input_ids && vocab_size > 0), "hash routing needs input_ids and vocab_size");
  if (n_tokens == 0) return DSV4_OK;
  if (int rc = bind_device_of(x_bf16, nullptr)) return rc;
  DSV4_CHECK_ARG(((uintptr_t)x_bf16 % 16) == 0 && ((uintptr_t)gate_w % 16) == 0, "x and gate_w must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const WsLayout& w = p->wl;
  bool launched = false;
  if (int rc = route_fused_launch(x_bf16, gate_w, bias, tid2eid, input_ids, vocab_size, n_tokens, p->H, E, topk,
                                  score_func, renormalize, route_scale, weights_out, indices_out,
                                  wsp<float>(p, w.rpart), wsp<int>(p, w.rbar), wsp<int>(p, w.status), st, &launched))
    return rc;
  if (launched) return DSV4_OK;
  return dsv4_route_topk(x_bf16, gate_w, bias, tid2eid, input_ids, vocab_size, n_tokens, p->H, E, topk, score_func,
                         renormalize, route_scale, weights_out, indices_out, wsp<uint8_t>(p, w.rpart),
                         route_fused_part_bytes(n_tokens, p->H, E), stream);
  DSV4_API_END
}

extern "C" int dsv4_moe_set_ffn_fusion(dsv4_moe_plan* p, int32_t enable) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(p, "null plan");
  DSV4_CHECK_ARG(enable >= -1 && enable <= 1, "enable must be -1, 0 or 1");
  p->fused_ffn = enable;
  DSV4_API_END
}

extern "C" int dsv4_moe_stage_times(dsv4_moe_plan* p, float* ms, int32_t n) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(p && ms, "null pointer");
  DSV4_CHECK_ARG(p->timing, "timing is not enabled on this plan");
  DSV4_CUDA_CHECK(cudaSetDevice(p->device));
  DSV4_CUDA_CHECK(cudaEventSynchronize(p->ev[5]));
  for (int i = 0; i < 5 && i < n; ++i) DSV4_CUDA_CHECK(cudaEventElapsedTime(&ms[i], p->ev[i], p->ev[i + 1]));
  DSV4_API_END
}

extern "C" int dsv4_moe_status(dsv4_moe_plan* p, void* stream) {
  if (!p) return fail(DSV4_EINVAL, "dsv4_moe_status: null plan");
  cudaSetDevice(p->device);
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return fail(DSV4_ECUDA, std::string("dsv4_moe_status: ") + cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpy(&v, p->ws + p->wl.status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(DSV4_ECUDA, std::string("dsv4_moe_status: ") + cudaGetErrorString(e));
  if (v != 0) {
    cudaMemset(p->ws + p->wl.status, 0, sizeof(int));
    return fail(v, "a kernel of the routed-expert layer reported this status");
  }
  return DSV4_OK;
}

extern "C" int dsv4_moe_debug_align(dsv4_moe_plan* p, int32_t** counts, int32_t** offsets, int32_t** sorted_flat,
                                    int32_t** inv, int32_t** active, int32_t** n_active) {
  if (!p) return fail(DSV4_EINVAL, "dsv4_moe_debug_align: null plan");
  if (counts) *counts = wsp<int32_t>(p, p->wl.counts);
  if (offsets) *offsets = wsp<int32_t>(p, p->wl.offsets);
  if (sorted_flat) *sorted_flat = wsp<int32_t>(p, p->wl.sorted_flat);
  if (inv) *inv = wsp<int32_t>(p, p->wl.inv);
  if (active) *active = wsp<int32_t>(p, p->wl.active);
  if (n_active) *n_active = wsp<int32_t>(p, p->wl.n_active);
  return DSV4_OK;
}

// Standalone moe_align entry point (the same kernel, no chunk outputs).
extern "C" int dsv4_moe_align(const int32_t* indices, int64_t n_tokens, int32_t topk, int32_t n_experts,
                              int32_t* counts, int32_t* offsets, int32_t* sorted_flat, int32_t* inv, int32_t* active,
                              int32_t* n_active, int* status, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(counts && offsets && active && n_active, "null pointer");
  DSV4_CHECK_ARG(n_tokens == 0 || (indices && sorted_flat && inv), "null pointer");
  DSV4_CHECK_ARG(n_experts > 0 && n_experts <= 1024 && topk > 0, "bad n_experts / topk");
  DSV4_CHECK_ARG(n_tokens >= 0 && n_tokens * topk < (1LL << 31), "too many assignments");
  int rc = bind_device_of(counts, nullptr);
  if (rc != 0) return rc;
  const size_t al_smem = (size_t)(2 * n_experts + 32 + AL_THREADS) * 4 + (size_t)32 * n_experts * 4;
  DSV4_CUDA_CHECK(
      cudaFuncSetAttribute(moe_align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)al_smem));
  moe_align_kernel<<<1, AL_THREADS, al_smem, (cudaStream_t)stream>>>(
      indices, (int)(n_tokens * topk), topk, n_experts, nullptr, counts, offsets, sorted_flat, inv, active, n_active,
      nullptr, nullptr, nullptr, 1, status, nullptr, topk, -1, nullptr, 0);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

extern "C" int dsv4_moe_combine_ordered(const void* rows_bf16, const int32_t* order, int64_t n_tokens, int32_t topk,
                                        int32_t hidden, void* y_bf16, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(n_tokens >= 0 && topk > 0 && hidden > 0 && hidden % 8 == 0, "bad sizes");
  if (n_tokens == 0) return DSV4_OK;
  DSV4_CHECK_ARG(rows_bf16 && order && y_bf16, "null pointer");
  DSV4_CHECK_ARG(((uintptr_t)rows_bf16 % 16) == 0 && ((uintptr_t)y_bf16 % 16) == 0, "rows and y must be 16-byte aligned");
  if (int rc = bind_device_of(y_bf16, nullptr)) return rc;
  combine_ordered_kernel<<<(unsigned)n_tokens, std::min(1024, hidden / 8), 0, (cudaStream_t)stream>>>(
      (const uint16_t*)rows_bf16, order, topk, hidden, (uint16_t*)y_bf16, n_tokens);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}
