// Expert parallelism: packing of the fixed-capacity dispatch (no counterpart
// in the reference, whose expert-parallel size is 1, deepseek_v4.py:82).
//
// Expert e lives on rank owner[e] (a placement map; without one, e / e_loc).
// Every rank sends `cap` rows to every
// peer (cap = T*k, the worst case), so the exchange has a shape known in
// advance and the layer can be captured in a CUDA graph.  For assignment
// a = t*k + j with destination d, its slot in the send buffer is
// d*cap + (number of earlier assignments with the same destination):
//   send_x[slot]    = x[t]                                  (bf16 row)
//   send_meta[slot] = (e, bits of the route weight)
// and padding slots get send_meta = (-1, 0), an empty assignment for the
// routed-expert kernels.  `ordered[t][0..k)` lists the slots of token t in
// ascending expert id order: the order in which the returned rows are added
// (deepseek_v4.py:195-197).
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"

namespace dsv4 {

constexpr int EP_THREADS = 1024;
constexpr int EP_MAX_WORLD = 64;

// One CTA.  Assignments are taken in rounds of 1024 (thread = assignment):
// the rank of an assignment among those of its destination is its rank among
// equal destinations of its warp (match) plus the count in earlier warps
// plus the count of earlier rounds.
__global__ void __launch_bounds__(EP_THREADS, 1)
    ep_pack_index_kernel(const int32_t* __restrict__ idx, const float* __restrict__ w, int64_t P, int topk,
                         int E, int e_loc, const int32_t* __restrict__ owner, int world, int64_t cap,
                         int32_t* __restrict__ pos, int32_t* __restrict__ meta, int32_t* __restrict__ ordered,
                         int* __restrict__ status) {
  __shared__ int wc[32][EP_MAX_WORLD];
  __shared__ int base[EP_MAX_WORLD];
  __shared__ int round_tot[EP_MAX_WORLD];
  griddep_wait();
  griddep_launch();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < world) base[tid] = 0;
  for (int64_t r0 = 0; r0 < P; r0 += EP_THREADS) {
    for (int i = tid; i < 32 * EP_MAX_WORLD; i += EP_THREADS) (&wc[0][0])[i] = 0;
    __syncthreads();
    const int64_t a = r0 + tid;
    int e = -1, d = -1;
    if (a < P) {
      e = idx[a];
      if (e < 0 || e >= E) {
        if (e != -1) set_status(status, DSV4_EINVAL);
        e = -1;
      } else {
        d = owner ? owner[e] : e / e_loc;
        if (d < 0 || d >= world) {
          set_status(status, DSV4_EINVAL);
          e = d = -1;
        }
      }
    }
    const unsigned same = __match_any_sync(0xffffffffu, d);
    const int rank = __popc(same & ((1u << lane) - 1u));
    if (d >= 0 && rank == 0) wc[warp][d] = __popc(same);
    __syncthreads();
    if (tid < world) {   // exclusive prefix over the warps, per destination
      int s = 0;
      for (int v = 0; v < 32; ++v) {
        const int c = wc[v][tid];
        wc[v][tid] = s;
        s += c;
      }
      round_tot[tid] = s;
    }
    __syncthreads();
    if (d >= 0) {
      const int64_t slot = (int64_t)d * cap + base[d] + wc[warp][d] + rank;
      pos[a] = (int32_t)slot;
      meta[2 * slot] = e;
      meta[2 * slot + 1] = __float_as_int(w[a]);
    } else if (a < P) {
      pos[a] = -1;
    }
    __syncthreads();
    if (tid < world) base[tid] += round_tot[tid];
    __syncthreads();
  }
  // padding slots of every destination block
  for (int64_t s = tid; s < (int64_t)world * cap; s += EP_THREADS) {
    const int d = (int)(s / cap);
    if (s - (int64_t)d * cap >= base[d]) {
      meta[2 * s] = -1;
      meta[2 * s + 1] = 0;
    }
  }
  // per token: its slots in ascending expert id order (insertion sort of k)
  for (int64_t t = tid; t < P / topk; t += EP_THREADS) {
    int ke[16], kp[16];
    int n = 0;
    for (int j = 0; j < topk; ++j) {
      const int e = idx[t * topk + j];
      const int p = pos[t * topk + j];
      if (p < 0) continue;
      int i = n++;
      while (i > 0 && ke[i - 1] > e) {
        ke[i] = ke[i - 1];
        kp[i] = kp[i - 1];
        --i;
      }
      ke[i] = e;
      kp[i] = p;
    }
    for (int j = 0; j < topk; ++j) ordered[t * topk + j] = j < n ? kp[j] : -1;
  }
}

// One warp per assignment: copy the token's bf16 row into its send slot.
__global__ void ep_pack_rows_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ pos, int64_t P,
                                    int topk, int H, uint16_t* __restrict__ send_x) {
  griddep_wait();
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t a = warp0; a < P; a += nwarps) {
    const int p = pos[a];
    if (p < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + (a / topk) * H);
    uint4* dst = reinterpret_cast<uint4*>(send_x + (int64_t)p * H);
    for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
  }
}

}  // namespace dsv4

using namespace dsv4;

extern "C" int dsv4_ep_dispatch_pack(const void* x_bf16, const float* route_weights, const int32_t* route_indices,
                                     int64_t n_tokens, int32_t topk, int32_t hidden, int32_t n_experts,
                                     int32_t world, const int32_t* expert_owner, void* send_x_bf16,
                                     int32_t* send_meta, int32_t* slot_of_assignment, int32_t* ordered_slots,
                                     int* status, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16 && route_weights && route_indices && send_x_bf16 && send_meta && slot_of_assignment &&
                     ordered_slots && status,
                 "null pointer");
  DSV4_CHECK_ARG(n_tokens >= 0 && topk > 0 && topk <= 16, "topk must be in [1, 16]");
  DSV4_CHECK_ARG(world > 0 && world <= EP_MAX_WORLD && n_experts > 0 && (expert_owner || n_experts % world == 0),
                 "world must be in [1, 64] and divide n_experts (or pass expert_owner)");
  DSV4_CHECK_ARG(hidden > 0 && hidden % 8 == 0, "hidden must be a positive multiple of 8");
  DSV4_CHECK_ARG(n_tokens * topk < (1LL << 31) / world, "too many assignments");
  DSV4_CHECK_ARG(((uintptr_t)x_bf16 % 16) == 0 && ((uintptr_t)send_x_bf16 % 16) == 0, "rows must be 16-byte aligned");
  if (n_tokens == 0) return DSV4_OK;
  if (int rc = bind_device_of(route_indices, nullptr)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = pdl_enabled();
  const int64_t P = n_tokens * topk;
  const int64_t cap = P;
  DSV4_CUDA_CHECK(launch_k(ep_pack_index_kernel, dim3(1), dim3(EP_THREADS), 0, st, pdl, route_indices, route_weights,
                           P, (int)topk, (int)n_experts, (int)(n_experts / world), expert_owner, (int)world, cap,
                           slot_of_assignment, send_meta, ordered_slots, status));
  const int64_t blocks = std::min<int64_t>((P * 32 + 255) / 256, 148 * 8);
  DSV4_CUDA_CHECK(launch_k(ep_pack_rows_kernel, dim3((unsigned)blocks), dim3(256), 0, st, pdl,
                           (const uint16_t*)x_bf16, (const int32_t*)slot_of_assignment, P, (int)topk, (int)hidden,
                           (uint16_t*)send_x_bf16));
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

namespace dsv4 {

// ---------------------------------------------------------------------------
// Exchange over NVLink peer memory (CUDA IPC): exact per-peer counts, and
// each token crosses once per destination rank, however many of its k
// experts live there.  Each rank owns one device block that its peers write
// into (T = the token capacity per source, k = top-k):
//   recv_x [world*T, H] bf16: the tokens dispatched to this rank, COMPACT:
//     source s fills rows off[s] .. off[s] + n[s->me), off[s] = the sum over
//     s' < s of n[s'->me];
//   recv_idx / recv_w [world*T, k]: each received token's k picks with the
//     experts of other ranks set to -1 (weight 0), recv_src [world*T] int2
//     (source rank, token index at the source);
//   back [T*k, H] bf16: expert outputs of this rank's own assignments; the
//     owner of assignment a = t*k + j writes row a;
//   cnt [world][world] int32: row s = the per-destination token counts of s;
//   flags [3][world]: per source, the epoch of its published counts, rows
//     and returned rows; ctrl: epoch, arrival counters, tokens received;
//   pos [T][world] int32 (local): the compact index of (token, destination).
// A step: (1) one CTA finds, per destination, the tokens with at least one
// expert there and their stable rank, writes its count row into every
// peer's cnt and publishes; (2) a wait for every source's counts; (3) each
// (token, destination) row, its masked picks and its source into the owner's
// block, then "rows published"; (4) a wait for every source's rows, which
// also sums the received count (the layer's device-side token count); after
// the layer (top-k over the received tokens, foreign experts -1) (5) every
// assignment's output goes back to its source's `back`, read from the
// layer's sorted output rows through inv, and (6) a wait.  Publishing is a
// system-scope release of the epoch after the writes are fenced; waiting is
// an acquire, bounded (DSV4_ETIMEOUT in *status).  A peer writes into this
// rank's block for step e+1 only after it received this rank's step-e
// return, which this rank sends after consuming step e, so one buffer set
// suffices.  After a timeout the step's data are undefined and a late peer
// may still write: the handle must be destroyed and created again.
// ---------------------------------------------------------------------------
struct EpBlock {
  int64_t off_back, off_idx, off_w, off_src, off_cnt, off_pos, off_dst, off_flags, off_ctrl, bytes;
};
static EpBlock ep_block(int world, int64_t tokens, int topk, int hidden) {
  auto al = [](int64_t v) { return (v + 255) / 256 * 256; };
  EpBlock b;
  const int64_t rows = (int64_t)world * tokens;
  b.off_back = al(rows * hidden * 2);
  b.off_idx = b.off_back + al(tokens * topk * hidden * 2);
  b.off_w = b.off_idx + al(rows * topk * 4);
  b.off_src = b.off_w + al(rows * topk * 4);
  b.off_cnt = b.off_src + al(rows * 8);
  b.off_pos = b.off_cnt + al((int64_t)world * world * 4);
  b.off_dst = b.off_pos + al(tokens * world * 4);
  b.off_flags = b.off_dst + al(rows * topk * 8);
  b.off_ctrl = b.off_flags + al(3 * (int64_t)world * 4);
  b.bytes = b.off_ctrl + 256;
  return b;
}
// ctrl words
constexpr int EPC_EPOCH = 0, EPC_ROWS = 1, EPC_BACK = 2, EPC_NRECV = 3;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ep_dest(int e, int e_loc, const int32_t* __restrict__ owner) {
  return owner ? owner[e] : e / e_loc;
}

// One CTA: epoch += 1; per destination, the tokens with an expert there and
// their stable rank among them (pos[t][d], or -1); this rank's count row
// into every peer's cnt, fenced and published.  (The combine order of each
// token's assignments is left to the rows kernel, a warp per token.)
__global__ void __launch_bounds__(EP_THREADS, 1)
    ep_p2p_index_kernel(const int32_t* __restrict__ idx, int64_t T, int topk, int E, int e_loc,
                        const int32_t* __restrict__ owner, int world, int my_rank, uint8_t* const* __restrict__ peers,
                        int64_t off_cnt, int64_t off_flags, uint32_t* __restrict__ ctrl, int32_t* __restrict__ pos,
                        int* __restrict__ status) {
  __shared__ int wc[32][EP_MAX_WORLD];
  __shared__ int base[EP_MAX_WORLD];
  __shared__ int round_tot[EP_MAX_WORLD];
  griddep_wait();
  griddep_launch();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned lt = (1u << lane) - 1u;
  if (tid == 0) ctrl[EPC_EPOCH] = ctrl[EPC_EPOCH] + 1u;   // this step's epoch
  if (tid < world) base[tid] = 0;
  for (int64_t t0 = 0; t0 < T; t0 += EP_THREADS) {
    const int64_t t = t0 + tid;
    unsigned long long mask = 0ull;   // destinations of this token
    if (t < T) {
      int ev[16];   // the token's picks, loaded together
#pragma unroll
      for (int j = 0; j < 16; ++j) ev[j] = j < topk ? idx[t * topk + j] : -1;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (j >= topk) break;
        const int e = ev[j];
        if (e >= 0 && e < E) {
          const int d = ep_dest(e, e_loc, owner);
          if (d >= 0 && d < world)
            mask |= 1ull << d;
          else
            set_status(status, DSV4_EINVAL);
        } else if (e != -1) {
          set_status(status, DSV4_EINVAL);
        }
      }
    }
    for (int d = 0; d < world; ++d) {
      const unsigned bal = __ballot_sync(0xffffffffu, (mask >> d) & 1ull);
      if (lane == 0) wc[warp][d] = __popc(bal);
    }
    __syncthreads();
    if (tid < world) {   // exclusive prefix over the warps, per destination
      int sum = 0;
      for (int v = 0; v < 32; ++v) {
        const int c = wc[v][tid];
        wc[v][tid] = sum;
        sum += c;
      }
      round_tot[tid] = sum;
    }
    __syncthreads();
    for (int d = 0; d < world; ++d) {
      const bool on = (mask >> d) & 1ull;
      const unsigned bal = __ballot_sync(0xffffffffu, on);
      if (t < T) pos[t * world + d] = on ? base[d] + wc[warp][d] + __popc(bal & lt) : -1;
    }
    __syncthreads();
    if (tid < world) base[tid] += round_tot[tid];
    __syncthreads();
  }
  // this rank's counts into row my_rank of every peer's count matrix
  for (int i = tid; i < world * world; i += EP_THREADS) {
    const int d = i / world, c = i - d * world;
    reinterpret_cast<int32_t*>(peers[d] + off_cnt)[my_rank * world + c] = base[c];
  }
  __threadfence_system();
  __syncthreads();
  if (tid == 0) {
    const uint32_t epoch = ctrl[EPC_EPOCH];
    for (int d = 0; d < world; ++d)
      st_release_sys(reinterpret_cast<uint32_t*>(peers[d] + off_flags) + 0 * world + my_rank, epoch);
  }
}

// After every CTA fenced its peer writes, the last CTA to finish publishes
// the epoch into slot `flag_slot` of every peer's flags.
__device__ __forceinline__ void ep_publish(uint32_t* __restrict__ ctrl, int counter, uint8_t* const* __restrict__ peers,
                                           int world, int64_t off_flags, int flag_slot) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&ctrl[counter], 1u);
    if (prev == gridDim.x - 1) {
      ctrl[counter] = 0u;
      __threadfence_system();
      const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&ctrl[EPC_EPOCH]);
      for (int d = 0; d < world; ++d)
        st_release_sys(reinterpret_cast<uint32_t*>(peers[d] + off_flags) + flag_slot, epoch);
    }
  }
}

// One warp per token: the row goes to every destination rank with at least
// one of its experts, at the compact row off[d] + pos[t][d] of the owner's
// block, with its picks (the other ranks' experts set to -1, weight 0) and
// its source.  The offsets come from this rank's copy of the count matrix
// (every source wrote its row before the wait that precedes this kernel).
// Row format (DSV4_ROWS_*): bf16 as it is, or quantised here once for all
// destinations exactly as the owner's quantise-gather would (FP8 per 128 /
// MXFP4 per 32), so that fewer bytes cross NVLink; the block scales follow
// the codes in the same row.
template <int FMT>
__global__ void ep_p2p_rows_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ idx,
                                   const float* __restrict__ w, const int32_t* __restrict__ pos, int64_t T, int topk,
                                   int H, int E, int e_loc, const int32_t* __restrict__ owner, int world, int my_rank,
                                   uint8_t* const* __restrict__ peers, EpBlock blk, const int32_t* __restrict__ cnt,
                                   uint32_t* __restrict__ ctrl, int64_t row_bytes, int32_t* __restrict__ ordered) {
  __shared__ int64_t off[EP_MAX_WORLD];
  griddep_wait();
  griddep_launch();
  if (threadIdx.x < world) {
    int64_t o = 0;
    for (int s = 0; s < my_rank; ++s) o += cnt[s * world + threadIdx.x];
    off[threadIdx.x] = o;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int kblk = H / 128;
  for (int64_t t = warp0; t < T; t += nwarps) {
    // destinations of this token: lane d < world holds its row there, or -1
    const int p = lane < world ? pos[t * world + lane] : -1;
    const int64_t my_row = p >= 0 ? off[lane] + p : -1;
    {
      // the token's combine order: its valid assignments t*k + j in ascending
      // expert id (equal ids by j), then -1; lane j ranks pick j
      const int e = lane < topk ? idx[t * topk + lane] : -1;
      const bool valid = e >= 0 && e < E && [&] {
        const int d = ep_dest(e, e_loc, owner);
        return d >= 0 && d < world;
      }();
      int rank = 0;
      for (int i = 0; i < topk; ++i) {
        const int ei = __shfl_sync(0xffffffffu, e, i);
        const int vi = __shfl_sync(0xffffffffu, valid ? 1 : 0, i);
        rank += (vi && (ei < e || (ei == e && i < lane))) ? 1 : 0;
      }
      const int nv = __popc(__ballot_sync(0xffffffffu, valid));
      if (valid) ordered[t * topk + rank] = (int)(t * topk + lane);
      if (lane >= nv && lane < topk) ordered[t * topk + lane] = -1;
    }
    const unsigned dests = __ballot_sync(0xffffffffu, p >= 0);
    if (dests == 0u) continue;
    uint32_t scl[2] = {0u, 0u};   // lane L: the scale(s) of block L (and L + 32)
    for (int kb0 = 0; kb0 < kblk; kb0 += 8) {
      // eight 128-column blocks' loads in flight together, then each block
      uint2 raws[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        raws[u] = kb0 + u < kblk ? *reinterpret_cast<const uint2*>(x + t * H + (kb0 + u) * 128 + lane * 4)
                                 : make_uint2(0u, 0u);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int kb = kb0 + u;
        if (kb >= kblk) break;
        const uint2 raw = raws[u];
        if constexpr (FMT == DSV4_ROWS_BF16) {
          for (unsigned m = dests; m; m &= m - 1u) {
            const int d = __ffs(m) - 1;
            const int64_t row = __shfl_sync(0xffffffffu, my_row, d);
            *reinterpret_cast<uint2*>(peers[d] + row * row_bytes + (int64_t)(kb * 128 + lane * 4) * 2) = raw;
          }
        } else {
          const float v[4] = {bf16_from_bits(raw.x & 0xffffu), bf16_from_bits(raw.x >> 16),
                              bf16_from_bits(raw.y & 0xffffu), bf16_from_bits(raw.y >> 16)};
          int e;
          if constexpr (FMT == DSV4_ROWS_FP8) {
            const uint32_t o = fp8_block_quant(v, &e);
            if (lane == (kb & 31)) scl[kb >> 5] = (uint32_t)(e + 127);
            for (unsigned m = dests; m; m &= m - 1u) {
              const int d = __ffs(m) - 1;
              const int64_t row = __shfl_sync(0xffffffffu, my_row, d);
              *reinterpret_cast<uint32_t*>(peers[d] + row * row_bytes + kb * 128 + lane * 4) = o;
            }
          } else {
            const uint32_t packed = mxfp4_block_quant(v, &e);
            const uint32_t sword = (uint32_t)(__shfl_sync(0xffffffffu, e, 0) + 127) |
                                   ((uint32_t)(__shfl_sync(0xffffffffu, e, 8) + 127) << 8) |
                                   ((uint32_t)(__shfl_sync(0xffffffffu, e, 16) + 127) << 16) |
                                   ((uint32_t)(__shfl_sync(0xffffffffu, e, 24) + 127) << 24);
            if (lane == (kb & 31)) scl[kb >> 5] = sword;
            for (unsigned m = dests; m; m &= m - 1u) {
              const int d = __ffs(m) - 1;
              const int64_t row = __shfl_sync(0xffffffffu, my_row, d);
              *reinterpret_cast<uint16_t*>(peers[d] + row * row_bytes + kb * 64 + lane * 2) = (uint16_t)packed;
            }
          }
        }
      }
    }
    if constexpr (FMT != DSV4_ROWS_BF16) {
      // the block scales after the codes: one byte (FP8) or one word of four
      // (MXFP4) per 128 columns, lane L storing block L's
      for (unsigned m = dests; m; m &= m - 1u) {
        const int d = __ffs(m) - 1;
        const int64_t row = __shfl_sync(0xffffffffu, my_row, d);
        uint8_t* base = peers[d] + row * row_bytes + (FMT == DSV4_ROWS_FP8 ? H : H / 2);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int kb = lane + 32 * h;
          if (kb < kblk) {
            if (FMT == DSV4_ROWS_FP8)
              base[kb] = (uint8_t)scl[h];
            else
              reinterpret_cast<uint32_t*>(base)[kb] = scl[h];
          }
        }
      }
    }
    // picks and source, per destination
    for (unsigned m = dests; m; m &= m - 1u) {
      const int d = __ffs(m) - 1;
      const int64_t row = __shfl_sync(0xffffffffu, my_row, d);
      if (lane < topk) {
        const int e = idx[t * topk + lane];
        const bool mine = e >= 0 && e < E && ep_dest(e, e_loc, owner) == d;
        reinterpret_cast<int32_t*>(peers[d] + blk.off_idx)[row * topk + lane] = mine ? e : -1;
        reinterpret_cast<float*>(peers[d] + blk.off_w)[row * topk + lane] = mine ? w[t * topk + lane] : 0.f;
      }
      if (lane == 0) reinterpret_cast<int2*>(peers[d] + blk.off_src)[row] = make_int2(my_rank, (int)t);
    }
  }
  ep_publish(ctrl, EPC_ROWS, peers, world, blk.off_flags, 1 * world + my_rank);
}

// One warp per (received token j < n_recv, pick s) with an expert of this
// rank: its output (row inv[j*k + s] of the layer's sorted output, or row
// j*k + s of y when inv is null) into the source's `back` row t*k + s.
__global__ void ep_p2p_return_kernel(const uint16_t* __restrict__ y, const int32_t* __restrict__ inv,
                                     const int32_t* __restrict__ recv_idx, const int2* __restrict__ src_of,
                                     const uint32_t* __restrict__ n_recv, int world, int my_rank, int64_t T, int topk,
                                     int H, uint8_t* const* __restrict__ peers, int64_t off_back, int64_t off_flags,
                                     uint32_t* __restrict__ ctrl) {
  griddep_wait();
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const int64_t n = (int64_t)*reinterpret_cast<const volatile uint32_t*>(n_recv) * topk;
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t a = warp0; a < n; a += nwarps) {
    if (recv_idx[a] < 0) continue;
    const int64_t j = a / topk;
    const int s = (int)(a - j * topk);
    const int2 st = src_of[j];
    if (st.x < 0 || st.x >= world || st.y < 0 || st.y >= T) continue;   // not written this step (after a timeout)
    const int64_t from_row = inv ? (int64_t)inv[a] : a;
    const uint4* from = reinterpret_cast<const uint4*>(y + from_row * H);
    uint4* dst = reinterpret_cast<uint4*>(peers[st.x] + off_back) + ((int64_t)st.y * topk + s) * (H / 8);
    for (int c = lane; c < H / 8; c += 32) dst[c] = from[c];
  }
  ep_publish(ctrl, EPC_BACK, peers, world, off_flags, 2 * world + my_rank);
}

// The return target of every received assignment a = j*k + s (an expert of
// this rank): row t*k + s of its source's `back`, as a device address (a
// peer's memory for the other ranks); null for the other ranks' picks.  The
// down GEMM in scatter mode stores each output row there directly.
__global__ void ep_p2p_targets_kernel(const int32_t* __restrict__ recv_idx, const int2* __restrict__ src_of,
                                      const uint32_t* __restrict__ n_recv, int world, int64_t T, int topk, int H,
                                      uint8_t* const* __restrict__ peers, int64_t off_back,
                                      uint16_t** __restrict__ dst) {
  griddep_wait();
  griddep_launch();
  const int64_t n = (int64_t)*reinterpret_cast<const volatile uint32_t*>(n_recv) * topk;
  for (int64_t a = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; a < n; a += (int64_t)gridDim.x * blockDim.x) {
    uint16_t* d = nullptr;
    if (recv_idx[a] >= 0) {
      const int64_t j = a / topk;
      const int s = (int)(a - j * topk);
      const int2 st = src_of[j];
      if (st.x >= 0 && st.x < world && st.y >= 0 && st.y < T)
        d = reinterpret_cast<uint16_t*>(peers[st.x] + off_back) + ((int64_t)st.y * topk + s) * H;
    }
    dst[a] = d;
  }
}

// One CTA: after the rows this rank wrote into its peers' `back` (the down
// GEMM in scatter mode, a finished kernel, its stores fenced system-wide),
// publish "returned" to every peer.
__global__ void ep_p2p_publish_back_kernel(uint32_t* __restrict__ ctrl, uint8_t* const* __restrict__ peers, int world,
                                           int64_t off_flags, int my_rank) {
  griddep_wait();
  griddep_launch();
  ep_publish(ctrl, EPC_BACK, peers, world, off_flags, 2 * world + my_rank);
}

// One thread: wait (bounded) until every source has published this step's
// epoch in flags[first .. first+world).  With `cnt`, also writes the number
// of tokens this rank receives (column my_rank of the count matrix) to *n_recv.
__global__ void ep_p2p_wait_kernel(const uint32_t* __restrict__ flags, const uint32_t* __restrict__ ctrl, int world,
                                   int* __restrict__ status, const int32_t* __restrict__ cnt, int my_rank,
                                   uint32_t* __restrict__ n_recv) {
  griddep_wait();
  griddep_launch();
  if (threadIdx.x != 0) return;
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(&ctrl[EPC_EPOCH]);
  const uint64_t t0 = globaltimer_ns();
  for (int s = 0; s < world; ++s) {
    while ((int32_t)(ld_acquire_sys(flags + s) - epoch) < 0) {
      if (globaltimer_ns() - t0 > DSV4_WAIT_NS) {
        set_status(status, DSV4_ETIMEOUT);
        if (n_recv) *n_recv = 0u;   // the layer then runs on no rows
        return;
      }
    }
  }
  if (n_recv) {
    uint32_t n = 0;
    for (int s = 0; s < world; ++s) n += (uint32_t)cnt[s * world + my_rank];
    *n_recv = n;
  }
}

}  // namespace dsv4

struct dsv4_ep {
  int rank = 0, world = 1, device = 0, hidden = 0, topk = 0;
  int64_t tokens = 0;   // token capacity per source
  dsv4::EpBlock blk{};
  uint8_t* base = nullptr;
  uint8_t** peers_dev = nullptr;
  std::vector<uint8_t*> opened;   // peer blocks opened through IPC
  ~dsv4_ep() {
    cudaSetDevice(device);
    for (uint8_t* p : opened)
      if (p) cudaIpcCloseMemHandle(p);
    if (peers_dev) cudaFree(peers_dev);
    if (base) cudaFree(base);
  }
};

namespace dsv4 {
namespace {
int ep_check(dsv4_ep* ep) {
  if (!ep) return fail(DSV4_EINVAL, "null expert-parallel handle");
  if (!ep->peers_dev) return fail(DSV4_EINVAL, "dsv4_ep_connect has not been called");
  return DSV4_OK;
}
}  // namespace
}  // namespace dsv4

extern "C" int dsv4_ep_create(dsv4_ep** out, int32_t device, int32_t rank, int32_t world, int64_t max_tokens,
                              int32_t topk, int32_t hidden, void* ipc_handle_out) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(out && ipc_handle_out, "null pointer");
  DSV4_CHECK_ARG(world > 0 && world <= EP_MAX_WORLD && rank >= 0 && rank < world, "rank/world out of range");
  DSV4_CHECK_ARG(max_tokens > 0 && max_tokens < (1LL << 30) && topk > 0 && topk <= 16 && hidden > 0 &&
                     hidden % 8 == 0,
                 "bad capacity / topk / hidden");
  std::unique_ptr<dsv4_ep> ep(new dsv4_ep);
  ep->device = device;
  DSV4_CUDA_CHECK(cudaSetDevice(device));
  ep->rank = rank;
  ep->world = world;
  ep->tokens = max_tokens;
  ep->topk = topk;
  ep->hidden = hidden;
  ep->blk = ep_block(world, max_tokens, topk, hidden);
  DSV4_CUDA_CHECK(cudaMalloc(&ep->base, (size_t)ep->blk.bytes));
  DSV4_CUDA_CHECK(cudaMemset(ep->base + ep->blk.off_idx, 0, (size_t)(ep->blk.bytes - ep->blk.off_idx)));
  cudaIpcMemHandle_t h;
  DSV4_CUDA_CHECK(cudaIpcGetMemHandle(&h, ep->base));
  memcpy(ipc_handle_out, &h, sizeof(h));
  *out = ep.release();
  DSV4_API_END
}

extern "C" int dsv4_ep_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

extern "C" int dsv4_ep_connect(dsv4_ep* ep, const void* handles) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(ep && handles, "null pointer");
  DSV4_CHECK_ARG(!ep->peers_dev, "already connected");
  DSV4_CUDA_CHECK(cudaSetDevice(ep->device));
  std::vector<uint8_t*> peers(ep->world, nullptr);
  for (int r = 0; r < ep->world; ++r) {
    if (r == ep->rank) {
      peers[r] = ep->base;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    DSV4_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    peers[r] = static_cast<uint8_t*>(p);
    ep->opened.push_back(peers[r]);
  }
  DSV4_CUDA_CHECK(cudaMalloc(&ep->peers_dev, sizeof(uint8_t*) * ep->world));
  DSV4_CUDA_CHECK(cudaMemcpy(ep->peers_dev, peers.data(), sizeof(uint8_t*) * ep->world, cudaMemcpyHostToDevice));
  DSV4_API_END
}

extern "C" int dsv4_ep_buffers(dsv4_ep* ep, void** recv_x, int32_t** recv_indices, float** recv_weights,
                               int32_t** n_recv, void** back) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(ep && recv_x && recv_indices && recv_weights && n_recv && back, "null pointer");
  *recv_x = ep->base;
  *back = ep->base + ep->blk.off_back;
  *recv_indices = reinterpret_cast<int32_t*>(ep->base + ep->blk.off_idx);
  *recv_weights = reinterpret_cast<float*>(ep->base + ep->blk.off_w);
  *n_recv = reinterpret_cast<int32_t*>(ep->base + ep->blk.off_ctrl) + EPC_NRECV;
  DSV4_API_END
}

extern "C" int64_t dsv4_ep_row_bytes(int32_t row_format, int32_t hidden) {
  if (hidden <= 0 || hidden % 128 != 0) return DSV4_EINVAL;
  const int64_t H = hidden;
  int64_t b;
  if (row_format == DSV4_ROWS_BF16)
    b = 2 * H;
  else if (row_format == DSV4_ROWS_FP8)
    b = H + H / 128;
  else if (row_format == DSV4_ROWS_MXFP4)
    b = H / 2 + H / 32;
  else
    return DSV4_EINVAL;
  return (b + 15) / 16 * 16;
}

extern "C" int dsv4_ep_dispatch(dsv4_ep* ep, const void* x_bf16, const float* route_weights,
                                const int32_t* route_indices, int64_t n_tokens, int32_t n_experts,
                                const int32_t* expert_owner, int32_t* ordered_assignments, int* status,
                                void* stream) {
  return dsv4_ep_dispatch_q(ep, x_bf16, route_weights, route_indices, n_tokens, n_experts, expert_owner,
                            ordered_assignments, DSV4_ROWS_BF16, status, stream);
}

extern "C" int dsv4_ep_dispatch_q(dsv4_ep* ep, const void* x_bf16, const float* route_weights,
                                  const int32_t* route_indices, int64_t n_tokens, int32_t n_experts,
                                  const int32_t* expert_owner, int32_t* ordered_assignments, int32_t row_format,
                                  int* status, void* stream) {
  DSV4_API_BEGIN
  if (int rc = ep_check(ep)) return rc;
  DSV4_CHECK_ARG(x_bf16 && route_weights && route_indices && ordered_assignments && status, "null pointer");
  DSV4_CHECK_ARG(row_format >= DSV4_ROWS_BF16 && row_format <= DSV4_ROWS_MXFP4, "unknown row format");
  DSV4_CHECK_ARG(ep->world <= 32, "the peer-memory exchange takes at most 32 ranks");
  DSV4_CHECK_ARG(ep->hidden % 128 == 0 && ep->hidden <= 8192, "hidden must be a multiple of 128, at most 8192");
  const int64_t row_bytes = dsv4_ep_row_bytes(row_format, ep->hidden);
  DSV4_CHECK_ARG(n_tokens >= 0 && n_tokens <= ep->tokens, "n_tokens must be in [0, the handle's max_tokens]");
  DSV4_CHECK_ARG(n_experts > 0 && (expert_owner || n_experts % ep->world == 0),
                 "n_experts must divide over the ranks (or pass expert_owner)");
  DSV4_CHECK_ARG(((uintptr_t)x_bf16 % 16) == 0, "rows must be 16-byte aligned");
  DSV4_CUDA_CHECK(cudaSetDevice(ep->device));
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = pdl_enabled();
  const int64_t T = n_tokens;
  const int k = ep->topk;
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(ep->base + ep->blk.off_ctrl);
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(ep->base + ep->blk.off_flags);
  const int32_t* cnt = reinterpret_cast<const int32_t*>(ep->base + ep->blk.off_cnt);
  int32_t* pos = reinterpret_cast<int32_t*>(ep->base + ep->blk.off_pos);
  uint8_t* const* peers = (uint8_t* const*)ep->peers_dev;
  const int e_loc = (int)(n_experts / ep->world);
  DSV4_CUDA_CHECK(launch_k(ep_p2p_index_kernel, dim3(1), dim3(EP_THREADS), 0, st, pdl, route_indices, T, k,
                           (int)n_experts, e_loc, expert_owner, ep->world, ep->rank, peers, ep->blk.off_cnt,
                           ep->blk.off_flags, ctrl, pos, status));
  DSV4_CUDA_CHECK(launch_k(ep_p2p_wait_kernel, dim3(1), dim3(32), 0, st, pdl, flags, (const uint32_t*)ctrl,
                           ep->world, status, (const int32_t*)nullptr, ep->rank, (uint32_t*)nullptr));
  // a warp per token
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((T * 32 + 255) / 256, 148 * 8));
  auto rows_kernel = row_format == DSV4_ROWS_FP8     ? ep_p2p_rows_kernel<DSV4_ROWS_FP8>
                     : row_format == DSV4_ROWS_MXFP4 ? ep_p2p_rows_kernel<DSV4_ROWS_MXFP4>
                                                     : ep_p2p_rows_kernel<DSV4_ROWS_BF16>;
  DSV4_CUDA_CHECK(launch_k(rows_kernel, dim3((unsigned)blocks), dim3(256), 0, st, pdl, (const uint16_t*)x_bf16,
                           route_indices, route_weights, (const int32_t*)pos, T, k, ep->hidden, (int)n_experts, e_loc,
                           expert_owner, ep->world, ep->rank, peers, ep->blk, cnt, ctrl, row_bytes,
                           ordered_assignments));
  DSV4_CUDA_CHECK(launch_k(ep_p2p_wait_kernel, dim3(1), dim3(32), 0, st, pdl, flags + ep->world,
                           (const uint32_t*)ctrl, ep->world, status, cnt, ep->rank, ctrl + EPC_NRECV));
  // the return targets of the received assignments (for the scatter-mode down GEMM)
  const int64_t assigns = (int64_t)ep->world * ep->tokens * ep->topk;
  const unsigned tblocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((assigns + 255) / 256, 148 * 4));
  DSV4_CUDA_CHECK(launch_k(ep_p2p_targets_kernel, dim3(tblocks), dim3(256), 0, st, pdl,
                           (const int32_t*)(ep->base + ep->blk.off_idx), (const int2*)(ep->base + ep->blk.off_src),
                           (const uint32_t*)(ctrl + EPC_NRECV), ep->world, ep->tokens, ep->topk, ep->hidden, peers,
                           ep->blk.off_back, reinterpret_cast<uint16_t**>(ep->base + ep->blk.off_dst)));
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

extern "C" int dsv4_ep_return_targets(dsv4_ep* ep, void*** assign_dst) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(ep && assign_dst, "null pointer");
  *assign_dst = reinterpret_cast<void**>(ep->base + ep->blk.off_dst);
  DSV4_API_END
}

extern "C" int dsv4_ep_return_published(dsv4_ep* ep, int* status, void* stream) {
  DSV4_API_BEGIN
  if (int rc = ep_check(ep)) return rc;
  DSV4_CHECK_ARG(status, "null pointer");
  DSV4_CUDA_CHECK(cudaSetDevice(ep->device));
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = pdl_enabled();
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(ep->base + ep->blk.off_ctrl);
  DSV4_CUDA_CHECK(launch_k(ep_p2p_publish_back_kernel, dim3(1), dim3(32), 0, st, pdl, ctrl,
                           (uint8_t* const*)ep->peers_dev, ep->world, ep->blk.off_flags, ep->rank));
  DSV4_CUDA_CHECK(launch_k(ep_p2p_wait_kernel, dim3(1), dim3(32), 0, st, pdl,
                           (const uint32_t*)(ep->base + ep->blk.off_flags) + 2 * ep->world, (const uint32_t*)ctrl,
                           ep->world, status, (const int32_t*)nullptr, ep->rank, (uint32_t*)nullptr));
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

extern "C" int dsv4_ep_return(dsv4_ep* ep, const void* rows_bf16, const int32_t* row_of_assignment, int* status,
                              void* stream) {
  DSV4_API_BEGIN
  if (int rc = ep_check(ep)) return rc;
  DSV4_CHECK_ARG(rows_bf16 && status, "null pointer");
  DSV4_CHECK_ARG(((uintptr_t)rows_bf16 % 16) == 0, "rows must be 16-byte aligned");
  DSV4_CUDA_CHECK(cudaSetDevice(ep->device));
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = pdl_enabled();
  uint32_t* ctrl = reinterpret_cast<uint32_t*>(ep->base + ep->blk.off_ctrl);
  const int64_t assigns = (int64_t)ep->world * ep->tokens * ep->topk;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((assigns * 32 + 255) / 256, 148 * 8));
  DSV4_CUDA_CHECK(launch_k(ep_p2p_return_kernel, dim3((unsigned)blocks), dim3(256), 0, st, pdl,
                           (const uint16_t*)rows_bf16, row_of_assignment,
                           (const int32_t*)(ep->base + ep->blk.off_idx), (const int2*)(ep->base + ep->blk.off_src),
                           (const uint32_t*)(ctrl + EPC_NRECV), ep->world, ep->rank, ep->tokens, ep->topk, ep->hidden,
                           (uint8_t* const*)ep->peers_dev, ep->blk.off_back, ep->blk.off_flags, ctrl));
  DSV4_CUDA_CHECK(launch_k(ep_p2p_wait_kernel, dim3(1), dim3(32), 0, st, pdl,
                           (const uint32_t*)(ep->base + ep->blk.off_flags) + 2 * ep->world, (const uint32_t*)ctrl,
                           ep->world, status, (const int32_t*)nullptr, ep->rank, (uint32_t*)nullptr));
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

extern "C" int dsv4_ep_destroy(dsv4_ep* ep) {
  delete ep;
  return DSV4_OK;
}
