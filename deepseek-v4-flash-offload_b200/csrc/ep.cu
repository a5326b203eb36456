// Expert parallelism: packing of the fixed-capacity dispatch (no counterpart
// in the reference, whose expert-parallel size is 1, deepseek_v4.py:82).
//
// Expert e lives on rank e / e_loc.  Every rank sends `cap` rows to every
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
#include <string>

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
                         int e_loc, int world, int64_t cap, int32_t* __restrict__ pos, int32_t* __restrict__ meta,
                         int32_t* __restrict__ ordered, int* __restrict__ status) {
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
      if (e < 0 || e >= e_loc * world) {
        set_status(status, DSV4_EINVAL);
        e = -1;
      } else {
        d = e / e_loc;
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
                                     int32_t world, void* send_x_bf16, int32_t* send_meta, int32_t* slot_of_assignment,
                                     int32_t* ordered_slots, int* status, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16 && route_weights && route_indices && send_x_bf16 && send_meta && slot_of_assignment &&
                     ordered_slots && status,
                 "null pointer");
  DSV4_CHECK_ARG(n_tokens >= 0 && topk > 0 && topk <= 16, "topk must be in [1, 16]");
  DSV4_CHECK_ARG(world > 0 && world <= EP_MAX_WORLD && n_experts > 0 && n_experts % world == 0,
                 "world must be in [1, 64] and divide n_experts");
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
                           P, (int)topk, (int)(n_experts / world), (int)world, cap, slot_of_assignment, send_meta,
                           ordered_slots, status));
  const int64_t blocks = std::min<int64_t>((P * 32 + 255) / 256, 148 * 8);
  DSV4_CUDA_CHECK(launch_k(ep_pack_rows_kernel, dim3((unsigned)blocks), dim3(256), 0, st, pdl,
                           (const uint16_t*)x_bf16, (const int32_t*)slot_of_assignment, P, (int)topk, (int)hidden,
                           (uint16_t*)send_x_bf16));
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}
