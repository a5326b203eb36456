// Tensor-core rate of the two block-scaled MMA kinds the grouped GEMM uses,
// measured on this GPU: the denominators of the prefill roofline.
//   kind 0: tcgen05.mma.kind::mxf4.block_scale.scale_vec::2X (a4w4 profile:
//           E2M1 x E2M1, 64 of K per instruction);
//   kind 1: tcgen05.mma.kind::mxf8f6f4.block_scale (bf16 profile: E2M1
//           weights x E4M3 activations, 32 of K per instruction).
// One CTA per SM; one thread issues MMAs of M = 128, N = n back to back from
// operands that stay in shared memory, accumulating into one TMEM tile, so
// only the tensor pipe limits the rate.  The operand bytes are zeros: the
// rate of the pipe does not depend on them.
#include <algorithm>

#include "capi_internal.h"
#include "common.cuh"

namespace dsv4 {

constexpr int MP_THREADS = 128;

template <int KIND>
__global__ void __launch_bounds__(MP_THREADS, 1) mma_peak_kernel(int64_t iters, int n, int* status) {
  extern __shared__ __align__(1024) uint8_t mp_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(mp_raw) + 1023) & ~uintptr_t(1023));
  constexpr int ROW = KIND == 0 ? 64 : 128;   // bytes per row of a 128-element k-tile
  uint8_t* sA = smem;                          // 128 rows
  uint8_t* sB = sA + 128 * ROW;                // n rows
  uint8_t* sSF = sB + 256 * ROW;               // 2 x 512 B scale atoms
  uint64_t* bar = reinterpret_cast<uint64_t*>(sSF + 1024);
  uint32_t* holder = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x;
  for (int i = tid; i < (128 * ROW + 256 * ROW + 1024) / 16; i += MP_THREADS)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (tid < 32) {
    tmem_alloc(holder, 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;
  if (tid == 0) {
    const uint32_t sfa = tmem + 256, sfb = tmem + 260;
    tc_cp_sf(sfa, desc_sf(smem_u32(sSF)));
    tc_cp_sf(sfb, desc_sf(smem_u32(sSF + 512)));
    const uint32_t aA = smem_u32(sA), aB = smem_u32(sB);
    for (int64_t it = 0; it < iters; ++it) {
      if constexpr (KIND == 0) {
        const uint64_t dA = desc_sw64(aA), dB = desc_sw64(aB);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint32_t sel = (2u * kb) << 30;
          tc_mma_mxf4(tmem, dA + 2u * kb, dB + 2u * kb, idesc_mxf4(n, 2u * kb), (it | kb) != 0 ? 1u : 0u,
                      sfa | sel, sfb | sel);
        }
      } else {
        const uint64_t dA = desc_sw128(aA), dB = desc_sw128(aB);
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          const uint32_t sel = (uint32_t)kb << 30;
          tc_mma_mxf8f6f4(tmem, dA + 2u * kb, dB + 2u * kb, idesc_mxf8f6f4(n, false, (uint32_t)kb),
                          (it | kb) != 0 ? 1u : 0u, sfa | sel, sfb | sel);
        }
      }
    }
    tc_commit(bar);
    if (!mbar_wait(bar, 0, status)) {
      // the MMAs did not drain in time: wait once more (bounded) before the
      // TMEM they write is freed
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(bar, 0) && globaltimer_ns() - t0 < DSV4_WAIT_NS) {
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (tid < 32) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace dsv4

using namespace dsv4;

extern "C" int dsv4_mma_peak(int32_t kind, int32_t n, int64_t iters, int32_t device, double* tflops_out,
                             double* ms_out) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(tflops_out, "null pointer");
  DSV4_CHECK_ARG(kind == 0 || kind == 1, "kind must be 0 (mxf4) or 1 (mxf8f6f4)");
  DSV4_CHECK_ARG(n >= 16 && n <= 256 && n % 16 == 0, "n must be a multiple of 16 in [16, 256]");
  DSV4_CHECK_ARG(iters > 0 && iters < (1LL << 40), "iters must be positive");
  DSV4_CUDA_CHECK(cudaSetDevice(device));
  int sms = 0;
  DSV4_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  const int row = kind == 0 ? 64 : 128;
  // at least 120 KB so that one CTA (and one 512-column TMEM allocation) sits on each SM
  const size_t smem = std::max<size_t>(1024 + (size_t)(128 + 256) * row + 1024 + 64, 120 * 1024);
  void (*k)(int64_t, int, int*) = kind == 0 ? mma_peak_kernel<0> : mma_peak_kernel<1>;
  DSV4_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int* status = nullptr;
  DSV4_CUDA_CHECK(cudaMalloc(&status, sizeof(int)));
  DSV4_CUDA_CHECK(cudaMemset(status, 0, sizeof(int)));
  cudaEvent_t e0, e1;
  DSV4_CUDA_CHECK(cudaEventCreate(&e0));
  DSV4_CUDA_CHECK(cudaEventCreate(&e1));
  k<<<sms, MP_THREADS, smem>>>(iters / 8 + 1, n, status);   // warm-up
  DSV4_CUDA_CHECK(cudaEventRecord(e0));
  k<<<sms, MP_THREADS, smem>>>(iters, n, status);
  DSV4_CUDA_CHECK(cudaEventRecord(e1));
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_CUDA_CHECK(cudaEventSynchronize(e1));
  float ms = 0.f;
  DSV4_CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
  int st = 0;
  DSV4_CUDA_CHECK(cudaMemcpy(&st, status, sizeof(int), cudaMemcpyDeviceToHost));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFree(status);
  if (st != 0) return fail(st, "dsv4_mma_peak: a bounded wait ran out");
  const double k_per_iter = 128.0;   // one 128-element k-tile per iteration
  const double flops = 2.0 * 128.0 * n * k_per_iter * (double)iters * sms;
  *tflops_out = flops / (ms * 1e-3) / 1e12;
  if (ms_out) *ms_out = ms;
  DSV4_API_END
}
