// Element-wise kernels: MXFP4 weight dequant (checkpoint layout and slot
// layout), FP8-E4M3 activation round trip, MXFP4 activation quantisation.
// All are HBM-bound: 128-bit loads/stores, one warp per 128-element block.
#include "capi_internal.h"
#include "common.cuh"
#include "slot_layout.h"

namespace dsv4 {

// ---------------------------------------------------------------------------
// dequant_fp4_weight (npu_ops.py:142-158): one thread = one 32-element scale
// block = 16 packed bytes in, 64 bytes of bf16 out.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void dequant_block32(const uint8_t* src16, uint32_t sbyte, uint16_t* dst32) {
  const uint4 raw = *reinterpret_cast<const uint4*>(src16);
  const float s = e8m0_value(sbyte);
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t o[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const uint32_t byte = (w[q] >> (8 * b)) & 0xffu;
      const uint32_t lo = bf16_bits(e2m1_value(byte & 0xfu) * s);
      const uint32_t hi = bf16_bits(e2m1_value(byte >> 4) * s);
      o[b] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(dst32 + q * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void dequant_mxfp4_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ s,
                                     uint16_t* __restrict__ out, int64_t rows, int64_t k) {
  const int64_t kb = k / 32;
  const int64_t n = rows * kb;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < n; c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = c / kb, b = c - r * kb;
    dequant_block32(w + r * (k / 2) + b * 16, s[c], out + r * k + b * 32);
  }
}

// Dequant of one matrix of a packed slot (layout in slot_layout.h); row r of
// the output is paired-matrix row (r/128)*pair_stride + pair_base + r%128.
__global__ void slot_dequant_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ sf,
                                    uint16_t* __restrict__ out, int64_t rows, int64_t k, int pair_stride,
                                    int pair_base) {
  const int64_t kb = k / 32;
  const int64_t n = rows * kb;
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < n; c += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = c / kb, b = c - r * kb;
    const int64_t R = (r / 128) * pair_stride + pair_base + r % 128;
    dequant_block32(w + w_pair_offset(R, b * 32, k), sf[sf_pair_offset(R, b, k)], out + r * k + b * 32);
  }
}

// ---------------------------------------------------------------------------
// act_quant in place (npu_ops.py:73-98): one warp per 128-element block, four
// elements per lane.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__global__ void act_quant_fp8_rt_kernel(uint16_t* __restrict__ x, int64_t rows, int64_t cols) {
  const int lane = threadIdx.x & 31;
  const int64_t nblk = rows * (cols / 128);
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = warp0; b < nblk; b += nwarps) {
    uint16_t* p = x + b * 128 + lane * 4;
    uint2 raw = *reinterpret_cast<const uint2*>(p);
    float v[4] = {bf16_from_bits(raw.x & 0xffffu), bf16_from_bits(raw.x >> 16), bf16_from_bits(raw.y & 0xffffu),
                  bf16_from_bits(raw.y >> 16)};
    float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    a = warp_max(a);
    const int e = fp8_scale_exp(a);
    const float inv = pow2i(-e), s = pow2i(e);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float q = fminf(fmaxf(v[i] * inv, -448.0f), 448.0f);
      o[i] = bf16_bits(e4m3_value(e4m3_byte(q)) * s);
    }
    *reinterpret_cast<uint2*>(p) = make_uint2(o[0] | (o[1] << 16), o[2] | (o[3] << 16));
  }
}

// ---------------------------------------------------------------------------
// MXFP4 activation quant: one warp per 128 elements = four 32-blocks of eight
// lanes; packed output low nibble = even element.
// ---------------------------------------------------------------------------
__global__ void act_quant_mxfp4_kernel(const uint16_t* __restrict__ x, int64_t rows, int64_t cols,
                                       uint8_t* __restrict__ q, uint8_t* __restrict__ sc) {
  const int lane = threadIdx.x & 31;
  const int64_t nblk = rows * (cols / 128);
  const int64_t warp0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t b = warp0; b < nblk; b += nwarps) {
    const uint2 raw = *reinterpret_cast<const uint2*>(x + b * 128 + lane * 4);
    float v[4] = {bf16_from_bits(raw.x & 0xffffu), bf16_from_bits(raw.x >> 16), bf16_from_bits(raw.y & 0xffffu),
                  bf16_from_bits(raw.y >> 16)};
    float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const int e = mx_scale_exp(a);
    const float inv = pow2_any(-e);
    const uint32_t c0 = e2m1_code(v[0] * inv), c1 = e2m1_code(v[1] * inv);
    const uint32_t c2 = e2m1_code(v[2] * inv), c3 = e2m1_code(v[3] * inv);
    const uint16_t packed = (uint16_t)(c0 | (c1 << 4) | (c2 << 8) | (c3 << 12));
    *reinterpret_cast<uint16_t*>(q + b * 64 + lane * 2) = packed;
    if ((lane & 7) == 0) sc[b * 4 + (lane >> 3)] = (uint8_t)(e + 127);
  }
}

static int grid_for(int64_t work_items, int threads) {
  int64_t g = (work_items + threads - 1) / threads;
  const int64_t cap = 148LL * 16;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace dsv4

using namespace dsv4;

extern "C" int dsv4_dequant_mxfp4(const uint8_t* w_packed, const uint8_t* scale, void* out_bf16, int64_t rows,
                                  int64_t k, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(w_packed && scale && out_bf16, "null pointer");
  DSV4_CHECK_ARG(rows >= 0 && k > 0 && k % 32 == 0, "k must be a positive multiple of 32");
  DSV4_CHECK_ARG(((uintptr_t)w_packed % 16) == 0 && ((uintptr_t)out_bf16 % 16) == 0,
                 "w_packed and out must be 16-byte aligned");
  if (rows == 0) return DSV4_OK;
  if (int rc = bind_device_of(w_packed, nullptr)) return rc;
  const int64_t items = rows * (k / 32);
  dequant_mxfp4_kernel<<<grid_for(items, 256), 256, 0, (cudaStream_t)stream>>>(w_packed, scale, (uint16_t*)out_bf16,
                                                                                rows, k);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

extern "C" int dsv4_slot_dequant(const uint8_t* slot, int32_t hidden, int32_t inter, void* w1, void* w2, void* w3,
                                 void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(slot && w1 && w2 && w3, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && inter > 0 && hidden % 256 == 0 && inter % 128 == 0,
                 "hidden must be a positive multiple of 256 and inter of 128");
  const SlotLayout L = slot_layout(hidden, inter);
  if (int rc = bind_device_of(slot, nullptr)) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t items13 = (int64_t)inter * (hidden / 32), items2 = (int64_t)hidden * (inter / 32);
  // w1 row r is paired row (r/128)*256 + r%128, w3 row r is (r/128)*256 + 128 + r%128, w2 row r is r
  slot_dequant_kernel<<<grid_for(items13, 256), 256, 0, st>>>(slot + L.w13p, slot + L.sf13, (uint16_t*)w1, inter,
                                                              hidden, 256, 0);
  slot_dequant_kernel<<<grid_for(items13, 256), 256, 0, st>>>(slot + L.w13p, slot + L.sf13, (uint16_t*)w3, inter,
                                                              hidden, 256, 128);
  slot_dequant_kernel<<<grid_for(items2, 256), 256, 0, st>>>(slot + L.w2p, slot + L.sf2, (uint16_t*)w2, hidden,
                                                             inter, 128, 0);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

extern "C" int dsv4_act_quant_fp8_rt(void* x_bf16, int64_t rows, int64_t cols, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16, "null pointer");
  DSV4_CHECK_ARG(rows >= 0 && cols > 0 && cols % 128 == 0, "cols must be a positive multiple of 128");
  DSV4_CHECK_ARG(((uintptr_t)x_bf16 % 8) == 0, "x must be 8-byte aligned");
  if (rows == 0) return DSV4_OK;
  if (int rc = bind_device_of(x_bf16, nullptr)) return rc;
  const int64_t warps = rows * (cols / 128);
  act_quant_fp8_rt_kernel<<<grid_for(warps * 32, 256), 256, 0, (cudaStream_t)stream>>>((uint16_t*)x_bf16, rows,
                                                                                        cols);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

extern "C" int dsv4_act_quant_mxfp4(const void* x_bf16, int64_t rows, int64_t cols, uint8_t* q_packed,
                                    uint8_t* scale, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(x_bf16 && q_packed && scale, "null pointer");
  DSV4_CHECK_ARG(rows >= 0 && cols > 0 && cols % 128 == 0, "cols must be a positive multiple of 128");
  DSV4_CHECK_ARG(((uintptr_t)x_bf16 % 8) == 0 && ((uintptr_t)q_packed % 2) == 0, "misaligned pointer");
  if (rows == 0) return DSV4_OK;
  if (int rc = bind_device_of(x_bf16, nullptr)) return rc;
  const int64_t warps = rows * (cols / 128);
  act_quant_mxfp4_kernel<<<grid_for(warps * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)x_bf16, rows, cols, q_packed, scale);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}
