// Shared device helpers for the sm_100a routed-expert kernels: status codes,
// number-format conversions (bf16 / E4M3 / E2M1 / E8M0) and thin inline-PTX
// wrappers for mbarrier, TMA and tcgen05 (TMEM) instructions.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dsv4moe.h"

#ifndef DSV4_WAIT_NS
// Upper bound of every device-side wait (mbarrier phase, cross-role hand-off).
// A wait that runs out records DSV4_ETIMEOUT in the kernel's status word and
// the kernel unwinds instead of spinning forever.
#define DSV4_WAIT_NS 2000000000ull
#endif

namespace dsv4 {

// ---------------------------------------------------------------------------
// number formats
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16r(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
__device__ __forceinline__ uint16_t bf16_bits(float x) {
  __nv_bfloat16 b = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&b);
}
__device__ __forceinline__ float bf16_from_bits(uint32_t b) {
  return __uint_as_float(b << 16);
}

// E2M1 code -> value; code 8 decodes to +0.0 like the reference table.
// Magnitude bits: exponent field e (2 bits), mantissa bit m; e == 0 is the
// subnormal 0 / 0.5, otherwise 2**(e-1) * (1 + m/2).
__device__ __forceinline__ float e2m1_value(uint32_t code) {
  const uint32_t e = (code >> 1) & 3u, m = code & 1u;
  uint32_t bits = e ? (((e + 126u) << 23) | (m << 22)) : (m ? 0x3F000000u : 0u);
  if ((code & 8u) && bits) bits |= 0x80000000u;
  return __uint_as_float(bits);
}

// E8M0 byte -> float 2**(s-127): s=0 is the subnormal 2**-127 and s=255
// overflows to +inf, the values torch.pow(2, s-127) gives in float32.
__device__ __forceinline__ float e8m0_value(uint32_t s) {
  if (s == 0u) return __uint_as_float(0x00400000u);
  if (s == 255u) return __uint_as_float(0x7f800000u);
  return __uint_as_float(s << 23);
}

// 2**k for integer k in [-126, 127].
__device__ __forceinline__ float pow2i(int k) { return __uint_as_float((uint32_t)(k + 127) << 23); }

// Exact ceil(log2(v)) for finite v > 0 (normal or subnormal).
__device__ __forceinline__ int ceil_log2_exact(float v) {
  uint32_t u = __float_as_uint(v);
  int e = (int)((u >> 23) & 0xffu);
  uint32_t m = u & 0x7fffffu;
  if (e == 0) {  // subnormal: v = m * 2**-149
    int msb = 31 - __clz(m);
    return (m == (1u << msb)) ? (msb - 149) : (msb - 148);
  }
  return (e - 127) + (m != 0u ? 1 : 0);
}

// Scale exponent of the per-128 FP8 activation quantisation (act_quant with
// "ue8m0"): amax clamped to >= 1e-4, v = amax * float(1/448), clamped to
// >= 2**-126, k = ceil(log2(v)).
__device__ __forceinline__ int fp8_scale_exp(float amax) {
  float a = fmaxf(amax, 1e-4f);
  float v = __fmul_rn(a, (float)(1.0 / 448.0));
  v = fmaxf(v, __uint_as_float(0x00800000u));
  return ceil_log2_exact(v);
}

// E4M3 (fn) byte of x, x already within [-448, 448]; round to nearest even.
__device__ __forceinline__ uint32_t e4m3_byte(float x) {
  return (uint32_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float e4m3_value(uint32_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

// MXFP4 activation scale exponent: floor(log2(amax/6)) computed exactly,
// clamped to [-127, 127]; amax == 0 gives -127.
__device__ __forceinline__ int mx_scale_exp(float amax) {
  if (!(amax > 0.0f)) return -127;
  uint32_t u = __float_as_uint(amax);
  int e = (int)((u >> 23) & 0xffu);
  int E;
  bool ge15;
  if (e == 0) {
    uint32_t m = u & 0x7fffffu;
    int msb = 31 - __clz(m);
    E = msb - 149;
    ge15 = msb >= 1 && ((m >> (msb - 1)) & 1u);
  } else {
    E = e - 127;
    ge15 = (u & 0x400000u) != 0u;  // mantissa >= 1.5
  }
  int k = E - 3 + (ge15 ? 1 : 0);
  return k < -127 ? -127 : (k > 127 ? 127 : k);
}

// 2**k as float for k in [-149, 127] (exact).
__device__ __forceinline__ float pow2_any(int k) {
  if (k >= -126) return __uint_as_float((uint32_t)(k + 127) << 23);
  return __uint_as_float(1u << (k + 149));
}

// E2M1 code of x (round to nearest, ties to even code, saturate at 6);
// zero results carry no sign bit.  One sm_100a conversion instruction
// (cvt.rn.satfinite.e2m1x2.f32: x into the low nibble, 0 into the high
// one), then a result of magnitude zero loses its sign bit.
__device__ __forceinline__ uint32_t e2m1_code(float x) {
  uint32_t w;
  asm("{\n\t.reg .b8 b;\n\tcvt.rn.satfinite.e2m1x2.f32 b, %2, %1;\n\tmov.b32 %0, {b, b, b, b};\n\t}"
      : "=r"(w)
      : "f"(x), "f"(0.0f));
  const uint32_t c = w & 0xfu;
  return (c & 7u) ? c : 0u;
}

// Activation quantisation of one 128-column block held by a warp, four
// consecutive columns per lane (lane L: columns 4L..4L+3), as the layer's
// quantise-gather does it (the reference's act_quant / dynamic MX quant):
//   FP8: one E4M3 byte per column, the block's scale 2^e with
//        e = fp8_scale_exp(amax of the 128); returns the lane's 4 bytes;
//   MXFP4: one E2M1 code per column, a scale 2^e per 32 columns (lanes
//        8g..8g+7), e = mx_scale_exp(amax of the 32); returns the lane's 4
//        codes packed low nibble first.
__device__ __forceinline__ uint32_t fp8_block_quant(const float v[4], int* e_out) {
  float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const int e = fp8_scale_exp(a);
  const float inv_s = pow2i(-e);
  uint32_t o = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) o |= e4m3_byte(fminf(fmaxf(v[i] * inv_s, -448.f), 448.f)) << (8 * i);
  *e_out = e;
  return o;
}
__device__ __forceinline__ uint32_t mxfp4_block_quant(const float v[4], int* e_out) {
  float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const int e = mx_scale_exp(a);
  const float inv_s = pow2_any(-e);
  *e_out = e;
  return e2m1_code(v[0] * inv_s) | (e2m1_code(v[1] * inv_s) << 4) | (e2m1_code(v[2] * inv_s) << 8) |
         (e2m1_code(v[3] * inv_s) << 12);
}

// ---------------------------------------------------------------------------
// status word shared by a kernel and its host wrapper
// ---------------------------------------------------------------------------
__device__ __forceinline__ void set_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}
__device__ __forceinline__ int read_status(const int* status) {
  return status ? *(volatile const int*)status : 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// programmatic dependent launch: a kernel waits for its stream predecessor
// (complete, memory visible) before reading its outputs, then lets its own
// successor start.  Waiting before releasing keeps every kernel older than
// the predecessor complete when a kernel starts.  Both are no-ops for a
// kernel launched without the programmatic-serialization attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// shared-memory addresses, mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0u;
}
// Bounded wait for the phase with the given parity.  Returns false (and
// records DSV4_ETIMEOUT) when the limit runs out or when another wait of the
// kernel already timed out; the caller then unwinds.  Other status codes
// (bad input) only mark the result invalid and do not stop the pipeline.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (read_status(status) == DSV4_ETIMEOUT) return false;
    if (globaltimer_ns() - t0 > DSV4_WAIT_NS) {
      set_status(status, DSV4_ETIMEOUT);
      return false;
    }
  }
}
// Counters between the CTAs of one grid: a release add after the counted
// stores, an acquire load before the dependent reads; the wait is bounded
// like mbar_wait (DSV4_ETIMEOUT, or another wait's timeout, ends it).
__device__ __forceinline__ void red_release_add(int* addr, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire(const int* addr) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ bool wait_count_geq(const int* addr, int target, int* status) {
  if (ld_acquire(addr) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    __nanosleep(64);
    if (ld_acquire(addr) >= target) return true;
    if (read_status(status) == DSV4_ETIMEOUT) return false;
    if (globaltimer_ns() - t0 > DSV4_WAIT_NS) {
      set_status(status, DSV4_ETIMEOUT);
      return false;
    }
  }
}
// generic-proxy stores made visible by an acquire, then read by TMA (the
// async proxy) in this thread
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// TMA and bulk copies (no cluster multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3, int c4, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 / TMEM
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// Copy a 32-row x 128-bit block of scale factors from shared memory into the
// 128 TMEM lanes (replicated into each 32-lane sub-partition).
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void tc_mma_mxf8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate, uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// Packed E2M1 x E2M1 (two elements per byte in shared memory), 64 of K per
// instruction, one E8M0 scale per 32 elements (two per row per instruction).
__device__ __forceinline__ void tc_mma_mxf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate, uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.scale_vec::2X [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// bf16 x bf16 -> fp32 in TMEM, both operands K-major in shared memory.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Instruction descriptor of kind::f16 with bf16 A and B, fp32 D, both K-major.
__host__ __device__ __forceinline__ uint32_t idesc_bf16(int m, int n) {
  uint32_t d = 0;
  d |= 1u << 4;                        // D format F32
  d |= 1u << 7;                        // A format BF16
  d |= 1u << 10;                       // B format BF16
  d |= ((uint32_t)(n >> 3) & 63u) << 17;
  d |= ((uint32_t)(m >> 4) & 31u) << 24;
  return d;
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 8 consecutive 32-bit columns -> 8 registers per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 lanes x 16 consecutive 32-bit columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row atoms of
// 128 B, atoms 1024 B apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}
// K-major, 64-byte swizzle: 8-row atoms of 64 B, atoms 512 B apart (packed
// E2M1: 128 elements per row).
__device__ __forceinline__ uint64_t desc_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(512u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)4u << 61;
  return d;
}
// Descriptor of a 32-row x 16-byte scale-factor block (no swizzle, 8-row
// core matrices 128 B apart), the source of tc_cp_sf.
__device__ __forceinline__ uint64_t desc_sf(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(128u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}
// Instruction descriptor of kind::mxf8f6f4.block_scale with A = E2M1 (or
// E4M3 with a_e4m3: the shared expert's FP8 weights), B = E4M3 (b_fp4 =
// false) or E2M1, M = 128, E8M0 scales, both K-major.
__host__ __device__ __forceinline__ uint32_t idesc_mxf8f6f4(int n, bool b_fp4, uint32_t sf_id, bool a_e4m3 = false) {
  uint32_t d = 0;
  d |= (sf_id & 3u) << 4;              // B scale-factor id
  d |= (a_e4m3 ? 0u : 5u) << 7;        // A format E4M3 / E2M1
  d |= (b_fp4 ? 5u : 0u) << 10;        // B format E2M1 / E4M3
  d |= ((uint32_t)(n >> 3) & 63u) << 17;
  d |= 1u << 23;                       // scale format UE8M0
  d |= (128u >> 4) << 24;              // M = 128
  d |= (sf_id & 3u) << 29;             // A scale-factor id
  return d;
}
// Instruction descriptor of kind::mxf4.block_scale.scale_vec::2X: A = B =
// E2M1 (format code 1 of this kind), M = 128, E8M0 scales, both K-major;
// sf_id 0 or 2 picks the scale byte pair of the 64-element K step.
__host__ __device__ __forceinline__ uint32_t idesc_mxf4(int n, uint32_t sf_id) {
  uint32_t d = 0;
  d |= (sf_id & 3u) << 4;              // B scale-factor id
  d |= 1u << 7;                        // A format E2M1
  d |= 1u << 10;                       // B format E2M1
  d |= ((uint32_t)(n >> 3) & 63u) << 17;
  d |= 1u << 23;                       // scale format UE8M0
  d |= (128u >> 4) << 24;              // M = 128
  d |= (sf_id & 3u) << 29;             // A scale-factor id
  return d;
}

}  // namespace dsv4
