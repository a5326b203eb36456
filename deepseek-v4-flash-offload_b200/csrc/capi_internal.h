// Host-side helpers shared by the C-ABI entry points: thread-local error
// string, argument / CUDA checks that turn into DSV4_E* return codes, and the
// packed expert slot layout.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/dsv4moe.h"

namespace dsv4 {

void set_error(int code, const std::string& msg);
int fail(int code, const std::string& msg);
// Make the device that owns `ptr` current for this library's CUDA runtime
// (the library links its own runtime, so it does not see the caller's
// cudaSetDevice).  Optionally returns the device ordinal.
int bind_device_of(const void* ptr, int* device);
// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// libcuda link): rank-D map over `base` with element strides of 1.
int make_map(CUtensorMap* m, CUtensorMapDataType dt, int rank, void* base, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box, const char* what,
             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// Launch with programmatic stream serialization (PDL) when `pdl`: the kernel
// may start while its stream predecessor finishes; it must call
// griddep_wait() before reading that predecessor's outputs.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Whether kernels are launched with PDL (env DSV4_PDL, default on).
bool pdl_enabled();

// The decode router in one launch (route.cu): partial logits into `part`
// ([H/128][T][E] fp32), a grid barrier on `bar` (two ints, zero before and
// after the launch), top-k.  Launches only when T < 256, E <= 256 and the
// whole grid fits on the GPU at once; *launched reports whether it did.
int route_fused_launch(const void* x_bf16, const float* gate_w, const float* bias, const int32_t* tid2eid,
                       const int64_t* input_ids, int64_t vocab, int64_t n_tokens, int hidden, int n_experts,
                       int topk, int score_func, int renormalize, float route_scale, float* weights_out,
                       int32_t* indices_out, float* part, int* bar, int* status, cudaStream_t st, bool* launched);
// Bytes of `part` for up to n_tokens (< 256) tokens.
inline int64_t route_fused_part_bytes(int64_t n_tokens, int hidden, int n_experts) {
  return (int64_t)(hidden / 128) * n_tokens * n_experts * 4;
}

// Byte layout of one packed expert slot (see include/dsv4moe.h).
struct SlotLayout {
  int64_t w13p;   // [2I, H/2] packed, w1 rows then w3 rows
  int64_t w2p;    // [H, I/2] packed
  int64_t sf13;   // scale atoms of the [2I, H] matrix
  int64_t sf2;    // scale atoms of the [H, I] matrix
  int64_t bytes;  // total
};
inline SlotLayout slot_layout(int64_t hidden, int64_t inter) {
  SlotLayout L;
  L.w13p = 0;
  L.w2p = L.w13p + 2 * inter * hidden / 2;
  L.sf13 = L.w2p + hidden * inter / 2;
  L.sf2 = L.sf13 + 2 * inter * hidden / 32;
  L.bytes = L.sf2 + hidden * inter / 32;
  return L;
}

// Byte layout of the shared expert's FP8 slot: [w13 E4M3 | w2 E4M3 | w13
// scale atoms | w2 scale atoms], blocks as the packed slot but 1 B / element.
inline SlotLayout shared_slot_layout(int64_t hidden, int64_t inter) {
  SlotLayout L;
  L.w13p = 0;
  L.w2p = L.w13p + 2 * inter * hidden;
  L.sf13 = L.w2p + hidden * inter;
  L.sf2 = L.sf13 + 2 * inter * hidden / 32;
  L.bytes = L.sf2 + hidden * inter / 32;
  return L;
}

}  // namespace dsv4

#define DSV4_API_BEGIN try {
#define DSV4_API_END                                              \
  return DSV4_OK;                                                 \
  }                                                               \
  catch (const std::exception& ex) {                              \
    return ::dsv4::fail(DSV4_EINVAL, ex.what());                  \
  }                                                               \
  catch (...) {                                                   \
    return ::dsv4::fail(DSV4_EINVAL, "unknown C++ exception");    \
  }

#define DSV4_CHECK_ARG(cond, msg)                                                     \
  do {                                                                                \
    if (!(cond)) return ::dsv4::fail(DSV4_EINVAL, std::string(__func__) + ": " + (msg)); \
  } while (0)

#define DSV4_CUDA_CHECK(expr)                                                                   \
  do {                                                                                          \
    cudaError_t _e = (expr);                                                                    \
    if (_e != cudaSuccess)                                                                      \
      return ::dsv4::fail(DSV4_ECUDA, std::string(__func__) + ": " + #expr + ": " +             \
                                          cudaGetErrorString(_e));                              \
  } while (0)
