// C-ABI basics: error reporting, ABI version and the host-side packing of a
// checkpoint expert (six tensors) into one kernel-native slot.
#include <stdlib.h>
#include <string.h>

#include <string>

#include "capi_internal.h"
#include "slot_layout.h"

namespace dsv4 {

static thread_local std::string g_last_error;

void set_error(int code, const std::string& msg) {
  g_last_error = "dsv4 error " + std::to_string(code) + ": " + msg;
}

int fail(int code, const std::string& msg) {
  set_error(code, msg);
  return code;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("DSV4_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

int bind_device_of(const void* ptr, int* device) {
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, ptr);
  if (e != cudaSuccess) return fail(DSV4_ECUDA, std::string("cudaPointerGetAttributes: ") + cudaGetErrorString(e));
  if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
    return fail(DSV4_EINVAL, "expected a device pointer");
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != a.device) {
    e = cudaSetDevice(a.device);
    if (e != cudaSuccess) return fail(DSV4_ECUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  }
  if (device) *device = a.device;
  return DSV4_OK;
}

// Checkpoint tensors [rows, k/2] packed weights and [rows, k/32] scales of
// one matrix -> the paired slot layout (slot_layout.h).  which_of(r) gives the
// paired-matrix row of checkpoint row r.
template <typename RowMap>
static void pack_matrix(const uint8_t* w, const uint8_t* s, int64_t rows, int64_t k, uint8_t* wdst, uint8_t* sdst,
                        RowMap row_of) {
  const int64_t kb_n = k / 32;
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t R = row_of(r);
    for (int64_t kt = 0; kt < k / 128; ++kt) memcpy(wdst + w_pair_offset(R, kt * 128, k), w + r * (k / 2) + kt * 64, 64);
    for (int64_t kb = 0; kb < kb_n; ++kb) sdst[sf_pair_offset(R, kb, k)] = s[r * kb_n + kb];
  }
}

template <typename RowMap>
static void unpack_matrix(const uint8_t* wsrc, const uint8_t* ssrc, int64_t rows, int64_t k, uint8_t* w, uint8_t* s,
                          RowMap row_of) {
  const int64_t kb_n = k / 32;
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t R = row_of(r);
    for (int64_t kt = 0; kt < k / 128; ++kt) memcpy(w + r * (k / 2) + kt * 64, wsrc + w_pair_offset(R, kt * 128, k), 64);
    for (int64_t kb = 0; kb < kb_n; ++kb) s[r * kb_n + kb] = ssrc[sf_pair_offset(R, kb, k)];
  }
}

}  // namespace dsv4

using namespace dsv4;

extern "C" const char* dsv4_last_error_string(void) { return g_last_error.c_str(); }

extern "C" int dsv4_abi_version(void) { return DSV4_ABI_VERSION; }

extern "C" int64_t dsv4_expert_slot_bytes(int32_t hidden, int32_t inter) {
  if (hidden <= 0 || inter <= 0 || hidden % 256 || inter % 128) return DSV4_EINVAL;
  return slot_layout(hidden, inter).bytes;
}

extern "C" int dsv4_pack_expert_host(const uint8_t* w1p, const uint8_t* w1s, const uint8_t* w2p,
                                     const uint8_t* w2s, const uint8_t* w3p, const uint8_t* w3s, int32_t hidden,
                                     int32_t inter, uint8_t* slot) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(w1p && w1s && w2p && w2s && w3p && w3s && slot, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && inter > 0 && hidden % 256 == 0 && inter % 128 == 0,
                 "hidden must be a positive multiple of 256 and inter of 128");
  const SlotLayout L = slot_layout(hidden, inter);
  const int64_t H = hidden, I = inter;
  pack_matrix(w1p, w1s, I, H, slot + L.w13p, slot + L.sf13, [](int64_t r) { return w13_pair_row(r, 0); });
  pack_matrix(w3p, w3s, I, H, slot + L.w13p, slot + L.sf13, [](int64_t r) { return w13_pair_row(r, 1); });
  pack_matrix(w2p, w2s, H, I, slot + L.w2p, slot + L.sf2, [](int64_t r) { return r; });
  DSV4_API_END
}

extern "C" int dsv4_unpack_expert_host(const uint8_t* slot, int32_t hidden, int32_t inter, uint8_t* w1p,
                                       uint8_t* w1s, uint8_t* w2p, uint8_t* w2s, uint8_t* w3p, uint8_t* w3s) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(w1p && w1s && w2p && w2s && w3p && w3s && slot, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && inter > 0 && hidden % 256 == 0 && inter % 128 == 0,
                 "hidden must be a positive multiple of 256 and inter of 128");
  const SlotLayout L = slot_layout(hidden, inter);
  const int64_t H = hidden, I = inter;
  unpack_matrix(slot + L.w13p, slot + L.sf13, I, H, w1p, w1s, [](int64_t r) { return w13_pair_row(r, 0); });
  unpack_matrix(slot + L.w13p, slot + L.sf13, I, H, w3p, w3s, [](int64_t r) { return w13_pair_row(r, 1); });
  unpack_matrix(slot + L.w2p, slot + L.sf2, H, I, w2p, w2s, [](int64_t r) { return r; });
  DSV4_API_END
}

// ---------------------------------------------------------------------------
// Shared expert (deepseek_v4.py:87-100; model_npu.py:469-491 Expert in "fp8"
// mode): w1 / w3 [I, H] and w2 [H, I] E4M3 with one E8M0 scale per 128 x 128
// block (npu_ops.py:161-167 dequant_fp8_weight), packed into the FP8 slot the
// grouped GEMM reads (slot_layout.h w8_pair_offset): the block scale is
// written as the per-32 scale of each of its four 32-element groups.
// ---------------------------------------------------------------------------
namespace dsv4 {
template <typename RowMap>
static void pack_matrix_fp8(const uint8_t* w, const uint8_t* s, int64_t rows, int64_t k, uint8_t* wdst, uint8_t* sdst,
                            RowMap row_of) {
  const int64_t kb_n = k / 32, sk = (k + 127) / 128;
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t R = row_of(r);
    for (int64_t kt = 0; kt < k / 128; ++kt) memcpy(wdst + w8_pair_offset(R, kt * 128, k), w + r * k + kt * 128, 128);
    for (int64_t kb = 0; kb < kb_n; ++kb) sdst[sf_pair_offset(R, kb, k)] = s[(r / 128) * sk + kb / 4];
  }
}
}  // namespace dsv4

extern "C" int64_t dsv4_shared_slot_bytes(int32_t hidden, int32_t inter) {
  if (hidden <= 0 || inter <= 0 || hidden % 256 || inter % 128) return DSV4_EINVAL;
  return shared_slot_layout(hidden, inter).bytes;
}

extern "C" int dsv4_pack_shared_host(const uint8_t* w1, const uint8_t* s1, const uint8_t* w2, const uint8_t* s2,
                                     const uint8_t* w3, const uint8_t* s3, int32_t hidden, int32_t inter,
                                     uint8_t* slot) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(w1 && s1 && w2 && s2 && w3 && s3 && slot, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && inter > 0 && hidden % 256 == 0 && inter % 128 == 0,
                 "hidden must be a positive multiple of 256 and inter of 128");
  const SlotLayout L = shared_slot_layout(hidden, inter);
  const int64_t H = hidden, I = inter;
  pack_matrix_fp8(w1, s1, I, H, slot + L.w13p, slot + L.sf13, [](int64_t r) { return w13_pair_row(r, 0); });
  pack_matrix_fp8(w3, s3, I, H, slot + L.w13p, slot + L.sf13, [](int64_t r) { return w13_pair_row(r, 1); });
  pack_matrix_fp8(w2, s2, H, I, slot + L.w2p, slot + L.sf2, [](int64_t r) { return r; });
  DSV4_API_END
}
