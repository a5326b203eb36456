// C-ABI basics: error reporting, ABI version and the host-side packing of a
// checkpoint expert (six tensors) into one kernel-native slot.
#include <string.h>

#include <string>

#include "capi_internal.h"

namespace dsv4 {

static thread_local std::string g_last_error;

void set_error(int code, const std::string& msg) {
  g_last_error = "dsv4 error " + std::to_string(code) + ": " + msg;
}

int fail(int code, const std::string& msg) {
  set_error(code, msg);
  return code;
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

// Scale bytes of a [rows, k] matrix (row-major [rows, k/32]) -> 512-byte
// atoms of 128 rows x 4 blocks: atom (r/128, kb/4) holds row r at byte
// (r%32)*16 + ((r%128)/32)*4 + kb%4.  This is the order in which the tensor
// cores read block scales from TMEM after a 32x128b.warpx4 copy.
static void tile_scales(const uint8_t* s, int64_t rows, int64_t k, uint8_t* dst, int64_t row_base) {
  const int64_t kb_n = k / 32, ktiles = k / 128;
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t R = row_base + r;
    for (int64_t kb = 0; kb < kb_n; ++kb) {
      const int64_t off = ((R / 128) * ktiles + kb / 4) * 512 + (R % 32) * 16 + ((R % 128) / 32) * 4 + (kb % 4);
      dst[off] = s[r * kb_n + kb];
    }
  }
}

static void untile_scales(const uint8_t* src, int64_t rows, int64_t k, uint8_t* s, int64_t row_base) {
  const int64_t kb_n = k / 32, ktiles = k / 128;
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t R = row_base + r;
    for (int64_t kb = 0; kb < kb_n; ++kb) {
      const int64_t off = ((R / 128) * ktiles + kb / 4) * 512 + (R % 32) * 16 + ((R % 128) / 32) * 4 + (kb % 4);
      s[r * kb_n + kb] = src[off];
    }
  }
}

// Packed weights [rows, k/2] (row-major, two E2M1 per byte) -> 8 KiB blocks of
// 128 rows x 128 elements: block (r/128, k/128) at ((r/128)*(k/128) + k/128)*8192,
// row r%128 of the block at (r%128)*64.  One TMA box = one contiguous block.
static void tile_weights(const uint8_t* w, int64_t rows, int64_t k, uint8_t* dst, int64_t row_base) {
  const int64_t kt_n = k / 128, row_bytes = k / 2;
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t R = row_base + r;
    for (int64_t kt = 0; kt < kt_n; ++kt)
      memcpy(dst + ((R / 128) * kt_n + kt) * 8192 + (R % 128) * 64, w + r * row_bytes + kt * 64, 64);
  }
}

static void untile_weights(const uint8_t* src, int64_t rows, int64_t k, uint8_t* w, int64_t row_base) {
  const int64_t kt_n = k / 128, row_bytes = k / 2;
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t R = row_base + r;
    for (int64_t kt = 0; kt < kt_n; ++kt)
      memcpy(w + r * row_bytes + kt * 64, src + ((R / 128) * kt_n + kt) * 8192 + (R % 128) * 64, 64);
  }
}

}  // namespace dsv4

using namespace dsv4;

extern "C" const char* dsv4_last_error_string(void) { return g_last_error.c_str(); }

extern "C" int dsv4_abi_version(void) { return DSV4_ABI_VERSION; }

extern "C" int64_t dsv4_expert_slot_bytes(int32_t hidden, int32_t inter) {
  if (hidden <= 0 || inter <= 0 || hidden % 128 || inter % 128) return DSV4_EINVAL;
  return slot_layout(hidden, inter).bytes;
}

extern "C" int dsv4_pack_expert_host(const uint8_t* w1p, const uint8_t* w1s, const uint8_t* w2p,
                                     const uint8_t* w2s, const uint8_t* w3p, const uint8_t* w3s, int32_t hidden,
                                     int32_t inter, uint8_t* slot) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(w1p && w1s && w2p && w2s && w3p && w3s && slot, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && inter > 0 && hidden % 128 == 0 && inter % 128 == 0,
                 "hidden and inter must be positive multiples of 128");
  const SlotLayout L = slot_layout(hidden, inter);
  const int64_t H = hidden, I = inter;
  tile_weights(w1p, I, H, slot + L.w13p, 0);
  tile_weights(w3p, I, H, slot + L.w13p, I);
  tile_weights(w2p, H, I, slot + L.w2p, 0);
  tile_scales(w1s, I, H, slot + L.sf13, 0);
  tile_scales(w3s, I, H, slot + L.sf13, I);
  tile_scales(w2s, H, I, slot + L.sf2, 0);
  DSV4_API_END
}

extern "C" int dsv4_unpack_expert_host(const uint8_t* slot, int32_t hidden, int32_t inter, uint8_t* w1p,
                                       uint8_t* w1s, uint8_t* w2p, uint8_t* w2s, uint8_t* w3p, uint8_t* w3s) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(w1p && w1s && w2p && w2s && w3p && w3s && slot, "null pointer");
  DSV4_CHECK_ARG(hidden > 0 && inter > 0 && hidden % 128 == 0 && inter % 128 == 0,
                 "hidden and inter must be positive multiples of 128");
  const SlotLayout L = slot_layout(hidden, inter);
  const int64_t H = hidden, I = inter;
  untile_weights(slot + L.w13p, I, H, w1p, 0);
  untile_weights(slot + L.w13p, I, H, w3p, I);
  untile_weights(slot + L.w2p, H, I, w2p, 0);
  untile_scales(slot + L.sf13, I, H, w1s, 0);
  untile_scales(slot + L.sf13, I, H, w3s, I);
  untile_scales(slot + L.sf2, H, I, w2s, 0);
  DSV4_API_END
}
