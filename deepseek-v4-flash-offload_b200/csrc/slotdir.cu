// Device-resident expert slot directory: the LRU of ExpertBank.get_packed
// (offload.py:103-129) kept in HBM, so that a layer whose experts are only
// partly resident never waits for the host.
//
// The host LRU (slotcache.cpp) needs the routing on the host: one device ->
// host copy and a stream synchronisation per layer, after which the host
// issues the copies of the missed experts.  Here the router's output stays
// on the device:
//   resolve  one CTA reads the layer's [T, k] expert ids, walks the active
//            experts in ascending id order exactly like the host LRU (a hit
//            moves the key to the most-recently-used end, a miss takes a free
//            slot, lowest index first, else evicts the least recently used
//            key that is not part of the batch), updates the (layer, expert)
//            -> slot table that the grouped GEMM reads, and lists the misses;
//   fetch    the GPU copies each missed expert's packed slot from the pinned
//            host pool (mapped into the device address space: zero-copy
//            reads over PCIe, 16 bytes per thread, many requests in flight)
//            into its HBM slot.
// Both are asynchronous on the caller's stream and have a fixed launch shape,
// so an offloaded decode step can be captured in a CUDA graph.
//
// Recency is a per-slot stamp from a global access clock: the i-th active
// expert of a batch gets stamp clock + 1 + i.  Because keys of the batch are
// never evicted by the batch, the m misses of a batch take the m non-batch
// slots of smallest (stamp, slot) (free slots have stamp 0), in order, which
// is the host LRU's choice key by key.
//
// Prefetch: a resolve in prefetch mode (the predicted experts of the next
// layer, on a side stream, while the current layer's GEMMs run) may only
// evict slots whose stamp is older than the last demand batch, so it never
// overwrites an expert that the layer in flight reads; when no such slot is
// left it skips the rest of its list.  Demand and prefetch keep separate
// miss lists.
#include <algorithm>
#include <memory>
#include <string>
#include <vector>

#include "capi_internal.h"
#include "common.cuh"

namespace dsv4 {

constexpr int SD_THREADS = 1024;
// 128 threads of at most 40 registers: one fetch CTA fits beside a grouped-GEMM
// CTA on an SM (352 threads x 168 registers, 221 KB of shared memory), so a
// prefetch runs under the GEMM instead of waiting for its SMs
constexpr int SD_FETCH_THREADS = 128;
constexpr int SD_STAT_N = 8;   // hits, misses, evictions, pf_hits, pf_fetched, pf_evictions, pf_skipped, batches

struct SdHeader {
  int status;
  int n_fetch[2];   // misses listed by the last demand (0) / prefetch (1) resolve
  int pad;
  long long clock;     // last stamp handed out
  long long protect;   // stamps >= protect belong to the demand batch in flight
  long long stats[SD_STAT_N];
};

struct SdPtrs {
  SdHeader* h;
  int32_t* dir;     // [L * E] slot of (layer, expert) or -1
  int32_t* key;     // [S] layer * E + expert held by the slot, or -1
  int64_t* stamp;   // [S] last access (0: free)
  const uint8_t* const* src;   // [L * E] device address of the pinned host slot, or null
  int2* list;       // [2][max_list] (slot, key) of the listed misses
  int max_list;
  int L, E, S;
};

__device__ __forceinline__ int sd_block_scan(int v, int* scratch, int* total) {
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
  *total = scratch[31];
  __syncthreads();
  return excl;
}

// One CTA of 1024 threads.  Shared memory (below the 48 KB default for
// E <= 1024 and S <= DSV4_SLOTDIR_MAX_SLOTS): the ascending lists of missing
// experts and of their batch positions, act[E] u8, inb[S] u8.
__global__ void __launch_bounds__(SD_THREADS, 1)
    slotdir_resolve_kernel(SdPtrs d, const int32_t* __restrict__ idx, int P, int layer, int mode) {
  extern __shared__ int sd_sm[];
  int* scratch = sd_sm;                     // 32
  int* bcast = scratch + 32;                // 4
  int* miss_e = bcast + 4;                  // E
  int* miss_pos = miss_e + d.E;             // E
  uint8_t* act = reinterpret_cast<uint8_t*>(miss_pos + d.E);   // E
  uint8_t* inb = act + d.E;                 // S
  const int tid = threadIdx.x;
  const int E = d.E, S = d.S;
  const int base = layer * E;
  for (int e = tid; e < E; e += SD_THREADS) act[e] = 0;
  for (int s = tid; s < S; s += SD_THREADS) inb[s] = 0;
  __syncthreads();
  for (int p = tid; p < P; p += SD_THREADS) {
    const int e = idx[p];
    if (e >= 0 && e < E) act[e] = 1;
  }
  __syncthreads();
  // ascending active list (E <= SD_THREADS: one expert per thread)
  const bool on = tid < E && act[tid];
  const int cur = on ? d.dir[base + tid] : -1;
  int nact = 0, nmiss = 0;
  const int pos = sd_block_scan(on ? 1 : 0, scratch, &nact);
  const bool miss = on && cur < 0;
  const int mpos = sd_block_scan(miss ? 1 : 0, scratch, &nmiss);
  if (nact > S) {   // the batch cannot be resident at once: nothing changes
    if (tid == 0) {
      if (mode == 0)
        set_status(&d.h->status, DSV4_ENOMEM);
      else
        d.h->stats[6] += nmiss;   // a prediction too large to hold is skipped
    }
    return;
  }
  const long long clock0 = d.h->clock;
  const long long protect = d.h->protect;
  if (miss) {
    miss_e[mpos] = tid;
    miss_pos[mpos] = pos;
  }
  if (on && cur >= 0) {   // hit: move to the most-recently-used end
    inb[cur] = 1;
    d.stamp[cur] = clock0 + 1 + pos;
  }
  __syncthreads();
  int fetched = 0, evicted = 0;
  for (int j = 0; j < nmiss; ++j) {
    // smallest (stamp, slot) among the slots this batch does not hold
    unsigned long long best = ~0ull;
    for (int s = tid; s < S; s += SD_THREADS) {
      if (inb[s]) continue;
      const long long st = d.stamp[s];
      if (mode == 1 && st >= protect) continue;   // read by the demand batch in flight
      const unsigned long long k = ((unsigned long long)st << 20) | (unsigned long long)s;
      best = k < best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, best, o);
      best = y < best ? y : best;
    }
    __shared__ unsigned long long wbest[32];
    if ((tid & 31) == 0) wbest[tid >> 5] = best;
    __syncthreads();
    if (tid < 32) {
      unsigned long long b = wbest[tid];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long y = __shfl_xor_sync(0xffffffffu, b, o);
        b = y < b ? y : b;
      }
      if (tid == 0) {
        if (b == ~0ull) {
          bcast[0] = -1;   // no slot left that may be evicted (prefetch only)
        } else {
          const int v = (int)(b & 0xfffffull);
          const int e = miss_e[j];
          const int old = d.key[v];
          if (old >= 0) {
            d.dir[old] = -1;
            ++evicted;
          }
          d.key[v] = base + e;
          d.dir[base + e] = v;
          d.stamp[v] = clock0 + 1 + miss_pos[j];
          d.list[mode * d.max_list + fetched] = make_int2(v, base + e);
          ++fetched;
          inb[v] = 1;
          bcast[0] = v;
        }
      }
    }
    __syncthreads();
    if (bcast[0] < 0) break;
  }
  if (tid == 0) {
    d.h->clock = clock0 + nact;
    d.h->n_fetch[mode] = fetched;
    long long* st = d.h->stats;
    if (mode == 0) {
      d.h->protect = clock0 + 1;
      st[0] += nact - nmiss;
      st[1] += nmiss;
      st[2] += evicted;
    } else {
      st[3] += nact - nmiss;
      st[4] += fetched;
      st[5] += evicted;
      st[6] += nmiss - fetched;
    }
    st[7] += 1;
  }
}

// Copies the listed misses from the pinned host pool into their HBM slots:
// every CTA walks the list, each thread moves 4 x 16 bytes per round.
__global__ void __launch_bounds__(SD_FETCH_THREADS, 16)
    slotdir_fetch_kernel(SdPtrs d, int mode, uint8_t* __restrict__ arena, int64_t slot_bytes) {
  const int n = *reinterpret_cast<volatile const int*>(&d.h->n_fetch[mode]);
  const int64_t nv = slot_bytes / 16;
  const int64_t stride = (int64_t)gridDim.x * SD_FETCH_THREADS;
  for (int i = 0; i < n; ++i) {
    const int2 it = d.list[mode * d.max_list + i];
    const uint4* src = reinterpret_cast<const uint4*>(d.src[it.y]);
    uint4* dst = reinterpret_cast<uint4*>(arena + (int64_t)it.x * slot_bytes);
    if (src == nullptr) {   // never registered: leave the slot, the GEMM reports the expert
      if (blockIdx.x == 0 && threadIdx.x == 0) set_status(&d.h->status, DSV4_ENOTFOUND);
      continue;
    }
    int64_t v = (int64_t)blockIdx.x * SD_FETCH_THREADS + threadIdx.x;
    for (; v + 3 * stride < nv; v += 4 * stride) {
      uint4 r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) r[u] = __ldcs(src + v + u * stride);
#pragma unroll
      for (int u = 0; u < 4; ++u) dst[v + u * stride] = r[u];
    }
    for (; v < nv; v += stride) dst[v] = __ldcs(src + v);
  }
}

__global__ void slotdir_clear_kernel(SdPtrs d) {
  const int64_t n = (int64_t)d.L * d.E;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    d.dir[i] = -1;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < d.S; s += (int64_t)gridDim.x * blockDim.x) {
    d.key[s] = -1;
    d.stamp[s] = 0;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    d.h->clock = 0;
    d.h->protect = 1;
    d.h->n_fetch[0] = d.h->n_fetch[1] = 0;
  }
}

static int64_t al256(int64_t v) { return (v + 255) / 256 * 256; }

struct SdLayout {
  int64_t dir, key, stamp, src, list, bytes;
  int max_list;
};

static SdLayout sd_layout(int64_t L, int64_t E, int64_t S) {
  SdLayout l;
  l.max_list = (int)std::min<int64_t>(E, S);
  int64_t o = al256(sizeof(SdHeader));
  l.dir = o;
  o = al256(o + 4 * L * E);
  l.key = o;
  o = al256(o + 4 * S);
  l.stamp = o;
  o = al256(o + 8 * S);
  l.src = o;
  o = al256(o + 8 * L * E);
  l.list = o;
  o = al256(o + 8 * 2 * (int64_t)l.max_list);
  l.bytes = o;
  return l;
}

}  // namespace dsv4

using namespace dsv4;

struct dsv4_slotdir {
  int device = 0;
  int num_sms = 148;
  SdPtrs p{};
  SdLayout lay{};
  uint8_t* ws = nullptr;
  uint8_t* arena = nullptr;
  int64_t slot_bytes = 0;
};

extern "C" int64_t dsv4_slotdir_workspace_bytes(int32_t n_layers, int32_t n_experts, int64_t n_slots) {
  if (n_layers <= 0 || n_experts <= 0 || n_experts > 1024 || n_slots <= 0 || n_slots > DSV4_SLOTDIR_MAX_SLOTS)
    return DSV4_EINVAL;
  return sd_layout(n_layers, n_experts, n_slots).bytes;
}

extern "C" int dsv4_slotdir_create(dsv4_slotdir** out, int32_t n_layers, int32_t n_experts, uint8_t* slot_arena,
                                   int64_t n_slots, int64_t slot_bytes, void* workspace, int64_t workspace_bytes) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(out && slot_arena && workspace, "null pointer");
  DSV4_CHECK_ARG(n_layers > 0 && (int64_t)n_layers * n_experts < (1 << 26), "n_layers must be positive");
  DSV4_CHECK_ARG(n_experts > 0 && n_experts <= 1024, "n_experts must be in [1, 1024]");
  DSV4_CHECK_ARG(n_slots > 0 && n_slots <= DSV4_SLOTDIR_MAX_SLOTS, "n_slots must be in [1, DSV4_SLOTDIR_MAX_SLOTS]");
  DSV4_CHECK_ARG(slot_bytes > 0 && slot_bytes % 256 == 0, "slot_bytes must be a positive multiple of 256");
  DSV4_CHECK_ARG(((uintptr_t)slot_arena % 256) == 0 && ((uintptr_t)workspace % 256) == 0,
                 "slot arena and workspace must be 256-byte aligned");
  const SdLayout lay = sd_layout(n_layers, n_experts, n_slots);
  DSV4_CHECK_ARG(workspace_bytes >= lay.bytes, "workspace too small");
  std::unique_ptr<dsv4_slotdir> d(new dsv4_slotdir());
  if (int rc = bind_device_of(slot_arena, &d->device)) return rc;
  DSV4_CUDA_CHECK(cudaDeviceGetAttribute(&d->num_sms, cudaDevAttrMultiProcessorCount, d->device));
  uint8_t* ws = (uint8_t*)workspace;
  d->ws = ws;
  d->lay = lay;
  d->arena = slot_arena;
  d->slot_bytes = slot_bytes;
  d->p.h = reinterpret_cast<SdHeader*>(ws);
  d->p.dir = reinterpret_cast<int32_t*>(ws + lay.dir);
  d->p.key = reinterpret_cast<int32_t*>(ws + lay.key);
  d->p.stamp = reinterpret_cast<int64_t*>(ws + lay.stamp);
  d->p.src = reinterpret_cast<const uint8_t* const*>(ws + lay.src);
  d->p.list = reinterpret_cast<int2*>(ws + lay.list);
  d->p.max_list = lay.max_list;
  d->p.L = n_layers;
  d->p.E = n_experts;
  d->p.S = (int)n_slots;
  DSV4_CUDA_CHECK(cudaMemset(workspace, 0, (size_t)lay.bytes));
  slotdir_clear_kernel<<<64, 256>>>(d->p);
  DSV4_CUDA_CHECK(cudaGetLastError());
  // a small shared-memory need must not force a carve-out that keeps the
  // copies off the SMs that a grouped GEMM occupies
  DSV4_CUDA_CHECK(cudaFuncSetAttribute(slotdir_fetch_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  DSV4_CUDA_CHECK(cudaDeviceSynchronize());
  *out = d.release();
  DSV4_API_END
}

extern "C" int dsv4_slotdir_destroy(dsv4_slotdir* d) {
  delete d;
  return DSV4_OK;
}

extern "C" int dsv4_slotdir_set_sources(dsv4_slotdir* d, int64_t n, const int32_t* layers, const int32_t* experts,
                                        const void* const* host_slots) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(d, "null directory");
  DSV4_CHECK_ARG(n >= 0 && (n == 0 || (layers && experts && host_slots)), "null pointer");
  DSV4_CUDA_CHECK(cudaSetDevice(d->device));
  std::vector<const void*> dev(n);
  for (int64_t i = 0; i < n; ++i) {
    DSV4_CHECK_ARG(layers[i] >= 0 && layers[i] < d->p.L && experts[i] >= 0 && experts[i] < d->p.E,
                   "layer or expert outside the directory");
    // the GPU reads the slot straight from host memory: it must be page-locked
    // memory that this device can address, over its whole length
    const uint8_t* hp = static_cast<const uint8_t*>(host_slots[i]);
    DSV4_CHECK_ARG(hp != nullptr, "null host slot");
    cudaPointerAttributes a0{}, a1{};
    DSV4_CUDA_CHECK(cudaPointerGetAttributes(&a0, hp));
    DSV4_CUDA_CHECK(cudaPointerGetAttributes(&a1, hp + d->slot_bytes - 1));
    DSV4_CHECK_ARG(a0.type == cudaMemoryTypeHost && a1.type == cudaMemoryTypeHost && a0.devicePointer &&
                       a1.devicePointer &&
                       (const uint8_t*)a1.devicePointer - (const uint8_t*)a0.devicePointer == d->slot_bytes - 1,
                   "host slot is not page-locked memory mapped for this device");
    DSV4_CHECK_ARG(((uintptr_t)a0.devicePointer % 16) == 0, "host slot must be 16-byte aligned");
    dev[i] = a0.devicePointer;
  }
  // scatter on the host into a copy of the table, then one upload
  const int64_t LE = (int64_t)d->p.L * d->p.E;
  std::vector<const void*> table(LE);
  DSV4_CUDA_CHECK(cudaMemcpy(table.data(), d->p.src, LE * sizeof(void*), cudaMemcpyDeviceToHost));
  for (int64_t i = 0; i < n; ++i) table[(int64_t)layers[i] * d->p.E + experts[i]] = dev[i];
  DSV4_CUDA_CHECK(cudaMemcpy((void*)d->p.src, table.data(), LE * sizeof(void*), cudaMemcpyHostToDevice));
  DSV4_API_END
}

extern "C" int dsv4_slotdir_acquire(dsv4_slotdir* d, int32_t layer, const int32_t* indices, int64_t n_assign,
                                    int32_t mode, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(d, "null directory");
  DSV4_CHECK_ARG(layer >= 0 && layer < d->p.L, "layer outside the directory");
  DSV4_CHECK_ARG(mode == DSV4_SLOTDIR_DEMAND || mode == DSV4_SLOTDIR_PREFETCH, "unknown mode");
  DSV4_CHECK_ARG(n_assign >= 0 && n_assign < (1LL << 31), "bad assignment count");
  DSV4_CHECK_ARG(n_assign == 0 || indices, "null indices");
  DSV4_CUDA_CHECK(cudaSetDevice(d->device));
  cudaStream_t st = (cudaStream_t)stream;
  const size_t smem = (size_t)(36 + 2 * d->p.E) * 4 + d->p.E + d->p.S;
  slotdir_resolve_kernel<<<1, SD_THREADS, smem, st>>>(d->p, indices, (int)n_assign, layer, mode);
  DSV4_CUDA_CHECK(cudaGetLastError());
  // enough requests in flight to cover the PCIe round trip, few enough SMs
  // that a grouped GEMM running beside a prefetch keeps its pace
  const int grid = std::max(8, d->num_sms / 2);
  slotdir_fetch_kernel<<<grid, SD_FETCH_THREADS, 0, st>>>(d->p, mode, d->arena, d->slot_bytes);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}

extern "C" int dsv4_slotdir_table(dsv4_slotdir* d, int32_t layer, int32_t** slot_of_out) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(d && slot_of_out, "null pointer");
  DSV4_CHECK_ARG(layer >= 0 && layer < d->p.L, "layer outside the directory");
  *slot_of_out = d->p.dir + (int64_t)layer * d->p.E;
  DSV4_API_END
}

extern "C" int dsv4_slotdir_stats(dsv4_slotdir* d, int64_t* out8, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(d && out8, "null pointer");
  DSV4_CUDA_CHECK(cudaSetDevice(d->device));
  DSV4_CUDA_CHECK(cudaStreamSynchronize((cudaStream_t)stream));
  SdHeader h;
  DSV4_CUDA_CHECK(cudaMemcpy(&h, d->p.h, sizeof(h), cudaMemcpyDeviceToHost));
  for (int i = 0; i < SD_STAT_N; ++i) out8[i] = h.stats[i];
  DSV4_API_END
}

extern "C" int dsv4_slotdir_status(dsv4_slotdir* d, void* stream) {
  if (!d) return fail(DSV4_EINVAL, "dsv4_slotdir_status: null directory");
  cudaSetDevice(d->device);
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return fail(DSV4_ECUDA, std::string("dsv4_slotdir_status: ") + cudaGetErrorString(e));
  int v = 0;
  e = cudaMemcpy(&v, &d->p.h->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(DSV4_ECUDA, std::string("dsv4_slotdir_status: ") + cudaGetErrorString(e));
  if (v != 0) {
    cudaMemset(&d->p.h->status, 0, sizeof(int));
    return fail(v, "the slot directory reported this status");
  }
  return DSV4_OK;
}

extern "C" int dsv4_slotdir_snapshot(dsv4_slotdir* d, int32_t* slot_key_out, int64_t* stamp_out, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(d && slot_key_out && stamp_out, "null pointer");
  DSV4_CUDA_CHECK(cudaSetDevice(d->device));
  DSV4_CUDA_CHECK(cudaStreamSynchronize((cudaStream_t)stream));
  DSV4_CUDA_CHECK(cudaMemcpy(slot_key_out, d->p.key, 4 * (size_t)d->p.S, cudaMemcpyDeviceToHost));
  DSV4_CUDA_CHECK(cudaMemcpy(stamp_out, d->p.stamp, 8 * (size_t)d->p.S, cudaMemcpyDeviceToHost));
  DSV4_API_END
}

extern "C" int dsv4_slotdir_clear(dsv4_slotdir* d, void* stream) {
  DSV4_API_BEGIN
  DSV4_CHECK_ARG(d, "null directory");
  DSV4_CUDA_CHECK(cudaSetDevice(d->device));
  slotdir_clear_kernel<<<64, 256, 0, (cudaStream_t)stream>>>(d->p);
  DSV4_CUDA_CHECK(cudaGetLastError());
  DSV4_API_END
}
