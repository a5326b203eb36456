// Grouped expert GEMM on the sm_100a tensor cores (tcgen05, TMEM, TMA).
//
// Swap-AB formulation: the weight rows of one expert are the MMA M side
// (128 rows per MMA, two MMAs per 256-row weight pair), the tokens routed to
// that expert are the N side (up to 64 per tile), K runs along the hidden (or
// intermediate) dimension:
//     D[w_row, token] = sum_k W[w_row, k] * X[token, k]
// A = packed E2M1 weights straight from the expert slot, one contiguous
// 16 KiB block per (256-row pair, 128 of K) (TMA type 16U4_ALIGN16B expands
// them to the one-byte-per-element shared-memory form the f8f6f4 tensor-core
// path reads), with their E8M0 per-32 scales;
// B = E4M3 activations (bf16 profile) or E2M1 activations (a4w4), with E8M0
// per-32 scales.  bf16 profile: one tcgen05.mma.kind::mxf8f6f4.block_scale
// per 32 of K.  a4w4: both operands stay packed (two E2M1 per byte, TMA
// type UINT8 with a 64-byte swizzle) and one kind::mxf4.block_scale per 64
// of K, half the instructions and half the shared-memory bytes per product.
// The products equal those of the reference's dequantised operands exactly,
// so only accumulation order differs.
//
// Decode MMAs are tiny (N = 16 tokens).  A tcgen05 instruction costs the
// thread that issues it about 60-70 cycles whatever N is (up to 128), while
// the tensor pipe itself stays mostly idle, so one issuing thread per CTA
// caps the weight stream well below HBM speed.  Each 128-row half of the
// weight pair therefore has its own issuing thread, scale copies and
// accumulator; the two run in parallel on every stage.
//
// Warp roles (352 threads, one CTA per SM, persistent over tiles):
//   warp 0     producer: TMA for A and B, bulk copies of the A and B scale
//              atoms, one mbarrier per stage;
//   warp 1     TMEM owner, MMA issuer for weight rows 0-127 of the pair;
//   warps 2-9  epilogue: TMEM -> registers -> fused math -> global; two
//              warps per TMEM lane quarter, each taking half the columns;
//   warp 10    MMA issuer for weight rows 128-255 of the pair.
// Every role walks the same tile sequence and loads the next tile's
// metadata (chunk, slot) one tile ahead, so tile boundaries cost no
// dependent global-memory round trip.
// Gate/up runs the gate (w1) and up (w3) rows of the same 128 intermediate
// rows into two accumulators; down runs two consecutive 128-row tiles of w2.
// Accumulators are double-buffered in TMEM so the epilogue of one tile
// overlaps the main loop of the next.
#pragma once

#include "common.cuh"

namespace dsv4 {

constexpr int G_BM = 128;
constexpr int G_BN = 64;    // decode tile: up to 64 tokens of one expert
constexpr int G_BK = 128;
constexpr int G_EPI_WARPS = 8;
constexpr int G_MMA2_WARP = 2 + G_EPI_WARPS;   // MMA issuer of weight rows 128-255
constexpr int G_THREADS = 32 * (G_MMA2_WARP + 1);
constexpr uint32_t G_TMEM_COLS = 512;

enum : int { EPI_SWIGLU_FP8 = 0, EPI_SWIGLU_MXFP4 = 1, EPI_STORE_BF16 = 2 };

// BN = tokens per tile: 64 (decode) or 112 (prefill: 1.75x the work per MMA
// instruction, whose issue cost does not grow with N).  112 is the widest
// tile whose two double-buffered accumulators (2 x 2 x 112 = 448 columns)
// leave room in TMEM for the 16 scale-factor columns, so the epilogue of one
// tile still overlaps the main loop of the next.
// With packed operands (PACKED: the a4w4 profile) a stage is 22-25 KB
// instead of 42-48 KB, so the ring is 8 stages deep.
template <int NUM_A, int BN = G_BN, bool PACKED = false>
struct GemmCfg {
  static_assert(BN == 64 || BN == 112, "tile of 64 or 112 tokens");
  static constexpr int ROW_BYTES = PACKED ? G_BK / 2 : G_BK;   // shared-memory bytes per row of a k-tile
  static constexpr int A_BYTES = G_BM * ROW_BYTES;  // 8 KB packed, 16 KB with E2M1 expanded to 1 B / element
  static constexpr int B_BYTES = BN * ROW_BYTES;
  static constexpr int SF_BYTES = 512;
  static constexpr int STAGE_RAW = NUM_A * A_BYTES + B_BYTES + (NUM_A + 1) * SF_BYTES;
  static constexpr int STAGE_BYTES = (STAGE_RAW + 1023) / 1024 * 1024;
  static constexpr int STAGES = PACKED ? 8 : (BN == 64 ? 5 : 4);
  static constexpr int ACC_BUFS = 2;
  static constexpr uint32_t SF_COL = ACC_BUFS * NUM_A * BN;   // A and B scales of each issuer: 16 columns
  static constexpr int BAR_BYTES = 256;
  static constexpr int RED_BYTES = 4 * BN * 4;                   // per-column amax of each lane quarter
  static constexpr int XPOSE_STRIDE = 36;                         // bytes per column row (32 + 4: no bank conflicts)
  static constexpr int XPOSE_BYTES = G_EPI_WARPS * 32 * XPOSE_STRIDE;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + RED_BYTES + XPOSE_BYTES + 1024;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(SF_COL + 16 <= G_TMEM_COLS, "scale columns above the accumulators");
};

struct GemmParams {
  const uint8_t* arena;      // slot arena base
  int64_t slot_bytes;
  int64_t sfa_off;           // byte offset of the A scale atoms inside a slot
  int k_tiles;               // K / 128
  int a_row_tiles;           // tiles per chunk = 256-row weight pairs of the matrix
  int out_tile_cols;         // output columns per tile (128: gate/up pair, 256: down pair)
  const uint8_t* b_sf;       // activation scale atoms: 512 B per (k-tile, BN-row block)
  int64_t rb_cap;            // BN-row blocks per k-tile in b_sf / out_sf
  const int4* chunks;        // {expert, row0, nrows, 1 when the expert has several chunks}
  const int* n_chunks;
  const int* slot_of;        // expert -> slot
  int n_slots;               // slots in the arena; other values are rejected
  const float* sorted_w;     // route weight per sorted row (gate/up epilogue)
  uint8_t* out_q;            // gate/up: next activation (E4M3 [p_cap][I] or E2M1 [p_cap][I/2])
  uint8_t* out_sf;           // gate/up: its scale atoms, same layout as b_sf
  uint16_t* out_bf16;        // down: [p_cap][H] bf16
  int out_ld;                // elements per output row (I or H)
  float swiglu_limit;
  int* status;
  // the shared expert (bf16 profile): chunks of expert `shared_expert` read
  // E4M3 weights from the FP8 slot at `shared_slot` (tensor map tmAsh)
  int shared_expert;         // -1: none
  const uint8_t* shared_slot;
  int64_t shared_sfa_off;    // byte offset of its A scale atoms
  // down GEMM, scatter mode (expert parallelism): the output row of sorted
  // row r goes to assign_dst[sorted_flat[r]] (any memory this GPU can store
  // to, a peer's buffer over NVLink included; null: dropped) instead of
  // out_bf16, so the return of the rows overlaps the GEMM tile by tile
  const int32_t* sorted_flat;
  uint16_t* const* assign_dst;
  // fused gate/up -> down launch: the gate/up epilogue of chunk c counts its
  // finished tiles in chunk_done[c]; a down tile of chunk c loads its
  // activations (the h rows) once the count reaches the gate/up tiles per
  // chunk.  Zeroed by the align of the same pass.
  int* chunk_done;
};

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// SiLU with the fast exponential and division intrinsics: relative error
// ~1e-6, far inside the layer's tolerance; v -> -inf gives -0.
__device__ __forceinline__ float silu_f(float v) { return __fdividef(v, 1.0f + __expf(-v)); }


struct TileInfo {
  int slot;   // < 0: skip (expert not resident)
  int row0;   // first row of the 64-row chunk
  int nrows;  // valid rows in the chunk
  int mt;     // 128-row tile of the weight matrix
  bool sh;    // the shared expert (FP8 weights)
  bool reuse; // the expert's weights feed several chunks
  int ph;     // 0: first GEMM of the launch (gate/up, or the only one); 1: down of a fused launch
  int c;      // chunk
};

__device__ __forceinline__ TileInfo load_tile(const GemmParams& p, int t, int n_tiles) {
  TileInfo ti{-1, 0, 0, 0, false, false, 0, 0};
  if (t < n_tiles) {
    const int c = t / p.a_row_tiles;
    ti.c = c;
    const int4 ch = p.chunks[c];
    if (ch.x == p.shared_expert) {
      ti.sh = true;
      ti.slot = 0;
    } else {
      const int s = p.slot_of[ch.x];
      ti.slot = (s >= 0 && s < p.n_slots) ? s : -1;
    }
    ti.row0 = ch.y;
    ti.nrows = ch.z;
    ti.reuse = ch.w != 0;
    ti.mt = t - c * p.a_row_tiles;
  }
  return ti;
}

// Tile t of a launch: the first GEMM's tiles [0, n0), then (fused launch)
// the down GEMM's [n0, n_all).
__device__ __forceinline__ TileInfo load_tile2(const GemmParams& p, const GemmParams& pd, int t, int n0, int n_all) {
  if (t < n0) return load_tile(p, t, n0);
  TileInfo ti = load_tile(pd, t - n0, n_all - n0);
  ti.ph = 1;
  return ti;
}

// Activation rows loaded per tile: the chunk's valid rows rounded up to 16,
// 32, 64 or the tile width (decode chunks are mostly short); also the MMA N.
// Column maxima of |h[n]| over a warp's 32 lanes, all 32 columns at once:
// five butterfly rounds each halve the columns a lane keeps (16, 8, 4, 2,
// 1) while exchanging the other half with its partner, so 31 shuffles
// leave lane L with column L's maximum.  The maximum is taken on the bit
// patterns (non-negative floats order like unsigned integers).  v is
// scratch (overwritten).
__device__ __forceinline__ float column_amax_transposed(const float* h, float* v, int lane) {
  uint32_t* u = reinterpret_cast<uint32_t*>(v);
#pragma unroll
  for (int n = 0; n < 32; ++n) u[n] = __float_as_uint(fabsf(h[n]));
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int j = 0; j < s; ++j) {
      const uint32_t send = upper ? u[j] : u[j + s];
      const uint32_t keep = upper ? u[j + s] : u[j];
      u[j] = max(keep, __shfl_xor_sync(0xffffffffu, send, s));
    }
  }
  return __uint_as_float(u[0]);
}

template <int BN>
__device__ __forceinline__ int b_rows_for(int nrows) {
  return nrows <= 16 ? 16 : (nrows <= 32 ? 32 : (nrows <= 64 ? 64 : BN));
}

// The tensor maps of one GEMM: weights (A), activations (B) by rows per
// tile, and the shared expert's FP8 weights.
struct GemmMaps {
  CUtensorMap A, B16, B32, B64, Bwide, Ash;
};

// FUSED: one launch runs the gate/up GEMM (epilogue EPI, params p, maps m0)
// and then the down GEMM (bf16 rows, params pd, maps m1) over the same
// chunks; each CTA takes its gate/up tiles first, so a down tile only ever
// waits for gate/up tiles, which never wait: no cycle, whatever the CTAs'
// residency.  Otherwise one GEMM (p, m0; m1 and pd unused).
template <int NUM_A, bool B_FP4, int EPI, int BN, bool FUSED>
__global__ void __launch_bounds__(G_THREADS, 1)
    moe_gemm_kernel(const __grid_constant__ GemmMaps m0, const __grid_constant__ GemmParams p,
                    const __grid_constant__ GemmMaps m1, const __grid_constant__ GemmParams pd) {
  static_assert(NUM_A == 2, "operand tiles come in 256-row pairs");
  static_assert(!FUSED || EPI != EPI_STORE_BF16, "a fused launch starts with the gate/up GEMM");
  using C = GemmCfg<NUM_A, BN, B_FP4>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::STAGES;
  uint64_t* accfull = bars + 2 * C::STAGES;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  int* epi_fail = reinterpret_cast<int*>(tmem_holder + 1);
  float* red = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES + C::BAR_BYTES);  // [4][BN]
  uint8_t* xpose_all = smem + C::STAGES * C::STAGE_BYTES + C::BAR_BYTES + C::RED_BYTES;  // [8 warps][32][36]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 2);   // one commit from each MMA issuer
    }
    for (int b = 0; b < C::ACC_BUFS; ++b) {
      mbar_init(&accfull[b], 2);
      mbar_init(&accempty[b], G_EPI_WARPS);
    }
    mbar_init(drain, 2);
    *epi_fail = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
#pragma unroll
    for (int g = 0; g < (FUSED ? 2 : 1); ++g) {
      const GemmMaps& m = g ? m1 : m0;
      prefetch_tensormap(&m.A);
      prefetch_tensormap(&m.B16);
      prefetch_tensormap(&m.B32);
      prefetch_tensormap(&m.B64);
      if (BN > 64) prefetch_tensormap(&m.Bwide);
      if (!B_FP4 && p.shared_expert >= 0) prefetch_tensormap(&m.Ash);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, G_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // The align outputs (chunks, counts) are two kernels back and complete;
  // the activations come from the immediate predecessor: wait for it, then
  // let the next kernel start its prologue.
  const int n_chunks_all = *p.n_chunks;
  const int n0 = n_chunks_all * p.a_row_tiles;                            // first GEMM's tiles
  const int n_tiles = FUSED ? n0 + n_chunks_all * pd.a_row_tiles : n0;   // all tiles of the launch
  const int step = gridDim.x;
  constexpr uint32_t a_tx = 2 * G_BM * G_BK / 2;      // packed bytes of the 256-row A box
  constexpr uint32_t a_tx_sh = 2 * G_BM * G_BK;       // the shared expert's E4M3 box
  // parameters and maps of a tile's GEMM
  auto P = [&](const TileInfo& ti) -> const GemmParams& { return (FUSED && ti.ph) ? pd : p; };
  auto M = [&](const TileInfo& ti) -> const GemmMaps& { return (FUSED && ti.ph) ? m1 : m0; };
  auto tile = [&](int t) -> TileInfo { return FUSED ? load_tile2(p, pd, t, n0, n_tiles) : load_tile(p, t, n_tiles); };
  // the shared expert exists only with FP8 activations (the bf16 profile)
  auto a_map = [&](const TileInfo& ti) -> const CUtensorMap* { return (!B_FP4 && ti.sh) ? &M(ti).Ash : &M(ti).A; };
  auto a_bytes = [&](const TileInfo& ti) -> uint32_t { return (!B_FP4 && ti.sh) ? a_tx_sh : a_tx; };
  auto a_sf = [&](const TileInfo& ti) -> const uint8_t* {
    const GemmParams& q = P(ti);
    return (!B_FP4 && ti.sh) ? q.shared_slot + q.shared_sfa_off
                             : q.arena + (int64_t)ti.slot * q.slot_bytes + q.sfa_off;
  };
  // The weights do not depend on the predecessor kernel: the producer puts
  // the first tile's first ring stages of weights and weight scales in
  // flight before it waits; that tile's activations follow after the wait.
  int pre = 0;
  if (warp == 0 && lane == 0) {
    const TileInfo first = tile(blockIdx.x);
    if (first.slot >= 0) {
      const uint64_t pol_w = first.reuse ? policy_evict_normal() : policy_evict_first();
      const uint8_t* sf_base = a_sf(first);
      const int k_tiles = P(first).k_tiles;
      const uint32_t b_tx = (uint32_t)b_rows_for<BN>(first.nrows) * (B_FP4 ? G_BK / 2 : G_BK);
      pre = k_tiles < C::STAGES ? k_tiles : C::STAGES;
      for (int kt = 0; kt < pre; ++kt) {   // stage kt, first phase: the ring is empty
        uint8_t* st = smem + kt * C::STAGE_BYTES;
        mbar_expect_tx(&full[kt], a_bytes(first) + 2 * C::SF_BYTES + b_tx + C::SF_BYTES);
        tma_load_5d(st, a_map(first), &full[kt], 0, 0, kt, first.mt, first.slot, pol_w);
        bulk_load(st + NUM_A * C::A_BYTES + C::B_BYTES,
                  sf_base + ((int64_t)first.mt * k_tiles + kt) * 2 * C::SF_BYTES, 2 * C::SF_BYTES, &full[kt], pol_w);
      }
    }
  }
  griddep_wait();
  griddep_launch();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      // weights stream through L2 once (evict first), except an expert's
      // whose weight tiles feed several chunks: the other chunks' tiles run
      // at about the same time on other CTAs and find them in L2
      const uint64_t pol_once = policy_evict_first(), pol_reuse = policy_evict_normal();
      const uint64_t pol_x = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      TileInfo cur = tile(blockIdx.x);
      for (int t = blockIdx.x; t < n_tiles && ok; t += step) {
        const TileInfo nxt = tile(t + step);
        if (cur.slot < 0) {
          set_status(p.status, DSV4_ENOTFOUND);
          cur = nxt;
          continue;
        }
        const GemmParams& q = P(cur);
        const GemmMaps& m = M(cur);
        const int k_tiles = q.k_tiles;
        const uint8_t* sf_base = a_sf(cur);
        const CUtensorMap* mA = a_map(cur);
        const uint32_t atx = a_bytes(cur);
        const uint8_t* sfb_base = q.b_sf + (int64_t)(cur.row0 / BN) * C::SF_BYTES;
        const int nb = b_rows_for<BN>(cur.nrows);
        const CUtensorMap* mB = nb == 16 ? &m.B16 : (nb == 32 ? &m.B32 : (nb == 64 ? &m.B64 : &m.Bwide));
        int early = t == (int)blockIdx.x ? pre : 0;   // stages whose weights are already in flight
        const uint64_t pol_w = cur.reuse ? pol_reuse : pol_once;
        if (FUSED && cur.ph) {
          // the h rows of this chunk come from the gate/up tiles of other
          // CTAs: until all of them have stored theirs, fill the ring
          // stages as they free up with this tile's weights (which do not
          // depend on them), then wait
          if (ld_acquire(p.chunk_done + cur.c) < p.a_row_tiles) {
            const int npre = k_tiles < C::STAGES ? k_tiles : C::STAGES;
            const uint32_t b_tx = (uint32_t)nb * (B_FP4 ? G_BK / 2 : G_BK);
            int s = stage;
            uint32_t ph = phase;
            for (int kt = 0; kt < npre; ++kt) {
              if (kt >= early) {
                if (!mbar_wait(&empty[s], ph ^ 1u, p.status)) {
                  ok = false;
                  break;
                }
                uint8_t* st = smem + s * C::STAGE_BYTES;
                mbar_expect_tx(&full[s], atx + 2 * C::SF_BYTES + b_tx + C::SF_BYTES);
                tma_load_5d(st, mA, &full[s], 0, 0, kt, cur.mt, cur.slot, pol_w);
                bulk_load(st + NUM_A * C::A_BYTES + C::B_BYTES,
                          sf_base + ((int64_t)cur.mt * k_tiles + kt) * 2 * C::SF_BYTES, 2 * C::SF_BYTES, &full[s],
                          pol_w);
              }
              if (++s == C::STAGES) {
                s = 0;
                ph ^= 1u;
              }
            }
            if (!ok) break;
            early = early > npre ? early : npre;
          }
          if (!wait_count_geq(p.chunk_done + cur.c, p.a_row_tiles, p.status)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();   // the TMA reads below see those stores
        }
        for (int kt = 0; kt < k_tiles; ++kt) {
          uint8_t* st = smem + stage * C::STAGE_BYTES;
          uint8_t* sA = st;                        // 256 rows: A0 then A1
          uint8_t* sB = st + NUM_A * C::A_BYTES;
          uint8_t* sSFA = sB + C::B_BYTES;         // 2 x 512 B
          uint8_t* sSFB = sSFA + NUM_A * C::SF_BYTES;
          if (kt >= early) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) {
              ok = false;
              break;
            }
            const uint32_t b_tx = (uint32_t)nb * (B_FP4 ? G_BK / 2 : G_BK);
            mbar_expect_tx(&full[stage], atx + 2 * C::SF_BYTES + b_tx + C::SF_BYTES);
            tma_load_5d(sA, mA, &full[stage], 0, 0, kt, cur.mt, cur.slot, pol_w);
            bulk_load(sSFA, sf_base + ((int64_t)cur.mt * k_tiles + kt) * 2 * C::SF_BYTES, 2 * C::SF_BYTES,
                      &full[stage], pol_w);
          }
          tma_load_2d(sB, mB, &full[stage], kt * C::ROW_BYTES, cur.row0, pol_x);
          // B scales: the atom of (k-tile kt, this 64-row chunk), already in tensor-core order
          bulk_load(sSFB, sfb_base + (int64_t)kt * q.rb_cap * C::SF_BYTES, C::SF_BYTES, &full[stage], pol_x);
          mbar_arrive(&full[stage]);
          ++issued;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        cur = nxt;
      }
      if (!ok) {
        // let copies already in flight land before the CTA can exit
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < C::STAGES && i < issued; ++i) {
          if (--s < 0) {
            s = C::STAGES - 1;
            ph ^= 1u;
          }
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[s], ph) && globaltimer_ns() - t0 < DSV4_WAIT_NS) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1 || warp == G_MMA2_WARP) {
    // ----------------------------------------------------------- MMA issuers
    if (lane == 0) {
      const int half = warp == 1 ? 0 : 1;   // weight rows 0-127 or 128-255 of the pair
      int stage = 0;
      uint32_t phase = 0;
      int abuf = 0;
      uint32_t aphase = 0;
      bool ok = true;
      // each issuer copies the scales it reads into its own TMEM columns:
      // tcgen05 operations of different threads are not ordered
      const uint32_t sfa = tmem + C::SF_COL + 8 * half, sfb = tmem + C::SF_COL + 8 * half + 4;
      TileInfo cur = tile(blockIdx.x);
      for (int t = blockIdx.x; t < n_tiles && ok; t += step) {
        const TileInfo nxt = tile(t + step);
        if (cur.slot < 0) {
          cur = nxt;
          continue;
        }
        const int nb = b_rows_for<BN>(cur.nrows);
        const bool a_e4m3 = !B_FP4 && cur.sh;
        const int k_tiles = P(cur).k_tiles;
        cur = nxt;
        if (!mbar_wait(&accempty[abuf], aphase ^ 1u, p.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)abuf * (NUM_A * BN) + (uint32_t)half * BN;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&full[stage], phase, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* st = smem + stage * C::STAGE_BYTES;
          const uint32_t aA = smem_u32(st + half * C::A_BYTES);
          const uint32_t aB = smem_u32(st + NUM_A * C::A_BYTES);
          const uint32_t aSFA = aB + C::B_BYTES + half * C::SF_BYTES;
          const uint32_t aSFB = aB + C::B_BYTES + NUM_A * C::SF_BYTES;
          tc_cp_sf(sfa, desc_sf(aSFA));
          tc_cp_sf(sfb, desc_sf(aSFB));
          if constexpr (B_FP4) {
            const uint64_t dA = desc_sw64(aA), dB = desc_sw64(aB);
#pragma unroll
            for (int kb = 0; kb < G_BK / 64; ++kb) {
              // scale bytes 2kb, 2kb+1 of each row's 32-bit column: sf_id 0 or 2
              const uint32_t idesc = idesc_mxf4(nb, 2u * kb);
              const uint32_t sel = (2u * kb) << 30;
              const uint32_t acc = (kt | kb) != 0 ? 1u : 0u;
              // +32 bytes (64 packed elements) of K per step inside the 64-byte swizzle row
              tc_mma_mxf4(d, dA + 2u * kb, dB + 2u * kb, idesc, acc, sfa | sel, sfb | sel);
            }
          } else {
            const uint64_t dA = desc_sw128(aA), dB = desc_sw128(aB);
#pragma unroll
            for (int kb = 0; kb < G_BK / 32; ++kb) {
              const uint32_t idesc = idesc_mxf8f6f4(nb, false, (uint32_t)kb, a_e4m3);
              const uint32_t sel = (uint32_t)kb << 30;
              const uint32_t acc = (kt | kb) != 0 ? 1u : 0u;
              // +32 bytes of K per step inside the 128-byte swizzle row
              tc_mma_mxf8f6f4(d, dA + 2u * kb, dB + 2u * kb, idesc, acc, sfa | sel, sfb | sel);
            }
          }
          tc_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&accfull[abuf]);
        if (++abuf == C::ACC_BUFS) {
          abuf = 0;
          aphase ^= 1u;
        }
      }
      // drain: every tcgen05 operation issued above has completed after this
      tc_commit(drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < DSV4_WAIT_NS) {
      }
    }
    __syncwarp();
  } else if (warp < 2 + G_EPI_WARPS) {
    // ------------------------------------------------------------ epilogue
    constexpr int HALF = BN / 2;       // columns per epilogue warp
    constexpr int SUB = 32;            // columns per pass (registers)
    const int q = warp & 3;            // TMEM lane quarter of this warp
    const int half = (warp - 2) >> 2;  // which half of the BN columns
    const int i = q * 32 + lane;       // row inside the 128-row tile
    const int c0 = half * HALF;        // first column of this warp
    uint8_t* xpose = xpose_all + (warp - 2) * 32 * C::XPOSE_STRIDE;   // [column][row] bytes of this warp
    int abuf = 0;
    uint32_t aphase = 0;
    float w[SUB];
    // route weights of 32 rows starting at cs (row0 + cs is a multiple of 8;
    // the sorted-weight buffer has a tile of slack after its last group)
    auto load_w = [&](int row0, int cs) {
      if constexpr (EPI != EPI_STORE_BF16) {
        const float4* wp = reinterpret_cast<const float4*>(p.sorted_w + row0 + cs);
#pragma unroll
        for (int j = 0; j < SUB / 4; ++j) {
          const float4 v = wp[j];
          w[4 * j] = v.x;
          w[4 * j + 1] = v.y;
          w[4 * j + 2] = v.z;
          w[4 * j + 3] = v.w;
        }
      }
    };
    TileInfo cur = tile(blockIdx.x);
    for (int t = blockIdx.x; t < n_tiles; t += step) {
      const TileInfo nxt = tile(t + step);
      if (cur.slot < 0) {
        cur = nxt;
        continue;
      }
      const int row0 = cur.row0, nrows = cur.nrows, mt = cur.mt, chunk = cur.c;
      // bf16 rows out: the down GEMM (alone, or the second half of a fused launch)
      const bool store_tile = EPI == EPI_STORE_BF16 || (FUSED && cur.ph);
      const GemmParams& gq = P(cur);
      cur = nxt;
      if (!store_tile) load_w(row0, c0);
      // all epilogue warps take the same decision: a failed wait in any of
      // them ends the loop for all (the named barriers below need all 8)
      if (!mbar_wait(&accfull[abuf], aphase, p.status) && lane == 0) atomicOr(epi_fail, 1);
      named_bar_sync(1, 32 * G_EPI_WARPS);
      if (*reinterpret_cast<volatile int*>(epi_fail) != 0) break;
      tc_fence_after();
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)abuf * (NUM_A * BN) + c0;
      constexpr int NPASS = (HALF + SUB - 1) / SUB;
#pragma unroll
      for (int sub = 0; sub < NPASS; ++sub) {
        const int cs = c0 + sub * SUB;   // first column of this pass
        const int width = HALF - sub * SUB < SUB ? HALF - sub * SUB : SUB;   // 32, or 24 (BN = 112)
        if (sub > 0 && !store_tile) load_w(row0, cs);
        float acc0[SUB];
        float acc1[NUM_A == 2 ? SUB : 1];
        (void)acc1;
        tmem_ld16(tbase + sub * SUB, acc0);
        if (width == 32)
          tmem_ld16(tbase + sub * SUB + 16, acc0 + 16);
        else
          tmem_ld8(tbase + sub * SUB + 16, acc0 + 16);
        if constexpr (NUM_A == 2) {
          tmem_ld16(tbase + BN + sub * SUB, acc1);
          if (width == 32)
            tmem_ld16(tbase + BN + sub * SUB + 16, acc1 + 16);
          else
            tmem_ld8(tbase + BN + sub * SUB + 16, acc1 + 16);
        }
        tc_wait_ld();
        if (width < SUB) {   // columns past the pass width were not loaded
#pragma unroll
          for (int n = 0; n < SUB; ++n)
            if (n >= width) acc0[n] = acc1[n] = 0.f;
        }
        if (sub == NPASS - 1) {   // this tile's accumulators are read out
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&accempty[abuf]);
        }

        if (store_tile) {
          // rows 0..127 of the pair -> acc0, rows 128..255 -> acc1
          if (gq.assign_dst) {
            // scatter: lane L fetches the destination of column cs+L, then
            // every column's row is stored where it belongs (plain stores,
            // 64 contiguous bytes per warp and column)
            uint16_t* mine = nullptr;
            if (lane < width && cs + lane < nrows) {
              const int a = gq.sorted_flat[row0 + cs + lane];
              mine = a >= 0 ? gq.assign_dst[a] : nullptr;
            }
            const unsigned long long mv = reinterpret_cast<unsigned long long>(mine);
#pragma unroll
            for (int n = 0; n < SUB; ++n) {
              const unsigned long long b = __shfl_sync(0xffffffffu, mv, n);
              if (b) {
                uint16_t* dst = reinterpret_cast<uint16_t*>(b) + mt * gq.out_tile_cols + i;
                dst[0] = bf16_bits(acc0[n]);
                if constexpr (NUM_A == 2) dst[G_BM] = bf16_bits(acc1[n]);
              }
            }
          } else {
            uint16_t* dst = gq.out_bf16 + (int64_t)(row0 + cs) * gq.out_ld + mt * gq.out_tile_cols + i;
#pragma unroll
            for (int n = 0; n < SUB; ++n)
              if (n < width && cs + n < nrows) dst[(int64_t)n * gq.out_ld] = bf16_bits(acc0[n]);
            if constexpr (NUM_A == 2) {
              uint16_t* dst1 = dst + G_BM;
#pragma unroll
              for (int n = 0; n < SUB; ++n)
                if (n < width && cs + n < nrows) dst1[(int64_t)n * gq.out_ld] = bf16_bits(acc1[n]);
            }
          }
        } else if constexpr (EPI != EPI_STORE_BF16) {
          // gate = bf16(w1 x), up = bf16(w3 x); clamp; h = silu(gate)*up*w_route;
          // bf16(h) is the input of the activation re-quantisation.
          const float lim = p.swiglu_limit;
#pragma unroll
          for (int n = 0; n < SUB; ++n) {
            float g = bf16r(acc0[n]);
            float u = bf16r(acc1[n]);
            if (lim > 0.f) {
              u = fminf(fmaxf(u, -lim), lim);
              g = fminf(g, lim);
            }
            acc0[n] = bf16r(silu_f(g) * u * w[n]);
          }
          if constexpr (EPI == EPI_SWIGLU_FP8) {
            // per-token amax over the 128 rows of this tile = one 128-block of I:
            // redux over the warp's 32 rows, then across the 4 lane quarters
            // lane L: max |h| of column cs+L over the warp's 32 rows
            const float mine = column_amax_transposed(acc0, acc1, lane);
            if (lane < width) red[q * BN + cs + lane] = mine;
            named_bar_sync(1, 32 * G_EPI_WARPS);
            const float amax_l = lane < width ? fmaxf(fmaxf(red[cs + lane], red[BN + cs + lane]),
                                                      fmaxf(red[2 * BN + cs + lane], red[3 * BN + cs + lane]))
                                              : 0.f;
            const int e_l = fp8_scale_exp(amax_l);
            // E4M3 bytes into [column][row], then lane L stores column L's 32 bytes
#pragma unroll
            for (int n = 0; n < SUB; ++n) {
              const int e = __shfl_sync(0xffffffffu, e_l, n);
              const float v = fminf(fmaxf(acc0[n] * pow2i(-e), -448.f), 448.f);
              xpose[n * C::XPOSE_STRIDE + lane] = (uint8_t)e4m3_byte(v);
            }
            __syncwarp();
            if (lane < width && cs + lane < nrows) {
              const uint32_t* src = reinterpret_cast<const uint32_t*>(xpose + lane * C::XPOSE_STRIDE);
              uint4* dst = reinterpret_cast<uint4*>(p.out_q + (int64_t)(row0 + cs + lane) * p.out_ld + mt * G_BM + q * 32);
              dst[0] = make_uint4(src[0], src[1], src[2], src[3]);
              dst[1] = make_uint4(src[4], src[5], src[6], src[7]);
            }
            __syncwarp();
            if (q == 0 && lane < width && cs + lane < nrows) {
              const int n = cs + lane;
              *reinterpret_cast<uint32_t*>(p.out_sf + ((int64_t)mt * p.rb_cap + row0 / BN) * 512 + (n & 31) * 16 +
                                           (n >> 5) * 4) = (uint32_t)(e_l + 127) * 0x01010101u;
            }
            named_bar_sync(1, 32 * G_EPI_WARPS);
          } else {
            // per-token amax over the 32 rows of this warp = one 32-block of I;
            // lane L holds column cs+L's
            const int e_l = mx_scale_exp(column_amax_transposed(acc0, acc1, lane));
            const bool col_ok = lane < width && cs + lane < nrows;
            if (col_ok) {
              const int cn = cs + lane;
              p.out_sf[((int64_t)mt * p.rb_cap + row0 / BN) * 512 + q + (cn & 31) * 16 + (cn >> 5) * 4] =
                  (uint8_t)(e_l + 127);
            }
            // E2M1 codes into [column][row], then lane L packs column L's 32
            // rows two per byte (even row in the low nibble) and stores 16 B
#pragma unroll
            for (int n = 0; n < SUB; ++n) {
              const int e = __shfl_sync(0xffffffffu, e_l, n);
              xpose[n * C::XPOSE_STRIDE + lane] = (uint8_t)e2m1_code(acc0[n] * pow2_any(-e));
            }
            __syncwarp();
            if (col_ok) {
              const uint32_t* src = reinterpret_cast<const uint32_t*>(xpose + lane * C::XPOSE_STRIDE);
              uint32_t o[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const uint32_t t0 = src[2 * k] | (src[2 * k] >> 4), t1 = src[2 * k + 1] | (src[2 * k + 1] >> 4);
                o[k] = __byte_perm(t0, t1, 0x6420);
              }
              *reinterpret_cast<uint4*>(p.out_q + (int64_t)(row0 + cs + lane) * (p.out_ld / 2) + (mt * G_BM + q * 32) / 2) =
                  make_uint4(o[0], o[1], o[2], o[3]);
            }
            __syncwarp();
          }
        }
      }
      if (FUSED && !store_tile) {
        // this gate/up tile's h columns and scales are stored: count it for
        // the down tiles of its chunk (stores, fence, barrier, then one add)
        __threadfence();
        named_bar_sync(1, 32 * G_EPI_WARPS);
        if (warp == 2 && lane == 0) red_release_add(p.chunk_done + chunk, 1);
      }
      if (++abuf == C::ACC_BUFS) {
        abuf = 0;
        aphase ^= 1u;
      }
    }
  }

  // scatter mode: the rows stored to other GPUs are visible system-wide
  // before this grid completes and a later kernel publishes them
  if ((EPI == EPI_STORE_BF16 && p.assign_dst) || (FUSED && pd.assign_dst)) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, G_TMEM_COLS);
  }
}

}  // namespace dsv4
