// Grouped expert GEMM on the sm_100a tensor cores (tcgen05, TMEM, TMA).
//
// Swap-AB formulation: the weight rows of one expert are the MMA M side
// (128 rows per tile), the tokens routed to that expert are the N side
// (64 per tile), K runs along the hidden (or intermediate) dimension:
//     D[w_row, token] = sum_k W[w_row, k] * X[token, k]
// A = packed E2M1 weights straight from the expert slot (TMA type
// 16U4_ALIGN16B expands them to the one-byte-per-element shared-memory form
// the f8f6f4 tensor-core path reads), with their E8M0 per-32 scales;
// B = E4M3 activations (bf16 profile) or E2M1 activations (a4w4), with E8M0
// per-32 scales.  One tcgen05.mma.kind::mxf8f6f4.block_scale per 32 of K.
// The products equal those of bf16(dequant(W)) x bf16(fp8_roundtrip(X)) of
// the reference exactly, so only accumulation order differs.
//
// Warp roles (192 threads, one CTA per SM, persistent over tiles):
//   warp 0     producer: TMA for A and B, bulk copy of A scales, gather of
//              B scales into the tensor-core order, one mbarrier per stage;
//   warp 1     TMEM owner and MMA issuer (one thread);
//   warps 2-5  epilogue: TMEM -> registers -> fused math -> global.
// NUM_A = 2 runs the gate (w1) and up (w3) projections of the same 128
// intermediate rows into two accumulators; NUM_A = 1 runs the down
// projection.  Accumulators are double-buffered in TMEM so the epilogue of
// one tile overlaps the main loop of the next.
#pragma once

#include "common.cuh"

namespace dsv4 {

constexpr int G_BM = 128;
constexpr int G_BN = 64;
constexpr int G_BK = 128;
constexpr int G_THREADS = 192;
constexpr uint32_t G_TMEM_COLS = 512;
constexpr uint32_t G_SF_COL = 256;   // TMEM columns 256..267 hold scale factors

enum : int { EPI_SWIGLU_FP8 = 0, EPI_SWIGLU_MXFP4 = 1, EPI_STORE_BF16 = 2 };

template <int NUM_A>
struct GemmCfg {
  static constexpr int A_BYTES = G_BM * G_BK;  // 16 KB (E2M1 expanded to 1 B / element)
  static constexpr int B_BYTES = G_BN * G_BK;  // 8 KB
  static constexpr int SF_BYTES = 512;
  static constexpr int STAGE_RAW = NUM_A * A_BYTES + B_BYTES + (NUM_A + 1) * SF_BYTES;
  static constexpr int STAGE_BYTES = (STAGE_RAW + 1023) / 1024 * 1024;
  static constexpr int STAGES = NUM_A == 2 ? 5 : 8;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + BAR_BYTES + 4 * G_BN * 4 + 1024;
};

struct GemmParams {
  const uint8_t* arena;      // slot arena base
  int64_t slot_bytes;
  int64_t sfa_off;           // byte offset of the A scale atoms inside a slot
  int k_tiles;               // K / 128
  int a_row_tiles;           // tiles of 128 rows per A matrix (= tiles per chunk)
  int a1_row_offset;         // row offset of the second A matrix (w3) in the map
  const uint32_t* b_sf;      // activation scales [k_tiles][p_cap], 4 bytes per row
  int64_t p_cap;
  const int4* chunks;        // {expert, row0, nrows, 0}
  const int* n_chunks;
  const int* slot_of;        // expert -> slot
  int n_slots;               // slots in the arena; other values are rejected
  const float* sorted_w;     // route weight per sorted row (gate/up epilogue)
  uint8_t* out_q;            // gate/up: next activation (E4M3 [p_cap][I] or E2M1 [p_cap][I/2])
  uint32_t* out_sf;          // gate/up: its scales [I/128][p_cap]
  uint16_t* out_bf16;        // down: [p_cap][H] bf16
  int out_ld;                // elements per output row (I or H)
  float swiglu_limit;
  int* status;
};

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

template <int NUM_A, bool B_FP4, int EPI>
__global__ void __launch_bounds__(G_THREADS, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const GemmParams p) {
  using C = GemmCfg<NUM_A>;
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
  float* red = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES + C::BAR_BYTES);  // [4][G_BN]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 4);
    }
    mbar_init(drain, 1);
    *epi_fail = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, G_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  const int n_tiles = (*p.n_chunks) * p.a_row_tiles;
  const int k_tiles = p.k_tiles;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    int stage = 0;
    uint32_t phase = 0;
    int issued = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
      const int c = t / p.a_row_tiles, mt = t - c * p.a_row_tiles;
      const int4 ch = p.chunks[c];
      const int slot = p.slot_of[ch.x];
      if (slot < 0 || slot >= p.n_slots) {
        set_status(p.status, DSV4_ENOTFOUND);
        continue;
      }
      const uint8_t* sf_base = p.arena + (int64_t)slot * p.slot_bytes + p.sfa_off;
      for (int kt = 0; kt < k_tiles; ++kt) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + stage * C::STAGE_BYTES;
        uint8_t* sA0 = st;
        uint8_t* sA1 = st + C::A_BYTES;
        uint8_t* sB = st + NUM_A * C::A_BYTES;
        uint8_t* sSFA = sB + C::B_BYTES;
        uint8_t* sSFB = sSFA + NUM_A * C::SF_BYTES;
        // B scales: row n of the tile -> byte (n%32)*16 + (n/32)*4
        const uint32_t* bsf = p.b_sf + (int64_t)kt * p.p_cap + ch.y;
#pragma unroll
        for (int h = 0; h < G_BN / 32; ++h) {
          const int n = lane + 32 * h;
          *reinterpret_cast<uint32_t*>(sSFB + (n & 31) * 16 + (n >> 5) * 4) = bsf[n];
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          constexpr uint32_t a_tx = G_BM * G_BK / 2;  // packed bytes of one A box
          constexpr uint32_t b_tx = B_FP4 ? G_BN * G_BK / 2 : G_BN * G_BK;
          mbar_expect_tx(&full[stage], NUM_A * (a_tx + C::SF_BYTES) + b_tx);
          tma_load_3d(sA0, &tmA, &full[stage], kt * G_BK, mt * G_BM, slot, pol_w);
          bulk_load(sSFA, sf_base + ((int64_t)mt * k_tiles + kt) * C::SF_BYTES, C::SF_BYTES, &full[stage], pol_w);
          if (NUM_A == 2) {
            tma_load_3d(sA1, &tmA, &full[stage], kt * G_BK, p.a1_row_offset + mt * G_BM, slot, pol_w);
            const int rt1 = p.a1_row_offset / G_BM + mt;
            bulk_load(sSFA + C::SF_BYTES, sf_base + ((int64_t)rt1 * k_tiles + kt) * C::SF_BYTES, C::SF_BYTES,
                      &full[stage], pol_w);
          }
          tma_load_2d(sB, &tmB, &full[stage], kt * G_BK, ch.y, pol_x);
          mbar_arrive(&full[stage]);
        }
        __syncwarp();
        ++issued;
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (!ok && lane == 0) {
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
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int abuf = 0;
      uint32_t aphase = 0;
      bool ok = true;
      const uint32_t sfa0 = tmem + G_SF_COL, sfa1 = tmem + G_SF_COL + 4, sfb = tmem + G_SF_COL + 8;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
        const int c = t / p.a_row_tiles;
        const int slot = p.slot_of[p.chunks[c].x];
        if (slot < 0 || slot >= p.n_slots) continue;
        if (!mbar_wait(&accempty[abuf], aphase ^ 1u, p.status)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)abuf * (NUM_A * G_BN);
        const uint32_t d1 = d0 + G_BN;
        for (int kt = 0; kt < k_tiles; ++kt) {
          if (!mbar_wait(&full[stage], phase, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint8_t* st = smem + stage * C::STAGE_BYTES;
          const uint32_t aA0 = smem_u32(st), aA1 = smem_u32(st + C::A_BYTES);
          const uint32_t aB = smem_u32(st + NUM_A * C::A_BYTES);
          const uint32_t aSFA = aB + C::B_BYTES;
          const uint32_t aSFB = aSFA + NUM_A * C::SF_BYTES;
          tc_cp_sf(sfa0, desc_sf(aSFA));
          if (NUM_A == 2) tc_cp_sf(sfa1, desc_sf(aSFA + C::SF_BYTES));
          tc_cp_sf(sfb, desc_sf(aSFB));
          const uint64_t dA0 = desc_sw128(aA0), dA1 = desc_sw128(aA1), dB = desc_sw128(aB);
#pragma unroll
          for (int kb = 0; kb < G_BK / 32; ++kb) {
            const uint32_t idesc = idesc_mxf8f6f4(G_BN, B_FP4, (uint32_t)kb);
            const uint32_t sel = (uint32_t)kb << 30;
            const uint32_t acc = (kt | kb) != 0 ? 1u : 0u;
            // +32 bytes of K per step inside the 128-byte swizzle row
            tc_mma_mxf8f6f4(d0, dA0 + 2u * kb, dB + 2u * kb, idesc, acc, sfa0 | sel, sfb | sel);
            if (NUM_A == 2) tc_mma_mxf8f6f4(d1, dA1 + 2u * kb, dB + 2u * kb, idesc, acc, sfa1 | sel, sfb | sel);
          }
          tc_commit(&empty[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&accfull[abuf]);
        if (++abuf == 2) {
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
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;            // TMEM lane quarter of this warp
    const int ew = warp - 2;           // 0..3
    const int i = q * 32 + lane;       // row inside the 128-row tile
    int abuf = 0;
    uint32_t aphase = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
      const int c = t / p.a_row_tiles, mt = t - c * p.a_row_tiles;
      const int4 ch = p.chunks[c];
      const int slot = p.slot_of[ch.x];
      if (slot < 0 || slot >= p.n_slots) continue;
      const int row0 = ch.y, nrows = ch.z;
      // all four epilogue warps take the same decision: a failed wait in any
      // of them ends the loop for all (the named barriers below need all 4)
      if (!mbar_wait(&accfull[abuf], aphase, p.status) && lane == 0) atomicOr(epi_fail, 1);
      named_bar_sync(1, 128);
      if (*reinterpret_cast<volatile int*>(epi_fail) != 0) break;
      tc_fence_after();
      float acc0[G_BN];
      float acc1[NUM_A == 2 ? G_BN : 1];
      (void)acc1;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)abuf * (NUM_A * G_BN);
#pragma unroll
      for (int j = 0; j < G_BN / 16; ++j) tmem_ld16(tbase + j * 16, acc0 + j * 16);
      if constexpr (NUM_A == 2) {
#pragma unroll
        for (int j = 0; j < G_BN / 16; ++j) tmem_ld16(tbase + G_BN + j * 16, acc1 + j * 16);
      }
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[abuf]);
      if (++abuf == 2) {
        abuf = 0;
        aphase ^= 1u;
      }

      if constexpr (EPI == EPI_STORE_BF16) {
        uint16_t* dst = p.out_bf16 + (int64_t)row0 * p.out_ld + mt * G_BM + i;
#pragma unroll
        for (int n = 0; n < G_BN; ++n)
          if (n < nrows) dst[(int64_t)n * p.out_ld] = bf16_bits(acc0[n]);
      } else {
        // gate = bf16(w1 x), up = bf16(w3 x); clamp; h = silu(gate)*up*w_route;
        // bf16(h) is the input of the activation re-quantisation.
        const float lim = p.swiglu_limit;
#pragma unroll
        for (int n = 0; n < G_BN; ++n) {
          float g = bf16r(acc0[n]);
          float u = bf16r(acc1[n]);
          if (lim > 0.f) {
            u = fminf(fmaxf(u, -lim), lim);
            g = fminf(g, lim);
          }
          const float w = (n < nrows) ? p.sorted_w[row0 + n] : 0.f;
          acc0[n] = bf16r(silu_f(g) * u * w);
        }
        if constexpr (EPI == EPI_SWIGLU_FP8) {
          // per-token amax over the 128 rows of this tile = one 128-block of I
#pragma unroll
          for (int n = 0; n < G_BN; ++n) {
            const float m = warp_max_f(fabsf(acc0[n]));
            if (lane == 0) red[ew * G_BN + n] = m;
          }
          named_bar_sync(1, 128);
          uint8_t* dst = p.out_q + (int64_t)row0 * p.out_ld + mt * G_BM + i;
#pragma unroll
          for (int n = 0; n < G_BN; ++n) {
            if (n < nrows) {
              const float amax = fmaxf(fmaxf(red[n], red[G_BN + n]), fmaxf(red[2 * G_BN + n], red[3 * G_BN + n]));
              const int e = fp8_scale_exp(amax);
              const float v = fminf(fmaxf(acc0[n] * pow2i(-e), -448.f), 448.f);
              dst[(int64_t)n * p.out_ld] = (uint8_t)e4m3_byte(v);
              if (i == 0) p.out_sf[(int64_t)mt * p.p_cap + row0 + n] = (uint32_t)(e + 127) * 0x01010101u;
            }
          }
          named_bar_sync(1, 128);
        } else {
          // per-token amax over the 32 rows of this warp = one 32-block of I
          uint8_t* dst = p.out_q + (int64_t)row0 * (p.out_ld / 2) + (mt * G_BM + i) / 2;
          uint8_t* sfd = reinterpret_cast<uint8_t*>(p.out_sf) + ((int64_t)mt * p.p_cap + row0) * 4 + q;
#pragma unroll
          for (int n = 0; n < G_BN; ++n) {
            if (n < nrows) {
              const float amax = warp_max_f(fabsf(acc0[n]));
              const int e = mx_scale_exp(amax);
              const uint32_t code = e2m1_code(acc0[n] * pow2_any(-e));
              const uint32_t hi = __shfl_down_sync(0xffffffffu, code, 1);
              if ((lane & 1) == 0) dst[(int64_t)n * (p.out_ld / 2)] = (uint8_t)(code | (hi << 4));
              if (lane == 0) sfd[(int64_t)n * 4] = (uint8_t)(e + 127);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, G_TMEM_COLS);
  }
}

}  // namespace dsv4
