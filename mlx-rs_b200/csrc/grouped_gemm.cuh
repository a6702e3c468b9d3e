// Grouped dequantising GEMM for the routed experts on sm_100a (tcgen05 +
// TMEM + TMA), shared by the gate/up (+SwiGLU) and down projections.
//
// Reference op: gather_qmm(x_sorted, w, scales, biases, rhs=expert ids,
// transpose=true, sorted_indices=true) as issued by SplitSwitchFfn::forward
// (crates/mlxr-lm/src/nn/switch.rs:417-441) through
// QuantizedSwitchLinear::apply (switch.rs:148-167), and for the gate/up pair
// the swiglu that follows (activations.rs:198-200).
//
// Orientation ("weights as M"): one work item is a 128-row slice of one
// expert's weight matrix (the A operand, K-major, dequantised into shared
// memory) times a tile of up to BN expert-sorted token rows (the B operand,
// K-major, loaded by TMA with 128-byte swizzle). The accumulator D[128, BN]
// lives in TMEM: lane = output feature, column = token. Decode batches use
// small BN (16/32), prefill BN = 128 (gate/up) or 256 (down).
//
// Warp roles (480 threads):
//   warps 0-3   epilogue: TMEM -> registers -> SwiGLU / plain -> bf16 global
//   warps 4-11  dequant: packed uint32 tile (smem) -> bf16 swizzled A tile
//   warp 12     TMA producer for packed weight tiles (raw ring)
//   warp 13     TMA producer for activation tiles (operand ring)
//   warp 14     TMEM allocator + single-thread tcgen05.mma issuer
// Accumulators are double-buffered in TMEM when they fit (2*NMAT*BN <= 512),
// so the epilogue of item i overlaps the main loop of item i+1.
#pragma once

#include "common.cuh"

#ifndef MLXR_RAW_WAR_FENCE
#define MLXR_RAW_WAR_FENCE 1
#endif

namespace mlxr {

// One entry of the device-built tile list: expert, first sorted row, rows.
struct GemmTile {
  int32_t expert;
  int32_t row_start;
  int32_t row_count;
  int32_t pad;
};

template <int NMAT, int BN, int BITS>
struct GG {
  static constexpr int BM = 128;
  static constexpr int BK = 64;  // == group size
  static constexpr int KW = BK * BITS / 32;               // packed words per row per k-step
  static constexpr int RAW_ROW = KW * 4;                  // bytes
  static constexpr int RAW_MAT = BM * RAW_ROW;
  static constexpr int RAW_STAGE = NMAT * RAW_MAT;
  static constexpr int A_MAT = BM * BK * 2;               // 16 KB bf16
  static constexpr int A_STAGE = NMAT * A_MAT;
  static constexpr int B_STAGE = BN * BK * 2;
  static constexpr int RS = RAW_STAGE <= 8192 ? 8 : 4;    // raw ring depth
  static constexpr int SMEM_BUDGET = 220 * 1024;
  static constexpr int OS_FIT = (SMEM_BUDGET - RS * RAW_STAGE) / (A_STAGE + B_STAGE);
  static constexpr int OS = OS_FIT > 4 ? 4 : OS_FIT;      // operand ring depth
  static_assert(OS >= 2, "shared memory budget too small");
  static constexpr int ACC_COLS = NMAT * BN;
  static constexpr int AB = (2 * ACC_COLS <= 512) ? 2 : 1;
  static constexpr int TMEM_NEED = AB * ACC_COLS;
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                   : TMEM_NEED <= 256 ? 256 : 512;
  static_assert(TMEM_NEED <= 512, "accumulators exceed tensor memory");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128 must be a multiple of 16 in [16, 256]");
  static constexpr int NUM_THREADS = 480;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + OS * A_STAGE;
  static constexpr int OFF_RAW = OFF_B + OS * B_STAGE;
  static constexpr int OFF_BAR = OFF_RAW + RS * RAW_STAGE;
  static constexpr int NUM_BARS = 2 * RS + 2 * OS + 2 * AB + 1;
  static constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16 + 1024;  // + alignment slack
  static constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN);
};

struct GemmArgs {
  const uint16_t* scales[2];  // bf16 [E*Nout, K/64]
  const uint16_t* biases[2];
  const GemmTile* tiles;
  const int32_t* num_tiles;
  uint16_t* out;              // bf16 [rows, Nout]
  int32_t n_out;              // Nout (multiple of 128)
  int32_t k_dim;              // K (multiple of 64)
  int32_t num_experts;
  int32_t max_tiles;
  int64_t out_rows;           // rows of `out` (and of the activation operand)
  int* status;
};

// A tile entry is used only if it names a valid expert and a row range inside
// the output; every role evaluates the same predicate and skips bad entries,
// so a corrupted tile list can never turn into a wild load or store.
__device__ inline bool tile_ok(const GemmTile& t, const GemmArgs& a) {
  return t.expert >= 0 && t.expert < a.num_experts && t.row_start >= 0 && t.row_count > 0 &&
         (int64_t)t.row_start + t.row_count <= a.out_rows;
}

// 4-bit word (8 codes) -> 8 bf16 values s*q + b (one rounding, bf16 fma).
__device__ inline uint4 dequant_word4(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 b2) {
  const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.0f, 128.0f);
  uint32_t t[4];
  t[0] = (w & 0x000F000Fu) | 0x43004300u;
  t[1] = ((w >> 4) & 0x000F000Fu) | 0x43004300u;
  t[2] = ((w >> 8) & 0x000F000Fu) | 0x43004300u;
  t[3] = ((w >> 12) & 0x000F000Fu) | 0x43004300u;
  uint32_t d[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&t[i]);
    v = __hsub2(v, k128);  // exact: (128 + q) - 128
    v = __hfma2(v, s2, b2);
    d[i] = *reinterpret_cast<uint32_t*>(&v);
  }
  // d[i] holds codes (i, i+4); reorder to (0,1) (2,3) (4,5) (6,7).
  uint4 o;
  o.x = __byte_perm(d[0], d[1], 0x5410);
  o.y = __byte_perm(d[2], d[3], 0x5410);
  o.z = __byte_perm(d[0], d[1], 0x7632);
  o.w = __byte_perm(d[2], d[3], 0x7632);
  return o;
}

// Two 8-bit words (8 codes) -> 8 bf16 values: codes made exact in fp32 via
// the 2^23 mantissa trick, fp32 fma, one rounding to bf16.
__device__ inline uint4 dequant_words8(uint32_t w0, uint32_t w1, float s, float b) {
  float v[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = __uint_as_float(__byte_perm(w0, 0x4B000000u, 0x7540 + j)) - 8388608.0f;
    v[4 + j] = __uint_as_float(__byte_perm(w1, 0x4B000000u, 0x7540 + j)) - 8388608.0f;
  }
  uint4 o;
  o.x = pack_bf16x2(__fmaf_rn(v[0], s, b), __fmaf_rn(v[1], s, b));
  o.y = pack_bf16x2(__fmaf_rn(v[2], s, b), __fmaf_rn(v[3], s, b));
  o.z = pack_bf16x2(__fmaf_rn(v[4], s, b), __fmaf_rn(v[5], s, b));
  o.w = pack_bf16x2(__fmaf_rn(v[6], s, b), __fmaf_rn(v[7], s, b));
  return o;
}

// After a producer stops (normally or on abort), wait (bounded) until every
// TMA load it issued into a ring of STAGES slots has landed, so no copy is
// still writing shared memory when the CTA exits. `issued` = loads issued.
template <int STAGES>
__device__ inline void drain_ring(uint64_t* full, uint32_t issued, volatile int* abort_flag, int* status) {
  for (uint32_t s = 0; s < (uint32_t)STAGES && s < issued; ++s) {
    const uint32_t last = issued - 1 - ((issued - 1 - s) % STAGES);
    int dummy_abort = 0;
    (void)abort_flag;
    mbar_wait(&full[s], (last / STAGES) & 1, &dummy_abort, status);
  }
}

template <int NMAT, int BN, int BITS>
__global__ void __launch_bounds__(480, 1)
    grouped_dequant_gemm_kernel(const __grid_constant__ CUtensorMap tm_a0, const __grid_constant__ CUtensorMap tm_a1,
                                const __grid_constant__ CUtensorMap tm_b, const GemmArgs args) {
  using C = GG<NMAT, BN, BITS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem + C::OFF_A;
  uint8_t* sB = smem + C::OFF_B;
  uint8_t* sRaw = smem + C::OFF_RAW;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + C::RS;
  uint64_t* op_full = raw_empty + C::RS;
  uint64_t* op_empty = op_full + C::OS;
  uint64_t* acc_full = op_empty + C::OS;
  uint64_t* acc_empty = acc_full + C::AB;
  uint64_t* fin_bar = acc_empty + C::AB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fin_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::RS; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], 8);
    }
    for (int i = 0; i < C::OS; ++i) {
      mbar_init(&op_full[i], 1 + 8);
      mbar_init(&op_empty[i], 1);
    }
    for (int i = 0; i < C::AB; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(fin_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 14) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 12 && lane == 0) {
    prefetch_tmap(&tm_a0);
    if (NMAT == 2) prefetch_tmap(&tm_a1);
    prefetch_tmap(&tm_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_out = args.n_out;
  const int mt_per_expert = n_out / C::BM;
  const int ksteps = args.k_dim / C::BK;
  int ntiles = *args.num_tiles;
  if (ntiles > args.max_tiles) ntiles = args.max_tiles;
  const int num_items = ntiles * mt_per_expert;

  if (warp == 12) {
    // ---------------------------------------------- raw weight producer --
    if (lane == 0) {
      uint32_t it = 0;
      for (int item = blockIdx.x; item < num_items && !*abort_flag; item += gridDim.x) {
        const GemmTile t = args.tiles[item / mt_per_expert];
        if (!tile_ok(t, args)) {
          atomicCAS(args.status, 0, (int)kDevBadIndex);
          continue;
        }
        const int a_row = t.expert * n_out + (item % mt_per_expert) * C::BM;
        for (int ks = 0; ks < ksteps; ++ks, ++it) {
          const int s = it % C::RS;
          if (!mbar_wait(&raw_empty[s], ((it / C::RS) & 1) ^ 1, abort_flag, args.status)) break;
          mbar_arrive_expect_tx(&raw_full[s], C::RAW_STAGE);
          tma_load_2d(sRaw + s * C::RAW_STAGE, &tm_a0, &raw_full[s], ks * C::KW, a_row);
          if (NMAT == 2) tma_load_2d(sRaw + s * C::RAW_STAGE + C::RAW_MAT, &tm_a1, &raw_full[s], ks * C::KW, a_row);
        }
      }
      drain_ring<C::RS>(raw_full, it, abort_flag, args.status);
    }
  } else if (warp == 13) {
    // ------------------------------------------- activation producer ----
    if (lane == 0) {
      uint32_t it = 0;
      for (int item = blockIdx.x; item < num_items && !*abort_flag; item += gridDim.x) {
        const GemmTile t = args.tiles[item / mt_per_expert];
        if (!tile_ok(t, args)) continue;
        for (int ks = 0; ks < ksteps; ++ks, ++it) {
          const int s = it % C::OS;
          if (!mbar_wait(&op_empty[s], ((it / C::OS) & 1) ^ 1, abort_flag, args.status)) break;
          mbar_arrive_expect_tx(&op_full[s], C::B_STAGE);
          tma_load_2d(sB + s * C::B_STAGE, &tm_b, &op_full[s], ks * C::BK, t.row_start);
        }
      }
      drain_ring<C::OS>(op_full, it, abort_flag, args.status);
    }
  } else if (warp == 14) {
    // ----------------------------------------------------- MMA issuer ----
    if (lane == 0) {
      uint32_t it = 0, li = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
        if (!tile_ok(args.tiles[item / mt_per_expert], args)) continue;
        const int ab = li % C::AB;
        const uint32_t acc_phase = (li / C::AB) & 1;
        ++li;  // counts valid items only, exactly like the epilogue
        if (!mbar_wait(&acc_empty[ab], acc_phase ^ 1, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t d0 = tmem_base + (uint32_t)(ab * C::ACC_COLS);
        for (int ks = 0; ks < ksteps; ++ks, ++it) {
          const int s = it % C::OS;
          if (!mbar_wait(&op_full[s], (it / C::OS) & 1, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * C::A_STAGE);
          const uint32_t b_base = smem_u32(sB + s * C::B_STAGE);
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk) {
            const uint64_t bdesc = umma_desc_sw128(b_base + kk * 32);
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
              const uint64_t adesc = umma_desc_sw128(a_base + m * C::A_MAT + kk * 32);
              umma_bf16(d0 + (uint32_t)(m * BN), adesc, bdesc, C::IDESC, (ks | kk) != 0 ? 1u : 0u);
            }
          }
          umma_commit(&op_empty[s]);
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
      // Quiesce the tensor pipe before TMEM is released.
      umma_commit(fin_bar);
      mbar_wait(fin_bar, 0, abort_flag, args.status);
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------- dequant ----
    const int dt = threadIdx.x - 128;          // 0..255
    const int mat = NMAT == 2 ? dt >> 7 : 0;   // gate / up
    const int row = dt & 127;
    const int c_lo = NMAT == 2 ? 0 : (dt >> 7) * 4;  // first 16 B chunk of this thread
    constexpr int NCH = NMAT == 2 ? 8 : 4;           // chunks per thread per k-step
    const int G = args.k_dim / 64;
    uint32_t rit = 0, oit = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
      const GemmTile t = args.tiles[item / mt_per_expert];
      if (!tile_ok(t, args)) continue;
      const int64_t srow = (int64_t)t.expert * n_out + (item % mt_per_expert) * C::BM + row;
      const uint16_t* sp = args.scales[mat] + srow * G;
      const uint16_t* bp = args.biases[mat] + srow * G;
      // Scale/bias prefetch ring (distance 2) held in registers.
      uint16_t s0 = __ldg(sp), b0 = __ldg(bp);
      uint16_t s1 = G > 1 ? __ldg(sp + 1) : 0, b1 = G > 1 ? __ldg(bp + 1) : 0;
      for (int ks = 0; ks < ksteps; ++ks, ++rit, ++oit) {
        uint16_t s2 = 0, b2v = 0;
        if (ks + 2 < G) {
          s2 = __ldg(sp + ks + 2);
          b2v = __ldg(bp + ks + 2);
        }
        // Packed codes of this thread's slice.
        const int rs = rit % C::RS;
        if (!mbar_wait(&raw_full[rs], (rit / C::RS) & 1, abort_flag, args.status)) {
          ok = false;
          break;
        }
        uint32_t wv[NCH * BITS / 4];
        {
          const uint4* src = reinterpret_cast<const uint4*>(sRaw + rs * C::RAW_STAGE + mat * C::RAW_MAT +
                                                            row * C::RAW_ROW + c_lo * BITS);
#pragma unroll
          for (int i = 0; i < NCH * BITS / 16; ++i) {
            const uint4 v = src[i];
            wv[4 * i + 0] = v.x;
            wv[4 * i + 1] = v.y;
            wv[4 * i + 2] = v.z;
            wv[4 * i + 3] = v.w;
          }
        }
#if MLXR_RAW_WAR_FENCE
        // The slot is refilled by TMA (async proxy) once all warps release it:
        // order this warp's generic-proxy reads before that write.
        fence_proxy_async_smem();
#endif
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);
        const int os = oit % C::OS;
        if (!mbar_wait(&op_empty[os], ((oit / C::OS) & 1) ^ 1, abort_flag, args.status)) {
          ok = false;
          break;
        }
        uint8_t* dstA = sA + os * C::A_STAGE + mat * C::A_MAT;
        if (BITS == 4) {
          const __nv_bfloat162 s2v = __halves2bfloat162(__ushort_as_bfloat16(s0), __ushort_as_bfloat16(s0));
          const __nv_bfloat162 b2 = __halves2bfloat162(__ushort_as_bfloat16(b0), __ushort_as_bfloat16(b0));
#pragma unroll
          for (int c = 0; c < NCH; ++c) {
            const uint4 o = dequant_word4(wv[c], s2v, b2);
            *reinterpret_cast<uint4*>(dstA + sw128_offset(row, c_lo + c)) = o;
          }
        } else {
          const float sf = bf16_bits_to_f32(s0), bf = bf16_bits_to_f32(b0);
#pragma unroll
          for (int c = 0; c < NCH; ++c) {
            const uint4 o = dequant_words8(wv[2 * c], wv[2 * c + 1], sf, bf);
            *reinterpret_cast<uint4*>(dstA + sw128_offset(row, c_lo + c)) = o;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&op_full[os]);
        s0 = s1; b0 = b1;
        s1 = s2; b1 = b2v;
      }
    }
  } else {
    // ------------------------------------------------------- epilogue ----
    const int q = warp;  // TMEM lane quarter 0..3
    uint32_t li = 0;
    for (int item = blockIdx.x; item < num_items; item += gridDim.x) {
      const GemmTile t = args.tiles[item / mt_per_expert];
      if (!tile_ok(t, args)) continue;
      const int ab = li % C::AB;
      const uint32_t acc_phase = (li / C::AB) & 1;
      ++li;
      if (!mbar_wait(&acc_full[ab], acc_phase, abort_flag, args.status)) break;
      tc_fence_after();
      const int f = (item % mt_per_expert) * C::BM + q * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * C::ACC_COLS);
      uint16_t* outp = args.out + (int64_t)t.row_start * n_out + f;
      const int rows = t.row_count < BN ? t.row_count : BN;
      constexpr int CW = BN >= 32 ? 32 : 16;  // TMEM columns per load
#pragma unroll 1
      for (int c = 0; c < BN / CW; ++c) {
        if (c * CW >= rows) break;
        uint32_t g[32];
        uint32_t u[32];
        if (CW == 32) {
          if (NMAT == 2) tmem_ld2_x32_wait(tbase + c * 32, tbase + BN + c * 32, g, u);
          else tmem_ld_x32_wait(tbase + c * 32, g);
        } else {
          if (NMAT == 2) tmem_ld2_x16_wait(tbase, tbase + BN, g, u);
          else tmem_ld_x16_wait(tbase, g);
        }
        const int nvalid = rows - c * CW < CW ? rows - c * CW : CW;
#pragma unroll
        for (int j = 0; j < CW; ++j) {
          if (j < nvalid) {
            float v = __uint_as_float(g[j]);
            if (NMAT == 2) v = silu_f32(v) * __uint_as_float(u[j]);
            outp[(int64_t)(c * CW + j) * n_out] = f32_to_bf16_bits(v);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 14) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace mlxr
