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
// expert's weight matrix (the A operand) times a tile of up to BN
// expert-sorted token rows (the B operand, K-major, loaded by TMA with
// 128-byte swizzle). The dequantised A operand lives in tensor memory, not in
// shared memory: the dequant thread that owns weight row r writes its bf16
// values into TMEM lane r with tcgen05.st and tcgen05.mma reads A from TMEM
// (the A-in-TMEM form). This keeps shared memory for the TMA streams only;
// with A in shared memory, writing it and the tensor core re-reading it made
// shared-memory bandwidth the limit of the decode path. The accumulator
// D[128, BN] lives in TMEM too: lane = output feature, column = token.
// Decode batches use small BN (16/32), prefill BN = 128 (gate/up) or 256 (down).
//
// Warp roles (736 threads, 768 with two weight matrices or narrow tiles):
//   warps 0-3   epilogue: TMEM -> registers -> SwiGLU / plain -> bf16 global
//   warps 4-19  dequant: packed uint32 tile (smem) -> bf16 A stage in TMEM;
//               NGRP = 2 (two matrices) or 4 (one) groups of warps take
//               turns by k-step, each thread a whole weight row of its
//               k-steps, so the groups run a stage apart and hide each
//               other's barrier, fence and TMEM-store latencies
//   warp 20     TMA producer for packed weight tiles (raw ring)
//   warp 21     TMA producer for activation tiles (B ring)
//   warps 22-   single-thread tcgen05.mma issuers: one per weight matrix, or
//               for narrow tiles (BN <= 32) one per k-step parity
//               (warp 22 also allocates TMEM)
// TMEM columns: [0, AB*NMAT*BN*KP) accumulators (double-buffered when they fit,
// so the epilogue of item i overlaps the main loop of item i+1), then OS
// stages of NMAT x 32 columns (128 rows x 64 bf16) of dequantised A. The
// activation tiles have their own, deeper ring of OSB shared-memory stages.
#pragma once

#include "common.cuh"

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
  static constexpr int B_STAGE = BN * BK * 2;
  // Narrow (decode) tiles split every accumulator by k-step parity: two
  // issuers, one per parity, each issue all NMAT matrices' MMAs of their own
  // k-steps into their own accumulators, and the epilogue adds the halves.
  // The fixed cost a thread pays per tcgen05.mma, commit and barrier wait,
  // not the tensor pipe, bounds a single issuer's k-step rate at these widths.
  static constexpr int KP = BN <= 32 ? 2 : 1;
  // Tensor memory: accumulators, then the A stages.
  static constexpr int ACC_COLS = NMAT * BN * KP;
  static constexpr int A_COLS = NMAT * 32;                // one A stage: NMAT x (128 x 64 bf16)
  static constexpr int AB = (2 * ACC_COLS + 2 * A_COLS <= 512) ? 2 : 1;
  static constexpr int OS_FIT = (512 - AB * ACC_COLS) / A_COLS;
  // Scales and biases staged in shared memory by TMA: one block holds SB_K
  // k-steps (groups) of the 128 rows' scales and biases of every matrix of
  // the item (a {SB_K x 128} bf16 box each, rows 16 bytes apart).
  static constexpr int SB_K = 8;
  static constexpr int SB_BOX = BM * SB_K * 2;
  static constexpr int SB_STAGE = NMAT * 2 * SB_BOX;
  static constexpr int SBS = 3;
  // Two rings per k-step, each released by the MMA commits of that k-step:
  // the dequantised A tile in TMEM (OS stages, bounded by tensor memory)
  // and the activation (B) tile in shared memory (OSB stages). The B ring
  // is deeper than the A ring: the activation tile's TMA load is the
  // longest round trip of a k-step (about 1.8 us on the 128-token prefill
  // tiles, issued only once its slot is free), so with the two rings tied
  // together at four stages a k-step took (TMA latency + MMA) / 4.
  static constexpr int SMEM_RINGS = 220 * 1024 - SBS * SB_STAGE;  // B + packed-weight rings
  static constexpr int OS_T = OS_FIT > 6 ? 6 : OS_FIT;
  static constexpr int OS = OS_T;
  static constexpr int OSB_ROOM = (SMEM_RINGS - 4 * RAW_STAGE) / B_STAGE;
  static constexpr int OSB = OSB_ROOM > 8 ? 8 : OSB_ROOM;
  // Packed-weight ring: up to 96 KB (16 stages) in what shared memory leaves.
  static constexpr int RS_ROOM = (SMEM_RINGS - OSB * B_STAGE) / RAW_STAGE;
  static constexpr int RS_WANT = (96 * 1024) / RAW_STAGE;
  static constexpr int RS_A = RS_WANT > 16 ? 16 : RS_WANT;
  static constexpr int RS = RS_A < RS_ROOM ? RS_A : RS_ROOM;
  static_assert(RS >= 4, "shared memory too small for the packed-weight ring");
  static_assert(OS >= 2, "tensor memory too small for two A stages");
  static_assert(OSB >= 2, "shared memory too small for two activation stages");
  static constexpr int A_BASE = AB * ACC_COLS;
  static constexpr int TMEM_NEED = A_BASE + OS * A_COLS;
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                   : TMEM_NEED <= 256 ? 256 : 512;
  static_assert(TMEM_NEED <= 512, "tensor memory exceeded");
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128 must be a multiple of 16 in [16, 256]");
  // One MMA-issuing thread per matrix: issuing a tcgen05.mma costs the issuing
  // thread tens of cycles whatever N is, so with narrow decode tiles a single
  // issuer, not the tensor pipe, bounds the k-step rate.
  static constexpr int ISSUERS = KP == 2 ? 2 : NMAT;
  static constexpr int STAGE_COMMITS = KP == 2 ? 1 : ISSUERS;  // commits that release one stage
  static constexpr int DQ_WARPS = 16;
  static constexpr int W_RAW = 4 + DQ_WARPS;  // raw weight producer warp
  static constexpr int W_B = W_RAW + 1;       // activation producer warp
  static constexpr int W_MMA = W_B + 1;       // first MMA issuer warp (allocates TMEM)
  static constexpr int NUM_THREADS = 32 * (W_MMA + ISSUERS);
  // Dequant groups: group g takes the k-steps it with it % NGRP == g.
  static constexpr int NGRP = (DQ_WARPS * 32) / (NMAT * BM);
  static constexpr int GRP_WARPS = DQ_WARPS / NGRP;  // arrivals per stage
  static constexpr int NCH = 8;                      // 8-weight chunks per row per k-step
  static constexpr int WBYTES = NCH * BITS;          // packed bytes per thread per k-step
  static constexpr int OFF_B = 0;
  static constexpr int OFF_RAW = OFF_B + OSB * B_STAGE;
  static constexpr int OFF_SB = OFF_RAW + RS * RAW_STAGE;
  static constexpr int OFF_BAR = OFF_SB + SBS * SB_STAGE;
  static constexpr int NUM_BARS = 2 * RS + 2 * OS + 2 * OSB + 2 * AB + 1 + 2 * SBS;
  static constexpr int SCHED_Q = 16;  // work-queue entries published ahead (shared-memory ring)
  // At least 120 KB so that two CTAs never share an SM: each CTA holds its
  // tensor memory for its whole (persistent) lifetime.
  static constexpr int SMEM_USED = OFF_BAR + NUM_BARS * 8 + 16 + (SCHED_Q + 2) * 4 + 1024;  // + alignment slack
  static constexpr int SMEM_BYTES = SMEM_USED > 120 * 1024 ? SMEM_USED : 120 * 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory exceeded");
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
  int perm_out;               // store out's feature axis in the 4-bit chunk K order
  int pair;                   // NMAT == 2 only: the two matrices are row blocks m and m+128
                              // of one weight (plain epilogue) instead of gate and up (SwiGLU)
  int32_t w_rows1;            // weight rows per expert of the first phase: Nout, or 2*Nout
                              // for a packed gate|up [E, 2*Nout, K] (up = rows Nout..)
  int* status;
  // Scales and biases come through the TMA staging ring (their tensor maps
  // are valid: 16-byte aligned rows of a multiple of 8 groups) for the items
  // of phase 1 / phase 2; otherwise every dequant thread loads its own.
  int sb1, sb2;
  // Split-K (splits > 1): every (tile, row slice) is split into `splits`
  // k-ranges; each writes its fp32 accumulators to `partial`, and the last
  // split to finish (per TMEM lane quarter, counted in `counters`, zero on
  // entry) adds them up in split order and runs the epilogue.
  int splits;
  int max_split_rows;         // row slices `partial` and `counters` hold
  float* partial;             // [row slices][splits][4 quarters][NMAT][BN][32]
  int32_t* counters;          // [row slices][4]
  // Fused launch (second phase): after the gate|up items (phase 1), the same
  // CTAs run the down projection items (phase 2: row pairs of the down weight,
  // plain epilogue) over the same tile list. A phase-2 item of tile j loads
  // its activation rows (h) once all phase-1 items of tile j have stored
  // them: tile_ready[j] counts their epilogue warps (zero on entry).
  const uint16_t* scales2;
  const uint16_t* biases2;
  uint16_t* out2;             // bf16 [rows, n_out2]
  int32_t n_out2;             // multiple of 256
  int32_t k_dim2;             // multiple of 64
  int32_t* tile_ready;        // [max_tiles]
  // Work queue: sched[0] counts the items handed out beyond each CTA's
  // first (item blockIdx.x), sched[1] the CTAs that finished; zero before the
  // launch, and the last CTA to finish zeroes both again.
  int32_t* sched;
};

// A tile entry is used only if it names a valid expert and a row range inside
// the output; every role evaluates the same predicate and skips bad entries,
// so a corrupted tile list can never turn into a wild load or store.
__device__ inline bool tile_ok(const GemmTile& t, const GemmArgs& a) {
  return t.expert >= 0 && t.expert < a.num_experts && t.row_start >= 0 && t.row_count > 0 &&
         (int64_t)t.row_start + t.row_count <= a.out_rows;
}

// K order inside every 8-element (16-byte) chunk of a 4-bit operand pair.
// The 4-bit dequantiser emits codes (0,4), (1,5), (2,6), (3,7) as bf16 pairs
// straight from the nibble masks, so A holds chunk elements in the order
// {0,4,1,5,2,6,3,7}. The tensor core only needs A and B to agree on the K
// order, so the activation operand is stored with the same order instead of
// re-shuffling every weight: element e of a chunk sits at position kperm(e).
__host__ __device__ inline int kperm_pos(int e) { return ((e & 3) << 1) | (e >> 2); }

// 4-bit word (8 codes) -> 4 bf16 pairs s*q + b (one rounding, bf16 fma) in
// the chunk order {0,4}, {1,5}, {2,6}, {3,7}.
__device__ inline void dequant_word4(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 b2, uint32_t* d) {
  const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.0f, 128.0f);
  uint32_t t[4];
  t[0] = (w & 0x000F000Fu) | 0x43004300u;
  t[1] = ((w >> 4) & 0x000F000Fu) | 0x43004300u;
  t[2] = ((w >> 8) & 0x000F000Fu) | 0x43004300u;
  t[3] = ((w >> 12) & 0x000F000Fu) | 0x43004300u;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&t[i]);
    v = __hsub2(v, k128);  // exact: (128 + q) - 128
    v = __hfma2(v, s2, b2);
    d[i] = *reinterpret_cast<uint32_t*>(&v);
  }
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

// Bounded wait until *p >= target (a counter other CTAs of this grid raise).
__device__ inline bool wait_counter_geq(const int32_t* p, int target, volatile int* abort_flag, int* status) {
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    if (v >= target) return true;
    if ((it & 63u) == 63u) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        atomicCAS(status, 0, (int)kDevTimeout);
        return false;
      }
    }
  }
}

// SPLITK: the split-K variant (args.splits > 1). FUSED: gate|up then down in
// one launch (NMAT == 2). The plain variant has both folded out. GLU: the
// gate|up epilogue applies gelu_approx (GeGLU) instead of silu (SwiGLU).
template <int NMAT, int BN, int BITS, bool SPLITK, bool FUSED, bool GLU>
__global__ void __launch_bounds__(GG<NMAT, BN, BITS>::NUM_THREADS, 1)
    grouped_dequant_gemm_kernel(const __grid_constant__ CUtensorMap tm_a0, const __grid_constant__ CUtensorMap tm_a1,
                                const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_a2,
                                const __grid_constant__ CUtensorMap tm_b2, const __grid_constant__ CUtensorMap tm_s0,
                                const __grid_constant__ CUtensorMap tm_z0, const __grid_constant__ CUtensorMap tm_s1,
                                const __grid_constant__ CUtensorMap tm_z1, const __grid_constant__ CUtensorMap tm_s2,
                                const __grid_constant__ CUtensorMap tm_z2, const GemmArgs args) {
  static_assert(!(SPLITK && FUSED), "split-K and the fused launch are separate variants");
  static_assert(!FUSED || NMAT == 2, "the fused launch pairs gate|up with row pairs of down");
  using C = GG<NMAT, BN, BITS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem + C::OFF_B;
  uint8_t* sRaw = smem + C::OFF_RAW;
  uint8_t* sSB = smem + C::OFF_SB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + C::RS;
  uint64_t* op_full = raw_empty + C::RS;   // dequantised A stage written to TMEM (dequant warps)
  uint64_t* op_empty = op_full + C::OS;     // A stage consumed (MMA commit)
  uint64_t* b_full = op_empty + C::OS;      // activation tile landed (TMA)
  uint64_t* b_empty = b_full + C::OSB;      // activation tile consumed (MMA commit)
  uint64_t* acc_full = b_empty + C::OSB;
  uint64_t* acc_empty = acc_full + C::AB;
  uint64_t* fin_bar = acc_empty + C::AB;
  uint64_t* sb_full = fin_bar + 1;          // scale/bias block landed (TMA)
  uint64_t* sb_empty = sb_full + C::SBS;    // block read by every dequant warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sb_empty + C::SBS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Work-queue ring: entry n of this CTA's item sequence in s_ring[n % Q];
  // s_pub = entries published, s_cons = entries the epilogue has finished.
  volatile int* s_ring = reinterpret_cast<volatile int*>(tmem_slot + 4);
  volatile int* s_pub = s_ring + C::SCHED_Q;
  volatile int* s_cons = s_pub + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::RS; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], C::GRP_WARPS);
    }
    for (int i = 0; i < C::OS; ++i) {
      mbar_init(&op_full[i], C::GRP_WARPS);
      mbar_init(&op_empty[i], C::STAGE_COMMITS);
    }
    for (int i = 0; i < C::OSB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], C::STAGE_COMMITS);
    }
    for (int i = 0; i < C::AB; ++i) {
      mbar_init(&acc_full[i], C::ISSUERS);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(fin_bar, C::ISSUERS);
    for (int i = 0; i < C::SBS; ++i) {
      mbar_init(&sb_full[i], 1);
      mbar_init(&sb_empty[i], C::DQ_WARPS);
    }
    *abort_flag = 0;
    *s_pub = 1;  // entry 0 is blockIdx.x, known to every role
    *s_cons = 0;
    fence_mbar_init();
  }
  if (warp == C::W_MMA) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == C::W_RAW && lane == 0) {
    prefetch_tmap(&tm_a0);
    if (NMAT == 2) prefetch_tmap(&tm_a1);
    prefetch_tmap(&tm_b);
    if (FUSED) {
      prefetch_tmap(&tm_a2);
      prefetch_tmap(&tm_b2);
    }
    if (!SPLITK && args.sb1) {
      prefetch_tmap(&tm_s0);
      prefetch_tmap(&tm_z0);
      if (NMAT == 2) {
        prefetch_tmap(&tm_s1);
        prefetch_tmap(&tm_z1);
      }
    }
    if (FUSED && args.sb2) {
      prefetch_tmap(&tm_s2);
      prefetch_tmap(&tm_z2);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above touched only this CTA's shared and tensor memory; the
  // tile list and operands come from the previous kernel.
  pdl_wait();
  pdl_launch_dependents();

  const int pair1 = NMAT == 2 ? args.pair : 0;
  const int mrows1 = pair1 ? 2 * C::BM : C::BM;  // output rows per work item
  const int mt1 = args.n_out / mrows1;
  const int ks1 = args.k_dim / C::BK;
  int ntiles = *args.num_tiles;
  if (ntiles > args.max_tiles) ntiles = args.max_tiles;
  const int S = SPLITK ? (args.splits > 1 ? args.splits : 1) : 1;
  const int n1 = ntiles * mt1 * S;
  const int mt2 = FUSED ? args.n_out2 / (2 * C::BM) : 1;
  const int ks2 = FUSED ? args.k_dim2 / C::BK : 0;
  const int num_items = n1 + (FUSED ? ntiles * mt2 : 0);
  // Work item -> tile, m-tile, k-range and phase. Phase 1: row slice
  // base = tile * mt1 + m, split s covers k-steps [s*ks1/S, (s+1)*ks1/S).
  // Phase 2 (fused launch): down row pairs of the same tiles.
  struct Item {
    int tile, m, base, split, k_lo, k_hi, ksteps, n_out, mrows, pair, wstride;
    bool ph2;
  };
  auto item_of = [&](int item) {
    Item d;
    if (!FUSED || item < n1) {
      d.base = item / S;
      d.split = item % S;
      d.tile = d.base / mt1;
      d.m = d.base % mt1;
      d.ksteps = ks1;
      d.k_lo = d.split * ks1 / S;
      d.k_hi = (d.split + 1) * ks1 / S;
      d.n_out = args.n_out;
      d.wstride = args.w_rows1;
      d.mrows = mrows1;
      d.pair = pair1;
      d.ph2 = false;
    } else {
      const int l = item - n1;
      d.base = l;
      d.split = 0;
      d.tile = l / mt2;
      d.m = l % mt2;
      d.ksteps = ks2;
      d.k_lo = 0;
      d.k_hi = ks2;
      d.n_out = args.n_out2;
      d.wstride = args.n_out2;
      d.mrows = 2 * C::BM;
      d.pair = 1;
      d.ph2 = true;
    }
    return d;
  };

  // Items whose scales and biases come through the staging ring: whole-K
  // items (no split) with a multiple of SB_K k-steps and valid maps. The
  // producer and the dequant warps evaluate the same predicate per item.
  auto item_sb = [&](const Item& d) -> bool {
    if (SPLITK) return false;
    return ((FUSED && d.ph2) ? args.sb2 : args.sb1) != 0 && d.ksteps % C::SB_K == 0 && d.k_lo == 0;
  };

  // Entry n of this CTA's work sequence (-1: no more). Entry 0 is item
  // blockIdx.x. Decode-width launches (their items are uneven: 32-k-step
  // gate|up items and 12-k-step down items, and a static round-robin left
  // whole gate|up items on a few CTAs at the end) take later entries from the
  // shared counter, fetched and published by the weight producer; wide tiles
  // keep the static round-robin (measured slightly faster there).
  const bool dynamic = C::KP == 2 && (int)gridDim.x < num_items;
  auto sched_item = [&](int n) -> int {
    if (!dynamic) {
      const int64_t it = (int64_t)blockIdx.x + (int64_t)n * gridDim.x;
      return it < num_items ? (int)it : -1;
    }
    if (n == 0) return (int)blockIdx.x < num_items ? (int)blockIdx.x : -1;
    if (*s_pub <= n) {
      const unsigned long long t0 = global_ns();
      for (uint32_t k = 1; *s_pub <= n; ++k) {
        __nanosleep(64);
        if ((k & 63u) == 0) {
          if (*abort_flag) return -1;
          if (global_ns() - t0 > kWaitLimitNs) {
            *abort_flag = 1;
            atomicCAS(args.status, 0, (int)kDevTimeout);
            return -1;
          }
        }
      }
    }
    __threadfence_block();
    return s_ring[n % C::SCHED_Q];
  };

  if (warp == C::W_RAW) {
    // ---------------------------------------------- raw weight producer --
    if (lane == 0) {
      uint32_t it = 0;
      uint32_t sbi = 0;  // scale/bias blocks issued
      for (int n = 0; !*abort_flag; ++n) {
        int item;
        if (n == 0 || !dynamic) {
          item = sched_item(n);
        } else {
          // Reuse ring slot n % Q once the epilogue has started entry n - Q + 1.
          const unsigned long long t0 = global_ns();
          bool ok = true;
          for (uint32_t k = 1; *s_cons < n - C::SCHED_Q + 1; ++k) {
            __nanosleep(64);
            if ((k & 63u) == 0 && (*abort_flag || global_ns() - t0 > kWaitLimitNs)) {
              if (!*abort_flag) atomicCAS(args.status, 0, (int)kDevTimeout);
              *abort_flag = 1;
              ok = false;
              break;
            }
          }
          if (!ok) break;
          item = (int)gridDim.x + atomicAdd(&args.sched[0], 1);
          if (item >= num_items) item = -1;
          s_ring[n % C::SCHED_Q] = item;
          __threadfence_block();
          *s_pub = n + 1;
        }
        if (item < 0) break;
        const Item d = item_of(item);
        const GemmTile t = args.tiles[d.tile];
        if (!tile_ok(t, args)) {
          atomicCAS(args.status, 0, (int)kDevBadIndex);
          continue;
        }
        const int a_row = t.expert * d.wstride + d.m * d.mrows;
        const CUtensorMap* ma = (FUSED && d.ph2) ? &tm_a2 : &tm_a0;
        const CUtensorMap* mb = (FUSED && d.ph2) ? &tm_a2 : &tm_a1;
        const bool use_sb = item_sb(d);
        const CUtensorMap* ms0 = (FUSED && d.ph2) ? &tm_s2 : &tm_s0;
        const CUtensorMap* mz0 = (FUSED && d.ph2) ? &tm_z2 : &tm_z0;
        const CUtensorMap* ms1 = (FUSED && d.ph2) ? &tm_s2 : &tm_s1;
        const CUtensorMap* mz1 = (FUSED && d.ph2) ? &tm_z2 : &tm_z1;
        const int row1 = a_row + (d.pair ? C::BM : 0);
        for (int ks = d.k_lo; ks < d.k_hi; ++ks, ++it) {
          if (use_sb && ks % C::SB_K == 0) {
            // The next SB_K groups of every matrix's scales and biases.
            const int q = sbi % C::SBS;
            if (!mbar_wait(&sb_empty[q], ((sbi / C::SBS) & 1) ^ 1, abort_flag, args.status)) break;
            mbar_arrive_expect_tx(&sb_full[q], C::SB_STAGE);
            uint8_t* dst = sSB + q * C::SB_STAGE;
            tma_load_2d(dst, ms0, &sb_full[q], ks, a_row);
            tma_load_2d(dst + C::SB_BOX, mz0, &sb_full[q], ks, a_row);
            if (NMAT == 2) {
              tma_load_2d(dst + 2 * C::SB_BOX, ms1, &sb_full[q], ks, row1);
              tma_load_2d(dst + 3 * C::SB_BOX, mz1, &sb_full[q], ks, row1);
            }
            ++sbi;
          }
          const int s = it % C::RS;
          if (!mbar_wait(&raw_empty[s], ((it / C::RS) & 1) ^ 1, abort_flag, args.status)) break;
          mbar_arrive_expect_tx(&raw_full[s], C::RAW_STAGE);
          tma_load_2d(sRaw + s * C::RAW_STAGE, ma, &raw_full[s], ks * C::KW, a_row);
          if (NMAT == 2)
            tma_load_2d(sRaw + s * C::RAW_STAGE + C::RAW_MAT, mb, &raw_full[s], ks * C::KW,
                        a_row + (d.pair ? C::BM : 0));
        }
      }
      drain_ring<C::RS>(raw_full, it, abort_flag, args.status);
      drain_ring<C::SBS>(sb_full, sbi, abort_flag, args.status);
    }
  } else if (warp == C::W_B) {
    // ------------------------------------------- activation producer ----
    if (lane == 0) {
      uint32_t it = 0;
      int s = 0;
      uint32_t ph = 0;
      for (int n = 0; !*abort_flag; ++n) {
        const int item = sched_item(n);
        if (item < 0) break;
        const Item d = item_of(item);
        const GemmTile t = args.tiles[d.tile];
        if (!tile_ok(t, args)) continue;
        const CUtensorMap* mbt = &tm_b;
        if constexpr (FUSED) {
          if (d.ph2) {
            // The tile's h rows come from phase-1 epilogues (generic stores,
            // possibly in other CTAs); order them before these TMA reads.
            if (!wait_counter_geq(args.tile_ready + d.tile, 4 * mt1, abort_flag, args.status)) break;
            asm volatile("fence.proxy.async.global;" ::: "memory");
            mbt = &tm_b2;
          }
        }
        for (int ks = d.k_lo; ks < d.k_hi; ++ks, ++it) {
          if (!mbar_wait(&b_empty[s], ph ^ 1, abort_flag, args.status)) break;
          mbar_arrive_expect_tx(&b_full[s], C::B_STAGE);
          tma_load_2d(sB + s * C::B_STAGE, mbt, &b_full[s], ks * C::BK, t.row_start);
          if (++s == C::OSB) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      drain_ring<C::OSB>(b_full, it, abort_flag, args.status);
    }
  } else if (warp >= C::W_MMA) {
    // ---------------------------------------------------- MMA issuers ----
    // Issuer mi issues the MMAs of matrix mi (gate / up) into its own
    // accumulator; every stage and accumulator barrier expects one commit
    // per issuer.
    const int mi = warp - C::W_MMA;
    if (C::KP == 2 && lane == 0) {
      // Issuer mi takes the k-steps of global parity mi (the same split as the
      // dequant groups) for every matrix, into accumulator half mi.
      const uint64_t bdesc0 = umma_desc_sw128(smem_u32(sB));
      const uint32_t a0 = tmem_base + (uint32_t)C::A_BASE;
      uint32_t li = 0, git = 0;
      int s = 0, sb = 0;         // A (TMEM) and activation (shared memory) stages
      uint32_t ph = 0, bph = 0;
      bool ok = true;
      for (int n = 0; ok; ++n) {
        const int item = sched_item(n);
        if (item < 0) break;
        const Item di = item_of(item);
        if (!tile_ok(args.tiles[di.tile], args)) continue;
        const int ab = li % C::AB;
        const uint32_t acc_phase = (li / C::AB) & 1;
        ++li;
        if (!mbar_wait(&acc_empty[ab], acc_phase ^ 1, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t d0 = tmem_base + (uint32_t)(ab * C::ACC_COLS + mi * BN);
        uint32_t acc = 0;
        for (int ks = di.k_lo; ks < di.k_hi; ++ks, ++git) {
          if ((git & 1u) == (uint32_t)mi) {
            if (!mbar_wait(&b_full[sb], bph, abort_flag, args.status) ||
                !mbar_wait(&op_full[s], ph, abort_flag, args.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t bd = bdesc0 + (uint64_t)(sb * (C::B_STAGE >> 4));
            const uint32_t as = a0 + (uint32_t)(s * C::A_COLS);
#pragma unroll
            for (int m = 0; m < NMAT; ++m)
              umma_bf16_ts_k64(d0 + (uint32_t)(m * 2 * BN), as + (uint32_t)(m * 32), bd, C::IDESC, acc);
            acc = 1;
            umma_commit(&op_empty[s]);
            umma_commit(&b_empty[sb]);
          }
          if (++s == C::OS) {
            s = 0;
            ph ^= 1;
          }
          if (++sb == C::OSB) {
            sb = 0;
            bph ^= 1;
          }
        }
        // (with no k-step of its parity in the item the commit arrives at once
        // and the half is never read: items have at least two k-steps)
        if (ok) umma_commit(&acc_full[ab]);
      }
      umma_commit(fin_bar);
      mbar_wait(fin_bar, 0, abort_flag, args.status);
    } else if (C::KP == 1 && lane == 0) {
      const uint64_t bdesc0 = umma_desc_sw128(smem_u32(sB));
      const uint32_t a0 = tmem_base + (uint32_t)(C::A_BASE + mi * 32);
      uint32_t li = 0;
      int s = 0, sb = 0;         // A (TMEM) and activation (shared memory) stages
      uint32_t ph = 0, bph = 0;
      bool ok = true;
      for (int n = 0; ok; ++n) {
        const int item = sched_item(n);
        if (item < 0) break;
        const Item di = item_of(item);
        if (!tile_ok(args.tiles[di.tile], args)) continue;
        const int ab = li % C::AB;
        const uint32_t acc_phase = (li / C::AB) & 1;
        ++li;  // counts valid items only, exactly like the epilogue
        if (!mbar_wait(&acc_empty[ab], acc_phase ^ 1, abort_flag, args.status)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(ab * C::ACC_COLS + mi * BN);
        const int k_lo = di.k_lo, k_hi = di.k_hi;
        for (int ks = k_lo; ks < k_hi; ++ks) {
          if (!mbar_wait(&b_full[sb], bph, abort_flag, args.status) ||
              !mbar_wait(&op_full[s], ph, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          umma_bf16_ts_k64(d, a0 + (uint32_t)(s * C::A_COLS), bdesc0 + (uint64_t)(sb * (C::B_STAGE >> 4)), C::IDESC,
                           ks != k_lo ? 1u : 0u);
          umma_commit(&op_empty[s]);
          umma_commit(&b_empty[sb]);
          if (++s == C::OS) {
            s = 0;
            ph ^= 1;
          }
          if (++sb == C::OSB) {
            sb = 0;
            bph ^= 1;
          }
        }
        if (ok) umma_commit(&acc_full[ab]);
      }
      // Quiesce the tensor pipe before TMEM is released.
      umma_commit(fin_bar);
      mbar_wait(fin_bar, 0, abort_flag, args.status);
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------- dequant ----
    // Thread dt owns weight row dt % 128 (TMEM lane = row, so warp % 4 is
    // the lane quarter) of matrix `mat`, and the k-steps of its group.
    const int dt = threadIdx.x - 128;  // 0..511
    const int row = dt & 127;
    const int sub = dt >> 7;           // 0..3
    const int mat = NMAT == 2 ? (sub & 1) : 0;
    const int grp = NMAT == 2 ? (sub >> 1) : sub;
    constexpr int NGRP = C::NGRP;
    const uint8_t* raw_mine = sRaw + mat * C::RAW_MAT + row * C::RAW_ROW;
    const uint32_t ta_mine = tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(C::A_BASE + mat * 32);
    int rs = 0, os = 0;          // ring slots of global k-step `it`, advanced incrementally
    uint32_t rph = 0, oph = 0;   // their phases
    uint32_t it = 0;
    uint32_t sbi = 0;            // scale/bias blocks finished by this warp
    bool ok = true;
    auto advance = [&](int n) {
      rs += n;
      if (rs >= C::RS) {
        rs -= C::RS;
        rph ^= 1;
      }
      os += n;
      if (os >= C::OS) {
        os -= C::OS;
        oph ^= 1;
      }
      it += n;
    };
    for (int n = 0; ok; ++n) {
      const int item = sched_item(n);
      if (item < 0) break;
      const Item d = item_of(item);
      const GemmTile t = args.tiles[d.tile];
      if (!tile_ok(t, args)) continue;
      const int64_t srow = (int64_t)t.expert * d.wstride + d.m * d.mrows + (d.pair ? mat * C::BM : 0) + row;
      // (select, not index: a runtime index into the kernel parameters would
      // copy them to local memory)
      const uint16_t* sbase = (FUSED && d.ph2) ? args.scales2 : (mat ? args.scales[1] : args.scales[0]);
      const uint16_t* bbase = (FUSED && d.ph2) ? args.biases2 : (mat ? args.biases[1] : args.biases[0]);
      const uint16_t* sp = sbase + srow * d.ksteps;
      const uint16_t* bp = bbase + srow * d.ksteps;
      // First k-step of this item that belongs to the group.
      const int k_lo = d.k_lo, k_hi = d.k_hi;
      const int first = (int)((grp - (int)(it % NGRP) + NGRP) % NGRP);
      int ks = k_lo + first;
      advance(ks < k_hi ? first : k_hi - k_lo);
      if (ks >= k_hi) continue;
      // Staged items: SB_K is a multiple of NGRP and items start at k-step 0,
      // so every group takes SB_K / NGRP k-steps of each block, the first at
      // position grp.
      const bool use_sb = item_sb(d);
      uint32_t s_nx = 0, b_nx = 0;
      if (!use_sb) {  // one k-step ahead
        s_nx = __ldg(sp + ks);
        b_nx = __ldg(bp + ks);
      }
      for (; ks < k_hi; ks += NGRP) {
        uint32_t s16 = s_nx, b16 = b_nx;
        const int kb = ks % C::SB_K;
        const int sq = sbi % C::SBS;
        if (use_sb) {
          if (kb < NGRP && !mbar_wait(&sb_full[sq], (sbi / C::SBS) & 1, abort_flag, args.status)) {
            ok = false;
            break;
          }
        } else if (ks + NGRP < k_hi) {
          s_nx = __ldg(sp + ks + NGRP);
          b_nx = __ldg(bp + ks + NGRP);
        }
        if (!mbar_wait(&raw_full[rs], rph, abort_flag, args.status)) {
          ok = false;
          break;
        }
        uint32_t wv[C::WBYTES / 4];
        {
          const uint4* src = reinterpret_cast<const uint4*>(raw_mine + rs * C::RAW_STAGE);
#pragma unroll
          for (int i = 0; i < C::WBYTES / 16; ++i) {
            const uint4 v = src[i];
            wv[4 * i + 0] = v.x;
            wv[4 * i + 1] = v.y;
            wv[4 * i + 2] = v.z;
            wv[4 * i + 3] = v.w;
          }
        }
        if (use_sb) {
          const uint16_t* sbm = reinterpret_cast<const uint16_t*>(sSB + sq * C::SB_STAGE + mat * 2 * C::SB_BOX);
          s16 = sbm[row * C::SB_K + kb];
          b16 = sbm[C::BM * C::SB_K + row * C::SB_K + kb];
        }
        uint32_t av[32];  // this thread's A row for the k-step, bf16 pairs
        if (BITS == 4) {
          const uint32_t s2w = s16 | (s16 << 16), b2w = b16 | (b16 << 16);
          const __nv_bfloat162 s2v = *reinterpret_cast<const __nv_bfloat162*>(&s2w);
          const __nv_bfloat162 b2v = *reinterpret_cast<const __nv_bfloat162*>(&b2w);
#pragma unroll
          for (int c = 0; c < 8; ++c) dequant_word4(wv[c], s2v, b2v, &av[4 * c]);
        } else {
          const float sfv = bf16_bits_to_f32((uint16_t)s16), bfv = bf16_bits_to_f32((uint16_t)b16);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 o = dequant_words8(wv[2 * c], wv[2 * c + 1], sfv, bfv);
            av[4 * c + 0] = o.x;
            av[4 * c + 1] = o.y;
            av[4 * c + 2] = o.z;
            av[4 * c + 3] = o.w;
          }
        }
        // The codes (and scale and bias) are in registers: release the raw
        // slot, and the scale/bias block after this group's last k-step in it
        // (TMA refills them through the async proxy, so order this warp's
        // generic reads first).
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&raw_empty[rs]);
        if (use_sb && kb + NGRP >= C::SB_K) {
          if (lane == 0) mbar_arrive(&sb_empty[sq]);
          ++sbi;
        }
        // Only the TMEM store needs the stage: wait for its release here, after
        // the arithmetic, so the dequantisation overlaps the MMA round trip.
        if (!mbar_wait(&op_empty[os], oph ^ 1, abort_flag, args.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st_x32(ta_mine + (uint32_t)(os * C::A_COLS), av);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&op_full[os]);
        const int step = ks + NGRP < k_hi ? NGRP : k_hi - ks;
        advance(step);
      }
    }
  } else {
    // ------------------------------------------------------- epilogue ----
    const int q = warp;  // TMEM lane quarter 0..3
    uint32_t li = 0;
    // TMEM columns per load (keeps the epilogue's registers small).
    constexpr int CW = C::KP == 2 ? 8 : 16;
    constexpr int PQ = NMAT * BN * 32;  // floats of one quarter's partial accumulators
    for (int n = 0;; ++n) {
      if (q == 0 && lane == 0) *s_cons = n;  // entries before n are finished
      const int item = sched_item(n);
      if (item < 0) break;
      const Item d = item_of(item);
      const int base = d.base, split = d.split;
      const GemmTile t = args.tiles[d.tile];
      if (!tile_ok(t, args)) continue;
      const int ab = li % C::AB;
      const uint32_t acc_phase = (li / C::AB) & 1;
      ++li;
      if (!mbar_wait(&acc_full[ab], acc_phase, abort_flag, args.status)) break;
      tc_fence_after();
      const int n_out = d.n_out;
      const int fn = d.m * d.mrows + q * 32 + lane;
      const int perm = (FUSED && d.ph2) ? 0 : args.perm_out;
      const int f = perm ? ((fn & ~7) | kperm_pos(fn & 7)) : fn;
      uint16_t* outb = (FUSED && d.ph2) ? args.out2 : args.out;
      uint16_t* outp2 = outb + (int64_t)t.row_start * n_out + fn + C::BM;  // pair mode: second row block
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * C::ACC_COLS);
      uint16_t* outp = outb + (int64_t)t.row_start * n_out + f;
      const int rows = t.row_count < BN ? t.row_count : BN;
      // Columns [c*CW, c*CW + CW) of both matrices' accumulators (halves added
      // for k-parity accumulators: half 0 + half 1, in that order).
      auto load_cols = [&](int c, float (&gv)[16], float (&uv)[16]) {
        const uint32_t tc = tbase + (uint32_t)(c * CW);
        if constexpr (C::KP == 2) {
          uint32_t r[32];
          if (NMAT == 2) tmem_ld4_x8_wait(tc, tc + BN, tc + 2 * BN, tc + 3 * BN, r);
          else tmem_ld2_x8_wait(tc, tc + BN, r);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            gv[j] = __uint_as_float(r[j]) + __uint_as_float(r[8 + j]);
            uv[j] = NMAT == 2 ? __uint_as_float(r[16 + j]) + __uint_as_float(r[24 + j]) : 0.0f;
          }
        } else {
          uint32_t g[32];
          uint32_t u[32];
          if (NMAT == 2) tmem_ld2_x16_wait(tc, tc + BN, g, u);
          else tmem_ld_x16_wait(tc, g);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            gv[j] = __uint_as_float(g[j]);
            uv[j] = NMAT == 2 ? __uint_as_float(u[j]) : 0.0f;
          }
        }
      };
      auto store = [&](int col, float gv, float uv) {
        if (NMAT == 2 && d.pair) {
          outp[(int64_t)col * n_out] = f32_to_bf16_bits(gv);
          outp2[(int64_t)col * n_out] = f32_to_bf16_bits(uv);
        } else {
          float v = gv;
          if constexpr (NMAT == 2) v = (GLU ? gelu_tanh_f32(v) : silu_f32(v)) * uv;
          outp[(int64_t)col * n_out] = f32_to_bf16_bits(v);
        }
      };
      if constexpr (SPLITK) {
        // Split-K: spill this split's accumulators, release TMEM, and let the
        // last split of the row slice (per lane quarter) finish it.
        const bool in_cap = base < args.max_split_rows;
        if (!in_cap && lane == 0) atomicCAS(args.status, 0, (int)kDevBadIndex);
        float* pq = args.partial + (((size_t)base * S + split) * 4 + q) * PQ;
#pragma unroll 1
        for (int c = 0; c < BN / CW && in_cap; ++c) {
          if (c * CW >= rows) break;
          float gv[16], uv[16];
          load_cols(c, gv, uv);
#pragma unroll
          for (int j = 0; j < CW; ++j) {
            pq[(c * CW + j) * 32 + lane] = gv[j];
            if (NMAT == 2) pq[(BN + c * CW + j) * 32 + lane] = uv[j];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[ab]);
        if (!in_cap) continue;
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          last = atomicAdd(&args.counters[base * 4 + q], 1) == S - 1;
          if (last) args.counters[base * 4 + q] = 0;  // clean for the next launch
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence();
        const float* p0 = args.partial + ((size_t)base * S * 4 + q) * PQ;
        const size_t sstride = (size_t)4 * PQ;
#pragma unroll 1
        for (int col = 0; col < rows; ++col) {
          float gv = 0.0f, uv = 0.0f;
          for (int sp_ = 0; sp_ < S; ++sp_) {
            gv += __ldcg(p0 + sp_ * sstride + col * 32 + lane);
            if (NMAT == 2) uv += __ldcg(p0 + sp_ * sstride + (BN + col) * 32 + lane);
          }
          store(col, gv, uv);
        }
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN / CW; ++c) {
        if (c * CW >= rows) break;
        float gv[16], uv[16];
        load_cols(c, gv, uv);
        const int nvalid = rows - c * CW < CW ? rows - c * CW : CW;
#pragma unroll
        for (int j = 0; j < CW; ++j)
          if (j < nvalid) store(c * CW + j, gv[j], uv[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      if constexpr (FUSED) {
        if (!d.ph2) {  // this warp's h rows of the tile are stored: count them
          __threadfence();
          __syncwarp();
          if (lane == 0) atomicAdd(args.tile_ready + d.tile, 1);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (dynamic && threadIdx.x == 0) {  // (a launch with no queued items never touches the counters)
    __threadfence();
    if (atomicAdd(&args.sched[1], 1) == (int)gridDim.x - 1) {  // last CTA: clean for the next launch
      args.sched[0] = 0;
      args.sched[1] = 0;
    }
  }
  if (warp == C::W_MMA) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace mlxr
