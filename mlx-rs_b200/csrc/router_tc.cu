// Router logits for large batches on the int8 tensor cores.
//
// The logit of token t and expert e is bf16(fp32(S) + bias[e]), where S is
// the exact dot product of the bf16 rows x[t] and wg[e] rounded once to fp32
// (exact_dot.cuh). Here S comes from integer digit planes:
//
//  * router_digits_kernel: row r (bf16) becomes an integer row X times 2^u,
//    u = (the row's largest element exponent) - 29, so |X[i]| < 2^30; bits
//    of an element below 2^u are truncated toward zero and the truncated
//    elements are counted. X is stored as four balanced base-256 int8 digit
//    planes, X = d0 2^24 + d1 2^16 + d2 2^8 + d3 with every d in [-128, 127]
//    (the Ozaki-style error-free splitting of a matrix product into exact
//    low-precision products).
//  * router_tc_kernel: per CTA 128 experts x 64 tokens. The 16 plane
//    products sum_i dw_l[i] dx_k[i] run as tcgen05.mma kind::i8 (s8 x s8 ->
//    s32, exact), added per weight 2^(8 (6 - k - l)) into 7 accumulators in
//    tensor memory (|sum| < 4 D 2^14 < 2^31 for D < 32768). The epilogue
//    forms the exact 128-bit V = sum_i X[i] W[i] and rounds V 2^(u_x + u_w)
//    to fp32. With truncated elements the true sum lies within
//    (n_x + n_w) 2^(30 + u_x + u_w) of that (n = truncated elements of each
//    row), and the logit is written when both ends of the interval give the
//    same bf16 value; otherwise, and for rows holding inf or NaN, the warp
//    computes the logit from the original rows (logit_warp: an fp64 sum with
//    its error bound, then the exact sum if that is still open). The
//    split-K form (small and mid batches) computes only the 13 products with
//    k + l <= 4 into 5 sums and bounds the other three (exact_dot.cuh); its
//    finish applies the wider interval test once per logit.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "exact_dot.cuh"
#include "gemm_launch.h"
#include "router_tc.h"

namespace mlxr {

constexpr int RG_BM = 128;                       // experts per CTA (MMA M)
constexpr int RG_BK = 64;                        // digits per k-block (one 64-byte swizzle row)
constexpr int RG_STAGES = 4;
constexpr int RG_A_PLANE = RG_BM * RG_BK;        // 8 KB
constexpr int RG_THREADS = 224;                   // warp 0 TMA, warp 1 MMA, warps 2..5 epilogue, warp 6 waiter
constexpr int RD_WARPS = 8;
// Token-tile width BN (MMA N): 64 for large batches (7 accumulators x 64 =
// 448 of the 512 tensor-memory columns), 16 for the small-batch split-K form.
template <int BN>
struct RgCfg {
  static constexpr int B_PLANE = BN * RG_BK;
  static constexpr int STAGE = 4 * RG_A_PLANE + 4 * B_PLANE;  // 48 KB (BN 64), 36 KB (BN 16)
  static constexpr int OFF_BAR = RG_STAGES * STAGE;
  static constexpr int SMEM = OFF_BAR + 128 + 1024;           // + barriers, + alignment slack
  static constexpr int TMEM_COLS = BN == 64 ? 512 : 128;
};

// bf16 rows -> digit planes dig[4][rows_pad][Dp] and info[r] = {u, n}
// (n = truncated elements, -1 when the row holds inf or NaN). Rows
// rows..rows_pad-1 and columns D..Dp-1 are written as zeros. RD_WARPS warps
// per row; D a multiple of 8, Dp a multiple of 128.
//
// Digits: for |X| < 2^30, Y = X + 0x808080 has the balanced base-256 digits
// of X in its bytes with the top bit of the three low bytes flipped
// (d_k = ((X + 2^(8k) 0x80...) >> 8k mod 256) - 128 for the low digits), so
// (X + 0x808080) ^ 0x808080 holds d3, d2, d1, d0 from the low byte up.
__device__ __forceinline__ int bf16_to_fixed(uint32_t b, int u, int& lost) {
  const int be = (int)((b >> 7) & 0xffu);
  const int mag = (int)(b & 0x7fu) | (be ? 0x80 : 0);
  const int sh = (be ? be : 1) - 134 - u;  // <= 22
  int X;
  if (sh >= 0) {
    X = mag << sh;
  } else {
    const int r = -sh < 31 ? -sh : 31;
    X = mag >> r;
    lost += (X << r) != mag;
  }
  return (b & 0x8000u) ? -X : X;
}

struct DigitRows {
  const uint16_t* src;
  int64_t rows, rows_pad;
  int8_t* dig;
  int2* info;
};

// One CTA per row of two row sets (the router rows, then the tokens).
__global__ void __launch_bounds__(RD_WARPS * 32) router_digits_kernel(DigitRows ra, DigitRows rb, int D, int Dp) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int s_top[RD_WARPS], s_nonfin[RD_WARPS], s_lost[RD_WARPS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool first = (int64_t)blockIdx.x < ra.rows_pad;
  const DigitRows& q = first ? ra : rb;
  const int64_t r = first ? (int64_t)blockIdx.x : (int64_t)blockIdx.x - ra.rows_pad;
  const uint16_t* src = q.src;
  const int64_t rows = q.rows, rows_pad = q.rows_pad;
  int8_t* dig = q.dig;
  int2* info = q.info;
  const size_t plane = (size_t)rows_pad * Dp;
  int8_t* out = dig + (size_t)r * Dp;
  const int nch = D / 8, npch = Dp / 8;
  if (r >= rows) {
    for (int c = threadIdx.x; c < npch; c += RD_WARPS * 32)
#pragma unroll
      for (int k = 0; k < 4; ++k) reinterpret_cast<uint2*>(out + k * plane)[c] = make_uint2(0u, 0u);
    if (threadIdx.x == 0) info[r] = make_int2(0, 0);
    return;
  }
  const uint4* row = reinterpret_cast<const uint4*>(src + r * (int64_t)D);
  // pass 1: the largest |bits| of the row, two halves per packed 16-bit max
  // (|bits| >= 0x7f80 means inf or NaN: such a row is flagged as a whole,
  // so those values may enter the max)
  uint32_t m2 = 0;
  for (int c = threadIdx.x; c < nch; c += RD_WARPS * 32) {
    const uint4 v = __ldg(row + c);
    m2 = __vmaxu2(m2, v.x & 0x7fff7fffu);
    m2 = __vmaxu2(m2, v.y & 0x7fff7fffu);
    m2 = __vmaxu2(m2, v.z & 0x7fff7fffu);
    m2 = __vmaxu2(m2, v.w & 0x7fff7fffu);
  }
  uint32_t mb = __reduce_max_sync(0xffffffffu, max(m2 & 0xffffu, m2 >> 16));
  uint32_t nonfin = mb >= 0x7f80u ? 1u : 0u;
  if (lane == 0) {
    s_top[warp] = (int)mb;
    s_nonfin[warp] = (int)nonfin;
  }
  __syncthreads();
  mb = 0;
  nonfin = 0;
#pragma unroll
  for (int w = 0; w < RD_WARPS; ++w) {
    mb = max(mb, (uint32_t)s_top[w]);
    nonfin |= (uint32_t)s_nonfin[w];
  }
  // exponent of the largest |element|: (be ? be : 1) - 127; u 29 below it
  const int be_max = (int)(mb >> 7);
  const int u = mb == 0 ? 0 : (be_max ? be_max : 1) - 127 - 29;
  int lost = 0;
  // Fast form: X = trunc(x 2^-u) as one fp32 multiply (exact: x 2^-u is an
  // integer of at most 30 bits, or 0, for every element that loses no bits)
  // and a truncating conversion, when 2^-u is a normal fp32 (u >= -127).
  // An element can lose bits only if its |bits| lie in (0, 128 (u + 134))
  // (exponent field below u + 134, or subnormal); a chunk holding one takes
  // the integer form, which also counts the truncated elements.
  const bool fast = u >= -127;
  const float scale = fast ? __uint_as_float((uint32_t)(127 - u) << 23) : 0.0f;
  const int thr = u + 134;
  const uint32_t lim = thr <= 0 ? 0u : (uint32_t)(thr * 128);  // <= 232 * 128 < 2^16
  const uint32_t lim2 = (lim << 16) | lim;
  for (int c = threadIdx.x; c < npch; c += RD_WARPS * 32) {
    uint32_t o[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};  // digit words of the 8 elements
    if (c < nch && !nonfin) {
      const uint4 v = __ldg(row + c);
      const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
      uint32_t cand = fast ? 0u : 1u;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t m = wd[q] & 0x7fff7fffu;
        cand |= __vcmpltu2(m, lim2) & __vcmpne2(m, 0u);
      }
      if (cand == 0u) {
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const uint32_t fb = (h & 1) ? (wd[h >> 1] & 0xffff0000u) : (wd[h >> 1] << 16);
          const int X = __float2int_rz(__uint_as_float(fb) * scale);
          o[h] = ((uint32_t)X + 0x808080u) ^ 0x808080u;
        }
      } else {
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const uint32_t b = (wd[h >> 1] >> ((h & 1) * 16)) & 0xffffu;
          o[h] = ((uint32_t)bf16_to_fixed(b, u, lost) + 0x808080u) ^ 0x808080u;
        }
      }
    }
    // plane k takes byte 3 - k of each element's word
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t sel = 3 - k;
      const uint32_t s01 = sel | ((sel + 4) << 4);  // byte sel of a, byte sel of b
      const uint32_t w01 = __byte_perm(o[0], o[1], s01), w23 = __byte_perm(o[2], o[3], s01);
      const uint32_t w45 = __byte_perm(o[4], o[5], s01), w67 = __byte_perm(o[6], o[7], s01);
      const uint2 pk = make_uint2(__byte_perm(w01, w23, 0x5410), __byte_perm(w45, w67, 0x5410));
      reinterpret_cast<uint2*>(out + k * plane)[c] = pk;
    }
  }
  lost = __reduce_add_sync(0xffffffffu, lost);
  if (lane == 0) s_lost[warp] = lost;
  __syncthreads();
  if (threadIdx.x == 0) {
    int n = 0;
#pragma unroll
    for (int w = 0; w < RD_WARPS; ++w) n += s_lost[w];
    info[r] = make_int2(u, nonfin ? -1 : n);
  }
}

// Seven 8-column TMEM loads (columns c0 + stride j .. +7, j < 7) in one wait.
__device__ inline void tmem_ld7_x8_wait(uint32_t t, uint32_t (&r)[56], uint32_t stride) {
  asm volatile(
      "{\n\t.reg .b32 t1, t2, t3, t4, t5, t6;\n\t"
      "add.u32 t1, %56, %57;\n\tadd.u32 t2, t1, %57;\n\tadd.u32 t3, t2, %57;\n\t"
      "add.u32 t4, t3, %57;\n\tadd.u32 t5, t4, %57;\n\tadd.u32 t6, t5, %57;\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%56];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8, %9, %10, %11, %12, %13, %14, %15}, [t1];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16, %17, %18, %19, %20, %21, %22, %23}, [t2];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%24, %25, %26, %27, %28, %29, %30, %31}, [t3];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%32, %33, %34, %35, %36, %37, %38, %39}, [t4];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%40, %41, %42, %43, %44, %45, %46, %47}, [t5];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%48, %49, %50, %51, %52, %53, %54, %55}, [t6];\n\t"
      "tcgen05.wait::ld.sync.aligned;\n\t}"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55])
      : "r"(t), "r"(stride)
      : "memory");
}

// Two K=32 int8 MMAs (one 64-byte k-block row) into accumulator d: A and B
// from 64-byte-swizzled K-major shared-memory tiles whose descriptors
// advance by 32 B (2 in units of 16 B) per step. The first MMA overwrites d
// when accumulate == 0.
__device__ inline void umma_i8_ss_k64(uint32_t d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                      uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t.reg .b64 a1, b1;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.b32 q, %4, %4;\n\t"
      "add.u64 a1, %1, 2;\n\tadd.u64 b1, %2, 2;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], a1, b1, %3, q;\n\t}" ::"r"(d),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand in the 64-byte
// swizzle canonical layout: rows of 64 B, 8-row atoms of 512 B
// (stride-dimension byte offset), layout type 4 = SWIZZLE_64B at bits 61-63,
// version 1 at bit 46; the leading-dimension offset is unused (1).
__device__ inline uint64_t umma_desc_sw64(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(512u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)4u << 61;
  return d;
}

// Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A s8 (7-9 = 1),
// B s8 (10-12 = 1), both K-major, N>>3 at bits 17-22, M>>4 at bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_s8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

struct RouterTcArgs {
  const uint16_t* x;
  const uint16_t* wg;
  const int2* xinfo;
  const int2* winfo;
  const float* bias;
  uint16_t* lg;
  int32_t* part;  // split-K form: [splits][kRouterSums][T][E] digit sums of each k-slice
  int64_t T;
  int E, D, nk, kps;  // k-blocks in all, per split
  int rows_pad_x, rows_pad_w;
  int* status;
};

// SPLIT: CTA (x, y, z) sums k-blocks [z kps, (z + 1) kps) and writes its 7
// digit sums per (token, expert) to part (logits_from_partials_kernel finishes);
// otherwise the epilogue forms the logits.
template <int BN, bool SPLIT>
__global__ void __launch_bounds__(RG_THREADS, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                     const RouterTcArgs a) {
  using G = RgCfg<BN>;
  // digit sums per logit: all 16 products directly; 13 in the split-K form,
  // whose finish (logits_from_partials_kernel) takes the wider interval test
  constexpr int NSUMS = SPLIT ? kRouterSums : 7;
  constexpr int RG_BN = BN;
  constexpr int RG_B_PLANE = G::B_PLANE;
  constexpr int RG_STAGE = G::STAGE;
  extern __shared__ __align__(1024) uint8_t rg_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rg_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::OFF_BAR);
  uint64_t* full = bars;                  // [RG_STAGES] digit tiles landed (TMA)
  uint64_t* empty = full + RG_STAGES;     // [RG_STAGES] stage consumed (MMA commit)
  uint64_t* acc_full = empty + RG_STAGES; // all MMAs done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* s_ready = tmem_slot + 2;  // k-blocks landed, published by the waiter warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * RG_BN, m0 = blockIdx.y * RG_BM;

  if (threadIdx.x == 0) {
    for (int i = 0; i < RG_STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    *s_ready = 0u;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, G::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w);
    prefetch_tmap(&tm_x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the digit planes and row info come from the previous kernels
  pdl_launch_dependents();
  const int kb0 = SPLIT ? (int)blockIdx.z * a.kps : 0;
  const int nkb = SPLIT ? min(a.kps, a.nk - kb0) : a.nk;  // k-blocks of this CTA (>= 1)

  if (warp == 0) {
    if (lane == 0) {
      uint32_t issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % RG_STAGES;
        const uint32_t ph = (uint32_t)(i / RG_STAGES) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.status)) break;
        uint8_t* st = smem + s * RG_STAGE;
        const int kx = (kb0 + i) * RG_BK;
        mbar_arrive_expect_tx(&full[s], RG_STAGE);
#pragma unroll
        for (int l = 0; l < 4; ++l) tma_load_2d(st + l * RG_A_PLANE, &tm_w, &full[s], kx, l * a.rows_pad_w + m0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          tma_load_2d(st + 4 * RG_A_PLANE + k * RG_B_PLANE, &tm_x, &full[s], kx, k * a.rows_pad_x + n0);
        ++issued;
      }
      drain_ring<RG_STAGES>(full, issued, abort_flag, a.status);
    }
  } else if (warp == 6) {
    // Waiter: takes the stage-landed waits off the MMA issuer (an mbarrier
    // wait in a thread with MMAs in flight lasts until they complete) and
    // publishes the count of landed k-blocks in shared memory.
    if (lane == 0) {
      for (int i = 0; i < nkb; ++i) {
        const int s = i % RG_STAGES;
        const uint32_t ph = (uint32_t)(i / RG_STAGES) & 1u;
        if (!mbar_wait(&full[s], ph, abort_flag, a.status)) break;
        asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(s_ready)), "r"((uint32_t)(i + 1))
                     : "memory");
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_s8(RG_BM, RG_BN);
      bool ok = true;
      for (int kb = 0; kb < nkb && ok; ++kb) {
        const int s = kb % RG_STAGES;
        // bounded poll of the waiter's count (plain shared-memory loads)
        const unsigned long long t0 = global_ns();
        for (uint32_t it = 1;; ++it) {
          uint32_t landed;
          asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(landed) : "r"(smem_u32(s_ready)) : "memory");
          if (landed >= (uint32_t)(kb + 1)) break;
          if ((it & 1023u) == 0) {
            if (*abort_flag) {
              ok = false;
              break;
            }
            if (global_ns() - t0 > kWaitLimitNs) {
              *abort_flag = 1;
              atomicCAS(a.status, 0, (int)kDevTimeout);
              ok = false;
              break;
            }
          }
        }
        if (!ok) break;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * RG_STAGE);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t bdesc = umma_desc_sw64(st + 4 * RG_A_PLANE + k * RG_B_PLANE);
#pragma unroll
          for (int l = 0; l < 4; ++l) {
            const int sg = k + l;
            if (sg >= NSUMS) continue;  // split-K form: the three lowest-weight products are bounded, not computed
            const int first_k = sg > 3 ? sg - 3 : 0;
            const uint32_t accum = (kb > 0 || k != first_k) ? 1u : 0u;
            umma_i8_ss_k64(tmem_base + (uint32_t)(sg * RG_BN), umma_desc_sw64(st + l * RG_A_PLANE), bdesc, idesc,
                           accum);
          }
        }
        umma_commit(&empty[s]);
      }
      // acc_full completes once every MMA issued above has completed (also
      // on abort); wait for it here too, so that no MMA is in flight when
      // the tensor memory is released.
      umma_commit(acc_full);
      mbar_wait(acc_full, 0, abort_flag, a.status);
    }
  } else {
    // Epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 = experts m0 + 32 (w % 4) + lane.
    const int q = warp & 3;
    const int e = m0 + 32 * q + lane;
    const bool e_ok = e < a.E;
    const int ec = e_ok ? e : a.E - 1;
    const int2 wi = a.winfo[ec];
    const float b = a.bias ? a.bias[ec] : 0.0f;
    bool ok = mbar_wait(acc_full, 0, abort_flag, a.status);
    tc_fence_after();
#pragma unroll 1
    for (int c8 = 0; c8 < RG_BN / 8 && ok; ++c8) {
      uint32_t r[56];
      tmem_ld7_x8_wait(tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(c8 * 8), r, RG_BN);
      uint32_t und = 0;  // bit j: this lane's logit of token j left undecided
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // unrolled: r stays in registers
        const int64_t t = n0 + c8 * 8 + j;
        const bool valid = e_ok && t < a.T;
        int32_t A[NSUMS];
#pragma unroll
        for (int g = 0; g < NSUMS; ++g) A[g] = (int32_t)r[g * 8 + j];
        if constexpr (SPLIT) {
          if (valid) {
            int32_t* pp = a.part + (((int64_t)blockIdx.z * kRouterSums) * a.T + t) * a.E + e;
#pragma unroll
            for (int g = 0; g < NSUMS; ++g) pp[(int64_t)g * a.T * a.E] = A[g];
          }
        } else {
          const int2 xi = a.xinfo[t < a.T ? t : a.T - 1];
          bool decided;
          const uint16_t lb = logit_from_digit_sums<NSUMS>(A, xi, wi, a.D, b, &decided);
          if (valid && decided) a.lg[t * a.E + e] = lb;
          und |= (uint32_t)(valid && !decided) << j;
        }
      }
      // Rare: logits the interval test left open, by the whole warp (logit_warp).
      uint32_t pend = __reduce_or_sync(0xffffffffu, und);
#pragma unroll 1
      while (pend) {
        const int j = __ffs(pend) - 1;
        pend &= pend - 1;
        const int64_t t = n0 + c8 * 8 + j;
        uint32_t need = __ballot_sync(0xffffffffu, (und >> j) & 1u);
        while (need) {
          const int src = __ffs(need) - 1;
          need &= need - 1;
          const int es = __shfl_sync(0xffffffffu, ec, src);
          const float bs = __shfl_sync(0xffffffffu, b, src);
          const uint16_t r = logit_warp(a.x + t * (int64_t)a.D, a.wg + (int64_t)es * a.D, a.D, bs, lane);
          if (lane == src) a.lg[t * a.E + e] = r;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, G::TMEM_COLS);
  }
}

RouterTcLayout router_tc_layout(int64_t T, int E, int D, size_t budget) {
  RouterTcLayout L;
  // 16-token tiles up to kRouterTcSplitMaxT tokens, else 64; the k range is
  // cut over CTAs while the tiles alone fill less than about one wave.
  L.bn = T <= kRouterTcSplitMaxT ? 16 : 64;
  L.Dp = (D + 127) / 128 * 128;
  L.rows_pad_x = (T + L.bn - 1) / L.bn * L.bn;
  L.rows_pad_w = (E + RG_BM - 1) / RG_BM * RG_BM;
  const int nk = (int)(L.Dp / RG_BK);
  const int sms = num_sms_current();
  const int64_t tiles = (L.rows_pad_x / L.bn) * (L.rows_pad_w / RG_BM);
  L.split = L.bn == 16 || tiles * 5 < (int64_t)sms * 4;
  // About one CTA per SM, at most 16 k-slices (each logit's finish reads
  // them all), fewer when the partial sums would not fit `budget`.
  int want = L.split ? (int)std::max<int64_t>(1, std::min<int64_t>(16, sms / std::max<int64_t>(tiles, 1))) : 1;
  for (;; --want) {
    L.kps = (nk + want - 1) / want;
    L.splits = L.split ? (nk + L.kps - 1) / L.kps : 1;
    size_t o = 0;
    auto take = [&](size_t bytes) {
      const size_t at = o;
      o = (o + bytes + 255) / 256 * 256;
      return at;
    };
    L.xdig = take((size_t)4 * L.rows_pad_x * L.Dp);
    L.wdig = take((size_t)4 * L.rows_pad_w * L.Dp);
    L.xinfo = take((size_t)L.rows_pad_x * sizeof(int2));
    L.winfo = take((size_t)L.rows_pad_w * sizeof(int2));
    L.part = L.split ? take((size_t)L.splits * kRouterSums * T * E * sizeof(int32_t)) : 0;
    L.total = o;
    if (L.total <= budget || want <= 1) break;
  }
  return L;
}

bool router_tc_supported(int D) { return D >= 8 && D % 8 == 0 && D < 32768; }

template <int BN, bool SPLIT>
static int launch_tc(const RouterTcLayout& L, const CUtensorMap& tw, const CUtensorMap& tx, const RouterTcArgs& a,
                     cudaStream_t st) {
  auto kern = router_tc_kernel<BN, SPLIT>;
  static std::atomic<uint64_t> attr_done{0};
  if (int rc = ensure_smem_attr(kern, RgCfg<BN>::SMEM, attr_done)) return rc;
  const dim3 grid((unsigned)(L.rows_pad_x / BN), (unsigned)(L.rows_pad_w / RG_BM), (unsigned)L.splits);
  launch_pdl(kern, grid, RG_THREADS, RgCfg<BN>::SMEM, st, tw, tx, a);
  MLXR_LAUNCH_CHECK("router_tc_kernel");
  return MLXR_CU_OK;
}

int launch_router_tc(const RouterTcProblem& p, cudaStream_t st) {
  if (!router_tc_supported(p.D))
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "router_tc: D=%d must be a multiple of 8 below 32768", p.D);
  if (p.T <= 0 || p.E <= 0) return MLXR_CU_OK;
  const RouterTcLayout L = router_tc_layout(p.T, p.E, p.D, p.budget);
  uint8_t* ws = static_cast<uint8_t*>(p.workspace);
  int8_t* xdig = reinterpret_cast<int8_t*>(ws + L.xdig);
  int8_t* wdig = reinterpret_cast<int8_t*>(ws + L.wdig);
  int2* xinfo = reinterpret_cast<int2*>(ws + L.xinfo);
  int2* winfo = reinterpret_cast<int2*>(ws + L.winfo);
  const DigitRows rw{p.wg, (int64_t)p.E, L.rows_pad_w, wdig, winfo};
  const DigitRows rx{p.x, p.T, L.rows_pad_x, xdig, xinfo};
  launch_pdl(router_digits_kernel, (unsigned)(L.rows_pad_w + L.rows_pad_x), RD_WARPS * 32, 0, st, rw, rx, p.D,
             (int)L.Dp);
  MLXR_LAUNCH_CHECK("router_digits_kernel");
  CUtensorMap tw, tx;
  if (int rc = make_map_2d(&tw, wdig, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)L.Dp, (uint64_t)4 * L.rows_pad_w,
                           RG_BK, RG_BM, CU_TENSOR_MAP_SWIZZLE_64B))
    return rc;
  if (int rc = make_map_2d(&tx, xdig, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)L.Dp, (uint64_t)4 * L.rows_pad_x,
                           RG_BK, (uint32_t)L.bn, CU_TENSOR_MAP_SWIZZLE_64B))
    return rc;
  RouterTcArgs a;
  a.x = p.x;
  a.wg = p.wg;
  a.xinfo = xinfo;
  a.winfo = winfo;
  a.bias = p.bias;
  a.lg = p.lg;
  a.part = L.split ? reinterpret_cast<int32_t*>(ws + L.part) : nullptr;
  a.T = p.T;
  a.E = p.E;
  a.D = p.D;
  a.nk = (int)(L.Dp / RG_BK);
  a.kps = L.kps;
  a.rows_pad_x = (int)L.rows_pad_x;
  a.rows_pad_w = (int)L.rows_pad_w;
  a.status = p.status;
  if (L.bn == 16) return launch_tc<16, true>(L, tw, tx, a, st);
  return L.split ? launch_tc<64, true>(L, tw, tx, a, st) : launch_tc<64, false>(L, tw, tx, a, st);
}

}  // namespace mlxr
