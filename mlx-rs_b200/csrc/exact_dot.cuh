// Exact dot products of bf16 vectors rounded once to fp32: the router
// logit's sum (logit = bf16(fp32(sum x_i * w_i) + bias)). The product of two
// bf16 values is exact, so the sum has one defined value whatever the
// summation order; every router kernel produces its correctly rounded fp32
// value (round to nearest, ties to even; an exact zero is +0).
//
//  * rn32_limbs: round a multi-limb integer times a power of two to fp32.
//  * dot_rn32_warp: the exact sum by one warp with fixed-point limb
//    accumulators (the fallback when a faster path cannot decide the result).
//  * logit_from_f64: the bf16 logit when the sum is only known to lie in an
//    interval; it is decided when both ends give the same bf16 value,
//    since fp32 rounding, the fp32 bias add and bf16 rounding are all
//    monotone non-decreasing.
//  * rn32_i128: the rounding of an exact integer sum (the tensor-core path).
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace mlxr {

// Round (-1)^neg * mag * 2^lsb to fp32, nearest-even. mag: n little-endian
// 64-bit limbs. Exact zero -> +0; a nonzero value that rounds to zero keeps
// its sign; overflow -> +-inf; subnormal results are rounded once at 2^-149.
__device__ inline float rn32_limbs(const uint64_t* mag, int n, int neg, int lsb) {
  int top = n - 1;
  while (top >= 0 && mag[top] == 0) --top;
  if (top < 0) return 0.0f;
  const int hb = top * 64 + 63 - __clzll((long long)mag[top]);
  const uint32_t sign = neg ? 0x80000000u : 0u;
  const int e = hb + lsb;
  if (e > 127) return __uint_as_float(sign | 0x7f800000u);
  int q = e - 23 < -149 ? -149 : e - 23;
  const int sh = q - lsb;  // bits of mag below the result's last place
  auto bits_at = [&](int pos) -> uint64_t {  // 64 bits of mag starting at bit pos (pos >= 0)
    const int li = pos >> 6, off = pos & 63;
    uint64_t v = li < n ? mag[li] >> off : 0u;
    if (off && li + 1 < n) v |= mag[li + 1] << (64 - off);
    return v;
  };
  uint64_t mant;
  if (sh <= 0) {
    mant = mag[0] << (-sh);  // the value is below 2^24 units of 2^q: one limb, exact
  } else {
    mant = bits_at(sh) & ((1ull << 25) - 1);
    const uint64_t rb = (bits_at(sh - 1)) & 1u;
    bool sticky = false;
    const int below = sh - 1;  // bits [0, below) are the sticky bits
    for (int li = 0; li < n && li * 64 < below && !sticky; ++li) {
      const int nb = below - li * 64;
      const uint64_t m = nb >= 64 ? ~0ull : ((1ull << nb) - 1);
      sticky = (mag[li] & m) != 0;
    }
    if (rb && (sticky || (mant & 1u))) ++mant;
  }
  if (mant == (1ull << 24)) {
    mant >>= 1;
    ++q;
  }
  if (mant >= (1ull << 23)) {
    if (q + 23 > 127) return __uint_as_float(sign | 0x7f800000u);
    return __uint_as_float(sign | ((uint32_t)(q + 150) << 23) | ((uint32_t)mant & 0x7fffffu));
  }
  return __uint_as_float(sign | (uint32_t)mant);
}

// bf16 logit of a sum s (fp32 already): bf16(s + bias).
__device__ __forceinline__ uint16_t logit_bits(float s, float bias) { return f32_to_bf16_bits(__fadd_rn(s, bias)); }

// The exact sum of x[i] * w[i] over i < D by the whole warp (every lane
// calls it with the same arguments; every lane gets the result). Lane j
// takes elements j, j+32, ...: each product m * 2^p (|m| < 2^16,
// p >= -266) is added into the lane's positive or negative 576-bit
// accumulator (last bit 2^-266); the accumulators are summed across the
// warp with carries, and the difference is rounded once. Infinite or NaN
// operands give NaN (a NaN product, or infinite products of both signs) or
// +-inf, as the real sum would.
static __device__ __noinline__ float dot_rn32_warp(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, int D,
                                           int lane) {
  constexpr int NL = 9;
  uint64_t pos[NL], neg[NL];
#pragma unroll
  for (int k = 0; k < NL; ++k) pos[k] = neg[k] = 0u;
  uint32_t cls = 0;  // bit 0: NaN product, bit 1: +inf product, bit 2: -inf product
  for (int i = lane; i < D; i += 32) {
    const uint32_t a = x[i], b = w[i];
    const bool fa = ((a >> 7) & 0xffu) == 0xffu, fb = ((b >> 7) & 0xffu) == 0xffu;
    if (fa || fb) {
      const bool na = fa && (a & 0x7fu), nb = fb && (b & 0x7fu);
      const bool za = (a & 0x7fffu) == 0, zb = (b & 0x7fffu) == 0;
      if (na || nb || (fa && zb) || (fb && za)) cls |= 1u;
      else cls |= (((a ^ b) & 0x8000u) == 0) ? 2u : 4u;
      continue;
    }
    const int bea = (a >> 7) & 0xff, beb = (b >> 7) & 0xff;
    const uint32_t ma = bea ? ((a & 0x7fu) | 0x80u) : (a & 0x7fu);
    const uint32_t mb = beb ? ((b & 0x7fu) | 0x80u) : (b & 0x7fu);
    const uint64_t m = (uint64_t)(ma * mb);
    if (m == 0) continue;
    const int at = ((bea ? bea : 1) - 134) + ((beb ? beb : 1) - 134) + 266;
    uint64_t* acc = ((a ^ b) & 0x8000u) ? neg : pos;
    const int li = at >> 6, off = at & 63;
    const uint64_t lo = m << off, hi = off ? (m >> (64 - off)) : 0u;
    uint64_t t = acc[li] + lo;
    uint32_t c = t < lo;
    acc[li] = t;
    if (li + 1 < NL) {
      const uint64_t t1 = acc[li + 1] + hi;
      const uint32_t c1 = t1 < hi;
      acc[li + 1] = t1 + c;
      c = c1 | (acc[li + 1] < t1);
      for (int k = li + 2; k < NL && c; ++k) {
        acc[k] += 1u;
        c = acc[k] == 0u;
      }
    }
  }
  cls = __reduce_or_sync(0xffffffffu, cls);
  if (cls & 1u || (cls & 6u) == 6u) return __uint_as_float(0x7fc00000u);
  if (cls & 2u) return __uint_as_float(0x7f800000u);
  if (cls & 4u) return __uint_as_float(0xff800000u);
  // Sum the accumulators over the warp (xor butterfly; every lane ends with the total).
#pragma unroll 1
  for (int s = 16; s >= 1; s >>= 1) {
    uint32_t cp = 0, cn = 0;
#pragma unroll
    for (int k = 0; k < NL; ++k) {
      const uint64_t op = __shfl_xor_sync(0xffffffffu, pos[k], s);
      const uint64_t on = __shfl_xor_sync(0xffffffffu, neg[k], s);
      const uint64_t tp = pos[k] + op, tn = neg[k] + on;
      const uint32_t c1p = tp < op, c1n = tn < on;
      pos[k] = tp + cp;
      neg[k] = tn + cn;
      cp = c1p | (pos[k] < tp);
      cn = c1n | (neg[k] < tn);
    }
  }
  int cmp = 0;
#pragma unroll
  for (int k = NL - 1; k >= 0; --k)
    if (cmp == 0) cmp = pos[k] > neg[k] ? 1 : (pos[k] < neg[k] ? -1 : 0);
  uint64_t mag[NL];
  uint32_t borrow = 0;
#pragma unroll
  for (int k = 0; k < NL; ++k) {
    const uint64_t big = cmp >= 0 ? pos[k] : neg[k], small = cmp >= 0 ? neg[k] : pos[k];
    const uint64_t t = big - small;
    const uint32_t b1 = big < small;
    mag[k] = t - borrow;
    borrow = b1 | (t < (uint64_t)borrow);
  }
  return rn32_limbs(mag, NL, cmp < 0, -266);
}

// fp32 rounding of a signed 128-bit integer times 2^lsb. Fast path: shift
// the magnitude right by k so that it fits 63 bits, folding the shifted-out
// bits into bit 0 (a sticky bit: with 39 or more bits below the fp32
// rounding position this keeps "below / at / above half" intact), convert
// with the hardware's correctly rounded int64 -> fp32, and scale by
// 2^(k + lsb) through the exponent field when the result is a normal number
// (exponent field 2..254, so the exact value was normal too).
__device__ __forceinline__ float rn32_i128(__int128 v, int lsb) {
  const bool neg = v < 0;
  const unsigned __int128 mag = neg ? (unsigned __int128)(-v) : (unsigned __int128)v;
  if (mag == 0) return 0.0f;
  const uint64_t hi = (uint64_t)(mag >> 64), lo = (uint64_t)mag;
  const int nbits = hi ? 128 - __clzll((long long)hi) : 64 - __clzll((long long)lo);
  const int k = nbits > 63 ? nbits - 63 : 0;
  uint64_t m;
  if (k == 0) {
    m = lo;
  } else {
    const unsigned __int128 sh = mag >> k;
    const unsigned __int128 lost = mag & ((((unsigned __int128)1) << k) - 1);
    m = (uint64_t)sh | (lost != 0 ? 1u : 0u);
  }
  const float f = __ll2float_rn((long long)m);
  const uint32_t fb = __float_as_uint(f);
  const int ex = (int)((fb >> 23) & 0xffu) + k + lsb;
  if (ex >= 2 && ex <= 254) return __uint_as_float((neg ? 0x80000000u : 0u) | (fb & 0x007fffffu) | ((uint32_t)ex << 23));
  const uint64_t limbs[2] = {lo, hi};
  return rn32_limbs(limbs, 2, neg, lsb);
}

// The bf16 logit of a sum known to lie within err of s (fp64): decided when
// both ends of [s - err, s + err] give the same logit. Returns false when
// the interval straddles a rounding boundary or s is not finite.
__device__ __forceinline__ bool logit_from_f64(double s, double err, float bias, uint16_t* out) {
  if (!isfinite(s) || !isfinite(err)) return false;
  const uint16_t a = logit_bits(__double2float_rn(__dsub_rd(s, err)), bias);
  const uint16_t b = logit_bits(__double2float_rn(__dadd_ru(s, err)), bias);
  *out = a;
  return a == b;
}

// The tensor-core router's digit sums: the plane products of digits k
// (token) and l (router row) are added per weight 2^(8 (6 - k - l)) into
// NS sums A[g], g = k + l < NS. NS = 7 keeps all 16 products; NS = 5 (the
// split-K form) drops the three with k + l = 5, 6, which add up to at most
// D (2 * 2^14 * 2^8 + 2^14) units of the last digit pair (every balanced
// digit is at most 128 in magnitude), and that bound joins the interval test.
constexpr int kRouterSums = 5;  // the split-K form's sums per logit

// Both ends of [V - B, V + B] give the logit lb (not inlined: it is called
// from unrolled loops).
static __device__ __noinline__ bool digit_interval_same(__int128 V, __int128 B, int lsb, float bias, uint32_t lb) {
  return logit_bits(rn32_i128(V - B, lsb), bias) == lb && logit_bits(rn32_i128(V + B, lsb), bias) == lb;
}

// The bf16 logit from the digit sums: V = sum_g A[g] 2^(8 (6 - g)), and the
// sum lies within B 2^(u_x + u_w) of V 2^(u_x + u_w), B = (n_x + n_w) 2^30
// (a truncated element adds at most 2^30 units; xi, wi = {u, truncated
// count}) plus D (2^23 + 2^14) when NS = 5. *decided is false when that
// interval straddles a bf16 logit boundary or a row holds inf or NaN (count
// -1): the caller then computes the exact sum.
template <int NS>
__device__ __forceinline__ uint16_t logit_from_digit_sums(const int32_t (&A)[NS], int2 xi, int2 wi, int D, float bias,
                                                          bool* decided) {
  static_assert(NS == 5 || NS == 7, "5 or 7 digit sums");
  *decided = false;
  if (xi.y < 0 || wi.y < 0) return 0;
  const int64_t hi = (int64_t)A[0] * (1ll << 24) + (int64_t)A[1] * (1ll << 16) + (int64_t)A[2] * (1ll << 8) + A[3];
  int64_t lo = (int64_t)A[4] * (1ll << 16);
  if constexpr (NS == 7) lo += (int64_t)A[5] * (1ll << 8) + A[6];
  const __int128 V = ((__int128)hi << 24) + (__int128)lo;
  const int lsb = xi.x + wi.x;
  if constexpr (NS == 5) {
    // First in fp64 (the three 128-bit roundings below cost more): |V| <
    // 2^80, so (V >> 32) 2^32 is exact and adding the low 32 bits rounds
    // once (relative error <= 2^-53); 2^lsb (lsb in [-310, 196]) scales
    // exactly. The sum lies within B 2^lsb + 2^-52 |s| of s, both rounded up.
    const double v = __dadd_rn(__ll2double_rn((long long)(V >> 32)) * 4294967296.0, (double)(uint32_t)V);
    const double p2 = __hiloint2double((lsb + 1023) << 20, 0);
    const double s = v * p2;
    const long long Bd = (long long)(xi.y + wi.y) * (1ll << 30) + (long long)D * ((1ll << 23) + (1ll << 14));
    const double err = __dadd_ru(__dmul_ru(__ll2double_ru(Bd), p2), __dmul_ru(fabs(s), 0x1p-52));
    uint16_t lf;
    if (logit_from_f64(s, err, bias, &lf)) {
      *decided = true;
      return lf;
    }
  }
  const uint16_t lb = logit_bits(rn32_i128(V, lsb), bias);
  __int128 B = (__int128)(xi.y + wi.y) * (1ll << 30);
  if constexpr (NS == 5) B += (__int128)D * ((1ll << 23) + (1ll << 14));
  *decided = B == 0 || digit_interval_same(V, B, lsb, bias, lb);
  return lb;
}

// bf16 (the low 16 bits of b) -> fp64, exact for every finite value: the
// bf16 exponent and fraction bits placed at the bottom of the fp64 exponent
// and the top of its fraction give the value times 2^-896 (a subnormal fp64
// for bf16 subnormals), and the power-of-two scale restores it exactly. inf
// and NaN come out finite (>= 2^128 in magnitude); callers detect them from
// the largest |bits| of the row (>= 0x7f80).
__device__ __forceinline__ double bf16_to_f64(uint32_t b) {
  const uint32_t hi = ((b & 0x7fffu) << 13) | ((b & 0x8000u) << 16);
  return __hiloint2double((int)hi, 0) * 0x1.0p+896;
}

// Error bound of an fp64 sum of D exact products that each went through at
// most `depth` roundings: |s - S| <= gamma_depth * sum|x_i w_i| with
// gamma_depth = depth 2^-53 / (1 - depth 2^-53), and sum|x_i w_i| <=
// D max|x| max|w|. mx, mw: the largest |bf16 bits| of each row (finite).
// The factor (depth + 8) 2^-52 covers gamma and the roundings of this bound.
__device__ __forceinline__ double f64_sum_err(int depth, int D, uint32_t mx, uint32_t mw) {
  const double f = (double)(depth + 8) * 0x1.0p-52 * (double)D;
  return __dmul_ru(__dmul_ru(f, bf16_to_f64(mx)), bf16_to_f64(mw));
}

// Class of the product a * b of two bf16 values (bits): 0 when both are
// finite, else bit 0 for NaN (a NaN operand, or inf times 0), bit 1 for
// +inf, bit 2 for -inf. A sum holding any non-finite product is NaN when a
// NaN product or infinite products of both signs occur, else the infinity
// of their sign (class_sum).
__device__ __forceinline__ uint32_t product_class(uint32_t a, uint32_t b) {
  const bool fa = (a & 0x7f80u) == 0x7f80u, fb = (b & 0x7f80u) == 0x7f80u;
  if (!(fa || fb)) return 0u;
  const bool na = fa && (a & 0x7fu), nb = fb && (b & 0x7fu);
  const bool za = (a & 0x7fffu) == 0, zb = (b & 0x7fffu) == 0;
  if (na || nb || (fa && zb) || (fb && za)) return 1u;
  return (((a ^ b) & 0x8000u) == 0) ? 2u : 4u;
}

__device__ __forceinline__ float class_sum(uint32_t cls) {
  if (cls & 1u || (cls & 6u) == 6u) return __uint_as_float(0x7fc00000u);
  return (cls & 2u) ? __uint_as_float(0x7f800000u) : __uint_as_float(0xff800000u);
}

// One pass of the whole warp over x . w (D % 8 == 0, both rows 16-byte
// aligned): lane j takes the 16-byte chunks j, j + 32, ..., two in flight,
// and returns (every lane) the fp64 sum of the exact products (one rounding
// per element, then an xor butterfly: depth 8 ceil(D / 256) + 5), the
// rows' largest |bf16 bits| and the OR of the product classes.
__device__ __forceinline__ double dot_f64_warp(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, int D,
                                               int lane, uint32_t* mx_out, uint32_t* mw_out, uint32_t* cls_out) {
  const int nch = D / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  double acc = 0.0;
  uint32_t mx = 0, mw = 0, cls = 0;
  for (int c0 = lane; c0 < nch; c0 += 64) {
    uint4 xv[2], wv[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = c0 + 32 * u;
      xv[u] = c < nch ? __ldg(xr + c) : make_uint4(0u, 0u, 0u, 0u);
      wv[u] = c < nch ? __ldg(wr + c) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint32_t xa[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w}, wa[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t a = h ? (xa[q] >> 16) : (xa[q] & 0xffffu);
          const uint32_t b = h ? (wa[q] >> 16) : (wa[q] & 0xffffu);
          mx = max(mx, a & 0x7fffu);
          mw = max(mw, b & 0x7fffu);
          cls |= product_class(a, b);
          acc = __fma_rn(bf16_to_f64(a), bf16_to_f64(b), acc);  // zero padding adds exactly 0
        }
    }
  }
  *mx_out = __reduce_max_sync(0xffffffffu, mx);
  *mw_out = __reduce_max_sync(0xffffffffu, mw);
  *cls_out = __reduce_or_sync(0xffffffffu, cls);
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, s));
  return acc;
}

// x . w by the whole warp when a row holds inf or NaN: every such element
// makes its product inf or NaN, so the element classes alone decide the sum
// (no limb sums). D % 8 == 0, both rows 16-byte aligned.
static __device__ __noinline__ float dot_nonfinite_warp(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                        int D, int lane) {
  uint32_t mx, mw, cls;
  (void)dot_f64_warp(x, w, D, lane, &mx, &mw, &cls);
  return class_sum(cls);
}

// The exact logit when the fp64 interval was not enough: the class pass for
// rows holding inf or NaN (mx, mw: the rows' largest |bf16 bits|), else the
// limb sum. Warp-uniform arguments; D % 8 == 0, rows 16-byte aligned.
__device__ __forceinline__ uint16_t logit_exact_warp(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                     int D, float bias, uint32_t mx, uint32_t mw, int lane) {
  const float v = (mx >= 0x7f80u || mw >= 0x7f80u) ? dot_nonfinite_warp(x, w, D, lane) : dot_rn32_warp(x, w, D, lane);
  return logit_bits(v, bias);
}

// The bf16 logit of x . w + bias by the whole warp (every lane calls it with
// the same arguments and gets the result), for logits an interval test left
// open: one dot_f64_warp pass decides rows holding inf or NaN from the
// product classes and the others from the fp64 interval (the bound of
// f64_sum_err); only when that interval also straddles a rounding boundary
// the exact sum (dot_rn32_warp, whose limb accumulators cost ~30 us per
// call at D = 4096 against ~1 us for this pass). D % 8 == 0, both rows
// 16-byte aligned.
static __device__ __noinline__ uint16_t logit_warp(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                   int D, float bias, int lane) {
  uint32_t mx, mw, cls;
  const double s = dot_f64_warp(x, w, D, lane, &mx, &mw, &cls);
  if (cls) return logit_bits(class_sum(cls), bias);
  uint16_t lb;
  if (logit_from_f64(s, f64_sum_err(8 * ((D / 8 + 31) / 32) + 5, D, mx, mw), bias, &lb)) return lb;
  return logit_bits(dot_rn32_warp(x, w, D, lane), bias);
}

}  // namespace mlxr
