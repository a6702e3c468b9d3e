// CPU oracle for the Qwen 3.5/3.6 MoE block hot path (and the Gemma 4 MoE
// branch that runs on the same kernels, orc_gemma4_block).
//
// TEST INFRASTRUCTURE ONLY. This file is the checker the tests compare the
// CUDA library against; it is never linked into, called by, or shipped with
// the product library (mlx-rs_b200/libmlxr_moe.so).
//
// PARITY STATUS: unpinned against the reference's own numbers. The
// reference's arithmetic lives in MLX C++ (ml-explore/mlx v0.31.2, pinned at
// crates/mlxr-sys Cargo.toml:50-52 of the reference), which is downloaded at
// build time (crates/mlxr-sys/build.rs:141) and is not present here, so no
// MLX output can be produced in this container. The oracle restates the
// reference's dataflow op by op and is pinned against the relations its own
// tests assert (crates/mlxr/src/ops/quantization.rs:299-421,
// crates/mlxr/src/ops/arithmetic.rs:3099-3196,
// crates/mlxr-lm/src/activations.rs:341-351), reproduced in tests/.
//
// What it restates (reference file:line):
//   * block forward: crates/mlxr-lm/src/qwen3_5/text/moe.rs:116-146
//   * routed experts: crates/mlxr-lm/src/nn/switch.rs:417-474 (forward,
//     forward_with_combine, fallback), :223-234 (combine_with_weights),
//     :499-517 (gather_sort / scatter_unsort)
//   * swiglu: crates/mlxr-lm/src/activations.rs:198-200; silu
//     crates/mlxr/src/layers/activation.rs:139
//   * shared expert: crates/mlxr-lm/src/nn/swiglu_mlp.rs:63-68
//   * quantized linear: crates/mlxr/src/layers/quantized.rs:356-371
//   * op family: crates/mlxr/src/ops/quantization.rs:47-221 (quantize,
//     quantized_matmul, dequantize, gather_qmm) and gather_mm
//     crates/mlxr/src/ops/arithmetic.rs:1577-1609
//   * Gemma 4 MoE branch (orc_gemma4_block): Router::forward
//     crates/mlxr-lm/src/gemma4/text/text.rs:622-664 with router_post
//     crates/mlxr-lm/src/activations.rs:309-331, the experts input norm
//     pre_feedforward_layernorm_2 (text.rs:907-911), PackedSwitchFfn
//     crates/mlxr-lm/src/nn/switch.rs:242-345 (gate_up_proj [E, 2I, D]) with
//     GegluActivation (switch.rs:195-206; gelu_approximate
//     crates/mlxr/src/layers/activation.rs:170-174)
//
// Two block modes:
//   mode 0 "mlx-staged": rounds to bf16 at every reference op boundary
//     (logits, probs, top-k weights, each gather_qmm output, swiglu, the
//     weighted product, the k-sum, the shared branch, the final add);
//     accumulation in fp64.
//   mode 1 "fused-fp32": the CUDA kernels' contract (weights dequantised to
//     bf16, fp32 accumulation, h and y stored bf16, fp32 combine).
// Routing (router contract) is identical in both modes and bit-exact with the
// CUDA router: see route_logit / route_token below.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API extern "C" __attribute__((visibility("default")))

namespace {

// ---------------------------------------------------------------- bf16 ----
inline float bf2f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline uint16_t f2bf(float f) {  // round to nearest even
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
inline float rbf(float f) { return bf2f(f2bf(f)); }
inline float u2f(uint32_t u) {
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

enum { DT_BF16 = 0, DT_F16 = 1, DT_F32 = 2 };

inline float h2f(uint16_t h) {  // IEEE binary16 -> float
  uint32_t s = (h >> 15) & 1, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  float v;
  if (e == 0) v = std::ldexp((float)m, -24);
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp((float)(m | 0x400), (int)e - 25);
  return s ? -v : v;
}
inline uint16_t f2h(float f) {  // float -> binary16, RNE (via double path)
  uint32_t u;
  std::memcpy(&u, &f, 4);
  uint32_t s = (u >> 16) & 0x8000u;
  float a = std::fabs(f);
  if (std::isnan(f)) return (uint16_t)(s | 0x7e00);
  if (a >= 65520.0f) return (uint16_t)(s | 0x7c00);
  if (a < 6.103515625e-05f) {  // subnormal: quantum 2^-24
    float q = std::nearbyint(a * 16777216.0f);
    return (uint16_t)(s | (uint32_t)q);
  }
  int ex;
  std::frexp(a, &ex);  // a = m * 2^ex, m in [0.5,1)
  float quant = std::ldexp(1.0f, ex - 11);
  float r = std::nearbyint(a / quant) * quant;
  uint32_t e2;
  int ex2;
  float m2 = std::frexp(r, &ex2);
  e2 = (uint32_t)(ex2 - 1 + 15);
  uint32_t mant = (uint32_t)std::ldexp(m2, 11) & 0x3ffu;
  return (uint16_t)(s | (e2 << 10) | mant);
}

inline float load_as_f32(const void* p, int dt, int64_t i) {
  switch (dt) {
    case DT_BF16: return bf2f(((const uint16_t*)p)[i]);
    case DT_F16: return h2f(((const uint16_t*)p)[i]);
    default: return ((const float*)p)[i];
  }
}
inline void store_from_f32(void* p, int dt, int64_t i, float v) {
  switch (dt) {
    case DT_BF16: ((uint16_t*)p)[i] = f2bf(v); break;
    case DT_F16: ((uint16_t*)p)[i] = f2h(v); break;
    default: ((float*)p)[i] = v;
  }
}

// -------------------------------------------------------------- Philox ----
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC'11). Counter = (pair_lo, pair_hi, stream_lo,
// stream_hi), key = (seed_lo, seed_hi).
inline void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c[0];
    uint64_t p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
    uint32_t n1 = (uint32_t)p1;
    uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    uint32_t n3 = (uint32_t)p0;
    c[0] = n0; c[1] = n1; c[2] = n2; c[3] = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// Two N(0,1) samples per Philox block (Box-Muller in fp64 on 53-bit uniforms).
inline void normal_pair(uint64_t seed, uint64_t stream, uint64_t pair, double* z0, double* z1) {
  uint32_t c[4] = {(uint32_t)pair, (uint32_t)(pair >> 32), (uint32_t)stream, (uint32_t)(stream >> 32)};
  philox(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  uint64_t a = ((((uint64_t)c[0]) << 32) | c[1]) >> 11;
  uint64_t b = ((((uint64_t)c[2]) << 32) | c[3]) >> 11;
  double u1 = ((double)a + 1.0) * 0x1.0p-53;  // (0, 1]
  double u2 = (double)b * 0x1.0p-53;          // [0, 1)
  double rad = std::sqrt(-2.0 * std::log(u1));
  double th = 6.283185307179586476925286766559 * u2;
  *z0 = rad * std::cos(th);
  *z1 = rad * std::sin(th);
}

// ---------------------------------------------------- router contract ----
// exp(x) for x <= 0 shared bit-for-bit with the CUDA router: Cody & Waite
// range reduction (Cody & Waite, "Software Manual for the Elementary
// Functions", 1980) with n = rint(x*log2 e), a two-part ln 2 whose high part
// has 12 trailing zero bits, and the degree-7 Taylor polynomial of e^r in
// Horner form with explicit fmaf. Scaling by 2^n is done with exponent bits;
// results below 2^-126 take a second exact scaling so that rounding happens
// once. Every operation is an IEEE-754 round-to-nearest basic operation.
inline float exp_route(float x) {
  if (!(x > -104.0f)) return 0.0f;
  const float t = x * 0x1.715476p+0f;
  const float n = std::rint(t);
  float r = std::fma(n, -0x1.62e4p-1f, x);
  r = std::fma(n, -0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;
  p = std::fma(p, r, 0x1.6c16c2p-10f);
  p = std::fma(p, r, 0x1.111112p-7f);
  p = std::fma(p, r, 0x1.555556p-5f);
  p = std::fma(p, r, 0x1.555556p-3f);
  p = std::fma(p, r, 0x1.0p-1f);
  p = std::fma(p, r, 1.0f);
  p = std::fma(p, r, 1.0f);
  const int ni = (int)n;
  if (ni >= -126) return p * u2f((uint32_t)(ni + 127) << 23);
  const float a = p * u2f((uint32_t)(ni + 64 + 127) << 23);
  return a * 0x1.0p-64f;
}

// Round (-1)^neg * mag * 2^lsb to fp32, to nearest with ties to even, where
// mag is an n-limb little-endian unsigned integer. An exact zero gives +0; a
// nonzero value that rounds to zero keeps its sign; above the fp32 range it
// gives +-inf. Subnormal results are rounded once, at 2^-149.
float rn32_limbs(const uint64_t* mag, int n, int neg, int lsb) {
  int top = n - 1;
  while (top >= 0 && mag[top] == 0) --top;
  if (top < 0) return 0.0f;
  const int hb = top * 64 + 63 - __builtin_clzll(mag[top]);  // highest set bit
  const uint32_t sign = neg ? 0x80000000u : 0u;
  const int e = hb + lsb;  // the value lies in [2^e, 2^(e+1))
  if (e > 127) return u2f(sign | 0x7f800000u);
  int q = std::max(e - 23, -149);  // exponent of the result's last place
  const int sh = q - lsb;          // bits of mag below that place
  auto bit = [&](int i) -> uint64_t { return (i >= 0 && i < 64 * n) ? (mag[i >> 6] >> (i & 63)) & 1u : 0u; };
  uint64_t mant = 0;
  for (int i = hb; i >= std::max(sh, 0); --i) mant = (mant << 1) | bit(i);
  if (sh < 0) mant <<= -sh;
  if (sh > 0) {
    const uint64_t rb = bit(sh - 1);
    bool sticky = false;
    for (int i = sh - 2; i >= 0 && !sticky; --i) sticky = bit(i) != 0;
    if (rb && (sticky || (mant & 1u))) ++mant;
  }
  if (mant == (1ull << 24)) {
    mant >>= 1;
    ++q;
  }
  if (mant >= (1ull << 23)) {
    if (q + 23 > 127) return u2f(sign | 0x7f800000u);
    return u2f(sign | ((uint32_t)(q + 150) << 23) | ((uint32_t)mant & 0x7fffffu));
  }
  return u2f(sign | (uint32_t)mant);  // subnormal (q == -149) or zero
}

// bf16 bits -> value = m * 2^p with m a signed integer, |m| < 2^8.
inline void bf16_mp(uint16_t b, int* m, int* p) {
  const int be = (b >> 7) & 0xff, f = b & 0x7f;
  const int mag = be ? (f | 0x80) : f;
  *p = (be ? be : 1) - 134;
  *m = (b & 0x8000) ? -mag : mag;
}

// The exact dot product of two bf16 vectors rounded once to fp32. Each
// product is an integer below 2^16 times 2^(px + pw) with px + pw >= -266, so
// the positive and the negative products are summed exactly in two 576-bit
// fixed-point accumulators whose last bit weighs 2^-266. With an infinite or
// NaN operand the result is NaN when a product is NaN (NaN operand or
// inf * 0) or when products of both signs are infinite, else +-inf: the value
// of the real sum, independent of order.
float dot_bf16_rn32(const uint16_t* x, const uint16_t* w, int D) {
  constexpr int NL = 9;
  uint64_t pos[NL] = {}, neg[NL] = {};
  bool nan = false, pinf = false, ninf = false;
  for (int i = 0; i < D; ++i) {
    const uint16_t a = x[i], b = w[i];
    const bool fa = ((a >> 7) & 0xff) == 0xff, fb = ((b >> 7) & 0xff) == 0xff;
    if (fa || fb) {
      const bool na = fa && (a & 0x7f), nb = fb && (b & 0x7f);
      const bool za = (a & 0x7fff) == 0, zb = (b & 0x7fff) == 0;
      if (na || nb || (fa && zb) || (fb && za)) nan = true;
      else if (((a ^ b) & 0x8000) == 0) pinf = true;
      else ninf = true;
      continue;
    }
    int ma, pa, mb, pb;
    bf16_mp(a, &ma, &pa);
    bf16_mp(b, &mb, &pb);
    const int64_t m = (int64_t)ma * mb;
    if (m == 0) continue;
    const int at = pa + pb + 266;
    uint64_t* acc = m > 0 ? pos : neg;
    const unsigned __int128 v = (unsigned __int128)(uint64_t)(m > 0 ? m : -m) << (at & 63);
    int li = at >> 6;
    uint64_t add[2] = {(uint64_t)v, (uint64_t)(v >> 64)};
    unsigned carry = 0;
    for (int k = li; k < NL; ++k) {
      const uint64_t ad = (k - li < 2) ? add[k - li] : 0u;
      const uint64_t t = acc[k] + ad;
      const unsigned c1 = t < ad;
      const uint64_t t2 = t + carry;
      const unsigned c2 = t2 < t;
      acc[k] = t2;
      carry = c1 | c2;
      if (k - li >= 1 && carry == 0) break;
    }
  }
  if (nan || (pinf && ninf)) return u2f(0x7fc00000u);
  if (pinf) return u2f(0x7f800000u);
  if (ninf) return u2f(0xff800000u);
  int cmp = 0;
  for (int k = NL - 1; k >= 0 && cmp == 0; --k) cmp = pos[k] > neg[k] ? 1 : pos[k] < neg[k] ? -1 : 0;
  const uint64_t* big = cmp >= 0 ? pos : neg;
  const uint64_t* small = cmp >= 0 ? neg : pos;
  uint64_t mag[NL];
  unsigned borrow = 0;
  for (int k = 0; k < NL; ++k) {
    const uint64_t t = big[k] - small[k];
    const unsigned b1 = big[k] < small[k];
    mag[k] = t - borrow;
    borrow = b1 | (t < (uint64_t)borrow);
  }
  return rn32_limbs(mag, NL, cmp < 0, -266);
}

// logit(t, e) = bf16_rne( fp32(sum) + bias[e] ): sum is the exact dot
// product of x[t] and wg[e] (every product of two bf16 values is exact),
// rounded once to fp32 (nearest, ties to even); the bias is added in fp32
// and the result rounded to bf16. The reference computes the gate in bf16
// with fp32 accumulation in an order it does not specify (MLX matmul,
// moe.rs:123); rounding the exact sum makes the logit independent of
// summation order, so tensor-core and CUDA-core kernels can all produce it.
float route_logit(const uint16_t* xr, const uint16_t* wr, int D, float bias) {
  return rbf(dot_bf16_rn32(xr, wr, D) + bias);
}

// Softmax (fp32 inside, bf16 out: moe.rs:124, softmax_axis precise=true),
// top-K by (prob desc, expert asc) in place of argpartition (moe.rs:128-132,
// whose in-partition order is undefined, sort.rs:235-237), then the
// renormalisation of moe.rs:136-138 with bf16 results at each op.
// Sum order for the softmax denominator: lane j sums experts e = j, j+32, ...
// ascending, then the same xor butterfly as route_logit.
void route_token(const float* logit, int E, int K, int renorm, int32_t* idx, uint16_t* w, uint16_t* probs_out) {
  float mx = -INFINITY;
  for (int e = 0; e < E; ++e) mx = std::max(mx, logit[e]);
  std::vector<float> s(E);
  float lane[32];
  for (int j = 0; j < 32; ++j) {
    float acc = 0.0f;
    for (int e = j; e < E; e += 32) {
      s[e] = exp_route(logit[e] - mx);
      acc = acc + s[e];
    }
    lane[j] = acc;
  }
  for (int st = 16; st >= 1; st >>= 1) {
    float nv[32];
    for (int j = 0; j < 32; ++j) nv[j] = lane[j] + lane[j ^ st];
    std::memcpy(lane, nv, sizeof(lane));
  }
  const float sum = lane[0];
  std::vector<uint32_t> key(E);
  for (int e = 0; e < E; ++e) {
    uint16_t pb = f2bf(s[e] / sum);
    if (probs_out) probs_out[e] = pb;
    key[e] = ((uint32_t)pb << 16) | (uint32_t)(0xffff - e);
  }
  std::vector<uint32_t> top(K);
  std::partial_sort_copy(key.begin(), key.end(), top.begin(), top.end(), [](uint32_t a, uint32_t b) { return a > b; });
  float denom = 0.0f;
  for (int k = 0; k < K; ++k) {
    idx[k] = 0xffff - (int)(top[k] & 0xffff);
    denom = denom + bf2f((uint16_t)(top[k] >> 16));
  }
  const float dbf = rbf(denom);
  for (int k = 0; k < K; ++k) {
    const float p = bf2f((uint16_t)(top[k] >> 16));
    w[k] = renorm ? f2bf(p / dbf) : (uint16_t)(top[k] >> 16);
  }
}

// ------------------------------------------------------ affine packing ----
// Packing: element j of a uint32 word sits in bits [bits*j, bits*j + bits)
// (the [E, N, Kin*bits/32] layout pinned by quantization.rs:307).
// Quantiser (quantization.rs:47-70 -> mlx_quantize, mode "affine"; the
// converter calls it at crates/mlxr-convert/src/quantize.rs:44). The
// arithmetic is MLX's published affine quantiser (ml-explore/mlx v0.31.2,
// `affine_quantize` in mlx/ops.cpp and its CPU kernel in
// mlx/backend/cpu/quantized.cpp), restated per group of gs consecutive
// elements of a row, all in fp32:
//   n_bins = 2^bits - 1; scale = max((max - min) / n_bins, 1e-7)
//   edge = the end (min or max) of larger magnitude; the scale is negative
//     when |min| <= |max| (edge = max), positive otherwise (edge = min)
//   q0 = rint(edge / scale); if q0 != 0: scale = edge / q0, bias = edge
//     (so that 0 = scale * (-q0) + bias is exactly representable);
//     else bias = 0
//   q = clamp(rint((w - bias) / scale), 0, n_bins) from the fp32 pair,
//   and only then scale and bias are rounded to the weight dtype.
// rint rounds halves to even (MLX's CPU kernel; its Metal kernel rounds
// halves away from zero, which differs only on exact .5 quotients).
// Dequantisation: w' = fmaf(scale, q, bias) in fp32.
inline bool bits_ok(int bits) { return bits == 2 || bits == 4 || bits == 8; }
inline bool gs_ok(int gs) { return gs == 32 || gs == 64 || gs == 128; }

inline uint32_t get_code(const uint32_t* row, int64_t k, int bits) {
  const int per = 32 / bits;
  return (row[k / per] >> ((k % per) * bits)) & ((1u << bits) - 1u);
}

// Dequantise one row of length len, grouped along the row, to fp32.
void dequant_row(const uint32_t* wq, const void* s, const void* b, int sdt, int64_t srow, int64_t len, int gs, int bits,
                 float* out) {
  for (int64_t k = 0; k < len; ++k) {
    const int64_t g = srow + k / gs;
    const float sc = load_as_f32(s, sdt, g), bi = load_as_f32(b, sdt, g);
    out[k] = std::fma(sc, (float)get_code(wq, k, bits), bi);
  }
}

// fp32 dot with 16 independent partial sums (vectorisable without
// reassociation); n must be a multiple of 16.
inline float dot16(const float* a, const float* b, int64_t n) {
  float acc[16] = {0};
  for (int64_t i = 0; i < n; i += 16)
    for (int j = 0; j < 16; ++j) acc[j] += a[i + j] * b[i + j];
  float s = 0.0f;
  for (int j = 0; j < 16; ++j) s += acc[j];
  return s;
}
inline double dot64(const float* a, const float* b, int64_t n) {
  double acc[8] = {0};
  int64_t i = 0;
  for (; i + 8 <= n; i += 8)
    for (int j = 0; j < 8; ++j) acc[j] += (double)a[i + j] * (double)b[i + j];
  double s = 0.0;
  for (; i < n; ++i) s += (double)a[i] * (double)b[i];
  for (int j = 0; j < 8; ++j) s += acc[j];
  return s;
}

inline float silu(float g) { return g / (1.0f + std::exp(-g)); }
inline float sigm(float g) { return 1.0f / (1.0f + std::exp(-g)); }

int g_threads = 0;
inline int nthreads() {
#ifdef _OPENMP
  return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
  return 1;
#endif
}

}  // namespace

// ============================================================ C ABI =====

ORC_API int orc_version(void) { return 1; }

ORC_API void orc_set_threads(int n) { g_threads = n; }

ORC_API int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

// Seeded N(0, stddev^2) samples rounded to bf16 (fp64 -> fp32 -> bf16).
// Element i uses Philox pair i/2 of the given stream; even i takes the
// cosine branch, odd i the sine branch.
ORC_API void orc_normal_bf16(uint64_t seed, uint64_t stream, int64_t n, float stddev, uint16_t* out) {
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t p = 0; p < (n + 1) / 2; ++p) {
    double z0, z1;
    normal_pair(seed, stream, (uint64_t)p, &z0, &z1);
    out[2 * p] = f2bf((float)(z0 * (double)stddev));
    if (2 * p + 1 < n) out[2 * p + 1] = f2bf((float)(z1 * (double)stddev));
  }
}

ORC_API void orc_f32_to_bf16(const float* in, int64_t n, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = f2bf(in[i]);
}
ORC_API void orc_exp_route(const float* in, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = exp_route(in[i]);
}

// Row-wise exact dot products: out[r] = dot_bf16_rn32(x[r], w[r], D).
ORC_API void orc_dot_rn32(const uint16_t* x, const uint16_t* w, int64_t rows, int D, float* out) {
  for (int64_t r = 0; r < rows; ++r) out[r] = dot_bf16_rn32(x + r * D, w + r * D, D);
}

// quantize: w [rows, cols] in dtype dt -> wq [rows, cols*bits/32],
// scales/biases [rows, cols/gs] in dtype dt (quantization.rs:47-70).
ORC_API int orc_quantize(const void* w, int dt, int64_t rows, int64_t cols, int gs, int bits, uint32_t* wq, void* scales,
                         void* biases) {
  if (!bits_ok(bits) || !gs_ok(gs) || cols % gs != 0 || rows < 0) return 1;
  const int per = 32 / bits;
  const int64_t ngroups = cols / gs;
  const float nbins = (float)((1 << bits) - 1);
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t r = 0; r < rows; ++r) {
    uint32_t* qrow = wq + r * (cols / per);
    std::memset(qrow, 0, sizeof(uint32_t) * (cols / per));
    for (int64_t g = 0; g < ngroups; ++g) {
      float mn = INFINITY, mx = -INFINITY;
      for (int i = 0; i < gs; ++i) {
        const float v = load_as_f32(w, dt, r * cols + g * gs + i);
        mn = std::min(mn, v);
        mx = std::max(mx, v);
      }
      const bool min_edge = std::fabs(mn) > std::fabs(mx);
      float sc = std::max((mx - mn) / nbins, 1e-7f);
      if (!min_edge) sc = -sc;
      const float edge = min_edge ? mn : mx;
      const float q0 = std::rint(edge / sc);
      float bi = 0.0f;
      if (q0 != 0.0f) {
        sc = edge / q0;
        bi = edge;
      }
      for (int i = 0; i < gs; ++i) {
        const float v = load_as_f32(w, dt, r * cols + g * gs + i);
        const float q = std::min(std::max(std::rint((v - bi) / sc), 0.0f), nbins);
        const int64_t k = g * gs + i;
        qrow[k / per] |= ((uint32_t)q) << ((k % per) * bits);
      }
      store_from_f32(scales, dt, r * ngroups + g, sc);
      store_from_f32(biases, dt, r * ngroups + g, bi);
    }
  }
  return 0;
}

// dequantize (quantization.rs:118-146): out[r][k] = fmaf(s, q, b), stored in out_dt.
ORC_API int orc_dequantize(const uint32_t* wq, const void* s, const void* b, int sdt, int64_t rows, int64_t cols, int gs,
                           int bits, void* out, int out_dt) {
  if (!bits_ok(bits) || !gs_ok(gs) || cols % gs != 0) return 1;
  const int64_t wpr = cols * bits / 32;
#pragma omp parallel num_threads(nthreads())
  {
    std::vector<float> row(cols);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      dequant_row(wq + r * wpr, s, b, sdt, r * (cols / gs), cols, gs, bits, row.data());
      for (int64_t k = 0; k < cols; ++k) store_from_f32(out, out_dt, r * cols + k, row[k]);
    }
  }
  return 0;
}

// Dequantise matrix `mat` of a [batch, ...] packed stack to a dense fp32
// [N, K] matrix (transpose=true layout; for transpose=false the packed
// matrix is [K, N] and is returned transposed to [N, K]).
static void dense_weight(const uint32_t* wq, const void* s, const void* b, int sdt, int64_t mat, int64_t N, int64_t K,
                         int transpose, int gs, int bits, float* out) {
  if (transpose) {
    const int64_t wpr = K * bits / 32, gpr = K / gs;
    for (int64_t n = 0; n < N; ++n)
      dequant_row(wq + (mat * N + n) * wpr, s, b, sdt, (mat * N + n) * gpr, K, gs, bits, out + n * K);
  } else {
    const int64_t wpr = N * bits / 32, gpr = N / gs;
    std::vector<float> row(N);
    for (int64_t k = 0; k < K; ++k) {
      dequant_row(wq + (mat * K + k) * wpr, s, b, sdt, (mat * K + k) * gpr, N, gs, bits, row.data());
      for (int64_t n = 0; n < N; ++n) out[n * K + k] = row[n];
    }
  }
}

// gather_qmm (quantization.rs:171-221) with flattened broadcast indices:
// out[p] = x[lhs[p]] @ dequant(w[rhs[p]])^T (transpose) — x is
// [x_batch, M, K] in x_dt, out [P, M, N] fp32 (fp64 accumulation).
// lhs/rhs may be NULL meaning identity (p).
ORC_API int orc_gather_qmm(const void* x, int x_dt, int64_t x_batch, int64_t M, int64_t K, const uint32_t* wq,
                           const void* s, const void* b, int sdt, int64_t w_batch, int64_t N, const int32_t* lhs,
                           const int32_t* rhs, int64_t P, int transpose, int gs, int bits, float* out) {
  if (!bits_ok(bits) || !gs_ok(gs)) return 1;
  if ((transpose ? K : N) % gs != 0) return 1;
  for (int64_t p = 0; p < P; ++p) {
    const int64_t li = lhs ? lhs[p] : p, ri = rhs ? rhs[p] : p;
    if (li < 0 || li >= x_batch || ri < 0 || ri >= w_batch) return 2;
  }
#pragma omp parallel num_threads(nthreads())
  {
    std::vector<float> W(N * K), xr(K);
#pragma omp for schedule(dynamic)
    for (int64_t p = 0; p < P; ++p) {
      const int64_t li = lhs ? lhs[p] : p, ri = rhs ? rhs[p] : p;
      dense_weight(wq, s, b, sdt, ri, N, K, transpose, gs, bits, W.data());
      for (int64_t m = 0; m < M; ++m) {
        for (int64_t k = 0; k < K; ++k) xr[k] = load_as_f32(x, x_dt, (li * M + m) * K + k);
        for (int64_t n = 0; n < N; ++n) out[(p * M + m) * N + n] = (float)dot64(xr.data(), W.data() + n * K, K);
      }
    }
  }
  return 0;
}

// quantized_matmul (quantization.rs:81-112; QuantizedLinear::forward
// layers/quantized.rs:356-371 uses transpose=true): x [M, K] -> out [M, N].
ORC_API int orc_quantized_matmul(const void* x, int x_dt, int64_t M, int64_t K, const uint32_t* wq, const void* s,
                                 const void* b, int sdt, int64_t N, int transpose, int gs, int bits, float* out) {
  int32_t zero = 0;
  // One weight matrix, one x "batch" of M rows.
  return orc_gather_qmm(x, x_dt, 1, M, K, wq, s, b, sdt, 1, N, &zero, &zero, 1, transpose, gs, bits, out);
}

// gather_mm (arithmetic.rs:1577-1609): a [a_batch, M, K], b [b_batch, K, N]
// fp32, out [P, M, N] fp32 with fp64 accumulation.
ORC_API int orc_gather_mm(const float* a, int64_t a_batch, int64_t M, int64_t K, const float* bm, int64_t b_batch,
                          int64_t N, const int32_t* lhs, const int32_t* rhs, int64_t P, float* out) {
  for (int64_t p = 0; p < P; ++p) {
    const int64_t li = lhs ? lhs[p] : p, ri = rhs ? rhs[p] : p;
    if (li < 0 || li >= a_batch || ri < 0 || ri >= b_batch) return 2;
  }
  for (int64_t p = 0; p < P; ++p) {
    const int64_t li = lhs ? lhs[p] : p, ri = rhs ? rhs[p] : p;
    for (int64_t m = 0; m < M; ++m)
      for (int64_t n = 0; n < N; ++n) {
        double acc = 0.0;
        for (int64_t k = 0; k < K; ++k) acc += (double)a[(li * M + m) * K + k] * (double)bm[(ri * K + k) * N + n];
        out[(p * M + m) * N + n] = (float)acc;
      }
  }
  return 0;
}

// Router contract (moe.rs:123-138). x [T, D] bf16, wg [E, D] bf16,
// bias [E] fp32 or NULL. Outputs idx [T, K] int32 in rank order, w [T, K]
// bf16; logits/probs [T, E] bf16 when non-NULL.
ORC_API int orc_router(const uint16_t* x, int64_t T, int D, const uint16_t* wg, int E, const float* bias, int K,
                       int renorm, int32_t* idx, uint16_t* w, uint16_t* logits_out, uint16_t* probs_out) {
  if (D % 8 != 0 || K < 1 || K > E || E > 65535) return 1;
#pragma omp parallel num_threads(nthreads())
  {
    std::vector<float> lg(E);
#pragma omp for schedule(dynamic, 4)
    for (int64_t t = 0; t < T; ++t) {
      for (int e = 0; e < E; ++e) {
        lg[e] = route_logit(x + t * D, wg + (int64_t)e * D, D, bias ? bias[e] : 0.0f);
        if (logits_out) logits_out[t * E + e] = f2bf(lg[e]);
      }
      route_token(lg.data(), E, K, renorm, idx + t * K, w + t * K, probs_out ? probs_out + t * E : nullptr);
    }
  }
  return 0;
}

// Permutation contract (gather_sort / scatter_unsort, switch.rs:499-517):
// rows f = t*K + k are stably sorted by expert id. counts[E],
// offsets[E+1] (exclusive prefix), sorted_flat[pos] = f, inv[f] = pos.
ORC_API int orc_permute(const int32_t* idx, int64_t T, int K, int E, int32_t* counts, int32_t* offsets,
                        int32_t* sorted_flat, int32_t* inv) {
  const int64_t R = T * K;
  std::vector<int32_t> cur(E, 0);
  for (int e = 0; e < E; ++e) counts[e] = 0;
  for (int64_t f = 0; f < R; ++f) {
    if (idx[f] < 0 || idx[f] >= E) return 2;
    counts[idx[f]]++;
  }
  offsets[0] = 0;
  for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + counts[e];
  for (int64_t f = 0; f < R; ++f) {
    const int e = idx[f];
    const int32_t pos = offsets[e] + cur[e]++;
    sorted_flat[pos] = (int32_t)f;
    inv[f] = pos;
  }
  return 0;
}

// ------------------------------------------------------------- block ----
struct OrcQuant {  // one quantised linear / switch linear
  const uint32_t* w;
  const uint16_t* s;  // bf16
  const uint16_t* b;  // bf16
};

struct OrcMoeConfig {
  int hidden;            // D
  int num_experts;       // E
  int top_k;             // K
  int moe_intermediate;  // I
  int shared_intermediate;  // Is (0 = no shared expert)
  int group_size;
  int bits;
  int shared_bits;  // bits of the shared expert
  int renorm;
  int shared_gate_bits;  // bits of shared_expert_gate; 0 = shared_bits
};

struct OrcMoeWeights {
  const uint16_t* router;      // [E, D] bf16
  const float* router_bias;    // [E] or NULL
  OrcQuant gate, up, down;     // [E, I, D*b/32] / [E, D, I*b/32]
  OrcQuant sh_gate, sh_up, sh_down;  // [Is, D..] / [D, Is..]
  OrcQuant sh_expert_gate;     // [1, D*b/32]
};

// One quantised projection of rows `in` (R x Kin, fp32) by matrix `mat`
// of a switch stack [*, N, Kin]; out (R x N). fused: weights rounded to bf16
// and fp32 accumulation; staged: exact fp32 weights and fp64 accumulation.
static void proj_rows(const OrcQuant& q, int64_t mat, int64_t N, int64_t Kin, int gs, int bits, const float* in, int64_t R,
                      float* out, bool fused, std::vector<float>& Wbuf) {
  Wbuf.resize(N * Kin);
  dense_weight(q.w, q.s, q.b, DT_BF16, mat, N, Kin, 1, gs, bits, Wbuf.data());
  if (fused)
    for (auto& v : Wbuf) v = rbf(v);
  for (int64_t r = 0; r < R; ++r)
    for (int64_t n = 0; n < N; ++n)
      out[r * N + n] = fused ? dot16(in + r * Kin, Wbuf.data() + n * Kin, Kin)
                             : (float)dot64(in + r * Kin, Wbuf.data() + n * Kin, Kin);
}

// Block forward (moe.rs:116-146). mode 0 = mlx-staged, 1 = fused-fp32.
// x [T, D] bf16 -> out [T, D] bf16. idx_out [T, K], w_out [T, K] optional.
ORC_API int orc_moe_block(const OrcMoeConfig* c, const OrcMoeWeights* wt, const uint16_t* x, int64_t T, int mode,
                          uint16_t* out, int32_t* idx_out, uint16_t* w_out) {
  const int D = c->hidden, E = c->num_experts, K = c->top_k, I = c->moe_intermediate, Is = c->shared_intermediate;
  const int gs = c->group_size, bits = c->bits, sbits = c->shared_bits;
  if (D % gs || I % gs || (Is && Is % gs) || !bits_ok(bits) || !gs_ok(gs)) return 1;
  const bool fused = mode == 1;
  const int64_t R = T * K;
  std::vector<int32_t> idx(R), counts(E), offsets(E + 1), sorted(R), inv(R);
  std::vector<uint16_t> wk(R);
  int rc = orc_router(x, T, D, wt->router, E, wt->router_bias, K, c->renorm, idx.data(), wk.data(), nullptr, nullptr);
  if (rc) return rc;
  orc_permute(idx.data(), T, K, E, counts.data(), offsets.data(), sorted.data(), inv.data());
  if (idx_out) std::memcpy(idx_out, idx.data(), sizeof(int32_t) * R);
  if (w_out) std::memcpy(w_out, wk.data(), sizeof(uint16_t) * R);

  std::vector<float> xf(T * D);
  for (int64_t i = 0; i < T * D; ++i) xf[i] = bf2f(x[i]);

  // Routed experts, grouped by expert through the sorted order (the same
  // rows gather_qmm(sorted_indices=true) sees after gather_sort).
  std::vector<uint16_t> y(R * (int64_t)D);  // y for sorted row pos, bf16
#pragma omp parallel num_threads(nthreads())
  {
    std::vector<float> Wb, xin, g, u, h, yy;
#pragma omp for schedule(dynamic)
    for (int e = 0; e < E; ++e) {
      const int64_t n = counts[e], o = offsets[e];
      if (!n) continue;
      xin.resize(n * D);
      for (int64_t r = 0; r < n; ++r) std::memcpy(&xin[r * D], &xf[(sorted[o + r] / K) * D], sizeof(float) * D);
      g.resize(n * I); u.resize(n * I); h.resize(n * I); yy.resize(n * D);
      proj_rows(wt->gate, e, I, D, gs, bits, xin.data(), n, g.data(), fused, Wb);
      proj_rows(wt->up, e, I, D, gs, bits, xin.data(), n, u.data(), fused, Wb);
      for (int64_t i = 0; i < n * I; ++i) {
        if (fused) h[i] = rbf(silu(g[i]) * u[i]);
        else h[i] = rbf(silu(rbf(g[i])) * rbf(u[i]));  // gather_qmm outputs are bf16
      }
      proj_rows(wt->down, e, D, I, gs, bits, h.data(), n, yy.data(), fused, Wb);
      for (int64_t i = 0; i < n * D; ++i) y[o * D + i] = f2bf(yy[i]);
    }
  }

  // Shared branch (moe.rs:118-120; swiglu_mlp.rs:63-68).
  std::vector<float> ysh, sig;
  if (Is > 0) {
    ysh.resize(T * (int64_t)D);
    sig.resize(T);
    std::vector<float> sg(Is * (int64_t)D), su(Is * (int64_t)D), sd((int64_t)D * Is), gw(D);
    dense_weight(wt->sh_gate.w, wt->sh_gate.s, wt->sh_gate.b, DT_BF16, 0, Is, D, 1, gs, sbits, sg.data());
    dense_weight(wt->sh_up.w, wt->sh_up.s, wt->sh_up.b, DT_BF16, 0, Is, D, 1, gs, sbits, su.data());
    dense_weight(wt->sh_down.w, wt->sh_down.s, wt->sh_down.b, DT_BF16, 0, D, Is, 1, gs, sbits, sd.data());
    dense_weight(wt->sh_expert_gate.w, wt->sh_expert_gate.s, wt->sh_expert_gate.b, DT_BF16, 0, 1, D, 1, gs,
                 c->shared_gate_bits ? c->shared_gate_bits : sbits, gw.data());
    if (fused) {
      for (auto& v : sg) v = rbf(v);
      for (auto& v : su) v = rbf(v);
      for (auto& v : sd) v = rbf(v);
    }
#pragma omp parallel num_threads(nthreads())
    {
      std::vector<float> hs(Is);
#pragma omp for schedule(static)
      for (int64_t t = 0; t < T; ++t) {
        const float* xr = &xf[t * D];
        for (int i = 0; i < Is; ++i) {
          if (fused) {
            const float gg = dot16(xr, &sg[(int64_t)i * D], D), uu = dot16(xr, &su[(int64_t)i * D], D);
            hs[i] = rbf(silu(gg) * uu);
          } else {
            const float gg = rbf((float)dot64(xr, &sg[(int64_t)i * D], D));
            const float uu = rbf((float)dot64(xr, &su[(int64_t)i * D], D));
            hs[i] = rbf(silu(gg) * uu);
          }
        }
        for (int d = 0; d < D; ++d)
          ysh[t * D + d] = rbf(fused ? dot16(hs.data(), &sd[(int64_t)d * Is], Is) : (float)dot64(hs.data(), &sd[(int64_t)d * Is], Is));
        const float z = fused ? (float)dot64(xr, gw.data(), D) : rbf((float)dot64(xr, gw.data(), D));
        sig[t] = fused ? sigm(z) : rbf(sigm(z));
      }
    }
  }

  // Combine (switch.rs:223-234 / 465-474) and the final add (moe.rs:145).
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t t = 0; t < T; ++t) {
    for (int d = 0; d < D; ++d) {
      float acc = 0.0f;
      for (int k = 0; k < K; ++k) {
        const float yk = bf2f(y[(int64_t)inv[t * K + k] * D + d]);
        const float wv = bf2f(wk[t * K + k]);
        if (fused) acc += wv * yk;
        else acc += rbf(wv * yk);
      }
      float o;
      if (fused) {
        o = Is > 0 ? acc + sig[t] * ysh[t * D + d] : acc;
      } else {
        const float routed = rbf(acc);
        o = Is > 0 ? rbf(ysh[t * D + d] * sig[t]) + routed : routed;
      }
      out[t * D + d] = f2bf(o);
    }
  }
  return 0;
}

// ------------------------------------------------------------ Gemma 4 ----
// Routing contract of the Gemma 4 MoE branch (bit-exact with the CUDA
// router), restating Router::forward (gemma4/text/text.rs:622-664):
//  1. inv(t) = 1 / sqrt(ss / D + eps) in IEEE fp32, where ss is the sum of
//     x[t][d]^2 in the logit order (lane j folds chunks j, j+32, ... with
//     fmaf, then the xor butterfly): fast::rms_norm's inverse RMS.
//  2. router input  xr[d] = bf16((x[d] * inv) * wr[d]), wr = Router.scale *
//     hidden^-0.5 (pre-multiplied once, text.rs:628-639);
//     experts input xe[d] = bf16((x[d] * inv) * we[d]), we =
//     pre_feedforward_layernorm_2.weight (text.rs:907-911).
//  3. scores = route_logit(xr, Wr[e]) (no bias): the bf16 scores.
//  4. top-K by (score desc, expert asc) in place of argpartition (text.rs:
//     647-651, order undefined there).
//  5. router_post (activations.rs:325-331): softmax over the K scores
//     (max = the first; exp_route; the sum in top-K order; IEEE division;
//     bf16), times per_expert_scale[idx] (bf16 x bf16 in fp32, bf16).
float gemma4_inv_rms(const uint16_t* xr, int D, float eps) {
  float lane[32];
  const int nchunks = D / 8;
  for (int j = 0; j < 32; ++j) {
    float acc = 0.0f;
    for (int c = j; c < nchunks; c += 32)
      for (int i = 0; i < 8; ++i) {
        const float v = bf2f(xr[c * 8 + i]);
        acc = std::fma(v, v, acc);
      }
    lane[j] = acc;
  }
  for (int s = 16; s >= 1; s >>= 1) {
    float nv[32];
    for (int j = 0; j < 32; ++j) nv[j] = lane[j] + lane[j ^ s];
    std::memcpy(lane, nv, sizeof(lane));
  }
  const float ms = lane[0] / (float)D;
  return 1.0f / std::sqrt(ms + eps);
}

// Order-preserving 16-bit key of a bf16 value (larger value, larger key).
inline uint32_t bf16_order_key(uint16_t b) { return (b & 0x8000u) ? (uint32_t)(uint16_t)~b : (uint32_t)(b | 0x8000u); }

void gemma4_route_token(const uint16_t* scores, const uint16_t* expert_scale, int E, int K, int32_t* idx, uint16_t* w) {
  std::vector<uint32_t> key(E);
  for (int e = 0; e < E; ++e) key[e] = (bf16_order_key(scores[e]) << 16) | (uint32_t)(0xffff - e);
  std::vector<uint32_t> top(K);
  std::partial_sort_copy(key.begin(), key.end(), top.begin(), top.end(), [](uint32_t a, uint32_t b) { return a > b; });
  std::vector<float> ex(K);
  float mx = 0.0f, sum = 0.0f;
  for (int k = 0; k < K; ++k) {
    idx[k] = 0xffff - (int)(top[k] & 0xffff);
    const float sc = bf2f(scores[idx[k]]);
    if (k == 0) mx = sc;
    ex[k] = exp_route(sc - mx);
    sum = sum + ex[k];
  }
  for (int k = 0; k < K; ++k) w[k] = f2bf(bf2f(f2bf(ex[k] / sum)) * bf2f(expert_scale[idx[k]]));
}

// gelu_approximate (activation.rs:170): 0.5 g (1 + tanh(sqrt(2/pi) (g + 0.044715 g^3))).
inline float gelu_tanh(float g) {
  const float y = 0.7978845608028654f * (g + 0.044715f * g * g * g);
  return 0.5f * g * (1.0f + std::tanh(y));
}

struct OrcGemma4Config {
  int hidden;            // D
  int num_experts;       // E
  int top_k;             // K
  int moe_intermediate;  // I (gate_up_proj has 2I rows per expert)
  int group_size;
  int bits;
  float eps;
};

struct OrcGemma4Weights {
  const uint16_t* router;        // Router.proj [E, D] bf16
  const uint16_t* router_norm;   // [D] bf16: Router.scale * hidden^-0.5
  const uint16_t* expert_scale;  // [E] bf16: Router.per_expert_scale
  const uint16_t* experts_norm;  // [D] bf16: pre_feedforward_layernorm_2.weight
  OrcQuant gate_up;              // [E, 2I, D*b/32]
  OrcQuant down;                 // [E, D, I*b/32]
};

// Gemma 4 MoE branch in the kernels' contract (fused-fp32: weights
// dequantised to bf16, fp32 accumulation, h and y stored bf16, fp32
// combine). x [T, D] is the router input h (text.rs:901-916); out [T, D] =
// sum_k w_k * down_k(geglu(gate_up_k(pre_ff_2(h)))), before
// post_feedforward_layernorm_2. out may be NULL (routing only).
ORC_API int orc_gemma4_block(const OrcGemma4Config* c, const OrcGemma4Weights* wt, const uint16_t* x, int64_t T,
                             uint16_t* out, int32_t* idx_out, uint16_t* w_out) {
  const int D = c->hidden, E = c->num_experts, K = c->top_k, I = c->moe_intermediate;
  const int gs = c->group_size, bits = c->bits;
  if (D % 8 || D % gs || I % gs || !bits_ok(bits) || !gs_ok(gs) || K < 1 || K > E || E > 0xffff) return 1;
  const int64_t R = T * K;
  std::vector<int32_t> idx(R), counts(E), offsets(E + 1), sorted(R), inv(R);
  std::vector<uint16_t> wk(R), xe((size_t)T * D);
#pragma omp parallel num_threads(nthreads())
  {
    std::vector<uint16_t> xr(D), sc(E);
#pragma omp for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
      const uint16_t* xt = x + t * D;
      const float iv = gemma4_inv_rms(xt, D, c->eps);
      for (int d = 0; d < D; ++d) {
        const float a = bf2f(xt[d]) * iv;
        xr[d] = f2bf(a * bf2f(wt->router_norm[d]));
        xe[t * D + d] = f2bf(a * bf2f(wt->experts_norm[d]));
      }
      for (int e = 0; e < E; ++e) sc[e] = f2bf(route_logit(xr.data(), wt->router + (int64_t)e * D, D, 0.0f));
      gemma4_route_token(sc.data(), wt->expert_scale, E, K, &idx[t * K], &wk[t * K]);
    }
  }
  if (idx_out) std::memcpy(idx_out, idx.data(), sizeof(int32_t) * R);
  if (w_out) std::memcpy(w_out, wk.data(), sizeof(uint16_t) * R);
  if (!out) return 0;
  orc_permute(idx.data(), T, K, E, counts.data(), offsets.data(), sorted.data(), inv.data());

  std::vector<uint16_t> y(R * (int64_t)D);
#pragma omp parallel num_threads(nthreads())
  {
    std::vector<float> Wb, xin, gu, h, yy;
#pragma omp for schedule(dynamic)
    for (int e = 0; e < E; ++e) {
      const int64_t n = counts[e], o = offsets[e];
      if (!n) continue;
      xin.resize(n * D);
      for (int64_t r = 0; r < n; ++r)
        for (int d = 0; d < D; ++d) xin[r * D + d] = bf2f(xe[(sorted[o + r] / K) * D + d]);
      gu.resize(n * 2 * I); h.resize(n * I); yy.resize(n * D);
      proj_rows(wt->gate_up, e, 2 * I, D, gs, bits, xin.data(), n, gu.data(), true, Wb);
      for (int64_t r = 0; r < n; ++r)
        for (int i = 0; i < I; ++i) h[r * I + i] = rbf(gelu_tanh(gu[r * 2 * I + i]) * gu[r * 2 * I + I + i]);
      proj_rows(wt->down, e, D, I, gs, bits, h.data(), n, yy.data(), true, Wb);
      for (int64_t i = 0; i < n * D; ++i) y[o * D + i] = f2bf(yy[i]);
    }
  }
#pragma omp parallel for schedule(static) num_threads(nthreads())
  for (int64_t t = 0; t < T; ++t)
    for (int d = 0; d < D; ++d) {
      float acc = 0.0f;
      for (int k = 0; k < K; ++k) acc += bf2f(wk[t * K + k]) * bf2f(y[(int64_t)inv[t * K + k] * D + d]);
      out[t * D + d] = f2bf(acc);
    }
  return 0;
}
