// Router, permutation and combine kernels of the MoE block.
//
// Router (Qwen35MoeBlock::forward, crates/mlxr-lm/src/qwen3_5/text/moe.rs:123-138):
// logits = x @ gate^T rounded to bf16, softmax (fp32 inside, bf16 out),
// top-K, renormalisation. The reference's argpartition leaves the order of
// equal probabilities undefined (crates/mlxr/src/ops/sort.rs:235-237); this
// implementation fixes the routing contract so that CPU and GPU agree bit for
// bit:
//   * logit(t, e) = bf16(fp32(S) + bias[e]), S the exact dot product of the
//     bf16 rows x[t] and gate[e] rounded once to fp32 (exact_dot.cuh): the
//     same value in whatever order a kernel sums, so the fp64 kernels below
//     and the int8 tensor-core kernels (router_tc.cu) all produce it.
//   * softmax: exact max, exp_route(l - max), lane sums over e = j, j+32, ...
//     then the same butterfly, IEEE division, bf16 probabilities.
//   * top-K by (probability desc, expert asc); denominator summed in rank
//     order; weights = bf16(p / bf16(denominator)).
// Permutation (gather_sort / scatter_unsort, crates/mlxr-lm/src/nn/switch.rs:
// 499-517): the flat rows f = t*K + k are stably sorted by expert (a counting
// sort: per-block histograms, one scan, stable in-block ranks by
// __match_any_sync; one CTA does all of it when the rows fit one block); a
// wide gather then builds the expert-sorted copy of x with 16-byte loads.
// Combine (combine_with_weights, switch.rs:223-234, plus the shared branch
// and final add, moe.rs:118-120,145): out[t] = sum_k w[t,k] * y[inv[t*K+k]]
// (+ sigmoid(x . g_s) * shared(x)), fp32 accumulation, one bf16 rounding.
#pragma once

#include "common.cuh"
#include "exact_dot.cuh"
#include "grouped_gemm.cuh"

namespace mlxr {

// exp for x <= 0 under the routing contract (Cody & Waite range reduction,
// degree-7 Taylor polynomial of e^r in Horner form with explicit fma, exact
// power-of-two scaling). Every step is an IEEE-754 round-to-nearest basic
// operation, so the host oracle reproduces it bit for bit.
__device__ inline float exp_route(float x) {
  if (!(x > -104.0f)) return 0.0f;
  const float t = __fmul_rn(x, 0x1.715476p+0f);
  const float n = rintf(t);
  float r = __fmaf_rn(n, -0x1.62e4p-1f, x);
  r = __fmaf_rn(n, -0x1.7f7d1cp-20f, r);
  float p = 0x1.a01a02p-13f;
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
  p = __fmaf_rn(p, r, 0x1.111112p-7f);
  p = __fmaf_rn(p, r, 0x1.555556p-5f);
  p = __fmaf_rn(p, r, 0x1.555556p-3f);
  p = __fmaf_rn(p, r, 0x1.0p-1f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = (int)n;
  if (ni >= -126) return __fmul_rn(p, __uint_as_float((uint32_t)(ni + 127) << 23));
  const float a = __fmul_rn(p, __uint_as_float((uint32_t)(ni + 64 + 127) << 23));
  return __fmul_rn(a, 0x1.0p-64f);
}

__device__ inline float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ inline float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// ------------------------------------------------------------ router ---
constexpr int RT_MAX_EXPERTS = 1024;  // routing lane arrays cover up to 32 groups of 32
constexpr int RT_MAXK = 32;

struct SharedGateArgs {
  const uint32_t* w;   // [1, D*bits/32]
  const uint16_t* s;   // [1, D/64]
  const uint16_t* b;
  int bits;
};

// Softmax + top-K + renormalisation of one token by one warp, from its bf16
// logits held as floats in shared memory (lrow[0..E)).
// Order-preserving 16-bit key of a bf16 value (larger value, larger key).
__device__ inline uint32_t bf16_order_key(uint32_t b) { return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u); }

// Gemma 4 routing of one token by one warp from its bf16 scores (router_post,
// crates/mlxr-lm/src/activations.rs:325-331, after the top-k of
// gemma4/text/text.rs:647-651): top-K by (score desc, expert asc); softmax
// over the K picked scores (max = the first pick, exp_route, the sum in pick
// order, IEEE division, bf16); times per_expert_scale[e] (bf16).
// MV: groups of 32 experts the lane arrays cover (MV * 32 >= E); sized per
// batch so that they stay in registers.
template <int MV>
__device__ inline void route_token_warp_gemma4(const float* lrow, int64_t t, int E, int K, int lane,
                                               int32_t* __restrict__ idx_out, uint16_t* __restrict__ w_out,
                                               const uint16_t* __restrict__ expert_scale) {
  constexpr int RT_MAXV = MV;
  uint32_t key[RT_MAXV];
#pragma unroll
  for (int m = 0; m < RT_MAXV; ++m) {
    const int e = lane + 32 * m;
    key[m] = e < E ? (bf16_order_key(f32_to_bf16_bits(lrow[e])) << 16) | (uint32_t)(0xFFFF - e) : 0u;
  }
  int my_e = 0;
  float my_x = 0.0f, mx = 0.0f, denom = 0.0f;
  for (int k = 0; k < K; ++k) {
    uint32_t best = 0u;
#pragma unroll
    for (int m = 0; m < RT_MAXV; ++m) best = best > key[m] ? best : key[m];
    best = __reduce_max_sync(0xffffffffu, best);
    const int e = 0xFFFF - (int)(best & 0xFFFFu);
    const float sc = lrow[e];
    if (lane == (e & 31)) {
#pragma unroll
      for (int m = 0; m < RT_MAXV; ++m)
        if (m == (e >> 5)) key[m] = 0u;
    }
    if (k == 0) mx = sc;
    const float ex = exp_route(__fsub_rn(sc, mx));
    denom = __fadd_rn(denom, ex);
    if (lane == k) {
      my_e = e;
      my_x = ex;
    }
  }
  if (lane < K) {
    const float p = bf16_bits_to_f32(f32_to_bf16_bits(__fdiv_rn(my_x, denom)));
    idx_out[t * K + lane] = my_e;
    w_out[t * K + lane] = f32_to_bf16_bits(__fmul_rn(p, bf16_bits_to_f32(expert_scale[my_e])));
  }
}

// expert_scale != NULL: the Gemma 4 routing above instead of this one.
template <int MV>
__device__ inline void route_token_warp_mv(const float* lrow, int64_t t, int E, int K, int renorm, int lane,
                                           int32_t* __restrict__ idx_out, uint16_t* __restrict__ w_out,
                                           uint16_t* __restrict__ probs_out, const uint16_t* __restrict__ expert_scale) {
  constexpr int RT_MAXV = MV;
  if (expert_scale) {
    route_token_warp_gemma4<MV>(lrow, t, E, K, lane, idx_out, w_out, expert_scale);
    return;
  }
  float lv[RT_MAXV];
  float mx = -INFINITY;
#pragma unroll
  for (int m = 0; m < RT_MAXV; ++m) {
    const int e = lane + 32 * m;
    lv[m] = e < E ? lrow[e] : -INFINITY;
    mx = fmaxf(mx, lv[m]);
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, s));
  float acc = 0.0f;
#pragma unroll
  for (int m = 0; m < RT_MAXV; ++m) {
    const int e = lane + 32 * m;
    if (e < E) {
      lv[m] = exp_route(__fsub_rn(lv[m], mx));
      acc = __fadd_rn(acc, lv[m]);
    }
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, s));
  uint32_t key[RT_MAXV];
#pragma unroll
  for (int m = 0; m < RT_MAXV; ++m) {
    const int e = lane + 32 * m;
    key[m] = 0u;
    if (e < E) {
      const uint16_t pb = f32_to_bf16_bits(__fdiv_rn(lv[m], acc));
      if (probs_out) probs_out[t * E + e] = pb;
      key[m] = ((uint32_t)pb << 16) | (uint32_t)(0xFFFF - e);
    }
  }
  int my_e = 0;
  float my_p = 0.0f;
  float denom = 0.0f;
  for (int k = 0; k < K; ++k) {
    uint32_t best = 0u;
#pragma unroll
    for (int m = 0; m < RT_MAXV; ++m) best = best > key[m] ? best : key[m];
    best = __reduce_max_sync(0xffffffffu, best);
    const int e = 0xFFFF - (int)(best & 0xFFFFu);
    const float p = bf16_bits_to_f32((uint16_t)(best >> 16));
    if (lane == (e & 31)) {
#pragma unroll
      for (int m = 0; m < RT_MAXV; ++m)
        if (m == (e >> 5)) key[m] = 0u;
    }
    if (lane == k) {
      my_e = e;
      my_p = p;
    }
    denom = __fadd_rn(denom, p);
  }
  if (lane < K) {
    const float dbf = bf16_bits_to_f32(f32_to_bf16_bits(denom));
    idx_out[t * K + lane] = my_e;
    w_out[t * K + lane] = renorm ? f32_to_bf16_bits(__fdiv_rn(my_p, dbf)) : f32_to_bf16_bits(my_p);
  }
}

// Routes one token (every lane of the warp calls it), with lane arrays sized for E.
__device__ inline void route_token_warp(const float* lrow, int64_t t, int E, int K, int renorm, int lane,
                                        int32_t* __restrict__ idx_out, uint16_t* __restrict__ w_out,
                                        uint16_t* __restrict__ probs_out, const uint16_t* __restrict__ expert_scale) {
  if (E <= 128) route_token_warp_mv<4>(lrow, t, E, K, renorm, lane, idx_out, w_out, probs_out, expert_scale);
  else if (E <= 256) route_token_warp_mv<8>(lrow, t, E, K, renorm, lane, idx_out, w_out, probs_out, expert_scale);
  else if (E <= 512) route_token_warp_mv<16>(lrow, t, E, K, renorm, lane, idx_out, w_out, probs_out, expert_scale);
  else route_token_warp_mv<32>(lrow, t, E, K, renorm, lane, idx_out, w_out, probs_out, expert_scale);
}

// sigmoid(x . dequant(g_s)) of one token by one warp (moe.rs:119-120).
__device__ inline void shared_gate_warp(const uint16_t* __restrict__ xr, int D, const SharedGateArgs& sg, int lane,
                                        float* out) {
  const int per = 32 / sg.bits;
  const uint32_t mask = (1u << sg.bits) - 1u;
  float z = 0.0f;
  for (int d = lane; d < D; d += 32) {
    const uint32_t q = (__ldg(sg.w + d / per) >> ((d % per) * sg.bits)) & mask;
    const float wv = __fmaf_rn(bf16_bits_to_f32(__ldg(sg.s + d / 64)), (float)q, bf16_bits_to_f32(__ldg(sg.b + d / 64)));
    z = fmaf(bf16_bits_to_f32(__ldg(xr + d)), wv, z);
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) z += __shfl_xor_sync(0xffffffffu, z, s);
  if (lane == 0) *out = 1.0f / (1.0f + __expf(-z));
}

// The whole router for TPB tokens in one CTA of 16 warps. Warp w computes
// the logits of expert groups w, w+16, ... (8 experts each) for the TPB
// tokens into shared memory: lane j sums the exact products of the 16-byte
// chunks j, j+32, ... of D in fp64, an xor butterfly adds the lanes, and the
// logit is taken from the error interval of that sum (or the exact warp sum
// when the interval straddles a rounding boundary). Warp t < TPB then
// routes token t.
constexpr int RT_THREADS = 512;

template <int TPB>
__global__ void __launch_bounds__(RT_THREADS) router_fused_kernel(
    const uint16_t* __restrict__ x, int64_t T, int D, const uint16_t* __restrict__ wg, int E,
    const float* __restrict__ bias, int K, int renorm, int32_t* __restrict__ idx_out, uint16_t* __restrict__ w_out,
    uint16_t* __restrict__ logits_out, uint16_t* __restrict__ probs_out, SharedGateArgs sg,
    float* __restrict__ sig_out, const uint16_t* __restrict__ expert_scale) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ float s_lg[];  // [TPB][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = (int64_t)blockIdx.x * TPB;
  const uint4* xr[TPB];
#pragma unroll
  for (int i = 0; i < TPB; ++i) xr[i] = reinterpret_cast<const uint4*>(x + (t0 + i < T ? t0 + i : T - 1) * D);
  const int nchunks = D / 8;
  const int ngroups = (E + 7) / 8;
  for (int g = warp; g < ngroups; g += RT_THREADS / 32) {
    const int e0 = g * 8;
    const uint4* wr[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) wr[j] = reinterpret_cast<const uint4*>(wg + (int64_t)(e0 + j < E ? e0 + j : E - 1) * D);
    // fp64 sums of the exact products (and of the squares, for the error
    // bound); the logit is decided from the interval or, failing that, by
    // the exact warp sum.
    double acc[TPB][8];
    uint32_t mx[TPB], mw[8];  // largest |bf16 bits| of each row (error bound, inf/NaN detection)
#pragma unroll
    for (int i = 0; i < TPB; ++i) {
      mx[i] = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.0;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) mw[j] = 0u;
#pragma unroll 2
    for (int c = lane; c < nchunks; c += 32) {
      uint4 xv[TPB], wv[8];
#pragma unroll
      for (int i = 0; i < TPB; ++i) xv[i] = __ldg(xr[i] + c);
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[j] = __ldg(wr[j] + c);
#pragma unroll
      for (int el = 0; el < 8; ++el) {
        double xf[TPB], wf[8];
#pragma unroll
        for (int i = 0; i < TPB; ++i) {
          const uint32_t wd = el < 2 ? xv[i].x : el < 4 ? xv[i].y : el < 6 ? xv[i].z : xv[i].w;
          const uint32_t b = (el & 1) ? (wd >> 16) : (wd & 0xffffu);
          xf[i] = bf16_to_f64(b);
          mx[i] = max(mx[i], b & 0x7fffu);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t wd = el < 2 ? wv[j].x : el < 4 ? wv[j].y : el < 6 ? wv[j].z : wv[j].w;
          const uint32_t b = (el & 1) ? (wd >> 16) : (wd & 0xffffu);
          wf[j] = bf16_to_f64(b);
          mw[j] = max(mw[j], b & 0x7fffu);
        }
#pragma unroll
        for (int i = 0; i < TPB; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = __fma_rn(xf[i], wf[j], acc[i][j]);
      }
    }
#pragma unroll
    for (int i = 0; i < TPB; ++i) mx[i] = __reduce_max_sync(0xffffffffu, mx[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) mw[j] = __reduce_max_sync(0xffffffffu, mw[j]);
    const int depth = 8 * ((nchunks + 31) / 32) + 5;
    uint16_t mine = 0;
#pragma unroll
    for (int i = 0; i < TPB; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        double v = acc[i][j];
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, s));
        const int e = e0 + j < E ? e0 + j : E - 1;
        const float b = bias ? bias[e] : 0.0f;
        uint16_t lb;
        if (mx[i] >= 0x7f80u || mw[j] >= 0x7f80u || !logit_from_f64(v, f64_sum_err(depth, D, mx[i], mw[j]), b, &lb)) {
          const int64_t t = t0 + i < T ? t0 + i : T - 1;
          lb = logit_exact_warp(x + t * D, wg + (int64_t)e * D, D, b, mx[i], mw[j], lane);
        }
        if (lane == i * 8 + j) mine = lb;
      }
    if (lane < TPB * 8) {
      const int i = lane >> 3, e = e0 + (lane & 7);
      if (e < E) {
        s_lg[i * E + e] = bf16_bits_to_f32(mine);
        if (logits_out && t0 + i < T) logits_out[(t0 + i) * E + e] = mine;
      }
    }
  }
  __syncthreads();
  if (warp < TPB && t0 + warp < T) {
    const int64_t t = t0 + warp;
    route_token_warp(s_lg + warp * E, t, E, K, renorm, lane, idx_out, w_out, probs_out, expert_scale);
    if (sig_out) shared_gate_warp(x + t * D, D, sg, lane, sig_out + t);
  }
}

// Small batches: the logits of TPB tokens are spread over many CTAs (warp w
// of CTA (gx, gy) computes the EPW experts of group RS_WARPS*gx + w for
// tokens gy*TPB ...), with router_fused_kernel's fp64 sums and interval
// test, into the bf16 logits buffer lg [T, E]. Each lane
// issues the loads of UNR chunk steps before using them, so a warp keeps
// (TPB + EPW) * UNR 16-byte loads in flight: with few tokens the kernel is
// bound by memory latency, not arithmetic. The CTA that finishes the last
// expert group of a token block (counter[gy], zero on entry) routes it.
constexpr int RS_WARPS = 4;

template <int TPB, int EPW, int UNR>
__global__ void __launch_bounds__(RS_WARPS * 32) router_split_kernel(
    const uint16_t* __restrict__ x, int64_t T, int D, const uint16_t* __restrict__ wg, int E,
    const float* __restrict__ bias, int K, int renorm, int32_t* __restrict__ idx_out, uint16_t* __restrict__ w_out,
    uint16_t* __restrict__ lg, uint16_t* __restrict__ probs_out, SharedGateArgs sg, float* __restrict__ sig_out,
    int* __restrict__ counter, const uint16_t* __restrict__ expert_scale) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ float s_lg[];  // [TPB][E] (last CTA of a token block only)
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = (int64_t)blockIdx.y * TPB;
  const int nchunks = D / 8;
  const int ngroups = (E + EPW - 1) / EPW;
  const int g = blockIdx.x * RS_WARPS + warp;
  if (g < ngroups) {
    const uint4* xr[TPB];
#pragma unroll
    for (int i = 0; i < TPB; ++i) xr[i] = reinterpret_cast<const uint4*>(x + (t0 + i < T ? t0 + i : T - 1) * D);
    const int e0 = g * EPW;
    const uint4* wr[EPW];
#pragma unroll
    for (int j = 0; j < EPW; ++j)
      wr[j] = reinterpret_cast<const uint4*>(wg + (int64_t)(e0 + j < E ? e0 + j : E - 1) * D);
    double acc[TPB][EPW];
    uint32_t mx[TPB], mw[EPW];  // largest |bf16 bits| of each row (error bound, inf/NaN detection)
#pragma unroll
    for (int i = 0; i < TPB; ++i) {
      mx[i] = 0u;
#pragma unroll
      for (int j = 0; j < EPW; ++j) acc[i][j] = 0.0;
    }
#pragma unroll
    for (int j = 0; j < EPW; ++j) mw[j] = 0u;
    for (int cb = 0; cb < nchunks; cb += 32 * UNR) {
      uint4 xv[UNR][TPB], wv[UNR][EPW];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int c = cb + 32 * u + lane;
        if (c < nchunks) {
#pragma unroll
          for (int i = 0; i < TPB; ++i) xv[u][i] = __ldg(xr[i] + c);
#pragma unroll
          for (int j = 0; j < EPW; ++j) wv[u][j] = __ldg(wr[j] + c);
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        if (cb + 32 * u + lane >= nchunks) break;
#pragma unroll
        for (int el = 0; el < 8; ++el) {
          double xf[TPB], wf[EPW];
#pragma unroll
          for (int i = 0; i < TPB; ++i) {
            const uint32_t wd = el < 2 ? xv[u][i].x : el < 4 ? xv[u][i].y : el < 6 ? xv[u][i].z : xv[u][i].w;
            const uint32_t b = (el & 1) ? (wd >> 16) : (wd & 0xffffu);
            xf[i] = bf16_to_f64(b);
            mx[i] = max(mx[i], b & 0x7fffu);
          }
#pragma unroll
          for (int j = 0; j < EPW; ++j) {
            const uint32_t wd = el < 2 ? wv[u][j].x : el < 4 ? wv[u][j].y : el < 6 ? wv[u][j].z : wv[u][j].w;
            const uint32_t b = (el & 1) ? (wd >> 16) : (wd & 0xffffu);
            wf[j] = bf16_to_f64(b);
            mw[j] = max(mw[j], b & 0x7fffu);
          }
#pragma unroll
          for (int i = 0; i < TPB; ++i)
#pragma unroll
            for (int j = 0; j < EPW; ++j) acc[i][j] = __fma_rn(xf[i], wf[j], acc[i][j]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < TPB; ++i) mx[i] = __reduce_max_sync(0xffffffffu, mx[i]);
#pragma unroll
    for (int j = 0; j < EPW; ++j) mw[j] = __reduce_max_sync(0xffffffffu, mw[j]);
    const int depth = 8 * ((nchunks + 31) / 32) + 5;
    uint16_t mine = 0;
#pragma unroll
    for (int i = 0; i < TPB; ++i)
#pragma unroll
      for (int j = 0; j < EPW; ++j) {
        double v = acc[i][j];
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, s));
        const int e = e0 + j < E ? e0 + j : E - 1;
        const float b = bias ? bias[e] : 0.0f;
        uint16_t lb;
        if (mx[i] >= 0x7f80u || mw[j] >= 0x7f80u || !logit_from_f64(v, f64_sum_err(depth, D, mx[i], mw[j]), b, &lb)) {
          const int64_t t = t0 + i < T ? t0 + i : T - 1;
          lb = logit_exact_warp(x + t * D, wg + (int64_t)e * D, D, b, mx[i], mw[j], lane);
        }
        if (lane == i * EPW + j) mine = lb;
      }
    if (lane < TPB * EPW) {
      const int i = lane / EPW, e = e0 + lane % EPW;
      if (e < E && t0 + i < T) lg[(t0 + i) * E + e] = mine;
    }
  }
  // Publish this CTA's logits; the last CTA of the token block routes it.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&counter[blockIdx.y], 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int ntok = (int)min((int64_t)TPB, T - t0);
  for (int i = threadIdx.x; i < ntok * E; i += blockDim.x)
    s_lg[i] = bf16_bits_to_f32(__ldcg(lg + t0 * E + i));
  __syncthreads();
  for (int i = warp; i < ntok; i += RS_WARPS) {
    const int64_t t = t0 + i;
    route_token_warp(s_lg + i * E, t, E, K, renorm, lane, idx_out, w_out, probs_out, expert_scale);
    if (sig_out) shared_gate_warp(x + t * D, D, sg, lane, sig_out + t);
  }
}

// Gemma 4 input norms of one token per warp (fast::rms_norm of the router,
// gemma4/text/text.rs:622-639, and pre_feedforward_layernorm_2, :907-911):
// inv = 1 / sqrt(ss / D + eps) in IEEE fp32, ss = sum of x^2 in the logit
// order (lane j folds chunks j, j+32, ... of 8 elements with fmaf, then the
// xor butterfly); xr = bf16((x * inv) * wr), xe = bf16((x * inv) * we).
// x, xr, xe 16-byte aligned, D a multiple of 8.
constexpr int G4_NORM_WARPS = 8;
__global__ void __launch_bounds__(G4_NORM_WARPS * 32) gemma4_norm_kernel(
    const uint16_t* __restrict__ x, int64_t T, int D, float eps, const uint16_t* __restrict__ wr,
    const uint16_t* __restrict__ we, uint16_t* __restrict__ xr, uint16_t* __restrict__ xe) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * G4_NORM_WARPS + warp;
  if (t >= T) return;
  const uint4* row = reinterpret_cast<const uint4*>(x + t * D);
  const int nchunks = D / 8;
  float acc = 0.0f;
  for (int c = lane; c < nchunks; c += 32) {
    const uint4 v = row[c];
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = bf_lo(w4[i]), b = bf_hi(w4[i]);
      acc = __fmaf_rn(a, a, acc);
      acc = __fmaf_rn(b, b, acc);
    }
  }
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, s));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)D), eps)));
  const uint4* wr4 = reinterpret_cast<const uint4*>(wr);
  const uint4* we4 = reinterpret_cast<const uint4*>(we);
  uint4* xr4 = reinterpret_cast<uint4*>(xr + t * D);
  uint4* xe4 = reinterpret_cast<uint4*>(xe + t * D);
  for (int c = lane; c < nchunks; c += 32) {
    const uint4 v = row[c], a4 = __ldg(wr4 + c), b4 = __ldg(we4 + c);
    const uint32_t xv[4] = {v.x, v.y, v.z, v.w}, av[4] = {a4.x, a4.y, a4.z, a4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
    uint32_t ro[4], eo[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x0 = __fmul_rn(bf_lo(xv[i]), inv), x1 = __fmul_rn(bf_hi(xv[i]), inv);
      ro[i] = (uint32_t)f32_to_bf16_bits(__fmul_rn(x0, bf_lo(av[i]))) |
              ((uint32_t)f32_to_bf16_bits(__fmul_rn(x1, bf_hi(av[i]))) << 16);
      eo[i] = (uint32_t)f32_to_bf16_bits(__fmul_rn(x0, bf_lo(bv[i]))) |
              ((uint32_t)f32_to_bf16_bits(__fmul_rn(x1, bf_hi(bv[i]))) << 16);
    }
    xr4[c] = make_uint4(ro[0], ro[1], ro[2], ro[3]);
    xe4[c] = make_uint4(eo[0], eo[1], eo[2], eo[3]);
  }
}

// Softmax / top-K / renormalisation (and the shared-expert gate) of one
// token per warp from the bf16 logits lg [T, E].
constexpr int RT_ROUTE_WARPS = 8;
template <int MV>
__global__ void __launch_bounds__(RT_ROUTE_WARPS * 32) route_rows_kernel(
    const uint16_t* __restrict__ lg, const uint16_t* __restrict__ x, int64_t T, int D, int E, int K, int renorm,
    int32_t* __restrict__ idx_out, uint16_t* __restrict__ w_out, uint16_t* __restrict__ probs_out, SharedGateArgs sg,
    float* __restrict__ sig_out, const uint16_t* __restrict__ expert_scale) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ float s_row[];  // [RT_ROUTE_WARPS][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * RT_ROUTE_WARPS + warp;
  if (t >= T) return;
  float* row = s_row + warp * E;
  for (int e = lane; e < E; e += 32) row[e] = bf16_bits_to_f32(lg[t * E + e]);
  __syncwarp();
  route_token_warp_mv<MV>(row, t, E, K, renorm, lane, idx_out, w_out, probs_out, expert_scale);
  if (sig_out) shared_gate_warp(x + t * D, D, sg, lane, sig_out + t);
}

// The tensor-core router's split-K form (router_tc.cu): part[s][g][t][e]
// (s < splits, g < kRouterSums) are the digit sums of k-slice s. One thread per
// (token, expert), experts fastest: the slices are added (exact integer
// sums) and the logit formed as router_tc_kernel's epilogue does; logits the
// interval test leaves open are computed by the whole warp (logit_warp)
// (each undecided lane's token and expert in turn). route_rows_kernel then
// routes the tokens.
__global__ void __launch_bounds__(256) logits_from_partials_kernel(
    const int32_t* __restrict__ part, int splits, const int2* __restrict__ xinfo, const int2* __restrict__ winfo,
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ wg, const float* __restrict__ bias, int64_t T, int D,
    int E, uint16_t* __restrict__ lg) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t n = T * (int64_t)E;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = i < n;
  const int64_t ic = valid ? i : n - 1;
  const int64_t t = ic / E;
  const int e = (int)(ic - t * E);
  const int64_t gstride = n, sstride = kRouterSums * n;
  int32_t A[kRouterSums] = {0, 0, 0, 0, 0};
  for (int sp = 0; sp < splits; ++sp)
#pragma unroll
    for (int g = 0; g < kRouterSums; ++g) A[g] += __ldg(part + sp * sstride + g * gstride + ic);
  const float b = bias ? bias[e] : 0.0f;
  bool decided;
  uint16_t lb = logit_from_digit_sums<kRouterSums>(A, xinfo[t], winfo[e], D, b, &decided);
  uint32_t need = __ballot_sync(0xffffffffu, valid && !decided);
  while (need) {
    const int src = __ffs(need) - 1;
    need &= need - 1;
    const int64_t ts = __shfl_sync(0xffffffffu, t, src);
    const int es = __shfl_sync(0xffffffffu, e, src);
    const float bs = __shfl_sync(0xffffffffu, b, src);
    const uint16_t r = logit_warp(x + ts * D, wg + (int64_t)es * D, D, bs, lane);
    if (lane == src) lb = r;
  }
  if (valid) lg[i] = lb;
}

// ------------------------------------------------------- permutation ----
constexpr int PERM_ROWS = 2048;  // flat rows per permute block (8 warps x 256)
constexpr int PERM_MAX_E = 1024;

// skip != 0: rows whose index is negative are left out of the permutation
// (their inv entry becomes -1); otherwise a negative index is an error.
__global__ void __launch_bounds__(256) permute_count_kernel(const int32_t* __restrict__ idx, int64_t R, int E,
                                                           int32_t* __restrict__ block_counts, int skip, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * PERM_ROWS;
  for (int i = threadIdx.x; i < PERM_ROWS; i += blockDim.x) {
    const int64_t f = base + i;
    if (f < R) {
      const int e = idx[f];
      if (e < 0 && skip) continue;
      if (e < 0 || e >= E) atomicCAS(status, 0, (int)kDevBadIndex);
      else atomicAdd(&hist[e], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) block_counts[(int64_t)blockIdx.x * E + e] = hist[e];
}

// Exclusive scan of one int per thread over a 1024-thread block.
__device__ inline int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int s = 1; s < 32; s <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, s);
    if (lane >= s) incl += o;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int ws = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
    int wi = ws;
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, wi, s);
      if (lane >= s) wi += o;
    }
    warp_sums[lane] = wi - ws;
    if (lane == 31) *total = wi;
  }
  __syncthreads();
  const int r = warp_sums[warp] + incl - v;
  __syncthreads();
  return r;
}

struct TileListOut {
  GemmTile* tiles;
  int32_t* count;
  int bn;
  int cap;  // entries the list holds; tiles beyond it are dropped (the gather flags the excess rows)
};

// Tile lists for the grouped GEMMs (one per tile width) and the dense
// shared-expert list, from each expert's total `tot` and offset `off`
// (thread e of a 1024-thread block owns expert e).
__device__ inline void build_tile_lists(int e, int E, int tot, int off, int64_t T, const TileListOut& l1,
                                        const TileListOut& l2, const TileListOut& lsh, int* warp_sums, int* total) {
  TileListOut lists[2] = {l1, l2};
  for (int li = 0; li < 2; ++li) {
    const TileListOut L = lists[li];
    const int nt = e < E ? (tot + L.bn - 1) / L.bn : 0;
    const int toff = block_exclusive_scan(nt, warp_sums, total);
    for (int j = 0; j < nt; ++j) {
      GemmTile g;
      g.expert = e;
      g.row_start = off + j * L.bn;
      g.row_count = min(L.bn, tot - j * L.bn);
      g.pad = 0;
      if (toff + j < L.cap) L.tiles[toff + j] = g;
    }
    if (e == 0) *L.count = min(*total, L.cap);
  }
  if (lsh.tiles) {
    const int nt = (int)((T + lsh.bn - 1) / lsh.bn);
    for (int j = e; j < nt && j < lsh.cap; j += blockDim.x) {
      GemmTile g;
      g.expert = 0;
      g.row_start = j * lsh.bn;
      g.row_count = (int)min((int64_t)lsh.bn, T - (int64_t)j * lsh.bn);
      g.pad = 0;
      lsh.tiles[j] = g;
    }
    if (e == 0) *lsh.count = min(nt, lsh.cap);
  }
}

// Single CTA of 1024 threads: expert totals, offsets, per-block bases and
// the GEMM tile lists (one per tile width) plus the dense shared-expert list.
__global__ void __launch_bounds__(1024) permute_scan_kernel(int32_t* __restrict__ zero, int nzero,
                                                           const int32_t* __restrict__ block_counts, int nblk, int E,
                                                           int64_t T, int32_t* __restrict__ block_base,
                                                           int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                                                           TileListOut l1, TileListOut l2, TileListOut lsh) {
  pdl_wait();
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;  // counters the GEMMs expect at zero
  __shared__ int warp_sums[32];
  __shared__ int total;
  const int e = threadIdx.x;
  int tot = 0;
  if (e < E)
    for (int b = 0; b < nblk; ++b) tot += block_counts[(int64_t)b * E + e];
  const int off = block_exclusive_scan(e < E ? tot : 0, warp_sums, &total);
  if (e < E) {
    counts[e] = tot;
    offsets[e] = off;
    int run = off;
    for (int b = 0; b < nblk; ++b) {
      const int c = block_counts[(int64_t)b * E + e];
      block_base[(int64_t)b * E + e] = run;
      run += c;
    }
  }
  if (e == 0) offsets[E] = total;
  build_tile_lists(e, E, tot, off, T, l1, l2, lsh, warp_sums, &total);
}

// Stable ranks of a warp's contiguous row range [wbeg, wend): each row f
// goes to position wbase[e] + (rows of the same expert before it), where
// wbase[e] (shared memory) holds the warp's first position per expert.
__device__ inline void rank_rows_warp(const int32_t* __restrict__ idx, int64_t wbeg, int64_t wend, int64_t R, int E,
                                      int* wbase, int lane, int32_t* __restrict__ sorted_rows,
                                      int32_t* __restrict__ inv) {
  const uint32_t lt_mask = (1u << lane) - 1u;
  for (int64_t c0 = wbeg; c0 < wend; c0 += 32) {
    const int64_t f = c0 + lane;
    int e = -1;
    if (f < wend) {
      e = idx[f];
      if (e < 0 || e >= E) e = -1;
    }
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    int pos = -1;
    if (e >= 0) pos = wbase[e] + __popc(peers & lt_mask);
    if (pos >= R) pos = -1;  // cannot happen for consistent counts; never write out of range
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) wbase[e] += __popc(peers);
    __syncwarp();
    if (pos >= 0) {
      sorted_rows[pos] = (int32_t)f;
      inv[f] = pos;
    } else if (f < wend) {
      inv[f] = -1;  // a skipped (or invalid, already flagged) row
    }
  }
}

// The whole permutation when every flat row fits one 2048-row block: count,
// scan, tile lists and the stable scatter in a single 1024-thread CTA.
__global__ void __launch_bounds__(1024) permute_small_kernel(const int32_t* __restrict__ idx, int64_t R, int E,
                                                            int64_t T, int32_t* __restrict__ counts,
                                                            int32_t* __restrict__ offsets,
                                                            int32_t* __restrict__ sorted_rows,
                                                            int32_t* __restrict__ inv, TileListOut l1, TileListOut l2,
                                                            TileListOut lsh, int skip, int* status,
                                                            int32_t* __restrict__ zero, int nzero,
                                                            const uint16_t* __restrict__ gx, int D, int K, int kperm,
                                                            uint16_t* __restrict__ x_sorted) {
  pdl_wait();
  pdl_launch_dependents();
  // Counters the GEMMs that follow expect at zero (split-K).
  for (int i = threadIdx.x; i < nzero; i += blockDim.x) zero[i] = 0;
  extern __shared__ int sm[];  // hist[E], then wcnt[8][E] (8 row ranges of 256)
  __shared__ int warp_sums[32];
  __shared__ int total;
  int* hist = sm;
  int* wcnt = sm + E;
  for (int i = threadIdx.x; i < 9 * E; i += blockDim.x) sm[i] = 0;
  __syncthreads();
  for (int64_t f = threadIdx.x; f < R; f += blockDim.x) {
    const int e = idx[f];
    if (e < 0 && skip) continue;
    if (e < 0 || e >= E) {
      atomicCAS(status, 0, (int)kDevBadIndex);
    } else {
      atomicAdd(&hist[e], 1);
      atomicAdd(&wcnt[(int)(f / (PERM_ROWS / 8)) * E + e], 1);
    }
  }
  __syncthreads();
  const int e = threadIdx.x;
  const int tot = e < E ? hist[e] : 0;
  const int off = block_exclusive_scan(tot, warp_sums, &total);
  if (e < E) {
    counts[e] = tot;
    offsets[e] = off;
    int run = off;
    for (int w = 0; w < 8; ++w) {
      const int c = wcnt[w * E + e];
      wcnt[w * E + e] = run;
      run += c;
    }
  }
  if (e == 0) offsets[E] = total;
  build_tile_lists(e, E, tot, off, T, l1, l2, lsh, warp_sums, &total);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < 8) {
    const int64_t wbeg = (int64_t)warp * (PERM_ROWS / 8);
    const int64_t wend = min(wbeg + PERM_ROWS / 8, R);
    rank_rows_warp(idx, wbeg, wend, R, E, wcnt + warp * E, lane, sorted_rows, inv);
  }
  if (x_sorted == nullptr) return;
  // Few rows (decode): the row gather here rather than in a second launch,
  // the same copy as permute_gather_kernel (one warp per row, 16-byte
  // accesses, 4-bit K order when kperm).
  __syncthreads();
  const int dvec = D / 8;
  for (int64_t pos = warp; pos < R; pos += 32) {
    const int32_t f = sorted_rows[pos];
    if (f < 0 || (int64_t)f >= R) continue;
    const uint4* src = reinterpret_cast<const uint4*>(gx + (int64_t)(f / K) * D);
    uint4* dst = reinterpret_cast<uint4*>(x_sorted + pos * D);
    for (int v = lane; v < dvec; v += 32) {
      uint4 a = __ldg(src + v);
      if (kperm) {
        uint4 b;
        b.x = __byte_perm(a.x, a.z, 0x5410);
        b.y = __byte_perm(a.x, a.z, 0x7632);
        b.z = __byte_perm(a.y, a.w, 0x5410);
        b.w = __byte_perm(a.y, a.w, 0x7632);
        a = b;
      }
      dst[v] = a;
    }
  }
}

// Stable in-block ranks. 8 warps; warp w owns flat rows
// [blk*2048 + w*256, +256).
__global__ void __launch_bounds__(256) permute_scatter_kernel(const int32_t* __restrict__ idx, int64_t R, int E,
                                                             const int32_t* __restrict__ block_base,
                                                             int32_t* __restrict__ sorted_rows,
                                                             int32_t* __restrict__ inv) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ int wcnt[];  // [8][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < 8 * E; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  const int64_t wbeg = (int64_t)blockIdx.x * PERM_ROWS + warp * (PERM_ROWS / 8);
  const int64_t wend = min(wbeg + PERM_ROWS / 8, R);
  for (int64_t f = wbeg + lane; f < wend; f += 32) {
    const int e = idx[f];
    if (e >= 0 && e < E) atomicAdd(&wcnt[warp * E + e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = block_base[(int64_t)blockIdx.x * E + e];
    for (int w = 0; w < 8; ++w) {
      const int c = wcnt[w * E + e];
      wcnt[w * E + e] = run;
      run += c;
    }
  }
  __syncthreads();
  rank_rows_warp(idx, wbeg, wend, R, E, wcnt + warp * E, lane, sorted_rows, inv);
}

// x_sorted[pos] = x[sorted_rows[pos] / K] (sorted_rows NULL: the identity)
// for pos < n_rows, one warp per row, 16-byte loads and stores, the whole
// grid streaming. sorted_rows entries must lie in [0, n_flat). With count
// (a permutation with skipped rows) only pos < *count is copied, and a count
// above n_rows (more rows than the destination holds) is an error. With
// kperm the 8 elements of every 16-byte chunk are stored in the 4-bit
// operand order {0,4,1,5,2,6,3,7} the grouped GEMM's dequantiser produces.
__global__ void __launch_bounds__(256) permute_gather_kernel(const int32_t* __restrict__ sorted_rows, int64_t n_rows,
                                                            int64_t n_flat, int K, const uint16_t* __restrict__ x,
                                                            int D, int kperm, uint16_t* __restrict__ x_sorted,
                                                            const int32_t* __restrict__ count, int* status,
                                                            int coherent) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dvec = D / 8;
  int64_t n = n_rows;
  if (count) {
    const int64_t c = *count;
    if (c > n_rows && blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(status, 0, (int)kDevBadIndex);
    n = min(n_rows, c);
  }
  // An output larger than half the L2 goes out with streaming (evict-first)
  // stores: it cannot stay in L2 for the GEMM anyway, and normal stores
  // would evict the x rows that the next K - 1 copies of each token read.
  const bool stream_out = n_rows * (int64_t)D * 2 > (int64_t)(64ll << 20);
  for (int64_t pos = (int64_t)blockIdx.x * 8 + warp; pos < n; pos += (int64_t)gridDim.x * 8) {
    int64_t src_row = pos;
    if (sorted_rows) {
      const int32_t f = sorted_rows[pos];
      if (f < 0 || (int64_t)f >= n_flat) continue;
      src_row = f / K;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + src_row * D);
    uint4* dst = reinterpret_cast<uint4*>(x_sorted + pos * D);
    // coherent: through L2 only (the rows were stored by a peer GPU);
    // otherwise the read-only path, which keeps rows gathered K times in L1.
    auto ld = [&](int v) { return coherent ? __ldcg(src + v) : __ldg(src + v); };
    auto st = [&](int v, uint4 a) {
      if (kperm) {
        uint4 b;
        b.x = __byte_perm(a.x, a.z, 0x5410);
        b.y = __byte_perm(a.x, a.z, 0x7632);
        b.z = __byte_perm(a.y, a.w, 0x5410);
        b.w = __byte_perm(a.y, a.w, 0x7632);
        a = b;
      }
      if (stream_out) __stcs(dst + v, a);
      else dst[v] = a;
    };
    // Eight 16-byte loads of the row in flight per lane before any store
    // (one load at a time left the copy latency-bound at half the HBM rate).
    int v = lane;
    for (; v + 7 * 32 < dvec; v += 8 * 32) {
      uint4 a[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = ld(v + j * 32);
#pragma unroll
      for (int j = 0; j < 8; ++j) st(v + j * 32, a[j]);
    }
    for (; v < dvec; v += 32) st(v, ld(v));
  }
}

// ------------------------------------------------------------ combine ---
__global__ void __launch_bounds__(256) combine_kernel(const uint16_t* __restrict__ y_sorted,
                                                     const int32_t* __restrict__ inv, const uint16_t* __restrict__ w,
                                                     int K, int D, int64_t T, const uint16_t* __restrict__ y_sh,
                                                     const float* __restrict__ sig, uint16_t* __restrict__ out,
                                                     int* status) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int rows[RT_MAXK];
  __shared__ float wk[RT_MAXK];
  const int64_t t = blockIdx.x;
  if (threadIdx.x < K) {
    int r = inv[t * K + threadIdx.x];
    float wv = bf16_bits_to_f32(w[t * K + threadIdx.x]);
    if (r < 0 || (int64_t)r >= T * K) {  // never for a permutation built by permute_scatter_kernel
      atomicCAS(status, 0, (int)kDevBadIndex);
      r = 0;
      wv = 0.0f;
    }
    rows[threadIdx.x] = r;
    wk[threadIdx.x] = wv;
  }
  __syncthreads();
  const float sg = y_sh ? sig[t] : 0.0f;
  const int dvec = D / 8;
  for (int v = threadIdx.x; v < dvec; v += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    for (int k0 = 0; k0 < K; k0 += 8) {
      uint4 yv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)  // all loads of the group first
        if (k0 + j < K) yv[j] = __ldg(reinterpret_cast<const uint4*>(y_sorted + (int64_t)rows[k0 + j] * D) + v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (k0 + j < K) {
          const float wj = wk[k0 + j];
          const uint32_t ww[4] = {yv[j].x, yv[j].y, yv[j].z, yv[j].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[2 * i] = fmaf(wj, bf_lo(ww[i]), acc[2 * i]);
            acc[2 * i + 1] = fmaf(wj, bf_hi(ww[i]), acc[2 * i + 1]);
          }
        }
      }
    }
    if (y_sh) {
      const uint4 yv = __ldg(reinterpret_cast<const uint4*>(y_sh + t * D) + v);
      const uint32_t ww[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = fmaf(sg, bf_lo(ww[i]), acc[2 * i]);
        acc[2 * i + 1] = fmaf(sg, bf_hi(ww[i]), acc[2 * i + 1]);
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + t * D)[v] = o;
  }
}

// ------------------------------------------------- expert parallelism ---
// Expert e lives on rank placement[e] >> 16 as its local expert
// placement[e] & 0xFFFF; without a placement table, on rank e % world as
// local expert e / world.
// Every token is sent once to each rank that owns at least one of its top-k
// experts (one "pair" per (token, rank)); the pair carries up to K slots of
// (local expert, top-k weight), and the receiving rank returns one partial
// row per pair: the weighted sum of its experts' outputs for that token.

// dest[t*K + k] = rank of expert idx[t*K + k] when k is the first of token t
// that goes to that rank, -1 otherwise (so a stable sort of the non-negative
// entries lists the pairs by rank, then token).
__device__ __forceinline__ int ep_rank_of(int e, int world, const int32_t* placement) {
  return placement ? (int)((uint32_t)placement[e] >> 16) : e % world;
}
__device__ __forceinline__ int ep_local_of(int e, int world, const int32_t* placement) {
  return placement ? (placement[e] & 0xFFFF) : e / world;
}

__global__ void ep_pair_dest_kernel(const int32_t* __restrict__ idx, int64_t T, int K, int world,
                                    const int32_t* __restrict__ placement, int32_t* __restrict__ dest, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (f >= T * K) return;
  const int64_t t = f / K;
  const int k = (int)(f - t * K);
  const int e = idx[f];
  if (e < 0) {
    atomicCAS(status, 0, (int)kDevBadIndex);
    dest[f] = -1;
    return;
  }
  const int r = ep_rank_of(e, world, placement);
  if (r < 0 || r >= world) {
    atomicCAS(status, 0, (int)kDevBadIndex);
    dest[f] = -1;
    return;
  }
  bool first = true;
  for (int j = 0; j < k; ++j) {
    const int ej = idx[t * K + j];
    if (ej >= 0 && ep_rank_of(ej, world, placement) == r) {
      first = false;
      break;
    }
  }
  dest[f] = first ? r : -1;
}

// send_counts[2r] = pairs sent to rank r (from the pair permutation),
// send_counts[2r + 1] = (token, k) rows those pairs carry. One CTA.
__global__ void __launch_bounds__(1024) ep_counts_kernel(const int32_t* __restrict__ idx, int64_t R, int world,
                                                        const int32_t* __restrict__ placement,
                                                        const int32_t* __restrict__ pair_counts,
                                                        int32_t* __restrict__ send_counts) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int hist[64];
  if (threadIdx.x < 64) hist[threadIdx.x] = 0;
  __syncthreads();
  for (int64_t f = threadIdx.x; f < R; f += blockDim.x) {
    const int e = idx[f];
    if (e >= 0) {
      const int r = ep_rank_of(e, world, placement);
      if (r >= 0 && r < world) atomicAdd(&hist[r], 1);
    }
  }
  __syncthreads();
  if (threadIdx.x < world) {
    send_counts[2 * threadIdx.x] = pair_counts[threadIdx.x];
    send_counts[2 * threadIdx.x + 1] = hist[threadIdx.x];
  }
}

__device__ __forceinline__ int32_t ep_slot(int local_expert, uint16_t weight_bits) {
  return (int32_t)(((uint32_t)local_expert << 16) | weight_bits);
}

// One thread per token: for each pair of the token (send position pos =
// pair_pos[t*K + k] of its first k), meta[pos*K + j] = the j-th of the
// token's experts on that rank in k order, packed as (local expert << 16) |
// bf16 weight bits; -1 fills the unused slots.
__global__ void ep_pair_meta_kernel(const int32_t* __restrict__ idx, const uint16_t* __restrict__ w,
                                    const int32_t* __restrict__ pair_pos, int64_t T, int K, int world,
                                    const int32_t* __restrict__ placement, int64_t max_pairs,
                                    int32_t* __restrict__ meta, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const int32_t* ti = idx + t * K;
  for (int k = 0; k < K; ++k) {
    const int64_t pos = pair_pos[t * K + k];
    if (pos < 0) continue;  // not the first k of its rank
    if (pos >= max_pairs || ti[k] < 0) {
      atomicCAS(status, 0, (int)kDevBadIndex);
      continue;
    }
    const int r = ep_rank_of(ti[k], world, placement);
    int j = 0;
    for (int k2 = k; k2 < K; ++k2) {
      const int e = ti[k2];
      if (e >= 0 && ep_rank_of(e, world, placement) == r)
        meta[pos * K + j++] = ep_slot(ep_local_of(e, world, placement), w[t * K + k2]);
    }
    for (; j < K; ++j) meta[pos * K + j] = -1;
  }
}

// Receiving side: idx_local[i] = local expert of slot i, -1 for an empty slot.
__global__ void ep_slot_expert_kernel(const int32_t* __restrict__ meta, int64_t n, int E_local,
                                      int32_t* __restrict__ idx_local, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t m = meta[i];
  int le = -1;
  if (m >= 0) {
    le = m >> 16;
    if (le >= E_local) {
      atomicCAS(status, 0, (int)kDevBadIndex);
      le = -1;
    }
  }
  idx_local[i] = le;
}

// acc[0..7] += sum_j wk[j] * rows_base[rows[j]][8v .. 8v+7] (fp32 fmaf, j
// ascending), with the loads of each group of 8 rows issued first.
__device__ __forceinline__ void weighted_rows_acc(const uint16_t* __restrict__ base, const int* rows,
                                                  const float* wk, int n, int D, int v, float acc[8]) {
  for (int k0 = 0; k0 < n; k0 += 8) {
    uint4 yv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (k0 + j < n) yv[j] = __ldcg(reinterpret_cast<const uint4*>(base + (int64_t)rows[k0 + j] * D) + v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (k0 + j < n) {
        const float wj = wk[k0 + j];
        const uint32_t ww[4] = {yv[j].x, yv[j].y, yv[j].z, yv[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[2 * i] = fmaf(wj, bf_lo(ww[i]), acc[2 * i]);
          acc[2 * i + 1] = fmaf(wj, bf_hi(ww[i]), acc[2 * i + 1]);
        }
      }
    }
  }
}

__device__ __forceinline__ void store_bf16x8(uint16_t* dst, const float acc[8]) {
  uint4 o;
  o.x = pack_bf16x2(acc[0], acc[1]);
  o.y = pack_bf16x2(acc[2], acc[3]);
  o.z = pack_bf16x2(acc[4], acc[5]);
  o.w = pack_bf16x2(acc[6], acc[7]);
  *reinterpret_cast<uint4*>(dst) = o;
}

// Receiving side, one CTA per received pair p: partial[p] = bf16(sum over
// the pair's filled slots j, in slot order, of w_j * y_sorted[inv[p*K + j]]).
__global__ void __launch_bounds__(256) ep_reduce_kernel(const uint16_t* __restrict__ y_sorted,
                                                       const int32_t* __restrict__ inv,
                                                       const int32_t* __restrict__ meta, int K, int D, int64_t rows,
                                                       uint16_t* __restrict__ partial, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int rws[RT_MAXK];
  __shared__ float wk[RT_MAXK];
  __shared__ int nk;
  const int64_t p = blockIdx.x;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int j = 0; j < K; ++j) {
      const int32_t m = meta[p * K + j];
      if (m < 0) continue;
      const int r = inv[p * K + j];
      if (r < 0 || (int64_t)r >= rows) {
        atomicCAS(status, 0, (int)kDevBadIndex);
        continue;
      }
      rws[n] = r;
      wk[n] = bf16_bits_to_f32((uint16_t)(m & 0xFFFF));
      ++n;
    }
    nk = n;
  }
  __syncthreads();
  const int n = nk;
  for (int v = threadIdx.x; v < D / 8; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    weighted_rows_acc(y_sorted, rws, wk, n, D, v, acc);
    store_bf16x8(partial + p * D + 8 * v, acc);
  }
}

// Owning side, one CTA per token: out[t] = bf16(sum of the token's returned
// partial rows, in the order of their first k, + sig[t] * y_sh[t]).
__global__ void __launch_bounds__(256) ep_combine_kernel(const uint16_t* __restrict__ partial,
                                                        const int32_t* __restrict__ pair_pos, int K, int D,
                                                        int64_t num_pairs, const uint16_t* __restrict__ y_sh,
                                                        const float* __restrict__ sig, uint16_t* __restrict__ out,
                                                        int* status) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int rws[RT_MAXK + 1];
  __shared__ float wk[RT_MAXK + 1];
  __shared__ int nk;
  const int64_t t = blockIdx.x;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int k = 0; k < K; ++k) {
      const int32_t pos = pair_pos[t * K + k];
      if (pos < 0) continue;
      if ((int64_t)pos >= num_pairs) {
        atomicCAS(status, 0, (int)kDevBadIndex);
        continue;
      }
      rws[n] = pos;
      wk[n] = 1.0f;
      ++n;
    }
    nk = n;
  }
  __syncthreads();
  const int n = nk;
  const float sg = y_sh ? sig[t] : 0.0f;
  for (int v = threadIdx.x; v < D / 8; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    weighted_rows_acc(partial, rws, wk, n, D, v, acc);
    if (y_sh) {
      const uint4 yv = __ldg(reinterpret_cast<const uint4*>(y_sh + t * D) + v);
      const uint32_t ww[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = fmaf(sg, bf_lo(ww[i]), acc[2 * i]);
        acc[2 * i + 1] = fmaf(sg, bf_hi(ww[i]), acc[2 * i + 1]);
      }
    }
    store_bf16x8(out + t * D + 8 * v, acc);
  }
}

// The dense shared-expert tile list alone (row tiles of width bn over T
// tokens), for callers that run the shared expert without a permute.
// sig[t] = sigmoid(x[t] . dequant(shared_expert_gate)) alone, one warp per
// token, for callers that run the combine without the router (the routers
// compute it in their own pass over x, with the same helper).
__global__ void __launch_bounds__(256) shared_gate_kernel(const uint16_t* __restrict__ x, int64_t T, int D,
                                                         SharedGateArgs sg, float* __restrict__ sig) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t < T) shared_gate_warp(x + t * D, D, sg, threadIdx.x & 31, sig + t);
}

__global__ void shared_tiles_kernel(GemmTile* __restrict__ tiles, int32_t* __restrict__ count, int64_t T, int bn,
                                    int cap) {
  pdl_wait();
  pdl_launch_dependents();
  const int nt = (int)((T + bn - 1) / bn);
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < nt && j < cap; j += gridDim.x * blockDim.x) {
    GemmTile g;
    g.expert = 0;
    g.row_start = j * bn;
    g.row_count = (int)min((int64_t)bn, T - (int64_t)j * bn);
    g.pad = 0;
    tiles[j] = g;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *count = min(nt, cap);
}

// ------------------------------------------------ peer-memory exchange ---
// Expert parallelism without a collective library: every rank owns one
// exchange buffer of the same layout, mapped into every other rank's address
// space (CUDA IPC over NVLink). Rank `me` stores the pairs it sends to rank r
// into r's buffer (recv_x / recv_meta block `me`), then the pair and slot
// counts and finally an epoch flag; r stores the partial rows it returns into
// me's buffer (back block r) and then a flag. Readers wait on the flags
// (bounded) and read the data through L2.
struct EpBufLayout {
  int64_t recv_x, recv_meta, back, counts, rows, flag_disp, flag_back, done, epoch, total;
};

__host__ __device__ inline EpBufLayout ep_buf_layout(int world, int64_t cap, int D, int K) {
  EpBufLayout b{};
  int64_t o = 0;
  auto take = [&](int64_t bytes) {
    const int64_t at = o;
    o += (bytes + 255) & ~(int64_t)255;
    return at;
  };
  b.recv_x = take((int64_t)world * cap * D * 2);
  b.recv_meta = take((int64_t)world * cap * K * 4);
  b.back = take((int64_t)world * cap * D * 2);
  b.counts = take((int64_t)world * 4);
  b.rows = take((int64_t)world * 4);
  b.flag_disp = take((int64_t)world * 4);
  b.flag_back = take((int64_t)world * 4);
  b.done = take(16);
  b.epoch = take(16);  // the device-resident step counter (steps called with epoch 0)
  b.total = o;
  return b;
}

constexpr int EP_MAX_WORLD = 64;
struct EpPeers {
  uint8_t* base[EP_MAX_WORLD];  // every rank's exchange buffer as seen from this GPU
};

// Flag values. A rank publishes the step's epoch (1 <= epoch < 2^31) when
// its side of the step went well, and the epoch with the top bit set (a
// poisoned flag) when its own status word was already non-zero: a wait that
// expired, or an index it skipped. Receivers that see a poisoned flag record
// kDevPeerFailed instead of reading the rows, so one rank's failure reaches
// every rank's status word rather than passing partial rows on as valid.
constexpr uint32_t EP_FLAG_POISON = 0x80000000u;

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Dispatch over peer memory: one warp per pair in destination order (pos in
// [offsets[r], offsets[r+1]) for rank r). The pair's x row and slot row go to
// rank r's recv block `me` at index pos - offsets[r]; pair_pos[f] (f = the
// pair's first (token, k)) becomes r * cap + that index, where the partial
// row will come back. The last CTA to finish publishes the counts and the
// flag on every rank.
__global__ void __launch_bounds__(256) ep_send_kernel(EpPeers peers, EpBufLayout bl, int me, int world, int64_t cap,
                                                      const uint16_t* __restrict__ x, int D, int K,
                                                      const int32_t* __restrict__ sorted,
                                                      const int32_t* __restrict__ offsets,
                                                      const int32_t* __restrict__ meta_local,
                                                      const int32_t* __restrict__ send_counts,
                                                      int32_t* __restrict__ pair_pos, uint32_t epoch,
                                                      int* __restrict__ done, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  if (epoch == 0) epoch = *reinterpret_cast<const volatile uint32_t*>(peers.base[me] + bl.epoch);
  __shared__ int s_off[EP_MAX_WORLD + 1];
  __shared__ int s_last;
  for (int i = threadIdx.x; i <= world; i += blockDim.x) s_off[i] = offsets[i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t npairs = s_off[world];
  for (int64_t pos = (int64_t)blockIdx.x * 8 + warp; pos < npairs; pos += (int64_t)gridDim.x * 8) {
    int r = 0;
    while (r + 1 < world && s_off[r + 1] <= pos) ++r;
    const int64_t pr = pos - s_off[r];
    const int32_t f = sorted[pos];
    if (pr >= cap || f < 0) {
      if (lane == 0) atomicCAS(status, 0, (int)kDevBadIndex);
      continue;
    }
    const int64_t t = f / K;
    if (lane == 0) pair_pos[f] = (int32_t)(r * cap + pr);
    const uint4* src = reinterpret_cast<const uint4*>(x + t * D);
    uint4* dst = reinterpret_cast<uint4*>(peers.base[r] + bl.recv_x + ((int64_t)me * cap + pr) * D * 2);
    for (int v = lane; v < D / 8; v += 32) dst[v] = __ldg(src + v);
    int32_t* dm = reinterpret_cast<int32_t*>(peers.base[r] + bl.recv_meta) + ((int64_t)me * cap + pr) * K;
    if (lane < K) dm[lane] = meta_local[pos * K + lane];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(done, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  if (threadIdx.x < world) {
    const int r = threadIdx.x;
    uint8_t* b = peers.base[r];
    reinterpret_cast<volatile int32_t*>(b + bl.counts)[me] = s_off[r + 1] - s_off[r];
    reinterpret_cast<volatile int32_t*>(b + bl.rows)[me] = send_counts[2 * r + 1];
    __threadfence_system();
    const uint32_t failed = *reinterpret_cast<volatile int*>(status) != 0 ? EP_FLAG_POISON : 0u;
    st_release_sys_u32(reinterpret_cast<uint32_t*>(b + bl.flag_disp) + me, epoch | failed);
  }
  if (threadIdx.x == 0) *done = 0;
}

// Steps called with epoch 0 use the device-resident counter in this rank's
// exchange buffer: the dispatch advances it first (one thread), and every
// kernel of the step reads it. Every rank advances its own counter once per
// step, so the counters agree as the host epochs would, and a captured CUDA
// graph of the step replays with a new epoch each time.
__global__ void ep_bump_epoch_kernel(uint8_t* local, EpBufLayout bl, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    uint32_t* slot = reinterpret_cast<uint32_t*>(local + bl.epoch);
    const uint32_t v = *slot + 1u;
    if (v >= EP_FLAG_POISON) atomicCAS(status, 0, (int)kDevBadIndex);  // 2^31 steps: recreate the comm
    else *slot = v;
  }
}

// One CTA: wait until every rank has published `epoch` in flags[0..world)
// (bounded; on expiry the status records a timeout and the data is not used).
// A poisoned flag of this epoch ends the wait for that rank with
// kDevPeerFailed in the status word.
__global__ void ep_wait_flags_kernel(const uint32_t* __restrict__ flags, int world, uint32_t epoch,
                                     const uint32_t* __restrict__ epoch_dev, unsigned long long limit_ns,
                                     int* status) {
  pdl_wait();
  pdl_launch_dependents();
  if (epoch == 0) epoch = *reinterpret_cast<const volatile uint32_t*>(epoch_dev);
  if (threadIdx.x < world) {
    const unsigned long long t0 = global_ns();
    for (uint32_t it = 0;; ++it) {
      const uint32_t v = ld_acquire_sys_u32(flags + threadIdx.x);
      const uint32_t e = v & ~EP_FLAG_POISON;
      if (e >= epoch) {
        if (v & EP_FLAG_POISON) atomicCAS(status, 0, (int)kDevPeerFailed);
        break;
      }
      if ((it & 63u) == 63u && global_ns() - t0 > limit_ns) {
        atomicCAS(status, 0, (int)kDevTimeout);
        break;
      }
    }
  }
  __threadfence_system();
}

// Receiving side over peer memory: slot f of the [world][cap][K] receive
// area is used when its pair index is below that source's count and the slot
// is filled; idx_local[f] = local expert or -1.
__global__ void ep_slot_expert_p2p_kernel(const int32_t* __restrict__ meta, const int32_t* __restrict__ counts,
                                          int world, int64_t cap, int K, int E_local,
                                          int32_t* __restrict__ idx_local, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t n = (int64_t)world * cap * K;
  for (int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; f < n; f += (int64_t)gridDim.x * blockDim.x) {
    const int64_t q = f / K;
    const int s = (int)(q / cap);
    const int64_t p = q - (int64_t)s * cap;
    int le = -1;
    const int c = __ldcg(counts + s);
    if (c < 0 || c > cap) {
      if (f == (int64_t)s * cap * K) atomicCAS(status, 0, (int)kDevBadIndex);
    } else if (p < c) {
      const int32_t m = __ldcg(meta + f);
      if (m >= 0) {
        le = m >> 16;
        if (le >= E_local) {
          atomicCAS(status, 0, (int)kDevBadIndex);
          le = -1;
        }
      }
    }
    idx_local[f] = le;
  }
}

// Pre-reduce each received pair and store the partial row straight into the
// owner's back block; the last CTA publishes the back flag on every rank.
__global__ void __launch_bounds__(256) ep_reduce_send_kernel(EpPeers peers, EpBufLayout bl, int me, int world,
                                                             int64_t cap, const uint16_t* __restrict__ y_sorted,
                                                             const int32_t* __restrict__ inv,
                                                             const int32_t* __restrict__ meta,
                                                             const int32_t* __restrict__ counts, int K, int D,
                                                             int64_t rows, uint32_t epoch, int* __restrict__ done,
                                                             int* status) {
  pdl_wait();
  pdl_launch_dependents();
  if (epoch == 0) epoch = *reinterpret_cast<const volatile uint32_t*>(peers.base[me] + bl.epoch);
  __shared__ int rws[RT_MAXK];
  __shared__ float wk[RT_MAXK];
  __shared__ int nk;
  __shared__ int s_last;
  const int64_t npairs = (int64_t)world * cap;
  for (int64_t q = blockIdx.x; q < npairs; q += gridDim.x) {
    const int s = (int)(q / cap);
    const int64_t p = q - (int64_t)s * cap;
    if (p >= __ldcg(counts + s)) continue;  // uniform over the CTA
    if (threadIdx.x == 0) {
      int n = 0;
      for (int j = 0; j < K; ++j) {
        const int32_t m = __ldcg(meta + q * K + j);
        if (m < 0) continue;
        const int r = inv[q * K + j];
        if (r < 0 || (int64_t)r >= rows) {
          atomicCAS(status, 0, (int)kDevBadIndex);
          continue;
        }
        rws[n] = r;
        wk[n] = bf16_bits_to_f32((uint16_t)(m & 0xFFFF));
        ++n;
      }
      nk = n;
    }
    __syncthreads();
    const int n = nk;
    uint16_t* dst = reinterpret_cast<uint16_t*>(peers.base[s] + bl.back) + ((int64_t)me * cap + p) * D;
    for (int v = threadIdx.x; v < D / 8; v += blockDim.x) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      weighted_rows_acc(y_sorted, rws, wk, n, D, v, acc);
      store_bf16x8(dst + 8 * v, acc);
    }
    __syncthreads();
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(done, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  if (threadIdx.x < world) {
    const uint32_t failed = *reinterpret_cast<volatile int*>(status) != 0 ? EP_FLAG_POISON : 0u;
    st_release_sys_u32(reinterpret_cast<uint32_t*>(peers.base[threadIdx.x] + bl.flag_back) + me, epoch | failed);
  }
  if (threadIdx.x == 0) *done = 0;
}

}  // namespace mlxr
