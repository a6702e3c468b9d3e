// Router, permutation and combine kernels of the MoE block.
//
// Router (Qwen35MoeBlock::forward, crates/mlxr-lm/src/qwen3_5/text/moe.rs:123-138):
// logits = x @ gate^T rounded to bf16, softmax (fp32 inside, bf16 out),
// top-K, renormalisation. The reference's argpartition leaves the order of
// equal probabilities undefined (crates/mlxr/src/ops/sort.rs:235-237); this
// implementation fixes the routing contract so that CPU and GPU agree bit for
// bit:
//   * logit(t, e): fp32 fma chains, one per lane j of a warp, over the 16-byte
//     chunks j, j+32, ... of the D axis (8 elements each, ascending), then an
//     xor butterfly over the 32 lanes (strides 16, 8, 4, 2, 1); + bias[e];
//     rounded to bf16.
//   * softmax: exact max, exp_route(l - max), lane sums over e = j, j+32, ...
//     then the same butterfly, IEEE division, bf16 probabilities.
//   * top-K by (probability desc, expert asc); denominator summed in rank
//     order; weights = bf16(p / bf16(denominator)).
// Permutation (gather_sort / scatter_unsort, crates/mlxr-lm/src/nn/switch.rs:
// 499-517): the flat rows f = t*K + k are stably sorted by expert (a counting
// sort: per-block histograms, one scan, stable in-block ranks by
// __match_any_sync); the expert-sorted copy of x is gathered in the same pass
// with 16-byte loads.
// Combine (combine_with_weights, switch.rs:223-234, plus the shared branch
// and final add, moe.rs:118-120,145): out[t] = sum_k w[t,k] * y[inv[t*K+k]]
// (+ sigmoid(x . g_s) * shared(x)), fp32 accumulation, one bf16 rounding.
#pragma once

#include "common.cuh"
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

// --------------------------------------------------------- logits -------
// A warp computes RT_TOK tokens x RT_EXP experts; a CTA of 8 warps covers
// RT_TOK tokens x 64 experts.
constexpr int RT_TOK = 4, RT_EXP = 8;

__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t* __restrict__ x, int64_t T, int D,
                                                           const uint16_t* __restrict__ wg, int E,
                                                           const float* __restrict__ bias,
                                                           uint16_t* __restrict__ logits) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t0 = (int64_t)blockIdx.y * RT_TOK;
  const int e0 = (blockIdx.x * 8 + warp) * RT_EXP;
  if (e0 >= E) return;
  float acc[RT_TOK][RT_EXP];
#pragma unroll
  for (int i = 0; i < RT_TOK; ++i)
#pragma unroll
    for (int j = 0; j < RT_EXP; ++j) acc[i][j] = 0.0f;
  const uint4* xr[RT_TOK];
  const uint4* wr[RT_EXP];
#pragma unroll
  for (int i = 0; i < RT_TOK; ++i) xr[i] = reinterpret_cast<const uint4*>(x + (t0 + i < T ? t0 + i : T - 1) * D);
#pragma unroll
  for (int j = 0; j < RT_EXP; ++j) wr[j] = reinterpret_cast<const uint4*>(wg + (int64_t)(e0 + j < E ? e0 + j : E - 1) * D);
  const int nchunks = D / 8;
  for (int c = lane; c < nchunks; c += 32) {
    uint4 xv[RT_TOK], wv[RT_EXP];
#pragma unroll
    for (int i = 0; i < RT_TOK; ++i) xv[i] = __ldg(xr[i] + c);
#pragma unroll
    for (int j = 0; j < RT_EXP; ++j) wv[j] = __ldg(wr[j] + c);
#pragma unroll
    for (int el = 0; el < 8; ++el) {
      float xf[RT_TOK], wf[RT_EXP];
#pragma unroll
      for (int i = 0; i < RT_TOK; ++i) {
        const uint32_t wd = el < 2 ? xv[i].x : el < 4 ? xv[i].y : el < 6 ? xv[i].z : xv[i].w;
        xf[i] = (el & 1) ? bf_hi(wd) : bf_lo(wd);
      }
#pragma unroll
      for (int j = 0; j < RT_EXP; ++j) {
        const uint32_t wd = el < 2 ? wv[j].x : el < 4 ? wv[j].y : el < 6 ? wv[j].z : wv[j].w;
        wf[j] = (el & 1) ? bf_hi(wd) : bf_lo(wd);
      }
#pragma unroll
      for (int i = 0; i < RT_TOK; ++i)
#pragma unroll
        for (int j = 0; j < RT_EXP; ++j) acc[i][j] = __fmaf_rn(xf[i], wf[j], acc[i][j]);
    }
  }
  float mine = 0.0f;
#pragma unroll
  for (int i = 0; i < RT_TOK; ++i)
#pragma unroll
    for (int j = 0; j < RT_EXP; ++j) {
      float v = acc[i][j];
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, s));
      if (lane == i * RT_EXP + j) mine = v;
    }
  const int i = lane / RT_EXP, j = lane % RT_EXP;
  const int64_t t = t0 + i;
  const int e = e0 + j;
  if (t < T && e < E) {
    const float b = bias ? bias[e] : 0.0f;
    logits[t * E + e] = f32_to_bf16_bits(__fadd_rn(mine, b));
  }
}

// ------------------------------------------------ softmax + top-K -------
constexpr int RT_MAXV = 32;  // E <= 1024
constexpr int RT_MAXK = 32;

struct SharedGateArgs {
  const uint32_t* w;   // [1, D*bits/32]
  const uint16_t* s;   // [1, D/64]
  const uint16_t* b;
  int bits;
};

// One warp per token.
__global__ void __launch_bounds__(256) router_topk_kernel(const uint16_t* __restrict__ logits, int64_t T, int E,
                                                         int K, int renorm, int32_t* __restrict__ idx_out,
                                                         uint16_t* __restrict__ w_out, uint16_t* __restrict__ probs_out,
                                                         const uint16_t* __restrict__ x, int D, SharedGateArgs sg,
                                                         float* __restrict__ sig_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 8 + warp;
  if (t >= T) return;
  const uint16_t* lrow = logits + t * E;
  float lv[RT_MAXV];
  float mx = -INFINITY;
#pragma unroll
  for (int m = 0; m < RT_MAXV; ++m) {
    const int e = lane + 32 * m;
    lv[m] = e < E ? bf16_bits_to_f32(lrow[e]) : -INFINITY;
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
  if (sig_out) {
    // sigmoid(x . dequant(g_s)) for the shared expert (moe.rs:119-120).
    const int per = 32 / sg.bits;
    const uint32_t mask = (1u << sg.bits) - 1u;
    const uint16_t* xr = x + t * D;
    float z = 0.0f;
    for (int d = lane; d < D; d += 32) {
      const uint32_t q = (__ldg(sg.w + d / per) >> ((d % per) * sg.bits)) & mask;
      const float wv = __fmaf_rn(bf16_bits_to_f32(__ldg(sg.s + d / 64)), (float)q, bf16_bits_to_f32(__ldg(sg.b + d / 64)));
      z = fmaf(bf16_bits_to_f32(__ldg(xr + d)), wv, z);
    }
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) z += __shfl_xor_sync(0xffffffffu, z, s);
    if (lane == 0) sig_out[t] = 1.0f / (1.0f + __expf(-z));
  }
}

// ------------------------------------------------------- permutation ----
constexpr int PERM_ROWS = 2048;  // flat rows per permute block (8 warps x 256)
constexpr int PERM_MAX_E = 1024;

__global__ void __launch_bounds__(256) permute_count_kernel(const int32_t* __restrict__ idx, int64_t R, int E,
                                                           int32_t* __restrict__ block_counts, int* status) {
  extern __shared__ int hist[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * PERM_ROWS;
  for (int i = threadIdx.x; i < PERM_ROWS; i += blockDim.x) {
    const int64_t f = base + i;
    if (f < R) {
      const int e = idx[f];
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
};

// Single CTA of 1024 threads: expert totals, offsets, per-block bases and
// the GEMM tile lists (one per tile width) plus the dense shared-expert list.
__global__ void __launch_bounds__(1024) permute_scan_kernel(const int32_t* __restrict__ block_counts, int nblk, int E,
                                                           int64_t T, int32_t* __restrict__ block_base,
                                                           int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                                                           TileListOut l1, TileListOut l2, TileListOut lsh) {
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
  TileListOut lists[2] = {l1, l2};
  for (int li = 0; li < 2; ++li) {
    const TileListOut L = lists[li];
    const int nt = e < E ? (tot + L.bn - 1) / L.bn : 0;
    const int toff = block_exclusive_scan(nt, warp_sums, &total);
    for (int j = 0; j < nt; ++j) {
      GemmTile g;
      g.expert = e;
      g.row_start = off + j * L.bn;
      g.row_count = min(L.bn, tot - j * L.bn);
      g.pad = 0;
      L.tiles[toff + j] = g;
    }
    if (e == 0) *L.count = total;
  }
  if (lsh.tiles) {
    const int nt = (int)((T + lsh.bn - 1) / lsh.bn);
    for (int j = e; j < nt; j += blockDim.x) {
      GemmTile g;
      g.expert = 0;
      g.row_start = j * lsh.bn;
      g.row_count = (int)min((int64_t)lsh.bn, T - (int64_t)j * lsh.bn);
      g.pad = 0;
      lsh.tiles[j] = g;
    }
    if (e == 0) *lsh.count = nt;
  }
}

// Stable in-block ranks. 8 warps; warp w owns flat rows
// [blk*2048 + w*256, +256).
__global__ void __launch_bounds__(256) permute_scatter_kernel(const int32_t* __restrict__ idx, int64_t R, int E,
                                                             const int32_t* __restrict__ block_base,
                                                             int32_t* __restrict__ sorted_rows,
                                                             int32_t* __restrict__ inv) {
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
    if (e >= 0) pos = wcnt[warp * E + e] + __popc(peers & lt_mask);
    if (pos >= R) pos = -1;  // cannot happen for consistent counts; never write out of range
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) wcnt[warp * E + e] += __popc(peers);
    __syncwarp();
    if (e >= 0) {
      sorted_rows[pos] = (int32_t)f;
      inv[f] = pos;
    }
  }
}

// x_sorted[pos] = x[sorted_rows[pos] / K] (sorted_rows NULL: the identity),
// one warp per row, 16-byte loads and stores, the whole grid streaming. With
// kperm the 8 elements of every 16-byte chunk are stored in the 4-bit
// operand order {0,4,1,5,2,6,3,7} the grouped GEMM's dequantiser produces.
__global__ void __launch_bounds__(256) permute_gather_kernel(const int32_t* __restrict__ sorted_rows, int64_t R, int K,
                                                            const uint16_t* __restrict__ x, int D, int kperm,
                                                            uint16_t* __restrict__ x_sorted) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dvec = D / 8;
  for (int64_t pos = (int64_t)blockIdx.x * 8 + warp; pos < R; pos += (int64_t)gridDim.x * 8) {
    int64_t src_row = pos;
    if (sorted_rows) {
      const int32_t f = sorted_rows[pos];
      if (f < 0 || (int64_t)f >= R) continue;
      src_row = f / K;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + src_row * D);
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

// ------------------------------------------------------------ combine ---
__global__ void __launch_bounds__(128) combine_kernel(const uint16_t* __restrict__ y_sorted,
                                                     const int32_t* __restrict__ inv, const uint16_t* __restrict__ w,
                                                     int K, int D, int64_t T, const uint16_t* __restrict__ y_sh,
                                                     const float* __restrict__ sig, uint16_t* __restrict__ out,
                                                     int* status) {
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
    for (int k = 0; k < K; ++k) {
      const uint4 yv = __ldg(reinterpret_cast<const uint4*>(y_sorted + (int64_t)rows[k] * D) + v);
      const uint32_t ww[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = fmaf(wk[k], bf_lo(ww[i]), acc[2 * i]);
        acc[2 * i + 1] = fmaf(wk[k], bf_hi(ww[i]), acc[2 * i + 1]);
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

}  // namespace mlxr
