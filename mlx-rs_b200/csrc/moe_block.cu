// MoE block orchestration and its C ABI: Qwen35MoeBlock::forward
// (crates/mlxr-lm/src/qwen3_5/text/moe.rs:116-146) on one device.
//
// Stream of work for x [T, D]:
//   router_logits -> router_topk (+ shared-gate sigmoid)
//   permute_count -> permute_scan (offsets, tile lists) -> permute_scatter
//   grouped GEMM gate|up + SwiGLU  (x_sorted -> h_sorted)
//   grouped GEMM down              (h_sorted -> y_sorted)
//   [shared expert: dense GEMMs over x with the same kernels]
//   combine (+ sigmoid-gated shared expert)
// model_kind 1 runs the Gemma 4 MoE branch (gemma4/text/text.rs:901-916) on
// the same stages: the input RMS norms first (router input, experts input),
// Gemma routing (top-k of the scores, softmax over k x per-expert scale),
// the experts' normed rows permuted, packed gate_up_proj with GeGLU, no
// shared expert.
// All scratch lives in the caller's workspace; nothing is allocated here.
#include <algorithm>
#include <cstring>
#include <type_traits>
#include <mutex>

#include "common.cuh"
#include "gemm_launch.h"
#include "router_tc.h"
#include "routing.cuh"

namespace mlxr {

static __device__ int g_op_status;

int* op_status_word() {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_op_status);
  if (e != cudaSuccess) {
    check_cuda(e, "cudaGetSymbolAddress(op status)");
    return nullptr;
  }
  return static_cast<int*>(p);
}

// Optional per-thread stage events (a profiling hook): when set, the block
// forward records events[i] on its stream at each stage boundary.
static thread_local cudaEvent_t t_stage_events[8];
static thread_local int t_stage_count = 0;

static inline void stage_mark(int i, cudaStream_t st) {
  // External records become event nodes when the stream is being captured.
  if (i < t_stage_count && t_stage_events[i]) cudaEventRecordWithFlags(t_stage_events[i], st, cudaEventRecordExternal);
}

static inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// The first 256 bytes of every workspace: the device status word, then the
// split router's per-token-block counters (ints 1..16), then the grouped
// GEMM launches' work-queue counters (ints 32..39), all cleared by the call
// that starts a forward (or an expert-parallel step).
constexpr size_t kStatusSlotBytes = 256;
constexpr int kSchedExperts1 = 32, kSchedExperts2 = 34, kSchedShared1 = 36, kSchedShared2 = 38;
constexpr int kSplitRouterMaxT = 64;   // batches up to this size use router_split_kernel

struct Layout {
  // R: flat (token, k) rows; rows: expert rows the buffers hold (R, or fewer
  // when some flat rows are skipped, as on the receiving side of expert parallelism).
  int64_t T = 0, R = 0, rows = 0, rows_pad = 0, sh_rows_pad = 0;
  int E = 0, K = 0, D = 0, I = 0, Is = 0, nblk = 0;
  int bn1 = 0, bn2 = 0, bns = 0;
  int s1 = 1, s2 = 1;          // split-K factors of the gate/up and down GEMMs
  int split_rows = 0;          // row slices the split buffers hold
  int fuse = 0;                // gate/up and down in one launch (same tile list, no split)
  int kind = 0;                // config model_kind (1 = Gemma 4 branch)
  int max_t1 = 0, max_t2 = 0, max_tsh = 0;
  size_t status = 0, logits = 0, idx = 0, w = 0, sig = 0, bcounts = 0, bbase = 0, counts = 0, offsets = 0,
         sorted = 0, inv = 0, t1 = 0, n1 = 0, t2 = 0, n2 = 0, tsh = 0, nsh = 0, xs = 0, h = 0, y = 0, xpad = 0,
         hsh = 0, ysh = 0, part = 0, cnt = 0, ready = 0, gxr = 0, gxe = 0, rtc = 0, total = 0;
};

// Token-tile width from the mean number of rows per expert.
static int pick_bn(double avg_rows, int max_bn) {
  int bn;
  if (avg_rows <= 12) bn = 16;
  else if (avg_rows <= 24) bn = 32;
  else if (avg_rows <= 48) bn = 64;
  else if (avg_rows <= 160) bn = 128;
  else bn = 256;
  return bn < max_bn ? bn : max_bn;
}

static int shared_gate_bits(const mlxr_cu_moe_config* c) {
  return c->shared_gate_bits ? c->shared_gate_bits : c->shared_bits;
}

static int validate(const mlxr_cu_moe_config* c, int64_t T) {
  MLXR_CHECK_ARG(c != nullptr, "moe: null config");
  MLXR_CHECK_ARG(T >= 0, "moe: negative token count");
  MLXR_CHECK_ARG(c->hidden_size > 0 && c->hidden_size % 128 == 0, "moe: hidden_size=%d must be a positive multiple of 128",
                 c->hidden_size);
  MLXR_CHECK_ARG(c->num_experts >= 1 && c->num_experts <= PERM_MAX_E, "moe: num_experts=%d must be in [1, %d]",
                 c->num_experts, PERM_MAX_E);
  MLXR_CHECK_ARG(c->num_experts_per_tok >= 1 && c->num_experts_per_tok <= RT_MAXK &&
                     c->num_experts_per_tok <= c->num_experts,
                 "moe: num_experts_per_tok=%d must be in [1, min(32, num_experts)]", c->num_experts_per_tok);
  MLXR_CHECK_ARG(c->moe_intermediate_size > 0 && c->moe_intermediate_size % 128 == 0,
                 "moe: moe_intermediate_size=%d must be a positive multiple of 128", c->moe_intermediate_size);
  MLXR_CHECK_ARG(c->shared_expert_intermediate_size >= 0 && c->shared_expert_intermediate_size % 128 == 0,
                 "moe: shared_expert_intermediate_size=%d must be a multiple of 128", c->shared_expert_intermediate_size);
  if (c->group_size != 64)
    return set_error(MLXR_CU_ERR_UNSUPPORTED, "moe: group_size=%d is not supported (64)", c->group_size);
  if (c->model_kind != 0 && c->model_kind != 1)
    return set_error(MLXR_CU_ERR_UNSUPPORTED, "moe: model_kind=%d is not supported (0 Qwen 3.5/3.6, 1 Gemma 4)",
                     c->model_kind);
  if (c->model_kind == 1) {
    MLXR_CHECK_ARG(c->shared_expert_intermediate_size == 0,
                   "moe: the Gemma 4 branch has no shared expert (shared_expert_intermediate_size=%d)",
                   c->shared_expert_intermediate_size);
    MLXR_CHECK_ARG(c->rms_norm_eps >= 0.0f && c->rms_norm_eps < 1.0f, "moe: rms_norm_eps=%g out of range",
                   (double)c->rms_norm_eps);
  }
  if (c->bits != 4 && c->bits != 8) return set_error(MLXR_CU_ERR_UNSUPPORTED, "moe: bits=%d is not supported (4, 8)", c->bits);
  if (c->shared_expert_intermediate_size > 0 && c->shared_bits != 4 && c->shared_bits != 8)
    return set_error(MLXR_CU_ERR_UNSUPPORTED, "moe: shared_bits=%d is not supported (4, 8)", c->shared_bits);
  if (c->shared_expert_intermediate_size > 0 && c->shared_gate_bits != 0 && c->shared_gate_bits != 4 &&
      c->shared_gate_bits != 8)
    return set_error(MLXR_CU_ERR_UNSUPPORTED, "moe: shared_gate_bits=%d is not supported (0, 4, 8)",
                     c->shared_gate_bits);
  MLXR_CHECK_ARG(T * (int64_t)c->num_experts_per_tok < (int64_t)1 << 30, "moe: T*K=%lld too large",
                 (long long)(T * c->num_experts_per_tok));
  return MLXR_CU_OK;
}

// Split-K factor for a GEMM with `items` work items of `ksteps` k-steps: only
// when the items would leave more than half of the SMs idle.
static int pick_splits(int64_t items, int ksteps) {
  const int sms = num_sms_current();
  if (items <= 0 || items * 2 > sms) return 1;
  int sp = (int)(sms / items);
  if (sp > ksteps / 4) sp = ksteps / 4;
  if (sp > 8) sp = 8;
  return sp < 1 ? 1 : sp;
}

// rows_cap: expert rows the buffers hold (default T*K); bn_rows: the rows
// the tile widths are chosen for (default: rows_cap).
static Layout make_layout(const mlxr_cu_moe_config* c, int64_t T, int64_t rows_cap = -1, int64_t bn_rows = -1) {
  Layout L;
  L.T = T;
  L.E = c->num_experts;
  L.K = c->num_experts_per_tok;
  L.D = c->hidden_size;
  L.I = c->moe_intermediate_size;
  L.Is = c->shared_expert_intermediate_size;
  L.kind = c->model_kind;
  L.R = T * L.K;
  L.rows = rows_cap >= 0 && rows_cap < L.R ? rows_cap : L.R;
  L.rows_pad = L.rows > 256 ? L.rows : 256;
  L.sh_rows_pad = T > 256 ? T : 256;
  L.nblk = (int)((L.R + PERM_ROWS - 1) / PERM_ROWS);
  if (L.nblk < 1) L.nblk = 1;
  const double avg = L.E > 0 ? (double)(bn_rows >= 0 ? bn_rows : L.rows) / L.E : 0.0;
  L.bn1 = pick_bn(avg, 128);
  L.bn2 = pick_bn(avg, (L.D % 256 == 0) ? 128 : 256);
  L.bns = pick_bn((double)T, 64);
  L.max_t1 = (int)(L.E + (L.rows + L.bn1 - 1) / L.bn1 + 1);
  L.max_t2 = (int)(L.E + (L.rows + L.bn2 - 1) / L.bn2 + 1);
  L.max_tsh = (int)((T + L.bns - 1) / L.bns + 1);
  // Split-K for small batches (the whole permutation in one CTA, which also
  // clears the split counters): expected non-empty experts min(E, rows).
  const int mt1 = L.I / 128, mt2 = (L.D % 256 == 0) ? L.D / 256 : L.D / 128;
  if (L.nblk == 1 && L.rows > 0) {
    const int64_t used = L.rows < L.E ? L.rows : L.E;
    if (L.bn1 <= 32) L.s1 = pick_splits(used * mt1, L.D / 64);
    if (L.bn2 <= 32) L.s2 = pick_splits(used * mt2, L.I / 64);
  }
  // One launch for both GEMMs when they share the tile list (equal token-tile
  // widths), the down weight goes in row pairs, and neither is split; only
  // for decode-width tiles, where the gate|up tail and the second launch's
  // ramp are a visible share of the time (measured: no gain for prefill).
  L.fuse = (L.s1 == 1 && L.s2 == 1 && L.D % 256 == 0 && L.bn1 <= 32 && L.bn1 == (L.bn2 < 128 ? L.bn2 : 128)) ? 1 : 0;
  if (L.s1 > 1 || L.s2 > 1) {
    // Tiles per GEMM are at most rows/bn + (non-empty experts) + 1.
    const int64_t t1 = std::min<int64_t>(L.max_t1, L.rows / L.bn1 + std::min<int64_t>(L.rows, L.E) + 1);
    const int64_t t2 = std::min<int64_t>(L.max_t2, L.rows / L.bn2 + std::min<int64_t>(L.rows, L.E) + 1);
    L.split_rows = (int)std::max(t1 * mt1, t2 * mt2);
  }
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align256(o + (bytes ? bytes : 1));
    return at;
  };
  L.status = take(kStatusSlotBytes);  // status word, then the split router's block counters
  L.logits = take((size_t)T * L.E * 2);
  L.idx = take((size_t)L.R * 4);
  L.w = take((size_t)L.R * 2);
  L.sig = take((size_t)T * 4);
  L.bcounts = take((size_t)L.nblk * L.E * 4);
  L.bbase = take((size_t)L.nblk * L.E * 4);
  L.counts = take((size_t)L.E * 4);
  L.offsets = take((size_t)(L.E + 1) * 4);
  L.sorted = take((size_t)L.R * 4);
  L.inv = take((size_t)L.R * 4);
  L.t1 = take((size_t)L.max_t1 * sizeof(GemmTile));
  L.n1 = take(4);
  L.t2 = take((size_t)L.max_t2 * sizeof(GemmTile));
  L.n2 = take(4);
  L.tsh = take((size_t)L.max_tsh * sizeof(GemmTile));
  L.nsh = take(4);
  L.xs = take((size_t)L.rows_pad * L.D * 2);
  L.h = take((size_t)L.rows_pad * L.I * 2);
  L.y = take((size_t)L.rows * L.D * 2);
  if (L.Is > 0) {
    L.xpad = take((T < 256 || c->shared_bits == 4) ? (size_t)L.sh_rows_pad * L.D * 2 : 0);
    L.hsh = take((size_t)L.sh_rows_pad * L.Is * 2);
    L.ysh = take((size_t)T * L.D * 2);
  }
  if (L.fuse) L.ready = take((size_t)L.max_t1 * sizeof(int32_t));
  if (L.kind == 1) {  // Gemma 4: the router's and the experts' RMS-normed inputs
    L.gxr = take((size_t)T * L.D * 2);
    L.gxe = take((size_t)T * L.D * 2);
  }
  // The tensor-core router's digit planes: in the x_sorted buffer when they
  // fit (the permute fills it only after the router has finished), else apart.
  if (T > kSplitRouterMaxT && router_tc_supported(L.D)) {
    const size_t xs_bytes = (size_t)L.rows_pad * L.D * 2;
    const size_t need = router_tc_layout(T, L.E, L.D, xs_bytes).total;
    L.rtc = need <= xs_bytes ? L.xs : take(need);
  }
  if (L.split_rows > 0) {
    const int smax = L.s1 > L.s2 ? L.s1 : L.s2;
    const int bmax = L.bn1 > L.bn2 ? L.bn1 : L.bn2;
    L.part = take((size_t)L.split_rows * smax * 4 * 2 * bmax * 32 * sizeof(float));
    L.cnt = take((size_t)L.split_rows * 4 * sizeof(int32_t));
  }
  L.total = o;
  return L;
}

template <typename P>
static inline P* at(void* ws, size_t off) {
  return reinterpret_cast<P*>(static_cast<uint8_t*>(ws) + off);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int check_ws(const Layout& L, void* ws, size_t bytes) {
  if (!ws) return set_error(MLXR_CU_ERR_WORKSPACE, "moe: workspace is NULL (need %zu bytes)", L.total);
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return set_error(MLXR_CU_ERR_WORKSPACE, "moe: workspace %p is not 256-byte aligned", ws);
  if (bytes < L.total) return set_error(MLXR_CU_ERR_WORKSPACE, "moe: workspace has %zu bytes, needs %zu", bytes, L.total);
  return MLXR_CU_OK;
}

// ------------------------------------------------------------ stages ----
static int run_router(const mlxr_cu_moe_config* c, const mlxr_cu_moe_weights* wt, const Layout& L, const void* x,
                      void* ws, uint16_t* logits, uint16_t* probs, cudaStream_t st) {
  if (L.T == 0) return MLXR_CU_OK;
  MLXR_CHECK_ARG(wt && wt->router_weight, "moe: router weight is NULL");
  MLXR_CHECK_ARG(aligned16(x) && aligned16(wt->router_weight), "moe: x and the router weight must be 16-byte aligned");
  SharedGateArgs sg{nullptr, nullptr, nullptr, 8};
  float* sig = nullptr;
  if (L.Is > 0) {
    MLXR_CHECK_ARG(wt->shared_expert_gate.weight && wt->shared_expert_gate.scales && wt->shared_expert_gate.biases,
                   "moe: shared_expert_gate is NULL");
    sg.w = wt->shared_expert_gate.weight;
    sg.s = static_cast<const uint16_t*>(wt->shared_expert_gate.scales);
    sg.b = static_cast<const uint16_t*>(wt->shared_expert_gate.biases);
    sg.bits = shared_gate_bits(c);
    sig = at<float>(ws, L.sig);
  }
  const uint16_t* xp = static_cast<const uint16_t*>(x);
  const uint16_t* wg = static_cast<const uint16_t*>(wt->router_weight);
  // Gemma 4: route the RMS-normed input (no bias) and write the experts'
  // normed input beside it; the routing ends in router_post.
  const float* rbias = wt->router_bias;
  const uint16_t* es = nullptr;
  if (c->model_kind == 1) {
    MLXR_CHECK_ARG(wt->router_norm && wt->expert_scale && wt->experts_norm,
                   "moe: Gemma 4 router_norm / expert_scale / experts_norm is NULL");
    MLXR_CHECK_ARG(aligned16(wt->router_norm) && aligned16(wt->experts_norm),
                   "moe: Gemma 4 router_norm and experts_norm must be 16-byte aligned");
    uint16_t* gxr = at<uint16_t>(ws, L.gxr);
    launch_pdl(gemma4_norm_kernel, (unsigned)((L.T + G4_NORM_WARPS - 1) / G4_NORM_WARPS), G4_NORM_WARPS * 32, 0, st, xp,
               L.T, L.D, c->rms_norm_eps, static_cast<const uint16_t*>(wt->router_norm),
               static_cast<const uint16_t*>(wt->experts_norm), gxr, at<uint16_t>(ws, L.gxe));
    MLXR_LAUNCH_CHECK("gemma4_norm_kernel");
    xp = gxr;
    rbias = nullptr;
    es = static_cast<const uint16_t*>(wt->expert_scale);
  }
  if (L.T > kSplitRouterMaxT && router_tc_supported(L.D)) {
    // The logits on the int8 tensor cores (router_tc.cu): from the kernel's
    // epilogue, or (split-K form) from its partial digit sums; then one
    // warp per token routes them.
    uint16_t* lg = logits ? logits : at<uint16_t>(ws, L.logits);
    const size_t budget = (size_t)L.rows_pad * L.D * 2;  // the same budget the workspace layout used
    const RouterTcLayout R = router_tc_layout(L.T, L.E, L.D, budget);
    RouterTcProblem rp{xp, L.T, wg, L.E, L.D, rbias, lg, at<void>(ws, L.rtc), at<int>(ws, L.status), budget};
    if (int rc = launch_router_tc(rp, st)) return rc;
    if (R.split) {
      uint8_t* rb = at<uint8_t>(ws, L.rtc);
      const int64_t n = L.T * (int64_t)L.E;
      launch_pdl(logits_from_partials_kernel, (unsigned)((n + 255) / 256), 256, 0, st,
                 reinterpret_cast<const int32_t*>(rb + R.part), R.splits, reinterpret_cast<const int2*>(rb + R.xinfo),
                 reinterpret_cast<const int2*>(rb + R.winfo), xp, wg, rbias, L.T, L.D, L.E, lg);
      MLXR_LAUNCH_CHECK("logits_from_partials_kernel");
    }
    const unsigned grid = (unsigned)((L.T + RT_ROUTE_WARPS - 1) / RT_ROUTE_WARPS);
    const size_t smem = RT_ROUTE_WARPS * L.E * sizeof(float);
    // lane arrays of the routing sized for E (registers, not local memory)
    auto route = [&](auto mv) {
      constexpr int MV = decltype(mv)::value;
      launch_pdl(route_rows_kernel<MV>, grid, RT_ROUTE_WARPS * 32, smem, st, lg, xp, L.T, L.D, L.E, L.K,
                 c->norm_topk_prob, at<int32_t>(ws, L.idx), at<uint16_t>(ws, L.w), probs, sg, sig, es);
    };
    if (L.E <= 128) route(std::integral_constant<int, 4>{});
    else if (L.E <= 256) route(std::integral_constant<int, 8>{});
    else if (L.E <= 512) route(std::integral_constant<int, 16>{});
    else route(std::integral_constant<int, 32>{});
    MLXR_LAUNCH_CHECK("route_rows_kernel");
    return MLXR_CU_OK;
  }
  // Small batches (latency: the tensor-core form costs more launches) and D
  // beyond the tensor-core path: fp64 sums on the CUDA cores. Up to 64
  // tokens the logits are spread over many CTAs and the last CTA of each
  // token block routes it; beyond, one token per CTA.
  if (L.T <= kSplitRouterMaxT) {
    // 2 experts per warp; 1, 2 or 4 tokens per block.
    const int tpb = L.T <= 4 ? 1 : L.T <= 16 ? 2 : 4;
    constexpr int EPW = 2;
    const int ngroups = (L.E + EPW - 1) / EPW;
    const dim3 grid((unsigned)((ngroups + RS_WARPS - 1) / RS_WARPS), (unsigned)((L.T + tpb - 1) / tpb));
    uint16_t* lg = logits ? logits : at<uint16_t>(ws, L.logits);
    int* counter = at<int>(ws, L.status) + 1;
    const size_t smem = (size_t)tpb * L.E * sizeof(float);
    const float* rb = rbias;
    int32_t* io = at<int32_t>(ws, L.idx);
    uint16_t* wo = at<uint16_t>(ws, L.w);
    const int rn = c->norm_topk_prob;
    if (tpb == 1)
      launch_pdl(router_split_kernel<1, EPW, 8>, grid, RS_WARPS * 32, smem, st, xp, L.T, L.D, wg, L.E, rb, L.K, rn, io, wo, lg,
                                                                        probs, sg, sig, counter, es);
    else if (tpb == 2)
      launch_pdl(router_split_kernel<2, EPW, 6>, grid, RS_WARPS * 32, smem, st, xp, L.T, L.D, wg, L.E, rb, L.K, rn, io, wo, lg,
                                                                        probs, sg, sig, counter, es);
    else
      launch_pdl(router_split_kernel<4, EPW, 4>, grid, RS_WARPS * 32, smem, st, xp, L.T, L.D, wg, L.E, rb, L.K, rn, io, wo, lg,
                                                                        probs, sg, sig, counter, es);
    MLXR_LAUNCH_CHECK("router_split_kernel");
    return MLXR_CU_OK;
  } else {
    launch_pdl(router_fused_kernel<1>, (unsigned)L.T, RT_THREADS, L.E * sizeof(float), st,
        xp, L.T, L.D, wg, L.E, rbias, L.K, c->norm_topk_prob, at<int32_t>(ws, L.idx), at<uint16_t>(ws, L.w),
        logits, probs, sg, sig, es);
  }
  MLXR_LAUNCH_CHECK("router_fused_kernel");
  return MLXR_CU_OK;
}

// skip != 0: rows with a negative index are left out (see permute_count_kernel).
static int run_permute(const Layout& L, const int32_t* idx, const void* x, void* ws, int32_t* counts, int32_t* offsets,
                       int32_t* sorted, int32_t* inv, uint16_t* xs, int kperm, cudaStream_t st, int skip = 0,
                       int coherent = 0) {
  int* status = at<int>(ws, L.status);
  TileListOut l1{at<GemmTile>(ws, L.t1), at<int32_t>(ws, L.n1), L.bn1, L.max_t1};
  TileListOut l2{at<GemmTile>(ws, L.t2), at<int32_t>(ws, L.n2), L.bn2, L.max_t2};
  TileListOut lsh{L.Is > 0 ? at<GemmTile>(ws, L.tsh) : nullptr, at<int32_t>(ws, L.nsh), L.bns, L.max_tsh};
  // Counters the expert GEMMs expect at zero: split-K arrivals or the fused
  // launch's per-tile readiness.
  int32_t* zero = nullptr;
  int nzero = 0;
  if (L.split_rows > 0) {
    zero = at<int32_t>(ws, L.cnt);
    nzero = L.split_rows * 4;
  } else if (L.fuse) {
    zero = at<int32_t>(ws, L.ready);
    nzero = L.max_t1;
  }
  // Up to this many rows the one-CTA permute also gathers them (one launch
  // fewer on the decode path).
  constexpr int64_t kGatherInSmall = 16;
  bool gathered = false;
  if (L.nblk == 1) {
    // Every flat row fits one block: count, scan, tile lists and ranks in one CTA.
    const bool g = xs && !skip && L.R > 0 && L.rows == L.R && L.R <= kGatherInSmall;
    launch_pdl(permute_small_kernel, 1, 1024, 9 * L.E * sizeof(int), st, idx, L.R, L.E, L.T, counts, offsets, sorted, inv, l1,
               l2, lsh, skip, status, zero, nzero, g ? static_cast<const uint16_t*>(x) : nullptr, L.D, L.K, kperm,
               g ? xs : nullptr);
    MLXR_LAUNCH_CHECK("permute_small_kernel");
    gathered = g;
  } else {
    launch_pdl(permute_count_kernel, L.nblk, 256, L.E * sizeof(int), st, idx, L.R, L.E, at<int32_t>(ws, L.bcounts), skip,
                                                                 status);
    MLXR_LAUNCH_CHECK("permute_count_kernel");
    launch_pdl(permute_scan_kernel, 1, 1024, 0, st, zero, nzero, at<int32_t>(ws, L.bcounts), L.nblk, L.E, L.T, at<int32_t>(ws, L.bbase),
                                            counts, offsets, l1, l2, lsh);
    MLXR_LAUNCH_CHECK("permute_scan_kernel");
    launch_pdl(permute_scatter_kernel, L.nblk, 256, 8 * L.E * sizeof(int), st, idx, L.R, L.E, at<int32_t>(ws, L.bbase),
                                                                       sorted, inv);
    MLXR_LAUNCH_CHECK("permute_scatter_kernel");
  }
  if (xs && !gathered && L.R > 0 && L.rows > 0) {
    const int64_t gblocks = (L.rows + 7) / 8;
    const int gather_grid = (int)(gblocks < 4 * 148 ? gblocks : 4 * 148);
    launch_pdl(permute_gather_kernel, gather_grid, 256, 0, st, sorted, L.rows, L.R, L.K, static_cast<const uint16_t*>(x), L.D,
                                                       kperm, xs, skip ? offsets + L.E : nullptr, status, coherent);
    MLXR_LAUNCH_CHECK("permute_gather_kernel");
  }
  return MLXR_CU_OK;
}

static int check_qlinear(const mlxr_cu_qlinear& q, const char* name) {
  MLXR_CHECK_ARG(q.weight && q.scales && q.biases, "moe: %s weight/scales/biases must be non-NULL", name);
  MLXR_CHECK_ARG(aligned16(q.weight), "moe: %s weight must be 16-byte aligned", name);
  MLXR_CHECK_ARG((reinterpret_cast<uintptr_t>(q.scales) & 3) == 0 && (reinterpret_cast<uintptr_t>(q.biases) & 3) == 0,
                 "moe: %s scales/biases must be 4-byte aligned", name);
  return MLXR_CU_OK;
}

static int run_experts(const mlxr_cu_moe_config* c, const mlxr_cu_moe_weights* wt, const Layout& L, void* ws,
                       cudaStream_t st, int mid_stage) {
  if (L.rows == 0) return MLXR_CU_OK;
  const bool packed = c->model_kind == 1;  // Gemma 4: one gate_up_proj [E, 2I, D*b/32]
  if (packed) {
    if (int rc = check_qlinear(wt->switch_gate_up, "switch_glu.gate_up_proj")) return rc;
  } else {
    if (int rc = check_qlinear(wt->switch_gate, "switch_mlp.gate_proj")) return rc;
    if (int rc = check_qlinear(wt->switch_up, "switch_mlp.up_proj")) return rc;
  }
  if (int rc = check_qlinear(wt->switch_down, "switch_mlp.down_proj")) return rc;
  int* status = at<int>(ws, L.status);
  GroupedGemmProblem p{};
  p.nmat = 2;
  p.bn = L.bn1;
  p.bits = c->bits;
  if (packed) {
    // Gate = rows 0..I-1 and up = rows I..2I-1 of each expert's 2I rows: the
    // second matrix's views start I rows into the same tensors.
    const auto& gu = wt->switch_gate_up;
    const int64_t wpr = (int64_t)L.D * c->bits / 32, gpr = L.D / 64;
    p.w[0] = gu.weight;
    p.w[1] = gu.weight + (int64_t)L.I * wpr;
    p.s[0] = static_cast<const uint16_t*>(gu.scales);
    p.s[1] = static_cast<const uint16_t*>(gu.scales) + (int64_t)L.I * gpr;
    p.b[0] = static_cast<const uint16_t*>(gu.biases);
    p.b[1] = static_cast<const uint16_t*>(gu.biases) + (int64_t)L.I * gpr;
    p.w_rows = (int64_t)L.E * 2 * L.I;
    p.w_rows1 = (int64_t)L.E * 2 * L.I - L.I;
    p.w_expert_rows = 2 * L.I;
    p.glu = 1;  // GeGLU (nn/switch.rs:195-206)
  } else {
    p.w[0] = wt->switch_gate.weight;
    p.w[1] = wt->switch_up.weight;
    p.s[0] = static_cast<const uint16_t*>(wt->switch_gate.scales);
    p.s[1] = static_cast<const uint16_t*>(wt->switch_up.scales);
    p.b[0] = static_cast<const uint16_t*>(wt->switch_gate.biases);
    p.b[1] = static_cast<const uint16_t*>(wt->switch_up.biases);
    p.w_rows = (int64_t)L.E * L.I;
  }
  p.n_out = L.I;
  p.k_dim = L.D;
  p.num_experts = L.E;
  p.act = at<uint16_t>(ws, L.xs);
  p.act_rows = L.rows_pad;
  p.tiles = at<GemmTile>(ws, L.t1);
  p.num_tiles = at<int32_t>(ws, L.n1);
  p.max_tiles = L.max_t1;
  p.out = at<uint16_t>(ws, L.h);
  p.out_rows = L.rows;
  p.perm_out = c->bits == 4;  // h is the 4-bit down projection's activation operand
  p.status = status;
  p.splits = L.s1;
  p.max_split_rows = L.split_rows;
  p.partial = L.split_rows ? at<float>(ws, L.part) : nullptr;
  p.counters = L.split_rows ? at<int32_t>(ws, L.cnt) : nullptr;
  p.sched = at<int32_t>(ws, L.status) + kSchedExperts1;
  if (L.fuse) {
    // gate|up then down (row pairs) in one launch over the same tiles.
    p.fused = 1;
    p.w2 = wt->switch_down.weight;
    p.s2 = static_cast<const uint16_t*>(wt->switch_down.scales);
    p.b2 = static_cast<const uint16_t*>(wt->switch_down.biases);
    p.w2_rows = (int64_t)L.E * L.D;
    p.n_out2 = L.D;
    p.k_dim2 = L.I;
    p.act2_rows = L.rows_pad;
    p.out2 = at<uint16_t>(ws, L.y);
    p.tile_ready = at<int32_t>(ws, L.ready);
    if (int rc = launch_grouped_gemm(p, st)) return rc;
    stage_mark(mid_stage, st);
    return MLXR_CU_OK;
  }
  if (int rc = launch_grouped_gemm(p, st)) return rc;
  stage_mark(mid_stage, st);

  GroupedGemmProblem q{};
  // Two 128-row blocks of the down weight per work item (two accumulators,
  // two MMA issuers) when D allows it.
  q.pair = (L.D % 256 == 0) ? 1 : 0;
  q.nmat = q.pair ? 2 : 1;
  q.bn = q.pair ? (L.bn2 < 128 ? L.bn2 : 128) : L.bn2;
  q.bits = c->bits;
  q.w[0] = q.w[1] = wt->switch_down.weight;
  q.s[0] = q.s[1] = static_cast<const uint16_t*>(wt->switch_down.scales);
  q.b[0] = q.b[1] = static_cast<const uint16_t*>(wt->switch_down.biases);
  q.w_rows = (int64_t)L.E * L.D;
  q.n_out = L.D;
  q.k_dim = L.I;
  q.num_experts = L.E;
  q.act = at<uint16_t>(ws, L.h);
  q.act_rows = L.rows_pad;
  q.tiles = at<GemmTile>(ws, L.t2);
  q.num_tiles = at<int32_t>(ws, L.n2);
  q.max_tiles = L.max_t2;
  q.out = at<uint16_t>(ws, L.y);
  q.out_rows = L.rows;
  q.perm_out = 0;
  q.status = status;
  q.splits = L.s2;
  q.max_split_rows = L.split_rows;
  q.partial = L.split_rows ? at<float>(ws, L.part) : nullptr;
  q.counters = L.split_rows ? at<int32_t>(ws, L.cnt) : nullptr;
  q.sched = at<int32_t>(ws, L.status) + kSchedExperts2;
  return launch_grouped_gemm(q, st);
}

static int run_shared(const mlxr_cu_moe_config* c, const mlxr_cu_moe_weights* wt, const Layout& L, const void* x,
                      void* ws, cudaStream_t st) {
  if (L.Is == 0 || L.T == 0) return MLXR_CU_OK;
  if (int rc = check_qlinear(wt->shared_gate, "shared_expert.gate_proj")) return rc;
  if (int rc = check_qlinear(wt->shared_up, "shared_expert.up_proj")) return rc;
  if (int rc = check_qlinear(wt->shared_down, "shared_expert.down_proj")) return rc;
  int* status = at<int>(ws, L.status);
  const uint16_t* act = static_cast<const uint16_t*>(x);
  int64_t act_rows = L.T;
  const int kperm = c->shared_bits == 4;
  if (L.T < 256 || kperm) {
    // A padded (>= 256 rows) and, for 4-bit weights, K-order-permuted copy.
    const int64_t gblocks = (L.T + 7) / 8;
    const int grid = (int)(gblocks < 4 * 148 ? gblocks : 4 * 148);
    launch_pdl(permute_gather_kernel, grid, 256, 0, st, nullptr, L.T, L.T, 1, static_cast<const uint16_t*>(x), L.D, kperm,
                                                at<uint16_t>(ws, L.xpad), nullptr, status, 0);
    MLXR_LAUNCH_CHECK("permute_gather_kernel(shared)");
    act = at<uint16_t>(ws, L.xpad);
    act_rows = L.sh_rows_pad;
  }
  GroupedGemmProblem p{};
  p.nmat = 2;
  p.bn = L.bns;
  p.bits = c->shared_bits;
  p.w[0] = wt->shared_gate.weight;
  p.w[1] = wt->shared_up.weight;
  p.s[0] = static_cast<const uint16_t*>(wt->shared_gate.scales);
  p.s[1] = static_cast<const uint16_t*>(wt->shared_up.scales);
  p.b[0] = static_cast<const uint16_t*>(wt->shared_gate.biases);
  p.b[1] = static_cast<const uint16_t*>(wt->shared_up.biases);
  p.w_rows = L.Is;
  p.n_out = L.Is;
  p.k_dim = L.D;
  p.num_experts = 1;
  p.act = act;
  p.act_rows = act_rows;
  p.tiles = at<GemmTile>(ws, L.tsh);
  p.num_tiles = at<int32_t>(ws, L.nsh);
  p.max_tiles = L.max_tsh;
  p.out = at<uint16_t>(ws, L.hsh);
  p.out_rows = L.T;
  p.perm_out = c->shared_bits == 4;
  p.status = status;
  p.sched = at<int32_t>(ws, L.status) + kSchedShared1;
  if (int rc = launch_grouped_gemm(p, st)) return rc;
  GroupedGemmProblem q{};
  q.pair = (L.D % 256 == 0) ? 1 : 0;
  q.nmat = q.pair ? 2 : 1;
  q.bn = L.bns;
  q.bits = c->shared_bits;
  q.w[0] = q.w[1] = wt->shared_down.weight;
  q.s[0] = q.s[1] = static_cast<const uint16_t*>(wt->shared_down.scales);
  q.b[0] = q.b[1] = static_cast<const uint16_t*>(wt->shared_down.biases);
  q.w_rows = L.D;
  q.n_out = L.D;
  q.k_dim = L.Is;
  q.num_experts = 1;
  q.act = at<uint16_t>(ws, L.hsh);
  q.act_rows = L.sh_rows_pad;
  q.tiles = at<GemmTile>(ws, L.tsh);
  q.num_tiles = at<int32_t>(ws, L.nsh);
  q.max_tiles = L.max_tsh;
  q.out = at<uint16_t>(ws, L.ysh);
  q.out_rows = L.T;
  q.perm_out = 0;
  q.status = status;
  q.sched = at<int32_t>(ws, L.status) + kSchedShared2;
  return launch_grouped_gemm(q, st);
}

// Dispatch scratch: the block layout's router and permute buffers, then the
// per-(token, k) destination ranks.
static size_t ep_dispatch_bytes(const mlxr_cu_moe_config* c, int64_t T, size_t* dest_off) {
  const Layout L = make_layout(c, T);
  *dest_off = L.total;
  return L.total + align256((size_t)(T * c->num_experts_per_tok) * 4 + 4);
}

// The rows a dispatch sends: x, or for the Gemma 4 branch the experts'
// RMS-normed input that run_router wrote beside the routing.
static const void* ep_send_rows(const Layout& L, const void* x, void* ws) {
  return L.kind == 1 ? static_cast<const void*>(at<uint16_t>(ws, L.gxe)) : x;
}

static int ep_check_world(const mlxr_cu_moe_config* cfg, int world) {
  MLXR_CHECK_ARG(world >= 1 && world <= 64 && world <= cfg->num_experts,
                 "moe_ep: world=%d must be in [1, min(64, num_experts=%d)]", world, cfg->num_experts);
  return MLXR_CU_OK;
}


// Receiving side: num_pairs pairs of K slots (flat rows), num_rows filled slots.
static Layout ep_experts_layout(const mlxr_cu_moe_config* lc, int64_t num_pairs, int64_t num_rows) {
  return make_layout(lc, num_pairs, num_rows);
}

// -------------------------------------------- gather_qmm on tensor cores --
// gather_qmm (crates/mlxr/src/ops/quantization.rs:171-221) as QuantizedSwitchLinear::apply
// (crates/mlxr-lm/src/nn/switch.rs:148-167) issues it: bf16 rows, weights [E, N, K] 4- or
// 8-bit with group 64, transpose. The rows f = p * M + m of the output are
// treated as single-expert "tokens" (top-1, expert rhs[p]) and run through the
// block's machinery: the counting sort by expert builds the expert-sorted
// order and tile list, the rows are gathered (x[lhs[p]][m]), one grouped
// dequantising GEMM (tcgen05, plain epilogue) computes the expert-sorted
// outputs, and a final copy puts them back in index order.

// flat[f] = rhs[f / M] (or f / M without rhs); an index outside [0, E) is
// reported and replaced by expert 0 so the pass stays in bounds.
__global__ void gqmm_flat_experts_kernel(const uint32_t* __restrict__ rhs, int64_t R, int64_t M, int E,
                                         int32_t* __restrict__ flat, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; f < R; f += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = f / M;
    const int64_t e = rhs ? (int64_t)rhs[p] : p;
    if (e < 0 || e >= E) {
      atomicCAS(status, 0, (int)kDevBadIndex);
      flat[f] = 0;
    } else {
      flat[f] = (int32_t)e;
    }
  }
}

// xs[pos] = x[lhs[p]][m] for f = sorted[pos] = p * M + m (lhs absent: p),
// one warp per row with eight 16-byte loads in flight per lane; kperm stores
// each 8-element chunk in the 4-bit dequantiser's K order {0,4,1,5,2,6,3,7}.
__global__ void __launch_bounds__(256) gqmm_gather_kernel(const int32_t* __restrict__ sorted, int64_t R,
                                                         const uint32_t* __restrict__ lhs, int64_t M,
                                                         int64_t x_batch, const uint16_t* __restrict__ x, int D,
                                                         int kperm, uint16_t* __restrict__ xs, int* status) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dvec = D / 8;
  for (int64_t pos = (int64_t)blockIdx.x * 8 + warp; pos < R; pos += (int64_t)gridDim.x * 8) {
    const int64_t f = sorted[pos];
    if (f < 0 || f >= R) {
      if (lane == 0) atomicCAS(status, 0, (int)kDevBadIndex);
      continue;
    }
    const int64_t p = f / M, m = f - p * M;
    const int64_t src = lhs ? (int64_t)lhs[p] : p;
    if (src < 0 || src >= x_batch) {
      if (lane == 0) atomicCAS(status, 0, (int)kDevBadIndex);
      continue;
    }
    const uint4* in = reinterpret_cast<const uint4*>(x + (src * M + m) * D);
    uint4* outp = reinterpret_cast<uint4*>(xs + pos * D);
    auto st = [&](int v, uint4 a) {
      if (kperm) {
        uint4 b;
        b.x = __byte_perm(a.x, a.z, 0x5410);
        b.y = __byte_perm(a.x, a.z, 0x7632);
        b.z = __byte_perm(a.y, a.w, 0x5410);
        b.w = __byte_perm(a.y, a.w, 0x7632);
        a = b;
      }
      outp[v] = a;
    };
    int v = lane;
    for (; v + 7 * 32 < dvec; v += 8 * 32) {
      uint4 a[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = __ldg(in + v + j * 32);
#pragma unroll
      for (int j = 0; j < 8; ++j) st(v + j * 32, a[j]);
    }
    for (; v < dvec; v += 32) st(v, __ldg(in + v));
  }
}

// out[f] = y[inv[f]] (N columns, 16-byte copies); the pass's device status
// is forwarded to the op family's status word at the end.
__global__ void __launch_bounds__(256) gqmm_unpermute_kernel(const uint16_t* __restrict__ y,
                                                            const int32_t* __restrict__ inv, int64_t R, int N,
                                                            uint16_t* __restrict__ out, const int* status,
                                                            int* op_status) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = N / 8;
  for (int64_t f = (int64_t)blockIdx.x * 8 + warp; f < R; f += (int64_t)gridDim.x * 8) {
    const int64_t r = inv[f];
    if (r < 0 || r >= R) {
      if (lane == 0) atomicCAS(op_status, 0, (int)kDevBadIndex);
      continue;
    }
    const uint4* in = reinterpret_cast<const uint4*>(y + r * N);
    uint4* o = reinterpret_cast<uint4*>(out + f * N);
    for (int v = lane; v < nvec; v += 32) o[v] = __ldg(in + v);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    const int s = *reinterpret_cast<const volatile int*>(status);
    if (s != 0) atomicCAS(op_status, 0, s);
  }
}

// The tensor-core path applies to bf16 rows, transposed weights, group 64,
// 4 or 8 bits, K and N multiples of 128, at most PERM_MAX_E experts.
static bool gqmm_fast_ok(mlxr_cu_dtype x_dtype, int64_t K, int64_t N, int64_t w_batch, int transpose, int gs,
                         int bits, int64_t R) {
  return x_dtype == MLXR_CU_BFLOAT16 && transpose && gs == 64 && (bits == 4 || bits == 8) && K % 128 == 0 &&
         N % 128 == 0 && K <= (int64_t)1 << 20 && N <= (int64_t)1 << 20 && w_batch >= 1 && w_batch <= PERM_MAX_E &&
         R > 0 && R < (int64_t)1 << 30;
}

static mlxr_cu_moe_config gqmm_cfg(int64_t K, int64_t N, int64_t w_batch, int bits) {
  mlxr_cu_moe_config c{};
  c.hidden_size = (int32_t)K;
  c.num_experts = (int32_t)w_batch;
  c.num_experts_per_tok = 1;
  c.moe_intermediate_size = (int32_t)N;
  c.group_size = 64;
  c.bits = bits;
  c.shared_bits = bits;
  c.norm_topk_prob = 1;
  return c;
}

// The pass's workspace: the block layout for R one-expert rows (its status
// slot, routing arrays, tile list, x_sorted [R, K] and the expert-sorted
// outputs in its h buffer [R, N]) plus the flat expert array.
struct GqmmLayout {
  Layout L;
  size_t flat = 0, total = 0;
};
static GqmmLayout gqmm_layout(const mlxr_cu_moe_config* c, int64_t R) {
  GqmmLayout g;
  g.L = make_layout(c, R);
  g.flat = align256(g.L.total);
  g.total = align256(g.flat + (size_t)R * 4);
  return g;
}

}  // namespace mlxr

using namespace mlxr;

extern "C" {

int mlxr_cu_moe_workspace_size(const mlxr_cu_moe_config* cfg, int64_t num_tokens, size_t* bytes) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  MLXR_CHECK_ARG(bytes != nullptr, "moe_workspace_size: bytes is NULL");
  *bytes = make_layout(cfg, num_tokens).total;
  return MLXR_CU_OK;
}

int mlxr_cu_moe_block_forward(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, const void* x,
                              int64_t num_tokens, void* out, const mlxr_cu_moe_routing* routing, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  MLXR_CHECK_ARG(weights != nullptr, "moe: weights is NULL");
  const Layout L = make_layout(cfg, num_tokens);
  if (int rc = check_ws(L, workspace, workspace_bytes)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  MLXR_CUDA_TRY(cudaMemsetAsync(at<int>(workspace, L.status), 0, kStatusSlotBytes, st));
  if (num_tokens == 0) return MLXR_CU_OK;
  MLXR_CHECK_ARG(x && out, "moe: x/out is NULL");
  MLXR_CHECK_ARG(aligned16(x) && aligned16(out), "moe: x and out must be 16-byte aligned");
  void* ws = workspace;
  stage_mark(0, st);
  if (int rc = run_router(cfg, weights, L, x, ws, nullptr, nullptr, st)) return rc;
  stage_mark(1, st);
  const void* xe = L.kind == 1 ? static_cast<const void*>(at<uint16_t>(ws, L.gxe)) : x;  // the experts' input
  if (int rc = run_permute(L, at<int32_t>(ws, L.idx), xe, ws, at<int32_t>(ws, L.counts), at<int32_t>(ws, L.offsets),
                           at<int32_t>(ws, L.sorted), at<int32_t>(ws, L.inv), at<uint16_t>(ws, L.xs), cfg->bits == 4, st))
    return rc;
  stage_mark(2, st);
  if (int rc = run_experts(cfg, weights, L, ws, st, 3)) return rc;
  stage_mark(4, st);
  if (int rc = run_shared(cfg, weights, L, x, ws, st)) return rc;
  stage_mark(5, st);
  launch_pdl(combine_kernel, (unsigned)L.T, L.D >= 2048 ? 256 : 128, 0, st, at<uint16_t>(ws, L.y), at<int32_t>(ws, L.inv), at<uint16_t>(ws, L.w),
                                                L.K, L.D, L.T, L.Is > 0 ? at<uint16_t>(ws, L.ysh) : nullptr,
                                                at<float>(ws, L.sig), static_cast<uint16_t*>(out),
                                                at<int>(ws, L.status));
  MLXR_LAUNCH_CHECK("combine_kernel");
  stage_mark(6, st);
  if (routing) {
    auto cp = [&](void* dst, size_t off, size_t bytes) -> int {
      if (dst && bytes) MLXR_CUDA_TRY(cudaMemcpyAsync(dst, at<uint8_t>(ws, off), bytes, cudaMemcpyDeviceToDevice, st));
      return MLXR_CU_OK;
    };
    if (int rc = cp(routing->indices, L.idx, (size_t)L.R * 4)) return rc;
    if (int rc = cp(routing->weights, L.w, (size_t)L.R * 2)) return rc;
    if (int rc = cp(routing->counts, L.counts, (size_t)L.E * 4)) return rc;
    if (int rc = cp(routing->offsets, L.offsets, (size_t)(L.E + 1) * 4)) return rc;
    if (int rc = cp(routing->sorted_rows, L.sorted, (size_t)L.R * 4)) return rc;
    if (int rc = cp(routing->inverse, L.inv, (size_t)L.R * 4)) return rc;
  }
  return MLXR_CU_OK;
}

int mlxr_cu_moe_set_stage_events(void* const* events, int count) {
  MLXR_CHECK_ARG(count >= 0 && count <= 8, "moe_set_stage_events: count=%d must be in [0, 8]", count);
  MLXR_CHECK_ARG(count == 0 || events != nullptr, "moe_set_stage_events: events is NULL");
  for (int i = 0; i < 8; ++i) t_stage_events[i] = i < count ? static_cast<cudaEvent_t>(events[i]) : nullptr;
  t_stage_count = count;
  return MLXR_CU_OK;
}

// ------------------------------------------------ allocation-free entry --
// Some callers of this library cannot allocate device memory when they call
// it: a serving engine that has reserved nearly all HBM for weights and KV
// cache up front and treats any later cudaMalloc as an error (or cannot
// afford its implicit device-wide synchronisation on a latency path), or a
// host runtime that binds this library over a plain C ABI and has no device
// allocator to hand it. For them mlxr_cu_moe_block_forward_noalloc runs the
// block forward with its scratch in the fixed-size array below, which lives
// in the library image: every GPU that loads the library holds
// kNoAllocScratchBytes of it until the process exits, and nothing on this
// path calls cudaMalloc, cudaFree or an allocating library routine.
constexpr size_t kNoAllocScratchBytes = size_t(24) << 20;  // 24 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Host code cannot use g_noalloc_scratch as a device address (in host code it
// names a host-side stand-in). The device address is looked up with
// cudaGetSymbolAddress once per device, with that device current, and cached
// together with the driver context it belongs to: the module (and with it the
// array) is loaded per context, so a caller that switches to another context
// on the same device (or recreates the primary one after cudaDeviceReset)
// gets a fresh lookup instead of a stale address.
typedef int (*PFN_ctx_get_current)(void**);

static PFN_ctx_get_current ctx_get_current_fn() {
  static PFN_ctx_get_current fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_ctx_get_current>(p);
  });
  return fn;
}

static void* noalloc_scratch(int* rc) {
  static std::mutex mu;
  static void* ptrs[128] = {};
  static void* ctxs[128] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *rc = check_cuda(e, "cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= 128) {
    *rc = set_error(MLXR_CU_ERR_CUDA, "moe_noalloc: device ordinal %d out of range", dev);
    return nullptr;
  }
  // Which driver context is current (cudaSetDevice makes the device's
  // primary context current when none is).
  void* ctx = nullptr;
  PFN_ctx_get_current get_ctx = ctx_get_current_fn();
  if (!get_ctx || get_ctx(&ctx) != 0) {
    *rc = set_error(MLXR_CU_ERR_CUDA, "moe_noalloc: cuCtxGetCurrent is not available from the driver");
    return nullptr;
  }
  if (!ctx) {
    e = cudaSetDevice(dev);
    if (e != cudaSuccess || get_ctx(&ctx) != 0 || !ctx) {
      *rc = check_cuda(e != cudaSuccess ? e : cudaErrorDeviceUninitialized, "cudaSetDevice (no current context)");
      return nullptr;
    }
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev] || ctxs[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *rc = check_cuda(e != cudaSuccess ? e : cudaErrorInvalidSymbol, "cudaGetSymbolAddress(noalloc scratch)");
      return nullptr;
    }
    ptrs[dev] = p;
    ctxs[dev] = ctx;
  }
  *rc = MLXR_CU_OK;
  return ptrs[dev];
}

int mlxr_cu_moe_block_forward_noalloc(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights,
                                      const void* x, int64_t num_tokens, void* out,
                                      const mlxr_cu_moe_routing* routing, int* device_status, void* stream) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  const Layout L = make_layout(cfg, num_tokens);
  if (L.total > kNoAllocScratchBytes)
    return set_error(MLXR_CU_ERR_WORKSPACE,
                     "moe_noalloc: %lld tokens need %zu bytes of scratch but the allocation-free entry point has %zu; "
                     "split the batch or call mlxr_cu_moe_block_forward with a workspace",
                     (long long)num_tokens, L.total, kNoAllocScratchBytes);
  int rc = MLXR_CU_OK;
  void* ws = noalloc_scratch(&rc);
  if (!ws) return rc;
  // The scratch keeps the previous call's contents; the forward clears its
  // status word itself and rebuilds every other buffer before reading it.
  if (int r2 = mlxr_cu_moe_block_forward(cfg, weights, x, num_tokens, out, routing, ws, kNoAllocScratchBytes, stream))
    return r2;
  if (device_status)
    MLXR_CUDA_TRY(cudaMemcpyAsync(device_status, at<int>(ws, L.status), sizeof(int), cudaMemcpyDeviceToDevice,
                                  static_cast<cudaStream_t>(stream)));
  return MLXR_CU_OK;
}

int mlxr_cu_moe_status(const void* workspace, void* stream) {
  MLXR_CHECK_ARG(workspace != nullptr, "moe_status: workspace is NULL");
  MLXR_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int v = 0;
  MLXR_CUDA_TRY(cudaMemcpy(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost));  // status is at offset 0
  switch (v) {
    case kDevOk: return MLXR_CU_OK;
    case kDevTimeout: return set_error(MLXR_CU_ERR_TIMEOUT, "moe: a device-side wait timed out");
    case kDevBadIndex: return set_error(MLXR_CU_ERR_DEVICE_INDEX, "moe: an expert index was outside [0, num_experts)");
    case kDevPeerFailed:
      return set_error(MLXR_CU_ERR_TIMEOUT,
                       "moe: another rank reported a failed step (its wait timed out or it skipped a bad index); "
                       "the rows it exchanged in this step are not valid");
    default: return set_error(MLXR_CU_ERR_CUDA, "moe: device status %d", v);
  }
}

int mlxr_cu_op_status(void* stream) {
  int* p = op_status_word();
  if (!p) return MLXR_CU_ERR_CUDA;
  MLXR_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  int v = 0;
  MLXR_CUDA_TRY(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  const int zero = 0;
  MLXR_CUDA_TRY(cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice));
  if (v == kDevBadIndex) return set_error(MLXR_CU_ERR_DEVICE_INDEX, "an index was outside its batch");
  if (v != 0) return set_error(MLXR_CU_ERR_CUDA, "device status %d", v);
  return MLXR_CU_OK;
}

int mlxr_cu_moe_router(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, const void* x,
                       int64_t num_tokens, int32_t* indices, void* topk_weights, void* logits, void* probs,
                       void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  const Layout L = make_layout(cfg, num_tokens);
  if (int rc = check_ws(L, workspace, workspace_bytes)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  MLXR_CUDA_TRY(cudaMemsetAsync(at<int>(workspace, L.status), 0, kStatusSlotBytes, st));
  if (num_tokens == 0) return MLXR_CU_OK;
  MLXR_CHECK_ARG(x && indices && topk_weights, "moe_router: x/indices/weights is NULL");
  uint16_t* lg = logits ? static_cast<uint16_t*>(logits) : at<uint16_t>(workspace, L.logits);
  mlxr_cu_moe_config c2 = *cfg;
  c2.shared_expert_intermediate_size = 0;  // the router alone does not evaluate the shared gate
  Layout L2 = L;
  L2.Is = 0;
  if (int rc = run_router(&c2, weights, L2, x, workspace, lg, static_cast<uint16_t*>(probs), st)) return rc;
  MLXR_CUDA_TRY(cudaMemcpyAsync(indices, at<int32_t>(workspace, L.idx), (size_t)L.R * 4, cudaMemcpyDeviceToDevice, st));
  MLXR_CUDA_TRY(cudaMemcpyAsync(topk_weights, at<uint16_t>(workspace, L.w), (size_t)L.R * 2, cudaMemcpyDeviceToDevice, st));
  return MLXR_CU_OK;
}

int mlxr_cu_moe_permute(const mlxr_cu_moe_config* cfg, const int32_t* indices, int64_t num_tokens, const void* x,
                        int32_t* counts, int32_t* offsets, int32_t* sorted_rows, int32_t* inverse, void* x_sorted,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  const Layout L = make_layout(cfg, num_tokens);
  if (int rc = check_ws(L, workspace, workspace_bytes)) return rc;
  MLXR_CHECK_ARG(indices && x && counts && offsets && sorted_rows && inverse && x_sorted, "moe_permute: NULL argument");
  MLXR_CHECK_ARG(aligned16(x) && aligned16(x_sorted), "moe_permute: x and x_sorted must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  MLXR_CUDA_TRY(cudaMemsetAsync(at<int>(workspace, L.status), 0, kStatusSlotBytes, st));
  return run_permute(L, indices, x, workspace, counts, offsets, sorted_rows, inverse, static_cast<uint16_t*>(x_sorted),
                     0, st);
}

int mlxr_cu_moe_experts(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, const int32_t* row_experts,
                        int64_t num_tokens, const void* x_rows, void* y_rows, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  MLXR_CHECK_ARG(weights != nullptr, "moe_experts: weights is NULL");
  const Layout L = make_layout(cfg, num_tokens);
  if (int rc = check_ws(L, workspace, workspace_bytes)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  MLXR_CUDA_TRY(cudaMemsetAsync(at<int>(workspace, L.status), 0, kStatusSlotBytes, st));
  if (num_tokens == 0) return MLXR_CU_OK;
  MLXR_CHECK_ARG(row_experts && x_rows && y_rows, "moe_experts: NULL argument");
  MLXR_CHECK_ARG(aligned16(x_rows) && aligned16(y_rows), "moe_experts: x_rows and y_rows must be 16-byte aligned");
  void* ws = workspace;
  // The T*K rows are grouped by expert as single-slot tokens (a stable sort:
  // the identity when they already are), gathered into the GEMM operand
  // buffer, run through the experts, and written back in the caller's order.
  Layout P = L;
  P.K = 1;
  P.T = L.R;
  P.Is = 0;
  if (int rc = run_permute(P, row_experts, x_rows, ws, at<int32_t>(ws, L.counts), at<int32_t>(ws, L.offsets),
                           at<int32_t>(ws, L.sorted), at<int32_t>(ws, L.inv), at<uint16_t>(ws, L.xs), cfg->bits == 4, st))
    return rc;
  if (int rc = run_experts(cfg, weights, L, ws, st, 3)) return rc;
  const int64_t gblocks = (L.R + 7) / 8;
  const int grid = (int)(gblocks < 4 * 148 ? gblocks : 4 * 148);
  launch_pdl(permute_gather_kernel, grid, 256, 0, st, at<int32_t>(ws, L.inv), L.R, L.R, 1, at<uint16_t>(ws, L.y), L.D, 0,
             static_cast<uint16_t*>(y_rows), nullptr, at<int>(ws, L.status), 0);
  MLXR_LAUNCH_CHECK("permute_gather_kernel(unsort)");
  return MLXR_CU_OK;
}

int mlxr_cu_moe_combine(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, const void* x,
                        int64_t num_tokens, const void* y_sorted, const int32_t* inverse, const void* topk_weights,
                        void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  const Layout L = make_layout(cfg, num_tokens);
  if (int rc = check_ws(L, workspace, workspace_bytes)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  MLXR_CUDA_TRY(cudaMemsetAsync(at<int>(workspace, L.status), 0, kStatusSlotBytes, st));
  if (num_tokens == 0) return MLXR_CU_OK;
  MLXR_CHECK_ARG(y_sorted && inverse && topk_weights && out, "moe_combine: NULL argument");
  MLXR_CHECK_ARG(aligned16(y_sorted) && aligned16(out), "moe_combine: y_sorted and out must be 16-byte aligned");
  void* ws = workspace;
  const uint16_t* ysh = nullptr;
  if (L.Is > 0) {
    MLXR_CHECK_ARG(weights != nullptr && x != nullptr && aligned16(x), "moe_combine: weights / x is NULL or misaligned");
    MLXR_CHECK_ARG(weights->shared_expert_gate.weight && weights->shared_expert_gate.scales &&
                       weights->shared_expert_gate.biases,
                   "moe_combine: shared_expert_gate is NULL");
    SharedGateArgs sg{weights->shared_expert_gate.weight,
                      static_cast<const uint16_t*>(weights->shared_expert_gate.scales),
                      static_cast<const uint16_t*>(weights->shared_expert_gate.biases), shared_gate_bits(cfg)};
    launch_pdl(shared_gate_kernel, (unsigned)((L.T + 7) / 8), 256, 0, st, static_cast<const uint16_t*>(x), L.T, L.D, sg,
               at<float>(ws, L.sig));
    MLXR_LAUNCH_CHECK("shared_gate_kernel");
    launch_pdl(shared_tiles_kernel, (unsigned)((L.max_tsh + 255) / 256), 256, 0, st, at<GemmTile>(ws, L.tsh),
               at<int32_t>(ws, L.nsh), L.T, L.bns, L.max_tsh);
    MLXR_LAUNCH_CHECK("shared_tiles_kernel");
    if (int rc = run_shared(cfg, weights, L, x, ws, st)) return rc;
    ysh = at<uint16_t>(ws, L.ysh);
  }
  launch_pdl(combine_kernel, (unsigned)L.T, L.D >= 2048 ? 256 : 128, 0, st, static_cast<const uint16_t*>(y_sorted), inverse,
             static_cast<const uint16_t*>(topk_weights), L.K, L.D, L.T, ysh, at<float>(ws, L.sig),
             static_cast<uint16_t*>(out), at<int>(ws, L.status));
  MLXR_LAUNCH_CHECK("combine_kernel");
  return MLXR_CU_OK;
}

// ------------------------------------------------ expert parallelism ---
// One rank's share of the block when its experts are spread over `world`
// ranks (expert e on rank e % world as local expert e / world). Per step:
// mlxr_cu_moe_ep_dispatch routes this rank's tokens and lists one pair per
// (token, destination rank) with its x row and its (local expert, weight)
// slots; the caller exchanges the pairs (all-to-all); mlxr_cu_moe_ep_experts
// runs the received pairs through this rank's experts and pre-reduces each
// pair to one partial row; the caller returns the partial rows (the reverse
// all-to-all); mlxr_cu_moe_ep_combine sums each token's partial rows and adds
// the shared expert.

int mlxr_cu_moe_ep_workspace_size(const mlxr_cu_moe_config* cfg, int world, int64_t num_tokens,
                                  int64_t max_recv_pairs, int64_t max_recv_rows, size_t* bytes) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  if (int rc = ep_check_world(cfg, world)) return rc;
  MLXR_CHECK_ARG(bytes != nullptr, "moe_ep_workspace_size: bytes is NULL");
  MLXR_CHECK_ARG(max_recv_pairs >= 0 && max_recv_rows >= 0, "moe_ep_workspace_size: negative receive bound");
  if (int rc = validate(cfg, max_recv_pairs)) return rc;
  mlxr_cu_moe_config lc = *cfg;  // any placement: up to all experts on this rank
  lc.shared_expert_intermediate_size = 0;
  size_t dest_off = 0;
  size_t need = ep_dispatch_bytes(cfg, num_tokens, &dest_off);
  const size_t e2 = ep_experts_layout(&lc, max_recv_pairs, max_recv_rows).total;
  const size_t e3 = make_layout(cfg, num_tokens).total;
  if (e2 > need) need = e2;
  if (e3 > need) need = e3;
  *bytes = need;
  return MLXR_CU_OK;
}

int mlxr_cu_moe_ep_dispatch(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, int world,
                            const int32_t* placement, const void* x, int64_t num_tokens, int32_t* send_counts, int32_t* pair_pos,
                            void* x_send, int32_t* meta_send, float* shared_gate, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  if (int rc = ep_check_world(cfg, world)) return rc;
  MLXR_CHECK_ARG(weights != nullptr, "moe_ep_dispatch: weights is NULL");
  size_t dest_off = 0;
  const size_t need = ep_dispatch_bytes(cfg, num_tokens, &dest_off);
  MLXR_CHECK_ARG(workspace && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0 && workspace_bytes >= need,
                 "moe_ep_dispatch: workspace NULL, not 256-byte aligned or smaller than %zu bytes", need);
  MLXR_CHECK_ARG(send_counts != nullptr, "moe_ep_dispatch: send_counts is NULL");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = workspace;
  const Layout L = make_layout(cfg, num_tokens);
  MLXR_CUDA_TRY(cudaMemsetAsync(at<int>(ws, L.status), 0, kStatusSlotBytes, st));
  if (num_tokens == 0) {
    MLXR_CUDA_TRY(cudaMemsetAsync(send_counts, 0, (size_t)world * 2 * 4, st));
    return MLXR_CU_OK;
  }
  MLXR_CHECK_ARG(x && pair_pos && x_send && meta_send && aligned16(x) && aligned16(x_send),
                 "moe_ep_dispatch: NULL or misaligned argument (x and x_send need 16-byte alignment)");
  MLXR_CHECK_ARG(cfg->shared_expert_intermediate_size == 0 || shared_gate, "moe_ep_dispatch: shared_gate is NULL");
  if (int rc = run_router(cfg, weights, L, x, ws, nullptr, nullptr, st)) return rc;
  const int K = cfg->num_experts_per_tok;
  const int64_t R = L.R;
  int32_t* dest = at<int32_t>(ws, dest_off);
  launch_pdl(ep_pair_dest_kernel, (unsigned)((R + 255) / 256), 256, 0, st, at<int32_t>(ws, L.idx), num_tokens, K, world, placement, dest,
                                                                    at<int>(ws, L.status));
  MLXR_LAUNCH_CHECK("ep_pair_dest_kernel");
  // Stable sort of the pairs by destination rank: the block permutation with
  // `world` buckets, the non-first (token, k) rows skipped, x rows gathered
  // unpermuted into x_send.
  Layout P = L;
  P.E = world;
  P.Is = 0;
  P.rows = num_tokens * (K < world ? K : world);
  P.bn1 = P.bn2 = 1 << 30;  // tile lists are not used here
  P.max_t1 = P.max_t2 = world + 1;
  if (int rc = run_permute(P, dest, ep_send_rows(L, x, ws), ws, at<int32_t>(ws, L.counts), at<int32_t>(ws, L.offsets),
                           at<int32_t>(ws, L.sorted), pair_pos, static_cast<uint16_t*>(x_send), 0, st, 1))
    return rc;
  launch_pdl(ep_counts_kernel, 1, 1024, 0, st, at<int32_t>(ws, L.idx), R, world, placement, at<int32_t>(ws, L.counts),
             send_counts);
  MLXR_LAUNCH_CHECK("ep_counts_kernel");
  launch_pdl(ep_pair_meta_kernel, (unsigned)((num_tokens + 127) / 128), 128, 0, st, 
      at<int32_t>(ws, L.idx), at<uint16_t>(ws, L.w), pair_pos, num_tokens, K, world, placement, P.rows, meta_send,
      at<int>(ws, L.status));
  MLXR_LAUNCH_CHECK("ep_pair_meta_kernel");
  if (cfg->shared_expert_intermediate_size > 0)
    MLXR_CUDA_TRY(cudaMemcpyAsync(shared_gate, at<float>(ws, L.sig), (size_t)num_tokens * 4, cudaMemcpyDeviceToDevice,
                                  st));
  return MLXR_CU_OK;
}

int mlxr_cu_moe_ep_experts(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* local_weights,
                           int num_local_experts, const void* x_recv, const int32_t* meta_recv, int64_t num_pairs,
                           int64_t num_rows, void* partial, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = validate(cfg, num_pairs)) return rc;
  MLXR_CHECK_ARG(num_local_experts >= 1 && num_local_experts <= cfg->num_experts,
                 "moe_ep_experts: num_local_experts=%d must be in [1, num_experts]", num_local_experts);
  mlxr_cu_moe_config lc = *cfg;
  lc.num_experts = num_local_experts;
  lc.shared_expert_intermediate_size = 0;
  MLXR_CHECK_ARG(local_weights != nullptr, "moe_ep_experts: weights is NULL");
  MLXR_CHECK_ARG(num_rows >= 0 && num_rows <= num_pairs * lc.num_experts_per_tok,
                 "moe_ep_experts: num_rows=%lld must be in [0, num_pairs * K]", (long long)num_rows);
  const Layout L = ep_experts_layout(&lc, num_pairs, num_rows);
  if (int rc = check_ws(L, workspace, workspace_bytes)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = workspace;  // the status word was cleared by this step's dispatch
  if (num_pairs == 0) return MLXR_CU_OK;
  MLXR_CHECK_ARG(x_recv && meta_recv && partial && aligned16(x_recv) && aligned16(partial),
                 "moe_ep_experts: NULL or misaligned argument (x_recv and partial need 16-byte alignment)");
  launch_pdl(ep_slot_expert_kernel, (unsigned)((L.R + 255) / 256), 256, 0, st, meta_recv, L.R, L.E, at<int32_t>(ws, L.idx),
                                                                        at<int>(ws, L.status));
  MLXR_LAUNCH_CHECK("ep_slot_expert_kernel");
  if (int rc = run_permute(L, at<int32_t>(ws, L.idx), x_recv, ws, at<int32_t>(ws, L.counts), at<int32_t>(ws, L.offsets),
                           at<int32_t>(ws, L.sorted), at<int32_t>(ws, L.inv), at<uint16_t>(ws, L.xs), lc.bits == 4, st, 1))
    return rc;
  if (int rc = run_experts(&lc, local_weights, L, ws, st, 7)) return rc;
  if (L.rows == 0) {
    MLXR_CUDA_TRY(cudaMemsetAsync(partial, 0, (size_t)num_pairs * L.D * 2, st));
    return MLXR_CU_OK;
  }
  launch_pdl(ep_reduce_kernel, (unsigned)num_pairs, L.D >= 2048 ? 256 : 128, 0, st, 
      at<uint16_t>(ws, L.y), at<int32_t>(ws, L.inv), meta_recv, L.K, L.D, L.rows, static_cast<uint16_t*>(partial),
      at<int>(ws, L.status));
  MLXR_LAUNCH_CHECK("ep_reduce_kernel");
  return MLXR_CU_OK;
}

int mlxr_cu_moe_ep_combine(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, const void* x,
                           int64_t num_tokens, const void* partial_back, int64_t num_pairs, const int32_t* pair_pos,
                           const float* shared_gate, void* out, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  const Layout L = make_layout(cfg, num_tokens);
  if (int rc = check_ws(L, workspace, workspace_bytes)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = workspace;  // the status word was cleared by this step's dispatch
  if (num_tokens == 0) return MLXR_CU_OK;
  MLXR_CHECK_ARG(x && pair_pos && out && aligned16(x) && aligned16(out) && (num_pairs == 0 || partial_back) &&
                     aligned16(partial_back),
                 "moe_ep_combine: NULL or misaligned argument");
  const uint16_t* ysh = nullptr;
  if (L.Is > 0) {
    MLXR_CHECK_ARG(shared_gate != nullptr && weights != nullptr, "moe_ep_combine: shared_gate / weights is NULL");
    // The block forward gets the shared tile list from its permute; here it is built alone.
    launch_pdl(shared_tiles_kernel, (unsigned)((L.max_tsh + 255) / 256), 256, 0, st, at<GemmTile>(ws, L.tsh),
                                                                             at<int32_t>(ws, L.nsh), L.T, L.bns,
                                                                             L.max_tsh);
    MLXR_LAUNCH_CHECK("shared_tiles_kernel");
    if (int rc = run_shared(cfg, weights, L, x, ws, st)) return rc;
    ysh = at<uint16_t>(ws, L.ysh);
  }
  launch_pdl(ep_combine_kernel, (unsigned)L.T, L.D >= 2048 ? 256 : 128, 0, st, 
      static_cast<const uint16_t*>(partial_back), pair_pos, L.K, L.D, num_pairs, ysh, shared_gate,
      static_cast<uint16_t*>(out), at<int>(ws, L.status));
  MLXR_LAUNCH_CHECK("ep_combine_kernel");
  return MLXR_CU_OK;
}

// ----------------------------------------- expert parallelism, peer memory --
// The same three steps with the exchange done by the kernels themselves
// over NVLink (see EpBufLayout in routing.cuh): no collective library and no
// host read of the counts. A communicator holds this rank's exchange buffer
// and every other rank's buffer mapped through CUDA IPC.

}  // extern "C"

namespace mlxr {
struct EpComm {
  int world = 0, rank = 0, D = 0, K = 0, device = -1;
  int64_t cap = 0;
  EpBufLayout bl{};
  uint8_t* local = nullptr;
  EpPeers peers{};
  bool opened[EP_MAX_WORLD] = {};
};

static int ep_comm_check(const void* comm, const mlxr_cu_moe_config* cfg) {
  MLXR_CHECK_ARG(comm != nullptr, "moe_ep_p2p: comm is NULL");
  const EpComm* c = static_cast<const EpComm*>(comm);
  MLXR_CHECK_ARG(c->local != nullptr, "moe_ep_p2p: comm is not initialised");
  MLXR_CHECK_ARG(cfg->hidden_size == c->D && cfg->num_experts_per_tok == c->K,
                 "moe_ep_p2p: comm was made for hidden=%d K=%d, block has hidden=%d K=%d", c->D, c->K,
                 cfg->hidden_size, cfg->num_experts_per_tok);
  for (int r = 0; r < c->world; ++r)
    MLXR_CHECK_ARG(c->peers.base[r] != nullptr, "moe_ep_p2p: rank %d's buffer is not connected", r);
  return MLXR_CU_OK;
}

// Dispatch scratch on top of the block layout: destinations, slot rows, counts.
struct EpP2PDispatch {
  size_t dest, meta, counts, total;
};
static EpP2PDispatch ep_p2p_dispatch_layout(const mlxr_cu_moe_config* c, int world, int64_t T) {
  EpP2PDispatch d{};
  const Layout L = make_layout(c, T);
  size_t o = L.total;
  const int K = c->num_experts_per_tok;
  auto take = [&](size_t bytes) {
    const size_t at_ = o;
    o = align256(o + (bytes ? bytes : 1));
    return at_;
  };
  d.dest = take((size_t)T * K * 4);
  d.meta = take((size_t)T * (K < world ? K : world) * K * 4);
  d.counts = take((size_t)world * 2 * 4);
  d.total = o;
  return d;
}
static Layout ep_p2p_experts_layout(const mlxr_cu_moe_config* c, int num_local, int world, int64_t cap,
                                    int64_t expected_rows) {
  mlxr_cu_moe_config lc = *c;
  lc.num_experts = num_local;
  lc.shared_expert_intermediate_size = 0;
  const int K = c->num_experts_per_tok;
  const int64_t pairs = (int64_t)world * cap;
  const int64_t rows = pairs * (K < num_local ? K : num_local);
  return make_layout(&lc, pairs, rows, expected_rows);
}
}  // namespace mlxr

extern "C" {

int mlxr_cu_ep_comm_create(int world, int rank, int64_t cap, int hidden, int k, void** comm, void* ipc_handle) {
  MLXR_CHECK_ARG(world >= 1 && world <= EP_MAX_WORLD && rank >= 0 && rank < world,
                 "ep_comm_create: world=%d rank=%d (world must be in [1, %d])", world, rank, EP_MAX_WORLD);
  MLXR_CHECK_ARG(cap >= 1 && hidden > 0 && hidden % 8 == 0 && k >= 1 && k <= RT_MAXK,
                 "ep_comm_create: cap=%lld hidden=%d k=%d", (long long)cap, hidden, k);
  MLXR_CHECK_ARG(comm && ipc_handle, "ep_comm_create: NULL output");
  EpComm* c = new EpComm();
  c->world = world;
  c->rank = rank;
  c->cap = cap;
  c->D = hidden;
  c->K = k;
  c->bl = ep_buf_layout(world, cap, hidden, k);
  cudaError_t e = cudaGetDevice(&c->device);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&c->local), (size_t)c->bl.total);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, (size_t)c->bl.total);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return check_cuda(e, "ep_comm_create");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == MLXR_CU_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(ipc_handle, &h, sizeof(h));
  c->peers.base[rank] = c->local;
  *comm = c;
  return MLXR_CU_OK;
}

int mlxr_cu_ep_comm_connect(void* comm, const void* ipc_handles) {
  MLXR_CHECK_ARG(comm && ipc_handles, "ep_comm_connect: NULL argument");
  EpComm* c = static_cast<EpComm*>(comm);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank || c->opened[r]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const uint8_t*>(ipc_handles) + (size_t)r * sizeof(h), sizeof(h));
    void* p = nullptr;
    MLXR_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    c->peers.base[r] = static_cast<uint8_t*>(p);
    c->opened[r] = true;
  }
  return MLXR_CU_OK;
}

int mlxr_cu_ep_comm_destroy(void* comm) {
  if (!comm) return MLXR_CU_OK;
  EpComm* c = static_cast<EpComm*>(comm);
  int rc = MLXR_CU_OK;
  for (int r = 0; r < c->world; ++r)
    if (c->opened[r]) {
      const cudaError_t e = cudaIpcCloseMemHandle(c->peers.base[r]);
      if (e != cudaSuccess && rc == MLXR_CU_OK) rc = check_cuda(e, "cudaIpcCloseMemHandle");
    }
  if (c->local) {
    const cudaError_t e = cudaFree(c->local);
    if (e != cudaSuccess && rc == MLXR_CU_OK) rc = check_cuda(e, "cudaFree(exchange buffer)");
  }
  delete c;
  return rc;
}

int mlxr_cu_moe_ep_p2p_workspace_size(const mlxr_cu_moe_config* cfg, const void* comm, int64_t num_tokens,
                                      int num_local_experts, int64_t expected_rows, size_t* bytes) {
  if (int rc = validate(cfg, num_tokens)) return rc;
  if (int rc = ep_comm_check(comm, cfg)) return rc;
  MLXR_CHECK_ARG(bytes && num_local_experts >= 1 && num_local_experts <= cfg->num_experts,
                 "moe_ep_p2p_workspace_size: bad num_local_experts=%d", num_local_experts);
  const EpComm* c = static_cast<const EpComm*>(comm);
  MLXR_CHECK_ARG(num_tokens <= c->cap, "moe_ep_p2p: %lld tokens exceed the comm capacity %lld",
                 (long long)num_tokens, (long long)c->cap);
  size_t need = ep_p2p_dispatch_layout(cfg, c->world, num_tokens).total;
  const size_t e2 = ep_p2p_experts_layout(cfg, num_local_experts, c->world, c->cap, expected_rows).total;
  const size_t e3 = make_layout(cfg, num_tokens).total;
  if (e2 > need) need = e2;
  if (e3 > need) need = e3;
  *bytes = need;
  return MLXR_CU_OK;
}

int mlxr_cu_moe_ep_dispatch_p2p(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, void* comm,
                                const int32_t* placement, const void* x, int64_t num_tokens, int32_t* pair_pos,
                                float* shared_gate, uint32_t epoch, void* workspace, size_t workspace_bytes,
                                void* stream) {
  MLXR_CHECK_ARG(epoch < EP_FLAG_POISON, "moe_ep: epoch=%u must be 0 (device counter) or in [1, 2^31)", epoch);
  if (int rc = validate(cfg, num_tokens)) return rc;
  if (int rc = ep_comm_check(comm, cfg)) return rc;
  EpComm* c = static_cast<EpComm*>(comm);
  const int world = c->world;
  MLXR_CHECK_ARG(num_tokens <= c->cap, "moe_ep_dispatch_p2p: %lld tokens exceed the comm capacity %lld",
                 (long long)num_tokens, (long long)c->cap);
  MLXR_CHECK_ARG(weights != nullptr, "moe_ep_dispatch_p2p: weights is NULL");
  const EpP2PDispatch dl = ep_p2p_dispatch_layout(cfg, world, num_tokens);
  MLXR_CHECK_ARG(workspace && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0 && workspace_bytes >= dl.total,
                 "moe_ep_dispatch_p2p: workspace NULL, not 256-byte aligned or smaller than %zu bytes", dl.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = workspace;
  const Layout L = make_layout(cfg, num_tokens);
  MLXR_CUDA_TRY(cudaMemsetAsync(at<int>(ws, L.status), 0, kStatusSlotBytes, st));
  if (epoch == 0) {  // device-resident step counter: advance it before any kernel of the step reads it
    launch_pdl(ep_bump_epoch_kernel, 1, 32, 0, st, c->local, c->bl, at<int>(ws, L.status));
    MLXR_LAUNCH_CHECK("ep_bump_epoch_kernel");
  }
  const int K = cfg->num_experts_per_tok;
  const int64_t R = L.R;
  int32_t* offsets = at<int32_t>(ws, L.offsets);
  int32_t* send_counts = at<int32_t>(ws, dl.counts);
  if (num_tokens == 0) {
    MLXR_CUDA_TRY(cudaMemsetAsync(offsets, 0, (size_t)(world + 1) * 4, st));
    MLXR_CUDA_TRY(cudaMemsetAsync(send_counts, 0, (size_t)world * 2 * 4, st));
  } else {
    MLXR_CHECK_ARG(x && pair_pos && aligned16(x), "moe_ep_dispatch_p2p: NULL or misaligned x / pair_pos");
    MLXR_CHECK_ARG(cfg->shared_expert_intermediate_size == 0 || shared_gate, "moe_ep_dispatch_p2p: shared_gate is NULL");
    if (int rc = run_router(cfg, weights, L, x, ws, nullptr, nullptr, st)) return rc;
    int32_t* dest = at<int32_t>(ws, dl.dest);
    launch_pdl(ep_pair_dest_kernel, (unsigned)((R + 255) / 256), 256, 0, st, at<int32_t>(ws, L.idx), num_tokens, K,
               world, placement, dest, at<int>(ws, L.status));
    MLXR_LAUNCH_CHECK("ep_pair_dest_kernel");
    Layout P = L;
    P.E = world;
    P.Is = 0;
    P.rows = num_tokens * (K < world ? K : world);
    P.bn1 = P.bn2 = 1 << 30;
    P.max_t1 = P.max_t2 = world + 1;
    if (int rc = run_permute(P, dest, x, ws, at<int32_t>(ws, L.counts), offsets, at<int32_t>(ws, L.sorted), pair_pos,
                             nullptr, 0, st, 1))
      return rc;
    launch_pdl(ep_counts_kernel, 1, 1024, 0, st, at<int32_t>(ws, L.idx), R, world, placement, at<int32_t>(ws, L.counts),
               send_counts);
    MLXR_LAUNCH_CHECK("ep_counts_kernel");
    launch_pdl(ep_pair_meta_kernel, (unsigned)((num_tokens + 127) / 128), 128, 0, st, at<int32_t>(ws, L.idx),
               at<uint16_t>(ws, L.w), pair_pos, num_tokens, K, world, placement, P.rows, at<int32_t>(ws, dl.meta),
               at<int>(ws, L.status));
    MLXR_LAUNCH_CHECK("ep_pair_meta_kernel");
    if (cfg->shared_expert_intermediate_size > 0)
      MLXR_CUDA_TRY(cudaMemcpyAsync(shared_gate, at<float>(ws, L.sig), (size_t)num_tokens * 4,
                                    cudaMemcpyDeviceToDevice, st));
  }
  const int64_t pairs_max = num_tokens * (K < world ? K : world);
  int grid = (int)((pairs_max + 7) / 8);
  if (grid > 4 * 148) grid = 4 * 148;
  if (grid < 1) grid = 1;
  launch_pdl(ep_send_kernel, grid, 256, 0, st, c->peers, c->bl, c->rank, world, c->cap,
             static_cast<const uint16_t*>(ep_send_rows(L, x, ws)), c->D, K, at<int32_t>(ws, L.sorted), offsets,
             at<int32_t>(ws, dl.meta),
             send_counts, pair_pos, epoch, reinterpret_cast<int*>(c->local + c->bl.done), at<int>(ws, L.status));
  MLXR_LAUNCH_CHECK("ep_send_kernel");
  return MLXR_CU_OK;
}

int mlxr_cu_moe_ep_experts_p2p(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* local_weights,
                               int num_local_experts, void* comm, int64_t expected_rows, uint32_t epoch,
                               void* workspace, size_t workspace_bytes, void* stream) {
  MLXR_CHECK_ARG(epoch < EP_FLAG_POISON, "moe_ep: epoch=%u must be 0 (device counter) or in [1, 2^31)", epoch);
  if (int rc = ep_comm_check(comm, cfg)) return rc;
  EpComm* c = static_cast<EpComm*>(comm);
  MLXR_CHECK_ARG(local_weights != nullptr && num_local_experts >= 1 && num_local_experts <= cfg->num_experts,
                 "moe_ep_experts_p2p: weights NULL or num_local_experts=%d out of range", num_local_experts);
  if (int rc = validate(cfg, (int64_t)c->world * c->cap)) return rc;
  mlxr_cu_moe_config lc = *cfg;
  lc.num_experts = num_local_experts;
  lc.shared_expert_intermediate_size = 0;
  const Layout L = ep_p2p_experts_layout(cfg, num_local_experts, c->world, c->cap, expected_rows);
  if (int rc = check_ws(L, workspace, workspace_bytes)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = workspace;  // the status word was cleared by this step's dispatch
  int* status = at<int>(ws, L.status);
  const uint8_t* b = c->local;
  launch_pdl(ep_wait_flags_kernel, 1, 64, 0, st, reinterpret_cast<const uint32_t*>(b + c->bl.flag_disp), c->world,
             epoch, reinterpret_cast<const uint32_t*>(b + c->bl.epoch), 5 * kWaitLimitNs, status);
  MLXR_LAUNCH_CHECK("ep_wait_flags_kernel(dispatch)");
  const int32_t* meta = reinterpret_cast<const int32_t*>(b + c->bl.recv_meta);
  const int32_t* counts = reinterpret_cast<const int32_t*>(b + c->bl.counts);
  launch_pdl(ep_slot_expert_p2p_kernel, (unsigned)((L.R + 255) / 256 < 4096 ? (L.R + 255) / 256 : 4096), 256, 0, st,
             meta, counts, c->world, c->cap, c->K, num_local_experts, at<int32_t>(ws, L.idx), status);
  MLXR_LAUNCH_CHECK("ep_slot_expert_p2p_kernel");
  if (int rc = run_permute(L, at<int32_t>(ws, L.idx), b + c->bl.recv_x, ws, at<int32_t>(ws, L.counts),
                           at<int32_t>(ws, L.offsets), at<int32_t>(ws, L.sorted), at<int32_t>(ws, L.inv),
                           at<uint16_t>(ws, L.xs), lc.bits == 4, st, 1, 1))
    return rc;
  if (int rc = run_experts(&lc, local_weights, L, ws, st, 7)) return rc;
  int grid = (int)(c->world * c->cap < 8 * 148 ? c->world * c->cap : 8 * 148);
  launch_pdl(ep_reduce_send_kernel, grid, L.D >= 2048 ? 256 : 128, 0, st, c->peers, c->bl, c->rank, c->world, c->cap,
             at<uint16_t>(ws, L.y), at<int32_t>(ws, L.inv), meta, counts, c->K, c->D, L.rows, epoch,
             reinterpret_cast<int*>(c->local + c->bl.done), status);
  MLXR_LAUNCH_CHECK("ep_reduce_send_kernel");
  return MLXR_CU_OK;
}

int mlxr_cu_moe_ep_combine_p2p(const mlxr_cu_moe_config* cfg, const mlxr_cu_moe_weights* weights, void* comm,
                               const void* x, int64_t num_tokens, const int32_t* pair_pos, const float* shared_gate,
                               void* out, uint32_t epoch, void* workspace, size_t workspace_bytes, void* stream) {
  MLXR_CHECK_ARG(epoch < EP_FLAG_POISON, "moe_ep: epoch=%u must be 0 (device counter) or in [1, 2^31)", epoch);
  if (int rc = validate(cfg, num_tokens)) return rc;
  if (int rc = ep_comm_check(comm, cfg)) return rc;
  EpComm* c = static_cast<EpComm*>(comm);
  const Layout L = make_layout(cfg, num_tokens);
  if (int rc = check_ws(L, workspace, workspace_bytes)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = workspace;  // the status word was cleared by this step's dispatch
  const uint16_t* ysh = nullptr;
  if (num_tokens > 0 && L.Is > 0) {
    MLXR_CHECK_ARG(x && shared_gate && weights && aligned16(x), "moe_ep_combine_p2p: x / shared_gate / weights");
    // The shared expert runs before the wait: it overlaps the other ranks' experts.
    launch_pdl(shared_tiles_kernel, (unsigned)((L.max_tsh + 255) / 256), 256, 0, st, at<GemmTile>(ws, L.tsh),
               at<int32_t>(ws, L.nsh), L.T, L.bns, L.max_tsh);
    MLXR_LAUNCH_CHECK("shared_tiles_kernel");
    if (int rc = run_shared(cfg, weights, L, x, ws, st)) return rc;
    ysh = at<uint16_t>(ws, L.ysh);
  }
  launch_pdl(ep_wait_flags_kernel, 1, 64, 0, st, reinterpret_cast<const uint32_t*>(c->local + c->bl.flag_back),
             c->world, epoch, reinterpret_cast<const uint32_t*>(c->local + c->bl.epoch), 5 * kWaitLimitNs,
             at<int>(ws, L.status));
  MLXR_LAUNCH_CHECK("ep_wait_flags_kernel(combine)");
  if (num_tokens == 0) return MLXR_CU_OK;
  MLXR_CHECK_ARG(pair_pos && out && aligned16(out), "moe_ep_combine_p2p: NULL or misaligned argument");
  launch_pdl(ep_combine_kernel, (unsigned)L.T, L.D >= 2048 ? 256 : 128, 0, st,
             reinterpret_cast<const uint16_t*>(c->local + c->bl.back), pair_pos, L.K, L.D,
             (int64_t)c->world * c->cap, ysh, shared_gate, static_cast<uint16_t*>(out), at<int>(ws, L.status));
  MLXR_LAUNCH_CHECK("ep_combine_kernel(p2p)");
  return MLXR_CU_OK;
}

int mlxr_cu_gather_qmm_workspace_size(mlxr_cu_dtype x_dtype, int64_t x_batch, int64_t M, int64_t K, int64_t w_batch,
                                      int64_t N, int64_t num_indices, int transpose, int group_size, int bits,
                                      size_t* bytes) {
  MLXR_CHECK_ARG(bytes != nullptr, "gather_qmm_workspace_size: bytes is NULL");
  MLXR_CHECK_ARG(M >= 0 && K > 0 && N > 0 && x_batch > 0 && w_batch > 0 && num_indices >= 0,
                 "gather_qmm_workspace_size: bad shape");
  group_size = group_size == 0 ? 64 : group_size;
  bits = bits == 0 ? 4 : bits;
  const int64_t R = num_indices * M;
  *bytes = 0;
  if (!gqmm_fast_ok(x_dtype, K, N, w_batch, transpose, group_size, bits, R)) return MLXR_CU_OK;
  const mlxr_cu_moe_config c = gqmm_cfg(K, N, w_batch, bits);
  *bytes = gqmm_layout(&c, R).total;
  return MLXR_CU_OK;
}

int mlxr_cu_gather_qmm_ws(const void* x, mlxr_cu_dtype x_dtype, int64_t x_batch, int64_t M, int64_t K,
                          const uint32_t* w, const void* scales, const void* biases, int64_t w_batch, int64_t N,
                          const uint32_t* lhs_indices, const uint32_t* rhs_indices, int64_t num_indices,
                          int transpose, int group_size, int bits, const char* mode, int sorted_indices, void* out,
                          void* workspace, size_t workspace_bytes, void* stream) {
  const int gs = group_size == 0 ? 64 : group_size;
  const int b = bits == 0 ? 4 : bits;
  const int64_t R = num_indices * M;
  const bool fast = (mode == nullptr || std::strcmp(mode, "affine") == 0) &&
                    gqmm_fast_ok(x_dtype, K, N, w_batch, transpose, gs, b, R) && x && w && scales && biases && out;
  if (!fast)  // every other shape: the general CUDA-core kernel (no workspace)
    return mlxr_cu_gather_qmm(x, x_dtype, x_batch, M, K, w, scales, biases, w_batch, N, lhs_indices, rhs_indices,
                              num_indices, transpose, group_size, bits, mode, sorted_indices, out, stream);
  MLXR_CHECK_ARG(lhs_indices || num_indices <= x_batch, "gather_qmm: num_indices exceeds x batch without lhs_indices");
  MLXR_CHECK_ARG(rhs_indices || num_indices <= w_batch, "gather_qmm: num_indices exceeds w batch without rhs_indices");
  MLXR_CHECK_ARG(aligned16(x) && aligned16(out) && aligned16(w), "gather_qmm_ws: x, out and w must be 16-byte aligned");
  MLXR_CHECK_ARG((reinterpret_cast<uintptr_t>(scales) & 3) == 0 && (reinterpret_cast<uintptr_t>(biases) & 3) == 0,
                 "gather_qmm_ws: scales/biases must be 4-byte aligned");
  const mlxr_cu_moe_config c = gqmm_cfg(K, N, w_batch, b);
  const GqmmLayout G = gqmm_layout(&c, R);
  const Layout& L = G.L;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0 || workspace_bytes < G.total)
    return set_error(MLXR_CU_ERR_WORKSPACE,
                     "gather_qmm_ws: workspace NULL, not 256-byte aligned or smaller than %zu bytes", G.total);
  int* op_status = op_status_word();
  if (!op_status) return MLXR_CU_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* ws = workspace;
  int* status = at<int>(ws, L.status);
  MLXR_CUDA_TRY(cudaMemsetAsync(status, 0, kStatusSlotBytes, st));
  int32_t* flat = at<int32_t>(ws, G.flat);
  const int fgrid = (int)std::min<int64_t>((R + 255) / 256, 4 * 148);
  launch_pdl(gqmm_flat_experts_kernel, fgrid, 256, 0, st, rhs_indices, R, M, (int)w_batch, flat, status);
  MLXR_LAUNCH_CHECK("gqmm_flat_experts_kernel");
  // Counting sort by expert (no row gather: the rows come through lhs below).
  if (int rc = run_permute(L, flat, nullptr, ws, at<int32_t>(ws, L.counts), at<int32_t>(ws, L.offsets),
                           at<int32_t>(ws, L.sorted), at<int32_t>(ws, L.inv), nullptr, 0, st))
    return rc;
  const int ggrid = (int)std::min<int64_t>((R + 7) / 8, 4 * 148);
  launch_pdl(gqmm_gather_kernel, ggrid, 256, 0, st, at<int32_t>(ws, L.sorted), R, lhs_indices, M, x_batch,
             static_cast<const uint16_t*>(x), (int)K, b == 4 ? 1 : 0, at<uint16_t>(ws, L.xs), status);
  MLXR_LAUNCH_CHECK("gqmm_gather_kernel");
  GroupedGemmProblem p{};
  // Two 128-row blocks of the weight per work item (two accumulators, two
  // MMA issuers, plain stores) when N allows it, as the block's down
  // projection runs.
  p.pair = (N % 256 == 0) ? 1 : 0;
  p.nmat = p.pair ? 2 : 1;
  p.bn = L.bn1;
  p.bits = b;
  p.w[0] = p.w[1] = w;
  p.s[0] = p.s[1] = static_cast<const uint16_t*>(scales);
  p.b[0] = p.b[1] = static_cast<const uint16_t*>(biases);
  p.w_rows = w_batch * N;
  p.n_out = (int)N;
  p.k_dim = (int)K;
  p.num_experts = (int)w_batch;
  p.act = at<uint16_t>(ws, L.xs);
  p.act_rows = L.rows_pad;
  p.tiles = at<GemmTile>(ws, L.t1);
  p.num_tiles = at<int32_t>(ws, L.n1);
  p.max_tiles = L.max_t1;
  p.out = at<uint16_t>(ws, L.h);
  p.out_rows = L.rows;
  p.perm_out = 0;
  p.status = status;
  p.splits = L.s1;
  p.max_split_rows = L.split_rows;
  p.partial = L.split_rows ? at<float>(ws, L.part) : nullptr;
  p.counters = L.split_rows ? at<int32_t>(ws, L.cnt) : nullptr;
  p.sched = status + kSchedExperts1;
  if (int rc = launch_grouped_gemm(p, st)) return rc;
  launch_pdl(gqmm_unpermute_kernel, ggrid, 256, 0, st, at<uint16_t>(ws, L.h), at<int32_t>(ws, L.inv), R, (int)N,
             static_cast<uint16_t*>(out), status, op_status);
  MLXR_LAUNCH_CHECK("gqmm_unpermute_kernel");
  return MLXR_CU_OK;
}

int mlxr_cu_quantized_matmul_ws(const void* x, mlxr_cu_dtype x_dtype, int64_t M, int64_t K, const uint32_t* w,
                                const void* scales, const void* biases, int64_t N, int transpose, int group_size,
                                int bits, const char* mode, void* out, void* workspace, size_t workspace_bytes,
                                void* stream) {
  // One weight matrix, M rows: the gather with one index and rows M.
  return mlxr_cu_gather_qmm_ws(x, x_dtype, 1, M, K, w, scales, biases, 1, N, nullptr, nullptr, 1, transpose,
                               group_size, bits, mode, 0, out, workspace, workspace_bytes, stream);
}

}  // extern "C"
