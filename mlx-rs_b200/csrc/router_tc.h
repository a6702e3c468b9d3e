// Launch interface of the tensor-core router logits (router_tc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mlxr {

// Workspace of one launch: digit planes of the tokens and of the router
// rows (4 int8 planes each, rows padded to the tile, D padded to 128) and
// the per-row exponent / truncation count.
// Batches up to this size use 16-token tiles (else 64). Whenever the tiles
// alone would fill less than about one wave of CTAs the launch takes the
// split-K form: the k range cut over CTAs, partial digit sums finished by
// logits_from_partials_kernel.
constexpr int64_t kRouterTcSplitMaxT = 256;

struct RouterTcLayout {
  bool split = false;
  int bn = 64, splits = 1, kps = 0;
  int64_t Dp = 0, rows_pad_x = 0, rows_pad_w = 0;
  size_t xdig = 0, wdig = 0, xinfo = 0, winfo = 0, part = 0, total = 0;
};
// budget: bytes the caller would like the layout to stay within (the k
// range is cut into fewer slices to get there; the total may still exceed
// it at one slice).
RouterTcLayout router_tc_layout(int64_t T, int E, int D, size_t budget = ~(size_t)0);
bool router_tc_supported(int D);

// logits lg [T, E] bf16 = bf16(fp32(exact x[t] . wg[e]) + bias[e]) (bias may
// be NULL). In the split-K form (router_tc_layout(...).split) it writes the
// partial digit sums instead (layout.part, [splits][5][T][E] int32) and
// logits_from_partials_kernel forms the logits.
struct RouterTcProblem {
  const uint16_t* x;   // [T, D] bf16, 16-byte aligned
  int64_t T;
  const uint16_t* wg;  // [E, D] bf16, 16-byte aligned
  int E;
  int D;
  const float* bias;
  uint16_t* lg;
  void* workspace;     // router_tc_layout(T, E, D, budget).total bytes, 256-byte aligned
  int* status;         // device status word (timeouts)
  size_t budget;       // the layout's budget (the same value sizes the workspace)
};
int launch_router_tc(const RouterTcProblem& p, cudaStream_t st);

}  // namespace mlxr
