// Launch interface of the grouped dequantising GEMM (grouped_gemm.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mlxr {

struct GemmTile;

struct GroupedGemmProblem {
  int nmat;                   // 2 = gate/up pair with SwiGLU epilogue, 1 = plain
  int bn;                     // token-tile width (16, 32, 64, 128, 256)
  int bits;                   // 4 or 8
  const uint32_t* w[2];       // packed weights, [w_rows, k_dim*bits/32]
  const uint16_t* s[2];       // bf16 scales [w_rows, k_dim/64]
  const uint16_t* b[2];       // bf16 biases
  int64_t w_rows;             // num_experts * n_out
  int n_out;                  // output features per expert (multiple of 128)
  int k_dim;                  // reduction length (multiple of 64)
  int num_experts;
  const uint16_t* act;        // bf16 activations [act_rows, k_dim] (sorted rows)
  int64_t act_rows;
  const GemmTile* tiles;      // device tile list
  const int32_t* num_tiles;   // device count
  int max_tiles;
  uint16_t* out;              // bf16 [out_rows, n_out]
  int64_t out_rows;
  int perm_out;               // 1: write out's feature axis in the 4-bit chunk K order
  int pair;                   // nmat 2 only: w[0] rows m and m+128 as the two matrices (plain store)
  int w_expert_rows;          // weight rows per expert (0 = n_out; 2*n_out for a packed gate|up
                              // whose w[1], s[1], b[1] point n_out rows into the same tensor)
  int64_t w_rows1;            // rows of matrix 1's tensor view (0 = w_rows)
  int glu;                    // nmat 2, not pair: 0 = SwiGLU, 1 = GeGLU (gelu_approx(gate) * up)
  int* status;
  int grid;                   // 0 = one CTA per SM
  int splits;                 // split-K factor (0/1 = none); needs partial and counters
  int max_split_rows;         // row slices (tile x m-tile) the split buffers hold
  float* partial;             // fp32 [max_split_rows][splits][4][nmat][bn][32]
  int32_t* counters;          // [max_split_rows][4], zero before the launch
  // Fused launch (nmat 2, not split): after this problem (gate|up + SwiGLU),
  // the down projection in row pairs over the same tiles: weights w2
  // [w2_rows, k_dim2*bits/32] (+ s2, b2), activations act2 = this problem's
  // out, output out2 [out_rows, n_out2]; tile_ready [max_tiles] zeroed.
  int fused;
  const uint32_t* w2;
  const uint16_t* s2;
  const uint16_t* b2;
  int64_t w2_rows;
  int n_out2;
  int k_dim2;
  int64_t act2_rows;
  uint16_t* out2;
  int32_t* tile_ready;
  int32_t* sched;             // 2 ints, zero before the launch (work queue; left zero after it)
};

int launch_grouped_gemm(const GroupedGemmProblem& p, cudaStream_t st);
// 2-D row-major TMA tensor map (grouped_gemm.cu): `inner` elements of
// elem_bytes per row, `rows` rows, box box_inner x box_rows.
int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                uint64_t rows, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz);
int num_sms_current();

}  // namespace mlxr
