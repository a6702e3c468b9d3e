// Host side of the grouped dequantising GEMM: tensor-map encoding and the
// dispatch over (matrices per item, token-tile width, bits).
#include <cudaTypedefs.h>

#include <mutex>

#include "gemm_launch.h"
#include "grouped_gemm.cuh"

namespace mlxr {

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D row-major tensor map: inner extent `inner` elements, `rows` rows.
int make_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                       uint64_t rows, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  auto enc = get_encode_fn();
  if (!enc) return set_error(MLXR_CU_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "TMA operand %p is not 16-byte aligned", base);
  if ((inner * elem_bytes) % 16 != 0)
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "TMA row pitch %llu bytes is not a multiple of 16",
                     (unsigned long long)(inner * elem_bytes));
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(MLXR_CU_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) inner=%llu rows=%llu box=%u x %u", (int)r,
                     (unsigned long long)inner, (unsigned long long)rows, box_inner, box_rows);
  return MLXR_CU_OK;
}

int num_sms_current() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <int NMAT, int BN, int BITS, bool SPLITK, bool FUSED, bool GLU = false>
static int launch_one(const GroupedGemmProblem& p, cudaStream_t st) {
  using C = GG<NMAT, BN, BITS>;
  CUtensorMap ta0, ta1, tb, ta2, tb2;
  const uint64_t kw = (uint64_t)p.k_dim * BITS / 32;
  if (int rc = make_map_2d(&ta0, p.w[0], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, kw, (uint64_t)p.w_rows, C::KW, C::BM,
                           CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  if (NMAT == 2) {
    if (int rc = make_map_2d(&ta1, p.w[1], CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, kw,
                             (uint64_t)(p.w_rows1 > 0 ? p.w_rows1 : p.w_rows), C::KW, C::BM,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
  } else {
    ta1 = ta0;
  }
  if (int rc = make_map_2d(&tb, p.act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)p.k_dim, (uint64_t)p.act_rows,
                           C::BK, BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return rc;
  if (FUSED) {
    if (int rc = make_map_2d(&ta2, p.w2, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, (uint64_t)p.k_dim2 * BITS / 32,
                             (uint64_t)p.w2_rows, C::KW, C::BM, CU_TENSOR_MAP_SWIZZLE_NONE))
      return rc;
    if (int rc = make_map_2d(&tb2, p.out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)p.k_dim2,
                             (uint64_t)p.act2_rows, C::BK, BN, CU_TENSOR_MAP_SWIZZLE_128B))
      return rc;
  } else {
    ta2 = ta0;
    tb2 = tb;
  }
  // Scale/bias maps for the staging ring: [rows, K/64] bf16 viewed as 2-D,
  // a {8 groups x 128 rows} box. TMA needs 16-byte aligned bases and row
  // pitches (a multiple of 8 groups); shapes that miss either keep the
  // per-thread loads (the flag stays 0 and the maps are not used).
  CUtensorMap ts0 = ta0, tz0 = ta0, ts1 = ta0, tz1 = ta0, ts2 = ta0, tz2 = ta0;
  auto sb_maps = [&](const uint16_t* sc, const uint16_t* bi, int64_t rows, int k_dim, CUtensorMap* ms,
                     CUtensorMap* mz) -> int {
    const int groups = k_dim / 64;
    if (SPLITK || groups % C::SB_K != 0 || !sc || !bi || (reinterpret_cast<uintptr_t>(sc) & 15) ||
        (reinterpret_cast<uintptr_t>(bi) & 15))
      return 0;
    if (make_map_2d(ms, sc, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (uint64_t)groups, (uint64_t)rows, C::SB_K, C::BM,
                    CU_TENSOR_MAP_SWIZZLE_NONE) ||
        make_map_2d(mz, bi, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (uint64_t)groups, (uint64_t)rows, C::SB_K, C::BM,
                    CU_TENSOR_MAP_SWIZZLE_NONE)) {
      mlxr_cu_clear_error();  // not an error: the kernel falls back to per-thread loads
      return 0;
    }
    return 1;
  };
  int sb1 = sb_maps(p.s[0], p.b[0], p.w_rows, p.k_dim, &ts0, &tz0);
  if (sb1 && NMAT == 2)
    sb1 = sb_maps(p.s[1], p.b[1], p.w_rows1 > 0 ? p.w_rows1 : p.w_rows, p.k_dim, &ts1, &tz1);
  else if (sb1) {
    ts1 = ts0;
    tz1 = tz0;
  }
  const int sb2 = FUSED ? sb_maps(p.s2, p.b2, p.w2_rows, p.k_dim2, &ts2, &tz2) : 0;
  auto kern = grouped_dequant_gemm_kernel<NMAT, BN, BITS, SPLITK, FUSED, GLU>;
  static std::atomic<uint64_t> attr_done{0};  // per instantiation and device
  if (int rc = ensure_smem_attr(kern, C::SMEM_BYTES, attr_done)) return rc;
  GemmArgs a;
  a.scales[0] = p.s[0];
  a.scales[1] = NMAT == 2 ? p.s[1] : p.s[0];
  a.biases[0] = p.b[0];
  a.biases[1] = NMAT == 2 ? p.b[1] : p.b[0];
  a.tiles = p.tiles;
  a.num_tiles = p.num_tiles;
  a.out = p.out;
  a.n_out = p.n_out;
  a.k_dim = p.k_dim;
  a.num_experts = p.num_experts;
  a.max_tiles = p.max_tiles;
  a.out_rows = p.out_rows;
  a.perm_out = p.perm_out;
  a.pair = p.pair;
  a.w_rows1 = p.w_expert_rows > 0 ? p.w_expert_rows : p.n_out;
  a.status = p.status;
  a.sb1 = sb1;
  a.sb2 = sb2;
  a.splits = p.splits > 1 ? p.splits : 1;
  a.max_split_rows = p.max_split_rows;
  a.partial = p.partial;
  a.counters = p.counters;
  if (a.splits > 1 && (!a.partial || !a.counters || a.max_split_rows <= 0))
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "grouped gemm: split-K needs partial and counter buffers");
  a.scales2 = p.s2;
  a.biases2 = p.b2;
  a.out2 = p.out2;
  a.n_out2 = p.n_out2;
  a.k_dim2 = p.k_dim2;
  a.tile_ready = p.tile_ready;
  a.sched = p.sched;
  if (!a.sched) return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "grouped gemm: no work-queue counters");
  if (FUSED && (!p.w2 || !p.s2 || !p.b2 || !p.out2 || !p.tile_ready || p.n_out2 % 256 != 0 || p.k_dim2 % 64 != 0 ||
                p.k_dim2 != p.n_out))
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "grouped gemm: bad fused second phase");
  // k-parity accumulators: every work item needs a k-step of each parity.
  if (C::KP == 2 && ((p.k_dim / C::BK) / a.splits < 2 || (FUSED && p.k_dim2 / C::BK < 2)))
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "grouped gemm: K=%d over %d splits leaves a work item one k-step",
                     p.k_dim, a.splits);
  const int grid = p.grid > 0 ? p.grid : num_sms_current();
  launch_pdl(kern, grid, C::NUM_THREADS, C::SMEM_BYTES, st, ta0, ta1, tb, ta2, tb2, ts0, tz0, ts1, tz1, ts2, tz2, a);
  MLXR_LAUNCH_CHECK("grouped_dequant_gemm_kernel");
  return MLXR_CU_OK;
}

int launch_grouped_gemm(const GroupedGemmProblem& p, cudaStream_t st) {
  if (p.pair && (p.nmat != 2 || p.n_out % 256 != 0))
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "grouped gemm: paired row blocks need nmat 2 and n_out %% 256 == 0");
  if (p.n_out % 128 != 0 || p.k_dim % 64 != 0)
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "grouped gemm: n_out=%d must be a multiple of 128 and K=%d of 64",
                     p.n_out, p.k_dim);
  // Split-K only for the decode tile widths (few work items come from few tokens).
  if (p.splits > 1 && p.bn > 32)
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "grouped gemm: split-K is built for bn <= 32 (bn=%d)", p.bn);
  if (p.fused && (p.nmat != 2 || p.splits > 1 || p.pair))
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "grouped gemm: the fused launch needs nmat 2, no split, no pair");
  if (p.glu && (p.nmat != 2 || p.pair))
    return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "grouped gemm: GeGLU needs a gate|up pair (nmat 2, no pair)");
  if (p.glu) {  // GeGLU gate|up instantiations (the Gemma 4 experts)
#define MLXR_GG_GLU(BNV, BT)                                                                                     \
  if (p.fused && p.bn == BNV && p.bits == BT) return launch_one<2, BNV, BT, false, true, true>(p, st);        \
  if (!p.fused && p.splits > 1 && p.bn == BNV && p.bits == BT && BNV <= 32)                                   \
    return launch_one<2, BNV, BT, (BNV <= 32), false, true>(p, st);                                           \
  if (!p.fused && p.splits <= 1 && p.bn == BNV && p.bits == BT) return launch_one<2, BNV, BT, false, false, true>(p, st);
    MLXR_GG_GLU(16, 4) MLXR_GG_GLU(32, 4) MLXR_GG_GLU(64, 4) MLXR_GG_GLU(128, 4)
    MLXR_GG_GLU(16, 8) MLXR_GG_GLU(32, 8) MLXR_GG_GLU(64, 8) MLXR_GG_GLU(128, 8)
#undef MLXR_GG_GLU
    return set_error(MLXR_CU_ERR_UNSUPPORTED, "grouped gemm: no GeGLU kernel for bn=%d bits=%d", p.bn, p.bits);
  }
#define MLXR_GG_FUSED(BNV, BT) \
  if (p.fused && p.bn == BNV && p.bits == BT) return launch_one<2, BNV, BT, false, true>(p, st);
  MLXR_GG_FUSED(16, 4) MLXR_GG_FUSED(32, 4) MLXR_GG_FUSED(64, 4) MLXR_GG_FUSED(128, 4)
  MLXR_GG_FUSED(16, 8) MLXR_GG_FUSED(32, 8) MLXR_GG_FUSED(64, 8) MLXR_GG_FUSED(128, 8)
#undef MLXR_GG_FUSED
#define MLXR_GG_SPLIT(NM, BNV, BT) \
  if (p.splits > 1 && p.nmat == NM && p.bn == BNV && p.bits == BT) return launch_one<NM, BNV, BT, true, false>(p, st);
  MLXR_GG_SPLIT(2, 16, 4) MLXR_GG_SPLIT(2, 32, 4) MLXR_GG_SPLIT(1, 16, 4) MLXR_GG_SPLIT(1, 32, 4)
  MLXR_GG_SPLIT(2, 16, 8) MLXR_GG_SPLIT(2, 32, 8) MLXR_GG_SPLIT(1, 16, 8) MLXR_GG_SPLIT(1, 32, 8)
#undef MLXR_GG_SPLIT
#define MLXR_GG_CASE(NM, BNV, BT) \
  if (p.nmat == NM && p.bn == BNV && p.bits == BT) return launch_one<NM, BNV, BT, false, false>(p, st);
  MLXR_GG_CASE(2, 16, 4) MLXR_GG_CASE(2, 32, 4) MLXR_GG_CASE(2, 64, 4) MLXR_GG_CASE(2, 128, 4)
  MLXR_GG_CASE(1, 16, 4) MLXR_GG_CASE(1, 32, 4) MLXR_GG_CASE(1, 64, 4) MLXR_GG_CASE(1, 128, 4) MLXR_GG_CASE(1, 256, 4)
  MLXR_GG_CASE(2, 16, 8) MLXR_GG_CASE(2, 32, 8) MLXR_GG_CASE(2, 64, 8) MLXR_GG_CASE(2, 128, 8)
  MLXR_GG_CASE(1, 16, 8) MLXR_GG_CASE(1, 32, 8) MLXR_GG_CASE(1, 64, 8) MLXR_GG_CASE(1, 128, 8) MLXR_GG_CASE(1, 256, 8)
#undef MLXR_GG_CASE
  return set_error(MLXR_CU_ERR_UNSUPPORTED, "grouped gemm: no kernel for nmat=%d bn=%d bits=%d", p.nmat, p.bn, p.bits);
}

}  // namespace mlxr
