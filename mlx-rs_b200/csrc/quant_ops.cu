// The quantised op family behind the C ABI: quantize, dequantize,
// quantized_matmul, gather_qmm, gather_mm (crates/mlxr/src/ops/quantization.rs
// and arithmetic.rs:1577 of the reference), plus the seeded input generator.
//
// These are the general-shape entry points (any M, N, K, batch and index
// pattern). The MoE block does not route through them: it runs the grouped
// tcgen05 kernels in grouped_gemm.cu on the expert-sorted rows.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "common.cuh"

namespace mlxr {

// ------------------------------------------------------------ errors ----
static thread_local std::string t_last_error;
static thread_local bool t_has_error = false;

int set_error(int status, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  t_has_error = true;
  return status;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MLXR_CU_OK;
  return set_error(MLXR_CU_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

static inline bool mode_ok(const char* mode) { return mode == nullptr || std::strcmp(mode, "affine") == 0; }

// ---------------------------------------------------------- dtype io ----
template <int DT>
struct IO;
template <>
struct IO<MLXR_CU_BFLOAT16> {
  static __device__ float load(const void* p, int64_t i) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  }
  static __device__ void store(void* p, int64_t i, float v) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  }
  static __device__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <>
struct IO<MLXR_CU_FLOAT16> {
  static __device__ float load(const void* p, int64_t i) { return __half2float(reinterpret_cast<const __half*>(p)[i]); }
  static __device__ void store(void* p, int64_t i, float v) { reinterpret_cast<__half*>(p)[i] = __float2half_rn(v); }
  static __device__ float round(float v) { return __half2float(__float2half_rn(v)); }
};
template <>
struct IO<MLXR_CU_FLOAT32> {
  static __device__ float load(const void* p, int64_t i) { return reinterpret_cast<const float*>(p)[i]; }
  static __device__ void store(void* p, int64_t i, float v) { reinterpret_cast<float*>(p)[i] = v; }
  static __device__ float round(float v) { return v; }
};

#define MLXR_DISPATCH_DTYPE(dt, DT, ...)                                      \
  switch (dt) {                                                               \
    case MLXR_CU_BFLOAT16: { constexpr int DT = MLXR_CU_BFLOAT16; __VA_ARGS__; break; } \
    case MLXR_CU_FLOAT16: { constexpr int DT = MLXR_CU_FLOAT16; __VA_ARGS__; break; }   \
    case MLXR_CU_FLOAT32: { constexpr int DT = MLXR_CU_FLOAT32; __VA_ARGS__; break; }   \
    default: return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "unknown dtype %d", (int)dt); \
  }

__device__ inline uint32_t get_code(const uint32_t* row, int64_t k, int bits) {
  const int per = 32 / bits;
  return (row[k / per] >> ((k % per) * bits)) & ((1u << bits) - 1u);
}

// ----------------------------------------------------------- quantize ---
// One thread per (row, group). MLX's affine quantiser (ml-explore/mlx
// v0.31.2, `affine_quantize` in mlx/ops.cpp and the CPU kernel in
// mlx/backend/cpu/quantized.cpp), in fp32 with explicitly rounded IEEE
// operations so that the bytes do not depend on the compiler's contraction
// or fast-math choices:
//   scale = max((max - min) / n_bins, 1e-7), negated unless |min| > |max|;
//   edge = min when |min| > |max|, else max;
//   q0 = rint(edge / scale); q0 != 0: scale = edge / q0, bias = edge (zero is
//   then exactly representable); q0 == 0: bias = 0;
//   q = clamp(rint((w - bias) / scale), 0, n_bins) from the fp32 pair; the
//   pair is rounded to the weight dtype only when stored.
// The group's elements are read 16 bytes at a time (vec != 0: w is 16-byte
// aligned; groups of 32, 64 or 128 elements are then 16-byte aligned too).
template <int DT>
struct QVec {
  static constexpr int N = DT == MLXR_CU_FLOAT32 ? 4 : 8;  // elements per 16-byte load
  static __device__ void load(const void* w, int64_t i, float (&v)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(w) + i * (16 / N)));
    const uint32_t a[4] = {u.x, u.y, u.z, u.w};
    if constexpr (DT == MLXR_CU_FLOAT32) {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = __uint_as_float(a[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[2 * j] = IO<DT>::load(&a[j], 0);
        v[2 * j + 1] = IO<DT>::load(&a[j], 1);
      }
    }
  }
};

template <int DT>
__global__ void quantize_kernel(const void* __restrict__ w, int64_t rows, int64_t cols, int gs, int bits,
                                uint32_t* __restrict__ wq, void* __restrict__ scales, void* __restrict__ biases,
                                int vec) {
  const int64_t ngroups = cols / gs;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= rows * ngroups) return;
  const int64_t r = gid / ngroups, g = gid % ngroups;
  const int64_t base = r * cols + g * gs;
  constexpr int NV = QVec<DT>::N;
  float mn = INFINITY, mx = -INFINITY;
  if (vec) {
    for (int i = 0; i < gs; i += NV) {
      float v[8];
      QVec<DT>::load(w, base + i, v);
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        mn = fminf(mn, v[j]);
        mx = fmaxf(mx, v[j]);
      }
    }
  } else {
    for (int i = 0; i < gs; ++i) {
      const float v = IO<DT>::load(w, base + i);
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
  }
  const float nbins = (float)((1 << bits) - 1);
  const bool min_edge = fabsf(mn) > fabsf(mx);
  float sc = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), nbins), 1e-7f);
  if (!min_edge) sc = -sc;
  const float edge = min_edge ? mn : mx;
  const float q0 = rintf(__fdiv_rn(edge, sc));
  float bi = 0.0f;
  if (q0 != 0.0f) {
    sc = __fdiv_rn(edge, q0);
    bi = edge;
  }
  const int per = 32 / bits;
  uint32_t* qrow = wq + r * (cols / per) + g * gs / per;
  auto code = [&](float v) {
    return (uint32_t)fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(v, bi), sc)), 0.0f), nbins);
  };
  if (vec) {
    // word wi holds elements [wi*per, wi*per + per); per (4, 8 or 16) and NV
    // (4 or 8) divide the group, so each load feeds whole or partial words.
    uint32_t word = 0;
    for (int i = 0; i < gs; i += NV) {
      float v[8];
      QVec<DT>::load(w, base + i, v);
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int e = i + j;
        word |= code(v[j]) << ((e % per) * bits);
        if (e % per == per - 1) {
          qrow[e / per] = word;
          word = 0;
        }
      }
    }
  } else {
    for (int wi = 0; wi < gs / per; ++wi) {
      uint32_t word = 0;
      for (int j = 0; j < per; ++j) word |= code(IO<DT>::load(w, base + wi * per + j)) << (j * bits);
      qrow[wi] = word;
    }
  }
  IO<DT>::store(scales, gid, sc);
  IO<DT>::store(biases, gid, bi);
}

// --------------------------------------------------------- dequantize ---
template <int SDT, int ODT>
__global__ void dequantize_kernel(const uint32_t* __restrict__ wq, const void* __restrict__ s,
                                  const void* __restrict__ b, int64_t rows, int64_t cols, int gs, int bits,
                                  void* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols, k = i % cols;
  const int64_t g = r * (cols / gs) + k / gs;
  const uint32_t q = get_code(wq + r * (cols * bits / 32), k, bits);
  IO<ODT>::store(out, i, __fmaf_rn(IO<SDT>::load(s, g), (float)q, IO<SDT>::load(b, g)));
}

// ----------------------------------------------------- gather_qmm (any) --
// Tiled CUDA-core kernel for arbitrary shapes: one CTA computes a 16 x 64
// output tile of batch entry p; K is walked in chunks of 32 with the weight
// chunk dequantised (fp32 fma) into shared memory.
constexpr int GQ_BM = 16, GQ_BN = 64, GQ_BK = 32;

template <int DT>
__global__ void __launch_bounds__(256) gather_qmm_kernel(const void* __restrict__ x, int64_t x_batch, int64_t M,
                                                        int64_t K, const uint32_t* __restrict__ w,
                                                        const void* __restrict__ s, const void* __restrict__ b,
                                                        int64_t w_batch, int64_t N, const uint32_t* __restrict__ lhs,
                                                        const uint32_t* __restrict__ rhs, int transpose, int gs,
                                                        int bits, void* __restrict__ out, int* __restrict__ status,
                                                        int64_t p_base) {
  __shared__ float xs[GQ_BM][GQ_BK + 1];
  __shared__ float ws[GQ_BN][GQ_BK + 1];
  const int64_t p = p_base + blockIdx.z;
  const int64_t li = lhs ? (int64_t)lhs[p] : p;
  const int64_t ri = rhs ? (int64_t)rhs[p] : p;
  if (li >= x_batch || ri >= w_batch) {
    if (threadIdx.x == 0) atomicCAS(status, 0, (int)kDevBadIndex);
    return;
  }
  const int64_t m0 = (int64_t)blockIdx.y * GQ_BM, n0 = (int64_t)blockIdx.x * GQ_BN;
  const int tid = threadIdx.x;
  const int tn = tid % GQ_BN, tm = tid / GQ_BN;  // 4 row-groups of 4 rows
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int64_t wpr = transpose ? K * bits / 32 : N * bits / 32;
  const int64_t gpr = transpose ? K / gs : N / gs;
  const int64_t wmat_rows = transpose ? N : K;
  for (int64_t k0 = 0; k0 < K; k0 += GQ_BK) {
    for (int i = tid; i < GQ_BM * GQ_BK; i += 256) {
      const int r = i / GQ_BK, c = i % GQ_BK;
      const int64_t m = m0 + r, k = k0 + c;
      xs[r][c] = (m < M && k < K) ? IO<DT>::load(x, (li * M + m) * K + k) : 0.0f;
    }
    for (int i = tid; i < GQ_BN * GQ_BK; i += 256) {
      const int r = i / GQ_BK, c = i % GQ_BK;
      const int64_t n = n0 + r, k = k0 + c;
      float v = 0.0f;
      if (n < N && k < K) {
        const int64_t wr = transpose ? n : k, wc = transpose ? k : n;
        const int64_t row = ri * wmat_rows + wr;
        const uint32_t q = get_code(w + row * wpr, wc, bits);
        const int64_t g = row * gpr + wc / gs;
        v = __fmaf_rn(IO<DT>::load(s, g), (float)q, IO<DT>::load(b, g));
      }
      ws[r][c] = v;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < GQ_BK; ++c) {
      const float wv = ws[tn][c];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = fmaf(xs[tm * 4 + j][c], wv, acc[j]);
    }
    __syncthreads();
  }
  const int64_t n = n0 + tn;
  if (n < N)
    for (int j = 0; j < 4; ++j) {
      const int64_t m = m0 + tm * 4 + j;
      if (m < M) IO<DT>::store(out, (p * M + m) * N + n, acc[j]);
    }
}

// ------------------------------------------------------------ gather_mm --
template <int DT>
__global__ void __launch_bounds__(256) gather_mm_kernel(const void* __restrict__ a, int64_t a_batch, int64_t M,
                                                       int64_t K, const void* __restrict__ bm, int64_t b_batch,
                                                       int64_t N, const uint32_t* __restrict__ lhs,
                                                       const uint32_t* __restrict__ rhs, void* __restrict__ out,
                                                       int* __restrict__ status, int64_t p_base) {
  __shared__ float as[GQ_BM][GQ_BK + 1];
  __shared__ float bs[GQ_BK][GQ_BN + 1];
  const int64_t p = p_base + blockIdx.z;
  const int64_t li = lhs ? (int64_t)lhs[p] : p;
  const int64_t ri = rhs ? (int64_t)rhs[p] : p;
  if (li >= a_batch || ri >= b_batch) {
    if (threadIdx.x == 0) atomicCAS(status, 0, (int)kDevBadIndex);
    return;
  }
  const int64_t m0 = (int64_t)blockIdx.y * GQ_BM, n0 = (int64_t)blockIdx.x * GQ_BN;
  const int tid = threadIdx.x, tn = tid % GQ_BN, tm = tid / GQ_BN;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t k0 = 0; k0 < K; k0 += GQ_BK) {
    for (int i = tid; i < GQ_BM * GQ_BK; i += 256) {
      const int r = i / GQ_BK, c = i % GQ_BK;
      const int64_t m = m0 + r, k = k0 + c;
      as[r][c] = (m < M && k < K) ? IO<DT>::load(a, (li * M + m) * K + k) : 0.0f;
    }
    for (int i = tid; i < GQ_BK * GQ_BN; i += 256) {
      const int r = i / GQ_BN, c = i % GQ_BN;
      const int64_t k = k0 + r, n = n0 + c;
      bs[r][c] = (k < K && n < N) ? IO<DT>::load(bm, (ri * K + k) * N + n) : 0.0f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < GQ_BK; ++c) {
      const float bv = bs[c][tn];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = fmaf(as[tm * 4 + j][c], bv, acc[j]);
    }
    __syncthreads();
  }
  const int64_t n = n0 + tn;
  if (n < N)
    for (int j = 0; j < 4; ++j) {
      const int64_t m = m0 + tm * 4 + j;
      if (m < M) IO<DT>::store(out, (p * M + m) * N + n, acc[j]);
    }
}

// -------------------------------------------------------------- synth ---
__device__ inline void philox10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
    const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

__global__ void synth_normal_kernel(uint64_t seed, uint64_t stream_id, int64_t n, float stddev,
                                    uint16_t* __restrict__ out) {
  const int64_t p = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (2 * p >= n) return;
  uint32_t c[4] = {(uint32_t)p, (uint32_t)((uint64_t)p >> 32), (uint32_t)stream_id, (uint32_t)(stream_id >> 32)};
  philox10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  const uint64_t a = ((((uint64_t)c[0]) << 32) | c[1]) >> 11;
  const uint64_t bb = ((((uint64_t)c[2]) << 32) | c[3]) >> 11;
  const double u1 = ((double)a + 1.0) * 0x1.0p-53;
  const double u2 = (double)bb * 0x1.0p-53;
  const double rad = sqrt(-2.0 * log(u1));
  const double th = 6.283185307179586476925286766559 * u2;
  out[2 * p] = f32_to_bf16_bits((float)(rad * cos(th) * (double)stddev));
  if (2 * p + 1 < n) out[2 * p + 1] = f32_to_bf16_bits((float)(rad * sin(th) * (double)stddev));
}

// Device address of the op family's status word (these ABIs take no
// workspace): one file-scope __device__ int per device, shared by every host
// thread and stream that calls the op family on that device. Ops running
// concurrently on several streams race on it: a bad index seen by one can be
// read (and cleared) by mlxr_cu_op_status called for another.
int* op_status_word();

}  // namespace mlxr

using namespace mlxr;

extern "C" {

const char* mlxr_cu_last_error(void) { return t_has_error ? t_last_error.c_str() : nullptr; }
void mlxr_cu_clear_error(void) {
  t_has_error = false;
  t_last_error.clear();
}
int mlxr_cu_abi_version(void) { return MLXR_CU_ABI_VERSION; }

static inline int default_gs(int gs) { return gs == 0 ? 64 : gs; }
static inline int default_bits(int bits) { return bits == 0 ? 4 : bits; }

static int check_q_args(int gs, int bits, const char* mode) {
  if (!mode_ok(mode)) return set_error(MLXR_CU_ERR_UNSUPPORTED, "mode '%s' is not supported (only \"affine\")", mode);
  if (!(bits == 2 || bits == 4 || bits == 8))
    return set_error(MLXR_CU_ERR_UNSUPPORTED, "bits=%d is not supported (2, 4, 8)", bits);
  if (!(gs == 32 || gs == 64 || gs == 128))
    return set_error(MLXR_CU_ERR_UNSUPPORTED, "group_size=%d is not supported (32, 64, 128)", gs);
  return MLXR_CU_OK;
}

int mlxr_cu_quantize(const void* w, mlxr_cu_dtype dtype, int64_t rows, int64_t cols, int group_size, int bits,
                     const char* mode, uint32_t* wq, void* scales, void* biases, void* stream) {
  group_size = default_gs(group_size);
  bits = default_bits(bits);
  if (int rc = check_q_args(group_size, bits, mode)) return rc;
  MLXR_CHECK_ARG(rows >= 0 && cols > 0, "quantize: bad shape [%lld, %lld]", (long long)rows, (long long)cols);
  MLXR_CHECK_ARG(cols % group_size == 0, "quantize: cols=%lld is not a multiple of group_size=%d", (long long)cols,
                 group_size);
  MLXR_CHECK_ARG(w && wq && scales && biases, "quantize: null pointer");
  if (rows == 0) return MLXR_CU_OK;
  const int64_t n = rows * (cols / group_size);
  cudaStream_t st = (cudaStream_t)stream;
  const int vec = (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  MLXR_DISPATCH_DTYPE(dtype, DT, quantize_kernel<DT><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
                                     w, rows, cols, group_size, bits, wq, scales, biases, vec));
  MLXR_LAUNCH_CHECK("quantize_kernel");
  return MLXR_CU_OK;
}

int mlxr_cu_dequantize(const uint32_t* wq, const void* scales, const void* biases, mlxr_cu_dtype sb_dtype,
                       int64_t rows, int64_t cols, int group_size, int bits, const char* mode, void* out,
                       mlxr_cu_dtype out_dtype, void* stream) {
  group_size = default_gs(group_size);
  bits = default_bits(bits);
  if (int rc = check_q_args(group_size, bits, mode)) return rc;
  MLXR_CHECK_ARG(rows >= 0 && cols > 0 && cols % group_size == 0, "dequantize: bad shape [%lld, %lld]",
                 (long long)rows, (long long)cols);
  MLXR_CHECK_ARG(wq && scales && biases && out, "dequantize: null pointer (affine needs biases)");
  if (rows == 0) return MLXR_CU_OK;
  const int64_t n = rows * cols;
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)((n + 255) / 256);
#define MLXR_DQ(SDT)                                                                                      \
  switch (out_dtype) {                                                                                    \
    case MLXR_CU_BFLOAT16: dequantize_kernel<SDT, MLXR_CU_BFLOAT16><<<grid, 256, 0, st>>>(wq, scales, biases, rows, cols, group_size, bits, out); break; \
    case MLXR_CU_FLOAT16: dequantize_kernel<SDT, MLXR_CU_FLOAT16><<<grid, 256, 0, st>>>(wq, scales, biases, rows, cols, group_size, bits, out); break;   \
    case MLXR_CU_FLOAT32: dequantize_kernel<SDT, MLXR_CU_FLOAT32><<<grid, 256, 0, st>>>(wq, scales, biases, rows, cols, group_size, bits, out); break;   \
    default: return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "unknown out dtype");                       \
  }
  switch (sb_dtype) {
    case MLXR_CU_BFLOAT16: MLXR_DQ(MLXR_CU_BFLOAT16); break;
    case MLXR_CU_FLOAT16: MLXR_DQ(MLXR_CU_FLOAT16); break;
    case MLXR_CU_FLOAT32: MLXR_DQ(MLXR_CU_FLOAT32); break;
    default: return set_error(MLXR_CU_ERR_INVALID_ARGUMENT, "unknown scales dtype");
  }
#undef MLXR_DQ
  MLXR_LAUNCH_CHECK("dequantize_kernel");
  return MLXR_CU_OK;
}

int mlxr_cu_gather_qmm(const void* x, mlxr_cu_dtype x_dtype, int64_t x_batch, int64_t M, int64_t K,
                       const uint32_t* w, const void* scales, const void* biases, int64_t w_batch, int64_t N,
                       const uint32_t* lhs_indices, const uint32_t* rhs_indices, int64_t num_indices, int transpose,
                       int group_size, int bits, const char* mode, int sorted_indices, void* out, void* stream) {
  (void)sorted_indices;  // a locality hint in the reference; results do not depend on it
  group_size = default_gs(group_size);
  bits = default_bits(bits);
  if (int rc = check_q_args(group_size, bits, mode)) return rc;
  MLXR_CHECK_ARG(x && w && scales && out, "gather_qmm: null pointer");
  MLXR_CHECK_ARG(biases, "gather_qmm: mode affine requires biases");
  MLXR_CHECK_ARG(M >= 0 && K > 0 && N > 0 && x_batch > 0 && w_batch > 0 && num_indices >= 0,
                 "gather_qmm: bad shape");
  MLXR_CHECK_ARG((transpose ? K : N) % group_size == 0,
                 "gather_qmm: the quantised axis (%lld) is not a multiple of group_size=%d",
                 (long long)(transpose ? K : N), group_size);
  MLXR_CHECK_ARG(lhs_indices || num_indices <= x_batch, "gather_qmm: num_indices exceeds x batch without lhs_indices");
  MLXR_CHECK_ARG(rhs_indices || num_indices <= w_batch, "gather_qmm: num_indices exceeds w batch without rhs_indices");
  if (num_indices == 0 || M == 0) return MLXR_CU_OK;
  int* status = op_status_word();
  if (!status) return MLXR_CU_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  MLXR_CHECK_ARG((M + GQ_BM - 1) / GQ_BM <= 65535, "gather_qmm: M=%lld too large", (long long)M);
  for (int64_t p0 = 0; p0 < num_indices; p0 += 65535) {
    const int64_t np = num_indices - p0 < 65535 ? num_indices - p0 : 65535;
    dim3 grid((unsigned)((N + GQ_BN - 1) / GQ_BN), (unsigned)((M + GQ_BM - 1) / GQ_BM), (unsigned)np);
    MLXR_DISPATCH_DTYPE(x_dtype, DT, gather_qmm_kernel<DT><<<grid, 256, 0, st>>>(
                                         x, x_batch, M, K, w, scales, biases, w_batch, N, lhs_indices, rhs_indices,
                                         transpose, group_size, bits, out, status, p0));
  }
  MLXR_LAUNCH_CHECK("gather_qmm_kernel");
  return MLXR_CU_OK;
}

int mlxr_cu_quantized_matmul(const void* x, mlxr_cu_dtype x_dtype, int64_t M, int64_t K, const uint32_t* w,
                             const void* scales, const void* biases, int64_t N, int transpose, int group_size,
                             int bits, const char* mode, void* out, void* stream) {
  return mlxr_cu_gather_qmm(x, x_dtype, 1, M, K, w, scales, biases, 1, N, nullptr, nullptr, 1, transpose, group_size,
                            bits, mode, 0, out, stream);
}

int mlxr_cu_gather_mm(const void* a, const void* b, mlxr_cu_dtype dtype, int64_t a_batch, int64_t M, int64_t K,
                      int64_t b_batch, int64_t N, const uint32_t* lhs_indices, const uint32_t* rhs_indices,
                      int64_t num_indices, int sorted_indices, void* out, void* stream) {
  (void)sorted_indices;
  MLXR_CHECK_ARG(a && b && out, "gather_mm: null pointer");
  MLXR_CHECK_ARG(M >= 0 && K > 0 && N > 0 && a_batch > 0 && b_batch > 0 && num_indices >= 0, "gather_mm: bad shape");
  MLXR_CHECK_ARG(lhs_indices || num_indices <= a_batch, "gather_mm: num_indices exceeds a batch without lhs_indices");
  MLXR_CHECK_ARG(rhs_indices || num_indices <= b_batch, "gather_mm: num_indices exceeds b batch without rhs_indices");
  if (num_indices == 0 || M == 0) return MLXR_CU_OK;
  int* status = op_status_word();
  if (!status) return MLXR_CU_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  MLXR_CHECK_ARG((M + GQ_BM - 1) / GQ_BM <= 65535, "gather_mm: M=%lld too large", (long long)M);
  for (int64_t p0 = 0; p0 < num_indices; p0 += 65535) {
    const int64_t np = num_indices - p0 < 65535 ? num_indices - p0 : 65535;
    dim3 grid((unsigned)((N + GQ_BN - 1) / GQ_BN), (unsigned)((M + GQ_BM - 1) / GQ_BM), (unsigned)np);
    MLXR_DISPATCH_DTYPE(dtype, DT, gather_mm_kernel<DT><<<grid, 256, 0, st>>>(a, a_batch, M, K, b, b_batch, N,
                                                                             lhs_indices, rhs_indices, out, status, p0));
  }
  MLXR_LAUNCH_CHECK("gather_mm_kernel");
  return MLXR_CU_OK;
}

int mlxr_cu_synth_normal_bf16(uint64_t seed, uint64_t stream_id, int64_t n, float stddev, void* out, void* stream) {
  MLXR_CHECK_ARG(out && n >= 0, "synth_normal_bf16: bad arguments");
  if (n == 0) return MLXR_CU_OK;
  const int64_t pairs = (n + 1) / 2;
  synth_normal_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, (cudaStream_t)stream>>>(seed, stream_id, n, stddev,
                                                                                          (uint16_t*)out);
  MLXR_LAUNCH_CHECK("synth_normal_kernel");
  return MLXR_CU_OK;
}

}  // extern "C"
