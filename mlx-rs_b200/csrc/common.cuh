// Shared helpers for the sm_100a MoE kernels: bf16 bit helpers, status
// reporting, and thin inline-PTX wrappers for mbarriers, TMA and tcgen05.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>

#include "../../include/mlxr_moe.h"

namespace mlxr {

// ------------------------------------------------------------ errors ----
// Thread-local last-error message plus a status return (the reference's
// Guarded::try_from_op contract, crates/mlxr/src/utils/guard.rs:31-51:
// status 0 = success, otherwise the message is fetched from a thread-local).
int set_error(int status, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device):
// `done` holds one bit per device ordinal (< 64) already configured.
template <typename F>
inline int ensure_smem_attr(F* func, int bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, "cudaGetDevice");
  const uint64_t bit = (dev >= 0 && dev < 64) ? (uint64_t(1) << dev) : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return MLXR_CU_OK;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  if (bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return MLXR_CU_OK;
}

// Programmatic dependent launch. Every kernel of the block is launched with
// launch_pdl (the launch may begin while the previous kernel in the stream
// is still running) and starts with pdl_wait() before it touches global
// memory: griddepcontrol.wait returns once the previous grid has completed
// and its writes are visible, so the overlap only hides launch latency and
// prologues (barrier set-up, tensor-memory allocation). pdl_launch_dependents()
// lets the next kernel begin launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

#define MLXR_CHECK_ARG(cond, ...)                                                  \
  do {                                                                             \
    if (!(cond)) return ::mlxr::set_error(MLXR_CU_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)
#define MLXR_CUDA_TRY(expr)                                      \
  do {                                                           \
    cudaError_t _e = (expr);                                     \
    if (_e != cudaSuccess) return ::mlxr::check_cuda(_e, #expr); \
  } while (0)
#define MLXR_LAUNCH_CHECK(name)                                   \
  do {                                                            \
    cudaError_t _e = cudaGetLastError();                          \
    if (_e != cudaSuccess) return ::mlxr::check_cuda(_e, name);   \
  } while (0)

// Device-side status codes written into the caller's status word.
enum DeviceStatus : int {
  kDevOk = 0,
  kDevTimeout = 1,      // a bounded wait gave up
  kDevBadIndex = 2,     // an index outside [0, E) or a row outside its range
  kDevTmemAlloc = 3,    // tensor-memory allocation failed
  kDevPeerFailed = 4,   // another rank published a poisoned flag: its side of the step failed
};

// ------------------------------------------------------------- bf16 -----
__host__ __device__ inline float bf16_bits_to_f32(uint16_t h) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(((uint32_t)h) << 16);
#else
  uint32_t u = ((uint32_t)h) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

__device__ inline uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ inline uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// --------------------------------------------------------- timeouts -----
// Every spin-wait in these kernels is bounded by wall-clock time read from
// %globaltimer (ns). On expiry the waiting thread records kDevTimeout in the
// status word and the kernel unwinds without touching its operands again.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ inline unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ inline uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// --------------------------------------------------------- mbarrier -----
__device__ inline void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ inline void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ inline void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ inline void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ inline bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or `ns` nanoseconds pass, instead of spinning. A spinning waiter
// takes issue slots from the warps that share its SM sub-partition: in the
// grouped GEMM a spinning producer warp left the dequant warps beside it
// thousands of cycles behind the others.
__device__ inline bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and raises the CTA's
// abort flag and the global status) when the limit expires or when another
// thread of the CTA has already aborted.
__device__ inline bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (*abort_flag) return false;
    if ((it & 15u) == 0 && global_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      atomicCAS(status, 0, (int)kDevTimeout);
      return false;
    }
  }
}

// After a producer stops (normally or on abort), wait (bounded) until every
// TMA load it issued into a ring of STAGES slots has landed, so no copy is
// still writing shared memory when the CTA exits. `issued` = loads issued.
template <int STAGES>
__device__ inline void drain_ring(uint64_t* full, uint32_t issued, volatile int* abort_flag, int* status) {
  for (uint32_t s = 0; s < (uint32_t)STAGES && s < issued; ++s) {
    const uint32_t last = issued - 1 - ((issued - 1 - s) % STAGES);
    int dummy_abort = 0;
    (void)abort_flag;
    mbar_wait(&full[s], (last / STAGES) & 1, &dummy_abort, status);
  }
}

// -------------------------------------------------------------- TMA -----
__device__ inline void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}
__device__ inline void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tensor-core operand reads through smem descriptors).
__device__ inline void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------- tcgen05 ----
__device__ inline void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ inline void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ inline void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ inline void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ inline void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// One 64-wide k-step as four K=16 MMAs from a single asm block: A from TMEM
// columns a, a+8, a+16, a+24; B from the 128-byte-swizzled K-major tile whose
// descriptor start address advances by 32 B (2 in units of 16 B) per step.
// The first MMA overwrites D when accumulate == 0; the rest accumulate.
__device__ inline void umma_bf16_ts_k64(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t.reg .b32 a1, a2, a3;\n\t.reg .b64 b1, b2, b3;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "setp.eq.b32 q, %4, %4;\n\t"
      "add.u32 a1, %1, 8;\n\tadd.u32 a2, %1, 16;\n\tadd.u32 a3, %1, 24;\n\t"
      "add.u64 b1, %2, 2;\n\tadd.u64 b2, %2, 4;\n\tadd.u64 b3, %2, 6;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %3, q;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ inline void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// TMEM -> registers. Each helper issues the tcgen05.ld(s) and the
// tcgen05.wait::ld in ONE asm statement: the destination registers are only
// defined once the wait has retired, so the compiler cannot schedule a use of
// them ahead of the wait. Warp w reads TMEM lanes 32*(w%4) .. +31; columns
// start at the column field of taddr.
__device__ inline void tmem_ld_x16_wait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ inline void tmem_ld2_x16_wait(uint32_t ta, uint32_t tb, uint32_t (&a)[32], uint32_t (&b)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]), "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15]),
        "=r"(b[0]), "=r"(b[1]), "=r"(b[2]), "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]), "=r"(b[8]), "=r"(b[9]), "=r"(b[10]), "=r"(b[11]), "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15])
      : "r"(ta), "r"(tb)
      : "memory");
}

// Two or four 8-column loads of this warp's lanes in one wait: r[8*i + j] =
// column j of region i.
__device__ inline void tmem_ld2_x8_wait(uint32_t t0, uint32_t t1, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%16];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8, %9, %10, %11, %12, %13, %14, %15}, [%17];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(t0), "r"(t1)
      : "memory");
}
__device__ inline void tmem_ld4_x8_wait(uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8, %9, %10, %11, %12, %13, %14, %15}, [%33];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16, %17, %18, %19, %20, %21, %22, %23}, [%34];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%24, %25, %26, %27, %28, %29, %30, %31}, [%35];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(t0), "r"(t1), "r"(t2), "r"(t3)
      : "memory");
}

// Registers -> TMEM: each thread writes N consecutive 32-bit columns of its
// own lane (lane = 32*(warp%4) + laneid). Completion is awaited with
// tmem_st_wait() before the data is handed to the tensor core.
__device__ inline void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
               : "memory");
}
__device__ inline void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand stored in the
// 128-byte swizzle canonical layout: rows of 128 B (64 bf16), 8-row atoms of
// 1024 B (stride-dimension byte offset), start address advanced by 32 B per
// K=16 step inside the atom. Bits: [0,14) addr>>4, [16,30) LBO>>4 (unused for
// swizzled K-major, set to 1), [32,46) SBO>>4, [46,48) version 1,
// [61,64) layout 2 = SWIZZLE_128B.
__device__ inline uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A bf16 (7-9 = 1),
// B bf16 (10-12 = 1), both K-major, N>>3 at bits 17-22, M>>4 at bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// g * sigmoid(g) with the fast exponential and division (a few ulp of fp32;
// the result is rounded to bf16 right after).
__device__ inline float silu_f32(float g) { return __fdividef(g, 1.0f + __expf(-g)); }
// gelu_approximate (crates/mlxr/src/layers/activation.rs:170-174):
// 0.5 g (1 + tanh(y)), y = sqrt(2/pi) (g + 0.044715 g^3), evaluated as the
// equal g / (1 + exp(-2y)).
__device__ inline float gelu_tanh_f32(float g) {
  const float z = 1.5957691216057308f * (g + 0.044715f * g * g * g);
  return __fdividef(g, 1.0f + __expf(-z));
}

}  // namespace mlxr
