// Shared device helpers for the sm_100a kernels: mbarriers, bulk (TMA-engine)
// copies, bounded waits, numeric conversions and the device status word.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <atomic>

#include "../../include/akt.h"

namespace akt {

// ---------------------------------------------------------------------------
// device status word: first error recorded by any kernel of this library.
// Kernels never trap; they record a code here and skip the offending access.
// ---------------------------------------------------------------------------
// Files built as whole-program device code (without -rdc, so that ptxas
// applies setmaxnreg register budgets) keep their own word, which the host
// status functions read and clear together with the shared one.
#ifdef AKT_WHOLE_PROGRAM
namespace {
__device__ unsigned int g_device_status_local = 0;
}
#define AKT_STATUS_WORD g_device_status_local
#else
extern __device__ unsigned int g_device_status;
#define AKT_STATUS_WORD g_device_status
#endif

enum DeviceStatus : unsigned int {
  kStatusOk = 0,
  kStatusWaitTimeout = 1,     // an mbarrier wait ran past its limit
  kStatusBadPage = 2,         // page id outside the pool
  kStatusBadToken = 3,        // token index outside the sequence
  kStatusBadIndptr = 4,       // indptr not monotone / past the index array
  kStatusListOverflow = 5,    // more kept tokens than the index list holds
};

__device__ __forceinline__ void record_status(unsigned int code) {
  atomicCAS(&AKT_STATUS_WORD, 0u, code);
}

// ---------------------------------------------------------------------------
// shared-memory addresses and mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Raise kernel Kern's dynamic shared-memory limit on the current device to at
// least `bytes`.  The driver call is made only when the value already set
// for this kernel and device is smaller (one static per kernel instantiation).
template <auto Kern>
cudaError_t ensure_smem_limit(size_t bytes) {
  static std::atomic<int> set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (set[dev].load(std::memory_order_relaxed) >= (int)bytes) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) {
    int cur = set[dev].load(std::memory_order_relaxed);
    while (cur < (int)bytes && !set[dev].compare_exchange_weak(cur, (int)bytes, std::memory_order_relaxed)) {
    }
  }
  return e;
}

// Programmatic dependent launch.  A kernel launched by launch_dependent() may
// start while the previous kernel in its stream still runs; before reading
// anything that kernel writes it calls grid_dep_wait(), which returns once the
// previous grid has completed with its writes visible.  The first kernel of a
// call is launched normally: it reads the caller's inputs.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args... args) {
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
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity to complete.  The wait is bounded:
// after ~kWaitLimitNs it records kStatusWaitTimeout and returns false; callers
// then stop issuing work and fall through to the kernel's exit path.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++it & 255u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) {
      record_status(kStatusWaitTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// bulk global->shared copy through the TMA engine (1-D, no tensor map).
// Both addresses 16-byte aligned, size a multiple of 16.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// named barrier over a subset of warps
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// numerics
// ---------------------------------------------------------------------------
template <typename T>
struct Elem;

template <>
struct Elem<__half> {
  using T2 = __half2;
  static __device__ __forceinline__ float2 to_float2(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
  }
  static __device__ __forceinline__ float to_float(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_float(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

template <>
struct Elem<__nv_bfloat16> {
  using T2 = __nv_bfloat162;
  static __device__ __forceinline__ float2 to_float2(uint32_t v) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
  }
  static __device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_float(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// packed fp32x2 fused multiply-add / multiply (sm_100 compiler builtins: the
// operands stay in register pairs, no repacking around the instruction)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) { return __fmul2_rn(a, b); }

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__host__ __device__ constexpr int cdiv(int a, int b) { return (a + b - 1) / b; }

// n / d for 32-bit unsigned n by multiply-high and shift (the round-up
// multiplier method of Granlund and Montgomery, "Division by invariant
// integers using multiplication", PLDI 1994): l = ceil(log2 d),
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (umulhi(n, m) + n) >> l with a
// 33-bit sum.  Built on the host for a divisor 1 <= d < 2^31.
struct FastDiv {
  uint32_t d, m, l;
};

inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while (l < 32 && (1ull << l) < d) ++l;
  const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
  return FastDiv{d, (uint32_t)m, l};
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
  return (uint32_t)(((uint64_t)__umulhi(n, f.m) + n) >> f.l);
}

}  // namespace akt
