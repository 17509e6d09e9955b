// Device primitives for the sm_100a sampling kernels: order-preserving keys,
// cluster / distributed-shared-memory helpers, bulk async copies with bounded
// mbarrier waits, block-wide scans and a shared-memory bitonic sort.
#pragma once

#include <cooperative_groups.h>
#include <cstdint>
#include <cuda_runtime.h>

namespace vb {

namespace cg = cooperative_groups;

constexpr int kThreads = 512;               // threads per CTA in every kernel
constexpr int kWarps = kThreads / 32;
constexpr int kMaxCluster = 8;              // portable cluster size
constexpr uint64_t kNoKey = ~0ull;          // sorts after every real key
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // bounded waits give up after 1 s

// ---------------------------------------------------------------- keys ----
// Sampler::pick orders candidates by value descending, index ascending
// (src/sampler.cpp:71) and compares -0.0 equal to +0.0.  A NaN logit makes the
// reference's std::sort undefined; here it is ordered as -inf.
__device__ __forceinline__ float canon(float v) {
  if (v != v) return -__int_as_float(0x7f800000);
  return v == 0.0f ? 0.0f : v;
}
// Monotone map float -> u32 (larger float -> larger code).
__device__ __forceinline__ uint32_t ord32(float cv) {
  const uint32_t b = __float_as_uint(cv);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unord32(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}
// 64-bit key whose ascending order is the reference's candidate order:
// high word = inverted value code, low word = global token id.
__device__ __forceinline__ uint64_t dkey(float v, uint32_t gid) {
  return (static_cast<uint64_t>(~ord32(canon(v))) << 32) | gid;
}
__device__ __forceinline__ float dval(uint64_t d) { return unord32(~static_cast<uint32_t>(d >> 32)); }
__device__ __forceinline__ uint32_t did(uint64_t d) { return static_cast<uint32_t>(d); }

// Repetition penalty, fp32 and correctly rounded (src/sampler.cpp:63).
__device__ __forceinline__ float penalize(float v, float rep) {
  return v > 0.0f ? __fdiv_rn(v, rep) : __fmul_rn(v, rep);
}

// --------------------------------------------------- cluster barriers -----
// The non-.aligned forms: a warp may reach them diverged (e.g. after a
// single-thread tail).  arrive.release / wait.acquire order the shared and
// distributed-shared memory accesses around the barrier.
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_all() {
  cluster_arrive();
  cluster_wait();
}

// ------------------------------------- programmatic dependent launch ------
// Without the launch attribute both are no-ops.  grid_wait blocks until the
// grids this one depends on have completed and their writes are visible (they
// contain no waits of their own); grid_release lets the dependent grid be
// scheduled before this one finishes.
__device__ __forceinline__ void grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------ timers ------
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// --------------------------------------------------- mbarrier + bulk copy -
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Waits for the phase with a time limit; returns false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = gtimer();
  while (!mbar_try_wait(bar, phase)) {
    if (gtimer() - t0 > kWaitLimitNs) return false;
  }
  return true;
}
// Global -> this CTA's shared memory, completion counted on `bar` in bytes.
// Both addresses 16-byte aligned, bytes a multiple of 16.  Never multicast.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 16-byte asynchronous copy global -> shared (both 16-byte aligned), L1
// bypassed; completion by cp_async_wait_all in the issuing thread.
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src_gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src_gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Streaming 16-byte load: read-only path, no L1 allocation, 256-byte L2 prefetch.
__device__ __forceinline__ float4 ld_stream(const float4* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_stream1(const float* p) {
  float v;
  asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

// ------------------------------------------------------------- scans ------
template <class T>
__device__ __forceinline__ T warp_incl_scan(T x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  return x;
}
template <class T>
__device__ __forceinline__ T warp_min(T x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    T y = __shfl_xor_sync(0xffffffffu, x, o);
    x = y < x ? y : x;
  }
  return x;
}
template <class T>
__device__ __forceinline__ T warp_max(T x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    T y = __shfl_xor_sync(0xffffffffu, x, o);
    x = y > x ? y : x;
  }
  return x;
}
template <class T>
__device__ __forceinline__ T warp_sum(T x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Block-wide exclusive scan of one value per thread.  `ws` holds kWarps
// entries of shared scratch.  Returns the exclusive prefix; *total gets the
// block total.  Contains two __syncthreads.
// NT = threads of the block (a multiple of 32, at most 1024).
template <class T, int NT = kThreads>
__device__ __forceinline__ T block_excl_scan(T x, T* ws, T* total) {
  constexpr int W = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T incl = warp_incl_scan(x);
  if (lane == 31) ws[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    T w = lane < W ? ws[lane] : T(0);
    w = warp_incl_scan(w);
    if (lane < W) ws[lane] = w;
  }
  __syncthreads();
  *total = ws[W - 1];
  return incl - x + (warp ? ws[warp - 1] : T(0));
}

template <class T, int NT = kThreads>
__device__ __forceinline__ T block_min(T x, T* ws) {
  constexpr int W = NT / 32;
  x = warp_min(x);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) ws[warp] = x;
  __syncthreads();
  T r = ws[0];
  for (int i = 1; i < W; ++i) r = ws[i] < r ? ws[i] : r;
  __syncthreads();
  return r;
}
template <class T, int NT = kThreads>
__device__ __forceinline__ T block_sum(T x, T* ws) {
  constexpr int W = NT / 32;
  x = warp_sum(x);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) ws[warp] = x;
  __syncthreads();
  T r = ws[0];
  for (int i = 1; i < W; ++i) r += ws[i];
  __syncthreads();
  return r;
}

// Ascending bitonic sort of n (a power of two) 64-bit keys in shared memory.
__device__ inline void bitonic_sort_u64(uint64_t* s, int n) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t a = s[i], b = s[ixj];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            s[i] = b;
            s[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

}  // namespace vb
