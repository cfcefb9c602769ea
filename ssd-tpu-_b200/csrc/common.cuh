// Shared device helpers for the verify-step kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <utility>

#include "../../include/ssd_verify.h"

namespace ssd {

using bf16 = __nv_bfloat16;

constexpr int kWarp = 32;

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(bf16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ bf16 from_f<bf16>(float x) { return __float2bfloat16_rn(x); }

// Round an fp32 value to bf16 precision, staying in fp32.
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <typename T> __device__ __forceinline__ float store_round(float x) { return x; }
template <> __device__ __forceinline__ float store_round<bf16>(float x) { return round_bf16(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

// Order-preserving map of fp32 onto uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}
// (value, index) packed so that max() picks the larger value, then the SMALLER index
// (first-occurrence argmax, as numpy/jnp/torch argmax).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  return ((unsigned long long)float_key(v) << 32) | (unsigned long long)(0xffffffffu - idx);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long k) {
  return 0xffffffffu - (uint32_t)(k & 0xffffffffu);
}
__device__ __forceinline__ float argmax_key_value(unsigned long long k) {
  return key_float((uint32_t)(k >> 32));
}

// Block-wide reductions; every thread receives the result.  `scratch` must hold
// 32 entries and may be reused after the call returns.
template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T* scratch, Op op) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  T r = scratch[0];
  for (int i = 1; i < nw; ++i) r = op(r, scratch[i]);
  return r;
}

struct OpSum { template <typename T> __device__ T operator()(T a, T b) const { return a + b; } };
struct OpMax {
  __device__ float operator()(float a, float b) const { return fmaxf(a, b); }
  __device__ unsigned long long operator()(unsigned long long a, unsigned long long b) const { return a > b ? a : b; }
};

// Acquire-release fetch-add at GPU scope (the ticket of a split reduction).
__device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int* a, unsigned int v) {
  unsigned int old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(a), "r"(v) : "memory");
  return old;
}

// "Last block done" ticket: returns true in exactly one block of the group once
// all `total` blocks of the group have called it.  The counter is reset to 0 by
// that block, so the workspace stays reusable without a memset.  Each block must
// have written its partial results before calling.  Ordering without per-thread
// fences: the first barrier puts the block's partial stores before thread 0's
// acq_rel ticket (release); in the last block the ticket also acquires every
// other block's partials and the second barrier passes that on to all of its
// threads, which must read the partials with L2 loads (__ldcg).
__device__ __forceinline__ bool last_block_of(unsigned int* counter, unsigned int total, bool* smem_flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atom_add_acq_rel_gpu(counter, 1u);
    const bool last = (prev == total - 1);
    if (last) *reinterpret_cast<volatile unsigned int*>(counter) = 0u;
    *smem_flag = last;
  }
  __syncthreads();
  return *smem_flag;
}

// Every workspace starts with a fixed-size region of ticket counters.  It is the
// only part of a workspace that must hold zeros between calls, and because its
// size does not depend on the call's shape, calls of different shapes can share
// one workspace: their partial-result regions never overlap any counter.
constexpr int kCounterCap = 16384;
constexpr size_t kCounterBytes = sizeof(unsigned int) * kCounterCap;

// 16-byte aligned vector of 8 bf16 values.
struct alignas(16) bf16x8 { __nv_bfloat162 h[4]; };

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// Loads of data that an earlier kernel of the stream wrote.  Every kernel is
// launched with programmatic dependent launch, so a grid is already resident
// while its predecessor still writes; the non-coherent read-only path
// (ld.global.nc, which the compiler may also pick for const __restrict__
// pointers) can then serve stale lines even after griddepcontrol.wait.
// Activations, logits, token ids, positions and page tables are therefore read
// through L2 (ld.global.cg); only weights and constant tables that no kernel
// writes use ldg_nc_v4.  Kernel parameters carry no __restrict__ for the same
// reason.
__device__ __forceinline__ uint4 ld_act_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
template <typename T>
__device__ __forceinline__ T ld_act(const T* p) {
  return __ldcg(p);
}

// Weights and constant tables only (see ld_act_v4).
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Programmatic dependent launch.  Every kernel of the verify path is launched
// with launch_pdl, so it may start while its predecessor in the stream is still
// draining.  pdl_wait() blocks until the predecessor grid has completed and its
// writes are visible: call it before reading anything an earlier kernel wrote
// (a no-op when the launch had no programmatic dependency).  pdl_trigger() lets
// the next kernel launch; kernels call it once their CTA's main work is issued.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
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
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// launch_pdl with a 1-D thread-block cluster of `cluster_x` CTAs.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                      unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace ssd

// Launch through launch_pdl and turn a launch failure into SSD_ERR_LAUNCH.
#define SSD_PDL(kern, grid, block, smem, st, ...)                                        \
  do {                                                                                   \
    if (::ssd::launch_pdl(kern, dim3(grid), dim3(block), (size_t)(smem), (cudaStream_t)(st), \
                          __VA_ARGS__) != cudaSuccess) {                                 \
      (void)cudaGetLastError();                                                          \
      return SSD_ERR_LAUNCH;                                                             \
    }                                                                                    \
  } while (0)

#define SSD_CHECK_LAUNCH()                               \
  do {                                                   \
    cudaError_t e__ = cudaGetLastError();                \
    if (e__ != cudaSuccess) return SSD_ERR_LAUNCH;       \
  } while (0)
