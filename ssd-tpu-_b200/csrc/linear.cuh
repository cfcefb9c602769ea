// Internal interface of the projection kernels (not part of the C ABI).
#pragma once
#include "common.cuh"

namespace ssd {

inline size_t align_up256(size_t x) { return (x + 255) & ~size_t(255); }

struct LinearPlan {
  int splits;     // split-K factor (from N, K only)
  int kc;         // K elements per split
  int tiles_max;  // upper bound on N tiles (ticket counters)
};

__device__ __forceinline__ float gelu_tanh_f(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
  const float c = 0.7978845608028654f;
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float in = __fmul_rn(c, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(in)));
}

template <typename T>
__device__ __forceinline__ void epilogue_store(int epi, void* y, int N, int m, int n, float acc, float acc_pair) {
  switch (epi) {
    case SSD_EPI_STORE:
      reinterpret_cast<T*>(y)[(int64_t)m * N + n] = from_f<T>(acc);
      break;
    case SSD_EPI_STORE_F32:
      reinterpret_cast<float*>(y)[(int64_t)m * N + n] = acc;
      break;
    case SSD_EPI_RESIDUAL: {
      T* p = reinterpret_cast<T*>(y) + (int64_t)m * N + n;
      *p = from_f<T>(__fadd_rn(to_f(*p), store_round<T>(acc)));
      break;
    }
    case SSD_EPI_GEGLU: {  // n even: acc = gate, acc_pair = up
      const float g = store_round<T>(acc), u = store_round<T>(acc_pair);
      const float a = store_round<T>(gelu_tanh_f(g));
      reinterpret_cast<T*>(y)[(int64_t)m * (N / 2) + n / 2] = from_f<T>(__fmul_rn(a, u));
      break;
    }
  }
}



LinearPlan plan_linear_cc(int N, int K, int elem_bytes);
size_t linear_cc_workspace(int M, int N, int K, int elem_bytes);
template <typename T>
int linear_cc(cudaStream_t st, const void* x, const void* w, void* y, int epi, int M, int N, int K, void* ws,
              size_t ws_bytes, int rowscale = 0, float eps = 0.f);

// tcgen05 weight-streaming path (bf16)
size_t linear_tc_workspace(int M, int N, int K);
int linear_tc(cudaStream_t st, const void* x, const void* w, void* y, int epi, int M, int N, int K, void* ws,
              size_t ws_bytes, int rowscale = 0, float eps = 0.f);
bool linear_tc_supported(int M, int N, int K);

}  // namespace ssd
