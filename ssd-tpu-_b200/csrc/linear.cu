// K3: skinny projections y = epilogue(x[M,K] w[N,K]^T) for the verify step.
//
// The verify forward multiplies a handful of token rows (M = B*(k+1), 5 for
// the 7B sd step) by every weight matrix of the model, so each projection is a
// pure weight stream: bytes = N*K*sizeof(w), flops = 2*M*N*K (about 5 flop per
// weight byte at M = 5, far under the tensor ridge).  This file holds the
// CUDA-core streamer used for fp32 weights (the toy pair) and as the
// split-K/epilogue machinery shared with the tcgen05 path:
//   * warp = ROWS output features; lanes stride K in 16-byte weight vectors
//     (ld.global.nc, no L1 allocation), x staged once per CTA in shared memory;
//   * split-K over `splits` CTAs chosen from (N, K) only, never from M, and a
//     fixed reduction order (lane-strided partials -> xor-shuffle tree -> split
//     order), so a row's result does not depend on how many rows ride along;
//   * the last CTA of an N-tile (atomic ticket, self-resetting) folds the
//     splits and applies the fused epilogue (store / fp32 store / residual add
//     / GeGLU on interleaved gate-up rows).
#include "common.cuh"
#include "linear.cuh"

namespace ssd {

namespace {

constexpr int kLinThreads = 256;
constexpr int kWarps = kLinThreads / 32;

template <typename T> struct WVec;
template <> struct WVec<bf16> {
  static constexpr int N = 8;
  __device__ static void load(const bf16* p, float* f) { unpack8(ldg_nc_v4(p), f); }
  __device__ static void load_smem(const bf16* p, float* f) { unpack8(*reinterpret_cast<const uint4*>(p), f); }
};
template <> struct WVec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float* f) {
    uint4 u = ldg_nc_v4(p);
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y); f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  }
  __device__ static void load_smem(const float* p, float* f) {
    float4 u = *reinterpret_cast<const float4*>(p);
    f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
  }
};

template <typename T, int MMAX, int ROWS>
__global__ void __launch_bounds__(kLinThreads)
linear_cc_kernel(const T* x, const T* w, void* y, int epi, int M, int N,
                 int K, int splits, int kc, float* ws, unsigned int* counters,
                 int rowscale, float eps) {
  constexpr int VN = WVec<T>::N;
  constexpr int STEP = 32 * VN;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* xs = reinterpret_cast<T*>(smem_raw);  // [M][kc]
  __shared__ bool is_last;
  __shared__ float inv_s[16];

  pdl_wait();
  const int tile = blockIdx.x, split = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int k0 = split * kc;
  const int klen = min(kc, K - k0);
  if (rowscale) {
    // RMS of each full token row (the (1 + w) factor is folded into the weights);
    // warp w takes rows w, w + 8; lane-strided sums and an xor tree: fixed order.
    for (int m = warp; m < M; m += kWarps) {
      float a = 0.f;
      for (int k = lane; k < K; k += 32) {
        const float v = to_f(x[(int64_t)m * K + k]);
        a = fmaf(v, v, a);
      }
      a = warp_sum(a);
      if (lane == 0) inv_s[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(a, (float)K), eps)));
    }
  }
  // stage x[:, k0:k0+klen]
  {
    const int pieces = klen / VN;
    for (int i = threadIdx.x; i < M * pieces; i += kLinThreads) {
      const int m = i / pieces, c = i % pieces;
      *reinterpret_cast<uint4*>(xs + (int64_t)m * kc + c * VN) =
          *reinterpret_cast<const uint4*>(x + (int64_t)m * K + k0 + c * VN);
    }
  }
  __syncthreads();

  const int n0 = (tile * kWarps + warp) * ROWS;
  float acc[ROWS][MMAX];
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int m = 0; m < MMAX; ++m) acc[r][m] = 0.f;

  for (int kk = lane * VN; kk < klen; kk += STEP) {
    float wv[ROWS][VN];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int n = n0 + r;
      if (n < N) WVec<T>::load(w + (int64_t)n * K + k0 + kk, wv[r]);
      else {
#pragma unroll
        for (int e = 0; e < VN; ++e) wv[r][e] = 0.f;
      }
    }
#pragma unroll
    for (int m = 0; m < MMAX; ++m) {
      if (m < M) {
        float xv[VN];
        WVec<T>::load_smem(xs + (int64_t)m * kc + kk, xv);
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
#pragma unroll
          for (int e = 0; e < VN; ++e) acc[r][m] = fmaf(wv[r][e], xv[e], acc[r][m]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS; ++r)
#pragma unroll
    for (int m = 0; m < MMAX; ++m) acc[r][m] = warp_sum(acc[r][m]);
  pdl_trigger();

  if (splits == 1) {
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const int n = n0 + r;
        if (n >= N) continue;
        if (epi == SSD_EPI_GEGLU && (r & 1)) continue;
#pragma unroll
        for (int m = 0; m < MMAX; ++m)
          if (m < M) {
            const float sc = rowscale ? inv_s[m] : 1.f;
            const float a0 = rowscale ? __fmul_rn(acc[r][m], sc) : acc[r][m];
            const float a1 = (r + 1 < ROWS) ? (rowscale ? __fmul_rn(acc[r + 1][m], sc) : acc[r + 1][m]) : 0.f;
            epilogue_store<T>(epi, y, N, m, n, a0, a1);
          }
      }
    }
    return;
  }
  // split-K partials: ws[split][m][n]
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const int n = n0 + r;
      if (n >= N) continue;
#pragma unroll
      for (int m = 0; m < MMAX; ++m)
        if (m < M) ws[((int64_t)split * M + m) * N + n] = acc[r][m];
    }
  }
  if (!last_block_of(&counters[tile], (unsigned)splits, &is_last)) return;
  const int tile_n0 = tile * kWarps * ROWS;
  const int tile_rows = min(kWarps * ROWS, N - tile_n0);
  for (int i = threadIdx.x; i < M * tile_rows; i += kLinThreads) {
    const int m = i / tile_rows, r = i % tile_rows, n = tile_n0 + r;
    if (epi == SSD_EPI_GEGLU && (n & 1)) continue;
    float s = 0.f, s2 = 0.f;
    for (int sp = 0; sp < splits; ++sp) {
      s += __ldcg(&ws[((int64_t)sp * M + m) * N + n]);
      if (epi == SSD_EPI_GEGLU) s2 += __ldcg(&ws[((int64_t)sp * M + m) * N + n + 1]);
    }
    if (rowscale) {
      s = __fmul_rn(s, inv_s[m]);
      s2 = __fmul_rn(s2, inv_s[m]);
    }
    epilogue_store<T>(epi, y, N, m, n, s, s2);
  }
}

}  // namespace

// Split plan from (N, K, rows per CTA): enough CTAs to cover the SMs twice
// and a K slice that fits the x stage in shared memory.
LinearPlan plan_linear_cc(int N, int K, int elem_bytes) {
  LinearPlan p;
  const int vn = 16 / elem_bytes;
  const int max_kc = (elem_bytes == 2) ? 4096 : 2048;
  const int tiles = (N + kWarps * 4 - 1) / (kWarps * 4);  // rows per CTA at ROWS = 4 (the smaller tile)
  int splits = (K + max_kc - 1) / max_kc;
  while (tiles * splits < 2 * 148 && K / (splits * 2) >= 512) splits *= 2;
  int kc = (K + splits - 1) / splits;
  kc = (kc + 32 * vn - 1) / (32 * vn) * (32 * vn);
  splits = (K + kc - 1) / kc;
  p.splits = splits;
  p.kc = kc;
  p.tiles_max = tiles;
  return p;
}

size_t linear_cc_workspace(int M, int N, int K, int elem_bytes) {
  const LinearPlan p = plan_linear_cc(N, K, elem_bytes);
  if (p.splits == 1) return 256;
  return kCounterBytes + align_up256(sizeof(float) * (size_t)p.splits * M * N);
}

template <typename T, int MMAX, int ROWS>
static int launch_cc(cudaStream_t st, const void* x, const void* w, void* y, int epi, int M, int N, int K,
                     const LinearPlan& p, void* ws, int rowscale, float eps) {
  const int tiles = (N + kWarps * ROWS - 1) / (kWarps * ROWS);
  const size_t smem = sizeof(T) * (size_t)M * p.kc;
  auto kern = linear_cc_kernel<T, MMAX, ROWS>;
  // opt in whenever the dynamic part alone comes near the 48 KB default (static smem adds to it)
  if (smem > 32 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return SSD_ERR_LAUNCH;
  unsigned int* counters = reinterpret_cast<unsigned int*>(ws);
  float* part = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + kCounterBytes);
  SSD_PDL(kern, dim3(tiles, p.splits), kLinThreads, smem, st, reinterpret_cast<const T*>(x), reinterpret_cast<const T*>(w),
                                                         y, epi, M, N, K, p.splits, p.kc, part, counters, rowscale, eps);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

template <typename T>
int linear_cc(cudaStream_t st, const void* x, const void* w, void* y, int epi, int M, int N, int K, void* ws,
              size_t ws_bytes, int rowscale, float eps) {
  if (M > 16) return SSD_ERR_UNSUPPORTED;
  const LinearPlan p = plan_linear_cc(N, K, sizeof(T));
  if (p.splits > 1 && (!ws || ws_bytes < linear_cc_workspace(M, N, K, sizeof(T)))) return SSD_ERR_WORKSPACE;
  if (sizeof(T) * (size_t)M * p.kc > 200 * 1024) return SSD_ERR_UNSUPPORTED;
  if (p.splits > 1 && p.tiles_max > kCounterCap) return SSD_ERR_UNSUPPORTED;
  if (M <= 1) return launch_cc<T, 1, 8>(st, x, w, y, epi, M, N, K, p, ws, rowscale, eps);
  if (M <= 2) return launch_cc<T, 2, 8>(st, x, w, y, epi, M, N, K, p, ws, rowscale, eps);
  if (M <= 4) return launch_cc<T, 4, 8>(st, x, w, y, epi, M, N, K, p, ws, rowscale, eps);
  if (M <= 8) return launch_cc<T, 8, 8>(st, x, w, y, epi, M, N, K, p, ws, rowscale, eps);
  return launch_cc<T, 16, 4>(st, x, w, y, epi, M, N, K, p, ws, rowscale, eps);
}

template int linear_cc<bf16>(cudaStream_t, const void*, const void*, void*, int, int, int, int, void*, size_t, int,
                             float);
template int linear_cc<float>(cudaStream_t, const void*, const void*, void*, int, int, int, int, void*, size_t, int,
                              float);

}  // namespace ssd
