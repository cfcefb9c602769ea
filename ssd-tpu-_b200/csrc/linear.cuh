// Internal interface of the projection kernels (not part of the C ABI).
#pragma once
#include <cuda.h>

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

// TMA map over a bf16 KV cache plane stack [plane_pages][block_size][hkv][D]: box = one
// page of one head, 64 dims wide (128-byte swizzle); D % 64 == 0.
bool make_kv_page_map(CUtensorMap* m, const void* pages, int plane_pages, int block_size, int hkv, int D);

// ssd_paged_verify_attention with `early`: nonzero when the previous kernel in
// the stream writes only q and this step's new K/V rows (the decoder forward),
// so that the TMA kernel may read the tables and stream the older pages before
// waiting for it (programmatic dependent launch).
int paged_verify_attention_impl(ssd_stream_t stream, const void* q, const void* pages, int dtype, int num_layers,
                                int num_blocks, int block_size, int num_kv_heads, int head_dim, int layer,
                                const int32_t* block_tables, int max_blocks, const int32_t* seq_lens,
                                const int32_t* q_lens, void* out, float scale, int B, int T, int num_heads,
                                int max_seq_len, void* workspace, size_t workspace_bytes, int early);

// ---- tensor-parallel collectives fused into the tcgen05 projection epilogue
constexpr int kMaxTP = 8;
constexpr int kFlagTiles = 2048;  // output tiles (128 rows of W) per collective
// Control block of a rank's symmetric heap: word 2 = error status; from byte
// 256 the per-tile counters (how many collectives this rank has finished for
// output tile t -- every rank makes the same calls, so the counts agree), then
// the arrival flags [kMaxTP source ranks][kFlagTiles]: flag[s][t] holds the
// count of the last tile t that rank s has delivered here.
constexpr size_t kCtrlCountersOffset = 256;
constexpr size_t kCtrlFlagsOffset = kCtrlCountersOffset + sizeof(uint32_t) * kFlagTiles;
constexpr size_t kCommCtrlBytes = kCtrlFlagsOffset + sizeof(uint32_t) * kMaxTP * kFlagTiles;
enum { COLL_NONE = 0, COLL_ALLREDUCE = 1, COLL_ALLGATHER = 2 };

struct CollArgs {
  int mode;             // COLL_*
  int rank, world;
  char* heaps[kMaxTP];  // every rank's heap base, mapped in this process
  size_t ctrl_off;      // control block offset (same on every rank)
  size_t dst_off;       // all-reduce: receive area; all-gather: the fp32 output [M, ldy]
  int ldy, col_off;     // all-gather: row pitch and first column of this rank's block
  int recv_rows, recv_tiles;  // all-reduce: receive slots [2][recv_tiles][world][recv_rows][128] (fp32 | count << 32)
  int form;                   // all-reduce: SSD_ALLREDUCE_*
};

// QKV projection epilogue with RoPE and the K/V page write (weights with q/k
// rows stored as rotation pairs, see ssd_gemma_weights.qk_pairs): the rounded
// q values are rotated into q_out [M, hq, D], k rotated and v copied into the
// token's page slot, exactly as ssd_rope_kv_write does from a stored qkv row.
struct RopeArgs {
  bf16* q_out;
  bf16* pages;
  const int32_t* pos;     // [M] token positions (-1: no K/V write)
  const int32_t* tables;  // [B, max_blocks]
  const float* cos_t;     // [rope_max_pos, D/2]
  const float* sin_t;
  int64_t plane;          // elements of one K (or V) plane: layers * blocks * block_size * hkv * D
  int layer, num_blocks, block_size, max_blocks, hq, hkv, D, T, rope_max_pos;
};
constexpr int kEpiRopeQkv = 100;  // internal epilogue code (not part of the C ABI)

int linear_tc_rope(cudaStream_t st, const void* x, const void* w, int M, int N, int K, void* ws, size_t ws_bytes,
                   float eps, const RopeArgs& ra);

// mode ALLREDUCE: y[M,N] (bf16, residual in/out) += round(sum over ranks of x_r w_r^T)
// mode ALLGATHER: out[M, col_off .. col_off+N) = x w^T (fp32), written on every rank
int linear_tc_coll(cudaStream_t st, const void* x, const void* w, void* y, int M, int N, int K, void* ws,
                   size_t ws_bytes, const CollArgs& ca);

}  // namespace ssd
