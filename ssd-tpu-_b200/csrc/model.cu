// Whole-model verify forward (native runtime) and the small fused ops it uses.
//
// ssd_gemma_forward replaces DecodeModelAdapter.verify / prefill / decode
// (jax_ssd/models/base.py:34-58) as implemented by GemmaAdapter
// (jax_ssd/models/gemma_adapter.py:81-143): one host call issues the whole
// layer stack on one stream, so it can be captured into a CUDA graph.  Per
// layer (5 launches): QKV projection with the input RMSNorm fused (norm weight
// folded into the weight columns, row rsqrt applied in the epilogue) -> RoPE +
// K/V page write -> paged attention -> O projection with the residual add fused
// -> gate/up projection with the MLP RMSNorm and GeGLU fused -> down projection
// with the residual add fused.  Numerics: bf16 storage between these ops, fp32
// math inside them.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "linear.cuh"

namespace ssd {
namespace {

template <typename T>
__global__ void embed_kernel(const int32_t* tokens, const T* E, T* x, int d,
                             int vocab, float scale) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  int tok = tokens[m];
  tok = tok < 0 ? 0 : (tok >= vocab ? vocab - 1 : tok);
  const T* e = E + (int64_t)tok * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) x[(int64_t)m * d + i] = from_f<T>(__fmul_rn(to_f(e[i]), scale));
}

// One CTA per row.  bf16 rows with d % 8 == 0 are read once as 16-byte vectors
// kept in registers (d <= 8 * 256 * 4); other shapes take the scalar loop.
template <typename T>
__global__ void rmsnorm_kernel(const T* x, const T* w, T* y, int d, float eps) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  const T* xr = x + (int64_t)m * d;
  float s = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float v = to_f(xr[i]);
    s = fmaf(v, v, s);
  }
  s = block_reduce(s, red, OpSum());
  const float ms = __fdiv_rn(s, (float)d);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    y[(int64_t)m * d + i] = from_f<T>(__fmul_rn(__fmul_rn(to_f(xr[i]), inv), __fadd_rn(1.0f, to_f(w[i]))));
}

__global__ void __launch_bounds__(256) rmsnorm_bf16_vec_kernel(const bf16* x, const bf16* w,
                                                              bf16* y, int d, float eps) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  const int nv = d / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (int64_t)m * d);
  float v[4][8];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < nv) {
      unpack8(xr[i], v[j]);
#pragma unroll
      for (int e = 0; e < 8; ++e) s = fmaf(v[j][e], v[j][e], s);
    }
  }
  s = block_reduce(s, red, OpSum());
  const float ms = __fdiv_rn(s, (float)d);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + (int64_t)m * d);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = threadIdx.x + j * blockDim.x;
    if (i < nv) {
      float wv[8];
      unpack8(wr[i], wv);
      uint4 o;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float a = __fmul_rn(__fmul_rn(v[j][2 * e], inv), __fadd_rn(1.0f, wv[2 * e]));
        const float c = __fmul_rn(__fmul_rn(v[j][2 * e + 1], inv), __fadd_rn(1.0f, wv[2 * e + 1]));
        oh[e] = __floats2bfloat162_rn(a, c);
      }
      yr[i] = o;
    }
  }
}

// positions[b*T+t] = seq_lens_before[b] + t for t < q_lens[b], else -1; seq_after[b].
__global__ void positions_kernel(const int32_t* slb, const int32_t* ql, int B, int T,
                                 int32_t* pos, int32_t* seq_after,
                                 int32_t* qlen_out) {
  pdl_wait();
  pdl_trigger();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < B * T; i += gridDim.x * blockDim.x) {
    const int b = i / T, t = i % T;
    const int q = ql ? ql[b] : T;
    pos[i] = t < q ? slb[b] + t : -1;
    if (t == 0) {
      seq_after[b] = slb[b] + q;
      qlen_out[b] = q;
    }
  }
}

// rows[b] = h[b*T + q_lens[b]-1]  (last valid token per sequence)
template <typename T>
__global__ void gather_last_kernel(const T* h, const int32_t* qlen, int tq, int d,
                                   T* out) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const int t = min(max(qlen[b] - 1, 0), tq - 1);
  for (int i = threadIdx.x; i < d; i += blockDim.x) out[(int64_t)b * d + i] = h[((int64_t)b * tq + t) * d + i];
}

inline size_t a256(size_t x) { return align_up256(x); }

struct Scratch {
  void *x, *h, *qkv, *q, *attn, *act, *hl;
  int32_t *pos, *seq_after, *qlen;
  void* lin_ws;
  size_t lin_ws_bytes;
  void* attn_ws;
  size_t attn_ws_bytes;
  size_t total;
};

int max_m() { return 256; }  // tcgen05 path; the CUDA-core path takes M <= 16

size_t linear_ws_any(int M, int N, int K, int dtype) {
  if (dtype == SSD_DTYPE_BF16 && linear_tc_supported(M, N, K)) return linear_tc_workspace(M, N, K);
  return linear_cc_workspace(M, N, K, dtype == SSD_DTYPE_BF16 ? 2 : 4);
}

Scratch carve(const ssd_gemma_weights* w, int B, int T, int max_seq_len, char* base) {
  Scratch s{};
  const size_t es = w->dtype == SSD_DTYPE_BF16 ? 2 : 4;
  const int M = B * T;
  const int d = w->d_model, D = w->head_dim, hq = w->num_heads, hkv = w->num_kv_heads, F = w->ffn;
  size_t off = 0;
  auto take = [&](size_t bytes) { char* p = base ? base + off : nullptr; off += a256(bytes); return (void*)p; };
  s.x = take(es * M * d);
  s.h = take(es * M * d);
  s.qkv = take(es * (size_t)M * (hq + 2 * hkv) * D);
  s.q = take(es * (size_t)M * hq * D);
  s.attn = take(es * (size_t)M * hq * D);
  s.act = take(es * (size_t)M * F);
  s.hl = take(es * (size_t)B * d);
  s.pos = (int32_t*)take(sizeof(int32_t) * M);
  s.seq_after = (int32_t*)take(sizeof(int32_t) * B);
  s.qlen = (int32_t*)take(sizeof(int32_t) * B);
  size_t lw = 0;
  auto upd = [&](int m, int n, int k) { lw = std::max(lw, linear_ws_any(m, n, k, w->dtype)); };
  upd(M, (hq + 2 * hkv) * D, d);
  upd(M, d, hq * D);
  upd(M, 2 * F, d);
  upd(M, d, F);
  upd(M, w->vocab, d);
  upd(B, w->vocab, d);
  s.lin_ws_bytes = lw;
  s.lin_ws = take(lw);
  s.attn_ws_bytes = ssd_paged_attention_workspace_size(B, T, hq, hkv, D, max_seq_len);
  s.attn_ws = take(s.attn_ws_bytes);
  s.total = off;
  return s;
}

}  // namespace

int linear_allreduce_impl(cudaStream_t st, const void* x, const void* w, void* y, int M, int N, int K, void* ws,
                          size_t ws_bytes, const ssd_comm* c);
int linear_allgather_impl(cudaStream_t st, const void* x, const void* w, float* y, int ldy, int M, int N, int K,
                          void* ws, size_t ws_bytes, const ssd_comm* c);

int linear_dispatch(cudaStream_t st, const void* x, const void* w, int dtype, void* y, int epi, int M, int N, int K,
                    void* ws, size_t ws_bytes, int rowscale = 0, float eps = 0.f) {
  if (dtype == SSD_DTYPE_BF16) {
    if (linear_tc_supported(M, N, K)) return linear_tc(st, x, w, y, epi, M, N, K, ws, ws_bytes, rowscale, eps);
    return linear_cc<bf16>(st, x, w, y, epi, M, N, K, ws, ws_bytes, rowscale, eps);
  }
  return linear_cc<float>(st, x, w, y, epi, M, N, K, ws, ws_bytes, rowscale, eps);
}

}  // namespace ssd

using namespace ssd;

extern "C" const char* ssd_status_string(int status) {
  switch (status) {
    case SSD_OK: return "ok";
    case SSD_ERR_INVALID: return "invalid argument";
    case SSD_ERR_LAUNCH: return "CUDA launch error";
    case SSD_ERR_TIMEOUT: return "device-side wait timed out";
    case SSD_ERR_UNSUPPORTED: return "shape outside compiled kernel limits";
    case SSD_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

extern "C" int ssd_abi_version(void) { return (1 << 16) | 1; }

extern "C" int ssd_linear_max_m(void) { return max_m(); }

extern "C" size_t ssd_linear_workspace_size(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  // large enough for either storage dtype
  return std::max(linear_ws_any(M, N, K, SSD_DTYPE_BF16), linear_ws_any(M, N, K, SSD_DTYPE_F32));
}

extern "C" int ssd_linear(ssd_stream_t stream, const void* x, const void* w, int dtype, void* y, int epilogue, int M,
                          int N, int K, void* workspace, size_t workspace_bytes) {
  if (M <= 0 || N <= 0 || K <= 0 || !x || !w || !y) return SSD_ERR_INVALID;
  if (M > max_m()) return SSD_ERR_UNSUPPORTED;
  if (epilogue < SSD_EPI_STORE || epilogue > SSD_EPI_GEGLU) return SSD_ERR_INVALID;
  if (epilogue == SSD_EPI_GEGLU && (N & 1)) return SSD_ERR_INVALID;
  if (dtype != SSD_DTYPE_BF16 && dtype != SSD_DTYPE_F32) return SSD_ERR_INVALID;
  const int vn = dtype == SSD_DTYPE_BF16 ? 8 : 4;
  if (K % vn) return SSD_ERR_UNSUPPORTED;
  return linear_dispatch((cudaStream_t)stream, x, w, dtype, y, epilogue, M, N, K, workspace, workspace_bytes);
}

extern "C" int ssd_linear_rownorm(ssd_stream_t stream, const void* x, const void* w, int dtype, void* y, int epilogue,
                                  int M, int N, int K, float eps, void* workspace, size_t workspace_bytes) {
  if (M <= 0 || N <= 0 || K <= 0 || !x || !w || !y || !(eps >= 0.f)) return SSD_ERR_INVALID;
  if (M > max_m()) return SSD_ERR_UNSUPPORTED;
  if (epilogue != SSD_EPI_STORE && epilogue != SSD_EPI_STORE_F32 && epilogue != SSD_EPI_GEGLU) return SSD_ERR_INVALID;
  if (epilogue == SSD_EPI_GEGLU && (N & 1)) return SSD_ERR_INVALID;
  if (dtype != SSD_DTYPE_BF16 && dtype != SSD_DTYPE_F32) return SSD_ERR_INVALID;
  const int vn = dtype == SSD_DTYPE_BF16 ? 8 : 4;
  if (K % vn) return SSD_ERR_UNSUPPORTED;
  return linear_dispatch((cudaStream_t)stream, x, w, dtype, y, epilogue, M, N, K, workspace, workspace_bytes, 1, eps);
}

extern "C" int ssd_embed(ssd_stream_t stream, const int32_t* tokens, const void* embed, int dtype, void* x, int M,
                         int d, int vocab) {
  if (M <= 0 || d <= 0 || vocab <= 0 || !tokens || !embed || !x) return SSD_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  float scale = sqrtf((float)d);
  if (dtype == SSD_DTYPE_BF16) {
    scale = __bfloat162float(__float2bfloat16_rn(scale));
    SSD_PDL(embed_kernel<bf16>, M, 256, 0, st, tokens, (const bf16*)embed, (bf16*)x, d, vocab, scale);
  } else if (dtype == SSD_DTYPE_F32) {
    SSD_PDL(embed_kernel<float>, M, 256, 0, st, tokens, (const float*)embed, (float*)x, d, vocab, scale);
  } else {
    return SSD_ERR_INVALID;
  }
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

extern "C" int ssd_rmsnorm(ssd_stream_t stream, const void* x, const void* w, int dtype, void* y, int M, int d,
                           float eps) {
  if (M <= 0 || d <= 0 || !x || !w || !y) return SSD_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec = (d % 8 == 0) && d <= 8 * 256 * 4 && !(reinterpret_cast<uintptr_t>(x) & 15) &&
                   !(reinterpret_cast<uintptr_t>(w) & 15) && !(reinterpret_cast<uintptr_t>(y) & 15);
  if (dtype == SSD_DTYPE_BF16 && vec)
    SSD_PDL(rmsnorm_bf16_vec_kernel, M, 256, 0, st, (const bf16*)x, (const bf16*)w, (bf16*)y, d, eps);
  else if (dtype == SSD_DTYPE_BF16)
    SSD_PDL(rmsnorm_kernel<bf16>, M, 256, 0, st, (const bf16*)x, (const bf16*)w, (bf16*)y, d, eps);
  else if (dtype == SSD_DTYPE_F32)
    SSD_PDL(rmsnorm_kernel<float>, M, 256, 0, st, (const float*)x, (const float*)w, (float*)y, d, eps);
  else
    return SSD_ERR_INVALID;
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

static bool weights_ok(const ssd_gemma_weights* w) {
  if (!w || w->num_layers <= 0 || w->d_model <= 0 || w->num_heads <= 0 || w->num_kv_heads <= 0 ||
      w->num_heads % w->num_kv_heads || w->head_dim <= 0 || w->ffn <= 0 || w->vocab <= 0)
    return false;
  if (w->dtype != SSD_DTYPE_BF16 && w->dtype != SSD_DTYPE_F32) return false;
  if (!w->embed || !w->final_norm || !w->w_qkv || !w->w_o || !w->w_gate_up || !w->w_down || !w->rope_cos ||
      !w->rope_sin || w->rope_max_pos <= 0)
    return false;
  for (int l = 0; l < w->num_layers; ++l)
    if (!w->w_qkv[l] || !w->w_o[l] || !w->w_gate_up[l] || !w->w_down[l]) return false;
  if (w->tp_world < 0 || w->tp_world > SSD_MAX_TP || w->tp_rank < 0 || (w->tp_world > 1 && w->tp_rank >= w->tp_world))
    return false;
  if (w->qk_pairs && (w->dtype != SSD_DTYPE_BF16 || (w->head_dim & 1) ||
                      !linear_tc_supported(max_m(), (w->num_heads + 2 * w->num_kv_heads) * w->head_dim, w->d_model)))
    return false;
  return true;
}

extern "C" size_t ssd_gemma_scratch_size(const ssd_gemma_weights* w, int B, int T, int max_seq_len) {
  if (!w || B <= 0 || T <= 0 || max_seq_len <= 0) return 0;
  return carve(w, B, T, max_seq_len, nullptr).total;
}

extern "C" int ssd_gemma_forward(ssd_stream_t stream, const ssd_gemma_weights* w, const ssd_gemma_batch* bt) {
  if (!weights_ok(w) || !bt) return SSD_ERR_INVALID;
  const int B = bt->B, T = bt->T, M = B * T;
  if (B <= 0 || T <= 0 || !bt->tokens || !bt->seq_lens_before || !bt->kv_pages || !bt->block_tables ||
      !bt->scratch || bt->max_seq_len <= 0 || bt->num_blocks <= 0 || bt->block_size <= 0)
    return SSD_ERR_INVALID;
  if (M > max_m()) return SSD_ERR_UNSUPPORTED;
  if ((int64_t)bt->max_blocks * bt->block_size < bt->max_seq_len) return SSD_ERR_INVALID;
  if (bt->max_seq_len > w->rope_max_pos) return SSD_ERR_INVALID;
  if (w->tp_world > 1 && !bt->comm) return SSD_ERR_INVALID;
  if (bt->comm) {
    const ssd_comm* c = bt->comm;
    if (c->world != std::max(w->tp_world, 1) || c->rank != w->tp_rank || w->dtype != SSD_DTYPE_BF16 ||
        w->vocab % c->world)
      return SSD_ERR_INVALID;
  }
  const Scratch s = carve(w, B, T, bt->max_seq_len, reinterpret_cast<char*>(bt->scratch));
  if (bt->scratch_bytes < s.total) return SSD_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const int dt = w->dtype;
  const int d = w->d_model, D = w->head_dim, hq = w->num_heads, hkv = w->num_kv_heads, F = w->ffn;
  const int L = w->num_layers;
  const float scale = 1.0f / sqrtf((float)D);
  int rc;
#define SSD_TRY(expr)              \
  do {                             \
    rc = (expr);                   \
    if (rc != SSD_OK) return rc;   \
  } while (0)
  int nprof = 0;
  // while the stream is being captured, timing events must be external records
  // (they stay timed event nodes in the graph); outside capture a plain record
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (bt->prof_events) cudaStreamIsCapturing(st, &cap);
  const bool capturing = cap == cudaStreamCaptureStatusActive;
  auto rec_event = [&](void* ev) {
    if (capturing) cudaEventRecordWithFlags((cudaEvent_t)ev, st, cudaEventRecordExternal);
    else cudaEventRecord((cudaEvent_t)ev, st);
  };
  auto timed = [&](int kind, auto&& launch) {
    const bool rec = bt->prof_events && nprof < bt->prof_capacity;
    if (rec) rec_event(bt->prof_events[2 * nprof]);
    const int r = launch();
    if (rec) {
      rec_event(bt->prof_events[2 * nprof + 1]);
      if (bt->prof_kind) bt->prof_kind[nprof] = kind;
      ++nprof;
      if (bt->prof_count) *bt->prof_count = nprof;
    }
    return r;
  };
  auto proj = [&](int kind, const void* x, const void* wt, void* y, int epi, int m, int n, int k, int rowscale) {
    return timed(kind, [&] {
      return linear_dispatch(st, x, wt, dt, y, epi, m, n, k, s.lin_ws, s.lin_ws_bytes, rowscale, w->eps);
    });
  };
  // row-parallel projection + residual: all-reduced over the tensor-parallel group when there is one
  const ssd_comm* comm = bt->comm;
  auto proj_rowpar = [&](int kind, const void* x, const void* wt, void* y, int m, int n, int k) {
    if (!comm) return proj(kind, x, wt, y, SSD_EPI_RESIDUAL, m, n, k, 0);
    return timed(kind, [&] { return linear_allreduce_impl(st, x, wt, y, m, n, k, s.lin_ws, s.lin_ws_bytes, comm); });
  };
  // tied LM head, vocab-parallel under tensor parallelism
  auto lm_head = [&](const void* x, int m) {
    if (!comm) return proj(4, x, w->embed, bt->logits, SSD_EPI_STORE_F32, m, w->vocab, d, 0);
    const int vloc = w->vocab / comm->world;
    const void* wt = reinterpret_cast<const bf16*>(w->embed) + (size_t)comm->rank * vloc * d;
    return timed(4, [&] {
      return linear_allgather_impl(st, x, wt, bt->logits, w->vocab, m, vloc, d, s.lin_ws, s.lin_ws_bytes, comm);
    });
  };
  if (bt->prof_count) *bt->prof_count = 0;

  SSD_PDL(positions_kernel, (M + 255) / 256, 256, 0, st, bt->seq_lens_before, bt->q_lens, B, T, s.pos, s.seq_after,
                                                     s.qlen);
  SSD_CHECK_LAUNCH();
  SSD_TRY(ssd_embed(stream, bt->tokens, w->embed, dt, s.x, M, d, w->vocab));
  for (int l = 0; l < L; ++l) {
    // RMSNorm folded: w_qkv carries (1 + attn_norm) in its columns, the projection
    // scales each token row by its rsqrt(mean(x^2) + eps)
    if (w->qk_pairs) {
      // RoPE and the K/V page write in the projection's epilogue (q/k rows stored as rotation pairs)
      RopeArgs ra;
      ra.q_out = reinterpret_cast<bf16*>(s.q);
      ra.pages = reinterpret_cast<bf16*>(bt->kv_pages);
      ra.pos = s.pos;
      ra.tables = bt->block_tables;
      ra.cos_t = w->rope_cos;
      ra.sin_t = w->rope_sin;
      ra.plane = (int64_t)L * bt->num_blocks * bt->block_size * hkv * D;
      ra.layer = l;
      ra.num_blocks = bt->num_blocks;
      ra.block_size = bt->block_size;
      ra.max_blocks = bt->max_blocks;
      ra.hq = hq;
      ra.hkv = hkv;
      ra.D = D;
      ra.T = T;
      ra.rope_max_pos = w->rope_max_pos;
      SSD_TRY(timed(0, [&] {
        return linear_tc_rope(st, s.x, w->w_qkv[l], M, (hq + 2 * hkv) * D, d, s.lin_ws, s.lin_ws_bytes, w->eps, ra);
      }));
    } else {
      SSD_TRY(proj(0, s.x, w->w_qkv[l], s.qkv, SSD_EPI_STORE, M, (hq + 2 * hkv) * D, d, 1));
      SSD_TRY(ssd_rope_kv_write(stream, s.qkv, s.q, bt->kv_pages, dt, L, bt->num_blocks, bt->block_size, hq, hkv, D,
                                l, bt->block_tables, bt->max_blocks, s.pos, w->rope_cos, w->rope_sin,
                                w->rope_max_pos, B, T));
    }
    // early = 1: the kernel before it (RoPE + K/V write, or the QKV projection that
    // does them) writes only q and the new rows
    SSD_TRY(paged_verify_attention_impl(stream, s.q, bt->kv_pages, dt, L, bt->num_blocks, bt->block_size, hkv, D, l,
                                       bt->block_tables, bt->max_blocks, s.seq_after, s.qlen, s.attn, scale, B, T,
                                       hq, bt->max_seq_len, s.attn_ws, s.attn_ws_bytes, 1));
    SSD_TRY(proj_rowpar(1, s.attn, w->w_o[l], s.x, M, d, hq * D));
    SSD_TRY(proj(2, s.x, w->w_gate_up[l], s.act, SSD_EPI_GEGLU, M, 2 * F, d, 1));  // mlp_norm folded likewise
    SSD_TRY(proj_rowpar(3, s.act, w->w_down[l], s.x, M, d, F));
  }
  if (!bt->logits) return SSD_OK;  // prompt chunk: only the K/V rows were needed
  SSD_TRY(ssd_rmsnorm(stream, s.x, w->final_norm, dt, s.h, M, d, w->eps));
  if (bt->logits_last_only) {
    if (dt == SSD_DTYPE_BF16)
      SSD_PDL(gather_last_kernel<bf16>, B, 256, 0, st, (const bf16*)s.h, s.qlen, T, d, (bf16*)s.hl);
    else
      SSD_PDL(gather_last_kernel<float>, B, 256, 0, st, (const float*)s.h, s.qlen, T, d, (float*)s.hl);
    SSD_CHECK_LAUNCH();
    SSD_TRY(lm_head(s.hl, B));
  } else {
    SSD_TRY(lm_head(s.h, M));
  }
#undef SSD_TRY
  return SSD_OK;
}
