// K1: multi-query paged verify attention; K2: KV-slot writes (plain and fused
// with RoPE).
//
// Semantics: jax_ssd/kernels/attention_ref.py:9-21 (softmax(q k^T * scale +
// mask) v) with the verify mask of jax_ssd/kernels/masks.py:33-40 and the page
// layout of jax_ssd/kernels/kv_cache.py:13 — pages[2][L][NB][BS][Hkv][D].
//
// Decomposition (flash-decoding): grid (split, kv_head x row_group, sequence).
// A CTA owns one KV head of one sequence, a fixed 256-position slice of its
// context, and up to 16 query rows (the G = Hq/Hkv query heads of that KV head
// times the T new tokens), so each K/V byte is read once per row group.  K/V
// tiles of 32 positions are double-buffered into shared memory with cp.async
// through the page table; scores, online softmax and P.V run on CUDA cores in
// fp32.  Each CTA leaves an unnormalised partial (o, m, l) per row; the last CTA
// of the (sequence, head, row group) folds the splits in split order.
//
// Batch invariance: split and tile boundaries sit at fixed absolute positions,
// each row's reductions run in a fixed order, and fully masked tiles / empty
// splits are exact no-ops, so a query's output does not depend on T or on the
// other rows — the greedy stream of a k+1-token verify equals the one-token
// decode stream bit for bit.
#include "common.cuh"

namespace ssd {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kRows = 16;      // query rows per CTA
constexpr int kTile = 32;      // positions per smem tile
constexpr int kChunk = 128;    // positions per split (fixed => batch invariant)
constexpr int kParts = 8;      // dim partitions for q.k (one warp each)

template <typename T> struct Vec16;
template <> struct Vec16<bf16> { static constexpr int N = 8; };
template <> struct Vec16<float> { static constexpr int N = 4; };

__device__ __forceinline__ void load16_to_f(const bf16* p, float* f) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  unpack8(u, f);
}
__device__ __forceinline__ void load16_to_f(const float* p, float* f) {
  float4 u = *reinterpret_cast<const float4*>(p);
  f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N> __device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

template <typename KV, int D>
struct AttnSmem {
  static constexpr int V16 = Vec16<KV>::N;
  static constexpr int KPAD = 16 / sizeof(KV);            // +16 B per K row: conflict-free
  static constexpr int KSTRIDE = D + KPAD;
  static constexpr size_t k_bytes = sizeof(KV) * kTile * KSTRIDE;
  static constexpr size_t v_bytes = sizeof(KV) * kTile * D;
  static constexpr size_t stage_bytes = k_bytes + v_bytes;
  static constexpr size_t q_bytes = sizeof(float) * kRows * D;
  static constexpr size_t spart_bytes = sizeof(float) * kParts * kRows * kTile;
  static constexpr size_t p_bytes = sizeof(float) * kRows * kTile;
  static constexpr size_t total = 2 * stage_bytes + q_bytes + spart_bytes + p_bytes + 3 * sizeof(float) * kRows + 64;
};

struct RowInfo {
  int nrows;        // rows in this CTA
  int pos[kRows];   // absolute position of each row's token (-1 = padding row)
};

// Fold the split partials of one (sequence, KV head, row group) in split order.
// Only splits that start before seq_len can hold keys; the per-row weights
// w_s = exp(m_s - M) and the normaliser L are computed once per row by one warp
// (lane-strided over splits, xor-tree sums: adding an empty split's exact zeros
// leaves them unchanged, so the result does not depend on how many empty splits
// exist), then every output element sums w_s * o_s in split order with
// independent loads in flight.
template <typename KV, int D>
__device__ __forceinline__ void attention_fold(const float* __restrict__ ws_o, const float2* __restrict__ ws_ml,
                                               KV* __restrict__ out, int64_t grp_id, int nsplit, int seq_len,
                                               int nrows, int row0, int G, int T, int hq, int kvh, int b,
                                               float* wsm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ns = max(1, min(nsplit, (seq_len + kChunk - 1) / kChunk));
  __shared__ float inv_l[kRows];
  // wsm: [kRows][ns] weights (ns <= 256 fits the score-partial region)
  for (int r = warp; r < nrows; r += kAttnThreads / 32) {
    const int64_t rb = grp_id * nsplit * kRows + r;
    float mloc = -INFINITY;
    for (int s = lane; s < ns; s += 32) mloc = fmaxf(mloc, __ldcg(&ws_ml[rb + (int64_t)s * kRows]).x);
    const float M = warp_max(mloc);
    float lsum = 0.f;
    for (int s = lane; s < ns; s += 32) {
      const float2 ml = __ldcg(&ws_ml[rb + (int64_t)s * kRows]);
      const float w = (ml.x == -INFINITY || M == -INFINITY) ? 0.f : expf(ml.x - M);
      wsm[r * 256 + s] = w;
      lsum += ml.y * w;
    }
    const float L = warp_sum(lsum);
    if (lane == 0) inv_l[r] = L;
  }
  __syncthreads();
  for (int i = tid; i < nrows * D; i += kAttnThreads) {
    const int r = i / D, d = i % D;
    const int64_t rb = grp_id * nsplit * kRows + r;
    const float* wr = wsm + r * 256;
    float O = 0.f;
    int s = 0;
    for (; s + 4 <= ns; s += 4) {
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = wr[s + j] != 0.f ? __ldcg(&ws_o[(rb + (int64_t)(s + j) * kRows) * D + d]) : 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) O += wr[s + j] * v[j];
    }
    for (; s < ns; ++s) O += wr[s] != 0.f ? wr[s] * __ldcg(&ws_o[(rb + (int64_t)s * kRows) * D + d]) : 0.f;
    const float L = inv_l[r];
    const float res = (L > 0.f) ? O / L : 0.f;
    const int gr = row0 + r, t = gr / G, g = gr % G;
    out[(((int64_t)b * T + t) * hq + kvh * G + g) * D + d] = from_f<KV>(res);
  }
}

template <typename KV, int D>
__global__ void __launch_bounds__(kAttnThreads)
paged_attention_kernel(const KV* __restrict__ q, const KV* __restrict__ pages, int num_layers, int num_blocks,
                       int block_size, int hkv, int layer, const int32_t* __restrict__ block_tables,
                       int max_blocks, const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ q_lens,
                       KV* __restrict__ out, float scale, int T, int hq, int row_groups, int nsplit,
                       float* __restrict__ ws_o, float2* __restrict__ ws_ml, unsigned int* __restrict__ counters) {
  using S = AttnSmem<KV, D>;
  constexpr int V16 = S::V16;
  extern __shared__ __align__(16) unsigned char smem[];
  KV* kbuf[2];
  KV* vbuf[2];
  kbuf[0] = reinterpret_cast<KV*>(smem);
  vbuf[0] = reinterpret_cast<KV*>(smem + S::k_bytes);
  kbuf[1] = reinterpret_cast<KV*>(smem + S::stage_bytes);
  vbuf[1] = reinterpret_cast<KV*>(smem + S::stage_bytes + S::k_bytes);
  float* qs = reinterpret_cast<float*>(smem + 2 * S::stage_bytes);
  float* spart = qs + kRows * D;
  float* ps = spart + kParts * kRows * kTile;
  float* m_s = ps + kRows * kTile;
  float* l_s = m_s + kRows;
  float* a_s = l_s + kRows;
  __shared__ RowInfo ri;
  __shared__ bool is_last;

  const int split = blockIdx.x;
  const int kvh = blockIdx.y / row_groups, rg = blockIdx.y % row_groups;
  const int b = blockIdx.z;
  const int G = hq / hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int seq_len = seq_lens[b];
  const int ql = q_lens ? q_lens[b] : T;
  const int total_rows = G * T;
  const int row0 = rg * kRows;

  if (tid == 0) {
    ri.nrows = min(kRows, total_rows - row0);
    for (int r = 0; r < kRows; ++r) {
      const int gr = row0 + r;          // row = t * G + g
      const int t = gr / G;
      ri.pos[r] = (r < ri.nrows && t < ql) ? seq_len - ql + t : -1;
    }
  }
  __syncthreads();
  const int nrows = ri.nrows;
  int kmax = 0;  // one past the last position any row of this CTA sees
  for (int r = 0; r < nrows; ++r) kmax = max(kmax, ri.pos[r] + 1);
  const int k_begin = split * kChunk;
  // positions beyond the table's reach are never read (guards a seq_len larger than the pages)
  const int k_end = min(min(min(k_begin + kChunk, kmax), seq_len), max_blocks * block_size);

  const int64_t grp_id = ((int64_t)b * hkv + kvh) * row_groups + rg;
  if (k_end <= k_begin) {
    // No key of this split is visible to any row: mark the rows empty (m = -inf,
    // l = 0; the fold then never reads their o) and take the ticket.
    if (tid < nrows) ws_ml[(grp_id * nsplit + split) * kRows + tid] = make_float2(-INFINITY, 0.f);
    if (!last_block_of(&counters[grp_id], (unsigned)nsplit, &is_last)) return;
    attention_fold<KV, D>(ws_o, ws_ml, out, grp_id, nsplit, seq_len, nrows, row0, G, T, hq, kvh, b, spart);
    return;
  }

  // q rows -> fp32 smem (zeros for padding rows)
  for (int i = tid; i < kRows * D; i += kAttnThreads) {
    const int r = i / D, d = i % D;
    float v = 0.f;
    if (r < nrows && ri.pos[r] >= 0) {
      const int gr = row0 + r, t = gr / G, g = gr % G;
      v = to_f(q[(((int64_t)b * T + t) * hq + kvh * G + g) * D + d]);
    }
    qs[i] = v;
  }
  if (tid < kRows) { m_s[tid] = -INFINITY; l_s[tid] = 0.f; }

  // per-thread output accumulators: dim pair dp, rows r = grp + k*groups
  constexpr int PAIRS = D / 2;
  constexpr int GROUPS = kAttnThreads / PAIRS;  // 2 (D=256), 4 (128), 8 (64)
  constexpr int RPT = kRows / GROUPS;           // rows per thread
  const int dp = tid % PAIRS, grp = tid / PAIRS;
  float acc0[RPT], acc1[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) { acc0[i] = 0.f; acc1[i] = 0.f; }

  const int64_t plane = (int64_t)num_layers * num_blocks * block_size * hkv * D;  // K -> V plane offset
  const KV* kbase = pages + (int64_t)layer * num_blocks * block_size * hkv * D;
  const int32_t* table = block_tables + (int64_t)b * max_blocks;

  auto issue_tile = [&](int stage, int t0) {
    // 32 positions x D elements of K and of V, 16-byte pieces
    constexpr int PIECES = D / V16;
    for (int i = tid; i < kTile * PIECES; i += kAttnThreads) {
      const int j = i / PIECES, c = i % PIECES;
      const int p = t0 + j;
      if (p < k_end) {
        int blk = table[p / block_size];
        if ((unsigned)blk >= (unsigned)num_blocks) blk = 0;  // unallocated entry: stay in bounds
        const KV* src = kbase + (((int64_t)blk * block_size + (p % block_size)) * hkv + kvh) * D + c * V16;
        cp_async16(kbuf[stage] + j * S::KSTRIDE + c * V16, src);
        cp_async16(vbuf[stage] + j * D + c * V16, src + plane);
      }
    }
    cp_async_commit();
  };

  const int ntiles = k_end > k_begin ? (k_end - k_begin + kTile - 1) / kTile : 0;
  if (ntiles > 0) issue_tile(0, k_begin);
  __syncthreads();

  for (int it = 0; it < ntiles; ++it) {
    const int stage = it & 1;
    const int t0 = k_begin + it * kTile;
    if (it + 1 < ntiles) { issue_tile(stage ^ 1, t0 + kTile); cp_async_wait<1>(); }
    else cp_async_wait<0>();
    __syncthreads();

    // ---- scores: warp = dim partition, lane = position
    {
      constexpr int DP = D / kParts;
      const KV* krow = kbuf[stage] + lane * S::KSTRIDE + warp * DP;
      float kv[DP];
#pragma unroll
      for (int c = 0; c < DP; c += V16) load16_to_f(krow + c, kv + c);
      for (int r = 0; r < nrows; ++r) {
        const float* qr = qs + r * D + warp * DP;
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < DP; ++c) s = fmaf(qr[c], kv[c], s);
        spart[(warp * kRows + r) * kTile + lane] = s;
      }
    }
    __syncthreads();
    // ---- online softmax: warp per row, lane = position
    for (int r = warp; r < nrows; r += kAttnThreads / 32) {
      const int p = t0 + lane;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kParts; ++w) s += spart[(w * kRows + r) * kTile + lane];
      const bool ok = (p < k_end) && (p <= ri.pos[r]);
      s = ok ? s * scale : -INFINITY;
      const float tmax = warp_max(s);
      const float m_old = m_s[r];
      const float m_new = fmaxf(m_old, tmax);
      float pr = 0.f, alpha = 1.f;
      if (m_new != -INFINITY) {
        pr = ok ? expf(s - m_new) : 0.f;
        alpha = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
      }
      const float psum = warp_sum(pr);
      ps[r * kTile + lane] = pr;
      if (lane == 0) {
        m_s[r] = m_new;
        l_s[r] = (m_new == -INFINITY) ? 0.f : l_s[r] * alpha + psum;
        a_s[r] = alpha;
      }
    }
    __syncthreads();
    // ---- o = o * alpha + P V
    {
      const KV* vb = vbuf[stage];
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const int r = grp + i * GROUPS;
        if (r < nrows) {
          const float al = a_s[r];
          acc0[i] *= al;
          acc1[i] *= al;
        }
      }
      const int jn = min(kTile, k_end - t0);
      for (int j = 0; j < jn; ++j) {
        const float v0 = to_f(vb[j * D + 2 * dp]);
        const float v1 = to_f(vb[j * D + 2 * dp + 1]);
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
          const int r = grp + i * GROUPS;
          if (r < nrows) {
            const float pj = ps[r * kTile + j];
            acc0[i] = fmaf(pj, v0, acc0[i]);
            acc1[i] = fmaf(pj, v1, acc1[i]);
          }
        }
      }
    }
    __syncthreads();
  }

  // ---- partials: ws_o[(((b*hkv + kvh)*row_groups + rg)*nsplit + split)*kRows + r][D]
  const int64_t base = (grp_id * nsplit + split) * kRows;
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = grp + i * GROUPS;
    if (r < nrows) {
      ws_o[(base + r) * D + 2 * dp] = acc0[i];
      ws_o[(base + r) * D + 2 * dp + 1] = acc1[i];
    }
  }
  if (tid < nrows) ws_ml[base + tid] = make_float2(m_s[tid], l_s[tid]);

  if (!last_block_of(&counters[grp_id], (unsigned)nsplit, &is_last)) return;

  attention_fold<KV, D>(ws_o, ws_ml, out, grp_id, nsplit, seq_len, nrows, row0, G, T, hq, kvh, b, spart);
}

// ---------------------------------------------------------------- K2
template <typename KV>
__global__ void kv_write_kernel(KV* __restrict__ pages, int num_layers, int num_blocks, int block_size, int hkv,
                                int D, int layer, const int32_t* __restrict__ block_tables, int max_blocks,
                                const int32_t* __restrict__ positions, const KV* __restrict__ k,
                                const KV* __restrict__ v, int T) {
  const int b = blockIdx.y, t = blockIdx.x;
  const int p = positions[(int64_t)b * T + t];
  if (p < 0 || p / block_size >= max_blocks) return;
  const int blk = block_tables[(int64_t)b * max_blocks + p / block_size];
  if ((unsigned)blk >= (unsigned)num_blocks) return;
  const int64_t plane = (int64_t)num_layers * num_blocks * block_size * hkv * D;
  KV* dst = pages + (((int64_t)layer * num_blocks + blk) * block_size + p % block_size) * hkv * D;
  const KV* ks = k + ((int64_t)b * T + t) * hkv * D;
  const KV* vs = v + ((int64_t)b * T + t) * hkv * D;
  for (int i = threadIdx.x; i < hkv * D; i += blockDim.x) {
    dst[i] = ks[i];
    dst[plane + i] = vs[i];
  }
}

// RoPE on q and k of a fused qkv row, q -> q_out, k (rotated) and v -> pages.
// grid (Hq + Hkv, T, B): one CTA per head of one token, one thread per rotation pair.
template <typename KV>
__global__ void rope_kv_write_kernel(const KV* __restrict__ qkv, KV* __restrict__ q_out, KV* __restrict__ pages,
                                     int num_layers, int num_blocks, int block_size, int hq, int hkv, int D,
                                     int layer, const int32_t* __restrict__ block_tables, int max_blocks,
                                     const int32_t* __restrict__ positions, const float* __restrict__ cos_t,
                                     const float* __restrict__ sin_t, int rope_max_pos, int T) {
  const int h = blockIdx.x, t = blockIdx.y, b = blockIdx.z;
  const int64_t m = (int64_t)b * T + t;
  const int p = positions[m];
  const int half = D / 2;
  const int width = (hq + 2 * hkv) * D;
  const KV* row = qkv + m * width;
  const int pc = (p < 0) ? 0 : min(p, rope_max_pos - 1);
  const float* cr = cos_t + (int64_t)pc * half;
  const float* sr = sin_t + (int64_t)pc * half;
  const int64_t plane = (int64_t)num_layers * num_blocks * block_size * hkv * D;
  KV* dst = nullptr;
  if (h >= hq && p >= 0 && p / block_size < max_blocks) {
    const int blk = block_tables[(int64_t)b * max_blocks + p / block_size];
    if ((unsigned)blk < (unsigned)num_blocks)
      dst = pages + (((int64_t)layer * num_blocks + blk) * block_size + p % block_size) * hkv * D;
  }
  const KV* src = row + h * D;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float x1 = to_f(src[i]), x2 = to_f(src[i + half]);
    const float c = cr[i], s = sr[i];
    // separate products, as the oracle's float32 expression evaluates them
    const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    const float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
    if (h < hq) {
      KV* qo = q_out + (m * hq + h) * D;
      qo[i] = from_f<KV>(y1);
      qo[i + half] = from_f<KV>(y2);
    } else if (dst) {
      KV* ko = dst + (h - hq) * D;
      ko[i] = from_f<KV>(y1);
      ko[i + half] = from_f<KV>(y2);
    }
  }
  if (dst) {  // the matching V head
    const KV* vsrc = row + (hq + hkv + (h - hq)) * D;
    KV* vo = dst + plane + (h - hq) * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) vo[i] = vsrc[i];
  }
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct AttnLayout {
  int row_groups, nsplit;
  size_t groups, off_cnt, off_o, off_ml, total;
};

inline AttnLayout attn_layout(int B, int T, int hq, int hkv, int D, int max_seq_len) {
  AttnLayout L;
  const int G = hq / hkv;
  L.row_groups = (G * T + kRows - 1) / kRows;
  L.nsplit = (max_seq_len + kChunk - 1) / kChunk;
  if (L.nsplit < 1) L.nsplit = 1;  // <= 256 (checked by the caller): the fold keeps one weight per split
  const size_t groups = (size_t)B * hkv * L.row_groups;
  const size_t rows = groups * L.nsplit * kRows;
  L.groups = groups;
  L.off_cnt = 0;
  L.off_o = kCounterBytes;
  L.off_ml = L.off_o + align256(sizeof(float) * rows * D);
  L.total = L.off_ml + align256(sizeof(float2) * rows);
  return L;
}

template <typename KV, int D>
int launch_attention(cudaStream_t st, const void* q, const void* pages, int num_layers, int num_blocks,
                     int block_size, int hkv, int layer, const int32_t* tables, int max_blocks,
                     const int32_t* seq_lens, const int32_t* q_lens, void* out, float scale, int B, int T, int hq,
                     const AttnLayout& L, void* ws) {
  using S = AttnSmem<KV, D>;
  auto kern = paged_attention_kernel<KV, D>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::total) != cudaSuccess)
    return SSD_ERR_LAUNCH;
  char* w = reinterpret_cast<char*>(ws);
  dim3 grid(L.nsplit, hkv * L.row_groups, B);
  kern<<<grid, kAttnThreads, S::total, st>>>(
      reinterpret_cast<const KV*>(q), reinterpret_cast<const KV*>(pages), num_layers, num_blocks, block_size, hkv,
      layer, tables, max_blocks, seq_lens, q_lens, reinterpret_cast<KV*>(out), scale, T, hq, L.row_groups,
      L.nsplit, reinterpret_cast<float*>(w + L.off_o), reinterpret_cast<float2*>(w + L.off_ml),
      reinterpret_cast<unsigned int*>(w + L.off_cnt));
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

}  // namespace
}  // namespace ssd

using namespace ssd;

extern "C" size_t ssd_paged_attention_workspace_size(int B, int T, int num_heads, int num_kv_heads, int head_dim,
                                                     int max_seq_len) {
  if (B <= 0 || T <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || head_dim <= 0 || max_seq_len <= 0)
    return 0;
  return attn_layout(B, T, num_heads, num_kv_heads, head_dim, max_seq_len).total;
}

extern "C" int ssd_paged_verify_attention(ssd_stream_t stream, const void* q, const void* pages, int dtype,
                                          int num_layers, int num_blocks, int block_size, int num_kv_heads,
                                          int head_dim, int layer, const int32_t* block_tables, int max_blocks,
                                          const int32_t* seq_lens, const int32_t* q_lens, void* out, float scale,
                                          int B, int T, int num_heads, int max_seq_len, void* workspace,
                                          size_t workspace_bytes) {
  if (B <= 0 || T <= 0 || num_kv_heads <= 0 || num_heads <= 0 || num_heads % num_kv_heads || layer < 0 ||
      layer >= num_layers || block_size <= 0 || max_blocks <= 0 || max_seq_len <= 0 || !q || !pages || !out ||
      !block_tables || !seq_lens)
    return SSD_ERR_INVALID;
  if ((int64_t)max_blocks * block_size < max_seq_len) return SSD_ERR_INVALID;
  if (max_seq_len > 256 * kChunk) return SSD_ERR_UNSUPPORTED;  // 32768 positions
  if (B > 65535 || (int64_t)num_kv_heads * ((num_heads / num_kv_heads * T + kRows - 1) / kRows) > 65535)
    return SSD_ERR_UNSUPPORTED;
  const AttnLayout L = attn_layout(B, T, num_heads, num_kv_heads, head_dim, max_seq_len);
  if (!workspace || workspace_bytes < L.total) return SSD_ERR_WORKSPACE;
  if (L.groups > (size_t)kCounterCap) return SSD_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
#define SSD_ATTN_CASE(KVT, DD)                                                                                  \
  return launch_attention<KVT, DD>(st, q, pages, num_layers, num_blocks, block_size, num_kv_heads, layer,       \
                                   block_tables, max_blocks, seq_lens, q_lens, out, scale, B, T, num_heads, L, \
                                   workspace)
  if (dtype == SSD_DTYPE_BF16) {
    if (head_dim == 256) SSD_ATTN_CASE(bf16, 256);
    if (head_dim == 128) SSD_ATTN_CASE(bf16, 128);
    if (head_dim == 64) SSD_ATTN_CASE(bf16, 64);
  } else if (dtype == SSD_DTYPE_F32) {
    if (head_dim == 256) SSD_ATTN_CASE(float, 256);
    if (head_dim == 128) SSD_ATTN_CASE(float, 128);
    if (head_dim == 64) SSD_ATTN_CASE(float, 64);
  }
#undef SSD_ATTN_CASE
  return SSD_ERR_UNSUPPORTED;
}

extern "C" int ssd_kv_write(ssd_stream_t stream, void* pages, int dtype, int num_layers, int num_blocks,
                            int block_size, int num_kv_heads, int head_dim, int layer, const int32_t* block_tables,
                            int max_blocks, const int32_t* positions, const void* k, const void* v, int B, int T) {
  if (B <= 0 || T <= 0 || layer < 0 || layer >= num_layers || !pages || !block_tables || !positions || !k || !v)
    return SSD_ERR_INVALID;
  if (B > 65535) return SSD_ERR_UNSUPPORTED;
  dim3 grid(T, B);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == SSD_DTYPE_BF16)
    kv_write_kernel<bf16><<<grid, 256, 0, st>>>(reinterpret_cast<bf16*>(pages), num_layers, num_blocks, block_size,
                                                num_kv_heads, head_dim, layer, block_tables, max_blocks, positions,
                                                reinterpret_cast<const bf16*>(k), reinterpret_cast<const bf16*>(v), T);
  else if (dtype == SSD_DTYPE_F32)
    kv_write_kernel<float><<<grid, 256, 0, st>>>(reinterpret_cast<float*>(pages), num_layers, num_blocks,
                                                 block_size, num_kv_heads, head_dim, layer, block_tables, max_blocks,
                                                 positions, reinterpret_cast<const float*>(k),
                                                 reinterpret_cast<const float*>(v), T);
  else
    return SSD_ERR_INVALID;
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

extern "C" int ssd_rope_kv_write(ssd_stream_t stream, const void* qkv, void* q_out, void* pages, int dtype,
                                 int num_layers, int num_blocks, int block_size, int num_heads, int num_kv_heads,
                                 int head_dim, int layer, const int32_t* block_tables, int max_blocks,
                                 const int32_t* positions, const float* rope_cos, const float* rope_sin,
                                 int rope_max_pos, int B, int T) {
  if (B <= 0 || T <= 0 || layer < 0 || layer >= num_layers || head_dim % 2 || !qkv || !q_out || !pages ||
      !block_tables || !positions || !rope_cos || !rope_sin || rope_max_pos <= 0)
    return SSD_ERR_INVALID;
  if (B > 65535 || T > 65535) return SSD_ERR_UNSUPPORTED;
  dim3 grid(num_heads + num_kv_heads, T, B);
  const int threads = head_dim / 2 < 32 ? 32 : (head_dim / 2 > 256 ? 256 : head_dim / 2);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == SSD_DTYPE_BF16)
    rope_kv_write_kernel<bf16><<<grid, threads, 0, st>>>(
        reinterpret_cast<const bf16*>(qkv), reinterpret_cast<bf16*>(q_out), reinterpret_cast<bf16*>(pages),
        num_layers, num_blocks, block_size, num_heads, num_kv_heads, head_dim, layer, block_tables, max_blocks,
        positions, rope_cos, rope_sin, rope_max_pos, T);
  else if (dtype == SSD_DTYPE_F32)
    rope_kv_write_kernel<float><<<grid, threads, 0, st>>>(
        reinterpret_cast<const float*>(qkv), reinterpret_cast<float*>(q_out), reinterpret_cast<float*>(pages),
        num_layers, num_blocks, block_size, num_heads, num_kv_heads, head_dim, layer, block_tables, max_blocks,
        positions, rope_cos, rope_sin, rope_max_pos, T);
  else
    return SSD_ERR_INVALID;
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}
