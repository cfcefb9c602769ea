// K1: multi-query paged verify attention; K2: KV-slot writes (plain and fused
// with RoPE).
//
// Semantics: jax_ssd/kernels/attention_ref.py:9-21 (softmax(q k^T * scale +
// mask) v) with the verify mask of jax_ssd/kernels/masks.py:33-40 and the page
// layout of jax_ssd/kernels/kv_cache.py:13 -- pages[2][L][NB][BS][Hkv][D].
//
// Decomposition (flash-decoding): grid (split, kv_head x row_group, sequence).
// A CTA owns one KV head of one sequence, a fixed 128-position slice of its
// context and up to 8 query rows (the G = Hq/Hkv query heads of that KV head
// times the new tokens), so each K/V byte is read once per row group.  Inside
// the CTA each of the 8 warps owns 16 consecutive positions and runs start to
// finish without CTA-wide synchronisation, with all of its loads in flight at
// once (decode attention is latency-bound: a few hundred positions):
//   * scores: 4 positions per round, 8 lanes per position each holding 16-byte
//     pieces of the K row (128-byte contiguous segments), q rows from shared
//     memory, a 3-step xor reduction per row;
//   * softmax statistics per row with two warp reductions (lane = position);
//   * P.V with lane = D/32 head dims: V rows read coalesced, p from a per-warp
//     shared-memory row.
// The warps' (m, l, o) are then combined in warp order, the CTA writes one
// partial per row, and the last CTA of the group folds the splits in split
// order (atomic ticket).
//
// Batch invariance: split and warp boundaries sit at fixed absolute positions,
// every reduction of a row runs in a fixed order, and fully masked warps or
// splits contribute exact zeros, so a query's output does not depend on T or
// on the other rows -- a k+1-token verify reproduces one-token decodes bit for bit.
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "linear.cuh"

namespace ssd {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kWarpsA = kAttnThreads / 32;
constexpr int kRows = 8;                       // query rows per CTA
constexpr int kWarpKeys = 16;                  // positions per warp
constexpr int kChunk = kWarpsA * kWarpKeys;    // positions per split (fixed => batch invariant)

template <typename T> struct Vec16;
template <> struct Vec16<bf16> { static constexpr int N = 8; };
template <> struct Vec16<float> { static constexpr int N = 4; };

// N consecutive elements (N * sizeof(KV) in {4, 8, 16} bytes, aligned) -> fp32
template <int N>
__device__ __forceinline__ void load_n(const bf16* p, float* f) {
  if constexpr (N == 8) {
    unpack8(ld_act_v4(p), f);
  } else if constexpr (N == 4) {
    uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = __bfloat162float(p[i]);
  }
}
template <int N>
__device__ __forceinline__ void load_n(const float* p, float* f) {
#pragma unroll
  for (int i = 0; i < N; ++i) f[i] = p[i];
}

template <typename KV, int D>
struct AttnSmem {
  static constexpr size_t q_bytes = sizeof(float) * kRows * D;
  static constexpr size_t p_bytes = sizeof(float) * kWarpsA * kRows * kWarpKeys;
  static constexpr size_t o_bytes = sizeof(float) * kWarpsA * kRows * D;
  static constexpr size_t ml_bytes = sizeof(float2) * kWarpsA * kRows;
  static constexpr size_t total = q_bytes + p_bytes + o_bytes + ml_bytes + 64;
};

struct RowInfo {
  int nrows;        // rows in this CTA
  int pos[kRows];   // absolute position of each row's token (-1 = padding row)
};

// Fold the split partials of one (sequence, KV head, row group) in split order.
// Only splits that start before seq_len can hold keys; the per-row weights
// w_s = exp(m_s - M) and the normaliser L are computed once per row by one warp
// (lane-strided over splits, xor-tree sums: an empty split's exact zeros leave
// them unchanged), then every output element sums w_s * o_s in split order.
template <typename KV, int D, int CHUNK = kChunk, int NTHREADS = kAttnThreads>
__device__ __forceinline__ void attention_fold(const float* ws_o, const float2* ws_ml,
                                               KV* out, int64_t grp_id, int nsplit, int seq_len,
                                               int nrows, int row0, int G, int T, int hq, int kvh, int b,
                                               float* wsm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ns = max(1, min(nsplit, (seq_len + CHUNK - 1) / CHUNK));
  __shared__ float inv_l[kRows];
  for (int r = warp; r < nrows; r += NTHREADS / 32) {
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
  for (int i = tid; i < nrows * D; i += NTHREADS) {
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
paged_attention_kernel(const KV* q, const KV* pages, int num_layers, int num_blocks,
                       int block_size, int hkv, int layer, const int32_t* block_tables,
                       int max_blocks, const int32_t* seq_lens, const int32_t* q_lens,
                       KV* out, float scale, int T, int hq, int row_groups, int nsplit,
                       float* ws_o, float2* ws_ml, unsigned int* counters) {
  using S = AttnSmem<KV, D>;
  constexpr int V16 = Vec16<KV>::N;      // elements per 16-byte load
  constexpr int DPL = D / 32;            // head dims per lane in P.V
  constexpr int KCH = D / (8 * V16);     // 16-byte K pieces per lane and position (8 lanes per position)
  static_assert(KCH >= 1, "head_dim too small");
  extern __shared__ __align__(16) unsigned char smem[];
  float* qs = reinterpret_cast<float*>(smem);                 // [kRows][D]
  float* ps = qs + kRows * D;                                 // [warp][kRows][kWarpKeys]
  float* os = ps + kWarpsA * kRows * kWarpKeys;               // [warp][kRows][D]
  float2* mls = reinterpret_cast<float2*>(os + kWarpsA * kRows * D);  // [warp][kRows]
  __shared__ RowInfo ri;
  __shared__ bool is_last;

  pdl_wait();
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
    // no key of this split is visible to any row: mark the rows empty and take the ticket
    if (tid < nrows) ws_ml[(grp_id * nsplit + split) * kRows + tid] = make_float2(-INFINITY, 0.f);
    pdl_trigger();
    if (!last_block_of(&counters[grp_id], (unsigned)nsplit, &is_last)) return;
    attention_fold<KV, D>(ws_o, ws_ml, out, grp_id, nsplit, seq_len, nrows, row0, G, T, hq, kvh, b, os);
    return;
  }

  const int64_t plane = (int64_t)num_layers * num_blocks * block_size * hkv * D;  // K -> V plane offset
  const KV* kbase = pages + (int64_t)layer * num_blocks * block_size * hkv * D;
  const int32_t* table = block_tables + (int64_t)b * max_blocks;
  const int t0 = k_begin + warp * kWarpKeys;
  const int jn = max(0, min(kWarpKeys, k_end - t0));   // positions of this warp that exist

  // Row offsets of this warp's positions: lane j (< kWarpKeys) resolves position t0 + j.
  int64_t my_off = 0;
  if (lane < jn) {
    const int key = t0 + lane;
    int blk = table[key / block_size];
    if ((unsigned)blk >= (unsigned)num_blocks) blk = 0;  // unallocated entry: stay in bounds
    my_off = (((int64_t)blk * block_size + key % block_size) * hkv + kvh) * D;
  }

  // ---- issue every K load of this warp before any arithmetic: 4 positions per
  // round (8 lanes each, 128-byte contiguous segments), KCH pieces per lane
  const int kq = lane >> 3, li = lane & 7;
  constexpr int ROUNDS = kWarpKeys / 4;
  uint4 kraw[ROUNDS][KCH];
#pragma unroll
  for (int rd = 0; rd < ROUNDS; ++rd) {
    const int j = rd * 4 + kq;
    const int64_t off = __shfl_sync(0xffffffffu, my_off, j);
#pragma unroll
    for (int c = 0; c < KCH; ++c)
      kraw[rd][c] = (j < jn) ? ld_act_v4(kbase + off + c * 8 * V16 + li * V16) : make_uint4(0, 0, 0, 0);
  }

  // q rows -> fp32 smem (zeros for padding rows), while the K loads are in flight
  for (int i = tid; i < kRows * D; i += kAttnThreads) {
    const int r = i / D, d = i % D;
    float v = 0.f;
    if (r < nrows && ri.pos[r] >= 0) {
      const int gr = row0 + r, t = gr / G, g = gr % G;
      v = to_f(q[(((int64_t)b * T + t) * hq + kvh * G + g) * D + d]);
    }
    qs[i] = v;
  }
  __syncthreads();

  // ---- scores: lane (kq, li) dots its pieces, the 8 lanes of a position reduce
  float* pw = ps + warp * kRows * kWarpKeys;
#pragma unroll
  for (int rd = 0; rd < ROUNDS; ++rd) {
    const int j = rd * 4 + kq;
    float part[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) part[r] = 0.f;
#pragma unroll
    for (int c = 0; c < KCH; ++c) {
      float kv[V16];
      if constexpr (V16 == 8) unpack8(kraw[rd][c], kv);
      else { kv[0] = __uint_as_float(kraw[rd][c].x); kv[1] = __uint_as_float(kraw[rd][c].y);
             kv[2] = __uint_as_float(kraw[rd][c].z); kv[3] = __uint_as_float(kraw[rd][c].w); }
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        if (r < nrows) {
          const float* qr = qs + r * D + c * 8 * V16 + li * V16;
#pragma unroll
          for (int e = 0; e < V16; ++e) part[r] = fmaf(qr[e], kv[e], part[r]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      if (r < nrows) {
        float v = part[r];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        if (li == 0) pw[r * kWarpKeys + j] = v;
      }
    }
  }

  // ---- V loads for P.V (lane = DPL dims), issued before the softmax math
  float vv[kWarpKeys][DPL];
#pragma unroll
  for (int j = 0; j < kWarpKeys; ++j) {
    const int64_t off = __shfl_sync(0xffffffffu, my_off, j);
    if (j < jn) load_n<DPL>(kbase + plane + off + lane * DPL, vv[j]);
    else {
#pragma unroll
      for (int e = 0; e < DPL; ++e) vv[j][e] = 0.f;
    }
  }
  __syncwarp();

  // ---- softmax statistics of this warp's positions, per row (lane = position)
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    if (r < nrows) {
      const int key = t0 + lane;
      const bool ok = lane < jn && key <= ri.pos[r];
      const float sc = ok ? pw[r * kWarpKeys + (lane & (kWarpKeys - 1))] * scale : -INFINITY;
      const float m = warp_max(sc);
      const float pr = (ok && m != -INFINITY) ? expf(sc - m) : 0.f;
      const float l = warp_sum(pr);
      __syncwarp();
      if (lane < kWarpKeys) pw[r * kWarpKeys + lane] = pr;
      if (lane == 0) mls[warp * kRows + r] = make_float2(m, l);
    }
  }
  __syncwarp();

  // ---- o = P.V
  float o[kRows][DPL];
#pragma unroll
  for (int r = 0; r < kRows; ++r)
#pragma unroll
    for (int e = 0; e < DPL; ++e) o[r][e] = 0.f;
#pragma unroll
  for (int j = 0; j < kWarpKeys; ++j) {
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      if (r < nrows) {
        const float pj = pw[r * kWarpKeys + j];
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[r][e] = fmaf(pj, vv[j][e], o[r][e]);
      }
    }
  }
  float* ow = os + warp * kRows * D;
#pragma unroll
  for (int r = 0; r < kRows; ++r)
    if (r < nrows)
#pragma unroll
      for (int e = 0; e < DPL; ++e) ow[r * D + lane * DPL + e] = o[r][e];
  __syncthreads();

  // ---- combine the warps in warp order -> this split's partial per row
  const int64_t base = (grp_id * nsplit + split) * kRows;
  for (int i = tid; i < nrows * D; i += kAttnThreads) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarpsA; ++w) M = fmaxf(M, mls[w * kRows + r].x);
    float O = 0.f, L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarpsA; ++w) {
        const float2 ml = mls[w * kRows + r];
        const float wt = (ml.x == -INFINITY) ? 0.f : expf(ml.x - M);
        L += ml.y * wt;
        O += os[(w * kRows + r) * D + d] * wt;
      }
    }
    ws_o[(base + r) * D + d] = O;
    if (d == 0) ws_ml[base + r] = make_float2(M, L);
  }
  pdl_trigger();

  if (!last_block_of(&counters[grp_id], (unsigned)nsplit, &is_last)) return;
  attention_fold<KV, D>(ws_o, ws_ml, out, grp_id, nsplit, seq_len, nrows, row0, G, T, hq, kvh, b, os);
}

// ---------------------------------------------------------------- K1, bf16 on tensor cores
// Same decomposition and partial/fold protocol as paged_attention_kernel, but
// each warp's 16 positions go through mma.sync m16n8k16 (bf16 in, fp32
// accumulate): S[16 rows x 16 positions] = Q K^T over D/16 k-steps, the row
// softmax of the warp's positions on the S fragments, then O[16 x D] += P V with
// P re-packed from the S accumulators as the A operand.  K/V rows of the warp are
// staged in shared memory with cp.async (positions past the end are
// zero-filled, so P = 0 never meets stale data), Q once per CTA; fragments come
// from ldmatrix (.trans for V).  P is rounded to bf16 before P.V.
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <int D>
struct TcSmem {
  static constexpr int STRIDE = D + 8;                         // bf16 elements per row (+16 B: ldmatrix conflict-free)
  static constexpr size_t q_bytes = 2ull * 16 * STRIDE;
  static constexpr size_t kv_bytes = 2ull * kWarpsA * kWarpKeys * STRIDE;   // per plane
  static constexpr size_t o_bytes = sizeof(float) * kWarpsA * kRows * D;   // aliases the K tiles
  static constexpr size_t ml_bytes = sizeof(float2) * kWarpsA * kRows;
  static constexpr size_t total = q_bytes + 2 * kv_bytes + ml_bytes + 128;
  static_assert(o_bytes <= kv_bytes, "warp outputs must fit in the K tiles");
};

template <int D>
__global__ void __launch_bounds__(kAttnThreads, 1)
paged_attention_tc_kernel(const bf16* q, const bf16* pages, int num_layers,
                          int num_blocks, int block_size, int hkv, int layer, const int32_t* block_tables,
                          int max_blocks, const int32_t* seq_lens, const int32_t* q_lens,
                          bf16* out, float scale, int T, int hq, int row_groups, int nsplit,
                          float* ws_o, float2* ws_ml, unsigned int* counters) {
  using S = TcSmem<D>;
  constexpr int ST = S::STRIDE;
  constexpr int KSTEPS = D / 16;
  constexpr int NT = D / 8;              // n-tiles of P.V
  extern __shared__ __align__(16) unsigned char smem[];
  bf16* qs = reinterpret_cast<bf16*>(smem);                                // [16][ST]
  bf16* ks = reinterpret_cast<bf16*>(smem + S::q_bytes);                   // [warp][16][ST]
  bf16* vs = reinterpret_cast<bf16*>(smem + S::q_bytes + S::kv_bytes);     // [warp][16][ST]
  float* os = reinterpret_cast<float*>(ks);                                // [warp][kRows][D] after P.V
  float2* mls = reinterpret_cast<float2*>(smem + S::q_bytes + 2 * S::kv_bytes);
  __shared__ RowInfo ri;
  __shared__ bool is_last;

  pdl_wait();
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
      const int gr = row0 + r;
      const int t = gr / G;
      ri.pos[r] = (r < ri.nrows && t < ql) ? seq_len - ql + t : -1;
    }
  }
  __syncthreads();
  const int nrows = ri.nrows;
  int kmax = 0;
  for (int r = 0; r < nrows; ++r) kmax = max(kmax, ri.pos[r] + 1);
  const int k_begin = split * kChunk;
  const int k_end = min(min(min(k_begin + kChunk, kmax), seq_len), max_blocks * block_size);
  const int64_t grp_id = ((int64_t)b * hkv + kvh) * row_groups + rg;
  if (k_end <= k_begin) {
    if (tid < nrows) ws_ml[(grp_id * nsplit + split) * kRows + tid] = make_float2(-INFINITY, 0.f);
    pdl_trigger();
    if (!last_block_of(&counters[grp_id], (unsigned)nsplit, &is_last)) return;
    attention_fold<bf16, D>(ws_o, ws_ml, out, grp_id, nsplit, seq_len, nrows, row0, G, T, hq, kvh, b,
                            reinterpret_cast<float*>(ks));
    return;
  }

  const int64_t plane = (int64_t)num_layers * num_blocks * block_size * hkv * D;
  const bf16* kbase = pages + (int64_t)layer * num_blocks * block_size * hkv * D;
  const int32_t* table = block_tables + (int64_t)b * max_blocks;
  const int t0 = k_begin + warp * kWarpKeys;
  const int jn = max(0, min(kWarpKeys, k_end - t0));

  // ---- stage this warp's K and V rows (16 B pieces, zero-fill past the end)
  {
    int64_t my_off = 0;
    if (lane < jn) {
      const int key = t0 + lane;
      int blk = table[key / block_size];
      if ((unsigned)blk >= (unsigned)num_blocks) blk = 0;
      my_off = (((int64_t)blk * block_size + key % block_size) * hkv + kvh) * D;
    }
    constexpr int PIECES = D / 8;                 // 16-byte pieces per row
    const uint32_t kw = (uint32_t)__cvta_generic_to_shared(ks + warp * kWarpKeys * ST);
    const uint32_t vw = (uint32_t)__cvta_generic_to_shared(vs + warp * kWarpKeys * ST);
#pragma unroll 4
    for (int i = lane; i < kWarpKeys * PIECES; i += 32) {
      const int j = i / PIECES, c = i % PIECES;
      const int64_t off = __shfl_sync(0xffffffffu, my_off, j);
      const bool valid = j < jn;
      const bf16* src = kbase + (valid ? off : 0) + c * 8;
      cp_async16_zfill(kw + (uint32_t)(j * ST + c * 8) * 2, src, valid);
      cp_async16_zfill(vw + (uint32_t)(j * ST + c * 8) * 2, src + plane, valid);
    }
    asm volatile("cp.async.commit_group;");
  }
  // ---- Q rows (bf16, zero padding rows) while the K/V copies are in flight
  for (int i = tid; i < 16 * (D / 8); i += kAttnThreads) {
    const int r = i / (D / 8), c = i % (D / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nrows && ri.pos[r] >= 0) {
      const int gr = row0 + r, t = gr / G, g = gr % G;
      v = *reinterpret_cast<const uint4*>(q + (((int64_t)b * T + t) * hq + kvh * G + g) * D + c * 8);
    }
    *reinterpret_cast<uint4*>(qs + r * ST + c * 8) = v;
  }
  asm volatile("cp.async.wait_group 0;");
  __syncthreads();

  // ---- S = Q K^T for the warp's 16 positions (2 n-tiles of 8)
  float sacc[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) sacc[nt][e] = 0.f;
  const uint32_t qaddr0 = (uint32_t)__cvta_generic_to_shared(qs);
  const uint32_t kaddr0 = (uint32_t)__cvta_generic_to_shared(ks + warp * kWarpKeys * ST);
  const uint32_t vaddr0 = (uint32_t)__cvta_generic_to_shared(vs + warp * kWarpKeys * ST);
  const int lr = lane & 7, lm = lane >> 3;     // ldmatrix: row within matrix, matrix index
#pragma unroll
  for (int ks_ = 0; ks_ < KSTEPS; ++ks_) {
    uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
    // A: rows lr + 8*(lm&1), dims 16ks + 8*(lm>>1)
    ldsm_x4(qaddr0 + (uint32_t)((lr + 8 * (lm & 1)) * ST + 16 * ks_ + 8 * (lm >> 1)) * 2, a0, a1, a2, a3);
    // B: positions 8*(lm>>1) + lr, dims 16ks + 8*(lm&1)
    ldsm_x4(kaddr0 + (uint32_t)((8 * (lm >> 1) + lr) * ST + 16 * ks_ + 8 * (lm & 1)) * 2, b0, b1, b2, b3);
    mma_bf16_16816(sacc[0], a0, a1, a2, a3, b0, b1);
    mma_bf16_16816(sacc[1], a0, a1, a2, a3, b2, b3);
  }
  // ---- softmax of the warp's positions per row (rows lane/4 and lane/4 + 8;
  // only rows < kRows = 8 are real, the upper half of the tile stays empty)
  const int rA = lane >> 2;
  const int prow = (rA < nrows) ? ri.pos[rA] : -1;
  float pa[2][2];
  float m = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = t0 + nt * 8 + (lane & 3) * 2 + e;
      const bool ok = (key < k_end) && (key <= prow);
      pa[nt][e] = ok ? sacc[nt][e] * scale : -INFINITY;
      m = fmaxf(m, pa[nt][e]);
    }
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  float l = 0.f;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float pv = (m == -INFINITY || pa[nt][e] == -INFINITY) ? 0.f : expf(pa[nt][e] - m);
      pa[nt][e] = pv;
      l += pv;
    }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  if ((lane & 3) == 0 && rA < kRows) mls[warp * kRows + rA] = make_float2(m, l);
  // P as the A operand (rows 8-15 are zero)
  const uint32_t pa0 = pack_bf16(pa[0][0], pa[0][1]), pa1 = 0u;
  const uint32_t pa2 = pack_bf16(pa[1][0], pa[1][1]), pa3 = 0u;

  // ---- O = P V: n-tiles of 8 dims, two per ldmatrix.trans
  float oacc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) oacc[nt][e] = 0.f;
#pragma unroll
  for (int np = 0; np < NT / 2; ++np) {
    uint32_t b0, b1, b2, b3;
    // matrices: (dims 16np + 8*(lm>>1), positions 8*(lm&1) + lr)
    ldsm_x4_t(vaddr0 + (uint32_t)((8 * (lm & 1) + lr) * ST + 16 * np + 8 * (lm >> 1)) * 2, b0, b1, b2, b3);
    mma_bf16_16816(oacc[2 * np], pa0, pa1, pa2, pa3, b0, b1);
    mma_bf16_16816(oacc[2 * np + 1], pa0, pa1, pa2, pa3, b2, b3);
  }
  __syncthreads();  // every warp is done reading its K tile: the outputs may overwrite it
  float* ow = os + warp * kRows * D;
  if (rA < nrows) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      ow[rA * D + nt * 8 + (lane & 3) * 2] = oacc[nt][0];
      ow[rA * D + nt * 8 + (lane & 3) * 2 + 1] = oacc[nt][1];
    }
  }
  __syncthreads();

  // ---- combine the warps in warp order -> this split's partial per row
  const int64_t base = (grp_id * nsplit + split) * kRows;
  for (int i = tid; i < nrows * D; i += kAttnThreads) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarpsA; ++w) M = fmaxf(M, mls[w * kRows + r].x);
    float O = 0.f, L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarpsA; ++w) {
        const float2 ml = mls[w * kRows + r];
        const float wt = (ml.x == -INFINITY) ? 0.f : expf(ml.x - M);
        L += ml.y * wt;
        O += os[(w * kRows + r) * D + d] * wt;
      }
    }
    ws_o[(base + r) * D + d] = O;
    if (d == 0) ws_ml[base + r] = make_float2(M, L);
  }
  pdl_trigger();
  if (!last_block_of(&counters[grp_id], (unsigned)nsplit, &is_last)) return;
  attention_fold<bf16, D>(ws_o, ws_ml, out, grp_id, nsplit, seq_len, nrows, row0, G, T, hq, kvh, b, os);
}

// ---------------------------------------------------------------- K1, bf16, TMA-pipelined
// The verify/decode attention for bf16 pages of 16 rows.  A CTA owns one
// (sequence, KV head, row group) and a fixed 256-position split (16 pages):
//   * warp 0 (one lane) is the producer: it reads the page table and streams
//     each page's K and V rows into a ring of shared-memory stages with TMA
//     (a 5-D tensor map over the cache, box = 16 rows x 64 dims, 128-byte
//     swizzle, no multicast), one mbarrier per stage;
//   * the other warps are consumers (3 at D = 256, 4 otherwise): consumer c
//     takes pages c, c+C, c+2C, ... and keeps an online-softmax state per query
//     row (running max, sum and the 16 x D accumulator in registers) across
//     its pages: S = Q K^T and O += P V with mma.sync m16n8k16 (bf16 in, fp32
//     accumulate), fragments via ldmatrix from the swizzled stages.  The stage
//     count is a multiple of C, so every stage belongs to one consumer, which
//     waits on it exactly one phase after its previous use (an mbarrier wait
//     only tells phases apart modulo 2);
//   * the consumers' states are combined in warp order; a group whose context
//     fits one split writes its output directly, otherwise the split writes a
//     partial and the group's last split folds them in split order.
// Rows of a page past the end of the context are zeroed in the stage before
// P.V (masked probabilities are exact zeros, stale rows must not be NaN).
// At D = 256: 128 threads and ~106 KB of shared memory, two CTAs per SM, up
// to 12 pages (192 KB) of K/V in flight per SM.  Models with at most two KV heads
// (a GQA draft, a tensor-parallel shard) launch only one or two CTAs per sequence
// at decode contexts, so each CTA's consumers walk their pages one after another:
// they get 6 consumers and 12 stages instead (224 threads, ~203 KB, one CTA per
// SM), which halves the pages per consumer.  The consumer count is a property of
// the model's shape, never of the batch or the query count, so batch invariance
// holds as for the other kernels: splits, page ownership and every reduction
// order are fixed.
constexpr int kTmaChunk = 256;                  // positions per split
constexpr int kTmaPage = 16;                    // rows per page (TMA box height)
// consumer warps per CTA for head size D; the stage count is a multiple of it
template <int D>
constexpr int tma_consumers() {
  return D == 256 ? 3 : 4;
}
constexpr int kTmaWideConsumers = 6;  // D = 256, at most two KV heads
template <int D, int C>
constexpr int tma_threads() {
  return 32 * (1 + C);
}
constexpr uint32_t kTmaWaitLimit = 1u << 24;

__device__ __forceinline__ void tmb_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void tmb_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tmb_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool tmb_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait; false after kTmaWaitLimit polls (the caller records the error and stops)
__device__ __forceinline__ bool tmb_wait(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kTmaWaitLimit; ++i)
    if (tmb_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], "
      "[%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

template <int D, int C>
struct TmaSmem {
  static constexpr int CONS = C;
  static constexpr int CHUNKS = D / 64;                          // 128-byte swizzle rows per page row
  static constexpr uint32_t PLANE = kTmaPage * D * 2;            // K (or V) of one page: 16 x D bf16
  static constexpr uint32_t STAGE = 2 * PLANE;
  static constexpr int STAGES = D == 256 ? 2 * C : D == 128 ? 12 : 16;
  static_assert(STAGES % CONS == 0, "every stage must belong to one consumer (mbarrier parity)");
  static constexpr int QST = D + 8;                              // padded Q rows (ldmatrix conflict-free)
  static constexpr size_t ring = (size_t)STAGES * STAGE;
  static constexpr size_t q_off = ring;
  static constexpr size_t q_bytes = 2ull * 16 * QST;
  static constexpr size_t bar_off = q_off + q_bytes;
  static constexpr size_t ml_off = bar_off + 8 * 2 * STAGES + 16;
  static constexpr size_t total = 1024 + ml_off + sizeof(float2) * CONS * kRows;
  static constexpr size_t o_bytes = sizeof(float) * CONS * kRows * D;   // aliases the ring
  static_assert(o_bytes <= ring, "consumer outputs must fit in the ring");
};

// byte offset of (row, dim) inside one page plane laid out as [chunk][row][128 B], 128-byte swizzle
__device__ __forceinline__ uint32_t sw_off(int row, int dim) {
  const int c = dim >> 6, u = (dim >> 3) & 7;
  return (uint32_t)(c * (kTmaPage * 128) + row * 128 + ((u ^ (row & 7)) << 4));
}

template <int D, int C>
__global__ void __launch_bounds__(tma_threads<D, C>(), C > 4 ? 1 : 2)
paged_attention_tma_kernel(const __grid_constant__ CUtensorMap kvmap, const bf16* q, int num_layers, int num_blocks,
                           int hkv, int layer, const int32_t* block_tables, int max_blocks, const int32_t* seq_lens,
                           const int32_t* q_lens, bf16* out, float scale, int T, int hq, int row_groups, int nsplit,
                           float* ws_o, float2* ws_ml, unsigned int* counters, unsigned int* err, int early) {
  using S = TmaSmem<D, C>;
  constexpr int KSTEPS = D / 16;
  constexpr int NT = D / 8;
  constexpr int NCONS = S::CONS;
  constexpr int NTHREADS = tma_threads<D, C>();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const uint32_t raw = (uint32_t)__cvta_generic_to_shared(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* gb = smem_raw + (base - raw);
  bf16* qs = reinterpret_cast<bf16*>(gb + S::q_off);
  float* os = reinterpret_cast<float*>(gb);                        // [consumer][kRows][D], after the ring is done
  float2* mls = reinterpret_cast<float2*>(gb + S::ml_off);
  const uint32_t bars = base + (uint32_t)S::bar_off;
  auto full = [&](int st) { return bars + 8u * st; };
  auto empty = [&](int st) { return bars + 8u * (S::STAGES + st); };
  __shared__ RowInfo ri;
  __shared__ bool is_last;
  __shared__ int s_abort;

  const int split = blockIdx.x;
  const int kvh = blockIdx.y / row_groups, rg = blockIdx.y % row_groups;
  const int b = blockIdx.z;
  const int G = hq / hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    for (int st = 0; st < S::STAGES; ++st) {
      tmb_init(full(st), 1);
      tmb_init(empty(st), 1);
    }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&kvmap) : "memory");
  }
  // early != 0: the caller guarantees that the previous kernel in the stream
  // writes neither the sequence lengths, q_lens, the page tables nor any K/V row
  // below seq_len - q_len (it writes only q and this step's new rows).  Those are
  // then read, and the pages below the new rows streamed, before waiting for it.
  if (!early) pdl_wait();
  const int seq_len = ld_act(seq_lens + b);
  const int ql = q_lens ? ld_act(q_lens + b) : T;
  const int total_rows = G * T;
  const int row0 = rg * kRows;
  if (tid == 0) {
    ri.nrows = min(kRows, total_rows - row0);
    for (int r = 0; r < kRows; ++r) {
      const int gr = row0 + r;
      const int t = gr / G;
      ri.pos[r] = (r < ri.nrows && t < ql) ? seq_len - ql + t : -1;
    }
  }
  __syncthreads();
  const int nrows = ri.nrows;
  int kmax = 0;
  for (int r = 0; r < nrows; ++r) kmax = max(kmax, ri.pos[r] + 1);
  const int k_begin = split * kTmaChunk;
  const int k_end = min(min(min(k_begin + kTmaChunk, kmax), seq_len), max_blocks * kTmaPage);
  const int64_t grp_id = ((int64_t)b * hkv + kvh) * row_groups + rg;
  const int ns = max(1, min(nsplit, (seq_len + kTmaChunk - 1) / kTmaChunk));
  if (split >= ns) {  // past this sequence's context: the fold neither waits for nor reads this split
    pdl_trigger();
    return;
  }
  const int npages = k_end > k_begin ? (k_end - k_begin + kTmaPage - 1) / kTmaPage : 0;

  int issued = 0;  // pages the producer lane has put in flight
  __shared__ int s_blk[kTmaChunk / kTmaPage];
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // the split's page-table entries in one parallel load (not one L2 round trip per page)
    if (lane < npages) {
      int blk = ld_act(block_tables + (int64_t)b * max_blocks + (k_begin / kTmaPage + lane));
      s_blk[lane] = ((unsigned)blk >= (unsigned)num_blocks) ? 0 : blk;
    }
    __syncwarp();
    if (lane == 0 && npages > 0) {
      const int stable_end = early ? seq_len - ql : 0;  // rows below it are not the previous kernel's
      bool waited = !early;
      for (int j = 0; j < npages; ++j, ++issued) {
        if (!waited && k_begin + (j + 1) * kTmaPage > stable_end) {
          pdl_wait();
          waited = true;
        }
        const int st = j % S::STAGES;
        if (j >= S::STAGES && !tmb_wait(empty(st), (uint32_t)((j / S::STAGES) - 1) & 1u)) {
          s_abort = 1;
          atomicExch(err, 1u);
          break;
        }
        const int blk = s_blk[j];
        const int kpage = layer * num_blocks + blk;                      // plane 0 (K)
        const int vpage = (num_layers + layer) * num_blocks + blk;       // plane 1 (V)
        const uint32_t dst = base + (uint32_t)st * S::STAGE;
        tmb_expect_tx(full(st), S::STAGE);
#pragma unroll
        for (int c = 0; c < S::CHUNKS; ++c) {
          tma_load_5d(dst + (uint32_t)c * (kTmaPage * 128), &kvmap, full(st), 0, c, kvh, 0, kpage);
          tma_load_5d(dst + S::PLANE + (uint32_t)c * (kTmaPage * 128), &kvmap, full(st), 0, c, kvh, 0, vpage);
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ consumers
    const int c = warp - 1;
    if (early) pdl_wait();  // q (and the new K/V rows) are the previous kernel's output
    // Q rows (bf16, zero padding rows) -- consumers share this work
    for (int i = tid - 32; i < 16 * (D / 8); i += 32 * NCONS) {
      const int r = i / (D / 8), cc = i % (D / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < nrows && ri.pos[r] >= 0) {
        const int gr = row0 + r, t = gr / G, g = gr % G;
        v = ld_act_v4(q + (((int64_t)b * T + t) * hq + kvh * G + g) * D + cc * 8);
      }
      *reinterpret_cast<uint4*>(qs + r * S::QST + cc * 8) = v;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(32 * NCONS) : "memory");
    const int rA = lane >> 2;
    const int prow = (rA < nrows) ? ri.pos[rA] : -1;
    float m_run = -INFINITY, l_run = 0.f;
    float oacc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) oacc[nt][e] = 0.f;
    const uint32_t qaddr0 = (uint32_t)__cvta_generic_to_shared(qs);
    const int lr = lane & 7, lm = lane >> 3;
    for (int j = c; j < npages; j += NCONS) {
      const int st = j % S::STAGES;
      if (!tmb_wait(full(st), (uint32_t)(j / S::STAGES) & 1u)) {
        s_abort = 1;
        atomicExch(err, 2u);
        break;
      }
      const uint32_t kbase = base + (uint32_t)st * S::STAGE, vbase = kbase + S::PLANE;
      const int t0 = k_begin + j * kTmaPage;
      const int valid = min(kTmaPage, k_end - t0);
      if (valid < kTmaPage) {
        // rows past the context: zero V (whole 128-byte lines, any swizzle)
        unsigned char* vg = gb + ((size_t)st * S::STAGE + S::PLANE);
        for (int i = lane; i < (kTmaPage - valid) * S::CHUNKS * 8; i += 32) {
          const int r = valid + i / (S::CHUNKS * 8), rest = i % (S::CHUNKS * 8), ch = rest / 8, u = rest % 8;
          *reinterpret_cast<uint4*>(vg + ch * (kTmaPage * 128) + r * 128 + u * 16) = make_uint4(0, 0, 0, 0);
        }
        __syncwarp();
      }
      // S = Q K^T (2 n-tiles of 8 positions)
      float sacc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sacc[nt][e] = 0.f;
#pragma unroll
      for (int ks_ = 0; ks_ < KSTEPS; ++ks_) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        ldsm_x4(qaddr0 + (uint32_t)((lr + 8 * (lm & 1)) * S::QST + 16 * ks_ + 8 * (lm >> 1)) * 2, a0, a1, a2, a3);
        ldsm_x4(kbase + sw_off(8 * (lm >> 1) + lr, 16 * ks_ + 8 * (lm & 1)), b0, b1, b2, b3);
        mma_bf16_16816(sacc[0], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(sacc[1], a0, a1, a2, a3, b2, b3);
      }
      // online softmax of row rA over this page (4 lanes share a row)
      float pa[2][2];
      float mp = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = t0 + nt * 8 + (lane & 3) * 2 + e;
          const bool ok = (key < k_end) && (key <= prow);
          pa[nt][e] = ok ? sacc[nt][e] * scale : -INFINITY;
          mp = fmaxf(mp, pa[nt][e]);
        }
      mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 1));
      mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 2));
      const float m_new = fmaxf(m_run, mp);
      const float alpha = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
      float lp = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pv = (m_new == -INFINITY || pa[nt][e] == -INFINITY) ? 0.f : expf(pa[nt][e] - m_new);
          pa[nt][e] = pv;
          lp += pv;
        }
      lp += __shfl_xor_sync(0xffffffffu, lp, 1);
      lp += __shfl_xor_sync(0xffffffffu, lp, 2);
      l_run = l_run * alpha + lp;
      m_run = m_new;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        oacc[nt][0] *= alpha;
        oacc[nt][1] *= alpha;
      }
      const uint32_t pa0 = pack_bf16(pa[0][0], pa[0][1]), pa2 = pack_bf16(pa[1][0], pa[1][1]);
      // O += P V
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + sw_off(8 * (lm & 1) + lr, 16 * np + 8 * (lm >> 1)), b0, b1, b2, b3);
        mma_bf16_16816(oacc[2 * np], pa0, 0u, pa2, 0u, b0, b1);
        mma_bf16_16816(oacc[2 * np + 1], pa0, 0u, pa2, 0u, b2, b3);
      }
      // stage free: generic writes (zeroing) before the next TMA fill of it
      if (valid < kTmaPage) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) tmb_arrive(empty(st));
    }
    // this consumer's state -> shared memory (after every consumer is done with the ring)
    asm volatile("bar.sync 1, %0;" ::"n"(32 * NCONS) : "memory");
    if ((lane & 3) == 0 && rA < kRows) mls[c * kRows + rA] = make_float2(m_run, l_run);
    float* ow = os + c * kRows * D;
    if (rA < nrows) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        ow[rA * D + nt * 8 + (lane & 3) * 2] = oacc[nt][0];
        ow[rA * D + nt * 8 + (lane & 3) * 2 + 1] = oacc[nt][1];
      }
    }
  }
  __syncthreads();
  if (s_abort) {
    // a bounded wait gave up (error recorded): let the copies still in flight land, then leave
    if (tid == 0)
      for (int j = max(0, issued - S::STAGES); j < issued; ++j) tmb_wait(full(j % S::STAGES), (uint32_t)(j / S::STAGES) & 1u);
    return;
  }

  // ---- combine the consumers in warp order
  const bool direct = (ns == 1);  // the group's context fits split 0, which writes the output
  const int64_t pbase = (grp_id * nsplit + split) * kRows;
  for (int i = tid; i < nrows * D; i += NTHREADS) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NCONS; ++w) M = fmaxf(M, mls[w * kRows + r].x);
    float O = 0.f, L = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NCONS; ++w) {
        const float2 ml = mls[w * kRows + r];
        const float wt = (ml.x == -INFINITY) ? 0.f : expf(ml.x - M);
        L += ml.y * wt;
        O += os[(w * kRows + r) * D + d] * wt;
      }
    }
    if (direct) {
      // one split: the fold would weight it by exp(0) = 1, so this is its result exactly
      const int gr = row0 + r, t = gr / G, g = gr % G;
      out[(((int64_t)b * T + t) * hq + kvh * G + g) * D + d] = from_f<bf16>((L > 0.f) ? O / L : 0.f);
    } else {
      ws_o[(pbase + r) * D + d] = O;
      if (d == 0) ws_ml[pbase + r] = make_float2(M, L);
    }
  }
  pdl_trigger();
  if (direct) return;
  // the ns splits that hold context take a ticket; the last one folds them in split order
  if (!last_block_of(&counters[grp_id], (unsigned)ns, &is_last)) return;
  attention_fold<bf16, D, kTmaChunk, NTHREADS>(ws_o, ws_ml, out, grp_id, nsplit, seq_len, nrows, row0, G, T, hq,
                                               kvh, b, os);
}

// ---------------------------------------------------------------- K2
template <typename KV>
__global__ void kv_write_kernel(KV* pages, int num_layers, int num_blocks, int block_size, int hkv,
                                int D, int layer, const int32_t* block_tables, int max_blocks,
                                const int32_t* positions, const KV* k,
                                const KV* v, int T) {
  pdl_wait();
  pdl_trigger();
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
__global__ void rope_kv_write_kernel(const KV* qkv, KV* q_out, KV* pages,
                                     int num_layers, int num_blocks, int block_size, int hq, int hkv, int D,
                                     int layer, const int32_t* block_tables, int max_blocks,
                                     const int32_t* positions, const float* cos_t,
                                     const float* sin_t, int rope_max_pos, int T) {
  pdl_wait();
  pdl_trigger();
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

// Workspace: ticket counters, an error word, split partials.  Sized for the
// 128-position splits of the CUDA-core / mma kernels, which covers the TMA
// kernel's 256-position splits too.
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
  L.off_o = kCounterBytes + 256;  // error word at kCounterBytes
  L.off_ml = L.off_o + align256(sizeof(float) * rows * D);
  L.total = L.off_ml + align256(sizeof(float2) * rows);
  return L;
}

template <int D>
int launch_attention_tc(cudaStream_t st, const void* q, const void* pages, int num_layers, int num_blocks,
                        int block_size, int hkv, int layer, const int32_t* tables, int max_blocks,
                        const int32_t* seq_lens, const int32_t* q_lens, void* out, float scale, int B, int T, int hq,
                        const AttnLayout& L, void* ws) {
  using S = TcSmem<D>;
  auto kern = paged_attention_tc_kernel<D>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::total) != cudaSuccess)
    return SSD_ERR_LAUNCH;
  char* w = reinterpret_cast<char*>(ws);
  dim3 grid(L.nsplit, hkv * L.row_groups, B);
  SSD_PDL(kern, grid, kAttnThreads, S::total, st, reinterpret_cast<const bf16*>(q),
          reinterpret_cast<const bf16*>(pages), num_layers, num_blocks, block_size, hkv, layer, tables, max_blocks,
          seq_lens, q_lens, reinterpret_cast<bf16*>(out), scale, T, hq, L.row_groups, L.nsplit,
          reinterpret_cast<float*>(w + L.off_o), reinterpret_cast<float2*>(w + L.off_ml),
          reinterpret_cast<unsigned int*>(w + L.off_cnt));
  return SSD_OK;
}

bool kv_map_cached(CUtensorMap* out, const void* pages, int plane_pages, int hkv, int D) {
  struct Key {
    const void* p;
    int n, h, d;
    bool operator==(const Key& o) const { return p == o.p && n == o.n && h == o.h && d == o.d; }
  };
  struct Hash {
    size_t operator()(const Key& k) const {
      return std::hash<const void*>()(k.p) ^ ((size_t)k.n * 0x9E3779B97F4A7C15ull) ^ ((size_t)k.h << 20) ^ (size_t)k.d;
    }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> cache;
  std::lock_guard<std::mutex> g(mu);
  const Key key{pages, plane_pages, hkv, D};
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  if (!make_kv_page_map(out, pages, plane_pages, kTmaPage, hkv, D)) return false;
  if (cache.size() > 1024) cache.clear();
  cache.emplace(key, *out);
  return true;
}

template <int D, int C>
int launch_attention_tma(cudaStream_t st, const void* q, const void* pages, int num_layers, int num_blocks, int hkv,
                         int layer, const int32_t* tables, int max_blocks, const int32_t* seq_lens,
                         const int32_t* q_lens, void* out, float scale, int B, int T, int hq, int max_seq_len,
                         const AttnLayout& L, void* ws, int early) {
  using S = TmaSmem<D, C>;
  CUtensorMap map;
  if (!kv_map_cached(&map, pages, 2 * num_layers * num_blocks, hkv, D)) return SSD_ERR_LAUNCH;
  auto kern = paged_attention_tma_kernel<D, C>;
  {
    // the shared-memory attribute belongs to each device's context: set it once per device
    static std::mutex mu;
    static uint64_t done = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SSD_ERR_LAUNCH;
    std::lock_guard<std::mutex> g(mu);
    if (!(done >> dev & 1ull)) {
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::total) != cudaSuccess) {
        (void)cudaGetLastError();
        return SSD_ERR_LAUNCH;
      }
      done |= 1ull << dev;
    }
  }
  char* w = reinterpret_cast<char*>(ws);
  const int nsplit = (max_seq_len + kTmaChunk - 1) / kTmaChunk;  // <= L.nsplit: fits the workspace
  dim3 grid(nsplit, hkv * L.row_groups, B);
  constexpr int threads = tma_threads<D, C>();
  SSD_PDL(kern, grid, threads, S::total, st, map, reinterpret_cast<const bf16*>(q), num_layers, num_blocks, hkv,
          layer, tables, max_blocks, seq_lens, q_lens, reinterpret_cast<bf16*>(out), scale, T, hq, L.row_groups,
          nsplit, reinterpret_cast<float*>(w + L.off_o), reinterpret_cast<float2*>(w + L.off_ml),
          reinterpret_cast<unsigned int*>(w + L.off_cnt), reinterpret_cast<unsigned int*>(w + kCounterBytes), early);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
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
  SSD_PDL(kern, grid, kAttnThreads, S::total, st, 
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
  return ssd::paged_verify_attention_impl(stream, q, pages, dtype, num_layers, num_blocks, block_size, num_kv_heads,
                                          head_dim, layer, block_tables, max_blocks, seq_lens, q_lens, out, scale, B,
                                          T, num_heads, max_seq_len, workspace, workspace_bytes, 0);
}

int ssd::paged_verify_attention_impl(ssd_stream_t stream, const void* q, const void* pages, int dtype,
                                     int num_layers, int num_blocks, int block_size, int num_kv_heads, int head_dim,
                                     int layer, const int32_t* block_tables, int max_blocks, const int32_t* seq_lens,
                                     const int32_t* q_lens, void* out, float scale, int B, int T, int num_heads,
                                     int max_seq_len, void* workspace, size_t workspace_bytes, int early) {
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
#define SSD_ATTN_TC(DD)                                                                                       \
  return launch_attention_tc<DD>(st, q, pages, num_layers, num_blocks, block_size, num_kv_heads, layer,        \
                                 block_tables, max_blocks, seq_lens, q_lens, out, scale, B, T, num_heads, L,  \
                                 workspace)
  const bool aligned16 = !(reinterpret_cast<uintptr_t>(q) & 15) && !(reinterpret_cast<uintptr_t>(pages) & 15);
#define SSD_ATTN_TMA_C(DD, CC)                                                                                  \
  return launch_attention_tma<DD, CC>(st, q, pages, num_layers, num_blocks, num_kv_heads, layer, block_tables,  \
                                      max_blocks, seq_lens, q_lens, out, scale, B, T, num_heads, max_seq_len, L, \
                                      workspace, early)
#define SSD_ATTN_TMA(DD) SSD_ATTN_TMA_C(DD, tma_consumers<DD>())
  if (dtype == SSD_DTYPE_BF16 && aligned16 && block_size == kTmaPage && (int64_t)2 * num_layers * num_blocks < (1ll << 31)) {
    if (head_dim == 256 && num_kv_heads <= 2) SSD_ATTN_TMA_C(256, kTmaWideConsumers);
    if (head_dim == 256) SSD_ATTN_TMA(256);
    if (head_dim == 128) SSD_ATTN_TMA(128);
    if (head_dim == 64) SSD_ATTN_TMA(64);
  }
#undef SSD_ATTN_TMA
#undef SSD_ATTN_TMA_C
  if (dtype == SSD_DTYPE_BF16 && aligned16) {
    if (head_dim == 256) SSD_ATTN_TC(256);
    if (head_dim == 128) SSD_ATTN_TC(128);
    if (head_dim == 64) SSD_ATTN_TC(64);
  }
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
#undef SSD_ATTN_TC
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
    SSD_PDL(kv_write_kernel<bf16>, grid, 256, 0, st, reinterpret_cast<bf16*>(pages), num_layers, num_blocks, block_size,
                                                num_kv_heads, head_dim, layer, block_tables, max_blocks, positions,
                                                reinterpret_cast<const bf16*>(k), reinterpret_cast<const bf16*>(v), T);
  else if (dtype == SSD_DTYPE_F32)
    SSD_PDL(kv_write_kernel<float>, grid, 256, 0, st, reinterpret_cast<float*>(pages), num_layers, num_blocks,
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
    SSD_PDL(rope_kv_write_kernel<bf16>, grid, threads, 0, st, 
        reinterpret_cast<const bf16*>(qkv), reinterpret_cast<bf16*>(q_out), reinterpret_cast<bf16*>(pages),
        num_layers, num_blocks, block_size, num_heads, num_kv_heads, head_dim, layer, block_tables, max_blocks,
        positions, rope_cos, rope_sin, rope_max_pos, T);
  else if (dtype == SSD_DTYPE_F32)
    SSD_PDL(rope_kv_write_kernel<float>, grid, threads, 0, st, 
        reinterpret_cast<const float*>(qkv), reinterpret_cast<float*>(q_out), reinterpret_cast<float*>(pages),
        num_layers, num_blocks, block_size, num_heads, num_kv_heads, head_dim, layer, block_tables, max_blocks,
        positions, rope_cos, rope_sin, rope_max_pos, T);
  else
    return SSD_ERR_INVALID;
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}
