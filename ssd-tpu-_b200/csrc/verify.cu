// K4: fused acceptance kernels — greedy verify, row argmax, rejection sampling
// with bonus / residual draw — plus the counter-based uniform / normal fills.
//
// Greedy follows jax_ssd/algorithm/verify.py:18-59; sampling follows
// verify.py:68-120 (see include/ssd_verify.h for the argument contract).
//
// All of these are HBM-bound vocabulary scans.  Each scan splits a row of V
// logits into `nchunks` slices so that the grid covers every SM several times;
// each CTA reduces its slice to a partial (argmax key, or max/sum-exp pair) in
// the workspace, and the last CTA of a group (atomic ticket, self-resetting)
// folds the partials in fixed chunk order, so results are deterministic.


#include "common.cuh"

namespace ssd {
namespace {

constexpr int kScanThreads = 256;
constexpr int kTargetCtas = 148 * 4;

inline int scan_chunks(int rows, int V) {
  if (rows <= 0 || V <= 0) return 1;
  int want = (kTargetCtas + rows - 1) / rows;
  int cap = (V + 2047) / 2048;  // at least 2K elements per CTA
  if (cap < 1) cap = 1;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return want;
}

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// The statistics pass of the sampling verify (one exp per element over 2K rows
// per sequence) is bound by instruction issue as much as by HBM: it gets twice
// the CTAs.  The residual and draw passes, over one row pair per sequence, keep
// scan_chunks (measured: twice the CTAs made both slower).
inline int sample_chunks(int rows, int V) {
  if (rows <= 0 || V <= 0) return 1;
  int want = (2 * kTargetCtas + rows - 1) / rows;
  int cap = (V + 1023) / 1024;  // at least 1K elements per CTA
  if (cap < 1) cap = 1;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return want;
}

// Chunk [lo, hi) of a row of V elements; bounds are multiples of 4 except the end.
__device__ __forceinline__ void chunk_bounds(int V, int nchunks, int c, int& lo, int& hi) {
  int per = (V + nchunks - 1) / nchunks;
  per = (per + 3) & ~3;
  lo = min(c * per, V);
  hi = min(lo + per, V);
}

// Thread-local first-occurrence argmax over x[lo:hi).
__device__ __forceinline__ void scan_argmax(const float* row, int lo, int hi, bool vec_ok,
                                            float& best, int& bidx) {
  best = -INFINITY;
  bidx = 0x7fffffff;
  if (vec_ok) {
    const int nv = (hi - lo) >> 2;
    const float4* p = reinterpret_cast<const float4*>(row + lo);
    int i = threadIdx.x;
    for (; i + 3 * kScanThreads < nv; i += 4 * kScanThreads) {
      float4 a[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = __ldcg(p + i + u * kScanThreads);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int base = lo + 4 * (i + u * kScanThreads);
        if (a[u].x > best) { best = a[u].x; bidx = base; }
        if (a[u].y > best) { best = a[u].y; bidx = base + 1; }
        if (a[u].z > best) { best = a[u].z; bidx = base + 2; }
        if (a[u].w > best) { best = a[u].w; bidx = base + 3; }
      }
    }
    for (; i < nv; i += kScanThreads) {
      float4 a = __ldcg(p + i);
      const int base = lo + 4 * i;
      if (a.x > best) { best = a.x; bidx = base; }
      if (a.y > best) { best = a.y; bidx = base + 1; }
      if (a.z > best) { best = a.z; bidx = base + 2; }
      if (a.w > best) { best = a.w; bidx = base + 3; }
    }
    for (int j = lo + 4 * nv + threadIdx.x; j < hi; j += kScanThreads) {
      float v = __ldcg(row + j);
      if (v > best) { best = v; bidx = j; }
    }
  } else {
    for (int j = lo + threadIdx.x; j < hi; j += kScanThreads) {
      float v = __ldcg(row + j);
      if (v > best) { best = v; bidx = j; }
    }
  }
}

__device__ __forceinline__ unsigned long long thread_key(float best, int bidx) {
  // A thread that saw no element contributes the minimum key.
  return bidx == 0x7fffffff ? 0ull : argmax_key(best, (uint32_t)bidx);
}

// ---------------------------------------------------------------- greedy
// grid (nchunks, rows); rows = B*(K+1) (verify) or rows (argmax_rows, K = 0).
// group = b for verify (all K+1 rows), row for argmax_rows.
__global__ void __launch_bounds__(kScanThreads)
greedy_scan_kernel(const float* x, int64_t ld, int V, int kp1, int nchunks,
                   bool vec_ok, unsigned int* counters,
                   unsigned long long* partial, const int32_t* spec,
                   int32_t* accept_until, int32_t* recovery,
                   uint8_t* mask, int32_t* target_tokens,
                   int32_t* argmax_out) {
  __shared__ unsigned long long red[32];
  __shared__ bool is_last;
  __shared__ int tt[64];
  __shared__ int s_spec[64];
  pdl_wait();
  const int row = blockIdx.y, c = blockIdx.x;
  const int group = row / kp1;
  // The drafted ids are read only by the group's last CTA, after the scan; every
  // CTA issues their load now, so it lands while the slice streams in.
  int my_spec = 0;
  if (!argmax_out && threadIdx.x < kp1) my_spec = __ldcg(spec + (int64_t)group * kp1 + threadIdx.x);
  int lo, hi;
  chunk_bounds(V, nchunks, c, lo, hi);
  float best;
  int bidx;
  scan_argmax(x + (int64_t)row * ld, lo, hi, vec_ok, best, bidx);
  unsigned long long key = block_reduce(thread_key(best, bidx), red, OpMax());
  if (threadIdx.x == 0) partial[(int64_t)row * nchunks + c] = key;
  pdl_trigger();

  if (!last_block_of(&counters[group], (unsigned)(kp1 * nchunks), &is_last)) return;

  // Fold the partials of every row of the group: one warp per row, all rows at
  // once (the max of (value, index) keys does not depend on the order).
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = warp; r < kp1; r += kScanThreads / 32) {
    unsigned long long k = 0ull;
    for (int i = lane; i < nchunks; i += 32) {
      const unsigned long long v = __ldcg(&partial[(int64_t)(group * kp1 + r) * nchunks + i]);
      k = v > k ? v : k;
    }
    k = warp_max_u64(k);
    if (lane == 0) tt[r] = k == 0ull ? 0 : (int)argmax_key_index(k);  // all-NaN row: token 0
  }
  if (threadIdx.x < kp1) s_spec[threadIdx.x] = my_spec;
  __syncthreads();
  if (threadIdx.x != 0) return;
  if (argmax_out) {  // argmax_rows: kp1 == 1
    argmax_out[group] = tt[0];
    return;
  }
  const int K = kp1 - 1;
  const int b = group;
  int acc = 0;
  while (acc < K && s_spec[acc + 1] == tt[acc]) ++acc;
  accept_until[b] = acc;
  recovery[b] = tt[acc];  // == tt[K] when every draft token is accepted
  if (mask) {
    mask[(int64_t)b * kp1] = 0;
    for (int j = 0; j < K; ++j) mask[(int64_t)b * kp1 + j + 1] = (j < acc) ? 1 : 0;
  }
  if (target_tokens)
    for (int j = 0; j < kp1; ++j) target_tokens[(int64_t)b * kp1 + j] = tt[j];
}

// ---------------------------------------------------------------- sampling
struct SampleDecision {
  int acc;        // accepted draft tokens
  int bonus;      // 1: all accepted, draw from softmax(lp[K]/Tp)
  int prow, qrow; // rows used for the final draw
  float mp, sp, mq, sq;  // softmax max / sum of those rows (temperature applied)
  float rsum;     // max(sum(residual), 1e-12)
  float pad[3];
};

// fp32 ops written out so the compiler cannot contract them into FMAs: the
// oracle evaluates the same expressions with separate roundings.
// x / T; at T = 1 the quotient is x exactly, so the division is skipped.
__device__ __forceinline__ float div_temp(float x, float temp) {
  return temp == 1.f ? x : __fdiv_rn(x, temp);
}
// The same for the per-element loops, with T = 1 known at compile time: a run-time
// test is compiled as a select that evaluates the division for every element anyway.
template <bool UNIT_T>
__device__ __forceinline__ float div_t(float x, float temp) {
  if constexpr (UNIT_T) {
    (void)temp;
    return x;
  } else {
    return __fdiv_rn(x, temp);
  }
}
__device__ __forceinline__ float prob_of(float logit, float temp, float m, float s) {
  return __fdiv_rn(expf(__fsub_rn(div_temp(logit, temp), m)), s);
}

// Pass 1: per-row (max, sum exp) of x/T for the rows the acceptance test reads,
// then (last CTA per sequence) the accept loop.  Rows per sequence: nP target
// rows (lp[off .. K]) followed by K draft rows (lq[0 .. K-1]).
// At T = 1 the pass fits 32 registers, so its 2 x 592 CTAs are resident in one wave
// (8 per SM); a general temperature keeps the compiler's choice.
template <bool UNIT_T>
__global__ void __launch_bounds__(kScanThreads, UNIT_T ? 8 : 1)
sample_stats_kernel(const float* lp, const float* lq, int K, int V,
                    int off, int nchunks, bool vec_ok, float tp, float tq,
                    unsigned int* counters, float2* part,
                    const int32_t* spec, const float* u_accept,
                    SampleDecision* dec) {
  __shared__ float redf[32];
  __shared__ bool is_last;
  __shared__ float2 stats[130];
  pdl_wait();
  const int nP = K + 1 - off, nR = nP + K;
  const int b = blockIdx.y / nR, r = blockIdx.y % nR;
  const bool is_p = r < nP;
  const float* row = is_p ? lp + ((int64_t)b * (K + 1) + off + r) * V
                          : lq + ((int64_t)b * K + (r - nP)) * V;
  const float temp = is_p ? tp : tq;
  int lo, hi;
  chunk_bounds(V, nchunks, blockIdx.x, lo, hi);
  // One pass, online per thread: (m, s) with s = sum exp(v - m), v = x / T.  The terms
  // use the __expf intrinsic (a few ulp; this pass is bound by instruction issue): s
  // is a sum of 10^5 terms whose order already differs from the oracle's, and the
  // accept test divides by it with an exact expf of its own 2K logits.
  // Sixteen loaded values at a time: their max moves m once (one rescale), then
  // each value adds exp(v - m) in four partial sums, without a branch per value.
  // A NaN logit is skipped (fmaxf ignores it, the select drops it) and a masked
  // (-inf) logit adds exp(-inf) = 0.
  float m = -INFINITY, s = 0.f;
  auto push = [&](float x) {
    const float v = div_t<UNIT_T>(x, temp);
    if (v > m) { s = (m == -INFINITY ? 0.f : s * expf(__fsub_rn(m, v))) + 1.f; m = v; }
    else if (v > -INFINITY) s += __expf(__fsub_rn(v, m));
  };
  if (vec_ok) {
    const int nv = (hi - lo) >> 2;
    const float4* p = reinterpret_cast<const float4*>(row + lo);
    int i = threadIdx.x;
    // four independent 16-byte loads in flight per thread before any exp
    for (; i + 3 * kScanThreads < nv; i += 4 * kScanThreads) {
      float v[16];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 a = __ldcg(p + i + u * kScanThreads);
        v[4 * u] = a.x; v[4 * u + 1] = a.y; v[4 * u + 2] = a.z; v[4 * u + 3] = a.w;
      }
      float lm = -INFINITY;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        v[e] = div_t<UNIT_T>(v[e], temp);
        lm = fmaxf(lm, v[e]);
      }
      if (lm > m) {
        s = (m == -INFINITY) ? 0.f : s * expf(__fsub_rn(m, lm));
        m = lm;
      }
      if (m != -INFINITY) {
        float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float ex = __expf(__fsub_rn(v[e], m));
          ps[e & 3] += (v[e] > -INFINITY) ? ex : 0.f;
        }
        s += (ps[0] + ps[1]) + (ps[2] + ps[3]);
      }
    }
    for (; i < nv; i += kScanThreads) {
      const float4 a = __ldcg(p + i);
      push(a.x); push(a.y); push(a.z); push(a.w);
    }
    for (int j = lo + 4 * nv + threadIdx.x; j < hi; j += kScanThreads) push(__ldcg(row + j));
  } else {
    for (int j = lo + threadIdx.x; j < hi; j += kScanThreads) push(__ldcg(row + j));
  }
  const float M = block_reduce(m, redf, OpMax());
  float sc = (m == -INFINITY) ? 0.f : s * expf(__fsub_rn(m, M));
  sc = block_reduce(sc, redf, OpSum());
  m = M;
  s = sc;
  if (threadIdx.x == 0) part[(int64_t)blockIdx.y * nchunks + blockIdx.x] = make_float2(m, s);
  pdl_trigger();

  if (!last_block_of(&counters[b], (unsigned)(nR * nchunks), &is_last)) return;
  // Fold chunk partials per row, one warp per row: M = max m_i, S = sum s_i * exp(m_i - M)
  // (lane-strided over the chunks, then a fixed xor tree: deterministic).
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int rr = warp; rr < nR; rr += kScanThreads / 32) {
      const float2* pr = part + (int64_t)(b * nR + rr) * nchunks;
      float M = -INFINITY;
      for (int i = lane; i < nchunks; i += 32) M = fmaxf(M, __ldcg(&pr[i].x));
      M = warp_max(M);
      float S = 0.f;
      for (int i = lane; i < nchunks; i += 32) {
        const float2 v = __ldcg(&pr[i]);
        if (v.y > 0.f) S += v.y * expf(v.x - M);
      }
      S = warp_sum(S);
      if (lane == 0) stats[rr] = make_float2(M, S);
    }
  }
  // the logits of the drafted tokens that the accept loop reads, all K in one go
  // (not one dependent round trip per position)
  __shared__ float s_xp[64], s_xq[64];
  __shared__ int s_tok_ok[64];
  for (int j = threadIdx.x; j < K; j += blockDim.x) {
    const int tok = spec[(int64_t)b * (K + 1) + j + 1];
    const bool ok = (unsigned)tok < (unsigned)V;  // not a token id: reject (never index with it)
    s_tok_ok[j] = ok ? 1 : 0;
    s_xp[j] = ok ? __ldcg(lp + ((int64_t)b * (K + 1) + j + off) * V + tok) : 0.f;
    s_xq[j] = ok ? __ldcg(lq + ((int64_t)b * K + j) * V + tok) : 0.f;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  int acc = 0;
  for (int j = 0; j < K; ++j) {
    if (!s_tok_ok[j]) break;
    const float2 pst = stats[j];  // target row j+off is stored at index j
    const float2 qst = stats[nP + j];
    const float pv = prob_of(s_xp[j], tp, pst.x, pst.y);
    const float qv = prob_of(s_xq[j], tq, qst.x, qst.y);
    const float ratio = fminf(1.0f, __fdiv_rn(pv, fmaxf(qv, 1e-12f)));
    if (u_accept[(int64_t)b * K + j] < ratio) ++acc; else break;
  }
  SampleDecision d;
  d.acc = acc;
  d.bonus = (acc == K) ? 1 : 0;
  d.prow = d.bonus ? K : acc + off;
  d.qrow = d.bonus ? 0 : acc;
  const float2 pst = stats[d.prow - off];
  d.mp = pst.x; d.sp = pst.y;
  if (!d.bonus) { const float2 q = stats[nP + acc]; d.mq = q.x; d.sq = q.y; } else { d.mq = 0.f; d.sq = 1.f; }
  d.rsum = 1.f;
  d.pad[0] = d.pad[1] = d.pad[2] = 0.f;
  dec[b] = d;
}

// Pass 2: residual mass sum_v max(p_v - x q_v, 0) (skipped for bonus rows), with
// p_v = e_v * (1 / s) where the oracle divides by s (the draw uses the same products).
template <bool UNIT_T>
__global__ void __launch_bounds__(kScanThreads)
sample_residual_kernel(const float* lp, const float* lq, int K, int V,
                       int nchunks, bool vec_ok, float tp, float tq, float sx, unsigned int* counters,
                       float* part, SampleDecision* dec) {
  __shared__ float redf[32];
  __shared__ bool is_last;
  pdl_wait();
  const int b = blockIdx.y;
  const SampleDecision d = dec[b];
  pdl_trigger();
  if (d.bonus) return;  // uniform over the group: no CTA touches the counter
  const float* prow = lp + ((int64_t)b * (K + 1) + d.prow) * V;
  const float* qrow = lq + ((int64_t)b * K + d.qrow) * V;
  int lo, hi;
  chunk_bounds(V, nchunks, blockIdx.x, lo, hi);
  float s = 0.f;
  // one reciprocal per row instead of a division per element (as in the draw pass)
  const float inv_sp = __frcp_rn(d.sp), inv_sq = __frcp_rn(d.sq);
  auto add = [&](float xp, float xq) {
    const float p = __fmul_rn(__expf(__fsub_rn(div_t<UNIT_T>(xp, tp), d.mp)), inv_sp);
    const float q = __fmul_rn(__expf(__fsub_rn(div_t<UNIT_T>(xq, tq), d.mq)), inv_sq);
    s += fmaxf(__fsub_rn(p, __fmul_rn(sx, q)), 0.f);
  };
  int j0 = lo;
  if (vec_ok) {
    // two float4 of each row (four 16-byte loads) in flight per thread
    const int nv = (hi - lo) >> 2;
    const float4* pp = reinterpret_cast<const float4*>(prow + lo);
    const float4* qq = reinterpret_cast<const float4*>(qrow + lo);
    int i = threadIdx.x;
    for (; i + kScanThreads < nv; i += 2 * kScanThreads) {
      const float4 a0 = __ldcg(pp + i), a1 = __ldcg(pp + i + kScanThreads);
      const float4 b0 = __ldcg(qq + i), b1 = __ldcg(qq + i + kScanThreads);
      add(a0.x, b0.x); add(a0.y, b0.y); add(a0.z, b0.z); add(a0.w, b0.w);
      add(a1.x, b1.x); add(a1.y, b1.y); add(a1.z, b1.z); add(a1.w, b1.w);
    }
    for (; i < nv; i += kScanThreads) {
      const float4 a0 = __ldcg(pp + i), b0 = __ldcg(qq + i);
      add(a0.x, b0.x); add(a0.y, b0.y); add(a0.z, b0.z); add(a0.w, b0.w);
    }
    j0 = lo + 4 * nv;
  }
  for (int j = j0 + threadIdx.x; j < hi; j += kScanThreads) add(__ldcg(prow + j), __ldcg(qrow + j));
  s = block_reduce(s, redf, OpSum());
  if (threadIdx.x == 0) part[(int64_t)b * nchunks + blockIdx.x] = s;
  if (!last_block_of(&counters[b], (unsigned)nchunks, &is_last)) return;
  // fold the chunk sums: every thread loads its share, then one fixed-order tree
  float tot = 0.f;
  for (int i = threadIdx.x; i < nchunks; i += kScanThreads) tot += __ldcg(&part[(int64_t)b * nchunks + i]);
  tot = block_reduce(tot, redf, OpSum());
  if (threadIdx.x == 0) dec[b].rsum = fmaxf(tot, 1e-12f);
}

// Pass 3: Gumbel-max categorical draw over log(r + 1e-12).
// The score of element j is log(r_j + 1e-12) + g_j with g_j = -log(-log u_j), the
// oracle's fp32 expression.  It is increasing in (r_j + 1e-12) / nl_j, nl_j = -log u_j,
// so a thread picks its best element by that ratio (compared by cross-multiplication:
// no division and one log per element) and evaluates the exact score for its best
// element only; threads and CTAs then compare exact scores.  The uniforms are an input
// of the call, not of the earlier passes: each thread takes -log u of its first 16
// elements before waiting for them.  r_j uses one reciprocal per row where the oracle
// divides (p = e / s, r = residual / sum): the choice can differ from the oracle's
// only where two scores agree to about the rounding of those products (a near-tie).
constexpr int kDrawPre = 4;  // float4 groups of uniforms a thread prepares before the wait
template <bool UNIT_T>
__global__ void __launch_bounds__(kScanThreads)
sample_draw_kernel(const float* lp, const float* lq,
                   const float* u_gumbel, int K, int V, int nchunks, bool vec_ok, float tp, float tq,
                   float sx, unsigned int* counters, unsigned long long* part,
                   const SampleDecision* dec, int32_t* accept_until,
                   int32_t* recovery, uint8_t* mask) {
  __shared__ unsigned long long red[32];
  __shared__ bool is_last;
  const int b = blockIdx.y;
  const float* urow = u_gumbel + (int64_t)b * V;
  int lo, hi;
  chunk_bounds(V, nchunks, blockIdx.x, lo, hi);
  const int nv = vec_ok ? (hi - lo) >> 2 : 0;
  const float4* uu = reinterpret_cast<const float4*>(urow + lo);
  float4 nlp[kDrawPre];  // -log u of this thread's first kDrawPre float4 groups
#pragma unroll
  for (int t = 0; t < kDrawPre; ++t) {
    const int i = threadIdx.x + t * kScanThreads;
    if (i < nv) {
      const float4 u = __ldcg(uu + i);
      nlp[t] = make_float4(-logf(u.x), -logf(u.y), -logf(u.z), -logf(u.w));
    }
  }
  pdl_wait();
  const SampleDecision d = dec[b];
  const float* prow = lp + ((int64_t)b * (K + 1) + d.prow) * V;
  const float* qrow = lq + ((int64_t)b * K + d.qrow) * V;
  const float inv_sp = __frcp_rn(d.sp), inv_sq = d.bonus ? 0.f : __frcp_rn(d.sq);
  const float inv_r = d.bonus ? 1.f : __frcp_rn(d.rsum);
  // best so far as the pair (num, nl): num = r + 1e-12 > 0, nl = -log u >= 0
  float bnum = 0.f, bnl = 1.f;
  int bidx = 0x7fffffff;
  // element j with its target logit xp, draft logit xq (unused for a bonus draw) and nl;
  // a thread visits its elements in increasing j, so ties keep the first index
  auto visit = [&](int j, float xp, float xq, float nl) {
    const float p = __fmul_rn(__expf(__fsub_rn(div_t<UNIT_T>(xp, tp), d.mp)), inv_sp);
    float r;
    if (d.bonus) {
      r = p;
    } else {
      const float q = __fmul_rn(__expf(__fsub_rn(div_t<UNIT_T>(xq, tq), d.mq)), inv_sq);
      r = __fmul_rn(fmaxf(__fsub_rn(p, __fmul_rn(sx, q)), 0.f), inv_r);
    }
    const float num = __fadd_rn(r, 1e-12f);
    // a candidate has a score above -inf that is not NaN: num not NaN, nl < inf (u > 0);
    // the first candidate is taken, a later one where num / nl > bnum / bnl, i.e.
    // num * bnl > bnum * nl (both sides finite: num <= 1 + 1e-12, nl < inf; nl = 0,
    // u = 1, is the oracle's +inf score, and the first of those stays)
    if (!(num == num) || !(nl < INFINITY)) return;
    if (bidx == 0x7fffffff || __fmul_rn(num, bnl) > __fmul_rn(bnum, nl)) {
      bnum = num;
      bnl = nl;
      bidx = j;
    }
  };
  int j0 = lo;
  if (vec_ok) {
    const float4* pp = reinterpret_cast<const float4*>(prow + lo);
    const float4* qq = reinterpret_cast<const float4*>(qrow + lo);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int t = 0; t < kDrawPre; ++t) {
      const int i = threadIdx.x + t * kScanThreads;
      if (i < nv) {
        const float4 a = __ldcg(pp + i);
        const float4 c = d.bonus ? zero : __ldcg(qq + i);
        const int j = lo + 4 * i;
        visit(j, a.x, c.x, nlp[t].x); visit(j + 1, a.y, c.y, nlp[t].y);
        visit(j + 2, a.z, c.z, nlp[t].z); visit(j + 3, a.w, c.w, nlp[t].w);
      }
    }
    for (int i = threadIdx.x + kDrawPre * kScanThreads; i < nv; i += kScanThreads) {
      const float4 a = __ldcg(pp + i);
      const float4 c = d.bonus ? zero : __ldcg(qq + i);
      const float4 u = __ldcg(uu + i);
      const int j = lo + 4 * i;
      visit(j, a.x, c.x, -logf(u.x)); visit(j + 1, a.y, c.y, -logf(u.y));
      visit(j + 2, a.z, c.z, -logf(u.z)); visit(j + 3, a.w, c.w, -logf(u.w));
    }
    j0 = lo + 4 * nv;
  }
  for (int j = j0 + threadIdx.x; j < hi; j += kScanThreads)
    visit(j, __ldcg(prow + j), d.bonus ? 0.f : __ldcg(qrow + j), -logf(__ldcg(urow + j)));
  // the exact score of this thread's best element: log(r + 1e-12) + (-log(-log u))
  const float best = bidx == 0x7fffffff ? -INFINITY : __fadd_rn(logf(bnum), -logf(bnl));
  unsigned long long key = block_reduce(thread_key(best, bidx), red, OpMax());
  if (threadIdx.x == 0) part[(int64_t)b * nchunks + blockIdx.x] = key;
  pdl_trigger();
  if (!last_block_of(&counters[b], (unsigned)nchunks, &is_last)) return;
  unsigned long long k = 0ull;
  for (int i = threadIdx.x; i < nchunks; i += kScanThreads) {
    const unsigned long long v = __ldcg(&part[(int64_t)b * nchunks + i]);
    k = v > k ? v : k;
  }
  k = block_reduce(k, red, OpMax());
  if (threadIdx.x == 0) {
    accept_until[b] = d.acc;
    recovery[b] = k == 0ull ? 0 : (int32_t)argmax_key_index(k);
    if (mask) {
      mask[(int64_t)b * (K + 1)] = 0;
      for (int j = 0; j < K; ++j) mask[(int64_t)b * (K + 1) + j + 1] = (j < d.acc) ? 1 : 0;
    }
  }
}

// ---------------------------------------------------------------- top-p (nucleus) mask
// One CTA per row.  The nucleus of softmax(x / T) at mass p is {x >= t*}, t* the
// largest logit value whose cumulative mass (all logits >= it, ties included)
// reaches p * Z.  Masses are fp64: w = exp(-(m - x) / T), m the row max.
//   1. m;
//   2. histogram of d = (m - x) / T over the near range [0, 8) nats in 2048 bins
//      of 1/256 nat; each mass is rounded to a multiple of 2^-44 and added with a
//      64-bit integer atomic (native in shared memory, order-independent, so the
//      bin sums are deterministic).  Logits further down only add to an fp64
//      register sum, so most of a row costs no atomic at all;
//   3. the cutoff bin: the first bin, walking down from the max, at which the
//      running mass reaches p * Z.  If the near range holds less than p * Z, a
//      second histogram covers [8, 40) nats in 1/64-nat bins the same way;
//   4. the cutoff bin's logits are compacted into shared memory and sorted
//      (descending); the walk continues through them to the exact t*;
//   5. every logit below t* (and every NaN) becomes -inf, in place.
// A cutoff beyond 40 nats (p within ~e^-40 * V / Z of 1) keeps every finite
// logit; a cutoff bin holding more than kTopPCap logits is kept whole.
constexpr int kTopPThreads = 1024;
constexpr int kTopPBins = 2048;
constexpr int kTopPCap = 4096;
constexpr double kTopPFix = 17592186044416.0;  // 2^44: V * 2^44 stays below 2^63 for V < 2^19
static_assert(kTopPBins == 2 * kTopPThreads, "the bin scan gives every thread two bins");

// ---- thread-block cluster helpers (distributed shared memory; all within one GPU)
__device__ __forceinline__ uint32_t tp_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// every thread of every CTA of the cluster: a hardware barrier, ordering shared-memory
// writes before it (release) with reads after it (acquire) across the cluster
__device__ __forceinline__ void tp_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
template <typename T>
__device__ __forceinline__ uint32_t tp_mapa(const T* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"((uint32_t)__cvta_generic_to_shared(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ unsigned long long tp_ld_u64(uint32_t a) {
  unsigned long long v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ double tp_ld_f64(uint32_t a) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ float tp_ld_f32(uint32_t a) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ int tp_ld_s32(uint32_t a) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}

// CL CTAs per row (a thread-block cluster when CL > 1): CTA r of the cluster streams
// the r-th contiguous part of the row.  The row max and the fp64 mass below the
// binned range are combined over the cluster in CTA order, every CTA sums the
// cluster's integer bin masses for its scan (exact, so each CTA finds the same
// cutoff bin), the first CTA gathers the cutoff bin's candidates from the others,
// sorts and walks them, and every CTA masks its part with the cutoff it publishes.
// With few rows (the draft rows of a batched decode) one CTA per row leaves most
// SMs idle; CL = 4 gives each row four.
template <int CL>
__global__ void __launch_bounds__(kTopPThreads)
top_p_mask_kernel(float* x, int64_t ld, int V, double inv_t, double top_p) {
  __shared__ unsigned long long massq[kTopPBins];  // bin masses in units of 2^-44; later candidate masses
  __shared__ float cand[kTopPCap];
  __shared__ float redf[32];
  __shared__ double redd[32];
  __shared__ unsigned long long wscan[32];
  __shared__ int s_bin, s_ncand, s_found;
  __shared__ double s_above;
  __shared__ float s_t;
  __shared__ float s_mx;     // CL > 1: this CTA's part of the row max
  __shared__ double s_below; // CL > 1: this CTA's part of the mass below the binned range
  pdl_wait();
  const uint32_t crank = CL > 1 ? tp_cluster_rank() : 0u;
  float* row = x + (int64_t)(blockIdx.x / CL) * ld;
  const int j_lo = (int)((int64_t)V * crank / CL), j_hi = (int)((int64_t)V * (crank + 1) / CL);
  float mloc = -INFINITY;
  for (int j = j_lo + threadIdx.x; j < j_hi; j += kTopPThreads) mloc = fmaxf(mloc, __ldcg(row + j));  // skips NaN
  float m = block_reduce(mloc, redf, OpMax());
  if constexpr (CL > 1) {
    if (threadIdx.x == 0) s_mx = m;
    tp_cluster_sync();
    for (int r = 0; r < CL; ++r) m = fmaxf(m, tp_ld_f32(tp_mapa(&s_mx, (uint32_t)r)));
    tp_cluster_sync();  // every CTA has read the others' parts (none exits before)
  }
  if (!(m > -INFINITY)) {  // no finite logit: nothing to rank (the same decision in every CTA)
    pdl_trigger();
    return;
  }
  const double md = (double)m;
  double lo = 0.0, scale = 256.0;  // level 0: [0, 8) nats, 256 bins per nat
  double above = 0.0;              // mass of the logits above the current range
  double target = 0.0;
  int b = -1;
  for (int level = 0; level < 2 && b < 0; ++level) {
    if (level == 1) {
      lo = 8.0;
      scale = 64.0;  // [8, 40) nats
    }
    const double hi = lo + kTopPBins / scale;
    for (int i = threadIdx.x; i < kTopPBins; i += kTopPThreads) massq[i] = 0ull;
    __syncthreads();
    double below = 0.0;  // mass of the logits below the range (fp64, per thread)
    for (int j = j_lo + threadIdx.x; j < j_hi; j += kTopPThreads) {
      const float v = __ldcg(row + j);
      if (!(v > -INFINITY)) continue;  // -inf and NaN carry no mass
      const double d = (md - (double)v) * inv_t;
      if (d < lo) continue;  // counted at the previous level
      const double w = exp(-d);
      if (d < hi) atomicAdd(&massq[(int)((d - lo) * scale)], (unsigned long long)__double2ll_rn(w * kTopPFix));
      else below += w;
    }
    below = block_reduce(below, redd, OpSum());
    // Inclusive prefix sums of the integer bin masses (exact, so any order gives the same
    // sums): thread i owns bins 2i and 2i + 1.  The cutoff bin is the first whose prefix
    // reaches the target -- the same test, on the same sums, as a walk down the bins.
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int b0i = 2 * threadIdx.x;
    unsigned long long q0 = massq[b0i], q1 = massq[b0i + 1];
    if constexpr (CL > 1) {
      // the cluster's bins (integer sums: any order, the same in every CTA) and the
      // mass below (fp64, summed in CTA order)
      if (threadIdx.x == 0) s_below = below;
      tp_cluster_sync();
      q0 = q1 = 0ull;
      below = 0.0;
      for (int r = 0; r < CL; ++r) {
        q0 += tp_ld_u64(tp_mapa(&massq[b0i], (uint32_t)r));
        q1 += tp_ld_u64(tp_mapa(&massq[b0i + 1], (uint32_t)r));
        below += tp_ld_f64(tp_mapa(&s_below, (uint32_t)r));
      }
      tp_cluster_sync();  // the histograms are read before any CTA clears or reuses them
    }
    unsigned long long incl = q0 + q1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) wscan[wid] = incl;
    if (threadIdx.x == 0) s_bin = kTopPBins;
    __syncthreads();
    if (wid == 0) {
      unsigned long long v = wscan[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      wscan[lane] = v;
    }
    __syncthreads();
    const unsigned long long excl = (wid > 0 ? wscan[wid - 1] : 0ull) + incl - (q0 + q1);  // bins < 2i
    const unsigned long long inq = wscan[31];
    const double in_range = (double)inq / kTopPFix;
    if (level == 0) target = top_p * (in_range + below);
    int mine = kTopPBins;
    if (above + (double)(excl + q0) / kTopPFix >= target) mine = b0i;
    else if (above + (double)(excl + q0 + q1) / kTopPFix >= target) mine = b0i + 1;
    if (mine < kTopPBins) atomicMin(&s_bin, mine);
    __syncthreads();
    const int bb = s_bin;
    if (bb < kTopPBins && bb == mine) s_above = above + (double)(mine == b0i ? excl : excl + q0) / kTopPFix;
    __syncthreads();
    if (bb < kTopPBins) {
      b = bb;
      above = s_above;
    } else {
      above += in_range;  // cutoff below this range
    }
    __syncthreads();  // s_bin and s_above are rewritten at the next level
  }
  if (threadIdx.x == 0) s_t = -INFINITY;  // cutoff below both ranges: keep every finite logit
  if (b >= 0) {
    if (threadIdx.x == 0) s_ncand = 0;
    __syncthreads();
    for (int j = j_lo + threadIdx.x; j < j_hi; j += kTopPThreads) {
      const float v = __ldcg(row + j);
      if (!(v > -INFINITY)) continue;
      const double d = (md - (double)v) * inv_t;
      if (d >= lo && (int)((d - lo) * scale) == b) {
        const int k = atomicAdd(&s_ncand, 1);
        if (k < kTopPCap) cand[k] = v;
      }
    }
    __syncthreads();
    unsigned int n = (unsigned int)s_ncand;
    if constexpr (CL > 1) {
      // the first CTA appends the others' candidates (their order does not matter: sorted next)
      tp_cluster_sync();
      if (crank == 0) {
        unsigned int off = min(n, (unsigned int)kTopPCap);
        for (int r = 1; r < CL; ++r) {
          const unsigned int nr = (unsigned int)tp_ld_s32(tp_mapa(&s_ncand, (uint32_t)r));
          for (unsigned int i = threadIdx.x; i < nr && off + i < (unsigned)kTopPCap; i += kTopPThreads)
            cand[off + i] = tp_ld_f32(tp_mapa(&cand[i], (uint32_t)r));
          n += nr;
          off = min(off + nr, (unsigned int)kTopPCap);
        }
      }
      tp_cluster_sync();  // the others' candidates have been read
    }
    if (CL == 1 || crank == 0) {
      if (n > (unsigned)kTopPCap) {
        // too many logits near the cutoff to sort here: keep the whole bin
        if (threadIdx.x == 0) s_t = (float)(md - (lo + (double)(b + 1) / scale) / inv_t);
      } else {
        int np2 = 1;
        while (np2 < (int)n) np2 <<= 1;
        for (int i = (int)n + threadIdx.x; i < np2; i += kTopPThreads) cand[i] = -INFINITY;
        __syncthreads();
        // bitonic sort, descending
        for (int size = 2; size <= np2; size <<= 1) {
          for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < np2; i += kTopPThreads) {
              const int jx = i ^ stride;
              if (jx > i) {
                const bool desc = (i & size) == 0;
                const float a = cand[i], c = cand[jx];
                if (desc ? (a < c) : (a > c)) {
                  cand[i] = c;
                  cand[jx] = a;
                }
              }
            }
            __syncthreads();
          }
        }
        // Walk down the sorted candidates until the running mass reaches the target: the masses
        // are computed by all threads (kTopPBins at a time, into the histogram's storage), the
        // running sum stays one thread's sequential fp64 sum, in candidate order.
        double* wv = reinterpret_cast<double*>(massq);
        double cum = above;  // thread 0's running mass
        if (threadIdx.x == 0) {
          s_found = 0;
          s_t = n > 0 ? cand[n - 1] : -INFINITY;
        }
        for (unsigned int base = 0; base < n; base += kTopPBins) {
          __syncthreads();  // the previous part has been walked (and s_found set)
          if (s_found) break;
          const unsigned int cnt = min(n - base, (unsigned int)kTopPBins);
          for (unsigned int i = threadIdx.x; i < cnt; i += kTopPThreads)
            wv[i] = exp(-(md - (double)cand[base + i]) * inv_t);
          __syncthreads();
          if (threadIdx.x == 0) {
            for (unsigned int i = 0; i < cnt; ++i) {
              cum += wv[i];
              if (cum >= target) {
                s_t = cand[base + i];
                s_found = 1;
                break;
              }
            }
          }
        }
      }
    }
  }
  __syncthreads();
  float t = s_t;
  if constexpr (CL > 1) {
    tp_cluster_sync();  // the first CTA's cutoff is published
    t = tp_ld_f32(tp_mapa(&s_t, 0u));
  }
  for (int j = j_lo + threadIdx.x; j < j_hi; j += kTopPThreads) {
    const float v = __ldcg(row + j);
    if (!(v >= t)) row[j] = -INFINITY;
  }
  if constexpr (CL > 1) tp_cluster_sync();  // no CTA leaves while another may still read its shared memory
  pdl_trigger();
}

// ---------------------------------------------------------------- RNG fills
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  // SplitMix64 finaliser (Steele, Lea, Flood 2014).
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float hash_uniform(uint64_t seed, uint64_t i) {
  const uint64_t h = mix64(seed ^ mix64(i));
  return ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0,1), 24-bit grid
}

// ---------------------------------------------------------------- row sampling
// token[r] = argmax_j (x[r][j] / T + G[r][j]), G = -log(-log(u)), u from the
// counter hash at (seed, offset + r * V + j): a draw from softmax(x[r] / T)
// (Gumbel-max), with no noise buffer in HBM.  Same chunked scan and ordered
// fold as the greedy kernels, so a row's draw is deterministic for a seed.
__global__ void __launch_bounds__(kScanThreads)
sample_rows_kernel(const float* x, int64_t ld, int V, int nchunks, float inv_t, uint64_t seed, uint64_t offset,
                   unsigned int* counters, unsigned long long* partial, int32_t* out) {
  __shared__ unsigned long long red[32];
  __shared__ bool is_last;
  pdl_wait();
  const int row = blockIdx.y, c = blockIdx.x;
  int lo, hi;
  chunk_bounds(V, nchunks, c, lo, hi);
  const float* xr = x + (int64_t)row * ld;
  const uint64_t base = offset + (uint64_t)row * (uint64_t)V;
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int j = lo + threadIdx.x; j < hi; j += kScanThreads) {
    const float u = hash_uniform(seed, base + (uint64_t)j);
    const float v = __ldcg(xr + j) * inv_t - logf(-logf(u));
    if (v > best) {
      best = v;
      bidx = j;
    }
  }
  unsigned long long key = block_reduce(thread_key(best, bidx), red, OpMax());
  if (threadIdx.x == 0) partial[(int64_t)row * nchunks + c] = key;
  pdl_trigger();
  if (!last_block_of(&counters[row], (unsigned)nchunks, &is_last)) return;
  unsigned long long k = 0ull;
  for (int i = threadIdx.x; i < nchunks; i += blockDim.x) {
    const unsigned long long v = __ldcg(&partial[(int64_t)row * nchunks + i]);
    k = v > k ? v : k;
  }
  k = block_reduce(k, red, OpMax());
  // no finite candidate in the row (all logits NaN): emit token 0 rather than an invalid id
  if (threadIdx.x == 0) out[row] = k == 0ull ? 0 : (int32_t)argmax_key_index(k);
}

__global__ void uniform_fill_kernel(float* out, int64_t n, uint64_t seed, uint64_t offset) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = hash_uniform(seed, offset + (uint64_t)i);
}

template <typename T>
__global__ void normal_fill_kernel(T* out, int64_t n, float std, uint64_t seed) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float u1 = hash_uniform(seed, 2 * (uint64_t)i);
    const float u2 = hash_uniform(seed, 2 * (uint64_t)i + 1);
    const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);  // Box-Muller
    out[i] = from_f<T>(z * std);
  }
}

}  // namespace
}  // namespace ssd

using namespace ssd;

// ------------------------------------------------------------------ C ABI
extern "C" size_t ssd_verify_greedy_workspace_size(int B, int K, int V) {
  if (B <= 0 || K < 0 || V <= 0) return 0;
  const int rows = B * (K + 1);
  const int nch = scan_chunks(rows, V);
  return kCounterBytes + sizeof(unsigned long long) * (size_t)rows * nch;
}

static int launch_greedy(cudaStream_t st, const float* x, int64_t ld, int rows, int kp1, int V,
                         const int32_t* spec, int32_t* acc, int32_t* rec, uint8_t* mask, int32_t* tt,
                         int32_t* amax, void* ws, size_t ws_bytes) {
  const int nch = scan_chunks(rows, V);
  const size_t need = kCounterBytes + sizeof(unsigned long long) * (size_t)rows * nch;
  if (ws_bytes < need || ws == nullptr) return SSD_ERR_WORKSPACE;
  if (rows > kCounterCap) return SSD_ERR_UNSUPPORTED;
  unsigned int* counters = reinterpret_cast<unsigned int*>(ws);
  unsigned long long* part = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(ws) + kCounterBytes);
  const bool vec_ok = (ld % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  dim3 grid(nch, rows);
  SSD_PDL(greedy_scan_kernel, grid, kScanThreads, 0, st, x, ld, V, kp1, nch, vec_ok, counters, part, spec, acc,
                                                     rec, mask, tt, amax);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

extern "C" int ssd_verify_greedy(ssd_stream_t stream, const float* logits_p, const int32_t* speculations,
                                 int32_t* accept_until, int32_t* recovery, uint8_t* accepted_mask,
                                 int32_t* target_tokens, void* workspace, size_t workspace_bytes, int B,
                                 int K, int V) {
  if (B <= 0 || K < 0 || K > 63 || V <= 0 || !logits_p || !speculations || !accept_until || !recovery)
    return SSD_ERR_INVALID;
  if ((int64_t)B * (K + 1) > 65535) return SSD_ERR_UNSUPPORTED;
  return launch_greedy((cudaStream_t)stream, logits_p, V, B * (K + 1), K + 1, V, speculations, accept_until,
                       recovery, accepted_mask, target_tokens, nullptr, workspace, workspace_bytes);
}

// ------------------------------------------------------------------ no-allocation variant
// Greedy acceptance for callers that cannot allocate device memory (an XLA
// custom call that is handed only its operands and no allocator, embedders
// with a fixed device-memory budget).  Its scratch -- the
// ticket counters and the per-chunk argmax partials -- lives in this file-scope
// device array instead of a caller workspace.  Every GPU that loads the library
// holds these 34 KB until the process exits.  Host code must not use the array's
// name as a pointer (on the host it is only a stand-in); the device address comes
// from cudaGetSymbolAddress, looked up on every call with the caller's device
// current (a cheap runtime query), so no stale address outlives a device reset.
constexpr int kNoAllocMaxRows = 512;       // B * (K + 1)
constexpr int kNoAllocMaxPartials = 4096;  // rows * chunks (at most 592 + rows in practice)
constexpr size_t kNoAllocCounterBytes = sizeof(unsigned int) * kNoAllocMaxRows;
static __device__ __align__(256) unsigned char g_greedy_scratch[kNoAllocCounterBytes +
                                                                sizeof(unsigned long long) * kNoAllocMaxPartials];

// Device address of g_greedy_scratch on the current device.
static int greedy_scratch_address(void** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_greedy_scratch) != cudaSuccess || p == nullptr) {
    (void)cudaGetLastError();
    return SSD_ERR_LAUNCH;
  }
  *out = p;
  return SSD_OK;
}

extern "C" int ssd_verify_greedy_noalloc(ssd_stream_t stream, const float* logits_p, const int32_t* speculations,
                                         int32_t* accept_until, int32_t* recovery, uint8_t* accepted_mask,
                                         int32_t* target_tokens, int B, int K, int V) {
  if (B <= 0 || K < 0 || K > 63 || V <= 0 || !logits_p || !speculations || !accept_until || !recovery)
    return SSD_ERR_INVALID;
  const int64_t rows = (int64_t)B * (K + 1);
  if (rows > kNoAllocMaxRows) return SSD_ERR_UNSUPPORTED;
  const int nch = scan_chunks((int)rows, V);
  if (rows * nch > kNoAllocMaxPartials) return SSD_ERR_UNSUPPORTED;
  void* base = nullptr;
  const int rc = greedy_scratch_address(&base);
  if (rc != SSD_OK) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  // the counters must start at zero whatever an earlier (possibly aborted) call left behind
  if (cudaMemsetAsync(base, 0, kNoAllocCounterBytes, st) != cudaSuccess) return SSD_ERR_LAUNCH;
  unsigned int* counters = reinterpret_cast<unsigned int*>(base);
  unsigned long long* part =
      reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(base) + kNoAllocCounterBytes);
  const bool vec_ok = (V % 4 == 0) && ((reinterpret_cast<uintptr_t>(logits_p) & 15) == 0);
  SSD_PDL(greedy_scan_kernel, dim3(nch, (unsigned)rows), kScanThreads, 0, st, logits_p, V, V, K + 1, nch, vec_ok, counters,
                                                                         part, speculations, accept_until, recovery,
                                                                         accepted_mask, target_tokens, nullptr);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

extern "C" int ssd_argmax_rows(ssd_stream_t stream, const float* x, int64_t ld, int rows, int V, int32_t* out,
                               void* workspace, size_t workspace_bytes) {
  if (rows <= 0 || rows > 65535 || V <= 0 || ld < V || !x || !out) return SSD_ERR_INVALID;
  return launch_greedy((cudaStream_t)stream, x, ld, rows, 1, V, nullptr, nullptr, nullptr, nullptr, nullptr, out,
                       workspace, workspace_bytes);
}

extern "C" int ssd_sample_rows(ssd_stream_t stream, const float* x, int64_t ld, int rows, int V, float temperature,
                               uint64_t seed, uint64_t offset, int32_t* out, void* workspace,
                               size_t workspace_bytes) {
  if (rows <= 0 || rows > 65535 || V <= 0 || ld < V || !x || !out || !(temperature > 0.f)) return SSD_ERR_INVALID;
  const int nch = scan_chunks(rows, V);
  const size_t need = kCounterBytes + sizeof(unsigned long long) * (size_t)rows * nch;
  if (!workspace || workspace_bytes < need) return SSD_ERR_WORKSPACE;
  if (rows > kCounterCap) return SSD_ERR_UNSUPPORTED;
  unsigned int* counters = reinterpret_cast<unsigned int*>(workspace);
  unsigned long long* part =
      reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(workspace) + kCounterBytes);
  cudaStream_t st = (cudaStream_t)stream;
  SSD_PDL(sample_rows_kernel, dim3(nch, rows), kScanThreads, 0, st, x, ld, V, nch, 1.0f / temperature, seed, offset,
          counters, part, out);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

extern "C" int ssd_top_p_mask(ssd_stream_t stream, float* x, int64_t ld, int rows, int V, float temperature,
                              float top_p) {
  if (rows <= 0 || V <= 0 || ld < V || !x || !(temperature > 0.f) || !(top_p > 0.f)) return SSD_ERR_INVALID;
  if (top_p >= 1.0f) return SSD_OK;  // the whole distribution
  if (V >= (1 << 19)) return SSD_ERR_UNSUPPORTED;  // fixed-point bin masses would overflow
  cudaStream_t st = (cudaStream_t)stream;
  const double inv_t = 1.0 / (double)temperature, p = (double)top_p;
  if (rows <= 74) {  // up to half the SMs' worth of rows: four CTAs per row
    if (launch_pdl_cluster(top_p_mask_kernel<4>, dim3(rows * 4), dim3(kTopPThreads), 0, st, 4u, x, ld, V, inv_t, p) !=
        cudaSuccess) {
      (void)cudaGetLastError();
      return SSD_ERR_LAUNCH;
    }
    return SSD_OK;
  }
  SSD_PDL(top_p_mask_kernel<1>, dim3(rows), kTopPThreads, 0, st, x, ld, V, inv_t, p);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

static void sample_layout(int B, int K, int V, int& nR, int& nch, size_t& off_part, size_t& off_dec,
                          size_t& total) {
  nR = 2 * K + 1;  // upper bound over both alignments
  nch = sample_chunks(B * nR, V);
  // the residual and draw passes scan B rows: give them the same chunk count
  off_part = kCounterBytes;
  const size_t p1 = sizeof(float2) * (size_t)B * nR * nch;
  const size_t p2 = sizeof(unsigned long long) * (size_t)B * scan_chunks(B, V);
  off_dec = off_part + align256(p1 > p2 ? p1 : p2);
  total = off_dec + align256(sizeof(SampleDecision) * (size_t)B);
}

extern "C" size_t ssd_verify_sample_workspace_size(int B, int K, int V) {
  if (B <= 0 || K < 0 || V <= 0) return 0;
  int nR, nch;
  size_t a, b, t;
  sample_layout(B, K, V, nR, nch, a, b, t);
  return t;
}

extern "C" int ssd_verify_sample(ssd_stream_t stream, const float* logits_p, const float* logits_q,
                                 const int32_t* speculations, const float* u_accept, const float* u_gumbel,
                                 float temperature_p, float temperature_q, float sampler_x, int alignment,
                                 int32_t* accept_until, int32_t* recovery, uint8_t* accepted_mask,
                                 void* workspace, size_t workspace_bytes, int B, int K, int V) {
  if (B <= 0 || K < 0 || K > 63 || V <= 0 || !logits_p || !speculations || !u_gumbel || !accept_until ||
      !recovery)
    return SSD_ERR_INVALID;
  if (K > 0 && (!logits_q || !u_accept)) return SSD_ERR_INVALID;
  if (!(temperature_p > 0.f) || !(temperature_q > 0.f)) return SSD_ERR_INVALID;
  if (alignment != SSD_ALIGN_REFERENCE && alignment != SSD_ALIGN_STANDARD) return SSD_ERR_INVALID;
  int nR, nch;
  size_t off_part, off_dec, total;
  sample_layout(B, K, V, nR, nch, off_part, off_dec, total);
  if (!workspace || workspace_bytes < total) return SSD_ERR_WORKSPACE;
  // K = 0 (verify.py:98-114 with k = 0): nothing to accept, so every row draws its
  // bonus token from softmax(lp[0] / Tp) -- the same under both alignments.  The
  // draft logits are never read for a bonus draw; the kernels still form a draft
  // row pointer, so they get the target rows instead of a possibly empty buffer.
  const int off = (alignment == SSD_ALIGN_REFERENCE && K > 0) ? 1 : 0;
  if (K == 0) logits_q = logits_p;
  const int rows = B * (2 * K + 1 - off);
  if (rows > 65535 || 3 * B > kCounterCap) return SSD_ERR_UNSUPPORTED;
  char* w = reinterpret_cast<char*>(workspace);
  unsigned int* c0 = reinterpret_cast<unsigned int*>(w);
  unsigned int* c1 = c0 + B;
  unsigned int* c2 = c1 + B;
  float2* part = reinterpret_cast<float2*>(w + off_part);
  SampleDecision* dec = reinterpret_cast<SampleDecision*>(w + off_dec);
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec_ok = (V % 4 == 0) && ((reinterpret_cast<uintptr_t>(logits_p) & 15) == 0) &&
                      ((reinterpret_cast<uintptr_t>(logits_q) & 15) == 0);
  const bool unit = temperature_p == 1.f && temperature_q == 1.f;
  SSD_PDL(unit ? sample_stats_kernel<true> : sample_stats_kernel<false>, dim3(nch, rows), kScanThreads, 0, st,
          logits_p, logits_q, K, V, off, nch, vec_ok, temperature_p, temperature_q, c0, part, speculations,
          u_accept, dec);
  SSD_CHECK_LAUNCH();
  const int nch_b = scan_chunks(B, V);
  const bool vec_b = vec_ok && ((reinterpret_cast<uintptr_t>(u_gumbel) & 15) == 0);
  SSD_PDL(unit ? sample_residual_kernel<true> : sample_residual_kernel<false>, dim3(nch_b, B), kScanThreads, 0, st,
          logits_p, logits_q, K, V, nch_b, vec_ok,
          temperature_p, temperature_q, sampler_x, c1, reinterpret_cast<float*>(part), dec);
  SSD_CHECK_LAUNCH();
  SSD_PDL(unit ? sample_draw_kernel<true> : sample_draw_kernel<false>, dim3(nch_b, B), kScanThreads, 0, st,
      logits_p, logits_q, u_gumbel, K, V, nch_b, vec_b, temperature_p, temperature_q, sampler_x, c2,
      reinterpret_cast<unsigned long long*>(part), dec, accept_until, recovery, accepted_mask);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

extern "C" int ssd_uniform_fill(ssd_stream_t stream, float* out, int64_t n, uint64_t seed, uint64_t offset) {
  if (n < 0 || (n > 0 && !out)) return SSD_ERR_INVALID;
  if (n == 0) return SSD_OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  SSD_PDL(uniform_fill_kernel, (unsigned)blocks, 256, 0, (cudaStream_t)stream, out, n, seed, offset);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

extern "C" int ssd_normal_fill(ssd_stream_t stream, void* out, int dtype, int64_t n, float std, uint64_t seed) {
  if (n < 0 || (n > 0 && !out)) return SSD_ERR_INVALID;
  if (n == 0) return SSD_OK;
  int64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == SSD_DTYPE_BF16)
    SSD_PDL(normal_fill_kernel<bf16>, (unsigned)blocks, 256, 0, st, reinterpret_cast<bf16*>(out), n, std, seed);
  else if (dtype == SSD_DTYPE_F32)
    SSD_PDL(normal_fill_kernel<float>, (unsigned)blocks, 256, 0, st, reinterpret_cast<float*>(out), n, std, seed);
  else
    return SSD_ERR_INVALID;
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}
