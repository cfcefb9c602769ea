// K3 on the 5th-generation tensor cores: y = epilogue(x[M,K] w[N,K]^T), bf16 in,
// fp32 accumulation in TMEM, for M <= 256 token rows.
//
// The verify forward is a weight stream (M = k+1 = 5 rows against every weight
// byte), so the kernel is built to keep HBM busy, not the tensor pipe:
//   * swap-AB: the weight tile is the UMMA A operand (M_mma = 128 weight rows),
//     the token rows are B (N_mma = MP = M rounded up to 16); D[128 x MP] fp32
//     lives in TMEM, double-buffered so one tile's epilogue overlaps the next
//     tile's loads;
//   * persistent stream-K: one CTA per SM walks a contiguous range of
//     (tile, 64-wide k-block) units, so every SM streams the same number of
//     weight bytes whatever N and K are;
//   * warp 0 issues TMA loads of 128x64 weight blocks and MPx64 token blocks
//     (SWIZZLE_128B, no multicast) into a STAGES-deep ring of shared memory;
//     warp 1 (one thread) issues tcgen05.mma and commits each stage back to the
//     producer; warps 2-5 read the accumulator with tcgen05.ld and run the fused
//     epilogue (store / fp32 store / residual add / GeGLU).
//   * a tile cut by a CTA boundary is finished by its last-arriving contributor
//     (atomic ticket), which sums the fp32 partials in CTA (= K) order, so the
//     result is deterministic and, because the unit split depends on (N, K) and
//     the SM count only, independent of M.
//   * shapes with at most as many tiles as SMs use a tile-split plan instead:
//     G CTAs per tile (up to two per SM), each one contiguous part of its k-blocks; for
//     M <= 16 they run as one thread-block cluster and fold in distributed
//     shared memory (see linear_tc_kernel's CLU parameter).
// Every mbarrier wait is bounded: on timeout the kernel records an error code,
// stops issuing work, drains what it issued and releases its TMEM.
//
// Tensor parallelism fuses the collective into the same kernel.  Every rank
// maps every other rank's symmetric heap (CUDA IPC over NVLink); the rank that
// finishes an output tile stores its values straight into the peers' heaps
// (plain stores, no TMA, no multicast), so tile i crosses NVLink while tile i+1
// is still being multiplied:
//   * all-reduce (row-parallel O / down): each value travels as one 64-bit word
//     (fp32 bits, delivery count) into a receive slot [parity][tile][source
//     rank][row][128]; the tile's owner on every rank polls the words of all
//     sources (data and tag arrive together: no flags, no fences), folds them
//     in rank order (so every rank holds bit-identical sums), adds the residual
//     and stores bf16;
//   * all-gather (vocab-parallel LM head): the fp32 logits columns land in the
//     same place of every rank's logits buffer, followed by one arrival flag
//     per peer and tile; the tile's owner waits for the peers' flags of that
//     tile, so the logits are complete when the kernel ends.
// Each rank counts, per output tile, the collectives it has finished (device
// memory, so CUDA-graph replays need no host state; every rank makes the same
// calls, so the counts agree).  A delivery of tile t carries the count as its
// flag value, and the all-reduce receive slots [parity][tile][source] alternate
// by the count's parity -- a rank can be at most one delivery of a tile ahead of
// another.  The tile's owner on every rank waits for all peers' deliveries of
// that tile, so a kernel ends only when all of its tiles have arrived.  Peer
// waits are bounded in time; on expiry the kernel records SSD_ERR_TIMEOUT in
// the control block and finishes without the missing data.
#include <cuda.h>

#include <mutex>
#include <unordered_map>

#include "linear.cuh"

namespace ssd {
namespace tc {

constexpr int BM = 128;       // weight rows per tile (UMMA M)
constexpr int BK = 64;        // bf16 per k-block: one 128-byte swizzle row
// warp 0 TMA, warp 1 MMA + TMEM owner, warps 2.. epilogue (Cfg<MP>::THREADS in all)
constexpr uint32_t kWaitLimit = 1u << 24;  // polls before a wait gives up (~seconds)

struct Params {
  void* y;
  const bf16* x;  // token rows (read directly only for the row norms)
  int rowscale;   // 1: scale row m of the result by rsqrt(mean(x[m]^2) + eps)
  float eps;
  const float* inv_g;  // rowscale with M > 16: the row scales, computed by row_inv_rms_kernel
  int epi, M, N, K;
  int KB;        // k-blocks per tile
  int U;         // total units = tiles * KB
  int base, rem; // units per CTA; the first `rem` CTAs take one more
  int G;         // tile-split plan: each tile's k-blocks cut into G parts, CTA c = tile * G + part (0: stream-K)
  float* part;   // [grid][2][ms / 4][BM][4] partial tiles: 4 rows of one column are 16 contiguous bytes,
                 // and a warp's 32 columns of those 4 rows 512 contiguous bytes
  int ms;        // M rounded up to 16
  unsigned int* counters;  // per tile (self-resetting)
  unsigned int* err;       // error word
  // fused collective (COLL_NONE: plain epilogue)
  int coll, rank, world, ldy, col_off, recv_rows, recv_tiles;
  int owner_fold;  // all-reduce over more than 16 rows: partials go to the tile's owner only (see coll_finish)
  char* heaps[kMaxTP];
  size_t ctrl_off, dst_off;
  RopeArgs rope;  // epi == kEpiRopeQkv
};

// First unit of CTA c.  Stream-K: contiguous ranges of base or base + 1 units.
// Tile-split: part j of a tile takes KB / G k-blocks, the first KB % G parts one
// more -- the same contiguous, K-ordered ranges, aligned to tiles.
__host__ __device__ inline int unit_begin(const Params& p, int c) {
  if (p.G) {
    const int tile = c / p.G, part = c - tile * p.G;
    const int b = p.KB / p.G, r = p.KB % p.G;
    return tile * p.KB + part * b + (part < r ? part : r);
  }
  return c * p.base + (c < p.rem ? c : p.rem);
}
__device__ inline int cta_of_unit(const Params& p, int u) {
  if (p.G) {
    const int tile = u / p.KB, kb = u - tile * p.KB;
    const int b = p.KB / p.G, r = p.KB % p.G, big = r * (b + 1);
    return tile * p.G + (kb < big ? kb / (b + 1) : r + (kb - big) / b);
  }
  const int big = p.rem * (p.base + 1);
  return u < big ? u / (p.base + 1) : p.rem + (u - big) / p.base;
}

__device__ __forceinline__ uint32_t smem_u32(const void* ptr) { return (uint32_t)__cvta_generic_to_shared(ptr); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
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

// Bounded wait.  Returns false when the CTA has been told to abort or when the
// poll budget runs out (then it raises the abort flag and records `code`).
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                             unsigned int* err, unsigned int code) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort_flag) return false;
  }
  *abort_flag = 1;
  atomicExch(err, code);
  return false;
}

// ---- thread-block cluster (distributed shared memory) helpers
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }
// the same shared-memory offset in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t mapa(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_dsmem(uint32_t caddr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(caddr) : "memory");
  return v;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t caddr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}
// bounded wait that acquires what other CTAs of the cluster released with their arrivals
__device__ __forceinline__ bool wait_cluster_bounded(uint32_t bar, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

// ---- cross-GPU signalling (system scope: the peers write over NVLink)
constexpr uint64_t kPeerWaitNs = 5000000000ull;  // a peer that is 5 s late is reported, not awaited
constexpr uint32_t kPeerWaitPolls = 1u << 27;

__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* a, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t* ctrl_of(const Params& p, int r) {
  return reinterpret_cast<uint32_t*>(p.heaps[r] + p.ctrl_off);
}
// arrival flag on rank `r` for (source rank, tile)
__device__ __forceinline__ uint32_t* flag_of(const Params& p, int r, int src, int tile) {
  return reinterpret_cast<uint32_t*>(p.heaps[r] + p.ctrl_off + kCtrlFlagsOffset) + ((size_t)src * kFlagTiles + tile);
}
// this rank's count of finished collectives for output tile `tile`
__device__ __forceinline__ uint32_t* tile_count_of(const Params& p, int tile) {
  return reinterpret_cast<uint32_t*>(p.heaps[p.rank] + p.ctrl_off + kCtrlCountersOffset) + tile;
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* a, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* a, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* a) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}
// Bounded wait for a flag another GPU writes; false on timeout.
__device__ bool wait_peer_flag(const uint32_t* f, uint32_t want) {
  if (ld_relaxed_sys(f) == want) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kPeerWaitPolls; ++i) {
    __nanosleep(32);
    if (ld_relaxed_sys(f) == want) return true;
    if ((i & 63u) == 63u && global_ns() - t0 > kPeerWaitNs) return false;
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 TMEM lanes x 16 fp32 columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: kind::f16, A = B = bf16, D = fp32, both K-major, M = 128, N = MP.
template <int MP>
__host__ __device__ constexpr uint32_t idesc_bf16() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(MP >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

template <int MP>
struct Cfg {
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = MP * BK * 2;
  static constexpr uint32_t STAGE = A_BYTES + B_BYTES;
  // MP <= 32: a ring small enough (<= 113 KB) that the next projection's CTA can
  // share the SM and prefetch its weights while this one drains (PDL).
  static constexpr int STAGES = MP <= 16 ? 6 : MP <= 32 ? 5 : MP <= 64 ? 8 : MP <= 128 ? 6 : 4;
  static constexpr uint32_t TMEM_COLS = 2 * MP < 32 ? 32 : 2 * MP;
  // barriers, TMEM slot and flags, row scales [256], RoPE row info [MP] (int + int64)
  static constexpr uint32_t BAR_BYTES = 8 * (2 * STAGES + 5) + 16 + 4 * 256 + 12 * MP;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE + BAR_BYTES;
  // Epilogue warps per TMEM lane quadrant.  The epilogue issues a few dozen dependent
  // instructions per output element; with one warp per scheduler nothing hides their
  // latency, so tiles of more than 16 token rows get two warps per quadrant (warps w and
  // w + 4 read the same TMEM lanes and take alternate 16-row chunks).  Up to 16 rows (one
  // chunk) stay at one: their CTAs are sized for two per SM, next to the next kernel's.
  static constexpr int REP = MP >= 32 ? 2 : 1;
  static constexpr int EPI = 128 * REP;  // epilogue threads
  static constexpr int THREADS = 64 + EPI;
};

template <int NT>
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory"); }

// kEpiRopeQkv: output (m, n) of the QKV projection with rotation-paired q/k rows;
// `pair` is the accumulator of row n ^ 1 (the other half of the rotation pair).
// Row m's table position (clamped) and the element offset of its K row in the
// pages (-1: no K/V write), computed once per CTA into shared memory.
__device__ __forceinline__ void rope_row_info(const RopeArgs& r, int m, int* pc, long long* off) {
  const int p = ld_act(r.pos + m);
  long long o = -1;
  if (p >= 0 && p / r.block_size < r.max_blocks) {
    const int blk = ld_act(r.tables + (int64_t)(m / r.T) * r.max_blocks + p / r.block_size);
    if ((unsigned)blk < (unsigned)r.num_blocks)
      o = (((long long)r.layer * r.num_blocks + blk) * r.block_size + p % r.block_size) * r.hkv * r.D;
  }
  pc[m] = p < 0 ? 0 : min(p, r.rope_max_pos - 1);
  off[m] = o;
}

__device__ __forceinline__ void rope_qkv_store(const RopeArgs& r, int m, int n, float acc, float pair, int pc,
                                               long long off) {
  const int D = r.D, half = D >> 1, qk = (r.hq + r.hkv) * D;
  if (n < qk) {
    const int h = n / D, rr = n - h * D, i = rr >> 1;
    const bool odd = rr & 1;
    // the stored (bf16) q/k values, as the separate RoPE step reads them
    const float self = store_round<bf16>(acc), other = store_round<bf16>(pair);
    const float x1 = odd ? other : self, x2 = odd ? self : other;
    const float c = __ldg(r.cos_t + (int64_t)pc * half + i), sn = __ldg(r.sin_t + (int64_t)pc * half + i);
    const float y = odd ? __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn)) : __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
    const int dim = i + (odd ? half : 0);
    if (h < r.hq) r.q_out[((int64_t)m * r.hq + h) * D + dim] = from_f<bf16>(y);
    else if (off >= 0) r.pages[off + (long long)(h - r.hq) * D + dim] = from_f<bf16>(y);
  } else if (off >= 0) {
    r.pages[r.plane + off + (n - qk)] = from_f<bf16>(acc);
  }
}

// The residual rows m0 .. m0+15 of output column n (SSD_EPI_RESIDUAL; zeros otherwise), loaded
// together before they are needed: a store loop that read each row's residual just before writing
// it paid one L2 round trip per row (it cannot hoist a load above a store to the same array).
// Every load is issued (rows past M and columns past N read a valid element instead and
// are discarded), so all 16 are in flight together.
__device__ __forceinline__ void load_residual16(const Params& p, int m0, int n, float* res) {
  if (p.epi != SSD_EPI_RESIDUAL) {
#pragma unroll
    for (int j = 0; j < 16; ++j) res[j] = 0.f;
    return;
  }
  const bf16* y = reinterpret_cast<const bf16*>(p.y) + min(n, p.N - 1);
  const int last = p.M - 1;
  uint16_t raw[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) raw[j] = __ldcg(reinterpret_cast<const unsigned short*>(y + (int64_t)min(m0 + j, last) * p.N));
#pragma unroll
  for (int j = 0; j < 16; ++j) res[j] = __bfloat162float(__ushort_as_bfloat16(raw[j]));
}

// every non-collective output store of the kernel; `res` is the prefetched residual (RESIDUAL)
template <bool ROPE>
__device__ __forceinline__ void store_out(const Params& p, int m, int n, float acc, float pair, float res,
                                          const int* rpc, const long long* roff) {
  if constexpr (ROPE) {
    rope_qkv_store(p.rope, m, n, acc, pair, rpc[m], roff[m]);
  } else if (p.epi == SSD_EPI_RESIDUAL) {
    reinterpret_cast<bf16*>(p.y)[(int64_t)m * p.N + n] = from_f<bf16>(__fadd_rn(res, store_round<bf16>(acc)));
  } else if (!(p.epi == SSD_EPI_GEGLU && (n & 1))) {
    epilogue_store<bf16>(p.epi, p.y, p.N, m, n, acc, pair);
  }
}

// rsqrt(mean(x^2) + eps) of one token row, by one warp: lanes stride K in 8-element
// vectors (lane l takes elements 8l .. 8l+7 of every 256), each lane sums its vectors
// in K order with fma, then an xor tree -- a fixed order, so every CTA and every M
// gets the same bits.  Eight vectors per lane are loaded before any is used (one L2
// round trip per 2048 elements of the row instead of one per 256).
__device__ __forceinline__ float row_inv_rms(const bf16* xr, int K, float eps, int lane) {
  constexpr int kBatch = 8;
  float acc = 0.f;
  for (int k0 = lane * 8; k0 < K; k0 += kBatch * 256) {
    uint4 buf[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) buf[i] = k0 + i * 256 < K ? ld_act_v4(xr + k0 + i * 256) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (k0 + i * 256 >= K) break;
      float f[8];
      unpack8(buf[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(f[e], f[e], acc);
    }
  }
  acc = warp_sum(acc);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)K), eps)));
}

// The row scales of M > 16 token rows, once per projection instead of once per CTA
// (every CTA needs all rows: at M = 224, K = 3072 that was 1.4 MB of reads per CTA
// and a chain of L2 round trips before its first store).  One warp per row.
__global__ void __launch_bounds__(128) row_inv_rms_kernel(const bf16* x, int M, int K, float eps, float* out) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (m >= M) return;
  const float r = row_inv_rms(x + (size_t)m * K, K, eps, lane);
  if (lane == 0) out[m] = r;
}

// COLL: instantiate the fused-collective epilogue (p.coll != COLL_NONE); the
// plain projection is compiled without it so that its code stays small.
// CLU: launched as clusters of p.G CTAs over the tile-split plan (one tile per
// cluster, one segment per CTA).  The parts of a tile meet in distributed
// shared memory instead of the global partial buffer: every non-leader leaves
// its fp32 partial in its own (idle) ring and arrives on the leader's mbarrier;
// the leader folds its own accumulator and the peers' partials in part (= K)
// order -- the same sums as the global fold, with no ticket and no L2 round trips.
// ROPE: the QKV projection's epilogue applies RoPE and writes the K/V rows
// (epi == kEpiRopeQkv); its own instantiation, so the plain kernels stay small.
// The collective and RoPE instantiations declare one resident CTA per SM as the
// minimum (two still fit): without it ptxas held them to 96 registers and spilled.
template <int MP, bool COLL, bool CLU, bool ROPE>
__global__ void __launch_bounds__(Cfg<MP>::THREADS, (COLL || ROPE) ? 1 : 0)
linear_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                 const Params p) {
  using C = Cfg<MP>;
  constexpr int S = C::STAGES;
  constexpr int REP = C::REP, EPI = C::EPI;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + S * C::STAGE;
  auto full = [&](int s) { return bars + 8u * s; };
  auto empty = [&](int s) { return bars + 8u * (S + s); };
  auto accf = [&](int b) { return bars + 8u * (2 * S + b); };
  auto acce = [&](int b) { return bars + 8u * (2 * S + 2 + b); };
  const uint32_t red_bar = bars + 8u * (2 * S + 4);  // CLU: the non-leaders' partials are ready
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + S * C::STAGE + 8 * (2 * S + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_slot + 2);
  float* inv_s = reinterpret_cast<float*>(tmem_slot + 4);  // [M] row scales
  int* rope_pc = reinterpret_cast<int*>(inv_s + 256);      // ROPE: [MP] positions, then [MP] K-row offsets
  long long* rope_off = reinterpret_cast<long long*>(rope_pc + MP);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const int u0 = unit_begin(p, cta), u1 = unit_begin(p, cta + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf(b), 1);
      mbar_init(acce(b), EPI);
    }
    if (CLU) mbar_init(red_bar, (uint32_t)(p.G - 1));
    *abort_flag = 0;
    *last_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // CLU: split-phase cluster barrier -- arrive now, wait before the first remote
  // access, so that the peers' mbarrier inits are visible by then.
  if (CLU) cluster_arrive();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&wmap) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&xmap) : "memory");
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      // Weights never depend on the previous kernel: start streaming the first
      // ring's worth of weight blocks before waiting for it (PDL), then add the
      // token blocks of those stages once its outputs are visible.
      const int pre = min(S, u1 - u0);
      for (int i = 0; i < pre; ++i) {
        const int u = u0 + i, tile = u / p.KB, kb = u - tile * p.KB;
        mbar_expect_tx(full(i), C::STAGE);
        tma_load_2d(base + i * C::STAGE, &wmap, full(i), kb * BK, tile * BM);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        const int u = u0 + i, kb = u - (u / p.KB) * p.KB;
        tma_load_2d(base + i * C::STAGE + C::A_BYTES, &xmap, full(i), kb * BK, 0);
      }
      issued = pre;
      stage = pre % S;
      phase = (pre == S) ? 1u : 0u;
      for (int u = u0 + pre; u < u1; ++u) {
        const int tile = u / p.KB, kb = u - tile * p.KB;
        if (!wait_bounded(empty(stage), phase ^ 1u, abort_flag, p.err, 1)) break;
        mbar_expect_tx(full(stage), C::STAGE);
        const uint32_t dst = base + stage * C::STAGE;
        tma_load_2d(dst, &wmap, full(stage), kb * BK, tile * BM);
        tma_load_2d(dst + C::A_BYTES, &xmap, full(stage), kb * BK, 0);
        ++issued;
        if (++stage == S) { stage = 0; phase ^= 1u; }
      }
      pdl_trigger();  // all loads issued: the next kernel may start its prologue
      if (*abort_flag) {
        // drain: wait (bounded, ignoring the abort flag) for the loads still in flight
        for (int i = 0; i < S && i < issued; ++i) {
          if (--stage < 0) { stage = S - 1; phase ^= 1u; }
          for (uint32_t t = 0; t < kWaitLimit && !mbar_try_wait(full(stage), phase); ++t) {}
        }
      }
    }
    __syncwarp();  // the whole warp meets the final barrier together
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16<MP>();
      int stage = 0;
      uint32_t phase = 0;
      int seg = 0;
      int u = u0;
      bool ok = true;
      while (ok && u < u1) {
        const int tile = u / p.KB;
        const int seg_end = min(u1, (tile + 1) * p.KB);
        const int buf = seg & 1;
        const uint32_t use = (uint32_t)(seg >> 1);
        if (!wait_bounded(acce(buf), (use & 1u) ^ 1u, abort_flag, p.err, 2)) break;
        tc_fence_after();
        const uint32_t dcol = tmem + (uint32_t)(buf * MP);
        bool first = true;
        for (; u < seg_end; ++u) {
          if (!wait_bounded(full(stage), phase, abort_flag, p.err, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a = base + stage * C::STAGE;
          const uint64_t ad = sw128_desc(a), bd = sw128_desc(a + C::A_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)  // +32 bytes along K inside the swizzle row
            umma_bf16(dcol, ad + 2 * k, bd + 2 * k, idesc, (first && k == 0) ? 0u : 1u);
          first = false;
          umma_commit(empty(stage));
          if (++stage == S) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(accf(buf));
        ++seg;
      }
      if (!ok || *abort_flag) {
        // let every issued MMA retire before TMEM is released: commit to an
        // accumulator barrier nobody else waits on any more and wait for it.
        const int buf = seg & 1;
        umma_commit(accf(buf));
        const uint32_t par = (uint32_t)((seg >> 1) & 1);
        for (uint32_t t = 0; t < kWaitLimit && !mbar_try_wait(accf(buf), par); ++t) {}
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    pdl_wait();  // outputs, residual inputs and the workspace belong to the previous kernel until it ends
    const int q = warp & 3;  // TMEM lane quadrant this warp may read
    const int row = q * 32 + lane;
    const int ew = warp - 2;   // epilogue warp 0 .. 4 * REP - 1
    // which of the quadrant's REP warps: takes 16-row chunks rep, rep + REP, ... (a compile-time 0
    // when REP is 1, so the one-warp loops keep their constant bounds)
    const int rep = REP == 1 ? 0 : ew >> 2;
    auto n_of = [&](int tile) { return tile * BM + row; };
    // ---- fused collective: pushes of a finished tile and its completion
    auto tile_count = [&](int tile) { return *reinterpret_cast<volatile uint32_t*>(tile_count_of(p, tile)) + 1u; };
    auto push = [&](uint32_t jt, int tile, int m, int n, float v) {  // value of output (m, n) to every rank
      if (p.coll == COLL_ALLREDUCE) {
        // one 64-bit word: fp32 bits | delivery count << 32 (single-copy atomic, so
        // the receiver polls the data itself -- no flag, no fence)
        const size_t o = p.dst_off + sizeof(uint64_t) * (((((size_t)(jt & 1u) * p.recv_tiles + tile) * p.world +
                                                           p.rank) * p.recv_rows + m) * BM + (n - tile * BM));
        const uint64_t w = ((uint64_t)jt << 32) | __float_as_uint(v);
        if (p.owner_fold) st_relaxed_sys_u64(reinterpret_cast<uint64_t*>(p.heaps[tile % p.world] + o), w);
        else
          for (int d = 0; d < p.world; ++d) st_relaxed_sys_u64(reinterpret_cast<uint64_t*>(p.heaps[d] + o), w);
      } else {
        const size_t o = p.dst_off + sizeof(float) * ((size_t)m * p.ldy + p.col_off + n);
        for (int d = 0; d < p.world; ++d) *reinterpret_cast<float*>(p.heaps[d] + o) = v;
      }
    };
    auto coll_finish = [&](uint32_t jt, int tile) {
      const int n = tile * BM + row;
      if (p.coll == COLL_ALLREDUCE) {
        // every thread polls its own (m, row) words of all sources -- the words it
        // pushed itself included, so no barrier orders the CTA's pushes -- and
        // folds them in rank order: bit-identical sums on every rank.
        // owner_fold (more than 16 rows): only the tile's owner rank (tile % world)
        // received the partials; it folds them the same way and sends each sum, as the
        // same kind of word, into the slot [tile][owner] of every other rank, where
        // nothing else is written for this tile; the other ranks poll that one word.
        // Every rank then adds its own copy of the residual (identical on all ranks):
        // the values are those of the all-to-all form, for about 2/world of its traffic.
        const int owner = p.owner_fold ? tile % p.world : p.rank;
        if (n < p.N && owner != p.rank) {
          const uint64_t* slot = reinterpret_cast<const uint64_t*>(p.heaps[p.rank] + p.dst_off) +
                                 ((((size_t)(jt & 1u) * p.recv_tiles + tile) * p.world + owner) * p.recv_rows) * BM +
                                 row;
          bool ok = true;
          for (int m0 = 16 * rep; m0 < p.M && ok; m0 += 16 * REP) {
            uint64_t w[16];
            float res[16];
            load_residual16(p, m0, n, res);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              w[i] = m0 + i < p.M ? ld_relaxed_sys_u64(slot + (size_t)(m0 + i) * BM) : ((uint64_t)jt << 32);
            for (uint32_t it = 0;; ++it) {  // late words: poll again (bounded)
              bool all = true;
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if ((uint32_t)(w[i] >> 32) != jt) {
                  all = false;
                  w[i] = ld_relaxed_sys_u64(slot + (size_t)(m0 + i) * BM);
                }
              if (all) break;
              if (it >= kPeerWaitPolls) {
                ok = false;
                break;
              }
              __nanosleep(32);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (m0 + i < p.M)
                reinterpret_cast<bf16*>(p.y)[(int64_t)(m0 + i) * p.N + n] =
                    from_f<bf16>(__fadd_rn(res[i], store_round<bf16>(__uint_as_float((uint32_t)w[i]))));
          }
          if (!ok) {
            atomicExch(p.err, 5u);
            atomicExch(ctrl_of(p, p.rank) + 2, (unsigned int)SSD_ERR_TIMEOUT);
          }
        } else if (n < p.N) {
          const uint64_t* slot = reinterpret_cast<const uint64_t*>(p.heaps[p.rank] + p.dst_off) +
                                 (((size_t)(jt & 1u) * p.recv_tiles + tile) * p.world) * p.recv_rows * BM + row;
          bool ok = true;
          const bf16* yres = reinterpret_cast<const bf16*>(p.y);
          for (int m0 = 4 * rep; m0 < p.M; m0 += 4 * REP) {
            uint64_t w[4][kMaxTP];
            float res[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)  // in flight together with the first poll
              res[i] = m0 + i < p.M ? __bfloat162float(__ldcg(yres + (int64_t)(m0 + i) * p.N + n)) : 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int r = 0; r < kMaxTP; ++r)
                w[i][r] = (m0 + i < p.M && r < p.world)
                              ? ld_relaxed_sys_u64(slot + ((size_t)r * p.recv_rows + m0 + i) * BM)
                              : ((uint64_t)jt << 32);
            for (uint32_t it = 0;; ++it) {  // late words: poll again (bounded)
              bool all = true;
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int r = 0; r < kMaxTP; ++r)
                  if ((uint32_t)(w[i][r] >> 32) != jt) {
                    all = false;
                    w[i][r] = ld_relaxed_sys_u64(slot + ((size_t)r * p.recv_rows + m0 + i) * BM);
                  }
              if (all) break;
              if (it >= kPeerWaitPolls) {
                ok = false;
                break;
              }
              __nanosleep(32);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              if (m0 + i >= p.M) break;
              float sum = 0.f;
#pragma unroll
              for (int r = 0; r < kMaxTP; ++r)
                if (r < p.world) sum += __uint_as_float((uint32_t)w[i][r]);
              reinterpret_cast<bf16*>(p.y)[(int64_t)(m0 + i) * p.N + n] =
                  from_f<bf16>(__fadd_rn(res[i], store_round<bf16>(sum)));
              if (p.owner_fold) {  // the sum to every other rank's slot [tile][owner]
                const size_t o = p.dst_off + sizeof(uint64_t) * (((((size_t)(jt & 1u) * p.recv_tiles + tile) *
                                                                     p.world + p.rank) * p.recv_rows + m0 + i) * BM + row);
                const uint64_t word = ((uint64_t)jt << 32) | __float_as_uint(sum);
                for (int d = 0; d < p.world; ++d)
                  if (d != p.rank) st_relaxed_sys_u64(reinterpret_cast<uint64_t*>(p.heaps[d] + o), word);
              }
            }
            if (!ok) break;
          }
          if (!ok) {
            atomicExch(p.err, 5u);
            atomicExch(ctrl_of(p, p.rank) + 2, (unsigned int)SSD_ERR_TIMEOUT);
          }
        }
        epi_bar<EPI>();  // every thread has read the tile count before it advances
        if (threadIdx.x == 64) *tile_count_of(p, tile) = jt;
        return;
      }
      // all-gather: the barrier puts every epilogue thread's pushes before thread
      // 64's system-scope fence and flag stores (cumulativity)
      epi_bar<EPI>();
      if (threadIdx.x == 64) {
        fence_acq_rel_sys();
        for (int d = 0; d < p.world; ++d) st_relaxed_sys(flag_of(p, d, p.rank, tile), jt);
      }
      if (warp == 2) {  // lane s waits for source rank s's delivery of this tile
        bool ok = true;
        if (lane < p.world && lane != p.rank) {
          ok = wait_peer_flag(flag_of(p, p.rank, lane, tile), jt);
          fence_acq_rel_sys();
        }
        ok = __all_sync(0xffffffffu, ok);
        if (lane == 0) {
          *tile_count_of(p, tile) = jt;
          if (!ok) {
            atomicExch(p.err, 5u);
            atomicExch(ctrl_of(p, p.rank) + 2, (unsigned int)SSD_ERR_TIMEOUT);
          }
        }
      }
    };
    if (p.rowscale && (!CLU || cluster_ctarank() == 0)) {
      // RMS of each token row (the (1 + w) factor is folded into the weights):
      // warp (q) takes rows m = q, q+4, ...; more than 16 rows were computed once
      // for all CTAs by row_inv_rms_kernel (the same function, so the same bits).
      if (p.inv_g) {
        for (int m = (int)threadIdx.x - 64; m < p.M; m += EPI) inv_s[m] = __ldcg(p.inv_g + m);
      } else {
        for (int m = REP == 1 ? q : ew; m < p.M; m += 4 * REP) {
          const float r = row_inv_rms(p.x + (size_t)m * p.K, p.K, p.eps, lane);
          if (lane == 0) inv_s[m] = r;
        }
      }
      epi_bar<EPI>();
    }
    if constexpr (ROPE) {
      if (!CLU || cluster_ctarank() == 0) {  // the CTAs that store outputs
        for (int m = (int)threadIdx.x - 64; m < p.M; m += EPI) rope_row_info(p.rope, m, rope_pc, rope_off);
        epi_bar<EPI>();
      }
    }
    if constexpr (CLU) {
      // ------------------------------------------------ cluster fold (one tile)
      cluster_wait();  // startup phase: every CTA of the cluster has initialised its barriers
      const uint32_t crank = cluster_ctarank();
      const int tile = cta / p.G;
      const int n = tile * BM + row;
      // the leader's tile count and residual rows, in flight while the MMAs finish
      const uint32_t jt = (COLL && crank == 0) ? tile_count(tile) : 0u;
      float res[16];
      if (!COLL && crank == 0) load_residual16(p, 0, n, res);
      float v[16];
      if (wait_bounded(accf(0), 0u, abort_flag, p.err, 4)) {
        tc_fence_after();
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16), v);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0.f;
      }
      // [M][BM] fp32 partial in ring stage 0: every MMA of this CTA has completed
      // (accf), so no operand lives there any more
      float* red = reinterpret_cast<float*>(gbase);
      if (crank != 0) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < p.M) red[j * BM + row] = v[j];
        // the barrier orders all epilogue threads' stores before thread 64's
        // cluster-scope release (cumulativity)
        epi_bar<EPI>();
        if (threadIdx.x == 64) mbar_arrive_remote(mapa(red_bar, 0));
      } else {
        if (!wait_cluster_bounded(red_bar, 0u, 4u * kWaitLimit)) {
          *abort_flag = 1;
          atomicExch(p.err, 6u);
        }
        // fold in part (= K) order, 4 peers' loads in flight at a time: the sums
        // of the global fold (0 + part 0 + part 1 + ...)
        float s[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) s[j] = 0.f + v[j];
        const uint32_t red_s = smem_u32(red) + 4u * (uint32_t)row;
        for (int c = 1; c < p.G; c += 4) {
          float r[4][16];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const uint32_t rb = mapa(red_s, (uint32_t)min(c + cc, p.G - 1));
#pragma unroll
            for (int j = 0; j < 16; ++j)
              r[cc][j] = (c + cc < p.G && j < p.M) ? ld_dsmem(rb + 4u * (uint32_t)(j * BM)) : 0.f;
          }
#pragma unroll
          for (int cc = 0; cc < 4; ++cc)
#pragma unroll
            for (int j = 0; j < 16; ++j) s[j] += r[cc][j];
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (p.rowscale && j < p.M) s[j] = __fmul_rn(s[j], inv_s[j]);
          const float up = __shfl_xor_sync(0xffffffffu, s[j], 1);  // row n ^ 1 (GeGLU up, RoPE pair)
          if constexpr (COLL) {
            if (j < p.M && n < p.N) push(jt, tile, j, n, s[j]);
          } else if (j < p.M && n < p.N) {
            store_out<ROPE>(p, j, n, s[j], up, res[j], rope_pc, rope_off);
          }
        }
        if constexpr (COLL) coll_finish(jt, tile);
      }
    }
    int seg = 0;
    int u = CLU ? u1 : u0;  // CLU: the tile was finished above
    const int first_tile = u0 / p.KB;
    while (u < u1) {
      const int tile = u / p.KB;
      const int kb_begin = u - tile * p.KB;
      const int seg_end = min(u1, (tile + 1) * p.KB);
      const int kb_end = seg_end - tile * p.KB;
      u = seg_end;
      const int buf = seg & 1;
      const uint32_t use = (uint32_t)(seg >> 1);
      ++seg;
      const bool whole = (kb_begin == 0 && kb_end == p.KB);
      const uint32_t jt_whole = (COLL && whole) ? tile_count(tile) : 0u;
      if (!wait_bounded(accf(buf), use & 1u, abort_flag, p.err, 4)) break;
      tc_fence_after();
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * MP);
      const int n = tile * BM + row;
      float* mine = p.part + (size_t)(cta * 2 + (tile == first_tile ? 0 : 1)) * p.ms * BM + 4 * row;
      const int cend = min(MP, (p.M + 15) & ~15);
      float nxt[16];  // this warp's next 16 accumulator columns, read while a chunk is stored
      if (REP == 1 || 16 * rep < cend) {  // (one warp: cend >= 16 always)
        tmem_ld16(taddr + 16 * rep, nxt);
        tmem_ld_wait();
      }
#pragma unroll 1
      for (int c0 = 16 * rep; c0 < cend; c0 += 16 * REP) {
        float v[16], res[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = nxt[j];
        if (c0 + 16 * REP < cend) tmem_ld16(taddr + c0 + 16 * REP, nxt);
        // the residual rows of this chunk are in flight together
        // (row-parallel shapes whose K is at most 8 k-blocks, e.g. O at TP8, take this path)
        if (!whole) {
          // this CTA's part of a split tile: 16 rows of column n, four 16-byte stores (rows past M
          // land in the padding and are never read)
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<float4*>(mine + (size_t)(c0 / 4 + i) * BM * 4) =
                make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else {
          if (!COLL) load_residual16(p, c0, n, res);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = c0 + j;
            if (p.rowscale && m < p.M) v[j] = __fmul_rn(v[j], inv_s[m]);
            const float up = __shfl_xor_sync(0xffffffffu, v[j], 1);  // row n ^ 1 (GeGLU up, RoPE pair)
            if (m >= p.M) continue;
            if constexpr (COLL) {
              if (n < p.N) push(jt_whole, tile, m, n, v[j]);
            } else if (n < p.N) {
              store_out<ROPE>(p, m, n, v[j], up, res[j], rope_pc, rope_off);
            }
          }
        }
        if (c0 + 16 * REP < cend) tmem_ld_wait();
      }
      tc_fence_before();
      mbar_arrive(acce(buf));
      if (whole) {
        if constexpr (COLL) coll_finish(jt_whole, tile);
        continue;
      }
      // ---- split tile: ticket, then the last contributor folds all partials in K order.
      // The barrier orders this CTA's partial stores before thread 64's ticket
      // (an acq_rel RMW: release of our partials, acquire of the others' for the
      // last contributor); the second barrier extends the acquire to all
      // epilogue threads, whose fold loads read L2 (.cg).  No per-thread fence.
      epi_bar<EPI>();
      const int c_first = cta_of_unit(p, tile * p.KB);
      const int c_last = cta_of_unit(p, tile * p.KB + p.KB - 1);
      if (threadIdx.x == 64) {
        const unsigned int prev = atom_add_acq_rel_gpu(&p.counters[tile], 1u);
        const bool last = prev == (unsigned int)(c_last - c_first);
        if (last) *reinterpret_cast<volatile unsigned int*>(&p.counters[tile]) = 0u;  // self-reset (stream-ordered)
        *last_flag = last ? 1 : 0;
      }
      epi_bar<EPI>();
      const bool last = *last_flag != 0;
      epi_bar<EPI>();  // everyone has read the flag before the next tile may rewrite it
      if (!last) continue;
      const uint32_t jt = COLL ? tile_count(tile) : 0u;
      // Fold the contributors in CTA (= K) order.  Rows are taken 16 at a time and
      // contributors 4 at a time so up to 64 independent L2 loads are in flight
      // per thread; the summation order per output stays c_first .. c_last.
      for (int m0 = 16 * rep; m0 < p.M; m0 += 16 * REP) {
        const int mn = min(16, p.M - m0);
        float s[16], res[16];
        if (!COLL) load_residual16(p, m0, n, res);
#pragma unroll
        for (int i = 0; i < 16; ++i) s[i] = 0.f;
        for (int c = c_first; c <= c_last; c += 4) {
          // all 16 vector loads are issued before the first add: contributors past c_last
          // read a valid partial (clamped index) whose value is never used
          float v[4][16];
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int ci = min(c + cc, c_last);
            const int e = tile == unit_begin(p, ci) / p.KB ? 0 : 1;
            const float* src = p.part + (size_t)(ci * 2 + e) * p.ms * BM + (size_t)(m0 / 4) * BM * 4 + 4 * row;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float4 t = __ldcg(reinterpret_cast<const float4*>(src + (size_t)i * BM * 4));
              v[cc][4 * i] = t.x;
              v[cc][4 * i + 1] = t.y;
              v[cc][4 * i + 2] = t.z;
              v[cc][4 * i + 3] = t.w;
            }
          }
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            if (c + cc > c_last) break;
#pragma unroll
            for (int i = 0; i < 16; ++i) s[i] += v[cc][i];
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          if (p.rowscale && i < mn) s[i] = __fmul_rn(s[i], inv_s[m0 + i]);
          const float up = __shfl_xor_sync(0xffffffffu, s[i], 1);  // row n ^ 1 (GeGLU up, RoPE pair)
          if constexpr (COLL) {
            if (i < mn && n < p.N) push(jt, tile, m0 + i, n, s[i]);
          } else if (i < mn && n < p.N) {
            store_out<ROPE>(p, m0 + i, n, s[i], up, res[i], rope_pc, rope_off);
          }
        }
      }
      if constexpr (COLL) coll_finish(jt, tile);
    }
  }

  if (CLU && warp < 2) cluster_wait();  // startup phase (the epilogue waited before its remote accesses)
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS) : "memory");
  }
  if (CLU) {  // no CTA leaves while the leader may still read its shared memory
    cluster_arrive();
    cluster_wait();
  }
}

// ------------------------------------------------------------------ host side
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(f);
  });
  return fn;
}

// rows x K bf16 row-major, box = box_rows x 64, 128-byte swizzle, zero fill out of bounds.
bool make_map(CUtensorMap* m, const void* ptr, int rows, int K, int box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct MapKey {
  const void* p;
  int n, k;
  bool operator==(const MapKey& o) const { return p == o.p && n == o.n && k == o.k; }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.p) ^ ((size_t)k.n * 0x9E3779B97F4A7C15ull) ^ (size_t)k.k;
  }
};

bool weight_map(CUtensorMap* out, const void* w, int N, int K) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  std::lock_guard<std::mutex> g(mu);
  MapKey key{w, N, K};
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  if (!make_map(out, w, N, K, BM)) return false;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return true;
}

int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  return n;
}

constexpr int kMaxParts = 16;  // cluster size limit (non-portable sizes above 8)

// Kernel attributes, set once per instantiation and device (not on every launch).
template <int MP, bool COLL, bool CLU, bool ROPE>
cudaError_t prepare_kernel() {
  static std::mutex mu;
  static uint64_t done = 0;  // bit d: attributes set on device d
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> g(mu);
  if (done >> dev & 1ull) return cudaSuccess;
  auto kern = linear_tc_kernel<MP, COLL, CLU, ROPE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg<MP>::SMEM);
  if (e == cudaSuccess && CLU) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess) done |= 1ull << dev;
  return e;
}

// True when `tiles` clusters of G CTAs of the M <= 16 kernel can all be resident
// at once on this device (so the tile-split plan runs in one wave).
bool clusters_fit(int G, int tiles) {
  static std::mutex mu;
  static std::unordered_map<int, int> cache;  // device * 32 + G -> max active clusters
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(dev * 32 + G);
  if (it == cache.end()) {
    int n = 0;
    if (prepare_kernel<16, false, true, false>() == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(G * tiles);
      cfg.blockDim = dim3(Cfg<16>::THREADS);
      cfg.dynamicSmemBytes = Cfg<16>::SMEM;
      cudaLaunchAttribute a[1];
      a[0].id = cudaLaunchAttributeClusterDimension;
      a[0].val.clusterDim.x = G;
      a[0].val.clusterDim.y = 1;
      a[0].val.clusterDim.z = 1;
      cfg.attrs = a;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, linear_tc_kernel<16, false, true, false>, &cfg) != cudaSuccess) n = 0;
    }
    (void)cudaGetLastError();
    it = cache.emplace(dev * 32 + G, n).first;
  }
  return it->second >= tiles;
}

// Tile-split plan for shapes with at most as many tiles as SMs: G parts per tile,
// up to two CTAs per SM (the largest G whose clusters all fit at once, else the
// arithmetic choice through the global fold).  Depends on (N, K) and the device only, never
// on M, so every M sums the same partials in the same order.
int split_parts(int tiles, int KB, int sms) {
  if (tiles > sms || KB < 2) return 0;
  // Few k-blocks per tile: the fold costs more than the parallelism buys.  Measured on B200 in
  // chains of launches at M = 5: a part's partial reaches the folding CTA in about one shared-memory
  // round trip per four parts (~1.3 us each), while a CTA streams a 16 KB k-block in well under
  // that.  So a tile of at most 8 k-blocks is one CTA (no fold: O at TP8 6.2 vs 6.6 us), and a
  // tile of at most 32 k-blocks takes at most four parts (2B O 7.7 vs 9.1 us, 2B QKV 7.9 vs 9.2).
  if (KB <= 8) return 1;
  int G = (2 * sms) / tiles;
  if (G > KB) G = KB;
  if (G > kMaxParts) G = kMaxParts;
  if (KB <= 32 && G > 4) G = 4;
  for (int g = G; g >= 2; --g)
    if (clusters_fit(g, tiles)) return g;
  return G;
}

void plan(int M, int N, int K, int sms, Params& p, int& grid) {
  const int tiles = (N + BM - 1) / BM;
  p.KB = (K + BK - 1) / BK;
  p.U = tiles * p.KB;
  p.G = split_parts(tiles, p.KB, sms);
  if (p.G) {
    grid = tiles * p.G;
    p.base = p.rem = 0;
    return;
  }
  grid = p.U < sms ? p.U : sms;
  p.base = p.U / grid;
  p.rem = p.U % grid;
  (void)M;
}

// Stream-K launches one CTA per SM, the tile-split plan up to two: the partial
// buffer [grid][2][M][BM] is sized for twice the SM count.
// Layout: tile counters | error word | partials [2 * SMs][2][M rounded up to 16][BM] | row scales [256].
size_t workspace_bytes(int M, int N, int K) {
  (void)N;
  (void)K;
  const size_t ms = (size_t)((M + 15) & ~15);
  return kCounterBytes + 256 + sizeof(float) * ((size_t)num_sms() * 4 * ms * BM + 256);
}

template <int MP>
int launch(cudaStream_t st, const void* x, const void* w, void* y, int epi, int M, int N, int K, void* ws,
           int rowscale, float eps, const CollArgs* ca, const RopeArgs* ra) {
  using C = Cfg<MP>;
  CUtensorMap wm, xm;
  if (!weight_map(&wm, w, N, K)) return SSD_ERR_LAUNCH;
  if (!make_map(&xm, x, M, K, MP)) return SSD_ERR_LAUNCH;
  Params p{};
  int grid;
  plan(M, N, K, num_sms(), p, grid);
  p.y = y;
  p.x = reinterpret_cast<const bf16*>(x);
  p.rowscale = rowscale;
  p.eps = eps;
  p.epi = epi;
  p.M = M;
  p.N = N;
  p.K = K;
  char* wsb = reinterpret_cast<char*>(ws);
  p.counters = reinterpret_cast<unsigned int*>(wsb);
  p.err = reinterpret_cast<unsigned int*>(wsb + kCounterBytes);
  p.part = reinterpret_cast<float*>(wsb + kCounterBytes + 256);
  p.ms = (M + 15) & ~15;
  p.inv_g = nullptr;
  if (rowscale && M > 16) {
    float* inv = p.part + (size_t)num_sms() * 4 * p.ms * BM;
    SSD_PDL(row_inv_rms_kernel, (M + 3) / 4, 128, 0, st, reinterpret_cast<const bf16*>(x), M, K, eps, inv);
    SSD_CHECK_LAUNCH();
    p.inv_g = inv;
  }
  p.coll = COLL_NONE;
  if (ra) p.rope = *ra;
  if (ca && ca->mode != COLL_NONE) {
    p.coll = ca->mode;
    p.rank = ca->rank;
    p.world = ca->world;
    p.ldy = ca->ldy;
    p.col_off = ca->col_off;
    for (int r = 0; r < kMaxTP; ++r) p.heaps[r] = r < ca->world ? ca->heaps[r] : nullptr;
    p.ctrl_off = ca->ctrl_off;
    p.dst_off = ca->dst_off;
    p.recv_rows = ca->recv_rows;
    p.recv_tiles = ca->recv_tiles;
    // The owner-fold form sends about 2 (world - 1) / world of a rank's partial bytes where the
    // all-to-all form sends world - 1 of them, for one more hop (a poll and a push, a few us).  It
    // is taken where that saves more than 4 MB per rank (about 6 us of NVLink), which needs at
    // least 4 ranks and many rows (e.g. 7B O/down at 8 ranks from 33 rows on); it is never
    // taken for 16 rows or fewer.  Both forms give the same bits (the caller may pick one).
    const double saved = (double)(ca->world - 1) * (ca->world - 2) / ca->world * M * N * sizeof(uint64_t);
    const bool owner = ca->form == SSD_ALLREDUCE_OWNER ||
                       (ca->form == SSD_ALLREDUCE_AUTO && M > 16 && saved > 4.0 * (1 << 20));
    p.owner_fold = (ca->mode == COLL_ALLREDUCE && ca->world > 1 && owner) ? 1 : 0;
  }
  if constexpr (MP == 16) {
    if (p.G >= 2 && clusters_fit(p.G, grid / p.G)) {
      const bool coll = p.coll != COLL_NONE, rope = epi == kEpiRopeQkv;
      if ((coll ? prepare_kernel<16, true, true, false>()
                : rope ? prepare_kernel<16, false, true, true>() : prepare_kernel<16, false, true, false>()) !=
          cudaSuccess)
        return SSD_ERR_LAUNCH;
      auto kern = coll ? linear_tc_kernel<16, true, true, false>
                       : rope ? linear_tc_kernel<16, false, true, true> : linear_tc_kernel<16, false, true, false>;
      if (launch_pdl_cluster(kern, dim3(grid), dim3(C::THREADS), C::SMEM, st, (unsigned)p.G, wm, xm, p) !=
          cudaSuccess) {
        (void)cudaGetLastError();
        return SSD_ERR_LAUNCH;
      }
      return SSD_OK;
    }
  }
  const bool coll = p.coll != COLL_NONE, rope = epi == kEpiRopeQkv;
  auto kern = coll ? linear_tc_kernel<MP, true, false, false>
                   : rope ? linear_tc_kernel<MP, false, false, true> : linear_tc_kernel<MP, false, false, false>;
  if ((coll ? prepare_kernel<MP, true, false, false>()
            : rope ? prepare_kernel<MP, false, false, true> () : prepare_kernel<MP, false, false, false>()) !=
      cudaSuccess)
    return SSD_ERR_LAUNCH;
  SSD_PDL(kern, grid, C::THREADS, C::SMEM, st, wm, xm, p);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

template <typename... A>
int launch_any(int M, A... a) {
  if (M <= 16) return launch<16>(a...);
  if (M <= 32) return launch<32>(a...);
  if (M <= 64) return launch<64>(a...);
  if (M <= 128) return launch<128>(a...);
  return launch<256>(a...);
}

}  // namespace tc

bool make_kv_page_map(CUtensorMap* m, const void* pages, int plane_pages, int block_size, int hkv, int D) {
  // pages [plane_pages][block_size][hkv][D] bf16 viewed as 5-D (d % 64, d / 64, head, row, page):
  // one box = 16 rows x 64 dims (128 B per row, 128-byte swizzle) of one head of one page
  tc::EncodeFn fn = tc::encode_fn();
  if (!fn || D % 64 || block_size > 256) return false;
  cuuint64_t dims[5] = {64, (cuuint64_t)(D / 64), (cuuint64_t)hkv, (cuuint64_t)block_size, (cuuint64_t)plane_pages};
  cuuint64_t strides[4] = {128, (cuuint64_t)D * 2, (cuuint64_t)hkv * D * 2, (cuuint64_t)block_size * hkv * D * 2};
  cuuint32_t box[5] = {64, 1, 1, (cuuint32_t)block_size, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(pages), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool linear_tc_supported(int M, int N, int K) {
  return M >= 1 && M <= 256 && N >= 1 && K >= 64 && (K % 8) == 0 && (N + tc::BM - 1) / tc::BM <= kCounterCap &&
         tc::encode_fn() != nullptr;
}

size_t linear_tc_workspace(int M, int N, int K) { return tc::workspace_bytes(M, N, K); }

int linear_tc(cudaStream_t st, const void* x, const void* w, void* y, int epi, int M, int N, int K, void* ws,
              size_t ws_bytes, int rowscale, float eps) {
  if (!ws || ws_bytes < tc::workspace_bytes(M, N, K)) return SSD_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) return SSD_ERR_UNSUPPORTED;
  return tc::launch_any(M, st, x, w, y, epi, M, N, K, ws, rowscale, eps, (const CollArgs*)nullptr,
                        (const RopeArgs*)nullptr);
}

int linear_tc_rope(cudaStream_t st, const void* x, const void* w, int M, int N, int K, void* ws, size_t ws_bytes,
                   float eps, const RopeArgs& ra) {
  if (!linear_tc_supported(M, N, K)) return SSD_ERR_UNSUPPORTED;
  if (!ws || ws_bytes < tc::workspace_bytes(M, N, K)) return SSD_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) return SSD_ERR_UNSUPPORTED;
  if (ra.D <= 0 || (ra.D & 1) || N != (ra.hq + 2 * ra.hkv) * ra.D || ra.T <= 0 || M % ra.T) return SSD_ERR_INVALID;
  return tc::launch_any(M, st, x, w, nullptr, kEpiRopeQkv, M, N, K, ws, 1, eps, (const CollArgs*)nullptr, &ra);
}

int linear_tc_coll(cudaStream_t st, const void* x, const void* w, void* y, int M, int N, int K, void* ws,
                   size_t ws_bytes, const CollArgs& ca) {
  if (!linear_tc_supported(M, N, K)) return SSD_ERR_UNSUPPORTED;
  if ((N + tc::BM - 1) / tc::BM > kFlagTiles) return SSD_ERR_UNSUPPORTED;
  if (!ws || ws_bytes < tc::workspace_bytes(M, N, K)) return SSD_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15)) return SSD_ERR_UNSUPPORTED;
  const int epi = ca.mode == COLL_ALLREDUCE ? SSD_EPI_RESIDUAL : SSD_EPI_STORE_F32;
  return tc::launch_any(M, st, x, w, y, epi, M, N, K, ws, 0, 0.f, &ca, (const RopeArgs*)nullptr);
}

}  // namespace ssd
