// K5: device mirror of the paged-KV block allocator (allocate / speculative
// rollback / free), bit-exact with jax_ssd/runtime/page_manager.py:21-70 when
// sequences are processed in index order.
//
// These are latency-bound integer kernels: one CTA of 1024 threads.  The
// sequential semantics of the reference (sequence 0 first, blocks popped from /
// pushed to the END of one LIFO free list, ref counts with "absent = 1" on
// release) are reproduced with scans instead of a serial loop:
//   allocate: an exclusive scan with the reference's all-or-nothing rule gives
//             each sequence its slice of the free-list top;
//   release:  each release event e of block x is the i-th event on x in
//             sequence order; starting from count r, rc' = max(rc,1)-1 applied
//             i times is max(r-i,0), so the event pushes x iff i >= r.  A scan
//             of those pushes gives each its free-list position.
#include "common.cuh"

namespace ssd {
namespace {

constexpr int kPageThreads = 1024;
constexpr int kEventCap = 1024;  // events handled per batch (one per thread)

__device__ __forceinline__ int block_exclusive_scan(int v, int* tmp, int* total) {
  // Hillis-Steele over blockDim.x <= 1024 entries in shared memory.
  const int t = threadIdx.x;
  tmp[t] = v;
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {
    int add = (t >= off) ? tmp[t - off] : 0;
    __syncthreads();
    tmp[t] += add;
    __syncthreads();
  }
  const int incl = tmp[t];
  if (total) *total = tmp[blockDim.x - 1];
  __syncthreads();
  return incl - v;
}

__global__ void __launch_bounds__(kPageThreads)
page_allocate_kernel(int32_t* tables, int32_t* lens, int max_blocks, int32_t* free_list, int32_t* free_top,
                     int32_t* ref_counts, int num_blocks, const int32_t* num_tokens, const int32_t* num_new,
                     uint8_t* ok, int block_size, int B) {
  __shared__ int s_extra[kPageThreads];
  __shared__ int s_start[kPageThreads];  // free-list top seen by the sequence
  __shared__ int s_top;
  pdl_wait();
  if (threadIdx.x == 0) s_top = *free_top;
  __syncthreads();
  for (int base = 0; base < B; base += kPageThreads) {
    const int b = base + threadIdx.x;
    int extra = 0;
    bool fits = true;
    if (b < B) {
      const int need = (num_tokens[b] + num_new[b] + block_size - 1) / block_size;
      extra = need - lens[b];
      if (extra < 0) extra = 0;
      if (lens[b] + extra > max_blocks) fits = false;  // table capacity (device-side guard)
    }
    s_extra[threadIdx.x] = fits ? extra : -1;
    __syncthreads();
    // The all-or-nothing rule makes this scan sequential; it is a few integer ops
    // per sequence on one thread, the pops below run in parallel.
    if (threadIdx.x == 0) {
      int top = s_top;
      const int n = min(kPageThreads, B - base);
      for (int i = 0; i < n; ++i) {
        const int e = s_extra[i];
        s_start[i] = top;
        if (e < 0 || e > top) { s_extra[i] = -1; continue; }
        top -= e;
      }
      s_top = top;
    }
    __syncthreads();
    if (b < B) {
      const int e = s_extra[threadIdx.x];
      if (ok) ok[b] = e >= 0 ? 1 : 0;
      if (e > 0) {
        const int top = s_start[threadIdx.x];
        int len = lens[b];
        for (int i = 0; i < e; ++i) {
          const int blk = free_list[top - 1 - i];
          free_list[top - 1 - i] = -1;
          tables[(int64_t)b * max_blocks + len + i] = blk;
          if (blk >= 0 && blk < num_blocks) atomicAdd(&ref_counts[blk], 1);
        }
        lens[b] = len + e;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *free_top = s_top;
  pdl_trigger();
}

// Release events in sequence order.  mode 0 = rollback (pop from the end while
// len > used), mode 1 = free (target table forward, then draft table forward).
__global__ void __launch_bounds__(kPageThreads)
page_release_kernel(int mode, int32_t* tables, int32_t* lens, int max_blocks, int32_t* dtables, int32_t* dlens,
                    int dmax_blocks, int32_t* free_list, int32_t* free_top, int32_t* ref_counts, int num_blocks,
                    const int32_t* num_tokens, const int32_t* accepted, int32_t* kv_lens, const uint8_t* release,
                    int block_size, int B) {
  __shared__ int s_tmp[kPageThreads];
  __shared__ int s_blk[kEventCap];
  __shared__ int s_off[kPageThreads];
  __shared__ int s_top;
  pdl_wait();
  if (threadIdx.x == 0) s_top = *free_top;
  __syncthreads();

  for (int base = 0; base < B; base += kPageThreads) {
    const int b = base + threadIdx.x;
    int n = 0, used = 0;
    if (b < B) {
      if (mode == 0) {
        used = (num_tokens[b] + accepted[b] + block_size - 1) / block_size;
        const int len = min(lens[b], max_blocks);
        n = len > used ? len - used : 0;
        if (kv_lens) kv_lens[b] = num_tokens[b] + accepted[b];
      } else if (release[b]) {
        n = min(lens[b], max_blocks) + (dtables ? min(dlens[b], dmax_blocks) : 0);
      }
    }
    int tot;
    const int off = block_exclusive_scan(n, s_tmp, &tot);
    s_off[threadIdx.x] = off;
    __syncthreads();
    // Walk the events of this group of sequences in batches of kEventCap.
    for (int e0 = 0; e0 < tot; e0 += kEventCap) {
      const int e = e0 + threadIdx.x;
      // locate the sequence of event e (binary search over s_off)
      int blk = -1;
      if (e < tot) {
        int lo = 0, hi = min(kPageThreads, B - base) - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_off[mid] <= e) lo = mid; else hi = mid - 1;
        }
        const int sb = base + lo, i = e - s_off[lo];
        const int len = min(lens[sb], max_blocks);
        if (mode == 0) {
          blk = tables[(int64_t)sb * max_blocks + len - 1 - i];
        } else {
          blk = i < len ? tables[(int64_t)sb * max_blocks + i] : dtables[(int64_t)sb * dmax_blocks + (i - len)];
        }
      }
      s_blk[threadIdx.x] = blk;
      __syncthreads();
      int push = 0;
      if (e < tot && blk >= 0 && blk < num_blocks) {
        int rank = 1;
        for (int j = 0; j < (int)threadIdx.x; ++j) rank += (s_blk[j] == blk);
        const int r = ref_counts[blk];
        push = rank >= r ? 1 : 0;
      }
      __syncthreads();  // every thread has read ref_counts before the updates below
      int npush;
      const int pos = block_exclusive_scan(push, s_tmp, &npush);
      if (push && s_top + pos < num_blocks) free_list[s_top + pos] = blk;
      // the last event on each block in this batch writes the block's new count
      if (e < tot && blk >= 0 && blk < num_blocks) {
        bool last = true;
        int cnt = 0;
        for (int j = 0; j < min(kEventCap, tot - e0); ++j) {
          if (s_blk[j] == blk) { ++cnt; if (j > (int)threadIdx.x) last = false; }
        }
        if (last) {
          const int r = ref_counts[blk];
          ref_counts[blk] = r > cnt ? r - cnt : 0;
        }
      }
      __syncthreads();
      if (threadIdx.x == 0) s_top += npush;
      __syncthreads();
    }
    // shrink the tables
    if (b < B && n > 0) {
      if (mode == 0) {
        for (int i = used; i < min(lens[b], max_blocks); ++i) tables[(int64_t)b * max_blocks + i] = -1;
        lens[b] = used;
      } else {
        for (int i = 0; i < min(lens[b], max_blocks); ++i) tables[(int64_t)b * max_blocks + i] = -1;
        lens[b] = 0;
        if (dtables) {
          for (int i = 0; i < min(dlens[b], dmax_blocks); ++i) dtables[(int64_t)b * dmax_blocks + i] = -1;
          dlens[b] = 0;
        }
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *free_top = s_top;
  pdl_trigger();
}

// Fork: dst rows dst_row0 .. dst_row0+n-1 (empty tables) take the first
// num_tokens tokens of row src_row -- its full blocks shared (ref count + 1 per
// sharer, absent counting as 1) and, when the last block is partial, a fresh
// block of their own popped from the free-list top in row order.  A row that
// would need a fresh block when none is left is left empty (ok = 0).
__global__ void __launch_bounds__(kPageThreads)
page_fork_kernel(int32_t* tables, int32_t* lens, int max_blocks, int32_t* free_list, int32_t* free_top,
                 int32_t* ref_counts, int num_blocks, int src_row, int dst_row0, int n, int num_tokens,
                 int block_size, uint8_t* ok) {
  __shared__ int s_nok;
  __shared__ uint8_t s_ok[kPageThreads];
  pdl_wait();
  const int full = num_tokens / block_size;
  const bool part = (num_tokens % block_size) != 0;
  const int need = full + (part ? 1 : 0);
  if (threadIdx.x == 0) {
    int top = *free_top;
    int nok = 0;
    for (int i = 0; i < n; ++i) {
      const int d = dst_row0 + i;
      const bool fits = need <= max_blocks && lens[src_row] >= need && (!part || top > 0);
      s_ok[i] = fits ? 1 : 0;
      if (ok) ok[i] = fits ? 1 : 0;
      if (!fits) continue;
      if (part) {
        const int blk = free_list[--top];
        free_list[top] = -1;
        tables[(int64_t)d * max_blocks + full] = blk;
        if (blk >= 0 && blk < num_blocks) ref_counts[blk] += 1;
      }
      lens[d] = need;
      ++nok;
    }
    *free_top = top;
    s_nok = nok;
  }
  __syncthreads();
  const int nok = s_nok;
  // shared full blocks: copy the table prefix into every row that forked, count the sharers
  for (int j = threadIdx.x; j < full && j < max_blocks; j += blockDim.x) {
    const int blk = tables[(int64_t)src_row * max_blocks + j];
    for (int i = 0; i < n; ++i)
      if (s_ok[i]) tables[(int64_t)(dst_row0 + i) * max_blocks + j] = blk;
    if (nok > 0 && blk >= 0 && blk < num_blocks) ref_counts[blk] = max(ref_counts[blk], 1) + nok;
  }
  pdl_trigger();
}

// Copy rows [0, rows) of row src_row's block `full` into each forked row's own
// block `full`, every layer and both planes of pages [2][L][NB][BS][Hkv][D].
template <typename KV>
__global__ void kv_fork_copy_kernel(KV* pages, int num_layers, int num_blocks, int block_size, int hkv, int D,
                                    const int32_t* tables, int max_blocks, int src_row, int dst_row0, int n, int full,
                                    int rows, const uint8_t* ok) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x;       // forked row
  const int lp = blockIdx.y;      // plane * num_layers + layer
  if (ok && !ok[i]) return;
  const int sblk = tables[(int64_t)src_row * max_blocks + full];
  const int dblk = tables[(int64_t)(dst_row0 + i) * max_blocks + full];
  if ((unsigned)sblk >= (unsigned)num_blocks || (unsigned)dblk >= (unsigned)num_blocks) return;
  const int64_t page = (int64_t)block_size * hkv * D;
  const KV* src = pages + ((int64_t)lp * num_blocks + sblk) * page;
  KV* dst = pages + ((int64_t)lp * num_blocks + dblk) * page;
  const int64_t count = (int64_t)rows * hkv * D;
  for (int64_t e = threadIdx.x; e < count; e += blockDim.x) dst[e] = src[e];
}

}  // namespace
}  // namespace ssd

using namespace ssd;

extern "C" int ssd_page_fork(ssd_stream_t stream, int32_t* block_tables, int32_t* table_lens, int max_blocks,
                             int32_t* free_list, int32_t* free_top, int32_t* ref_counts, int num_blocks, int src_row,
                             int dst_row0, int n, int num_tokens, int block_size, uint8_t* ok, void* kv_pages,
                             int dtype, int num_layers, int num_kv_heads, int head_dim) {
  if (n < 0 || max_blocks <= 0 || num_blocks <= 0 || block_size <= 0 || num_tokens < 0 || src_row < 0 ||
      dst_row0 < 0 || (src_row >= dst_row0 && src_row < dst_row0 + n))
    return SSD_ERR_INVALID;
  if (n == 0) return SSD_OK;
  if (!block_tables || !table_lens || !free_list || !free_top || !ref_counts) return SSD_ERR_INVALID;
  if (kv_pages && (num_layers <= 0 || num_kv_heads <= 0 || head_dim <= 0 || !ok)) return SSD_ERR_INVALID;
  if (n > kPageThreads) return SSD_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  SSD_PDL(page_fork_kernel, 1, kPageThreads, 0, st, block_tables, table_lens, max_blocks, free_list, free_top,
          ref_counts, num_blocks, src_row, dst_row0, n, num_tokens, block_size, ok);
  SSD_CHECK_LAUNCH();
  const int rows = num_tokens % block_size;
  if (kv_pages && rows > 0) {
    const int full = num_tokens / block_size;
    dim3 grid(n, 2 * num_layers);
    if (dtype == SSD_DTYPE_BF16)
      SSD_PDL(kv_fork_copy_kernel<bf16>, grid, 256, 0, st, reinterpret_cast<bf16*>(kv_pages), num_layers,
              num_blocks, block_size, num_kv_heads, head_dim, block_tables, max_blocks, src_row, dst_row0, n, full,
              rows, ok);
    else if (dtype == SSD_DTYPE_F32)
      SSD_PDL(kv_fork_copy_kernel<float>, grid, 256, 0, st, reinterpret_cast<float*>(kv_pages), num_layers,
              num_blocks, block_size, num_kv_heads, head_dim, block_tables, max_blocks, src_row, dst_row0, n, full,
              rows, ok);
    else
      return SSD_ERR_INVALID;
    SSD_CHECK_LAUNCH();
  }
  return SSD_OK;
}

extern "C" int ssd_page_allocate(ssd_stream_t stream, int32_t* block_tables, int32_t* table_lens, int max_blocks,
                                 int32_t* free_list, int32_t* free_top, int32_t* ref_counts, int num_blocks,
                                 const int32_t* num_tokens, const int32_t* num_new, uint8_t* ok, int block_size,
                                 int B) {
  if (B < 0 || max_blocks <= 0 || num_blocks <= 0 || block_size <= 0) return SSD_ERR_INVALID;
  if (B == 0) return SSD_OK;
  if (!block_tables || !table_lens || !free_list || !free_top || !ref_counts || !num_tokens || !num_new)
    return SSD_ERR_INVALID;
  SSD_PDL(page_allocate_kernel, 1, kPageThreads, 0, (cudaStream_t)stream, block_tables, table_lens, max_blocks,
                                                                     free_list, free_top, ref_counts, num_blocks,
                                                                     num_tokens, num_new, ok, block_size, B);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

extern "C" int ssd_page_rollback(ssd_stream_t stream, int32_t* block_tables, int32_t* table_lens, int max_blocks,
                                 int32_t* free_list, int32_t* free_top, int32_t* ref_counts, int num_blocks,
                                 const int32_t* num_tokens, const int32_t* accepted, int32_t* kv_lens,
                                 int block_size, int B) {
  if (B < 0 || max_blocks <= 0 || num_blocks <= 0 || block_size <= 0) return SSD_ERR_INVALID;
  if (B == 0) return SSD_OK;
  if (!block_tables || !table_lens || !free_list || !free_top || !ref_counts || !num_tokens || !accepted)
    return SSD_ERR_INVALID;
  SSD_PDL(page_release_kernel, 1, kPageThreads, 0, (cudaStream_t)stream, 
      0, block_tables, table_lens, max_blocks, nullptr, nullptr, 0, free_list, free_top, ref_counts, num_blocks,
      num_tokens, accepted, kv_lens, nullptr, block_size, B);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}

extern "C" int ssd_page_free(ssd_stream_t stream, int32_t* block_tables, int32_t* table_lens, int max_blocks,
                             int32_t* draft_tables, int32_t* draft_lens, int draft_max_blocks, int32_t* free_list,
                             int32_t* free_top, int32_t* ref_counts, int num_blocks, const uint8_t* release, int B) {
  if (B < 0 || max_blocks <= 0 || num_blocks <= 0) return SSD_ERR_INVALID;
  if (B == 0) return SSD_OK;
  if (!block_tables || !table_lens || !free_list || !free_top || !ref_counts || !release) return SSD_ERR_INVALID;
  if (draft_tables && (!draft_lens || draft_max_blocks <= 0)) return SSD_ERR_INVALID;
  SSD_PDL(page_release_kernel, 1, kPageThreads, 0, (cudaStream_t)stream, 
      1, block_tables, table_lens, max_blocks, draft_tables, draft_lens, draft_max_blocks, free_list, free_top,
      ref_counts, num_blocks, nullptr, nullptr, nullptr, release, 1, B);
  SSD_CHECK_LAUNCH();
  return SSD_OK;
}
