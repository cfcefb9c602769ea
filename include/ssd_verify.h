/*
 * ssd_verify.h — C ABI of the B200 (sm_100a) speculative-decoding verify path.
 *
 * Conventions (all entry points):
 *   - Every pointer argument is DEVICE memory unless the comment says "host".
 *   - Calls are stream-ordered on `stream` and never allocate device memory:
 *     buffers, including `workspace`, are owned by the caller.
 *   - Workspaces must be zero-filled once when the caller allocates them; every
 *     call leaves its workspace zero-filled again (self-resetting counters), so a
 *     workspace can be reused by later calls on the same stream.  Calls that
 *     share one workspace must not overlap on the GPU.
 *   - Return value: SSD_OK (0) or an SSD_ERR_* code; invalid sizes are rejected
 *     on the host before any launch.
 *   - bf16 tensors are passed as `ssd_bf16` (raw bfloat16 bits); `dtype`
 *     selects SSD_DTYPE_BF16 or SSD_DTYPE_F32 storage where both exist.
 *
 * Citations are to TinevimboMusingadi/ssd-tpu- (paths within that project).
 */
#ifndef SSD_VERIFY_H_
#define SSD_VERIFY_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct CUstream_st* ssd_stream_t; /* == cudaStream_t */
typedef uint16_t ssd_bf16;

enum {
  SSD_OK = 0,
  SSD_ERR_INVALID = 1,     /* bad size / null pointer / unsupported shape */
  SSD_ERR_LAUNCH = 2,      /* CUDA launch error */
  SSD_ERR_TIMEOUT = 3,     /* a bounded device-side wait gave up */
  SSD_ERR_UNSUPPORTED = 4, /* shape outside the compiled kernel limits */
  SSD_ERR_WORKSPACE = 5    /* workspace too small */
};

enum { SSD_DTYPE_BF16 = 0, SSD_DTYPE_F32 = 1 };

/* Human-readable text for a status code (static storage). */
const char* ssd_status_string(int status);
/* ABI version: (major << 16) | minor. */
int ssd_abi_version(void);

/* ------------------------------------------------------------------ K4: acceptance */

/* Workspace bytes for ssd_verify_greedy / ssd_argmax_rows. */
size_t ssd_verify_greedy_workspace_size(int B, int K, int V);

/*
 * Greedy verification over K+1 positions.
 * Replaces jax_ssd/algorithm/verify.py:18-59 (verify_greedy) and
 * reference/cuda_ssd/verify_torch.py:8-45.
 *   logits_p      [B, K+1, V] fp32 target logits
 *   speculations  [B, K+1] int32; column 0 = previous recovery, 1..K = draft
 *   accept_until  [B] int32 out: leading draft tokens equal to the target argmax
 *   recovery      [B] int32 out: target argmax at position accept_until
 *   accepted_mask [B, K+1] uint8 out (may be NULL): [b,0]=0, [b,j+1]=(j<accept_until)
 *   target_tokens [B, K+1] int32 out (may be NULL): argmax of every row
 * argmax ties resolve to the first index.  0 <= K <= 63 (else SSD_ERR_INVALID).
 */
int ssd_verify_greedy(ssd_stream_t stream, const float* logits_p, const int32_t* speculations,
                      int32_t* accept_until, int32_t* recovery, uint8_t* accepted_mask,
                      int32_t* target_tokens, void* workspace, size_t workspace_bytes, int B, int K,
                      int V);

/*
 * ssd_verify_greedy without a workspace argument, for callers that cannot
 * allocate device memory (an XLA custom call handed only its operands,
 * embedders with a fixed device-memory budget).  No
 * counterpart in the reference: it is an addition of this library.
 * Outputs and argument meaning are those of ssd_verify_greedy; it allocates
 * nothing.  Its scratch is a 34 KB array in the library's device data that
 * every GPU loading the library holds until exit.  Limits: B*(K+1) <= 512
 * (larger calls return SSD_ERR_UNSUPPORTED).  Every call looks up the array's
 * device address on the caller's current device (no address is cached, so a
 * device reset leaves nothing stale); call it with the device of `stream`
 * current.  All calls share the array, so calls
 * that overlap on the GPU (different streams, or different host threads
 * without ordering) race and give wrong results.
 */
int ssd_verify_greedy_noalloc(ssd_stream_t stream, const float* logits_p,
                              const int32_t* speculations, int32_t* accept_until,
                              int32_t* recovery, uint8_t* accepted_mask, int32_t* target_tokens,
                              int B, int K, int V);

/*
 * Row-wise argmax (first index on ties) of x[rows, V] (row stride `ld`
 * elements), e.g. the draft's greedy token.  Replaces the jnp.argmax calls of
 * jax_ssd/runtime/engine.py:224 and jax_ssd/models/gemma_adapter.py:127.
 * Uses the ssd_verify_greedy workspace sizing with B=rows, K=0.
 */
int ssd_argmax_rows(ssd_stream_t stream, const float* x, int64_t ld, int rows, int V, int32_t* out,
                    void* workspace, size_t workspace_bytes);

/*
 * Row-wise sample from softmax(x[r] / temperature) (temperature > 0), e.g. the
 * draft token of sampled speculative decoding (the reference drafts greedily,
 * jax_ssd/models/gemma_adapter.py:127; sampled drafting is what verify_sample,
 * jax_ssd/algorithm/verify.py:68-120, assumes).  Gumbel-max: out[r] = argmax_j
 * (x[r][j] / temperature - log(-log(u))), u from a counter hash at
 * (seed, offset + r * V + j), so the draw is reproducible and no noise buffer
 * is read.  rows <= 16384.  Uses the ssd_verify_greedy workspace sizing with B=rows, K=0.
 */
int ssd_sample_rows(ssd_stream_t stream, const float* x, int64_t ld, int rows, int V, float temperature,
                    uint64_t seed, uint64_t offset, int32_t* out, void* workspace, size_t workspace_bytes);

/*
 * Top-p (nucleus) filter of softmax(x[r] / temperature), in place: every
 * logit below the row's cutoff t* (and every NaN) becomes -inf, so the
 * sampling and acceptance kernels above see the renormalised nucleus.  t* is
 * the largest logit value whose cumulative mass -- over all logits >= it,
 * ties included, fp64 masses exp((x - max) / temperature) -- reaches
 * top_p * Z.  top_p >= 1 leaves the rows untouched; V < 524288.  Not in the reference (its
 * SamplingParams has no top-p); the batched serving workload (T = 1.0,
 * top-p 0.95) asks for it.  No workspace.
 */
int ssd_top_p_mask(ssd_stream_t stream, float* x, int64_t ld, int rows, int V, float temperature, float top_p);

/* Workspace bytes for ssd_verify_sample. */
size_t ssd_verify_sample_workspace_size(int B, int K, int V);

enum { SSD_ALIGN_REFERENCE = 0, SSD_ALIGN_STANDARD = 1 };

/*
 * Sampling-mode verification (rejection sampling, bonus token, residual).
 * Replaces jax_ssd/algorithm/verify.py:68-120 (verify_sample, _verify_sample_row)
 * with the JAX threefry draws replaced by explicit uniforms:
 *   u_accept [B, K] in [0,1): draft token j is accepted iff u < min(1, p/max(q,1e-12))
 *   u_gumbel [B, V] in (0,1): categorical draw = argmax(log(r + 1e-12) - log(-log u))
 *   logits_q [B, K, V] fp32 draft logits; temperatures must be > 0; 0 <= K <= 63.
 *   alignment SSD_ALIGN_REFERENCE judges draft token j+1 with target row j+1
 *   (verify.py:103 as written); SSD_ALIGN_STANDARD uses row j.
 *   K = 0 (as the reference allows): nothing is accepted and every row draws its
 *   bonus token from softmax(lp[0] / Tp); logits_q and u_accept may then be NULL.
 */
int ssd_verify_sample(ssd_stream_t stream, const float* logits_p, const float* logits_q,
                      const int32_t* speculations, const float* u_accept, const float* u_gumbel,
                      float temperature_p, float temperature_q, float sampler_x, int alignment,
                      int32_t* accept_until, int32_t* recovery, uint8_t* accepted_mask,
                      void* workspace, size_t workspace_bytes, int B, int K, int V);

/*
 * Fill out[n] with counter-based uniforms in (0,1): a stateless hash of
 * (seed, offset + i).  Stands in for jax.random.split/uniform
 * (jax_ssd/algorithm/verify.py:80,100,107) when the caller passes a seed.
 */
int ssd_uniform_fill(ssd_stream_t stream, float* out, int64_t n, uint64_t seed, uint64_t offset);

/* ---------------------------------------------------------- K5: paged-KV blocks */
/*
 * Device mirror of the host page manager (jax_ssd/runtime/page_manager.py).
 * State: block_tables [B, max_blocks] int32 (unused entries -1), table_lens [B],
 * free_list [num_blocks] used as a stack free_list[0:*free_top] (pop/push at the
 * top, i.e. the END of the reference's Python list), ref_counts [num_blocks]
 * (0 = absent from the reference's dict).  Sequences are processed in index
 * order, exactly as successive per-sequence calls of the reference.
 */

/* PageManager.allocate / allocate_draft (page_manager.py:21-47): grow each table to
 * ceil((num_tokens+num_new)/block_size) blocks popped from the free-list top;
 * a sequence that does not fit is left unchanged and gets ok[b]=0. */
int ssd_page_allocate(ssd_stream_t stream, int32_t* block_tables, int32_t* table_lens,
                      int max_blocks, int32_t* free_list, int32_t* free_top, int32_t* ref_counts,
                      int num_blocks, const int32_t* num_tokens, const int32_t* num_new,
                      uint8_t* ok, int block_size, int B);

/* PageManager.rollback_speculative (page_manager.py:49-56, _free_block :66-70):
 * pop blocks from the END of each table while len > ceil((num_tokens+accepted)/bs);
 * each popped block's ref count drops (absent counts as 1) and at 0 it is pushed
 * on the free list.  kv_lens (may be NULL) receives num_tokens+accepted, the
 * truncated valid KV length. */
int ssd_page_rollback(ssd_stream_t stream, int32_t* block_tables, int32_t* table_lens,
                      int max_blocks, int32_t* free_list, int32_t* free_top, int32_t* ref_counts,
                      int num_blocks, const int32_t* num_tokens, const int32_t* accepted,
                      int32_t* kv_lens, int block_size, int B);

/* PageManager.free_sequence (page_manager.py:58-64) for every b with
 * release[b] != 0: target table in forward order, then the draft table
 * (draft_tables may be NULL). */
int ssd_page_free(ssd_stream_t stream, int32_t* block_tables, int32_t* table_lens, int max_blocks,
                  int32_t* draft_tables, int32_t* draft_lens, int draft_max_blocks,
                  int32_t* free_list, int32_t* free_top, int32_t* ref_counts, int num_blocks,
                  const uint8_t* release, int B);

/*
 * Fork for branch decoding (async SSD fan-out; the reference builds dense branch
 * masks instead, jax_ssd/kernels/masks.py:8-30, pallas_attention.py:16-35):
 * rows dst_row0 .. dst_row0+n-1 (empty tables, n <= 1024) take the first
 * num_tokens tokens of row src_row.  Its full blocks are shared (ref count + 1
 * per sharer, absent counting as 1, as page_manager.py:66-70 reads it); when the
 * last block is partial each row gets a fresh block popped from the free-list top
 * in row order, and (kv_pages != NULL) the partial block's first num_tokens %
 * block_size rows are copied into it for every layer and both planes.  A row that
 * cannot get its block is left empty with ok[i] = 0 (ok is required with kv_pages).
 * Paged attention over the forked rows then sees the trunk plus each branch's own
 * tokens -- the branch mask -- with no trunk copy.  Releasing a forked row with
 * ssd_page_free decrements the shared counts.
 */
int ssd_page_fork(ssd_stream_t stream, int32_t* block_tables, int32_t* table_lens, int max_blocks,
                  int32_t* free_list, int32_t* free_top, int32_t* ref_counts, int num_blocks,
                  int src_row, int dst_row0, int n, int num_tokens, int block_size, uint8_t* ok,
                  void* kv_pages, int dtype, int num_layers, int num_kv_heads, int head_dim);

/* ------------------------------------------------------------ speculation cache */
/*
 * SpecCache.lookup (jax_ssd/algorithm/spec_cache.py:43-66) on the device.
 *   keys [N,3] int32, valid [N] uint8, tokens [N,K] int32, logits [N,K,V] fp32 (may be
 *   NULL when out_logits is NULL); request_keys [B,3].
 *   hit [B] uint8, idx [B] int32 (-1 on a miss), out_tokens [B,K] (0 on a miss),
 *   out_logits [B,K,V] (may be NULL; zeros on a miss).
 * A request hits the first valid slot whose three key fields all match.
 */
int ssd_spec_cache_lookup(ssd_stream_t stream, const int32_t* keys, const uint8_t* valid,
                          const int32_t* tokens, const float* logits, int N, int K, int V,
                          const int32_t* request_keys, int B, uint8_t* hit, int32_t* idx,
                          int32_t* out_tokens, float* out_logits);

/* --------------------------------------------------------------- K2: KV write */
/*
 * Write K/V rows of new tokens into the paged cache.
 * Replaces jax_ssd/kernels/kv_cache.py:39-58 (write_kv_slots); layout
 * kv_cache.py:13,28-31: pages [2, num_layers, num_blocks, block_size, Hkv, D].
 *   positions [B, T] int32 (-1 = skip); slot = block_tables[b][p/bs]*bs + p%bs
 *   k, v      [B, T, Hkv, D] in the cache dtype
 */
int ssd_kv_write(ssd_stream_t stream, void* pages, int dtype, int num_layers, int num_blocks,
                 int block_size, int num_kv_heads, int head_dim, int layer,
                 const int32_t* block_tables, int max_blocks, const int32_t* positions,
                 const void* k, const void* v, int B, int T);

/* --------------------------------------------------- K1: paged verify attention */

size_t ssd_paged_attention_workspace_size(int B, int T, int num_heads, int num_kv_heads,
                                          int head_dim, int max_seq_len);

/*
 * Multi-query attention of each sequence's new tokens against its pages.
 * Replaces jax_ssd/kernels/attention_ref.py:9-21 with the mask of
 * jax_ssd/kernels/masks.py:33-40 and the page layout of kv_cache.py:13.
 *   q        [B, T, Hq, D]; out [B, T, Hq, D] (cache dtype)
 *   seq_lens [B]: cached tokens INCLUDING the new ones (already written)
 *   q_lens   [B] or NULL (= T): valid new tokens; new token t sits at position
 *            seq_lens[b] - q_lens[b] + t and sees positions 0..that position.
 *   GQA: query head h reads KV head h / (Hq / Hkv).  max_seq_len bounds seq_lens.
 *   Rows t >= q_lens[b] are written as zeros.
 */
int ssd_paged_verify_attention(ssd_stream_t stream, const void* q, const void* pages, int dtype,
                               int num_layers, int num_blocks, int block_size, int num_kv_heads,
                               int head_dim, int layer, const int32_t* block_tables, int max_blocks,
                               const int32_t* seq_lens, const int32_t* q_lens, void* out,
                               float scale, int B, int T, int num_heads, int max_seq_len,
                               void* workspace, size_t workspace_bytes);

/* ------------------------------------------------------- K3: skinny projections */

enum {
  SSD_EPI_STORE = 0,     /* y[M,N] = x w^T in the activation dtype */
  SSD_EPI_STORE_F32 = 1, /* y[M,N] fp32 (logits) */
  SSD_EPI_RESIDUAL = 2,  /* y[M,N] (in/out) = round(y + round(x w^T)) */
  SSD_EPI_GEGLU = 3      /* w rows interleaved (gate_i, up_i): y[M,N/2] =
                            round(round(gelu_tanh(round(g))) * round(u)) */
};

size_t ssd_linear_workspace_size(int M, int N, int K);
/* Largest M (tokens x sequences) one ssd_linear / ssd_gemma_forward call takes. */
int ssd_linear_max_m(void);

/*
 * y = epilogue(x[M,K] w[N,K]^T) with fp32 accumulation; w row-major like the
 * reference's Gemma projections (HF Flax Gemma, called from
 * jax_ssd/models/gemma_adapter.py:81-102).
 */
int ssd_linear(ssd_stream_t stream, const void* x, const void* w, int dtype, void* y,
               int epilogue, int M, int N, int K, void* workspace, size_t workspace_bytes);

/*
 * Projection of RMS-normalised token rows with the norm weight folded into w:
 * y = epilogue(rsqrt(mean(x[m]^2) + eps) * (x[m] w^T)), where w = W * (1 + g)
 * column-wise for the Gemma RMSNorm weight g.  Fuses the input / MLP RMSNorm of
 * jax_ssd/models/gemma_adapter.py:81-102 (HF Gemma) into the QKV and gate/up
 * projections.  Epilogues: SSD_EPI_STORE, SSD_EPI_STORE_F32, SSD_EPI_GEGLU.
 * Uses the ssd_linear_workspace_size workspace.
 */
int ssd_linear_rownorm(ssd_stream_t stream, const void* x, const void* w, int dtype, void* y,
                       int epilogue, int M, int N, int K, float eps, void* workspace,
                       size_t workspace_bytes);

/* ------------------------------------------------------------ tensor parallelism */
/*
 * Tensor-parallel projections with the collective fused into the projection
 * kernel (no reference counterpart: the reference shards with XLA GSPMD,
 * jax_ssd/models/sharding.py:10-31, and its collectives are XLA's).  One
 * process per GPU; every rank owns a "symmetric heap" -- a device buffer of the
 * same size, carved identically on every rank -- and maps every peer's heap
 * into its address space (ssd_ipc_export / ssd_ipc_import, CUDA IPC over
 * NVLink).  The kernels store fp32 tiles straight into the peers' heaps and
 * signal per-tile arrival flags held in each heap's control block.
 * All ranks must issue the same collective calls in the same order on one
 * stream each; a rank that is more than about 5 s late makes the others give up,
 * record SSD_ERR_TIMEOUT in word 2 of their control block and finish with
 * incomplete results (nothing hangs).  The control block also holds per-tile
 * delivery counts and flags (device state, so CUDA graphs replay the calls).
 */
#define SSD_MAX_TP 8
typedef struct {
  int rank, world;                 /* this rank, ranks in the group (1..SSD_MAX_TP) */
  void* heaps[SSD_MAX_TP];         /* heap of rank r as mapped in this process; heaps[rank] = own */
  size_t heap_bytes;               /* size of every rank's heap */
  size_t ctrl_offset;              /* control block (ssd_comm_ctrl_bytes), zero-filled before first use */
  size_t recv_offset, recv_bytes;  /* all-reduce receive area (>= ssd_comm_recv_bytes) */
  int recv_rows, recv_tiles;       /* its shape: the max_m and ceil(max_n / 128) it was sized for */
  int allreduce_form;              /* SSD_ALLREDUCE_AUTO (0), _ALL_TO_ALL or _OWNER; same on every rank */
} ssd_comm;
/* Forms of the fused all-reduce (ssd_linear_allreduce); every form gives the same bits. */
enum { SSD_ALLREDUCE_AUTO = 0, SSD_ALLREDUCE_ALL_TO_ALL = 1, SSD_ALLREDUCE_OWNER = 2 };

/* Bytes of the control block (multiple of 256). */
size_t ssd_comm_ctrl_bytes(void);
/* Bytes of the all-reduce receive area for projections of up to max_m x max_n outputs. */
size_t ssd_comm_recv_bytes(int world, int max_m, int max_n);

/* CUDA IPC: a 64-byte handle of the allocation holding `ptr` and ptr's offset in it. */
int ssd_ipc_export(const void* ptr, void* handle, size_t* offset);
/* Map a peer's exported buffer: *ptr = mapped allocation + offset. */
int ssd_ipc_import(const void* handle, size_t offset, void** ptr);
/* Unmap a buffer mapped by ssd_ipc_import. */
int ssd_ipc_close(void* ptr, size_t offset);


/*
 * Row-parallel projection + all-reduce + residual (the O and down projections
 * of a tensor-parallel layer): y[M,N] += round_bf16(sum over ranks r, in rank
 * order, of x_r[M,K] w_r[N,K]^T), where x_r / w_r are rank r's column shards.
 * bf16 only; every rank ends with bit-identical y.  Uses the
 * ssd_linear_workspace_size(M, N, K) workspace.
 * Forms (comm->allreduce_form): ALL_TO_ALL -- every rank sends each fp32 partial
 * to every rank, which folds all of them (one hop); OWNER -- each partial goes to
 * the output tile's owner rank (tile % world) only, which folds and sends the sum
 * to the others (two hops, about 2/world of the bytes); AUTO takes OWNER where it
 * saves more than 4 MB per rank and M > 16, else ALL_TO_ALL.
 */
int ssd_linear_allreduce(ssd_stream_t stream, const void* x, const void* w, void* y, int M, int N, int K,
                         void* workspace, size_t workspace_bytes, const ssd_comm* comm);

/*
 * Column-parallel projection + all-gather (the vocab-parallel LM head):
 * y[m, rank*N + n] = x[m] . w[n] in fp32, written into y on every rank.  y is a
 * [M, ldy] fp32 buffer inside the heap, at the same offset on every rank; when
 * the call's kernel ends, every rank's columns are present.  bf16 only.
 */
int ssd_linear_allgather(ssd_stream_t stream, const void* x, const void* w, float* y, int ldy, int M, int N,
                         int K, void* workspace, size_t workspace_bytes, const ssd_comm* comm);

/* ------------------------------------------------ fused small ops of the forward */

/* x[m] = round(embed[tokens[m]] * round(sqrt(d))) ; tokens [M] int32 */
int ssd_embed(ssd_stream_t stream, const int32_t* tokens, const void* embed, int dtype, void* x,
              int M, int d, int vocab);
/* y[m] = round(x * rsqrt(mean(x^2) + eps) * (1 + w)) (Gemma RMSNorm) */
int ssd_rmsnorm(ssd_stream_t stream, const void* x, const void* w, int dtype, void* y, int M,
                int d, float eps);
/*
 * RoPE (rotate-half, table cos/sin [max_pos, D/2] fp32) on the q and k parts
 * of qkv [B*T, (Hq+2Hkv)*D], q written to q_out [B*T, Hq, D], rotated k and v
 * written into the pages (fused K2).  positions as in ssd_kv_write.
 */
int ssd_rope_kv_write(ssd_stream_t stream, const void* qkv, void* q_out, void* pages, int dtype,
                      int num_layers, int num_blocks, int block_size, int num_heads,
                      int num_kv_heads, int head_dim, int layer, const int32_t* block_tables,
                      int max_blocks, const int32_t* positions, const float* rope_cos,
                      const float* rope_sin, int rope_max_pos, int B, int T);

/* --------------------------------------------------- whole-model verify forward */

typedef struct {
  int num_layers, d_model, num_heads, num_kv_heads, head_dim, ffn, vocab;
  float eps;
  int dtype;                       /* storage dtype of weights, activations and KV */
  const void* embed;               /* [vocab, d] (tied LM head) */
  const void* final_norm;          /* [d] */
  /* The input and MLP RMSNorm weights are folded into the projections that
   * consume them: w_qkv = W_qkv * (1 + attn_norm) and w_gate_up = W_gu *
   * (1 + mlp_norm), column-wise, rounded to the storage dtype. */
  const void* const* w_qkv;        /* host array [L] of device [(Hq+2Hkv)*D, d] */
  const void* const* w_o;          /* host array [L] of device [d, Hq*D] */
  const void* const* w_gate_up;    /* host array [L] of device [2F, d], rows (gate_i, up_i) */
  const void* const* w_down;       /* host array [L] of device [d, F] */
  const float* rope_cos;           /* [rope_max_pos, D/2] */
  const float* rope_sin;
  int rope_max_pos;
  /* Tensor parallelism: with tp_world > 1 the struct describes rank tp_rank's
   * shard -- num_heads, num_kv_heads and ffn are per-rank counts (a single KV
   * head is replicated), w_o / w_down hold the matching column blocks, vocab is
   * the full vocabulary and embed the full (replicated) table, whose rows
   * [tp_rank*vocab/tp_world, ...) are this rank's LM-head block. */
  int tp_rank, tp_world;
  /* 1: within every q and k head of w_qkv the rows are stored as rotation
   * pairs -- row 2i holds dimension i, row 2i+1 dimension i + D/2 (v rows
   * unchanged) -- and the forward applies RoPE and writes the K/V rows in the
   * QKV projection's epilogue (bf16 weights only).  0: canonical row order and
   * the separate ssd_rope_kv_write step. */
  int qk_pairs;
} ssd_gemma_weights;

typedef struct {
  int B, T;                        /* sequences, new tokens per sequence (padded) */
  const int32_t* tokens;           /* [B, T] */
  const int32_t* seq_lens_before;  /* [B] tokens already cached */
  const int32_t* q_lens;           /* [B] valid new tokens, or NULL (= T) */
  void* kv_pages;                  /* [2, L, num_blocks, block_size, Hkv, D] */
  int num_blocks, block_size;
  const int32_t* block_tables;     /* [B, max_blocks] */
  int max_blocks;
  int max_seq_len;                 /* bound on seq_lens_before + T */
  float* logits;                   /* [B, T, V] fp32, [B, V] with logits_last_only, or NULL
                                      (prompt chunks: K/V only, no final norm / LM head) */
  int logits_last_only;            /* 1: logits of each sequence's last valid token only */
  void* scratch;                   /* activations + workspaces, zero-filled once */
  size_t scratch_bytes;
  /* Optional launch timing of the projections (all NULL/0 to disable): host
   * array of 2*prof_capacity cudaEvent_t; event 2i / 2i+1 are recorded on
   * `stream` around the i-th projection, prof_kind[i] names it (0 qkv, 1 o,
   * 2 gate_up, 3 down, 4 lm_head) and *prof_count receives the number used. */
  void* const* prof_events;
  int prof_capacity;
  int* prof_count;
  int* prof_kind;
  /* Tensor parallelism (NULL: none).  When set, the O and down projections
   * run as ssd_linear_allreduce and the LM head as ssd_linear_allgather, so
   * `logits` must lie in comm's heap, at the same offset on every rank. */
  const ssd_comm* comm;
} ssd_gemma_batch;

size_t ssd_gemma_scratch_size(const ssd_gemma_weights* w, int B, int T, int max_seq_len);

/*
 * Target (or draft) forward over the new tokens of B sequences against the paged
 * cache: writes their K/V rows and the fp32 logits.  Replaces
 * DecodeModelAdapter.verify/prefill/decode (jax_ssd/models/base.py:34-58) as
 * implemented by GemmaAdapter (jax_ssd/models/gemma_adapter.py:81-143).
 * `w` and the pointer arrays it holds are host memory read during the call.
 */
int ssd_gemma_forward(ssd_stream_t stream, const ssd_gemma_weights* w, const ssd_gemma_batch* b);

/* Seeded N(0, std^2) init of n elements (counter-based hash + Box-Muller). */
int ssd_normal_fill(ssd_stream_t stream, void* out, int dtype, int64_t n, float std, uint64_t seed);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#ifdef __cplusplus
}
#endif

#endif /* SSD_VERIFY_H_ */
