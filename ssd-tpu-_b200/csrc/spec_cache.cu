// Speculation-cache lookup on the device (jax_ssd/algorithm/spec_cache.py:43-66).
//
// A request key [seq_id, accepted_index, recovery_token] hits the FIRST valid
// slot whose key matches in all three fields; hits copy that slot's draft tokens
// (and, when requested, its draft logits) into the outputs, misses write -1 /
// zeros.  One warp per request scans the slots (lane-strided, min-index
// reduction); the logits copy is a grid-stride loop over the hit rows.
#include "common.cuh"

namespace ssd {
namespace {

__global__ void spec_lookup_kernel(const int32_t* keys, const uint8_t* valid, int N,
                                   const int32_t* req, int B, const int32_t* tokens, int K,
                                   uint8_t* hit, int32_t* idx,
                                   int32_t* out_tokens) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= B) return;
  const int a = req[warp * 3], c = req[warp * 3 + 1], d = req[warp * 3 + 2];
  int best = 0x7fffffff;
  for (int i = lane; i < N; i += 32)
    if (valid[i] && keys[i * 3] == a && keys[i * 3 + 1] == c && keys[i * 3 + 2] == d) { best = i; break; }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
  const bool h = best != 0x7fffffff;
  if (lane == 0) {
    hit[warp] = h ? 1 : 0;
    idx[warp] = h ? best : -1;
  }
  for (int j = lane; j < K; j += 32) out_tokens[(int64_t)warp * K + j] = h ? tokens[(int64_t)best * K + j] : 0;
}

__global__ void spec_gather_logits_kernel(const float* logits, int64_t row, const int32_t* idx,
                                          int B, float* out) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = (int64_t)B * row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / row);
    const int s = idx[b];
    out[i] = s >= 0 ? logits[(int64_t)s * row + (i % row)] : 0.f;
  }
}

}  // namespace
}  // namespace ssd

using namespace ssd;

extern "C" int ssd_spec_cache_lookup(ssd_stream_t stream, const int32_t* keys, const uint8_t* valid,
                                     const int32_t* tokens, const float* logits, int N, int K, int V,
                                     const int32_t* request_keys, int B, uint8_t* hit, int32_t* idx,
                                     int32_t* out_tokens, float* out_logits) {
  if (N <= 0 || K <= 0 || B < 0 || !keys || !valid || !tokens || !request_keys || !hit || !idx || !out_tokens)
    return SSD_ERR_INVALID;
  if (B == 0) return SSD_OK;
  if (out_logits && (!logits || V <= 0)) return SSD_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  const int warps_per_block = 4;
  SSD_PDL(spec_lookup_kernel, (B + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, st, keys, valid,
          N, request_keys, B, tokens, K, hit, idx, out_tokens);
  if (out_logits) {
    const int64_t row = (int64_t)K * V;
    int64_t blocks = ((int64_t)B * row + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    SSD_PDL(spec_gather_logits_kernel, (unsigned)blocks, 256, 0, st, logits, row, idx, B, out_logits);
  }
  return SSD_OK;
}
