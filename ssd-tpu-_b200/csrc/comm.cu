// Tensor-parallel plumbing: CUDA IPC mapping of the symmetric heaps and the
// C entry points of the collective projections (the kernels live in
// linear_tc.cu).  No reference counterpart: the reference shards with XLA
// GSPMD (jax_ssd/models/sharding.py:10-31).
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "linear.cuh"

namespace ssd {
namespace {

using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetRangeFn get_range_fn() {
  static GetRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetRangeFn>(f);
  });
  return fn;
}

bool comm_ok(const ssd_comm* c) {
  if (!c || c->world < 1 || c->world > SSD_MAX_TP || c->rank < 0 || c->rank >= c->world) return false;
  for (int r = 0; r < c->world; ++r)
    if (!c->heaps[r]) return false;
  if (c->ctrl_offset % 256 || c->ctrl_offset + kCommCtrlBytes > c->heap_bytes) return false;
  return true;
}

CollArgs coll_args(const ssd_comm* c, int mode) {
  CollArgs a{};
  a.mode = mode;
  a.rank = c->rank;
  a.world = c->world;
  for (int r = 0; r < kMaxTP; ++r) a.heaps[r] = r < c->world ? reinterpret_cast<char*>(c->heaps[r]) : nullptr;
  a.ctrl_off = c->ctrl_offset;
  return a;
}

}  // namespace

static_assert(SSD_MAX_TP == kMaxTP, "SSD_MAX_TP mismatch");

int linear_allreduce_impl(cudaStream_t st, const void* x, const void* w, void* y, int M, int N, int K, void* ws,
                          size_t ws_bytes, const ssd_comm* c) {
  if (!comm_ok(c) || !x || !w || !y || M <= 0 || N <= 0 || K <= 0) return SSD_ERR_INVALID;
  const int tiles = (N + 127) / 128;
  if (M > c->recv_rows || tiles > c->recv_tiles || c->recv_offset % 256 ||
      ssd_comm_recv_bytes(c->world, c->recv_rows, c->recv_tiles * 128) > c->recv_bytes ||
      c->recv_offset + c->recv_bytes > c->heap_bytes)
    return SSD_ERR_INVALID;
  CollArgs a = coll_args(c, COLL_ALLREDUCE);
  a.dst_off = c->recv_offset;
  a.recv_rows = c->recv_rows;
  a.recv_tiles = c->recv_tiles;
  if (c->allreduce_form < SSD_ALLREDUCE_AUTO || c->allreduce_form > SSD_ALLREDUCE_OWNER) return SSD_ERR_INVALID;
  a.form = c->allreduce_form;
  return linear_tc_coll(st, x, w, y, M, N, K, ws, ws_bytes, a);
}

int linear_allgather_impl(cudaStream_t st, const void* x, const void* w, float* y, int ldy, int M, int N, int K,
                          void* ws, size_t ws_bytes, const ssd_comm* c) {
  if (!comm_ok(c) || !x || !w || !y || M <= 0 || N <= 0 || K <= 0) return SSD_ERR_INVALID;
  if ((int64_t)N * c->world > ldy) return SSD_ERR_INVALID;
  const char* own = reinterpret_cast<const char*>(c->heaps[c->rank]);
  const char* yp = reinterpret_cast<const char*>(y);
  if (yp < own || (reinterpret_cast<uintptr_t>(y) & 3)) return SSD_ERR_INVALID;
  const size_t off = (size_t)(yp - own);
  if (off + sizeof(float) * (size_t)M * ldy > c->heap_bytes) return SSD_ERR_INVALID;
  CollArgs a = coll_args(c, COLL_ALLGATHER);
  a.dst_off = off;
  a.ldy = ldy;
  a.col_off = c->rank * N;
  return linear_tc_coll(st, x, w, nullptr, M, N, K, ws, ws_bytes, a);
}

}  // namespace ssd

using namespace ssd;

extern "C" size_t ssd_comm_ctrl_bytes(void) { return align_up256(kCommCtrlBytes); }

extern "C" size_t ssd_comm_recv_bytes(int world, int max_m, int max_n) {
  if (world <= 0 || max_m <= 0 || max_n <= 0) return 0;
  const size_t tiles = (size_t)(max_n + 127) / 128;  // slots [2][tiles][world][max_m][128] of 64-bit words
  return align_up256(sizeof(uint64_t) * 2 * tiles * world * (size_t)max_m * 128);
}

extern "C" int ssd_ipc_export(const void* ptr, void* handle, size_t* offset) {
  if (!ptr || !handle || !offset) return SSD_ERR_INVALID;
  GetRangeFn fn = get_range_fn();
  if (!fn) return SSD_ERR_LAUNCH;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return SSD_ERR_INVALID;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) {
    cudaGetLastError();
    return SSD_ERR_LAUNCH;
  }
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = (size_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return SSD_OK;
}

extern "C" int ssd_ipc_import(const void* handle, size_t offset, void** ptr) {
  if (!handle || !ptr) return SSD_ERR_INVALID;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return SSD_ERR_LAUNCH;
  }
  *ptr = reinterpret_cast<char*>(base) + offset;
  return SSD_OK;
}

extern "C" int ssd_ipc_close(void* ptr, size_t offset) {
  if (!ptr) return SSD_ERR_INVALID;
  if (cudaIpcCloseMemHandle(reinterpret_cast<char*>(ptr) - offset) != cudaSuccess) {
    cudaGetLastError();
    return SSD_ERR_LAUNCH;
  }
  return SSD_OK;
}

extern "C" int ssd_linear_allreduce(ssd_stream_t stream, const void* x, const void* w, void* y, int M, int N, int K,
                                    void* workspace, size_t workspace_bytes, const ssd_comm* comm) {
  return linear_allreduce_impl((cudaStream_t)stream, x, w, y, M, N, K, workspace, workspace_bytes, comm);
}

extern "C" int ssd_linear_allgather(ssd_stream_t stream, const void* x, const void* w, float* y, int ldy, int M,
                                    int N, int K, void* workspace, size_t workspace_bytes, const ssd_comm* comm) {
  return linear_allgather_impl((cudaStream_t)stream, x, w, y, ldy, M, N, K, workspace, workspace_bytes, comm);
}
