// Key-key importance without any caller-supplied or runtime-allocated scratch.
//
// Some callers cannot allocate device memory at the point where they need the
// importance scores: code running inside a memory pool or allocator that must
// not re-enter it, engines that reserve all device memory up front and hand out
// only fixed buffers, or embedders whose host language has no binding for
// cudaMalloc.  nq_score_keykey_noalloc serves them: it runs the same kernels as
// nq_score_keykey, but its scratch lives in a fixed array compiled into this
// library (NQ_NOALLOC_SCRATCH_BYTES per GPU, resident from load until exit).
//
// Notes for users:
//  - The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current).  Make that first call
//    before any stream capture.
//  - Every call on a device shares the one array.  Calls whose work overlaps on
//    the GPU (different streams, or different host threads) race on it and must
//    be serialised by the caller.
//  - The kernels fully overwrite the scratch they read (tile maxima and sums,
//    row statistics, per-head column sums), so nothing is cleared between calls.
//  - The address is cached per device ordinal for the life of the process.  A
//    cudaDeviceReset (or anything else that destroys and recreates the device's
//    primary context) makes the cached address stale: callers that reset a device
//    must not call this entry point on it afterwards.
#include <cmath>
#include <mutex>

#include "../../include/nexusquant_b200.h"
#include "nq_internal.h"

namespace {

// Scratch for one call; the score kernels align their carve-up to 256 bytes.
static __device__ __align__(256) unsigned char g_noalloc_scratch[NQ_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (set up once per device).
nq_status_t scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NQ_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return NQ_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return NQ_ERR_CUDA;
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return NQ_OK;
}

}  // namespace

extern "C" nq_status_t nq_score_keykey_noalloc(const void* k, int32_t in_dtype, int32_t batch, int32_t heads,
                                               int32_t seq, int32_t head_dim, int64_t stride_b, int64_t stride_h,
                                               int64_t stride_t, int32_t obs_window, int32_t head_begin,
                                               int32_t head_end, int32_t per_head, float* out, nq_stream_t stream) {
  if (!k || !out || batch < 0 || heads <= 0 || seq < 0 || obs_window <= 0) return NQ_ERR_INVALID_ARG;
  if (in_dtype < 0 || in_dtype > 2) return NQ_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 96 && head_dim != 128) return NQ_ERR_UNSUPPORTED;
  if (head_begin < 0 || head_end > heads || head_begin >= head_end) return NQ_ERR_INVALID_ARG;
  if (batch == 0 || seq == 0) return NQ_OK;
  const int hr = head_end - head_begin;
  const int n_q = obs_window < seq ? obs_window : seq;
  const size_t sbytes = nq::score_workspace_bytes(batch, hr, n_q, seq);
  const size_t cbytes = per_head ? 0 : (size_t)batch * hr * seq * sizeof(float) + 256;
  if (sbytes + cbytes > (size_t)NQ_NOALLOC_SCRATCH_BYTES) return NQ_ERR_TOO_LARGE;
  void* ws = nullptr;
  const nq_status_t st = scratch_address(&ws);
  if (st != NQ_OK) return st;

  nq::ScoreArgs a{};
  a.q = nullptr; a.k = k; a.in_dtype = in_dtype;
  a.batch = batch; a.q_heads = heads; a.heads = heads; a.n_q = n_q; a.seq = seq; a.head_dim = head_dim;
  a.k_stride_b = stride_b; a.k_stride_h = stride_h; a.k_stride_t = stride_t;
  a.causal = 0; a.q_pos0 = 0; a.head_begin = head_begin; a.head_end = head_end;
  a.scale = static_cast<float>(std::pow(static_cast<double>(head_dim), -0.5));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* colsum = per_head ? out
                           : reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(ws) + sbytes + 255) & ~uintptr_t(255));
  if (nq::launch_score_colsums(a, colsum, ws, sbytes, s) != cudaSuccess) return NQ_ERR_CUDA;
  if (!per_head && nq::launch_reduce_heads(colsum, batch, hr, seq, static_cast<float>(heads), 0, out, s) != cudaSuccess)
    return NQ_ERR_CUDA;
  return NQ_OK;
}
