// Keep-set selection (nexusquant/pipeline.py:895-959, _build_keep_mask):
// BOS + last `sliding_window` tokens + top-n_keep of importance[1:prefix]
// + protected positions, emitted as ascending token indices.
//
// One CTA per batch row.  The top-k threshold is found with an MSB-first radix
// select over order-preserving 32-bit keys of the fp32 scores (4 passes of 8
// bits, per-warp histograms in shared memory).  Ties at the threshold are
// resolved toward the lower index.  The compaction is a two-pass segmented
// scan: each thread owns a contiguous run of tokens, so the output order is
// the token order.
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ bool is_protected(const int32_t* prot, int n, int t) {
  int lo = 0, hi = n - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    const int v = prot[mid];
    if (v == t) return true;
    if (v < t) lo = mid + 1; else hi = mid - 1;
  }
  return false;
}

// Exclusive block scan of one int per thread; returns the total in *total.
__device__ int block_exclusive_scan(int v, int* sh, int* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int s = lane < kSelWarps ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    sh[lane] = s;  // inclusive warp totals
  }
  __syncthreads();
  const int before = (wid > 0 ? sh[wid - 1] : 0) + x - v;
  *total = sh[kSelWarps - 1];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(kSelThreads) select_kernel(const float* imp, int seq, int sw, int n_keep,
                                                             const int32_t* prot, int n_prot, int32_t* kept_idx,
                                                             int32_t* kept_count) {
  __shared__ uint32_t hist[kSelWarps][256];
  __shared__ uint32_t tot[256];
  __shared__ uint32_t s_pref, s_rem;
  __shared__ int scan_sh[32];
  const int b = blockIdx.x;
  const float* x = imp + (int64_t)b * seq;
  const int prefix = max(seq - sw, 0);
  const int k = (prefix > 1 && n_keep > 0) ? min(n_keep, prefix - 1) : 0;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;

  // ---- radix select: threshold key of the k-th largest score in [1, prefix)
  uint32_t pref = 0, mask = 0;
  uint32_t rem = (uint32_t)k;
  if (k > 0) {
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < kSelWarps * 256; i += kSelThreads) (&hist[0][0])[i] = 0u;
      __syncthreads();
      for (int t0 = 1; t0 < prefix; t0 += kSelThreads) {
        const int t = t0 + threadIdx.x;
        bool act = false;
        uint32_t dig = 0;
        if (t < prefix) {
          const uint32_t key = order_key(x[t]);
          if ((key & mask) == pref) { act = true; dig = (key >> shift) & 0xFFu; }
        }
        const uint32_t am = __ballot_sync(0xffffffffu, act);
        if (act) {
          const uint32_t peers = __match_any_sync(am, dig);
          if ((__ffs(peers) - 1) == lane) hist[wid][dig] += __popc(peers);
        }
      }
      __syncthreads();
      if (threadIdx.x < 256) {
        uint32_t s = 0;
        for (int w = 0; w < kSelWarps; ++w) s += hist[w][threadIdx.x];
        tot[threadIdx.x] = s;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        uint32_t above = 0;
        int d = 255;
        for (; d > 0; --d) {
          if (above + tot[d] >= rem) break;
          above += tot[d];
        }
        s_pref = pref | ((uint32_t)d << shift);
        s_rem = rem - above;
      }
      __syncthreads();
      pref = s_pref;
      rem = s_rem;
      mask |= 0xFFu << shift;
      __syncthreads();
    }
  }
  const uint32_t thr = pref;   // exact key of the k-th largest
  const int need_eq = (int)rem; // how many threshold-equal scores to keep (lowest index first)

  // ---- compaction over contiguous per-thread runs
  const int per = (seq + kSelThreads - 1) / kSelThreads;
  const int t_begin = min(seq, threadIdx.x * per), t_end = min(seq, t_begin + per);
  int n_eq = 0;
  if (k > 0)
    for (int t = max(t_begin, 1); t < min(t_end, prefix); ++t) n_eq += (order_key(x[t]) == thr);
  int eq_total;
  const int eq_before = block_exclusive_scan(n_eq, scan_sh, &eq_total);
  // pass A: count kept tokens of this run
  auto keep_at = [&](int t, int& eq_rank) -> bool {
    bool keep = (t == 0) || (sw > 0 && t >= seq - sw);
    if (!keep && k > 0 && t >= 1 && t < prefix) {
      const uint32_t key = order_key(x[t]);
      if (key > thr) keep = true;
      else if (key == thr) { keep = eq_rank < need_eq; ++eq_rank; }
    } else if (k > 0 && t >= 1 && t < prefix && order_key(x[t]) == thr) {
      ++eq_rank;
    }
    if (!keep && n_prot > 0) keep = is_protected(prot, n_prot, t);
    return keep;
  };
  int cnt = 0;
  {
    int er = eq_before;
    for (int t = t_begin; t < t_end; ++t) cnt += keep_at(t, er) ? 1 : 0;
  }
  int total;
  const int out_before = block_exclusive_scan(cnt, scan_sh, &total);
  {
    int er = eq_before;
    int o = out_before;
    int32_t* dst = kept_idx + (int64_t)b * seq;
    for (int t = t_begin; t < t_end; ++t)
      if (keep_at(t, er)) dst[o++] = t;
  }
  if (threadIdx.x == 0) kept_count[b] = total;
  (void)eq_total;
}

size_t select_workspace_bytes(int, int) { return 0; }

cudaError_t launch_select(const float* imp, int batch, int seq, int sw, int n_keep, const int32_t* prot, int n_prot,
                          int32_t* kept_idx, int32_t* kept_count, void*, cudaStream_t s) {
  if (batch == 0) return cudaSuccess;
  select_kernel<<<batch, kSelThreads, 0, s>>>(imp, seq, sw, n_keep, prot, n_prot, kept_idx, kept_count);
  return cudaGetLastError();
}

}  // namespace nq
