// Keep-set selection (nexusquant/pipeline.py:895-959, _build_keep_mask):
// BOS + last `sliding_window` tokens + top-n_keep of importance[1:prefix]
// + protected positions, emitted as ascending token indices.
//
// One CTA of 1024 threads per batch row; every pass reads the row with
// coalesced 16-byte loads (4 scores per thread per step).
//  1. MSB-first radix select of the k-th largest order-preserving key over
//     3 digits (11, 11, 10 bits); per-warp aggregated shared-memory histograms.
//     After the first digit only the keys that still match the prefix count.
//  2. Ordered compaction in chunks of 4096 tokens: a block scan of threshold ties
//     (only in chunks that hold one) ranks them, lowest index first, and a block
//     scan of kept counts gives each thread its output offset.
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

constexpr int kSelThreads = 1024;
constexpr int kSelWarps = kSelThreads / 32;
constexpr int kSelChunk = kSelThreads * 4;

// Order-preserving unsigned key; -0.0 and +0.0 compare equal (one tie class), as in a float compare.
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = f == 0.0f ? 0u : __float_as_uint(f);
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

// Inclusive block scan of one int per thread (1024 threads); returns the inclusive value,
// *total gets the block sum.
__device__ __forceinline__ int block_scan_incl(int v, int* sh, int* total) {
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
    int s = sh[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    sh[lane] = s;
  }
  __syncthreads();
  const int r = x + (wid > 0 ? sh[wid - 1] : 0);
  *total = sh[kSelWarps - 1];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float4 load4(const float* x, int t0, int n) {
  if (t0 + 3 < n && ((reinterpret_cast<uintptr_t>(x + t0) & 15) == 0)) return *reinterpret_cast<const float4*>(x + t0);
  float4 r;
  r.x = t0 < n ? x[t0] : 0.0f;
  r.y = t0 + 1 < n ? x[t0 + 1] : 0.0f;
  r.z = t0 + 2 < n ? x[t0 + 2] : 0.0f;
  r.w = t0 + 3 < n ? x[t0 + 3] : 0.0f;
  return r;
}

__global__ void __launch_bounds__(kSelThreads) select_kernel(const float* imp, int seq, int sw, int n_keep,
                                                             const int32_t* prot, int n_prot, int32_t* kept_idx,
                                                             int32_t* kept_count) {
  __shared__ uint32_t hist[2048];
  __shared__ uint32_t s_pref, s_rem;
  __shared__ int scan_sh[32];
  const int b = blockIdx.x;
  const float* x = imp + (int64_t)b * seq;
  const int prefix = max(seq - sw, 0);
  const int k = (prefix > 1 && n_keep > 0) ? min(n_keep, prefix - 1) : 0;
  const int lane = threadIdx.x & 31;

  // ---- radix select over digits [31:21], [20:10], [9:0]
  uint32_t pref = 0, mask = 0, rem = (uint32_t)k;
  if (k > 0) {
    const int shifts[3] = {21, 10, 0};
    const int bits[3] = {11, 11, 10};
    for (int p = 0; p < 3; ++p) {
      const int sh = shifts[p], nb = 1 << bits[p];
      for (int i = threadIdx.x; i < nb; i += kSelThreads) hist[i] = 0u;
      __syncthreads();
      for (int c0 = 0; c0 < prefix; c0 += kSelChunk) {
        const int t0 = c0 + threadIdx.x * 4;
        const float4 v4 = load4(x, t0, prefix);
        const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int t = t0 + u;
          const uint32_t key = order_key(vv[u]);
          const bool act = t >= 1 && t < prefix && (key & mask) == pref;
          const uint32_t dig = (key >> sh) & (uint32_t)(nb - 1);
          const uint32_t am = __ballot_sync(0xffffffffu, act);
          if (act) {
            const uint32_t peers = __match_any_sync(am, dig);
            if ((__ffs(peers) - 1) == lane) atomicAdd(&hist[dig], (uint32_t)__popc(peers));
          }
        }
      }
      __syncthreads();
      if (threadIdx.x < 32) {
        // warp 0: find the digit holding the rem-th largest key (scan bins from the top)
        const int per = nb / 32;
        uint32_t cnt = 0;
        const int hi0 = nb - 1 - lane * per;  // this lane's bins: hi0 down to hi0 - per + 1
        for (int i = 0; i < per; ++i) cnt += hist[hi0 - i];
        // exclusive prefix of counts over lanes (lane 0 = highest bins)
        uint32_t inc = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
          if (lane >= o) inc += y;
        }
        const uint32_t exc = inc - cnt;
        if (exc < rem && rem <= inc) {
          uint32_t above = exc;
          int d = hi0;
          for (int i = 0; i < per; ++i, --d) {
            const uint32_t hcount = hist[d];
            if (above + hcount >= rem) break;
            above += hcount;
          }
          s_pref = pref | ((uint32_t)d << sh);
          s_rem = rem - above;
        }
      }
      __syncthreads();
      pref = s_pref;
      rem = s_rem;
      mask |= (uint32_t)(nb - 1) << sh;
      __syncthreads();
    }
  }
  const uint32_t thr = pref;    // exact key of the k-th largest prefix score
  const int need_eq = (int)rem; // threshold-equal scores to keep, lowest index first

  // ---- ordered compaction, 4096 tokens per chunk
  int out_base = 0, eq_base = 0;
  int32_t* dst = kept_idx + (int64_t)b * seq;
  for (int c0 = 0; c0 < seq; c0 += kSelChunk) {
    const int t0 = c0 + threadIdx.x * 4;
    const float4 v4 = load4(x, t0, seq);
    const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
    // keep[u]: BOS, window, above threshold or protected; tie[u]: equal to the threshold key
    bool keep[4], tie[4];
    int n_tie_l = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = t0 + u;
      bool kp = false, eq = false;
      if (t < seq) {
        if (t == 0 || (sw > 0 && t >= seq - sw)) {
          kp = true;
        } else if (k > 0 && t < prefix) {
          const uint32_t key = order_key(vv[u]);
          kp = key > thr;
          eq = key == thr;
        }
        if (!kp && n_prot > 0) kp = is_protected(prot, n_prot, t);
      }
      keep[u] = kp;
      tie[u] = eq;
      n_tie_l += eq;
    }
    // Tie ranks: only the first need_eq threshold ties of the row (lowest index) are top-k members.
    // A __syncthreads_or keeps the common no-tie chunks to a single barrier.
    if (__syncthreads_or(n_tie_l)) {
      int chunk_ties;
      int r = eq_base + block_scan_incl(n_tie_l, scan_sh, &chunk_ties) - n_tie_l;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (tie[u]) keep[u] = keep[u] || r < need_eq;
        r += tie[u];
      }
      eq_base += chunk_ties;
    }
    const int n_out_l = (int)keep[0] + (int)keep[1] + (int)keep[2] + (int)keep[3];
    int chunk_out;
    int o = out_base + block_scan_incl(n_out_l, scan_sh, &chunk_out) - n_out_l;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (keep[u]) dst[o++] = t0 + u;
    out_base += chunk_out;
  }
  if (threadIdx.x == 0) kept_count[b] = out_base;
}

size_t select_workspace_bytes(int, int) { return 0; }

cudaError_t launch_select(const float* imp, int batch, int seq, int sw, int n_keep, const int32_t* prot, int n_prot,
                          int32_t* kept_idx, int32_t* kept_count, void*, cudaStream_t s) {
  if (batch == 0) return cudaSuccess;
  select_kernel<<<batch, kSelThreads, 0, s>>>(imp, seq, sw, n_keep, prot, n_prot, kept_idx, kept_count);
  return cudaGetLastError();
}

}  // namespace nq
