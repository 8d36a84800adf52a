// Keep-set selection (nexusquant/pipeline.py:895-959, _build_keep_mask):
// BOS + last `sliding_window` tokens + top-n_keep of importance[1:prefix]
// + protected positions, emitted as ascending token indices.
//
// One thread-block cluster of 16 CTAs (1024 threads each; 8 for short rows or where
// clusters of 16 are not available) per batch row;
// CTA c owns the c-th slice of the row.  Every pass reads the row with
// coalesced 16-byte loads (after the first pass they hit L2).
//  1. MSB-first radix select of the k-th largest order-preserving key over 3
//     digits (11, 11, 10 bits).  Each CTA builds a warp-aggregated histogram
//     of its slice and adds it into CTA 0's histogram through distributed
//     shared memory; CTA 0 picks the digit.  After the first digit only keys
//     that still match the prefix count.
//  2. Ordered compaction: the CTAs exchange their slice's kept and tie counts
//     (ties are kept lowest index first), then each compacts its slice in
//     chunks of 4096 tokens with block scans, writing at its own offset.
#include <cooperative_groups.h>

#include <mutex>

#include "nq_common.cuh"
#include "nq_internal.h"

namespace cg = cooperative_groups;

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

// Inclusive block scan of one int per thread (1024 threads); *total gets the block sum.
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

// Ordered compaction of the slice [lo, hi) in chunks of 4096 tokens: kept = BOS, window,
// above threshold, protected, or a threshold tie whose row rank (lowest index first, from
// eq_base) is below need_eq.  WRITE: store indices from out_base; returns the slice count.
template <bool WRITE>
__device__ __forceinline__ int compact_slice(const float* x, int seq, int sw, int prefix, int k, uint32_t thr,
                                             int need_eq, const int32_t* prot, int n_prot, int lo, int hi,
                                             int eq_base, int out_base, int32_t* dst, int* scan_sh) {
  int count = 0;
  for (int c0 = lo; c0 < hi; c0 += kSelChunk) {
    const int t0 = c0 + threadIdx.x * 4;
    const float4 v4 = load4(x, t0, hi);
    const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
    bool keep[4], tie[4];
    int n_tie = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = t0 + u;
      bool kp = false, eq = false;
      if (t < hi) {
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
      n_tie += eq;
    }
    if (__syncthreads_or(n_tie)) {
      int chunk_ties;
      int r = eq_base + block_scan_incl(n_tie, scan_sh, &chunk_ties) - n_tie;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (tie[u]) keep[u] = keep[u] || r < need_eq;
        r += tie[u];
      }
      eq_base += chunk_ties;
    }
    const int n_out = (int)keep[0] + (int)keep[1] + (int)keep[2] + (int)keep[3];
    int chunk_out;
    const int before = block_scan_incl(n_out, scan_sh, &chunk_out) - n_out;
    if (WRITE) {
      int o = out_base + count + before;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (keep[u]) dst[o++] = t0 + u;
    }
    count += chunk_out;
  }
  return count;
}

// CS CTAs per row form one thread-block cluster (set at launch).
template <int CS>
__global__ void __launch_bounds__(kSelThreads)
    select_kernel(const float* imp, int seq, int sw, int n_keep, const int32_t* prot, int n_prot, int32_t* kept_idx,
                  int32_t* kept_count) {
  __shared__ uint32_t hist[2048];   // this CTA's histogram
  __shared__ uint32_t ghist[2048];  // CTA 0: the cluster's histogram
  __shared__ uint32_t s_pref, s_rem;
  __shared__ int scan_sh[32];
  __shared__ int cnt_keep[CS], cnt_tie[CS];  // CTA 0: per-slice counts
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int b = blockIdx.x / CS;
  const float* x = imp + (int64_t)b * seq;
  const int prefix = max(seq - sw, 0);
  const int k = (prefix > 1 && n_keep > 0) ? min(n_keep, prefix - 1) : 0;
  const int lane = threadIdx.x & 31;
  // this CTA's slice [lo, hi), a multiple of 4 tokens wide
  const int per = ((seq + CS - 1) / CS + 3) & ~3;
  const int lo = min(seq, rank * per), hi = min(seq, lo + per);
  uint32_t* g0 = cluster.map_shared_rank(ghist, 0);
  uint32_t* pref0 = cluster.map_shared_rank(&s_pref, 0);
  uint32_t* rem0 = cluster.map_shared_rank(&s_rem, 0);

  // ---- radix select over digits [31:21], [20:10], [9:0]
  uint32_t pref = 0, mask = 0, rem = (uint32_t)k;
  if (k > 0) {
    const int shifts[3] = {21, 10, 0};
    const int bits[3] = {11, 11, 10};
    const int pend = min(hi, prefix);
    for (int p = 0; p < 3; ++p) {
      const int sh = shifts[p], nb = 1 << bits[p];
      for (int i = threadIdx.x; i < nb; i += kSelThreads) {
        hist[i] = 0u;
        if (rank == 0) ghist[i] = 0u;
      }
      cluster.sync();  // CTA 0's cluster histogram is zero before anyone adds to it
      for (int c0 = lo; c0 < pend; c0 += kSelChunk) {
        const int t0 = c0 + threadIdx.x * 4;
        const float4 v4 = load4(x, t0, pend);
        const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int t = t0 + u;
          const uint32_t key = order_key(vv[u]);
          const bool act = t >= 1 && t < pend && (key & mask) == pref;
          const uint32_t dig = (key >> sh) & (uint32_t)(nb - 1);
          const uint32_t am = __ballot_sync(0xffffffffu, act);
          if (act) {
            const uint32_t peers = __match_any_sync(am, dig);
            if ((__ffs(peers) - 1) == lane) atomicAdd(&hist[dig], (uint32_t)__popc(peers));
          }
        }
      }
      __syncthreads();
      for (int i = threadIdx.x; i < nb; i += kSelThreads)
        if (hist[i]) atomicAdd(g0 + i, hist[i]);
      cluster.sync();  // the cluster histogram is complete
      if (rank == 0 && threadIdx.x < 32) {
        // warp 0 of CTA 0: the digit holding the rem-th largest key (bins scanned from the top)
        const int pl = nb / 32;
        uint32_t cnt = 0;
        const int hi0 = nb - 1 - lane * pl;  // this lane's bins: hi0 down to hi0 - pl + 1
        for (int i = 0; i < pl; ++i) cnt += ghist[hi0 - i];
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
          for (int i = 0; i < pl; ++i, --d) {
            const uint32_t hcount = ghist[d];
            if (above + hcount >= rem) break;
            above += hcount;
          }
          s_pref = pref | ((uint32_t)d << sh);
          s_rem = rem - above;
        }
      }
      cluster.sync();  // the digit is published
      pref = *pref0;
      rem = *rem0;
      mask |= (uint32_t)(nb - 1) << sh;
    }
  }
  const uint32_t thr = pref;     // exact key of the k-th largest prefix score
  const int need_eq = (int)rem;  // threshold-equal scores to keep, lowest index first

  // ---- slice counts without protection: N1 (BOS, window, above threshold) and T (threshold ties)
  int n1_l = 0, nt_l = 0;
  for (int c0 = lo; c0 < hi; c0 += kSelChunk) {
    const int t0 = c0 + threadIdx.x * 4;
    const float4 v4 = load4(x, t0, hi);
    const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = t0 + u;
      if (t >= hi) continue;
      if (t == 0 || (sw > 0 && t >= seq - sw)) {
        ++n1_l;
      } else if (k > 0 && t < prefix) {
        const uint32_t key = order_key(vv[u]);
        n1_l += key > thr;
        nt_l += key == thr;
      }
    }
  }
  int n1, nt;
  block_scan_incl(n1_l, scan_sh, &n1);
  block_scan_incl(nt_l, scan_sh, &nt);
  if (threadIdx.x == 0) {
    cluster.map_shared_rank(cnt_keep, 0)[rank] = n1;
    cluster.map_shared_rank(cnt_tie, 0)[rank] = nt;
  }
  cluster.sync();
  int eq_base = 0;  // global tie rank of this slice's first tie
  int out_r = 0;    // this slice's output count when nothing is protected
  {
    const int* ck = cluster.map_shared_rank(cnt_keep, 0);
    const int* ct = cluster.map_shared_rank(cnt_tie, 0);
    for (int r = 0; r < rank; ++r) eq_base += ct[r];
    out_r = ck[rank] + max(0, min(need_eq - eq_base, ct[rank]));
  }
  if (n_prot > 0) out_r = compact_slice<false>(x, seq, sw, prefix, k, thr, need_eq, prot, n_prot, lo, hi, eq_base, 0,
                                                nullptr, scan_sh);
  cluster.sync();  // everyone has read the first counts
  if (threadIdx.x == 0) cluster.map_shared_rank(cnt_keep, 0)[rank] = out_r;
  cluster.sync();
  int out_base = 0;
  {
    const int* ck = cluster.map_shared_rank(cnt_keep, 0);
    int total = 0;
    for (int r = 0; r < CS; ++r) {
      if (r == rank) out_base = total;
      total += ck[r];
    }
    if (rank == 0 && threadIdx.x == 0) kept_count[b] = total;
  }
  compact_slice<true>(x, seq, sw, prefix, k, thr, need_eq, prot, n_prot, lo, hi, eq_base, out_base,
                      kept_idx + (int64_t)b * seq, scan_sh);
  cluster.sync();  // CTA 0's shared memory outlives every remote reader
}

size_t select_workspace_bytes(int, int) { return 0; }

template <int CS>
static cudaError_t launch_cs(const float* imp, int batch, int seq, int sw, int n_keep, const int32_t* prot,
                             int n_prot, int32_t* kept_idx, int32_t* kept_count, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(batch * CS);
  cfg.blockDim = dim3(kSelThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, select_kernel<CS>, imp, seq, sw, n_keep, prot, n_prot, kept_idx, kept_count);
}

// 16 CTAs per row where the device schedules clusters of 16 (a non-portable size), else 8.
// The attribute that allows the size is set per device, so the answer is cached per device
// ordinal, each entry set once under a mutex (several host threads may select at once).
static bool cluster16_ok() {
  constexpr int kMaxDev = 64;
  static std::mutex mu;
  static signed char ok[kMaxDev] = {};  // 0 unknown, 1 yes, -1 no
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    cudaGetLastError();
    return false;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (ok[dev] == 0) {
    ok[dev] = -1;
    if (cudaFuncSetAttribute(select_kernel<16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(16);
      cfg.blockDim = dim3(kSelThreads);
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 16;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, select_kernel<16>, &cfg) == cudaSuccess && clusters > 0)
        ok[dev] = 1;
    }
    cudaGetLastError();
  }
  return ok[dev] == 1;
}

cudaError_t launch_select(const float* imp, int batch, int seq, int sw, int n_keep, const int32_t* prot, int n_prot,
                          int32_t* kept_idx, int32_t* kept_count, void*, cudaStream_t s) {
  if (batch == 0) return cudaSuccess;
  if (seq >= 16 * kSelChunk && cluster16_ok())
    return launch_cs<16>(imp, batch, seq, sw, n_keep, prot, n_prot, kept_idx, kept_count, s);
  return launch_cs<8>(imp, batch, seq, sw, n_keep, prot, n_prot, kept_idx, kept_count, s);
}

}  // namespace nq
