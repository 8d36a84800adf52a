// Merge eviction's nearest kept token on the tensor cores, exact (nq_merge_nearest_unit).
//
// nearest[i] = argmax_j u[evict_pos[i]] . u[kept_pos[j]], first j on ties (torch.argmax,
// nexusquant/pipeline.py:1023-1024), with the dot products defined as the exact kernel of
// nq_merge_nearest computes them: fp32 fmaf in coordinate order 0 .. 127.  Rows are unit
// vectors (norm <= 1 + 1e-6, as nq_merge_centroid_normalize writes them).
//
//  1. screening: CTA = 128 evicted rows, 256 threads.  The evicted tile (fp32,
//     K-major, 128-byte swizzle) stays in shared memory; kept tiles of 128 rows stream through
//     two cp.async stages; one thread issues tcgen05.mma kind::tf32 (M = 128 evicted rows,
//     N = 128 kept rows, K = 128, fp32 accumulation) into one of two TMEM accumulators, so
//     the MMA of tile i+1 overlaps the scan of tile i.  For unit rows the tf32 value differs
//     from the exact one by at most 2^-9 (1 + 2^-9) (operands truncated to 10 mantissa bits)
//     plus the fp32 summation error of either order (< 4e-5): kMargin = 0.005 is more than
//     twice that bound, so the exact argmax always satisfies approx >= max approx - kMargin.
//     Each thread (one row, one half of the columns) keeps, in column order, every column
//     within kMargin of its running maximum (12 slots, compacted when full).
//  2. exact re-check in the same CTA: each candidate within kMargin of the row maximum is
//     recomputed with the exact kernel's fmaf order; the best (first column on ties) wins.
//  3. rows whose slots overflowed, that saw a NaN or infinite similarity, or whose evicted row
//     is not a unit vector are marked -1 and re-scanned exactly over every kept row by
//     nearest_fix_kernel.
#include "../../include/nexusquant_b200.h"
#include "nq_common.cuh"
#include "nq_internal.h"
#include "nq_umma.cuh"

namespace nq {
namespace {

constexpr int kMD = 128;          // head_dim
constexpr int kMT = 128;          // rows per tile (evicted: MMA M; kept: MMA N)
constexpr int kMSlots = 12;       // candidate slots per (row, half)
constexpr float kMargin = 0.005f;
constexpr int kMThreads = 256;

struct MtSmem {
  static constexpr int kTile = kMT * kMD * 4;          // 64 KB: 4 column blocks x 128 rows x 128 B
  static constexpr int kE = 0;
  static constexpr int kK0 = kTile;
  static constexpr int kK1 = 2 * kTile;
  static constexpr int kCandIdx = 3 * kTile;           // [slot][thread] int
  static constexpr int kCandVal = kCandIdx + kMSlots * kMThreads * 4;
  static constexpr int kBytes = kCandVal + kMSlots * kMThreads * 4 + 1024;  // + alignment slack
};

// Byte offset of 16-byte chunk j (0..31) of row r in a swizzled fp32 tile.
__device__ __forceinline__ uint32_t mt_chunk(int r, int j) {
  return (uint32_t)((j >> 3) * (kMT * 128) + r * 128 + (((j & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(valid ? 16 : 0)
               : "memory");
}

// Row index this lane fetches for a tile: lane l (< 16) of warp w holds rows[8 l + w], the row
// that warp w copies in step l of mt_load_tile (one global load per lane, issued ahead).
__device__ __forceinline__ int mt_row_index(const int32_t* rows, int n) {
  const int lane = threadIdx.x & 31, r = 8 * lane + (threadIdx.x >> 5);
  return (lane < 16 && r < n) ? rows[r] : 0;
}

// Rows rows[0..n) of unit (or zeros past n) -> swizzled tile; every thread issues 16 copies,
// taking the row index of step k from lane k of its warp.
__device__ __forceinline__ void mt_load_tile(uint8_t* tile, const float* unit, int my_index, int n) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < kMT * 32 / kMThreads; ++k) {
    const int r = 8 * k + warp;
    const int src_row = __shfl_sync(0xffffffffu, my_index, k);
    const bool ok = r < n;
    cp_async16_zfill(tile + mt_chunk(r, lane), unit + (ok ? (int64_t)src_row * kMD + 4 * lane : 0), ok);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Exact dot product, the order of nearest_kernel: fmaf over coordinates 0 .. 127.
__device__ __forceinline__ float mt_exact(const uint8_t* etile, int r, const float* krow) {
  float acc = 0.0f;
#pragma unroll 4
  for (int j = 0; j < 32; ++j) {
    const float4 a = *reinterpret_cast<const float4*>(etile + mt_chunk(r, j));
    const float4 b = __ldg(reinterpret_cast<const float4*>(krow) + j);
    acc = __fmaf_rn(a.x, b.x, acc);
    acc = __fmaf_rn(a.y, b.y, acc);
    acc = __fmaf_rn(a.z, b.z, acc);
    acc = __fmaf_rn(a.w, b.w, acc);
  }
  return acc;
}

__global__ void __launch_bounds__(kMThreads, 1)
    nearest_tc_kernel(const float* __restrict__ unit, const int32_t* __restrict__ evict_pos, int n_evict,
                      const int32_t* __restrict__ kept_pos, int n_kept, int32_t* __restrict__ nearest) {
  extern __shared__ uint8_t mt_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(mt_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* E = sm + MtSmem::kE;
  int* cidx = reinterpret_cast<int*>(sm + MtSmem::kCandIdx);
  float* cval = reinterpret_cast<float*>(sm + MtSmem::kCandVal);
  __shared__ uint64_t mbar[2];
  __shared__ uint32_t tmem_base;
  __shared__ int err;
  __shared__ float rmax[2][kMT];
  __shared__ float bval[2][kMT];
  __shared__ int bcol[2][kMT];
  __shared__ int rbad[kMT];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int row = quarter * 32 + lane;  // TMEM lane = evicted row of the tile
  const int e0 = blockIdx.x * kMT;
  const int n_e = min(kMT, n_evict - e0);
  const int tiles = (n_kept + kMT - 1) / kMT;

  if (tid == 0) {
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    fence_mbar_init();
    err = 0;
  }
  if (tid < kMT) rbad[tid] = 0;
  if (warp == 0) tmem_alloc(&tmem_base, 256);
  mt_load_tile(E, unit, mt_row_index(evict_pos + e0, n_e), n_e);
  mt_load_tile(sm + MtSmem::kK0, unit, mt_row_index(kept_pos, n_kept), min(kMT, n_kept));
  if (tiles > 1) mt_load_tile(sm + MtSmem::kK1, unit, mt_row_index(kept_pos + kMT, n_kept - kMT), min(kMT, n_kept - kMT));
  // row indices of the next tile to copy (tile 2), fetched one tile ahead
  int next_index = tiles > 2 ? mt_row_index(kept_pos + 2 * kMT, n_kept - 2 * kMT) : 0;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;
  constexpr uint32_t kIdesc = f16_idesc(2, kMT, kMT);  // tf32 x tf32 -> fp32

  float amax = -INFINITY;
  int cnt = 0;
  bool bad = false;
  auto issue_mma = [&](int i) {
    const uint8_t* ks = sm + ((i & 1) ? MtSmem::kK1 : MtSmem::kK0);
    const uint32_t d = tbase + (uint32_t)((i & 1) * kMT);
#pragma unroll
    for (int k = 0; k < kMD / 8; ++k) {
      const int blk = k >> 2, off = (k & 3) * 32;
      umma_tf32(d, sw128_desc(E + blk * (kMT * 128) + off), sw128_desc(ks + blk * (kMT * 128) + off), kIdesc,
                k > 0 ? 1u : 0u);
    }
    umma_commit(&mbar[i & 1]);
  };
  auto scan = [&](int i) {
    if (!mbar_wait(&mbar[i & 1], (i >> 1) & 1)) err = 1;
    tc_fence_after();
    __syncwarp();
    float v[64];
    {
      float a[32], b[32];
      const uint32_t t = tbase + ((uint32_t)(quarter * 32) << 16) + (uint32_t)((i & 1) * kMT + 64 * half);
      tmem_ld32(t, a);
      tmem_ld32(t + 32, b);
#pragma unroll
      for (int j = 0; j < 32; ++j) { v[j] = a[j]; v[32 + j] = b[j]; }
    }
    const int c0 = i * kMT + 64 * half;
    const int nv = min(64, n_kept - c0);  // valid columns of this thread's half-tile
    if (nv < 64) {
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (j >= nv) v[j] = -1e30f;
    }
    // tile maximum; NaN propagates, so a NaN or infinite similarity shows in m
    float m = v[0];
#pragma unroll
    for (int j = 1; j < 63; j += 2) m = max3_nan(m, v[j], v[j + 1]);
    m = max3_nan(m, v[63], v[63]);
    if (nv <= 0) return;
    if (!(fabsf(m) <= 1e30f) || !(m > -1e29f)) {  // NaN, inf, or only -inf: the exact scan decides
      bad = true;
      return;
    }
    amax = fmaxf(amax, m);
    const float thr = amax - kMargin;
    if (m < thr) return;  // nothing of this tile is near the running maximum (the common case)
    // drop the slots that fell below the threshold, then append this tile's near-maximum columns
    int w = 0;
    for (int s2 = 0; s2 < cnt; ++s2) {
      const float cv = cval[s2 * kMThreads + tid];
      if (cv >= thr) {
        cval[w * kMThreads + tid] = cv;
        cidx[w * kMThreads + tid] = cidx[s2 * kMThreads + tid];
        ++w;
      }
    }
    cnt = w;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      if (v[j] >= thr) {  // masked columns hold -1e30 < thr
        if (cnt < kMSlots) {
          cval[cnt * kMThreads + tid] = v[j];
          cidx[cnt * kMThreads + tid] = c0 + j;
          ++cnt;
        } else {
          bad = true;  // more near-ties than slots: the exact scan decides this row
        }
      }
    }
  };

  for (int i = 0; i < tiles; ++i) {
    // tile i has landed (only tile i+1 may still be in flight)
    if (i + 1 < tiles) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else asm volatile("cp.async.wait_group 0;" ::: "memory");
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && !err) {
      tc_fence_after();
      issue_mma(i);
    }
    if (i > 0) scan(i - 1);
    // stage i & 1 is free once MMA i completed: copy tile i + 2 into it
    if (i + 2 < tiles) {
      if (!mbar_wait(&mbar[i & 1], (i >> 1) & 1)) err = 1;
      mt_load_tile(sm + ((i & 1) ? MtSmem::kK1 : MtSmem::kK0), unit, next_index, min(kMT, n_kept - (i + 2) * kMT));
      if (i + 3 < tiles) next_index = mt_row_index(kept_pos + (i + 3) * kMT, n_kept - (i + 3) * kMT);
    }
    if (err) break;
  }
  if (!err && tiles > 0) scan(tiles - 1);

  // ---- exact re-check of the candidates within kMargin of the row maximum
  rmax[half][row] = amax;
  if (bad) rbad[row] = 1;
  if (half == 0) {
    float ss = 0.0f;
#pragma unroll 4
    for (int j = 0; j < 32; ++j) {
      const float4 a = *reinterpret_cast<const float4*>(E + mt_chunk(row, j));
      ss = fmaf(a.x, a.x, fmaf(a.y, a.y, fmaf(a.z, a.z, fmaf(a.w, a.w, ss))));
    }
    if (ss > 1.0001f) rbad[row] = 1;  // not a unit row: the screening bound does not hold
  }
  __syncthreads();
  const float thr = fmaxf(rmax[0][row], rmax[1][row]) - kMargin;
  float best = -INFINITY;
  int bc = 0x7fffffff;
  if (row < n_e && !err && !rbad[row]) {
    for (int s = 0; s < cnt; ++s) {
      if (cval[s * kMThreads + tid] < thr) continue;
      const int col = cidx[s * kMThreads + tid];
      if (col < 0 || col >= n_kept) continue;  // cannot happen: only valid columns are appended
      const float x = mt_exact(E, row, unit + (int64_t)kept_pos[col] * kMD);
      if (x > best || (x == best && col < bc)) { best = x; bc = col; }
    }
  }
  bval[half][row] = best;
  bcol[half][row] = bc;
  __syncthreads();
  if (half == 0 && row < n_e) {
    float b = bval[0][row];
    int c = bcol[0][row];
    const float b1 = bval[1][row];
    const int c1 = bcol[1][row];
    if (b1 > b || (b1 == b && c1 < c)) { b = b1; c = c1; }
    nearest[e0 + row] = (err || rbad[row] || c == 0x7fffffff) ? -1 : c;
  }
  if (tid == 0 && err) {
    mbar_wait(&mbar[0], 0, 1u << 20);
    mbar_wait(&mbar[1], 0, 1u << 20);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, 256);
}

// Rows marked -1: the exact scan of nearest_kernel over every kept row, one warp per row.
__global__ void __launch_bounds__(256) nearest_fix_kernel(const float* __restrict__ unit,
                                                          const int32_t* __restrict__ evict_pos, int n_evict,
                                                          const int32_t* __restrict__ kept_pos, int n_kept,
                                                          int32_t* __restrict__ nearest) {
  const int e = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (e >= n_evict || nearest[e] != -1) return;
  const float* er = unit + (int64_t)evict_pos[e] * kMD;
  float best = -INFINITY;
  int bc = 0x7fffffff;
  for (int col = lane; col < n_kept; col += 32) {
    const float* kr = unit + (int64_t)kept_pos[col] * kMD;
    float acc = 0.0f;
    for (int j = 0; j < kMD / 4; ++j) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(er) + j);
      const float4 b = __ldg(reinterpret_cast<const float4*>(kr) + j);
      acc = __fmaf_rn(a.x, b.x, acc);
      acc = __fmaf_rn(a.y, b.y, acc);
      acc = __fmaf_rn(a.z, b.z, acc);
      acc = __fmaf_rn(a.w, b.w, acc);
    }
    if (acc > best || (acc == best && col < bc)) { best = acc; bc = col; }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oc = __shfl_xor_sync(0xffffffffu, bc, o);
    if (ov > best || (ov == best && oc < bc)) { best = ov; bc = oc; }
  }
  // rows whose similarities are all NaN keep index 0, as torch.argmax would
  if (lane == 0) nearest[e] = bc == 0x7fffffff ? 0 : bc;
}

}  // namespace
}  // namespace nq

extern "C" nq_status_t nq_merge_nearest_unit(const float* unit_rows, int32_t head_dim, const int32_t* evict_pos,
                                             int32_t n_evict, const int32_t* kept_pos, int32_t n_kept,
                                             int32_t* nearest, nq_stream_t stream) {
  if (!unit_rows || n_evict < 0 || n_kept < 0) return NQ_ERR_INVALID_ARG;
  if (head_dim != nq::kMD) return NQ_ERR_UNSUPPORTED;
  if (n_evict == 0) return NQ_OK;
  if (!evict_pos || !nearest || !kept_pos || n_kept == 0) return NQ_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(unit_rows) & 15u) return NQ_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaFuncSetAttribute(nq::nearest_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, nq::MtSmem::kBytes) !=
      cudaSuccess)
    return NQ_ERR_CUDA;
  const unsigned blocks = (unsigned)((n_evict + nq::kMT - 1) / nq::kMT);
  nq::nearest_tc_kernel<<<blocks, nq::kMThreads, nq::MtSmem::kBytes, s>>>(unit_rows, evict_pos, n_evict, kept_pos,
                                                                          n_kept, nearest);
  if (cudaGetLastError() != cudaSuccess) return NQ_ERR_CUDA;
  const unsigned fb = (unsigned)(((int64_t)n_evict * 32 + 255) / 256);
  nq::nearest_fix_kernel<<<fb, 256, 0, s>>>(unit_rows, evict_pos, n_evict, kept_pos, n_kept, nearest);
  return cudaGetLastError() == cudaSuccess ? NQ_OK : NQ_ERR_CUDA;
}
