// Merge eviction (MergingPress-style value merging), NexusQuantEvict._apply_merge_eviction
// (nexusquant/pipeline.py:961-1048), for one batch element at a time:
//
//  1. centroid[t, :] = mean over layers of (mean over heads of V_l[h, t, :]), fp32, layers of
//     the full sequence only (pipeline.py:996-1011); rows normalised as F.normalize does
//     (pipeline.py:1019-1020).
//  2. For every evicted token e, the kept token whose unit centroid has the largest dot product
//     with e's, first kept index on ties (torch.argmax, pipeline.py:1023-1024).  Fused tile
//     GEMM + running argmax: the n_evict x n_kept similarity matrix is never written.
//  3. For every kept token s, V_l[h, s, :] += w * V_l[h, e, :] over its evicted tokens e in
//     ascending order, w = fp32(imp[e] / (imp[s] + imp[e] + 1e-8)) computed in double as the
//     reference's Python floats are, the product and the sum each rounded to fp32, the result
//     rounded once to the cache dtype (pipeline.py:1026-1048).  Survivors are never evicted,
//     so the update is in place and race-free.
#include "../../include/nexusquant_b200.h"
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {
namespace {

constexpr int kMergeLayers = 96;  // layer pointers per launch (kernel parameter space)

struct MergeLayers {
  const void* v[kMergeLayers];
};

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }

template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }

// ---- 1a. acc[t, i] (+)= mean_h V_l[h, t, i] for the layers of this launch, in layer order.
// One thread per 8 consecutive coordinates of one token.
template <typename T>
__global__ void centroid_accumulate_kernel(MergeLayers L, int n_layers, int heads, int seq, int head_dim,
                                           int64_t sh, int64_t st, int accumulate, float* __restrict__ acc) {
  const int chunks = head_dim / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)seq * chunks) return;
  const int t = (int)(i / chunks), c = (int)(i % chunks);
  float a[8];
  float* dst = acc + (int64_t)t * head_dim + 8 * c;
  if (accumulate) {
    const float4 x = reinterpret_cast<const float4*>(dst)[0], y = reinterpret_cast<const float4*>(dst)[1];
    a[0] = x.x; a[1] = x.y; a[2] = x.z; a[3] = x.w; a[4] = y.x; a[5] = y.y; a[6] = y.z; a[7] = y.w;
  }
  const float hf = (float)heads;
  for (int l = 0; l < n_layers; ++l) {
    const T* base = static_cast<const T*>(L.v[l]) + (int64_t)t * st + 8 * c;
    float s[8];
    load8(base, s);
    for (int h = 1; h < heads; ++h) {
      float x[8];
      load8(base + (int64_t)h * sh, x);
#pragma unroll
      for (int k = 0; k < 8; ++k) s[k] = __fadd_rn(s[k], x[k]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float m = __fdiv_rn(s[k], hf);
      a[k] = (accumulate || l > 0) ? __fadd_rn(a[k], m) : m;
    }
  }
  reinterpret_cast<float4*>(dst)[0] = make_float4(a[0], a[1], a[2], a[3]);
  reinterpret_cast<float4*>(dst)[1] = make_float4(a[4], a[5], a[6], a[7]);
}

// ---- 1b. unit[t, :] = c / max(||c||, 1e-12) with c = acc[t, :] / n_layers.  One warp per token.
__global__ void centroid_normalize_kernel(const float* __restrict__ acc, int seq, int head_dim, int n_layers,
                                          float* __restrict__ unit) {
  const int warp = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (warp >= seq) return;
  const float* r = acc + (int64_t)warp * head_dim;
  const float n = (float)n_layers;
  float ss = 0.0f;
  for (int i = lane; i < head_dim; i += 32) {
    const float c = __fdiv_rn(r[i], n);
    ss = __fmaf_rn(c, c, ss);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float den = fmaxf(__fsqrt_rn(ss), 1e-12f);
  float* u = unit + (int64_t)warp * head_dim;
  for (int i = lane; i < head_dim; i += 32) u[i] = __fdiv_rn(__fdiv_rn(r[i], n), den);
}

// ---- 2. nearest kept token of every evicted token.
// A CTA owns 128 evicted rows (whole unit rows, transposed in shared memory) and walks the kept
// rows in tiles of 128, 32 coordinates at a time.  Thread (ty, tx) of 16 x 16 holds an 8 x 8
// block of dot products -- rows {4ty..4ty+3, 64+4ty..64+4ty+3}, columns likewise from tx, so
// every shared-memory read is a conflict-free float4 -- and a running (max, first index) per row.
constexpr int kNT = 128, kNK = 32, kNP = kNT + 4;  // tile rows, coordinates per step, padded stride

__global__ void __launch_bounds__(256, 2) nearest_kernel(const float* __restrict__ unit, int head_dim,
                                                      const int32_t* __restrict__ evict_pos, int n_evict,
                                                      const int32_t* __restrict__ kept_pos, int n_kept,
                                                      int32_t* __restrict__ nearest) {
  extern __shared__ __align__(16) float sm[];
  float* Es = sm;                       // [head_dim][kNP]
  float* Ks = sm + head_dim * kNP;      // [kNK][kNP]
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int e0 = blockIdx.x * kNT;
  const int q4 = head_dim / 4;
  for (int idx = tid; idx < kNT * q4; idx += 256) {
    const int row = idx % kNT, q = idx / kNT;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e0 + row < n_evict) x = reinterpret_cast<const float4*>(unit + (int64_t)evict_pos[e0 + row] * head_dim)[q];
    Es[(4 * q + 0) * kNP + row] = x.x;
    Es[(4 * q + 1) * kNP + row] = x.y;
    Es[(4 * q + 2) * kNP + row] = x.z;
    Es[(4 * q + 3) * kNP + row] = x.w;
  }
  float best[8];
  int bidx[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) { best[i] = -INFINITY; bidx[i] = 0x7fffffff; }

  for (int k0 = 0; k0 < n_kept; k0 += kNT) {
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    for (int d0 = 0; d0 < head_dim; d0 += kNK) {
      __syncthreads();  // previous step's readers are done with Ks (and Es is written, first time)
      for (int idx = tid; idx < kNT * (kNK / 4); idx += 256) {
        const int row = idx % kNT, q = idx / kNT;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k0 + row < n_kept)
          x = reinterpret_cast<const float4*>(unit + (int64_t)kept_pos[k0 + row] * head_dim + d0)[q];
        Ks[(4 * q + 0) * kNP + row] = x.x;
        Ks[(4 * q + 1) * kNP + row] = x.y;
        Ks[(4 * q + 2) * kNP + row] = x.z;
        Ks[(4 * q + 3) * kNP + row] = x.w;
      }
      __syncthreads();
#pragma unroll 4
      for (int kk = 0; kk < kNK; ++kk) {
        const float* er = Es + (d0 + kk) * kNP;
        const float* kr = Ks + kk * kNP;
        const float4 a0 = *reinterpret_cast<const float4*>(er + 4 * ty);
        const float4 a1 = *reinterpret_cast<const float4*>(er + 64 + 4 * ty);
        const float4 b0 = *reinterpret_cast<const float4*>(kr + 4 * tx);
        const float4 b1 = *reinterpret_cast<const float4*>(kr + 64 + 4 * tx);
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
      }
    }
    // columns in ascending order (first index wins on ties)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = k0 + (j < 4 ? 4 * tx + j : 64 + 4 * tx + (j - 4));
      if (col < n_kept) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (acc[i][j] > best[i] || (acc[i][j] == best[i] && col < bidx[i])) { best[i] = acc[i][j]; bidx[i] = col; }
      }
    }
  }
  // reduce over the 16 tx lanes that share ty (lanes 0-15 and 16-31 of the warp)
#pragma unroll
  for (int i = 0; i < 8; ++i) {
#pragma unroll
    for (int o = 8; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best[i], o);
      const int oi = __shfl_xor_sync(0xffffffffu, bidx[i], o);
      if (ov > best[i] || (ov == best[i] && oi < bidx[i])) { best[i] = ov; bidx[i] = oi; }
    }
    const int e = e0 + (i < 4 ? 4 * ty + i : 64 + 4 * ty + (i - 4));
    // rows whose similarities are all NaN keep index 0, as torch.argmax would
    if (tx == 0 && e < n_evict) nearest[e] = bidx[i] == 0x7fffffff ? 0 : bidx[i];
  }
}

// ---- 3. survivors absorb their evicted tokens' values.  One warp per (kept token, layer, head)
// row, 4 coordinates per lane; block y walks (layer, head) pairs 8 at a time.
template <typename T>
__global__ void __launch_bounds__(256) merge_apply_kernel(MergeLayers L, int n_layers, int heads, int head_dim,
                                                          int64_t sh, int64_t st, const float* __restrict__ imp,
                                                          const int32_t* __restrict__ kept_pos,
                                                          const int32_t* __restrict__ seg_start,
                                                          const int32_t* __restrict__ seg_evicted) {
  const int j = blockIdx.x;
  const int s0 = seg_start[j], s1 = seg_start[j + 1];
  if (s0 == s1) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int lh = blockIdx.y * 8 + warp;
  if (lh >= n_layers * heads) return;
  const int l = lh / heads, h = lh % heads;
  T* base = const_cast<T*>(static_cast<const T*>(L.v[l])) + (int64_t)h * sh;
  const int s = kept_pos[j];
  const double imp_s = (double)imp[s];
  for (int c0 = 4 * lane; c0 < head_dim; c0 += 128) {
    T* ps = base + (int64_t)s * st + c0;
    float a[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) a[k] = to_f<T>(ps[k]);
    for (int q = s0; q < s1; ++q) {
      const int e = seg_evicted[q];
      const double imp_e = (double)imp[e];
      const float w = (float)(imp_e / (imp_s + imp_e + 1e-8));
      const T* pe = base + (int64_t)e * st + c0;
#pragma unroll
      for (int k = 0; k < 4; ++k) a[k] = __fadd_rn(a[k], __fmul_rn(w, to_f<T>(pe[k])));
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) ps[k] = from_f<T>(a[k]);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int ebytes(int dtype) { return dtype == NQ_F32 ? 4 : 2; }

size_t nearest_smem_bytes(int head_dim) { return (size_t)(head_dim + kNK) * kNP * sizeof(float); }

nq_status_t cuda_st(cudaError_t e) { return e == cudaSuccess ? NQ_OK : NQ_ERR_CUDA; }

nq_status_t check_values(const void* const* values, int32_t n_layers, int32_t dtype, int32_t heads, int32_t seq,
                         int32_t head_dim, int64_t sh, int64_t st, bool need16) {
  if (!values || n_layers < 0 || heads <= 0 || seq < 0 || dtype < 0 || dtype > 2) return NQ_ERR_INVALID_ARG;
  if (head_dim <= 0 || head_dim % 8 || head_dim > 1024) return NQ_ERR_UNSUPPORTED;
  if (sh < 0 || st < head_dim) return NQ_ERR_INVALID_ARG;
  const int eb = ebytes(dtype);
  for (int l = 0; l < n_layers; ++l) {
    if (!values[l]) return NQ_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(values[l]) % (need16 ? 16 : eb)) return NQ_ERR_ALIGNMENT;
  }
  if (need16 && ((sh * eb) % 16 || (st * eb) % 16)) return NQ_ERR_ALIGNMENT;
  return NQ_OK;
}

}  // namespace
}  // namespace nq

using namespace nq;

extern "C" {

nq_status_t nq_merge_centroid_accumulate(const void* const* values, int32_t n_layers, int32_t dtype, int32_t heads,
                                         int32_t seq, int32_t head_dim, int64_t stride_h, int64_t stride_t,
                                         int32_t accumulate, float* centroid_sum, nq_stream_t stream) {
  nq_status_t st = check_values(values, n_layers, dtype, heads, seq, head_dim, stride_h, stride_t, true);
  if (st != NQ_OK) return st;
  if (!centroid_sum) return NQ_ERR_INVALID_ARG;
  if (!al16(centroid_sum)) return NQ_ERR_ALIGNMENT;
  if (seq == 0 || n_layers == 0) return NQ_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t threads = (int64_t)seq * (head_dim / 8);
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  for (int l0 = 0; l0 < n_layers; l0 += kMergeLayers) {
    const int n = n_layers - l0 < kMergeLayers ? n_layers - l0 : kMergeLayers;
    MergeLayers L{};
    for (int i = 0; i < n; ++i) L.v[i] = values[l0 + i];
    const int acc = (accumulate || l0 > 0) ? 1 : 0;
    switch (dtype) {
      case NQ_F16:
        centroid_accumulate_kernel<__half><<<blocks, 256, 0, s>>>(L, n, heads, seq, head_dim, stride_h, stride_t, acc,
                                                                   centroid_sum);
        break;
      case NQ_BF16:
        centroid_accumulate_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(L, n, heads, seq, head_dim, stride_h,
                                                                          stride_t, acc, centroid_sum);
        break;
      default:
        centroid_accumulate_kernel<float><<<blocks, 256, 0, s>>>(L, n, heads, seq, head_dim, stride_h, stride_t, acc,
                                                                  centroid_sum);
    }
    st = cuda_st(cudaGetLastError());
    if (st != NQ_OK) return st;
  }
  return NQ_OK;
}

nq_status_t nq_merge_centroid_normalize(const float* centroid_sum, int32_t seq, int32_t head_dim,
                                        int32_t n_layers, float* unit_rows, nq_stream_t stream) {
  if (!centroid_sum || !unit_rows || seq < 0 || n_layers <= 0) return NQ_ERR_INVALID_ARG;
  if (head_dim <= 0 || head_dim % 8 || head_dim > 1024) return NQ_ERR_UNSUPPORTED;
  if (seq == 0) return NQ_OK;
  const unsigned blocks = (unsigned)(((int64_t)seq * 32 + 255) / 256);
  centroid_normalize_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(centroid_sum, seq, head_dim,
                                                                                   n_layers, unit_rows);
  return cuda_st(cudaGetLastError());
}

nq_status_t nq_merge_nearest(const float* unit_rows, int32_t head_dim, const int32_t* evict_pos, int32_t n_evict,
                             const int32_t* kept_pos, int32_t n_kept, int32_t* nearest, nq_stream_t stream) {
  if (!unit_rows || n_evict < 0 || n_kept < 0) return NQ_ERR_INVALID_ARG;
  if (head_dim <= 0 || head_dim % kNK || head_dim > 256) return NQ_ERR_UNSUPPORTED;
  if (n_evict == 0) return NQ_OK;
  if (!evict_pos || !nearest || !kept_pos || n_kept == 0) return NQ_ERR_INVALID_ARG;
  if (!al16(unit_rows)) return NQ_ERR_ALIGNMENT;
  const size_t smem = nearest_smem_bytes(head_dim);
  if (smem > 48 * 1024) {  // 84.5 KB at head_dim 128, 152 KB at 256
    const cudaError_t e = cudaFuncSetAttribute(nearest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return NQ_ERR_CUDA;
  }
  const unsigned blocks = (unsigned)((n_evict + kNT - 1) / kNT);
  nearest_kernel<<<blocks, 256, smem, static_cast<cudaStream_t>(stream)>>>(unit_rows, head_dim, evict_pos, n_evict,
                                                                           kept_pos, n_kept, nearest);
  return cuda_st(cudaGetLastError());
}

nq_status_t nq_merge_apply(const void* const* values, int32_t n_layers, int32_t dtype, int32_t heads, int32_t seq,
                           int32_t head_dim, int64_t stride_h, int64_t stride_t, const float* importance,
                           const int32_t* kept_pos, int32_t n_kept, const int32_t* seg_start,
                           const int32_t* seg_evicted, nq_stream_t stream) {
  nq_status_t st = check_values(values, n_layers, dtype, heads, seq, head_dim, stride_h, stride_t, false);
  if (st != NQ_OK) return st;
  if (n_kept < 0) return NQ_ERR_INVALID_ARG;
  if (n_layers == 0 || n_kept == 0) return NQ_OK;
  if (!importance || !kept_pos || !seg_start || !seg_evicted) return NQ_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int l0 = 0; l0 < n_layers; l0 += kMergeLayers) {
    const int n = n_layers - l0 < kMergeLayers ? n_layers - l0 : kMergeLayers;
    MergeLayers L{};
    for (int i = 0; i < n; ++i) L.v[i] = values[l0 + i];
    const dim3 grid((unsigned)n_kept, (unsigned)((n * heads + 7) / 8));
    switch (dtype) {
      case NQ_F16:
        merge_apply_kernel<__half><<<grid, 256, 0, s>>>(L, n, heads, head_dim, stride_h, stride_t, importance,
                                                         kept_pos, seg_start, seg_evicted);
        break;
      case NQ_BF16:
        merge_apply_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(L, n, heads, head_dim, stride_h, stride_t, importance,
                                                                kept_pos, seg_start, seg_evicted);
        break;
      default:
        merge_apply_kernel<float><<<grid, 256, 0, s>>>(L, n, heads, head_dim, stride_h, stride_t, importance, kept_pos,
                                                        seg_start, seg_evicted);
    }
    st = cuda_st(cudaGetLastError());
    if (st != NQ_OK) return st;
  }
  return NQ_OK;
}

}  // extern "C"
