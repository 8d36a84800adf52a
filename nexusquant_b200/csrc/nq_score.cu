// Token-importance kernels: softmax column sums of (queries x keys).
//
// Key-key proxy (nexusquant/pipeline.py:756-782): queries are the last
// `obs_window` keys of the same head, no mask.  Real-attention restatement
// (pipeline.py:784-836): explicit queries at positions q_pos0.., causal mask.
//
// Three deterministic passes per (batch, query head):
//   1. per key tile: logits for every query, tile max and tile sum of exp
//   2. per query: combine tiles -> row max M and row sum Z
//   3. per key tile: colsum[t] = sum_q exp(l[q,t] - M[q]) / Z[q] (query order fixed)
// then a head reduction in head order.  Nothing uses atomics, so every rank of
// a multi-GPU job reproduces the same importance bit for bit.
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

constexpr int kScoreThreads = 128;  // one key per thread
constexpr int kQChunk = 32;         // queries per register chunk

struct ScoreWs {
  float* pm;   // [B, Hr, tiles, nq] tile max
  float* pl;   // [B, Hr, tiles, nq] tile sum
  float* M;    // [B, Hr, nq]
  float* Z;    // [B, Hr, nq]
};

static inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t score_workspace_bytes(int batch, int n_heads, int n_q, int seq) {
  const size_t tiles = (seq + kScoreThreads - 1) / kScoreThreads;
  const size_t part = (size_t)batch * n_heads * tiles * n_q * sizeof(float);
  const size_t stat = (size_t)batch * n_heads * n_q * sizeof(float);
  return 2 * align256(part) + 2 * align256(stat) + 256;
}

static ScoreWs carve(void* ws, int batch, int n_heads, int n_q, int seq) {
  const size_t tiles = (seq + kScoreThreads - 1) / kScoreThreads;
  const size_t part = align256((size_t)batch * n_heads * tiles * n_q * sizeof(float));
  const size_t stat = align256((size_t)batch * n_heads * n_q * sizeof(float));
  uint8_t* p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  ScoreWs w;
  w.pm = reinterpret_cast<float*>(p);
  w.pl = reinterpret_cast<float*>(p + part);
  w.M = reinterpret_cast<float*>(p + 2 * part);
  w.Z = reinterpret_cast<float*>(p + 2 * part + stat);
  return w;
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }

// Logits of this thread's key against queries [q0, q0 + kQChunk).
template <typename T, int D>
__device__ __forceinline__ void chunk_logits(const float (&kr)[D], const float* qs, int nqc, float scale,
                                             float (&lg)[kQChunk]) {
#pragma unroll
  for (int q = 0; q < kQChunk; ++q) lg[q] = 0.0f;
#pragma unroll
  for (int i = 0; i < D; i += 4) {
#pragma unroll
    for (int q = 0; q < kQChunk; ++q) {
      if (q < nqc) {
        const float4 qv = *reinterpret_cast<const float4*>(qs + q * D + i);
        float a = lg[q];
        a = __fmaf_rn(kr[i], qv.x, a);
        a = __fmaf_rn(kr[i + 1], qv.y, a);
        a = __fmaf_rn(kr[i + 2], qv.z, a);
        a = __fmaf_rn(kr[i + 3], qv.w, a);
        lg[q] = a;
      }
    }
  }
#pragma unroll
  for (int q = 0; q < kQChunk; ++q) lg[q] = __fmul_rn(lg[q], scale);
}

template <typename T, int D>
__device__ __forceinline__ void load_queries(const ScoreArgs& a, int b, int qh, int q0, int nqc, float* qs) {
  const int grp = a.q_heads / a.heads;
  for (int e = threadIdx.x; e < nqc * D; e += blockDim.x) {
    const int q = e / D, i = e % D;
    const int qi = q0 + q;
    float v;
    if (a.q) {
      const T* p = static_cast<const T*>(a.q) + (int64_t)b * a.q_stride_b + (int64_t)qh * a.q_stride_h +
                   (int64_t)qi * a.q_stride_t;
      v = to_f<T>(p[i]);
    } else {
      const int kh = qh / grp;
      const int t = a.seq - a.n_q + qi;
      const T* p = static_cast<const T*>(a.k) + (int64_t)b * a.k_stride_b + (int64_t)kh * a.k_stride_h +
                   (int64_t)t * a.k_stride_t;
      v = to_f<T>(p[i]);
    }
    qs[q * D + i] = v;
  }
}

template <typename T, int D>
__device__ __forceinline__ void load_key(const ScoreArgs& a, int b, int kh, int t, float (&kr)[D]) {
  const T* p = static_cast<const T*>(a.k) + (int64_t)b * a.k_stride_b + (int64_t)kh * a.k_stride_h +
               (int64_t)t * a.k_stride_t;
#pragma unroll
  for (int i = 0; i < D; ++i) kr[i] = to_f<T>(p[i]);
}

// Pass 1: tile max and tile sum-exp for every query.
template <typename T, int D>
__global__ void __launch_bounds__(kScoreThreads) score_pass1(const ScoreArgs a, ScoreWs w) {
  __shared__ __align__(16) float qs[kQChunk * D];
  __shared__ float lt[kScoreThreads][kQChunk + 1];
  __shared__ float red[4][kQChunk];
  const int tile = blockIdx.x, hr = blockIdx.y, b = blockIdx.z;
  const int qh = a.head_begin + hr;
  const int Hr = a.head_end - a.head_begin;
  const int kh = qh / (a.q_heads / a.heads);
  const int tiles = gridDim.x;
  const int t = tile * kScoreThreads + threadIdx.x;
  float kr[D];
  if (t < a.seq) load_key<T, D>(a, b, kh, t, kr);
  for (int q0 = 0; q0 < a.n_q; q0 += kQChunk) {
    const int nqc = min(kQChunk, a.n_q - q0);
    __syncthreads();
    load_queries<T, D>(a, b, qh, q0, nqc, qs);
    __syncthreads();
    float lg[kQChunk];
    if (t < a.seq) {
      chunk_logits<T, D>(kr, qs, nqc, a.scale, lg);
#pragma unroll
      for (int q = 0; q < kQChunk; ++q) {
        const bool vis = q < nqc && (!a.causal || t <= a.q_pos0 + q0 + q);
        lt[threadIdx.x][q] = vis ? lg[q] : -INFINITY;
      }
    } else {
#pragma unroll
      for (int q = 0; q < kQChunk; ++q) lt[threadIdx.x][q] = -INFINITY;
    }
    __syncthreads();
    const int q = threadIdx.x & 31, part = threadIdx.x >> 5;
    float m = -INFINITY;
    for (int r = part * 32; r < part * 32 + 32; ++r) m = fmaxf(m, lt[r][q]);
    red[part][q] = m;
    __syncthreads();
    const float mt = fmaxf(fmaxf(red[0][q], red[1][q]), fmaxf(red[2][q], red[3][q]));
    float s = 0.0f;
    for (int r = part * 32; r < part * 32 + 32; ++r) {
      const float v = lt[r][q];
      if (v != -INFINITY) s = __fadd_rn(s, expf(__fsub_rn(v, mt)));
    }
    __syncthreads();
    red[part][q] = s;
    __syncthreads();
    if (threadIdx.x < 32 && q < nqc) {
      const float st = __fadd_rn(__fadd_rn(red[0][q], red[1][q]), __fadd_rn(red[2][q], red[3][q]));
      const int64_t o = (((int64_t)b * Hr + hr) * tiles + tile) * a.n_q + q0 + q;
      w.pm[o] = mt;
      w.pl[o] = st;
    }
  }
}

// Pass 2: combine tiles per query.
__global__ void score_pass2(const ScoreArgs a, ScoreWs w, int tiles) {
  const int hr = blockIdx.x, b = blockIdx.y;
  const int Hr = a.head_end - a.head_begin;
  for (int q = threadIdx.x; q < a.n_q; q += blockDim.x) {
    const int64_t base = ((int64_t)b * Hr + hr) * tiles * a.n_q + q;
    float M = -INFINITY;
    for (int t = 0; t < tiles; ++t) M = fmaxf(M, w.pm[base + (int64_t)t * a.n_q]);
    float Z = 0.0f;
    for (int t = 0; t < tiles; ++t) {
      const float mt = w.pm[base + (int64_t)t * a.n_q];
      if (mt != -INFINITY) Z = __fadd_rn(Z, __fmul_rn(w.pl[base + (int64_t)t * a.n_q], expf(__fsub_rn(mt, M))));
    }
    const int64_t o = ((int64_t)b * Hr + hr) * a.n_q + q;
    w.M[o] = M;
    w.Z[o] = Z;
  }
}

// Pass 3: column sums of the normalised probabilities.
template <typename T, int D>
__global__ void __launch_bounds__(kScoreThreads) score_pass3(const ScoreArgs a, ScoreWs w, float* colsum) {
  __shared__ __align__(16) float qs[kQChunk * D];
  __shared__ float sM[kQChunk], sZ[kQChunk];
  const int tile = blockIdx.x, hr = blockIdx.y, b = blockIdx.z;
  const int qh = a.head_begin + hr;
  const int Hr = a.head_end - a.head_begin;
  const int kh = qh / (a.q_heads / a.heads);
  const int t = tile * kScoreThreads + threadIdx.x;
  float kr[D];
  if (t < a.seq) load_key<T, D>(a, b, kh, t, kr);
  float acc = 0.0f;
  for (int q0 = 0; q0 < a.n_q; q0 += kQChunk) {
    const int nqc = min(kQChunk, a.n_q - q0);
    __syncthreads();
    load_queries<T, D>(a, b, qh, q0, nqc, qs);
    if (threadIdx.x < nqc) {
      const int64_t o = ((int64_t)b * Hr + hr) * a.n_q + q0 + threadIdx.x;
      sM[threadIdx.x] = w.M[o];
      sZ[threadIdx.x] = w.Z[o];
    }
    __syncthreads();
    if (t < a.seq) {
      float lg[kQChunk];
      chunk_logits<T, D>(kr, qs, nqc, a.scale, lg);
#pragma unroll
      for (int q = 0; q < kQChunk; ++q) {
        if (q < nqc && (!a.causal || t <= a.q_pos0 + q0 + q))
          acc = __fadd_rn(acc, __fdiv_rn(expf(__fsub_rn(lg[q], sM[q])), sZ[q]));
      }
    }
  }
  if (t < a.seq) colsum[((int64_t)b * Hr + hr) * a.seq + t] = acc;
}

__global__ void reduce_heads_kernel(const float* colsum, int batch, int n_heads, int seq, float divisor,
                                    int accumulate, float* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)batch * seq) return;
  const int b = (int)(i / seq), t = (int)(i % seq);
  float s = 0.0f;
  for (int h = 0; h < n_heads; ++h) s = __fadd_rn(s, colsum[((int64_t)b * n_heads + h) * seq + t]);
  const float v = __fdiv_rn(s, divisor);
  out[i] = accumulate ? __fadd_rn(out[i], v) : v;
}

template <typename T, int D>
static cudaError_t run_score(const ScoreArgs& a, float* colsum, void* ws, cudaStream_t s) {
  const int Hr = a.head_end - a.head_begin;
  const int tiles = (a.seq + kScoreThreads - 1) / kScoreThreads;
  ScoreWs w = carve(ws, a.batch, Hr, a.n_q, a.seq);
  dim3 g(tiles, Hr, a.batch);
  score_pass1<T, D><<<g, kScoreThreads, 0, s>>>(a, w);
  score_pass2<<<dim3(Hr, a.batch), 64, 0, s>>>(a, w, tiles);
  score_pass3<T, D><<<g, kScoreThreads, 0, s>>>(a, w, colsum);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t score_dim(const ScoreArgs& a, float* colsum, void* ws, cudaStream_t s) {
  switch (a.head_dim) {
    case 64: return run_score<T, 64>(a, colsum, ws, s);
    case 96: return run_score<T, 96>(a, colsum, ws, s);
    case 128: return run_score<T, 128>(a, colsum, ws, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_score_colsums(const ScoreArgs& a, float* colsum, void* ws, size_t, cudaStream_t s) {
  if (score_umma_supported(a)) {
    // cudaErrorNotSupported: the tensor maps could not be encoded; nothing was launched
    const cudaError_t e = launch_score_umma(a, colsum, ws, s);
    if (e != cudaErrorNotSupported) return e;
  }
  switch (a.in_dtype) {
    case 0: return score_dim<__half>(a, colsum, ws, s);
    case 1: return score_dim<__nv_bfloat16>(a, colsum, ws, s);
    case 2: return score_dim<float>(a, colsum, ws, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_reduce_heads(const float* colsum, int batch, int n_heads, int seq, float divisor, int accumulate,
                                float* out, cudaStream_t s) {
  const int64_t n = (int64_t)batch * seq;
  if (n == 0) return cudaSuccess;
  reduce_heads_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(colsum, batch, n_heads, seq, divisor, accumulate,
                                                                   out);
  return cudaGetLastError();
}

}  // namespace nq
