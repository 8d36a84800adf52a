// Tensor-core token-importance kernels for fp16 / bf16 caches.
//
// Same three-pass structure as nq_score.cu (tile statistics, per-query
// combine, normalised column sums), but the logits Q K^T come from mma.sync
// m16n8k16 (fp16 or bf16 inputs, fp32 accumulation) on key tiles staged in
// shared memory by the TMA engine, and the softmax runs in base 2
// (2^(l * log2 e - m)) on the ex2 unit.  All reductions have a fixed order, so
// the result is deterministic and identical on every rank.
//
// CTA: 4 warps, 128 keys per tile (32 per warp = 2 m16 tiles), all queries
// (n_q <= 64, padded to a multiple of 8) of one (batch, query head); a CTA walks
// a run of consecutive tiles of that head with a two-stage copy pipeline.
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

constexpr int kTcThreads = 128;
constexpr int kTcKeys = 128;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

struct TcWs {
  float* pm;  // [B, Hr, tiles, nq] tile max (base-2 logits)
  float* pl;  // [B, Hr, tiles, nq] tile sum of 2^(l - max)
  float* M;   // [B, Hr, nq]
  float* Z;   // [B, Hr, nq]
};

template <int D>
struct TcLayout {
  static constexpr int kStride = D * 2 + 16;            // padded rows: conflict-free ldmatrix / LDS
  static constexpr int kTile = kTcKeys * kStride;       // one key tile
  static constexpr int kQ = 64 * kStride;               // up to 64 query rows
  static constexpr int kSmem = 2 * kTile + kQ;
};

// Logits of this warp's 32 keys x NT*8 queries: acc[m][n][4] (m16n8 C layout).
template <typename T, int D, int NT>
__device__ __forceinline__ void tile_logits(const uint8_t* ktile, const uint8_t* qs, float (&acc)[2][NT][4]) {
  using Lo = TcLayout<D>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[m][n][i] = 0.0f;
  // ldmatrix lane address: matrices (rows 0-7, k0), (rows 8-15, k0), (rows 0-7, k0+8), (rows 8-15, k0+8)
  const int lr = (lane & 7) + ((lane >> 3) & 1) * 8;
  const int lk = (lane >> 4) * 8;
#pragma unroll
  for (int k0 = 0; k0 < D; k0 += 16) {
    uint32_t a[2][4];
#pragma unroll
    for (int m = 0; m < 2; ++m)
      ldsm_x4(a[m], ktile + (warp * 32 + m * 16 + lr) * Lo::kStride + (k0 + lk) * 2);
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const uint8_t* qrow = qs + (n * 8 + (lane >> 2)) * Lo::kStride + (k0 + (lane & 3) * 2) * 2;
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(qrow);
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(qrow + 16);
#pragma unroll
      for (int m = 0; m < 2; ++m) mma16816<T>(acc[m][n], a[m], b0, b1);
    }
  }
}

// Load this CTA's query rows (n_q of them; the padding rows are zero) into shared memory.
template <typename T, int D>
__device__ __forceinline__ void load_q(const ScoreArgs& a, int b, int qh, int nqp, uint8_t* qs) {
  using Lo = TcLayout<D>;
  const int grp = a.q_heads / a.heads;
  for (int e = threadIdx.x; e < nqp * (D / 8); e += kTcThreads) {
    const int q = e / (D / 8), c = e % (D / 8);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (q < a.n_q) {
      const T* p;
      if (a.q) {
        p = static_cast<const T*>(a.q) + (int64_t)b * a.q_stride_b + (int64_t)qh * a.q_stride_h +
            (int64_t)q * a.q_stride_t;
      } else {
        const int t = a.seq - a.n_q + q;
        p = static_cast<const T*>(a.k) + (int64_t)b * a.k_stride_b + (int64_t)(qh / grp) * a.k_stride_h +
            (int64_t)t * a.k_stride_t;
      }
      v = *reinterpret_cast<const uint4*>(p + 8 * c);
    }
    *reinterpret_cast<uint4*>(qs + q * Lo::kStride + c * 16) = v;
  }
}

// Copy key tile `tile` (rows tile*128 ..) of kv head kh into a stage; thread r copies row r.
template <typename T, int D>
__device__ __forceinline__ void issue_keys(const ScoreArgs& a, int b, int kh, int tile, uint8_t* stage,
                                           uint64_t* bar) {
  using Lo = TcLayout<D>;
  const int t = tile * kTcKeys + threadIdx.x;
  if (threadIdx.x == 0) {
    const int rows = min(kTcKeys, a.seq - tile * kTcKeys);
    mbar_arrive_expect_tx(bar, (uint32_t)rows * D * 2);
  }
  __syncthreads();
  if (t < a.seq) {
    const T* p = static_cast<const T*>(a.k) + (int64_t)b * a.k_stride_b + (int64_t)kh * a.k_stride_h +
                 (int64_t)t * a.k_stride_t;
    bulk_g2s(stage + threadIdx.x * Lo::kStride, p, D * 2, bar);
  }
}

// PASS 1: per tile, per query: max of base-2 logits and sum of 2^(l - max).
// PASS 3: per key: sum over queries of 2^(l - M_q) / Z_q.
template <typename T, int D, int NT, int PASS>
__global__ void __launch_bounds__(kTcThreads) score_tc(const ScoreArgs a, TcWs w, float* colsum, int tiles_per_cta) {
  using Lo = TcLayout<D>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar[2];
  __shared__ float red[4][64];
  __shared__ float sM[64], sZ[64];
  const int hr = blockIdx.y, b = blockIdx.z;
  const int qh = a.head_begin + hr;
  const int Hr = a.head_end - a.head_begin;
  const int kh = qh / (a.q_heads / a.heads);
  const int tiles = (a.seq + kTcKeys - 1) / kTcKeys;
  const int t0 = blockIdx.x * tiles_per_cta;
  const int t1 = min(tiles, t0 + tiles_per_cta);
  if (t0 >= t1) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int NQP = NT * 8;
  uint8_t* qs = smem + 2 * Lo::kTile;
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
  }
  load_q<T, D>(a, b, qh, NQP, qs);
  if (PASS == 3 && threadIdx.x < NQP) {
    const bool ok = threadIdx.x < a.n_q;
    const int64_t o = ((int64_t)b * Hr + hr) * a.n_q + threadIdx.x;
    sM[threadIdx.x] = ok ? w.M[o] : 0.0f;
    sZ[threadIdx.x] = ok ? __frcp_rn(w.Z[o]) : 0.0f;  // 1 / Z
  }
  issue_keys<T, D>(a, b, kh, t0, smem, &bar[0]);
  const float sc2 = a.scale * kLog2e;
  for (int tile = t0, it = 0; tile < t1; ++tile, ++it) {
    const int s = it & 1;
    __syncthreads();  // stage s^1 is free (its tile was consumed in the previous iteration)
    if (tile + 1 < t1) issue_keys<T, D>(a, b, kh, tile + 1, smem + (s ^ 1) * Lo::kTile, &bar[s ^ 1]);
    if (!mbar_wait(&bar[s], (it >> 1) & 1)) {
      if (tile + 1 < t1) mbar_wait(&bar[s ^ 1], ((it + 1) >> 1) & 1);
      return;
    }
    float acc[2][NT][4];
    tile_logits<T, D, NT>(smem + s * Lo::kTile, qs, acc);
    // element (m, n, i): key = tile*128 + warp*32 + m*16 + lane/4 + (i>=2)*8, query = n*8 + (lane&3)*2 + (i&1)
    const int kbase = tile * kTcKeys + warp * 32 + (lane >> 2);
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int key = kbase + m * 16 + (i >> 1) * 8;
          const int q = n * 8 + (lane & 3) * 2 + (i & 1);
          const bool vis = key < a.seq && q < a.n_q && (!a.causal || key <= a.q_pos0 + q);
          acc[m][n][i] = vis ? __fmul_rn(acc[m][n][i], sc2) : -INFINITY;
        }
    if (PASS == 1) {
      // per-query max over this tile: in-thread (4 keys), lanes with equal lane&3, then warps
      float mx[NT][2];
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          float v = fmaxf(fmaxf(acc[0][n][j], acc[0][n][j + 2]), fmaxf(acc[1][n][j], acc[1][n][j + 2]));
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
          mx[n][j] = v;
        }
      if (lane < 4)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int j = 0; j < 2; ++j) red[warp][n * 8 + lane * 2 + j] = mx[n][j];
      __syncthreads();
      float sm[NT][2];
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int q = n * 8 + (lane & 3) * 2 + j;
          const float mt = fmaxf(fmaxf(red[0][q], red[1][q]), fmaxf(red[2][q], red[3][q]));
          mx[n][j] = mt;
          float v = 0.0f;
          if (mt != -INFINITY) {
#pragma unroll
            for (int m = 0; m < 2; ++m) {
              v = __fadd_rn(v, ex2(__fsub_rn(acc[m][n][j], mt)));
              v = __fadd_rn(v, ex2(__fsub_rn(acc[m][n][j + 2], mt)));
            }
          }
          v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
          v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 8));
          v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 16));
          sm[n][j] = v;
        }
      __syncthreads();
      if (lane < 4)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int j = 0; j < 2; ++j) red[warp][n * 8 + lane * 2 + j] = sm[n][j];
      __syncthreads();
      if (warp == 0 && lane < 4) {
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int q = n * 8 + lane * 2 + j;
            if (q < a.n_q) {
              const float st = __fadd_rn(__fadd_rn(red[0][q], red[1][q]), __fadd_rn(red[2][q], red[3][q]));
              const int64_t o = (((int64_t)b * Hr + hr) * tiles + tile) * a.n_q + q;
              w.pm[o] = mx[n][j];
              w.pl[o] = st;
            }
          }
      }
    } else {
      // column sums: sum over queries of 2^(l - M_q) / Z_q, for each of the thread's 4 keys
      float cs[2][2];
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          float v = 0.0f;
#pragma unroll
          for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const int q = n * 8 + (lane & 3) * 2 + j;
              v = __fadd_rn(v, __fmul_rn(ex2(__fsub_rn(acc[m][n][r * 2 + j], sM[q])), sZ[q]));
            }
          v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
          v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
          cs[m][r] = v;
        }
      if ((lane & 3) == 0) {
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const int key = kbase + m * 16 + r * 8;
            if (key < a.seq) colsum[((int64_t)b * Hr + hr) * a.seq + key] = cs[m][r];
          }
      }
    }
  }
}

// Per query: combine tile statistics -> M (base-2 max) and Z (sum of 2^(l - M)).  One warp per query.
__global__ void score_tc_combine(const ScoreArgs a, TcWs w, int tiles) {
  const int q = blockIdx.x, hr = blockIdx.y, b = blockIdx.z;
  const int Hr = a.head_end - a.head_begin;
  const int lane = threadIdx.x;
  const int64_t base = ((int64_t)b * Hr + hr) * tiles * a.n_q + q;
  float m = -INFINITY, s = 0.0f;
  for (int t = lane; t < tiles; t += 32) {
    const float mt = w.pm[base + (int64_t)t * a.n_q], st = w.pl[base + (int64_t)t * a.n_q];
    if (mt == -INFINITY) continue;
    if (mt > m) {
      s = __fadd_rn(__fmul_rn(s, ex2(__fsub_rn(m, mt))), st);
      m = mt;
    } else {
      s = __fadd_rn(s, __fmul_rn(st, ex2(__fsub_rn(mt, m))));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    float v = 0.0f;
    if (m != -INFINITY) v = __fmul_rn(s, ex2(__fsub_rn(m, mm)));
    if (m2 != -INFINITY) v = __fadd_rn(v, __fmul_rn(s2, ex2(__fsub_rn(m2, mm))));
    m = mm;
    s = v;
  }
  if (lane == 0) {
    const int64_t o = ((int64_t)b * Hr + hr) * a.n_q + q;
    w.M[o] = m;
    w.Z[o] = s;
  }
}

template <typename T, int D, int NT>
static cudaError_t run_tc(const ScoreArgs& a, float* colsum, void* ws, cudaStream_t s) {
  using Lo = TcLayout<D>;
  const int Hr = a.head_end - a.head_begin;
  const int tiles = (a.seq + kTcKeys - 1) / kTcKeys;
  // tile workspace layout identical to nq_score.cu (tiles of 128 keys)
  const size_t part = ((size_t)a.batch * Hr * tiles * a.n_q * sizeof(float) + 255) & ~size_t(255);
  const size_t stat = ((size_t)a.batch * Hr * a.n_q * sizeof(float) + 255) & ~size_t(255);
  uint8_t* p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  TcWs w{reinterpret_cast<float*>(p), reinterpret_cast<float*>(p + part), reinterpret_cast<float*>(p + 2 * part),
         reinterpret_cast<float*>(p + 2 * part + stat)};
  int dev = 0, sms = 0;
  cudaError_t e;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  // about 4 CTAs per SM in total, each walking a run of tiles of one head
  const long long heads = (long long)a.batch * Hr;
  int tpc = (int)((tiles * heads + 4LL * sms - 1) / (4LL * sms));
  tpc = max(1, min(tpc, tiles));
  const int chunks = (tiles + tpc - 1) / tpc;
  const size_t smem = Lo::kSmem;
  auto k1 = score_tc<T, D, NT, 1>;
  auto k3 = score_tc<T, D, NT, 3>;
  if ((e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(k3, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess) return e;
  dim3 g(chunks, Hr, a.batch);
  k1<<<g, kTcThreads, smem, s>>>(a, w, colsum, tpc);
  score_tc_combine<<<dim3(a.n_q, Hr, a.batch), 32, 0, s>>>(a, w, tiles);
  k3<<<g, kTcThreads, smem, s>>>(a, w, colsum, tpc);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t tc_nt(const ScoreArgs& a, float* colsum, void* ws, cudaStream_t s) {
  if (a.n_q <= 32) return run_tc<T, D, 4>(a, colsum, ws, s);
  if (a.n_q <= 64) return run_tc<T, D, 8>(a, colsum, ws, s);
  return cudaErrorInvalidValue;
}

template <typename T>
static cudaError_t tc_dim(const ScoreArgs& a, float* colsum, void* ws, cudaStream_t s) {
  switch (a.head_dim) {
    case 64: return tc_nt<T, 64>(a, colsum, ws, s);
    case 96: return tc_nt<T, 96>(a, colsum, ws, s);
    case 128: return tc_nt<T, 128>(a, colsum, ws, s);
  }
  return cudaErrorInvalidValue;
}

// fp16 / bf16 caches with n_q <= 64 and 16-byte aligned rows; returns false when not applicable.
bool score_tc_supported(const ScoreArgs& a) {
  if (a.in_dtype != 0 && a.in_dtype != 1) return false;
  if (a.n_q < 1 || a.n_q > 64) return false;
  if ((a.k_stride_t * 2) % 16 || (a.k_stride_h * 2) % 16 || (a.k_stride_b * 2) % 16) return false;
  if (a.q && ((a.q_stride_t * 2) % 16 || (a.q_stride_h * 2) % 16 || (a.q_stride_b * 2) % 16)) return false;
  if ((reinterpret_cast<uintptr_t>(a.k) & 15) || (a.q && (reinterpret_cast<uintptr_t>(a.q) & 15))) return false;
  return true;
}

cudaError_t launch_score_tc(const ScoreArgs& a, float* colsum, void* ws, cudaStream_t s) {
  return a.in_dtype == 0 ? tc_dim<__half>(a, colsum, ws, s) : tc_dim<__nv_bfloat16>(a, colsum, ws, s);
}

}  // namespace nq
