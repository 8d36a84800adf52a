// Decode attention straight from the compressed layout (no fp16 K/V materialised).
//
// Semantics of NexusQuantPagedAttention.forward (nexusquant/integrations/vllm_backend.py:
// 692-765): one query token per sequence, keys and values dequantized as decompress_page
// does (:398-429, keys re-rotated at their stored positions and optionally sharpened), then
// softmax(q K^T / sqrt(d)) V in fp32, fp16 output.  Query heads are grouped over the KV
// heads (q head g*G .. g*G+G-1 reads KV head g; G = 1 is the reference's case).
//
// Split-K over tokens, two kernels:
//  * attend_partial: CTA = (token split, KV head, batch), 128 threads.  Per tile of 128
//    tokens each thread decodes one key in registers (unpack -> exact half2 butterfly ->
//    scale -> RoPE -> sharpen -> fp16, as the dequantize kernel) and dots it with the G
//    queries (base-2 logits).  Values stay in the code domain: because the inverse
//    Hadamard is linear, sum_t p_t v_t = h/2 * H^T (sum_t p_t s_t c_t), so the CTA
//    accumulates p_t * scale_t * codes_t per dimension (thread j owns dimension j) with
//    online-softmax rescaling, and writes (max, sum, accumulator) per query head.
//  * attend_combine: per (batch, query head) merges the splits, divides by the softmax
//    sum, applies the inverse Walsh-Hadamard butterfly once and scales by h/2.
// Fixed reduction orders throughout: deterministic.
#include <algorithm>

#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

namespace {

constexpr int kAtTok = 128;  // tokens per tile = threads per CTA
constexpr int kAtD = 128;    // head_dim = d_p
constexpr float kAtLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2a(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ __half2 ah2_bits(uint32_t u) {
  __half2 h;
  *reinterpret_cast<uint32_t*>(&h) = u;
  return h;
}
__device__ __forceinline__ __half2 ah2c(float a) { return __floats2half2_rn(a, a); }

// Codes of coordinates {q, q + 64} (q < 64) as half2 integers from a packed row.
template <int FMT>
__device__ __forceinline__ void at_unpack(const uint8_t* p, __half2 (&R)[64]) {
  if constexpr (FMT == 0) {
    uint32_t w[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + k);
      w[4 * k] = u.x; w[4 * k + 1] = u.y; w[4 * k + 2] = u.z; w[4 * k + 3] = u.w;
    }
#pragma unroll
    for (int q = 0; q < 64; q += 2) {
      const int m = q >> 3, byte = (q & 7) >> 1;
      const uint32_t u = __byte_perm(w[m], w[m + 8], (uint32_t)((4 + byte) << 8 | byte));
      R[q] = __hadd2(ah2_bits((u & 0x000F000Fu) | 0x64006400u), ah2c(-1032.0f));
      R[q + 1] = __hfma2(ah2_bits((u & 0x00F000F0u) | 0x64006400u), ah2c(1.0f / 16.0f), ah2c(-72.0f));
    }
  } else if constexpr (FMT == 1) {
    uint32_t w[20];
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + k);
      w[4 * k] = u.x; w[4 * k + 1] = u.y; w[4 * k + 2] = u.z; w[4 * k + 3] = u.w;
    }
#pragma unroll
    for (int q = 0; q < 64; ++q) {
      const int bit = 5 * q, k = bit >> 5, s = bit & 31;
      uint32_t lo, hi;
      if (s + 5 <= 32) {
        lo = w[k] >> s;
        hi = w[k + 10] >> s;
      } else {
        lo = __funnelshift_r(w[k], w[k + 1], s);
        hi = __funnelshift_r(w[k + 10], w[k + 11], s);
      }
      const uint32_t u = __byte_perm(lo, hi, 0x5410u);
      R[q] = __hadd2(ah2_bits((u & 0x001F001Fu) | 0x64006400u), ah2c(-1032.0f));
    }
  } else {
    uint32_t w[32];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + k);
      w[4 * k] = u.x; w[4 * k + 1] = u.y; w[4 * k + 2] = u.z; w[4 * k + 3] = u.w;
    }
#pragma unroll
    for (int q = 0; q < 64; ++q) {
      const int m = q >> 2, byte = q & 3;
      const uint32_t u = __byte_perm(w[m], w[m + 16], (uint32_t)((4 + byte) << 8 | byte));
      R[q] = __hadd2(ah2_bits((u & 0x00FF00FFu) ^ 0x64806480u), ah2c(-1152.0f));
    }
  }
}

// Code (integer) of coordinate j of a packed row.
template <int FMT>
__device__ __forceinline__ int at_code(const uint8_t* row, int j) {
  if constexpr (FMT == 0) return (int)((row[j >> 1] >> ((j & 1) * 4)) & 0xF) - 8;
  else if constexpr (FMT == 1) {
    const int bit = 5 * j, byte = bit >> 3, s = bit & 7;
    const uint32_t v = (uint32_t)row[byte] | (s > 3 ? ((uint32_t)row[byte + 1] << 8) : 0u);  // stays in the row
    return (int)((v >> s) & 0x1F) - 8;
  } else {
    return (int)(int8_t)row[j];
  }
}

template <int FMT>
constexpr int at_pb() { return FMT == 0 ? 64 : (FMT == 1 ? 80 : 128); }

}  // namespace


// 3 CTAs per SM: the register cap (170) costs 16 bytes of spill at G = 8 and lifts occupancy
// from 8 to 12 warps; the kernel is latency-bound (scoreboard stalls), and on B200 this is
// 83 us against 93 us at 2 CTAs for a config-4 layer.  attend_splits sizes the grid to one wave.
template <int FMTK, int FMTV, int G>
__global__ void __launch_bounds__(kAtTok, 3) attend_partial(const AttendArgs a) {
  constexpr int PBV = at_pb<FMTV>();
  __shared__ float qs[G][kAtD];                     // queries * scale * log2 e
  __shared__ __align__(16) uint8_t vrow[kAtTok][PBV];  // value codes of the tile
  __shared__ float wgt[G][kAtTok];                  // p_t * value scale_t
  __shared__ float red[G][4];
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int count = a.count ? min(a.count[b], a.n_tokens) : a.n_tokens;
  const int t0 = split * a.tokens_per_split, t1 = min(count, t0 + a.tokens_per_split);
  const float qscale = a.scale * kAtLog2e;
  for (int e = tid; e < G * kAtD; e += kAtTok) {
    const int g = e / kAtD, j = e % kAtD;
    qs[g][j] = __half2float(a.q[(int64_t)b * a.q_stride_b + (int64_t)(kh * G + g) * a.q_stride_h + j]) * qscale;
  }
  float m[G], l[G], acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) { m[g] = -INFINITY; l[g] = 0.0f; acc[g] = 0.0f; }
  const int64_t row0 = ((int64_t)b * a.heads + kh) * a.n_tokens;
  const float coef_h = 0.5f * hadamard_entry(kAtD);
  __syncthreads();
  for (int base = t0; base < t1; base += kAtTok) {
    const int t = base + tid;
    const bool valid = t < t1;
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = -INFINITY;
    float sv = 0.0f;
    if (valid) {
      // key: decode as the dequantize kernel does, then dot with the queries
      __half2 R[64];
      at_unpack<FMTK>(a.k_codes + (row0 + t) * at_pb<FMTK>(), R);
#pragma unroll
      for (int st = 1; st < 64; st <<= 1)
#pragma unroll
        for (int q = 0; q < 64; ++q)
          if ((q & st) == 0) {
            const __half2 x = R[q], y = R[q + st];
            R[q] = __hadd2(x, y);
            R[q + st] = __hsub2(x, y);
          }
      const __half2 pm = __floats2half2_rn(1.0f, -1.0f);
#pragma unroll
      for (int q = 0; q < 64; ++q) R[q] = __hfma2(__high2half2(R[q]), pm, __low2half2(R[q]));
      const float coef = __fmul_rn(__half2float(__ushort_as_half(a.k_scales[row0 + t])), coef_h);
      const int pos = min(max(a.positions[(int64_t)b * a.n_tokens + t], 0), a.rope_rows - 1);
      const float* cs = a.rope_cos + (int64_t)pos * (kAtD / 2);
      const float* sn = a.rope_sin + (int64_t)pos * (kAtD / 2);
#pragma unroll
      for (int g = 0; g < G; ++g) s[g] = 0.0f;
#pragma unroll
      for (int i = 0; i < 64; i += 4) {
        const float4 c4 = __ldg(reinterpret_cast<const float4*>(cs + i));
        const float4 s4 = __ldg(reinterpret_cast<const float4*>(sn + i));
        const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float z1 = __fmul_rn(__low2float(R[i + u]), coef), z2 = __fmul_rn(__high2float(R[i + u]), coef);
          float k1 = __fsub_rn(__fmul_rn(z1, cc[u]), __fmul_rn(z2, ss[u]));
          float k2 = __fadd_rn(__fmul_rn(z1, ss[u]), __fmul_rn(z2, cc[u]));
          if (a.key_sharpen != 1.0f) {
            k1 = __fmul_rn(k1, a.key_sharpen);
            k2 = __fmul_rn(k2, a.key_sharpen);
          }
          k1 = __half2float(__float2half_rn(k1));  // the fp16 key the dequantize path stores
          k2 = __half2float(__float2half_rn(k2));
#pragma unroll
          for (int g = 0; g < G; ++g) s[g] = fmaf(qs[g][i + u], k1, fmaf(qs[g][i + u + 64], k2, s[g]));
        }
      }
      sv = __half2float(__ushort_as_half(a.v_scales[row0 + t]));
      const uint4* src = reinterpret_cast<const uint4*>(a.v_codes + (row0 + t) * PBV);
#pragma unroll
      for (int k = 0; k < PBV / 16; ++k) reinterpret_cast<uint4*>(vrow[tid])[k] = __ldg(src + k);
    }
    // tile maxima -> new running maxima (same value in every thread)
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float v = s[g];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
      if (lane == 0) red[g][warp] = v;
    }
    __syncthreads();
    float alpha[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float tm = fmaxf(fmaxf(red[g][0], red[g][1]), fmaxf(red[g][2], red[g][3]));
      const float mn = fmaxf(m[g], tm);
      alpha[g] = m[g] == -INFINITY ? 0.0f : ex2a(m[g] - mn);
      m[g] = mn;
      const float p = valid ? ex2a(s[g] - mn) : 0.0f;
      wgt[g][tid] = p * sv;
      s[g] = p;
    }
    __syncthreads();
    // tile sums of p
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float v = s[g];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[g][warp] = v;
    }
    __syncthreads();
    const int nt = min(kAtTok, t1 - base);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      l[g] = l[g] * alpha[g] + ((red[g][0] + red[g][1]) + (red[g][2] + red[g][3]));
      acc[g] *= alpha[g];
    }
    // values in the code domain: thread tid owns dimension tid
    for (int u = 0; u < nt; ++u) {
      const float c = (float)at_code<FMTV>(vrow[u], tid);
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = fmaf(wgt[g][u], c, acc[g]);
    }
    __syncthreads();
  }
  const int64_t o = ((int64_t)b * a.q_heads + kh * G) * a.splits + split;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int64_t og = o + (int64_t)g * a.splits;
    if (tid == 0) {
      a.ws_m[og] = m[g];
      a.ws_l[og] = l[g];
    }
    a.ws_acc[og * kAtD + tid] = acc[g];
  }
}

__global__ void __launch_bounds__(kAtD) attend_combine(const AttendArgs a) {
  __shared__ float y[kAtD];
  const int qh = blockIdx.x, b = blockIdx.y, j = threadIdx.x;
  const int64_t o = ((int64_t)b * a.q_heads + qh) * a.splits;
  float M = -INFINITY;
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, a.ws_m[o + s]);
  float L = 0.0f, v = 0.0f;
  if (M != -INFINITY) {
    for (int s = 0; s < a.splits; ++s) {
      const float ms = a.ws_m[o + s];
      if (ms == -INFINITY) continue;
      const float f = ex2a(ms - M);
      L = fmaf(a.ws_l[o + s], f, L);
      v = fmaf(a.ws_acc[(o + s) * kAtD + j], f, v);
    }
  }
  y[j] = L > 0.0f ? v / L : 0.0f;
  __syncthreads();
  // inverse Walsh-Hadamard (stride 1, 2, ... 64) across the 128 threads
  for (int st = 1; st < kAtD; st <<= 1) {
    const float mine = y[j], other = y[j ^ st];
    __syncthreads();
    y[j] = (j & st) ? other - mine : mine + other;
    __syncthreads();
  }
  const float r = y[j] * (0.5f * hadamard_entry(kAtD));
  a.out[(int64_t)b * a.out_stride_b + (int64_t)qh * a.out_stride_h + j] = __float2half_rn(r);
}

size_t attend_workspace_bytes(int batch, int q_heads, int splits) {
  const size_t n = (size_t)batch * q_heads * splits;
  return n * sizeof(float) * (2 + kAtD) + 3 * 256;
}

int attend_splits(int batch, int heads, int n_tokens) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = (n_tokens + kAtTok - 1) / kAtTok;
  // one wave of attend_partial at 3 resident CTAs per SM
  const long long want = (3LL * sms + (long long)batch * heads - 1) / ((long long)batch * heads);
  return (int)std::max(1LL, std::min<long long>(tiles, want));
}

template <int FMTK, int FMTV>
static cudaError_t attend_g(const AttendArgs& a, int G, cudaStream_t s) {
  const dim3 grid(a.splits, a.heads, a.batch);
  switch (G) {
    case 1: attend_partial<FMTK, FMTV, 1><<<grid, kAtTok, 0, s>>>(a); break;
    case 2: attend_partial<FMTK, FMTV, 2><<<grid, kAtTok, 0, s>>>(a); break;
    case 4: attend_partial<FMTK, FMTV, 4><<<grid, kAtTok, 0, s>>>(a); break;
    case 8: attend_partial<FMTK, FMTV, 8><<<grid, kAtTok, 0, s>>>(a); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_attend(const AttendArgs& in, int fk, int fv, void* ws, cudaStream_t s) {
  AttendArgs a = in;
  const size_t n = (size_t)a.batch * a.q_heads * a.splits;
  uint8_t* p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  a.ws_m = reinterpret_cast<float*>(p);
  a.ws_l = a.ws_m + n;
  a.ws_acc = a.ws_l + n;
  const int G = a.q_heads / a.heads;
  cudaError_t e;
#define NQ_AT(K_, V_) \
  if (fk == K_ && fv == V_) e = attend_g<K_, V_>(a, G, s); else
  NQ_AT(0, 0) NQ_AT(1, 0) NQ_AT(0, 1) NQ_AT(1, 1) NQ_AT(2, 0) NQ_AT(2, 1) NQ_AT(2, 2) NQ_AT(0, 2) NQ_AT(1, 2)
  return cudaErrorInvalidValue;
#undef NQ_AT
  if (e != cudaSuccess) return e;
  attend_combine<<<dim3(a.q_heads, a.batch), kAtD, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace nq
