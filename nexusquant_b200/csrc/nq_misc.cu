// Protected-layer row gather and temporal delta coding of lattice codes.
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

// out[b, h, j, :] = fp16(in[b, h, kept_idx[b, j], :]); one thread per 8 elements, grid rows
// walking the (b, h) pairs so the index arithmetic is 32-bit.
// Replaces the protected-layer branch of NexusQuantEvict(Truncate).compress
// (nexusquant/pipeline.py:1206-1210, :1363-1368).
template <typename T>
__global__ void gather_rows_kernel(const T* in, int batch, int heads, int head_dim, int64_t isb, int64_t ish, int64_t ist,
                                   const int32_t* kept_idx, const int32_t* kept_count, int n_kept, __half* out,
                                   int64_t osb, int64_t osh, int64_t ost) {
  const int chunks = head_dim / 8;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int j = i / chunks, c = i - j * chunks;
  for (int bh = blockIdx.y; bh < batch * heads; bh += gridDim.y) {
  const int b = bh / heads, h = bh - b * heads;
  const int cnt = kept_count ? min(kept_count[b], n_kept) : n_kept;
  if (j >= cnt) continue;
  const int src = kept_idx ? kept_idx[(int64_t)b * n_kept + j] : j;
  const T* p = in + b * isb + h * ish + (int64_t)src * ist + 8 * c;
  float v[8];
  load8(p, v);
  __half2 h0 = __floats2half2_rn(v[0], v[1]), h1 = __floats2half2_rn(v[2], v[3]);
  __half2 h2 = __floats2half2_rn(v[4], v[5]), h3 = __floats2half2_rn(v[6], v[7]);
  uint4 u;
  u.x = *reinterpret_cast<uint32_t*>(&h0);
  u.y = *reinterpret_cast<uint32_t*>(&h1);
  u.z = *reinterpret_cast<uint32_t*>(&h2);
  u.w = *reinterpret_cast<uint32_t*>(&h3);
  *reinterpret_cast<uint4*>(out + b * osb + h * osh + (int64_t)j * ost + 8 * c) = u;
  }
}

cudaError_t launch_gather_rows(const void* in, int dtype, int batch, int heads, int head_dim, int64_t isb,
                               int64_t ish, int64_t ist, const int32_t* kept_idx, const int32_t* kept_count,
                               int n_kept, uint16_t* out, int64_t osb, int64_t osh, int64_t ost, cudaStream_t s) {
  const int64_t per_head = (int64_t)n_kept * (head_dim / 8);
  if (per_head == 0 || batch == 0 || heads == 0) return cudaSuccess;
  if (per_head > 0x7fffffffLL - 256 || (int64_t)batch * heads > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  const int64_t bh = (int64_t)batch * heads;
  const dim3 grid((unsigned)((per_head + 255) / 256), (unsigned)(bh < 65535 ? bh : 65535));
  __half* o = reinterpret_cast<__half*>(out);
  switch (dtype) {
    case 0:
      gather_rows_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(in), batch, heads, head_dim, isb, ish, ist,
                                                      kept_idx, kept_count, n_kept, o, osb, osh, ost);
      break;
    case 1:
      gather_rows_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(in), batch, heads, head_dim,
                                                             isb, ish, ist, kept_idx, kept_count, n_kept, o, osb,
                                                             osh, ost);
      break;
    case 2:
      gather_rows_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(in), batch, heads, head_dim, isb, ish, ist,
                                                     kept_idx, kept_count, n_kept, o, osb, osh, ost);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// Unpack the 8 codes of group g of a packed row.
__device__ __forceinline__ void unpack_group(const uint8_t* row, int g, int levels, int (&c)[8]) {
  if (levels <= 4) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + 4 * g);
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = (int)((w >> (4 * i)) & 0xFu) - 8;
  } else if (levels == 8) {
    uint64_t w = 0;
#pragma unroll
    for (int k = 0; k < 5; ++k) w |= (uint64_t)row[5 * g + k] << (8 * k);
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = (int)((w >> (5 * i)) & 31u) - 8;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = (int8_t)row[8 * g + i];
  }
}

// delta[s, t, :] = code[s, t, :] - code[s, t-1, :] (int8), delta[s, 0, :] = code[s, 0, :]
// (nexusquant/core/temporal_codec.py:48-52).  One thread per 8-group.
__global__ void delta_kernel(const uint8_t* codes, int n_streams, int n_tokens, int dp, int levels, int8_t* delta) {
  const int G = dp / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)n_streams * n_tokens * G;
  if (i >= total) return;
  const int g = (int)(i % G);
  const int64_t row = i / G;  // stream * n_tokens + t
  const int t = (int)(row % n_tokens);
  const int pb = levels <= 4 ? dp / 2 : (levels == 8 ? dp * 5 / 8 : dp);
  int c[8], p[8];
  unpack_group(codes + row * pb, g, levels, c);
  if (t > 0) unpack_group(codes + (row - 1) * pb, g, levels, p);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    lo |= ((uint32_t)(t > 0 ? c[k] - p[k] : c[k]) & 0xFFu) << (8 * k);
    hi |= ((uint32_t)(t > 0 ? c[4 + k] - p[4 + k] : c[4 + k]) & 0xFFu) << (8 * k);
  }
  *reinterpret_cast<uint2*>(delta + row * dp + 8 * g) = make_uint2(lo, hi);
}

cudaError_t launch_delta(const uint8_t* codes, int n_streams, int n_tokens, int dp, int levels, int8_t* delta,
                         cudaStream_t s) {
  const int64_t total = (int64_t)n_streams * n_tokens * (dp / 8);
  if (total == 0) return cudaSuccess;
  delta_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(codes, n_streams, n_tokens, dp, levels, delta);
  return cudaGetLastError();
}

// rANS symbol pass (nexusquant/core/entropy_coder.py:35-75 applied to the lattice codes).
// mode 0: counts[c + L] += #rows with code c (c in [-L, L]; 2L + 1 bins, shared-memory
//         histogram per CTA, one global atomic per bin and CTA).
// mode 1: symbols[i] = half ? c + L : c / 2 + L / 2 (uint8, row-major [rows, d_p]), the
//         reference's shift for half-integer (doubled) or integer coordinates.
// Symbols are clipped to the alphabet as the reference clips them.
__device__ __forceinline__ uint32_t rans_symbol(int c, int levels, int half) {
  return half ? (uint32_t)min(max(c + levels, 0), 2 * levels)
              : (uint32_t)min(max((c >> 1) + levels / 2, 0), levels);
}

__global__ void code_symbols_kernel(const uint8_t* codes, int64_t rows, int dp, int levels, int mode, int half,
                                    unsigned int* counts, uint8_t* symbols) {
  __shared__ unsigned int h[33];
  if (mode == 0)
    for (int i = threadIdx.x; i < 33; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int G = dp / 8;
  const int pb = levels <= 4 ? dp / 2 : (levels == 8 ? dp * 5 / 8 : dp);
  const int64_t total = rows * G;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / G;
    const int g = (int)(i - row * G);
    int c[8];
    unpack_group(codes + row * pb, g, levels, c);
    if (mode == 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) atomicAdd(&h[min(max(c[k] + levels, 0), 2 * levels)], 1u);
    } else {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        lo |= rans_symbol(c[k], levels, half) << (8 * k);
        hi |= rans_symbol(c[4 + k], levels, half) << (8 * k);
      }
      *reinterpret_cast<uint2*>(symbols + row * dp + 8 * g) = make_uint2(lo, hi);
    }
  }
  if (mode == 0) {
    __syncthreads();
    for (int i = threadIdx.x; i < 2 * levels + 1; i += blockDim.x)
      if (h[i]) atomicAdd(&counts[i], h[i]);
  }
}

cudaError_t launch_code_symbols(const uint8_t* codes, int64_t rows, int dp, int levels, int mode, int half,
                                unsigned int* counts, uint8_t* symbols, cudaStream_t s) {
  const int64_t total = rows * (dp / 8);
  if (total == 0) return cudaSuccess;
  int dev = 0, sms = 0;
  cudaError_t e;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  long long grid = (total + 255) / 256;
  if (grid > 8LL * sms) grid = 8LL * sms;
  code_symbols_kernel<<<(unsigned)grid, 256, 0, s>>>(codes, rows, dp, levels, mode, half, counts, symbols);
  return cudaGetLastError();
}

}  // namespace nq
