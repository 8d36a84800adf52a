// Byte layouts of the paged (vLLM-style) interface, nexusquant/integrations/vllm_backend.py:
//  * CompressedPage.key_codes / value_codes hold one int8 per coordinate, code = 2 x lattice
//    point (vllm_backend.py:73-101, :267-316).  nq_unpack_codes turns the library's packed rows
//    (nibbles for L <= 4, 5-bit fields for L = 8, int8 for L = 16) into that layout.
//  * pack_codes_nibble / unpack_codes_nibble (vllm_backend.py:476-540): byte k of a row holds
//    clamp(c[2k] + 8, 0, 15) in its low nibble and clamp(c[2k+1] + 8, 0, 15) in its high nibble,
//    an odd last coordinate is paired with a zero nibble; unpacking subtracts 8.
// All three are one pass of byte work, one thread per output word or byte.
#include "../../include/nexusquant_b200.h"
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {
namespace {

// One thread per 8-group of one row: 8 int8 codes out (one 8-byte store).
template <int FMT>
__global__ void unpack_codes_kernel(const uint8_t* __restrict__ packed, int64_t rows, int dp, int pb,
                                    int8_t* __restrict__ codes) {
  const int G = dp / 8;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * G) return;
  const int64_t r = i / G;
  const int g = (int)(i % G);
  const uint8_t* row = packed + r * pb;
  int c[8];
  if constexpr (FMT == 0) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row + 4 * g);
#pragma unroll
    for (int k = 0; k < 8; ++k) c[k] = (int)((w >> (4 * k)) & 0xFu) - 8;
  } else if constexpr (FMT == 1) {
    uint64_t w = 0;
#pragma unroll
    for (int k = 0; k < 5; ++k) w |= (uint64_t)row[5 * g + k] << (8 * k);
#pragma unroll
    for (int k = 0; k < 8; ++k) c[k] = (int)((w >> (5 * k)) & 31u) - 8;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) c[k] = (int8_t)row[8 * g + k];
  }
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    lo |= ((uint32_t)c[k] & 0xFFu) << (8 * k);
    hi |= ((uint32_t)c[4 + k] & 0xFFu) << (8 * k);
  }
  *reinterpret_cast<uint2*>(codes + r * dp + 8 * g) = make_uint2(lo, hi);
}

__device__ __forceinline__ uint32_t nib(int c) {
  c += 8;
  return (uint32_t)(c < 0 ? 0 : (c > 15 ? 15 : c));
}

// One thread per output byte.
__global__ void pack_nibbles_kernel(const int8_t* __restrict__ codes, int64_t rows, int d,
                                    uint8_t* __restrict__ packed) {
  const int pb = (d + 1) / 2;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * pb) return;
  const int64_t r = i / pb;
  const int k = (int)(i % pb);
  const int8_t* row = codes + r * d;
  const uint32_t lo = nib(row[2 * k]);
  const uint32_t hi = 2 * k + 1 < d ? nib(row[2 * k + 1]) : 0u;  // padding nibble is 0
  packed[i] = (uint8_t)(lo | (hi << 4));
}

// One thread per output code.
__global__ void unpack_nibbles_kernel(const uint8_t* __restrict__ packed, int64_t rows, int d,
                                      int8_t* __restrict__ codes) {
  const int pb = (d + 1) / 2;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * d) return;
  const int64_t r = i / d;
  const int j = (int)(i % d);
  const uint32_t b = packed[r * pb + j / 2];
  codes[i] = (int8_t)((int)((j & 1) ? (b >> 4) & 0xFu : b & 0xFu) - 8);
}

unsigned blocks_for(int64_t n) { return (unsigned)((n + 255) / 256); }

}  // namespace
}  // namespace nq

using namespace nq;

extern "C" {

nq_status_t nq_unpack_codes(const uint8_t* packed, int64_t rows, int32_t head_dim_padded, int32_t levels,
                            int8_t* codes, nq_stream_t stream) {
  if (!packed || !codes || rows < 0) return NQ_ERR_INVALID_ARG;
  if (levels != 2 && levels != 4 && levels != 8 && levels != 16) return NQ_ERR_INVALID_ARG;
  if (head_dim_padded <= 0 || head_dim_padded % 8) return NQ_ERR_INVALID_ARG;
  const int fmt = levels <= 4 ? 0 : (levels == 8 ? 1 : 2);  // the compress kernel's packing formats
  const int pb = fmt == 0 ? head_dim_padded / 2 : (fmt == 1 ? head_dim_padded * 5 / 8 : head_dim_padded);
  if ((reinterpret_cast<uintptr_t>(codes) & 7u) || (fmt == 0 && (reinterpret_cast<uintptr_t>(packed) & 3u)))
    return NQ_ERR_ALIGNMENT;
  if (rows == 0) return NQ_OK;
  const int64_t n = rows * (head_dim_padded / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (fmt == 0) unpack_codes_kernel<0><<<blocks_for(n), 256, 0, s>>>(packed, rows, head_dim_padded, pb, codes);
  else if (fmt == 1) unpack_codes_kernel<1><<<blocks_for(n), 256, 0, s>>>(packed, rows, head_dim_padded, pb, codes);
  else unpack_codes_kernel<2><<<blocks_for(n), 256, 0, s>>>(packed, rows, head_dim_padded, pb, codes);
  return cudaGetLastError() == cudaSuccess ? NQ_OK : NQ_ERR_CUDA;
}

nq_status_t nq_pack_nibbles(const int8_t* codes, int64_t rows, int32_t d, uint8_t* packed, nq_stream_t stream) {
  if (!codes || !packed || rows < 0 || d <= 0) return NQ_ERR_INVALID_ARG;
  if (rows == 0) return NQ_OK;
  const int64_t n = rows * ((d + 1) / 2);
  pack_nibbles_kernel<<<blocks_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(codes, rows, d, packed);
  return cudaGetLastError() == cudaSuccess ? NQ_OK : NQ_ERR_CUDA;
}

nq_status_t nq_unpack_nibbles(const uint8_t* packed, int64_t rows, int32_t d, int8_t* codes, nq_stream_t stream) {
  if (!codes || !packed || rows < 0 || d <= 0) return NQ_ERR_INVALID_ARG;
  if (rows == 0) return NQ_OK;
  const int64_t n = rows * d;
  unpack_nibbles_kernel<<<blocks_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(packed, rows, d, codes);
  return cudaGetLastError() == cudaSuccess ? NQ_OK : NQ_ERR_CUDA;
}

}  // extern "C"
