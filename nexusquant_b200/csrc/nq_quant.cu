// Fused KV compress and dequantize kernels (sm_100a).
//
// Compress, per vector (one (layer, K|V, batch, head, kept token) row):
//   load row (TMA bulk copy -> shared) -> fp32 -> [keys] inverse split-half RoPE
//   at the source position -> zero pad to d_p -> Walsh-Hadamard butterfly in
//   registers -> * fl32(1/sqrt(d_p)) -> amax, sc = amax / (L/2) -> x / sc
//   (correctly rounded) -> relaxed-E8 nearest point per 8-group -> clamp ->
//   pack codes, fp16 scale [-> fake-quant reconstruction].
// Reference: nexusquant/pipeline.py:1218-1236, nexusquant/core/e8_lattice.py:27-124,
// nexusquant/core/rope_utils.py:75-122, nexusquant/integrations/vllm_backend.py:267-316.
//
// Work decomposition: one thread owns one vector (d_p <= 128 fp32 values in
// registers), so the butterfly and the lattice step need no cross-thread
// exchange.  A CTA of 128 threads owns a tile of HG heads x (128/HG) tokens of
// one (layer, K|V, batch); threads of a warp that share a token also share the
// RoPE table row, which is then a shared-memory broadcast.  All layers of a
// call go in one launch (per-layer pointers travel in the kernel parameters).
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

// --------------------------------------------------------------------------
// Relaxed-E8 nearest point of one 8-group (nexusquant/core/e8_lattice.py:27-69),
// emitted as codes = 2 * lattice point clamped to [-levels, levels].
//
// A = round-half-even(x) with, when sum(A) is odd, the coordinate of smallest
// gap (first index on ties) moved one step toward x; B = round(fl(x - 0.5)) + 0.5.
// B is chosen iff d_half < d_int, evaluated exactly as
//   sum_i g_i + odd * (1 - 2 g_min) > 2,   g_i = |x_i - round(x_i)|
// (d_half - d_int = sum_i (1/4 - g_i) - odd * (1 - 2 g_min)), in fp32 with the
// sum taken in index order -- the same arithmetic as the CPU oracle.
// --------------------------------------------------------------------------
__device__ __forceinline__ void e8_group(const float (&n)[8], int levels, int (&code)[8]) {
  float af[8], g[8];
  uint32_t sbits[8], bbits[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float s = __fadd_rn(n[i], kMagic);
    sbits[i] = __float_as_uint(s);
    af[i] = __fsub_rn(s, kMagic);
    g[i] = fabsf(__fsub_rn(n[i], af[i]));
    float t = __fsub_rn(n[i], 0.5f);
    bbits[i] = __float_as_uint(__fadd_rn(t, kMagic));
  }
  float gsum = g[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) gsum = __fadd_rn(gsum, g[i]);
  float gmin = g[0];
  int idx = 0;
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    if (g[i] < gmin) { gmin = g[i]; idx = i; }
  }
  uint32_t par = sbits[0] ^ sbits[1] ^ sbits[2] ^ sbits[3] ^ sbits[4] ^ sbits[5] ^ sbits[6] ^ sbits[7];
  const bool odd = (par & 1u) != 0u;
  float lhs = gsum;
  if (odd) lhs = __fadd_rn(lhs, __fsub_rn(1.0f, __fmul_rn(2.0f, gmin)));
  const bool use_b = lhs > 2.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int a = static_cast<int>(sbits[i] - kMagicBits);
    int bp = static_cast<int>(bbits[i] - kMagicBits);
    int c;
    if (use_b) {
      c = 2 * bp + 1;
    } else {
      c = 2 * a;
      if (odd && i == idx) c += (__fsub_rn(n[i], af[i]) >= 0.0f) ? 2 : -2;
    }
    c = min(max(c, -levels), levels);
    code[i] = c;
  }
}

// Packed bytes of one vector.
__host__ __device__ constexpr int packed_bytes_of(int dp, int levels) {
  return levels <= 4 ? dp / 2 : (levels == 8 ? dp * 5 / 8 : dp);
}

// Pack 8 codes of group g into the row words (little-endian byte order).
template <int DP>
__device__ __forceinline__ void pack_group(uint32_t* w, int g, const int (&c)[8], int levels) {
  if (levels <= 4) {
    uint32_t v = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) v |= (static_cast<uint32_t>(c[i] + 8) & 0xFu) << (4 * i);
    w[g] = v;
  } else if (levels == 8) {
    uint64_t v = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) v |= static_cast<uint64_t>(c[i] + 8) << (5 * i);
    const int bit = 40 * g;
    const int wi = bit >> 5, sh = bit & 31;
    // bits of the 40-bit field land in at most 3 words
    w[wi] |= static_cast<uint32_t>(v << sh);
    uint64_t rest = v >> (32 - sh);
    w[wi + 1] |= static_cast<uint32_t>(rest);
    if (sh > 24) w[wi + 2] |= static_cast<uint32_t>(rest >> 32);
  } else {
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lo |= (static_cast<uint32_t>(c[i]) & 0xFFu) << (8 * i);
      hi |= (static_cast<uint32_t>(c[4 + i]) & 0xFFu) << (8 * i);
    }
    w[2 * g] = lo;
    w[2 * g + 1] = hi;
  }
}

// Unnormalised in-register Walsh-Hadamard butterfly, stages of stride 1, 2, 4 ...
template <int DP>
__device__ __forceinline__ void fwht_regs(float (&x)[DP]) {
#pragma unroll
  for (int h = 1; h < DP; h <<= 1) {
#pragma unroll
    for (int i = 0; i < DP; ++i) {
      if ((i & h) == 0) {
        float a = x[i], b = x[i + h];
        x[i] = __fadd_rn(a, b);
        x[i + h] = __fsub_rn(a, b);
      }
    }
  }
}

// Store BYTES (a multiple of 8) from the row words to global; compile-time size
// keeps the words in registers.
template <int BYTES>
__device__ __forceinline__ void store_row(uint8_t* dst, const uint32_t* w) {
  if constexpr ((BYTES & 15) == 0) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int k = 0; k < BYTES / 16; ++k) d[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
  } else {
    uint2* d = reinterpret_cast<uint2*>(dst);
#pragma unroll
    for (int k = 0; k < BYTES / 8; ++k) d[k] = make_uint2(w[2 * k], w[2 * k + 1]);
  }
}

// Reconstruct (fake-quant) from integer codes held as floats in x[], write fp16.
template <int D, int DP>
__device__ __forceinline__ void reconstruct_store(float (&x)[DP], float scale, bool key, const float* cosr,
                                                  const float* sinr, float sharpen, __half* out,
                                                  bool rotate = true) {
  if (rotate) fwht_regs<DP>(x);
  const float coef = __fmul_rn(scale, rotate ? 0.5f * hadamard_entry(DP) : 0.5f);
#pragma unroll
  for (int i = 0; i < D; ++i) x[i] = __fmul_rn(x[i], coef);
  constexpr int DH = D / 2;
  if (key) {
#pragma unroll
    for (int i = 0; i < DH; ++i) {
      const float c = __ldg(cosr + i), s = __ldg(sinr + i);
      const float z1 = x[i], z2 = x[i + DH];
      x[i] = __fsub_rn(__fmul_rn(z1, c), __fmul_rn(z2, s));
      x[i + DH] = __fadd_rn(__fmul_rn(z1, s), __fmul_rn(z2, c));
    }
    if (sharpen != 1.0f) {
#pragma unroll
      for (int i = 0; i < D; ++i) x[i] = __fmul_rn(x[i], sharpen);
    }
  }
#pragma unroll
  for (int k = 0; k < D / 8; ++k) {
    __half2 h0 = __floats2half2_rn(x[8 * k], x[8 * k + 1]);
    __half2 h1 = __floats2half2_rn(x[8 * k + 2], x[8 * k + 3]);
    __half2 h2 = __floats2half2_rn(x[8 * k + 4], x[8 * k + 5]);
    __half2 h3 = __floats2half2_rn(x[8 * k + 6], x[8 * k + 7]);
    uint4 u;
    u.x = *reinterpret_cast<uint32_t*>(&h0);
    u.y = *reinterpret_cast<uint32_t*>(&h1);
    u.z = *reinterpret_cast<uint32_t*>(&h2);
    u.w = *reinterpret_cast<uint32_t*>(&h3);
    reinterpret_cast<uint4*>(out)[k] = u;
  }
}

// --------------------------------------------------------------------------
// Dequantize kernel: one thread per vector, codes read straight from global.
// --------------------------------------------------------------------------
template <int D, int DP>
__global__ void __launch_bounds__(kCompressThreads, 3) decompress_kernel(const DecompressArgs args) {
  const int HG = args.head_group;
  const int TOK = kCompressThreads / HG;
  int bid = blockIdx.x;
  const int t_tiles = (args.n_tokens + TOK - 1) / TOK;
  const int h_groups = (args.heads + HG - 1) / HG;
  const int tt = bid % t_tiles; bid /= t_tiles;
  const int hg = bid % h_groups; bid /= h_groups;
  const int b = bid % args.batch; bid /= args.batch;
  const int kv = bid & 1;
  const int layer = bid >> 1;
  const DLayerIO& L = args.layers[layer];
  const bool key = (kv == 0);
  const uint8_t* codes = key ? L.k_codes : L.v_codes;
  if (codes == nullptr) return;
  const int levels = key ? L.key_levels : L.value_levels;
  const int tid = threadIdx.x;
  const int j = tt * TOK + tid / HG;
  const int head = hg * HG + tid % HG;
  const int count = args.count ? min(args.count[b], args.n_tokens) : args.n_tokens;
  if (j >= count || head >= args.heads) return;

  const int64_t vrow = ((int64_t)b * args.heads + head) * args.n_tokens + j;
  const int pb = packed_bytes_of(DP, levels);
  const uint8_t* p = codes + vrow * pb;
  float x[DP];
  if (levels <= 4) {
#pragma unroll
    for (int k = 0; k < DP / 32; ++k) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + k);
      const uint32_t ww[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          x[32 * k + 8 * q + i] = static_cast<float>(static_cast<int>((ww[q] >> (4 * i)) & 0xFu) - 8);
    }
  } else if (levels == 8) {
    uint32_t ww[DP * 5 / 32];
    if ((pb & 15) == 0) {
#pragma unroll
      for (int k = 0; k < DP * 5 / 128; ++k) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + k);
        ww[4 * k] = u.x; ww[4 * k + 1] = u.y; ww[4 * k + 2] = u.z; ww[4 * k + 3] = u.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < DP * 5 / 64; ++k) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(p) + k);
        ww[2 * k] = u.x; ww[2 * k + 1] = u.y;
      }
    }
#pragma unroll
    for (int g = 0; g < DP / 8; ++g) {
      const int bit = 40 * g;
      const int wi = bit >> 5, sh = bit & 31;
      uint64_t v = (static_cast<uint64_t>(ww[wi + 1]) << 32 | ww[wi]) >> sh;
      if (sh > 24) v |= static_cast<uint64_t>(ww[wi + 2]) << (64 - sh);
#pragma unroll
      for (int i = 0; i < 8; ++i) x[8 * g + i] = static_cast<float>(static_cast<int>((v >> (5 * i)) & 31u) - 8);
    }
  } else {
#pragma unroll
    for (int k = 0; k < DP / 16; ++k) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + k);
      const uint32_t ww[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          x[16 * k + 4 * q + i] = static_cast<float>(static_cast<int8_t>((ww[q] >> (8 * i)) & 0xFFu));
    }
  }
  const uint16_t* s16 = key ? L.k_scales : L.v_scales;
  const float scale = __half2float(__ushort_as_half(s16[vrow]));
  const int pos = key ? args.positions[(int64_t)b * args.n_tokens + j] : 0;
  uint16_t* out = key ? L.k_out : L.v_out;
  __half* o = reinterpret_cast<__half*>(out) + (int64_t)b * args.out_stride_b + (int64_t)head * args.out_stride_h +
              (int64_t)j * args.out_stride_t;
  constexpr int DH = D / 2;
  reconstruct_store<D, DP>(x, scale, key, args.rope_cos + (int64_t)pos * DH, args.rope_sin + (int64_t)pos * DH,
                           args.key_sharpen, o);
}

// --------------------------------------------------------------------------
// Launchers
// --------------------------------------------------------------------------
cudaError_t launch_decompress(const DecompressArgs& a, int n_layers, cudaStream_t s) {
  const int tok = kCompressThreads / a.head_group;
  const long long blocks = (long long)n_layers * 2 * a.batch * ((a.heads + a.head_group - 1) / a.head_group) *
                           ((a.n_tokens + tok - 1) / tok);
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  if (a.head_dim == 128 && a.head_dim_padded == 128)
    decompress_kernel<128, 128><<<(int)blocks, kCompressThreads, 0, s>>>(a);
  else if (a.head_dim == 96 && a.head_dim_padded == 128)
    decompress_kernel<96, 128><<<(int)blocks, kCompressThreads, 0, s>>>(a);
  else if (a.head_dim == 64 && a.head_dim_padded == 64)
    decompress_kernel<64, 64><<<(int)blocks, kCompressThreads, 0, s>>>(a);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace nq
