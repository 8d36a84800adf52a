// Dequantize kernel (sm_100a): packed lattice codes -> fp16 K / V rows.
//
// Per vector: unpack codes c (= 2 * lattice point, integers in [-16, 16]) ->
// inverse Walsh-Hadamard -> * fl32(scale * 0.5 / sqrt(d_p)) -> [keys] forward
// split-half RoPE at the token's position -> [keys] * sharpen -> fp16.
// Reference: nexusquant/integrations/vllm_backend.py:319-338 (_dequantize_perhead),
// :398-429 (decompress_page); nexusquant/core/rope_utils.py:75-122.
//
// Design:
//  * One thread per vector.  The butterfly runs on the integer codes, whose
//    partial sums stay within +-16 * d_p <= 2048: every intermediate is an
//    integer that fp16 represents exactly, so the transform runs as packed
//    half2 adds (two coordinates per instruction, half the registers of fp32)
//    and equals the fp32 transform bit for bit.  Register q holds coordinates
//    {q, q + d_p/2}; the last stage is one HFMA2 inside the register.
//  * Codes become half2 integers without any int->float conversion: a field f
//    placed in the mantissa of 1024.0 (bits 0x6400 | f) is the half 1024 + f,
//    and one HADD2 / HFMA2 removes the bias.
//  * Scale, RoPE and sharpening run in fp32 (packed f32x2 where both lanes
//    share the operation), in the same order and rounding as the CPU oracle.
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

__device__ __forceinline__ __half2 h2_bits(uint32_t u) {
  __half2 h;
  *reinterpret_cast<uint32_t*>(&h) = u;
  return h;
}
__device__ __forceinline__ __half2 h2_const(float a) { return __floats2half2_rn(a, a); }

// {f_lo - 8, f_hi - 8} from 4-bit fields at bit SH (0 or 4) of the two 16-bit lanes of u.
template <int SH>
__device__ __forceinline__ __half2 nibble_pair(uint32_t u) {
  const __half2 h = h2_bits((u & (0x000F000Fu << SH)) | 0x64006400u);  // 1024 + f * 2^SH
  if constexpr (SH == 0) return __hadd2(h, h2_const(-1032.0f));
  else return __hfma2(h, h2_const(1.0f / 16.0f), h2_const(-72.0f));   // 64 + f - 72
}

// Load the packed row (PB bytes, 16-byte aligned) into words.
template <int PB>
__device__ __forceinline__ void load_row(const uint8_t* p, uint32_t (&w)[PB / 4]) {
  if constexpr (PB % 16 == 0) {
#pragma unroll
    for (int k = 0; k < PB / 16; ++k) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + k);
      w[4 * k] = u.x; w[4 * k + 1] = u.y; w[4 * k + 2] = u.z; w[4 * k + 3] = u.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < PB / 8; ++k) {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(p) + k);
      w[2 * k] = u.x; w[2 * k + 1] = u.y;
    }
  }
}

// Codes of coordinates {q, q + DP/2} as half2 integers, for every q < DP/2.
// FMT: 0 = nibbles (field = c + 8), 1 = 5-bit fields (c + 8), 2 = int8 (c).
template <int DP, int FMT>
__device__ __forceinline__ void unpack_codes(const uint8_t* p, __half2 (&R)[DP / 2]) {
  constexpr int HR = DP / 2;
  if constexpr (FMT == 0) {
    uint32_t w[DP / 8];
    load_row<DP / 2>(p, w);
#pragma unroll
    for (int q = 0; q < HR; q += 2) {
      const int m = q >> 3, byte = (q & 7) >> 1;
      const uint32_t u = __byte_perm(w[m], w[m + HR / 8], (uint32_t)((4 + byte) << 8 | byte));
      R[q] = nibble_pair<0>(u);
      R[q + 1] = nibble_pair<4>(u);
    }
  } else if constexpr (FMT == 1) {
    uint32_t w[DP * 5 / 32];
    load_row<DP * 5 / 8>(p, w);
    constexpr int OFF = 5 * HR / 32;  // word offset of coordinate q + DP/2
#pragma unroll
    for (int q = 0; q < HR; ++q) {
      const int bit = 5 * q, k = bit >> 5, s = bit & 31;
      uint32_t lo, hi;
      if (s + 5 <= 32) {
        lo = w[k] >> s;
        hi = w[k + OFF] >> s;
      } else {
        lo = __funnelshift_r(w[k], w[k + 1], s);
        hi = __funnelshift_r(w[k + OFF], w[k + OFF + 1], s);
      }
      const uint32_t u = __byte_perm(lo, hi, 0x5410u);
      R[q] = __hadd2(h2_bits((u & 0x001F001Fu) | 0x64006400u), h2_const(-1032.0f));
    }
  } else {
    uint32_t w[DP / 4];
    load_row<DP>(p, w);
#pragma unroll
    for (int q = 0; q < HR; ++q) {
      const int m = q >> 2, byte = q & 3;
      const uint32_t u = __byte_perm(w[m], w[m + HR / 4], (uint32_t)((4 + byte) << 8 | byte));
      // signed byte c -> 0x6400 | (c + 128) = half(1152 + c)
      R[q] = __hadd2(h2_bits((u & 0x00FF00FFu) ^ 0x64806480u), h2_const(-1152.0f));
    }
  }
}

// Unnormalised Walsh-Hadamard butterfly (stride 1, 2, 4, ...) on exact half2 integers.
template <int DP>
__device__ __forceinline__ void fwht_half2(__half2 (&R)[DP / 2]) {
  constexpr int HR = DP / 2;
#pragma unroll
  for (int st = 1; st < HR; st <<= 1) {
#pragma unroll
    for (int q = 0; q < HR; ++q) {
      if ((q & st) == 0) {
        const __half2 a = R[q], b = R[q + st];
        R[q] = __hadd2(a, b);
        R[q + st] = __hsub2(a, b);
      }
    }
  }
  // stride DP/2: {lo, hi} -> {lo + hi, lo - hi}
  const __half2 pm = __floats2half2_rn(1.0f, -1.0f);
#pragma unroll
  for (int q = 0; q < HR; ++q) R[q] = __hfma2(__high2half2(R[q]), pm, __low2half2(R[q]));
}

// Coordinate k of the transformed vector, as float.
template <int DP>
__device__ __forceinline__ float coord(const __half2 (&R)[DP / 2], int k) {
  return k < DP / 2 ? __low2float(R[k]) : __high2float(R[k - DP / 2]);
}

__device__ __forceinline__ uint32_t h2u(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void st_global_v8(void* p, const uint32_t (&v)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// Scale, [RoPE, sharpen] and store coordinates [0, D) as fp16.  Chunk c (outputs W*c ..
// W*c + W-1) is paired with chunk c + D/(2W), their RoPE partners at + D/2.  W = 16 with
// 32-byte stores (one full sector per lane) when the rows are 32-byte aligned, else 8.
template <int D, int DP, bool KEY, bool V8>
__device__ __forceinline__ void finish_store(const __half2 (&R)[DP / 2], float coef, const float* cosr,
                                             const float* sinr, float sharpen, __half* out) {
  constexpr int DH = D / 2;
  constexpr int W = V8 ? 16 : 8;
  static_assert(DH % W == 0, "chunk width must divide D/2");
  const u64 coef2 = pk(coef, coef), sh2 = pk(sharpen, sharpen);
#pragma unroll
  for (int c = 0; c < DH / W; ++c) {
    uint32_t o1[W / 2], o2[W / 2];
#pragma unroll
    for (int u = 0; u < W; u += 2) {
      float y1[2], y2[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = W * c + u + e;
        u64 z = mul2(pk(coord<DP>(R, i), coord<DP>(R, i + DH)), coef2);  // {z1, z2}
        if constexpr (KEY) {
          // cosr / sinr point into shared memory
          const float cu = cosr[i], su = sinr[i];
          float m1, m2, n1, n2;
          upk(mul2(z, pk(cu, cu)), m1, m2);  // z1 c, z2 c
          upk(mul2(z, pk(su, su)), n1, n2);  // z1 s, z2 s
          z = pk(__fsub_rn(m1, n2), __fadd_rn(n1, m2));
          if (sharpen != 1.0f) z = mul2(z, sh2);
        }
        upk(z, y1[e], y2[e]);
      }
      o1[u / 2] = h2u(y1[0], y1[1]);
      o2[u / 2] = h2u(y2[0], y2[1]);
    }
    if constexpr (V8) {
      st_global_v8(out + W * c, o1);
      st_global_v8(out + DH + W * c, o2);
    } else {
      reinterpret_cast<uint4*>(out)[c] = make_uint4(o1[0], o1[1], o1[2], o1[3]);
      reinterpret_cast<uint4*>(out + DH)[c] = make_uint4(o2[0], o2[1], o2[2], o2[3]);
    }
  }
}

// --------------------------------------------------------------------------
// One CTA: HG heads x (128 / HG) tokens of one (layer, K|V, batch); one thread per vector.
// --------------------------------------------------------------------------
// RoPE rows of a tile in shared memory: per token cos[D/2] then sin[D/2], rows padded by
// 16 bytes so the HG-lane broadcasts of different tokens fall in different banks.
template <int D>
struct RopeSmem {
  static constexpr int kRow = 4 * D + 16;
  static constexpr int kChunks = 4 * D / 16;  // 16-byte chunks per token (cos + sin)
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

template <int D, int DP, bool KEY, int FMT, bool V8>
__device__ __forceinline__ void decompress_vector(const DecompressArgs& args, const DLayerIO& L, int b, int head,
                                                  int j, bool valid, uint8_t* rope_smem) {
  const int64_t vrow = ((int64_t)b * args.heads + head) * args.n_tokens + j;
  constexpr int DH = D / 2;
  const int HG = args.head_group;
  float* trow = nullptr;
  if constexpr (KEY) {
    // the HG threads of this token copy its cos / sin rows into shared memory while the
    // butterfly runs (they are consecutive lanes of one warp)
    trow = reinterpret_cast<float*>(rope_smem + (threadIdx.x / HG) * RopeSmem<D>::kRow);
    if (valid) {
      const int pos = min(max(args.positions[(int64_t)b * args.n_tokens + j], 0), args.rope_rows - 1);
      const int hl = threadIdx.x % HG;
      for (int c = hl; c < RopeSmem<D>::kChunks; c += HG) {
        const int half = c / (RopeSmem<D>::kChunks / 2), k = c % (RopeSmem<D>::kChunks / 2);
        const float* src = (half ? args.rope_sin : args.rope_cos) + (int64_t)pos * DH + 4 * k;
        cp_async16(trow + half * DH + 4 * k, src);
      }
    }
  }
  constexpr int PB = FMT == 0 ? DP / 2 : (FMT == 1 ? DP * 5 / 8 : DP);
  __half2 R[DP / 2];
  float coef = 0.0f;
  if (valid) {
    unpack_codes<DP, FMT>((KEY ? L.k_codes : L.v_codes) + vrow * PB, R);
    fwht_half2<DP>(R);
    const float scale = __half2float(__ushort_as_half((KEY ? L.k_scales : L.v_scales)[vrow]));
    coef = __fmul_rn(scale, 0.5f * hadamard_entry(DP));
  }
  if constexpr (KEY) {
    cp_async_wait_all();
    __syncwarp();
  }
  if (!valid) return;
  __half* o = reinterpret_cast<__half*>(KEY ? L.k_out : L.v_out) + (int64_t)b * args.out_stride_b +
              (int64_t)head * args.out_stride_h + (int64_t)j * args.out_stride_t;
  finish_store<D, DP, KEY, V8>(R, coef, trow, trow + DH, args.key_sharpen, o);
}

// KEY: this launch covers the key rows (true) or the value rows (false) of every layer; one
// half per kernel keeps each kernel's code (three packing formats) small for the i-cache.
// 5 CTAs per SM for keys (93 registers) and 6 for values (80; 5 at d = 96), without spills:
// the kernel is latency-bound on its code loads, and the extra warps hide it (4 CTAs: 0.625
// of the measured HBM peak on config 3, 5: 0.679).
template <int D, int DP, bool V8, bool KEY>
__global__ void __launch_bounds__(kCompressThreads, (KEY || D == 96) ? 5 : 6) decompress_kernel(const DecompressArgs args) {
  extern __shared__ __align__(16) uint8_t rope_smem[];
  const int HG = args.head_group;
  const int TOK = kCompressThreads / HG;
  int bid = blockIdx.x;
  const int t_tiles = (args.n_tokens + TOK - 1) / TOK;
  const int h_groups = (args.heads + HG - 1) / HG;
  const int tt = bid % t_tiles; bid /= t_tiles;
  const int hg = bid % h_groups; bid /= h_groups;
  const int b = bid % args.batch; bid /= args.batch;
  const int layer = bid;
  const DLayerIO& L = args.layers[layer];
  if ((KEY ? L.k_codes : L.v_codes) == nullptr) return;
  const int j = tt * TOK + threadIdx.x / HG;
  const int head = hg * HG + threadIdx.x % HG;
  const int count = args.count ? min(args.count[b], args.n_tokens) : args.n_tokens;
  // invalid threads stay until the warp-level barrier of the key path
  const bool valid = j < count && head < args.heads;
  const int levels = KEY ? L.key_levels : L.value_levels;
  const int fmt = levels <= 4 ? 0 : (levels == 8 ? 1 : 2);
  if (fmt == 0) decompress_vector<D, DP, KEY, 0, V8>(args, L, b, head, j, valid, rope_smem);
  else if (fmt == 1) decompress_vector<D, DP, KEY, 1, V8>(args, L, b, head, j, valid, rope_smem);
  else decompress_vector<D, DP, KEY, 2, V8>(args, L, b, head, j, valid, rope_smem);
}

template <int D, int DP, bool V8>
static cudaError_t launch_dq_t(const DecompressArgs& a, long long blocks, cudaStream_t s) {
  const int smem = (kCompressThreads / a.head_group) * RopeSmem<D>::kRow;
  cudaError_t e =
      cudaFuncSetAttribute(decompress_kernel<D, DP, V8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  decompress_kernel<D, DP, V8, true><<<(int)blocks, kCompressThreads, smem, s>>>(a);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  decompress_kernel<D, DP, V8, false><<<(int)blocks, kCompressThreads, 0, s>>>(a);  // values: no RoPE rows
  return cudaGetLastError();
}

// 32-byte stores need every output row and half-row to start on a 32-byte boundary.
static bool rows_32b_aligned(const DecompressArgs& a, int n_layers) {
  if ((a.out_stride_b * 2) % 32 || (a.out_stride_h * 2) % 32 || (a.out_stride_t * 2) % 32 || a.head_dim % 32)
    return false;
  for (int l = 0; l < n_layers; ++l) {
    if ((reinterpret_cast<uintptr_t>(a.layers[l].k_out) | reinterpret_cast<uintptr_t>(a.layers[l].v_out)) & 31)
      return false;
  }
  return true;
}

template <int D, int DP>
static cudaError_t launch_dq(const DecompressArgs& a, int n_layers, long long blocks, cudaStream_t s) {
  return rows_32b_aligned(a, n_layers) ? launch_dq_t<D, DP, true>(a, blocks, s) : launch_dq_t<D, DP, false>(a, blocks, s);
}

// --------------------------------------------------------------------------
// Launcher
// --------------------------------------------------------------------------
cudaError_t launch_decompress(const DecompressArgs& a, int n_layers, cudaStream_t s) {
  const int tok = kCompressThreads / a.head_group;
  const long long blocks = (long long)n_layers * a.batch * ((a.heads + a.head_group - 1) / a.head_group) *
                           ((a.n_tokens + tok - 1) / tok);
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  if (a.head_dim == 128 && a.head_dim_padded == 128) return launch_dq<128, 128>(a, n_layers, blocks, s);
  if (a.head_dim == 96 && a.head_dim_padded == 128) return launch_dq<96, 128>(a, n_layers, blocks, s);
  if (a.head_dim == 64 && a.head_dim_padded == 64) return launch_dq<64, 64>(a, n_layers, blocks, s);
  return cudaErrorInvalidValue;
}

}  // namespace nq
