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
//  * A warp owns 32 consecutive tokens of one head.  The tile's RoPE rows are
//    copied to shared memory by cp.async while the butterfly runs, and the
//    warp's fp16 rows are staged in shared memory and leave as contiguous
//    512-byte stores (thread-per-row stores reach only ~80 % of the HBM
//    bandwidth that coalesced ones do for this 1:4 read:write mix).
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

// Packed row bytes and words of one vector.
template <int DP, int FMT>
struct Packed {
  static constexpr int kBytes = FMT == 0 ? DP / 2 : (FMT == 1 ? DP * 5 / 8 : DP);
  static constexpr int kWords = kBytes / 4;
};

// Codes of coordinates {q, q + DP/2} as half2 integers, for every q < DP/2, from the
// row's words.  FMT: 0 = nibbles (field = c + 8), 1 = 5-bit fields (c + 8), 2 = int8 (c).
template <int DP, int FMT>
__device__ __forceinline__ void unpack_codes(const uint32_t (&w)[Packed<DP, FMT>::kWords], __half2 (&R)[DP / 2]) {
  constexpr int HR = DP / 2;
  if constexpr (FMT == 0) {
#pragma unroll
    for (int q = 0; q < HR; q += 2) {
      const int m = q >> 3, byte = (q & 7) >> 1;
      const uint32_t u = __byte_perm(w[m], w[m + HR / 8], (uint32_t)((4 + byte) << 8 | byte));
      R[q] = nibble_pair<0>(u);
      R[q + 1] = nibble_pair<4>(u);
    }
  } else if constexpr (FMT == 1) {
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

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ float4 ld_shared_f4(const void* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ uint4 ld_shared_u4(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}

// --------------------------------------------------------------------------
// Tile geometry.  A CTA of 4 warps covers HGT heads x (128 / HGT) tokens of one
// (layer, K|V, batch), HGT = min(4, head_group); warp w takes head w % HGT and the
// 32 consecutive tokens of block w / HGT, one token per lane.  A warp's output rows
// are then one head's consecutive tokens: they go through shared memory and leave
// as 512-byte contiguous stores, and its code rows / scales are contiguous loads.
// --------------------------------------------------------------------------
template <int D>
struct DqSmem {
  static constexpr int kOutRow = 2 * D + 16;                 // fp16 row + pad (conflict-free 16-byte access)
  static constexpr int kOut = 4 * 32 * kOutRow;              // staging of the 4 warps
  static constexpr int kRopeRow = 4 * D + 16;                // cos[D/2], sin[D/2], pad
  static constexpr int kRopeChunks = 4 * D / 16;
  static int bytes(int hgt) { return kOut + (128 / hgt) * kRopeRow; }
};

__host__ __device__ __forceinline__ int dq_heads_per_tile(int head_group) { return head_group < 4 ? head_group : 4; }
static inline int dq_heads_per_tile_host(int head_group) { return dq_heads_per_tile(head_group); }

// Scale, [RoPE, sharpen], convert to fp16 and write the row into shared memory.  Output
// chunk c (outputs 8c .. 8c+7) is paired with chunk c + D/16 (RoPE partners at + D/2).
template <int D, int DP, bool KEY, bool SHARP>
__device__ __forceinline__ void finish_row(const __half2 (&R)[DP / 2], float coef, const uint8_t* trow,
                                           float sharpen, uint8_t* srow) {
  constexpr int DH = D / 2;
  const u64 coef2 = pk(coef, coef), sh2 = pk(sharpen, sharpen);
#pragma unroll
  for (int c = 0; c < DH / 8; ++c) {
    uint32_t o1[4], o2[4];
#pragma unroll
    for (int u = 0; u < 8; u += 4) {
      float4 cv = make_float4(0.f, 0.f, 0.f, 0.f), sv = cv;
      if constexpr (KEY) {
        cv = ld_shared_f4(trow + 4 * (8 * c + u));
        sv = ld_shared_f4(trow + 4 * (DH + 8 * c + u));
      }
      const float cc[4] = {cv.x, cv.y, cv.z, cv.w}, ss[4] = {sv.x, sv.y, sv.z, sv.w};
      float y1[4], y2[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 8 * c + u + e;
        u64 z = mul2(pk(coord<DP>(R, i), coord<DP>(R, i + DH)), coef2);  // {z1, z2}
        if constexpr (KEY) {
          float m1, m2, n1, n2;
          upk(mul2(z, pk(cc[e], cc[e])), m1, m2);  // z1 c, z2 c
          upk(mul2(z, pk(ss[e], ss[e])), n1, n2);  // z1 s, z2 s
          z = pk(__fsub_rn(m1, n2), __fadd_rn(n1, m2));
          if constexpr (SHARP) z = mul2(z, sh2);
        }
        upk(z, y1[e], y2[e]);
      }
      o1[u / 2] = h2u(y1[0], y1[1]); o1[u / 2 + 1] = h2u(y1[2], y1[3]);
      o2[u / 2] = h2u(y2[0], y2[1]); o2[u / 2 + 1] = h2u(y2[2], y2[3]);
    }
    st_shared_v4(srow + 16 * c, o1[0], o1[1], o1[2], o1[3]);
    st_shared_v4(srow + 2 * DH + 16 * c, o2[0], o2[1], o2[2], o2[3]);
  }
}

template <int D, int DP, bool KEY, int FMT, bool SHARP>
__device__ __forceinline__ void decompress_tile(const DecompressArgs& args, const DLayerIO& L, int b, int hgi,
                                                int tt, int count, uint8_t* smem) {
  using S = DqSmem<D>;
  constexpr int DH = D / 2;
  const int HGT = dq_heads_per_tile(args.head_group);
  const int TOK = kCompressThreads / HGT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = hgi * HGT + warp % HGT;
  const int j0w = tt * TOK + (warp / HGT) * 32;  // first token of this warp
  const int j = j0w + lane;
  const bool valid = j < count && head < args.heads;
  uint8_t* rope = smem + S::kOut;
  const int64_t vrow = ((int64_t)b * args.heads + head) * args.n_tokens + j;
  using P = Packed<DP, FMT>;
  uint32_t w[P::kWords];
  uint16_t sbits = 0;
  if (valid) {
    load_row<P::kBytes>((KEY ? L.k_codes : L.v_codes) + vrow * P::kBytes, w);
    sbits = (KEY ? L.k_scales : L.v_scales)[vrow];
  }
  if constexpr (KEY) {
    // cos / sin rows of the tile's tokens -> shared memory, overlapping the code loads and
    // the butterfly: the CTA's threads split evenly over the tile's tokens, one position each
    const int tok0 = tt * TOK;
    const int n_tok = min(TOK, count - tok0);
    const int tpt = kCompressThreads / TOK;  // threads per token (1, 2 or 4)
    const int t = threadIdx.x / tpt;
    if (t < n_tok) {
      const int pos = args.positions[(int64_t)b * args.n_tokens + tok0 + t];
      for (int k = threadIdx.x % tpt; k < S::kRopeChunks; k += tpt) {
        const int half = k / (S::kRopeChunks / 2), q = k % (S::kRopeChunks / 2);
        cp_async16(rope + t * S::kRopeRow + half * 4 * DH + 16 * q,
                   (half ? args.rope_sin : args.rope_cos) + (int64_t)pos * DH + 4 * q);
      }
    }
  }
  __half2 R[DP / 2];
  float coef = 0.0f;
  if (valid) {
    unpack_codes<DP, FMT>(w, R);
    fwht_half2<DP>(R);
    coef = __fmul_rn(__half2float(__ushort_as_half(sbits)), 0.5f * hadamard_entry(DP));
  }
  if constexpr (KEY) {
    cp_async_wait_all();
    __syncthreads();  // rope rows are shared across warps
  }
  uint8_t* sw = smem + warp * 32 * S::kOutRow;
  if (valid)
    finish_row<D, DP, KEY, SHARP>(R, coef, rope + ((warp / HGT) * 32 + lane) * S::kRopeRow, args.key_sharpen,
                                  sw + lane * S::kOutRow);
  __syncwarp();
  // the warp's rows leave as 16-byte chunks, each row written by 2*D/16 consecutive lanes
  if (head < args.heads) {
    constexpr int CPR = 2 * D / 16;  // chunks per row
    constexpr int RPI = 32 / CPR;    // rows per instruction
    __half* base = reinterpret_cast<__half*>(KEY ? L.k_out : L.v_out) + (int64_t)b * args.out_stride_b +
                   (int64_t)head * args.out_stride_h;
    const int cr = lane % CPR;
#pragma unroll
    for (int k = 0; k < 32 / RPI; ++k) {
      const int r = k * RPI + lane / CPR;
      if (j0w + r < count) {
        const uint4 v = ld_shared_u4(sw + r * S::kOutRow + 16 * cr);
        reinterpret_cast<uint4*>(base + (int64_t)(j0w + r) * args.out_stride_t)[cr] = v;
      }
    }
  }
}

template <int D, int DP, bool SHARP>
__global__ void __launch_bounds__(kCompressThreads, 4) decompress_kernel(const DecompressArgs args) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int HGT = dq_heads_per_tile(args.head_group);
  const int TOK = kCompressThreads / HGT;
  int bid = blockIdx.x;
  const int t_tiles = (args.n_tokens + TOK - 1) / TOK;
  const int h_groups = (args.heads + HGT - 1) / HGT;
  const int tt = bid % t_tiles; bid /= t_tiles;
  const int hgi = bid % h_groups; bid /= h_groups;
  const int b = bid % args.batch; bid /= args.batch;
  const int kv = bid & 1;
  const int layer = bid >> 1;
  const DLayerIO& L = args.layers[layer];
  const bool key = kv == 0;
  if ((key ? L.k_codes : L.v_codes) == nullptr) return;
  const int count = args.count ? min(args.count[b], args.n_tokens) : args.n_tokens;
  if (tt * TOK >= count) return;  // uniform over the CTA
  const int levels = key ? L.key_levels : L.value_levels;
  const int fmt = levels <= 4 ? 0 : (levels == 8 ? 1 : 2);
  if (key) {
    if (fmt == 0) decompress_tile<D, DP, true, 0, SHARP>(args, L, b, hgi, tt, count, smem);
    else if (fmt == 1) decompress_tile<D, DP, true, 1, SHARP>(args, L, b, hgi, tt, count, smem);
    else decompress_tile<D, DP, true, 2, SHARP>(args, L, b, hgi, tt, count, smem);
  } else {
    if (fmt == 0) decompress_tile<D, DP, false, 0, SHARP>(args, L, b, hgi, tt, count, smem);
    else if (fmt == 1) decompress_tile<D, DP, false, 1, SHARP>(args, L, b, hgi, tt, count, smem);
    else decompress_tile<D, DP, false, 2, SHARP>(args, L, b, hgi, tt, count, smem);
  }
}

template <int D, int DP>
static cudaError_t launch_dq(const DecompressArgs& a, long long blocks, cudaStream_t s) {
  const int smem = DqSmem<D>::bytes(dq_heads_per_tile_host(a.head_group));
  auto kern = a.key_sharpen != 1.0f ? decompress_kernel<D, DP, true> : decompress_kernel<D, DP, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<(unsigned)blocks, kCompressThreads, smem, s>>>(a);
  return cudaGetLastError();
}

// --------------------------------------------------------------------------
// Launcher
// --------------------------------------------------------------------------
cudaError_t launch_decompress(const DecompressArgs& a, int n_layers, cudaStream_t s) {
  const int hgt = dq_heads_per_tile_host(a.head_group);
  const int tok = kCompressThreads / hgt;
  const long long blocks = (long long)n_layers * 2 * a.batch * ((a.heads + hgt - 1) / hgt) *
                           ((a.n_tokens + tok - 1) / tok);
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  if (a.head_dim == 128 && a.head_dim_padded == 128) return launch_dq<128, 128>(a, blocks, s);
  if (a.head_dim == 96 && a.head_dim_padded == 128) return launch_dq<96, 128>(a, blocks, s);
  if (a.head_dim == 64 && a.head_dim_padded == 64) return launch_dq<64, 64>(a, blocks, s);
  return cudaErrorInvalidValue;
}

}  // namespace nq
