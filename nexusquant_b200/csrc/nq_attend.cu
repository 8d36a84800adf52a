// Decode attention straight from the compressed layout (no fp16 K/V materialised).
//
// Semantics of NexusQuantPagedAttention.forward (nexusquant/integrations/vllm_backend.py:
// 692-765): one query token per sequence, keys and values dequantized as decompress_page
// does (:398-429, keys re-rotated at their stored positions and optionally sharpened), then
// softmax(q K^T / sqrt(d)) V in fp32, fp16 output.  Query heads are grouped over the KV
// heads (q head g*G .. g*G+G-1 reads KV head g; G = 1 is the reference's case).
//
// Split-K over tokens, two kernels:
//  * attend_partial: CTA = (token split, KV head, batch), 256 threads, both contractions on
//    the 5th-generation tensor cores (tcgen05.mma kind::f16, fp32 accumulators in TMEM).
//    Per tile of 128 tokens:
//      - the two threads of token t decode its key in registers, half of the coordinate
//        pairs each (unpack -> exact half2 butterfly, one stage across the pair by shuffle ->
//        scale -> RoPE -> sharpen -> fp16, the dequantize kernel's arithmetic) into a K-major,
//        128-byte-swizzled shared tile, and convert half of value t's codes each (small
//        integers, exact in fp16) into an MN-major swizzled tile;
//      - one thread issues S = K Q^T (M = 128 tokens, N = 16 >= G query heads, K = 128);
//        thread t of warps 0-3 reads token t's logits back from TMEM lane t;
//      - online softmax over the tile; the weights p_t * s_t (value scale) go to shared
//        memory as fp16;
//      - one thread issues O = C^T W^T (M = 128 dimensions, N = 16, K = 128 tokens): values
//        stay in the code domain because the inverse Hadamard is linear,
//        sum_t p_t v_t = h/2 * H^T (sum_t p_t s_t c_t); thread j reads dimension j from
//        TMEM and folds it into its running accumulator with the softmax rescale.
//    It writes (max, sum, accumulator) per query head and split.
//  * attend_combine: per (batch, query head) merges the splits, divides by the softmax
//    sum, applies the inverse Walsh-Hadamard butterfly once and scales by h/2.
// Fixed reduction orders throughout: deterministic.
#include <algorithm>

#include "nq_common.cuh"
#include "nq_internal.h"
#include "nq_umma.cuh"

namespace nq {

namespace {

constexpr int kAtTok = 128;  // tokens per tile = TMEM lanes
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

template <int FMT>
constexpr int at_pb() { return FMT == 0 ? 64 : (FMT == 1 ? 80 : 128); }

}  // namespace


// Device error word of the attention kernel's bounded waits (bit 2 of nq_device_error).
__device__ unsigned int g_attend_wait_error;

// Shared-memory plan of attend_partial (offsets from a 1024-byte aligned base).
struct AtSmem {
  static constexpr int kK = 0;          // keys: 2 column blocks x 128 rows x 128 B, K-major SW128
  static constexpr int kV = 32768;      // value codes: 2 M blocks (64 dims) x 16 groups of 8 tokens x 1024 B
  static constexpr int kQ = 65536;      // queries: 2 column blocks x 16 rows x 128 B
  static constexpr int kW = 69632;      // weights: 2 token blocks x 16 rows x 128 B
  static constexpr int kBytes = 73728 + 1024;  // + alignment slack
  static constexpr int kN = 16;         // MMA N (query heads, zero rows above G)
};

// Byte offset of element (row, col) of a K-major SW128 operand with 128-byte rows grouped
// in column blocks of 64 elements (block stride `blk`): 16-byte chunk index XOR row % 8.
__device__ __forceinline__ uint32_t sw128_off(int row, int col, int blk) {
  return (uint32_t)((col >> 6) * blk + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2);
}

// Value codes of dimensions 2p, 2p + 1 as a half2 of exact integers, from a packed row in words.
template <int FMT>
__device__ __forceinline__ uint32_t at_code_pair(const uint32_t* w, int p) {
  if constexpr (FMT == 0) {
    // byte p holds dimensions 2p (low nibble) and 2p + 1 (high nibble): [byte, 0, byte, 0]
    const uint32_t x = __byte_perm(w[p >> 2], 0u, 0x4040u + (uint32_t)(p & 3) * 0x0101u);
    const __half2 h = __hfma2(ah2_bits((x & 0x00F0000Fu) | 0x64006400u), __floats2half2_rn(1.0f, 1.0f / 16.0f),
                              __floats2half2_rn(-1032.0f, -72.0f));
    return *reinterpret_cast<const uint32_t*>(&h);
  } else if constexpr (FMT == 1) {
    uint32_t f[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int bit = 5 * (2 * p + e), k = bit >> 5, sh = bit & 31;
      f[e] = (sh + 5 <= 32 ? (w[k] >> sh) : __funnelshift_r(w[k], w[k + 1], sh)) & 31u;
    }
    const __half2 h = __hadd2(ah2_bits(f[0] | (f[1] << 16) | 0x64006400u), ah2c(-1032.0f));
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const uint32_t x = __byte_perm(w[p >> 1], 0u, (p & 1) ? 0x4342u : 0x4140u);
    const __half2 h = __hadd2(ah2_bits((x ^ 0x00800080u) | 0x64006400u), ah2c(-1152.0f));
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

// Codes of coordinates {q, q + 64} for the 32 pairs q in [32 h, 32 h + 32) of a packed row, as
// half2 integers (R[q - 32 h]): the half of the key that thread h of a token's pair decodes.
template <int FMT>
__device__ __forceinline__ void at_unpack_half(const uint8_t* p, int h, bool valid, __half2 (&R)[32]) {
  if constexpr (FMT == 0) {
    // dims [32h, 32h + 32): bytes [16h, 16h + 16); dims + 64: bytes [32 + 16h, 48 + 16h)
    uint32_t wl[4] = {0u, 0u, 0u, 0u}, wh[4] = {0u, 0u, 0u, 0u};
    if (valid) {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(p + 16 * h));
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(p + 32 + 16 * h));
      wl[0] = a.x; wl[1] = a.y; wl[2] = a.z; wl[3] = a.w;
      wh[0] = b.x; wh[1] = b.y; wh[2] = b.z; wh[3] = b.w;
    }
#pragma unroll
    for (int q = 0; q < 32; q += 2) {
      const int m = q >> 3, byte = (q & 7) >> 1;
      const uint32_t u = __byte_perm(wl[m], wh[m], (uint32_t)((4 + byte) << 8 | byte));
      R[q] = __hadd2(ah2_bits((u & 0x000F000Fu) | 0x64006400u), ah2c(-1032.0f));
      R[q + 1] = __hfma2(ah2_bits((u & 0x00F000F0u) | 0x64006400u), ah2c(1.0f / 16.0f), ah2c(-72.0f));
    }
  } else if constexpr (FMT == 1) {
    // dims [32h, 32h + 32): bits [160h, 160h + 160) = bytes [20h, 20h + 20); dims + 64: + 40 bytes
    uint32_t wl[6] = {0u, 0u, 0u, 0u, 0u, 0u}, wh[6] = {0u, 0u, 0u, 0u, 0u, 0u};
    if (valid) {
      const uint32_t* pl = reinterpret_cast<const uint32_t*>(p + 20 * h);
      const uint32_t* ph = reinterpret_cast<const uint32_t*>(p + 40 + 20 * h);
#pragma unroll
      for (int k = 0; k < 5; ++k) { wl[k] = __ldg(pl + k); wh[k] = __ldg(ph + k); }
    }
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      const int bit = 5 * q, k = bit >> 5, s = bit & 31;
      const uint32_t lo = __funnelshift_r(wl[k], wl[k + 1], s), hi = __funnelshift_r(wh[k], wh[k + 1], s);
      const uint32_t u = __byte_perm(lo, hi, 0x5410u);
      R[q] = __hadd2(ah2_bits((u & 0x001F001Fu) | 0x64006400u), ah2c(-1032.0f));
    }
  } else {
    // dims [32h, 32h + 32): bytes [32h, 32h + 32); dims + 64: bytes [64 + 32h, 96 + 32h)
    uint32_t wl[8], wh[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) { wl[k] = 0u; wh[k] = 0u; }
    if (valid) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(p + 32 * h) + k);
        const uint4 b = __ldg(reinterpret_cast<const uint4*>(p + 64 + 32 * h) + k);
        wl[4 * k] = a.x; wl[4 * k + 1] = a.y; wl[4 * k + 2] = a.z; wl[4 * k + 3] = a.w;
        wh[4 * k] = b.x; wh[4 * k + 1] = b.y; wh[4 * k + 2] = b.z; wh[4 * k + 3] = b.w;
      }
    }
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      const int m = q >> 2, byte = q & 3;
      const uint32_t u = __byte_perm(wl[m], wh[m], (uint32_t)((4 + byte) << 8 | byte));
      R[q] = __hadd2(ah2_bits((u & 0x00FF00FFu) ^ 0x64806480u), ah2c(-1152.0f));
    }
  }
}

// 256 threads: two per token for the decode (thread h of the pair takes pairs [32h, 32h + 32)
// of the key and dimensions [64h, 64h + 64) of the value); warps 0-3 (one thread per TMEM lane)
// run the softmax and the accumulator.  2 CTAs per SM (74 KB of shared memory each), one wave
// (attend_splits).
constexpr int kAtThreads = 256;

template <int FMTK, int FMTV, int G>
__global__ void __launch_bounds__(kAtThreads, 2) attend_partial(const AttendArgs a) {
  constexpr int PBV = at_pb<FMTV>();
  extern __shared__ uint8_t at_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(at_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kb = sm + AtSmem::kK;
  uint8_t* vb = sm + AtSmem::kV;
  uint8_t* qb = sm + AtSmem::kQ;
  uint8_t* wb = sm + AtSmem::kW;
  __shared__ uint64_t barS, barO;
  __shared__ uint32_t tmem_base;
  __shared__ float red[G][4];
  __shared__ int err;
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tok = tid >> 1, hh = tid & 1;  // decode: token of the tile, half
  const bool smx = warp < 4;               // softmax / accumulator thread: TMEM lane tid
  const int count = a.count ? min(a.count[b], a.n_tokens) : a.n_tokens;
  const int t0 = split * a.tokens_per_split, t1 = min(count, t0 + a.tokens_per_split);
  const float qscale = a.scale * kAtLog2e;

  // queries (fp16, exact) and the zero rows G..15 of the query and weight operands
  for (int e = tid; e < (AtSmem::kW + 4096 - AtSmem::kQ) / 16; e += kAtThreads)
    reinterpret_cast<uint4*>(qb)[e] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    mbar_init(&barS, 1);
    mbar_init(&barO, 1);
    fence_mbar_init();
    err = 0;
  }
  if (warp == 0) tmem_alloc(&tmem_base, 32);
  __syncthreads();
  for (int e = tid; e < G * kAtD; e += kAtThreads) {
    const int g = e / kAtD, j = e % kAtD;
    *reinterpret_cast<__half*>(qb + sw128_off(g, j, 2048)) =
        a.q[(int64_t)b * a.q_stride_b + (int64_t)(kh * G + g) * a.q_stride_h + j];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tS = tmem_base, tO = tmem_base + 16;
  const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
  constexpr uint32_t kIdescQK = f16_idesc(0, 128, AtSmem::kN);
  constexpr uint32_t kIdescPV = f16_idesc(0, 128, AtSmem::kN) | (1u << 15);  // A (value codes) MN-major

  float m[G], lsum[G], acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) { m[g] = -INFINITY; lsum[g] = 0.0f; acc[g] = 0.0f; }
  const int64_t row0 = ((int64_t)b * a.heads + kh) * a.n_tokens;
  const float coef_h = 0.5f * hadamard_entry(kAtD);
  const __half2 sg = hh ? ah2c(-1.0f) : ah2c(1.0f);
  uint32_t ph = 0;
  for (int base = t0; base < t1; base += kAtTok, ph ^= 1u) {
    const int t = base + tok;
    const bool valid = t < t1;  // shared by both threads of the pair: the shuffle below is uniform
    // ---- key t, pairs [32 hh, 32 hh + 32) -> row tok of the key tile
    {
      __half2 R[32];
      at_unpack_half<FMTK>(a.k_codes + (row0 + (valid ? t : t0)) * at_pb<FMTK>(), hh, valid, R);
#pragma unroll
      for (int st = 1; st < 32; st <<= 1)
#pragma unroll
        for (int q = 0; q < 32; ++q)
          if ((q & st) == 0) {
            const __half2 x = R[q], y = R[q + st];
            R[q] = __hadd2(x, y);
            R[q + st] = __hsub2(x, y);
          }
      // stride 32 crosses the pair: lower thread x + y, upper thread x - y (x = lower's value)
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        const uint32_t mine = *reinterpret_cast<const uint32_t*>(&R[q]);
        const uint32_t o = __shfl_xor_sync(0xffffffffu, mine, 1);
        R[q] = __hfma2(R[q], sg, ah2_bits(o));
      }
      const __half2 pm = __floats2half2_rn(1.0f, -1.0f);
#pragma unroll
      for (int q = 0; q < 32; ++q) R[q] = __hfma2(__high2half2(R[q]), pm, __low2half2(R[q]));
      if (valid) {
        const float coef = __fmul_rn(__half2float(__ushort_as_half(a.k_scales[row0 + t])), coef_h);
        const int pos = min(max(a.positions[(int64_t)b * a.n_tokens + t], 0), a.rope_rows - 1);
        const float* cs = a.rope_cos + (int64_t)pos * (kAtD / 2) + 32 * hh;
        const float* sn = a.rope_sin + (int64_t)pos * (kAtD / 2) + 32 * hh;
        const u64 coef2 = pk(coef, coef), sh2 = pk(a.key_sharpen, a.key_sharpen);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          const float4 c0 = __ldg(reinterpret_cast<const float4*>(cs + i));
          const float4 c1 = __ldg(reinterpret_cast<const float4*>(cs + i + 4));
          const float4 s0 = __ldg(reinterpret_cast<const float4*>(sn + i));
          const float4 s1 = __ldg(reinterpret_cast<const float4*>(sn + i + 4));
          const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
          const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int u = 0; u < 8; u += 2) {
            float k1[2], k2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float2 r = __half22float2(R[i + u + e]);
              float z1, z2, m1, m2, n1, n2;
              upk(mul2(pk(r.x, r.y), coef2), z1, z2);
              upk(mul2(pk(z1, z2), pk(cc[u + e], cc[u + e])), m1, m2);
              upk(mul2(pk(z1, z2), pk(ss[u + e], ss[u + e])), n1, n2);
              u64 kk = pk(__fsub_rn(m1, n2), __fadd_rn(n1, m2));
              if (a.key_sharpen != 1.0f) kk = mul2(kk, sh2);
              upk(kk, k1[e], k2[e]);
            }
            const __half2 hl = __floats2half2_rn(k1[0], k1[1]), hv = __floats2half2_rn(k2[0], k2[1]);
            lo[u / 2] = *reinterpret_cast<const uint32_t*>(&hl);
            hi[u / 2] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          const int c = 4 * hh + (i >> 3);  // 16-byte chunk of dimensions 32 hh + i ..
          *reinterpret_cast<uint4*>(kb + tok * 128 + ((c ^ (tok & 7)) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          *reinterpret_cast<uint4*>(kb + 16384 + tok * 128 + ((c ^ (tok & 7)) << 4)) =
              make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
      } else {
#pragma unroll
        for (int c = 4 * hh; c < 4 * hh + 4; ++c) {
          *reinterpret_cast<uint4*>(kb + tok * 128 + (c << 4)) = make_uint4(0u, 0u, 0u, 0u);
          *reinterpret_cast<uint4*>(kb + 16384 + tok * 128 + (c << 4)) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
    }
    // ---- value t's codes, dimensions [64 hh, 64 hh + 64) -> M block hh of the value tile
    {
      // this half's codes: dims [64 hh, 64 hh + 64) = bytes [PBV/2 hh, PBV/2 (hh + 1)) (local words)
      constexpr int HW = PBV / 8;  // words per half row
      uint32_t w[HW + 1];
#pragma unroll
      for (int k = 0; k <= HW; ++k) w[k] = 0u;
      if (valid) {
        const uint32_t* src = reinterpret_cast<const uint32_t*>(a.v_codes + (row0 + t) * PBV + hh * (PBV / 2));
        if constexpr (FMTV == 1) {
#pragma unroll
          for (int k = 0; k < HW; ++k) w[k] = __ldg(src + k);  // 40-byte halves: 4-byte aligned
        } else {
#pragma unroll
          for (int k = 0; k < HW / 4; ++k) {
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(src) + k);
            w[4 * k] = u.x; w[4 * k + 1] = u.y; w[4 * k + 2] = u.z; w[4 * k + 3] = u.w;
          }
        }
      }
      uint8_t* vrow = vb + hh * 16384 + (tok >> 3) * 1024 + (tok & 7) * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 8 dimensions per 16-byte chunk
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (valid) {
          const int p0 = 4 * c;  // first dimension pair of the chunk, within this half
          v.x = at_code_pair<FMTV>(w, p0);
          v.y = at_code_pair<FMTV>(w, p0 + 1);
          v.z = at_code_pair<FMTV>(w, p0 + 2);
          v.w = at_code_pair<FMTV>(w, p0 + 3);
        }
        *reinterpret_cast<uint4*>(vrow + ((c ^ (tok & 7)) << 4)) = v;
      }
    }
    const bool vs = smx && base + tid < t1;  // softmax token tid of the tile
    const float sv = vs ? __half2float(__ushort_as_half(a.v_scales[row0 + base + tid])) : 0.0f;
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- S = K Q^T
    if (tid == 0 && !err) {
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < kAtD / 16; ++k) {
        const int blk = k >> 2, off = (k & 3) * 32;
        umma_f16(tS, sw128_desc(kb + blk * 16384 + off), sw128_desc(qb + blk * 2048 + off), kIdescQK, k > 0 ? 1u : 0u);
      }
      umma_commit(&barS);
    }
    float s[G];
    if (smx) {
      if (!mbar_wait(&barS, ph)) err = 1;
      tc_fence_after();
      float x[16];
      tmem_ld16(tS + lane_off, x);
      // ---- online softmax over the tile (base-2 logits), thread tid = token tid
#pragma unroll
      for (int g = 0; g < G; ++g) {
        s[g] = vs ? x[g] * qscale : -INFINITY;
        float v = s[g];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[g][warp] = v;
      }
    }
    __syncthreads();
    float alpha[G];
    if (smx) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float tm = fmaxf(fmaxf(red[g][0], red[g][1]), fmaxf(red[g][2], red[g][3]));
        const float mn = fmaxf(m[g], tm);
        alpha[g] = m[g] == -INFINITY ? 0.0f : ex2a(m[g] - mn);
        m[g] = mn;
        const float p = vs ? ex2a(s[g] - mn) : 0.0f;
        lsum[g] = fmaf(lsum[g], alpha[g], p);
        *reinterpret_cast<__half*>(wb + sw128_off(g, tid, 2048)) = __float2half_rn(vs ? p * sv : 0.0f);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- O = C^T W^T (value codes, M = dimensions)
    if (tid == 0 && !err) {
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < kAtTok / 16; ++k) {
        const int blk = k >> 2, off = (k & 3) * 32;
        umma_f16(tO, sw128_mn_desc(vb + k * 2048, 16384, 1024), sw128_desc(wb + blk * 2048 + off), kIdescPV,
                 k > 0 ? 1u : 0u);
      }
      umma_commit(&barO);
    }
    if (smx) {
      if (!mbar_wait(&barO, ph)) err = 1;
      tc_fence_after();
      float o[16];
      tmem_ld16(tO + lane_off, o);
#pragma unroll
      for (int g = 0; g < G; ++g) acc[g] = fmaf(acc[g], alpha[g], o[g]);
    }
    tc_fence_before();
    __syncthreads();  // the tiles and TMEM columns are free for the next tile
    if (err) break;
  }
  // ---- per query head: running max, softmax sum (fixed-order reduction), accumulator
  const int64_t o = ((int64_t)b * a.q_heads + kh * G) * a.splits + split;
  if (smx) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float v = lsum[g];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) red[g][warp] = v;
    }
  }
  __syncthreads();
  if (smx) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int64_t og = o + (int64_t)g * a.splits;
      if (tid == 0) {
        a.ws_m[og] = m[g];
        a.ws_l[og] = (red[g][0] + red[g][1]) + (red[g][2] + red[g][3]);
      }
      a.ws_acc[og * kAtD + tid] = acc[g];
    }
  }
  if (tid == 0 && err) {
    // a tile whose MMA was not waited for must finish before TMEM is freed
    mbar_wait(&barS, ph, 1u << 20);
    mbar_wait(&barO, ph, 1u << 20);
    atomicOr(&g_attend_wait_error, 1u);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_base, 32);
}

// Merge of the splits: split weights f_s = 2^(m_s - M) computed once per split in parallel,
// then every dimension sums its accumulators in split order with independent loads.
constexpr int kAtMaxSplits = 1024;

__global__ void __launch_bounds__(kAtD) attend_combine(const AttendArgs a) {
  __shared__ float y[kAtD];
  __shared__ float f[kAtMaxSplits];
  __shared__ float red[kAtD / 32];
  const int qh = blockIdx.x, b = blockIdx.y, j = threadIdx.x, lane = j & 31, warp = j >> 5;
  const int S = a.splits;
  const int64_t o = ((int64_t)b * a.q_heads + qh) * S;
  float M = -INFINITY;
  for (int s = j; s < S; s += kAtD) M = fmaxf(M, a.ws_m[o + s]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  if (lane == 0) red[warp] = M;
  __syncthreads();
  M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  __syncthreads();
  float L = 0.0f;
  for (int s = j; s < S; s += kAtD) {
    const float ms = a.ws_m[o + s];
    const float fs = (ms == -INFINITY || M == -INFINITY) ? 0.0f : ex2a(ms - M);
    f[s] = fs;
    L = fmaf(a.ws_l[o + s], fs, L);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  if (lane == 0) red[warp] = L;
  __syncthreads();
  L = (red[0] + red[1]) + (red[2] + red[3]);
  const float* accp = a.ws_acc + o * kAtD + j;
  float v0 = 0.0f, v1 = 0.0f, v2 = 0.0f, v3 = 0.0f;
  int s = 0;
  for (; s + 4 <= S; s += 4) {
    const float x0 = accp[(int64_t)s * kAtD], x1 = accp[(int64_t)(s + 1) * kAtD];
    const float x2 = accp[(int64_t)(s + 2) * kAtD], x3 = accp[(int64_t)(s + 3) * kAtD];
    v0 = fmaf(x0, f[s], v0);
    v1 = fmaf(x1, f[s + 1], v1);
    v2 = fmaf(x2, f[s + 2], v2);
    v3 = fmaf(x3, f[s + 3], v3);
  }
  for (; s < S; ++s) v0 = fmaf(accp[(int64_t)s * kAtD], f[s], v0);
  const float v = (v0 + v1) + (v2 + v3);
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

cudaError_t attend_take_error(unsigned int* bits, cudaStream_t s) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_attend_wait_error, sizeof(v), 0, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && v) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_attend_wait_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  *bits = v;
  return e;
}

size_t attend_workspace_bytes(int batch, int q_heads, int splits) {
  const size_t n = (size_t)batch * q_heads * splits;
  return n * sizeof(float) * (2 + kAtD) + 3 * 256;
}

int attend_splits(int batch, int heads, int n_tokens) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tiles = (n_tokens + kAtTok - 1) / kAtTok;
  // one wave of attend_partial at 2 resident CTAs per SM
  const long long want = (2LL * sms + (long long)batch * heads - 1) / ((long long)batch * heads);
  return (int)std::max(1LL, std::min<long long>(std::min<long long>(tiles, want), kAtMaxSplits));
}

template <int FMTK, int FMTV>
static cudaError_t attend_g(const AttendArgs& a, int G, cudaStream_t s) {
  const dim3 grid(a.splits, a.heads, a.batch);
  cudaError_t e = cudaSuccess;
  auto run = [&](auto kern) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, AtSmem::kBytes);
    if (e == cudaSuccess) kern<<<grid, kAtThreads, AtSmem::kBytes, s>>>(a);
  };
  switch (G) {
    case 1: run(attend_partial<FMTK, FMTV, 1>); break;
    case 2: run(attend_partial<FMTK, FMTV, 2>); break;
    case 4: run(attend_partial<FMTK, FMTV, 4>); break;
    case 8: run(attend_partial<FMTK, FMTV, 8>); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
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
