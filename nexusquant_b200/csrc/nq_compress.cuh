// Fused KV compress kernel (sm_100a).
//
// Per vector (one (layer, K|V, batch, head, kept token) row of d values):
//   TMA bulk copy row -> shared -> fp32 -> [keys] inverse split-half RoPE at the
//   source position -> zero pad to d_p -> Walsh-Hadamard butterfly in registers
//   -> * fl32(1/sqrt(d_p)) -> amax, sc = amax / (L/2) -> x / sc (correctly
//   rounded) -> relaxed-E8 nearest point per 8-group -> clamp -> packed codes,
//   fp16 scale [-> fake-quant reconstruction].
// Reference: nexusquant/pipeline.py:1218-1236, nexusquant/core/e8_lattice.py:27-124,
// nexusquant/core/rope_utils.py:75-122, nexusquant/integrations/vllm_backend.py:267-316.
//
// Design:
//  * One thread owns one vector.  Coordinates are held as pairs
//    P[j] = {x[j], x[j + d_p/2]} in 64-bit registers so the RoPE products, the
//    first log2(d_p)-1 butterfly stages, the scale, the division and half of
//    the lattice arithmetic run as sm_100 packed f32x2 instructions (two
//    IEEE-rounded fp32 results per instruction, bit-identical to scalar code).
//    Group g (low lanes) and group g + d_p/16 (high lanes) go through the
//    lattice step together.
//  * K vs V and the packing format are template parameters, so the per-vector
//    code is one branch-free basic block.
//  * Persistent CTAs (2 per SM) walk the tile list; each has a two-stage
//    shared-memory pipeline: while tile i is computed, the rows of tile i+1 are
//    in flight through the TMA engine (cp.async.bulk, no multicast).
//  * A tile is HG heads x (128/HG) tokens of one (layer, K|V, batch); threads of
//    a warp that share a token read the same RoPE row (shared-memory broadcast).
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

typedef unsigned long long u64;

__device__ __forceinline__ u64 pk(float a, float b) {
  u64 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk(u64 p, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(p));
}
__device__ __forceinline__ u64 add2(u64 a, u64 b) {
  u64 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 sub2(u64 a, u64 b) {
  u64 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 mul2(u64 a, u64 b) {
  u64 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
  u64 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Packing formats: 0 = nibbles (L <= 4), 1 = 5-bit fields (L = 8), 2 = int8 (L = 16).
__host__ __device__ constexpr int fmt_of(int levels) { return levels <= 4 ? 0 : (levels == 8 ? 1 : 2); }
template <int FMT, int DP>
struct Fmt {
  static constexpr int kBytes = FMT == 0 ? DP / 2 : (FMT == 1 ? DP * 5 / 8 : DP);
  static constexpr int kWords = kBytes / 4;
};

// Relaxed-E8 choice for one 8-group (nexusquant/core/e8_lattice.py:27-69), from
// the per-coordinate gaps e = x - round(x) and the bit patterns of x + M and
// fl(x - 0.5) + M (M = 1.5 * 2^23, whose low bits hold the rounded integers).
// Emits fields f = code + 8 with code = 2 * lattice point clamped to [-L, L].
// B is chosen iff sum_i |e_i| + odd * (1 - 2 min_i |e_i|) > 2 (fp32, pairwise sum):
// the same arithmetic as the CPU oracle.
__device__ __forceinline__ void e8_fields(const float (&e)[8], const uint32_t (&sb)[8], const uint32_t (&bb)[8],
                                          int levels, int (&f)[8]) {
  // pairwise sum ((g0+g1)+(g2+g3))+((g4+g5)+(g6+g7)): depth 3 instead of 7
  float g[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) g[i] = fabsf(e[i]);
  const float gsum = __fadd_rn(__fadd_rn(__fadd_rn(g[0], g[1]), __fadd_rn(g[2], g[3])),
                               __fadd_rn(__fadd_rn(g[4], g[5]), __fadd_rn(g[6], g[7])));
  // tournament argmin keeping the left entry on ties = first index of the minimum
  float tg[4], te[4];
  int ti[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const bool r = g[2 * k + 1] < g[2 * k];
    tg[k] = r ? g[2 * k + 1] : g[2 * k];
    te[k] = r ? e[2 * k + 1] : e[2 * k];
    ti[k] = r ? 2 * k + 1 : 2 * k;
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const bool r = tg[2 * k + 1] < tg[2 * k];
    tg[k] = r ? tg[2 * k + 1] : tg[2 * k];
    te[k] = r ? te[2 * k + 1] : te[2 * k];
    ti[k] = r ? ti[2 * k + 1] : ti[2 * k];
  }
  const bool r = tg[1] < tg[0];
  const float gmin = r ? tg[1] : tg[0];
  const float emin = r ? te[1] : te[0];
  const int idx = r ? ti[1] : ti[0];
  const uint32_t par = (sb[0] ^ sb[1] ^ sb[2] ^ sb[3] ^ sb[4] ^ sb[5] ^ sb[6] ^ sb[7]) & 1u;
  const float lhs = par ? __fadd_rn(gsum, __fsub_rn(1.0f, __fmul_rn(2.0f, gmin))) : gsum;
  const bool use_b = lhs > 2.0f;
  // field = 2 * round + 8 (A) or 2 * round(x - 0.5) + 9 (B); the magic offset cancels mod 2^32
  const uint32_t off = (use_b ? 9u : 8u) - 2u * kMagicBits;
  const int fix = (par && !use_b) ? (emin >= 0.0f ? 2 : -2) : 0;
  const int lo = 8 - levels, hi = 8 + levels;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t base = use_b ? bb[i] : sb[i];
    int v = static_cast<int>(2u * base + off);
    v += (i == idx) ? fix : 0;
    f[i] = min(max(v, lo), hi);
  }
}

template <int FMT, int DP>
__device__ __forceinline__ void pack_fields(uint32_t* w, int g, const int (&f)[8]) {
  if constexpr (FMT == 0) {
    uint32_t v = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) v |= static_cast<uint32_t>(f[i]) << (4 * i);
    w[g] = v;
  } else if constexpr (FMT == 1) {
    uint64_t v = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) v |= static_cast<uint64_t>(f[i]) << (5 * i);
    const int bit = 40 * g;
    const int wi = bit >> 5, sh = bit & 31;  // sh is 0, 8, 16 or 24
    w[wi] |= static_cast<uint32_t>(v << sh);
    w[wi + 1] |= static_cast<uint32_t>(v >> (32 - sh));
  } else {
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lo |= (static_cast<uint32_t>(f[i] - 8) & 0xFFu) << (8 * i);
      hi |= (static_cast<uint32_t>(f[4 + i] - 8) & 0xFFu) << (8 * i);
    }
    w[2 * g] = lo;
    w[2 * g + 1] = hi;
  }
}

template <int BYTES>
__device__ __forceinline__ void store_words(uint8_t* dst, const uint32_t* w) {
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

// Fake-quant reconstruction from the fields (codes + 8), written as fp16.
template <int D, int DP>
__device__ __forceinline__ void recon_store(float (&x)[DP], float sc, bool key, const float* cosr,
                                            const float* sinr, float sharpen, bool rotate, __half* out) {
  if (rotate) {
#pragma unroll
    for (int h = 1; h < DP; h <<= 1) {
#pragma unroll
      for (int i = 0; i < DP; ++i) {
        if ((i & h) == 0) {
          const float a = x[i], b = x[i + h];
          x[i] = __fadd_rn(a, b);
          x[i + h] = __fsub_rn(a, b);
        }
      }
    }
  }
  const float coef = __fmul_rn(sc, rotate ? 0.5f * hadamard_entry(DP) : 0.5f);
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
// Tile geometry shared by the load and compute phases.
// --------------------------------------------------------------------------
struct Tile {
  int layer, kv, b, hg, tt;
};

__device__ __forceinline__ Tile decode_tile(const CompressArgs& a, int n_layers, long long t) {
  const int TOK = kCompressThreads / a.head_group;
  const int t_tiles = (a.n_kept + TOK - 1) / TOK;
  const int h_groups = (a.heads + a.head_group - 1) / a.head_group;
  Tile r;
  r.tt = (int)(t % t_tiles); t /= t_tiles;
  r.hg = (int)(t % h_groups); t /= h_groups;
  r.b = (int)(t % a.batch); t /= a.batch;
  r.layer = (int)(t % n_layers); t /= n_layers;
  r.kv = (int)t;  // K tiles first, then V tiles
  return r;
}

template <typename TIn, int D>
struct Smem {
  static constexpr int kRowBytes = D * InTraits<TIn>::kBytes;
  static constexpr int kRowStride = kRowBytes + 16;  // padded: conflict-free 16-byte reads
  static constexpr int kTabStride = 2 * (D / 2) * 4 + 16;
  static constexpr int kRows = kCompressThreads * kRowStride;
  // rows + one RoPE row per token of the tile, rounded to 128 bytes
  __host__ __device__ static constexpr int stage(int head_group) {
    return (kRows + (kCompressThreads / head_group) * kTabStride + 127) & ~127;
  }
};

// Issue the TMA copies of one tile into a stage (all threads; thread 0 posts the byte count first).
template <typename TIn, int D>
__device__ __forceinline__ void issue_tile(const CompressArgs& a, int n_layers, long long tile, uint8_t* stage,
                                           uint64_t* bar) {
  using S = Smem<TIn, D>;
  const Tile t = decode_tile(a, n_layers, tile);
  const LayerIO& L = a.layers[t.layer];
  const bool key = t.kv == 0;
  const TIn* src = static_cast<const TIn*>(key ? L.k : L.v);
  const int HG = a.head_group, TOK = kCompressThreads / HG;
  const int count = a.kept_count ? min(a.kept_count[t.b], a.n_kept) : a.n_kept;
  const int tid = threadIdx.x;
  const int tok_l = tid / HG, head_l = tid % HG;
  const int j = t.tt * TOK + tok_l;
  const int head = t.hg * HG + head_l;
  const bool valid = src != nullptr && j < count && head < a.heads;
  if (valid) {
    const int row = a.kept_idx ? a.kept_idx[(int64_t)t.b * a.n_kept + j] : j;
    const TIn* g = src + (int64_t)t.b * a.in_stride_b + (int64_t)head * a.in_stride_h + (int64_t)row * a.in_stride_t;
    bulk_g2s(stage + tid * S::kRowStride, g, S::kRowBytes, bar);
    if (key && head_l == 0) {
      const int pos = a.positions ? a.positions[(int64_t)t.b * a.n_kept + j] : row;
      uint8_t* trow = stage + S::kRows + tok_l * S::kTabStride;
      bulk_g2s(trow, a.rope_cos + (int64_t)pos * (D / 2), (D / 2) * 4, bar);
      bulk_g2s(trow + (D / 2) * 4, a.rope_sin + (int64_t)pos * (D / 2), (D / 2) * 4, bar);
    }
  }
}

template <typename TIn, int D>
__device__ __forceinline__ uint32_t tile_bytes(const CompressArgs& a, int n_layers, long long tile) {
  const Tile t = decode_tile(a, n_layers, tile);
  const LayerIO& L = a.layers[t.layer];
  const bool key = t.kv == 0;
  if ((key ? L.k : L.v) == nullptr) return 0;
  const int HG = a.head_group, TOK = kCompressThreads / HG;
  const int count = a.kept_count ? min(a.kept_count[t.b], a.n_kept) : a.n_kept;
  const int toks = max(0, min(TOK, count - t.tt * TOK));
  const int heads = min(HG, a.heads - t.hg * HG);
  uint32_t bytes = (uint32_t)(toks * heads) * Smem<TIn, D>::kRowBytes;
  if (key) bytes += (uint32_t)toks * (D / 2) * 8;
  return bytes;
}

// --------------------------------------------------------------------------
// Per-vector body for one tile (K or V, one packing format).
// --------------------------------------------------------------------------
template <typename TIn, int D, int DP, bool KEY, int FMT, bool RECON>
__device__ __forceinline__ void compress_tile(const CompressArgs& a, int n_layers, long long tile,
                                              const uint8_t* stage) {
  using S = Smem<TIn, D>;
  constexpr int H2 = DP / 2;  // pairs
  const Tile t = decode_tile(a, n_layers, tile);
  const LayerIO& L = a.layers[t.layer];
  const int levels = KEY ? L.key_levels : L.value_levels;
  const int HG = a.head_group, TOK = kCompressThreads / HG;
  const int count = a.kept_count ? min(a.kept_count[t.b], a.n_kept) : a.n_kept;
  const int tid = threadIdx.x;
  const int tok_l = tid / HG, head_l = tid % HG;
  const int j = t.tt * TOK + tok_l;
  const int head = t.hg * HG + head_l;
  if (j >= count || head >= a.heads || (KEY ? L.k : L.v) == nullptr) return;

  // ---- load, widen, inverse RoPE -> pairs P[q] = {x[q], x[q + DP/2]}
  u64 P[H2];
  const TIn* r = reinterpret_cast<const TIn*>(stage + tid * S::kRowStride);
  const float* cs = reinterpret_cast<const float*>(stage + S::kRows + tok_l * S::kTabStride);
  const float* sn = cs + D / 2;
  if constexpr (D == DP) {
#pragma unroll
    for (int k = 0; k < H2 / 8; ++k) {
      float lo[8], hi[8];
      load8(r + 8 * k, lo);
      load8(r + H2 + 8 * k, hi);
#pragma unroll
      for (int i = 0; i < 8; ++i) P[8 * k + i] = pk(lo[i], hi[i]);
    }
    if constexpr (KEY) {
      // pair (q, q + D/2) is P[q]: y1 = x1 c + x2 s, y2 = x2 c - x1 s
#pragma unroll
      for (int q = 0; q < H2; q += 4) {
        const float4 c4 = *reinterpret_cast<const float4*>(cs + q);
        const float4 s4 = *reinterpret_cast<const float4*>(sn + q);
        const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
        const float ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float m1, m2, n1, n2;
          upk(mul2(P[q + u], pk(cc[u], cc[u])), m1, m2);  // x1 c, x2 c
          upk(mul2(P[q + u], pk(ss[u], ss[u])), n1, n2);  // x1 s, x2 s
          P[q + u] = pk(__fadd_rn(m1, n2), __fsub_rn(m2, n1));
        }
      }
    }
  } else {
    // D < DP (96 -> 128): RoPE pairs (i, i + D/2) do not line up with the register pairs
    float x[D];
#pragma unroll
    for (int k = 0; k < D / 8; ++k) load8(r + 8 * k, &x[8 * k]);
    if constexpr (KEY) {
#pragma unroll
      for (int i = 0; i < D / 2; ++i) {
        const float c = cs[i], s = sn[i];
        const float x1 = x[i], x2 = x[i + D / 2];
        x[i] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        x[i + D / 2] = __fsub_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
      }
    }
#pragma unroll
    for (int q = 0; q < H2; ++q) P[q] = pk(x[q], q + H2 < D ? x[q + H2] : 0.0f);
  }

  // ---- rotate (stages 1 .. DP/4 on pairs, stage DP/2 inside each pair), scale
  float amax = 0.0f;
  if (a.rotate) {
#pragma unroll
    for (int h = 1; h < H2; h <<= 1) {
#pragma unroll
      for (int q = 0; q < H2; ++q) {
        if ((q & h) == 0) {
          const u64 u = P[q], v = P[q + h];
          P[q] = add2(u, v);
          P[q + h] = sub2(u, v);
        }
      }
    }
    const u64 hh = pk(hadamard_entry(DP), hadamard_entry(DP));
#pragma unroll
    for (int q = 0; q < H2; ++q) {
      float u, v;
      upk(P[q], u, v);
      P[q] = mul2(pk(__fadd_rn(u, v), __fsub_rn(u, v)), hh);
      float y0, y1;
      upk(P[q], y0, y1);
      amax = max3(amax, fabsf(y0), fabsf(y1));
    }
  } else {
#pragma unroll
    for (int q = 0; q < H2; ++q) {
      float y0, y1;
      upk(P[q], y0, y1);
      amax = max3(amax, fabsf(y0), fabsf(y1));
    }
  }
  amax = fmaxf(amax, 1e-8f);
  const float sc = __fmul_rn(amax, 2.0f / static_cast<float>(levels));
  const float rcp = __frcp_rn(sc);
  const u64 r2 = pk(rcp, rcp), nsc2 = pk(-sc, -sc);
  const u64 M2 = pk(kMagic, kMagic), half2 = pk(0.5f, 0.5f);

  // ---- lattice: groups g (low lanes) and g + DP/16 (high lanes) together
  constexpr int G = DP / 8;
  uint32_t w[Fmt<FMT, DP>::kWords];
#pragma unroll
  for (int i = 0; i < Fmt<FMT, DP>::kWords; ++i) w[i] = 0u;
  float xr[RECON ? DP : 1];
#pragma unroll
  for (int g = 0; g < G / 2; ++g) {
    float elo[8], ehi[8];
    uint32_t slo[8], shi[8], blo[8], bhi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const u64 y = P[8 * g + i];
      // correctly rounded y / sc (Markstein): q = y r; rem = y - q sc; q + rem r
      const u64 q0 = mul2(y, r2);
      const u64 rem = fma2(q0, nsc2, y);
      const u64 n = fma2(rem, r2, q0);
      const u64 s = add2(n, M2);
      const u64 e = sub2(n, sub2(s, M2));
      const u64 sb = add2(sub2(n, half2), M2);
      float s0, s1, b0, b1;
      upk(e, elo[i], ehi[i]);
      upk(s, s0, s1);
      upk(sb, b0, b1);
      slo[i] = __float_as_uint(s0); shi[i] = __float_as_uint(s1);
      blo[i] = __float_as_uint(b0); bhi[i] = __float_as_uint(b1);
    }
    int flo[8], fhi[8];
    e8_fields(elo, slo, blo, levels, flo);
    e8_fields(ehi, shi, bhi, levels, fhi);
    pack_fields<FMT, DP>(w, g, flo);
    pack_fields<FMT, DP>(w, g + G / 2, fhi);
    if constexpr (RECON) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        xr[8 * g + i] = static_cast<float>(flo[i] - 8);
        xr[8 * (g + G / 2) + i] = static_cast<float>(fhi[i] - 8);
      }
    }
  }

  // ---- outputs
  const int64_t vrow = ((int64_t)t.b * a.heads + head) * a.n_kept + j;
  uint8_t* codes = KEY ? L.k_codes : L.v_codes;
  constexpr int PB = Fmt<FMT, DP>::kBytes;
  if (codes) store_words<PB>(codes + vrow * PB, w);
  uint16_t* sc16 = KEY ? L.k_scales : L.v_scales;
  if (sc16) sc16[vrow] = __half_as_ushort(__float2half_rn(sc));
  float* sc32 = KEY ? L.k_scales_f32 : L.v_scales_f32;
  if (sc32) sc32[vrow] = sc;
  if constexpr (RECON) {
    uint16_t* out = KEY ? L.k_out : L.v_out;
    if (out) {
      const int src_row = a.kept_idx ? a.kept_idx[(int64_t)t.b * a.n_kept + j] : j;
      const int pos = a.positions ? a.positions[(int64_t)t.b * a.n_kept + j] : src_row;
      const int orow = a.out_row_mode == 1 ? j : src_row;
      int opos = pos;
      if (a.out_positions) opos = a.out_positions[(int64_t)t.b * a.n_kept + j];
      else if (a.out_row_mode == 1) opos = j;
      __half* o = reinterpret_cast<__half*>(out) + (int64_t)t.b * a.out_stride_b + (int64_t)head * a.out_stride_h +
                  (int64_t)orow * a.out_stride_t;
      recon_store<D, DP>(xr, sc, KEY, a.rope_cos + (int64_t)opos * (D / 2), a.rope_sin + (int64_t)opos * (D / 2),
                         a.key_sharpen, a.rotate != 0, o);
    }
  }
}

// --------------------------------------------------------------------------
// Persistent kernel: two-stage TMA pipeline over the tile list.
// --------------------------------------------------------------------------
template <typename TIn, int D, int DP, int FMTK, int FMTV, bool RECON>
__global__ void __launch_bounds__(kCompressThreads, 2) compress_kernel(const CompressArgs args, int n_layers,
                                                                        long long n_tiles, int ns) {
  using S = Smem<TIn, D>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar[2];
  const long long first = blockIdx.x;
  if (first >= n_tiles) return;
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&bar[0], tile_bytes<TIn, D>(args, n_layers, first));
  }
  __syncthreads();
  issue_tile<TIn, D>(args, n_layers, first, smem, &bar[0]);
  int it = 0;
  // ns = 2: tile i+1 is loaded into the other stage while tile i is computed;
  // ns = 1 (rows too large for two stages): load and compute alternate.
  for (long long tile = first; tile < n_tiles; tile += gridDim.x, ++it) {
    const int s = ns == 2 ? (it & 1) : 0;
    const uint32_t ph = ns == 2 ? ((it >> 1) & 1) : (it & 1);
    const long long next = tile + gridDim.x;
    // everyone has finished the tile that used stage s^1 (previous iteration) here
    __syncthreads();
    if (ns == 2 && next < n_tiles) {
      if (threadIdx.x == 0) mbar_arrive_expect_tx(&bar[s ^ 1], tile_bytes<TIn, D>(args, n_layers, next));
      __syncthreads();
      issue_tile<TIn, D>(args, n_layers, next, smem + (s ^ 1) * S::stage(args.head_group), &bar[s ^ 1]);
    }
    if (!mbar_wait(&bar[s], ph)) {
      if (args.error_flag) atomicExch(args.error_flag, 1);
      if (ns == 2 && next < n_tiles) mbar_wait(&bar[s ^ 1], ((it + 1) >> 1) & 1);  // let in-flight copies land
      return;
    }
    const uint8_t* stage = smem + s * S::stage(args.head_group);
    const Tile t = decode_tile(args, n_layers, tile);
    if (t.kv == 0) compress_tile<TIn, D, DP, true, FMTK, RECON>(args, n_layers, tile, stage);
    else compress_tile<TIn, D, DP, false, FMTV, RECON>(args, n_layers, tile, stage);
    if (ns == 1 && next < n_tiles) {
      __syncthreads();
      if (threadIdx.x == 0) mbar_arrive_expect_tx(&bar[0], tile_bytes<TIn, D>(args, n_layers, next));
      __syncthreads();
      issue_tile<TIn, D>(args, n_layers, next, smem, &bar[0]);
    }
  }
}

// --------------------------------------------------------------------------
// Launch
// --------------------------------------------------------------------------
template <typename TIn, int D, int DP, int FMTK, int FMTV>
static cudaError_t launch_fmt(const CompressArgs& a, int n_layers, long long n_tiles, cudaStream_t s, bool recon) {
  using S = Smem<TIn, D>;
  int dev = 0, sms = 0, per_sm = 0, max_smem = 0;
  cudaError_t e;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return e;
  const int ns = 2 * (size_t)S::stage(a.head_group) + 64 <= (size_t)max_smem ? 2 : 1;
  const size_t smem = ns * (size_t)S::stage(a.head_group);
  auto kern = recon ? compress_kernel<TIn, D, DP, FMTK, FMTV, true> : compress_kernel<TIn, D, DP, FMTK, FMTV, false>;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kCompressThreads, smem)) != cudaSuccess)
    return e;
  long long grid = (long long)sms * (per_sm > 0 ? per_sm : 1);
  if (grid > n_tiles) grid = n_tiles;
  kern<<<(unsigned)grid, kCompressThreads, smem, s>>>(a, n_layers, n_tiles, ns);
  return cudaGetLastError();
}

template <typename TIn, int D, int DP>
static cudaError_t launch_dims(const CompressArgs& a, int n_layers, long long n_tiles, int fk, int fv,
                               cudaStream_t s, bool recon) {
#define NQ_FMT_CASE(K_, V_) \
  if (fk == K_ && fv == V_) return launch_fmt<TIn, D, DP, K_, V_>(a, n_layers, n_tiles, s, recon);
  NQ_FMT_CASE(0, 0) NQ_FMT_CASE(1, 0) NQ_FMT_CASE(1, 1) NQ_FMT_CASE(0, 1) NQ_FMT_CASE(2, 0) NQ_FMT_CASE(2, 1)
  NQ_FMT_CASE(2, 2) NQ_FMT_CASE(0, 2) NQ_FMT_CASE(1, 2)
#undef NQ_FMT_CASE
  return cudaErrorInvalidValue;
}

// Instantiated once per input dtype in nq_compress_{f16,bf16,f32}.cu (parallel builds).
template <typename TIn>
cudaError_t launch_compress_t(const CompressArgs& a, int n_layers, long long n_tiles, int fk, int fv, cudaStream_t s,
                              bool recon) {
  if (a.head_dim == 128 && a.head_dim_padded == 128) return launch_dims<TIn, 128, 128>(a, n_layers, n_tiles, fk, fv, s, recon);
  if (a.head_dim == 96 && a.head_dim_padded == 128) return launch_dims<TIn, 96, 128>(a, n_layers, n_tiles, fk, fv, s, recon);
  if (a.head_dim == 64 && a.head_dim_padded == 64) return launch_dims<TIn, 64, 64>(a, n_layers, n_tiles, fk, fv, s, recon);
  return cudaErrorInvalidValue;
}

}  // namespace nq
