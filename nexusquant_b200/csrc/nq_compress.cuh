// Fused KV compress kernel (sm_100a).
//
// Per vector (one (layer, K|V, batch, head, kept token) row of d values):
//   cp.async row -> shared -> fp32 -> [keys] inverse split-half RoPE at the
//   source position -> zero pad to d_p -> Walsh-Hadamard butterfly in registers
//   -> * fl32(1/sqrt(d_p)) -> amax, sc = amax / (L/2) -> x / sc (correctly
//   rounded) -> relaxed-E8 nearest point per 8-group -> clamp -> packed codes,
//   fp16 scale [-> fake-quant reconstruction].
// Reference: nexusquant/pipeline.py:1218-1236, nexusquant/core/e8_lattice.py:27-124,
// nexusquant/core/rope_utils.py:75-122, nexusquant/integrations/vllm_backend.py:267-316.
//
// Design:
//  * Two threads own one vector.  Coordinates are held as pairs
//    P[j] = {x[j], x[j + d_p/2]} in 64-bit registers so the RoPE products, the
//    butterfly stages, the scale, the division and half of the lattice
//    arithmetic run as sm_100 packed f32x2 instructions (two IEEE-rounded fp32
//    results per instruction, bit-identical to scalar code).  Each thread holds
//    half of the pairs; one butterfly stage crosses the thread pair (shuffle).
//    Group g (low lanes) and group g + d_p/16 (high lanes) go through the
//    lattice step together.
//  * K vs V and the packing format are template parameters, so the per-vector
//    code is one branch-free basic block.
//  * Persistent CTAs walk the tile list; each has a two-stage shared-memory
//    pipeline: while tile i is computed, the rows of tile i+1 are in flight as
//    16-byte cp.async copies (per-lane operands: no per-row issue loop, and a
//    warp barrier suffices because each warp copies the rows it computes).
//  * A tile is HG heads x (64/HG) tokens of one (layer, K|V, batch); threads of
//    a warp that share a token read the same RoPE row (shared-memory broadcast).
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

// Packing formats: 0 = nibbles (L <= 4), 1 = 5-bit fields (L = 8), 2 = int8 (L = 16).
__host__ __device__ constexpr int fmt_of(int levels) { return levels <= 4 ? 0 : (levels == 8 ? 1 : 2); }
template <int FMT, int DP>
struct Fmt {
  static constexpr int kBytes = FMT == 0 ? DP / 2 : (FMT == 1 ? DP * 5 / 8 : DP);
  static constexpr int kWords = kBytes / 4;
};

// Packed-field layout of one 8-group.  Field i sits at bit sh(i) of word wd(i); an
// A field is f = 2a + BIAS and a B field f = 2k + 1 + BIAS, with a = rint(x) and
// k = rint(x - 1/2), so code = 2 * lattice point = f - BIAS.  Formats 0 and 1 keep
// f (nibbles / 5-bit fields, BIAS 8); format 2 turns f into the signed code byte.
template <int FMT>
struct GF {
  static constexpr int kWords = FMT == 0 ? 1 : 2;
  static constexpr int kBias = FMT == 2 ? 32 : 8;
  static constexpr int kWidth = FMT == 0 ? 4 : (FMT == 1 ? 5 : 8);
  static constexpr int kPer = FMT == 0 ? 8 : 4;  // fields per word
  static constexpr uint32_t kMask = (1u << kWidth) - 1u;
  __host__ __device__ static constexpr int sh(int i) { return kWidth * (i % kPer); }
  __host__ __device__ static constexpr int wd(int i) { return i / kPer; }
  // c replicated into every field of a word (mod 2^32)
  __host__ __device__ static constexpr uint32_t rep(uint32_t c) {
    uint32_t r = 0;
    for (int i = 0; i < kPer; ++i) r += c << (kWidth * i);
    return r;
  }
  static constexpr uint32_t kBit0 = rep(1u), kBit1 = rep(2u);
  // Accumulator seeds: sum_i bits(x_i + M) * 2^(sh(i)+1) + seed = sum_i field_i << sh(i),
  // because bits(x + M) = kMagicBits + round(x) and the magic part cancels mod 2^32.
  static constexpr uint32_t kSeedA = rep((uint32_t)kBias) - rep(2u * kMagicBits);
  static constexpr uint32_t kSeedB = rep((uint32_t)kBias + 1u) - rep(2u * kMagicBits);
};

__device__ __forceinline__ uint32_t umin(uint32_t a, uint32_t b) { return a < b ? a : b; }

// Relaxed-E8 nearest point of one 8-group (nexusquant/core/e8_lattice.py:27-69), packed.
//
// Inputs per coordinate: e = x - round(x), sa = bits(x + M), sb = bits(fl(x - 1/2) + M)
// (M = 1.5 * 2^23).  Decision, as in the CPU oracle: B iff
//   sum_i |e_i| (pairwise) + odd * (1 - 2 min_i |e_i|) > 2,
// and for A with an odd coordinate sum the first coordinate of smallest |e| moves one step
// toward x.  Everything after the gaps runs on the packed words:
//  * the A and B fields of the whole group are accumulated with one IMAD per coordinate;
//  * parity = popcount of the A fields' bit 1;
//  * argmin: unsigned minima of (bits(|e_i|) << 2 | i mod 4) per half (first index on
//    ties), then the halves compared on |e|;
//  * the step's direction is fB - fA at that coordinate (+1 when e = 0);
//  * clamping to [-L, L]: with L a power of two, sc = amax * 2/L is exact and |x| <= L/2,
//    so a field leaves the range only as B at x = +L/2 (L >= 4, f = L + 9 + BIAS - 8),
//    B at x = -L/2 (L = 2, f = 5), or the A step at a = +L/2 -- each is patched directly.
template <int FMT, int LEV>
__device__ __forceinline__ void e8_group(const float (&e)[8], const uint32_t (&sa)[8], const uint32_t (&sb)[8],
                                         uint32_t (&w)[GF<FMT>::kWords]) {
  using F = GF<FMT>;
  constexpr int NW = F::kWords;
  const float gsum = __fadd_rn(__fadd_rn(__fadd_rn(fabsf(e[0]), fabsf(e[1])), __fadd_rn(fabsf(e[2]), fabsf(e[3]))),
                               __fadd_rn(__fadd_rn(fabsf(e[4]), fabsf(e[5])), __fadd_rn(fabsf(e[6]), fabsf(e[7]))));
  uint32_t key[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) key[i] = (__float_as_uint(e[i]) << 2) | (uint32_t)(i & 3);  // |e| <= 1/2: bit 30 is 0
  const uint32_t kl = umin(umin(key[0], key[1]), umin(key[2], key[3]));
  const uint32_t kh = umin(umin(key[4], key[5]), umin(key[6], key[7]));
  const bool in_hi = (kh >> 2) < (kl >> 2);
  const uint32_t km = in_hi ? kh : kl;
  const uint32_t gbits = km >> 2;
  const int idx = (in_hi ? 4 : 0) + (int)(km & 3u);
  // sign bits of e (bit 7 - i for coordinate i), for the direction of the A step
  uint32_t neg = 0u;
#pragma unroll
  for (int i = 0; i < 8; ++i) neg = __funnelshift_l(__float_as_uint(e[i]), neg, 1);

  uint32_t wa[NW], wb[NW];
#pragma unroll
  for (int k = 0; k < NW; ++k) { wa[k] = F::kSeedA; wb[k] = F::kSeedB; }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    wa[F::wd(i)] += sa[i] * (2u << F::sh(i));
    wb[F::wd(i)] += sb[i] * (2u << F::sh(i));
  }
  uint32_t par;
  if constexpr (NW == 1) par = __popc(wa[0] & F::kBit1) & 1u;
  else par = __popc((wa[0] ^ wa[1]) & F::kBit1) & 1u;
  const float lhs = par ? __fadd_rn(gsum, __fmaf_rn(-2.0f, __uint_as_float(gbits), 1.0f)) : gsum;
  const bool use_b = lhs > 2.0f;

  // A step at coordinate idx: one step toward x, up when e_idx >= 0 (e8_lattice.py:42-43;
  // e = -0 only for x = -0, whose gap is 0 and which steps up).  The sign is read from e
  // itself: the B field (fA + 1 for e > 0, fA - 1 for e < 0) says otherwise where fl(x - 1/2)
  // rounded onto a half-way point (x just below 0, x = -1 + 2^-24).
  const int sh = F::kWidth * (FMT == 0 ? idx : (idx & 3));
  const uint32_t wa_i = (NW == 1 || idx < 4) ? wa[0] : wa[NW - 1];
  const uint32_t fa = (wa_i >> sh) & F::kMask;
  const bool up = gbits == 0u || ((neg >> (7 - idx)) & 1u) == 0u;
  // a = +L/2 cannot step up: the reference's clamp (e8_lattice.py:120) takes it back
  const bool step = par && !use_b && !(up && fa == (uint32_t)(F::kBias + LEV));
  const uint32_t delta = step ? ((up ? 2u : 0xfffffffeu) << sh) : 0u;

  // B clamps (compile-time level count)
#pragma unroll
  for (int k = 0; k < NW; ++k) {
    const uint32_t x = wb[k];
    if constexpr (FMT == 0) {
      if constexpr (LEV == 4) wb[k] = x - (x & (x >> 2) & (x >> 3) & F::kBit0);  // 13 -> 12
      else wb[k] = x + (x & (x >> 2) & ~(x >> 1) & F::kBit0);                     // L = 2: 5 -> 6
    } else if constexpr (FMT == 1) {
      wb[k] = x - (x & (x >> 4) & F::kBit0);                                      // 17 -> 16
    } else {
      wb[k] = x - (x & (x >> 4) & (x >> 5) & F::kBit0);                           // 49 -> 48
    }
  }
#pragma unroll
  for (int k = 0; k < NW; ++k) {
    const bool mine = NW == 1 || ((idx >> 2) == k);
    uint32_t v = use_b ? wb[k] : wa[k] + (mine ? delta : 0u);
    if constexpr (FMT == 2) {
      // f = c + 32 in [16, 48] -> signed code byte: f ^ 32 is c for c >= 0 and c + 64 for
      // c < 0, which then needs 0xC0 on top
      const uint32_t y = v ^ 0x20202020u;
      v = y + (y & 0x20202020u) * 6u;
    }
    w[k] = v;
  }
}

// Place a group's packed words into the row words of its region.
template <int FMT>
__device__ __forceinline__ void place_group(uint32_t* r, int g, const uint32_t (&w)[GF<FMT>::kWords]) {
  if constexpr (FMT == 0) {
    r[g] = w[0];
  } else if constexpr (FMT == 1) {
    const uint64_t v = (uint64_t)w[0] | ((uint64_t)w[1] << 20);
    const int bit = 40 * g;
    const int wi = bit >> 5, sh = bit & 31;  // sh is 0, 8, 16 or 24
    r[wi] |= static_cast<uint32_t>(v << sh);
    r[wi + 1] |= static_cast<uint32_t>(v >> (32 - sh));
  } else {
    r[2 * g] = w[0];
    r[2 * g + 1] = w[1];
  }
}

// Code (2 * lattice point) of coordinate i from a group's packed words.
template <int FMT>
__device__ __forceinline__ int group_code(const uint32_t (&w)[GF<FMT>::kWords], int i) {
  using F = GF<FMT>;
  const uint32_t f = (w[F::wd(i)] >> F::sh(i)) & F::kMask;
  if constexpr (FMT == 2) return (int)(int8_t)f;
  else return (int)f - 8;
}


// Store BYTES bytes of words to dst using G-byte stores (G divides BYTES and dst's alignment).
template <int BYTES, int G>
__device__ __forceinline__ void store_region(uint8_t* dst, const uint32_t* w) {
  if constexpr (G == 16) {
#pragma unroll
    for (int k = 0; k < BYTES / 16; ++k)
      reinterpret_cast<uint4*>(dst)[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
  } else if constexpr (G == 8) {
#pragma unroll
    for (int k = 0; k < BYTES / 8; ++k) reinterpret_cast<uint2*>(dst)[k] = make_uint2(w[2 * k], w[2 * k + 1]);
  } else if constexpr (G == 4) {
#pragma unroll
    for (int k = 0; k < BYTES / 4; ++k) reinterpret_cast<uint32_t*>(dst)[k] = w[k];
  } else {
#pragma unroll
    for (int k = 0; k < BYTES / 2; ++k)
      reinterpret_cast<uint16_t*>(dst)[k] = static_cast<uint16_t>(w[k >> 1] >> (16 * (k & 1)));
  }
}

__host__ __device__ constexpr int largest_pow2_div(int a) { return a % 16 == 0 ? 16 : a % 8 == 0 ? 8 : a % 4 == 0 ? 4 : 2; }
__host__ __device__ constexpr int gcd_pow2(int a, int b) {
  return largest_pow2_div(a) < largest_pow2_div(b) ? largest_pow2_div(a) : largest_pow2_div(b);
}

// Fake-quant reconstruction of a full vector of codes (as floats), written as fp16.
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
// Tile geometry: a tile is HG heads x (kCompressVecs/HG) tokens of one
// (layer, K|V, batch); vector v of the tile is owned by threads 2v and 2v+1.
// --------------------------------------------------------------------------
struct Tile {
  int layer, kv, b, hg, tt;
};

// Tile-list geometry of one launch half, fixed per launch.
struct TileGeom {
  int tt_n;  // token tiles per (layer, batch, head group)
  int hg_n;  // head groups
};

__device__ __forceinline__ TileGeom tile_geom(const CompressArgs& a) {
  const int TOK = kCompressVecs >> a.hg_shift;
  return TileGeom{(a.n_kept + TOK - 1) / TOK, (a.heads + a.head_group - 1) >> a.hg_shift};
}

// Decoded once per CTA (32-bit: the host keeps the tile count below 2^31).
__device__ __forceinline__ Tile decode_tile(const CompressArgs& a, const TileGeom& g, int n_layers, int t) {
  Tile r;
  int q = t / g.tt_n;
  r.tt = t - q * g.tt_n;
  t = q; q = t / g.hg_n;
  r.hg = t - q * g.hg_n;
  t = q; q = t / a.batch;
  r.b = t - q * a.batch;
  t = q; q = t / n_layers;
  r.layer = t - q * n_layers;
  r.kv = q;  // K tiles first, then V tiles
  return r;
}

// Advance a decoded tile by `step` tiles without dividing (the carry loop runs about
// step / tt_n + 1 times; the layer index may run past the end, which the caller bounds).
__device__ __forceinline__ void advance_tile(Tile& r, const CompressArgs& a, const TileGeom& g, int step) {
  r.tt += step;
  while (r.tt >= g.tt_n) {
    r.tt -= g.tt_n;
    if (++r.hg == g.hg_n) {
      r.hg = 0;
      if (++r.b == a.batch) {
        r.b = 0;
        ++r.layer;
      }
    }
  }
}

template <typename TIn, int D>
struct Smem {
  static constexpr int kRowBytes = D * InTraits<TIn>::kBytes;
  static constexpr int kRowStride = kRowBytes + 16;  // padded: conflict-free 16-byte reads
  static constexpr int kTabStride = 2 * (D / 2) * 4 + 16;
  static constexpr int kRows = kCompressVecs * kRowStride;
  // rows + one RoPE row per token of the tile, rounded to 128 bytes
  __host__ __device__ static constexpr int stage(int head_group) {
    return (kRows + (kCompressVecs / head_group) * kTabStride + 127) & ~127;
  }
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Copy one tile's rows (and, for keys, its tokens' RoPE rows) into a stage with 16-byte
// cp.async.  A warp copies exactly the rows of its own 16 vectors (and of their tokens), so
// a warp barrier orders the copies and their readers; consecutive lanes take consecutive
// chunks of a row, so every copy instruction moves whole contiguous rows (good coalescing,
// and few large reads when the layers sit in host memory behind PCIe).
template <typename TIn, int D>
__device__ __forceinline__ void issue_tile(const CompressArgs& a, const Tile& t, uint8_t* stage) {
  using S = Smem<TIn, D>;
  constexpr int CPR = S::kRowBytes / 16;  // 16-byte chunks per row
  constexpr int WV = 16;                  // vectors per warp
  const LayerIO& L = a.layers[t.layer];
  const bool key = t.kv == 0;
  const TIn* src = static_cast<const TIn*>(key ? L.k : L.v);
  if (src == nullptr) return;
  const int HG = a.head_group, TOK = kCompressVecs >> a.hg_shift;
  const int count = a.kept_count ? min(a.kept_count[t.b], a.n_kept) : a.n_kept;
  const int lane = threadIdx.x & 31, wv0 = (threadIdx.x >> 5) * WV;  // the warp's first vector
  // this lane's vector (lanes 2v, 2v+1 own vector v): its row address and RoPE position
  const int v = threadIdx.x >> 1;
  const int tok_l = v >> a.hg_shift, head_l = v & (HG - 1);
  const int j = t.tt * TOK + tok_l;
  const int head = t.hg * HG + head_l;
  const bool vj = j < count;
  const int row = vj ? (a.kept_idx ? a.kept_idx[(int64_t)t.b * a.n_kept + j] : j) : 0;
  const bool valid = vj && head < a.heads;
  const uint8_t* g = valid ? reinterpret_cast<const uint8_t*>(src + (int64_t)t.b * a.in_stride_b +
                                                              (int64_t)head * a.in_stride_h +
                                                              (int64_t)row * a.in_stride_t)
                           : nullptr;
#pragma unroll
  for (int i = 0; i < WV * CPR / 32; ++i) {
    const int c = i * 32 + lane;
    const int rv = c / CPR, ck = c % CPR;  // row (vector) within the warp, chunk within the row
    const uint8_t* gr = reinterpret_cast<const uint8_t*>(
        __shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(g), 2 * rv));
    if (gr) cp_async16(stage + (wv0 + rv) * S::kRowStride + 16 * ck, gr + 16 * ck);
  }
  if (key) {
    // the warp's tokens: vectors wv0 .. wv0+15 -> tokens wv0/HG .. (wv0+15)/HG
    constexpr int HALF = (D / 2) * 4 / 16;  // chunks of one cos (or sin) row
    // clamped into the table: a position past it must not read outside the RoPE rows
    const int pos = vj ? min(max(a.positions ? a.positions[(int64_t)t.b * a.n_kept + j] : row, 0), a.rope_rows - 1)
                       : -1;
    const int tw0 = wv0 >> a.hg_shift, ntw = (WV + HG - 1) >> a.hg_shift;  // tokens of this warp
    const int n_chunks = ntw * 2 * HALF;
    for (int c0 = 0; c0 < n_chunks; c0 += 32) {  // uniform trip count: the shuffle needs every lane
      const int c = c0 + lane;
      const int tk = min(c / (2 * HALF), ntw - 1), k = c % (2 * HALF);
      // position of token tw0 + tk, held by the lanes of its first vector (HG divides 16)
      const int p = __shfl_sync(0xffffffffu, pos, 2 * tk * HG);
      if (c >= n_chunks || p < 0 || tw0 + tk >= TOK) continue;
      uint8_t* trow = stage + S::kRows + (tw0 + tk) * S::kTabStride;
      if (k < HALF) cp_async16(trow + 16 * k, a.rope_cos + (int64_t)p * (D / 2) + 4 * k);
      else cp_async16(trow + 16 * k, a.rope_sin + (int64_t)p * (D / 2) + 4 * (k - HALF));
    }
  }
}

// Coordinates j0 .. j0+7 of a staged row (j0 a multiple of 8), widened to fp32 and, for keys,
// inverse-rotated at the row's position: y_i = x_i c + x_{i+HF} s, y_{i+HF} = x_{i+HF} c - x_i s,
// each rounded as the whole-row rotation rounds it.
template <typename TIn, bool KEY, int HF>
__device__ __forceinline__ void chunk_in(const TIn* r, const float* cs, const float* sn, int j0, float (&x)[8]) {
  load8(r + j0, x);
  if constexpr (KEY) {
    const bool up = j0 < HF;
    const int i0 = up ? j0 : j0 - HF;
    float pr[8];
    load8(r + (up ? j0 + HF : i0), pr);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float c = cs[i0 + u], s = sn[i0 + u];
      const float a = __fmul_rn(x[u], c), b = __fmul_rn(pr[u], s);
      x[u] = up ? __fadd_rn(a, b) : __fsub_rn(a, b);
    }
  }
}

// --------------------------------------------------------------------------
// Per-vector body (two threads per vector), one tile of K or V, one format.
// Thread h of the pair owns pairs P[q] = {x[q], x[q + DP/2]} for q in
// [h*DP/4, (h+1)*DP/4): all butterfly stages but one are in-thread, the stage
// of stride DP/4 crosses the pair through one shuffle per register.
// --------------------------------------------------------------------------
template <typename TIn, int D, int DP, bool KEY, int LEV, bool RECON>
__device__ __forceinline__ void compress_tile(const CompressArgs& a, const Tile& t, const uint8_t* stage) {
  using S = Smem<TIn, D>;
  constexpr int H2 = DP / 2;  // pairs per vector
  constexpr int HP = H2 / 2;  // pairs per thread
  const LayerIO& L = a.layers[t.layer];
  if ((KEY ? L.k : L.v) == nullptr) return;  // uniform over the CTA
  constexpr int FMT = fmt_of(LEV);
  const int HG = a.head_group, TOK = kCompressVecs >> a.hg_shift;
  const int count = a.kept_count ? min(a.kept_count[t.b], a.n_kept) : a.n_kept;
  const int v = threadIdx.x >> 1, h = threadIdx.x & 1;
  const int tok_l = v >> a.hg_shift, head_l = v & (HG - 1);
  const int j = t.tt * TOK + tok_l;
  const int head = t.hg * HG + head_l;
  // both threads of every pair run the whole body (they exchange data); invalid ones store nothing
  const bool valid = j < count && head < a.heads;

  // ---- load, widen, inverse RoPE -> this thread's pairs
  u64 P[HP];
  const TIn* r = reinterpret_cast<const TIn*>(stage + v * S::kRowStride);
  const float* cs = reinterpret_cast<const float*>(stage + S::kRows + tok_l * S::kTabStride);
  const float* sn = cs + D / 2;
  const int q0 = h * HP;
  if constexpr (D == DP) {
#pragma unroll
    for (int k = 0; k < HP / 8; ++k) {
      float lo[8], hi[8];
      load8(r + q0 + 8 * k, lo);
      load8(r + H2 + q0 + 8 * k, hi);
#pragma unroll
      for (int i = 0; i < 8; ++i) P[8 * k + i] = pk(lo[i], hi[i]);
    }
    if constexpr (KEY) {
      // pair (q, q + D/2) is P[q]: y1 = x1 c + x2 s, y2 = x2 c - x1 s
#pragma unroll
      for (int q = 0; q < HP; q += 4) {
        const float4 c4 = *reinterpret_cast<const float4*>(cs + q0 + q);
        const float4 s4 = *reinterpret_cast<const float4*>(sn + q0 + q);
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
    // D < DP (96 -> 128): thread h needs coordinates j = h*HP + q (low) and H2 + h*HP + q
    // (high; past D they are the zero pad).  Chunks of 8 coordinates never straddle D/2 or D,
    // so each thread loads (and, for keys, inverse-rotates) only the chunks it owns: the chunk
    // addresses differ between the two threads of a pair, the code does not.
    constexpr int HF = D / 2;
    static_assert(HF % 8 == 0 && (D - H2) % 8 == 0 && D >= H2 && HP % 8 == 0, "chunking of the padded path");
#pragma unroll
    for (int k = 0; k < HP / 8; ++k) {
      const int jl = h * HP + 8 * k;
      const int jh0 = H2 + h * HP + 8 * k;
      const bool vh = jh0 < D;
      float lo[8], hi[8];
      chunk_in<TIn, KEY, HF>(r, cs, sn, jl, lo);
      chunk_in<TIn, KEY, HF>(r, cs, sn, vh ? jh0 : jl, hi);  // a valid chunk; replaced by the pad
#pragma unroll
      for (int i = 0; i < 8; ++i) P[8 * k + i] = pk(lo[i], vh ? hi[i] : 0.0f);
    }
  }

  // ---- rotate: stages 1 .. HP/2 in-thread, stage HP across the pair, stage H2 inside each register
  float amax = 0.0f;
  if (a.rotate) {
#pragma unroll
    for (int st = 1; st < HP; st <<= 1) {
#pragma unroll
      for (int q = 0; q < HP; ++q) {
        if ((q & st) == 0) {
          const u64 u = P[q], w2 = P[q + st];
          P[q] = add2(u, w2);
          P[q + st] = sub2(u, w2);
        }
      }
    }
    // lower thread: a + b; upper thread: a - b  (a = lower thread's value)  == fma(mine, +-1, other)
    const float sg = h ? -1.0f : 1.0f;
    const u64 sg2 = pk(sg, sg);
#pragma unroll
    for (int q = 0; q < HP; ++q) {
      const u64 o = __shfl_xor_sync(0xffffffffu, P[q], 1);
      P[q] = fma2(P[q], sg2, o);
    }
    const u64 hh = pk(hadamard_entry(DP), hadamard_entry(DP));
#pragma unroll
    for (int q = 0; q < HP; ++q) {
      float u, w2;
      upk(P[q], u, w2);
      P[q] = mul2(pk(__fadd_rn(u, w2), __fsub_rn(u, w2)), hh);
      float y0, y1;
      upk(P[q], y0, y1);
      amax = max3(amax, fabsf(y0), fabsf(y1));
    }
  } else {
#pragma unroll
    for (int q = 0; q < HP; ++q) {
      float y0, y1;
      upk(P[q], y0, y1);
      amax = max3(amax, fabsf(y0), fabsf(y1));
    }
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, 1e-8f);
  const float sc = __fmul_rn(amax, 2.0f / static_cast<float>(LEV));  // 2 / L: exact (power of two)
  const float rcp = __frcp_rn(sc);
  const u64 r2 = pk(rcp, rcp), nsc2 = pk(-sc, -sc);

  // ---- lattice: this thread's groups g (low lanes) and g + DP/16 (high lanes)
  constexpr int GT = HP / 8;                  // groups per lane type per thread
  constexpr int GB = FMT == 0 ? 4 : (FMT == 1 ? 5 : 8);  // bytes per group
  constexpr int REG = GT * GB;                // bytes per region (low / high)
  constexpr int RW = (REG + 3) / 4;           // words per region
  uint32_t wl[RW], wh[RW];
#pragma unroll
  for (int i = 0; i < RW; ++i) { wl[i] = 0u; wh[i] = 0u; }
  uint32_t gl_all[RECON ? GT : 1][GF<FMT>::kWords], gh_all[RECON ? GT : 1][GF<FMT>::kWords];
#pragma unroll
  for (int g = 0; g < GT; ++g) {
    float elo[8], ehi[8];
    uint32_t slo[8], shi[8], blo[8], bhi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const u64 y = P[8 * g + i];
      // correctly rounded y / sc (Markstein): q = y r; rem = y - q sc; q + rem r
      const u64 q1 = mul2(y, r2);
      const u64 rem = fma2(q1, nsc2, y);
      const u64 n = fma2(rem, r2, q1);
      // the roundings, packed: s = n + M (rint in the low bits), e = n - (s - M), and
      // b = fl(n - 1/2) + M for the half-integer candidate
      const u64 M2 = pk(kMagic, kMagic);
      const u64 s2 = add2(n, M2);
      const u64 e2 = sub2(n, sub2(s2, M2));
      const u64 b2 = add2(sub2(n, pk(0.5f, 0.5f)), M2);
      float s0, s1, b0, b1;
      upk(s2, s0, s1);
      upk(e2, elo[i], ehi[i]);
      upk(b2, b0, b1);
      slo[i] = __float_as_uint(s0); shi[i] = __float_as_uint(s1);
      blo[i] = __float_as_uint(b0); bhi[i] = __float_as_uint(b1);
    }
    uint32_t glo[GF<FMT>::kWords], ghi[GF<FMT>::kWords];
    e8_group<FMT, LEV>(elo, slo, blo, glo);
    e8_group<FMT, LEV>(ehi, shi, bhi, ghi);
    place_group<FMT>(wl, g, glo);
    place_group<FMT>(wh, g, ghi);
    if constexpr (RECON) {
#pragma unroll
      for (int k = 0; k < GF<FMT>::kWords; ++k) { gl_all[g][k] = glo[k]; gh_all[g][k] = ghi[k]; }
    }
  }

  // ---- outputs
  const int64_t vrow = ((int64_t)t.b * a.heads + head) * a.n_kept + j;
  uint8_t* codes = KEY ? L.k_codes : L.v_codes;
  constexpr int PB = Fmt<FMT, DP>::kBytes;
  constexpr int HOFF = (H2 / 8) * GB;  // byte offset of the high-lane groups
  constexpr int G = gcd_pow2(gcd_pow2(REG, HOFF), PB);
  if (valid && codes) {
    uint8_t* row = codes + vrow * PB;
    store_region<REG, G>(row + h * REG, wl);
    store_region<REG, G>(row + HOFF + h * REG, wh);
  }
  if (valid && h == 0) {
    uint16_t* sc16 = KEY ? L.k_scales : L.v_scales;
    if (sc16) sc16[vrow] = __half_as_ushort(__float2half_rn(sc));
    float* sc32 = KEY ? L.k_scales_f32 : L.v_scales_f32;
    if (sc32) sc32[vrow] = sc;
  }
  if constexpr (RECON && D == DP) {
    // Fake-quant reconstruction, split like the forward path: this thread rebuilds its own
    // pairs {x[q], x[q + DP/2]} (q in [h HP, (h + 1) HP)) from its groups' codes; the inverse
    // butterfly runs on exact integers (|partial sums| <= 16 DP), so its order does not change
    // a bit; then * fl(sc / 2 * h), forward RoPE at the output position, sharpening and fp16,
    // each rounded as recon_store rounds them.
    uint16_t* out = KEY ? L.k_out : L.v_out;
    if (out) {
      u64 R[HP];
#pragma unroll
      for (int g = 0; g < GT; ++g)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          R[8 * g + i] = pk(static_cast<float>(group_code<FMT>(gl_all[g], i)),
                            static_cast<float>(group_code<FMT>(gh_all[g], i)));
      if (a.rotate) {
#pragma unroll
        for (int st = 1; st < HP; st <<= 1) {
#pragma unroll
          for (int q = 0; q < HP; ++q) {
            if ((q & st) == 0) {
              const u64 u = R[q], w2 = R[q + st];
              R[q] = add2(u, w2);
              R[q + st] = sub2(u, w2);
            }
          }
        }
        const float sg = h ? -1.0f : 1.0f;
        const u64 sg2 = pk(sg, sg);
#pragma unroll
        for (int q = 0; q < HP; ++q) {
          const u64 o = __shfl_xor_sync(0xffffffffu, R[q], 1);
          R[q] = fma2(R[q], sg2, o);
        }
#pragma unroll
        for (int q = 0; q < HP; ++q) {
          float u, w2;
          upk(R[q], u, w2);
          R[q] = pk(__fadd_rn(u, w2), __fsub_rn(u, w2));
        }
      }
      if (valid) {
        const int src_row = a.kept_idx ? a.kept_idx[(int64_t)t.b * a.n_kept + j] : j;
        const int pos = min(max(a.positions ? a.positions[(int64_t)t.b * a.n_kept + j] : src_row, 0), a.rope_rows - 1);
        const int orow = a.out_row_mode == 1 ? j : src_row;
        int opos = pos;
        if (a.out_positions) opos = a.out_positions[(int64_t)t.b * a.n_kept + j];
        else if (a.out_row_mode == 1) opos = j;
        opos = min(max(opos, 0), a.rope_rows - 1);
        __half* o = reinterpret_cast<__half*>(out) + (int64_t)t.b * a.out_stride_b +
                    (int64_t)head * a.out_stride_h + (int64_t)orow * a.out_stride_t;
        const float coef = __fmul_rn(sc, a.rotate ? 0.5f * hadamard_entry(DP) : 0.5f);
        const u64 coef2 = pk(coef, coef), sh2 = pk(a.key_sharpen, a.key_sharpen);
        const float* cr = a.rope_cos + (int64_t)opos * (D / 2) + q0;
        const float* sr = a.rope_sin + (int64_t)opos * (D / 2) + q0;
#pragma unroll
        for (int k = 0; k < HP / 8; ++k) {
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int u = 0; u < 8; u += 2) {
            float y1[2], y2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int q = 8 * k + u + e;
              u64 z = mul2(R[q], coef2);
              if constexpr (KEY) {
                const float c = __ldg(cr + q), sn2 = __ldg(sr + q);
                float m1, m2, n1, n2;
                upk(mul2(z, pk(c, c)), m1, m2);
                upk(mul2(z, pk(sn2, sn2)), n1, n2);
                z = pk(__fsub_rn(m1, n2), __fadd_rn(n1, m2));
                if (a.key_sharpen != 1.0f) z = mul2(z, sh2);
              }
              upk(z, y1[e], y2[e]);
            }
            const __half2 hl = __floats2half2_rn(y1[0], y1[1]), hv = __floats2half2_rn(y2[0], y2[1]);
            lo[u / 2] = *reinterpret_cast<const uint32_t*>(&hl);
            hi[u / 2] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          reinterpret_cast<uint4*>(o + q0)[k] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          reinterpret_cast<uint4*>(o + H2 + q0)[k] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        }
      }
    }
  } else if constexpr (RECON) {
    uint16_t* out = KEY ? L.k_out : L.v_out;
    if (out) {
      // assemble the full code vector in the lower thread of the pair
      float x[DP];
#pragma unroll
      for (int g = 0; g < GT; ++g)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int mine_l = group_code<FMT>(gl_all[g], i), mine_h = group_code<FMT>(gh_all[g], i);
          const int oth_l = __shfl_xor_sync(0xffffffffu, mine_l, 1);
          const int oth_h = __shfl_xor_sync(0xffffffffu, mine_h, 1);
          const int q = 8 * g + i;
          x[q] = static_cast<float>(mine_l);             // valid in the lower thread
          x[q + HP] = static_cast<float>(oth_l);
          x[q + H2] = static_cast<float>(mine_h);
          x[q + HP + H2] = static_cast<float>(oth_h);
        }
      if (valid && h == 0) {
        const int src_row = a.kept_idx ? a.kept_idx[(int64_t)t.b * a.n_kept + j] : j;
        const int pos = min(max(a.positions ? a.positions[(int64_t)t.b * a.n_kept + j] : src_row, 0), a.rope_rows - 1);
        const int orow = a.out_row_mode == 1 ? j : src_row;
        int opos = pos;
        if (a.out_positions) opos = a.out_positions[(int64_t)t.b * a.n_kept + j];
        else if (a.out_row_mode == 1) opos = j;
        opos = min(max(opos, 0), a.rope_rows - 1);
        __half* o = reinterpret_cast<__half*>(out) + (int64_t)t.b * a.out_stride_b +
                    (int64_t)head * a.out_stride_h + (int64_t)orow * a.out_stride_t;
        recon_store<D, DP>(x, sc, KEY, a.rope_cos + (int64_t)opos * (D / 2), a.rope_sin + (int64_t)opos * (D / 2),
                           a.key_sharpen, a.rotate != 0, o);
      }
    }
  }
}

// --------------------------------------------------------------------------
// Persistent kernel: 1- or 2-stage cp.async pipeline over the tile list.  KVS selects the
// key tiles (0, the first half of the tile list) or the value tiles (1): each instantiation
// holds one per-vector body, half the code of a kernel that handles both, which keeps the
// instruction cache from thrashing.
// --------------------------------------------------------------------------
template <typename TIn, int D, int DP, int LEV, bool RECON, int KVS>
__global__ void __launch_bounds__(kCompressThreads, 4) compress_kernel(const CompressArgs args, int n_layers,
                                                                        int n_tiles, int ns) {
  using S = Smem<TIn, D>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int first = blockIdx.x;
  if (first >= n_tiles) return;
  const int base = KVS * n_tiles;  // n_tiles = tiles of this half
  const int stage_bytes = S::stage(args.head_group);
  const TileGeom geom = tile_geom(args);
  const int step = (int)gridDim.x;
  Tile cur = decode_tile(args, geom, n_layers, base + first);
  issue_tile<TIn, D>(args, cur, smem);
  cp_async_commit();
  int it = 0;
  // ns = 2: tile i+1 is copied into the other stage while tile i is computed;
  // ns = 1 (rows too large for two stages): copy and compute alternate.
  for (int tile = first; tile < n_tiles; tile += step, ++it) {
    const int s = ns == 2 ? (it & 1) : 0;
    const bool has_next = tile + step < n_tiles;
    Tile nt = cur;
    if (has_next) advance_tile(nt, args, geom, step);
    if (ns == 2) {
      __syncwarp();  // this warp is done with stage s^1 (previous tile)
      if (has_next) issue_tile<TIn, D>(args, nt, smem + (s ^ 1) * stage_bytes);
      cp_async_commit();
      cp_async_wait<1>();  // everything but the newest group: the current tile has landed
    } else {
      cp_async_wait<0>();
    }
    __syncwarp();
    const uint8_t* stage = smem + s * stage_bytes;
    compress_tile<TIn, D, DP, KVS == 0, LEV, RECON>(args, cur, stage);
    if (ns == 1 && has_next) {
      __syncwarp();
      issue_tile<TIn, D>(args, nt, smem);
      cp_async_commit();
    }
    cur = nt;
  }
}

// --------------------------------------------------------------------------
// Launch
// --------------------------------------------------------------------------
// One half of the tile list (kvs 0: key tiles, 1: value tiles) at level count LEV.
template <typename TIn, int D, int DP, int LEV>
static cudaError_t launch_half(const CompressArgs& a, int n_layers, long long half, int kvs, cudaStream_t s,
                               bool recon) {
  using S = Smem<TIn, D>;
  int dev = 0, sms = 0, per_sm = 0, max_smem = 0;
  cudaError_t e;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return e;
  const int ns = 2 * (size_t)S::stage(a.head_group) + 64 <= (size_t)max_smem ? 2 : 1;
  const size_t smem = ns * (size_t)S::stage(a.head_group);
  auto kern = kvs == 0 ? (recon ? compress_kernel<TIn, D, DP, LEV, true, 0> : compress_kernel<TIn, D, DP, LEV, false, 0>)
                       : (recon ? compress_kernel<TIn, D, DP, LEV, true, 1> : compress_kernel<TIn, D, DP, LEV, false, 1>);
  if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kCompressThreads, smem)) != cudaSuccess)
    return e;
  long long grid = (long long)sms * (per_sm > 0 ? per_sm : 1);
  if (grid > half) grid = half;
  if (grid > 0) kern<<<(unsigned)grid, kCompressThreads, smem, s>>>(a, n_layers, (int)half, ns);
  return cudaGetLastError();
}

template <typename TIn, int D, int DP>
static cudaError_t launch_dims(const CompressArgs& a, int n_layers, long long n_tiles, int lk, int lv,
                               cudaStream_t s, bool recon) {
  // key tiles (first half of the tile list), then value tiles, one kernel each
  const long long half = n_tiles / 2;
  for (int kvs = 0; kvs < 2; ++kvs) {
    const int lev = kvs == 0 ? lk : lv;
    if (lev == 0) continue;  // no layer of this launch has this tensor
    cudaError_t e = cudaErrorInvalidValue;
    switch (lev) {
      case 2: e = launch_half<TIn, D, DP, 2>(a, n_layers, half, kvs, s, recon); break;
      case 4: e = launch_half<TIn, D, DP, 4>(a, n_layers, half, kvs, s, recon); break;
      case 8: e = launch_half<TIn, D, DP, 8>(a, n_layers, half, kvs, s, recon); break;
      case 16: e = launch_half<TIn, D, DP, 16>(a, n_layers, half, kvs, s, recon); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Instantiated once per input dtype in nq_compress_{f16,bf16,f32}.cu (parallel builds).
template <typename TIn>
cudaError_t launch_compress_t(const CompressArgs& a, int n_layers, long long n_tiles, int lk, int lv, cudaStream_t s,
                              bool recon) {
  if (a.head_dim == 128 && a.head_dim_padded == 128) return launch_dims<TIn, 128, 128>(a, n_layers, n_tiles, lk, lv, s, recon);
  if (a.head_dim == 96 && a.head_dim_padded == 128) return launch_dims<TIn, 96, 128>(a, n_layers, n_tiles, lk, lv, s, recon);
  if (a.head_dim == 64 && a.head_dim_padded == 64) return launch_dims<TIn, 64, 64>(a, n_layers, n_tiles, lk, lv, s, recon);
  return cudaErrorInvalidValue;
}

}  // namespace nq
