// Token-importance kernels on the 5th-generation tensor cores (tcgen05 / TMEM).
//
// Computes, per (batch, query head), the softmax column sums of the logits
// Q K^T * scale over the keys (nexusquant/pipeline.py:756-782 key-key proxy,
// :784-836 real-attention scorer), in two passes over the keys plus a combine:
//   PASS 1  per CTA chunk of key tiles, per query: max of base-2 logits and the
//           sum of 2^(l - max) (written per chunk);
//   combine per query: chunk statistics -> M (max) and Z (sum);
//   PASS 3  per key: sum over queries of 2^(l - M_q) / Z_q.
//
// Per key tile (128 keys):
//  * TMA (cp.async.bulk.tensor, no multicast) copies the tile as 128-byte
//    swizzled rows of 64 head-dim elements into one of three shared stages;
//    the query tile (32 or 64 rows) is loaded the same way once per CTA.
//  * One thread issues tcgen05.mma (kind::f16, M = 128 keys, N = queries,
//    K = 16 per instruction, fp32 accumulation) into one of two TMEM
//    accumulators, so the MMA of tile i+1 overlaps the softmax of tile i.
//  * Warp w reads TMEM lanes 32*(w%4) .. (its keys) with tcgen05.ld: every
//    thread owns one key and 32 queries (warps 4..7 take queries 32..63), so
//    PASS 3 sums over queries inside the thread and PASS 1 keeps per-thread
//    running (max, sum) per query, merged across threads once per chunk.
// All reductions have a fixed order: the result is deterministic.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "../../include/nexusquant_b200.h"
#include "nq_common.cuh"
#include "nq_internal.h"
#include "nq_umma.cuh"

namespace nq {

namespace {

constexpr int kUmKeys = 128;     // keys per tile (MMA M)

// Device error word of this library's bounded waits (one per device): bit 0 a scorer wait,
// bit 1 the wait self-test.  Read and cleared by nq_device_error().
__device__ unsigned int g_wait_error;
constexpr unsigned int kWaitErrScore = 1u, kWaitErrSelfTest = 2u;
constexpr int kUmStages = 3;     // key-tile stages
constexpr float kLog2eU = 1.4426950408889634f;

__device__ __forceinline__ float ex2u(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace

// Shared-memory layout: key stages (1024-aligned), query tile, barriers.
template <int D, int NQP>
struct UmLayout {
  static constexpr int kBlocks = (D + 63) / 64;            // 64-element (128-byte) column blocks
  static constexpr int kKeyBlock = kUmKeys * 128;          // one column block of a key tile
  static constexpr int kStage = kBlocks * kKeyBlock;
  static constexpr int kQBlock = NQP * 128;
  static constexpr int kQ = kBlocks * kQBlock;
  static constexpr int kThreadsQ = 128 * (NQP / 32);
  static constexpr int kScratch = kThreadsQ * 32 * 2 * 4;  // PASS 1 end-of-chunk merge (reuses the stages)
  static constexpr int kMain = kUmStages * kStage + kQ;
  static constexpr int kBytes = (kMain > kScratch ? kMain : kScratch) + 1024;  // + alignment slack
  static constexpr int kThreads = 128 * (NQP / 32);
  static constexpr uint32_t kTmemCols = 2 * NQP < 32 ? 32 : 2 * NQP;  // power of two >= 32
};

struct UmWs {
  float* pm;  // [B, Hr, chunks, nq] chunk max (base-2 logits)
  float* pl;  // [B, Hr, chunks, nq] chunk sum of 2^(l - max)
  float* M;   // [B, Hr, nq]
  float* Z;   // [B, Hr, nq]
};

template <int D, int NQP, int PASS>
__global__ void __launch_bounds__(UmLayout<D, NQP>::kThreads, 1)
    score_umma(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap qmap, const ScoreArgs a,
               UmWs w, float* colsum, int tiles_per_cta, uint32_t idesc) {
  using Lo = UmLayout<D, NQP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem + kUmStages * Lo::kStage;
  __shared__ uint64_t kbar[kUmStages], mbar[2], qbar;
  __shared__ uint32_t tmem_base;
  __shared__ int err;
  __shared__ float sM[NQP], sZi[NQP];

  const int hr = blockIdx.y, b = blockIdx.z;
  const int qh = a.head_begin + hr;
  const int Hr = a.head_end - a.head_begin;
  const int kh = qh / (a.q_heads / a.heads);
  const int tiles = (a.seq + kUmKeys - 1) / kUmKeys;
  const int t0 = blockIdx.x * tiles_per_cta;
  const int t1 = min(tiles, t0 + tiles_per_cta);
  if (t0 >= t1) return;
  const int n_t = t1 - t0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3;                    // TMEM lane quarter of this warp
  const int qoff = (warp >> 2) * 32;            // this thread's 32 queries
  const uint32_t stage_tx = (uint32_t)Lo::kStage, q_tx = (uint32_t)Lo::kQ;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kUmStages; ++i) mbar_init(&kbar[i], 1);
    mbar_init(&mbar[0], 1);
    mbar_init(&mbar[1], 1);
    mbar_init(&qbar, 1);
    fence_mbar_init();
    err = 0;
  }
  if (warp == 0) tmem_alloc(&tmem_base, Lo::kTmemCols);
  if (PASS == 3 && threadIdx.x < NQP) {
    const bool ok = threadIdx.x < a.n_q;
    const int64_t o = ((int64_t)b * Hr + hr) * a.n_q + threadIdx.x;
    sM[threadIdx.x] = ok ? w.M[o] : 0.0f;
    sZi[threadIdx.x] = ok ? __frcp_rn(w.Z[o]) : 0.0f;  // 1 / Z
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;

  // producer: thread 0 issues the TMA copies and the MMAs
  auto issue_keys = [&](int i) {  // tile t0 + i -> stage i % kUmStages
    const int st = i % kUmStages;
    mbar_arrive_expect_tx(&kbar[st], stage_tx);
    for (int blk = 0; blk < Lo::kBlocks; ++blk)
      tma_load_4d(smem + st * Lo::kStage + blk * Lo::kKeyBlock, &kmap, blk * 64, (t0 + i) * kUmKeys, kh, b,
                  &kbar[st]);
  };
  auto issue_mma = [&](int i) {  // tile t0 + i from stage i % 3 -> TMEM accumulator i & 1
    const uint8_t* ks = smem + (i % kUmStages) * Lo::kStage;
    const uint32_t dacc = tbase + (uint32_t)((i & 1) * NQP);
#pragma unroll
    for (int k = 0; k < D / 16; ++k) {
      const int blk = k >> 2, off = (k & 3) * 32;
      umma_f16(dacc, sw128_desc(ks + blk * Lo::kKeyBlock + off), sw128_desc(qs + blk * Lo::kQBlock + off), idesc,
               k > 0 ? 1u : 0u);
    }
    umma_commit(&mbar[i & 1]);
  };

  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&qbar, q_tx);
    const int qrow = a.q ? 0 : a.seq - a.n_q;
    const int qhead = a.q ? qh : kh;
    for (int blk = 0; blk < Lo::kBlocks; ++blk)
      tma_load_4d(qs + blk * Lo::kQBlock, &qmap, blk * 64, qrow, qhead, b, &qbar);
    issue_keys(0);
    if (n_t > 1) issue_keys(1);
    if (!mbar_wait(&qbar, 0) || !mbar_wait(&kbar[0], 0)) {
      err = 1;
    } else {
      tc_fence_after();
      issue_mma(0);
    }
  }

  const float sc2 = a.scale * kLog2eU;
  float rm[32], rs[32];  // PASS 1 running statistics of this thread's key lane
#pragma unroll
  for (int q = 0; q < 32; ++q) { rm[q] = -INFINITY; rs[q] = 0.0f; }

  for (int i = 0; i < n_t; ++i) {
    // producer: MMA for tile i+1 (its stage has landed), keys for tile i+2
    if (threadIdx.x == 0 && !err) {
      if (i + 1 < n_t) {
        if (!mbar_wait(&kbar[(i + 1) % kUmStages], ((i + 1) / kUmStages) & 1)) {
          err = 1;
        } else {
          tc_fence_after();
          issue_mma(i + 1);
        }
      }
      if (i + 2 < n_t && !err) issue_keys(i + 2);  // stage of tile i-1, whose MMA was consumed
    }
    // consumers: logits of tile i
    const bool ok = mbar_wait(&mbar[i & 1], (i >> 1) & 1);
    if (!ok) err = 1;
    tc_fence_after();
    __syncwarp();  // tcgen05.ld is warp-collective; thread 0 arrives from the producer branch
    float x[32];
    tmem_ld32(tbase + ((uint32_t)(quad * 32) << 16) + (uint32_t)((i & 1) * NQP + qoff), x);
    const int key = (t0 + i) * kUmKeys + quad * 32 + lane;
    if (PASS == 1) {
      if (ok) {
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const int qq = qoff + q;
          const bool vis = key < a.seq && qq < a.n_q && (!a.causal || key <= a.q_pos0 + qq);
          if (vis) {
            const float l = __fmul_rn(x[q], sc2);
            const float d = __fsub_rn(l, rm[q]);
            const float e = ex2u(-fabsf(d));
            // l <= max: s += 2^(l - max); l > max: s = s * 2^(max - l) + 1, max = l
            rs[q] = d > 0.0f ? __fmaf_rn(rs[q], e, 1.0f) : __fadd_rn(rs[q], e);
            rm[q] = fmaxf(rm[q], l);
          }
        }
      }
    } else {
      float v = 0.0f;
      if (ok) {
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const int qq = qoff + q;
          const bool vis = qq < a.n_q && (!a.causal || key <= a.q_pos0 + qq);
          if (vis) v = __fadd_rn(v, __fmul_rn(ex2u(__fsub_rn(__fmul_rn(x[q], sc2), sM[qq])), sZi[qq]));
        }
      }
      if (NQP == 32) {
        if (ok && key < a.seq) colsum[((int64_t)b * Hr + hr) * a.seq + key] = v;
      } else {
        // queries 32..63 (warps 4..7) hand their partial sums to warps 0..3 through the consumed
        // stage of tile i (the MMA reading it has completed; tile i+3 is copied in only after the
        // end-of-iteration barrier)
        float* part = reinterpret_cast<float*>(smem + (i % kUmStages) * Lo::kStage);
        if (warp >= 4) part[threadIdx.x - 128] = v;
        __syncthreads();
        if (warp < 4 && ok && key < a.seq)
          colsum[((int64_t)b * Hr + hr) * a.seq + key] = __fadd_rn(v, part[threadIdx.x]);
      }
    }
    tc_fence_before();
    __syncthreads();  // accumulator i & 1 and stage i % 3 are free for tile i + 2 / i + 3
    tc_fence_after();
    if (err) break;
  }

  if (PASS == 1 && !err) {
    // merge the per-thread statistics of each query over the 128 key lanes, lane order
    float* sm = reinterpret_cast<float*>(smem);  // all stages are consumed
    float* ss = sm + Lo::kThreads * 32;
#pragma unroll
    for (int q = 0; q < 32; ++q) {
      sm[q * Lo::kThreads + threadIdx.x] = rm[q];
      ss[q * Lo::kThreads + threadIdx.x] = rs[q];
    }
    __syncthreads();
    if (threadIdx.x < NQP && threadIdx.x < a.n_q) {
      const int q = threadIdx.x;
      const int col = q & 31, half = q >> 5;  // stored by threads 128*half .. 128*half+127
      float m = -INFINITY, s = 0.0f;
      for (int t = 0; t < 128; ++t) {
        const int src = col * Lo::kThreads + half * 128 + t;
        const float mt = sm[src], st = ss[src];
        if (mt == -INFINITY) continue;
        if (mt > m) {
          s = __fadd_rn(__fmul_rn(s, ex2u(__fsub_rn(m, mt))), st);
          m = mt;
        } else {
          s = __fadd_rn(s, __fmul_rn(st, ex2u(__fsub_rn(mt, m))));
        }
      }
      const int64_t o = (((int64_t)b * Hr + hr) * gridDim.x + blockIdx.x) * a.n_q + q;
      w.pm[o] = m;
      w.pl[o] = s;
    }
  }
  // drain: the MMA issued for a tile that was not consumed must finish before TMEM is freed;
  // the expired wait is recorded in the device error word (nq_device_error)
  if (threadIdx.x == 0 && err) {
    mbar_wait(&mbar[0], 0, 1u << 20);
    mbar_wait(&mbar[1], 0, 1u << 20);
    atomicOr(&g_wait_error, kWaitErrScore);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tbase, Lo::kTmemCols);
}

// Per query: combine chunk statistics -> M and Z (one warp per query, fixed order).
__global__ void score_umma_combine(const ScoreArgs a, UmWs w, int chunks) {
  const int q = blockIdx.x, hr = blockIdx.y, b = blockIdx.z;
  const int Hr = a.head_end - a.head_begin;
  const int lane = threadIdx.x;
  const int64_t base = ((int64_t)b * Hr + hr) * chunks * a.n_q + q;
  float m = -INFINITY, s = 0.0f;
  for (int t = lane; t < chunks; t += 32) {
    const float mt = w.pm[base + (int64_t)t * a.n_q], st = w.pl[base + (int64_t)t * a.n_q];
    if (mt == -INFINITY) continue;
    if (mt > m) {
      s = __fadd_rn(__fmul_rn(s, ex2u(__fsub_rn(m, mt))), st);
      m = mt;
    } else {
      s = __fadd_rn(s, __fmul_rn(st, ex2u(__fsub_rn(mt, m))));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mm = fmaxf(m, m2);
    float v = 0.0f;
    if (m != -INFINITY) v = __fmul_rn(s, ex2u(__fsub_rn(m, mm)));
    if (m2 != -INFINITY) v = __fadd_rn(v, __fmul_rn(s2, ex2u(__fsub_rn(m2, mm))));
    m = mm;
    s = v;
  }
  if (lane == 0) {
    const int64_t o = ((int64_t)b * Hr + hr) * a.n_q + q;
    w.M[o] = m;
    w.Z[o] = s;
  }
}

// ------------------------------------------------------------------- host side
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 4-D map over [batch, heads, rows, D] (innermost last) with a box of 64 x box_rows, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, int dtype, int D, int rows, int heads, int batch, int64_t st,
              int64_t sh, int64_t sb, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)heads, (cuuint64_t)batch};
  const cuuint64_t strides[3] = {(cuuint64_t)st * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(m, dtype == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int D, int NQP>
cudaError_t run_umma(const ScoreArgs& a, float* colsum, void* ws, cudaStream_t s) {
  using Lo = UmLayout<D, NQP>;
  const int Hr = a.head_end - a.head_begin;
  const int tiles = (a.seq + kUmKeys - 1) / kUmKeys;
  const size_t part = ((size_t)a.batch * Hr * tiles * a.n_q * sizeof(float) + 255) & ~size_t(255);
  const size_t stat = ((size_t)a.batch * Hr * a.n_q * sizeof(float) + 255) & ~size_t(255);
  uint8_t* p = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  UmWs w{reinterpret_cast<float*>(p), reinterpret_cast<float*>(p + part), reinterpret_cast<float*>(p + 2 * part),
         reinterpret_cast<float*>(p + 2 * part + stat)};
  CUtensorMap kmap, qmap;
  // a layout the tensor-map encoder refuses (extents, strides) goes to the CUDA-core scorer
  if (!make_map(&kmap, a.k, a.in_dtype, D, a.seq, a.heads, a.batch, a.k_stride_t, a.k_stride_h, a.k_stride_b,
                kUmKeys))
    return cudaErrorNotSupported;
  const bool qmap_ok =
      a.q ? make_map(&qmap, a.q, a.in_dtype, D, a.n_q, a.q_heads, a.batch, a.q_stride_t, a.q_stride_h, a.q_stride_b,
                     NQP)
          : make_map(&qmap, a.k, a.in_dtype, D, a.seq, a.heads, a.batch, a.k_stride_t, a.k_stride_h, a.k_stride_b,
                     NQP);
  if (!qmap_ok) return cudaErrorNotSupported;
  int dev = 0, sms = 0;
  cudaError_t e;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  auto k1 = score_umma<D, NQP, 1>;
  auto k3 = score_umma<D, NQP, 3>;
  const int smem = Lo::kBytes;
  if ((e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(k3, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
  // all of the unified L1/shared array as shared memory, so two CTAs fit per SM
  if ((e = cudaFuncSetAttribute(k1, cudaFuncAttributePreferredSharedMemoryCarveout, 100)) != cudaSuccess) return e;
  if ((e = cudaFuncSetAttribute(k3, cudaFuncAttributePreferredSharedMemoryCarveout, 100)) != cudaSuccess) return e;
  // one wave: each (batch, head) row gets `chunks` CTAs walking equal runs of its tiles, with
  // chunks x rows at most the resident CTA slots (more rows than slots: one CTA per row)
  const long long rows = (long long)a.batch * Hr;
  // resident CTAs per SM: two of the 32-query kernel, one of the 64-query kernel (registers);
  // (measured: planning the 32-query kernel for two beats the occupancy query's answer of one)
  const long long slots = (long long)sms * (NQP == 32 ? 2 : 1);
  long long want = slots / (rows > 0 ? rows : 1);
  want = want < 1 ? 1 : (want > tiles ? tiles : want);
  const int tpc = (int)((tiles + want - 1) / want);
  const int chunks = (tiles + tpc - 1) / tpc;
  const uint32_t idesc = f16_idesc(a.in_dtype, kUmKeys, NQP);
  const dim3 g(chunks, Hr, a.batch);
  k1<<<g, Lo::kThreads, smem, s>>>(kmap, qmap, a, w, colsum, tpc, idesc);
  score_umma_combine<<<dim3(a.n_q, Hr, a.batch), 32, 0, s>>>(a, w, chunks);
  k3<<<g, Lo::kThreads, smem, s>>>(kmap, qmap, a, w, colsum, tpc, idesc);
  return cudaGetLastError();
}

template <int D>
cudaError_t umma_nq(const ScoreArgs& a, float* colsum, void* ws, cudaStream_t s) {
  if (a.n_q <= 32) return run_umma<D, 32>(a, colsum, ws, s);
  return run_umma<D, 64>(a, colsum, ws, s);
}

}  // namespace

bool score_umma_supported(const ScoreArgs& a) {
  if (a.in_dtype != 0 && a.in_dtype != 1) return false;
  if (a.n_q < 1 || a.n_q > 64) return false;
  if (a.head_dim != 64 && a.head_dim != 96 && a.head_dim != 128) return false;
  if ((a.k_stride_t * 2) % 16 || (a.k_stride_h * 2) % 16 || (a.k_stride_b * 2) % 16) return false;
  if (a.q && ((a.q_stride_t * 2) % 16 || (a.q_stride_h * 2) % 16 || (a.q_stride_b * 2) % 16)) return false;
  if ((reinterpret_cast<uintptr_t>(a.k) & 15) || (a.q && (reinterpret_cast<uintptr_t>(a.q) & 15))) return false;
  return encode_fn() != nullptr;
}

cudaError_t launch_score_umma(const ScoreArgs& a, float* colsum, void* ws, cudaStream_t s) {
  if (a.head_dim == 128) return umma_nq<128>(a, colsum, ws, s);
  if (a.head_dim == 96) return umma_nq<96>(a, colsum, ws, s);
  return umma_nq<64>(a, colsum, ws, s);
}

// A bounded wait that is made to expire on purpose: one CTA waits on an mbarrier nothing
// arrives on, with nothing else in flight, and records the expiry like a real kernel would.
__global__ void wait_selftest_kernel(uint32_t max_iters) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait(&bar, 0, max_iters)) atomicOr(&g_wait_error, kWaitErrSelfTest);
}

}  // namespace nq

extern "C" nq_status_t nq_device_error(int32_t* bits, nq_stream_t stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, nq::g_wait_error, sizeof(v), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return NQ_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return NQ_ERR_CUDA;
  if (v) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbolAsync(nq::g_wait_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return NQ_ERR_CUDA;
  }
  unsigned int at = 0;
  if (nq::attend_take_error(&at, s) != cudaSuccess) return NQ_ERR_CUDA;
  if (at) v |= 4u;  // decode attention
  if (bits) *bits = static_cast<int32_t>(v);
  return v ? NQ_ERR_TIMEOUT : NQ_OK;
}

extern "C" nq_status_t nq_wait_selftest(uint32_t max_iters, nq_stream_t stream) {
  if (max_iters == 0 || max_iters > (1u << 20)) return NQ_ERR_INVALID_ARG;
  nq::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(max_iters);
  return cudaGetLastError() == cudaSuccess ? NQ_OK : NQ_ERR_CUDA;
}
