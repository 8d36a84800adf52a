// Internal (non-ABI) declarations shared by the kernels and the C entry points.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nq {

constexpr int kCompressThreads = 128;   // threads per compress / dequantize CTA
constexpr int kCompressVecs = 64;       // vectors per compress tile (two threads per vector)
constexpr int kMaxLayersPerLaunch = 96; // per-layer pointers travel in the kernel parameters

struct LayerIO {
  const void* k;
  const void* v;
  uint8_t* k_codes;
  uint8_t* v_codes;
  uint16_t* k_scales;
  uint16_t* v_scales;
  float* k_scales_f32;
  float* v_scales_f32;
  uint16_t* k_out;
  uint16_t* v_out;
  int32_t key_levels, value_levels;
};

struct CompressArgs {
  int32_t batch, heads, seq, head_dim, head_dim_padded, n_kept;
  int32_t head_group;  // heads per CTA tile (1, 2, 4 or 8)
  int32_t hg_shift;    // log2(head_group), set by launch_compress
  const int32_t* kept_idx;
  const int32_t* kept_count;
  const int32_t* positions;
  const float* rope_cos;
  const float* rope_sin;
  int32_t rope_rows;
  int32_t in_dtype;
  int64_t in_stride_b, in_stride_h, in_stride_t;
  int64_t out_stride_b, out_stride_h, out_stride_t;
  int32_t out_row_mode;
  const int32_t* out_positions;
  float key_sharpen;
  int32_t rotate;
  int32_t* error_flag;
  LayerIO layers[kMaxLayersPerLaunch];
};

struct DLayerIO {
  const uint8_t* k_codes;
  const uint8_t* v_codes;
  const uint16_t* k_scales;
  const uint16_t* v_scales;
  uint16_t* k_out;
  uint16_t* v_out;
  int32_t key_levels, value_levels;
};

struct DecompressArgs {
  int32_t batch, heads, n_tokens, head_dim, head_dim_padded;
  int32_t head_group;
  const int32_t* count;
  const int32_t* positions;
  const float* rope_cos;
  const float* rope_sin;
  int32_t rope_rows;  // positions are clamped to [0, rope_rows - 1] before indexing the tables
  int64_t out_stride_b, out_stride_h, out_stride_t;
  float key_sharpen;
  DLayerIO layers[kMaxLayersPerLaunch];
};

cudaError_t launch_compress(const CompressArgs& a, int n_layers, cudaStream_t s, bool recon);
cudaError_t launch_decompress(const DecompressArgs& a, int n_layers, cudaStream_t s);

// scoring (nq_score.cu)
struct ScoreArgs {
  const void* q;   // explicit queries, or nullptr for key-key (queries = last obs keys)
  const void* k;
  int32_t in_dtype;
  int32_t batch, q_heads, heads, n_q, seq, head_dim;
  int64_t q_stride_b, q_stride_h, q_stride_t;
  int64_t k_stride_b, k_stride_h, k_stride_t;
  int32_t causal;      // 1: key t visible to query i when t <= q_pos0 + i
  int32_t q_pos0;
  int32_t head_begin, head_end;  // query heads scored
  float scale;
};
size_t score_workspace_bytes(int batch, int n_heads, int n_q, int seq);
// Per-head column sums colsum[b, h - head_begin, t] into the workspace-backed buffer `colsum`.
// tcgen05 / TMEM path (nq_score_umma.cu) for fp16 / bf16 caches
bool score_umma_supported(const ScoreArgs& a);
cudaError_t launch_score_umma(const ScoreArgs& a, float* colsum, void* ws, cudaStream_t s);
cudaError_t launch_score_colsums(const ScoreArgs& a, float* colsum, void* ws, size_t ws_bytes, cudaStream_t s);
// out[b, t] (=|+=) weight * sum_h colsum[b, h, t] in head order.
cudaError_t launch_reduce_heads(const float* colsum, int batch, int n_heads, int seq, float weight, int accumulate,
                                float* out, cudaStream_t s);

// selection (nq_select.cu)
size_t select_workspace_bytes(int batch, int seq);
cudaError_t launch_select(const float* imp, int batch, int seq, int sliding_window, int n_keep,
                          const int32_t* prot, int n_prot, int32_t* kept_idx, int32_t* kept_count, void* ws,
                          cudaStream_t s);

// misc (nq_misc.cu)
cudaError_t launch_gather_rows(const void* in, int dtype, int batch, int heads, int head_dim, int64_t isb,
                               int64_t ish, int64_t ist, const int32_t* kept_idx, const int32_t* kept_count,
                               int n_kept, uint16_t* out, int64_t osb, int64_t osh, int64_t ost, cudaStream_t s);
cudaError_t launch_code_symbols(const uint8_t* codes, int64_t rows, int dp, int levels, int mode, int half,
                                unsigned int* counts, uint8_t* symbols, cudaStream_t s);
cudaError_t launch_delta(const uint8_t* codes, int n_streams, int n_tokens, int dp, int levels, int8_t* delta,
                         cudaStream_t s);

// compressed-domain decode attention (nq_attend.cu)
struct AttendArgs {
  int32_t batch, q_heads, heads, n_tokens, splits, tokens_per_split;
  const int32_t* count;
  const __half* q;
  int64_t q_stride_b, q_stride_h;
  const uint8_t* k_codes;
  const uint8_t* v_codes;
  const uint16_t* k_scales;
  const uint16_t* v_scales;
  const int32_t* positions;
  const float* rope_cos;
  const float* rope_sin;
  int32_t rope_rows;  // positions are clamped to [0, rope_rows - 1] before indexing the tables
  float key_sharpen, scale;
  float* ws_m;    // [b, hq, splits]
  float* ws_l;    // [b, hq, splits]
  float* ws_acc;  // [b, hq, splits, 128]
  __half* out;
  int64_t out_stride_b, out_stride_h;
};
int attend_splits(int batch, int heads, int n_tokens);
size_t attend_workspace_bytes(int batch, int q_heads, int splits);
cudaError_t attend_take_error(unsigned int* bits, cudaStream_t s);  // read and clear its wait-error word
cudaError_t launch_attend(const AttendArgs& a, int fmt_k, int fmt_v, void* ws, cudaStream_t s);

}  // namespace nq
