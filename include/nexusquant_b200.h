/*
 * nexusquant_b200.h -- C ABI of the B200 (sm_100a) KV-cache compression path.
 *
 * Drop-in replacement for the torch math behind NexusQuant's post-prefill
 * compression (jagmarques/nexusquant v0.5.0): the per-layer loops of
 * nexusquant/pipeline.py, nexusquant/core/{e8_lattice,hadamard,rope_utils}.py
 * and the Triton kernels of nexusquant/kernels/e8_triton.py.
 *
 * Conventions
 *   - All pointers are device pointers unless stated otherwise; sizes are in
 *     elements, strides in elements.  Tensors are [batch, heads, tokens, dim]
 *     with a unit innermost stride (the layout of a HuggingFace DynamicCache
 *     layer), addressed through (stride_b, stride_h, stride_t).
 *   - Every entry point is stream-ordered on `stream` (a cudaStream_t; NULL is
 *     the legacy default stream), returns an nq_status_t, never throws, and
 *     validates its arguments on the host before launching anything.
 *   - No entry point allocates device memory: scratch space is passed in by the
 *     caller, sized by the matching *_workspace_size() query.
 *   - Lattice codes are 2 * (E8 lattice point), integers in [-L, L] for L =
 *     2^bits levels (nexusquant/integrations/vllm_backend.py:309-315).  Packed
 *     formats per vector of d_p codes (d_p = head_dim rounded up to a power of 2):
 *       L <= 4 : nibbles, byte k = (c[2k] + 8) | (c[2k+1] + 8) << 4
 *                (vllm_backend.py:476-513, pack_codes_nibble);      d_p/2 bytes
 *       L == 8 : 5-bit fields c + 8, 8 codes per 5 bytes, little endian; 5*d_p/8
 *       L == 16: int8 codes (CompressedPage.key_codes, vllm_backend.py:79-85); d_p
 *   - Scales are fp16 bit patterns (CompressedPage.key_scales, vllm_backend.py:392).
 */
#ifndef NEXUSQUANT_B200_H
#define NEXUSQUANT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NQ_ABI_VERSION 2

typedef int32_t nq_status_t;
enum {
  NQ_OK = 0,
  NQ_ERR_INVALID_ARG = -1,   /* bad pointer, size, stride or level (reference: ValueError) */
  NQ_ERR_UNSUPPORTED = -2,   /* shape outside what the kernels support (e.g. head_dim > 128) */
  NQ_ERR_CUDA = -3,          /* a CUDA launch or query failed */
  NQ_ERR_TIMEOUT = -4,       /* a bounded device-side wait expired */
  NQ_ERR_WORKSPACE = -5,     /* workspace missing or smaller than *_workspace_size() */
  NQ_ERR_ALIGNMENT = -6,     /* a pointer or stride breaks the 16-byte alignment rule */
  NQ_ERR_TOO_LARGE = -7      /* problem needs more than the library's built-in scratch */
};

typedef enum { NQ_F16 = 0, NQ_BF16 = 1, NQ_F32 = 2 } nq_dtype_t;

typedef void *nq_stream_t; /* cudaStream_t */

/* Human-readable text for a status code (static storage). */
const char *nq_status_string(nq_status_t status);
/* NQ_ABI_VERSION of the loaded library. */
int32_t nq_abi_version(void);
/* Packed bytes of one vector of d_p codes at `levels` (2, 4, 8 or 16); -1 if unsupported. */
int32_t nq_packed_bytes(int32_t d_p, int32_t levels);

/*
 * Compress layers (all in one launch): inverse RoPE on keys (at each token's source position),
 * zero-pad head_dim to d_p, orthonormal Walsh-Hadamard transform, per-vector
 * scale amax/(L/2), relaxed-E8 nearest point per 8-group with the clamp to
 * [-L/2, L/2], then pack codes and store fp16 scales.  Optionally also writes
 * the fake-quantized fp16 reconstruction the reference pipelines write back.
 *
 * Replaces the per-layer loop body of NexusQuantEvict.compress
 * (nexusquant/pipeline.py:1190-1244), NexusQuantQuantOnly.compress
 * (pipeline.py:236-263), NexusQuantSimple.compress (pipeline.py:130-166),
 * NexusQuantEvictTruncate.compress (pipeline.py:1349-1399) and
 * NexusQuantKVCompressor.compress_page (vllm_backend.py:344-396), together with
 * E8Lattice.quantize_perhead (nexusquant/core/e8_lattice.py:97-124) and the
 * Triton e8_encode_kernel (nexusquant/kernels/e8_triton.py:238-324).
 */
/* Per-layer tensors of one compress call.  Any pointer may be NULL to skip
 * that output (or, for k / v, that half of the layer). */
typedef struct nq_layer_io {
  const void *k, *v;                /* [batch, heads, seq, head_dim] in in_dtype, strided */
  uint8_t *k_codes, *v_codes;       /* [batch, heads, n_kept, packed_bytes] */
  uint16_t *k_scales, *v_scales;    /* fp16 [batch, heads, n_kept] */
  float *k_scales_f32, *v_scales_f32; /* fp32 [batch, heads, n_kept] */
  uint16_t *k_out, *v_out;          /* fake-quant fp16 reconstruction (strided, see out_*) */
  int32_t key_levels, value_levels; /* 2, 4, 8 or 16 (2^bits) */
} nq_layer_io_t;

typedef struct nq_compress_params {
  int32_t batch, heads, seq;     /* layer shape (seq = tokens held by each layer) */
  int32_t head_dim;              /* d: 64, 96 or 128 */
  int32_t head_dim_padded;       /* d_p: power of two >= d (64 or 128) */
  int32_t n_kept;                /* tokens compressed per batch row */
  const int32_t *kept_idx;       /* [batch, n_kept] source token indices; NULL = 0..n_kept-1 */
  const int32_t *kept_count;     /* [batch] valid entries (<= n_kept); NULL = n_kept for every row */
  const int32_t *positions;      /* [batch, n_kept] RoPE positions of the kept tokens; NULL = token index */
  /* RoPE tables [rope_rows, head_dim/2] fp32, row p = cos / sin(p * inv_freq)
   * (nexusquant/core/rope_utils.py:106-112); required when any k is given. */
  const float *rope_cos;
  const float *rope_sin;
  int32_t rope_rows;
  int32_t in_dtype;              /* nq_dtype_t */
  int64_t in_stride_b, in_stride_h, in_stride_t;
  int64_t out_stride_b, out_stride_h, out_stride_t;   /* for k_out / v_out */
  int32_t out_row_mode;          /* 0: reconstruction row = source index (masked layout)
                                    1: row = j, keys re-encoded at position j (truncated layout,
                                       pipeline.py:1376-1388) */
  const int32_t *out_positions;  /* optional [batch, n_kept] re-encoding positions */
  float key_sharpen;             /* multiplies reconstructed keys (1.0 = off) */
  int32_t rotate;                /* 1: Walsh-Hadamard rotation (the pipelines' path);
                                    0: quantize the (RoPE-removed) rows as given, as
                                       E8Lattice.quantize_perhead does (e8_lattice.py:97-124) */
  int32_t inputs_host;           /* 0: k / v are device memory.  1: k / v are pinned host memory
                                    mapped into the device address space (UVA: the host pointer
                                    is the device pointer); the kernel then reads only the kept
                                    rows across PCIe.  Checked with cudaPointerGetAttributes:
                                    anything else returns NQ_ERR_INVALID_ARG. */
  int32_t *error_flag;           /* optional device int32; unused: the compress kernels have no
                                    device-side waits.  Expired waits of the scorer are reported
                                    by nq_device_error(). */
  const nq_layer_io_t *layers;   /* HOST array [n_layers] */
  int32_t n_layers;
} nq_compress_params_t;

nq_status_t nq_compress_layers(const nq_compress_params_t *params, nq_stream_t stream);

/*
 * Dequantize layers from the compressed layout: unpack -> code * 0.5 * scale
 * -> inverse Walsh-Hadamard -> (keys) RoPE at the stored positions -> optional
 * key sharpening -> fp16.
 *
 * Replaces NexusQuantKVCompressor.decompress_page (vllm_backend.py:398-429) and
 * _dequantize_perhead (vllm_backend.py:319-338), and the Triton
 * e8_decode_kernel (nexusquant/kernels/e8_triton.py:331-355).
 */
typedef struct nq_dlayer_io {
  const uint8_t *k_codes, *v_codes;     /* either may be NULL */
  const uint16_t *k_scales, *v_scales;  /* fp16 */
  uint16_t *k_out, *v_out;              /* fp16 [batch, heads, n_tokens, head_dim] (strided) */
  int32_t key_levels, value_levels;
} nq_dlayer_io_t;

typedef struct nq_decompress_params {
  int32_t batch, heads, n_tokens;  /* compressed rows per (batch, head) */
  int32_t head_dim, head_dim_padded;
  const int32_t *count;            /* [batch] valid rows; NULL = n_tokens */
  const int32_t *positions;        /* [batch, n_tokens] RoPE positions (required for keys) */
  const float *rope_cos, *rope_sin;
  int32_t rope_rows;
  int64_t out_stride_b, out_stride_h, out_stride_t;
  float key_sharpen;               /* 1.0 or sqrt(1.05) (README.md:75; paper section 3.6) */
  const nq_dlayer_io_t *layers;    /* HOST array [n_layers] */
  int32_t n_layers;
} nq_decompress_params_t;

nq_status_t nq_decompress_layers(const nq_decompress_params_t *params, nq_stream_t stream);


/*
 * Key-key token importance (SnapKV-style proxy): the last min(obs_window, seq)
 * keys of each head attend, without a mask and with scale head_dim^-1/2, to all
 * `seq` keys; the importance of token t is the softmax column sum over those
 * queries, averaged over heads.  Replaces NexusQuantEvict._score_importance
 * (nexusquant/pipeline.py:756-782).
 *   per_head == 0: out[batch, seq]  = (sum over h in [head_begin, head_end) of colsum_h) / heads
 *   per_head == 1: out[batch, head_end - head_begin, seq] = colsum_h
 * (A rank of a multi-GPU job scores its head range with per_head = 1; after an
 * all-gather, nq_reduce_heads forms the same mean on every rank.)
 */
nq_status_t nq_score_keykey(const void *k, int32_t in_dtype, int32_t batch, int32_t heads, int32_t seq,
                            int32_t head_dim, int64_t stride_b, int64_t stride_h, int64_t stride_t,
                            int32_t obs_window, int32_t head_begin, int32_t head_end, int32_t per_head,
                            float *out, void *workspace, size_t workspace_bytes, nq_stream_t stream);
/* Workspace for nq_score_keykey over `heads` scored heads. */
size_t nq_score_keykey_workspace_size(int32_t batch, int32_t heads, int32_t seq, int32_t obs_window);

/*
 * Real-attention importance from explicit queries: q [batch, q_heads, n_q, d]
 * at positions q_pos0 .. q_pos0 + n_q - 1 attend causally (key t visible when
 * t <= position) to k [batch, heads, seq, d]; q_heads is a multiple of heads
 * (grouped-query layout, query head i reads key head i / (q_heads / heads)).
 *   importance[b, t] (=, or += when accumulate) mean over query heads of the
 *   softmax column sums.
 * One call per layer with accumulate = 1, then dividing by the layer count, is
 * NexusQuantEvict._score_importance_real (nexusquant/pipeline.py:784-836)
 * restated on synthetic queries.
 */
nq_status_t nq_score_attention(const void *q, const void *k, int32_t in_dtype, int32_t batch, int32_t q_heads,
                               int32_t heads, int32_t n_q, int32_t seq, int32_t head_dim, int64_t q_stride_b,
                               int64_t q_stride_h, int64_t q_stride_t, int64_t k_stride_b, int64_t k_stride_h,
                               int64_t k_stride_t, int32_t q_pos0, int32_t accumulate, float *importance,
                               void *workspace, size_t workspace_bytes, nq_stream_t stream);
size_t nq_score_attention_workspace_size(int32_t batch, int32_t q_heads, int32_t n_q, int32_t seq);

/*
 * nq_score_keykey without any scratch from the caller or from cudaMalloc.
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory when they score (inside an allocator or memory pool that must not be
 * re-entered, engines that pre-reserve all device memory, bindings without a
 * cudaMalloc): the scratch is a fixed array inside this library, of
 * NQ_NOALLOC_SCRATCH_BYTES per GPU, held from load until exit.  Same arguments
 * and results as nq_score_keykey minus the workspace.  Returns NQ_ERR_TOO_LARGE
 * when the problem needs more scratch than that: roughly
 * batch * (head_end - head_begin) * seq * (4 + 8 * min(obs_window, seq) / 128)
 * bytes (without the first term when per_head = 1); 8 MiB covers one 128K-token,
 * 8-head layer.  The first call on a device looks up the array's address with
 * that device current; make it before any stream capture.  All calls on a device
 * share the array: calls that overlap on the GPU race and must be serialised.
 */
#define NQ_NOALLOC_SCRATCH_BYTES (8u << 20)
nq_status_t nq_score_keykey_noalloc(const void *k, int32_t in_dtype, int32_t batch, int32_t heads, int32_t seq,
                                    int32_t head_dim, int64_t stride_b, int64_t stride_h, int64_t stride_t,
                                    int32_t obs_window, int32_t head_begin, int32_t head_end, int32_t per_head,
                                    float *out, nq_stream_t stream);

/*
 * out[b, t] (=, or += when accumulate) (sum over h = 0 .. heads-1, in order, of
 * per_head[b, h, t]) / divisor.  The head mean of pipeline.py:781 and :834.
 */
nq_status_t nq_reduce_heads(const float *per_head, int32_t batch, int32_t heads, int32_t seq, float divisor,
                            int32_t accumulate, float *out, nq_stream_t stream);

/*
 * Keep set: BOS, the last `sliding_window` tokens, the top-n_keep tokens of
 * importance[b, 1 : seq - sliding_window] (ties toward the lower index) and the
 * sorted `protected_pos` list.  Writes the kept token indices in ascending
 * order to kept_idx[b, :] and their number to kept_count[b].
 * Replaces NexusQuantEvict._build_keep_mask (nexusquant/pipeline.py:895-959).
 * n_keep is max(1, int(prefix * (1.0 - rate))) computed by the caller in IEEE
 * double (pipeline.py:918-920).
 */
nq_status_t nq_select_keep(const float *importance, int32_t batch, int32_t seq, int32_t sliding_window,
                           int32_t n_keep, const int32_t *protected_pos, int32_t n_protected,
                           int32_t *kept_idx, int32_t *kept_count, void *workspace, size_t workspace_bytes,
                           nq_stream_t stream);
size_t nq_select_keep_workspace_size(int32_t batch, int32_t seq);

/*
 * Gather kept rows of a boundary-protected layer into fp16 (no quantization):
 * out[b, h, j, :] = in[b, h, kept_idx[b, j], :].
 * Replaces the protected-layer branch of NexusQuantEvict.compress
 * (nexusquant/pipeline.py:1206-1210) and NexusQuantEvictTruncate.compress
 * (pipeline.py:1363-1368).
 */
nq_status_t nq_gather_rows(const void *in, int32_t in_dtype, int32_t batch, int32_t heads, int32_t head_dim,
                           int64_t in_stride_b, int64_t in_stride_h, int64_t in_stride_t, const int32_t *kept_idx,
                           const int32_t *kept_count, int32_t n_kept, uint16_t *out, int64_t out_stride_b,
                           int64_t out_stride_h, int64_t out_stride_t, nq_stream_t stream);

/*
 * Temporal delta of lattice codes along tokens, per (batch, head) stream:
 * delta[.., 0, :] = code[.., 0, :], delta[.., t, :] = code[.., t, :] - code[.., t-1, :]
 * as int8, from packed codes [streams, n_tokens, packed_bytes].
 * Replaces temporal_delta_encode (nexusquant/core/temporal_codec.py:30-52) and
 * the delta step of compression_accounting._compress_with_delta_zstd
 * (nexusquant/core/compression_accounting.py:49-62).
 */
nq_status_t nq_delta_codes(const uint8_t *codes, int32_t n_streams, int32_t n_tokens, int32_t head_dim_padded,
                           int32_t levels, int8_t *delta, nq_stream_t stream);

/*
 * rANS entropy coding of the lattice codes (nexusquant/core/entropy_coder.py), split as the
 * work splits: the symbol and frequency pass over every code runs on the device, only the
 * inherently serial state loop on the host.
 *   nq_code_histogram: counts[c + L] += number of codes equal to c, c in [-L, L] (2L + 1
 *     device uint32 bins, accumulated: zero them first).  An odd code means the stream has
 *     half-integer lattice coordinates (_lattice_to_symbols, entropy_coder.py:35-75).
 *   nq_code_symbols: uint8 symbols [rows, d_p] (8-byte aligned), c + L when half != 0 (alphabet
 *     2L + 1), else c / 2 + L / 2 (alphabet L + 1) -- the reference's shift of doubled or
 *     integer coordinates.
 *   nq_rans_encode / nq_rans_decode (HOST pointers, host code): the reference's 32-bit-state,
 *     16-bit-word rANS with a 12-bit frequency table summing to 4096 (_rans_encode /
 *     _rans_decode, entropy_coder.py:246-345); words in stream order, *out_len words written,
 *     NQ_ERR_TOO_LARGE when out_cap is too small (n + 2 words always suffice).
 */
nq_status_t nq_code_histogram(const uint8_t *codes, int64_t rows, int32_t head_dim_padded, int32_t levels,
                              uint32_t *counts, nq_stream_t stream);
nq_status_t nq_code_symbols(const uint8_t *codes, int64_t rows, int32_t head_dim_padded, int32_t levels,
                            int32_t half, uint8_t *symbols, nq_stream_t stream);
nq_status_t nq_rans_encode(const uint8_t *symbols, int64_t n, const uint32_t *freqs, int32_t alphabet,
                           uint16_t *out, int64_t out_cap, int64_t *out_len);
nq_status_t nq_rans_decode(const uint16_t *words, int64_t n_words, int64_t n, const uint32_t *freqs,
                           int32_t alphabet, uint8_t *symbols);

/*
 * Decode attention straight from the compressed layout: one query token per sequence,
 * softmax(q K^T * scale) V with K / V dequantized on the fly as nq_decompress_layers
 * would (keys re-rotated at their positions, sharpened, rounded to fp16), fp16 output.
 * Replaces NexusQuantPagedAttention.forward (vllm_backend.py:692-765), which
 * decompresses every page to fp16 first.  head_dim = head_dim_padded = 128; query head
 * g*G + i attends KV head g, G = q_heads / heads in {1, 2, 4, 8}; a sequence with
 * count 0 gets a zero output, as in the reference.  Both contractions run on the tensor cores
 * (fp16 operands, fp32 accumulation): the fp16 keys against the fp16 queries, and the value
 * codes (exact in fp16) against the softmax weights times the value scales rounded to fp16;
 * the result agrees with dequantize-then-attend within rel-L2 1e-3.
 */
typedef struct {
  int32_t batch, q_heads, heads, head_dim, head_dim_padded, n_tokens;
  const int32_t *count;          /* [batch] valid tokens (<= n_tokens); NULL = n_tokens */
  const uint16_t *q;             /* fp16 [batch, q_heads, head_dim], row stride 1 */
  int64_t q_stride_b, q_stride_h;
  const uint8_t *k_codes, *v_codes;      /* [batch, heads, n_tokens, packed bytes] */
  const uint16_t *k_scales, *v_scales;   /* fp16 [batch, heads, n_tokens] */
  int32_t key_levels, value_levels;
  const int32_t *positions;      /* [batch, n_tokens] RoPE positions of the stored keys */
  const float *rope_cos, *rope_sin;  /* [rope_rows, head_dim/2], as for nq_compress_layers */
  int32_t rope_rows;
  float key_sharpen;             /* 1.0 = off */
  float scale;                   /* logit scale; 0 = 1/sqrt(head_dim) as the reference */
  uint16_t *out;                 /* fp16 [batch, q_heads, head_dim], row stride 1 */
  int64_t out_stride_b, out_stride_h;
} nq_attend_params_t;

size_t nq_attend_compressed_workspace_size(int32_t batch, int32_t q_heads, int32_t heads, int32_t n_tokens);
nq_status_t nq_attend_compressed(const nq_attend_params_t *params, void *workspace, size_t workspace_bytes,
                                 nq_stream_t stream);

/*
 * Merge eviction, the value merging of NexusQuantEvict(merge_eviction=True)
 * (nexusquant/pipeline.py:961-1048, called at :1186-1187 before hard eviction).  Four
 * stream-ordered steps per batch element, all on device memory:
 *
 *   nq_merge_centroid_accumulate  centroid_sum[t, :] (+)= mean over heads of V_l[h, t, :] for
 *                                 each given layer in order (accumulate = 0 starts the sum with
 *                                 the first layer).  values: host array of n_layers device
 *                                 pointers, each [heads, seq, head_dim] of one batch element with
 *                                 strides (stride_h, stride_t, 1) in elements; 16-byte aligned.
 *   nq_merge_centroid_normalize   unit_rows = (centroid_sum / n_layers) / max(||.||, 1e-12) per row
 *                                 (pipeline.py:1013-1020); unit_rows may alias centroid_sum.
 *   nq_merge_nearest              nearest[i] = argmax_j unit[evict_pos[i]] . unit[kept_pos[j]],
 *                                 first j on ties (pipeline.py:1023-1024); head_dim a multiple of
 *                                 32, at most 256.
 *   nq_merge_apply                for each j with seg_start[j] < seg_start[j+1]:
 *                                 V_l[h, kept_pos[j], :] += w * V_l[h, e, :] for e in
 *                                 seg_evicted[seg_start[j] .. seg_start[j+1]) in that order,
 *                                 w = fp32(imp[e] / (imp[s] + imp[e] + 1e-8)) in double, product
 *                                 and sum rounded to fp32, stored once in the cache dtype
 *                                 (pipeline.py:1026-1048).  In place; importance is fp32 [seq].
 */
nq_status_t nq_merge_centroid_accumulate(const void *const *values, int32_t n_layers, int32_t dtype, int32_t heads,
                                         int32_t seq, int32_t head_dim, int64_t stride_h, int64_t stride_t,
                                         int32_t accumulate, float *centroid_sum, nq_stream_t stream);
nq_status_t nq_merge_centroid_normalize(const float *centroid_sum, int32_t seq, int32_t head_dim,
                                        int32_t n_layers, float *unit_rows, nq_stream_t stream);
/* Same result as nq_merge_nearest for head_dim 128 and rows of norm <= 1 + 1e-6 (what
 * nq_merge_centroid_normalize writes); no counterpart in the reference.  The similarities are
 * screened on the tensor cores (tf32, fp32 accumulation) keeping every column within 0.005 of
 * the row maximum (more than twice the tf32 error bound for unit rows); those candidates are
 * re-computed in the exact kernel's fp32 order, so the chosen indices are identical.  Rows that
 * run out of candidate slots, contain NaN or are not unit rows fall back to the exact scan. */
nq_status_t nq_merge_nearest_unit(const float *unit_rows, int32_t head_dim, const int32_t *evict_pos,
                                  int32_t n_evict, const int32_t *kept_pos, int32_t n_kept, int32_t *nearest,
                                  nq_stream_t stream);
nq_status_t nq_merge_nearest(const float *unit_rows, int32_t head_dim, const int32_t *evict_pos, int32_t n_evict,
                             const int32_t *kept_pos, int32_t n_kept, int32_t *nearest, nq_stream_t stream);
nq_status_t nq_merge_apply(const void *const *values, int32_t n_layers, int32_t dtype, int32_t heads, int32_t seq,
                           int32_t head_dim, int64_t stride_h, int64_t stride_t, const float *importance,
                           const int32_t *kept_pos, int32_t n_kept, const int32_t *seg_start,
                           const int32_t *seg_evicted, nq_stream_t stream);

/*
 * Byte layouts of the paged interface (nexusquant/integrations/vllm_backend.py):
 *   nq_unpack_codes    packed lattice codes [rows, nq_packed_bytes(d_p, levels)] -> int8
 *                      [rows, d_p] with code = 2 x lattice point, the layout of
 *                      CompressedPage.key_codes / value_codes (vllm_backend.py:73-101).
 *                      codes must be 8-byte aligned.
 *   nq_pack_nibbles    NexusQuantKVCompressor.pack_codes_nibble (vllm_backend.py:476-513):
 *                      int8 [rows, d] -> uint8 [rows, (d + 1) / 2], byte k = clamp(c[2k] + 8)
 *                      | clamp(c[2k+1] + 8) << 4 (clamp to [0, 15]; an odd d pads a 0 nibble).
 *   nq_unpack_nibbles  unpack_codes_nibble (vllm_backend.py:515-540): the inverse, nibble - 8.
 * Replace the reference's torch byte manipulation on the page path; one pass each.
 */
nq_status_t nq_unpack_codes(const uint8_t *packed, int64_t rows, int32_t head_dim_padded, int32_t levels,
                            int8_t *codes, nq_stream_t stream);
nq_status_t nq_pack_nibbles(const int8_t *codes, int64_t rows, int32_t d, uint8_t *packed, nq_stream_t stream);
nq_status_t nq_unpack_nibbles(const uint8_t *packed, int64_t rows, int32_t d, int8_t *codes, nq_stream_t stream);

/*
 * Device-side failure reporting (no counterpart in the reference, which has no device code).
 *
 * Every device-side wait in this library (the tensor-core scorer's waits on TMA and MMA
 * completion, the decode attention's waits on MMA completion) has an iteration limit.  A wait
 * that runs out makes its kernel stop early, release what it holds and OR a bit into a
 * per-device error word; the scores or outputs it leaves are then not valid.  nq_device_error synchronizes `stream`, stores the word in *bits (if bits is
 * not NULL), clears it, and returns NQ_ERR_TIMEOUT if any bit was set, else NQ_OK.
 * Bits: 1 = scorer wait, 2 = nq_wait_selftest, 4 = decode attention wait.
 */
nq_status_t nq_device_error(int32_t *bits, nq_stream_t stream);
/* Test hook: one CTA waits on an mbarrier that nothing arrives on, for max_iters (1..2^20)
 * tries, then records the expiry (bit 2) -- the failure path without any copy in flight. */
nq_status_t nq_wait_selftest(uint32_t max_iters, nq_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* NEXUSQUANT_B200_H */
