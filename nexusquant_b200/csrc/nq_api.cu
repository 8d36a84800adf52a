// extern "C" entry points of libnexusquant_b200.so (declared in include/nexusquant_b200.h).
// Every function validates its arguments on the host, launches stream-ordered
// work, never throws and never allocates device memory.
#include <cmath>
#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/nexusquant_b200.h"
#include "nq_internal.h"

namespace {

using nq::kMaxLayersPerLaunch;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool valid_levels(int l) { return l == 2 || l == 4 || l == 8 || l == 16; }
int elem_bytes(int dtype) { return dtype == NQ_F32 ? 4 : 2; }
bool supported_dims(int d, int dp) { return (d == 128 && dp == 128) || (d == 96 && dp == 128) || (d == 64 && dp == 64); }

int head_group_for(int heads) {
  int hg = 1;
  while (hg * 2 <= heads && hg < 8) hg *= 2;
  return hg;
}

nq_status_t cuda_status(cudaError_t e) { return e == cudaSuccess ? NQ_OK : NQ_ERR_CUDA; }

}  // namespace

extern "C" {

const char* nq_status_string(nq_status_t s) {
  switch (s) {
    case NQ_OK: return "ok";
    case NQ_ERR_INVALID_ARG: return "invalid argument";
    case NQ_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case NQ_ERR_CUDA: return "CUDA error";
    case NQ_ERR_TIMEOUT: return "device-side wait timed out";
    case NQ_ERR_WORKSPACE: return "workspace missing or too small";
    case NQ_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case NQ_ERR_TOO_LARGE: return "problem exceeds the library's built-in scratch size";
  }
  return "unknown status";
}

int32_t nq_abi_version(void) { return NQ_ABI_VERSION; }

int32_t nq_packed_bytes(int32_t d_p, int32_t levels) {
  if (!valid_levels(levels) || d_p <= 0 || (d_p & 7)) return -1;
  return levels <= 4 ? d_p / 2 : (levels == 8 ? d_p * 5 / 8 : d_p);
}

nq_status_t nq_compress_layers(const nq_compress_params_t* p, nq_stream_t stream) {
  if (!p || !p->layers || p->n_layers < 0) return NQ_ERR_INVALID_ARG;
  if (p->batch < 0 || p->heads < 0 || p->seq < 0 || p->n_kept < 0) return NQ_ERR_INVALID_ARG;
  if (p->in_dtype < 0 || p->in_dtype > 2) return NQ_ERR_INVALID_ARG;
  if (!supported_dims(p->head_dim, p->head_dim_padded)) return NQ_ERR_UNSUPPORTED;
  if (p->kept_idx == nullptr && p->n_kept > p->seq) return NQ_ERR_INVALID_ARG;
  if (p->n_layers == 0 || p->batch == 0 || p->heads == 0 || p->n_kept == 0) return NQ_OK;
  const int eb = elem_bytes(p->in_dtype);
  // 16-byte cp.async copies need 16-byte aligned rows
  if ((p->in_stride_b * eb) % 16 || (p->in_stride_h * eb) % 16 || (p->in_stride_t * eb) % 16) return NQ_ERR_ALIGNMENT;
  if ((p->out_stride_b * 2) % 16 || (p->out_stride_h * 2) % 16 || (p->out_stride_t * 2) % 16) return NQ_ERR_ALIGNMENT;
  bool any_key = false, any_out = false;
  for (int l = 0; l < p->n_layers; ++l) {
    const nq_layer_io_t& L = p->layers[l];
    if (L.k && !valid_levels(L.key_levels)) return NQ_ERR_INVALID_ARG;
    if (L.v && !valid_levels(L.value_levels)) return NQ_ERR_INVALID_ARG;
    const void* ptrs[] = {L.k, L.v, L.k_codes, L.v_codes, L.k_out, L.v_out};
    for (const void* q : ptrs)
      if (q && !aligned16(q)) return NQ_ERR_ALIGNMENT;
    if ((L.k_codes && !L.k) || (L.v_codes && !L.v)) return NQ_ERR_INVALID_ARG;
    if (p->inputs_host) {
      // host-resident layers must be pinned and mapped at the same address (UVA)
      for (const void* q : {L.k, L.v}) {
        if (!q) continue;
        cudaPointerAttributes at;
        if (cudaPointerGetAttributes(&at, q) != cudaSuccess || at.type != cudaMemoryTypeHost ||
            at.devicePointer != q) {
          cudaGetLastError();
          return NQ_ERR_INVALID_ARG;
        }
      }
    }
    any_key |= (L.k != nullptr);
    any_out |= (L.k_out || L.v_out);
  }
  if (any_key && (!p->rope_cos || !p->rope_sin || p->rope_rows <= 0)) return NQ_ERR_INVALID_ARG;
  if (!aligned16(p->rope_cos) || !aligned16(p->rope_sin)) return NQ_ERR_ALIGNMENT;
  if (((p->head_dim / 2) * 4) % 16) return NQ_ERR_ALIGNMENT;

  nq::CompressArgs a;
  std::memset(&a, 0, sizeof(a));
  a.batch = p->batch; a.heads = p->heads; a.seq = p->seq;
  a.head_dim = p->head_dim; a.head_dim_padded = p->head_dim_padded; a.n_kept = p->n_kept;
  a.head_group = head_group_for(p->heads);
  a.kept_idx = p->kept_idx; a.kept_count = p->kept_count; a.positions = p->positions;
  a.rope_cos = p->rope_cos; a.rope_sin = p->rope_sin; a.rope_rows = p->rope_rows;
  a.in_dtype = p->in_dtype;
  a.in_stride_b = p->in_stride_b; a.in_stride_h = p->in_stride_h; a.in_stride_t = p->in_stride_t;
  a.out_stride_b = p->out_stride_b; a.out_stride_h = p->out_stride_h; a.out_stride_t = p->out_stride_t;
  a.out_row_mode = p->out_row_mode; a.out_positions = p->out_positions;
  a.key_sharpen = p->key_sharpen == 0.0f ? 1.0f : p->key_sharpen;
  a.rotate = p->rotate;
  a.error_flag = p->error_flag;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // one launch per (key level count, value level count) group of layers (the kernels are
  // specialised on the level count), at most kMaxLayersPerLaunch layers each
  auto group_key = [&](int l) {
    const nq_layer_io_t& L = p->layers[l];
    return (L.k ? L.key_levels : 0) * 32 + (L.v ? L.value_levels : 0);
  };
  std::vector<int> order(p->n_layers);
  for (int l = 0; l < p->n_layers; ++l) order[l] = l;
  std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return group_key(x) < group_key(y); });
  for (int l0 = 0; l0 < p->n_layers;) {
    const int key0 = group_key(order[l0]);
    int n = 0;
    while (l0 + n < p->n_layers && n < kMaxLayersPerLaunch && group_key(order[l0 + n]) == key0) ++n;
    for (int i = 0; i < n; ++i) {
      const nq_layer_io_t& L = p->layers[order[l0 + i]];
      nq::LayerIO& d = a.layers[i];
      d.k = L.k; d.v = L.v; d.k_codes = L.k_codes; d.v_codes = L.v_codes;
      d.k_scales = L.k_scales; d.v_scales = L.v_scales;
      d.k_scales_f32 = L.k_scales_f32; d.v_scales_f32 = L.v_scales_f32;
      d.k_out = L.k_out; d.v_out = L.v_out;
      d.key_levels = L.key_levels; d.value_levels = L.value_levels;
    }
    const nq_status_t st = cuda_status(nq::launch_compress(a, n, s, any_out));
    if (st != NQ_OK) return st;
    l0 += n;
  }
  return NQ_OK;
}

nq_status_t nq_decompress_layers(const nq_decompress_params_t* p, nq_stream_t stream) {
  if (!p || !p->layers || p->n_layers < 0) return NQ_ERR_INVALID_ARG;
  if (p->batch < 0 || p->heads < 0 || p->n_tokens < 0) return NQ_ERR_INVALID_ARG;
  if (!supported_dims(p->head_dim, p->head_dim_padded)) return NQ_ERR_UNSUPPORTED;
  if (p->n_layers == 0 || p->batch == 0 || p->heads == 0 || p->n_tokens == 0) return NQ_OK;
  if ((p->out_stride_b * 2) % 16 || (p->out_stride_h * 2) % 16 || (p->out_stride_t * 2) % 16) return NQ_ERR_ALIGNMENT;
  bool any_key = false;
  for (int l = 0; l < p->n_layers; ++l) {
    const nq_dlayer_io_t& L = p->layers[l];
    if (L.k_codes && (!valid_levels(L.key_levels) || !L.k_scales || !L.k_out)) return NQ_ERR_INVALID_ARG;
    if (L.v_codes && (!valid_levels(L.value_levels) || !L.v_scales || !L.v_out)) return NQ_ERR_INVALID_ARG;
    const void* ptrs[] = {L.k_codes, L.v_codes, L.k_out, L.v_out};
    for (const void* q : ptrs)
      if (q && !aligned16(q)) return NQ_ERR_ALIGNMENT;
    any_key |= (L.k_codes != nullptr);
  }
  if (any_key && (!p->positions || !p->rope_cos || !p->rope_sin || p->rope_rows <= 0)) return NQ_ERR_INVALID_ARG;
  nq::DecompressArgs a;
  std::memset(&a, 0, sizeof(a));
  a.batch = p->batch; a.heads = p->heads; a.n_tokens = p->n_tokens;
  a.head_dim = p->head_dim; a.head_dim_padded = p->head_dim_padded;
  a.head_group = head_group_for(p->heads);
  a.count = p->count; a.positions = p->positions;
  a.rope_cos = p->rope_cos; a.rope_sin = p->rope_sin; a.rope_rows = p->rope_rows;
  a.out_stride_b = p->out_stride_b; a.out_stride_h = p->out_stride_h; a.out_stride_t = p->out_stride_t;
  a.key_sharpen = p->key_sharpen == 0.0f ? 1.0f : p->key_sharpen;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int l0 = 0; l0 < p->n_layers; l0 += kMaxLayersPerLaunch) {
    const int n = std::min(kMaxLayersPerLaunch, p->n_layers - l0);
    for (int i = 0; i < n; ++i) {
      const nq_dlayer_io_t& L = p->layers[l0 + i];
      nq::DLayerIO& d = a.layers[i];
      d.k_codes = L.k_codes; d.v_codes = L.v_codes; d.k_scales = L.k_scales; d.v_scales = L.v_scales;
      d.k_out = L.k_out; d.v_out = L.v_out; d.key_levels = L.key_levels; d.value_levels = L.value_levels;
    }
    const nq_status_t st = cuda_status(nq::launch_decompress(a, n, s));
    if (st != NQ_OK) return st;
  }
  return NQ_OK;
}

size_t nq_score_keykey_workspace_size(int32_t batch, int32_t heads, int32_t seq, int32_t obs_window) {
  if (batch <= 0 || heads <= 0 || seq <= 0) return 0;
  const int obs = std::min(obs_window, seq);
  return nq::score_workspace_bytes(batch, heads, obs, seq) + (size_t)batch * heads * seq * sizeof(float) + 256;
}

static nq_status_t score_common(const nq::ScoreArgs& a, int per_head, float divisor, int accumulate, float* out,
                                void* ws, size_t ws_bytes, size_t need, cudaStream_t s) {
  if (!ws || ws_bytes < need) return NQ_ERR_WORKSPACE;
  const int Hr = a.head_end - a.head_begin;
  const size_t sbytes = nq::score_workspace_bytes(a.batch, Hr, a.n_q, a.seq);
  float* colsum = per_head ? out
                           : reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(ws) + sbytes + 255) & ~uintptr_t(255));
  cudaError_t e = nq::launch_score_colsums(a, colsum, ws, sbytes, s);
  if (e != cudaSuccess) return NQ_ERR_CUDA;
  if (!per_head) e = nq::launch_reduce_heads(colsum, a.batch, Hr, a.seq, divisor, accumulate, out, s);
  return cuda_status(e);
}

nq_status_t nq_score_keykey(const void* k, int32_t in_dtype, int32_t batch, int32_t heads, int32_t seq,
                            int32_t head_dim, int64_t stride_b, int64_t stride_h, int64_t stride_t,
                            int32_t obs_window, int32_t head_begin, int32_t head_end, int32_t per_head,
                            float* out, void* workspace, size_t workspace_bytes, nq_stream_t stream) {
  if (!k || !out || batch < 0 || heads <= 0 || seq < 0 || obs_window <= 0) return NQ_ERR_INVALID_ARG;
  if (in_dtype < 0 || in_dtype > 2) return NQ_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 96 && head_dim != 128) return NQ_ERR_UNSUPPORTED;
  if (head_begin < 0 || head_end > heads || head_begin >= head_end) return NQ_ERR_INVALID_ARG;
  if (batch == 0 || seq == 0) return NQ_OK;
  nq::ScoreArgs a;
  std::memset(&a, 0, sizeof(a));
  a.q = nullptr; a.k = k; a.in_dtype = in_dtype;
  a.batch = batch; a.q_heads = heads; a.heads = heads; a.n_q = std::min(obs_window, seq); a.seq = seq;
  a.head_dim = head_dim;
  a.k_stride_b = stride_b; a.k_stride_h = stride_h; a.k_stride_t = stride_t;
  a.causal = 0; a.q_pos0 = 0; a.head_begin = head_begin; a.head_end = head_end;
  a.scale = static_cast<float>(std::pow(static_cast<double>(head_dim), -0.5));
  const size_t need = nq_score_keykey_workspace_size(batch, head_end - head_begin, seq, obs_window);
  return score_common(a, per_head, static_cast<float>(heads), 0, out, workspace, workspace_bytes, need,
                      static_cast<cudaStream_t>(stream));
}

size_t nq_score_attention_workspace_size(int32_t batch, int32_t q_heads, int32_t n_q, int32_t seq) {
  if (batch <= 0 || q_heads <= 0 || seq <= 0 || n_q <= 0) return 0;
  return nq::score_workspace_bytes(batch, q_heads, n_q, seq) + (size_t)batch * q_heads * seq * sizeof(float) + 256;
}

nq_status_t nq_score_attention(const void* q, const void* k, int32_t in_dtype, int32_t batch, int32_t q_heads,
                               int32_t heads, int32_t n_q, int32_t seq, int32_t head_dim, int64_t q_stride_b,
                               int64_t q_stride_h, int64_t q_stride_t, int64_t k_stride_b, int64_t k_stride_h,
                               int64_t k_stride_t, int32_t q_pos0, int32_t accumulate, float* importance,
                               void* workspace, size_t workspace_bytes, nq_stream_t stream) {
  if (!q || !k || !importance || batch < 0 || heads <= 0 || q_heads <= 0 || n_q <= 0 || seq < 0)
    return NQ_ERR_INVALID_ARG;
  if (q_heads % heads) return NQ_ERR_INVALID_ARG;
  if (in_dtype < 0 || in_dtype > 2) return NQ_ERR_INVALID_ARG;
  if (head_dim != 64 && head_dim != 96 && head_dim != 128) return NQ_ERR_UNSUPPORTED;
  if (q_pos0 < 0) return NQ_ERR_INVALID_ARG;
  if (batch == 0 || seq == 0) return NQ_OK;
  nq::ScoreArgs a;
  std::memset(&a, 0, sizeof(a));
  a.q = q; a.k = k; a.in_dtype = in_dtype;
  a.batch = batch; a.q_heads = q_heads; a.heads = heads; a.n_q = n_q; a.seq = seq; a.head_dim = head_dim;
  a.q_stride_b = q_stride_b; a.q_stride_h = q_stride_h; a.q_stride_t = q_stride_t;
  a.k_stride_b = k_stride_b; a.k_stride_h = k_stride_h; a.k_stride_t = k_stride_t;
  a.causal = 1; a.q_pos0 = q_pos0; a.head_begin = 0; a.head_end = q_heads;
  a.scale = static_cast<float>(std::pow(static_cast<double>(head_dim), -0.5));
  const size_t need = nq_score_attention_workspace_size(batch, q_heads, n_q, seq);
  return score_common(a, 0, static_cast<float>(q_heads), accumulate, importance, workspace, workspace_bytes, need,
                      static_cast<cudaStream_t>(stream));
}

nq_status_t nq_reduce_heads(const float* per_head, int32_t batch, int32_t heads, int32_t seq, float divisor,
                            int32_t accumulate, float* out, nq_stream_t stream) {
  if (!per_head || !out || batch < 0 || heads <= 0 || seq < 0 || !(divisor > 0.0f)) return NQ_ERR_INVALID_ARG;
  return cuda_status(
      nq::launch_reduce_heads(per_head, batch, heads, seq, divisor, accumulate, out, static_cast<cudaStream_t>(stream)));
}

size_t nq_select_keep_workspace_size(int32_t batch, int32_t seq) { return nq::select_workspace_bytes(batch, seq); }

nq_status_t nq_select_keep(const float* importance, int32_t batch, int32_t seq, int32_t sliding_window,
                           int32_t n_keep, const int32_t* protected_pos, int32_t n_protected, int32_t* kept_idx,
                           int32_t* kept_count, void* workspace, size_t workspace_bytes, nq_stream_t stream) {
  if (!importance || !kept_idx || !kept_count || batch < 0 || seq < 0 || sliding_window < 0 || n_keep < 0)
    return NQ_ERR_INVALID_ARG;
  if (n_protected < 0 || (n_protected > 0 && !protected_pos)) return NQ_ERR_INVALID_ARG;
  if (workspace_bytes < nq::select_workspace_bytes(batch, seq)) return NQ_ERR_WORKSPACE;
  if (batch == 0) return NQ_OK;
  return cuda_status(nq::launch_select(importance, batch, seq, sliding_window, n_keep, protected_pos, n_protected,
                                       kept_idx, kept_count, workspace, static_cast<cudaStream_t>(stream)));
}

nq_status_t nq_gather_rows(const void* in, int32_t in_dtype, int32_t batch, int32_t heads, int32_t head_dim,
                           int64_t in_stride_b, int64_t in_stride_h, int64_t in_stride_t, const int32_t* kept_idx,
                           const int32_t* kept_count, int32_t n_kept, uint16_t* out, int64_t out_stride_b,
                           int64_t out_stride_h, int64_t out_stride_t, nq_stream_t stream) {
  if (!in || !out || batch < 0 || heads < 0 || n_kept < 0 || head_dim <= 0 || (head_dim & 7))
    return NQ_ERR_INVALID_ARG;
  if (in_dtype < 0 || in_dtype > 2) return NQ_ERR_INVALID_ARG;
  const int eb = elem_bytes(in_dtype);
  if (!aligned16(in) || !aligned16(out) || (in_stride_b * eb) % 16 || (in_stride_h * eb) % 16 ||
      (in_stride_t * eb) % 16 || (out_stride_b * 2) % 16 || (out_stride_h * 2) % 16 || (out_stride_t * 2) % 16)
    return NQ_ERR_ALIGNMENT;
  {
    // device memory, or pinned host memory mapped at the same address (UVA); nothing else
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, in) != cudaSuccess ||
        (at.type != cudaMemoryTypeDevice && at.type != cudaMemoryTypeManaged &&
         !(at.type == cudaMemoryTypeHost && at.devicePointer == in))) {
      cudaGetLastError();
      return NQ_ERR_INVALID_ARG;
    }
  }
  return cuda_status(nq::launch_gather_rows(in, in_dtype, batch, heads, head_dim, in_stride_b, in_stride_h,
                                            in_stride_t, kept_idx, kept_count, n_kept, out, out_stride_b,
                                            out_stride_h, out_stride_t, static_cast<cudaStream_t>(stream)));
}

nq_status_t nq_delta_codes(const uint8_t* codes, int32_t n_streams, int32_t n_tokens, int32_t head_dim_padded,
                           int32_t levels, int8_t* delta, nq_stream_t stream) {
  if (!codes || !delta || n_streams < 0 || n_tokens < 0 || !valid_levels(levels)) return NQ_ERR_INVALID_ARG;
  if (head_dim_padded <= 0 || (head_dim_padded & 7)) return NQ_ERR_INVALID_ARG;
  if (!aligned16(delta) || !aligned16(codes)) return NQ_ERR_ALIGNMENT;
  return cuda_status(
      nq::launch_delta(codes, n_streams, n_tokens, head_dim_padded, levels, delta, static_cast<cudaStream_t>(stream)));
}

nq_status_t nq_code_histogram(const uint8_t* codes, int64_t rows, int32_t head_dim_padded, int32_t levels,
                              uint32_t* counts, nq_stream_t stream) {
  if (!codes || !counts || rows < 0 || !valid_levels(levels)) return NQ_ERR_INVALID_ARG;
  if (head_dim_padded <= 0 || (head_dim_padded & 7)) return NQ_ERR_INVALID_ARG;
  return cuda_status(nq::launch_code_symbols(codes, rows, head_dim_padded, levels, 0, 0, counts, nullptr,
                                             static_cast<cudaStream_t>(stream)));
}

nq_status_t nq_code_symbols(const uint8_t* codes, int64_t rows, int32_t head_dim_padded, int32_t levels,
                            int32_t half, uint8_t* symbols, nq_stream_t stream) {
  if (!codes || !symbols || rows < 0 || !valid_levels(levels)) return NQ_ERR_INVALID_ARG;
  if (head_dim_padded <= 0 || (head_dim_padded & 7)) return NQ_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(symbols) & 7) return NQ_ERR_ALIGNMENT;
  return cuda_status(nq::launch_code_symbols(codes, rows, head_dim_padded, levels, 1, half != 0, nullptr, symbols,
                                             static_cast<cudaStream_t>(stream)));
}

// rANS, 32-bit state, 16-bit words, M = 2^12, state in [2^16, 2^32)
// (nexusquant/core/entropy_coder.py:246-295 encode, :298-345 decode).  Host code.
nq_status_t nq_rans_encode(const uint8_t* symbols, int64_t n, const uint32_t* freqs, int32_t alphabet,
                           uint16_t* out, int64_t out_cap, int64_t* out_len) {
  if ((!symbols && n) || !freqs || !out || !out_len || alphabet <= 0 || alphabet > 256 || n < 0) return NQ_ERR_INVALID_ARG;
  uint32_t cum[257];
  cum[0] = 0;
  for (int s = 0; s < alphabet; ++s) cum[s + 1] = cum[s] + freqs[s];
  if (cum[alphabet] != 4096u) return NQ_ERR_INVALID_ARG;
  int64_t k = 0;  // words written, in reverse order
  uint64_t state = 1u << 16;
  for (int64_t i = n - 1; i >= 0; --i) {
    const unsigned s = symbols[i];
    if (s >= (unsigned)alphabet || freqs[s] == 0) return NQ_ERR_INVALID_ARG;
    const uint64_t fs = freqs[s];
    const uint64_t threshold = fs << 20;
    while (state >= threshold) {
      if (k >= out_cap) return NQ_ERR_TOO_LARGE;
      out[k++] = (uint16_t)(state & 0xFFFFu);
      state >>= 16;
    }
    state = (state / fs) * 4096u + (state % fs) + cum[s];
  }
  if (k + 2 > out_cap) return NQ_ERR_TOO_LARGE;
  out[k++] = (uint16_t)(state & 0xFFFFu);
  out[k++] = (uint16_t)((state >> 16) & 0xFFFFu);
  for (int64_t a = 0, b = k - 1; a < b; ++a, --b) {
    const uint16_t t = out[a];
    out[a] = out[b];
    out[b] = t;
  }
  *out_len = k;
  return NQ_OK;
}

nq_status_t nq_rans_decode(const uint16_t* words, int64_t n_words, int64_t n, const uint32_t* freqs,
                           int32_t alphabet, uint8_t* symbols) {
  if (!words || n_words < 2 || !freqs || (!symbols && n) || alphabet <= 0 || alphabet > 256 || n < 0)
    return NQ_ERR_INVALID_ARG;
  uint32_t cum[257];
  cum[0] = 0;
  for (int s = 0; s < alphabet; ++s) cum[s + 1] = cum[s] + freqs[s];
  if (cum[alphabet] != 4096u) return NQ_ERR_INVALID_ARG;
  static thread_local uint8_t slot2sym[4096];
  for (int s = 0; s < alphabet; ++s)
    for (uint32_t c = cum[s]; c < cum[s + 1]; ++c) slot2sym[c] = (uint8_t)s;
  int64_t pos = 2;
  uint64_t state = ((uint64_t)words[0] << 16) | words[1];
  for (int64_t i = 0; i < n; ++i) {
    const uint32_t slot = (uint32_t)(state & 4095u);
    const unsigned s = slot2sym[slot];
    state = freqs[s] * (state >> 12) + slot - cum[s];
    while (state < (1u << 16) && pos < n_words) state = (state << 16) | words[pos++];
    symbols[i] = (uint8_t)s;
  }
  return NQ_OK;
}

}  // extern "C"

extern "C" {
size_t nq_attend_compressed_workspace_size(int32_t batch, int32_t q_heads, int32_t heads, int32_t n_tokens) {
  if (batch <= 0 || q_heads <= 0 || heads <= 0 || n_tokens <= 0) return 0;
  return nq::attend_workspace_bytes(batch, q_heads, nq::attend_splits(batch, heads, n_tokens));
}

nq_status_t nq_attend_compressed(const nq_attend_params_t* p, void* workspace, size_t workspace_bytes,
                                 nq_stream_t stream) {
  if (!p) return NQ_ERR_INVALID_ARG;
  if (p->batch < 0 || p->q_heads <= 0 || p->heads <= 0 || p->n_tokens < 0) return NQ_ERR_INVALID_ARG;
  if (p->head_dim != 128 || p->head_dim_padded != 128) return NQ_ERR_UNSUPPORTED;
  const int g = p->q_heads % p->heads ? 0 : p->q_heads / p->heads;
  if (g != 1 && g != 2 && g != 4 && g != 8) return NQ_ERR_UNSUPPORTED;
  if (!valid_levels(p->key_levels) || !valid_levels(p->value_levels)) return NQ_ERR_INVALID_ARG;
  if (p->batch == 0) return NQ_OK;
  if (p->n_tokens == 0) {
    // empty code tensors may carry null pointers: only the output is needed
    if (!p->out) return NQ_ERR_INVALID_ARG;
    // nothing to attend: zero the [q_heads, 128] fp16 rows of each batch element (one strided
    // memset per batch element)
    if (p->out_stride_h < 128) return NQ_ERR_INVALID_ARG;
    for (int b = 0; b < p->batch; ++b) {
      const cudaError_t e = cudaMemset2DAsync(p->out + b * p->out_stride_b, (size_t)p->out_stride_h * 2, 0, 256,
                                              (size_t)p->q_heads, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return NQ_ERR_CUDA;
    }
    return NQ_OK;
  }
  if (!p->q || !p->out || !p->k_codes || !p->v_codes || !p->k_scales || !p->v_scales || !p->positions ||
      !p->rope_cos || !p->rope_sin || p->rope_rows <= 0)
    return NQ_ERR_INVALID_ARG;
  const void* al[] = {p->k_codes, p->v_codes, p->rope_cos, p->rope_sin};
  for (const void* q : al)
    if (!aligned16(q)) return NQ_ERR_ALIGNMENT;
  const int splits = nq::attend_splits(p->batch, p->heads, p->n_tokens);
  if (!workspace || workspace_bytes < nq::attend_workspace_bytes(p->batch, p->q_heads, splits))
    return NQ_ERR_WORKSPACE;
  nq::AttendArgs a{};
  a.batch = p->batch; a.q_heads = p->q_heads; a.heads = p->heads; a.n_tokens = p->n_tokens;
  a.splits = splits;
  const int tiles = (p->n_tokens + 127) / 128;
  a.tokens_per_split = ((tiles + splits - 1) / splits) * 128;
  a.count = p->count;
  a.q = reinterpret_cast<const __half*>(p->q);
  a.q_stride_b = p->q_stride_b; a.q_stride_h = p->q_stride_h;
  a.k_codes = p->k_codes; a.v_codes = p->v_codes; a.k_scales = p->k_scales; a.v_scales = p->v_scales;
  a.positions = p->positions; a.rope_cos = p->rope_cos; a.rope_sin = p->rope_sin; a.rope_rows = p->rope_rows;
  a.key_sharpen = p->key_sharpen == 0.0f ? 1.0f : p->key_sharpen;
  a.scale = p->scale == 0.0f ? 1.0f / sqrtf((float)p->head_dim) : p->scale;
  a.out = reinterpret_cast<__half*>(p->out);
  a.out_stride_b = p->out_stride_b; a.out_stride_h = p->out_stride_h;
  auto fmt = [](int levels) { return levels <= 4 ? 0 : (levels == 8 ? 1 : 2); };
  return cuda_status(nq::launch_attend(a, fmt(p->key_levels), fmt(p->value_levels), workspace,
                                       static_cast<cudaStream_t>(stream)));
}
}  // extern "C"
