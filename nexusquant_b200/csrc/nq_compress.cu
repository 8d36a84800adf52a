// Host dispatch of the compress kernels by input dtype (kernels in nq_compress.cuh).
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

template <typename TIn>
cudaError_t launch_compress_t(const CompressArgs& a, int n_layers, long long n_tiles, int fk, int fv, cudaStream_t s,
                              bool recon);

// All layers of `a` must share the key level count and the value level count (0 for a half
// whose layers all lack that tensor: its kernel is skipped).
cudaError_t launch_compress(const CompressArgs& args, int n_layers, cudaStream_t s, bool recon) {
  CompressArgs a = args;
  a.hg_shift = 0;
  while ((1 << a.hg_shift) < a.head_group) ++a.hg_shift;
  if ((1 << a.hg_shift) != a.head_group || a.head_group > 8) return cudaErrorInvalidValue;
  const int tok = kCompressVecs / a.head_group;
  const long long tiles = 2LL * n_layers * a.batch * ((a.heads + a.head_group - 1) / a.head_group) *
                          ((a.n_kept + tok - 1) / tok);
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;  // kernels index tiles with 32-bit ints
  int lk = 0, lv = 0;
  for (int l = 0; l < n_layers; ++l) {
    if (a.layers[l].k) lk = a.layers[l].key_levels;
    if (a.layers[l].v) lv = a.layers[l].value_levels;
  }
  switch (a.in_dtype) {
    case 0: return launch_compress_t<__half>(a, n_layers, tiles, lk, lv, s, recon);
    case 1: return launch_compress_t<__nv_bfloat16>(a, n_layers, tiles, lk, lv, s, recon);
    case 2: return launch_compress_t<float>(a, n_layers, tiles, lk, lv, s, recon);
  }
  return cudaErrorInvalidValue;
}

}  // namespace nq
