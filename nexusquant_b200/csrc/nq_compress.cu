// Host dispatch of the compress kernels by input dtype (kernels in nq_compress.cuh).
#include "nq_common.cuh"
#include "nq_internal.h"

namespace nq {

template <typename TIn>
cudaError_t launch_compress_t(const CompressArgs& a, int n_layers, long long n_tiles, int fk, int fv, cudaStream_t s,
                              bool recon);

static int fmt_of_levels(int levels) { return levels <= 4 ? 0 : (levels == 8 ? 1 : 2); }

// All layers of `a` must share the key packing format and the value packing format.
cudaError_t launch_compress(const CompressArgs& a, int n_layers, cudaStream_t s, bool recon) {
  const int tok = kCompressVecs / a.head_group;
  const long long tiles = 2LL * n_layers * a.batch * ((a.heads + a.head_group - 1) / a.head_group) *
                          ((a.n_kept + tok - 1) / tok);
  if (tiles <= 0) return cudaSuccess;
  if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;  // kernels index tiles with 32-bit ints
  const int fk = fmt_of_levels(a.layers[0].key_levels), fv = fmt_of_levels(a.layers[0].value_levels);
  switch (a.in_dtype) {
    case 0: return launch_compress_t<__half>(a, n_layers, tiles, fk, fv, s, recon);
    case 1: return launch_compress_t<__nv_bfloat16>(a, n_layers, tiles, fk, fv, s, recon);
    case 2: return launch_compress_t<float>(a, n_layers, tiles, fk, fv, s, recon);
  }
  return cudaErrorInvalidValue;
}

}  // namespace nq
