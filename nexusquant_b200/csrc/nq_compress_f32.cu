// Compress kernels for float caches (see nq_compress.cuh).
#include "nq_compress.cuh"

namespace nq {
template cudaError_t launch_compress_t<float>(const CompressArgs&, int, long long, int, int, cudaStream_t, bool);
}  // namespace nq
