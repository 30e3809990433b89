// Slice of a packed exact-token store: out = packed[start:end].
//
// Reference (pkhairkh/gfst-hmb-public): exact_block_materialize_forward
// (src/gfst_hmb_mpuc/csrc/sm120_stub.cu:225-245), called from
// GfstDecodeState._materialize_exact_block (src/gfst_hmb_mpuc/state.py:553-632)
// to read one block's token ids out of the packed pool.  The bytes of the
// range are copied by a grid-stride kernel: 16-byte vectors when source and
// destination line up, else single bytes.
#include "gfst_common.cuh"

namespace gfst {
namespace {

constexpr int kCopyThreads = 256;

__global__ void __launch_bounds__(kCopyThreads) copy_vec16_kernel(const uint4* __restrict__ src,
                                                                 uint4* __restrict__ dst, int64_t n_vec) {
  for (int64_t i = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; i < n_vec; i += (int64_t)gridDim.x * kCopyThreads)
    dst[i] = src[i];
}

__global__ void __launch_bounds__(kCopyThreads) copy_bytes_kernel(const unsigned char* __restrict__ src,
                                                                 unsigned char* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kCopyThreads)
    dst[i] = src[i];
}

unsigned grid_for(int64_t units) {
  const int64_t blocks = (units + kCopyThreads - 1) / kCopyThreads;
  return (unsigned)(blocks < 148 * 8 ? (blocks < 1 ? 1 : blocks) : 148 * 8);
}

}  // namespace
}  // namespace gfst

extern "C" int gfst_exact_block_materialize(const void* packed, int64_t n_elements, int elem_size, int64_t start,
                                            int64_t end, void* out, cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_elements >= 0 && elem_size >= 1, GFST_ERR_ARG, "bad sizes (n=%lld, elem_size=%d)",
               (long long)n_elements, elem_size);
  GFST_REQUIRE(start >= 0, GFST_ERR_ARG, "start must be nonnegative");
  GFST_REQUIRE(end >= start, GFST_ERR_ARG, "end must be >= start");
  GFST_REQUIRE(end <= n_elements, GFST_ERR_ARG, "end %lld > %lld elements", (long long)end, (long long)n_elements);
  const int64_t bytes = (end - start) * (int64_t)elem_size;
  if (bytes == 0) return GFST_OK;
  GFST_REQUIRE(packed && out, GFST_ERR_ARG, "null buffer");
  const unsigned char* src = static_cast<const unsigned char*>(packed) + start * (int64_t)elem_size;
  unsigned char* dst = static_cast<unsigned char*>(out);
  if (aligned16(src) && aligned16(dst) && bytes % 16 == 0) {
    copy_vec16_kernel<<<grid_for(bytes / 16), kCopyThreads, 0, stream>>>(reinterpret_cast<const uint4*>(src),
                                                                         reinterpret_cast<uint4*>(dst), bytes / 16);
    return check_launch("copy_vec16_kernel");
  }
  copy_bytes_kernel<<<grid_for(bytes), kCopyThreads, 0, stream>>>(src, dst, bytes);
  return check_launch("copy_bytes_kernel");
}
