// C-ABI entry of the coarse block retrieval (score + top-k).
#include "block_topk.cuh"

extern "C" int gfst_block_topk(const void* Q, const void* Ksum, int64_t n_streams, int n_queries, int n_blocks,
                               int n_blocks_stride, int d, int k, int dtype, float* top_scores, int32_t* top_idx,
                               cudaStream_t stream) {
  using namespace gfst;
  GFST_REQUIRE(n_streams >= 0 && n_queries >= 0 && n_blocks >= 0, GFST_ERR_ARG, "negative size");
  GFST_REQUIRE(n_blocks_stride >= n_blocks, GFST_ERR_ARG, "n_blocks_stride %d < n_blocks %d", n_blocks_stride,
               n_blocks);
  GFST_REQUIRE(k >= 1 && k <= 32, GFST_ERR_SHAPE, "k=%d outside [1, 32]", k);
  GFST_REQUIRE(d >= 1 && d <= 256, GFST_ERR_SHAPE, "d=%d outside [1, 256]", d);
  GFST_REQUIRE(dtype == GFST_F32 || dtype == GFST_BF16, GFST_ERR_DTYPE, "unsupported dtype %d", dtype);
  if (n_streams == 0 || n_queries == 0) return GFST_OK;
  GFST_REQUIRE(Q && top_scores && top_idx && (Ksum || n_blocks == 0), GFST_ERR_ARG, "null buffer");
  if (dtype == GFST_BF16)
    return block_topk_tc(Q, Ksum, n_streams, n_queries, n_blocks, n_blocks_stride, d, k, top_scores, top_idx,
                         stream);
  return block_topk_simt(Q, Ksum, n_streams, n_queries, n_blocks, n_blocks_stride, d, k, dtype, top_scores,
                         top_idx, stream);
}

extern "C" int gfst_debug_bounded_wait(int64_t cycles, cudaStream_t stream) {
  GFST_REQUIRE(cycles >= 1 && cycles <= 2000000000LL, GFST_ERR_ARG, "cycles=%lld outside [1, 2e9]",
               (long long)cycles);
  return gfst::launch_bounded_wait_probe((long long)cycles, stream);
}

extern "C" int gfst_check_device_errors(int clear) {
  // every stream of the current device, the library's non-blocking ones included
  const cudaError_t se = cudaDeviceSynchronize();
  GFST_REQUIRE(se == cudaSuccess, GFST_ERR_DEVICE, "cudaDeviceSynchronize: %s", cudaGetErrorString(se));
  unsigned int v = 0, w = 0;
  int st = gfst::read_device_error(clear, &v);
  if (st != GFST_OK) return st;
  st = gfst::read_readout_error(clear, &w);
  if (st != GFST_OK) return st;
  v = v != 0 ? v : w;
  st = gfst::read_commit_error(clear, &w);
  if (st != GFST_OK) return st;
  v = v != 0 ? v : w;
  st = gfst::read_score_error(clear, &w);
  if (st != GFST_OK) return st;
  v = v != 0 ? v : w;
  st = gfst::read_scan_error(clear, &w);
  if (st != GFST_OK) return st;
  v = v != 0 ? v : w;
  if (v != 0) {
    gfst::set_last_error("a kernel gave up a bounded wait (device error word %u)", v);
    return (int)v;
  }
  return GFST_OK;
}
