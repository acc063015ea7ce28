// Row gather/scatter between request tensors and the fused batch.
//
// build_microbatch (lorafusion/scheduler/data_batcher.py:18-87) concatenates row slices of the
// request tensors in fused-row order; scatter_outputs (data_batcher.py:90-103) splits the fused
// output back per request.  Both are the same operation: a list of runs, each copying `rows`
// consecutive rows of `row_bytes` bytes from one strided matrix to another.  The host builds the
// run list from the packing (a few hundred runs at most); one launch moves every row.
//
// Layout of the work: one warp per row, 16-byte vector copies when every address and stride of
// the run allows it (decided per run, so the branch is warp-uniform), else 4-byte or byte copies.
// The copy is byte-exact.  It is HBM-bound: each row is read once and written once.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lorafusion_b200.h"

namespace {

constexpr int kRowThreads = 256;  // 8 warps, one row each per step

__device__ __forceinline__ int find_run(const lf_row_run* runs, int n_runs, int64_t g) {
  int lo = 0, hi = n_runs - 1;  // last run with row0 <= g
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (runs[mid].row0 <= g) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kRowThreads) copy_rows_kernel(const lf_row_run* __restrict__ runs, int n_runs,
                                                                int64_t row_bytes, int64_t total_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kRowThreads / 32);
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * (kRowThreads / 32) + (threadIdx.x >> 5); g < total_rows;
       g += warps) {
    const lf_row_run r = runs[find_run(runs, n_runs, g)];
    const int64_t i = g - r.row0;
    if (i < 0 || i >= r.rows) continue;  // row not covered (runs with gaps): nothing to copy
    const char* src = reinterpret_cast<const char*>(r.src) + i * r.src_stride;
    char* dst = reinterpret_cast<char*>(r.dst) + i * r.dst_stride;
    const uint64_t align = reinterpret_cast<uint64_t>(src) | reinterpret_cast<uint64_t>(dst) |
                           static_cast<uint64_t>(row_bytes);
    if ((align & 15) == 0) {
      const int64_t n = row_bytes >> 4;
      const uint4* s = reinterpret_cast<const uint4*>(src);
      uint4* d = reinterpret_cast<uint4*>(dst);
      for (int64_t k = lane; k < n; k += 32) d[k] = __ldcs(s + k);
    } else if ((align & 3) == 0) {
      const int64_t n = row_bytes >> 2;
      const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
      uint32_t* d = reinterpret_cast<uint32_t*>(dst);
      for (int64_t k = lane; k < n; k += 32) d[k] = s[k];
    } else {
      for (int64_t k = lane; k < row_bytes; k += 32) dst[k] = src[k];
    }
  }
}

}  // namespace

extern "C" int lf_copy_rows(const lf_row_run* runs_dev, int32_t n_runs, int64_t row_bytes, int64_t total_rows,
                            lf_stream_t stream) {
  if (n_runs < 0 || row_bytes < 0 || total_rows < 0) return LF_ERR_INVALID_ARG;
  if (n_runs == 0 || row_bytes == 0 || total_rows == 0) return LF_OK;
  if (!runs_dev) return LF_ERR_INVALID_ARG;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LF_ERR_CUDA;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return LF_ERR_CUDA;
  const int64_t want = (total_rows + (kRowThreads / 32) - 1) / (kRowThreads / 32);
  const int64_t cap = static_cast<int64_t>(sms) * 8;  // 8 CTAs of 8 warps per SM in flight
  const int grid = static_cast<int>(want < cap ? want : cap);
  copy_rows_kernel<<<grid, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(runs_dev, n_runs, row_bytes,
                                                                                 total_rows);
  return cudaGetLastError() == cudaSuccess ? LF_OK : LF_ERR_CUDA;
}
