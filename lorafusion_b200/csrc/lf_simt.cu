// CUDA-core kernels of the fused LoRA op: products of the input values summed in f64, one
// rounding to the output type at the end.  They carry the float32 problems (where tensor cores
// cannot meet a 1e-5 bound: a float32 result within a few float32 ulps of the exact value) and
// any shape the TMA path cannot address (rows not 16-byte aligned).  Same decomposition as the
// tensor-core path: routed shrink -> S_ext (f64), base GEMM with the LoRA expand in its
// epilogue, segmented gram for dA/dB.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "lf_internal.cuh"

namespace lf {
namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// One warp per (segment tile, row).  Lanes split K, then tree-reduce.
template <typename T>
__global__ void __launch_bounds__(256) simt_shrink_kernel(const T* __restrict__ P, int64_t ldp, int Kred,
                                                          const T* __restrict__ apk, Tables tb,
                                                          double* __restrict__ s_ext) {
  const int st = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.y * 8 + warp;  // row inside the 128-row tile
  const int r_pad = tb.r_pad;
  double* out = s_ext + (static_cast<int64_t>(st) * LF_TILE_ROWS + row) * r_pad;
  const int lo = tb.st_lo(st), hi = tb.st_hi(st);
  if (row < lo || row >= hi) {
    for (int j = lane; j < r_pad; j += 32) out[j] = 0.0;
    return;
  }
  const int slot = tb.st_slot(st);
  const float scale = tb.st_scale(st);
  const int64_t grow = static_cast<int64_t>(tb.st_tile(st)) * LF_TILE_ROWS + row;
  const T* xr = P + grow * ldp;
  const T* a = apk + static_cast<int64_t>(slot) * r_pad * Kred;
  for (int j0 = 0; j0 < r_pad; j0 += 16) {
    double acc[16];
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) acc[jj] = 0.0;
    for (int k = lane; k < Kred; k += 32) {
      const double xv = to_f(xr[k]);
#pragma unroll
      for (int jj = 0; jj < 16; ++jj)
        acc[jj] = fma(xv, static_cast<double>(to_f(a[static_cast<int64_t>(j0 + jj) * Kred + k])), acc[jj]);
    }
#pragma unroll
    for (int jj = 0; jj < 16; ++jj) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[jj] += __shfl_xor_sync(0xffffffffu, acc[jj], o);
    }
    if (lane < 16) {
      double v = acc[0];
#pragma unroll
      for (int jj = 1; jj < 16; ++jj)
        if (lane == jj) v = acc[jj];
      out[j0 + lane] = static_cast<double>(scale) * v;
    }
  }
}

// 64x64 output tile, 256 threads, 4x4 per thread, K chunks of 16.
constexpr int SG_BM = 64, SG_BN = 64, SG_BK = 16;

template <typename T>
__global__ void __launch_bounds__(256) simt_gemm_kernel(const T* __restrict__ P, int64_t ldp,
                                                        const T* __restrict__ Q, int64_t qsn, int64_t qsk, int Trows,
                                                        int Nout, int Kred, const double* __restrict__ s_ext,
                                                        const T* __restrict__ lpk, Tables tb, T* __restrict__ out,
                                                        int64_t ldo) {
  __shared__ float ps[SG_BK][SG_BM + 4];
  __shared__ float qs[SG_BK][SG_BN + 4];
  const int m0 = blockIdx.y * SG_BM, n0 = blockIdx.x * SG_BN;
  const int tid = threadIdx.x;
  const int tr = tid / 16, tc = tid % 16;  // 16x16 threads, 4x4 each
  double acc[4][4] = {};
  for (int k0 = 0; k0 < Kred; k0 += SG_BK) {
    for (int e = tid; e < SG_BM * SG_BK; e += 256) {
      const int r = e / SG_BK, k = e % SG_BK;
      const int gr = m0 + r, gk = k0 + k;
      ps[k][r] = (gr < Trows && gk < Kred) ? to_f(P[static_cast<int64_t>(gr) * ldp + gk]) : 0.f;
    }
    for (int e = tid; e < SG_BN * SG_BK; e += 256) {
      int n, k;
      if (qsk == 1) {
        n = e / SG_BK;
        k = e % SG_BK;
      } else {
        k = e / SG_BN;
        n = e % SG_BN;
      }
      const int gn = n0 + n, gk = k0 + k;
      qs[k][n] = (gn < Nout && gk < Kred) ? to_f(Q[static_cast<int64_t>(gn) * qsn + static_cast<int64_t>(gk) * qsk])
                                          : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < SG_BK; ++k) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = ps[k][tr * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = qs[k][tc * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma(static_cast<double>(a[i]), static_cast<double>(b[j]), acc[i][j]);
    }
    __syncthreads();
  }
  // LoRA expand: each row adds S_ext[st][row] . L[slot][n][:] for every segment tile st holding the
  // row (one per virtual slot of its adapter), in segment-tile order
  const int r_pad = tb.r_pad;
  if (lpk != nullptr) {
    const int tile = m0 / LF_TILE_ROWS;
    const int st_b = tb.tile_st(tile), st_e = tb.tile_st(tile + 1);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int gr = m0 + tr * 4 + i;
      if (gr >= Trows) continue;
      const int row = gr - tile * LF_TILE_ROWS;
      for (int st = st_b; st < st_e; ++st) {
        if (row < tb.st_lo(st) || row >= tb.st_hi(st)) continue;
        const double* srow = s_ext + (static_cast<int64_t>(st) * LF_TILE_ROWS + row) * r_pad;
        const T* lb = lpk + static_cast<int64_t>(tb.st_slot(st)) * Nout * r_pad;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int gn = n0 + tc * 4 + j;
          if (gn >= Nout) continue;
          double d = 0.0;
          for (int q = 0; q < r_pad; ++q)
            d = fma(srow[q], static_cast<double>(to_f(lb[static_cast<int64_t>(gn) * r_pad + q])), d);
          acc[i][j] += d;
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gr = m0 + tr * 4 + i;
    if (gr >= Trows) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tc * 4 + j;
      if (gn < Nout) out[static_cast<int64_t>(gr) * ldo + gn] = from_f<T>(static_cast<float>(acc[i][j]));
    }
  }
}

// One thread per output column c of one slot; accumulators over the padded rank.  O: output type.
template <typename T, typename O, int R>
__global__ void __launch_bounds__(128) simt_gram_kernel(const T* __restrict__ D, int64_t ldd, int C,
                                                        const double* __restrict__ s_ext, Tables tb,
                                                        O* __restrict__ out, int transpose_out) {
  const int slot = blockIdx.x;
  const int c = blockIdx.y * 128 + threadIdx.x;
  double acc[R];
#pragma unroll
  for (int j = 0; j < R; ++j) acc[j] = 0.0;
  const int b = tb.slot_st(slot), e = tb.slot_st(slot + 1);
  for (int i = b; i < e; ++i) {
    const int st = tb.slot_list(i);
    const int lo = tb.st_lo(st), hi = tb.st_hi(st);
    const int64_t row0 = static_cast<int64_t>(tb.st_tile(st)) * LF_TILE_ROWS;
    for (int r = lo; r < hi; ++r) {
      const double d = (c < C) ? static_cast<double>(to_f(D[(row0 + r) * ldd + c])) : 0.0;
      const double* s = s_ext + (static_cast<int64_t>(st) * LF_TILE_ROWS + r) * R;
#pragma unroll
      for (int j = 0; j < R; ++j) acc[j] = fma(d, s[j], acc[j]);
    }
  }
  if (c >= C) return;
  const int rank = tb.slot_rank(slot);
  O* o = out + static_cast<int64_t>(tb.rank_prefix(slot)) * C;
#pragma unroll
  for (int j = 0; j < R; ++j) {
    if (j >= rank) break;
    if (transpose_out)
      o[static_cast<int64_t>(j) * C + c] = from_f<O>(static_cast<float>(acc[j]));
    else
      o[static_cast<int64_t>(c) * rank + j] = from_f<O>(static_cast<float>(acc[j]));
  }
}

template <typename T, typename O>
cudaError_t gram_dispatch(const void* D, int64_t ldd, int C, const double* s_ext, const Tables& tb, void* out,
                          int transpose_out, cudaStream_t st) {
  dim3 grid(tb.n_slots, (C + 127) / 128);
  if (tb.n_slots == 0 || C == 0) return cudaSuccess;
  switch (tb.r_pad) {
    case 16:
      simt_gram_kernel<T, O, 16><<<grid, 128, 0, st>>>((const T*)D, ldd, C, s_ext, tb, (O*)out, transpose_out);
      break;
    case 32:
      simt_gram_kernel<T, O, 32><<<grid, 128, 0, st>>>((const T*)D, ldd, C, s_ext, tb, (O*)out, transpose_out);
      break;
    default:
      simt_gram_kernel<T, O, 64><<<grid, 128, 0, st>>>((const T*)D, ldd, C, s_ext, tb, (O*)out, transpose_out);
      break;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t simt_shrink(int dtype, const void* P, int64_t ldp, int Kred, const void* apk, const Tables& tb,
                        double* s_ext, cudaStream_t st) {
  if (tb.n_segtiles == 0) return cudaSuccess;
  dim3 grid(tb.n_segtiles, LF_TILE_ROWS / 8);
  switch (dtype) {
    case LF_F32:
      simt_shrink_kernel<float><<<grid, 256, 0, st>>>((const float*)P, ldp, Kred, (const float*)apk, tb, s_ext);
      break;
    case LF_BF16:
      simt_shrink_kernel<__nv_bfloat16>
          <<<grid, 256, 0, st>>>((const __nv_bfloat16*)P, ldp, Kred, (const __nv_bfloat16*)apk, tb, s_ext);
      break;
    default:
      simt_shrink_kernel<__half><<<grid, 256, 0, st>>>((const __half*)P, ldp, Kred, (const __half*)apk, tb, s_ext);
      break;
  }
  return cudaGetLastError();
}

cudaError_t simt_gemm(int dtype, const void* P, int64_t ldp, const void* Q, int64_t qsn, int64_t qsk, int T, int Nout,
                      int Kred, const double* s_ext, const void* lpk, const Tables& tb, void* out, int64_t ldo,
                      cudaStream_t st) {
  if (T == 0 || Nout == 0) return cudaSuccess;
  dim3 grid((Nout + SG_BN - 1) / SG_BN, (T + SG_BM - 1) / SG_BM);
  switch (dtype) {
    case LF_F32:
      simt_gemm_kernel<float><<<grid, 256, 0, st>>>((const float*)P, ldp, (const float*)Q, qsn, qsk, T, Nout, Kred,
                                                    s_ext, (const float*)lpk, tb, (float*)out, ldo);
      break;
    case LF_BF16:
      simt_gemm_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
          (const __nv_bfloat16*)P, ldp, (const __nv_bfloat16*)Q, qsn, qsk, T, Nout, Kred, s_ext,
          (const __nv_bfloat16*)lpk, tb, (__nv_bfloat16*)out, ldo);
      break;
    default:
      simt_gemm_kernel<__half><<<grid, 256, 0, st>>>((const __half*)P, ldp, (const __half*)Q, qsn, qsk, T, Nout, Kred,
                                                     s_ext, (const __half*)lpk, tb, (__half*)out, ldo);
      break;
  }
  return cudaGetLastError();
}

cudaError_t simt_gram(int dtype, const void* D, int64_t ldd, int C, const double* s_ext, const Tables& tb, void* out,
                      int transpose_out, int out_f32, cudaStream_t st) {
  switch (dtype) {
    case LF_F32:
      return gram_dispatch<float, float>(D, ldd, C, s_ext, tb, out, transpose_out, st);
    case LF_BF16:
      return out_f32 ? gram_dispatch<__nv_bfloat16, float>(D, ldd, C, s_ext, tb, out, transpose_out, st)
                     : gram_dispatch<__nv_bfloat16, __nv_bfloat16>(D, ldd, C, s_ext, tb, out, transpose_out, st);
    default:
      return out_f32 ? gram_dispatch<__half, float>(D, ldd, C, s_ext, tb, out, transpose_out, st)
                     : gram_dispatch<__half, __half>(D, ldd, C, s_ext, tb, out, transpose_out, st);
  }
}

// ------------------------------------------------------------------ packing
namespace {
template <typename S, typename T>
__global__ void pack_kernel(const uint64_t* __restrict__ src_ptrs, const int32_t* __restrict__ ranks, int rank_dim,
                            int other_dim, int transpose, int d0, int d1, T* __restrict__ dst, int64_t total) {
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t per = static_cast<int64_t>(d0) * d1;
    const int s = static_cast<int>(e / per);
    const int64_t rem = e - s * per;
    const int i = static_cast<int>(rem / d1), j = static_cast<int>(rem % d1);
    const int r = ranks[s];
    const int rows = rank_dim == 0 ? r : other_dim;
    const int cols = rank_dim == 0 ? other_dim : r;
    const int si = transpose ? j : i, sj = transpose ? i : j;
    float v = 0.f;
    if (si < rows && sj < cols) {
      const S* src = reinterpret_cast<const S*>(src_ptrs[s]);
      v = to_f(src[static_cast<int64_t>(si) * cols + sj]);
    }
    dst[e] = from_f<T>(v);
  }
}

template <typename S>
cudaError_t pack_dst(int dst_dtype, const uint64_t* src_ptrs, const int32_t* ranks, int n_slots, int rank_dim,
                     int other_dim, int transpose, int d0, int d1, void* dst, cudaStream_t st) {
  const int64_t total = static_cast<int64_t>(n_slots) * d0 * d1;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks64 = (total + threads - 1) / threads;
  const int blocks = static_cast<int>(blocks64 > 148 * 32 ? 148 * 32 : blocks64);
  switch (dst_dtype) {
    case LF_F32:
      pack_kernel<S, float><<<blocks, threads, 0, st>>>(src_ptrs, ranks, rank_dim, other_dim, transpose, d0, d1,
                                                        (float*)dst, total);
      break;
    case LF_BF16:
      pack_kernel<S, __nv_bfloat16><<<blocks, threads, 0, st>>>(src_ptrs, ranks, rank_dim, other_dim, transpose, d0,
                                                                d1, (__nv_bfloat16*)dst, total);
      break;
    default:
      pack_kernel<S, __half><<<blocks, threads, 0, st>>>(src_ptrs, ranks, rank_dim, other_dim, transpose, d0, d1,
                                                         (__half*)dst, total);
      break;
  }
  return cudaGetLastError();
}
}  // namespace

cudaError_t pack_adapters(int src_dtype, int dst_dtype, const uint64_t* src_ptrs, const int32_t* ranks, int n_slots,
                          int rank_dim, int other_dim, int transpose, int d0, int d1, void* dst, cudaStream_t st) {
  switch (src_dtype) {
    case LF_F32:
      return pack_dst<float>(dst_dtype, src_ptrs, ranks, n_slots, rank_dim, other_dim, transpose, d0, d1, dst, st);
    case LF_BF16:
      return pack_dst<__nv_bfloat16>(dst_dtype, src_ptrs, ranks, n_slots, rank_dim, other_dim, transpose, d0, d1, dst,
                                     st);
    default:
      return pack_dst<__half>(dst_dtype, src_ptrs, ranks, n_slots, rank_dim, other_dim, transpose, d0, d1, dst, st);
  }
}

}  // namespace lf
