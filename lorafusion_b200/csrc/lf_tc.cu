// sm_100a tensor-core kernels of the fused multi-adapter LoRA op (bf16 / f16 in, f32 accumulate).
//
// All three kernels share one structure: warp 0 is the TMA producer (one elected lane),
// warp 1 allocates TMEM and issues tcgen05.mma (one elected lane), warps 2..5 drain the
// TMEM accumulator.  Stages are handed over with mbarriers; every wait is bounded.
//
//  tc_gemm   out = P Q^T + sum_segments S_ext[seg] L[slot(seg)]^T
//            Forward: P = x, Q = W (K-major), S_ext = scaled x A_i^T, L = B_i.
//            dX:      P = g, Q = W read MN-major (no transposed copy), S_ext = scaled g B_i, L = A_i^T.
//            The LoRA expand is extra K-steps into the same TMEM accumulator, one per
//            segment tile, so the output is written exactly once.
//  tc_shrink S_ext[seg] = mask_rows(scale * P_tile A_slot^T), K split across a thread-block
//            cluster and reduced through distributed shared memory in a fixed order.
//  tc_gram   grad[slot] = sum over the slot's segment tiles of D_tile^T S_ext[seg]
//            (dB: D = g, S = forward S_ext;  dA: D = x, S = backward S_ext), both operands
//            read MN-major straight from the row-major activations.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "lf_internal.cuh"
#include "lf_ptx.cuh"

namespace lf {
namespace {

constexpr int kBM = 128;  // rows per tile = TMEM lanes
constexpr int kBK = 64;   // K elements per stage = one 128-byte swizzle row
constexpr int kThreads = 192;
constexpr int kGemmBN = 256;
constexpr int kGemmStages = 4;
constexpr int kShrStages = 3;
constexpr int kGramStages = 4;

template <typename OutT>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  return pack_bf16x2(a, b);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  return pack_f16x2(a, b);
}
template <typename OutT>
__device__ __forceinline__ OutT cvt_out(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half cvt_out<__half>(float v) {
  return __float2half_rn(v);
}

// Time-bounded wait used only while unwinding after an abort: ignores the abort flag.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_error(err, kErrTimeoutDrain);
      return;
    }
  }
}

// Bounded wait done by lane 0 and broadcast, so the warp stays converged for tcgen05.ld.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort_flag, err, code) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
}

// ========================================================================== GEMM
struct GemmParams {
  void* out;
  int64_t ldo;
  int T, Nout, Kred;
  int n_mtiles, n_ntiles, group_m;
  int lora, r_pad;
  uint32_t idesc_main, idesc_lora;
  uint32_t lora_layout, lora_sbo;
  Tables tb;
};

__device__ __forceinline__ void gemm_raster(int t, const GemmParams& p, int& m, int& n) {
  const int per_group = p.group_m * p.n_ntiles;
  const int g = t / per_group;
  const int first_m = g * p.group_m;
  const int gsize = min(p.n_mtiles - first_m, p.group_m);
  const int r = t - g * per_group;
  m = first_m + r % gsize;
  n = r / gsize;
}

constexpr int kGemmABytes = kBM * kBK * 2;       // 16 KB
constexpr int kGemmBBytes = kGemmBN * kBK * 2;   // 32 KB
constexpr int kGemmSmem = 1024 + kGemmStages * (kGemmABytes + kGemmBBytes) + 256;

template <bool kQMN, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_p, const __grid_constant__ CUtensorMap map_q,
                   const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_l,
                   const GemmParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kGemmStages * kGemmABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kGemmStages * kGemmBBytes);
  uint64_t* empty = full + kGemmStages;
  uint64_t* tfull = empty + kGemmStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = prm.n_mtiles * prm.n_ntiles;
  const int nkb = (prm.Kred + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_p);
    tma_prefetch_desc(&map_q);
    if (prm.lora) {
      tma_prefetch_desc(&map_s);
      tma_prefetch_desc(&map_l);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, last_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int m, n;
        gemm_raster(t, prm, m, n);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, prm.tb.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kGemmABytes + kGemmBBytes);
          tma_load_2d(sA + stage * kGemmABytes, &map_p, &full[stage], kb * kBK, m * kBM);
          if (kQMN) {
#pragma unroll
            for (int j = 0; j < kGemmBN / 64; ++j)
              tma_load_2d(sB + stage * kGemmBBytes + j * (64 * kBK * 2), &map_q, &full[stage], n * kGemmBN + j * 64,
                          kb * kBK);
          } else {
            tma_load_2d(sB + stage * kGemmBBytes, &map_q, &full[stage], kb * kBK, n * kGemmBN);
          }
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kGemmStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok || !prm.lora) continue;
        const int sb = prm.tb.tile_st(m), se = prm.tb.tile_st(m + 1);
        const uint32_t bytes = static_cast<uint32_t>((kBM + kGemmBN) * prm.r_pad * 2);
        for (int j = sb; j < se; ++j) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, prm.tb.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], bytes);
          tma_load_2d(sA + stage * kGemmABytes, &map_s, &full[stage], 0, j * kBM);
          tma_load_2d(sB + stage * kGemmBBytes, &map_l, &full[stage], 0,
                      prm.tb.st_slot(j) * prm.Nout + n * kGemmBN);
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kGemmStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {  // let every copy this thread started land before the CTA exits
        for (int s = 0; s < kGemmStages; ++s)
          if (issued_mask & (1u << s)) drain_wait(&full[s], (last_parity >> s) & 1u, prm.tb.err);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool issued_any = false;
      const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
      int it = 0;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++it) {
        int m, n;
        gemm_raster(t, prm, m, n);
        const int buf = it & 1;
        if (!mbar_wait(&tempty[buf], ((it >> 1) & 1) ^ 1, abort_flag, prm.tb.err, kErrTimeoutAcc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * kGemmBN);
        uint32_t acc = 0;
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, prm.tb.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = a_base + stage * kGemmABytes, b0 = b_base + stage * kGemmBBytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = umma_sdesc(a0 + k * 32, 16, 1024, 2);
            const uint64_t bdesc = kQMN ? umma_sdesc(b0 + k * 2048, 64 * kBK * 2, 1024, 2)
                                        : umma_sdesc(b0 + k * 32, 16, 1024, 2);
            umma_f16(d, adesc, bdesc, prm.idesc_main, acc);
            acc = 1;
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == kGemmStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok && prm.lora) {
          const int sb = prm.tb.tile_st(m), se = prm.tb.tile_st(m + 1);
          for (int j = sb; j < se; ++j) {
            if (!mbar_wait(&full[stage], phase, abort_flag, prm.tb.err, kErrTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = a_base + stage * kGemmABytes, b0 = b_base + stage * kGemmBBytes;
            for (int k = 0; k < prm.r_pad / 16; ++k) {
              const uint64_t adesc = umma_sdesc(a0 + k * 32, 16, prm.lora_sbo, prm.lora_layout);
              const uint64_t bdesc = umma_sdesc(b0 + k * 32, 16, prm.lora_sbo, prm.lora_layout);
              umma_f16(d, adesc, bdesc, prm.idesc_lora, acc);
              acc = 1;
            }
            issued_any = true;
            umma_commit(&empty[stage]);
            if (++stage == kGemmStages) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
      if (!ok && issued_any) {  // wait for in-flight MMAs before TMEM is released
        umma_commit(drain);
        drain_wait(drain, 0, prm.tb.err);
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      int m, n;
      gemm_raster(t, prm, m, n);
      const int buf = it & 1;
      if (!warp_wait(&tfull[buf], (it >> 1) & 1, abort_flag, prm.tb.err, kErrTimeoutAcc)) break;
      tc_fence_after();
      const int row = m * kBM + q * 32 + lane;
      OutT* orow = reinterpret_cast<OutT*>(prm.out) + static_cast<int64_t>(row) * prm.ldo;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * kGemmBN);
#pragma unroll 1
      for (int c = 0; c < kGemmBN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tbase + c * 32, v);
        tmem_wait_ld();
        const int col0 = n * kGemmBN + c * 32;
        if (row < prm.T) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            if (col0 + g * 8 < prm.Nout) {
              uint4 pk;
              pk.x = pack2<OutT>(__uint_as_float(v[g * 8 + 0]), __uint_as_float(v[g * 8 + 1]));
              pk.y = pack2<OutT>(__uint_as_float(v[g * 8 + 2]), __uint_as_float(v[g * 8 + 3]));
              pk.z = pack2<OutT>(__uint_as_float(v[g * 8 + 4]), __uint_as_float(v[g * 8 + 5]));
              pk.w = pack2<OutT>(__uint_as_float(v[g * 8 + 6]), __uint_as_float(v[g * 8 + 7]));
              *reinterpret_cast<uint4*>(orow + col0 + g * 8) = pk;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ========================================================================== shrink
struct ShrinkParams {
  void* s_ext;
  int ab_fmt;
  int Kred;
  int kb_per_split;
  int cluster;
  int r_pad;
  Tables tb;
};

constexpr int kShrABytes = kBM * kBK * 2;    // 16 KB
constexpr int kShrBBytes = 128 * kBK * 2;    // N <= 128 rows
constexpr int kShrSmem = 1024 + kShrStages * (kShrABytes + kShrBBytes) + 256;
constexpr int kPartLd = kBM + 1;             // column-major partial sums, odd stride
static_assert(128 * kPartLd * 4 <= kShrStages * (kShrABytes + kShrBBytes), "partials must fit the stage area");

template <typename OutT>
__global__ void __launch_bounds__(kThreads, 2)
    tc_shrink_kernel(const __grid_constant__ CUtensorMap map_p, const __grid_constant__ CUtensorMap map_a,
                     const ShrinkParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kShrStages * kShrABytes;
  float* partial = reinterpret_cast<float*>(smem);  // reused once every stage is consumed
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kShrStages * kShrBBytes);
  uint64_t* empty = full + kShrStages;
  uint64_t* tfull = empty + kShrStages;
  uint64_t* drain = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Tables& tb = prm.tb;
  const int unit = blockIdx.x / prm.cluster;
  const uint32_t crank = cluster_ctarank();
  const int tile = tb.unit_tile(unit), st0 = tb.unit_st0(unit), nst = tb.unit_nst(unit);
  const int r_pad = prm.r_pad;
  const int N = nst * r_pad;
  const int nkb = (prm.Kred + kBK - 1) / kBK;
  const int kb0 = static_cast<int>(crank) * prm.kb_per_split;
  const int kb1 = min(nkb, kb0 + prm.kb_per_split);
  const bool has_k = kb1 > kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kShrStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_p);
    tma_prefetch_desc(&map_a);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && has_k) {
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, last_parity = 0;
      bool ok = true;
      const uint32_t bytes = static_cast<uint32_t>(kShrABytes + N * kBK * 2);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, prm.tb.err, kErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], bytes);
        tma_load_2d(sA + stage * kShrABytes, &map_p, &full[stage], kb * kBK, tile * kBM);
        for (int j = 0; j < nst; ++j)
          tma_load_2d(sB + stage * kShrBBytes + j * r_pad * (kBK * 2), &map_a, &full[stage], kb * kBK,
                      tb.st_slot(st0 + j) * r_pad);
        issued_mask |= 1u << stage;
        last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == kShrStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok)
        for (int s = 0; s < kShrStages; ++s)
          if (issued_mask & (1u << s)) drain_wait(&full[s], (last_parity >> s) & 1u, prm.tb.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && has_k) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued_any = false;
      const uint32_t idesc = umma_idesc_f16(kBM, N, prm.ab_fmt, 0, 0);
      const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
      uint32_t acc = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, prm.tb.err, kErrTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = a_base + stage * kShrABytes, b0 = b_base + stage * kShrBBytes;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          umma_f16(tmem_base, umma_sdesc(a0 + k * 32, 16, 1024, 2), umma_sdesc(b0 + k * 32, 16, 1024, 2), idesc, acc);
          acc = 1;
        }
        issued_any = true;
        umma_commit(&empty[stage]);
        if (++stage == kShrStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (ok)
        umma_commit(tfull);
      else if (issued_any) {
        umma_commit(drain);
        drain_wait(drain, 0, prm.tb.err);
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    bool ok = true;
    if (has_k) ok = warp_wait(tfull, 0, abort_flag, prm.tb.err, kErrTimeoutAcc);
    if (ok && has_k) {
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
      for (int c = 0; c < N; c += 16) {
        uint32_t v[16];
        tmem_ld16(tbase + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) partial[(c + jj) * kPartLd + row] = __uint_as_float(v[jj]);
      }
    } else {
      for (int c = 0; c < N; ++c) partial[c * kPartLd + row] = 0.f;
    }
  }

  // all partial sums of the cluster are visible after this barrier
  tc_fence_before();
  cluster_sync_all();

  {
    const int rows_per = kBM / prm.cluster;
    const int r0 = static_cast<int>(crank) * rows_per;
    const int total = rows_per * N;
    const uint32_t part_base = smem_u32(partial);
    OutT* out = reinterpret_cast<OutT*>(prm.s_ext);
    for (int e = threadIdx.x; e < total; e += kThreads) {
      const int row = r0 + e / N, col = e % N;
      const uint32_t off = static_cast<uint32_t>((col * kPartLd + row) * 4);
      float sum = 0.f;
      for (int qr = 0; qr < prm.cluster; ++qr) sum += ld_cluster_f32(map_to_cta(part_base + off, qr));
      const int j = col / r_pad, jj = col - j * r_pad;
      const int st = st0 + j;
      const bool in = row >= tb.st_lo(st) && row < tb.st_hi(st);
      const float v = in ? tb.st_scale(st) * sum : 0.f;
      out[(static_cast<int64_t>(st) * kBM + row) * r_pad + jj] = cvt_out<OutT>(v);
    }
  }

  // keep this CTA's shared memory alive until every peer has read it
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 128);
  }
}

// ========================================================================== gram (dA / dB)
struct GramParams {
  void* out;
  int C;
  int n_cblk;
  int transpose_out;
  int r_pad;
  uint32_t idesc;
  uint32_t s_layout, s_sbo, s_kstep;
  Tables tb;
};

constexpr int kGramDBytes = kBM * 128 * 2;  // 128 rows x 128 columns
constexpr int kGramSBytes = kBM * 64 * 2;   // 128 rows x r_pad (<= 64)
constexpr int kGramSmem = 1024 + kGramStages * (kGramDBytes + kGramSBytes) + 256;

template <typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gram_kernel(const __grid_constant__ CUtensorMap map_d, const __grid_constant__ CUtensorMap map_s,
                   const GramParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sD = smem;
  uint8_t* sS = smem + kGramStages * kGramDBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sS + kGramStages * kGramSBytes);
  uint64_t* empty = full + kGramStages;
  uint64_t* tfull = empty + kGramStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Tables& tb = prm.tb;
  const int total = tb.n_slots * prm.n_cblk;
  const int r_pad = prm.r_pad;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGramStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_d);
    tma_prefetch_desc(&map_s);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, last_parity = 0;
      bool ok = true;
      const uint32_t bytes = static_cast<uint32_t>(kGramDBytes + kBM * r_pad * 2);
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const int slot = tb.slot_order(u / prm.n_cblk);
        const int cb = u % prm.n_cblk;
        for (int i = tb.slot_st(slot); i < tb.slot_st(slot + 1); ++i) {
          const int st = tb.slot_list(i);
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, prm.tb.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], bytes);
          const int row0 = tb.st_tile(st) * kBM;
          tma_load_2d(sD + stage * kGramDBytes, &map_d, &full[stage], cb * 128, row0);
          tma_load_2d(sD + stage * kGramDBytes + kGramDBytes / 2, &map_d, &full[stage], cb * 128 + 64, row0);
          tma_load_2d(sS + stage * kGramSBytes, &map_s, &full[stage], 0, st * kBM);
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kGramStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok)
        for (int s = 0; s < kGramStages; ++s)
          if (issued_mask & (1u << s)) drain_wait(&full[s], (last_parity >> s) & 1u, prm.tb.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued_any = false;
      const uint32_t d_base = smem_u32(sD), s_base = smem_u32(sS);
      int it = 0;
      for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
        const int slot = tb.slot_order(u / prm.n_cblk);
        const int b = tb.slot_st(slot), e = tb.slot_st(slot + 1);
        if (b == e) continue;  // adapter with only empty routes: epilogue writes zeros
        const int buf = it & 1;
        if (!mbar_wait(&tempty[buf], ((it >> 1) & 1) ^ 1, abort_flag, prm.tb.err, kErrTimeoutAcc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dt = tmem_base + static_cast<uint32_t>(buf * 64);
        uint32_t acc = 0;
        for (int i = b; i < e; ++i) {
          if (!mbar_wait(&full[stage], phase, abort_flag, prm.tb.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = d_base + stage * kGramDBytes, b0 = s_base + stage * kGramSBytes;
#pragma unroll
          for (int k = 0; k < kBM / 16; ++k) {
            const uint64_t adesc = umma_sdesc(a0 + k * 2048, kGramDBytes / 2, 1024, 2);
            const uint64_t bdesc = umma_sdesc(b0 + k * prm.s_kstep, kBM * r_pad * 2, prm.s_sbo, prm.s_layout);
            umma_f16(dt, adesc, bdesc, prm.idesc, acc);
            acc = 1;
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == kGramStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
        ++it;
      }
      if (!ok && issued_any) {
        umma_commit(drain);
        drain_wait(drain, 0, prm.tb.err);
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    int it = 0;
    OutT* out = reinterpret_cast<OutT*>(prm.out);
    for (int u = blockIdx.x; u < total; u += gridDim.x) {
      const int slot = tb.slot_order(u / prm.n_cblk);
      const int cb = u % prm.n_cblk;
      const int c = cb * 128 + q * 32 + lane;
      const int rank = tb.slot_rank(slot);
      OutT* o = out + static_cast<int64_t>(tb.rank_prefix(slot)) * prm.C;
      const bool empty_slot = tb.slot_st(slot) == tb.slot_st(slot + 1);
      if (empty_slot) {
        if (c < prm.C)
          for (int j = 0; j < rank; ++j) {
            if (prm.transpose_out)
              o[static_cast<int64_t>(j) * prm.C + c] = cvt_out<OutT>(0.f);
            else
              o[static_cast<int64_t>(c) * rank + j] = cvt_out<OutT>(0.f);
          }
        continue;
      }
      const int buf = it & 1;
      if (!warp_wait(&tfull[buf], (it >> 1) & 1, abort_flag, prm.tb.err, kErrTimeoutAcc)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * 64);
      for (int j0 = 0; j0 < r_pad; j0 += 16) {
        uint32_t v[16];
        tmem_ld16(tbase + j0, v);
        tmem_wait_ld();
        if (c < prm.C) {
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = j0 + jj;
            if (j < rank) {
              const OutT val = cvt_out<OutT>(__uint_as_float(v[jj]));
              if (prm.transpose_out)
                o[static_cast<int64_t>(j) * prm.C + c] = val;
              else
                o[static_cast<int64_t>(c) * rank + j] = val;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
      ++it;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 128);
  }
}

// Opt-in to large dynamic shared memory once per (kernel, device).
struct SmemOptIn {
  const void* fn;
  int dev;
};
SmemOptIn g_smem_optin[64];
int g_smem_optin_n = 0;

template <typename K>
cudaError_t ensure_smem(K kernel, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const void* fn = reinterpret_cast<const void*>(kernel);
  for (int i = 0; i < g_smem_optin_n; ++i)
    if (g_smem_optin[i].fn == fn && g_smem_optin[i].dev == dev) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && g_smem_optin_n < 64) g_smem_optin[g_smem_optin_n++] = SmemOptIn{fn, dev};
  return e;
}

uint32_t sw_sbo(int r_pad) { return static_cast<uint32_t>(8 * r_pad * 2); }

}  // namespace

cudaError_t tc_gemm(int dtype, bool q_mn_major, const TcMaps& maps, int T, int Nout, int Kred, bool lora,
                    const Tables& tb, void* out, int64_t ldo, int num_sms, cudaStream_t st) {
  GemmParams p{};
  p.out = out;
  p.ldo = ldo;
  p.T = T;
  p.Nout = Nout;
  p.Kred = Kred;
  p.n_mtiles = (T + kBM - 1) / kBM;
  p.n_ntiles = (Nout + kGemmBN - 1) / kGemmBN;
  p.group_m = 8;
  p.lora = lora ? 1 : 0;
  p.r_pad = tb.r_pad;
  const int fmt = dtype == LF_BF16 ? 1 : 0;
  p.idesc_main = umma_idesc_f16(kBM, kGemmBN, fmt, 0, q_mn_major ? 1 : 0);
  p.idesc_lora = umma_idesc_f16(kBM, kGemmBN, fmt, 0, 0);
  p.lora_layout = umma_layout_for_span(tb.r_pad * 2);
  p.lora_sbo = sw_sbo(tb.r_pad);
  p.tb = tb;
  const int total = p.n_mtiles * p.n_ntiles;
  if (total == 0) return cudaSuccess;
  const int grid = total < num_sms ? total : num_sms;
  cudaError_t e;
#define LF_LAUNCH_GEMM(QMN, OT, IDX)                                                                  \
  e = ensure_smem(tc_gemm_kernel<QMN, OT>, kGemmSmem);                                               \
  if (e != cudaSuccess) return e;                                                                    \
  tc_gemm_kernel<QMN, OT><<<grid, kThreads, kGemmSmem, st>>>(maps.p, maps.q, maps.s, maps.l, p);
  if (dtype == LF_BF16) {
    if (q_mn_major) {
      LF_LAUNCH_GEMM(true, __nv_bfloat16, 0)
    } else {
      LF_LAUNCH_GEMM(false, __nv_bfloat16, 0)
    }
  } else {
    if (q_mn_major) {
      LF_LAUNCH_GEMM(true, __half, 0)
    } else {
      LF_LAUNCH_GEMM(false, __half, 0)
    }
  }
#undef LF_LAUNCH_GEMM
  return cudaGetLastError();
}

cudaError_t tc_shrink(int dtype, const CUtensorMap& p_map, const CUtensorMap& a_map, int Kred, const Tables& tb,
                      void* s_ext, int num_sms, cudaStream_t st) {
  if (tb.n_units == 0) return cudaSuccess;
  const int nkb = (Kred + kBK - 1) / kBK;
  // split K across a cluster until there are about two CTAs per SM
  int cluster = 1;
  while (cluster < 8 && tb.n_units * cluster * 2 <= 2 * num_sms && nkb >= 2 * cluster * 2) cluster *= 2;
  ShrinkParams p{};
  p.s_ext = s_ext;
  p.ab_fmt = dtype == LF_BF16 ? 1 : 0;
  p.Kred = Kred;
  p.cluster = cluster;
  p.kb_per_split = (nkb + cluster - 1) / cluster;
  p.r_pad = tb.r_pad;
  p.tb = tb;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tb.n_units * cluster);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kShrSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (dtype == LF_BF16) {
    e = ensure_smem(tc_shrink_kernel<__nv_bfloat16>, kShrSmem);
    if (e != cudaSuccess) return e;
    e = cudaLaunchKernelEx(&cfg, tc_shrink_kernel<__nv_bfloat16>, p_map, a_map, p);
  } else {
    e = ensure_smem(tc_shrink_kernel<__half>, kShrSmem);
    if (e != cudaSuccess) return e;
    e = cudaLaunchKernelEx(&cfg, tc_shrink_kernel<__half>, p_map, a_map, p);
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t tc_gram(int dtype, const CUtensorMap& d_map, const CUtensorMap& s_map, int C, const Tables& tb, void* out,
                    int transpose_out, int num_sms, cudaStream_t st) {
  GramParams p{};
  p.out = out;
  p.C = C;
  p.n_cblk = (C + 127) / 128;
  p.transpose_out = transpose_out;
  p.r_pad = tb.r_pad;
  const int fmt = dtype == LF_BF16 ? 1 : 0;
  p.idesc = umma_idesc_f16(kBM, tb.r_pad, fmt, 1, 1);
  p.s_layout = umma_layout_for_span(tb.r_pad * 2);
  p.s_sbo = sw_sbo(tb.r_pad);
  p.s_kstep = static_cast<uint32_t>(16 * tb.r_pad * 2);
  p.tb = tb;
  const int total = tb.n_slots * p.n_cblk;
  if (total == 0) return cudaSuccess;
  const int grid = total < num_sms ? total : num_sms;
  cudaError_t e;
  if (dtype == LF_BF16) {
    e = ensure_smem(tc_gram_kernel<__nv_bfloat16>, kGramSmem);
    if (e != cudaSuccess) return e;
    tc_gram_kernel<__nv_bfloat16><<<grid, kThreads, kGramSmem, st>>>(d_map, s_map, p);
  } else {
    e = ensure_smem(tc_gram_kernel<__half>, kGramSmem);
    if (e != cudaSuccess) return e;
    tc_gram_kernel<__half><<<grid, kThreads, kGramSmem, st>>>(d_map, s_map, p);
  }
  return cudaGetLastError();
}

}  // namespace lf
