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
constexpr int kShrStages = 8;
constexpr int kGramStages = 3;

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
__device__ __forceinline__ float cvt_in(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float cvt_in(__half v) { return __half2float(v); }

// S values enter the dA/dB sums as hi + lo (both in the input type): hi = round(v) is what the
// LoRA expand reads, lo = round(v - hi) restores the bits hi dropped.
template <typename OutT>
__device__ __forceinline__ void split_hi_lo(float v, OutT& hi, OutT& lo) {
  hi = cvt_out<OutT>(v);
  lo = cvt_out<OutT>(v - cvt_in(hi));
}
// Pack 8 values as hi (pk_hi) and lo (pk_lo) halves of two uint4 each.
template <typename OutT>
__device__ __forceinline__ void pack8_hi_lo(const float* v, uint4& pk_hi, uint4& pk_lo) {
  uint32_t* h = reinterpret_cast<uint32_t*>(&pk_hi);
  uint32_t* l = reinterpret_cast<uint32_t*>(&pk_lo);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    OutT h0, l0, h1, l1;
    split_hi_lo<OutT>(v[2 * e], h0, l0);
    split_hi_lo<OutT>(v[2 * e + 1], h1, l1);
    h[e] = static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&h0)) |
           (static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&h1)) << 16);
    l[e] = static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&l0)) |
           (static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&l1)) << 16);
  }
}

// Time-bounded wait used only while unwinding after an abort: ignores the abort flag.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = wait_limit(err);
  while (!mbar_try_wait_sleep(bar, parity, kWaitSleepNs)) {
    if (globaltimer_ns() - t0 > limit) {
      record_error(err, kErrTimeoutDrain);
      return;
    }
  }
}

// Global load issued at this point in program order (an asm volatile is never moved past the
// other asm statements), so a value needed only after a k-loop is fetched before the loop.
__device__ __forceinline__ int ld_early(const int32_t* p) {
  int v;
  asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
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
        int sb = 0, se = 0, sl[4] = {0, 0, 0, 0};
        if (prm.lora) {  // the LoRA stages' table entries, fetched while the k-loop runs
          sb = ld_early(prm.tb.base + prm.tb.off_tile_st + m);
          se = ld_early(prm.tb.base + prm.tb.off_tile_st + m + 1);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            sl[q] = ld_early(prm.tb.base + prm.tb.off_st_slot + min(sb + q, prm.tb.n_segtiles - 1));
        }
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
        const uint32_t bytes = static_cast<uint32_t>((kBM + kGemmBN) * prm.r_pad * 2);
        for (int j = sb; j < se; ++j) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, prm.tb.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int jj = j - sb;
          const int slot = jj == 0 ? sl[0] : jj == 1 ? sl[1] : jj == 2 ? sl[2] : jj == 3 ? sl[3] : prm.tb.st_slot(j);
          mbar_arrive_expect_tx(&full[stage], bytes);
          tma_load_2d(sA + stage * kGemmABytes, &map_s, &full[stage], 0, j * kBM);
          tma_load_2d(sB + stage * kGemmBBytes, &map_l, &full[stage], 0, slot * prm.Nout + n * kGemmBN);
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
        int n_lora = 0;
        if (prm.lora)
          n_lora = ld_early(prm.tb.base + prm.tb.off_tile_st + m + 1) - ld_early(prm.tb.base + prm.tb.off_tile_st + m);
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
          for (int j = 0; j < n_lora; ++j) {
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

// ========================================================================== pair GEMM
// Same product as tc_gemm_kernel with 256x256 output tiles computed by a CTA pair
// (cluster of 2, tcgen05 cta_group::2).  CTA r of the pair loads rows [128r, 128r+128) of the
// tile's P rows and the N-half [128r, 128r+128) of Q into its own shared memory; the even CTA
// issues M=256/N=256 MMAs that read both CTAs' tiles, and each CTA's TMEM receives its 128
// rows.  Per CTA and k-block this moves 32 KB for 2x the FLOPs of the 48 KB single-CTA stage.
// Every TMA completes on the even CTA's `full` barrier; the MMA thread commits to the `empty`
// and `tfull` barriers of both CTAs; both CTAs' epilogue warps arrive on the even CTA's `tempty`.
constexpr int kPairStages = 6;
constexpr int kPairABytes = kBM * kBK * 2;   // 16 KB: this CTA's 128 rows of P
constexpr int kPairBBytes = 128 * kBK * 2;   // 16 KB: this CTA's 128-row half of Q
constexpr int kPairOutBytes = 4 * 2 * 32 * 64 * 2;  // epilogue staging: 4 warps x 2 buffers x (32 rows x 64 cols)
// The shrink role lays the same shared memory out as deeper stages of one x tile (16 KB) plus
// <= 64 rows of packed A (8 KB): more bytes in flight per SM while it competes with the GEMM.
constexpr int kRoleStageBytes = kPairABytes + 64 * kBK * 2;
constexpr int kRoleStages = 9;
// Accumulation chains of one shrink item: K step i of the item goes to accumulator i % chains and
// the epilogue adds the chains in fixed order.  A tcgen05 fp32 accumulation adds an error of
// about 2^-25 of the running sum per MMA, with a bias that does not average out, so a sum over
// thousands of K steps (K = 28672 is 1792 of them) loses ~1e-4 relative; c chains cut that c-fold
// (each chain's sum is shorter and smaller, and their errors have independent signs).
constexpr int kRoleChains = 4;                   // x 2 accumulator buffers x 64 columns = 512
constexpr int kShrChains = 8;                    // standalone shrink: 8 x 64 columns = 512
constexpr int kPairBars = kRoleStages;  // barrier array length shared by both roles
static_assert(kRoleStages * kRoleStageBytes <= kPairStages * (kPairABytes + kPairBBytes) + kPairOutBytes,
              "shrink-role stages must fit the pair kernel's shared memory");
// LoRA table entries of one tile (slot, segment tile) staged by the producer warp; a tile with
// more entries reads the rest from the table.
constexpr int kPairEntPerLane = 6;
constexpr int kPairEntBytes = 32 * kPairEntPerLane * 2 * 4;
// barriers: the GEMM's (and a dedicated shrink role's) at +0, a shrink prologue's at +256
constexpr int kPairBarBytes = 512;
// ... and the split tail's partial-tile loads (two buffers per epilogue warp) at +448
constexpr int kPairTailBarOff = 448;
static_assert((2 * kPairBars + 4 + 2) * 8 + 8 <= 256 && 256 + (2 * kRoleStages + 6) * 8 <= kPairTailBarOff &&
                  kPairTailBarOff + 8 * 8 <= kPairBarBytes,
              "barrier area");
// The last part of a split tail tile reads the earlier parts' partial tiles into the pipeline
// ring (idle once its last unit's MMAs are done): per epilogue warp two buffers, each one 64-column
// chunk (32 rows x 64 fp32 = 8 KB) of every earlier part (at most three).
constexpr int kTailChunkBytes = 32 * 64 * 4;
constexpr int kTailBufBytes = 3 * kTailChunkBytes;
static_assert(4 * 2 * kTailBufBytes <= kPairStages * (kPairABytes + kPairBBytes), "tail buffers fit the ring");
constexpr int kPairSmem = 1024 + kPairStages * (kPairABytes + kPairBBytes) + kPairOutBytes + kPairBarBytes + kPairEntBytes;
static_assert(kPairSmem <= 227 * 1024, "pair kernel shared memory");

struct PairParams {
  void* out;
  int64_t ldo;
  int T, Nout, Kred;
  int n_mpairs, n_ntiles, group_m;
  int lora, r_pad;
  int lora_per_stage;  // LoRA items (S tile + B tile, kBM x r_pad each) one pipeline stage holds
  // K-split tail: when the last round of tiles would leave at least half of the pairs idle, each
  // of its tiles is computed by tail_parts pairs over consecutive K ranges.  Parts before the last
  // leave fp32 partial tiles in tail_partial and release their tail_flag words; the last part
  // (which also runs the tile's LoRA stages) adds them, in part order, before it stores.
  int tail_parts;         // 1: no split
  float* tail_partial;    // [slot][2 CTAs][4 epilogue warps][4 chunks][16 float4][32 rows]
  uint64_t* tail_flag;    // [slot][2 CTAs][4 epilogue warps] = gen once that partial is written
  uint32_t idesc_main, idesc_lora;
  uint32_t lora_layout, lora_sbo;
  // co-scheduled shrink: the first 2*n_shrink_pairs CTAs compute S_ext (P . A_slot^T) and publish
  // one ready flag per shrink unit; 0 = S_ext was produced by an earlier launch ...
  int n_shrink_pairs;
  // ... or, with shrink_prologue, every CTA runs its share of the shrink items first
  int shrink_prologue;
  int ab_fmt;
  void* s_ext;
  uint64_t* unit_ready;  // one flag per (unit, K half) item
  uint64_t gen;
  uint64_t ready_gen;    // value GEMM CTAs wait for on unit_ready: gen (a test hook may change it)
  // S_ext planes the LoRA stages sum: 1 = the full product; 2 = two K-half partial products
  // (written by the co-scheduled shrink), plane p starting at S map row p * s_plane_rows
  int s_planes, s_plane_rows;
  // optional second shrink job (own activations/slab/K), items after the first job's
  int job2, Kred2;
  void* s_ext2;
  Tables tb;
};

__device__ __forceinline__ void pair_raster(int t, const PairParams& p, int& mp, int& n) {
  const int per_group = p.group_m * p.n_ntiles;
  const int g = t / per_group;
  const int first = g * p.group_m;
  const int gsize = min(p.n_mpairs - first, p.group_m);
  const int r = t - g * per_group;
  mp = first + r % gsize;
  n = r / gsize;
}

// k-blocks the last part of a split tail tile runs beyond an even share (about the time an
// earlier part takes to write its fp32 partial tile and release it)
constexpr int kTailSkew = 6;

// Work units of one GEMM pair: the full tiles t = pair + k * n_pairs of the first `rounds`
// rounds, then at most one tail unit.  Tail unit v (counted from the last pair down) is part
// v % parts of tail tile v / parts; partial slot = tail tile * (parts - 1) + part.
struct PairSched {
  int rounds, tail_base, n_tail, parts;
};
__device__ __forceinline__ PairSched pair_sched(const PairParams& p, int n_pairs) {
  const int total = p.n_mpairs * p.n_ntiles;
  PairSched s;
  s.rounds = total / n_pairs;
  s.tail_base = s.rounds * n_pairs;
  const int rem = total - s.tail_base;
  s.parts = rem > 0 && p.tail_parts > 1 ? p.tail_parts : 1;
  s.n_tail = rem * s.parts;
  return s;
}
struct PairUnit {
  int mp, n;
  int kb0, kb1;   // K blocks of this unit
  int part;       // -1: whole tile; else part of a split tail tile
  int slot0;      // first partial slot of that tile
  bool last;      // stores the output (whole tile, or the tile's last part)
};
__device__ __forceinline__ PairUnit pair_unit(const PairParams& p, const PairSched& s, int pair, int n_pairs,
                                              int k, int nkb) {
  PairUnit u;
  if (k < s.rounds) {
    pair_raster(pair + k * n_pairs, p, u.mp, u.n);
    u.kb0 = 0;
    u.kb1 = nkb;
    u.part = -1;
    u.slot0 = 0;
    u.last = true;
    return u;
  }
  const int v = n_pairs - 1 - pair;
  const int j = v / s.parts, q = v - j * s.parts;
  pair_raster(s.tail_base + j, p, u.mp, u.n);
  // The last part (which adds the others' partials) gets `skew` extra k-blocks, so the earlier
  // parts' partial tiles are written while it still runs its k-loop.
  const int skew = min(kTailSkew, nkb / (4 * s.parts));
  u.kb0 = q * (nkb - skew) / s.parts;
  u.kb1 = q == s.parts - 1 ? nkb : (q + 1) * (nkb - skew) / s.parts;
  u.part = s.parts > 1 ? q : -1;
  u.slot0 = j * (s.parts - 1);
  u.last = q == s.parts - 1;
  return u;
}

// Bounded wait until ready[u] == gen for every u in [u0, u1) (acquire).
__device__ __forceinline__ bool wait_units_ready(const uint64_t* ready, int u0, int u1, uint64_t gen,
                                                 volatile int* abort_flag, int* err) {
  for (int u = u0; u < u1; ++u) {
    if (ld_acquire_u64(ready + u) == gen) continue;
    const uint64_t t0 = globaltimer_ns();
    const uint64_t limit = wait_limit(err);
    while (ld_acquire_u64(ready + u) != gen) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > limit) {
        record_error(err, kErrTimeoutFlag);
        *abort_flag = 1;
        return false;
      }
      __nanosleep(200);
    }
  }
  return true;
}

// Shrink role of the co-scheduled pair kernel, run by CTAs [0, 2*n_shrink_pairs) for the whole
// launch, or (kPrologue) by every CTA before its GEMM tiles: items (job, unit = row tile and
// <= 64/r_pad segment tiles, K half h) on single CTAs, S written straight from TMEM (scaled,
// masked per segment) as hi in plane h and lo in plane 2 + h (bf16/f16), then the item's ready
// flag is released.  The epilogue warps of CTA 0
// also write the all-zero block before releasing item 0.  In prologue mode the role keeps the
// TMEM allocation permit (the GEMM allocates after it) and its barriers are its own.
template <typename OutT, bool kPrologue>
__device__ __forceinline__ void pair_shrink_role(const PairParams& prm, const CUtensorMap& map_p,
                                                 const CUtensorMap& map_a, const CUtensorMap& map_p2,
                                                 const CUtensorMap& map_a2, uint8_t* sA, uint8_t* sB, uint64_t* full,
                                                 uint64_t* empty, uint64_t* tfull, uint64_t* tempty, uint64_t* drain,
                                                 uint64_t* pub, uint32_t* tmem_slot, volatile int* abort_flag) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Tables& tb = prm.tb;
  const int me = static_cast<int>(blockIdx.x), n_me = kPrologue ? static_cast<int>(gridDim.x) : 2 * prm.n_shrink_pairs;
  const int r_pad = prm.r_pad;
  // item = (job, unit, K half): half h of a job covers its k-blocks [h*half, min(nkb, (h+1)*half))
  const int n_items = (prm.job2 ? 4 : 2) * tb.n_units;
  const int64_t plane_elems = static_cast<int64_t>(prm.s_plane_rows) * r_pad;
  auto job_nkb = [&](int job) { return ((job ? prm.Kred2 : prm.Kred) + kBK - 1) / kBK; };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRoleStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    mbar_init(pub, 4);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_p);
    tma_prefetch_desc(&map_a);
    if (prm.job2) {
      tma_prefetch_desc(&map_p2);
      tma_prefetch_desc(&map_a2);
    }
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, 2 * kRoleChains * 64);
    if (!kPrologue) tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  if (!kPrologue) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, last_parity = 0;
      bool ok = true;
      for (int item = me; item < n_items && ok; item += n_me) {
        const int job = item >= 2 * tb.n_units ? 1 : 0;
        const int u = (item - job * 2 * tb.n_units) >> 1, h = item & 1;
        const CUtensorMap* mp = job ? &map_p2 : &map_p;
        const CUtensorMap* ma = job ? &map_a2 : &map_a;
        const int nkb = job_nkb(job), nkb_half = (nkb + 1) / 2;
        const int tile = tb.unit_tile(u), st0 = tb.unit_st0(u), nst = tb.unit_nst(u);
        int arow[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) arow[j] = j < nst ? tb.st_slot(st0 + j) * r_pad : 0;
        const uint32_t bytes = static_cast<uint32_t>(kPairABytes + nst * r_pad * kBK * 2);
        const int kb_end = min(nkb, (h + 1) * nkb_half);
        for (int kb = h * nkb_half; kb < kb_end; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, tb.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], bytes);
          uint8_t* sx = sA + stage * kRoleStageBytes;
          tma_load_2d(sx, mp, &full[stage], kb * kBK, tile * kBM);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (j < nst)
              tma_load_2d(sx + kPairABytes + j * r_pad * (kBK * 2), ma, &full[stage], kb * kBK, arow[j]);
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kRoleStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok)
        for (int s = 0; s < kRoleStages; ++s)
          if (issued_mask & (1u << s)) drain_wait(&full[s], (last_parity >> s) & 1u, tb.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued_any = false;
      const uint32_t a_base = smem_u32(sA);
      int it = 0;
      for (int item = me; item < n_items && ok; item += n_me, ++it) {
        const int job = item >= 2 * tb.n_units ? 1 : 0;
        const int u = (item - job * 2 * tb.n_units) >> 1, h = item & 1;
        const int nkb = job_nkb(job), nkb_half = (nkb + 1) / 2;
        const int N = tb.unit_nst(u) * r_pad;
        const uint32_t idesc = umma_idesc_f16(kBM, N, prm.ab_fmt, 0, 0);
        const int buf = it & 1;
        if (!mbar_wait(&tempty[buf], ((it >> 1) & 1) ^ 1, abort_flag, tb.err, kErrTimeoutAcc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * kRoleChains * 64);
        uint32_t started = 0;  // chains holding a partial sum
        int step = 0;
        const int kb_end = min(nkb, (h + 1) * nkb_half);
        for (int kb = h * nkb_half; kb < kb_end; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, tb.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = a_base + stage * kRoleStageBytes, b0 = a0 + kPairABytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k, ++step) {
            const int ch = step % kRoleChains;
            umma_f16(d + ch * 64, umma_sdesc(a0 + k * 32, 16, 1024, 2), umma_sdesc(b0 + k * 32, 16, 1024, 2), idesc,
                     (started >> ch) & 1u);
            started |= 1u << ch;
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == kRoleStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
      if (!ok && issued_any) {  // wait for in-flight MMAs before TMEM is released
        umma_commit(drain);
        drain_wait(drain, 0, tb.err);
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    OutT* s_ext = reinterpret_cast<OutT*>(prm.s_ext);
    if (me == 0)  // the all-zero segment tile of both planes, published with item 0
      for (int e = threadIdx.x - 64; e < kBM * r_pad; e += 128) {
        s_ext[static_cast<int64_t>(tb.n_segtiles) * kBM * r_pad + e] = cvt_out<OutT>(0.f);
        s_ext[plane_elems + static_cast<int64_t>(tb.n_segtiles) * kBM * r_pad + e] = cvt_out<OutT>(0.f);
      }
    int it = 0;
    for (int item = me; item < n_items; item += n_me, ++it) {
      const int job = item >= 2 * tb.n_units ? 1 : 0;
      const int u = (item - job * 2 * tb.n_units) >> 1, h = item & 1;
      const int nkb = job_nkb(job), nkb_half = (nkb + 1) / 2;
      const bool has_k = h * nkb_half < nkb;  // an empty K half contributes zeros
      OutT* s_out = reinterpret_cast<OutT*>(job ? prm.s_ext2 : prm.s_ext);
      const int st0 = tb.unit_st0(u), nst = tb.unit_nst(u);
      int lo[4], hi[4];
      float sc[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int st = st0 + min(j, nst - 1);
        lo[j] = tb.st_lo(st);
        hi[j] = tb.st_hi(st);
        sc[j] = tb.st_scale(st);
      }
      const int buf = it & 1;
      // chains the MMA thread started for this item (4 K steps per k-block)
      const int n_ch = has_k ? min(kRoleChains, 4 * (min(nkb, (h + 1) * nkb_half) - h * nkb_half)) : 0;
      if (!warp_wait(&tfull[buf], (it >> 1) & 1, abort_flag, tb.err, kErrTimeoutAcc)) break;
      tc_fence_after();
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * kRoleChains * 64);
      for (int j = 0; j < nst; ++j) {
        const bool in = has_k && row >= (j == 0 ? lo[0] : j == 1 ? lo[1] : j == 2 ? lo[2] : lo[3]) &&
                        row < (j == 0 ? hi[0] : j == 1 ? hi[1] : j == 2 ? hi[2] : hi[3]);
        const float scale = j == 0 ? sc[0] : j == 1 ? sc[1] : j == 2 ? sc[2] : sc[3];
        OutT* dst = s_out + h * plane_elems + (static_cast<int64_t>(st0 + j) * kBM + row) * r_pad;
        OutT* dst_lo = dst + 2 * plane_elems;
        for (int c = 0; c < r_pad; c += 16) {
          float f[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) f[e] = 0.f;
          for (int ch = 0; ch < n_ch; ++ch) {  // chains added in fixed order
            uint32_t v[16];
            tmem_ld16(tbase + ch * 64 + j * r_pad + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) f[e] += __uint_as_float(v[e]);
          }
#pragma unroll
          for (int e = 0; e < 16; ++e) f[e] = in ? scale * f[e] : 0.f;
          uint4 hi0, lo0, hi1, lo1;
          pack8_hi_lo<OutT>(f, hi0, lo0);
          pack8_hi_lo<OutT>(f + 8, hi1, lo1);
          *reinterpret_cast<uint4*>(dst + c) = hi0;
          *reinterpret_cast<uint4*>(dst + c + 8) = hi1;
          *reinterpret_cast<uint4*>(dst_lo + c) = lo0;
          *reinterpret_cast<uint4*>(dst_lo + c + 8) = lo1;
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
      // publish: each warp orders its stores, then thread 64 sees all four warps and releases
      __threadfence();
      __syncwarp();
      if (lane == 0) mbar_arrive(pub);
      if (warp == 2) {
        int ok = 1;
        if (lane == 0) {
          ok = mbar_wait(pub, static_cast<uint32_t>(it) & 1u, abort_flag, tb.err, kErrTimeoutAcc) ? 1 : 0;
          if (ok) {
            __threadfence();
            fence_proxy_async_global();
            st_release_u64(prm.unit_ready + item, prm.gen);
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (!kPrologue) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kRoleChains * 64);
  }
  if (kPrologue) __syncthreads();
}

template <bool kQMN, typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_p, const __grid_constant__ CUtensorMap map_q,
                        const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_l,
                        const __grid_constant__ CUtensorMap map_o, const __grid_constant__ CUtensorMap map_a,
                        const __grid_constant__ CUtensorMap map_p2, const __grid_constant__ CUtensorMap map_a2,
                        const PairParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kPairStages * kPairABytes;
  uint8_t* sOut = sB + kPairStages * kPairBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + kPairOutBytes);
  uint64_t* empty = full + kPairBars;
  uint64_t* tfull = empty + kPairBars;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* pub = drain + 1;  // shrink role: all epilogue warps finished writing a unit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pub + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // a shrink prologue's barriers: never re-initialized while its last arrivals may be in flight
  uint64_t* rfull = reinterpret_cast<uint64_t*>(sOut + kPairOutBytes + 256);
  uint64_t* rempty = rfull + kRoleStages;
  uint64_t* rtfull = rempty + kRoleStages;
  uint64_t* rtempty = rtfull + 2;
  uint64_t* rdrain = rtempty + 2;
  uint64_t* rpub = rdrain + 1;
  uint64_t* tail_bar = reinterpret_cast<uint64_t*>(sOut + kPairOutBytes + kPairTailBarOff);
  int* pair_ent = reinterpret_cast<int*>(sOut + kPairOutBytes + kPairBarBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (static_cast<int>(blockIdx.x) < 2 * prm.n_shrink_pairs) {
    pair_shrink_role<OutT, false>(prm, map_p, map_a, map_p2, map_a2, sA, sB, full, empty, tfull, tempty, drain, pub,
                                  tmem_slot, abort_flag);
    return;
  }
  if (prm.shrink_prologue && static_cast<int>(blockIdx.x) < (prm.job2 ? 4 : 2) * prm.tb.n_units)
    pair_shrink_role<OutT, true>(prm, map_p, map_a, map_p2, map_a2, sA, sB, rfull, rempty, rtfull, rtempty, rdrain,
                                 rpub, tmem_slot, abort_flag);
  const uint32_t crank = cluster_ctarank();  // 0: issues the MMAs
  const int pair = static_cast<int>(blockIdx.x >> 1) - prm.n_shrink_pairs;
  const int n_pairs = static_cast<int>(gridDim.x >> 1) - prm.n_shrink_pairs;
  const int nkb = (prm.Kred + kBK - 1) / kBK;
  const PairSched sched = pair_sched(prm, n_pairs);
  const int n_units = sched.rounds + (n_pairs - 1 - pair < sched.n_tail ? 1 : 0);
  const Tables& tb = prm.tb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // one arrive per epilogue warp of both CTAs
    }
    for (int b = 0; b < 8; ++b) mbar_init(&tail_bar[b], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_p);
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_o);
    if (prm.lora) {
      tma_prefetch_desc(&map_s);
      tma_prefetch_desc(&map_l);
    }
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t full_lead = map_to_cta(smem_u32(full), 0);
  const uint32_t tempty_lead = map_to_cta(smem_u32(tempty), 0);

  if (warp == 0) {
    // Lane 0 issues every copy.  Each tile's LoRA table entries (slot, segment tile) are fetched
    // by the whole warp before the tile's k-loop and staged in shared memory after it, so the
    // LoRA copies that follow the k-loop wait on no table load.
    int stage = 0;
    uint32_t phase = 0, issued_mask = 0, last_parity = 0;
    bool ok = true;
    const uint32_t main_bytes = 2u * (kPairABytes + kPairBBytes);
    const uint32_t lora_bytes = static_cast<uint32_t>(2 * 2 * kBM * prm.r_pad * 2);
    const int lora_item_bytes = kBM * prm.r_pad * 2;  // one operand of one item, this CTA
    const int32_t* st_of = tb.base + (crank ? tb.off_pl_b : tb.off_pl_a);
    const int32_t* pl_slot = tb.base + tb.off_pl_slot;
    for (int k = 0; k < n_units; ++k) {
      const PairUnit un = pair_unit(prm, sched, pair, n_pairs, k, nkb);
      const int mp = un.mp, n = un.n;
      const bool lora = prm.lora && un.last;  // the LoRA stages belong to the part that stores
      const int mtile = 2 * mp + static_cast<int>(crank);
      int pb = 0, pe = 0;
      int e_slot[kPairEntPerLane], e_st[kPairEntPerLane];
      if (lora) {  // fetched while the k-loop runs
        pb = ld_early(tb.base + tb.off_pair_lora + mp);
        pe = ld_early(tb.base + tb.off_pair_lora + mp + 1);
#pragma unroll
        for (int q = 0; q < kPairEntPerLane; ++q) {
          const int i = pb + lane + 32 * q;
          e_slot[q] = i < pe ? ld_early(pl_slot + i) : 0;
          e_st[q] = i < pe ? ld_early(st_of + i) : 0;
        }
      }
      // ready flags this tile's LoRA stages need, read early (relaxed) while the k-loop runs
      int it0 = 0, it1 = 0;
      uint64_t fl[9];
      if (lane == 0) {
        if (lora && (prm.n_shrink_pairs > 0 || prm.shrink_prologue)) {
          it0 = 2 * ld_early(tb.base + tb.off_tile_unit + 2 * mp);
          it1 = 2 * ld_early(tb.base + tb.off_tile_unit + min(2 * mp + 2, tb.n_tiles));
          fl[0] = ld_relaxed_u64(prm.unit_ready);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            fl[q + 1] = it0 + q < it1 ? ld_relaxed_u64(prm.unit_ready + it0 + q) : prm.ready_gen;
        }
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, tb.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (crank == 0) mbar_arrive_expect_tx(&full[stage], main_bytes);
          const uint32_t fb = full_lead + static_cast<uint32_t>(stage * 8);
          tma_load_2d_pair(sA + stage * kPairABytes, &map_p, fb, kb * kBK, mtile * kBM);
          if (kQMN) {
            tma_load_2d_pair(sB + stage * kPairBBytes, &map_q, fb, n * 256 + static_cast<int>(crank) * 128, kb * kBK);
            tma_load_2d_pair(sB + stage * kPairBBytes + 64 * kBK * 2, &map_q, fb,
                             n * 256 + static_cast<int>(crank) * 128 + 64, kb * kBK);
          } else {
            tma_load_2d_pair(sB + stage * kPairBBytes, &map_q, fb, kb * kBK, n * 256 + static_cast<int>(crank) * 128);
          }
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      if (!lora) continue;
      // lane 0 issued the previous tile's LoRA copies before this k-loop: the entries are free
#pragma unroll
      for (int q = 0; q < kPairEntPerLane; ++q) {
        const int e = lane + 32 * q;
        if (pb + e < pe) {
          pair_ent[2 * e] = e_slot[q];
          pair_ent[2 * e + 1] = e_st[q];
        }
      }
      __syncwarp();
      if (lane == 0) {
        if ((prm.n_shrink_pairs > 0 || prm.shrink_prologue) && pe > pb) {  // S_ext of both row tiles (and the zero block) published?
          bool seen = it1 - it0 <= 8;
#pragma unroll
          for (int q = 0; q < 9; ++q) seen = seen && fl[q] == prm.ready_gen;
          if (seen) {
            fence_acquire_gpu();  // the early loads saw every release: acquire them
          } else if (!wait_units_ready(prm.unit_ready, 0, 1, prm.ready_gen, abort_flag, tb.err) ||
                     !wait_units_ready(prm.unit_ready, it0, it1, prm.ready_gen, abort_flag, tb.err)) {
            ok = false;
          }
          fence_proxy_async_global();
        }
        // LoRA items (pair-table entry, S plane), entry-major, packed lora_per_stage to a stage
        const int n_items = (pe - pb) * prm.s_planes;
        for (int i0 = 0; i0 < n_items && ok; i0 += prm.lora_per_stage) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, tb.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int cnt = min(prm.lora_per_stage, n_items - i0);
          if (crank == 0) mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(cnt) * lora_bytes);
          const uint32_t fb = full_lead + static_cast<uint32_t>(stage * 8);
          for (int c = 0; c < cnt; ++c) {
            const int item = i0 + c;
            const int e = item / prm.s_planes, pl = item - e * prm.s_planes;
            const bool staged = e < 32 * kPairEntPerLane;
            const int slot = staged ? pair_ent[2 * e] : pl_slot[pb + e];
            const int st = staged ? pair_ent[2 * e + 1] : st_of[pb + e];
            tma_load_2d_pair(sA + stage * kPairABytes + c * lora_item_bytes, &map_s, fb, 0,
                             pl * prm.s_plane_rows + st * kBM);
            tma_load_2d_pair(sB + stage * kPairBBytes + c * lora_item_bytes, &map_l, fb, 0,
                             slot * prm.Nout + n * 256 + static_cast<int>(crank) * 128);
          }
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
    }
    if (lane == 0 && !ok && crank == 0)  // copies of both CTAs complete on the even CTA's barriers
      for (int s = 0; s < kPairStages; ++s)
        if (issued_mask & (1u << s)) drain_wait(&full[s], (last_parity >> s) & 1u, tb.err);
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && crank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued_any = false;
      const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
      const uint32_t empty_local = smem_u32(empty), tfull_local = smem_u32(tfull);  // same offsets in both CTAs
      const uint32_t lora_item_bytes = static_cast<uint32_t>(kBM * prm.r_pad * 2);
      int it = 0;
      for (int k = 0; k < n_units && ok; ++k, ++it) {
        const PairUnit un = pair_unit(prm, sched, pair, n_pairs, k, nkb);
        const int mp = un.mp;
        const int buf = it & 1;
        int n_lora = 0;
        if (prm.lora && un.last)
          n_lora = (ld_early(tb.base + tb.off_pair_lora + mp + 1) - ld_early(tb.base + tb.off_pair_lora + mp)) *
                   prm.s_planes;
        if (!mbar_wait(&tempty[buf], ((it >> 1) & 1) ^ 1, abort_flag, tb.err, kErrTimeoutAcc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * 256);
        uint32_t acc = 0;
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, tb.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = a_base + stage * kPairABytes, b0 = b_base + stage * kPairBBytes;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t adesc = umma_sdesc(a0 + k * 32, 16, 1024, 2);
            const uint64_t bdesc = kQMN ? umma_sdesc(b0 + k * 2048, 64 * kBK * 2, 1024, 2)
                                        : umma_sdesc(b0 + k * 32, 16, 1024, 2);
            umma_f16_pair(d, adesc, bdesc, prm.idesc_main, acc);
            acc = 1;
          }
          issued_any = true;
          umma_commit_pair_both(empty_local + stage * 8);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        for (int j = 0; ok && j < n_lora; j += prm.lora_per_stage) {
          if (!mbar_wait(&full[stage], phase, abort_flag, tb.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int cnt = min(prm.lora_per_stage, n_lora - j);
          for (int c = 0; c < cnt; ++c) {
            const uint32_t a0 = a_base + stage * kPairABytes + c * lora_item_bytes;
            const uint32_t b0 = b_base + stage * kPairBBytes + c * lora_item_bytes;
            for (int k = 0; k < prm.r_pad / 16; ++k) {
              const uint64_t adesc = umma_sdesc(a0 + k * 32, 16, prm.lora_sbo, prm.lora_layout);
              const uint64_t bdesc = umma_sdesc(b0 + k * 32, 16, prm.lora_sbo, prm.lora_layout);
              umma_f16_pair(d, adesc, bdesc, prm.idesc_lora, acc);
              acc = 1;
            }
          }
          issued_any = true;
          umma_commit_pair_both(empty_local + stage * 8);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_both(tfull_local + buf * 8);
      }
      if (!ok && issued_any) {
        umma_commit_pair(map_to_cta(smem_u32(drain), 0));
        drain_wait(drain, 0, tb.err);
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    int it = 0;
    int n_stores = 0;
    const int wslot = static_cast<int>(crank) * 4 + q;  // this warp's 32 rows of a partial tile
    uint32_t tail_pending = 0, tail_par = 0;  // lane 0: partial-tile copies in flight per buffer, their parity
    for (int k = 0; k < n_units; ++k, ++it) {
      const PairUnit un = pair_unit(prm, sched, pair, n_pairs, k, nkb);
      const int mp = un.mp, n = un.n;
      const int buf = it & 1;
      if (!warp_wait(&tfull[buf], (it >> 1) & 1, abort_flag, tb.err, kErrTimeoutAcc)) break;
      tc_fence_after();
      // Split tail tiles move their fp32 partials through this warp's share of the ring (idle in
      // the pair's last unit, which a tail unit always is).  An earlier part stages each chunk
      // there and bulk-copies it out.  The last part copies the earlier parts' chunks in: all
      // four at once after one earlier part, else chunk c into buffer c & 1 while c - 1 is added.
      const bool tail_last = un.part > 0 && un.last;
      uint8_t* tail_w = sA + q * (2 * kTailBufBytes);  // this warp's share of the ring
      auto tail_chunk = [&](int c, int p) {  // chunk c of earlier part p in shared memory
        return tail_w + (un.part == 1 ? c : (c & 1) * un.part + p) * kTailChunkBytes;
      };
      auto tail_src = [&](int c, int p) {  // ... and in the partial tiles
        return prm.tail_partial + (static_cast<size_t>(un.slot0 + p) * 8 + wslot) * (4 * 2048) +
               static_cast<size_t>(c) * 2048;
      };
      auto tail_load = [&](int c) {  // lane 0: chunk c, or all chunks after one earlier part
        const int nc = un.part == 1 ? 256 / 64 : 1;
        uint64_t* bar = tail_bar + 2 * q + (c & 1);
        mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nc * un.part * kTailChunkBytes));
        for (int cc = c; cc < c + nc; ++cc)
          for (int p = 0; p < un.part; ++p) bulk_load(tail_chunk(cc, p), tail_src(cc, p), kTailChunkBytes, bar);
        tail_pending |= 1u << (c & 1);
        tail_par = (tail_par & ~(1u << (c & 1))) | (static_cast<uint32_t>((c >> 1) & 1) << (c & 1));
      };
      if (tail_last) {  // the earlier parts of this tile have published their partials?
        int ok = 1;
        if (lane == 0) {
          for (int p = 0; p < un.part && ok; ++p)
            ok = wait_units_ready(prm.tail_flag, (un.slot0 + p) * 8 + wslot, (un.slot0 + p) * 8 + wslot + 1,
                                  prm.gen, abort_flag, tb.err) ? 1 : 0;
          if (ok) {
            fence_proxy_async_global();  // the acquired partials, read by the copy engine
            tail_load(0);
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        __syncwarp();
      }
      bool tail_ok = true;
      // rows [row0, row0+32) of this CTA's tile: TMEM -> registers -> swizzled staging -> TMA store
      const int row0 = (2 * mp + static_cast<int>(crank)) * kBM + q * 32;
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * 256);
      uint8_t* stage_w = sOut + (warp - 2) * (2 * 32 * 64 * 2);
      // The pair's last unit: the ring is idle (every MMA of the pair is done), so each warp
      // stages all four chunks there, after its partial-tile buffers, and no store waits for an
      // earlier one to have read its buffer.
      const bool ring_stage = k == n_units - 1 && un.part <= 2;
      uint8_t* ring_w = tail_w + (tail_last ? (un.part == 1 ? 4 : 2 * un.part) * kTailChunkBytes : 0);
#pragma unroll 1
      for (int c = 0; c < 256 / 64; ++c) {
        uint32_t v[64];
        tmem_ld32(tbase + c * 64, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(tbase + c * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_ld();
        if (c == 256 / 64 - 1) {  // accumulator fully read: hand it back to the MMA thread
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(tempty_lead + buf * 8);
        }
        if (un.part >= 0) {
          // partial tiles: slot, warp rows, 64-column chunk c; float4 i of lane (row) l at
          // i * 32 + l, so each warp-wide access covers 512 contiguous bytes
          const size_t chunk_off = static_cast<size_t>(c) * 2048;
          if (!un.last) {
            float4* stg = reinterpret_cast<float4*>(tail_w + c * kTailChunkBytes) + lane;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              stg[i * 32] = make_float4(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1]),
                                        __uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3]));
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              bulk_store(prm.tail_partial + (static_cast<size_t>(un.slot0 + un.part) * 8 + wslot) * (4 * 2048) +
                             chunk_off,
                         tail_w + c * kTailChunkBytes, kTailChunkBytes);
              bulk_commit();
            }
            continue;
          }
          if (un.part > 1 && lane == 0 && c + 1 < 256 / 64) {  // buffer (c + 1) & 1 was read for chunk c - 1
            fence_proxy_async_smem();
            tail_load(c + 1);
          }
          if (un.part > 1 || c == 0) {
            // every lane acquires the copy's completion (bounded wait) before reading the buffer
            tail_ok = __all_sync(0xffffffffu, mbar_wait(tail_bar + 2 * q + (c & 1), (c >> 1) & 1, abort_flag, tb.err,
                                                        kErrTimeoutFull));
            if (!tail_ok) break;
            if (lane == 0) tail_pending &= ~(1u << (c & 1));
          }
          for (int p = 0; p < un.part; ++p) {  // add the earlier parts in part order
            const float4* src = reinterpret_cast<const float4*>(tail_chunk(c, p)) + lane;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float4 f = src[i * 32];
              v[4 * i] = __float_as_uint(__uint_as_float(v[4 * i]) + f.x);
              v[4 * i + 1] = __float_as_uint(__uint_as_float(v[4 * i + 1]) + f.y);
              v[4 * i + 2] = __float_as_uint(__uint_as_float(v[4 * i + 2]) + f.z);
              v[4 * i + 3] = __float_as_uint(__uint_as_float(v[4 * i + 3]) + f.w);
            }
          }
          __syncwarp();  // the buffer is free for the copy of chunk c + 2
        }
        const int col0 = n * 256 + c * 64;
        if (row0 >= prm.T || col0 >= prm.Nout) continue;
        uint8_t* sbuf = ring_stage ? ring_w + c * (32 * 64 * 2) : stage_w + (n_stores & 1) * (32 * 64 * 2);
        if (!ring_stage && lane == 0) bulk_wait_read<1>();  // the store that used this buffer has read it
        __syncwarp();
        uint8_t* rowp = sbuf + lane * 128;
#pragma unroll
        for (int g = 0; g < 8; ++g) {  // 16-byte granule g of the row goes to slot g ^ (row % 8)
          uint4 pk;
          pk.x = pack2<OutT>(__uint_as_float(v[g * 8 + 0]), __uint_as_float(v[g * 8 + 1]));
          pk.y = pack2<OutT>(__uint_as_float(v[g * 8 + 2]), __uint_as_float(v[g * 8 + 3]));
          pk.z = pack2<OutT>(__uint_as_float(v[g * 8 + 4]), __uint_as_float(v[g * 8 + 5]));
          pk.w = pack2<OutT>(__uint_as_float(v[g * 8 + 6]), __uint_as_float(v[g * 8 + 7]));
          *reinterpret_cast<uint4*>(rowp + ((g ^ (lane & 7)) << 4)) = pk;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_o, sbuf, col0, row0);
          bulk_commit();
        }
        ++n_stores;
      }
      if (!tail_ok) break;
      if (un.part >= 0 && !un.last) {  // publish this warp's share of the partial tile
        if (lane == 0) {
          bulk_wait_all();             // the bulk copies have written it
          fence_proxy_async_global();  // ... ordered before the release
          __threadfence();
          st_release_u64(prm.tail_flag + (un.slot0 + un.part) * 8 + wslot, prm.gen);
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      bulk_wait_all();
      for (int b = 0; b < 2; ++b)  // partial-tile copies still in flight after an abort
        if (tail_pending & (1u << b)) drain_wait(tail_bar + 2 * q + b, (tail_par >> b) & 1u, tb.err);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

// ========================================================================== shrink
struct ShrinkParams {
  void* s_ext;           // hi plane; the lo plane follows at + plane_elems
  int64_t plane_elems;
  int ab_fmt;
  int Kred;
  int kb_per_split;
  int cluster;
  int r_pad;
  Tables tb;
};

constexpr int kShrABytes = kBM * kBK * 2;    // 16 KB
constexpr int kShrBBytes = 64 * kBK * 2;     // N <= 64 rows (unit = <= 64 / r_pad segment tiles)
constexpr int kShrSmem = 1024 + kShrStages * (kShrABytes + kShrBBytes) + 256;
constexpr int kPartLd = kBM + 1;             // column-major partial sums, odd stride
constexpr int kMaxShrCluster = 4;             // K split across at most 4 CTAs (all resident at once)
static_assert(64 * kPartLd * 4 <= kShrStages * (kShrABytes + kShrBBytes), "partials must fit the stage area");

template <typename OutT>
__global__ void __launch_bounds__(kThreads, 1)
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
  int* seg_lo = reinterpret_cast<int*>(tmem_slot + 2);  // per segment tile of the unit (<= 4)
  int* seg_hi = seg_lo + 8;
  float* seg_scale = reinterpret_cast<float*>(seg_hi + 8);

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
  if (threadIdx.x >= 32 && threadIdx.x < 32 + nst) {  // segment bounds for the reduction step
    const int j = threadIdx.x - 32;
    seg_lo[j] = tb.st_lo(st0 + j);
    seg_hi[j] = tb.st_hi(st0 + j);
    seg_scale[j] = tb.st_scale(st0 + j);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, kShrChains * 64);
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
      int arow[4];  // first packed-A row of every segment's adapter, read once
#pragma unroll
      for (int j = 0; j < 4; ++j) arow[j] = j < nst ? tb.st_slot(st0 + j) * r_pad : 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, prm.tb.err, kErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[stage], bytes);
        tma_load_2d(sA + stage * kShrABytes, &map_p, &full[stage], kb * kBK, tile * kBM);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (j < nst)
            tma_load_2d(sB + stage * kShrBBytes + j * r_pad * (kBK * 2), &map_a, &full[stage], kb * kBK, arow[j]);
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
      uint32_t started = 0;  // accumulation chains holding a partial sum
      int step = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, prm.tb.err, kErrTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = a_base + stage * kShrABytes, b0 = b_base + stage * kShrBBytes;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k, ++step) {
          const int ch = step % kShrChains;
          umma_f16(tmem_base + ch * 64, umma_sdesc(a0 + k * 32, 16, 1024, 2), umma_sdesc(b0 + k * 32, 16, 1024, 2),
                   idesc, (started >> ch) & 1u);
          started |= 1u << ch;
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
      const int n_ch = min(kShrChains, 4 * (kb1 - kb0));
      for (int c = 0; c < N; c += 16) {
        float f[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) f[jj] = 0.f;
        for (int ch = 0; ch < n_ch; ++ch) {  // chains added in fixed order
          uint32_t v[16];
          tmem_ld16(tbase + ch * 64 + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) f[jj] += __uint_as_float(v[jj]);
        }
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) partial[(c + jj) * kPartLd + row] = f[jj];
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
      float part[kMaxShrCluster];
#pragma unroll
      for (int qr = 0; qr < kMaxShrCluster; ++qr)  // issue every peer load before summing
        part[qr] = qr < prm.cluster ? ld_cluster_f32(map_to_cta(part_base + off, qr)) : 0.f;
      float sum = 0.f;
#pragma unroll
      for (int qr = 0; qr < kMaxShrCluster; ++qr) sum += part[qr];
      const int j = col / r_pad, jj = col - j * r_pad;
      const int st = st0 + j;
      const bool in = row >= seg_lo[j] && row < seg_hi[j];
      const float v = in ? seg_scale[j] * sum : 0.f;
      OutT hi, lo;
      split_hi_lo<OutT>(v, hi, lo);
      const int64_t idx = (static_cast<int64_t>(st) * kBM + row) * r_pad + jj;
      out[idx] = hi;
      out[prm.plane_elems + idx] = lo;
    }
  }

  if (blockIdx.x == 0) {  // the all-zero segment tile the pair GEMM pads odd row tiles with
    OutT* zero = reinterpret_cast<OutT*>(prm.s_ext) + static_cast<int64_t>(tb.n_segtiles) * kBM * r_pad;
    for (int e = threadIdx.x; e < kBM * r_pad; e += kThreads) zero[e] = cvt_out<OutT>(0.f);
  }

  // keep this CTA's shared memory alive until every peer has read it
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kShrChains * 64);
  }
}

// ========================================================================== gram (dA / dB)
// grad[slot] = sum over the slot's segment tiles of D_tile^T . S_ext[seg] for up to two jobs in one
// launch (the backward's dB: D = g, C = N, S = s.x.A^T; and dA: D = x, C = K, S = s.g.B).
struct GramJob {
  void* out;
  int C, n_cblk, transpose_out, out_f32;
};
struct GramParams {
  GramJob job[2];
  int n_jobs;
  int planes, s_plane_rows;  // S_ext planes summed (2: K-half partial products)
  int r_pad;
  int n_stages, stage_bytes;  // ring of stages: 128x128 D tile, then `planes` S tiles
  // One MMA per 16-row K step covers every plane (N = planes * r_pad: the planes are consecutive
  // MN chunks of the B operand).  K steps rotate over `chains` accumulators so that consecutive
  // MMAs do not wait on each other; the epilogue adds chains and planes in fixed order.
  int chains, acc_cols, tmem_cols;  // acc_cols = chains * planes * r_pad per buffer
  int n_bufs;                       // accumulator buffers (<= kGramMaxBufs, n_bufs * acc_cols <= tmem_cols)
  uint32_t idesc;
  uint32_t s_layout, s_sbo, s_kstep;
  // Load balance: a slot with more than `cap` segment tiles is split into parts of about equal
  // size (0: never split).  Parts of a split slot write fp32 partial sums; per (job, slot, column
  // block, epilogue warp) the last part to arrive adds them up in part order.
  int cap;
  float* partial;      // [kGramMaxPartials][128][r_pad]
  uint64_t* counters;  // [kGramMaxCounters][4] arrival words, generation in the high half
  uint32_t gen32;
  GramPeer peer;       // exchange of spanning adapters' blocks with the other GPUs (world 0: none)
  Tables tb;
};

constexpr int kGramDBytes = kBM * 128 * 2;  // 128 rows x 128 columns
constexpr int kGramMaxStages = 8;
constexpr int kGramRingBytes = 3 * (kGramDBytes + 2 * kBM * 64 * 2);  // 3 stages at r_pad 64 with 2 planes

// Work units of one CTA (job, slot part, column block), staged in shared memory once with the
// segment tiles each one streams, so no role waits on a dependent table load per unit.
constexpr int kGramMaxUnits = 64;
constexpr int kGramMaxBufs = 8;    // TMEM accumulators (as many as 512 columns hold)
struct GramUnit {
  int job, slot, b, e, rank, rank_prefix, cb;
  int parts;  // parts of this slot (1: written straight from TMEM)
  int pid;    // partial block of this part
  int pbase;  // partial block of part 0; part p is pbase + p * n_cblk
  int cid;    // counter row (x4 warps)
};
// Per slot position (slot_order index), read from the table once per CTA: the slot's metadata and,
// per job, prefix sums of parts, split parts and split slots.  Only when n_slots <= kGramMaxSlots
// (`cached`); otherwise units are decoded from the table and never split.
struct GramSlotPrefix {
  int slot[kGramMaxSlots], b0[kGramMaxSlots], nst[kGramMaxSlots], rank[kGramMaxSlots], rprefix[kGramMaxSlots];
  int part[2][kGramMaxSlots + 1];
  int split_part[2][kGramMaxSlots + 1];
  int split_slot[2][kGramMaxSlots + 1];
  int units[2];           // units of each job
  int pid_off, cid_off;   // job 1's partial blocks and counter rows follow job 0's
  int use_split, cached;
};
// Warps of the gram kernel: TMA producer, MMA issuer, then two sets of four epilogue warps that
// drain alternate units (set s the units k = s, s + 2, ... through accumulator buffer s), so one
// set's tensor-memory loads and global stores overlap the other's.
constexpr int kGramEpiSets = 2;
constexpr int kGramThreads = 64 + kGramEpiSets * 128;
// epilogue staging of a [rank, C] block in the input type: per epilogue warp 16 ranks x 32 columns
constexpr int kGramStageTrBytes = kGramEpiSets * 4 * 16 * 32 * 2;
constexpr int kGramSmem = 1024 + kGramRingBytes + kGramMaxUnits * static_cast<int>(sizeof(GramUnit)) +
                          static_cast<int>(sizeof(GramSlotPrefix)) + kGramStageTrBytes + 512;
static_assert(kGramSmem <= 227 * 1024, "gram kernel shared memory");

// Unit k of the combined list (job 0's units, then job 1's): part k / n_cblk of the job's parts,
// listed slot after slot in slot_order, column block k % n_cblk.
__device__ __forceinline__ GramUnit gram_unit(const GramParams& prm, const GramSlotPrefix& sp, int k) {
  const Tables& tb = prm.tb;
  GramUnit g;
  g.job = k < sp.units[0] ? 0 : 1;
  const int kl = k - (g.job ? sp.units[0] : 0);
  const int n_cblk = prm.job[g.job].n_cblk;
  const int pg = kl / n_cblk;
  g.cb = kl - pg * n_cblk;
  g.parts = 1;
  g.pid = g.pbase = g.cid = 0;
  if (!sp.cached) {
    g.slot = tb.slot_order(pg);
    g.b = tb.slot_st(g.slot);
    g.e = tb.slot_st(g.slot + 1);
    g.rank = tb.slot_rank(g.slot);
    g.rank_prefix = tb.rank_prefix(g.slot);
    return g;
  }
  int pos = pg, p = 0;
  if (sp.use_split) {  // last slot position whose first part is <= pg
    const int* part = sp.part[g.job];
    int lo = 0, hi = tb.n_slots - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (part[mid] <= pg) lo = mid;
      else hi = mid - 1;
    }
    pos = lo;
    p = pg - part[pos];
    g.parts = part[pos + 1] - part[pos];
  }
  g.slot = sp.slot[pos];
  const int b0 = sp.b0[pos], nst = sp.nst[pos];
  g.b = b0 + static_cast<int>(static_cast<int64_t>(p) * nst / g.parts);
  g.e = b0 + static_cast<int>(static_cast<int64_t>(p + 1) * nst / g.parts);
  g.rank = sp.rank[pos];
  g.rank_prefix = sp.rprefix[pos];
  if (g.parts > 1) {
    g.pbase = (g.job ? sp.pid_off : 0) + sp.split_part[g.job][pos] * n_cblk + g.cb;
    g.pid = g.pbase + p * n_cblk;
    g.cid = (g.job ? sp.cid_off : 0) + sp.split_slot[g.job][pos] * n_cblk + g.cb;
  }
  return g;
}

// k-th unit of CTA `me` among `G`: units are dealt zig-zag (0..G-1, then G-1..0, ...) so that,
// listed largest first, every CTA gets a similar share.
__device__ __forceinline__ int gram_zigzag(int r, int me, int G) { return r * G + ((r & 1) ? G - 1 - me : me); }

// Exchange entries (see peer_half_bytes): entry (src, blk, jp, col) holds elements 2jp and 2jp+1 of
// column col of block blk as rank src computed it, each as {gen << 32 | float bits}.  A warp's 32
// columns of one pair are 512 contiguous bytes.
__device__ __forceinline__ size_t span_entry(const GramPeer& pr, int src, int blk, int jp, int col) {
  return ((static_cast<size_t>(src) * pr.n_blocks + blk) * (pr.xr / 2) + jp) * 128 + col;
}
// Elements j0 .. j0+15 of this lane's column of block `blk`, into every rank's exchange buffer
// (this rank's entries there); plain stores, no fence: each word carries the generation.
__device__ __forceinline__ void span_put16(const GramPeer& pr, size_t half, int blk, int col, int j0, const float* v) {
  const uint64_t tag = static_cast<uint64_t>(static_cast<uint32_t>(pr.gen)) << 32;
  const size_t e0 = span_entry(pr, pr.rank, blk, j0 / 2, col);
  for (int d = 0; d < pr.world; ++d) {
    uint8_t* base = pr.xbuf[d] + half;
#pragma unroll 2
    for (int t = 0; t < 8; ++t)
      st_volatile_v2u64(base + (e0 + static_cast<size_t>(t) * 128) * 16, tag | __float_as_uint(v[2 * t]),
                        tag | __float_as_uint(v[2 * t + 1]));
  }
}
// Adds rank src's elements j0 .. j0+15 of this lane's column of block `blk` (local exchange buffer)
// to acc, once they carry this call's generation: all eight entries are loaded at once, those not
// yet written are polled (bounded).  False after a timeout or an abort.
__device__ __forceinline__ bool span_add16(const GramPeer& pr, const uint8_t* base, int src, int blk, int col, int j0,
                                           float* acc, volatile int* abort_flag, int* err) {
  const uint32_t gen = static_cast<uint32_t>(pr.gen);
  const uint8_t* p = base + span_entry(pr, src, blk, j0 / 2, col) * 16;
  uint64_t w[16];
#pragma unroll
  for (int t = 0; t < 8; ++t) ld_volatile_v2u64(p + static_cast<size_t>(t) * 128 * 16, w[2 * t], w[2 * t + 1]);
  bool ready = true;
#pragma unroll
  for (int i = 0; i < 16; ++i) ready = ready && static_cast<uint32_t>(w[i] >> 32) == gen;
  if (!ready) {
    const uint64_t t0 = globaltimer_ns();
    const uint64_t limit = wait_limit(err);
#pragma unroll
    for (int t = 0; t < 8; ++t)
      while (static_cast<uint32_t>(w[2 * t] >> 32) != gen || static_cast<uint32_t>(w[2 * t + 1] >> 32) != gen) {
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > limit) {
          record_error(err, kErrTimeoutFlag);
          *abort_flag = 1;
          return false;
        }
        __nanosleep(128);
        ld_volatile_v2u64(p + static_cast<size_t>(t) * 128 * 16, w[2 * t], w[2 * t + 1]);
      }
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] += __uint_as_float(static_cast<uint32_t>(w[i]));
  return true;
}

// Arrival on a per-launch counter word (generation in the high 32 bits); returns the count after
// this arrival, or 0 after a bounded number of failed tries (error recorded).
__device__ __forceinline__ uint32_t gen_arrive(uint64_t* ctr, uint32_t gen32, int* err) {
  unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(ctr);
  for (int i = 0; i < (1 << 20); ++i) {
    const bool same = static_cast<uint32_t>(cur >> 32) == gen32;
    const unsigned long long next = same ? cur + 1ull : ((static_cast<unsigned long long>(gen32) << 32) | 1ull);
    const unsigned long long seen = atomicCAS(reinterpret_cast<unsigned long long*>(ctr), cur, next);
    if (seen == cur) return static_cast<uint32_t>(next);
    cur = seen;
  }
  record_error(err, kErrTimeoutFlag);
  return 0;
}

template <typename OutT>
__global__ void __launch_bounds__(kGramThreads)
    tc_gram_kernel(const __grid_constant__ CUtensorMap map_d0, const __grid_constant__ CUtensorMap map_s0,
                   const __grid_constant__ CUtensorMap map_d1, const __grid_constant__ CUtensorMap map_s1,
                   const GramParams prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  GramUnit* units = reinterpret_cast<GramUnit*>(ring + kGramRingBytes);
  GramSlotPrefix& sp = *reinterpret_cast<GramSlotPrefix*>(units + kGramMaxUnits);
  OutT* stage_tr = reinterpret_cast<OutT*>((reinterpret_cast<uintptr_t>(&sp + 1) + 15) & ~uintptr_t(15));
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(stage_tr) + kGramStageTrBytes);
  uint64_t* empty = full + kGramMaxStages;
  uint64_t* tfull = empty + kGramMaxStages;
  uint64_t* tempty = tfull + kGramMaxBufs;
  uint64_t* drain = tempty + kGramMaxBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Tables& tb = prm.tb;
  const int me = static_cast<int>(blockIdx.x), G = static_cast<int>(gridDim.x);
  const int r_pad = prm.r_pad;
  const int n_stages = prm.n_stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < prm.n_bufs; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_d0);
    tma_prefetch_desc(&map_s0);
    if (prm.n_jobs > 1) {
      tma_prefetch_desc(&map_d1);
      tma_prefetch_desc(&map_s1);
    }
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(tmem_slot, static_cast<uint32_t>(prm.tmem_cols));
    tmem_relinquish();
  }

  const bool cached = tb.n_slots <= kGramMaxSlots;
  // Every thread reads table entries in parallel (one short chain of dependent loads each): each
  // slot position's metadata.
  if (cached)
    for (int i = threadIdx.x; i < tb.n_slots; i += kGramThreads) {
      const int sl = tb.slot_order(i);
      const int b0 = tb.slot_st(sl);
      sp.slot[i] = sl;
      sp.b0[i] = b0;
      sp.nst[i] = tb.slot_st(sl + 1) - b0;
      sp.rank[i] = tb.slot_rank(sl);
      sp.rprefix[i] = tb.rank_prefix(sl);
    }
  __syncthreads();
  // Parts per slot position (warp 2, from shared memory): slots with more than `cap` segment
  // tiles are split, unless the partial blocks or counters that needs would not fit; every CTA
  // decides the same way.
  if (warp == 2) {
    int tp[2] = {0, 0}, ts[2] = {0, 0}, tss[2] = {0, 0};
    const bool try_split = cached && prm.cap > 0 && prm.partial != nullptr;
    if (cached) {
      for (int i0 = 0; i0 < tb.n_slots; i0 += 32) {
        const int i = i0 + lane;
        const int nst = i < tb.n_slots ? sp.nst[i] : 0;
        // parts are the same for both jobs (one cap); lanes past the end count nothing
        const int P = i >= tb.n_slots ? 0 : (try_split && nst > prm.cap) ? (nst + prm.cap - 1) / prm.cap : 1;
        int a = P, b = P > 1 ? P : 0, c = P > 1 ? 1 : 0;  // inclusive warp scans
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int ua = __shfl_up_sync(0xffffffffu, a, d), ub = __shfl_up_sync(0xffffffffu, b, d),
                    uc = __shfl_up_sync(0xffffffffu, c, d);
          if (lane >= d) {
            a += ua;
            b += ub;
            c += uc;
          }
        }
        if (i < tb.n_slots)
          for (int j = 0; j < 2; ++j) {
            sp.part[j][i] = tp[j] + a - P;
            sp.split_part[j][i] = ts[j] + b - (P > 1 ? P : 0);
            sp.split_slot[j][i] = tss[j] + c - (P > 1 ? 1 : 0);
          }
        const int ta = __shfl_sync(0xffffffffu, a, 31), tb2 = __shfl_sync(0xffffffffu, b, 31),
                  tc = __shfl_sync(0xffffffffu, c, 31);
        for (int j = 0; j < 2; ++j) {
          tp[j] += ta;
          ts[j] += tb2;
          tss[j] += tc;
        }
      }
    }
    int64_t need_p = 0, need_c = 0;
    for (int j = 0; j < prm.n_jobs; ++j) {
      need_p += static_cast<int64_t>(ts[j]) * prm.job[j].n_cblk;
      need_c += static_cast<int64_t>(tss[j]) * prm.job[j].n_cblk;
    }
    const bool fits = try_split && ts[0] > 0 && need_p <= kGramMaxPartials && need_c <= kGramMaxCounters;
    if (!fits && cached) {  // one part per slot
      for (int i = lane; i < tb.n_slots; i += 32) sp.part[0][i] = sp.part[1][i] = i;
      tp[0] = tp[1] = tb.n_slots;
    }
    if (lane == 0) {
      sp.cached = cached ? 1 : 0;
      sp.use_split = fits ? 1 : 0;
      if (cached) sp.part[0][tb.n_slots] = sp.part[1][tb.n_slots] = tp[0];
      const int slots_or_parts = cached ? tp[0] : tb.n_slots;
      sp.units[0] = slots_or_parts * prm.job[0].n_cblk;
      sp.units[1] = prm.n_jobs > 1 ? slots_or_parts * prm.job[1].n_cblk : 0;
      sp.pid_off = ts[0] * prm.job[0].n_cblk;
      sp.cid_off = tss[0] * prm.job[0].n_cblk;
    }
  }
  __syncthreads();
  const int total = sp.units[0] + sp.units[1];
  int n_mine = 0;
  for (int r = 0; r * G < total; ++r) n_mine += gram_zigzag(r, me, G) < total ? 1 : 0;
  const int n_staged = n_mine < kGramMaxUnits ? n_mine : kGramMaxUnits;
  if (warp >= 2) {  // stage this CTA's units
    for (int k = threadIdx.x - 64; k < n_staged; k += kGramThreads - 64)
      units[k] = gram_unit(prm, sp, gram_zigzag(k, me, G));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  auto unit = [&](int k) -> GramUnit { return k < kGramMaxUnits ? units[k] : gram_unit(prm, sp, gram_zigzag(k, me, G)); };

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, last_parity = 0;
      bool ok = true;
      const uint32_t s_bytes = static_cast<uint32_t>(kBM * r_pad * 2);
      const uint32_t bytes = static_cast<uint32_t>(kGramDBytes) + prm.planes * s_bytes;
      for (int k = 0; k < n_mine && ok; ++k) {
        const GramUnit g = unit(k);
        const CUtensorMap* md = g.job ? &map_d1 : &map_d0;
        const CUtensorMap* ms = g.job ? &map_s1 : &map_s0;
        for (int i = g.b; i < g.e && ok; ++i) {
          const int st = tb.slot_list(i);
          const int row0 = tb.st_tile(st) * kBM;
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, tb.err, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], bytes);
          uint8_t* sD = ring + stage * prm.stage_bytes;
          tma_load_2d(sD, md, &full[stage], g.cb * 128, row0);
          tma_load_2d(sD + kGramDBytes / 2, md, &full[stage], g.cb * 128 + 64, row0);
          for (int pl = 0; pl < prm.planes; ++pl)
            tma_load_2d(sD + kGramDBytes + pl * s_bytes, ms, &full[stage], 0, pl * prm.s_plane_rows + st * kBM);
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == n_stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok)
        for (int s = 0; s < n_stages; ++s)
          if (issued_mask & (1u << s)) drain_wait(&full[s], (last_parity >> s) & 1u, tb.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued_any = false;
      const uint32_t ring_base = smem_u32(ring);
      const uint32_t s_bytes = static_cast<uint32_t>(kBM * r_pad * 2);
      for (int k = 0; k < n_mine && ok; ++k) {
        const GramUnit g = unit(k);
        // unit k goes through accumulator buffer k % n_bufs to epilogue set k % 2
        const int buf = k % prm.n_bufs;
        if (!mbar_wait(&tempty[buf], ((k / prm.n_bufs) & 1) ^ 1, abort_flag, tb.err, kErrTimeoutAcc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (g.b == g.e) {  // adapter with only empty routes: nothing to add, the epilogue writes zeros
          mbar_arrive(&tfull[buf]);
          continue;
        }
        const uint32_t dt = tmem_base + static_cast<uint32_t>(buf * prm.acc_cols);
        const uint32_t chain_cols = static_cast<uint32_t>(prm.acc_cols / prm.chains);
        uint32_t started = 0;  // chains that hold a partial sum already
        for (int i = g.b; i < g.e; ++i) {
          if (!mbar_wait(&full[stage], phase, abort_flag, tb.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = ring_base + stage * prm.stage_bytes;
          const uint32_t b0 = a0 + kGramDBytes;
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk) {
            const int ch = kk % prm.chains;
            const uint64_t adesc = umma_sdesc(a0 + kk * 2048, kGramDBytes / 2, 1024, 2);
            const uint64_t bdesc = umma_sdesc(b0 + kk * prm.s_kstep, s_bytes, prm.s_sbo, prm.s_layout);
            umma_f16(dt + ch * chain_cols, adesc, bdesc, prm.idesc, (started >> ch) & 1u);
            started |= 1u << ch;
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == n_stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[buf]);
      }
      if (!ok && issued_any) {
        umma_commit(drain);
        drain_wait(drain, 0, tb.err);
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3;  // the TMEM lane quadrant this warp may access
    const int col = q * 32 + lane;
    const int set = (warp - 2) >> 2;
    // Elements (j0 .. j0+15, column cb * 128 + col) of a slot's block, [rank, C] (transposed) or
    // [C, rank], in the input type or (out_f32) in float, written with 16-byte stores where the layout
    // allows (C is a multiple of 8 on this path): a [C, rank] row segment from registers; a [rank, C]
    // block in the input type through this warp's staging tile (16 ranks x 32 columns) as 16-byte
    // row pieces; [rank, C] in float as one 128-byte row piece per warp and rank.  The whole warp
    // calls it (same block, converged).
    auto store16 = [&](int job, int rank_prefix, int rank, int cb, int j0, const float* v) {
      const GramJob& jb = prm.job[job];
      const int c = cb * 128 + col;
      const int64_t obase = static_cast<int64_t>(rank_prefix) * jb.C;
      if (jb.transpose_out && !jb.out_f32) {
        OutT* stg = stage_tr + (warp - 2) * 16 * 32;
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) stg[jj * 32 + lane] = cvt_out<OutT>(v[jj]);
        __syncwarp();
        OutT* o = reinterpret_cast<OutT*>(jb.out) + obase;
        const int cw = cb * 128 + q * 32;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int idx = lane + 32 * t, rr = idx >> 2, ch = idx & 3;
          const int j = j0 + rr, c8 = cw + ch * 8;
          if (j < rank && c8 < jb.C)
            *reinterpret_cast<uint4*>(o + static_cast<int64_t>(j) * jb.C + c8) =
                *reinterpret_cast<const uint4*>(stg + rr * 32 + ch * 8);
        }
        __syncwarp();
        return;
      }
      if (c >= jb.C) return;
      if (jb.transpose_out) {
        float* o = reinterpret_cast<float*>(jb.out) + obase;
#pragma unroll
        for (int jj = 0; jj < 16; ++jj)
          if (j0 + jj < rank) o[static_cast<int64_t>(j0 + jj) * jb.C + c] = v[jj];
        return;
      }
      const int64_t row = obase + static_cast<int64_t>(c) * rank;
      if (jb.out_f32) {
        float* o = reinterpret_cast<float*>(jb.out) + row;
#pragma unroll
        for (int q4 = 0; q4 < 16; q4 += 4) {
          const int j = j0 + q4;
          if (rank % 4 == 0 && j + 4 <= rank)
            *reinterpret_cast<float4*>(o + j) = make_float4(v[q4], v[q4 + 1], v[q4 + 2], v[q4 + 3]);
          else
            for (int e = 0; e < 4; ++e)
              if (j + e < rank) o[j + e] = v[q4 + e];
        }
        return;
      }
      OutT* o = reinterpret_cast<OutT*>(jb.out) + row;
#pragma unroll
      for (int q8 = 0; q8 < 16; q8 += 8) {
        const int j = j0 + q8;
        if (rank % 8 == 0 && j + 8 <= rank) {
          uint4 pk;
          pk.x = pack2<OutT>(v[q8], v[q8 + 1]);
          pk.y = pack2<OutT>(v[q8 + 2], v[q8 + 3]);
          pk.z = pack2<OutT>(v[q8 + 4], v[q8 + 5]);
          pk.w = pack2<OutT>(v[q8 + 6], v[q8 + 7]);
          *reinterpret_cast<uint4*>(o + j) = pk;
        } else {
          for (int e = 0; e < 8; ++e)
            if (j + e < rank) o[j + e] = cvt_out<OutT>(v[q8 + e]);
        }
      }
    };
    for (int k = set; k < n_mine; k += kGramEpiSets) {
      const GramUnit g = unit(k);
      const GramJob& jb = prm.job[g.job];
      const int buf = k % prm.n_bufs;
      const int rank = g.rank;
      if (!warp_wait(&tfull[buf], (k / prm.n_bufs) & 1, abort_flag, tb.err, kErrTimeoutAcc)) break;
      tc_fence_after();
      if (g.b == g.e) {
        float zeros[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) zeros[jj] = 0.f;
        for (int j0 = 0; j0 < rank; j0 += 16) store16(g.job, g.rank_prefix, rank, g.cb, j0, zeros);
        tc_fence_before();
        mbar_arrive(&tempty[buf]);
        continue;
      }
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * prm.acc_cols);
      const int chain_cols = prm.acc_cols / prm.chains;
      // 16 columns j0.. of this thread's row: chains and planes added in fixed order (chain-major);
      // two tensor-memory loads are in flight per wait
      auto load_sum16 = [&](int j0, float* out16) {
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) out16[jj] = 0.f;
        const int n = prm.chains * prm.planes;
        for (int i0 = 0; i0 < n; i0 += 2) {
          uint32_t v[2][16];
#pragma unroll
          for (int u = 0; u < 2; ++u)
            if (i0 + u < n) {
              const int ch = (i0 + u) / prm.planes, pl = (i0 + u) - ch * prm.planes;
              tmem_ld16(tbase + ch * chain_cols + pl * r_pad + j0, v[u]);
            }
          tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < 2; ++u)
            if (i0 + u < n) {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) out16[jj] += __uint_as_float(v[u][jj]);
            }
        }
      };
      // A spanning slot's block (this warp's 32 columns, summed over this rank's rows) goes to every
      // rank's exchange buffer; the sums over the ranks are formed after the units.  A split
      // slot's last part pushes the parts' sum.
      const int sv = prm.peer.world > 0 ? prm.peer.slot_span[g.slot] : -1;
      if (sv >= 0 && g.parts == 1) {
        const GramPeer& pr = prm.peer;
        const int blk = sv * pr.blocks_per_span + (jb.transpose_out ? pr.cblk_b : 0) + g.cb;
        const size_t half = peer_half_bytes(pr.world, pr.n_blocks, pr.xr) * static_cast<size_t>(pr.gen & 1);
        for (int j0 = 0; j0 < pr.xr; j0 += 16) {
          float v[16];
          if (j0 < r_pad) {
            load_sum16(j0, v);
          } else {
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) v[jj] = 0.f;
          }
          span_put16(pr, half, blk, col, j0, v);
        }
        tc_fence_before();
        mbar_arrive(&tempty[buf]);
        continue;
      }
      if (g.parts > 1) {
        // part of a split slot: fp32 partial of this warp's 32 columns; the last of the slot's
        // parts to arrive (per column block and warp) adds the parts in part order
        float* mine = prm.partial + (static_cast<int64_t>(g.pid) * 128 + col) * r_pad;
        for (int j0 = 0; j0 < r_pad; j0 += 16) {
          float v[16];
          load_sum16(j0, v);
#pragma unroll
          for (int jj = 0; jj < 16; jj += 4)
            *reinterpret_cast<float4*>(mine + j0 + jj) = make_float4(v[jj], v[jj + 1], v[jj + 2], v[jj + 3]);
        }
        tc_fence_before();
        mbar_arrive(&tempty[buf]);
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0)
          last = gen_arrive(prm.counters + static_cast<int64_t>(g.cid) * 4 + q, prm.gen32, tb.err) ==
                         static_cast<uint32_t>(g.parts)
                     ? 1
                     : 0;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence();
        if (sv >= 0) {  // spanning slot: the parts' sum goes to the exchange (zeros past r_pad)
          const GramPeer& pr = prm.peer;
          const int blk = sv * pr.blocks_per_span + (jb.transpose_out ? pr.cblk_b : 0) + g.cb;
          const size_t half = peer_half_bytes(pr.world, pr.n_blocks, pr.xr) * static_cast<size_t>(pr.gen & 1);
          for (int j0 = 0; j0 < pr.xr; j0 += 16) {
            float acc[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) acc[jj] = 0.f;
            if (j0 < r_pad)
              for (int pp = 0; pp < g.parts; ++pp) {
                const float4* src = reinterpret_cast<const float4*>(
                    prm.partial + (static_cast<int64_t>(g.pbase + pp * jb.n_cblk) * 128 + col) * r_pad + j0);
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                  const float4 f = __ldcg(src + t);
                  acc[4 * t] += f.x;
                  acc[4 * t + 1] += f.y;
                  acc[4 * t + 2] += f.z;
                  acc[4 * t + 3] += f.w;
                }
              }
            span_put16(pr, half, blk, col, j0, acc);
          }
          continue;
        }
        for (int j0 = 0; j0 < r_pad; j0 += 16) {  // 16 sums per step, parts added in order
          float acc[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) acc[jj] = 0.f;
          for (int pp = 0; pp < g.parts; ++pp) {
            const float4* src = reinterpret_cast<const float4*>(
                prm.partial + (static_cast<int64_t>(g.pbase + pp * jb.n_cblk) * 128 + col) * r_pad + j0);
            float4 v4[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) v4[t] = __ldcg(src + t);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              acc[4 * t] += v4[t].x;
              acc[4 * t + 1] += v4[t].y;
              acc[4 * t + 2] += v4[t].z;
              acc[4 * t + 3] += v4[t].w;
            }
          }
          if (j0 < rank) store16(g.job, g.rank_prefix, rank, g.cb, j0, acc);
        }
        continue;
      }
      // 16 rank columns at a time: their tensor-memory loads, then their 16-byte stores (measured
      // faster than reading the whole row before the first store)
      for (int j0 = 0; j0 < r_pad; j0 += 16) {
        float v[16];
        load_sum16(j0, v);
        if (j0 < rank) store16(g.job, g.rank_prefix, rank, g.cb, j0, v);
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
    if (prm.peer.world > 0 && !*abort_flag) {
      // Sums of the spanning blocks of this launch's jobs (held here or not): block t goes to set
      // t % 2 of CTA t / 2 (mod the grid); each lane adds its column's entries from the holders
      // in rank order, as they arrive, and the warp writes the sums like a local block.
      const GramPeer& pr = prm.peer;
      const size_t half = peer_half_bytes(pr.world, pr.n_blocks, pr.xr) * static_cast<size_t>(pr.gen & 1);
      const uint8_t* base = pr.xbuf[pr.rank] + half;
      const int n_sum0 = pr.n_span * prm.job[0].n_cblk;
      const int n_sum = n_sum0 + (prm.n_jobs > 1 ? pr.n_span * prm.job[1].n_cblk : 0);
      bool ok = true;
      for (int t = me * kGramEpiSets + set; t < n_sum && ok; t += G * kGramEpiSets) {
        const int j = t < n_sum0 ? 0 : 1;
        const GramJob& jb = prm.job[j];
        const int tt = t - (j ? n_sum0 : 0);
        const int sv = tt / jb.n_cblk, cb = tt - sv * jb.n_cblk;
        const int blk = sv * pr.blocks_per_span + (jb.transpose_out ? pr.cblk_b : 0) + cb;
        const int out_prefix = pr.span_info[3 * sv], rank = pr.span_info[3 * sv + 1];
        const uint32_t holders = static_cast<uint32_t>(pr.span_info[3 * sv + 2]);
        for (int j0 = 0; j0 < pr.xr && j0 < rank; j0 += 16) {
          float acc[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) acc[jj] = 0.f;
          for (int src = 0; src < pr.world && ok; ++src)
            if ((holders >> src) & 1u) ok = span_add16(pr, base, src, blk, col, j0, acc, abort_flag, tb.err);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          store16(j, out_prefix, rank, cb, j0, acc);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, static_cast<uint32_t>(prm.tmem_cols));
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

int pair_spare_pairs(int T, int Nout, int num_sms, int n_units) {
  const int n_mtiles = (T + kBM - 1) / kBM;
  const int total = ((n_mtiles + 1) / 2) * ((Nout + 255) / 256);
  const int pairs = num_sms / 2;
  if (total == 0 || n_units == 0) return 0;
  const int rounds = (total + pairs - 1) / pairs;
  const int gemm_pairs = (total + rounds - 1) / rounds;
  const int spare = pairs - gemm_pairs;
  return spare >= 4 ? spare : 0;  // below 8 SMs the shrink would hold up the first round
}

cudaError_t tc_gemm_pair(int dtype, bool q_mn_major, const TcMaps& maps, int T, int Nout, int Kred, bool lora,
                         const Tables& tb, void* out, int64_t ldo, int num_sms, cudaStream_t st,
                         const PairShrink* shrink, const PairTail* tail) {
  PairParams p{};
  p.out = out;
  p.ldo = ldo;
  p.T = T;
  p.Nout = Nout;
  p.Kred = Kred;
  const int n_mtiles = (T + kBM - 1) / kBM;
  p.n_mpairs = (n_mtiles + 1) / 2;
  p.n_ntiles = (Nout + 255) / 256;
  // Raster groups of row pairs (tiles of a group go column block by column block, the row pairs
  // fastest).  With a co-scheduled shrink the first round touches few row tiles, whose shrink
  // units are ready first; otherwise 16 row pairs, whose P rows stay in L2 while the group sweeps
  // Q, so large problems re-read Q from HBM once per 16 row pairs (measured at 32768 x 8192 ->
  // 28672 under the power cap: 13.3 ms against 14.2 ms with groups of 4).
  p.group_m = 16;
  p.lora = lora ? 1 : 0;
  p.r_pad = tb.r_pad;
  const int fmt = dtype == LF_BF16 ? 1 : 0;
  p.ab_fmt = fmt;
  p.s_planes = 1;
  p.s_plane_rows = (tb.n_segtiles + 1) * kBM;
  p.idesc_main = umma_idesc_f16(256, 256, fmt, 0, q_mn_major ? 1 : 0);
  p.idesc_lora = umma_idesc_f16(256, 256, fmt, 0, 0);
  p.lora_layout = umma_layout_for_span(tb.r_pad * 2);
  p.lora_sbo = sw_sbo(tb.r_pad);
  p.lora_per_stage = tb.r_pad > 0 ? kPairABytes / (kBM * tb.r_pad * 2) : 1;  // 4, 2, 1 for r_pad 16, 32, 64
  static_assert(kPairABytes / kBM == kPairBBytes / 128, "S and B items split a stage alike");
  p.tb = tb;
  p.tail_parts = 1;
  const int total = p.n_mpairs * p.n_ntiles;
  if (total == 0) return cudaSuccess;
  const int all_pairs = num_sms / 2;
  const int nkb = (Kred + kBK - 1) / kBK;
  int gemm_pairs = total < all_pairs ? total : all_pairs;
  const CUtensorMap* a_map = &maps.p;  // unused unless a shrink is co-scheduled
  const CUtensorMap* p2_map = &maps.p;
  const CUtensorMap* a2_map = &maps.p;
  if (shrink != nullptr && (shrink->n_pairs > 0 || shrink->prologue)) {
    p.group_m = 4;
    p.shrink_prologue = shrink->prologue ? 1 : 0;
    p.n_shrink_pairs = shrink->prologue ? 0 : shrink->n_pairs;
    p.s_planes = 2;
    p.s_ext = shrink->s_ext;
    p.unit_ready = shrink->unit_ready;
    p.gen = shrink->gen;
    p.ready_gen = shrink->wait_gen;
    a_map = &shrink->a_map;
    if (shrink->job2) {
      p.job2 = 1;
      p.Kred2 = shrink->K2;
      p.s_ext2 = shrink->s_ext2;
      p2_map = &shrink->p2_map;
      a2_map = &shrink->a2_map;
    }
    if (!shrink->prologue) {  // the GEMM keeps its round count on the pairs the shrink leaves
      const int rounds = (total + all_pairs - 1) / all_pairs;
      gemm_pairs = (total + rounds - 1) / rounds;
    }
  }
  if (tail != nullptr && tail->slots > 0) {
    // Cut the tail tiles along K when the last round is at most half full (or there are fewer
    // tiles than pairs), into as many parts (<= 4, each >= 2 k-blocks) as the idle pairs and the
    // partial slots allow.
    const bool few = total < gemm_pairs || (p.n_shrink_pairs == 0 && total < all_pairs);
    const int avail = few && p.n_shrink_pairs == 0 ? all_pairs : gemm_pairs;
    const int rem = few ? total : total - (total / gemm_pairs) * gemm_pairs;
    int parts = rem > 0 && 2 * rem <= avail ? avail / rem : 1;
    if (parts > 4) parts = 4;
    while (parts > 1 && (rem * (parts - 1) > tail->slots || nkb < 2 * parts)) --parts;
    if (parts > 1) {
      if (few) gemm_pairs = total * parts;  // every tile is a tail tile, one part per pair
      p.tail_parts = parts;
      p.tail_partial = tail->partial;
      p.tail_flag = tail->flags;
      if (p.n_shrink_pairs == 0 && !p.shrink_prologue) p.gen = tail->gen;  // else the shrink's serves both
    }
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * (gemm_pairs + p.n_shrink_pairs));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kPairSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // GEMM pairs wait on the shrink CTAs' flags, last tail parts on the earlier parts' flags: all
  // CTAs must be resident at once
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.n_shrink_pairs > 0 || p.shrink_prologue || p.tail_parts > 1 ? 2 : 1;
  cudaError_t e;
#define LF_LAUNCH_PAIR(QMN, OT)                                                                  \
  e = ensure_smem(tc_gemm_pair_kernel<QMN, OT>, kPairSmem);                                     \
  if (e != cudaSuccess) return e;                                                               \
  e = cudaLaunchKernelEx(&cfg, tc_gemm_pair_kernel<QMN, OT>, maps.p, maps.q, maps.s, maps.l, maps.o, *a_map, *p2_map, \
                         *a2_map, p);
  if (dtype == LF_BF16) {
    if (q_mn_major) {
      LF_LAUNCH_PAIR(true, __nv_bfloat16)
    } else {
      LF_LAUNCH_PAIR(false, __nv_bfloat16)
    }
  } else {
    if (q_mn_major) {
      LF_LAUNCH_PAIR(true, __half)
    } else {
      LF_LAUNCH_PAIR(false, __half)
    }
  }
#undef LF_LAUNCH_PAIR
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t tc_shrink(int dtype, const CUtensorMap& p_map, const CUtensorMap& a_map, int Kred, const Tables& tb,
                      void* s_ext, int num_sms, cudaStream_t st) {
  if (tb.n_units == 0) return cudaSuccess;
  const int nkb = (Kred + kBK - 1) / kBK;
  // split K across a cluster while every CTA still fits on the GPU at once (one per SM)
  // and each keeps at least four k-blocks
  int cluster = 1;
  while (cluster < kMaxShrCluster && tb.n_units * cluster * 2 <= num_sms && nkb >= 4 * cluster * 2) cluster *= 2;
  ShrinkParams p{};
  p.s_ext = s_ext;
  p.plane_elems = static_cast<int64_t>(tb.n_segtiles + 1) * kBM * tb.r_pad;
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

cudaError_t tc_gram(int dtype, const GramJobDesc* jobs, int n_jobs, const Tables& tb, int num_sms, cudaStream_t st,
                    int planes, void* scratch, uint64_t gen, const GramPeer* peer) {
  if (n_jobs < 1 || n_jobs > 2) return cudaErrorInvalidValue;
  GramParams p{};
  if (peer != nullptr) p.peer = *peer;
  p.n_jobs = n_jobs;
  int64_t steps = 0, most = 0;
  for (int j = 0; j < n_jobs; ++j) {
    p.job[j].out = jobs[j].out;
    p.job[j].C = jobs[j].C;
    p.job[j].n_cblk = (jobs[j].C + 127) / 128;
    p.job[j].transpose_out = jobs[j].transpose_out;
    p.job[j].out_f32 = jobs[j].out_f32;
    steps += static_cast<int64_t>(tb.n_segtiles) * p.job[j].n_cblk;
    most += static_cast<int64_t>(tb.n_segtiles + tb.n_slots) * p.job[j].n_cblk;  // units once split
  }
  p.planes = planes;
  p.s_plane_rows = (tb.n_segtiles + 1) * kBM;
  p.r_pad = tb.r_pad;
  p.stage_bytes = kGramDBytes + planes * kBM * tb.r_pad * 2;
  p.n_stages = kGramRingBytes / p.stage_bytes;
  if (p.n_stages > kGramMaxStages) p.n_stages = kGramMaxStages;
  const int fmt = dtype == LF_BF16 ? 1 : 0;
  const int width = planes * tb.r_pad;  // MMA N
  // Accumulator buffers, each with its accumulation chains (rotating over K steps, added in fixed
  // order: see kRoleChains).  The epilogue (tensor-memory reads and stores of a unit) takes longer
  // than a short unit's MMAs, so where four buffers fit the MMA runs up to four units ahead of the
  // epilogue sets, with one chain (each chain is more columns for the epilogue to read: one chain
  // measured faster than two or four, and than eight buffers); otherwise two buffers with as many
  // chains as fit, up to four.
  if (4 * width <= 512) {
    p.n_bufs = 4;
    p.chains = 1;
  } else {
    p.n_bufs = 2;
    p.chains = 4;
    while (p.chains > 1 && 2 * p.chains * width > 512) p.chains >>= 1;
  }
  p.acc_cols = p.chains * width;
  p.tmem_cols = 512;  // one CTA per SM: the whole TMEM
  p.idesc = umma_idesc_f16(kBM, width, fmt, 1, 1);
  p.s_layout = umma_layout_for_span(tb.r_pad * 2);
  p.s_sbo = sw_sbo(tb.r_pad);
  p.s_kstep = static_cast<uint32_t>(16 * tb.r_pad * 2);
  p.tb = tb;
  if (tb.n_slots == 0 || most == 0) return cudaSuccess;
  const int grid = static_cast<int>(most < num_sms ? most : num_sms);
  if (scratch != nullptr && tb.n_slots <= kGramMaxSlots) {
    // Parts of at most ~an eighth of a CTA's even share of segment-tile steps: dealt zig-zag,
    // largest first, parts that small leave the busiest CTA within ~10% of the mean (a quarter
    // share: ~25%; a half share: ~40% at 16 Zipf-sized adapters).
    const int64_t share = (steps + 8 * grid - 1) / (8 * grid);
    p.cap = static_cast<int>(share < 2 ? 2 : share);
    p.partial = static_cast<float*>(scratch);
    p.counters = reinterpret_cast<uint64_t*>(static_cast<char*>(scratch) +
                                             static_cast<size_t>(kGramMaxPartials) * 128 * tb.r_pad * 4);
    p.gen32 = static_cast<uint32_t>(gen);
  }
  const CUtensorMap& d1 = jobs[n_jobs - 1].d_map;
  const CUtensorMap& s1 = jobs[n_jobs - 1].s_map;
  cudaError_t e;
  if (dtype == LF_BF16) {
    e = ensure_smem(tc_gram_kernel<__nv_bfloat16>, kGramSmem);
    if (e != cudaSuccess) return e;
    tc_gram_kernel<__nv_bfloat16><<<grid, kGramThreads, kGramSmem, st>>>(jobs[0].d_map, jobs[0].s_map, d1, s1, p);
  } else {
    e = ensure_smem(tc_gram_kernel<__half>, kGramSmem);
    if (e != cudaSuccess) return e;
    tc_gram_kernel<__half><<<grid, kGramThreads, kGramSmem, st>>>(jobs[0].d_map, jobs[0].s_map, d1, s1, p);
  }
  return cudaGetLastError();
}

}  // namespace lf
