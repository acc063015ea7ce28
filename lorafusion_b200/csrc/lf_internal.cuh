// Internal declarations shared by the kernel translation units and the C ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lorafusion_b200.h"

namespace lf {

// Device view of the routing table (see lf_plan_info for the sections).
struct Tables {
  const int32_t* base;
  int32_t off_tile_st, off_st_tile, off_st_lo, off_st_hi, off_st_slot, off_st_scale;
  int32_t off_slot_st, off_slot_list, off_slot_rank, off_rank_prefix, off_slot_order;
  int32_t off_unit_tile, off_unit_st0, off_unit_nst;
  int32_t off_pair_lora, off_pl_a, off_pl_b, off_pl_slot, off_tile_unit;
  int32_t n_tiles, n_segtiles, n_slots, n_units, r_pad;
  int* err;  // device status word for bounded-wait timeouts

  __device__ __forceinline__ int32_t tile_st(int t) const { return base[off_tile_st + t]; }
  __device__ __forceinline__ int32_t st_tile(int j) const { return base[off_st_tile + j]; }
  __device__ __forceinline__ int32_t st_lo(int j) const { return base[off_st_lo + j]; }
  __device__ __forceinline__ int32_t st_hi(int j) const { return base[off_st_hi + j]; }
  __device__ __forceinline__ int32_t st_slot(int j) const { return base[off_st_slot + j]; }
  __device__ __forceinline__ float st_scale(int j) const { return __int_as_float(base[off_st_scale + j]); }
  __device__ __forceinline__ int32_t slot_st(int s) const { return base[off_slot_st + s]; }
  __device__ __forceinline__ int32_t slot_list(int i) const { return base[off_slot_list + i]; }
  __device__ __forceinline__ int32_t slot_rank(int s) const { return base[off_slot_rank + s]; }
  __device__ __forceinline__ int32_t rank_prefix(int s) const { return base[off_rank_prefix + s]; }
  __device__ __forceinline__ int32_t slot_order(int i) const { return base[off_slot_order + i]; }
  __device__ __forceinline__ int32_t unit_tile(int u) const { return base[off_unit_tile + u]; }
  __device__ __forceinline__ int32_t unit_st0(int u) const { return base[off_unit_st0 + u]; }
  __device__ __forceinline__ int32_t unit_nst(int u) const { return base[off_unit_nst + u]; }
  __device__ __forceinline__ int32_t pair_lora(int p) const { return base[off_pair_lora + p]; }
  __device__ __forceinline__ int32_t pl_a(int i) const { return base[off_pl_a + i]; }
  __device__ __forceinline__ int32_t pl_b(int i) const { return base[off_pl_b + i]; }
  __device__ __forceinline__ int32_t pl_slot(int i) const { return base[off_pl_slot + i]; }
  __device__ __forceinline__ int32_t tile_unit(int t) const { return base[off_tile_unit + t]; }
};

Tables make_tables(const lf_plan_info* info, const int32_t* table_dev);

// --------------------------------------------------------------- SIMT (any dtype, f64 sums)
// S_ext[st][row][j] = (row in segment) ? scale * sum_k P[tile*128+row][k] * Apk[slot][j][k] : 0
cudaError_t simt_shrink(int dtype, const void* P, int64_t ldp, int Kred, const void* apk, const Tables& tb,
                        double* s_ext, cudaStream_t st);
// out[t][n] = sum_k P[t][k] Q(n,k) + sum_j S_ext[st(t)][row][j] * L[slot][n][j],  Q(n,k) = Q[n*qsn + k*qsk]
cudaError_t simt_gemm(int dtype, const void* P, int64_t ldp, const void* Q, int64_t qsn, int64_t qsk, int T, int Nout,
                      int Kred, const double* s_ext, const void* lpk, const Tables& tb, void* out, int64_t ldo,
                      cudaStream_t st);
// grad[slot] = sum_{rows of slot} D[row][c] * S_ext[..][row][j]; layout [C][rank] or [rank][C] (transpose_out),
// in the input type or (out_f32) in float
cudaError_t simt_gram(int dtype, const void* D, int64_t ldd, int C, const double* s_ext, const Tables& tb,
                      void* out, int transpose_out, int out_f32, cudaStream_t st);

// --------------------------------------------------------------- tcgen05 (bf16 / f16)
struct TcMaps {
  CUtensorMap p;   // [T, Kred] box (64, 128)
  CUtensorMap q;   // K-major: [Nout, Kred] box (64, 256);  MN-major: [Kred, Nout] box (64, 64)
  CUtensorMap s;   // S_ext [n_st*128, r_pad] box (r_pad, 128)
  CUtensorMap l;   // L [n_slots*Nout, r_pad] box (r_pad, 256)
  CUtensorMap o;   // output [T, Nout] box (64, 32), 128-byte swizzle (pair GEMM epilogue stores)
};

cudaError_t tc_shrink(int dtype, const CUtensorMap& p_map, const CUtensorMap& a_map, int Kred, const Tables& tb,
                      void* s_ext, int num_sms, cudaStream_t st);
cudaError_t tc_gemm(int dtype, bool q_mn_major, const TcMaps& maps, int T, int Nout, int Kred, bool lora,
                    const Tables& tb, void* out, int64_t ldo, int num_sms, cudaStream_t st);
// Same product with 256x256 tiles computed by CTA pairs (cta_group::2).  Maps: p box (64,128),
// q K-major box (64,128) / MN-major box (64,64), s box (r_pad,128), l box (r_pad,128).
// Optional routed shrink run by spare CTA pairs of the same launch (S_ext = s.P.A_slot^T).
// The GEMM's own LoRA operand comes from the first job (P = the GEMM's P); an optional second
// job (its own P, slab and K) is computed afterwards for a later launch (the backward's x.A^T).
struct PairShrink {
  CUtensorMap a_map;     // packed slab [n_slots*r_pad, Kred] box (64, r_pad), job 1
  void* s_ext;           // two K-half planes written by the launch, job 1
  uint64_t* unit_ready;  // [2*n_units] ready flags of job 1 (then [2*n_units] of job 2)
  uint64_t gen;          // value the flags take in this launch
  uint64_t wait_gen;     // value the GEMM CTAs wait for (gen; a test hook makes it one nobody writes)
  int n_pairs;           // CTA pairs given to the shrink (dedicated mode)
  bool prologue;         // instead: every CTA runs its share of the shrink before its GEMM tiles
  bool job2;             // second job present
  CUtensorMap p2_map;    // job 2 activations [T, K2] box (64, 128)
  CUtensorMap a2_map;    // job 2 slab [n_slots*r_pad, K2] box (64, r_pad)
  void* s_ext2;
  int K2;
};
// K-split tail of the pair GEMM (the last round of 256x256 tiles cut along K when it would
// leave at least half of the CTA pairs idle): fp32 partial tiles and their release flags, in
// caller scratch after the fixed workspace sections.  `slots` partial tiles fit there; `gen`
// must differ from every earlier launch's on the same flags.
constexpr int kTailSlots = 80;                              // >= the CTA pairs of a B200 (74)
constexpr size_t kTailPartialBytes = size_t(256) * 256 * 4;  // one fp32 256x256 tile
constexpr size_t kTailFlagBytes = (size_t(kTailSlots) * 8 * 8 + 255) & ~size_t(255);
inline size_t tail_scratch_bytes() { return kTailFlagBytes + kTailSlots * kTailPartialBytes; }
struct PairTail {
  uint64_t* flags;  // [slot][2 CTAs][4 epilogue warps]
  float* partial;   // [slot][256 x 256]
  int slots;
  uint64_t gen;
};
// CTA pairs the pair GEMM can leave to a co-scheduled shrink without adding a round (0: none).
int pair_spare_pairs(int T, int Nout, int num_sms, int n_units);
// `tail` (optional) enables the K-split tail; the launch is then cooperative.
cudaError_t tc_gemm_pair(int dtype, bool q_mn_major, const TcMaps& maps, int T, int Nout, int Kred, bool lora,
                         const Tables& tb, void* out, int64_t ldo, int num_sms, cudaStream_t st,
                         const PairShrink* shrink = nullptr, const PairTail* tail = nullptr);
// Forward workspace without the tail scratch (the least lf_forward accepts).
size_t forward_min_workspace_bytes(const lf_plan_info* info);
// Gram load balance: slots (slot_order positions) the kernel can split into parts, and the
// capacity of the fp32 partial blocks ([128][r_pad] each) and arrival counters (x4) it may use.
constexpr int kGramMaxSlots = 512;
constexpr int kGramMaxPartials = 640;
constexpr int kGramMaxCounters = 1280;
inline size_t gram_scratch_bytes(int r_pad) {
  return (static_cast<size_t>(kGramMaxPartials) * 128 * r_pad * 4 + static_cast<size_t>(kGramMaxCounters) * 4 * 8 +
          255) & ~size_t(255);
}
// planes: S_ext planes to sum (1, or 2 when the K-half partial products of the co-scheduled
// shrink are read); s_map must then cover both planes.
// Gram jobs (dB: D = g, C = N, S = s.x.A^T, grad [N, r] blocks; dA: D = x, C = K, S = s.g.B,
// transposed [r, K] blocks), up to two in one launch.  `scratch` (gram_scratch_bytes(r_pad), any
// contents) holds the partial sums of split slots; nullptr disables splitting.  `gen` must differ
// from every earlier launch's on that scratch.  planes: S_ext planes to sum (1, or 2 when the
// K-half partial products of the co-scheduled shrink are read); s maps must then cover both.
struct GramJobDesc {
  CUtensorMap d_map;  // D [T, C] box (64, 128)
  CUtensorMap s_map;  // S_ext planes [planes * (n_st+1) * 128, r_pad] box (r_pad, 128)
  int C;
  void* out;
  int transpose_out;
  int out_f32;  // write the gradient blocks as float instead of the input type
};
// In-kernel exchange of the dA/dB blocks of adapters whose rows span the GPUs of one node.  The
// gram pushes each block it computes for a spanning virtual slot (128 columns x r_pad, fp32) into
// every rank's exchange buffer over peer mappings and releases a flag per (block, epilogue warp)
// there; afterwards every CTA sums, in rank order, blocks that all their holders have released,
// and writes them like ordinary gradient blocks.  Exchange buffer of each rank, per half (calls
// alternate by `gen` parity): flags [world][n_blocks][4] u64, then data
// [world][n_blocks][128][xr] float.
constexpr int kMaxPeers = 8;
struct GramPeer {
  int world = 0, rank = 0;   // world 0: no exchange
  uint8_t* xbuf[kMaxPeers];  // every rank's exchange buffer as mapped in this process
  const int32_t* slot_span;  // [n_slots] spanning virtual slot of each local slot, -1 else (device)
  const int32_t* span_info;  // [n_span][3] output rank prefix, rank, holder mask (device)
  int n_span, n_blocks;      // n_blocks = n_span * blocks_per_span
  int blocks_per_span;       // column blocks of dB (ceil(N/128)) then of dA (ceil(K/128))
  int cblk_b;                // ceil(N/128): where a slot's dA blocks start
  int xr;                    // rank columns of an exchanged block (the same on every rank)
  uint64_t gen;
};
// One half of an exchange buffer: per (source rank, block, rank-column pair, column) one 16-byte
// entry of two 64-bit words {generation << 32 | float bits}.
__host__ __device__ inline size_t peer_half_bytes(int world, int n_blocks, int r_pad) {
  return (static_cast<size_t>(world) * n_blocks * 128 * r_pad * 8 + 255) & ~size_t(255);
}
cudaError_t tc_gram(int dtype, const GramJobDesc* jobs, int n_jobs, const Tables& tb, int num_sms, cudaStream_t st,
                    int planes = 1, void* scratch = nullptr, uint64_t gen = 0, const GramPeer* peer = nullptr);

// --------------------------------------------------------------- packing
cudaError_t pack_adapters(int src_dtype, int dst_dtype, const uint64_t* src_ptrs, const int32_t* ranks,
                          int n_slots, int rank_dim, int other_dim, int transpose, int d0, int d1, void* dst,
                          cudaStream_t st);

}  // namespace lf
