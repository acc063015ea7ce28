/*
 * lorafusion_b200 — C ABI of the B200 (sm_100a) fused multi-adapter LoRA operator.
 *
 * The operator computes, for a fused batch whose rows are routed to adapters by
 * contiguous row ranges ("routes"):
 *
 *   forward   y        = x W^T + s_i (x A_i^T) B_i^T                 (rows of route -> adapter i)
 *   backward  grad_x   = g W   + s_i (g B_i) A_i
 *             grad_B_i = s_i sum_rows g^T (x A_i^T)
 *             grad_A_i = s_i sum_rows (g B_i)^T x
 *
 * with x [T,K], W [N,K], A_i [r_i,K], B_i [N,r_i], g = grad_out [T,N], s_i = alpha_i / r_i.
 * This is lorafusion's op contract (lorafusion/ops/mock_ops.py:15-95); the Python module
 * lorafusion_b200.b200_ops exposes it with the reference's exact call signature
 * (fused_lora_forward / fused_lora_backward) on top of these entry points.
 *
 * Conventions
 *  - Every pointer argument named *_dev is device memory; everything else is host memory.
 *  - Matrices are dense row-major.  The caller owns every buffer; the library allocates
 *    nothing per call (scratch space is the caller's `workspace`).
 *  - Every entry point returns an lf_status; nothing aborts or traps.
 *  - Work is enqueued on the given stream; calls do not synchronize.
 */
#ifndef LORAFUSION_B200_H
#define LORAFUSION_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LF_API __attribute__((visibility("default")))
#else
#define LF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void* lf_stream_t; /* a cudaStream_t */

typedef enum lf_status {
  LF_OK = 0,
  LF_ERR_INVALID_ARG = 1,   /* null pointer, bad shape/stride, bad enum             -> ValueError   */
  LF_ERR_ROUTING = 2,       /* routes do not tile [0,T) in order, slot out of range -> ValueError   */
  LF_ERR_UNSUPPORTED = 3,   /* dtype/rank/alignment this build does not handle      -> ValueError   */
  LF_ERR_CUDA = 4,          /* a CUDA runtime/driver call failed                    -> RuntimeError */
  LF_ERR_CAPACITY = 5,      /* a caller buffer (table, workspace) is too small      -> ValueError   */
  LF_ERR_DEVICE = 6         /* a kernel reported a bounded-wait timeout             -> RuntimeError */
} lf_status;

typedef enum lf_dtype { LF_F32 = 0, LF_BF16 = 1, LF_F16 = 2 } lf_dtype;

/* Rows per fused-row tile used by every kernel's routing tables. */
#define LF_TILE_ROWS 128

/* Sizes and section offsets (in int32 words) of a routing table built by lf_plan_tables. */
typedef struct lf_plan_info {
  int32_t total_rows;      /* T */
  int32_t n_routes;
  int32_t n_slots;         /* (virtual) slots: the input slots, one of rank r > 64 as ceil(r/64) */
  int32_t n_tiles;         /* ceil(T / LF_TILE_ROWS) */
  int32_t n_segtiles;      /* route x tile intersections ("segment tiles") */
  int32_t r_pad;           /* padded rank shared by every (virtual) slot: 16, 32 or 64 */
  int32_t max_rank;        /* largest input slot rank */
  int32_t rank_total;      /* sum of slot ranks: rows of the concatenated grad_a blocks */
  int32_t n_shrink_units;  /* (tile, run of <= 64/r_pad segment tiles) work units of the shrink */
  int32_t table_words;     /* int32 words of the table in use */
  /* section offsets */
  int32_t off_tile_st;     /* [n_tiles+1]  CSR: segment tiles of each row tile */
  int32_t off_st_tile;     /* [n_segtiles] row tile of each segment tile */
  int32_t off_st_lo;       /* [n_segtiles] first row inside the tile */
  int32_t off_st_hi;       /* [n_segtiles] one past the last row inside the tile */
  int32_t off_st_slot;     /* [n_segtiles] adapter slot */
  int32_t off_st_route;    /* [n_segtiles] index of the route it came from */
  int32_t off_st_scale;    /* [n_segtiles] float bits of the slot's scaling */
  int32_t off_slot_st;     /* [n_slots+1]  CSR: segment tiles of each slot, in route order */
  int32_t off_slot_list;   /* [n_segtiles] */
  int32_t off_slot_rank;   /* [n_slots]    rank of each slot */
  int32_t off_rank_prefix; /* [n_slots+1]  exclusive prefix sum of ranks */
  int32_t off_slot_order;  /* [n_slots]    slots by descending segment-tile count */
  int32_t off_unit_tile;   /* [n_shrink_units] */
  int32_t off_unit_st0;    /* [n_shrink_units] */
  int32_t off_unit_nst;    /* [n_shrink_units] */
  /* Row tiles taken two at a time (rows 256p .. 256p+255) by the CTA-pair GEMM: per pair, one
   * LoRA stage per adapter slot present in either tile, holding each tile's segment tile of
   * that slot or the all-zero segment tile n_segtiles (the workspace's last block). */
  int32_t n_pair_lora;     /* LoRA stages over all pairs */
  int32_t off_pair_lora;   /* [ceil(n_tiles/2)+1] CSR: stages of each pair */
  int32_t off_pl_a;        /* [n_pair_lora] segment tile of the even row tile */
  int32_t off_pl_b;        /* [n_pair_lora] segment tile of the odd row tile */
  int32_t off_pl_slot;     /* [n_pair_lora] adapter slot */
  int32_t off_tile_unit;   /* [n_tiles+1]  CSR: shrink units of each row tile */
} lf_plan_info;

/* Upper bound on the int32 words lf_plan_tables needs when every slot rank is at most 64 (with
 * larger ranks lf_plan_tables reports the words it needs: LF_ERR_CAPACITY, info->table_words). */
LF_API int32_t lf_plan_table_words(int32_t n_routes, int32_t total_rows, int32_t n_slots);

/*
 * Build the device routing table on the host.
 * Replaces the per-route Python loops of lorafusion/ops/triton_ops.py:398-407 and :435-466
 * (and the row-range walk of mock_ops.py:40-46, :71-93): routes are
 * TileRoutingConfig.routes (lorafusion/ops/config.py:29-47) mapped to adapter slots.
 * Checks what TileRoutingConfig.validate checks (config.py:55-69) -> LF_ERR_ROUTING.
 *   route_start/route_end/route_slot : [n_routes]
 *   slot_rank/slot_scale             : [n_slots] rank r_i (any positive rank, as mock_ops allows) and
 *                                      scaling alpha_i/r_i
 *   table                            : host buffer of table_capacity int32 words
 * A slot of rank r > 64 is carried as ceil(r/64) consecutive virtual slots of ranks 64, ..., 64,
 * r - 64 (ceil(r/64) - 1): slot s's virtual slots follow those of slots < s, each over all of s's
 * rows (the LoRA product is the sum over the chunks).  Everything indexed by slot below (the
 * packed slabs of lf_pack_adapters, grad_a / grad_b blocks, info->n_slots) is per virtual slot;
 * a slot's grad_a rows are its virtual slots' rows, consecutive.
 * The caller copies `table` (info->table_words words) to device memory.  A table_capacity below the
 * need returns LF_ERR_CAPACITY with info->table_words set to the need.
 */
LF_API int lf_plan_tables(const int32_t* route_start, const int32_t* route_end, const int32_t* route_slot,
                   int32_t n_routes, int32_t total_rows, const int32_t* slot_rank, const float* slot_scale,
                   int32_t n_slots, int32_t* table, int32_t table_capacity, lf_plan_info* info);

/* Operands of one projection. */
typedef struct lf_problem {
  int32_t dtype;        /* lf_dtype of x, W, grad_out, outputs and packed adapters */
  int32_t T, K, N;      /* rows, in_features, out_features */
  const void* x_dev;    /* [T,K] */
  const void* w_dev;    /* [N,K] */
  const void* a_pack_dev;  /* [n_slots, r_pad, K]  A_i rows, zero padded   (forward shrink)  */
  const void* b_pack_dev;  /* [n_slots, N, r_pad]  B_i, zero padded columns (forward expand) */
  const void* bt_pack_dev; /* [n_slots, r_pad, N]  B_i^T                     (backward shrink) */
  const void* at_pack_dev; /* [n_slots, K, r_pad]  A_i^T                     (backward expand) */
} lf_problem;

/*
 * Workspace bytes the forward / backward use for this table and dtype.  The workspace starts with
 * S_ext, the routed shrink's output per segment tile: on the tensor-core path four bf16/f16 planes
 * of [n_segtiles + 1][128][r_pad] (each value v stored as hi = round(v) and lo = round(v - hi), for
 * one or two K-half partial products: planes [hi..., lo...]), on the float32 / CUDA-core path one
 * f64 buffer of the same shape.  About 20 MiB of it is
 * the scratch of the GEMM's K-split tail (fp32 partial tiles of a last round cut along K);
 * a smaller workspace that still holds the fixed sections is accepted, and the tail then
 * splits only as far as the partial tiles fit (not at all below one tile).
 */
LF_API size_t lf_forward_workspace_bytes(const lf_plan_info* info, int32_t dtype);
LF_API size_t lf_backward_workspace_bytes(const lf_plan_info* info, int32_t dtype);

/*
 * Pack per-adapter matrices into one zero-padded slab (one launch for all slots).
 * Replaces the memoized fp16 transposed copies of lorafusion/ops/triton_ops.py:114-152.
 * For slot s, src_ptrs_dev[s] points at a row-major matrix whose rank dimension is
 * dim `rank_dim` (0: [r_s, other], 1: [other, r_s]).  The slab is [n_slots, d0, d1]:
 *   transpose = 0: dst[s][i][j] = src_s[i][j]
 *   transpose = 1: dst[s][i][j] = src_s[j][i]
 * and zero wherever the source index is outside the matrix.
 */
LF_API int lf_pack_adapters(int32_t src_dtype, int32_t dst_dtype, const uint64_t* src_ptrs_dev,
                     const int32_t* slot_rank_dev, int32_t n_slots, int32_t rank_dim, int32_t other_dim,
                     int32_t transpose, int32_t d0, int32_t d1, void* dst_dev, lf_stream_t stream);

/*
 * Forward: y [T,N] (dtype of the problem).
 * Replaces triton_ops.fused_lora_forward (lorafusion/ops/triton_ops.py:373-409) and
 * mock_ops.fused_lora_forward (lorafusion/ops/mock_ops.py:15-48).
 */
LF_API int lf_forward(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev, void* y_dev,
               void* workspace_dev, size_t workspace_bytes, lf_stream_t stream);

/*
 * The forward in separately launchable stages (same arguments as lf_forward), so a caller
 * can time or overlap them.  `stages` is a bit mask:
 *   LF_STAGE_SHRINK   routed shrink: workspace <- s_i x A_i^T, masked per segment tile
 *   LF_STAGE_EXPAND   fused base GEMM + LoRA expand into y (reads the shrink's workspace)
 *   LF_STAGE_BASE     base GEMM only, y = x W^T (the "LoRA disabled" yardstick)
 *   LF_STAGE_SINGLE_CTA  with EXPAND or BASE: use 128x256 tiles on single CTAs instead of the
 *                     default 256x256 tiles on CTA pairs (bf16/f16 only; for comparisons)
 *   LF_STAGE_SEPARATE with SHRINK|EXPAND: run them as two ordinary launches instead of one
 *                     cooperative launch (for profilers and SM-partitioned GPUs, which refuse
 *                     cooperative launches)
 * lf_forward == lf_forward_stages(..., LF_STAGE_SHRINK | LF_STAGE_EXPAND).
 * Has no counterpart in the reference (its forward is one call per route).
 */
#define LF_STAGE_SHRINK 1
#define LF_STAGE_EXPAND 2
#define LF_STAGE_BASE 4
#define LF_STAGE_SINGLE_CTA 8
#define LF_STAGE_SEPARATE 16
LF_API int lf_forward_stages(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev, void* y_dev,
                             void* workspace_dev, size_t workspace_bytes, int32_t stages, lf_stream_t stream);

/*
 * The part of lf_forward_workspace_bytes that holds S_ext and the co-scheduling flags; the rest
 * (lf_forward_workspace_bytes minus this) is the K-split tail's scratch, needed only while a
 * forward runs.
 */
LF_API size_t lf_forward_fixed_workspace_bytes(const lf_plan_info* info, int32_t dtype);

/*
 * lf_forward with the K-split tail's scratch in a buffer of its own (`tail_dev`, `tail_bytes`:
 * up to lf_forward_workspace_bytes - lf_forward_fixed_workspace_bytes, 16-byte aligned, else the
 * tail is not split; null/0 = take it from the workspace as lf_forward does), so a caller can keep the workspace, which then needs only
 * lf_forward_fixed_workspace_bytes, for a later lf_backward_sf while the tail buffer is reused.
 * Also reports, in *s_f_planes, the K-half planes of S_f = s_i x A_i^T the call left in the
 * workspace: 2 when the shrink ran inside the GEMM launch, 1 when it ran as a launch of its own, 0
 * when the workspace holds no tensor-core S_f (float32 / CUDA-core path, empty problem).  That
 * value, taken from the call that filled the workspace, is what lf_backward_sf needs.  No
 * counterpart in the reference (it recomputes x A_i^T in the backward).
 */
LF_API int lf_forward_sf(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev, void* y_dev,
                         void* workspace_dev, size_t workspace_bytes, void* tail_dev, size_t tail_bytes,
                         int32_t* s_f_planes, lf_stream_t stream);

/*
 * Kernel launches lf_forward makes for this problem on the current device: 1 when the routed
 * shrink runs on CTA pairs the fused GEMM's round count leaves idle (same launch), else 2.
 * Returns a negative lf_status on bad arguments.  No counterpart in the reference.
 */
LF_API int lf_forward_launch_count(const lf_problem* prob, const lf_plan_info* info);

/*
 * Kernel launches lf_backward makes for this problem on the current device: 2 when both routed
 * shrinks run on CTA pairs the grad_x GEMM leaves idle (that GEMM, then one launch for both
 * grams dA and dB), 4 when the shrinks run as launches of their own, 1 with no routed rows
 * (5 on the float32 path).  Negative lf_status on bad arguments.  No counterpart in the reference.
 */
LF_API int lf_backward_launch_count(const lf_problem* prob, const lf_plan_info* info);

/*
 * Process-wide switch for the co-scheduled (cooperative) launches:
 *   1 (default) the routed shrinks run inside the GEMM's launch on CTA pairs the GEMM's round
 *     count leaves idle (when there are at least four), the GEMM on the others; the GEMM's last
 *     round may be K-split over idle CTA pairs;
 *   2  the same, but every CTA first computes its share of the shrink items and then its GEMM
 *     tiles (which wait only for the S tiles they read), so the GEMM has every CTA pair;
 *   0  no cooperative launches: each routed shrink is an ordinary launch of its own and no tail
 *     is K-split.  For profilers and SM-partitioned GPUs, which refuse cooperative launches (a
 *     refused launch also turns co-scheduling off for that device by itself).
 * Other values return LF_ERR_INVALID_ARG.  The default is 1, or 0 when a CUDA tool (Nsight Compute,
 * compute-sanitizer) is injected into the process: its injection variables are set or its
 * injection library is mapped when the library loads.
 * No counterpart in the reference.
 */
LF_API int lf_set_co_scheduling(int32_t enable);

/*
 * The process-wide co-scheduling mode (*mode, as lf_set_co_scheduling takes it) and, for the
 * current device, the cudaError_t a refused cooperative launch returned (*refused_error; 0 while
 * no launch was refused there).  No counterpart in the reference.
 */
LF_API int lf_get_co_scheduling(int32_t* mode, int32_t* refused_error);

/*
 * Backward: grad_x [T,K]; grad_a = concatenated [r_s, K] blocks and grad_b = concatenated
 * [N, r_s] blocks, slot after slot (slot s starts at rank_prefix[s]*K and rank_prefix[s]*N).
 * Replaces triton_ops.fused_lora_backward (triton_ops.py:412-468) and
 * mock_ops.fused_lora_backward (mock_ops.py:51-95).
 */
LF_API int lf_backward(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                const void* grad_out_dev, void* grad_x_dev, void* grad_a_dev, void* grad_b_dev,
                void* workspace_dev, size_t workspace_bytes, lf_stream_t stream);

/*
 * lf_backward with S_f = s_i x A_i^T taken from a forward instead of recomputed: `s_f_dev` is the
 * workspace a lf_forward_sf call on the same x, adapters and tables filled, and `s_f_planes` the
 * value that call reported (1 or 2 K-half planes, each stored as hi and lo).  The caller keeps
 * that workspace unchanged until this call's work is done.  bf16/f16 only: the float32 path
 * recomputes S_f.
 * Saves the backward's x . A^T shrink (reference: mock_ops.py:79-80 recomputes it per route).
 */
LF_API int lf_backward_sf(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                          const void* grad_out_dev, const void* s_f_dev, int32_t s_f_planes, void* grad_x_dev,
                          void* grad_a_dev, void* grad_b_dev, void* workspace_dev, size_t workspace_bytes,
                          lf_stream_t stream);

/*
 * lf_backward / lf_backward_sf with the dtype of grad_a and grad_b chosen: `grad_ab_dtype` is the
 * problem's dtype or LF_F32 (float gradient blocks, summed in float before any rounding: what a
 * multi-GPU caller all-reduces).  `s_f_dev` may be null (S_f recomputed; `s_f_planes` ignored).
 * Replaces triton_ops.fused_lora_backward (lorafusion/ops/triton_ops.py:412-468), whose grads
 * come back in the input dtype (:453-455); LF_F32 has no counterpart there.
 */
LF_API int lf_backward_ex(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                          const void* grad_out_dev, const void* s_f_dev, int32_t s_f_planes, int32_t grad_ab_dtype,
                          void* grad_x_dev, void* grad_a_dev, void* grad_b_dev, void* workspace_dev,
                          size_t workspace_bytes, lf_stream_t stream);

/*
 * Multi-GPU backward with the gradient exchange inside the gram kernel.  One process per GPU of a
 * node; adapters whose rows span GPUs ("spanning") need dA/dB summed over the GPUs that hold
 * them, and every GPU receives those sums.  Instead of a separate all-reduce, the dA/dB kernel
 * pushes each fp32 block (128 columns x r_pad) it computes for a spanning virtual slot into every
 * rank's exchange buffer over peer mappings (NVLink), and then sums, in rank order, the blocks of
 * every spanning virtual slot as their holders' entries arrive.  Every rank gets the same sums, bit
 * for bit.  Each 64-bit entry carries the call's generation beside the value, so the push needs
 * no fence and no flag.
 *
 *   exchange[r]    rank r's exchange buffer as mapped here (lf_peer_alloc there, lf_ipc_handle /
 *                  lf_ipc_open here; this rank's own: the local pointer), at least
 *                  lf_peer_exchange_bytes(world, n_span * (ceil(N/128) + ceil(K/128)), r_pad_x) bytes
 *   r_pad_x        16, 32 or 64, at least every spanning virtual slot's rank, the same on every rank
 *                  (blocks are exchanged with that many rank columns)
 *   slot_span_dev  [info->n_slots] index of each (virtual) slot among the spanning virtual slots, -1
 *                  for the others (numbering shared by every rank)
 *   span_info_dev  [n_span][3] per spanning virtual slot: its first row in this call's grad_a/grad_b
 *                  layout (those of slots not held here follow info->rank_total), its rank, and the
 *                  mask of ranks that hold it
 *   gen            low 32 bits nonzero, different on consecutive calls, the same on every rank
 *                  (calls alternate between the two halves of the buffers by its parity)
 *
 * Every rank makes the same sequence of calls; a rank whose peers do not arrive stops after the
 * wait limit (lf_set_wait_limit) and lf_device_error reports it.  Tensor-core problems with routed
 * rows only: LF_ERR_UNSUPPORTED otherwise.  No counterpart in the reference (it is single-GPU).
 */
#define LF_MAX_PEERS 8
#define LF_IPC_HANDLE_BYTES 64
typedef struct lf_peer_reduce {
  int32_t world;
  int32_t rank;
  void* exchange[LF_MAX_PEERS];
  const int32_t* slot_span_dev;
  const int32_t* span_info_dev;
  int32_t n_span;
  int32_t r_pad_x;
  uint64_t gen;
} lf_peer_reduce;

LF_API size_t lf_peer_exchange_bytes(int32_t world, int32_t n_blocks, int32_t r_pad);
LF_API int lf_backward_peer(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                            const void* grad_out_dev, const void* s_f_dev, int32_t s_f_planes, int32_t grad_ab_dtype,
                            void* grad_x_dev, void* grad_a_dev, void* grad_b_dev, void* workspace_dev,
                            size_t workspace_bytes, const lf_peer_reduce* peer, lf_stream_t stream);

/* Device memory for an exchange buffer (zeroed), its inter-process handle, and a peer's buffer
 * mapped into this process (cudaIpc*; processes on one node). */
LF_API int lf_peer_alloc(size_t bytes, void** dev_ptr);
LF_API int lf_peer_free(void* dev_ptr);
LF_API int lf_ipc_handle(const void* dev_ptr, void* handle);
LF_API int lf_ipc_open(const void* handle, void** dev_ptr);
LF_API int lf_ipc_close(void* dev_ptr);

/*
 * The backward in separately launchable stages (arguments as lf_backward_ex), for callers that
 * time them or overlap them with other work (e.g. a gradient all-reduce with the grad_x GEMM).
 * `stages` is a bit mask; each stage is a launch of its own and the routed shrinks are never
 * co-scheduled inside the grad_x launch:
 *   LF_BSTAGE_SHRINK   S_b = s_i g B_i (and S_f = s_i x A_i^T unless s_f_dev is given) into the
 *                      workspace
 *   LF_BSTAGE_GRAD_X   grad_x = g W + S_b A (reads S_b from the workspace)
 *   LF_BSTAGE_GRAD_AB  grad_a / grad_b, the segmented grams (read S_f and S_b)
 * A GRAD_X or GRAD_AB call reads what an earlier SHRINK call on the same workspace, tables and
 * inputs left there; stages passed together run in the order above.  No counterpart in the
 * reference.
 */
#define LF_BSTAGE_SHRINK 1
#define LF_BSTAGE_GRAD_X 2
#define LF_BSTAGE_GRAD_AB 4
LF_API int lf_backward_stages(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                              const void* grad_out_dev, const void* s_f_dev, int32_t s_f_planes,
                              int32_t grad_ab_dtype, void* grad_x_dev, void* grad_a_dev, void* grad_b_dev,
                              void* workspace_dev, size_t workspace_bytes, int32_t stages, lf_stream_t stream);

/*
 * Forward of a batch that lives in host memory, streamed in row chunks: chunk i is copied to
 * x_dev on `h2d_stream` while chunk i-1 is computed on `stream` and chunk i-2 is copied back to
 * y_host on `d2h_stream`, so both PCIe directions and the GPU work overlap.  All copies and
 * launches are enqueued by this one call (no per-chunk host round trips); `stream` waits for
 * the last copy back, so synchronizing `stream` makes y_host valid.
 *  - prob: the whole batch (T rows, K, N, dtype, w_dev and the adapter slabs); prob->x_dev is
 *    ignored.  x_host [T,K] and y_host [T,N] should be pinned; x_dev [T,K] and y_dev [T,N] are
 *    device buffers the call fills.
 *  - chunks: rows [row0, row0 + rows) in order, each with tables of its own routes (rows rebased
 *    to the chunk) built over the whole batch's slots, so every chunk reads the same slabs.
 *  - workspace: at least the largest lf_forward_workspace_bytes of the chunks' tables; chunks
 *    run one after another on `stream` and share it.
 *  - The copies start after the work already enqueued on `stream` (they wait for it).
 * Returns the first failing chunk's status (nothing after it is enqueued).  No counterpart in
 * the reference (its ops take device tensors).
 */
typedef struct lf_host_chunk {
  int32_t row0;
  int32_t rows;
  const lf_plan_info* info;
  const int32_t* table_dev;
} lf_host_chunk;
LF_API int lf_forward_host(const lf_problem* prob, const lf_host_chunk* chunks, int32_t n_chunks,
                           const void* x_host, void* y_host, void* x_dev, void* y_dev, void* workspace_dev,
                           size_t workspace_bytes, lf_stream_t stream, lf_stream_t h2d_stream,
                           lf_stream_t d2h_stream);

/*
 * Forward for callers that cannot allocate device memory: same inputs, output and result as
 * lf_forward, but no workspace argument.  The scratch lives in a fixed array of
 * LF_NOALLOC_SCRATCH_BYTES that the library declares in device memory; every GPU that loads the
 * library holds that array until the process exits.  No counterpart in the reference (its ops
 * allocate freely through torch).
 *  - Returns LF_ERR_CAPACITY when the workspace's fixed sections exceed the array (the
 *    K-split tail scratch is optional and uses what is left).
 *  - Allocates nothing: no cudaMalloc/cudaFree and no allocating library call.
 *  - The first call on each device looks up the array's device address (with that device
 *    current); make that first call before any stream capture.
 *  - All calls on a device share the one array: calls whose work overlaps on the GPU (other
 *    streams, other host threads) race on it and must be serialized by the caller.
 *  - The array's address is kept per device ordinal for the life of the process: do not use this
 *    entry point (or the library) across a cudaDeviceReset of that device.
 */
#define LF_NOALLOC_SCRATCH_BYTES (16u << 20)
LF_API int lf_forward_noalloc(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                              void* y_dev, lf_stream_t stream);

/*
 * One run of lf_copy_rows.  Flattened row g of the copy belongs to the run with the largest
 * row0 <= g; runs are sorted by row0, and a run covers flattened rows [row0, row0 + rows).
 */
typedef struct lf_row_run {
  uint64_t src;       /* device address of the run's first source row */
  uint64_t dst;       /* device address of the run's first destination row */
  int64_t src_stride; /* bytes between consecutive source rows */
  int64_t dst_stride; /* bytes between consecutive destination rows */
  int64_t rows;       /* rows in the run */
  int64_t row0;       /* flattened index of the run's first row (running sum of `rows`) */
} lf_row_run;

/*
 * Copy the rows of every run (row_bytes bytes each, byte-exact) in one launch; `runs_dev` is
 * device memory holding n_runs entries and total_rows = sum of their rows.  Gathers request rows
 * into the fused batch (replaces the torch.cat of lorafusion/scheduler/data_batcher.py:61-80)
 * and splits fused output rows back per request (replaces the per-row loop of
 * data_batcher.py:90-103).  Enqueued on `stream`; never synchronizes.
 */
LF_API int lf_copy_rows(const lf_row_run* runs_dev, int32_t n_runs, int64_t row_bytes, int64_t total_rows,
                        lf_stream_t stream);

/*
 * First-fit-decreasing packing of per-adapter row counts (host only), identical to greedy_pack
 * (lorafusion/scheduler/milp_packer.py:36-72): adapters in the given order are cut into chunks of
 * at most tile_capacity rows, the chunks are stably sorted by size, largest first, and each goes
 * into the first bin with room, else into a new bin at the end.  Adapters with rows <= 0 give no
 * chunk.  Result (CSR): bin b holds entries [bin_start[b], bin_start[b+1]) of
 * entry_adapter / entry_rows in insertion order; *n_entries and *n_bins are set.  Needs
 * max_entries >= the chunk count (bin_start has max_entries + 1 slots); otherwise returns
 * LF_ERR_CAPACITY with *n_entries = the chunk count.  tile_capacity <= 0: LF_ERR_INVALID_ARG.
 */
LF_API int lf_greedy_pack(const int32_t* adapter_ids, const int32_t* rows, int32_t n_adapters, int32_t tile_capacity,
                          int32_t max_entries, int32_t* bin_start, int32_t* entry_adapter, int32_t* entry_rows,
                          int32_t* n_entries, int32_t* n_bins);

/*
 * Row -> rank assignment for one process per GPU (host only).  No counterpart in the reference
 * (it runs on one device).  Input: the packing (CSR of lf_greedy_pack), whose entries in bin order
 * are the global fused rows.  Every rank may hold its even share of the rows rounded up to whole
 * `granule_rows` (the fused GEMM's row tile).  Adapters, most rows first (ties: first appearance),
 * go whole to the rank they fit best (least room left, then lowest rank); an adapter that fits
 * nowhere is cut over the ranks with most room (then lowest rank), each taking what it has room
 * for, so only such adapters span ranks.  An adapter's rows go to its parts in global row order.
 * Output: global row ranges [range_start, range_end) with their rank, ascending, adjacent ranges
 * of one rank merged; *n_ranges is set (LF_ERR_CAPACITY when more than max_ranges: call again with
 * that many).  Deterministic: every rank computes the same ranges without communicating.
 */
LF_API int lf_assign_rows(const int32_t* bin_start, const int32_t* entry_adapter, const int32_t* entry_rows,
                          int32_t n_bins, int32_t world_size, int32_t granule_rows, int32_t max_ranges,
                          int64_t* range_start, int64_t* range_end, int32_t* range_rank, int32_t* n_ranges);

/*
 * Read and clear the device-side error word (bounded-wait timeouts inside kernels: codes 0x101 ..
 * 0x105).  Synchronizes the current device.  *code = 0 when no kernel reported a problem; after a
 * nonzero code the outputs of the calls since the previous read are undefined.
 */
LF_API int lf_device_error(int32_t* code);

/*
 * Bound of every wait inside this library's kernels on the current device, in nanoseconds
 * (0 = the default, about 1 s; otherwise 1 ms .. 60 s).  A wait that runs out records its code in
 * the device status word (lf_device_error), makes its CTA stop, lets the copies and MMAs it
 * started finish, frees its tensor memory and returns; nothing traps.  Synchronous; call it while
 * no kernel of this library runs on the device.  No counterpart in the reference.
 */
LF_API int lf_set_wait_limit(uint64_t limit_ns);

/*
 * Test hook for the failure path: the next `launches` co-scheduled GEMM launches (shrink inside the
 * GEMM launch) make their GEMM CTAs wait for a ready value that no shrink item publishes, so those
 * waits run out after the wait limit and the launch reports a timeout through lf_device_error; the
 * launch's outputs are then undefined.  0 cancels.  No counterpart in the reference.
 */
LF_API int lf_inject_stale_ready(int32_t launches);

/* Static description of a status code. */
LF_API const char* lf_status_string(int status);

/* Build identification: "lorafusion_b200 <version> sm_100a". */
LF_API const char* lf_version(void);

/*
 * Release what the library itself holds on every device: lf_forward_host's stream-ordering
 * events.  Work already enqueued is unaffected (a destroyed event that a stream still waits on
 * is freed when it completes); later calls recreate what they need.  The caller owns every other
 * buffer.  Returns LF_OK.
 */
LF_API int lf_release(void);

#ifdef __cplusplus
}
#endif

#endif /* LORAFUSION_B200_H */
