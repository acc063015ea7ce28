// C ABI of the fused multi-adapter LoRA operator: argument checks, TMA descriptors,
// kernel dispatch.  No torch types cross this boundary; see include/lorafusion_b200.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "lf_internal.cuh"
#include "lf_ptx.cuh"

namespace lf {

// Device control word (one per device context): the status bounded waits inside the kernels
// record, and the wait limit they read.
__device__ DeviceCtl g_device_ctl = {0, 0, kWaitLimitNs};

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct DeviceState {
  bool ready = false;
  int num_sms = 0;
  int* status = nullptr;      // address of g_device_ctl.status on this device
  std::atomic<bool> no_cosched{false};  // the co-scheduled (cooperative) launch was refused here once
  std::atomic<int> refusal{0};          // the cudaError_t that refused launch returned
  std::vector<cudaEvent_t> events;  // lf_forward_host's stream-ordering events (grown on demand)
  std::mutex ev_mu;
};

std::mutex g_mu;
DeviceState g_dev[64];

// A profiling or checking tool injected into the process replays or serializes kernels, and a
// co-scheduled launch (whose CTAs wait on each other) then fails, so the default is "no
// co-scheduled launches" when one is present.  Signs of one: the variables CUDA tools set for
// their injection (CUDA_INJECTION64_PATH; Nsight Compute's NV_NSIGHT_INJECTION_* and
// NV_COMPUTE_PROFILER_PERFWORKS_DIR; NVIDIA_PROCESS_INJECTION_*), or an injection library mapped
// into the process.
bool tool_injected() {
  for (const char* v : {"CUDA_INJECTION64_PATH", "NV_NSIGHT_INJECTION_TRANSPORT_TYPE", "NV_COMPUTE_PROFILER_PERFWORKS_DIR",
                        "NVIDIA_PROCESS_INJECTION_CRASH_REPORTING"}) {
    const char* x = std::getenv(v);
    if (x != nullptr && x[0] != '\0') return true;
  }
  if (FILE* f = std::fopen("/proc/self/maps", "r")) {
    char line[1024];
    bool found = false;
    while (!found && std::fgets(line, sizeof(line), f))
      found = std::strstr(line, "libcuda-injection") != nullptr || std::strstr(line, "InjectionTarget") != nullptr;
    std::fclose(f);
    if (found) return true;
  }
  return false;
}
int default_cosched_mode() { return tool_injected() ? 0 : 1; }
// process-wide switch (lf_set_co_scheduling): 0 off, 1 dedicated, 2 prologue
std::atomic<int> g_cosched_mode{default_cosched_mode()};

// Test hook (lf_inject_stale_ready): co-scheduled launches that still make their GEMM CTAs wait
// for a ready value no shrink item publishes.
std::atomic<int> g_stale_ready{0};
uint64_t wait_generation(uint64_t gen) {
  int n = g_stale_ready.load();
  while (n > 0 && !g_stale_ready.compare_exchange_weak(n, n - 1)) {
  }
  return n > 0 ? gen + 2 : gen;
}

bool cosched_allowed(const DeviceState* ds) { return !ds->no_cosched.load() && g_cosched_mode.load() != 0; }

// A cooperative launch that returned `e` ran nothing: clear the (non-sticky) launch error, keep
// the code for lf_get_co_scheduling and use ordinary launches on this device from now on.
void refuse_cosched(DeviceState* ds, cudaError_t e) {
  (void)cudaGetLastError();
  int expect = 0;
  ds->refusal.compare_exchange_strong(expect, static_cast<int>(e));
  ds->no_cosched.store(true);
}
// Shrink inside the GEMM launch: on CTA pairs the GEMM's round count leaves idle (default, when
// there are at least four), or as every CTA's prologue (mode 2).
bool cosched_prologue() { return g_cosched_mode.load() == 2; }
EncodeTiledFn g_encode = nullptr;

int elem_bytes(int dtype) { return dtype == LF_F32 ? 4 : 2; }

cudaError_t device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& d = g_dev[dev];
  if (!d.ready) {
    e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.status), g_device_ctl);
    if (e != cudaSuccess) return e;
    d.ready = true;
  }
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return e != cudaSuccess ? e : cudaErrorUnknown;
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  *out = &d;
  return cudaSuccess;
}

// 2-D tile map over a row-major [outer, inner] matrix with row pitch `pitch_bytes`.
bool make_map(CUtensorMap* m, int dtype, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch_bytes,
              uint32_t box_inner, uint32_t box_outer) {
  const uint32_t span = box_inner * static_cast<uint32_t>(elem_bytes(dtype));
  CUtensorMapSwizzle sw = span == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                          : span == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                       : CU_TENSOR_MAP_SWIZZLE_32B;
  if (span != 128 && span != 64 && span != 32) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == LF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  std::memset(m, 0, sizeof(*m));
  CUresult r = g_encode(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int to_status(cudaError_t e) { return e == cudaSuccess ? LF_OK : LF_ERR_CUDA; }

// segment tiles plus one all-zero block (index n_segtiles) the pair GEMM pads with
size_t segtile_elems(const lf_plan_info* info) {
  return static_cast<size_t>(info->n_segtiles + 1) * LF_TILE_ROWS * static_cast<size_t>(info->r_pad);
}

// One S_ext buffer, 256-byte multiple: f64 for the CUDA-core path, or four bf16/f16 planes for
// the tensor-core path.  A tensor-core shrink writes each value v as hi = round(v) in plane h and
// lo = round(v - hi) in plane kh + h, where kh (1 or 2) counts its K-half partial products (two
// when it runs inside the GEMM launch): planes [hi of each K half..., lo of each K half...].  The
// LoRA expand reads the hi planes; the dA/dB grams read all 2*kh planes, so S enters the
// gradient sums with about 16 significant bits instead of 8.
size_t sext_bytes(const lf_plan_info* info) { return (segtile_elems(info) * 8 + 255) & ~size_t(255); }

constexpr int kSextPlanes = 4;  // planes one tensor-core S_ext buffer holds

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// ready flags of the (job, unit, K half) items when shrinks run inside the GEMM launch
// (one job in the forward, two in the backward)
size_t flag_bytes(const lf_plan_info* info, int jobs = 1) {
  return (static_cast<size_t>(info->n_shrink_units) * 2 * 8 * jobs + 255) & ~size_t(255);
}

// Per-launch flag value: unique within the process, so flags left in a reused workspace by an
// earlier launch never read as ready; a stray equal 64-bit value in fresh memory is the only
// (negligible) collision.
uint64_t next_generation() {
  static std::atomic<uint64_t> gen{
      (static_cast<uint64_t>(std::chrono::steady_clock::now().time_since_epoch().count()) << 1) | 1u};
  return gen.fetch_add(2, std::memory_order_relaxed) + 2;
}

int check_problem(const lf_problem* p, const lf_plan_info* info, const int32_t* table_dev) {
  if (!p || !info || (!table_dev && info->table_words > 0)) return LF_ERR_INVALID_ARG;
  if (p->dtype != LF_F32 && p->dtype != LF_BF16 && p->dtype != LF_F16) return LF_ERR_INVALID_ARG;
  if (p->T < 0 || p->K < 0 || p->N < 0) return LF_ERR_INVALID_ARG;
  if (p->T != info->total_rows) return LF_ERR_ROUTING;
  if (info->r_pad != 16 && info->r_pad != 32 && info->r_pad != 64) return LF_ERR_INVALID_ARG;
  return LF_OK;
}

// Tensor-core path: bf16/f16 with every row pitch and base 16-byte aligned (TMA).
bool tc_eligible(const lf_problem* p, std::initializer_list<const void*> ptrs) {
  if (p->dtype == LF_F32) return false;
  if (p->K == 0 || p->N == 0 || p->K % 8 != 0 || p->N % 8 != 0) return false;
  for (const void* q : ptrs)
    if (q && !aligned16(q)) return false;
  return true;
}

}  // namespace

Tables make_tables(const lf_plan_info* info, const int32_t* table_dev) {
  Tables t{};
  t.base = table_dev;
  t.off_tile_st = info->off_tile_st;
  t.off_st_tile = info->off_st_tile;
  t.off_st_lo = info->off_st_lo;
  t.off_st_hi = info->off_st_hi;
  t.off_st_slot = info->off_st_slot;
  t.off_st_scale = info->off_st_scale;
  t.off_slot_st = info->off_slot_st;
  t.off_slot_list = info->off_slot_list;
  t.off_slot_rank = info->off_slot_rank;
  t.off_rank_prefix = info->off_rank_prefix;
  t.off_slot_order = info->off_slot_order;
  t.off_unit_tile = info->off_unit_tile;
  t.off_unit_st0 = info->off_unit_st0;
  t.off_unit_nst = info->off_unit_nst;
  t.off_pair_lora = info->off_pair_lora;
  t.off_pl_a = info->off_pl_a;
  t.off_pl_b = info->off_pl_b;
  t.off_pl_slot = info->off_pl_slot;
  t.off_tile_unit = info->off_tile_unit;
  t.n_tiles = info->n_tiles;
  t.n_segtiles = info->n_segtiles;
  t.n_slots = info->n_slots;
  t.n_units = info->n_shrink_units;
  t.r_pad = info->r_pad;
  t.err = nullptr;
  return t;
}

}  // namespace lf

using namespace lf;

namespace lf {
size_t forward_min_workspace_bytes(const lf_plan_info* info) {
  return info ? align256(sext_bytes(info) + flag_bytes(info)) : 0;
}
}  // namespace lf

namespace {
size_t backward_min_workspace_bytes(const lf_plan_info* info) {
  return info ? align256(2 * sext_bytes(info) + flag_bytes(info, 2) +
                         gram_scratch_bytes(info->r_pad > 0 ? info->r_pad : 16))
              : 0;
}

// The K-split tail's scratch at byte `off` of a workspace of `bytes`: as many partial tiles as
// fit there (none: no split).
PairTail tail_scratch(void* ws, size_t bytes, size_t off) {
  PairTail t{};
  if (ws == nullptr || bytes < off + kTailFlagBytes + kTailPartialBytes) return t;
  char* base = static_cast<char*>(ws) + off;
  if (!aligned16(base)) return t;  // partial tiles are moved by bulk copies: no split tail
  t.flags = reinterpret_cast<uint64_t*>(base);
  t.partial = reinterpret_cast<float*>(base + kTailFlagBytes);
  const size_t fit = (bytes - off - kTailFlagBytes) / kTailPartialBytes;
  t.slots = static_cast<int>(fit < static_cast<size_t>(kTailSlots) ? fit : kTailSlots);
  t.gen = next_generation();
  return t;
}
}  // namespace

extern "C" size_t lf_forward_workspace_bytes(const lf_plan_info* info, int32_t dtype) {
  (void)dtype;
  return info ? forward_min_workspace_bytes(info) + tail_scratch_bytes() : 0;
}

extern "C" size_t lf_backward_workspace_bytes(const lf_plan_info* info, int32_t dtype) {
  (void)dtype;
  return info ? backward_min_workspace_bytes(info) + tail_scratch_bytes() : 0;
}

extern "C" int lf_pack_adapters(int32_t src_dtype, int32_t dst_dtype, const uint64_t* src_ptrs_dev,
                                const int32_t* slot_rank_dev, int32_t n_slots, int32_t rank_dim, int32_t other_dim,
                                int32_t transpose, int32_t d0, int32_t d1, void* dst_dev, lf_stream_t stream) {
  if (src_dtype < 0 || src_dtype > 2 || dst_dtype < 0 || dst_dtype > 2) return LF_ERR_INVALID_ARG;
  if (n_slots < 0 || d0 < 0 || d1 < 0 || other_dim < 0 || (rank_dim != 0 && rank_dim != 1)) return LF_ERR_INVALID_ARG;
  if (n_slots == 0 || d0 == 0 || d1 == 0) return LF_OK;
  if (!src_ptrs_dev || !slot_rank_dev || !dst_dev) return LF_ERR_INVALID_ARG;
  return to_status(pack_adapters(src_dtype, dst_dtype, src_ptrs_dev, slot_rank_dev, n_slots, rank_dim, other_dim,
                                 transpose, d0, d1, dst_dev, static_cast<cudaStream_t>(stream)));
}

namespace {
// The forward stages; *sf_planes (if given) receives the K-half planes of S_f the shrink left in
// the workspace (2 when it ran inside the GEMM launch, 1 as a launch of its own, 0 without a
// tensor-core shrink), the value lf_backward_sf needs.
int forward_impl(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev, void* y_dev,
                 void* workspace_dev, size_t workspace_bytes, void* tail_dev, size_t tail_bytes, int32_t stages,
                 lf_stream_t stream, int32_t* sf_planes) {
  if (sf_planes) *sf_planes = 0;
  int rc = check_problem(prob, info, table_dev);
  if (rc != LF_OK) return rc;
  if (stages <= 0 || stages > 31 || ((stages & LF_STAGE_EXPAND) && (stages & LF_STAGE_BASE))) return LF_ERR_INVALID_ARG;
  const int T = prob->T, K = prob->K, N = prob->N;
  if (T == 0 || N == 0) return LF_OK;
  if (!prob->x_dev || !prob->w_dev || !prob->a_pack_dev || !prob->b_pack_dev || !y_dev) return LF_ERR_INVALID_ARG;
  if (workspace_bytes < forward_min_workspace_bytes(info) || !workspace_dev) return LF_ERR_CAPACITY;
  DeviceState* ds = nullptr;
  cudaError_t e = device_state(&ds);
  if (e != cudaSuccess) return LF_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Tables tb = make_tables(info, table_dev);
  tb.err = ds->status;
  const int dt = prob->dtype;
  const int rp = info->r_pad;
  const bool do_shrink = (stages & LF_STAGE_SHRINK) != 0;
  const bool do_gemm = (stages & (LF_STAGE_EXPAND | LF_STAGE_BASE)) != 0;
  const bool lora = (stages & LF_STAGE_EXPAND) != 0 && info->n_segtiles > 0;

  if (tc_eligible(prob, {prob->x_dev, prob->w_dev, prob->a_pack_dev, prob->b_pack_dev, y_dev, workspace_dev})) {
    const bool single = (stages & LF_STAGE_SINGLE_CTA) != 0;
    const uint32_t nbox = single ? 256 : 128;  // rows of W / B_i per CTA and tile
    TcMaps maps;
    CUtensorMap a_map;
    const size_t es = 2;
    const uint64_t s_rows = kSextPlanes * static_cast<uint64_t>(info->n_segtiles + 1) * LF_TILE_ROWS;
    bool ok = make_map(&maps.p, dt, prob->x_dev, K, T, K * es, 64, 128) &&
              make_map(&maps.q, dt, prob->w_dev, K, N, K * es, 64, nbox) &&
              make_map(&a_map, dt, prob->a_pack_dev, K, static_cast<uint64_t>(info->n_slots) * rp, K * es, 64, rp);
    if (info->n_segtiles > 0)
      ok = ok && make_map(&maps.s, dt, workspace_dev, rp, s_rows, rp * es, rp, 128) &&
           make_map(&maps.l, dt, prob->b_pack_dev, rp, static_cast<uint64_t>(info->n_slots) * N, rp * es, rp, nbox);
    else
      maps.s = maps.l = maps.p;
    ok = ok && make_map(&maps.o, dt, y_dev, N, T, N * es, 64, 32);
    if (!ok) return LF_ERR_UNSUPPORTED;
    // Shrink and expand requested together: run the shrink on CTA pairs the GEMM's round count
    // leaves idle, inside the same launch, when there are enough of them.
    const bool separate = (stages & LF_STAGE_SEPARATE) != 0;
    const bool fuse = !single && !separate && do_shrink && lora && cosched_allowed(ds);
    const int spare = fuse && !cosched_prologue() ? pair_spare_pairs(T, N, ds->num_sms, info->n_shrink_units) : 0;
    // the K-split tail needs a cooperative launch too
    const PairTail tail = tail_dev ? tail_scratch(tail_dev, tail_bytes, 0)
                                   : tail_scratch(workspace_dev, workspace_bytes, forward_min_workspace_bytes(info));
    if (fuse && (spare > 0 || cosched_prologue())) {
      PairShrink sh{};
      sh.a_map = a_map;
      sh.s_ext = workspace_dev;
      sh.unit_ready = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace_dev) + sext_bytes(info));
      sh.gen = next_generation();
      sh.wait_gen = wait_generation(sh.gen);
      sh.n_pairs = spare;
      sh.prologue = cosched_prologue();
      e = tc_gemm_pair(dt, false, maps, T, N, K, lora, tb, y_dev, N, ds->num_sms, st, &sh, &tail);
      if (e == cudaSuccess) {
        if (sf_planes) *sf_planes = 2;
        return LF_OK;
      }
      // The cooperative launch was refused (e.g. other work holds SMs, or a profiler
      // serializes launches): nothing ran; use the two-launch path from now on.
      refuse_cosched(ds, e);
    }
    if (do_shrink) {
      e = tc_shrink(dt, maps.p, a_map, K, tb, workspace_dev, ds->num_sms, st);
      if (e != cudaSuccess) return LF_ERR_CUDA;
      if (sf_planes) *sf_planes = 1;
    }
    if (do_gemm) {
      if (single) {
        e = tc_gemm(dt, false, maps, T, N, K, lora, tb, y_dev, N, ds->num_sms, st);
      } else {
        e = tc_gemm_pair(dt, false, maps, T, N, K, lora, tb, y_dev, N, ds->num_sms, st, nullptr,
                         cosched_allowed(ds) ? &tail : nullptr);
        if (e != cudaSuccess && cosched_allowed(ds)) {  // cooperative launch refused: nothing ran
          refuse_cosched(ds, e);
          e = tc_gemm_pair(dt, false, maps, T, N, K, lora, tb, y_dev, N, ds->num_sms, st);
        }
      }
    }
    return to_status(e);
  }

  double* s_ext = static_cast<double*>(workspace_dev);
  if (do_shrink) {
    e = simt_shrink(dt, prob->x_dev, K, K, prob->a_pack_dev, tb, s_ext, st);
    if (e != cudaSuccess) return LF_ERR_CUDA;
  }
  if (do_gemm)
    e = simt_gemm(dt, prob->x_dev, K, prob->w_dev, K, 1, T, N, K, s_ext, lora ? prob->b_pack_dev : nullptr, tb, y_dev,
                  N, st);
  return to_status(e);
}
}  // namespace

extern "C" int lf_forward_stages(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                                 void* y_dev, void* workspace_dev, size_t workspace_bytes, int32_t stages,
                                 lf_stream_t stream) {
  return forward_impl(prob, info, table_dev, y_dev, workspace_dev, workspace_bytes, nullptr, 0, stages, stream,
                      nullptr);
}

extern "C" int lf_forward_sf(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev, void* y_dev,
                             void* workspace_dev, size_t workspace_bytes, void* tail_dev, size_t tail_bytes,
                             int32_t* s_f_planes, lf_stream_t stream) {
  if (!s_f_planes) return LF_ERR_INVALID_ARG;
  return forward_impl(prob, info, table_dev, y_dev, workspace_dev, workspace_bytes, tail_dev, tail_bytes,
                      LF_STAGE_SHRINK | LF_STAGE_EXPAND, stream, s_f_planes);
}

extern "C" size_t lf_forward_fixed_workspace_bytes(const lf_plan_info* info, int32_t dtype) {
  (void)dtype;
  return forward_min_workspace_bytes(info);
}

extern "C" int lf_forward_launch_count(const lf_problem* prob, const lf_plan_info* info) {
  if (!prob || !info) return -LF_ERR_INVALID_ARG;
  if (prob->T == 0 || prob->N == 0) return 0;
  DeviceState* ds = nullptr;
  if (device_state(&ds) != cudaSuccess) return -LF_ERR_CUDA;
  const bool tc = prob->dtype != LF_F32 && prob->K > 0 && prob->K % 8 == 0 && prob->N % 8 == 0;
  if (tc && info->n_segtiles > 0 && cosched_allowed(ds) &&
      (cosched_prologue() || pair_spare_pairs(prob->T, prob->N, ds->num_sms, info->n_shrink_units) > 0))
    return 1;
  return 2;
}

extern "C" int lf_backward_launch_count(const lf_problem* prob, const lf_plan_info* info) {
  if (!prob || !info) return -LF_ERR_INVALID_ARG;
  if (prob->T == 0) return 0;
  DeviceState* ds = nullptr;
  if (device_state(&ds) != cudaSuccess) return -LF_ERR_CUDA;
  const bool tc = prob->dtype != LF_F32 && prob->K > 0 && prob->K % 8 == 0 && prob->N % 8 == 0;
  const bool lora = info->n_segtiles > 0 && info->n_slots > 0;
  if (!tc) return 5;
  if (!lora) return 1;
  return (cosched_allowed(ds) &&
          (cosched_prologue() || pair_spare_pairs(prob->T, prob->K, ds->num_sms, info->n_shrink_units) > 0))
             ? 2
             : 4;
}

extern "C" int lf_set_co_scheduling(int32_t enable) {
  if (enable < 0 || enable > 2) return LF_ERR_INVALID_ARG;
  g_cosched_mode.store(enable);
  return LF_OK;
}

extern "C" int lf_set_wait_limit(uint64_t limit_ns) {
  if (limit_ns != 0 && (limit_ns < 1000000ull || limit_ns > 60000000000ull)) return LF_ERR_INVALID_ARG;
  const unsigned long long v = limit_ns == 0 ? kWaitLimitNs : limit_ns;
  DeviceState* ds = nullptr;
  if (device_state(&ds) != cudaSuccess) return LF_ERR_CUDA;
  if (cudaMemcpyToSymbol(g_device_ctl, &v, sizeof(v), offsetof(DeviceCtl, wait_limit_ns)) != cudaSuccess)
    return LF_ERR_CUDA;
  return LF_OK;
}

extern "C" int lf_inject_stale_ready(int32_t launches) {
  if (launches < 0) return LF_ERR_INVALID_ARG;
  g_stale_ready.store(launches);
  return LF_OK;
}

extern "C" int lf_get_co_scheduling(int32_t* mode, int32_t* refused_error) {
  if (!mode || !refused_error) return LF_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  if (device_state(&ds) != cudaSuccess) return LF_ERR_CUDA;
  *mode = g_cosched_mode.load();
  *refused_error = ds->no_cosched.load() ? ds->refusal.load() : 0;
  return LF_OK;
}

extern "C" int lf_release(void) {
  for (DeviceState& d : g_dev) {
    std::lock_guard<std::mutex> lk(d.ev_mu);
    for (cudaEvent_t ev : d.events) (void)cudaEventDestroy(ev);
    d.events.clear();
  }
  return LF_OK;
}

extern "C" int lf_forward_host(const lf_problem* prob, const lf_host_chunk* chunks, int32_t n_chunks,
                               const void* x_host, void* y_host, void* x_dev, void* y_dev, void* workspace_dev,
                               size_t workspace_bytes, lf_stream_t stream, lf_stream_t h2d_stream,
                               lf_stream_t d2h_stream) {
  if (!prob || n_chunks < 0 || (n_chunks > 0 && (!chunks || !x_host || !y_host || !x_dev || !y_dev)))
    return LF_ERR_INVALID_ARG;
  if (prob->dtype != LF_F32 && prob->dtype != LF_BF16 && prob->dtype != LF_F16) return LF_ERR_INVALID_ARG;
  const size_t es = static_cast<size_t>(elem_bytes(prob->dtype));
  // Every chunk is checked before anything is enqueued, with the checks lf_forward makes, so a
  // bad chunk list fails with nothing in flight.
  int end = 0;
  for (int32_t c = 0; c < n_chunks; ++c) {
    const lf_host_chunk& ch = chunks[c];
    if (ch.row0 != end || ch.rows < 0 || !ch.info || ch.info->total_rows != ch.rows) return LF_ERR_INVALID_ARG;
    lf_problem pc = *prob;
    pc.T = ch.rows;
    const int rc = check_problem(&pc, ch.info, ch.table_dev);
    if (rc != LF_OK) return rc;
    if (ch.rows > 0 && prob->N > 0 && (workspace_bytes < forward_min_workspace_bytes(ch.info) || !workspace_dev))
      return LF_ERR_CAPACITY;
    end += ch.rows;
  }
  if (end != prob->T) return LF_ERR_INVALID_ARG;
  if (n_chunks == 0) return LF_OK;
  if (prob->N > 0 && (!prob->w_dev || !prob->a_pack_dev || !prob->b_pack_dev)) return LF_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  if (device_state(&ds) != cudaSuccess) return LF_ERR_CUDA;
  const size_t n_ev = 2 * static_cast<size_t>(n_chunks) + 3;
  std::lock_guard<std::mutex> lk(ds->ev_mu);  // one enqueue at a time per device shares the events
  while (ds->events.size() < n_ev) {
    cudaEvent_t ev;
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return LF_ERR_CUDA;
    ds->events.push_back(ev);
  }
  cudaEvent_t* ev = ds->events.data();
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  cudaStream_t si = static_cast<cudaStream_t>(h2d_stream);
  cudaStream_t so = static_cast<cudaStream_t>(d2h_stream);
  // the copies come after the work already on `stream` (earlier readers of x_dev / y_dev)
  if (cudaEventRecord(ev[0], cs) != cudaSuccess || cudaStreamWaitEvent(si, ev[0], 0) != cudaSuccess ||
      cudaStreamWaitEvent(so, ev[0], 0) != cudaSuccess)
    return LF_ERR_CUDA;
  const char* xh = static_cast<const char*>(x_host);
  char* yh = static_cast<char*>(y_host);
  char* xd = static_cast<char*>(x_dev);
  char* yd = static_cast<char*>(y_dev);
  const size_t row_in = static_cast<size_t>(prob->K) * es, row_out = static_cast<size_t>(prob->N) * es;
  int rc = LF_OK;
  for (int32_t c = 0; c < n_chunks && rc == LF_OK; ++c) {
    const lf_host_chunk& ch = chunks[c];
    const size_t r0 = static_cast<size_t>(ch.row0), nr = static_cast<size_t>(ch.rows);
    cudaEvent_t ev_in = ev[3 + 2 * c], ev_out = ev[4 + 2 * c];
    if (cudaMemcpyAsync(xd + r0 * row_in, xh + r0 * row_in, nr * row_in, cudaMemcpyHostToDevice, si) != cudaSuccess ||
        cudaEventRecord(ev_in, si) != cudaSuccess || cudaStreamWaitEvent(cs, ev_in, 0) != cudaSuccess) {
      rc = LF_ERR_CUDA;
      break;
    }
    lf_problem pc = *prob;
    pc.T = ch.rows;
    pc.x_dev = xd + r0 * row_in;
    rc = lf_forward(&pc, ch.info, ch.table_dev, yd + r0 * row_out, workspace_dev, workspace_bytes, stream);
    if (rc != LF_OK) break;
    if (cudaEventRecord(ev_out, cs) != cudaSuccess || cudaStreamWaitEvent(so, ev_out, 0) != cudaSuccess ||
        cudaMemcpyAsync(yh + r0 * row_out, yd + r0 * row_out, nr * row_out, cudaMemcpyDeviceToHost, so) != cudaSuccess)
      rc = LF_ERR_CUDA;
  }
  // `stream` waits for both copy streams, also after a failure part-way: the caller may release
  // x_dev / y_dev / the host buffers once `stream` has passed this point.
  const bool joined = cudaEventRecord(ev[1], so) == cudaSuccess && cudaStreamWaitEvent(cs, ev[1], 0) == cudaSuccess &&
                      cudaEventRecord(ev[2], si) == cudaSuccess && cudaStreamWaitEvent(cs, ev[2], 0) == cudaSuccess;
  if (rc == LF_OK && !joined) rc = LF_ERR_CUDA;
  return rc;
}

extern "C" int lf_forward(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev, void* y_dev,
                          void* workspace_dev, size_t workspace_bytes, lf_stream_t stream) {
  return lf_forward_stages(prob, info, table_dev, y_dev, workspace_dev, workspace_bytes,
                           LF_STAGE_SHRINK | LF_STAGE_EXPAND, stream);
}

namespace {
// The backward; `sf_given` (planes `sf_planes`) is S_f = s x A_i^T as a forward left it in its
// workspace (tensor-core path only), or null to compute it here.
// `stages` 0: the whole backward (routed shrinks inside the grad_x launch when co-scheduling
// allows); otherwise the LF_BSTAGE_* bits, each a launch of its own (shrinks never co-scheduled).
int backward_impl(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev, const void* grad_out_dev,
                  const void* sf_given, int sf_planes, int grad_f32, void* grad_x_dev, void* grad_a_dev,
                  void* grad_b_dev, void* workspace_dev, size_t workspace_bytes, lf_stream_t stream,
                  int stages = 0, const lf_peer_reduce* peer = nullptr) {
  int rc = check_problem(prob, info, table_dev);
  if (rc != LF_OK) return rc;
  GramPeer gp{};
  if (peer != nullptr) {  // spanning adapters' blocks exchanged by the gram: tensor-core path only
    if (peer->world < 2 || peer->world > LF_MAX_PEERS || peer->rank < 0 || peer->rank >= peer->world ||
        peer->n_span <= 0 || !peer->slot_span_dev || !peer->span_info_dev || static_cast<uint32_t>(peer->gen) == 0 ||
        (peer->r_pad_x != 16 && peer->r_pad_x != 32 && peer->r_pad_x != 64))
      return LF_ERR_INVALID_ARG;
    for (int r = 0; r < peer->world; ++r)
      if (!peer->exchange[r] || !aligned16(peer->exchange[r])) return LF_ERR_INVALID_ARG;
    if (prob->dtype == LF_F32 || prob->T == 0 || info->n_segtiles == 0 || info->n_slots == 0)
      return LF_ERR_UNSUPPORTED;
    gp.world = peer->world;
    gp.rank = peer->rank;
    for (int r = 0; r < peer->world; ++r) gp.xbuf[r] = static_cast<uint8_t*>(peer->exchange[r]);
    gp.slot_span = peer->slot_span_dev;
    gp.span_info = peer->span_info_dev;
    gp.n_span = peer->n_span;
    gp.cblk_b = (prob->N + 127) / 128;
    gp.blocks_per_span = gp.cblk_b + (prob->K + 127) / 128;
    gp.n_blocks = gp.n_span * gp.blocks_per_span;
    gp.xr = peer->r_pad_x;
    gp.gen = peer->gen;
  }
  const GramPeer* gpp = peer != nullptr ? &gp : nullptr;
  const bool staged = stages != 0;
  const bool do_shrink = !staged || (stages & LF_BSTAGE_SHRINK) != 0;
  const bool do_gx = !staged || (stages & LF_BSTAGE_GRAD_X) != 0;
  const bool do_gab = !staged || (stages & LF_BSTAGE_GRAD_AB) != 0;
  const int T = prob->T, K = prob->K, N = prob->N;
  const size_t sb = sext_bytes(info);
  if (workspace_bytes < backward_min_workspace_bytes(info) || !workspace_dev) return LF_ERR_CAPACITY;
  DeviceState* ds = nullptr;
  cudaError_t e = device_state(&ds);
  if (e != cudaSuccess) return LF_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int dt = prob->dtype;
  const size_t es = static_cast<size_t>(elem_bytes(dt));
  if (do_gab && info->n_slots > 0 && (!grad_a_dev || !grad_b_dev)) return LF_ERR_INVALID_ARG;
  if (do_gab && (T == 0 || info->n_segtiles == 0)) {  // adapters whose routes are all empty: zero gradients
    const size_t ra = static_cast<size_t>(info->rank_total);
    const size_t gs = grad_f32 ? 4 : es;
    if (ra > 0 && K > 0 && cudaMemsetAsync(grad_a_dev, 0, ra * K * gs, st) != cudaSuccess) return LF_ERR_CUDA;
    if (ra > 0 && N > 0 && cudaMemsetAsync(grad_b_dev, 0, ra * N * gs, st) != cudaSuccess) return LF_ERR_CUDA;
  }
  if (T == 0) return LF_OK;
  if (!prob->x_dev || !prob->w_dev || !grad_out_dev || (do_gx && !grad_x_dev)) return LF_ERR_INVALID_ARG;
  if (info->n_slots > 0 && (!prob->a_pack_dev || !prob->bt_pack_dev || !prob->at_pack_dev))
    return LF_ERR_INVALID_ARG;
  Tables tb = make_tables(info, table_dev);
  tb.err = ds->status;
  const int rp = info->r_pad;
  char* ws = static_cast<char*>(workspace_dev);
  void* s_f = ws;
  void* s_b = ws + sb;
  const bool reuse_sf = sf_given != nullptr && prob->dtype != LF_F32 && (sf_planes == 1 || sf_planes == 2);
  if (reuse_sf) s_f = const_cast<void*>(sf_given);

  const bool tc_path = tc_eligible(prob, {prob->x_dev, prob->w_dev, prob->a_pack_dev, prob->bt_pack_dev,
                                          prob->at_pack_dev, grad_out_dev, grad_x_dev, workspace_dev});
  if (peer != nullptr && !tc_path) return LF_ERR_UNSUPPORTED;
  if (tc_path) {
    CUtensorMap p_x, p_g, a_map, bt_map, sf_map, sb_map;
    TcMaps dx;
    const PairTail tail = tail_scratch(workspace_dev, workspace_bytes, backward_min_workspace_bytes(info));
    const uint64_t s_rows = kSextPlanes * static_cast<uint64_t>(info->n_segtiles + 1) * LF_TILE_ROWS;
    bool ok = make_map(&p_x, dt, prob->x_dev, K, T, K * es, 64, 128) &&
              make_map(&p_g, dt, grad_out_dev, N, T, N * es, 64, 128) &&
              make_map(&dx.q, dt, prob->w_dev, K, N, K * es, 64, 64);
    const bool lora = info->n_segtiles > 0 && info->n_slots > 0;
    if (lora)
      ok = ok &&
           make_map(&a_map, dt, prob->a_pack_dev, K, static_cast<uint64_t>(info->n_slots) * rp, K * es, 64, rp) &&
           make_map(&bt_map, dt, prob->bt_pack_dev, N, static_cast<uint64_t>(info->n_slots) * rp, N * es, 64, rp) &&
           make_map(&sf_map, dt, s_f, rp, s_rows, rp * es, rp, 128) &&
           make_map(&sb_map, dt, s_b, rp, s_rows, rp * es, rp, 128) &&
           make_map(&dx.l, dt, prob->at_pack_dev, rp, static_cast<uint64_t>(info->n_slots) * K, rp * es, rp, 128);
    if (do_gx) ok = ok && make_map(&dx.o, dt, grad_x_dev, K, T, K * es, 64, 32);
    if (!ok) return LF_ERR_UNSUPPORTED;
    dx.p = p_g;
    int planes = 1;  // S_b's K-half planes (S_f's: sf_planes when reused, else the same as S_b's)
    bool gemm_done = !do_gx;
    if (lora && staged) {
      dx.s = sb_map;
      if (do_shrink) {
        if (!reuse_sf) {
          e = tc_shrink(dt, p_x, a_map, K, tb, s_f, ds->num_sms, st);
          if (e != cudaSuccess) return LF_ERR_CUDA;
        }
        e = tc_shrink(dt, p_g, bt_map, N, tb, s_b, ds->num_sms, st);
        if (e != cudaSuccess) return LF_ERR_CUDA;
      }
    } else if (lora) {
      dx.s = sb_map;
      // The shrinks inside the dX GEMM launch, on CTA pairs its round count leaves idle: job 1 =
      // S_b (g . B_i, needed by the dX tiles), job 2 = S_f (x . A_i^T, read by the dB gram) unless
      // the forward's is reused.
      const int spare =
          cosched_allowed(ds) && !cosched_prologue() ? pair_spare_pairs(T, K, ds->num_sms, info->n_shrink_units) : 0;
      if (cosched_allowed(ds) && (spare > 0 || cosched_prologue())) {
        PairShrink sh{};
        sh.a_map = bt_map;
        sh.s_ext = s_b;
        sh.unit_ready = reinterpret_cast<uint64_t*>(ws + 2 * sb);
        sh.gen = next_generation();
        sh.wait_gen = wait_generation(sh.gen);
        sh.n_pairs = spare;
        sh.prologue = cosched_prologue();
        sh.job2 = !reuse_sf;
        sh.p2_map = p_x;
        sh.a2_map = a_map;
        sh.s_ext2 = s_f;
        sh.K2 = K;
        e = tc_gemm_pair(dt, true, dx, T, K, N, lora, tb, grad_x_dev, K, ds->num_sms, st, &sh, &tail);
        if (e == cudaSuccess) {
          planes = 2;
          gemm_done = true;
        } else {
          refuse_cosched(ds, e);  // cooperative launch refused: nothing ran
        }
      }
      if (!gemm_done) {
        if (!reuse_sf) {
          e = tc_shrink(dt, p_x, a_map, K, tb, s_f, ds->num_sms, st);
          if (e != cudaSuccess) return LF_ERR_CUDA;
        }
        e = tc_shrink(dt, p_g, bt_map, N, tb, s_b, ds->num_sms, st);
        if (e != cudaSuccess) return LF_ERR_CUDA;
      }
    } else {
      dx.s = dx.l = p_g;
    }
    if (!gemm_done) {
      e = tc_gemm_pair(dt, true, dx, T, K, N, lora, tb, grad_x_dev, K, ds->num_sms, st, nullptr,
                       cosched_allowed(ds) ? &tail : nullptr);
      if (e != cudaSuccess && cosched_allowed(ds)) {  // cooperative launch refused: nothing ran
        refuse_cosched(ds, e);
        e = tc_gemm_pair(dt, true, dx, T, K, N, lora, tb, grad_x_dev, K, ds->num_sms, st);
      }
      if (e != cudaSuccess) return LF_ERR_CUDA;
    }
    if (lora && do_gab) {  // dB and dA in one launch
      GramJobDesc jobs[2];
      jobs[0].d_map = p_g;
      jobs[0].s_map = sf_map;
      jobs[0].C = N;
      jobs[0].out = grad_b_dev;
      jobs[0].transpose_out = 0;
      jobs[0].out_f32 = grad_f32;
      jobs[1].d_map = p_x;
      jobs[1].s_map = sb_map;
      jobs[1].C = K;
      jobs[1].out = grad_a_dev;
      jobs[1].transpose_out = 1;
      jobs[1].out_f32 = grad_f32;
      void* scratch = ws + 2 * sb + flag_bytes(info, 2);
      // the grams read hi and lo planes: 2 per K half
      const int f_planes = reuse_sf ? sf_planes : planes;
      if (f_planes == planes) {
        e = tc_gram(dt, jobs, 2, tb, ds->num_sms, st, 2 * planes, scratch, next_generation(), gpp);
      } else {  // S_f and S_b hold different plane counts: one launch each
        e = tc_gram(dt, &jobs[0], 1, tb, ds->num_sms, st, 2 * f_planes, scratch, next_generation(), gpp);
        if (e == cudaSuccess)
          e = tc_gram(dt, &jobs[1], 1, tb, ds->num_sms, st, 2 * planes, scratch, next_generation(), gpp);
      }
      if (e != cudaSuccess) return LF_ERR_CUDA;
    }
    return LF_OK;
  }

  double* sf = reinterpret_cast<double*>(ws);  // the CUDA-core path computes its own f64 S_f
  double* sbp = static_cast<double*>(s_b);
  if (do_shrink) {
    e = simt_shrink(dt, prob->x_dev, K, K, prob->a_pack_dev, tb, sf, st);
    if (e != cudaSuccess) return LF_ERR_CUDA;
    e = simt_shrink(dt, grad_out_dev, N, N, prob->bt_pack_dev, tb, sbp, st);
    if (e != cudaSuccess) return LF_ERR_CUDA;
  }
  if (do_gx) {  // grad_x = g W + S_b . A   (Q(c, m) = W[m][c])
    e = simt_gemm(dt, grad_out_dev, N, prob->w_dev, 1, K, T, K, N, sbp, prob->at_pack_dev, tb, grad_x_dev, K, st);
    if (e != cudaSuccess) return LF_ERR_CUDA;
  }
  if (do_gab) {
    e = simt_gram(dt, grad_out_dev, N, N, sf, tb, grad_b_dev, 0, grad_f32, st);
    if (e != cudaSuccess) return LF_ERR_CUDA;
    e = simt_gram(dt, prob->x_dev, K, K, sbp, tb, grad_a_dev, 1, grad_f32, st);
  }
  return to_status(e);
}
}  // namespace

extern "C" int lf_backward(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                           const void* grad_out_dev, void* grad_x_dev, void* grad_a_dev, void* grad_b_dev,
                           void* workspace_dev, size_t workspace_bytes, lf_stream_t stream) {
  return backward_impl(prob, info, table_dev, grad_out_dev, nullptr, 0, 0, grad_x_dev, grad_a_dev, grad_b_dev,
                       workspace_dev, workspace_bytes, stream);
}

extern "C" int lf_backward_sf(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                              const void* grad_out_dev, const void* s_f_dev, int32_t s_f_planes, void* grad_x_dev,
                              void* grad_a_dev, void* grad_b_dev, void* workspace_dev, size_t workspace_bytes,
                              lf_stream_t stream) {
  if (!s_f_dev || (s_f_planes != 1 && s_f_planes != 2)) return LF_ERR_INVALID_ARG;
  return backward_impl(prob, info, table_dev, grad_out_dev, s_f_dev, s_f_planes, 0, grad_x_dev, grad_a_dev,
                       grad_b_dev, workspace_dev, workspace_bytes, stream);
}

extern "C" int lf_backward_stages(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                                  const void* grad_out_dev, const void* s_f_dev, int32_t s_f_planes,
                                  int32_t grad_ab_dtype, void* grad_x_dev, void* grad_a_dev, void* grad_b_dev,
                                  void* workspace_dev, size_t workspace_bytes, int32_t stages, lf_stream_t stream) {
  if (!prob) return LF_ERR_INVALID_ARG;
  if (stages <= 0 || stages > (LF_BSTAGE_SHRINK | LF_BSTAGE_GRAD_X | LF_BSTAGE_GRAD_AB)) return LF_ERR_INVALID_ARG;
  if (s_f_dev && s_f_planes != 1 && s_f_planes != 2) return LF_ERR_INVALID_ARG;
  if (grad_ab_dtype != prob->dtype && grad_ab_dtype != LF_F32) return LF_ERR_INVALID_ARG;
  return backward_impl(prob, info, table_dev, grad_out_dev, s_f_dev, s_f_dev ? s_f_planes : 0,
                       grad_ab_dtype == LF_F32 ? 1 : 0, grad_x_dev, grad_a_dev, grad_b_dev, workspace_dev,
                       workspace_bytes, stream, stages);
}

extern "C" int lf_backward_ex(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                              const void* grad_out_dev, const void* s_f_dev, int32_t s_f_planes, int32_t grad_ab_dtype,
                              void* grad_x_dev, void* grad_a_dev, void* grad_b_dev, void* workspace_dev,
                              size_t workspace_bytes, lf_stream_t stream) {
  if (!prob) return LF_ERR_INVALID_ARG;
  if (s_f_dev && s_f_planes != 1 && s_f_planes != 2) return LF_ERR_INVALID_ARG;
  if (grad_ab_dtype != prob->dtype && grad_ab_dtype != LF_F32) return LF_ERR_INVALID_ARG;
  return backward_impl(prob, info, table_dev, grad_out_dev, s_f_dev, s_f_dev ? s_f_planes : 0,
                       grad_ab_dtype == LF_F32 ? 1 : 0, grad_x_dev, grad_a_dev, grad_b_dev, workspace_dev,
                       workspace_bytes, stream);
}

extern "C" int lf_backward_peer(const lf_problem* prob, const lf_plan_info* info, const int32_t* table_dev,
                                const void* grad_out_dev, const void* s_f_dev, int32_t s_f_planes,
                                int32_t grad_ab_dtype, void* grad_x_dev, void* grad_a_dev, void* grad_b_dev,
                                void* workspace_dev, size_t workspace_bytes, const lf_peer_reduce* peer,
                                lf_stream_t stream) {
  if (!prob || !peer) return LF_ERR_INVALID_ARG;
  if (s_f_dev && s_f_planes != 1 && s_f_planes != 2) return LF_ERR_INVALID_ARG;
  if (grad_ab_dtype != prob->dtype && grad_ab_dtype != LF_F32) return LF_ERR_INVALID_ARG;
  return backward_impl(prob, info, table_dev, grad_out_dev, s_f_dev, s_f_dev ? s_f_planes : 0,
                       grad_ab_dtype == LF_F32 ? 1 : 0, grad_x_dev, grad_a_dev, grad_b_dev, workspace_dev,
                       workspace_bytes, stream, 0, peer);
}

extern "C" size_t lf_peer_exchange_bytes(int32_t world, int32_t n_blocks, int32_t r_pad) {
  if (world < 1 || world > LF_MAX_PEERS || n_blocks < 0 || (r_pad != 16 && r_pad != 32 && r_pad != 64)) return 0;
  return 2 * peer_half_bytes(world, n_blocks, r_pad);
}

extern "C" int lf_peer_alloc(size_t bytes, void** dev_ptr) {
  if (!dev_ptr || bytes == 0) return LF_ERR_INVALID_ARG;
  *dev_ptr = nullptr;
  if (cudaMalloc(dev_ptr, bytes) != cudaSuccess) return LF_ERR_CUDA;
  if (cudaMemset(*dev_ptr, 0, bytes) != cudaSuccess) return LF_ERR_CUDA;  // flags start below any generation
  return LF_OK;
}

extern "C" int lf_peer_free(void* dev_ptr) { return cudaFree(dev_ptr) == cudaSuccess ? LF_OK : LF_ERR_CUDA; }

extern "C" int lf_ipc_handle(const void* dev_ptr, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == LF_IPC_HANDLE_BYTES, "IPC handle size");
  if (!dev_ptr || !handle) return LF_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)) != cudaSuccess) return LF_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return LF_OK;
}

extern "C" int lf_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return LF_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *dev_ptr = nullptr;
  return cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? LF_OK : LF_ERR_CUDA;
}

extern "C" int lf_ipc_close(void* dev_ptr) {
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? LF_OK : LF_ERR_CUDA;
}

extern "C" int lf_device_error(int32_t* code) {
  if (!code) return LF_ERR_INVALID_ARG;
  DeviceState* ds = nullptr;
  if (device_state(&ds) != cudaSuccess) return LF_ERR_CUDA;
  if (cudaDeviceSynchronize() != cudaSuccess) return LF_ERR_CUDA;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_ctl, sizeof(int), offsetof(DeviceCtl, status)) != cudaSuccess)
    return LF_ERR_CUDA;
  const int zero = 0;
  if (cudaMemcpyToSymbol(g_device_ctl, &zero, sizeof(int), offsetof(DeviceCtl, status)) != cudaSuccess)
    return LF_ERR_CUDA;
  *code = v;
  return LF_OK;
}

extern "C" const char* lf_status_string(int status) {
  switch (status) {
    case LF_OK:
      return "ok";
    case LF_ERR_INVALID_ARG:
      return "invalid argument";
    case LF_ERR_ROUTING:
      return "routes do not tile the fused rows";
    case LF_ERR_UNSUPPORTED:
      return "unsupported dtype, rank or alignment";
    case LF_ERR_CUDA:
      return "CUDA call failed";
    case LF_ERR_CAPACITY:
      return "buffer too small";
    case LF_ERR_DEVICE:
      return "a kernel gave up waiting (device timeout)";
    default:
      return "unknown status";
  }
}

extern "C" const char* lf_version(void) { return "lorafusion_b200 0.1.0 sm_100a"; }
