// C ABI of liblp_b200.so (declared in include/lp_logprob.h): argument checks, tensor-map
// construction, tile planning and kernel launches. No torch or Python types cross it.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/lp_logprob.h"
#include "lp_gemm.cuh"
#include "lp_plan.cuh"
#include "lp_small_kernels.cuh"

namespace {

using namespace lpk;

thread_local std::string g_last_error;
std::atomic<long long> g_launches{0};

// Optional per-kernel timing: CUDA events recorded on the launching stream around every
// kernel this library launches, summed per kernel name by lp_profile_read().
struct ProfRecord {
  const char* tag;
  cudaEvent_t start, stop;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRecord> g_prof_records;
std::vector<cudaEvent_t> g_prof_pool;

cudaEvent_t prof_event() {
  if (!g_prof_pool.empty()) {
    cudaEvent_t e = g_prof_pool.back();
    g_prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

struct ProfScope {
  cudaStream_t st;
  const char* tag;
  cudaEvent_t start = nullptr;
  ProfScope(cudaStream_t s, const char* t) : st(s), tag(t) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (g_prof_on) {
      start = prof_event();
      cudaEventRecord(start, st);
    }
  }
  ~ProfScope() {
    if (start == nullptr) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    cudaEvent_t stop = prof_event();
    cudaEventRecord(stop, st);
    g_prof_records.push_back({tag, start, stop});
  }
};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define LP_CUDA_TRY(expr)                                                                   \
  do {                                                                                      \
    cudaError_t e_ = (expr);                                                                \
    if (e_ != cudaSuccess) return fail(LP_ECUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

#define LP_LAUNCH_CHECK(name)                                                                  \
  do {                                                                                         \
    cudaError_t e_ = cudaGetLastError();                                                       \
    if (e_ != cudaSuccess) return fail(LP_ECUDA, "launch %s: %s", name, cudaGetErrorString(e_)); \
    g_launches.fetch_add(1, std::memory_order_relaxed);                                        \
  } while (0)

constexpr int kMaxDevices = 64;

// Tensor-core CTA group of the GEMMs: 2 = CTA pairs with 256x256 tiles, 1 = single CTAs with
// 128x256 tiles. By default each GEMM uses the group that measured faster for it;
// LP_B200_CTA_GROUP=1|2 or lp_set_cta_group(1|2) forces one group for every GEMM.
// 0 = per-GEMM default (below); 1 / 2 = force every GEMM to that CTA group.
// Optional pipeline counters of the GEMM kernels (a tuning aid): one 8-counter block per CTA
// and per GEMM kind, allocated on the first lp_debug_enable(1) of a device.
constexpr int kDbgKinds = 5;  // fwd, dz, dh, dw, other
std::atomic<bool> g_dbg_on{false};
unsigned long long* g_dbg_buf[kMaxDevices] = {};
int dbg_kind(const char* tag) {
  if (!strcmp(tag, "fwd_lse_gemm")) return 0;
  if (!strcmp(tag, "bwd_dz_gemm")) return 1;
  if (!strcmp(tag, "bwd_dh_gemm")) return 2;
  if (!strcmp(tag, "bwd_dw_gemm")) return 3;
  return 4;
}
unsigned long long* dbg_ptr(const char* tag) {
  if (!g_dbg_on.load()) return nullptr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices || g_dbg_buf[dev] == nullptr) return nullptr;
  return g_dbg_buf[dev] + (size_t)dbg_kind(tag) * 256 * 8;
}

std::atomic<int> g_cg{-1};

int forced_cta_group() {
  int v = g_cg.load();
  if (v < 0) {
    const char* e = getenv("LP_B200_CTA_GROUP");
    v = (e != nullptr && (e[0] == '1' || e[0] == '2')) ? e[0] - '0' : 0;
    g_cg.store(v);
  }
  return v;
}

// CTA group per GEMM. A pair's 256x256 tile takes a third less operand data from L2 per FLOP
// than two single-CTA 128x256 tiles, and at the 1 kW power cap the energy saved comes back as
// SM clock. With one multicast commit per K block the pair's MMA issue is as fast as a single
// CTA's (forward: 659 vs 652 cycles per K block); a whole config-2 step with every GEMM as
// pairs measured fastest, although the dZ recompute alone is ~2 % faster as single CTAs.
// The sampler head (a few decode rows) and the generic GEMM hook use single CTAs.
enum CgUse { CG_FWD, CG_DZ, CG_DH, CG_DW, CG_HOOK, CG_HEAD };
int cta_group_for(CgUse k) {
  const int f = forced_cta_group();
  if (f) return f;
  // tuning: LP_B200_CG_PER_GEMM="fzhw" (four digits 1 / 2: forward, dZ, dH, dW)
  static const char* per = getenv("LP_B200_CG_PER_GEMM");
  if (per != nullptr && k < CG_HOOK && (int)strlen(per) >= 4 && (per[k] == '1' || per[k] == '2')) return per[k] - '0';
  return (k == CG_HOOK || k == CG_HEAD) ? 1 : 2;
}
int cta_group() { return forced_cta_group(); }

// The dW GEMM's K is the chunk's token count. With few tokens (e.g. T = 256) each tile is a
// few K blocks and the pair's cross-SM hand-offs (both CTAs' loads, both epilogues) are not
// amortised: single CTAs measured faster there (T = 256: 0.35 vs 0.43 ms, the bf16 dW stores
// at 0.86 of the write-only HBM bandwidth), pairs faster at thousands of tokens.
int cta_group_dw(int64_t k_tokens) {
  const int cg = cta_group_for(CG_DW);
  if (forced_cta_group() != 0 || getenv("LP_B200_CG_PER_GEMM") != nullptr) return cg;
  return k_tokens <= 1024 ? 1 : cg;
}

struct DeviceInfo {
  int sms = 0;
  int major = 0, minor = 0;
  int pairs = 0;  // CTA pairs of the pair GEMMs that can be resident at once
  bool ready = false;
};

// Persistent workers of a launch: SMs for CG = 1, co-resident CTA pairs for CG = 2.
// LP_B200_MAX_CTAS caps the CTAs of a GEMM launch (a tuning aid: fewer SMs share L2 / HBM).
int workers(const DeviceInfo* di, int cg) {
  static const int cap = [] {
    const char* e = getenv("LP_B200_MAX_CTAS");
    return (e != nullptr && atoi(e) > 0) ? atoi(e) : 0;
  }();
  const int w = cg == 1 ? di->sms : di->pairs;
  return cap > 0 ? std::max(1, std::min(w, cap / cg)) : w;
}
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

// How many 2-CTA clusters of the largest pair GEMM (most shared memory) fit on the GPU at
// once; the persistent pair kernels launch at most this many pairs.
int max_resident_pairs(int sms, int* pairs) {
  auto kern = tc_gemm_kernel<2, EPI_BWD_DZ, false, false, true>;
  constexpr int smem = gemm_smem_bytes<2, EPI_BWD_DZ>();
  LP_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms, 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  LP_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
  *pairs = std::max(1, std::min(n, sms / 2));
  return LP_OK;
}

// Host-visible device error codes: one int per device in mapped, pinned host memory, which
// kernels write (besides g_lp_device_error) when they record an error. Reading a slot is a
// plain host load, so callers can check for errors at points where they already wait for
// the GPU without another synchronisation.
int* g_host_errors = nullptr;  // [kMaxDevices], allocated on the first device set-up

int setup_host_error_mirror(int dev) {
  if (g_host_errors == nullptr) {
    void* p = nullptr;
    LP_CUDA_TRY(cudaHostAlloc(&p, kMaxDevices * sizeof(int), cudaHostAllocMapped | cudaHostAllocPortable));
    std::memset(p, 0, kMaxDevices * sizeof(int));
    g_host_errors = static_cast<int*>(p);
  }
  int* dptr = nullptr;
  LP_CUDA_TRY(cudaHostGetDevicePointer(reinterpret_cast<void**>(&dptr), g_host_errors + dev, 0));
  LP_CUDA_TRY(cudaMemcpyToSymbol(g_lp_host_error, &dptr, sizeof(dptr)));
  return LP_OK;
}

int current_device_info(DeviceInfo** out) {
  int dev = 0;
  LP_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(LP_EINVAL, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    LP_CUDA_TRY(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    LP_CUDA_TRY(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev));
    LP_CUDA_TRY(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev));
    d.pairs = d.sms / 2;
    if (d.major == 10 && d.minor == 0) {
      int rc = max_resident_pairs(d.sms, &d.pairs);
      if (rc) return rc;
      if ((rc = setup_host_error_mirror(dev))) return rc;
    }
    d.ready = true;
  }
  if (d.major != 10 || d.minor != 0)
    return fail(LP_EUNSUPPORTED, "liblp_b200 needs an sm_100 (B200) device, device %d is sm_%d%d", dev, d.major,
                d.minor);
  *out = &d;
  return LP_OK;
}

// --------------------------------------------------------------------------- tensor maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D tiled map, 128-byte swizzle, zero fill out of bounds. `inner`/`outer` in elements,
// `row_bytes` = byte stride between outer rows.
int make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize, uint64_t inner, uint64_t outer,
             uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, const char* what,
             CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(LP_ECUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  if (inner == 0 || outer == 0) return fail(LP_EINVAL, "%s: empty tensor", what);
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return fail(LP_EINVAL, "%s: base pointer not 16-byte aligned", what);
  if (row_bytes % 16 != 0) return fail(LP_EINVAL, "%s: row stride %llu bytes not a multiple of 16", what,
                                       (unsigned long long)row_bytes);
  if (row_bytes < inner * (uint64_t)esize) return fail(LP_EINVAL, "%s: row stride smaller than a row", what);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LP_ECUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)r);
  return LP_OK;
}

int map_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_elems, uint32_t bi,
             uint32_t bo, const char* what) {
  return make_map(m, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, inner, outer, ld_elems * 2, bi, bo, what);
}

// MN-major bf16 operand [k_extent rows][mn_extent columns] (row stride ld_elems) as a 3-D
// map: dims (64 columns, K rows, mn_extent / 64 column chunks), box (64, 64, chunks), 128-byte
// swizzle. One box lands in shared memory as `chunks` consecutive 8 KB [64 K rows x 128 B]
// blocks, the layout of `chunks` 2-D 64x64 boxes side by side. Only for mn_extent % 64 == 0,
// so the box never reaches past the tensor.
int map_mn3d(CUtensorMap* m, const void* base, uint64_t mn_extent, uint64_t k_extent, uint64_t ld_elems,
             uint32_t chunks, const char* what) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(LP_ECUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  if (mn_extent % 64 != 0 || k_extent == 0) return fail(LP_EINVAL, "%s: 3-D map needs 64-column chunks", what);
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return fail(LP_EINVAL, "%s: base pointer not 16-byte aligned", what);
  if ((ld_elems * 2) % 16 != 0 || ld_elems < mn_extent) return fail(LP_EINVAL, "%s: bad row stride", what);
  cuuint64_t dims[3] = {64, k_extent, mn_extent / 64};
  cuuint64_t strides[2] = {ld_elems * 2, 128};
  cuuint32_t box[3] = {64, 64, chunks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LP_ECUDA, "%s: cuTensorMapEncodeTiled (3-D) failed (%d)", what, (int)r);
  return LP_OK;
}

// 3-D MN-major operand maps (LP_B200_MN3D=0 keeps the per-chunk 2-D boxes, for tuning).
bool mn3d_enabled() {
  static const bool on = [] {
    const char* e = getenv("LP_B200_MN3D");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

// Epilogue store targets: one 32-row box per warp and piece, rows of `box_row_bytes` (64 or
// 128, the store_row_bytes of the GEMM) with the swizzle of that width, matching the staging
// layout of the GEMM epilogue.
int map_store_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                   const char* what, int box_row_bytes = 64) {
  return make_map(m, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, inner, outer, ld_elems * 2, box_row_bytes / 2, 32,
                  what, box_row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}
int map_store_f32(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                  const char* what, int box_row_bytes = 64) {
  return make_map(m, base, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, inner, outer, ld_elems * 4, box_row_bytes / 4, 32,
                  what, box_row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

// store_row_bytes of the plain-store GEMM (EPI_STORE) at CTA group cg.
int store_box_bytes(int cg) { return cg == 2 ? store_row_bytes<2, EPI_STORE>() : store_row_bytes<1, EPI_STORE>(); }

// Planning (tile plans, split-K, backward token chunks, workspace layout): lp_plan.cuh.

// --------------------------------------------------------------------------- launches
}  // namespace

// Work-unit counters of the GEMM kernels (each launch claims its units with atomicAdd on
// one slot). Slots rotate so that launches in flight on different streams use different
// counters; a launch zeroes its slot on its own stream just before it starts.
constexpr int kSchedSlots = 4096;
static __device__ unsigned int g_lp_sched[kSchedSlots];

namespace {

unsigned int* g_sched_ptr[kMaxDevices] = {};
std::mutex g_sched_mu;
std::atomic<unsigned> g_sched_next{0};

int sched_slot(cudaStream_t st, unsigned int** out) {
  int dev = 0;
  LP_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(LP_EINVAL, "device ordinal %d out of range", dev);
  unsigned int* base;
  {
    std::lock_guard<std::mutex> lk(g_sched_mu);
    if (g_sched_ptr[dev] == nullptr) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_lp_sched);
      if (e != cudaSuccess || p == nullptr)
        return fail(LP_ECUDA, "cudaGetSymbolAddress(work counters) on device %d: %s", dev, cudaGetErrorString(e));
      g_sched_ptr[dev] = static_cast<unsigned int*>(p);
    }
    base = g_sched_ptr[dev];
  }
  unsigned int* slot = base + g_sched_next.fetch_add(1u) % kSchedSlots;
  LP_CUDA_TRY(cudaMemsetAsync(slot, 0, sizeof(unsigned int), st));
  *out = slot;
  return LP_OK;
}

template <int CG, int EPI, bool A_MN, bool B_MN, bool CAP>
int launch_gemm_cg(cudaStream_t st, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& o,
                   const GemmParams& p, const DeviceInfo* di, const char* tag) {
  auto kern = tc_gemm_kernel<CG, EPI, A_MN, B_MN, CAP>;
  constexpr int smem = gemm_smem_bytes<CG, EPI>();
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  LP_CUDA_TRY(cudaGetDevice(&dev));
  if (!configured[dev]) {
    LP_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if (CG == 2) LP_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0));
    configured[dev] = true;
  }
  const int grid = CG * std::max(1, std::min(p.s.num_units, workers(di, CG)));
  GemmParams pp = p;
  pp.dbg = dbg_ptr(tag);
  if (int rc = sched_slot(st, &pp.sched)) return rc;
  ProfScope prof(st, tag);
  if constexpr (CG == 1) {
    kern<<<grid, NUM_THREADS, smem, st>>>(a, b, o, pp);
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    LP_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a, b, o, pp));
  }
  LP_LAUNCH_CHECK("tc_gemm_kernel");
  return LP_OK;
}

template <int EPI, bool A_MN, bool B_MN, bool CAP>
int launch_gemm(cudaStream_t st, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& o,
                const GemmParams& p, const DeviceInfo* di, const char* tag) {
  return p.s.bm == 256 ? launch_gemm_cg<2, EPI, A_MN, B_MN, CAP>(st, a, b, o, p, di, tag)
                       : launch_gemm_cg<1, EPI, A_MN, B_MN, CAP>(st, a, b, o, p, di, tag);
}

template <int EPI, bool A_MN, bool B_MN>
int launch_gemm_cap(bool cap, cudaStream_t st, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& o,
                    const GemmParams& p, const DeviceInfo* di, const char* tag) {
  return cap ? launch_gemm<EPI, A_MN, B_MN, true>(st, a, b, o, p, di, tag)
             : launch_gemm<EPI, A_MN, B_MN, false>(st, a, b, o, p, di, tag);
}

// L2 eviction priorities of the A / B loads of each GEMM (0 normal = plain load,
// 1 evict_first, 2 evict_last). Measured (ncu DRAM bytes per launch at the config-2 size):
// plain loads keep the forward and the dZ recompute near their algorithmic traffic;
// evict_first on an operand that concurrent CTAs share (W) multiplies HBM reads, and an
// explicit evict_normal policy is not the same as no hint. With the dynamic scheduler the
// dW GEMM is also faster with plain loads than with evict_last on its H chunk (715 vs 734
// cycles per K block, pipeline counters). LP_B200_L2HINTS="fA fB zA zB hA hB wA wB"
// (8 digits: forward, dZ recompute, dH, dW) overrides them for tuning.
enum GemmKind { G_FWD = 0, G_DZ = 1, G_DH = 2, G_DW = 3 };
int l2_hint(GemmKind k, int operand) {
  static int table[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  static std::once_flag once;
  std::call_once(once, [] {
    const char* e = getenv("LP_B200_L2HINTS");
    if (e == nullptr) return;
    int i = 0;
    for (const char* c = e; *c && i < 8; ++c)
      if (*c >= '0' && *c <= '2') table[i++] = *c - '0';
  });
  return table[2 * (int)k + operand];
}

void set_hints(GemmParams& p, GemmKind k) {
  p.e.a_l2 = l2_hint(k, 0);
  p.e.b_l2 = l2_hint(k, 1);
}

// Box height of a K-major B operand: the rows of B one CTA stages.
uint32_t b_box_rows(int cg) { return (uint32_t)(BN / cg); }

int check_common(const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs, const int32_t* y) {
  if (T < 0 || d <= 0 || Vs <= 0) return fail(LP_EINVAL, "bad sizes T=%lld d=%lld Vs=%lld", (long long)T, (long long)d,
                                               (long long)Vs);
  if (T > (int64_t)1 << 30 || Vs > (int64_t)1 << 30) return fail(LP_EINVAL, "T or Vs above 2^30");
  if (d % 8 != 0) return fail(LP_EINVAL, "hidden size d=%lld must be a multiple of 8", (long long)d);
  if (ldh < d || ldh % 8 != 0) return fail(LP_EINVAL, "ldh=%lld must be >= d and a multiple of 8", (long long)ldh);
  if (T > 0 && (H == nullptr || y == nullptr)) return fail(LP_EINVAL, "null hidden or targets");
  if (W == nullptr) return fail(LP_EINVAL, "null embedding");
  return LP_OK;
}

// Few rows for many partials: the forward's finalize runs one block per row instead of one
// thread per row (fewer rows than fill the GPU with 256-row blocks).
bool few_rows(int64_t T, const DeviceInfo* di) { return cdiv(T, 256) < di->sms; }

}  // namespace

// ============================================================================= C ABI
extern "C" {

int lp_version(void) { return 100; }

const char* lp_last_error(void) { return g_last_error.c_str(); }

long long lp_launch_count(void) { return g_launches.load(); }

int lp_debug_enable(int on) {
  int dev = 0;
  LP_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(LP_EINVAL, "device ordinal out of range");
  if (on && g_dbg_buf[dev] == nullptr) {
    LP_CUDA_TRY(cudaMalloc(&g_dbg_buf[dev], (size_t)kDbgKinds * 256 * 8 * sizeof(unsigned long long)));
  }
  if (g_dbg_buf[dev] != nullptr)
    LP_CUDA_TRY(cudaMemset(g_dbg_buf[dev], 0, (size_t)kDbgKinds * 256 * 8 * sizeof(unsigned long long)));
  g_dbg_on.store(on != 0);
  return LP_OK;
}

int lp_debug_read(unsigned long long* out) {
  int dev = 0;
  LP_CUDA_TRY(cudaGetDevice(&dev));
  if (out == nullptr) return fail(LP_EINVAL, "null out");
  if (dev < 0 || dev >= kMaxDevices || g_dbg_buf[dev] == nullptr) return fail(LP_EINVAL, "debug counters not enabled");
  std::vector<unsigned long long> h((size_t)kDbgKinds * 256 * 8);
  LP_CUDA_TRY(cudaMemcpy(h.data(), g_dbg_buf[dev], h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
  for (int k = 0; k < kDbgKinds; ++k)
    for (int i = 0; i < 8; ++i) {
      unsigned long long t = 0;
      for (int c = 0; c < 256; ++c) t += h[((size_t)k * 256 + c) * 8 + i];
      out[k * 8 + i] = t;
    }
  return LP_OK;
}

int lp_device_pairs(void) {
  DeviceInfo* di = nullptr;
  return current_device_info(&di) == LP_OK ? di->pairs : -1;
}

int lp_set_cta_group(int cg) {
  if (cg != 0 && cg != 1 && cg != 2) return fail(LP_EINVAL, "cta group must be 0, 1 or 2, got %d", cg);
  g_cg.store(cg);
  return LP_OK;
}

int lp_get_cta_group(void) { return cta_group(); }

int lp_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (auto& r : g_prof_records) {
    g_prof_pool.push_back(r.start);
    g_prof_pool.push_back(r.stop);
  }
  g_prof_records.clear();
  g_prof_on = on != 0;
  return LP_OK;
}

int lp_profile_read(int max_tags, char* names, double* total_ms, long long* launches, int* n_tags) {
  if (max_tags <= 0 || names == nullptr || total_ms == nullptr || launches == nullptr || n_tags == nullptr)
    return fail(LP_EINVAL, "bad lp_profile_read arguments");
  std::lock_guard<std::mutex> lk(g_prof_mu);
  int n = 0;
  std::vector<std::string> tags;
  for (auto& r : g_prof_records) {
    LP_CUDA_TRY(cudaEventSynchronize(r.stop));
    float ms = 0.f;
    LP_CUDA_TRY(cudaEventElapsedTime(&ms, r.start, r.stop));
    int k = 0;
    while (k < n && tags[k] != r.tag) ++k;
    if (k == n) {
      if (n == max_tags) continue;
      tags.push_back(r.tag);
      total_ms[n] = 0.0;
      launches[n] = 0;
      ++n;
    }
    total_ms[k] += ms;
    launches[k] += 1;
  }
  for (int k = 0; k < n; ++k) {
    std::strncpy(names + 32 * k, tags[k].c_str(), 31);
    names[32 * k + 31] = 0;
  }
  *n_tags = n;
  return LP_OK;
}

int lp_device_error(int device, int* code) {
  int prev = 0;
  LP_CUDA_TRY(cudaGetDevice(&prev));
  LP_CUDA_TRY(cudaSetDevice(device));
  int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_lp_device_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_lp_device_error, &zero, sizeof(int));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(LP_ECUDA, "lp_device_error: %s", cudaGetErrorString(e));
  if (g_host_errors != nullptr && device >= 0 && device < kMaxDevices) {
    if (v == 0) v = reinterpret_cast<volatile int*>(g_host_errors)[device];
    reinterpret_cast<volatile int*>(g_host_errors)[device] = 0;
  }
  if (code) *code = v;
  return LP_OK;
}

int lp_device_error_poll(int device) {
  if (device < 0 || device >= kMaxDevices || g_host_errors == nullptr) return 0;
  return reinterpret_cast<volatile int*>(g_host_errors)[device];
}

size_t lp_fwd_workspace_bytes(int64_t T, int64_t Vs) {
  DeviceInfo* di = nullptr;
  int sms = 148;
  if (current_device_info(&di) == LP_OK) sms = di->sms;
  if (T <= 0 || Vs <= 0) return 256;
  const int cg = cta_group_for(CG_FWD);
  GemmSched s = plan_fwd(T, Vs, 64, di != nullptr ? workers(di, cg) : (cg == 1 ? sms : sms / 2), 128 * cg);
  // partials, target logits, and the [3, T] triples lp_fwd_sum merges first when T is small
  return align_up((size_t)2 * s.n_groups * T * sizeof(float2), 256) + align_up((size_t)T * 4, 256) +
         align_up((size_t)T * 12, 256);
}

int lp_fwd(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs, int64_t v_off,
           const int32_t* y, float softcap, float* stats, float* logp, void* workspace, size_t workspace_bytes) {
  int rc = check_common(H, T, d, ldh, W, Vs, y);
  if (rc) return rc;
  if (T == 0) return LP_OK;
  if (stats == nullptr) return fail(LP_EINVAL, "null stats");
  DeviceInfo* di = nullptr;
  if ((rc = current_device_info(&di))) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int cg = cta_group_for(CG_FWD);
  GemmSched s = plan_fwd(T, Vs, d, workers(di, cg), 128 * cg);
  const size_t part_bytes = align_up((size_t)2 * s.n_groups * T * sizeof(float2), 256);
  const size_t need = part_bytes + align_up((size_t)T * 4, 256);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(LP_EWORKSPACE, "lp_fwd needs %zu workspace bytes, got %zu", need, workspace_bytes);
  float2* part = reinterpret_cast<float2*>(workspace);
  float* tgt = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + part_bytes);

  alignas(64) CUtensorMap ta, tb;
  if ((rc = map_bf16(&ta, H, d, T, ldh, BK, 128, "hidden"))) return rc;
  if ((rc = map_bf16(&tb, W, d, Vs, d, BK, b_box_rows(cg), "embedding"))) return rc;
  GemmParams p{};
  p.s = s;
  p.e.y = y;
  p.e.v_off = v_off;
  p.e.softcap = softcap;
  p.e.part = part;
  p.e.tgt = tgt;
  set_hints(p, G_FWD);
  if ((rc = launch_gemm_cap<EPI_FWD_LSE, false, false>(softcap > 0.f, st, ta, tb, ta, p, di, "fwd_lse_gemm"))) return rc;
  ProfScope prof(st, "fwd_finalize");
  if (few_rows(T, di)) {
    fwd_finalize_rows_kernel<<<(unsigned)T, 128, 0, st>>>(part, 2 * s.n_groups, (int)T, tgt, y, v_off, Vs, stats, logp);
    LP_LAUNCH_CHECK("fwd_finalize_rows_kernel");
  } else {
    fwd_finalize_kernel<<<(unsigned)cdiv(T, 256), 256, 0, st>>>(part, 2 * s.n_groups, (int)T, tgt, y, v_off, Vs, stats,
                                                                logp);
    LP_LAUNCH_CHECK("fwd_finalize_kernel");
  }
  return LP_OK;
}

int lp_fwd_sum(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs,
               int64_t v_off, const int32_t* y, float softcap, void* exchange, void* exchange_multicast,
               int64_t ld_exchange, unsigned* counter, unsigned* counter_multicast, unsigned* arrivals,
               unsigned epoch, int rank, int world, int timeout_ms, float* logp, float* norm, void* workspace,
               size_t workspace_bytes) {
  int rc = check_common(H, T, d, ldh, W, Vs, y);
  if (rc) return rc;
  if (world < 1 || rank < 0 || rank >= world) return fail(LP_EINVAL, "bad rank %d / world %d", rank, world);
  if (exchange == nullptr || exchange_multicast == nullptr || counter == nullptr || counter_multicast == nullptr ||
      arrivals == nullptr)
    return fail(LP_EINVAL, "null exchange buffer, counter or arrival counter");
  if (((reinterpret_cast<uintptr_t>(exchange) | reinterpret_cast<uintptr_t>(exchange_multicast)) & 15) != 0)
    return fail(LP_EINVAL, "the exchange buffer and its multicast address must be 16-byte aligned");
  if (ld_exchange < T) return fail(LP_EINVAL, "ld_exchange=%lld < T=%lld", (long long)ld_exchange, (long long)T);
  if (epoch == 0 || (unsigned long long)epoch * (unsigned)world > 0xffffffffull)
    return fail(LP_EINVAL, "epoch %u out of range for world %d", epoch, world);
  if (timeout_ms <= 0) return fail(LP_EINVAL, "timeout_ms must be positive");
  if (T == 0) return LP_OK;
  if (logp == nullptr && norm == nullptr) return fail(LP_EINVAL, "null logp and norm");
  DeviceInfo* di = nullptr;
  if ((rc = current_device_info(&di))) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int cg = cta_group_for(CG_FWD);
  GemmSched s = plan_fwd(T, Vs, d, workers(di, cg), 128 * cg);
  const size_t part_bytes = align_up((size_t)2 * s.n_groups * T * sizeof(float2), 256);
  const size_t tgt_bytes = align_up((size_t)T * 4, 256);
  const size_t need = part_bytes + tgt_bytes + align_up((size_t)T * 12, 256);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(LP_EWORKSPACE, "lp_fwd_sum needs %zu workspace bytes, got %zu", need, workspace_bytes);
  float2* part = reinterpret_cast<float2*>(workspace);
  float* tgt = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + part_bytes);
  float* pre = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + part_bytes + tgt_bytes);

  alignas(64) CUtensorMap ta, tb;
  if ((rc = map_bf16(&ta, H, d, T, ldh, BK, 128, "hidden"))) return rc;
  if ((rc = map_bf16(&tb, W, d, Vs, d, BK, b_box_rows(cg), "embedding"))) return rc;
  GemmParams p{};
  p.s = s;
  p.e.y = y;
  p.e.v_off = v_off;
  p.e.softcap = softcap;
  p.e.part = part;
  p.e.tgt = tgt;
  set_hints(p, G_FWD);
  if ((rc = launch_gemm_cap<EPI_FWD_LSE, false, false>(softcap > 0.f, st, ta, tb, ta, p, di, "fwd_lse_gemm"))) return rc;
  // one block per SM at most: every block must be resident while the blocks wait for the
  // other ranks
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(T, 256), di->sms);
  ProfScope prof(st, "fwd_finalize_mesh");
  const bool merge_first = few_rows(T, di);
  if (merge_first) {
    fwd_finalize_rows_kernel<<<(unsigned)T, 128, 0, st>>>(part, 2 * s.n_groups, (int)T, tgt, y, v_off, Vs, pre,
                                                          nullptr);
    LP_LAUNCH_CHECK("fwd_finalize_rows_kernel");
  }
  fwd_finalize_mesh_kernel<<<grid, 256, 0, st>>>(
      part, 2 * s.n_groups, (int)T, tgt, y, v_off, Vs, reinterpret_cast<float4*>(exchange_multicast),
      reinterpret_cast<const float4*>(exchange), ld_exchange, counter_multicast, counter, arrivals,
      epoch * (unsigned)world, rank, world, (unsigned long long)timeout_ms * 1000000ull, merge_first ? pre : nullptr,
      logp, norm);
  LP_LAUNCH_CHECK("fwd_finalize_mesh_kernel");
  return LP_OK;
}

}  // extern "C"

namespace {

// Sampler head plan: the forward's chunk-major order with one vocabulary tile per unit, so
// a decode batch (one or two M tiles) still spreads over every SM.
GemmSched plan_head(int64_t B, int64_t V, int64_t d, int bm) {
  GemmSched s = plan_fwd(B, V, d, 0, bm);
  s.n_group = 1;
  s.n_groups = s.tiles_n;
  s.num_units = s.tiles_m * s.n_groups;
  return s;
}

size_t head_part_bytes(const GemmSched& s, int64_t B) { return align_up((size_t)2 * s.n_groups * B * sizeof(float2), 256); }

}  // namespace

extern "C" {

size_t lp_head_workspace_bytes(int64_t B, int64_t V) {
  if (B <= 0 || V <= 0) return 256;
  const int cg = cta_group_for(CG_HEAD);
  return 2 * head_part_bytes(plan_head(B, V, 64, 128 * cg), B);
}

int lp_head(void* stream, const void* H, int64_t B, int64_t d, int64_t ldh, const void* W, int64_t V, float softcap,
            float* logits, int64_t ld_logits, int flags, float* norm, int32_t* argmax, float* argmax_logp,
            void* workspace, size_t workspace_bytes) {
  if (B < 0 || d <= 0 || V <= 0) return fail(LP_EINVAL, "bad sizes B=%lld d=%lld V=%lld", (long long)B, (long long)d,
                                              (long long)V);
  if (B > (int64_t)1 << 30 || V > (int64_t)1 << 30) return fail(LP_EINVAL, "B or V above 2^30");
  if (d % 8 != 0) return fail(LP_EINVAL, "hidden size d=%lld must be a multiple of 8", (long long)d);
  if (ldh < d || ldh % 8 != 0) return fail(LP_EINVAL, "ldh=%lld must be >= d and a multiple of 8", (long long)ldh);
  if (W == nullptr || (B > 0 && H == nullptr)) return fail(LP_EINVAL, "null hidden or embedding");
  if (flags & ~LP_HEAD_LOGPROBS) return fail(LP_EINVAL, "unknown lp_head flags %d", flags);
  if (logits != nullptr) {
    if (ld_logits < V || ld_logits % 4 != 0) return fail(LP_EINVAL, "ld_logits must be >= V and a multiple of 4");
    if ((reinterpret_cast<uintptr_t>(logits) & 15) != 0) return fail(LP_EINVAL, "logits must be 16-byte aligned");
  } else if (flags & LP_HEAD_LOGPROBS) {
    return fail(LP_EINVAL, "LP_HEAD_LOGPROBS needs a logits buffer");
  }
  if ((flags & LP_HEAD_LOGPROBS) && norm == nullptr) return fail(LP_EINVAL, "LP_HEAD_LOGPROBS needs norm");
  if (B == 0) return LP_OK;
  DeviceInfo* di = nullptr;
  int rc = current_device_info(&di);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int cg = cta_group_for(CG_HEAD);
  GemmSched s = plan_head(B, V, d, 128 * cg);
  const size_t pb = head_part_bytes(s, B);
  if (workspace == nullptr || workspace_bytes < 2 * pb)
    return fail(LP_EWORKSPACE, "lp_head needs %zu workspace bytes, got %zu", 2 * pb, workspace_bytes);
  float2* part = reinterpret_cast<float2*>(workspace);
  float2* best = reinterpret_cast<float2*>(reinterpret_cast<char*>(workspace) + pb);

  alignas(64) CUtensorMap ta, tb, to;
  if ((rc = map_bf16(&ta, H, d, B, ldh, BK, 128, "hidden"))) return rc;
  if ((rc = map_bf16(&tb, W, d, V, d, BK, b_box_rows(cg), "embedding"))) return rc;
  if (logits != nullptr) {
    if ((rc = map_store_f32(&to, logits, V, B, ld_logits, "logits store"))) return rc;
  } else {
    to = ta;  // not used: no logits are stored
  }
  GemmParams p{};
  p.s = s;
  p.e.softcap = softcap;
  p.e.part = part;
  p.e.best = best;
  p.e.store_logits = logits != nullptr ? 1 : 0;
  set_hints(p, G_FWD);
  if ((rc = launch_gemm_cap<EPI_HEAD, false, false>(softcap > 0.f, st, ta, tb, to, p, di, "head_gemm"))) return rc;
  {
    ProfScope prof(st, "head_finalize");
    head_finalize_kernel<<<(unsigned)B, 256, 0, st>>>(part, best, 2 * s.n_groups, (int)B, norm, argmax, argmax_logp);
    LP_LAUNCH_CHECK("head_finalize_kernel");
  }
  if (flags & LP_HEAD_LOGPROBS) {
    ProfScope prof(st, "logits_to_logprobs");
    const unsigned gx = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(V / 4 + 1, 256), 64));
    const unsigned gy = (unsigned)std::min<int64_t>(B, 65535);
    logits_to_logprobs_kernel<<<dim3(gx, gy), 256, 0, st>>>(logits, ld_logits, (int)B, V, norm);
    LP_LAUNCH_CHECK("logits_to_logprobs_kernel");
  }
  return LP_OK;
}

int lp_combine(void* stream, const float* shard_stats, int P, int64_t T, float* logp, float* norm) {
  if (P <= 0 || T < 0) return fail(LP_EINVAL, "bad P=%d or T=%lld", P, (long long)T);
  if (T == 0) return LP_OK;
  if (shard_stats == nullptr) return fail(LP_EINVAL, "null shard_stats");
  DeviceInfo* di = nullptr;
  if (int rc = current_device_info(&di)) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ProfScope prof(st, "combine");
  combine_kernel<<<(unsigned)cdiv(T, 256), 256, 0, st>>>(shard_stats, P, (int)T, logp, norm);
  LP_LAUNCH_CHECK("combine_kernel");
  return LP_OK;
}

size_t lp_bwd_workspace_bytes(int64_t T, int64_t d, int64_t Vs, int64_t token_chunk, int flags) {
  DeviceInfo* di = nullptr;
  int sms = 148;
  if (current_device_info(&di) == LP_OK) sms = di->sms;
  if (T <= 0 || Vs <= 0 || d <= 0) return 256;
  const int cg = cta_group_for(CG_DH);  // the split-K partials follow the dH GEMM's tiles
  return bwd_layout(T, d, Vs, token_chunk, flags, di != nullptr ? workers(di, cg) : (cg == 1 ? sms : sms / 2),
                    128 * cg).total +
         256;
}

}  // extern "C"

namespace {

// The dH sum over the vocabulary mesh inside the dH GEMM (lp_bwd_sum).
struct MeshSum {
  void* dh_mc;
  unsigned* cnt_local;
  unsigned* cnt_mc;
  int rank, world;
  unsigned long long limit_ns;
};

int bwd_impl(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs, int64_t v_off,
             const int32_t* y, float softcap, const float* norm, const float* g, void* dH, int64_t ld_dh, void* dW,
             int flags, int64_t token_chunk, void* workspace, size_t workspace_bytes, const MeshSum* ms) {
  int rc = check_common(H, T, d, ldh, W, Vs, y);
  if (rc) return rc;
  const bool want_dh = !(flags & LP_BWD_NO_DH), want_dw = !(flags & LP_BWD_NO_DW);
  const bool dh_f32 = flags & LP_BWD_DH_F32, dw_bf16 = flags & LP_BWD_DW_BF16;
  if (want_dh && (dH == nullptr || ld_dh < d || ld_dh % 8 != 0))
    return fail(LP_EINVAL, "dH must be non-null with ld_dh >= d and ld_dh %% 8 == 0");
  if (want_dw && dW == nullptr) return fail(LP_EINVAL, "null dW");
  if (T > 0 && (norm == nullptr || g == nullptr)) return fail(LP_EINVAL, "null norm or g");
  DeviceInfo* di = nullptr;
  if ((rc = current_device_info(&di))) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (T == 0) {
    // no tokens: dW is zero
    if (want_dw) LP_CUDA_TRY(cudaMemsetAsync(dW, 0, (size_t)Vs * d * (dw_bf16 ? 2 : 4), st));
    return LP_OK;
  }
  const int cg_dz = cta_group_for(CG_DZ), cg_dh = cta_group_for(CG_DH);
  if (ms != nullptr && want_dh) {
    // chunks start on 256-row boundaries (the row-block counters are per 128 rows)
    if (token_chunk <= 0) token_chunk = default_token_chunk(T, Vs, d);
    if (token_chunk < T) token_chunk = std::max<int64_t>(256, token_chunk / 256 * 256);
  }
  const BwdLayout L = bwd_layout(T, d, Vs, token_chunk, flags, workers(di, cg_dh), 128 * cg_dh);
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(LP_EWORKSPACE, "lp_bwd needs %zu workspace bytes, got %zu", L.total, workspace_bytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & 1023) != 0) return fail(LP_EINVAL, "workspace must be 1024-byte aligned");
  char* ws = reinterpret_cast<char*>(workspace);
  __nv_bfloat16* dz = reinterpret_cast<__nv_bfloat16*>(ws + L.dz_off);
  float* part = reinterpret_cast<float*>(ws + L.part_off);
  float* dw_acc = (want_dw && dw_bf16 && L.chunks > 1) ? reinterpret_cast<float*>(ws + L.dwacc_off)
                                                        : reinterpret_cast<float*>(dW);
  const bool cap = softcap > 0.f;
  const __nv_bfloat16* Hb = reinterpret_cast<const __nv_bfloat16*>(H);

  for (int64_t c = 0; c < L.chunks; ++c) {
    const int64_t t0 = c * L.tc;
    const int64_t tcur = std::min<int64_t>(L.tc, T - t0);
    const __nv_bfloat16* Hc = Hb + t0 * ldh;

    // 1) recompute logits tile by tile and write dZ (bf16) for this chunk
    {
      alignas(64) CUtensorMap ta, tb, to;
      if ((rc = map_bf16(&ta, Hc, d, tcur, ldh, BK, 128, "hidden chunk"))) return rc;
      if ((rc = map_bf16(&tb, W, d, Vs, d, BK, b_box_rows(cg_dz), "embedding"))) return rc;
      if ((rc = map_store_bf16(&to, dz, Vs, tcur, L.ldz, "dZ store"))) return rc;
      GemmParams p{};
      p.s = plan_dz(tcur, Vs, d, workers(di, cg_dz), 128 * cg_dz);
      p.e.y = y + t0;
      p.e.v_off = v_off;
      p.e.softcap = softcap;
      p.e.g = g + t0;
      p.e.stats = norm + t0;
      p.e.stats_ld = T;
      set_hints(p, G_DZ);
      if ((rc = launch_gemm_cap<EPI_BWD_DZ, false, false>(cap, st, ta, tb, to, p, di, "bwd_dz_gemm"))) return rc;
    }
    // 2) dH[t0:t0+tcur] = dZ . W
    if (want_dh) {
      alignas(64) CUtensorMap ta, tb, to;
      if ((rc = map_bf16(&ta, dz, Vs, tcur, L.ldz, BK, 128, "dZ as A"))) return rc;
      GemmParams p{};
      p.b_mn3d = mn3d_enabled() && d % 64 == 0;
      if (p.b_mn3d) rc = map_mn3d(&tb, W, d, Vs, d, b_box_rows(cg_dh) / 64, "embedding as MN-major B");
      else rc = map_bf16(&tb, W, d, Vs, d, 64, 64, "embedding as MN-major B");
      if (rc) return rc;
      const int wk = workers(di, cg_dh);
      p.s = plan_gemm(tcur, d, Vs, wk, ms == nullptr, 1, 128 * cg_dh);
      char* dh_c = reinterpret_cast<char*>(dH) + (size_t)t0 * ld_dh * (dh_f32 ? 4 : 2);
      if (ms != nullptr) {
        // partial tiles stored (bf16) into this rank's copy, summed across ranks by the
        // reduce items of the same launch
        if ((rc = map_store_bf16(&to, dh_c, d, tcur, ld_dh, "dH partial store", store_box_bytes(cg_dh)))) return rc;
        p.e.store_mode = STORE_BF16;
        p.e.split_rows = 0;
        p.s.red_lag = std::min(p.s.tiles_m, (int)cdiv(3 * (int64_t)wk, p.s.tiles_n) + 2);
        p.s.num_units = p.s.tiles_m * p.s.tiles_n + p.s.tiles_m;
        p.e.sum_mc = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<char*>(ms->dh_mc) + (size_t)t0 * ld_dh * 2);
        p.e.sum_local = reinterpret_cast<__nv_bfloat16*>(dh_c);
        p.e.sum_ld = ld_dh;
        p.e.cnt_local = ms->cnt_local + t0 / 128;
        p.e.cnt_mc = ms->cnt_mc + t0 / 128;
        p.e.cnt_target = (unsigned)(ms->world * p.s.tiles_n * EPI_WARPS * cg_dh);
        p.e.sum_rank = ms->rank;
        p.e.sum_world = ms->world;
        p.e.peer_limit_ns = ms->limit_ns;
      } else if (p.s.k_splits == 1) {
        if (dh_f32) {
          if ((rc = map_store_f32(&to, dh_c, d, tcur, ld_dh, "dH store", store_box_bytes(cg_dh)))) return rc;
          p.e.store_mode = STORE_F32;
        } else {
          if ((rc = map_store_bf16(&to, dh_c, d, tcur, ld_dh, "dH store", store_box_bytes(cg_dh)))) return rc;
          p.e.store_mode = STORE_BF16;
        }
        p.e.split_rows = 0;
      } else {
        if ((rc = map_store_f32(&to, part, d, (uint64_t)p.s.k_splits * L.mpad, d, "dH partials",
                                store_box_bytes(cg_dh))))
          return rc;
        p.e.store_mode = STORE_F32;
        p.e.split_rows = (int)L.mpad;
      }
      set_hints(p, G_DH);
      if ((rc = launch_gemm<EPI_STORE, false, true, false>(st, ta, tb, to, p, di, "bwd_dh_gemm"))) return rc;
      if (p.s.k_splits > 1) {
        const int64_t total = tcur * (d / 4);
        const unsigned grid = (unsigned)std::min<int64_t>(cdiv(total, 256), (int64_t)di->sms * 8);
        ProfScope prof(st, "splitk_reduce");
        splitk_reduce_kernel<<<grid, 256, 0, st>>>(part, p.s.k_splits, tcur, d, L.mpad, dh_c, ld_dh, dh_f32 ? 0 : 1);
        LP_LAUNCH_CHECK("splitk_reduce_kernel");
      }
    }
    // 3) dW (+)= dZ^T . H_chunk
    if (want_dw) {
      const int cg_dw = cta_group_dw(tcur);
      alignas(64) CUtensorMap ta, tb, to;
      GemmParams p{};
      p.a_mn3d = mn3d_enabled() && Vs % 64 == 0;
      p.b_mn3d = mn3d_enabled() && d % 64 == 0;
      if (p.a_mn3d) rc = map_mn3d(&ta, dz, Vs, tcur, L.ldz, 2, "dZ as MN-major A");
      else rc = map_bf16(&ta, dz, Vs, tcur, L.ldz, 64, 64, "dZ as MN-major A");
      if (rc) return rc;
      if (p.b_mn3d) rc = map_mn3d(&tb, Hc, d, tcur, ldh, b_box_rows(cg_dw) / 64, "hidden as MN-major B");
      else rc = map_bf16(&tb, Hc, d, tcur, ldh, 64, 64, "hidden as MN-major B");
      if (rc) return rc;
      p.s = plan_gemm(Vs, d, tcur, workers(di, cg_dw), false, 1, 128 * cg_dw);
      const bool direct_bf16 = dw_bf16 && L.chunks == 1;
      if (direct_bf16) {
        if ((rc = map_store_bf16(&to, dW, d, Vs, d, "dW store", store_box_bytes(cg_dw)))) return rc;
        p.e.store_mode = STORE_BF16;
      } else {
        if ((rc = map_store_f32(&to, dw_acc, d, Vs, d, "dW store", store_box_bytes(cg_dw)))) return rc;
        p.e.store_mode = c == 0 ? STORE_F32 : STORE_F32_ADD;
      }
      set_hints(p, G_DW);
      if ((rc = launch_gemm<EPI_STORE, true, true, false>(st, ta, tb, to, p, di, "bwd_dw_gemm"))) return rc;
    }
  }
  if (want_dw && dw_bf16 && L.chunks > 1) {
    const int64_t n = Vs * d;
    const unsigned grid = (unsigned)std::min<int64_t>(cdiv(n / 4 + 1, 256), (int64_t)di->sms * 8);
    ProfScope prof(st, "f32_to_bf16");
    f32_to_bf16_kernel<<<grid, 256, 0, st>>>(dw_acc, reinterpret_cast<__nv_bfloat16*>(dW), n);
    LP_LAUNCH_CHECK("f32_to_bf16_kernel");
  }
  return LP_OK;
}

}  // namespace

extern "C" {

int lp_bwd(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs, int64_t v_off,
           const int32_t* y, float softcap, const float* norm, const float* g, void* dH, int64_t ld_dh, void* dW,
           int flags, int64_t token_chunk, void* workspace, size_t workspace_bytes) {
  return bwd_impl(stream, H, T, d, ldh, W, Vs, v_off, y, softcap, norm, g, dH, ld_dh, dW, flags, token_chunk,
                  workspace, workspace_bytes, nullptr);
}

size_t lp_bwd_sum_counters(int64_t T) { return T > 0 ? (size_t)cdiv(T, 128) + 2 : 0; }

int lp_bwd_sum(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs,
               int64_t v_off, const int32_t* y, float softcap, const float* norm, const float* g, void* dH,
               void* dH_multicast, int64_t ld_dh, unsigned* counters, unsigned* counters_multicast, int rank,
               int world, int timeout_ms, void* dW, int flags, int64_t token_chunk, void* workspace,
               size_t workspace_bytes) {
  if (flags & (LP_BWD_DH_F32 | LP_BWD_NO_DH))
    return fail(LP_EINVAL, "lp_bwd_sum sums a bf16 dH: LP_BWD_DH_F32 / LP_BWD_NO_DH do not apply");
  if (dH_multicast == nullptr || counters == nullptr || counters_multicast == nullptr)
    return fail(LP_EINVAL, "null multicast dH or counters");
  if (((reinterpret_cast<uintptr_t>(dH) | reinterpret_cast<uintptr_t>(dH_multicast)) & 15) != 0)
    return fail(LP_EINVAL, "dH and its multicast address must be 16-byte aligned");
  if (world < 1 || rank < 0 || rank >= world) return fail(LP_EINVAL, "bad rank %d / world %d", rank, world);
  if (timeout_ms <= 0) return fail(LP_EINVAL, "timeout_ms must be positive");
  const MeshSum ms{dH_multicast, counters, counters_multicast, rank, world, (unsigned long long)timeout_ms * 1000000ull};
  return bwd_impl(stream, H, T, d, ldh, W, Vs, v_off, y, softcap, norm, g, dH, ld_dh, dW, flags, token_chunk,
                  workspace, workspace_bytes, &ms);
}

int lp_gemm_bf16(void* stream, const void* A, int64_t M, int64_t K, int64_t lda, int a_mn, const void* B, int64_t N,
                 int64_t ldb, int b_mn, float* D, int64_t ldd) {
  if (M <= 0 || N <= 0 || K <= 0) return fail(LP_EINVAL, "bad GEMM sizes");
  if (A == nullptr || B == nullptr || D == nullptr) return fail(LP_EINVAL, "null GEMM operand");
  if (ldd < N || ldd % 4 != 0) return fail(LP_EINVAL, "ldd must be >= N and a multiple of 4");
  if (N % 4 != 0) return fail(LP_EINVAL, "N must be a multiple of 4");
  DeviceInfo* di = nullptr;
  int rc = current_device_info(&di);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  alignas(64) CUtensorMap ta, tb, to;
  // K-major A: [M rows][K], MN-major A: [K rows][M]; likewise B with N.
  if (a_mn) rc = map_bf16(&ta, A, M, K, lda, 64, 64, "A (MN-major)");
  else rc = map_bf16(&ta, A, K, M, lda, BK, 128, "A (K-major)");
  if (rc) return rc;
  const int cg = cta_group_for(CG_HOOK);
  if (b_mn) rc = map_bf16(&tb, B, N, K, ldb, 64, 64, "B (MN-major)");
  else rc = map_bf16(&tb, B, K, N, ldb, BK, b_box_rows(cg), "B (K-major)");
  if (rc) return rc;
  if ((rc = map_store_f32(&to, D, N, M, ldd, "D", store_box_bytes(cg)))) return rc;
  GemmParams p{};
  p.s = plan_gemm(M, N, K, workers(di, cg), false, 0, 128 * cg);
  p.e.store_mode = STORE_F32;
  if (!a_mn && !b_mn) return launch_gemm<EPI_STORE, false, false, false>(st, ta, tb, to, p, di, "gemm");
  if (!a_mn && b_mn) return launch_gemm<EPI_STORE, false, true, false>(st, ta, tb, to, p, di, "gemm");
  if (a_mn && b_mn) return launch_gemm<EPI_STORE, true, true, false>(st, ta, tb, to, p, di, "gemm");
  return launch_gemm<EPI_STORE, true, false, false>(st, ta, tb, to, p, di, "gemm");
}

size_t lp_compact_workspace_bytes(int64_t B, int64_t N) {
  const int64_t slots = std::max<int64_t>(B * N, 1);
  return align_up((size_t)cdiv(slots, kCompactBlock) * 4, 256) * 2;
}

int lp_compact(void* stream, const uint8_t* mask, int64_t B, int64_t N, const void* hidden, int64_t hidden_bstride,
               int64_t hidden_rstride, int64_t row_offset, int64_t d, const int32_t* ids, void* H_out, int32_t* y_out,
               int32_t* idx, int32_t* pos, int32_t* count, void* workspace, size_t workspace_bytes) {
  if (B < 0 || N < 0) return fail(LP_EINVAL, "bad B=%lld N=%lld", (long long)B, (long long)N);
  const int64_t slots = B * N;
  if (slots > ((int64_t)1 << 31) - 1) return fail(LP_EINVAL, "too many slots");
  if (mask == nullptr || idx == nullptr || pos == nullptr || count == nullptr)
    return fail(LP_EINVAL, "null mask / idx / pos / count");
  if (hidden != nullptr) {
    if (d <= 0 || d % 8 != 0) return fail(LP_EINVAL, "d=%lld must be a positive multiple of 8", (long long)d);
    if (H_out == nullptr) return fail(LP_EINVAL, "null H_out");
    if (hidden_rstride % 8 != 0 || hidden_bstride % 8 != 0) return fail(LP_EINVAL, "hidden strides must be multiples of 8");
    if ((reinterpret_cast<uintptr_t>(hidden) & 15) || (reinterpret_cast<uintptr_t>(H_out) & 15))
      return fail(LP_EINVAL, "hidden / H_out must be 16-byte aligned");
    if (y_out != nullptr && ids == nullptr) return fail(LP_EINVAL, "y_out needs ids");
  }
  const size_t need = lp_compact_workspace_bytes(B, N);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(LP_EWORKSPACE, "lp_compact needs %zu workspace bytes, got %zu", need, workspace_bytes);
  DeviceInfo* di = nullptr;
  if (int rc = current_device_info(&di)) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (slots == 0) {
    LP_CUDA_TRY(cudaMemsetAsync(count, 0, sizeof(int32_t), st));
    return LP_OK;
  }
  const int nblocks = (int)cdiv(slots, kCompactBlock);
  ProfScope prof(st, "compact");
  int* block_counts = reinterpret_cast<int*>(workspace);
  int* block_offsets = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + need / 2);
  compact_count_kernel<<<nblocks, 256, 0, st>>>(mask, slots, block_counts);
  LP_LAUNCH_CHECK("compact_count_kernel");
  compact_scan_kernel<<<1, 1024, 0, st>>>(block_counts, nblocks, block_offsets, count);
  LP_LAUNCH_CHECK("compact_scan_kernel");
  compact_write_kernel<<<nblocks, 256, 0, st>>>(mask, slots, block_offsets, idx, pos);
  LP_LAUNCH_CHECK("compact_write_kernel");
  if (hidden != nullptr) {
    const int64_t warps = std::min<int64_t>(slots, (int64_t)di->sms * 32);
    compact_gather_kernel<<<(unsigned)cdiv(warps * 32, 256), 256, 0, st>>>(
        idx, count, N, reinterpret_cast<const __nv_bfloat16*>(hidden), hidden_bstride, hidden_rstride, row_offset, d,
        ids, reinterpret_cast<__nv_bfloat16*>(H_out), y_out);
    LP_LAUNCH_CHECK("compact_gather_kernel");
  }
  return LP_OK;
}

int lp_scatter_rows(void* stream, const void* src, int64_t src_stride, const int32_t* pos, int64_t slots,
                    int64_t width, int elem_bytes, void* out, int64_t out_stride, int64_t rows_per_group,
                    int64_t group_stride, int out_elem_bytes) {
  if (slots < 0 || width <= 0 || (elem_bytes != 2 && elem_bytes != 4))
    return fail(LP_EINVAL, "bad slots / width / elem_bytes");
  if (out_elem_bytes != elem_bytes && !(elem_bytes == 4 && out_elem_bytes == 2))
    return fail(LP_EINVAL, "out_elem_bytes must equal elem_bytes, or be 2 for f32 -> bf16");
  if (rows_per_group <= 0) return fail(LP_EINVAL, "rows_per_group must be positive");
  if (slots == 0) return LP_OK;
  if (src == nullptr || pos == nullptr || out == nullptr) return fail(LP_EINVAL, "null src / pos / out");
  DeviceInfo* di = nullptr;
  if (int rc = current_device_info(&di)) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (out_elem_bytes != elem_bytes) {
    if (width % 8 != 0 || src_stride % 4 != 0 || out_stride % 8 != 0 || group_stride % 8 != 0 ||
        (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
      return fail(LP_EINVAL, "f32 -> bf16 scatter needs width % 8 == 0 and 16-byte aligned rows");
    ProfScope prof(st, "scatter_rows");
    const int64_t warps = std::min<int64_t>(slots, 148 * 64);
    scatter_rows_f32_to_bf16_kernel<<<(unsigned)cdiv(warps * 32, 256), 256, 0, st>>>(
        reinterpret_cast<const float*>(src), src_stride, pos, slots, width, reinterpret_cast<__nv_bfloat16*>(out),
        out_stride, rows_per_group, group_stride);
    LP_LAUNCH_CHECK("scatter_rows_f32_to_bf16_kernel");
    return LP_OK;
  }
  const int64_t row_bytes = width * elem_bytes;
  ProfScope prof(st, "scatter_rows");
  const bool vec = row_bytes % 16 == 0 && (src_stride * elem_bytes) % 16 == 0 && (out_stride * elem_bytes) % 16 == 0 &&
                   (group_stride * elem_bytes) % 16 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  if (vec) {
    const int64_t warps = std::min<int64_t>(slots, 148 * 64);
    scatter_rows_vec_kernel<<<(unsigned)cdiv(warps * 32, 256), 256, 0, st>>>(
        reinterpret_cast<const uint8_t*>(src), src_stride * elem_bytes, pos, slots, row_bytes,
        reinterpret_cast<uint8_t*>(out), out_stride * elem_bytes, rows_per_group, group_stride * elem_bytes);
    LP_LAUNCH_CHECK("scatter_rows_vec_kernel");
  } else {
    const int64_t total = slots * width;
    const unsigned grid = (unsigned)std::min<int64_t>(cdiv(total, 256), 148 * 16);
    scatter_rows_elem_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const uint8_t*>(src), src_stride, pos, slots,
                                                   width, elem_bytes, reinterpret_cast<uint8_t*>(out), out_stride,
                                                   rows_per_group, group_stride);
    LP_LAUNCH_CHECK("scatter_rows_elem_kernel");
  }
  return LP_OK;
}

int lp_peer_barrier(void* stream, const unsigned long long* signal_pads, int rank, int world, int channel,
                    int timeout_ms) {
  if (signal_pads == nullptr) return fail(LP_EINVAL, "null signal_pads");
  if (world < 1 || world > 1024 || rank < 0 || rank >= world) return fail(LP_EINVAL, "bad rank %d / world %d", rank, world);
  if (channel < 0 || timeout_ms <= 0) return fail(LP_EINVAL, "bad channel %d or timeout %d ms", channel, timeout_ms);
  DeviceInfo* di = nullptr;
  if (int rc = current_device_info(&di)) return rc;  // device set-up (host-visible error slot)
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int threads = (world + 31) / 32 * 32;
  ProfScope prof(st, "peer_barrier");
  peer_barrier_kernel<<<1, threads, 0, st>>>(signal_pads, rank, world, channel,
                                             (unsigned long long)timeout_ms * 1000000ull);
  LP_LAUNCH_CHECK("peer_barrier_kernel");
  return LP_OK;
}

}  // extern "C"

// ============================================================================= no-alloc forward
// lp_fwd_noalloc: the forward of lp_fwd for callers that cannot allocate device memory at
// the call site. Its scratch (the per-row partial max / sum of every vocabulary group and
// the owned target logit) lives in one file-scope device array that every GPU which loads
// this library holds until the process exits. Host code must not hand the array's name to
// a kernel (in host code it is only a stand-in symbol): the device address is looked up
// once per device with cudaGetSymbolAddress and cached.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(LP_NOALLOC_SCRATCH_BYTES);
}  // namespace

static __device__ __align__(256) unsigned char g_lp_noalloc_scratch[kNoAllocScratchBytes];

namespace {

void* g_noalloc_scratch_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of the scratch array on the current device (set up on first use there).
int noalloc_scratch(void** out) {
  int dev = 0;
  LP_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(LP_EINVAL, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_lp_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(LP_ECUDA, "cudaGetSymbolAddress(no-alloc scratch) on device %d: %s", dev, cudaGetErrorString(e));
    g_noalloc_scratch_ptr[dev] = p;
  }
  *out = g_noalloc_scratch_ptr[dev];
  return LP_OK;
}


}  // namespace

extern "C" int lp_fwd_noalloc(void* stream, const void* H, int64_t T, int64_t d, int64_t ldh, const void* W, int64_t Vs,
                              int64_t v_off, const int32_t* y, float softcap, float* stats, float* logp) {
  int rc = check_common(H, T, d, ldh, W, Vs, y);
  if (rc) return rc;
  if (T == 0) return LP_OK;
  if (stats == nullptr) return fail(LP_EINVAL, "null stats");
  DeviceInfo* di = nullptr;
  if ((rc = current_device_info(&di))) return rc;
  // Same tile plan as lp_fwd, with the vocabulary groups widened until the partials fit
  // the fixed scratch; too many tokens for even one group is refused.
  const int cg = cta_group_for(CG_FWD);
  GemmSched s = plan_fwd(T, Vs, d, workers(di, cg), 128 * cg);
  size_t part_bytes = 0;
  const size_t need = widen_fwd_groups(&s, T, kNoAllocScratchBytes, &part_bytes);
  if (need > kNoAllocScratchBytes)
    return fail(LP_EINVAL,
                "lp_fwd_noalloc: T=%lld tokens need %zu scratch bytes, above its fixed limit of %zu bytes "
                "(LP_NOALLOC_SCRATCH_BYTES); use lp_fwd with a workspace",
                (long long)T, need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(&scratch))) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float2* part = reinterpret_cast<float2*>(scratch);
  float* tgt = reinterpret_cast<float*>(reinterpret_cast<char*>(scratch) + part_bytes);

  alignas(64) CUtensorMap ta, tb;
  if ((rc = map_bf16(&ta, H, d, T, ldh, BK, 128, "hidden"))) return rc;
  if ((rc = map_bf16(&tb, W, d, Vs, d, BK, b_box_rows(cg), "embedding"))) return rc;
  GemmParams p{};
  p.s = s;
  p.e.y = y;
  p.e.v_off = v_off;
  p.e.softcap = softcap;
  p.e.part = part;
  p.e.tgt = tgt;
  set_hints(p, G_FWD);
  if ((rc = launch_gemm_cap<EPI_FWD_LSE, false, false>(softcap > 0.f, st, ta, tb, ta, p, di, "fwd_lse_gemm"))) return rc;
  ProfScope prof(st, "fwd_finalize");
  fwd_finalize_kernel<<<(unsigned)cdiv(T, 256), 256, 0, st>>>(part, 2 * s.n_groups, (int)T, tgt, y, v_off, Vs, stats,
                                                              logp);
  LP_LAUNCH_CHECK("fwd_finalize_kernel");
  return LP_OK;
}
