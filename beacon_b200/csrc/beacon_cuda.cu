// beacon_cuda.cu -- libbeacon_cuda.so: the extern "C" boundary (include/beacon_cuda.h)
// over the sm_100a kernels.  One translation unit so every kernel shares the
// device fault words in sm100.cuh.
//
// Host-side responsibilities: argument validation (mirroring LaunchParams::validate,
// crates/beacon-cuda/src/launch.rs:78-97, plus shape/alignment checks), TMA tensor-map
// encoding, tile-shape selection, workspace management and error mapping onto
// LaunchError (crates/beacon-cuda/src/error.rs:4-13).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/beacon_cuda.h"
#include "attention.cuh"
#include "attention_bwd.cuh"
#include "diag.cuh"
#include "elementwise.cuh"
#include "gemm.cuh"
#include "gemm_fp8.cuh"
#include "sm100.cuh"

using namespace beacon;
using bf16 = __nv_bfloat16;

// ===========================================================================
// errors
// ===========================================================================
namespace {

thread_local std::string t_last_error;
thread_local int t_last_status = BEACON_OK;
std::atomic<uint64_t> g_launches{0};

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  t_last_status = status;
  return status;
}

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(BEACON_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return BEACON_OK;
}

// ---------------------------------------------------------------------------
// Per-kernel device timing: when enabled, the tensor-core kernels are bracketed by
// CUDA events recorded on the stream they are launched on; beacon_profile_read()
// synchronises on those events and returns the accumulated time per kernel name.
// ---------------------------------------------------------------------------
struct ProfRec {
  const char* name;
  cudaEvent_t e0, e1;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRec> g_prof_pending;
std::vector<cudaEvent_t> g_prof_pool;
struct ProfTotal {
  std::string name;
  double ms;
  uint64_t count;
};
std::vector<ProfTotal> g_prof_totals;

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
  const char* name = nullptr;
  cudaStream_t st = nullptr;
  cudaEvent_t e0 = nullptr;
  ProfScope(const char* n, cudaStream_t s) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (!g_prof_on) return;
    name = n;
    st = s;
    e0 = prof_event();
    cudaEventRecord(e0, st);
  }
  ~ProfScope() {
    if (!e0) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    cudaEvent_t e1 = prof_event();
    cudaEventRecord(e1, st);
    g_prof_pending.push_back(ProfRec{name, e0, e1});
  }
};

#define BEACON_TRY(expr)             \
  do {                               \
    int _rc = (expr);                \
    if (_rc != BEACON_OK) return _rc; \
  } while (0)

// ===========================================================================
// devices
// ===========================================================================
struct DeviceInfo {
  int sms = 0;
  int major = 0, minor = 0;
  bool init = false;
};
std::mutex g_dev_mu;
DeviceInfo g_dev[64];

int current_device(int* dev, DeviceInfo** info) {
  int d = 0;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) return fail(BEACON_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (d < 0 || d >= 64) return fail(BEACON_ERR_CUDA, "device ordinal %d out of range", d);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo& di = g_dev[d];
  if (!di.init) {
    cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, d);
    cudaDeviceGetAttribute(&di.major, cudaDevAttrComputeCapabilityMajor, d);
    cudaDeviceGetAttribute(&di.minor, cudaDevAttrComputeCapabilityMinor, d);
    di.init = true;
  }
  if (di.major != 10 || di.minor != 0)
    return fail(BEACON_ERR_MODULE_LOAD, "device %d is sm_%d%d; this library is built for sm_100a only", d, di.major,
                di.minor);
  *dev = d;
  *info = &di;
  return BEACON_OK;
}

// The work-counter slot (g_sched) of the next persistent launch on device `dev`.
std::atomic<unsigned> g_sched_next[64];
int sched_slot(int dev) { return (int)(g_sched_next[dev].fetch_add(1u) % (unsigned)kSchedSlots); }

// ===========================================================================
// TMA tensor maps
// ===========================================================================
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor of `rank` dims (dims[0] innermost, contiguous); bf16 with 128-byte swizzle unless
// given another element type / swizzle.
int make_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides_bytes,
             const uint32_t* box, CUtensorMapDataType type = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(BEACON_ERR_MODULE_LOAD, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) s[i] = strides_bytes[i];
  CUresult r = fn(m, type, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return BEACON_OK;
}

int make_map_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                uint32_t box_inner, uint32_t box_outer) {
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {ld_elems * 2};
  const uint32_t box[2] = {box_inner, box_outer};
  return make_map(m, base, 2, dims, strides, box);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ===========================================================================
// workspace: grow-only, one per device
// ===========================================================================
struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::mutex g_ws_mu;
Workspace g_ws[64];

// While beacon_launch dispatches a kernel ID, the arena's own workspace stands in for the
// library's: an entry point that needs scratch and was given none takes the arena's, and
// fails with OutOfMemory instead of allocating when the arena has too little.
struct ArenaScope {
  bool active = false;
  void* ws = nullptr;
  size_t bytes = 0;
};
thread_local ArenaScope t_arena;

int get_workspace(int dev, size_t need, void* user, size_t user_bytes, void** out) {
  if (need == 0) {
    *out = user;
    return BEACON_OK;
  }
  if (user != nullptr) {
    if (user_bytes < need)
      return fail(BEACON_ERR_OUT_OF_MEMORY, "workspace of %zu bytes given, %zu needed", user_bytes, need);
    *out = user;
    return BEACON_OK;
  }
  if (t_arena.active) {
    if (t_arena.bytes < need)
      return fail(BEACON_ERR_OUT_OF_MEMORY,
                  "out of device memory: requested %zu bytes of arena workspace, %zu available "
                  "(reserve it once with beacon_workspace_create)",
                  need, t_arena.bytes);
    *out = t_arena.ws;
    return BEACON_OK;
  }
  std::lock_guard<std::mutex> lk(g_ws_mu);
  Workspace& w = g_ws[dev];
  if (w.bytes < need) {
    if (w.ptr) {
      cudaDeviceSynchronize();
      cudaFree(w.ptr);
      w.ptr = nullptr;
      w.bytes = 0;
    }
    cudaError_t e = cudaMalloc(&w.ptr, need);
    if (e != cudaSuccess) {
      cudaGetLastError();
      size_t fr = 0, tot = 0;
      cudaMemGetInfo(&fr, &tot);
      t_last_error = "workspace allocation failed";
      t_last_status = BEACON_ERR_OUT_OF_MEMORY;
      return fail(BEACON_ERR_OUT_OF_MEMORY, "out of device memory: requested %zu bytes, %zu available", need, fr);
    }
    w.bytes = need;
  }
  *out = w.ptr;
  return BEACON_OK;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ===========================================================================
// GEMM dispatch
// ===========================================================================
struct Operand {
  const void* ptr;
  bool mn_major;  // A: [K][M] storage (else [M][K]);  B: [K][N] storage (else [N][K])
  int64_t ld;     // elements between consecutive storage rows
};

template <int BN, bool A_MN, bool B_MN>
int launch_gemm_tc_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2, const GemmParams& p,
                     int sms, cudaStream_t st) {
  using Cfg = GemmCfg<BN>;
  auto kern = k_gemm_bf16_tc<BN, A_MN, B_MN>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return fail(BEACON_ERR_CUDA, "gemm smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = tiles < sms ? tiles : sms;
  {
    ProfScope prof("k_gemm_bf16_tc", st);
    kern<<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, st>>>(ta, tb, tb2, p);
  }
  return check_launch("k_gemm_bf16_tc");
}

template <int BN>
int launch_gemm_tc_bn(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2,
                      const GemmParams& p, int sms, cudaStream_t st) {
  if (!a_mn && b_mn) return launch_gemm_tc_t<BN, false, true>(ta, tb, tb2, p, sms, st);
  if (!a_mn && !b_mn) return launch_gemm_tc_t<BN, false, false>(ta, tb, tb2, p, sms, st);
  if (a_mn && b_mn) return launch_gemm_tc_t<BN, true, true>(ta, tb, tb2, p, sms, st);
  return launch_gemm_tc_t<BN, true, false>(ta, tb, tb2, p, sms, st);
}

template <bool A_MN, bool B_MN, int BN>
int launch_gemm_tc2_t(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2, const GemmParams& p,
                      int sms, cudaStream_t st) {
  using Cfg = GemmCfg2<BN>;
  auto kern = k_gemm_bf16_tc2<A_MN, B_MN, BN>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return fail(BEACON_ERR_CUDA, "gemm2 smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  const int pairs = std::min(tiles, sms / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  {
    ProfScope prof("k_gemm_bf16_tc", st);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tb2, p);
    if (e != cudaSuccess) return fail(BEACON_ERR_CUDA, "k_gemm_bf16_tc2 launch: %s", cudaGetErrorString(e));
  }
  return check_launch("k_gemm_bf16_tc2");
}

template <int BN>
int launch_gemm_tc2_bn(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb2,
                       const GemmParams& p, int sms, cudaStream_t st) {
  if (!a_mn && b_mn) return launch_gemm_tc2_t<false, true, BN>(ta, tb, tb2, p, sms, st);
  if (!a_mn && !b_mn) return launch_gemm_tc2_t<false, false, BN>(ta, tb, tb2, p, sms, st);
  if (a_mn && b_mn) return launch_gemm_tc2_t<true, true, BN>(ta, tb, tb2, p, sms, st);
  return launch_gemm_tc2_t<true, false, BN>(ta, tb, tb2, p, sms, st);
}

// Kernel choice override for tests: BEACON_GEMM_PATH = "1sm" | "2sm" (256x256 pair tiles) |
// "2sm128" (256x128 pair tiles); default: by shape.
int gemm_path_override() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("BEACON_GEMM_PATH");
    v = (e && !strcmp(e, "1sm")) ? 1 : (e && !strcmp(e, "2sm")) ? 2 : (e && !strcmp(e, "2sm128")) ? 3 : 0;
  }
  return v;
}

// SM-wave efficiency of `tiles` work units over `slots` parallel slots.
double wave_eff(int64_t tiles, int64_t slots) {
  const int64_t waves = (tiles + slots - 1) / slots;
  return (double)tiles / (double)(waves * slots);
}

// Pick the N tile: the widest tile keeps shared-memory traffic per FLOP lowest,
// narrower tiles win back idle SMs when the tile count is a poor multiple of the SM count.
int choose_bn(int64_t M, int64_t Nout, bool swiglu, int sms) {
  const int cands[3] = {256, 128, 64};
  const double cost[3] = {1.0, 0.93, 0.80};
  int best = 256;
  double best_score = -1.0;
  for (int i = 0; i < 3; ++i) {
    const int bn = cands[i];
    if (swiglu && bn < 128) continue;
    const int64_t cols = swiglu ? bn / 2 : bn;
    const int64_t tiles = ((M + 127) / 128) * ((Nout + cols - 1) / cols);
    const int64_t waves = (tiles + sms - 1) / sms;
    const double eff = (double)tiles / (double)(waves * sms);
    const double score = eff * cost[i];
    if (score > best_score + 1e-9) {
      best_score = score;
      best = bn;
    }
  }
  return best;
}

// The tile shape of a bf16 GEMM: 2-SM pair tiles of 256 x pair_bn, or (pair_bn = 0) 1-SM
// tiles of 128 x bn.
struct GemmPlan {
  int pair_bn = 0, bn = 0;
};
GemmPlan gemm_plan(int64_t M, int64_t N, bool swiglu, int sms, int force_bn) {
  // 2-SM pair tiles halve each SM's operand stream; they win whenever their wave
  // efficiency is close to the best 1-SM tile's.  Per SM and 64-deep K step a 128x128 1-SM
  // tile needs 32 KB for 71-cycle MMAs, more than TMA delivers to one SM (measured ~58 B per
  // clock in that kernel); a 256x128 pair tile needs 24 KB and a 256x256 one 32 KB for MMAs
  // twice as long.  Scores: wave efficiency x the rows the tiles cover (M padded to 128 or
  // 256 rows) x a per-shape credit.
  GemmPlan plan;
  {
    const int ov = gemm_path_override();
    const double rows1 = (double)M / (double)(((M + 127) / 128) * 128);
    const double rows2 = (double)M / (double)(((M + 255) / 256) * 256);
    const int64_t cols2 = swiglu ? 128 : 256;
    const int64_t tiles2 = ((M + 255) / 256) * ((N + cols2 - 1) / cols2);
    const double score2 = wave_eff(tiles2, sms / 2) * rows2 * 1.15;
    const int64_t tiles2n = ((M + 255) / 256) * ((N + 127) / 128);
    const double score2n = swiglu ? 0.0 : wave_eff(tiles2n, sms / 2) * rows2 * 0.97;
    const int bn1 = choose_bn(M, N, swiglu, sms);
    const int64_t c1 = swiglu ? bn1 / 2 : bn1;
    const double cost1 = bn1 == 256 ? 1.0 : bn1 == 128 ? 0.93 : 0.80;
    const double score1 = wave_eff(((M + 127) / 128) * ((N + c1 - 1) / c1), sms) * rows1 * cost1;
    if (ov == 2 || (ov == 3 && swiglu)) {
      plan.pair_bn = 256;
    } else if (ov == 3) {
      plan.pair_bn = 128;
    } else if (ov == 0 && !force_bn) {
      if (score2 > score1 && score2 >= score2n) plan.pair_bn = 256;
      else if (score2n > score1) plan.pair_bn = 128;
    }
    plan.bn = plan.pair_bn ? plan.pair_bn : (force_bn ? force_bn : bn1);
  }
  return plan;
}

// C[M,N] = A . B (+ epilogue) with bf16 operands.  `B2` is the up-projection for the tile-pair
// (SwiGLU) epilogues, or the second K range of B when p.k_split > 0 (C = A . [B ; B2]).
int gemm_bf16(const Operand& A, const Operand& B, const Operand* B2, GemmParams p, cudaStream_t st, int force_bn = 0) {
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  if (p.M == 0 || p.N == 0) return BEACON_OK;
  const bool swiglu = epi_tile_pairs(p.epi);
  const bool two_b = swiglu || p.k_split > 0;
  if (p.k_split > 0 && (p.k_split % 64 != 0 || p.k_split >= p.K || swiglu))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "K-split GEMM: split %d of K %d must be a multiple of 64", p.k_split,
                p.K);
  const bool tma_ok = aligned16(A.ptr) && aligned16(B.ptr) && (A.ld % 8 == 0) && (B.ld % 8 == 0) &&
                      (!two_b || (aligned16(B2->ptr) && B2->ld % 8 == 0)) && p.K > 0;
  if (!tma_ok) {
    if (two_b || p.sc_hd > 0 || p.epi == kEpiSwigluBwd || p.out2 != nullptr)
      return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "fused GEMM epilogue needs 16-byte aligned rows");
    // exact SIMT path for shapes TMA cannot describe
    const long long sam = A.mn_major ? 1 : A.ld, sak = A.mn_major ? A.ld : 1;
    const long long sbk = B.mn_major ? B.ld : 1, sbn = B.mn_major ? 1 : B.ld;
    dim3 grid((unsigned)((p.N + 63) / 64), (unsigned)((p.M + 63) / 64));
    k_gemm_simt<bf16><<<grid, 256, 0, st>>>(reinterpret_cast<const bf16*>(A.ptr), sam, sak,
                                            reinterpret_cast<const bf16*>(B.ptr), sbk, sbn, p);
    return check_launch("k_gemm_simt<bf16>");
  }
  const int pair_bn = gemm_plan(p.M, p.N, swiglu, di->sms, force_bn).pair_bn;  // 0: 1-SM tiles
  if (pair_bn) {
    p.tiles_m = (p.M + 255) / 256;
    p.tiles_n = swiglu ? (p.N + 127) / 128 : (p.N + pair_bn - 1) / pair_bn;
    CUtensorMap ta, tb, tb2;
    if (!A.mn_major)
      BEACON_TRY(make_map_2d(&ta, A.ptr, (uint64_t)p.K, (uint64_t)p.M, (uint64_t)A.ld, 64, 128));
    else
      BEACON_TRY(make_map_2d(&ta, A.ptr, (uint64_t)p.M, (uint64_t)p.K, (uint64_t)A.ld, 64, 64));
    // with a K split each B tensor holds its own K range (extent k_split / K - k_split)
    const uint64_t k1 = p.k_split > 0 ? (uint64_t)p.k_split : (uint64_t)p.K;
    const uint64_t k2 = p.k_split > 0 ? (uint64_t)(p.K - p.k_split) : (uint64_t)p.K;
    auto map_b2 = [&](CUtensorMap* m, const Operand& op, uint64_t kext) -> int {
      if (op.mn_major) return make_map_2d(m, op.ptr, (uint64_t)p.N, kext, (uint64_t)op.ld, 64, 64);
      return make_map_2d(m, op.ptr, kext, (uint64_t)p.N, (uint64_t)op.ld, 64, (uint32_t)(pair_bn / 2));
    };
    BEACON_TRY(map_b2(&tb, B, k1));
    if (two_b) {
      if (B2->mn_major != B.mn_major) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "B operands differ in major");
      BEACON_TRY(map_b2(&tb2, *B2, k2));
    } else {
      tb2 = tb;
    }
    if (pair_bn == 128) return launch_gemm_tc2_bn<128>(A.mn_major, B.mn_major, ta, tb, tb2, p, di->sms, st);
    return launch_gemm_tc2_bn<256>(A.mn_major, B.mn_major, ta, tb, tb2, p, di->sms, st);
  }
  const int bn = force_bn ? force_bn : choose_bn(p.M, p.N, swiglu, di->sms);
  const int cols = swiglu ? bn / 2 : bn;
  p.tiles_m = (p.M + 127) / 128;
  p.tiles_n = (p.N + cols - 1) / cols;
  CUtensorMap ta, tb, tb2;
  // A logical [M,K]
  if (!A.mn_major)
    BEACON_TRY(make_map_2d(&ta, A.ptr, (uint64_t)p.K, (uint64_t)p.M, (uint64_t)A.ld, 64, 128));
  else
    BEACON_TRY(make_map_2d(&ta, A.ptr, (uint64_t)p.M, (uint64_t)p.K, (uint64_t)A.ld, 64, 64));
  // B logical [K,N]; for SwiGLU the tensor's N is the hidden width F; with a K split each
  // B tensor holds its own K range
  const uint64_t k1 = p.k_split > 0 ? (uint64_t)p.k_split : (uint64_t)p.K;
  const uint64_t k2 = p.k_split > 0 ? (uint64_t)(p.K - p.k_split) : (uint64_t)p.K;
  auto map_b = [&](CUtensorMap* m, const Operand& op, uint64_t kext) -> int {
    if (op.mn_major) return make_map_2d(m, op.ptr, (uint64_t)p.N, kext, (uint64_t)op.ld, 64, 64);
    return make_map_2d(m, op.ptr, kext, (uint64_t)p.N, (uint64_t)op.ld, 64, (uint32_t)cols);
  };
  BEACON_TRY(map_b(&tb, B, k1));
  if (two_b) {
    if (B2->mn_major != B.mn_major) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "B operands differ in major");
    BEACON_TRY(map_b(&tb2, *B2, k2));
  } else {
    tb2 = tb;
  }
  switch (bn) {
    case 256: return launch_gemm_tc_bn<256>(A.mn_major, B.mn_major, ta, tb, tb2, p, di->sms, st);
    case 128: return launch_gemm_tc_bn<128>(A.mn_major, B.mn_major, ta, tb, tb2, p, di->sms, st);
    default: return launch_gemm_tc_bn<64>(A.mn_major, B.mn_major, ta, tb, tb2, p, di->sms, st);
  }
}

int gemm_f32(const Operand& A, const Operand& B, GemmParams p, cudaStream_t st) {
  if (p.M == 0 || p.N == 0) return BEACON_OK;
  const long long sam = A.mn_major ? 1 : A.ld, sak = A.mn_major ? A.ld : 1;
  const long long sbk = B.mn_major ? B.ld : 1, sbn = B.mn_major ? 1 : B.ld;
  dim3 grid((unsigned)((p.N + 63) / 64), (unsigned)((p.M + 63) / 64));
  k_gemm_simt<float><<<grid, 256, 0, st>>>(reinterpret_cast<const float*>(A.ptr), sam, sak,
                                           reinterpret_cast<const float*>(B.ptr), sbk, sbn, p);
  return check_launch("k_gemm_simt<f32>");
}

GemmParams gemm_params(int64_t M, int64_t N, int64_t K, void* out, int64_t ldo, bool out_f32) {
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.out = out;
  p.ldo = ldo;
  p.out_f32 = out_f32 ? 1 : 0;
  p.epi = kEpiStore;
  p.aux_f32 = out_f32 ? 1 : 0;
  p.out_scale = 1.0f;
  return p;
}

int check_dtype_gemm(int dtype) {
  if (dtype != BEACON_BF16 && dtype != BEACON_F32)
    return fail(BEACON_ERR_UNIMPLEMENTED, "dtype %d: the GEMM family supports f32 and bf16", dtype);
  return BEACON_OK;
}

int check_dims(const char* what, int64_t a, int64_t b, int64_t c) {
  if (a < 0 || b < 0 || c < 0) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "%s: negative dimension", what);
  if (a > INT32_MAX || b > INT32_MAX || c > INT32_MAX)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "%s: dimension exceeds 2^31-1", what);
  return BEACON_OK;
}

int zero_fill(void* p, size_t bytes, cudaStream_t st) {
  if (!p || bytes == 0) return BEACON_OK;
  cudaError_t e = cudaMemsetAsync(p, 0, bytes, st);
  if (e != cudaSuccess) return fail(BEACON_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  return BEACON_OK;
}

// One logical C = A.B with the given storage of A and B, dtype-dispatched.
int gemm_any(int dtype, const Operand& A, const Operand& B, GemmParams p, cudaStream_t st) {
  if (p.K == 0) {  // empty reduction: out = epilogue(0)
    const size_t es = p.out_f32 ? 4 : 2;
    if (p.epi == kEpiStore || (p.epi == kEpiBias && p.bias == nullptr)) {
      if ((int64_t)p.ldo == p.N) return zero_fill(p.out, (size_t)p.M * p.N * es, st);
    }
  }
  if (dtype == BEACON_F32) return gemm_f32(A, B, p, st);
  return gemm_bf16(A, B, nullptr, p, st);
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int grid_for(int64_t work, int threads, int sms) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = (int64_t)sms * 8;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

}  // namespace

// ===========================================================================
// library
// ===========================================================================
extern "C" int beacon_version(void) { return 100; }

extern "C" int beacon_last_error(char* buf, size_t len) {
  if (buf && len) {
    strncpy(buf, t_last_error.c_str(), len - 1);
    buf[len - 1] = '\0';
  }
  return t_last_status;
}

extern "C" uint64_t beacon_launch_count(void) { return g_launches.load(); }

extern "C" void beacon_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof_on = on != 0;
}

extern "C" int beacon_profile_read(const char* kernel, double* total_ms, uint64_t* count) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (const ProfRec& r : g_prof_pending) {
    cudaEventSynchronize(r.e1);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, r.e0, r.e1);
    bool found = false;
    for (ProfTotal& t : g_prof_totals)
      if (t.name == r.name) {
        t.ms += ms;
        t.count += 1;
        found = true;
      }
    if (!found) g_prof_totals.push_back(ProfTotal{r.name, (double)ms, 1});
    g_prof_pool.push_back(r.e0);
    g_prof_pool.push_back(r.e1);
  }
  g_prof_pending.clear();
  if (total_ms) *total_ms = 0.0;
  if (count) *count = 0;
  if (kernel == nullptr) {  // reset
    g_prof_totals.clear();
    return BEACON_OK;
  }
  for (const ProfTotal& t : g_prof_totals)
    if (t.name == kernel) {
      if (total_ms) *total_ms = t.ms;
      if (count) *count = t.count;
    }
  return BEACON_OK;
}

extern "C" int beacon_device_status(int device, unsigned int out[3]) {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail(BEACON_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  e = cudaDeviceSynchronize();
  unsigned int w[4] = {0, 0, 0, 0};
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(w, g_beacon_status, sizeof(w));
  const unsigned int zero[4] = {0, 0, 0, 0};
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_beacon_status, zero, sizeof(zero));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(BEACON_ERR_CUDA, "device status: %s", cudaGetErrorString(e));
  if (out) {
    out[0] = w[0];
    out[1] = w[1];
    out[2] = w[2];
  }
  if (w[0] != 0) return fail(BEACON_ERR_CUDA, "device fault code %u at site 0x%x (%u faults)", w[0], w[1], w[2]);
  return BEACON_OK;
}

extern "C" int beacon_diag_wait_timeout(uint64_t limit_ns, unsigned int* out, void* stream) {
  if (!out) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "diag_wait_timeout: null pointer");
  if (limit_ns == 0 || limit_ns > 1000000000ull)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "diag_wait_timeout: limit must be in (0, 1 s]");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  k_diag_wait_timeout<<<1, 32, 0, as_stream(stream)>>>(limit_ns, reinterpret_cast<uint32_t*>(out));
  return check_launch("k_diag_wait_timeout");
}

extern "C" int beacon_diag_exp2_poly(float* out, const float* in, int64_t n, void* stream) {
  if (n < 0 || (n & 1)) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "diag_exp2_poly: n must be even");
  if (n == 0) return BEACON_OK;
  if (!out || !in) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "diag_exp2_poly: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  k_diag_exp2_poly<<<grid_for(n / 2, 256, di->sms), 256, 0, as_stream(stream)>>>(out, in, n);
  return check_launch("k_diag_exp2_poly");
}

// ===========================================================================
// matmul / linear
// ===========================================================================
namespace {

int launch_gemm_fp8w_tc2(const void* lhs, const void* rhs_fp8, GemmParams p, int sms, cudaStream_t st) {
  using Cfg = GemmFp8Cfg;
  CUtensorMap ta, tw;
  BEACON_TRY(make_map_2d(&ta, lhs, (uint64_t)p.K, (uint64_t)p.M, (uint64_t)p.K, 64, 128));
  {  // the fp8 weight [K][N] as bytes: boxes of 128 columns x 64 K rows, not swizzled
    const uint64_t dims[2] = {(uint64_t)p.N, (uint64_t)p.K};
    const uint64_t strides[1] = {(uint64_t)p.N};
    const uint32_t box[2] = {128, 64};
    BEACON_TRY(make_map(&tw, rhs_fp8, 2, dims, strides, box, CU_TENSOR_MAP_DATA_TYPE_UINT8,
                        CU_TENSOR_MAP_SWIZZLE_NONE));
  }
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_gemm_fp8w_tc2, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return fail(BEACON_ERR_CUDA, "fp8 gemm smem attribute: %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  p.tiles_m = (p.M + 255) / 256;
  p.tiles_n = (p.N + 255) / 256;
  const int pairs = std::min(p.tiles_m * p.tiles_n, sms / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  {
    ProfScope prof("k_gemm_fp8w_tc2", st);
    cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_fp8w_tc2, ta, tw, p);
    if (e != cudaSuccess) return fail(BEACON_ERR_CUDA, "k_gemm_fp8w_tc2 launch: %s", cudaGetErrorString(e));
  }
  return check_launch("k_gemm_fp8w_tc2");
}

// fp8 e4m3 weights [k, n] (crates/beacon-core/src/dtype.rs:134-195):
// out = (lhs . decode(rhs)) * scale (* *scale_dev) (+ bias).  Where TMA can describe the
// operands (16-byte aligned, k % 8 == 0, n % 16 == 0) the weights are decoded inside the
// GEMM pipeline (k_gemm_fp8w_tc2: each weight byte is read from HBM once); otherwise they
// are decoded to a bf16 copy in the library workspace and the bf16 GEMM runs on that.
int gemm_fp8w(void* out, const void* lhs, const void* rhs_fp8, float scale, const float* scale_dev,
              const void* bias, int64_t m, int64_t k, int64_t n, cudaStream_t st) {
  BEACON_TRY(check_dims("fp8-weight GEMM", m, k, n));
  if (m == 0 || n == 0) return BEACON_OK;
  if (!out || (k && (!lhs || !rhs_fp8))) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "fp8-weight GEMM: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  if (k > 0 && k % 8 == 0 && n % 16 == 0 && aligned16(lhs) && aligned16(rhs_fp8) && aligned16(out) &&
      gemm_path_override() != 1) {
    GemmParams p = gemm_params(m, n, k, out, n, false);
    p.out_scale = scale;
    p.out_scale_dev = scale_dev;
    if (bias) {
      p.epi = kEpiBias;
      p.bias = bias;
    }
    return launch_gemm_fp8w_tc2(lhs, rhs_fp8, p, di->sms, st);
  }
  void* ws = nullptr;
  const size_t wbytes = align256((size_t)k * n * 2);
  BEACON_TRY(get_workspace(dev, wbytes, nullptr, 0, &ws));
  if (k > 0) {
    if (!aligned16(rhs_fp8))
      return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "fp8-weight GEMM: weights must be 16-byte aligned");
    k_fp8_to_bf16<<<grid_for(k * n / 16 + 1, 256, di->sms), 256, 0, st>>>(
        reinterpret_cast<uint16_t*>(ws), reinterpret_cast<const uint8_t*>(rhs_fp8), k * n);
    BEACON_TRY(check_launch("k_fp8_to_bf16"));
  }
  GemmParams p = gemm_params(m, n, k, out, n, false);
  p.out_scale = scale;
  p.out_scale_dev = scale_dev;
  if (bias) {
    p.epi = kEpiBias;
    p.bias = bias;
  }
  return gemm_any(BEACON_BF16, Operand{lhs, false, k}, Operand{ws, true, n}, p, st);
}

}  // namespace

extern "C" int beacon_matmul_fp8w_fwd(void* out, const void* lhs, const void* rhs_fp8, float rhs_scale, int64_t m,
                                      int64_t k, int64_t n, void* stream) {
  return gemm_fp8w(out, lhs, rhs_fp8, rhs_scale, nullptr, nullptr, m, k, n, as_stream(stream));
}

extern "C" int beacon_linear_fp8w_fwd(void* out, const void* x, const void* weight_fp8, float weight_scale,
                                      const void* bias, int64_t m, int64_t k, int64_t n, void* stream) {
  return gemm_fp8w(out, x, weight_fp8, weight_scale, nullptr, bias, m, k, n, as_stream(stream));
}

extern "C" int beacon_linear_fp8w_fwd_devscale(void* out, const void* x, const void* weight_fp8,
                                               const float* weight_scale_dev, const void* bias, int64_t m, int64_t k,
                                               int64_t n, void* stream) {
  if (!weight_scale_dev) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "linear_fp8w_fwd_devscale: null pointer");
  return gemm_fp8w(out, x, weight_fp8, 1.0f, weight_scale_dev, bias, m, k, n, as_stream(stream));
}

extern "C" int beacon_quantize_fp8e4m3(void* out_fp8, float* scale, float* amax, const float* src, int64_t n,
                                       void* stream) {
  if (n < 0) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "quantize_fp8e4m3: negative n");
  if (!scale || !amax || (n > 0 && (!out_fp8 || !src)))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "quantize_fp8e4m3: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  cudaStream_t st = as_stream(stream);
  BEACON_TRY(zero_fill(amax, 4, st));
  if (n > 0) {
    k_absmax<<<grid_for(n / 4 + 1, 256, di->sms), 256, 0, st>>>(reinterpret_cast<unsigned int*>(amax), src, n);
    BEACON_TRY(check_launch("k_absmax"));
  }
  k_quantize_fp8<<<grid_for(std::max<int64_t>(n, 1), 256, di->sms), 256, 0, st>>>(
      reinterpret_cast<uint8_t*>(out_fp8), scale, amax, src, n);
  return check_launch("k_quantize_fp8");
}

extern "C" int beacon_matmul_plan(int64_t m, int64_t k, int64_t n, int32_t* out) {
  if (!out) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "matmul_plan: null output");
  if (m <= 0 || n <= 0 || k < 0 || m > INT32_MAX || n > INT32_MAX)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "matmul_plan: bad shape m=%lld k=%lld n=%lld", (long long)m,
                (long long)k, (long long)n);
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  const GemmPlan pl = gemm_plan(m, n, false, di->sms, 0);
  const int64_t tm = pl.pair_bn ? 256 : 128, tn = pl.pair_bn ? pl.pair_bn : pl.bn;
  out[0] = (int32_t)tm;
  out[1] = (int32_t)tn;
  out[2] = (int32_t)(((m + tm - 1) / tm) * ((n + tn - 1) / tn));
  out[3] = pl.pair_bn ? 2 : 1;
  out[4] = di->sms;
  return BEACON_OK;
}

extern "C" int beacon_matmul_fwd(void* out, const void* lhs, const void* rhs, int64_t m, int64_t k, int64_t n,
                                 int dtype, void* stream) {
  if (dtype == BEACON_FP8E4M3) return gemm_fp8w(out, lhs, rhs, 1.0f, nullptr, nullptr, m, k, n, as_stream(stream));
  BEACON_TRY(check_dtype_gemm(dtype));
  BEACON_TRY(check_dims("matmul_fwd", m, k, n));
  if (m && n && (!out || (k && (!lhs || !rhs))))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "matmul_fwd: null pointer");
  GemmParams p = gemm_params(m, n, k, out, n, dtype == BEACON_F32);
  return gemm_any(dtype, Operand{lhs, false, k}, Operand{rhs, true, n}, p, as_stream(stream));
}

extern "C" int beacon_matmul_bwd(void* dlhs, void* drhs, const void* dout, const void* lhs, const void* rhs,
                                 int64_t m, int64_t k, int64_t n, int dtype, void* stream) {
  BEACON_TRY(check_dtype_gemm(dtype));
  BEACON_TRY(check_dims("matmul_bwd", m, k, n));
  if ((dlhs && m && k && n && (!dout || !rhs)) || (drhs && k && n && m && (!lhs || !dout)))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "matmul_bwd: null pointer");
  cudaStream_t st = as_stream(stream);
  const bool f32 = dtype == BEACON_F32;
  if (dlhs) {  // dlhs[m,k] = dout[m,n] . rhs[k,n]^T   (B stored [N=k][K=n]: K-major)
    GemmParams p = gemm_params(m, k, n, dlhs, k, f32);
    BEACON_TRY(gemm_any(dtype, Operand{dout, false, n}, Operand{rhs, false, n}, p, st));
  }
  if (drhs) {  // drhs[k,n] = lhs[m,k]^T . dout[m,n]  (A stored [K=m][M=k]: MN-major; B [K=m][N=n]: MN-major)
    GemmParams p = gemm_params(k, n, m, drhs, n, f32);
    BEACON_TRY(gemm_any(dtype, Operand{lhs, true, k}, Operand{dout, true, n}, p, st));
  }
  return BEACON_OK;
}

extern "C" int beacon_linear_fwd(void* out, const void* x, const void* weight, const void* bias, int64_t m,
                                 int64_t k, int64_t n, int dtype, void* stream) {
  if (dtype == BEACON_FP8E4M3) return gemm_fp8w(out, x, weight, 1.0f, nullptr, bias, m, k, n, as_stream(stream));
  BEACON_TRY(check_dtype_gemm(dtype));
  BEACON_TRY(check_dims("linear_fwd", m, k, n));
  if (m && n && (!out || (k && (!x || !weight))))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "linear_fwd: null pointer");
  GemmParams p = gemm_params(m, n, k, out, n, dtype == BEACON_F32);
  if (bias) {
    p.epi = kEpiBias;
    p.bias = bias;
  }
  return gemm_any(dtype, Operand{x, false, k}, Operand{weight, true, n}, p, as_stream(stream));
}

extern "C" int beacon_linear_bwd(void* dx, void* dweight, void* dbias, const void* dout, const void* x,
                                 const void* weight, int64_t m, int64_t k, int64_t n, int dtype, void* stream) {
  BEACON_TRY(check_dtype_gemm(dtype));
  BEACON_TRY(check_dims("linear_bwd", m, k, n));
  if (dbias && n > 0 && m > 0 && !dout) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "linear_bwd: null pointer");
  BEACON_TRY(beacon_matmul_bwd(dx, dweight, dout, x, weight, m, k, n, dtype, stream));
  if (dbias && n > 0) {
    int dev;
    DeviceInfo* di;
    BEACON_TRY(current_device(&dev, &di));
    cudaStream_t st = as_stream(stream);
    const int parts = (int)std::min<int64_t>(std::max<int64_t>(m, 1), (int64_t)di->sms * 2);
    void* ws = nullptr;
    BEACON_TRY(get_workspace(dev, (size_t)parts * n * 4, nullptr, 0, &ws));
    float* part = reinterpret_cast<float*>(ws);
    if (dtype == BEACON_F32) {
      k_colsum_partial<float><<<parts, 256, 0, st>>>(part, reinterpret_cast<const float*>(dout), m, (int)n);
      BEACON_TRY(check_launch("k_colsum_partial"));
      k_colsum<float><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(reinterpret_cast<float*>(dbias), part, parts,
                                                                     (int)n);
    } else {
      k_colsum_partial<bf16><<<parts, 256, 0, st>>>(part, reinterpret_cast<const bf16*>(dout), m, (int)n);
      BEACON_TRY(check_launch("k_colsum_partial"));
      k_colsum<bf16><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(reinterpret_cast<bf16*>(dbias), part, parts,
                                                                    (int)n);
    }
    BEACON_TRY(check_launch("k_colsum"));
  }
  return BEACON_OK;
}

// ===========================================================================
// elementwise
// ===========================================================================
extern "C" int beacon_residual_add_fwd(void* out, const void* a, const void* b, int64_t n, int dtype,
                                       void* stream) {
  if (n < 0) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "residual_add: negative n");
  if (n == 0) return BEACON_OK;
  if (dtype != BEACON_BF16 && dtype != BEACON_F32) return fail(BEACON_ERR_UNIMPLEMENTED, "residual_add: dtype %d", dtype);
  if (!out || !a || !b) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "residual_add: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  cudaStream_t st = as_stream(stream);
  const bool vec_ok = aligned16(out) && aligned16(a) && aligned16(b);
  if (dtype == BEACON_BF16) {
    if (!vec_ok) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "residual_add: pointers must be 16-byte aligned");
    k_add_bf16<<<grid_for(n / 8 + 1, 256, di->sms), 256, 0, st>>>(
        reinterpret_cast<bf16*>(out), reinterpret_cast<const bf16*>(a), reinterpret_cast<const bf16*>(b), n);
  } else if (dtype == BEACON_F32) {
    if (!vec_ok) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "residual_add: pointers must be 16-byte aligned");
    k_add_f32<<<grid_for(n / 4 + 1, 256, di->sms), 256, 0, st>>>(
        reinterpret_cast<float*>(out), reinterpret_cast<const float*>(a), reinterpret_cast<const float*>(b), n);
  } else {
    return fail(BEACON_ERR_UNIMPLEMENTED, "residual_add: dtype %d", dtype);
  }
  return check_launch("residual_add_fwd");
}

extern "C" int beacon_residual_add_bwd(void* d_a, void* d_b, const void* d_out, int64_t n, int dtype,
                                       void* stream) {
  if (n < 0) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "residual_add_bwd: negative n");
  if (n == 0) return BEACON_OK;
  if (dtype < 0 || dtype > 3) return fail(BEACON_ERR_UNIMPLEMENTED, "residual_add_bwd: dtype %d", dtype);
  const int es[4] = {4, 2, 2, 1};
  if (!d_out) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "residual_add_bwd: null pointer");
  if (!aligned16(d_out) || (d_a && !aligned16(d_a)) || (d_b && !aligned16(d_b)))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "residual_add_bwd: pointers must be 16-byte aligned");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  const long long nbytes = n * es[dtype];
  k_fanout2<<<grid_for(nbytes / 16 + 1, 256, di->sms), 256, 0, as_stream(stream)>>>(
      reinterpret_cast<uint8_t*>(d_a), reinterpret_cast<uint8_t*>(d_b), reinterpret_cast<const uint8_t*>(d_out),
      nbytes);
  return check_launch("residual_add_bwd");
}

extern "C" int beacon_cast(void* dst, const void* src, int64_t n, int kind, void* stream) {
  if (n < 0) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "cast: negative n");
  if (kind < 0 || kind > 3) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "cast: unknown kind %d", kind);
  if (n == 0) return BEACON_OK;
  if (!dst || !src) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "cast: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  k_cast<<<grid_for(n, 256, di->sms), 256, 0, as_stream(stream)>>>(dst, src, n, kind);
  return check_launch("cast");
}

// ===========================================================================
// embedding lookup / dropout
// ===========================================================================
namespace {
constexpr unsigned int kSiteEmbFwd = 0x601, kSiteEmbBwd = 0x602;

int embedding_check(const char* what, const void* a, const void* b, const void* idx, int64_t tokens, int64_t dim,
                    int64_t vocab, int dtype) {
  if (tokens < 0 || dim <= 0 || dim > INT32_MAX || vocab < 0)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "%s: bad shape tokens=%lld dim=%lld vocab=%lld", what,
                (long long)tokens, (long long)dim, (long long)vocab);
  if (dtype != BEACON_BF16 && dtype != BEACON_F32) return fail(BEACON_ERR_UNIMPLEMENTED, "%s: dtype %d", what, dtype);
  if (tokens > 0 && (!a || !b || !idx)) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "%s: null pointer", what);
  return BEACON_OK;
}
}  // namespace

extern "C" int beacon_embedding_lookup_fwd(void* out, const void* table, const uint32_t* indices, int64_t tokens,
                                           int64_t dim, int64_t vocab, int dtype, void* stream) {
  BEACON_TRY(embedding_check("embedding_lookup_fwd", out, table, indices, tokens, dim, vocab, dtype));
  if (tokens == 0) return BEACON_OK;
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  const int es = dtype == BEACON_F32 ? 4 : 2;
  const int vec = aligned16(out) && aligned16(table) && (dim * es) % 16 == 0;
  const int grid = grid_for(tokens * 32, 256, di->sms);
  if (dtype == BEACON_BF16)
    k_embedding_fwd<bf16><<<grid, 256, 0, as_stream(stream)>>>((bf16*)out, (const bf16*)table, indices, tokens,
                                                                 (int)dim, vocab, vec, kSiteEmbFwd);
  else
    k_embedding_fwd<float><<<grid, 256, 0, as_stream(stream)>>>((float*)out, (const float*)table, indices, tokens,
                                                                  (int)dim, vocab, vec, kSiteEmbFwd);
  return check_launch("k_embedding_fwd");
}

extern "C" int beacon_embedding_lookup_bwd(void* d_table, const void* d_out, const uint32_t* indices, int64_t tokens,
                                           int64_t dim, int64_t vocab, int dtype, void* stream) {
  BEACON_TRY(embedding_check("embedding_lookup_bwd", d_table, d_out, indices, tokens, dim, vocab, dtype));
  if (tokens == 0) return BEACON_OK;
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  const int grid = grid_for(tokens * 32, 256, di->sms);
  if (dtype == BEACON_BF16)
    k_embedding_bwd<bf16><<<grid, 256, 0, as_stream(stream)>>>((bf16*)d_table, (const bf16*)d_out, indices, tokens,
                                                                 (int)dim, vocab, kSiteEmbBwd);
  else
    k_embedding_bwd<float><<<grid, 256, 0, as_stream(stream)>>>((float*)d_table, (const float*)d_out, indices,
                                                                  tokens, (int)dim, vocab, kSiteEmbBwd);
  return check_launch("k_embedding_bwd");
}

extern "C" int beacon_dropout_fwd(void* out, const void* input, void* mask, int64_t n, float p, uint64_t seed,
                                  int dtype, void* stream) {
  if (n < 0 || !(p >= 0.0f)) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "dropout_fwd: n %lld, p %g", (long long)n, p);
  if (dtype != BEACON_BF16 && dtype != BEACON_F32) return fail(BEACON_ERR_UNIMPLEMENTED, "dropout_fwd: dtype %d", dtype);
  if (n == 0) return BEACON_OK;
  if (!out || !input || !mask) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "dropout_fwd: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  if (aligned16(out) && aligned16(mask) && aligned16(input)) {  // eight elements per thread
    const int grid = grid_for((n + 7) / 8, 256, di->sms);
    if (dtype == BEACON_BF16)
      k_dropout_fwd_vec<bf16><<<grid, 256, 0, as_stream(stream)>>>((bf16*)out, (bf16*)mask, (const bf16*)input, n, p,
                                                                   seed);
    else
      k_dropout_fwd_vec<float><<<grid, 256, 0, as_stream(stream)>>>((float*)out, (float*)mask, (const float*)input, n,
                                                                    p, seed);
    return check_launch("k_dropout_fwd_vec");
  }
  const int grid = grid_for(n, 256, di->sms);
  if (dtype == BEACON_BF16)
    k_dropout_fwd<bf16><<<grid, 256, 0, as_stream(stream)>>>((bf16*)out, (bf16*)mask, (const bf16*)input, n, p, seed);
  else
    k_dropout_fwd<float><<<grid, 256, 0, as_stream(stream)>>>((float*)out, (float*)mask, (const float*)input, n, p,
                                                               seed);
  return check_launch("k_dropout_fwd");
}

extern "C" int beacon_dropout_bwd(void* d_in, const void* d_out, const void* mask, int64_t n, int dtype,
                                  void* stream) {
  if (n < 0) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "dropout_bwd: negative n");
  if (dtype != BEACON_BF16 && dtype != BEACON_F32) return fail(BEACON_ERR_UNIMPLEMENTED, "dropout_bwd: dtype %d", dtype);
  if (n == 0) return BEACON_OK;
  if (!d_in || !d_out || !mask) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "dropout_bwd: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  if (aligned16(d_in) && aligned16(d_out) && aligned16(mask)) {  // eight elements per thread
    const int grid = grid_for((n + 7) / 8, 256, di->sms);
    if (dtype == BEACON_BF16)
      k_dropout_bwd_vec<bf16><<<grid, 256, 0, as_stream(stream)>>>((bf16*)d_in, (const bf16*)d_out,
                                                                   (const bf16*)mask, n);
    else
      k_dropout_bwd_vec<float><<<grid, 256, 0, as_stream(stream)>>>((float*)d_in, (const float*)d_out,
                                                                    (const float*)mask, n);
    return check_launch("k_dropout_bwd_vec");
  }
  const int grid = grid_for(n, 256, di->sms);
  if (dtype == BEACON_BF16)
    k_dropout_bwd<bf16><<<grid, 256, 0, as_stream(stream)>>>((bf16*)d_in, (const bf16*)d_out, (const bf16*)mask, n);
  else
    k_dropout_bwd<float><<<grid, 256, 0, as_stream(stream)>>>((float*)d_in, (const float*)d_out, (const float*)mask,
                                                               n);
  return check_launch("k_dropout_bwd");
}

// ===========================================================================
// RMSNorm
// ===========================================================================
extern "C" int beacon_rmsnorm_adjoint_fwd(void* out, const void* x, const void* weight, float* rms,
                                          int64_t tokens, int64_t dim, float eps, int dtype, void* stream) {
  if (tokens < 0 || dim <= 0 || dim > INT32_MAX)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_fwd: bad shape tokens=%lld dim=%lld",
                (long long)tokens, (long long)dim);
  if (dtype != BEACON_BF16 && dtype != BEACON_F32) return fail(BEACON_ERR_UNIMPLEMENTED, "rmsnorm_fwd: dtype %d", dtype);
  if (tokens == 0) return BEACON_OK;
  if (!out || !x || !weight || !rms) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_fwd: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  cudaStream_t st = as_stream(stream);
  const int grid = (int)std::min<int64_t>(tokens, (int64_t)di->sms * 16);
  const bool vec = aligned16(out) && aligned16(x) && aligned16(weight) && dim % 8 == 0;
  const int d = (int)dim;
#define RMS_FWD(T, V) \
  k_rmsnorm_fwd<T, V><<<grid, 256, 0, st>>>((T*)out, rms, (const T*)x, (const T*)weight, tokens, d, eps)
  // an odd count of 256-column chunks above 8 does not split over two warps: the CTA-per-row kernel
  if (dtype == BEACON_BF16 && vec && dim % 256 == 0 && dim <= 4096 && (dim / 256 <= 8 || (dim / 256) % 2 == 0)) {
    // k_rmsnorm_fwd_warp: one warp per row up to 2048 columns, two warps per row above;
    // 8-warp CTAs, at most two per SM by their register use
    const int wpr = dim > 2048 ? 2 : 1;
    const int slots = 8 / wpr;
    const int wgrid = (int)std::min<int64_t>((tokens + slots - 1) / slots, (int64_t)di->sms * 2);
    const bf16 *xb = (const bf16*)x, *wb = (const bf16*)weight;
    bf16* yb = (bf16*)out;
    switch (dim / 256) {
#define RMS_WARP(N, W) \
  case N: k_rmsnorm_fwd_warp<N / W, W><<<wgrid, 256, 0, st>>>(yb, rms, xb, wb, tokens, d, eps); break;
      RMS_WARP(1, 1) RMS_WARP(2, 1) RMS_WARP(3, 1) RMS_WARP(4, 1) RMS_WARP(5, 1) RMS_WARP(6, 1) RMS_WARP(7, 1)
      RMS_WARP(8, 1) RMS_WARP(10, 2) RMS_WARP(12, 2) RMS_WARP(14, 2) RMS_WARP(16, 2)
#undef RMS_WARP
    }
  } else if (dtype == BEACON_BF16) {
    if (vec && dim <= 256 * 8 * 1) RMS_FWD(bf16, 1);
    else if (vec && dim <= 256 * 8 * 2) RMS_FWD(bf16, 2);
    else if (vec && dim <= 256 * 8 * 4) RMS_FWD(bf16, 4);
    else if (vec && dim <= 256 * 8 * 8) RMS_FWD(bf16, 8);
    else k_rmsnorm_fwd_any<bf16><<<grid, 256, 0, st>>>((bf16*)out, rms, (const bf16*)x, (const bf16*)weight, tokens, d, eps);
  } else if (dtype == BEACON_F32) {
    if (vec && dim <= 256 * 8 * 1) RMS_FWD(float, 1);
    else if (vec && dim <= 256 * 8 * 2) RMS_FWD(float, 2);
    else if (vec && dim <= 256 * 8 * 4) RMS_FWD(float, 4);
    else k_rmsnorm_fwd_any<float><<<grid, 256, 0, st>>>((float*)out, rms, (const float*)x, (const float*)weight, tokens, d, eps);
  } else {
    return fail(BEACON_ERR_UNIMPLEMENTED, "rmsnorm_fwd: dtype %d", dtype);
  }
#undef RMS_FWD
  return check_launch("rmsnorm_fwd");
}

extern "C" int beacon_rmsnorm_adjoint_bwd(void* dx, void* dweight, const void* dy, const void* x, const float* rms,
                                          const void* weight, int64_t tokens, int64_t dim, int dtype,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  if (tokens < 0 || dim <= 0 || dim > INT32_MAX)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_bwd: bad shape");
  if (dtype != BEACON_BF16 && dtype != BEACON_F32) return fail(BEACON_ERR_UNIMPLEMENTED, "rmsnorm_bwd: dtype %d", dtype);
  if (tokens > 0 && (!dx || !dy || !x || !rms || !weight))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_bwd: null pointer");
  const bool vec = aligned16(dx) && aligned16(x) && aligned16(dy) && aligned16(weight);
  if (!vec) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_bwd: pointers must be 16-byte aligned");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  cudaStream_t st = as_stream(stream);
  const int es = dtype == BEACON_F32 ? 4 : 2;
  if (tokens == 0) {
    if (dweight) return zero_fill(dweight, (size_t)dim * es, st);
    return BEACON_OK;
  }
  // bf16 rows of 256 x NCH x WPR columns (NCH <= 4; WPR 1, 2 or 4 warps per row, the
  // fewest that fit) up to 4096: one to four warps per row (k_rmsnorm_bwd_warp).
  if (dtype == BEACON_BF16 && dim % 256 == 0 && dim <= 4096) {
    const int nch = (int)(dim / 256);
    const void* fn = nullptr;
    int wpr = 0;
#define RMS_BWD_WARP_PICK(N, W)                                \
  if (!fn && nch == (N) * (W)) {                               \
    fn = (const void*)k_rmsnorm_bwd_warp<N, W>;                \
    wpr = W;                                                   \
  }
    RMS_BWD_WARP_PICK(1, 1) RMS_BWD_WARP_PICK(2, 1) RMS_BWD_WARP_PICK(3, 1) RMS_BWD_WARP_PICK(4, 1)
    RMS_BWD_WARP_PICK(3, 2) RMS_BWD_WARP_PICK(4, 2)
    RMS_BWD_WARP_PICK(3, 4) RMS_BWD_WARP_PICK(4, 4)
#undef RMS_BWD_WARP_PICK
    if (fn) {
      int nb = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, 256, 0) != cudaSuccess || nb <= 0) nb = 2;
      cudaGetLastError();
      const int slots = 8 / wpr;
      const int grid = (int)std::min<int64_t>((tokens + slots - 1) / slots, (int64_t)di->sms * nb);
      float* part = nullptr;
      bool ok = true;
      if (dweight) {
        void* ws = nullptr;
        BEACON_TRY(get_workspace(dev, (size_t)grid * dim * 4, workspace, workspace_bytes, &ws));
        ok = aligned16(ws);
        part = reinterpret_cast<float*>(ws);
      }
      if (ok) {
#define RMS_BWD_WARP(N, W)                                                                                       \
  if (fn == (const void*)k_rmsnorm_bwd_warp<N, W>)                                                               \
    k_rmsnorm_bwd_warp<N, W><<<grid, 256, 0, st>>>((bf16*)dx, part, (const bf16*)dy, (const bf16*)x, rms,        \
                                                   (const bf16*)weight, tokens, (int)dim);
        RMS_BWD_WARP(1, 1) RMS_BWD_WARP(2, 1) RMS_BWD_WARP(3, 1) RMS_BWD_WARP(4, 1)
        RMS_BWD_WARP(3, 2) RMS_BWD_WARP(4, 2)
        RMS_BWD_WARP(3, 4) RMS_BWD_WARP(4, 4)
#undef RMS_BWD_WARP
        BEACON_TRY(check_launch("rmsnorm_bwd"));
        if (dweight) {
          k_colsum_split2<bf16><<<dim3((unsigned)((dim + 31) / 32), 1), 256, 0, st>>>((bf16*)dweight, part, nullptr,
                                                                                      nullptr, grid, (int)dim);
          BEACON_TRY(check_launch("rmsnorm_bwd colsum"));
        }
        return BEACON_OK;
      }
    }
  }
  // Register-resident rows (k_rmsnorm_bwd_rows) up to 8192 bf16 / 4096 f32 columns;
  // beyond that, for dim % 8 != 0 or with a misaligned workspace, k_rmsnorm_bwd.
  int rows_vec = 0;
  if (dim % 8 == 0) {
    if (dim <= 256 * 8) rows_vec = 1;
    else if (dim <= 256 * 8 * 2) rows_vec = 2;
    else if (dim <= 256 * 8 * 4 && dtype == BEACON_BF16) rows_vec = 4;
  }
  const void* rows_fn = nullptr;
  if (rows_vec == 1) rows_fn = dtype == BEACON_BF16 ? (const void*)k_rmsnorm_bwd_rows<bf16, 1>
                                                    : (const void*)k_rmsnorm_bwd_rows<float, 1>;
  if (rows_vec == 2) rows_fn = dtype == BEACON_BF16 ? (const void*)k_rmsnorm_bwd_rows<bf16, 2>
                                                    : (const void*)k_rmsnorm_bwd_rows<float, 2>;
  if (rows_vec == 4) rows_fn = (const void*)k_rmsnorm_bwd_rows<bf16, 4>;
  int per_sm = 4;  // resident CTAs per SM for the grid (one wave)
  if (rows_fn) {
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, rows_fn, 256, 0) == cudaSuccess && nb > 0) per_sm = nb;
    cudaGetLastError();
  }
  const int grid = (int)std::min<int64_t>(tokens, (int64_t)di->sms * per_sm);
  float* part = nullptr;
  if (dweight) {
    void* ws = nullptr;
    BEACON_TRY(get_workspace(dev, (size_t)grid * dim * 4, workspace, workspace_bytes, &ws));
    if (!aligned16(ws)) rows_fn = nullptr;
    part = reinterpret_cast<float*>(ws);
  }
#define RMS_BWD_ROWS(T, V)                                                                                  \
  k_rmsnorm_bwd_rows<T, V><<<grid, 256, 0, st>>>((T*)dx, part, (const T*)dy, (const T*)x, rms, (const T*)weight, \
                                                 tokens, (int)dim)
  if (dtype == BEACON_BF16) {
    if (rows_fn && rows_vec == 1) RMS_BWD_ROWS(bf16, 1);
    else if (rows_fn && rows_vec == 2) RMS_BWD_ROWS(bf16, 2);
    else if (rows_fn && rows_vec == 4) RMS_BWD_ROWS(bf16, 4);
    else
      k_rmsnorm_bwd<bf16><<<grid, 256, 0, st>>>((bf16*)dx, part, (const bf16*)dy, (const bf16*)x, rms,
                                                (const bf16*)weight, tokens, (int)dim);
    BEACON_TRY(check_launch("rmsnorm_bwd"));
    if (dweight)
      k_colsum_split2<bf16><<<dim3((unsigned)((dim + 31) / 32), 1), 256, 0, st>>>((bf16*)dweight, part, nullptr,
                                                                                  nullptr, grid, (int)dim);
  } else {
    if (rows_fn && rows_vec == 1) RMS_BWD_ROWS(float, 1);
    else if (rows_fn && rows_vec == 2) RMS_BWD_ROWS(float, 2);
    else
      k_rmsnorm_bwd<float><<<grid, 256, 0, st>>>((float*)dx, part, (const float*)dy, (const float*)x, rms,
                                                 (const float*)weight, tokens, (int)dim);
    BEACON_TRY(check_launch("rmsnorm_bwd"));
    if (dweight)
      k_colsum_split2<float><<<dim3((unsigned)((dim + 31) / 32), 1), 256, 0, st>>>((float*)dweight, part, nullptr,
                                                                                   nullptr, grid, (int)dim);
  }
#undef RMS_BWD_ROWS
  if (dweight) BEACON_TRY(check_launch("rmsnorm_bwd colsum"));
  return BEACON_OK;
}

// ===========================================================================
// RMSNorm folded into the GEMM that follows it
//   rmsnorm(x, g) . W = diag(1 / rms) . x . (diag(g) . W)
// The gain is folded into W's rows once per weight version (beacon_rmsnorm_fold_weight);
// each call then runs one row-statistics pass over x (k_rms_stats: reads x, writes rms)
// and the GEMM on raw x with 1 / rms applied to the accumulator in its epilogue, instead
// of writing and re-reading a normalised copy of x.
// ===========================================================================
namespace {

int rms_stats(float* rms, float* sumsq, const void* x, int64_t T, int64_t dim, float eps, int dtype, int sms,
              cudaStream_t st) {
  const int grid = (int)std::min<int64_t>((T + 7) / 8, (int64_t)sms * 16);
  const int vec = aligned16(x) && dim % 8 == 0;
  if (dtype == BEACON_BF16)
    k_rms_stats<bf16><<<grid, 256, 0, st>>>(rms, sumsq, (const bf16*)x, T, (int)dim, eps, vec);
  else
    k_rms_stats<float><<<grid, 256, 0, st>>>(rms, sumsq, (const float*)x, T, (int)dim, eps, vec);
  return check_launch("k_rms_stats");
}

}  // namespace

extern "C" int beacon_rmsnorm_fold_weight(void* w_out, const void* gain, const void* w, int64_t k, int64_t n,
                                          int dtype, void* stream) {
  BEACON_TRY(check_dims("rmsnorm_fold_weight", k, n, 1));
  if (dtype != BEACON_BF16 && dtype != BEACON_F32)
    return fail(BEACON_ERR_UNIMPLEMENTED, "rmsnorm_fold_weight: dtype %d", dtype);
  if (k == 0 || n == 0) return BEACON_OK;
  if (!w_out || !gain || !w) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_fold_weight: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  const int grid = grid_for(k * n, 256, di->sms);
  if (dtype == BEACON_BF16)
    k_fold_gain<bf16><<<grid, 256, 0, as_stream(stream)>>>((bf16*)w_out, (const bf16*)gain, (const bf16*)w, k, n);
  else
    k_fold_gain<float><<<grid, 256, 0, as_stream(stream)>>>((float*)w_out, (const float*)gain, (const float*)w, k,
                                                            n);
  return check_launch("k_fold_gain");
}

extern "C" int beacon_rmsnorm_linear_fwd(void* out, float* rms, const void* x, const void* w_folded,
                                         const void* bias, int64_t m, int64_t k, int64_t n, float eps, int dtype,
                                         void* stream) {
  BEACON_TRY(check_dtype_gemm(dtype));
  BEACON_TRY(check_dims("rmsnorm_linear_fwd", m, k, n));
  if (k == 0) return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_linear_fwd: k (the normalised width) is 0");
  if (m == 0) return BEACON_OK;
  if (!rms || !x || (n && (!out || !w_folded)))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_linear_fwd: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  cudaStream_t st = as_stream(stream);
  BEACON_TRY(rms_stats(rms, nullptr, x, m, k, eps, dtype, di->sms, st));
  if (n == 0) return BEACON_OK;
  GemmParams p = gemm_params(m, n, k, out, n, dtype == BEACON_F32);
  p.row_rms = rms;
  if (bias) {
    p.epi = kEpiBias;
    p.bias = bias;
  }
  return gemm_any(dtype, Operand{x, false, k}, Operand{w_folded, true, n}, p, st);
}

// ===========================================================================
// LayerNorm
// ===========================================================================
extern "C" int beacon_layernorm_adjoint_fwd(void* out, const void* x, const void* weight, const void* bias,
                                            float* mean, float* invstd, int64_t tokens, int64_t dim, float eps,
                                            int dtype, void* stream) {
  if (tokens < 0 || dim <= 0 || dim > INT32_MAX)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "layernorm_fwd: bad shape tokens=%lld dim=%lld",
                (long long)tokens, (long long)dim);
  if (dtype != BEACON_BF16 && dtype != BEACON_F32)
    return fail(BEACON_ERR_UNIMPLEMENTED, "layernorm_fwd: dtype %d", dtype);
  if (tokens == 0) return BEACON_OK;
  if (!out || !x || !weight || !bias || !mean || !invstd)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "layernorm_fwd: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  cudaStream_t st = as_stream(stream);
  const int grid = (int)std::min<int64_t>(tokens, (int64_t)di->sms * 16);
  const bool vec = aligned16(out) && aligned16(x) && aligned16(weight) && aligned16(bias) && dim % 8 == 0;
  const int d = (int)dim;
#define LN_FWD(T, V)                                                                                          \
  k_layernorm_fwd<T, V><<<grid, 256, 0, st>>>((T*)out, mean, invstd, (const T*)x, (const T*)weight,           \
                                              (const T*)bias, tokens, d, eps)
#define LN_FWD_ANY(T)                                                                                         \
  k_layernorm_fwd_any<T><<<grid, 256, 0, st>>>((T*)out, mean, invstd, (const T*)x, (const T*)weight,          \
                                               (const T*)bias, tokens, d, eps)
  const bool warp_rows = dtype == BEACON_BF16 && vec && dim % 256 == 0 && dim <= 4096 && (dim / 256 <= 8 ||
                                                                                            (dim / 256) % 2 == 0);
  if (warp_rows) {
    // k_layernorm_fwd_warp: one warp per row up to 2048 columns, two warps per row above
    const int wpr = dim > 2048 ? 2 : 1;
    const int slots = 8 / wpr;
    const int wgrid = (int)std::min<int64_t>((tokens + slots - 1) / slots, (int64_t)di->sms * 2);
    const bf16 *xb = (const bf16*)x, *wb = (const bf16*)weight, *bb = (const bf16*)bias;
    bf16* yb = (bf16*)out;
    switch (dim / 256) {
#define LN_WARP(N, W) \
  case N: k_layernorm_fwd_warp<N / W, W><<<wgrid, 256, 0, st>>>(yb, mean, invstd, xb, wb, bb, tokens, d, eps); break;
      LN_WARP(1, 1) LN_WARP(2, 1) LN_WARP(3, 1) LN_WARP(4, 1) LN_WARP(5, 1) LN_WARP(6, 1) LN_WARP(7, 1)
      LN_WARP(8, 1) LN_WARP(10, 2) LN_WARP(12, 2) LN_WARP(14, 2) LN_WARP(16, 2)
#undef LN_WARP
    }
  } else if (dtype == BEACON_BF16) {
    if (vec && dim <= 256 * 8 * 1) LN_FWD(bf16, 1);
    else if (vec && dim <= 256 * 8 * 2) LN_FWD(bf16, 2);
    else if (vec && dim <= 256 * 8 * 4) LN_FWD(bf16, 4);
    else if (vec && dim <= 256 * 8 * 8) LN_FWD(bf16, 8);
    else LN_FWD_ANY(bf16);
  } else {
    if (vec && dim <= 256 * 8 * 1) LN_FWD(float, 1);
    else if (vec && dim <= 256 * 8 * 2) LN_FWD(float, 2);
    else if (vec && dim <= 256 * 8 * 4) LN_FWD(float, 4);
    else LN_FWD_ANY(float);
  }
#undef LN_FWD
#undef LN_FWD_ANY
  return check_launch("layernorm_fwd");
}

extern "C" int beacon_layernorm_adjoint_bwd(void* dx, void* dweight, void* dbias, const void* dy, const void* x,
                                            const float* mean, const float* invstd, const void* weight,
                                            int64_t tokens, int64_t dim, int dtype, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  if (tokens < 0 || dim <= 0 || dim > INT32_MAX)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "layernorm_bwd: bad shape tokens=%lld dim=%lld",
                (long long)tokens, (long long)dim);
  if (dtype != BEACON_BF16 && dtype != BEACON_F32)
    return fail(BEACON_ERR_UNIMPLEMENTED, "layernorm_bwd: dtype %d", dtype);
  if (tokens > 0 && (!dx || !dy || !x || !mean || !invstd || !weight))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "layernorm_bwd: null pointer");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  cudaStream_t st = as_stream(stream);
  const int es = dtype == BEACON_F32 ? 4 : 2;
  if (tokens == 0) {  // empty sums
    if (dweight) BEACON_TRY(zero_fill(dweight, (size_t)dim * es, st));
    if (dbias) BEACON_TRY(zero_fill(dbias, (size_t)dim * es, st));
    return BEACON_OK;
  }
  const bool vec = aligned16(dx) && aligned16(dy) && aligned16(x) && aligned16(weight) && dim % 8 == 0;
  // Register-resident rows (k_layernorm_bwd_rows) up to 8192 bf16 / 4096 f32 columns;
  // beyond that, or with a misaligned workspace, the partials go through global memory.
  int rows_vec = 0;
  if (vec) {
    if (dim <= 256 * 8) rows_vec = 1;
    else if (dim <= 256 * 8 * 2) rows_vec = 2;
    else if (dim <= 256 * 8 * 4 && dtype == BEACON_BF16) rows_vec = 4;
  }
  const void* rows_fn = nullptr;
  if (rows_vec == 1) rows_fn = dtype == BEACON_BF16 ? (const void*)k_layernorm_bwd_rows<bf16, 1>
                                                    : (const void*)k_layernorm_bwd_rows<float, 1>;
  if (rows_vec == 2) rows_fn = dtype == BEACON_BF16 ? (const void*)k_layernorm_bwd_rows<bf16, 2>
                                                    : (const void*)k_layernorm_bwd_rows<float, 2>;
  if (rows_vec == 4) rows_fn = (const void*)k_layernorm_bwd_rows<bf16, 4>;
  int per_sm = 4;  // resident CTAs per SM for the grid (one wave)
  if (rows_fn) {
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, rows_fn, 256, 0) == cudaSuccess && nb > 0) per_sm = nb;
    cudaGetLastError();
  }
  const int grid = (int)std::min<int64_t>(tokens, (int64_t)di->sms * per_sm);
  const size_t part_bytes = (size_t)grid * dim * 4;
  const int nparts = (dweight ? 1 : 0) + (dbias ? 1 : 0);
  float *part_w = nullptr, *part_b = nullptr;
  if (nparts) {
    void* ws = nullptr;
    BEACON_TRY(get_workspace(dev, part_bytes * nparts, workspace, workspace_bytes, &ws));
    if (!aligned16(ws)) rows_fn = nullptr;
    float* p = reinterpret_cast<float*>(ws);
    if (dweight) part_w = p, p += (size_t)grid * dim;
    if (dbias) part_b = p;
  }
  const dim3 cgrid((unsigned)((dim + 31) / 32), 2);
#define LN_BWD_ROWS(T, V)                                                                                       \
  k_layernorm_bwd_rows<T, V><<<grid, 256, 0, st>>>((T*)dx, part_w, part_b, (const T*)dy, (const T*)x, mean,     \
                                                   invstd, (const T*)weight, tokens, (int)dim)
  if (dtype == BEACON_BF16) {
    if (rows_fn && rows_vec == 1) LN_BWD_ROWS(bf16, 1);
    else if (rows_fn && rows_vec == 2) LN_BWD_ROWS(bf16, 2);
    else if (rows_fn && rows_vec == 4) LN_BWD_ROWS(bf16, 4);
    else
      k_layernorm_bwd<bf16><<<grid, 256, 0, st>>>((bf16*)dx, part_w, part_b, (const bf16*)dy, (const bf16*)x, mean,
                                                  invstd, (const bf16*)weight, tokens, (int)dim, vec);
    BEACON_TRY(check_launch("layernorm_bwd"));
    if (nparts)
      k_colsum_split2<bf16><<<cgrid, 256, 0, st>>>((bf16*)dweight, part_w, (bf16*)dbias, part_b, grid, (int)dim);
  } else {
    if (rows_fn && rows_vec == 1) LN_BWD_ROWS(float, 1);
    else if (rows_fn && rows_vec == 2) LN_BWD_ROWS(float, 2);
    else
      k_layernorm_bwd<float><<<grid, 256, 0, st>>>((float*)dx, part_w, part_b, (const float*)dy, (const float*)x,
                                                   mean, invstd, (const float*)weight, tokens, (int)dim, vec);
    BEACON_TRY(check_launch("layernorm_bwd"));
    if (nparts)
      k_colsum_split2<float><<<cgrid, 256, 0, st>>>((float*)dweight, part_w, (float*)dbias, part_b, grid, (int)dim);
  }
  if (nparts) BEACON_TRY(check_launch("layernorm_bwd colsum"));
#undef LN_BWD_ROWS
  return BEACON_OK;
}

// ===========================================================================
// RMSNorm backward without any allocation.
//
// For callers that cannot allocate device memory on their own: a launcher that
// hands out only pointers into one preallocated arena (the reference's model,
// crates/beacon-core/src/arena.rs), a latency-critical path where a first-call
// cudaMalloc and its device synchronisation are not acceptable, or a host under
// an allocator that forbids allocations it does not see.  beacon_rmsnorm_adjoint_bwd
// takes a workspace from the caller or grows its own with cudaMalloc; this variant
// keeps the dweight partial sums in a fixed array compiled into the library.
//
// The array is a file-scope __device__ buffer of kNoAllocScratchFloats floats
// (4 MiB).  Every GPU that loads this library holds it until the process exits.
// Its address is looked up once per device, on the first call made with that
// device current (cudaGetSymbolAddress); make that first call before any stream
// capture.  All calls share the one array and it keeps the last call's contents:
// each CTA zeroes its own partial row before accumulating, so nothing carries
// over, but two calls that overlap on the GPU (different streams, or different
// host threads on one device) race on it and must be serialised by the caller.
// ===========================================================================
namespace {

constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;  // 4 MiB
static __device__ __align__(256) float g_rmsnorm_bwd_scratch[kNoAllocScratchFloats];

std::mutex g_noalloc_mu;
float* g_noalloc_ptr[64] = {};

int noalloc_scratch(int dev, float** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_rmsnorm_bwd_scratch);  // device `dev` is current
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return fail(BEACON_ERR_CUDA, "rmsnorm_bwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = reinterpret_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return BEACON_OK;
}

}  // namespace

extern "C" int beacon_rmsnorm_adjoint_bwd_noalloc(void* dx, void* dweight, const void* dy, const void* x,
                                                  const float* rms, const void* weight, int64_t tokens, int64_t dim,
                                                  int dtype, void* stream) {
  if (tokens < 0 || dim <= 0 || dim > INT32_MAX)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_bwd_noalloc: bad shape");
  if ((size_t)dim > kNoAllocScratchFloats)
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG,
                "rmsnorm_bwd_noalloc: dim %lld exceeds the fixed scratch of %zu floats (4 MiB); "
                "use beacon_rmsnorm_adjoint_bwd with a workspace",
                (long long)dim, kNoAllocScratchFloats);
  if (dtype != BEACON_BF16 && dtype != BEACON_F32)
    return fail(BEACON_ERR_UNIMPLEMENTED, "rmsnorm_bwd_noalloc: dtype %d", dtype);
  if (tokens > 0 && (!dx || !dy || !x || !rms || !weight))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_bwd_noalloc: null pointer");
  if (!(aligned16(dx) && aligned16(x) && aligned16(dy) && aligned16(weight)))
    return fail(BEACON_ERR_INVALID_LAUNCH_CONFIG, "rmsnorm_bwd_noalloc: pointers must be 16-byte aligned");
  int dev;
  DeviceInfo* di;
  BEACON_TRY(current_device(&dev, &di));
  cudaStream_t st = as_stream(stream);
  if (tokens == 0) {  // empty batch: dweight = 0 (a memset, no allocation)
    if (dweight) return zero_fill(dweight, (size_t)dim * (dtype == BEACON_F32 ? 4 : 2), st);
    return BEACON_OK;
  }
  // partial rows: as many CTAs as the fixed scratch holds rows of `dim` floats
  const int64_t cap_rows = (int64_t)(kNoAllocScratchFloats / (size_t)dim);
  const int grid = (int)std::min<int64_t>(std::min<int64_t>(tokens, (int64_t)di->sms * 4), cap_rows);
  float* part = nullptr;
  if (dweight) BEACON_TRY(noalloc_scratch(dev, &part));
  if (dtype == BEACON_BF16) {
    k_rmsnorm_bwd<bf16><<<grid, 256, 0, st>>>((bf16*)dx, part, (const bf16*)dy, (const bf16*)x, rms,
                                              (const bf16*)weight, tokens, (int)dim);
    BEACON_TRY(check_launch("rmsnorm_bwd_noalloc"));
    if (dweight) k_colsum<bf16><<<(unsigned)((dim + 255) / 256), 256, 0, st>>>((bf16*)dweight, part, grid, (int)dim);
  } else {
    k_rmsnorm_bwd<float><<<grid, 256, 0, st>>>((float*)dx, part, (const float*)dy, (const float*)x, rms,
                                               (const float*)weight, tokens, (int)dim);
    BEACON_TRY(check_launch("rmsnorm_bwd_noalloc"));
    if (dweight) k_colsum<float><<<(unsigned)((dim + 255) / 256), 256, 0, st>>>((float*)dweight, part, grid, (int)dim);
  }
  if (dweight) BEACON_TRY(check_launch("rmsnorm_bwd_noalloc colsum"));
  return BEACON_OK;
}

#include "abi_attention.inc"
#include "abi_swiglu.inc"
#include "abi_block.inc"
#include "abi_arena.inc"
