// libsandmuon_b200.cu -- host runtime and C-ABI of the SandMuon B200 engine.
//
// One translation unit: the kernels (sm_gemm.cuh, sm_kernels.cuh), the plan
// executor that sequences a whole optimizer step from a single C call, and the
// extern "C" entry points declared in include/sandmuon_b200.h.
//
// Memory: the library allocates nothing on the device.  Callers pass every
// buffer; a plan carves its workspace into per-shape-group buffers:
//   xh|xl  BF16 [B, rp, cp] x2  hi/lo planes of the S8 iterate: stages 1, 3, 5
//                               read it (stage 5 reads the hi plane only)
//   xa|xb  BF16 [B, rp, cp] x2  hi/lo planes of the iterate of stages 2 and 4;
//                               the S8 output Q (BF16 [B, rp, cp]) reuses the
//                               xa plane
//   gh, gl BF16 [B, rp, rp]     stage 1: gram hi/lo, then P hi/lo in place;
//                               stages 2-4: shifted gram H = G + beta I hi/lo;
//                               stage 5: gh = H, gl = polynomial P
//   g2     FP32 [B, rp, rp]     stage-1 gram^2; stages 2-4: P hi/lo planes
//   + per-row float2 statistics, per-tile partial sums, per-matrix scalars.
// rp, cp are the oriented rows/cols (rows <= cols) padded to multiples of 128;
// padding is zeroed at plan creation and stays zero through every stage.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <queue>
#include <string>
#include <vector>

#include "sm_common.cuh"
#include "sm_gemm.cuh"
#include "sm_kernels.cuh"

namespace smb {

// S8 constants (sandmuon/coefficients.py:3-10).
constexpr float kS8Margin = 1.35f;
constexpr double kS8Coeff[5][3] = {
    {11.062126275847973, -56.051653229128085, 72.32081107619855},
    {4.100720073616268, -2.9324183165353577, 0.5339692084282731},
    {3.930310192522361, -2.873509793709714, 0.5366557527206212},
    {3.280567968245866, -2.414925589994015, 0.48635134757825227},
    {2.282741575232451, -1.6302296637355072, 0.40275720810675486},
};

thread_local std::string t_last_error;

static int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

#define SM_CUDA(call)                                                                       \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) return fail(SM_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

#define SM_LAUNCHED()                                                                        \
  do {                                                                                       \
    cudaError_t e_ = cudaGetLastError();                                                     \
    if (e_ != cudaSuccess) return fail(SM_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e_)); \
  } while (0)

#define SM_TRY(expr)          \
  do {                        \
    int rc_ = (expr);         \
    if (rc_ != SM_OK) return rc_; \
  } while (0)

// Launches issued while t_pdl is set (the kernels of an optimizer step after
// its first) carry the programmatic-stream-serialization attribute: each may
// start launching while its predecessor drains, and waits in grid_dep_wait()
// before it reads or writes global memory.
thread_local bool t_pdl = false;

struct PdlScope {
  bool saved;
  explicit PdlScope(bool on) : saved(t_pdl) { t_pdl = on; }
  ~PdlScope() { t_pdl = saved; }
};

// Fills `attrs` with the attributes of the current launch mode plus an
// optional cluster of `cluster` CTAs; returns how many were written.
static unsigned launch_attrs(cudaLaunchAttribute* attrs, int cluster) {
  unsigned n = 0;
  if (cluster > 1) {
    memset(&attrs[n], 0, sizeof(attrs[n]));
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = static_cast<unsigned>(cluster);
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = 1;
    ++n;
  }
  if (t_pdl) {
    memset(&attrs[n], 0, sizeof(attrs[n]));
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  return n;
}

template <typename... KArgs, typename... Args>
static int launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                         Args... args) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cudaLaunchAttribute attrs[2];
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attrs;
  cfg.numAttrs = launch_attrs(attrs, 1);
  SM_CUDA(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
  return SM_OK;
}

static inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
static inline int64_t round_up(int64_t a, int64_t b) { return cdiv(a, b) * b; }

// ------------------------------------------------------------ device info

struct DeviceInfo {
  int sms = 0;
  bool attrs_set = false;
  int pair_workers = -1;  // CTA pairs of the GEMM that can be resident at once (0: no pair mode)
};
static std::mutex g_dev_mutex;
static DeviceInfo g_dev[64];

static int current_device_info(DeviceInfo** out) {
  int dev = 0;
  SM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(SM_ERR_UNSUPPORTED, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  DeviceInfo& d = g_dev[dev];
  if (d.sms == 0) {
    int major = 0, minor = 0;
    SM_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    SM_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (major != 10 || minor != 0)
      return fail(SM_ERR_UNSUPPORTED, "libsandmuon_b200 requires an sm_100 (B200) GPU; found sm_" +
                                          std::to_string(major) + std::to_string(minor));
    SM_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
  }
  *out = &d;
  return SM_OK;
}

// ------------------------------------------------------------- tensor maps

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_encode(PFN_cuTensorMapEncodeTiled_v12000* out) {
  static std::once_flag once;
  static int status = SM_OK;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
      status = SM_ERR_UNSUPPORTED;
    } else {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  if (status != SM_OK) return fail(status, "cuTensorMapEncodeTiled is unavailable");
  *out = g_encode;
  return SM_OK;
}

// 3-D BF16 tensor [batch, outer, inner] (inner contiguous), box
// {64, box_outer, 1} with the 128-byte swizzle (one box row = 128 bytes).
// inner * 2 bytes must be a multiple of 16.
static int make_map(CUtensorMap* m, const void* base, int64_t inner, int64_t outer, int64_t batch,
                    uint32_t box_inner, uint32_t box_outer) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  SM_TRY(get_encode(&enc));
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return fail(SM_ERR_ARG, "TMA base not 16-byte aligned");
  if ((inner * 2) % 16 != 0) return fail(SM_ERR_ARG, "TMA row stride not a multiple of 16 bytes");
  if (box_inner != 64) return fail(SM_ERR_ARG, "TMA box inner extent must be 64 (128-byte swizzle)");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(inner * 2), static_cast<cuuint64_t>(inner * outer * 2)};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapSwizzle swz = box_inner == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SM_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return SM_OK;
}

// ------------------------------------------------------------ GEMM launch

// K extent of one pipeline stage: 64 BF16 = 128-byte rows with the 128-byte
// swizzle (measured faster per MMA than 32 / 64-byte rows).  The ring holds as
// many stages as fit next to the epilogue staging: BN=256 compensated 2 x 96 KB,
// BN=128 compensated 3 x 64 KB, plain 4 x 48 KB or 6 x 32 KB.  The SMB_*
// macros exist for tuning sweeps; the defaults are the shipped configuration.
#ifndef SMB_COMP_STAGES
#define SMB_COMP_STAGES 8
#endif
#ifndef SMB_PLAIN_STAGES
#define SMB_PLAIN_STAGES 8
#endif
#ifndef SMB_BN_MAX
#define SMB_BN_MAX 256
#endif
#ifndef SMB_USE_SCHEDULE
#define SMB_USE_SCHEDULE 1
#endif
// S8 GEMMs of groups whose padded row count is a multiple of 256 run on CTA
// pairs (256-row tiles, tcgen05 cta_group::2).
#ifndef SMB_PAIR
#define SMB_PAIR 1
#endif
// Every operand tile uses the 128-byte swizzle and 64-deep k-blocks (measured:
// 32-deep stages, with twice as many in the ring, are 10-30% slower, and an
// MN-major A reads no faster than a K-major one).  The ring holds as many
// stages as fit next to the epilogue staging.  The SMB_* macros exist for
// tuning sweeps; the defaults are the shipped configuration.
constexpr int kBkK = 64;   // every launch of the S8 path (K-major A)
constexpr int kBkMN = 64;  // launches whose A and B are both MN-major (unit tests)
constexpr uint32_t kChunk = Swz::kChunkElems;

// Ring depth of a configuration: the configured depth, capped by what fits in
// 227 KB of shared memory next to the epilogue staging.
template <int BN, int BK, bool COMP, int CG>
struct GemmConfig {
  static constexpr int kStageBytes = GemmSmem<BN, BK, COMP, 1, CG>::kStageBytes;
  static constexpr int kFit = (232448 - 1024 - 256 - GemmSmem<BN, BK, COMP, 1, CG>::kStagingBytes) / kStageBytes;
  static constexpr int kWant = COMP ? SMB_COMP_STAGES : SMB_PLAIN_STAGES;
  static constexpr int kStages = kWant < kFit ? kWant : kFit;
  using S = GemmSmem<BN, BK, COMP, kStages, CG>;
  static_assert(S::kTotal <= 232448, "shared memory budget");
};

template <int BN, int BK, bool COMP, bool A_MN, bool B_MN, int EPI, int CG>
static int gemm_kernel(void (**out)(GemmLaunch), int* smem_bytes) {
  using C = GemmConfig<BN, BK, COMP, CG>;
  auto kern = k_gemm_bf16<BN, BK, COMP, A_MN, B_MN, C::kStages, EPI, CG>;
  static bool attr_done[64] = {};
  int dev = 0;
  SM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(SM_ERR_UNSUPPORTED, "device ordinal out of range");
  if (!attr_done[dev]) {
    SM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::S::kTotal));
    attr_done[dev] = true;
  }
  *out = kern;
  *smem_bytes = C::S::kTotal;
  return SM_OK;
}

// `attr` holds room for two attributes: the pair cluster and, in a plan
// step, programmatic serialisation.
static void pair_launch_config(cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr, int grid, int smem,
                               cudaStream_t st) {
  memset(cfg, 0, sizeof(*cfg));
  cfg->gridDim = dim3(static_cast<unsigned>(grid));
  cfg->blockDim = dim3(kGemmThreads);
  cfg->dynamicSmemBytes = static_cast<size_t>(smem);
  cfg->stream = st;
  cfg->attrs = attr;
  cfg->numAttrs = launch_attrs(attr, 2);
}

template <int BN, int BK, bool COMP, bool A_MN, bool B_MN, int EPI, int CG>
static int launch_gemm_t(const GemmLaunch& L, int grid, cudaStream_t st) {
  void (*kern)(GemmLaunch);
  int smem = 0;
  SM_TRY((gemm_kernel<BN, BK, COMP, A_MN, B_MN, EPI, CG>(&kern, &smem)));
  if (L.total_tiles == 0 || grid == 0) return SM_OK;
  if (CG == 1) {
    SM_TRY(launch_kernel(kern, dim3(grid), dim3(kGemmThreads), static_cast<size_t>(smem), st, L));
  } else {
    if (grid % 2 != 0) return fail(SM_ERR_ARG, "a CTA-pair GEMM needs an even grid");
    cudaLaunchConfig_t cfg;
    cudaLaunchAttribute attr[2];
    pair_launch_config(&cfg, attr, grid, smem, st);
    SM_CUDA(cudaLaunchKernelEx(&cfg, kern, L));
  }
  SM_LAUNCHED();
  return SM_OK;
}

// How many CTA pairs of the GEMM can be resident at once on this device (one
// CTA per SM; pairs are placed within a GPC, so this can be below sms / 2).
// Every pair configuration holds one CTA per SM, so the largest stands for all.
static int pair_workers(DeviceInfo* di, int* out) {
  if (di->pair_workers < 0) {
    int n = 0;
    if (SMB_PAIR) {
      void (*kern)(GemmLaunch);
      int smem = 0;
      SM_TRY((gemm_kernel<256, 64, true, false, false, kEpiF32, 2>(&kern, &smem)));
      cudaLaunchConfig_t cfg;
      cudaLaunchAttribute attr[2];
      PdlScope plain(false);
      pair_launch_config(&cfg, attr, 2 * std::max(1, di->sms / 2), smem, nullptr);
      SM_CUDA(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    }
    di->pair_workers = std::max(0, n);
  }
  *out = di->pair_workers;
  return SM_OK;
}

// Operand layouts: 0 = A and B K-major; 1 = A K-major, B MN-major; 2 = both MN-major.
enum GemmLayout : int { kLayoutKK = 0, kLayoutKM = 1, kLayoutMM = 2 };

template <int BN, int CG>
static int dispatch_gemm_bn(bool comp, int layout, int epi, const GemmLaunch& L, int grid, cudaStream_t st) {
  if (layout == kLayoutKK) {
    if (comp) {
      switch (epi) {
        case kEpiF32: return launch_gemm_t<BN, kBkK, true, false, false, kEpiF32, CG>(L, grid, st);
        case kEpiBF16: return launch_gemm_t<BN, kBkK, true, false, false, kEpiBF16, CG>(L, grid, st);
        case kEpiHiLo: return launch_gemm_t<BN, kBkK, true, false, false, kEpiHiLo, CG>(L, grid, st);
        case kEpiF32Norm: return launch_gemm_t<BN, kBkK, true, false, false, kEpiF32Norm, CG>(L, grid, st);
        case kEpiPolyHiLo: return launch_gemm_t<BN, kBkK, true, false, false, kEpiPolyHiLo, CG>(L, grid, st);
        default: break;
      }
    } else {
      switch (epi) {
        case kEpiF32: return launch_gemm_t<BN, kBkK, false, false, false, kEpiF32, CG>(L, grid, st);
        case kEpiBF16: return launch_gemm_t<BN, kBkK, false, false, false, kEpiBF16, CG>(L, grid, st);
        case kEpiPoly: return launch_gemm_t<BN, kBkK, false, false, false, kEpiPoly, CG>(L, grid, st);
        default: break;
      }
    }
  } else if (layout == kLayoutKM) {
    if (comp) {
      switch (epi) {
        case kEpiF32: return launch_gemm_t<BN, kBkK, true, false, true, kEpiF32, CG>(L, grid, st);
        case kEpiBF16: return launch_gemm_t<BN, kBkK, true, false, true, kEpiBF16, CG>(L, grid, st);
        case kEpiHiLo: return launch_gemm_t<BN, kBkK, true, false, true, kEpiHiLo, CG>(L, grid, st);
        default: break;
      }
    } else {
      switch (epi) {
        case kEpiF32: return launch_gemm_t<BN, kBkK, false, false, true, kEpiF32, CG>(L, grid, st);
        case kEpiBF16: return launch_gemm_t<BN, kBkK, false, false, true, kEpiBF16, CG>(L, grid, st);
        default: break;
      }
    }
  } else if (layout == kLayoutMM && CG == 1) {
    if (epi == kEpiF32) {
      return comp ? launch_gemm_t<BN, kBkMN, true, true, true, kEpiF32, CG>(L, grid, st)
                  : launch_gemm_t<BN, kBkMN, false, true, true, kEpiF32, CG>(L, grid, st);
    }
  }
  return fail(SM_ERR_ARG, "unsupported GEMM mode combination (compensated=" + std::to_string(comp) +
                              ", layout=" + std::to_string(layout) + ", epilogue=" + std::to_string(epi) +
                              ", cta pair=" + std::to_string(CG == 2) + ")");
}

static int dispatch_gemm(int bn, int cg, bool comp, int layout, int epi, const GemmLaunch& L, int grid,
                         cudaStream_t st) {
  if (cg == 1 && bn == 256) return dispatch_gemm_bn<256, 1>(comp, layout, epi, L, grid, st);
  if (cg == 1 && bn == 128) return dispatch_gemm_bn<128, 1>(comp, layout, epi, L, grid, st);
  if (cg == 2 && bn == 256) return dispatch_gemm_bn<256, 2>(comp, layout, epi, L, grid, st);
  if (cg == 2 && bn == 128) return dispatch_gemm_bn<128, 2>(comp, layout, epi, L, grid, st);
  return fail(SM_ERR_ARG, "BN must be 128 or 256 and the CTA group 1 or 2");
}

static inline int pick_bn(int64_t n) { return (n % 256 == 0 && SMB_BN_MAX >= 256) ? 256 : 128; }

static GemmProblem gemm_problem(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh,
                                const CUtensorMap& bl, int m, int n, int k, int batch, int bn, int cg, int sym) {
  GemmProblem p;
  memset(&p, 0, sizeof(p));
  p.sym = sym;
  p.a_hi = ah;
  p.a_lo = al;
  p.b_hi = bh;
  p.b_lo = bl;
  p.m = m;
  p.n = n;
  p.k = k;
  p.batch = batch;
  p.tiles_m = m / (kGemmBM * cg);
  p.tiles_n = n / bn;
  p.scale = 1.0f;
  return p;
}

// Tiles of one problem: the full grid, or its upper triangle when symmetric.
// Tiles of the upper block triangle of a symmetric product: row tile mi needs
// the column tiles from R * mi on (R = tn / tm: 1 for square tiles, 2 for
// 256 x 128 pair tiles).
static int64_t sym_tiles(int64_t tm, int64_t tn) {
  const int64_t r = tn / tm;
  return tm * tn - r * tm * (tm - 1) / 2;
}

static int64_t problem_tiles(const GemmProblem& p) {
  if (p.sym) return sym_tiles(p.tiles_m, p.tiles_n) * p.batch;
  return static_cast<int64_t>(p.tiles_m) * p.tiles_n * p.batch;
}

// Executed tensor FLOPs (symmetric products count only the tiles computed).
static double problem_flops(const GemmProblem& p, bool comp) {
  const double tile = 2.0 * (static_cast<double>(p.m) / p.tiles_m) * (static_cast<double>(p.n) / p.tiles_n) * p.k;
  return tile * static_cast<double>(problem_tiles(p)) * (comp ? 3.0 : 1.0);
}

// Balanced static tile schedule for problems given as (tiles, k-blocks per
// tile), laid out back to back in launch-global tile order.  Tiles are taken
// longest first and dealt to the least-loaded worker (CTA or CTA pair; ties to
// the lowest); each worker keeps its tiles in that order.  Output: [grid + 1]
// offsets then the tile lists, grid = the number of workers.
static void lpt_schedule(const std::vector<std::pair<int64_t, int>>& probs, int grid, std::vector<int>& out) {
  std::vector<std::pair<int, int>> tiles;  // (k-blocks, global tile)
  int64_t base = 0;
  for (const auto& pr : probs) {
    for (int64_t t = 0; t < pr.first; ++t) tiles.push_back({pr.second, static_cast<int>(base + t)});
    base += pr.first;
  }
  std::stable_sort(tiles.begin(), tiles.end(), [](const auto& a, const auto& b) { return a.first > b.first; });
  std::vector<std::vector<int>> lists(grid);
  std::vector<int64_t> load(grid, 0);
  // min-heap on (load, cta)
  std::vector<std::pair<int64_t, int>> heap;
  for (int c = 0; c < grid; ++c) heap.push_back({0, c});
  auto cmp = [](const std::pair<int64_t, int>& a, const std::pair<int64_t, int>& b) {
    return a.first != b.first ? a.first > b.first : a.second > b.second;
  };
  std::make_heap(heap.begin(), heap.end(), cmp);
  for (const auto& t : tiles) {
    std::pop_heap(heap.begin(), heap.end(), cmp);
    auto top = heap.back();
    lists[top.second].push_back(t.second);
    top.first += t.first;
    heap.back() = top;
    std::push_heap(heap.begin(), heap.end(), cmp);
  }
  out.assign(grid + 1 + tiles.size(), 0);
  int off = 0;
  for (int c = 0; c < grid; ++c) {
    out[c] = off;
    for (int t : lists[c]) out[grid + 1 + off++] = t;
  }
  out[grid] = off;
}

// ------------------------------------------------------------------- timing

struct Timer {
  bool enabled = false;
  std::vector<cudaEvent_t> pool;
  struct Rec {
    int cls;
    cudaEvent_t a, b;
    double flops;
  };
  std::vector<Rec> recs;
  size_t next = 0;

  // Records the opening event; *idx = record index (or -1 when disabled).
  int begin(int cls, double flops, cudaStream_t st, long* idx) {
    *idx = -1;
    if (!enabled) return SM_OK;
    while (pool.size() < next + 2) {
      cudaEvent_t e;
      SM_CUDA(cudaEventCreate(&e));
      pool.push_back(e);
    }
    Rec r{cls, pool[next], pool[next + 1], flops};
    next += 2;
    SM_CUDA(cudaEventRecord(r.a, st));
    recs.push_back(r);
    *idx = static_cast<long>(recs.size()) - 1;
    return SM_OK;
  }
  int end(long idx, cudaStream_t st) {
    if (idx < 0) return SM_OK;
    SM_CUDA(cudaEventRecord(recs[idx].b, st));
    return SM_OK;
  }
};

// Runs `body` bracketed by timing events of class `cls` when timing is on.
#define SM_TIMED(timer, cls, flops, stream, body)        \
  do {                                                   \
    long rec_ = -1;                                      \
    if ((timer) != nullptr) SM_TRY((timer)->begin((cls), (flops), (stream), &rec_)); \
    SM_TRY(body);                                        \
    if ((timer) != nullptr) SM_TRY((timer)->end(rec_, (stream))); \
  } while (0)

// ------------------------------------------------------------------ groups

struct Group {
  int r = 0, c = 0;      // oriented shape, r <= c
  int rp = 0, cp = 0;    // padded to multiples of 128
  bool pair_ok = false;  // rp % 256 == 0 and CTA pairs fit: 256-row pair tiles possible
  int tile_cg[3] = {1, 1, 1};        // per GEMM kind: 1 = one CTA, 128-row tiles; 2 = CTA pair, 256-row
  int tile_bn[3] = {128, 128, 128};  // per GEMM kind: N extent of a tile
  int batch = 0;
  int mat_off = 0;       // first descriptor of this group in the MatDev table
  bool rank1 = false;
  int dmax = 0;          // leading dimension of the per-row statistic arrays
  __nv_bfloat16 *xh = nullptr, *xl = nullptr, *xa = nullptr, *xb = nullptr, *gh = nullptr, *gl = nullptr;
  __nv_bfloat16 *ph = nullptr, *pl = nullptr;
  __nv_bfloat16* q = nullptr;  // S8 output Q, BF16 [B, rp, cp] (param layout when transposed)
  float *g2 = nullptr, *partials = nullptr;
  // plane scale 2^k of the stored stage-1 input, its stage-1 alphas (rho for
  // X = rho * planes, rho^2 for X X^T, rho / s for P X), S8 scale s, 1/s, graft
  float *pre = nullptr, *rho = nullptr, *rho2 = nullptr, *px_alpha = nullptr;
  float *s = nullptr, *s_inv = nullptr, *gamma = nullptr;
  bool fused_ok = false;  // every matrix fits k_whiten_fused (rows in shared memory)
  int fused_blocks = 0;   // grid x of k_whiten_fused: the most row blocks of a matrix
  // Untransposed matrices (d_out = r, d_in = c) on the row stream
  // (k_whiten_rows) when rows_ok; the transposed ones then take
  // k_whiten_fused alone, with grid x fused_blocks_t.
  bool rows_ok = false;
  int rows_count = 0, rows_threads = 0, rows_grid = 0, fused_blocks_t = 0, fused_blocks_u = 0;
  int* rows_slots = nullptr;  // [rows_count] slots of the untransposed matrices
  std::vector<int> host_rows_slots;
  // Transposed matrices (d_out = c, d_in = r) on the block stream
  // (k_whiten_cols) when cols_ok.
  bool cols_ok = false;
  int cols_count = 0, cols_threads = 0, cols_grid = 0;
  int* cols_slots = nullptr;  // [cols_count] slots of the transposed matrices
  std::vector<int> host_cols_slots;
  float2 *rs_white = nullptr, *rs_map = nullptr;
  int* tmask = nullptr;  // [B] 1 = transposed matrix: its Q is stored in param layout
  unsigned *tk_white = nullptr, *tk_map = nullptr;  // [B] last-CTA tickets (zero between launches)
  std::vector<int> host_tmask;
  // K-major boxes {64, 128}: the iterate as both operands of X X^T, and G / P
  // (128-row tiles of A; G also as the 128-row B tiles of G G)
  CUtensorMap xh_K, xl_K, xa_K, xb_K;
  CUtensorMap gh_K, gl_K, ph_K, pl_K;
  // K-major boxes {64, 64}: the B operand of a symmetric product on 256 x 128
  // CTA-pair tiles, where each CTA stages 64 B rows
  CUtensorMap xh_K64, xl_K64, xa_K64, xb_K64, gh_K64, gl_K64;
  // MN-major boxes {64, 64}: the iterate as the B of P X
  CUtensorMap xh_MN, xl_MN, xa_MN, xb_MN;
};

// Bump allocator over a caller workspace (or a null base to measure).
struct Carver {
  uint8_t* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <typename T>
  T* take(size_t count) {
    off = round_up(static_cast<int64_t>(off), 256);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

enum GemmKind : int { kGram = 0, kGramSq = 1, kPX = 2 };

// Tile shapes of the three GEMM kinds, chosen per plan (choose_tilings):
//   X X^T, G G (symmetric, upper block triangle): one CTA with 128 x 128
//     tiles; a CTA pair with 256 x 256 tiles; or a CTA pair with 256 x 128
//     block-row tiles (each CTA stages 64 B rows: the *_K64 tensor maps);
//   P X: one CTA or a CTA pair (128 / 256 rows) with BN = 128 or 256.
static int kind_cg(const Group& g, int kind) { return g.tile_cg[kind]; }
static int kind_bn(const Group& g, int kind) { return g.tile_bn[kind]; }

// F32Norm partial sums of one matrix's G*G (its tiles_m x tiles_n grid).
static int norm_slots_per_matrix(const Group& g) {
  const int tm = g.rp / (kGemmBM * kind_cg(g, kGramSq));
  const int tn = g.rp / kind_bn(g, kGramSq);
  return tm * tn * kNormSlots;
}

// Room for the partials of the finest tiling (128 x 128 tiles), so a plan's
// layout does not depend on the tiling it picks.
static int norm_slots_capacity(const Group& g) {
  const int t = g.rp / kGemmBM;
  return t * t * kNormSlots;
}

static void carve_group(Carver& cv, Group& g) {
  const size_t xs = static_cast<size_t>(g.batch) * g.rp * g.cp;
  const size_t gs = static_cast<size_t>(g.batch) * g.rp * g.rp;
  g.xh = cv.take<__nv_bfloat16>(2 * xs);  // xh | xl contiguous
  g.xl = g.xh ? g.xh + xs : nullptr;
  g.xa = cv.take<__nv_bfloat16>(2 * xs);  // xa | xb contiguous; q aliases both planes
  g.xb = g.xa ? g.xa + xs : nullptr;
  g.q = g.xa;
  g.gh = cv.take<__nv_bfloat16>(gs);
  g.gl = cv.take<__nv_bfloat16>(gs);
  g.g2 = cv.take<float>(gs);
  g.ph = reinterpret_cast<__nv_bfloat16*>(g.g2);  // P hi | P lo in the g2 bytes
  g.pl = g.ph ? g.ph + gs : nullptr;
  g.partials = cv.take<float>(static_cast<size_t>(g.batch) * norm_slots_capacity(g));
  g.pre = cv.take<float>(g.batch);
  g.rho = cv.take<float>(g.batch);
  g.rho2 = cv.take<float>(g.batch);
  g.px_alpha = cv.take<float>(g.batch);
  g.s = cv.take<float>(g.batch);
  g.s_inv = cv.take<float>(g.batch);
  g.gamma = cv.take<float>(g.batch);
  g.rs_white = cv.take<float2>(static_cast<size_t>(g.batch) * g.dmax);
  g.rs_map = cv.take<float2>(static_cast<size_t>(g.batch) * g.dmax);
  g.tmask = cv.take<int>(g.batch);
  g.tk_white = cv.take<unsigned>(g.batch);
  g.rows_slots = cv.take<int>(g.batch);
  g.cols_slots = cv.take<int>(g.batch);
  g.tk_map = cv.take<unsigned>(g.batch);
}

static int encode_group_maps(Group& g) {
  SM_TRY(make_map(&g.xh_K, g.xh, g.cp, g.rp, g.batch, kBkK, kGemmBM));
  SM_TRY(make_map(&g.xl_K, g.xl, g.cp, g.rp, g.batch, kBkK, kGemmBM));
  SM_TRY(make_map(&g.xa_K, g.xa, g.cp, g.rp, g.batch, kBkK, kGemmBM));
  SM_TRY(make_map(&g.xb_K, g.xb, g.cp, g.rp, g.batch, kBkK, kGemmBM));
  SM_TRY(make_map(&g.gh_K, g.gh, g.rp, g.rp, g.batch, kBkK, kGemmBM));
  SM_TRY(make_map(&g.gl_K, g.gl, g.rp, g.rp, g.batch, kBkK, kGemmBM));
  SM_TRY(make_map(&g.ph_K, g.ph, g.rp, g.rp, g.batch, kBkK, kGemmBM));
  SM_TRY(make_map(&g.pl_K, g.pl, g.rp, g.rp, g.batch, kBkK, kGemmBM));
  SM_TRY(make_map(&g.xh_K64, g.xh, g.cp, g.rp, g.batch, kBkK, kGemmBM / 2));
  SM_TRY(make_map(&g.xl_K64, g.xl, g.cp, g.rp, g.batch, kBkK, kGemmBM / 2));
  SM_TRY(make_map(&g.xa_K64, g.xa, g.cp, g.rp, g.batch, kBkK, kGemmBM / 2));
  SM_TRY(make_map(&g.xb_K64, g.xb, g.cp, g.rp, g.batch, kBkK, kGemmBM / 2));
  SM_TRY(make_map(&g.gh_K64, g.gh, g.rp, g.rp, g.batch, kBkK, kGemmBM / 2));
  SM_TRY(make_map(&g.gl_K64, g.gl, g.rp, g.rp, g.batch, kBkK, kGemmBM / 2));
  SM_TRY(make_map(&g.xh_MN, g.xh, g.cp, g.rp, g.batch, kChunk, kBkK));
  SM_TRY(make_map(&g.xl_MN, g.xl, g.cp, g.rp, g.batch, kChunk, kBkK));
  SM_TRY(make_map(&g.xa_MN, g.xa, g.cp, g.rp, g.batch, kChunk, kBkK));
  SM_TRY(make_map(&g.xb_MN, g.xb, g.cp, g.rp, g.batch, kChunk, kBkK));
  return SM_OK;
}

// Shape fields and the default tiling (pair tiles where possible: 256 x 256
// for the symmetric products, BN = 256 for P X when the columns allow it);
// choose_tilings may replace the tiling for a plan's batch sizes.
static void init_group_shape(Group& g, int r, int c, int batch, bool pair_ok) {
  g.r = r;
  g.c = c;
  g.rp = static_cast<int>(round_up(r, 128));
  g.cp = static_cast<int>(round_up(c, 128));
  g.pair_ok = SMB_PAIR && g.rp % 256 == 0 && pair_ok;
  for (int kind = 0; kind < 2; ++kind) {
    g.tile_cg[kind] = g.pair_ok ? 2 : 1;
    g.tile_bn[kind] = g.pair_ok ? 2 * kGemmBM : kGemmBM;
  }
  g.tile_cg[2] = g.pair_ok ? 2 : 1;
  g.tile_bn[2] = pick_bn(g.cp);
  g.batch = batch;
  g.dmax = c;
}

// --------------------------------------------------------- S8 launch plan
// Stage schedule of the S8 polynomial: stages 1-4 compensated (hi/lo operand
// planes, three BF16 products, FP32 accumulation), stage 5 plain BF16.
// Keeping stage 2-4 iterates at ~16 significant bits holds the map within
// 1e-2 relative Frobenius error of the FP32 reference even for rank-deficient
// inputs, whose near-zero singular values the later stages amplify ~120x.
constexpr int kCompensatedStages = 4;


// Groups whose products share a launch (same BN), longest K first, with an
// optional balanced tile schedule in device memory.
struct LaunchSet {
  std::vector<int> groups;
  int bn = 0;
  int cg = 1;
  int grid = 0;  // CTAs (cg per worker)
  int* sched = nullptr;
  std::vector<int> h_sched;
};

struct S8Launches {
  std::vector<LaunchSet> sets[3];
};

// beta = b / (2c) of S8 stage `stage` (0-based, stages 1-4): the shift that
// turns a I + b G + c G^2 into c (G + beta I)^2 + (a - c beta^2) I.
static double s8_shift(int stage) { return kS8Coeff[stage][1] / (2.0 * kS8Coeff[stage][2]); }

static int kind_k(const Group& g, int kind) { return kind == kGram ? g.cp : g.rp; }
static int kind_n(const Group& g, int kind) { return kind == kPX ? g.cp : g.rp; }

// ------------------------------------------------- tiling by cost model
// A plan's GEMM launches are persistent: each worker (a CTA, or a CTA pair)
// takes its share of the launch's tiles from an LPT schedule, so a launch
// lasts as long as its most loaded worker.  Pair tiles are the most
// efficient per SM, but with few matrices per launch (a rank's share of a
// sharded step) a handful of long tiles leaves most workers idle.  Per GEMM
// kind, choose_tilings estimates that makespan for every tiling the plan's
// groups support and keeps the shortest.
//
// Relative cost of one 64-deep k-block of one tile, in units of a CTA-pair
// 256 x 256 tile's k-block: tile area / (per-SM efficiency x SMs).  The
// per-SM efficiencies relative to the 256 x 256 pair tile come from
// config-1 ncu launch lists on B200 (compensated G G: 79 us per launch on
// pair tiles, 89 us on single-CTA 128 x 128 tiles at 4.4 and 7.7 tile waves,
// i.e. 0.71); the 256 x 128 and 128 x 256 figures are interpolated.
static double kblock_cost(int cg, int bn) {
  const double area = static_cast<double>(kGemmBM * cg) * bn / (256.0 * 256.0);
  double eff;
  if (cg == 2) eff = bn == 256 ? 1.0 : 0.80;
  else eff = bn == 256 ? 0.85 : 0.71;
  return area / (eff * cg / 2.0);
}

// LPT makespan of `costs` over `workers` (the schedule lpt_schedule builds).
static double lpt_makespan(std::vector<double> costs, int workers) {
  if (costs.empty() || workers <= 0) return 0.0;
  std::sort(costs.begin(), costs.end(), [](double a, double b) { return a > b; });
  std::priority_queue<double, std::vector<double>, std::greater<double>> load;
  for (int w = 0; w < workers; ++w) load.push(0.0);
  double worst = 0.0;
  for (double c : costs) {
    double l = load.top() + c;
    load.pop();
    load.push(l);
    worst = std::max(worst, l);
  }
  return worst;
}

// Estimated duration of one stage's launches of `kind` with the groups'
// current tile choices: groups sharing a (cg, bn) share a launch (as in
// build_s8_launches); launches run one after another, each paying a fixed
// ramp of about two k-blocks.
static double kind_cost(const std::vector<Group>& groups, int kind, int sms, int pairs) {
  std::vector<std::pair<int, int>> keys;
  for (const Group& g : groups) {
    const std::pair<int, int> key{kind_cg(g, kind), kind_bn(g, kind)};
    if (std::find(keys.begin(), keys.end(), key) == keys.end()) keys.push_back(key);
  }
  double total = 0.0;
  for (const auto& key : keys) {
    std::vector<double> costs;
    const double unit = kblock_cost(key.first, key.second);
    for (const Group& g : groups) {
      if (kind_cg(g, kind) != key.first || kind_bn(g, kind) != key.second) continue;
      const int64_t tm = g.rp / (kGemmBM * key.first);
      const int64_t tn = kind_n(g, kind) / key.second;
      const int64_t tiles = (kind == kPX ? tm * tn : sym_tiles(tm, tn)) * g.batch;
      const double c = unit * (kind_k(g, kind) / kBkK);
      for (int64_t t = 0; t < tiles; ++t) costs.push_back(c);
    }
    total += lpt_makespan(costs, key.first == 2 ? pairs : sms) + 2.0;
  }
  return total;
}

// Picks, per GEMM kind, the tiling with the shortest estimated launches for
// these groups (the same candidate for every group that supports it; the
// others keep one-CTA tiles).  The default (first candidate: pair tiles)
// stays unless another is estimated at least 10% faster, since the
// efficiencies above are estimates.  SMB_TILE_MODEL=0 keeps the defaults
// (for measuring the model against them).
#ifndef SMB_TILE_MODEL
#define SMB_TILE_MODEL 1
#endif
static void choose_tilings(std::vector<Group>& groups, int sms, int pairs) {
  if (!SMB_TILE_MODEL) return;
  for (int kind = 0; kind < 3; ++kind) {
    const std::pair<int, int> sym_options[] = {{2, 256}, {2, 128}, {1, 128}};
    const std::pair<int, int> px_options[] = {{2, 256}, {2, 128}, {1, 256}, {1, 128}};
    const std::pair<int, int>* options = kind == kPX ? px_options : sym_options;
    const int n_options = kind == kPX ? 4 : 3;
    double best = -1.0;
    std::vector<std::pair<int, int>> best_pick;
    for (int o = 0; o < n_options; ++o) {
      std::vector<std::pair<int, int>> pick;
      for (Group& g : groups) {
        int cg = options[o].first, bn = options[o].second;
        const bool ok = (cg == 1 || (g.pair_ok && pairs > 0)) && kind_n(g, kind) % bn == 0;
        if (!ok) {
          cg = 1;
          bn = kind == kPX ? pick_bn(g.cp) : kGemmBM;
        }
        g.tile_cg[kind] = cg;
        g.tile_bn[kind] = bn;
        pick.push_back({cg, bn});
      }
      const double cost = kind_cost(groups, kind, sms, pairs) * (o == 0 ? 0.9 : 1.0);
      if (best < 0.0 || cost < best) {
        best = cost;
        best_pick = pick;
      }
    }
    for (size_t i = 0; i < groups.size(); ++i) {
      groups[i].tile_cg[kind] = best_pick[i].first;
      groups[i].tile_bn[kind] = best_pick[i].second;
    }
  }
}

// Builds the launch sets of every GEMM kind.  With `cv` the tile schedules
// are carved from the workspace (measured when cv.base is null).  `pairs` is
// the number of CTA pairs that can be resident at once.
static void build_s8_launches(const std::vector<Group>& groups, int sms, int pairs, Carver* cv, S8Launches* out) {
  for (int kind = 0; kind < 3; ++kind) {
    std::vector<LaunchSet>& sets = out->sets[kind];
    sets.clear();
    for (int gi = 0; gi < static_cast<int>(groups.size()); ++gi) {
      const int bn = kind_bn(groups[gi], kind);
      const int cg = kind_cg(groups[gi], kind);
      LaunchSet* set = nullptr;
      for (auto& s : sets)
        if (s.bn == bn && s.cg == cg && static_cast<int>(s.groups.size()) < kMaxProblems) set = &s;
      if (set == nullptr) {
        sets.push_back(LaunchSet());
        set = &sets.back();
        set->bn = bn;
        set->cg = cg;
      }
      set->groups.push_back(gi);
    }
    for (auto& set : sets) {
      std::stable_sort(set.groups.begin(), set.groups.end(), [&](int a, int b) {
        return kind_k(groups[a], kind) > kind_k(groups[b], kind);
      });
      std::vector<std::pair<int64_t, int>> probs;
      int64_t total = 0;
      for (int gi : set.groups) {
        const Group& g = groups[gi];
        const int64_t tm = g.rp / (kGemmBM * set.cg);
        const int64_t tn = kind_n(g, kind) / set.bn;
        const int64_t tiles = (kind == kPX ? tm * tn : sym_tiles(tm, tn)) * g.batch;
        probs.push_back({tiles, kind_k(g, kind) / kBkK});
        total += tiles;
      }
      const int workers = static_cast<int>(std::min<int64_t>(total, set.cg == 2 ? pairs : sms));
      set.grid = workers * set.cg;
      if (cv != nullptr && workers > 0 && SMB_USE_SCHEDULE) {
        lpt_schedule(probs, workers, set.h_sched);
        set.sched = cv->take<int>(set.h_sched.size());
      }
    }
  }
}

// The GEMM of `kind` in S8 stage `stage` (0-based) for group g: operands,
// outputs and epilogue.  Iterates alternate between the xa|xb and xh|xl pairs.
static GemmProblem s8_problem(const Group& g, int kind, int stage, int bn, int* epi) {
  const bool comp = stage < kCompensatedStages;
  const bool in_a = (stage % 2) == 1;  // stages 2 and 4 read xa|xb
  const CUtensorMap& xK_h = in_a ? g.xa_K : g.xh_K;
  const CUtensorMap& xK_l = in_a ? g.xb_K : g.xl_K;
  const CUtensorMap& xMN_h = in_a ? g.xa_MN : g.xh_MN;
  const CUtensorMap& xMN_l = in_a ? g.xb_MN : g.xl_MN;
  GemmProblem p;
  // B rows staged per CTA: 64 on 256 x 128 pair tiles, else 128
  const bool b64 = kind_cg(g, kind) == 2 && bn == kGemmBM;
  if (kind == kGram) {
    // X X^T: A = B = X, K-major, symmetric tiles
    const CUtensorMap& bK_h = b64 ? (in_a ? g.xa_K64 : g.xh_K64) : xK_h;
    const CUtensorMap& bK_l = b64 ? (in_a ? g.xb_K64 : g.xl_K64) : xK_l;
    p = gemm_problem(xK_h, comp ? xK_l : xK_h, bK_h, comp ? bK_l : bK_h, g.rp, g.rp, g.cp, g.batch, bn,
                     kind_cg(g, kind), 1);
    p.out0 = g.gh;
    p.out1 = g.gl;
    *epi = comp ? kEpiHiLo : kEpiBF16;
    // stages 2-5 store the shifted gram H = G + beta I (see the G H product);
    // stage 1 scales the planes' product by rho^2 (normalised input)
    if (stage > 0) p.diag = static_cast<float>(s8_shift(stage));
    else p.alpha = g.rho2;
  } else if (kind == kGramSq) {
    // G G with G symmetric: B = G read K-major as G^T
    const CUtensorMap& bG_h = b64 ? g.gh_K64 : g.gh_K;
    const CUtensorMap& bG_l = b64 ? g.gl_K64 : g.gl_K;
    p = gemm_problem(g.gh_K, comp ? g.gl_K : g.gh_K, bG_h, comp ? bG_l : bG_h, g.rp, g.rp, g.rp, g.batch,
                     bn, kind_cg(g, kind), 1);
    if (stage == 0) {
      p.out0 = g.g2;
      p.partials = g.partials;
      *epi = kEpiF32Norm;
    } else {
      // Stages 2-5: with H = G + beta I and beta = b / (2c), the polynomial
      //   P = a I + b G + c G^2 = c H^2 + (a - c beta^2) I,
      // so this product squares the shifted gram the X X^T epilogue stored and
      // its epilogue only scales and adds to the diagonal: no gram re-read.
      const double a = kS8Coeff[stage][0], c = kS8Coeff[stage][2], beta = s8_shift(stage);
      p.scale = static_cast<float>(c);
      p.diag = static_cast<float>(a - c * beta * beta);
      if (comp) {
        p.out0 = g.ph;
        p.out1 = g.pl;
        *epi = kEpiHiLo;
      } else {
        p.out0 = g.gl;
        *epi = kEpiBF16;
      }
    }
  } else {
    // P X with X read MN-major; P lives in gh|gl (stage 1, written by
    // k_poly_stage1), in the g2 bytes (stages 2-4) or in gl (stage 5).
    const CUtensorMap& pA_h = stage == 0 ? g.gh_K : (comp ? g.ph_K : g.gl_K);
    const CUtensorMap& pA_l = stage == 0 ? g.gl_K : (comp ? g.pl_K : g.gl_K);
    p = gemm_problem(pA_h, pA_l, xMN_h, comp ? xMN_l : xMN_h, g.rp, g.cp, g.rp, g.batch, bn, kind_cg(g, kind), 0);
    const bool last = stage == 4;
    const bool next_comp = stage + 1 < kCompensatedStages;
    if (last) {
      // Q rounded to BF16 (2^-9 relative per element, uncorrelated with the
      // S8 error: ~0.1% of the update in quadrature) halves what this
      // product writes and both mapback passes read
      p.out0 = g.q;  // over the xa plane; stage 5 reads xh
      p.tmask = g.tmask;  // transposed matrices: Q stored in param layout
      *epi = kEpiBF16;
    } else {
      p.out0 = in_a ? g.xh : g.xa;
      p.out1 = in_a ? g.xl : g.xb;
      *epi = next_comp ? kEpiHiLo : kEpiBF16;
    }
    if (stage == 0) p.alpha = g.px_alpha;  // X2 = (P rho planes) / s
  }
  return p;
}

static int launch_s8_kind(const std::vector<Group>& groups, const S8Launches& plan, int kind, int stage,
                          cudaStream_t st, Timer* tm, int64_t* launches) {
  const bool comp = stage < kCompensatedStages;
  for (const LaunchSet& set : plan.sets[kind]) {
    GemmLaunch L;
    memset(&L, 0, sizeof(L));
    int epi = -1;
    int begin = 0;
    double flops = 0.0;
    for (int gi : set.groups) {
      int e = -1;
      GemmProblem p = s8_problem(groups[gi], kind, stage, set.bn, &e);
      if (epi >= 0 && e != epi) return fail(SM_ERR_ARG, "mixed epilogues in one launch");
      epi = e;
      p.tile_begin = begin;
      begin += static_cast<int>(problem_tiles(p));
      flops += problem_flops(p, comp);
      L.p[L.n_problems++] = p;
    }
    L.total_tiles = begin;
    L.sched = set.sched;
    const int layout = kind == kPX ? kLayoutKM : kLayoutKK;
    SM_TIMED(tm, SM_TCLASS_GEMM, flops, st, dispatch_gemm(set.bn, set.cg, comp, layout, epi, L, set.grid, st));
    ++*launches;
  }
  return SM_OK;
}

// The five-stage S8 polynomial of every group: inputs are the stage-1 planes
// xh/xl (normalised, oriented, zero-padded); outputs BF16 Q [B, rp, cp] in
// each group's q.  Mirrors _s8_fp32 (sandmuon/optimizer.py:79-91); every GEMM
// of a stage covers all groups in one launch.
static int run_s8(const std::vector<Group>& groups, const S8Launches& plan, cudaStream_t st, Timer* tm,
                  int64_t* launches) {
  for (int stage = 0; stage < 5; ++stage) {
    SM_TRY(launch_s8_kind(groups, plan, kGram, stage, st, tm, launches));
    SM_TRY(launch_s8_kind(groups, plan, kGramSq, stage, st, tm, launches));
    if (stage == 0) {
      // s = max(1.35 |G2|_F^(1/4), 1e-30); P = a I + b G/s/s + c G2/s/s/s/s (hi/lo in place of G)
      for (const Group& g : groups) {
        const int per_mat = norm_slots_per_matrix(g);
        const int64_t per = static_cast<int64_t>(g.rp) * g.rp;
        const int blocks = static_cast<int>(std::min<int64_t>(cdiv(per / 4, 1024), 512));
        SM_TIMED(tm, SM_TCLASS_ELEMWISE, 0.0, st, ([&]() -> int {
                   SM_TRY(launch_kernel(k_poly_stage1, dim3(blocks, g.batch), dim3(256), 0, st, g.gh, g.gl, g.g2,
                                        g.partials, per_mat, kS8Margin, g.s, g.s_inv, g.rho, g.px_alpha, g.rp,
                                        (float)kS8Coeff[0][0], (float)kS8Coeff[0][1], (float)kS8Coeff[0][2]));
                   return SM_OK;
                 }()));
        *launches += 1;
      }
    }
    SM_TRY(launch_s8_kind(groups, plan, kPX, stage, st, tm, launches));
  }
  return SM_OK;
}

// Whitening / normalisation front end for one group (N3 passes 1 and 2).
// Raises k_whiten_fused's dynamic shared-memory limit once per device and
// instantiation (at plan creation, outside any capture).
static int prepare_front_fused(bool rank1) {
  static std::mutex mutex;
  static bool done[2][64] = {};
  int dev = 0;
  SM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(SM_ERR_UNSUPPORTED, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(mutex);
  if (!done[rank1][dev]) {
    auto kern = rank1 ? k_whiten_fused<true> : k_whiten_fused<false>;
    SM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kFusedSmemBytes));
    done[rank1][dev] = true;
  }
  return SM_OK;
}

// SMB_FRONT_ROWS=0 keeps every matrix of a fused-eligible group on
// k_whiten_fused (the untransposed row stream off).
#ifndef SMB_FRONT_ROWS
#define SMB_FRONT_ROWS 1
#endif
constexpr bool kFrontRows = SMB_FRONT_ROWS != 0;
// SMB_FRONT_COLS=0 keeps the transposed matrices on k_whiten_fused.
#ifndef SMB_FRONT_COLS
#define SMB_FRONT_COLS 1
#endif
constexpr bool kFrontCols = SMB_FRONT_COLS != 0;

// Sizes the row stream of group g (k_whiten_rows): raises the kernel's
// dynamic shared-memory limit once per device and instantiation, then takes
// as many CTAs as fit on the device at once, at most one per row.  At plan
// creation, outside any capture.
static int prepare_front_rows(Group& g, int sms) {
  static std::mutex mutex;
  static bool done[2][64] = {};
  int dev = 0;
  SM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(SM_ERR_UNSUPPORTED, "device ordinal out of range");
  auto kern = g.rank1 ? k_whiten_rows<true> : k_whiten_rows<false>;
  {
    std::lock_guard<std::mutex> lock(mutex);
    if (!done[g.rank1][dev]) {
      SM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, rows_smem_bytes(32 * 8 * kRowsKMax * 4)));
      SM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
      done[g.rank1][dev] = true;
    }
  }
  int per_sm = 0;
  SM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, g.rows_threads,
                                                        static_cast<size_t>(rows_smem_bytes(g.c))));
  if (per_sm < 1) {
    g.rows_ok = false;
    return SM_OK;
  }
  const int64_t rows = static_cast<int64_t>(g.rows_count) * g.r;
  g.rows_grid = static_cast<int>(std::min<int64_t>(rows, static_cast<int64_t>(per_sm) * sms));
  return SM_OK;
}

// Sizes the block stream of group g (k_whiten_cols): one CTA per SM, at
// most one per block.  At plan creation, outside any capture.
static int prepare_front_cols(Group& g, int sms) {
  static std::mutex mutex;
  static bool done[2][64] = {};
  int dev = 0;
  SM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(SM_ERR_UNSUPPORTED, "device ordinal out of range");
  auto kern = g.rank1 ? k_whiten_cols<true> : k_whiten_cols<false>;
  {
    std::lock_guard<std::mutex> lock(mutex);
    if (!done[g.rank1][dev]) {
      SM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 196608));
      SM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
      done[g.rank1][dev] = true;
    }
  }
  int per_sm = 0;
  SM_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, g.cols_threads,
                                                        static_cast<size_t>(cols_smem_bytes(g.r))));
  if (per_sm < 1) {
    g.cols_ok = false;
    return SM_OK;
  }
  const int64_t blocks = static_cast<int64_t>(g.cols_count) * cdiv(g.c, kColsRows);
  g.cols_grid = static_cast<int>(std::min<int64_t>(blocks, static_cast<int64_t>(per_sm) * sms));
  return SM_OK;
}

// One launch of the fused front end (k_whiten_fused) for group g: every
// matrix, or those of one orientation when a stream takes the other.
static int launch_front_fused(const Group& g, const MatDev* mats, float mom_beta, float mom_omb, int which,
                              cudaStream_t st) {
  auto kern = g.rank1 ? k_whiten_fused<true> : k_whiten_fused<false>;
  const int gx = which == 1 ? g.fused_blocks_t : which == 2 ? g.fused_blocks_u : g.fused_blocks;
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(g.batch));
  return launch_kernel(kern, grid, dim3(256), static_cast<size_t>(kFusedSmemBytes), st, mats, mom_beta, mom_omb,
                       g.rs_white, g.dmax, g.pre, g.rho, g.rho2, g.tk_white, g.xh, g.xl,
                       static_cast<int64_t>(g.rp), static_cast<int64_t>(g.cp), which);
}

// One launch of the transposed block stream (k_whiten_cols) for group g.
static int launch_front_cols(const Group& g, const MatDev* mats, float mom_beta, float mom_omb, cudaStream_t st) {
  auto kern = g.rank1 ? k_whiten_cols<true> : k_whiten_cols<false>;
  return launch_kernel(kern, dim3(static_cast<unsigned>(g.cols_grid)), dim3(static_cast<unsigned>(g.cols_threads)),
                       static_cast<size_t>(cols_smem_bytes(g.r)), st, mats, g.cols_slots, g.cols_count, g.c, g.r,
                       mom_beta, mom_omb, g.rs_white, g.dmax, g.pre, g.rho, g.rho2, g.tk_white, g.xh, g.xl,
                       static_cast<int64_t>(g.rp), static_cast<int64_t>(g.cp));
}

// One launch of the untransposed row stream (k_whiten_rows) for group g.
static int launch_front_rows(const Group& g, const MatDev* mats, float mom_beta, float mom_omb, cudaStream_t st) {
  auto kern = g.rank1 ? k_whiten_rows<true> : k_whiten_rows<false>;
  return launch_kernel(kern, dim3(static_cast<unsigned>(g.rows_grid)), dim3(static_cast<unsigned>(g.rows_threads)),
                       static_cast<size_t>(rows_smem_bytes(g.c)), st, mats, g.rows_slots, g.rows_count, g.r, g.c,
                       mom_beta, mom_omb, g.rs_white, g.dmax, g.pre, g.rho, g.rho2, g.tk_white, g.xh, g.xl,
                       static_cast<int64_t>(g.rp), static_cast<int64_t>(g.cp));
}

// Whitening / normalisation front end for one group (N3).  `fused`: one pass
// (k_whiten_fused) when the group qualifies (16-byte aligned rows that fit
// its shared memory) -- it scales the planes by the previous step's plane
// scale, so a plan's first step always takes the two passes, which derive
// the scale from this step's norm.  Both paths store the same planes up to
// the power-of-two scale and set the same stage-1 alphas.
static int run_front(const Group& g, const MatDev* d_mats, float mom_beta, float mom_omb, bool vec4, bool fused,
                     cudaStream_t st, Timer* tm, int64_t* launches) {
  const int B = g.batch;
  const int ld = g.dmax;
  const MatDev* mats = d_mats + g.mat_off;
  if (fused && vec4 && g.fused_ok) {
    // untransposed matrices: row stream; transposed: block stream; what
    // neither takes goes through k_whiten_fused
    if (g.rows_ok) {
      SM_TIMED(tm, SM_TCLASS_ELEMWISE, 0.0, st, launch_front_rows(g, mats, mom_beta, mom_omb, st));
      *launches += 1;
    }
    if (g.cols_ok) {
      SM_TIMED(tm, SM_TCLASS_ELEMWISE, 0.0, st, launch_front_cols(g, mats, mom_beta, mom_omb, st));
      *launches += 1;
    }
    const bool rest_u = g.rows_count > 0 && !g.rows_ok, rest_t = g.cols_count > 0 && !g.cols_ok;
    if (rest_u || rest_t) {
      const int which = rest_u && rest_t ? 0 : rest_t ? 1 : 2;
      SM_TIMED(tm, SM_TCLASS_ELEMWISE, 0.0, st, launch_front_fused(g, mats, mom_beta, mom_omb, which, st));
      *launches += 1;
    }
    return SM_OK;
  }
  SM_TIMED(tm, SM_TCLASS_ELEMWISE, 0.0, st, ([&]() -> int {
             dim3 grid(static_cast<unsigned>(cdiv(g.dmax, 8 * kWhitenRows)), B);
             auto kern = g.rank1 ? (vec4 ? k_whiten_rowstats<4, true> : k_whiten_rowstats<1, true>)
                                 : (vec4 ? k_whiten_rowstats<4, false> : k_whiten_rowstats<1, false>);
             SM_TRY(launch_kernel(kern, grid, dim3(256), 0, st, mats, mom_beta, mom_omb, g.rs_white, ld, g.pre,
                                  g.rho, g.rho2, g.tk_white));
             return SM_OK;
           }()));
  SM_TIMED(tm, SM_TCLASS_ELEMWISE, 0.0, st, ([&]() -> int {
             // 32 x 64 tiles of a matrix in either orientation of the group's shape
             const int64_t tiles = std::max(cdiv(g.c, 64) * cdiv(g.r, 32), cdiv(g.r, 64) * cdiv(g.c, 32));
             dim3 grid(static_cast<unsigned>(tiles), B);
             auto kern = g.rank1 ? (vec4 ? k_whiten_write<true, true> : k_whiten_write<true, false>)
                                 : (vec4 ? k_whiten_write<false, true> : k_whiten_write<false, false>);
             SM_TRY(launch_kernel(kern, grid, dim3(256), 0, st, mats, mom_beta, mom_omb, g.rs_white, ld, g.pre,
                                  g.xh, g.xl, static_cast<int64_t>(g.rp), static_cast<int64_t>(g.cp)));
             return SM_OK;
           }()));
  *launches += 2;
  return SM_OK;
}

// Mapback + graft + update back end for one group (N7 passes 1 and 2).
static int run_back(const Group& g, const MatDev* d_mats, bool vec4, int sms, const PeerSet& peers, cudaStream_t st,
                    Timer* tm, int64_t* launches) {
  const int B = g.batch;
  const int ld = g.dmax;
  const MatDev* mats = d_mats + g.mat_off;
  SM_TIMED(tm, SM_TCLASS_ELEMWISE, 0.0, st, ([&]() -> int {
             dim3 grid(static_cast<unsigned>(cdiv(g.dmax, 8 * kMapbackRows)), B);
             auto kern = g.rank1 ? k_mapback_rowstats<true> : k_mapback_rowstats<false>;
             SM_TRY(launch_kernel(kern, grid, dim3(256), 0, st, mats, g.q, static_cast<int64_t>(g.rp),
                                  static_cast<int64_t>(g.cp), g.rs_map, ld, g.gamma, g.tk_map));
             return SM_OK;
           }()));
  SM_TIMED(tm, SM_TCLASS_ELEMWISE, 0.0, st, ([&]() -> int {
             // ~4 iterations per thread over the largest matrix of the group
             const int64_t per = static_cast<int64_t>(g.r) * g.c / (vec4 ? 4 : 1);
             const unsigned gx = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(cdiv(per, 1024), 8 * sms)));
             dim3 grid(gx, B);
             auto kern = g.rank1 ? (vec4 ? k_mapback_apply<true, true> : k_mapback_apply<true, false>)
                                 : (vec4 ? k_mapback_apply<false, true> : k_mapback_apply<false, false>);
             SM_TRY(launch_kernel(kern, grid, dim3(256), 0, st, mats, g.q, static_cast<int64_t>(g.rp),
                                  static_cast<int64_t>(g.cp), g.rs_map, ld, g.gamma, peers));
             return SM_OK;
           }()));
  *launches += 2;
  return SM_OK;
}

}  // namespace smb

using namespace smb;

// ==================================================================== plan

#ifndef SMB_PDL
#define SMB_PDL 1
#endif

struct SmPlan {
  int device = 0;
  std::vector<SmMatrixSpec> mats;
  std::vector<SmStatSpec> stats;
  std::vector<Group> groups;
  std::vector<int> order;        // table position -> matrix index
  std::vector<int> mat_group;    // matrix index -> group
  std::vector<int> mat_slot;     // matrix index -> slot within group
  float stat_beta = 0.97f, stat_omb = 0.03f;
  int export_mode = SM_EXPORT_WEIGHTS;
  float mom_beta = 0.8f, mom_omb = 0.2f;
  MatDev* d_mats = nullptr;
  StatDev* d_stats = nullptr;
  size_t table_bytes = 0;
  std::vector<uint8_t> h_table;
  // per-stat outputs
  std::vector<float*> s_inv, s_z, s_zeta, s_scal;
  S8Launches s8;
  Timer timer;
  int64_t launches_last = 0;
  // Graph replay: from the second step on, the step's launches run as one
  // CUDA graph (captured on a private stream; kernel choices depend only on
  // the plan and on the per-group vec4 flags, which key the capture).  The
  // per-step descriptor table is uploaded before each replay.
  bool replay = true;
  bool pdl = SMB_PDL != 0;  // programmatic dependent launch between the step's kernels
  int64_t steps_done = 0;
  cudaStream_t cap_stream = nullptr;
  cudaGraphExec_t exec = nullptr;
  std::vector<uint8_t> exec_vec4;
  int64_t exec_launches = 0;
  // Peer-mirrored weight range (sm_plan_set_peers): weights inside
  // [peer_lo, peer_hi) are also stored at each peer's copy.
  PeerSet peers{};
  const char* peer_lo = nullptr;
  const char* peer_hi = nullptr;
};

namespace smb {

__global__ void k_fill(float* p, int64_t n, float v) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = v;
}

static int plan_layout(const SmPlanSpec* spec, void* ws, SmPlan* plan, size_t* bytes) {
  if (spec == nullptr || spec->n_matrices < 0 || spec->n_stats < 0)
    return fail(SM_ERR_ARG, "null or negative plan spec");
  Carver cv(ws);
  const int nm = spec->n_matrices, ns = spec->n_stats;
  // group discovery (oriented shape, first-appearance order)
  std::vector<std::pair<int, int>> shapes;
  std::vector<int> mg(nm), slot(nm);
  std::vector<int> counts;
  for (int i = 0; i < nm; ++i) {
    const SmMatrixSpec& m = spec->matrices[i];
    if (m.d_out <= 0 || m.d_in <= 0) return fail(SM_ERR_ARG, "matrix with empty shape");
    if (m.a_stat < 0 || m.a_stat >= ns || m.b_stat < 0 || m.b_stat >= ns)
      return fail(SM_ERR_ARG, "matrix statistic index out of range");
    const SmStatSpec& sa = spec->stats[m.a_stat];
    const SmStatSpec& sb = spec->stats[m.b_stat];
    if (sa.kind == SM_STAT_B || sb.kind != SM_STAT_B) return fail(SM_ERR_ARG, "statistic kinds do not match sides");
    if (sa.n != m.d_in || sb.n != m.d_out) return fail(SM_ERR_ARG, "statistic length does not match matrix shape");
    const int r = std::min(m.d_out, m.d_in), c = std::max(m.d_out, m.d_in);
    int g = -1;
    for (size_t k = 0; k < shapes.size(); ++k)
      if (shapes[k].first == r && shapes[k].second == c) g = static_cast<int>(k);
    if (g < 0) {
      g = static_cast<int>(shapes.size());
      shapes.push_back({r, c});
      counts.push_back(0);
    }
    mg[i] = g;
    slot[i] = counts[g]++;
  }
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  int pairs = 0;
  SM_TRY(pair_workers(di, &pairs));
  std::vector<Group> groups(shapes.size());
  int off = 0;
  for (size_t g = 0; g < shapes.size(); ++g) {
    init_group_shape(groups[g], shapes[g].first, shapes[g].second, counts[g], pairs > 0);
    groups[g].mat_off = off;
    off += counts[g];
    bool any_r1 = false, any_diag = false;
    for (int i = 0; i < nm; ++i) {
      if (mg[i] != static_cast<int>(g)) continue;
      const int kind = spec->stats[spec->matrices[i].a_stat].kind;
      if (kind == SM_STAT_A_RANK1) any_r1 = true;
      else any_diag = true;
    }
    if (any_r1 && any_diag) return fail(SM_ERR_ARG, "a shape group mixes rank-one and diagonal A statistics");
    groups[g].rank1 = any_r1;
    // The fused front end needs every matrix's rows in shared memory (at
    // least 4 rows per CTA for a transposed matrix, whose rows become X
    // columns); the rows' 16-byte alignment is checked per step (vec4).
    bool fused_ok = true;
    int fused_blocks = 0;
    for (int i = 0; i < nm; ++i) {
      if (mg[i] != static_cast<int>(g)) continue;
      const SmMatrixSpec& m = spec->matrices[i];
      const int rows = fused_rows(m.d_in);
      if (m.d_in % 4 != 0 || rows < (m.d_out > m.d_in ? 4 : 1)) {
        fused_ok = false;
        break;
      }
      fused_blocks = std::max(fused_blocks, static_cast<int>(cdiv(m.d_out, rows)));
    }
    groups[g].fused_ok = fused_ok;
    groups[g].fused_blocks = fused_blocks;
    // row stream for the untransposed matrices (slot order), k_whiten_fused for the rest
    groups[g].host_rows_slots.clear();
    groups[g].host_cols_slots.clear();
    int fused_blocks_t = 0, fused_blocks_u = 0;
    for (int i = 0; i < nm; ++i) {  // slots rise with i within a group
      if (mg[i] != static_cast<int>(g)) continue;
      const SmMatrixSpec& m = spec->matrices[i];
      const int nblk = static_cast<int>(cdiv(m.d_out, std::max(1, fused_rows(m.d_in))));
      if (m.d_out > m.d_in) {
        fused_blocks_t = std::max(fused_blocks_t, nblk);
        groups[g].host_cols_slots.push_back(slot[i]);
      } else {
        fused_blocks_u = std::max(fused_blocks_u, nblk);
        groups[g].host_rows_slots.push_back(slot[i]);
      }
    }
    groups[g].rows_count = static_cast<int>(groups[g].host_rows_slots.size());
    groups[g].cols_count = static_cast<int>(groups[g].host_cols_slots.size());
    groups[g].fused_blocks_t = fused_blocks_t;
    groups[g].fused_blocks_u = fused_blocks_u;
    groups[g].rows_ok = kFrontRows && fused_ok && groups[g].rows_count > 0 && rows_stream_fits(groups[g].c);
    groups[g].rows_threads = 32 * rows_team_warps(groups[g].c);
    groups[g].cols_ok = kFrontCols && fused_ok && groups[g].cols_count > 0 && cols_stream_fits(groups[g].r);
    groups[g].cols_threads = cols_threads(groups[g].r);
  }
  choose_tilings(groups, di->sms, pairs);
  MatDev* d_mats = cv.take<MatDev>(nm);
  StatDev* d_stats = cv.take<StatDev>(ns);
  std::vector<float*> s_inv(ns), s_z(ns), s_zeta(ns), s_scal(ns);
  for (int s = 0; s < ns; ++s) {
    const SmStatSpec& st = spec->stats[s];
    if (st.n <= 0) return fail(SM_ERR_ARG, "statistic with empty length");
    s_inv[s] = cv.take<float>(st.n);
    s_z[s] = st.kind == SM_STAT_A_RANK1 ? cv.take<float>(st.n) : nullptr;
    s_zeta[s] = st.kind == SM_STAT_A_RANK1 ? cv.take<float>(st.n) : nullptr;
    s_scal[s] = cv.take<float>(4);
  }
  for (auto& g : groups) carve_group(cv, g);
  S8Launches s8;
  build_s8_launches(groups, di->sms, pairs, &cv, &s8);
  *bytes = round_up(static_cast<int64_t>(cv.off), 256);
  if (plan != nullptr) {
    plan->s8 = s8;
    plan->mats.assign(spec->matrices, spec->matrices + nm);
    plan->stats.assign(spec->stats, spec->stats + ns);
    plan->groups = groups;
    plan->mat_group = mg;
    plan->mat_slot = slot;
    plan->order.assign(nm, 0);
    for (int i = 0; i < nm; ++i) plan->order[groups[mg[i]].mat_off + slot[i]] = i;
    plan->d_mats = d_mats;
    plan->d_stats = d_stats;
    plan->table_bytes = reinterpret_cast<uint8_t*>(d_stats + ns) - reinterpret_cast<uint8_t*>(d_mats);
    plan->s_inv = s_inv;
    plan->s_z = s_z;
    plan->s_zeta = s_zeta;
    plan->s_scal = s_scal;
  }
  return SM_OK;
}

// A statistics workspace starts with kStatsTicketWords tickets (one per
// column group of the TMA kernel; zero between calls), then the partial rows.
constexpr int kStatsTicketWords = 4096;
constexpr size_t kStatsTicketBytes = kStatsTicketWords * sizeof(unsigned);

// Statistics launch geometry.  CB column blocks (of 32 * vec columns) per CTA
// when that divides the block count; row splits for about
// SMB_STATS_CTAS_PER_SM CTAs per SM, each warp covering at least one
// unrolled batch of rows.
#ifndef SMB_STATS_UNROLL
#define SMB_STATS_UNROLL 8
#endif
#ifndef SMB_STATS_CTAS_PER_SM
#define SMB_STATS_CTAS_PER_SM 2
#endif
#ifndef SMB_STATS_CB_MAX
#define SMB_STATS_CB_MAX 4
#endif

struct StatsGeometry {
  int cb = 1;
  int64_t groups = 0, splits = 0, rows_per_split = 0;
};

static StatsGeometry stats_geometry(int64_t n_rows, int64_t n_cols, int vec, int sms, int64_t max_splits) {
  StatsGeometry g;
  const int64_t blocks = cdiv(n_cols, 32 * vec);
  for (int c : {4, 2}) {
    if (c <= SMB_STATS_CB_MAX && blocks % c == 0) {
      g.cb = c;
      break;
    }
  }
  g.groups = blocks / g.cb;
  const int64_t row_groups = 8 / g.cb;
  int64_t splits = cdiv(static_cast<int64_t>(SMB_STATS_CTAS_PER_SM) * sms, g.groups);
  splits = std::min<int64_t>(splits, cdiv(n_rows, row_groups * SMB_STATS_UNROLL));
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, max_splits));
  g.rows_per_split = cdiv(n_rows, splits);
  g.splits = cdiv(n_rows, g.rows_per_split);
  return g;
}

template <typename T, int VEC, bool FIRST>
static void colstats_partial(const StatsGeometry& g, const T* x, int64_t n_rows, int64_t n_cols, int64_t rs,
                             int64_t cs, float* part_sq, float* part_s, cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>(g.groups), static_cast<unsigned>(g.splits));
  constexpr int U = SMB_STATS_UNROLL;
  if (g.cb == 4)
    k_colstats_partial<T, VEC, FIRST, 4, U><<<grid, 256, 0, st>>>(x, n_rows, n_cols, rs, cs, g.rows_per_split,
                                                                  part_sq, part_s);
  else if (g.cb == 2)
    k_colstats_partial<T, VEC, FIRST, 2, U><<<grid, 256, 0, st>>>(x, n_rows, n_cols, rs, cs, g.rows_per_split,
                                                                  part_sq, part_s);
  else
    k_colstats_partial<T, VEC, FIRST, 1, U><<<grid, 256, 0, st>>>(x, n_rows, n_cols, rs, cs, g.rows_per_split,
                                                                  part_sq, part_s);
}

// Both kernels of one accumulation: partials into `partials` (capacity
// max_splits rows of the partial table), then the ordered finish.  (A single
// launch whose last CTA per column group runs the finish was measured slower:
// 37 us instead of 15 + 8 us for a 16384 x 768 FP32 call, the last CTA's
// serial sum over ~100 row splits outweighing the saved launch.)
template <typename T>
static int stats_run(const T* x, int64_t n_rows, int64_t n_cols, int64_t rs, int64_t cs, float* sum_sq, float* sum,
                     float* partials, int64_t max_splits, cudaStream_t st, int sms) {
  constexpr int kVec = 16 / sizeof(T);
  const bool vec_ok = cs == 1 && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                      ((rs * static_cast<int64_t>(sizeof(T))) % 16 == 0) && (n_cols % kVec == 0);
  const int vec = vec_ok ? kVec : 1;
  const StatsGeometry g = stats_geometry(n_rows, n_cols, vec, sms, max_splits);
  float* part_sq = partials;
  float* part_s = sum ? partials + static_cast<size_t>(g.splits) * n_cols : nullptr;
  if (vec_ok) {
    if (sum) colstats_partial<T, kVec, true>(g, x, n_rows, n_cols, rs, cs, part_sq, part_s, st);
    else colstats_partial<T, kVec, false>(g, x, n_rows, n_cols, rs, cs, part_sq, part_s, st);
  } else {
    if (sum) colstats_partial<T, 1, true>(g, x, n_rows, n_cols, rs, cs, part_sq, part_s, st);
    else colstats_partial<T, 1, false>(g, x, n_rows, n_cols, rs, cs, part_sq, part_s, st);
  }
  SM_LAUNCHED();
  k_colstats_finish<<<static_cast<unsigned>(cdiv(n_cols, 32)), 256, 0, st>>>(part_sq, part_s,
                                                                          static_cast<int>(g.splits), n_cols,
                                                                          sum_sq, sum);
  SM_LAUNCHED();
  return SM_OK;
}

// ------------------------------------- statistics in one cluster launch
#ifndef SMB_STATS_CLUSTER
#define SMB_STATS_CLUSTER 1
#endif
// k_colstats_cluster for contiguous rows with 16-byte-aligned starts and
// n_cols a multiple of the vector width: a cluster of `cl` CTAs per 128-byte
// column slab, cl a power of two <= 16 chosen for about two CTAs per SM
// (<= 8 where the device cannot co-schedule 16-CTA clusters of this kernel).
static int stats_cluster_max(int* out) {
  static int cached[64] = {};
  int dev = 0;
  SM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(SM_ERR_UNSUPPORTED, "device ordinal out of range");
  if (cached[dev] == 0) {
    auto kern = k_colstats_cluster<float, true>;
    int best = 8;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
      cudaLaunchConfig_t cfg;
      memset(&cfg, 0, sizeof(cfg));
      cudaLaunchAttribute attr;
      memset(&attr, 0, sizeof(attr));
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 16;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.gridDim = dim3(16);
      cfg.blockDim = dim3(256);
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) best = 16;
    }
    cudaGetLastError();  // a refused query leaves no error behind
    cached[dev] = best;
  }
  *out = cached[dev];
  return SM_OK;
}

template <typename T, bool FIRST>
static int stats_cluster_run(const T* x, int64_t n_rows, int64_t n_cols, int64_t rs, float* sum_sq, float* sum,
                             cudaStream_t st, int sms) {
  constexpr int kSlab = 8 * (16 / static_cast<int>(sizeof(T)));
  const int64_t slabs = cdiv(n_cols, kSlab);
  int cmax = 8;
  SM_TRY(stats_cluster_max(&cmax));
  int cl = 1;
  while (cl < cmax && slabs * cl < 2 * static_cast<int64_t>(sms) && cl < n_rows) cl *= 2;
  if (slabs * cl > (int64_t{1} << 31) - 1) return fail(SM_ERR_ARG, "too many columns for the statistics grid");
  auto kern = k_colstats_cluster<T, FIRST>;
  static bool attr_done[64] = {};
  int dev = 0;
  SM_CUDA(cudaGetDevice(&dev));
  if (!attr_done[dev]) {
    SM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cudaLaunchAttribute attr;
  memset(&attr, 0, sizeof(attr));
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = static_cast<unsigned>(cl);
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(slabs * cl));
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  SM_CUDA(cudaLaunchKernelEx(&cfg, kern, x, n_rows, n_cols, rs, cl, sum_sq, sum));
  return SM_OK;
}

// Whether an input takes the one-launch cluster kernel.
template <typename T>
static bool stats_cluster_eligible(const T* x, int64_t n_cols, int64_t rs, int64_t cs) {
  constexpr int kVec = 16 / sizeof(T);
  return cs == 1 && rs >= n_cols && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
         ((rs * static_cast<int64_t>(sizeof(T))) % 16 == 0) && (n_cols % kVec == 0);
}

// Largest number of row splits any input geometry of this shape may use.
static int64_t stats_max_splits(int64_t n_rows, int64_t n_cols, int sms) {
  int64_t splits = 0;
  for (int vec : {1, 2, 4, 8})
    splits = std::max(splits, stats_geometry(n_rows, n_cols, vec, sms, INT64_MAX).splits);
  return splits;
}

// --------------------------------------------------- TMA statistics path
// Contiguous, 16-byte-aligned inputs of at least SMB_STATS_TMA_MIN_MB take
// the single-reduction-launch TMA kernel (k_colstats_tma); smaller or other
// layouts the two-kernel path above.  Measured per call on B200 as fixed
// cost + bytes / rate: TMA ~10 us + bytes / 6.5-6.8 TB/s, two-kernel
// ~6.3 us + bytes / 5.3-6.0 TB/s, so the TMA kernel wins from ~128 MB.  A
// workspace starts with kStatsTicketWords tickets, then the partial rows.
// The tickets a call uses are zeroed in stream order before its kernel (a
// caller workspace may hold anything); the kernel leaves them zero.
#ifndef SMB_STATS_TMA_MIN_MB
#define SMB_STATS_TMA_MIN_MB 128
#endif

// Box rows: kStatsCols x rows = SMB_STATS_BOX_KB kilobytes.
#ifndef SMB_STATS_BOX_KB
#define SMB_STATS_BOX_KB 32
#endif
template <typename T>
struct StatsTmaType;
template <>
struct StatsTmaType<float> {
  static constexpr int kRows = SMB_STATS_BOX_KB * 1024 / (kStatsCols * 4);
  static constexpr CUtensorMapDataType kType = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
};
template <>
struct StatsTmaType<__nv_bfloat16> {
  static constexpr int kRows = SMB_STATS_BOX_KB * 1024 / (kStatsCols * 2);
  static constexpr CUtensorMapDataType kType = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
};
template <>
struct StatsTmaType<__half> {
  static constexpr int kRows = SMB_STATS_BOX_KB * 1024 / (kStatsCols * 2);
  static constexpr CUtensorMapDataType kType = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
};
template <>
struct StatsTmaType<double> {
  static constexpr int kRows = SMB_STATS_BOX_KB * 1024 / (kStatsCols * 8);
  static constexpr CUtensorMapDataType kType = CU_TENSOR_MAP_DATA_TYPE_FLOAT64;
};

struct StatsTmaGeometry {
  int groups = 0, splits = 0, row_blocks = 0;
};

// One CTA per SM: the column groups share the SMs, each taking an equal
// slice of the row blocks.
static StatsTmaGeometry stats_tma_geometry(int64_t n_rows, int64_t n_cols, int rows_per_box, int sms) {
  StatsTmaGeometry g;
  g.groups = static_cast<int>(cdiv(n_cols, kStatsCols));
  g.row_blocks = static_cast<int>(cdiv(n_rows, rows_per_box));
  g.splits = std::max(1, std::min(sms / std::max(1, g.groups), g.row_blocks));
  return g;
}

template <typename T>
static bool stats_tma_eligible(const T* x, int64_t n_rows, int64_t n_cols, int64_t rs, int64_t cs) {
  const int64_t row_bytes = rs * static_cast<int64_t>(sizeof(T));
  return cs == 1 && rs >= n_cols && (reinterpret_cast<uintptr_t>(x) % 16 == 0) && row_bytes % 16 == 0 &&
         row_bytes < (int64_t{1} << 40) && n_rows < (int64_t{1} << 31) &&
         cdiv(n_cols, kStatsCols) <= kStatsTicketWords;
}

// Partial floats the TMA path needs for this shape (0: not eligible).
static int64_t stats_tma_partial_floats(int64_t n_rows, int64_t n_cols, int rows_per_box, int sms) {
  const StatsTmaGeometry g = stats_tma_geometry(n_rows, n_cols, rows_per_box, sms);
  return static_cast<int64_t>(g.groups) * g.splits * kStatsCols * 2;
}

template <typename T, bool FIRST>
static int stats_tma_launch(const CUtensorMap& map, const StatsTmaArgs& args, int grid, cudaStream_t st) {
  constexpr int BR = StatsTmaType<T>::kRows;
  auto kern = k_colstats_tma<T, FIRST, BR>;
  static bool attr_done[64] = {};
  int dev = 0;
  SM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(SM_ERR_UNSUPPORTED, "device ordinal out of range");
  if (!attr_done[dev]) {
    SM_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, StatsTmaSmem<T, BR>::kBytes));
    attr_done[dev] = true;
  }
  kern<<<grid, kStatsThreads, StatsTmaSmem<T, BR>::kBytes, st>>>(map, args);
  SM_LAUNCHED();
  return SM_OK;
}

// Runs the TMA path when the input qualifies and the partial capacity
// suffices; *done says whether it ran.
// zero_tickets: clear the call's tickets first, in stream order.
template <typename T>
static int stats_tma_run(const T* x, int64_t n_rows, int64_t n_cols, int64_t rs, int64_t cs, float* sum_sq,
                         float* sum, unsigned* tickets, bool zero_tickets, float* partials, int64_t partial_floats,
                         cudaStream_t st, int sms, bool* done) {
  *done = false;
  if (!stats_tma_eligible(x, n_rows, n_cols, rs, cs)) return SM_OK;
  if (n_rows * n_cols * static_cast<int64_t>(sizeof(T)) < (int64_t{SMB_STATS_TMA_MIN_MB} << 20)) return SM_OK;
  constexpr int BR = StatsTmaType<T>::kRows;
  StatsTmaGeometry g = stats_tma_geometry(n_rows, n_cols, BR, sms);
  const int64_t per_split = static_cast<int64_t>(g.groups) * kStatsCols * (sum ? 2 : 1);
  if (per_split > partial_floats) return SM_OK;
  g.splits = static_cast<int>(std::min<int64_t>(g.splits, partial_floats / per_split));
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  SM_TRY(get_encode(&enc));
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(n_cols), static_cast<cuuint64_t>(n_rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(rs * static_cast<int64_t>(sizeof(T)))};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kStatsCols), static_cast<cuuint32_t>(BR)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&map, StatsTmaType<T>::kType, 2, const_cast<T*>(x), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SM_ERR_CUDA, "cuTensorMapEncodeTiled (statistics) failed: " + std::to_string(r));
  StatsTmaArgs a;
  a.n_cols = n_cols;
  a.groups = g.groups;
  a.splits = g.splits;
  a.row_blocks = g.row_blocks;
  a.part_sq = partials;
  a.part_sum = sum ? partials + static_cast<int64_t>(g.groups) * g.splits * kStatsCols : nullptr;
  a.tickets = tickets;
  a.sum_sq = sum_sq;
  a.sum = sum;
  const int grid = g.groups * g.splits;
  if (zero_tickets) SM_CUDA(cudaMemsetAsync(tickets, 0, sizeof(unsigned) * g.groups, st));
  if (sum) SM_TRY((stats_tma_launch<T, true>(map, a, grid, st)));
  else SM_TRY((stats_tma_launch<T, false>(map, a, grid, st)));
  *done = true;
  return SM_OK;
}

template <typename T>
static int stats_launch(const T* x, int64_t n_rows, int64_t n_cols, int64_t rs, int64_t cs, float* sum_sq,
                        float* sum, void* ws, size_t ws_bytes, cudaStream_t st, int sms) {
  if (ws == nullptr || ws_bytes < kStatsTicketBytes) return fail(SM_ERR_WORKSPACE, "statistics workspace too small");
  unsigned* tickets = static_cast<unsigned*>(ws);
  float* partials = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + kStatsTicketBytes);
  const int64_t cap = static_cast<int64_t>((ws_bytes - kStatsTicketBytes) / sizeof(float));
  bool done = false;
  SM_TRY(stats_tma_run(x, n_rows, n_cols, rs, cs, sum_sq, sum, tickets, true, partials, cap, st, sms, &done));
  if (done) return SM_OK;
  if (SMB_STATS_CLUSTER && stats_cluster_eligible(x, n_cols, rs, cs))
    return sum ? stats_cluster_run<T, true>(x, n_rows, n_cols, rs, sum_sq, sum, st, sms)
               : stats_cluster_run<T, false>(x, n_rows, n_cols, rs, sum_sq, sum, st, sms);
  const int64_t per_split = n_cols * (sum ? 2 : 1);
  const int64_t max_splits = cap / per_split;
  if (max_splits < stats_max_splits(n_rows, n_cols, sms)) return fail(SM_ERR_WORKSPACE, "statistics workspace too small");
  return stats_run(x, n_rows, n_cols, rs, cs, sum_sq, sum, partials, max_splits, st, sms);
}

// ------------------------------------------ statistics without a workspace
// Library-owned scratch for sm_stats_accumulate_noalloc: the per-split
// partial sums live here instead of in a caller workspace.  One copy per
// device, kept until the process exits.  Host code must not use the symbol as
// a pointer: its device address comes from cudaGetSymbolAddress, looked up
// once per device with that device current.
static __device__ __align__(256) float g_noalloc_scratch[SM_STATS_NOALLOC_SCRATCH_FLOATS];
// last-CTA tickets of the TMA path; each call clears the ones it uses
// (cudaMemsetAsync, in stream order) before its kernel, so a ticket left
// non-zero by two overlapping calls cannot affect later ones
static __device__ __align__(256) unsigned g_noalloc_tickets[kStatsTicketWords];
static std::mutex g_noalloc_mutex;
static float* g_noalloc_addr[64] = {};
static unsigned* g_noalloc_ticket_addr[64] = {};

static int noalloc_scratch_address(float** out, unsigned** tickets) {
  int dev = 0;
  SM_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(SM_ERR_UNSUPPORTED, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    void* q = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&q, g_noalloc_tickets);
    if (e != cudaSuccess || p == nullptr || q == nullptr)
      return fail(SM_ERR_CUDA, std::string("cudaGetSymbolAddress(noalloc scratch): ") + cudaGetErrorString(e));
    g_noalloc_addr[dev] = static_cast<float*>(p);
    g_noalloc_ticket_addr[dev] = static_cast<unsigned*>(q);
  }
  *out = g_noalloc_addr[dev];
  *tickets = g_noalloc_ticket_addr[dev];
  return SM_OK;
}

// Same kernels as stats_launch; the number of row splits is capped so the
// partials fit the fixed scratch array.  Every partial is written before it
// is read, so stale contents never leak; the TMA path's tickets are cleared
// by each call (a memset allocates nothing).
template <typename T>
static int stats_launch_noalloc(const T* x, int64_t n_rows, int64_t n_cols, int64_t rs, int64_t cs, float* sum_sq,
                                float* sum, float* scratch, unsigned* tickets, cudaStream_t st, int sms) {
  bool done = false;
  SM_TRY(stats_tma_run(x, n_rows, n_cols, rs, cs, sum_sq, sum, tickets, true, scratch,
                       static_cast<int64_t>(SM_STATS_NOALLOC_SCRATCH_FLOATS), st, sms, &done));
  if (done) return SM_OK;
  if (SMB_STATS_CLUSTER && stats_cluster_eligible(x, n_cols, rs, cs))
    return sum ? stats_cluster_run<T, true>(x, n_rows, n_cols, rs, sum_sq, sum, st, sms)
               : stats_cluster_run<T, false>(x, n_rows, n_cols, rs, sum_sq, sum, st, sms);
  const int64_t per_split = n_cols * (sum ? 2 : 1);
  const int64_t cap = static_cast<int64_t>(SM_STATS_NOALLOC_SCRATCH_FLOATS) / per_split;
  if (cap < 1) return fail(SM_ERR_ARG, "too many columns for the no-allocation scratch");
  return stats_run(x, n_rows, n_cols, rs, cs, sum_sq, sum, scratch, cap, st, sms);
}

// Layout: Group buffers, then MatDev table [batch], ones [max(rows, cols)].
static int s8_layout(int32_t batch, int32_t rows, int32_t cols, bool pair_ok, void* ws, Group* g, MatDev** d_mats,
                     float** ones, size_t* bytes) {
  Carver cv(ws);
  init_group_shape(*g, std::min(rows, cols), std::max(rows, cols), batch, pair_ok);
  g->rank1 = false;
  g->mat_off = 0;
  *d_mats = cv.take<MatDev>(batch);
  *ones = cv.take<float>(std::max(rows, cols));
  carve_group(cv, *g);
  *bytes = round_up(static_cast<int64_t>(cv.off), 256);
  return SM_OK;
}

}  // namespace smb

// =============================================================== C-ABI

extern "C" {

int sm_version(void) { return SM_ABI_VERSION; }

const char* sm_last_error(void) { return t_last_error.c_str(); }

int sm_init_device(void) {
  DeviceInfo* di;
  return current_device_info(&di);
}

int sm_device_status(int* status_out, void* stream) {
  if (status_out == nullptr) return fail(SM_ERR_ARG, "null status_out");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0, zero = 0;
  SM_CUDA(cudaMemcpyFromSymbolAsync(&v, g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st));
  SM_CUDA(cudaMemcpyToSymbolAsync(g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st));
  SM_CUDA(cudaStreamSynchronize(st));
  *status_out = v;
  return SM_OK;
}

// ------------------------------------------------------------ N1 stats

size_t sm_stats_workspace_bytes(int64_t n_rows, int64_t n_cols) {
  if (n_rows <= 0 || n_cols <= 0) return 0;
  int sms = 148;
  DeviceInfo* di;
  if (current_device_info(&di) == SM_OK) sms = di->sms;
  int64_t floats = stats_max_splits(n_rows, n_cols, sms) * n_cols * 2;
  for (int rows_per_box : {StatsTmaType<double>::kRows, StatsTmaType<float>::kRows, StatsTmaType<__half>::kRows})
    floats = std::max(floats, stats_tma_partial_floats(n_rows, n_cols, rows_per_box, sms));
  return kStatsTicketBytes + static_cast<size_t>(floats) * sizeof(float);
}

int sm_stats_accumulate(const void* rows, int dtype, int64_t n_rows, int64_t n_cols, int64_t row_stride,
                        int64_t col_stride, float* sum_sq, float* sum, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (n_rows < 0 || n_cols < 0) return fail(SM_ERR_ARG, "negative shape");
  if (n_rows == 0 || n_cols == 0) return SM_OK;
  if (rows == nullptr || sum_sq == nullptr) return fail(SM_ERR_ARG, "null input or output");
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SM_DTYPE_F32:
      return stats_launch(static_cast<const float*>(rows), n_rows, n_cols, row_stride, col_stride, sum_sq, sum,
                          workspace, workspace_bytes, st, di->sms);
    case SM_DTYPE_BF16:
      return stats_launch(static_cast<const __nv_bfloat16*>(rows), n_rows, n_cols, row_stride, col_stride, sum_sq,
                          sum, workspace, workspace_bytes, st, di->sms);
    case SM_DTYPE_F16:
      return stats_launch(static_cast<const __half*>(rows), n_rows, n_cols, row_stride, col_stride, sum_sq, sum,
                          workspace, workspace_bytes, st, di->sms);
    case SM_DTYPE_F64:
      return stats_launch(static_cast<const double*>(rows), n_rows, n_cols, row_stride, col_stride, sum_sq, sum,
                          workspace, workspace_bytes, st, di->sms);
    default:
      return fail(SM_ERR_ARG, "unsupported dtype code " + std::to_string(dtype));
  }
}

int sm_stats_accumulate_noalloc(const void* rows, int dtype, int64_t n_rows, int64_t n_cols, int64_t row_stride,
                                int64_t col_stride, float* sum_sq, float* sum, void* stream) {
  if (n_rows < 0 || n_cols < 0) return fail(SM_ERR_ARG, "negative shape");
  if (n_cols > SM_STATS_NOALLOC_MAX_COLS)
    return fail(SM_ERR_ARG, "sm_stats_accumulate_noalloc supports at most " +
                                std::to_string(SM_STATS_NOALLOC_MAX_COLS) + " columns; got " + std::to_string(n_cols) +
                                " (use sm_stats_accumulate with a caller workspace)");
  if (n_rows == 0 || n_cols == 0) return SM_OK;
  if (rows == nullptr || sum_sq == nullptr) return fail(SM_ERR_ARG, "null input or output");
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  float* scratch = nullptr;
  unsigned* tickets = nullptr;
  SM_TRY(noalloc_scratch_address(&scratch, &tickets));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SM_DTYPE_F32:
      return stats_launch_noalloc(static_cast<const float*>(rows), n_rows, n_cols, row_stride, col_stride, sum_sq,
                                  sum, scratch, tickets, st, di->sms);
    case SM_DTYPE_BF16:
      return stats_launch_noalloc(static_cast<const __nv_bfloat16*>(rows), n_rows, n_cols, row_stride, col_stride,
                                  sum_sq, sum, scratch, tickets, st, di->sms);
    case SM_DTYPE_F16:
      return stats_launch_noalloc(static_cast<const __half*>(rows), n_rows, n_cols, row_stride, col_stride, sum_sq,
                                  sum, scratch, tickets, st, di->sms);
    case SM_DTYPE_F64:
      return stats_launch_noalloc(static_cast<const double*>(rows), n_rows, n_cols, row_stride, col_stride, sum_sq,
                                  sum, scratch, tickets, st, di->sms);
    default:
      return fail(SM_ERR_ARG, "unsupported dtype code " + std::to_string(dtype));
  }
}

// ------------------------------------------------------------------ plan

int sm_plan_workspace_bytes(const SmPlanSpec* spec, size_t* bytes_out) {
  if (bytes_out == nullptr) return fail(SM_ERR_ARG, "null bytes_out");
  return plan_layout(spec, nullptr, nullptr, bytes_out);
}

int sm_plan_create(const SmPlanSpec* spec, void* workspace, size_t workspace_bytes, void* stream,
                   SmPlan** plan_out) {
  if (plan_out == nullptr) return fail(SM_ERR_ARG, "null plan_out");
  *plan_out = nullptr;
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(SM_ERR_ARG, "workspace must be a 256-byte aligned device pointer");
  if (spec == nullptr || (spec->export_mode != SM_EXPORT_WEIGHTS && spec->export_mode != SM_EXPORT_BF16_DELTA))
    return fail(SM_ERR_ARG, "null plan spec or unknown export mode");
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  for (int i = 0; i < spec->n_matrices; ++i) {
    const SmMatrixSpec& m = spec->matrices[i];
    if (m.weight == nullptr || m.momentum == nullptr) return fail(SM_ERR_ARG, "null weight or momentum");
  }
  for (int s = 0; s < spec->n_stats; ++s) {
    const SmStatSpec& st = spec->stats[s];
    if (st.sum == nullptr || st.ema == nullptr) return fail(SM_ERR_ARG, "null statistic buffer");
    if (st.kind == SM_STAT_A_RANK1 && (st.first_sum == nullptr || st.mean_ema == nullptr))
      return fail(SM_ERR_ARG, "rank-one statistic without first-moment buffers");
  }
  size_t need = 0;
  SM_TRY(plan_layout(spec, nullptr, nullptr, &need));
  if (workspace_bytes < need) return fail(SM_ERR_WORKSPACE, "plan workspace too small");
  SmPlan* p = new SmPlan();
  int rc = plan_layout(spec, workspace, p, &need);
  if (rc == SM_OK) {
    SM_CUDA(cudaGetDevice(&p->device));
    p->stat_beta = spec->statistic_beta;
    p->stat_omb = static_cast<float>(1.0 - static_cast<double>(spec->statistic_beta));
    p->mom_beta = spec->momentum;
    p->export_mode = spec->export_mode;
    p->mom_omb = static_cast<float>(1.0 - static_cast<double>(spec->momentum));
    // Zero the whole workspace once: padding of every S8 plane must be zero.
    cudaError_t e = cudaMemsetAsync(workspace, 0, need, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) rc = fail(SM_ERR_CUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
    for (auto& g : p->groups) {
      if (rc != SM_OK) break;
      rc = encode_group_maps(g);
      if (rc == SM_OK && g.fused_ok) rc = prepare_front_fused(g.rank1);
      if (rc == SM_OK && g.rows_ok) {
        DeviceInfo* di = nullptr;
        rc = current_device_info(&di);
        if (rc == SM_OK) rc = prepare_front_rows(g, di->sms);
      }
      if (rc == SM_OK && g.cols_ok) {
        DeviceInfo* di = nullptr;
        rc = current_device_info(&di);
        if (rc == SM_OK) rc = prepare_front_cols(g, di->sms);
      }
    }
    for (size_t gi = 0; gi < p->groups.size() && rc == SM_OK; ++gi) {
      Group& g = p->groups[gi];
      g.host_tmask.assign(g.batch, 0);
      for (int i = 0; i < spec->n_matrices; ++i)
        if (p->mat_group[i] == static_cast<int>(gi))
          g.host_tmask[p->mat_slot[i]] = spec->matrices[i].d_out > spec->matrices[i].d_in ? 1 : 0;
      e = cudaMemcpyAsync(g.tmask, g.host_tmask.data(), g.batch * sizeof(int), cudaMemcpyHostToDevice,
                          static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) rc = fail(SM_ERR_CUDA, std::string("tmask upload: ") + cudaGetErrorString(e));
      if (rc == SM_OK && g.rows_count > 0) {
        e = cudaMemcpyAsync(g.rows_slots, g.host_rows_slots.data(), g.rows_count * sizeof(int),
                            cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) rc = fail(SM_ERR_CUDA, std::string("row slot upload: ") + cudaGetErrorString(e));
      }
      if (rc == SM_OK && g.cols_count > 0) {
        e = cudaMemcpyAsync(g.cols_slots, g.host_cols_slots.data(), g.cols_count * sizeof(int),
                            cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) rc = fail(SM_ERR_CUDA, std::string("block slot upload: ") + cudaGetErrorString(e));
      }
    }
    for (int kind = 0; kind < 3 && rc == SM_OK; ++kind) {
      for (const LaunchSet& set : p->s8.sets[kind]) {
        if (set.sched == nullptr || set.h_sched.empty()) continue;
        e = cudaMemcpyAsync(set.sched, set.h_sched.data(), set.h_sched.size() * sizeof(int), cudaMemcpyHostToDevice,
                            static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) {
          rc = fail(SM_ERR_CUDA, std::string("schedule upload: ") + cudaGetErrorString(e));
          break;
        }
      }
    }
    p->h_table.resize(p->table_bytes);
    if (rc == SM_OK) {
      e = cudaStreamCreateWithFlags(&p->cap_stream, cudaStreamNonBlocking);
      if (e != cudaSuccess) rc = fail(SM_ERR_CUDA, std::string("capture stream: ") + cudaGetErrorString(e));
    }
  }
  if (rc != SM_OK) {
    sm_plan_destroy(p);
    return rc;
  }
  *plan_out = p;
  return SM_OK;
}

static int launch_step(SmPlan* p, const std::vector<uint8_t>& vec4, bool first, cudaStream_t st, Timer* tm,
                       int64_t* out);

int sm_plan_step(SmPlan* p, const SmStepArgs* args, void* stream) {
  if (p == nullptr || args == nullptr || args->grads == nullptr || args->lrs == nullptr || args->counts == nullptr ||
      args->ema_init == nullptr)
    return fail(SM_ERR_ARG, "null plan or step argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nm = static_cast<int>(p->mats.size());
  const int ns = static_cast<int>(p->stats.size());
  Timer* tm = p->timer.enabled ? &p->timer : nullptr;
  int64_t launches = 0;

  // ---- host table: per-matrix descriptors in group/slot order + statistics
  MatDev* hm = reinterpret_cast<MatDev*>(p->h_table.data());
  StatDev* hs = reinterpret_cast<StatDev*>(p->h_table.data() +
                                          (reinterpret_cast<uint8_t*>(p->d_stats) - reinterpret_cast<uint8_t*>(p->d_mats)));
  std::vector<uint8_t> vec4(p->groups.size(), 1);
  for (int t = 0; t < nm; ++t) {
    const int i = p->order[t];
    const SmMatrixSpec& m = p->mats[i];
    if (args->grads[i] == nullptr) return fail(SM_ERR_ARG, "null gradient for matrix " + std::to_string(i));
    MatDev& d = hm[t];
    memset(&d, 0, sizeof(d));
    d.grad = args->grads[i];
    d.mom = m.momentum;
    d.weight = m.weight;
    d.export_to = m.export_to;
    d.export_bf16 = (p->export_mode == SM_EXPORT_BF16_DELTA && m.export_to != nullptr) ? 1 : 0;
    {
      const char* w = reinterpret_cast<const char*>(m.weight);
      const int64_t wbytes = static_cast<int64_t>(m.d_out) * m.d_in * 4;
      d.peer = (p->peers.n > 0 && w >= p->peer_lo && w + wbytes <= p->peer_hi) ? 1 : 0;
    }
    d.inv_a = p->s_inv[m.a_stat];
    d.z_a = p->s_z[m.a_stat];
    d.zeta_a = p->s_zeta[m.a_stat];
    d.scal_a = p->s_scal[m.a_stat];
    d.inv_b = p->s_inv[m.b_stat];
    d.d_out = m.d_out;
    d.d_in = m.d_in;
    d.transposed = m.d_out > m.d_in ? 1 : 0;
    d.slot = p->mat_slot[i];
    d.lr = args->lrs[i];
    d.sqrt_rows = static_cast<float>(std::sqrt(static_cast<double>(m.d_out)));
    const bool aligned = (m.d_in % 4 == 0) && (reinterpret_cast<uintptr_t>(d.grad) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(d.mom) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(d.weight) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(d.export_to) % (d.export_bf16 ? 8 : 16) == 0);
    if (!aligned) vec4[p->mat_group[i]] = 0;
  }
  for (int s = 0; s < ns; ++s) {
    const SmStatSpec& sp = p->stats[s];
    if (args->counts[s] < 1) return fail(SM_ERR_ARG, "statistic " + std::to_string(s) + " has no rows");
    StatDev& d = hs[s];
    memset(&d, 0, sizeof(d));
    d.sum = sp.sum;
    d.first_sum = sp.first_sum;
    d.ema = sp.ema;
    d.mean_ema = sp.mean_ema;
    d.inv = p->s_inv[s];
    d.z = p->s_z[s];
    d.zeta = p->s_zeta[s];
    d.scal = p->s_scal[s];
    d.count = args->counts[s];
    d.count_dev = args->device_counts != nullptr ? args->device_counts + s : nullptr;
    d.n = sp.n;
    d.kind = sp.kind;
    d.init = args->ema_init[s] ? 1 : 0;
  }
  // A caller's graph capture would freeze this step's arguments (uploaded
  // from host memory below) into every replay: refuse it.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  SM_CUDA(cudaStreamIsCapturing(st, &cap));
  if (cap != cudaStreamCaptureStatusNone)
    return fail(SM_ERR_UNSUPPORTED, "sm_plan_step cannot be captured into a CUDA graph: its per-step "
                                    "arguments are uploaded from host memory at call time");
  // Pageable source on purpose: the runtime stages this small table through
  // the command stream before returning (so h_table may be rewritten at
  // once), where a pinned source would queue on a copy engine behind any
  // bulk host-to-device copy the caller has in flight on another stream.
  SM_CUDA(cudaMemcpyAsync(p->d_mats, p->h_table.data(), p->table_bytes, cudaMemcpyHostToDevice, st));

  const bool use_graph = p->replay && tm == nullptr && p->steps_done > 0;
  const bool first = p->steps_done == 0;
  ++p->steps_done;
  if (use_graph) {
    if (p->exec != nullptr && p->exec_vec4 != vec4) {
      SM_CUDA(cudaGraphExecDestroy(p->exec));
      p->exec = nullptr;
    }
    if (p->exec == nullptr) {
      int64_t n = 0;
      SM_CUDA(cudaStreamBeginCapture(p->cap_stream, cudaStreamCaptureModeThreadLocal));
      const int rc = launch_step(p, vec4, false, p->cap_stream, nullptr, &n);
      cudaGraph_t graph = nullptr;
      const cudaError_t e = cudaStreamEndCapture(p->cap_stream, &graph);
      if (rc != SM_OK) {
        if (graph != nullptr) cudaGraphDestroy(graph);
        return rc;
      }
      if (e != cudaSuccess) return fail(SM_ERR_CUDA, std::string("step capture: ") + cudaGetErrorString(e));
      const cudaError_t ei = cudaGraphInstantiate(&p->exec, graph, 0);
      cudaGraphDestroy(graph);
      if (ei != cudaSuccess) {
        p->exec = nullptr;
        return fail(SM_ERR_CUDA, std::string("step graph instantiate: ") + cudaGetErrorString(ei));
      }
      p->exec_vec4 = vec4;
      p->exec_launches = n;
    }
    SM_CUDA(cudaGraphLaunch(p->exec, st));
    p->launches_last = p->exec_launches;
    return SM_OK;
  }
  SM_TRY(launch_step(p, vec4, first, st, tm, &launches));
  p->launches_last = launches;
  return SM_OK;
}

// Every kernel of one step, in stream order on `st`.  `first`: the plan's
// first step (the two-pass front end; see run_front).
static int launch_step(SmPlan* p, const std::vector<uint8_t>& vec4, bool first, cudaStream_t st, Timer* tm,
                       int64_t* out) {
  const int ns = static_cast<int>(p->stats.size());
  int64_t launches = 0;
  // The first kernel follows the descriptor upload in plain stream order;
  // every later one may launch early (programmatic dependent launch).
  PdlScope plain(false);
  SM_TIMED(tm, SM_TCLASS_STATS, 0.0, st, ([&]() -> int {
             if (ns > 0) SM_TRY(launch_kernel(k_stats_finish, dim3(ns), dim3(256), 0, st, p->d_stats,
                                              p->stat_beta, p->stat_omb));
             return SM_OK;
           }()));
  ++launches;
  PdlScope rest(p->pdl);
  for (size_t gi = 0; gi < p->groups.size(); ++gi)
    SM_TRY(run_front(p->groups[gi], p->d_mats, p->mom_beta, p->mom_omb, vec4[gi] != 0, !first, st, tm,
                     &launches));
  SM_TRY(run_s8(p->groups, p->s8, st, tm, &launches));
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  for (size_t gi = 0; gi < p->groups.size(); ++gi)
    SM_TRY(run_back(p->groups[gi], p->d_mats, vec4[gi] != 0, di->sms, p->peers, st, tm, &launches));
  *out = launches;
  return SM_OK;
}

int sm_plan_set_replay(SmPlan* p, int enabled) {
  if (p == nullptr) return fail(SM_ERR_ARG, "null plan");
  p->replay = enabled != 0;
  return SM_OK;
}

int sm_plan_set_timing(SmPlan* p, int enabled) {
  if (p == nullptr) return fail(SM_ERR_ARG, "null plan");
  p->timer.enabled = enabled != 0;
  return SM_OK;
}

int sm_plan_timing_read(SmPlan* p, double* ms_out, int64_t* launches_out, double* gemm_flops_out) {
  if (p == nullptr || ms_out == nullptr || launches_out == nullptr) return fail(SM_ERR_ARG, "null argument");
  for (int c = 0; c < SM_TCLASS_COUNT; ++c) {
    ms_out[c] = 0.0;
    launches_out[c] = 0;
  }
  double flops = 0.0;
  if (!p->timer.recs.empty()) SM_CUDA(cudaEventSynchronize(p->timer.recs.back().b));
  for (const auto& r : p->timer.recs) {
    float ms = 0.f;
    SM_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
    ms_out[r.cls] += ms;
    launches_out[r.cls] += 1;
    flops += r.flops;
  }
  if (gemm_flops_out != nullptr) *gemm_flops_out = flops;
  p->timer.recs.clear();
  p->timer.next = 0;
  return SM_OK;
}

int sm_plan_launches_per_step(const SmPlan* p, int64_t* out) {
  if (p == nullptr || out == nullptr) return fail(SM_ERR_ARG, "null argument");
  *out = p->launches_last;
  return SM_OK;
}

int sm_plan_destroy(SmPlan* p) {
  if (p == nullptr) return SM_OK;
  for (cudaEvent_t e : p->timer.pool) cudaEventDestroy(e);
  if (p->exec != nullptr) cudaGraphExecDestroy(p->exec);
  if (p->cap_stream != nullptr) cudaStreamDestroy(p->cap_stream);
  delete p;
  return SM_OK;
}

// -------------------------------------------------------------- S8 batch

size_t sm_s8_workspace_bytes(int32_t batch, int32_t rows, int32_t cols) {
  if (batch <= 0 || rows <= 0 || cols <= 0) return 0;
  Group g;
  MatDev* dm;
  float* ones;
  size_t bytes = 0;
  // Sized for single-CTA tiles, whose norm partials outnumber a pair's.
  s8_layout(batch, rows, cols, false, nullptr, &g, &dm, &ones, &bytes);
  return bytes;
}

int sm_s8_polar(const float* x, float* out, int32_t batch, int32_t rows, int32_t cols, void* workspace,
                size_t workspace_bytes, void* stream) {
  if (batch < 0 || rows < 0 || cols < 0) return fail(SM_ERR_ARG, "negative shape");
  if (batch == 0 || rows == 0 || cols == 0) return SM_OK;
  if (x == nullptr || out == nullptr) return fail(SM_ERR_ARG, "null input or output");
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(SM_ERR_ARG, "workspace must be a 256-byte aligned device pointer");
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  int pairs = 0;
  SM_TRY(pair_workers(di, &pairs));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Group g;
  MatDev* d_mats;
  float* ones;
  size_t need = 0;
  s8_layout(batch, rows, cols, pairs > 0, nullptr, &g, &d_mats, &ones, &need);
  if (workspace_bytes < need) return fail(SM_ERR_WORKSPACE, "S8 workspace too small");
  s8_layout(batch, rows, cols, pairs > 0, workspace, &g, &d_mats, &ones, &need);
  {
    std::vector<Group> one(1, g);
    choose_tilings(one, di->sms, pairs);
    g = one[0];
  }
  SM_TRY(encode_group_maps(g));
  SM_CUDA(cudaMemsetAsync(workspace, 0, need, st));
  const int64_t nmax = std::max(rows, cols);
  k_fill<<<static_cast<unsigned>(cdiv(nmax, 256)), 256, 0, st>>>(ones, nmax, 1.0f);
  SM_LAUNCHED();
  k_fill<<<1, 256, 0, st>>>(g.gamma, batch, 1.0f);
  SM_LAUNCHED();
  std::vector<MatDev> hm(batch);
  const int64_t per = static_cast<int64_t>(rows) * cols;
  bool vec4 = (cols % 4 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
  for (int b = 0; b < batch; ++b) {
    MatDev& d = hm[b];
    memset(&d, 0, sizeof(d));
    d.grad = x + b * per;
    d.mom = nullptr;  // S8 input is used as is (no momentum)
    d.weight = out + b * per;
    d.inv_a = ones;
    d.inv_b = ones;
    d.d_out = rows;
    d.d_in = cols;
    d.transposed = rows > cols ? 1 : 0;
    d.slot = b;
    d.lr = -1.0f;  // out = 0 - (-1) * 1 * Q
    d.sqrt_rows = 1.0f;
  }
  SM_CUDA(cudaMemcpyAsync(d_mats, hm.data(), sizeof(MatDev) * batch, cudaMemcpyHostToDevice, st));
  g.host_tmask.assign(batch, rows > cols ? 1 : 0);
  SM_CUDA(cudaMemcpyAsync(g.tmask, g.host_tmask.data(), sizeof(int) * batch, cudaMemcpyHostToDevice, st));
  int64_t launches = 0;
  SM_TRY(run_front(g, d_mats, 0.0f, 1.0f, vec4, false, st, nullptr, &launches));
  std::vector<Group> groups(1, g);
  S8Launches s8;
  build_s8_launches(groups, di->sms, pairs, nullptr, &s8);  // round-robin tiles: no schedule tables
  SM_TRY(run_s8(groups, s8, st, nullptr, &launches));
  SM_CUDA(cudaMemsetAsync(out, 0, sizeof(float) * batch * per, st));
  {
    const bool out_vec4 = vec4 && (reinterpret_cast<uintptr_t>(out) % 16 == 0);
    dim3 grid(static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(cdiv(per, 1024), 8 * di->sms))), batch);
    const PeerSet none{};  // hm[].peer is 0: no peer stores
    if (out_vec4)
      k_mapback_apply<false, true><<<grid, 256, 0, st>>>(d_mats, g.q, g.rp, g.cp, g.rs_map, g.dmax, g.gamma, none);
    else
      k_mapback_apply<false, false><<<grid, 256, 0, st>>>(d_mats, g.q, g.rp, g.cp, g.rs_map, g.dmax, g.gamma, none);
    SM_LAUNCHED();
  }
  return SM_OK;
}

int sm_s8_executed_flops(int32_t batch, int32_t rows, int32_t cols, double* flops_out) {
  if (flops_out == nullptr) return fail(SM_ERR_ARG, "null output");
  *flops_out = 0.0;
  if (batch < 0 || rows < 0 || cols < 0) return fail(SM_ERR_ARG, "negative shape");
  if (batch == 0 || rows == 0 || cols == 0) return SM_OK;
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  int pairs = 0;
  SM_TRY(pair_workers(di, &pairs));
  std::vector<Group> one(1);
  init_group_shape(one[0], std::min(rows, cols), std::max(rows, cols), batch, pairs > 0);
  choose_tilings(one, di->sms, pairs);
  const Group& g = one[0];
  double total = 0.0;
  for (int stage = 0; stage < 5; ++stage) {
    for (int kind = 0; kind < 3; ++kind) {
      int epi = -1;
      const GemmProblem p = s8_problem(g, kind, stage, kind_bn(g, kind), &epi);
      total += problem_flops(p, stage < kCompensatedStages);
    }
  }
  *flops_out = total;
  return SM_OK;
}

// ------------------------------------------------------- multi-tensor copy

int sm_copy_multi(const SmCopySpec* copies, int32_t count, void* stream) {
  if (count < 0 || (count > 0 && copies == nullptr)) return fail(SM_ERR_ARG, "bad copy list");
  if (count == 0) return SM_OK;
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int start = 0; start < count; start += kCopyMax) {
    CopyBatch b;
    memset(&b, 0, sizeof(b));
    b.count = std::min(kCopyMax, count - start);
    for (int t = 0; t < b.count; ++t) {
      const SmCopySpec& c = copies[start + t];
      if (c.bytes < 0 || (c.bytes > 0 && (c.dst == nullptr || c.src == nullptr)))
        return fail(SM_ERR_ARG, "bad copy " + std::to_string(start + t));
      b.dst[t] = static_cast<uint8_t*>(c.dst);
      b.src[t] = static_cast<const uint8_t*>(c.src);
      b.bytes[t] = c.bytes;
      b.chunk_start[t + 1] = b.chunk_start[t] + cdiv(c.bytes, kCopyChunk);
    }
    const int64_t chunks = b.chunk_start[b.count];
    if (chunks == 0) continue;
    k_copy_multi<<<static_cast<int>(std::min<int64_t>(chunks, 8 * di->sms)), 256, 0, st>>>(b);
    SM_LAUNCHED();
  }
  return SM_OK;
}

// ------------------------------------------------------- BF16 delta apply

int sm_apply_bf16_delta_multi(const SmDeltaSpec* items, int32_t count, void* stream) {
  if (count < 0 || (count > 0 && items == nullptr)) return fail(SM_ERR_ARG, "bad delta list");
  if (count == 0) return SM_OK;
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int start = 0; start < count; start += kCopyMax) {
    DeltaBatch b;
    memset(&b, 0, sizeof(b));
    b.count = std::min(kCopyMax, count - start);
    for (int t = 0; t < b.count; ++t) {
      const SmDeltaSpec& c = items[start + t];
      if (c.numel < 0 || (c.numel > 0 && (c.weight == nullptr || c.delta == nullptr)))
        return fail(SM_ERR_ARG, "bad delta entry " + std::to_string(start + t));
      b.weight[t] = c.weight;
      b.delta[t] = static_cast<const __nv_bfloat16*>(c.delta);
      b.numel[t] = c.numel;
      b.chunk_start[t + 1] = b.chunk_start[t] + cdiv(c.numel, kDeltaChunk);
    }
    const int64_t chunks = b.chunk_start[b.count];
    if (chunks == 0) continue;
    k_apply_bf16_delta<<<static_cast<int>(std::min<int64_t>(chunks, 8 * di->sms)), 256, 0, st>>>(b);
    SM_LAUNCHED();
  }
  return SM_OK;
}

// ------------------------------------------------------------------ AdamW

int sm_adamw_multi(const SmAdamTensor* tensors, int32_t count, float lr, float beta1, float beta2, float eps,
                   float decay_factor, void* stream) {
  if (count < 0 || (count > 0 && tensors == nullptr)) return fail(SM_ERR_ARG, "bad tensor list");
  if (count == 0) return SM_OK;
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float omb1 = static_cast<float>(1.0 - static_cast<double>(beta1));
  const float omb2 = static_cast<float>(1.0 - static_cast<double>(beta2));
  for (int start = 0; start < count; start += kAdamMaxTensors) {
    AdamBatch b;
    memset(&b, 0, sizeof(b));
    b.count = std::min(kAdamMaxTensors, count - start);
    b.chunk_start[0] = 0;
    for (int t = 0; t < b.count; ++t) {
      const SmAdamTensor& s = tensors[start + t];
      if (s.numel < 0 || (s.numel > 0 && (s.param == nullptr || s.grad == nullptr || s.exp_avg == nullptr ||
                                          s.exp_avg_sq == nullptr)))
        return fail(SM_ERR_ARG, "bad AdamW tensor " + std::to_string(start + t));
      b.param[t] = s.param;
      b.grad[t] = s.grad;
      b.m1[t] = s.exp_avg;
      b.m2[t] = s.exp_avg_sq;
      b.numel[t] = s.numel;
      b.bc1[t] = s.bias_correction1;
      b.bc2[t] = s.bias_correction2;
      b.chunk_start[t + 1] = b.chunk_start[t] + cdiv(s.numel, kAdamChunk);
    }
    const int64_t chunks = b.chunk_start[b.count];
    if (chunks == 0) continue;
    const int grid = static_cast<int>(std::min<int64_t>(chunks, 8 * di->sms));
    k_adamw_multi<<<grid, 256, 0, st>>>(b, lr, beta1, omb1, beta2, omb2, eps, decay_factor);
    SM_LAUNCHED();
  }
  return SM_OK;
}

// ------------------------------------------------------------------- GEMM

int sm_gemm_bf16(const void* a_hi, const void* a_lo, const void* b_hi, const void* b_lo, int layout, int32_t batch,
                 int32_t m, int32_t n, int32_t k, int epilogue, void* out0, void* out1, const float* alpha,
                 const void* aux, const void* aux_lo, float pa, float pb, float pc, float* partials,
                 void* stream) {
  if (batch <= 0 || m <= 0 || n <= 0 || k <= 0) return fail(SM_ERR_ARG, "empty GEMM");
  if (m % 128 != 0 || n % 128 != 0 || k % 64 != 0) return fail(SM_ERR_ARG, "GEMM needs M%128, N%128, K%64 == 0");
  if (a_hi == nullptr || b_hi == nullptr || out0 == nullptr) return fail(SM_ERR_ARG, "null operand");
  const bool b_kmajor = (layout & SM_GEMM_B_KMAJOR) != 0;
  const bool a_mn = (layout & SM_GEMM_A_MNMAJOR) != 0;
  const int cg = (layout & SM_GEMM_PAIR) ? 2 : 1;
  const bool narrow = (layout & SM_GEMM_BN128) != 0;
  if (a_mn && b_kmajor) return fail(SM_ERR_ARG, "an MN-major A needs an MN-major B");
  if (cg == 2 && m % 256 != 0) return fail(SM_ERR_ARG, "CTA-pair tiles need M%256 == 0");
  if (cg == 2 && a_mn) return fail(SM_ERR_ARG, "CTA-pair tiles need a K-major A");
  const int sym = (epilogue & SM_EPI_SYMMETRIC) ? 1 : 0;
  epilogue &= ~SM_EPI_SYMMETRIC;
  if (sym && (m != n || !b_kmajor)) return fail(SM_ERR_ARG, "symmetric output needs M == N and K-major B");
  const bool comp = a_lo != nullptr;
  if (comp && b_lo == nullptr) return fail(SM_ERR_ARG, "compensated mode needs both lo planes");
  if (epilogue == SM_EPI_HILO && out1 == nullptr) return fail(SM_ERR_ARG, "hi/lo epilogue needs out1");
  if (epilogue == SM_EPI_POLY && aux == nullptr) return fail(SM_ERR_ARG, "poly epilogue needs aux");
  if (epilogue == SM_EPI_POLY_HILO && (aux == nullptr || aux_lo == nullptr || out1 == nullptr))
    return fail(SM_ERR_ARG, "hi/lo poly epilogue needs aux, aux_lo and out1");
  if (epilogue == SM_EPI_F32_NORM && partials == nullptr) return fail(SM_ERR_ARG, "norm epilogue needs partials");
  DeviceInfo* di;
  SM_TRY(current_device_info(&di));
  int workers = di->sms;
  if (cg == 2) {
    SM_TRY(pair_workers(di, &workers));
    if (workers <= 0) return fail(SM_ERR_UNSUPPORTED, "no CTA pair of the GEMM fits on this device");
  }
  const int bn = narrow ? kGemmBM : (sym ? kGemmBM * cg : pick_bn(n));
  const int b_box = bn / cg;  // K-major B rows one CTA stages
  const int bk = a_mn ? kBkMN : kBkK;
  CUtensorMap ah, al, bh, bl;
  // A: K-major [batch, M, K]; MN-major [batch, K, M].  B: K-major [batch, N, K]; MN-major [batch, K, N].
  if (!a_mn) SM_TRY(make_map(&ah, a_hi, k, m, batch, kChunk, kGemmBM));
  else SM_TRY(make_map(&ah, a_hi, m, k, batch, kChunk, bk));
  al = ah;
  if (comp) {
    if (!a_mn) SM_TRY(make_map(&al, a_lo, k, m, batch, kChunk, kGemmBM));
    else SM_TRY(make_map(&al, a_lo, m, k, batch, kChunk, bk));
  }
  if (b_kmajor) SM_TRY(make_map(&bh, b_hi, k, n, batch, kChunk, b_box));
  else SM_TRY(make_map(&bh, b_hi, n, k, batch, kChunk, bk));
  bl = bh;
  if (comp) {
    if (b_kmajor) SM_TRY(make_map(&bl, b_lo, k, n, batch, kChunk, b_box));
    else SM_TRY(make_map(&bl, b_lo, n, k, batch, kChunk, bk));
  }
  GemmLaunch L;
  memset(&L, 0, sizeof(L));
  GemmProblem& p = L.p[0];
  p = gemm_problem(ah, al, bh, bl, m, n, k, batch, bn, cg, sym);
  p.out0 = out0;
  p.out1 = out1;
  p.alpha = alpha;
  p.aux = static_cast<const __nv_bfloat16*>(aux);
  p.aux_lo = static_cast<const __nv_bfloat16*>(aux_lo);
  p.pa = pa;
  p.pb = pb;
  p.pc = pc;
  p.partials = partials;
  L.n_problems = 1;
  L.total_tiles = static_cast<int>(problem_tiles(p));
  L.sched = nullptr;
  const int grid = std::min(L.total_tiles, workers) * cg;
  const int lay = a_mn ? kLayoutMM : (b_kmajor ? kLayoutKK : kLayoutKM);
  return dispatch_gemm(bn, cg, comp, lay, epilogue, L, grid, static_cast<cudaStream_t>(stream));
}

int sm_plan_set_peers(SmPlan* p, const void* local_base, int64_t bytes, const void* const* peer_bases,
                      int32_t n_peers) {
  if (p == nullptr) return fail(SM_ERR_ARG, "null plan");
  if (n_peers < 0 || n_peers > kMaxPeers) return fail(SM_ERR_ARG, "n_peers must be in [0, 15]");
  if (n_peers > 0 && (local_base == nullptr || bytes <= 0 || peer_bases == nullptr))
    return fail(SM_ERR_ARG, "peer delivery needs a local range and the peers' bases");
  PeerSet ps{};
  ps.n = n_peers;
  for (int r = 0; r < n_peers; ++r) {
    if (peer_bases[r] == nullptr) return fail(SM_ERR_ARG, "null peer base");
    ps.delta[r] = reinterpret_cast<const char*>(peer_bases[r]) - reinterpret_cast<const char*>(local_base);
  }
  p->peers = ps;
  p->peer_lo = static_cast<const char*>(local_base);
  p->peer_hi = p->peer_lo + (n_peers > 0 ? bytes : 0);
  // the peer set is a launch argument: the next replay re-captures the step
  if (p->exec != nullptr) {
    SM_CUDA(cudaGraphExecDestroy(p->exec));
    p->exec = nullptr;
  }
  return SM_OK;
}

static PFN_cuMemGetAddressRange_v3020 g_addr_range = nullptr;

int sm_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr) return fail(SM_ERR_ARG, "null argument");
  if (g_addr_range == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    const cudaError_t e = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return fail(SM_ERR_UNSUPPORTED, "cuMemGetAddressRange is unavailable");
    g_addr_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(SM_ERR_CUDA, "cuMemGetAddressRange failed: " + std::to_string(r));
  cudaIpcMemHandle_t h;
  SM_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return SM_OK;
}

int sm_ipc_open(const void* handle, void** base_out) {
  if (handle == nullptr || base_out == nullptr) return fail(SM_ERR_ARG, "null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  SM_CUDA(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess));
  return SM_OK;
}

int sm_ipc_close(void* base) {
  if (base == nullptr) return fail(SM_ERR_ARG, "null base");
  SM_CUDA(cudaIpcCloseMemHandle(base));
  return SM_OK;
}

}  // extern "C"
