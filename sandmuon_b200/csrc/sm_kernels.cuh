// sm_kernels.cuh -- HBM-bound kernels of the SandMuon step on sm_100a.
//
//   N1  k_colstats_partial / k_colstats_finish : hook column statistics
//   N2  k_stats_finish                         : EMA + inverse square roots
//   N3  k_whiten_rowstats / k_whiten_write     : Nesterov momentum, two-sided
//                                                whitening, stage-1 hi/lo split
//   N5  k_poly_stage1                          : stage-1 scale s and first S8 polynomial (hi/lo)
//   N7  k_mapback_rowstats / k_mapback_apply   : mapback, graft, weight update
//   N8  k_adamw_multi                          : auxiliary AdamW
//   --  k_reduce_*                             : per-matrix scalar reductions
//
// All reductions use a fixed order (no float atomics) so results are
// bit-reproducible run to run.
#pragma once

#include "sm_common.cuh"

namespace smb {

// The last of `count` CTAs to arrive on `ticket` returns true (after a fence
// that makes every other CTA's prior global writes visible to it) and resets
// the ticket to zero.  Call from all threads after the CTA's writes.
__device__ __forceinline__ bool last_cta_of(unsigned* ticket, unsigned count) {
  __shared__ unsigned s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned t = atomicAdd(ticket, 1u);
    s_last = (t + 1u == count) ? 1u : 0u;
    if (s_last) {
      __threadfence();
      *ticket = 0u;
    }
  }
  __syncthreads();
  return s_last != 0u;
}

// ============================================================ N1: statistics
// sum_sq[c] += sum_r x[r,c]^2 ; sum[c] += sum_r x[r,c]
// (sandmuon/optimizer.py:156-168 forward hook, :170-178 cotangent hook).
// Pass 1: grid (column groups, row splits).  A CTA's 8 warps cover CB
// adjacent column blocks of 32*VEC columns (lane l owns VEC consecutive
// columns, one 16-byte vector) and 8/CB interleaved row groups; each warp
// keeps U row loads in flight.  So a CTA streams CB * 512 contiguous bytes of
// every row it visits.  Partials [split][col] go to the workspace in a fixed
// order; pass 2 sums them in split order (FP64) into the accumulators.

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<double>(double v) { return static_cast<float>(v); }

template <typename T, int VEC>
__device__ __forceinline__ void load_vec(const T* p, int64_t cs, float (&out)[VEC]) {
  if constexpr (VEC * sizeof(T) == 16) {
    const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(p));  // streamed once: evict first
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < VEC; ++i) out[i] = to_f32<T>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) out[i] = to_f32<T>(p[i * cs]);
  }
}

template <typename T, int VEC, bool FIRST, int CB, int U>
__global__ void __launch_bounds__(256, 2)
    k_colstats_partial(const T* __restrict__ x, int64_t n_rows, int64_t n_cols, int64_t rs, int64_t cs,
                       int64_t rows_per_split, float* __restrict__ part_sq, float* __restrict__ part_sum) {
  constexpr int kRowGroups = 8 / CB;
  constexpr int kCols = 32 * VEC * CB;  // columns of one CTA
  __shared__ float sh_sq[8][32 * VEC];
  __shared__ float sh_s[FIRST ? 8 : 1][FIRST ? 32 * VEC : 1];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cbl = warp % CB;   // column block of this warp within the CTA
  const int rg = warp / CB;    // row group
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * kCols + cbl * 32 * VEC + lane * VEC;
  const int64_t r_begin = static_cast<int64_t>(blockIdx.y) * rows_per_split;
  const int64_t r_end = min(r_begin + rows_per_split, n_rows);
  float acc_sq[VEC], acc_s[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc_sq[i] = acc_s[i] = 0.0f;
  // The vector path requires n_cols % VEC == 0 (host-checked), so a lane's
  // VEC columns are either all in range or all out.
  if (col0 < n_cols) {
    const T* base = x + col0 * cs;
    int64_t r = r_begin + rg;
    for (; r + (U - 1) * kRowGroups < r_end; r += U * kRowGroups) {
      float v[U][VEC];
#pragma unroll
      for (int u = 0; u < U; ++u) load_vec<T, VEC>(base + (r + u * kRowGroups) * rs, cs, v[u]);
#pragma unroll
      for (int u = 0; u < U; ++u) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          acc_sq[i] += v[u][i] * v[u][i];
          if (FIRST) acc_s[i] += v[u][i];
        }
      }
    }
    for (; r < r_end; r += kRowGroups) {
      float v[VEC];
      load_vec<T, VEC>(base + r * rs, cs, v);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        acc_sq[i] += v[i] * v[i];
        if (FIRST) acc_s[i] += v[i];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    sh_sq[warp][lane * VEC + i] = acc_sq[i];
    if (FIRST) sh_s[warp][lane * VEC + i] = acc_s[i];
  }
  __syncthreads();
  // column c of the CTA: block c / (32 VEC), summed over its row groups in order
  for (int c = threadIdx.x; c < kCols; c += blockDim.x) {
    const int64_t col = static_cast<int64_t>(blockIdx.x) * kCols + c;
    if (col >= n_cols) continue;
    const int cb = c / (32 * VEC), cc = c - cb * 32 * VEC;
    float s2 = 0.0f, s1 = 0.0f;
#pragma unroll
    for (int g = 0; g < kRowGroups; ++g) {
      s2 += sh_sq[g * CB + cb][cc];
      if (FIRST) s1 += sh_s[g * CB + cb][cc];
    }
    part_sq[static_cast<int64_t>(blockIdx.y) * n_cols + col] = s2;
    if (FIRST) part_sum[static_cast<int64_t>(blockIdx.y) * n_cols + col] = s1;
  }
}

// Pass 2: 32 columns per CTA; warp w sums the partial rows w, w + 8, ... of
// its columns (coalesced 128-byte rows, FP64), then warp 0 combines the 8
// warp sums in order.  Fixed order throughout, so results are reproducible.
__global__ void __launch_bounds__(256)
    k_colstats_finish(const float* __restrict__ part_sq, const float* __restrict__ part_sum, int splits,
                      int64_t n_cols, float* __restrict__ sum_sq, float* __restrict__ sum) {
  __shared__ double sh_sq[8][33];
  __shared__ double sh_s[8][33];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  double s2 = 0.0, s1 = 0.0;
  if (c < n_cols) {
#pragma unroll 4
    for (int p = warp; p < splits; p += 8) {
      s2 += part_sq[static_cast<int64_t>(p) * n_cols + c];
      if (sum != nullptr) s1 += part_sum[static_cast<int64_t>(p) * n_cols + c];
    }
  }
  sh_sq[warp][lane] = s2;
  sh_s[warp][lane] = s1;
  __syncthreads();
  if (warp == 0 && c < n_cols) {
    double t2 = 0.0, t1 = 0.0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      t2 += sh_sq[w][lane];
      t1 += sh_s[w][lane];
    }
    sum_sq[c] += static_cast<float>(t2);
    if (sum != nullptr) sum[c] += static_cast<float>(t1);
  }
}

// ------------------------------------- N1, one launch reduced in a cluster
// For contiguous rows with 16-byte-aligned starts and n_cols a multiple of
// the vector width (16 bytes of T).  A cluster of CL CTAs owns one slab of
// 128 bytes of every row (32 FP32 / 64 BF16 columns); its CTAs split the
// rows in contiguous ranges.  In a CTA, 8 lanes cover a row's slab with one
// 16-byte load each, so the 256 threads are 32 row lanes x 8 column lanes,
// each keeping kStatsUnroll loads in flight.  Sums: FP32 per thread over its
// rows, then FP64 over the 32 row lanes in order, then the cluster's leader
// adds its CTAs' FP64 sums in rank order through distributed shared memory
// and accumulates into sum_sq / sum.  One launch per call, no workspace,
// reproducible results.
// Loads in flight per thread.  Measured on B200 (one config-1 microbatch of
// hook calls, CUDA-graph replay): 16 against 8, BF16 inputs 1.155 against
// 1.280 ms, FP32 inputs unchanged (1.62 ms).
#ifndef SMB_STATS_CLUSTER_UNROLL
#define SMB_STATS_CLUSTER_UNROLL 16
#endif
constexpr int kStatsUnroll = SMB_STATS_CLUSTER_UNROLL;

template <typename T, bool FIRST>
__global__ void __launch_bounds__(256)
    k_colstats_cluster(const T* __restrict__ x, int64_t n_rows, int64_t n_cols, int64_t rs, int cl,
                       float* __restrict__ sum_sq, float* __restrict__ sum) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int kSlab = 8 * VEC;  // columns of one cluster
  // row-lane sums; the leader reuses them for the cluster's FP64 sums
  // (16 x kSlab doubles fit in 32 x (kSlab + 1) floats)
  __shared__ __align__(8) float sh_sq[32][kSlab + 1];
  __shared__ __align__(8) float sh_s[FIRST ? 32 : 1][FIRST ? kSlab + 1 : 1];
  __shared__ double cta_sq[kSlab];
  __shared__ double cta_s[FIRST ? kSlab : 1];
  const int rank = static_cast<int>(cluster_ctarank());
  const int64_t slab = blockIdx.x / cl;
  const int cl_lane = threadIdx.x & 7;   // 16-byte column lane
  const int row_lane = threadIdx.x >> 3;  // 0..31
  const int64_t col0 = slab * kSlab + cl_lane * VEC;
  const int64_t per = (n_rows + cl - 1) / cl;
  const int64_t r_begin = min(static_cast<int64_t>(rank) * per, n_rows);
  const int64_t r_end = min(r_begin + per, n_rows);
  float acc_sq[VEC], acc_s[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc_sq[i] = acc_s[i] = 0.0f;
  if (col0 < n_cols) {
    const T* base = x + col0;
    int64_t r = r_begin + row_lane;
    for (; r + (kStatsUnroll - 1) * 32 < r_end; r += kStatsUnroll * 32) {
      float v[kStatsUnroll][VEC];
#pragma unroll
      for (int u = 0; u < kStatsUnroll; ++u) load_vec<T, VEC>(base + (r + u * 32) * rs, 1, v[u]);
#pragma unroll
      for (int u = 0; u < kStatsUnroll; ++u) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          acc_sq[i] += v[u][i] * v[u][i];
          if (FIRST) acc_s[i] += v[u][i];
        }
      }
    }
    for (; r < r_end; r += 32) {
      float v[VEC];
      load_vec<T, VEC>(base + r * rs, 1, v);
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        acc_sq[i] += v[i] * v[i];
        if (FIRST) acc_s[i] += v[i];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    sh_sq[row_lane][cl_lane * VEC + i] = acc_sq[i];
    if (FIRST) sh_s[row_lane][cl_lane * VEC + i] = acc_s[i];
  }
  __syncthreads();
  if (threadIdx.x < kSlab) {
    double t2 = 0.0, t1 = 0.0;
#pragma unroll 8
    for (int l = 0; l < 32; ++l) {
      t2 += static_cast<double>(sh_sq[l][threadIdx.x]);
      if (FIRST) t1 += static_cast<double>(sh_s[l][threadIdx.x]);
    }
    cta_sq[threadIdx.x] = t2;
    if (FIRST) cta_s[threadIdx.x] = t1;
  }
  // every CTA's sums are in its shared memory before the leader reads them
  cluster_sync_all();
  if (rank == 0) {
    // all of the cluster's sums fetched at once (one round of remote loads),
    // then added in rank order
    double* all_sq = reinterpret_cast<double*>(&sh_sq[0][0]);  // [cl][kSlab], reusing the staging
    double* all_s = FIRST ? reinterpret_cast<double*>(&sh_s[0][0]) : nullptr;
    for (int e = threadIdx.x; e < cl * kSlab; e += blockDim.x) {
      const int k = e / kSlab, c = e - k * kSlab;
      all_sq[e] = ld_shared_cluster_f64(mapa_shared(smem_u32(&cta_sq[c]), static_cast<uint32_t>(k)));
      if (FIRST) all_s[e] = ld_shared_cluster_f64(mapa_shared(smem_u32(&cta_s[c]), static_cast<uint32_t>(k)));
    }
    __syncthreads();
    const int64_t col = slab * kSlab + threadIdx.x;
    if (threadIdx.x < kSlab && col < n_cols) {
      double t2 = 0.0, t1 = 0.0;
      for (int k = 0; k < cl; ++k) {
        t2 += all_sq[k * kSlab + threadIdx.x];
        if (FIRST) t1 += all_s[k * kSlab + threadIdx.x];
      }
      sum_sq[col] += static_cast<float>(t2);
      if (FIRST) sum[col] += static_cast<float>(t1);
    }
  }
  // no CTA leaves while the leader may still read its shared memory
  cluster_sync_all();
}

// ------------------------------------------------ N1, TMA-fed single launch
// For contiguous 16-byte-aligned rows.  A persistent CTA (one per SM) takes
// one column group (kStatsCols columns) and a contiguous range of its row
// blocks, streams them through a kStatsStages-deep ring of 2-D TMA boxes
// (kStatsCols x BR elements, 32 KB) filled by one producer thread, and
// reduces each box from shared memory, one column per consumer thread, so
// the bytes in flight do not depend on registers.  The CTA's column sums
// become one partial row of the workspace; the last CTA of the group to
// finish (an integer ticket per group, zero at launch and reset by that CTA)
// adds the group's partial rows in order (FP64) into the accumulators.  One
// reduction launch per call, reproducible results.

constexpr int kStatsCols = 256;
#ifndef SMB_STATS_STAGES
#define SMB_STATS_STAGES 4
#endif
constexpr int kStatsStages = SMB_STATS_STAGES;
constexpr int kStatsThreads = kStatsCols + 32;  // consumer threads + one producer warp

struct StatsTmaArgs {
  int64_t n_cols;
  int groups;          // column groups of kStatsCols columns
  int splits;          // CTAs per group
  int row_blocks;      // boxes per group: ceil(n_rows / BR)
  float* part_sq;      // [groups * splits, kStatsCols]
  float* part_sum;     // same, or null
  unsigned* tickets;   // [groups], zero at launch; reset to zero by the last CTA
  float* sum_sq;       // [n_cols] accumulators
  float* sum;          // or null
};

template <typename T, int BR>
struct StatsTmaSmem {
  static constexpr uint32_t kBoxBytes = kStatsCols * BR * sizeof(T);
  static constexpr int kBytes = kStatsStages * kBoxBytes + 2 * kStatsStages * 8 + 16 + 1024;
};

template <typename T, bool FIRST, int BR>
__global__ void __launch_bounds__(kStatsThreads, 1)
    k_colstats_tma(const __grid_constant__ CUtensorMap map, const StatsTmaArgs a) {
  using S = StatsTmaSmem<T, BR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const T* ring = reinterpret_cast<const T*>(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStatsStages * S::kBoxBytes);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * kStatsStages);
  __shared__ int sh_last;
  const uint32_t bar_base = smem_u32(bars);
  auto bar_full = [&](int st) { return bar_base + 8u * st; };
  auto bar_empty = [&](int st) { return bar_base + 8u * (kStatsStages + st); };

  const int g = static_cast<int>(blockIdx.x) % a.groups;
  const int s = static_cast<int>(blockIdx.x) / a.groups;
  const int rb_begin = static_cast<int>(static_cast<int64_t>(a.row_blocks) * s / a.splits);
  const int rb_end = static_cast<int>(static_cast<int64_t>(a.row_blocks) * (s + 1) / a.splits);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int st = 0; st < kStatsStages; ++st) {
      mbar_init(bar_full(st), 1);
      mbar_init(bar_empty(st), kStatsCols / 32);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  __syncthreads();

  if (tid >= kStatsCols) {
    // ------------------------------------------------------------ producer
    if (tid == kStatsCols) {
      tma_prefetch_desc(&map);
      int stage = 0;
      uint32_t phase = 0;
      for (int rb = rb_begin; rb < rb_end; ++rb) {
        if (!mbar_wait(bar_empty(stage), phase ^ 1u, abort_flag, kStatusTimeoutStatsLoad)) break;
        mbar_arrive_expect_tx(bar_full(stage), S::kBoxBytes);
        tma_load_2d(smem_u32(ring + static_cast<size_t>(stage) * BR * kStatsCols), &map, bar_full(stage),
                    g * kStatsCols, rb * BR);
        if (++stage == kStatsStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // ----------------------------------------------------------- consumers
    // FP32 within a box, FP64 across boxes (a CTA may see thousands of rows)
    double acc_sq = 0.0, acc_s = 0.0;
    int stage = 0;
    uint32_t phase = 0;
    for (int rb = rb_begin; rb < rb_end; ++rb) {
      // the vote keeps each warp uniform (and on the same side of a timeout)
      const bool ready = mbar_wait(bar_full(stage), phase, abort_flag, kStatusTimeoutStatsReduce);
      if (!__all_sync(0xffffffffu, ready)) break;
      const T* box = ring + static_cast<size_t>(stage) * BR * kStatsCols + tid;
      float box_sq = 0.0f, box_s = 0.0f;
#pragma unroll 8
      for (int r = 0; r < BR; ++r) {
        const float v = to_f32<T>(box[r * kStatsCols]);
        box_sq += v * v;
        if (FIRST) box_s += v;
      }
      acc_sq += box_sq;
      if (FIRST) acc_s += box_s;
      __syncwarp();
      if ((tid & 31) == 0) mbar_arrive(bar_empty(stage));
      if (++stage == kStatsStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    const int64_t prow = (static_cast<int64_t>(g) * a.splits + s) * kStatsCols;
    a.part_sq[prow + tid] = static_cast<float>(acc_sq);
    if (FIRST) a.part_sum[prow + tid] = static_cast<float>(acc_s);
    __threadfence();
  }
  __syncthreads();
  if (tid == 0) sh_last = atomicAdd(&a.tickets[g], 1u) == static_cast<unsigned>(a.splits - 1);
  __syncthreads();
  if (sh_last && tid < kStatsCols) {
    // every partial row of the group is visible: sum them in split order
    __threadfence();
    const float* psq = a.part_sq + static_cast<int64_t>(g) * a.splits * kStatsCols + tid;
    const float* ps = FIRST ? a.part_sum + static_cast<int64_t>(g) * a.splits * kStatsCols + tid : nullptr;
    double t2 = 0.0, t1 = 0.0;
#pragma unroll 16
    for (int p = 0; p < a.splits; ++p) {
      t2 += __ldcg(psq + static_cast<int64_t>(p) * kStatsCols);
      if (FIRST) t1 += __ldcg(ps + static_cast<int64_t>(p) * kStatsCols);
    }
    const int64_t col = static_cast<int64_t>(g) * kStatsCols + tid;
    if (col < a.n_cols) {
      a.sum_sq[col] += static_cast<float>(t2);
      if (FIRST) a.sum[col] += static_cast<float>(t1);
    }
    if (tid == 0) a.tickets[g] = 0u;
  }
}

// ====================================================== N2: statistics finish
// One CTA per statistic vector; kind-specific arithmetic of
//   _finish_a + diagonal_inverse_sqrt / rank1_inverse_sqrt
//   (sandmuon/optimizer.py:182-207, :19-35) and
//   _finish_b (sandmuon/optimizer.py:209-222).

struct StatDev {
  float* sum;
  float* first_sum;
  float* ema;
  float* mean_ema;
  float* inv;     // out [n]
  float* z;       // out [n] (rank-one)
  float* zeta;    // out [n] = inv * z (rank-one)
  float* scal;    // out [4]: {coefficient, sum(zeta^2), sum(z^2), 0}
  const int64_t* count_dev;  // device row count, or null: use `count`
  int64_t count;
  int32_t n;
  int32_t kind;
  int32_t init;
  int32_t pad;
};

template <int NT>
__device__ __forceinline__ double block_sum_d(double v, double* sh) {
  v = warp_sum_d(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  double t = 0.0;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) t += sh[w];
  return t;
}

constexpr float kFltTiny = 1.17549435e-38f;  // torch.finfo(torch.float32).tiny

// Vectors of up to 256 * kFinishK elements: each thread loads its elements
// once and the three passes below run from registers (one memory round trip
// instead of three); the arithmetic and reduction orders are those of the
// loop path.
constexpr int kFinishK = 12;

template <bool RANK1_A, bool KIND_B>
__device__ __forceinline__ void stats_finish_regs(const StatDev& d, int n, float count, float beta, float omb,
                                                  double* sh) {
  float sum[kFinishK], ema[kFinishK], first[kFinishK], mema[kFinishK];
#pragma unroll
  for (int k = 0; k < kFinishK; ++k) {
    const int i = threadIdx.x + 256 * k;
    const bool in = i < n;
    sum[k] = in ? d.sum[i] : 0.0f;
    ema[k] = (in && !d.init) ? d.ema[i] : 0.0f;
    first[k] = (RANK1_A && in) ? d.first_sum[i] : 0.0f;
    mema[k] = (RANK1_A && in && !d.init) ? d.mean_ema[i] : 0.0f;
  }
  if (KIND_B) {
    // b = sum / count ; b /= max(mean(b), tiny)
    double acc = 0.0;
#pragma unroll
    for (int k = 0; k < kFinishK; ++k)
      if (threadIdx.x + 256 * k < n) acc += static_cast<double>(sum[k] / count);
    const float mean_b = static_cast<float>(block_sum_d<256>(acc, sh) / n);
    const float denom = fmaxf(mean_b, kFltTiny);
    double acc_e = 0.0;
#pragma unroll
    for (int k = 0; k < kFinishK; ++k) {
      const int i = threadIdx.x + 256 * k;
      if (i < n) {
        const float bv = (sum[k] / count) / denom;
        ema[k] = d.init ? bv : ema[k] * beta + omb * bv;
        d.ema[i] = ema[k];
        d.sum[i] = 0.0f;
        acc_e += ema[k];
      }
    }
    __syncthreads();  // sh reuse
    const float mean_e = static_cast<float>(block_sum_d<256>(acc_e, sh) / n);
#pragma unroll
    for (int k = 0; k < kFinishK; ++k) {
      const int i = threadIdx.x + 256 * k;
      if (i < n) {
        const float nrm = fmaxf(ema[k], mean_e * 1e-6f) / fmaxf(mean_e, kFltTiny);
        d.inv[i] = 1.0f / sqrtf(fmaxf(nrm, 1e-6f));
      }
    }
    return;
  }
  double acc = 0.0;
#pragma unroll
  for (int k = 0; k < kFinishK; ++k) {
    const int i = threadIdx.x + 256 * k;
    if (i < n) {
      const float second = sum[k] / count;
      ema[k] = d.init ? second : ema[k] * beta + omb * second;
      d.ema[i] = ema[k];
      d.sum[i] = 0.0f;
      if (RANK1_A) {
        const float mean = first[k] / count;
        mema[k] = d.init ? mean : mema[k] * beta + omb * mean;
        d.mean_ema[i] = mema[k];
        d.first_sum[i] = 0.0f;
      }
      acc += ema[k];
    }
  }
  const float mean_e = static_cast<float>(block_sum_d<256>(acc, sh) / n);
  if (!RANK1_A) {
#pragma unroll
    for (int k = 0; k < kFinishK; ++k) {
      const int i = threadIdx.x + 256 * k;
      if (i < n) {
        const float nrm = fmaxf(ema[k], mean_e * 1e-6f) / fmaxf(mean_e, kFltTiny);
        d.inv[i] = 1.0f / sqrtf(fmaxf(nrm, 1e-6f));
      }
    }
    if (threadIdx.x == 0) {
      d.scal[0] = 0.0f;
      d.scal[1] = 0.0f;
      d.scal[2] = 0.0f;
      d.scal[3] = 0.0f;
    }
    return;
  }
  // rank1_inverse_sqrt (sandmuon/optimizer.py:27-35)
  const float scale = fmaxf(mean_e, kFltTiny);
  const float root_scale = sqrtf(scale);
  double acc_z = 0.0, acc_zeta = 0.0;
#pragma unroll
  for (int k = 0; k < kFinishK; ++k) {
    const int i = threadIdx.x + 256 * k;
    if (i < n) {
      const float mu = mema[k];
      const float var = fmaxf(ema[k] - mu * mu, 0.0f);
      const float inv = 1.0f / sqrtf(fmaxf(var / scale, 1e-6f));
      const float z = inv * (mu / root_scale);
      d.inv[i] = inv;
      d.z[i] = z;
      d.zeta[i] = inv * z;
      acc_z += static_cast<double>(z) * z;
      acc_zeta += static_cast<double>(inv * z) * (inv * z);
    }
  }
  __syncthreads();  // sh reuse
  const double kz = block_sum_d<256>(acc_z, sh);
  __syncthreads();
  const double kzeta = block_sum_d<256>(acc_zeta, sh);
  if (threadIdx.x == 0) {
    const float root = sqrtf(1.0f + static_cast<float>(kz));
    d.scal[0] = -1.0f / (root * (root + 1.0f));
    d.scal[1] = static_cast<float>(kzeta);
    d.scal[2] = static_cast<float>(kz);
    d.scal[3] = 0.0f;
  }
}

__global__ void __launch_bounds__(256) k_stats_finish(const StatDev* __restrict__ stats, float beta, float omb) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ double sh[8];
  const StatDev d = stats[blockIdx.x];
  const int n = d.n;
  const float count = static_cast<float>(d.count_dev != nullptr ? *d.count_dev : d.count);
  if (n <= 256 * kFinishK) {
    if (d.kind == SM_STAT_B) stats_finish_regs<false, true>(d, n, count, beta, omb, sh);
    else if (d.kind == SM_STAT_A_RANK1) stats_finish_regs<true, false>(d, n, count, beta, omb, sh);
    else stats_finish_regs<false, false>(d, n, count, beta, omb, sh);
    return;
  }

  if (d.kind == SM_STAT_B) {
    // b = sum / count ; b /= max(mean(b), tiny)
    double acc = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) acc += static_cast<double>(d.sum[i] / count);
    const float mean_b = static_cast<float>(block_sum_d<256>(acc, sh) / n);
    const float denom = fmaxf(mean_b, kFltTiny);
    double acc_e = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float b = (d.sum[i] / count) / denom;
      const float e = d.init ? b : d.ema[i] * beta + omb * b;
      d.ema[i] = e;
      d.sum[i] = 0.0f;
      acc_e += e;
    }
    const float mean_e = static_cast<float>(block_sum_d<256>(acc_e, sh) / n);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float e = d.ema[i];
      const float nrm = fmaxf(e, mean_e * 1e-6f) / fmaxf(mean_e, kFltTiny);
      d.inv[i] = 1.0f / sqrtf(fmaxf(nrm, 1e-6f));
    }
    return;
  }

  // A statistics: second = a_sum / count (and mean = a_first_sum / count)
  const bool rank1 = d.kind == SM_STAT_A_RANK1;
  double acc = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float second = d.sum[i] / count;
    const float e = d.init ? second : d.ema[i] * beta + omb * second;
    d.ema[i] = e;
    d.sum[i] = 0.0f;
    if (rank1) {
      const float mean = d.first_sum[i] / count;
      d.mean_ema[i] = d.init ? mean : d.mean_ema[i] * beta + omb * mean;
      d.first_sum[i] = 0.0f;
    }
    acc += e;
  }
  const float mean_e = static_cast<float>(block_sum_d<256>(acc, sh) / n);
  if (!rank1) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const float nrm = fmaxf(d.ema[i], mean_e * 1e-6f) / fmaxf(mean_e, kFltTiny);
      d.inv[i] = 1.0f / sqrtf(fmaxf(nrm, 1e-6f));
    }
    if (threadIdx.x == 0) {
      d.scal[0] = 0.0f;
      d.scal[1] = 0.0f;
      d.scal[2] = 0.0f;
      d.scal[3] = 0.0f;
    }
    return;
  }
  // rank1_inverse_sqrt (sandmuon/optimizer.py:27-35)
  const float scale = fmaxf(mean_e, kFltTiny);
  const float root_scale = sqrtf(scale);
  double acc_z = 0.0, acc_zeta = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float mu = d.mean_ema[i];
    const float var = fmaxf(d.ema[i] - mu * mu, 0.0f);
    const float inv = 1.0f / sqrtf(fmaxf(var / scale, 1e-6f));
    const float z = inv * (mu / root_scale);
    d.inv[i] = inv;
    d.z[i] = z;
    d.zeta[i] = inv * z;
    acc_z += static_cast<double>(z) * z;
    acc_zeta += static_cast<double>(inv * z) * (inv * z);
  }
  const double kz = block_sum_d<256>(acc_z, sh);
  const double kzeta = block_sum_d<256>(acc_zeta, sh);
  if (threadIdx.x == 0) {
    const float root = sqrtf(1.0f + static_cast<float>(kz));
    d.scal[0] = -1.0f / (root * (root + 1.0f));
    d.scal[1] = static_cast<float>(kzeta);
    d.scal[2] = static_cast<float>(kz);
    d.scal[3] = 0.0f;
  }
}

// ===================================================== per-matrix descriptor

struct MatDev {
  const float* grad;    // [d_out, d_in]
  float* mom;           // [d_out, d_in]
  float* weight;        // [d_out, d_in]
  float* export_to;     // [d_out, d_in] copy of the updated weight (FP32), or of the
                        // BF16 update delta when export_bf16; or null
  const float* inv_a;   // [d_in]
  const float* z_a;     // [d_in] or null (diagonal A)
  const float* zeta_a;  // [d_in] inv_a * z_a or null
  const float* scal_a;  // {coefficient, sum(zeta^2), ...}
  const float* inv_b;   // [d_out]
  int32_t d_out, d_in;
  int32_t transposed;   // d_out > d_in: oriented matrix is the transpose
  int32_t slot;
  float lr;
  float sqrt_rows;      // sqrt(d_out): the graft norm
  int32_t export_bf16;  // 1: export_to holds bf16 D = bf16(lr * direction), W -= float(D)
  int32_t peer;         // 1: the weight lies in the plan's peer-mirrored range (PeerSet)
};

// ========================================== N3 pass 1: whitening row stats
// Per param row o (contiguous, d_in long):
//   m' = .8 m + .2 g ; s = .8 m' + .2 g          (sandmuon/optimizer.py:246-248)
//   y  = inv_b[o] * s * inv_a                    (whitening diagonals)
//   rs[o] = { y . z_a , |y| }   (|y| from an FP64 sum of squares, so rows of
//                                tiny or huge gradients neither underflow nor
//                                overflow on the way to the matrix norm)
// The rank-one whitening correction V = Y + c (Y z) z^T acts along d_in in
// both orientations, so its dot products are row dots of the param layout.
// The last CTA of a matrix to finish (an integer ticket per matrix, zero
// between launches: that CTA resets it) also reduces the matrix's |y|^2 row
// sums, in row order, into the matrix's plane scale and stage-1 alphas
// (plane_scale_for, set_stage1_alphas below).
//
// Normalisation.  The S8 input is x = v / max(|v|_F, 1e-30)
// (sandmuon/optimizer.py:77-78).  The S8 map is invariant to the scale of
// its input (stage 1 divides by s = 1.35 |G^2|_F^(1/4)), so any norm that
// keeps X in range reproduces it; |Y|_F bounds |V|_F within the factor
// sqrt(1 + |z|^2) of the rank-one whitener and never cancels.  The hi/lo
// planes hold v * 2^k, a power-of-two scale near 1 / |Y|_F (exact: the split
// commutes with it), and the stage-1 products take the remaining factor
// rho = (1 / max(|Y|_F, 1e-30)) / 2^k as their alpha: rho^2 for X X^T, rho / s
// for P X.  Every result is then bitwise independent of k.

// 2^k with norm * 2^k in [1, 2), k clamped to [-126, 126]; 1 for a zero or
// non-finite norm.
__device__ __forceinline__ float plane_scale_for(double norm) {
  if (!(norm > 0.0) || !isfinite(norm)) return 1.0f;
  int e = 0;
  frexp(norm, &e);  // norm in [2^(e-1), 2^e)
  return ldexpf(1.0f, min(max(1 - e, -126), 126));
}

// Stage-1 alphas of planes written as v * `used`: rho = (1 / max(norm, 1e-30))
// / used, exactly (used is a power of two), and rho^2; 0 for a zero matrix.
__device__ __forceinline__ void set_stage1_alphas(double norm, float used, float* rho, float* rho2, int b) {
  const float inv = 1.0f / fmaxf(static_cast<float>(norm), 1e-30f);
  const float r = norm > 0.0 ? inv / used : 0.0f;
  rho[b] = r;
  rho2[b] = r * r;
}

// Sum over rows 0..n of rs[row].y^2 in a fixed order (FP64), whole CTA.
__device__ __forceinline__ double rows_sum_sq_y(const float2* rs, int n, double* sh) {
  double acc = 0.0;
  for (int o = threadIdx.x; o < n; o += blockDim.x) {
    const double v = static_cast<double>(__ldcg(&rs[o].y));
    acc += v * v;
  }
  acc = warp_sum_d(acc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[warp] = acc;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += sh[w];
  return t;
}

// Sum over rows 0..n of rs[row].y in a fixed order (FP64), whole CTA.
__device__ __forceinline__ double rows_sum_y(const float2* rs, int n, double* sh) {
  double acc = 0.0;
  for (int o = threadIdx.x; o < n; o += blockDim.x) acc += static_cast<double>(__ldcg(&rs[o].y));
  acc = warp_sum_d(acc);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[warp] = acc;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += sh[w];
  return t;
}

// Each warp reduces ROWS consecutive param rows, so one CTA covers 8 * ROWS
// rows and the whitening vectors loaded per column group serve all of a
// warp's rows.  Rows past d_out repeat the last row and are not stored.
// Measured on B200 (config 1, ncu): mapback row statistics 111 -> 105 us
// with 4 rows per warp; the whitening pass, which streams two arrays per
// row, 106 -> 141 us, so it keeps one row per warp.
#ifndef SMB_MAPBACK_ROWS
#define SMB_MAPBACK_ROWS 4
#endif
constexpr int kWhitenRows = 1;
constexpr int kMapbackRows = SMB_MAPBACK_ROWS;

template <int VEC, bool RANK1>
__global__ void __launch_bounds__(256)
    k_whiten_rowstats(const MatDev* __restrict__ mats, float mom_beta, float omb, float2* __restrict__ rs,
                      int ld_rs, float* __restrict__ pre, float* __restrict__ rho, float* __restrict__ rho2,
                      unsigned* __restrict__ tickets) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ double sh[8];
  const MatDev md = mats[blockIdx.y];
  const int o0 = blockIdx.x * 8 * kWhitenRows;
  if (o0 >= md.d_out) return;  // whole CTA: it takes no part in the matrix's ticket
  const int obase = o0 + (threadIdx.x >> 5) * kWhitenRows;
  const int lane = threadIdx.x & 31;
  float2* rsb = rs + static_cast<int64_t>(blockIdx.y) * ld_rs;
  if (obase < md.d_out) {
    // A null momentum means "use the input as is" (the batch S8 entry point).
    const bool has_mom = md.mom != nullptr;
    const float* g[kWhitenRows];
    const float* m[kWhitenRows];
    float ib[kWhitenRows], dot[kWhitenRows];
    double sq[kWhitenRows];
#pragma unroll
    for (int r = 0; r < kWhitenRows; ++r) {
      const int o = min(obase + r, md.d_out - 1);
      g[r] = md.grad + static_cast<int64_t>(o) * md.d_in;
      m[r] = has_mom ? md.mom + static_cast<int64_t>(o) * md.d_in : g[r];
      ib[r] = md.inv_b[o];
      dot[r] = 0.0f;
      sq[r] = 0.0f;
    }
#pragma unroll 2
    for (int i = lane * VEC; i < md.d_in; i += 32 * VEC) {
      float av[VEC], zv[VEC];
      if constexpr (VEC == 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(md.inv_a + i);
        av[0] = a4.x; av[1] = a4.y; av[2] = a4.z; av[3] = a4.w;
        if (RANK1) {
          const float4 z4 = *reinterpret_cast<const float4*>(md.z_a + i);
          zv[0] = z4.x; zv[1] = z4.y; zv[2] = z4.z; zv[3] = z4.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          av[e] = md.inv_a[i + e];
          if (RANK1) zv[e] = md.z_a[i + e];
        }
      }
#pragma unroll
      for (int r = 0; r < kWhitenRows; ++r) {
        float gv[VEC], mv[VEC];
        if constexpr (VEC == 4) {
          const float4 g4 = *reinterpret_cast<const float4*>(g[r] + i);
          const float4 m4 = *reinterpret_cast<const float4*>(m[r] + i);
          gv[0] = g4.x; gv[1] = g4.y; gv[2] = g4.z; gv[3] = g4.w;
          mv[0] = m4.x; mv[1] = m4.y; mv[2] = m4.z; mv[3] = m4.w;
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            gv[e] = g[r][i + e];
            mv[e] = m[r][i + e];
          }
        }
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float mn = mom_beta * mv[e] + omb * gv[e];
          const float src = has_mom ? mom_beta * mn + omb * gv[e] : gv[e];
          const float y = (src * ib[r]) * av[e];
          sq[r] += static_cast<double>(y) * y;
          if (RANK1) dot[r] += y * zv[e];
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kWhitenRows; ++r) {
      const double s_r = warp_sum_d(sq[r]);
      const float d_r = RANK1 ? warp_sum(dot[r]) : 0.0f;
      if (lane == 0 && obase + r < md.d_out) rsb[obase + r] = make_float2(d_r, static_cast<float>(sqrt(s_r)));
    }
  }
  if (last_cta_of(tickets + blockIdx.y, static_cast<unsigned>((md.d_out + 8 * kWhitenRows - 1) / (8 * kWhitenRows)))) {
    const double t = rows_sum_sq_y(rsb, md.d_out, sh);
    // k_whiten_write writes the planes with the scale set here
    if (threadIdx.x == 0) {
      const double norm = sqrt(t);
      const float used = plane_scale_for(norm);
      pre[blockIdx.y] = used;
      set_stage1_alphas(norm, used, rho, rho2, blockIdx.y);
    }
  }
}

// ========================================== N3 pass 2: whiten + split write
// Tile of 32 param rows x 64 param columns per CTA (256 threads); grid
// (tiles of the group's largest matrix, matrices).
//   m' written back ; v = y + c * dot[o] * z[i] ; x = v * pre[b]
//   X_hi/X_lo at the oriented position: (o, i), or (i, o) when transposed
//   (staged through shared memory so both reads and writes are coalesced).
template <bool RANK1, bool VEC4>
__global__ void __launch_bounds__(256)
    k_whiten_write(const MatDev* __restrict__ mats, float mom_beta, float omb, const float2* __restrict__ rs, int ld_rs,
                   const float* __restrict__ pre, __nv_bfloat16* __restrict__ xh,
                   __nv_bfloat16* __restrict__ xl, int64_t rp, int64_t cp) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ uint32_t sh_hi[64][17];  // [i][o/2] packed bf16 pairs, transposed staging
  __shared__ uint32_t sh_lo[64][17];
  // blockIdx.x numbers this matrix's 32 x 64 tiles row-major; a grid sized
  // for the group's largest tile count leaves the surplus CTAs idle.
  const int b = blockIdx.y;
  const MatDev md = mats[b];
  const int tiles_x = (md.d_in + 63) / 64;
  const int o0 = static_cast<int>(blockIdx.x / tiles_x) * 32;
  const int i0 = static_cast<int>(blockIdx.x % tiles_x) * 64;
  if (o0 >= md.d_out) return;
  const float scale = pre[b];
  const float coef = RANK1 ? md.scal_a[0] : 0.0f;
  const bool has_mom = md.mom != nullptr;
  const int tx = threadIdx.x & 15;   // 4 consecutive columns
  const int ty = threadIdx.x >> 4;   // rows ty and ty + 16
  const int64_t plane = static_cast<int64_t>(b) * rp * cp;
  const bool trans = md.transposed != 0;

#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int ol = ty + 16 * half;
    const int o = o0 + ol;
    const int ib = i0 + tx * 4;
    float xv[4] = {0.f, 0.f, 0.f, 0.f};
    if (o < md.d_out) {
      const float invb = md.inv_b[o];
      const float cw = RANK1 ? coef * rs[static_cast<int64_t>(b) * ld_rs + o].x : 0.0f;
      const int64_t row = static_cast<int64_t>(o) * md.d_in;
      if (VEC4 && ib + 3 < md.d_in) {
        const float4 g4 = *reinterpret_cast<const float4*>(md.grad + row + ib);
        const float4 m4 = has_mom ? *reinterpret_cast<const float4*>(md.mom + row + ib) : g4;
        const float4 a4 = *reinterpret_cast<const float4*>(md.inv_a + ib);
        const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
        const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
        float zv[4] = {0.f, 0.f, 0.f, 0.f};
        if (RANK1) {
          const float4 z4 = *reinterpret_cast<const float4*>(md.z_a + ib);
          zv[0] = z4.x; zv[1] = z4.y; zv[2] = z4.z; zv[3] = z4.w;
        }
        float mn[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          mn[e] = mom_beta * mv[e] + omb * gv[e];
          const float src = has_mom ? mom_beta * mn[e] + omb * gv[e] : gv[e];
          float v = (src * invb) * av[e];
          if (RANK1) v += cw * zv[e];
          xv[e] = v * scale;
        }
        if (has_mom) *reinterpret_cast<float4*>(md.mom + row + ib) = make_float4(mn[0], mn[1], mn[2], mn[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = ib + e;
          if (i < md.d_in) {
            const float gv = md.grad[row + i];
            float src = gv;
            if (has_mom) {
              const float mn = mom_beta * md.mom[row + i] + omb * gv;
              md.mom[row + i] = mn;
              src = mom_beta * mn + omb * gv;
            }
            float v = (src * invb) * md.inv_a[i];
            if (RANK1) v += cw * md.z_a[i];
            xv[e] = v * scale;
          }
        }
      }
    }
    float h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) split_hilo(xv[e], h[e], l[e]);
    if (!trans) {
      if (o < md.d_out) {
        __nv_bfloat16* dh = xh + plane + static_cast<int64_t>(o) * cp;
        __nv_bfloat16* dl = xl + plane + static_cast<int64_t>(o) * cp;
        if (ib + 3 < md.d_in) {
          *reinterpret_cast<uint2*>(dh + ib) = make_uint2(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]));
          *reinterpret_cast<uint2*>(dl + ib) = make_uint2(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]));
        } else {
          for (int e = 0; e < 4; ++e) {
            if (ib + e < md.d_in) {
              dh[ib + e] = __float2bfloat16_rn(h[e]);
              dl[ib + e] = __float2bfloat16_rn(l[e]);
            }
          }
        }
      }
    } else {
      // stage (i, o) pairs: element (il, ol) -> packed word [il][ol/2], half ol&1
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int il = tx * 4 + e;
        __nv_bfloat16* ph = reinterpret_cast<__nv_bfloat16*>(&sh_hi[il][ol >> 1]) + (ol & 1);
        __nv_bfloat16* pl = reinterpret_cast<__nv_bfloat16*>(&sh_lo[il][ol >> 1]) + (ol & 1);
        *ph = __float2bfloat16_rn(h[e]);
        *pl = __float2bfloat16_rn(l[e]);
      }
    }
  }
  if (trans) {
    __syncthreads();
    // oriented X row = i (d_in index), columns = o; 64 rows x 32 bf16 each.
    const int il = threadIdx.x >> 2;       // 0..63
    const int oc = (threadIdx.x & 3) * 8;  // 0, 8, 16, 24
    const int i = i0 + il;
    if (i < md.d_in) {
      __nv_bfloat16* dh = xh + plane + static_cast<int64_t>(i) * cp + o0 + oc;
      __nv_bfloat16* dl = xl + plane + static_cast<int64_t>(i) * cp + o0 + oc;
      if (o0 + oc + 7 < md.d_out) {
        uint4 vh, vl;
        vh.x = sh_hi[il][oc / 2 + 0]; vh.y = sh_hi[il][oc / 2 + 1];
        vh.z = sh_hi[il][oc / 2 + 2]; vh.w = sh_hi[il][oc / 2 + 3];
        vl.x = sh_lo[il][oc / 2 + 0]; vl.y = sh_lo[il][oc / 2 + 1];
        vl.z = sh_lo[il][oc / 2 + 2]; vl.w = sh_lo[il][oc / 2 + 3];
        *reinterpret_cast<uint4*>(dh) = vh;
        *reinterpret_cast<uint4*>(dl) = vl;
      } else {
        for (int e = 0; e < 8; ++e) {
          if (o0 + oc + e < md.d_out) {
            dh[e] = reinterpret_cast<const __nv_bfloat16*>(&sh_hi[il][0])[oc + e];
            dl[e] = reinterpret_cast<const __nv_bfloat16*>(&sh_lo[il][0])[oc + e];
          }
        }
      }
    }
  }
}

// ======================================== N3 in one pass: fused front end
// From a plan's second step on, one kernel replaces the two above for groups
// whose rows are 16-byte aligned.  A CTA owns R consecutive param rows of one
// matrix (R = fused_rows(d_in): as many as fit kFusedSmemBytes, a power of
// two <= 16):
//   1. one thread copies the R gradient rows and R momentum rows into shared
//      memory with bulk async copies (cp.async.bulk, no multicast)
//      completing on one mbarrier (a bounded wait);
//   2. row statistics from shared memory: y . z_a and |y| (FP64 sum of
//      squares; rows split over 8 / R warps when R < 8, combined in order);
//   3. m' is written back and the hi/lo planes of x = v * pre[b] at the
//      oriented position; the param rows of a transposed matrix are columns
//      of X, so there each thread writes the R consecutive bf16 of one X row.
// DRAM traffic: g and m read once, m' and the planes written once (16 bytes
// per param, against 24 for the two passes).  Measured on B200 (config 1,
// ncu launch lists): 86 us for the 36 x 768^2 group (two passes 111 us) and
// 188 us for the 18 x 768 x 3072 group (213 us).  pre[b] is the previous
// step's plane scale; the last CTA of a matrix to finish (an integer ticket
// per matrix, zero between launches) reduces the row norms into the stage-1
// alphas for it and the next step's pre[b].  If |Y|_F * pre[b] falls outside
// [2^-60, 2^60] (the norm moved that far since the previous step, so the
// planes may have lost range) it sets kStatusFrontRange.
constexpr int kFusedSmemBytes = 96 * 1024;

__host__ __device__ constexpr int fused_rows(int d_in) {
  int r = 16;
  while (r > 0 && static_cast<int64_t>(r) * d_in * 8 > kFusedSmemBytes) r >>= 1;
  return r;
}

// (y . z, |y|^2) of one row segment
struct FrontSeg {
  float dot;
  double sq;
};

template <bool RANK1>
__global__ void __launch_bounds__(256)
    k_whiten_fused(const MatDev* __restrict__ mats, float mom_beta, float omb, float2* __restrict__ rs, int ld_rs,
                   float* __restrict__ pre, float* __restrict__ rho, float* __restrict__ rho2,
                   unsigned* __restrict__ tickets, __nv_bfloat16* __restrict__ xh, __nv_bfloat16* __restrict__ xl,
                   int64_t rp, int64_t cp, int which) {
  extern __shared__ __align__(128) uint8_t fused_smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ FrontSeg s_seg[8];
  __shared__ float s_dot[16], s_ib[16];
  __shared__ double sh[8];
  __shared__ int s_abort;
  grid_dep_wait();
  grid_dep_launch();
  const int b = blockIdx.y;
  const MatDev md = mats[b];
  const int R = fused_rows(md.d_in);
  const int o0 = blockIdx.x * R;
  // whole CTA: it takes no part in the matrix's ticket.  which: 0 every
  // matrix, 1 only transposed ones, 2 only untransposed ones (the streams
  // k_whiten_rows / k_whiten_cols take the others)
  if (o0 >= md.d_out || (which == 1 && !md.transposed) || (which == 2 && md.transposed)) return;
  const int rows = min(R, md.d_out - o0);
  const int n = md.d_in;
  const int n4 = n / 4;
  float* sg = reinterpret_cast<float*>(fused_smem);
  float* sm = sg + static_cast<size_t>(R) * n;
  const float scale = pre[b];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float2* rsb = rs + static_cast<int64_t>(b) * ld_rs;

  // ---- 1. the rows into shared memory
  const uint32_t bar_a = smem_u32(&bar);
  if (threadIdx.x == 0) {
    mbar_init(bar_a, 1);
    s_abort = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < rows) s_ib[threadIdx.x] = md.inv_b[o0 + threadIdx.x];
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t row_bytes = static_cast<uint32_t>(n) * 4u;
    mbar_arrive_expect_tx(bar_a, 2u * static_cast<uint32_t>(rows) * row_bytes);
    for (int r = 0; r < rows; ++r) {
      const int64_t off = static_cast<int64_t>(o0 + r) * n;
      bulk_load(smem_u32(sg + static_cast<size_t>(r) * n), md.grad + off, row_bytes, bar_a);
      bulk_load(smem_u32(sm + static_cast<size_t>(r) * n), md.mom + off, row_bytes, bar_a);
    }
  }
  bool ok = mbar_wait(bar_a, 0, &s_abort, kStatusTimeoutFrontLoad);
  ok = __syncthreads_and(ok) != 0;
  if (!ok) {
    // let the copies in flight land (bounded) before this CTA's shared memory goes
    mbar_wait(bar_a, 0, nullptr, kStatusTimeoutFrontLoad);
  } else {
    // ---- 2. row statistics: segment = (row, part), S parts per row
    const int S = R >= 8 ? 1 : 8 / R;
    for (int seg = warp; seg < rows * S; seg += 8) {
      const int r = seg / S, part = seg - r * S;
      const int lo4 = part * n4 / S, hi4 = (part + 1) * n4 / S;
      const float4* g4 = reinterpret_cast<const float4*>(sg + static_cast<size_t>(r) * n);
      const float4* m4 = reinterpret_cast<const float4*>(sm + static_cast<size_t>(r) * n);
      const float ib = s_ib[r];
      float dot = 0.0f;
      double sq = 0.0;
      for (int i4 = lo4 + lane; i4 < hi4; i4 += 32) {
        const float4 gv = g4[i4], mv = m4[i4];
        const float4 av = *reinterpret_cast<const float4*>(md.inv_a + 4 * i4);
        float4 zv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (RANK1) zv = *reinterpret_cast<const float4*>(md.z_a + 4 * i4);
        const float ge[4] = {gv.x, gv.y, gv.z, gv.w}, me[4] = {mv.x, mv.y, mv.z, mv.w};
        const float ae[4] = {av.x, av.y, av.z, av.w}, ze[4] = {zv.x, zv.y, zv.z, zv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mn = mom_beta * me[e] + omb * ge[e];
          const float src = mom_beta * mn + omb * ge[e];
          const float y = (src * ib) * ae[e];
          sq += static_cast<double>(y) * y;
          if (RANK1) dot += y * ze[e];
        }
      }
      sq = warp_sum_d(sq);
      dot = RANK1 ? warp_sum(dot) : 0.0f;
      if (lane == 0) {
        s_seg[seg & 7].dot = dot;
        s_seg[seg & 7].sq = sq;
        if (S == 1) {
          s_dot[r] = dot;
          rsb[o0 + r] = make_float2(dot, static_cast<float>(sqrt(sq)));
        }
      }
    }
    __syncthreads();
    if (S > 1 && threadIdx.x < rows) {
      const int r = threadIdx.x;
      float dot = 0.0f;
      double sq = 0.0;
      for (int part = 0; part < S; ++part) {
        dot += s_seg[r * S + part].dot;
        sq += s_seg[r * S + part].sq;
      }
      s_dot[r] = dot;
      rsb[o0 + r] = make_float2(dot, static_cast<float>(sqrt(sq)));
    }
    __syncthreads();

    // ---- 3. momentum and planes
    const float coef = RANK1 ? md.scal_a[0] : 0.0f;
    const int64_t plane = static_cast<int64_t>(b) * rp * cp;
    if (!md.transposed) {
      for (int it = threadIdx.x; it < rows * n4; it += blockDim.x) {
        const int r = it / n4, i4 = it - r * n4;
        const int o = o0 + r;
        const float4 gv = reinterpret_cast<const float4*>(sg + static_cast<size_t>(r) * n)[i4];
        const float4 mv = reinterpret_cast<const float4*>(sm + static_cast<size_t>(r) * n)[i4];
        const float4 av = *reinterpret_cast<const float4*>(md.inv_a + 4 * i4);
        float4 zv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (RANK1) zv = *reinterpret_cast<const float4*>(md.z_a + 4 * i4);
        const float ge[4] = {gv.x, gv.y, gv.z, gv.w}, me[4] = {mv.x, mv.y, mv.z, mv.w};
        const float ae[4] = {av.x, av.y, av.z, av.w}, ze[4] = {zv.x, zv.y, zv.z, zv.w};
        const float ib = s_ib[r], cw = coef * s_dot[r];
        float mn[4], h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          mn[e] = mom_beta * me[e] + omb * ge[e];
          const float src = mom_beta * mn[e] + omb * ge[e];
          float v = (src * ib) * ae[e];
          if (RANK1) v += cw * ze[e];
          split_hilo(v * scale, h[e], l[e]);
        }
        *reinterpret_cast<float4*>(md.mom + static_cast<int64_t>(o) * n + 4 * i4) =
            make_float4(mn[0], mn[1], mn[2], mn[3]);
        const int64_t xo = plane + static_cast<int64_t>(o) * cp + 4 * i4;
        *reinterpret_cast<uint2*>(xh + xo) = make_uint2(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]));
        *reinterpret_cast<uint2*>(xl + xo) = make_uint2(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]));
      }
    } else {
      // X row i = param column i; this CTA's rows are X columns o0 .. o0+rows
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float a = md.inv_a[i];
        const float z = RANK1 ? md.z_a[i] : 0.0f;
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int r = 0; r < 16; r += 2) {
          float h2[2] = {0.f, 0.f}, l2[2] = {0.f, 0.f};
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const int rr = r + q;
            if (rr < rows) {
              const float gv = sg[static_cast<size_t>(rr) * n + i];
              const float mv = sm[static_cast<size_t>(rr) * n + i];
              const float mn = mom_beta * mv + omb * gv;
              md.mom[static_cast<int64_t>(o0 + rr) * n + i] = mn;
              const float src = mom_beta * mn + omb * gv;
              float v = (src * s_ib[rr]) * a;
              if (RANK1) v += coef * s_dot[rr] * z;
              split_hilo(v * scale, h2[q], l2[q]);
            }
          }
          hw[r / 2] = pack_bf16x2(h2[0], h2[1]);
          lw[r / 2] = pack_bf16x2(l2[0], l2[1]);
        }
        __nv_bfloat16* dh = xh + plane + static_cast<int64_t>(i) * cp + o0;
        __nv_bfloat16* dl = xl + plane + static_cast<int64_t>(i) * cp + o0;
        if (rows == 16) {  // o0 % 16 == 0: 32-byte aligned
          reinterpret_cast<uint4*>(dh)[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          reinterpret_cast<uint4*>(dh)[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
          reinterpret_cast<uint4*>(dl)[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
          reinterpret_cast<uint4*>(dl)[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
        } else if (rows == 8) {  // o0 % 8 == 0: 16-byte aligned
          reinterpret_cast<uint4*>(dh)[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          reinterpret_cast<uint4*>(dl)[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        } else if (rows % 2 == 0) {  // o0 is even: 4-byte aligned pairs
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            if (2 * w < rows) {
              reinterpret_cast<uint32_t*>(dh)[w] = hw[w];
              reinterpret_cast<uint32_t*>(dl)[w] = lw[w];
            }
          }
        } else {
#pragma unroll
          for (int r = 0; r < 16; ++r) {
            if (r < rows) {
              const uint32_t wh = hw[r / 2], wl = lw[r / 2];
              dh[r] = __ushort_as_bfloat16(static_cast<unsigned short>((r & 1) ? (wh >> 16) : (wh & 0xFFFFu)));
              dl[r] = __ushort_as_bfloat16(static_cast<unsigned short>((r & 1) ? (wl >> 16) : (wl & 0xFFFFu)));
            }
          }
        }
      }
    }
  }
  // ---- 4. the matrix's last CTA: stage-1 alphas for these planes, next scale
  if (last_cta_of(tickets + b, static_cast<unsigned>((md.d_out + R - 1) / R))) {
    const double t = rows_sum_sq_y(rsb, md.d_out, sh);
    if (threadIdx.x == 0) {
      const double norm = sqrt(t);
      set_stage1_alphas(norm, scale, rho, rho2, b);
      const double placed = norm * scale;
      if (norm > 0.0 && !(placed > 0x1p-60 && placed < 0x1p60)) atomicExch(&g_status, kStatusFrontRange);
      pre[b] = plane_scale_for(norm);
    }
  }
}

// ===================================== N3 in one pass: untransposed row stream
// The matrices of a group whose param rows are X rows (d_out <= d_in) all
// have the group's shape r x n (n = d_in).  Their r * count rows form one
// stream; CTA c of the persistent grid takes the contiguous range
// [c * total / grid, (c+1) * total / grid) of it.  A CTA is one team of
// TW = rows_team_warps(n) warps, so every thread holds at most kRowsKMax
// float4 of a row: thread t owns the float4 columns t, t + 32 TW, ...  and
// keeps the matrix's inv_a (and z_a) for them in registers.  Rows arrive in
// a ring of kRowsStages shared-memory buffers (g row, m row) by bulk async
// copies (cp.async.bulk, no multicast) that thread 0 issues kRowsStages - 1
// rows ahead; each buffer completes on its own mbarrier (a bounded wait).
// Per row: (y . z_a, |y|) from registers-held columns (FP64 squares), then m'
// and the hi/lo planes of x = v * pre[b] at X[o, :] -- the same arithmetic
// as k_whiten_fused.  No CTA-wide phase separates loading from writing, so
// copies stay in flight while a row is written.  A matrix's ticket counts
// rows: a CTA adds its row count once per matrix segment it covers, and the
// CTA that completes the count reduces the row norms into the stage-1 alphas
// and the next plane scale.
constexpr int kRowsKMax = 8;     // float4 per thread per row
constexpr int kRowsStages = 3;   // row buffers per CTA

__host__ __device__ constexpr int rows_team_warps(int n) {
  int tw = 1;
  while (tw < 8 && n / 4 > 32 * tw * kRowsKMax) tw <<= 1;
  return tw;
}
// n that the row stream takes: float4 rows of at most 32 * 8 * kRowsKMax float4
__host__ __device__ constexpr bool rows_stream_fits(int n) { return n % 4 == 0 && n > 0 && n / 4 <= 32 * 8 * kRowsKMax; }
__host__ __device__ constexpr int rows_smem_bytes(int n) { return kRowsStages * 2 * n * 4; }

template <bool RANK1>
__global__ void __launch_bounds__(256)
    k_whiten_rows(const MatDev* __restrict__ mats, const int* __restrict__ slots, int count, int r, int n,
                  float mom_beta, float omb, float2* __restrict__ rs, int ld_rs, float* __restrict__ pre,
                  float* __restrict__ rho, float* __restrict__ rho2, unsigned* __restrict__ tickets,
                  __nv_bfloat16* __restrict__ xh, __nv_bfloat16* __restrict__ xl, int64_t rp, int64_t cp) {
  extern __shared__ __align__(128) uint8_t rows_smem[];
  __shared__ __align__(8) uint64_t full[kRowsStages];
  __shared__ FrontSeg s_part[2][8];
  __shared__ double sh[8];
  __shared__ unsigned s_last;
  __shared__ int s_abort;
  grid_dep_wait();
  grid_dep_launch();
  const int T = blockDim.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, TW = T >> 5;
  const int64_t total = static_cast<int64_t>(count) * r;
  const int64_t j0 = total * blockIdx.x / gridDim.x, j1 = total * (blockIdx.x + 1) / gridDim.x;
  const int rows = static_cast<int>(j1 - j0);
  if (rows <= 0) return;
  const int n4 = n / 4;
  const uint32_t row_bytes = static_cast<uint32_t>(n) * 4u;
  float* ring = reinterpret_cast<float*>(rows_smem);  // buffer s: g at ring + 2 n s, m after it

  // thread 0: bulk copies of stream row q (0-based in this CTA's range) into buffer q % S
  auto issue = [&](int q) {
    const int64_t j = j0 + q;
    const int k = static_cast<int>(j / r), o = static_cast<int>(j - static_cast<int64_t>(k) * r);
    const MatDev& m = mats[slots[k]];
    const int s = q % kRowsStages;
    const uint32_t bar = smem_u32(&full[s]);
    float* dst = ring + static_cast<size_t>(2 * s) * n;
    mbar_arrive_expect_tx(bar, 2u * row_bytes);
    bulk_load(smem_u32(dst), m.grad + static_cast<int64_t>(o) * n, row_bytes, bar);
    bulk_load(smem_u32(dst + n), m.mom + static_cast<int64_t>(o) * n, row_bytes, bar);
  };

  if (tid == 0) {
    for (int s = 0; s < kRowsStages; ++s) mbar_init(smem_u32(&full[s]), 1);
    s_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  int issued = min(kRowsStages, rows);
  if (tid == 0)
    for (int q = 0; q < issued; ++q) issue(q);

  float4 a_reg[kRowsKMax], z_reg[kRowsKMax];
  int cur_k = -1, b = 0, seg = 0;
  float scale = 1.0f, coef = 0.0f;
  const float* inv_b = nullptr;
  float* mom = nullptr;
  float2* rsb = nullptr;
  int64_t plane = 0;
  bool alive = true;
  int q_fail = rows;  // first row whose copies did not arrive

  // closes this CTA's segment of matrix b: its rows join the matrix's ticket
  auto close_segment = [&]() {
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      const unsigned t = atomicAdd(tickets + b, static_cast<unsigned>(seg));
      s_last = (t + static_cast<unsigned>(seg) == static_cast<unsigned>(r)) ? 1u : 0u;
      if (s_last) {
        __threadfence();
        tickets[b] = 0u;
      }
    }
    __syncthreads();
    if (s_last) {
      const double t = rows_sum_sq_y(rsb, r, sh);
      if (tid == 0) {
        const double norm = sqrt(t);
        set_stage1_alphas(norm, scale, rho, rho2, b);
        const double placed = norm * scale;
        if (norm > 0.0 && !(placed > 0x1p-60 && placed < 0x1p60)) atomicExch(&g_status, kStatusFrontRange);
        pre[b] = plane_scale_for(norm);
      }
      __syncthreads();
    }
  };

  for (int q = 0; q < rows; ++q) {
    const int64_t j = j0 + q;
    const int k = static_cast<int>(j / r), o = static_cast<int>(j - static_cast<int64_t>(k) * r);
    if (k != cur_k) {
      if (cur_k >= 0) close_segment();
      cur_k = k;
      b = slots[k];
      const MatDev& m = mats[b];
      inv_b = m.inv_b;
      mom = m.mom;
      coef = RANK1 ? m.scal_a[0] : 0.0f;
      scale = pre[b];
      rsb = rs + static_cast<int64_t>(b) * ld_rs;
      plane = static_cast<int64_t>(b) * rp * cp;
      seg = 0;
#pragma unroll
      for (int kk = 0; kk < kRowsKMax; ++kk) {
        const int i4 = tid + kk * T;
        a_reg[kk] = i4 < n4 ? reinterpret_cast<const float4*>(m.inv_a)[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
        z_reg[kk] = (RANK1 && i4 < n4) ? reinterpret_cast<const float4*>(m.z_a)[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    ++seg;
    const int s = q % kRowsStages;
    bool ok = alive && mbar_wait(smem_u32(&full[s]), static_cast<uint32_t>((q / kRowsStages) & 1), &s_abort,
                                 kStatusTimeoutFrontLoad);
    ok = __syncthreads_and(ok) != 0;
    if (!ok) {
      if (alive) q_fail = q;
      alive = false;
      continue;
    }
    // every thread is past row q - 1: its buffer takes the next row
    if (tid == 0 && q >= 1 && issued < rows) issue(issued++);
    const float4* g4 = reinterpret_cast<const float4*>(ring + static_cast<size_t>(2 * s) * n);
    const float4* m4 = g4 + n4;
    const float ib = inv_b[o];

    // row statistics
    float dot = 0.0f;
    double sq = 0.0;
#pragma unroll
    for (int kk = 0; kk < kRowsKMax; ++kk) {
      const int i4 = tid + kk * T;
      if (i4 < n4) {
        const float4 gv = g4[i4], mv = m4[i4];
        const float ge[4] = {gv.x, gv.y, gv.z, gv.w}, me[4] = {mv.x, mv.y, mv.z, mv.w};
        const float ae[4] = {a_reg[kk].x, a_reg[kk].y, a_reg[kk].z, a_reg[kk].w};
        const float ze[4] = {z_reg[kk].x, z_reg[kk].y, z_reg[kk].z, z_reg[kk].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mn = mom_beta * me[e] + omb * ge[e];
          const float src = mom_beta * mn + omb * ge[e];
          const float y = (src * ib) * ae[e];
          sq += static_cast<double>(y) * y;
          if (RANK1) dot += y * ze[e];
        }
      }
    }
    sq = warp_sum_d(sq);
    dot = RANK1 ? warp_sum(dot) : 0.0f;
    if (TW > 1) {
      if (lane == 0) {
        s_part[q & 1][warp].dot = dot;
        s_part[q & 1][warp].sq = sq;
      }
      __syncthreads();
      dot = 0.0f;
      sq = 0.0;
      for (int w = 0; w < TW; ++w) {
        dot += s_part[q & 1][w].dot;
        sq += s_part[q & 1][w].sq;
      }
    }
    if (tid == 0) rsb[o] = make_float2(dot, static_cast<float>(sqrt(sq)));

    // momentum and planes
    const float cw = coef * dot;
    float* mrow = mom + static_cast<int64_t>(o) * n;
    const int64_t xrow = plane + static_cast<int64_t>(o) * cp;
#pragma unroll
    for (int kk = 0; kk < kRowsKMax; ++kk) {
      const int i4 = tid + kk * T;
      if (i4 < n4) {
        const float4 gv = g4[i4], mv = m4[i4];
        const float ge[4] = {gv.x, gv.y, gv.z, gv.w}, me[4] = {mv.x, mv.y, mv.z, mv.w};
        const float ae[4] = {a_reg[kk].x, a_reg[kk].y, a_reg[kk].z, a_reg[kk].w};
        const float ze[4] = {z_reg[kk].x, z_reg[kk].y, z_reg[kk].z, z_reg[kk].w};
        float mn[4], h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          mn[e] = mom_beta * me[e] + omb * ge[e];
          const float src = mom_beta * mn[e] + omb * ge[e];
          float v = (src * ib) * ae[e];
          if (RANK1) v += cw * ze[e];
          split_hilo(v * scale, h[e], l[e]);
        }
        reinterpret_cast<float4*>(mrow)[i4] = make_float4(mn[0], mn[1], mn[2], mn[3]);
        const int64_t xo = xrow + 4 * i4;
        *reinterpret_cast<uint2*>(xh + xo) = make_uint2(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]));
        *reinterpret_cast<uint2*>(xl + xo) = make_uint2(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]));
      }
    }
  }
  close_segment();
  if (!alive && tid == 0) {
    // the copies still in flight land (bounded) before this CTA's shared memory goes
    for (int q = q_fail; q < issued; ++q) {
      const int s = q % kRowsStages;
      mbar_wait(smem_u32(&full[s]), static_cast<uint32_t>((q / kRowsStages) & 1), nullptr, kStatusTimeoutFrontLoad);
    }
  }
}

// ===================================== N3 in one pass: transposed block stream
// The transposed matrices of a group (d_out = c > d_in = n = r) have param
// rows that are X columns.  Their 16-row blocks form one stream; CTA c of the
// persistent grid (one CTA per SM) takes a contiguous range of blocks.  A
// block's g rows and m rows are contiguous in memory: one bulk async copy
// each (cp.async.bulk, no multicast) into a 2-stage ring, thread 0 issuing
// the next block while the current one is processed (bounded mbarrier waits).
// Thread = (4 consecutive X rows i..i+3, part p of kColsParts row parts of
// 16 / kColsParts param rows): the 32 / kColsParts lanes of a part take
// consecutive float4 columns, so the 16-byte shared loads are conflict-free,
// and the parts of a warp together write whole 32-byte sectors of their X
// rows (16 bf16: the block's 16 param rows).  One thread per item, so a
// thread keeps its columns' inv_a (and z_a) in registers for the whole
// matrix and its rows' inv_b for the block.
//   1. per param row: (y . z_a, |y|^2) partial sums over the thread's
//      columns, reduced over the lanes of a part (shuffles), then over the
//      warps in warp order (shared memory): deterministic;
//   2. m' and the hi/lo planes of x = v * pre[b], as k_whiten_fused.
// A matrix's ticket counts blocks: a CTA adds its block count once per
// matrix segment; the CTA that completes the count reduces the row norms.
#ifndef SMB_COLS_PARTS
#define SMB_COLS_PARTS 4
#endif
constexpr int kColsRows = 16;   // param rows per block
constexpr int kColsStages = 2;
constexpr int kColsParts = SMB_COLS_PARTS;       // 2 or 4
constexpr int kColsPartRows = kColsRows / kColsParts;
constexpr int kColsLanes = 32 / kColsParts;     // lanes per part
static_assert(kColsParts == 2 || kColsParts == 4, "2 or 4 row parts");
// 4 parts: up to 24 warps of at most 80 registers; 2 parts: 16 of at most 128
constexpr int kColsMaxThreads = kColsParts == 4 ? 768 : 512;

__host__ __device__ constexpr int cols_smem_bytes(int n) { return kColsStages * 2 * kColsRows * n * 4; }
// items (= threads): the float4 columns rounded up to whole parts, times the parts
__host__ __device__ constexpr int cols_threads(int n) { return ((n / 4 + kColsLanes - 1) / kColsLanes) * 32; }
__host__ __device__ constexpr bool cols_stream_fits(int n) {
  return n % 4 == 0 && n > 0 && cols_smem_bytes(n) <= 196608 && cols_threads(n) <= kColsMaxThreads;
}

template <bool RANK1>
__global__ void __launch_bounds__(kColsMaxThreads, 1)
    k_whiten_cols(const MatDev* __restrict__ mats, const int* __restrict__ slots, int count, int c, int n,
                  float mom_beta, float omb, float2* __restrict__ rs, int ld_rs, float* __restrict__ pre,
                  float* __restrict__ rho, float* __restrict__ rho2, unsigned* __restrict__ tickets,
                  __nv_bfloat16* __restrict__ xh, __nv_bfloat16* __restrict__ xl, int64_t rp, int64_t cp) {
  extern __shared__ __align__(128) uint8_t cols_smem[];
  __shared__ __align__(8) uint64_t full[kColsStages];
  __shared__ float s_pdot[32][kColsRows];   // [warp][row] partials
  __shared__ double s_psq[32][kColsRows];
  __shared__ float s_dot[kColsRows];
  __shared__ double sh[32];
  __shared__ unsigned s_last;
  __shared__ int s_abort;
  grid_dep_wait();
  grid_dep_launch();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, NW = blockDim.x >> 5;
  const int nb = (c + kColsRows - 1) / kColsRows;  // blocks per matrix
  const int64_t total = static_cast<int64_t>(count) * nb;
  const int64_t j0 = total * blockIdx.x / gridDim.x, j1 = total * (blockIdx.x + 1) / gridDim.x;
  const int blocks = static_cast<int>(j1 - j0);
  if (blocks <= 0) return;
  const int n4 = n / 4;
  float* ring = reinterpret_cast<float*>(cols_smem);  // stage s: g rows at ring + 2 R n s, m rows after
  const int part = lane / kColsLanes;
  const int i4 = warp * kColsLanes + (lane % kColsLanes);  // this thread's float4 column
  const bool has = i4 < n4;
  const int r0 = part * kColsPartRows;                     // its first row of a block

  auto issue = [&](int q) {
    const int64_t j = j0 + q;
    const int k = static_cast<int>(j / nb), blk = static_cast<int>(j - static_cast<int64_t>(k) * nb);
    const int o0 = blk * kColsRows, rows = min(kColsRows, c - o0);
    const MatDev& m = mats[slots[k]];
    const int s = q % kColsStages;
    const uint32_t bar = smem_u32(&full[s]);
    float* dst = ring + static_cast<size_t>(2 * s) * kColsRows * n;
    const uint32_t bytes = static_cast<uint32_t>(rows) * static_cast<uint32_t>(n) * 4u;
    mbar_arrive_expect_tx(bar, 2u * bytes);
    bulk_load(smem_u32(dst), m.grad + static_cast<int64_t>(o0) * n, bytes, bar);
    bulk_load(smem_u32(dst + kColsRows * n), m.mom + static_cast<int64_t>(o0) * n, bytes, bar);
  };

  if (tid == 0) {
    for (int s = 0; s < kColsStages; ++s) mbar_init(smem_u32(&full[s]), 1);
    s_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  int issued = min(kColsStages, blocks);
  if (tid == 0)
    for (int q = 0; q < issued; ++q) issue(q);

  int cur_k = -1, b = 0, seg = 0;
  float scale = 1.0f, coef = 0.0f;
  const MatDev* md = nullptr;
  float2* rsb = nullptr;
  int64_t plane = 0;
  float4 av = make_float4(0.f, 0.f, 0.f, 0.f), zv = make_float4(0.f, 0.f, 0.f, 0.f);
  bool alive = true;
  int q_fail = blocks;

  auto close_segment = [&]() {
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      const unsigned t = atomicAdd(tickets + b, static_cast<unsigned>(seg));
      s_last = (t + static_cast<unsigned>(seg) == static_cast<unsigned>(nb)) ? 1u : 0u;
      if (s_last) {
        __threadfence();
        tickets[b] = 0u;
      }
    }
    __syncthreads();
    if (s_last) {
      const double t = rows_sum_sq_y(rsb, c, sh);
      if (tid == 0) {
        const double norm = sqrt(t);
        set_stage1_alphas(norm, scale, rho, rho2, b);
        const double placed = norm * scale;
        if (norm > 0.0 && !(placed > 0x1p-60 && placed < 0x1p60)) atomicExch(&g_status, kStatusFrontRange);
        pre[b] = plane_scale_for(norm);
      }
      __syncthreads();
    }
  };

  for (int q = 0; q < blocks; ++q) {
    const int64_t j = j0 + q;
    const int k = static_cast<int>(j / nb), blk = static_cast<int>(j - static_cast<int64_t>(k) * nb);
    if (k != cur_k) {
      if (cur_k >= 0) close_segment();
      cur_k = k;
      b = slots[k];
      md = mats + b;
      coef = RANK1 ? md->scal_a[0] : 0.0f;
      scale = pre[b];
      rsb = rs + static_cast<int64_t>(b) * ld_rs;
      plane = static_cast<int64_t>(b) * rp * cp;
      seg = 0;
      if (has) {
        av = reinterpret_cast<const float4*>(md->inv_a)[i4];
        if (RANK1) zv = reinterpret_cast<const float4*>(md->z_a)[i4];
      }
    }
    ++seg;
    const int o0 = blk * kColsRows, rows = min(kColsRows, c - o0);
    float ib[kColsPartRows];
#pragma unroll
    for (int r = 0; r < kColsPartRows; ++r) ib[r] = r0 + r < rows ? md->inv_b[o0 + r0 + r] : 0.0f;
    const int s = q % kColsStages;
    bool ok = alive && mbar_wait(smem_u32(&full[s]), static_cast<uint32_t>((q / kColsStages) & 1), &s_abort,
                                 kStatusTimeoutFrontLoad);
    ok = __syncthreads_and(ok) != 0;
    if (!ok) {
      if (alive) q_fail = q;
      alive = false;
      continue;
    }
    if (tid == 0 && q >= 1 && issued < blocks) issue(issued++);
    const float* sg = ring + static_cast<size_t>(2 * s) * kColsRows * n;
    const float* smo = sg + kColsRows * n;
    const float ae[4] = {av.x, av.y, av.z, av.w}, ze[4] = {zv.x, zv.y, zv.z, zv.w};

    // 1. row statistics of this part's rows over the thread's columns
    float pdot[kColsPartRows];
    double psq[kColsPartRows];
#pragma unroll
    for (int r = 0; r < kColsPartRows; ++r) {
      pdot[r] = 0.0f;
      psq[r] = 0.0;
      const int rr = r0 + r;
      if (has && rr < rows) {
        const float4 gv = reinterpret_cast<const float4*>(sg + static_cast<size_t>(rr) * n)[i4];
        const float4 mv = reinterpret_cast<const float4*>(smo + static_cast<size_t>(rr) * n)[i4];
        const float ge[4] = {gv.x, gv.y, gv.z, gv.w}, me[4] = {mv.x, mv.y, mv.z, mv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mn = mom_beta * me[e] + omb * ge[e];
          const float src = mom_beta * mn + omb * ge[e];
          const float y = (src * ib[r]) * ae[e];
          psq[r] += static_cast<double>(y) * y;
          if (RANK1) pdot[r] += y * ze[e];
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kColsPartRows; ++r) {
#pragma unroll
      for (int off = kColsLanes / 2; off > 0; off >>= 1) {
        psq[r] += __shfl_xor_sync(0xffffffffu, psq[r], off);
        if (RANK1) pdot[r] += __shfl_xor_sync(0xffffffffu, pdot[r], off);
      }
    }
    if (lane % kColsLanes == 0) {
#pragma unroll
      for (int r = 0; r < kColsPartRows; ++r) {
        s_pdot[warp][r0 + r] = pdot[r];
        s_psq[warp][r0 + r] = psq[r];
      }
    }
    __syncthreads();
    if (tid < kColsRows) {
      float dot = 0.0f;
      double sq = 0.0;
      for (int w = 0; w < NW; ++w) {
        dot += s_pdot[w][tid];
        sq += s_psq[w][tid];
      }
      s_dot[tid] = dot;
      if (tid < rows) rsb[o0 + tid] = make_float2(dot, static_cast<float>(sqrt(sq)));
    }
    __syncthreads();

    // 2. momentum and this part's 16 / kColsParts X columns of rows i..i+3
    if (has) {
      uint32_t hw[4][kColsPartRows / 2], lw[4][kColsPartRows / 2];  // [X row e][bf16 pair of param rows]
      float* mom = md->mom + static_cast<int64_t>(o0) * n;
#pragma unroll
      for (int w2 = 0; w2 < kColsPartRows / 2; ++w2) {
        float hv[2][4], lv[2][4];
#pragma unroll
        for (int q2 = 0; q2 < 2; ++q2) {
          const int r = 2 * w2 + q2, rr = r0 + r;
          if (rr < rows) {
            const float4 gv = reinterpret_cast<const float4*>(sg + static_cast<size_t>(rr) * n)[i4];
            const float4 mv = reinterpret_cast<const float4*>(smo + static_cast<size_t>(rr) * n)[i4];
            const float cw = coef * s_dot[rr];
            const float ge[4] = {gv.x, gv.y, gv.z, gv.w}, me[4] = {mv.x, mv.y, mv.z, mv.w};
            float mn[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              mn[e] = mom_beta * me[e] + omb * ge[e];
              const float src = mom_beta * mn[e] + omb * ge[e];
              float v = (src * ib[r]) * ae[e];
              if (RANK1) v += cw * ze[e];
              split_hilo(v * scale, hv[q2][e], lv[q2][e]);
            }
            reinterpret_cast<float4*>(mom + static_cast<int64_t>(rr) * n)[i4] = make_float4(mn[0], mn[1], mn[2], mn[3]);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              hv[q2][e] = 0.0f;
              lv[q2][e] = 0.0f;
            }
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          hw[e][w2] = pack_bf16x2(hv[0][e], hv[1][e]);
          lw[e][w2] = pack_bf16x2(lv[0][e], lv[1][e]);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t xo = plane + static_cast<int64_t>(4 * i4 + e) * cp + o0 + r0;
        if constexpr (kColsPartRows == 8) {
          *reinterpret_cast<uint4*>(xh + xo) = make_uint4(hw[e][0], hw[e][1], hw[e][2], hw[e][3]);
          *reinterpret_cast<uint4*>(xl + xo) = make_uint4(lw[e][0], lw[e][1], lw[e][2], lw[e][3]);
        } else {
          *reinterpret_cast<uint2*>(xh + xo) = make_uint2(hw[e][0], hw[e][1]);
          *reinterpret_cast<uint2*>(xl + xo) = make_uint2(lw[e][0], lw[e][1]);
        }
      }
    }
  }
  close_segment();
  if (!alive && tid == 0) {
    for (int q = q_fail; q < issued; ++q) {
      const int s = q % kColsStages;
      mbar_wait(smem_u32(&full[s]), static_cast<uint32_t>((q / kColsStages) & 1), nullptr, kStatusTimeoutFrontLoad);
    }
  }
}

// ================================================ S8 stage-1 scale and poly
// s[b] = max(1.35 * |G2_b|_F^(1/4), 1e-30) from the per-tile partial sums of
// squares written by the G*G epilogue (sandmuon/optimizer.py:81), then
// P = a I + b G / s / s + c G2 / s / s / s / s (sandmuon/optimizer.py:83-84),
// emitted as hi/lo BF16 planes in place of the G hi/lo planes.  Every CTA of
// matrix b reduces the matrix's partials itself (a few hundred floats from
// L2, in one fixed order, so every CTA derives the same s); the matrix's
// first CTA also stores s, 1/s and the stage-1 P X alpha rho[b] / s[b].
// Four consecutive elements (one row, rp % 4 == 0) per thread and iteration.
__global__ void __launch_bounds__(256)
    k_poly_stage1(__nv_bfloat16* __restrict__ gh, __nv_bfloat16* __restrict__ gl, const float* __restrict__ g2,
                  const float* __restrict__ partials, int per_mat, float margin, float* __restrict__ s,
                  float* __restrict__ s_inv, const float* __restrict__ rho, float* __restrict__ px_alpha, int rp,
                  float pa, float pb, float pc) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ double sh[8];
  const int b = blockIdx.y;
  double acc = 0.0;
  for (int p = threadIdx.x; p < per_mat; p += blockDim.x) acc += partials[static_cast<int64_t>(b) * per_mat + p];
  const double t = block_sum_d<256>(acc, sh);
  const float sv = fmaxf(margin * powf(static_cast<float>(sqrt(t)), 0.25f), 1e-30f);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    s[b] = sv;
    s_inv[b] = 1.0f / sv;
    // stage-1 P X: (P x) / s with x = rho * (stored planes)
    px_alpha[b] = rho[b] * (1.0f / sv);
  }
  const int64_t per4 = static_cast<int64_t>(rp) * rp / 4;
  // Multiplications by 1/s, one at a time: for a zero matrix (s = 1e-30, so
  // 1/s = 1e30 while 1/s^2 would overflow) every partial product stays 0 and
  // P = a I exactly; for a normalised input s is O(1).
  const float is = 1.0f / sv;
  const int64_t base = static_cast<int64_t>(b) * rp * rp;
  for (int64_t i4 = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i4 < per4;
       i4 += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i4 * 4;
    const int r = static_cast<int>(e / rp);
    const int c = static_cast<int>(e - static_cast<int64_t>(r) * rp);
    const uint2 wh = *reinterpret_cast<const uint2*>(gh + base + e);
    const uint2 wl = *reinterpret_cast<const uint2*>(gl + base + e);
    const float4 w2 = *reinterpret_cast<const float4*>(g2 + base + e);
    const float gv[4] = {bf16_lo_to_f(wh.x) + bf16_lo_to_f(wl.x), bf16_hi_to_f(wh.x) + bf16_hi_to_f(wl.x),
                         bf16_lo_to_f(wh.y) + bf16_lo_to_f(wl.y), bf16_hi_to_f(wh.y) + bf16_hi_to_f(wl.y)};
    const float g2v[4] = {w2.x, w2.y, w2.z, w2.w};
    float hi[4], lo[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float t1 = (gv[q] * is) * is;
      const float t2 = (((g2v[q] * is) * is) * is) * is;
      const float p = (r == c + q ? pa : 0.0f) + pb * t1 + pc * t2;
      split_hilo(p, hi[q], lo[q]);
    }
    *reinterpret_cast<uint2*>(gh + base + e) = make_uint2(pack_bf16x2(hi[0], hi[1]), pack_bf16x2(hi[2], hi[3]));
    *reinterpret_cast<uint2*>(gl + base + e) = make_uint2(pack_bf16x2(lo[0], lo[1]), pack_bf16x2(lo[2], lo[3]));
  }
}

// ============================================ N7 pass 1: mapback row stats
// Mapback U = diag(inv_b) (Q + c (Q z) z^T) diag(inv_a) in param coordinates
// (rank1_mapback, sandmuon/optimizer.py:48-60, both orientations: the last S8
// GEMM stores Q of a transposed matrix already transposed, so Q is always in
// the param layout [d_out, d_in] with row stride ldq = transposed ? rp : cp).
// Per param row o (one warp, 16-byte loads):
//   t = sum_i z_i Q_oi, S1 = sum_i a_i^2 Q_oi^2, S2 = sum_i a_i^2 z_i Q_oi
//   |U_o|^2 = inv_b_o^2 (S1 + 2 c t S2 + c^2 t^2 sum_i a_i^2 z_i^2)
// out[o] = {t, |U_o|^2}.
__device__ __forceinline__ int64_t q_ld(const MatDev& md, int64_t rp, int64_t cp) {
  return md.transposed ? rp : cp;
}

#ifndef SMB_MAPBACK_MINB
#define SMB_MAPBACK_MINB 3  // 80 registers, 3 CTAs per SM: 62 -> 56 us on config 1
#endif
template <bool RANK1>
__global__ void __launch_bounds__(256, SMB_MAPBACK_MINB)
    k_mapback_rowstats(const MatDev* __restrict__ mats, const __nv_bfloat16* __restrict__ q, int64_t rp, int64_t cp,
                       float2* __restrict__ out, int ld_out, float* __restrict__ gamma,
                       unsigned* __restrict__ tickets) {
  grid_dep_wait();
  grid_dep_launch();
  __shared__ double sh[8];
  const int b = blockIdx.y;
  const MatDev md = mats[b];
  const int o0 = blockIdx.x * 8 * kMapbackRows;
  if (o0 >= md.d_out) return;  // whole CTA: it takes no part in the matrix's ticket
  const int obase = o0 + (threadIdx.x >> 5) * kMapbackRows;
  const int lane = threadIdx.x & 31;
  float2* outb = out + static_cast<int64_t>(b) * ld_out;
  if (obase < md.d_out) {
    const __nv_bfloat16* qr[kMapbackRows];
    float t[kMapbackRows], s1[kMapbackRows], s2[kMapbackRows];
#pragma unroll
    for (int r = 0; r < kMapbackRows; ++r) {
      const int o = min(obase + r, md.d_out - 1);
      qr[r] = q + static_cast<int64_t>(b) * rp * cp + static_cast<int64_t>(o) * q_ld(md, rp, cp);
      t[r] = 0.f;
      s1[r] = 0.f;
      s2[r] = 0.f;
    }
    // 8 BF16 (16 bytes) per lane and row: Q rows are 16-byte aligned (row
    // strides are multiples of 128 elements); the rows' tails go one by one
    const int n8 = md.d_in & ~7;
    for (int i = lane * 8; i < n8; i += 256) {
      float aa[8], zz[8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float4 a = *reinterpret_cast<const float4*>(md.inv_a + i + 4 * h);
        aa[4 * h + 0] = a.x * a.x; aa[4 * h + 1] = a.y * a.y; aa[4 * h + 2] = a.z * a.z; aa[4 * h + 3] = a.w * a.w;
        float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        if (RANK1) z = *reinterpret_cast<const float4*>(md.z_a + i + 4 * h);
        zz[4 * h + 0] = z.x; zz[4 * h + 1] = z.y; zz[4 * h + 2] = z.z; zz[4 * h + 3] = z.w;
      }
      uint4 raw[kMapbackRows];
#pragma unroll
      for (int r = 0; r < kMapbackRows; ++r) raw[r] = *reinterpret_cast<const uint4*>(qr[r] + i);
#pragma unroll
      for (int r = 0; r < kMapbackRows; ++r) {
        const uint32_t w[4] = {raw[r].x, raw[r].y, raw[r].z, raw[r].w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float v = (e & 1) ? bf16_hi_to_f(w[e >> 1]) : bf16_lo_to_f(w[e >> 1]);
          s1[r] += aa[e] * v * v;
          if (RANK1) {
            t[r] += zz[e] * v;
            s2[r] += aa[e] * zz[e] * v;
          }
        }
      }
    }
    for (int i = n8 + lane; i < md.d_in; i += 32) {
      const float a2 = md.inv_a[i] * md.inv_a[i];
      const float z = RANK1 ? md.z_a[i] : 0.f;
#pragma unroll
      for (int r = 0; r < kMapbackRows; ++r) {
        const float v = __bfloat162float(qr[r][i]);
        s1[r] += a2 * v * v;
        if (RANK1) {
          t[r] += z * v;
          s2[r] += a2 * z * v;
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kMapbackRows; ++r) {
      const float s1r = warp_sum(s1[r]);
      const float tr = RANK1 ? warp_sum(t[r]) : 0.f;
      const float s2r = RANK1 ? warp_sum(s2[r]) : 0.f;
      const int o = obase + r;
      if (lane == 0 && o < md.d_out) {
        const double ib = md.inv_b[o];
        double row = s1r;
        if (RANK1) {
          const double c = md.scal_a[0], k2 = md.scal_a[1];
          row = s1r + 2.0 * c * tr * s2r + c * c * static_cast<double>(tr) * tr * k2;
        }
        outb[o] = make_float2(tr, static_cast<float>(ib * ib * row));
      }
    }
  }
  // gamma[b] = sqrt(d_out) / max(|U_b|_F, tiny)  (_graft_direction,
  // sandmuon/optimizer.py:63-66), by the matrix's last CTA
  if (last_cta_of(tickets + b, static_cast<unsigned>((md.d_out + 8 * kMapbackRows - 1) / (8 * kMapbackRows)))) {
    const double total = rows_sum_y(outb, md.d_out, sh);
    if (threadIdx.x == 0) gamma[b] = md.sqrt_rows / fmaxf(static_cast<float>(sqrt(total)), kFltTiny);
  }
}

// Peer delivery of updated weights (a sharded step's weight exchange done by
// the update kernel itself): every updated weight of a matrix flagged
// MatDev::peer is also stored at byte offset delta[r] from its local address,
// the same position in peer r's copy of the flat weight buffer, mapped into
// this device's address space (plain stores over NVLink; no multicast).
constexpr int kMaxPeers = 15;
struct PeerSet {
  int32_t n;
  int32_t pad;
  int64_t delta[kMaxPeers];
};

// ======================================== N7 pass 2: mapback + update apply
// W[o,i] -= lr * gamma * inv_b[o] * inv_a[i] * (Q[o,i] + c t[o] z[i])
// (sandmuon/optimizer.py:303-315).  Grid-stride over the matrix (blockIdx.y)
// in 16-byte groups when d_in % 4 == 0, else element by element.
template <bool RANK1, bool VEC4>
__global__ void __launch_bounds__(256)
    k_mapback_apply(const MatDev* __restrict__ mats, const __nv_bfloat16* __restrict__ q, int64_t rp, int64_t cp,
                    const float2* __restrict__ rs, int ld_rs, const float* __restrict__ gamma, const PeerSet peers) {
  grid_dep_wait();
  grid_dep_launch();
  const int b = blockIdx.y;
  const MatDev md = mats[b];
  const __nv_bfloat16* qb = q + static_cast<int64_t>(b) * rp * cp;
  const int64_t ldq = q_ld(md, rp, cp);
  const float step = md.lr * gamma[b];
  const float coef = RANK1 ? md.scal_a[0] : 0.0f;
  const int per_row = VEC4 ? md.d_in / 4 : md.d_in;
  const int n_peers = md.peer ? peers.n : 0;
  const int64_t total = static_cast<int64_t>(md.d_out) * per_row;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int o = static_cast<int>(idx / per_row);
    const int col = static_cast<int>(idx - static_cast<int64_t>(o) * per_row);
    const float ib = md.inv_b[o];
    const float ct = RANK1 ? coef * rs[static_cast<int64_t>(b) * ld_rs + o].x : 0.0f;
    if (VEC4) {
      const int i = col * 4;
      const uint2 raw = *reinterpret_cast<const uint2*>(qb + static_cast<int64_t>(o) * ldq + i);
      const float4 v = make_float4(bf16_lo_to_f(raw.x), bf16_hi_to_f(raw.x), bf16_lo_to_f(raw.y),
                                   bf16_hi_to_f(raw.y));
      const float4 a = *reinterpret_cast<const float4*>(md.inv_a + i);
      float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      if (RANK1) z = *reinterpret_cast<const float4*>(md.z_a + i);
      float4* wp = reinterpret_cast<float4*>(md.weight + static_cast<int64_t>(o) * md.d_in + i);
      float4 w = *wp;
      float4 d = make_float4(step * (((v.x + ct * z.x) * ib) * a.x), step * (((v.y + ct * z.y) * ib) * a.y),
                             step * (((v.z + ct * z.z) * ib) * a.z), step * (((v.w + ct * z.w) * ib) * a.w));
      if (md.export_bf16) {
        // every rank applies the same rounded delta (k_apply_bf16_delta)
        const uint2 packed = make_uint2(pack_bf16x2(d.x, d.y), pack_bf16x2(d.z, d.w));
        d = make_float4(bf16_lo_to_f(packed.x), bf16_hi_to_f(packed.x), bf16_lo_to_f(packed.y),
                        bf16_hi_to_f(packed.y));
        *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(md.export_to) +
                                  static_cast<int64_t>(o) * md.d_in + i) = packed;
      }
      w.x = w.x - d.x;
      w.y = w.y - d.y;
      w.z = w.z - d.z;
      w.w = w.w - d.w;
      *wp = w;
      for (int r = 0; r < n_peers; ++r)
        *reinterpret_cast<float4*>(reinterpret_cast<char*>(wp) + peers.delta[r]) = w;
      if (md.export_to != nullptr && !md.export_bf16)
        *reinterpret_cast<float4*>(md.export_to + static_cast<int64_t>(o) * md.d_in + i) = w;
    } else {
      const int i = col;
      float v = __bfloat162float(qb[static_cast<int64_t>(o) * ldq + i]);
      if (RANK1) v += ct * md.z_a[i];
      const float u = (v * ib) * md.inv_a[i];
      const int64_t wi = static_cast<int64_t>(o) * md.d_in + i;
      float d = step * u;
      if (md.export_bf16) {
        const __nv_bfloat16 db = __float2bfloat16_rn(d);
        reinterpret_cast<__nv_bfloat16*>(md.export_to)[wi] = db;
        d = __bfloat162float(db);
      }
      const float w = md.weight[wi] - d;
      md.weight[wi] = w;
      for (int r = 0; r < n_peers; ++r)
        *reinterpret_cast<float*>(reinterpret_cast<char*>(md.weight + wi) + peers.delta[r]) = w;
      if (md.export_to != nullptr && !md.export_bf16) md.export_to[wi] = w;
    }
  }
}

// ======================================================= multi-tensor copy
constexpr int kCopyMax = 64;

struct CopyBatch {
  uint8_t* dst[kCopyMax];
  const uint8_t* src[kCopyMax];
  int64_t bytes[kCopyMax];
  int64_t chunk_start[kCopyMax + 1];  // prefix sums of 64 KB chunks
  int32_t count;
};

constexpr int64_t kCopyChunk = 65536;

__global__ void __launch_bounds__(256) k_copy_multi(const CopyBatch batch) {
  const int64_t total = batch.chunk_start[batch.count];
  for (int64_t ch = blockIdx.x; ch < total; ch += gridDim.x) {
    int t = 0;
    while (batch.chunk_start[t + 1] <= ch) ++t;
    const int64_t base = (ch - batch.chunk_start[t]) * kCopyChunk;
    const int64_t end = min(base + kCopyChunk, batch.bytes[t]);
    const uint8_t* s = batch.src[t];
    uint8_t* d = batch.dst[t];
    const bool vec = ((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d) | batch.bytes[t]) & 15) == 0;
    if (vec) {
      for (int64_t o = base + threadIdx.x * 16; o < end; o += blockDim.x * 16)
        *reinterpret_cast<uint4*>(d + o) = *reinterpret_cast<const uint4*>(s + o);
    } else {
      for (int64_t o = base + threadIdx.x; o < end; o += blockDim.x) d[o] = s[o];
    }
  }
}

// ============================================= multi-tensor BF16 delta apply
struct DeltaBatch {
  float* weight[kCopyMax];
  const __nv_bfloat16* delta[kCopyMax];
  int64_t numel[kCopyMax];
  int64_t chunk_start[kCopyMax + 1];  // prefix sums of kDeltaChunk-element chunks
  int32_t count;
};

constexpr int64_t kDeltaChunk = 8192;

// weight[i] -= float(delta[i]): the update a sharded step's owner applied to
// its own copy (k_mapback_apply with export_bf16), replayed on another rank.
__global__ void __launch_bounds__(256) k_apply_bf16_delta(const DeltaBatch batch) {
  const int64_t total = batch.chunk_start[batch.count];
  for (int64_t ch = blockIdx.x; ch < total; ch += gridDim.x) {
    int t = 0;
    while (batch.chunk_start[t + 1] <= ch) ++t;
    const int64_t base = (ch - batch.chunk_start[t]) * kDeltaChunk;
    const int64_t end = min(base + kDeltaChunk, batch.numel[t]);
    float* w = batch.weight[t];
    const __nv_bfloat16* d = batch.delta[t];
    const bool vec = ((reinterpret_cast<uintptr_t>(w) & 15) | (reinterpret_cast<uintptr_t>(d) & 7) |
                      (batch.numel[t] & 3)) == 0;
    if (vec) {
      for (int64_t i = base + threadIdx.x * 4; i < end; i += blockDim.x * 4) {
        const uint2 p = *reinterpret_cast<const uint2*>(d + i);
        float4 v = *reinterpret_cast<float4*>(w + i);
        v.x -= bf16_lo_to_f(p.x);
        v.y -= bf16_hi_to_f(p.x);
        v.z -= bf16_lo_to_f(p.y);
        v.w -= bf16_hi_to_f(p.y);
        *reinterpret_cast<float4*>(w + i) = v;
      }
    } else {
      for (int64_t i = base + threadIdx.x; i < end; i += blockDim.x) w[i] -= __bfloat162float(d[i]);
    }
  }
}

// ============================================================ N8: AdamW
constexpr int kAdamMaxTensors = 24;

struct AdamBatch {
  float* param[kAdamMaxTensors];
  const float* grad[kAdamMaxTensors];
  float* m1[kAdamMaxTensors];
  float* m2[kAdamMaxTensors];
  int64_t numel[kAdamMaxTensors];
  int64_t chunk_start[kAdamMaxTensors + 1];  // prefix sums of 4096-element chunks
  float bc1[kAdamMaxTensors];
  float bc2[kAdamMaxTensors];
  int32_t count;
};

constexpr int kAdamChunk = 4096;

__global__ void __launch_bounds__(256)
    k_adamw_multi(const AdamBatch batch, float lr, float beta1, float omb1, float beta2, float omb2, float eps,
                  float decay) {
  const int64_t total_chunks = batch.chunk_start[batch.count];
  for (int64_t ch = blockIdx.x; ch < total_chunks; ch += gridDim.x) {
    int t = 0;
    while (batch.chunk_start[t + 1] <= ch) ++t;
    const int64_t base = (ch - batch.chunk_start[t]) * kAdamChunk;
    const int64_t end = min(base + kAdamChunk, batch.numel[t]);
    float* p = batch.param[t];
    const float* g = batch.grad[t];
    float* m1 = batch.m1[t];
    float* m2 = batch.m2[t];
    const float bc1 = batch.bc1[t], bc2 = batch.bc2[t];
    for (int64_t e = base + threadIdx.x; e < end; e += blockDim.x) {
      const float gv = g[e];
      const float a = m1[e] * beta1 + omb1 * gv;
      const float v = m2[e] * beta2 + omb2 * (gv * gv);
      m1[e] = a;
      m2[e] = v;
      const float upd = (a / bc1) / (sqrtf(v / bc2) + eps);
      const float pv = p[e] * decay;
      p[e] = pv - lr * upd;
    }
  }
}

}  // namespace smb
