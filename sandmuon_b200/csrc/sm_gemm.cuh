// sm_gemm.cuh -- batched BF16 GEMM on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// C[b] = A[b] * op(B[b]) for every matrix b of up to kMaxProblems batches in
// one launch: the dense products of the S8 polynomial (x x^T, gram gram, p x;
// sandmuon/optimizer.py:79-91) for every shape group of an optimizer at once.
//
// Design (one persistent CTA per SM, 10 warps):
//   warp 0      TMA producer: streams A/B k-blocks (128-byte swizzle, BK = 64)
//               into a STAGES-deep shared-memory ring.
//   warp 1      MMA issuer: owns the TMEM allocation; one thread issues
//               tcgen05.mma (M=128, N=BN, K=16) into a double-buffered FP32
//               accumulator in TMEM and releases ring slots with tcgen05.commit.
//   warps 2..9  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows; the two warps of a lane quarter take
//               alternate 32-column chunks), apply the fused epilogue, store.
// CTA-pair mode (CG = 2, clusters of two CTAs): a pair computes a 256 x BN
// tile with tcgen05 cta_group::2 (M = 256).  Each CTA streams its own 128 A
// rows and BN/2 of the B columns, so a ring slot holds half the B bytes of
// the single-CTA mode and one SM's operand traffic per FLOP drops by a third
// (compensated BN=256: 64 KB per slot instead of 96 KB, three slots instead
// of two).  Both CTAs' TMA loads complete on the leader's full barrier; the
// leader alone issues the MMAs and multicasts its commits to both CTAs' ring
// and accumulator barriers; each CTA's epilogue drains its own TMEM rows and
// arrives on the leader's accumulator-empty barrier.
// Compensated mode (stages 1-4 of S8) loads hi and lo BF16 planes of both
// operands and issues three MMAs per k-step into the same accumulator:
//   acc += A_hi*B_lo; acc += A_lo*B_hi; acc += A_hi*B_hi
// (the three-product order of the historical compensated kernel,
// reproduction/odl/ops/bf16_compensated_mm_fast.py:64-66).
// Operands are K-major ([M or N, K] rows: x for x x^T) or MN-major ([K, M or
// N] rows: x for p x, and the symmetric p and g read as their own transposes).
// No cluster multicast is used.
// Tiles are visited in a host-computed per-CTA order (longest first, balanced
// by k-blocks) when a schedule is given, else round-robin.
#pragma once

#include "sm_common.cuh"

namespace smb {

constexpr int kGemmBM = 128;
constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr int kMaxProblems = 4;
// F32Norm partial slots per output tile: one per epilogue warp and CTA of a pair.
constexpr int kNormSlots = SM_EPI_NORM_SLOTS;
static_assert(kNormSlots == 2 * kEpiWarps, "norm partial slots");

enum GemmEpi : int {
  kEpiF32 = SM_EPI_F32,
  kEpiBF16 = SM_EPI_BF16,
  kEpiHiLo = SM_EPI_HILO,
  kEpiF32Norm = SM_EPI_F32_NORM,
  kEpiPoly = SM_EPI_POLY,
  kEpiPolyHiLo = SM_EPI_POLY_HILO,
};

// One batched problem of a launch: its TMA descriptors and epilogue operands.
struct GemmProblem {
  CUtensorMap a_hi, a_lo, b_hi, b_lo;
  int m, n, k;          // per-matrix problem (multiples of 128 / BN / BK)
  int batch;
  int tiles_m, tiles_n;
  int tile_begin;       // first launch-global tile index of this problem
  int sym;              // 1: C is symmetric (m == n): only the upper block triangle
                        // is computed (square tiles, or 256 x 128 pair tiles) and
                        // the blocks above the diagonal also store C^T
  void* out0;           // [batch, m, n] FP32 or BF16 (hi plane for hi/lo outputs)
  void* out1;           // lo plane for hi/lo outputs
  const float* alpha;   // [batch] scale of the accumulator, or null (= 1)
  // aux / aux_lo / pa / pb / pc: the polynomial epilogues, reachable through
  // sm_gemm_bf16 (the optimizer's S8 uses scale / diag with a shifted gram)
  const __nv_bfloat16* aux;     // [batch, m, n] BF16 gram (hi plane) for the poly epilogues
  const __nv_bfloat16* aux_lo;  // lo plane of the gram for the hi/lo poly epilogue
  float pa, pb, pc;     // poly coefficients: out = pa*I + pb*gram + pc*acc
  float scale;          // F32 / BF16 / hi-lo epilogues: out = scale*alpha*acc + diag*I
  float diag;
  float* partials;      // [batch, tiles_m*tiles_n*kNormSlots] sum of squares (F32Norm)
  const int* tmask;     // [batch] or null: 1 = store this matrix's result transposed
                        // ([n, m], row stride m) -- F32 and BF16 epilogues only
};

struct GemmLaunch {
  GemmProblem p[kMaxProblems];
  int n_problems;
  int total_tiles;
  // Optional schedule over workers (CTAs, or CTA pairs in pair mode):
  // sched[0..workers] = per-worker offsets into sched[workers+1..] (launch-
  // global tile indices).  Null: worker w visits w, w + workers, ...
  const int* sched;
};

template <int BN, int BK, bool COMP, int STAGES, int CG>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * BK * 2;       // this CTA's 128 A rows
  static constexpr int kBBytes = (BN / CG) * BK * 2;     // this CTA's share of B
  static constexpr int kOps = COMP ? 2 : 1;
  static constexpr int kStageBytes = kOps * (kABytes + kBBytes);
  static constexpr int kBarrierBytes = (2 * STAGES + 4) * 8 + 16;
  // Epilogue staging: per epilogue warp one 32 x 32 FP32 chunk padded to 33
  // floats per row, so row writes and column reads are both conflict-free.
  static constexpr int kStageWords = 32 * 33;
  static constexpr int kStagingBytes = kEpiWarps * kStageWords * 4;
  // +1024 for manual alignment of the dynamic shared memory base.
  static constexpr int kTotal = STAGES * kStageBytes + kBarrierBytes + kStagingBytes + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN;
};

// Launch-global tile index -> (problem, matrix, m-tile, n-tile); `slot` is
// the tile's index among the `per` tiles computed for one matrix.
struct TileCoord {
  int q, b, mi, ni, slot, per;
};

__device__ __forceinline__ TileCoord decode_tile(const GemmLaunch& L, int t) {
  int q = 0;
#pragma unroll
  for (int i = 1; i < kMaxProblems; ++i)
    if (i < L.n_problems && t >= L.p[i].tile_begin) q = i;
  const GemmProblem& P = L.p[q];
  const int local = t - P.tile_begin;
  TileCoord c;
  c.q = q;
  if (P.sym) {
    // The upper block triangle, row tile by row tile: row tile mi needs the
    // column tiles ni >= R * mi, R = tiles_n / tiles_m (1 for square tiles,
    // 2 for 256 x 128 pair tiles).
    const int R = P.tiles_n / P.tiles_m;
    const int per = P.tiles_m * P.tiles_n - R * P.tiles_m * (P.tiles_m - 1) / 2;
    c.b = local / per;
    int u = local - c.b * per;
    c.slot = u;
    c.per = per;
    int mi = 0;
    while (u >= P.tiles_n - R * mi) {
      u -= P.tiles_n - R * mi;
      ++mi;
    }
    c.mi = mi;
    c.ni = R * mi + u;
  } else {
    const int per = P.tiles_m * P.tiles_n;
    c.b = local / per;
    const int rem = local - c.b * per;
    c.slot = rem;
    c.per = per;
    c.mi = rem / P.tiles_n;
    c.ni = rem - c.mi * P.tiles_n;
  }
  return c;
}

// The sequence of tiles a worker (CTA, or CTA pair) visits; identical for
// all three warp roles and both CTAs of a pair.
template <int CG>
struct TileIter {
  const int* list;
  int pos, end, step;
  __device__ __forceinline__ explicit TileIter(const GemmLaunch& L) {
    const int worker = static_cast<int>(blockIdx.x) / CG;
    const int workers = static_cast<int>(gridDim.x) / CG;
    if (L.sched != nullptr) {
      list = L.sched + workers + 1;
      pos = L.sched[worker];
      end = L.sched[worker + 1];
      step = 1;
    } else {
      list = nullptr;
      pos = worker;
      end = L.total_tiles;
      step = workers;
    }
  }
  __device__ __forceinline__ bool valid() const { return pos < end; }
  __device__ __forceinline__ int tile() const { return list != nullptr ? list[pos] : pos; }
  __device__ __forceinline__ void next() { pos += step; }
};

template <int BN, int BK, bool COMP, bool A_MN, bool B_MN, int STAGES, int EPI, int CG>
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm_bf16(const __grid_constant__ GemmLaunch L) {
  using S = GemmSmem<BN, BK, COMP, STAGES, CG>;
  using W = Swz;
  static_assert((A_MN || BK == 64) && (B_MN || BK == 64), "K-major operands need BK = 64");
  static_assert(CG == 1 || CG == 2, "one CTA or a CTA pair per tile");
  static_assert(!B_MN || (BN / CG) % W::kChunkElems == 0, "an MN-major B share is whole 64-column chunks");
  constexpr bool kPair = CG == 2;
  constexpr int kTileM = kGemmBM * CG;  // output rows of one tile (both CTAs of a pair)
  constexpr int kBRows = BN / CG;       // B rows / columns this CTA stages
  constexpr int kKSteps = BK / 16;
  constexpr uint32_t kChunk = W::chunk_bytes(BK);
  constexpr uint32_t kIdesc = umma_idesc_bf16(kTileM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  // bars[0, S): full, [S, 2S): empty, [2S, 2S+2): tmem full, [2S+2, 2S+4): tmem empty
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* staging = reinterpret_cast<uint32_t*>(smem + STAGES * S::kStageBytes + S::kBarrierBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;  // 0 = the pair's MMA leader
  const uint32_t bar_base = smem_u32(bars);
  auto bar_full = [&](int s) { return bar_base + 8u * s; };
  auto bar_empty = [&](int s) { return bar_base + 8u * (STAGES + s); };
  auto bar_tfull = [&](int a) { return bar_base + 8u * (2 * STAGES + a); };
  auto bar_tempty = [&](int a) { return bar_base + 8u * (2 * STAGES + 2 + a); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_tfull(a), 1);
      mbar_init(bar_tempty(a), kEpiWarps * CG);  // the epilogue warps of both CTAs of a pair
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  __syncwarp();
  // A pair's CTAs signal each other's barriers: both are initialised first.
  if (kPair) cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    if (kPair) tmem_alloc_pair(smem_u32(tmem_slot), S::kTmemCols);
    else tmem_alloc(smem_u32(tmem_slot), S::kTmemCols);
  }
  if (warp == 0 && lane == 0) {
    for (int q = 0; q < L.n_problems; ++q) {
      tma_prefetch_desc(&L.p[q].a_hi);
      tma_prefetch_desc(&L.p[q].b_hi);
      if (COMP) {
        tma_prefetch_desc(&L.p[q].a_lo);
        tma_prefetch_desc(&L.p[q].b_lo);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above is private to this CTA; operands and outputs may belong
  // to the previous kernel of the stream until here.
  grid_dep_wait();
  grid_dep_launch();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (TileIter<CG> it(L); it.valid() && ok; it.next()) {
        const TileCoord tc = decode_tile(L, it.tile());
        const GemmProblem& P = L.p[tc.q];
        const int kblocks = P.k / BK;
        const int a_row = tc.mi * kTileM + static_cast<int>(rank) * kGemmBM;
        const int b_row = tc.ni * BN + static_cast<int>(rank) * kBRows;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(bar_empty(stage), phase ^ 1u, abort_flag, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          // The leader's full barrier counts the bytes of both CTAs of a pair.
          const uint32_t fb = bar_full(stage);
          const uint32_t fb_tx = kPair ? mapa_shared(fb, 0) : fb;
          if (rank == 0) mbar_arrive_expect_tx(fb, CG * S::kStageBytes);
          auto load = [&](uint32_t dst, const CUtensorMap* map, int c0, int c1) {
            if (kPair) tma_load_3d_pair(dst, map, fb_tx, c0, c1, tc.b);
            else tma_load_3d(dst, map, fb, c0, c1, tc.b);
          };
          const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + S::kOps * S::kABytes;
          const int kc = kb * BK;
          if (!A_MN) {
            load(sa, &P.a_hi, kc, a_row);
            if (COMP) load(sa + S::kABytes, &P.a_lo, kc, a_row);
          } else {
#pragma unroll
            for (int j = 0; j < kGemmBM / W::kChunkElems; ++j) {
              const int mc = a_row + W::kChunkElems * j;
              load(sa + j * kChunk, &P.a_hi, mc, kc);
              if (COMP) load(sa + S::kABytes + j * kChunk, &P.a_lo, mc, kc);
            }
          }
          if (!B_MN) {
            load(sb, &P.b_hi, kc, b_row);
            if (COMP) load(sb + S::kBBytes, &P.b_lo, kc, b_row);
          } else {
#pragma unroll
            for (int j = 0; j < kBRows / W::kChunkElems; ++j) {
              const int nc = b_row + W::kChunkElems * j;
              load(sb + j * kChunk, &P.b_hi, nc, kc);
              if (COMP) load(sb + S::kBBytes + j * kChunk, &P.b_lo, nc, kc);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every ring slot's last release (a commit, from the peer's
      // leader in a pair) has arrived before this CTA may leave.
      for (int i = 0; i < STAGES && ok; ++i) {
        ok = mbar_wait(bar_empty(stage), phase ^ 1u, abort_flag, kStatusTimeoutProducer);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    // (the leader's thread only, for both CTAs of a pair)
    if (lane == 0 && rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (TileIter<CG> it(L); it.valid() && ok; it.next(), ++local) {
        const TileCoord tc = decode_tile(L, it.tile());
        const int kblocks = L.p[tc.q].k / BK;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(bar_tempty(acc), acc_phase ^ 1u, abort_flag, kStatusTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(bar_full(stage), phase, abort_flag, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + S::kOps * S::kABytes;
#pragma unroll
          for (int ks = 0; ks < kKSteps; ++ks) {
            auto opdesc = [&](uint32_t base, bool mn) -> uint64_t {
              return mn ? umma_desc(base + ks * W::kMnStepBytes, kChunk, W::kSbo, W::kLayout)
                        : umma_desc(base + ks * 32, 16, W::kSbo, W::kLayout);
            };
            auto mma = [&](uint64_t a, uint64_t b, uint32_t accumulate) {
              if (kPair) umma_bf16_pair(d_tmem, a, b, kIdesc, accumulate);
              else umma_bf16(d_tmem, a, b, kIdesc, accumulate);
            };
            const uint64_t a_hi = opdesc(sa, A_MN);
            const uint64_t b_hi = opdesc(sb, B_MN);
            const uint32_t accumulate = (kb > 0 || ks > 0) ? 1u : 0u;
            if (COMP) {
              const uint64_t a_lo = opdesc(sa + S::kABytes, A_MN);
              const uint64_t b_lo = opdesc(sb + S::kBBytes, B_MN);
              mma(a_hi, b_lo, accumulate);
              mma(a_lo, b_hi, 1u);
              mma(a_hi, b_hi, 1u);
            } else {
              mma(a_hi, b_hi, accumulate);
            }
          }
          // Ring slot `stage` is free in both CTAs once these MMAs complete.
          if (kPair) umma_commit_pair(bar_empty(stage), 0x3);
          else umma_commit(bar_empty(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (kPair) umma_commit_pair(bar_tfull(acc), 0x3);
        else umma_commit(bar_tfull(acc));
      }
      // Drain: both accumulators released by every epilogue warp (the
      // peer's arrive remotely) before the leader may leave.
      for (int i = 0; i < 2 && ok; ++i, ++local) {
        ok = mbar_wait(bar_tempty(local & 1), ((local >> 1) & 1) ^ 1u, abort_flag, kStatusTimeoutMma);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;          // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;      // which alternate column chunks it takes
    // the leader's accumulator-empty barriers (shared::cluster addresses)
    const uint32_t tempty_leader0 = kPair ? mapa_shared(bar_tempty(0), 0) : bar_tempty(0);
    int local = 0;
    for (TileIter<CG> it(L); it.valid(); it.next(), ++local) {
      const TileCoord tc = decode_tile(L, it.tile());
      const GemmProblem& P = L.p[tc.q];
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // Every lane polls; the vote keeps the warp converged (and uniform on
      // timeout) before the .sync.aligned TMEM loads below.
      const bool ready = mbar_wait(bar_tfull(acc), acc_phase, abort_flag, kStatusTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();

      // first row of this warp's slab: the tile, this CTA's half of a pair, the lane quarter
      const int row0 = tc.mi * kTileM + static_cast<int>(rank) * kGemmBM + quarter * 32;
      const int row = row0 + lane;                        // the TMEM lane = tile row of this thread
      const size_t mat_off = static_cast<size_t>(tc.b) * P.m * P.n;
      const float alpha = (P.alpha != nullptr ? P.alpha[tc.b] : 1.0f) * P.scale;
      // Symmetric output: a block above the diagonal is also stored transposed.
      // With 256 x 128 pair tiles a CTA's block is 128 x 128 (row block rb);
      // the one below the diagonal in a diagonal tile is skipped, its
      // transpose coming from the tile to its right.
      bool mirror = false, skip = false;
      if (P.sym) {
        if (kTileM == BN) {
          mirror = tc.ni != tc.mi;
        } else {
          const int rb = tc.mi * CG + static_cast<int>(rank);
          mirror = tc.ni > rb;
          skip = tc.ni < rb;
        }
      }
      float sumsq = 0.0f;
      float* stg = reinterpret_cast<float*>(staging) + (warp - 2) * S::kStageWords;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
      if (skip) {
        // Nothing of this block is stored: release the accumulator at once.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (kPair) mbar_arrive_cluster(tempty_leader0 + 8u * acc);
          else mbar_arrive(bar_tempty(acc));
        }
      }
#pragma unroll 1
      for (int j = half; j < BN / 32 && !skip; j += 2) {
        uint32_t r[32];
        tmem_ld_32x32(t_row + j * 32, r);
        tmem_wait_ld();
        if (j + 2 >= BN / 32) {
          // Accumulator fully read into registers: hand it back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if (kPair) mbar_arrive_cluster(tempty_leader0 + 8u * acc);
            else mbar_arrive(bar_tempty(acc));
          }
        }
        const int col0 = tc.ni * BN + j * 32;
        float v[32];
        if (EPI == kEpiPoly || EPI == kEpiPolyHiLo) {
          // The gram chunk (32 rows x 32 BF16), loaded coalesced (4 lanes x 8
          // elements per row), combined hi + lo, staged, read back by rows.
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int rr = 8 * it + (lane >> 2);
            const int c8 = (lane & 3) * 8;
            const size_t off = mat_off + static_cast<size_t>(row0 + rr) * P.n + col0 + c8;
            const uint4 gh = *reinterpret_cast<const uint4*>(P.aux + off);
            const uint32_t wh[4] = {gh.x, gh.y, gh.z, gh.w};
            float g[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              g[2 * e] = bf16_lo_to_f(wh[e]);
              g[2 * e + 1] = bf16_hi_to_f(wh[e]);
            }
            if (EPI == kEpiPolyHiLo) {
              const uint4 gl = *reinterpret_cast<const uint4*>(P.aux_lo + off);
              const uint32_t wl[4] = {gl.x, gl.y, gl.z, gl.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                g[2 * e] += bf16_lo_to_f(wl[e]);
                g[2 * e + 1] += bf16_hi_to_f(wl[e]);
              }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) stg[rr * 33 + c8 + e] = g[e];
          }
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            v[c] = P.pb * stg[lane * 33 + c] + P.pc * __uint_as_float(r[c]);
            if (col0 + c == row) v[c] += P.pa;
          }
          __syncwarp();
        } else {
          // the chunk's columns col0 .. col0+31 hold this row's diagonal element
          const bool diag_here = P.diag != 0.0f && row >= col0 && row < col0 + 32;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            v[c] = alpha * __uint_as_float(r[c]);
            if (diag_here && col0 + c == row) v[c] += P.diag;
          }
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          stg[lane * 33 + c] = v[c];
          if (EPI == kEpiF32Norm) sumsq += v[c] * v[c];
        }
        __syncwarp();
        // Coalesced stores of the chunk (rows row0.., cols col0..) and, for an
        // off-diagonal tile of a symmetric product or a matrix whose FP32
        // result is stored transposed, of its transpose (rows col0.., cols
        // row0..), read from the staging tile by columns.
        const bool tout = (EPI == kEpiF32 || EPI == kEpiBF16) && P.tmask != nullptr && P.tmask[tc.b] != 0;
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
          if (pass == 0 && tout) continue;
          if (pass == 1 && !mirror && !tout) break;
          const int orow0 = pass == 0 ? row0 : col0;
          const int ocol0 = pass == 0 ? col0 : row0;
          if (EPI == kEpiF32 || EPI == kEpiF32Norm) {
            float* out = static_cast<float*>(P.out0) + mat_off;
            const size_t ld = tout ? P.m : P.n;
#pragma unroll
            for (int it = 0; it < 8; ++it) {
              const int rr = 4 * it + (lane >> 3);
              const int c4 = (lane & 7) * 4;
              float4 o;
              if (pass == 0) {
                o = make_float4(stg[rr * 33 + c4], stg[rr * 33 + c4 + 1], stg[rr * 33 + c4 + 2],
                                stg[rr * 33 + c4 + 3]);
              } else {
                o = make_float4(stg[c4 * 33 + rr], stg[(c4 + 1) * 33 + rr], stg[(c4 + 2) * 33 + rr],
                                stg[(c4 + 3) * 33 + rr]);
              }
              *reinterpret_cast<float4*>(out + static_cast<size_t>(orow0 + rr) * ld + ocol0 + c4) = o;
            }
          } else {
            constexpr bool kTwo = (EPI == kEpiHiLo || EPI == kEpiPolyHiLo);
            __nv_bfloat16* out_h = static_cast<__nv_bfloat16*>(P.out0) + mat_off;
            __nv_bfloat16* out_l = kTwo ? static_cast<__nv_bfloat16*>(P.out1) + mat_off : nullptr;
#pragma unroll
            for (int it = 0; it < 4; ++it) {
              const int rr = 8 * it + (lane >> 2);
              const int c8 = (lane & 3) * 8;
              float x[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) x[e] = pass == 0 ? stg[rr * 33 + c8 + e] : stg[(c8 + e) * 33 + rr];
              const size_t ld = tout ? P.m : P.n;
              const size_t off = static_cast<size_t>(orow0 + rr) * ld + ocol0 + c8;
              if (kTwo) {
                float h[8], l[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) split_hilo(x[e], h[e], l[e]);
                *reinterpret_cast<uint4*>(out_h + off) = make_uint4(
                    pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]), pack_bf16x2(h[6], h[7]));
                *reinterpret_cast<uint4*>(out_l + off) = make_uint4(
                    pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]), pack_bf16x2(l[4], l[5]), pack_bf16x2(l[6], l[7]));
              } else {
                *reinterpret_cast<uint4*>(out_h + off) = make_uint4(
                    pack_bf16x2(x[0], x[1]), pack_bf16x2(x[2], x[3]), pack_bf16x2(x[4], x[5]), pack_bf16x2(x[6], x[7]));
              }
            }
          }
        }
        __syncwarp();
      }
      if (EPI == kEpiF32Norm) {
        // A block above the diagonal stands for itself and its mirror (a
        // skipped one for nothing).  A single CTA also clears the slots a
        // pair's second CTA would use; the tiles_m x tiles_n slots past the
        // `per` computed tiles of a symmetric product are cleared by tile
        // slot - per (per >= half the grid), so the matrix sum stays exact.
        sumsq = warp_sum(sumsq);
        if (lane == 0) {
          const int slot = static_cast<int>(rank) * kEpiWarps + (warp - 2);
          float* part = P.partials + static_cast<size_t>(tc.b) * P.tiles_m * P.tiles_n * kNormSlots;
          const size_t own = static_cast<size_t>(tc.slot) * kNormSlots;
          part[own + slot] = mirror ? 2.0f * sumsq : sumsq;
          if (!kPair) part[own + kEpiWarps + slot] = 0.0f;
          const int spare = tc.slot + tc.per;
          if (spare < P.tiles_m * P.tiles_n) {
            part[static_cast<size_t>(spare) * kNormSlots + slot] = 0.0f;
            if (!kPair) part[static_cast<size_t>(spare) * kNormSlots + kEpiWarps + slot] = 0.0f;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // Neither CTA of a pair frees TMEM or leaves while the other may still
  // signal its barriers or the leader's MMAs may still read its operands.
  if (kPair) cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if (kPair) tmem_dealloc_pair(tmem_base, S::kTmemCols);
    else tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace smb
