// sm_gemm.cuh -- batched BF16 GEMM on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// C[b] = A[b] * op(B[b]) for every matrix b of up to kMaxProblems batches in
// one launch: the dense products of the S8 polynomial (x x^T, gram gram, p x;
// sandmuon/optimizer.py:79-91) for every shape group of an optimizer at once.
//
// Design (one persistent CTA per SM, 10 warps):
//   warp 0      TMA producer: streams A/B k-blocks (128-byte swizzle; BK = 64
//               for K-major operands, BK = 32 when both operands are MN-major)
//               into a STAGES-deep shared-memory ring.
//   warp 1      MMA issuer: owns the TMEM allocation; one thread issues
//               tcgen05.mma (M=128, N=BN, K=16) into a double-buffered FP32
//               accumulator in TMEM and releases ring slots with tcgen05.commit.
//   warps 2..9  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows; the two warps of a lane quarter take
//               alternate 32-column chunks), apply the fused epilogue, store.
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
  int sym;              // 1: C is symmetric (m == n, BN == 128): only tiles with
                        // ni >= mi are computed, off-diagonal ones also store C^T
  void* out0;           // [batch, m, n] FP32 or BF16 (hi plane for hi/lo outputs)
  void* out1;           // lo plane for hi/lo outputs
  const float* alpha;   // [batch] scale of the accumulator, or null (= 1)
  const __nv_bfloat16* aux;     // [batch, m, n] BF16 gram (hi plane) for the poly epilogues
  const __nv_bfloat16* aux_lo;  // lo plane of the gram for the hi/lo poly epilogue
  float pa, pb, pc;     // poly coefficients: out = pa*I + pb*gram + pc*acc
  float* partials;      // [batch, tiles_m*tiles_n*kEpiWarps] sum of squares (F32Norm)
  const int* tmask;     // [batch] or null: 1 = store this matrix's FP32 result
                        // transposed ([n, m], row stride m) -- F32 epilogue only
};

struct GemmLaunch {
  GemmProblem p[kMaxProblems];
  int n_problems;
  int total_tiles;
  // Optional schedule: sched[0..grid] = per-CTA offsets into sched[grid+1..]
  // (launch-global tile indices).  Null: CTA c visits c, c + grid, ...
  const int* sched;
};

template <int BN, int BK, bool COMP, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
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

// Launch-global tile index -> (problem, matrix, m-tile, n-tile).
struct TileCoord {
  int q, b, mi, ni, local;
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
    // upper-triangular tiles of a tiles_m x tiles_m grid, row by row
    const int per = P.tiles_m * (P.tiles_m + 1) / 2;
    c.b = local / per;
    int u = local - c.b * per;
    int mi = 0;
    while (u >= P.tiles_m - mi) {
      u -= P.tiles_m - mi;
      ++mi;
    }
    c.mi = mi;
    c.ni = mi + u;
  } else {
    const int per = P.tiles_m * P.tiles_n;
    c.b = local / per;
    const int rem = local - c.b * per;
    c.mi = rem / P.tiles_n;
    c.ni = rem - c.mi * P.tiles_n;
  }
  c.local = c.mi * P.tiles_n + c.ni;
  return c;
}

// The sequence of tiles a CTA visits; identical for all three warp roles.
struct TileIter {
  const int* list;
  int pos, end, step;
  __device__ __forceinline__ explicit TileIter(const GemmLaunch& L) {
    if (L.sched != nullptr) {
      list = L.sched + gridDim.x + 1;
      pos = L.sched[blockIdx.x];
      end = L.sched[blockIdx.x + 1];
      step = 1;
    } else {
      list = nullptr;
      pos = blockIdx.x;
      end = L.total_tiles;
      step = gridDim.x;
    }
  }
  __device__ __forceinline__ bool valid() const { return pos < end; }
  __device__ __forceinline__ int tile() const { return list != nullptr ? list[pos] : pos; }
  __device__ __forceinline__ void next() { pos += step; }
};

template <int BN, int BK, bool COMP, bool A_MN, bool B_MN, int STAGES, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm_bf16(const __grid_constant__ GemmLaunch L) {
  using S = GemmSmem<BN, BK, COMP, STAGES>;
  using W = Swz;
  static_assert((A_MN || BK == 64) && (B_MN || BK == 64), "K-major operands need BK = 64");
  constexpr int kKSteps = BK / 16;
  constexpr uint32_t kChunk = W::chunk_bytes(BK);
  constexpr uint32_t kIdesc = umma_idesc_bf16(kGemmBM, BN, A_MN, B_MN);

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
      mbar_init(bar_tempty(a), kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), S::kTmemCols);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (TileIter it(L); it.valid() && ok; it.next()) {
        const TileCoord tc = decode_tile(L, it.tile());
        const GemmProblem& P = L.p[tc.q];
        const int kblocks = P.k / BK;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(bar_empty(stage), phase ^ 1u, abort_flag, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar_full(stage);
          mbar_arrive_expect_tx(fb, S::kStageBytes);
          const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + S::kOps * S::kABytes;
          const int kc = kb * BK;
          if (!A_MN) {
            tma_load_3d(sa, &P.a_hi, fb, kc, tc.mi * kGemmBM, tc.b);
            if (COMP) tma_load_3d(sa + S::kABytes, &P.a_lo, fb, kc, tc.mi * kGemmBM, tc.b);
          } else {
#pragma unroll
            for (int j = 0; j < kGemmBM / W::kChunkElems; ++j) {
              const int mc = tc.mi * kGemmBM + W::kChunkElems * j;
              tma_load_3d(sa + j * kChunk, &P.a_hi, fb, mc, kc, tc.b);
              if (COMP) tma_load_3d(sa + S::kABytes + j * kChunk, &P.a_lo, fb, mc, kc, tc.b);
            }
          }
          if (!B_MN) {
            tma_load_3d(sb, &P.b_hi, fb, kc, tc.ni * BN, tc.b);
            if (COMP) tma_load_3d(sb + S::kBBytes, &P.b_lo, fb, kc, tc.ni * BN, tc.b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / W::kChunkElems; ++j) {
              const int nc = tc.ni * BN + W::kChunkElems * j;
              tma_load_3d(sb + j * kChunk, &P.b_hi, fb, nc, kc, tc.b);
              if (COMP) tma_load_3d(sb + S::kBBytes + j * kChunk, &P.b_lo, fb, nc, kc, tc.b);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (TileIter it(L); it.valid() && ok; it.next(), ++local) {
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
            const uint64_t a_hi = opdesc(sa, A_MN);
            const uint64_t b_hi = opdesc(sb, B_MN);
            const uint32_t accumulate = (kb > 0 || ks > 0) ? 1u : 0u;
            if (COMP) {
              const uint64_t a_lo = opdesc(sa + S::kABytes, A_MN);
              const uint64_t b_lo = opdesc(sb + S::kBBytes, B_MN);
              umma_bf16(d_tmem, a_hi, b_lo, kIdesc, accumulate);
              umma_bf16(d_tmem, a_lo, b_hi, kIdesc, 1u);
              umma_bf16(d_tmem, a_hi, b_hi, kIdesc, 1u);
            } else {
              umma_bf16(d_tmem, a_hi, b_hi, kIdesc, accumulate);
            }
          }
          umma_commit(bar_empty(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(bar_tfull(acc));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;          // TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;      // which alternate column chunks it takes
    int local = 0;
    for (TileIter it(L); it.valid(); it.next(), ++local) {
      const TileCoord tc = decode_tile(L, it.tile());
      const GemmProblem& P = L.p[tc.q];
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // Every lane polls; the vote keeps the warp converged (and uniform on
      // timeout) before the .sync.aligned TMEM loads below.
      const bool ready = mbar_wait(bar_tfull(acc), acc_phase, abort_flag, kStatusTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();

      const int row0 = tc.mi * kGemmBM + quarter * 32;  // first row of this warp's slab
      const int row = row0 + lane;                        // the TMEM lane = tile row of this thread
      const size_t mat_off = static_cast<size_t>(tc.b) * P.m * P.n;
      const float alpha = P.alpha != nullptr ? P.alpha[tc.b] : 1.0f;
      const bool mirror = P.sym && tc.ni != tc.mi;
      float sumsq = 0.0f;
      float* stg = reinterpret_cast<float*>(staging) + (warp - 2) * S::kStageWords;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int j = half; j < BN / 32; j += 2) {
        uint32_t r[32];
        tmem_ld_32x32(t_row + j * 32, r);
        tmem_wait_ld();
        if (j + 2 >= BN / 32) {
          // Accumulator fully read into registers: hand it back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_tempty(acc));
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
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = alpha * __uint_as_float(r[c]);
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
        const bool tout = (EPI == kEpiF32) && P.tmask != nullptr && P.tmask[tc.b] != 0;
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
              const size_t off = static_cast<size_t>(orow0 + rr) * P.n + ocol0 + c8;
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
        // An off-diagonal tile stands for itself and its mirror; the mirror's
        // partial slots are cleared so the per-matrix sum stays exact.
        sumsq = warp_sum(sumsq);
        if (lane == 0) {
          const int slot = warp - 2;
          float* part = P.partials + static_cast<size_t>(tc.b) * P.tiles_m * P.tiles_n * kEpiWarps;
          part[tc.local * kEpiWarps + slot] = mirror ? 2.0f * sumsq : sumsq;
          if (mirror) part[(tc.ni * P.tiles_n + tc.mi) * kEpiWarps + slot] = 0.0f;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace smb
