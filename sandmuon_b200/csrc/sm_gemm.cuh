// sm_gemm.cuh -- batched BF16 GEMM on sm_100a tensor cores (tcgen05 + TMEM + TMA).
//
// C[b] = A[b] * op(B[b]) for every matrix b of a batch, the dense products of
// the S8 polynomial (x x^T, gram gram, p x; sandmuon/optimizer.py:79-91).
//
// Design (one persistent CTA per SM, 6 warps):
//   warp 0      TMA producer: streams A/B k-blocks (64 BF16 = 128 B rows,
//               128-byte swizzle) into a STAGES-deep shared-memory ring.
//   warp 1      MMA issuer: owns the TMEM allocation; one thread issues
//               tcgen05.mma (M=128, N=BN, K=16) into a double-buffered FP32
//               accumulator in TMEM and releases ring slots with tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31 = tile rows), apply the fused epilogue, store.
// Compensated mode (stage 1 of S8) loads hi and lo BF16 planes of both
// operands and issues three MMAs per k-step into the same accumulator:
//   acc += A_hi*B_lo; acc += A_lo*B_hi; acc += A_hi*B_hi
// (the three-product order of the historical compensated kernel,
// reproduction/odl/ops/bf16_compensated_mm_fast.py:64-66).
// B is either K-major ([N, K] rows, for x x^T and the symmetric gram gram) or
// MN-major ([K, N] rows, for p x).  No cluster multicast is used.
#pragma once

#include "sm_common.cuh"

namespace smb {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;

enum GemmEpi : int {
  kEpiF32 = SM_EPI_F32,
  kEpiBF16 = SM_EPI_BF16,
  kEpiHiLo = SM_EPI_HILO,
  kEpiF32Norm = SM_EPI_F32_NORM,
  kEpiPoly = SM_EPI_POLY,
  kEpiPolyHiLo = SM_EPI_POLY_HILO,
};

struct GemmArgs {
  int m, n, k;          // per-matrix problem (multiples of 128 / BN / 64)
  int batch;
  int tiles_m, tiles_n;
  void* out0;           // [batch, m, n] FP32 or BF16 (hi plane for HiLo)
  void* out1;           // lo plane for HiLo
  const float* alpha;   // [batch] scale of the accumulator, or null (= 1)
  const __nv_bfloat16* aux;     // [batch, m, n] BF16 gram (hi plane) for the poly epilogues
  const __nv_bfloat16* aux_lo;  // lo plane of the gram for the hi/lo poly epilogue
  float pa, pb, pc;     // poly coefficients: out = pa*I + pb*aux + pc*acc
  float* partials;      // [batch, tiles_m*tiles_n*4] sum of squares (F32Norm)
};

template <int BN, bool COMP, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kOps = COMP ? 2 : 1;
  static constexpr int kStageBytes = kOps * (kABytes + kBBytes);
  static constexpr int kBarrierBytes = (2 * STAGES + 4) * 8 + 16;
  // +1024 for manual alignment of the dynamic shared memory base.
  static constexpr int kTotal = STAGES * kStageBytes + kBarrierBytes + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN;
};

template <int BN, bool COMP, bool B_MN, int STAGES, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm_bf16(const __grid_constant__ CUtensorMap tm_a_hi, const __grid_constant__ CUtensorMap tm_a_lo,
                const __grid_constant__ CUtensorMap tm_b_hi, const __grid_constant__ CUtensorMap tm_b_lo,
                const GemmArgs args) {
  using L = GemmSmem<BN, COMP, STAGES>;
  constexpr int kKSteps = kGemmBK / 16;
  constexpr uint32_t kIdesc = umma_idesc_bf16(kGemmBM, BN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
  // bars[0, S): full, [S, 2S): empty, [2S, 2S+2): tmem full, [2S+2, 2S+4): tmem empty
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
      mbar_init(bar_tempty(a), 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a_hi);
    tma_prefetch_desc(&tm_b_hi);
    if (COMP) {
      tma_prefetch_desc(&tm_a_lo);
      tma_prefetch_desc(&tm_b_lo);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_per_mat = args.tiles_m * args.tiles_n;
  const int total_tiles = tiles_per_mat * args.batch;
  const int kblocks = args.k / kGemmBK;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        const int b = tile / tiles_per_mat;
        const int rem = tile - b * tiles_per_mat;
        const int mi = rem / args.tiles_n;
        const int ni = rem - mi * args.tiles_n;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(bar_empty(stage), phase ^ 1u, abort_flag, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar_full(stage);
          mbar_arrive_expect_tx(fb, L::kStageBytes);
          const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t sb = sa + L::kOps * L::kABytes;
          const int kc = kb * kGemmBK;
          tma_load_3d(sa, &tm_a_hi, fb, kc, mi * kGemmBM, b);
          if (COMP) tma_load_3d(sa + L::kABytes, &tm_a_lo, fb, kc, mi * kGemmBM, b);
          if (!B_MN) {
            tma_load_3d(sb, &tm_b_hi, fb, kc, ni * BN, b);
            if (COMP) tma_load_3d(sb + L::kBBytes, &tm_b_lo, fb, kc, ni * BN, b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) {
              tma_load_3d(sb + j * 8192, &tm_b_hi, fb, ni * BN + 64 * j, kc, b);
              if (COMP) tma_load_3d(sb + L::kBBytes + j * 8192, &tm_b_lo, fb, ni * BN + 64 * j, kc, b);
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
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x, ++local) {
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
          const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t sb = sa + L::kOps * L::kABytes;
#pragma unroll
          for (int ks = 0; ks < kKSteps; ++ks) {
            const uint64_t a_hi = umma_desc_sw128(sa + ks * 32, 16, 1024);
            uint64_t b_hi;
            if (B_MN) {
              b_hi = umma_desc_sw128(sb + ks * 2048, 8192, 1024);
            } else {
              b_hi = umma_desc_sw128(sb + ks * 32, 16, 1024);
            }
            const uint32_t accumulate = (kb > 0 || ks > 0) ? 1u : 0u;
            if (COMP) {
              const uint64_t a_lo = umma_desc_sw128(sa + L::kABytes + ks * 32, 16, 1024);
              uint64_t b_lo;
              if (B_MN) {
                b_lo = umma_desc_sw128(sb + L::kBBytes + ks * 2048, 8192, 1024);
              } else {
                b_lo = umma_desc_sw128(sb + L::kBBytes + ks * 32, 16, 1024);
              }
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
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++local) {
      const int b = tile / tiles_per_mat;
      const int rem = tile - b * tiles_per_mat;
      const int mi = rem / args.tiles_n;
      const int ni = rem - mi * args.tiles_n;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      // Every lane polls; the vote keeps the warp converged (and uniform on
      // timeout) before the .sync.aligned TMEM loads below.
      const bool ready = mbar_wait(bar_tfull(acc), acc_phase, abort_flag, kStatusTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();

      const int row = mi * kGemmBM + quarter * 32 + lane;
      const size_t mat_off = static_cast<size_t>(b) * args.m * args.n;
      const size_t row_off = mat_off + static_cast<size_t>(row) * args.n;
      const float alpha = args.alpha != nullptr ? args.alpha[b] : 1.0f;
      float sumsq = 0.0f;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int j = 0; j < BN / 32; ++j) {
        uint32_t r[32];
        tmem_ld_32x32(t_row + j * 32, r);
        tmem_wait_ld();
        if (j == BN / 32 - 1) {
          // Accumulator fully read into registers: hand it back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_tempty(acc));
        }
        const int col0 = ni * BN + j * 32;
        if (EPI == kEpiF32 || EPI == kEpiF32Norm) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(args.out0) + row_off + col0);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4 v;
            v.x = alpha * __uint_as_float(r[4 * q + 0]);
            v.y = alpha * __uint_as_float(r[4 * q + 1]);
            v.z = alpha * __uint_as_float(r[4 * q + 2]);
            v.w = alpha * __uint_as_float(r[4 * q + 3]);
            if (EPI == kEpiF32Norm) sumsq += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            dst[q] = v;
          }
        } else if (EPI == kEpiBF16) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(args.out0) + row_off + col0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 v;
            v.x = pack_bf16x2(alpha * __uint_as_float(r[8 * q + 0]), alpha * __uint_as_float(r[8 * q + 1]));
            v.y = pack_bf16x2(alpha * __uint_as_float(r[8 * q + 2]), alpha * __uint_as_float(r[8 * q + 3]));
            v.z = pack_bf16x2(alpha * __uint_as_float(r[8 * q + 4]), alpha * __uint_as_float(r[8 * q + 5]));
            v.w = pack_bf16x2(alpha * __uint_as_float(r[8 * q + 6]), alpha * __uint_as_float(r[8 * q + 7]));
            dst[q] = v;
          }
        } else if (EPI == kEpiHiLo) {
          uint4* dhi = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(args.out0) + row_off + col0);
          uint4* dlo = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(args.out1) + row_off + col0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float h[8], l[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) split_hilo(alpha * __uint_as_float(r[8 * q + e]), h[e], l[e]);
            uint4 vh, vl;
            vh.x = pack_bf16x2(h[0], h[1]); vh.y = pack_bf16x2(h[2], h[3]);
            vh.z = pack_bf16x2(h[4], h[5]); vh.w = pack_bf16x2(h[6], h[7]);
            vl.x = pack_bf16x2(l[0], l[1]); vl.y = pack_bf16x2(l[2], l[3]);
            vl.z = pack_bf16x2(l[4], l[5]); vl.w = pack_bf16x2(l[6], l[7]);
            dhi[q] = vh;
            dlo[q] = vl;
          }
        } else if (EPI == kEpiPolyHiLo) {
          // P = pa*I + pb*G + pc*acc with G = hi + lo, emitted as hi/lo planes
          const uint4* srch = reinterpret_cast<const uint4*>(args.aux + row_off + col0);
          const uint4* srcl = reinterpret_cast<const uint4*>(args.aux_lo + row_off + col0);
          uint4* dhi = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(args.out0) + row_off + col0);
          uint4* dlo = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(args.out1) + row_off + col0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 gh = srch[q];
            const uint4 gl = srcl[q];
            const uint32_t wh[4] = {gh.x, gh.y, gh.z, gh.w};
            const uint32_t wl[4] = {gl.x, gl.y, gl.z, gl.w};
            float h[8], l[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int c0 = col0 + 8 * q + 2 * e;
              const float g0 = bf16_lo_to_f(wh[e]) + bf16_lo_to_f(wl[e]);
              const float g1 = bf16_hi_to_f(wh[e]) + bf16_hi_to_f(wl[e]);
              float v0 = args.pb * g0 + args.pc * __uint_as_float(r[8 * q + 2 * e]);
              float v1 = args.pb * g1 + args.pc * __uint_as_float(r[8 * q + 2 * e + 1]);
              if (c0 == row) v0 += args.pa;
              if (c0 + 1 == row) v1 += args.pa;
              split_hilo(v0, h[2 * e], l[2 * e]);
              split_hilo(v1, h[2 * e + 1], l[2 * e + 1]);
            }
            uint4 vh, vl;
            vh.x = pack_bf16x2(h[0], h[1]); vh.y = pack_bf16x2(h[2], h[3]);
            vh.z = pack_bf16x2(h[4], h[5]); vh.w = pack_bf16x2(h[6], h[7]);
            vl.x = pack_bf16x2(l[0], l[1]); vl.y = pack_bf16x2(l[2], l[3]);
            vl.z = pack_bf16x2(l[4], l[5]); vl.w = pack_bf16x2(l[6], l[7]);
            dhi[q] = vh;
            dlo[q] = vl;
          }
        } else if (EPI == kEpiPoly) {
          const uint4* src = reinterpret_cast<const uint4*>(args.aux + row_off + col0);
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(args.out0) + row_off + col0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 g = src[q];
            const uint32_t gw[4] = {g.x, g.y, g.z, g.w};
            float p[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int c0 = col0 + 8 * q + 2 * e;
              float v0 = args.pb * bf16_lo_to_f(gw[e]) + args.pc * __uint_as_float(r[8 * q + 2 * e]);
              float v1 = args.pb * bf16_hi_to_f(gw[e]) + args.pc * __uint_as_float(r[8 * q + 2 * e + 1]);
              if (c0 == row) v0 += args.pa;
              if (c0 + 1 == row) v1 += args.pa;
              p[2 * e] = v0;
              p[2 * e + 1] = v1;
            }
            uint4 v;
            v.x = pack_bf16x2(p[0], p[1]); v.y = pack_bf16x2(p[2], p[3]);
            v.z = pack_bf16x2(p[4], p[5]); v.w = pack_bf16x2(p[6], p[7]);
            dst[q] = v;
          }
        }
      }
      if (EPI == kEpiF32Norm) {
        sumsq = warp_sum(sumsq);
        if (lane == 0) {
          args.partials[static_cast<size_t>(b) * tiles_per_mat * 4 + rem * 4 + quarter] = sumsq;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

}  // namespace smb
