// The router GEMM, the step before the routed path: S = x . W_router^T, bf16 x bf16 -> f32, on 5th-gen
// tensor cores (tcgen05.mma kind::f16, TMEM accumulators, TMA-fed 128-byte-swizzled operand tiles).  It replaces
// the reference's `router` projection (scripts/gen_stage.py:1130: gemm(L + "router", normed, w_router,
// router_partial, EXPERTS, H), bound to extern:cublas_bf16_tn_f32, gen_stage.py:244-247): C[m, n] =
// A[m, k] . W[n, k]^T with f32 out, whose rows feed the router top-k.
//
// Tiles.  A unit is 128 token rows x BN experts (BN a multiple of 16 dividing E, at most 256: 224 for E = 896,
// four units across); a persistent grid walks the units, the four expert tiles of a token block side by side
// so the x rows are read from L2.  Stages of 64 K elements (128 bytes a row: one swizzle atom wide), a 4-stage
// mbarrier ring.  Roles (320 threads): warp 0 lane 0 issues the two TMA boxes a stage, warp 1 lane 0 the MMAs
// (M = 128, N = BN, K = 16, four a stage) into one of two TMEM accumulators, warps 2-9 drain an accumulator
// (two warps a TMEM sub-partition, half of the columns each) while the MMAs fill the other.  Rows past T are
// zero-filled by the loads and not stored.  Every wait is bounded and reports instead of hanging.
#pragma once
#include "common.cuh"

namespace k3 {

namespace rgemm {
constexpr int BM = 128;                 // token rows a unit (the MMA's M)
constexpr int BN_MAX = 256;             // expert columns a unit, at most (the MMA's N)
constexpr int BK = 64;                  // K elements a stage: 128 bytes of bf16
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;    // 16 KB
constexpr int B_BYTES = BN_MAX * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr u32 ACC_COLS = 256;           // one accumulator; two of them double-buffer the units
constexpr u32 TMEM_COLS = 512;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 32 * (2 + EPI_WARPS);
}  // namespace rgemm

struct RouterParams {
  float* S;      // [T, lds] f32
  int lds;
  int T;         // token rows
  int K;         // reduction length (H), a multiple of 64
  int bn;        // expert columns a unit
  int n_tiles;   // E / bn
  int m_tiles;   // ceil(T / 128)
  u32* err;
};

// kind::f16 instruction descriptor: f32 accumulator, bf16 A and B, both K-major, M x N
__device__ __forceinline__ u32 rg_idesc(int m, int n) {
  return 1u << 4 | 1u << 7 | 1u << 10 | (u32)(n >> 3) << 17 | (u32)(m >> 4) << 24;
}
__device__ __forceinline__ void rg_mma(u32 d_tmem, u64 adesc, u64 bdesc, u32 idesc, u32 accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 16 consecutive columns of this warp's 32 lanes
__device__ __forceinline__ void rg_ld16(u32 taddr, u32 (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__global__ void __launch_bounds__(rgemm::THREADS, 1)
    router_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                       RouterParams p) {
  using namespace rgemm;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  u64* bars = reinterpret_cast<u64*>(smem + STAGES * STAGE_BYTES);
  u64* full = bars;                     // [STAGES]
  u64* empty = bars + STAGES;           // [STAGES]
  u64* acc_full = bars + 2 * STAGES;    // [2]
  u64* acc_empty = bars + 2 * STAGES + 2;  // [2]
  u64* drain = bars + 2 * STAGES + 4;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 5);
  u32* tmem_slot = reinterpret_cast<u32*>(bars + 2 * STAGES + 6);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmW);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const u32 tmem_base = *tmem_slot;
  const int units = p.m_tiles * p.n_tiles;
  const int kstages = p.K / BK;
  const u32 tx = (u32)(A_BYTES + p.bn * BK * 2);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      u32 phase = 0;
      int armed[STAGES] = {0, 0, 0, 0};
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        const int tm = u / p.n_tiles, tn = u % p.n_tiles;
        for (int ks = 0; ks < kstages; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, 0xC00u)) break;
          uint8_t* st = smem + stage * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], tx);
          ++armed[stage];
          tma_load_2d(st, &tmX, &full[stage], ks * BK, tm * BM);
          tma_load_2d(st + A_BYTES, &tmW, &full[stage], ks * BK, tn * p.bn);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (armed[s]) mbar_wait(&full[s], (u32)(armed[s] - 1) & 1u, nullptr, p.err, 0xC10u, 100000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0;
      u32 phase = 0;
      u32 acc_phase[2] = {0u, 0u};
      int buf = 0;
      bool issued = false;
      const u32 idesc = rg_idesc(BM, p.bn);
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        if (!mbar_wait(&acc_empty[buf], acc_phase[buf] ^ 1u, abort_flag, p.err, 0xC20u)) break;
        tc_fence_after();
        const u32 d = tmem_base + (u32)buf * ACC_COLS;
        bool ok = true;
        for (int ks = 0; ks < kstages; ++ks) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, 0xC30u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const u32 st = smem_u32(smem + stage * STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            rg_mma(d, sdesc_k_sw128(st + kk * 32), sdesc_k_sw128(st + A_BYTES + kk * 32), idesc, (ks | kk) != 0);
          tc_commit(&empty[stage]);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[buf]);
        acc_phase[buf] ^= 1u;
        buf ^= 1;
      }
      if (issued) {
        tc_commit(drain);
        mbar_wait(drain, 0, nullptr, p.err, 0xC40u, 100000000ull);
      }
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..9): sub-partition, column half
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;
    const u32 lane_base = (u32)(sub * 32) << 16;
    const int cols = p.bn / 2;  // a multiple of 8
    u32 acc_phase[2] = {0u, 0u};
    int buf = 0;
    for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
      const int tm = u / p.n_tiles, tn = u % p.n_tiles;
      if (!mbar_wait(&acc_full[buf], acc_phase[buf], abort_flag, p.err, 0xC50u)) break;
      tc_fence_after();
      const int row = tm * BM + sub * 32 + lane;
      float* dst = p.S + (long long)row * p.lds + tn * p.bn + half * cols;
      const u32 c0 = (u32)buf * ACC_COLS + (u32)(half * cols);
      for (int c = 0; c < cols; c += 16) {
        u32 v[16];
        if (c + 16 <= cols) {
          rg_ld16(tmem_base + lane_base + c0 + c, v);
          tmem_wait_ld();
          if (row < p.T) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<uint4*>(dst + c + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          }
        } else {  // the last 8 columns of a half (bn / 2 an odd multiple of 8)
          u32 w[8];
          asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                       : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]),
                         "=r"(w[7])
                       : "r"(tmem_base + lane_base + c0 + c)
                       : "memory");
          tmem_wait_ld();
          if (row < p.T) {
            *reinterpret_cast<uint4*>(dst + c) = make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4*>(dst + c + 4) = make_uint4(w[4], w[5], w[6], w[7]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      acc_phase[buf] ^= 1u;
      buf ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace k3
