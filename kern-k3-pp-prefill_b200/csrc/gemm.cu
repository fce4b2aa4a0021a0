// Grouped (per-expert) block-scaled GEMMs of the routed MoE on 5th-gen tensor
// cores: FC1 = [gate; up] x act -> SwiGLU -> MXFP8 (E4M3 + UE8M0 per 32), and
// FC2 = down x act1 -> bf16.  They replace the two TRT-LLM-gen batched-GEMM
// cubins of the reference (kernels.toml:1-9; op arguments
// scripts/k3_moe_bmm.py:131-134, 167-169; contract docs/k3-kernel-abi.md:535-565).
//
// Operands.  A = expert weights, MXFP4 (E2M1 packed two a byte, UE8M0 per 32
// along K), loaded by TMA with the 16U4_ALIGN16B type that unpacks them into
// the byte-per-element shared-memory form kind::mxf8f6f4 reads.  B = the
// activations, MXFP8 rows in permuted (expert-grouped) order.  The weight is
// the MMA's M side (128 rows an accumulator) and the tokens its N side, so a
// tile of n routed rows issues N = roundup(n, 8) columns, not a padded 128.
//
// Tiles.  The routing tables (cta_batch / cta_limit / num_non_exiting, the
// reference's format) cut every expert's rows into 128-row token tiles; a
// work unit is (token tile c, feature block fb).  FC1's unit holds the gate
// and the up accumulator of 128 features (two M=128 accumulators); FC2's holds
// 256 output features.  A persistent grid walks the units round-robin.
//
// Roles (192 threads): warp 0 lane 0 issues TMA (operands) and bulk copies
// (scale atoms); warp 1 lane 0 copies the scale atoms into tensor memory
// (tcgen05.cp) and issues the MMAs; warps 2-5 are the epilogue, each reading
// its 32-lane sub-partition of the accumulators.  A 4-stage mbarrier ring
// carries K blocks of 128; every wait is bounded and reports instead of
// hanging.
#include "common.cuh"

namespace k3 {

namespace gemm {
constexpr int BM = 128;                  // weight rows an accumulator
constexpr int BN = 128;                  // token rows a tile (the routing tile)
constexpr int BK = 128;                  // K elements a stage
constexpr int NACC = 2;                  // accumulators a tile
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;         // unpacked E2M1: a byte an element in shared memory
constexpr int B_BYTES = BN * BK;
constexpr int SF_BYTES = 512;            // one 128-row x 4-group scale atom
constexpr int OPS_STAGE = NACC * A_BYTES + B_BYTES;          // 48 KB, 1024-aligned
constexpr int SF_STAGE = (NACC + 1) * SF_BYTES;               // 1.5 KB
// bytes a stage's copies complete on its barrier: a 16U4_ALIGN16B load counts
// the packed (global) bytes, half the unpacked tile it writes
constexpr u32 STAGE_TX = NACC * A_BYTES / 2 + B_BYTES + SF_STAGE;
constexpr int SMEM_BYTES = STAGES * (OPS_STAGE + SF_STAGE) + 1024 /*align*/ + 256 /*barriers*/;
constexpr u32 TMEM_COLS = 512;
constexpr int SF_TMEM_COL = NACC * BN;   // scale columns after the accumulators
constexpr int THREADS = 192;
}  // namespace gemm

enum { MODE_FC1 = 0, MODE_FC2 = 1 };

struct GemmParams {
  const uint8_t* sfa;       // weight scales, tiled over all weight rows, K/128 atoms a row block
  const uint8_t* sfb;       // activation scales, tiled over permuted rows
  const int* cta_batch;     // [ctas] local expert of token tile c
  const int* cta_limit;     // [ctas] end of tile c's real rows
  const int* meta;          // meta[0] = num_non_exiting
  uint8_t* out_q;           // FC1: [cap_rows, out_cols] E4M3
  uint8_t* out_sf;          // FC1: tiled scales over permuted rows
  bf16* out_bf16;           // FC2: [cap_rows, out_cols]
  u32* err;
  int K;                    // reduction length (elements), multiple of 128
  int rows_per_expert;      // weight rows an expert: FC1 2I, FC2 H
  int n_experts;            // experts the weight tensor holds
  int nfb;                  // feature blocks a token tile
  int out_cols;             // FC1 I, FC2 H
  int cap_rows;             // permuted-row capacity of B and the outputs
  int max_ctas;             // capacity of the CTA tables
};

struct Unit {
  int valid, e, row0, n, fb;
};

__device__ __forceinline__ Unit decode_unit(const GemmParams& p, int u) {
  Unit w;
  const int c = u / p.nfb;
  w.fb = u % p.nfb;
  w.e = p.cta_batch[c];
  w.row0 = c * gemm::BN;
  w.n = p.cta_limit[c] - w.row0;
  w.valid = c < p.max_ctas && w.e >= 0 && w.e < p.n_experts && w.n > 0 && w.n <= gemm::BN &&
            w.row0 + gemm::BN <= p.cap_rows;
  return w;
}

// weight row of accumulator a of unit w
template <int MODE>
__device__ __forceinline__ int weight_row(const GemmParams& p, const Unit& w, int a) {
  if (MODE == MODE_FC1) return w.e * p.rows_per_expert + a * (p.rows_per_expert / 2) + w.fb * gemm::BM;
  return w.e * p.rows_per_expert + (w.fb * gemm::NACC + a) * gemm::BM;
}

template <int MODE>
__global__ void __launch_bounds__(gemm::THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        GemmParams p) {
  using namespace gemm;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ops = smem;                                  // [STAGES][A0 | A1 | B]
  uint8_t* sfs = smem + STAGES * OPS_STAGE;             // [STAGES][SFA0 | SFA1 | SFB]
  u64* bars = reinterpret_cast<u64*>(sfs + STAGES * SF_STAGE);
  u64* full = bars;                                     // [STAGES]
  u64* empty = bars + STAGES;                           // [STAGES]
  u64* acc_full = bars + 2 * STAGES;
  u64* acc_empty = bars + 2 * STAGES + 1;
  u64* drain = bars + 2 * STAGES + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 3);
  u32* tmem_slot = reinterpret_cast<u32*>(bars + 2 * STAGES + 4);

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
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const u32 tmem_base = *tmem_slot;

  const int nne = min(p.meta[0], p.max_ctas);
  const int units = nne * p.nfb;
  const int kstages = p.K / BK;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      u32 phase = 0;
      int armed[STAGES] = {0, 0, 0, 0};
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        const Unit w = decode_unit(p, u);
        if (!w.valid) {
          report_error(p.err, ERR_BAD_TABLE, 0x100u + MODE);
          continue;
        }
        int arow[NACC];
#pragma unroll
        for (int a = 0; a < NACC; ++a) arow[a] = weight_row<MODE>(p, w, a);
        for (int ks = 0; ks < kstages; ++ks) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, 0x200u + MODE)) break;
          uint8_t* st = ops + stage * OPS_STAGE;
          uint8_t* sf = sfs + stage * SF_STAGE;
          mbar_arrive_expect_tx(&full[stage], STAGE_TX);
          ++armed[stage];
#pragma unroll
          for (int a = 0; a < NACC; ++a) {
            tma_load_2d(st + a * A_BYTES, &tmA, &full[stage], ks * BK, arow[a]);
            bulk_load(sf + a * SF_BYTES, p.sfa + ((long long)(arow[a] / BM) * kstages + ks) * SF_BYTES, SF_BYTES,
                      &full[stage]);
          }
          tma_load_2d(st + NACC * A_BYTES, &tmB, &full[stage], ks * BK, w.row0);
          bulk_load(sf + NACC * SF_BYTES, p.sfb + ((long long)(w.row0 / BN) * kstages + ks) * SF_BYTES, SF_BYTES,
                    &full[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // every armed stage's last fill has landed before the block may exit
      for (int s = 0; s < STAGES; ++s)
        if (armed[s]) mbar_wait(&full[s], (u32)(armed[s] - 1) & 1u, nullptr, p.err, 0x300u + MODE, 100000000ull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0;
      u32 phase = 0, acc_phase = 0;
      bool issued = false;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        const Unit w = decode_unit(p, u);
        if (!w.valid) continue;
        const int N = (w.n + 7) & ~7;
        if (!mbar_wait(acc_empty, acc_phase ^ 1u, abort_flag, p.err, 0x400u + MODE)) break;
        tc_fence_after();
        bool ok = true;
        for (int ks = 0; ks < kstages; ++ks) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, 0x500u + MODE)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const u32 st = smem_u32(ops + stage * OPS_STAGE);
          const u32 sf = smem_u32(sfs + stage * SF_STAGE);
          const u32 sf_col = tmem_base + SF_TMEM_COL + stage * 16;
#pragma unroll
          for (int a = 0; a <= NACC; ++a) tmem_cp_32x128b_x4(sf_col + 4 * a, sdesc_sf(sf + a * SF_BYTES));
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const u32 idesc = idesc_mxf8f6f4(N, (u32)kk, (u32)kk);
            const u64 bdesc = sdesc_k_sw128(st + NACC * A_BYTES + kk * 32);
#pragma unroll
            for (int a = 0; a < NACC; ++a) {
              const u64 adesc = sdesc_k_sw128(st + a * A_BYTES + kk * 32);
              mma_mxf8f6f4(tmem_base + a * BN, adesc, bdesc, idesc, (sf_col + 4 * a) | ((u32)kk << 30),
                           (sf_col + 4 * NACC) | ((u32)kk << 30), (ks | kk) != 0);
            }
          }
          tc_commit(&empty[stage]);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(acc_full);
        acc_phase ^= 1u;
      }
      if (issued) {
        // all issued tensor-core work has finished before the block may exit
        tc_commit(drain);
        mbar_wait(drain, 0, nullptr, p.err, 0x600u + MODE, 100000000ull);
      }
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2..5)
    const int sub = warp & 3;                 // tensor-memory sub-partition of this warp
    const u32 lane_base = (u32)(sub * 32) << 16;
    u32 acc_phase = 0;
    for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
      const Unit w = decode_unit(p, u);
      if (!w.valid) continue;
      if (!mbar_wait(acc_full, acc_phase, abort_flag, p.err, 0x700u + MODE)) break;
      tc_fence_after();
      if (MODE == MODE_FC1) {
        const int f = w.fb * BM + sub * 32 + lane;  // this lane's feature
        const int kb = (w.fb * BM + sub * 32) / 32;
        const int kg4 = p.out_cols / 128;
        for (int j0 = 0; j0 < w.n; j0 += 32) {
          u32 g[32], v[32];
          tmem_ld32(tmem_base + lane_base + (u32)j0, g);
          tmem_ld32(tmem_base + lane_base + (u32)(BN + j0), v);
          tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            if (j0 + jj < w.n) {
              const float gf = __uint_as_float(g[jj]);
              const float uf = __uint_as_float(v[jj]);
              const float h = gf / (1.0f + __expf(-gf)) * uf;
              const u32 am = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(h)));
              const int e = mx8_exponent(__uint_as_float(am));
              const float s = exp2f((float)-e);
              const long long r = w.row0 + j0 + jj;
              p.out_q[r * p.out_cols + f] = (uint8_t)(e4m3x2_sat(h * s, 0.f) & 0xffu);
              if (lane == 0) p.out_sf[sf_tiled_offset(r, kb, kg4)] = (uint8_t)(e + 127);
            }
          }
        }
      } else {
        for (int a = 0; a < NACC; ++a) {
          const int f = (w.fb * NACC + a) * BM + sub * 32 + lane;
          for (int j0 = 0; j0 < w.n; j0 += 32) {
            u32 v[32];
            tmem_ld32(tmem_base + lane_base + (u32)(a * BN + j0), v);
            tmem_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              if (j0 + jj < w.n) {
                const long long r = w.row0 + j0 + jj;
                p.out_bf16[r * p.out_cols + f] = __float2bfloat16_rn(__uint_as_float(v[jj]));
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      acc_phase ^= 1u;
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
