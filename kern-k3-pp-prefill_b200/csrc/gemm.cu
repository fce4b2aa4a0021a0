// Grouped (per-expert) block-scaled GEMMs of the routed MoE on 5th-gen tensor
// cores: FC1 = act x [gate; up]^T -> SwiGLU -> MXFP8 (E4M3 + UE8M0 per 32),
// and FC2 = act1 x down^T -> bf16.  They replace the two TRT-LLM-gen
// batched-GEMM cubins of the reference (kernels.toml:1-9; op arguments
// scripts/k3_moe_bmm.py:131-134, 167-169; contract docs/k3-kernel-abi.md:535-565).
//
// Operands.  A = the activations: 128 permuted token rows of MXFP8 (one
// routing tile).  B = 256 rows of expert weights, MXFP4 (E2M1 packed two a
// byte, UE8M0 per 32 along K), loaded by TMA with the 16U4_ALIGN16B type that
// unpacks them into the byte-per-element form kind::mxf8f6f4 reads.  One MMA
// is M=128 x N=256 x K=32: the full-rate shape (an M=128 MMA costs the same
// ~75 cycles for any N <= 128, so weight rows are put on the N side, 256 at a
// time, and the tokens of a tile on M).  FC1's 256 weight rows are the gate
// and the up rows of the same 128 features, so every accumulator row holds a
// token's gate and up values side by side.
//
// Tiles.  The routing tables (cta_batch / cta_limit / num_non_exiting, the
// reference's format) cut every expert's rows into 128-row token tiles; a work
// unit is (token tile c, 256-row weight block fb).  A persistent grid walks
// the units round-robin, so the weight blocks of one tile run side by side
// and its activation tile is read from L2.
//
// Roles (384 threads): warp 0 lane 0 issues the TMA boxes (activation tile,
// two weight tiles); warps 10-11 bring the three scale atoms of a stage with
// cp.async; warp 1 lane 0 copies the atoms into tensor memory (tcgen05.cp)
// and issues the MMAs; warps 2-9 are the epilogue.  An epilogue
// warp reads its sub-partition's 32 token rows and one half of the columns
// into registers, releases the accumulator, and only then computes and
// stores, so the next unit's MMAs overlap the math and the stores.  A 4-stage
// mbarrier ring carries K blocks of 128; every wait is bounded and reports
// instead of hanging.
#pragma once
#include "common.cuh"

namespace k3 {

namespace gemm {
constexpr int BM = 128;                  // token rows a tile (the routing tile): the MMA's M
constexpr int BN = 256;                  // weight rows a unit: the MMA's N
constexpr int BK = 128;                  // K elements a stage
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;         // activation tile (E4M3)
constexpr int W_TILE = 128 * BK;         // one 128-row weight tile, unpacked E2M1 (a byte an element)
constexpr int B_BYTES = 2 * W_TILE;
constexpr int SF_BYTES = 512;            // one 128-row x 4-group scale atom
constexpr int OPS_STAGE = A_BYTES + B_BYTES;                  // 48 KB, 1024-aligned
constexpr int SF_STAGE = 3 * SF_BYTES;                        // activation atom + two weight atoms
// bytes a stage's copies complete on its barrier: a 16U4_ALIGN16B load counts
// the packed (global) bytes, half the unpacked tile it writes
#ifndef K3MOE_LDGSTS
#define K3MOE_LDGSTS 1
#endif
// 1: a stage's three 512-byte scale atoms travel by cp.async (LDGSTS) from two loader warps, leaving the
// TMA unit three large boxes a stage (measured 1.5% faster a layer than six TMA operations); 0: all by TMA.
// Moving the 16 KB activation tile to cp.async as well starved the MMA (FC1 3.06 -> 3.94 ms).
constexpr int LDGSTS = K3MOE_LDGSTS;
constexpr u32 STAGE_TX = LDGSTS ? A_BYTES + B_BYTES / 2 : A_BYTES + B_BYTES / 2 + SF_STAGE;
constexpr int SMEM_BYTES = STAGES * (OPS_STAGE + SF_STAGE) + 1024 /*align*/ + 256 /*barriers*/;
constexpr u32 TMEM_COLS = 512;
constexpr int SF_TMEM_COL = BN;          // scale columns after the accumulator
constexpr int EPI_WARPS = 8;
constexpr int LOADER_WARPS = LDGSTS ? 2 : 0;
constexpr int LOADER_THREADS = 32 * LOADER_WARPS;
constexpr int THREADS = 32 * (2 + EPI_WARPS + LOADER_WARPS);
}  // namespace gemm

enum { MODE_FC1 = 0, MODE_FC2 = 1 };

struct GemmParams {
  const uint8_t* sfw;       // weight scales, tiled over all weight rows (atom t of data tile t)
  const uint8_t* sfa;       // activation scales, tiled over permuted rows
  const int* cta_batch;     // [ctas] local expert of token tile c
  const int* cta_limit;     // [ctas] end of tile c's real rows
  const int* meta;          // meta[0] = num_non_exiting
  uint8_t* out_q;           // FC1: [cap_rows, out_cols] E4M3, tile-major
  uint8_t* out_sf;          // FC1: tiled scales over permuted rows
  bf16* out_bf16;           // FC2: [cap_rows, out_cols] row-major
  const int* out_rows;      // FC2: permuted row r is stored at row out_rows[r] (null: at r)
  u32* err;
  int K;                    // reduction length (elements), multiple of 128
  int rows_per_expert;      // weight rows an expert: FC1 2I, FC2 H
  int n_experts;            // experts the weight tensor holds
  int nfb;                  // weight blocks a token tile: FC1 I/128, FC2 H/256
  int out_cols;             // FC1 I, FC2 H
  int cap_rows;             // permuted-row capacity of the activations and the outputs
  int max_ctas;             // capacity of the CTA tables
  unsigned long long* trace;  // optional per-role cycle counters (16 a mode), or null
  int act;                  // FC1 gate: 0 SwiGLU silu(g)*u, 1 K3's SiTU a tanh(g/a) sigmoid(g) * b tanh(u/b)
  int fb0;                  // FC2: the first 256-column block computed (a column slice [256 fb0, 256 (fb0 + nfb)))
  const float* alpha;       // SiTU: per-expert a and b (f32 [n_experts]), or null for K3's a = 4, b = 25
  const float* beta;
  const unsigned long long* out_ptrs;  // FC2: permuted row r is stored at the address out_ptrs[r] (a row of H
                                       // columns, possibly another GPU's memory), or null (out_rows / out_bf16)
};

// FC1's gated activation of (gate g, up u); SiTU with a = 4, b = 25 is K3's gate.  ra, rb are 1/a, 1/b
// (exact for a = 4; the nearest float to 1/25 for b = 25, the same value as the literal 0.04f).
__device__ __forceinline__ float gated_act(float g, float u, int act, float a = 4.0f, float ra = 0.25f,
                                           float b = 25.0f, float rb = 0.04f) {
  const float sg = __fdividef(1.0f, 1.0f + __expf(-g));
  if (act == 0) return g * sg * u;
  return a * tanhf(ra * g) * sg * (b * tanhf(rb * u));
}

struct Unit {
  int valid, e, row0, n, fb;
};

__device__ __forceinline__ Unit decode_unit(const GemmParams& p, int u) {
  Unit w;
  const int c = u / p.nfb;
  w.fb = u % p.nfb;
  w.e = p.cta_batch[c];
  w.row0 = c * gemm::BM;
  w.n = p.cta_limit[c] - w.row0;
  w.valid = c < p.max_ctas && w.e >= 0 && w.e < p.n_experts && w.n > 0 && w.n <= gemm::BM &&
            w.row0 + gemm::BM <= p.cap_rows;
  return w;
}

// first weight row of the h-th 128-row half of unit w's weight block:
// FC1 pairs the gate rows of features [128 fb, 128 fb + 128) with their up rows
template <int MODE>
__device__ __forceinline__ int weight_row(const GemmParams& p, const Unit& w, int h) {
  if (MODE == MODE_FC1) return w.e * p.rows_per_expert + h * (p.rows_per_expert / 2) + w.fb * 128;
  return w.e * p.rows_per_expert + (p.fb0 + w.fb) * gemm::BN + h * 128;
}

// The kernel body: tmW / tmA point at the weight and activation tensor maps (kernel parameters for the C-ABI
// launch, a global-memory descriptor buffer for the module entries of module_gemm.cu).
template <int MODE>
__device__ __forceinline__ void grouped_gemm_body(const CUtensorMap* tmW, const CUtensorMap* tmA, const GemmParams& p) {
  using namespace gemm;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ops = smem;                                  // [STAGES][A | W0 | W1]
  uint8_t* sfs = smem + STAGES * OPS_STAGE;             // [STAGES][SFA | SFW0 | SFW1]
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
      mbar_init(&full[s], 1 + LOADER_THREADS);  // the TMA producer's arrive + one per loader thread
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, EPI_WARPS);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(tmW);
    prefetch_tmap(tmA);
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
      const long long t_role = clock64();
      long long t_wait = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        const Unit w = decode_unit(p, u);
        if (!w.valid) {
          report_error(p.err, ERR_BAD_TABLE, 0x100u + MODE);
          continue;
        }
        int wrow[2];
        wrow[0] = weight_row<MODE>(p, w, 0);
        wrow[1] = weight_row<MODE>(p, w, 1);
        for (int ks = 0; ks < kstages; ++ks) {
          const long long t0 = clock64();
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, 0x200u + MODE)) break;
          t_wait += clock64() - t0;
          uint8_t* st = ops + stage * OPS_STAGE;
          uint8_t* sf = sfs + stage * SF_STAGE;
          mbar_arrive_expect_tx(&full[stage], STAGE_TX);
          ++armed[stage];
          // tile-major operands: tile t = row_block * kstages + ks is rows [128 t, 128 t + 128) of the
          // maps (one contiguous chunk), and its scales are the 512-byte atom t
          const int ta = (w.row0 / BM) * kstages + ks;
          tma_load_2d(st, tmA, &full[stage], 0, ta * BM);
          if (!LDGSTS) bulk_load(sf, p.sfa + (long long)ta * SF_BYTES, SF_BYTES, &full[stage]);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int t = (wrow[h] / 128) * kstages + ks;
            tma_load_2d(st + A_BYTES + h * W_TILE, tmW, &full[stage], 0, t * 128);
            if (!LDGSTS) bulk_load(sf + (1 + h) * SF_BYTES, p.sfw + (long long)t * SF_BYTES, SF_BYTES, &full[stage]);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // every armed stage's last fill has landed before the block may exit
      for (int s = 0; s < STAGES; ++s)
        if (armed[s]) mbar_wait(&full[s], (u32)(armed[s] - 1) & 1u, nullptr, p.err, 0x300u + MODE, 100000000ull);
      if (p.trace) {
        atomicAdd(p.trace + MODE * 16 + 0, (unsigned long long)(clock64() - t_role));
        atomicAdd(p.trace + MODE * 16 + 1, (unsigned long long)t_wait);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      int stage = 0;
      u32 phase = 0, acc_phase = 0;
      bool issued = false;
      const long long t_role = clock64();
      long long t_wfull = 0, t_wacc = 0, n_units = 0;
      for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
        const Unit w = decode_unit(p, u);
        if (!w.valid) continue;
        long long t0 = clock64();
        if (!mbar_wait(acc_empty, acc_phase ^ 1u, abort_flag, p.err, 0x400u + MODE)) break;
        t_wacc += clock64() - t0;
        ++n_units;
        tc_fence_after();
        bool ok = true;
        for (int ks = 0; ks < kstages; ++ks) {
          t0 = clock64();
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, 0x500u + MODE)) {
            ok = false;
            break;
          }
          t_wfull += clock64() - t0;
          // the loader warps' cp.async writes (generic proxy) before the tensor core's reads (async proxy)
          if (LDGSTS) fence_proxy_async_shared();
          tc_fence_after();
          const u32 st = smem_u32(ops + stage * OPS_STAGE);
          const u32 sf = smem_u32(sfs + stage * SF_STAGE);
          const u32 sf_col = tmem_base + SF_TMEM_COL + stage * 16;
          // scale columns: [0,4) the activation atom, [4,8) and [8,12) the two weight atoms
#pragma unroll
          for (int q = 0; q < 3; ++q) tmem_cp_32x128b_x4(sf_col + 4 * q, sdesc_sf(sf + q * SF_BYTES));
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const u32 idesc = idesc_mxf8f6f4(BN, (u32)kk, (u32)kk, FMT_E4M3, FMT_E2M1);
            const u64 adesc = sdesc_k_sw128(st + kk * 32);
            const u64 bdesc = sdesc_k_sw128(st + A_BYTES + kk * 32);
            mma_mxf8f6f4(tmem_base, adesc, bdesc, idesc, sf_col | ((u32)kk << 30), (sf_col + 4) | ((u32)kk << 30),
                         (ks | kk) != 0);
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
      if (p.trace) {
        atomicAdd(p.trace + MODE * 16 + 2, (unsigned long long)(clock64() - t_role));
        atomicAdd(p.trace + MODE * 16 + 3, (unsigned long long)t_wfull);
        atomicAdd(p.trace + MODE * 16 + 4, (unsigned long long)t_wacc);
        atomicAdd(p.trace + MODE * 16 + 7, (unsigned long long)n_units);
      }
    }
  } else if (warp >= 2 + EPI_WARPS) {
    // ------------------------------------------------ cp.async loaders (warps 10, 11): a stage's scale atoms
    // (the activation atom, then the two weight atoms), 16 bytes a thread-copy
    const int lt = threadIdx.x - 32 * (2 + EPI_WARPS);
    int stage = 0;
    u32 phase = 0;
    bool stop = false;
    for (int u = blockIdx.x; u < units && !stop && !*abort_flag; u += gridDim.x) {
      const Unit w = decode_unit(p, u);
      if (!w.valid) continue;
      const int wt0 = weight_row<MODE>(p, w, 0) / 128, wt1 = weight_row<MODE>(p, w, 1) / 128;
      for (int ks = 0; ks < kstages; ++ks) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err, 0x800u + MODE)) {
          stop = true;
          break;
        }
        const u32 sf = smem_u32(sfs + stage * SF_STAGE);
        const int ta = (w.row0 / BM) * kstages + ks;
        for (int c = lt; c < SF_STAGE / 16; c += LOADER_THREADS) {
          const int q = c >> 5;  // atom: 0 activation, 1 and 2 the weight tiles
          const long long t = q == 0 ? ta : (long long)(q == 1 ? wt0 : wt1) * kstages + ks;
          const uint8_t* a = (q == 0 ? p.sfa : p.sfw) + t * SF_BYTES;
          cp_async16(sf + c * 16, a + (c & 31) * 16);
        }
        cp_async_mbar_arrive_noinc(&full[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    cp_async_wait_all();
  } else {
    // ------------------------------------------------ epilogue (warps 2..9)
    // warp -> (sub-partition, column half): its thread i owns token row 32*sub + i of the tile
    const int sub = warp & 3;
    const int half = (warp - 2) >> 2;
    const u32 lane_base = (u32)(sub * 32) << 16;
    const int row = sub * 32 + lane;
    u32 acc_phase = 0;
    const long long t_role = clock64();
    long long t_wait = 0;
    for (int u = blockIdx.x; u < units && !*abort_flag; u += gridDim.x) {
      const Unit w = decode_unit(p, u);
      if (!w.valid) continue;
      const long long t0 = clock64();
      // the warp leaves together (its tensor-memory loads and shuffles below take every lane)
      if (!__all_sync(0xffffffffu, mbar_wait(acc_full, acc_phase, abort_flag, p.err, 0x700u + MODE))) break;
      t_wait += clock64() - t0;
      tc_fence_after();
      u32 v[4][32];
      if (MODE == MODE_FC1) {
        // gate of features [64 half, 64 half + 64) in columns 64 half.., their up 128 columns later
        const u32 c0 = (u32)(64 * half);
        tmem_ld32(tmem_base + lane_base + c0, v[0]);
        tmem_ld32(tmem_base + lane_base + c0 + 32, v[1]);
        tmem_ld32(tmem_base + lane_base + c0 + 128, v[2]);
        tmem_ld32(tmem_base + lane_base + c0 + 160, v[3]);
      } else {
        const u32 c0 = (u32)(128 * half);
#pragma unroll
        for (int q = 0; q < 4; ++q) tmem_ld32(tmem_base + lane_base + c0 + 32 * q, v[q]);
      }
      tmem_wait_ld();
      // the accumulator is in registers: release it to the next unit's MMAs
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      acc_phase ^= 1u;
      if (MODE == MODE_FC2) {
        // The thread's 128 columns of its token row, as bf16.  Stored one row a lane, a warp's store would
        // touch 32 lines (32 L1 wavefronts for 1 KB); instead each group of 8 lanes transposes its 8 rows'
        // 16-byte chunks (lane i gets chunk i of each row) and stores whole 128-byte lines: 4 lines a store.
        bf16* dst = nullptr;
        if (row < w.n) {
          const long long r = w.row0 + row;
          if (p.out_ptrs != nullptr) {
            dst = reinterpret_cast<bf16*>(p.out_ptrs[r]) + (p.fb0 + w.fb) * BN + 128 * half;
          } else {
            const long long ro = p.out_rows ? (long long)p.out_rows[r] : r;
            dst = p.out_bf16 + ro * p.out_cols + w.fb * BN + 128 * half;
          }
        }
        const unsigned long long mine = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
        for (int g = 0; g < 2; ++g) {  // 64 columns at a time: 8 chunks of 16 bytes
          uint4 a[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const u32* src = v[2 * g + c / 4] + 8 * (c % 4);
            a[c] = make_uint4(f2_to_bf16x2(__uint_as_float(src[0]), __uint_as_float(src[1])),
                              f2_to_bf16x2(__uint_as_float(src[2]), __uint_as_float(src[3])),
                              f2_to_bf16x2(__uint_as_float(src[4]), __uint_as_float(src[5])),
                              f2_to_bf16x2(__uint_as_float(src[6]), __uint_as_float(src[7])));
          }
          // 8 x 8 transpose within each 8-lane group: swap off-diagonal blocks of 4, then 2, then 1
#pragma unroll
          for (int d = 4; d >= 1; d >>= 1) {
            const bool upper = (lane & d) != 0;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              if (c & d) continue;
              const uint4 send = upper ? a[c] : a[c | d];
              uint4 got;
              got.x = __shfl_xor_sync(0xffffffffu, send.x, d);
              got.y = __shfl_xor_sync(0xffffffffu, send.y, d);
              got.z = __shfl_xor_sync(0xffffffffu, send.z, d);
              got.w = __shfl_xor_sync(0xffffffffu, send.w, d);
              if (upper) a[c] = got;
              else a[c | d] = got;
            }
          }
#pragma unroll
          for (int m = 0; m < 8; ++m) {  // row (group base + m), chunk (lane % 8)
            const unsigned long long rp = __shfl_sync(0xffffffffu, mine, (lane & ~7) | m);
            if (rp != 0ull) *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(rp) + 64 * g + 8 * (lane & 7)) = a[m];
          }
        }
      } else if (row < w.n) {
        const long long r = w.row0 + row;
        {
          const int kg4 = p.out_cols / 128;
          // SiTU's a, b: per expert from the caller's buffers (the module entry), else K3's 4 and 25
          float ga = 4.0f, gra = 0.25f, gb = 25.0f, grb = 0.04f;
          if (p.alpha != nullptr) {
            ga = p.alpha[w.e];
            gb = p.beta[w.e];
            gra = __frcp_rn(ga);
            grb = __frcp_rn(gb);
          }
          u32 sfw = 0;
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            float hv[32];
            float amax = 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float gf = __uint_as_float(v[g][j]);
              const float uf = __uint_as_float(v[2 + g][j]);
              hv[j] = gated_act(gf, uf, p.act, ga, gra, gb, grb);
              amax = fmaxf(amax, fabsf(hv[j]));
            }
            const int e = mx8_exponent_ocp(amax);
            const float s = pow2_normal(-e);
            u32 q[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              q[j] = (u32)e4m3x2_sat(hv[4 * j] * s, hv[4 * j + 1] * s) |
                     ((u32)e4m3x2_sat(hv[4 * j + 2] * s, hv[4 * j + 3] * s) << 16);
            const int f = w.fb * 128 + 64 * half + 32 * g;
            st_global_v8(p.out_q + op8_offset(r, f, p.out_cols), q);  // the group's 32 bytes, contiguous
            sfw |= (u32)(e + 127) << (8 * g);
          }
          // the two groups' scales are adjacent bytes of one atom row (kb even)
          const int kb = (w.fb * 128 + 64 * half) / 32;
          *reinterpret_cast<unsigned short*>(p.out_sf + sf_tiled_offset(r, kb, kg4)) = (unsigned short)sfw;
        }
      }
    }
    // rows stored at caller addresses may sit in a peer GPU's memory: order them at system scope before the
    // kernel's end (a later kernel on this stream signals the peer)
    if (MODE == MODE_FC2 && p.out_ptrs != nullptr) __threadfence_system();
    if (p.trace && lane == 0 && warp == 2) {
      atomicAdd(p.trace + MODE * 16 + 5, (unsigned long long)(clock64() - t_role));
      atomicAdd(p.trace + MODE * 16 + 6, (unsigned long long)t_wait);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int MODE>
__global__ void __launch_bounds__(gemm::THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA,
                        GemmParams p) {
  grouped_gemm_body<MODE>(&tmW, &tmA, p);
}

}  // namespace k3
