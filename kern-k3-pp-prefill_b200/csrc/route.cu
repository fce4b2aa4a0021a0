// Bandwidth kernels of the routed-MoE path: router top-k, routing tables,
// MXFP8 activation quantisation (plain and fused with the permutation), the
// routing-weighted combine, and the MXFP4 weight quantiser.
//
// Reference semantics (file:line inside the reference project):
//   top-k        source/k3_moe_route.cu:117-221, 372-385; source/k3_prefill_glue.cu:504-557
//   tables       source/k3_moe_prefill.cu:97-204 (count / tables / scatter), source/k3_moe_route.cu:457-519
//   quant        source/k3_moe_prefill.cu:66-95; source/k3_mxfp8.cu:20-54
//   combine      source/k3_moe_prefill.cu:206-234
// The MXFP4 weight quantiser has no reference counterpart (the reference
// consumes pre-quantised checkpoints); it follows the OCP MX rule.
#include "common.cuh"

namespace k3 {

// ============================================================ router top-k
// One warp a row.  Lane l holds experts e = j*32 + l: key = ord(sig + bias), sig = 1/(1+expf(-s)) (an
// IEEE reciprocal).  The K largest keys, ties to the smaller expert, lane r ending with the r-th pick;
// weights sig / (butterfly sum over the K picks + 1e-20) * rs.  K must be a power of two <= 16.
//
// Selection: tau = the K-th largest of the 32 lane maxima (a bitonic sort across the warp) bounds the
// K-th largest key from below (K lanes hold a key >= tau), so only keys >= tau are candidates; they are
// compacted into shared memory and each ranked by counting the candidates ahead of it.  With more than
// TOPK_CAND candidates (ties on a large scale), K rounds of warp max / min over the registers instead.
#define TOPK_MAX_EPL 32  // experts per lane: E <= 1024
#define TOPK_CAND 64     // candidate slots a warp (shared memory)

__device__ __forceinline__ float router_sigmoid(float s) { return __frcp_rn(1.0f + expf(-s)); }

// Returns this lane's pick (lanes < K).
template <int EPL>
__device__ __forceinline__ int topk_warp(const float* __restrict__ row, const float* __restrict__ bias, int E, int K,
                                         float rsv, int lane, u32* __restrict__ ck, int* __restrict__ ce,
                                         int* __restrict__ idx_out, float* __restrict__ wts_out) {
  u32 o[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int e = j * 32 + lane;
    o[j] = e < E ? ord_f32(router_sigmoid(row[e]) + bias[e]) : 0u;  // 0: below every real key
  }
  // tau: bitonic sort of the lane maxima, descending; lane K-1 holds the K-th largest
  u32 v = o[0];
#pragma unroll
  for (int j = 1; j < EPL; ++j) v = max(v, o[j]);
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const u32 p = __shfl_xor_sync(0xffffffffu, v, j);
      const bool up = ((lane & k) == 0) == ((lane & j) == 0);  // keep the larger in the lower lane of a pair
      v = up ? max(v, p) : min(v, p);
    }
  const u32 tau = __shfl_sync(0xffffffffu, v, K - 1);
  int c = 0;
#pragma unroll
  for (int j = 0; j < EPL; ++j) c += o[j] >= tau;
  int incl = c;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  const int n = __shfl_sync(0xffffffffu, incl, 31);
  int pick = 0;
  if (n <= TOPK_CAND) {
    int at = incl - c;
#pragma unroll
    for (int j = 0; j < EPL; ++j)
      if (o[j] >= tau) {
        ck[at] = o[j];
        ce[at] = j * 32 + lane;
        ++at;
      }
    __syncwarp();
    // candidate i's rank: the candidates with a larger key, or the same key and a smaller expert
    int rk[TOPK_CAND / 32], ex[TOPK_CAND / 32];
#pragma unroll
    for (int h = 0; h < TOPK_CAND / 32; ++h) {
      const int i = lane + 32 * h;
      rk[h] = K;
      if (i < n) {
        const u32 ki = ck[i];
        const int ei = ce[i];
        int r = 0;
        for (int q = 0; q < n; ++q) {
          const u32 kq = ck[q];
          r += (kq > ki) | ((kq == ki) & (ce[q] < ei));
        }
        rk[h] = r;
        ex[h] = ei;
      }
    }
    __syncwarp();
#pragma unroll
    for (int h = 0; h < TOPK_CAND / 32; ++h)
      if (rk[h] < K) ce[rk[h]] = ex[h];
    __syncwarp();
    if (lane < K) pick = ce[lane];
    __syncwarp();
  } else {
    for (int r = 0; r < K; ++r) {
      u32 m = o[0];
#pragma unroll
      for (int j = 1; j < EPL; ++j) m = max(m, o[j]);
      m = __reduce_max_sync(0xffffffffu, m);
      u32 mine = 0xffffffffu;
#pragma unroll
      for (int j = EPL - 1; j >= 0; --j)
        if (o[j] == m) mine = (u32)(j * 32 + lane);
      const u32 ew = __reduce_min_sync(0xffffffffu, mine);
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (j * 32 + lane == (int)ew) o[j] = 0u;
      if (lane == r) pick = (int)ew;
    }
  }
  const float w = lane < K ? router_sigmoid(row[pick]) : 0.f;
  float den = w;
  for (int off = K / 2; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
  if (lane < K) {
    wts_out[lane] = (w / (den + 1e-20f)) * rsv;
    idx_out[lane] = pick;
  }
  return pick;
}

template <int EPL>
__global__ void __launch_bounds__(256) topk_kernel(const float* __restrict__ S, int lds, const float* __restrict__ bias,
                                                   const bf16* __restrict__ rs, int T, int E, int K,
                                                   int* __restrict__ idx, float* __restrict__ wts) {
  __shared__ u32 ck[8][TOPK_CAND];
  __shared__ int ce[8][TOPK_CAND];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const float rsv = __bfloat162float(rs[0]);
  for (int t = blockIdx.x * warps + warp; t < T; t += gridDim.x * warps)
    topk_warp<EPL>(S + (long long)t * lds, bias, E, K, rsv, lane, ck[warp], ce[warp], idx + (long long)t * K,
                   wts + (long long)t * K);
}

// ============================================================ routing tables
// Rows are processed in blocks of TB = 256.  A row r has K ids (global expert
// indices); the ones in [first, first + E) are local expert id - first, the
// others are foreign (exp2perm = -1).  With `shared`, a further expert E
// (the shared expert) takes every row.  Within an expert the permuted rows are
// in row order, so every table is the same bytes on every run.
#define TB 256

// blockcount[b][e] for e in [0, E + shared): the local picks of block b.
__global__ void __launch_bounds__(TB) route_count_kernel(const int* __restrict__ ids, int R, int K, int first, int E,
                                                          int shared, int* __restrict__ blockcount,
                                                          u32* __restrict__ err) {
  extern __shared__ int hist[];
  const int EL = E + shared;
  for (int i = threadIdx.x; i < EL; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int r0 = blockIdx.x * TB;
  const int nrows = min(TB, R - r0);
  for (int i = threadIdx.x; i < nrows * K; i += blockDim.x) {
    const int e = ids[(long long)r0 * K + i] - first;
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  if (shared && threadIdx.x == 0) hist[E] = nrows;
  __syncthreads();
  for (int i = threadIdx.x; i < EL; i += blockDim.x) blockcount[(long long)blockIdx.x * EL + i] = hist[i];
}

// One block of 1024 threads.  count[e] = sum over blocks; CTA counts
// ceil(count/tile) exclusive-scanned into off[e]; cta c of expert e covers
// permuted rows [tile*c, tile*(c+1)), real up to cta_limit[c] =
// min(tile*(c+1), tile*off[e] + count[e]); padding rows route row 0.
// blockoff[b][e] = picks of e in the blocks before b; blockcount[0][e] (read, then reused) = tile*off[e].
// meta[0] = num_non_exiting, meta[1] = total_padded, meta[2] = the shared
// expert's first permuted row (tile*off[E]) or -1.
__global__ void __launch_bounds__(1024) route_tables_kernel(int* __restrict__ blockcount, int blocks, int E,
                                                             int shared, int tile, int* __restrict__ blockoff,
                                                             int* __restrict__ counts, int* __restrict__ cta_batch,
                                                             int* __restrict__ cta_limit, int* __restrict__ meta,
                                                             int* __restrict__ route_map) {
  __shared__ int s_cnt[2048 + 1];
  __shared__ int s_off[2048 + 1];
  __shared__ int s_wsum[32];
  const int EL = E + shared;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  // an expert's picks before each block (its column of blockcount, loads 8 at a time so they overlap)
  for (int e = t; e < EL; e += blockDim.x) {
    int run = 0, b = 0;
    for (; b + 8 <= blocks; b += 8) {
      int c[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) c[i] = blockcount[(long long)(b + i) * EL + e];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        blockoff[(long long)(b + i) * EL + e] = run;
        run += c[i];
      }
    }
    for (; b < blocks; ++b) {
      const int c = blockcount[(long long)b * EL + e];
      blockoff[(long long)b * EL + e] = run;
      run += c;
    }
    s_cnt[e] = run;
    counts[e] = run;
  }
  __syncthreads();
  // exclusive scan of ctas over experts: thread t owns experts 2t, 2t+1 (EL <= 2048)
  int c0 = 0, c1 = 0;
  if (2 * t < EL) c0 = (s_cnt[2 * t] + tile - 1) / tile;
  if (2 * t + 1 < EL) c1 = (s_cnt[2 * t + 1] + tile - 1) / tile;
  int incl = c0 + c1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_wsum[warp] = incl;
  __syncthreads();
  int base = 0, total = 0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    const int s = s_wsum[w];
    base += w < warp ? s : 0;
    total += s;
  }
  if (2 * t < EL) s_off[2 * t] = base + incl - c0 - c1;
  if (2 * t + 1 < EL) s_off[2 * t + 1] = base + incl - c1;
  if (t == 0) s_off[EL] = total;
  __syncthreads();
  if (t == 0) {
    meta[0] = total;
    meta[1] = total * tile;
    meta[2] = shared ? s_off[E] * tile : -1;
  }
  for (int e = t; e < EL; e += blockDim.x) {
    const int o = s_off[e], n = s_off[e + 1] - o, cnt = s_cnt[e];
    // tile 1 plans positions only (the all-to-all send order): no CTA tables
    for (int c = 0; c < n && tile > 1; ++c) {
      cta_batch[o + c] = e;
      cta_limit[o + c] = min((o + c + 1) * tile, o * tile + cnt);
    }
    for (int r = o * tile + cnt; r < (o + n) * tile; ++r) route_map[r] = 0;
    // the expert's first permuted row, for the scatter: row 0 of blockcount is spent, its column e is reused
    blockcount[e] = o * tile;
  }
}

// The permuted row of pick (r, k) is ebase[e] (the expert's first row) + blockoff[b][e] + the picks of e
// by rows of the block before r (a bitmap popcount): route_map[row] = r, exp2perm[r*K+k] = row.
// Shared-expert rows are tile*off[E] + r and go to route_map only.
__global__ void __launch_bounds__(TB) route_scatter_kernel(const int* __restrict__ ids, int R, int K, int first, int E,
                                                            int shared, const int* __restrict__ ebase,
                                                            const int* __restrict__ blockoff,
                                                            int* __restrict__ route_map, int* __restrict__ exp2perm) {
  extern __shared__ u32 bits[];  // [E][TB/32]
  const int EL = E + shared;
  constexpr int W = TB / 32;
  for (int i = threadIdx.x; i < E * W; i += blockDim.x) bits[i] = 0u;
  __syncthreads();
  const int r0 = blockIdx.x * TB;
  const int nrows = min(TB, R - r0);
  for (int i = threadIdx.x; i < nrows * K; i += blockDim.x) {
    const int e = ids[(long long)r0 * K + i] - first;
    if (e >= 0 && e < E) {
      const int lr = i / K;
      atomicOr(&bits[e * W + (lr >> 5)], 1u << (lr & 31));
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nrows * K; i += blockDim.x) {
    const int e = ids[(long long)r0 * K + i] - first;
    const long long gi = (long long)r0 * K + i;
    if (e < 0 || e >= E) {
      exp2perm[gi] = -1;
      continue;
    }
    const int lr = i / K;
    int rank = 0;
    for (int w = 0; w < (lr >> 5); ++w) rank += __popc(bits[e * W + w]);
    rank += __popc(bits[e * W + (lr >> 5)] & ((1u << (lr & 31)) - 1u));
    const int row = ebase[e] + blockoff[(long long)blockIdx.x * EL + e] + rank;
    exp2perm[gi] = row;
    route_map[row] = r0 + lr;
  }
  if (shared) {
    const int sb = ebase[E] + blockoff[(long long)blockIdx.x * EL + E];
    for (int lr = threadIdx.x; lr < nrows; lr += blockDim.x) route_map[sb + lr] = r0 + lr;
  }
}

// ============================================================ MXFP8 quantisation
// Four lanes hold one 32-element group (8 bf16 each); the group's exponent is
// the one of k3_moe_prefill.cu:66-95 (e = ceil(log2(amax/448)), clamp
// [-127,127]) and the elements are cvt.rn.satfinite.e4m3(x * 2^-e).
__device__ __forceinline__ uint2 quant8_lanes(const uint4 u, int& sfbyte) {
  const u32* p = reinterpret_cast<const u32*>(&u);
  float2 v[4];
  float amax = 0.f;
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    v[l] = bf16x2_to_f2(p[l]);
    amax = fmaxf(amax, fmaxf(fabsf(v[l].x), fabsf(v[l].y)));
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const int e = mx8_exponent(amax);
  const float s = exp2f((float)-e);
  sfbyte = e + 127;
  uint2 w;
  w.x = (u32)e4m3x2_sat(v[0].x * s, v[0].y * s) | ((u32)e4m3x2_sat(v[1].x * s, v[1].y * s) << 16);
  w.y = (u32)e4m3x2_sat(v[2].x * s, v[2].y * s) | ((u32)e4m3x2_sat(v[3].x * s, v[3].y * s) << 16);
  return w;
}

// Quantise rows of x (row stride ldx elements, `cols` a multiple of 256) and
// write q/sf to every permuted row the row is routed to (exp2perm, plus the
// shared expert's row).  q in the tile-major operand layout (op8_offset), SF in
// the 128x4-tiled layout over permuted rows.
// One warp a row; a lane covers 8 columns of each 256-column piece.
__device__ __forceinline__ void quant_permute_rows(const bf16* __restrict__ x, int ldx, int R, int cols, int K,
                                                   const int* __restrict__ exp2perm, const int* __restrict__ meta,
                                                   uint8_t* __restrict__ qp, uint8_t* __restrict__ sfp) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int kt = cols / 128, kg4 = (cols / 32 + 3) / 4;
  const int shared_base = meta[2];
  const int nd = K + (shared_base >= 0 ? 1 : 0);  // destination slots: the K picks, then the shared expert's row
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < R; r += gridDim.x * warps) {
    // lane d < nd holds destination d's permuted row (or -1) and its row bases in q and in the scales
    int p = -1;
    if (lane < K) p = exp2perm[(long long)r * K + lane];
    else if (lane == K && shared_base >= 0) p = shared_base + r;
    const long long qrow = p >= 0 ? (long long)(p >> 7) * kt * (128 * 128) + (p & 127) * 128 : 0;
    const long long srow = p >= 0 ? (long long)(p >> 7) * kg4 * 512 + (p & 31) * 16 + ((p & 127) >> 5) * 4 : 0;
    const bf16* xr = x + (long long)r * ldx;
    // the row's pieces four at a time: their loads in flight together
    for (int c00 = 0; c00 < cols; c00 += 4 * 256) {
      uint4 ub[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (c00 + i * 256 < cols) ub[i] = *reinterpret_cast<const uint4*>(xr + c00 + i * 256 + lane * 8);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
      const int c0 = c00 + i * 256;
      if (c0 >= cols) break;
      const int c = c0 + lane * 8;
      const uint4 u = ub[i];
      int sfb;
      const uint2 w = quant8_lanes(u, sfb);
      // gather the 4 groups' scale bytes of this 128-column half into lane 0 / 16
      const int kb = c / 32;
      u32 sfw = (u32)sfb << (8 * (kb & 3));
      sfw |= __shfl_down_sync(0xffffffffu, sfw, 4);
      sfw |= __shfl_down_sync(0xffffffffu, sfw, 8);
      const int qcol = (c >> 7) * (128 * 128) + (c & 127);
      const int scol = (kb >> 2) * 512;
      for (int d = 0; d < nd; ++d) {
        const int pd = __shfl_sync(0xffffffffu, p, d);
        if (pd < 0) continue;  // the same for the whole warp
        const long long qd = __shfl_sync(0xffffffffu, qrow, d);
        const long long sd = __shfl_sync(0xffffffffu, srow, d);
        *reinterpret_cast<uint2*>(qp + qd + qcol) = w;
        if ((lane & 15) == 0) *reinterpret_cast<u32*>(sfp + sd + scol) = sfw;
      }
      }
    }
  }
}

__global__ void __launch_bounds__(256) quant_permute_kernel(const bf16* __restrict__ x, int ldx, int R, int cols, int K,
                                                            const int* __restrict__ exp2perm,
                                                            const int* __restrict__ meta, uint8_t* __restrict__ qp,
                                                            uint8_t* __restrict__ sfp) {
  quant_permute_rows(x, ldx, R, cols, K, exp2perm, meta, qp, sfp);
}

// Linear-SF quantiser (kern_k3_moe_quant's layout): q [rows, cols], sf [rows, cols/32].
__global__ void __launch_bounds__(256) quant_linear_kernel(const bf16* __restrict__ x, int ldx, int rows, int cols,
                                                           uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int per_row = cols / 256;
  const long long n = (long long)rows * per_row;
  for (long long i = (long long)blockIdx.x * warps + (threadIdx.x >> 5); i < n; i += (long long)gridDim.x * warps) {
    const long long r = i / per_row;
    const int c = (int)(i % per_row) * 256 + lane * 8;
    const uint4 u = *reinterpret_cast<const uint4*>(x + r * ldx + c);
    int sfb;
    const uint2 w = quant8_lanes(u, sfb);
    *reinterpret_cast<uint2*>(q + r * cols + c) = w;
    if ((lane & 3) == 0) sf[r * (cols / 32) + c / 32] = (uint8_t)sfb;
  }
}

// Tiled-SF quantiser (kern_k3_mxfp8_quant's layout) over a row range.
__global__ void __launch_bounds__(256) quant_tiled_kernel(const bf16* __restrict__ x, int ldx, int rows, int cols,
                                                          uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int per_row = cols / 256;
  const int kg4 = (cols / 32 + 3) / 4;
  const long long n = (long long)rows * per_row;
  for (long long i = (long long)blockIdx.x * warps + (threadIdx.x >> 5); i < n; i += (long long)gridDim.x * warps) {
    const long long r = i / per_row;
    const int c = (int)(i % per_row) * 256 + lane * 8;
    const uint4 u = *reinterpret_cast<const uint4*>(x + r * ldx + c);
    int sfb;
    const uint2 w = quant8_lanes(u, sfb);
    const int kb = c / 32;
    u32 sfw = (u32)sfb << (8 * (kb & 3));
    sfw |= __shfl_down_sync(0xffffffffu, sfw, 4);
    sfw |= __shfl_down_sync(0xffffffffu, sfw, 8);
    *reinterpret_cast<uint2*>(q + r * cols + c) = w;
    if ((lane & 15) == 0) *reinterpret_cast<u32*>(sf + sf_tiled_offset(r, kb, kg4)) = sfw;
  }
}

// ============================================================ combine
// out[t] = bf16( sum_{k=0..K-1, p>=0} fma(w[t,k], fc2[p], acc)  (+ fc2[shared_base+t]) ),
// f32, k in order, the shared expert (weight 1) last.  Rows t >= T are zero.
// One block a row, 8 columns a thread a step.
__device__ __forceinline__ void combine_row(const bf16* __restrict__ fc2, const int* __restrict__ exp2perm,
                                            const float* __restrict__ wts, const int* __restrict__ meta,
                                            bf16* __restrict__ out, int ldo, int T, int K, int cols, int t) {
  __shared__ int sp[17];
  __shared__ float sw[17];
  const int shared_base = meta ? meta[2] : -1;
  int n = 0;
  if (t < T) {
    if (threadIdx.x < K) {
      sp[threadIdx.x] = exp2perm[(long long)t * K + threadIdx.x];
      sw[threadIdx.x] = wts[(long long)t * K + threadIdx.x];
    }
    if (threadIdx.x == 0) {
      sp[K] = shared_base >= 0 ? shared_base + t : -1;
      sw[K] = 1.0f;
    }
    n = K + 1;
  }
  __syncthreads();
  for (int h = threadIdx.x; h < cols / 8; h += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < n; ++k) {
      const int p = sp[k];
      if (p < 0) continue;
      const float w = sw[k];
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(fc2 + (long long)p * cols) + h);
      const u32* pv = reinterpret_cast<const u32*>(&u);
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const float2 f = bf16x2_to_f2(pv[l]);
        acc[2 * l] = fmaf(w, f.x, acc[2 * l]);
        acc[2 * l + 1] = fmaf(w, f.y, acc[2 * l + 1]);
      }
    }
    uint4 o;
    o.x = f2_to_bf16x2(acc[0], acc[1]);
    o.y = f2_to_bf16x2(acc[2], acc[3]);
    o.z = f2_to_bf16x2(acc[4], acc[5]);
    o.w = f2_to_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + (long long)t * ldo)[h] = o;
  }
}

__global__ void __launch_bounds__(256) combine_kernel(const bf16* __restrict__ fc2, const int* __restrict__ exp2perm,
                                                      const float* __restrict__ wts, const int* __restrict__ meta,
                                                      bf16* __restrict__ out, int ldo, int T, int K, int cols) {
  combine_row(fc2, exp2perm, wts, meta, out, ldo, T, K, cols, blockIdx.x);
}

// ============================================================ MXFP4 weights
// OCP MX rule for E2M1 elements with a UE8M0 scale per 32 along K:
// shared exponent X = floor(log2(amax)) - 2 (E2M1's largest power is 2^2),
// scale byte X + 127 clamped to [0, 254] (amax = 0 gives byte 0), elements
// v / 2^X rounded to nearest even on the E2M1 grid {0,.5,1,1.5,2,3,4,6},
// saturated at 6.  All arithmetic is exact (scaling by powers of two, integer
// exponent extraction), so the host restatement gives the same bytes.
__host__ __device__ __forceinline__ int floor_log2_f32(float a) {
  // a > 0 and finite
  u32 b;
#ifdef __CUDA_ARCH__
  b = __float_as_uint(a);
#else
  memcpy(&b, &a, 4);
#endif
  const int ex = (int)((b >> 23) & 0xff);
  if (ex != 0) return ex - 127;
  // subnormal: position of the top mantissa bit
  const u32 m = b & 0x7fffffu;
  int top = 31;
  while (!((m >> top) & 1u)) --top;
  return top - 149;
}

// 2^n exactly, n in [-149, 127]
__host__ __device__ __forceinline__ float pow2i(int n) {
  const u32 b = n >= -126 ? (u32)(n + 127) << 23 : 1u << (n + 149);
  float f;
#ifdef __CUDA_ARCH__
  f = __uint_as_float(b);
#else
  memcpy(&f, &b, 4);
#endif
  return f;
}

__host__ __device__ __forceinline__ u32 e2m1_code(float y) {
  // y already scaled; round to nearest even on the E2M1 grid, saturate at 6
  const u32 sign = y < 0.f ? 8u : 0u;
  const float a = fabsf(y);
  u32 c;
  if (a <= 0.25f) c = 0;        // 0.25 ties to 0 (even)
  else if (a < 0.75f) c = 1;    // 0.5
  else if (a <= 1.25f) c = 2;   // 1.0 (0.75 ties up to 1.0, 1.25 ties down to 1.0)
  else if (a < 1.75f) c = 3;    // 1.5
  else if (a <= 2.5f) c = 4;    // 2.0 (1.75 ties up, 2.5 ties down)
  else if (a < 3.5f) c = 5;     // 3.0
  else if (a <= 5.0f) c = 6;    // 4.0 (3.5 ties up, 5 ties down)
  else c = 7;                   // 6.0 (saturate)
  return sign | c;
}

__host__ __device__ __forceinline__ int mx4_exponent(float amax) {
  if (!(amax > 0.f)) return -127;
  int x = floor_log2_f32(amax) - 2;
  return x < -127 ? -127 : (x > 127 ? 127 : x);
}

// w f32 [rows, K] -> packed E2M1 (element 2i in the low nibble of byte i) in
// the tile-major operand layout (op4_offset; rows a multiple of 128) and
// scales in the 128x4-tiled layout: the scale of (row r, group kb) is at
// sf_tiled_offset(r, kb, K/128).  One thread a 32-element group.
__global__ void __launch_bounds__(256) quant_mxfp4_kernel(const float* __restrict__ w, long long rows, int K,
                                                          uint8_t* __restrict__ packed, uint8_t* __restrict__ sf) {
  const int kbn = K / 32, kg4 = (kbn + 3) / 4;
  const long long n = rows * kbn;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / kbn;
    const int kb = (int)(i % kbn);
    const float4* src = reinterpret_cast<const float4*>(w + r * K + kb * 32);
    float v[32];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 f = src[j];
      v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
    }
    const int x = mx4_exponent(amax);
    const float inv = pow2i(-x);
    u32 out[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 32; ++j) out[j >> 3] |= e2m1_code(v[j] * inv) << (4 * (j & 7));
    uint4* dst = reinterpret_cast<uint4*>(packed + op4_offset(r, kb * 32, K));
    *dst = make_uint4(out[0], out[1], out[2], out[3]);
    sf[sf_tiled_offset(r, kb, kg4)] = (uint8_t)(x + 127);
  }
}

// Deterministic synthetic weights: value (row r, column c) of stream `seed`
// is an Irwin-Hall(4) draw scaled to standard deviation `sd`, made from the
// splitmix64 hash of (seed, r, c) with integer sums and one correctly rounded
// conversion, so host and device produce the same f32 bits.
__host__ __device__ __forceinline__ u64 splitmix64(u64 z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__host__ __device__ __forceinline__ float synth_value(u64 seed, long long r, int c, float sd) {
  const u64 h1 = splitmix64(seed * 0x100000001B3ull ^ ((u64)r << 20) ^ (u64)c);
  const u64 h2 = splitmix64(h1);
  // four 24-bit uniforms, centred: |s| < 2^25; the sum's standard deviation is 2^24 / sqrt(3)
  const long long s = (long long)(h1 & 0xFFFFFF) + (long long)((h1 >> 32) & 0xFFFFFF) + (long long)(h2 & 0xFFFFFF) +
                      (long long)((h2 >> 32) & 0xFFFFFF) - (2ll << 24);
  const float scale = sd * 1.7320508f / 16777216.0f;
  return (float)s * scale;  // one conversion (round to nearest) and one multiply
}

// Generate + quantise in one pass: rows [row0, row0 + rows) of stream `seed`.
__global__ void __launch_bounds__(256) synth_mxfp4_kernel(u64 seed, long long row0, long long rows, int K, float sd,
                                                          uint8_t* __restrict__ packed, uint8_t* __restrict__ sf) {
  const int kbn = K / 32, kg4 = (kbn + 3) / 4;
  const long long n = rows * kbn;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / kbn;
    const int kb = (int)(i % kbn);
    float v[32];
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      v[j] = synth_value(seed, row0 + r, kb * 32 + j, sd);
      amax = fmaxf(amax, fabsf(v[j]));
    }
    const int x = mx4_exponent(amax);
    const float inv = pow2i(-x);
    u32 out[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 32; ++j) out[j >> 3] |= e2m1_code(v[j] * inv) << (4 * (j & 7));
    *reinterpret_cast<uint4*>(packed + op4_offset(r, kb * 32, K)) = make_uint4(out[0], out[1], out[2], out[3]);
    sf[sf_tiled_offset(r, kb, kg4)] = (uint8_t)(x + 127);
  }
}

}  // namespace k3
