// Drop-in kernel entries: the reference's module entry names, argument lists
// and launch geometry (docs/k3-kernel-abi.md §0 conventions; kernels.toml), so
// a manifest that binds the reference's modules can bind this one instead.
// Every entry computes with this project's own kernels' arithmetic and matches
// the reference entry byte for byte (tests/test_gpu_dropin.py).  TOPK is 16 and
// LATENT 3584, as compiled into the reference modules.
//
//   kern_k3_moe_quant           source/k3_moe_prefill.cu:66   grid ceil(rows*cols/32/256), block 256
//   kern_k3_mxfp8_quant         source/k3_mxfp8.cu:20         any grid, block 256
//   kern_k3g_router_topk        source/k3_prefill_glue.cu:504 grid ceil(B/4), block 128 (E = 896)
//   kern_k3_router_topk         source/k3_router_argmax.cu:110 grid B, block 1024 (E = 896)
//   kern_k3_moe_route_count     source/k3_moe_prefill.cu:97   grid ceil(T/256), block 256
//   kern_k3_moe_route_tables    source/k3_moe_prefill.cu:115  grid 1, block 1024
//   kern_k3_moe_route_scatter   source/k3_moe_prefill.cu:155  grid ceil(T/256), block 256
//   kern_k3_moe_finalize        source/k3_moe_prefill.cu:206  grid rows, any block
//   kern_k3g_finalize_rms       source/k3_prefill_glue.cu:573 grid rows, block cols/8
//   kern_k3g_moe_finalize_rms   source/k3_moe_route.cu:538    grid rows, block 448
//   kern_k3g_moe_route          source/k3_moe_route.cu:338    grid 64 (B <= 256) or 288, block 512 (grid barrier)
//   kern_k3g_moe_route_init     source/k3_moe_route.cu:522    any grid, block 1024
//   kern_k3g_situ               source/k3_prefill_glue.cu:668 grid (B, ceil(n/2048)), block 256
//   kern_k3_moe_w_shuffle       source/k3_moe_prefill.cu:242  grid ceil(experts*n*row_bytes/16/block)
//   kern_k3_moe_sf_shuffle      source/k3_moe_prefill.cu:252  grid ceil(experts*n*kg/block)
//   kern_k3_moe_front           source/k3_moe_front.cu:358    grid T + NSH/64 (T <= 64), block 1024, F_SMEM
//                                                             dynamic shared bytes, PDL dependent
#include "common.cuh"

namespace k3 {
namespace dropin {
constexpr int TOPK = 16;
constexpr int N_EXPERTS = 896;
constexpr int LATENT = 3584;
constexpr int MAX_LOCAL = 1024;  // local experts the table entries handle (the reference's: 64)
}  // namespace dropin

// 32 elements a thread: the MXFP8 rule over one group, 32 E4M3 bytes + the scale
__device__ __forceinline__ void quant32(const bf16* __restrict__ src, uint8_t* __restrict__ q, uint8_t* __restrict__ sf) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  u32 w[16];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 u = s[j];
    w[4 * j] = u.x; w[4 * j + 1] = u.y; w[4 * j + 2] = u.z; w[4 * j + 3] = u.w;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float2 f = bf16x2_to_f2(w[j]);
    amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  const int e = mx8_exponent(amax);
  const float sc = exp2f((float)-e);
  *sf = (uint8_t)(e + 127);
  u32 o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 a = bf16x2_to_f2(w[2 * j]), b = bf16x2_to_f2(w[2 * j + 1]);
    o[j] = (u32)e4m3x2_sat(a.x * sc, a.y * sc) | ((u32)e4m3x2_sat(b.x * sc, b.y * sc) << 16);
  }
  uint4* d = reinterpret_cast<uint4*>(q);
  d[0] = make_uint4(o[0], o[1], o[2], o[3]);
  d[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

}  // namespace k3

using namespace k3;

extern "C" __global__ void __launch_bounds__(256) kern_k3_moe_quant(const bf16* __restrict__ x, uint8_t* __restrict__ q,
                                                                    uint8_t* __restrict__ sf, int rows, int cols) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * cols / 32) return;
  quant32(x + i * 32, q + i * 32, sf + i);
}

extern "C" __global__ void __launch_bounds__(256) kern_k3_mxfp8_quant(const bf16* __restrict__ x, int ld,
                                                                      uint8_t* __restrict__ q, uint8_t* __restrict__ sf,
                                                                      int rows, int cols) {
  const int kb = cols / 32, kg4 = (kb + 3) / 4;
  const long long n = (long long)rows * kb;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / kb;
    const int b = (int)(i % kb);
    uint8_t s;
    quant32(x + r * ld + b * 32, q + i * 32, &s);
    sf[sf_tiled_offset(r, b, kg4)] = s;
  }
}

extern "C" __global__ void __launch_bounds__(128) kern_k3g_router_topk(const float* __restrict__ S,
                                                                       const float* __restrict__ bias,
                                                                       const bf16* __restrict__ rs,
                                                                       int* __restrict__ idx, float* __restrict__ wts,
                                                                       int B) {
  __shared__ u32 ck[4][TOPK_CAND];
  __shared__ int ce[4][TOPK_CAND];
  const int warp = threadIdx.x >> 5, b = blockIdx.x * 4 + warp;
  if (b >= B) return;
  topk_warp<dropin::N_EXPERTS / 32>(S + (long long)b * dropin::N_EXPERTS, bias, dropin::N_EXPERTS, dropin::TOPK,
                                  __bfloat162float(rs[0]), threadIdx.x & 31, ck[warp], ce[warp],
                                  idx + (long long)b * dropin::TOPK, wts + (long long)b * dropin::TOPK);
}

// kern_k3_router_topk (source/k3_router_argmax.cu:110-206): the decode router's top-16 of S [B, 896], one block
// a row, grid (B), block 1024 (the reference's launch: the experts rounded up to 256); warp 0 runs the same
// selection as kern_k3g_router_topk, so the picks and weight bits are that entry's.
extern "C" __global__ void __launch_bounds__(1024, 1) kern_k3_router_topk(const float* __restrict__ S,
                                                                          const float* __restrict__ bias,
                                                                          const bf16* __restrict__ rs,
                                                                          int* __restrict__ idx, float* __restrict__ wts,
                                                                          int B) {
  __shared__ u32 ck[TOPK_CAND];
  __shared__ int ce[TOPK_CAND];
  const int b = blockIdx.x;
  if (b >= B || threadIdx.x >= 32) return;
  topk_warp<dropin::N_EXPERTS / 32>(S + (long long)b * dropin::N_EXPERTS, bias, dropin::N_EXPERTS, dropin::TOPK,
                                    __bfloat162float(rs[0]), threadIdx.x, ck, ce, idx + (long long)b * dropin::TOPK,
                                    wts + (long long)b * dropin::TOPK);
}

// ------------------------------------------------------------------ EP-slice routing tables (top-16)
// Local experts are [rank*E, rank*E + E); the entries keep the reference's
// buffers (blockcount / blockoff [blocks][E], num_non_exiting, total_padded).
extern "C" __global__ void __launch_bounds__(256) kern_k3_moe_route_count(const int* __restrict__ ids, int T, int rank,
                                                                          int E, int* __restrict__ blockcount) {
  __shared__ int hist[dropin::MAX_LOCAL];
  for (int i = threadIdx.x; i < E; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int r0 = blockIdx.x * 256, nrows = min(256, T - r0), first = rank * E;
  for (int i = threadIdx.x; i < nrows * dropin::TOPK; i += blockDim.x) {
    const int e = ids[(long long)r0 * dropin::TOPK + i] - first;
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x) blockcount[(long long)blockIdx.x * E + i] = hist[i];
}

extern "C" __global__ void __launch_bounds__(1024) kern_k3_moe_route_tables(
    const int* __restrict__ blockcount, int blocks, int E, int tile, int* __restrict__ blockoff,
    int* __restrict__ cta_batch, int* __restrict__ cta_limit, int* __restrict__ num_non_exiting,
    int* __restrict__ total_padded, int* __restrict__ route_map) {
  __shared__ int s_cnt[dropin::MAX_LOCAL], s_off[dropin::MAX_LOCAL + 1];
  const int t = threadIdx.x;
  for (int e = t; e < E; e += blockDim.x) {
    int run = 0;
    for (int b = 0; b < blocks; ++b) {
      const int c = blockcount[(long long)b * E + e];
      blockoff[(long long)b * E + e] = run;
      run += c;
    }
    s_cnt[e] = run;
  }
  __syncthreads();
  if (t == 0) {  // at most MAX_LOCAL experts: a serial scan is a few microseconds
    int run = 0;
    for (int e = 0; e < E; ++e) {
      s_off[e] = run;
      run += (s_cnt[e] + tile - 1) / tile;
    }
    s_off[E] = run;
    num_non_exiting[0] = run;
    total_padded[0] = run * tile;
  }
  __syncthreads();
  for (int e = t; e < E; e += blockDim.x) {
    const int o = s_off[e], n = s_off[e + 1] - o, cnt = s_cnt[e];
    for (int c = 0; c < n; ++c) {
      cta_batch[o + c] = e;
      cta_limit[o + c] = min((o + c + 1) * tile, o * tile + cnt);
    }
    for (int r = o * tile + cnt; r < (o + n) * tile; ++r) route_map[r] = 0;
    for (int b = 0; b < blocks; ++b) blockoff[(long long)b * E + e] += o * tile;
  }
}

extern "C" __global__ void __launch_bounds__(256) kern_k3_moe_route_scatter(const int* __restrict__ ids,
                                                                            const int* __restrict__ blockoff, int T,
                                                                            int rank, int E,
                                                                            int* __restrict__ route_map,
                                                                            int* __restrict__ exp2perm) {
  __shared__ u32 bits[dropin::MAX_LOCAL * 8];  // [expert][256 rows / 32]
  for (int i = threadIdx.x; i < E * 8; i += blockDim.x) bits[i] = 0u;
  __syncthreads();
  const int r0 = blockIdx.x * 256, nrows = min(256, T - r0), first = rank * E;
  for (int i = threadIdx.x; i < nrows * dropin::TOPK; i += blockDim.x) {
    const int e = ids[(long long)r0 * dropin::TOPK + i] - first;
    if (e >= 0 && e < E) {
      const int lr = i / dropin::TOPK;
      atomicOr(&bits[e * 8 + (lr >> 5)], 1u << (lr & 31));
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nrows * dropin::TOPK; i += blockDim.x) {
    const long long gi = (long long)r0 * dropin::TOPK + i;
    const int e = ids[gi] - first;
    if (e < 0 || e >= E) {
      exp2perm[gi] = -1;
      continue;
    }
    const int lr = i / dropin::TOPK;
    int rank_in = 0;
    for (int w = 0; w < (lr >> 5); ++w) rank_in += __popc(bits[e * 8 + w]);
    rank_in += __popc(bits[e * 8 + (lr >> 5)] & ((1u << (lr & 31)) - 1u));
    const int row = blockoff[(long long)blockIdx.x * E + e] + rank_in;
    exp2perm[gi] = row;
    route_map[row] = r0 + lr;
  }
}

// ------------------------------------------------------------------ combine entries
extern "C" __global__ void __launch_bounds__(1024) kern_k3_moe_finalize(const bf16* __restrict__ fc2,
                                                                        const int* __restrict__ exp2perm,
                                                                        const float* __restrict__ wts,
                                                                        bf16* __restrict__ out, int T, int cols) {
  // rows t >= T come out zero (the gathered chunk's tail)
  combine_row(fc2, exp2perm, wts, nullptr, out, cols, T, dropin::TOPK, cols, blockIdx.x);
}

// the combine of one row normed by gamma: y = bf16(combine); r = rsqrt(mean(y^2) + 1e-5);
// out = bf16(bf16(y * r) * gamma).  The sum of squares runs in the reference's order
// (a thread's 8 columns in turn, then an xor butterfly in the warp, then over the
// warps' sums), so the bytes match.  One thread a group of 8 columns: block = cols/8.
__device__ __forceinline__ void finalize_rms_row(const bf16* __restrict__ fc2, const int* __restrict__ exp2perm,
                                                 const float* __restrict__ wts, const bf16* __restrict__ gamma,
                                                 bf16* __restrict__ orow, int T, int cols) {
  __shared__ float sm[33];
  __shared__ int sp[dropin::TOPK];
  __shared__ float sw[dropin::TOPK];
  const int t = blockIdx.x, h = threadIdx.x, lane = h & 31, warp = h >> 5;
  if (h < dropin::TOPK && t < T) {
    sp[h] = exp2perm[(long long)t * dropin::TOPK + h];
    sw[h] = wts[(long long)t * dropin::TOPK + h];
  }
  __syncthreads();
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (t < T) {
    for (int k = 0; k < dropin::TOPK; ++k) {
      const int p = sp[k];
      if (p < 0) continue;
      const float w = sw[k];
      const uint4 u = reinterpret_cast<const uint4*>(fc2 + (long long)p * cols)[h];
      const u32* pv = reinterpret_cast<const u32*>(&u);
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const float2 f = bf16x2_to_f2(pv[l]);
        acc[2 * l] = fmaf(w, f.x, acc[2 * l]);
        acc[2 * l + 1] = fmaf(w, f.y, acc[2 * l + 1]);
      }
    }
  }
  u32 y[4];
  float sum = 0.f;
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    y[l] = f2_to_bf16x2(acc[2 * l], acc[2 * l + 1]);
    const float2 f = bf16x2_to_f2(y[l]);
    sum = fmaf(f.x, f.x, sum);
    sum = fmaf(f.y, f.y, sum);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) sm[warp] = sum;
  if (h < 32 && h >= (int)(blockDim.x >> 5)) sm[h] = 0.f;
  __syncthreads();
  if (warp == 0) {
    float v = sm[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sm[32] = v;
  }
  __syncthreads();
  const float r = rsqrtf(sm[32] / (float)cols + 1e-5f);
  const uint4 gw = reinterpret_cast<const uint4*>(gamma)[h];
  const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&gw);
  uint4 o;
  __nv_bfloat162* ov = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const float2 f = bf16x2_to_f2(y[l]);
    ov[l] = __hmul2(__floats2bfloat162_rn(f.x * r, f.y * r), g[l]);
  }
  reinterpret_cast<uint4*>(orow)[h] = o;
}

extern "C" __global__ void __launch_bounds__(1024) kern_k3g_finalize_rms(const bf16* __restrict__ fc2,
                                                                         const int* __restrict__ exp2perm,
                                                                         const float* __restrict__ wts,
                                                                         const bf16* __restrict__ gamma,
                                                                         bf16* __restrict__ out, int T, int cols) {
  finalize_rms_row(fc2, exp2perm, wts, gamma, out + (long long)blockIdx.x * cols, T, cols);
}

extern "C" __global__ void __launch_bounds__(dropin::LATENT / 8) kern_k3g_moe_finalize_rms(
    const bf16* __restrict__ fc2, const int* __restrict__ exp2perm, const float* __restrict__ wts,
    const bf16* __restrict__ gamma, bf16* __restrict__ out, int ldo, int T) {
  finalize_rms_row(fc2, exp2perm, wts, gamma, out + (long long)blockIdx.x * ldo, T, dropin::LATENT);
}

// ------------------------------------------------------------------ the fused prefill front (one launch)
// kern_k3g_moe_route (source/k3_moe_route.cu:338-520, op scripts/k3_moe_bmm.py:96-100): router top-16,
// the latent in MXFP8 (linear scales), the shared expert's SiTU activation and the routing tables of a rank
// holding every expert, `tile` rows a CTA, in one launch.  Grid 64 (B <= 256) or 288 blocks of 512 threads,
// two an SM, every block resident: phase 1 (rows' top-k and their marks in this call's table; the latent
// and shared-activation pieces) | grid barrier | phase 2 (counts scanned into CTA offsets, the CTA tables,
// every pick's permuted row in row order).
//
// `sync` (SYNC_WORDS u32, zeroed once by kern_k3g_moe_route_init): word 0 the barrier's arrivals, word 32
// its generation, word 1 an error word (nonzero: a barrier wait ran out, the outputs are incomplete), then
// two routing tables picked by the generation's parity: [E] pick counts, [E][32] counts per 256-row chunk,
// [E][256] row bitmaps.  A call zeroes the other parity's table for the next call, so calls of any B need no
// re-initialisation.  The sizes are the reference's (the manifest allocates the buffer).
namespace k3 {
namespace dropin {
constexpr int SHARED_W = 6144;               // the shared expert's width: gu = [gate | up], act = SiTU(gate, up)
constexpr int MAX_ROWS = 8192;
constexpr int CHUNK = 256, CHUNKS = MAX_ROWS / CHUNK, WORDS = MAX_ROWS / 32;
constexpr int TABLE = N_EXPERTS * (1 + CHUNKS + WORDS);
constexpr int ARRIVE_AT = 0, ERR_AT = 1, GEN_AT = 32, TABLES_AT = 64;
constexpr int SYNC_WORDS = TABLES_AT + 2 * TABLE + 2;
constexpr int RT_THREADS = 512, RT_WARPS = RT_THREADS / 32;
constexpr u64 BARRIER_LIMIT_NS = 2000000000ull;
}  // namespace dropin

__device__ __forceinline__ u32 ld_acquire_gpu(const u32* p) {
  u32 v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(u32* p, u32 v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float tanh_approx(float x) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// The shared expert's activation as the reference's fused front computes it (source/k3_moe_route.cu:257-269,
// k3_prefill_glue.cu's kern_k3g_situ): e^-g by the __expf intrinsic, the sigmoid an IEEE reciprocal, the tanh
// terms tanh.approx, every product and sum rounded on its own: (4 tanh(g/4) * sigmoid(g)) * 25 tanh(u/25).
__device__ __forceinline__ float situ_front(float g, float u) {
  const float d = __fadd_rn(__expf(-g), 1.0f);
  const float a = __fmul_rn(tanh_approx(__fmul_rn(g, 0.25f)), 4.0f);
  const float c = __fmul_rn(tanh_approx(__fmul_rn(u, 0.04f)), 25.0f);
  return __fmul_rn(__fmul_rn(a, __frcp_rn(d)), c);
}

}  // namespace k3

extern "C" __global__ void __launch_bounds__(dropin::RT_THREADS, 2) kern_k3g_moe_route(
    const float* __restrict__ S, const float* __restrict__ bias, const bf16* __restrict__ rs,
    const bf16* __restrict__ x, int ldx, const bf16* __restrict__ gu, int ldgu, uint8_t* __restrict__ q,
    uint8_t* __restrict__ sf, int* __restrict__ idx, float* __restrict__ wts, bf16* __restrict__ act, int ldact,
    u32* __restrict__ sync, int* __restrict__ cta_batch, int* __restrict__ cta_limit,
    int* __restrict__ num_non_exiting, int* __restrict__ total_padded, int* __restrict__ route_map,
    int* __restrict__ exp2perm, int tile, int B) {
  using namespace k3::dropin;
  __shared__ u32 s_gen, s_ok;
  __shared__ int s_cnt[N_EXPERTS], s_off[N_EXPERTS];
  __shared__ int s_wsum[RT_WARPS];
  __shared__ u32 s_ck[RT_WARPS][TOPK_CAND];
  __shared__ int s_ce[RT_WARPS][TOPK_CAND];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int nthreads = gridDim.x * RT_THREADS, gt = blockIdx.x * RT_THREADS + t;
  const int gwarp = blockIdx.x * RT_WARPS + warp, nwarps = gridDim.x * RT_WARPS;
  if (B < 0 || B > MAX_ROWS || tile < 1) return;  // every block returns alike: no barrier is entered

  if (t == 0) s_gen = ld_acquire_gpu(sync + GEN_AT);
  __syncthreads();
  const u32 gen = s_gen;
  u32* cur = sync + TABLES_AT + (gen & 1u) * TABLE;
  u32* nxt = sync + TABLES_AT + (~gen & 1u) * TABLE;
  int* tot = reinterpret_cast<int*>(cur);
  int* chunk = tot + N_EXPERTS;
  u32* bits = cur + N_EXPERTS * (1 + CHUNKS);
  for (int i = gt; i < TABLE; i += nthreads) nxt[i] = 0u;  // the next call's table

  // ---- phase 1a: a warp a row: top-16, marked in this call's table
  const float rsv = __bfloat162float(rs[0]);
  for (int b = gwarp; b < B; b += nwarps) {
    const int e = topk_warp<N_EXPERTS / 32>(S + (long long)b * N_EXPERTS, bias, N_EXPERTS, TOPK, rsv, lane, s_ck[warp],
                                          s_ce[warp], idx + (long long)b * TOPK, wts + (long long)b * TOPK);
    if (lane < TOPK) {
      atomicAdd(tot + e, 1);
      atomicAdd(chunk + e * CHUNKS + b / CHUNK, 1);
      atomicOr(bits + e * WORDS + b / 32, 1u << (b & 31));
    }
  }
  // ---- phase 1b: 256-column pieces, a warp a piece: the latent's MXFP8 (kern_k3_moe_quant's bytes) and
  // the shared expert's SiTU activation
  const int nq = B * (LATENT / 256), ns = B * (SHARED_W / 256);
  for (int i = gwarp; i < nq + ns; i += nwarps) {
    if (i < nq) {
      const int b = i / (LATENT / 256), c = (i % (LATENT / 256)) * 256 + lane * 8;
      int sfb;
      const uint2 w = quant8_lanes(*reinterpret_cast<const uint4*>(x + (long long)b * ldx + c), sfb);
      *reinterpret_cast<uint2*>(q + (long long)b * LATENT + c) = w;
      if ((lane & 3) == 0) sf[(long long)b * (LATENT / 32) + c / 32] = (uint8_t)sfb;
    } else {
      const int j = i - nq, b = j / (SHARED_W / 256), c = (j % (SHARED_W / 256)) * 256 + lane * 8;
      const uint4 gv = *reinterpret_cast<const uint4*>(gu + (long long)b * ldgu + c);
      const uint4 uv = *reinterpret_cast<const uint4*>(gu + (long long)b * ldgu + SHARED_W + c);
      const u32* gp = reinterpret_cast<const u32*>(&gv);
      const u32* up = reinterpret_cast<const u32*>(&uv);
      uint4 o;
      u32* op = reinterpret_cast<u32*>(&o);
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const float2 g2 = bf16x2_to_f2(gp[l]), u2 = bf16x2_to_f2(up[l]);
        op[l] = f2_to_bf16x2(situ_front(g2.x, u2.x), situ_front(g2.y, u2.y));
      }
      *reinterpret_cast<uint4*>(act + (long long)b * ldact + c) = o;
    }
  }

  // ---- grid barrier (every block resident); a wait that runs out marks the error word and leaves
  __syncthreads();
  if (t == 0) {
    __threadfence();
    s_ok = 1u;
    if (atomicAdd(sync + ARRIVE_AT, 1u) == gridDim.x - 1) {
      atomicExch(sync + ARRIVE_AT, 0u);
      __threadfence();
      st_release_gpu(sync + GEN_AT, gen + 1u);
    } else {
      const u64 t0 = globaltimer_ns();
      while (ld_acquire_gpu(sync + GEN_AT) == gen) {
        if (globaltimer_ns() - t0 > BARRIER_LIMIT_NS) {
          atomicOr(sync + ERR_AT, 1u);
          s_ok = 0u;
          break;
        }
        __nanosleep(64);
      }
    }
    __threadfence();
  }
  __syncthreads();
  if (!s_ok) return;

  // ---- phase 2: CTA counts of the experts exclusive-scanned (thread t: experts 2t and 2t + 1)
  int c0 = 0, c1 = 0;
  if (2 * t < N_EXPERTS) {
    s_cnt[2 * t] = __ldcg(tot + 2 * t);
    s_cnt[2 * t + 1] = __ldcg(tot + 2 * t + 1);
    c0 = (s_cnt[2 * t] + tile - 1) / tile;
    c1 = (s_cnt[2 * t + 1] + tile - 1) / tile;
  }
  int incl = c0 + c1;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) s_wsum[warp] = incl;
  __syncthreads();
  int before = 0, total = 0;
  for (int w = 0; w < RT_WARPS; ++w) {
    before += w < warp ? s_wsum[w] : 0;
    total += s_wsum[w];
  }
  if (2 * t < N_EXPERTS) {
    s_off[2 * t] = before + incl - c0 - c1;
    s_off[2 * t + 1] = before + incl - c1;
  }
  __syncthreads();
  if (gt == 0) {
    num_non_exiting[0] = total;
    total_padded[0] = total * tile;
  }
  for (int e = gt; e < N_EXPERTS; e += nthreads) {
    const int n = (s_cnt[e] + tile - 1) / tile, o = s_off[e];
    for (int c = 0; c < n; ++c) {
      cta_batch[o + c] = e;
      cta_limit[o + c] = min((o + c + 1) * tile, o * tile + s_cnt[e]);
    }
  }
  // a pick's place among its expert's rows: its picks in the chunks before the row's chunk, then in the
  // chunk's bitmap words before the row's word, then in that word below the row (row order, every run alike)
  for (int b = gwarp; b < B; b += nwarps) {
    const int mine = lane < TOPK ? idx[(long long)b * TOPK + lane] : 0;
    const int bc = b / CHUNK, bw = b / 32;
    int place = 0;
    for (int k = 0; k < TOPK; ++k) {
      const int e = __shfl_sync(0xffffffffu, mine, k);
      int v = lane < bc ? __ldcg(chunk + e * CHUNKS + lane) : 0;
      const int w = bc * (CHUNK / 32) + lane;
      if (w <= bw) {
        const u32 word = __ldcg(bits + e * WORDS + w);
        v += __popc(w < bw ? word : (word & ((1u << (b & 31)) - 1u)));
      }
      v = __reduce_add_sync(0xffffffffu, v);
      if (lane == k) place = v;
    }
    if (lane < TOPK) {
      const int p = s_off[mine] * tile + place;
      exp2perm[(long long)b * TOPK + lane] = p;
      route_map[p] = b;
    }
  }
}

// kern_k3g_moe_route_init (source/k3_moe_route.cu:522): zero the sync words before a stage's first call
extern "C" __global__ void __launch_bounds__(1024) kern_k3g_moe_route_init(u32* __restrict__ sync) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dropin::SYNC_WORDS; i += gridDim.x * blockDim.x) sync[i] = 0u;
}

// K3's shared-expert SiTU on landed bf16 operands (kern_k3g_situ, source/k3_prefill_glue.cu:668-686): p = [gate |
// up] rows of 2n bf16, act [B, n] bf16.  Grid (B, ceil(n / 2048)), block 256, 8 columns a thread (n a
// multiple of 8); the fused front's arithmetic (situ_front).  The reference entry switches a warp to an
// approximate reciprocal with one Newton step when every gate is >= -87; the reference records that step equal
// to the correctly rounded reciprocal for every d in [2^-126, 2^126) (source/k3_moe_route.cu:78-80, checked
// over all of them), which holds 1 + e^-g there, so __frcp_rn on every lane gives the same bytes.
extern "C" __global__ void __launch_bounds__(256) kern_k3g_situ(const bf16* __restrict__ p, bf16* __restrict__ act,
                                                                 int n, int B) {
  const int b = blockIdx.x;
  const int j = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (b >= B || j >= n) return;
  const uint4 gv = *reinterpret_cast<const uint4*>(p + (long long)b * 2 * n + j);
  const uint4 uv = *reinterpret_cast<const uint4*>(p + (long long)b * 2 * n + n + j);
  const u32* gp = reinterpret_cast<const u32*>(&gv);
  const u32* up = reinterpret_cast<const u32*>(&uv);
  uint4 o;
  u32* op = reinterpret_cast<u32*>(&o);
#pragma unroll
  for (int l = 0; l < 4; ++l) {
    const float2 g2 = bf16x2_to_f2(gp[l]), u2 = bf16x2_to_f2(up[l]);
    op[l] = f2_to_bf16x2(situ_front(g2.x, u2.x), situ_front(g2.y, u2.y));
  }
  *reinterpret_cast<uint4*>(act + (long long)b * n + j) = o;
}

// ------------------------------------------------------------------ load-time weight re-layouts
// kern_k3_moe_w_shuffle / kern_k3_moe_sf_shuffle (source/k3_moe_prefill.cu:237-259, registered by
// scripts/k3_moe_bmm.py:176-184): the checkpoint's expert rows into the row order the TRT-LLM-gen GEMMs'
// epilogue expects, and (sf) the row scales into the 128x4-tiled layout.  Within each 32-row group, GEMM
// row r takes the checkpoint row whose position is (r % 8) * 4 + (r % 32) / 8 (a transpose of the 8 x 4
// arrangement); `gated` interleaves the two halves [up | gate] of FC1's 2I rows, even positions from the
// first half, odd from the second.  The layout is the consumer's (the prebuilt GEMMs), so the map is fixed.
__device__ __forceinline__ int gemm_row_source(int r, int n, int gated) {
  const int pos = (r & ~31) + (r & 7) * 4 + ((r & 31) >> 3);
  if (!gated) return pos;
  return (pos & 1) * (n / 2) + (pos >> 1);
}

// grid ceil(experts * n * row_bytes / 16 / block), any block: one 16-byte chunk a thread
extern "C" __global__ void kern_k3_moe_w_shuffle(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                 int experts, int n, int row_bytes, int gated) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int chunks = row_bytes / 16;
  if (i >= (long long)experts * n * chunks) return;
  const long long row = i / chunks;  // expert * n + r
  const int c = (int)(i - row * chunks);
  const int e = (int)(row / n), r = (int)(row - (long long)e * n);
  const uint4* s = reinterpret_cast<const uint4*>(src + ((long long)e * n + gemm_row_source(r, n, gated)) * row_bytes);
  reinterpret_cast<uint4*>(dst)[i] = s[c];
}

// grid ceil(experts * n * kg / block), any block: one scale byte a thread (kg = K / 32 groups a row)
extern "C" __global__ void kern_k3_moe_sf_shuffle(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                  int experts, int n, int kg, int gated) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)experts * n * kg) return;
  const long long row = i / kg;
  const int c = (int)(i - row * kg);
  const int e = (int)(row / n), r = (int)(row - (long long)e * n);
  dst[(long long)e * n * kg + sf_tiled_offset(r, c, kg / 4)] = src[((long long)e * n + gemm_row_source(r, n, gated)) * kg + c];
}

// ------------------------------------------------------------------ load-time re-layout for this build's GEMMs
// The same inputs as the two shuffles above (the checkpoint's MXFP4 `weight_packed` rows, E2M1 two a byte with
// element 2i in the low nibble, and their UE8M0 `weight_scale` bytes, [n rows, K/32] an expert; FC1 bound as
// [w3 (up); w1 (gate)], scripts/gen_stage.py:681-702) and the same parameter lists, so a derive program binds
// them by changing only the entry name; the outputs are the layout k3moe's grouped GEMMs read instead of the
// TRT-LLM-gen one.  `gated` (FC1) swaps the halves: rows [gate (the checkpoint's second half); up (its first)].
// Rows stay in order otherwise (the GEMMs need no epilogue permutation).  n and K multiples of 128.
__device__ __forceinline__ int tile_row_source(int r, int n, int gated) {
  if (!gated) return r;
  return r < n / 2 ? r + n / 2 : r - n / 2;
}

// grid ceil(experts * n * row_bytes / 16 / block), any block: one 16-byte chunk of the output a thread.  The
// output is tile-major (128 x 128-element tiles of 8 KB, tile (R/128, k/128) at (R/128) * (K/128) + k/128 over
// the flattened rows R = e * n + r), so a thread's chunk is 16 bytes of one tile row.
extern "C" __global__ void kern_k3_moe_w_tiles(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                               int experts, int n, int row_bytes, int gated) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)experts * n * (row_bytes / 16)) return;
  const long long t = i >> 9;                  // 8 KB tile: 512 chunks
  const int within = (int)(i & 511);
  const int kt_n = row_bytes / 64;             // tiles along K
  const long long R = (t / kt_n) * 128 + (within >> 2);
  const int b = (int)(t % kt_n) * 64 + (within & 3) * 16;
  const int e = (int)(R / n), r = (int)(R - (long long)e * n);
  reinterpret_cast<uint4*>(dst)[i] =
      *reinterpret_cast<const uint4*>(src + ((long long)e * n + tile_row_source(r, n, gated)) * row_bytes + b);
}

// grid ceil(experts * n * kg / 4 / block), any block: four scale bytes a thread (groups 4j..4j+3 of one row,
// adjacent in both layouts), into the 128x4-tiled layout over the flattened rows (kg = K / 32, a multiple of 4).
extern "C" __global__ void kern_k3_moe_sf_tiles(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                int experts, int n, int kg, int gated) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int q = kg / 4;
  if (i >= (long long)experts * n * q) return;
  const long long R = i / q;
  const int c = (int)(i - R * q) * 4;
  const int e = (int)(R / n), r = (int)(R - (long long)e * n);
  const u32 v = *reinterpret_cast<const u32*>(src + ((long long)e * n + tile_row_source(r, n, gated)) * kg + c);
  *reinterpret_cast<u32*>(dst + sf_tiled_offset(R, c, q)) = v;
}

// ------------------------------------------------------------------ the decode front (one launch)
// kern_k3_moe_front (source/k3_moe_front.cu:358-471; op scripts/gen_stage.py:416-428, 1080-1087): a decode
// step's MoE front over T <= 64 rows of the front GEMM's f32 output (F_LDS columns a row: router | latent |
// this rank's shared gate | up).  Grid T + NSH/64 blocks of 1024 threads, F_SMEM bytes of dynamic shared
// memory, launched as a programmatic dependent of the front GEMM (it waits at entry, then releases FC1).
//   row block b < T   top-16 of the router columns (idx, wts: kern_k3g_router_topk's picks and bits); the
//                     latent landed to bf16 and quantised to MXFP8 with linear scales (q, sf:
//                     kern_k3_moe_quant's bytes); the shared expert's SiTU row (act); with more than
//                     F_LOCAL_SITU_ROWS rows a flag to every shared-expert block once the act row is in
//                     (ready), and always the row's two lowest local picks to the shared-expert blocks'
//                     prefetchers (ids); the last row block to arrive (done) builds the
//                     routing tables of this rank's experts first + j * STRIDE (j < EXPERTS / STRIDE), TILE
//                     rows a CTA, an expert's rows in token order (the reference leaves them in atomic order;
//                     the GEMMs compute each row on its own), padding rows routing token 0, exp2perm -1 for
//                     another rank's expert.
//   block T + c       sh_out[:, 64c, 64c + 64) = act . Wsh[64c, 64c + 64)^T on the tensor cores: bf16
//                     operands, one f32 accumulation chain over K in 16-element steps in order (the order
//                     cuBLASLt sums this shape in), rounded to bf16; its last warp pulls a share of the
//                     first two touched experts' FC1 weights and scales into L2 while HBM is idle.
// Carries (the manifest zeroes them once): ready / ids [NSH/64][64] i32 (each consumer clears what it read),
// done i32 (the last row block resets the count).  Every wait is bounded (2 s); one that runs out sets bit 30
// of done (kept until the host clears it; the count is the low 16 bits) and its block skips the work that
// needed it instead of spinning.  The row blocks never wait and have the lower indices, so they are
// dispatched first.  The compile-time shape takes the reference module's defines (EXPERTS, LDS, SH, STRIDE,
// NSH) when given; the defaults are its own.
#ifdef EXPERTS
#define K3F_EXPERTS (EXPERTS)
#else
#define K3F_EXPERTS 896
#endif
#ifdef LDS
#define K3F_LDS (LDS)
#else
#define K3F_LDS 6016
#endif
#ifdef SH
#define K3F_SH (SH)
#else
#define K3F_SH 768
#endif
#ifdef STRIDE
#define K3F_STRIDE (STRIDE)
#else
#define K3F_STRIDE 8
#endif
#ifdef NSH
#define K3F_NSH (NSH)
#else
#define K3F_NSH 7168
#endif

namespace k3 {
namespace dropin {
constexpr int F_EXPERTS = K3F_EXPERTS, F_LDS = K3F_LDS, F_SH = K3F_SH, F_STRIDE = K3F_STRIDE, F_NSH = K3F_NSH;
constexpr int F_LOCAL = F_EXPERTS / F_STRIDE;  // this rank's experts
constexpr int F_TILE = 16, F_MAX_ROWS = 64;
// CTAs of the tables: ceil(rows / F_TILE) an expert, at most one partial CTA a local expert
constexpr int F_MAX_CTAS = F_LOCAL + F_MAX_ROWS * TOPK / F_TILE;
constexpr int F_READERS = F_NSH / 64;           // shared-expert blocks
constexpr int F_THREADS = 1024, F_WORKERS = F_THREADS - 32;
constexpr int F_SORT_WARPS = F_EXPERTS / 32;    // an expert a thread
constexpr int F_QUANT_WARPS = LATENT / 8 / 32;  // 8 latent columns a thread
constexpr int F_RANK_WARPS = F_SORT_WARPS - F_QUANT_WARPS;
constexpr int F_SITU_THREADS = F_SH / 4;        // 4 shared columns a thread
constexpr int F_ATOM_COL = 64 * 128;            // 64 rows of 128-byte swizzle atoms
constexpr int F_OPERAND = F_SH / 64 * F_ATOM_COL;
constexpr int F_SMEM = 1024 + 2 * F_OPERAND + 64 * 64 * 2;
// a row block's scratch in the dynamic shared memory: sigmoids, candidate keys and experts, warp maxima, picks,
// the candidate count, per-warp counts, then the tables' expert masks, CTA offsets and CTA limits
static_assert((3 * F_EXPERTS + 32 + 16 + 16 + 32) * 4 + F_LOCAL * 8 + (F_LOCAL + 1 + F_MAX_CTAS) * 4 <= F_SMEM,
              "a row block's scratch fits the dynamic shared memory");
constexpr int F_EPI_WARPS = F_WORKERS / 128 * 4;  // warps moving accumulator tiles out (whole lane quarters)
constexpr long long F_FC1_W = 2LL * 3072 * (LATENT / 2), F_FC1_SF = 2LL * 3072 * (LATENT / 32);
constexpr int F_ERR = 1 << 30, F_COUNT = 0xffff;
constexpr u64 F_WAIT_NS = 2000000000ull;
static_assert(F_EXPERTS % 32 == 0 && F_EXPERTS / 32 <= TOPK_MAX_EPL && F_EXPERTS % F_STRIDE == 0, "router shape");
static_assert(F_LOCAL <= F_THREADS - F_SORT_WARPS * 32 && F_MAX_ROWS * TOPK <= F_THREADS,
              "an expert mask a SiTU thread to zero, one pick a thread");
static_assert(F_MAX_ROWS <= 64, "an expert's picking rows fit a 64-bit mask");
static_assert(F_SORT_WARPS % 4 == 0, "warp maxima read four at a time");

// Up to this many rows every shared-expert block computes the SiTU rows itself instead of waiting for the row
// blocks' flags
// (16 rows, two chunks a thread, was slower from 8 rows up: 7.66 -> 8.55 us at 16 rows, the extra S reads
// costing more than the flag wait they save)
constexpr int F_LOCAL_SITU_ROWS = 8;
constexpr int F_ACT_CHUNKS = (F_LOCAL_SITU_ROWS * (F_SH / 8) + F_WORKERS - 1) / F_WORKERS;  // a thread
static_assert(F_ACT_CHUNKS <= 2, "at most two act chunks a thread");
static_assert(F_RANK_WARPS >= 2 && F_SORT_WARPS <= 31 && F_SORT_WARPS >= TOPK,
              "ranking warps, a warp left for the SiTU, at least TOPK warp maxima");
static_assert(F_SH % 64 == 0 && F_NSH % 64 == 0 && F_LDS % 4 == 0, "whole swizzle atoms, 16-byte rows");
static_assert(F_READERS <= F_WORKERS && (F_FC1_W / F_READERS) % 16 == 0 && (F_FC1_SF / F_READERS) % 16 == 0,
              "16-byte prefetch shares");
}  // namespace dropin

__device__ __forceinline__ u32 dynamic_smem_size() {
  u32 r;
  asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
  return r;
}
__device__ __forceinline__ int ld_acquire_i32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_relaxed_i32(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_i32(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_i32(int* p, int v) {
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int r;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(r) : "l"(p), "r"(v) : "memory");
  return r;
}
// Wait (bounded) for *flag != 0; returns the value, 0 when the limit passed first.
template <bool ACQUIRE>
__device__ __forceinline__ int wait_nonzero(const int* flag) {
  int v = ACQUIRE ? ld_acquire_i32(flag) : ld_relaxed_i32(flag);
  if (v != 0) return v;
  const u64 t0 = globaltimer_ns();
  while ((v = ACQUIRE ? ld_acquire_i32(flag) : ld_relaxed_i32(flag)) == 0) {
    if (globaltimer_ns() - t0 > dropin::F_WAIT_NS) return 0;
    __nanosleep(128);
  }
  return v;
}

// Two SiTU outputs as a bf16 pair: gate and up landed to bf16 first (the decode front's rounding sequence)
__device__ __forceinline__ u32 situ_bf16x2(float g_lo, float g_hi, float u_lo, float u_hi) {
  const float2 g = bf16x2_to_f2(f2_to_bf16x2(g_lo, g_hi)), u = bf16x2_to_f2(f2_to_bf16x2(u_lo, u_hi));
  return f2_to_bf16x2(situ_front(g.x, u.x), situ_front(g.y, u.y));
}

// Byte offset of row r's 16-byte chunk k (8 bf16) in a K-major operand of 128-byte swizzle atoms, 64-row
// atom columns 8 KB apart (the tensor core's SWIZZLE_128B pattern: chunk index XOR row mod 8).
__device__ __forceinline__ u32 front_swizzle(int r, int k) {
  return (u32)((k >> 3) * dropin::F_ATOM_COL + r * 128 + (((k & 7) ^ (r & 7)) << 4));
}
// kind::f16 instruction descriptor: f32 accumulator, bf16 A and B, both K-major, M x N
__device__ __forceinline__ u32 idesc_bf16(int m, int n) {
  return 1u << 4 | 1u << 7 | 1u << 10 | (u32)(n >> 3) << 17 | (u32)(m >> 4) << 24;
}
__device__ __forceinline__ void mma_bf16(u32 d_tmem, u64 adesc, u64 bdesc, u32 idesc, u32 accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 8 consecutive columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld8(u32 taddr, u32 (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void front_work_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(dropin::F_WORKERS) : "memory");
}

// The last row block's routing tables over the T x 16 picks, thread i the pick i = row * 16 + k.  An
// expert's rows are kept as a 64-bit mask of the picking rows (T <= 64; a row picks an expert at most once),
// so its count is a popcount and a pick's slot within the expert is the number of picking rows before its
// own: an expert's rows come in token order.  Scratch in the (otherwise unused) dynamic shared memory, the
// masks zeroed by the caller.
__device__ __forceinline__ void front_tables(const int* __restrict__ idx, int first, int T, u64* __restrict__ scratch,
                                             int* __restrict__ cta_batch, int* __restrict__ cta_limit,
                                             int* __restrict__ num_non_exiting, int* __restrict__ total_padded,
                                             int* __restrict__ route_map, int* __restrict__ exp2perm, int own_row,
                                             const int* __restrict__ own_picks) {
  using namespace dropin;
  u64* rows = scratch;                                   // [F_LOCAL] the rows picking each expert
  int* off = reinterpret_cast<int*>(rows + F_LOCAL);     // [F_LOCAL + 1] first CTA of each expert
  int* clim = off + F_LOCAL + 1;                         // [F_MAX_CTAS] end of each CTA's real rows
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31, r = t / TOPK;
  int j = -1;
  if (t < T * TOPK) {
    // this block's own row from shared memory; the others' from L2, where their blocks stored them before
    // counting in
    const int d = (r == own_row ? own_picks[t - r * TOPK] : __ldcg(idx + t)) - first;
    if (d >= 0 && d % F_STRIDE == 0 && d / F_STRIDE < F_LOCAL) j = d / F_STRIDE;
  }
  if (j >= 0) atomicOr(rows + j, 1ull << r);  // rows[] zeroed by the caller before its last barrier
  __syncthreads();
  if (warp == 0) {  // off: exclusive scan of the experts' CTA counts, EPL consecutive experts a lane
    constexpr int EPL = (F_LOCAL + 31) / 32;
    int ctas[EPL], sum = 0;
#pragma unroll
    for (int k = 0; k < EPL; ++k) {
      const int e = lane * EPL + k;
      ctas[k] = e < F_LOCAL ? (__popcll(rows[e]) + F_TILE - 1) / F_TILE : 0;
      sum += ctas[k];
    }
    int incl = sum;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    int run = incl - sum;
#pragma unroll
    for (int k = 0; k < EPL; ++k) {
      const int e = lane * EPL + k;
      if (e < F_LOCAL) off[e] = run;
      run += ctas[k];
    }
    if (lane == 31) {
      off[F_LOCAL] = incl;
      num_non_exiting[0] = incl;
      total_padded[0] = incl * F_TILE;
    }
  }
  __syncthreads();
  if (t < F_LOCAL) {
    const int o0 = off[t], o1 = off[t + 1], lim = o0 * F_TILE + __popcll(rows[t]);
    for (int c = o0; c < o1; ++c) {
      const int l = min((c + 1) * F_TILE, lim);
      cta_batch[c] = t;
      cta_limit[c] = l;
      clim[c] = l;
    }
  }
  if (t < T * TOPK) {
    int row = -1;
    if (j >= 0) {
      row = off[j] * F_TILE + __popcll(rows[j] & ((1ull << r) - 1ull));
      route_map[row] = r;
    }
    exp2perm[t] = row;
  }
  __syncthreads();
  // the padding rows (route token 0), one a thread over all CTAs' slots
  for (int i = t; i < off[F_LOCAL] * F_TILE; i += blockDim.x)
    if (i >= clim[i / F_TILE]) route_map[i] = 0;
}

// Warp 31 of shared-expert block c: the rows' lowest local picks (clearing their flags), then this block's
// share of the two least touched experts' FC1 weights and scales (the reference's FC1 layout: expert e's
// [2 x 3072, LATENT] packed MXFP4 at e * F_FC1_W) into L2.
__device__ __forceinline__ void front_prefetch(int* __restrict__ ids, int* __restrict__ done, int T, int c,
                                               const uint8_t* __restrict__ w13, const uint8_t* __restrict__ w13_sf) {
  using namespace dropin;
  const int lane = threadIdx.x & 31;
  int a = F_LOCAL, a2 = F_LOCAL;  // this lane's two least distinct local experts
  bool ok = true;
  for (int r = lane; r < T; r += 32) {
    int* flag = ids + c * 64 + r;
    const int v = wait_nonzero<false>(flag);
    if (v == 0) {
      ok = false;
      continue;
    }
    *flag = 0;
    const int two[2] = {(v - 1) % 256, (v - 1) / 256};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int x = two[h];
      if (x == a || x == a2) continue;
      if (x < a) {
        a2 = a;
        a = x;
      } else if (x < a2) {
        a2 = x;
      }
    }
  }
  if (!__all_sync(0xffffffffu, ok)) {
    if (lane == 0) atomicOr(done, F_ERR);
    return;
  }
  const int j = __reduce_min_sync(0xffffffffu, a);
  const int k = __reduce_min_sync(0xffffffffu, a == j ? a2 : a);
  if (lane < 2) {
    const int e = lane ? k : j;
    if (e < F_LOCAL) {
      bulk_prefetch(w13 + e * F_FC1_W + c * (F_FC1_W / F_READERS), (u32)(F_FC1_W / F_READERS));
      bulk_prefetch(w13_sf + e * F_FC1_SF + c * (F_FC1_SF / F_READERS), (u32)(F_FC1_SF / F_READERS));
    }
  }
}

}  // namespace k3

extern "C" __global__ void __launch_bounds__(dropin::F_THREADS, 1) kern_k3_moe_front(
    const float* __restrict__ S, const float* __restrict__ bias, const bf16* __restrict__ rs, int* __restrict__ idx,
    float* __restrict__ wts, uint8_t* __restrict__ q, uint8_t* __restrict__ sf, bf16* __restrict__ act,
    int* __restrict__ ready, int* __restrict__ ids, int* __restrict__ done, int* __restrict__ cta_batch,
    int* __restrict__ cta_limit, int* __restrict__ num_non_exiting, int* __restrict__ total_padded,
    int* __restrict__ route_map, int* __restrict__ exp2perm, const bf16* __restrict__ wsh, bf16* __restrict__ sh_out,
    const uint8_t* __restrict__ w13, const uint8_t* __restrict__ w13_sf, int first, int T) {
  using namespace k3::dropin;
  extern __shared__ __align__(16) uint8_t f_dyn[];
  __shared__ int s_last, s_fail;
  __shared__ u32 s_tmem;
  __shared__ __align__(8) u64 s_bar;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  const int b = blockIdx.x, t = threadIdx.x, warp = t >> 5, lane = t & 31;
  if (T < 1 || T > F_MAX_ROWS || dynamic_smem_size() < (u32)F_SMEM) {  // a launch outside the contract
    if (b == 0 && t == 0) atomicOr(done, F_ERR);
    return;
  }

  if (b < T) {
    // ---------------------------------------------------------------- row block b
    // Warps [0, F_SORT_WARPS) hold one expert a thread: sigmoid, key, the warp maxima; tau (the 16th largest
    // warp maximum, computed by every warp alike) bounds the top 16 from below, so only keys >= tau are
    // candidates; they are compacted into shared memory and ranked in parallel (a warp a candidate, its
    // lanes counting the candidates ahead of it), the ranks < 16 giving the picks in order.  The latent's
    // MXFP8 runs on warps [F_RANK_WARPS, F_SORT_WARPS) meanwhile, the SiTU on the remaining warps from the
    // start.
    const float* row = S + (long long)b * F_LDS;
    float* s_sig = reinterpret_cast<float*>(f_dyn);                 // [F_EXPERTS]
    u32* c_key = reinterpret_cast<u32*>(s_sig + F_EXPERTS);         // candidates [F_EXPERTS]
    int* c_e = reinterpret_cast<int*>(c_key + F_EXPERTS);           // [F_EXPERTS]
    u32* s_wmax = reinterpret_cast<u32*>(c_e + F_EXPERTS);          // [32]
    int* s_pick = reinterpret_cast<int*>(s_wmax + 32);              // [TOPK]
    int* s_n = s_pick + TOPK;                                       // [1] candidates
    int* s_ccnt = s_n + 16;                                         // [32] candidates a warp (16-byte aligned)
    u64* table_scratch = reinterpret_cast<u64*>(s_ccnt + 32);
    if (warp < F_SORT_WARPS) {
      // the latent's loads in flight from the start (quantised after the ranking)
      float4 lat_lo = make_float4(0.f, 0.f, 0.f, 0.f), lat_hi = lat_lo;
      const int u = t - F_RANK_WARPS * 32;
      if (warp >= F_RANK_WARPS) {
        lat_lo = reinterpret_cast<const float4*>(row + F_EXPERTS)[2 * u];
        lat_hi = reinterpret_cast<const float4*>(row + F_EXPERTS)[2 * u + 1];
      }
      const float rsv = __bfloat162float(rs[0]);
      const float sg = router_sigmoid(row[t]);
      const u32 key = ord_f32(sg + bias[t]);
      s_sig[t] = sg;
      const u32 m = __reduce_max_sync(0xffffffffu, key);
      if (lane == 0) s_wmax[warp] = m;
      asm volatile("bar.sync 2, %0;" ::"n"(F_SORT_WARPS * 32) : "memory");
      // tau: lane l ranks warp l's maximum among all of them (ties by warp index); rank TOPK - 1 is tau
      const u32 wm = lane < F_SORT_WARPS ? s_wmax[lane] : 0u;
      int wrank = 0;
#pragma unroll
      for (int q4 = 0; q4 < F_SORT_WARPS / 4; ++q4) {
        const uint4 m4 = reinterpret_cast<const uint4*>(s_wmax)[q4];
        const u32 mq[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) wrank += (mq[h] > wm) | ((mq[h] == wm) & (4 * q4 + h < lane));
      }
      const u32 tau = __shfl_sync(0xffffffffu, wm, __ffs(__ballot_sync(0xffffffffu, wrank == TOPK - 1)) - 1);
      // the candidates compacted in warp order: a warp's slots start after the lower warps' candidates
      const bool cand = key >= tau;
      const u32 bal = __ballot_sync(0xffffffffu, cand);
      if (lane == 0) s_ccnt[warp] = __popc(bal);
      asm volatile("bar.sync 2, %0;" ::"n"(F_SORT_WARPS * 32) : "memory");
      int base = 0;
#pragma unroll
      for (int q4 = 0; q4 < F_SORT_WARPS / 4; ++q4) {
        const int4 c4 = reinterpret_cast<const int4*>(s_ccnt)[q4];
        base += (4 * q4 < warp ? c4.x : 0) + (4 * q4 + 1 < warp ? c4.y : 0) + (4 * q4 + 2 < warp ? c4.z : 0) +
                (4 * q4 + 3 < warp ? c4.w : 0);
      }
      if (cand) {
        const int at = base + __popc(bal & ((1u << lane) - 1u));
        c_key[at] = key;
        c_e[at] = t;
      }
      if (warp == F_SORT_WARPS - 1 && lane == 0) *s_n = base + __popc(bal);
      asm volatile("bar.sync 2, %0;" ::"n"(F_SORT_WARPS * 32) : "memory");
      {
        // candidate i's rank: the candidates with a larger key, or the same key and a smaller expert
        const int n = *s_n;
        for (int i = warp; i < n; i += F_SORT_WARPS) {
          const u32 ki = c_key[i];
          const int ei = c_e[i];
          int ahead = 0;
          for (int qq = lane; qq < n; qq += 32) {
            const u32 kq = c_key[qq];
            ahead += (kq > ki) | ((kq == ki) & (c_e[qq] < ei));
          }
          ahead = __reduce_add_sync(0xffffffffu, ahead);
          if (lane == 0 && ahead < TOPK) s_pick[ahead] = ei;
        }
      }
      asm volatile("bar.sync 2, %0;" ::"n"(F_SORT_WARPS * 32) : "memory");
      if (warp == 0) {
        const int pick = lane < TOPK ? s_pick[lane] : 0;
        // the row's two lowest local picks, to every shared-expert block's prefetcher (which the launch's
        // end waits for), first
        const int d = pick - first;
        const int mine = lane < TOPK && d >= 0 && d % F_STRIDE == 0 ? d / F_STRIDE : F_LOCAL;
        const int j = __reduce_min_sync(0xffffffffu, mine);
        const int j2 = __reduce_min_sync(0xffffffffu, mine == j ? F_LOCAL : mine);
        for (int c = lane; c < F_READERS; c += 32) st_relaxed_i32(ids + c * 64 + b, 1 + j + 256 * j2);
        if (lane < TOPK) idx[(long long)b * TOPK + lane] = pick;
        // warp 1 counts the row in once the picks are stored; this warp goes on with the weights
        asm volatile("bar.arrive 4, 64;" ::: "memory");
        const float w = lane < TOPK ? s_sig[pick] : 0.f;
        float den = w;
#pragma unroll
        for (int off = TOPK / 2; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
        if (lane < TOPK) wts[(long long)b * TOPK + lane] = (w / (den + 1e-20f)) * rsv;
      } else if (warp == 1) {
        asm volatile("bar.sync 4, 64;" ::: "memory");
        if (lane == 0) {  // the row's picks are out: count it in (release them, acquire the other rows')
          const int n = atom_add_acq_rel(done, 1);
          s_last = (n & F_COUNT) == T - 1;
        }
      } else if (warp >= F_RANK_WARPS) {
        // the latent: 8 columns a thread (four threads a 32-column group), landed to bf16, then MXFP8
        const uint4 lv = make_uint4(f2_to_bf16x2(lat_lo.x, lat_lo.y), f2_to_bf16x2(lat_lo.z, lat_lo.w),
                                    f2_to_bf16x2(lat_hi.x, lat_hi.y), f2_to_bf16x2(lat_hi.z, lat_hi.w));
        int sfb;
        const uint2 w = quant8_lanes(lv, sfb);
        reinterpret_cast<uint2*>(q + (long long)b * LATENT)[u] = w;
        if ((u & 3) == 0) sf[(long long)b * (LATENT / 32) + (u >> 2)] = (uint8_t)sfb;
      }
    } else {
      // the shared expert's SiTU, 4 columns a thread, gate and up landed to bf16 first; every pass's loads
      // in flight before the first is used
      constexpr int LANES = F_THREADS - F_SORT_WARPS * 32, PASSES = (F_SITU_THREADS + LANES - 1) / LANES;
      const int k0 = t - F_SORT_WARPS * 32;
      float4 g[PASSES], u[PASSES];
#pragma unroll
      for (int p = 0; p < PASSES; ++p)
        if (k0 + p * LANES < F_SITU_THREADS) {
          g[p] = reinterpret_cast<const float4*>(row + F_EXPERTS + LATENT)[k0 + p * LANES];
          u[p] = reinterpret_cast<const float4*>(row + F_EXPERTS + LATENT + F_SH)[k0 + p * LANES];
        }
#pragma unroll
      for (int p = 0; p < PASSES; ++p)
        if (k0 + p * LANES < F_SITU_THREADS)
          reinterpret_cast<uint2*>(act + (long long)b * F_SH)[k0 + p * LANES] =
              make_uint2(situ_bf16x2(g[p].x, g[p].y, u[p].x, u[p].y), situ_bf16x2(g[p].z, g[p].w, u[p].z, u[p].w));
      if (k0 < F_LOCAL) table_scratch[k0] = 0ull;  // the tables' expert masks, should this block be the last
      // the row is in: one flag to each shared-expert block (a release after the barrier: cumulative over
      // the SiTU warps' stores), unless those blocks compute the rows themselves
      if (T > F_LOCAL_SITU_ROWS) {
        asm volatile("bar.sync 3, %0;" ::"n"(LANES) : "memory");
        for (int c = k0; c < F_READERS; c += LANES) st_release_i32(ready + c * 64 + b, 1);
      }
    }
    __syncthreads();
    if (!s_last) return;
    front_tables(idx, first, T, table_scratch, cta_batch, cta_limit, num_non_exiting, total_padded,
                 route_map, exp2perm, b, s_pick);
    __syncthreads();
    if (t == 0) atomicAnd(done, F_ERR);  // the count back to zero, a recorded error kept
    return;
  }

  // ------------------------------------------------------------------ block T + c: shared down projection
  const int c = b - T, n0 = c * 64;
  if (warp == 31) {
    front_prefetch(ids, done, T, c, w13, w13_sf);
    return;
  }
  uint8_t* sw = f_dyn + ((1024u - (smem_u32(f_dyn) & 1023u)) & 1023u);  // Wsh rows, 1 KB aligned
  uint8_t* sa = sw + F_OPERAND;                                       // the T act rows
  bf16* tile = reinterpret_cast<bf16*>(sa + F_OPERAND);               // out [T][64]
  const u32 sw_at = smem_u32(sw), sa_at = smem_u32(sa);
  // Few rows: every block computes the act rows itself from the front GEMM's gate | up (bit for bit as the
  // row blocks do), 8-column chunks (t + m F_WORKERS), their loads in flight before anything else
  const bool local_act = T <= F_LOCAL_SITU_ROWS;
  float4 g0[F_ACT_CHUNKS], g1[F_ACT_CHUNKS], u0[F_ACT_CHUNKS], u1[F_ACT_CHUNKS];
#pragma unroll
  for (int m = 0; m < F_ACT_CHUNKS; ++m) {
    const int i = t + m * F_WORKERS, ar = i / (F_SH / 8), ak = i % (F_SH / 8);
    g0[m] = g1[m] = u0[m] = u1[m] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (local_act && i < T * (F_SH / 8)) {
      const float* gp = S + (long long)ar * F_LDS + F_EXPERTS + LATENT + ak * 8;
      g0[m] = reinterpret_cast<const float4*>(gp)[0];
      g1[m] = reinterpret_cast<const float4*>(gp)[1];
      u0[m] = reinterpret_cast<const float4*>(gp + F_SH)[0];
      u1[m] = reinterpret_cast<const float4*>(gp + F_SH)[1];
    }
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, 64);
    tmem_relinquish();
  }
  // Wsh's 64 rows (one contiguous 96 KB run) go straight into the swizzled operand, 16 bytes a cp.async, in
  // flight with the act rows' loads.  (Staging them with one bulk copy and swizzling them in shared memory was
  // 0.6 us slower a launch at 8 rows.)
  for (int i = t; i < 64 * (F_SH / 8); i += F_WORKERS) {
    const int r = i / (F_SH / 8), k = i % (F_SH / 8);
    cp_async16(sw_at + front_swizzle(r, k), wsh + (long long)(n0 + r) * F_SH + k * 8);
  }
  if (t == 0) {
    s_fail = 0;
    mbar_init(&s_bar, 1);
    fence_mbar_init();
  }
  front_work_sync();
  if (local_act) {
#pragma unroll
    for (int m = 0; m < F_ACT_CHUNKS; ++m) {
      const int i = t + m * F_WORKERS, ar = i / (F_SH / 8), ak = i % (F_SH / 8);
      if (i < T * (F_SH / 8))
        *reinterpret_cast<uint4*>(sa + front_swizzle(ar, ak)) =
            make_uint4(situ_bf16x2(g0[m].x, g0[m].y, u0[m].x, u0[m].y), situ_bf16x2(g0[m].z, g0[m].w, u0[m].z, u0[m].w),
                       situ_bf16x2(g1[m].x, g1[m].y, u1[m].x, u1[m].y), situ_bf16x2(g1[m].z, g1[m].w, u1[m].z, u1[m].w));
    }
    cp_async_wait_all();
  } else {
    if (t < T) {
      int* flag = ready + c * 64 + t;
      if (wait_nonzero<true>(flag) != 0) {
        *flag = 0;
      } else {
        s_fail = 1;
        atomicOr(done, F_ERR);
      }
    }
    front_work_sync();
    if (!*reinterpret_cast<volatile int*>(&s_fail))
      for (int i = t; i < T * (F_SH / 8); i += F_WORKERS) {
        const int r = i / (F_SH / 8), k = i % (F_SH / 8);
        cp_async16(sa_at + front_swizzle(r, k), act + (long long)r * F_SH + k * 8);
      }
    cp_async_wait_all();
  }
  fence_proxy_async_shared();  // both operands (generic-proxy writes), to the tensor core's reads
  tc_fence_before();
  front_work_sync();
  tc_fence_after();
  const bool fail = *reinterpret_cast<volatile int*>(&s_fail) != 0;
  const int tiles = (T + 7) / 8;
  if (!fail) {
    if (t == 0) {
      const u32 idesc = idesc_bf16(64, tiles * 8);
      for (int s = 0; s < F_SH / 16; ++s) {  // K in 16-element steps, one accumulation chain in order
        const u32 off = (u32)((s >> 2) * F_ATOM_COL + (s & 3) * 32);
        mma_bf16(s_tmem, sdesc_k_sw128(sw_at + off), sdesc_k_sw128(sa_at + off), idesc, s > 0 ? 1u : 0u);
      }
      tc_commit(&s_bar);
    }
    __syncwarp();
    if (warp < F_EPI_WARPS && mbar_wait(&s_bar, 0, nullptr, nullptr, 0, F_WAIT_NS)) {
      tc_fence_after();
      // M = 64: accumulator row m (output column n0 + m) sits in lane 32 (m / 16) + m % 16, column = token
      const int quarter = warp & 3;
      for (int j = warp >> 2; j < tiles; j += F_EPI_WARPS / 4) {
        u32 v[8];
        tmem_ld8(s_tmem + ((u32)(32 * quarter) << 16) + 8 * j, v);
        tmem_wait_ld();
        if (lane < 16)
#pragma unroll
          for (int i = 0; i < 8; ++i)
            tile[(8 * j + i) * 64 + 16 * quarter + lane] = __float2bfloat16(__uint_as_float(v[i]));
      }
    }
  }
  tc_fence_before();
  cp_async_wait_all();  // nothing of this block's in flight past here
  front_work_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(s_tmem, 64);
  }
  if (!*reinterpret_cast<volatile int*>(&s_fail))
    for (int i = t; i < T * 8; i += F_WORKERS) {
      const int r = i >> 3, col = i & 7;
      reinterpret_cast<uint4*>(sh_out + (long long)r * F_NSH + n0)[col] = reinterpret_cast<const uint4*>(tile + r * 64)[col];
    }
}
