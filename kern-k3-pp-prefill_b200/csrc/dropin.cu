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
//   kern_k3_moe_route_count     source/k3_moe_prefill.cu:97   grid ceil(T/256), block 256
//   kern_k3_moe_route_tables    source/k3_moe_prefill.cu:115  grid 1, block 1024
//   kern_k3_moe_route_scatter   source/k3_moe_prefill.cu:155  grid ceil(T/256), block 256
//   kern_k3_moe_finalize        source/k3_moe_prefill.cu:206  grid rows, any block
//   kern_k3g_finalize_rms       source/k3_prefill_glue.cu:573 grid rows, block cols/8
//   kern_k3g_moe_finalize_rms   source/k3_moe_route.cu:538    grid rows, block 448
//   kern_k3g_moe_route          source/k3_moe_route.cu:338    grid 64 (B <= 256) or 288, block 512 (grid barrier)
//   kern_k3g_moe_route_init     source/k3_moe_route.cu:522    any grid, block 1024
//   kern_k3_moe_w_shuffle       source/k3_moe_prefill.cu:242  grid ceil(experts*n*row_bytes/16/block)
//   kern_k3_moe_sf_shuffle      source/k3_moe_prefill.cu:252  grid ceil(experts*n*kg/block)
#include "common.cuh"

namespace k3 {
namespace dropin {
constexpr int TOPK = 16;
constexpr int EXPERTS = 896;
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
  topk_warp<dropin::EXPERTS / 32>(S + (long long)b * dropin::EXPERTS, bias, dropin::EXPERTS, dropin::TOPK,
                                  __bfloat162float(rs[0]), threadIdx.x & 31, ck[warp], ce[warp],
                                  idx + (long long)b * dropin::TOPK, wts + (long long)b * dropin::TOPK);
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
constexpr int TABLE = EXPERTS * (1 + CHUNKS + WORDS);
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
__device__ __forceinline__ float ex2_approx_ftz(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// The shared expert's activation as the reference's fused front computes it (source/k3_moe_route.cu:257-269,
// k3_prefill_glue.cu's kern_k3g_situ): e^-g as ex2.approx.ftz(g * -log2 e), the sigmoid an IEEE reciprocal,
// the tanh terms tanh.approx, every product and sum rounded on its own: (4 tanh(g/4) * sigmoid(g)) * 25 tanh(u/25).
__device__ __forceinline__ float situ_front(float g, float u) {
  const float d = __fadd_rn(ex2_approx_ftz(__fmul_rn(g, -1.44269502f)), 1.0f);
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
  __shared__ int s_cnt[EXPERTS], s_off[EXPERTS];
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
  int* chunk = tot + EXPERTS;
  u32* bits = cur + EXPERTS * (1 + CHUNKS);
  for (int i = gt; i < TABLE; i += nthreads) nxt[i] = 0u;  // the next call's table

  // ---- phase 1a: a warp a row: top-16, marked in this call's table
  const float rsv = __bfloat162float(rs[0]);
  for (int b = gwarp; b < B; b += nwarps) {
    const int e = topk_warp<EXPERTS / 32>(S + (long long)b * EXPERTS, bias, EXPERTS, TOPK, rsv, lane, s_ck[warp],
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
  if (2 * t < EXPERTS) {
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
  if (2 * t < EXPERTS) {
    s_off[2 * t] = before + incl - c0 - c1;
    s_off[2 * t + 1] = before + incl - c1;
  }
  __syncthreads();
  if (gt == 0) {
    num_non_exiting[0] = total;
    total_padded[0] = total * tile;
  }
  for (int e = gt; e < EXPERTS; e += nthreads) {
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
