// Drop-in kernel entries: the reference's module entry names, argument lists
// and launch geometry (docs/k3-kernel-abi.md §0 conventions; kernels.toml), so
// a manifest that binds the reference's modules can bind this one instead.
// Every entry computes with this project's own kernels' arithmetic and matches
// the reference entry byte for byte (tests/test_gpu_ref.py).  TOPK is 16 and
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
  const int b = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (b >= B) return;
  topk_warp<dropin::EXPERTS / 32>(S + (long long)b * dropin::EXPERTS, bias, dropin::EXPERTS, dropin::TOPK,
                                  __bfloat162float(rs[0]), threadIdx.x & 31, idx + (long long)b * dropin::TOPK,
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
