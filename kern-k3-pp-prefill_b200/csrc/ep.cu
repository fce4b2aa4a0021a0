// Expert-parallel data movement kernels: pack routed rows for the all-to-all
// dispatch, unpack received rows into the GEMMs' permuted operand, and the
// owner-side combine.  (The reference has no MoE all-to-all: its decode EP
// replicates the batch and all-reduces, roofline/decode.md:164-166; this is the
// token-sharded layout of the benchmark configurations.)
//
// Packed row (dispatch wire format), `stride` = roundup(H + H/32 + 4, 16) bytes:
//   [0, H)            E4M3 elements (MXFP8, the rule of k3moe_quant_mxfp8)
//   [H, H + H/32)     UE8M0 scale per 32 elements, linear
//   [H + H/32, +4)    local expert id at the destination (int32)
//   the rest          unused (rows stay 16-byte aligned)
#include "common.cuh"

namespace k3 {

// `split` warps a source row, each a contiguous share of its 256-column pieces: quantise the row once and
// write it to each of its destination slots: slot send_pos[t*K + k] with id idx[t*K + k] - dest*E_local
// (dest = idx / E_local), or, with send_pos null, slot t with id `fixed_eid`.  (A decode step has a few
// dozen rows: several warps a row keep more of the GPU busy.)
__global__ void __launch_bounds__(256) ep_pack_kernel(const bf16* __restrict__ x, int ldx, int T, int H, int K,
                                                      const int* __restrict__ idx, const int* __restrict__ send_pos,
                                                      int E_local, int fixed_eid, uint8_t* __restrict__ dst,
                                                      int stride, int split) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int pieces = H / 256, share = (pieces + split - 1) / split;
  for (int g = blockIdx.x * warps + (threadIdx.x >> 5); g < T * split; g += gridDim.x * warps) {
    const int t = g / split, part = g - t * split;
    long long pos[16];
    int eid[16];
    int nd = 0;
    if (send_pos) {
      for (int k = 0; k < K; ++k) {
        const int p = send_pos[(long long)t * K + k];
        if (p < 0) continue;
        const int g = idx[(long long)t * K + k];
        pos[nd] = p;
        eid[nd] = g % E_local;
        ++nd;
      }
    } else {
      pos[0] = t;
      eid[0] = fixed_eid;
      nd = 1;
    }
    const bf16* xr = x + (long long)t * ldx;
    const int c_end = min(H, (part + 1) * share * 256);
    for (int c0 = part * share * 256; c0 < c_end; c0 += 256) {
      const int c = c0 + lane * 8;
      const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
      int sfb;
      const uint2 w = quant8_lanes(u, sfb);
      const int kb = c / 32;
      u32 sfw = (u32)sfb << (8 * (kb & 3));
      sfw |= __shfl_down_sync(0xffffffffu, sfw, 4);
      sfw |= __shfl_down_sync(0xffffffffu, sfw, 8);
      for (int d = 0; d < nd; ++d) {
        uint8_t* row = dst + pos[d] * stride;
        *reinterpret_cast<uint2*>(row + c) = w;
        if ((lane & 15) == 0) *reinterpret_cast<u32*>(row + H + kb) = sfw;
      }
    }
    if (part == 0 && lane < nd) *reinterpret_cast<int*>(dst + pos[lane] * stride + H + H / 32) = eid[lane];
  }
}

// ids[i] = the local expert id field of packed row i
__global__ void __launch_bounds__(256) ep_ids_kernel(const uint8_t* __restrict__ rows, int stride, int R, int H,
                                                     int* __restrict__ ids) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < R; i += gridDim.x * blockDim.x)
    ids[i] = *reinterpret_cast<const int*>(rows + (long long)i * stride + H + H / 32);
}

// Packed row i -> permuted row perm[i] of the tile-major operand (q) and the
// 128x4-tiled scales; rows with perm < 0 are skipped.  One warp a row.
__global__ void __launch_bounds__(256) ep_unpack_kernel(const uint8_t* __restrict__ rows, int stride, int R, int H,
                                                        const int* __restrict__ perm, uint8_t* __restrict__ qp,
                                                        uint8_t* __restrict__ sfp) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int kg4 = H / 128;
  for (int i = blockIdx.x * warps + (threadIdx.x >> 5); i < R; i += gridDim.x * warps) {
    const int p = perm[i];
    if (p < 0) continue;
    const uint8_t* row = rows + (long long)i * stride;
    // 16 bytes a lane: 8 lanes a 128-byte tile row, 4 tile rows a step
    for (int c = lane * 16; c < H; c += 512)
      *reinterpret_cast<uint4*>(qp + op8_offset(p, c, H)) = *reinterpret_cast<const uint4*>(row + c);
    // 4 scale bytes (4 consecutive groups) are one u32 of the tiled atom row
    for (int g = lane; g < H / 128; g += 32)
      *reinterpret_cast<u32*>(sfp + sf_tiled_offset(p, 4 * g, kg4)) = *reinterpret_cast<const u32*>(row + H + 4 * g);
  }
}

// out[t] = bf16( sum_{k, pos>=0} fma(w[t,k], back[pos[t,k]], acc) (+ shared[t]) ), f32, k in order:
// the single-GPU combine's arithmetic, over rows returned by the combine all-to-all.
__global__ void __launch_bounds__(256) combine_ep_kernel(const bf16* __restrict__ back, const int* __restrict__ pos,
                                                         const float* __restrict__ wts,
                                                         const bf16* __restrict__ shared_rows, int ld_shared,
                                                         bf16* __restrict__ out, int ldo, int T, int K, int cols) {
  __shared__ int sp[16];
  __shared__ float sw[16];
  const int t = blockIdx.x;
  if (threadIdx.x < K) {
    sp[threadIdx.x] = pos[(long long)t * K + threadIdx.x];
    sw[threadIdx.x] = wts[(long long)t * K + threadIdx.x];
  }
  __syncthreads();
  for (int h = threadIdx.x; h < cols / 8; h += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < K; ++k) {
      const int p = sp[k];
      if (p < 0) continue;
      const float w = sw[k];
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(back + (long long)p * cols) + h);
      const u32* pv = reinterpret_cast<const u32*>(&u);
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const float2 f = bf16x2_to_f2(pv[l]);
        acc[2 * l] = fmaf(w, f.x, acc[2 * l]);
        acc[2 * l + 1] = fmaf(w, f.y, acc[2 * l + 1]);
      }
    }
    if (shared_rows) {
      const uint4 u = *(reinterpret_cast<const uint4*>(shared_rows + (long long)t * ld_shared) + h);
      const u32* pv = reinterpret_cast<const u32*>(&u);
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const float2 f = bf16x2_to_f2(pv[l]);
        acc[2 * l] = fmaf(1.0f, f.x, acc[2 * l]);
        acc[2 * l + 1] = fmaf(1.0f, f.y, acc[2 * l + 1]);
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

}  // namespace k3
