// Expert-parallel data movement kernels: pack routed rows for the all-to-all
// dispatch, unpack received rows into the GEMMs' permuted operand, and the
// owner-side combine.  (The reference has no MoE all-to-all: its decode EP
// replicates the batch and all-reduces, roofline/decode.md:164-166; this is the
// token-sharded layout of the benchmark configurations.)
//
// One row a pick (the fixed-block dispatch of decode-sized batches), `stride` = roundup(H + H/32 + 4, 16) bytes:
//   [0, H)            E4M3 elements (MXFP8, the rule of k3moe_quant_mxfp8)
//   [H, H + H/32)     UE8M0 scale per 32 elements, linear
//   [H + H/32, +4)    local expert id at the destination (int32)
//   the rest          unused (rows stay 16-byte aligned)
//
// Per-destination rows (the counts-exchange dispatch): a token is sent once to each rank holding any of its
// picks, stride roundup(H + H/32 + 2 K, 16):
//   [0, H + H/32)     as above
//   [H + H/32, +2K)   the local expert ids (int16) of the token's picks on that rank, in pick order, -1 after
// The receiver routes each row to all its experts; FC2's results go back one row a pick, in (token, pick)
// order, so the owner's combine is unchanged.
#pragma once
#include "common.cuh"

namespace k3 {

constexpr int EP_MAX_RANKS = 16;

// 64-bit bases a rank (or a block of rows), passed by value: the peer-memory transport's destinations.
struct EpBases {
  unsigned long long base[EP_MAX_RANKS + 1];
  long long start[EP_MAX_RANKS + 2];  // row-number ranges [start[s], start[s+1]) of block s
};

// pair_ids[t*W + d] = d when token t has a pick on rank d, else -1 (W <= 64)
__global__ void __launch_bounds__(256) ep_pairs_kernel(const int* __restrict__ dest, int T, int K, int W,
                                                       int* __restrict__ pair_ids) {
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += gridDim.x * blockDim.x) {
    unsigned long long on = 0ull;
    for (int k = 0; k < K; ++k) {
      const int d = dest[(long long)t * K + k];
      if (d >= 0 && d < W) on |= 1ull << d;
    }
    for (int d = 0; d < W; ++d) pair_ids[(long long)t * W + d] = ((on >> d) & 1ull) ? d : -1;
  }
}

// `split` warps a source row: quantise token t once and write it to the slot pair_pos[t*W + d] of every rank d
// it goes to, headed by the local ids of its picks there (lid[t*K + k] where dest[t*K + k] == d, in k order);
// with pair_pos null, slot t headed by `fixed_eid` alone.  Slot p of rank d is row p of dst, or with
// use_bases, the row at bases.base[d] + p * stride (rank d's receive buffer, possibly in another GPU's memory).
// With shared_eid >= 0 (use_bases) the token also goes to slot t of bases.base[W], headed by shared_eid alone
// (the rank's own shared-expert rows).  With pair_back, rank d's row also carries pair_back[t*W + d] (int32) at
// byte back_col: where the results of the token's picks there go back to.  Stores into peer memory are
// ordered at system scope before the kernel ends (a later kernel on the stream signals the peers).
// With tail_bytes > 0 (= stride - H, a multiple of 16) and split 1, each warp builds a row's tail (scales, ids,
// return index, zero padding) in tail_bytes of dynamic shared memory and stores it as 16-byte chunks, whole
// 128-byte lines where the rows are line-aligned, instead of one 4-byte store a scale word and one 2-byte
// store an id: a row bound for another GPU crosses NVLink as full lines only.
__global__ void __launch_bounds__(256) ep_pack_pairs_kernel(const bf16* __restrict__ x, int ldx, int T, int H, int K,
                                                            const int* __restrict__ dest, const int* __restrict__ lid,
                                                            const int* __restrict__ pair_pos, int W, int fixed_eid,
                                                            uint8_t* __restrict__ dst, int stride, int split,
                                                            EpBases bases, int use_bases, int shared_eid = -1,
                                                            const int* __restrict__ pair_back = nullptr,
                                                            int back_col = 0, int tail_bytes = 0) {
  extern __shared__ __align__(16) uint8_t pack_tails[];
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int pieces = H / 256, share = (pieces + split - 1) / split;
  const bool whole_tail = tail_bytes > 0 && split == 1;
  uint8_t* tail = pack_tails + (threadIdx.x >> 5) * tail_bytes;
  for (int g = blockIdx.x * warps + (threadIdx.x >> 5); g < T * split; g += gridDim.x * warps) {
    const int t = g / split, part = g - t * split;
    // lane d < W: rank d's slot for this token (or -1)
    long long my_pos = -1;
    if (pair_pos == nullptr) {
      if (lane == 0) my_pos = t;
    } else if (lane < W) {
      my_pos = pair_pos[(long long)t * W + lane];
    } else if (lane == W && shared_eid >= 0) {
      my_pos = t;
    }
    const unsigned live = __ballot_sync(0xffffffffu, my_pos >= 0);
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
      for (unsigned m = live; m; m &= m - 1) {
        const int d = __ffs(m) - 1;
        const long long pd = __shfl_sync(0xffffffffu, my_pos, d);
        uint8_t* row = (use_bases ? reinterpret_cast<uint8_t*>(bases.base[d]) : dst) + pd * stride;
        *reinterpret_cast<uint2*>(row + c) = w;
        if (!whole_tail && (lane & 15) == 0) *reinterpret_cast<u32*>(row + H + kb) = sfw;
      }
      if (whole_tail && (lane & 15) == 0) *reinterpret_cast<u32*>(tail + kb) = sfw;
    }
    if (whole_tail) {
      // per destination: its ids and return index into the tail image, then the tail out in 16-byte chunks
      for (unsigned m = live; m; m &= m - 1) {
        const int d = __ffs(m) - 1;
        __syncwarp();
        if (lane == d) {
          short* ids = reinterpret_cast<short*>(tail + H / 32);
          int n = 0;
          if (pair_pos == nullptr) {
            ids[n++] = (short)fixed_eid;
          } else if (lane == W) {
            ids[n++] = (short)shared_eid;
          } else {
            for (int k = 0; k < K; ++k)
              if (dest[(long long)t * K + k] == lane) ids[n++] = (short)lid[(long long)t * K + k];
          }
          for (; n < K; ++n) ids[n] = -1;
          for (int b = H / 32 + 2 * K; b < tail_bytes; b += 2) *reinterpret_cast<short*>(tail + b) = 0;
          if (pair_back != nullptr && lane < W)
            *reinterpret_cast<int*>(tail + (back_col - H)) = pair_back[(long long)t * W + lane];
        }
        __syncwarp();
        const long long pd = __shfl_sync(0xffffffffu, my_pos, d);
        uint8_t* row = (use_bases ? reinterpret_cast<uint8_t*>(bases.base[d]) : dst) + pd * stride;
        for (int q = lane; q < tail_bytes / 16; q += 32)
          *reinterpret_cast<uint4*>(row + H + 16 * q) = reinterpret_cast<const uint4*>(tail)[q];
      }
      __syncwarp();
      continue;
    }
    if (part == 0 && my_pos >= 0) {  // lane d writes its rank's id list
      uint8_t* row = (use_bases ? reinterpret_cast<uint8_t*>(bases.base[lane]) : dst) + my_pos * stride;
      short* ids = reinterpret_cast<short*>(row + H + H / 32);
      int n = 0;
      if (pair_pos == nullptr) {
        ids[n++] = (short)fixed_eid;
      } else if (lane == W) {
        ids[n++] = (short)shared_eid;
      } else {
        for (int k = 0; k < K; ++k)
          if (dest[(long long)t * K + k] == lane) ids[n++] = (short)lid[(long long)t * K + k];
        if (pair_back != nullptr) *reinterpret_cast<int*>(row + back_col) = pair_back[(long long)t * W + lane];
      }
      for (; n < K; ++n) ids[n] = -1;
    }
  }
  if (use_bases) __threadfence_system();
}

// ids[i*KH + j] = the j-th local expert id (int16, -1 none) of per-destination row i.  With region_counts, the
// rows come in regions of region_rows rows, region s holding region_counts[s] rows (the rest stale): rows past
// a region's count get no ids.
__global__ void __launch_bounds__(256) ep_ids_k_kernel(const uint8_t* __restrict__ rows, int stride, int R, int H,
                                                       int KH, int* __restrict__ ids,
                                                       const u32* __restrict__ region_counts = nullptr,
                                                       int region_rows = 0) {
  const long long n = (long long)R * KH;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const long long i = e / KH;
    const int j = (int)(e - i * KH);
    if (region_counts != nullptr) {
      const long long s = i / region_rows;
      if (i - s * region_rows >= (long long)min(region_counts[s], (u32)region_rows)) {
        ids[e] = -1;
        continue;
      }
    }
    ids[e] = reinterpret_cast<const short*>(rows + i * stride + H + H / 32)[j];
  }
}

// Per-destination row i -> permuted rows perm[i*KH + j] (j < KH, -1 skipped) of the tile-major operand and
// the tiled scales.  One warp a row: each 16-byte piece is read once and written to every destination.
__global__ void __launch_bounds__(256) ep_unpack_k_kernel(const uint8_t* __restrict__ rows, int stride, int R, int H,
                                                          int KH, const int* __restrict__ perm,
                                                          uint8_t* __restrict__ qp, uint8_t* __restrict__ sfp) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int kg4 = H / 128;
  for (int i = blockIdx.x * warps + (threadIdx.x >> 5); i < R; i += gridDim.x * warps) {
    const int my_p = lane < KH ? perm[(long long)i * KH + lane] : -1;
    const unsigned live = __ballot_sync(0xffffffffu, my_p >= 0);
    if (!live) continue;
    const uint8_t* row = rows + (long long)i * stride;
    for (int c0 = 0; c0 < H; c0 += 512) {  // whole warp in step (H may end mid-step): the shuffles need every lane
      const int c = c0 + lane * 16;
      const uint4 v = c < H ? *reinterpret_cast<const uint4*>(row + c) : make_uint4(0u, 0u, 0u, 0u);
      for (unsigned m = live; m; m &= m - 1) {
        const int p = __shfl_sync(0xffffffffu, my_p, __ffs(m) - 1);
        if (c < H) *reinterpret_cast<uint4*>(qp + op8_offset(p, c, H)) = v;
      }
    }
    for (int g0 = 0; g0 < H / 128; g0 += 32) {  // whole warp in step: the shuffles below need every lane
      const int g = g0 + lane;
      const u32 v = g < H / 128 ? *reinterpret_cast<const u32*>(row + H + 4 * g) : 0u;
      for (unsigned m = live; m; m &= m - 1) {
        const int p = __shfl_sync(0xffffffffu, my_p, __ffs(m) - 1);
        if (g < H / 128) *reinterpret_cast<u32*>(sfp + sf_tiled_offset(p, 4 * g, kg4)) = v;
      }
    }
  }
}

// The return row of every routed (row, id) pair: pairs numbered in (row, j) order over the valid ids, so
// out_rows[perm[i*KH + j]] = (valid ids in rows before i) + (valid ids before j in row i).  One block; each
// thread a contiguous run of rows, a block scan of the runs' counts between two passes.
__global__ void __launch_bounds__(1024) ep_return_rows_kernel(const int* __restrict__ perm, int R, int KH,
                                                              int* __restrict__ out_rows) {
  __shared__ int warp_sum[32];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nt = blockDim.x;
  const int per = (R + nt - 1) / nt, r0 = t * per, r1 = min(R, r0 + per);
  int cnt = 0;
  for (int i = r0; i < r1; ++i)
    for (int j = 0; j < KH; ++j) cnt += perm[(long long)i * KH + j] >= 0;
  int incl = cnt;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) warp_sum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int v = lane < (nt >> 5) ? warp_sum[lane] : 0;
    int wi = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, wi, d);
      if (lane >= d) wi += y;
    }
    if (lane < (nt >> 5)) warp_sum[lane] = wi - v;
  }
  __syncthreads();
  int next = warp_sum[warp] + incl - cnt;
  for (int i = r0; i < r1; ++i)
    for (int j = 0; j < KH; ++j) {
      const int p = perm[(long long)i * KH + j];
      if (p >= 0) out_rows[p] = next++;
    }
}

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
// the single-GPU combine's arithmetic, over rows returned by the combine all-to-all.  The returned rows (and
// the shared rows) may come as column chunks of chunk_cols columns: chunk j of row p at
// back + j * back_cs + p * back_ld (shared: shared_rows + j * shared_cs + t * ld_shared).
__global__ void __launch_bounds__(256) combine_ep_kernel(const bf16* __restrict__ back, const int* __restrict__ pos,
                                                         const float* __restrict__ wts,
                                                         const bf16* __restrict__ shared_rows, int ld_shared,
                                                         bf16* __restrict__ out, int ldo, int T, int K, int cols,
                                                         int chunk_cols, long long back_cs, int back_ld,
                                                         long long shared_cs) {
  __shared__ int sp[16];
  __shared__ float sw[16];
  const int t = blockIdx.x;
  if (threadIdx.x < K) {
    sp[threadIdx.x] = pos[(long long)t * K + threadIdx.x];
    sw[threadIdx.x] = wts[(long long)t * K + threadIdx.x];
  }
  __syncthreads();
  for (int h = threadIdx.x; h < cols / 8; h += blockDim.x) {
    const int ch = (8 * h) / chunk_cols, within = 8 * h - ch * chunk_cols;
    const bf16* bk = back + ch * back_cs + within;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < K; ++k) {
      const int p = sp[k];
      if (p < 0) continue;
      const float w = sw[k];
      const uint4 u = __ldcs(reinterpret_cast<const uint4*>(bk + (long long)p * back_ld));
      const u32* pv = reinterpret_cast<const u32*>(&u);
#pragma unroll
      for (int l = 0; l < 4; ++l) {
        const float2 f = bf16x2_to_f2(pv[l]);
        acc[2 * l] = fmaf(w, f.x, acc[2 * l]);
        acc[2 * l + 1] = fmaf(w, f.y, acc[2 * l + 1]);
      }
    }
    if (shared_rows) {
      const uint4 u = *reinterpret_cast<const uint4*>(shared_rows + ch * shared_cs + (long long)t * ld_shared + within);
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
