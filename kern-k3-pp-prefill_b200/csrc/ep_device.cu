// The device-resident expert-parallel step (k3moe_ep_forward): every rank's buffer that its peers store into
// has FIXED regions, so no rank needs another rank's counts before it sends, and the step has no host
// synchronisation (a whole step can be captured in a CUDA graph).
//
// One rank's peer buffer (mapped into every rank through CUDA IPC):
//   recv   (W + 1) * T_max rows of `stride` bytes: region s < W the rows source rank s sent this step (the pair
//          rows of ep_pack_pairs_kernel plus, at byte back_col, the int32 return index of the row's first pick),
//          region W this rank's own tokens for the shared expert;
//   back   T_max * K rows of H bf16: FC2's results of this rank's picks, grouped by the rank that computed them
//          and in (token, pick) order within one (the picks plan below numbers them);
//   counts W + 1 u32: rows region s holds this step (count s written by source s before its flag);
//   flags  2W u32: flag (phase, s) = the step number when source s's stores of that phase are complete.
// The receiver reads a region's first counts[s] rows only; the return index carried by each row tells the
// computing rank where in the owner's back buffer its results go, so FC2's epilogue stores them there directly.
#pragma once
#include "ep_peer.cu"

namespace k3 {

constexpr int PLAN_THREADS = 1024;

// Block-wide exclusive scan of one 64-bit value a thread (1024 threads); `total` gets the block's sum.
__device__ __forceinline__ unsigned long long block_exclusive_scan_u64(unsigned long long v, unsigned long long* s_warp,
                                                                       unsigned long long& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long incl = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const unsigned long long wv = s_warp[lane];
    unsigned long long wi = wv;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, wi, d);
      if (lane >= d) wi += y;
    }
    s_warp[lane] = wi - wv;
    if (lane == 31) s_warp[32] = wi;
  }
  __syncthreads();
  const unsigned long long r = s_warp[warp] + incl - v;
  total = s_warp[32];
  __syncthreads();  // s_warp reused by the next scan
  return r;
}

// The sender's plans, one block of PLAN_THREADS threads, thread i the tokens [i * per, (i + 1) * per):
//   dest[t*K + k], lid[t*K + k]   rank and local expert id of each pick (owner / local maps, or E_local blocks)
//   pair_pos[t*W + d]             the token's row in its region of rank d's receive buffer (its number among
//                                 the tokens with a pick on d, in token order), -1 when it has none there
//   pair_back[t*W + d]            the return index of the token's first pick on d
//   send_pos[t*K + k]             each pick's return index: picks grouped by destination rank, (token, pick)
//                                 order within one (the combine reads back[send_pos])
//   rows_to[d]                    rows this rank sends rank d (delivered as d's count of this source)
// and, once a step, the step number (*epoch += 1) and this rank's own shared-region count (shared_rows).
__global__ void __launch_bounds__(PLAN_THREADS) ep_plan_kernel(
    const int* __restrict__ idx, int T, int K, int W, int E_local, const int* __restrict__ owner,
    const int* __restrict__ local, int* __restrict__ dest, int* __restrict__ lid, int* __restrict__ pair_pos,
    int* __restrict__ pair_back, int* __restrict__ send_pos, int* __restrict__ rows_to, u32* __restrict__ epoch,
    u32* __restrict__ shared_count, int shared_rows, int E, u32* __restrict__ err) {
  __shared__ unsigned long long s_warp[33];
  __shared__ int s_first[EP_MAX_RANKS];  // first return index of each destination's picks
  const int per = (T + PLAN_THREADS - 1) / PLAN_THREADS;
  const int t0 = min(T, (int)threadIdx.x * per), t1 = min(T, t0 + per);
  // pass 1: each pick's destination; this thread's rows (low 32 bits) and picks (high) a destination
  unsigned long long mine[EP_MAX_RANKS];
#pragma unroll
  for (int d = 0; d < EP_MAX_RANKS; ++d) mine[d] = 0ull;
  for (int t = t0; t < t1; ++t) {
    u32 on = 0;
    for (int k = 0; k < K; ++k) {
      const int e = idx[(long long)t * K + k];
      int d = -1, l = -1;
      if (e >= 0 && e < E) {
        d = owner ? owner[e] : e / E_local;
        l = local ? local[e] : e - d * E_local;
      }
      if (d < 0 || d >= W) {
        report_error(err, ERR_BAD_EXPERT, 0xC00u);
        d = -1;
        l = -1;
      }
      dest[(long long)t * K + k] = d;
      lid[(long long)t * K + k] = l;
      if (d >= 0) on |= 1u << d;
#pragma unroll
      for (int q = 0; q < EP_MAX_RANKS; ++q)
        if (q == d) mine[q] += 1ull << 32;
    }
#pragma unroll
    for (int q = 0; q < EP_MAX_RANKS; ++q) mine[q] += (on >> q) & 1u;
  }
  // exclusive prefixes over the threads (token order), and the destinations' totals
  unsigned long long run[EP_MAX_RANKS];
  long long first = 0;
#pragma unroll
  for (int q = 0; q < EP_MAX_RANKS; ++q) {
    if (q >= W) {
      run[q] = 0ull;
      continue;
    }
    unsigned long long total;
    run[q] = block_exclusive_scan_u64(mine[q], s_warp, total);
    if (threadIdx.x == 0) {
      s_first[q] = (int)first;
      rows_to[q] = (int)(total & 0xffffffffull);
    }
    first += (long long)(total >> 32);
  }
  if (threadIdx.x == 0) {
    *epoch += 1u;
    *shared_count = (u32)shared_rows;
  }
  __syncthreads();
  // pass 2: the positions, token by token in order
  for (int t = t0; t < t1; ++t) {
    u32 on = 0;
    for (int k = 0; k < K; ++k) {
      const int d = dest[(long long)t * K + k];
      if (d >= 0) on |= 1u << d;
    }
#pragma unroll
    for (int q = 0; q < EP_MAX_RANKS; ++q) {
      if (q >= W) continue;
      const bool has = (on >> q) & 1u;
      pair_pos[(long long)t * W + q] = has ? (int)(run[q] & 0xffffffffull) : -1;
      pair_back[(long long)t * W + q] = has ? s_first[q] + (int)(run[q] >> 32) : -1;
      if (has) run[q] += 1ull;
    }
    for (int k = 0; k < K; ++k) {
      const int d = dest[(long long)t * K + k];
      int pos = -1;
#pragma unroll
      for (int q = 0; q < EP_MAX_RANKS; ++q)
        if (q == d) {
          pos = s_first[q] + (int)(run[q] >> 32);
          run[q] += 1ull << 32;
        }
      send_pos[(long long)t * K + k] = pos;
    }
  }
}

// One phase of the exchange, thread s < W: with rows_to, store rows_to[s] into count `me` of rank s's peer
// buffer (a local store for s == me); then (s != me) a system-scope fence and a release store of the step
// number into flag (phase, me) of rank s; then wait, at most budget_ns, for flag (phase, s) of this rank to
// reach the step number (serial-number order).  A source still late is recorded (ERR_WAIT_TIMEOUT, site
// 0xA00 + 0x10 * phase + s) and the kernel returns.  The step's data stores were made by earlier kernels on
// this stream, each ending with a system-scope fence.
__global__ void ep_exchange_kernel(EpBases peer, long long counts_off, long long flags_off, int W, int me, int phase,
                                   const int* __restrict__ rows_to, const u32* __restrict__ epoch,
                                   unsigned long long budget_ns, u32* __restrict__ err) {
  const int s = threadIdx.x;
  if (s >= W) return;
  const u32 step = *epoch;
  uint8_t* theirs = reinterpret_cast<uint8_t*>(peer.base[s]);
  if (rows_to != nullptr) reinterpret_cast<volatile u32*>(theirs + counts_off)[me] = (u32)rows_to[s];
  if (s == me) return;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  st_release_sys(reinterpret_cast<u32*>(theirs + flags_off) + phase * W + me, step);
  const u32* flag = reinterpret_cast<const u32*>(reinterpret_cast<const uint8_t*>(peer.base[me]) + flags_off) +
                    phase * W + s;
  const u64 t0 = globaltimer_ns();
  for (;;) {
    if ((int)(ld_acquire_sys(flag) - step) >= 0) return;
    if (globaltimer_ns() - t0 > budget_ns) {
      report_error(err, ERR_WAIT_TIMEOUT, 0xA00u + 0x10u * (u32)phase + (u32)s);
      return;
    }
    __nanosleep(128);
  }
}

// The address of every FC2 result row: pick j of received row r (permuted row p = perm[r*K + j] >= 0) goes to
// rank s's back buffer (back.base[s], s = r / region_rows) at row (return index carried by row r) + j, or, for
// a row of the shared region (r >= W * region_rows), to shared_base + (r - W * region_rows) * row_bytes.  A
// return index outside [0, back_rows) is recorded (ERR_BAD_TABLE, site 0xB10) and its row sent to `sink`.
__global__ void __launch_bounds__(256) ep_step_ptrs_kernel(const int* __restrict__ perm, long long n, int K,
                                                           const uint8_t* __restrict__ rows, int stride, int back_col,
                                                           int region_rows, int W, EpBases back, long long back_rows,
                                                           unsigned long long shared_base, long long row_bytes,
                                                           unsigned long long sink,
                                                           unsigned long long* __restrict__ ptrs,
                                                           u32* __restrict__ err) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const int p = perm[e];
    if (p < 0) continue;
    const long long r = e / K;
    const int j = (int)(e - r * K);
    unsigned long long a;
    if (r < (long long)W * region_rows) {
      const int s = (int)(r / region_rows);
      const long long b = (long long)*reinterpret_cast<const int*>(rows + r * stride + back_col) + j;
      if (b >= 0 && b < back_rows) {
        a = back.base[s] + (unsigned long long)(b * row_bytes);
      } else {
        report_error(err, ERR_BAD_TABLE, 0xB10u);
        a = sink;
      }
    } else {
      a = shared_base + (unsigned long long)((r - (long long)W * region_rows) * row_bytes);
    }
    ptrs[p] = a;
  }
}

}  // namespace k3
