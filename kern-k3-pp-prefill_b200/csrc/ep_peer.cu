// Expert-parallel transport over peer memory (NVLink / NVSwitch, CUDA IPC mappings): the dispatch rows and
// FC2's results are stored straight into the receiving rank's buffers by the kernels that make them (the pack
// kernel, FC2's epilogue), so neither all-to-all runs as a separate pass; a flag a (source rank, phase) then
// tells the receiver that a source's stores are complete.  The combine that follows reads only local memory:
// the combine is folded into the receive side of the collective.
//
// Ordering.  A source's data stores are made by kernels that complete before its signal kernel starts (the
// same stream); the signal kernel fences at system scope and stores the flag with release semantics; the
// receiver's wait kernel loads it with acquire semantics before the kernels that read the data start.
// Every wait is bounded by a %globaltimer budget: on expiry it records ERR_WAIT_TIMEOUT (site 0xA00 + the
// late source) in the error words and returns; nothing traps.  No TMA touches peer memory.
#pragma once
#include "ep.cu"

namespace k3 {

__device__ __forceinline__ void st_release_sys(u32* p, u32 v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ u32 ld_acquire_sys(const u32* p) {
  u32 v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread s < W (s != me): store `epoch` into slot `slot0 + me` of rank s's flag array (flag_base.base[s]).
__global__ void ep_signal_kernel(EpBases flag_base, int W, int me, int slot0, u32 epoch) {
  const int s = threadIdx.x;
  if (s >= W || s == me) return;
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  st_release_sys(reinterpret_cast<u32*>(flag_base.base[s]) + slot0 + me, epoch);
}

// Lane s < W (s != skip) waits until flags[s] has reached `epoch` (serial-number order), at most budget_ns;
// a source that stays late is recorded (ERR_WAIT_TIMEOUT, site 0xA00 + s) and the wait returns.
__global__ void ep_wait_kernel(const u32* __restrict__ flags, int W, int skip, u32 epoch, unsigned long long budget_ns,
                               u32* __restrict__ err) {
  const int s = threadIdx.x;
  if (s >= W || s == skip) return;
  const u64 t0 = globaltimer_ns();
  for (;;) {
    if ((int)(ld_acquire_sys(flags + s) - epoch) >= 0) return;
    if (globaltimer_ns() - t0 > budget_ns) {
      report_error(err, ERR_WAIT_TIMEOUT, 0xA00u + (u32)s);
      return;
    }
    __nanosleep(256);
  }
}

// The destination address of every FC2 result row: permuted row perm[i*KH + j] (>= 0) carries the (i, j) pair
// numbered q = out_rows[perm]; q falls in block s ([start[s], start[s+1])), whose rows go to base[s] + (q -
// start[s]) * row_bytes.  A q outside every block is recorded (ERR_BAD_TABLE) and its row sent to `sink`.
__global__ void __launch_bounds__(256) ep_row_ptrs_kernel(const int* __restrict__ perm, long long n, int nblocks,
                                                          const int* __restrict__ out_rows, EpBases blocks,
                                                          long long row_bytes, unsigned long long sink,
                                                          unsigned long long* __restrict__ ptrs, u32* __restrict__ err) {
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const int p = perm[e];
    if (p < 0) continue;
    const long long q = out_rows[p];
    unsigned long long a = sink;
    bool ok = false;
    for (int s = 0; s < nblocks; ++s)
      if (q >= blocks.start[s] && q < blocks.start[s + 1]) {
        a = blocks.base[s] + (unsigned long long)((q - blocks.start[s]) * row_bytes);
        ok = true;
        break;
      }
    if (!ok) report_error(err, ERR_BAD_TABLE, 0xB00u);
    ptrs[p] = a;
  }
}

}  // namespace k3
