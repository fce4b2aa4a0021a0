// Shared device helpers for the k3moe kernels (sm_100a only).
//
// Everything here is a thin wrapper over one PTX instruction or a small exact
// bit manipulation; the kernels in route.cu / gemm.cu build on them.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include <cstring>

#if defined(__CUDA_ARCH__) && !defined(__CUDA_ARCH_FEAT_SM100_ALL)
#error "k3moe kernels are written for sm_100a (compile with -gencode arch=compute_100a,code=sm_100a)"
#endif

namespace k3 {

typedef __nv_bfloat16 bf16;
typedef unsigned int u32;
typedef unsigned long long u64;

// ---------------------------------------------------------------- error word
// The first word of the caller's error buffer collects a bitmask of failures
// seen on the device; the second records the first failing site.  Kernels
// never trap: a wait that runs out of time writes here and returns.
enum : u32 {
  ERR_WAIT_TIMEOUT = 1u << 0,   // an mbarrier wait ran past its time limit
  ERR_BAD_TABLE = 1u << 1,      // a routing-table entry was out of range (skipped)
  ERR_BAD_EXPERT = 1u << 2,     // a top-k id outside [0, E) reached a table kernel (skipped)
  ERR_BAD_ARGS = 1u << 3,       // a module entry's arguments failed its checks (nothing was computed)
};

__device__ __forceinline__ void report_error(u32* err, u32 code, u32 site) {
  if (err == nullptr) return;
  atomicOr(err, code);
  atomicCAS(err + 1, 0u, site);
}

__device__ __forceinline__ u64 globaltimer_ns() {
  u64 t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- ordering keys
// Monotone f32 -> u32 map: a > b (as floats, no NaN) iff ord(a) > ord(b).
__device__ __forceinline__ u32 ord_f32(float f) {
  const u32 b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// ---------------------------------------------------------------- fp8 / scale helpers
// E4M3 of two floats (round to nearest even, saturate to +-448); lo in the low byte.
__device__ __forceinline__ unsigned short e4m3x2_sat(float lo, float hi) {
  unsigned short d;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(d) : "f"(hi), "f"(lo));
  return d;
}

// The MXFP8 block exponent for a 32-element group with absolute maximum `amax`:
// e = ceil(log2(amax / 448)) (0 when amax is 0), clamped to [-127, 127].
// The UE8M0 byte is e + 127 and the elements are scaled by 2^-e.
__device__ __forceinline__ int mx8_exponent(float amax) {
  int e = amax > 0.f ? (int)ceilf(log2f(amax / 448.f)) : 0;
  return min(max(e, -127), 127);
}

// The block exponent of FC1's output requantisation: the OCP MX rule, e = floor(log2(amax)) - 8 (E4M3's largest
// power of two is 2^8), clamped to [-127, 127]; the scaled group's largest values then lie in [256, 512) and
// the conversion saturates them at 448.  This is the rule of the reference's FC1 (the TRT-LLM-gen batched GEMM
// family): an fp32 restatement with it reproduces that GEMM's outputs on the same operands to 5e-5 rel-L2,
// where ceil(log2(amax / 448)) (the activation quantiser's rule) leaves 2.5%.  Exact: floor(log2(amax)) is the
// unbiased exponent field of a normal f32; zero and subnormal amax give -127.
__device__ __forceinline__ int mx8_exponent_ocp(float amax) {
  const int eb = (int)((__float_as_uint(amax) >> 23) & 0xffu);
  return min(max(eb - 127 - 8, -127), 127);
}

// 2^n as an f32 built from its bits, n in [-126, 127]
__device__ __forceinline__ float pow2_normal(int n) { return __uint_as_float((u32)(n + 127) << 23); }

// bf16 pairs as bits: a bf16 is the top half of its f32.
__device__ __forceinline__ float2 bf16x2_to_f2(u32 u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
__device__ __forceinline__ u32 f2_to_bf16x2(float lo, float hi) {
  u32 r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Offset of scale byte (row r, 32-group kb) in the 128x4-tiled scale layout:
// 512-byte atoms of 128 rows x 4 groups, atom (r/128, kb/4) at
// ((r/128) * kgroups4 + kb/4) * 512, inside it (r%32)*16 + (r%128/32)*4 + kb%4.
// kgroups4 = ceil(K/32 / 4).  This is cuBLAS's block-scaled layout and the one
// the tensor-core scale copy (tcgen05.cp 32x128b.warpx4) reads atom by atom.
__host__ __device__ __forceinline__ long long sf_tiled_offset(long long r, int kb, int kgroups4) {
  return ((r >> 7) * kgroups4 + (kb >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (kb & 3);
}

// Tile-major operand layout of the grouped GEMMs: a [rows, K] matrix (rows and
// K multiples of 128) is stored as 128 x 128-element tiles, tile (r/128, k/128)
// at index (r/128) * (K/128) + k/128, each tile row-major.  One pipeline
// stage's TMA box is then one contiguous chunk (16 KB of E4M3, 8 KB of packed
// E2M1), and the tile index equals the index of its 512-byte scale atom.
__host__ __device__ __forceinline__ long long op8_offset(long long r, int k, int K) {
  return (((r >> 7) * (K >> 7) + (k >> 7)) << 14) + ((r & 127) << 7) + (k & 127);
}
// packed E2M1 (two elements a byte, element 2i in the low nibble of byte i): byte of element k
__host__ __device__ __forceinline__ long long op4_offset(long long r, int k, int K) {
  return (((r >> 7) * (K >> 7) + (k >> 7)) << 13) + ((r & 127) << 6) + ((k & 127) >> 1);
}

// ---------------------------------------------------------------- shared memory / mbarrier
__device__ __forceinline__ u32 smem_u32(const void* p) { return (u32)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(u64* bar, u32 count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(u64* bar, u32 bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(u64* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(u64* bar, u32 parity) {
  u32 ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and reports) when `limit_ns` passes first, or
// when another role of the block already gave up (`*abort` set; a null
// `abort` waits out the limit regardless, for draining copies in flight).
__device__ __forceinline__ bool mbar_wait(u64* bar, u32 parity, volatile int* abort, u32* err, u32 site,
                                          u64 limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const u64 t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort != nullptr && *abort) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      if (abort != nullptr) *abort = 1;
      report_error(err, ERR_WAIT_TIMEOUT, site);
      return false;
    }
  }
}

// 32 bytes to global memory in one store (sm_100's 256-bit vector store); `p` 32-byte aligned.  A warp's
// stores to 32 different rows then fill whole 32-byte sectors and take half the store instructions of
// 16-byte ones.
__device__ __forceinline__ void st_global_v8(void* p, const u32 (&v)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, u64* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// plain bulk copy global -> shared, 16-byte aligned addresses, size a multiple of 16
__device__ __forceinline__ void bulk_load(void* dst, const void* src, u32 bytes, u64* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// bring a tensor-map box into L2 (no shared memory, no completion to wait on)
__device__ __forceinline__ void tma_prefetch_2d(const void* tmap, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(tmap), "r"(c0), "r"(c1)
               : "memory");
}
// bring `bytes` (a multiple of 16, 16-byte aligned) into L2
__device__ __forceinline__ void bulk_prefetch(const void* src, u32 bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------- cp.async (LDGSTS)
// 16 bytes global -> shared, through L2 only; both addresses 16-byte aligned
__device__ __forceinline__ void cp_async16(u32 dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// arrive on `bar` once every cp.async this thread issued so far has landed (the barrier counts the arrival)
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(u64* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// order this thread's view of generic-proxy shared-memory writes before its later async-proxy accesses
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(u32* dst_smem, u32 ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(u32 taddr, u32 ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(u64* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[smem] x B[smem]^T with per-32 UE8M0 scales read from tmem.
__device__ __forceinline__ void mma_mxf8f6f4(u32 d_tmem, u64 adesc, u64 bdesc, u32 idesc, u32 sfa_tmem, u32 sfb_tmem,
                                             u32 accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Copy a 32-row x 16-byte block of shared memory into tmem lanes 0..31 of every
// sub-partition (replicated x4), 4 columns wide.
__device__ __forceinline__ void tmem_cp_32x128b_x4(u32 taddr, u64 sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive columns of this warp's 32 lanes: thread i gets lane (base + i), columns c..c+31.
__device__ __forceinline__ void tmem_ld32(u32 taddr, u32 (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row x 128-byte
// atoms 1024 bytes apart.  The tile base must be 1024-byte aligned; stepping
// the start address by 32 bytes selects the next 32-element K block.
__device__ __forceinline__ u64 sdesc_k_sw128(u32 saddr) {
  u64 d = (u64)((saddr >> 4) & 0x3FFFu);
  d |= (u64)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (u64)(1024 >> 4) << 32;   // stride byte offset: next 8-row group
  d |= (u64)1 << 46;             // descriptor version for sm_100
  d |= (u64)2 << 61;             // SWIZZLE_128B
  return d;
}
// Descriptor of a 32-row x 16-byte scale block (no swizzle, rows 16 bytes apart,
// 8-row groups 128 bytes apart), the source of tcgen05.cp 32x128b.
__device__ __forceinline__ u64 sdesc_sf(u32 saddr) {
  u64 d = (u64)((saddr >> 4) & 0x3FFFu);
  d |= (u64)(128 >> 4) << 32;
  d |= (u64)1 << 46;
  return d;
}

// Instruction descriptor of kind::mxf8f6f4 with UE8M0 scales, K-major A and B,
// M = 128, N = n (multiple of 8, <= 256).  Formats: 0 = E4M3, 5 = E2M1.
// The scale-factor ids select the byte of the scale column (the K block).
enum : u32 { FMT_E4M3 = 0, FMT_E2M1 = 5 };
__device__ __forceinline__ u32 idesc_mxf8f6f4(int n, u32 a_sf_id, u32 b_sf_id, u32 a_fmt = FMT_E2M1,
                                              u32 b_fmt = FMT_E4M3) {
  u32 d = 0;
  d |= (b_sf_id & 3u) << 4;
  d |= a_fmt << 7;               // A format
  d |= b_fmt << 10;              // B format
  d |= (u32)(n >> 3) << 17;      // N >> 3
  d |= 1u << 23;                 // scale type UE8M0
  d |= (128u >> 4) << 24;        // M >> 4
  d |= (a_sf_id & 3u) << 29;
  return d;
}

}  // namespace k3
