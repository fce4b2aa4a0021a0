// Module entries of the two grouped GEMMs, for a manifest that binds FC1 / FC2 as plain kernel launches in
// place of the TRT-LLM-gen batched GEMMs (kernels.toml:1-9; scripts/k3_moe_bmm.py:112-113 `trtllm_bmm.op`).
// They take the reference ops' logical parameters in the reference's order (scripts/k3_moe_bmm.py:131-134,
// 167-169: FC1 a, sf_a, b, sf_b, c, sf_c, route_map, alpha, beta, num_non_exiting, total_padded, cta_batch,
// cta_limit; FC2 a, sf_a, b, sf_b, c, num_non_exiting, total_padded, cta_batch, cta_limit), then the GEMM's
// shape and this build's own: `maps`, a global-memory buffer of two TMA descriptors (the weights', then the
// activations') that k3moe_gemm_tensor_maps fills once at load time (the buffers are bound at fixed
// addresses, as the TRT-LLM-gen parameter block's descriptors are), and `err`, two error words.
//
//   a / sf_a   the expert weights (MXFP4, tile-major) and their tiled scales: the maps' first descriptor covers a
//   b / sf_b   the activations: MXFP8 rows in permuted order, tile-major (kern_k3_moe_quant_permute's output,
//              or k3moe_quant_permute's); the second descriptor covers b.  The rows are already permuted, so
//              route_map is accepted for the argument list and not read.
//   c / sf_c   FC1: MXFP8 [padded, m/2] tile-major + tiled scales; FC2: bf16 [padded, m] row-major
//   alpha/beta FC1 with act = 1: SiTU's per-expert a, b (K3: 4 and 25, the reference's `fill_f32` carries);
//              act = 0: SwiGLU (the buffers are not read).
//   m, k       weight rows an expert (FC1 2I, FC2 H) and the reduction length (FC1 H, FC2 I)
// Launch: grid = the SM count (a persistent walk over the tables' units; 148 on B200), block gemm::THREADS
// (384), dynamic shared memory gemm::SMEM_BYTES.  The outputs are those of k3moe_fc1_act / k3moe_fc2 byte for
// byte (tests/test_gpu_dropin.py).
#include "gemm.cu"

namespace k3 {

// The descriptors were written through the generic proxy (a copy into global memory): order them before the
// tensor-map proxy's reads of this thread (the TMA producer).
__device__ __forceinline__ void acquire_tmaps(const CUtensorMap* maps) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(maps) : "memory");
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(maps + 1) : "memory");
}

// The host checks of gemm_launch, made on the device (a module launch has no host code): m a multiple of 256
// (FC1: 128 gate + 128 up rows a unit; FC2: 256 outputs), k of 256, the output 32-byte aligned (256-bit
// stores), the descriptors 64-byte aligned.
__device__ __forceinline__ bool module_gemm_args_ok(int m, int k, int num_experts, int cap_rows, int max_ctas,
                                                    const CUtensorMap* maps, const void* out) {
  return m > 0 && m % 256 == 0 && k > 0 && k % 256 == 0 && num_experts > 0 && cap_rows > 0 &&
         cap_rows % 128 == 0 && max_ctas > 0 && (long long)max_ctas * 128 <= cap_rows && maps != nullptr &&
         (reinterpret_cast<uintptr_t>(maps) & 63) == 0 && out != nullptr && (reinterpret_cast<uintptr_t>(out) & 31) == 0;
}

}  // namespace k3

// The activations of FC1's `b` / `sf_b`: every row of x (bf16, row stride ldx) quantised to MXFP8 and written to
// each permuted row it is routed to (exp2perm, [R, K]; and the shared expert's row meta[2] + r when meta[2] >= 0),
// tile-major with tiled scales (k3moe_quant_permute's output).  In the reference chain the GEMM gathers the
// quantised rows itself through route_map; here this launch does it before FC1.  Grid any (a persistent walk,
// one warp a row), block 256; cols a multiple of 256.
extern "C" __global__ void __launch_bounds__(256) kern_k3_moe_quant_permute(
    const k3::bf16* __restrict__ x, int ldx, int R, int cols, int K, const int* __restrict__ exp2perm,
    const int* __restrict__ meta, uint8_t* __restrict__ q_perm, uint8_t* __restrict__ sf_perm) {
  if (cols <= 0 || cols % 256 || ldx < cols || K < 1 || K > 16) return;
  k3::quant_permute_rows(x, ldx, R, cols, K, exp2perm, meta, q_perm, sf_perm);
}

extern "C" __global__ void __launch_bounds__(k3::gemm::THREADS, 1) kern_k3_moe_fc1(
    const uint8_t* __restrict__ a, const uint8_t* __restrict__ sf_a, const uint8_t* __restrict__ b,
    const uint8_t* __restrict__ sf_b, uint8_t* __restrict__ c, uint8_t* __restrict__ sf_c,
    const int* __restrict__ route_map, const float* __restrict__ alpha, const float* __restrict__ beta,
    const int* __restrict__ num_non_exiting, const int* __restrict__ total_padded, const int* __restrict__ cta_batch,
    const int* __restrict__ cta_limit, int m, int k, int num_experts, int cap_rows, int max_ctas, int act,
    const CUtensorMap* __restrict__ maps, unsigned* __restrict__ err) {
  using namespace k3;
  (void)a;
  (void)b;
  (void)route_map;
  (void)total_padded;
  if (!module_gemm_args_ok(m, k, num_experts, cap_rows, max_ctas, maps, c) || (act != 0 && act != 1)) {
    if (threadIdx.x == 0) report_error(err, ERR_BAD_ARGS, 0x910u);
    return;
  }
  if (threadIdx.x == 0) acquire_tmaps(maps);
  GemmParams p;
  p.sfw = sf_a;
  p.sfa = sf_b;
  p.cta_batch = cta_batch;
  p.cta_limit = cta_limit;
  p.meta = num_non_exiting;
  p.out_q = c;
  p.out_sf = sf_c;
  p.out_bf16 = nullptr;
  p.out_rows = nullptr;
  p.err = err;
  p.K = k;
  p.rows_per_expert = m;
  p.n_experts = num_experts;
  p.nfb = m / 2 / 128;
  p.out_cols = m / 2;
  p.cap_rows = cap_rows;
  p.max_ctas = max_ctas;
  p.trace = nullptr;
  p.act = act;
  p.fb0 = 0;
  p.alpha = act == 1 ? alpha : nullptr;
  p.beta = act == 1 ? beta : nullptr;
  p.out_ptrs = nullptr;
  grouped_gemm_body<MODE_FC1>(maps, maps + 1, p);
}

extern "C" __global__ void __launch_bounds__(k3::gemm::THREADS, 1) kern_k3_moe_fc2(
    const uint8_t* __restrict__ a, const uint8_t* __restrict__ sf_a, const uint8_t* __restrict__ b,
    const uint8_t* __restrict__ sf_b, k3::bf16* __restrict__ c, const int* __restrict__ num_non_exiting,
    const int* __restrict__ total_padded, const int* __restrict__ cta_batch, const int* __restrict__ cta_limit, int m,
    int k, int num_experts, int cap_rows, int max_ctas, const CUtensorMap* __restrict__ maps,
    unsigned* __restrict__ err) {
  using namespace k3;
  (void)a;
  (void)b;
  (void)total_padded;
  if (!module_gemm_args_ok(m, k, num_experts, cap_rows, max_ctas, maps, c)) {
    if (threadIdx.x == 0) report_error(err, ERR_BAD_ARGS, 0x920u);
    return;
  }
  if (threadIdx.x == 0) acquire_tmaps(maps);
  GemmParams p;
  p.sfw = sf_a;
  p.sfa = sf_b;
  p.cta_batch = cta_batch;
  p.cta_limit = cta_limit;
  p.meta = num_non_exiting;
  p.out_q = nullptr;
  p.out_sf = nullptr;
  p.out_bf16 = c;
  p.out_rows = nullptr;
  p.err = err;
  p.K = k;
  p.rows_per_expert = m;
  p.n_experts = num_experts;
  p.nfb = m / gemm::BN;
  p.out_cols = m;
  p.cap_rows = cap_rows;
  p.max_ctas = max_ctas;
  p.trace = nullptr;
  p.act = 0;
  p.fb0 = 0;
  p.alpha = nullptr;
  p.beta = nullptr;
  p.out_ptrs = nullptr;
  grouped_gemm_body<MODE_FC2>(maps, maps + 1, p);
}
