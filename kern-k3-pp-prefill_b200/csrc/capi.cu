// Host side of the k3moe C ABI (include/k3moe.h): argument checks, launch
// geometry, TMA tensor-map encoding and the layer chain.  One translation unit
// holds every kernel so the library needs no relocatable device code.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <vector>

#include "../../include/k3moe.h"
#include "gemm.cu"
#include "route.cu"
#include "ep.cu"
#include "ep_peer.cu"
#include "ep_device.cu"
#include "router.cu"
#include "dropin.cu"

using namespace k3;

static_assert(gemm::THREADS == K3MOE_GEMM_THREADS && gemm::SMEM_BYTES == K3MOE_GEMM_SMEM_BYTES,
              "the module GEMM entries' launch geometry in include/k3moe.h");

namespace {

constexpr int kMaxDevices = 64;

int num_sms(int dev) {
  static int cache[kMaxDevices] = {0};
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

// Kernel attributes are per device: set them once per (device, kernel).
template <typename F>
bool set_smem_once(F kernel, int bytes, int slot) {
  static std::mutex mu;
  static bool done[kMaxDevices][8] = {};
  const int dev = current_device();
  std::lock_guard<std::mutex> g(mu);
  if (dev >= 0 && dev < kMaxDevices && done[dev][slot]) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  if (dev >= 0 && dev < kMaxDevices) done[dev][slot] = true;
  return true;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Map over a tile-major operand (rows x k, both multiples of 128): viewed as
// rows*k/128 rows of 128 elements, so one 128 x 128 box is one stored tile
// (a contiguous 16 KB of E4M3 or 8 KB of packed E2M1); 128-byte swizzle.
int encode_operand(CUtensorMap* m, const void* base, long long rows, int k, bool fp4) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return K3MOE_EDRIVER;
  const cuuint64_t dims[2] = {128, (cuuint64_t)(rows * (k / 128))};
  const cuuint64_t strides[1] = {(cuuint64_t)(fp4 ? 64 : 128)};
  const cuuint32_t box[2] = {128, 128};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, fp4 ? CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? K3MOE_OK : K3MOE_ETMAP;
}

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange: the base of the allocation holding a pointer (an IPC handle names a whole allocation)
AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(p);
  });
  return fn;
}

unsigned long long* g_trace = nullptr;  // k3moe_set_trace

int launch_status() { return cudaGetLastError() == cudaSuccess ? K3MOE_OK : K3MOE_ELAUNCH; }

inline long long cdiv(long long a, long long b) { return (a + b - 1) / b; }
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

template <int EPL>
void launch_topk(const float* S, int lds, const float* bias, const bf16* rs, int T, int E, int K, int* idx,
                 float* wts, cudaStream_t s) {
  const int warps = 8;
  const long long blocks = cdiv(T, warps);
  topk_kernel<EPL><<<(unsigned)blocks, warps * 32, 0, s>>>(S, lds, bias, rs, T, E, K, idx, wts);
}

// FC2 may compute a column slice [col0, col0 + ncols) of its output into a buffer of row stride ldo (ncols 0:
// all H columns, row stride H), with at most grid_cap persistent blocks (0: one an SM).
int gemm_launch(int mode, const uint8_t* w, const uint8_t* w_sf, const uint8_t* act, const uint8_t* act_sf,
                const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, uint8_t* out_q,
                uint8_t* out_sf, void* out_bf16, int H, int I, int n_experts, int cap_rows, int max_ctas,
                uint32_t* err, cudaStream_t stream, const int32_t* out_rows = nullptr, int activation = 0,
                int col0 = 0, int ncols = 0, int ldo = 0, int grid_cap = 0, const uint64_t* out_ptrs = nullptr) {
  if (activation != 0 && activation != 1) return K3MOE_EINVAL;
  if (ncols == 0) {
    ncols = H;
    ldo = H;
  }
  if (col0 < 0 || col0 % gemm::BN || ncols <= 0 || ncols % gemm::BN || col0 + ncols > H || ldo < ncols || ldo % 16 ||
      grid_cap < 0)
    return K3MOE_EINVAL;
  if (H <= 0 || I <= 0 || H % 256 || I % 256 || n_experts <= 0 || cap_rows <= 0 || cap_rows % 128 || max_ctas <= 0 ||
      (long long)max_ctas * 128 > cap_rows)
    return K3MOE_EINVAL;
  // the epilogues store 32 bytes at a time (256-bit stores): the outputs must start 32-byte aligned
  const void* out0 = mode == MODE_FC1 ? static_cast<const void*>(out_q) : out_ptrs ? out_ptrs : out_bf16;
  if (out0 == nullptr || reinterpret_cast<uintptr_t>(out0) % 32 != 0) return K3MOE_EINVAL;
  const int K = mode == MODE_FC1 ? H : I;
  const int rows_per_expert = mode == MODE_FC1 ? 2 * I : H;
  CUtensorMap ta, tb;
  int rc = encode_operand(&ta, w, (long long)n_experts * rows_per_expert, K, true);
  if (rc) return rc;
  rc = encode_operand(&tb, act, cap_rows, K, false);
  if (rc) return rc;
  GemmParams p;
  p.sfw = w_sf;
  p.sfa = act_sf;
  p.cta_batch = cta_batch;
  p.cta_limit = cta_limit;
  p.meta = meta;
  p.out_q = out_q;
  p.out_sf = out_sf;
  p.out_bf16 = reinterpret_cast<bf16*>(out_bf16);
  p.out_rows = out_rows;
  p.act = activation;
  p.alpha = nullptr;  // SiTU at K3's a = 4, b = 25
  p.beta = nullptr;
  p.out_ptrs = reinterpret_cast<const unsigned long long*>(out_ptrs);
  p.err = err;
  p.K = K;
  p.rows_per_expert = rows_per_expert;
  p.n_experts = n_experts;
  p.nfb = mode == MODE_FC1 ? I / 128 : ncols / gemm::BN;  // FC1: 128 features (gate + up rows), FC2: 256 outputs
  p.fb0 = mode == MODE_FC1 ? 0 : col0 / gemm::BN;
  p.out_cols = mode == MODE_FC1 ? I : ldo;
  p.cap_rows = cap_rows;
  p.max_ctas = max_ctas;
  p.trace = g_trace;
  const long long max_units = (long long)max_ctas * p.nfb;
  const int sms = num_sms(current_device());
  const int grid = (int)std::min<long long>(grid_cap > 0 ? std::min(grid_cap, sms) : sms, max_units);
  if (mode == MODE_FC1) {
    if (!set_smem_once(grouped_gemm_kernel<MODE_FC1>, gemm::SMEM_BYTES, 0)) return K3MOE_ELAUNCH;
    grouped_gemm_kernel<MODE_FC1><<<grid, gemm::THREADS, gemm::SMEM_BYTES, stream>>>(ta, tb, p);
  } else {
    if (!set_smem_once(grouped_gemm_kernel<MODE_FC2>, gemm::SMEM_BYTES, 1)) return K3MOE_ELAUNCH;
    grouped_gemm_kernel<MODE_FC2><<<grid, gemm::THREADS, gemm::SMEM_BYTES, stream>>>(ta, tb, p);
  }
  return launch_status();
}

struct LayerLayout {
  size_t off[14];
  size_t total;
  int max_ctas, cap_rows, nb, EL;
  size_t blockcount, blockoff;  // inside the route scratch
};

enum { L_IDX, L_WTS, L_COUNTS, L_CTA_BATCH, L_CTA_LIMIT, L_META, L_ROUTE_MAP, L_EXP2PERM, L_QP, L_SFP, L_FC1Q,
       L_FC1SF, L_FC2, L_ERR };

LayerLayout layer_layout(int T, int H, int I, int E, int K, int shared) {
  LayerLayout L;
  L.EL = E + shared;
  L.nb = (int)cdiv(T, TB);
  L.max_ctas = k3moe_max_ctas(T, K, E, shared, 128);
  L.cap_rows = L.max_ctas * 128;
  size_t at = 0;
  auto take = [&](size_t bytes) {
    const size_t o = at;
    at = align_up(at + bytes, 1024);
    return o;
  };
  L.off[L_IDX] = take((size_t)T * K * 4);
  L.off[L_WTS] = take((size_t)T * K * 4);
  L.off[L_COUNTS] = take((size_t)L.EL * 4);
  L.off[L_CTA_BATCH] = take((size_t)L.max_ctas * 4);
  L.off[L_CTA_LIMIT] = take((size_t)L.max_ctas * 4);
  L.off[L_META] = take(16);
  L.off[L_ROUTE_MAP] = take((size_t)L.cap_rows * 4);
  L.off[L_EXP2PERM] = take((size_t)T * K * 4);
  L.off[L_QP] = take((size_t)L.cap_rows * H);
  L.off[L_SFP] = take((size_t)L.cap_rows * H / 32);
  L.off[L_FC1Q] = take((size_t)L.cap_rows * I);
  L.off[L_FC1SF] = take((size_t)L.cap_rows * I / 32);
  L.off[L_FC2] = take((size_t)L.cap_rows * H * 2);
  L.off[L_ERR] = take(16);
  L.blockcount = take((size_t)L.nb * L.EL * 4);
  L.blockoff = take((size_t)L.nb * L.EL * 4);
  L.total = at;
  return L;
}

}  // namespace

extern "C" {

int k3moe_abi_version(void) { return 1; }

int k3moe_route_topk(const float* S, int lds, const float* bias, const void* rs_bf16, int T, int E_total, int K,
                     int32_t* idx, float* wts, k3moe_stream_t stream) {
  if (T < 0 || E_total < K || E_total > 1024 || K < 1 || K > 16 || (K & (K - 1)) || lds < E_total) return K3MOE_EINVAL;
  if (T == 0) return K3MOE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bf16* rs = reinterpret_cast<const bf16*>(rs_bf16);
  const int epl = (E_total + 31) / 32;
  if (epl <= 1) launch_topk<1>(S, lds, bias, rs, T, E_total, K, idx, wts, s);
  else if (epl <= 2) launch_topk<2>(S, lds, bias, rs, T, E_total, K, idx, wts, s);
  else if (epl <= 4) launch_topk<4>(S, lds, bias, rs, T, E_total, K, idx, wts, s);
  else if (epl <= 8) launch_topk<8>(S, lds, bias, rs, T, E_total, K, idx, wts, s);
  else if (epl <= 16) launch_topk<16>(S, lds, bias, rs, T, E_total, K, idx, wts, s);
  else if (epl <= 28) launch_topk<28>(S, lds, bias, rs, T, E_total, K, idx, wts, s);
  else launch_topk<32>(S, lds, bias, rs, T, E_total, K, idx, wts, s);
  return launch_status();
}

int k3moe_max_ctas(int R, int K, int E, int shared, int tile) {
  if (R < 0 || K < 1 || E < 1 || tile < 1) return 0;
  const long long rows = (long long)R * K + (long long)(shared ? R : 0);
  return (int)(E + (shared ? 1 : 0) + cdiv(rows, tile));
}

size_t k3moe_route_scratch_bytes(int R, int E, int shared) {
  const size_t nb = (size_t)cdiv(R, TB);
  return 2 * align_up(nb * (E + (shared ? 1 : 0)) * 4, 256);
}

int k3moe_route_tables(const int32_t* idx, int R, int K, int first, int E, int shared, int tile, void* scratch,
                       int32_t* counts, int32_t* cta_batch, int32_t* cta_limit, int32_t* meta, int32_t* route_map,
                       int32_t* exp2perm, k3moe_stream_t stream) {
  shared = shared ? 1 : 0;
  if (R < 1 || K < 1 || K > 16 || E < 1 || E + shared > 2048 || tile < 1 || tile > 1024) return K3MOE_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int nb = (int)cdiv(R, TB), EL = E + shared;
  int* blockcount = reinterpret_cast<int*>(scratch);
  int* blockoff = reinterpret_cast<int*>(reinterpret_cast<char*>(scratch) + align_up((size_t)nb * EL * 4, 256));
  route_count_kernel<<<nb, TB, EL * 4, s>>>(idx, R, K, first, E, shared, blockcount, nullptr);
  route_tables_kernel<<<1, 1024, 0, s>>>(blockcount, nb, E, shared, tile, blockoff, counts, cta_batch, cta_limit, meta,
                                         route_map);
  const int sc_smem = E * (TB / 32) * 4;
  if (sc_smem > 48 * 1024 && !set_smem_once(route_scatter_kernel, sc_smem, 2)) return K3MOE_ELAUNCH;
  route_scatter_kernel<<<nb, TB, sc_smem, s>>>(idx, R, K, first, E, shared, blockcount, blockoff, route_map, exp2perm);
  return launch_status();
}

int k3moe_quant_mxfp8(const void* x_bf16, int ldx, int rows, int cols, uint8_t* q, uint8_t* sf, int tiled_sf,
                      k3moe_stream_t stream) {
  if (rows < 0 || cols <= 0 || cols % 256 || ldx < cols || ldx % 8) return K3MOE_EINVAL;
  if (rows == 0) return K3MOE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long pieces = (long long)rows * (cols / 256);
  const int grid = (int)std::min<long long>(cdiv(pieces, 8), (long long)num_sms(current_device()) * 16);
  const bf16* x = reinterpret_cast<const bf16*>(x_bf16);
  if (tiled_sf) quant_tiled_kernel<<<grid, 256, 0, s>>>(x, ldx, rows, cols, q, sf);
  else quant_linear_kernel<<<grid, 256, 0, s>>>(x, ldx, rows, cols, q, sf);
  return launch_status();
}

int k3moe_quant_permute(const void* x_bf16, int ldx, int R, int cols, int K, const int32_t* exp2perm,
                        const int32_t* meta, uint8_t* q_perm, uint8_t* sf_perm, k3moe_stream_t stream) {
  if (R < 0 || cols <= 0 || cols % 256 || ldx < cols || ldx % 8 || K < 1 || K > 16) return K3MOE_EINVAL;
  if (R == 0) return K3MOE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int grid = (int)std::min<long long>(cdiv(R, 8), (long long)num_sms(current_device()) * 8);
  quant_permute_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const bf16*>(x_bf16), ldx, R, cols, K, exp2perm, meta,
                                            q_perm, sf_perm);
  return launch_status();
}

int k3moe_fc1(const uint8_t* w13, const uint8_t* w13_sf, const uint8_t* q_perm, const uint8_t* sf_perm,
              const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, uint8_t* fc1_q,
              uint8_t* fc1_sf, int H, int I, int n_experts, int cap_rows, int max_ctas, uint32_t* err,
              k3moe_stream_t stream) {
  return gemm_launch(MODE_FC1, w13, w13_sf, q_perm, sf_perm, cta_batch, cta_limit, meta, fc1_q, fc1_sf, nullptr, H, I,
                     n_experts, cap_rows, max_ctas, err, reinterpret_cast<cudaStream_t>(stream));
}

int k3moe_fc1_act(const uint8_t* w13, const uint8_t* w13_sf, const uint8_t* q_perm, const uint8_t* sf_perm,
                  const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, uint8_t* fc1_q,
                  uint8_t* fc1_sf, int H, int I, int n_experts, int cap_rows, int max_ctas, uint32_t* err,
                  int activation, k3moe_stream_t stream) {
  return gemm_launch(MODE_FC1, w13, w13_sf, q_perm, sf_perm, cta_batch, cta_limit, meta, fc1_q, fc1_sf, nullptr, H, I,
                     n_experts, cap_rows, max_ctas, err, reinterpret_cast<cudaStream_t>(stream), nullptr, activation);
}

int k3moe_fc2(const uint8_t* w2, const uint8_t* w2_sf, const uint8_t* fc1_q, const uint8_t* fc1_sf,
              const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, void* fc2_bf16, int H, int I,
              int n_experts, int cap_rows, int max_ctas, uint32_t* err, k3moe_stream_t stream) {
  return gemm_launch(MODE_FC2, w2, w2_sf, fc1_q, fc1_sf, cta_batch, cta_limit, meta, nullptr, nullptr, fc2_bf16, H, I,
                     n_experts, cap_rows, max_ctas, err, reinterpret_cast<cudaStream_t>(stream));
}

int k3moe_combine(const void* fc2_bf16, const int32_t* exp2perm, const float* wts, const int32_t* meta, void* out_bf16,
                  int ldo, int T, int out_rows, int K, int cols, k3moe_stream_t stream) {
  if (T < 0 || out_rows < T || K < 1 || K > 16 || cols <= 0 || cols % 8 || ldo < cols || ldo % 8) return K3MOE_EINVAL;
  if (out_rows == 0) return K3MOE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  combine_kernel<<<out_rows, 256, 0, s>>>(reinterpret_cast<const bf16*>(fc2_bf16), exp2perm, wts, meta,
                                          reinterpret_cast<bf16*>(out_bf16), ldo, T, K, cols);
  return launch_status();
}

int k3moe_quant_mxfp4(const float* w, long long rows, int K, uint8_t* packed, uint8_t* sf, k3moe_stream_t stream) {
  if (rows < 0 || rows % 128 || K <= 0 || K % 128) return K3MOE_EINVAL;
  if (rows == 0) return K3MOE_OK;
  const long long groups = rows * (K / 32);
  const int grid = (int)std::min<long long>(cdiv(groups, 256), (long long)num_sms(current_device()) * 32);
  quant_mxfp4_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(w, rows, K, packed, sf);
  return launch_status();
}

int k3moe_synth_mxfp4(uint64_t seed, long long row0, long long rows, int K, float sd, uint8_t* packed, uint8_t* sf,
                      k3moe_stream_t stream) {
  if (rows < 0 || rows % 128 || row0 < 0 || K <= 0 || K % 128 || row0 % 128) return K3MOE_EINVAL;
  if (rows == 0) return K3MOE_OK;
  const long long groups = rows * (K / 32);
  const int grid = (int)std::min<long long>(cdiv(groups, 256), (long long)num_sms(current_device()) * 32);
  // the tiled scale offsets are relative to row0 (a multiple of 128): callers pass sf at row0's atom
  synth_mxfp4_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(seed, row0, rows, K, sd, packed, sf);
  return launch_status();
}

int k3moe_router_gemm(const void* x_bf16, int ldx, const void* w_bf16, int ldw, int T, int E, int H, float* S, int lds,
                      uint32_t* err, k3moe_stream_t stream) {
  if (!x_bf16 || !w_bf16 || !S || T < 1 || E < 16 || E % 16 || H < 64 || H % 64 || ldx < H || ldx % 8 ||
      ldw < H || ldw % 8 || lds < E || lds % 4 || reinterpret_cast<uintptr_t>(x_bf16) % 16 ||
      reinterpret_cast<uintptr_t>(w_bf16) % 16 || reinterpret_cast<uintptr_t>(S) % 16)
    return K3MOE_EINVAL;
  // expert columns a unit: the largest multiple of 16 up to 256 dividing E (224 for 896)
  int bn = 16;
  for (int c = rgemm::BN_MAX; c >= 16; c -= 16)
    if (E % c == 0) {
      bn = c;
      break;
    }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return K3MOE_EDRIVER;
  CUtensorMap mx, mw;
  const cuuint32_t estr[2] = {1, 1};
  {
    const cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)T};
    const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
    const cuuint32_t box[2] = {rgemm::BK, rgemm::BM};
    if (fn(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x_bf16), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return K3MOE_ETMAP;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)E};
    const cuuint64_t strides[1] = {(cuuint64_t)ldw * 2};
    const cuuint32_t box[2] = {rgemm::BK, (cuuint32_t)bn};
    if (fn(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w_bf16), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return K3MOE_ETMAP;
  }
  RouterParams p;
  p.S = S;
  p.lds = lds;
  p.T = T;
  p.K = H;
  p.bn = bn;
  p.n_tiles = E / bn;
  p.m_tiles = (int)cdiv(T, rgemm::BM);
  p.err = err;
  const int units = p.m_tiles * p.n_tiles;
  const int grid = std::min(units, num_sms(current_device()));
  if (!set_smem_once(router_gemm_kernel, rgemm::SMEM_BYTES, 3)) return K3MOE_ELAUNCH;
  router_gemm_kernel<<<grid, rgemm::THREADS, rgemm::SMEM_BYTES, reinterpret_cast<cudaStream_t>(stream)>>>(mx, mw, p);
  return launch_status();
}

int k3moe_gemm_tensor_maps(int mode, const uint8_t* w, const uint8_t* act, int n_experts, int H, int I, int cap_rows,
                           void* maps_dev, k3moe_stream_t stream) {
  if ((mode != 0 && mode != 1) || !w || !act || !maps_dev || n_experts < 1 || H < 256 || H % 256 || I < 256 ||
      I % 256 || cap_rows < 128 || cap_rows % 128 || reinterpret_cast<uintptr_t>(maps_dev) % 64)
    return K3MOE_EINVAL;
  const int K = mode == 0 ? H : I;
  const int rows_per_expert = mode == 0 ? 2 * I : H;
  CUtensorMap maps[2];
  static_assert(sizeof(maps) == K3MOE_GEMM_MAPS_BYTES, "the descriptor buffer's size in include/k3moe.h");
  int rc = encode_operand(&maps[0], w, (long long)n_experts * rows_per_expert, K, true);
  if (rc) return rc;
  rc = encode_operand(&maps[1], act, cap_rows, K, false);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(maps_dev, maps, sizeof(maps), cudaMemcpyHostToDevice, s) != cudaSuccess) return K3MOE_ELAUNCH;
  return cudaStreamSynchronize(s) == cudaSuccess ? K3MOE_OK : K3MOE_ELAUNCH;
}

int k3moe_import_mxfp4(const uint8_t* packed_rows, const uint8_t* scale_rows, int experts, int rows_per_expert,
                       int K, int gated, uint8_t* packed, uint8_t* sf, k3moe_stream_t stream) {
  if (experts < 1 || rows_per_expert < 128 || rows_per_expert % 128 || K < 128 || K % 128 || !packed_rows ||
      !scale_rows || !packed || !sf || reinterpret_cast<uintptr_t>(packed_rows) % 16 ||
      reinterpret_cast<uintptr_t>(packed) % 16 || reinterpret_cast<uintptr_t>(scale_rows) % 4 ||
      reinterpret_cast<uintptr_t>(sf) % 4)
    return K3MOE_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long chunks = (long long)experts * rows_per_expert * (K / 32);  // 16-byte chunks (K/2 bytes a row)
  const long long quads = (long long)experts * rows_per_expert * (K / 128);  // 4-byte scale pieces
  kern_k3_moe_w_tiles<<<(unsigned)cdiv(chunks, 256), 256, 0, s>>>(packed_rows, packed, experts, rows_per_expert,
                                                                  K / 2, gated ? 1 : 0);
  kern_k3_moe_sf_tiles<<<(unsigned)cdiv(quads, 256), 256, 0, s>>>(scale_rows, sf, experts, rows_per_expert, K / 32,
                                                                  gated ? 1 : 0);
  return launch_status();
}

size_t k3moe_layer_workspace_size(int T, int H, int I, int E, int K, int shared) {
  if (T < 1 || H < 256 || I < 256 || E < 1 || K < 1) return 0;
  return layer_layout(T, H, I, E, K, shared ? 1 : 0).total;
}

int k3moe_layer_workspace_offsets(int T, int H, int I, int E, int K, int shared, size_t* offsets14) {
  if (T < 1 || H < 256 || I < 256 || E < 1 || K < 1 || !offsets14) return K3MOE_EINVAL;
  const LayerLayout L = layer_layout(T, H, I, E, K, shared ? 1 : 0);
  for (int i = 0; i < 14; ++i) offsets14[i] = L.off[i];
  return K3MOE_OK;
}

int k3moe_layer_forward_events(const k3moe_layer_args* a, void* workspace, size_t ws_bytes, k3moe_stream_t stream,
                               void* const* events, int n_events) {
  if (!a || !workspace || (n_events > 0 && !events)) return K3MOE_EINVAL;
  const int shared = a->shared ? 1 : 0;
  if (a->T < 1 || a->H % 256 || a->I % 256 || a->E < a->K || a->E > 1024 || a->ldx < a->H || a->ldo < a->H)
    return K3MOE_EINVAL;
  const LayerLayout L = layer_layout(a->T, a->H, a->I, a->E, a->K, shared);
  if (ws_bytes < L.total) return K3MOE_ENOSPACE;
  char* ws = reinterpret_cast<char*>(workspace);
  auto I32 = [&](int i) { return reinterpret_cast<int32_t*>(ws + L.off[i]); };
  auto U8 = [&](int i) { return reinterpret_cast<uint8_t*>(ws + L.off[i]); };
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto mark = [&](int i) {
    if (i < n_events && events[i]) cudaEventRecord(reinterpret_cast<cudaEvent_t>(events[i]), s);
  };
  uint32_t* err = reinterpret_cast<uint32_t*>(ws + L.off[L_ERR]);
  if (cudaMemsetAsync(err, 0, 8, s) != cudaSuccess) return K3MOE_ELAUNCH;
  float* wts = reinterpret_cast<float*>(ws + L.off[L_WTS]);
  mark(0);
  int rc = k3moe_route_topk(a->S, a->lds, a->bias, a->rs, a->T, a->E, a->K, I32(L_IDX), wts, stream);
  if (rc) return rc;
  mark(1);
  // the route scratch (block counts / offsets) sits at the end of the layout
  rc = k3moe_route_tables(I32(L_IDX), a->T, a->K, 0, a->E, shared, 128, ws + L.blockcount, I32(L_COUNTS),
                          I32(L_CTA_BATCH), I32(L_CTA_LIMIT), I32(L_META), I32(L_ROUTE_MAP), I32(L_EXP2PERM), stream);
  if (rc) return rc;
  mark(2);
  rc = k3moe_quant_permute(a->x, a->ldx, a->T, a->H, a->K, I32(L_EXP2PERM), I32(L_META), U8(L_QP), U8(L_SFP), stream);
  if (rc) return rc;
  mark(3);
  const int nexp = a->E + shared;
  rc = k3moe_fc1_act(a->w13, a->w13_sf, U8(L_QP), U8(L_SFP), I32(L_CTA_BATCH), I32(L_CTA_LIMIT), I32(L_META),
                     U8(L_FC1Q), U8(L_FC1SF), a->H, a->I, nexp, L.cap_rows, L.max_ctas, err, a->activation, stream);
  if (rc) return rc;
  mark(4);
  rc = k3moe_fc2(a->w2, a->w2_sf, U8(L_FC1Q), U8(L_FC1SF), I32(L_CTA_BATCH), I32(L_CTA_LIMIT), I32(L_META),
                 ws + L.off[L_FC2], a->H, a->I, nexp, L.cap_rows, L.max_ctas, err, stream);
  if (rc) return rc;
  mark(5);
  rc = k3moe_combine(ws + L.off[L_FC2], I32(L_EXP2PERM), wts, I32(L_META), a->out, a->ldo, a->T, a->T, a->K, a->H,
                     stream);
  mark(6);
  return rc;
}

int k3moe_layer_forward(const k3moe_layer_args* a, void* workspace, size_t ws_bytes, k3moe_stream_t stream) {
  return k3moe_layer_forward_events(a, workspace, ws_bytes, stream, nullptr, 0);
}

int k3moe_fc2_to_rows(const uint8_t* w2, const uint8_t* w2_sf, const uint8_t* fc1_q, const uint8_t* fc1_sf,
                      const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, const int32_t* out_rows,
                      void* out_bf16, int H, int I, int n_experts, int cap_rows, int max_ctas, uint32_t* err,
                      k3moe_stream_t stream) {
  if (!out_rows) return K3MOE_EINVAL;
  return gemm_launch(MODE_FC2, w2, w2_sf, fc1_q, fc1_sf, cta_batch, cta_limit, meta, nullptr, nullptr, out_bf16, H, I,
                     n_experts, cap_rows, max_ctas, err, reinterpret_cast<cudaStream_t>(stream), out_rows);
}

int k3moe_fc2_to_ptrs(const uint8_t* w2, const uint8_t* w2_sf, const uint8_t* fc1_q, const uint8_t* fc1_sf,
                      const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, const uint64_t* row_ptrs,
                      int H, int I, int n_experts, int cap_rows, int max_ctas, uint32_t* err, k3moe_stream_t stream) {
  if (!row_ptrs) return K3MOE_EINVAL;
  return gemm_launch(MODE_FC2, w2, w2_sf, fc1_q, fc1_sf, cta_batch, cta_limit, meta, nullptr, nullptr, nullptr, H, I,
                     n_experts, cap_rows, max_ctas, err, reinterpret_cast<cudaStream_t>(stream), nullptr, 0, 0, 0, 0, 0,
                     row_ptrs);
}

int k3moe_fc2_cols(const uint8_t* w2, const uint8_t* w2_sf, const uint8_t* fc1_q, const uint8_t* fc1_sf,
                   const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, const int32_t* out_rows,
                   void* out_bf16, int ldo, int col0, int ncols, int H, int I, int n_experts, int cap_rows,
                   int max_ctas, int grid_cap, uint32_t* err, k3moe_stream_t stream) {
  if (ncols <= 0) return K3MOE_EINVAL;
  return gemm_launch(MODE_FC2, w2, w2_sf, fc1_q, fc1_sf, cta_batch, cta_limit, meta, nullptr, nullptr, out_bf16, H, I,
                     n_experts, cap_rows, max_ctas, err, reinterpret_cast<cudaStream_t>(stream), out_rows, 0, col0,
                     ncols, ldo, grid_cap);
}

int k3moe_ep_row_stride(int H) { return H > 0 && H % 256 == 0 ? (H + H / 32 + 4 + 15) / 16 * 16 : 0; }

int k3moe_ep_pack(const void* x_bf16, int ldx, int T, int H, int K, const int32_t* idx, const int32_t* send_pos,
                  int E_local, int fixed_eid, uint8_t* dst, int stride, k3moe_stream_t stream) {
  if (T < 0 || H <= 0 || H % 256 || ldx < H || ldx % 8 || stride < k3moe_ep_row_stride(H) || stride % 16 ||
      (send_pos && (K < 1 || K > 16 || !idx || E_local < 1)))
    return K3MOE_EINVAL;
  if (T == 0) return K3MOE_OK;
  // several warps a row when there are few rows (a decode step): about four warps an SM in all
  const int sms = num_sms(current_device());
  const int split = (int)std::max<long long>(1, std::min<long long>(H / 256, cdiv(4LL * sms, T)));
  const int grid = (int)std::min<long long>(cdiv((long long)T * split, 8), (long long)sms * 8);
  ep_pack_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const bf16*>(x_bf16), ldx, T, H, K, idx, send_pos, E_local, fixed_eid, dst, stride, split);
  return launch_status();
}

int k3moe_ep_ids(const uint8_t* rows, int stride, int R, int H, int32_t* ids, k3moe_stream_t stream) {
  if (R < 0 || H <= 0 || stride < k3moe_ep_row_stride(H)) return K3MOE_EINVAL;
  if (R == 0) return K3MOE_OK;
  ep_ids_kernel<<<(unsigned)cdiv(R, 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(rows, stride, R, H, ids);
  return launch_status();
}

int k3moe_ep_unpack(const uint8_t* rows, int stride, int R, int H, const int32_t* perm, uint8_t* q_perm,
                    uint8_t* sf_perm, k3moe_stream_t stream) {
  if (R < 0 || H <= 0 || H % 256 || stride < k3moe_ep_row_stride(H) || stride % 16) return K3MOE_EINVAL;
  if (R == 0) return K3MOE_OK;
  const int grid = (int)std::min<long long>(cdiv(R, 8), (long long)num_sms(current_device()) * 8);
  ep_unpack_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(rows, stride, R, H, perm, q_perm, sf_perm);
  return launch_status();
}

int k3moe_ep_pair_row_stride(int H, int K) {
  return H > 0 && H % 256 == 0 && K >= 1 && K <= 16 ? (H + H / 32 + 2 * K + 15) / 16 * 16 : 0;
}

int k3moe_ep_pairs(const int32_t* dest, int T, int K, int W, int32_t* pair_ids, k3moe_stream_t stream) {
  if (T < 0 || K < 1 || K > 16 || W < 1 || W > 32 || !dest || !pair_ids) return K3MOE_EINVAL;
  if (T == 0) return K3MOE_OK;
  const int grid = (int)std::min<long long>(cdiv(T, 256), (long long)num_sms(current_device()) * 4);
  ep_pairs_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(dest, T, K, W, pair_ids);
  return launch_status();
}

int k3moe_ep_pack_pairs(const void* x_bf16, int ldx, int T, int H, int K, const int32_t* dest, const int32_t* lid,
                        const int32_t* pair_pos, int W, int fixed_eid, uint8_t* dst, int stride,
                        k3moe_stream_t stream) {
  if (T < 0 || H <= 0 || H % 256 || ldx < H || ldx % 8 || K < 1 || K > 16 || !dst ||
      stride < k3moe_ep_pair_row_stride(H, K) || stride % 16 || (pair_pos && (W < 1 || W > 32 || !dest || !lid)) ||
      (!pair_pos && (fixed_eid < -32768 || fixed_eid > 32767)))
    return K3MOE_EINVAL;
  if (T == 0) return K3MOE_OK;
  const int sms = num_sms(current_device());
  const int split = (int)std::max<long long>(1, std::min<long long>(H / 256, cdiv(4LL * sms, T)));
  const int grid = (int)std::min<long long>(cdiv((long long)T * split, 8), (long long)sms * 8);
  const int tail = split == 1 ? stride - H : 0;  // one warp a token: row tails built in shared memory
  ep_pack_pairs_kernel<<<grid, 256, 8 * tail, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const bf16*>(x_bf16), ldx, T, H, K, dest, lid, pair_pos, W, fixed_eid, dst, stride, split,
      EpBases{}, 0, -1, nullptr, 0, tail);
  return launch_status();
}

int k3moe_ep_pack_pairs_to(const void* x_bf16, int ldx, int T, int H, int K, const int32_t* dest, const int32_t* lid,
                           const int32_t* pair_pos, int W, const uint64_t* row_base, int stride,
                           k3moe_stream_t stream) {
  if (T < 0 || H <= 0 || H % 256 || ldx < H || ldx % 8 || K < 1 || K > 16 || !dest || !lid || !pair_pos ||
      !row_base || W < 1 || W > EP_MAX_RANKS || stride < k3moe_ep_pair_row_stride(H, K) || stride % 16)
    return K3MOE_EINVAL;
  if (T == 0) return K3MOE_OK;
  EpBases b{};
  for (int d = 0; d < W; ++d) {
    if (row_base[d] % 16) return K3MOE_EINVAL;
    b.base[d] = row_base[d];
  }
  const int sms = num_sms(current_device());
  const int split = (int)std::max<long long>(1, std::min<long long>(H / 256, cdiv(4LL * sms, T)));
  const int grid = (int)std::min<long long>(cdiv((long long)T * split, 8), (long long)sms * 8);
  const int tail = split == 1 ? stride - H : 0;  // one warp a token: row tails built in shared memory
  ep_pack_pairs_kernel<<<grid, 256, 8 * tail, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const bf16*>(x_bf16), ldx, T, H, K, dest, lid, pair_pos, W, 0, nullptr, stride, split, b, 1,
      -1, nullptr, 0, tail);
  return launch_status();
}

int k3moe_ep_row_ptrs(const int32_t* perm, int R, int K, const int32_t* out_rows, int nblocks,
                      const uint64_t* block_base, const int64_t* block_start, int64_t row_bytes, void* sink,
                      uint64_t* row_ptrs, uint32_t* err, k3moe_stream_t stream) {
  if (R < 0 || K < 1 || K > 16 || !perm || !out_rows || !row_ptrs || !sink || nblocks < 1 ||
      nblocks > EP_MAX_RANKS + 1 || !block_base || !block_start || row_bytes <= 0 || row_bytes % 32)
    return K3MOE_EINVAL;
  if (R == 0) return K3MOE_OK;
  EpBases b{};
  for (int s = 0; s < nblocks; ++s) {
    if (block_base[s] % 32 || block_start[s + 1] < block_start[s]) return K3MOE_EINVAL;
    b.base[s] = block_base[s];
    b.start[s] = block_start[s];
  }
  b.start[nblocks] = block_start[nblocks];
  const long long n = (long long)R * K;
  const int grid = (int)std::min<long long>(cdiv(n, 256), (long long)num_sms(current_device()) * 8);
  ep_row_ptrs_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      perm, n, nblocks, out_rows, b, row_bytes, reinterpret_cast<unsigned long long>(sink),
      reinterpret_cast<unsigned long long*>(row_ptrs), err);
  return launch_status();
}

int k3moe_ep_signal(const uint64_t* flag_bases, int W, int me, int slot0, uint32_t epoch, k3moe_stream_t stream) {
  if (!flag_bases || W < 1 || W > EP_MAX_RANKS || me < 0 || me >= W || slot0 < 0) return K3MOE_EINVAL;
  EpBases b{};
  for (int s = 0; s < W; ++s) {
    if (s != me && (flag_bases[s] == 0 || flag_bases[s] % 4)) return K3MOE_EINVAL;
    b.base[s] = flag_bases[s];
  }
  ep_signal_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(b, W, me, slot0, epoch);
  return launch_status();
}

int k3moe_ep_wait(const uint32_t* flags, int W, int skip, uint32_t epoch, uint64_t budget_ns, uint32_t* err,
                  k3moe_stream_t stream) {
  if (!flags || W < 1 || W > 32 || budget_ns == 0) return K3MOE_EINVAL;
  ep_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(flags, W, skip, epoch,
                                                                        (unsigned long long)budget_ns, err);
  return launch_status();
}

int k3moe_ep_ids_k(const uint8_t* rows, int stride, int R, int H, int K, int32_t* ids, k3moe_stream_t stream) {
  if (R < 0 || H <= 0 || H % 256 || K < 1 || K > 16 || stride < k3moe_ep_pair_row_stride(H, K)) return K3MOE_EINVAL;
  if (R == 0) return K3MOE_OK;
  const long long n = (long long)R * K;
  const int grid = (int)std::min<long long>(cdiv(n, 256), (long long)num_sms(current_device()) * 8);
  ep_ids_k_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(rows, stride, R, H, K, ids);
  return launch_status();
}

int k3moe_ep_unpack_k(const uint8_t* rows, int stride, int R, int H, int K, const int32_t* perm, uint8_t* q_perm,
                      uint8_t* sf_perm, k3moe_stream_t stream) {
  if (R < 0 || H <= 0 || H % 256 || K < 1 || K > 16 || stride < k3moe_ep_pair_row_stride(H, K) || stride % 16)
    return K3MOE_EINVAL;
  if (R == 0) return K3MOE_OK;
  const int grid = (int)std::min<long long>(cdiv(R, 8), (long long)num_sms(current_device()) * 8);
  ep_unpack_k_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(rows, stride, R, H, K, perm, q_perm,
                                                                               sf_perm);
  return launch_status();
}

int k3moe_ep_return_rows(const int32_t* perm, int R, int K, int32_t* out_rows, k3moe_stream_t stream) {
  if (R < 0 || K < 1 || K > 16 || !perm || !out_rows) return K3MOE_EINVAL;
  if (R == 0) return K3MOE_OK;
  ep_return_rows_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(perm, R, K, out_rows);
  return launch_status();
}

int k3moe_combine_ep(const void* back_bf16, const int32_t* pos, const float* wts, const void* shared_bf16,
                     int ld_shared, void* out_bf16, int ldo, int T, int K, int cols, k3moe_stream_t stream) {
  if (T < 0 || K < 1 || K > 16 || cols <= 0 || cols % 8 || ldo < cols || ldo % 8 ||
      (shared_bf16 && (ld_shared < cols || ld_shared % 8)))
    return K3MOE_EINVAL;
  if (T == 0) return K3MOE_OK;
  combine_ep_kernel<<<T, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const bf16*>(back_bf16), pos, wts, reinterpret_cast<const bf16*>(shared_bf16), ld_shared,
      reinterpret_cast<bf16*>(out_bf16), ldo, T, K, cols, cols, 0, cols, 0);
  return launch_status();
}

int k3moe_combine_ep_chunked(const void* back_bf16, long long back_chunk_stride, int back_ld, const int32_t* pos,
                             const float* wts, const void* shared_bf16, long long shared_chunk_stride, int ld_shared,
                             void* out_bf16, int ldo, int T, int K, int cols, int chunk_cols, k3moe_stream_t stream) {
  if (T < 0 || K < 1 || K > 16 || cols <= 0 || cols % 8 || ldo < cols || ldo % 8 || chunk_cols <= 0 ||
      chunk_cols % 8 || cols % chunk_cols || back_ld < chunk_cols || back_ld % 8 || back_chunk_stride % 8 ||
      (shared_bf16 && (ld_shared < chunk_cols || ld_shared % 8 || shared_chunk_stride % 8)))
    return K3MOE_EINVAL;
  if (T == 0) return K3MOE_OK;
  combine_ep_kernel<<<T, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const bf16*>(back_bf16), pos, wts, reinterpret_cast<const bf16*>(shared_bf16), ld_shared,
      reinterpret_cast<bf16*>(out_bf16), ldo, T, K, cols, chunk_cols, back_chunk_stride, back_ld,
      shared_chunk_stride);
  return launch_status();
}

int k3moe_ipc_export(const void* dev_ptr, void* handle64, uint64_t* offset) {
  if (!dev_ptr || !handle64 || !offset) return K3MOE_EINVAL;
  AddressRangeFn range = address_range_fn();
  if (!range) return K3MOE_EDRIVER;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return K3MOE_EINVAL;
  cudaIpcMemHandle_t h;
  static_assert(sizeof(h) == 64, "a CUDA IPC handle is 64 bytes");
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return K3MOE_ELAUNCH;
  std::memcpy(handle64, &h, sizeof(h));
  *offset = (uint64_t)(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return K3MOE_OK;
}

int k3moe_ipc_import(const void* handle64, uint64_t offset, void** dev_ptr) {
  if (!handle64 || !dev_ptr) return K3MOE_EINVAL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return K3MOE_ELAUNCH;
  *dev_ptr = static_cast<char*>(p) + offset;
  return K3MOE_OK;
}

int k3moe_ipc_release(void* dev_ptr, uint64_t offset) {
  if (!dev_ptr) return K3MOE_EINVAL;
  return cudaIpcCloseMemHandle(static_cast<char*>(dev_ptr) - offset) == cudaSuccess ? K3MOE_OK : K3MOE_ELAUNCH;
}

int k3moe_set_trace(uint64_t* counters) {
  g_trace = reinterpret_cast<unsigned long long*>(counters);
  return K3MOE_OK;
}

int k3moe_read_error(uint32_t* err, uint32_t* out2, int clear, k3moe_stream_t stream) {
  if (!err || !out2) return K3MOE_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(out2, err, 8, cudaMemcpyDeviceToHost, s) != cudaSuccess) return K3MOE_ELAUNCH;
  if (clear && cudaMemsetAsync(err, 0, 8, s) != cudaSuccess) return K3MOE_ELAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return K3MOE_ELAUNCH;
  return (out2[0] | out2[1]) ? K3MOE_EDEVICE : K3MOE_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- the device-resident expert-parallel step
namespace {

struct EpPeerLayout {
  long long stride, back_col, recv_off, back_off, counts_off, flags_off, total;
};

EpPeerLayout ep_peer_layout(const k3moe_ep_config& c) {
  EpPeerLayout L;
  L.back_col = ((long long)c.H + c.H / 32 + 2LL * c.K + 3) / 4 * 4;  // the int32 after the ids, 4-byte aligned
  L.stride = (L.back_col + 4 + 15) / 16 * 16;
  L.recv_off = 0;
  L.back_off = (long long)align_up((size_t)(c.world + 1) * c.max_tokens * L.stride, 256);
  L.counts_off = L.back_off + (long long)align_up((size_t)c.max_tokens * c.K * c.H * 2, 256);
  L.flags_off = L.counts_off + 256;
  L.total = L.flags_off + 256;
  return L;
}

enum { EW_EPOCH, EW_ERR, EW_OWNER, EW_LOCAL, EW_IDX, EW_WTS, EW_DEST, EW_LID, EW_SEND_POS, EW_PAIR_POS, EW_PAIR_BACK,
       EW_ROWS_TO, EW_IDS, EW_COUNTS, EW_CTA_BATCH, EW_CTA_LIMIT, EW_META, EW_ROUTE_MAP, EW_EXP2PERM, EW_SCRATCH,
       EW_QP, EW_SFP, EW_FC1Q, EW_FC1SF, EW_PTRS, EW_SHARED, EW_N };

struct EpWsLayout {
  size_t off[EW_N];
  size_t total;
  int El, nexp, R_all, max_ctas, cap_rows;
};

EpWsLayout ep_ws_layout(const k3moe_ep_config& c) {
  EpWsLayout L;
  const int W = c.world, T = c.max_tokens, K = c.K;
  L.El = c.E / W;
  L.nexp = L.El + (c.shared ? 1 : 0);
  L.R_all = (W + 1) * T;
  // permuted rows: the picks a rank can receive (every source's every pick, at most one a local expert) and
  // its own shared rows, padded to 128 an expert
  const long long picks = (long long)W * T * std::min(K, L.El) + (c.shared ? T : 0);
  L.max_ctas = (int)(L.nexp + cdiv(picks, 128));
  L.cap_rows = L.max_ctas * 128;
  size_t at = 0;
  auto take = [&](size_t bytes) {
    const size_t o = at;
    at = align_up(at + bytes, 1024);
    return o;
  };
  L.off[EW_EPOCH] = take(16);
  L.off[EW_ERR] = take(16);
  L.off[EW_OWNER] = take((size_t)c.E * 4);
  L.off[EW_LOCAL] = take((size_t)c.E * 4);
  L.off[EW_IDX] = take((size_t)T * K * 4);
  L.off[EW_WTS] = take((size_t)T * K * 4);
  L.off[EW_DEST] = take((size_t)T * K * 4);
  L.off[EW_LID] = take((size_t)T * K * 4);
  L.off[EW_SEND_POS] = take((size_t)T * K * 4);
  L.off[EW_PAIR_POS] = take((size_t)T * W * 4);
  L.off[EW_PAIR_BACK] = take((size_t)T * W * 4);
  L.off[EW_ROWS_TO] = take((size_t)(W + 1) * 4);
  L.off[EW_IDS] = take((size_t)L.R_all * K * 4);
  L.off[EW_COUNTS] = take((size_t)L.nexp * 4);
  L.off[EW_CTA_BATCH] = take((size_t)L.max_ctas * 4);
  L.off[EW_CTA_LIMIT] = take((size_t)L.max_ctas * 4);
  L.off[EW_META] = take(16);
  L.off[EW_ROUTE_MAP] = take((size_t)L.cap_rows * 4);
  L.off[EW_EXP2PERM] = take((size_t)L.R_all * K * 4);
  L.off[EW_SCRATCH] = take(k3moe_route_scratch_bytes(L.R_all, L.nexp, 0));
  L.off[EW_QP] = take((size_t)L.cap_rows * c.H);
  L.off[EW_SFP] = take((size_t)L.cap_rows * c.H / 32);
  L.off[EW_FC1Q] = take((size_t)L.cap_rows * c.I);
  L.off[EW_FC1SF] = take((size_t)L.cap_rows * c.I / 32);
  L.off[EW_PTRS] = take((size_t)L.cap_rows * 8);
  L.off[EW_SHARED] = take((size_t)(T + 1) * c.H * 2);  // the last row: the sink of a bad return index
  L.total = at;
  return L;
}

bool ep_config_ok(const k3moe_ep_config* c) {
  return c && c->world >= 1 && c->world <= EP_MAX_RANKS && c->rank >= 0 && c->rank < c->world && c->H > 0 &&
         c->H % 256 == 0 && c->I > 0 && c->I % 256 == 0 && c->E >= 1 && c->E <= 1024 && c->E % c->world == 0 &&
         c->K >= 1 && c->K <= 16 && (c->K & (c->K - 1)) == 0 && c->K <= c->E && c->max_tokens >= 1 &&
         c->max_tokens <= 65536 && (c->activation == 0 || c->activation == 1) &&
         (long long)(c->world + 1) * c->max_tokens * c->K < (1LL << 31);
}

}  // namespace

struct k3moe_ep {
  k3moe_ep_config c;
  EpPeerLayout P;
  EpWsLayout L;
  char* ws;
  uint8_t* peer;
  const uint8_t *w13, *w13_sf, *w2, *w2_sf;
  EpBases recv_base;  // [d < W]: rank d's region of this rank's rows; [W]: this rank's shared region
  EpBases back_base;  // [s]: rank s's return buffer
  EpBases peer_base;  // [s]: rank s's peer buffer
  bool use_owner;
};

extern "C" {

size_t k3moe_ep_peer_bytes(const k3moe_ep_config* c) {
  return ep_config_ok(c) ? (size_t)ep_peer_layout(*c).total : 0;
}

size_t k3moe_ep_workspace_bytes(const k3moe_ep_config* c) { return ep_config_ok(c) ? ep_ws_layout(*c).total : 0; }

int k3moe_ep_create(const k3moe_ep_config* c, const int32_t* owner, const uint8_t* w13, const uint8_t* w13_sf,
                    const uint8_t* w2, const uint8_t* w2_sf, void* peer_buffer, const uint64_t* peer_bases,
                    void* workspace, size_t ws_bytes, k3moe_stream_t stream, k3moe_ep** out) {
  if (!ep_config_ok(c) || !out || !w13 || !w13_sf || !w2 || !w2_sf || !peer_buffer || !peer_bases || !workspace)
    return K3MOE_EINVAL;
  const EpPeerLayout P = ep_peer_layout(*c);
  const EpWsLayout L = ep_ws_layout(*c);
  if (ws_bytes < L.total) return K3MOE_ENOSPACE;
  if (reinterpret_cast<uintptr_t>(peer_buffer) % 256 || reinterpret_cast<uintptr_t>(workspace) % 256 ||
      peer_bases[c->rank] != reinterpret_cast<uint64_t>(peer_buffer))
    return K3MOE_EINVAL;
  for (int s = 0; s < c->world; ++s)
    if (peer_bases[s] == 0 || peer_bases[s] % 256) return K3MOE_EINVAL;
  const int El = c->E / c->world;
  std::vector<int32_t> own(c->E), loc(c->E);
  if (owner) {
    std::vector<int> seen(c->world, 0);
    for (int e = 0; e < c->E; ++e) {
      if (owner[e] < 0 || owner[e] >= c->world) return K3MOE_EINVAL;
      own[e] = owner[e];
      loc[e] = seen[owner[e]]++;
    }
    for (int r = 0; r < c->world; ++r)
      if (seen[r] != El) return K3MOE_EINVAL;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = reinterpret_cast<char*>(workspace);
  uint8_t* pb = reinterpret_cast<uint8_t*>(peer_buffer);
  if (cudaMemsetAsync(ws + L.off[EW_EPOCH], 0, 16, s) != cudaSuccess ||
      cudaMemsetAsync(ws + L.off[EW_ERR], 0, 16, s) != cudaSuccess ||
      cudaMemsetAsync(pb + P.counts_off, 0, (size_t)(P.total - P.counts_off), s) != cudaSuccess)
    return K3MOE_ELAUNCH;
  if (owner && (cudaMemcpyAsync(ws + L.off[EW_OWNER], own.data(), (size_t)c->E * 4, cudaMemcpyHostToDevice, s) !=
                    cudaSuccess ||
                cudaMemcpyAsync(ws + L.off[EW_LOCAL], loc.data(), (size_t)c->E * 4, cudaMemcpyHostToDevice, s) !=
                    cudaSuccess))
    return K3MOE_ELAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return K3MOE_ELAUNCH;
  // kernel attributes now, so that a later stream capture needs none
  if (!set_smem_once(grouped_gemm_kernel<MODE_FC1>, gemm::SMEM_BYTES, 0) ||
      !set_smem_once(grouped_gemm_kernel<MODE_FC2>, gemm::SMEM_BYTES, 1))
    return K3MOE_ELAUNCH;
  const int sc_smem = L.nexp * (TB / 32) * 4;
  if (sc_smem > 48 * 1024 && !set_smem_once(route_scatter_kernel, sc_smem, 2)) return K3MOE_ELAUNCH;
  k3moe_ep* ep = new k3moe_ep();
  ep->c = *c;
  if (ep->c.wait_budget_ns == 0) ep->c.wait_budget_ns = 5000000000ull;
  ep->P = P;
  ep->L = L;
  ep->ws = ws;
  ep->peer = pb;
  ep->w13 = w13;
  ep->w13_sf = w13_sf;
  ep->w2 = w2;
  ep->w2_sf = w2_sf;
  ep->use_owner = owner != nullptr;
  for (int d = 0; d < c->world; ++d) {
    ep->recv_base.base[d] = peer_bases[d] + (uint64_t)P.recv_off + (uint64_t)c->rank * c->max_tokens * P.stride;
    ep->back_base.base[d] = peer_bases[d] + (uint64_t)P.back_off;
    ep->peer_base.base[d] = peer_bases[d];
  }
  ep->recv_base.base[c->world] = peer_bases[c->rank] + (uint64_t)P.recv_off + (uint64_t)c->world * c->max_tokens * P.stride;
  *out = ep;
  return launch_status();
}

int k3moe_ep_forward_events(k3moe_ep* ep, const float* S, int lds, const float* bias, const void* rs_bf16,
                            const void* x_bf16, int ldx, int T, void* out_bf16, int ldo, k3moe_stream_t stream,
                            void* const* events, int n_events) {
  if (!ep || !S || !bias || !rs_bf16 || !x_bf16 || !out_bf16 || (n_events > 0 && !events)) return K3MOE_EINVAL;
  const k3moe_ep_config& c = ep->c;
  const EpPeerLayout& P = ep->P;
  const EpWsLayout& L = ep->L;
  if (T < 1 || T > c.max_tokens || lds < c.E || ldx < c.H || ldx % 8 || ldo < c.H || ldo % 8) return K3MOE_EINVAL;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = ep->ws;
  auto I32 = [&](int i) { return reinterpret_cast<int32_t*>(ws + L.off[i]); };
  auto U8 = [&](int i) { return reinterpret_cast<uint8_t*>(ws + L.off[i]); };
  auto mark = [&](int i) {
    if (i < n_events && events[i]) cudaEventRecord(reinterpret_cast<cudaEvent_t>(events[i]), s);
  };
  const int W = c.world, me = c.rank, K = c.K, H = c.H;
  u32* err = reinterpret_cast<u32*>(ws + L.off[EW_ERR]);
  u32* epoch = reinterpret_cast<u32*>(ws + L.off[EW_EPOCH]);
  u32* counts = reinterpret_cast<u32*>(ep->peer + P.counts_off);
  const int sms = num_sms(current_device());
  mark(0);
  int rc = k3moe_route_topk(S, lds, bias, rs_bf16, T, c.E, K, I32(EW_IDX), reinterpret_cast<float*>(ws + L.off[EW_WTS]),
                            stream);
  if (rc) return rc;
  ep_plan_kernel<<<1, PLAN_THREADS, 0, s>>>(I32(EW_IDX), T, K, W, L.El, ep->use_owner ? I32(EW_OWNER) : nullptr,
                                            ep->use_owner ? I32(EW_LOCAL) : nullptr, I32(EW_DEST), I32(EW_LID),
                                            I32(EW_PAIR_POS), I32(EW_PAIR_BACK), I32(EW_SEND_POS), I32(EW_ROWS_TO),
                                            epoch, counts + W, c.shared ? T : 0, c.E, err);
  mark(1);
  {
    const int split = (int)std::max<long long>(1, std::min<long long>(H / 256, cdiv(4LL * sms, T)));
    const int grid = (int)std::min<long long>(cdiv((long long)T * split, 8), (long long)sms * 8);
    const int tail = split == 1 ? (int)P.stride - H : 0;  // one warp a token: row tails in shared memory
    ep_pack_pairs_kernel<<<grid, 256, 8 * tail, s>>>(reinterpret_cast<const bf16*>(x_bf16), ldx, T, H, K,
                                                     I32(EW_DEST), I32(EW_LID), I32(EW_PAIR_POS), W, 0, nullptr,
                                                     (int)P.stride, split, ep->recv_base, 1, c.shared ? L.El : -1,
                                                     I32(EW_PAIR_BACK), (int)P.back_col, tail);
  }
  ep_exchange_kernel<<<1, 32, 0, s>>>(ep->peer_base, P.counts_off, P.flags_off, W, me, 0, I32(EW_ROWS_TO), epoch,
                                      (unsigned long long)c.wait_budget_ns, err);
  mark(2);
  const uint8_t* rows = ep->peer + P.recv_off;
  {
    const long long n = (long long)L.R_all * K;
    const int grid = (int)std::min<long long>(cdiv(n, 256), (long long)sms * 8);
    ep_ids_k_kernel<<<grid, 256, 0, s>>>(rows, (int)P.stride, L.R_all, H, K, I32(EW_IDS), counts, c.max_tokens);
  }
  rc = k3moe_route_tables(I32(EW_IDS), L.R_all, K, 0, L.nexp, 0, 128, ws + L.off[EW_SCRATCH], I32(EW_COUNTS),
                          I32(EW_CTA_BATCH), I32(EW_CTA_LIMIT), I32(EW_META), I32(EW_ROUTE_MAP), I32(EW_EXP2PERM),
                          stream);
  if (rc) return rc;
  {
    const int grid = (int)std::min<long long>(cdiv(L.R_all, 8), (long long)sms * 8);
    ep_unpack_k_kernel<<<grid, 256, 0, s>>>(rows, (int)P.stride, L.R_all, H, K, I32(EW_EXP2PERM), U8(EW_QP),
                                            U8(EW_SFP));
  }
  mark(3);
  rc = gemm_launch(MODE_FC1, ep->w13, ep->w13_sf, U8(EW_QP), U8(EW_SFP), I32(EW_CTA_BATCH), I32(EW_CTA_LIMIT),
                   I32(EW_META), U8(EW_FC1Q), U8(EW_FC1SF), nullptr, H, c.I, L.nexp, L.cap_rows, L.max_ctas, err, s,
                   nullptr, c.activation);
  if (rc) return rc;
  mark(4);
  {
    const long long n = (long long)L.R_all * K;
    const int grid = (int)std::min<long long>(cdiv(n, 256), (long long)sms * 8);
    const unsigned long long shared_rows = reinterpret_cast<unsigned long long>(ws + L.off[EW_SHARED]);
    ep_step_ptrs_kernel<<<grid, 256, 0, s>>>(I32(EW_EXP2PERM), n, K, rows, (int)P.stride, (int)P.back_col,
                                             c.max_tokens, W, ep->back_base, (long long)c.max_tokens * K, shared_rows,
                                             2LL * H, shared_rows + 2ull * H * c.max_tokens,
                                             reinterpret_cast<unsigned long long*>(ws + L.off[EW_PTRS]), err);
  }
  rc = gemm_launch(MODE_FC2, ep->w2, ep->w2_sf, U8(EW_FC1Q), U8(EW_FC1SF), I32(EW_CTA_BATCH), I32(EW_CTA_LIMIT),
                   I32(EW_META), nullptr, nullptr, nullptr, H, c.I, L.nexp, L.cap_rows, L.max_ctas, err, s, nullptr,
                   0, 0, 0, 0, 0, reinterpret_cast<const uint64_t*>(ws + L.off[EW_PTRS]));
  if (rc) return rc;
  mark(5);
  ep_exchange_kernel<<<1, 32, 0, s>>>(ep->peer_base, P.counts_off, P.flags_off, W, me, 1, nullptr, epoch,
                                      (unsigned long long)c.wait_budget_ns, err);
  mark(6);
  combine_ep_kernel<<<T, 256, 0, s>>>(reinterpret_cast<const bf16*>(ep->peer + P.back_off), I32(EW_SEND_POS),
                                      reinterpret_cast<const float*>(ws + L.off[EW_WTS]),
                                      c.shared ? reinterpret_cast<const bf16*>(ws + L.off[EW_SHARED]) : nullptr, H,
                                      reinterpret_cast<bf16*>(out_bf16), ldo, T, K, H, H, 0, H, 0);
  mark(7);
  return launch_status();
}

int k3moe_ep_forward(k3moe_ep* ep, const float* S, int lds, const float* bias, const void* rs_bf16,
                     const void* x_bf16, int ldx, int T, void* out_bf16, int ldo, k3moe_stream_t stream) {
  return k3moe_ep_forward_events(ep, S, lds, bias, rs_bf16, x_bf16, ldx, T, out_bf16, ldo, stream, nullptr, 0);
}

uint32_t* k3moe_ep_errors(k3moe_ep* ep) { return ep ? reinterpret_cast<uint32_t*>(ep->ws + ep->L.off[EW_ERR]) : nullptr; }

const uint32_t* k3moe_ep_counts(k3moe_ep* ep) {
  return ep ? reinterpret_cast<const uint32_t*>(ep->peer + ep->P.counts_off) : nullptr;
}

const int32_t* k3moe_ep_expert_rows(k3moe_ep* ep) {
  return ep ? reinterpret_cast<const int32_t*>(ep->ws + ep->L.off[EW_COUNTS]) : nullptr;
}

const int32_t* k3moe_ep_meta(k3moe_ep* ep) {
  return ep ? reinterpret_cast<const int32_t*>(ep->ws + ep->L.off[EW_META]) : nullptr;
}

void k3moe_ep_destroy(k3moe_ep* ep) { delete ep; }

}  // extern "C"

#include "noalloc.cu"
