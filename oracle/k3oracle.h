/* k3oracle — CPU restatement of the Kimi-K3 routed-MoE path, TEST
 * INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load this library; the product (libk3moe.so) never does.
 *
 * Each function names the reference code it restates (paths inside the
 * reference project).  Pins: the router top-k against golden vectors made by
 * the reference's own CPU reference (harness/k3/ref.h, see
 * tests/golden/make_golden.py); the byte-level stages (quantisation, tables,
 * combine) against the reference's kernels built from source and run on the
 * GPU box (oracle/_ref, tests/test_gpu_ref.py).  The MXFP4 weight quantiser
 * and the GEMM rounding chain have no reference code (parity unpinned there;
 * the GEMMs are compared with tolerances). */
#ifndef K3ORACLE_H
#define K3ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* number formats */
float orc_bf16_to_f32(uint16_t b);
uint16_t orc_f32_to_bf16(float f);           /* round to nearest even */
uint8_t orc_f32_to_e4m3_sat(float f);        /* RNE, saturate to +-448, NaN -> 0x7f|sign */
float orc_e4m3_to_f32(uint8_t b);
float orc_e2m1_to_f32(uint8_t nibble);
int orc_mx8_exponent(float amax);            /* ceil(log2(amax/448)) clamped, 0 for amax 0 */
int orc_mx8_exponent_ocp(float amax);        /* FC1's output: floor(log2(amax)) - 8 clamped, -127 for 0 */
long long orc_sf_tiled_offset(long long r, int kb, int kg4);
/* tile-major GEMM operands (128 x 128-element tiles, tile (r/128, k/128) at
 * index (r/128)*(K/128) + k/128, row-major inside): byte of E4M3 element (r, k),
 * byte of packed E2M1 element (r, k) */
long long orc_op8_offset(long long r, int k, int K);
long long orc_op4_offset(long long r, int k, int K);

/* router top-k: source/k3_moe_route.cu:117-221, 372-385; source/k3_prefill_glue.cu:504-557 */
void orc_topk(const float* S, int lds, const float* bias, uint16_t rs_bits, int T, int E, int K, int32_t* idx,
              float* wts);

/* routing tables: source/k3_moe_prefill.cu:97-204 (row order within an expert,
 * as source/k3_moe_route.cu:39-44, 496-519) */
void orc_tables(const int32_t* idx, int R, int K, int first, int E, int shared, int tile, int32_t* counts,
                int32_t* cta_batch, int32_t* cta_limit, int32_t* meta, int32_t* route_map, int32_t* exp2perm);

/* MXFP8: source/k3_moe_prefill.cu:66-95 (linear sf), source/k3_mxfp8.cu:20-54 (tiled sf) */
void orc_quant_mxfp8(const uint16_t* x, int ldx, int rows, int cols, uint8_t* q, uint8_t* sf, int tiled);
/* the same, written to permuted rows (exp2perm and the shared expert's rows) */
void orc_quant_permute(const uint16_t* x, int ldx, int R, int cols, int K, const int32_t* exp2perm,
                       const int32_t* meta, uint8_t* q_perm, uint8_t* sf_perm);

/* MXFP4 weights (OCP MX rule; no reference code) */
void orc_quant_mxfp4(const float* w, long long rows, int K, uint8_t* packed, uint8_t* sf);
void orc_synth_f32(uint64_t seed, long long row0, long long rows, int K, float sd, float* out);

/* combine: source/k3_moe_prefill.cu:206-234 */
void orc_combine(const uint16_t* fc2, const int32_t* exp2perm, const float* wts, const int32_t* meta, uint16_t* out,
                 int ldo, int T, int out_rows, int K, int cols);

/* FC1 / FC2 over the tables: fp32 dequantise-and-matmul of the same quantised
 * operands (the reference GEMMs are closed cubins; their family, run through
 * FlashInfer's TRT-LLM-gen MoE on the same operands, pins this restatement:
 * oracle/flashinfer_ref.py, tests/test_gpu_flashinfer_ref.py).
 * Rows of tiles c in [c0, c1) only.  fc1: the gate, then MXFP8 with the OCP
 * exponent rule (orc_mx8_exponent_ocp), the reference FC1's. */
void orc_fc1(const uint8_t* w13, const uint8_t* w13_sf, const uint8_t* q_perm, const uint8_t* sf_perm,
             const int32_t* cta_batch, const int32_t* cta_limit, int c0, int c1, int H, int I, uint8_t* fc1_q,
             uint8_t* fc1_sf);
/* act: 0 SwiGLU, 1 K3's SiTU (harness/k3/ref.h:97-101) */
void orc_fc1_act(const uint8_t* w13, const uint8_t* w13_sf, const uint8_t* q_perm, const uint8_t* sf_perm,
                 const int32_t* cta_batch, const int32_t* cta_limit, int c0, int c1, int H, int I, uint8_t* fc1_q,
                 uint8_t* fc1_sf, int act);
void orc_fc2(const uint8_t* w2, const uint8_t* w2_sf, const uint8_t* fc1_q, const uint8_t* fc1_sf,
             const int32_t* cta_batch, const int32_t* cta_limit, int c0, int c1, int H, int I, uint16_t* fc2);

/* threads the OpenMP loops may use (0 = the runtime default); returns the count in effect */
int orc_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
