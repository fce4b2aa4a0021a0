/* k3oracle GEMM stages — TEST INFRASTRUCTURE ONLY (see k3oracle.h).
 * fp32 dequantise-and-matmul of the quantised operands the device GEMMs read:
 * weights MXFP4 (E2M1 * 2^(sf-127)), activations MXFP8 (E4M3 * 2^(sf-127)),
 * both exact in f32; f32 dot products (vectorised partial sums).  The device
 * accumulates in a different order, so these stages are compared with
 * tolerances, never bit for bit. */
#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#include "k3oracle.h"

static float ue8m0(uint8_t s) { return s == 255 ? NAN : ldexpf(1.0f, (int)s - 127); }

/* weight row r (flattened over experts) of K elements -> f32 */
static void dequant_w_row(const uint8_t* w, const uint8_t* w_sf, long long r, int K, float* out) {
  const int kg4 = (K / 32 + 3) / 4;
  for (int kb = 0; kb < K / 32; ++kb) {
    const float s = ue8m0(w_sf[orc_sf_tiled_offset(r, kb, kg4)]);
    const uint8_t* grp = w + orc_op4_offset(r, kb * 32, K);
    for (int j = 0; j < 16; ++j) {
      const uint8_t b = grp[j];
      out[kb * 32 + 2 * j] = orc_e2m1_to_f32(b & 15) * s;
      out[kb * 32 + 2 * j + 1] = orc_e2m1_to_f32(b >> 4) * s;
    }
  }
}

/* permuted activation row p of K elements (E4M3 + tiled sf) -> f32 */
static void dequant_a_row(const uint8_t* q, const uint8_t* sf, long long p, int K, float* out) {
  const int kg4 = (K / 32 + 3) / 4;
  for (int kb = 0; kb < K / 32; ++kb) {
    const float s = ue8m0(sf[orc_sf_tiled_offset(p, kb, kg4)]);
    const uint8_t* grp = q + orc_op8_offset(p, kb * 32, K);
    for (int j = 0; j < 32; ++j) out[kb * 32 + j] = orc_e4m3_to_f32(grp[j]) * s;
  }
}

static float dot(const float* a, const float* b, int n) {
  float acc[16] = {0};
  int i = 0;
  for (; i + 16 <= n; i += 16)
    for (int j = 0; j < 16; ++j) acc[j] += a[i + j] * b[i + j];
  float s = 0.f;
  for (int j = 0; j < 16; ++j) s += acc[j];
  for (; i < n; ++i) s += a[i] * b[i];
  return s;
}

/* the gate: 0 SwiGLU silu(g) * u; 1 K3's SiTU 4 tanh(g/4) sigmoid(g) * 25 tanh(u/25)
 * (harness/k3/ref.h:97-101), in double */
static float gated_act(float g, float u, int act) {
  const double gd = g, ud = u, sg = 1.0 / (1.0 + exp(-gd));
  if (act == 0) return (float)(gd * sg * ud);
  return (float)(4.0 * tanh(gd / 4.0) * sg * 25.0 * tanh(ud / 25.0));
}

void orc_fc1(const uint8_t* w13, const uint8_t* w13_sf, const uint8_t* q_perm, const uint8_t* sf_perm,
             const int32_t* cta_batch, const int32_t* cta_limit, int c0, int c1, int H, int I, uint8_t* fc1_q,
             uint8_t* fc1_sf) {
  orc_fc1_act(w13, w13_sf, q_perm, sf_perm, cta_batch, cta_limit, c0, c1, H, I, fc1_q, fc1_sf, 0);
}

/* Every tile c in [c0, c1): expert e = cta_batch[c], rows [128c, cta_limit[c]). */
void orc_fc1_act(const uint8_t* w13, const uint8_t* w13_sf, const uint8_t* q_perm, const uint8_t* sf_perm,
                 const int32_t* cta_batch, const int32_t* cta_limit, int c0, int c1, int H, int I, uint8_t* fc1_q,
                 uint8_t* fc1_sf, int act) {
  const int kg4_out = (I / 32 + 3) / 4;
  for (int c = c0; c < c1; ++c) {
    const int e = cta_batch[c], row0 = c * 128, n = cta_limit[c] - row0;
    if (n <= 0) continue;
    float* xa = (float*)malloc(sizeof(float) * (size_t)n * H);
    float* h = (float*)malloc(sizeof(float) * (size_t)n * I);
    for (int j = 0; j < n; ++j) dequant_a_row(q_perm, sf_perm, row0 + j, H, xa + (size_t)j * H);
#pragma omp parallel
    {
      float* wg = (float*)malloc(sizeof(float) * H);
      float* wu = (float*)malloc(sizeof(float) * H);
#pragma omp for schedule(static)
      for (int f = 0; f < I; ++f) {
        dequant_w_row(w13, w13_sf, (long long)e * 2 * I + f, H, wg);
        dequant_w_row(w13, w13_sf, (long long)e * 2 * I + I + f, H, wu);
        for (int j = 0; j < n; ++j) {
          const float g = dot(wg, xa + (size_t)j * H, H);
          const float u = dot(wu, xa + (size_t)j * H, H);
          h[(size_t)j * I + f] = gated_act(g, u, act);
        }
      }
      free(wg);
      free(wu);
    }
    for (int j = 0; j < n; ++j)
      for (int kb = 0; kb < I / 32; ++kb) {
        float amax = 0.f;
        for (int i = 0; i < 32; ++i) {
          const float a = fabsf(h[(size_t)j * I + kb * 32 + i]);
          if (a > amax) amax = a;
        }
        const int ex = orc_mx8_exponent_ocp(amax);
        const float s = ldexpf(1.0f, -ex);
        uint8_t* grp = fc1_q + orc_op8_offset(row0 + j, kb * 32, I);
        for (int i = 0; i < 32; ++i) grp[i] = orc_f32_to_e4m3_sat(h[(size_t)j * I + kb * 32 + i] * s);
        fc1_sf[orc_sf_tiled_offset(row0 + j, kb, kg4_out)] = (uint8_t)(ex + 127);
      }
    free(xa);
    free(h);
  }
}

void orc_fc2(const uint8_t* w2, const uint8_t* w2_sf, const uint8_t* fc1_q, const uint8_t* fc1_sf,
             const int32_t* cta_batch, const int32_t* cta_limit, int c0, int c1, int H, int I, uint16_t* fc2) {
  for (int c = c0; c < c1; ++c) {
    const int e = cta_batch[c], row0 = c * 128, n = cta_limit[c] - row0;
    if (n <= 0) continue;
    float* act = (float*)malloc(sizeof(float) * (size_t)n * I);
    for (int j = 0; j < n; ++j) dequant_a_row(fc1_q, fc1_sf, row0 + j, I, act + (size_t)j * I);
#pragma omp parallel
    {
      float* wr = (float*)malloc(sizeof(float) * I);
#pragma omp for schedule(static)
      for (int o = 0; o < H; ++o) {
        dequant_w_row(w2, w2_sf, (long long)e * H + o, I, wr);
        for (int j = 0; j < n; ++j) fc2[(size_t)(row0 + j) * H + o] = orc_f32_to_bf16(dot(wr, act + (size_t)j * I, I));
      }
      free(wr);
    }
    free(act);
  }
}
