/* k3oracle exact stages — TEST INFRASTRUCTURE ONLY (see k3oracle.h).
 * Compiled with -ffp-contract=off: every float operation is the single IEEE
 * operation written, so the bit-exact stages mirror the device rounding. */
#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

#include "k3oracle.h"

float orc_bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

uint16_t orc_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)(((u >> 16) & 0x8000u) | 0x7fc0u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* E4M3 (bias 7, no infinities, max 448 = 1.75 * 2^8): nearest even, saturating. */
uint8_t orc_f32_to_e4m3_sat(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
  if (isnan(f)) return (uint8_t)(sign | 0x7f);
  const float a = fabsf(f);
  if (a >= 448.0f) return (uint8_t)(sign | 0x7e);
  if (a < 0.015625f) { /* below 2^-6: the subnormal grid k * 2^-9, k = 0..8 (8 is 2^-6) */
    const float k = rintf(a * 512.0f);
    return (uint8_t)(sign | (uint8_t)k);
  }
  int ex;
  frexpf(a, &ex); /* a = m * 2^ex, m in [0.5, 1) -> a in [2^(ex-1), 2^ex) */
  int e = ex - 1; /* -6 .. 8 */
  int mi = (int)rintf(ldexpf(a, 3 - e)); /* 8 .. 16: 3 fraction bits, exact scaling */
  if (mi == 16) {
    mi = 8;
    ++e;
  }
  if (e > 8 || (e == 8 && mi > 14)) return (uint8_t)(sign | 0x7e);
  return (uint8_t)(sign | (uint8_t)((e + 7) << 3) | (uint8_t)(mi - 8));
}

float orc_e4m3_to_f32(uint8_t b) {
  const int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
  float v;
  if (e == 15 && m == 7) return NAN;
  if (e == 0) v = ldexpf((float)m, -9);
  else v = ldexpf((float)(8 + m), e - 10);
  return s ? -v : v;
}

float orc_e2m1_to_f32(uint8_t nib) {
  static const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float v = mag[nib & 7];
  return (nib & 8) ? -v : v;
}

/* e = ceil(log2(amax / 448)) with the quotient rounded to f32 first (as the
 * kernels divide in f32); exact: a power of two gives its exponent, anything
 * else the next one up. */
int orc_mx8_exponent(float amax) {
  if (!(amax > 0.f)) return 0;
  const float y = amax / 448.0f;
  int ex;
  const float m = frexpf(y, &ex); /* y = m * 2^ex, m in [0.5, 1) */
  int e = (m == 0.5f) ? ex - 1 : ex;
  if (e < -127) e = -127;
  if (e > 127) e = 127;
  return e;
}

/* FC1's output rule (the reference's TRT-LLM-gen FC1): OCP MX, e = floor(log2(amax)) - 8, clamped; zero and
 * subnormal amax give -127.  frexp: amax = m 2^ex with m in [0.5, 1), so floor(log2(amax)) = ex - 1. */
int orc_mx8_exponent_ocp(float amax) {
  if (!(amax >= 1.17549435e-38f)) return -127;
  int ex;
  frexpf(amax, &ex);
  int e = ex - 1 - 8;
  if (e < -127) e = -127;
  if (e > 127) e = 127;
  return e;
}

long long orc_sf_tiled_offset(long long r, int kb, int kg4) {
  return ((r / 128) * kg4 + kb / 4) * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + kb % 4;
}

long long orc_op8_offset(long long r, int k, int K) {
  return ((r / 128) * (K / 128) + k / 128) * 16384 + (r % 128) * 128 + k % 128;
}

long long orc_op4_offset(long long r, int k, int K) {
  return ((r / 128) * (K / 128) + k / 128) * 8192 + (r % 128) * 64 + (k % 128) / 2;
}

static uint32_t ord_f32(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

/* Restates source/k3_prefill_glue.cu:504-557 / source/k3_moe_route.cu:117-221,
 * 372-385: sig = 1/(1 + expf(-s)); keys sig + bias; K largest, ties to the
 * smaller expert; wts = sig / (xor-butterfly sum over the K picks + 1e-20) * rs. */
void orc_topk(const float* S, int lds, const float* bias, uint16_t rs_bits, int T, int E, int K, int32_t* idx,
              float* wts) {
  const float rsv = orc_bf16_to_f32(rs_bits);
#pragma omp parallel
  {
    float* sig = (float*)malloc(sizeof(float) * E);
    uint32_t* key = (uint32_t*)malloc(sizeof(uint32_t) * E);
#pragma omp for schedule(static)
    for (int t = 0; t < T; ++t) {
      for (int e = 0; e < E; ++e) {
        const float sg = 1.0f / (1.0f + expf(-S[(size_t)t * lds + e]));
        sig[e] = sg;
        key[e] = ord_f32(sg + bias[e]);
      }
      int pe[16];
      float pw[16], v[16], nv[16];
      for (int r = 0; r < K; ++r) {
        int best = -1;
        for (int e = 0; e < E; ++e)
          if (key[e] != 0u && (best < 0 || key[e] > key[best])) best = e;
        pe[r] = best;
        pw[r] = sig[best];
        key[best] = 0u;
      }
      for (int r = 0; r < K; ++r) v[r] = pw[r];
      for (int o = K / 2; o > 0; o >>= 1) {
        for (int r = 0; r < K; ++r) nv[r] = v[r] + v[r ^ o];
        for (int r = 0; r < K; ++r) v[r] = nv[r];
      }
      const float den = v[0];
      for (int r = 0; r < K; ++r) {
        idx[(size_t)t * K + r] = pe[r];
        wts[(size_t)t * K + r] = (pw[r] / (den + 1e-20f)) * rsv;
      }
    }
    free(sig);
    free(key);
  }
}

/* Restates source/k3_moe_prefill.cu:97-204 with the row order of
 * source/k3_moe_route.cu:496-519: counts; ctas = ceil(count/tile) scanned
 * into offsets; cta_batch / cta_limit; padding rows route row 0; a pick's
 * permuted row is its expert's offset plus the earlier rows that picked it. */
void orc_tables(const int32_t* idx, int R, int K, int first, int E, int shared, int tile, int32_t* counts,
                int32_t* cta_batch, int32_t* cta_limit, int32_t* meta, int32_t* route_map, int32_t* exp2perm) {
  const int EL = E + (shared ? 1 : 0);
  int* off = (int*)calloc((size_t)EL + 1, sizeof(int));
  int* fill = (int*)calloc((size_t)EL, sizeof(int));
  for (int e = 0; e < EL; ++e) counts[e] = 0;
  for (long long i = 0; i < (long long)R * K; ++i) {
    const int e = idx[i] - first;
    if (e >= 0 && e < E) counts[e]++;
  }
  if (shared) counts[E] = R;
  for (int e = 0; e < EL; ++e) off[e + 1] = off[e] + (counts[e] + tile - 1) / tile;
  meta[0] = off[EL];
  meta[1] = off[EL] * tile;
  meta[2] = shared ? off[E] * tile : -1;
  for (int e = 0; e < EL; ++e) {
    for (int c = off[e]; c < off[e + 1]; ++c) {
      cta_batch[c] = e;
      const int lim = off[e] * tile + counts[e];
      cta_limit[c] = (c + 1) * tile < lim ? (c + 1) * tile : lim;
    }
    for (int r = off[e] * tile + counts[e]; r < off[e + 1] * tile; ++r) route_map[r] = 0;
  }
  for (int r = 0; r < R; ++r) {
    for (int k = 0; k < K; ++k) {
      const int e = idx[(size_t)r * K + k] - first;
      if (e < 0 || e >= E) {
        exp2perm[(size_t)r * K + k] = -1;
        continue;
      }
      const int row = off[e] * tile + fill[e]++;
      exp2perm[(size_t)r * K + k] = row;
      route_map[row] = r;
    }
    if (shared) route_map[off[E] * tile + r] = r;
  }
  free(off);
  free(fill);
}

/* one 32-element group: the scale byte and 32 E4M3 bytes */
static uint8_t quant_group(const uint16_t* x, uint8_t* q) {
  float amax = 0.f;
  for (int j = 0; j < 32; ++j) {
    const float a = fabsf(orc_bf16_to_f32(x[j]));
    if (a > amax) amax = a;
  }
  const int e = orc_mx8_exponent(amax);
  const float s = ldexpf(1.0f, -e); /* exact: 2^-e, e in [-127, 127] */
  for (int j = 0; j < 32; ++j) q[j] = orc_f32_to_e4m3_sat(orc_bf16_to_f32(x[j]) * s);
  return (uint8_t)(e + 127);
}

/* Restates source/k3_moe_prefill.cu:66-95 (tiled = 0) and source/k3_mxfp8.cu:20-54 (tiled = 1). */
void orc_quant_mxfp8(const uint16_t* x, int ldx, int rows, int cols, uint8_t* q, uint8_t* sf, int tiled) {
  const int kbn = cols / 32, kg4 = (kbn + 3) / 4;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; ++r)
    for (int kb = 0; kb < kbn; ++kb) {
      const uint8_t s = quant_group(x + (size_t)r * ldx + kb * 32, q + (size_t)r * cols + kb * 32);
      if (tiled) sf[orc_sf_tiled_offset(r, kb, kg4)] = s;
      else sf[(size_t)r * kbn + kb] = s;
    }
}

void orc_quant_permute(const uint16_t* x, int ldx, int R, int cols, int K, const int32_t* exp2perm,
                       const int32_t* meta, uint8_t* q_perm, uint8_t* sf_perm) {
  const int kbn = cols / 32, kg4 = (kbn + 3) / 4;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < R; ++r) {
    int dst[17], nd = 0;
    for (int k = 0; k < K; ++k)
      if (exp2perm[(size_t)r * K + k] >= 0) dst[nd++] = exp2perm[(size_t)r * K + k];
    if (meta[2] >= 0) dst[nd++] = meta[2] + r;
    uint8_t qg[32];
    for (int kb = 0; kb < kbn; ++kb) {
      const uint8_t s = quant_group(x + (size_t)r * ldx + kb * 32, qg);
      for (int d = 0; d < nd; ++d) {
        memcpy(q_perm + orc_op8_offset(dst[d], kb * 32, cols), qg, 32);
        sf_perm[orc_sf_tiled_offset(dst[d], kb, kg4)] = s;
      }
    }
  }
}

/* OCP MX, E2M1 elements: X = floor(log2 amax) - 2 (clamped to [-127, 127],
 * -127 for amax 0), elements v / 2^X rounded to the nearest point of
 * {0, .5, 1, 1.5, 2, 3, 4, 6} (ties to the even code), saturating at 6. */
static uint8_t e2m1_round(float y) {
  static const float grid[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float a = fabsf(y);
  int best = 0;
  for (int c = 1; c < 8; ++c) {
    const float dc = fabsf(a - grid[c]), db = fabsf(a - grid[best]);
    if (dc < db || (dc == db && (c & 1) == 0)) best = c;
  }
  if (a > 6.f) best = 7;
  return (uint8_t)((y < 0.f ? 8 : 0) | best);
}

void orc_quant_mxfp4(const float* w, long long rows, int K, uint8_t* packed, uint8_t* sf) {
  const int kbn = K / 32, kg4 = (kbn + 3) / 4;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < rows; ++r)
    for (int kb = 0; kb < kbn; ++kb) {
      const float* v = w + r * K + kb * 32;
      float amax = 0.f;
      for (int j = 0; j < 32; ++j)
        if (fabsf(v[j]) > amax) amax = fabsf(v[j]);
      int X = -127;
      if (amax > 0.f) {
        int ex;
        frexpf(amax, &ex); /* amax in [2^(ex-1), 2^ex) */
        X = ex - 1 - 2;
        if (X < -127) X = -127;
        if (X > 127) X = 127;
      }
      uint8_t* out = packed + orc_op4_offset(r, kb * 32, K);
      for (int j = 0; j < 16; ++j) {
        const uint8_t lo = e2m1_round(ldexpf(v[2 * j], -X));
        const uint8_t hi = e2m1_round(ldexpf(v[2 * j + 1], -X));
        out[j] = (uint8_t)(lo | (hi << 4));
      }
      sf[orc_sf_tiled_offset(r, kb, kg4)] = (uint8_t)(X + 127);
    }
}

static uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* The synthetic weight stream of k3moe_synth_mxfp4 (input generation, not an
 * algorithm): an Irwin-Hall(4) draw from splitmix64(seed, r, c), std sd. */
void orc_synth_f32(uint64_t seed, long long row0, long long rows, int K, float sd, float* out) {
  const float scale = sd * 1.7320508f / 16777216.0f;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < rows; ++r)
    for (int c = 0; c < K; ++c) {
      const uint64_t h1 = splitmix64(seed * 0x100000001B3ull ^ ((uint64_t)(row0 + r) << 20) ^ (uint64_t)c);
      const uint64_t h2 = splitmix64(h1);
      const long long s = (long long)(h1 & 0xFFFFFF) + (long long)((h1 >> 32) & 0xFFFFFF) +
                          (long long)(h2 & 0xFFFFFF) + (long long)((h2 >> 32) & 0xFFFFFF) - (2ll << 24);
      out[r * K + c] = (float)s * scale;
    }
}

/* Restates source/k3_moe_prefill.cu:206-234: f32 FMA in k order over the local
 * picks, then the shared expert's row (weight 1); rows past T are zero. */
void orc_combine(const uint16_t* fc2, const int32_t* exp2perm, const float* wts, const int32_t* meta, uint16_t* out,
                 int ldo, int T, int out_rows, int K, int cols) {
  const int sb = meta ? meta[2] : -1;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < out_rows; ++t) {
    for (int c = 0; c < cols; ++c) {
      float acc = 0.f;
      if (t < T) {
        for (int k = 0; k < K; ++k) {
          const int p = exp2perm[(size_t)t * K + k];
          if (p < 0) continue;
          acc = fmaf(wts[(size_t)t * K + k], orc_bf16_to_f32(fc2[(size_t)p * cols + c]), acc);
        }
        if (sb >= 0) acc = fmaf(1.0f, orc_bf16_to_f32(fc2[(size_t)(sb + t) * cols + c]), acc);
      }
      out[(size_t)t * ldo + c] = orc_f32_to_bf16(acc);
    }
  }
}

int orc_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
}
