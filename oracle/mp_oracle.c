/*
 * TEST INFRASTRUCTURE — the CPU oracle for the projection hot path. Only the
 * tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this;
 * the product path never does.
 *
 * A plain-C, fp64 restatement of what one projection of the Ming-Image DiT
 * computes in the reference (vpipe-ming-image, paths relative to it):
 *
 *   y[m, n] = sum_k x[m, k] * deq(W)[n, k]
 *           + sum over live slots i of s_i * sum_j (sum_k x[m, k] A_i[j, k]) B_i[n, j]
 *
 *   - `lin` = lin_base + lora::Applier::apply      src/ming-dit.cc:1763-1771
 *   - biasless block projections                    src/ming-dit.cc:454-456
 *   - live slots: bound and strength != 0           src/ming-dit.cc:3007-3022
 *                                                   (lora::Stack::add drops 0)
 *   - alpha folded into A ("W x + scale * B (A x)") src/ming-dit.cc:2845-2851,
 *                                                   src/ming-model-config-stage.cc:48-63
 *   - packed weight = U32 codes [N, K*bits/32] + scales/biases [N, K/64]
 *                                                   src/ming-dit.cc:802-831,
 *                                                   tests/ming-quant-test.cc:526-530
 *
 * PARITY PARTLY UNPINNED. The dequant kernels (affine_dequant_w{4,8}g64,
 * affine_qmm_steel_w{4,8}g64) belong to the vpipe host SDK, which is not in
 * the reference tree, and no golden vector for them exists there. The rule
 * restated here is the one the reference's tensor names and shapes imply
 * (MLX-style affine, codes LSB-first in each U32 word):
 *       w[n, k] = scale[n, k/64] * q[n, k] + bias[n, k/64],
 *       q[n, k] = (codes[n][k*bits/32] >> ((k % (32/bits)) * bits)) & (2^bits - 1).
 * The signed-symmetric 8-bit mode (not a reference format)
 * reads the same byte as a two's-complement int8 and has no bias.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

double mpo_bf16_to_f64(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return (double)f;
}

/* Round-to-nearest-even float -> bf16 bits (NaN kept quiet). */
uint16_t mpo_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* codes U32 [n, k*bits/32] -> integer code values q [n, k]. For symmetric
 * 8-bit codes the value is the signed byte. */
void mpo_unpack_codes(const uint32_t* codes, int n, int k, int bits, int symmetric, int32_t* q) {
  const int per = 32 / bits;
  const int words = k / per;
  const uint32_t mask = (1u << bits) - 1u;
  for (int r = 0; r < n; ++r) {
    for (int c = 0; c < k; ++c) {
      const uint32_t w = codes[(size_t)r * words + c / per];
      const uint32_t v = (w >> ((c % per) * bits)) & mask;
      q[(size_t)r * k + c] = symmetric ? (int32_t)(int8_t)(uint8_t)v : (int32_t)v;
    }
  }
}

/* q [n, k] -> codes U32 [n, k*bits/32], LSB first. */
void mpo_pack_codes(const int32_t* q, int n, int k, int bits, uint32_t* codes) {
  const int per = 32 / bits;
  const int words = k / per;
  const uint32_t mask = (1u << bits) - 1u;
  for (int r = 0; r < n; ++r) {
    for (int wi = 0; wi < words; ++wi) {
      uint32_t w = 0;
      for (int j = 0; j < per; ++j)
        w |= ((uint32_t)q[(size_t)r * k + wi * per + j] & mask) << (j * bits);
      codes[(size_t)r * words + wi] = w;
    }
  }
}

/* Dequantized weight in fp64: bits 0 = dense bf16 `data`. */
void mpo_dequant(const void* data, const uint16_t* scales, const uint16_t* biases, int n, int k,
                 int bits, int symmetric, double* w) {
  if (bits == 0) {
    const uint16_t* d = (const uint16_t*)data;
    for (size_t i = 0; i < (size_t)n * k; ++i) w[i] = mpo_bf16_to_f64(d[i]);
    return;
  }
  int32_t* q = (int32_t*)malloc(sizeof(int32_t) * (size_t)n * k);
  mpo_unpack_codes((const uint32_t*)data, n, k, bits, symmetric, q);
  const int g = k / 64;
  for (int r = 0; r < n; ++r) {
    for (int c = 0; c < k; ++c) {
      const double s = mpo_bf16_to_f64(scales[(size_t)r * g + c / 64]);
      const double b = biases ? mpo_bf16_to_f64(biases[(size_t)r * g + c / 64]) : 0.0;
      w[(size_t)r * k + c] = s * (double)q[(size_t)r * k + c] + b;
    }
  }
  free(q);
}

/*
 * The projection for rows [0, m) of x (bf16, leading dimension ldx), fp64
 * throughout. `n_slots` adapters: a[i] bf16 [rank[i], k], b[i] bf16
 * [n, rank[i]], strength s[i] (a slot with strength exactly 0 contributes
 * nothing, as the reference's Stack::add drops it). Output y fp64 [m, n].
 */
void mpo_projection(const uint16_t* x, int64_t ldx, int m, const void* data,
                    const uint16_t* scales, const uint16_t* biases, int n, int k, int bits,
                    int symmetric, int n_slots, const uint16_t* const* a,
                    const uint16_t* const* b, const int32_t* rank, const double* s, double* y) {
  double* w = (double*)malloc(sizeof(double) * (size_t)n * k);
  mpo_dequant(data, scales, biases, n, k, bits, symmetric, w);
  double* xr = (double*)malloc(sizeof(double) * (size_t)m * k);
  for (int r = 0; r < m; ++r)
    for (int c = 0; c < k; ++c) xr[(size_t)r * k + c] = mpo_bf16_to_f64(x[(size_t)r * ldx + c]);
#pragma omp parallel for schedule(static)
  for (int r = 0; r < m; ++r) {
    const double* xrow = xr + (size_t)r * k;
    for (int c = 0; c < n; ++c) {
      const double* wrow = w + (size_t)c * k;
      double acc = 0.0;
      for (int i = 0; i < k; ++i) acc += xrow[i] * wrow[i];
      y[(size_t)r * n + c] = acc;
    }
    for (int sl = 0; sl < n_slots; ++sl) {
      if (s[sl] == 0.0 || rank[sl] <= 0) continue;
      const int rk = rank[sl];
      double t[1024];
      for (int j = 0; j < rk; ++j) {
        double acc = 0.0;
        for (int i = 0; i < k; ++i) acc += xrow[i] * mpo_bf16_to_f64(a[sl][(size_t)j * k + i]);
        t[j] = acc * s[sl];
      }
      for (int c = 0; c < n; ++c) {
        double acc = 0.0;
        for (int j = 0; j < rk; ++j) acc += t[j] * mpo_bf16_to_f64(b[sl][(size_t)c * rk + j]);
        y[(size_t)r * n + c] += acc;
      }
    }
  }
  free(xr);
  free(w);
}

/*
 * Batched adaLN modulation of one block, fp64: mods = W temb + bias
 * (reference fill_mod, src/ming-dit.cc:2266-2273). temb bf16 [m, k].
 */
void mpo_modulation(const uint16_t* temb, int m, const void* data, const uint16_t* scales,
                    const uint16_t* biases, const uint16_t* bias, int n, int k, int bits,
                    int symmetric, double* mods) {
  double* w = (double*)malloc(sizeof(double) * (size_t)n * k);
  mpo_dequant(data, scales, biases, n, k, bits, symmetric, w);
  for (int r = 0; r < m; ++r) {
    for (int c = 0; c < n; ++c) {
      double acc = 0.0;
      for (int i = 0; i < k; ++i)
        acc += mpo_bf16_to_f64(temb[(size_t)r * k + i]) * w[(size_t)c * k + i];
      mods[(size_t)r * n + c] = acc + mpo_bf16_to_f64(bias[c]);
    }
  }
  free(w);
}

int mpo_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
