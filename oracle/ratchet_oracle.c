/*
 * ratchet_oracle.c — CPU restatement of the reference ratchet-linear hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product package links or calls this file; it is the
 * checker for the CUDA kernels (tests/, __graft_entry__.smoke()) and the timed CPU baseline of
 * bench.py.  It is pinned against golden vectors produced by the reference itself
 * (tests/golden/make_golden.py).
 *
 * Every function cites the reference code (LoomNode/local-ai-training, src/local_ai_training/)
 * whose arithmetic it restates.  Where the reference leaves an order unspecified (a row sum), the
 * order is the one the CUDA kernels use, described at canonical_sum(), so that CUDA and oracle
 * agree bit for bit; against the reference the same rows agree up to that order.
 *
 * Build: gcc -O2 -ffp-contract=off -fno-fast-math -fPIC -shared (see oracle/build.py).
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

/* ---------- bf16 round-to-nearest-even (torch .to(torch.bfloat16)) ---------- */
float or_bf16_round(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
    u |= 0x00400000u; /* quiet NaN */
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
  }
  u &= 0xffff0000u;
  memcpy(&f, &u, 4);
  return f;
}

/* ---------- Philox4x32-10 (Salmon et al., SC'11) ---------- */
void or_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
  uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
  uint32_t k0 = key_in[0], k1 = key_in[1];
  const uint32_t A = 0xD2511F53u, B = 0xCD9E8D57u;
  for (int r = 0; r < 10; ++r) {
    const uint64_t pb = (uint64_t)B * c2, pa = (uint64_t)A * c0;
    const uint32_t n0 = (uint32_t)(pb >> 32) ^ c1 ^ k0;
    const uint32_t n2 = (uint32_t)(pa >> 32) ^ c3 ^ k1;
    c0 = n0;
    c1 = (uint32_t)pb;
    c2 = n2;
    c3 = (uint32_t)pa;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  out[0] = c0, out[1] = c1, out[2] = c2, out[3] = c3;
}

/* This library's stochastic-rounding draw for linear element index e (see the header of the
 * CUDA library): 16-bit half (e & 1) (0 = low) of word ((e & 7) >> 1) of
 * Philox(ctr = (e>>3, (e>>3)>>32, step, "RATC"), key = (seed, (seed>>32) ^ layer)), mapped to
 * u = (h + 1/2) * 2^-16.  The reference draws tl.rand(seed, m*K + n) with a fresh host seed per
 * call (int8_matmul.py:143-145, 200); its stream is not reproducible, so only the distribution
 * of the rounding is shared. */
float or_sr_uniform(uint64_t seed, uint32_t step, uint32_t layer, uint64_t e) {
  const uint64_t block = e >> 3;
  const uint32_t ctr[4] = {(uint32_t)block, (uint32_t)(block >> 32), step, 0x52415443u};
  const uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32) ^ layer};
  uint32_t out[4];
  or_philox4x32_10(ctr, key, out);
  const uint32_t word = out[(e & 7) >> 1];
  const uint32_t h = (e & 1) ? (word >> 16) : (word & 0xFFFFu);
  return (float)(2u * h + 1u) * 7.62939453125e-06f; /* 2^-17, exact */
}

/* ---------- canonical row sum ----------
 * The row is cut into 8-element chunks (chunk c = elements 8c..8c+7).
 *   level 1: 256 partials T_t (t = 0..255); T_t adds the elements of chunks c = t (mod 256) in
 *            increasing index order, starting from +0.0f;
 *   level 2: 32 partials S_s = ((T_s + T_s+32) + (T_s+64 + T_s+96)) + ((T_s+128 + T_s+160) +
 *            (T_s+192 + T_s+224));
 *   level 3: xor butterfly over S_0..S_31 (offsets 16, 8, 4, 2, 1); the result is lane 0's value.
 * All arithmetic fp32 round-to-nearest.  A warp per row (each lane keeping 8 level-1 partials) and
 * a CTA per row (one partial per thread) both realise this order exactly. */
static float canonical_sum(const float *terms, int64_t n) {
  float T[256];
  for (int i = 0; i < 256; ++i) T[i] = 0.0f;
  const int64_t chunks = (n + 7) / 8;
  for (int64_t c = 0; c < chunks; ++c)
    for (int j = 0; j < 8; ++j) {
      const int64_t i = 8 * c + j;
      if (i < n) T[c % 256] = T[c % 256] + terms[i];
    }
  float v[32], nv[32];
  for (int s = 0; s < 32; ++s) {
    const float a = T[s] + T[s + 32], b = T[s + 64] + T[s + 96];
    const float c = T[s + 128] + T[s + 160], d = T[s + 192] + T[s + 224];
    v[s] = (a + b) + (c + d);
  }
  for (int o = 16; o > 0; o >>= 1) {
    for (int l = 0; l < 32; ++l) nv[l] = v[l] + v[l ^ o];
    for (int l = 0; l < 32; ++l) v[l] = nv[l];
  }
  return v[0];
}

/* ---------- row quantisation: int8_matmul.py:82-84, 106-150, 225-239 ----------
 * x: (rows, cols) fp32 values (bf16 inputs are passed widened, exactly). */
void or_quantize_rows(const float *x, int64_t rows, int64_t cols, const float *col_scale,
                      int stochastic, uint64_t seed, uint32_t step, uint32_t layer, int8_t *q,
                      float *scale_out) {
  for (int64_t r = 0; r < rows; ++r) {
    float amax = 0.0f;
    for (int64_t k = 0; k < cols; ++k) {
      float v = x[r * cols + k];
      if (col_scale) v = v * col_scale[k];
      const float a = fabsf(v);
      if (a > amax) amax = a;
    }
    float scale = amax / 127.0f;
    if (scale < FLT_MIN) scale = FLT_MIN;
    scale_out[r] = scale;
    for (int64_t k = 0; k < cols; ++k) {
      float v = x[r * cols + k];
      if (col_scale) v = v * col_scale[k];
      float rq;
      if (stochastic) {
        const float u = or_sr_uniform(seed, step, layer, (uint64_t)(r * cols + k));
        const float y = v / scale;
        rq = floorf(y + u);
      } else {
        rq = rintf(v / scale);
      }
      if (rq < -127.0f) rq = -127.0f;
      if (rq > 127.0f) rq = 127.0f;
      q[r * cols + k] = (int8_t)(int)rq;
    }
  }
}

/* ---------- scaled int8 GEMM: int8_matmul.py:64-79 ----------
 * lhs (M,K), rhs (K,N) row-major; out = bf16((float(acc) * ls[m]) * rs[n]) returned as fp32. */
void or_scaled_int8_mm(const int8_t *lhs, const int8_t *rhs, const float *ls, const float *rs,
                       int64_t M, int64_t N, int64_t K, float *out, int32_t *acc_out) {
  for (int64_t m = 0; m < M; ++m)
    for (int64_t n = 0; n < N; ++n) {
      int32_t acc = 0;
      for (int64_t k = 0; k < K; ++k) acc += (int32_t)lhs[m * K + k] * (int32_t)rhs[k * N + n];
      if (acc_out) acc_out[m * N + n] = acc;
      float v = (float)acc * ls[m];
      if (rs) v = v * rs[n];
      out[m * N + n] = or_bf16_round(v);
    }
}

/* ---------- activation dequant for grad_weight: ratchet.py:73-76 ---------- */
void or_dequant_rows(const int8_t *q, const float *s, int64_t rows, int64_t cols, float *out) {
  for (int64_t r = 0; r < rows; ++r) {
    const float sb = or_bf16_round(s[r]);
    for (int64_t k = 0; k < cols; ++k) out[r * cols + k] = or_bf16_round((float)q[r * cols + k] * sb);
  }
}

/* ---------- grad_weight: ratchet.py:148-163 ----------
 * gw[n,k] = sum_m g[m,n] * x[m,k], accumulated in double (an order-free reference for the
 * tolerance checks of the fp32-accumulating tensor-core GEMM). */
void or_grad_weight(const float *g, const float *x, int64_t Mt, int64_t N, int64_t K, float *out) {
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k) {
      double acc = 0.0;
      for (int64_t m = 0; m < Mt; ++m) acc += (double)g[m * N + n] * (double)x[m * K + k];
      out[n * K + k] = (float)acc;
    }
}

/* ---------- ratchet update: ratchet.py:185-199 (nibbles), 248-262 (bucket), 265-301 (core),
 *            539-556 (_normalize), 487-537 (per-row statistics) ---------- */
static uint8_t ratchet_one(uint8_t old, float z, int max_code, int T, float low, float high,
                           int64_t counts[4]) {
  const float mag = fabsf(z);
  const int bucket = mag >= high ? 2 : (mag >= low ? 1 : 0);
  const int sgn = (z > 0.0f) - (z < 0.0f);
  const int inc = -sgn * bucket;
  int code = (int)(old & 0x0F) - max_code;
  int p = (int)(old >> 4) - 7 + inc;
  const int pos_req = p >= T, neg_req = p <= -T;
  const int pos_mv = pos_req && code < max_code, neg_mv = neg_req && code > -max_code;
  code += pos_mv - neg_mv;
  p -= pos_req * T;
  p += neg_req * T;
  if (p < -128) p = -128;
  if (p > 127) p = 127;
  counts[0] += pos_mv;
  counts[1] += neg_mv;
  counts[2] += pos_req && !pos_mv;
  counts[3] += neg_req && !neg_mv;
  return (uint8_t)(((code + max_code) & 0x0F) | (((p + 7) & 0x0F) << 4));
}

/* grad: (rows, cols) fp32 values; round_bf16 applies the bf16 rounding of the reference's
 * bf16 GEMM output first.  normalize == 0 treats grad as already normalised
 * (apply_normalized_gradient).  Returns the number of rows skipped for NaN/Inf. */
int64_t or_ratchet_update(const float *grad, int round_bf16, int64_t rows, int64_t cols,
                          uint8_t *packed, int8_t *code_out, int normalize, float *rms_ema,
                          double beta, int max_code, int T, double bucket_low, double bucket_high,
                          double eps, int64_t counts[4], float *row_rms, float *grad_scale,
                          float *scratch /* 2*cols floats */) {
  const float low = (float)bucket_low, high = (float)bucket_high, epsf = (float)eps;
  const float betaf = (float)beta, ombf = (float)(1.0 - beta);
  int64_t skipped = 0;
  float *g = scratch, *terms = scratch + cols;
  for (int64_t r = 0; r < rows; ++r) {
    int bad = 0;
    for (int64_t k = 0; k < cols; ++k) {
      float v = grad[r * cols + k];
      if (round_bf16) v = or_bf16_round(v);
      g[k] = v;
      if (!isfinite(v)) bad = 1;
    }
    for (int64_t k = 0; k < cols; ++k) terms[k] = g[k] * g[k];
    const float ms = canonical_sum(terms, cols) / (float)cols;
    float gs = 0.0f;
    if (grad_scale) {
      for (int64_t k = 0; k < cols; ++k)
        terms[k] = g[k] * (float)((int)(packed[r * cols + k] & 0x0F) - max_code);
      gs = canonical_sum(terms, cols);
      grad_scale[r] = gs;
    }
    float denom_rms = sqrtf(ms);
    if (rms_ema && beta > 0.0 && !bad) {
      const float ema_old = rms_ema[r];
      const float upd = ema_old == 0.0f ? ms : betaf * ema_old + ombf * ms;
      const float ema = ms > 0.0f ? upd : ema_old;
      rms_ema[r] = ema;
      denom_rms = sqrtf(ema);
    }
    const float denom = denom_rms + epsf;
    if (row_rms) row_rms[r] = sqrtf(ms);
    if (bad) {
      ++skipped;
    } else {
      for (int64_t k = 0; k < cols; ++k) {
        const float z = normalize ? g[k] / denom : g[k];
        packed[r * cols + k] = ratchet_one(packed[r * cols + k], z, max_code, T, low, high, counts);
      }
    }
    if (code_out)
      for (int64_t k = 0; k < cols; ++k)
        code_out[r * cols + k] = (int8_t)((int)(packed[r * cols + k] & 0x0F) - max_code);
  }
  return skipped;
}

/* pressure leak: ratchet.py:613-625 */
void or_ratchet_leak(uint8_t *packed, int64_t n) {
  for (int64_t i = 0; i < n; ++i) {
    const uint8_t v = packed[i];
    int p = (int)(v >> 4) - 7;
    p -= (p > 0) - (p < 0);
    packed[i] = (uint8_t)((v & 0x0F) | (((p + 7) & 0x0F) << 4));
  }
}

/* ---------- fused producers: int8_fused.py, int8_backward.py ---------- */
/* y = (x * r) * w, r = 1 / sqrt(mean(x^2) + eps) with IEEE sqrt/division, then RN row quant. */
void or_rmsnorm_quantize(const float *x, const float *w, double eps, int64_t rows, int64_t cols,
                         int8_t *q, float *scale_out, float *scratch /* cols */) {
  const float epsf = (float)eps;
  for (int64_t r = 0; r < rows; ++r) {
    const float *xr = x + r * cols;
    for (int64_t k = 0; k < cols; ++k) scratch[k] = xr[k] * xr[k];
    const float var = canonical_sum(scratch, cols) / (float)cols;
    const float rr = 1.0f / sqrtf(var + epsf);
    for (int64_t k = 0; k < cols; ++k) scratch[k] = (xr[k] * rr) * w[k];
    or_quantize_rows(scratch, 1, cols, 0, 0, 0, 0, 0, q + r * cols, scale_out + r);
  }
}

static float gelu_tanh(float x) {
  const float c = 0.7978845608028654f;
  const float cube = ((0.044715f * x) * x) * x;
  const float inner = c * (x + cube);
  const float th = tanhf(inner);
  return (0.5f * x) * (1.0f + th);
}

void or_gelu_quantize(const float *x, int64_t rows, int64_t cols, int8_t *q, float *scale_out,
                      float *scratch /* cols */) {
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t k = 0; k < cols; ++k) scratch[k] = gelu_tanh(x[r * cols + k]);
    or_quantize_rows(scratch, 1, cols, 0, 0, 0, 0, 0, q + r * cols, scale_out + r);
  }
}

void or_rmsnorm_backward(const float *gy, const float *x, const float *w, double eps, int64_t rows,
                         int64_t cols, float *dx, float *scratch /* cols */) {
  const float epsf = (float)eps;
  for (int64_t r = 0; r < rows; ++r) {
    const float *xr = x + r * cols, *gr = gy + r * cols;
    for (int64_t k = 0; k < cols; ++k) scratch[k] = xr[k] * xr[k];
    const float var = canonical_sum(scratch, cols) / (float)cols;
    for (int64_t k = 0; k < cols; ++k) scratch[k] = (gr[k] * w[k]) * xr[k];
    const float dsum = canonical_sum(scratch, cols);
    const float rr = 1.0f / sqrtf(var + epsf);
    const float dvar = (dsum * -0.5f) * ((rr * rr) * rr);
    for (int64_t k = 0; k < cols; ++k) {
      const float dh = gr[k] * w[k];
      dx[r * cols + k] = or_bf16_round(dh * rr + ((dvar * 2.0f) * xr[k]) / (float)cols);
    }
  }
}

void or_gelu_backward(const float *gy, const float *x, int64_t n, float *dx) {
  const float c = 0.7978845608028654f;
  for (int64_t i = 0; i < n; ++i) {
    const float xv = x[i];
    const float x2 = xv * xv;
    const float inner = c * (xv + (0.044715f * xv) * x2);
    const float th = tanhf(inner);
    const float t1 = 0.5f * (1.0f + th);
    const float t2 = (((0.5f * xv) * (1.0f - th * th)) * c) * (1.0f + 0.134145f * x2);
    dx[i] = or_bf16_round(gy[i] * (t1 + t2));
  }
}
