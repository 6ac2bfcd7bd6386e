// rt_rowops.cuh — HBM-bound row kernels: per-token int8 quantisation (round-to-nearest and
// Philox stochastic rounding), the ratchet update, pressure leak, unpack, validation, the
// activation dequant of the grad_weight operand and the fused producers of pre-quantised inputs.
//
// Canonical row reduction order (mirrored bit-for-bit by oracle/ratchet_oracle.c):
//   a row of `cols` elements is split into 4-element groups; group g belongs to slot g % 256;
//   each slot sums its elements in increasing index order starting from +0.0f (fp32, RN);
//   slots 32w..32w+31 are combined by an xor butterfly (offsets 16,8,4,2,1);
//   the 8 warp sums w0..w7 are combined as ((w0+w1)+(w2+w3))+((w4+w5)+(w6+w7)).
// Every kernel that needs a row sum (mean square for the ratchet normalisation, RMSNorm) uses one
// 256-thread CTA per row and this order.
#pragma once

#include <cfloat>

#include "rt_common.cuh"

namespace rt {

constexpr int ROW_THREADS = 256;

// -------------------------------------------------------------------------------------------
// Generic element access.
// -------------------------------------------------------------------------------------------
__device__ __forceinline__ float load_elem(const void *p, int dtype, int64_t idx) {
  if (dtype == RT_F32) return __ldg(static_cast<const float *>(p) + idx);
  return bf16_from_bits(__ldg(static_cast<const unsigned short *>(p) + idx));
}
__device__ __forceinline__ void store_elem(void *p, int dtype, int64_t idx, float v) {
  if (dtype == RT_F32)
    static_cast<float *>(p)[idx] = v;
  else
    static_cast<unsigned short *>(p)[idx] = bf16_bits(v);
}

// Fixed-order CTA sum (see header).  `red` is 8 floats of shared memory.
__device__ __forceinline__ float cta_sum_canonical(float partial, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float w = warp_sum_butterfly(partial);
  __syncthreads();  // protect `red` from a previous use
  if (lane == 0) red[warp] = w;
  __syncthreads();
  const float a = __fadd_rn(red[0], red[1]), b = __fadd_rn(red[2], red[3]);
  const float c = __fadd_rn(red[4], red[5]), d = __fadd_rn(red[6], red[7]);
  return __fadd_rn(__fadd_rn(a, b), __fadd_rn(c, d));
}
__device__ __forceinline__ float cta_max(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int i = 1; i < ROW_THREADS / 32; ++i) m = fmaxf(m, red[i]);
  return m;
}

// quantisation of one value given the row scale (int8_matmul.py:139-148).
__device__ __forceinline__ int8_t quant_rn(float v, float scale) {
  float r = rintf(__fdiv_rn(v, scale));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(r));
}
__device__ __forceinline__ int8_t quant_sr(float v, float scale, float u) {
  float r = floorf(__fadd_rn(__fdiv_rn(v, scale), u));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(r));
}
__device__ __forceinline__ float row_scale_of(float amax) {
  return fmaxf(__fdiv_rn(amax, 127.0f), FLT_MIN);
}

// ===========================================================================================
// Row quantisation (int8_matmul.py:106-150).
// ===========================================================================================
struct QuantArgs {
  const void *x;
  int64_t rows, cols, stride_row, stride_col;
  const float *col_scale;
  int stochastic;
  uint64_t seed;
  uint32_t step, layer;
  int8_t *q;
  int64_t ldq;
  float *row_scale;
  unsigned short *xbf16;
  int64_t ld_xbf16;
};

// Vectorised, register-resident variant: RT threads per row, each holding VPT vectors of W
// consecutive elements (16-byte loads).  Rows, columns and outputs are 16-byte aligned.
template <typename T, int RT, int VPT>
__global__ void __launch_bounds__(256) quant_rows_vec_kernel(QuantArgs a) {
  constexpr int W = 16 / sizeof(T);
  constexpr int RPC = 256 / RT;  // rows per CTA
  constexpr int NW = RT / 32;    // warps per row
  __shared__ float red[256 / 32];
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * RPC + sub;
  const bool live = row < a.rows;
  const int64_t nchunk = a.cols / W;
  const T *xr = static_cast<const T *>(a.x) + (live ? row : 0) * a.stride_row;

  float v[VPT][W];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (live && c < nchunk) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(xr + c * W));
      if constexpr (sizeof(T) == 4) {
        v[i][0] = __uint_as_float(raw.x);
        v[i][1] = __uint_as_float(raw.y);
        v[i][2] = __uint_as_float(raw.z);
        v[i][3] = __uint_as_float(raw.w);
      } else {
        const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[i][2 * j] = __uint_as_float(w4[j] << 16);
          v[i][2 * j + 1] = __uint_as_float(w4[j] & 0xFFFF0000u);
        }
      }
      if (a.xbf16 != nullptr) {  // bf16(x), unscaled: the grad_weight GEMM operand
        unsigned short hb[W];
#pragma unroll
        for (int j = 0; j < W; ++j) hb[j] = bf16_bits(v[i][j]);
        unsigned short *dst = a.xbf16 + row * a.ld_xbf16 + c * W;
        if constexpr (W == 8) {
          uint4 o;
          o.x = hb[0] | (uint32_t(hb[1]) << 16);
          o.y = hb[2] | (uint32_t(hb[3]) << 16);
          o.z = hb[4] | (uint32_t(hb[5]) << 16);
          o.w = hb[6] | (uint32_t(hb[7]) << 16);
          *reinterpret_cast<uint4 *>(dst) = o;
        } else {
          uint2 o;
          o.x = hb[0] | (uint32_t(hb[1]) << 16);
          o.y = hb[2] | (uint32_t(hb[3]) << 16);
          *reinterpret_cast<uint2 *>(dst) = o;
        }
      }
      if (a.col_scale != nullptr) {
#pragma unroll
        for (int j = 0; j < W; j += 4) {
          const float4 cs = __ldg(reinterpret_cast<const float4 *>(a.col_scale + c * W + j));
          v[i][j] = __fmul_rn(v[i][j], cs.x);
          v[i][j + 1] = __fmul_rn(v[i][j + 1], cs.y);
          v[i][j + 2] = __fmul_rn(v[i][j + 2], cs.z);
          v[i][j + 3] = __fmul_rn(v[i][j + 3], cs.w);
        }
      }
#pragma unroll
      for (int j = 0; j < W; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j) v[i][j] = 0.0f;
    }
  }
  // row amax across the RT threads of this row
  amax = warp_max(amax);
  if constexpr (NW > 1) {
    __syncthreads();
    if ((t & 31) == 0) red[sub * NW + (t >> 5)] = amax;
    __syncthreads();
    amax = red[sub * NW];
#pragma unroll
    for (int w = 1; w < NW; ++w) amax = fmaxf(amax, red[sub * NW + w]);
  }
  if (!live) return;
  const float scale = row_scale_of(amax);
  if (t == 0) a.row_scale[row] = scale;
  int8_t *qr = a.q + row * a.ldq;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (c >= nchunk) continue;
    int8_t o[W];
    if (a.stochastic) {
      const uint64_t e0 = static_cast<uint64_t>(row) * a.cols + c * W;  // multiple of 4
#pragma unroll
      for (int j = 0; j < W; j += 4) {
        const Philox4 p = sr_block(a.seed, a.step, a.layer, (e0 + j) >> 2);
        o[j] = quant_sr(v[i][j], scale, u24(p.x));
        o[j + 1] = quant_sr(v[i][j + 1], scale, u24(p.y));
        o[j + 2] = quant_sr(v[i][j + 2], scale, u24(p.z));
        o[j + 3] = quant_sr(v[i][j + 3], scale, u24(p.w));
      }
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j) o[j] = quant_rn(v[i][j], scale);
    }
    if constexpr (W == 8) {
      uint2 packed8;
      packed8.x = uint32_t(uint8_t(o[0])) | (uint32_t(uint8_t(o[1])) << 8) |
                  (uint32_t(uint8_t(o[2])) << 16) | (uint32_t(uint8_t(o[3])) << 24);
      packed8.y = uint32_t(uint8_t(o[4])) | (uint32_t(uint8_t(o[5])) << 8) |
                  (uint32_t(uint8_t(o[6])) << 16) | (uint32_t(uint8_t(o[7])) << 24);
      *reinterpret_cast<uint2 *>(qr + c * W) = packed8;
    } else {
      *reinterpret_cast<uint32_t *>(qr + c * W) =
          uint32_t(uint8_t(o[0])) | (uint32_t(uint8_t(o[1])) << 8) |
          (uint32_t(uint8_t(o[2])) << 16) | (uint32_t(uint8_t(o[3])) << 24);
    }
  }
}

// Generic variant: any strides/alignment, one 256-thread CTA per row, two passes (the second
// pass re-reads the row, normally from L2).
template <typename T>
__global__ void __launch_bounds__(256) quant_rows_generic_kernel(QuantArgs a) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const T *xr = static_cast<const T *>(a.x) + row * a.stride_row;
  float amax = 0.0f;
  for (int64_t k = threadIdx.x; k < a.cols; k += 256) {
    float v = load_as_float<T>(xr + k * a.stride_col);
    if (a.xbf16 != nullptr) a.xbf16[row * a.ld_xbf16 + k] = bf16_bits(v);
    if (a.col_scale != nullptr) v = __fmul_rn(v, __ldg(a.col_scale + k));
    amax = fmaxf(amax, fabsf(v));
  }
  amax = cta_max(amax, red);
  const float scale = row_scale_of(amax);
  if (threadIdx.x == 0) a.row_scale[row] = scale;
  for (int64_t k = threadIdx.x; k < a.cols; k += 256) {
    float v = load_as_float<T>(xr + k * a.stride_col);
    if (a.col_scale != nullptr) v = __fmul_rn(v, __ldg(a.col_scale + k));
    int8_t o;
    if (a.stochastic) {
      const uint64_t e = static_cast<uint64_t>(row) * a.cols + k;
      const Philox4 p = sr_block(a.seed, a.step, a.layer, e >> 2);
      o = quant_sr(v, scale, u24(philox_word(p, static_cast<int>(e & 3))));
    } else {
      o = quant_rn(v, scale);
    }
    a.q[row * a.ldq + k] = o;
  }
}

template <typename T, int RT>
static void launch_quant_vec(const QuantArgs &a, int vpt, cudaStream_t s) {
  const int rpc = 256 / RT;
  const dim3 grid(static_cast<unsigned>((a.rows + rpc - 1) / rpc));
  switch (vpt) {
    case 1: quant_rows_vec_kernel<T, RT, 1><<<grid, 256, 0, s>>>(a); break;
    case 2: quant_rows_vec_kernel<T, RT, 2><<<grid, 256, 0, s>>>(a); break;
    case 4: quant_rows_vec_kernel<T, RT, 4><<<grid, 256, 0, s>>>(a); break;
    case 8: quant_rows_vec_kernel<T, RT, 8><<<grid, 256, 0, s>>>(a); break;
    default: quant_rows_vec_kernel<T, RT, 16><<<grid, 256, 0, s>>>(a); break;
  }
}

static inline int pow2_at_least(int64_t v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

template <typename T>
static int quant_rows_dispatch(const QuantArgs &a, cudaStream_t s) {
  constexpr int W = 16 / sizeof(T);
  const bool vec = a.stride_col == 1 && aligned16(a.x) &&
                   (a.stride_row * static_cast<int64_t>(sizeof(T))) % 16 == 0 && a.cols % W == 0 &&
                   (reinterpret_cast<uintptr_t>(a.q) % W) == 0 && a.ldq % W == 0 &&
                   (a.col_scale == nullptr || aligned16(a.col_scale)) &&
                   (a.xbf16 == nullptr ||
                    ((reinterpret_cast<uintptr_t>(a.xbf16) % (2 * W)) == 0 && a.ld_xbf16 % W == 0));
  const int64_t nchunk = a.cols / W;
  if (vec && nchunk <= 32 * 8) {
    launch_quant_vec<T, 32>(a, pow2_at_least((nchunk + 31) / 32), s);
  } else if (vec && nchunk <= 256 * 16) {
    launch_quant_vec<T, 256>(a, pow2_at_least((nchunk + 255) / 256), s);
  } else {
    quant_rows_generic_kernel<T><<<static_cast<unsigned>(a.rows), 256, 0, s>>>(a);
  }
  return check_launch("rt_quantize_rows");
}

// ===========================================================================================
// Ratchet update (ratchet.py:248-301, 487-556, 582-611): one 256-thread CTA per row; the row's
// 4-element groups are held in registers (VPT groups per thread), so HBM sees one read of the
// gradient and of `packed`, one write of `packed` and (optionally) of the int8 code mirror.
// ===========================================================================================
struct UpdateArgs {
  const void *grad;
  int grad_dtype, round_bf16;
  int64_t ldg, rows, cols;
  uint8_t *packed;
  int64_t ldp;
  int8_t *code_out;
  int64_t ldc;
  int normalize;
  float *rms_ema;
  float beta, one_minus_beta;
  int max_code, threshold;
  float low, high, eps;
  unsigned long long *counts;
  float *row_rms, *grad_scale;
};

struct Moves {
  int pos, neg, bpos, bneg;
};

// One weight: returns the new packed byte (ratchet.py:277-294).
__device__ __forceinline__ uint8_t ratchet_one(uint8_t old, float z, const UpdateArgs &a,
                                               Moves &m) {
  const float mag = fabsf(z);
  const int bucket = mag >= a.high ? 2 : (mag >= a.low ? 1 : 0);
  const int sgn = (z > 0.0f) - (z < 0.0f);
  const int inc = -sgn * bucket;
  int code = static_cast<int>(old & 0x0F) - a.max_code;
  int p = static_cast<int>(old >> 4) - 7 + inc;
  const bool pos_req = p >= a.threshold, neg_req = p <= -a.threshold;
  const bool pos_mv = pos_req && code < a.max_code, neg_mv = neg_req && code > -a.max_code;
  code += static_cast<int>(pos_mv) - static_cast<int>(neg_mv);
  p -= static_cast<int>(pos_req) * a.threshold;
  p += static_cast<int>(neg_req) * a.threshold;
  p = min(max(p, -128), 127);
  m.pos += pos_mv;
  m.neg += neg_mv;
  m.bpos += pos_req && !pos_mv;
  m.bneg += neg_req && !neg_mv;
  return static_cast<uint8_t>(((code + a.max_code) & 0x0F) | (((p + 7) & 0x0F) << 4));
}

__device__ __forceinline__ float grad_value(const UpdateArgs &a, int64_t idx) {
  float g = load_elem(a.grad, a.grad_dtype, idx);
  if (a.round_bf16) g = bf16_round(g);
  return g;
}

// VEC: fp32/bf16 gradient rows, `packed` and `code_out` allow 4-element vector access.
template <int VPT, bool VEC>
__global__ void __launch_bounds__(256) ratchet_update_kernel(UpdateArgs a) {
  __shared__ float red[8];
  __shared__ int redi[8][4];
  __shared__ float bcast[2];
  const int t = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int64_t ngroups = (a.cols + 3) / 4;

  float g[VPT][4];
  uint32_t pk[VPT];
  bool bad = false;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t grp = t + static_cast<int64_t>(i) * ROW_THREADS;
    const int64_t c0 = grp * 4;
    pk[i] = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) g[i][j] = 0.0f;
    if (grp >= ngroups) continue;
    if constexpr (VEC) {
      if (a.grad_dtype == RT_F32) {
        const float4 f = __ldg(
            reinterpret_cast<const float4 *>(static_cast<const float *>(a.grad) + row * a.ldg + c0));
        g[i][0] = f.x, g[i][1] = f.y, g[i][2] = f.z, g[i][3] = f.w;
      } else {
        const uint2 h = __ldg(reinterpret_cast<const uint2 *>(
            static_cast<const unsigned short *>(a.grad) + row * a.ldg + c0));
        g[i][0] = __uint_as_float(h.x << 16), g[i][1] = __uint_as_float(h.x & 0xFFFF0000u);
        g[i][2] = __uint_as_float(h.y << 16), g[i][3] = __uint_as_float(h.y & 0xFFFF0000u);
      }
      if (a.round_bf16) {
#pragma unroll
        for (int j = 0; j < 4; ++j) g[i][j] = bf16_round(g[i][j]);
      }
      pk[i] = *reinterpret_cast<const uint32_t *>(a.packed + row * a.ldp + c0);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (c0 + j < a.cols) {
          g[i][j] = grad_value(a, row * a.ldg + c0 + j);
          pk[i] |= static_cast<uint32_t>(a.packed[row * a.ldp + c0 + j]) << (8 * j);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) bad |= !isfinite(g[i][j]);
  }
  bad = __syncthreads_or(bad) != 0;

  // mean square in the canonical order; the trainable-scale gradient uses the same order.
  float ss = 0.0f, gs = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ss = __fadd_rn(ss, __fmul_rn(g[i][j], g[i][j]));
      if (a.grad_scale != nullptr) {
        const int code = static_cast<int>((pk[i] >> (8 * j)) & 0x0Fu) - a.max_code;
        gs = __fadd_rn(gs, __fmul_rn(g[i][j], static_cast<float>(code)));
      }
    }
  }
  const float total = cta_sum_canonical(ss, red);
  float gsum = 0.0f;
  if (a.grad_scale != nullptr) gsum = cta_sum_canonical(gs, red);
  const float ms = __fdiv_rn(total, static_cast<float>(a.cols));

  if (t == 0) {
    float denom_rms = __fsqrt_rn(ms);
    if (a.rms_ema != nullptr && !bad) {
      const float ema_old = a.rms_ema[row];
      const float upd = ema_old == 0.0f
                            ? ms
                            : __fadd_rn(__fmul_rn(a.beta, ema_old), __fmul_rn(a.one_minus_beta, ms));
      const float ema = ms > 0.0f ? upd : ema_old;
      a.rms_ema[row] = ema;
      denom_rms = __fsqrt_rn(ema);
    }
    bcast[0] = __fadd_rn(denom_rms, a.eps);
    if (a.row_rms != nullptr) a.row_rms[row] = __fsqrt_rn(ms);
    if (a.grad_scale != nullptr) a.grad_scale[row] = gsum;
    if (bad) raise_status(RT_STATUS_NONFINITE_GRADIENT);
  }
  __syncthreads();
  const float denom = bcast[0];

  Moves m = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t grp = t + static_cast<int64_t>(i) * ROW_THREADS;
    const int64_t c0 = grp * 4;
    if (grp >= ngroups) continue;
    uint32_t out = pk[i];
    if (!bad) {
      out = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint8_t old = static_cast<uint8_t>(pk[i] >> (8 * j));
        if (c0 + j < a.cols) {
          const float z = a.normalize ? __fdiv_rn(g[i][j], denom) : g[i][j];
          out |= static_cast<uint32_t>(ratchet_one(old, z, a, m)) << (8 * j);
        }
      }
    }
    uint32_t codes = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      codes |= static_cast<uint32_t>(static_cast<uint8_t>(
                   static_cast<int8_t>(static_cast<int>((out >> (8 * j)) & 0x0Fu) - a.max_code)))
               << (8 * j);
    if constexpr (VEC) {
      if (!bad) *reinterpret_cast<uint32_t *>(a.packed + row * a.ldp + c0) = out;
      if (a.code_out != nullptr)
        *reinterpret_cast<uint32_t *>(a.code_out + row * a.ldc + c0) = codes;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (c0 + j >= a.cols) break;
        if (!bad) a.packed[row * a.ldp + c0 + j] = static_cast<uint8_t>(out >> (8 * j));
        if (a.code_out != nullptr)
          a.code_out[row * a.ldc + c0 + j] = static_cast<int8_t>(codes >> (8 * j));
      }
    }
  }
  // move counters: warp sums, then one atomic per counter per CTA
  const int lane = t & 31, warp = t >> 5;
  m.pos = warp_isum(m.pos), m.neg = warp_isum(m.neg);
  m.bpos = warp_isum(m.bpos), m.bneg = warp_isum(m.bneg);
  if (lane == 0) {
    redi[warp][0] = m.pos, redi[warp][1] = m.neg, redi[warp][2] = m.bpos, redi[warp][3] = m.bneg;
  }
  __syncthreads();
  if (t < 4 && a.counts != nullptr) {
    int s = 0;
    for (int w = 0; w < 8; ++w) s += redi[w][t];
    if (s != 0) atomicAdd(a.counts + t, static_cast<unsigned long long>(s));
  }
}

// Rows longer than 8192: same arithmetic and reduction order, gradient re-read per pass.
__global__ void __launch_bounds__(256) ratchet_update_long_kernel(UpdateArgs a) {
  __shared__ float red[8];
  __shared__ int redi[8][4];
  __shared__ float bcast[1];
  const int t = threadIdx.x;
  const int64_t row = blockIdx.x;
  const int64_t ngroups = (a.cols + 3) / 4;
  float ss = 0.0f, gs = 0.0f;
  bool bad = false;
  for (int64_t grp = t; grp < ngroups; grp += ROW_THREADS) {
    for (int j = 0; j < 4; ++j) {
      const int64_t c = grp * 4 + j;
      if (c >= a.cols) break;
      const float g = grad_value(a, row * a.ldg + c);
      bad |= !isfinite(g);
      ss = __fadd_rn(ss, __fmul_rn(g, g));
      if (a.grad_scale != nullptr) {
        const int code = static_cast<int>(a.packed[row * a.ldp + c] & 0x0F) - a.max_code;
        gs = __fadd_rn(gs, __fmul_rn(g, static_cast<float>(code)));
      }
    }
  }
  bad = __syncthreads_or(bad) != 0;
  const float total = cta_sum_canonical(ss, red);
  float gsum = 0.0f;
  if (a.grad_scale != nullptr) gsum = cta_sum_canonical(gs, red);
  const float ms = __fdiv_rn(total, static_cast<float>(a.cols));
  if (t == 0) {
    float denom_rms = __fsqrt_rn(ms);
    if (a.rms_ema != nullptr && !bad) {
      const float ema_old = a.rms_ema[row];
      const float upd = ema_old == 0.0f
                            ? ms
                            : __fadd_rn(__fmul_rn(a.beta, ema_old), __fmul_rn(a.one_minus_beta, ms));
      const float ema = ms > 0.0f ? upd : ema_old;
      a.rms_ema[row] = ema;
      denom_rms = __fsqrt_rn(ema);
    }
    bcast[0] = __fadd_rn(denom_rms, a.eps);
    if (a.row_rms != nullptr) a.row_rms[row] = __fsqrt_rn(ms);
    if (a.grad_scale != nullptr) a.grad_scale[row] = gsum;
    if (bad) raise_status(RT_STATUS_NONFINITE_GRADIENT);
  }
  __syncthreads();
  const float denom = bcast[0];
  Moves m = {0, 0, 0, 0};
  for (int64_t c = t; c < a.cols; c += ROW_THREADS) {
    uint8_t v = a.packed[row * a.ldp + c];
    if (!bad) {
      const float g = grad_value(a, row * a.ldg + c);
      const float z = a.normalize ? __fdiv_rn(g, denom) : g;
      v = ratchet_one(v, z, a, m);
      a.packed[row * a.ldp + c] = v;
    }
    if (a.code_out != nullptr)
      a.code_out[row * a.ldc + c] = static_cast<int8_t>(static_cast<int>(v & 0x0F) - a.max_code);
  }
  const int lane = t & 31, warp = t >> 5;
  m.pos = warp_isum(m.pos), m.neg = warp_isum(m.neg);
  m.bpos = warp_isum(m.bpos), m.bneg = warp_isum(m.bneg);
  if (lane == 0) {
    redi[warp][0] = m.pos, redi[warp][1] = m.neg, redi[warp][2] = m.bpos, redi[warp][3] = m.bneg;
  }
  __syncthreads();
  if (t < 4 && a.counts != nullptr) {
    int s = 0;
    for (int w = 0; w < 8; ++w) s += redi[w][t];
    if (s != 0) atomicAdd(a.counts + t, static_cast<unsigned long long>(s));
  }
}

// ===========================================================================================
// Small elementwise state kernels.
// ===========================================================================================
__global__ void leak_kernel(uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const uint8_t v = packed[r * ldp + c];
    int p = static_cast<int>(v >> 4) - 7;
    p -= (p > 0) - (p < 0);
    packed[r * ldp + c] = static_cast<uint8_t>((v & 0x0F) | (((p + 7) & 0x0F) << 4));
  }
}

__global__ void unpack_kernel(const uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols,
                              int max_code, int8_t *code, int64_t ldc, int8_t *pressure,
                              int64_t ldpr) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const uint8_t v = __ldg(packed + r * ldp + c);
    if (code) code[r * ldc + c] = static_cast<int8_t>(static_cast<int>(v & 0x0F) - max_code);
    if (pressure) pressure[r * ldpr + c] = static_cast<int8_t>(static_cast<int>(v >> 4) - 7);
  }
}

// Contiguous fast path of the unpack used to refresh the int8 code mirror (16 weights / thread).
__global__ void unpack_codes_vec_kernel(const uint4 *packed, int64_t n16, int max_code,
                                        uint4 *code) {
  const uint32_t bias = 0x01010101u * static_cast<uint32_t>(max_code);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint4 v = __ldg(packed + i);
    // per byte: (v & 0x0F) - max_code; the low nibble is >= 0, so a bytewise subtraction with a
    // borrow-free formulation is done via __vsub4.
    v.x = __vsub4(v.x & 0x0F0F0F0Fu, bias);
    v.y = __vsub4(v.y & 0x0F0F0F0Fu, bias);
    v.z = __vsub4(v.z & 0x0F0F0F0Fu, bias);
    v.w = __vsub4(v.w & 0x0F0F0F0Fu, bias);
    code[i] = v;
  }
}

__global__ void validate_kernel(const uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols,
                                int max_code, const float *scale) {
  uint32_t bits = 0;
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const uint8_t v = __ldg(packed + r * ldp + c);
    const int code = static_cast<int>(v & 0x0F) - max_code;
    const int p = static_cast<int>(v >> 4) - 7;
    if (code < -max_code || code > max_code) bits |= RT_STATUS_CODE_RANGE;
    if (p > 7 || p < -7) bits |= RT_STATUS_PRESSURE_RANGE;
  }
  if (scale != nullptr) {
    for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < rows;
         r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const float s = scale[r];
      if (!(s > 0.0f) || !isfinite(s)) bits |= RT_STATUS_SCALE_INVALID;
    }
  }
  bits = __reduce_or_sync(0xffffffffu, bits);
  if ((threadIdx.x & 31) == 0 && bits) raise_status(bits);
}

// out[m,k] = bf16(bf16(q) * bf16(s[m])) (ratchet.py:73-76); 8 elements per thread when aligned.
__global__ void dequant_vec_kernel(const int8_t *q, int64_t ldq, const float *s, uint16_t *out,
                                   int64_t ldo, int64_t rows, int64_t cols8) {
  const int64_t n = rows * cols8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols8, c = (i % cols8) * 8;
    const float sb = bf16_round(__ldg(s + r));
    const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(q + r * ldq + c));
    const uint32_t w[2] = {raw.x, raw.y};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int8_t lo = static_cast<int8_t>((w[j >> 1] >> (16 * (j & 1))) & 0xFF);
      const int8_t hi = static_cast<int8_t>((w[j >> 1] >> (16 * (j & 1) + 8)) & 0xFF);
      o[j] = bf16_bits(__fmul_rn(static_cast<float>(lo), sb)) |
             (static_cast<uint32_t>(bf16_bits(__fmul_rn(static_cast<float>(hi), sb))) << 16);
    }
    *reinterpret_cast<uint4 *>(out + r * ldo + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}
__global__ void dequant_kernel(const int8_t *q, int64_t ldq, const float *s, uint16_t *out,
                               int64_t ldo, int64_t rows, int64_t cols) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const float sb = bf16_round(__ldg(s + r));
    out[r * ldo + c] = bf16_bits(__fmul_rn(static_cast<float>(q[r * ldq + c]), sb));
  }
}

// ===========================================================================================
// Fused producers (int8_fused.py, int8_backward.py).  One 256-thread CTA per row, row values
// re-read from L2 for the second pass.
// ===========================================================================================
// rmsnorm: y = (x * r) * w with r = 1 / sqrt(mean(x^2) + eps) (IEEE sqrt and division).
__global__ void __launch_bounds__(256)
    rmsnorm_quant_kernel(const void *x, int dtype, int64_t ldx, const float *w, float eps,
                         int64_t cols, int8_t *q, int64_t ldq, float *row_scale) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const int64_t ngroups = (cols + 3) / 4;
  float ss = 0.0f;
  for (int64_t grp = threadIdx.x; grp < ngroups; grp += 256)
    for (int j = 0; j < 4; ++j) {
      const int64_t c = grp * 4 + j;
      if (c >= cols) break;
      const float v = load_elem(x, dtype, row * ldx + c);
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
  const float total = cta_sum_canonical(ss, red);
  const float var = __fdiv_rn(total, static_cast<float>(cols));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  float amax = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += 256) {
    const float y = __fmul_rn(__fmul_rn(load_elem(x, dtype, row * ldx + c), r), __ldg(w + c));
    amax = fmaxf(amax, fabsf(y));
  }
  amax = cta_max(amax, red);
  const float scale = row_scale_of(amax);
  if (threadIdx.x == 0) row_scale[row] = scale;
  for (int64_t c = threadIdx.x; c < cols; c += 256) {
    const float y = __fmul_rn(__fmul_rn(load_elem(x, dtype, row * ldx + c), r), __ldg(w + c));
    q[row * ldq + c] = quant_rn(y, scale);
  }
}

// tanh-approximate GELU with the reference's operation order (int8_fused.py:70-75).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float c = 0.7978845608028654f;
  const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  const float inner = __fmul_rn(c, __fadd_rn(x, cube));
  const float th = tanhf(inner);
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, th));
}

__global__ void __launch_bounds__(256)
    gelu_quant_kernel(const void *x, int dtype, int64_t ldx, int64_t cols, int8_t *q, int64_t ldq,
                      float *row_scale) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  float amax = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += 256)
    amax = fmaxf(amax, fabsf(gelu_tanh(load_elem(x, dtype, row * ldx + c))));
  amax = cta_max(amax, red);
  const float scale = row_scale_of(amax);
  if (threadIdx.x == 0) row_scale[row] = scale;
  for (int64_t c = threadIdx.x; c < cols; c += 256)
    q[row * ldq + c] = quant_rn(gelu_tanh(load_elem(x, dtype, row * ldx + c)), scale);
}

__global__ void __launch_bounds__(256)
    transpose_quant_kernel(const void *x, int dtype, int64_t heads, int64_t seq, int64_t head_dim,
                           int64_t sb, int64_t sh, int64_t ss, int64_t sd, int8_t *q, int64_t ldq,
                           float *row_scale) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;  // row = b * seq + s
  const int64_t b = row / seq, s = row % seq;
  const int64_t channels = heads * head_dim;
  float amax = 0.0f;
  for (int64_t c = threadIdx.x; c < channels; c += 256) {
    const int64_t h = c / head_dim, d = c % head_dim;
    amax = fmaxf(amax, fabsf(load_elem(x, dtype, b * sb + h * sh + s * ss + d * sd)));
  }
  amax = cta_max(amax, red);
  const float scale = row_scale_of(amax);
  if (threadIdx.x == 0) row_scale[row] = scale;
  for (int64_t c = threadIdx.x; c < channels; c += 256) {
    const int64_t h = c / head_dim, d = c % head_dim;
    q[row * ldq + c] = quant_rn(load_elem(x, dtype, b * sb + h * sh + s * ss + d * sd), scale);
  }
}

// RMSNorm backward dx (int8_backward.py:7-27), stored through bf16 as the reference does.
__global__ void __launch_bounds__(256)
    rmsnorm_bwd_kernel(const void *gy, int gdt, const void *x, int xdt, const float *w, float eps,
                       int64_t cols, void *dx, int dxdt) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const int64_t ngroups = (cols + 3) / 4;
  float ss = 0.0f, dot = 0.0f;
  for (int64_t grp = threadIdx.x; grp < ngroups; grp += 256)
    for (int j = 0; j < 4; ++j) {
      const int64_t c = grp * 4 + j;
      if (c >= cols) break;
      const float xv = load_elem(x, xdt, row * cols + c);
      const float dh = __fmul_rn(load_elem(gy, gdt, row * cols + c), __ldg(w + c));
      ss = __fadd_rn(ss, __fmul_rn(xv, xv));
      dot = __fadd_rn(dot, __fmul_rn(dh, xv));
    }
  const float total = cta_sum_canonical(ss, red);
  const float dsum = cta_sum_canonical(dot, red);
  const float var = __fdiv_rn(total, static_cast<float>(cols));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  const float dvar = __fmul_rn(__fmul_rn(dsum, -0.5f), __fmul_rn(__fmul_rn(r, r), r));
  for (int64_t c = threadIdx.x; c < cols; c += 256) {
    const float xv = load_elem(x, xdt, row * cols + c);
    const float dh = __fmul_rn(load_elem(gy, gdt, row * cols + c), __ldg(w + c));
    const float v = __fadd_rn(__fmul_rn(dh, r),
                              __fdiv_rn(__fmul_rn(__fmul_rn(dvar, 2.0f), xv), static_cast<float>(cols)));
    store_elem(dx, dxdt, row * cols + c, bf16_round(v));
  }
}

// tanh-GELU backward (int8_backward.py:53-74), stored through bf16 as the reference does.
__global__ void gelu_bwd_kernel(const void *gy, int gdt, const void *x, int xdt, int64_t n,
                                void *dx, int dxdt) {
  const float c = 0.7978845608028654f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float xv = load_elem(x, xdt, i);
    const float g = load_elem(gy, gdt, i);
    const float x2 = __fmul_rn(xv, xv);
    const float inner = __fmul_rn(c, __fadd_rn(xv, __fmul_rn(__fmul_rn(0.044715f, xv), x2)));
    const float th = tanhf(inner);
    const float t1 = __fmul_rn(0.5f, __fadd_rn(1.0f, th));
    const float t2 = __fmul_rn(
        __fmul_rn(__fmul_rn(__fmul_rn(0.5f, xv), __fsub_rn(1.0f, __fmul_rn(th, th))), c),
        __fadd_rn(1.0f, __fmul_rn(0.134145f, x2)));
    store_elem(dx, dxdt, i, bf16_round(__fmul_rn(g, __fadd_rn(t1, t2))));
  }
}

static inline unsigned grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 32) b = 148 * 32;
  if (b < 1) b = 1;
  return static_cast<unsigned>(b);
}

}  // namespace rt

// ===========================================================================================
// C ABI
// ===========================================================================================
using namespace rt;

extern "C" int rt_quantize_rows(const void *x, int x_dtype, int64_t rows, int64_t cols,
                                int64_t stride_row, int64_t stride_col, const float *col_scale,
                                int stochastic, uint64_t seed, uint32_t step, uint32_t layer,
                                int8_t *q, int64_t ldq, float *row_scale, void *x_bf16_out,
                                int64_t ld_xbf16, void *stream) {
  if (rows < 0 || cols < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_quantize_rows: negative shape");
  if (rows == 0) return RT_OK;
  if (x == nullptr || q == nullptr || row_scale == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_quantize_rows: null pointer");
  if (x_dtype != RT_F32 && x_dtype != RT_BF16)
    return fail(RT_ERR_DTYPE, "rt_quantize_rows: input must be float32 or bfloat16");
  if (cols == 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_quantize_rows: zero columns");
  QuantArgs a{x,   rows,      cols,      stride_row, stride_col, col_scale,
              stochastic, seed, step, layer, q, ldq, row_scale,
              static_cast<unsigned short *>(x_bf16_out), ld_xbf16};
  cudaStream_t s = as_stream(stream);
  return x_dtype == RT_F32 ? quant_rows_dispatch<float>(a, s)
                           : quant_rows_dispatch<__nv_bfloat16>(a, s);
}

extern "C" int rt_dequant_rows_bf16(const int8_t *q, int64_t ldq, const float *row_scale,
                                    void *out, int64_t ldo, int64_t rows, int64_t cols,
                                    void *stream) {
  if (rows < 0 || cols < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_dequant_rows_bf16: shape");
  if (rows == 0 || cols == 0) return RT_OK;
  cudaStream_t s = as_stream(stream);
  uint16_t *o = static_cast<uint16_t *>(out);
  if (cols % 8 == 0 && ldq % 8 == 0 && ldo % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(q) & 7) == 0 && aligned16(out)) {
    dequant_vec_kernel<<<grid_for(rows * (cols / 8), 256), 256, 0, s>>>(q, ldq, row_scale, o, ldo,
                                                                         rows, cols / 8);
  } else {
    dequant_kernel<<<grid_for(rows * cols, 256), 256, 0, s>>>(q, ldq, row_scale, o, ldo, rows,
                                                              cols);
  }
  return check_launch("rt_dequant_rows_bf16");
}

extern "C" int rt_ratchet_update(const void *grad, int grad_dtype, int round_bf16, int64_t ldg,
                                 int64_t rows, int64_t cols, uint8_t *packed, int64_t ldp,
                                 int8_t *code_out, int64_t ldc, int normalize, float *rms_ema,
                                 double ema_beta, int max_code, int threshold, double bucket_low,
                                 double bucket_high, double eps, int64_t *counts, float *row_rms,
                                 float *grad_scale, void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_update: shape");
  if (rows == 0) return RT_OK;
  if (grad == nullptr || packed == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_update: null pointer");
  if (grad_dtype != RT_F32 && grad_dtype != RT_BF16)
    return fail(RT_ERR_DTYPE, "rt_ratchet_update: gradient must be float32 or bfloat16");
  if (max_code < 1 || max_code > 7)
    return fail(RT_ERR_INVALID_ARGUMENT, "max_code must be in 1..7 (3..15 states)");
  if (threshold <= 0 || threshold > 127)
    return fail(RT_ERR_INVALID_ARGUMENT, "pressure_threshold must be in [1, 127]");
  if (!(0.0 <= bucket_low && bucket_low < bucket_high))
    return fail(RT_ERR_INVALID_ARGUMENT, "bucket thresholds must satisfy 0 <= low < high");
  UpdateArgs a;
  a.grad = grad, a.grad_dtype = grad_dtype, a.round_bf16 = round_bf16, a.ldg = ldg;
  a.rows = rows, a.cols = cols, a.packed = packed, a.ldp = ldp, a.code_out = code_out;
  a.ldc = ldc, a.normalize = normalize, a.rms_ema = (ema_beta > 0.0) ? rms_ema : nullptr;
  a.beta = static_cast<float>(ema_beta);
  a.one_minus_beta = static_cast<float>(1.0 - ema_beta);
  a.max_code = max_code, a.threshold = threshold;
  a.low = static_cast<float>(bucket_low), a.high = static_cast<float>(bucket_high);
  a.eps = static_cast<float>(eps);
  a.counts = reinterpret_cast<unsigned long long *>(counts);
  a.row_rms = row_rms, a.grad_scale = grad_scale;
  cudaStream_t s = as_stream(stream);
  const size_t esz = grad_dtype == RT_F32 ? 4 : 2;
  const bool vec = cols % 4 == 0 && ldg % 4 == 0 && ldp % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(grad) % (4 * esz)) == 0 &&
                   (reinterpret_cast<uintptr_t>(packed) & 3) == 0 &&
                   (code_out == nullptr || ((reinterpret_cast<uintptr_t>(code_out) & 3) == 0 &&
                                            ldc % 4 == 0));
  const int64_t per_thread = (cols + 4 * ROW_THREADS - 1) / (4 * ROW_THREADS);
  const dim3 grid(static_cast<unsigned>(rows));
#define RT_UPD(VPT)                                                      \
  (vec ? (ratchet_update_kernel<VPT, true><<<grid, ROW_THREADS, 0, s>>>(a)) \
       : (ratchet_update_kernel<VPT, false><<<grid, ROW_THREADS, 0, s>>>(a)))
  if (per_thread <= 1)
    RT_UPD(1);
  else if (per_thread <= 2)
    RT_UPD(2);
  else if (per_thread <= 4)
    RT_UPD(4);
  else if (per_thread <= 8)
    RT_UPD(8);
  else
    ratchet_update_long_kernel<<<grid, ROW_THREADS, 0, s>>>(a);
#undef RT_UPD
  return check_launch("rt_ratchet_update");
}

extern "C" int rt_ratchet_leak(uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols,
                               int max_code, void *stream) {
  (void)max_code;
  if (rows < 0 || cols < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_leak: shape");
  if (rows * cols == 0) return RT_OK;
  leak_kernel<<<grid_for(rows * cols, 256), 256, 0, as_stream(stream)>>>(packed, ldp, rows, cols);
  return check_launch("rt_ratchet_leak");
}

extern "C" int rt_unpack_code_pressure(const uint8_t *packed, int64_t ldp, int64_t rows,
                                       int64_t cols, int max_code, int8_t *code, int64_t ldc,
                                       int8_t *pressure, int64_t ldpr, void *stream) {
  if (rows < 0 || cols < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_unpack_code_pressure: shape");
  if (rows * cols == 0) return RT_OK;
  cudaStream_t s = as_stream(stream);
  const int64_t n = rows * cols;
  if (pressure == nullptr && code != nullptr && ldp == cols && ldc == cols && n % 16 == 0 &&
      aligned16(packed) && aligned16(code)) {
    unpack_codes_vec_kernel<<<grid_for(n / 16, 256), 256, 0, s>>>(
        reinterpret_cast<const uint4 *>(packed), n / 16, max_code, reinterpret_cast<uint4 *>(code));
  } else {
    unpack_kernel<<<grid_for(n, 256), 256, 0, s>>>(packed, ldp, rows, cols, max_code, code, ldc,
                                                   pressure, ldpr);
  }
  return check_launch("rt_unpack_code_pressure");
}

extern "C" int rt_ratchet_validate(const uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols,
                                   int max_code, const float *scale, void *stream) {
  if (rows < 0 || cols < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_validate: shape");
  if (rows * cols == 0) return RT_OK;
  validate_kernel<<<grid_for(rows * cols, 256), 256, 0, as_stream(stream)>>>(packed, ldp, rows,
                                                                             cols, max_code, scale);
  return check_launch("rt_ratchet_validate");
}

extern "C" int rt_rmsnorm_quantize(const void *x, int x_dtype, int64_t ldx, const float *weight,
                                   double eps, int64_t rows, int64_t cols, int8_t *q, int64_t ldq,
                                   float *row_scale, void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_rmsnorm_quantize: shape");
  if (x_dtype != RT_F32 && x_dtype != RT_BF16) return fail(RT_ERR_DTYPE, "rt_rmsnorm_quantize: dtype");
  if (rows == 0) return RT_OK;
  rmsnorm_quant_kernel<<<static_cast<unsigned>(rows), 256, 0, as_stream(stream)>>>(
      x, x_dtype, ldx, weight, static_cast<float>(eps), cols, q, ldq, row_scale);
  return check_launch("rt_rmsnorm_quantize");
}

extern "C" int rt_gelu_quantize(const void *x, int x_dtype, int64_t ldx, int64_t rows,
                                int64_t cols, int8_t *q, int64_t ldq, float *row_scale,
                                void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_gelu_quantize: shape");
  if (x_dtype != RT_F32 && x_dtype != RT_BF16) return fail(RT_ERR_DTYPE, "rt_gelu_quantize: dtype");
  if (rows == 0) return RT_OK;
  gelu_quant_kernel<<<static_cast<unsigned>(rows), 256, 0, as_stream(stream)>>>(x, x_dtype, ldx,
                                                                                cols, q, ldq,
                                                                                row_scale);
  return check_launch("rt_gelu_quantize");
}

extern "C" int rt_transpose_quantize(const void *x, int x_dtype, int64_t batch, int64_t heads,
                                     int64_t seq, int64_t head_dim, int64_t stride_b,
                                     int64_t stride_h, int64_t stride_s, int64_t stride_d,
                                     int8_t *q, int64_t ldq, float *row_scale, void *stream) {
  if (batch < 0 || heads <= 0 || seq < 0 || head_dim <= 0)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_transpose_quantize: shape");
  if (x_dtype != RT_F32 && x_dtype != RT_BF16)
    return fail(RT_ERR_DTYPE, "rt_transpose_quantize: dtype");
  if (batch * seq == 0) return RT_OK;
  transpose_quant_kernel<<<static_cast<unsigned>(batch * seq), 256, 0, as_stream(stream)>>>(
      x, x_dtype, heads, seq, head_dim, stride_b, stride_h, stride_s, stride_d, q, ldq, row_scale);
  return check_launch("rt_transpose_quantize");
}

extern "C" int rt_rmsnorm_backward(const void *grad_y, int gy_dtype, const void *x, int x_dtype,
                                   const float *weight, double eps, int64_t rows, int64_t cols,
                                   void *dx, int dx_dtype, void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_rmsnorm_backward: shape");
  if (rows == 0) return RT_OK;
  rmsnorm_bwd_kernel<<<static_cast<unsigned>(rows), 256, 0, as_stream(stream)>>>(
      grad_y, gy_dtype, x, x_dtype, weight, static_cast<float>(eps), cols, dx, dx_dtype);
  return check_launch("rt_rmsnorm_backward");
}

extern "C" int rt_gelu_backward(const void *grad_y, int gy_dtype, const void *x, int x_dtype,
                                int64_t rows, int64_t cols, void *dx, int dx_dtype, void *stream) {
  if (rows < 0 || cols < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_gelu_backward: shape");
  if (rows * cols == 0) return RT_OK;
  gelu_bwd_kernel<<<grid_for(rows * cols, 256), 256, 0, as_stream(stream)>>>(
      grad_y, gy_dtype, x, x_dtype, rows * cols, dx, dx_dtype);
  return check_launch("rt_gelu_backward");
}
