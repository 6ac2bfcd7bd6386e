// rt_loss.cuh — token cross-entropy over the lm_head logits (model.py:244-249 calls
// F.cross_entropy(logits, targets) with mean reduction and ignore_index -100).
//
// Forward, one CTA per row: row max, logsum = log(sum exp(x - max)), loss_row = logsum - (x_t - max)
// (the log_softmax form log p = (x - max) - logsum, torch's LogSoftMax epilogue order).
// Backward, one CTA per row, writes the bf16 gradient the lm_head GEMMs consume directly:
//   g_j = RN(exp(log p_j) · w) - [j == t] · w   with w = grad_loss / count,
// the value torch's nll + log_softmax backward produce in fp32, then rounded to bf16 as the
// reference does before its grad GEMMs.  Rows whose target is ignore_index get zero loss and
// gradient.  An optional fp32 gradient arriving for the logits themselves is added before the
// rounding.
#pragma once

#include "rt_common.cuh"

namespace rt {

constexpr int CE_THREADS = 256;
constexpr int CE_VEC = 8;  // float4 chunks per thread held in registers (rows up to 8192 floats)

__device__ __forceinline__ float ce_block_max(float v, float *sm) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sm[w] = v;
  __syncthreads();
  float m = sm[0];
#pragma unroll
  for (int i = 1; i < CE_THREADS / 32; ++i) m = fmaxf(m, sm[i]);
  return m;
}
// fixed-order sum: each warp's butterfly, then the eight warp sums in warp order
__device__ __forceinline__ float ce_block_sum(float v, float *sm) {
  v = warp_sum_butterfly(v);
  const int w = threadIdx.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sm[w] = v;
  __syncthreads();
  float s = sm[0];
#pragma unroll
  for (int i = 1; i < CE_THREADS / 32; ++i) s = __fadd_rn(s, sm[i]);
  return s;
}

template <typename T>
__device__ __forceinline__ float ce_load(const T *p) {
  if constexpr (sizeof(T) == 4)
    return *p;
  else
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(p));
}

struct CeArgs {
  const void *logits;
  int64_t ld, rows, cols;
  const int64_t *targets;
  int64_t ignore_index;
  float *row_max, *row_logsum, *row_loss;
  const float *grad_loss, *count;  // backward: device scalars
  const float *extra;              // backward: optional fp32 gradient of the logits
  int64_t ld_extra;
  uint16_t *out;  // backward: bf16 gradient
  int64_t ldo;
};

// Four logits as floats: an fp32 float4, or four bf16 widened (exact).
__device__ __forceinline__ float4 ce_load4(const float *x, int c) {
  return __ldcs(reinterpret_cast<const float4 *>(x) + c);
}
__device__ __forceinline__ float4 ce_load4(const uint16_t *x, int c) {
  const uint2 u = __ldcs(reinterpret_cast<const uint2 *>(x) + c);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
}

// Register-resident rows: cols % 4 == 0, cols <= CE_THREADS·4·CE_VEC, rows aligned to 4 logits
// (16 bytes fp32, 8 bytes bf16).  Each thread takes the same groups of four in either dtype, so
// bf16 logits give the bits that fp32 logits of the same values give.
template <typename T>
__global__ void __launch_bounds__(CE_THREADS) ce_fwd_vec_kernel(CeArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sm[CE_THREADS / 32];
  const int64_t row = blockIdx.x;
  const T *x = static_cast<const T *>(a.logits) + row * a.ld;
  const int nq = static_cast<int>(a.cols / 4);
  float4 v[CE_VEC];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < CE_VEC; ++i) {
    const int c = threadIdx.x + i * CE_THREADS;
    if (c < nq) {
      v[i] = ce_load4(x, c);
      m = fmaxf(m, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
    }
  }
  m = ce_block_max(m, sm);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < CE_VEC; ++i) {
    const int c = threadIdx.x + i * CE_THREADS;
    if (c < nq) {
      s = __fadd_rn(s, expf(__fsub_rn(v[i].x, m)));
      s = __fadd_rn(s, expf(__fsub_rn(v[i].y, m)));
      s = __fadd_rn(s, expf(__fsub_rn(v[i].z, m)));
      s = __fadd_rn(s, expf(__fsub_rn(v[i].w, m)));
    }
  }
  s = ce_block_sum(s, sm);
  if (threadIdx.x == 0) {
    const float logsum = logf(s);
    const int64_t t = a.targets[row];
    a.row_max[row] = m;
    a.row_logsum[row] = logsum;
    float loss = 0.0f;
    if (t != a.ignore_index) {
      if (t < 0 || t >= a.cols) {
        raise_status(RT_STATUS_CODE_RANGE);
      } else {
        loss = -__fsub_rn(__fsub_rn(ce_load(x + t), m), logsum);
      }
    }
    a.row_loss[row] = loss;
  }
}

// Any layout: two passes over the row in global memory.
template <typename T>
__global__ void __launch_bounds__(CE_THREADS) ce_fwd_generic_kernel(CeArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sm[CE_THREADS / 32];
  const int64_t row = blockIdx.x;
  const T *x = static_cast<const T *>(a.logits) + row * a.ld;
  float m = -INFINITY;
  for (int64_t j = threadIdx.x; j < a.cols; j += CE_THREADS) m = fmaxf(m, ce_load(x + j));
  m = ce_block_max(m, sm);
  float s = 0.0f;
  for (int64_t j = threadIdx.x; j < a.cols; j += CE_THREADS)
    s = __fadd_rn(s, expf(__fsub_rn(ce_load(x + j), m)));
  s = ce_block_sum(s, sm);
  if (threadIdx.x == 0) {
    const float logsum = logf(s);
    const int64_t t = a.targets[row];
    a.row_max[row] = m;
    a.row_logsum[row] = logsum;
    float loss = 0.0f;
    if (t != a.ignore_index) {
      if (t < 0 || t >= a.cols) {
        raise_status(RT_STATUS_CODE_RANGE);
      } else {
        loss = -__fsub_rn(__fsub_rn(ce_load(x + t), m), logsum);
      }
    }
    a.row_loss[row] = loss;
  }
}

__device__ __forceinline__ float ce_grad(float xv, float m, float logsum, float w, bool is_target) {
  const float p = expf(__fsub_rn(__fsub_rn(xv, m), logsum));
  const float g = __fmul_rn(p, w);
  return is_target ? __fsub_rn(g, w) : g;
}

template <typename T>
__global__ void __launch_bounds__(CE_THREADS) ce_bwd_kernel(CeArgs a) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const T *x = static_cast<const T *>(a.logits) + row * a.ld;
  uint16_t *o = a.out + row * a.ldo;
  const float *e = a.extra != nullptr ? a.extra + row * a.ld_extra : nullptr;
  const int64_t t = a.targets[row];
  const bool ignored = t == a.ignore_index || t < 0 || t >= a.cols;
  const float w = __fdiv_rn(__ldg(a.grad_loss), __ldg(a.count));
  const float m = a.row_max[row], logsum = a.row_logsum[row];
  const auto a16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = a.cols % 8 == 0 && (a.ld % 8) == 0 && (a.ldo % 8) == 0 && a16(x) && a16(o) &&
                   (e == nullptr || ((a.ld_extra % 4) == 0 && a16(e)));
  if (vec) {
    for (int64_t c = threadIdx.x; c < a.cols / 8; c += CE_THREADS) {
      float xs[8];
      if constexpr (sizeof(T) == 4) {
        const float4 v0 = __ldcs(reinterpret_cast<const float4 *>(x) + 2 * c);
        const float4 v1 = __ldcs(reinterpret_cast<const float4 *>(x) + 2 * c + 1);
        xs[0] = v0.x, xs[1] = v0.y, xs[2] = v0.z, xs[3] = v0.w;
        xs[4] = v1.x, xs[5] = v1.y, xs[6] = v1.z, xs[7] = v1.w;
      } else {
        const uint4 u = __ldcs(reinterpret_cast<const uint4 *>(x) + c);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          xs[2 * j] = __uint_as_float(w[j] << 16);
          xs[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
        }
      }
      float g[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t col = 8 * c + j;
        g[j] = ignored ? 0.0f : ce_grad(xs[j], m, logsum, w, col == t);
      }
      if (e != nullptr) {
        const float4 e0 = reinterpret_cast<const float4 *>(e)[2 * c];
        const float4 e1 = reinterpret_cast<const float4 *>(e)[2 * c + 1];
        const float es[8] = {e0.x, e0.y, e0.z, e0.w, e1.x, e1.y, e1.z, e1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = __fadd_rn(g[j], es[j]);
      }
      uint4 u;
      u.x = pack_bf16x2(g[0], g[1]);
      u.y = pack_bf16x2(g[2], g[3]);
      u.z = pack_bf16x2(g[4], g[5]);
      u.w = pack_bf16x2(g[6], g[7]);
      reinterpret_cast<uint4 *>(o)[c] = u;
    }
  } else {
    for (int64_t j = threadIdx.x; j < a.cols; j += CE_THREADS) {
      float g = ignored ? 0.0f : ce_grad(ce_load(x + j), m, logsum, w, j == t);
      if (e != nullptr) g = __fadd_rn(g, e[j]);
      o[j] = bf16_bits(g);
    }
  }
}

}  // namespace rt

using namespace rt;

extern "C" int rt_cross_entropy_fwd(const void *logits, int dtype, int64_t ld, int64_t rows,
                                    int64_t cols, const int64_t *targets, int64_t ignore_index,
                                    float *row_max, float *row_logsum, float *row_loss,
                                    void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "cross_entropy: shape");
  if (dtype != RT_F32 && dtype != RT_BF16)
    return fail(RT_ERR_DTYPE, "cross_entropy: logits must be float32 or bfloat16");
  if (rows == 0) return RT_OK;
  if (logits == nullptr || targets == nullptr || row_max == nullptr || row_logsum == nullptr ||
      row_loss == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "cross_entropy: null pointer");
  if (rows > INT32_MAX) return fail(RT_ERR_UNSUPPORTED, "cross_entropy: too many rows");
  CeArgs a{};
  a.logits = logits, a.ld = ld, a.rows = rows, a.cols = cols, a.targets = targets;
  a.ignore_index = ignore_index, a.row_max = row_max, a.row_logsum = row_logsum;
  a.row_loss = row_loss;
  cudaStream_t s = as_stream(stream);
  const bool vec = cols % 4 == 0 && ld % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(logits) & (dtype == RT_F32 ? 15 : 7)) == 0 &&
                   cols <= static_cast<int64_t>(CE_THREADS) * 4 * CE_VEC;
  const unsigned grid = static_cast<unsigned>(rows);
  if (vec && dtype == RT_F32)
    launch_k(ce_fwd_vec_kernel<float>, grid, CE_THREADS, 0, s, a);
  else if (vec)
    launch_k(ce_fwd_vec_kernel<uint16_t>, grid, CE_THREADS, 0, s, a);
  else if (dtype == RT_F32)
    launch_k(ce_fwd_generic_kernel<float>, grid, CE_THREADS, 0, s, a);
  else
    launch_k(ce_fwd_generic_kernel<uint16_t>, grid, CE_THREADS, 0, s, a);
  return check_launch("cross_entropy_fwd");
}

extern "C" int rt_cross_entropy_bwd(const void *logits, int dtype, int64_t ld, int64_t rows,
                                    int64_t cols, const int64_t *targets, int64_t ignore_index,
                                    const float *row_max, const float *row_logsum,
                                    const float *grad_loss, const float *count,
                                    const float *extra_grad, int64_t ld_extra, void *grad_bf16,
                                    int64_t ldo, void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "cross_entropy: shape");
  if (dtype != RT_F32 && dtype != RT_BF16)
    return fail(RT_ERR_DTYPE, "cross_entropy: logits must be float32 or bfloat16");
  if (rows == 0) return RT_OK;
  if (logits == nullptr || targets == nullptr || row_max == nullptr || row_logsum == nullptr ||
      grad_loss == nullptr || count == nullptr || grad_bf16 == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "cross_entropy: null pointer");
  if (rows > INT32_MAX) return fail(RT_ERR_UNSUPPORTED, "cross_entropy: too many rows");
  CeArgs a{};
  a.logits = logits, a.ld = ld, a.rows = rows, a.cols = cols, a.targets = targets;
  a.ignore_index = ignore_index;
  a.row_max = const_cast<float *>(row_max), a.row_logsum = const_cast<float *>(row_logsum);
  a.grad_loss = grad_loss, a.count = count, a.extra = extra_grad, a.ld_extra = ld_extra;
  a.out = static_cast<uint16_t *>(grad_bf16), a.ldo = ldo;
  cudaStream_t s = as_stream(stream);
  const unsigned grid = static_cast<unsigned>(rows);
  if (dtype == RT_F32)
    launch_k(ce_bwd_kernel<float>, grid, CE_THREADS, 0, s, a);
  else
    launch_k(ce_bwd_kernel<uint16_t>, grid, CE_THREADS, 0, s, a);
  return check_launch("cross_entropy_bwd");
}
