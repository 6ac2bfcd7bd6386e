// rt_rowops.cuh — HBM-bound row kernels: per-token int8 quantisation (round-to-nearest and
// Philox stochastic rounding), the ratchet update, pressure leak, unpack, validation, the
// activation dequant of the grad_weight operand and the fused producers of pre-quantised inputs
// with their backwards.
//
// Layout: a row is cut into 8-element chunks (one 16-byte load for bf16, two for fp32).  RT
// threads serve a row (32: a warp per row, 8 rows per 256-thread CTA; 128: 2 rows per CTA; 256: one
// row per CTA) and each thread keeps VPT chunks in registers (chunk c = t + RT·i), so HBM sees one
// read of every input and one write of every output.  Rows whose pointers or strides do not allow
// 16-byte access, or that are longer than 256·8·8 elements, run the generic kernels (one CTA per
// row, chunk loop) with identical arithmetic.
//
// Canonical row sum (mirrored bit-for-bit by oracle/ratchet_oracle.c canonical_sum):
//   level 1  256 partials T_t; T_t adds the elements of chunks c ≡ t (mod 256) in index order from
//            +0.0f (a warp-per-row lane keeps 8 of them, a CTA-per-row thread one);
//   level 2  S_s = ((T_s+T_s+32)+(T_s+64+T_s+96)) + ((T_s+128+T_s+160)+(T_s+192+T_s+224)), s<32;
//   level 3  xor butterfly over S_0..S_31 (offsets 16, 8, 4, 2, 1).
// Every sum a kernel here takes over a row (mean squares, dot products) uses this order.
#pragma once

#include <cfloat>
#include <mutex>

#include "rt_common.cuh"

namespace rt {

constexpr int CTA = 256;

// ------------------------------------------------------------------------------------ chunk I/O
__device__ __forceinline__ void ld8(const float *p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
  const float4 b = __ldg(reinterpret_cast<const float4 *>(p) + 1);
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
__device__ __forceinline__ void ld8(const __nv_bfloat16 *p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4 *>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[2 * j] = __uint_as_float(w[j] << 16);
    v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ void st8(float *p, const float (&v)[8]) {
  reinterpret_cast<float4 *>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4 *>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);  // one paired RN conversion
  return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ void st8(__nv_bfloat16 *p, const float (&v)[8]) {
  uint4 u;
  u.x = bf16x2_bits(v[0], v[1]);
  u.y = bf16x2_bits(v[2], v[3]);
  u.z = bf16x2_bits(v[4], v[5]);
  u.w = bf16x2_bits(v[6], v[7]);
  *reinterpret_cast<uint4 *>(p) = u;
}
__device__ __forceinline__ uint2 pack_i8x8(const int8_t (&q)[8]) {
  uint2 o;
  o.x = uint32_t(uint8_t(q[0])) | (uint32_t(uint8_t(q[1])) << 8) | (uint32_t(uint8_t(q[2])) << 16) |
        (uint32_t(uint8_t(q[3])) << 24);
  o.y = uint32_t(uint8_t(q[4])) | (uint32_t(uint8_t(q[5])) << 8) | (uint32_t(uint8_t(q[6])) << 16) |
        (uint32_t(uint8_t(q[7])) << 24);
  return o;
}
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

// --------------------------------------------------------------------------- row reductions
__device__ __forceinline__ float tree8(const float (&a)[8]) {
  return __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                   __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
}
// acc[k] is the level-1 partial T_{t + RT·k}.  `sm` holds (CTA/RT)·CTA floats and `smb` CTA/RT
// floats when RT > 32.  Every thread of the CTA must call it (it synchronises the CTA).
template <int RT>
__device__ __forceinline__ float row_sum(const float (&acc)[CTA / RT], float *sm, float *smb,
                                         int sub, int t) {
  if constexpr (RT == 32) {
    return warp_sum_butterfly(tree8(acc));
  } else {
    constexpr int NT = CTA / RT;
    float *rowsm = sm + sub * CTA;
#pragma unroll
    for (int k = 0; k < NT; ++k) rowsm[t + RT * k] = acc[k];
    __syncthreads();
    if (t < 32) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = rowsm[t + 32 * j];
      const float s = warp_sum_butterfly(tree8(v));
      if (t == 0) smb[sub] = s;
    }
    __syncthreads();
    return smb[sub];
  }
}
// row maximum (order-free); `smx` holds (CTA/RT)·8 floats when RT > 32.
template <int RT>
__device__ __forceinline__ float row_max(float v, float *smx, int sub, int t) {
  v = warp_max(v);
  if constexpr (RT == 32) {
    return v;
  } else {
    __syncthreads();
    if ((t & 31) == 0) smx[sub * 8 + (t >> 5)] = v;
    __syncthreads();
    float m = smx[sub * 8];
#pragma unroll
    for (int w = 1; w < RT / 32; ++w) m = fmaxf(m, smx[sub * 8 + w]);
    return m;
  }
}
// CTA-per-row versions (RT = 256, one level-1 partial per thread) for the generic kernels.
__device__ __forceinline__ float cta_row_sum(float partial, float *sm, float *smb) {
  const float acc[1] = {partial};
  return row_sum<CTA>(acc, sm, smb, 0, threadIdx.x);
}
__device__ __forceinline__ float cta_max(float v, float *smx) {
  return row_max<CTA>(v, smx, 0, threadIdx.x);
}

// --------------------------------------------------------------------------- quantisation
// int8_matmul.py:139-148.  The reference rounds RN(v / scale); only its rounding decision
// matters, so the quotient is first formed as v · RN(1/scale) (within 1.5 ulp of RN(v / scale),
// i.e. below 2^-15 since |v / scale| <= 127.5) and the IEEE division is taken only when that
// estimate lies within 2^-12 of a rounding boundary (a half-integer for rint, an integer after
// adding u for stochastic rounding) — the result is the one of the exact quotient.
constexpr float kBoundaryWindow = 2.44140625e-4f;  // 2^-12
constexpr float kRoundMagic = 12582912.0f;            // 1.5 * 2^23
// Round-to-nearest-even quant of one value, as an int in [-127, 127].  The estimate is clamped
// first (clamping commutes with rounding at the integer bounds) and rounded by adding 1.5·2^23,
// whose low mantissa bits then hold the integer.
__device__ __forceinline__ int quant_rn_i(float v, float scale, float rcp) {
  const float y = fminf(fmaxf(__fmul_rn(v, rcp), -127.0f), 127.0f);
  const float t = __fadd_rn(y, kRoundMagic);
  if (fabsf(__fsub_rn(y, __fsub_rn(t, kRoundMagic))) >= 0.5f - kBoundaryWindow)
    return static_cast<int>(rintf(fminf(fmaxf(__fdiv_rn(v, scale), -127.0f), 127.0f)));
  return __float_as_int(t) - 0x4B400000;
}
// Stochastic rounding floor(RN(RN(v / scale) + u)), as an int in [-127, 127], given um = u - 1/2.
// th = fma(v, rcp, um) lies within 2^-15 of RN(v / scale) + u - 1/2 (the reciprocal estimate,
// the division's and the fma's roundings), so RN(th), taken through the rounding magic, is
// floor(RN(RN(v / scale) + u)) unless th lies within the window of a half-integer; those
// elements go to the IEEE division, the reference's two roundings, floor and clamp.  Outside the
// window the estimate stays within (-128, 128), so the fast path needs no clamp.
__device__ __forceinline__ int quant_sr_i(float v, float scale, float rcp, float um) {
  const float th = __fmaf_rn(v, rcp, um);
  const float z = __fadd_rn(th, kRoundMagic);
  if (fabsf(__fsub_rn(th, __fsub_rn(z, kRoundMagic))) >= 0.5f - kBoundaryWindow) {
    const float t = __fadd_rn(__fdiv_rn(v, scale), __fadd_rn(um, 0.5f));  // u exact
    return min(max(__float2int_rd(t), -127), 127);
  }
  return __float_as_int(z) - 0x4B400000;
}
// quant_rn_i that also returns the rounded value as a float (exact: a small integer), which the
// rounding magic has produced already -- no int-to-float conversion for the dequantised copy.
__device__ __forceinline__ int quant_rn_if(float v, float scale, float rcp, float &qf) {
  const float y = fminf(fmaxf(__fmul_rn(v, rcp), -127.0f), 127.0f);
  const float t = __fadd_rn(y, kRoundMagic);
  qf = __fsub_rn(t, kRoundMagic);
  if (fabsf(__fsub_rn(y, qf)) >= 0.5f - kBoundaryWindow) {
    qf = rintf(fminf(fmaxf(__fdiv_rn(v, scale), -127.0f), 127.0f));
    return static_cast<int>(qf);
  }
  return __float_as_int(t) - 0x4B400000;
}
__device__ __forceinline__ int8_t quant_rn(float v, float scale, float rcp) {
  return static_cast<int8_t>(quant_rn_i(v, scale, rcp));
}
__device__ __forceinline__ int8_t quant_sr(float v, float scale, float rcp, float um) {
  return static_cast<int8_t>(quant_sr_i(v, scale, rcp, um));
}
// Four ints in [-128, 127] -> one word of int8 bytes (two byte permutes and a merge).
__device__ __forceinline__ uint32_t pack4_i8(int a, int b, int c, int d) {
  const uint32_t lo = __byte_perm(static_cast<uint32_t>(a), static_cast<uint32_t>(b), 0x0040);
  const uint32_t hi = __byte_perm(static_cast<uint32_t>(c), static_cast<uint32_t>(d), 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}
__device__ __forceinline__ float row_scale_of(float amax) {
  return fmaxf(__fdiv_rn(amax, 127.0f), FLT_MIN);
}

// Round-to-nearest quant of eight values into one 8-byte int8 chunk; with dq, also the chunk of
// bf16(bf16(q) · sb), sb = bf16(row scale): the grad_weight operand that the backward otherwise
// dequantises from the saved int8 rows (ratchet.py:73-76), written here from registers.
__device__ __forceinline__ void quant_rn_store8(int8_t *qp, unsigned short *dq, const float (&v)[8],
                                                float scale, float rcp, float sb) {
  int qi[8];
  float qf[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) qi[j] = quant_rn_if(v[j], scale, rcp, qf[j]);
  uint2 o;
  o.x = pack4_i8(qi[0], qi[1], qi[2], qi[3]);
  o.y = pack4_i8(qi[4], qi[5], qi[6], qi[7]);
  *reinterpret_cast<uint2 *>(qp) = o;
  if (dq != nullptr) {
    float d[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) d[j] = __fmul_rn(qf[j], sb);
    st8(reinterpret_cast<__nv_bfloat16 *>(dq), d);
  }
}

// Row-kernel configuration: threads per row and chunks per thread for a row of `nch` chunks.
struct RowCfg {
  int rt, vpt;  // rt == 0: generic kernel
};
static inline int pow2_at_least(int64_t v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}
// At most two chunks per thread while a CTA per row allows it: the row stays in registers
// without capping occupancy (eight chunks held 86 registers and left a quarter of the warp
// slots in use), and more resident warps hide each row's load -> reduce -> store chain.  Few
// rows get more threads each (up to a CTA per row) so that the grid fills the GPU.
static inline RowCfg row_cfg(int64_t nch, int64_t rows = INT64_MAX) {
  const int64_t want_threads = 148 * 2048;
  if (nch > 256 * 8) return {0, 0};
  int rt = nch <= 32 * 2 ? 32 : (nch <= 128 * 2 ? 128 : 256);
  // (rows < want / rt, not rows * rt < want: the default row count would overflow the product)
  while (rt < 256 && rows < want_threads / rt && nch > rt) rt = rt == 32 ? 128 : 256;
  return {rt, pow2_at_least((nch + rt - 1) / rt)};
}
// Kernels holding four row arrays per chunk (RMSNorm backward) keep at most 2 chunks per thread.
static inline RowCfg row_cfg_narrow(int64_t nch) {
  if (nch <= 32) return {32, 1};
  if (nch <= 64) return {32, 2};
  if (nch <= 256) return {128, 2};
  if (nch <= 512) return {256, 2};
  return {0, 0};
}
// Resident 256-thread CTAs per SM of the grid-striding row kernels, whose launch bounds give
// four at up to two chunks a thread, two at four, one at eight.
static inline unsigned resident_ctas(int vpt) { return vpt <= 2 ? 4u : (vpt == 4 ? 2u : 1u); }
// Grid of the persistent update kernels: the row blocks, at most the CTAs resident at once.
static inline unsigned update_grid(unsigned blocks, int vpt) {
  int sms = 0;
  if (rt_sm_count(&sms) != RT_OK || sms <= 0) sms = 148;
  const unsigned cap = static_cast<unsigned>(sms) * resident_ctas(vpt);
  return blocks < cap ? blocks : cap;
}
static inline unsigned row_grid(int64_t rows, int rt) {
  const int64_t rpc = CTA / rt;
  return static_cast<unsigned>((rows + rpc - 1) / rpc);
}

#define RT_DISPATCH_ROW(cfg, KERNEL, T, GRID, ...)                                 \
  do {                                                                               \
    switch ((cfg).rt * 16 + (cfg).vpt) {                                             \
      case 32 * 16 + 1: launch_k(KERNEL<T, 32, 1>, GRID, CTA, 0, s, __VA_ARGS__); break;   \
      case 32 * 16 + 2: launch_k(KERNEL<T, 32, 2>, GRID, CTA, 0, s, __VA_ARGS__); break;   \
      case 32 * 16 + 4: launch_k(KERNEL<T, 32, 4>, GRID, CTA, 0, s, __VA_ARGS__); break;   \
      case 32 * 16 + 8: launch_k(KERNEL<T, 32, 8>, GRID, CTA, 0, s, __VA_ARGS__); break;   \
      case 128 * 16 + 1: launch_k(KERNEL<T, 128, 1>, GRID, CTA, 0, s, __VA_ARGS__); break; \
      case 128 * 16 + 2: launch_k(KERNEL<T, 128, 2>, GRID, CTA, 0, s, __VA_ARGS__); break; \
      case 128 * 16 + 4: launch_k(KERNEL<T, 128, 4>, GRID, CTA, 0, s, __VA_ARGS__); break; \
      case 128 * 16 + 8: launch_k(KERNEL<T, 128, 8>, GRID, CTA, 0, s, __VA_ARGS__); break; \
      case 256 * 16 + 1: launch_k(KERNEL<T, 256, 1>, GRID, CTA, 0, s, __VA_ARGS__); break; \
      case 256 * 16 + 2: launch_k(KERNEL<T, 256, 2>, GRID, CTA, 0, s, __VA_ARGS__); break; \
      case 256 * 16 + 4: launch_k(KERNEL<T, 256, 4>, GRID, CTA, 0, s, __VA_ARGS__); break; \
      default: launch_k(KERNEL<T, 256, 8>, GRID, CTA, 0, s, __VA_ARGS__); break;           \
    }                                                                                \
  } while (0)

#define RT_DISPATCH_ROW_NARROW(cfg, KERNEL, T, GRID, ...)                           \
  do {                                                                               \
    switch ((cfg).rt * 16 + (cfg).vpt) {                                             \
      case 32 * 16 + 1: launch_k(KERNEL<T, 32, 1>, GRID, CTA, 0, s, __VA_ARGS__); break;   \
      case 32 * 16 + 2: launch_k(KERNEL<T, 32, 2>, GRID, CTA, 0, s, __VA_ARGS__); break;   \
      case 128 * 16 + 2: launch_k(KERNEL<T, 128, 2>, GRID, CTA, 0, s, __VA_ARGS__); break; \
      default: launch_k(KERNEL<T, 256, 2>, GRID, CTA, 0, s, __VA_ARGS__); break;           \
    }                                                                                \
  } while (0)

#define RT_DISPATCH_ROW_NARROW_SMEM(cfg, KERNEL, T, GRID, SMEM, ...)                        \
  do {                                                                                        \
    switch ((cfg).rt * 16 + (cfg).vpt) {                                                      \
      case 32 * 16 + 1: launch_k(KERNEL<T, 32, 1>, GRID, CTA, SMEM, s, __VA_ARGS__); break;         \
      case 32 * 16 + 2: launch_k(KERNEL<T, 32, 2>, GRID, CTA, SMEM, s, __VA_ARGS__); break;         \
      case 128 * 16 + 2: launch_k(KERNEL<T, 128, 2>, GRID, CTA, SMEM, s, __VA_ARGS__); break;       \
      default: launch_k(KERNEL<T, 256, 2>, GRID, CTA, SMEM, s, __VA_ARGS__); break;                 \
    }                                                                                         \
  } while (0)

// ===========================================================================================
// Row quantisation (int8_matmul.py:106-150).
// ===========================================================================================
struct QuantArgs {
  const void *x;
  int64_t rows, cols, stride_row, stride_col;
  const float *col_scale;
  int stochastic;
  int round_bf16;  // fp32 input rounded to bf16 before anything else
  uint64_t seed;
  uint32_t step, layer;
  uint32_t *step_dev;
  int8_t *q;
  int64_t ldq;
  float *row_scale;
  unsigned short *xbf16;
  int64_t ld_xbf16;
};

// Step of the stochastic-rounding stream: step_dev[0] when given (read by every thread at the
// start).  After all its threads have used it, each CTA reports on step_dev[1]; the last CTA of
// the launch resets that count and advances step_dev[0] by one, so consecutive calls draw fresh
// streams with no host work per call (a captured graph advances it on every replay).
__device__ __forceinline__ uint32_t sr_step_read(const QuantArgs &a) {
  return a.step_dev != nullptr ? *reinterpret_cast<const volatile uint32_t *>(a.step_dev)
                               : a.step;
}
// Whole CTA, after the last use of `step`.
__device__ __forceinline__ void sr_step_arrive(const QuantArgs &a, uint32_t step) {
  if (a.step_dev == nullptr) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.step_dev + 1, 1u) == gridDim.x - 1) {
      a.step_dev[1] = 0u;
      __threadfence();
      atomicExch(a.step_dev, step + 1u);
    }
  }
}

// Two entry points over one body.  The resident-sized grid of the dispatch counts on four CTAs
// per SM at up to two chunks a thread: the bf16 variants compile to 64 registers unforced, the
// fp32 ones (70 registers unforced) are held to it by their launch bounds.  Forcing the bf16
// variants too cost 11 % (more instructions at the same register count); leaving them unbounded
// under an explicit minimum of one CTA gave 92 registers and 80 instead of 55 us (2048 wide).
template <typename T, int RT, int VPT>
__device__ __forceinline__ void quant_rows_body(const QuantArgs &a);
template <typename T, int RT, int VPT>
__global__ void __launch_bounds__(CTA) quant_rows_kernel(QuantArgs a) {
  pdl_wait();
  pdl_trigger();
  quant_rows_body<T, RT, VPT>(a);
}
template <typename T, int RT, int VPT>
__global__ void __launch_bounds__(CTA, 4) quant_rows_f32_kernel(QuantArgs a) {
  pdl_wait();
  pdl_trigger();
  quant_rows_body<T, RT, VPT>(a);
}
template <typename T, int RT, int VPT>
__device__ __forceinline__ void quant_rows_body(const QuantArgs &a) {
  // grid-stride over groups of RPC rows: a resident-sized grid (few CTAs, so that the step
  // ticket of sr_step_arrive costs one atomic per resident CTA)
  constexpr int RPC = CTA / RT;
  __shared__ float smx[RPC * 8];
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t nch = a.cols / 8;
  const int64_t groups = (a.rows + RPC - 1) / RPC;
  const uint32_t step = sr_step_read(a);
  // this thread's chunks are the same columns in every row: their scales stay in registers
  float cs[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (a.col_scale != nullptr && c < nch) {
      ld8(a.col_scale + 8 * c, cs[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) cs[i][j] = 1.0f;
    }
  }
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t row = grp * RPC + sub;
    const bool live = row < a.rows;
    const T *xr = static_cast<const T *>(a.x) + (live ? row : 0) * a.stride_row;
    float v[VPT][8];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t c = t + static_cast<int64_t>(i) * RT;
      if (live && c < nch) {
        ld8(xr + 8 * c, v[i]);
        if (a.round_bf16) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = bf16_round(v[i][j]);
        }
        if (a.xbf16 != nullptr)
          st8(reinterpret_cast<__nv_bfloat16 *>(a.xbf16 + row * a.ld_xbf16 + 8 * c), v[i]);
        if (a.col_scale != nullptr) {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[i][j] = __fmul_rn(v[i][j], cs[i][j]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
      }
    }
    amax = row_max<RT>(amax, smx, sub, t);  // CTA-uniform trip count: its barriers are safe
    const float scale = row_scale_of(amax);
    const float rcp = __frcp_rn(scale);
    if (live && t == 0) a.row_scale[row] = scale;
    int8_t *qr = a.q + (live ? row : 0) * a.ldq;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t c = t + static_cast<int64_t>(i) * RT;
      if (!live || c >= nch) continue;
      uint2 o;
      if (a.stochastic) {
        const uint64_t e0 = static_cast<uint64_t>(row) * a.cols + 8 * c;  // multiple of 8
        const Philox4 p = sr_block(a.seed, step, a.layer, e0 >> 3);
        o.x = pack4_i8(quant_sr_i(v[i][0], scale, rcp, sr_um_lo(p.x)),
                       quant_sr_i(v[i][1], scale, rcp, sr_um_hi(p.x)),
                       quant_sr_i(v[i][2], scale, rcp, sr_um_lo(p.y)),
                       quant_sr_i(v[i][3], scale, rcp, sr_um_hi(p.y)));
        o.y = pack4_i8(quant_sr_i(v[i][4], scale, rcp, sr_um_lo(p.z)),
                       quant_sr_i(v[i][5], scale, rcp, sr_um_hi(p.z)),
                       quant_sr_i(v[i][6], scale, rcp, sr_um_lo(p.w)),
                       quant_sr_i(v[i][7], scale, rcp, sr_um_hi(p.w)));
      } else {
        o.x = pack4_i8(quant_rn_i(v[i][0], scale, rcp), quant_rn_i(v[i][1], scale, rcp),
                       quant_rn_i(v[i][2], scale, rcp), quant_rn_i(v[i][3], scale, rcp));
        o.y = pack4_i8(quant_rn_i(v[i][4], scale, rcp), quant_rn_i(v[i][5], scale, rcp),
                       quant_rn_i(v[i][6], scale, rcp), quant_rn_i(v[i][7], scale, rcp));
      }
      *reinterpret_cast<uint2 *>(qr + 8 * c) = o;
    }
  }
  sr_step_arrive(a, step);
}

// Generic: any strides, one CTA per row, two passes (the second normally hits L2).
template <typename T>
__global__ void __launch_bounds__(CTA) quant_rows_generic_kernel(QuantArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ float smx[8];
  const int64_t row = blockIdx.x;
  const T *xr = static_cast<const T *>(a.x) + row * a.stride_row;
  const uint32_t step = sr_step_read(a);
  float amax = 0.0f;
  for (int64_t k = threadIdx.x; k < a.cols; k += CTA) {
    float v = load_as_float<T>(xr + k * a.stride_col);
    if (a.round_bf16) v = bf16_round(v);
    if (a.xbf16 != nullptr) a.xbf16[row * a.ld_xbf16 + k] = bf16_bits(v);
    if (a.col_scale != nullptr) v = __fmul_rn(v, __ldg(a.col_scale + k));
    amax = fmaxf(amax, fabsf(v));
  }
  amax = cta_max(amax, smx);
  const float scale = row_scale_of(amax);
  const float rcp = __frcp_rn(scale);
  if (threadIdx.x == 0) a.row_scale[row] = scale;
  for (int64_t k = threadIdx.x; k < a.cols; k += CTA) {
    float v = load_as_float<T>(xr + k * a.stride_col);
    if (a.round_bf16) v = bf16_round(v);
    if (a.col_scale != nullptr) v = __fmul_rn(v, __ldg(a.col_scale + k));
    int8_t o;
    if (a.stochastic) {
      const uint64_t e = static_cast<uint64_t>(row) * a.cols + k;
      const Philox4 p = sr_block(a.seed, step, a.layer, e >> 3);
      const uint32_t w = philox_word(p, static_cast<int>((e & 7) >> 1));
      o = quant_sr(v, scale, rcp, (e & 1) ? sr_um_hi(w) : sr_um_lo(w));
    } else {
      o = quant_rn(v, scale, rcp);
    }
    a.q[row * a.ldq + k] = o;
  }
  sr_step_arrive(a, step);
}

// ---- Fixed-point stochastic rounding (the staged quantiser and the fused producer backwards).
// Same results as quant_sr_i (floor(RN(RN(v / scale) + u)), clamped), with the rounding decision
// made in fixed point.  With R = RN(1/scale)·2^15 (exact scaling),
//    t = fma(v, R, 1.5·2^23 + 2) rounds v·R + 2 to an integer T + 2 (|v·R| < 2^22 keeps t in
//    [2^23, 2^24), where consecutive integers have consecutive bit patterns).  For the element's
//    16-bit draw h (u = (h + 1/2)·2^-16),  W = 2·bits(t) + h + 2^23  equals
//    0x97000000 + Z + 4 (mod 2^32) with Z = 2T + h, the sum RN(v/scale)·2^16 + h + 1/2 estimated
//    to within 2.25 units (reciprocal 0.25·2, integer rounding 0.5·2, the quotient's rounding
//    2^-18·2^16).  The reference sum RN(q0 + u) moves by at most 0.5 more, so unless Z lies within
//    2.75 of a multiple of 2^16 — exactly when the low 16 bits of W are below 7 — floor(sum) is
//    Z >> 16, whose low byte is byte 2 of W.  Those elements take the IEEE division instead.
//    |q0| <= 127 + 2^-17 and u <= 1 - 2^-17 bound the sum by 128, and a sum within 2.75 units of
//    ±127 or 128 is always re-done exactly, so the fast path needs no clamp.
//    Zero rows take R = 0 (every value 0, t = 2^23·1.5 + 2); rows whose reciprocal exceeds 2^100
//    (amax below ~1e-28) are done exactly throughout.
constexpr float kSrFixedMagic = 12582914.0f;  // 1.5·2^23 + 2

// int8 bytes of eight fast-path words (byte 2 of each) and whether any needs the exact path.
__device__ __forceinline__ uint2 sr_fixed_pack(const uint32_t (&w)[8]) {
  const uint32_t a = __byte_perm(w[0], w[1], 0x0062), b = __byte_perm(w[2], w[3], 0x0062);
  const uint32_t c = __byte_perm(w[4], w[5], 0x0062), d = __byte_perm(w[6], w[7], 0x0062);
  return make_uint2(__byte_perm(a, b, 0x5410), __byte_perm(c, d, 0x5410));
}
// (the low 16 bits of each word moved to the top by a multiply, then three-way minima)
__device__ __forceinline__ bool sr_fixed_ambiguous(const uint32_t (&w)[8]) {
  uint32_t m = __vimin3_u32(w[0] * 65536u, w[1] * 65536u, w[2] * 65536u);
  m = __vimin3_u32(m, w[3] * 65536u, w[4] * 65536u);
  m = __vimin3_u32(m, w[5] * 65536u, w[6] * 65536u);
  return min(m, w[7] * 65536u) < (7u << 16);
}
// h + 2^23 for the low / high 16-bit half of a Philox word (one byte permute each).
__device__ __forceinline__ uint32_t sr_h_lo(uint32_t word) {
  return __byte_perm(word, 0x00800000u, 0x7610);
}
__device__ __forceinline__ uint32_t sr_h_hi(uint32_t word) {
  return __byte_perm(word, 0x00800000u, 0x7632);
}
// The exact path for one element: the reference's two roundings, floor and clamp.
__device__ __forceinline__ int sr_exact(float v, float scale, uint32_t hbits) {
  // hbits = h + 2^23; u = (h + 1/2)·2^-16 built exactly in a float's mantissa
  const float u = __uint_as_float(0x3F800040u | ((hbits & 0xFFFFu) << 7)) - 1.0f;
  const float t = __fadd_rn(__fdiv_rn(v, scale), u);
  return min(max(__float2int_rd(t), -127), 127);
}

// ---- pieces of the stochastic-rounding row quantisation shared by the fused gradient producers
// (a producer that already holds a layer's output-gradient row in registers quantises it for
// the layer's int8 grad_input GEMM in the same pass, with the arithmetic of quant_rows_kernel).
template <int RT, int VPT>
__device__ __forceinline__ void sr_load_col_scales(const QuantArgs &a, int t, int64_t nch,
                                                   float (&cs)[VPT][8]) {
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (a.col_scale != nullptr && c < nch) {
      ld8(a.col_scale + 8 * c, cs[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) cs[i][j] = 1.0f;
    }
  }
}
// One chunk of the gradient as the layer receives it -> the value the quantiser rounds: the
// optional bf16 rounding, the bf16 copy (grad_weight operand), the column scale; amax updated.
__device__ __forceinline__ void sr_prepare_chunk(const QuantArgs &a, int64_t row, int64_t c,
                                                 float (&v)[8], const float (&cs)[8],
                                                 float &amax) {
  if (a.round_bf16) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = bf16_round(v[j]);
  }
  if (a.xbf16 != nullptr)
    st8(reinterpret_cast<__nv_bfloat16 *>(a.xbf16 + row * a.ld_xbf16 + 8 * c), v);
  if (a.col_scale != nullptr) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __fmul_rn(v[j], cs[j]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
}
// The int8 row of prepared values with the row's scale already known: fixed-point decisions, then
// a warp-uniform pass that redraws the flagged chunks and overwrites them with the exact result
// (whole warps call it: RT >= 32 keeps each row's threads in whole warps).
template <int RT, int VPT>
__device__ __forceinline__ void sr_fixed_store_row(const QuantArgs &a, uint32_t step, int64_t row,
                                                   int t, int64_t nch, const float (&v)[VPT][8],
                                                   float amax, float scale, float rcp, bool live) {
  const bool row_exact = amax != 0.0f && rcp > 0x1p100f;
  const float r15 = (amax == 0.0f || row_exact) ? 0.0f : __fmul_rn(rcp, 32768.0f);
  int8_t *qr = a.q + (live ? row : 0) * a.ldq;
  uint32_t redo = 0;  // this thread's chunks whose bytes the exact path re-does
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (!live || c >= nch) continue;
    const uint64_t e0 = static_cast<uint64_t>(row) * a.cols + 8 * c;  // multiple of 8
    const Philox4 p = sr_block(a.seed, step, a.layer, e0 >> 3);
    const uint32_t pw[4] = {p.x, p.y, p.z, p.w};
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      w[j] = __float_as_uint(__fmaf_rn(v[i][j], r15, kSrFixedMagic)) * 2u +
             ((j & 1) ? sr_h_hi(pw[j >> 1]) : sr_h_lo(pw[j >> 1]));
    if (row_exact || sr_fixed_ambiguous(w)) redo |= 1u << i;
    *reinterpret_cast<uint2 *>(qr + 8 * c) = sr_fixed_pack(w);
  }
  // rare (a few elements in 10^4, or a row of tiny maximum)
  if (__any_sync(0xffffffffu, redo != 0)) {
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      if (((redo >> i) & 1u) == 0) continue;
      const int64_t c = t + static_cast<int64_t>(i) * RT;
      const uint64_t e0 = static_cast<uint64_t>(row) * a.cols + 8 * c;
      const Philox4 p = sr_block(a.seed, step, a.layer, e0 >> 3);
      const uint32_t pw[4] = {p.x, p.y, p.z, p.w};
      int q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        q[j] = sr_exact(v[i][j], scale, (j & 1) ? sr_h_hi(pw[j >> 1]) : sr_h_lo(pw[j >> 1]));
      *reinterpret_cast<uint2 *>(qr + 8 * c) =
          make_uint2(pack4_i8(q[0], q[1], q[2], q[3]), pack4_i8(q[4], q[5], q[6], q[7]));
    }
  }
}
// Row scale and int8 row from the prepared values (amax already reduced over the row).
template <int RT, int VPT>
__device__ __forceinline__ void sr_quant_store_row(const QuantArgs &a, uint32_t step, int64_t row,
                                                   int t, int64_t nch, const float (&v)[VPT][8],
                                                   float amax) {
  const float scale = row_scale_of(amax);
  const float rcp = __frcp_rn(scale);
  if (t == 0) a.row_scale[row] = scale;
  sr_fixed_store_row<RT, VPT>(a, step, row, t, nch, v, amax, scale, rcp, true);
}
// ---- Staged stochastic-rounding quantiser: the layer gradients of the int8 backward.
// Every thread copies its chunks of the row groups S-1 iterations ahead into its own slots of
// shared memory with cp.async, so HBM reads stay in flight while the current rows compute; the
// rounding is sr_fixed_store_row's.
template <typename T, int RT, int VPT, int S>
__global__ void __launch_bounds__(CTA) quant_sr_staged_kernel(QuantArgs a) {
  constexpr int RPC = CTA / RT;
  constexpr int P = static_cast<int>(sizeof(T)) / 2;  // 16-byte pieces per chunk: 1 bf16, 2 fp32
  extern __shared__ uint4 stage[];                     // [S][VPT][P][CTA] own slots
  __shared__ float smx[RPC * 8];
  pdl_wait();
  pdl_trigger();
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t nch = a.cols / 8;
  const int64_t groups = (a.rows + RPC - 1) / RPC;
  const uint32_t step = sr_step_read(a);
  const char *xbase = static_cast<const char *>(a.x);
  const int64_t row_bytes = a.stride_row * static_cast<int64_t>(sizeof(T));
  // up to two chunks a thread the column scales stay in registers; wider rows re-read them
  // (L1) for each row
  constexpr bool kCsRegs = VPT <= 2;
  float csr[kCsRegs ? VPT : 1][8];
  if constexpr (kCsRegs) sr_load_col_scales<RT, VPT>(a, t, nch, csr);

  auto issue = [&](int64_t grp, int st) {
    const int64_t row = grp * RPC + sub;
    if (grp < groups && row < a.rows) {
      const char *xr = xbase + row * row_bytes;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t c = t + static_cast<int64_t>(i) * RT;
        if (c < nch) {
#pragma unroll
          for (int p = 0; p < P; ++p)
            cp_async16(&stage[((st * VPT + i) * P + p) * CTA + threadIdx.x],
                       xr + c * (8 * static_cast<int64_t>(sizeof(T))) + 16 * p);
        }
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s = 0; s < S - 1; ++s) issue(blockIdx.x + static_cast<int64_t>(s) * gridDim.x, s);

  int st = 0;
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    issue(grp + static_cast<int64_t>(S - 1) * gridDim.x, st == 0 ? S - 1 : st - 1);
    cp_async_wait<S - 1>();
    const int64_t row = grp * RPC + sub;
    const bool live = row < a.rows;
    float v[VPT][8];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t c = t + static_cast<int64_t>(i) * RT;
      if (live && c < nch) {
        const uint4 *slot = &stage[((st * VPT + i) * P) * CTA + threadIdx.x];
        if constexpr (sizeof(T) == 2) {
          const uint4 u = slot[0];
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            v[i][2 * j] = __uint_as_float(w[j] << 16);
            v[i][2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
          }
        } else {
          const float4 lo = *reinterpret_cast<const float4 *>(slot);
          const float4 hi = *reinterpret_cast<const float4 *>(slot + CTA);
          v[i][0] = lo.x, v[i][1] = lo.y, v[i][2] = lo.z, v[i][3] = lo.w;
          v[i][4] = hi.x, v[i][5] = hi.y, v[i][6] = hi.z, v[i][7] = hi.w;
          if (a.round_bf16) {
            uint32_t pb[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              pb[j] = pack_bf16x2(v[i][2 * j], v[i][2 * j + 1]);
              v[i][2 * j] = __uint_as_float(pb[j] << 16);
              v[i][2 * j + 1] = __uint_as_float(pb[j] & 0xFFFF0000u);
            }
            if (a.xbf16 != nullptr)
              *reinterpret_cast<uint4 *>(a.xbf16 + row * a.ld_xbf16 + 8 * c) =
                  make_uint4(pb[0], pb[1], pb[2], pb[3]);
          } else if (a.xbf16 != nullptr) {
            st8(reinterpret_cast<__nv_bfloat16 *>(a.xbf16 + row * a.ld_xbf16 + 8 * c), v[i]);
          }
        }
        if constexpr (sizeof(T) == 2) {
          if (a.xbf16 != nullptr)
            *reinterpret_cast<uint4 *>(a.xbf16 + row * a.ld_xbf16 + 8 * c) = slot[0];
        }
        if (a.col_scale != nullptr) {
          float cs[8];
          if constexpr (kCsRegs) {
#pragma unroll
            for (int j = 0; j < 8; ++j) cs[j] = csr[kCsRegs ? i : 0][j];
          } else {
            ld8(a.col_scale + 8 * c, cs);
          }
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const float2 r = __fmul2_rn(make_float2(v[i][j], v[i][j + 1]),
                                        make_float2(cs[j], cs[j + 1]));
            v[i][j] = r.x, v[i][j + 1] = r.y;
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
      }
    }
    amax = row_max<RT>(amax, smx, sub, t);  // CTA-uniform trip count: its barriers are safe
    const float scale = row_scale_of(amax);
    const float rcp = __frcp_rn(scale);
    if (live && t == 0) a.row_scale[row] = scale;
    sr_fixed_store_row<RT, VPT>(a, step, row, t, nch, v, amax, scale, rcp, live);
    st = st == S - 1 ? 0 : st + 1;
  }
  cp_async_wait<0>();
  sr_step_arrive(a, step);
}

// Host: the vectorised kernels' layout conditions on the quantiser outputs.
static inline bool sr_outputs_vec(const QuantArgs &a) {
  return (reinterpret_cast<uintptr_t>(a.q) & 7) == 0 && a.ldq % 8 == 0 &&
         (a.col_scale == nullptr || aligned16(a.col_scale)) &&
         (a.xbf16 == nullptr || (aligned16(a.xbf16) && a.ld_xbf16 % 8 == 0));
}

// Resident CTAs per SM of one staged-kernel instance (its shared stages and registers), asked of
// the runtime once per instance and device (the shared-memory attribute is set on each device
// the kernel runs on; the cache is per template instance: one per kernel).
template <auto kernel>
static unsigned staged_resident(size_t smem) {
  static std::mutex mu;
  static int per_sm[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  std::lock_guard<std::mutex> lock(mu);
  if (per_sm[dev] == 0) {
    // static and dynamic shared memory together may pass the default 48 KB
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, CTA, smem) != cudaSuccess || n < 1)
      n = 1;
    per_sm[dev] = n;
  }
  int sms = 0;
  if (rt_sm_count(&sms) != RT_OK || sms <= 0) sms = 148;
  return static_cast<unsigned>(sms) * static_cast<unsigned>(per_sm[dev]);
}
template <typename T, int RT, int VPT>
static void launch_quant_sr_staged(const QuantArgs &a, cudaStream_t s) {
  constexpr int P = static_cast<int>(sizeof(T)) / 2;
  constexpr int S = VPT * P <= 2 ? 6 : 3;  // 24-48 KB of stages per CTA
  constexpr size_t smem = static_cast<size_t>(S) * VPT * P * CTA * 16;
  const unsigned resident = staged_resident<quant_sr_staged_kernel<T, RT, VPT, S>>(smem);
  const unsigned groups = row_grid(a.rows, RT);
  launch_k(quant_sr_staged_kernel<T, RT, VPT, S>, groups < resident ? groups : resident, CTA, smem,
           s, a);
}
// The staged kernel takes the vectorised stochastic cases whose chunks fit 48 KB of stages.
template <typename T>
static bool quant_sr_staged(const QuantArgs &a, const RowCfg &cfg, cudaStream_t s) {
  if (!a.stochastic || !staged_enabled()) return false;
  switch (cfg.rt * 16 + cfg.vpt * static_cast<int>(sizeof(T)) / 2) {
    case 32 * 16 + 1: launch_quant_sr_staged<T, 32, 1>(a, s); return true;
    case 128 * 16 + 1: launch_quant_sr_staged<T, 128, 1>(a, s); return true;
    case 256 * 16 + 1: launch_quant_sr_staged<T, 256, 1>(a, s); return true;
    case 32 * 16 + 2: launch_quant_sr_staged<T, 32, sizeof(T) == 2 ? 2 : 1>(a, s); return true;
    case 128 * 16 + 2: launch_quant_sr_staged<T, 128, sizeof(T) == 2 ? 2 : 1>(a, s); return true;
    case 256 * 16 + 2: launch_quant_sr_staged<T, 256, sizeof(T) == 2 ? 2 : 1>(a, s); return true;
    case 32 * 16 + 4: launch_quant_sr_staged<T, 32, sizeof(T) == 2 ? 4 : 2>(a, s); return true;
    case 128 * 16 + 4: launch_quant_sr_staged<T, 128, sizeof(T) == 2 ? 4 : 2>(a, s); return true;
    case 256 * 16 + 4: launch_quant_sr_staged<T, 256, sizeof(T) == 2 ? 4 : 2>(a, s); return true;
    default: return false;
  }
}

template <typename T>
static int quant_rows_dispatch(const QuantArgs &a, cudaStream_t s) {
  const size_t es = sizeof(T);
  const bool vec = a.stride_col == 1 && aligned16(a.x) && (a.stride_row * es) % 16 == 0 &&
                   a.cols % 8 == 0 && (reinterpret_cast<uintptr_t>(a.q) & 7) == 0 && a.ldq % 8 == 0 &&
                   (a.col_scale == nullptr || aligned16(a.col_scale)) &&
                   (a.xbf16 == nullptr || (aligned16(a.xbf16) && a.ld_xbf16 % 8 == 0));
  const RowCfg cfg = vec ? row_cfg(a.cols / 8, a.rows) : RowCfg{0, 0};
  if (cfg.rt != 0 && quant_sr_staged<T>(a, cfg, s)) {
    // launched
  } else if (cfg.rt != 0) {
    int sms = 0;
    if (int rc = rt_sm_count(&sms)) return rc;
    // CTAs per SM that stay resident (the kernels' launch bounds: 4 up to two chunks a thread)
    const unsigned resident = static_cast<unsigned>(sms) * resident_ctas(cfg.vpt);
    const unsigned groups = row_grid(a.rows, cfg.rt);
    const unsigned grid = groups < resident ? groups : resident;
    if (sizeof(T) == 4 && cfg.vpt <= 2)
      RT_DISPATCH_ROW(cfg, quant_rows_f32_kernel, T, grid, a);
    else
      RT_DISPATCH_ROW(cfg, quant_rows_kernel, T, grid, a);
  } else {
    launch_k(quant_rows_generic_kernel<T>, static_cast<unsigned>(a.rows), CTA, 0, s, a);
  }
  return check_launch("rt_quantize_rows");
}

// ===========================================================================================
// Ratchet update (ratchet.py:248-301, 487-556, 582-611).
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
  float *row_rms, *rms_sum, *grad_scale;
  // grad_W as split-K partial tiles of the grad_weight GEMM instead of `grad`: element (n, k) is
  // the sum, in split order, of ws[s·ws_split_stride + ((n/128)·ws_tiles_n + k/ws_bn)·128·ws_bn
  // + (n%128)·ws_bn + k%ws_bn] (the order of the split-K reduce)
  const float *ws;
  int ws_splits, ws_tiles_n, ws_bn;
  int64_t ws_split_stride;
  // the gradient is multiplied by grad_mul after the optional bf16 rounding (1: untouched); the
  // mean over ranks / micro-batches of summed gradients, exact for powers of two
  float grad_mul;
  // optional: gradient row r updates state row row_ids[r] (packed, code, rms_ema, row outputs);
  // rows with row_ids[r] < 0 are skipped (the row-sparse embedding update)
  const int64_t *row_ids;
};

struct Moves {
  int pos, neg, bpos, bneg;
};

// Pressure increment of one weight (ratchet.py:248-262): -sign(z) · bucket(|z|) with
// z = RN(g / denom).  Only the two threshold comparisons depend on the quotient, so it is formed
// as g · RN(1/denom) (relative error below 2^-22) and the IEEE division is taken only when that
// estimate lies within a relative 2^-20 of a threshold.  sign(z) = sign(g) since denom > 0.
__device__ __forceinline__ int pressure_increment(float g, float denom, float rcp, int normalize,
                                                  float low, float high) {
  float mag = normalize ? fabsf(__fmul_rn(g, rcp)) : fabsf(g);
  if (normalize) {
    const float win = __fmul_rn(mag, 9.5367431640625e-07f);  // 2^-20
    if (fabsf(__fsub_rn(mag, high)) <= win || fabsf(__fsub_rn(mag, low)) <= win)
      mag = fabsf(__fdiv_rn(g, denom));
  }
  // z rounding to ±0 has sign 0 (and with low = 0 would otherwise reach bucket 1)
  if (mag == 0.0f) return 0;
  const int bucket = mag >= high ? 2 : (mag >= low ? 1 : 0);
  const int sgn = (g > 0.0f) - (g < 0.0f);
  return -sgn * bucket;
}

// One weight: the new packed byte (ratchet.py:277-294).
__device__ __forceinline__ uint8_t ratchet_one(uint8_t old, int inc, const UpdateArgs &a,
                                               Moves &m) {
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
__device__ __forceinline__ int8_t code_of(uint8_t packed, int max_code) {
  return static_cast<int8_t>(static_cast<int>(packed & 0x0F) - max_code);
}

// The whole code/pressure step of one weight as a table lookup.  Entry (old << 3 | bucket << 1
// | negative) for a packed byte `old`, a bucket in {0, 1, 2} and the gradient's sign holds what
// ratchet_one computes for the increment -sign(g)·bucket: bits 0-15 the four move counts as
// 4-bit fields (positive, negative, blocked positive, blocked negative), bits 16-23 the new
// packed byte, bits 24-31 its int8 code.  Built by each CTA from ratchet_one itself, so the
// lookup and the direct computation agree by construction.
constexpr int kUpdateLut = 256 * 8;
__device__ __forceinline__ void build_update_lut(uint32_t *lut, const UpdateArgs &a) {
  for (int e = threadIdx.x; e < kUpdateLut; e += blockDim.x) {
    const int old = e >> 3, bucket = (e >> 1) & 3, negative = e & 1;
    uint32_t v = 0;
    if (bucket <= 2) {
      Moves m = {0, 0, 0, 0};
      const uint8_t nb = ratchet_one(static_cast<uint8_t>(old), negative ? bucket : -bucket, a, m);
      v = static_cast<uint32_t>(m.pos) | (static_cast<uint32_t>(m.neg) << 4) |
          (static_cast<uint32_t>(m.bpos) << 8) | (static_cast<uint32_t>(m.bneg) << 12) |
          (static_cast<uint32_t>(nb) << 16) |
          (static_cast<uint32_t>(static_cast<uint8_t>(code_of(nb, a.max_code))) << 24);
    }
    lut[e] = v;
  }
  __syncthreads();
}
// Table index of one weight: the bucket of |z| (z = g / denom, formed as in pressure_increment)
// and the sign of g; z == ±0 moves nothing (bucket 0).
__device__ __forceinline__ uint32_t lut_index(uint32_t old, float g, float denom, float rcp,
                                              int normalize, float low, float high) {
  float mag = normalize ? fabsf(__fmul_rn(g, rcp)) : fabsf(g);
  if (normalize) {
    const float win = __fmul_rn(mag, 9.5367431640625e-07f);  // 2^-20
    if (fabsf(__fsub_rn(mag, high)) <= win || fabsf(__fsub_rn(mag, low)) <= win)
      mag = fabsf(__fdiv_rn(g, denom));
  }
  const uint32_t bucket =
      mag == 0.0f ? 0u : static_cast<uint32_t>(mag >= high) + static_cast<uint32_t>(mag >= low);
  return (old << 3) | (bucket << 1) | static_cast<uint32_t>(g < 0.0f);
}

// Per-row normaliser (ratchet.py:539-556); returns rms + eps.  Only `writer` stores rms_ema.
__device__ __forceinline__ float row_denominator(const UpdateArgs &a, int64_t row, float ms,
                                                 float ema_old, bool bad, bool writer) {
  float rms = __fsqrt_rn(ms);
  if (a.rms_ema != nullptr && !bad) {
    const float upd = ema_old == 0.0f
                          ? ms
                          : __fadd_rn(__fmul_rn(a.beta, ema_old), __fmul_rn(a.one_minus_beta, ms));
    const float ema = ms > 0.0f ? upd : ema_old;
    if (writer) a.rms_ema[row] = ema;
    rms = __fsqrt_rn(ema);
  }
  return __fadd_rn(rms, a.eps);
}

// The CTA's move counts (and, with rrs, the sum of its rows' gradient rms: RPC values) go to
// the global counters with one atomic each per CTA.
__device__ __forceinline__ void publish_moves(Moves m, int (*redi)[4], const UpdateArgs &a,
                                              const float *rrs = nullptr, int nrr = 0) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  m.pos = warp_isum(m.pos), m.neg = warp_isum(m.neg);
  m.bpos = warp_isum(m.bpos), m.bneg = warp_isum(m.bneg);
  __syncthreads();
  if (lane == 0) {
    redi[warp][0] = m.pos, redi[warp][1] = m.neg, redi[warp][2] = m.bpos, redi[warp][3] = m.bneg;
  }
  __syncthreads();
  if (threadIdx.x < 4 && a.counts != nullptr) {
    int sum = 0;
#pragma unroll
    for (int w = 0; w < CTA / 32; ++w) sum += redi[w][threadIdx.x];
    if (sum != 0) atomicAdd(a.counts + threadIdx.x, static_cast<unsigned long long>(sum));
  }
  if (threadIdx.x == 32 && rrs != nullptr && a.rms_sum != nullptr) {
    float sum = 0.0f;
    for (int r = 0; r < nrr; ++r) sum = __fadd_rn(sum, rrs[r]);
    atomicAdd(a.rms_sum, sum);
  }
}

// Eight gradient values of row `row`, chunk c: from `grad`, or (WS) summed over the split-K
// partial tiles in split order.
template <typename G, bool WS>
__device__ __forceinline__ void load_grad8(const UpdateArgs &a, const G *gr, int64_t row,
                                           int64_t c, float (&v)[8]) {
  if constexpr (WS) {
    const int64_t k0 = 8 * c;
    const int64_t tile = (row >> 7) * a.ws_tiles_n + k0 / a.ws_bn;
    const float *src = a.ws + (tile * 128 + (row & 127)) * a.ws_bn + k0 % a.ws_bn;
    ld8(src, v);
    for (int sp = 1; sp < a.ws_splits; ++sp) {
      float f[8];
      ld8(src + sp * a.ws_split_stride, f);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], f[j]);
    }
  } else {
    ld8(gr + 8 * c, v);
  }
}

template <typename G, int RT, int VPT, bool WS>
__device__ __forceinline__ void ratchet_update_body(const UpdateArgs &a, int64_t block,
                                                    const uint32_t *lut) {
  constexpr int RPC = CTA / RT, NT = CTA / RT;
  __shared__ float sm[RT == 32 ? 1 : RPC * CTA];
  __shared__ float smb[RPC];
  __shared__ float smx[RPC * 8];
  __shared__ int redi[CTA / 32][4];
  __shared__ float rrs[RPC];  // the rows' gradient rms, summed once per CTA
  // a CTA runs this once per row block: the shared arrays of the previous block are read
  // by every thread before any thread writes them again
  __syncthreads();
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t grow = block * RPC + sub;  // gradient row
  const int64_t srow = (grow < a.rows && a.row_ids != nullptr) ? a.row_ids[grow] : grow;
  const bool live = grow < a.rows && srow >= 0;
  const int64_t row = live ? srow : 0;  // state row
  const int64_t nch = a.cols / 8;
  const G *gr = static_cast<const G *>(a.grad) + (live ? grow : 0) * a.ldg;
  const uint8_t *pr = a.packed + row * a.ldp;

  float g[VPT][8];
  uint2 pk[VPT];
  bool bad = false;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    pk[i] = make_uint2(0, 0);
    if (live && c < nch) {
      load_grad8<G, WS>(a, gr, grow, c, g[i]);
      if (a.round_bf16) {
#pragma unroll
        for (int j = 0; j < 8; ++j) g[i][j] = bf16_round(g[i][j]);
      }
      if (a.grad_mul != 1.0f) {
#pragma unroll
        for (int j = 0; j < 8; ++j) g[i][j] = __fmul_rn(g[i][j], a.grad_mul);
      }
      pk[i] = *reinterpret_cast<const uint2 *>(pr + 8 * c);
#pragma unroll
      for (int j = 0; j < 8; ++j) bad |= !isfinite(g[i][j]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) g[i][j] = 0.0f;
    }
  }
  const float ema_old = (a.rms_ema != nullptr && live) ? a.rms_ema[row] : 0.0f;
  bad = row_max<RT>(bad ? 1.0f : 0.0f, smx, sub, t) > 0.0f;

  float ss[NT], gsa[NT];
#pragma unroll
  for (int k = 0; k < NT; ++k) ss[k] = 0.0f, gsa[k] = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ss[i % NT] = __fadd_rn(ss[i % NT], __fmul_rn(g[i][j], g[i][j]));
      if (a.grad_scale != nullptr) {
        const uint32_t word = j < 4 ? pk[i].x : pk[i].y;
        const float code = static_cast<float>(code_of(static_cast<uint8_t>(word >> (8 * (j & 3))),
                                                      a.max_code));
        gsa[i % NT] = __fadd_rn(gsa[i % NT], __fmul_rn(g[i][j], code));
      }
    }
  }
  const float total = row_sum<RT>(ss, sm, smb, sub, t);
  const float gsum = a.grad_scale != nullptr ? row_sum<RT>(gsa, sm, smb, sub, t) : 0.0f;
  const float ms = __fdiv_rn(total, static_cast<float>(a.cols));
  if (RT == 32) __syncwarp();
  const float denom = row_denominator(a, row, ms, ema_old, bad, live && t == 0);
  const float rcp = __frcp_rn(denom);
  if (t == 0) rrs[sub] = 0.0f;
  if (live && t == 0) {
    const float rr = __fsqrt_rn(ms);
    if (a.row_rms != nullptr) a.row_rms[row] = rr;
    rrs[sub] = rr;
    if (a.grad_scale != nullptr) a.grad_scale[row] = gsum;
    if (bad) raise_status(RT_STATUS_NONFINITE_GRADIENT);
  }

  Moves m = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (!live || c >= nch) continue;
    if (!bad) {
      // eight table lookups; the new packed and code bytes are gathered from the entries with
      // byte permutes, the move counts summed as 4-bit fields (at most 8 per chunk)
      uint32_t e[8];
      uint32_t counts = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t word = j < 4 ? pk[i].x : pk[i].y;
        const uint32_t old = (word >> (8 * (j & 3))) & 0xFFu;
        e[j] = lut[lut_index(old, g[i][j], denom, rcp, a.normalize, a.low, a.high)];
        counts += e[j];
      }
      const uint32_t t01 = __byte_perm(e[0], e[1], 0x7362), t23 = __byte_perm(e[2], e[3], 0x7362);
      const uint32_t t45 = __byte_perm(e[4], e[5], 0x7362), t67 = __byte_perm(e[6], e[7], 0x7362);
      const uint2 out = make_uint2(__byte_perm(t01, t23, 0x5410), __byte_perm(t45, t67, 0x5410));
      *reinterpret_cast<uint2 *>(a.packed + row * a.ldp + 8 * c) = out;
      if (a.code_out != nullptr)
        *reinterpret_cast<uint2 *>(a.code_out + row * a.ldc + 8 * c) =
            make_uint2(__byte_perm(t01, t23, 0x7632), __byte_perm(t45, t67, 0x7632));
      m.pos += counts & 0xF;
      m.neg += (counts >> 4) & 0xF;
      m.bpos += (counts >> 8) & 0xF;
      m.bneg += (counts >> 12) & 0xF;
    } else if (a.code_out != nullptr) {
      uint32_t cw[2] = {0, 0};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t word = j < 4 ? pk[i].x : pk[i].y;
        cw[j >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(
                          code_of(static_cast<uint8_t>(word >> (8 * (j & 3))), a.max_code)))
                      << (8 * (j & 3));
      }
      *reinterpret_cast<uint2 *>(a.code_out + row * a.ldc + 8 * c) = make_uint2(cw[0], cw[1]);
    }
  }
  publish_moves(m, redi, a, rrs, RPC);
}
// The vectorised update kernels stride a resident-sized grid over row blocks (each CTA builds
// the lookup table once and then serves many rows).
template <typename G, int RT, int VPT>
__global__ void __launch_bounds__(CTA) ratchet_update_kernel(UpdateArgs a) {
  __shared__ uint32_t lut[kUpdateLut];
  pdl_trigger();
  build_update_lut(lut, a);  // from the launch arguments only: overlaps the previous kernel
  pdl_wait();
  const int64_t blocks = (a.rows + (CTA / RT) - 1) / (CTA / RT);
  for (int64_t b = blockIdx.x; b < blocks; b += gridDim.x)
    ratchet_update_body<G, RT, VPT, false>(a, b, lut);
}
template <typename G, int RT, int VPT>
__global__ void __launch_bounds__(CTA) ratchet_update_ws_kernel(UpdateArgs a) {
  __shared__ uint32_t lut[kUpdateLut];
  pdl_trigger();
  build_update_lut(lut, a);
  pdl_wait();
  const int64_t blocks = (a.rows + (CTA / RT) - 1) / (CTA / RT);
  for (int64_t b = blockIdx.x; b < blocks; b += gridDim.x)
    ratchet_update_body<G, RT, VPT, true>(a, b, lut);
}

// Grouped update: the rows of up to kUpdateGroup layers (same row length, dtype and ratchet
// parameters) in one launch.  Layer l owns blocks [block0[l], block0[l+1]); each block runs the
// single-layer body on that layer's rows, so the arithmetic is the per-layer kernel's.
constexpr int kUpdateGroup = 64;
struct GroupLayer {
  const void *grad;
  int64_t ldg, rows;
  uint8_t *packed;
  int64_t ldp;
  int8_t *code_out;
  int64_t ldc;
  float *rms_ema;
  unsigned long long *counts;
  float *rms_sum;
  float grad_mul;
  int block0;
};
struct GroupArgs {
  UpdateArgs common;  // row length, dtype and ratchet parameters shared by the group
  int n;
  int blocks;  // total blocks of the group (block0 of a virtual layer n)
  GroupLayer L[kUpdateGroup];
};
template <typename G, int RT, int VPT>
__global__ void __launch_bounds__(CTA) ratchet_update_grouped_kernel(const __grid_constant__ GroupArgs g) {
  __shared__ uint32_t lut[kUpdateLut];
  pdl_trigger();
  build_update_lut(lut, g.common);
  pdl_wait();
  int l = 0;
  for (int b = static_cast<int>(blockIdx.x); b < g.blocks; b += static_cast<int>(gridDim.x)) {
    while (l + 1 < g.n && g.L[l + 1].block0 <= b) ++l;  // blocks only grow: resume the search
    const GroupLayer &L = g.L[l];
    UpdateArgs a = g.common;
    a.grad = L.grad, a.ldg = L.ldg, a.rows = L.rows, a.packed = L.packed, a.ldp = L.ldp;
    a.code_out = L.code_out, a.ldc = L.ldc, a.rms_ema = L.rms_ema, a.counts = L.counts;
    a.rms_sum = L.rms_sum, a.grad_mul = L.grad_mul;
    a.row_rms = nullptr, a.grad_scale = nullptr, a.ws = nullptr, a.row_ids = nullptr;
    ratchet_update_body<G, RT, VPT, false>(a, b - L.block0, lut);
  }
}

// ---- Staged update: the same results as the kernels above, from three changes.
//  * Exact bucket thresholds per row.  RN(|g| / denom) is non-decreasing in |g|, so "its bucket
//    reaches low (high)" is |g| >= T_low (T_high) for the least float T with RN(T / denom) >= low
//    (high).  T lies within a few ulps of RN(low · denom): lanes 0-15 of a warp try the 16 floats
//    from 8 below it, lanes 16-31 those around RN(high · denom), one IEEE division each, and a
//    ballot picks the first that reaches the bound.  Each weight then needs two comparisons
//    instead of a product, a window test and a possible division.  Rows where the candidates
//    leave the finite positive floats (a denominator of inf, thresholds underflowing) keep the
//    per-weight path of lut_index.  With normalize off the thresholds are low and high.  A bound
//    of 0 becomes the least positive float: z = ±0 has sign 0 and moves nothing, so bucket 1
//    starts where z becomes nonzero (at the least positive |g| when denom <= 1, where g / denom
//    >= g).
//  * Non-finite gradients: a row's sum of squares is finite unless some gradient is not finite
//    or the sum overflows; only when one of the CTA's rows has a non-finite sum are the rows
//    scanned element by element.
//  * Every thread copies its chunks of the gradient and packed rows S-1 blocks ahead into its own
//    shared-memory slots (cp.async); the move counts and rms sums go to the layer's counters once
//    per CTA and layer instead of once per block.
// Single-layer calls run as a group of one layer (row_rms, grad_scale and row_ids from common).
__device__ __forceinline__ void cp_async8(void *smem, const void *gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
// Eight table entries of one chunk -> its new packed and code bytes and the move counts.
__device__ __forceinline__ void store_update_chunk(const GroupLayer &L, int64_t row, int64_t c,
                                                   const uint32_t (&e)[8], Moves &m) {
  uint32_t counts = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) counts += e[j];
  const uint32_t t01 = __byte_perm(e[0], e[1], 0x7362), t23 = __byte_perm(e[2], e[3], 0x7362);
  const uint32_t t45 = __byte_perm(e[4], e[5], 0x7362), t67 = __byte_perm(e[6], e[7], 0x7362);
  *reinterpret_cast<uint2 *>(L.packed + row * L.ldp + 8 * c) =
      make_uint2(__byte_perm(t01, t23, 0x5410), __byte_perm(t45, t67, 0x5410));
  if (L.code_out != nullptr)
    *reinterpret_cast<uint2 *>(L.code_out + row * L.ldc + 8 * c) =
        make_uint2(__byte_perm(t01, t23, 0x7632), __byte_perm(t45, t67, 0x7632));
  m.pos += counts & 0xF;
  m.neg += (counts >> 4) & 0xF;
  m.bpos += (counts >> 8) & 0xF;
  m.bneg += (counts >> 12) & 0xF;
}
// Bucket thresholds of one row (every lane of the warp gets both); false: no exact pair found.
__device__ __forceinline__ bool bucket_thresholds(float denom, float low, float high,
                                                  int normalize, float &tlo, float &thi) {
  constexpr float kLeastPositive = 1.40129846e-45f;
  if (!normalize) {
    tlo = fmaxf(low, kLeastPositive), thi = fmaxf(high, kLeastPositive);
    return true;
  }
  const int lane = threadIdx.x & 31;
  const float lo_bound = low > 0.0f ? low : kLeastPositive;
  const float hi_bound = high > 0.0f ? high : kLeastPositive;
  const float bound = lane < 16 ? lo_bound : hi_bound;
  const float c0 = __fmul_rn(bound, denom);
  const int32_t b = __float_as_int(c0) + ((lane & 15) - 8);
  const bool in_range = c0 > 0.0f && __float_as_int(c0) >= 8 && b < 0x7F800000 &&
                        denom > 0.0f && denom < INFINITY;
  const float cand = __int_as_float(b);
  const bool reach = in_range && __fdiv_rn(cand, denom) >= bound;
  const uint32_t mask = __ballot_sync(0xffffffffu, reach);
  const uint32_t ok = __ballot_sync(0xffffffffu, in_range);
  const uint32_t lo = mask & 0xFFFFu, hi = mask >> 16;
  const int klo = __ffs(lo) - 1, khi = __ffs(hi) - 1;
  const float tl = __shfl_sync(0xffffffffu, cand, klo < 0 ? 0 : klo);
  const float th = __shfl_sync(0xffffffffu, cand, khi < 0 ? 16 : 16 + khi);
  // the candidate range must straddle each threshold: first candidate below, the rest monotone
  const bool tiny_lo = low <= 0.0f && denom > 0.0f && denom <= 1.0f;
  const bool lo_ok = tiny_lo || (klo >= 1 && lo == (0xFFFFu & ~((1u << klo) - 1u)) &&
                                 (ok & 0xFFFFu) == 0xFFFFu);
  const bool hi_ok = khi >= 1 && hi == (0xFFFFu & ~((1u << khi) - 1u)) && (ok >> 16) == 0xFFFFu;
  tlo = tiny_lo ? kLeastPositive : tl;
  thi = th;
  return lo_ok && hi_ok;
}
// Move counts and rms sum of the CTA's blocks of one layer -> its counters (whole CTA).
__device__ __forceinline__ void publish_layer(Moves m, float rr_acc, unsigned long long *counts,
                                              float *rms_sum, int (*redi)[4], float *rrs, int sub,
                                              int t, int rpc) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  m.pos = warp_isum(m.pos), m.neg = warp_isum(m.neg);
  m.bpos = warp_isum(m.bpos), m.bneg = warp_isum(m.bneg);
  __syncthreads();
  if (lane == 0) {
    redi[warp][0] = m.pos, redi[warp][1] = m.neg, redi[warp][2] = m.bpos, redi[warp][3] = m.bneg;
  }
  if (t == 0) rrs[sub] = rr_acc;
  __syncthreads();
  if (threadIdx.x < 4 && counts != nullptr) {
    int sum = 0;
#pragma unroll
    for (int w = 0; w < CTA / 32; ++w) sum += redi[w][threadIdx.x];
    if (sum != 0) atomicAdd(counts + threadIdx.x, static_cast<unsigned long long>(sum));
  }
  if (threadIdx.x == 32 && rms_sum != nullptr) {
    float sum = 0.0f;
    for (int r = 0; r < rpc; ++r) sum = __fadd_rn(sum, rrs[r]);
    if (sum != 0.0f) atomicAdd(rms_sum, sum);
  }
}

template <typename G, int RT, int VPT, int S>
__global__ void __launch_bounds__(CTA) ratchet_update_staged_kernel(const __grid_constant__ GroupArgs g) {
  constexpr int RPC = CTA / RT, NT = CTA / RT;
  constexpr int P = static_cast<int>(sizeof(G)) / 2;  // 16-byte gradient pieces per chunk
  __shared__ uint32_t lut[kUpdateLut];
  __shared__ float sm[RT == 32 ? 1 : RPC * CTA];
  __shared__ float smb[RPC];
  __shared__ float smx[RPC * 8];
  __shared__ int redi[CTA / 32][4];
  __shared__ float rrs[RPC];
  extern __shared__ uint4 stage[];  // gradient [S][VPT][P][CTA], then packed [S][VPT][CTA] (8 B)
  uint2 *pstage = reinterpret_cast<uint2 *>(stage + S * VPT * P * CTA);
  pdl_trigger();
  build_update_lut(lut, g.common);  // from the launch arguments only: overlaps the previous kernel
  pdl_wait();
  const UpdateArgs &a = g.common;
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t nch = a.cols / 8;

  int lp = 0;  // layer cursor of the copies (blocks only grow)
  auto issue = [&](int b, int st) {
    if (b < g.blocks) {
      while (lp + 1 < g.n && g.L[lp + 1].block0 <= b) ++lp;
      const GroupLayer &L = g.L[lp];
      const int64_t grow = static_cast<int64_t>(b - L.block0) * RPC + sub;
      if (grow < L.rows) {
        const int64_t srow = a.row_ids != nullptr ? __ldg(a.row_ids + grow) : grow;
        if (srow >= 0) {
          const char *gr = static_cast<const char *>(L.grad) + grow * L.ldg * static_cast<int64_t>(sizeof(G));
          const uint8_t *pr = L.packed + srow * L.ldp;
#pragma unroll
          for (int i = 0; i < VPT; ++i) {
            const int64_t c = t + static_cast<int64_t>(i) * RT;
            if (c < nch) {
#pragma unroll
              for (int p = 0; p < P; ++p)
                cp_async16(&stage[((st * VPT + i) * P + p) * CTA + threadIdx.x],
                           gr + c * (8 * static_cast<int64_t>(sizeof(G))) + 16 * p);
              cp_async8(&pstage[(st * VPT + i) * CTA + threadIdx.x], pr + 8 * c);
            }
          }
        }
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s = 0; s < S - 1; ++s) issue(static_cast<int>(blockIdx.x + s * gridDim.x), s);

  int l = 0, cur = -1;
  Moves m = {0, 0, 0, 0};
  float rr_acc = 0.0f;
  int st = 0;
  for (int b = static_cast<int>(blockIdx.x); b < g.blocks; b += static_cast<int>(gridDim.x)) {
    issue(b + (S - 1) * static_cast<int>(gridDim.x), st == 0 ? S - 1 : st - 1);
    while (l + 1 < g.n && g.L[l + 1].block0 <= b) ++l;
    if (l != cur) {  // CTA-uniform
      if (cur >= 0)
        publish_layer(m, rr_acc, g.L[cur].counts, g.L[cur].rms_sum, redi, rrs, sub, t, RPC);
      m = Moves{0, 0, 0, 0}, rr_acc = 0.0f, cur = l;
    }
    const GroupLayer &L = g.L[l];
    const int64_t grow = static_cast<int64_t>(b - L.block0) * RPC + sub;
    const int64_t srow = grow < L.rows ? (a.row_ids != nullptr ? __ldg(a.row_ids + grow) : grow) : -1;
    const bool live = srow >= 0;
    const int64_t row = live ? srow : 0;
    const float ema_old = (L.rms_ema != nullptr && live) ? L.rms_ema[row] : 0.0f;
    cp_async_wait<S - 1>();

    float gv[VPT][8];
    uint2 pk[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t c = t + static_cast<int64_t>(i) * RT;
      pk[i] = make_uint2(0, 0);
      if (live && c < nch) {
        const uint4 *slot = &stage[((st * VPT + i) * P) * CTA + threadIdx.x];
        if constexpr (sizeof(G) == 2) {
          const uint4 u = slot[0];
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            gv[i][2 * j] = __uint_as_float(w[j] << 16);
            gv[i][2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
          }
        } else {
          const float4 lo = *reinterpret_cast<const float4 *>(slot);
          const float4 hi = *reinterpret_cast<const float4 *>(slot + CTA);
          gv[i][0] = lo.x, gv[i][1] = lo.y, gv[i][2] = lo.z, gv[i][3] = lo.w;
          gv[i][4] = hi.x, gv[i][5] = hi.y, gv[i][6] = hi.z, gv[i][7] = hi.w;
          if (a.round_bf16) {
#pragma unroll
            for (int j = 0; j < 8; ++j) gv[i][j] = bf16_round(gv[i][j]);
          }
        }
        if (L.grad_mul != 1.0f) {
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const float2 r = __fmul2_rn(make_float2(gv[i][j], gv[i][j + 1]),
                                        make_float2(L.grad_mul, L.grad_mul));
            gv[i][j] = r.x, gv[i][j + 1] = r.y;
          }
        }
        pk[i] = pstage[(st * VPT + i) * CTA + threadIdx.x];
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) gv[i][j] = 0.0f;
      }
    }
    st = st == S - 1 ? 0 : st + 1;

    float ss[NT], gsa[NT];
#pragma unroll
    for (int k = 0; k < NT; ++k) ss[k] = 0.0f, gsa[k] = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float2 sq = __fmul2_rn(make_float2(gv[i][j], gv[i][j + 1]),
                                     make_float2(gv[i][j], gv[i][j + 1]));
        ss[i % NT] = __fadd_rn(ss[i % NT], sq.x);
        ss[i % NT] = __fadd_rn(ss[i % NT], sq.y);
      }
      if (a.grad_scale != nullptr) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t word = j < 4 ? pk[i].x : pk[i].y;
          const float code = static_cast<float>(
              code_of(static_cast<uint8_t>(word >> (8 * (j & 3))), a.max_code));
          gsa[i % NT] = __fadd_rn(gsa[i % NT], __fmul_rn(gv[i][j], code));
        }
      }
    }
    const float total = row_sum<RT>(ss, sm, smb, sub, t);
    const float gsum = a.grad_scale != nullptr ? row_sum<RT>(gsa, sm, smb, sub, t) : 0.0f;
    bool bad = false;
    if (__syncthreads_or(live && !isfinite(total))) {  // rare: scan the CTA's rows
      bool lb = false;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) lb |= !isfinite(gv[i][j]);
      bad = row_max<RT>(lb ? 1.0f : 0.0f, smx, sub, t) > 0.0f;
    }
    const float ms = __fdiv_rn(total, static_cast<float>(a.cols));
    UpdateArgs la = a;
    la.rms_ema = L.rms_ema;
    const float denom = row_denominator(la, row, ms, ema_old, bad, live && t == 0);
    float tlo, thi;
    const bool fast = bucket_thresholds(denom, a.low, a.high, a.normalize, tlo, thi);
    const float rcp = fast ? 0.0f : __frcp_rn(denom);
    if (live && t == 0) {
      const float rr = __fsqrt_rn(ms);
      if (a.row_rms != nullptr) a.row_rms[row] = rr;
      rr_acc = __fadd_rn(rr_acc, rr);
      if (a.grad_scale != nullptr) a.grad_scale[row] = gsum;
      if (bad) raise_status(RT_STATUS_NONFINITE_GRADIENT);
    }

    // (fast and bad are uniform over the row's warps: each variant is a loop of its own)
    if (!bad && fast) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t c = t + static_cast<int64_t>(i) * RT;
        if (!live || c >= nch) continue;
        uint32_t e[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t word = j < 4 ? pk[i].x : pk[i].y;
          const uint32_t old = __byte_perm(word, 0u, 0x4440 + (j & 3));
          const float ax = fabsf(gv[i][j]);
          uint32_t idx = (old << 3) | (__float_as_uint(gv[i][j]) >> 31);
          idx += ax >= tlo ? 2u : 0u;
          idx += ax >= thi ? 2u : 0u;
          e[j] = lut[idx];
        }
        store_update_chunk(L, row, c, e, m);
      }
    } else if (!bad) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t c = t + static_cast<int64_t>(i) * RT;
        if (!live || c >= nch) continue;
        uint32_t e[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t word = j < 4 ? pk[i].x : pk[i].y;
          const uint32_t old = __byte_perm(word, 0u, 0x4440 + (j & 3));
          e[j] = lut[lut_index(old, gv[i][j], denom, rcp, a.normalize, a.low, a.high)];
        }
        store_update_chunk(L, row, c, e, m);
      }
    }
    if (bad && L.code_out != nullptr) {  // the row stays; its code mirror is still written
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t c = t + static_cast<int64_t>(i) * RT;
        if (!live || c >= nch) continue;
        uint32_t cw[2] = {0, 0};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t word = j < 4 ? pk[i].x : pk[i].y;
          cw[j >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(
                            code_of(static_cast<uint8_t>(word >> (8 * (j & 3))), a.max_code)))
                        << (8 * (j & 3));
        }
        *reinterpret_cast<uint2 *>(L.code_out + row * L.ldc + 8 * c) = make_uint2(cw[0], cw[1]);
      }
    }
  }
  if (cur >= 0) publish_layer(m, rr_acc, g.L[cur].counts, g.L[cur].rms_sum, redi, rrs, sub, t, RPC);
  cp_async_wait<0>();
}

template <typename G, int RT, int VPT>
static void launch_update_staged(const GroupArgs &g, cudaStream_t s) {
  constexpr int P = static_cast<int>(sizeof(G)) / 2;
  constexpr int STAGE = VPT * (16 * P + 8) * CTA;  // one block's gradient and packed chunks
  constexpr int S = 49152 / STAGE < 2 ? 2 : (49152 / STAGE > 4 ? 4 : 49152 / STAGE);
  constexpr size_t smem = static_cast<size_t>(S) * STAGE;
  const unsigned resident = staged_resident<ratchet_update_staged_kernel<G, RT, VPT, S>>(smem);
  const unsigned blocks = static_cast<unsigned>(g.blocks);
  launch_k(ratchet_update_staged_kernel<G, RT, VPT, S>, blocks < resident ? blocks : resident, CTA,
           smem, s, g);
}
template <typename G>
static bool update_staged(const GroupArgs &g, const RowCfg &cfg, cudaStream_t s) {
  switch (cfg.rt * 16 + cfg.vpt) {
    case 32 * 16 + 1: launch_update_staged<G, 32, 1>(g, s); return true;
    case 32 * 16 + 2: launch_update_staged<G, 32, 2>(g, s); return true;
    case 32 * 16 + 4: launch_update_staged<G, 32, 4>(g, s); return true;
    case 128 * 16 + 1: launch_update_staged<G, 128, 1>(g, s); return true;
    case 128 * 16 + 2: launch_update_staged<G, 128, 2>(g, s); return true;
    case 128 * 16 + 4: launch_update_staged<G, 128, 4>(g, s); return true;
    case 256 * 16 + 1: launch_update_staged<G, 256, 1>(g, s); return true;
    case 256 * 16 + 2: launch_update_staged<G, 256, 2>(g, s); return true;
    case 256 * 16 + 4: launch_update_staged<G, 256, 4>(g, s); return true;
    case 256 * 16 + 8: launch_update_staged<G, 256, 8>(g, s); return true;
    default: return false;
  }
}

// Generic update: any alignment and row length, one CTA per row, same arithmetic and order.
__global__ void __launch_bounds__(CTA) ratchet_update_generic_kernel(UpdateArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sm[CTA];
  __shared__ float smb[1];
  __shared__ float smx[8];
  __shared__ int redi[CTA / 32][4];
  const int t = threadIdx.x;
  const int64_t grow = blockIdx.x;  // gradient row; the state row is row_ids[grow] if given
  const int64_t row = a.row_ids != nullptr ? a.row_ids[grow] : grow;
  if (row < 0) return;  // uniform over the CTA: before any barrier
  const int64_t nch = (a.cols + 7) / 8;
  float ss = 0.0f, gs = 0.0f;
  bool bad = false;
  for (int64_t c = t; c < nch; c += CTA)
    for (int j = 0; j < 8; ++j) {
      const int64_t k = 8 * c + j;
      if (k >= a.cols) break;
      float gv = load_elem(a.grad, a.grad_dtype, grow * a.ldg + k);
      if (a.round_bf16) gv = bf16_round(gv);
      if (a.grad_mul != 1.0f) gv = __fmul_rn(gv, a.grad_mul);
      bad |= !isfinite(gv);
      ss = __fadd_rn(ss, __fmul_rn(gv, gv));
      if (a.grad_scale != nullptr)
        gs = __fadd_rn(gs, __fmul_rn(gv, static_cast<float>(code_of(a.packed[row * a.ldp + k],
                                                                      a.max_code))));
    }
  const float ema_old = a.rms_ema != nullptr ? a.rms_ema[row] : 0.0f;
  bad = cta_max(bad ? 1.0f : 0.0f, smx) > 0.0f;
  const float total = cta_row_sum(ss, sm, smb);
  const float gsum = a.grad_scale != nullptr ? cta_row_sum(gs, sm, smb) : 0.0f;
  const float ms = __fdiv_rn(total, static_cast<float>(a.cols));
  const float denom = row_denominator(a, row, ms, ema_old, bad, t == 0);
  const float rcp = __frcp_rn(denom);
  if (t == 0) {
    const float rr = __fsqrt_rn(ms);
    if (a.row_rms != nullptr) a.row_rms[row] = rr;
    if (a.rms_sum != nullptr) atomicAdd(a.rms_sum, rr);
    if (a.grad_scale != nullptr) a.grad_scale[row] = gsum;
    if (bad) raise_status(RT_STATUS_NONFINITE_GRADIENT);
  }
  Moves m = {0, 0, 0, 0};
  for (int64_t k = t; k < a.cols; k += CTA) {
    uint8_t v = a.packed[row * a.ldp + k];
    if (!bad) {
      float gv = load_elem(a.grad, a.grad_dtype, grow * a.ldg + k);
      if (a.round_bf16) gv = bf16_round(gv);
      if (a.grad_mul != 1.0f) gv = __fmul_rn(gv, a.grad_mul);
      v = ratchet_one(v, pressure_increment(gv, denom, rcp, a.normalize, a.low, a.high), a, m);
      a.packed[row * a.ldp + k] = v;
    }
    if (a.code_out != nullptr) a.code_out[row * a.ldc + k] = code_of(v, a.max_code);
  }
  publish_moves(m, redi, a);
}

// ===========================================================================================
// Small state kernels.
// ===========================================================================================
__global__ void leak_kernel(uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols) {
  pdl_wait();
  pdl_trigger();
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
  pdl_wait();
  pdl_trigger();
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const uint8_t v = __ldg(packed + r * ldp + c);
    if (code) code[r * ldc + c] = code_of(v, max_code);
    if (pressure) pressure[r * ldpr + c] = static_cast<int8_t>(static_cast<int>(v >> 4) - 7);
  }
}

// Contiguous fast path of the unpack used to refresh the int8 code mirror (16 weights/thread).
__global__ void unpack_codes_vec_kernel(const uint4 *packed, int64_t n16, int max_code,
                                        uint4 *code) {
  pdl_wait();
  pdl_trigger();
  const uint32_t bias = 0x01010101u * static_cast<uint32_t>(max_code);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint4 v = __ldg(packed + i);
    // per byte (v & 0x0F) - max_code, as a bytewise modular subtraction
    v.x = __vsub4(v.x & 0x0F0F0F0Fu, bias);
    v.y = __vsub4(v.y & 0x0F0F0F0Fu, bias);
    v.z = __vsub4(v.z & 0x0F0F0F0Fu, bias);
    v.w = __vsub4(v.w & 0x0F0F0F0Fu, bias);
    code[i] = v;
  }
}

__global__ void validate_kernel(const uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols,
                                int max_code, const float *scale) {
  pdl_wait();
  pdl_trigger();
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
      const float sv = scale[r];
      if (!(sv > 0.0f) || !isfinite(sv)) bits |= RT_STATUS_SCALE_INVALID;
    }
  }
  bits = __reduce_or_sync(0xffffffffu, bits);
  if ((threadIdx.x & 31) == 0 && bits) raise_status(bits);
}

// out[m,k] = bf16(bf16(q) * bf16(s[m])) (ratchet.py:73-76); 8 elements per thread, 32-bit
// indexing when the tensor allows it.
template <typename I>
__global__ void dequant_vec_kernel(const int8_t *q, int64_t ldq, const float *s, __nv_bfloat16 *out,
                                   int64_t ldo, I rows, I cols8) {
  pdl_wait();
  pdl_trigger();
  const I n = rows * cols8;
  for (I i = blockIdx.x * static_cast<I>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<I>(gridDim.x) * blockDim.x) {
    const I r = i / cols8, c = (i - r * cols8) * 8;
    const float sb = bf16_round(__ldg(s + r));
    const uint2 raw = __ldg(reinterpret_cast<const uint2 *>(q + r * ldq + c));
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t word = j < 4 ? raw.x : raw.y;
      v[j] = __fmul_rn(static_cast<float>(static_cast<int8_t>(word >> (8 * (j & 3)))), sb);
    }
    st8(out + r * ldo + c, v);
  }
}
__global__ void dequant_kernel(const int8_t *q, int64_t ldq, const float *s, uint16_t *out,
                               int64_t ldo, int64_t rows, int64_t cols) {
  pdl_wait();
  pdl_trigger();
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const float sb = bf16_round(__ldg(s + r));
    out[r * ldo + c] = bf16_bits(__fmul_rn(static_cast<float>(q[r * ldq + c]), sb));
  }
}

// ===========================================================================================
// Fused producers (int8_fused.py) and their backwards (int8_backward.py).
// ===========================================================================================
// tanh-approximate GELU with the reference's operation order (int8_fused.py:70-75).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float c = 0.7978845608028654f;
  const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  const float inner = __fmul_rn(c, __fadd_rn(x, cube));
  const float th = tanhf(inner);
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, th));
}
// its derivative times the incoming gradient, stored through bf16 (int8_backward.py:66-75)
__device__ __forceinline__ float gelu_tanh_grad(float xv, float g) {
  const float c = 0.7978845608028654f;
  const float x2 = __fmul_rn(xv, xv);
  const float inner = __fmul_rn(c, __fadd_rn(xv, __fmul_rn(__fmul_rn(0.044715f, xv), x2)));
  const float th = tanhf(inner);
  const float t1 = __fmul_rn(0.5f, __fadd_rn(1.0f, th));
  const float t2 =
      __fmul_rn(__fmul_rn(__fmul_rn(__fmul_rn(0.5f, xv), __fsub_rn(1.0f, __fmul_rn(th, th))), c),
                __fadd_rn(1.0f, __fmul_rn(0.134145f, x2)));
  return bf16_round(__fmul_rn(g, __fadd_rn(t1, t2)));
}

struct ProdArgs {
  const void *x;
  int64_t ldx, rows, cols;
  const float *w;
  float eps;
  int8_t *q;
  int64_t ldq;
  float *row_scale;
  unsigned short *xdq;  // optional bf16 dequantised copy (row stride ld_dq)
  int64_t ld_dq;
};

// RMSNorm -> quant: y = (x · r) · w, r = 1 / sqrt(mean(x²) + eps) (IEEE sqrt and division).
template <typename T, int RT, int VPT>
__global__ void __launch_bounds__(CTA) rmsnorm_quant_kernel(ProdArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int RPC = CTA / RT, NT = CTA / RT;
  __shared__ float sm[RT == 32 ? 1 : RPC * CTA];
  __shared__ float smb[RPC];
  __shared__ float smx[RPC * 8];
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * RPC + sub;
  const bool live = row < a.rows;
  const int64_t nch = a.cols / 8;
  const T *xr = static_cast<const T *>(a.x) + (live ? row : 0) * a.ldx;
  float v[VPT][8];
  float ss[NT];
#pragma unroll
  for (int k = 0; k < NT; ++k) ss[k] = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (live && c < nch) {
      ld8(xr + 8 * c, v[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss[i % NT] = __fadd_rn(ss[i % NT], __fmul_rn(v[i][j], v[i][j]));
  }
  const float total = row_sum<RT>(ss, sm, smb, sub, t);
  const float var = __fdiv_rn(total, static_cast<float>(a.cols));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.eps)));
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (c < nch) {
      float wv[8];
      ld8(a.w + 8 * c, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i][j] = __fmul_rn(__fmul_rn(v[i][j], r), wv[j]);
        amax = fmaxf(amax, fabsf(v[i][j]));
      }
    }
  }
  amax = row_max<RT>(amax, smx, sub, t);
  if (!live) return;
  const float scale = row_scale_of(amax);
  const float rcp = __frcp_rn(scale);
  const float sb = bf16_round(scale);
  if (t == 0) a.row_scale[row] = scale;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (c >= nch) continue;
    quant_rn_store8(a.q + row * a.ldq + 8 * c, a.xdq == nullptr ? nullptr : a.xdq + row * a.ld_dq + 8 * c,
                    v[i], scale, rcp, sb);
  }
}

template <typename T, int RT, int VPT>
__global__ void __launch_bounds__(CTA) gelu_quant_kernel(ProdArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int RPC = CTA / RT;
  __shared__ float smx[RPC * 8];
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * RPC + sub;
  const bool live = row < a.rows;
  const int64_t nch = a.cols / 8;
  const T *xr = static_cast<const T *>(a.x) + (live ? row : 0) * a.ldx;
  float v[VPT][8];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (live && c < nch) {
      ld8(xr + 8 * c, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i][j] = gelu_tanh(v[i][j]);
        amax = fmaxf(amax, fabsf(v[i][j]));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
    }
  }
  amax = row_max<RT>(amax, smx, sub, t);
  if (!live) return;
  const float scale = row_scale_of(amax);
  const float rcp = __frcp_rn(scale);
  const float sb = bf16_round(scale);
  if (t == 0) a.row_scale[row] = scale;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (c >= nch) continue;
    quant_rn_store8(a.q + row * a.ldq + 8 * c, a.xdq == nullptr ? nullptr : a.xdq + row * a.ld_dq + 8 * c,
                    v[i], scale, rcp, sb);
  }
}

// The same producer over a persistent grid: every thread copies its chunks of the row groups S-1
// iterations ahead into its own shared-memory slots (cp.async), so the tanh-bound arithmetic of
// one row runs while the next rows' reads are in flight.  Per element the arithmetic is
// gelu_quant_kernel's (gelu_tanh, quant_rn_store8): identical results.
template <typename T, int RT, int VPT, int S>
__global__ void __launch_bounds__(CTA) gelu_quant_staged_kernel(ProdArgs a) {
  constexpr int RPC = CTA / RT;
  constexpr int P = static_cast<int>(sizeof(T)) / 2;  // 16-byte pieces per chunk
  extern __shared__ uint4 stage[];                     // [S][VPT][P][CTA] own slots
  __shared__ float smx[RPC * 8];
  pdl_wait();
  pdl_trigger();
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t nch = a.cols / 8;
  const int64_t groups = (a.rows + RPC - 1) / RPC;
  const int64_t row_bytes = a.ldx * static_cast<int64_t>(sizeof(T));
  auto issue = [&](int64_t grp, int st) {
    const int64_t row = grp * RPC + sub;
    if (grp < groups && row < a.rows) {
      const char *xr = static_cast<const char *>(a.x) + row * row_bytes;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t c = t + static_cast<int64_t>(i) * RT;
        if (c < nch) {
#pragma unroll
          for (int p = 0; p < P; ++p)
            cp_async16(&stage[((st * VPT + i) * P + p) * CTA + threadIdx.x],
                       xr + c * (8 * static_cast<int64_t>(sizeof(T))) + 16 * p);
        }
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s2 = 0; s2 < S - 1; ++s2) issue(blockIdx.x + static_cast<int64_t>(s2) * gridDim.x, s2);
  int st = 0;
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    issue(grp + static_cast<int64_t>(S - 1) * gridDim.x, st == 0 ? S - 1 : st - 1);
    cp_async_wait<S - 1>();
    const int64_t row = grp * RPC + sub;
    const bool live = row < a.rows;
    float v[VPT][8];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t c = t + static_cast<int64_t>(i) * RT;
      if (live && c < nch) {
        const uint4 *slot = &stage[((st * VPT + i) * P) * CTA + threadIdx.x];
        if constexpr (sizeof(T) == 2) {
          const uint4 u = slot[0];
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            v[i][2 * j] = __uint_as_float(w[j] << 16);
            v[i][2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
          }
        } else {
          const float4 lo = *reinterpret_cast<const float4 *>(slot);
          const float4 hi = *reinterpret_cast<const float4 *>(slot + CTA);
          v[i][0] = lo.x, v[i][1] = lo.y, v[i][2] = lo.z, v[i][3] = lo.w;
          v[i][4] = hi.x, v[i][5] = hi.y, v[i][6] = hi.z, v[i][7] = hi.w;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[i][j] = gelu_tanh(v[i][j]);
          amax = fmaxf(amax, fabsf(v[i][j]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
      }
    }
    amax = row_max<RT>(amax, smx, sub, t);  // CTA-uniform trip count: its barriers are safe
    if (live) {
      const float scale = row_scale_of(amax);
      const float rcp = __frcp_rn(scale);
      const float sb = bf16_round(scale);
      if (t == 0) a.row_scale[row] = scale;
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t c = t + static_cast<int64_t>(i) * RT;
        if (c >= nch) continue;
        quant_rn_store8(a.q + row * a.ldq + 8 * c,
                        a.xdq == nullptr ? nullptr : a.xdq + row * a.ld_dq + 8 * c, v[i], scale,
                        rcp, sb);
      }
    }
    st = st == S - 1 ? 0 : st + 1;
  }
  cp_async_wait<0>();
}

// Generic producers: one CTA per row, the row re-read from L2 between passes.
__global__ void __launch_bounds__(CTA)
    rmsnorm_quant_generic_kernel(ProdArgs a, int dtype) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sm[CTA];
  __shared__ float smb[1];
  __shared__ float smx[8];
  const int64_t row = blockIdx.x;
  const int64_t nch = (a.cols + 7) / 8;
  float ss = 0.0f;
  for (int64_t c = threadIdx.x; c < nch; c += CTA)
    for (int j = 0; j < 8; ++j) {
      const int64_t k = 8 * c + j;
      if (k >= a.cols) break;
      const float v = load_elem(a.x, dtype, row * a.ldx + k);
      ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
  const float total = cta_row_sum(ss, sm, smb);
  const float var = __fdiv_rn(total, static_cast<float>(a.cols));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.eps)));
  float amax = 0.0f;
  for (int64_t k = threadIdx.x; k < a.cols; k += CTA)
    amax = fmaxf(amax, fabsf(__fmul_rn(__fmul_rn(load_elem(a.x, dtype, row * a.ldx + k), r),
                                       __ldg(a.w + k))));
  amax = cta_max(amax, smx);
  const float scale = row_scale_of(amax);
  const float rcp = __frcp_rn(scale);
  const float sb = bf16_round(scale);
  if (threadIdx.x == 0) a.row_scale[row] = scale;
  for (int64_t k = threadIdx.x; k < a.cols; k += CTA) {
    const int8_t qv = quant_rn(
        __fmul_rn(__fmul_rn(load_elem(a.x, dtype, row * a.ldx + k), r), __ldg(a.w + k)), scale,
        rcp);
    a.q[row * a.ldq + k] = qv;
    if (a.xdq != nullptr) a.xdq[row * a.ld_dq + k] = bf16_bits(__fmul_rn(static_cast<float>(qv), sb));
  }
}

__global__ void __launch_bounds__(CTA) gelu_quant_generic_kernel(ProdArgs a, int dtype) {
  pdl_wait();
  pdl_trigger();
  __shared__ float smx[8];
  const int64_t row = blockIdx.x;
  float amax = 0.0f;
  for (int64_t k = threadIdx.x; k < a.cols; k += CTA)
    amax = fmaxf(amax, fabsf(gelu_tanh(load_elem(a.x, dtype, row * a.ldx + k))));
  amax = cta_max(amax, smx);
  const float scale = row_scale_of(amax);
  const float rcp = __frcp_rn(scale);
  const float sb = bf16_round(scale);
  if (threadIdx.x == 0) a.row_scale[row] = scale;
  for (int64_t k = threadIdx.x; k < a.cols; k += CTA) {
    const int8_t qv = quant_rn(gelu_tanh(load_elem(a.x, dtype, row * a.ldx + k)), scale, rcp);
    a.q[row * a.ldq + k] = qv;
    if (a.xdq != nullptr) a.xdq[row * a.ld_dq + k] = bf16_bits(__fmul_rn(static_cast<float>(qv), sb));
  }
}

// [B,H,T,D] heads -> rows b·T+t of H·D channels (int8_fused.py:103-131).
struct TransArgs {
  const void *x;
  int64_t batch, heads, seq, head_dim, sb, sh, ss, sd;
  int8_t *q;
  int64_t ldq;
  float *row_scale;
  unsigned short *xdq;  // optional bf16 dequantised copy (row stride ld_dq)
  int64_t ld_dq;
};
template <typename T, int RT, int VPT>
__global__ void __launch_bounds__(CTA) transpose_quant_kernel(TransArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int RPC = CTA / RT;
  __shared__ float smx[RPC * 8];
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * RPC + sub;
  const bool live = row < a.batch * a.seq;
  // row -> (b, s) and chunk -> (head, d) in 32-bit unsigned arithmetic (the launch checks that
  // rows and channels fit), a shift when head_dim is a power of two
  const uint32_t seq = static_cast<uint32_t>(a.seq), hd = static_cast<uint32_t>(a.head_dim);
  const uint32_t r32 = live ? static_cast<uint32_t>(row) : 0u;
  const uint32_t b = r32 / seq, s = r32 - b * seq;
  const bool hd_pow2 = (hd & (hd - 1)) == 0;
  const int hd_shift = __ffs(static_cast<int>(hd)) - 1;
  const int64_t nch = a.heads * a.head_dim / 8;
  const T *base = static_cast<const T *>(a.x) + b * a.sb + s * a.ss;
  float v[VPT][8];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (live && c < nch) {
      const uint32_t ch = 8u * static_cast<uint32_t>(c);
      const uint32_t h = hd_pow2 ? ch >> hd_shift : ch / hd, d = ch - h * hd;
      ld8(base + h * a.sh + d, v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
    }
  }
  amax = row_max<RT>(amax, smx, sub, t);
  if (!live) return;
  const float scale = row_scale_of(amax);
  const float rcp = __frcp_rn(scale);
  const float sb = bf16_round(scale);
  if (t == 0) a.row_scale[row] = scale;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (c >= nch) continue;
    quant_rn_store8(a.q + row * a.ldq + 8 * c, a.xdq == nullptr ? nullptr : a.xdq + row * a.ld_dq + 8 * c,
                    v[i], scale, rcp, sb);
  }
}
__global__ void __launch_bounds__(CTA) transpose_quant_generic_kernel(TransArgs a, int dtype) {
  pdl_wait();
  pdl_trigger();
  __shared__ float smx[8];
  const int64_t row = blockIdx.x;
  const int64_t b = row / a.seq, s = row % a.seq;
  const int64_t channels = a.heads * a.head_dim;
  float amax = 0.0f;
  for (int64_t c = threadIdx.x; c < channels; c += CTA) {
    const int64_t h = c / a.head_dim, d = c % a.head_dim;
    amax = fmaxf(amax, fabsf(load_elem(a.x, dtype, b * a.sb + h * a.sh + s * a.ss + d * a.sd)));
  }
  amax = cta_max(amax, smx);
  const float scale = row_scale_of(amax);
  const float rcp = __frcp_rn(scale);
  const float sbf = bf16_round(scale);
  if (threadIdx.x == 0) a.row_scale[row] = scale;
  for (int64_t c = threadIdx.x; c < channels; c += CTA) {
    const int64_t h = c / a.head_dim, d = c % a.head_dim;
    const int8_t qv =
        quant_rn(load_elem(a.x, dtype, b * a.sb + h * a.sh + s * a.ss + d * a.sd), scale, rcp);
    a.q[row * a.ldq + c] = qv;
    if (a.xdq != nullptr) a.xdq[row * a.ld_dq + c] = bf16_bits(__fmul_rn(static_cast<float>(qv), sbf));
  }
}

// RMSNorm backward (int8_backward.py:7-27): dx stored through bf16 (the reference stores the
// Triton kernel's bf16 value); dw[k] += Σ_rows (gy·x)·r accumulated with fp32 reductions.
struct RmsBwdArgs {
  const void *gy;
  const void *x;
  const float *w;
  float eps;
  int64_t rows, cols;
  void *dx;
  int dx_dtype;
  float *dw;
  const float *dx_add;  // optional fp32 gradient added to dx (the residual branch), may be dx
  QuantArgs sq;         // SRQ: stochastic-rounding quantisation of dx for the layer it feeds
  // dw != null: per-CTA partial rows of dw (vectorised kernel, [gridDim.x][cols]) or per-row
  // rsqrt values (generic kernel, [rows]); a second kernel sums them in a fixed order into dw
  float *dw_work;
};
// X: input dtype, G: incoming-gradient dtype (fp32 or bf16 each).  SRQ: dx (the output gradient
// of the ratchet layer whose output is this norm's input) is also quantised with stochastic
// rounding for that layer's int8 grad_input GEMM (a.sq: column scales, Philox key, int8 rows,
// row scales, bf16 copy), exactly as quant_rows_kernel would quantise the stored dx.
template <typename X, typename G, int RT, int VPT, bool SRQ>
__global__ void __launch_bounds__(CTA, 2) rmsnorm_bwd_kernel(RmsBwdArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int RPC = CTA / RT, NT = CTA / RT;
  __shared__ float sm[RT == 32 ? 1 : RPC * CTA];
  __shared__ float smb[RPC];
  __shared__ float smx[SRQ ? RPC * 8 : 1];
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t nch = a.cols / 8;
  const int64_t groups = (a.rows + RPC - 1) / RPC;
  float dwp[VPT][8], wv[VPT][8];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t c = t + static_cast<int64_t>(i) * RT;
    if (c < nch) {
      ld8(a.w + 8 * c, wv[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[i][j] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) dwp[i][j] = 0.0f;
  }
  // column scales are re-read per row (L1 hits) rather than held: two CTAs per SM stay resident
  const uint32_t step = SRQ ? sr_step_read(a.sq) : 0u;
  // x / cols as a multiply when cols is a power of two (then exact, the same value)
  const bool cols_pow2 = (a.cols & (a.cols - 1)) == 0;
  const float inv_cols = 1.0f / static_cast<float>(a.cols);
  // rows are visited in groups of RPC by a grid-stride loop (uniform across the CTA), so each
  // thread accumulates the weight gradient of its own columns over many rows
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t row = grp * RPC + sub;
    const bool live = row < a.rows;
    const X *xr = static_cast<const X *>(a.x) + (live ? row : 0) * a.cols;
    const G *gr = static_cast<const G *>(a.gy) + (live ? row : 0) * a.cols;
    float xv[VPT][8], gv[VPT][8], ad[VPT][8];
    float ss[NT], dot[NT];
#pragma unroll
    for (int k = 0; k < NT; ++k) ss[k] = 0.0f, dot[k] = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t c = t + static_cast<int64_t>(i) * RT;
      if (live && c < nch) {
        ld8(xr + 8 * c, xv[i]);
        ld8(gr + 8 * c, gv[i]);
        // the residual branch's gradient, requested with the row (it may alias dx: each element
        // is read before this thread stores it)
        if (a.dx_add != nullptr) ld8(a.dx_add + row * a.cols + 8 * c, ad[i]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) xv[i][j] = 0.0f, gv[i][j] = 0.0f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float dh = __fmul_rn(gv[i][j], wv[i][j]);
        ss[i % NT] = __fadd_rn(ss[i % NT], __fmul_rn(xv[i][j], xv[i][j]));
        dot[i % NT] = __fadd_rn(dot[i % NT], __fmul_rn(dh, xv[i][j]));
      }
    }
    const float total = row_sum<RT>(ss, sm, smb, sub, t);
    const float dsum = row_sum<RT>(dot, sm, smb, sub, t);
    const float var = __fdiv_rn(total, static_cast<float>(a.cols));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.eps)));
    const float dvar = __fmul_rn(__fmul_rn(dsum, -0.5f), __fmul_rn(__fmul_rn(r, r), r));
    float qv[SRQ ? VPT : 1][8];
    float amax = 0.0f;
    if (live) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t c = t + static_cast<int64_t>(i) * RT;
        if (c >= nch) continue;
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float dh = __fmul_rn(gv[i][j], wv[i][j]);
          const float num = __fmul_rn(__fmul_rn(dvar, 2.0f), xv[i][j]);
          const float q = cols_pow2 ? __fmul_rn(num, inv_cols)
                                    : __fdiv_rn(num, static_cast<float>(a.cols));
          o[j] = bf16_round(__fadd_rn(__fmul_rn(dh, r), q));
          dwp[i][j] = __fadd_rn(dwp[i][j], __fmul_rn(__fmul_rn(gv[i][j], xv[i][j]), r));
        }
        if (a.dx_add != nullptr) {  // summed as autograd sums the two branches
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = __fadd_rn(ad[i][j], o[j]);
        }
        if (a.dx_dtype == RT_F32)
          st8(static_cast<float *>(a.dx) + row * a.cols + 8 * c, o);
        else
          st8(static_cast<__nv_bfloat16 *>(a.dx) + row * a.cols + 8 * c, o);
        if constexpr (SRQ) {
          // the stored value (a bf16 dx stores the bf16-exact o unchanged)
#pragma unroll
          for (int j = 0; j < 8; ++j) qv[i][j] = o[j];
          float cs[8];
          if (a.sq.col_scale != nullptr) ld8(a.sq.col_scale + 8 * c, cs);
          sr_prepare_chunk(a.sq, row, c, qv[i], cs, amax);
        }
      }
    }
    if constexpr (SRQ) {
      amax = row_max<RT>(amax, smx, sub, t);  // CTA-uniform trip count: its barriers are safe
      if (live) sr_quant_store_row<RT, VPT>(a.sq, step, row, t, nch, qv, amax);
    }
  }
  if (a.dw != nullptr) {
    // the CTA's partial row of dw: its RPC sub-row partials summed in shared memory in sub
    // order, stored to this CTA's row of the workspace; dw_partials_reduce_kernel then adds the
    // CTA rows in index order (deterministic, unlike one atomic per column per CTA)
    float *part = a.dw_work + static_cast<int64_t>(blockIdx.x) * a.cols;
    extern __shared__ float dws[];  // [RPC][cols] when RPC > 1
    if constexpr (RPC > 1) {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t c = t + static_cast<int64_t>(i) * RT;
        if (c >= nch) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) dws[sub * a.cols + 8 * c + j] = dwp[i][j];
      }
      __syncthreads();
      for (int64_t k = threadIdx.x; k < a.cols; k += CTA) {
        float acc = dws[k];
        for (int r2 = 1; r2 < RPC; ++r2) acc = __fadd_rn(acc, dws[r2 * a.cols + k]);
        part[k] = acc;
      }
    } else {
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int64_t c = t + static_cast<int64_t>(i) * RT;
        if (c >= nch) continue;
        st8(part + 8 * c, dwp[i]);
      }
    }
  }
  if constexpr (SRQ) sr_step_arrive(a.sq, step);
}

__global__ void __launch_bounds__(CTA)
    rmsnorm_bwd_generic_kernel(RmsBwdArgs a, int gdt, int xdt) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sm[CTA];
  __shared__ float smb[1];
  const int64_t row = blockIdx.x;
  const int64_t nch = (a.cols + 7) / 8;
  float ss = 0.0f, dot = 0.0f;
  for (int64_t c = threadIdx.x; c < nch; c += CTA)
    for (int j = 0; j < 8; ++j) {
      const int64_t k = 8 * c + j;
      if (k >= a.cols) break;
      const float xv = load_elem(a.x, xdt, row * a.cols + k);
      const float dh = __fmul_rn(load_elem(a.gy, gdt, row * a.cols + k), __ldg(a.w + k));
      ss = __fadd_rn(ss, __fmul_rn(xv, xv));
      dot = __fadd_rn(dot, __fmul_rn(dh, xv));
    }
  const float total = cta_row_sum(ss, sm, smb);
  const float dsum = cta_row_sum(dot, sm, smb);
  const float var = __fdiv_rn(total, static_cast<float>(a.cols));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.eps)));
  const float dvar = __fmul_rn(__fmul_rn(dsum, -0.5f), __fmul_rn(__fmul_rn(r, r), r));
  for (int64_t k = threadIdx.x; k < a.cols; k += CTA) {
    const float xv = load_elem(a.x, xdt, row * a.cols + k);
    const float g = load_elem(a.gy, gdt, row * a.cols + k);
    const float dh = __fmul_rn(g, __ldg(a.w + k));
    const float v = __fadd_rn(__fmul_rn(dh, r), __fdiv_rn(__fmul_rn(__fmul_rn(dvar, 2.0f), xv),
                                                          static_cast<float>(a.cols)));
    float o = bf16_round(v);
    if (a.dx_add != nullptr) o = __fadd_rn(a.dx_add[row * a.cols + k], o);
    store_elem(a.dx, a.dx_dtype, row * a.cols + k, o);
  }
  if (a.dw != nullptr && threadIdx.x == 0) a.dw_work[row] = r;  // dw_rows_reduce_kernel's input
}

// dw[k] += the fixed-order sum of part[0..parts-1][k], the vectorised RMSNorm backward's per-CTA
// partial rows.  A CTA covers 32 columns with 8 lanes groups: group g sums the partials
// p = g, g + 8, g + 16, ... in order (loads issued eight at a time), then the eight group sums
// are added in g order -- the same tree on every call.
__global__ void __launch_bounds__(256)
    dw_partials_reduce_kernel(const float *__restrict__ part, int parts, int64_t cols, float *dw) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sums[8][33];
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int64_t k = blockIdx.x * 32ll + lane;
  float acc = 0.0f;
  if (k < cols) {
    int p = g;
    for (; p + 56 < parts; p += 64) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __ldg(part + static_cast<int64_t>(p + 8 * j) * cols + k);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, v[j]);
    }
    for (; p < parts; p += 8) acc = __fadd_rn(acc, __ldg(part + static_cast<int64_t>(p) * cols + k));
  }
  sums[g][lane] = acc;
  __syncthreads();
  if (g == 0 && k < cols) {
    float t = sums[0][lane];
#pragma unroll
    for (int j = 1; j < 8; ++j) t = __fadd_rn(t, sums[j][lane]);
    dw[k] = __fadd_rn(dw[k], t);
  }
}
// dw[k] += sum over rows (in order) of (gy·x)·r[row]: the generic kernel's weight gradient.
__global__ void __launch_bounds__(256)
    dw_rows_reduce_kernel(const void *gy, int gdt, const void *x, int xdt, const float *r,
                          int64_t rows, int64_t cols, float *dw) {
  pdl_wait();
  pdl_trigger();
  const int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (k >= cols) return;
  float acc = 0.0f;
  for (int64_t row = 0; row < rows; ++row)
    acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(load_elem(gy, gdt, row * cols + k),
                                             load_elem(x, xdt, row * cols + k)), r[row]));
  dw[k] = __fadd_rn(dw[k], acc);
}

template <typename T>
__global__ void gelu_bwd_vec_kernel(const T *gy, const T *x, int64_t n8, T *dx) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float xv[8], g[8], o[8];
    ld8(x + 8 * i, xv);
    ld8(gy + 8 * i, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = gelu_tanh_grad(xv[j], g[j]);
    st8(dx + 8 * i, o);
  }
}
__global__ void gelu_bwd_kernel(const void *gy, int gdt, const void *x, int xdt, int64_t n,
                                void *dx, int dxdt) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    store_elem(dx, dxdt, i, gelu_tanh_grad(load_elem(x, xdt, i), load_elem(gy, gdt, i)));
}

// tanh-GELU backward fused with the stochastic-rounding quantisation of its result, the output
// gradient of the expanding ratchet layer (int8_backward.py:53-89 followed by the layer's
// ratchet.py:117-134 quantisation): dx is written once and quantised from registers.  Rows are
// contiguous (a.sq.cols elements); grid-stride over row groups with a resident-sized grid.
struct GeluBwdQArgs {
  const void *gy;
  const void *x;
  void *dx;
  QuantArgs sq;
};
template <typename T, int RT, int VPT>
__global__ void __launch_bounds__(CTA, VPT <= 2 ? 4 : (VPT == 4 ? 2 : 1)) gelu_bwd_sr_kernel(GeluBwdQArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int RPC = CTA / RT;
  __shared__ float smx[RPC * 8];
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t nch = a.sq.cols / 8;
  const int64_t groups = (a.sq.rows + RPC - 1) / RPC;
  const uint32_t step = sr_step_read(a.sq);
  float cs[VPT][8];
  sr_load_col_scales<RT, VPT>(a.sq, t, nch, cs);
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t row = grp * RPC + sub;
    const bool live = row < a.sq.rows;
    const int64_t off = (live ? row : 0) * a.sq.cols;
    const T *xr = static_cast<const T *>(a.x) + off;
    const T *gr = static_cast<const T *>(a.gy) + off;
    T *dr = static_cast<T *>(a.dx) + off;
    float v[VPT][8];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t c = t + static_cast<int64_t>(i) * RT;
      if (live && c < nch) {
        float xv[8], g[8];
        ld8(xr + 8 * c, xv);
        ld8(gr + 8 * c, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = gelu_tanh_grad(xv[j], g[j]);
        st8(dr + 8 * c, v[i]);  // bf16-exact values: a bf16 dx stores them unchanged
        sr_prepare_chunk(a.sq, row, c, v[i], cs[i], amax);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
      }
    }
    amax = row_max<RT>(amax, smx, sub, t);
    if (live) sr_quant_store_row<RT, VPT>(a.sq, step, row, t, nch, v, amax);
  }
  sr_step_arrive(a.sq, step);
}

// Gradients of the three [B, H, T, D] head views of a fused q|k|v projection output gathered
// into its [B·T, 3·H·D] output gradient (the concatenation autograd forms for `.chunk(3)` of
// model.py:61-70 and the head transposes), fused with the stochastic-rounding quantisation of
// that gradient for the projection's int8 grad_input GEMM.  Part p of a row holds the channels
// h·D + d of source p; every source needs unit stride along D and D % 8 == 0.
struct HeadsQArgs {
  const void *src[3];
  int64_t sb[3], sh[3], ss[3];
  int64_t seq, head_dim, width;  // width = H·D channels per part
  void *out;
  int64_t ldo;
  QuantArgs sq;  // rows = B·T, cols = 3·width
};
template <typename T, int RT, int VPT>
__global__ void __launch_bounds__(CTA, VPT <= 2 ? 4 : (VPT == 4 ? 2 : 1)) heads3_sr_kernel(HeadsQArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int RPC = CTA / RT;
  __shared__ float smx[RPC * 8];
  const int sub = threadIdx.x / RT, t = threadIdx.x % RT;
  const int64_t nch = a.sq.cols / 8;
  const int64_t groups = (a.sq.rows + RPC - 1) / RPC;
  const uint32_t step = sr_step_read(a.sq);
  float cs[VPT][8];
  sr_load_col_scales<RT, VPT>(a.sq, t, nch, cs);
  // this thread's chunks sit at the same (part, head, d) in every row
  int part[VPT];
  int64_t coff[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t ch = 8 * (t + static_cast<int64_t>(i) * RT);
    const int64_t p = ch / a.width, w = ch - p * a.width;
    const int64_t h = w / a.head_dim, d = w - h * a.head_dim;
    part[i] = static_cast<int>(p < 3 ? p : 2);
    coff[i] = h * (p == 0 ? a.sh[0] : (p == 1 ? a.sh[1] : a.sh[2])) + d;
  }
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x) {
    const int64_t row = grp * RPC + sub;
    const bool live = row < a.sq.rows;
    const uint32_t r32 = live ? static_cast<uint32_t>(row) : 0u;  // rows < 2^31 (launch)
    const int64_t b = r32 / static_cast<uint32_t>(a.seq), s = r32 - b * a.seq;
    const T *base0 = static_cast<const T *>(a.src[0]) + b * a.sb[0] + s * a.ss[0];
    const T *base1 = static_cast<const T *>(a.src[1]) + b * a.sb[1] + s * a.ss[1];
    const T *base2 = static_cast<const T *>(a.src[2]) + b * a.sb[2] + s * a.ss[2];
    T *orow = static_cast<T *>(a.out) + (live ? row : 0) * a.ldo;
    float v[VPT][8];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int64_t c = t + static_cast<int64_t>(i) * RT;
      if (live && c < nch) {
        const T *src = part[i] == 0 ? base0 : (part[i] == 1 ? base1 : base2);
        ld8(src + coff[i], v[i]);
        st8(orow + 8 * c, v[i]);
        sr_prepare_chunk(a.sq, row, c, v[i], cs[i], amax);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
      }
    }
    amax = row_max<RT>(amax, smx, sub, t);
    if (live) sr_quant_store_row<RT, VPT>(a.sq, step, row, t, nch, v, amax);
  }
  sr_step_arrive(a.sq, step);
}

static inline unsigned grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  if (b > 148 * 32) b = 148 * 32;
  if (b < 1) b = 1;
  return static_cast<unsigned>(b);
}


// ===========================================================================================
// Ratchet embedding (ratchet.py:688-749) and uint16 token windows (data.py:238-287).
// ===========================================================================================
// out[t, :] = float(code(packed[tok[t], :])) * scale[tok[t]] -- the reference's
// F.embedding(tokens, code.float() * scale[:, None]) without the [rows, dim] effective weight.
// A warp per token; 8 codes per 8-byte load when the rows allow it.  Tokens outside [0, rows)
// give zero rows and set RT_STATUS_INDEX_RANGE.
__global__ void __launch_bounds__(256)
    embedding_forward_kernel(const uint8_t *packed, int64_t ldp, const float *scale, int max_code,
                             const int64_t *tokens, int64_t n_tok, int64_t rows, int64_t dim,
                             float *out, int64_t ldo, int vec) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * 8ll + (threadIdx.x >> 5);
  if (t >= n_tok) return;
  const int64_t tok = tokens[t];
  float *o = out + t * ldo;
  if (tok < 0 || tok >= rows) {
    for (int64_t k = lane; k < dim; k += 32) o[k] = 0.0f;
    if (lane == 0) raise_status(RT_STATUS_INDEX_RANGE);
    return;
  }
  const float sc = __ldg(scale + tok);
  const uint8_t *pr = packed + tok * ldp;
  if (vec) {
    for (int64_t c = lane; c < dim / 8; c += 32) {
      const uint2 w = __ldg(reinterpret_cast<const uint2 *>(pr + 8 * c));
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t word = j < 4 ? w.x : w.y;
        v[j] = __fmul_rn(static_cast<float>(code_of(static_cast<uint8_t>(word >> (8 * (j & 3))),
                                                    max_code)),
                         sc);
      }
      st8(o + 8 * c, v);
    }
  } else {
    for (int64_t k = lane; k < dim; k += 32)
      o[k] = __fmul_rn(static_cast<float>(code_of(pr[k], max_code)), sc);
  }
}

// The embedding's weight gradient, row-sparse: sorted_tokens / order are the token ids sorted
// stably and their positions (equal tokens keep position order).  The position at sorted index i that starts a
// run of equal tokens writes, into grad_rows[i], the sum of the run's gradient rows in position
// order from +0 (the order of the reference's CPU embedding backward, which adds each
// position's row into its token's row in position order), and row_ids[i] = its token; every
// other sorted index writes row_ids[i] = -1.  A warp per sorted index.
__global__ void __launch_bounds__(256)
    embedding_grad_rows_kernel(const float *grad, int64_t ldg, const int64_t *sorted_tokens,
                               const int64_t *order, int64_t n_tok, int64_t rows, int64_t dim,
                               float *grad_rows, int64_t ldr, int64_t *row_ids) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t i = blockIdx.x * 8ll + (threadIdx.x >> 5);
  if (i >= n_tok) return;
  const int64_t tok = sorted_tokens[i];
  const bool start = i == 0 || sorted_tokens[i - 1] != tok;
  if (!start || tok < 0 || tok >= rows) {
    if (lane == 0) row_ids[i] = -1;
    if (start && lane == 0) raise_status(RT_STATUS_INDEX_RANGE);
    return;
  }
  int64_t end = i + 1;
  while (end < n_tok && sorted_tokens[end] == tok) ++end;
  float *dst = grad_rows + i * ldr;
  for (int64_t k = lane; k < dim; k += 32) {
    float acc = 0.0f;
    for (int64_t j = i; j < end; ++j) acc = __fadd_rn(acc, __ldg(grad + order[j] * ldg + k));
    dst[k] = acc;
  }
  if (lane == 0) row_ids[i] = tok;
}

// inputs[b, t] = data[starts[b] + t], targets[b, t] = data[starts[b] + t + 1] (uint16 token ids
// widened to int64): the reference's batch_from_starts on a device-resident uint16 shard.
// Windows reaching past the data write zeros and set RT_STATUS_INDEX_RANGE.
__global__ void token_windows_kernel(const uint16_t *data, int64_t n, const int64_t *starts,
                                     int64_t batch, int64_t block, int64_t *inputs,
                                     int64_t *targets) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = batch * block;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t b = e / block, t = e - b * block;
    const int64_t idx = starts[b] + t;
    if (idx < 0 || idx + 1 >= n) {
      inputs[e] = 0;
      targets[e] = 0;
      raise_status(RT_STATUS_INDEX_RANGE);
      continue;
    }
    inputs[e] = data[idx];
    targets[e] = data[idx + 1];
  }
}

}  // namespace rt

// ===========================================================================================
// C ABI
// ===========================================================================================
using namespace rt;

extern "C" int rt_quantize_rows(const void *x, int x_dtype, int64_t rows, int64_t cols,
                                int64_t stride_row, int64_t stride_col, const float *col_scale,
                                int stochastic, int round_input_bf16, uint64_t seed,
                                uint32_t step, uint32_t layer, uint32_t *step_dev, int8_t *q,
                                int64_t ldq,
                                float *row_scale, void *x_bf16_out, int64_t ld_xbf16,
                                void *stream) {
  if (rows < 0 || cols < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_quantize_rows: negative shape");
  if (rows == 0) return RT_OK;
  if (x == nullptr || q == nullptr || row_scale == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_quantize_rows: null pointer");
  if (x_dtype != RT_F32 && x_dtype != RT_BF16)
    return fail(RT_ERR_DTYPE, "rt_quantize_rows: input must be float32 or bfloat16");
  if (cols == 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_quantize_rows: zero columns");
  QuantArgs a{x,          rows,   cols,     stride_row, stride_col, col_scale, stochastic,
              x_dtype == RT_F32 && round_input_bf16, seed, step, layer, step_dev, q, ldq,
              row_scale,  static_cast<unsigned short *>(x_bf16_out), ld_xbf16};
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
  if (cols % 8 == 0 && ldq % 8 == 0 && ldo % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(q) & 7) == 0 && aligned16(out)) {
    const int64_t n8 = rows * (cols / 8);
    auto *o = static_cast<__nv_bfloat16 *>(out);
    if (n8 < (int64_t(1) << 30) && rows * ldq < (int64_t(1) << 31) && rows * ldo < (int64_t(1) << 31))
      launch_k(dequant_vec_kernel<int32_t>, grid_for(n8, 256), 256, 0, s, 
          q, ldq, row_scale, o, ldo, static_cast<int32_t>(rows), static_cast<int32_t>(cols / 8));
    else
      launch_k(dequant_vec_kernel<int64_t>, grid_for(n8, 256), 256, 0, s, q, ldq, row_scale, o, ldo,
                                                                    rows, cols / 8);
  } else {
    launch_k(dequant_kernel, grid_for(rows * cols, 256), 256, 0, s, 
        q, ldq, row_scale, static_cast<uint16_t *>(out), ldo, rows, cols);
  }
  return check_launch("rt_dequant_rows_bf16");
}

static int ratchet_update_check(int64_t rows, int64_t cols, int max_code, int threshold,
                                double bucket_low, double bucket_high) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_update: shape");
  if (max_code < 1 || max_code > 7)
    return fail(RT_ERR_INVALID_ARGUMENT, "max_code must be in 1..7 (3..15 states)");
  if (threshold <= 0 || threshold > 127)
    return fail(RT_ERR_INVALID_ARGUMENT, "pressure_threshold must be in [1, 127]");
  if (!(0.0 <= bucket_low && bucket_low < bucket_high))
    return fail(RT_ERR_INVALID_ARGUMENT, "bucket thresholds must satisfy 0 <= low < high");
  return RT_OK;
}

static UpdateArgs update_args(const void *grad, int grad_dtype, int round_bf16, int64_t ldg,
                              int64_t rows, int64_t cols, uint8_t *packed, int64_t ldp,
                              int8_t *code_out, int64_t ldc, int normalize, float *rms_ema,
                              double ema_beta, int max_code, int threshold, double bucket_low,
                              double bucket_high, double eps, int64_t *counts, float *row_rms,
                              float *rms_sum, float *grad_scale) {
  UpdateArgs a{};
  a.grad = grad, a.grad_dtype = grad_dtype, a.round_bf16 = round_bf16, a.ldg = ldg;
  a.rows = rows, a.cols = cols, a.packed = packed, a.ldp = ldp, a.code_out = code_out;
  a.ldc = ldc, a.normalize = normalize, a.rms_ema = (ema_beta > 0.0) ? rms_ema : nullptr;
  a.beta = static_cast<float>(ema_beta);
  a.one_minus_beta = static_cast<float>(1.0 - ema_beta);
  a.max_code = max_code, a.threshold = threshold;
  a.low = static_cast<float>(bucket_low), a.high = static_cast<float>(bucket_high);
  a.eps = static_cast<float>(eps);
  a.counts = reinterpret_cast<unsigned long long *>(counts);
  a.row_rms = row_rms, a.rms_sum = rms_sum, a.grad_scale = grad_scale;
  a.grad_mul = 1.0f;
  a.row_ids = nullptr;
  return a;
}

// Launch of the update over a.rows rows (a.ws set: from split-K partial tiles).
static int ratchet_update_launch(const UpdateArgs &a, cudaStream_t s) {
  const int64_t rows = a.rows, cols = a.cols;
  const bool ws_ok = a.ws == nullptr || (aligned16(a.ws) && a.ws_bn % 8 == 0);
  const bool vec = cols % 8 == 0 && (a.ws != nullptr || (a.ldg % 8 == 0 && aligned16(a.grad))) &&
                   a.ldp % 8 == 0 && ws_ok && (reinterpret_cast<uintptr_t>(a.packed) & 7) == 0 &&
                   (a.code_out == nullptr ||
                    ((reinterpret_cast<uintptr_t>(a.code_out) & 7) == 0 && a.ldc % 8 == 0));
  // a warp per row up to four chunks a lane: the row's reductions are shuffles only (the
  // update's layers have few rows, so its time is the latency of one row's chain, and a CTA per
  // row pair spent it in barriers)
  RowCfg cfg = vec ? row_cfg(cols / 8, rows) : RowCfg{0, 0};
  if (cfg.rt != 0 && cols / 8 <= 32 * 4) cfg = RowCfg{32, pow2_at_least((cols / 8 + 31) / 32)};
  if (a.ws != nullptr) {
    if (cfg.rt == 0)
      return fail(RT_ERR_UNSUPPORTED, "rt_grad_weight_ratchet_update: rows need 8-element chunks");
    RT_DISPATCH_ROW(cfg, ratchet_update_ws_kernel, float, update_grid(row_grid(rows, cfg.rt), cfg.vpt), a);
  } else if (cfg.rt != 0 && staged_enabled()) {
    GroupArgs g;
    g.common = a;
    g.n = 1;
    g.blocks = static_cast<int>(row_grid(rows, cfg.rt));
    GroupLayer &d = g.L[0];
    d.grad = a.grad, d.ldg = a.ldg, d.rows = rows, d.packed = a.packed, d.ldp = a.ldp;
    d.code_out = a.code_out, d.ldc = a.ldc, d.rms_ema = a.rms_ema, d.counts = a.counts;
    d.rms_sum = a.rms_sum, d.grad_mul = a.grad_mul, d.block0 = 0;
    const bool ok = a.grad_dtype == RT_F32 ? update_staged<float>(g, cfg, s)
                                           : update_staged<__nv_bfloat16>(g, cfg, s);
    if (!ok) return fail(RT_ERR_UNSUPPORTED, "rt_ratchet_update: row configuration");
  } else if (cfg.rt != 0) {
    const unsigned grid = update_grid(row_grid(rows, cfg.rt), cfg.vpt);
    if (a.grad_dtype == RT_F32)
      RT_DISPATCH_ROW(cfg, ratchet_update_kernel, float, grid, a);
    else
      RT_DISPATCH_ROW(cfg, ratchet_update_kernel, __nv_bfloat16, grid, a);
  } else {
    launch_k(ratchet_update_generic_kernel, static_cast<unsigned>(rows), CTA, 0, s, a);
  }
  return check_launch("rt_ratchet_update");
}

extern "C" int rt_ratchet_update(const void *grad, int grad_dtype, int round_bf16, int64_t ldg,
                                 int64_t rows, int64_t cols, uint8_t *packed, int64_t ldp,
                                 int8_t *code_out, int64_t ldc, int normalize, float *rms_ema,
                                 double ema_beta, int max_code, int threshold, double bucket_low,
                                 double bucket_high, double eps, int64_t *counts, float *row_rms,
                                 float *rms_sum, float *grad_scale, void *stream) {
  if (int rc = ratchet_update_check(rows, cols, max_code, threshold, bucket_low, bucket_high))
    return rc;
  if (rows == 0) return RT_OK;
  if (grad == nullptr || packed == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_update: null pointer");
  if (grad_dtype != RT_F32 && grad_dtype != RT_BF16)
    return fail(RT_ERR_DTYPE, "rt_ratchet_update: gradient must be float32 or bfloat16");
  const UpdateArgs a = update_args(grad, grad_dtype, round_bf16, ldg, rows, cols, packed, ldp,
                                   code_out, ldc, normalize, rms_ema, ema_beta, max_code,
                                   threshold, bucket_low, bucket_high, eps, counts, row_rms,
                                   rms_sum, grad_scale);
  return ratchet_update_launch(a, as_stream(stream));
}

extern "C" int rt_ratchet_update_grouped(const rt_update_layer *layers, int n_layers,
                                         int grad_dtype, int round_bf16, int64_t cols,
                                         int normalize, double ema_beta, int max_code,
                                         int threshold, double bucket_low, double bucket_high,
                                         double eps, void *stream) {
  if (n_layers < 0 || (n_layers > 0 && layers == nullptr))
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_update_grouped: layer list");
  if (int rc = ratchet_update_check(0, cols, max_code, threshold, bucket_low, bucket_high))
    return rc;
  if (grad_dtype != RT_F32 && grad_dtype != RT_BF16)
    return fail(RT_ERR_DTYPE, "rt_ratchet_update_grouped: gradient must be float32 or bfloat16");
  cudaStream_t s = as_stream(stream);
  const size_t es = grad_dtype == RT_F32 ? 4 : 2;
  UpdateArgs common = update_args(nullptr, grad_dtype, round_bf16, 0, 0, cols, nullptr, 0, nullptr,
                                  0, normalize, nullptr, ema_beta, max_code, threshold, bucket_low,
                                  bucket_high, eps, nullptr, nullptr, nullptr, nullptr);
  // every layer must take the vectorised path (8-element chunks, 16-byte gradient rows, 8-byte
  // packed and code rows); otherwise the layers run one launch each
  bool vec = cols % 8 == 0 && cols / 8 <= 256 * 8;
  for (int i = 0; i < n_layers && vec; ++i) {
    const rt_update_layer &L = layers[i];
    if (L.rows < 0 || L.rows > INT32_MAX / 2)
      return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_update_grouped: layer %d rows", i);
    if (L.rows > 0 && (L.grad == nullptr || L.packed == nullptr))
      return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_update_grouped: layer %d null pointer", i);
    vec = vec && (L.rows == 0 || (aligned16(L.grad) && (L.ldg * es) % 16 == 0 &&
                                  (reinterpret_cast<uintptr_t>(L.packed) & 7) == 0 &&
                                  L.ldp % 8 == 0 &&
                                  (L.code_out == nullptr ||
                                   ((reinterpret_cast<uintptr_t>(L.code_out) & 7) == 0 &&
                                    L.ldc % 8 == 0))));
  }
  if (!vec) {
    for (int i = 0; i < n_layers; ++i) {
      const rt_update_layer &L = layers[i];
      if (L.rows == 0) continue;
      UpdateArgs a = common;
      a.grad = L.grad, a.ldg = L.ldg, a.rows = L.rows, a.packed = L.packed, a.ldp = L.ldp;
      a.code_out = L.code_out, a.ldc = L.ldc;
      a.rms_ema = ema_beta > 0.0 ? L.rms_ema : nullptr;
      a.counts = reinterpret_cast<unsigned long long *>(L.counts);
      a.rms_sum = L.rms_sum, a.grad_mul = L.grad_mul;
      if (int rc = ratchet_update_launch(a, s)) return rc;
    }
    return RT_OK;
  }
  // one configuration for the whole group: a warp per row up to four chunks a lane (as the
  // single-layer launch), else the row configuration of the group's total row count
  int64_t total_rows = 0;
  for (int i = 0; i < n_layers; ++i) total_rows += layers[i].rows;
  RowCfg cfg = row_cfg(cols / 8, total_rows);
  if (cols / 8 <= 32 * 4) cfg = RowCfg{32, pow2_at_least((cols / 8 + 31) / 32)};
  const int rpc = CTA / cfg.rt;
  for (int first = 0; first < n_layers;) {
    GroupArgs g;
    g.common = common;
    g.n = 0;
    int blocks = 0;
    for (; first < n_layers && g.n < kUpdateGroup; ++first) {
      const rt_update_layer &L = layers[first];
      if (L.rows == 0) continue;
      GroupLayer &d = g.L[g.n++];
      d.grad = L.grad, d.ldg = L.ldg, d.rows = L.rows, d.packed = L.packed, d.ldp = L.ldp;
      d.code_out = L.code_out, d.ldc = L.ldc;
      d.rms_ema = ema_beta > 0.0 ? L.rms_ema : nullptr;
      d.counts = reinterpret_cast<unsigned long long *>(L.counts);
      d.rms_sum = L.rms_sum, d.grad_mul = L.grad_mul;
      d.block0 = blocks;
      blocks += static_cast<int>((L.rows + rpc - 1) / rpc);
    }
    g.blocks = blocks;
    if (g.n == 0) continue;
    if (staged_enabled()) {
      const bool ok = grad_dtype == RT_F32 ? update_staged<float>(g, cfg, s)
                                           : update_staged<__nv_bfloat16>(g, cfg, s);
      if (!ok) return fail(RT_ERR_UNSUPPORTED, "rt_ratchet_update_grouped: row configuration");
      if (int rc = check_launch("rt_ratchet_update_grouped")) return rc;
      continue;
    }
    const unsigned grid = update_grid(static_cast<unsigned>(blocks), cfg.vpt);
    if (grad_dtype == RT_F32)
      RT_DISPATCH_ROW(cfg, ratchet_update_grouped_kernel, float, grid, g);
    else
      RT_DISPATCH_ROW(cfg, ratchet_update_grouped_kernel, __nv_bfloat16, grid, g);
    if (int rc = check_launch("rt_ratchet_update_grouped")) return rc;
  }
  return RT_OK;
}

extern "C" int rt_ratchet_leak(uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols,
                               int max_code, void *stream) {
  (void)max_code;
  if (rows < 0 || cols < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_leak: shape");
  if (rows * cols == 0) return RT_OK;
  launch_k(leak_kernel, grid_for(rows * cols, 256), 256, 0, as_stream(stream), packed, ldp, rows, cols);
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
    launch_k(unpack_codes_vec_kernel, grid_for(n / 16, 256), 256, 0, s, 
        reinterpret_cast<const uint4 *>(packed), n / 16, max_code, reinterpret_cast<uint4 *>(code));
  } else {
    launch_k(unpack_kernel, grid_for(n, 256), 256, 0, s, packed, ldp, rows, cols, max_code, code, ldc,
                                                   pressure, ldpr);
  }
  return check_launch("rt_unpack_code_pressure");
}

extern "C" int rt_ratchet_validate(const uint8_t *packed, int64_t ldp, int64_t rows, int64_t cols,
                                   int max_code, const float *scale, void *stream) {
  if (rows < 0 || cols < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_ratchet_validate: shape");
  if (rows * cols == 0) return RT_OK;
  launch_k(validate_kernel, grid_for(rows * cols, 256), 256, 0, as_stream(stream), packed, ldp, rows,
                                                                             cols, max_code, scale);
  return check_launch("rt_ratchet_validate");
}

extern "C" int rt_rmsnorm_quantize(const void *x, int x_dtype, int64_t ldx, const float *weight,
                                   double eps, int64_t rows, int64_t cols, int8_t *q, int64_t ldq,
                                   float *row_scale, void *dq_out, int64_t ld_dq, void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_rmsnorm_quantize: shape");
  if (x_dtype != RT_F32 && x_dtype != RT_BF16) return fail(RT_ERR_DTYPE, "rt_rmsnorm_quantize: dtype");
  if (rows == 0) return RT_OK;
  cudaStream_t s = as_stream(stream);
  ProdArgs a{x, ldx, rows, cols, weight, static_cast<float>(eps), q, ldq, row_scale,
             static_cast<unsigned short *>(dq_out), ld_dq};
  const size_t es = x_dtype == RT_F32 ? 4 : 2;
  const bool vec = cols % 8 == 0 && aligned16(x) && (ldx * es) % 16 == 0 && aligned16(weight) &&
                   (reinterpret_cast<uintptr_t>(q) & 7) == 0 && ldq % 8 == 0 &&
                   (dq_out == nullptr || (aligned16(dq_out) && ld_dq % 8 == 0));
  const RowCfg cfg = vec ? row_cfg(cols / 8) : RowCfg{0, 0};
  if (cfg.rt != 0) {
    if (x_dtype == RT_F32)
      RT_DISPATCH_ROW(cfg, rmsnorm_quant_kernel, float, row_grid(rows, cfg.rt), a);
    else
      RT_DISPATCH_ROW(cfg, rmsnorm_quant_kernel, __nv_bfloat16, row_grid(rows, cfg.rt), a);
  } else {
    launch_k(rmsnorm_quant_generic_kernel, static_cast<unsigned>(rows), CTA, 0, s, a, x_dtype);
  }
  return check_launch("rt_rmsnorm_quantize");
}

template <typename T, int RT, int VPT>
static void launch_gelu_quant_staged(const ProdArgs &a, cudaStream_t s) {
  constexpr int P = static_cast<int>(sizeof(T)) / 2;
  constexpr int S = VPT * P <= 2 ? 6 : 3;  // 24-48 KB of stages per CTA
  constexpr size_t smem = static_cast<size_t>(S) * VPT * P * CTA * 16;
  const unsigned resident = staged_resident<gelu_quant_staged_kernel<T, RT, VPT, S>>(smem);
  const unsigned groups = row_grid(a.rows, RT);
  launch_k(gelu_quant_staged_kernel<T, RT, VPT, S>, groups < resident ? groups : resident, CTA,
           smem, s, a);
}
// The staged producer takes the wide rows (four chunks a thread: 8192 bf16 values and up),
// where it measured 3 % faster; at 2048-wide rows the one-row-group-per-CTA kernel was as fast.
template <typename T>
static bool gelu_quant_staged(const ProdArgs &a, const RowCfg &cfg, cudaStream_t s) {
  if (cfg.vpt < 4) return false;
  switch (cfg.rt * 16 + cfg.vpt * static_cast<int>(sizeof(T)) / 2) {
    case 32 * 16 + 1: launch_gelu_quant_staged<T, 32, 1>(a, s); return true;
    case 128 * 16 + 1: launch_gelu_quant_staged<T, 128, 1>(a, s); return true;
    case 256 * 16 + 1: launch_gelu_quant_staged<T, 256, 1>(a, s); return true;
    case 32 * 16 + 2: launch_gelu_quant_staged<T, 32, sizeof(T) == 2 ? 2 : 1>(a, s); return true;
    case 128 * 16 + 2: launch_gelu_quant_staged<T, 128, sizeof(T) == 2 ? 2 : 1>(a, s); return true;
    case 256 * 16 + 2: launch_gelu_quant_staged<T, 256, sizeof(T) == 2 ? 2 : 1>(a, s); return true;
    case 32 * 16 + 4: launch_gelu_quant_staged<T, 32, sizeof(T) == 2 ? 4 : 2>(a, s); return true;
    case 128 * 16 + 4: launch_gelu_quant_staged<T, 128, sizeof(T) == 2 ? 4 : 2>(a, s); return true;
    case 256 * 16 + 4: launch_gelu_quant_staged<T, 256, sizeof(T) == 2 ? 4 : 2>(a, s); return true;
    default: return false;
  }
}

extern "C" int rt_gelu_quantize(const void *x, int x_dtype, int64_t ldx, int64_t rows,
                                int64_t cols, int8_t *q, int64_t ldq, float *row_scale,
                                void *dq_out, int64_t ld_dq, void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_gelu_quantize: shape");
  if (x_dtype != RT_F32 && x_dtype != RT_BF16) return fail(RT_ERR_DTYPE, "rt_gelu_quantize: dtype");
  if (rows == 0) return RT_OK;
  cudaStream_t s = as_stream(stream);
  ProdArgs a{x, ldx, rows, cols, nullptr, 0.0f, q, ldq, row_scale,
             static_cast<unsigned short *>(dq_out), ld_dq};
  const size_t es = x_dtype == RT_F32 ? 4 : 2;
  const bool vec = cols % 8 == 0 && aligned16(x) && (ldx * es) % 16 == 0 &&
                   (reinterpret_cast<uintptr_t>(q) & 7) == 0 && ldq % 8 == 0 &&
                   (dq_out == nullptr || (aligned16(dq_out) && ld_dq % 8 == 0));
  const RowCfg cfg = vec ? row_cfg(cols / 8) : RowCfg{0, 0};
  if (cfg.rt != 0 && staged_enabled() &&
      (x_dtype == RT_F32 ? gelu_quant_staged<float>(a, cfg, s)
                         : gelu_quant_staged<__nv_bfloat16>(a, cfg, s))) {
    // launched
  } else if (cfg.rt != 0) {
    if (x_dtype == RT_F32)
      RT_DISPATCH_ROW(cfg, gelu_quant_kernel, float, row_grid(rows, cfg.rt), a);
    else
      RT_DISPATCH_ROW(cfg, gelu_quant_kernel, __nv_bfloat16, row_grid(rows, cfg.rt), a);
  } else {
    launch_k(gelu_quant_generic_kernel, static_cast<unsigned>(rows), CTA, 0, s, a, x_dtype);
  }
  return check_launch("rt_gelu_quantize");
}

extern "C" int rt_transpose_quantize(const void *x, int x_dtype, int64_t batch, int64_t heads,
                                     int64_t seq, int64_t head_dim, int64_t stride_b,
                                     int64_t stride_h, int64_t stride_s, int64_t stride_d,
                                     int8_t *q, int64_t ldq, float *row_scale, void *dq_out,
                                     int64_t ld_dq, void *stream) {
  if (batch < 0 || heads <= 0 || seq < 0 || head_dim <= 0)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_transpose_quantize: shape");
  if (x_dtype != RT_F32 && x_dtype != RT_BF16)
    return fail(RT_ERR_DTYPE, "rt_transpose_quantize: dtype");
  if (batch * seq == 0) return RT_OK;
  cudaStream_t s = as_stream(stream);
  TransArgs a{x, batch, heads, seq, head_dim, stride_b, stride_h, stride_s, stride_d, q, ldq,
              row_scale, static_cast<unsigned short *>(dq_out), ld_dq};
  const int64_t es = x_dtype == RT_F32 ? 4 : 2;
  const bool vec = stride_d == 1 && head_dim % 8 == 0 && aligned16(x) &&
                   (stride_b * es) % 16 == 0 && (stride_h * es) % 16 == 0 &&
                   (stride_s * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(q) & 7) == 0 &&
                   ldq % 8 == 0 && (dq_out == nullptr || (aligned16(dq_out) && ld_dq % 8 == 0));
  const int64_t rows = batch * seq;
  const bool fits32 = rows < (int64_t(1) << 31) && heads * head_dim < (int64_t(1) << 31);
  const RowCfg cfg = vec && fits32 ? row_cfg(heads * head_dim / 8) : RowCfg{0, 0};
  if (cfg.rt != 0) {
    if (x_dtype == RT_F32)
      RT_DISPATCH_ROW(cfg, transpose_quant_kernel, float, row_grid(rows, cfg.rt), a);
    else
      RT_DISPATCH_ROW(cfg, transpose_quant_kernel, __nv_bfloat16, row_grid(rows, cfg.rt), a);
  } else {
    launch_k(transpose_quant_generic_kernel, static_cast<unsigned>(rows), CTA, 0, s, a, x_dtype);
  }
  return check_launch("rt_transpose_quantize");
}

// Launch shape of the RMSNorm backward: cfg.rt == 0 for the generic kernel (one CTA per row).
static RowCfg rmsnorm_bwd_cfg(const RmsBwdArgs &a, bool srq) {
  const bool vec = a.cols % 8 == 0 && aligned16(a.x) && aligned16(a.gy) && aligned16(a.dx) &&
                   aligned16(a.w) && (a.dw == nullptr || aligned16(a.dw)) &&
                   (a.dx_add == nullptr || aligned16(a.dx_add)) && (!srq || sr_outputs_vec(a.sq)) &&
                   (a.dw == nullptr || aligned16(a.dw_work));
  return vec ? row_cfg_narrow(a.cols / 8) : RowCfg{0, 0};
}
static int64_t rmsnorm_bwd_grid(int64_t rows, const RowCfg &cfg) {
  if (cfg.rt == 0) return rows;
  int sms = 0;
  rt_sm_count(&sms);
  const int64_t groups = (rows + (CTA / cfg.rt) - 1) / (CTA / cfg.rt);
  const int64_t cap = static_cast<int64_t>(sms > 0 ? sms : 148) * 2;
  return groups < cap ? groups : cap;
}
// Workspace of the weight gradient: per-CTA partial rows (vectorised) or per-row rsqrt (generic);
// the larger of the two, so that it does not depend on the operands' alignment.
static int64_t rmsnorm_bwd_work_bytes(int64_t rows, int64_t cols) {
  const RowCfg cfg = row_cfg_narrow(cols / 8);
  const int64_t vec = cfg.rt == 0 || cols % 8 ? 0 : rmsnorm_bwd_grid(rows, cfg) * cols * 4;
  const int64_t gen = rows * 4;
  return vec > gen ? vec : gen;
}

static int rmsnorm_backward_launch(const RmsBwdArgs &a, int gy_dtype, int x_dtype, bool srq,
                                   const char *who, cudaStream_t s) {
  const RowCfg cfg = rmsnorm_bwd_cfg(a, srq);
  if (cfg.rt == 0) {
    if (srq) return fail(RT_ERR_UNSUPPORTED, "rt_rmsnorm_backward_sr: rows need 16-byte chunks");
    launch_k(rmsnorm_bwd_generic_kernel, static_cast<unsigned>(a.rows), CTA, 0, s, a, gy_dtype, x_dtype);
    if (int rc = check_launch(who)) return rc;
    if (a.dw != nullptr) {
      launch_k(dw_rows_reduce_kernel, static_cast<unsigned>((a.cols + 255) / 256), 256, 0, s, a.gy,
               gy_dtype, a.x, x_dtype, static_cast<const float *>(a.dw_work), a.rows, a.cols, a.dw);
      return check_launch(who);
    }
    return RT_OK;
  }
  const unsigned grid = static_cast<unsigned>(rmsnorm_bwd_grid(a.rows, cfg));
  const size_t dsm = (a.dw != nullptr && cfg.rt < CTA) ? (CTA / cfg.rt) * a.cols * sizeof(float) : 0;
  if (dsm > 48 * 1024) return fail(RT_ERR_UNSUPPORTED, "rt_rmsnorm_backward: row too long");
  const int combo = (x_dtype == RT_F32 ? 0 : 2) + (gy_dtype == RT_F32 ? 0 : 1);
#define RT_RMSB(X, G, Q)                                                                      \
  switch (cfg.rt * 16 + cfg.vpt) {                                                            \
    case 32 * 16 + 1: launch_k(rmsnorm_bwd_kernel<X, G, 32, 1, Q>, grid, CTA, dsm, s, a); break;     \
    case 32 * 16 + 2: launch_k(rmsnorm_bwd_kernel<X, G, 32, 2, Q>, grid, CTA, dsm, s, a); break;     \
    case 128 * 16 + 2: launch_k(rmsnorm_bwd_kernel<X, G, 128, 2, Q>, grid, CTA, dsm, s, a); break;   \
    default: launch_k(rmsnorm_bwd_kernel<X, G, 256, 2, Q>, grid, CTA, dsm, s, a); break;             \
  }
  if (srq) {
    switch (combo) {
      case 0: RT_RMSB(float, float, true) break;
      case 1: RT_RMSB(float, __nv_bfloat16, true) break;
      case 2: RT_RMSB(__nv_bfloat16, float, true) break;
      default: RT_RMSB(__nv_bfloat16, __nv_bfloat16, true) break;
    }
  } else {
    switch (combo) {
      case 0: RT_RMSB(float, float, false) break;
      case 1: RT_RMSB(float, __nv_bfloat16, false) break;
      case 2: RT_RMSB(__nv_bfloat16, float, false) break;
      default: RT_RMSB(__nv_bfloat16, __nv_bfloat16, false) break;
    }
  }
#undef RT_RMSB
  if (int rc = check_launch(who)) return rc;
  if (a.dw != nullptr) {
    launch_k(dw_partials_reduce_kernel, static_cast<unsigned>((a.cols + 31) / 32), 256, 0, s,
             static_cast<const float *>(a.dw_work), static_cast<int>(grid), a.cols, a.dw);
    return check_launch(who);
  }
  return RT_OK;
}

extern "C" int64_t rt_rmsnorm_backward_workspace_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return rmsnorm_bwd_work_bytes(rows, cols);
}

static int rmsnorm_dw_work_check(float *dw, float *work, int64_t work_bytes, int64_t rows,
                                 int64_t cols, const char *who) {
  if (dw != nullptr && (work == nullptr || work_bytes < rmsnorm_bwd_work_bytes(rows, cols)))
    return fail(RT_ERR_INVALID_ARGUMENT,
                "%s: the weight gradient needs a workspace of rt_rmsnorm_backward_workspace_bytes",
                who);
  return RT_OK;
}

extern "C" int rt_rmsnorm_backward(const void *grad_y, int gy_dtype, const void *x, int x_dtype,
                                   const float *weight, double eps, int64_t rows, int64_t cols,
                                   void *dx, int dx_dtype, float *dw, const float *dx_add,
                                   float *dw_work, int64_t dw_work_bytes, void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_rmsnorm_backward: shape");
  if (rows == 0) return RT_OK;
  if (dx_add != nullptr && dx_dtype != RT_F32)
    return fail(RT_ERR_DTYPE, "rt_rmsnorm_backward: an added gradient needs a float32 dx");
  if (int rc = rmsnorm_dw_work_check(dw, dw_work, dw_work_bytes, rows, cols, "rt_rmsnorm_backward"))
    return rc;
  RmsBwdArgs a{grad_y, x, weight, static_cast<float>(eps), rows, cols, dx, dx_dtype, dw, dx_add,
               QuantArgs{}, dw_work};
  return rmsnorm_backward_launch(a, gy_dtype, x_dtype, false, "rt_rmsnorm_backward",
                                 as_stream(stream));
}

extern "C" int rt_rmsnorm_backward_sr(const void *grad_y, int gy_dtype, const void *x, int x_dtype,
                                      const float *weight, double eps, int64_t rows, int64_t cols,
                                      void *dx, int dx_dtype, float *dw, const float *dx_add,
                                      const float *col_scale, int round_input_bf16, uint64_t seed,
                                      uint32_t step, uint32_t layer, uint32_t *step_dev, int8_t *q,
                                      int64_t ldq, float *row_scale, void *x_bf16_out,
                                      int64_t ld_xbf16, float *dw_work, int64_t dw_work_bytes,
                                      void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_rmsnorm_backward_sr: shape");
  if (rows == 0) return RT_OK;
  if (int rc = rmsnorm_dw_work_check(dw, dw_work, dw_work_bytes, rows, cols,
                                     "rt_rmsnorm_backward_sr"))
    return rc;
  if (dx_add != nullptr && dx_dtype != RT_F32)
    return fail(RT_ERR_DTYPE, "rt_rmsnorm_backward_sr: an added gradient needs a float32 dx");
  if (q == nullptr || row_scale == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_rmsnorm_backward_sr: null pointer");
  QuantArgs sq{dx, rows, cols, cols, 1, col_scale, 1,
               dx_dtype == RT_F32 && round_input_bf16, seed, step, layer, step_dev, q, ldq,
               row_scale, static_cast<unsigned short *>(x_bf16_out), ld_xbf16};
  RmsBwdArgs a{grad_y, x, weight, static_cast<float>(eps), rows, cols, dx, dx_dtype, dw, dx_add, sq,
               dw_work};
  return rmsnorm_backward_launch(a, gy_dtype, x_dtype, true, "rt_rmsnorm_backward_sr",
                                 as_stream(stream));
}

extern "C" int rt_gelu_backward(const void *grad_y, int gy_dtype, const void *x, int x_dtype,
                                int64_t rows, int64_t cols, void *dx, int dx_dtype, void *stream) {
  if (rows < 0 || cols < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_gelu_backward: shape");
  const int64_t n = rows * cols;
  if (n == 0) return RT_OK;
  cudaStream_t s = as_stream(stream);
  if (gy_dtype == x_dtype && dx_dtype == x_dtype && n % 8 == 0 && aligned16(grad_y) &&
      aligned16(x) && aligned16(dx)) {
    if (x_dtype == RT_F32)
      launch_k(gelu_bwd_vec_kernel<float>, grid_for(n / 8, 256), 256, 0, s, 
          static_cast<const float *>(grad_y), static_cast<const float *>(x), n / 8,
          static_cast<float *>(dx));
    else
      launch_k(gelu_bwd_vec_kernel<__nv_bfloat16>, grid_for(n / 8, 256), 256, 0, s, 
          static_cast<const __nv_bfloat16 *>(grad_y), static_cast<const __nv_bfloat16 *>(x), n / 8,
          static_cast<__nv_bfloat16 *>(dx));
  } else {
    launch_k(gelu_bwd_kernel, grid_for(n, 256), 256, 0, s, grad_y, gy_dtype, x, x_dtype, n, dx, dx_dtype);
  }
  return check_launch("rt_gelu_backward");
}

extern "C" int rt_gelu_backward_sr(const void *grad_y, const void *x, int dtype, int64_t rows,
                                   int64_t cols, void *dx, const float *col_scale, uint64_t seed,
                                   uint32_t step, uint32_t layer, uint32_t *step_dev, int8_t *q,
                                   int64_t ldq, float *row_scale, void *x_bf16_out,
                                   int64_t ld_xbf16, void *stream) {
  if (rows < 0 || cols <= 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_gelu_backward_sr: shape");
  if (dtype != RT_F32 && dtype != RT_BF16) return fail(RT_ERR_DTYPE, "rt_gelu_backward_sr: dtype");
  if (rows == 0) return RT_OK;
  if (grad_y == nullptr || x == nullptr || dx == nullptr || q == nullptr || row_scale == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_gelu_backward_sr: null pointer");
  QuantArgs sq{dx, rows, cols, cols, 1, col_scale, 1, 0, seed, step, layer, step_dev, q, ldq,
               row_scale, static_cast<unsigned short *>(x_bf16_out), ld_xbf16};
  GeluBwdQArgs a{grad_y, x, dx, sq};
  const size_t es = dtype == RT_F32 ? 4 : 2;
  const bool vec = cols % 8 == 0 && aligned16(grad_y) && aligned16(x) && aligned16(dx) &&
                   (cols * es) % 16 == 0 && sr_outputs_vec(sq);
  const RowCfg cfg = vec ? row_cfg(cols / 8, rows) : RowCfg{0, 0};
  if (cfg.rt == 0) return fail(RT_ERR_UNSUPPORTED, "rt_gelu_backward_sr: rows need 16-byte chunks");
  int sms = 0;
  if (int rc = rt_sm_count(&sms)) return rc;
  const unsigned resident = static_cast<unsigned>(sms) * resident_ctas(cfg.vpt);
  const unsigned groups = row_grid(rows, cfg.rt);
  const unsigned grid = groups < resident ? groups : resident;
  cudaStream_t s = as_stream(stream);
  if (dtype == RT_F32)
    RT_DISPATCH_ROW(cfg, gelu_bwd_sr_kernel, float, grid, a);
  else
    RT_DISPATCH_ROW(cfg, gelu_bwd_sr_kernel, __nv_bfloat16, grid, a);
  return check_launch("rt_gelu_backward_sr");
}

extern "C" int rt_heads_gather_sr(const void *const *src, const int64_t *strides, int dtype,
                                  int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                                  void *out, int64_t ldo, const float *col_scale, uint64_t seed,
                                  uint32_t step, uint32_t layer, uint32_t *step_dev, int8_t *q,
                                  int64_t ldq, float *row_scale, void *x_bf16_out,
                                  int64_t ld_xbf16, void *stream) {
  if (batch < 0 || seq < 0 || heads <= 0 || head_dim <= 0)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_heads_gather_sr: shape");
  if (dtype != RT_F32 && dtype != RT_BF16) return fail(RT_ERR_DTYPE, "rt_heads_gather_sr: dtype");
  const int64_t rows = batch * seq;
  if (rows == 0) return RT_OK;
  if (src == nullptr || strides == nullptr || out == nullptr || q == nullptr ||
      row_scale == nullptr || src[0] == nullptr || src[1] == nullptr || src[2] == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_heads_gather_sr: null pointer");
  const int64_t width = heads * head_dim, cols = 3 * width;
  QuantArgs sq{out, rows, cols, ldo, 1, col_scale, 1, 0, seed, step, layer, step_dev, q, ldq,
               row_scale, static_cast<unsigned short *>(x_bf16_out), ld_xbf16};
  HeadsQArgs a;
  const int64_t es = dtype == RT_F32 ? 4 : 2;
  bool vec = head_dim % 8 == 0 && aligned16(out) && (ldo * es) % 16 == 0 && sr_outputs_vec(sq);
  for (int p = 0; p < 3; ++p) {
    a.src[p] = src[p];
    a.sb[p] = strides[4 * p], a.sh[p] = strides[4 * p + 1], a.ss[p] = strides[4 * p + 2];
    vec = vec && strides[4 * p + 3] == 1 && aligned16(src[p]) && (a.sb[p] * es) % 16 == 0 &&
          (a.sh[p] * es) % 16 == 0 && (a.ss[p] * es) % 16 == 0;
  }
  a.seq = seq, a.head_dim = head_dim, a.width = width, a.out = out, a.ldo = ldo, a.sq = sq;
  const RowCfg cfg = vec && rows < (int64_t(1) << 31) ? row_cfg(cols / 8, rows) : RowCfg{0, 0};
  if (cfg.rt == 0) return fail(RT_ERR_UNSUPPORTED, "rt_heads_gather_sr: heads need 16-byte chunks");
  int sms = 0;
  if (int rc = rt_sm_count(&sms)) return rc;
  const unsigned resident = static_cast<unsigned>(sms) * resident_ctas(cfg.vpt);
  const unsigned groups = row_grid(rows, cfg.rt);
  const unsigned grid = groups < resident ? groups : resident;
  cudaStream_t s = as_stream(stream);
  if (dtype == RT_F32)
    RT_DISPATCH_ROW(cfg, heads3_sr_kernel, float, grid, a);
  else
    RT_DISPATCH_ROW(cfg, heads3_sr_kernel, __nv_bfloat16, grid, a);
  return check_launch("rt_heads_gather_sr");
}

extern "C" int rt_embedding_forward(const uint8_t *packed, int64_t ldp, const float *scale,
                                    int max_code, const int64_t *tokens, int64_t n_tok,
                                    int64_t rows, int64_t dim, float *out, int64_t ldo,
                                    void *stream) {
  if (n_tok < 0 || rows <= 0 || dim <= 0)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_embedding_forward: shape");
  if (n_tok == 0) return RT_OK;
  if (packed == nullptr || scale == nullptr || tokens == nullptr || out == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_embedding_forward: null pointer");
  const int vec = dim % 8 == 0 && ldp % 8 == 0 && (reinterpret_cast<uintptr_t>(packed) & 7) == 0 &&
                  aligned16(out) && ldo % 4 == 0;
  launch_k(embedding_forward_kernel, static_cast<unsigned>((n_tok + 7) / 8), 256, 0,
           as_stream(stream), packed, ldp, scale, max_code, tokens, n_tok, rows, dim, out, ldo,
           vec);
  return check_launch("rt_embedding_forward");
}

extern "C" int64_t rt_embedding_update_workspace_bytes(int64_t n_tok, int64_t dim) {
  if (n_tok <= 0 || dim <= 0) return 0;
  const int64_t grads = ((n_tok * dim * 4 + 255) / 256) * 256;
  return grads + n_tok * 8;
}

extern "C" int rt_embedding_ratchet_update(
    const float *grad, int64_t ldg, const int64_t *sorted_tokens, const int64_t *order,
    int64_t n_tok, int64_t rows, int64_t dim, void *workspace, int64_t workspace_bytes,
    uint8_t *packed, int64_t ldp, int8_t *code_out, int64_t ldc, float *rms_ema, double ema_beta,
    int max_code, int threshold, double bucket_low, double bucket_high, double eps,
    int64_t *counts, float *rms_sum, void *stream) {
  if (int rc = ratchet_update_check(rows, dim, max_code, threshold, bucket_low, bucket_high))
    return rc;
  if (n_tok < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_embedding_ratchet_update: shape");
  if (n_tok == 0) return RT_OK;
  if (grad == nullptr || sorted_tokens == nullptr || order == nullptr || packed == nullptr ||
      workspace == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_embedding_ratchet_update: null pointer");
  if (workspace_bytes < rt_embedding_update_workspace_bytes(n_tok, dim) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(RT_ERR_INVALID_ARGUMENT,
                "rt_embedding_ratchet_update: workspace of rt_embedding_update_workspace_bytes, "
                "256-byte aligned");
  cudaStream_t s = as_stream(stream);
  float *grad_rows = static_cast<float *>(workspace);
  int64_t *row_ids = reinterpret_cast<int64_t *>(
      static_cast<uint8_t *>(workspace) + ((n_tok * dim * 4 + 255) / 256) * 256);
  launch_k(embedding_grad_rows_kernel, static_cast<unsigned>((n_tok + 7) / 8), 256, 0, s, grad,
           ldg, sorted_tokens, order, n_tok, rows, dim, grad_rows, dim, row_ids);
  if (int rc = check_launch("rt_embedding_ratchet_update")) return rc;
  // the update over the run-start rows: row r of grad_rows updates state row row_ids[r]
  UpdateArgs a = update_args(grad_rows, RT_F32, 0, dim, n_tok, dim, packed, ldp, code_out, ldc, 1,
                             rms_ema, ema_beta, max_code, threshold, bucket_low, bucket_high, eps,
                             counts, nullptr, rms_sum, nullptr);
  a.row_ids = row_ids;
  return ratchet_update_launch(a, s);
}

extern "C" int rt_token_windows(const uint16_t *data, int64_t n, const int64_t *starts,
                                int64_t batch, int64_t block, int64_t *inputs, int64_t *targets,
                                void *stream) {
  if (n < 0 || batch < 0 || block <= 0)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_token_windows: shape");
  if (batch == 0) return RT_OK;
  if (data == nullptr || starts == nullptr || inputs == nullptr || targets == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_token_windows: null pointer");
  launch_k(token_windows_kernel, grid_for(batch * block, 256), 256, 0, as_stream(stream), data, n,
           starts, batch, block, inputs, targets);
  return check_launch("rt_token_windows");
}
