// rt_gemm.cuh — tcgen05 GEMMs for sm_100a.
//
//   int8  (kind::i8, s32 accumulate in TMEM):  forward  out = q · codeᵀ       (K-major × K-major)
//                                              grad_in  out = g_q · code       (K-major × MN-major)
//   bf16  (kind::f16, f32 accumulate in TMEM): grad_W   gw  = g_bf16ᵀ · x̂      (MN-major × MN-major)
//
// One persistent, warp-specialised kernel per configuration:
//   warp 0      TMA producer (one elected thread): 128-byte-swizzled tiles into a STAGES-deep ring
//   warp 1      TMEM allocator + MMA issuer (one thread): 4 tcgen05.mma per stage, commit frees the
//               stage, a final commit hands the accumulator to the epilogue
//   warps 2..5  epilogue: tcgen05.ld 32x32b → fp32 → dequant/round → 128-byte-swizzled staging
//               in shared memory → TMA stores (plain lane-per-row stores when the output rows
//               are not 16-byte aligned or it accumulates), running on one TMEM accumulator
//               while the MMA fills the other (2 × BN columns).
// Tiles are BM=128 rows × BN columns; each stage covers 128 bytes of K (128 int8 or 64 bf16).
// Every CTA loads its own tiles (no clusters, no shared-tile loads between CTAs).
#pragma once

#include <cstring>
#include <mutex>

#include "rt_common.cuh"

namespace rt {

// EPI_SPLIT: split-K partial tiles (fp32) go to a workspace by TMA store; a second kernel sums
// them in split order 0..S-1 into the output — deterministic, and no CTA ever waits for another.
enum EpiMode : int { EPI_SCALED = 0, EPI_SPLIT = 1, EPI_F32_STORE = 2, EPI_BF16_STORE = 3 };

struct GemmArgs {
  int M, N, K;  // out is M × N, contraction over K
  int tiles_m, tiles_n, splits, kblocks;
  const float *a_scale;  // EPI_SCALED: per-row scale (M)
  const float *b_scale;  // EPI_SCALED: per-column scale (N) or null (== 1)
  const float *residual;  // EPI_SCALED, fp32 out: out = residual + value (M x N, ld_res) or null
  int64_t ld_res;
  int res_vec;            // residual rows are 16-byte aligned
  void *out;
  int64_t ldo;
  int out_dtype;  // EPI_SCALED: RT_BF16 or RT_F32 (bf16-rounded value widened)
  int epi;
  int accumulate;  // EPI_F32_STORE: out += result
  int vec_store;   // out rows are 16-byte aligned
  int tma_store;   // epilogue stages 32-row groups in shared memory and stores them with TMA
  int acc_small;   // int8: every |accumulator| < 2^22 (K·127·max|rhs| below it), 2-op conversion
  float *workspace;  // EPI_SPLIT: [splits][tiles][BM][BN] fp32 partial tiles
  // EPI_F32_STORE / EPI_BF16_STORE: out = round(addend + result) (M x N fp32, ld_add), or null
  const float *addend;
  int64_t ld_add;
};

template <typename T>
struct KindOf;
template <>
struct KindOf<int8_t> {
  static constexpr uint32_t dfmt = 2;  // S32
  static constexpr uint32_t abfmt = 1; // signed 8-bit
};
template <>
struct KindOf<__nv_bfloat16> {
  static constexpr uint32_t dfmt = 1;  // F32
  static constexpr uint32_t abfmt = 1; // BF16
};

template <typename T, bool A_MN, bool B_MN, int BN, int STAGES, int EPI = 8, int CG = 1>
struct GemmCfg {
  // CG = 2: a CTA pair (cluster of two) computes one (2·BM) x BN tile; each CTA holds BM rows of
  // A, BN/2 rows of B and BM accumulator rows x BN columns in its tensor memory
  static constexpr int BM = 128;
  static constexpr int TILE_M = BM * CG;
  static constexpr int ES = sizeof(T);
  static constexpr int KE = 128 / ES;  // K elements per stage
  static constexpr int UK = 32 / ES;   // K elements per tcgen05.mma
  static constexpr int B_ROWS = BN / CG;  // B rows (N) this CTA loads
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = B_ROWS * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  // EPI epilogue warps (8 or 16): EPI/4 per TMEM lane quarter, each taking BN/(EPI/4) columns
  static constexpr int EPI_WARPS = EPI;
  static constexpr int COLW = BN / (EPI / 4);
  static_assert(EPI == 8 || EPI == 16, "EPI");
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  // per epilogue warp: one 32-row x 128-byte staging buffer for TMA stores
  static constexpr int EPI_BYTES = EPI_WARPS * 4096;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 + 256;
  // Instruction descriptor: D format, A/B formats, majorness, N>>3 at [17,23), M>>4 at [24,29).
  static constexpr uint32_t IDESC = (KindOf<T>::dfmt << 4) | (KindOf<T>::abfmt << 7) |
                                    (KindOf<T>::abfmt << 10) | ((A_MN ? 1u : 0u) << 15) |
                                    ((B_MN ? 1u : 0u) << 16) |
                                    (static_cast<uint32_t>(BN >> 3) << 17) |
                                    (static_cast<uint32_t>(TILE_M >> 4) << 24);
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(CG == 1 || CG == 2, "CG");
  static_assert(B_ROWS % (128 / ES) == 0 || !B_MN, "MN-major B half: whole 128-byte boxes");
  static_assert(TMEM_COLS <= 512, "TMEM");
};

// K-major operand tile (rows × 128 B, 128B swizzle): 8-row groups 1024 B apart (SBO); the k-th
// MMA step starts 32 bytes further inside the swizzle atom.
// MN-major operand tile: boxes of (KE k-rows × 128 B) side by side along MN (LBO = KE·128 B);
// 8-k-row groups 1024 B apart (SBO); the k-th MMA step starts UK k-rows (UK·128 B) further.
template <bool MN, int KE, int UK>
__device__ __forceinline__ uint64_t operand_desc(uint32_t tile_addr, int kstep) {
  if constexpr (MN) {
    return make_sw128_desc(tile_addr + kstep * UK * 128, KE * 128, 1024);
  } else {
    return make_sw128_desc(tile_addr + kstep * 32, 16, 1024);
  }
}

template <bool MN, int ROWS, int KE, int ES>
__device__ __forceinline__ void load_operand(const CUtensorMap *map, uint64_t *bar, uint8_t *dst,
                                             int row0, int k0) {
  if constexpr (MN) {
    constexpr int PER_BOX = 128 / ES;  // MN elements per 128-byte box row
#pragma unroll
    for (int j = 0; j < ROWS / PER_BOX; ++j)
      tma_load_2d(map, bar, dst + j * (KE * 128), row0 + j * PER_BOX, k0);
  } else {
    tma_load_2d(map, bar, dst, k0, row0);
  }
}

// The same loads for a CTA pair: into this CTA's shared memory, completion counted on the
// barrier at cluster-window address bar0 (rank 0's).
template <bool MN, int ROWS, int KE, int ES>
__device__ __forceinline__ void load_operand_pair(const CUtensorMap *map, uint32_t bar0,
                                                  uint8_t *dst, int row0, int k0) {
  if constexpr (MN) {
    constexpr int PER_BOX = 128 / ES;
#pragma unroll
    for (int j = 0; j < ROWS / PER_BOX; ++j)
      tma_load_2d_pair(map, bar0, dst + j * (KE * 128), row0 + j * PER_BOX, k0);
  } else {
    tma_load_2d_pair(map, bar0, dst, k0, row0);
  }
}

// Exact int32 -> fp32 (round to nearest even) on the ALU and FMA pipes instead of the
// conversion unit, which a 128 x 256 tile's 32K conversions would otherwise saturate: with
// acc = hi·2^16 + lo (lo in [0, 2^16)) both halves are exact floats built in a mantissa, and one
// FMA rounds hi·2^16 + lo once.
__device__ __forceinline__ float i32_to_f32_rn(int acc) {
  const float hi = __int_as_float((acc >> 16) + 0x4B400000) - 12582912.0f;
  const float lo = __int_as_float((acc & 0xFFFF) | 0x4B000000) - 8388608.0f;
  return __fmaf_rn(hi, 65536.0f, lo);
}

template <typename T>
__device__ __forceinline__ float acc_to_float(uint32_t bits) {
  if constexpr (sizeof(T) == 1)
    return i32_to_f32_rn(static_cast<int>(bits));
  else
    return __uint_as_float(bits);
}

template <typename T>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs &p, int epi, int row, int n0,
                                               const uint32_t (&r)[32]) {
  if (row >= p.M) return;
  const bool full = p.vec_store && (n0 + 32 <= p.N);
  if (epi == EPI_SCALED) {
    const float ls = __ldg(p.a_scale + row);
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(acc_to_float<T>(r[j]), ls);
    if (p.b_scale != nullptr) {
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 s4 = __ldg(reinterpret_cast<const float4 *>(p.b_scale + n0 + j));
          v[j] = __fmul_rn(v[j], s4.x);
          v[j + 1] = __fmul_rn(v[j + 1], s4.y);
          v[j + 2] = __fmul_rn(v[j + 2], s4.z);
          v[j + 3] = __fmul_rn(v[j + 3], s4.w);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n0 + j < p.N) v[j] = __fmul_rn(v[j], __ldg(p.b_scale + n0 + j));
      }
    }
    if (p.out_dtype == RT_BF16) {
      uint16_t *o = static_cast<uint16_t *>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 w;
          w.x = bf16_bits(v[j]) | (uint32_t(bf16_bits(v[j + 1])) << 16);
          w.y = bf16_bits(v[j + 2]) | (uint32_t(bf16_bits(v[j + 3])) << 16);
          w.z = bf16_bits(v[j + 4]) | (uint32_t(bf16_bits(v[j + 5])) << 16);
          w.w = bf16_bits(v[j + 6]) | (uint32_t(bf16_bits(v[j + 7])) << 16);
          *reinterpret_cast<uint4 *>(o + j) = w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n0 + j < p.N) o[j] = bf16_bits(v[j]);
      }
    } else {
      float *o = static_cast<float *>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
      const float *res =
          p.residual != nullptr ? p.residual + static_cast<int64_t>(row) * p.ld_res + n0 : nullptr;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = bf16_round(v[j]);
        if (res != nullptr && n0 + j < p.N) v[j] = __fadd_rn(__ldg(res + j), v[j]);
      }
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          *reinterpret_cast<float4 *>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n0 + j < p.N) o[j] = v[j];
      }
    }
    return;
  }
  if (p.addend != nullptr) {  // out = round(addend + result), fp32 or bf16
    const float *ad = p.addend + static_cast<int64_t>(row) * p.ld_add + n0;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j)
      v[j] = (n0 + j < p.N) ? __fadd_rn(__ldg(ad + j), acc_to_float<T>(r[j])) : 0.0f;
    if (epi == EPI_BF16_STORE) {
      uint16_t *o = static_cast<uint16_t *>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) o[j] = bf16_bits(v[j]);
    } else {
      float *o = static_cast<float *>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) o[j] = v[j];
    }
    return;
  }
  if (epi == EPI_BF16_STORE) {
    uint16_t *o = static_cast<uint16_t *>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 w;
        w.x = bf16_bits(acc_to_float<T>(r[j])) | (uint32_t(bf16_bits(acc_to_float<T>(r[j + 1]))) << 16);
        w.y = bf16_bits(acc_to_float<T>(r[j + 2])) | (uint32_t(bf16_bits(acc_to_float<T>(r[j + 3]))) << 16);
        w.z = bf16_bits(acc_to_float<T>(r[j + 4])) | (uint32_t(bf16_bits(acc_to_float<T>(r[j + 5]))) << 16);
        w.w = bf16_bits(acc_to_float<T>(r[j + 6])) | (uint32_t(bf16_bits(acc_to_float<T>(r[j + 7]))) << 16);
        *reinterpret_cast<uint4 *>(o + j) = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < p.N) o[j] = bf16_bits(acc_to_float<T>(r[j]));
    }
    return;
  }
  float *o = static_cast<float *>(p.out) + static_cast<int64_t>(row) * p.ldo + n0;
  // EPI_F32_STORE
  if (full) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float4 w = make_float4(acc_to_float<T>(r[j]), acc_to_float<T>(r[j + 1]),
                             acc_to_float<T>(r[j + 2]), acc_to_float<T>(r[j + 3]));
      if (p.accumulate) {
        const float4 old = *reinterpret_cast<const float4 *>(o + j);
        w.x = __fadd_rn(old.x, w.x), w.y = __fadd_rn(old.y, w.y);
        w.z = __fadd_rn(old.z, w.z), w.w = __fadd_rn(old.w, w.w);
      }
      *reinterpret_cast<float4 *>(o + j) = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < p.N) o[j] = p.accumulate ? __fadd_rn(o[j], acc_to_float<T>(r[j]))
                                            : acc_to_float<T>(r[j]);
  }
}

// One 32-row group of 64 bf16 / 32 fp32 output columns through the warp's staging buffer:
// 128-byte swizzled rows (conflict-free 16-byte shared stores), then one TMA store that clips
// rows/columns outside the output.  `words` holds the 32 packed words of this lane's row.
__device__ __forceinline__ void stage_write(uint8_t *b, int lane, const uint32_t (&words)[32]) {
  if (lane == 0) bulk_wait_read_all();  // the warp's previous store has read the buffer
  __syncwarp();
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4 *>(b + lane * 128 + ((c ^ (lane & 7)) << 4)) =
        make_uint4(words[4 * c], words[4 * c + 1], words[4 * c + 2], words[4 * c + 3]);
  fence_proxy_async_smem();
  __syncwarp();
}
__device__ __forceinline__ void stage_issue(const CUtensorMap *map, uint8_t *b, int lane, int x,
                                            int y) {
  if (lane == 0) {
    tma_store_2d(map, b, x, y);
    bulk_commit_group();
  }
}
__device__ __forceinline__ void stage_and_store(const CUtensorMap *map, uint8_t *b, int lane,
                                                const uint32_t (&words)[32], int x, int y) {
  stage_write(b, lane, words);
  stage_issue(map, b, lane, x, y);
}

// Accumulator word -> fp32.  CONV 0: fp32 bits (kind::f16); 1: int32 known to lie in
// (-2^22, 2^22), exact through the 1.5·2^23 mantissa (one integer add, one float add);
// 2: any int32, exact round-to-nearest (i32_to_f32_rn).
template <int CONV>
__device__ __forceinline__ float cvt_acc(uint32_t b) {
  if constexpr (CONV == 0)
    return __uint_as_float(b);
  else if constexpr (CONV == 1)
    return __int_as_float(static_cast<int>(b) + 0x4B400000) - 12582912.0f;
  else
    return i32_to_f32_rn(static_cast<int>(b));
}

// One warp's share of a tile (32 rows, HALF columns from TMEM column t_row) through its staging
// buffer: bf16 groups of 64 columns or fp32 groups of 32, optionally scaled by the row scale a_s
// and the column scales bs[] (bf16-rounded like the reference when scaled).
// rmap (fp32 output only, or null): the residual, whose tile of each group is TMA-loaded into
// the staging buffer (completion on rbar, parity rphase) while the accumulators are read, then
// added after the rounding.
// The warp hands its accumulator columns back to the MMA warp (arrive on tempty_bar) as soon as
// its last TMEM read has completed, not after its stores, so the next MMA into this accumulator
// overlaps the conversion and stores: a bf16 group waits in the staging buffer, its TMA store
// deferred, while the next group is read from TMEM.
// tempty_addr: the barrier's address in the cluster shared window (this CTA's own barrier, or
// rank 0's when a CTA pair shares the accumulator-free barrier).
__device__ __forceinline__ void release_accumulator(uint32_t tempty_addr, int lane) {
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive_cluster(tempty_addr);
}
// Returns whether it arrived on tempty_bar (not when the warp's columns lie past the output).
template <int CONV, int HALF>
__device__ __forceinline__ bool epilogue_tma(const CUtensorMap *map, uint8_t *staging, int lane,
                                             uint32_t t_row, int x0, int x_end, int y,
                                             bool bf16_out, bool scaled, float a_s,
                                             const float *bs, const CUtensorMap *rmap,
                                             uint64_t *rbar, uint32_t &rphase,
                                             uint32_t tempty_bar) {
  if (bf16_out) {
    if (x0 >= x_end) return false;
    int pending = -1;  // column of the group staged but not yet stored
#pragma unroll 1
    for (int g = 0; g < HALF / 64; ++g) {
      const int n0 = x0 + g * 64;
      if (n0 >= x_end) break;  // warp-uniform
      // the group's two 32-column halves, each read, converted and packed before the next is
      // read (32 accumulator registers live, not 64)
      const bool last = g == HALF / 64 - 1 || n0 + 64 >= x_end;
      uint32_t w[32];
      const float4 *bs4 = reinterpret_cast<const float4 *>(bs + g * 64);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(g * 64 + 32 * h), r);
        tmem_ld_wait_regs(r);
        if (h == 1) {
          if (last) release_accumulator(tempty_bar, lane);
          if (pending >= 0) stage_issue(map, staging, lane, pending, y);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // columns 32h + 4j .. 32h + 4j + 3
          float v[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = cvt_acc<CONV>(r[4 * j + e]);
          if (scaled) {
            const float4 sc = bs4[8 * h + j];  // 16-byte broadcast read
            v[0] = __fmul_rn(__fmul_rn(v[0], a_s), sc.x), v[1] = __fmul_rn(__fmul_rn(v[1], a_s), sc.y);
            v[2] = __fmul_rn(__fmul_rn(v[2], a_s), sc.z), v[3] = __fmul_rn(__fmul_rn(v[3], a_s), sc.w);
          }
          w[16 * h + 2 * j] = pack_bf16x2(v[0], v[1]);
          w[16 * h + 2 * j + 1] = pack_bf16x2(v[2], v[3]);
        }
      }
      stage_write(staging, lane, w);
      if (last) {
        stage_issue(map, staging, lane, n0, y);
        pending = -1;
      } else {
        pending = n0;
      }
    }
    return true;
  } else {
    const int groups = min(HALF / 32, (x_end - x0 + 31) / 32);
#pragma unroll 1
    for (int g = 0; g < groups; ++g) {
      const int n0 = x0 + g * 32;
      if (rmap != nullptr && lane == 0) {
        bulk_wait_read_all();  // the previous store has read the staging buffer
        mbar_arrive_expect_tx(rbar, 4096);
        tma_load_2d(rmap, rbar, staging, n0, y);
      }
      uint32_t r[32];
      tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(g * 32), r);
      tmem_ld_wait_regs(r);
      if (g == groups - 1) release_accumulator(tempty_bar, lane);
      uint32_t w[32];
      const float4 *bs4 = reinterpret_cast<const float4 *>(bs + g * 32);
      bool res_ok = true;
      if (rmap != nullptr) {
        res_ok = mbar_wait(rbar, rphase);
        rphase ^= 1u;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = cvt_acc<CONV>(r[4 * j + e]);
        if (scaled) {
          const float4 sc = bs4[j];
          v[0] = bf16_round(__fmul_rn(__fmul_rn(v[0], a_s), sc.x));
          v[1] = bf16_round(__fmul_rn(__fmul_rn(v[1], a_s), sc.y));
          v[2] = bf16_round(__fmul_rn(__fmul_rn(v[2], a_s), sc.z));
          v[3] = bf16_round(__fmul_rn(__fmul_rn(v[3], a_s), sc.w));
        }
        if (rmap != nullptr && res_ok) {  // out = residual + value, the reference's fp32 add
          const float4 r4 = *reinterpret_cast<const float4 *>(staging + lane * 128 +
                                                              ((j ^ (lane & 7)) << 4));
          v[0] = __fadd_rn(r4.x, v[0]), v[1] = __fadd_rn(r4.y, v[1]);
          v[2] = __fadd_rn(r4.z, v[2]), v[3] = __fadd_rn(r4.w, v[3]);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) w[4 * j + e] = __float_as_uint(v[e]);
      }
      stage_and_store(map, staging, lane, w, n0, y);
    }
    return groups > 0;
  }
}

template <typename T, bool A_MN, bool B_MN, int BN, int STAGES, int EPI, int CG>
__global__ void __launch_bounds__(64 + 32 * EPI, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_c,
                     const __grid_constant__ CUtensorMap tma_r, GemmArgs p) {
  using C = GemmCfg<T, A_MN, B_MN, BN, STAGES, EPI, CG>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *a_tiles = smem;
  uint8_t *b_tiles = smem + STAGES * C::A_BYTES;
  uint8_t *staging_all = smem + STAGES * C::STAGE_BYTES;  // 1024-byte aligned
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * C::STAGE_BYTES + C::EPI_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + STAGES;
  uint64_t *tfull = bars + 2 * STAGES;
  uint64_t *tempty = bars + 2 * STAGES + 2;
  uint64_t *rfull = bars + 2 * STAGES + 4;  // per epilogue warp: its residual tile has landed
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4 + C::EPI_WARPS);
  __shared__ __align__(16) float s_bscale[BN];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // CTA pair: rank 0 issues the MMAs of the pair; both ranks load and run the epilogue
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  const int group = CG == 2 ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int groups = CG == 2 ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  pdl_trigger();  // the next kernel may launch and set itself up while this one runs
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      // rank 0's barrier collects the epilogue warps of both CTAs of a pair
      mbar_init(&tempty[b], C::EPI_WARPS * CG);
    }
    for (int w = 0; w < C::EPI_WARPS; ++w) mbar_init(&rfull[w], 1);
    fence_barrier_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    if (p.tma_store) tma_prefetch_desc(&tma_c);
    if (p.residual != nullptr && p.tma_store) tma_prefetch_desc(&tma_r);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (CG == 2)
    cluster_sync();  // both CTAs' barriers exist before either signals the other's
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // set-up above touches no global memory; operands, scales and outputs only after the
  // preceding kernel has completed
  pdl_wait();

  const int units = p.tiles_m * p.tiles_n * p.splits;
  // Unit u -> (tile n, tile m, split) and the split's k-block range, in 32-bit unsigned
  // arithmetic (split * kblocks stays far below 2^32): the single MMA-issuing thread runs this
  // between tiles while the tensor pipe drains, so it must be short (64-bit divisions there
  // left the tensor pipe idle ~0.9 us per tile).
  const uint32_t tiles_n = static_cast<uint32_t>(p.tiles_n);
  const uint32_t tiles_mn = static_cast<uint32_t>(p.tiles_m) * tiles_n;
  const uint32_t kblocks = static_cast<uint32_t>(p.kblocks);
  const uint32_t splits = static_cast<uint32_t>(p.splits);
  auto k_range = [&](uint32_t uu, int &kb0, int &kb1) {
    if (splits == 1) {
      kb0 = 0, kb1 = static_cast<int>(kblocks);
    } else {
      const uint32_t split = uu / tiles_mn;
      kb0 = static_cast<int>(split * kblocks / splits);
      kb1 = static_cast<int>((split + 1) * kblocks / splits);
    }
  };
  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = group; u < units && ok; u += groups) {
        const uint32_t uu = static_cast<uint32_t>(u);
        const uint32_t rest = uu / tiles_n;
        const int tn = static_cast<int>(uu - rest * tiles_n);
        const int tm = static_cast<int>(rest % static_cast<uint32_t>(p.tiles_m));
        int kb0, kb1;
        k_range(uu, kb0, kb1);
        const int a_row = tm * C::TILE_M + static_cast<int>(rank) * C::BM;
        const int b_row = tn * BN + static_cast<int>(rank) * C::B_ROWS;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1)) {
            ok = false;
            break;
          }
          if constexpr (CG == 2) {
            // both CTAs' loads complete on rank 0's full barrier, which expects the bytes of both
            const uint32_t bar0 = mapa_shared(smem_u32(&full[stage]), 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            load_operand_pair<A_MN, C::BM, C::KE, C::ES>(&tma_a, bar0,
                                                         a_tiles + stage * C::A_BYTES, a_row,
                                                         kb * C::KE);
            load_operand_pair<B_MN, C::B_ROWS, C::KE, C::ES>(&tma_b, bar0,
                                                             b_tiles + stage * C::B_BYTES, b_row,
                                                             kb * C::KE);
          } else {
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            load_operand<A_MN, C::BM, C::KE, C::ES>(&tma_a, &full[stage],
                                                    a_tiles + stage * C::A_BYTES, a_row,
                                                    kb * C::KE);
            load_operand<B_MN, BN, C::KE, C::ES>(&tma_b, &full[stage],
                                                 b_tiles + stage * C::B_BYTES, b_row, kb * C::KE);
          }
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
      }
      if constexpr (CG == 2) {
        // producer tail: every stage this CTA filled has been released (rank 0's MMA commits
        // arrive on this CTA's barriers) before the CTA can leave
        for (int i = 0; i < STAGES && ok; ++i) {
          ok = mbar_wait(&empty[stage], phase ^ 1);
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t a_base = smem_u32(a_tiles), b_base = smem_u32(b_tiles);
      for (int u = group; u < units && ok; u += groups) {
        int kb0, kb1;
        k_range(static_cast<uint32_t>(u), kb0, kb1);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = a_base + stage * C::A_BYTES;
          const uint32_t b_addr = b_base + stage * C::B_BYTES;
#pragma unroll
          for (int j = 0; j < C::KE / C::UK; ++j) {
            const uint64_t ad = operand_desc<A_MN, C::KE, C::UK>(a_addr, j);
            const uint64_t bd = operand_desc<B_MN, C::KE, C::UK>(b_addr, j);
            const uint32_t accumulate = (kb > kb0 || j > 0) ? 1u : 0u;
            if constexpr (CG == 2) {
              if constexpr (sizeof(T) == 1)
                umma_i8_pair(d_tmem, ad, bd, C::IDESC, accumulate);
              else
                umma_f16_pair(d_tmem, ad, bd, C::IDESC, accumulate);
            } else if constexpr (sizeof(T) == 1) {
              umma_i8(d_tmem, ad, bd, C::IDESC, accumulate);
            } else {
              umma_f16(d_tmem, ad, bd, C::IDESC, accumulate);
            }
          }
          // the stage is free in both CTAs once these MMAs have read it
          if constexpr (CG == 2)
            umma_commit_pair(&empty[stage]);
          else
            umma_commit(&empty[stage]);
          if (++stage == STAGES) stage = 0, phase ^= 1;
        }
        if constexpr (CG == 2)
          umma_commit_pair(&tfull[acc]);
        else
          umma_commit(&tfull[acc]);
        if (++acc == 2) acc = 0, acc_phase ^= 1;
      }
    }
  } else {
    // epilogue warps 2..9: TMEM lane quarter (warp % 4) holds accumulator rows 32·(warp%4)..+31;
    // warps 2..5 take the tile's first COLW columns, warps 6..9 the next COLW, and so on
    constexpr int HALF = C::COLW;  // columns of this warp
    const int sub = warp & 3;
    const int col0 = ((warp - 2) >> 2) * HALF;  // first tile column of this warp
    const int ep_tid = threadIdx.x - 64;        // 0..255 across the epilogue warps
    uint8_t *staging = staging_all + (warp - 2) * 4096;
    const bool split_mode = p.epi == EPI_SPLIT;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t rphase = 0;  // parity of this warp's residual barrier
    // the accumulator-free barriers live in rank 0 (its MMA thread waits on them)
    const uint32_t tempty0 = CG == 2 ? mapa_shared(smem_u32(&tempty[0]), 0) : smem_u32(&tempty[0]);
    const uint32_t tempty1 = CG == 2 ? mapa_shared(smem_u32(&tempty[1]), 0) : smem_u32(&tempty[1]);
    for (int u = group; u < units; u += groups) {
      const uint32_t uu = static_cast<uint32_t>(u);
      const uint32_t rest = uu / tiles_n;
      const int tn = static_cast<int>(uu - rest * tiles_n);
      const int tm = static_cast<int>(rest % static_cast<uint32_t>(p.tiles_m));
      const int split = static_cast<int>(uu / tiles_mn);
      const int tile = tm * p.tiles_n + tn;
      const int trow = sub * 32 + lane;
      const int row = tm * C::TILE_M + static_cast<int>(rank) * C::BM + trow;
      // this tile's scales, requested before the wait so that their latency overlaps the MMA
      const bool scaled = p.epi == EPI_SCALED && p.tma_store;
      static_assert(BN <= 32 * C::EPI_WARPS, "one column scale per epilogue thread");
      float col_scale = 1.0f, a_s = 1.0f;
      if (scaled) {
        const int n = tn * BN + ep_tid;
        if (ep_tid < BN && p.b_scale != nullptr && n < p.N) col_scale = __ldg(p.b_scale + n);
        if (row < p.M) a_s = __ldg(p.a_scale + row);
      }
      // every lane polls; the warp proceeds only if all lanes saw the phase complete, so the
      // .sync.aligned TMEM loads below are always executed by the full warp
      const bool lane_ok = mbar_wait(&tfull[acc], acc_phase);
      // the epilogue warps agree (barrier 1), so a timed-out wait can never leave some of them
      // inside the column-scale barrier below
      uint32_t all_ok;
      asm volatile(
          "{\n\t.reg .pred p, q;\n\t"
          "setp.ne.u32 p, %1, 0;\n\t"
          "bar.red.and.pred q, 1, %2, p;\n\t"
          "selp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(all_ok)
          : "r"(static_cast<uint32_t>(lane_ok)), "n"(32 * C::EPI_WARPS)
          : "memory");
      if (!all_ok) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) +
                             static_cast<uint32_t>(acc * BN + col0);
      bool released = false;  // the epilogue has arrived on tempty[acc] itself
      const uint32_t tempty_addr = acc == 0 ? tempty0 : tempty1;
      if (p.tma_store) {
        // column scales of this tile in shared memory; the barrier above also guarantees that
        // every warp has finished reading the previous tile's (barrier 1: the epilogue warps)
        if (scaled) {
          if (ep_tid < BN) s_bscale[ep_tid] = col_scale;
          asm volatile("bar.sync 1, %0;" ::"n"(32 * C::EPI_WARPS) : "memory");
        }
        const bool bf16_out =
            !split_mode && (p.out_dtype == RT_BF16 || p.epi == EPI_BF16_STORE);
        // split mode: the fp32 partial tile goes to its own 128 x BN block of the workspace
        const int y = split_mode
                          ? (split * p.tiles_m * p.tiles_n + tile) * C::TILE_M +
                                static_cast<int>(rank) * C::BM + sub * 32
                          : tm * C::TILE_M + static_cast<int>(rank) * C::BM + sub * 32;
        const int x0 = (split_mode ? 0 : tn * BN) + col0;
        const int x_end = split_mode ? BN : p.N;
        const float *bs = s_bscale + col0;
        const CUtensorMap *rmap = (p.residual != nullptr && !bf16_out) ? &tma_r : nullptr;
        uint64_t *rbar = &rfull[warp - 2];
        if (!split_mode && y >= p.M) {
          // this warp's 32 rows lie past the output: nothing to store
        } else if constexpr (sizeof(T) == 1) {
          if (p.acc_small)
            released = epilogue_tma<1, HALF>(&tma_c, staging, lane, t_row, x0, x_end, y,
                                             bf16_out, scaled, a_s, bs, rmap, rbar, rphase,
                                             tempty_addr);
          else
            released = epilogue_tma<2, HALF>(&tma_c, staging, lane, t_row, x0, x_end, y,
                                             bf16_out, scaled, a_s, bs, rmap, rbar, rphase,
                                             tempty_addr);
        } else {
          released = epilogue_tma<0, HALF>(&tma_c, staging, lane, t_row, x0, x_end, y, bf16_out,
                                           scaled, a_s, bs, rmap, rbar, rphase, tempty_addr);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < HALF / 32; ++c) {
          const int n0 = tn * BN + col0 + c * 32;
          if (n0 >= p.N) break;
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c * 32), r);
          tmem_ld_wait_regs(r);
          epilogue_chunk<T>(p, p.epi, row, n0, r);
        }
      }
      if (!released) release_accumulator(tempty_addr, lane);
      if (++acc == 2) acc = 0, acc_phase ^= 1;
    }
    if (p.tma_store && lane == 0) bulk_wait_all();  // staged stores done before the CTA exits
  }
  __syncwarp();
  tc_fence_before();
  if constexpr (CG == 2) {
    // neither CTA leaves while the other may still signal its barriers or read its tiles
    cluster_sync();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    }
  } else {
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
  }
}

// -------------------------------------------------------------------------------------------
// SIMT kernels with the same arithmetic, for operands TMA cannot address (unaligned strides).
// -------------------------------------------------------------------------------------------
__global__ void simt_scaled_i8_kernel(const int8_t *lhs, int64_t slm, int64_t slk,
                                      const int8_t *rhs, int64_t srk, int64_t srn,
                                      const float *ls, const float *rs, void *out, int out_dtype,
                                      int64_t ldo, int64_t M, int64_t N, int64_t K,
                                      const float *residual, int64_t ld_res) {
  pdl_wait();
  pdl_trigger();
  const int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t m = blockIdx.y * static_cast<int64_t>(blockDim.y) + threadIdx.y;
  if (m >= M || n >= N) return;
  int acc = 0;
  for (int64_t k = 0; k < K; ++k)
    acc += static_cast<int>(lhs[m * slm + k * slk]) * static_cast<int>(rhs[k * srk + n * srn]);
  float v = __fmul_rn(__int2float_rn(acc), __ldg(ls + m));
  if (rs != nullptr) v = __fmul_rn(v, __ldg(rs + n));
  if (out_dtype == RT_BF16) {
    static_cast<uint16_t *>(out)[m * ldo + n] = bf16_bits(v);
  } else {
    v = bf16_round(v);
    if (residual != nullptr) v = __fadd_rn(residual[m * ld_res + n], v);
    static_cast<float *>(out)[m * ldo + n] = v;
  }
}

__global__ void simt_gradw_kernel(const uint16_t *g, int64_t ldg, const uint16_t *x, int64_t ldx,
                                  void *out, int out_dtype, int64_t ldo, int64_t Mt, int64_t N,
                                  int64_t K, int accumulate, const float *addend, int64_t ld_add) {
  pdl_wait();
  pdl_trigger();
  const int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t n = blockIdx.y * static_cast<int64_t>(blockDim.y) + threadIdx.y;
  if (n >= N || k >= K) return;
  float acc = 0.0f;
  for (int64_t m = 0; m < Mt; ++m)
    acc = __fadd_rn(acc, __fmul_rn(bf16_from_bits(g[m * ldg + n]), bf16_from_bits(x[m * ldx + k])));
  if (addend != nullptr) acc = __fadd_rn(addend[n * ld_add + k], acc);
  if (out_dtype == RT_F32) {
    float *o = static_cast<float *>(out) + n * ldo + k;
    *o = accumulate ? __fadd_rn(*o, acc) : acc;
  } else {
    static_cast<uint16_t *>(out)[n * ldo + k] = bf16_bits(acc);
  }
}

__global__ void simt_matmul_bf16_kernel(const uint16_t *a, int64_t lda, const uint16_t *b,
                                        int64_t ldb, void *out, int out_dtype, int64_t ldo,
                                        int64_t M, int64_t N, int64_t K) {
  pdl_wait();
  pdl_trigger();
  const int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t m = blockIdx.y * static_cast<int64_t>(blockDim.y) + threadIdx.y;
  if (m >= M || n >= N) return;
  float acc = 0.0f;
  for (int64_t k = 0; k < K; ++k)
    acc = __fadd_rn(acc, __fmul_rn(bf16_from_bits(a[m * lda + k]), bf16_from_bits(b[k * ldb + n])));
  if (out_dtype == RT_F32)
    static_cast<float *>(out)[m * ldo + n] = acc;
  else
    static_cast<uint16_t *>(out)[m * ldo + n] = bf16_bits(acc);
}

// -------------------------------------------------------------------------------------------
// Host side: tensor maps (driver entry point fetched once), launch helpers.
// -------------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 2-D map over a row-major matrix: `inner` contiguous elements per row, `outer` rows,
// `row_bytes` between rows; box = box_inner × box_outer with 128-byte swizzle, zero OOB fill.
static int make_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner,
                    uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr) return fail(RT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RT_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return RT_OK;
}

// Operand description for the UMMA path.  A is (M,K), B is (N,K) in GEMM terms.
struct Operand {
  const void *ptr;
  bool mn;           // MN-major (MN index contiguous) vs K-major
  int64_t ld;        // elements between consecutive rows of the stored matrix
  int64_t rows_mn;   // extent along M (or N)
  int64_t extent_k;  // extent along K
};

template <typename T, bool MN>
static int operand_map(CUtensorMap *map, const Operand &o, int tile_rows) {
  using Cfg = GemmCfg<T, false, false, 128, 1>;
  const CUtensorMapDataType dt =
      sizeof(T) == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if constexpr (MN)
    return make_map(map, dt, o.ptr, o.rows_mn, o.extent_k, o.ld * sizeof(T), 128 / sizeof(T),
                    Cfg::KE);
  else
    return make_map(map, dt, o.ptr, o.extent_k, o.rows_mn, o.ld * sizeof(T), Cfg::KE, tile_rows);
}

template <typename T, bool A_MN, bool B_MN, int BN, int STAGES, int EPI = 8, int CG = 1>
static int launch_umma(const Operand &a, const Operand &b, GemmArgs args, cudaStream_t s) {
  using C = GemmCfg<T, A_MN, B_MN, BN, STAGES, EPI, CG>;
  CUtensorMap ma, mb, mc, mr;
  memset(&mr, 0, sizeof(mr));
  memset(&mc, 0, sizeof(mc));
  int rc = operand_map<T, A_MN>(&ma, a, C::BM);
  if (rc) return rc;
  rc = operand_map<T, B_MN>(&mb, b, C::B_ROWS);
  if (rc) return rc;
  if (CG == 2 && args.splits > 1)
    return fail(RT_ERR_UNSUPPORTED, "umma_gemm: CTA-pair tiles take no split-K");
  args.tiles_m = static_cast<int>((args.M + C::TILE_M - 1) / C::TILE_M);
  args.tiles_n = static_cast<int>((args.N + BN - 1) / BN);
  args.kblocks = static_cast<int>((args.K + C::KE - 1) / C::KE);
  if (args.splits < 1) args.splits = 1;
  if (args.splits > args.kblocks) args.splits = args.kblocks;
  // TMA-store epilogue: 16-byte aligned rows and a plain store (no accumulate), or the split-K
  // partial tiles (fp32, BN columns, one 128-row block per split and tile)
  const bool out_bf16 = args.out_dtype == RT_BF16 || args.epi == EPI_BF16_STORE;
  if (args.epi == EPI_SPLIT) {
    args.tma_store = 1;
    rc = make_map(&mc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, args.workspace, static_cast<uint64_t>(BN),
                  static_cast<uint64_t>(args.splits) * args.tiles_m * args.tiles_n * C::BM,
                  static_cast<uint64_t>(BN) * 4, 32, 32);
    if (rc) return rc;
  } else {
    args.tma_store = args.vec_store && args.addend == nullptr &&
                     (args.epi == EPI_SCALED || args.epi == EPI_BF16_STORE ||
                      (args.epi == EPI_F32_STORE && !args.accumulate));
  }
  if (args.tma_store && args.epi != EPI_SPLIT) {
    const size_t es = out_bf16 ? 2 : 4;
    rc = make_map(&mc, out_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                  args.out, static_cast<uint64_t>(args.N), static_cast<uint64_t>(args.M),
                  static_cast<uint64_t>(args.ldo) * es, static_cast<uint32_t>(128 / es), 32);
    if (rc) return rc;
  }
  if (args.tma_store && args.residual != nullptr) {
    // the residual tile of each fp32 output group, loaded by TMA into the group's staging buffer
    if (!args.res_vec) {
      args.tma_store = 0;  // unaligned residual rows: the lane-per-row epilogue adds it
    } else {
      rc = make_map(&mr, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, args.residual,
                    static_cast<uint64_t>(args.N), static_cast<uint64_t>(args.M),
                    static_cast<uint64_t>(args.ld_res) * 4, 32, 32);
      if (rc) return rc;
    }
  }

  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  if ((rc = rt_sm_count(&sms)) != RT_OK) return rc;
  static std::mutex mu;
  static bool configured[64] = {false};
  static int pair_slots[64] = {0};  // co-resident CTA pairs of this kernel per device
  auto kernel = umma_gemm_kernel<T, A_MN, B_MN, BN, STAGES, EPI, CG>;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
      cudaError_t e =
          cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
      if (e != cudaSuccess)
        return fail(RT_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      if constexpr (CG == 2) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1));
        cfg.blockDim = dim3(C::THREADS);
        cfg.dynamicSmemBytes = C::SMEM_BYTES;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr, cfg.numAttrs = 1;
        int clusters = 0;
        e = cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg);
        if (e != cudaSuccess || clusters < 1)
          return fail(RT_ERR_CUDA, "cudaOccupancyMaxActiveClusters: %s (%d)",
                      cudaGetErrorString(e), clusters);
        pair_slots[dev] = clusters;
      }
      configured[dev] = true;
    }
  }
  const int64_t units = static_cast<int64_t>(args.tiles_m) * args.tiles_n * args.splits;
  if constexpr (CG == 2) {
    const int64_t slots = dev >= 0 && dev < 64 ? pair_slots[dev] : sms / 2;
    const int pairs = static_cast<int>(units < slots ? units : slots);
    launch_k_cluster2(kernel, 2 * pairs, C::THREADS, C::SMEM_BYTES, s, ma, mb, mc, mr, args);
  } else {
    const int grid = static_cast<int>(units < sms ? units : sms);
    launch_k(kernel, grid, C::THREADS, C::SMEM_BYTES, s, ma, mb, mc, mr, args);
  }
  return check_launch("umma_gemm_kernel");
}

template <typename T>
static int kblocks_of(int64_t K) {
  return static_cast<int>((K + (128 / sizeof(T)) - 1) / (128 / sizeof(T)));
}

}  // namespace rt

// ===========================================================================================
// C ABI
// ===========================================================================================
using namespace rt;

extern "C" int rt_scaled_int8_mm(const int8_t *lhs, int64_t lhs_stride_m, int64_t lhs_stride_k,
                                 const int8_t *rhs, int64_t rhs_stride_k, int64_t rhs_stride_n,
                                 const float *lhs_scale, const float *rhs_scale, void *out,
                                 int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                                 int rhs_abs_max, const float *residual, int64_t ld_residual,
                                 void *stream) {
  if (M < 0 || N < 0 || K < 0) return fail(RT_ERR_INVALID_ARGUMENT, "scaled_int8_mm: negative shape");
  if (out_dtype != RT_BF16 && out_dtype != RT_F32)
    return fail(RT_ERR_DTYPE, "scaled_int8_mm: output must be bfloat16 or float32");
  if (residual != nullptr && out_dtype != RT_F32)
    return fail(RT_ERR_DTYPE, "scaled_int8_mm: a residual needs a float32 output");
  if (M == 0 || N == 0) return RT_OK;
  if (lhs == nullptr || rhs == nullptr || lhs_scale == nullptr || out == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "scaled_int8_mm: null pointer");
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2)
    return fail(RT_ERR_UNSUPPORTED, "scaled_int8_mm: dimension too large");
  cudaStream_t s = as_stream(stream);
  const size_t osz = out_dtype == RT_BF16 ? 2 : 4;
  GemmArgs args{};
  args.M = static_cast<int>(M), args.N = static_cast<int>(N), args.K = static_cast<int>(K);
  args.a_scale = lhs_scale, args.b_scale = rhs_scale, args.out = out, args.ldo = ldo;
  args.residual = residual, args.ld_res = ld_residual;
  args.res_vec = residual != nullptr && aligned16(residual) && ld_residual % 4 == 0;
  args.out_dtype = out_dtype, args.epi = EPI_SCALED, args.splits = 1;
  const int64_t rhs_bound = (rhs_abs_max <= 0 || rhs_abs_max > 128) ? 128 : rhs_abs_max;
  args.acc_small = K * 128 * rhs_bound < (int64_t(1) << 22);
  args.vec_store = aligned16(out) && (ldo * static_cast<int64_t>(osz)) % 16 == 0 &&
                   (rhs_scale == nullptr || aligned16(rhs_scale));
  // operand majorness from strides, as the reference kernel addresses them
  const bool a_k = lhs_stride_k == 1, a_mn = !a_k && lhs_stride_m == 1;
  const bool b_k = rhs_stride_k == 1, b_mn = !b_k && rhs_stride_n == 1;
  const bool a_ok = aligned16(lhs) && K > 0 &&
                    ((a_k && lhs_stride_m % 16 == 0) || (a_mn && lhs_stride_k % 16 == 0));
  const bool b_ok = aligned16(rhs) && K > 0 &&
                    ((b_k && rhs_stride_n % 16 == 0) || (b_mn && rhs_stride_k % 16 == 0));
  if (a_ok && b_ok) {
    Operand A{lhs, a_mn, a_k ? lhs_stride_m : lhs_stride_k, M, K};
    Operand B{rhs, b_mn, b_k ? rhs_stride_n : rhs_stride_k, N, K};
    const bool narrow = N <= 128;
    // fp32 outputs (twice the bytes per tile, and the residual tiles) run sixteen epilogue warps;
    // bf16 outputs eight (measured faster each way).  Wide tiles run on CTA pairs: 256 x 256
    // per pair, each SM loading 128 rows of A and 128 of B per stage instead of 128 + 256
#define RT_GO(AMN, BMN)                                                                     \
  if (narrow) return launch_umma<int8_t, AMN, BMN, 128, 6>(A, B, args, s);                  \
  if (pair) return wide_epi ? launch_umma<int8_t, AMN, BMN, 256, 5, 16, 2>(A, B, args, s)   \
                            : launch_umma<int8_t, AMN, BMN, 256, 6, 8, 2>(A, B, args, s);   \
  return wide_epi ? launch_umma<int8_t, AMN, BMN, 256, 3, 16>(A, B, args, s)                \
                  : launch_umma<int8_t, AMN, BMN, 256, 4>(A, B, args, s)
    const bool wide_epi = out_dtype == RT_F32;
    // pairs pay off where the MMA sets the pace (long contractions); at K = 512 the tile period
    // is the epilogue's and the pair's cluster set-up only adds to it (measured both ways)
    const bool pair = pair_enabled() && M > 128 && K >= 1024;
    if (!a_mn && !b_mn) {
      RT_GO(false, false);
    }
    if (!a_mn && b_mn) {
      RT_GO(false, true);
    }
    if (a_mn && !b_mn) {
      RT_GO(true, false);
    }
    RT_GO(true, true);
#undef RT_GO
  }
  const dim3 block(32, 8);
  const dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((M + 7) / 8));
  launch_k(simt_scaled_i8_kernel, grid, block, 0, s, lhs, lhs_stride_m, lhs_stride_k, rhs, rhs_stride_k,
                                                rhs_stride_n, lhs_scale, rhs_scale, out, out_dtype,
                                                ldo, M, N, K, residual, ld_residual);
  return check_launch("simt_scaled_i8_kernel");
}

extern "C" int rt_matmul_bf16(const void *a, int64_t lda, const void *b, int64_t ldb, void *out,
                              int out_dtype, int64_t ldo, int64_t M, int64_t N, int64_t K,
                              void *stream) {
  if (M < 0 || N < 0 || K < 0) return fail(RT_ERR_INVALID_ARGUMENT, "matmul_bf16: negative shape");
  if (out_dtype != RT_BF16 && out_dtype != RT_F32)
    return fail(RT_ERR_DTYPE, "matmul_bf16: output must be bfloat16 or float32");
  if (M == 0 || N == 0) return RT_OK;
  if (a == nullptr || b == nullptr || out == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "matmul_bf16: null pointer");
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX / 2)
    return fail(RT_ERR_UNSUPPORTED, "matmul_bf16: dimension too large");
  cudaStream_t s = as_stream(stream);
  const size_t osz = out_dtype == RT_BF16 ? 2 : 4;
  if (K == 0) {
    cudaError_t e = cudaMemset2DAsync(out, ldo * osz, 0, N * osz, M, s);
    return e == cudaSuccess ? RT_OK : fail(RT_ERR_CUDA, "matmul_bf16 memset: %s", cudaGetErrorString(e));
  }
  // A (M x K) row-major is K-major; B (K x N) row-major is MN-major: the tcgen05 kind::f16 GEMM
  // reads both in place (no transposed or padded copies).  Rows TMA cannot address (not 16-byte
  // aligned) take a SIMT kernel with fp32 accumulation.
  if (!aligned16(a) || !aligned16(b) || (lda * 2) % 16 != 0 || (ldb * 2) % 16 != 0) {
    const dim3 block(32, 8);
    const dim3 grid(static_cast<unsigned>((N + 31) / 32), static_cast<unsigned>((M + 7) / 8));
    launch_k(simt_matmul_bf16_kernel, grid, block, 0, s, static_cast<const uint16_t *>(a), lda,
             static_cast<const uint16_t *>(b), ldb, out, out_dtype, ldo, M, N, K);
    return check_launch("simt_matmul_bf16_kernel");
  }
  GemmArgs args{};
  args.M = static_cast<int>(M), args.N = static_cast<int>(N), args.K = static_cast<int>(K);
  args.out = out, args.ldo = ldo, args.out_dtype = out_dtype, args.splits = 1;
  args.epi = out_dtype == RT_F32 ? EPI_F32_STORE : EPI_BF16_STORE;
  args.vec_store = aligned16(out) && (ldo * static_cast<int64_t>(osz)) % 16 == 0;
  Operand A{a, false, lda, M, K};
  Operand B{b, true, ldb, N, K};
  if (N <= 128) return launch_umma<__nv_bfloat16, false, true, 128, 6>(A, B, args, s);
  if (pair_enabled() && M > 128 && K >= 1024)
    return launch_umma<__nv_bfloat16, false, true, 256, 6, 8, 2>(A, B, args, s);
  return launch_umma<__nv_bfloat16, false, true, 256, 4>(A, B, args, s);
}

namespace rt {
constexpr int GW_BN = 256;
constexpr int64_t GW_TILE_BYTES = 128 * GW_BN * 4;
static int64_t gw_tiles(int64_t N, int64_t K) { return ((N + 127) / 128) * ((K + GW_BN - 1) / GW_BN); }
// Split-K reduction of the grad_weight partial tiles: out[n, k] (+)= sum over splits, in split
// order, of ws[split][tile(n, k)][n % 128][k % BN].  Four consecutive k per thread, so both the
// partial-tile reads and the output writes are coalesced.
template <int BN>
__global__ void __launch_bounds__(256)
    splitk_reduce_kernel(const float *__restrict__ ws, int splits, int tiles_m, int tiles_n,
                         int rows, int cols, void *out, int out_dtype, int64_t ldo,
                         int accumulate, int vec_out, const float *addend, int64_t ld_add) {
  pdl_wait();
  pdl_trigger();
  const int groups = (cols + 3) >> 2;
  const int64_t total = static_cast<int64_t>(rows) * groups;
  const int64_t split_stride = static_cast<int64_t>(tiles_m) * tiles_n * 128 * BN;
  const bool idx32 = total <= static_cast<int64_t>(UINT32_MAX);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    // element group -> (row, col): a 32-bit division whenever the index fits (a 64-bit one is a
    // long instruction sequence per four elements)
    const int row = idx32 ? static_cast<int>(static_cast<uint32_t>(i) / static_cast<uint32_t>(groups))
                          : static_cast<int>(i / groups);
    const int col = static_cast<int>(i - static_cast<int64_t>(row) * groups) * 4;
    const int tile = (row >> 7) * tiles_n + col / BN;
    const float *src = ws + (static_cast<int64_t>(tile) * 128 + (row & 127)) * BN + col % BN;
    float4 v = splits > 0 ? __ldcs(reinterpret_cast<const float4 *>(src))
                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 4
    for (int sp = 1; sp < splits; ++sp) {
      const float4 f = __ldcs(reinterpret_cast<const float4 *>(src + sp * split_stride));
      v.x = __fadd_rn(v.x, f.x), v.y = __fadd_rn(v.y, f.y);
      v.z = __fadd_rn(v.z, f.z), v.w = __fadd_rn(v.w, f.w);
    }
    if (addend != nullptr) {  // out = round(addend + sum), the order of `accumulate`
      const float *ad = addend + static_cast<int64_t>(row) * ld_add + col;
      v.x = __fadd_rn(ad[0], v.x);
      if (col + 1 < cols) v.y = __fadd_rn(ad[1], v.y);
      if (col + 2 < cols) v.z = __fadd_rn(ad[2], v.z);
      if (col + 3 < cols) v.w = __fadd_rn(ad[3], v.w);
    }
    const float r[4] = {v.x, v.y, v.z, v.w};
    if (out_dtype == RT_F32) {
      float *o = static_cast<float *>(out) + static_cast<int64_t>(row) * ldo + col;
      if (vec_out && col + 4 <= cols) {
        float4 w = v;
        if (accumulate) {
          const float4 old = *reinterpret_cast<const float4 *>(o);
          w.x = __fadd_rn(old.x, w.x), w.y = __fadd_rn(old.y, w.y);
          w.z = __fadd_rn(old.z, w.z), w.w = __fadd_rn(old.w, w.w);
        }
        *reinterpret_cast<float4 *>(o) = w;
      } else {
        for (int j = 0; j < 4 && col + j < cols; ++j) o[j] = accumulate ? __fadd_rn(o[j], r[j]) : r[j];
      }
    } else {
      uint16_t *o = static_cast<uint16_t *>(out) + static_cast<int64_t>(row) * ldo + col;
      if (vec_out && col + 4 <= cols) {
        *reinterpret_cast<uint2 *>(o) =
            make_uint2(bf16_bits(r[0]) | (uint32_t(bf16_bits(r[1])) << 16),
                       bf16_bits(r[2]) | (uint32_t(bf16_bits(r[3])) << 16));
      } else {
        for (int j = 0; j < 4 && col + j < cols; ++j) o[j] = bf16_bits(r[j]);
      }
    }
  }
}

// split count: enough units to cover every SM, bounded by the K blocks and the workspace
static int gw_splits(int64_t M_tok, int64_t N, int64_t K, int sms, int64_t workspace_bytes) {
  const int64_t tiles = gw_tiles(N, K);
  const int64_t kb = (M_tok + 63) / 64;
  if (tiles >= sms) return 1;
  int64_t s = sms / tiles;
  if (s > kb) s = kb;
  const int64_t fit = workspace_bytes > 0 ? workspace_bytes / (tiles * GW_TILE_BYTES) : 0;
  if (s > fit) s = fit;
  return s < 2 ? 1 : static_cast<int>(s);
}
}  // namespace rt

extern "C" int64_t rt_grad_weight_workspace_bytes(int64_t M_tok, int64_t N, int64_t K) {
  int sms = 0;
  if (rt_sm_count(&sms) != RT_OK || M_tok <= 0 || N <= 0 || K <= 0) return 0;
  const int s = gw_splits(M_tok, N, K, sms, INT64_MAX / 4);
  if (s <= 1) return 0;
  const int64_t tiles = gw_tiles(N, K);
  return static_cast<int64_t>(s) * tiles * GW_TILE_BYTES;
}

namespace rt {
static int grad_weight_impl(const void *g, int64_t ldg, const void *x, int64_t ldx, void *out,
                            int out_dtype, int64_t ldo, int64_t M_tok, int64_t N, int64_t K,
                            int accumulate, const float *addend, int64_t ld_add, void *workspace,
                            int64_t workspace_bytes, void *stream) {
  if (M_tok < 0 || N < 0 || K < 0) return fail(RT_ERR_INVALID_ARGUMENT, "grad_weight: shape");
  if (addend != nullptr && accumulate)
    return fail(RT_ERR_INVALID_ARGUMENT, "grad_weight: accumulate and an addend exclude each other");
  if (out_dtype != RT_F32 && out_dtype != RT_BF16)
    return fail(RT_ERR_DTYPE, "grad_weight: output must be float32 or bfloat16");
  if (out_dtype == RT_BF16 && accumulate)
    return fail(RT_ERR_UNSUPPORTED, "grad_weight: accumulate needs a float32 output");
  if (N == 0 || K == 0) return RT_OK;
  if (out == nullptr || (M_tok > 0 && (g == nullptr || x == nullptr)))
    return fail(RT_ERR_INVALID_ARGUMENT, "grad_weight: null pointer");
  if (workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(RT_ERR_ALIGNMENT, "grad_weight: workspace must be 256-byte aligned");
  cudaStream_t s = as_stream(stream);
  const size_t osz = out_dtype == RT_BF16 ? 2 : 4;
  if (M_tok == 0 && addend != nullptr) {
    // nothing to add: out = round(addend), through the split-K reduce with no splits read
    launch_k(splitk_reduce_kernel<GW_BN>, 1u, 256, 0, s, static_cast<const float *>(nullptr), 0,
             0, 0, static_cast<int>(N), static_cast<int>(K), out, out_dtype, ldo, 0, 0, addend,
             ld_add);
    return check_launch("splitk_reduce_kernel");
  }
  if (M_tok == 0) {
    if (accumulate) return RT_OK;
    cudaError_t e = cudaMemset2DAsync(out, ldo * osz, 0, K * osz, N, s);
    return e == cudaSuccess ? RT_OK : fail(RT_ERR_CUDA, "grad_weight memset: %s", cudaGetErrorString(e));
  }
  const bool tma_ok = aligned16(g) && aligned16(x) && (ldg * 2) % 16 == 0 && (ldx * 2) % 16 == 0 &&
                      N <= INT32_MAX / 2 && K <= INT32_MAX / 2 && M_tok <= INT32_MAX / 2;
  if (tma_ok) {
    int sms = 0;
    int rc = rt_sm_count(&sms);
    if (rc) return rc;
    GemmArgs args{};
    args.M = static_cast<int>(N), args.N = static_cast<int>(K), args.K = static_cast<int>(M_tok);
    args.out = out, args.ldo = ldo, args.out_dtype = out_dtype, args.accumulate = accumulate;
    args.addend = addend, args.ld_add = ld_add;
    args.vec_store = aligned16(out) && (ldo * static_cast<int64_t>(osz)) % 16 == 0;
    const int splits =
        workspace == nullptr ? 1 : gw_splits(M_tok, N, K, sms, workspace_bytes);
    args.splits = splits;
    if (splits > 1) {
      args.epi = EPI_SPLIT;
      args.workspace = static_cast<float *>(workspace);
    } else {
      args.epi = out_dtype == RT_F32 ? EPI_F32_STORE : EPI_BF16_STORE;
    }
    // A = gᵀ: (N × M_tok) with N contiguous (MN-major); B = x: (K × M_tok) with K contiguous.
    Operand A{g, true, ldg, N, M_tok};
    Operand B{x, true, ldx, K, M_tok};
    if (splits == 1 && pair_enabled() && N > 128 && M_tok >= 1024)
      return launch_umma<__nv_bfloat16, true, true, 256, 6, 8, 2>(A, B, args, s);
    rc = launch_umma<__nv_bfloat16, true, true, GW_BN, 4>(A, B, args, s);
    if (rc || splits == 1) return rc;
    // the partial tiles, summed in split order into the output
    const int64_t work = N * ((K + 3) / 4);
    int64_t blocks = (work + 255) / 256;
    if (blocks > static_cast<int64_t>(sms) * 8) blocks = static_cast<int64_t>(sms) * 8;
    const int tiles_m = static_cast<int>((N + 127) / 128);
    const int tiles_n = static_cast<int>((K + GW_BN - 1) / GW_BN);
    launch_k(splitk_reduce_kernel<GW_BN>, static_cast<unsigned>(blocks), 256, 0, s, 
        static_cast<const float *>(workspace), splits, tiles_m, tiles_n, static_cast<int>(N),
        static_cast<int>(K), out, out_dtype, ldo, accumulate, args.vec_store, addend, ld_add);
    return check_launch("splitk_reduce_kernel");
  }
  const dim3 block(32, 8);
  const dim3 grid(static_cast<unsigned>((K + 31) / 32), static_cast<unsigned>((N + 7) / 8));
  launch_k(simt_gradw_kernel, grid, block, 0, s, static_cast<const uint16_t *>(g), ldg,
           static_cast<const uint16_t *>(x), ldx, out, out_dtype, ldo, M_tok, N, K, accumulate,
           addend, ld_add);
  return check_launch("simt_gradw_kernel");
}
}  // namespace rt

extern "C" int rt_grad_weight_bf16(const void *g, int64_t ldg, const void *x, int64_t ldx,
                                   void *out, int out_dtype, int64_t ldo, int64_t M_tok, int64_t N,
                                   int64_t K, int accumulate, void *workspace,
                                   int64_t workspace_bytes, void *stream) {
  return grad_weight_impl(g, ldg, x, ldx, out, out_dtype, ldo, M_tok, N, K, accumulate, nullptr, 0,
                          workspace, workspace_bytes, stream);
}

extern "C" int rt_grad_weight_bf16_add(const void *g, int64_t ldg, const void *x, int64_t ldx,
                                       const float *addend, int64_t ld_addend, void *out,
                                       int out_dtype, int64_t ldo, int64_t M_tok, int64_t N,
                                       int64_t K, void *workspace, int64_t workspace_bytes,
                                       void *stream) {
  if (addend == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "grad_weight_add: null addend");
  return grad_weight_impl(g, ldg, x, ldx, out, out_dtype, ldo, M_tok, N, K, 0, addend, ld_addend,
                          workspace, workspace_bytes, stream);
}

extern "C" int64_t rt_grad_weight_update_workspace_bytes(int64_t M_tok, int64_t N, int64_t K) {
  int sms = 0;
  if (rt_sm_count(&sms) != RT_OK || M_tok <= 0 || N <= 0 || K <= 0) return 0;
  const int s = gw_splits(M_tok, N, K, sms, INT64_MAX / 4);
  return static_cast<int64_t>(s < 1 ? 1 : s) * gw_tiles(N, K) * GW_TILE_BYTES;
}

// grad_W = gᵀ·x (bf16 operands, fp32 accumulation) straight into the ratchet update: the GEMM
// writes its fp32 partial tiles (one split or more) to the workspace and the update kernel sums
// them in split order as it reads each row -- the values the split-K reduce would store, without
// storing them, and without its launch.
extern "C" int rt_grad_weight_ratchet_update(
    const void *g, int64_t ldg, const void *x, int64_t ldx, int64_t M_tok, int64_t rows,
    int64_t cols, void *workspace, int64_t workspace_bytes, uint8_t *packed, int64_t ldp,
    int8_t *code_out, int64_t ldc, float *rms_ema, double ema_beta, int max_code, int threshold,
    double bucket_low, double bucket_high, double eps, int64_t *counts, float *row_rms,
    float *rms_sum, float *grad_scale, void *stream) {
  if (int rc = ratchet_update_check(rows, cols, max_code, threshold, bucket_low, bucket_high))
    return rc;
  if (M_tok < 0) return fail(RT_ERR_INVALID_ARGUMENT, "rt_grad_weight_ratchet_update: shape");
  if (rows == 0) return RT_OK;
  if (g == nullptr || x == nullptr || packed == nullptr || workspace == nullptr)
    return fail(RT_ERR_INVALID_ARGUMENT, "rt_grad_weight_ratchet_update: null pointer");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(RT_ERR_ALIGNMENT, "rt_grad_weight_ratchet_update: workspace must be 256-byte aligned");
  const bool tma_ok = M_tok > 0 && aligned16(g) && aligned16(x) && (ldg * 2) % 16 == 0 &&
                      (ldx * 2) % 16 == 0 && rows <= INT32_MAX / 2 && cols <= INT32_MAX / 2 &&
                      M_tok <= INT32_MAX / 2 && cols % 8 == 0;
  if (!tma_ok)
    return fail(RT_ERR_UNSUPPORTED, "rt_grad_weight_ratchet_update: operands need 16-byte rows");
  int sms = 0;
  if (int rc = rt_sm_count(&sms)) return rc;
  int splits = gw_splits(M_tok, rows, cols, sms, workspace_bytes);
  if (splits < 1) splits = 1;
  const int64_t tiles = gw_tiles(rows, cols);
  if (workspace_bytes < splits * tiles * GW_TILE_BYTES)
    return fail(RT_ERR_UNSUPPORTED, "rt_grad_weight_ratchet_update: workspace too small");
  cudaStream_t s = as_stream(stream);
  GemmArgs args{};
  args.M = static_cast<int>(rows), args.N = static_cast<int>(cols), args.K = static_cast<int>(M_tok);
  args.out_dtype = RT_F32, args.splits = splits, args.epi = EPI_SPLIT;
  args.workspace = static_cast<float *>(workspace);
  Operand A{g, true, ldg, rows, M_tok};
  Operand B{x, true, ldx, cols, M_tok};
  if (int rc = launch_umma<__nv_bfloat16, true, true, GW_BN, 4>(A, B, args, s)) return rc;
  UpdateArgs a = update_args(nullptr, RT_F32, 1, 0, rows, cols, packed, ldp, code_out, ldc, 1,
                             rms_ema, ema_beta, max_code, threshold, bucket_low, bucket_high, eps,
                             counts, row_rms, rms_sum, grad_scale);
  a.ws = static_cast<const float *>(workspace);
  a.ws_splits = static_cast<int>(splits > (M_tok + 63) / 64 ? (M_tok + 63) / 64 : splits);
  a.ws_tiles_n = static_cast<int>((cols + GW_BN - 1) / GW_BN);
  a.ws_bn = GW_BN;
  a.ws_split_stride = tiles * 128 * GW_BN;
  return ratchet_update_launch(a, s);
}

// ---------------------------------------------------------------------------------------------
// rt_grad_weight_bf16 without a caller-provided workspace: the split-K partial tiles live in a
// fixed device array of this library.  Nothing is allocated per call.
namespace rt {
// Split-K never needs more than SMs x 128 KiB of partial tiles (gw_splits caps splits x tiles at
// the SM count): 20 MiB covers every part with up to 160 SMs (B200: 148 -> 18.5 MiB at most),
// so the size check in rt_grad_weight_bf16_noalloc only rejects shapes on larger parts.
constexpr int64_t kGwScratchBytes = int64_t(20) << 20;
static_assert(kGwScratchBytes >= int64_t(148) * GW_TILE_BYTES, "scratch below B200's split-K need");
static __device__ __align__(256) uint8_t g_gw_scratch[kGwScratchBytes];

using CtxGetCurrentFn = CUresult (*)(CUcontext *);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long *);

// Unique id of the CUDA context current on this thread (0 when none is current).  Ids are never
// reused within a process, so a context created after a cudaDeviceReset, or another context an
// FFI host makes current on the same device, gets a fresh one.
static int current_context_id(unsigned long long *id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (get_current == nullptr || get_id == nullptr)
    return fail(RT_ERR_CUDA, "grad_weight_noalloc: cuCtxGetCurrent/cuCtxGetId are unavailable");
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS)
    return fail(RT_ERR_CUDA, "grad_weight_noalloc: cuCtxGetCurrent failed");
  *id = 0;
  if (ctx != nullptr && get_id(ctx, id) != CUDA_SUCCESS)
    return fail(RT_ERR_CUDA, "grad_weight_noalloc: cuCtxGetId failed");
  return RT_OK;
}

// Address of g_gw_scratch in the context current on this thread.  The symbol's address belongs
// to one context (the module is loaded once per context), so it is looked up once per context
// -- the first call with that context current -- and cached under the context's unique id.
static int gw_scratch_address(void **out) {
  constexpr int kEntries = 64;
  static std::mutex mu;
  static unsigned long long ids[kEntries] = {};
  static void *addrs[kEntries] = {};
  static int next = 0;
  unsigned long long id = 0;
  if (int rc = current_context_id(&id)) return rc;
  std::lock_guard<std::mutex> lock(mu);
  if (id != 0)
    for (int i = 0; i < kEntries; ++i)
      if (ids[i] == id) {
        *out = addrs[i];
        return RT_OK;
      }
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_gw_scratch);  // initialises the context if needed
  if (e != cudaSuccess || p == nullptr)
    return fail(RT_ERR_CUDA, "grad_weight_noalloc: scratch address lookup failed: %s",
                cudaGetErrorString(e));
  if (id == 0 && (current_context_id(&id) != RT_OK || id == 0)) {
    *out = p;  // no id to key it under: use it for this call only
    return RT_OK;
  }
  ids[next] = id;
  addrs[next] = p;
  next = (next + 1) % kEntries;
  *out = p;
  return RT_OK;
}
}  // namespace rt

extern "C" int rt_grad_weight_bf16_noalloc(const void *g, int64_t ldg, const void *x, int64_t ldx,
                                           void *out, int out_dtype, int64_t ldo, int64_t M_tok,
                                           int64_t N, int64_t K, int accumulate, void *stream) {
  if (M_tok <= 0 || N <= 0 || K <= 0)  // nothing to split: the plain path handles it
    return rt_grad_weight_bf16(g, ldg, x, ldx, out, out_dtype, ldo, M_tok, N, K, accumulate,
                               nullptr, 0, stream);
  const int64_t need = rt_grad_weight_workspace_bytes(M_tok, N, K);
  if (need > kGwScratchBytes)
    return fail(RT_ERR_UNSUPPORTED,
                "grad_weight_noalloc: this shape needs %lld bytes of scratch, the static scratch "
                "holds %lld",
                static_cast<long long>(need), static_cast<long long>(kGwScratchBytes));
  void *scratch = nullptr;
  if (need > 0) {
    int rc = gw_scratch_address(&scratch);
    if (rc) return rc;
    // nothing in the scratch needs to start at zero: every partial tile is written before it
    // is read, within the call
  }
  return rt_grad_weight_bf16(g, ldg, x, ldx, out, out_dtype, ldo, M_tok, N, K, accumulate, scratch,
                             need, stream);
}
