// Linear layers: C = epi(A . W^T + bias).
//
// bf16 and int8 operands run on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM, operands staged by TMA with 128-byte
// swizzle); f32 operands run on a SIMT kernel (the f32 compute precision,
// whose parity bar is 1e-4 and which tf32 tensor cores would not meet).
//
// tcgen05 kernel structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: A tile [128 x 128 B] + W tile [BN x 128 B] per stage
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2..   epilogue (kEpiWarps, an equal number per TMEM lane quarter,
//               each on a share of the tile's columns): tcgen05.ld of the
//               accumulator, dequant / bias / activation / residual,
//               coalesced global stores through a per-warp shared buffer
// The accumulator is double-buffered in TMEM (2 x BN columns), so the
// epilogue of tile i overlaps the main loop of tile i+1.  The epilogue is
// latency-bound, so it loads what it can one step ahead: the next tile's
// bias / weight scales / token scales during the current tile, and each
// unit's residual rows during the previous unit.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>

#include "jb_common.cuh"
#include "jb_internal.h"

namespace jb {
namespace {

constexpr int kBM = 128;
constexpr int kRowBytes = 128;   // one 128-byte swizzle row of K per stage
#ifndef JB_EPI_WARPS
#define JB_EPI_WARPS 8
#endif
#ifndef JB_EPI_UNIT_COLS
#define JB_EPI_UNIT_COLS 32
#endif
constexpr int kEpiWarps = JB_EPI_WARPS;  // kEpiWarps / 4 per TMEM lane quarter
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kGemmThreads = 64 + kEpiThreads;  // TMA warp + MMA warp + epilogue
constexpr int kEpiBarrier = 1;   // named barrier among the epilogue warps

// MAXST caps the operand stages: the int8 linears with short K (one tile's
// main loop is 6-8 stages of 128 K-bytes) measured 3-5% faster with three
// stages than with four (the shared memory left over goes to L1).
template <int BN, int MAXST = 8>
struct TcCfg {
  static constexpr int A_BYTES = kBM * kRowBytes;
  static constexpr int B_BYTES = BN * kRowBytes;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  // per accumulator buffer: bias[BN] and weight scale[BN] of the tile, f32
  static constexpr int PARAM_BYTES = 2 * 2 * BN * 4;
  // one 32-row bf16 output unit per epilogue warp
  static constexpr int CHUNK_BYTES = kEpiWarps * 32 * JB_EPI_UNIT_COLS * 2;
  // as many operand stages (at most 8) as fit in 227 KB beside the rest
  static constexpr int STAGES_FIT =
      (232448 - PARAM_BYTES - CHUNK_BYTES - (8 * (2 * 8 + 4) + 16) - 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > MAXST ? MAXST : STAGES_FIT;
  static constexpr int BAR_BYTES = 8 * (2 * STAGES + 4) + 16;
  static constexpr int SMEM = STAGES * STAGE_BYTES + PARAM_BYTES + CHUNK_BYTES + BAR_BYTES + 1024;
};

struct EpiParams {
  void* C;
  int ldc;
  int c_dtype;
  int epi;
  const float* bias;
  const void* resid;
  int ldr;
  const float* a_scale;
  const float* w_scale;
  int M;
  const int* dM;
  int N;
  int K;
  int* err;
  unsigned int* row_max;
  int h16;  // 16-bit operands, output and residual are f16 (else bf16)
};

// SIMT path: CUDA's erff / expf.
__device__ __forceinline__ float apply_epi(float v, int epi) {
  if (epi == JB_EPI_GELU) return gelu_erf(v);
  if (epi == JB_EPI_QUICK_GELU) return quick_gelu(v);
  return v;
}

// Named barrier over the epilogue warps that also ANDs a predicate across them.
__device__ __forceinline__ bool epi_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "n"(kEpiBarrier), "n"(kEpiThreads)
      : "memory");
  return r != 0;
}

// ── coalesced bf16 epilogue ─────────────────────────────────────────────────
// The epilogue works in units of 32 rows x kUnitCols columns (one tcgen05.ld
// 32x32b).  Each epilogue warp owns a shared buffer holding one unit in bf16
// (32 rows of kSlots 16-byte slots).  Slot q of row r lives at
// r*kUnitCols*2 + ((q ^ ((r >> kSwzShift) & (kSlots-1)))*16): both the
// row-per-thread pattern (thread r touches row r) and the coalesced pattern
// (lane l touches row kRowsPerIns*i + l/kSlots, slot l%kSlots, so each row's
// segment is whole sectors) are free of bank conflicts.
constexpr int kUnitCols = JB_EPI_UNIT_COLS;
static_assert(kUnitCols == 16 || kUnitCols == 32, "unit of 16 or 32 columns");
constexpr int kSlots = kUnitCols / 8;
constexpr int kRowsPerIns = 32 / kSlots;
constexpr int kSwzShift = kSlots == 4 ? 1 : 2;
constexpr int kUnitBytes = 32 * kUnitCols * 2;
__device__ __forceinline__ uint32_t unit_slot(uint32_t buf, int row, int q) {
  return buf + row * (kUnitCols * 2) + ((q ^ ((row >> kSwzShift) & (kSlots - 1))) << 4);
}
// Two f32 values as one 16-bit pair (f16 or bf16), and back.
__device__ __forceinline__ uint32_t pack16(float lo, float hi, bool h16) {
  if (h16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}
__device__ __forceinline__ float2 unpack16(uint32_t w, bool h16) {
  if (h16) return __half22float2(*reinterpret_cast<const __half2*>(&w));
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
template <int W>
__device__ __forceinline__ void tmem_ld_unit(uint32_t taddr, uint32_t (&r)[W]) {
  if constexpr (W == 16) tmem_ld_32x32b_x16(taddr, r);
  else tmem_ld_32x32b_x32(taddr, r);
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(a)
               : "memory");
  return v;
}

// Residual rows of one unit in the coalesced pattern (lane l holds row
// row0 + kRowsPerIns*i + l/kSlots, 16-byte slot l%kSlots); rows >= M read
// as zero.
__device__ __forceinline__ void load_resid_unit(const EpiParams& p, int row0, int lane, int M,
                                                int col0, uint4 (&rres)[kSlots]) {
#pragma unroll
  for (int i = 0; i < kSlots; ++i) {
    const int rr = row0 + i * kRowsPerIns + lane / kSlots;
    rres[i] = make_uint4(0, 0, 0, 0);
    if (rr < M)
      rres[i] = __ldg(reinterpret_cast<const uint4*>(static_cast<const bf16*>(p.resid) +
                                                      static_cast<size_t>(rr) * p.ldr + col0 +
                                                      (lane % kSlots) * 8));
  }
}

// Accumulator -> f32 value before the activation: int8 dequantisation
// (per-token x per-channel scale) or the f32 accumulator, plus bias.
template <bool S8, int W>
__device__ __forceinline__ void dequant_bias(const uint32_t (&r)[W], const float* sb,
                                             const float* ss, float as, float (&v)[W]) {
#pragma unroll
  for (int j = 0; j < W; j += 4) {
    const float4 b = *reinterpret_cast<const float4*>(sb + j);
    // packed f32x2 arithmetic: one instruction per two columns
    if constexpr (S8) {
      const float4 s = *reinterpret_cast<const float4*>(ss + j);
      const float2 s01 = __fmul2_rn(f2(as), make_float2(s.x, s.y));
      const float2 s23 = __fmul2_rn(f2(as), make_float2(s.z, s.w));
      const float2 v01 = __ffma2_rn(make_float2(__int2float_rn(static_cast<int>(r[j + 0])),
                                                __int2float_rn(static_cast<int>(r[j + 1]))),
                                    s01, make_float2(b.x, b.y));
      const float2 v23 = __ffma2_rn(make_float2(__int2float_rn(static_cast<int>(r[j + 2])),
                                                __int2float_rn(static_cast<int>(r[j + 3]))),
                                    s23, make_float2(b.z, b.w));
      v[j + 0] = v01.x; v[j + 1] = v01.y; v[j + 2] = v23.x; v[j + 3] = v23.y;
    } else {
      const float2 v01 = __fadd2_rn(make_float2(__uint_as_float(r[j + 0]), __uint_as_float(r[j + 1])),
                                    make_float2(b.x, b.y));
      const float2 v23 = __fadd2_rn(make_float2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])),
                                    make_float2(b.z, b.w));
      v[j + 0] = v01.x; v[j + 1] = v01.y; v[j + 2] = v23.x; v[j + 3] = v23.y;
    }
  }
}
template <int W>
__device__ __forceinline__ void activation(int epi, float (&v)[W]) {
  if (epi == JB_EPI_GELU) {
#pragma unroll
    for (int j = 0; j < W; j += 2) {
      const float2 g = gelu_tc2(make_float2(v[j], v[j + 1]));
      v[j] = g.x;
      v[j + 1] = g.y;
    }
  } else if (epi == JB_EPI_QUICK_GELU) {
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = quick_gelu_tc(v[j]);
  }
}

// One unit of a bf16 output whose columns all lie inside N: rows row0 ..
// row0+31 (thread `lane` owns row0+lane).  The residual (loaded ahead by the
// caller with load_resid_unit) moves through `buf` so that its global reads
// are whole row segments; the output is laid out in `buf` in the tensor
// map's swizzled box layout and written by one TMA store (rows past the
// map's extent are not written).
template <bool S8, bool H16>
__device__ __forceinline__ void epi_unit_bf16(const EpiParams& p, const CUtensorMap* tmC, int row0,
                                              int lane, int col0, const uint32_t (&r)[kUnitCols],
                                              const float* sb, const float* ss, float as,
                                              uint32_t buf, const uint4 (&rres)[kSlots], float& vmax) {
  float v[kUnitCols];
  dequant_bias<S8, kUnitCols>(r, sb, ss, as, v);
  activation<kUnitCols>(p.epi, v);
  // the previous unit's store must have read the buffer before it is reused
  if (lane == 0) bulk_wait_read_all();
  __syncwarp();
  if (p.epi == JB_EPI_RESIDUAL) {
#pragma unroll
    for (int i = 0; i < kSlots; ++i)
      sts128(unit_slot(buf, i * kRowsPerIns + lane / kSlots, lane % kSlots), rres[i]);
    __syncwarp();
    // Thread `lane` reads, then overwrites below, only row `lane`'s slots.
#pragma unroll
    for (int q = 0; q < kSlots; ++q) {
      const uint4 raw = lds128(unit_slot(buf, lane, q));
      const uint32_t w4[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack16(w4[e], H16);
        v[8 * q + 2 * e] += f.x;
        v[8 * q + 2 * e + 1] += f.y;
      }
    }
  }
  if (p.row_max) {  // the largest value before bf16 rounding rounds to the largest stored one
#pragma unroll
    for (int j = 0; j < kUnitCols; ++j) vmax = fmaxf(vmax, v[j]);
  }
#pragma unroll
  for (int q = 0; q < kSlots; ++q) {
    uint4 out;
    out.x = pack16(v[8 * q + 0], v[8 * q + 1], H16);
    out.y = pack16(v[8 * q + 2], v[8 * q + 3], H16);
    out.z = pack16(v[8 * q + 4], v[8 * q + 5], H16);
    out.w = pack16(v[8 * q + 6], v[8 * q + 7], H16);
    sts128(unit_slot(buf, lane, q), out);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmC, buf, col0, row0);
    bulk_commit();
  }
}

// One row's kUnitCols accumulator columns -> stored outputs, for every case
// the coalesced bf16 unit does not take: s32 (raw accumulator) and f32
// outputs, and bf16 units that cross N.  sb / ss are the tile's staged bias
// and weight scales for these columns (zero past N).
template <bool S8>
__device__ __forceinline__ void epi_unit(const EpiParams& p, int row, int col0,
                                         const uint32_t (&r)[kUnitCols], const float* sb,
                                         const float* ss, float as, float& vmax) {
  constexpr int W = kUnitCols;
  const int ncols = min(W, p.N - col0);
  const bool full = ncols == W;
  const size_t off = static_cast<size_t>(row) * p.ldc + col0;
  if (p.c_dtype == JB_DT_S32) {
    int* c = static_cast<int*>(p.C) + off;
    if (full) {
#pragma unroll
      for (int j = 0; j < W; j += 4)
        *reinterpret_cast<int4*>(c + j) = make_int4(r[j], r[j + 1], r[j + 2], r[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (j < ncols) c[j] = static_cast<int>(r[j]);
    }
    return;
  }
  float v[W];
  dequant_bias<S8, W>(r, sb, ss, as, v);
  activation<W>(p.epi, v);
  const size_t roff = static_cast<size_t>(row) * p.ldr + col0;
  if (p.c_dtype == JB_DT_BF16) {
    bf16* c = static_cast<bf16*>(p.C) + off;
    const bf16* rs = static_cast<const bf16*>(p.resid) + roff;
#pragma unroll
    for (int j = 0; j < W; ++j) {
      if (j < ncols) {
        float x = v[j];
        if (p.epi == JB_EPI_RESIDUAL) x += __bfloat162float(rs[j]);
        vmax = fmaxf(vmax, x);
        c[j] = __float2bfloat16_rn(x);
      }
    }
  } else if (p.c_dtype == JB_DT_F16) {
    f16* c = static_cast<f16*>(p.C) + off;
    const f16* rs = static_cast<const f16*>(p.resid) + roff;
#pragma unroll
    for (int j = 0; j < W; ++j) {
      if (j < ncols) {
        float x = v[j];
        if (p.epi == JB_EPI_RESIDUAL) x += __half2float(rs[j]);
        c[j] = __float2half_rn(x);
      }
    }
  } else {  // f32 output
    float* c = static_cast<float*>(p.C) + off;
    const float* rs = static_cast<const float*>(p.resid) + roff;
    if (full) {
#pragma unroll
      for (int j = 0; j < W; j += 4) {
        float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        if (p.epi == JB_EPI_RESIDUAL) {
          const float4 q = *reinterpret_cast<const float4*>(rs + j);
          o.x += q.x; o.y += q.y; o.z += q.z; o.w += q.w;
        }
        *reinterpret_cast<float4*>(c + j) = o;
      }
    } else {
#pragma unroll
      for (int j = 0; j < W; ++j)
        if (j < ncols) c[j] = v[j] + (p.epi == JB_EPI_RESIDUAL ? rs[j] : 0.f);
    }
  }
}

// H16: 16-bit operands / output / residual are f16 (bf16 otherwise; int8
// operands always write bf16).
template <bool S8, int BN, int MAXST, bool H16 = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const EpiParams p) {
  using Cfg = TcCfg<BN, MAXST>;
  constexpr int kElemsPerRow = S8 ? 128 : 64;  // K elements per 128-byte row
  constexpr int kSteps = 4;                    // 32-byte MMA K steps per row
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  // layout: [stages][A | B] | params [2][bias BN | scale BN] | epilogue chunks |
  //         barriers | tmem slot | abort flag
  float* params = reinterpret_cast<float*>(gbase + Cfg::STAGES * Cfg::STAGE_BYTES);
  const uint32_t chunks = base + Cfg::STAGES * Cfg::STAGE_BYTES + Cfg::PARAM_BYTES;
  const uint32_t bars = chunks + Cfg::CHUNK_BYTES;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (Cfg::STAGES + s); };
  auto tfull_bar = [&](int i) { return bars + 8u * (2 * Cfg::STAGES + i); };
  auto tempty_bar = [&](int i) { return bars + 8u * (2 * Cfg::STAGES + 2 + i); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + Cfg::STAGES * Cfg::STAGE_BYTES +
                                                    Cfg::PARAM_BYTES + Cfg::CHUNK_BYTES +
                                                    8 * (2 * Cfg::STAGES + 4));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = p.dM ? min(*p.dM, p.M) : p.M;
  const int m_tiles = (M + kBM - 1) / kBM;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int total = m_tiles * n_tiles;
  const int kb_count = (p.K + kElemsPerRow - 1) / kElemsPerRow;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(tfull_bar(i), 1);
      mbar_init(tempty_bar(i), kEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    if (p.c_dtype == JB_DT_BF16 || p.c_dtype == JB_DT_F16) prefetch_tensormap(&tmC);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && kb_count > 0) {
      int stage = 0;
      uint32_t ph = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const int mb = t / n_tiles, nb = t % n_tiles;
        bool ok = true;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(empty_bar(stage), ph ^ 1u, abort_flag)) { ok = false; break; }
          const uint32_t sa = base + stage * Cfg::STAGE_BYTES;
          mbar_arrive_expect_tx(full_bar(stage), Cfg::STAGE_BYTES);
          tma_load_2d(sa, &tmA, kb * kElemsPerRow, mb * kBM, full_bar(stage));
          tma_load_2d(sa + Cfg::A_BYTES, &tmB, kb * kElemsPerRow, nb * BN, full_bar(stage));
          if (++stage == Cfg::STAGES) { stage = 0; ph ^= 1u; }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && kb_count > 0) {
      constexpr uint32_t idesc = S8 ? idesc_s8_s32(kBM, BN)
                                    : (H16 ? idesc_f16_f32(kBM, BN) : idesc_bf16_f32(kBM, BN));
      int stage = 0;
      uint32_t ph = 0;
      int acc = 0;
      uint32_t acc_ph = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        if (!mbar_wait(tempty_bar(acc), acc_ph ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < kb_count; ++kb) {
          if (!mbar_wait(full_bar(stage), ph, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = base + stage * Cfg::STAGE_BYTES;
#pragma unroll
          for (int k = 0; k < kSteps; ++k) {
            const uint64_t ad = umma_desc_sw128(sa + 32u * k);
            const uint64_t bd = umma_desc_sw128(sa + Cfg::A_BYTES + 32u * k);
            if constexpr (S8)
              mma_s8(d_tmem, ad, bd, idesc, (kb | k) != 0);
            else
              mma_bf16(d_tmem, ad, bd, idesc, (kb | k) != 0);
          }
          mma_commit(empty_bar(stage));
          if (++stage == Cfg::STAGES) { stage = 0; ph ^= 1u; }
        }
        if (!ok) break;
        mma_commit(tfull_bar(acc));
        acc ^= 1;
        if (acc == 0) acc_ph ^= 1u;
      }
    }
  } else {
    // Epilogue warps 2..(1 + kEpiWarps).  Warp w may read TMEM lanes
    // 32*(w%4)..+31; the kEpiWarps/4 warps of a lane quarter take an equal
    // share of the tile's columns each.
    const int quarter = warp & 3;
    const int etid = threadIdx.x - 64;
    const int part = (warp - 2) >> 2;
    constexpr int kPartCols = BN / (kEpiWarps / 4);
    const uint32_t my_buf = chunks + static_cast<uint32_t>(etid >> 5) * kUnitBytes;
    const bool fast_out = p.c_dtype == JB_DT_BF16 || p.c_dtype == JB_DT_F16;
    const bool res_ahead = fast_out && p.epi == JB_EPI_RESIDUAL;
    // Per-column parameters of a tile: thread etid < BN owns column etid.
    auto load_params = [&](int t, float& b, float& sc) {
      const int col = (t % n_tiles) * BN + etid;
      const bool in = etid < BN && col < p.N;
      b = (in && p.bias) ? __ldg(p.bias + col) : 0.f;
      sc = (S8 && in && p.w_scale) ? __ldg(p.w_scale + col) : 0.f;
    };
    auto load_ascale = [&](int t) {
      const int row = (t / n_tiles) * kBM + quarter * 32 + lane;
      return (S8 && p.a_scale && row < M) ? __ldg(p.a_scale + row) : 0.f;
    };
    auto stage_params = [&](int buf, float b, float sc) {
      if (etid < BN) {
        params[buf * 2 * BN + etid] = b;
        params[buf * 2 * BN + BN + etid] = sc;
      }
    };
    int acc = 0;
    uint32_t acc_ph = 0;
    float as = 0.f;
    if (blockIdx.x < total && kb_count > 0) {
      float b, sc;
      load_params(blockIdx.x, b, sc);
      stage_params(0, b, sc);  // ordered by the first tile's barrier
      as = load_ascale(blockIdx.x);
    }
    for (int t = blockIdx.x; t < total && kb_count > 0; t += gridDim.x) {
      const int mb = t / n_tiles, nb = t % n_tiles;
      const int t_next = t + gridDim.x;
      // The next tile's parameters are loaded now and staged into the other
      // buffer after this tile, ordered by the next tile's barrier.
      float nb_b = 0.f, nb_s = 0.f, as_next = 0.f;
      if (t_next < total) {
        load_params(t_next, nb_b, nb_s);
        as_next = load_ascale(t_next);
      }
      const float* pb = params + acc * 2 * BN;
      const float* ps = pb + BN;
      const int row0 = mb * kBM + quarter * 32;
      const int c_begin = part * kPartCols, c_end = c_begin + kPartCols;
      auto fast = [&](int c) { return fast_out && nb * BN + c + kUnitCols <= p.N; };  // warp-uniform
      uint4 rres[kSlots] = {};
      if (res_ahead && fast(c_begin)) load_resid_unit(p, row0, lane, M, nb * BN + c_begin, rres);
      // One barrier orders the staged parameters and makes the
      // accumulator-ready decision the same for every epilogue warp (so none
      // can be left waiting at a later barrier after an abort).
      const bool ok = epi_bar_and(mbar_wait(tfull_bar(acc), acc_ph, abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      float vmax = 0.f;  // this thread's row: largest output of its columns (row_max)
#pragma unroll 1
      for (int c = c_begin; c < c_end; c += kUnitCols) {
        const int col0 = nb * BN + c;
        if (col0 >= p.N) break;  // warp-uniform
        uint32_t r[kUnitCols];
        tmem_ld_unit(tbase + c, r);
        // the next unit's residual rows load while this unit computes
        uint4 rnext[kSlots] = {};
        if (res_ahead && c + kUnitCols < c_end && fast(c + kUnitCols))
          load_resid_unit(p, row0, lane, M, col0 + kUnitCols, rnext);
        tmem_wait_ld();
        if (fast(c))
          epi_unit_bf16<S8, H16>(p, &tmC, row0, lane, col0, r, pb + c, ps + c, as, my_buf, rres, vmax);
        else if (row0 + lane < M)
          epi_unit<S8>(p, row0 + lane, col0, r, pb + c, ps + c, as, vmax);
#pragma unroll
        for (int i = 0; i < kSlots; ++i) rres[i] = rnext[i];
      }
      if (p.row_max && vmax > 0.f && row0 + lane < M)
        atomicMax(p.row_max + row0 + lane, __float_as_uint(__bfloat162float(__float2bfloat16_rn(vmax))));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      stage_params(acc ^ 1, nb_b, nb_s);
      as = as_next;
      acc ^= 1;
      if (acc == 0) acc_ph ^= 1u;
    }
    if (lane == 0) bulk_wait_all();  // this warp's output stores are complete
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag && p.err) atomicOr(p.err, kErrTimeout);
}

// ── f32 SIMT kernel ─────────────────────────────────────────────────────────
constexpr int kSimtTile = 64;
constexpr int kSimtK = 16;

__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A,
                                                       const float* __restrict__ W, EpiParams p) {
  __shared__ float As[kSimtK][kSimtTile + 4];
  __shared__ float Ws[kSimtK][kSimtTile + 4];
  const int M = p.dM ? min(*p.dM, p.M) : p.M;
  const int m0 = blockIdx.y * kSimtTile, n0 = blockIdx.x * kSimtTile;
  if (m0 >= M) return;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < p.K; k0 += kSimtK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = threadIdx.x + i * 256;
      const int r = idx / kSimtK, kk = idx % kSimtK;
      const int gk = k0 + kk;
      As[kk][r] = (m0 + r < M && gk < p.K) ? A[static_cast<size_t>(m0 + r) * p.K + gk] : 0.f;
      Ws[kk][r] = (n0 + r < p.N && gk < p.K) ? W[static_cast<size_t>(n0 + r) * p.K + gk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSimtK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = m0 + ty * 4 + i;
    if (row >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = n0 + tx * 4 + j;
      if (col >= p.N) continue;
      float v = acc[i][j] + (p.bias ? p.bias[col] : 0.f);
      v = apply_epi(v, p.epi);
      if (p.epi == JB_EPI_RESIDUAL) {
        const size_t ro = static_cast<size_t>(row) * p.ldr + col;
        v += (p.c_dtype == JB_DT_BF16) ? __bfloat162float(static_cast<const bf16*>(p.resid)[ro])
                                       : static_cast<const float*>(p.resid)[ro];
      }
      const size_t o = static_cast<size_t>(row) * p.ldc + col;
      if (p.c_dtype == JB_DT_BF16)
        static_cast<bf16*>(p.C)[o] = __float2bfloat16_rn(v);
      else
        static_cast<float*>(p.C)[o] = v;
    }
  }
}

// ── host side ───────────────────────────────────────────────────────────────
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 2-D K-major map over [rows, k_elems] with a (128-byte x box_rows) box.
bool make_map(CUtensorMap* map, const void* ptr, bool s8, bool h16, int rows, int k_elems,
              int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  const int esz = s8 ? 1 : 2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k_elems), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k_elems) * esz};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kRowBytes / esz), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = s8    ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : (h16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  CUresult r = enc(map, dt, 2,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Store map over a 16-bit output [rows, cols] with row stride ld elements: one
// epilogue unit (32 rows x kUnitCols columns) per box, swizzled to match
// unit_slot (64-byte rows: SWIZZLE_64B; 32-byte rows: SWIZZLE_32B).
bool make_store_map(CUtensorMap* map, void* ptr, bool h16, int rows, int cols, int ld) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kUnitCols), 32u};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, h16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   ptr, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   kUnitCols == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool S8, int BN, int MAXST = 8, bool H16 = false>
cudaError_t launch_tc(const GemmArgs& g, const EpiParams& p, cudaStream_t s, std::string* why) {
  using Cfg = TcCfg<BN, MAXST>;
  CUtensorMap ma, mb, mc;
  memset(&mc, 0, sizeof(mc));  // unused unless the output is 16-bit
  constexpr bool h16 = H16;
  if (!make_map(&ma, g.A, S8, h16, g.M, g.K, kBM) || !make_map(&mb, g.W, S8, h16, g.N, g.K, BN) ||
      ((p.c_dtype == JB_DT_BF16 || p.c_dtype == JB_DT_F16) &&
       !make_store_map(&mc, g.C, p.c_dtype == JB_DT_F16, g.M, g.N, p.ldc))) {
    if (why) *why = "cuTensorMapEncodeTiled failed (pointer alignment or shape)";
    return cudaErrorInvalidValue;
  }
  auto kern = gemm_tc_kernel<S8, BN, MAXST, H16>;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
  if (e != cudaSuccess) return e;
  const int m_tiles = (g.M + kBM - 1) / kBM;
  const int n_tiles = (g.N + BN - 1) / BN;
  const int grid = std::min(num_sms(dev), m_tiles * n_tiles);
  kern<<<grid, kGemmThreads, Cfg::SMEM, s>>>(ma, mb, mc, p);
  return cudaGetLastError();
}

}  // namespace

int num_sms(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (!cached[device]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    cached[device] = n > 0 ? n : 148;
  }
  return cached[device];
}

cudaError_t launch_gemm(const GemmArgs& g, cudaStream_t s, std::string* why) {
  if (g.M < 0 || g.N <= 0 || g.K <= 0) {
    if (why) *why = "linear: M, N, K must be positive";
    return cudaErrorInvalidValue;
  }
  if (g.M == 0) return cudaSuccess;
  EpiParams p;
  p.C = g.C;
  p.ldc = g.ldc ? g.ldc : g.N;
  p.c_dtype = g.c_dtype;
  p.epi = g.epi;
  p.bias = g.bias;
  p.resid = g.resid;
  p.ldr = g.ldr ? g.ldr : g.N;
  p.a_scale = g.a_scale;
  p.w_scale = g.w_scale;
  p.M = g.M;
  p.dM = g.dM;
  p.N = g.N;
  p.K = g.K;
  p.err = g.err;
  p.row_max = g.row_max;
  p.h16 = 0;
  if (g.epi == JB_EPI_RESIDUAL && !g.resid) {
    if (why) *why = "linear: residual epilogue without a residual tensor";
    return cudaErrorInvalidValue;
  }
  if (g.ab_dtype == JB_DT_F32) {
    if (g.c_dtype != JB_DT_F32 && g.c_dtype != JB_DT_BF16) {
      if (why) *why = "linear(f32): output must be f32 or bf16";
      return cudaErrorInvalidValue;
    }
    dim3 grid((g.N + kSimtTile - 1) / kSimtTile, (g.M + kSimtTile - 1) / kSimtTile);
    gemm_f32_kernel<<<grid, 256, 0, s>>>(static_cast<const float*>(g.A),
                                         static_cast<const float*>(g.W), p);
    return cudaGetLastError();
  }
  const bool s8 = g.ab_dtype == JB_DT_S8;
  if (!s8 && g.ab_dtype != JB_DT_BF16 && g.ab_dtype != JB_DT_F16) {
    if (why) *why = "linear: unsupported operand dtype";
    return cudaErrorInvalidValue;
  }
  // 16-bit outputs and residuals have the operands' 16-bit type (bf16 for int8)
  p.h16 = g.ab_dtype == JB_DT_F16 ? 1 : 0;
  if ((g.ab_dtype == JB_DT_F16 && g.c_dtype != JB_DT_F16 && g.c_dtype != JB_DT_F32) ||
      (g.ab_dtype != JB_DT_F16 && g.c_dtype == JB_DT_F16)) {
    if (why) *why = "linear: an f16 output needs f16 operands, and f16 operands an f16 or f32 output";
    return cudaErrorInvalidValue;
  }
  // TMA: row strides must be multiples of 16 bytes, bases 16-byte aligned.
  const int esz = s8 ? 1 : 2;
  if ((g.K * esz) % 16 != 0 || (reinterpret_cast<uintptr_t>(g.A) & 15) ||
      (reinterpret_cast<uintptr_t>(g.W) & 15)) {
    if (why) *why = "linear: K*elem_size must be a multiple of 16 and A/W 16-byte aligned";
    return cudaErrorInvalidValue;
  }
  if (s8 && g.c_dtype != JB_DT_S32 && (!g.a_scale || !g.w_scale)) {
    if (why) *why = "linear(int8): dequantised output needs a_scale and w_scale";
    return cudaErrorInvalidValue;
  }
  if (!s8 && g.c_dtype == JB_DT_S32) {
    if (why) *why = "linear(bf16): s32 output is only defined for int8 operands";
    return cudaErrorInvalidValue;
  }
  if ((p.ldc % 8) || (reinterpret_cast<uintptr_t>(g.C) & 15) ||
      (g.resid && ((p.ldr % 8) || (reinterpret_cast<uintptr_t>(g.resid) & 15)))) {
    if (why) *why = "linear: C/residual must be 16-byte aligned with row strides multiple of 8";
    return cudaErrorInvalidValue;
  }
  if (p.h16) {  // f16 operands
    if (g.N >= 512 || g.N % 256 == 0) return launch_tc<false, 256, 8, true>(g, p, s, why);
    if (g.N >= 128) return launch_tc<false, 128, 8, true>(g, p, s, why);
    return launch_tc<false, 64, 8, true>(g, p, s, why);
  }
  if (g.N >= 512 || g.N % 256 == 0) {
    if (s8 && g.K <= 1024) return launch_tc<true, 256, 3>(g, p, s, why);
    return s8 ? launch_tc<true, 256>(g, p, s, why) : launch_tc<false, 256>(g, p, s, why);
  }
  if (g.N >= 128)
    return s8 ? launch_tc<true, 128>(g, p, s, why) : launch_tc<false, 128>(g, p, s, why);
  return s8 ? launch_tc<true, 64>(g, p, s, why) : launch_tc<false, 64>(g, p, s, why);
}

}  // namespace jb
