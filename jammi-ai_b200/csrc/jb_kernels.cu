// Memory-bound kernels of the encoder forward: embeddings + LayerNorm,
// (residual +) LayerNorm with optional fused per-token int8 quantisation,
// per-row int8 quantisation, pooling + L2 normalisation, and the ViT
// patch / CLS / pooling helpers.  One warp per row with 16-byte vector
// loads; all statistics in f32.
#include <algorithm>
#include <cfloat>
#include <mutex>

#include "jb_common.cuh"
#include "jb_internal.h"

namespace jb {
namespace {

constexpr int kRowsPerBlock = 8;  // warps per 256-thread block

// 16-byte vector of T: 8 bf16 or 4 f32.
template <typename T> struct Vec;
template <> struct Vec<bf16> {
  static constexpr int N = 8;
  __device__ static void load(const bf16* p, float* v) {
    unpack(*reinterpret_cast<const uint4*>(p), v);
  }
  __device__ static void unpack(const uint4& raw, float* v) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __bfloat1622float2(h[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
  }
  __device__ static uint4 pack(const float* v) {
    uint4 raw;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    return raw;
  }
  __device__ static void store(bf16* p, const float* v) { *reinterpret_cast<uint4*>(p) = pack(v); }
  // value as it will be read back after the store (bf16 rounding)
  __device__ static float rounded(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};
template <> struct Vec<f16> {
  static constexpr int N = 8;
  __device__ static void load(const f16* p, float* v) {
    unpack(*reinterpret_cast<const uint4*>(p), v);
  }
  __device__ static void unpack(const uint4& raw, float* v) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 f = __half22float2(h[e]);
      v[2 * e] = f.x;
      v[2 * e + 1] = f.y;
    }
  }
  __device__ static uint4 pack(const float* v) {
    uint4 raw;
    __half2* h = reinterpret_cast<__half2*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
    return raw;
  }
  __device__ static void store(f16* p, const float* v) { *reinterpret_cast<uint4*>(p) = pack(v); }
  __device__ static float rounded(float x) { return __half2float(__float2half_rn(x)); }
};
template <> struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float* v) {
    float4 f = *reinterpret_cast<const float4*>(p);
    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
  }
  __device__ static void unpack(const uint4& raw, float* v) {
    v[0] = __uint_as_float(raw.x); v[1] = __uint_as_float(raw.y);
    v[2] = __uint_as_float(raw.z); v[3] = __uint_as_float(raw.w);
  }
  __device__ static uint4 pack(const float* v) {
    return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                      __float_as_uint(v[3]));
  }
  __device__ static void store(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
  __device__ static float rounded(float x) { return x; }
};

// Per-token symmetric int8 quantisation of values already rounded to the
// stored dtype: scale = amax/127, q = clamp(rint(x * (127/amax)), -127, 127).
// With |x| <= amax the product is at most 127 (1 + 2^-24), so the clamp never
// acts; rint of |y| < 2^22 is the low bits of y + 1.5 * 2^23 (the addition
// rounds to the nearest integer, ties to even), whose low byte is the int8
// code.  quant4 packs four codes with byte permutes: no conversion
// instructions.
__device__ __forceinline__ uint32_t quant4(float a, float b, float c, float d, float inv) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  // __fmul_rn / __fadd_rn: two roundings, never contracted into one fma
  // (the packed f32x2 forms are not held to that and break bit-exactness)
  const uint32_t qa = __float_as_uint(__fadd_rn(__fmul_rn(a, inv), kMagic));
  const uint32_t qb = __float_as_uint(__fadd_rn(__fmul_rn(b, inv), kMagic));
  const uint32_t qc = __float_as_uint(__fadd_rn(__fmul_rn(c, inv), kMagic));
  const uint32_t qd = __float_as_uint(__fadd_rn(__fmul_rn(d, inv), kMagic));
  return __byte_perm(__byte_perm(qa, qb, 0x0040), __byte_perm(qc, qd, 0x0040), 0x5410);
}

// Normalises the row held in v[] (nvec vectors of Vec<T>::N per lane slot),
// writes y (and optionally int8 + scale).  Called by one full warp; gamma
// and beta are read as float4 (16-byte aligned, shared or global memory).
template <typename T, int MAXV>
__device__ __forceinline__ void ln_finish(float (&v)[MAXV * Vec<T>::N], int nvec, int cols, int lane,
                                          const float* gamma, const float* beta, float eps, T* yrow,
                                          int8_t* qrow, float* scale_out) {
  constexpr int VN = Vec<T>::N;
  // sums over column pairs in packed f32x2 (two partial sums per lane)
  float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < MAXV; ++i)
    if (lane + i * 32 < nvec)
#pragma unroll
      for (int e = 0; e < VN; e += 2) s2 = __fadd2_rn(s2, make_float2(v[i * VN + e], v[i * VN + e + 1]));
  const float mean = warp_sum(s2.x + s2.y) / static_cast<float>(cols);
  float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < MAXV; ++i)
    if (lane + i * 32 < nvec)
#pragma unroll
      for (int e = 0; e < VN; e += 2) {
        const float2 d = __fadd2_rn(make_float2(v[i * VN + e], v[i * VN + e + 1]), f2(-mean));
        ss2 = __ffma2_rn(d, d, ss2);
      }
  const float var = warp_sum(ss2.x + ss2.y) / static_cast<float>(cols);
  const float rstd = 1.0f / sqrtf(var + eps);
  float amax = 0.f;
  const float nm = -mean * rstd;  // (x - mean) rstd = x rstd - mean rstd, one packed fma per pair
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = lane + i * 32;
    if (vi < nvec) {
      float o[VN];
      const float4* g4 = reinterpret_cast<const float4*>(gamma + vi * VN);
      const float4* b4 = reinterpret_cast<const float4*>(beta + vi * VN);
#pragma unroll
      for (int q = 0; q < VN / 4; ++q) {
        const float4 g = g4[q], b = b4[q];
        const float2 t01 = __ffma2_rn(make_float2(v[i * VN + 4 * q + 0], v[i * VN + 4 * q + 1]), f2(rstd), f2(nm));
        const float2 t23 = __ffma2_rn(make_float2(v[i * VN + 4 * q + 2], v[i * VN + 4 * q + 3]), f2(rstd), f2(nm));
        const float2 o01 = __ffma2_rn(t01, make_float2(g.x, g.y), make_float2(b.x, b.y));
        const float2 o23 = __ffma2_rn(t23, make_float2(g.z, g.w), make_float2(b.z, b.w));
        o[4 * q + 0] = o01.x; o[4 * q + 1] = o01.y; o[4 * q + 2] = o23.x; o[4 * q + 3] = o23.y;
      }
      // stored once; the quantiser reads the stored (rounded) values back
      // from the packed bits, not through a second conversion
      const uint4 packed = Vec<T>::pack(o);
      Vec<T>::unpack(packed, v + i * VN);
      *reinterpret_cast<uint4*>(yrow + vi * VN) = packed;
#pragma unroll
      for (int e = 0; e < VN; ++e) amax = fmaxf(amax, fabsf(v[i * VN + e]));
    }
  }
  if (qrow) {
    amax = warp_max(amax);
    const float inv = amax > 0.f ? 127.0f / amax : 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = lane + i * 32;
      if (vi < nvec) {
#pragma unroll
        for (int e = 0; e < VN / 4; ++e)
          reinterpret_cast<uint32_t*>(qrow + vi * VN)[e] =
              quant4(v[i * VN + 4 * e], v[i * VN + 4 * e + 1], v[i * VN + 4 * e + 2],
                     v[i * VN + 4 * e + 3], inv);
      }
    }
    if (lane == 0) *scale_out = amax / 127.0f;
  }
}

constexpr int kLnMaxCols = 1024;

// Stages gamma / beta (cols <= 1024 floats each) in shared memory.
__device__ __forceinline__ void stage_params(float* sg, float* sb, const float* gamma,
                                             const float* beta, int cols) {
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    sg[c] = gamma[c];
    sb[c] = beta[c];
  }
  __syncthreads();
}

// Persistent over rows: warp w of block b handles rows b*8+w, +gridDim*8, ...
template <typename T, int MAXV>
__global__ void __launch_bounds__(256) layernorm_kernel(LnArgs a) {
  constexpr int VN = Vec<T>::N;
  __shared__ __align__(16) float sg[kLnMaxCols];
  __shared__ __align__(16) float sb[kLnMaxCols];
  stage_params(sg, sb, a.gamma, a.beta, a.cols);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = a.drows ? min(*a.drows, a.rows) : a.rows;
  const int nvec = a.cols / VN;
  for (int row = blockIdx.x * kRowsPerBlock + warp; row < R; row += gridDim.x * kRowsPerBlock) {
    const T* x = static_cast<const T*>(a.x) + static_cast<size_t>(row) * a.cols;
    const T* r = a.resid ? static_cast<const T*>(a.resid) + static_cast<size_t>(row) * a.cols : nullptr;
    float v[MAXV * VN];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = lane + i * 32;
      if (vi < nvec) {
        Vec<T>::load(x + vi * VN, v + i * VN);
        if (r) {
          float t[VN];
          Vec<T>::load(r + vi * VN, t);
#pragma unroll
          for (int e = 0; e < VN; ++e) v[i * VN + e] += t[e];
        }
      }
    }
    ln_finish<T, MAXV>(v, nvec, a.cols, lane, sg, sb, a.eps,
                       static_cast<T*>(a.y) + static_cast<size_t>(row) * a.cols,
                       a.yq ? a.yq + static_cast<size_t>(row) * a.cols : nullptr,
                       a.yscale ? a.yscale + row : nullptr);
    if (a.zero_rows && lane == 0) a.zero_rows[row] = 0u;
  }
}

// 16-bit (bf16 or f16) rows of up to MAXV x 256 columns, persistent over
// rows like layernorm_kernel, but each warp loads its next row (and residual
// row) into registers before it normalises the current one, so the memory
// latency of one row overlaps the reductions and stores of the other.
template <int MAXV, bool RES, typename T = bf16>
__global__ void __launch_bounds__(256) layernorm_bf16_kernel(LnArgs a) {
  __shared__ __align__(16) float sg[kLnMaxCols];
  __shared__ __align__(16) float sb[kLnMaxCols];
  stage_params(sg, sb, a.gamma, a.beta, a.cols);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = a.drows ? min(*a.drows, a.rows) : a.rows;
  const int nvec = a.cols / 8;
  const int stride = gridDim.x * kRowsPerBlock;
  auto fetch = [&](int row, uint4 (&xr)[MAXV], uint4 (&rr)[MAXV]) {
    const uint4* x = reinterpret_cast<const uint4*>(static_cast<const T*>(a.x) +
                                                    static_cast<size_t>(row) * a.cols);
    const uint4* r = RES ? reinterpret_cast<const uint4*>(static_cast<const T*>(a.resid) +
                                                         static_cast<size_t>(row) * a.cols)
                         : nullptr;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = lane + i * 32;
      if (vi < nvec) {
        xr[i] = x[vi];
        if constexpr (RES) rr[i] = r[vi];
      }
    }
  };
  uint4 nx[MAXV], nr[MAXV];
  int row = blockIdx.x * kRowsPerBlock + warp;
  if (row < R) fetch(row, nx, nr);
  for (; row < R; row += stride) {
    float v[MAXV * 8];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (lane + i * 32 < nvec) {
        Vec<T>::unpack(nx[i], v + i * 8);
        if constexpr (RES) {
          float t[8];
          Vec<T>::unpack(nr[i], t);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[i * 8 + e] += t[e];
        }
      }
    }
    if (row + stride < R) fetch(row + stride, nx, nr);
    ln_finish<T, MAXV>(v, nvec, a.cols, lane, sg, sb, a.eps,
                       static_cast<T*>(a.y) + static_cast<size_t>(row) * a.cols,
                          a.yq ? a.yq + static_cast<size_t>(row) * a.cols : nullptr,
                          a.yscale ? a.yscale + row : nullptr);
    if (a.zero_rows && lane == 0) a.zero_rows[row] = 0u;
  }
}

// Persistent over (row b, position p) slots; padding slots are skipped.
template <typename T, int MAXV>
__global__ void __launch_bounds__(256) embed_ln_kernel(EmbedArgs a) {
  constexpr int VN = Vec<T>::N;
  __shared__ __align__(16) float sg[kLnMaxCols];
  __shared__ __align__(16) float sb[kLnMaxCols];
  if (a.gamma) stage_params(sg, sb, a.gamma, a.beta, a.H);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = a.H / VN;
  const int slots = a.batch * a.max_seq;
  for (int pos_idx = blockIdx.x * kRowsPerBlock + warp; pos_idx < slots;
       pos_idx += gridDim.x * kRowsPerBlock) {
    const int b = pos_idx / a.max_seq, p = pos_idx % a.max_seq;
    const int start = a.cu[b], len = a.cu[b + 1] - start;
    if (p >= len) continue;  // warp-uniform
    uint32_t id = a.ids[static_cast<size_t>(b) * a.max_seq + p];
    if (id >= static_cast<uint32_t>(a.vocab)) {
      if (lane == 0 && a.err) atomicOr(a.err, 2);
      id = 0;
    }
    const T* w = static_cast<const T*>(a.word) + static_cast<size_t>(id) * a.H;
    const T* pe = a.pos ? static_cast<const T*>(a.pos) + static_cast<size_t>(p) * a.H : nullptr;
    const T* te = static_cast<const T*>(a.type0);
    float v[MAXV * VN];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = lane + i * 32;
      if (vi < nvec) {
        float t1[VN], t2[VN];
        Vec<T>::load(w + vi * VN, v + i * VN);
        if (!pe) continue;  // token embedding alone (ModernBERT, modernbert.rs:331-332)
        Vec<T>::load(pe + vi * VN, t2);
        if (te) {
          Vec<T>::load(te + vi * VN, t1);
#pragma unroll
          for (int e = 0; e < VN; ++e) v[i * VN + e] = (v[i * VN + e] + t1[e]) + t2[e];
        } else {
#pragma unroll
          for (int e = 0; e < VN; ++e) v[i * VN + e] += t2[e];
        }
      }
    }
    const size_t row = static_cast<size_t>(start + p);
    T* yrow = static_cast<T*>(a.y) + row * a.H;
    if (!a.gamma) {  // token + position only (OpenCLIP text, clip_text.rs:309-312)
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int vi = lane + i * 32;
        if (vi < nvec) Vec<T>::store(yrow + vi * VN, v + i * VN);
      }
      continue;
    }
    ln_finish<T, MAXV>(v, nvec, a.H, lane, sg, sb, a.eps, yrow,
                       a.yq ? a.yq + row * a.H : nullptr, a.yscale ? a.yscale + row : nullptr);
  }
}

// The GELU quantiser is ALU-bound: it is compiled for this many resident
// 256-thread blocks per SM, trading unrolled temporaries for warps.
#ifndef JB_GELU_Q_BLOCKS
#define JB_GELU_Q_BLOCKS 3
#endif

// The value quantised for input x: x itself, or (ACT == JB_EPI_GELU) the
// GELU of x rounded to T -- what a stored activation tensor of type T holds.
template <typename T, int ACT>
__device__ __forceinline__ float pre_quant(float x) {
  if constexpr (ACT == JB_EPI_GELU) return Vec<T>::rounded(gelu_tc(x));
  else return x;
}

// One warp per row, optionally applying an activation first.  Rows of up to
// MAXV 16-byte vectors per lane are held in registers (after the
// activation), so each element is read from memory and activated once;
// MAXV == 0 is the general two-pass form for longer rows.
template <typename T, int MAXV, int ACT>
__global__ void __launch_bounds__(256, (ACT == JB_EPI_GELU ? JB_GELU_Q_BLOCKS : 1)) quantize_rows_kernel(const T* __restrict__ x, int8_t* q,
                                                            float* scale, int rows,
                                                            const int* drows, int cols) {
  constexpr int VN = Vec<T>::N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerBlock + warp;
  const int R = drows ? min(*drows, rows) : rows;
  if (row >= R) return;
  const T* xr = x + static_cast<size_t>(row) * cols;
  const int nvec = cols / VN;
  int8_t* qr = q + static_cast<size_t>(row) * cols;
  if constexpr (MAXV > 0) {
    uint4 raw[MAXV];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = lane + i * 32;
      if (vi < nvec) raw[i] = __ldg(reinterpret_cast<const uint4*>(xr + vi * VN));
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (lane + i * 32 < nvec) {
        float v[VN];
        Vec<T>::unpack(raw[i], v);
        if constexpr (ACT == JB_EPI_GELU) {
#pragma unroll
          for (int e = 0; e < VN; e += 2) {
            const float2 g = gelu_tc2(make_float2(v[e], v[e + 1]));
            v[e] = Vec<T>::rounded(g.x);
            v[e + 1] = Vec<T>::rounded(g.y);
          }
        }
#pragma unroll
        for (int e = 0; e < VN; ++e) amax = fmaxf(amax, fabsf(v[e]));
        if constexpr (ACT != JB_EPI_NONE) raw[i] = Vec<T>::pack(v);  // exact: v is T-rounded
      }
    }
    amax = warp_max(amax);
    const float inv = amax > 0.f ? 127.0f / amax : 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = lane + i * 32;
      if (vi < nvec) {
        float v[VN];
        Vec<T>::unpack(raw[i], v);
#pragma unroll
        for (int e = 0; e < VN / 4; ++e)
          reinterpret_cast<uint32_t*>(qr + vi * VN)[e] =
              quant4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3], inv);
      }
    }
    if (lane == 0) scale[row] = amax / 127.0f;
    return;
  }
  float amax = 0.f;
  for (int vi = lane; vi < nvec; vi += 32) {
    float v[VN];
    Vec<T>::load(xr + vi * VN, v);
#pragma unroll
    for (int e = 0; e < VN; ++e) amax = fmaxf(amax, fabsf(pre_quant<T, ACT>(v[e])));
  }
  amax = warp_max(amax);
  const float inv = amax > 0.f ? 127.0f / amax : 0.f;
  for (int vi = lane; vi < nvec; vi += 32) {
    float v[VN];
    Vec<T>::load(xr + vi * VN, v);
#pragma unroll
    for (int e = 0; e < VN; ++e) v[e] = pre_quant<T, ACT>(v[e]);
#pragma unroll
    for (int e = 0; e < VN / 4; ++e)
      reinterpret_cast<uint32_t*>(qr + vi * VN)[e] =
          quant4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3], inv);
  }
  if (lane == 0) scale[row] = amax / 127.0f;
}

// ── GELU by table, fused into the per-token quantiser ───────────────────────
// Every bf16 input has one correctly rounded bf16 GELU: bf16(x * Phi(x)) with
// Phi from CUDA's double-precision erf, tabulated once per device (65536
// entries, 128 KB).  The FFN2-input quantiser stages the table in shared
// memory and looks every value up: one function for every element, rising
// on the positives, so a row's largest GELU is the GELU of its largest x.
__device__ __align__(16) uint16_t g_gelu_bf16[65536];

__global__ void gelu_table_kernel() {
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= 65536) return;
  __nv_bfloat16_raw r;
  r.x = static_cast<unsigned short>(u);
  const double x = static_cast<double>(__bfloat162float(__nv_bfloat16(r)));
  const double g = 0.5 * x * (1.0 + erf(x * 0.70710678118654752440));
  const __nv_bfloat16 b = __double2bfloat16(g);
  g_gelu_bf16[u] = static_cast<__nv_bfloat16_raw>(b).x;
}

constexpr int kGeluQThreads = 512;
constexpr int kGeluTableBytes = 65536 * 2;
// A row whose largest x reaches this has amax = GELU(largest x): GELU(0.5) =
// 0.35 exceeds |GELU| anywhere on the negatives (at most 0.17, near -0.75).
constexpr float kGeluRowMaxFast = 0.5f;

// GELU of the two bf16 halves of w by lookup (table in shared memory).
__device__ __forceinline__ uint32_t gelu_lookup2(const uint16_t* tab, uint32_t w) {
  const uint32_t lo = tab[w & 0xFFFFu], hi = tab[w >> 16];
  return lo | (hi << 16);
}

// Per-token int8 of bf16(GELU(x)), x bf16 [rows, cols] (cols a multiple of
// 8): one warp per row, persistent (one 512-thread block per SM with the
// table in shared memory).  row_max[row] holds the row's largest x (f32
// bits, 0 when none is positive).  At >= kGeluRowMaxFast the row's amax is a
// single lookup and the row is read once; each lane holds its MAXV 16-byte
// vectors of the row in registers and loads those of its next row while it
// quantises the current one (rows of up to 12 vectors per lane), so a whole
// row's loads are in flight behind the lookups.  Other rows first take the
// amax over the held values.
template <int MAXV>
__global__ void __launch_bounds__(kGeluQThreads, 1)
    gelu_quantize_kernel(const bf16* __restrict__ x, const unsigned int* row_max, int8_t* q,
                         float* scale, int rows, const int* drows, int cols) {
  extern __shared__ __align__(16) uint16_t tab[];
  {
    const uint4* src = reinterpret_cast<const uint4*>(g_gelu_bf16);
    uint4* dst = reinterpret_cast<uint4*>(tab);
    for (int i = threadIdx.x; i < kGeluTableBytes / 16; i += kGeluQThreads) dst[i] = src[i];
  }
  __syncthreads();
  constexpr int kWarps = kGeluQThreads / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = drows ? min(*drows, rows) : rows;
  const int nvec = cols / 8;
  const int stride = gridDim.x * kWarps;
  auto fetch = [&](int row, uint4 (&r)[MAXV]) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * cols);
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
      if (lane + 32 * i < nvec) r[i] = __ldg(xr + lane + 32 * i);
  };
  // the next row's vectors fit beside the current ones up to 12 per lane
  constexpr bool kPrefetch = MAXV <= 12;
  uint4 cur[MAXV];
  int row = blockIdx.x * kWarps + warp;
  if (kPrefetch && row < R) fetch(row, cur);
  for (; row < R; row += stride) {
    const float xm = __uint_as_float(row_max[row]);
    uint4 nxt[kPrefetch ? MAXV : 1];
    if constexpr (kPrefetch) {
      if (row + stride < R) fetch(row + stride, nxt);
    } else {
      fetch(row, cur);
    }
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (lane + 32 * i < nvec) {
        cur[i].x = gelu_lookup2(tab, cur[i].x);
        cur[i].y = gelu_lookup2(tab, cur[i].y);
        cur[i].z = gelu_lookup2(tab, cur[i].z);
        cur[i].w = gelu_lookup2(tab, cur[i].w);
      }
    }
    float amax;
    if (xm >= kGeluRowMaxFast) {
      amax = __uint_as_float(static_cast<uint32_t>(tab[__float_as_uint(xm) >> 16]) << 16);
    } else {
      // the largest |GELU| as bf16 magnitude bits (integer order of
      // non-negative bf16 bit patterns is their numeric order)
      uint32_t mx2 = 0;
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        if (lane + 32 * i < nvec) {
          mx2 = __vmaxu2(mx2, cur[i].x & 0x7FFF7FFFu);
          mx2 = __vmaxu2(mx2, cur[i].y & 0x7FFF7FFFu);
          mx2 = __vmaxu2(mx2, cur[i].z & 0x7FFF7FFFu);
          mx2 = __vmaxu2(mx2, cur[i].w & 0x7FFF7FFFu);
        }
      }
      amax = warp_max(fmaxf(__uint_as_float(mx2 << 16), __uint_as_float(mx2 & 0xFFFF0000u)));
    }
    const float inv = amax > 0.f ? 127.0f / amax : 0.f;
    uint2* qr = reinterpret_cast<uint2*>(q + static_cast<size_t>(row) * cols);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (lane + 32 * i < nvec) {
        float v[8];
        Vec<bf16>::unpack(cur[i], v);
        qr[lane + 32 * i] = make_uint2(quant4(v[0], v[1], v[2], v[3], inv), quant4(v[4], v[5], v[6], v[7], inv));
      }
    }
    if (lane == 0) scale[row] = amax / 127.0f;
    if constexpr (kPrefetch) {
#pragma unroll
      for (int i = 0; i < MAXV; ++i) cur[i] = nxt[i];
    }
  }
}

// Each row's largest bf16 value (f32 bits, 0 when none is positive): the
// row_max the quantiser above takes, for callers without a linear's epilogue
// to record it.  One warp per row.
__global__ void __launch_bounds__(256) row_max_bf16_kernel(const bf16* __restrict__ x, unsigned int* out,
                                                           int rows, const int* drows, int cols) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerBlock + warp;
  const int R = drows ? min(*drows, rows) : rows;
  if (row >= R) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * cols);
  float m = 0.f;
  for (int vi = lane; vi < cols / 8; vi += 32) {
    float v[8];
    Vec<bf16>::unpack(__ldg(xr + vi), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) m = fmaxf(m, v[e]);
  }
  m = warp_max(m);
  if (lane == 0) out[row] = __float_as_uint(m);
}

// ── elementwise exact-erf GELU, in place ──────────────────────────────────
// Rows < *drows of x [rows, cols] (cols a multiple of the 16-byte vector).
template <typename T>
__global__ void __launch_bounds__(256) gelu_rows_kernel(T* x, int rows, const int* drows, int cols) {
  constexpr int VN = Vec<T>::N;
  const int R = drows ? min(*drows, rows) : rows;
  const size_t nv = static_cast<size_t>(R) * (cols / VN);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float v[VN];
    Vec<T>::load(x + i * VN, v);
#pragma unroll
    for (int e = 0; e < VN; ++e) v[e] = gelu_erf(v[e]);
    Vec<T>::store(x + i * VN, v);
  }
}

// RoPE on the Q and K blocks of packed qkv rows [T, 3H], in place
// (RotaryEmbedding::apply, modernbert.rs:133-163): for head h and i < d/2,
//   (x_i, x_{i+d/2}) -> (x_i c - x_{i+d/2} s, x_{i+d/2} c + x_i s),
// c, s = cos / sin[p][i] of the token's position p in its row.  One warp per
// token, persistent over the (row, position) slots; padding slots skipped.
template <typename T>
__global__ void __launch_bounds__(256) rope_qk_kernel(T* qkv, const int* __restrict__ cu, int batch,
                                                      int max_seq, int heads, int d,
                                                      const float* __restrict__ cos_t,
                                                      const float* __restrict__ sin_t) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = d >> 1, H = heads * d, pairs = 2 * heads * half;
  const int slots = batch * max_seq;
  for (int slot = blockIdx.x * 8 + warp; slot < slots; slot += gridDim.x * 8) {
    const int b = slot / max_seq, p = slot % max_seq;
    const int start = cu[b];
    if (p >= cu[b + 1] - start) continue;  // warp-uniform
    T* row = qkv + static_cast<size_t>(start + p) * 3 * H;
    const float* cr = cos_t + static_cast<size_t>(p) * half;
    const float* sr = sin_t + static_cast<size_t>(p) * half;
    for (int j = lane; j < pairs; j += 32) {
      const int h = j / half, i = j - h * half;  // h < heads: Q, else K (contiguous)
      T* x = row + h * d + i;
      const float x1 = to_f(x[0]), x2 = to_f(x[half]);
      const float c = cr[i], sn = sr[i];
      x[0] = from_f<T>(x1 * c - x2 * sn);
      x[half] = from_f<T>(x2 * c + x1 * sn);
    }
  }
}

// GeGLU of ModernBertMlp::forward (modernbert.rs:241-254): up_gate [rows, 2I]
// -> out[r, j] = gelu_erf(up_gate[r, j]) * up_gate[r, I + j], out [rows, I].
template <typename T>
__global__ void __launch_bounds__(256) geglu_kernel(const T* __restrict__ ug, T* __restrict__ out,
                                                    int rows, const int* drows, int I) {
  constexpr int VN = Vec<T>::N;
  const int R = drows ? min(*drows, rows) : rows;
  const int vpr = I / VN;
  const size_t nv = static_cast<size_t>(R) * vpr;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < nv;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t r = i / vpr;
    const int c = static_cast<int>(i - r * vpr) * VN;
    float g[VN], u[VN];
    Vec<T>::load(ug + r * 2 * I + c, g);
    Vec<T>::load(ug + r * 2 * I + I + c, u);
#pragma unroll
    for (int e = 0; e < VN; ++e) g[e] = gelu_erf(g[e]) * u[e];
    Vec<T>::store(out + r * I + c, g);
  }
}

// ── pooling + L2 (pooling.rs:31-148) ──────────────────────────────────────
constexpr int kPoolThreads = 128;

__device__ __forceinline__ float block_sum_128(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kPoolThreads / 32; ++i) t += red[i];
  return t;
}

// One block per row: warp w accumulates tokens w, w+8, ... over all columns
// (each lane owns 16-byte column vectors lane, lane+32, ...); the eight
// partial vectors meet in shared memory, then the block forms the L2 norm.
constexpr int kPoolWarps = 8;
constexpr int kPoolMaxH = 1024;

template <typename T>
__global__ void __launch_bounds__(kPoolWarps * 32) pool_normalize_kernel(const T* __restrict__ hidden,
                                                                         const int* __restrict__ cu,
                                                                         float* __restrict__ out, int H,
                                                                         int pooling) {
  constexpr int VN = Vec<T>::N;
  constexpr int MAXV = kPoolMaxH / (32 * VN);
  __shared__ float part[kPoolWarps][kPoolMaxH];
  __shared__ float red[kPoolWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x;
  const int start = cu[b], n = cu[b + 1] - start;
  const int nvec = H / VN;
  const bool is_max = pooling == JB_POOL_MAX;
  float acc[MAXV * VN];
#pragma unroll
  for (int k = 0; k < MAXV * VN; ++k) acc[k] = is_max ? -1e30f : 0.f;
  // CLS reads token 0 only; an all-padding row has none and stays zero.
  const int t_end = pooling == JB_POOL_CLS ? min(n, 1) : n;
  auto add_token = [&](int t, const uint4 (&raw)[MAXV]) {
    const float w = pooling == JB_POOL_WEIGHTED_MEAN ? static_cast<float>(t + 1) : 1.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (lane + 32 * i < nvec) {
        float x[VN];
        Vec<T>::unpack(raw[i], x);
#pragma unroll
        for (int e = 0; e < VN; ++e)
          acc[i * VN + e] = is_max ? fmaxf(acc[i * VN + e], x[e]) : fmaf(x[e], w, acc[i * VN + e]);
      }
    }
  };
  auto load_token = [&](int t, uint4 (&raw)[MAXV]) {
    const uint4* hr = reinterpret_cast<const uint4*>(hidden + static_cast<size_t>(start + t) * H);
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
      if (lane + 32 * i < nvec) raw[i] = __ldg(hr + lane + 32 * i);
  };
  // Warp w takes tokens w, w+8, ... in order; bf16 rows load four tokens at
  // a time (the accumulation order, hence the result, is unchanged).
  constexpr int kUnroll = sizeof(T) == 2 ? 4 : 1;
  int t = warp;
  for (; t + (kUnroll - 1) * kPoolWarps < t_end; t += kUnroll * kPoolWarps) {
    uint4 raw[kUnroll][MAXV];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) load_token(t + u * kPoolWarps, raw[u]);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) add_token(t + u * kPoolWarps, raw[u]);
  }
  for (; t < t_end; t += kPoolWarps) {
    uint4 raw[MAXV];
    load_token(t, raw);
    add_token(t, raw);
  }
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec)
#pragma unroll
      for (int e = 0; e < VN; ++e) part[warp][vi * VN + e] = acc[i * VN + e];
  }
  __syncthreads();
  float den = 1.f;
  if (pooling == JB_POOL_MEAN) den = fmaxf(static_cast<float>(n), 1.f);
  if (pooling == JB_POOL_WEIGHTED_MEAN)
    den = fmaxf(0.5f * static_cast<float>(n) * static_cast<float>(n + 1), 1.f);
  constexpr int kPer = kPoolMaxH / (kPoolWarps * 32);
  float vals[kPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int c = threadIdx.x + k * kPoolWarps * 32;
    float v = 0.f;
    if (c < H) {
      v = part[0][c];
#pragma unroll
      for (int w = 1; w < kPoolWarps; ++w) v = is_max ? fmaxf(v, part[w][c]) : v + part[w][c];
      if (!is_max) v = v / den;
      ss += v * v;
    }
    vals[k] = v;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  ss = 0.f;
#pragma unroll
  for (int w = 0; w < kPoolWarps; ++w) ss += red[w];
  // clamp(||x||, 1e-12, f32::MAX): an overflowing square sum (the -1e30
  // max-pool sentinel of an all-padding row) clamps to f32::MAX.
  const float norm = fminf(fmaxf(sqrtf(ss), 1e-12f), FLT_MAX);
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int c = threadIdx.x + k * kPoolWarps * 32;
    if (c < H) out[static_cast<size_t>(b) * H + c] = vals[k] / norm;
  }
}

__global__ void l2_rows_kernel(float* x, int cols) {
  __shared__ float red[kPoolThreads / 32];
  float* r = x + static_cast<size_t>(blockIdx.x) * cols;
  float ss = 0.f;
  for (int c = threadIdx.x; c < cols; c += kPoolThreads) ss += r[c] * r[c];
  ss = block_sum_128(ss, red);
  const float norm = fmaxf(sqrtf(ss), 1e-12f);
  for (int c = threadIdx.x; c < cols; c += kPoolThreads) r[c] = r[c] / norm;
}

// Exclusive scan of clamped lengths into cu[0..batch]; one 1024-thread block.
__global__ void __launch_bounds__(1024) lens_to_cu_kernel(const uint32_t* lens, int batch,
                                                          int max_seq, int* cu, int* total,
                                                          int* err) {
  __shared__ int part[1024];
  const int per = (batch + 1023) / 1024;
  const int b0 = threadIdx.x * per;
  int s = 0;
  for (int i = 0; i < per; ++i) {
    const int b = b0 + i;
    if (b < batch) {
      uint32_t l = lens[b];
      if (l > static_cast<uint32_t>(max_seq)) {
        if (err) atomicOr(err, 4);
        l = max_seq;
      }
      s += static_cast<int>(l);
    }
  }
  part[threadIdx.x] = s;
  __syncthreads();
  for (int off = 1; off < 1024; off <<= 1) {
    const int v = threadIdx.x >= off ? part[threadIdx.x - off] : 0;
    __syncthreads();
    part[threadIdx.x] += v;
    __syncthreads();
  }
  int run = part[threadIdx.x] - s;  // exclusive prefix of this thread's chunk
  for (int i = 0; i < per; ++i) {
    const int b = b0 + i;
    if (b < batch) {
      cu[b] = run;
      run += static_cast<int>(min(lens[b], static_cast<uint32_t>(max_seq)));
    }
  }
  if (threadIdx.x == 1023) {
    cu[batch] = part[1023];
    if (total) *total = part[1023];
  }
}

template <typename T>
__global__ void unpack_hidden_kernel(const T* packed, const int* cu, float* out, int batch,
                                     int max_seq, int H) {
  const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t total = static_cast<size_t>(batch) * max_seq * H;
  if (idx >= total) return;
  const int c = idx % H;
  const int p = (idx / H) % max_seq;
  const int b = idx / (static_cast<size_t>(H) * max_seq);
  const int start = cu[b], n = cu[b + 1] - start;
  out[idx] = p < n ? to_f(packed[static_cast<size_t>(start + p) * H + c]) : 0.f;
}

template <typename T>
__global__ void patchify_kernel(const float* px, T* out, int batch, int image, int patch) {
  const int g = image / patch;
  const int K = 3 * patch * patch;
  const size_t idx = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t total = static_cast<size_t>(batch) * g * g * K;
  if (idx >= total) return;
  const int k = idx % K;
  const size_t prow = idx / K;
  const int b = prow / (g * g);
  const int pidx = prow % (g * g);
  const int gy = pidx / g, gx = pidx % g;
  const int c = k / (patch * patch), ky = (k / patch) % patch, kx = k % patch;
  const float v = px[((static_cast<size_t>(b) * 3 + c) * image + gy * patch + ky) * image +
                     gx * patch + kx];
  out[idx] = from_f<T>(v);
}

// The same gather for patch and image sides that are multiples of 8: one
// thread per 8 consecutive pixels of one source row of image blockIdx.y
// (two 16-byte loads, consecutive threads along the row), written as 8
// consecutive elements of one patch row (one 16-byte store for 16-bit T).
// 32-bit index arithmetic inside one image.
template <typename T>
__global__ void __launch_bounds__(256) patchify8_kernel(const float* __restrict__ px, T* __restrict__ out,
                                                        int image, int patch) {
  const int xv = image >> 3, pv = patch >> 3, g = image / patch;
  const int u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= 3 * image * xv) return;
  const int b = blockIdx.y;
  const int x8 = u % xv, cy = u / xv, y = cy % image, c = cy / image;
  const float4* src = reinterpret_cast<const float4*>(
      px + ((static_cast<size_t>(b) * 3 + c) * image + y) * image + x8 * 8);
  const float4 a0 = __ldg(src), a1 = __ldg(src + 1);
  const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  const int gy = y / patch, ky = y - gy * patch, gx = x8 / pv, kx = (x8 - gx * pv) * 8;
  const size_t prow = static_cast<size_t>(b) * g * g + gy * g + gx;
  T* dst = out + prow * (3 * patch * patch) + (c * patch + ky) * patch + kx;
  constexpr int VN = Vec<T>::N;
#pragma unroll
  for (int i = 0; i < 8; i += VN) Vec<T>::store(dst + i, v + i);
}

template <typename T, int MAXV>
__global__ void __launch_bounds__(256) vit_embed_ln_kernel(const T* patch_out, const T* cls,
                                                           const T* pos, const float* gamma,
                                                           const float* beta, T* y, int batch,
                                                           int tokens, int W, float eps) {
  constexpr int VN = Vec<T>::N;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerBlock + warp;
  if (row >= batch * tokens) return;
  const int b = row / tokens, i = row % tokens;
  const T* src = i == 0 ? cls : patch_out + (static_cast<size_t>(b) * (tokens - 1) + i - 1) * W;
  const T* pe = pos + static_cast<size_t>(i) * W;
  const int nvec = W / VN;
  float v[MAXV * VN];
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int vi = lane + k * 32;
    if (vi < nvec) {
      float t[VN];
      Vec<T>::load(src + vi * VN, v + k * VN);
      Vec<T>::load(pe + vi * VN, t);
#pragma unroll
      for (int e = 0; e < VN; ++e) v[k * VN + e] += t[e];
    }
  }
  ln_finish<T, MAXV>(v, nvec, W, lane, gamma, beta, eps, y + static_cast<size_t>(row) * W, nullptr,
                     nullptr);
}

template <typename T, int MAXV>
__global__ void __launch_bounds__(32) vit_pool_ln_kernel(const T* x, const float* gamma,
                                                         const float* beta, T* y, int tokens,
                                                         int W, int gap, float eps,
                                                         const int* cu) {
  constexpr int VN = Vec<T>::N;
  const int lane = threadIdx.x;
  const int b = blockIdx.x;
  const int nvec = W / VN;
  float v[MAXV * VN];
#pragma unroll
  for (int k = 0; k < MAXV * VN; ++k) v[k] = 0.f;
  const int t0 = gap ? 1 : 0, t1 = gap ? tokens : 1;
  for (int t = t0; t < t1; ++t) {
    // cu: packed rows, the row's last token; else fixed rows of `tokens`
    const T* xr = cu ? x + static_cast<size_t>(cu[b + 1] - 1) * W
                     : x + (static_cast<size_t>(b) * tokens + t) * W;
#pragma unroll
    for (int k = 0; k < MAXV; ++k) {
      const int vi = lane + k * 32;
      if (vi < nvec) {
        float tmp[VN];
        Vec<T>::load(xr + vi * VN, tmp);
#pragma unroll
        for (int e = 0; e < VN; ++e) v[k * VN + e] += tmp[e];
      }
    }
  }
  if (gap) {
    const float inv_n = 1.0f / static_cast<float>(tokens - 1);
#pragma unroll
    for (int k = 0; k < MAXV * VN; ++k) v[k] *= inv_n;
  }
  ln_finish<T, MAXV>(v, nvec, W, lane, gamma, beta, eps, y + static_cast<size_t>(b) * W, nullptr,
                     nullptr);
}

// One warp per row: len[b] = 1 + the first position of the row's largest id
// (argmax(input_ids, dim=1), clip_text.rs:322-326; OpenCLIP's <|endoftext|>
// has the largest id, so the row ends at its EOT token).
__global__ void __launch_bounds__(256) eot_lens_kernel(const uint32_t* __restrict__ ids, int batch,
                                                       int S, uint32_t* __restrict__ lens) {
  const int b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (b >= batch) return;
  const uint32_t* r = ids + static_cast<size_t>(b) * S;
  uint32_t best = 0;
  int at = S;  // S: none seen yet (every real position compares below)
  for (int p = lane; p < S; p += 32) {
    const uint32_t v = r[p];
    if (at == S || v > best) {  // positions rise per lane: the first maximum wins
      best = v;
      at = p;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const uint32_t ob = __shfl_xor_sync(0xffffffffu, best, off);
    const int oa = __shfl_xor_sync(0xffffffffu, at, off);
    if (oa < S && (at == S || ob > best || (ob == best && oa < at))) {
      best = ob;
      at = oa;
    }
  }
  if (lane == 0) lens[b] = static_cast<uint32_t>(at < S ? at + 1 : 0);
}

__global__ void fill_cu_uniform_kernel(int* cu, int batch, int tokens) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b <= batch) cu[b] = b * tokens;
}

inline unsigned blocks_for(size_t n, unsigned per) { return static_cast<unsigned>((n + per - 1) / per); }

}  // namespace

// Persistent row kernels run one wave of 256-thread blocks: as many per SM
// as the kernel's registers and shared memory let reside (asked of the
// occupancy calculator once per kernel), so no block waits for a second wave.
template <auto Kern>
unsigned persistent_grid(size_t rows) {
  static const int per_sm = [] {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, Kern, 256, 0) != cudaSuccess || n < 1)
      n = 1;
    return n;
  }();
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned cap = static_cast<unsigned>(num_sms(dev)) * static_cast<unsigned>(per_sm);
  const unsigned need = blocks_for(rows, kRowsPerBlock);
  return need < cap ? need : cap;
}

cudaError_t launch_layernorm(const LnArgs& a, cudaStream_t s) {
  if (a.rows == 0) return cudaSuccess;
  if (a.cols > kLnMaxCols) return cudaErrorInvalidValue;
  if (a.dtype == JB_DT_BF16) {
    if (a.cols % 8 || a.cols > 1024) return cudaErrorInvalidValue;
    if (a.cols <= 768) {
      if (a.resid)
        layernorm_bf16_kernel<3, true>
            <<<persistent_grid<layernorm_bf16_kernel<3, true>>(a.rows), 256, 0, s>>>(a);
      else
        layernorm_bf16_kernel<3, false>
            <<<persistent_grid<layernorm_bf16_kernel<3, false>>(a.rows), 256, 0, s>>>(a);
    } else {
      if (a.resid)
        layernorm_bf16_kernel<4, true>
            <<<persistent_grid<layernorm_bf16_kernel<4, true>>(a.rows), 256, 0, s>>>(a);
      else
        layernorm_bf16_kernel<4, false>
            <<<persistent_grid<layernorm_bf16_kernel<4, false>>(a.rows), 256, 0, s>>>(a);
    }
  } else if (a.dtype == JB_DT_F16) {
    if (a.cols % 8 || a.cols > 1024 || a.yq) return cudaErrorInvalidValue;
    if (a.cols <= 768) {
      if (a.resid)
        layernorm_bf16_kernel<3, true, f16>
            <<<persistent_grid<layernorm_bf16_kernel<3, true, f16>>(a.rows), 256, 0, s>>>(a);
      else
        layernorm_bf16_kernel<3, false, f16>
            <<<persistent_grid<layernorm_bf16_kernel<3, false, f16>>(a.rows), 256, 0, s>>>(a);
    } else {
      if (a.resid)
        layernorm_bf16_kernel<4, true, f16>
            <<<persistent_grid<layernorm_bf16_kernel<4, true, f16>>(a.rows), 256, 0, s>>>(a);
      else
        layernorm_bf16_kernel<4, false, f16>
            <<<persistent_grid<layernorm_bf16_kernel<4, false, f16>>(a.rows), 256, 0, s>>>(a);
    }
  } else if (a.dtype == JB_DT_F32) {
    if (a.cols % 4 || a.cols > 1024) return cudaErrorInvalidValue;
    layernorm_kernel<float, 8><<<persistent_grid<layernorm_kernel<float, 8>>(a.rows), 256, 0, s>>>(a);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_embed_ln(const EmbedArgs& a, cudaStream_t s) {
  const size_t n = static_cast<size_t>(a.batch) * a.max_seq;
  if (n == 0) return cudaSuccess;
  if (a.dtype == JB_DT_BF16) {
    if (a.H % 8 || a.H > 1024) return cudaErrorInvalidValue;
    embed_ln_kernel<bf16, 4><<<persistent_grid<embed_ln_kernel<bf16, 4>>(n), 256, 0, s>>>(a);
  } else if (a.dtype == JB_DT_F16) {
    if (a.H % 8 || a.H > 1024) return cudaErrorInvalidValue;
    embed_ln_kernel<f16, 4><<<persistent_grid<embed_ln_kernel<f16, 4>>(n), 256, 0, s>>>(a);
  } else if (a.dtype == JB_DT_F32) {
    if (a.H % 4 || a.H > 1024) return cudaErrorInvalidValue;
    embed_ln_kernel<float, 8><<<persistent_grid<embed_ln_kernel<float, 8>>(n), 256, 0, s>>>(a);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

namespace {
template <int ACT>
cudaError_t launch_quantize_act(const void* x, int dtype, int8_t* q, float* scale, int rows,
                                const int* drows, int cols, cudaStream_t s) {
  const unsigned grid = blocks_for(rows, kRowsPerBlock);
  if (dtype == JB_DT_BF16) {
    if (cols % 8) return cudaErrorInvalidValue;
    const bf16* xb = static_cast<const bf16*>(x);
    const int per_lane = (cols / 8 + 31) / 32;
    if (per_lane <= 4)
      quantize_rows_kernel<bf16, 4, ACT><<<grid, 256, 0, s>>>(xb, q, scale, rows, drows, cols);
    else if (per_lane <= 8)
      quantize_rows_kernel<bf16, 8, ACT><<<grid, 256, 0, s>>>(xb, q, scale, rows, drows, cols);
    else if (per_lane <= 12)
      quantize_rows_kernel<bf16, 12, ACT><<<grid, 256, 0, s>>>(xb, q, scale, rows, drows, cols);
    else if (per_lane <= 16)
      quantize_rows_kernel<bf16, 16, ACT><<<grid, 256, 0, s>>>(xb, q, scale, rows, drows, cols);
    else
      quantize_rows_kernel<bf16, 0, ACT><<<grid, 256, 0, s>>>(xb, q, scale, rows, drows, cols);
  } else if (dtype != JB_DT_F32) {
    return cudaErrorInvalidValue;  // int8 inputs come from bf16 or f32 rows
  } else {
    if (cols % 4) return cudaErrorInvalidValue;
    quantize_rows_kernel<float, 0, ACT><<<grid, 256, 0, s>>>(static_cast<const float*>(x), q,
                                                             scale, rows, drows, cols);
  }
  return cudaGetLastError();
}
}  // namespace

namespace {
std::mutex g_gelu_mu;
bool g_gelu_ready[64] = {};

template <int MAXV>
cudaError_t launch_gelu_quantize_v(const bf16* x, const unsigned int* row_max, int8_t* q, float* scale,
                                   int rows, const int* drows, int cols, cudaStream_t s) {
  auto kern = gelu_quantize_kernel<MAXV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kGeluTableBytes);
  if (e != cudaSuccess) return e;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned need = blocks_for(rows, kGeluQThreads / 32);
  const unsigned grid = std::min<unsigned>(need, static_cast<unsigned>(num_sms(dev)));
  kern<<<grid, kGeluQThreads, kGeluTableBytes, s>>>(x, row_max, q, scale, rows, drows, cols);
  return cudaGetLastError();
}
// Rows of up to 16 vectors per lane (4096 columns) held in registers.
cudaError_t launch_gelu_quantize(const bf16* x, const unsigned int* row_max, int8_t* q, float* scale,
                                 int rows, const int* drows, int cols, cudaStream_t s) {
  const int per_lane = (cols / 8 + 31) / 32;
  if (per_lane <= 4) return launch_gelu_quantize_v<4>(x, row_max, q, scale, rows, drows, cols, s);
  if (per_lane <= 8) return launch_gelu_quantize_v<8>(x, row_max, q, scale, rows, drows, cols, s);
  if (per_lane <= 12) return launch_gelu_quantize_v<12>(x, row_max, q, scale, rows, drows, cols, s);
  if (per_lane <= 16) return launch_gelu_quantize_v<16>(x, row_max, q, scale, rows, drows, cols, s);
  return cudaErrorInvalidValue;
}
}  // namespace

cudaError_t init_gelu_table(cudaStream_t s) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(g_gelu_mu);
  if (dev >= 0 && dev < 64 && g_gelu_ready[dev]) return cudaSuccess;
  // Built once, synchronously, so that work on any stream may use it after.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(s, &cap);
  if (e != cudaSuccess) return e;
  if (cap != cudaStreamCaptureStatusNone) return cudaErrorStreamCaptureUnsupported;
  gelu_table_kernel<<<65536 / 256, 256, 0, s>>>();
  e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && dev >= 0 && dev < 64) g_gelu_ready[dev] = true;
  return e;
}

cudaError_t launch_quantize_rows(const void* x, int dtype, int8_t* q, float* scale, int rows,
                                 const int* drows, int cols, cudaStream_t s, int activation) {
  if (rows == 0) return cudaSuccess;
  if (activation == JB_EPI_GELU && dtype == JB_DT_BF16 && cols % 8 == 0) {
    cudaError_t e = init_gelu_table(s);  // no-op after the first call on this device
    if (e != cudaSuccess) return e;
    // the rows' largest values go to `scale` first (the quantiser reads a
    // row's entry before it writes the row's scale there)
    const bf16* xb = static_cast<const bf16*>(x);
    unsigned int* rmax = reinterpret_cast<unsigned int*>(scale);
    row_max_bf16_kernel<<<blocks_for(rows, kRowsPerBlock), 256, 0, s>>>(xb, rmax, rows, drows, cols);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_gelu_quantize(xb, rmax, q, scale, rows, drows, cols, s);
  }
  if (activation == JB_EPI_GELU)
    return launch_quantize_act<JB_EPI_GELU>(x, dtype, q, scale, rows, drows, cols, s);
  if (activation != JB_EPI_NONE) return cudaErrorInvalidValue;
  return launch_quantize_act<JB_EPI_NONE>(x, dtype, q, scale, rows, drows, cols, s);
}

cudaError_t launch_gelu_quantize_rowmax(const void* x, const unsigned int* row_max, int8_t* q,
                                        float* scale, int rows, const int* drows, int cols,
                                        cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (cols % 8) return cudaErrorInvalidValue;
  cudaError_t e = init_gelu_table(s);  // no-op after the first call on this device
  if (e != cudaSuccess) return e;
  return launch_gelu_quantize(static_cast<const bf16*>(x), row_max, q, scale, rows, drows, cols, s);
}

cudaError_t launch_gelu_rows(void* x, int dtype, int rows, const int* drows, int cols,
                             cudaStream_t s) {
  if (dtype != JB_DT_BF16 && dtype != JB_DT_F32) return cudaErrorInvalidValue;  // not an f16 kernel
  if (rows == 0) return cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned grid = static_cast<unsigned>(num_sms(dev)) * 8u;
  if (dtype == JB_DT_BF16) {
    if (cols % 8) return cudaErrorInvalidValue;
    gelu_rows_kernel<bf16><<<grid, 256, 0, s>>>(static_cast<bf16*>(x), rows, drows, cols);
  } else {
    if (cols % 4) return cudaErrorInvalidValue;
    gelu_rows_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(x), rows, drows, cols);
  }
  return cudaGetLastError();
}

cudaError_t launch_rope_qk(void* qkv, int dtype, const int* cu, int batch, int max_seq, int heads,
                           int d, const float* cos_t, const float* sin_t, cudaStream_t s) {
  if (dtype != JB_DT_BF16 && dtype != JB_DT_F32) return cudaErrorInvalidValue;  // not an f16 kernel
  const size_t slots = static_cast<size_t>(batch) * max_seq;
  if (slots == 0) return cudaSuccess;
  if (d % 2) return cudaErrorInvalidValue;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned grid = std::min<unsigned>(blocks_for(slots, 8), static_cast<unsigned>(num_sms(dev)) * 8u);
  if (dtype == JB_DT_BF16)
    rope_qk_kernel<bf16><<<grid, 256, 0, s>>>(static_cast<bf16*>(qkv), cu, batch, max_seq, heads, d,
                                              cos_t, sin_t);
  else
    rope_qk_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(qkv), cu, batch, max_seq, heads,
                                               d, cos_t, sin_t);
  return cudaGetLastError();
}

cudaError_t launch_geglu(const void* ug, void* out, int dtype, int rows, const int* drows, int I,
                         cudaStream_t s) {
  if (dtype != JB_DT_BF16 && dtype != JB_DT_F32) return cudaErrorInvalidValue;  // not an f16 kernel
  if (rows == 0) return cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned grid = static_cast<unsigned>(num_sms(dev)) * 8u;
  if (dtype == JB_DT_BF16) {
    if (I % 8) return cudaErrorInvalidValue;
    geglu_kernel<bf16><<<grid, 256, 0, s>>>(static_cast<const bf16*>(ug), static_cast<bf16*>(out),
                                            rows, drows, I);
  } else {
    if (I % 4) return cudaErrorInvalidValue;
    geglu_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(ug), static_cast<float*>(out),
                                             rows, drows, I);
  }
  return cudaGetLastError();
}

cudaError_t launch_pool_normalize(const void* hidden, int dtype, const int* cu, float* out,
                                  int batch, int H, int pooling, cudaStream_t s) {
  if (batch == 0) return cudaSuccess;
  if (H > kPoolMaxH || pooling < 0 || pooling > 3) return cudaErrorInvalidValue;
  if (dtype == JB_DT_BF16) {
    if (H % 8) return cudaErrorInvalidValue;
    pool_normalize_kernel<bf16><<<batch, kPoolWarps * 32, 0, s>>>(static_cast<const bf16*>(hidden),
                                                                  cu, out, H, pooling);
  } else if (dtype == JB_DT_F16) {
    if (H % 8) return cudaErrorInvalidValue;
    pool_normalize_kernel<f16><<<batch, kPoolWarps * 32, 0, s>>>(static_cast<const f16*>(hidden),
                                                                 cu, out, H, pooling);
  } else if (dtype != JB_DT_F32) {
    return cudaErrorInvalidValue;
  } else {
    if (H % 4) return cudaErrorInvalidValue;
    pool_normalize_kernel<float><<<batch, kPoolWarps * 32, 0, s>>>(
        static_cast<const float*>(hidden), cu, out, H, pooling);
  }
  return cudaGetLastError();
}

cudaError_t launch_lens_to_cu(const uint32_t* lens, int batch, int max_seq, int* cu, int* d_total,
                              int* err, cudaStream_t s) {
  lens_to_cu_kernel<<<1, 1024, 0, s>>>(lens, batch, max_seq, cu, d_total, err);
  return cudaGetLastError();
}

cudaError_t launch_unpack_hidden(const void* packed, int dtype, const int* cu, float* out,
                                 int batch, int max_seq, int H, cudaStream_t s) {
  const size_t n = static_cast<size_t>(batch) * max_seq * H;
  if (n == 0) return cudaSuccess;
  if (dtype == JB_DT_BF16)
    unpack_hidden_kernel<bf16><<<blocks_for(n, 256), 256, 0, s>>>(static_cast<const bf16*>(packed),
                                                                  cu, out, batch, max_seq, H);
  else if (dtype == JB_DT_F16)
    unpack_hidden_kernel<f16><<<blocks_for(n, 256), 256, 0, s>>>(static_cast<const f16*>(packed),
                                                                 cu, out, batch, max_seq, H);
  else if (dtype != JB_DT_F32)
    return cudaErrorInvalidValue;
  else
    unpack_hidden_kernel<float><<<blocks_for(n, 256), 256, 0, s>>>(
        static_cast<const float*>(packed), cu, out, batch, max_seq, H);
  return cudaGetLastError();
}

cudaError_t launch_patchify(const float* px, void* patches, int dtype, int batch, int image,
                            int patch, cudaStream_t s) {
  if (dtype != JB_DT_BF16 && dtype != JB_DT_F32) return cudaErrorInvalidValue;  // not an f16 kernel
  const int g = image / patch;
  const size_t n = static_cast<size_t>(batch) * g * g * 3 * patch * patch;
  if (n == 0) return cudaSuccess;
  if (patch % 8 == 0 && image % 8 == 0 && image % patch == 0 && (reinterpret_cast<uintptr_t>(px) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(patches) & 15) == 0) {
    const unsigned per_image = blocks_for(static_cast<size_t>(3) * image * (image / 8), 256);
    for (int b0 = 0; b0 < batch; b0 += 65535) {  // grid.y: one image each
      const int nb = std::min(batch - b0, 65535);
      const size_t px_off = static_cast<size_t>(b0) * 3 * image * image;
      const size_t out_off = static_cast<size_t>(b0) * g * g * 3 * patch * patch;
      if (dtype == JB_DT_BF16)
        patchify8_kernel<bf16><<<dim3(per_image, nb), 256, 0, s>>>(
            px + px_off, static_cast<bf16*>(patches) + out_off, image, patch);
      else
        patchify8_kernel<float><<<dim3(per_image, nb), 256, 0, s>>>(
            px + px_off, static_cast<float*>(patches) + out_off, image, patch);
    }
    return cudaGetLastError();
  }
  if (dtype == JB_DT_BF16)
    patchify_kernel<bf16><<<blocks_for(n, 256), 256, 0, s>>>(px, static_cast<bf16*>(patches), batch,
                                                             image, patch);
  else
    patchify_kernel<float><<<blocks_for(n, 256), 256, 0, s>>>(px, static_cast<float*>(patches),
                                                              batch, image, patch);
  return cudaGetLastError();
}

cudaError_t launch_vit_embed_ln(const void* patch_out, const void* cls, const void* pos,
                                const float* gamma, const float* beta, void* y, int dtype,
                                int batch, int tokens, int W, float eps, cudaStream_t s) {
  if (dtype != JB_DT_BF16 && dtype != JB_DT_F32) return cudaErrorInvalidValue;  // not an f16 kernel
  const size_t n = static_cast<size_t>(batch) * tokens;
  if (n == 0) return cudaSuccess;
  const unsigned grid = blocks_for(n, kRowsPerBlock);
  if (dtype == JB_DT_BF16) {
    if (W % 8 || W > 1024) return cudaErrorInvalidValue;
    vit_embed_ln_kernel<bf16, 4><<<grid, 256, 0, s>>>(
        static_cast<const bf16*>(patch_out), static_cast<const bf16*>(cls),
        static_cast<const bf16*>(pos), gamma, beta, static_cast<bf16*>(y), batch, tokens, W, eps);
  } else {
    if (W % 4 || W > 1024) return cudaErrorInvalidValue;
    vit_embed_ln_kernel<float, 8><<<grid, 256, 0, s>>>(
        static_cast<const float*>(patch_out), static_cast<const float*>(cls),
        static_cast<const float*>(pos), gamma, beta, static_cast<float*>(y), batch, tokens, W, eps);
  }
  return cudaGetLastError();
}

cudaError_t launch_vit_pool_ln(const void* x, const float* gamma, const float* beta, void* y,
                               int dtype, int batch, int tokens, int W, int gap, float eps,
                               cudaStream_t s, const int* cu) {
  if (dtype != JB_DT_BF16 && dtype != JB_DT_F32) return cudaErrorInvalidValue;  // not an f16 kernel
  if (batch == 0) return cudaSuccess;
  if (cu && gap) return cudaErrorInvalidValue;
  if (dtype == JB_DT_BF16) {
    if (W % 8 || W > 1024) return cudaErrorInvalidValue;
    vit_pool_ln_kernel<bf16, 4><<<batch, 32, 0, s>>>(static_cast<const bf16*>(x), gamma, beta,
                                                     static_cast<bf16*>(y), tokens, W, gap, eps, cu);
  } else {
    if (W % 4 || W > 1024) return cudaErrorInvalidValue;
    vit_pool_ln_kernel<float, 8><<<batch, 32, 0, s>>>(static_cast<const float*>(x), gamma, beta,
                                                      static_cast<float*>(y), tokens, W, gap, eps, cu);
  }
  return cudaGetLastError();
}

cudaError_t launch_eot_lens(const uint32_t* ids, int batch, int S, uint32_t* lens, cudaStream_t s) {
  if (batch == 0) return cudaSuccess;
  eot_lens_kernel<<<blocks_for(static_cast<size_t>(batch), 8), 256, 0, s>>>(ids, batch, S, lens);
  return cudaGetLastError();
}

cudaError_t launch_fill_cu_uniform(int* cu, int batch, int tokens, cudaStream_t s) {
  fill_cu_uniform_kernel<<<blocks_for(static_cast<size_t>(batch) + 1, 256), 256, 0, s>>>(cu, batch, tokens);
  return cudaGetLastError();
}

cudaError_t launch_l2_rows(float* x, int rows, int cols, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  l2_rows_kernel<<<rows, kPoolThreads, 0, s>>>(x, cols);
  return cudaGetLastError();
}

}  // namespace jb
