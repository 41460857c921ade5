// The vector side of the ANN sidecar and of exact search, on the device:
// the produced embeddings go from HBM into the index formats without a trip
// through host loops.
//
// * Binary threshold tau (fit_binary_threshold, crates/jammi-db/src/index/
//   sidecar.rs:162-216): per dimension over the first min(rows, 100000)
//   rows, either the mean -- an f64 sum taken in row order, divided by the
//   row count, rounded to f32 -- or the median under f32 total order (the
//   two central values averaged in f32 for an even count).  The mean runs
//   one thread per dimension so its additions happen in the reference's
//   order (bit-identical); the median is a radix select over the total-order
//   keys, exact by construction.
// * Threshold sign-packing (pack_threshold_bits, sidecar.rs:232-241): bit i
//   of a row is v[i] > tau[i], LSB-first in ceil(dim / 8) bytes, padding 0.
// * Exact search (exact_vector_search, crates/jammi-db/src/index/
//   exact.rs:119-175, with cosine_distance, crates/jammi-numerics/src/
//   distance.rs:6-21): distance = 1 - dot / (sqrt(|a|^2) sqrt(|b|^2)), or 1
//   when that denominator is below f32 epsilon; the three sums accumulate in
//   f32 in dimension order, each product and sum one IEEE rounding (explicit
//   _rn intrinsics: no fused multiply-adds), so every distance equals the
//   reference's bit for bit.  The k best per query under (distance, row-id
//   rank) -- the reference breaks distance ties by ascending _row_id; the
//   caller passes each row's rank in that order, or none for row order --
//   come from a radix select over 64-bit (distance key, rank) keys, then a
//   rank sort of the k survivors.
#include <algorithm>
#include <cfloat>
#include <cstdint>

#include "jb_common.cuh"
#include "jb_internal.h"

namespace jb {
namespace {

// f32 total order (Rust's f32::total_cmp) as an unsigned key order.
__device__ __forceinline__ uint32_t total_key(float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float from_total_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// ---- binary threshold -------------------------------------------------------

__global__ void mean_threshold_kernel(const float* __restrict__ v, int64_t rows, int dim,
                                      float* __restrict__ tau) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= dim) return;
  const float* p = v + d;
  double s = 0.0;
  int64_t r = 0;
  for (; r + 16 <= rows; r += 16) {  // sixteen loads in flight, the additions in row order
    float x[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) x[u] = __ldg(p + (r + u) * dim);
#pragma unroll
    for (int u = 0; u < 16; ++u) s = __dadd_rn(s, static_cast<double>(x[u]));
  }
  for (; r < rows; ++r) s = __dadd_rn(s, static_cast<double>(__ldg(p + r * dim)));
  const double n = rows > 0 ? static_cast<double>(rows) : 1.0;
  tau[d] = __double2float_rn(__ddiv_rn(s, n));
}

// Median: a radix select over f32 total-order keys, four 8-bit passes, the
// two central order statistics of an even count side by side.  Each pass is
// two launches: median_hist_kernel spreads the rows over a grid of
// (32-dimension groups) x (row splits); each CTA histograms the next byte of
// the keys that match each statistic's prefix so far, in shared memory laid
// out [statistic][bin][lane] (lane = dimension: no two lanes of a warp share
// a word), then adds its non-zero bins to the global histograms.
// median_select_kernel then has one thread per (statistic, dimension) scan
// its 256 bins for the bin holding its remaining rank, extend the prefix and
// clear the histogram for the next pass.  Exact by construction.
constexpr int kMedLanes = 32;
constexpr int kMedThreads = 256;
constexpr int kMedBins = 256;

struct MedianScratch {
  uint32_t* hist;       // [2][dim][256]
  uint32_t* prefix;     // [2][dim]
  int64_t* remaining;   // [2][dim]
};

size_t median_scratch_bytes_(int dim) {
  return size_t(2) * dim * kMedBins * sizeof(uint32_t) + size_t(2) * dim * sizeof(uint32_t) +
         size_t(2) * dim * sizeof(int64_t) + 64;
}

MedianScratch carve_median(void* p, int dim) {
  MedianScratch m;
  char* c = static_cast<char*>(p);
  m.remaining = reinterpret_cast<int64_t*>(c);
  c += size_t(2) * dim * sizeof(int64_t);
  m.hist = reinterpret_cast<uint32_t*>(c);
  c += size_t(2) * dim * kMedBins * sizeof(uint32_t);
  m.prefix = reinterpret_cast<uint32_t*>(c);
  return m;
}

__global__ void median_init_kernel(int dim, int64_t rows, int nstats, MedianScratch m) {
  const int64_t total = int64_t(2) * dim * kMedBins;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x)
    m.hist[i] = 0;
  const int64_t mid = rows / 2;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < 2 * int64_t(dim);
       i += int64_t(gridDim.x) * blockDim.x) {
    const int st = static_cast<int>(i / dim);
    m.prefix[i] = 0;
    // 0-based ranks: mid - 1 and mid for an even count, mid for an odd one
    const int64_t rank = (nstats == 2 && st == 0) ? mid - 1 : mid;
    m.remaining[i] = rank + 1;
  }
}

__global__ void __launch_bounds__(kMedThreads)
median_hist_kernel(const float* __restrict__ v, int64_t rows, int dim, int nstats, int pass,
                   int64_t rows_per_split, MedianScratch m) {
  extern __shared__ uint32_t h[];  // [nstats][256][32]
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int entries = nstats * kMedBins * kMedLanes;
  for (int e = t; e < entries; e += kMedThreads) h[e] = 0;
  __syncthreads();
  const int d = blockIdx.x * kMedLanes + lane;
  const int shift = 24 - 8 * pass;
  const uint32_t mask = pass == 0 ? 0u : (0xFFFFFFFFu << (32 - 8 * pass));
  if (d < dim) {
    const uint32_t p0 = m.prefix[d];
    // adjacent order statistics mostly share their prefix: one histogram then
    const uint32_t p1 = (nstats == 2 && m.prefix[dim + d] != p0) ? m.prefix[dim + d] : 0xFFFFFFFFu;
    const int64_t r_end = min(rows, (blockIdx.y + int64_t(1)) * rows_per_split);
    int64_t r = blockIdx.y * rows_per_split + warp;
    constexpr int W = kMedThreads / 32;
    for (; r + 7 * W < r_end; r += 8 * W) {  // eight loads in flight
      float x[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) x[u] = __ldg(v + (r + u * W) * dim + d);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t key = total_key(x[u]);
        const uint32_t bin = (key >> shift) & 255u;
        if ((key & mask) == p0) atomicAdd(&h[bin * kMedLanes + lane], 1u);
        if (p1 != 0xFFFFFFFFu && (key & mask) == p1) atomicAdd(&h[(kMedBins + bin) * kMedLanes + lane], 1u);
      }
    }
    for (; r < r_end; r += W) {
      const uint32_t key = total_key(__ldg(v + r * dim + d));
      const uint32_t bin = (key >> shift) & 255u;
      if ((key & mask) == p0) atomicAdd(&h[bin * kMedLanes + lane], 1u);
      if (p1 != 0xFFFFFFFFu && (key & mask) == p1) atomicAdd(&h[(kMedBins + bin) * kMedLanes + lane], 1u);
    }
  }
  __syncthreads();
  for (int e = t; e < entries; e += kMedThreads) {
    const uint32_t c = h[e];
    if (!c) continue;
    const int st = e / (kMedBins * kMedLanes);
    const int bin = (e / kMedLanes) % kMedBins;
    const int dd = blockIdx.x * kMedLanes + (e % kMedLanes);
    if (dd < dim) atomicAdd(&m.hist[(size_t(st) * dim + dd) * kMedBins + bin], c);
  }
}

// One warp per dimension: for each statistic, lane l sums bins [8l, 8l + 8)
// of its histogram (the first statistic's when both shared a prefix this
// pass), a warp scan finds the lane whose range holds the remaining rank and
// that lane walks its eight bins; the histograms are cleared for the next
// pass.
__global__ void median_select_kernel(int dim, int nstats, int pass, MedianScratch m) {
  const int d = static_cast<int>((blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (d >= dim) return;  // whole warps
  const int shift = 24 - 8 * pass;
  const bool shared = nstats == 2 && m.prefix[dim + d] == m.prefix[d];
  for (int st = 0; st < nstats; ++st) {
    const int i = st * dim + d;
    const uint4* hh = reinterpret_cast<const uint4*>(m.hist + size_t((st == 1 && shared) ? d : i) * kMedBins);
    const uint4 a = hh[2 * lane], b = hh[2 * lane + 1];
    const uint32_t c[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    int64_t sum = 0;
#pragma unroll
    for (int u = 0; u < 8; ++u) sum += c[u];
    int64_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    const int64_t excl = incl - sum;
    const int64_t rem = m.remaining[i];
    if (excl < rem && rem <= incl) {  // exactly one lane: its bins hold the rank
      int64_t cum = excl;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (cum + c[u] >= rem) {
          m.prefix[i] |= static_cast<uint32_t>(8 * lane + u) << shift;
          m.remaining[i] = rem - cum;
          break;
        }
        cum += c[u];
      }
    }
  }
  __syncwarp();
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int st = 0; st < nstats; ++st) {
    uint4* hh = reinterpret_cast<uint4*>(m.hist + (size_t(st) * dim + d) * kMedBins);
    hh[2 * lane] = z;
    hh[2 * lane + 1] = z;
  }
}

__global__ void median_final_kernel(int dim, int64_t rows, int nstats, MedianScratch m, float* __restrict__ tau) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= dim) return;
  if (rows == 0) {
    tau[d] = 0.0f;
    return;
  }
  const float a = from_total_key(m.prefix[d]);
  tau[d] = nstats == 2 ? __fdiv_rn(__fadd_rn(a, from_total_key(m.prefix[dim + d])), 2.0f) : a;
}

// Widths that are a multiple of 8 on a 16-byte aligned base: each output
// byte's eight values and thresholds as two 16-byte loads each.
__global__ void pack_threshold_bits8_kernel(const float* __restrict__ v, int64_t rows, int dim,
                                            const float* __restrict__ tau, uint8_t* __restrict__ out) {
  const int nb = dim / 8;
  const int64_t total = rows * nb;
  const float4* v4 = reinterpret_cast<const float4*>(v);
  const float4* t4 = reinterpret_cast<const float4*>(tau);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i % nb);
    const float4 x0 = __ldg(v4 + 2 * i), x1 = __ldg(v4 + 2 * i + 1);  // row r, byte b: floats 8i .. 8i + 7
    const float4 a0 = __ldg(t4 + 2 * b), a1 = __ldg(t4 + 2 * b + 1);
    const uint32_t byte = (x0.x > a0.x ? 1u : 0u) | (x0.y > a0.y ? 2u : 0u) | (x0.z > a0.z ? 4u : 0u) |
                          (x0.w > a0.w ? 8u : 0u) | (x1.x > a1.x ? 16u : 0u) | (x1.y > a1.y ? 32u : 0u) |
                          (x1.z > a1.z ? 64u : 0u) | (x1.w > a1.w ? 128u : 0u);
    out[i] = static_cast<uint8_t>(byte);
  }
}

__global__ void pack_threshold_bits_kernel(const float* __restrict__ v, int64_t rows, int dim,
                                           const float* __restrict__ tau, uint8_t* __restrict__ out) {
  const int nb = (dim + 7) / 8;
  const int64_t total = rows * nb;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / nb;
    const int b = static_cast<int>(i - r * nb);
    uint32_t byte = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int dd = b * 8 + k;
      if (dd < dim && __ldg(v + r * dim + dd) > __ldg(tau + dd)) byte |= 1u << k;
    }
    out[i] = static_cast<uint8_t>(byte);
  }
}

// ---- exact search -----------------------------------------------------------

constexpr int kDistRows = 128;  // corpus rows per CTA, one per thread
constexpr int kDistQ = 8;       // queries per CTA
constexpr int kDistChunk = 32;  // dimensions staged per step

// dist[q][row] for queries [q0, q0 + kDistQ) x rows [row0, row0 + 128).
__global__ void __launch_bounds__(kDistRows)
cosine_distance_kernel(const float* __restrict__ corpus, int64_t n, int dim,
                       const float* __restrict__ queries, int nq, float* __restrict__ dist) {
  __shared__ float tile[kDistRows][kDistChunk + 1];
  __shared__ float qs[kDistQ][kDistChunk];
  __shared__ float s_qnorm[kDistQ];
  const int t = threadIdx.x;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kDistRows;
  const int q0 = blockIdx.y * kDistQ;
  const int64_t row = row0 + t;
  float dot[kDistQ];
#pragma unroll
  for (int j = 0; j < kDistQ; ++j) dot[j] = 0.0f;
  float nb = 0.0f, na = 0.0f;  // na: query t's squared norm, threads t < kDistQ
  for (int d0 = 0; d0 < dim; d0 += kDistChunk) {
    const int w = min(kDistChunk, dim - d0);
    for (int e = t; e < kDistRows * kDistChunk; e += kDistRows) {
      const int r = e / kDistChunk, c = e % kDistChunk;
      const int64_t gr = row0 + r;
      tile[r][c] = (gr < n && c < w) ? __ldg(corpus + gr * dim + d0 + c) : 0.0f;
    }
    for (int e = t; e < kDistQ * kDistChunk; e += kDistRows) {
      const int j = e / kDistChunk, c = e % kDistChunk;
      qs[j][c] = (q0 + j < nq && c < w) ? __ldg(queries + static_cast<int64_t>(q0 + j) * dim + d0 + c) : 0.0f;
    }
    __syncthreads();
    for (int c = 0; c < w; ++c) {
      const float x = tile[t][c];
      nb = __fadd_rn(nb, __fmul_rn(x, x));
#pragma unroll
      for (int j = 0; j < kDistQ; ++j) dot[j] = __fadd_rn(dot[j], __fmul_rn(qs[j][c], x));
    }
    if (t < kDistQ)
      for (int c = 0; c < w; ++c) na = __fadd_rn(na, __fmul_rn(qs[t][c], qs[t][c]));
    __syncthreads();
  }
  if (t < kDistQ) s_qnorm[t] = na;
  __syncthreads();
  if (row >= n) return;
  const float sb = __fsqrt_rn(nb);
#pragma unroll
  for (int j = 0; j < kDistQ; ++j) {
    if (q0 + j >= nq) break;
    const float denom = __fmul_rn(__fsqrt_rn(s_qnorm[j]), sb);
    const float dd = denom < FLT_EPSILON ? 1.0f : __fsub_rn(1.0f, __fdiv_rn(dot[j], denom));
    dist[static_cast<int64_t>(q0 + j) * n + row] = dd;
  }
}

constexpr int kTopkThreads = 1024;

// Total-order key of a distance with ties equal: -0 reads as +0, every NaN
// as the positive quiet NaN (after all numbers).
__device__ __forceinline__ uint64_t search_key(float d, uint32_t rank) {
  if (d == 0.0f) d = 0.0f;
  if (d != d) d = __uint_as_float(0x7FC00000u);
  return (static_cast<uint64_t>(total_key(d)) << 32) | rank;
}

constexpr int kTopkCompact = 8192;  // keys a CTA narrows down to in shared memory
constexpr int kTopkDynSmem = kTopkCompact * (8 + 4);

// One CTA per query: the k-th smallest key by radix select (eight 8-bit
// passes), then the keys at or below it, ordered by counting smaller keys.
// Once a pass leaves at most kTopkCompact keys on the chosen prefix, one more
// scan of the row moves them into shared memory (and the keys below the
// prefix, all among the k best, straight to the candidates); the remaining
// passes and the final gather then read shared memory only.
__global__ void __launch_bounds__(kTopkThreads)
topk_kernel(const float* __restrict__ dist, int64_t n, const uint32_t* __restrict__ tie_rank, int k,
            int64_t* __restrict__ out_idx, float* __restrict__ out_dist, int* err) {
  __shared__ uint32_t hist[256];
  __shared__ uint64_t s_prefix, s_mask;
  __shared__ int64_t s_remaining;
  __shared__ uint32_t s_bin_count;
  __shared__ uint64_t cand_key[kMaxSearchK];
  __shared__ int64_t cand_idx[kMaxSearchK];
  __shared__ unsigned s_count, s_m;
  extern __shared__ __align__(16) unsigned char topk_dyn[];
  uint64_t* comp_key = reinterpret_cast<uint64_t*>(topk_dyn);             // [kTopkCompact]
  uint32_t* comp_idx = reinterpret_cast<uint32_t*>(comp_key + kTopkCompact);  // [kTopkCompact]
  const int q = blockIdx.x, t = threadIdx.x;
  const float* dq = dist + static_cast<int64_t>(q) * n;
  const int kk = static_cast<int>(min(static_cast<int64_t>(k), n));
  auto key_of = [&](int64_t i) {
    return search_key(dq[i], tie_rank ? tie_rank[i] : static_cast<uint32_t>(i));
  };
  // f(key, index) over the whole row, eight independent loads in flight per
  // thread (one CTA streams the row alone: latency, not bandwidth, bounds it)
  auto scan_row = [&](auto&& f) {
    constexpr int U = 8;
    const int64_t step = blockDim.x;
    int64_t i = t;
    for (; i + (U - 1) * step < n; i += U * step) {
      float d[U];
      uint32_t rk[U];
#pragma unroll
      for (int u = 0; u < U; ++u) d[u] = __ldg(dq + i + u * step);
#pragma unroll
      for (int u = 0; u < U; ++u)
        rk[u] = tie_rank ? __ldg(tie_rank + i + u * step) : static_cast<uint32_t>(i + u * step);
#pragma unroll
      for (int u = 0; u < U; ++u) f(search_key(d[u], rk[u]), i + u * step);
    }
    for (; i < n; i += step) f(key_of(i), i);
  };
  for (int s = kk + t; s < k; s += blockDim.x) {
    out_idx[static_cast<int64_t>(q) * k + s] = -1;
    out_dist[static_cast<int64_t>(q) * k + s] = __uint_as_float(0x7F800000u);
  }
  if (kk == 0) return;
  if (t == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_remaining = kk;
    s_count = 0;
    s_m = 0;
  }
  bool compacted = false;  // the same in every thread (decided from shared state)
  for (int pass = 0; pass < 8; ++pass) {
    const int shift = 56 - 8 * pass;
    for (int b = t; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    const uint64_t pfx = s_prefix, msk = s_mask;
    auto count = [&](uint64_t key, int64_t) {
      if ((key & msk) == pfx) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    };
    if (!compacted) {
      scan_row(count);
    } else {
      const unsigned m = s_m;
      for (unsigned j = t; j < m; j += blockDim.x) count(comp_key[j], 0);
    }
    __syncthreads();
    if (t == 0) {
      int64_t cum = 0;
      for (int b = 0; b < 256; ++b) {
        if (cum + hist[b] >= s_remaining) {
          s_prefix = pfx | (static_cast<uint64_t>(b) << shift);
          s_mask = msk | (0xFFull << shift);
          s_remaining -= cum;
          s_bin_count = hist[b];
          break;
        }
        cum += hist[b];
      }
    }
    __syncthreads();
    if (!compacted && pass < 7 && s_bin_count <= static_cast<uint32_t>(kTopkCompact)) {
      const uint64_t npfx = s_prefix, nmsk = s_mask;
      scan_row([&](uint64_t key, int64_t i) {
        const uint64_t top = key & nmsk;
        if (top == npfx) {
          const unsigned slot = atomicAdd(&s_m, 1u);
          if (slot < static_cast<unsigned>(kTopkCompact)) {
            comp_key[slot] = key;
            comp_idx[slot] = static_cast<uint32_t>(i);
          }
        } else if (top < npfx) {  // below the prefix: among the k best
          const unsigned slot = atomicAdd(&s_count, 1u);
          if (slot < static_cast<unsigned>(kMaxSearchK)) {
            cand_key[slot] = key;
            cand_idx[slot] = i;
          }
        }
      });
      compacted = true;
      __syncthreads();
    }
  }
  const uint64_t kth = s_prefix;
  if (compacted) {
    const unsigned m = s_m;
    for (unsigned j = t; j < m; j += blockDim.x) {
      const uint64_t key = comp_key[j];
      if (key <= kth) {
        const unsigned slot = atomicAdd(&s_count, 1u);
        if (slot < static_cast<unsigned>(kMaxSearchK)) {
          cand_key[slot] = key;
          cand_idx[slot] = comp_idx[j];
        }
      }
    }
  } else {
    scan_row([&](uint64_t key, int64_t i) {
      if (key <= kth) {
        const unsigned slot = atomicAdd(&s_count, 1u);
        if (slot < static_cast<unsigned>(kMaxSearchK)) {
          cand_key[slot] = key;
          cand_idx[slot] = i;
        }
      }
    });
  }
  __syncthreads();
  if (s_count != static_cast<unsigned>(kk)) {  // repeated ranks: no total order
    if (t == 0) atomicOr(err, kErrTieRank);
    return;
  }
  bool dup = false;
  for (int s = t; s < kk; s += blockDim.x) {
    const uint64_t key = cand_key[s];
    int pos = 0;
    for (int j = 0; j < kk; ++j) {
      pos += cand_key[j] < key || (cand_key[j] == key && j < s);  // a permutation even with repeats
      dup |= j != s && cand_key[j] == key;
    }
    out_idx[static_cast<int64_t>(q) * k + pos] = cand_idx[s];
    out_dist[static_cast<int64_t>(q) * k + pos] = dq[cand_idx[s]];
  }
  if (dup) atomicOr(err, kErrTieRank);  // repeated ranks inside the k: their order is arbitrary
}

}  // namespace

size_t fit_threshold_scratch_bytes(int dim) { return dim > 0 ? median_scratch_bytes_(dim) : 0; }

cudaError_t launch_fit_binary_threshold(const float* v, int64_t rows, int dim, int kind, float* tau,
                                        void* scratch, cudaStream_t s) {
  if (dim <= 0) return cudaSuccess;
  rows = rows < kThresholdSampleCap ? rows : kThresholdSampleCap;
  if (kind == 0) {
    mean_threshold_kernel<<<(dim + 127) / 128, 128, 0, s>>>(v, rows, dim, tau);
    return cudaGetLastError();
  }
  const int nstats = (rows > 0 && rows % 2 == 0) ? 2 : 1;
  const MedianScratch m = carve_median(scratch, dim);
  const unsigned gx = static_cast<unsigned>((dim + kMedLanes - 1) / kMedLanes);
  if (rows > 0) {
    median_init_kernel<<<64, 256, 0, s>>>(dim, rows, nstats, m);
    // about three CTAs per SM over the (dimension group, row split) grid
    const int64_t splits_want = std::max<int64_t>(1, (148 * 3 + gx - 1) / gx);
    int64_t per = (rows + splits_want - 1) / splits_want;
    per = std::max<int64_t>(per, 256);
    const unsigned gy = static_cast<unsigned>((rows + per - 1) / per);
    const int smem = nstats * kMedBins * kMedLanes * static_cast<int>(sizeof(uint32_t));
    cudaError_t e = cudaFuncSetAttribute(median_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    for (int pass = 0; pass < 4; ++pass) {
      median_hist_kernel<<<dim3(gx, gy), kMedThreads, smem, s>>>(v, rows, dim, nstats, pass, per, m);
      median_select_kernel<<<(dim + 7) / 8, 256, 0, s>>>(dim, nstats, pass, m);
    }
  }
  median_final_kernel<<<(dim + 127) / 128, 128, 0, s>>>(dim, rows, nstats, m, tau);
  return cudaGetLastError();
}

cudaError_t launch_pack_threshold_bits(const float* v, int64_t rows, int dim, const float* tau,
                                       uint8_t* out, cudaStream_t s) {
  const int64_t total = rows * ((dim + 7) / 8);
  if (total <= 0) return cudaSuccess;
  const int64_t blocks = (total + 255) / 256;
  const unsigned grid = static_cast<unsigned>(blocks < 148 * 64 ? blocks : 148 * 64);
  if (dim % 8 == 0 && reinterpret_cast<uintptr_t>(v) % 16 == 0 && reinterpret_cast<uintptr_t>(tau) % 16 == 0)
    pack_threshold_bits8_kernel<<<grid, 256, 0, s>>>(v, rows, dim, tau, out);
  else
    pack_threshold_bits_kernel<<<grid, 256, 0, s>>>(v, rows, dim, tau, out);
  return cudaGetLastError();
}

cudaError_t launch_exact_search(const float* corpus, int64_t n, int dim, const uint32_t* tie_rank,
                                const float* queries, int nq, int k, float* scratch, int64_t* out_idx,
                                float* out_dist, int* err, cudaStream_t s) {
  if (nq <= 0 || k <= 0) return cudaSuccess;
  if (n > 0) {
    const dim3 grid(static_cast<unsigned>((n + kDistRows - 1) / kDistRows), (nq + kDistQ - 1) / kDistQ);
    cosine_distance_kernel<<<grid, kDistRows, 0, s>>>(corpus, n, dim, queries, nq, scratch);
  }
  const cudaError_t e = cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTopkDynSmem);
  if (e != cudaSuccess) return e;
  topk_kernel<<<nq, kTopkThreads, kTopkDynSmem, s>>>(scratch, n, tie_rank, k, out_idx, out_dist, err);
  return cudaGetLastError();
}

cudaError_t launch_topk(const float* dist, int64_t n, const uint32_t* tie_rank, int nq, int k,
                        int64_t* out_idx, float* out_dist, int* err, cudaStream_t s) {
  if (nq <= 0 || k <= 0) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTopkDynSmem);
  if (e != cudaSuccess) return e;
  topk_kernel<<<nq, kTopkThreads, kTopkDynSmem, s>>>(dist, n, tie_rank, k, out_idx, out_dist, err);
  return cudaGetLastError();
}

}  // namespace jb
