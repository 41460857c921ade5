// Variable-length self-attention over packed rows.
//
// BertSelfAttention::forward (crates/jammi-encoders/src/bert.rs:135-155)
// computes softmax(Q K^T / sqrt(d) + mask) V on the padded [B, h, S, S]
// score tensor with an additive -10000 mask (mask.rs:14-20).  exp(s - 10000
// - max) underflows to exactly 0 in f32 for |s| << 10^4, so excluding padded
// keys reproduces it; padded query rows are never read by the pooling.  Here
// every (row, head, 64-query block) is one CTA that streams the row's valid
// keys only, with an online softmax in f32 registers.
//
//   flash_attn_bf16_d64: head_dim 64, bf16; QK^T and PV on mma.sync
//                        m16n8k16 tensor-core tiles, K/V double-buffered
//                        through cp.async into 128-byte-swizzled smem.
//   attn_simt:           any head_dim in {8,16,32,64}, f32 or bf16 (the f32
//                        compute precision and the tiny fixtures).
#include <algorithm>
#include <cmath>
#include <atomic>
#include <mutex>
#include <cstring>

#include <cudaTypedefs.h>

#include "jb_common.cuh"
#include "jb_internal.h"

namespace jb {
namespace {

constexpr int kFaRows = 64;     // queries per CTA (16 per warp)
constexpr int kFaKeys = 64;     // keys per pipeline stage
constexpr int kFaThreads = 128;
constexpr int kTileBytes = 64 * 128;  // 64 rows x 64 bf16

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
// Two f32 values as an f16 pair (H16) or a bf16 pair.
template <bool H16>
__device__ __forceinline__ uint32_t pack16(float lo, float hi) {
  if constexpr (H16) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    return pack_bf16(lo, hi);
  }
}
// 64 rows x 8 chunks of 16 B; chunk index XOR (row & 7) avoids bank conflicts.
__device__ __forceinline__ uint32_t swz(uint32_t tile, int row, int chunk) {
  return tile + row * 128 + ((chunk ^ (row & 7)) << 4);
}
// Rows >= rows_valid are zero-filled (cp.async with source size 0).
__device__ __forceinline__ void load_tile(uint32_t tile, const bf16* g, int ld, int rows_valid,
                                          int tid) {
#pragma unroll
  for (int i = tid; i < 64 * 8; i += kFaThreads) {
    const int r = i >> 3, c = i & 7;
    const bool ok = r < rows_valid;
    cp_async16(swz(tile, r, c), ok ? g + static_cast<size_t>(r) * ld + c * 8 : g, ok);
  }
}

// Four CTAs per SM (128 registers, 40 KB shared memory each): the rows are
// short, so the kernel is latency-bound and occupancy is what hides it.
// TMA = false: tiles by cp.async, rows past the row's end zero-filled.
// TMA = true:  one thread loads each tile with one TMA copy (the tensor map
// covers the buffer's row capacity; rows past the row's end hold other rows'
// values and are masked: K by the -inf scores, V zeroed in shared memory in
// the row's last key block so that 0 * V stays 0).
template <bool TMA>
__global__ void __launch_bounds__(kFaThreads, 4)
    flash_attn_bf16_d64(const bf16* __restrict__ qkv, const int* __restrict__ cu,
                        bf16* __restrict__ ctx, int heads, float scale_log2,
                        const __grid_constant__ CUtensorMap tm, int* err, int causal, int skip_le) {
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int start = cu[b], n = cu[b + 1] - start;
  const int q0 = qb * kFaRows;
  if (q0 >= n || n <= skip_le) return;  // rows of <= skip_le keys: the tcgen05 kernel
  const int H = heads * 64, ld = 3 * H;
  __shared__ __align__(1024) uint8_t sm[5 * kTileBytes];
  __shared__ __align__(8) uint64_t bars[2];
  const uint32_t sQ = smem_u32(sm);
  const uint32_t sK0 = sQ + kTileBytes, sV0 = sQ + 2 * kTileBytes;
  const uint32_t sK1 = sQ + 3 * kTileBytes, sV1 = sQ + 4 * kTileBytes;
  const bf16* gQ = qkv + static_cast<size_t>(start + q0) * ld + h * 64;
  const bf16* gK = qkv + static_cast<size_t>(start) * ld + H + h * 64;
  const bf16* gV = gK + H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bar0 = smem_u32(&bars[0]), bar1 = smem_u32(&bars[1]);

  if constexpr (TMA) {
    if (tid == 0) {
      mbar_init(bar0, 1);
      mbar_init(bar1, 1);
      fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
      mbar_arrive_expect_tx(bar0, 3 * kTileBytes);
      tma_load_2d(sQ, &tm, h * 64, start + q0, bar0);
      tma_load_2d(sK0, &tm, H + h * 64, start, bar0);
      tma_load_2d(sV0, &tm, 2 * H + h * 64, start, bar0);
    }
  } else {
    load_tile(sQ, gQ, ld, n - q0, tid);
    load_tile(sK0, gK, ld, n, tid);
    load_tile(sV0, gV, ld, n, tid);
    cp_async_commit();
  }

  // causal: this block's queries see keys up to its own last query, so the
  // key blocks stop at the diagonal one (kFaKeys == kFaRows)
  const int nkb = causal ? min(qb + 1, (n + kFaKeys - 1) / kFaKeys) : (n + kFaKeys - 1) / kFaKeys;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qf[4][4];

  for (int kb = 0; kb < nkb; ++kb) {
    const uint32_t sK = (kb & 1) ? sK1 : sK0, sV = (kb & 1) ? sV1 : sV0;
    if constexpr (TMA) {
      // the other buffer was last read in the previous iteration, which
      // ended with a CTA barrier
      if (kb + 1 < nkb && tid == 0) {
        const uint32_t bar = (kb & 1) ? bar0 : bar1;
        const int row = start + (kb + 1) * kFaKeys;
        mbar_arrive_expect_tx(bar, 2 * kTileBytes);
        tma_load_2d((kb & 1) ? sK0 : sK1, &tm, H + h * 64, row, bar);
        tma_load_2d((kb & 1) ? sV0 : sV1, &tm, 2 * H + h * 64, row, bar);
      }
      // all threads wait for this stage (bounded); a CTA whose wait gave up
      // reports it and leaves as a whole
      volatile int no_abort = 0;
      const bool ok = mbar_wait((kb & 1) ? bar1 : bar0, (kb >> 1) & 1, &no_abort);
      if (__syncthreads_or(!ok)) {
        if (tid == 0 && err) atomicOr(err, kErrTimeout);
        return;
      }
      const int valid = n - kb * kFaKeys;  // V rows of this block inside the row
      if (valid < kFaKeys) {
        for (int i = tid; i < (kFaKeys - valid) * 8; i += kFaThreads) {
          const int r = valid + (i >> 3), c = i & 7;
          asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(swz(sV, r, c)), "r"(0)
                       : "memory");
        }
        __syncthreads();
      }
    } else {
      if (kb + 1 < nkb) {
        const size_t off = static_cast<size_t>(kb + 1) * kFaKeys * ld;
        load_tile((kb & 1) ? sK0 : sK1, gK + off, ld, n - (kb + 1) * kFaKeys, tid);
        load_tile((kb & 1) ? sV0 : sV1, gV + off, ld, n - (kb + 1) * kFaKeys, tid);
        cp_async_commit();
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
    }
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int c = 2 * ks + (lane >> 4);
        ldsm_x4(swz(sQ, r, c), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
      }
    }
    if (q0 + warp * 16 < n) {  // warps past the row's end only load
      // S = Q K^T for this warp's 16 queries x 64 keys
      float s[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[i][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          const int r = np * 16 + (lane & 7) + 8 * (lane >> 4);
          const int c = 2 * ks + ((lane >> 3) & 1);
          ldsm_x4(swz(sK, r, c), b0, b1, b2, b3);
          mma16816(s[2 * np], qf[ks], b0, b1);
          mma16816(s[2 * np + 1], qf[ks], b2, b3);
        }
      }
      // Keys past the row's end (last block only) score -inf; then the online
      // softmax in log2 units, p = 2^(s * scale_log2 - m), the scale folded
      // into one fma per score.
      const int kbase = kb * kFaKeys;
      if (kbase + kFaKeys > n) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (kbase + nt * 8 + 2 * (lane & 3) + (e & 1) >= n) s[nt][e] = -INFINITY;
      }
      if (causal && kb == qb) {  // the diagonal block: key j > query i scores -inf
        const int qr = q0 + warp * 16 + (lane >> 2);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (kbase + nt * 8 + 2 * (lane & 3) + (e & 1) > qr + 8 * (e >> 1)) s[nt][e] = -INFINITY;
      }
      // row maxima and sums as trees (depth 4, not 8): short dependency chains
      float t0[8], t1[8];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        t0[nt] = fmaxf(s[nt][0], s[nt][1]);
        t1[nt] = fmaxf(s[nt][2], s[nt][3]);
      }
#pragma unroll
      for (int w = 4; w > 0; w >>= 1)
#pragma unroll
        for (int nt = 0; nt < w; ++nt) {
          t0[nt] = fmaxf(t0[nt], t0[nt + w]);
          t1[nt] = fmaxf(t1[nt], t1[nt + w]);
        }
      float mx0 = t0[0], mx1 = t1[0];
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0 * scale_log2), mn1 = fmaxf(m1, mx1 * scale_log2);
      const float a0 = ex2_approx(m0 - mn0), a1 = ex2_approx(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      float2 rs[8];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float2 e01 = __ffma2_rn(make_float2(s[nt][0], s[nt][1]), f2(scale_log2), f2(-mn0));
        const float2 e23 = __ffma2_rn(make_float2(s[nt][2], s[nt][3]), f2(scale_log2), f2(-mn1));
        s[nt][0] = ex2_approx(e01.x);
        s[nt][1] = ex2_approx(e01.y);
        s[nt][2] = ex2_approx(e23.x);
        s[nt][3] = ex2_approx(e23.y);
        rs[nt] = __fadd2_rn(make_float2(s[nt][0], s[nt][2]), make_float2(s[nt][1], s[nt][3]));
      }
#pragma unroll
      for (int w = 4; w > 0; w >>= 1)
#pragma unroll
        for (int nt = 0; nt < w; ++nt) rs[nt] = __fadd2_rn(rs[nt], rs[nt + w]);
      const float rs0 = rs[0].x, rs1 = rs[0].y;
      l0 = l0 * a0 + rs0;
      l1 = l1 * a1 + rs1;
      // o is zero before the first block, and unchanged when no row max moved
      if (kb > 0 && __any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
          const float2 o01 = __fmul2_rn(make_float2(o[dt][0], o[dt][1]), f2(a0));
          const float2 o23 = __fmul2_rn(make_float2(o[dt][2], o[dt][3]), f2(a1));
          o[dt][0] = o01.x; o[dt][1] = o01.y; o[dt][2] = o23.x; o[dt][3] = o23.y;
        }
      }
      // O += P V
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
        a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
        a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int dp = 0; dp < 4; ++dp) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
          const int c = 2 * dp + (lane >> 4);
          ldsm_x4_t(swz(sV, r, c), b0, b1, b2, b3);
          mma16816(o[2 * dp], a, b0, b1);
          mma16816(o[2 * dp + 1], a, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = 1.f / l0, i1 = 1.f / l1;
  const int r0 = q0 + warp * 16 + (lane >> 2), r1 = r0 + 8;
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) {
    const int col = h * 64 + dt * 8 + 2 * (lane & 3);
    if (r0 < n)
      *reinterpret_cast<__nv_bfloat162*>(ctx + static_cast<size_t>(start + r0) * H + col) =
          __floats2bfloat162_rn(o[dt][0] * i0, o[dt][1] * i0);
    if (r1 < n)
      *reinterpret_cast<__nv_bfloat162*>(ctx + static_cast<size_t>(start + r1) * H + col) =
          __floats2bfloat162_rn(o[dt][2] * i1, o[dt][3] * i1);
  }
}

// ── tcgen05 attention, any row length ──────────────────────────────────────
// A persistent, warp-specialised kernel: one CTA per SM pulls (row, head)
// units from a device counter, splits each into items of 128 queries, and
// streams the row's keys through each item in blocks of 128 with an online
// softmax.
//   warp 0  (TMA): takes the next unit (the counter read two units ahead,
//           the row offsets one unit ahead), publishes each item in a
//           4-entry ring in shared memory (an end entry per slot finishes
//           the walk), loads the item's Q (64-row boxes) into its slot's Q
//           buffer, then each key block's K and V into a 4-stage ring.
//   warps 1, 2 (MMA, one per slot): S = Q K_j^T (kind::f16, M = 128, N = the block's
//           keys rounded up to 16, four K = 16 steps) into the slot's TMEM
//           columns [0, 128), S_{j+1} as soon as the softmax has read S_j
//           (before it computes P_j, so the next S is ready when it ends);
//           once P_j is written (bf16 pairs, columns [192, 256)), O (+)=
//           P_j V_j with A = P from TMEM and B = V_j MN-major straight from
//           its TMA tile, into columns [128, 192).  One issuing thread per
//           slot, so the two slots' MMAs are issued side by side.
//   warps 3-10 and 11-18 (softmax, one group per slot; items alternate
//           slots): warp w reads TMEM lanes 32 (w % 4) .. + 31, and the two
//           warps of a group on the same lane quarter split each row's key
//           chunks (even / odd 16-key chunks), so two threads serve a query
//           row and exchange their partial maxima and sums through shared
//           memory (an mbarrier of two arrivals per exchange).  Per key block a thread
//           reads its chunks of S twice, two 16-key chunks at a time (once
//           for the maximum, once for the exponentials), masks keys past the
//           row's end (and
//           past the query when causal) in the block that has them, takes the
//           block maximum, and computes p = 2^(s log2(e) / 8 - m) against a
//           reference maximum m: the first block's maximum, raised only when
//           a later block exceeds it by more than 8 (2^8: p stays far inside
//           bf16 and f32), the row of O in TMEM and the running sum rescaled
//           then (lazy rescaling; P_{j-1} V is waited for before O or P is
//           touched).  P goes to TMEM as bf16 pairs.  After the last block,
//           O / sum is stored.
//           The group also zeroes V rows past the row's end in the block's
//           tile (other rows' values: 0 * V must stay 0).
// Every wait is bounded; on a timeout each role stops, the TMA and MMA
// threads wait (bounded) for their copies and MMAs in flight, the error flag
// is set and TMEM is freed.
constexpr int kAtQ = 128;            // queries per item
constexpr int kAtKB = 128;           // keys per block
constexpr int kAtStages = 4;         // K / V ring
constexpr int kAtSlotCols = 256;     // TMEM columns per slot; two slots
constexpr int kAtOCol = 128;         // O's first column inside a slot (S at [0, 128))
constexpr int kAtPCol = 192;         // P's first column inside a slot (bf16 pairs)
constexpr int kAtGroupWarps = 8;     // two warps per TMEM lane quarter: two threads per row
constexpr int kAtThreads = 96 + 2 * 32 * kAtGroupWarps;  // TMA warp, two MMA warps, softmax
constexpr int kAtQBytes = kAtQ * 128;                  // 16 KB
constexpr int kAtKBytes = kAtKB * 128;                 // 16 KB (K or V of a block)
constexpr int kAtMetaBytes = 512 + 2 * 2 * 4 * 2 * 32 * 4 + 2 * 4 * 2 * 32 * 4;  // barriers, ring, exchange
constexpr int kAtSmem = 1024 + 2 * kAtQBytes + kAtStages * 2 * kAtKBytes + kAtMetaBytes;
constexpr float kAtRescale = 8.f;    // lazy-rescaling threshold, log2 units

// One published work item (idx < 0: no more for this slot).  b0 = index of
// its first key block in the K / V stream, nb = its key blocks.
struct AtItem {
  int idx, start, n, h, q0, b0, nb;
};

// A bounded barrier wait whose outcome is the same for every lane of the
// warp (false if any lane gave up), so that no warp-collective tcgen05
// instruction after it is reached by only part of the warp.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort));
}

__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_32x32b_x16_at(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// H16: Q, K, V, P and the context are f16 (else bf16).
template <bool H16>
__global__ void __launch_bounds__(kAtThreads, 1)
    attn_tc_kernel(const int* __restrict__ cu, bf16* __restrict__ ctx, int batch, int heads,
                   float scale_log2, const __grid_constant__ CUtensorMap tm, int* err,
                   int causal, unsigned int* work) {
  const int H = heads * 64;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  const uint32_t sQ0 = base;                                   // [2][16 KB]
  const uint32_t sKV0 = base + 2 * kAtQBytes;                  // [4][K 16 KB | V 16 KB]
  uint8_t* meta = smem_raw + (sKV0 + kAtStages * 2 * kAtKBytes - raw);
  const uint32_t bars = smem_u32(meta);
  // barriers: q_full[2] q_empty[2] s_full[2] p_full[2] o_full[2] s_used[2]
  // k_full[4] v_full[4] kv_empty[4] spare[2] pair[8][2]
  auto qfull = [&](int s) { return bars + 8u * (0 + s); };
  auto qempty = [&](int s) { return bars + 8u * (2 + s); };
  auto sfull = [&](int s) { return bars + 8u * (4 + s); };
  auto pfull = [&](int s) { return bars + 8u * (6 + s); };
  auto ofull = [&](int s) { return bars + 8u * (8 + s); };
  auto sused = [&](int s) { return bars + 8u * (10 + s); };  // the softmax has read S_j
  auto kfull = [&](int st) { return bars + 8u * (12 + st); };
  auto vfull = [&](int st) { return bars + 8u * (16 + st); };
  auto kvempty = [&](int st) { return bars + 8u * (20 + st); };
  const uint32_t spare = bars + 8u * 24;  // [2], one per MMA warp
  // the two warps of a row meet here to exchange maxima and sums: [2 g][4 q]
  auto pairbar = [&](int g, int q) { return bars + 8u * (26 + 4 * g + q); };
  uint32_t* tslot_ptr = reinterpret_cast<uint32_t*>(meta + 8 * 34);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(meta + 8 * 34 + 4);
  volatile AtItem* ring = reinterpret_cast<volatile AtItem*>(meta + 384);  // [4]
  // the two threads of a row exchange their partial maxima (per key block,
  // double-buffered by block parity) and sums (per item) here
  volatile float* xmax = reinterpret_cast<volatile float*>(meta + 512);       // [2 g][2 par][4 q][2 half][32]
  volatile float* xsum = xmax + 2 * 2 * 4 * 2 * 32;                            // [2 g][4 q][2 half][32]
  static_assert(8 * 34 + 8 <= 384 && 384 + 4 * sizeof(AtItem) <= 512, "meta layout");
  auto sK = [&](int st) { return sKV0 + static_cast<uint32_t>(st) * 2 * kAtKBytes; };
  auto sV = [&](int st) { return sKV0 + static_cast<uint32_t>(st) * 2 * kAtKBytes + kAtKBytes; };

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(qfull(s), 1);
      mbar_init(qempty(s), 1 + kAtGroupWarps);  // the last S MMA's commit + the group's warps
      mbar_init(sfull(s), 1);
      mbar_init(pfull(s), kAtGroupWarps);
      mbar_init(ofull(s), 1);
      mbar_init(sused(s), kAtGroupWarps);
    }
    for (int st = 0; st < kAtStages; ++st) {
      mbar_init(kfull(st), 1);
      mbar_init(vfull(st), 1);
      mbar_init(kvempty(st), 1);
    }
    mbar_init(spare, 1);
    mbar_init(spare + 8u, 1);
    for (int i = 0; i < 8; ++i) mbar_init(pairbar(i >> 2, i & 3), 2);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tslot_ptr), 2 * kAtSlotCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot_ptr;

  if (warp == 0) {
    if (lane == 0) {  // ── TMA producer
      // Work units are (row, head) pairs from the device counter, expanded
      // here into their 128-query items.  The counter is read two units
      // ahead and a unit's row offsets one unit ahead, so neither round trip
      // sits between two items.
      const unsigned units = static_cast<unsigned>(batch) * heads;
      // a_next < a_after < later fetches (one thread's atomics return
      // increasing values), so a_next >= units means this CTA has no units left
      unsigned a_next = atomicAdd(work, 1u);
      unsigned a_after = atomicAdd(work, 1u);  // the unit after the next
      int next_start = 0, next_n = 0;
      if (a_next < units) {
        const int b = static_cast<int>(a_next) / heads;
        next_start = cu[b];
        next_n = cu[b + 1] - next_start;
      }
      int k = 0, bc = 0, ends = 0;
      int cur_start = 0, cur_n = 0, cur_h = 0, cur_q0 = 0, cur_qend = 0;  // items q0 < cur_qend left
      bool ok = true;
      while (ends < 2 && ok) {
        const int sl = k & 1;
        if (!mbar_wait(qempty(sl), ((k >> 1) & 1) ^ 1u, abort_flag)) break;
        AtItem it{-1, 0, 0, 0, 0, 0, 0};
        if (ends == 0) {
          while (cur_q0 >= cur_qend && a_next < units) {  // the next unit with rows
            cur_start = next_start;
            cur_n = next_n;
            cur_h = static_cast<int>(a_next) % heads;
            cur_q0 = 0;
            cur_qend = cur_n;
            a_next = a_after;  // returned long ago: issued a unit earlier
            if (a_next < units) {
              const int b = static_cast<int>(a_next) / heads;
              next_start = cu[b];  // used one unit later
              next_n = cu[b + 1] - next_start;
              a_after = atomicAdd(work, 1u);
            }
          }
          if (cur_q0 < cur_qend) {
            const int nk = (cur_n + kAtKB - 1) / kAtKB;
            const int qb = cur_q0 / kAtQ;
            it = AtItem{1, cur_start, cur_n, cur_h, cur_q0, bc, causal ? min(nk, qb + 1) : nk};
            cur_q0 += kAtQ;
          }
        }
        volatile AtItem& e = ring[k & 3];
        e.idx = it.idx;
        e.start = it.start;
        e.n = it.n;
        e.h = it.h;
        e.q0 = it.q0;
        e.b0 = it.b0;
        e.nb = it.nb;
        if (it.idx < 0) {  // published by the barrier's release
          mbar_arrive(qfull(sl));
          ++ends;
          ++k;
          continue;
        }
        const uint32_t sQ = sQ0 + static_cast<uint32_t>(sl) * kAtQBytes;
        const int qboxes = min(2, (it.n - it.q0 + 63) >> 6);
        mbar_arrive_expect_tx(qfull(sl), static_cast<uint32_t>(qboxes) * kTileBytes);
        for (int i = 0; i < qboxes; ++i)
          tma_load_2d(sQ + i * kTileBytes, &tm, it.h * 64, it.start + it.q0 + 64 * i, qfull(sl));
        for (int j = 0; j < it.nb; ++j, ++bc) {
          const int st = bc % kAtStages;
          if (!mbar_wait(kvempty(st), ((bc / kAtStages) & 1) ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          const int kn = min(kAtKB, it.n - kAtKB * j);
          const int boxes = (((kn + 15) & ~15) + 63) >> 6;
          const int row = it.start + kAtKB * j;
          mbar_arrive_expect_tx(kfull(st), static_cast<uint32_t>(boxes) * kTileBytes);
          for (int i = 0; i < boxes; ++i)
            tma_load_2d(sK(st) + i * kTileBytes, &tm, H + it.h * 64, row + 64 * i, kfull(st));
          mbar_arrive_expect_tx(vfull(st), static_cast<uint32_t>(boxes) * kTileBytes);
          for (int i = 0; i < boxes; ++i)
            tma_load_2d(sV(st) + i * kTileBytes, &tm, 2 * H + it.h * 64, row + 64 * i, vfull(st));
        }
        ++k;
      }
      if (*abort_flag) {
        // copies in flight land before the CTA leaves (bounded)
        volatile int no_abort = 0;
        for (int i = max(0, k - 2); i < k; ++i) mbar_wait(qfull(i & 1), (i >> 1) & 1, &no_abort);
        for (int b = max(0, bc - kAtStages); b < bc; ++b) {
          mbar_wait(kfull(b % kAtStages), (b / kAtStages) & 1, &no_abort);
          mbar_wait(vfull(b % kAtStages), (b / kAtStages) & 1, &no_abort);
        }
      }
    }
  } else if (warp <= 2) {
    if (lane == 0) {  // ── MMA issuer of slot warp - 1 (items k with k % 2 == slot)
      const int sl = warp - 1;
      const uint32_t slot = tbase + static_cast<uint32_t>(sl * kAtSlotCols);
      const uint32_t sQ = sQ0 + static_cast<uint32_t>(sl) * kAtQBytes;
      // B (V) MN-major
      const uint32_t idesc_pv = (H16 ? idesc_f16_f32(kAtQ, 64) : idesc_bf16_f32(kAtQ, 64)) | (1u << 16);
      int bs = 0;  // key blocks done in this slot (P V issued)
      int su = 0;  // S issued in this slot (each but the latest released by s_used before the next)
      bool ok = true;
      for (int ti = 0; ok; ++ti) {
        const int k = 2 * ti + sl;
        if (!mbar_wait(qfull(sl), ti & 1, abort_flag)) {
          ok = false;
          break;
        }
        if (ring[k & 3].idx < 0) break;  // the walk is over
        const int n = ring[k & 3].n, b0 = ring[k & 3].b0, nb = ring[k & 3].nb;
        // S_j overwrites S_{j-1} as soon as the softmax has read it (s_used),
        // which is before it computes P_{j-1}: S_j is issued while those
        // exponentials run, and P_{j-1} V once P_{j-1} is written.  The
        // softmax waits for P_{j-1} V before it writes P_j or touches O (and
        // P_0 V, which overwrites O, follows P_0, written after the previous
        // item's epilogue read O).
        auto issue_s = [&](int j) -> bool {
          const int b = b0 + j, st = b % kAtStages;
          const int kn = min(kAtKB, n - kAtKB * j), kpad = (kn + 15) & ~15;
          if ((su > 0 && !mbar_wait(sused(sl), (su - 1) & 1, abort_flag)) ||
              !mbar_wait(kfull(st), (b / kAtStages) & 1, abort_flag))
            return false;
          tc_fence_after();
          const uint32_t idesc = H16 ? idesc_f16_f32(kAtQ, kpad) : idesc_bf16_f32(kAtQ, kpad);
          // a 32-byte K step advances each descriptor's start address by 2
          const uint64_t dq = umma_desc_sw128(sQ), dk = umma_desc_sw128(sK(st));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_bf16(slot, dq + 2u * kk, dk + 2u * kk, idesc, kk != 0);
          mma_commit(sfull(sl));
          if (j == nb - 1) mma_commit(qempty(sl));  // Q read by the item's last S
          ++su;
          return true;
        };
        if (!issue_s(0)) {
          ok = false;
          break;
        }
        for (int j = 0; j < nb && ok; ++j, ++bs) {
          const int b = b0 + j, st = b % kAtStages;
          const int kn = min(kAtKB, n - kAtKB * j), kpad = (kn + 15) & ~15;
          if ((j + 1 < nb && !issue_s(j + 1)) || !mbar_wait(pfull(sl), bs & 1, abort_flag) ||
              !mbar_wait(vfull(st), (b / kAtStages) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // 16 keys of V (16 rows of 128 bytes) advance the start address by 128
          const uint64_t dv = umma_desc_sw128(sV(st));
#pragma unroll 1
          for (int c = 0; c < (kpad >> 4); ++c)
            mma_bf16_ta(slot + kAtOCol, slot + kAtPCol + 8u * c, dv + 128u * c, idesc_pv,
                        (j > 0 || c > 0) ? 1u : 0u);
          mma_commit(ofull(sl));
          mma_commit(kvempty(st));
        }
      }
      if (!ok) {
        // every MMA issued completes before TMEM is freed (bounded)
        volatile int no_abort = 0;
        mma_commit(spare + 8u * sl);
        mbar_wait(spare + 8u * sl, 0, &no_abort);
      }
    }
  } else {  // ── softmax / epilogue groups
    const int gw = (warp - 3) % kAtGroupWarps;
    const int g = (warp - 3) / kAtGroupWarps;          // slot: items k with k % 2 == g
    const int quarter = warp & 3;                       // TMEM lanes 32 quarter .. + 31
    const int half = gw >> 2;                           // this thread's key chunks: t % 2 == half
    const int gtid = tid - 96 - g * 32 * kAtGroupWarps;  // 0 .. 255
    const int r = 32 * quarter + lane;                  // query row of the item
    const uint32_t trow = tbase + static_cast<uint32_t>(g * kAtSlotCols) + (static_cast<uint32_t>(32 * quarter) << 16);
    auto xm = [&](int par, int hf) { return xmax + (((g * 2 + par) * 4 + quarter) * 2 + hf) * 32 + lane; };
    auto xs = [&](int hf) { return xsum + ((g * 4 + quarter) * 2 + hf) * 32 + lane; };
    // the row's other warp has written its half too (bounded: a partner that
    // gave up cannot strand this warp)
    int pairs = 0;
    auto pair_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(pairbar(g, quarter));
      return warp_wait(pairbar(g, quarter), (pairs++) & 1, abort_flag);
    };
    int bs = 0;  // key blocks done in this slot
    bool ok = true;
    for (int ti = 0; ok; ++ti) {
      const int k = 2 * ti + g;
      if (!warp_wait(qfull(g), ti & 1, abort_flag)) break;
      const int idx = ring[k & 3].idx;
      const int start = ring[k & 3].start, n = ring[k & 3].n, h = ring[k & 3].h, q0 = ring[k & 3].q0;
      const int b0 = ring[k & 3].b0, nb = ring[k & 3].nb;
      __syncwarp();
      if (idx < 0) break;  // the walk is over
      if (lane == 0) mbar_arrive(qempty(g));  // this warp has read the ring entry
      const int qi = q0 + r;
      const bool wactive = q0 + 32 * quarter < n;  // uniform over the row's two warps
      const int kmax = qi < n ? (causal ? min(n, qi + 1) : n) : 0;  // keys this row sees
      float mref = -INFINITY, l = 0.f;
      for (int jb = 0; jb < nb; ++jb, ++bs) {
        const int kbase = kAtKB * jb, kn = min(kAtKB, n - kbase), kpad = (kn + 15) & ~15;
        if (kpad > kn) {  // the row's last block: V rows [kn, kpad) -> 0
          const int b = b0 + jb, st = b % kAtStages;
          if (!warp_wait(vfull(st), (b / kAtStages) & 1, abort_flag)) {
            ok = false;
            break;
          }
          for (int i = gtid; i < (kpad - kn) * 8; i += 32 * kAtGroupWarps) {
            const uint32_t a = sV(st) + static_cast<uint32_t>(kn + (i >> 3)) * 128 + (i & 7) * 16;
            asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0) : "memory");
          }
          fence_proxy_async_smem();
        }
        if (!warp_wait(sfull(g), bs & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // this block's S read (all of it, by this warp): S_{j+1} may go in
        bool s_released = false;
        auto release_s = [&]() {
          if (!s_released) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sused(g));
            s_released = true;
          }
        };
        // this thread's chunks: t = half + 2u, u < mine; read in pairs (32
        // values live), once for the maximum and once for the exponentials
        const int chunks = kpad >> 4, mine = (chunks - half + 1) >> 1;
        const int lim = kmax - kbase;  // this row's valid columns in the block
        float m = -INFINITY;
        if (wactive) {
#pragma unroll
          for (int u0 = 0; u0 < 4; u0 += 2) {
            if (u0 < mine) {
              uint32_t v[2][16];
#pragma unroll
              for (int uu = 0; uu < 2; ++uu)
                if (u0 + uu < mine) tmem_ld_32x32b_x16_at(trow + 16 * (2 * (u0 + uu) + half), v[uu]);
              tmem_wait_ld();
#pragma unroll
              for (int uu = 0; uu < 2; ++uu) {
                if (u0 + uu < mine) {
                  const int c0 = 16 * (2 * (u0 + uu) + half);
                  if (c0 + 16 <= lim) {  // no masked key in this chunk
                    float a = fmaxf(__uint_as_float(v[uu][0]), __uint_as_float(v[uu][1]));
#pragma unroll
                    for (int e = 2; e < 16; e += 2)
                      a = fmaxf(a, fmaxf(__uint_as_float(v[uu][e]), __uint_as_float(v[uu][e + 1])));
                    m = fmaxf(m, a);
                  } else {
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                      if (c0 + e < lim) m = fmaxf(m, __uint_as_float(v[uu][e]));
                  }
                }
              }
            }
          }
          *xm(bs & 1, half) = m;
          if (!pair_sync()) {
            ok = false;
            break;
          }
          m = fmaxf(m, *xm(bs & 1, half ^ 1));
        }
        // P_{j-1} V is complete before this block writes P or touches O
        if (jb > 0) {
          if (!warp_wait(ofull(g), (bs - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (wactive) {
          const float mb = m * scale_log2;
          if (jb == 0) {
            mref = mb == -INFINITY ? 0.f : mb;  // a row with no key here keeps p = 0
          } else {
            // lazy rescaling: a row whose block maximum exceeds its reference
            // by more than the threshold moves O and the sum to the new
            // reference; each thread of the row rescales its half of O
            // (columns 32 half .. + 31) and its partial sum.  TMEM loads and
            // stores are warp-collective: the whole warp runs the loop, with
            // alpha = 1 on other rows (both warps of a row decide alike).
            const bool up = mb > mref + kAtRescale;
            if (__any_sync(0xffffffffu, up)) {
              const float alpha = up ? ex2_approx(mref - mb) : 1.f;
              l *= alpha;
#pragma unroll 1
              for (int c = 0; c < 32; c += 8) {
                uint32_t w8[8];
                tmem_ld_32x32b_x8(trow + kAtOCol + 32 * half + c, w8);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 8; ++e) w8[e] = __float_as_uint(__uint_as_float(w8[e]) * alpha);
                tmem_st_32x32b_x8(trow + kAtOCol + 32 * half + c, w8);
              }
              tmem_wait_st();
              if (up) mref = mb;
            }
          }
          float lsum0 = 0.f, lsum1 = 0.f;
#pragma unroll
          for (int u0 = 0; u0 < 4; u0 += 2) {
            if (u0 < mine) {
              uint32_t v[2][16];
#pragma unroll
              for (int uu = 0; uu < 2; ++uu)
                if (u0 + uu < mine) tmem_ld_32x32b_x16_at(trow + 16 * (2 * (u0 + uu) + half), v[uu]);
              tmem_wait_ld();
              if (u0 + 2 >= mine) release_s();  // the last of this thread's S reads
#pragma unroll
              for (int uu = 0; uu < 2; ++uu) {
                if (u0 + uu < mine) {
                  const int t = 2 * (u0 + uu) + half, c0 = 16 * t;
                  const bool full = c0 + 16 <= lim;  // no masked key in this chunk
                  uint32_t pk[8];
#pragma unroll
                  for (int e = 0; e < 16; e += 2) {
                    float2 z = __ffma2_rn(make_float2(__uint_as_float(v[uu][e]), __uint_as_float(v[uu][e + 1])),
                                          f2(scale_log2), f2(-mref));
                    if (!full) {  // keys past the row's end (or the query)
                      if (c0 + e >= lim) z.x = -INFINITY;
                      if (c0 + e + 1 >= lim) z.y = -INFINITY;
                    }
                    const float p0 = ex2_approx(z.x), p1 = ex2_approx(z.y);
                    lsum0 += p0;
                    lsum1 += p1;
                    pk[e >> 1] = pack16<H16>(p0, p1);
                  }
                  tmem_st_32x32b_x8(trow + kAtPCol + 8 * t, pk);
                }
              }
            }
          }
          l += lsum0 + lsum1;
          tmem_wait_st();
        }
        release_s();  // warps without reads in this pass
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pfull(g));
      }
      if (!ok) break;
      if (!warp_wait(ofull(g), (bs - 1) & 1, abort_flag)) break;
      tc_fence_after();
      if (wactive) {
        *xs(half) = l;
        if (!pair_sync()) break;
        const float inv_l = 1.f / (l + *xs(half ^ 1));
        uint32_t o[32];
        tmem_ld_32x32b_x32(trow + kAtOCol + 32 * half, o);
        tmem_wait_ld();
        if (qi < n) {
          uint4* dst = reinterpret_cast<uint4*>(ctx + static_cast<size_t>(start + qi) * H + h * 64 + 32 * half);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 wv;
            wv.x = pack16<H16>(__uint_as_float(o[8 * q + 0]) * inv_l, __uint_as_float(o[8 * q + 1]) * inv_l);
            wv.y = pack16<H16>(__uint_as_float(o[8 * q + 2]) * inv_l, __uint_as_float(o[8 * q + 3]) * inv_l);
            wv.z = pack16<H16>(__uint_as_float(o[8 * q + 4]) * inv_l, __uint_as_float(o[8 * q + 5]) * inv_l);
            wv.w = pack16<H16>(__uint_as_float(o[8 * q + 6]) * inv_l, __uint_as_float(o[8 * q + 7]) * inv_l);
            dst[q] = wv;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag && err) atomicOr(err, kErrTimeout);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 2 * kAtSlotCols);
  }
}

constexpr int kSimtRows = 64;
constexpr int kSimtKeys = 64;

template <typename T, int D>
__global__ void __launch_bounds__(kSimtRows) attn_simt(const T* __restrict__ qkv,
                                                      const int* __restrict__ cu,
                                                      T* __restrict__ ctx, int heads, float scale,
                                                      int causal) {
  const int b = blockIdx.z, h = blockIdx.y;
  const int start = cu[b], n = cu[b + 1] - start;
  if (blockIdx.x * kSimtRows >= n) return;
  const int q = blockIdx.x * kSimtRows + threadIdx.x;
  const int H = heads * D, ld = 3 * H;
  __shared__ float Ks[kSimtKeys][D + 1];
  __shared__ float Vs[kSimtKeys][D + 1];
  const bool active = q < n;
  float qv[D], o[D];
  float m = -INFINITY, l = 0.f;
#pragma unroll
  for (int d = 0; d < D; ++d) {
    qv[d] = active ? to_f(qkv[static_cast<size_t>(start + q) * ld + h * D + d]) : 0.f;
    o[d] = 0.f;
  }
  for (int k0 = 0; k0 < n; k0 += kSimtKeys) {
    __syncthreads();
    for (int i = threadIdx.x; i < kSimtKeys * D; i += kSimtRows) {
      const int r = i / D, d = i % D;
      const bool ok = k0 + r < n;
      const size_t base = static_cast<size_t>(start + k0 + r) * ld + h * D + d;
      Ks[r][d] = ok ? to_f(qkv[base + H]) : 0.f;
      Vs[r][d] = ok ? to_f(qkv[base + 2 * H]) : 0.f;
    }
    __syncthreads();
    if (active) {
      const int kn = causal ? min(min(kSimtKeys, n - k0), q - k0 + 1) : min(kSimtKeys, n - k0);
      for (int j = 0; j < kn; ++j) {
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < D; ++d) s = fmaf(qv[d], Ks[j][d], s);
        s *= scale;
        const float mn = fmaxf(m, s);
        const float corr = expf(m - mn);
        const float p = expf(s - mn);
        l = l * corr + p;
#pragma unroll
        for (int d = 0; d < D; ++d) o[d] = fmaf(p, Vs[j][d], o[d] * corr);
        m = mn;
      }
    }
  }
  if (active) {
    const float inv = 1.f / l;
#pragma unroll
    for (int d = 0; d < D; ++d)
      ctx[static_cast<size_t>(start + q) * H + h * D + d] = from_f<T>(o[d] * inv);
  }
}

template <typename T>
cudaError_t launch_simt(const void* qkv, const int* cu, void* ctx, int batch, int heads, int d,
                        int max_len, cudaStream_t s, std::string* why, int causal) {
  dim3 grid((max_len + kSimtRows - 1) / kSimtRows, heads, batch);
  const float scale = 1.0f / sqrtf(static_cast<float>(d));
  const T* q = static_cast<const T*>(qkv);
  T* c = static_cast<T*>(ctx);
  switch (d) {
    case 8: attn_simt<T, 8><<<grid, kSimtRows, 0, s>>>(q, cu, c, heads, scale, causal); break;
    case 16: attn_simt<T, 16><<<grid, kSimtRows, 0, s>>>(q, cu, c, heads, scale, causal); break;
    case 32: attn_simt<T, 32><<<grid, kSimtRows, 0, s>>>(q, cu, c, heads, scale, causal); break;
    case 64: attn_simt<T, 64><<<grid, kSimtRows, 0, s>>>(q, cu, c, heads, scale, causal); break;
    default:
      if (why) *why = "attention: head_dim must be 8, 16, 32 or 64";
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// 2-D map over qkv [rows, 3 * H] bf16 with one 64 x 64 box (128-byte rows,
// 128-byte swizzle: the layout swz() reads).
bool make_qkv_map(CUtensorMap* map, const void* qkv, int rows, int H, bool h16 = false) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  if (!enc || (reinterpret_cast<uintptr_t>(qkv) & 15)) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(3) * H, static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(3) * H * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, h16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
             const_cast<void*>(qkv), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

std::atomic<int> g_attn_tc{1};  // jb_set_attention_tcgen05 (on by default)
bool attn_tc_enabled() { return g_attn_tc.load(std::memory_order_relaxed) != 0; }

template <bool H16>
cudaError_t launch_tc(int grid, cudaStream_t s, const int* cu, bf16* ctx, int batch, int heads,
                      float scale_log2, const CUtensorMap& tm, int* err, int causal,
                      unsigned int* work) {
  // the shared-memory opt-in is a property of each device's context
  static std::atomic<uint8_t> attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev].load(std::memory_order_acquire)) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_tc_kernel<H16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kAtSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev].store(1, std::memory_order_release);
  }
  attn_tc_kernel<H16><<<grid, kAtThreads, kAtSmem, s>>>(cu, ctx, batch, heads, scale_log2, tm, err,
                                                    causal, work);
  return cudaGetLastError();
}

// Work counters for callers that pass none (the single-op entry points):
// one slot per call, round robin over kWorkSlots, so calls that overlap on the
// GPU get distinct counters unless kWorkSlots of them are in flight at once.
constexpr int kWorkSlots = 64;
__device__ unsigned int g_attn_work[kWorkSlots];
unsigned int* shared_work_counter() {
  static std::mutex mu;
  static unsigned int* base[64] = {};
  static unsigned next = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!base[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_attn_work) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    base[dev] = static_cast<unsigned int*>(p);
  }
  return base[dev] + (next++ % kWorkSlots);
}

}  // namespace

void set_attention_tcgen05(bool on) { g_attn_tc.store(on ? 1 : 0, std::memory_order_relaxed); }

cudaError_t launch_attention(const void* qkv, const int* cu, void* ctx, int dtype, int batch,
                             int heads, int head_dim, int max_len, cudaStream_t s,
                             std::string* why, int rows_cap, int* err, int causal, int* work) {
  if (batch == 0 || max_len == 0) return cudaSuccess;
  if (batch > 65535 || heads > 65535) {
    if (why) *why = "attention: batch and heads must be <= 65535";
    return cudaErrorInvalidValue;
  }
  const bool h16 = dtype == JB_DT_F16;
  if ((dtype == JB_DT_BF16 || h16) && head_dim == 64) {
    dim3 grid((max_len + kFaRows - 1) / kFaRows, heads, batch);
    const float scale_log2 = 1.4426950408889634f / sqrtf(64.f);
    CUtensorMap tm;
    memset(&tm, 0, sizeof(tm));
    const bool tma = rows_cap > 0 && make_qkv_map(&tm, qkv, rows_cap, heads * 64, h16);
    if (tma && attn_tc_enabled()) {
      // every row on tcgen05: 128-query items, keys streamed in blocks of 128
      unsigned int* w = work ? reinterpret_cast<unsigned int*>(work) : shared_work_counter();
      if (!w) {
        if (why) *why = "attention: no work counter";
        return cudaErrorInvalidValue;
      }
      cudaError_t e = cudaMemsetAsync(w, 0, sizeof(unsigned int), s);
      if (e != cudaSuccess) return e;
      int dev = 0;
      cudaGetDevice(&dev);
      int sms = 0;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      const long long units = static_cast<long long>(batch) * heads;  // (row, head) pairs
      const int grid = static_cast<int>(std::max(1ll, std::min<long long>(units, sms > 0 ? sms : 148)));
      return h16 ? launch_tc<true>(grid, s, cu, static_cast<bf16*>(ctx), batch, heads, scale_log2, tm,
                                   err, causal, w)
                 : launch_tc<false>(grid, s, cu, static_cast<bf16*>(ctx), batch, heads, scale_log2, tm,
                                    err, causal, w);
    }
    if (h16) {
      if (why)
        *why = "attention(f16, head_dim 64): runs on the tcgen05 kernel only (a row capacity and "
               "jb_set_attention_tcgen05(1))";
      return cudaErrorInvalidValue;
    }
    const int skip_le = 0;
    auto kern = tma ? flash_attn_bf16_d64<true> : flash_attn_bf16_d64<false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                         cudaSharedmemCarveoutMaxShared);
    kern<<<grid, kFaThreads, 0, s>>>(static_cast<const bf16*>(qkv), cu, static_cast<bf16*>(ctx),
                                     heads, scale_log2, tm, err, causal, skip_le);
    return cudaGetLastError();
  }
  if (dtype == JB_DT_BF16)
    return launch_simt<bf16>(qkv, cu, ctx, batch, heads, head_dim, max_len, s, why, causal);
  if (h16) return launch_simt<f16>(qkv, cu, ctx, batch, heads, head_dim, max_len, s, why, causal);
  if (dtype != JB_DT_F32) {
    if (why) *why = "attention: unsupported dtype";
    return cudaErrorInvalidValue;
  }
  return launch_simt<float>(qkv, cu, ctx, batch, heads, head_dim, max_len, s, why, causal);
}

}  // namespace jb
