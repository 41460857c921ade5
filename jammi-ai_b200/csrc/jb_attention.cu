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

// ── tcgen05 attention for rows of at most 256 keys ──────────────────────────
// A persistent, warp-specialised kernel: one CTA per SM pulls work items
// (row, head, 128-query block) of rows with at most MAXK keys from a device
// counter (dynamic schedule: no SM idles while another still has a queue).
// A row's keys all fit one accumulator, so its softmax is exact in one pass
// (no running rescale).
//   warp 0  (TMA): takes the next item from the counter, publishes it to the
//           other roles in a shared-memory ring beside its stage (an empty
//           entry, twice, ends the walk), and loads Q and K onto one
//           mbarrier, V onto a second, 64-row boxes, into STAGES stages.
//   warp 1  (MMA): S = Q K^T, four kind::f16 MMAs (K = 16) into the item's
//           TMEM slot, columns [0, n_pad), n_pad = the row length rounded up
//           to 16; once the softmax has written P: O = P V, one MMA per
//           16-key chunk with A = P read from TMEM and B = V straight from its
//           TMA tile (MN-major, 128-byte swizzle), into the slot's columns
//           [128, 192).  Each is issued as soon as its inputs are ready
//           (non-blocking probes of the barriers).
//   warps 2-5 and 6-9 (softmax, two groups ping-ponging on alternate items,
//           each with its own 256-column TMEM slot): warp w reads TMEM lanes
//           32 (w % 4) .. + 31, one thread per query row.  The group zeroes
//           the V rows past the row's end (other rows' values: 0 * V must
//           stay 0), reads S in register batches (max; then
//           2^(s log2(e) / 8 - m) and the sum), writes chunk c's P as bf16
//           pairs into columns [8c, 8c + 8) (S columns already consumed: the
//           chunks are read in ascending batches before their P is written;
//           P ends below column 128, where O starts) and, after
//           O = P V, scales the O row by 1 / sum and stores it (128 B).  While
//           one group waits for its O, the other runs its softmax.
// causal != 0 masks keys after the query.  MAXK = 192 keeps three 64 KB
// stages, MAXK = 256 two 80 KB ones.  Longer rows are left to the mma.sync
// kernel; the choice is per row, so a row's result does not depend on its
// batch.  Every wait is bounded; on a timeout each role stops, the
// TMA and MMA threads wait (bounded) for their copies and MMAs in flight,
// the error flag is set and TMEM is freed.
constexpr int kTcQ = 128;         // queries per item
constexpr int kTcSlotCols = 256;  // TMEM columns per slot; two slots
constexpr int kTcOCol = 128;      // O's first column inside a slot
constexpr int kTcGroupWarps = 4;
constexpr int kTcThreads = 64 + 2 * 32 * kTcGroupWarps;
constexpr int kTcBatch = 6;  // 16-column chunks per register batch
template <int MAXK>
constexpr int tc_stage_bytes() { return (kTcQ + 2 * MAXK) * 128; }
template <int MAXK, int STAGES>
constexpr int tc_smem() { return STAGES * tc_stage_bytes<MAXK>() + 1024 + 256 + STAGES * 32; }

// One published work item (or idx < 0: no more).
struct TcItem {
  int idx, start, n, h, q0;
};

template <int MAXK, int STAGES>
__global__ void __launch_bounds__(kTcThreads, 1)
    attn_tc_kernel(const int* __restrict__ cu, bf16* __restrict__ ctx, int batch, int heads,
                   float scale_log2, const __grid_constant__ CUtensorMap tm, int* err, int causal,
                   unsigned int* work) {
  constexpr int kTcStages = STAGES, kTcMaxKeys = MAXK;
  constexpr int kTcStageBytes = tc_stage_bytes<MAXK>();
  const int H = heads * 64;
  const int items = batch * heads * 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t stage0 = (raw + 1023u) & ~1023u;
  uint8_t* meta = smem_raw + (stage0 + kTcStages * kTcStageBytes - raw);
  const uint32_t bars = smem_u32(meta);
  // stage barriers (3 each): ld_qk, ld_v, smem_empty; slot barriers (2 each):
  // s_full, p_full, o_full, tmem_free; one spare
  auto sbar = [&](int kind, int st) { return bars + 8u * (kind * kTcStages + st); };
  auto tbar = [&](int kind, int sl) { return bars + 8u * (3 * kTcStages + kind * 2 + sl); };
  enum { kLdQK = 0, kLdV = 1, kSEmpty = 2 };
  enum { kSFull = 0, kPFull = 1, kOFull = 2, kTFree = 3 };
  const uint32_t spare = bars + 8u * (3 * kTcStages + 8);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(meta + 8 * 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(meta + 8 * 24 + 4);
  volatile TcItem* ring = reinterpret_cast<volatile TcItem*>(meta + 256);  // [STAGES]

  if (tid == 0) {
    for (int st = 0; st < kTcStages; ++st) {
      mbar_init(sbar(kLdQK, st), 1);
      mbar_init(sbar(kLdV, st), 1);
      mbar_init(sbar(kSEmpty, st), 1);
    }
    for (int sl = 0; sl < 2; ++sl) {
      mbar_init(tbar(kSFull, sl), 1);
      mbar_init(tbar(kPFull, sl), kTcGroupWarps);
      mbar_init(tbar(kOFull, sl), 1);
      mbar_init(tbar(kTFree, sl), kTcGroupWarps);
    }
    mbar_init(spare, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(tslot), 2 * kTcSlotCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  auto stage_of = [&](int k) { return stage0 + static_cast<uint32_t>(k % kTcStages) * kTcStageBytes; };

  if (warp == 0) {
    if (lane == 0) {  // ── TMA producer
      int k = 0, ends = 0;
      while (ends < 2) {
        const int st = k % kTcStages;
        const uint32_t ph = (k / kTcStages) & 1;
        if (!mbar_wait(sbar(kSEmpty, st), ph ^ 1u, abort_flag)) break;
        TcItem it{-1, 0, 0, 0, 0};
        if (ends == 0) {
          while (true) {
            const int idx = static_cast<int>(atomicAdd(work, 1u));
            if (idx >= items) break;
            const int bh = idx >> 1, b = bh / heads;
            const int q0 = (idx & 1) * kTcQ, start = cu[b], n = cu[b + 1] - start;
            if (q0 < n && n <= kTcMaxKeys) {
              it = TcItem{idx, start, n, bh - b * heads, q0};
              break;
            }
          }
        }
        ring[st].idx = it.idx;
        ring[st].start = it.start;
        ring[st].n = it.n;
        ring[st].h = it.h;
        ring[st].q0 = it.q0;
        if (it.idx < 0) {  // published by the barriers' release
          mbar_arrive(sbar(kLdQK, st));
          mbar_arrive(sbar(kLdV, st));
          ++ends;
          ++k;
          continue;
        }
        const uint32_t sQ = stage_of(k), sK = sQ + kTcQ * 128, sV = sK + kTcMaxKeys * 128;
        const int n_pad = (it.n + 15) & ~15;
        const int kboxes = (n_pad + 63) >> 6;
        const int qboxes = min(2, (it.n - it.q0 + 63) >> 6);
        mbar_arrive_expect_tx(sbar(kLdQK, st), static_cast<uint32_t>(qboxes + kboxes) * kTileBytes);
        for (int i = 0; i < qboxes; ++i) tma_load_2d(sQ + i * kTileBytes, &tm, it.h * 64, it.start + it.q0 + 64 * i, sbar(kLdQK, st));
        for (int i = 0; i < kboxes; ++i) tma_load_2d(sK + i * kTileBytes, &tm, H + it.h * 64, it.start + 64 * i, sbar(kLdQK, st));
        mbar_arrive_expect_tx(sbar(kLdV, st), static_cast<uint32_t>(kboxes) * kTileBytes);
        for (int i = 0; i < kboxes; ++i) tma_load_2d(sV + i * kTileBytes, &tm, 2 * H + it.h * 64, it.start + 64 * i, sbar(kLdV, st));
        ++k;
      }
      if (*abort_flag) {
        // copies in flight land before the CTA leaves (bounded)
        volatile int no_abort = 0;
        for (int j = max(0, k - kTcStages); j < k; ++j) {
          mbar_wait(sbar(kLdQK, j % kTcStages), (j / kTcStages) & 1, &no_abort);
          mbar_wait(sbar(kLdV, j % kTcStages), (j / kTcStages) & 1, &no_abort);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ── MMA issuer
      // items k with S issued (< ks) and with O = P V issued (< kp); ns[]
      // remembers the row lengths of the items in flight; an empty ring entry
      // (once its Q/K barrier has completed) ends the walk
      int ks = 0, kp = 0;
      int ns[4] = {0, 0, 0, 0};
      bool more = true, ok = true;
      const uint64_t t_limit = kWaitLimitNs;
      uint64_t t0 = global_timer_ns();
      while (ok) {
        bool progress = false;
        // next item whose S can go: its slot free and its Q, K loaded
        if (more && ks - kp < 2) {
          const int sl = ks & 1, st = ks % kTcStages;
          // one probe of the Q/K barrier, then the ring entry decides: an
          // empty entry (n = 0) must never reach an MMA (N = 0 is invalid)
          if (mbar_test_wait(sbar(kLdQK, st), (ks / kTcStages) & 1)) {
            const int n = ring[st].idx < 0 ? 0 : ring[st].n;
            if (n <= 0) {
              more = false;
            } else if (mbar_test_wait(tbar(kTFree, sl), ((ks >> 1) & 1) ^ 1u)) {
              tc_fence_after();
              const uint32_t sQ = stage_of(ks), sK = sQ + kTcQ * 128;
              const uint32_t idesc = idesc_bf16_f32(kTcQ, (n + 15) & ~15);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_bf16(tbase + static_cast<uint32_t>(sl * kTcSlotCols), umma_desc_sw128(sQ + 32u * kk),
                         umma_desc_sw128(sK + 32u * kk), idesc, kk != 0);
              mma_commit(tbar(kSFull, sl));
              ns[ks & 3] = n;
              ++ks;
              progress = true;
            }
          }
        }
        // O = P V of the oldest item whose P is written
        if (kp < ks && mbar_test_wait(tbar(kPFull, kp & 1), (kp >> 1) & 1)) {
          tc_fence_after();
          const int sl = kp & 1;
          const uint32_t sV = stage_of(kp) + kTcQ * 128 + kTcMaxKeys * 128;
          const uint32_t slot = tbase + static_cast<uint32_t>(sl * kTcSlotCols);
          const uint32_t idesc = idesc_bf16_f32(kTcQ, 64) | (1u << 16);  // B (V) MN-major
          const int chunks = ((ns[kp & 3] + 15) & ~15) >> 4;
#pragma unroll 1
          for (int c = 0; c < chunks; ++c)
            mma_bf16_ta(slot + kTcOCol, slot + 8u * c, umma_desc_sw128(sV + 2048u * c), idesc, c != 0);
          mma_commit(tbar(kOFull, sl));
          mma_commit(sbar(kSEmpty, kp % kTcStages));
          ++kp;
          progress = true;
        }
        if (!more && kp == ks) break;
        if (progress) {
          t0 = global_timer_ns();
        } else if (*abort_flag || global_timer_ns() - t0 > t_limit) {
          *abort_flag = 1;
          ok = false;
        }
      }
      // the last commit's arrival lands before the CTA leaves (bounded)
      if (ok && kp > 0) ok = mbar_wait(sbar(kSEmpty, (kp - 1) % kTcStages), ((kp - 1) / kTcStages) & 1, abort_flag);
      if (!ok) {
        // every MMA issued completes before TMEM is freed (bounded)
        volatile int no_abort = 0;
        mma_commit(spare);
        mbar_wait(spare, 0, &no_abort);
      }
    }
  } else {  // ── softmax / epilogue groups
    const int group = (warp - 2) / kTcGroupWarps;       // items k with k % 2 == group
    const int quarter = warp & 3;
    const int gtid = tid - 64 - group * 32 * kTcGroupWarps;  // 0 .. 127
    const int row = 32 * quarter + lane;
    for (int kk = group;; kk += 2) {
      const int st = kk % kTcStages;
      const uint32_t sph = (kk / kTcStages) & 1, tph = (kk >> 1) & 1;
      if (!mbar_wait(sbar(kLdV, st), sph, abort_flag)) break;
      const int idx = ring[st].idx;
      if (idx < 0) break;  // the walk is over
      const int start = ring[st].start, n = ring[st].n, h = ring[st].h, q0 = ring[st].q0;
      const uint32_t sV = stage_of(kk) + kTcQ * 128 + kTcMaxKeys * 128;
      const uint32_t trow = tbase + static_cast<uint32_t>(group * kTcSlotCols) +
                            (static_cast<uint32_t>(32 * quarter) << 16);
      const int n_pad = (n + 15) & ~15, chunks = n_pad >> 4;
      // V rows [n, n_pad) -> 0 (whole 128-byte rows, so the swizzle is moot)
      for (int i = gtid; i < (n_pad - n) * 8; i += 32 * kTcGroupWarps) {
        const uint32_t a = sV + static_cast<uint32_t>(n + (i >> 3)) * 128 + (i & 7) * 16;
        asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0) : "memory");
      }
      fence_proxy_async_smem();
      if (!mbar_wait(tbar(kSFull, group), tph, abort_flag)) break;
      tc_fence_after();
      const int qi = q0 + row;
      const bool active = q0 + 32 * quarter < n;  // warp-uniform
      const int kmax = causal ? min(n, qi + 1) : n;
      float l = 0.f;
      if (active) {
        float m = -INFINITY;
        uint32_t r[kTcBatch][16];
#pragma unroll 1
        for (int c0 = 0; c0 < chunks; c0 += kTcBatch) {
#pragma unroll
          for (int t = 0; t < kTcBatch; ++t)
            if (c0 + t < chunks) tmem_ld_32x32b_x16(trow + 16 * (c0 + t), r[t]);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < kTcBatch; ++t) {
            if (c0 + t < chunks) {
#pragma unroll
              for (int j = 0; j < 16; ++j)
                if (16 * (c0 + t) + j < kmax) m = fmaxf(m, __uint_as_float(r[t][j]));
            }
          }
        }
        const float mb = m * scale_log2;
#pragma unroll 1
        for (int c0 = 0; c0 < chunks; c0 += kTcBatch) {
#pragma unroll
          for (int t = 0; t < kTcBatch; ++t)
            if (c0 + t < chunks) tmem_ld_32x32b_x16(trow + 16 * (c0 + t), r[t]);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < kTcBatch; ++t) {
            if (c0 + t < chunks) {
              const int c = 16 * (c0 + t);
              uint32_t pk[8];
#pragma unroll
              for (int j = 0; j < 16; j += 2) {
                const float p0 = c + j < kmax ? ex2_approx(fmaf(__uint_as_float(r[t][j]), scale_log2, -mb)) : 0.f;
                const float p1 = c + j + 1 < kmax ? ex2_approx(fmaf(__uint_as_float(r[t][j + 1]), scale_log2, -mb)) : 0.f;
                l += p0 + p1;
                pk[j >> 1] = pack_bf16(p0, p1);
              }
              tmem_st_32x32b_x8(trow + (c >> 1), pk);  // consumed S columns [8c', 8c' + 8)
            }
          }
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tbar(kPFull, group));
      if (!mbar_wait(tbar(kOFull, group), tph, abort_flag)) break;
      tc_fence_after();
      if (active) {
        const float inv_l = 1.f / l;
        uint32_t o[32];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          tmem_ld_32x32b_x32(trow + kTcOCol + 32 * half, o);
          tmem_wait_ld();
          if (qi < n) {
            uint4* dst = reinterpret_cast<uint4*>(ctx + static_cast<size_t>(start + qi) * H + h * 64 + 32 * half);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 wv;
              wv.x = pack_bf16(__uint_as_float(o[8 * v + 0]) * inv_l, __uint_as_float(o[8 * v + 1]) * inv_l);
              wv.y = pack_bf16(__uint_as_float(o[8 * v + 2]) * inv_l, __uint_as_float(o[8 * v + 3]) * inv_l);
              wv.z = pack_bf16(__uint_as_float(o[8 * v + 4]) * inv_l, __uint_as_float(o[8 * v + 5]) * inv_l);
              wv.w = pack_bf16(__uint_as_float(o[8 * v + 6]) * inv_l, __uint_as_float(o[8 * v + 7]) * inv_l);
              dst[v] = wv;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tbar(kTFree, group));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag && err) atomicOr(err, kErrTimeout);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 2 * kTcSlotCols);
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
bool make_qkv_map(CUtensorMap* map, const void* qkv, int rows, int H) {
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
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(qkv), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

std::atomic<int> g_attn_tc{0};  // jb_set_attention_tcgen05
bool attn_tc_enabled() { return g_attn_tc.load(std::memory_order_relaxed) != 0; }

template <int MAXK, int STAGES>
cudaError_t launch_tc(int grid, cudaStream_t s, const int* cu, bf16* ctx, int batch, int heads,
                      float scale_log2, const CUtensorMap& tm, int* err, int causal,
                      unsigned int* work) {
  static const bool attr = cudaFuncSetAttribute(attn_tc_kernel<MAXK, STAGES>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                tc_smem<MAXK, STAGES>()) == cudaSuccess;
  if (!attr) return cudaErrorInvalidConfiguration;
  attn_tc_kernel<MAXK, STAGES><<<grid, kTcThreads, tc_smem<MAXK, STAGES>(), s>>>(
      cu, ctx, batch, heads, scale_log2, tm, err, causal, work);
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
  if (dtype == JB_DT_BF16 && head_dim == 64) {
    dim3 grid((max_len + kFaRows - 1) / kFaRows, heads, batch);
    const float scale_log2 = 1.4426950408889634f / sqrtf(64.f);
    CUtensorMap tm;
    memset(&tm, 0, sizeof(tm));
    const bool tma = rows_cap > 0 && make_qkv_map(&tm, qkv, rows_cap, heads * 64);
    int skip_le = 0;  // rows the tcgen05 kernel takes
    if (tma && attn_tc_enabled()) {
      // rows of up to 256 keys: S and P V on tcgen05 (one softmax pass)
      unsigned int* w = work ? reinterpret_cast<unsigned int*>(work) : shared_work_counter();
      cudaError_t e = w ? cudaMemsetAsync(w, 0, sizeof(unsigned int), s) : cudaErrorInvalidValue;
      if (e == cudaSuccess) {
        int dev = 0;
        cudaGetDevice(&dev);
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int items = batch * heads * 2;
        const int grid = std::max(1, std::min(items, sms > 0 ? sms : 148));
        if (max_len <= 192) {
          e = launch_tc<192, 3>(grid, s, cu, static_cast<bf16*>(ctx), batch, heads, scale_log2, tm,
                                err, causal, w);
          skip_le = 192;
        } else {
          e = launch_tc<256, 2>(grid, s, cu, static_cast<bf16*>(ctx), batch, heads, scale_log2, tm,
                                err, causal, w);
          skip_le = 256;
        }
        if (e != cudaSuccess) return e;
        if (max_len <= skip_le) return cudaSuccess;
      } else {
        cudaGetLastError();
      }
    }
    auto kern = tma ? flash_attn_bf16_d64<true> : flash_attn_bf16_d64<false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                         cudaSharedmemCarveoutMaxShared);
    kern<<<grid, kFaThreads, 0, s>>>(static_cast<const bf16*>(qkv), cu, static_cast<bf16*>(ctx),
                                     heads, scale_log2, tm, err, causal, skip_le);
    return cudaGetLastError();
  }
  if (dtype == JB_DT_BF16)
    return launch_simt<bf16>(qkv, cu, ctx, batch, heads, head_dim, max_len, s, why, causal);
  return launch_simt<float>(qkv, cu, ctx, batch, heads, head_dim, max_len, s, why, causal);
}

}  // namespace jb
