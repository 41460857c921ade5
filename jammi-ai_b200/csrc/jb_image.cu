// Image preprocessing on the device: decoded RGB8 images of any sizes ->
// the vision tower's f32 [B, 3, T, T] input.
//
// preprocess_image_batch (crates/jammi-ai/src/inference/image_preprocess.rs:15-51):
// pad to a white square centred at ((P - w) / 2, (P - h) / 2) (pad_to_square,
// :54-75), resize_exact to T x T with FilterType::CatmullRom, then
// (pixel / 255 - mean) / std per channel.  The resampling is the image crate's
// (0.25.10) separable filter: a vertical pass into an f32 intermediate, then
// a horizontal pass whose sums are clamped to [0, 255] and rounded half away
// from zero.  For output coordinate o, ratio r = P / T, s = max(r, 1):
//   c = (o + 0.5) r;  taps [clamp(floor(c - 2s), 0, P - 1), clamp(ceil(c + 2s), left + 1, P));
//   w_i = k((i - (c - 0.5)) / s) / sum_j w_j,  k the Catmull-Rom cubic
//   (Mitchell-Netravali B = 0, C = 1/2),
// each sum taken over the taps in order.  Every operation is one IEEE f32
// rounding (explicit _rn intrinsics: no contraction into fused multiply-adds),
// so the result equals the f32 restatement bit for bit.
//
// One CTA per (output row, image): the CTA's threads weight the row's
// vertical taps into shared memory, form the intermediate row (3 P values,
// coalesced byte reads of the source rows; the padding reads as 255), then
// each thread resamples output columns horizontally and writes the three
// normalised channels.
#include <cstdint>

#include "jb_common.cuh"
#include "jb_internal.h"

namespace jb {
namespace {

constexpr int kImgThreads = 256;

// Catmull-Rom: ((A a^3 + B a^2) + C a + D) / 6 with (A, B, C, D) =
// (9, -15, 0, 6) for a < 1 and (-3, 15, -24, 12) for 1 <= a < 2.
__device__ __forceinline__ float catmull_rom(float x) {
  const float a = fabsf(x);
  const float a2 = __fmul_rn(a, a);
  const float a3 = __fmul_rn(a2, a);
  float k;
  if (a < 1.0f) {
    k = __fadd_rn(__fadd_rn(__fmul_rn(9.0f, a3), __fmul_rn(-15.0f, a2)), 6.0f);
  } else if (a < 2.0f) {
    k = __fadd_rn(__fmul_rn(-3.0f, a3), __fmul_rn(15.0f, a2));
    k = __fadd_rn(k, __fmul_rn(-24.0f, a));
    k = __fadd_rn(k, 12.0f);
  } else {
    k = 0.0f;
  }
  return __fdiv_rn(k, 6.0f);
}

struct Taps {
  int left, n;
  float centre, sratio;
};
__device__ __forceinline__ Taps tap_range(int o, int src, int dst) {
  const float ratio = __fdiv_rn(static_cast<float>(src), static_cast<float>(dst));
  const float sratio = ratio < 1.0f ? 1.0f : ratio;
  const float support = __fmul_rn(2.0f, sratio);
  const float c = __fmul_rn(__fadd_rn(static_cast<float>(o), 0.5f), ratio);
  long long left = static_cast<long long>(floorf(__fsub_rn(c, support)));
  left = left < 0 ? 0 : (left > src - 1 ? src - 1 : left);
  long long right = static_cast<long long>(ceilf(__fadd_rn(c, support)));
  right = right < left + 1 ? left + 1 : (right > src ? src : right);
  Taps t;
  t.left = static_cast<int>(left);
  t.n = static_cast<int>(right - left);
  t.centre = __fsub_rn(c, 0.5f);
  t.sratio = sratio;
  return t;
}
__device__ __forceinline__ float tap_weight(const Taps& t, int i) {
  return catmull_rom(__fdiv_rn(__fsub_rn(static_cast<float>(t.left + i), t.centre), t.sratio));
}

__global__ void __launch_bounds__(kImgThreads) preprocess_rgb8_kernel(
    const uint8_t* __restrict__ bytes, const int64_t* __restrict__ offsets,
    const int* __restrict__ widths, const int* __restrict__ heights, int T, float3 mean,
    float3 stdv, float* __restrict__ out) {
  extern __shared__ float sm[];  // [3 P] intermediate row, then the vertical weights
  const int oy = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int w = widths[b], h = heights[b], P = max(w, h);
  const int offx = (P - w) / 2, offy = (P - h) / 2;
  const uint8_t* img = bytes + offsets[b];
  float* inter = sm;
  float* vw = sm + 3 * P;

  // vertical weights of this output row, normalised by their ordered sum
  const Taps tv = tap_range(oy, P, T);
  for (int i = tid; i < tv.n; i += kImgThreads) vw[i] = tap_weight(tv, i);
  __syncthreads();
  if (tid == 0) {
    float sum = 0.0f;
    for (int i = 0; i < tv.n; ++i) sum = __fadd_rn(sum, vw[i]);
    vw[tv.n] = sum;
  }
  __syncthreads();
  const float vsum = vw[tv.n];
  __syncthreads();
  for (int i = tid; i < tv.n; i += kImgThreads) vw[i] = __fdiv_rn(vw[i], vsum);
  __syncthreads();

  // intermediate row: value j = 3 x + c of the canvas, vertical sum over taps
  for (int j = tid; j < 3 * P; j += kImgThreads) {
    const int ix = j / 3 - offx;
    const bool in_x = ix >= 0 && ix < w;
    const int64_t col = static_cast<int64_t>(ix) * 3 + (j - (j / 3) * 3);
    float t = 0.0f;
    for (int i = 0; i < tv.n; ++i) {
      const int iy = tv.left + i - offy;
      const float v = (in_x && iy >= 0 && iy < h)
                          ? static_cast<float>(img[static_cast<int64_t>(iy) * w * 3 + col])
                          : 255.0f;
      t = __fadd_rn(t, __fmul_rn(v, vw[i]));
    }
    inter[j] = t;
  }
  __syncthreads();

  // horizontal pass, clamp, round half away from zero, normalise
  const size_t plane = static_cast<size_t>(T) * T;
  float* ob = out + static_cast<size_t>(b) * 3 * plane + static_cast<size_t>(oy) * T;
  for (int ox = tid; ox < T; ox += kImgThreads) {
    const Taps th = tap_range(ox, P, T);
    float sum = 0.0f;
    for (int i = 0; i < th.n; ++i) sum = __fadd_rn(sum, tap_weight(th, i));
    float t0 = 0.0f, t1 = 0.0f, t2 = 0.0f;
    for (int i = 0; i < th.n; ++i) {
      const float wi = __fdiv_rn(tap_weight(th, i), sum);
      const float* p = inter + 3 * (th.left + i);
      t0 = __fadd_rn(t0, __fmul_rn(p[0], wi));
      t1 = __fadd_rn(t1, __fmul_rn(p[1], wi));
      t2 = __fadd_rn(t2, __fmul_rn(p[2], wi));
    }
    const float q0 = roundf(fminf(fmaxf(t0, 0.0f), 255.0f));
    const float q1 = roundf(fminf(fmaxf(t1, 0.0f), 255.0f));
    const float q2 = roundf(fminf(fmaxf(t2, 0.0f), 255.0f));
    ob[ox] = __fdiv_rn(__fsub_rn(__fdiv_rn(q0, 255.0f), mean.x), stdv.x);
    ob[plane + ox] = __fdiv_rn(__fsub_rn(__fdiv_rn(q1, 255.0f), mean.y), stdv.y);
    ob[2 * plane + ox] = __fdiv_rn(__fsub_rn(__fdiv_rn(q2, 255.0f), mean.z), stdv.z);
  }
}

}  // namespace

size_t preprocess_smem_bytes(int max_side, int target) {
  // taps per coordinate < 4 max(P / T, 1) + 2 (the f32 ratio and the rounded
  // interval ends can add one each), plus one slot for the sum
  const double r = static_cast<double>(max_side) / target;
  const size_t taps = static_cast<size_t>(4.0 * (r > 1.0 ? r : 1.0)) + 8;
  return (3 * static_cast<size_t>(max_side) + taps) * sizeof(float);
}

cudaError_t launch_preprocess_rgb8(const uint8_t* d_bytes, const int64_t* d_offsets,
                                   const int* d_widths, const int* d_heights, int batch,
                                   int max_side, int target, const float* mean, const float* stdv,
                                   float* d_out, cudaStream_t s, std::string* why) {
  if (batch == 0) return cudaSuccess;
  if (target <= 0 || batch > 65535 || max_side <= 0) {
    if (why) *why = "image preprocessing: bad target size, batch or image size";
    return cudaErrorInvalidValue;
  }
  const size_t smem = preprocess_smem_bytes(max_side, target);
  if (smem > kImgMaxSmem) {
    if (why) *why = "image preprocessing: an image side of " + std::to_string(max_side) +
                    " pixels exceeds the on-chip row buffer";
    return cudaErrorInvalidValue;
  }
  cudaFuncSetAttribute(preprocess_rgb8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(kImgMaxSmem));
  dim3 grid(target, batch);
  preprocess_rgb8_kernel<<<grid, kImgThreads, smem, s>>>(
      d_bytes, d_offsets, d_widths, d_heights, target, make_float3(mean[0], mean[1], mean[2]),
      make_float3(stdv[0], stdv[1], stdv[2]), d_out);
  return cudaGetLastError();
}

}  // namespace jb
