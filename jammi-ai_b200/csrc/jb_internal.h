// Internal launcher interface shared by the kernels and the host runtime.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/jammi_b200.h"

namespace jb {

// Device error flag bits (atomicOr into a caller-owned int): 1 = a bounded
// wait gave up, 2 = token id out of range, 4 = row length above max_seq,
// 8 = exact search given repeated tie ranks.
constexpr int kErrTimeout = 1;
constexpr int kErrTieRank = 8;

// y = epi(A[M,K] . W[N,K]^T (+ bias)) with an optional residual; see
// jb_op_linear / jb_op_linear_s8 for the meaning of every field.
struct GemmArgs {
  const void* A = nullptr;
  const void* W = nullptr;
  int ab_dtype = JB_DT_BF16;  // JB_DT_F32 | JB_DT_BF16 | JB_DT_S8 (A and W alike)
  int M = 0;                  // rows the buffers hold (upper bound of the live count)
  const int* dM = nullptr;    // optional live row count in device memory (<= M)
  int N = 0, K = 0;
  const float* bias = nullptr;
  const void* resid = nullptr;
  int ldr = 0;
  const float* a_scale = nullptr;  // int8: per-row activation scale
  const float* w_scale = nullptr;  // int8: per-column weight scale
  void* C = nullptr;
  int ldc = 0;
  int c_dtype = JB_DT_BF16;
  int epi = JB_EPI_NONE;
  int* err = nullptr;  // device flag set when a bounded wait gives up
  // optional (tcgen05 path, bf16 output): per output row, atomicMax of the
  // row's largest stored value as f32 bits when it is positive (the bits of
  // non-negative floats order as the values do); rows must start at 0
  unsigned int* row_max = nullptr;
};

// Returns cudaSuccess or an error; *why receives a message for invalid shapes.
cudaError_t launch_gemm(const GemmArgs& g, cudaStream_t s, std::string* why);

struct LnArgs {
  const void* x = nullptr;
  const void* resid = nullptr;
  const float* gamma = nullptr;
  const float* beta = nullptr;
  void* y = nullptr;
  int8_t* yq = nullptr;   // optional fused per-row int8 quantisation of y
  float* yscale = nullptr;
  int dtype = JB_DT_BF16;
  int rows = 0;
  const int* drows = nullptr;
  int cols = 0;
  float eps = 1e-12f;
  unsigned int* zero_rows = nullptr;  // optional: set to 0 for every normalised row
};
cudaError_t launch_layernorm(const LnArgs& a, cudaStream_t s);

// Tabulates the bf16 GELU on the current device (once; later calls return at
// once).  The first int8 BERT forward or GELU quantisation on a device needs
// it: model loading calls it so that no forward (or graph capture) does.
cudaError_t init_gelu_table(cudaStream_t s);
cudaError_t launch_quantize_rows(const void* x, int dtype, int8_t* q, float* scale, int rows,
                                 const int* drows, int cols, cudaStream_t s,
                                 int activation = JB_EPI_NONE);
// The FFN2 input of the int8 forward: bf16(GELU(x)) per-token int8, with each
// row's largest x already known (row_max, as a linear's epilogue records it):
// a row whose largest x is >= 0.5 has amax = GELU(that x) (GELU rises on the
// positives and stays above -0.17 on the negatives), so the row is quantised
// in one streaming pass; other rows take two passes.
cudaError_t launch_gelu_quantize_rowmax(const void* x, const unsigned int* row_max, int8_t* q,
                                        float* scale, int rows, const int* drows, int cols,
                                        cudaStream_t s);

// BERT embeddings: word[ids] + type[0] + pos[p] -> LayerNorm, written packed
// at row cu[b] + p for p < len[b].  type0 == null: no type row; gamma == null:
// no LayerNorm (the sum is stored).
struct EmbedArgs {
  const uint32_t* ids = nullptr;  // [batch, max_seq]
  const int* cu = nullptr;        // [batch + 1]
  const void* word = nullptr;     // [vocab, H]
  const void* pos = nullptr;      // [max_pos, H]
  const void* type0 = nullptr;    // [H]
  const float* gamma = nullptr;
  const float* beta = nullptr;
  void* y = nullptr;
  int8_t* yq = nullptr;
  float* yscale = nullptr;
  int dtype = JB_DT_BF16;
  int batch = 0, max_seq = 0, H = 0, vocab = 0;
  float eps = 1e-12f;
  int* err = nullptr;  // set (bit 2) on an out-of-range token id
};
cudaError_t launch_embed_ln(const EmbedArgs& a, cudaStream_t s);

// bf16 head_dim-64 rows with TMA on the tcgen05 kernel (on by default) or the
// mma.sync one; process-wide.  The tcgen05 kernel takes its work units from
// a device counter: `work` (one int the caller owns, zeroed on the stream
// before the launch; the model forwards pass one in their workspace), or,
// when null, a slot of a small static pool.
void set_attention_tcgen05(bool on);
// causal != 0: query i attends to keys j <= i of its row (the OpenCLIP text
// mask, clip_text.rs:350-362).
cudaError_t launch_attention(const void* qkv, const int* cu, void* ctx, int dtype, int batch,
                             int heads, int head_dim, int max_len, cudaStream_t s,
                             std::string* why,
                             int rows_cap = 0, int* err = nullptr, int causal = 0,
                             int* work = nullptr);

// Bounded wait of one thread until *flag == expect, at most limit_ms; on
// expiry kErrTimeout in *err (jb_wait.cu).
cudaError_t launch_flag_wait(const int* flag, int expect, int limit_ms, int* err, cudaStream_t s);

// ANN sidecar vector formats and exact search (jb_index.cu).
constexpr int64_t kThresholdSampleCap = 100000;  // rows a binary threshold is fit over
constexpr int kMaxSearchK = 1024;
// scratch: fit_threshold_scratch_bytes(dim) bytes of device memory (the
// median's histograms; unused by the mean).
size_t fit_threshold_scratch_bytes(int dim);
cudaError_t launch_fit_binary_threshold(const float* v, int64_t rows, int dim, int kind, float* tau,
                                        void* scratch, cudaStream_t s);
cudaError_t launch_pack_threshold_bits(const float* v, int64_t rows, int dim, const float* tau,
                                       uint8_t* out, cudaStream_t s);
// scratch: f32 [nq, n]; out_idx / out_dist [nq, k]; repeated tie ranks set
// kErrTieRank in *err.
cudaError_t launch_exact_search(const float* corpus, int64_t n, int dim, const uint32_t* tie_rank,
                                const float* queries, int nq, int k, float* scratch, int64_t* out_idx,
                                float* out_dist, int* err, cudaStream_t s);
// The k smallest of each row of dist f32 [nq, n] under (distance, tie rank),
// the selection stage of launch_exact_search on its own.
cudaError_t launch_topk(const float* dist, int64_t n, const uint32_t* tie_rank, int nq, int k,
                        int64_t* out_idx, float* out_dist, int* err, cudaStream_t s);

cudaError_t launch_pool_normalize(const void* hidden, int dtype, const int* cu, float* out,
                                  int batch, int H, int pooling, cudaStream_t s);

// cu[0] = 0, cu[b+1] = cu[b] + min(len[b], max_seq); total also to *d_total.
// Lengths above max_seq set bit 4 of *err.
cudaError_t launch_lens_to_cu(const uint32_t* lens, int batch, int max_seq, int* cu, int* d_total,
                              int* err, cudaStream_t s);

// Scatter packed f32-converted hidden rows back to a zero-filled [B, S, H].
cudaError_t launch_unpack_hidden(const void* packed, int dtype, const int* cu, float* out,
                                 int batch, int max_seq, int H, cudaStream_t s);

// ViT: pixels [B,3,I,I] f32 -> patches [B*g*g, 3*p*p] (dtype), (c, ky, kx) order.
cudaError_t launch_patchify(const float* px, void* patches, int dtype, int batch, int image,
                            int patch, cudaStream_t s);
// ViT: x[b, 0] = cls + pos[0]; x[b, i] = patch_out[b, i-1] + pos[i]; then LN.
cudaError_t launch_vit_embed_ln(const void* patch_out, const void* cls, const void* pos,
                                const float* gamma, const float* beta, void* y, int dtype,
                                int batch, int tokens, int W, float eps, cudaStream_t s);
// ViT pooling before ln_post: CLS token (gap = 0) or mean of tokens 1.. (gap = 1), then LN.
// cu != null: packed rows, each row's last token (gap must be 0).
cudaError_t launch_vit_pool_ln(const void* x, const float* gamma, const float* beta, void* y,
                               int dtype, int batch, int tokens, int W, int gap, float eps,
                               cudaStream_t s, const int* cu = nullptr);
// lens[b] = 1 + argmax(ids[b, :S]) (first maximum): OpenCLIP text rows end at
// their <|endoftext|> token.
cudaError_t launch_eot_lens(const uint32_t* ids, int batch, int S, uint32_t* lens, cudaStream_t s);
// cu[b] = b * tokens for b in [0, batch] (fixed-length rows, e.g. ViT tokens).
cudaError_t launch_fill_cu_uniform(int* cu, int batch, int tokens, cudaStream_t s);
// Row-wise x / clamp(||x||, 1e-12) over f32 [rows, cols], in place.
cudaError_t launch_l2_rows(float* x, int rows, int cols, cudaStream_t s);
// Image preprocessing (image_preprocess.rs:15-75): RGB8 images packed at
// d_offsets (HWC bytes, widths x heights) -> pad to a white square, Catmull-Rom
// resize to target x target, (x / 255 - mean) / std -> f32 [batch, 3, target, target].
// max_side = the largest max(w, h) of the batch (sizes the on-chip row buffer).
constexpr size_t kImgMaxSmem = 232448;
size_t preprocess_smem_bytes(int max_side, int target);
cudaError_t launch_preprocess_rgb8(const uint8_t* d_bytes, const int64_t* d_offsets,
                                   const int* d_widths, const int* d_heights, int batch,
                                   int max_side, int target, const float* mean, const float* stdv,
                                   float* d_out, cudaStream_t s, std::string* why);
// ModernBERT: RoPE on the Q and K column blocks of packed qkv [T, 3 * heads * d]
// in place; cos_t / sin_t f32 [max_pos, d/2], position = index within the row.
cudaError_t launch_rope_qk(void* qkv, int dtype, const int* cu, int batch, int max_seq, int heads,
                           int d, const float* cos_t, const float* sin_t, cudaStream_t s);
// ModernBERT GeGLU: out[r, j] = gelu_erf(ug[r, j]) * ug[r, I + j], rows < *drows.
cudaError_t launch_geglu(const void* ug, void* out, int dtype, int rows, const int* drows, int I,
                         cudaStream_t s);
// x = gelu_erf(x) in place over rows < *drows (drows may be null).
cudaError_t launch_gelu_rows(void* x, int dtype, int rows, const int* drows, int cols,
                             cudaStream_t s);

int num_sms(int device);

}  // namespace jb
