/*
 * jammi_b200.h -- C ABI of the B200 (sm_100a) embedding-generation library.
 *
 * The library replaces the tensor runtime beneath the reference's encoder
 * forward (candle 0.11 CPU/cuBLAS/PTX).  Every entry point takes plain
 * pointers and sizes; no framework types cross the boundary.  Each
 * declaration names the reference interface it stands in for (paths are
 * relative to the f-inverse/jammi-ai checkout).
 *
 * Conventions
 *  - Every call returns a jb_status; on failure jb_last_error() returns a
 *    thread-local message.  An allocation failure returns JB_ERR_OOM and its
 *    message contains "out of memory", the substring the reference's batch
 *    halving keys on (crates/jammi-ai/src/inference/runner.rs:243-256).
 *  - "stream" is a cudaStream_t (NULL = the legacy default stream).
 *  - *_device entry points take device pointers and do not synchronise;
 *    host-pointer entry points copy in, run and copy out on "stream" and
 *    return after the result is on the host.
 *  - A jb_model is bound to one device.  Calls on one handle are serialised
 *    by an internal mutex (the reference shares one model across tasks,
 *    crates/jammi-ai/src/model/backend/candle.rs:39 `Send + Sync`).
 */
#ifndef JAMMI_B200_H
#define JAMMI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  JB_OK = 0,
  JB_ERR_OOM = 1,             /* message contains "out of memory" */
  JB_ERR_INVALID = 2,         /* bad argument / unsupported shape */
  JB_ERR_CUDA = 3,            /* CUDA runtime error */
  JB_ERR_TIMEOUT = 4,         /* a bounded device-side wait gave up */
  JB_ERR_SEQ_TOO_LONG = 5,    /* EncoderError::SequenceTooLong, crates/jammi-encoders/src/bert.rs:263-268 */
  JB_ERR_IO = 6,              /* weights / config could not be read */
  JB_ERR_NO_DEVICE = 7        /* require_gpu failed, crates/jammi-ai/src/model/backend/candle.rs:2168-2172 */
} jb_status;

/* Weight / compute format.  F32 and BF16 mirror ComputePrecision
 * (crates/jammi-numerics/src/precision.rs:36-51); INT8 is new: int8 weights
 * with per-output-channel scales and per-token int8 activations for the six
 * per-layer linears, bf16 everywhere else. */
typedef enum { JB_FMT_F32 = 0, JB_FMT_BF16 = 1, JB_FMT_INT8 = 2 } jb_format;

/* Pooling (crates/jammi-encoders/src/pooling.rs:14-30). */
typedef enum {
  JB_POOL_MEAN = 0,
  JB_POOL_CLS = 1,
  JB_POOL_MAX = 2,
  JB_POOL_WEIGHTED_MEAN = 3
} jb_pooling;

typedef enum { JB_FAMILY_BERT = 0, JB_FAMILY_CLIP_VISION = 1 } jb_family;

typedef struct jb_model jb_model;

typedef struct {
  int32_t family;          /* jb_family */
  int32_t format;          /* jb_format */
  int32_t device;
  int32_t hidden;          /* H (BERT) or width (ViT) */
  int32_t output_dim;      /* H (BERT) or embed_dim (ViT) */
  int32_t layers;
  int32_t heads;
  int32_t ffn;
  int32_t max_seq;         /* max_position_embeddings, or tokens per image */
  int32_t image_size;      /* ViT only */
  int64_t weight_bytes;    /* device bytes held by the weights */
} jb_model_info;

/* ── lifecycle ─────────────────────────────────────────────────────────── */

/* Load a safetensors checkpoint onto `device`.  `config_json` is the text of
 * HF config.json (BERT family) or open_clip_config.json (ViT, detected by its
 * "model_cfg" key).  Replaces CandleBackend::load's BERT and OpenCLIP arms
 * (crates/jammi-ai/src/model/backend/candle.rs:1585-1604, 1474-1501) and
 * Bert::builder().build (crates/jammi-encoders/src/bert.rs:489-587),
 * including the "bert." prefix probe (bert.rs:508-517).  For JB_FMT_INT8, a
 * linear whose checkpoint carries "<name>.weight_q" (I8) and
 * "<name>.weight_scale" (F32 [out]) is loaded as is; float weights are
 * quantised per output channel on load. */
jb_status jb_model_load(const char* safetensors_path, const char* config_json,
                        int device, int format, jb_model** out);
void jb_model_free(jb_model* model);
jb_status jb_model_get_info(const jb_model* model, jb_model_info* out);
const char* jb_last_error(void);
/* Device bytes one forward of (batch, seq) needs beyond the weights; the
 * per-batch counterpart of ModelDimensions::estimate_activation_memory
 * (crates/jammi-ai/src/model/mod.rs:295-301). */
size_t jb_estimate_batch_bytes(const jb_model* model, int batch, int seq);
/* Reads and clears the device error flag set by a bounded wait that gave up
 * in an earlier asynchronous *_device call.  Synchronises the stream. */
jb_status jb_model_sync(jb_model* model, void* stream);

/* Kernel timing: when enabled, every launch of a forward on this handle is
 * bracketed by CUDA events on its stream.  Enabling (or disabling) resets the
 * record.  jb_model_profile_read waits for the recorded events and returns,
 * per kernel class [0 linear (tensor-core GEMM), 1 attention, 2 memory-bound
 * (embeddings, LayerNorm, quantisation, pooling)], the summed device
 * milliseconds and launch counts.  New (the reference records only per-batch
 * wall time, crates/jammi-ai/src/inference/runner.rs:195-198). */
jb_status jb_model_profile_enable(jb_model* model, int enable);
jb_status jb_model_profile_read(jb_model* model, double ms[3], int32_t launches[3]);

/* ── text encoder (BERT family) ────────────────────────────────────────── */

/* Pooled, L2-normalised embeddings for `batch` rows of right-padded token
 * ids [batch, max_seq] with valid lengths lens[batch] (the attention mask of
 * BatchEncoding is a prefix of ones, crates/jammi-ai/src/model/tokenizer.rs:82-93).
 * out: host f32 [batch, H].  Replaces CandleTextForward::forward_pooled ->
 * Bert::forward -> pool_and_normalize (candle.rs:156-165, bert.rs:279-282,
 * pooling.rs:31-43), including tokens_to_tensor (H2D) and to_vec2 (D2H),
 * candle.rs:808-809, 838-840. */
jb_status jb_encode_text(jb_model* model, const uint32_t* ids, const uint32_t* lens,
                         int batch, int max_seq, int pooling, float* out, void* stream);
/* Same, with ids/lens/out in device memory; asynchronous on `stream`. */
jb_status jb_encode_text_device(jb_model* model, const uint32_t* d_ids, const uint32_t* d_lens,
                                int batch, int max_seq, int pooling, float* d_out, void* stream);
/* The same forward as jb_encode_text_device for callers that must not
 * allocate device memory: cudaMalloc/cudaFree synchronise the whole device
 * (a latency-critical query encoder sharing a GPU with a bulk embedding job
 * would stall behind it), and a process whose device memory is reserved by
 * another runtime's pool has none to allocate.  No counterpart in the
 * reference.  It calls no cudaMalloc, cudaFree or allocating library
 * routine; its scratch is a 64 MiB file-scope device array that every GPU
 * loading this library holds until exit.  Requests whose
 * jb_estimate_batch_bytes exceeds 64 MiB return JB_ERR_INVALID.  All calls on
 * a device share that array (it keeps the previous call's contents): calls
 * that overlap on the GPU race.  The first call on a device looks up the
 * array's device address; make it before any stream capture. */
jb_status jb_encode_text_device_noalloc(jb_model* model, const uint32_t* d_ids,
                                        const uint32_t* d_lens, int batch, int max_seq,
                                        int pooling, float* d_out, void* stream);
/* Bert::forward_hidden (bert.rs:257-276): last hidden states as f32
 * [batch, max_seq, H] in device memory; padded positions are written as 0. */
jb_status jb_forward_hidden_device(jb_model* model, const uint32_t* d_ids, const uint32_t* d_lens,
                                   int batch, int max_seq, float* d_hidden, void* stream);

/* ── vision encoder (OpenCLIP ViT) ─────────────────────────────────────── */

/* L2-normalised image embeddings for normalised pixels [batch, 3, S, S]
 * (host f32); out host f32 [batch, embed_dim].  Replaces
 * CandleVisionForward::forward_image -> OpenClipVisionTransformer::forward
 * plus l2_normalize (open_clip_vit.rs:309-353; candle.rs:425-438, 911). */
jb_status jb_encode_image(jb_model* model, const float* pixels, int batch,
                          float* out, void* stream);
jb_status jb_encode_image_device(jb_model* model, const float* d_pixels, int batch,
                                 float* d_out, void* stream);

/* ── single ops (device pointers) ──────────────────────────────────────── */
/* dtype codes for the op entry points */
typedef enum { JB_DT_F32 = 0, JB_DT_BF16 = 1, JB_DT_S8 = 2, JB_DT_S32 = 3 } jb_dtype;

/* Epilogues applied to acc (+ bias) before the store. */
typedef enum {
  JB_EPI_NONE = 0,        /* y = acc (+ bias if given) */
  JB_EPI_GELU = 1,        /* y = gelu_erf(acc + bias), bert.rs:187-190 */
  JB_EPI_QUICK_GELU = 2,  /* y = z * sigmoid(1.702 z), open_clip_vit.rs:123-125 */
  JB_EPI_RESIDUAL = 3     /* y = acc + bias + residual, bert.rs:164-167, 199-202 */
} jb_epilogue;

/* C[M,N] = epi(A[M,K] . W[N,K]^T + bias[N]) -- candle_nn::Linear as called by
 * MaybeLoraLinear::Frozen (crates/jammi-lora/src/wrapper.rs:29-42).
 * a_dtype/w_dtype: F32 (SIMT path) or BF16 (tcgen05 path); c_dtype F32 or
 * BF16; residual has c's dtype and row stride N.  bias may be NULL. */
jb_status jb_op_linear(const void* A, int a_dtype, const void* W, int w_dtype,
                       const float* bias, const void* residual, void* C, int c_dtype,
                       int M, int N, int K, int epilogue, void* stream);
/* int8 Linear: acc = Aq[M,K] . Wq[N,K]^T in int32 (tcgen05 kind::i8, exact).
 * c_dtype S32 stores acc itself; F32/BF16 store
 * epi(acc * a_scale[m] * w_scale[n] + bias[n]).  No reference counterpart
 * (the reference has no int8 matmul). */
jb_status jb_op_linear_s8(const int8_t* Aq, const float* a_scale, const int8_t* Wq,
                          const float* w_scale, const float* bias, const void* residual,
                          void* C, int c_dtype, int M, int N, int K, int epilogue, void* stream);
/* Per-row symmetric int8 quantisation of x[rows, cols] (F32 or BF16):
 * scale = amax/127, q = clamp(rint(x * (127/amax)), -127, 127). */
jb_status jb_op_quantize_rows(const void* x, int x_dtype, int8_t* q, float* scale,
                              int rows, int cols, void* stream);
/* y = LayerNorm(x (+ residual)) over the last dim, in place allowed
 * (crates/jammi-encoders/src/layer_norm.rs:55-84).  x/y dtype F32 or BF16. */
jb_status jb_op_layernorm(const void* x, const void* residual, const float* gamma,
                          const float* beta, void* y, int dtype, int rows, int cols,
                          float eps, void* stream);
/* Variable-length self-attention over packed rows: qkv [T, 3*heads*d] (Q|K|V
 * column blocks, head-major inside each), cu_seqlens [batch+1] (int32),
 * ctx [T, heads*d].  softmax(Q K^T / sqrt(d)) V per (row, head) over the row's
 * valid tokens -- BertSelfAttention::forward (bert.rs:135-155) with the
 * additive -10000 mask (mask.rs:14-20) realised by excluding padding.
 * dtype F32 or BF16; max_len bounds every row's length. */
jb_status jb_op_attention(const void* qkv, const int* cu_seqlens, void* ctx, int dtype,
                          int batch, int heads, int head_dim, int max_len, void* stream);
/* Synchronises `stream` and reads (then clears) the current device's error
 * flag shared by the single-op entry points: JB_ERR_TIMEOUT if a bounded
 * device-side wait gave up in an earlier op. */
jb_status jb_op_sync(void* stream);
/* pool_and_normalize over packed hidden [T, H] (dtype F32/BF16) with
 * cu_seqlens [batch+1]: out f32 [batch, H] (pooling.rs:31-148). */
jb_status jb_op_pool_normalize(const void* hidden, int dtype, const int* cu_seqlens,
                               float* out, int batch, int H, int pooling, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* JAMMI_B200_H */
