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

/* Weight / compute format.  F32, BF16 and F16 mirror ComputePrecision
 * (crates/jammi-numerics/src/precision.rs:36-51); INT8 is new: int8 weights
 * with per-output-channel scales and per-token int8 activations for the six
 * per-layer linears, bf16 everywhere else.  F16 is defined for the BERT and
 * DistilBERT encoders (no LoRA adapters); other families answer
 * JB_ERR_INVALID. */
typedef enum { JB_FMT_F32 = 0, JB_FMT_BF16 = 1, JB_FMT_INT8 = 2, JB_FMT_F16 = 3 } jb_format;

/* Pooling (crates/jammi-encoders/src/pooling.rs:14-30). */
typedef enum {
  JB_POOL_MEAN = 0,
  JB_POOL_CLS = 1,
  JB_POOL_MAX = 2,
  JB_POOL_WEIGHTED_MEAN = 3
} jb_pooling;

/* JB_FAMILY_CLIP_TEXT: the OpenCLIP text tower (crates/jammi-encoders/src/clip_text.rs),
 * loaded from the same checkpoint as the vision tower (root-level keys). */
typedef enum { JB_FAMILY_BERT = 0, JB_FAMILY_CLIP_VISION = 1, JB_FAMILY_CLIP_TEXT = 2 } jb_family;
/* BERT-family text encoders: BERT (crates/jammi-encoders/src/bert.rs) and
 * DistilBERT (crates/jammi-encoders/src/distilbert.rs: no token-type table,
 * config keys dim / n_layers / n_heads / hidden_dim, weights under "distilbert.")
 * share one forward; ModernBERT (crates/jammi-encoders/src/modernbert.rs,
 * "model_type": "modernbert": RoPE, GeGLU, bias-free pre-norm layers, weights
 * under "model.") has its own, behind the same text entry points. */
typedef enum { JB_TEXT_BERT = 0, JB_TEXT_DISTILBERT = 1, JB_TEXT_MODERNBERT = 2 } jb_text_variant;

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
  int32_t projection_rank; /* rank of the installed projection head, 0 if none */
  int32_t variant;         /* text family: jb_text_variant */
  float preprocess_mean[3]; /* vision: preprocess_cfg.mean (OpenAI CLIP defaults) */
  float preprocess_std[3];  /* vision: preprocess_cfg.std */
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
/* The same with the tower named: `family` JB_FAMILY_BERT, JB_FAMILY_CLIP_VISION
 * or JB_FAMILY_CLIP_TEXT (-1: detect, as jb_model_load).  An OpenCLIP
 * checkpoint holds both towers; CandleBackend::load builds both from it
 * (candle.rs:1474-1501): load it once per tower.  CLIP text models take
 * f32 or bf16 weights (ClipTextConfig::from_open_clip_config,
 * clip_text.rs:53-102: model_cfg.embed_dim, model_cfg.text_cfg). */
jb_status jb_model_load_family(const char* safetensors_path, const char* config_json,
                               int device, int format, int family, jb_model** out);
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
 * loading this library holds until exit.  BERT-family handles only (BERT,
 * DistilBERT, ModernBERT); an OpenCLIP text or vision handle returns
 * JB_ERR_INVALID.  Requests whose jb_estimate_batch_bytes exceeds 64 MiB
 * return JB_ERR_INVALID.  All calls on a device share that array (it keeps
 * the previous call's contents): calls that overlap on the GPU race.  The
 * first call on a device looks up the array's device address; make it
 * before any stream capture.  Like jb_encode_text_device it queues work and
 * returns: an out-of-vocabulary id or a length above max_seq found on the
 * device is reported by the handle's next synchronising call.  A handle
 * does not survive cudaDeviceReset (its weights are gone), and neither does
 * the looked-up address. */
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
/* Decoded RGB8 images (HWC bytes, image b at bytes + offsets[b], widths[b] x
 * heights[b], all inside n_bytes) -> host f32 [batch, embed_dim]: the whole of
 * CandleModel::forward_image_embedding (candle.rs:858-925) after decoding.
 * preprocess_image_batch (image_preprocess.rs:15-75: pad to a white square,
 * Catmull-Rom resize to image_size, (x / 255 - mean) / std with the model's
 * preprocess_cfg) runs on the device, on raw bytes copied once.  A side above
 * about 19,000 pixels answers JB_ERR_INVALID. */
jb_status jb_encode_image_rgb8(jb_model* model, const uint8_t* bytes, size_t n_bytes,
                               const int64_t* offsets, const int32_t* widths,
                               const int32_t* heights, int batch, float* out, void* stream);
/* The preprocessing alone on device buffers: -> f32 [batch, 3, target, target].
 * max_side = the largest max(width, height) of the batch; mean / std_ are host
 * float[3]. */
jb_status jb_op_preprocess_rgb8(const uint8_t* d_bytes, const int64_t* d_offsets,
                                const int32_t* d_widths, const int32_t* d_heights, int batch,
                                int max_side, int target, const float* mean, const float* std_,
                                float* d_out, void* stream);
jb_status jb_encode_image_device(jb_model* model, const float* d_pixels, int batch,
                                 float* d_out, void* stream);

/* ── single ops (device pointers) ──────────────────────────────────────── */
/* dtype codes for the op entry points */
typedef enum { JB_DT_F32 = 0, JB_DT_BF16 = 1, JB_DT_S8 = 2, JB_DT_S32 = 3, JB_DT_F16 = 4 } jb_dtype;

/* Epilogues applied to acc (+ bias) before the store. */
typedef enum {
  JB_EPI_NONE = 0,        /* y = acc (+ bias if given) */
  JB_EPI_GELU = 1,        /* y = gelu_erf(acc + bias), bert.rs:187-190 */
  JB_EPI_QUICK_GELU = 2,  /* y = z * sigmoid(1.702 z), open_clip_vit.rs:123-125 */
  JB_EPI_RESIDUAL = 3     /* y = acc + bias + residual, bert.rs:164-167, 199-202 */
} jb_epilogue;

/* C[M,N] = epi(A[M,K] . W[N,K]^T + bias[N]) -- candle_nn::Linear as called by
 * MaybeLoraLinear::Frozen (crates/jammi-lora/src/wrapper.rs:29-42).
 * a_dtype/w_dtype: F32 (SIMT path), or BF16 or F16 (tcgen05 path, both the
 * same); c_dtype F32, or the operands' 16-bit type; residual has c's dtype
 * and row stride N.  bias may be NULL. */
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
/* jb_op_quantize_rows of act(x): activation JB_EPI_GELU quantises
 * gelu_erf(x) rounded to x's dtype (the int8 FFN input: BertIntermediate,
 * bert.rs:187-190, followed by the per-token quantiser); JB_EPI_NONE is
 * jb_op_quantize_rows.  No reference counterpart (int8 format). */
jb_status jb_op_quantize_rows_act(const void* x, int x_dtype, int activation, int8_t* q,
                                  float* scale, int rows, int cols, void* stream);
/* y = LayerNorm(x (+ residual)) over the last dim, in place allowed
 * (crates/jammi-encoders/src/layer_norm.rs:55-84).  x/y dtype F32, BF16 or F16. */
jb_status jb_op_layernorm(const void* x, const void* residual, const float* gamma,
                          const float* beta, void* y, int dtype, int rows, int cols,
                          float eps, void* stream);
/* Variable-length self-attention over packed rows: qkv [T, 3*heads*d] (Q|K|V
 * column blocks, head-major inside each), cu_seqlens [batch+1] (int32),
 * ctx [T, heads*d].  softmax(Q K^T / sqrt(d)) V per (row, head) over the row's
 * valid tokens -- BertSelfAttention::forward (bert.rs:135-155) with the
 * additive -10000 mask (mask.rs:14-20) realised by excluding padding.
 * dtype F32, BF16 or F16 (F16 with head_dim 64 runs only on the tcgen05
 * kernel: jb_op_attention_rows); max_len bounds every row's length. */
jb_status jb_op_attention(const void* qkv, const int* cu_seqlens, void* ctx, int dtype,
                          int batch, int heads, int head_dim, int max_len, void* stream);
/* The same under the causal mask of the OpenCLIP text tower: query i of a row
 * attends to keys j <= i (clip_text.rs:133-162, mask :350-362). */
jb_status jb_op_attention_causal(const void* qkv, const int* cu_seqlens, void* ctx, int dtype,
                                 int batch, int heads, int head_dim, int max_len, void* stream);
/* The same with the row count of qkv known (rows >= cu_seqlens[batch]):
 * bf16 / f16 head_dim 64 then loads its tiles by TMA (the model forwards' path). */
jb_status jb_op_attention_rows(const void* qkv, const int* cu_seqlens, void* ctx, int dtype,
                               int batch, int heads, int head_dim, int max_len, int rows,
                               int causal, void* stream);
/* Process-wide choice for bf16 head_dim-64 attention with TMA (model forwards;
 * f16 always runs on the tcgen05 kernel, and is refused when it is off)
 * and jb_op_attention_rows): on != 0 (the default) runs every row on the
 * tcgen05 kernel (S = QK^T and O = PV as tcgen05.mma with S, P and O in
 * TMEM; keys streamed in blocks of 128 with an online softmax; a persistent
 * TMA / MMA / softmax warp-specialised CTA per SM pulling (row, head,
 * 128-query) items from a device counter); 0 runs every row on the mma.sync
 * kernel.  Single-op calls share a small pool of counters: more than 64 of
 * them in flight at once on one device race.  New (the reference runs
 * candle's batched matmuls and softmax, crates/jammi-encoders/src/bert.rs:143-152). */
void jb_set_attention_tcgen05(int on);
/* Synchronises `stream` and reads (then clears) the current device's error
 * flag shared by the single-op entry points: JB_ERR_TIMEOUT if a bounded
 * device-side wait gave up in an earlier op. */
jb_status jb_op_sync(void* stream);
/* A bounded device-side wait (one thread, %globaltimer): until *d_flag ==
 * expect, at most limit_ms (<= 2000).  On expiry the next jb_op_sync answers
 * JB_ERR_TIMEOUT and the context stays usable -- the same limit-then-report
 * rule as every spin inside the library's kernels, as an op that exercises
 * failure detection without a fault.  No reference counterpart. */
jb_status jb_op_wait_flag(const int* d_flag, int expect, int limit_ms, void* stream);
/* pool_and_normalize over packed hidden [T, H] (dtype F32/BF16/F16) with
 * cu_seqlens [batch+1]: out f32 [batch, H] (pooling.rs:31-148). */
jb_status jb_op_pool_normalize(const void* hidden, int dtype, const int* cu_seqlens,
                               float* out, int batch, int H, int pooling, void* stream);

/* ── post-pool projection head ───────────────────────────────────────────
 * The projection head of a fine-tuned embedding adapter (CandleModel's
 * projection_head, crates/jammi-ai/src/model/backend/candle.rs:823-829, built by
 * load_projection_head, candle.rs:1857-1892): a LoraLinear over an identity
 * base applied to the pooled, L2-normalised text embedding,
 *   y = x + (lora_alpha / rank) * (x A^T) B^T   (lora_linear.rs:206-305),
 * not re-normalised afterwards.  lora_a [rank, H] and lora_b [H, rank] are f32
 * host arrays; rank 0 removes the head.  Text (BERT) models only; every text
 * entry point that returns pooled embeddings applies it. */
jb_status jb_model_set_projection_head(jb_model* model, const float* lora_a, const float* lora_b,
                                       int rank, double lora_alpha);
/* The same from an adapter safetensors file holding "projection.lora_a" and
 * "projection.lora_b" (any float dtype).  A file without them installs no
 * head and returns JB_OK, like the reference's Ok(None). */
jb_status jb_model_load_projection_head(jb_model* model, const char* adapter_path,
                                        double lora_alpha);

/* ── LoRA adapters inside the encoder linears ────────────────────────────
 * An encoder adapter (SavedAdapter::EncoderAdapters, crates/jammi-ai/src/
 * fine_tune/target.rs:221-230) wraps a layer's linears in LoraLinear
 * (crates/jammi-lora/src/lora_linear.rs:226-305, sites built by LoraSite::build,
 * crates/jammi-encoders/src/bert.rs:590-640 and distilbert.rs):
 *   y = base(x) + scaling * (x A^T) B^T,
 * scaling = lora_alpha / rank, or lora_alpha / sqrt(rank) with use_rslora.
 * The FFN-in site adds before the GELU.  f32 and bf16 formats only (an int8
 * model answers JB_ERR_INVALID); text (BERT / DistilBERT) models only. */
typedef enum {
  JB_LORA_QUERY = 0,     /* query    | q_lin   */
  JB_LORA_KEY = 1,       /* key      | k_lin   */
  JB_LORA_VALUE = 2,     /* value    | v_lin   */
  JB_LORA_ATTN_OUT = 3,  /* dense    | out_lin */
  JB_LORA_FFN_IN = 4,    /* intermediate_dense | lin1 */
  JB_LORA_FFN_OUT = 5    /* output_dense       | lin2 */
} jb_lora_site;
/* Install (rank > 0) or remove (rank 0) the adapter of one site of one layer.
 * lora_a [rank, in_features], lora_b [out_features, rank], f32 host arrays;
 * `scaling` multiplies (x A^T) B^T as given. */
jb_status jb_model_set_lora(jb_model* model, int layer, int site, const float* lora_a,
                            const float* lora_b, int rank, double scaling);
/* Every adapter of an adapter.safetensors file: keys
 * "layer.{n}.{module}.lora_a" / ".lora_b" (bert.rs:299-346, distilbert.rs:
 * 245-296; module names per the site enum above), rank from lora_a's rows.
 * *n_sites (may be NULL) receives the number of sites installed; a file with
 * none installs nothing and returns JB_OK. */
jb_status jb_model_load_lora(jb_model* model, const char* adapter_path, double lora_alpha,
                             int use_rslora, int* n_sites);

/* ── memory-budget admission ──────────────────────────────────────────────
 * GpuScheduler (crates/jammi-ai/src/concurrency/gpu_scheduler.rs:11-218):
 * budget = total * (1 - headroom_fraction); reservations by compare-and-swap;
 * a release wakes blocked acquirers; priority is accepted and ignored. */
typedef struct jb_scheduler jb_scheduler;
/* GpuScheduler::new; NULL (and jb_last_error) when headroom is outside [0, 1]. */
jb_scheduler* jb_scheduler_new(uint64_t total_bytes, double headroom_fraction);
/* GpuScheduler::new_unlimited (CPU, or a failed memory probe). */
jb_scheduler* jb_scheduler_new_unlimited(void);
/* GpuScheduler::for_device (gpu_scheduler.rs:114-145): cudaMemGetInfo on
 * `device`, headroom = 1 - memory_fraction clamped to [0, 1]; device < 0 or a
 * failed probe gives an unlimited scheduler. */
jb_scheduler* jb_scheduler_for_device(int device, double memory_fraction);
void jb_scheduler_free(jb_scheduler* s);
int jb_scheduler_is_unlimited(const jb_scheduler* s);
uint64_t jb_scheduler_available(const jb_scheduler* s);
/* GpuScheduler::try_acquire: 1 when reserved, 0 when it would exceed the budget. */
int jb_scheduler_try_acquire(jb_scheduler* s, uint64_t bytes);
/* GpuScheduler::acquire: blocks until the bytes fit (woken by releases).
 * Requests larger than the whole budget fail at once with JB_ERR_OOM;
 * timeout_ms < 0 waits indefinitely, otherwise JB_ERR_TIMEOUT. */
jb_status jb_scheduler_acquire(jb_scheduler* s, uint64_t bytes, int priority, int64_t timeout_ms);
/* Drop of GpuPermit: returns the bytes and wakes waiters. */
void jb_scheduler_release(jb_scheduler* s, uint64_t bytes);

/* ── chunked runner ───────────────────────────────────────────────────────
 * InferenceRunner::run_chunks (crates/jammi-ai/src/inference/runner.rs:176-241):
 * forward(user, start, count, msg, msg_len) runs rows [start, start+count)
 * and returns a jb_status, writing a message on failure.  When the message is
 * an OOM (is_oom_error, runner.rs:243-256: "out of memory", "out_of_memory",
 * "outofmemory" or "oom", case-insensitive) and *batch_size > 1, the batch
 * size halves and the same slice is retried; any other failure, or an OOM at
 * batch size 1, is returned.  *batch_size keeps the final size. */
typedef int (*jb_forward_cb)(void* user, int64_t start, int64_t count, char* msg, size_t msg_len);
jb_status jb_run_chunks(int64_t rows, int* batch_size, jb_forward_cb forward, void* user);
int jb_is_oom_message(const char* msg);

/* ── pooling declared by a checkpoint (host) ──────────────────────────────
 * pooling_from_config (crates/jammi-ai/src/model/backend/candle.rs:440-538):
 * the JB_POOL_* strategy a sentence-transformers 1_Pooling/config.json
 * declares.  jb_pooling_from_config takes the file's text (NULL: no file ->
 * JB_POOL_MEAN); jb_pooling_from_model_dir reads <dir>/1_Pooling/config.json
 * (absent -> JB_POOL_MEAN; read_local_pooling_config, crates/jammi-ai/src/
 * model/resolver.rs:473-500).  The true pooling_mode_* flags must all name
 * one representable strategy (mean_sqrt_len_tokens counts as mean);
 * anything else answers JB_ERR_INVALID (JB_ERR_IO: present but unreadable),
 * never a silent mean. */
jb_status jb_pooling_from_config(const char* pooling_config_json, int* pooling);
jb_status jb_pooling_from_model_dir(const char* model_dir, int* pooling);

/* ── ANN sidecar vector formats and exact search (device) ─────────────────
 * The vector side of the reference's index module on device buffers.
 * jb_op_fit_binary_threshold: the per-dimension threshold tau a Binary
 * sidecar sign-packs against (fit_binary_threshold, crates/jammi-db/src/
 * index/sidecar.rs:162-216) over the first min(rows, 100000) rows of
 * d_vectors [rows, dim]: JB_THRESHOLD_MEAN (f64 sum in row order / count,
 * rounded to f32; bit-identical) or JB_THRESHOLD_MEDIAN (f32 total order,
 * the central pair averaged for an even count); zeros for no rows.
 * jb_op_pack_threshold_bits: pack_threshold_bits (sidecar.rs:232-241), bit i
 * = v[i] > tau[i], LSB-first, d_packed [rows, ceil(dim / 8)] bytes.
 * jb_op_exact_search: exact_vector_search (crates/jammi-db/src/index/
 * exact.rs:119-175) -- cosine_distance (crates/jammi-numerics/src/
 * distance.rs:6-21) of every query to every corpus row, bit-identical to the
 * reference's f32 loop, and the k nearest per query in ascending (distance,
 * tie rank) order: d_tie_rank [n] is each row's position in ascending
 * _row_id order (distinct; NULL = row order).  d_scratch holds
 * n_queries x n floats; d_idx / d_dist are [n_queries, k], entries past the
 * corpus size -1 / +inf.  k <= 1024.  Repeated tie ranks surface as
 * JB_ERR_INVALID from jb_op_sync. */
enum { JB_THRESHOLD_MEAN = 0, JB_THRESHOLD_MEDIAN = 1 };
jb_status jb_op_fit_binary_threshold(const float* d_vectors, int64_t rows, int dim, int kind,
                                     float* d_tau, void* stream);
jb_status jb_op_pack_threshold_bits(const float* d_vectors, int64_t rows, int dim,
                                    const float* d_tau, uint8_t* d_packed, void* stream);
jb_status jb_op_exact_search(const float* d_corpus, int64_t n, int dim, const uint32_t* d_tie_rank,
                             const float* d_queries, int n_queries, int k, float* d_scratch,
                             int64_t* d_idx, float* d_dist, void* stream);

/* ── ANN sidecar insert and search (device-resident SidecarIndex) ─────────
 * A sidecar index whose vector store lives on one device, fed straight from
 * the embedding job's output.  Keys are internal ids 0, 1, 2, ... in add
 * order (the reference's usearch key = position in row_map); the caller
 * keeps the key -> _row_id map.  Every pointer argument may be host
 * (pageable or pinned) or device memory.  Calls on one handle are
 * serialised by its lock and run on its own stream; each returns when its
 * work is done.
 * jb_sidecar_create: SidecarIndex::new (crates/jammi-db/src/index/
 *   sidecar.rs:407-430) for `dim`-wide vectors at JB_STORAGE_F32 or
 *   JB_STORAGE_BINARY (StoragePrecision, crates/jammi-db/src/config.rs:
 *   455-469; F16 and Int8 are quantised inside the graph library and answer
 *   JB_ERR_INVALID).
 * jb_sidecar_add: ResultSink::write_batch (crates/jammi-ai/src/pipeline/
 *   result_sink.rs:61-83) feeding SidecarIndex::add (sidecar.rs:754-790) --
 *   the rows of vectors [rows, dim] whose bit in `validity` is set
 *   (LSB-first, the bitmap jb_generate_embeddings writes; NULL = every row)
 *   are appended in row order; *first_key / *added (either may be NULL)
 *   receive the first key given and how many rows were taken.  An add after
 *   a build clears it (and its tie ranks): build again before searching a
 *   Binary sidecar.
 * jb_sidecar_build: SidecarIndex::build (sidecar.rs:792-824) -- a Binary
 *   sidecar fits tau over its first min(len, 100000) vectors
 *   (JB_THRESHOLD_MEAN / JB_THRESHOLD_MEDIAN; the reference builds with the
 *   median) and sign-packs every vector against it.  tie_rank [len] (NULL =
 *   key order) is each key's position in ascending _row_id order, the order
 *   the reference breaks equal distances in; ranks must be distinct.
 * jb_sidecar_search: SidecarIndex::search (sidecar.rs:826-864) for
 *   n_queries queries [n_queries, dim] -> keys int64 / dist f32
 *   [n_queries, k], nearest first: Binary by Hamming distance (differing
 *   bits of the codes, as f32), F32 by cosine distance (crates/jammi-
 *   numerics/src/distance.rs:6-21, bit-identical).  Every key is scanned,
 *   so the result is the exact k nearest (the reference's usearch HNSW
 *   graph returns approximate ones).  Slots past len hold -1 / +inf.
 *   k <= 1024.
 * jb_sidecar_search_final: SegmentedIndex::search_final (crates/jammi-db/
 *   src/index/segment.rs:239-264) -- an F32 sidecar answers as
 *   jb_sidecar_search; a Binary one retrieves k x oversample candidates
 *   (at least k; oversample below 1 counts as 1, the reference's Binary
 *   default is 32) by Hamming distance, rescores each with the exact cosine
 *   distance to its stored f32 vector and keeps the k best under (distance
 *   in f32 total order, tie rank).  k x oversample <= 1024.
 * jb_sidecar_export: the bundle's vector files -- exact f32 vectors
 *   [len, dim] in key order (the .rawf32 rescore companion, sidecar.rs:
 *   262-281), the codes [len, ceil(dim / 8)] each key would be inserted into
 *   a usearch b1x8 graph with (sidecar.rs:806-815) and tau [dim] (the
 *   .threshold companion); NULL skips one.  Codes and tau exist only for a
 *   built Binary sidecar with at least one vector. */
enum { JB_STORAGE_F32 = 0, JB_STORAGE_BINARY = 3 };
typedef struct jb_sidecar jb_sidecar;
jb_status jb_sidecar_create(int device, int dim, int precision, jb_sidecar** out);
jb_status jb_sidecar_add(jb_sidecar* sidecar, const float* vectors, const uint8_t* validity, int64_t rows,
                         int64_t* first_key, int64_t* added);
jb_status jb_sidecar_build(jb_sidecar* sidecar, int threshold_kind, const uint32_t* tie_rank);
int64_t jb_sidecar_len(const jb_sidecar* sidecar);
jb_status jb_sidecar_search(jb_sidecar* sidecar, const float* queries, int n_queries, int k, int64_t* keys,
                            float* dist);
jb_status jb_sidecar_search_final(jb_sidecar* sidecar, const float* queries, int n_queries, int k,
                                  int oversample, int64_t* keys, float* dist);
jb_status jb_sidecar_export(jb_sidecar* sidecar, float* exact, uint8_t* codes, float* tau);
void jb_sidecar_free(jb_sidecar* sidecar);

/* ── tokenizer (host) ─────────────────────────────────────────────────────
 * A model's tokenizer.json through the HuggingFace `tokenizers` pipeline the
 * reference runs in TokenizerWrapper (crates/jammi-ai/src/model/
 * tokenizer.rs:21-78): added tokens (normalized / lstrip / rstrip /
 * single_word), normalisers BertNormalizer, NFC, NFD, NFKC, NFKD, Lowercase,
 * StripAccents, Strip, Prepend, Replace (string patterns, regexes \s+ and
 * ' {2,}'), Precompiled (sentencepiece character maps) and Sequences,
 * pre-tokenisers BertPreTokenizer, ByteLevel, Whitespace, WhitespaceSplit,
 * Punctuation, Digits, Split (string patterns; the CLIP, GPT-2 and \s+
 * regexes), Metaspace and Sequences, models WordLevel, Unigram, WordPiece
 * and BPE (byte-level or character-level: unknown token, fuse_unk,
 * byte_fallback, subword prefix / suffix, ignore_merges), post-processors
 * TemplateProcessing, BertProcessing, RobertaProcessing, ByteLevel (and
 * Sequences), truncation to max_length (special ids included) or else the
 * file's own.  That covers the BERT (with RoBERTa, CamemBERT, XLM-RoBERTa),
 * DistilBERT, ModernBERT and CLIP families; other components (other regexes,
 * UnicodeScripts, ...) answer JB_ERR_INVALID at load.  Output is the ragged layout of jb_generate_embeddings: ids of text i
 * at ids[offsets[i] .. offsets[i+1]). */
typedef struct jb_tokenizer jb_tokenizer;
jb_status jb_tokenizer_load(const char* tokenizer_json_path, jb_tokenizer** out);
/* The OpenCLIP text tower's BPE from OpenCLIP's merges file (the
 * bpe_simple_vocab_16e6.txt.gz shipped with OpenCLIP checkpoints; gzip or
 * plain text): load_open_clip_bpe (crates/jammi-ai/src/model/clip_bpe.rs:
 * 52-217) -- byte symbols, "</w>" word ends, the CLIP regex pre-tokeniser, no
 * normaliser, <|startoftext|> ... <|endoftext|> (ids vocab-2 and vocab-1).
 * The first 48894 merges are read, as OpenCLIP does; a shorter file gives a
 * smaller vocabulary with the same layout. */
jb_status jb_tokenizer_load_clip_bpe(const char* merges_path, jb_tokenizer** out);
void jb_tokenizer_free(jb_tokenizer* tokenizer);
/* texts: n UTF-8 strings of text_bytes[i] bytes (invalid sequences read as
 * U+FFFD); max_length <= 0 applies the tokenizer.json's own truncation, if
 * any (with its direction), else none.  offsets [n + 1] is always
 * filled; ids may be NULL (a size query: offsets[n] ids are needed), else it
 * holds ids_capacity ids.  Long batches are tokenised on all host cores. */
jb_status jb_tokenize(const jb_tokenizer* tokenizer, const char* const* texts,
                      const uint64_t* text_bytes, int64_t n, int max_length, uint32_t* ids,
                      uint64_t ids_capacity, uint64_t* offsets);
/* jb_tokenize with CandleModel::forward_embedding's row rule (crates/jammi-ai/
 * src/model/backend/candle.rs:779-806): a NULL or empty text is a row with no
 * tokens -- the null row jb_generate_embeddings emits as a zero vector with a
 * cleared validity bit -- instead of an encoding of the empty string; pass
 * the model's max_seq as max_length, as the reference truncates to it. */
jb_status jb_tokenize_rows(const jb_tokenizer* tokenizer, const char* const* texts,
                           const uint64_t* text_bytes, int64_t n, int max_length, uint32_t* ids,
                           uint64_t ids_capacity, uint64_t* offsets);

/* ── multi-device embedding generation ────────────────────────────────────
 * The generate_embeddings driver (crates/jammi-ai/src/pipeline/embedding.rs:47-282
 * -> runner.rs:176-241 -> candle.rs:764-856) over one model handle per device:
 * rows are given as ragged token ids (values + row offsets, the layout of an
 * Arrow list array); empty rows are excluded and come out as zero vectors
 * with a null validity bit (candle.rs:785-797); the rest are length-bucketed
 * (longest first), cut into batches of batch_rows, and pulled by one worker
 * thread per device (one stream each, pinned double-buffered staging,
 * OOM batch-halving).  Embeddings land in row order in out[rows, H] -- the
 * values buffer of an Arrow FixedSizeList<Float32>[H]
 * (crates/jammi-ai/src/inference/adapter/embedding.rs:32-55) -- and
 * validity[(rows+7)/8] is the Arrow bitmap (may be NULL).
 * memory_fraction > 0 enables per-device admission (jb_scheduler_for_device). */
typedef struct {
  int32_t batch_rows;      /* rows per batch, e.g. 256 */
  int32_t pooling;         /* jb_pooling */
  int32_t sort_by_length;  /* length bucketing, longest first */
  int32_t pad_multiple;    /* pad each batch's width up to a multiple (>= 1) */
  double memory_fraction;  /* GpuConfig::memory_fraction; <= 0 disables admission */
} jb_generate_opts;
typedef struct {
  int64_t rows, valid_rows, batches, tokens, oom_retries;
  double seconds;
  /* where the time went (new; the reference records per-batch wall time
   * only, crates/jammi-ai/src/inference/runner.rs:195-198): */
  int64_t h2d_bytes, d2h_bytes;  /* host->device ids + lengths, device->host embeddings */
  double prepare_seconds;        /* validation, length bucketing, null rows (one thread) */
  double pack_seconds;           /* packing ids into pinned staging, summed over workers */
  double scatter_seconds;        /* pinned staging -> out in row order, summed over workers */
  double wait_seconds;           /* workers blocked on their device, summed */
  double worker_seconds_max;     /* the slowest worker's wall time */
  double worker_seconds_min;     /* the fastest worker's (max - min: the tail) */
  double enqueue_seconds;        /* copies + forward enqueued (CUDA graph capture included), summed */
  double setup_seconds;          /* staging allocation, summed (0 once a handle's staging fits) */
} jb_generate_stats;
jb_status jb_generate_embeddings(jb_model** models, int n_models, const uint32_t* ids,
                                 const uint64_t* offsets, int64_t rows,
                                 const jb_generate_opts* opts, float* out, uint8_t* validity,
                                 jb_generate_stats* stats);

#ifdef __cplusplus
}
#endif
#endif /* JAMMI_B200_H */
