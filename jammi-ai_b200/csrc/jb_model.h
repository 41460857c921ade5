// Host-side model handle: device weights, workspace and the encoder forward.
#pragma once

#include <cuda_runtime.h>

#include <functional>
#include <mutex>
#include <string>
#include <vector>

#include "jb_internal.h"

namespace jb {

// Thrown inside the library and turned into a jb_status at the C boundary.
struct Error {
  jb_status status;
  std::string msg;
};
[[noreturn]] void fail(jb_status st, const std::string& msg);
// Sets the calling thread's jb_last_error() message and returns `st`.
jb_status record_error(jb_status st, const std::string& msg);
void check_cuda(cudaError_t e, const char* what);

// Sets the calling thread's current device for a scope, restoring it after.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev);
  ~DeviceGuard();
};

struct Linear {
  void* w = nullptr;         // [N, K] in the operand dtype
  int dtype = JB_DT_BF16;    // JB_DT_F32 | JB_DT_BF16 | JB_DT_S8
  float* w_scale = nullptr;  // int8: [N]
  float* bias = nullptr;     // [N] or null
  int N = 0, K = 0;
};

struct BertLayerW {
  Linear qkv, o, ffn1, ffn2;
  float *ln1_g = nullptr, *ln1_b = nullptr, *ln2_g = nullptr, *ln2_b = nullptr;
};

// LoRA adapters of one encoder layer (the six sites of bert.rs:437-446:
// query, key, value, attention-output dense, intermediate dense, output
// dense).  Host copies per site rebuild the device matrices the forward uses:
// the q/k/v adapters fused into one [R, H] A and one block-diagonal [3H, R] B,
// each B pre-scaled, rank dimensions padded to a multiple of 8 with zeros.
struct LoraSiteHost {
  std::vector<float> a, b;  // A [rank, in], B [out, rank]
  int rank = 0;
  double scaling = 0;
};
struct LoraLayerW {
  LoraSiteHost site[6];
  Linear a_qkv, b_qkv, a_o, b_o, a_1, b_1, a_2, b_2;  // w == nullptr: no adapter
};
constexpr int kLoraSites = 6;

struct ClipBlockW {
  Linear qkv, o, fc, proj;
  float *ln1_g = nullptr, *ln1_b = nullptr, *ln2_g = nullptr, *ln2_b = nullptr;
};

// Kernel classes timed by the profiler.
enum ProfKind { kProfLinear = 0, kProfAttention = 1, kProfMemory = 2, kProfKinds = 3 };
struct ProfRec {
  int kind;
  cudaEvent_t a, b;
};

struct Workspace {
  int batch_cap = 0, seq_cap = 0;
  size_t bytes = 0;
  std::vector<void*> bufs;
  // shared
  uint32_t* ids = nullptr;
  uint32_t* lens = nullptr;
  int* cu = nullptr;
  int* total = nullptr;
  float* out = nullptr;
  void *x = nullptr, *x1 = nullptr, *y = nullptr, *qkv = nullptr, *ctx = nullptr, *hf = nullptr;
  int8_t* aq = nullptr;
  float* as = nullptr;
  unsigned int* rowmax = nullptr;  // int8: each row's largest FFN1 output (f32 bits)
  // vision
  float* head_t = nullptr;  // projection head: x A^T, [batch, rank] f32
  void* lora_t = nullptr;   // LoRA: x A^T, [rows, lora_width] in the activation dtype
  float* pixels = nullptr;
  void *patches = nullptr, *patch_out = nullptr, *pooled = nullptr;
};

}  // namespace jb

namespace jb {
// A whole forward captured as a CUDA graph on workspace buffers, replayed for
// every later call of the same shape (kind: 0 pooled text, 1 image).
struct GraphEntry {
  int kind = 0, batch = 0, seq = 0, pooling = 0;
  int seen = 0;                    // calls with this shape so far
  cudaGraphExec_t exec = nullptr;  // captured on the second call
  uint64_t last_use = 0;
};
// The multi-device driver's staging on one device, kept by the handle from
// one jb_generate_embeddings call to the next (pinned allocations and their
// release are slow and synchronise the device): a stream and two slots of
// pinned ids / lengths / embeddings with their device copies.
struct DriverSlot {
  uint32_t *h_ids = nullptr, *h_lens = nullptr, *d_ids = nullptr, *d_lens = nullptr;
  float *h_out = nullptr, *d_out = nullptr;
  cudaEvent_t done = nullptr;
};
struct DriverStage {
  cudaStream_t stream = nullptr;
  DriverSlot slot[2];
  size_t ids_cap = 0, rows_cap = 0, out_cap = 0;  // elements per slot
};
void free_driver_stage(DriverStage& st);
}  // namespace jb

struct jb_model {
  int family = JB_FAMILY_BERT;
  int variant = JB_TEXT_BERT;  // text family: BERT or DistilBERT weights / config
  int format = JB_FMT_BF16;
  int device = 0;
  int act = JB_DT_BF16;  // activation storage dtype
  // architecture
  int hidden = 0, layers = 0, heads = 0, ffn = 0, vocab = 0, max_pos = 0, type_vocab = 2;
  float eps = 1e-12f;
  int image_size = 0, patch = 0, embed_dim = 0, tokens = 0;
  bool gap = false;
  // BERT weights
  void *word = nullptr, *pos = nullptr, *type0 = nullptr;
  float *emb_ln_g = nullptr, *emb_ln_b = nullptr;
  // ModernBERT: final_norm, RoPE tables f32 [max_pos, head_dim / 2] (the layers
  // reuse BertLayerW: qkv = Wqkv, o = attn.Wo, ffn1 = Wi [2I, H], ffn2 = mlp.Wo,
  // ln1 = attn_norm (null in layer 0), ln2 = mlp_norm; betas all zero)
  float *final_ln_g = nullptr, *final_ln_b = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  std::vector<jb::BertLayerW> bert_layers;
  // ViT weights (the text tower reuses word / pos for its token and
  // positional tables, clip_blocks, ln_post for ln_final, proj for
  // text_projection)
  jb::Linear conv, proj;
  void *cls = nullptr, *vpos = nullptr;
  float *ln_pre_g = nullptr, *ln_pre_b = nullptr, *ln_post_g = nullptr, *ln_post_b = nullptr;
  std::vector<jb::ClipBlockW> clip_blocks;
  // preprocess_cfg mean / std of the vision tower (open_clip_vit.rs:15-16, 98-99)
  float img_mean[3] = {0.48145466f, 0.4578275f, 0.40821073f};
  float img_std[3] = {0.26862954f, 0.26130258f, 0.27577711f};
  // device copy of the raw RGB8 images of the last jb_encode_image_rgb8 call
  // (bytes, then offsets / widths / heights), grown on demand
  void* img_buf = nullptr;
  size_t img_cap = 0;
  // LoRA adapters (empty: none) and the widest padded rank of a fused site
  std::vector<jb::LoraLayerW> lora;
  int lora_width = 0;
  // post-pool projection head: A [rank, H], B [H, rank] pre-scaled by alpha / rank
  float *head_a = nullptr, *head_b = nullptr;
  int head_rank = 0;
  // bookkeeping
  std::vector<void*> weight_allocs;
  int64_t weight_bytes = 0;
  int* d_err = nullptr;
  int* h_err = nullptr;  // pinned host copy of *d_err, read after each synchronous call
  jb::Workspace ws;
  std::mutex mu;
  // driver staging (jb_generate_embeddings), held by one job at a time
  std::mutex drv_mu;
  jb::DriverStage drv;
  // CUDA-event timing of every launch (off unless enabled)
  bool prof_on = false;
  std::vector<jb::ProfRec> prof_recs;
  std::vector<cudaEvent_t> prof_free;
  // forward graphs (jb::run_graphed): private capture / replay stream and the
  // events that order it after, and before, the caller's stream
  std::vector<jb::GraphEntry> graphs;
  uint64_t graph_clock = 0;
  cudaStream_t graph_stream = nullptr;
  cudaEvent_t graph_in = nullptr, graph_out = nullptr;
  // jb_encode_image's chunked H2D: a copy stream, an event ordering it after
  // the caller's stream, and one event per chunk (grown on demand)
  cudaStream_t copy_stream = nullptr;
  std::vector<cudaEvent_t> copy_ev;
};

namespace jb {

// family -1: OpenCLIP vision when the config has "model_cfg", else BERT family.
jb_model* model_load(const char* path, const char* config_json, int device, int format,
                     int family = -1);
void model_free(jb_model* m);
size_t estimate_batch_bytes(const jb_model* m, int batch, int seq);
// Forward passes on device buffers (the workspace must already hold them).
void bert_forward_device(jb_model* m, const uint32_t* d_ids, const uint32_t* d_lens, int batch,
                         int max_seq, int pooling, float* d_out, float* d_hidden, cudaStream_t s);
void clip_forward_device(jb_model* m, const float* d_px, int batch, float* d_out, cudaStream_t s);
// OpenCLIP text: ids [batch, S] on device (rows end at their largest id, the
// EOT token) -> L2-normalised [batch, embed_dim] f32.
void clip_text_forward_device(jb_model* m, const uint32_t* d_ids, int batch, int S, float* d_out,
                              cudaStream_t s);
// Embedding width of the pooled output: H (BERT family) or embed_dim (CLIP).
inline int output_dim(const jb_model* m);
void ensure_workspace(jb_model* m, int batch, int seq);
// A workspace for (batch, seq) laid out over caller-owned device memory at
// `base` (estimate_batch_bytes(m, batch, seq) bytes, 256-byte aligned); the
// layout is the one ensure_workspace allocates.  Allocates nothing.
Workspace carve_workspace(const jb_model* m, void* base, int batch, int seq);
// Records CUDA events around one launch when profiling is on.
struct ProfScope {
  jb_model* m;
  cudaStream_t s;
  ProfRec rec;
  bool on;
  ProfScope(jb_model* m, int kind, cudaStream_t s);
  ~ProfScope();
};
void profile_enable(jb_model* m, bool on);
void profile_read(jb_model* m, double* ms, int* launches);
// Synchronises `s` and turns the device error flag into an Error.
void check_device_flag(jb_model* m, cudaStream_t s);
// Runs forward(stream), a whole forward over workspace buffers only, ordered
// after the work already queued on `s` and before the work queued next.  The
// first call of a shape (kind, batch, seq, pooling) launches it directly; the
// second captures it as a CUDA graph on the model's private stream; later
// calls replay the graph (one launch instead of ~110).  Profiling runs direct.
void run_graphed(jb_model* m, int kind, int batch, int seq, int pooling, cudaStream_t s,
                 const std::function<void(cudaStream_t)>& forward);
// Drops every captured graph (their pointers die with the workspace).
void clear_graphs(jb_model* m);
// Installs (rank > 0) or removes the projection head; drops the workspace
// (its layout depends on the rank) and the graphs.
void set_projection_head(jb_model* m, const float* a, const float* b, int rank, double alpha);
void load_projection_head(jb_model* m, const char* path, double alpha);
// Installs (rank > 0) or removes the LoRA adapter of one site; drops the
// workspace and the graphs.  f32 / bf16 formats.
void set_lora(jb_model* m, int layer, int site, const float* a, const float* b, int rank,
              double scaling);
// Every layer.{n}.{site}.lora_a / lora_b pair of an adapter file, scaling
// lora_alpha / rank (use_rslora: lora_alpha / sqrt(rank)).  Returns the count.
int load_lora(jb_model* m, const char* path, double alpha, bool rslora);

}  // namespace jb

inline int jb::output_dim(const jb_model* m) {
  return m->family == JB_FAMILY_BERT ? m->hidden : m->embed_dim;
}
