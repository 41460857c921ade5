// The C ABI (include/jammi_b200.h): argument checks, exception -> status
// mapping, the thread-local error message and the per-handle lock.
#include <cstring>
#include <mutex>
#include <string>

#include "jb_model.h"

namespace {

thread_local std::string g_last_error;

jb_status set_error(jb_status st, const std::string& msg) {
  g_last_error = msg;
  return st;
}

template <typename F>
jb_status guarded(F&& f) {
  try {
    f();
    g_last_error.clear();
    return JB_OK;
  } catch (const jb::Error& e) {
    return set_error(e.status, e.msg);
  } catch (const std::bad_alloc&) {
    return set_error(JB_ERR_OOM, "host out of memory");
  } catch (const std::exception& e) {
    return set_error(JB_ERR_INVALID, e.what());
  }
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// One error flag per device for the single-op entry points.
int* op_flag(int device) {
  static std::mutex mu;
  static int* flags[64] = {nullptr};
  if (device < 0 || device >= 64) jb::fail(JB_ERR_INVALID, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(mu);
  if (!flags[device]) {
    jb::check_cuda(cudaMalloc(&flags[device], sizeof(int)), "op error flag");
    jb::check_cuda(cudaMemset(flags[device], 0, sizeof(int)), "op error flag");
  }
  return flags[device];
}
int current_device() {
  int d = 0;
  jb::check_cuda(cudaGetDevice(&d), "cudaGetDevice");
  return d;
}

void check_text_args(const jb_model* m, int batch, int max_seq, int pooling) {
  if (!m) jb::fail(JB_ERR_INVALID, "null model");
  if (m->family != JB_FAMILY_BERT && m->family != JB_FAMILY_CLIP_TEXT)
    jb::fail(JB_ERR_INVALID, "model is not a text encoder");
  if (batch < 0 || max_seq < 0) jb::fail(JB_ERR_INVALID, "batch and max_seq must be >= 0");
  if (pooling < JB_POOL_MEAN || pooling > JB_POOL_WEIGHTED_MEAN) jb::fail(JB_ERR_INVALID, "unknown pooling");
  // SequenceTooLong: Bert::forward_hidden (bert.rs:263-268), ClipText::forward
  // (clip_text.rs:302-308, against context_length)
  if (max_seq > m->max_pos)
    jb::fail(JB_ERR_SEQ_TOO_LONG, "sequence length " + std::to_string(max_seq) + " exceeds " +
                                      (m->family == JB_FAMILY_CLIP_TEXT ? "context_length "
                                                                        : "max_position_embeddings ") +
                                      std::to_string(m->max_pos));
  if (static_cast<int64_t>(batch) * max_seq > (int64_t(1) << 30))
    jb::fail(JB_ERR_INVALID, "batch * max_seq too large");
}

}  // namespace

jb_status jb::record_error(jb_status st, const std::string& msg) { return set_error(st, msg); }

extern "C" {

const char* jb_last_error(void) { return g_last_error.c_str(); }

jb_status jb_model_load(const char* safetensors_path, const char* config_json, int device,
                        int format, jb_model** out) {
  return guarded([&] {
    if (!out) jb::fail(JB_ERR_INVALID, "null output handle");
    *out = nullptr;
    *out = jb::model_load(safetensors_path, config_json, device, format);
  });
}

jb_status jb_model_load_family(const char* safetensors_path, const char* config_json, int device,
                               int format, int family, jb_model** out) {
  return guarded([&] {
    if (!out) jb::fail(JB_ERR_INVALID, "null output handle");
    *out = nullptr;
    if (family < -1 || family > JB_FAMILY_CLIP_TEXT) jb::fail(JB_ERR_INVALID, "unknown model family");
    *out = jb::model_load(safetensors_path, config_json, device, format, family);
  });
}

void jb_model_free(jb_model* model) {
  try {
    jb::model_free(model);
  } catch (...) {
  }
}

jb_status jb_model_get_info(const jb_model* m, jb_model_info* out) {
  return guarded([&] {
    if (!m || !out) jb::fail(JB_ERR_INVALID, "null argument");
    std::memset(out, 0, sizeof(*out));
    out->family = m->family;
    out->format = m->format;
    out->device = m->device;
    out->hidden = m->hidden;
    out->output_dim = jb::output_dim(m);
    out->layers = m->layers;
    out->heads = m->heads;
    out->ffn = m->ffn;
    out->max_seq = m->max_pos;
    out->image_size = m->image_size;
    out->weight_bytes = m->weight_bytes;
    out->projection_rank = m->head_rank;
    out->variant = m->variant;
    for (int i = 0; i < 3; ++i) {
      out->preprocess_mean[i] = m->img_mean[i];
      out->preprocess_std[i] = m->img_std[i];
    }
  });
}

jb_status jb_model_set_projection_head(jb_model* m, const float* lora_a, const float* lora_b,
                                       int rank, double lora_alpha) {
  return guarded([&] {
    if (!m) jb::fail(JB_ERR_INVALID, "null model");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    jb::set_projection_head(m, lora_a, lora_b, rank, lora_alpha);
  });
}

jb_status jb_model_load_projection_head(jb_model* m, const char* adapter_path, double lora_alpha) {
  return guarded([&] {
    if (!m || !adapter_path) jb::fail(JB_ERR_INVALID, "null argument");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    jb::load_projection_head(m, adapter_path, lora_alpha);
  });
}

jb_status jb_model_set_lora(jb_model* m, int layer, int site, const float* lora_a,
                            const float* lora_b, int rank, double scaling) {
  return guarded([&] {
    if (!m) jb::fail(JB_ERR_INVALID, "null model");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    jb::set_lora(m, layer, site, lora_a, lora_b, rank, scaling);
  });
}

jb_status jb_model_load_lora(jb_model* m, const char* adapter_path, double lora_alpha,
                             int use_rslora, int* n_sites) {
  return guarded([&] {
    if (!m || !adapter_path) jb::fail(JB_ERR_INVALID, "null argument");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    const int n = jb::load_lora(m, adapter_path, lora_alpha, use_rslora != 0);
    if (n_sites) *n_sites = n;
  });
}

size_t jb_estimate_batch_bytes(const jb_model* m, int batch, int seq) {
  if (!m || batch < 0 || seq < 0) return 0;
  return jb::estimate_batch_bytes(m, batch, seq);
}

jb_status jb_model_sync(jb_model* m, void* stream) {
  return guarded([&] {
    if (!m) jb::fail(JB_ERR_INVALID, "null model");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    jb::check_device_flag(m, as_stream(stream));
  });
}

jb_status jb_model_profile_enable(jb_model* m, int enable) {
  return guarded([&] {
    if (!m) jb::fail(JB_ERR_INVALID, "null model");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    jb::profile_enable(m, enable != 0);
  });
}

jb_status jb_model_profile_read(jb_model* m, double ms[3], int32_t launches[3]) {
  return guarded([&] {
    if (!m || !ms || !launches) jb::fail(JB_ERR_INVALID, "null argument");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    int l[jb::kProfKinds];
    jb::profile_read(m, ms, l);
    for (int k = 0; k < jb::kProfKinds; ++k) launches[k] = l[k];
  });
}

jb_status jb_encode_text(jb_model* m, const uint32_t* ids, const uint32_t* lens, int batch,
                         int max_seq, int pooling, float* out, void* stream) {
  return guarded([&] {
    check_text_args(m, batch, max_seq, pooling);
    if (batch == 0) return;
    // CLIP text ignores lengths and pooling (clip_text.rs:287-295: the rows
    // end at their EOT token, which is also where they are pooled)
    const bool clip = m->family == JB_FAMILY_CLIP_TEXT;
    if (!ids || (!lens && !clip) || !out) jb::fail(JB_ERR_INVALID, "null buffer");
    if (clip && max_seq == 0) jb::fail(JB_ERR_INVALID, "OpenCLIP text rows need at least one token");
    for (int b = 0; b < batch && !clip; ++b)
      if (lens[b] > static_cast<uint32_t>(max_seq)) jb::fail(JB_ERR_INVALID, "a row length exceeds max_seq");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    cudaStream_t s = as_stream(stream);
    jb::ensure_workspace(m, batch, std::max(max_seq, 1));
    jb::Workspace& ws = m->ws;
    jb::check_cuda(cudaMemcpyAsync(ws.ids, ids, size_t(batch) * max_seq * 4, cudaMemcpyHostToDevice, s), "H2D ids");
    if (!clip)
      jb::check_cuda(cudaMemcpyAsync(ws.lens, lens, size_t(batch) * 4, cudaMemcpyHostToDevice, s), "H2D lens");
    jb::run_graphed(m, 0, batch, max_seq, clip ? 0 : pooling, s, [&](cudaStream_t gs) {
      if (clip)
        jb::clip_text_forward_device(m, ws.ids, batch, max_seq, ws.out, gs);
      else
        jb::bert_forward_device(m, ws.ids, ws.lens, batch, max_seq, pooling, ws.out, nullptr, gs);
    });
    jb::check_cuda(cudaMemcpyAsync(out, ws.out, size_t(batch) * jb::output_dim(m) * 4, cudaMemcpyDeviceToHost, s), "D2H");
    jb::check_device_flag(m, s);
  });
}

jb_status jb_encode_text_device(jb_model* m, const uint32_t* d_ids, const uint32_t* d_lens,
                                int batch, int max_seq, int pooling, float* d_out, void* stream) {
  return guarded([&] {
    check_text_args(m, batch, max_seq, pooling);
    if (batch == 0) return;
    const bool clip = m->family == JB_FAMILY_CLIP_TEXT;
    if (!d_ids || (!d_lens && !clip) || !d_out) jb::fail(JB_ERR_INVALID, "null buffer");
    if (clip && max_seq == 0) jb::fail(JB_ERR_INVALID, "OpenCLIP text rows need at least one token");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    jb::ensure_workspace(m, batch, std::max(max_seq, 1));
    // The forward runs on workspace copies of the inputs, so that one CUDA
    // graph per shape serves every caller buffer.
    cudaStream_t s = as_stream(stream);
    jb::Workspace& ws = m->ws;
    jb::check_cuda(cudaMemcpyAsync(ws.ids, d_ids, size_t(batch) * max_seq * 4, cudaMemcpyDeviceToDevice, s), "ids");
    if (!clip)
      jb::check_cuda(cudaMemcpyAsync(ws.lens, d_lens, size_t(batch) * 4, cudaMemcpyDeviceToDevice, s), "lens");
    jb::run_graphed(m, 0, batch, max_seq, clip ? 0 : pooling, s, [&](cudaStream_t gs) {
      if (clip)
        jb::clip_text_forward_device(m, ws.ids, batch, max_seq, ws.out, gs);
      else
        jb::bert_forward_device(m, ws.ids, ws.lens, batch, max_seq, pooling, ws.out, nullptr, gs);
    });
    jb::check_cuda(cudaMemcpyAsync(d_out, ws.out, size_t(batch) * jb::output_dim(m) * 4, cudaMemcpyDeviceToDevice, s), "out");
  });
}

jb_status jb_forward_hidden_device(jb_model* m, const uint32_t* d_ids, const uint32_t* d_lens,
                                   int batch, int max_seq, float* d_hidden, void* stream) {
  return guarded([&] {
    check_text_args(m, batch, max_seq, JB_POOL_MEAN);
    // OpenClipTextForward::forward_hidden (open_clip_text.rs:27-44)
    if (m->family == JB_FAMILY_CLIP_TEXT)
      jb::fail(JB_ERR_INVALID, "OpenCLIP text encoder does not support forward_hidden");
    if (batch == 0) return;
    if (!d_ids || !d_lens || !d_hidden) jb::fail(JB_ERR_INVALID, "null buffer");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    jb::ensure_workspace(m, batch, std::max(max_seq, 1));
    jb::bert_forward_device(m, d_ids, d_lens, batch, max_seq, JB_POOL_MEAN, nullptr, d_hidden,
                            as_stream(stream));
  });
}

// Images per chunk of jb_encode_image's overlapped pixel copy (77 MB of f32
// pixels at 224 x 224, about as long on the host link as its forward).
constexpr int kImageChunk = 128;

jb_status jb_encode_image(jb_model* m, const float* pixels, int batch, float* out, void* stream) {
  return guarded([&] {
    if (!m || m->family != JB_FAMILY_CLIP_VISION) jb::fail(JB_ERR_INVALID, "model is not a vision encoder");
    if (batch < 0) jb::fail(JB_ERR_INVALID, "batch must be >= 0");
    if (batch == 0) return;
    if (!pixels || !out) jb::fail(JB_ERR_INVALID, "null buffer");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    cudaStream_t s = as_stream(stream);
    jb::ensure_workspace(m, batch, m->tokens);
    jb::Workspace& ws = m->ws;
    const size_t px = size_t(3) * m->image_size * m->image_size;  // floats per image
    const int chunks = (batch + kImageChunk - 1) / kImageChunk;
    if (chunks == 1) {
      jb::check_cuda(cudaMemcpyAsync(ws.pixels, pixels, batch * px * 4, cudaMemcpyHostToDevice, s), "H2D pixels");
      jb::run_graphed(m, 1, batch, m->tokens, 0, s, [&](cudaStream_t gs) {
        jb::clip_forward_device(m, ws.pixels, batch, ws.out, gs);
      });
    } else {
      // Chunk i's pixels go to their own part of the staging buffer on a copy
      // stream while chunk i - 1's forward runs; images never interact, so
      // each row's embedding is the one the whole-batch forward gives.  Each
      // chunk keeps its own CUDA graph (kind 2 + i: its buffers' offsets).
      if (!m->copy_stream)
        jb::check_cuda(cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking), "copy stream");
      while (m->copy_ev.size() < static_cast<size_t>(chunks) + 1) {
        cudaEvent_t e;
        jb::check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "copy event");
        m->copy_ev.push_back(e);
      }
      // the caller's earlier work on s may still read the staging buffer
      jb::check_cuda(cudaEventRecord(m->copy_ev[0], s), "copy order");
      jb::check_cuda(cudaStreamWaitEvent(m->copy_stream, m->copy_ev[0], 0), "copy order");
      for (int i = 0; i < chunks; ++i) {
        const int b0 = i * kImageChunk, nb = std::min(kImageChunk, batch - b0);
        float* d_px = ws.pixels + b0 * px;
        float* d_out = ws.out + size_t(b0) * m->embed_dim;
        jb::check_cuda(cudaMemcpyAsync(d_px, pixels + b0 * px, nb * px * 4, cudaMemcpyHostToDevice,
                                       m->copy_stream), "H2D pixels");
        jb::check_cuda(cudaEventRecord(m->copy_ev[1 + i], m->copy_stream), "copy order");
        jb::check_cuda(cudaStreamWaitEvent(s, m->copy_ev[1 + i], 0), "copy order");
        jb::run_graphed(m, 2 + i, nb, m->tokens, 0, s, [&](cudaStream_t gs) {
          jb::clip_forward_device(m, d_px, nb, d_out, gs);
        });
      }
    }
    jb::check_cuda(cudaMemcpyAsync(out, ws.out, size_t(batch) * m->embed_dim * 4, cudaMemcpyDeviceToHost, s), "D2H");
    jb::check_device_flag(m, s);
  });
}

namespace {
// Checks one packed RGB8 batch (offsets / sizes inside n_bytes) and returns
// the largest image side.
int check_rgb8_batch(const uint8_t* bytes, size_t n_bytes, const int64_t* offsets,
                     const int32_t* widths, const int32_t* heights, int batch) {
  if (!bytes || !offsets || !widths || !heights) jb::fail(JB_ERR_INVALID, "null image buffer");
  int max_side = 0;
  for (int b = 0; b < batch; ++b) {
    const int64_t w = widths[b], h = heights[b], off = offsets[b];
    if (w <= 0 || h <= 0) jb::fail(JB_ERR_INVALID, "image " + std::to_string(b) + " is empty");
    if (off < 0 || static_cast<uint64_t>(off) + static_cast<uint64_t>(w * h * 3) > n_bytes)
      jb::fail(JB_ERR_INVALID, "image " + std::to_string(b) + " lies outside the byte buffer");
    max_side = std::max<int>(max_side, static_cast<int>(std::max(w, h)));
  }
  return max_side;
}
}  // namespace

jb_status jb_encode_image_rgb8(jb_model* m, const uint8_t* bytes, size_t n_bytes,
                               const int64_t* offsets, const int32_t* widths,
                               const int32_t* heights, int batch, float* out, void* stream) {
  return guarded([&] {
    if (!m || m->family != JB_FAMILY_CLIP_VISION) jb::fail(JB_ERR_INVALID, "model is not a vision encoder");
    if (batch < 0) jb::fail(JB_ERR_INVALID, "batch must be >= 0");
    if (batch == 0) return;
    if (!out) jb::fail(JB_ERR_INVALID, "null buffer");
    const int max_side = check_rgb8_batch(bytes, n_bytes, offsets, widths, heights, batch);
    if (jb::preprocess_smem_bytes(max_side, m->image_size) > jb::kImgMaxSmem)
      jb::fail(JB_ERR_INVALID, "an image side of " + std::to_string(max_side) + " pixels is too large");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    cudaStream_t s = as_stream(stream);
    jb::ensure_workspace(m, batch, m->tokens);
    jb::Workspace& ws = m->ws;
    // raw bytes, then offsets (8-byte aligned), widths, heights
    const size_t meta_at = (n_bytes + 15) & ~size_t(15);
    const size_t need = meta_at + size_t(batch) * 16;
    if (need > m->img_cap) {
      jb::check_cuda(cudaStreamSynchronize(s), "image buffer");
      if (m->img_buf) cudaFree(m->img_buf);
      m->img_buf = nullptr;
      m->img_cap = 0;
      jb::check_cuda(cudaMalloc(&m->img_buf, need), "image buffer");
      m->img_cap = need;
    }
    uint8_t* d_bytes = static_cast<uint8_t*>(m->img_buf);
    int64_t* d_off = reinterpret_cast<int64_t*>(d_bytes + meta_at);
    int32_t* d_w = reinterpret_cast<int32_t*>(d_off + batch);
    int32_t* d_h = d_w + batch;
    jb::check_cuda(cudaMemcpyAsync(d_bytes, bytes, n_bytes, cudaMemcpyHostToDevice, s), "H2D images");
    jb::check_cuda(cudaMemcpyAsync(d_off, offsets, size_t(batch) * 8, cudaMemcpyHostToDevice, s), "H2D offsets");
    jb::check_cuda(cudaMemcpyAsync(d_w, widths, size_t(batch) * 4, cudaMemcpyHostToDevice, s), "H2D widths");
    jb::check_cuda(cudaMemcpyAsync(d_h, heights, size_t(batch) * 4, cudaMemcpyHostToDevice, s), "H2D heights");
    std::string why;
    cudaError_t e = jb::launch_preprocess_rgb8(d_bytes, d_off, d_w, d_h, batch, max_side, m->image_size,
                                               m->img_mean, m->img_std, ws.pixels, s, &why);
    if (e != cudaSuccess) {
      if (!why.empty()) jb::fail(JB_ERR_INVALID, why);
      jb::check_cuda(e, "image preprocessing");
    }
    jb::run_graphed(m, 1, batch, m->tokens, 0, s, [&](cudaStream_t gs) {
      jb::clip_forward_device(m, ws.pixels, batch, ws.out, gs);
    });
    jb::check_cuda(cudaMemcpyAsync(out, ws.out, size_t(batch) * m->embed_dim * 4, cudaMemcpyDeviceToHost, s), "D2H");
    jb::check_device_flag(m, s);
  });
}

jb_status jb_op_preprocess_rgb8(const uint8_t* d_bytes, const int64_t* d_offsets,
                                const int32_t* d_widths, const int32_t* d_heights, int batch,
                                int max_side, int target, const float* mean, const float* stdv,
                                float* d_out, void* stream) {
  return guarded([&] {
    if (!d_bytes || !d_offsets || !d_widths || !d_heights || !mean || !stdv || !d_out || batch < 0)
      jb::fail(JB_ERR_INVALID, "jb_op_preprocess_rgb8: bad argument");
    std::string why;
    cudaError_t e = jb::launch_preprocess_rgb8(d_bytes, d_offsets, d_widths, d_heights, batch, max_side,
                                               target, mean, stdv, d_out, as_stream(stream), &why);
    if (e != cudaSuccess) {
      if (!why.empty()) jb::fail(JB_ERR_INVALID, why);
      jb::check_cuda(e, "jb_op_preprocess_rgb8");
    }
  });
}

jb_status jb_encode_image_device(jb_model* m, const float* d_pixels, int batch, float* d_out,
                                 void* stream) {
  return guarded([&] {
    if (!m || m->family != JB_FAMILY_CLIP_VISION) jb::fail(JB_ERR_INVALID, "model is not a vision encoder");
    if (batch < 0) jb::fail(JB_ERR_INVALID, "batch must be >= 0");
    if (batch == 0) return;
    if (!d_pixels || !d_out) jb::fail(JB_ERR_INVALID, "null buffer");
    std::lock_guard<std::mutex> lk(m->mu);
    jb::DeviceGuard g(m->device);
    jb::ensure_workspace(m, batch, m->tokens);
    jb::clip_forward_device(m, d_pixels, batch, d_out, as_stream(stream));
  });
}

// ── single ops ──────────────────────────────────────────────────────────────

jb_status jb_op_sync(void* stream) {
  return guarded([&] {
    int* flag = op_flag(current_device());
    jb::check_cuda(cudaStreamSynchronize(as_stream(stream)), "op");
    int v = 0;
    jb::check_cuda(cudaMemcpy(&v, flag, sizeof(int), cudaMemcpyDeviceToHost), "op flag");
    if (v) {
      cudaMemset(flag, 0, sizeof(int));
      if (v & jb::kErrTieRank) jb::fail(JB_ERR_INVALID, "exact search: tie ranks must be distinct");
      jb::fail(v & jb::kErrTimeout ? JB_ERR_TIMEOUT : JB_ERR_CUDA, "device-side wait exceeded its limit");
    }
  });
}

jb_status jb_op_linear(const void* A, int a_dtype, const void* W, int w_dtype, const float* bias,
                       const void* residual, void* C, int c_dtype, int M, int N, int K,
                       int epilogue, void* stream) {
  return guarded([&] {
    if (a_dtype != w_dtype || (a_dtype != JB_DT_F32 && a_dtype != JB_DT_BF16 && a_dtype != JB_DT_F16))
      jb::fail(JB_ERR_INVALID, "jb_op_linear: A and W must both be f32, both bf16 or both f16");
    if (c_dtype != JB_DT_F32 && c_dtype != JB_DT_BF16 && c_dtype != JB_DT_F16)
      jb::fail(JB_ERR_INVALID, "jb_op_linear: C must be f32, bf16 or f16");
    if (epilogue < JB_EPI_NONE || epilogue > JB_EPI_RESIDUAL) jb::fail(JB_ERR_INVALID, "unknown epilogue");
    if (!A || !W || !C || M < 0) jb::fail(JB_ERR_INVALID, "jb_op_linear: null buffer or negative M");
    jb::GemmArgs g;
    g.A = A;
    g.W = W;
    g.ab_dtype = a_dtype;
    g.M = M;
    g.N = N;
    g.K = K;
    g.bias = bias;
    g.resid = residual;
    g.C = C;
    g.c_dtype = c_dtype;
    g.epi = epilogue;
    g.err = op_flag(current_device());
    std::string why;
    cudaError_t e = jb::launch_gemm(g, as_stream(stream), &why);
    if (e != cudaSuccess) {
      if (!why.empty()) jb::fail(JB_ERR_INVALID, why);
      jb::check_cuda(e, "jb_op_linear");
    }
  });
}

jb_status jb_op_linear_s8(const int8_t* Aq, const float* a_scale, const int8_t* Wq,
                          const float* w_scale, const float* bias, const void* residual, void* C,
                          int c_dtype, int M, int N, int K, int epilogue, void* stream) {
  return guarded([&] {
    if (c_dtype != JB_DT_F32 && c_dtype != JB_DT_BF16 && c_dtype != JB_DT_S32)
      jb::fail(JB_ERR_INVALID, "jb_op_linear_s8: C must be s32, f32 or bf16");
    if (epilogue < JB_EPI_NONE || epilogue > JB_EPI_RESIDUAL) jb::fail(JB_ERR_INVALID, "unknown epilogue");
    if (!Aq || !Wq || !C || M < 0) jb::fail(JB_ERR_INVALID, "jb_op_linear_s8: null buffer or negative M");
    jb::GemmArgs g;
    g.A = Aq;
    g.W = Wq;
    g.ab_dtype = JB_DT_S8;
    g.M = M;
    g.N = N;
    g.K = K;
    g.bias = bias;
    g.resid = residual;
    g.a_scale = a_scale;
    g.w_scale = w_scale;
    g.C = C;
    g.c_dtype = c_dtype;
    g.epi = epilogue;
    g.err = op_flag(current_device());
    std::string why;
    cudaError_t e = jb::launch_gemm(g, as_stream(stream), &why);
    if (e != cudaSuccess) {
      if (!why.empty()) jb::fail(JB_ERR_INVALID, why);
      jb::check_cuda(e, "jb_op_linear_s8");
    }
  });
}

jb_status jb_op_quantize_rows(const void* x, int x_dtype, int8_t* q, float* scale, int rows,
                              int cols, void* stream) {
  return guarded([&] {
    if (!x || !q || !scale || rows < 0 || cols <= 0) jb::fail(JB_ERR_INVALID, "jb_op_quantize_rows: bad argument");
    if (x_dtype != JB_DT_F32 && x_dtype != JB_DT_BF16) jb::fail(JB_ERR_INVALID, "x must be f32 or bf16");
    jb::check_cuda(jb::launch_quantize_rows(x, x_dtype, q, scale, rows, nullptr, cols, as_stream(stream)),
                   "jb_op_quantize_rows");
  });
}

jb_status jb_op_quantize_rows_act(const void* x, int x_dtype, int activation, int8_t* q,
                                  float* scale, int rows, int cols, void* stream) {
  return guarded([&] {
    if (!x || !q || !scale || rows < 0 || cols <= 0)
      jb::fail(JB_ERR_INVALID, "jb_op_quantize_rows_act: bad argument");
    if (x_dtype != JB_DT_F32 && x_dtype != JB_DT_BF16) jb::fail(JB_ERR_INVALID, "x must be f32 or bf16");
    if (activation != JB_EPI_NONE && activation != JB_EPI_GELU)
      jb::fail(JB_ERR_INVALID, "activation must be JB_EPI_NONE or JB_EPI_GELU");
    jb::check_cuda(jb::launch_quantize_rows(x, x_dtype, q, scale, rows, nullptr, cols,
                                            as_stream(stream), activation),
                   "jb_op_quantize_rows_act");
  });
}

jb_status jb_op_layernorm(const void* x, const void* residual, const float* gamma,
                          const float* beta, void* y, int dtype, int rows, int cols, float eps,
                          void* stream) {
  return guarded([&] {
    if (!x || !gamma || !beta || !y || rows < 0 || cols <= 0) jb::fail(JB_ERR_INVALID, "jb_op_layernorm: bad argument");
    if (dtype != JB_DT_F32 && dtype != JB_DT_BF16 && dtype != JB_DT_F16)
      jb::fail(JB_ERR_INVALID, "dtype must be f32, bf16 or f16");
    jb::LnArgs a;
    a.x = x;
    a.resid = residual;
    a.gamma = gamma;
    a.beta = beta;
    a.y = y;
    a.dtype = dtype;
    a.rows = rows;
    a.cols = cols;
    a.eps = eps;
    jb::check_cuda(jb::launch_layernorm(a, as_stream(stream)), "jb_op_layernorm");
  });
}

namespace {
jb_status op_attention(const void* qkv, const int* cu_seqlens, void* ctx, int dtype, int batch,
                       int heads, int head_dim, int max_len, int causal, void* stream,
                       int rows = 0) {
  return guarded([&] {
    if (!qkv || !cu_seqlens || !ctx || batch < 0 || heads <= 0 || head_dim <= 0 || max_len < 0)
      jb::fail(JB_ERR_INVALID, "jb_op_attention: bad argument");
    if (dtype != JB_DT_F32 && dtype != JB_DT_BF16 && dtype != JB_DT_F16)
      jb::fail(JB_ERR_INVALID, "dtype must be f32, bf16 or f16");
    std::string why;
    cudaError_t e = jb::launch_attention(qkv, cu_seqlens, ctx, dtype, batch, heads, head_dim, max_len,
                                         as_stream(stream), &why, rows, op_flag(current_device()), causal);
    if (e != cudaSuccess) {
      if (!why.empty()) jb::fail(JB_ERR_INVALID, why);
      jb::check_cuda(e, "jb_op_attention");
    }
  });
}
}  // namespace

jb_status jb_op_attention(const void* qkv, const int* cu_seqlens, void* ctx, int dtype, int batch,
                          int heads, int head_dim, int max_len, void* stream) {
  return op_attention(qkv, cu_seqlens, ctx, dtype, batch, heads, head_dim, max_len, 0, stream);
}

jb_status jb_op_attention_causal(const void* qkv, const int* cu_seqlens, void* ctx, int dtype,
                                 int batch, int heads, int head_dim, int max_len, void* stream) {
  return op_attention(qkv, cu_seqlens, ctx, dtype, batch, heads, head_dim, max_len, 1, stream);
}

void jb_set_attention_tcgen05(int on) { jb::set_attention_tcgen05(on != 0); }

jb_status jb_op_attention_rows(const void* qkv, const int* cu_seqlens, void* ctx, int dtype,
                               int batch, int heads, int head_dim, int max_len, int rows,
                               int causal, void* stream) {
  if (rows < 0) return jb::record_error(JB_ERR_INVALID, "jb_op_attention_rows: rows must be >= 0");
  return op_attention(qkv, cu_seqlens, ctx, dtype, batch, heads, head_dim, max_len, causal ? 1 : 0,
                      stream, rows);
}

jb_status jb_op_wait_flag(const int* d_flag, int expect, int limit_ms, void* stream) {
  return guarded([&] {
    if (!d_flag || limit_ms < 0 || limit_ms > 2000) jb::fail(JB_ERR_INVALID, "jb_op_wait_flag: bad argument");
    jb::check_cuda(jb::launch_flag_wait(d_flag, expect, limit_ms, op_flag(current_device()), as_stream(stream)),
                   "jb_op_wait_flag");
  });
}

jb_status jb_op_fit_binary_threshold(const float* d_vectors, int64_t rows, int dim, int kind, float* d_tau,
                                     void* stream) {
  return guarded([&] {
    if (rows < 0 || dim < 0 || (kind != JB_THRESHOLD_MEAN && kind != JB_THRESHOLD_MEDIAN))
      jb::fail(JB_ERR_INVALID, "jb_op_fit_binary_threshold: bad argument");
    if (dim > 0 && (!d_tau || (rows > 0 && !d_vectors))) jb::fail(JB_ERR_INVALID, "jb_op_fit_binary_threshold: null buffer");
    // the median's histograms: stream-ordered scratch, released behind the launches
    void* scratch = nullptr;
    const bool median = kind == JB_THRESHOLD_MEDIAN && rows > 0 && dim > 0;
    if (median)
      jb::check_cuda(cudaMallocAsync(&scratch, jb::fit_threshold_scratch_bytes(dim), as_stream(stream)),
                     "jb_op_fit_binary_threshold: scratch");
    const cudaError_t e = jb::launch_fit_binary_threshold(d_vectors, rows, dim, kind, d_tau, scratch,
                                                          as_stream(stream));
    if (scratch) cudaFreeAsync(scratch, as_stream(stream));
    jb::check_cuda(e, "jb_op_fit_binary_threshold");
  });
}

jb_status jb_op_pack_threshold_bits(const float* d_vectors, int64_t rows, int dim, const float* d_tau,
                                    uint8_t* d_packed, void* stream) {
  return guarded([&] {
    if (rows < 0 || dim < 0) jb::fail(JB_ERR_INVALID, "jb_op_pack_threshold_bits: bad argument");
    if (rows > 0 && dim > 0 && (!d_vectors || !d_tau || !d_packed))
      jb::fail(JB_ERR_INVALID, "jb_op_pack_threshold_bits: null buffer");
    jb::check_cuda(jb::launch_pack_threshold_bits(d_vectors, rows, dim, d_tau, d_packed, as_stream(stream)),
                   "jb_op_pack_threshold_bits");
  });
}

jb_status jb_op_exact_search(const float* d_corpus, int64_t n, int dim, const uint32_t* d_tie_rank,
                             const float* d_queries, int n_queries, int k, float* d_scratch,
                             int64_t* d_idx, float* d_dist, void* stream) {
  return guarded([&] {
    if (n < 0 || dim <= 0 || n_queries < 0 || k < 0)
      jb::fail(JB_ERR_INVALID, "jb_op_exact_search: bad argument");
    if (k > jb::kMaxSearchK)
      jb::fail(JB_ERR_INVALID, "jb_op_exact_search: k above " + std::to_string(jb::kMaxSearchK));
    if (n > static_cast<int64_t>(UINT32_MAX)) jb::fail(JB_ERR_INVALID, "jb_op_exact_search: corpus above 2^32 rows");
    if (n_queries > 65535 * 8) jb::fail(JB_ERR_INVALID, "jb_op_exact_search: too many queries in one call");
    if (n_queries > 0 && k > 0 && (!d_idx || !d_dist || (n > 0 && (!d_corpus || !d_queries || !d_scratch))))
      jb::fail(JB_ERR_INVALID, "jb_op_exact_search: null buffer");
    jb::check_cuda(jb::launch_exact_search(d_corpus, n, dim, d_tie_rank, d_queries, n_queries, k, d_scratch,
                                           d_idx, d_dist, op_flag(current_device()), as_stream(stream)),
                   "jb_op_exact_search");
  });
}

jb_status jb_op_pool_normalize(const void* hidden, int dtype, const int* cu_seqlens, float* out,
                               int batch, int H, int pooling, void* stream) {
  return guarded([&] {
    if (!hidden || !cu_seqlens || !out || batch < 0 || H <= 0) jb::fail(JB_ERR_INVALID, "jb_op_pool_normalize: bad argument");
    if (pooling < JB_POOL_MEAN || pooling > JB_POOL_WEIGHTED_MEAN) jb::fail(JB_ERR_INVALID, "unknown pooling");
    if (dtype != JB_DT_F32 && dtype != JB_DT_BF16 && dtype != JB_DT_F16)
      jb::fail(JB_ERR_INVALID, "dtype must be f32, bf16 or f16");
    jb::check_cuda(jb::launch_pool_normalize(hidden, dtype, cu_seqlens, out, batch, H, pooling, as_stream(stream)),
                   "jb_op_pool_normalize");
  });
}

}  // extern "C"
