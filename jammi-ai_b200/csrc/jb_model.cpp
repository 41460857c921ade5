// Model loading (safetensors + HF / OpenCLIP config), weight packing and the
// encoder forward passes.
//
// BERT: CandleBackend::load BERT arm (crates/jammi-ai/src/model/backend/candle.rs:1585-1604)
//       -> Bert::builder().build (crates/jammi-encoders/src/bert.rs:489-587).
// ViT:  OpenCLIP arm (candle.rs:1474-1501) -> OpenClipVisionTransformer::load
//       (crates/jammi-ai/src/model/backend/open_clip_vit.rs:258-303).
#include "jb_model.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>

#include "jb_json.h"

namespace jb {

[[noreturn]] void fail(jb_status st, const std::string& msg) { throw Error{st, msg}; }

void check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return;
  cudaGetLastError();  // clear a sticky-free launch error
  if (e == cudaErrorMemoryAllocation)
    fail(JB_ERR_OOM, std::string(what) + ": CUDA out of memory");
  fail(JB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

DeviceGuard::DeviceGuard(int dev) {
  cudaGetDevice(&prev);
  if (prev != dev) check_cuda(cudaSetDevice(dev), "cudaSetDevice");
}
DeviceGuard::~DeviceGuard() {
  int cur = -1;
  cudaGetDevice(&cur);
  if (prev >= 0 && cur != prev) cudaSetDevice(prev);
}

namespace {

// ── safetensors ────────────────────────────────────────────────────────────
struct StTensor {
  std::string dtype;
  std::vector<int64_t> shape;
  size_t begin = 0, end = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
};

float half_to_float(uint16_t h) {
  const uint32_t sign = (h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: renormalise
      int e = -1;
      do { ++e; man <<= 1; } while (!(man & 0x400));
      bits = sign | ((127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t float_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;  // NaN
  u += 0x7FFFu + ((u >> 16) & 1u);                      // round to nearest even
  return static_cast<uint16_t>(u >> 16);
}

// IEEE binary16, round to nearest even.  Normal results: the exponent is
// rebiased (127 -> 15, i.e. minus 112 << 23) and the 13 dropped mantissa bits
// rounded by adding 0xFFF plus the kept LSB; a carry moves into the exponent.
// Magnitudes from 65520 up round to infinity; below 2^-14 the result is a
// subnormal multiple of 2^-24 (the scaling by 2^24 is exact, nearbyint rounds
// half to even).
uint16_t float_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint16_t sign = static_cast<uint16_t>((x >> 16) & 0x8000u);
  x &= 0x7FFFFFFFu;
  if (x > 0x7F800000u) return sign | 0x7E00u;  // NaN
  if (x >= 0x477FF000u) return sign | 0x7C00u;  // infinity, or rounds to it
  if (x < 0x38800000u) {
    float a;
    std::memcpy(&a, &x, 4);
    return sign | static_cast<uint16_t>(std::nearbyint(a * 16777216.0f));
  }
  return sign | static_cast<uint16_t>((x + 0x0FFFu + ((x >> 13) & 1u) - 0x38000000u) >> 13);
}

// The model's 16-bit activation / weight encoding of a float.
uint16_t to_half_bits(int dt, float f) { return dt == JB_DT_F16 ? float_to_f16(f) : float_to_bf16(f); }

struct SafeTensors {
  std::vector<char> file;
  size_t data_start = 0;
  std::map<std::string, StTensor> t;

  explicit SafeTensors(const std::string& path) {
    std::ifstream in(path, std::ios::binary | std::ios::ate);
    if (!in) fail(JB_ERR_IO, "cannot open weights file " + path);
    const std::streamsize size = in.tellg();
    in.seekg(0);
    file.resize(static_cast<size_t>(size));
    if (!in.read(file.data(), size)) fail(JB_ERR_IO, "cannot read weights file " + path);
    if (file.size() < 8) fail(JB_ERR_IO, "safetensors file too short");
    uint64_t hlen = 0;
    std::memcpy(&hlen, file.data(), 8);
    if (8 + hlen > file.size()) fail(JB_ERR_IO, "safetensors header length out of range");
    data_start = 8 + hlen;
    Json h;
    try {
      h = Json::parse(std::string(file.data() + 8, hlen));
    } catch (const std::exception& e) {
      fail(JB_ERR_IO, std::string("safetensors header: ") + e.what());
    }
    for (auto& kv : h.obj) {
      if (kv.first == "__metadata__") continue;
      StTensor st;
      st.dtype = kv.second.str_or("dtype", "");
      if (const Json* sh = kv.second.get("shape"))
        for (auto& d : sh->arr) st.shape.push_back(static_cast<int64_t>(d.num));
      const Json* off = kv.second.get("data_offsets");
      if (!off || off->arr.size() != 2) fail(JB_ERR_IO, "safetensors: bad offsets for " + kv.first);
      st.begin = static_cast<size_t>(off->arr[0].num);
      st.end = static_cast<size_t>(off->arr[1].num);
      if (data_start + st.end > file.size() || st.begin > st.end)
        fail(JB_ERR_IO, "safetensors: tensor out of range: " + kv.first);
      t[kv.first] = st;
    }
  }
  bool has(const std::string& k) const { return t.count(k) != 0; }
  const StTensor& get(const std::string& k) const {
    auto it = t.find(k);
    if (it == t.end()) fail(JB_ERR_IO, "missing tensor " + k);
    return it->second;
  }
  const char* ptr(const StTensor& s) const { return file.data() + data_start + s.begin; }

  std::vector<float> f32(const std::string& k, int64_t expect) const {
    const StTensor& s = get(k);
    if (s.numel() != expect)
      fail(JB_ERR_IO, "tensor " + k + " has " + std::to_string(s.numel()) + " elements, expected " +
                          std::to_string(expect));
    std::vector<float> out(static_cast<size_t>(expect));
    const char* p = ptr(s);
    if (s.dtype == "F32") {
      std::memcpy(out.data(), p, expect * 4);
    } else if (s.dtype == "BF16") {
      for (int64_t i = 0; i < expect; ++i) {
        uint16_t v;
        std::memcpy(&v, p + 2 * i, 2);
        const uint32_t u = static_cast<uint32_t>(v) << 16;
        std::memcpy(&out[i], &u, 4);
      }
    } else if (s.dtype == "F16") {
      for (int64_t i = 0; i < expect; ++i) {
        uint16_t v;
        std::memcpy(&v, p + 2 * i, 2);
        out[i] = half_to_float(v);
      }
    } else if (s.dtype == "F64") {
      for (int64_t i = 0; i < expect; ++i) {
        double v;
        std::memcpy(&v, p + 8 * i, 8);
        out[i] = static_cast<float>(v);
      }
    } else {
      fail(JB_ERR_IO, "tensor " + k + ": unsupported dtype " + s.dtype);
    }
    return out;
  }
  std::vector<float> f32_or(const std::string& k, int64_t n, float fill) const {
    return has(k) ? f32(k, n) : std::vector<float>(static_cast<size_t>(n), fill);
  }
  std::vector<int8_t> i8(const std::string& k, int64_t expect) const {
    const StTensor& s = get(k);
    if (s.numel() != expect || (s.dtype != "I8" && s.dtype != "U8"))
      fail(JB_ERR_IO, "tensor " + k + " must be I8 with " + std::to_string(expect) + " elements");
    std::vector<int8_t> out(static_cast<size_t>(expect));
    std::memcpy(out.data(), ptr(s), expect);
    return out;
  }
};

// ── device uploads ─────────────────────────────────────────────────────────
void* dev_alloc(jb_model* m, size_t bytes) {
  void* p = nullptr;
  check_cuda(cudaMalloc(&p, std::max<size_t>(bytes, 16)), "weight allocation");
  m->weight_allocs.push_back(p);
  m->weight_bytes += static_cast<int64_t>(bytes);
  return p;
}
void* upload_bytes(jb_model* m, const void* src, size_t bytes) {
  void* p = dev_alloc(m, bytes);
  check_cuda(cudaMemcpy(p, src, bytes, cudaMemcpyHostToDevice), "weight upload");
  return p;
}
float* upload_f32(jb_model* m, const std::vector<float>& v) {
  return static_cast<float*>(upload_bytes(m, v.data(), v.size() * 4));
}
// Upload in the model's activation dtype (f32, bf16 or f16).
void* upload_act(jb_model* m, const std::vector<float>& v) {
  if (m->act == JB_DT_F32) return upload_f32(m, v);
  std::vector<uint16_t> h(v.size());
  for (size_t i = 0; i < v.size(); ++i) h[i] = to_half_bits(m->act, v[i]);
  return upload_bytes(m, h.data(), h.size() * 2);
}

// Symmetric per-row int8: amax/127 scale, rint(w * 127/amax), f32 arithmetic.
void quantize_rows_host(const float* w, int rows, int cols, int8_t* q, float* scale) {
  for (int r = 0; r < rows; ++r) {
    const float* x = w + static_cast<size_t>(r) * cols;
    float amax = 0.f;
    for (int c = 0; c < cols; ++c) amax = std::max(amax, std::fabs(x[c]));
    const float inv = amax > 0.f ? 127.0f / amax : 0.f;
    for (int c = 0; c < cols; ++c) {
      const float v = std::nearbyint(x[c] * inv);
      q[static_cast<size_t>(r) * cols + c] = static_cast<int8_t>(std::max(-127.f, std::min(127.f, v)));
    }
    scale[r] = amax / 127.0f;
  }
}

// A linear whose output rows are the concatenation of `names` (each
// "<prefix>.weight" [n_i, K] + "<prefix>.bias" [n_i]).
Linear load_linear(jb_model* m, const SafeTensors& st, const std::vector<std::string>& names,
                   const std::vector<int>& rows, int K, bool has_bias, int fmt_dtype,
                   bool transpose_src = false) {
  Linear L;
  L.K = K;
  L.dtype = fmt_dtype;
  for (int r : rows) L.N += r;
  std::vector<float> bias;
  if (fmt_dtype == JB_DT_S8) {
    std::vector<int8_t> q(static_cast<size_t>(L.N) * K);
    std::vector<float> sc(L.N);
    int r0 = 0;
    for (size_t i = 0; i < names.size(); ++i) {
      const std::string& nm = names[i];
      const size_t n = static_cast<size_t>(rows[i]) * K;
      if (st.has(nm + ".weight_q")) {
        auto qi = st.i8(nm + ".weight_q", static_cast<int64_t>(n));
        auto si = st.f32(nm + ".weight_scale", rows[i]);
        std::memcpy(q.data() + static_cast<size_t>(r0) * K, qi.data(), n);
        std::memcpy(sc.data() + r0, si.data(), rows[i] * 4);
      } else {
        auto w = st.f32(nm + ".weight", static_cast<int64_t>(n));
        quantize_rows_host(w.data(), rows[i], K, q.data() + static_cast<size_t>(r0) * K,
                           sc.data() + r0);
      }
      r0 += rows[i];
    }
    L.w = upload_bytes(m, q.data(), q.size());
    L.w_scale = upload_f32(m, sc);
  } else {
    std::vector<float> w;
    w.reserve(static_cast<size_t>(L.N) * K);
    for (size_t i = 0; i < names.size(); ++i) {
      auto wi = st.f32(names[i] + (transpose_src ? "" : ".weight"),
                       static_cast<int64_t>(rows[i]) * K);
      if (transpose_src) {  // stored [K, N] (OpenCLIP proj) -> [N, K]
        std::vector<float> t(wi.size());
        for (int k = 0; k < K; ++k)
          for (int n = 0; n < rows[i]; ++n) t[static_cast<size_t>(n) * K + k] = wi[static_cast<size_t>(k) * rows[i] + n];
        wi.swap(t);
      }
      w.insert(w.end(), wi.begin(), wi.end());
    }
    if (fmt_dtype == JB_DT_F32) {
      L.w = upload_f32(m, w);
    } else {
      std::vector<uint16_t> h(w.size());
      for (size_t i = 0; i < w.size(); ++i) h[i] = to_half_bits(fmt_dtype, w[i]);
      L.w = upload_bytes(m, h.data(), h.size() * 2);
    }
  }
  if (has_bias) {
    for (size_t i = 0; i < names.size(); ++i) {
      auto b = st.f32_or(names[i] + ".bias", rows[i], 0.f);
      bias.insert(bias.end(), b.begin(), b.end());
    }
    L.bias = upload_f32(m, bias);
  }
  return L;
}

int linear_dtype(int format) {
  if (format == JB_FMT_F32) return JB_DT_F32;
  if (format == JB_FMT_INT8) return JB_DT_S8;
  return format == JB_FMT_F16 ? JB_DT_F16 : JB_DT_BF16;
}

// BERT and DistilBERT share the forward (post-LN encoder, exact-erf GELU,
// additive mask); DistilBERT (crates/jammi-encoders/src/distilbert.rs:1-13)
// has no token-type table and its own config and weight names.
struct TextNames {
  std::string prefix, type_table, layer, q, k, v, o, ln1, ffn1, ffn2, ln2;
};

// ModernBert::builder().build (modernbert.rs:495-625) with ModernBertConfig's
// serde defaults (:72-90): layer_norm_eps 1e-5, global_rope_theta 160000 for
// every layer; LayerNorms without bias, linears without bias.
void load_modernbert(jb_model* m, const SafeTensors& st, const Json& cfg) {
  m->family = JB_FAMILY_BERT;
  m->variant = JB_TEXT_MODERNBERT;
  m->hidden = static_cast<int>(cfg.num_or("hidden_size", 0));
  m->layers = static_cast<int>(cfg.num_or("num_hidden_layers", 0));
  m->heads = static_cast<int>(cfg.num_or("num_attention_heads", 0));
  m->ffn = static_cast<int>(cfg.num_or("intermediate_size", 0));
  m->vocab = static_cast<int>(cfg.num_or("vocab_size", 0));
  m->max_pos = static_cast<int>(cfg.num_or("max_position_embeddings", 0));
  m->eps = static_cast<float>(cfg.num_or("layer_norm_eps", 1e-5));
  m->type_vocab = 0;
  const double theta = cfg.num_or("global_rope_theta", 160000.0);
  const int H = m->hidden, I = m->ffn;
  if (H <= 0 || m->layers <= 0 || m->heads <= 0 || I <= 0 || m->vocab <= 0 || m->max_pos <= 0)
    fail(JB_ERR_INVALID, "config.json: incomplete ModernBERT dimensions");
  if (H % m->heads)  // ModernBertBuilder::build (modernbert.rs:502-511)
    fail(JB_ERR_INVALID, "hidden_size (" + std::to_string(H) + ") must be divisible by num_attention_heads (" +
                             std::to_string(m->heads) + ")");
  if (H > 1024 || H % 8 || I % 8) fail(JB_ERR_INVALID, "ModernBERT: hidden_size and intermediate_size must be multiples of 8, hidden_size <= 1024");
  if (m->format == JB_FMT_INT8) fail(JB_ERR_INVALID, "int8 weights are defined for BERT and DistilBERT encoders");
  if (m->format == JB_FMT_F16) fail(JB_ERR_INVALID, "f16 is defined for BERT and DistilBERT encoders");
  const int d = H / m->heads;
  if (d % 2) fail(JB_ERR_INVALID, "ModernBERT: head_dim must be even (RoPE pairs)");
  const std::string p = st.has("model.embeddings.tok_embeddings.weight") ? "model." : "";
  const int ld = linear_dtype(m->format);
  const std::vector<float> zeros(H, 0.f);
  m->word = upload_act(m, st.f32(p + "embeddings.tok_embeddings.weight", int64_t(m->vocab) * H));
  m->emb_ln_g = upload_f32(m, st.f32(p + "embeddings.norm.weight", H));
  m->emb_ln_b = upload_f32(m, zeros);
  for (int l = 0; l < m->layers; ++l) {
    const std::string q = p + "layers." + std::to_string(l) + ".";
    BertLayerW w;
    w.qkv = load_linear(m, st, {q + "attn.Wqkv"}, {3 * H}, H, false, ld);
    w.o = load_linear(m, st, {q + "attn.Wo"}, {H}, H, false, ld);
    w.ffn1 = load_linear(m, st, {q + "mlp.Wi"}, {2 * I}, H, false, ld);
    w.ffn2 = load_linear(m, st, {q + "mlp.Wo"}, {H}, I, false, ld);
    if (l > 0) w.ln1_g = upload_f32(m, st.f32(q + "attn_norm.weight", H));  // layer 0: identity
    w.ln1_b = m->emb_ln_b;
    w.ln2_g = upload_f32(m, st.f32(q + "mlp_norm.weight", H));
    w.ln2_b = m->emb_ln_b;
    m->bert_layers.push_back(w);
  }
  m->final_ln_g = upload_f32(m, st.f32(p + "final_norm.weight", H));
  m->final_ln_b = m->emb_ln_b;
  // RotaryEmbedding::new (modernbert.rs:106-131): theta in f64, tables in f32
  const int half = d / 2;
  std::vector<float> c(static_cast<size_t>(m->max_pos) * half), sn(c.size());
  for (int pos = 0; pos < m->max_pos; ++pos)
    for (int i = 0; i < half; ++i) {
      const double t = static_cast<double>(pos) * std::pow(theta, -2.0 * i / static_cast<double>(d));
      c[static_cast<size_t>(pos) * half + i] = static_cast<float>(std::cos(t));
      sn[static_cast<size_t>(pos) * half + i] = static_cast<float>(std::sin(t));
    }
  m->rope_cos = upload_f32(m, c);
  m->rope_sin = upload_f32(m, sn);
}

void load_bert(jb_model* m, const SafeTensors& st, const Json& cfg) {
  m->family = JB_FAMILY_BERT;
  if (cfg.str_or("model_type", "") == "modernbert") return load_modernbert(m, st, cfg);
  const bool distil = cfg.str_or("model_type", "") == "distilbert" ||
                      (cfg.get("dim") && cfg.get("n_layers"));
  m->variant = distil ? JB_TEXT_DISTILBERT : JB_TEXT_BERT;
  TextNames nm;
  if (distil) {  // DistilBertConfig (distilbert.rs:32-57), weights under "distilbert."
    m->hidden = static_cast<int>(cfg.num_or("dim", 0));
    m->layers = static_cast<int>(cfg.num_or("n_layers", 0));
    m->heads = static_cast<int>(cfg.num_or("n_heads", 0));
    m->ffn = static_cast<int>(cfg.num_or("hidden_dim", 0));
    m->type_vocab = 0;
    nm = {"distilbert.", "", "transformer.layer.", "attention.q_lin", "attention.k_lin",
          "attention.v_lin", "attention.out_lin", "sa_layer_norm", "ffn.lin1", "ffn.lin2",
          "output_layer_norm"};
  } else {
    m->hidden = static_cast<int>(cfg.num_or("hidden_size", 0));
    m->layers = static_cast<int>(cfg.num_or("num_hidden_layers", 0));
    m->heads = static_cast<int>(cfg.num_or("num_attention_heads", 0));
    m->ffn = static_cast<int>(cfg.num_or("intermediate_size", 0));
    m->type_vocab = static_cast<int>(cfg.num_or("type_vocab_size", 2));
    // the "bert." prefix probe of BertBuilder::build (bert.rs:508-517)
    nm = {st.has("bert.embeddings.word_embeddings.weight") ? "bert." : "",
          "embeddings.token_type_embeddings.weight", "encoder.layer.", "attention.self.query",
          "attention.self.key", "attention.self.value", "attention.output.dense",
          "attention.output.LayerNorm", "intermediate.dense", "output.dense", "output.LayerNorm"};
  }
  m->vocab = static_cast<int>(cfg.num_or("vocab_size", 0));
  m->max_pos = static_cast<int>(cfg.num_or("max_position_embeddings", 0));
  m->eps = static_cast<float>(cfg.num_or("layer_norm_eps", 1e-12));
  const int H = m->hidden, F = m->ffn;
  if (H <= 0 || m->layers <= 0 || m->heads <= 0 || F <= 0 || m->vocab <= 0 || m->max_pos <= 0 ||
      H % m->heads)
    fail(JB_ERR_INVALID, "config.json: incomplete or inconsistent encoder dimensions");
  if (H > 1024 || H % 8) fail(JB_ERR_INVALID, "hidden_size must be a multiple of 8 and <= 1024");
  const std::string& p = nm.prefix;
  m->word = upload_act(m, st.f32(p + "embeddings.word_embeddings.weight", int64_t(m->vocab) * H));
  m->pos = upload_act(m, st.f32(p + "embeddings.position_embeddings.weight", int64_t(m->max_pos) * H));
  std::vector<float> tt(H, 0.f);  // token_type_ids are all zero (bert.rs:269); none in DistilBERT
  if (!nm.type_table.empty()) {
    tt = st.f32(p + nm.type_table, int64_t(m->type_vocab) * H);
    tt.resize(H);
  }
  m->type0 = upload_act(m, tt);
  m->emb_ln_g = upload_f32(m, st.f32_or(p + "embeddings.LayerNorm.weight", H, 1.f));
  m->emb_ln_b = upload_f32(m, st.f32_or(p + "embeddings.LayerNorm.bias", H, 0.f));
  const int ld = linear_dtype(m->format);
  for (int l = 0; l < m->layers; ++l) {
    const std::string q = p + nm.layer + std::to_string(l) + ".";
    BertLayerW w;
    w.qkv = load_linear(m, st, {q + nm.q, q + nm.k, q + nm.v}, {H, H, H}, H, true, ld);
    w.o = load_linear(m, st, {q + nm.o}, {H}, H, true, ld);
    w.ffn1 = load_linear(m, st, {q + nm.ffn1}, {F}, H, true, ld);
    w.ffn2 = load_linear(m, st, {q + nm.ffn2}, {H}, F, true, ld);
    w.ln1_g = upload_f32(m, st.f32_or(q + nm.ln1 + ".weight", H, 1.f));
    w.ln1_b = upload_f32(m, st.f32_or(q + nm.ln1 + ".bias", H, 0.f));
    w.ln2_g = upload_f32(m, st.f32_or(q + nm.ln2 + ".weight", H, 1.f));
    w.ln2_b = upload_f32(m, st.f32_or(q + nm.ln2 + ".bias", H, 0.f));
    m->bert_layers.push_back(w);
  }
}

void load_clip_blocks(jb_model* m, const SafeTensors& st, const std::string& p);

void load_clip(jb_model* m, const SafeTensors& st, const Json& cfg) {
  m->family = JB_FAMILY_CLIP_VISION;
  const Json* mc = cfg.get("model_cfg");
  const Json* vc = mc ? mc->get("vision_cfg") : nullptr;
  if (!mc || !vc) fail(JB_ERR_INVALID, "OpenCLIP config missing 'model_cfg.vision_cfg'");
  if (!mc->get("embed_dim")) fail(JB_ERR_INVALID, "OpenCLIP config missing 'model_cfg.embed_dim'");
  // defaults of OpenClipVisionConfig::from_open_clip_config (open_clip_vit.rs:45-101)
  m->hidden = static_cast<int>(vc->num_or("width", 768));
  m->layers = static_cast<int>(vc->num_or("layers", 12));
  m->heads = static_cast<int>(vc->num_or("heads", m->hidden / 64));
  m->ffn = static_cast<int>(m->hidden * vc->num_or("mlp_ratio", 4.0));
  m->image_size = static_cast<int>(vc->num_or("image_size", 224));
  m->patch = static_cast<int>(vc->num_or("patch_size", 32));
  m->embed_dim = static_cast<int>(mc->num_or("embed_dim", 0));
  m->gap = vc->bool_or("global_average_pool", false);
  m->eps = 1e-5f;
  // preprocess_cfg.mean / .std, three numbers each, else the OpenAI CLIP
  // defaults (open_clip_vit.rs:98-99, parse_f32_array :105-120)
  if (const Json* pc = cfg.get("preprocess_cfg")) {
    for (const char* key : {"mean", "std"}) {
      const Json* a = pc->get(key);
      if (!a || a->kind != Json::Arr || a->arr.size() < 3) continue;
      bool nums = true;
      for (int i = 0; i < 3; ++i) nums = nums && a->arr[i].kind == Json::Num;
      if (!nums) continue;
      float* dst = key[0] == 'm' ? m->img_mean : m->img_std;
      for (int i = 0; i < 3; ++i) dst[i] = static_cast<float>(a->arr[i].num);
    }
  }
  const int W = m->hidden, P = m->patch, g = m->image_size / m->patch;
  m->tokens = g * g + 1;
  m->max_pos = m->tokens;
  if (W <= 0 || W % m->heads || W % 8 || W > 1024 || m->embed_dim <= 0 || g <= 0)
    fail(JB_ERR_INVALID, "OpenCLIP config: unsupported vision dimensions");
  if (m->format == JB_FMT_INT8) fail(JB_ERR_INVALID, "int8 weights are only defined for BERT encoders");
  if (m->format == JB_FMT_F16) fail(JB_ERR_INVALID, "f16 is defined for BERT and DistilBERT encoders");
  const std::string p = st.has("visual.conv1.weight") ? "visual." : "";
  const int ld = linear_dtype(m->format);
  m->conv = load_linear(m, st, {p + "conv1"}, {W}, 3 * P * P, false, ld);
  m->cls = upload_act(m, st.f32(p + "class_embedding", W));
  m->vpos = upload_act(m, st.f32(p + "positional_embedding", int64_t(m->tokens) * W));
  m->ln_pre_g = upload_f32(m, st.f32(p + "ln_pre.weight", W));
  m->ln_pre_b = upload_f32(m, st.f32(p + "ln_pre.bias", W));
  load_clip_blocks(m, st, p);
  m->ln_post_g = upload_f32(m, st.f32(p + "ln_post.weight", W));
  m->ln_post_b = upload_f32(m, st.f32(p + "ln_post.bias", W));
  m->proj = load_linear(m, st, {p + "proj"}, {m->embed_dim}, W, false, ld, /*transpose_src=*/true);
}

// ResidualAttentionBlock weights under p + "transformer.resblocks.{l}."
// (open_clip_vit.rs:203-224, clip_text.rs:192-205: the same layout).
void load_clip_blocks(jb_model* m, const SafeTensors& st, const std::string& p) {
  const int W = m->hidden, F = m->ffn;
  const int ld = linear_dtype(m->format);
  for (int l = 0; l < m->layers; ++l) {
    const std::string q = p + "transformer.resblocks." + std::to_string(l) + ".";
    ClipBlockW w;
    // in_proj_weight / in_proj_bias use underscores (open_clip_vit.rs:139-141)
    {
      Linear L;
      L.N = 3 * W;
      L.K = W;
      L.dtype = ld;
      auto wv = st.f32(q + "attn.in_proj_weight", int64_t(3) * W * W);
      if (ld == JB_DT_F32) {
        L.w = upload_f32(m, wv);
      } else {
        std::vector<uint16_t> h(wv.size());
        for (size_t i = 0; i < wv.size(); ++i) h[i] = float_to_bf16(wv[i]);
        L.w = upload_bytes(m, h.data(), h.size() * 2);
      }
      L.bias = upload_f32(m, st.f32(q + "attn.in_proj_bias", 3 * W));
      w.qkv = L;
    }
    w.o = load_linear(m, st, {q + "attn.out_proj"}, {W}, W, true, ld);
    w.fc = load_linear(m, st, {q + "mlp.c_fc"}, {F}, W, true, ld);
    w.proj = load_linear(m, st, {q + "mlp.c_proj"}, {W}, F, true, ld);
    w.ln1_g = upload_f32(m, st.f32(q + "ln_1.weight", W));
    w.ln1_b = upload_f32(m, st.f32(q + "ln_1.bias", W));
    w.ln2_g = upload_f32(m, st.f32(q + "ln_2.weight", W));
    w.ln2_b = upload_f32(m, st.f32(q + "ln_2.bias", W));
    m->clip_blocks.push_back(w);
  }
}

// ClipText::load (clip_text.rs:251-283) with ClipTextConfig::from_open_clip_config
// (:53-102): width and layers required, heads width/64, context_length 77 and
// vocab_size 49408 by default; MLP 4 x width (:194-195); LayerNorm eps 1e-5.
void load_clip_text(jb_model* m, const SafeTensors& st, const Json& cfg) {
  m->family = JB_FAMILY_CLIP_TEXT;
  const Json* mc = cfg.get("model_cfg");
  const Json* tc = mc ? mc->get("text_cfg") : nullptr;
  if (!mc) fail(JB_ERR_INVALID, "OpenCLIP config missing 'model_cfg'");
  if (!tc) fail(JB_ERR_INVALID, "OpenCLIP config missing 'model_cfg.text_cfg'");
  if (!mc->get("embed_dim")) fail(JB_ERR_INVALID, "OpenCLIP config missing 'model_cfg.embed_dim'");
  if (!tc->get("width")) fail(JB_ERR_INVALID, "OpenCLIP config missing 'model_cfg.text_cfg.width'");
  if (!tc->get("layers")) fail(JB_ERR_INVALID, "OpenCLIP config missing 'model_cfg.text_cfg.layers'");
  m->hidden = static_cast<int>(tc->num_or("width", 0));
  m->layers = static_cast<int>(tc->num_or("layers", 0));
  m->heads = static_cast<int>(tc->num_or("heads", m->hidden / 64));
  m->max_pos = static_cast<int>(tc->num_or("context_length", 77));
  m->vocab = static_cast<int>(tc->num_or("vocab_size", 49408));
  m->embed_dim = static_cast<int>(mc->num_or("embed_dim", 0));
  m->ffn = 4 * m->hidden;
  m->eps = 1e-5f;
  const int W = m->hidden;
  if (W <= 0 || m->heads <= 0 || W % m->heads || W % 8 || W > 1024 || m->embed_dim <= 0 ||
      m->max_pos <= 0 || m->vocab <= 0 || m->layers < 0)
    fail(JB_ERR_INVALID, "OpenCLIP config: unsupported text dimensions");
  if (m->format == JB_FMT_INT8) fail(JB_ERR_INVALID, "int8 weights are only defined for BERT encoders");
  if (m->format == JB_FMT_F16) fail(JB_ERR_INVALID, "f16 is defined for BERT and DistilBERT encoders");
  const int ld = linear_dtype(m->format);
  m->word = upload_act(m, st.f32("token_embedding.weight", int64_t(m->vocab) * W));
  m->pos = upload_act(m, st.f32("positional_embedding", int64_t(m->max_pos) * W));
  load_clip_blocks(m, st, "");
  m->ln_post_g = upload_f32(m, st.f32("ln_final.weight", W));
  m->ln_post_b = upload_f32(m, st.f32("ln_final.bias", W));
  m->proj = load_linear(m, st, {"text_projection"}, {m->embed_dim}, W, false, ld, /*transpose_src=*/true);
}

void free_workspace(Workspace& ws) {
  for (void* p : ws.bufs) cudaFree(p);
  ws = Workspace();
}

size_t esz(int dt) { return dt == JB_DT_F32 ? 4 : 2; }

// Sizes of every workspace buffer for (batch, seq); shared by the allocator
// and jb_estimate_batch_bytes.
struct WsPlan {
  size_t ids, lens, cu, total, out, x, qkv, hf, aq, as, rowmax, head_t, lora_t, pixels, patches,
      patch_out, pooled;
  size_t sum() const {
    return ids + lens + cu + total + out + 4 * x + qkv + hf + aq + as + rowmax + head_t + lora_t +
           pixels + patches + patch_out + pooled;
  }
};
size_t round_up(size_t v) { return (v + 255) & ~size_t(255); }
WsPlan plan_workspace(const jb_model* m, int batch, int seq) {
  WsPlan p{};
  const size_t B = batch, S = seq, T = B * S, e = esz(m->act);
  const size_t H = m->hidden, F = m->ffn;
  p.ids = round_up(B * S * 4);
  p.lens = round_up(B * 4);
  p.cu = round_up((B + 1) * 4);
  p.total = 256;
  p.out = round_up(B * std::max<size_t>(H, m->embed_dim) * 4);
  p.x = round_up(T * H * e);
  const bool modern = m->family == JB_FAMILY_BERT && m->variant == JB_TEXT_MODERNBERT;
  // ModernBERT: hf holds Wi's [T, 2I]; the GeGLU output [T, I] reuses qkv
  p.qkv = round_up(T * (modern ? std::max(3 * H, F) : 3 * H) * e);
  p.hf = round_up(T * (modern ? 2 * F : F) * e);
  p.head_t = m->head_rank > 0 ? round_up(B * m->head_rank * 4) : 0;
  p.lora_t = m->lora_width > 0 ? round_up(T * m->lora_width * e) : 0;
  if (m->format == JB_FMT_INT8) {
    p.aq = round_up(T * std::max(H, F));
    p.as = round_up(T * 4);
    p.rowmax = round_up(T * 4);
  }
  if (m->family == JB_FAMILY_CLIP_TEXT) p.pooled = round_up(B * H * e);
  if (m->family == JB_FAMILY_CLIP_VISION) {
    const size_t g = m->image_size / m->patch;
    p.pixels = round_up(B * 3 * m->image_size * m->image_size * 4);
    p.patches = round_up(B * g * g * 3 * m->patch * m->patch * e);
    p.patch_out = round_up(B * g * g * H * e);
    p.pooled = round_up(B * H * e);
  }
  return p;
}

}  // namespace

void free_driver_stage(DriverStage& st) {
  if (st.stream) cudaStreamSynchronize(st.stream);
  for (DriverSlot& s : st.slot) {
    if (s.h_ids) cudaFreeHost(s.h_ids);
    if (s.h_lens) cudaFreeHost(s.h_lens);
    if (s.h_out) cudaFreeHost(s.h_out);
    if (s.d_ids) cudaFree(s.d_ids);
    if (s.d_lens) cudaFree(s.d_lens);
    if (s.d_out) cudaFree(s.d_out);
    if (s.done) cudaEventDestroy(s.done);
    s = DriverSlot{};
  }
  if (st.stream) cudaStreamDestroy(st.stream);
  st = DriverStage{};
}

size_t estimate_batch_bytes(const jb_model* m, int batch, int seq) {
  if (m->family == JB_FAMILY_CLIP_VISION) seq = m->tokens;
  return plan_workspace(m, batch, seq).sum();
}

void ensure_workspace(jb_model* m, int batch, int seq) {
  Workspace& ws = m->ws;
  if (batch <= ws.batch_cap && seq <= ws.seq_cap) return;
  const int nb = std::max(batch, ws.batch_cap), ns = std::max(seq, ws.seq_cap);
  clear_graphs(m);
  free_workspace(ws);
  const WsPlan p = plan_workspace(m, nb, ns);
  char* base = nullptr;
  const size_t total = p.sum();
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&base), total);
  if (e != cudaSuccess) {
    cudaGetLastError();
    fail(JB_ERR_OOM, "CUDA out of memory: workspace of " + std::to_string(total) + " bytes for batch " +
                         std::to_string(nb) + " x seq " + std::to_string(ns));
  }
  ws.bufs.push_back(base);
  ws.bytes = total;
  ws.batch_cap = nb;
  ws.seq_cap = ns;
  size_t off = 0;
  auto take = [&](size_t bytes) -> void* {
    if (!bytes) return nullptr;
    void* r = base + off;
    off += bytes;
    return r;
  };
  ws.ids = static_cast<uint32_t*>(take(p.ids));
  ws.lens = static_cast<uint32_t*>(take(p.lens));
  ws.cu = static_cast<int*>(take(p.cu));
  ws.total = static_cast<int*>(take(p.total));
  ws.out = static_cast<float*>(take(p.out));
  ws.x = take(p.x);
  ws.x1 = take(p.x);
  ws.y = take(p.x);
  ws.ctx = take(p.x);
  ws.qkv = take(p.qkv);
  ws.hf = take(p.hf);
  ws.aq = static_cast<int8_t*>(take(p.aq));
  ws.as = static_cast<float*>(take(p.as));
  ws.rowmax = static_cast<unsigned int*>(take(p.rowmax));
  ws.head_t = static_cast<float*>(take(p.head_t));
  ws.lora_t = take(p.lora_t);
  ws.pixels = static_cast<float*>(take(p.pixels));
  ws.patches = take(p.patches);
  ws.patch_out = take(p.patch_out);
  ws.pooled = take(p.pooled);
}

Workspace carve_workspace(const jb_model* m, void* base_ptr, int batch, int seq) {
  Workspace ws;
  const WsPlan p = plan_workspace(m, batch, seq);
  char* base = static_cast<char*>(base_ptr);
  size_t off = 0;
  auto take = [&](size_t bytes) -> void* {
    if (!bytes) return nullptr;
    void* r = base + off;
    off += bytes;
    return r;
  };
  ws.batch_cap = batch;
  ws.seq_cap = seq;
  ws.bytes = p.sum();
  ws.ids = static_cast<uint32_t*>(take(p.ids));
  ws.lens = static_cast<uint32_t*>(take(p.lens));
  ws.cu = static_cast<int*>(take(p.cu));
  ws.total = static_cast<int*>(take(p.total));
  ws.out = static_cast<float*>(take(p.out));
  ws.x = take(p.x);
  ws.x1 = take(p.x);
  ws.y = take(p.x);
  ws.ctx = take(p.x);
  ws.qkv = take(p.qkv);
  ws.hf = take(p.hf);
  ws.aq = static_cast<int8_t*>(take(p.aq));
  ws.as = static_cast<float*>(take(p.as));
  ws.rowmax = static_cast<unsigned int*>(take(p.rowmax));
  ws.head_t = static_cast<float*>(take(p.head_t));
  ws.lora_t = take(p.lora_t);
  ws.pixels = static_cast<float*>(take(p.pixels));
  ws.patches = take(p.patches);
  ws.patch_out = take(p.patch_out);
  ws.pooled = take(p.pooled);
  return ws;
}

jb_model* model_load(const char* path, const char* config_json, int device, int format, int family) {
  if (!path || !config_json) fail(JB_ERR_INVALID, "weights path and config must be non-null");
  if (format < JB_FMT_F32 || format > JB_FMT_F16) fail(JB_ERR_INVALID, "unknown weight format");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    fail(JB_ERR_NO_DEVICE, "no CUDA device available (require_gpu)");
  }
  if (device < 0 || device >= ndev) fail(JB_ERR_NO_DEVICE, "device ordinal out of range");
  cudaDeviceProp prop;
  check_cuda(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10)
    fail(JB_ERR_NO_DEVICE, "this library is built for sm_100a (B200); device is sm_" +
                               std::to_string(prop.major * 10 + prop.minor));
  Json cfg;
  try {
    cfg = Json::parse(config_json);
  } catch (const std::exception& e) {
    fail(JB_ERR_INVALID, std::string("config json: ") + e.what());
  }
  DeviceGuard guard(device);
  std::unique_ptr<jb_model> m(new jb_model());
  m->device = device;
  m->format = format;
  m->act = format == JB_FMT_F32 ? JB_DT_F32 : (format == JB_FMT_F16 ? JB_DT_F16 : JB_DT_BF16);
  try {
    SafeTensors st(path);
    if (family < 0) family = cfg.get("model_cfg") ? JB_FAMILY_CLIP_VISION : JB_FAMILY_BERT;
    if (family == JB_FAMILY_CLIP_VISION)
      load_clip(m.get(), st, cfg);
    else if (family == JB_FAMILY_CLIP_TEXT)
      load_clip_text(m.get(), st, cfg);
    else
      load_bert(m.get(), st, cfg);
    check_cuda(cudaMalloc(&m->d_err, sizeof(int)), "error flag");
    check_cuda(cudaMemset(m->d_err, 0, sizeof(int)), "error flag");
    check_cuda(cudaMallocHost(&m->h_err, sizeof(int)), "error flag");
    *m->h_err = 0;
    // the int8 FFN2 input quantiser looks the GELU up in a per-device table
    if (m->family == JB_FAMILY_BERT && m->format == JB_FMT_INT8)
      check_cuda(init_gelu_table(nullptr), "GELU table");
  } catch (...) {
    for (void* p : m->weight_allocs) cudaFree(p);
    if (m->d_err) cudaFree(m->d_err);
    if (m->h_err) cudaFreeHost(m->h_err);
    throw;
  }
  return m.release();
}

void model_free(jb_model* m) {
  if (!m) return;
  {
    DeviceGuard guard(m->device);
    cudaDeviceSynchronize();
    clear_graphs(m);
    if (m->graph_stream) cudaStreamDestroy(m->graph_stream);
    if (m->graph_in) cudaEventDestroy(m->graph_in);
    if (m->graph_out) cudaEventDestroy(m->graph_out);
    if (m->copy_stream) cudaStreamDestroy(m->copy_stream);
    for (cudaEvent_t e : m->copy_ev) cudaEventDestroy(e);
    free_workspace(m->ws);
    free_driver_stage(m->drv);
    if (m->img_buf) cudaFree(m->img_buf);
    for (void* p : m->weight_allocs) cudaFree(p);
    if (m->d_err) cudaFree(m->d_err);
    if (m->h_err) cudaFreeHost(m->h_err);
    profile_enable(m, false);
    for (cudaEvent_t e : m->prof_free) cudaEventDestroy(e);
  }
  delete m;
}

namespace {
cudaEvent_t take_event(jb_model* m) {
  if (!m->prof_free.empty()) {
    cudaEvent_t e = m->prof_free.back();
    m->prof_free.pop_back();
    return e;
  }
  cudaEvent_t e;
  check_cuda(cudaEventCreate(&e), "cudaEventCreate");
  return e;
}
}  // namespace

ProfScope::ProfScope(jb_model* m_, int kind, cudaStream_t s_) : m(m_), s(s_), on(m_->prof_on) {
  if (!on) return;
  rec.kind = kind;
  rec.a = take_event(m);
  rec.b = take_event(m);
  cudaEventRecord(rec.a, s);
}
ProfScope::~ProfScope() {
  if (!on) return;
  cudaEventRecord(rec.b, s);
  m->prof_recs.push_back(rec);
}

void profile_enable(jb_model* m, bool on) {
  for (auto& r : m->prof_recs) {
    m->prof_free.push_back(r.a);
    m->prof_free.push_back(r.b);
  }
  m->prof_recs.clear();
  m->prof_on = on;
}

void profile_read(jb_model* m, double* ms, int* launches) {
  for (int k = 0; k < kProfKinds; ++k) {
    ms[k] = 0;
    launches[k] = 0;
  }
  for (auto& r : m->prof_recs) {
    check_cuda(cudaEventSynchronize(r.b), "profile");
    float t = 0;
    check_cuda(cudaEventElapsedTime(&t, r.a, r.b), "profile");
    ms[r.kind] += t;
    launches[r.kind] += 1;
  }
}

void clear_graphs(jb_model* m) {
  for (GraphEntry& g : m->graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  m->graphs.clear();
}

void run_graphed(jb_model* m, int kind, int batch, int seq, int pooling, cudaStream_t s,
                 const std::function<void(cudaStream_t)>& forward) {
  if (m->prof_on) {
    forward(s);
    return;
  }
  constexpr size_t kMaxShapes = 64;
  GraphEntry* g = nullptr;
  for (GraphEntry& e : m->graphs)
    if (e.kind == kind && e.batch == batch && e.seq == seq && e.pooling == pooling) g = &e;
  if (!g) {
    if (m->graphs.size() >= kMaxShapes) {  // forget the least recently used shape
      auto lru = std::min_element(m->graphs.begin(), m->graphs.end(),
                                  [](const GraphEntry& a, const GraphEntry& b) {
                                    return a.last_use < b.last_use;
                                  });
      if (lru->exec) cudaGraphExecDestroy(lru->exec);
      m->graphs.erase(lru);
    }
    GraphEntry e;
    e.kind = kind;
    e.batch = batch;
    e.seq = seq;
    e.pooling = pooling;
    m->graphs.push_back(e);
    g = &m->graphs.back();
  }
  g->last_use = ++m->graph_clock;
  if (++g->seen < 2) {  // a shape seen once may never come back: no capture yet
    forward(s);
    return;
  }
  if (!m->graph_stream) {
    check_cuda(cudaStreamCreateWithFlags(&m->graph_stream, cudaStreamNonBlocking), "graph stream");
    check_cuda(cudaEventCreateWithFlags(&m->graph_in, cudaEventDisableTiming), "graph event");
    check_cuda(cudaEventCreateWithFlags(&m->graph_out, cudaEventDisableTiming), "graph event");
  }
  cudaStream_t gs = m->graph_stream;
  if (!g->exec) {
    check_cuda(cudaStreamBeginCapture(gs, cudaStreamCaptureModeRelaxed), "graph capture");
    cudaGraph_t graph = nullptr;
    try {
      forward(gs);
    } catch (...) {
      cudaStreamEndCapture(gs, &graph);
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      throw;
    }
    check_cuda(cudaStreamEndCapture(gs, &graph), "graph capture");
    const cudaError_t e = cudaGraphInstantiate(&g->exec, graph, 0);
    cudaGraphDestroy(graph);
    check_cuda(e, "graph instantiate");
  }
  check_cuda(cudaEventRecord(m->graph_in, s), "graph order");
  check_cuda(cudaStreamWaitEvent(gs, m->graph_in, 0), "graph order");
  check_cuda(cudaGraphLaunch(g->exec, gs), "graph launch");
  check_cuda(cudaEventRecord(m->graph_out, gs), "graph order");
  check_cuda(cudaStreamWaitEvent(s, m->graph_out, 0), "graph order");
}

void set_projection_head(jb_model* m, const float* a, const float* b, int rank, double alpha) {
  if (m->family != JB_FAMILY_BERT) fail(JB_ERR_INVALID, "projection heads apply to text models");
  if (rank < 0 || (rank > 0 && (!a || !b))) fail(JB_ERR_INVALID, "projection head: bad arguments");
  cudaDeviceSynchronize();  // no forward may still read the old head or workspace
  clear_graphs(m);
  free_workspace(m->ws);
  m->weight_bytes -= 2ll * m->head_rank * m->hidden * 4;
  auto drop = [&](float*& p) {
    if (!p) return;
    cudaFree(p);
    m->weight_allocs.erase(std::remove(m->weight_allocs.begin(), m->weight_allocs.end(),
                                       static_cast<void*>(p)),
                           m->weight_allocs.end());
    p = nullptr;
  };
  drop(m->head_a);
  drop(m->head_b);
  m->head_rank = 0;
  if (rank == 0) return;
  const size_t n = static_cast<size_t>(rank) * m->hidden;
  const float scale = static_cast<float>(alpha / rank);  // LoraLinear::from_loaded
  std::vector<float> bs(b, b + n);
  for (float& v : bs) v *= scale;
  m->head_a = static_cast<float*>(upload_bytes(m, a, n * 4));
  m->head_b = static_cast<float*>(upload_bytes(m, bs.data(), n * 4));
  m->head_rank = rank;
}

namespace {
// Frees a device matrix that upload_* allocated for this model.
void drop_dev(jb_model* m, void*& p, size_t bytes) {
  if (!p) return;
  cudaFree(p);
  m->weight_allocs.erase(std::remove(m->weight_allocs.begin(), m->weight_allocs.end(), p),
                         m->weight_allocs.end());
  m->weight_bytes -= static_cast<int64_t>(bytes);
  p = nullptr;
}
size_t linear_bytes(const jb_model* m, const Linear& L) {
  return static_cast<size_t>(L.N) * L.K * (m->act == JB_DT_F32 ? 4 : 2);
}
int pad8(int r) { return (r + 7) / 8 * 8; }

// A [Rp, in] stacking the sites' A rows (zeros after), B [sum(out), Rp]
// block-diagonal with each site's scaling folded in; Linear in the activation
// dtype (w == nullptr when every site has rank 0).
void build_fused(jb_model* m, const LoraSiteHost* const* sites, const int* outs, int n, int in,
                 Linear& A, Linear& B) {
  drop_dev(m, A.w, linear_bytes(m, A));
  drop_dev(m, B.w, linear_bytes(m, B));
  A = Linear();
  B = Linear();
  int R = 0, O = 0;
  for (int i = 0; i < n; ++i) {
    R += sites[i]->rank;
    O += outs[i];
  }
  if (R == 0) return;
  const int Rp = pad8(R);
  std::vector<float> a(static_cast<size_t>(Rp) * in, 0.f), b(static_cast<size_t>(O) * Rp, 0.f);
  int r0 = 0, o0 = 0;
  for (int i = 0; i < n; ++i) {
    const LoraSiteHost& st = *sites[i];
    for (int r = 0; r < st.rank; ++r)
      std::copy(st.a.begin() + static_cast<size_t>(r) * in, st.a.begin() + static_cast<size_t>(r + 1) * in,
                a.begin() + static_cast<size_t>(r0 + r) * in);
    for (int o = 0; o < outs[i] && st.rank; ++o)
      for (int r = 0; r < st.rank; ++r)
        b[static_cast<size_t>(o0 + o) * Rp + r0 + r] =
            static_cast<float>(st.b[static_cast<size_t>(o) * st.rank + r] * st.scaling);
    r0 += st.rank;
    o0 += outs[i];
  }
  A.w = upload_act(m, a);
  A.dtype = m->act;
  A.N = Rp;
  A.K = in;
  B.w = upload_act(m, b);
  B.dtype = m->act;
  B.N = O;
  B.K = Rp;
}
}  // namespace

void set_lora(jb_model* m, int layer, int site, const float* a, const float* b, int rank,
              double scaling) {
  if (m->family != JB_FAMILY_BERT) fail(JB_ERR_INVALID, "LoRA adapters apply to text encoders");
  if (m->format == JB_FMT_INT8 || m->format == JB_FMT_F16)
    fail(JB_ERR_INVALID, "LoRA adapters run in the f32 and bf16 formats");
  if (m->variant == JB_TEXT_MODERNBERT)
    fail(JB_ERR_INVALID, "LoRA adapters are wired for the BERT and DistilBERT layer layout");
  if (layer < 0 || layer >= m->layers || site < 0 || site >= kLoraSites || rank < 0 ||
      (rank > 0 && (!a || !b)))
    fail(JB_ERR_INVALID, "LoRA: bad layer, site or rank");
  const int H = m->hidden, F = m->ffn;
  const int in[kLoraSites] = {H, H, H, H, H, F};
  const int out[kLoraSites] = {H, H, H, H, F, H};
  cudaDeviceSynchronize();  // no forward may still read the old matrices or workspace
  clear_graphs(m);
  free_workspace(m->ws);
  if (m->lora.empty()) m->lora.resize(m->layers);
  LoraLayerW& L = m->lora[layer];
  LoraSiteHost& st = L.site[site];
  st.rank = rank;
  st.scaling = scaling;
  st.a.assign(a ? a : nullptr, a ? a + static_cast<size_t>(rank) * in[site] : nullptr);
  st.b.assign(b ? b : nullptr, b ? b + static_cast<size_t>(out[site]) * rank : nullptr);
  if (site < 3) {
    const LoraSiteHost* qkv[3] = {&L.site[0], &L.site[1], &L.site[2]};
    const int outs[3] = {H, H, H};
    build_fused(m, qkv, outs, 3, H, L.a_qkv, L.b_qkv);
  } else {
    const LoraSiteHost* one[1] = {&st};
    const int outs[1] = {out[site]};
    Linear& A = site == 3 ? L.a_o : site == 4 ? L.a_1 : L.a_2;
    Linear& B = site == 3 ? L.b_o : site == 4 ? L.b_1 : L.b_2;
    build_fused(m, one, outs, 1, in[site], A, B);
  }
  m->lora_width = 0;
  for (const LoraLayerW& l : m->lora)
    for (const Linear* A : {&l.a_qkv, &l.a_o, &l.a_1, &l.a_2}) m->lora_width = std::max(m->lora_width, A->N);
}

int load_lora(jb_model* m, const char* path, double alpha, bool rslora) {
  // Adapter keys: layer.{n}.{module}.lora_a / .lora_b (bert.rs:299-346,
  // distilbert.rs:245-296), sites in the order query, key, value, attention
  // output, FFN in, FFN out.
  static const char* kBertSites[kLoraSites] = {"query", "key", "value", "dense",
                                                "intermediate_dense", "output_dense"};
  static const char* kDistilSites[kLoraSites] = {"q_lin", "k_lin", "v_lin", "out_lin", "lin1", "lin2"};
  const char* const* kSites = m->variant == JB_TEXT_DISTILBERT ? kDistilSites : kBertSites;
  SafeTensors st(path);
  int n = 0;
  for (int l = 0; l < m->layers; ++l)
    for (int s = 0; s < kLoraSites; ++s) {
      const std::string k = "layer." + std::to_string(l) + "." + kSites[s];
      if (!st.has(k + ".lora_a") || !st.has(k + ".lora_b")) continue;
      const StTensor& ta = st.get(k + ".lora_a");
      if (ta.shape.size() != 2) fail(JB_ERR_IO, k + ".lora_a must be [rank, in]");
      const int rank = static_cast<int>(ta.shape[0]);
      const int64_t in = ta.shape[1];
      const int64_t outd = (s == 4 ? m->ffn : m->hidden);
      if (in != (s == 5 ? m->ffn : m->hidden)) fail(JB_ERR_IO, k + ".lora_a has the wrong width");
      const std::vector<float> a = st.f32(k + ".lora_a", rank * in);
      const std::vector<float> b = st.f32(k + ".lora_b", rank * outd);
      const double scaling = rslora ? alpha / std::sqrt(static_cast<double>(rank)) : alpha / rank;
      set_lora(m, l, s, a.data(), b.data(), rank, scaling);
      ++n;
    }
  return n;
}

void load_projection_head(jb_model* m, const char* path, double alpha) {
  SafeTensors st(path);
  if (!st.has("projection.lora_a") || !st.has("projection.lora_b")) return;  // Ok(None)
  const StTensor& ta = st.get("projection.lora_a");
  if (ta.shape.size() != 2 || ta.shape[1] != m->hidden)
    fail(JB_ERR_IO, "projection.lora_a must be [rank, hidden]");
  const int rank = static_cast<int>(ta.shape[0]);
  const std::vector<float> a = st.f32("projection.lora_a", static_cast<int64_t>(rank) * m->hidden);
  const std::vector<float> b = st.f32("projection.lora_b", static_cast<int64_t>(rank) * m->hidden);
  set_projection_head(m, a.data(), b.data(), rank, alpha);
}

void check_device_flag(jb_model* m, cudaStream_t s) {
  // the flag rides the stream behind the forward's own copies: one wait
  check_cuda(cudaMemcpyAsync(m->h_err, m->d_err, sizeof(int), cudaMemcpyDeviceToHost, s), "error flag read");
  check_cuda(cudaStreamSynchronize(s), "forward");
  const int flag = *m->h_err;
  if (!flag) return;
  cudaMemset(m->d_err, 0, sizeof(int));
  if (flag & kErrTimeout) fail(JB_ERR_TIMEOUT, "a device-side wait exceeded its limit");
  if (flag & 2) fail(JB_ERR_INVALID, "token id out of range for the vocabulary");
  if (flag & 4) fail(JB_ERR_INVALID, "a row length exceeds max_seq");
  fail(JB_ERR_CUDA, "device error flag " + std::to_string(flag));
}

#define PROF_MEM_CALL(expr, name)        \
  do {                                   \
    ProfScope ps_(m, kProfMemory, s);    \
    check_cuda((expr), name);            \
  } while (0)

namespace {
void run_linear(jb_model* m, const Linear& L, const void* A, const float* a_scale, int Mcap,
                const int* dM, void* C, int c_dtype, int epi, const void* resid, cudaStream_t s,
                unsigned int* row_max = nullptr) {
  GemmArgs g;
  g.row_max = row_max;
  g.A = A;
  g.W = L.w;
  g.ab_dtype = L.dtype;
  g.M = Mcap;
  g.dM = dM;
  g.N = L.N;
  g.K = L.K;
  g.bias = L.bias;
  g.resid = resid;
  g.a_scale = a_scale;
  g.w_scale = L.w_scale;
  g.C = C;
  g.c_dtype = c_dtype;
  g.epi = epi;
  g.err = m->d_err;
  std::string why;
  ProfScope ps(m, kProfLinear, s);
  cudaError_t e = launch_gemm(g, s, &why);
  if (e != cudaSuccess) {
    if (!why.empty()) fail(JB_ERR_INVALID, why);
    check_cuda(e, "linear");
  }
}
void run_ln(jb_model* m, const void* x, const void* resid, const float* g, const float* b, void* y, int8_t* yq,
            float* ys, int dtype, int rows, const int* drows, int cols, float eps, cudaStream_t s,
            unsigned int* zero_rows = nullptr) {
  LnArgs a;
  a.zero_rows = zero_rows;
  a.x = x;
  a.resid = resid;
  a.gamma = g;
  a.beta = b;
  a.y = y;
  a.yq = yq;
  a.yscale = ys;
  a.dtype = dtype;
  a.rows = rows;
  a.drows = drows;
  a.cols = cols;
  a.eps = eps;
  ProfScope ps(m, kProfMemory, s);
  check_cuda(launch_layernorm(a, s), "layernorm");
}
}  // namespace

namespace {
// The attention kernels' work counter: 128 bytes into the workspace's 256-byte
// `total` slot, whose first int is the packed row count.
int* attn_work(const Workspace& ws) { return ws.total + 32; }
}  // namespace

namespace {
// ModernBert::forward_hidden (modernbert.rs:318-340) over packed rows, cu in
// ws.cu: embedding norm; per layer x += Wo(attn(rope(Wqkv(attn_norm(x)))))
// (layer 0 without attn_norm) and x += mlp.Wo(geglu(Wi(mlp_norm(x))));
// final_norm.  Returns the buffer holding the final hidden states.
void* modernbert_forward(jb_model* m, const uint32_t* d_ids, int batch, int max_seq, cudaStream_t s) {
  Workspace& ws = m->ws;
  const int H = m->hidden, I = m->ffn, Mcap = batch * max_seq, act = m->act;
  EmbedArgs ea;
  ea.ids = d_ids;
  ea.cu = ws.cu;
  ea.word = m->word;
  ea.gamma = m->emb_ln_g;
  ea.beta = m->emb_ln_b;
  ea.y = ws.x;
  ea.dtype = act;
  ea.batch = batch;
  ea.max_seq = max_seq;
  ea.H = H;
  ea.vocab = m->vocab;
  ea.eps = m->eps;
  ea.err = m->d_err;
  PROF_MEM_CALL(launch_embed_ln(ea, s), "embeddings");
  for (const BertLayerW& w : m->bert_layers) {
    // ModernBertAttention::forward (modernbert.rs:178-227)
    const void* h = ws.x;
    if (w.ln1_g) {
      run_ln(m, ws.x, nullptr, w.ln1_g, w.ln1_b, ws.x1, nullptr, nullptr, act, Mcap, ws.total, H, m->eps, s);
      h = ws.x1;
    }
    run_linear(m, w.qkv, h, nullptr, Mcap, ws.total, ws.qkv, act, JB_EPI_NONE, nullptr, s);
    PROF_MEM_CALL(launch_rope_qk(ws.qkv, act, ws.cu, batch, max_seq, m->heads, H / m->heads, m->rope_cos,
                                 m->rope_sin, s),
                  "rope");
    std::string why;
    cudaError_t e;
    {
      ProfScope ps(m, kProfAttention, s);
      e = launch_attention(ws.qkv, ws.cu, ws.ctx, act, batch, m->heads, H / m->heads, max_seq, s, &why,
                           Mcap, m->d_err, 0, attn_work(ws));
    }
    if (e != cudaSuccess) {
      if (!why.empty()) fail(JB_ERR_INVALID, why);
      check_cuda(e, "attention");
    }
    run_linear(m, w.o, ws.ctx, nullptr, Mcap, ws.total, ws.y, act, JB_EPI_RESIDUAL, ws.x, s);
    // ModernBertMlp::forward (modernbert.rs:241-254); the GeGLU output reuses qkv
    run_ln(m, ws.y, nullptr, w.ln2_g, w.ln2_b, ws.x1, nullptr, nullptr, act, Mcap, ws.total, H, m->eps, s);
    run_linear(m, w.ffn1, ws.x1, nullptr, Mcap, ws.total, ws.hf, act, JB_EPI_NONE, nullptr, s);
    PROF_MEM_CALL(launch_geglu(ws.hf, ws.qkv, act, Mcap, ws.total, I, s), "geglu");
    run_linear(m, w.ffn2, ws.qkv, nullptr, Mcap, ws.total, ws.x, act, JB_EPI_RESIDUAL, ws.y, s);
  }
  run_ln(m, ws.x, nullptr, m->final_ln_g, m->final_ln_b, ws.x1, nullptr, nullptr, act, Mcap, ws.total, H,
         m->eps, s);
  return ws.x1;
}
}  // namespace

void bert_forward_device(jb_model* m, const uint32_t* d_ids, const uint32_t* d_lens, int batch,
                         int max_seq, int pooling, float* d_out, float* d_hidden, cudaStream_t s) {
  Workspace& ws = m->ws;
  const int H = m->hidden, Mcap = batch * max_seq;
  const bool q8 = m->format == JB_FMT_INT8;
  const int act = m->act;
  PROF_MEM_CALL(launch_lens_to_cu(d_lens, batch, max_seq, ws.cu, ws.total, m->d_err, s), "lengths");
  void* hid = ws.x;  // the final hidden states
  if (m->variant == JB_TEXT_MODERNBERT) {
    hid = modernbert_forward(m, d_ids, batch, max_seq, s);
  } else {
    EmbedArgs ea;
    ea.ids = d_ids;
    ea.cu = ws.cu;
    ea.word = m->word;
    ea.pos = m->pos;
    ea.type0 = m->type0;
    ea.gamma = m->emb_ln_g;
    ea.beta = m->emb_ln_b;
    ea.y = ws.x;
    ea.yq = q8 ? ws.aq : nullptr;
    ea.yscale = q8 ? ws.as : nullptr;
    ea.dtype = act;
    ea.batch = batch;
    ea.max_seq = max_seq;
    ea.H = H;
    ea.vocab = m->vocab;
    ea.eps = m->eps;
    ea.err = m->d_err;
    PROF_MEM_CALL(launch_embed_ln(ea, s), "embeddings");
    int layer_idx = 0;
    for (const BertLayerW& w : m->bert_layers) {
      const LoraLayerW* lw = m->lora.empty() ? nullptr : &m->lora[layer_idx];
      ++layer_idx;
      // base(x) + scaling (x A^T) B^T: T = x A^T, then C += T B^T in place
      auto lora = [&](const Linear& A, const Linear& B, const void* x, void* C) {
        if (!A.w) return;
        run_linear(m, A, x, nullptr, Mcap, ws.total, ws.lora_t, act, JB_EPI_NONE, nullptr, s);
        run_linear(m, B, ws.lora_t, nullptr, Mcap, ws.total, C, act, JB_EPI_RESIDUAL, C, s);
      };
      // BertSelfAttention (bert.rs:135-155): fused QKV projection
      run_linear(m, w.qkv, q8 ? ws.aq : ws.x, ws.as, Mcap, ws.total, ws.qkv, act, JB_EPI_NONE, nullptr, s);
      if (lw) lora(lw->a_qkv, lw->b_qkv, ws.x, ws.qkv);
      std::string why;
      cudaError_t e;
      {
        ProfScope ps(m, kProfAttention, s);
        e = launch_attention(ws.qkv, ws.cu, ws.ctx, act, batch, m->heads, H / m->heads, max_seq, s,
                             &why, Mcap, m->d_err, 0, attn_work(ws));
      }
      if (e != cudaSuccess) {
        if (!why.empty()) fail(JB_ERR_INVALID, why);
        check_cuda(e, "attention");
      }
      if (q8) PROF_MEM_CALL(launch_quantize_rows(ws.ctx, act, ws.aq, ws.as, Mcap, ws.total, H, s), "quantize");
      // BertSelfOutput (bert.rs:164-167): LN(dense(ctx) + x)
      run_linear(m, w.o, q8 ? ws.aq : ws.ctx, ws.as, Mcap, ws.total, ws.y, act, JB_EPI_RESIDUAL, ws.x, s);
      if (lw) lora(lw->a_o, lw->b_o, ws.ctx, ws.y);
      run_ln(m, ws.y, nullptr, w.ln1_g, w.ln1_b, ws.x1, q8 ? ws.aq : nullptr, q8 ? ws.as : nullptr, act,
             Mcap, ws.total, H, m->eps, s, q8 ? ws.rowmax : nullptr);
      // BertIntermediate (bert.rs:187-190): gelu_erf(dense(x1)).  int8: the
      // GELU runs in the quantiser that FFN2's input needs anyway, on the bf16
      // dense output (the reference's bf16 order: Linear -> bf16 -> gelu);
      // the dense's epilogue records each row's largest output (rows zeroed
      // by the LayerNorm above), which fixes the row's scale in advance.
      const bool lora1 = lw && lw->a_1.w;  // the adapter adds before the activation
      run_linear(m, w.ffn1, q8 ? ws.aq : ws.x1, ws.as, Mcap, ws.total, ws.hf, act,
                 (q8 || lora1) ? JB_EPI_NONE : JB_EPI_GELU, nullptr, s, q8 ? ws.rowmax : nullptr);
      if (lora1) {
        lora(lw->a_1, lw->b_1, ws.x1, ws.hf);
        PROF_MEM_CALL(launch_gelu_rows(ws.hf, act, Mcap, ws.total, m->ffn, s), "gelu");
      }
      if (q8)
        PROF_MEM_CALL(launch_gelu_quantize_rowmax(ws.hf, ws.rowmax, ws.aq, ws.as, Mcap, ws.total,
                                                  m->ffn, s),
                      "quantize");
      // BertOutput (bert.rs:199-202): LN(dense(h) + x1)
      run_linear(m, w.ffn2, q8 ? ws.aq : ws.hf, ws.as, Mcap, ws.total, ws.y, act, JB_EPI_RESIDUAL, ws.x1, s);
      if (lw) lora(lw->a_2, lw->b_2, ws.hf, ws.y);
      run_ln(m, ws.y, nullptr, w.ln2_g, w.ln2_b, ws.x, q8 ? ws.aq : nullptr, q8 ? ws.as : nullptr, act,
             Mcap, ws.total, H, m->eps, s);
    }
  }
  if (d_hidden)
    PROF_MEM_CALL(launch_unpack_hidden(hid, act, ws.cu, d_hidden, batch, max_seq, H, s), "unpack");
  if (d_out) {
    PROF_MEM_CALL(launch_pool_normalize(hid, act, ws.cu, d_out, batch, H, pooling, s), "pooling");
    if (m->head_rank > 0) {  // projection head: d_out += (d_out A^T) (s B)^T, f32
      Linear la, lb;
      la.w = m->head_a;
      la.dtype = JB_DT_F32;
      la.N = m->head_rank;
      la.K = H;
      lb.w = m->head_b;
      lb.dtype = JB_DT_F32;
      lb.N = H;
      lb.K = m->head_rank;
      run_linear(m, la, d_out, nullptr, batch, nullptr, ws.head_t, JB_DT_F32, JB_EPI_NONE, nullptr, s);
      run_linear(m, lb, ws.head_t, nullptr, batch, nullptr, d_out, JB_DT_F32, JB_EPI_RESIDUAL, d_out, s);
    }
  }
}

namespace {
// The ResidualAttentionBlock stack (open_clip_vit.rs:226-236; clip_text.rs:207-217
// with the causal mask) over packed rows: the input in ws.x, rows <= rows_cap
// (*d_rows when given), cu in ws.cu.  Returns the buffer holding the output.
void* clip_blocks_forward(jb_model* m, int rows_cap, const int* d_rows, int batch, int max_len,
                          int causal, cudaStream_t s) {
  Workspace& ws = m->ws;
  const int W = m->hidden, act = m->act;
  void* x = ws.x;
  void* y = ws.y;
  for (const ClipBlockW& w : m->clip_blocks) {
    run_ln(m, x, nullptr, w.ln1_g, w.ln1_b, ws.x1, nullptr, nullptr, act, rows_cap, d_rows, W, m->eps, s);
    run_linear(m, w.qkv, ws.x1, nullptr, rows_cap, d_rows, ws.qkv, act, JB_EPI_NONE, nullptr, s);
    std::string why;
    cudaError_t e;
    {
      ProfScope ps(m, kProfAttention, s);
      e = launch_attention(ws.qkv, ws.cu, ws.ctx, act, batch, m->heads, W / m->heads, max_len, s, &why,
                           rows_cap, m->d_err, causal, attn_work(ws));
    }
    if (e != cudaSuccess) {
      if (!why.empty()) fail(JB_ERR_INVALID, why);
      check_cuda(e, "attention");
    }
    run_linear(m, w.o, ws.ctx, nullptr, rows_cap, d_rows, y, act, JB_EPI_RESIDUAL, x, s);
    std::swap(x, y);
    run_ln(m, x, nullptr, w.ln2_g, w.ln2_b, ws.x1, nullptr, nullptr, act, rows_cap, d_rows, W, m->eps, s);
    run_linear(m, w.fc, ws.x1, nullptr, rows_cap, d_rows, ws.hf, act, JB_EPI_QUICK_GELU, nullptr, s);
    run_linear(m, w.proj, ws.hf, nullptr, rows_cap, d_rows, y, act, JB_EPI_RESIDUAL, x, s);
    std::swap(x, y);
  }
  return x;
}
}  // namespace

void clip_text_forward_device(jb_model* m, const uint32_t* d_ids, int batch, int S, float* d_out,
                              cudaStream_t s) {
  Workspace& ws = m->ws;
  const int W = m->hidden, act = m->act, Mcap = batch * S;
  // rows end at their EOT token: under the causal mask no later position
  // reaches the pooled one, so only the prefix up to it is computed
  PROF_MEM_CALL(launch_eot_lens(d_ids, batch, S, ws.lens, s), "eot");
  PROF_MEM_CALL(launch_lens_to_cu(ws.lens, batch, S, ws.cu, ws.total, m->d_err, s), "lengths");
  // token_embedding(ids) + positional_embedding[..S] (clip_text.rs:309-312)
  EmbedArgs ea;
  ea.ids = d_ids;
  ea.cu = ws.cu;
  ea.word = m->word;
  ea.pos = m->pos;
  ea.y = ws.x;
  ea.dtype = act;
  ea.batch = batch;
  ea.max_seq = S;
  ea.H = W;
  ea.vocab = m->vocab;
  ea.err = m->d_err;
  PROF_MEM_CALL(launch_embed_ln(ea, s), "embeddings");
  void* x = clip_blocks_forward(m, Mcap, ws.total, batch, S, 1, s);
  // ln_final at the EOT position, @ text_projection, L2 (clip_text.rs:319-330, 379-389)
  PROF_MEM_CALL(launch_vit_pool_ln(x, m->ln_post_g, m->ln_post_b, ws.pooled, act, batch, 0, W, 0,
                                   m->eps, s, ws.cu),
                "eot pool");
  run_linear(m, m->proj, ws.pooled, nullptr, batch, nullptr, d_out, JB_DT_F32, JB_EPI_NONE, nullptr, s);
  PROF_MEM_CALL(launch_l2_rows(d_out, batch, m->embed_dim, s), "l2");
}

void clip_forward_device(jb_model* m, const float* d_px, int batch, float* d_out, cudaStream_t s) {
  Workspace& ws = m->ws;
  const int W = m->hidden, T = m->tokens, g = m->image_size / m->patch, act = m->act;
  const int Mrows = batch * T, Prows = batch * g * g;
  PROF_MEM_CALL(launch_patchify(d_px, ws.patches, act, batch, m->image_size, m->patch, s), "patchify");
  // conv1: kernel = stride = patch, no bias (open_clip_vit.rs:259-269, 313)
  run_linear(m, m->conv, ws.patches, nullptr, Prows, nullptr, ws.patch_out, act, JB_EPI_NONE, nullptr, s);
  // CLS cat + positional add + ln_pre (open_clip_vit.rs:319-330)
  PROF_MEM_CALL(launch_vit_embed_ln(ws.patch_out, m->cls, m->vpos, m->ln_pre_g, m->ln_pre_b, ws.x, act,
                                 batch, T, W, m->eps, s),
             "vit embed");
  PROF_MEM_CALL(launch_fill_cu_uniform(ws.cu, batch, T, s), "cu");
  void* x = clip_blocks_forward(m, Mrows, nullptr, batch, T, 0, s);
  // CLS (or GAP) pool -> ln_post -> proj (open_clip_vit.rs:339-352), then l2_normalize (candle.rs:425-438)
  PROF_MEM_CALL(launch_vit_pool_ln(x, m->ln_post_g, m->ln_post_b, ws.pooled, act, batch, T, W,
                                m->gap ? 1 : 0, m->eps, s),
             "vit pool");
  run_linear(m, m->proj, ws.pooled, nullptr, batch, nullptr, d_out, JB_DT_F32, JB_EPI_NONE, nullptr, s);
  PROF_MEM_CALL(launch_l2_rows(d_out, batch, m->embed_dim, s), "l2");
}

}  // namespace jb
