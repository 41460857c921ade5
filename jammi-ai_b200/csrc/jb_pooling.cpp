// The pooling a sentence-transformers checkpoint declares in
// 1_Pooling/config.json, mapped to a JB_POOL_* strategy the way the reference
// selects it when it loads a text encoder (pooling_from_config,
// crates/jammi-ai/src/model/backend/candle.rs:440-538, reading the file as
// read_local_pooling_config, crates/jammi-ai/src/model/resolver.rs:473-500):
//   no file                      -> mean (the bare BERT repo default);
//   a present file               -> a JSON object whose pooling_mode_* flags
//                                   that are boolean true all name one
//                                   strategy: cls_token -> cls, mean_tokens and
//                                   mean_sqrt_len_tokens -> mean (the L2
//                                   normalisation makes the two identical),
//                                   max_tokens -> max, weightedmean_tokens ->
//                                   weighted mean;
//   anything else (not an object, no true flag, an unrepresentable flag such
//   as pooling_mode_lasttoken, two strategies at once, an unreadable or
//   unparseable file) is an error, never a silent mean.
#include <cerrno>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include <sys/stat.h>

#include "jb_json.h"
#include "jb_model.h"

namespace jb {
namespace {

int pooling_of(const Json& cfg) {
  if (cfg.kind != Json::Obj) fail(JB_ERR_INVALID, "1_Pooling/config.json is not a JSON object");
  static const struct {
    const char* flag;
    int pooling;
  } kRecognized[] = {
      {"pooling_mode_cls_token", JB_POOL_CLS},
      {"pooling_mode_mean_tokens", JB_POOL_MEAN},
      {"pooling_mode_max_tokens", JB_POOL_MAX},
      {"pooling_mode_weightedmean_tokens", JB_POOL_WEIGHTED_MEAN},
      {"pooling_mode_mean_sqrt_len_tokens", JB_POOL_MEAN},
  };
  std::vector<std::string> true_flags, unsupported;
  for (const auto& kv : cfg.obj)
    if (kv.first.rfind("pooling_mode_", 0) == 0 && kv.second.kind == Json::Bool && kv.second.b)
      true_flags.push_back(kv.first);
  if (true_flags.empty())
    fail(JB_ERR_INVALID, "1_Pooling/config.json is present but declares no true pooling_mode_* flag");
  std::vector<int> distinct;
  for (const std::string& f : true_flags) {
    int p = -1;
    for (const auto& r : kRecognized)
      if (f == r.flag) p = r.pooling;
    if (p < 0) {
      unsupported.push_back(f);
      continue;
    }
    bool seen = false;
    for (int d : distinct) seen |= d == p;
    if (!seen) distinct.push_back(p);
  }
  if (!unsupported.empty()) {
    std::string names;
    for (const std::string& u : unsupported) names += (names.empty() ? "" : ", ") + u;
    fail(JB_ERR_INVALID, "unsupported pooling mode(s) " + names +
                             " declared in 1_Pooling/config.json: the engine cannot serve this encoder correctly");
  }
  if (distinct.size() > 1)
    fail(JB_ERR_INVALID, "1_Pooling/config.json declares " + std::to_string(distinct.size()) +
                             " distinct pooling strategies; concatenated modes are not representable");
  return distinct[0];
}

int pooling_of_text(const std::string& text) {
  Json j;
  try {
    j = Json::parse(text);
  } catch (const std::exception& e) {
    fail(JB_ERR_INVALID, std::string("1_Pooling/config.json is present but unparseable: ") + e.what());
  }
  return pooling_of(j);
}

template <typename F>
jb_status guarded_pooling(int* out, F&& f) {
  if (!out) return record_error(JB_ERR_INVALID, "null output");
  try {
    *out = f();
    return JB_OK;
  } catch (const Error& e) {
    return record_error(e.status, e.msg);
  } catch (const std::exception& e) {
    return record_error(JB_ERR_INVALID, e.what());
  }
}

}  // namespace
}  // namespace jb

extern "C" {

jb_status jb_pooling_from_config(const char* pooling_config_json, int* pooling) {
  return jb::guarded_pooling(pooling, [&] {
    return pooling_config_json ? jb::pooling_of_text(pooling_config_json) : static_cast<int>(JB_POOL_MEAN);
  });
}

jb_status jb_pooling_from_model_dir(const char* model_dir, int* pooling) {
  return jb::guarded_pooling(pooling, [&] {
    if (!model_dir) jb::fail(JB_ERR_INVALID, "null model directory");
    const std::string path = std::string(model_dir) + "/1_Pooling/config.json";
    struct stat st;
    if (stat(path.c_str(), &st) != 0) {
      if (errno == ENOENT || errno == ENOTDIR) return static_cast<int>(JB_POOL_MEAN);  // genuinely absent
      jb::fail(JB_ERR_IO, "1_Pooling/config.json is present but could not be opened: " +
                              std::string(std::strerror(errno)));
    }
    std::ifstream f(path, std::ios::binary);
    if (!f || S_ISDIR(st.st_mode))
      jb::fail(JB_ERR_IO, "1_Pooling/config.json is present but could not be opened");
    std::stringstream ss;
    ss << f.rdbuf();
    return jb::pooling_of_text(ss.str());
  });
}

}  // extern "C"
