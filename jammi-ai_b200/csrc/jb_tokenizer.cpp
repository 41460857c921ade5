// BERT WordPiece tokenizer on the host: texts -> token ids in the ragged
// layout jb_generate_embeddings takes, so a caller goes from text to
// embeddings without another runtime.
//
// The reference tokenises with the HuggingFace `tokenizers` crate from a
// model's tokenizer.json (TokenizerWrapper, crates/jammi-ai/src/model/
// tokenizer.rs:21-78; encode_batch with add_special_tokens and optional
// truncation).  This restates that crate's pipeline for the BERT family's
// tokenizer.json layout:
//   added tokens   special tokens ([CLS], [SEP], [MASK], ...) are matched in
//                  the raw text first, leftmost, longest at a position, and
//                  become their own ids;
//   BertNormalizer clean_text (drop NUL, U+FFFD and category C* except
//                  \t \n \r; whitespace -> ' '), handle_chinese_chars
//                  (spaces around CJK ideographs), strip_accents (NFD, then
//                  drop category Mn; on by default when lowercase is), then
//                  lowercase (one code point at a time);
//   BertPreTokenizer split on White_Space, each punctuation character
//                  (ASCII punctuation or category P*) a word of its own;
//   WordPiece      greedy longest-match-first per word, continuation pieces
//                  prefixed ("##"), a word longer than max_input_chars_per_word
//                  or with no full cover -> the unknown token;
//   post-processor TemplateProcessing "[CLS] $A [SEP]" or BertProcessing:
//                  the special ids around the sequence;
//   truncation     max_length counts the special ids; the sequence's tail is
//                  cut.
// Unicode data (categories, lowercase, canonical decompositions and
// combining classes) comes from jb_unicode_tables.h.
#include <algorithm>
#include <cstring>
#include <fstream>
#include <memory>
#include <sstream>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "jb_json.h"
#include "jb_model.h"
#include "jb_unicode_tables.h"

struct jb_tokenizer {
  bool clean_text = true, handle_chinese = true, strip_accents = true, lowercase = true;
  std::unordered_map<std::string, uint32_t> vocab;
  uint32_t unk_id = 0;
  std::string prefix = "##";
  int max_chars = 100;
  std::vector<uint32_t> before, after;  // special ids around the sequence
  std::vector<std::pair<std::string, uint32_t>> added;  // matched in the raw text
};

namespace jb {
namespace {

using uni::CpRange;

bool in_ranges(const CpRange* r, size_t n, uint32_t cp) {
  size_t lo = 0, hi = n;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (cp < r[mid].lo)
      hi = mid;
    else if (cp > r[mid].hi)
      lo = mid + 1;
    else
      return true;
  }
  return false;
}
template <size_t N>
bool in_table(const CpRange (&r)[N], uint32_t cp) {
  return in_ranges(r, N, cp);
}
template <size_t N>
const uni::SeqEntry* find_seq(const uni::SeqEntry (&t)[N], uint32_t cp) {
  const uni::SeqEntry* it =
      std::lower_bound(t, t + N, cp, [](const uni::SeqEntry& e, uint32_t c) { return e.cp < c; });
  return (it != t + N && it->cp == cp) ? it : nullptr;
}
uint8_t ccc(uint32_t cp) {
  const size_t n = sizeof(uni::kCcc) / sizeof(uni::kCcc[0]);
  const uni::CccEntry* it = std::lower_bound(
      uni::kCcc, uni::kCcc + n, cp, [](const uni::CccEntry& e, uint32_t c) { return e.cp < c; });
  return (it != uni::kCcc + n && it->cp == cp) ? it->ccc : 0;
}

// The White_Space property.
bool is_whitespace(uint32_t c) {
  return (c >= 0x9 && c <= 0xD) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
         (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F ||
         c == 0x205F || c == 0x3000;
}
bool is_control(uint32_t c) {  // category C*, \t \n \r excepted
  if (c == '\t' || c == '\n' || c == '\r') return false;
  return in_table(uni::kOther, c);
}
bool is_punct(uint32_t c) {
  if ((c >= 33 && c <= 47) || (c >= 58 && c <= 64) || (c >= 91 && c <= 96) || (c >= 123 && c <= 126))
    return true;
  return in_table(uni::kPunct, c);
}
bool is_cjk(uint32_t c) {
  return (c >= 0x4E00 && c <= 0x9FFF) || (c >= 0x3400 && c <= 0x4DBF) ||
         (c >= 0x20000 && c <= 0x2A6DF) || (c >= 0x2A700 && c <= 0x2B73F) ||
         (c >= 0x2B740 && c <= 0x2B81F) || (c >= 0x2B920 && c <= 0x2CEAF) ||
         (c >= 0xF900 && c <= 0xFAFF) || (c >= 0x2F800 && c <= 0x2FA1F);
}

// UTF-8 -> code points; an invalid byte sequence decodes to U+FFFD.
void decode_utf8(const char* s, size_t n, std::vector<uint32_t>& out) {
  const unsigned char* p = reinterpret_cast<const unsigned char*>(s);
  size_t i = 0;
  while (i < n) {
    const unsigned char b = p[i];
    uint32_t cp = 0xFFFD;
    int len = 1;
    if (b < 0x80) {
      cp = b;
    } else if ((b >> 5) == 0x6 && i + 1 < n && (p[i + 1] >> 6) == 0x2) {
      cp = ((b & 0x1F) << 6) | (p[i + 1] & 0x3F);
      len = 2;
      if (cp < 0x80) cp = 0xFFFD;
    } else if ((b >> 4) == 0xE && i + 2 < n && (p[i + 1] >> 6) == 0x2 && (p[i + 2] >> 6) == 0x2) {
      cp = ((b & 0x0F) << 12) | ((p[i + 1] & 0x3F) << 6) | (p[i + 2] & 0x3F);
      len = 3;
      if (cp < 0x800 || (cp >= 0xD800 && cp <= 0xDFFF)) cp = 0xFFFD;
    } else if ((b >> 3) == 0x1E && i + 3 < n && (p[i + 1] >> 6) == 0x2 && (p[i + 2] >> 6) == 0x2 &&
               (p[i + 3] >> 6) == 0x2) {
      cp = ((b & 0x07) << 18) | ((p[i + 1] & 0x3F) << 12) | ((p[i + 2] & 0x3F) << 6) | (p[i + 3] & 0x3F);
      len = 4;
      if (cp < 0x10000 || cp > 0x10FFFF) cp = 0xFFFD;
    }
    out.push_back(cp);
    i += len;
  }
}
void append_utf8(uint32_t c, std::string& s) {
  if (c < 0x80) {
    s.push_back(static_cast<char>(c));
  } else if (c < 0x800) {
    s.push_back(static_cast<char>(0xC0 | (c >> 6)));
    s.push_back(static_cast<char>(0x80 | (c & 0x3F)));
  } else if (c < 0x10000) {
    s.push_back(static_cast<char>(0xE0 | (c >> 12)));
    s.push_back(static_cast<char>(0x80 | ((c >> 6) & 0x3F)));
    s.push_back(static_cast<char>(0x80 | (c & 0x3F)));
  } else {
    s.push_back(static_cast<char>(0xF0 | (c >> 18)));
    s.push_back(static_cast<char>(0x80 | ((c >> 12) & 0x3F)));
    s.push_back(static_cast<char>(0x80 | ((c >> 6) & 0x3F)));
    s.push_back(static_cast<char>(0x80 | (c & 0x3F)));
  }
}

// Canonical decomposition (NFD): full decompositions from the table, Hangul
// syllables by the Unicode algorithm, then the canonical ordering of each run
// of combining marks by combining class (stable).
void nfd(const std::vector<uint32_t>& in, std::vector<uint32_t>& out) {
  out.clear();
  for (uint32_t c : in) {
    if (c >= 0xAC00 && c < 0xAC00 + 11172) {
      const uint32_t s = c - 0xAC00;
      out.push_back(0x1100 + s / 588);
      out.push_back(0x1161 + (s % 588) / 28);
      if (s % 28) out.push_back(0x11A7 + s % 28);
    } else if (const uni::SeqEntry* e = find_seq(uni::kDecomp, c)) {
      out.insert(out.end(), uni::kDecomp_seq + e->off, uni::kDecomp_seq + e->off + e->n);
    } else {
      out.push_back(c);
    }
  }
  for (size_t i = 0; i < out.size();) {
    if (ccc(out[i]) == 0) {
      ++i;
      continue;
    }
    size_t j = i;
    while (j < out.size() && ccc(out[j]) != 0) ++j;
    std::stable_sort(out.begin() + i, out.begin() + j,
                     [](uint32_t a, uint32_t b) { return ccc(a) < ccc(b); });
    i = j;
  }
}

void normalize(const jb_tokenizer& t, std::vector<uint32_t>& cps) {
  std::vector<uint32_t> tmp;
  if (t.clean_text) {
    tmp.clear();
    for (uint32_t c : cps) {
      if (c == 0 || c == 0xFFFD || is_control(c)) continue;
      tmp.push_back(is_whitespace(c) ? 0x20 : c);
    }
    cps.swap(tmp);
  }
  if (t.handle_chinese) {
    tmp.clear();
    for (uint32_t c : cps) {
      if (is_cjk(c)) {
        tmp.push_back(0x20);
        tmp.push_back(c);
        tmp.push_back(0x20);
      } else {
        tmp.push_back(c);
      }
    }
    cps.swap(tmp);
  }
  if (t.strip_accents) {
    nfd(cps, tmp);
    cps.clear();
    for (uint32_t c : tmp)
      if (!in_table(uni::kMarkNonspacing, c)) cps.push_back(c);
  }
  if (t.lowercase) {
    tmp.clear();
    for (uint32_t c : cps) {
      if (const uni::SeqEntry* e = find_seq(uni::kLower, c))
        tmp.insert(tmp.end(), uni::kLower_seq + e->off, uni::kLower_seq + e->off + e->n);
      else
        tmp.push_back(c);
    }
    cps.swap(tmp);
  }
}

void wordpiece(const jb_tokenizer& t, const std::vector<uint32_t>& word, std::vector<uint32_t>& ids) {
  if (word.empty()) return;
  if (static_cast<int>(word.size()) > t.max_chars) {
    ids.push_back(t.unk_id);
    return;
  }
  std::vector<uint32_t> pieces;
  size_t start = 0;
  std::string sub;
  while (start < word.size()) {
    size_t end = word.size();
    bool found = false;
    uint32_t id = 0;
    while (start < end) {
      sub.clear();
      if (start > 0) sub = t.prefix;
      for (size_t k = start; k < end; ++k) append_utf8(word[k], sub);
      auto it = t.vocab.find(sub);
      if (it != t.vocab.end()) {
        found = true;
        id = it->second;
        break;
      }
      --end;
    }
    if (!found) {
      ids.push_back(t.unk_id);
      return;
    }
    pieces.push_back(id);
    start = end;
  }
  ids.insert(ids.end(), pieces.begin(), pieces.end());
}

// One segment of text between added tokens: normalise, pre-tokenise, WordPiece.
void encode_segment(const jb_tokenizer& t, const char* s, size_t n, std::vector<uint32_t>& ids) {
  std::vector<uint32_t> cps;
  decode_utf8(s, n, cps);
  normalize(t, cps);
  std::vector<uint32_t> word;
  for (uint32_t c : cps) {
    if (is_whitespace(c)) {
      wordpiece(t, word, ids);
      word.clear();
    } else if (is_punct(c)) {
      wordpiece(t, word, ids);
      word.assign(1, c);
      wordpiece(t, word, ids);
      word.clear();
    } else {
      word.push_back(c);
    }
  }
  wordpiece(t, word, ids);
}

void encode(const jb_tokenizer& t, const char* s, size_t n, int max_length,
            std::vector<uint32_t>& out) {
  std::vector<uint32_t> ids;
  size_t seg = 0;
  for (size_t i = 0; i < n;) {
    size_t best = 0;
    uint32_t best_id = 0;
    for (const auto& a : t.added)
      if (a.first.size() > best && a.first.size() <= n - i && std::memcmp(s + i, a.first.data(), a.first.size()) == 0) {
        best = a.first.size();
        best_id = a.second;
      }
    if (best) {
      encode_segment(t, s + seg, i - seg, ids);
      ids.push_back(best_id);
      i += best;
      seg = i;
    } else {
      ++i;
    }
  }
  encode_segment(t, s + seg, n - seg, ids);
  const size_t specials = t.before.size() + t.after.size();
  if (max_length > 0) {
    const size_t keep = static_cast<size_t>(max_length) > specials ? max_length - specials : 0;
    if (ids.size() > keep) ids.resize(keep);
  }
  out.clear();
  out.insert(out.end(), t.before.begin(), t.before.end());
  out.insert(out.end(), ids.begin(), ids.end());
  out.insert(out.end(), t.after.begin(), t.after.end());
}

uint32_t token_id(const jb_tokenizer& t, const std::string& tok) {
  auto it = t.vocab.find(tok);
  if (it == t.vocab.end()) fail(JB_ERR_IO, "tokenizer.json: special token " + tok + " is not in the vocabulary");
  return it->second;
}

jb_tokenizer* load(const char* path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) fail(JB_ERR_IO, std::string("cannot open ") + path);
  std::stringstream ss;
  ss << f.rdbuf();
  Json j;
  try {
    j = Json::parse(ss.str());
  } catch (const std::exception& e) {
    fail(JB_ERR_IO, std::string("tokenizer.json: ") + e.what());
  }
  std::unique_ptr<jb_tokenizer> t(new jb_tokenizer());
  const Json* model = j.get("model");
  if (!model || model->str_or("type", "") != "WordPiece")
    fail(JB_ERR_INVALID, "tokenizer.json: only the WordPiece model (BERT family) is supported");
  const Json* vocab = model->get("vocab");
  if (!vocab || vocab->kind != Json::Obj) fail(JB_ERR_IO, "tokenizer.json: model.vocab missing");
  for (const auto& kv : vocab->obj) t->vocab[kv.first] = static_cast<uint32_t>(kv.second.num);
  t->prefix = model->str_or("continuing_subword_prefix", "##");
  t->max_chars = static_cast<int>(model->num_or("max_input_chars_per_word", 100));
  t->unk_id = token_id(*t, model->str_or("unk_token", "[UNK]"));
  if (const Json* nz = j.get("normalizer"); nz && nz->kind == Json::Obj) {
    if (nz->str_or("type", "") != "BertNormalizer")
      fail(JB_ERR_INVALID, "tokenizer.json: only the BertNormalizer is supported");
    t->clean_text = nz->bool_or("clean_text", true);
    t->handle_chinese = nz->bool_or("handle_chinese_chars", true);
    t->lowercase = nz->bool_or("lowercase", true);
    const Json* sa = nz->get("strip_accents");
    t->strip_accents = (sa && sa->kind == Json::Bool) ? sa->b : t->lowercase;
  } else {
    t->clean_text = t->handle_chinese = t->strip_accents = t->lowercase = false;
  }
  if (const Json* pt = j.get("pre_tokenizer"); pt && pt->kind == Json::Obj &&
                                              pt->str_or("type", "") != "BertPreTokenizer")
    fail(JB_ERR_INVALID, "tokenizer.json: only the BertPreTokenizer is supported");
  if (const Json* pp = j.get("post_processor"); pp && pp->kind == Json::Obj) {
    const std::string type = pp->str_or("type", "");
    if (type == "BertProcessing") {
      const Json* cls = pp->get("cls");
      const Json* sep = pp->get("sep");
      if (!cls || !sep || cls->arr.size() < 2 || sep->arr.size() < 2)
        fail(JB_ERR_IO, "tokenizer.json: BertProcessing needs cls and sep");
      t->before.push_back(static_cast<uint32_t>(cls->arr[1].num));
      t->after.push_back(static_cast<uint32_t>(sep->arr[1].num));
    } else if (type == "TemplateProcessing") {
      const Json* single = pp->get("single");
      const Json* specials = pp->get("special_tokens");
      if (!single || single->kind != Json::Arr) fail(JB_ERR_IO, "tokenizer.json: template without 'single'");
      bool seen_seq = false;
      for (const Json& item : single->arr) {
        if (item.get("Sequence")) {
          seen_seq = true;
          continue;
        }
        const Json* sp = item.get("SpecialToken");
        if (!sp) fail(JB_ERR_INVALID, "tokenizer.json: unsupported template item");
        const std::string name = sp->str_or("id", "");
        const Json* def = specials ? specials->get(name) : nullptr;
        const Json* ids = def ? def->get("ids") : nullptr;
        std::vector<uint32_t> v;
        if (ids && ids->kind == Json::Arr)
          for (const Json& x : ids->arr) v.push_back(static_cast<uint32_t>(x.num));
        else
          v.push_back(token_id(*t, name));
        auto& dst = seen_seq ? t->after : t->before;
        dst.insert(dst.end(), v.begin(), v.end());
      }
    } else {
      fail(JB_ERR_INVALID, "tokenizer.json: unsupported post-processor " + type);
    }
  }
  if (const Json* added = j.get("added_tokens"); added && added->kind == Json::Arr)
    for (const Json& a : added->arr) {
      const std::string content = a.str_or("content", "");
      if (!content.empty()) t->added.emplace_back(content, static_cast<uint32_t>(a.num_or("id", 0)));
    }
  return t.release();
}

}  // namespace
}  // namespace jb

extern "C" {

jb_status jb_tokenizer_load(const char* tokenizer_json_path, jb_tokenizer** out) {
  if (!out) return jb::record_error(JB_ERR_INVALID, "null output handle");
  *out = nullptr;
  try {
    if (!tokenizer_json_path) jb::fail(JB_ERR_INVALID, "null path");
    *out = jb::load(tokenizer_json_path);
    return JB_OK;
  } catch (const jb::Error& e) {
    return jb::record_error(e.status, e.msg);
  } catch (const std::exception& e) {
    return jb::record_error(JB_ERR_INVALID, e.what());
  }
}

void jb_tokenizer_free(jb_tokenizer* t) { delete t; }

jb_status jb_tokenize(const jb_tokenizer* t, const char* const* texts, const uint64_t* text_bytes,
                      int64_t n, int max_length, uint32_t* ids, uint64_t ids_capacity,
                      uint64_t* offsets) {
  try {
    if (!t || n < 0 || !offsets || (n > 0 && (!texts || !text_bytes)))
      jb::fail(JB_ERR_INVALID, "jb_tokenize: bad argument");
    std::vector<std::vector<uint32_t>> rows(static_cast<size_t>(n));
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const int64_t workers = n >= 256 ? std::min<int64_t>(hw, (n + 127) / 128) : 1;
    auto work = [&](int64_t w) {
      for (int64_t i = w; i < n; i += workers)
        jb::encode(*t, texts[i] ? texts[i] : "", texts[i] ? text_bytes[i] : 0, max_length, rows[i]);
    };
    if (workers == 1) {
      work(0);
    } else {
      std::vector<std::thread> pool;
      for (int64_t w = 0; w < workers; ++w) pool.emplace_back(work, w);
      for (auto& th : pool) th.join();
    }
    offsets[0] = 0;
    for (int64_t i = 0; i < n; ++i) offsets[i + 1] = offsets[i] + rows[i].size();
    if (!ids) return JB_OK;  // size query
    if (offsets[n] > ids_capacity)
      jb::fail(JB_ERR_INVALID, "jb_tokenize: the ids buffer holds " + std::to_string(ids_capacity) +
                                   " ids, the texts need " + std::to_string(offsets[n]));
    for (int64_t i = 0; i < n; ++i) std::copy(rows[i].begin(), rows[i].end(), ids + offsets[i]);
    return JB_OK;
  } catch (const jb::Error& e) {
    return jb::record_error(e.status, e.msg);
  } catch (const std::exception& e) {
    return jb::record_error(JB_ERR_INVALID, e.what());
  }
}

}  // extern "C"
