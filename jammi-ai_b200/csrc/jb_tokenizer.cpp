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
//
// The OpenCLIP text tower's tokenizer is the reference's load_open_clip_bpe
// (crates/jammi-ai/src/model/clip_bpe.rs:52-217), a `tokenizers` BPE built from
// OpenCLIP's merges file: vocabulary = the 256 byte symbols of the GPT-2 /
// CLIP byte-to-printable-code-point table, the same with the "</w>"
// end-of-word suffix, each merge joined, then <|startoftext|> and
// <|endoftext|>; no normaliser; the CLIP regex as an isolating pre-tokeniser
// (the special-token literals, the contractions 's 't 're 've 'm 'll 'd,
// letter runs, single digits, runs of other non-space characters; the spans
// between matches are pre-tokens too); per pre-token, each character a symbol
// (the last one with "</w>"), characters outside the vocabulary dropped (the
// model has no unknown token), then the lowest-ranked adjacent pair merged
// first (leftmost on ties) until none applies; <|startoftext|> ... <|endoftext|>
// around the sequence.
#include <algorithm>
#include <cstring>
#include <fstream>
#include <zlib.h>
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
  int kind = 0;  // 0: BERT WordPiece, 1: OpenCLIP BPE
  // BPE: (left id, right id) -> (rank, merged id)
  std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> merges;
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

bool is_letter(uint32_t c) { return in_table(uni::kLetter, c); }
bool is_number(uint32_t c) { return in_table(uni::kNumber, c); }

// Length (in code points) of the CLIP pre-tokeniser's match at position i,
// 0 if no alternative matches there; alternatives are tried in the regex's
// order, the first that matches wins.
size_t clip_match(const std::vector<uint32_t>& c, size_t i) {
  static const char* const kLiterals[] = {"<|startoftext|>", "<|endoftext|>", "'s", "'t", "'re",
                                          "'ve", "'m", "'ll", "'d"};
  for (const char* lit : kLiterals) {
    const size_t len = std::strlen(lit);
    if (i + len > c.size()) continue;
    size_t k = 0;
    while (k < len && c[i + k] == static_cast<unsigned char>(lit[k])) ++k;
    if (k == len) return len;
  }
  if (is_letter(c[i])) {
    size_t j = i + 1;
    while (j < c.size() && is_letter(c[j])) ++j;
    return j - i;
  }
  if (is_number(c[i])) return 1;
  if (is_whitespace(c[i])) return 0;
  size_t j = i + 1;
  while (j < c.size() && !is_whitespace(c[j]) && !is_letter(c[j]) && !is_number(c[j])) ++j;
  return j - i;
}

void bpe_word(const jb_tokenizer& t, const std::vector<uint32_t>& c, size_t b, size_t e,
              std::vector<uint32_t>& ids) {
  std::vector<uint32_t> sym;
  std::string s;
  for (size_t k = b; k < e; ++k) {
    s.clear();
    append_utf8(c[k], s);
    if (k + 1 == e) s += "</w>";
    auto it = t.vocab.find(s);
    if (it != t.vocab.end()) sym.push_back(it->second);  // unknown characters are dropped
  }
  while (sym.size() > 1) {
    uint32_t best_rank = UINT32_MAX, best_id = 0;
    size_t best_pos = 0;
    for (size_t k = 0; k + 1 < sym.size(); ++k) {
      auto it = t.merges.find((static_cast<uint64_t>(sym[k]) << 32) | sym[k + 1]);
      if (it != t.merges.end() && it->second.first < best_rank) {
        best_rank = it->second.first;
        best_id = it->second.second;
        best_pos = k;
      }
    }
    if (best_rank == UINT32_MAX) break;
    sym[best_pos] = best_id;
    sym.erase(sym.begin() + best_pos + 1);
  }
  ids.insert(ids.end(), sym.begin(), sym.end());
}

void encode_clip(const jb_tokenizer& t, const char* s, size_t n, std::vector<uint32_t>& ids) {
  std::vector<uint32_t> c;
  decode_utf8(s, n, c);
  size_t seg = 0;
  for (size_t i = 0; i < c.size();) {
    const size_t len = clip_match(c, i);
    if (len == 0) {
      ++i;
      continue;
    }
    if (seg < i) bpe_word(t, c, seg, i, ids);  // the span between matches
    bpe_word(t, c, i, i + len, ids);
    i += len;
    seg = i;
  }
  if (seg < c.size()) bpe_word(t, c, seg, c.size(), ids);
}

// One segment of text between added tokens: normalise, pre-tokenise, WordPiece.
void encode_segment(const jb_tokenizer& t, const char* s, size_t n, std::vector<uint32_t>& ids) {
  if (t.kind == 1) return encode_clip(t, s, n, ids);
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

// The GPT-2 / CLIP byte-to-printable-code-point table: bytes 33-126, 161-172
// and 174-255 map to themselves, the other 68 bytes, in ascending order, to
// 256, 257, ...
std::vector<uint32_t> byte_symbols() {
  std::vector<uint32_t> out(256);
  uint32_t extra = 0;
  for (uint32_t b = 0; b < 256; ++b) {
    const bool direct = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
    out[b] = direct ? b : 256 + extra++;
  }
  return out;
}

std::string read_maybe_gzip(const char* path) {
  gzFile f = gzopen(path, "rb");  // reads plain files unchanged
  if (!f) fail(JB_ERR_IO, std::string("cannot open ") + path);
  std::string data;
  char buf[1 << 16];
  int n;
  while ((n = gzread(f, buf, sizeof(buf))) > 0) data.append(buf, static_cast<size_t>(n));
  const bool bad = n < 0;
  gzclose(f);
  if (bad) fail(JB_ERR_IO, std::string("cannot decompress ") + path);
  return data;
}

jb_tokenizer* load_clip(const char* path) {
  // OpenCLIP's vocabulary: 49408 = 256 + 256 + 48894 merges + 2 specials
  constexpr size_t kMaxMerges = 49408 - 256 - 2 - 256;
  const std::string text = read_maybe_gzip(path);
  std::vector<std::pair<std::string, std::string>> merges;
  size_t line = 0;
  for (size_t pos = 0; pos <= text.size() && merges.size() < kMaxMerges;) {
    size_t nl = text.find('\n', pos);
    if (nl == std::string::npos) nl = text.size();
    if (line++ > 0) {  // line 0 is a header
      std::istringstream ls(text.substr(pos, nl - pos));
      std::string a, b;
      if (ls >> a >> b) merges.emplace_back(a, b);
    }
    pos = nl + 1;
  }
  if (merges.empty()) fail(JB_ERR_IO, std::string("no BPE merges in ") + path);
  std::unique_ptr<jb_tokenizer> t(new jb_tokenizer());
  t->kind = 1;
  const std::vector<uint32_t> bytes = byte_symbols();
  std::vector<std::string> vocab;
  for (uint32_t c : bytes) {
    std::string s;
    append_utf8(c, s);
    vocab.push_back(s);
  }
  for (uint32_t c : bytes) {
    std::string s;
    append_utf8(c, s);
    vocab.push_back(s + "</w>");
  }
  for (const auto& m : merges) vocab.push_back(m.first + m.second);
  vocab.push_back("<|startoftext|>");
  vocab.push_back("<|endoftext|>");
  for (size_t i = 0; i < vocab.size(); ++i) t->vocab[vocab[i]] = static_cast<uint32_t>(i);
  for (size_t r = 0; r < merges.size(); ++r) {
    auto a = t->vocab.find(merges[r].first), b = t->vocab.find(merges[r].second);
    auto ab = t->vocab.find(merges[r].first + merges[r].second);
    if (a == t->vocab.end() || b == t->vocab.end() || ab == t->vocab.end())
      fail(JB_ERR_IO, "BPE merge " + std::to_string(r + 1) + " names a symbol not in the vocabulary");
    t->merges[(static_cast<uint64_t>(a->second) << 32) | b->second] =
        {static_cast<uint32_t>(r), ab->second};
  }
  t->before.push_back(static_cast<uint32_t>(vocab.size() - 2));
  t->after.push_back(static_cast<uint32_t>(vocab.size() - 1));
  return t.release();
}

}  // namespace
}  // namespace jb

extern "C" {

jb_status jb_tokenizer_load_clip_bpe(const char* merges_path, jb_tokenizer** out) {
  if (!out) return jb::record_error(JB_ERR_INVALID, "null output handle");
  *out = nullptr;
  try {
    if (!merges_path) jb::fail(JB_ERR_INVALID, "null path");
    *out = jb::load_clip(merges_path);
    return JB_OK;
  } catch (const jb::Error& e) {
    return jb::record_error(e.status, e.msg);
  } catch (const std::exception& e) {
    return jb::record_error(JB_ERR_INVALID, e.what());
  }
}

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
