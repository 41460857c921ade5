// Host tokenizers: texts -> token ids in the ragged layout
// jb_generate_embeddings takes, so a caller goes from text to embeddings
// without another runtime.
//
// The reference tokenises with the HuggingFace `tokenizers` crate from a
// model's tokenizer.json, any architecture (TokenizerWrapper, crates/jammi-ai/
// src/model/tokenizer.rs:21-78; encode_batch with add_special_tokens and
// optional truncation), or from OpenCLIP's merges file (load_open_clip_bpe,
// crates/jammi-ai/src/model/clip_bpe.rs:52-217).  This restates that crate's
// pipeline for the tokenizer.json components the encoder families use:
//   added tokens   matched leftmost-longest, first those flagged
//                  normalized=false in the raw text, then those flagged
//                  normalized=true in each normalised piece between them;
//                  lstrip / rstrip swallow the whitespace beside a match,
//                  single_word rejects a match inside a word;
//   normaliser     BertNormalizer: clean_text (drop NUL, U+FFFD and
//                  category C* except \t \n \r; whitespace -> ' '),
//                  handle_chinese_chars (spaces around CJK ideographs),
//                  strip_accents (NFD, then drop category Mn; on by default
//                  when lowercase is), lowercase (one code point at a time);
//                  NFC, NFD, NFKC, NFKD, Lowercase, StripAccents (drop category M*, no
//                  decomposition of its own), Strip, Prepend (non-empty
//                  pieces), Replace (string patterns, or the regexes \s+
//                  and ' {2,}'), Precompiled (sentencepiece's character map,
//                  a darts-clone double array, applied per UAX #29 extended
//                  grapheme cluster of under 6 bytes, else per character,
//                  shortest matching key first), and Sequences;
//   pre-tokeniser  (a Sequence applies its steps in order, each to the words
//                  the previous one produced)
//                  BertPreTokenizer: split on White_Space, each punctuation
//                  character (ASCII punctuation or category P*) a word of its
//                  own; ByteLevel: an optional leading space (add_prefix_space,
//                  per piece), the GPT-2 regex ('s 't 're 've 'm 'll 'd,
//                  ' ?' + letters / numbers / other, whitespace runs that
//                  leave their last space to the next word), each word's
//                  UTF-8 bytes mapped to the byte-symbol alphabet below;
//                  Whitespace: the matches of \w+|[^\w\s]+; WhitespaceSplit;
//                  Punctuation with its split behaviour (isolated, removed,
//                  merged with the previous / next word, contiguous); Digits
//                  (each digit, or digit runs); Split on a literal string
//                  (the empty one matches at every character boundary) or on
//                  the CLIP, GPT-2 or \s+ regular expression, matched by
//                  hand (any other regex is refused), inverted or not, with
//                  any split behaviour; Metaspace (' ' -> the replacement,
//                  prepended always / at the text's start / never, split
//                  before each replacement);
//                  OpenCLIP's regex (the special-token literals, the
//                  contractions, letter runs, single digits, runs of other
//                  non-space characters; the spans between matches are words
//                  too);
//   model          WordPiece: greedy longest-match-first per word,
//                  continuation pieces prefixed ("##"), a word longer than
//                  max_input_chars_per_word or with no full cover -> the
//                  unknown token.  BPE: each character a symbol (continuing
//                  prefix on all but the first, end-of-word suffix on the
//                  last), a character outside the vocabulary -> its
//                  <0xXX> byte tokens (byte_fallback), else the unknown token
//                  (consecutive ones fused with fuse_unk), else dropped; then
//                  the lowest-ranked adjacent pair merged first (leftmost on
//                  ties) until none applies; ignore_merges takes a word found
//                  whole in the vocabulary as one token.  WordLevel: the word's
//                  id, else the unknown token's, else an error.  Unigram:
//                  Viterbi over the vocabulary's scores (below);
//   post-processor TemplateProcessing, BertProcessing, RobertaProcessing,
//                  ByteLevel (ids unchanged) and Sequences of these: special
//                  ids around the sequence;
//   truncation     max_length counts the special ids and cuts the sequence's
//                  tail; without one, tokenizer.json's own truncation (with
//                  its direction) applies.
// OpenCLIP's merges file becomes the same structure: vocabulary = the 256
// byte symbols, the same with the "</w>" end-of-word suffix, each merge
// joined, then <|startoftext|> and <|endoftext|>; no normaliser; the OpenCLIP
// regex; BPE with "</w>" and no unknown token; <|startoftext|> ...
// <|endoftext|> around the sequence.
// Unicode data (categories, lowercase, canonical decompositions, combining
// classes, NFC composites, word characters) comes from jb_unicode_tables.h.

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <queue>
#include <sstream>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include <zlib.h>

#include "jb_json.h"
#include "jb_model.h"
#include "jb_unicode_tables.h"

namespace jb {
namespace {

struct AddedToken {
  std::string content;
  uint32_t id = 0;
  bool lstrip = false, rstrip = false, single_word = false;
};

// Added tokens indexed by first byte, longest first within a byte, so a
// position's leftmost-longest match is the first candidate that matches.
struct AddedSet {
  std::vector<AddedToken> toks;
  std::vector<std::vector<uint32_t>> by_first = std::vector<std::vector<uint32_t>>(256);
  void add(const AddedToken& t) {
    toks.push_back(t);
    auto& v = by_first[static_cast<unsigned char>(t.content[0])];
    v.push_back(static_cast<uint32_t>(toks.size() - 1));
    std::stable_sort(v.begin(), v.end(), [this](uint32_t a, uint32_t b) {
      return toks[a].content.size() > toks[b].content.size();
    });
  }
};

enum NormOp { kNormBert, kNormNfc, kNormNfd, kNormNfkc, kNormNfkd, kNormLower, kNormStripAccents, kNormStrip, kNormPrepend, kNormReplace,
              kNormReplaceSpaceRuns, kNormReplaceSpaces2, kNormPrecompiled };
struct NormStep {
  int op = kNormBert;
  bool left = false, right = false;  // Strip
  std::vector<uint32_t> a, b;        // Prepend: a; Replace: a -> b
};
enum PreKind { kPreBert, kPreByteLevel, kPreClip, kPreWhitespace, kPreWhitespaceSplit, kPrePunctuation, kPreDigits,
               kPreSplit, kPreMetaspace };
enum PrependScheme { kPrependAlways, kPrependFirst, kPrependNever };
enum Behavior { kIsolated, kRemoved, kMergedWithPrevious, kMergedWithNext, kContiguous };
// Split patterns: a literal string, or one of the regular expressions the
// encoder families' tokenizer.json files use, matched by hand.
enum Pattern { kPatLiteral, kPatClip, kPatClipSpecials, kPatGpt2, kPatSpaceRuns };
struct PreStep {
  int kind = kPreBert;
  bool add_prefix_space = false, use_regex = true;  // ByteLevel
  int behavior = kIsolated;                         // Punctuation, Split
  bool individual_digits = false;                   // Digits
  int pattern = kPatLiteral;                        // Split
  std::vector<uint32_t> literal;                    // Split, kPatLiteral
  bool invert = false;                              // Split
  uint32_t replacement = 0x2581;                    // Metaspace
  int prepend_scheme = kPrependAlways;              // Metaspace
  bool split = true;                                // Metaspace
};
enum ModelKind { kWordPiece, kBpe, kWordLevel, kUnigram };

// sentencepiece's precompiled character map: a darts-clone double array
// over UTF-8 keys whose values index NUL-terminated replacements.
struct CharsMap {
  std::vector<uint32_t> units;
  std::string normalized;
};

// The Unigram vocabulary as a byte trie: edges (parent << 8 | byte) ->
// child, sorted for binary search; piece[node] = vocabulary id or -1.
struct PieceTrie {
  std::vector<std::pair<uint64_t, uint32_t>> edges;
  std::vector<int32_t> piece;
};

}  // namespace
}  // namespace jb

struct jb_tokenizer {
  int model = jb::kWordPiece;
  // normaliser and pre-tokeniser steps, applied in order
  std::vector<jb::NormStep> norm;
  bool clean_text = true, handle_chinese = true, strip_accents = true, lowercase = true;
  std::vector<jb::PreStep> pre;
  std::unordered_map<std::string, uint32_t> vocab;
  bool has_unk = false;
  uint32_t unk_id = 0;
  // WordPiece
  std::string prefix = "##";
  int max_chars = 100;
  // BPE: (left id, right id) -> (rank, merged id)
  std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> merges;
  std::string bpe_prefix, bpe_suffix;
  bool fuse_unk = false, byte_fallback = false, ignore_merges = false;
  // Unigram: scores by id, the piece trie, the lowest score
  std::vector<double> scores;
  jb::PieceTrie trie;
  double min_score = 0.0;
  jb::CharsMap charsmap;  // Precompiled normaliser
  std::vector<uint32_t> before, after;  // special ids around the sequence
  jb::AddedSet raw_added, norm_added;
  int file_max_length = 0;
  bool file_trunc_left = false;
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

// The White_Space property (also the regex \s of both pre-tokenisers).
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
bool is_letter(uint32_t c) { return in_table(uni::kLetter, c); }
bool is_number(uint32_t c) { return in_table(uni::kNumber, c); }
bool is_word_char(uint32_t c) { return in_table(uni::kWord, c); }

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
std::string to_utf8(const std::vector<uint32_t>& cps) {
  std::string s;
  for (uint32_t c : cps) append_utf8(c, s);
  return s;
}

// The GPT-2 / CLIP byte-to-printable-code-point table: bytes 33-126, 161-172
// and 174-255 map to themselves, the other 68 bytes, in ascending order, to
// 256, 257, ...
const std::vector<uint32_t>& byte_symbols() {
  static const std::vector<uint32_t> table = [] {
    std::vector<uint32_t> out(256);
    uint32_t extra = 0;
    for (uint32_t b = 0; b < 256; ++b) {
      const bool direct = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
      out[b] = direct ? b : 256 + extra++;
    }
    return out;
  }();
  return table;
}

// Canonical decomposition (NFD): full decompositions from the table, Hangul
// syllables by the Unicode algorithm, then the canonical ordering of each run
// of combining marks by combining class (stable).
void nfd(const std::vector<uint32_t>& in, std::vector<uint32_t>& out, bool compat = false) {
  out.clear();
  for (uint32_t c : in) {
    const uni::SeqEntry* k = compat ? find_seq(uni::kCompatDecomp, c) : nullptr;
    if (k) {
      out.insert(out.end(), uni::kCompatDecomp_seq + k->off, uni::kCompatDecomp_seq + k->off + k->n);
    } else if (c >= 0xAC00 && c < 0xAC00 + 11172) {
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

// The primary composite of (a, b), 0 if none: Hangul L+V and LV+T by the
// Unicode algorithm, the rest from the table.
uint32_t compose_pair(uint32_t a, uint32_t b) {
  if (a >= 0x1100 && a < 0x1100 + 19 && b >= 0x1161 && b < 0x1161 + 21)
    return 0xAC00 + ((a - 0x1100) * 21 + (b - 0x1161)) * 28;
  if (a >= 0xAC00 && a < 0xAC00 + 11172 && (a - 0xAC00) % 28 == 0 && b > 0x11A7 && b < 0x11A7 + 28)
    return a + (b - 0x11A7);
  const size_t n = sizeof(uni::kCompose) / sizeof(uni::kCompose[0]);
  const uni::ComposeEntry* it = std::lower_bound(
      uni::kCompose, uni::kCompose + n, std::make_pair(a, b),
      [](const uni::ComposeEntry& e, const std::pair<uint32_t, uint32_t>& k) {
        return e.first < k.first || (e.first == k.first && e.second < k.second);
      });
  return (it != uni::kCompose + n && it->first == a && it->second == b) ? it->composite : 0;
}

// NFC: NFD, then the canonical composition algorithm -- each character joins
// the last starter unless a character between them has combining class 0 or
// a class >= its own (blocked).
void nfc(const std::vector<uint32_t>& in, std::vector<uint32_t>& out, bool compat = false) {
  std::vector<uint32_t> d;
  nfd(in, d, compat);
  out.clear();
  long starter = -1;
  for (uint32_t c : d) {
    const uint8_t cc = ccc(c);
    if (starter >= 0) {
      const bool adjacent = static_cast<size_t>(starter) + 1 == out.size();
      const uint8_t last = adjacent ? 0 : ccc(out.back());
      if (adjacent || (last != 0 && last < cc)) {
        if (const uint32_t comp = compose_pair(out[starter], c)) {
          out[starter] = comp;
          continue;
        }
      }
    }
    if (cc == 0) starter = static_cast<long>(out.size());
    out.push_back(c);
  }
}

void lowercase_cps(std::vector<uint32_t>& cps) {
  std::vector<uint32_t> tmp;
  for (uint32_t c : cps) {
    if (const uni::SeqEntry* e = find_seq(uni::kLower, c))
      tmp.insert(tmp.end(), uni::kLower_seq + e->off, uni::kLower_seq + e->off + e->n);
    else
      tmp.push_back(c);
  }
  cps.swap(tmp);
}

template <size_t N>
uint8_t class_of(const uni::ClassRange (&r)[N], uint32_t cp) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (cp < r[mid].lo) hi = mid;
    else if (cp > r[mid].hi) lo = mid + 1;
    else return r[mid].cls;
  }
  return 0;
}

// End of the extended grapheme cluster (UAX #29, GB3-GB13 with GB9c) that
// starts at i.
size_t grapheme_end(const std::vector<uint32_t>& c, size_t i) {
  enum { CR = 1, LF, Control, Extend, ZWJ, RI, Prepend, SpacingMark, L, V, T, LV, LVT };
  const size_t n = c.size();
  uint8_t prev = class_of(uni::kGcb, c[i]);
  int ri = prev == RI;
  bool pict = in_table(uni::kExtPict, c[i]), pict_zwj = false;
  const uint8_t ib0 = class_of(uni::kIncb, c[i]);
  int conj = ib0 == 1 ? 1 : 0;  // 1: consonant [extend|linker]*, 2: ... with a linker
  size_t j = i + 1;
  for (; j < n; ++j) {
    const uint8_t cur = class_of(uni::kGcb, c[j]);
    const uint8_t ib = class_of(uni::kIncb, c[j]);
    const bool ext_pict = in_table(uni::kExtPict, c[j]);
    bool join;
    if (prev == CR && cur == LF) join = true;
    else if (prev == Control || prev == CR || prev == LF) join = false;
    else if (cur == Control || cur == CR || cur == LF) join = false;
    else if (prev == L && (cur == L || cur == V || cur == LV || cur == LVT)) join = true;
    else if ((prev == LV || prev == V) && (cur == V || cur == T)) join = true;
    else if ((prev == LVT || prev == T) && cur == T) join = true;
    else if (cur == Extend || cur == ZWJ || cur == SpacingMark || prev == Prepend) join = true;
    else if (conj == 2 && ib == 1) join = true;
    else if (pict_zwj && ext_pict) join = true;
    else if (prev == RI && cur == RI && ri % 2 == 1) join = true;
    else join = false;
    if (!join) break;
    ri = cur == RI ? ri + 1 : 0;
    if (ext_pict) {
      pict = true;
      pict_zwj = false;
    } else if (cur == Extend && pict) {
      pict_zwj = false;
    } else if (cur == ZWJ && pict) {
      pict = false;
      pict_zwj = true;
    } else {
      pict = pict_zwj = false;
    }
    if (ib == 1) conj = 1;
    else if (ib == 3 && conj) conj = 2;
    else if (ib != 2) conj = 0;
    prev = cur;
  }
  return j;
}

// darts-clone's common-prefix search, shortest key first; the replacement of
// the shortest key that prefixes `key`, if any.
bool charsmap_transform(const CharsMap& m, const std::string& key, std::string& out) {
  const std::vector<uint32_t>& a = m.units;
  auto offset = [](uint32_t u) { return (u >> 10) << ((u & (1u << 9)) >> 6); };
  if (a.empty()) return false;
  size_t node = offset(a[0]);
  for (unsigned char ch : key) {
    if (ch == 0) return false;
    node ^= ch;
    if (node >= a.size()) return false;
    const uint32_t unit = a[node];
    if ((unit & (0x80000000u | 0xFFu)) != ch) return false;
    node ^= offset(unit);
    if ((unit >> 8) & 1u) {
      if (node >= a.size()) return false;
      const size_t idx = a[node] & 0x7FFFFFFFu;
      if (idx > m.normalized.size()) return false;
      const size_t end = m.normalized.find('\0', idx);
      out.assign(m.normalized, idx, (end == std::string::npos ? m.normalized.size() : end) - idx);
      return true;
    }
  }
  return false;
}

// The Precompiled normaliser: per grapheme cluster shorter than 6 bytes the
// map's replacement of the whole cluster, else per character.
void precompiled_normalize(const CharsMap& m, std::vector<uint32_t>& cps) {
  std::string out, unit, rep;
  for (size_t i = 0; i < cps.size();) {
    const size_t e = grapheme_end(cps, i);
    unit.clear();
    for (size_t k = i; k < e; ++k) append_utf8(cps[k], unit);
    if (unit.size() < 6 && charsmap_transform(m, unit, rep)) {
      out += rep;
    } else {
      for (size_t k = i; k < e; ++k) {
        unit.clear();
        append_utf8(cps[k], unit);
        if (charsmap_transform(m, unit, rep)) {
          out += rep;
        } else {
          out += unit;
        }
      }
    }
    i = e;
  }
  cps.clear();
  decode_utf8(out.data(), out.size(), cps);
}

void bert_normalize(const jb_tokenizer& t, std::vector<uint32_t>& cps) {
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
  if (t.lowercase) lowercase_cps(cps);
}

void replace_all(std::vector<uint32_t>& cps, const std::vector<uint32_t>& pat, const std::vector<uint32_t>& with) {
  if (pat.empty() || cps.size() < pat.size()) return;
  std::vector<uint32_t> out;
  size_t i = 0;
  while (i < cps.size()) {
    if (i + pat.size() <= cps.size() && std::equal(pat.begin(), pat.end(), cps.begin() + i)) {
      out.insert(out.end(), with.begin(), with.end());
      i += pat.size();
    } else {
      out.push_back(cps[i++]);
    }
  }
  cps.swap(out);
}

void normalize(const jb_tokenizer& t, std::vector<uint32_t>& cps) {
  std::vector<uint32_t> tmp;
  for (const NormStep& st : t.norm) {
    switch (st.op) {
      case kNormBert: bert_normalize(t, cps); break;
      case kNormPrecompiled: precompiled_normalize(t.charsmap, cps); break;
      case kNormReplaceSpaces2: {  // regex " {2,}" -> content
        tmp.clear();
        for (size_t i = 0; i < cps.size();) {
          size_t j = i;
          while (j < cps.size() && cps[j] == ' ') ++j;
          if (j - i >= 2) {
            tmp.insert(tmp.end(), st.b.begin(), st.b.end());
            i = j;
          } else {
            tmp.push_back(cps[i++]);
          }
        }
        cps.swap(tmp);
        break;
      }
      case kNormNfc: nfc(cps, tmp); cps.swap(tmp); break;
      case kNormNfd: nfd(cps, tmp); cps.swap(tmp); break;
      case kNormNfkc: nfc(cps, tmp, true); cps.swap(tmp); break;
      case kNormNfkd: nfd(cps, tmp, true); cps.swap(tmp); break;
      case kNormLower: lowercase_cps(cps); break;
      case kNormStripAccents:  // every combining mark (category M*), no decomposition first
        tmp.clear();
        for (uint32_t c : cps)
          if (!in_table(uni::kMark, c)) tmp.push_back(c);
        cps.swap(tmp);
        break;
      case kNormStrip: {
        size_t b = 0, e = cps.size();
        if (st.left)
          while (b < e && is_whitespace(cps[b])) ++b;
        if (st.right)
          while (e > b && is_whitespace(cps[e - 1])) --e;
        cps = std::vector<uint32_t>(cps.begin() + b, cps.begin() + e);
        break;
      }
      case kNormPrepend:
        if (!cps.empty()) cps.insert(cps.begin(), st.a.begin(), st.a.end());
        break;
      case kNormReplace: replace_all(cps, st.a, st.b); break;
      case kNormReplaceSpaceRuns: {  // regex \s+ -> content
        tmp.clear();
        for (size_t i = 0; i < cps.size();) {
          if (!is_whitespace(cps[i])) {
            tmp.push_back(cps[i++]);
            continue;
          }
          while (i < cps.size() && is_whitespace(cps[i])) ++i;
          tmp.insert(tmp.end(), st.b.begin(), st.b.end());
        }
        cps.swap(tmp);
        break;
      }
    }
  }
}

// ---- models -----------------------------------------------------------------

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

// Applies the merges to a word's symbols, lowest rank first and leftmost on
// ties, in O(n log n): the symbols form a linked list and the candidate pairs
// sit in a min-heap keyed (rank, position); a popped pair that no longer
// exists (a side was merged away or changed) is skipped.
void merge_symbols(const jb_tokenizer& t, std::vector<uint32_t>& sym) {
  const int n = static_cast<int>(sym.size());
  if (n < 2) return;
  std::vector<int> prev(n), next(n);
  std::vector<char> live(n, 1);
  for (int i = 0; i < n; ++i) {
    prev[i] = i - 1;
    next[i] = i + 1 < n ? i + 1 : -1;
  }
  struct Cand {
    uint32_t rank;
    int pos;
    uint32_t id;
    bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : pos > o.pos; }
  };
  std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
  auto lookup = [&](int a) {
    const int b = next[a];
    if (b < 0) return;
    auto it = t.merges.find((static_cast<uint64_t>(sym[a]) << 32) | sym[b]);
    if (it != t.merges.end()) heap.push({it->second.first, a, it->second.second});
  };
  for (int i = 0; i + 1 < n; ++i) lookup(i);
  while (!heap.empty()) {
    const Cand c = heap.top();
    heap.pop();
    const int a = c.pos;
    if (!live[a] || next[a] < 0) continue;
    const int b = next[a];
    auto it = t.merges.find((static_cast<uint64_t>(sym[a]) << 32) | sym[b]);
    if (it == t.merges.end() || it->second.second != c.id || it->second.first != c.rank) continue;
    sym[a] = c.id;
    live[b] = 0;
    next[a] = next[b];
    if (next[b] >= 0) prev[next[b]] = a;
    if (prev[a] >= 0) lookup(prev[a]);
    lookup(a);
  }
  std::vector<uint32_t> out;
  for (int i = 0; i >= 0; i = next[i]) out.push_back(sym[i]);
  sym.swap(out);
}

void bpe(const jb_tokenizer& t, const std::vector<uint32_t>& word, std::vector<uint32_t>& ids) {
  if (word.empty()) return;
  if (t.ignore_merges) {
    auto it = t.vocab.find(to_utf8(word));
    if (it != t.vocab.end()) {
      ids.push_back(it->second);
      return;
    }
  }
  std::vector<uint32_t> sym;
  bool unk_pending = false;
  std::string s;
  for (size_t k = 0; k < word.size(); ++k) {
    s.clear();
    if (k > 0) s = t.bpe_prefix;
    append_utf8(word[k], s);
    if (k + 1 == word.size()) s += t.bpe_suffix;
    auto it = t.vocab.find(s);
    if (it != t.vocab.end()) {
      if (unk_pending) sym.push_back(t.unk_id);
      unk_pending = false;
      sym.push_back(it->second);
      continue;
    }
    if (t.byte_fallback) {
      std::vector<uint32_t> bytes;
      char code[8];
      for (unsigned char b : s) {
        std::snprintf(code, sizeof(code), "<0x%02X>", b);
        auto bt = t.vocab.find(code);
        if (bt == t.vocab.end()) break;
        bytes.push_back(bt->second);
      }
      if (bytes.size() == s.size()) {  // a pending unknown token stays pending
        sym.insert(sym.end(), bytes.begin(), bytes.end());
        continue;
      }
    }
    if (t.has_unk) {
      if (unk_pending && !t.fuse_unk) sym.push_back(t.unk_id);
      unk_pending = true;
    }
    // no unknown token: the character is dropped
  }
  if (unk_pending) sym.push_back(t.unk_id);
  merge_symbols(t, sym);
  ids.insert(ids.end(), sym.begin(), sym.end());
}

// Unigram: the best segmentation by Viterbi over byte positions (the
// crate's encode_optimized): every vocabulary piece that prefixes the rest
// of the word from each character boundary, score added to the best path
// there, the first path found kept on ties; a character with no piece of
// its own length gets the unknown token at (lowest score - 10); consecutive
// unknown pieces fuse into one.  Pieces map to ids, the fused unknown runs
// to <0xXX> byte tokens (byte_fallback) or the unknown id.
void unigram(const jb_tokenizer& t, const std::vector<uint32_t>& word, std::vector<uint32_t>& ids) {
  if (word.empty()) return;
  const std::string s = to_utf8(word);
  const size_t n = s.size();
  struct Node {
    double score = 0.0;
    long start = -1;
    int32_t id = 0;
  };
  std::vector<Node> best(n + 1);
  best[0].start = 0;
  const double unk_score = t.min_score - 10.0;
  const auto& edges = t.trie.edges;
  for (size_t at = 0; at < n;) {
    size_t mblen = 1;
    while (at + mblen < n && (static_cast<unsigned char>(s[at + mblen]) & 0xC0) == 0x80) ++mblen;
    const double base = best[at].score;
    bool single = false;
    uint32_t node = 0;
    for (size_t k = at; k < n; ++k) {
      const uint64_t key = (static_cast<uint64_t>(node) << 8) | static_cast<unsigned char>(s[k]);
      auto it = std::lower_bound(edges.begin(), edges.end(), std::make_pair(key, 0u),
                                 [](const std::pair<uint64_t, uint32_t>& a, const std::pair<uint64_t, uint32_t>& b) {
                                   return a.first < b.first;
                                 });
      if (it == edges.end() || it->first != key) break;
      node = it->second;
      const int32_t id = t.trie.piece[node];
      if (id < 0) continue;
      const size_t end = k + 1;
      const double cand = base + t.scores[id];
      if (best[end].start < 0 || cand > best[end].score) best[end] = {cand, static_cast<long>(at), id};
      if (end - at == mblen) single = true;
    }
    if (!single) {
      if (!t.has_unk) fail(JB_ERR_INVALID, "Unigram: a character has no piece and there is no unknown token");
      const double cand = base + unk_score;
      Node& tgt = best[at + mblen];
      if (tgt.start < 0 || cand > tgt.score) tgt = {cand, static_cast<long>(at), static_cast<int32_t>(t.unk_id)};
    }
    at += mblen;
  }
  std::vector<std::pair<size_t, size_t>> pieces;  // byte ranges, reversed
  size_t end = n, unk_end = 0;
  bool in_unk = false;
  while (end > 0) {
    const Node& nd = best[end];
    const size_t start = static_cast<size_t>(nd.start);
    if (t.has_unk && static_cast<uint32_t>(nd.id) == t.unk_id) {
      if (!in_unk) unk_end = end;
      in_unk = true;
    } else {
      if (in_unk) pieces.emplace_back(end, unk_end);
      in_unk = false;
      pieces.emplace_back(start, end);
    }
    end = start;
  }
  if (in_unk) pieces.emplace_back(0, unk_end);
  for (size_t k = pieces.size(); k-- > 0;) {
    const std::string piece = s.substr(pieces[k].first, pieces[k].second - pieces[k].first);
    auto it = t.vocab.find(piece);
    if (it != t.vocab.end()) {
      ids.push_back(it->second);
      continue;
    }
    if (t.byte_fallback) {
      std::vector<uint32_t> bytes;
      char code[8];
      for (unsigned char b : piece) {
        std::snprintf(code, sizeof(code), "<0x%02X>", b);
        auto bt = t.vocab.find(code);
        if (bt == t.vocab.end()) break;
        bytes.push_back(bt->second);
      }
      if (bytes.size() == piece.size()) {
        ids.insert(ids.end(), bytes.begin(), bytes.end());
        continue;
      }
    }
    if (!t.has_unk) fail(JB_ERR_INVALID, "Unigram: no unknown token");
    ids.push_back(t.unk_id);
  }
}

void model(const jb_tokenizer& t, const std::vector<uint32_t>& word, std::vector<uint32_t>& ids) {
  if (t.model == kWordPiece) return wordpiece(t, word, ids);
  if (t.model == kUnigram) return unigram(t, word, ids);
  if (t.model == kBpe) return bpe(t, word, ids);
  if (word.empty()) return;  // WordLevel: the word itself, else the unknown token
  auto it = t.vocab.find(to_utf8(word));
  if (it != t.vocab.end()) {
    ids.push_back(it->second);
  } else {
    if (!t.has_unk) fail(JB_ERR_INVALID, "WordLevel: a word is not in the vocabulary and there is no unknown token");
    ids.push_back(t.unk_id);
  }
}

// ---- pre-tokenisers ---------------------------------------------------------

// Length (in code points) of OpenCLIP's regex match at position i, 0 if no
// alternative matches there (whitespace); alternatives are tried in the
// regex's order, the first that matches wins.
size_t clip_match(const std::vector<uint32_t>& c, size_t i, bool specials = true) {
  static const char* const kLiterals[] = {"<|startoftext|>", "<|endoftext|>", "'s", "'t", "'re",
                                          "'ve", "'m", "'ll", "'d"};
  for (const char* lit : kLiterals) {
    if (!specials && lit[0] == '<') continue;
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

// Length of the GPT-2 regex's match at position i:
// 's|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+
size_t gpt2_match(const std::vector<uint32_t>& c, size_t i) {
  const size_t n = c.size();
  if (c[i] == '\'' && i + 1 < n) {
    const uint32_t a = c[i + 1], b = i + 2 < n ? c[i + 2] : 0;
    if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
    if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
  }
  const size_t j0 = i + (c[i] == ' ' ? 1 : 0);
  if (j0 < n) {
    size_t j = j0;
    if (is_letter(c[j])) {
      while (j < n && is_letter(c[j])) ++j;
      return j - i;
    }
    if (is_number(c[j])) {
      while (j < n && is_number(c[j])) ++j;
      return j - i;
    }
    auto other = [](uint32_t x) { return !is_whitespace(x) && !is_letter(x) && !is_number(x); };
    if (other(c[j])) {
      while (j < n && other(c[j])) ++j;
      return j - i;
    }
  }
  // c[i] is whitespace here
  size_t j = i;
  while (j < n && is_whitespace(c[j])) ++j;
  if (j == n || j - i == 1) return j - i;
  return j - 1 - i;  // the last space goes to the next word
}

// Words of one piece, each with whether it starts at the text's offset 0
// (Metaspace's "first" prepend scheme asks).
struct Words {
  std::vector<std::vector<uint32_t>> w;
  std::vector<char> at0;
  void add(const std::vector<uint32_t>& src, size_t b, size_t e, bool parent_at0) {
    w.emplace_back(src.begin() + b, src.begin() + e);
    at0.push_back(parent_at0 && b == 0);
  }
  void add(std::vector<uint32_t>&& v, bool flag) {
    w.push_back(std::move(v));
    at0.push_back(flag);
  }
};

// The crate's split of one word: a list of (segment, is-match) covering it,
// then `behavior` keeps, drops or merges the matches; empty pieces vanish.
struct Seg {
  size_t b, e;
  bool m;
};

void emit(const std::vector<uint32_t>& w, bool at0, const std::vector<Seg>& segs, int behavior, Words& out) {
  std::vector<Seg> merged;
  bool prev = false;
  switch (behavior) {
    case kIsolated:
    case kRemoved:
      merged = segs;
      break;
    case kContiguous:
      for (const Seg& g : segs) {
        if (!merged.empty() && g.m == prev) merged.back().e = g.e;
        else merged.push_back({g.b, g.e, false});
        prev = g.m;
      }
      break;
    case kMergedWithPrevious:
      for (const Seg& g : segs) {
        if (g.m && !prev && !merged.empty()) merged.back().e = g.e;
        else merged.push_back({g.b, g.e, false});
        prev = g.m;
      }
      break;
    case kMergedWithNext:
      for (size_t k = segs.size(); k-- > 0;) {
        const Seg& g = segs[k];
        if (g.m && !prev && !merged.empty()) merged.back().b = g.b;
        else merged.push_back({g.b, g.e, false});
        prev = g.m;
      }
      std::reverse(merged.begin(), merged.end());
      break;
  }
  for (const Seg& g : merged)
    if (g.e > g.b && !(behavior == kRemoved && g.m)) out.add(w, g.b, g.e, at0);
}

// Each character that satisfies the predicate is a match of its own.
template <typename Pred>
std::vector<Seg> char_segments(const std::vector<uint32_t>& w, Pred is_delim) {
  std::vector<Seg> segs;
  size_t run = 0;
  for (size_t i = 0; i < w.size(); ++i)
    if (is_delim(w[i])) {
      if (run < i) segs.push_back({run, i, false});
      segs.push_back({i, i + 1, true});
      run = i + 1;
    }
  if (run < w.size()) segs.push_back({run, w.size(), false});
  return segs;
}

template <typename Pred>
void split_chars(const std::vector<uint32_t>& w, bool at0, Pred is_delim, int behavior, Words& out) {
  emit(w, at0, char_segments(w, is_delim), behavior, out);
}

// Length of the pattern's match starting at i (0: none there).
size_t pattern_match(const PreStep& st, const std::vector<uint32_t>& c, size_t i) {
  switch (st.pattern) {
    case kPatClip: return clip_match(c, i, false);
    case kPatClipSpecials: return clip_match(c, i, true);
    case kPatGpt2: return gpt2_match(c, i);
    case kPatSpaceRuns: {
      size_t j = i;
      while (j < c.size() && is_whitespace(c[j])) ++j;
      return j - i;
    }
    default: {
      const std::vector<uint32_t>& lit = st.literal;
      return (i + lit.size() <= c.size() && std::equal(lit.begin(), lit.end(), c.begin() + i)) ? lit.size() : 0;
    }
  }
}

// A regex scan's matches in order with the gaps between them; the empty
// pattern matches the empty string at every boundary, end included.
std::vector<Seg> pattern_segments(const PreStep& st, const std::vector<uint32_t>& w) {
  std::vector<Seg> segs;
  if (w.empty()) return segs;
  size_t prev = 0;
  auto add_match = [&](size_t b, size_t e) {
    if (prev != b) segs.push_back({prev, b, false});
    segs.push_back({b, e, true});
    prev = e;
  };
  if (st.pattern == kPatLiteral && st.literal.empty()) {
    for (size_t b = 0; b <= w.size(); ++b) add_match(b, b);
  } else {
    for (size_t i = 0; i < w.size();) {
      const size_t len = pattern_match(st, w, i);
      if (len == 0) {
        ++i;
        continue;
      }
      add_match(i, i + len);
      i += len;
    }
  }
  if (prev != w.size()) segs.push_back({prev, w.size(), false});
  if (st.invert)
    for (Seg& g : segs) g.m = !g.m;
  return segs;
}

void pre_step(const PreStep& st, const std::vector<uint32_t>& w, bool at0, Words& out) {
  switch (st.kind) {
    case kPreBert: {  // split on White_Space (removed), each punctuation character isolated
      Words parts;
      split_chars(w, at0, is_whitespace, kRemoved, parts);
      for (size_t k = 0; k < parts.w.size(); ++k) split_chars(parts.w[k], parts.at0[k], is_punct, kIsolated, out);
      return;
    }
    case kPreWhitespaceSplit:
      split_chars(w, at0, is_whitespace, kRemoved, out);
      return;
    case kPrePunctuation:
      split_chars(w, at0, is_punct, st.behavior, out);
      return;
    case kPreDigits:
      split_chars(w, at0, is_number, st.individual_digits ? kIsolated : kContiguous, out);
      return;
    case kPreSplit:
      emit(w, at0, pattern_segments(st, w), st.behavior, out);
      return;
    case kPreMetaspace: {  // ' ' -> replacement, the prepend scheme, then split before each replacement
      std::vector<uint32_t> c = w;
      for (uint32_t& x : c)
        if (x == ' ') x = st.replacement;
      const bool prepend = st.prepend_scheme == kPrependAlways || (st.prepend_scheme == kPrependFirst && at0);
      if (prepend && (c.empty() || c[0] != st.replacement)) c.insert(c.begin(), st.replacement);
      if (!st.split) {
        out.add(std::move(c), at0);
        return;
      }
      const uint32_t r = st.replacement;
      split_chars(c, at0, [r](uint32_t x) { return x == r; }, kMergedWithNext, out);
      return;
    }
    case kPreWhitespace: {  // the matches of \w+|[^\w\s]+; the rest dropped
      auto word = [](uint32_t c) { return is_word_char(c); };
      for (size_t i = 0; i < w.size();) {
        if (is_whitespace(w[i])) {
          ++i;
          continue;
        }
        const bool wd = word(w[i]);
        size_t j = i + 1;
        while (j < w.size() && !is_whitespace(w[j]) && word(w[j]) == wd) ++j;
        out.add(w, i, j, at0);
        i = j;
      }
      return;
    }
    case kPreClip: {
      size_t seg = 0;
      for (size_t i = 0; i < w.size();) {
        const size_t len = clip_match(w, i);
        if (len == 0) {
          ++i;
          continue;
        }
        if (seg < i) out.add(w, seg, i, at0);
        out.add(w, i, i + len, at0);
        i += len;
        seg = i;
      }
      if (seg < w.size()) out.add(w, seg, w.size(), at0);
      return;
    }
    case kPreByteLevel: {
      std::vector<uint32_t> c = w;
      if (st.add_prefix_space && !c.empty() && c[0] != ' ') c.insert(c.begin(), ' ');
      const std::vector<uint32_t>& bs = byte_symbols();
      std::string utf8;
      for (size_t i = 0; i < c.size();) {
        const size_t len = st.use_regex ? gpt2_match(c, i) : c.size();
        utf8.clear();
        for (size_t k = i; k < i + len; ++k) append_utf8(c[k], utf8);
        std::vector<uint32_t> sym;
        for (unsigned char b : utf8) sym.push_back(bs[b]);
        out.add(std::move(sym), at0 && i == 0);
        i += len;
      }
      return;
    }
  }
}

void pre_tokenize_and_model(const jb_tokenizer& t, const std::string& piece, bool at0, std::vector<uint32_t>& ids) {
  Words words;
  std::vector<uint32_t> c;
  decode_utf8(piece.data(), piece.size(), c);
  if (c.empty()) return;
  words.add(std::move(c), at0);
  for (const PreStep& st : t.pre) {
    Words next;
    for (size_t k = 0; k < words.w.size(); ++k) pre_step(st, words.w[k], words.at0[k], next);
    words = std::move(next);
  }
  for (const auto& w : words.w) model(t, w, ids);
}

// ---- added tokens -----------------------------------------------------------

struct Piece {
  size_t begin, end;
  long id;  // -1: text
};

size_t prev_char_start(const std::string& s, size_t i) {  // i > 0
  do --i;
  while (i > 0 && (static_cast<unsigned char>(s[i]) & 0xC0) == 0x80);
  return i;
}
uint32_t char_at(const std::string& s, size_t i, size_t* len) {
  size_t n = 1;
  while (i + n < s.size() && n < 4 && (static_cast<unsigned char>(s[i + n]) & 0xC0) == 0x80) ++n;
  std::vector<uint32_t> c;
  decode_utf8(s.data() + i, n, c);
  if (len) *len = n;
  return c.empty() ? 0 : c[0];
}

// Splits s on the added tokens: leftmost-longest matches in one pass, as the
// crate's Aho-Corasick scan does (a match dropped by single_word still ends
// the scan step), lstrip back to the previous piece, rstrip forward.
std::vector<Piece> split_added(const std::string& s, const AddedSet& added) {
  std::vector<Piece> out;
  size_t start_offset = 0;
  for (size_t i = 0; i < s.size() && !added.toks.empty();) {
    const AddedToken* best = nullptr;
    for (uint32_t k : added.by_first[static_cast<unsigned char>(s[i])]) {
      const AddedToken& a = added.toks[k];
      if (a.content.size() <= s.size() - i && std::memcmp(s.data() + i, a.content.data(), a.content.size()) == 0) {
        best = &a;
        break;
      }
    }
    if (!best) {
      ++i;
      continue;
    }
    size_t start = i, stop = i + best->content.size();
    i = stop;
    if (best->single_word) {
      const bool word_before = start > 0 && is_word_char(char_at(s, prev_char_start(s, start), nullptr));
      const bool word_after = stop < s.size() && is_word_char(char_at(s, stop, nullptr));
      if (word_before || word_after) continue;
    }
    if (best->lstrip) {
      size_t ns = start;
      while (ns > 0) {
        const size_t p = prev_char_start(s, ns);
        if (!is_whitespace(char_at(s, p, nullptr))) break;
        ns = p;
      }
      start = std::max(ns, start_offset);
    }
    if (best->rstrip) {
      size_t len = 0;
      while (stop < s.size() && is_whitespace(char_at(s, stop, &len))) stop += len;
      i = std::max(i, stop);
    }
    if (start_offset < start) out.push_back({start_offset, start, -1});
    out.push_back({start, stop, static_cast<long>(best->id)});
    start_offset = stop;
  }
  if (start_offset < s.size()) out.push_back({start_offset, s.size(), -1});
  return out;
}

void encode(const jb_tokenizer& t, const char* s, size_t n, int max_length, std::vector<uint32_t>& out) {
  std::vector<uint32_t> ids;
  const std::string text(s, n);
  std::vector<uint32_t> cps;
  for (const Piece& p : split_added(text, t.raw_added)) {
    if (p.id >= 0) {
      ids.push_back(static_cast<uint32_t>(p.id));
      continue;
    }
    cps.clear();
    decode_utf8(text.data() + p.begin, p.end - p.begin, cps);
    normalize(t, cps);
    const std::string normed = to_utf8(cps);
    for (const Piece& q : split_added(normed, t.norm_added)) {
      if (q.id >= 0)
        ids.push_back(static_cast<uint32_t>(q.id));
      else  // a piece at the text's start stays there whatever the normaliser deleted
        pre_tokenize_and_model(t, normed.substr(q.begin, q.end - q.begin), p.begin == 0 && q.begin == 0, ids);
    }
  }
  const size_t specials = t.before.size() + t.after.size();
  const int limit = max_length > 0 ? max_length : t.file_max_length;
  if (limit > 0) {
    const size_t keep = static_cast<size_t>(limit) > specials ? limit - specials : 0;
    if (ids.size() > keep) {
      if (max_length <= 0 && t.file_trunc_left)
        ids.erase(ids.begin(), ids.end() - keep);
      else
        ids.resize(keep);
    }
  }
  out.clear();
  out.insert(out.end(), t.before.begin(), t.before.end());
  out.insert(out.end(), ids.begin(), ids.end());
  out.insert(out.end(), t.after.begin(), t.after.end());
}

// ---- loading ----------------------------------------------------------------

uint32_t token_id(const jb_tokenizer& t, const std::string& tok) {
  auto it = t.vocab.find(tok);
  if (it == t.vocab.end()) fail(JB_ERR_IO, "tokenizer.json: token " + tok + " is not in the vocabulary");
  return it->second;
}

void add_merge(jb_tokenizer& t, size_t rank, const std::string& a, const std::string& b) {
  const std::string joined = a + b.substr(std::min(t.bpe_prefix.size(), b.size()));
  auto ia = t.vocab.find(a), ib = t.vocab.find(b), iab = t.vocab.find(joined);
  if (ia == t.vocab.end() || ib == t.vocab.end() || iab == t.vocab.end())
    fail(JB_ERR_IO, "BPE merge " + std::to_string(rank + 1) + " (" + a + " " + b +
                        ") names a symbol not in the vocabulary");
  t.merges[(static_cast<uint64_t>(ia->second) << 32) | ib->second] = {static_cast<uint32_t>(rank),
                                                                        iab->second};
}

std::string base64_decode(const std::string& in) {
  auto val = [](char c) -> int {
    if (c >= 'A' && c <= 'Z') return c - 'A';
    if (c >= 'a' && c <= 'z') return c - 'a' + 26;
    if (c >= '0' && c <= '9') return c - '0' + 52;
    if (c == '+' || c == '-') return 62;
    if (c == '/' || c == '_') return 63;
    return -1;
  };
  std::string out;
  uint32_t acc = 0;
  int bits = 0;
  for (char c : in) {
    const int v = val(c);
    if (v < 0) continue;  // padding, whitespace
    acc = (acc << 6) | static_cast<uint32_t>(v);
    bits += 6;
    if (bits >= 8) {
      bits -= 8;
      out.push_back(static_cast<char>((acc >> bits) & 0xFF));
    }
  }
  return out;
}

// The charsmap blob: u32 little-endian trie size in bytes, the double array,
// then the NUL-separated replacement strings.
CharsMap parse_charsmap(const std::string& b64) {
  const std::string raw = base64_decode(b64);
  if (raw.size() < 4) fail(JB_ERR_IO, "tokenizer.json: Precompiled charsmap too short");
  uint32_t trie_bytes = 0;
  std::memcpy(&trie_bytes, raw.data(), 4);
  if (trie_bytes % 4 || 4 + static_cast<size_t>(trie_bytes) > raw.size())
    fail(JB_ERR_IO, "tokenizer.json: Precompiled charsmap is malformed");
  CharsMap m;
  m.units.resize(trie_bytes / 4);
  std::memcpy(m.units.data(), raw.data() + 4, trie_bytes);
  m.normalized = raw.substr(4 + trie_bytes);
  return m;
}

std::vector<uint32_t> cps_of(const std::string& u) {
  std::vector<uint32_t> c;
  decode_utf8(u.data(), u.size(), c);
  return c;
}

void parse_normalizer(jb_tokenizer& t, const Json& nz) {
  const std::string type = nz.str_or("type", "");
  NormStep st;
  if (type == "Sequence") {
    if (const Json* seq = nz.get("normalizers"); seq && seq->kind == Json::Arr)
      for (const Json& x : seq->arr) parse_normalizer(t, x);
    return;
  } else if (type == "BertNormalizer") {
    t.clean_text = nz.bool_or("clean_text", true);
    t.handle_chinese = nz.bool_or("handle_chinese_chars", true);
    t.lowercase = nz.bool_or("lowercase", true);
    const Json* sa = nz.get("strip_accents");
    t.strip_accents = (sa && sa->kind == Json::Bool) ? sa->b : t.lowercase;
    st.op = kNormBert;
  } else if (type == "NFC") {
    st.op = kNormNfc;
  } else if (type == "NFD") {
    st.op = kNormNfd;
  } else if (type == "NFKC") {
    st.op = kNormNfkc;
  } else if (type == "NFKD") {
    st.op = kNormNfkd;
  } else if (type == "Lowercase") {
    st.op = kNormLower;
  } else if (type == "StripAccents") {
    st.op = kNormStripAccents;
  } else if (type == "Precompiled") {
    st.op = kNormPrecompiled;
    t.charsmap = parse_charsmap(nz.str_or("precompiled_charsmap", ""));
  } else if (type == "Strip") {
    st.op = kNormStrip;
    st.left = nz.bool_or("strip_left", true);
    st.right = nz.bool_or("strip_right", true);
  } else if (type == "Prepend") {
    st.op = kNormPrepend;
    st.a = cps_of(nz.str_or("prepend", ""));
  } else if (type == "Replace") {
    const Json* pat = nz.get("pattern");
    const Json* lit = pat ? pat->get("String") : nullptr;
    const Json* re = pat ? pat->get("Regex") : nullptr;
    st.b = cps_of(nz.str_or("content", ""));
    if (lit && lit->kind == Json::Str) {
      st.op = kNormReplace;
      st.a = cps_of(lit->str);
    } else if (re && re->kind == Json::Str && re->str == "\\s+") {
      st.op = kNormReplaceSpaceRuns;
    } else if (re && re->kind == Json::Str && re->str == " {2,}") {
      st.op = kNormReplaceSpaces2;
    } else {
      fail(JB_ERR_INVALID, "tokenizer.json: Replace supports string patterns and the regexes \\s+ and ' {2,}'");
    }
  } else {
    fail(JB_ERR_INVALID, "tokenizer.json: unsupported normalizer " + type);
  }
  t.norm.push_back(st);
}

int behavior_of(const std::string& b) {
  if (b == "Isolated") return kIsolated;
  if (b == "Removed") return kRemoved;
  if (b == "MergedWithPrevious") return kMergedWithPrevious;
  if (b == "MergedWithNext") return kMergedWithNext;
  if (b == "Contiguous") return kContiguous;
  fail(JB_ERR_INVALID, "tokenizer.json: unknown split behavior " + b);
}

// The regular expressions this library matches by hand; any other is refused.
int known_regex(const std::string& re) {
  static const std::string kClip = "'s|'t|'re|'ve|'m|'ll|'d|[\\p{L}]+|[\\p{N}]|[^\\s\\p{L}\\p{N}]+";
  static const std::string kClipSpecials = "<\\|startoftext\\|>|<\\|endoftext\\|>|" + kClip;
  static const std::string kGpt2 =
      "'s|'t|'re|'ve|'m|'ll|'d| ?\\p{L}+| ?\\p{N}+| ?[^\\s\\p{L}\\p{N}]+|\\s+(?!\\S)|\\s+";
  if (re == kClip) return kPatClip;
  if (re == kClipSpecials) return kPatClipSpecials;
  if (re == kGpt2) return kPatGpt2;
  if (re == "\\s+") return kPatSpaceRuns;
  fail(JB_ERR_INVALID, "tokenizer.json: unsupported regex pattern " + re);
}

void parse_pre_tokenizer(jb_tokenizer& t, const Json& pt) {
  const std::string type = pt.str_or("type", "");
  PreStep st;
  if (type == "Sequence") {
    if (const Json* seq = pt.get("pretokenizers"); seq && seq->kind == Json::Arr)
      for (const Json& x : seq->arr) parse_pre_tokenizer(t, x);
    return;
  } else if (type == "BertPreTokenizer") {
    st.kind = kPreBert;
  } else if (type == "ByteLevel") {
    st.kind = kPreByteLevel;
    st.add_prefix_space = pt.bool_or("add_prefix_space", true);
    st.use_regex = pt.bool_or("use_regex", true);
  } else if (type == "Whitespace") {
    st.kind = kPreWhitespace;
  } else if (type == "WhitespaceSplit") {
    st.kind = kPreWhitespaceSplit;
  } else if (type == "Punctuation") {
    st.kind = kPrePunctuation;
    st.behavior = behavior_of(pt.str_or("behavior", "Isolated"));
  } else if (type == "Split") {
    st.kind = kPreSplit;
    st.behavior = behavior_of(pt.str_or("behavior", "Isolated"));
    st.invert = pt.bool_or("invert", false);
    const Json* pat = pt.get("pattern");
    const Json* lit = pat ? pat->get("String") : nullptr;
    const Json* re = pat ? pat->get("Regex") : nullptr;
    if (lit && lit->kind == Json::Str) {
      st.pattern = kPatLiteral;
      st.literal = cps_of(lit->str);
    } else if (re && re->kind == Json::Str) {
      st.pattern = known_regex(re->str);
    } else {
      fail(JB_ERR_INVALID, "tokenizer.json: Split without a pattern");
    }
  } else if (type == "Metaspace") {
    st.kind = kPreMetaspace;
    const std::vector<uint32_t> rep = cps_of(pt.str_or("replacement", "\xE2\x96\x81"));
    if (rep.size() != 1) fail(JB_ERR_INVALID, "tokenizer.json: Metaspace replacement must be one character");
    st.replacement = rep[0];
    const std::string scheme = pt.str_or("prepend_scheme", "");
    if (scheme == "always") st.prepend_scheme = kPrependAlways;
    else if (scheme == "first") st.prepend_scheme = kPrependFirst;
    else if (scheme == "never") st.prepend_scheme = kPrependNever;
    else if (scheme.empty()) st.prepend_scheme = pt.bool_or("add_prefix_space", true) ? kPrependAlways : kPrependNever;
    else fail(JB_ERR_INVALID, "tokenizer.json: unknown Metaspace prepend_scheme " + scheme);
    st.split = pt.bool_or("split", true);
  } else if (type == "Digits") {
    st.kind = kPreDigits;
    st.individual_digits = pt.bool_or("individual_digits", false);
  } else {
    fail(JB_ERR_INVALID, "tokenizer.json: unsupported pre-tokenizer " + type);
  }
  t.pre.push_back(st);
}

uint32_t id_of_pair(const Json* p, const char* what) {
  if (!p || p->kind != Json::Arr || p->arr.size() < 2)
    fail(JB_ERR_IO, std::string("tokenizer.json: post-processor needs ") + what);
  return static_cast<uint32_t>(p->arr[1].num);
}

// One post-processor's special ids around the sequence; a Sequence applies
// its processors in order, each wrapping the previous result.
void parse_post(const jb_tokenizer& t, const Json& pp, std::vector<uint32_t>& before,
                std::vector<uint32_t>& after) {
  const std::string type = pp.str_or("type", "");
  std::vector<uint32_t> b, a;
  if (type == "BertProcessing" || type == "RobertaProcessing") {
    b.push_back(id_of_pair(pp.get("cls"), "cls"));
    a.push_back(id_of_pair(pp.get("sep"), "sep"));
  } else if (type == "TemplateProcessing") {
    const Json* single = pp.get("single");
    const Json* specials = pp.get("special_tokens");
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
        v.push_back(token_id(t, name));
      auto& dst = seen_seq ? a : b;
      dst.insert(dst.end(), v.begin(), v.end());
    }
  } else if (type == "ByteLevel") {
    // offsets only
  } else if (type == "Sequence") {
    if (const Json* seq = pp.get("processors"); seq && seq->kind == Json::Arr)
      for (const Json& x : seq->arr) parse_post(t, x, before, after);
    return;
  } else {
    fail(JB_ERR_INVALID, "tokenizer.json: unsupported post-processor " + type);
  }
  before.insert(before.begin(), b.begin(), b.end());
  after.insert(after.end(), a.begin(), a.end());
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
  const std::string type = model ? model->str_or("type", "") : "";
  if (type != "WordPiece" && type != "BPE" && type != "WordLevel" && type != "Unigram")
    fail(JB_ERR_INVALID, "tokenizer.json: unsupported model '" + type + "' (WordPiece, BPE, WordLevel and Unigram are supported)");
  t->model = type == "WordPiece" ? kWordPiece : type == "BPE" ? kBpe : type == "WordLevel" ? kWordLevel : kUnigram;
  const Json* vocab = model->get("vocab");
  if (t->model == kUnigram) {  // [[piece, score], ...]; ids are positions
    if (!vocab || vocab->kind != Json::Arr) fail(JB_ERR_IO, "tokenizer.json: Unigram vocab missing");
    std::unordered_map<uint64_t, uint32_t> edges;
    t->trie.piece.assign(1, -1);
    t->min_score = vocab->arr.empty() ? 0.0 : 1e300;
    for (size_t id = 0; id < vocab->arr.size(); ++id) {
      const Json& e = vocab->arr[id];
      if (e.kind != Json::Arr || e.arr.size() < 2 || e.arr[0].kind != Json::Str)
        fail(JB_ERR_IO, "tokenizer.json: bad Unigram vocabulary entry");
      const std::string& piece = e.arr[0].str;
      t->vocab[piece] = static_cast<uint32_t>(id);
      t->scores.push_back(e.arr[1].num);
      t->min_score = std::min(t->min_score, e.arr[1].num);
      uint32_t node = 0;
      for (unsigned char ch : piece) {
        const uint64_t key = (static_cast<uint64_t>(node) << 8) | ch;
        auto it = edges.find(key);
        if (it == edges.end()) {
          const uint32_t child = static_cast<uint32_t>(t->trie.piece.size());
          t->trie.piece.push_back(-1);
          it = edges.emplace(key, child).first;
        }
        node = it->second;
      }
      if (node) t->trie.piece[node] = static_cast<int32_t>(id);
    }
    t->trie.edges.assign(edges.begin(), edges.end());
    std::sort(t->trie.edges.begin(), t->trie.edges.end());
    if (const Json* u = model->get("unk_id"); u && u->kind == Json::Num) {
      if (u->num < 0 || u->num >= static_cast<double>(vocab->arr.size()))
        fail(JB_ERR_IO, "tokenizer.json: Unigram unk_id out of range");
      t->unk_id = static_cast<uint32_t>(u->num);
      t->has_unk = true;
    }
    t->byte_fallback = model->bool_or("byte_fallback", false);
  } else {
    if (!vocab || vocab->kind != Json::Obj) fail(JB_ERR_IO, "tokenizer.json: model.vocab missing");
    for (const auto& kv : vocab->obj) t->vocab[kv.first] = static_cast<uint32_t>(kv.second.num);
  }
  if (t->model == kUnigram) {
    // parsed above
  } else if (t->model == kWordLevel) {
    if (const Json* unk = model->get("unk_token"); unk && unk->kind == Json::Str) {
      auto it = t->vocab.find(unk->str);
      t->has_unk = it != t->vocab.end();
      if (t->has_unk) t->unk_id = it->second;
    }
  } else if (t->model == kWordPiece) {
    t->prefix = model->str_or("continuing_subword_prefix", "##");
    t->max_chars = static_cast<int>(model->num_or("max_input_chars_per_word", 100));
    t->unk_id = token_id(*t, model->str_or("unk_token", "[UNK]"));
    t->has_unk = true;
  } else {
    if (const Json* d = model->get("dropout"); d && d->kind == Json::Num && d->num > 0)
      fail(JB_ERR_INVALID, "tokenizer.json: BPE dropout is not supported");
    if (const Json* unk = model->get("unk_token"); unk && unk->kind == Json::Str) {
      t->unk_id = token_id(*t, unk->str);
      t->has_unk = true;
    }
    if (const Json* p = model->get("continuing_subword_prefix"); p && p->kind == Json::Str) t->bpe_prefix = p->str;
    if (const Json* p = model->get("end_of_word_suffix"); p && p->kind == Json::Str) t->bpe_suffix = p->str;
    t->fuse_unk = model->bool_or("fuse_unk", false);
    t->byte_fallback = model->bool_or("byte_fallback", false);
    t->ignore_merges = model->bool_or("ignore_merges", false);
    const Json* merges = model->get("merges");
    if (!merges || merges->kind != Json::Arr) fail(JB_ERR_IO, "tokenizer.json: model.merges missing");
    for (size_t r = 0; r < merges->arr.size(); ++r) {
      const Json& m = merges->arr[r];
      if (m.kind == Json::Arr && m.arr.size() == 2) {  // ["a", "b"]
        add_merge(*t, r, m.arr[0].str, m.arr[1].str);
      } else if (m.kind == Json::Str) {  // "a b"
        const size_t sp = m.str.find(' ', 1);
        if (sp == std::string::npos) fail(JB_ERR_IO, "tokenizer.json: bad merge " + m.str);
        add_merge(*t, r, m.str.substr(0, sp), m.str.substr(sp + 1));
      } else {
        fail(JB_ERR_IO, "tokenizer.json: bad merge entry");
      }
    }
  }
  if (const Json* nz = j.get("normalizer"); nz && nz->kind == Json::Obj) parse_normalizer(*t, *nz);
  if (const Json* pt = j.get("pre_tokenizer"); pt && pt->kind == Json::Obj) parse_pre_tokenizer(*t, *pt);
  if (const Json* pp = j.get("post_processor"); pp && pp->kind == Json::Obj)
    parse_post(*t, *pp, t->before, t->after);
  if (const Json* added = j.get("added_tokens"); added && added->kind == Json::Arr)
    for (const Json& a : added->arr) {
      AddedToken tok;
      tok.content = a.str_or("content", "");
      if (tok.content.empty()) continue;
      tok.id = static_cast<uint32_t>(a.num_or("id", 0));
      tok.lstrip = a.bool_or("lstrip", false);
      tok.rstrip = a.bool_or("rstrip", false);
      tok.single_word = a.bool_or("single_word", false);
      (a.bool_or("normalized", false) ? t->norm_added : t->raw_added).add(tok);
    }
  if (const Json* tr = j.get("truncation"); tr && tr->kind == Json::Obj) {
    t->file_max_length = static_cast<int>(tr->num_or("max_length", 0));
    t->file_trunc_left = tr->str_or("direction", "Right") == "Left";
  }
  return t.release();
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
  t->model = kBpe;
  t->pre.push_back(PreStep{kPreClip});
  t->bpe_suffix = "</w>";
  std::vector<std::string> vocab;
  for (uint32_t c : byte_symbols()) {
    std::string s;
    append_utf8(c, s);
    vocab.push_back(s);
  }
  for (uint32_t c : byte_symbols()) {
    std::string s;
    append_utf8(c, s);
    vocab.push_back(s + "</w>");
  }
  for (const auto& m : merges) vocab.push_back(m.first + m.second);
  vocab.push_back("<|startoftext|>");
  vocab.push_back("<|endoftext|>");
  for (size_t i = 0; i < vocab.size(); ++i) t->vocab[vocab[i]] = static_cast<uint32_t>(i);
  for (size_t r = 0; r < merges.size(); ++r) add_merge(*t, r, merges[r].first, merges[r].second);
  t->before.push_back(static_cast<uint32_t>(vocab.size() - 2));
  t->after.push_back(static_cast<uint32_t>(vocab.size() - 1));
  return t.release();
}

template <typename F>
jb_status guarded_load(const char* path, jb_tokenizer** out, F&& loader) {
  if (!out) return record_error(JB_ERR_INVALID, "null output handle");
  *out = nullptr;
  try {
    if (!path) fail(JB_ERR_INVALID, "null path");
    *out = loader(path);
    return JB_OK;
  } catch (const Error& e) {
    return record_error(e.status, e.msg);
  } catch (const std::exception& e) {
    return record_error(JB_ERR_INVALID, e.what());
  }
}

}  // namespace
}  // namespace jb

namespace {
jb_status tokenize_impl(const jb_tokenizer* t, const char* const* texts, const uint64_t* text_bytes,
                        int64_t n, int max_length, uint32_t* ids, uint64_t ids_capacity,
                        uint64_t* offsets, bool empty_rows) {
  try {
    if (!t || n < 0 || !offsets || (n > 0 && (!texts || !text_bytes)))
      jb::fail(JB_ERR_INVALID, "jb_tokenize: bad argument");
    std::vector<std::vector<uint32_t>> rows(static_cast<size_t>(n));
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const int64_t workers = n >= 256 ? std::min<int64_t>(hw, (n + 127) / 128) : 1;
    std::mutex mu;
    std::string first_error;
    jb_status first_status = JB_OK;
    auto work = [&](int64_t w) {
      try {
        for (int64_t i = w; i < n; i += workers) {
          const bool empty = !texts[i] || text_bytes[i] == 0;
          if (empty && empty_rows) continue;  // a null row: no tokens at all
          jb::encode(*t, texts[i] ? texts[i] : "", texts[i] ? text_bytes[i] : 0, max_length, rows[i]);
        }
      } catch (const jb::Error& e) {
        std::lock_guard<std::mutex> lk(mu);
        if (first_status == JB_OK) first_status = e.status, first_error = e.msg;
      } catch (const std::exception& e) {
        std::lock_guard<std::mutex> lk(mu);
        if (first_status == JB_OK) first_status = JB_ERR_INVALID, first_error = e.what();
      }
    };
    if (workers == 1) {
      work(0);
    } else {
      std::vector<std::thread> pool;
      for (int64_t w = 0; w < workers; ++w) pool.emplace_back(work, w);
      for (auto& th : pool) th.join();
    }
    if (first_status != JB_OK) jb::fail(first_status, first_error);
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

}  // namespace

extern "C" {

jb_status jb_tokenizer_load(const char* tokenizer_json_path, jb_tokenizer** out) {
  return jb::guarded_load(tokenizer_json_path, out, jb::load);
}

jb_status jb_tokenizer_load_clip_bpe(const char* merges_path, jb_tokenizer** out) {
  return jb::guarded_load(merges_path, out, jb::load_clip);
}

void jb_tokenizer_free(jb_tokenizer* t) { delete t; }

jb_status jb_tokenize(const jb_tokenizer* t, const char* const* texts, const uint64_t* text_bytes,
                      int64_t n, int max_length, uint32_t* ids, uint64_t ids_capacity,
                      uint64_t* offsets) {
  return tokenize_impl(t, texts, text_bytes, n, max_length, ids, ids_capacity, offsets, false);
}

jb_status jb_tokenize_rows(const jb_tokenizer* t, const char* const* texts, const uint64_t* text_bytes,
                           int64_t n, int max_length, uint32_t* ids, uint64_t ids_capacity,
                           uint64_t* offsets) {
  return tokenize_impl(t, texts, text_bytes, n, max_length, ids, ids_capacity, offsets, true);
}

}  // extern "C"
