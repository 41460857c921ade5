"""Generates jb_unicode_tables.h: the Unicode data the host tokenizers'
normalisers (BERT, NFC, NFD, lowercase), pre-tokenisers (BERT, byte-level,
OpenCLIP) and added-token matching need (jb_tokenizer.cpp), from Python's
unicodedata:

* per-code-point lowercase mappings (one code point at a time, as the HF
  normaliser lowercases, so there is no final-sigma context),
* compatibility decompositions (full NFKD of each character, where it differs
  from the canonical one; for NFKC / NFKD),
* canonical decompositions (full, recursive; Hangul syllables are decomposed
  algorithmically in the C++ code) and canonical combining classes (for the
  canonical reordering of NFD),
* the ranges of general categories C* (other, including unassigned),
  P* (punctuation), Mn (nonspacing marks), L* (letters) and N* (numbers),
* the ranges of general category M* (marks, for StripAccents),
* the Grapheme_Cluster_Break classes, Extended_Pictographic and
  Indic_Conjunct_Break of UAX #29 (the extended grapheme clusters the
  Precompiled normaliser works on; from the regex module's properties),
* the ranges of regex word characters (\\w: Alphabetic, marks, decimal
  digits, connector punctuation, joiners; from the `regex` module), the
  \\w of the Whitespace pre-tokeniser and of an added token's single_word
  boundaries (the regex module's Unicode data is newer than unicodedata's,
  closer to the tokenizers crate's),
* the primary composites of NFC: (first, second) -> composite for every
  two-code-point canonical decomposition that NFC recomposes (composition
  exclusions and singletons left out; Hangul is algorithmic).

    python jammi-ai_b200/csrc/gen_unicode_tables.py   # rewrites jb_unicode_tables.h
"""
import os
import sys
import unicodedata

MAX_CP = 0x110000
HANGUL = range(0xAC00, 0xAC00 + 11172)


def ranges(pred):
    out, start = [], None
    for cp in range(MAX_CP):
        if pred(cp):
            if start is None:
                start = cp
        elif start is not None:
            out.append((start, cp - 1))
            start = None
    if start is not None:
        out.append((start, MAX_CP - 1))
    return out


def cat(cp):
    return unicodedata.category(chr(cp))


def main():
    here = os.path.dirname(os.path.abspath(__file__))
    other = ranges(lambda cp: cat(cp).startswith("C"))
    punct = ranges(lambda cp: cat(cp).startswith("P"))
    mark_nonspacing = ranges(lambda cp: cat(cp) == "Mn")
    letter = ranges(lambda cp: cat(cp).startswith("L"))
    number = ranges(lambda cp: cat(cp).startswith("N"))
    mark = ranges(lambda cp: cat(cp).startswith("M"))
    import regex
    word_re = regex.compile(r"\w")
    word = ranges(lambda cp: not 0xD800 <= cp <= 0xDFFF and word_re.match(chr(cp)) is not None)

    # Grapheme_Cluster_Break classes (UAX #29), Extended_Pictographic and
    # Indic_Conjunct_Break, from the regex module's property support
    gcb_names = ["CR", "LF", "Control", "Extend", "ZWJ", "Regional_Indicator", "Prepend", "SpacingMark",
                 "L", "V", "T", "LV", "LVT"]
    gcb_res = [(k + 1, regex.compile(r"\p{GCB=%s}" % n)) for k, n in enumerate(gcb_names)]
    incb_res = [(k + 1, regex.compile(r"\p{InCB=%s}" % n)) for k, n in enumerate(["Consonant", "Extend", "Linker"])]

    def classify(res):
        def f(cp):
            if 0xD800 <= cp <= 0xDFFF:
                return 0
            for k, r in res:
                if r.match(chr(cp)):
                    return k
            return 0
        return f

    def class_ranges(fn):
        out, start, cur = [], None, 0
        for cp in range(MAX_CP):
            k = fn(cp)
            if k != cur:
                if cur:
                    out.append((start, cp - 1, cur))
                start, cur = cp, k
        if cur:
            out.append((start, MAX_CP - 1, cur))
        return out

    gcb = class_ranges(classify(gcb_res))
    incb = class_ranges(classify(incb_res))
    ext_pict_re = regex.compile(r"\p{Extended_Pictographic}")
    ext_pict = ranges(lambda cp: not 0xD800 <= cp <= 0xDFFF and ext_pict_re.match(chr(cp)) is not None)

    compose = []  # (first, second, composite)
    for cp in range(MAX_CP):
        if 0xD800 <= cp <= 0xDFFF or cp in HANGUL:
            continue
        d = unicodedata.decomposition(chr(cp))
        if not d or d.startswith("<"):
            continue
        parts = [int(x, 16) for x in d.split()]
        if len(parts) == 2 and unicodedata.normalize("NFC", chr(cp)) == chr(cp):
            compose.append((parts[0], parts[1], cp))
    compose.sort()

    lower = []  # (cp, [mapped...])
    for cp in range(MAX_CP):
        if 0xD800 <= cp <= 0xDFFF:
            continue
        lo = chr(cp).lower()
        if lo != chr(cp):
            lower.append((cp, [ord(c) for c in lo]))

    decomp = []  # (cp, [decomposed...]) canonical, full
    for cp in range(MAX_CP):
        if 0xD800 <= cp <= 0xDFFF or cp in HANGUL:
            continue
        d = unicodedata.normalize("NFD", chr(cp))
        if d != chr(cp):
            decomp.append((cp, [ord(c) for c in d]))

    kdecomp = []  # (cp, [decomposed...]) compatibility, full, where it differs from the canonical one
    for cp in range(MAX_CP):
        if 0xD800 <= cp <= 0xDFFF or cp in HANGUL:
            continue
        k = unicodedata.normalize("NFKD", chr(cp))
        if k != unicodedata.normalize("NFD", chr(cp)):
            kdecomp.append((cp, [ord(c) for c in k]))

    ccc = [(cp, unicodedata.combining(chr(cp))) for cp in range(MAX_CP)
           if not 0xD800 <= cp <= 0xDFFF and unicodedata.combining(chr(cp))]

    def seq_table(name, entries):
        flat, rows = [], []
        for cp, seq in entries:
            rows.append((cp, len(flat), len(seq)))
            flat.extend(seq)
        s = [f"static const uint32_t {name}_seq[] = {{"]
        for i in range(0, len(flat), 12):
            s.append("  " + ", ".join(f"0x{v:X}" for v in flat[i:i + 12]) + ",")
        s.append("};")
        s.append(f"static const SeqEntry {name}[] = {{")
        for cp, off, n in rows:
            s.append(f"  {{0x{cp:X}, {off}, {n}}},")
        s.append("};")
        return "\n".join(s)

    def range_table(name, rs):
        s = [f"static const CpRange {name}[] = {{"]
        for a, b in rs:
            s.append(f"  {{0x{a:X}, 0x{b:X}}},")
        s.append("};")
        return "\n".join(s)

    lines = [
        "// Generated by gen_unicode_tables.py from Python's unicodedata "
        f"(Unicode {unicodedata.unidata_version}); do not edit.",
        "#pragma once",
        "#include <cstdint>",
        "",
        "namespace jb {",
        "namespace uni {",
        "struct CpRange { uint32_t lo, hi; };",
        "struct SeqEntry { uint32_t cp, off, n; };",
        "struct CccEntry { uint32_t cp; uint8_t ccc; };",
        "struct ComposeEntry { uint32_t first, second, composite; };",
        "struct ClassRange { uint32_t lo, hi; uint8_t cls; };",
        "// Grapheme_Cluster_Break: 1 CR, 2 LF, 3 Control, 4 Extend, 5 ZWJ, 6 Regional_Indicator,",
        "// 7 Prepend, 8 SpacingMark, 9 L, 10 V, 11 T, 12 LV, 13 LVT (0: Other)",
        "// Indic_Conjunct_Break: 1 Consonant, 2 Extend, 3 Linker (0: None)",
        f'static const char kUnicodeVersion[] = "{unicodedata.unidata_version}";',
        range_table("kOther", other),
        range_table("kPunct", punct),
        range_table("kMarkNonspacing", mark_nonspacing),
        range_table("kLetter", letter),
        range_table("kNumber", number),
        range_table("kWord", word),
        range_table("kMark", mark),
        range_table("kExtPict", ext_pict),
        "static const ClassRange kGcb[] = {",
        *[f"  {{0x{a:X}, 0x{b:X}, {c}}}," for a, b, c in gcb],
        "};",
        "static const ClassRange kIncb[] = {",
        *[f"  {{0x{a:X}, 0x{b:X}, {c}}}," for a, b, c in incb],
        "};",
        "static const ComposeEntry kCompose[] = {",
        *[f"  {{0x{a:X}, 0x{b:X}, 0x{c:X}}}," for a, b, c in compose],
        "};",
        seq_table("kLower", lower),
        seq_table("kDecomp", decomp),
        seq_table("kCompatDecomp", kdecomp),
        "static const CccEntry kCcc[] = {",
        *[f"  {{0x{cp:X}, {c}}}," for cp, c in ccc],
        "};",
        "}  // namespace uni",
        "}  // namespace jb",
        "",
    ]
    out = os.path.join(here, "jb_unicode_tables.h")
    with open(out, "w") as f:
        f.write("\n".join(lines))
    print("wrote", out, len(other), len(punct), len(mark_nonspacing), len(letter), len(number), len(word), len(compose), len(lower),
          len(decomp), len(ccc), file=sys.stderr)


if __name__ == "__main__":
    main()
