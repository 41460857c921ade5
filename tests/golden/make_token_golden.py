"""Generate tests/golden/reference_tiny_bert_tokens.json (run once, here, on CPU).

    JAMMI_REFERENCE=<reference checkout> python tests/golden/make_token_golden.py

Token ids of seeded synthetic texts under the reference's own fixture
tokenizers (cookbook/fixtures/tiny_bert/tokenizer.json: Lowercase +
StripAccents, Whitespace pre-tokeniser, WordPiece, [CLS]/[SEP]; and
tests/fixtures/tiny_open_clip/tokenizer.json: WordLevel over single
characters, '$A <|endoftext|>'), computed by
HuggingFace `tokenizers` -- the crate the reference tokenises with -- with
and without truncation.  Only texts and ids are written; the tokenizer files
stay in the reference checkout.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.environ.get("JAMMI_REFERENCE", "")
REF_TOKENIZER = os.path.join(REF_ROOT, "cookbook", "fixtures", "tiny_bert", "tokenizer.json")
REF_CLIP_TOKENIZER = os.path.join(REF_ROOT, "tests", "fixtures", "tiny_open_clip", "tokenizer.json")

ALPHABET = ("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789     .,;:!?'\"()-_/"
            "àáâäãåæçèéêëìíîïñòóôöõøùúûüýÿßÀÉÎÕÜ" "αβγΣσ" "東京数据" "̣́̈" "\t\n　" "😀€…—«»")
WORDS = ["the", "model", "embedding", "vector", "search", "query", "document", "naïve", "café",
         "CAFÉ", "résumé", "data", "fine-tune", "e-mail", "don't", "2024", "B200", "GPU's"]


def texts(seed=0, n=120):
    rng = np.random.default_rng(seed)
    out = ["", "Hello World", "naïve CAFÉ Ünïcödé", "  spaces\tand\nlines  ", "a-b_c.d,e!f?"]
    chars = list(ALPHABET)
    while len(out) < n:
        parts = []
        for _ in range(int(rng.integers(1, 10))):
            if rng.random() < 0.6:
                parts.append(WORDS[int(rng.integers(0, len(WORDS)))])
            else:
                k = int(rng.integers(1, 8))
                parts.append("".join(chars[i] for i in rng.integers(0, len(chars), size=k)))
        out.append(" ".join(parts))
    return out


def main():
    from tokenizers import Tokenizer
    if not REF_ROOT or not os.path.exists(REF_TOKENIZER):
        sys.exit("reference checkout not present")
    tok = Tokenizer.from_file(REF_TOKENIZER)
    ts = texts()
    doc = {"source": "cookbook/fixtures/tiny_bert/tokenizer.json", "texts": ts,
           "ids": [e.ids for e in tok.encode_batch(ts)]}
    for max_len in (4, 9):
        tok.enable_truncation(max_length=max_len)
        doc[f"ids_max{max_len}"] = [e.ids for e in tok.encode_batch(ts)]
    clip = Tokenizer.from_file(REF_CLIP_TOKENIZER)
    doc["clip_source"] = "tests/fixtures/tiny_open_clip/tokenizer.json"
    doc["clip_ids"] = [e.ids for e in clip.encode_batch(ts)]
    with open(os.path.join(HERE, "reference_tiny_bert_tokens.json"), "w", encoding="utf-8") as f:
        json.dump(doc, f, ensure_ascii=False)


if __name__ == "__main__":
    main()
