"""The library's OpenCLIP BPE tokenizer (jb_tokenizer_load_clip_bpe) against
HuggingFace `tokenizers` configured as the reference's load_open_clip_bpe
(crates/jammi-ai/src/model/clip_bpe.rs:52-217) configures it, id for id, on
merges files built here by a small BPE trainer over seeded synthetic text
(OpenCLIP's own merges file is not used).  CPU only."""
import gzip

import numpy as np
import pytest

tokenizers = pytest.importorskip("tokenizers")
regex = pytest.importorskip("regex")

CLIP_REGEX = (r"<\|startoftext\|>|<\|endoftext\|>|'s|'t|'re|'ve|'m|'ll|'d|"
              r"[\p{L}]+|[\p{N}]|[^\s\p{L}\p{N}]+")
SOT, EOT = "<|startoftext|>", "<|endoftext|>"
FULL_MERGES = 49408 - 256 - 2 - 256

ALPHABET = (
    "abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789"
    "      .,;:!?'\"()[]{}-_/\\@#$%^&*+=<>|~`"
    "àáâäãåæçèéêëìíîïñòóôöõøùúûüýÿßÀÉÎÕÜ¼½²³µ"
    "αβγΣσ" "абвгЖЯ" "東京数据" "한국" "ｆｕｌｌ" "٣٤"
    "̣́̈" "\t\n\r 　  " "\u0000\u0007​﻿" "😀€£¥©®™…—«»¿¡"
)
WORDS = ["the", "photo", "of", "a", "cat", "dog", "it's", "don't", "we're", "I've", "I'm",
         "you'll", "he'd", "café", "naïve", "2024", "!!!", "...", "<|endoftext|>", "Über"]


def byte_chars():
    direct = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    extra, out = 0, []
    for b in range(256):
        if b in direct:
            out.append(chr(b))
        else:
            out.append(chr(256 + extra))
            extra += 1
    return out


def random_texts(seed, n, max_len=60):
    rng = np.random.default_rng(seed)
    chars = list(ALPHABET)
    out = []
    for _ in range(n):
        parts = []
        for _ in range(int(rng.integers(0, 12))):
            if rng.random() < 0.6:
                parts.append(WORDS[int(rng.integers(0, len(WORDS)))])
            else:
                k = int(rng.integers(1, max_len // 6 + 2))
                parts.append("".join(chars[i] for i in rng.integers(0, len(chars), size=k)))
        out.append(" ".join(parts) if rng.random() < 0.7 else "".join(parts))
    return out


def train_merges(texts, n_merges):
    """Greedy BPE over the CLIP pre-tokens of `texts`: each pre-token a list of
    its characters that are in the byte alphabet, "</w>" on the last; the most
    frequent adjacent pair merged first (ties by first appearance)."""
    alphabet = set(byte_chars())
    counts = {}
    for t in texts:
        for m in regex.finditer(CLIP_REGEX, t):
            w = [c for c in m.group() if c in alphabet]
            if w:
                w[-1] += "</w>"
                counts[tuple(w)] = counts.get(tuple(w), 0) + 1
    words = [list(w) for w in counts]
    freq = list(counts.values())
    merges = []
    while len(merges) < n_merges:
        pairs = {}
        for w, f in zip(words, freq):
            for a, b in zip(w, w[1:]):
                pairs[(a, b)] = pairs.get((a, b), 0) + f
        if not pairs:
            break
        best = max(pairs.items(), key=lambda kv: kv[1])[0]
        merges.append(best)
        for w in words:
            i = 0
            while i + 1 < len(w):
                if (w[i], w[i + 1]) == best:
                    w[i:i + 2] = [w[i] + w[i + 1]]
                i += 1
    return merges


def write_merges(path, merges, compress):
    text = "#version: synthetic\n" + "".join(f"{a} {b}\n" for a, b in merges)
    if compress:
        with gzip.open(path, "wt", encoding="utf-8") as f:
            f.write(text)
    else:
        path.write_text(text, encoding="utf-8")


def hf_clip_tokenizer(merges):
    """The reference's construction (clip_bpe.rs:85-204) through the Python
    bindings of the same crate."""
    from tokenizers import Regex, Tokenizer, models, pre_tokenizers, processors
    bc = byte_chars()
    vocab_list = bc + [c + "</w>" for c in bc] + [a + b for a, b in merges] + [SOT, EOT]
    vocab = {t: i for i, t in enumerate(vocab_list)}
    tok = Tokenizer(models.BPE(vocab=vocab, merges=list(merges), end_of_word_suffix="</w>"))
    tok.pre_tokenizer = pre_tokenizers.Split(Regex(CLIP_REGEX), behavior="isolated", invert=False)
    n = len(vocab_list)
    tok.post_processor = processors.TemplateProcessing(
        single=f"{SOT}:0 $A:0 {EOT}:0", special_tokens=[(SOT, n - 2), (EOT, n - 1)])
    return tok


CASES = [
    "a photo of a cat", "", "   ", "it's I'M we're 'hello' ''s", "2024-12-02 v1.2.3",
    "café naïve Über ÀÉÎ", "東京 data 数据", "<|startoftext|>a cat<|endoftext|>", "!!!...???",
    "tab\tnew\nline\r　ideographic sep", "x\u0000y​z﻿", "😀 emoji… — «q»",
    "½ ² ³ µ ٣٤ ｆｕｌｌ", "don'tdon't", "aaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaaa",
]


@pytest.fixture(scope="module")
def merges():
    return train_merges(random_texts(1, 3000), 1500)


@pytest.mark.parametrize("compress", [True, False])
def test_matches_hf_tokenizers(tmp_path, merges, compress):
    from jammi_b200 import Tokenizer
    path = tmp_path / ("bpe.txt.gz" if compress else "bpe.txt")
    write_merges(path, merges, compress)
    hf = hf_clip_tokenizer(merges)
    ours = Tokenizer.clip_bpe(str(path))
    texts = CASES + random_texts(7, 500)
    got = ours(texts)
    bad = [(t, hf.encode(t).ids, list(g)) for t, g in zip(texts, got) if hf.encode(t).ids != list(g)]
    assert not bad, bad[:3]


def test_truncation_keeps_sot_and_eot(tmp_path, merges):
    """max_length counts <|startoftext|> and <|endoftext|> (OpenCLIP's context
    length is 77 with both), so the EOT the text tower pools on survives."""
    from jammi_b200 import Tokenizer
    path = tmp_path / "bpe.txt.gz"
    write_merges(path, merges, True)
    hf = hf_clip_tokenizer(merges)
    ours = Tokenizer.clip_bpe(str(path))
    texts = random_texts(9, 80, 200)
    n = len(merges) + 512 + 2
    for max_len in (2, 5, 77):
        hf.enable_truncation(max_length=max_len)
        ids, offsets = ours.encode_ragged(texts, max_length=max_len)
        for i, t in enumerate(texts):
            row = list(ids[offsets[i]:offsets[i + 1]])
            assert row == hf.encode(t).ids
            assert len(row) <= max_len and row[0] == n - 2 and row[-1] == n - 1


def test_merges_beyond_openclip_vocab_are_ignored(tmp_path):
    """OpenCLIP reads 48894 merges (a 49408-token vocabulary); later lines are
    not merges and the specials stay at ids 49406 and 49407."""
    from jammi_b200 import Tokenizer
    filler = [c for c in byte_chars() if c.isalpha() and c not in "abcd"]
    pairs = [(x, y) for x in filler for y in filler] + [(x, y + "</w>") for x in filler for y in filler]
    merges = pairs[:FULL_MERGES - 1] + [("a", "b</w>"), ("c", "d</w>"), ("a", "c</w>")]
    path = tmp_path / "big.txt.gz"
    write_merges(path, merges, True)
    ours = Tokenizer.clip_bpe(str(path))
    assert list(ours([""])[0]) == [49406, 49407]
    assert list(ours(["ab"])[0]) == [49406, 49405, 49407]        # the last merge read
    assert list(ours(["cd"])[0]) == [49406, ord("c"), 256 + ord("d"), 49407]  # past the limit
    hf = hf_clip_tokenizer(merges[:FULL_MERGES])
    for text in ("ab", "cd", "ac", "abcd ab cd", "a photo of a cat"):
        assert list(ours([text])[0]) == hf.encode(text).ids


def test_bad_merges_files_are_rejected(tmp_path):
    from jammi_b200 import Tokenizer
    from jammi_b200._lib import JbError
    with pytest.raises(JbError):
        Tokenizer.clip_bpe(str(tmp_path / "missing.txt.gz"))
    empty = tmp_path / "empty.txt"
    empty.write_text("#version: 0.2\n")
    with pytest.raises(JbError):
        Tokenizer.clip_bpe(str(empty))
    unknown = tmp_path / "unknown.txt"
    unknown.write_text("#version: 0.2\nzz y\n")  # "zz" is neither a byte symbol nor a merge
    with pytest.raises(JbError):
        Tokenizer.clip_bpe(str(unknown))
