"""The library's tokenizer.json BPE path (jb_tokenizer_load on a BPE model:
byte-level as RoBERTa / GPT-2 / ModernBERT checkpoints ship it, or
character-level with an unknown token, byte fallback, subword affixes)
against HuggingFace `tokenizers` -- the crate the reference loads any
tokenizer.json with (crates/jammi-ai/src/model/tokenizer.rs:21-78) -- id for
id, on tokenizer.json files trained here from seeded synthetic text.
CPU only."""
import json

import numpy as np
import pytest

tokenizers = pytest.importorskip("tokenizers")

from test_tokenizer import random_texts  # noqa: E402

SPECIALS = ["[UNK]", "[CLS]", "[SEP]", "[PAD]", "[MASK]"]
CASES = [
    "Hello World", "", " ", "   leading and trailing   ", "it's don't we're I've I'm you'll he'd",
    "'S 'LL' 's", "tabs\tand\nnewlines\r\n  x", "naïve café ÜBER Straße", "é ä ộ",
    "각 한", "東京の数据 GPU!", "😀 emoji… — «quotes»", "1234567 12.5%",
    "a<mask> b <mask>c", "<sep>   after <sep>", "foo foobar _foo foo_ (foo)", "HELLO hello Hello",
    "x  y   z    w", "[CLS] inside [SEP] text [MASK]", "Ǆ ǅ İstanbul ΣΑΣ", "a playedunp b",
]


def train_texts():
    return random_texts(1, 2000, 40) + ["reading played unplayable café naïve hello foo"] * 5


def added_tokens():
    from tokenizers import AddedToken
    return [
        AddedToken("<mask>", lstrip=True, normalized=False, special=True),
        AddedToken("<sep>", rstrip=True, normalized=False, special=True),
        AddedToken("  ", normalized=True, special=False),
        AddedToken("foo", single_word=True, normalized=True, special=False),
        AddedToken("hello", normalized=True, special=False),
    ]


def post_processor(kind, tok):
    from tokenizers import processors
    cls, sep = tok.token_to_id("[CLS]"), tok.token_to_id("[SEP]")
    template = processors.TemplateProcessing(single="[CLS] $A [SEP]",
                                             special_tokens=[("[CLS]", cls), ("[SEP]", sep)])
    if kind == "template":
        return template
    if kind == "roberta":
        return processors.RobertaProcessing(("[SEP]", sep), ("[CLS]", cls))
    if kind == "sequence":
        return processors.Sequence([processors.ByteLevel(trim_offsets=True), template])
    return None


def normalizer(kind):
    from tokenizers import normalizers
    return {"none": None, "nfc": normalizers.NFC(), "nfd": normalizers.NFD(),
            "nfc_lower": normalizers.Sequence([normalizers.NFC(), normalizers.Lowercase()])}[kind]


def save(tok, path, edit=None):
    tok.save(str(path))
    if edit is not None:
        doc = json.loads(path.read_text(encoding="utf-8"))
        edit(doc)
        path.write_text(json.dumps(doc), encoding="utf-8")  # ASCII with \\u escapes
        tok = tokenizers.Tokenizer.from_file(str(path))
    return tok, str(path)


def build_byte_level(tmp_path, norm="nfc", add_prefix_space=False, post="template", with_added=True):
    from tokenizers import Tokenizer, models, pre_tokenizers, trainers
    tok = Tokenizer(models.BPE())
    n = normalizer(norm)
    if n is not None:
        tok.normalizer = n
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=add_prefix_space, use_regex=True)
    trainer = trainers.BpeTrainer(vocab_size=1200, special_tokens=SPECIALS, show_progress=False,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    tok.train_from_iterator(train_texts(), trainer=trainer)
    pp = post_processor(post, tok)
    if pp is not None:
        tok.post_processor = pp
    if with_added:
        tok.add_tokens(added_tokens())
    return tok


def assert_same(ours, hf, texts):
    got = ours(texts)
    bad = [(t, hf.encode(t).ids, list(g)) for t, g in zip(texts, got) if hf.encode(t).ids != list(g)]
    assert not bad, bad[:3]


@pytest.mark.parametrize("norm,add_prefix_space,post", [
    ("nfc", False, "template"), ("none", True, "roberta"), ("nfc_lower", False, "sequence"),
    ("nfd", True, None), ("nfc", True, "template"),
])
def test_byte_level_matches_hf_tokenizers(tmp_path, norm, add_prefix_space, post):
    from jammi_b200 import Tokenizer
    hf, path = save(build_byte_level(tmp_path, norm, add_prefix_space, post), tmp_path / "tok.json")
    assert_same(Tokenizer(path), hf, CASES + random_texts(7, 400))


def test_merges_as_strings_ignore_merges_and_escaped_json(tmp_path):
    """Older tokenizer.json files list merges as "a b" strings; ignore_merges
    takes a word found whole in the vocabulary as one token; a file written
    with \\u escapes (surrogate pairs included) reads the same."""
    from jammi_b200 import Tokenizer

    def to_strings(doc):
        doc["model"]["merges"] = [" ".join(m) if isinstance(m, list) else m for m in doc["model"]["merges"]]

    def ignore(doc):
        to_strings(doc)
        doc["model"]["ignore_merges"] = True
        n = len(doc["model"]["vocab"])  # a whole-word entry no merge path reaches; the
        doc["model"]["vocab"]["Ġplayedunp"] = n  # added tokens after the vocabulary move up one
        for a in doc["added_tokens"]:
            a["id"] += a["id"] >= n

    for edit in (to_strings, ignore):
        hf, path = save(build_byte_level(tmp_path), tmp_path / "tok.json", edit)
        assert_same(Tokenizer(path), hf, CASES + random_texts(8, 200))


def build_char_level(tmp_path, prefix=None, suffix=None, fuse_unk=False):
    """Character-level BPE over BERT-style pre-tokens with a limited alphabet,
    so rare characters hit the unknown token."""
    from tokenizers import Tokenizer, models, normalizers, pre_tokenizers, trainers
    kw = {}
    if prefix:
        kw["continuing_subword_prefix"] = prefix
    if suffix:
        kw["end_of_word_suffix"] = suffix
    tok = Tokenizer(models.BPE(unk_token="[UNK]", fuse_unk=fuse_unk, **kw))
    tok.normalizer = normalizers.BertNormalizer(lowercase=False)
    tok.pre_tokenizer = pre_tokenizers.BertPreTokenizer()
    trainer = trainers.BpeTrainer(vocab_size=900, special_tokens=SPECIALS, show_progress=False,
                                  limit_alphabet=70, **kw)
    tok.train_from_iterator(train_texts(), trainer=trainer)
    tok.post_processor = post_processor("template", tok)
    return tok


@pytest.mark.parametrize("prefix,suffix,fuse_unk", [
    (None, None, False), (None, None, True), ("##", None, False), (None, "</w>", True), ("##", "</w>", False),
])
def test_char_level_unknowns_and_affixes(tmp_path, prefix, suffix, fuse_unk):
    from jammi_b200 import Tokenizer
    hf, path = save(build_char_level(tmp_path, prefix, suffix, fuse_unk), tmp_path / "tok.json")
    assert_same(Tokenizer(path), hf, CASES + random_texts(9, 300))


@pytest.mark.parametrize("fuse_unk", [False, True])
def test_byte_fallback(tmp_path, fuse_unk):
    """Characters outside the vocabulary become their <0xXX> byte tokens when
    every byte has one (bytes 0x00-0xEF here, so four-byte characters fall
    through to the unknown token)."""
    from jammi_b200 import Tokenizer

    def add_bytes(doc):
        vocab = doc["model"]["vocab"]
        nxt = max(vocab.values()) + 1
        for b in range(0xF0):
            vocab[f"<0x{b:02X}>"] = nxt + b
        doc["model"]["byte_fallback"] = True

    hf, path = save(build_char_level(tmp_path, fuse_unk=fuse_unk), tmp_path / "tok.json", add_bytes)
    assert_same(Tokenizer(path), hf, CASES + random_texts(10, 300))


def test_truncation_from_the_file(tmp_path):
    """Without max_length the file's own truncation applies, direction
    included; a max_length given to the call cuts the tail."""
    from jammi_b200 import Tokenizer
    hf = build_byte_level(tmp_path)
    hf.enable_truncation(max_length=7, direction="left")
    hf, path = save(hf, tmp_path / "tok.json")
    ours = Tokenizer(path)
    texts = random_texts(11, 60, 80)
    assert_same(ours, hf, texts)
    hf.enable_truncation(max_length=5)
    ids, offsets = ours.encode_ragged(texts, max_length=5)
    for i, t in enumerate(texts):
        assert list(ids[offsets[i]:offsets[i + 1]]) == hf.encode(t).ids


def test_many_texts_threads_keep_order(tmp_path):
    from jammi_b200 import Tokenizer
    hf, path = save(build_byte_level(tmp_path), tmp_path / "tok.json")
    texts = random_texts(12, 2000, 30)
    got = Tokenizer(path)(texts)
    assert [list(g) for g in got] == [e.ids for e in hf.encode_batch(texts)]
    assert all(isinstance(g, np.ndarray) for g in got[:3])


def test_escaped_astral_added_token(tmp_path):
    """A tokenizer.json written with \\u escapes spells characters outside
    the BMP as surrogate pairs; they decode to the one character."""
    from tokenizers import AddedToken
    from jammi_b200 import Tokenizer
    hf = build_byte_level(tmp_path)
    hf.add_tokens([AddedToken("😀🚀", normalized=False, special=True)])
    hf, path = save(hf, tmp_path / "tok.json", edit=lambda doc: None)
    assert "\\ud83d" in open(path).read()
    assert_same(Tokenizer(path), hf, ["a😀🚀b", "😀 🚀", "x 😀🚀😀🚀"])


def test_long_unbroken_words(tmp_path):
    """Words thousands of symbols long (URLs, base64, repeated letters) merge
    in the crate's order; the heap-ordered merge keeps this fast."""
    import time
    from jammi_b200 import Tokenizer
    hf, path = save(build_byte_level(tmp_path), tmp_path / "tok.json")
    rng = np.random.default_rng(3)
    letters = np.array(list("abcdefghijklmnopqrstuvwxyz"))
    texts = ["a" * 5000, "ab" * 2500, "".join(rng.choice(letters, 6000)),
             "https://example.com/" + "x".join(rng.choice(letters, 3000)),
             "".join(rng.choice(list("ABCDEFGHIJKLMNOPQRSTUVWXYZabcdefghijklmnopqrstuvwxyz0123456789+/"), 8000))]
    t0 = time.perf_counter()
    assert_same(Tokenizer(path), hf, texts)
    assert time.perf_counter() - t0 < 30
