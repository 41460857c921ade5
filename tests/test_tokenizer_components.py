"""The remaining tokenizer.json components the native tokenizer reads --
StripAccents, Strip, Prepend, Replace, NFKC and NFKD normalisers;
Whitespace, WhitespaceSplit, Punctuation (every split behaviour), Digits and
Split pre-tokenisers; Sequences of them; the WordLevel model -- against
HuggingFace `tokenizers`, id for id, and the reference's own fixture
tokenizers (cookbook/fixtures/tiny_bert: Lowercase + StripAccents,
Whitespace, WordPiece; tests/fixtures/tiny_open_clip: WordLevel over
characters).  CPU only."""
import json
import os

import pytest

tokenizers = pytest.importorskip("tokenizers")

from conftest import reference_path  # noqa: E402
from test_tokenizer import CASES, random_texts  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_tiny_bert_tokens.json")
REF_TOKENIZER = reference_path("cookbook", "fixtures", "tiny_bert", "tokenizer.json")

EXTRA = CASES + [
    "Mc: कः  Me: a⃝  Mn: é", "  padded both ends  ", "x__y _z_ a-b-c", "...!!!???", "a1b22c333 4444",
    "१२३ ٣٤ ½ ²", "don't stop", "[CLS] [SEP]", "ab" * 30,
    "ｆｕｌｌ ① ㍻ ﬁ ¼ Å Ǆ ᾯ ẛ̣ 가각 ㈜ ⅷ",
]


def _train(tok, model_kind, tmp_path, name):
    from tokenizers import trainers
    specials = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"]
    if model_kind == "wordpiece":
        trainer = trainers.WordPieceTrainer(vocab_size=1200, special_tokens=specials)
    else:
        trainer = trainers.BpeTrainer(vocab_size=900, special_tokens=specials, show_progress=False,
                                      limit_alphabet=120)
    tok.train_from_iterator(random_texts(1, 2000, 40) + ["reading played 12345 naïve"] * 5, trainer=trainer)
    from tokenizers import processors
    cls, sep = tok.token_to_id("[CLS]"), tok.token_to_id("[SEP]")
    tok.post_processor = processors.TemplateProcessing(single="[CLS] $A [SEP]",
                                                       special_tokens=[("[CLS]", cls), ("[SEP]", sep)])
    path = tmp_path / name
    tok.save(str(path))
    return tok, str(path)


def _same(path, hf, texts):
    from jammi_b200 import Tokenizer
    got = Tokenizer(path)(texts)
    bad = [(t, hf.encode(t).ids, list(g)) for t, g in zip(texts, got) if hf.encode(t).ids != list(g)]
    assert not bad, bad[:3]


def _normalizers():
    from tokenizers import normalizers as n
    return {
        "lower_stripaccents": n.Sequence([n.Lowercase(), n.StripAccents()]),
        "nfd_stripaccents": n.Sequence([n.NFD(), n.StripAccents()]),
        "strip_both": n.Strip(),
        "strip_left": n.Strip(left=True, right=False),
        "prepend_replace": n.Sequence([n.Replace(" ", "_"), n.Prepend("_")]),
        "replace_multi": n.Sequence([n.Replace("ab", "X"), n.Replace("  ", " ")]),
        "nfkc": n.NFKC(),
        "nfkd_lower": n.Sequence([n.NFKD(), n.Lowercase()]),
    }


def _pre_tokenizers():
    from tokenizers import pre_tokenizers as p
    return {
        "whitespace": p.Whitespace(),
        "whitespace_split": p.WhitespaceSplit(),
        "punct_isolated": p.Sequence([p.WhitespaceSplit(), p.Punctuation()]),
        "punct_removed": p.Sequence([p.WhitespaceSplit(), p.Punctuation("removed")]),
        "punct_prev": p.Sequence([p.WhitespaceSplit(), p.Punctuation("merged_with_previous")]),
        "punct_next": p.Sequence([p.WhitespaceSplit(), p.Punctuation("merged_with_next")]),
        "punct_contiguous": p.Sequence([p.WhitespaceSplit(), p.Punctuation("contiguous")]),
        "digits_each": p.Sequence([p.Whitespace(), p.Digits(individual_digits=True)]),
        "digits_runs": p.Sequence([p.WhitespaceSplit(), p.Digits(individual_digits=False)]),
        "digits_bytelevel": p.Sequence([p.Digits(individual_digits=True), p.ByteLevel(add_prefix_space=False)]),
    }


@pytest.mark.parametrize("norm", sorted(_normalizers()))
def test_normalizers(tmp_path, norm):
    from tokenizers import Tokenizer, models, pre_tokenizers
    tok = Tokenizer(models.WordPiece(unk_token="[UNK]"))
    tok.normalizer = _normalizers()[norm]
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    hf, path = _train(tok, "wordpiece", tmp_path, "tok.json")
    _same(path, hf, EXTRA + random_texts(3, 300))


@pytest.mark.parametrize("pre", sorted(_pre_tokenizers()))
def test_pre_tokenizers(tmp_path, pre):
    from tokenizers import Tokenizer, models
    kind = "bpe" if "bytelevel" in pre else "wordpiece"
    tok = Tokenizer(models.BPE(unk_token="[UNK]") if kind == "bpe" else models.WordPiece(unk_token="[UNK]"))
    tok.pre_tokenizer = _pre_tokenizers()[pre]
    hf, path = _train(tok, kind, tmp_path, "tok.json")
    _same(path, hf, EXTRA + random_texts(4, 300))


def test_reference_fixture_tokenizer_golden_ids():
    """The reference's own tiny_bert tokenizer (Lowercase + StripAccents,
    Whitespace, WordPiece, [CLS]/[SEP]): ids committed from HF `tokenizers`
    by tests/golden/make_token_golden.py; the file is re-read from the
    reference checkout when present."""
    if not REF_TOKENIZER or not os.path.exists(REF_TOKENIZER):
        pytest.skip("reference checkout not present")
    from jammi_b200 import Tokenizer
    g = json.load(open(GOLDEN, encoding="utf-8"))
    ours = Tokenizer(REF_TOKENIZER)
    got = [list(map(int, r)) for r in ours(g["texts"])]
    assert got == g["ids"]
    for max_len in (4, 9):
        got = [list(map(int, r)) for r in ours(g["texts"], max_length=max_len)]
        assert got == g[f"ids_max{max_len}"]


def test_unsupported_components_still_fail_loudly(tmp_path):
    from jammi_b200 import Tokenizer
    from jammi_b200._lib import JbError
    base = {"model": {"type": "WordPiece", "vocab": {"[UNK]": 0, "a": 1}, "unk_token": "[UNK]"}}
    for extra in ({"normalizer": {"type": "ByteLevel"}},
                  {"normalizer": {"type": "Replace", "pattern": {"Regex": "a+"}, "content": "b"}},
                  {"pre_tokenizer": {"type": "CharDelimiterSplit", "delimiter": "_"}},
                  {"pre_tokenizer": {"type": "Punctuation", "behavior": "Sideways"}}):
        path = tmp_path / "bad.json"
        path.write_text(json.dumps({**base, **extra}))
        with pytest.raises(JbError):
            Tokenizer(str(path))


REF_CLIP_TOKENIZER = reference_path("tests", "fixtures", "tiny_open_clip", "tokenizer.json")
CLIP_PATTERN = r"'s|'t|'re|'ve|'m|'ll|'d|[\p{L}]+|[\p{N}]|[^\s\p{L}\p{N}]+"


def test_reference_open_clip_fixture_tokenizer_golden_ids():
    """The reference's tiny OpenCLIP fixture tokenizer (WordLevel with '<pad>'
    as the unknown token, Split on the empty string inverted -- one word per
    character -- and '$A <|endoftext|>'): ids committed from HF `tokenizers`."""
    if not REF_CLIP_TOKENIZER or not os.path.exists(REF_CLIP_TOKENIZER):
        pytest.skip("reference checkout not present")
    from jammi_b200 import Tokenizer
    g = json.load(open(GOLDEN, encoding="utf-8"))
    got = [list(map(int, r)) for r in Tokenizer(REF_CLIP_TOKENIZER)(g["texts"])]
    assert got == g["clip_ids"]


def test_hf_format_clip_tokenizer(tmp_path):
    """CLIP's tokenizer.json as HF hubs ship it: NFC, whitespace runs -> ' ',
    Lowercase; Split on the CLIP regex (removed, inverted) then ByteLevel
    without its regex; BPE with '</w>' word ends; RobertaProcessing."""
    from tokenizers import Regex, Tokenizer, models, normalizers, pre_tokenizers, processors, trainers
    tok = Tokenizer(models.BPE(unk_token="<|endoftext|>", end_of_word_suffix="</w>"))
    tok.normalizer = normalizers.Sequence([normalizers.NFC(), normalizers.Replace(Regex(r"\s+"), " "),
                                           normalizers.Lowercase()])
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(CLIP_PATTERN), behavior="removed", invert=True),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    trainer = trainers.BpeTrainer(vocab_size=1200, special_tokens=["<|startoftext|>", "<|endoftext|>"],
                                  end_of_word_suffix="</w>", show_progress=False,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet())
    tok.train_from_iterator(random_texts(1, 2000, 40) + ["a photo of a cat"] * 5, trainer=trainer)
    tok.post_processor = processors.RobertaProcessing(("<|endoftext|>", 1), ("<|startoftext|>", 0))
    path = tmp_path / "clip.json"
    tok.save(str(path))
    _same(str(path), tok, EXTRA + random_texts(5, 300))


@pytest.mark.parametrize("pattern,behavior,invert", [
    ("-", "isolated", False), ("-", "removed", False), ("-", "merged_with_previous", False),
    ("-", "merged_with_next", False), ("-", "contiguous", False), ("ab", "isolated", True),
    ("", "isolated", True), ("", "removed", False), ("", "contiguous", True),
    ("regex:\\s+", "removed", False), ("regex:\\s+", "merged_with_next", False),
    ("regex:gpt2", "isolated", False), ("regex:clip", "removed", True),
])
def test_split_pre_tokenizer(tmp_path, pattern, behavior, invert):
    from tokenizers import Regex, Tokenizer, models, pre_tokenizers
    if pattern == "regex:gpt2":
        pat = Regex(r"'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+")
    elif pattern == "regex:clip":
        pat = Regex(CLIP_PATTERN)
    elif pattern.startswith("regex:"):
        pat = Regex(pattern[6:])
    else:
        pat = pattern
    tok = Tokenizer(models.WordPiece(unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Split(pat, behavior=behavior, invert=invert)
    hf, path = _train(tok, "wordpiece", tmp_path, "tok.json")
    _same(path, hf, EXTRA + ["a-b--c-", "-x-", "abab-ab", "  a  b  "] + random_texts(6, 200))


def test_word_level(tmp_path):
    from tokenizers import Tokenizer, models, pre_tokenizers, trainers
    tok = Tokenizer(models.WordLevel(unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.train_from_iterator(random_texts(1, 500, 30),
                            trainer=trainers.WordLevelTrainer(vocab_size=300, special_tokens=["[UNK]"]))
    path = tmp_path / "wl.json"
    tok.save(str(path))
    _same(str(path), tok, EXTRA + random_texts(7, 200))


def test_word_level_without_unknown_token_fails_on_every_thread_count(tmp_path):
    """A word outside a WordLevel vocabulary without an unknown token is an
    error (the crate's "Missing [UNK] token"), raised from the tokenizing
    threads as a status, for one text and for a batch split across cores."""
    from jammi_b200 import Tokenizer
    from jammi_b200._lib import JbError
    path = tmp_path / "wl.json"
    path.write_text(json.dumps({"model": {"type": "WordLevel", "vocab": {"a": 0, "b": 1}, "unk_token": "[UNK]"},
                                "pre_tokenizer": {"type": "WhitespaceSplit"}}))
    tok = Tokenizer(str(path))
    assert [list(map(int, r)) for r in tok(["a b a"])] == [[0, 1, 0]]
    for texts in (["a c"], ["a b"] * 600 + ["zzz"]):
        with pytest.raises(JbError, match="WordLevel"):
            tok(texts)
