"""The library's WordPiece tokenizer (jb_tokenizer_*) against HuggingFace
`tokenizers` -- the crate the reference tokenises with
(crates/jammi-ai/src/model/tokenizer.rs) -- id for id, on tokenizer.json files
built here from seeded synthetic text.  CPU only."""
import json

import numpy as np
import pytest

tokenizers = pytest.importorskip("tokenizers")

ALPHABET = (
    "abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789"
    "     .,;:!?'\"()[]{}-_/\\@#$%^&*+=<>|~`"
    "àáâäãåæçèéêëìíîïñòóôöõøùúûüýÿßÀÉÎÕÜŒœŁł"
    "αβγδεζηθΣσςΩΑΒ" "абвгдежзийклмнопрстЖЩЯ"
    "東京数据中文字符语言模型" "한국어문장" "ｆｕｌｌｗｉｄｔｈ"
    "̣́̈"          # combining marks
    "\t\n\r 　 "    # whitespace
    "\u0000\u0007​﻿"    # controls / format characters
    "😀🚀€£¥©®™…—–«»¿¡"
)


def random_texts(seed, n, max_len=60):
    rng = np.random.default_rng(seed)
    chars = list(ALPHABET)
    out = []
    for _ in range(n):
        k = int(rng.integers(0, max_len))
        out.append("".join(chars[i] for i in rng.integers(0, len(chars), size=k)))
    return out


def build(tmp_path, name, lowercase=True, strip_accents=None, processor="template"):
    from tokenizers import Tokenizer, models, normalizers, pre_tokenizers, processors, trainers
    tok = Tokenizer(models.WordPiece(unk_token="[UNK]", max_input_chars_per_word=40))
    tok.normalizer = normalizers.BertNormalizer(clean_text=True, handle_chinese_chars=True,
                                                strip_accents=strip_accents, lowercase=lowercase)
    tok.pre_tokenizer = pre_tokenizers.BertPreTokenizer()
    trainer = trainers.WordPieceTrainer(vocab_size=1500, special_tokens=[
        "[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"])
    tok.train_from_iterator(random_texts(1, 3000, 40) + ["reading played unplayable café naïve"] * 5,
                            trainer=trainer)
    cls, sep = tok.token_to_id("[CLS]"), tok.token_to_id("[SEP]")
    if processor == "template":
        tok.post_processor = processors.TemplateProcessing(
            single="[CLS] $A [SEP]", special_tokens=[("[CLS]", cls), ("[SEP]", sep)])
    elif processor == "bert":
        tok.post_processor = processors.BertProcessing(("[SEP]", sep), ("[CLS]", cls))
    path = tmp_path / name
    tok.save(str(path))
    return tok, str(path)


CASES = [
    "Hello World", "naïve café ÜBER Straße", "東京の数据 GPU!", "", "  spaces\t\ttabs\nnew  ",
    "unplayable reading,played.", "a" * 80, "[CLS] hello [SEP] [MASK]", "x\u0000y​z�",
    "Ǆ ǅ İstanbul ΣΑΣ ΌΣΟΣ", "한국어 문장입니다", "é ẹ́ ẹ́", "😀 emoji… — «quotes»",
]


@pytest.mark.parametrize("lowercase,strip_accents,processor", [
    (True, None, "template"), (False, None, "template"), (False, True, "bert"), (True, False, "bert"),
    (True, None, None),
])
def test_matches_hf_tokenizers(tmp_path, lowercase, strip_accents, processor):
    from jammi_b200 import Tokenizer
    hf, path = build(tmp_path, "tok.json", lowercase, strip_accents, processor)
    ours = Tokenizer(path)
    texts = CASES + random_texts(7, 400)
    got = ours(texts)
    bad = [(t, hf.encode(t).ids, list(g)) for t, g in zip(texts, got) if hf.encode(t).ids != list(g)]
    assert not bad, bad[:3]


def test_truncation_and_ragged_layout(tmp_path):
    """max_length counts [CLS] and [SEP] and cuts the sequence's tail (the
    reference's encode_batch with TruncationParams); the ragged output is the
    values / offsets layout of jb_generate_embeddings."""
    from jammi_b200 import Tokenizer
    hf, path = build(tmp_path, "tok.json")
    texts = random_texts(9, 50, 80)
    ours = Tokenizer(path)
    for max_len in (3, 8, 17):
        hf.enable_truncation(max_length=max_len)
        ids, offsets = ours.encode_ragged(texts, max_length=max_len)
        assert offsets[0] == 0 and offsets.size == len(texts) + 1 and ids.size == offsets[-1]
        for i, t in enumerate(texts):
            assert list(ids[offsets[i]:offsets[i + 1]]) == hf.encode(t).ids
            assert offsets[i + 1] - offsets[i] <= max_len


def test_many_texts_use_all_cores_in_order(tmp_path):
    from jammi_b200 import Tokenizer
    hf, path = build(tmp_path, "tok.json")
    texts = random_texts(11, 3000, 30)
    got = Tokenizer(path)(texts)
    assert [list(g) for g in got] == [e.ids for e in hf.encode_batch(texts)]


def test_unsupported_tokenizer_is_rejected(tmp_path):
    from jammi_b200 import Tokenizer
    from jammi_b200._lib import JbError
    for doc in ({"model": {"type": "SomethingElse", "vocab": [["a", 0.0]]}},
                {"model": {"type": "BPE", "vocab": {"a": 0}, "merges": []},
                 "pre_tokenizer": {"type": "UnicodeScripts"}},
                {"model": {"type": "BPE", "vocab": {"a": 0}, "merges": []},
                 "normalizer": {"type": "ByteLevel"}},
                {"model": {"type": "BPE", "vocab": {"a": 0}, "merges": ["a b"]}}):
        path = tmp_path / "bad.json"
        path.write_text(json.dumps(doc))
        with pytest.raises(JbError):
            Tokenizer(str(path))
    with pytest.raises(JbError):
        Tokenizer(str(tmp_path / "missing.json"))


def test_tokenize_rows_null_rows(tmp_path):
    """jb_tokenize_rows: None / empty texts are rows without tokens (the
    embedding path's null rows, candle.rs:779-806); the others are
    jb_tokenize's ids, truncated to max_length."""
    from jammi_b200 import Tokenizer
    hf, path = build(tmp_path, "tok.json")
    texts = ["hello world", "", None, "naïve café " * 20, "x"] + random_texts(12, 300)
    ours = Tokenizer(path)
    ids, offsets = ours.encode_ragged(texts, max_length=16, null_rows=True)
    hf.enable_truncation(max_length=16)
    for i, t in enumerate(texts):
        row = list(ids[offsets[i]:offsets[i + 1]])
        assert row == ([] if not t else hf.encode(t).ids)
