"""sentencepiece-style tokenizer.json files -- the XLM-RoBERTa / CamemBERT
layout the reference's BERT family loads (crates/jammi-encoders/src/bert.rs:1,
model types xlm-roberta and camembert): the Precompiled normaliser (the
sentencepiece character map over grapheme clusters), Strip, Replace(' {2,}'),
the Metaspace pre-tokeniser and the Unigram model -- against HuggingFace
`tokenizers`, id for id.  The files come from a sentencepiece model trained
here on seeded synthetic text with the nmt_nfkc rule, converted by
`transformers`' XLM-RoBERTa converter.  CPU only."""
import json

import pytest

tokenizers = pytest.importorskip("tokenizers")
spm = pytest.importorskip("sentencepiece")
pytest.importorskip("transformers")

from test_tokenizer import random_texts  # noqa: E402

CASES = [
    "Hello  World", "", " ", "   lead and trail   ", "naïve café Ünïcödé", "é ä́ x̣̂",
    "ｆｕｌｌｗｉｄｔｈ ① ② ㍻ ﬁ ¼", "tab\there\r\nCRLF", "東京の数据 GPU!", "😀 👍🏽 🇺🇸 emoji",
    "क्षत्रिय नमस्ते", "한국어 문장", "ΣΑΣ σας", "<s> </s> <unk> <pad>", "reading played unplayable", "a" * 50,
    "\u0000\u0007 ctrl", "​ zero‍width", "ﷺ ﷽", "Å Å Å",
]


@pytest.fixture(scope="module")
def converted(tmp_path_factory):
    from transformers import XLMRobertaTokenizer
    from transformers.convert_slow_tokenizer import convert_slow_tokenizer
    d = tmp_path_factory.mktemp("spm")
    texts = random_texts(1, 3000, 60) + ["reading played unplayable café naïve ｆｕｌｌ ① ㍻ ﬁ Å"] * 20
    (d / "corpus.txt").write_text("\n".join(t.replace("\n", " ") for t in texts), encoding="utf-8")
    spm.SentencePieceTrainer.train(input=str(d / "corpus.txt"), model_prefix=str(d / "m"), vocab_size=800,
                                   model_type="unigram", normalization_rule_name="nmt_nfkc",
                                   character_coverage=0.9995, minloglevel=2)
    fast = convert_slow_tokenizer(XLMRobertaTokenizer(vocab_file=str(d / "m.model")))
    path = d / "xlmr.json"
    fast.save(str(path))
    return d, json.loads(path.read_text(encoding="utf-8"))


def _check(d, doc, name, texts):
    from jammi_b200 import Tokenizer
    path = d / name
    path.write_text(json.dumps(doc), encoding="utf-8")
    hf = tokenizers.Tokenizer.from_file(str(path))
    got = Tokenizer(str(path))(texts)
    bad = [(t, hf.encode(t).ids, list(g)) for t, g in zip(texts, got) if hf.encode(t).ids != list(g)]
    assert not bad, bad[:3]


def test_xlm_roberta_layout(converted):
    d, doc = converted
    assert doc["model"]["type"] == "Unigram"
    assert [n["type"] for n in doc["normalizer"]["normalizers"]][0] == "Precompiled"
    _check(d, doc, "a.json", CASES + random_texts(7, 500))


@pytest.mark.parametrize("scheme,split", [("first", True), ("never", True), ("always", False), ("first", False)])
def test_metaspace_variants(converted, scheme, split):
    d, doc = converted
    doc = json.loads(json.dumps(doc))
    doc["pre_tokenizer"]["prepend_scheme"] = scheme
    doc["pre_tokenizer"]["split"] = split
    _check(d, doc, f"m_{scheme}_{split}.json", CASES + ["<s>x", " <s> y", "z</s>"] + random_texts(8, 200))


def test_legacy_layout_whitespace_split_then_metaspace(converted):
    """Older converted files: Replace(' {2,}', ' ') and WhitespaceSplit +
    Metaspace(add_prefix_space) instead of the prepend scheme."""
    d, doc = converted
    doc = json.loads(json.dumps(doc))
    doc["normalizer"]["normalizers"] = [doc["normalizer"]["normalizers"][0],
                                        {"type": "Replace", "pattern": {"Regex": " {2,}"}, "content": " "}]
    doc["pre_tokenizer"] = {"type": "Sequence", "pretokenizers": [
        {"type": "WhitespaceSplit"}, {"type": "Metaspace", "replacement": "▁", "add_prefix_space": True}]}
    _check(d, doc, "legacy.json", CASES + random_texts(9, 200))


@pytest.mark.parametrize("fallback", [True, False])
def test_unknown_runs_and_byte_fallback(converted, fallback):
    """Characters without a piece fuse into one unknown run, which maps to
    the unknown id or, with byte_fallback, to <0xXX> tokens."""
    d, doc = converted
    doc = json.loads(json.dumps(doc))
    vocab = doc["model"]["vocab"]
    if fallback:
        vocab.extend([[f"<0x{b:02X}>", -50.0] for b in range(256)])
    doc["model"]["byte_fallback"] = fallback
    _check(d, doc, f"bf_{fallback}.json", CASES + ["東京東京 x 数据", "😀😀 a 😀"] + random_texts(10, 200))
