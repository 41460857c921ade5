"""Pooling declared by a checkpoint (jb_pooling_from_config /
jb_pooling_from_model_dir) against the reference's own cases for
pooling_from_config (crates/jammi-ai/src/model/backend/candle.rs:2390-2470)
and read_local_pooling_config (crates/jammi-ai/src/model/resolver.rs:473-500).
CPU only."""
import json

import pytest


def _p():
    from jammi_b200.encoders import pooling_from_config, pooling_from_model_dir
    return pooling_from_config, pooling_from_model_dir


def test_absent_file_falls_back_to_mean(tmp_path):
    cfg, model_dir = _p()
    assert cfg(None) == "mean"
    assert model_dir(str(tmp_path)) == "mean"


@pytest.mark.parametrize("flags,want", [
    ({"pooling_mode_cls_token": True, "pooling_mode_mean_tokens": False}, "cls"),
    ({"pooling_mode_cls_token": False, "pooling_mode_mean_sqrt_len_tokens": True}, "mean"),
    ({"pooling_mode_mean_tokens": True, "pooling_mode_mean_sqrt_len_tokens": True}, "mean"),
    ({"pooling_mode_max_tokens": True, "word_embedding_dimension": 384}, "max"),
    ({"pooling_mode_weightedmean_tokens": True, "pooling_mode_cls_token": "true"}, "weighted_mean"),
])
def test_declared_strategy(flags, want):
    cfg, _ = _p()
    assert cfg(flags) == want
    assert cfg(json.dumps(flags)) == want


@pytest.mark.parametrize("bad,needle", [
    ({"pooling_mode_cls_token": False, "pooling_mode_lasttoken": True}, "pooling_mode_lasttoken"),
    ({"pooling_mode_cls_token": True, "pooling_mode_mean_tokens": True}, "distinct"),
    ({"pooling_mode_cls_token": False, "pooling_mode_mean_tokens": False}, "no true"),
    (["not", "an", "object"], "not a JSON object"),
    ("{not json", "unparseable"),
])
def test_declarations_that_fail_loudly(bad, needle):
    from jammi_b200._lib import JbError
    cfg, _ = _p()
    with pytest.raises(JbError) as e:
        cfg(bad if isinstance(bad, str) else json.dumps(bad))
    assert needle in str(e.value)


def test_model_dir_reads_the_declaration(tmp_path):
    from jammi_b200._lib import JbError
    _, model_dir = _p()
    (tmp_path / "1_Pooling").mkdir()
    f = tmp_path / "1_Pooling" / "config.json"
    f.write_text(json.dumps({"pooling_mode_cls_token": True}))
    assert model_dir(str(tmp_path)) == "cls"
    f.write_text('{"pooling_mode_cls_token": tr')  # truncated: a hard error, not mean
    with pytest.raises(JbError):
        model_dir(str(tmp_path))
