"""Decision-endpoint helpers (native decider_prepare / decider_answer): prompts keep option order and
render like Python's json.dumps(ensure_ascii=False); answers mask extra readout rows, apply the
temperature once and reduce to choice / score / yes-no answers with confidences."""
import json
import math

import pytest

from vllm_suffix_hybrid_b200 import _native

BODY = {"model": "decider", "state": {"z": "Grüße", "a": [1, 0.000001]},
        "questions": {"route": {"type": "choice", "criteria": {"second": "billing", "first": None}},
                      "truth": {"type": "noul"},
                      "severity": {"type": "score", "criteria": ["low", "mid", "high"]}}}
BODY_S = json.dumps(BODY, ensure_ascii=False)


def test_prompt_order_unicode_and_python_spacing():
    out = json.loads(_native.decider_prepare(BODY_S, json.dumps(["A", "B", "C"]), "pplx"))
    text = out["rows"][0]["messages"][1]["content"][0]["text"]
    assert "State:\n" + json.dumps(BODY["state"], ensure_ascii=False) in text
    assert 'State:\n{"z": "Grüße", "a": [1, 1e-06]}' in text
    assert "Options:\nA: second: billing\nB: first" in text
    assert out["identifiers"] == ["route", "truth", "severity"]
    assert [r["option_count"] for r in out["rows"]] == [2, 2, 3]
    assert out["rows"][1]["messages"][1]["content"][0]["text"].endswith(
        "A: No / false\nB: Yes / true\n\nReturn only the letter code of the best option.")


@pytest.mark.parametrize("v", [1e-06, 1.5e-07, 0.0001, 123.25, 1e15, 1e16, 2.5e+20, -3.0, 0.1 + 0.2])
def test_floats_render_like_python(v):
    body = {"model": "m", "state": {"x": v}, "questions": {"q": {"type": "noul"}}}
    text = json.loads(_native.decider_prepare(json.dumps(body), '["A","B"]', "pplx"))["rows"][0]["messages"][1][
        "content"][0]["text"]
    assert 'State:\n{"x": ' + repr(v) + "}" in text


def test_answers_mask_extra_rows_and_apply_temperature_once():
    r = json.loads(_native.decider_answer(BODY_S, json.dumps([[0, 2, 9999], [0, 0, 9999], [0, 0, 0, 9999]]), 2.0,
                                          "pplx"))
    assert r["answers"]["route"]["choice"] == "first"
    assert abs(r["answers"]["route"]["probabilities"]["first"] - 1.0 / (1.0 + math.exp(-1.0))) < 1e-12
    assert r["answers"]["truth"]["noul"] == 0.5
    assert r["answers"]["severity"]["score"] == 1.0
    assert r["model"] == "decider" and list(r["answers"]) == ["route", "truth", "severity"]


def test_d3_empty_state_media_and_entropy_confidence():
    body = {"model": "d3", "questions": {"s": {"type": "score", "criteria": [1, {"b": 2, "a": "x, y"}]},
                                         "c": {"type": "choice", "criteria": {"k": 3}}}}
    bs = json.dumps(body)
    prep = json.loads(_native.decider_prepare(bs, '["A","B"]', "d3"))
    assert prep["rows"][0]["messages"][0]["content"].startswith("You are a decision engine.")
    prompt = prep["rows"][0]["messages"][1]["content"]
    assert prompt.startswith("State:\n(empty)\n\nQuestion:\nChoose the best matching option.")
    assert prompt.endswith('Options:\nA: 1\nB: {"b": 2, "a": "x, y"}\n\nReply with only the code of the best option.')
    ans = json.loads(_native.decider_answer(bs, "[[0,0],[5]]", 1.0, "d3"))
    assert ans["answers"]["s"]["confidence"] == 0.0
    assert ans["answers"]["s"]["legend"]["1"] == '{"a":"x, y","b":2}'
    assert ans["answers"]["c"]["confidence"] == 1.0
    with pytest.raises(ValueError):
        _native.decider_prepare(bs, '["A","B"]', "pplx")
    media = json.dumps({"model": "d3", "state": "s", "images": ["a", "b"], "videos": ["v"],
                        "questions": {"q": {"type": "noul"}}})
    content = json.loads(_native.decider_prepare(media, '["A","B"]', "d3"))["rows"][0]["messages"][1]["content"]
    assert content[:3] == [{"type": "image"}, {"type": "image"}, {"type": "video"}]
    assert content[3]["text"].startswith("State:\ns\n")
    with pytest.raises(ValueError):
        _native.decider_prepare(media, '["A","B"]', "pplx")


def test_big_integers_keep_their_digits():
    body = '{"model":"decider","state":{"number":123456789012345678901234567890},"questions":{"q":{"type":"noul"}}}'
    text = json.loads(_native.decider_prepare(body, '["A","B"]', "pplx"))["rows"][0]["messages"][1]["content"][0][
        "text"]
    assert "123456789012345678901234567890" in text


def test_invalid_requests_fail_closed():
    with_images = dict(BODY, images=["x"])
    with pytest.raises(ValueError):
        _native.decider_prepare(json.dumps(with_images), '["A","B","C"]', "pplx")
    with pytest.raises(ValueError):
        _native.decider_answer(BODY_S, "[]", 1.0, "pplx")
    with pytest.raises(ValueError):
        _native.decider_answer(BODY_S, "[[0,1],[0,1],[0,1,2]]", float("nan"), "pplx")
    with pytest.raises(ValueError):
        _native.decider_prepare(BODY_S, '["A","A","B"]', "pplx")
    with pytest.raises(ValueError):
        _native.decider_prepare(BODY_S, '["A","B","C"]', "other")
    with pytest.raises(ValueError):
        _native.decider_prepare('{"model": "m", "state": "s", "questions": {"q": {"type": "rank"}}}', '["A"]')
