"""Table tests of the Anthropic <-> OpenAI translation: tool choices,
content blocks (thinking skipped, tool results with errors, mixed text and
tool results), sampling and metadata passthrough, finish-reason mapping,
responses with bad tool arguments or no content."""

import json

import pytest

from infera_b200.api.anthropic import (TranslationError, anthropic_to_openai_request, map_finish_reason,
                                       openai_to_anthropic_response)


def _req(messages, **kw):
    return anthropic_to_openai_request({"model": "m", "max_tokens": 16, "messages": messages, **kw})


@pytest.mark.parametrize("tc,want", [
    ("auto", "auto"), ({"type": "auto"}, "auto"), ({"type": "any"}, "required"), ({"type": "none"}, "none"),
    ({"type": "tool", "name": "f"}, {"type": "function", "function": {"name": "f"}}),
])
def test_tool_choice_mapping(tc, want):
    out = _req([{"role": "user", "content": "x"}], tool_choice=tc,
               tools=[{"name": "f", "input_schema": {"type": "object"}}])
    assert out["tool_choice"] == want


@pytest.mark.parametrize("tc", [{"type": "tool"}, {"type": "bogus"}])
def test_bad_tool_choice_rejected(tc):
    with pytest.raises(TranslationError):
        _req([{"role": "user", "content": "x"}], tool_choice=tc)


def test_tool_without_schema_gets_an_empty_object_schema():
    out = _req([{"role": "user", "content": "x"}], tools=[{"name": "g"}])
    assert out["tools"][0]["function"] == {"name": "g", "parameters": {"type": "object", "properties": {}}}


def test_content_blocks():
    out = _req([
        {"role": "user", "content": [{"type": "text", "text": "a"}, {"type": "text", "text": "b"}]},
        {"role": "assistant", "content": [{"type": "thinking", "thinking": "hmm"}, {"type": "text", "text": "ok"}]},
        {"role": "user", "content": [{"type": "text", "text": "before "},
                                     {"type": "tool_result", "tool_use_id": "t9", "is_error": True,
                                      "content": [{"type": "text", "text": "boom"}]}]},
    ])
    assert out["messages"][0] == {"role": "user", "content": "ab"}
    assert out["messages"][1] == {"role": "assistant", "content": "ok"}       # thinking dropped
    assert out["messages"][2] == {"role": "user", "content": "before "}
    assert out["messages"][3] == {"role": "tool", "tool_call_id": "t9", "content": "[error] boom"}


@pytest.mark.parametrize("messages", [
    [{"role": "user", "content": [{"type": "tool_use", "id": "x", "name": "f", "input": {}}]}],   # wrong role
    [{"role": "user", "content": [{"type": "video"}]}],
    [{"role": "user", "content": 42}],
    [{"role": "robot", "content": "hi"}],
])
def test_invalid_messages_rejected(messages):
    with pytest.raises(TranslationError):
        _req(messages)


def test_sampling_stream_and_metadata_passthrough():
    out = _req([{"role": "user", "content": "x"}], temperature=0.3, top_p=0.9, top_k=20, stream=True,
               metadata={"user_id": "u-1"}, stop_sequences=["\n\n", "END"])
    assert (out["temperature"], out["top_p"], out["top_k"]) == (0.3, 0.9, 20)
    assert out["stream"] and out["stream_options"] == {"include_usage": True}
    assert out["user"] == "u-1" and out["stop"] == ["\n\n", "END"] and out["max_tokens"] == 16


@pytest.mark.parametrize("finish,want", [("stop", "end_turn"), ("length", "max_tokens"), ("tool_calls", "tool_use"),
                                         ("content_filter", "end_turn"), (None, None), ("weird", "end_turn")])
def test_finish_reason_mapping(finish, want):
    assert map_finish_reason(finish) == want


def test_response_edge_cases():
    r = openai_to_anthropic_response({"model": "m", "choices": [{"message": {"content": None, "tool_calls": [
        {"id": "c", "function": {"name": "f", "arguments": "not json"}}]}, "finish_reason": "tool_calls"}]})
    assert r["content"] == [{"type": "tool_use", "id": "c", "name": "f", "input": {"_raw": "not json"}}]
    r = openai_to_anthropic_response({"choices": [{"message": {}, "finish_reason": "stop"}]}, model="mm")
    assert r["content"] == [{"type": "text", "text": ""}] and r["model"] == "mm"
    assert r["usage"] == {"input_tokens": 0, "output_tokens": 0}
    r = openai_to_anthropic_response({"choices": [{"message": {"content": "x"}, "finish_reason": "stop",
                                                   "stop_reason": "END"}]})
    assert r["stop_reason"] == "stop_sequence" and r["stop_sequence"] == "END"
    assert json.loads(json.dumps(r)) == r
