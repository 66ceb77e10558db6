"""Mid-stream migration bookkeeping (token-id continuation, text fallback
for chat and string prompts, poisoning, hop limit) and data-parallel rank
addressing (header, room alignment, route keys)."""

import json

from infera_b200.common.worker_pool import WorkerInfo
from infera_b200.router.dp_routing import (DP_RANK_HEADER, align_room_to_prefill_rank, disagg_prefill_dp_rank,
                                           dp_rank_header)
from infera_b200.router.migration import MigrationState, as_chat_chunk
from infera_b200.router.policy.target import RouteTarget, expand_targets
from infera_b200.router.token_ids import parse_sse_json, to_sse


def _ev(text, ids=None, finish=None, **extra):
    ch = {"index": 0, "text": text, "finish_reason": finish}
    if ids is not None:
        ch["token_ids"] = ids
    return to_sse({"id": "c", "created": 1, "model": "m", "choices": [ch], **extra})


def test_token_id_continuation_and_stripping():
    st = MigrationState({"prompt": [1, 2, 3], "max_tokens": 10, "stream": True}, limit=2, path="/v1/completions",
                        prompt_ids=[1, 2, 3])
    out = st.observe(_ev("a", [7]))
    assert "token_ids" not in json.dumps(parse_sse_json(out))        # ids never reach the client
    st.observe(_ev("b", [8, 9]))
    c = st.next_continuation()
    assert c.path == "/v1/completions" and c.body["prompt"] == [1, 2, 3, 7, 8, 9]
    assert c.body["max_tokens"] == 7 and c.body["return_token_ids"] and not c.reshape_to_chat
    assert st.can_migrate()
    st.next_continuation()
    assert not st.can_migrate()                                      # hop limit


def test_chat_text_fallback_and_finish():
    st = MigrationState({"messages": [{"role": "user", "content": "hi"}], "max_completion_tokens": 8,
                         "_infera_cache_hints": object()}, limit=3, path="/v1/chat/completions")
    st.observe(_ev("Hello wor"))                                     # text only: no ids
    c = st.next_continuation()
    assert c.body["messages"][-1] == {"role": "assistant", "content": "Hello wor"}
    assert c.body["continue_final_message"] and not c.body["add_generation_prompt"]
    assert "_infera_cache_hints" not in c.body and c.body["max_tokens"] >= 1
    st.observe(_ev("ld", finish="stop"))
    assert st.finished and not st.can_migrate()


def test_string_prompt_appends_text_and_token_list_without_ids_poisons():
    st = MigrationState({"prompt": "Once", "max_tokens": 4}, limit=3, path="/v1/completions")
    st.observe(_ev(" upon"))
    assert st.next_continuation().body["prompt"] == "Once upon"
    st2 = MigrationState({"prompt": [5, 6], "max_tokens": 4}, limit=3, path="/v1/completions")
    st2.prompt_ids = None
    st2.observe(_ev("x"))                                            # text without ids, no prompt ids
    st2.next_continuation()
    assert st2.poisoned and not st2.can_migrate()


def test_chat_chunk_reshape():
    obj = parse_sse_json(as_chat_chunk(_ev("tok", finish="length")))
    assert obj["object"] == "chat.completion.chunk"
    assert obj["choices"][0]["delta"] == {"content": "tok"} and obj["choices"][0]["finish_reason"] == "length"
    assert as_chat_chunk(b"data: [DONE]\n\n") == b"data: [DONE]\n\n"


def test_dp_rank_addressing():
    w = WorkerInfo(worker_id="w", url="http://w", model_name="m", dp_size=4)
    ts = expand_targets([w])
    assert [t.route_key for t in ts] == ["w#dp0", "w#dp1", "w#dp2", "w#dp3"]
    t2 = ts[2]
    assert dp_rank_header(t2) == {DP_RANK_HEADER: "2"} and disagg_prefill_dp_rank(t2) == 2
    for room in (0, 5, 17, 1000003):
        r = align_room_to_prefill_rank(room, t2)
        assert r % 4 == 2 and abs(r - room) < 4
    single = RouteTarget(WorkerInfo(worker_id="s", url="http://s", model_name="m"), None)
    assert dp_rank_header(single) == {} and align_room_to_prefill_rank(9, single) == 9
    assert disagg_prefill_dp_rank(single) is None
