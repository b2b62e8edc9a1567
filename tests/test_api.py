"""HTTP API on a tiny CPU model: OpenAI routes, SSE, tools, auth, validation, ops routes."""
import json
import os

import pytest
from fastapi.testclient import TestClient

from vramancer_b200.pipeline import InferencePipeline
from vramancer_b200.serving.api import create_app
from vramancer_b200.serving.security import sign_request


@pytest.fixture(scope="module")
def client():
    os.environ["VRM_API_TOKEN"] = "testtoken"
    os.environ["VRM_DISABLE_RATE_LIMIT"] = "1"
    pipe = InferencePipeline(enable_metrics=True).load("tiny-qwen2", device="cpu", max_model_len=256, max_batch=4)
    app = create_app(pipe)
    with TestClient(app) as c:
        c.headers.update({"Authorization": "Bearer testtoken"})
        yield c
    pipe.shutdown()


def test_public_ops(client):
    assert client.get("/health").json()["model_loaded"] is True
    assert client.get("/ready").status_code == 200
    assert client.get("/live").json()["live"] is True
    assert "vrm_" in client.get("/metrics").text
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny-qwen2"


def test_auth_required(client):
    r = client.post("/v1/completions", json={"prompt": "hi"}, headers={"Authorization": "Bearer nope"})
    assert r.status_code == 401


def test_completion_and_usage(client):
    r = client.post("/v1/completions", json={"prompt": "hello world", "max_tokens": 5})
    j = r.json()
    assert r.status_code == 200, j
    assert j["usage"]["completion_tokens"] == 5
    assert j["choices"][0]["finish_reason"] in ("length", "stop")


def test_chat_and_stream(client):
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4})
    assert r.status_code == 200
    assert r.json()["choices"][0]["message"]["role"] == "assistant"
    with client.stream("POST", "/v1/chat/completions",
                       json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4,
                             "stream": True}) as s:
        lines = [l for l in s.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    assert json.loads(lines[0][6:])["object"] == "chat.completion.chunk"


def test_validation_and_context(client):
    assert client.post("/v1/completions", json={"prompt": "x", "max_tokens": 0}).status_code == 400
    assert client.post("/v1/completions", json={"prompt": "x", "temperature": 9}).status_code == 400
    r = client.post("/v1/completions", json={"prompt": "x" * 400, "max_tokens": 4})
    assert r.status_code == 400 and r.json()["error"]["code"] == "context_length_exceeded"


def test_batch_infer_status(client):
    r = client.post("/v1/batch/completions", json={"prompts": ["a", "b", "c"], "max_tokens": 3})
    assert len(r.json()["choices"]) == 3
    r = client.post("/api/infer", json={"input_ids": [1, 2, 3, 4], "top": 5})
    assert len(r.json()["top"]) == 5
    st = client.get("/api/status").json()
    assert st["loaded"] and st["engine"]["finished"] >= 4
    assert "kv" in client.get("/api/batcher/stats").json()
    assert client.get("/api/history").json()["requests"]


def test_tool_calls_parsing():
    from vramancer_b200.serving.tool_calls import build_chat_message, build_chat_prompt, detect_tool_loop
    msg, fin = build_chat_message('<think>x</think><tool_call>{"name": "f", "arguments": {"a": 1},}</tool_call>')
    assert fin == "tool_calls" and msg["tool_calls"][0]["function"]["name"] == "f"
    p = build_chat_prompt([{"role": "user", "content": "q"}], tools=[{"type": "function",
                                                                     "function": {"name": "f"}}])
    assert "<tools>" in p and p.endswith("<|im_start|>assistant\n")
    h = [{"tool_calls": [{"function": {"name": "f", "arguments": "{}"}}]}] * 3
    assert detect_tool_loop(h)


def test_hmac_signing():
    from vramancer_b200.serving.security import verify_signature
    ts, sig = sign_request("s3", "POST", "/v1/completions", b"{}")
    assert verify_signature("s3", "POST", "/v1/completions", b"{}", ts, sig)
    assert not verify_signature("s3", "POST", "/v1/completions", b"{1}", ts, sig)


def test_stop_strings_and_n(client):
    """OpenAI `stop` (text cut before the first stop string, finish_reason "stop") and
    `n` independent choices; streaming ends before a stop string too."""
    base = client.post("/v1/completions", json={"prompt": "hello world", "max_tokens": 12}).json()
    full = base["choices"][0]["text"]
    assert len(full) > 4
    stop = full[2:4]
    r = client.post("/v1/completions", json={"prompt": "hello world", "max_tokens": 12, "stop": [stop]}).json()
    c = r["choices"][0]
    assert c["finish_reason"] == "stop" and stop not in c["text"] and full.startswith(c["text"])
    r = client.post("/v1/completions", json={"prompt": "hello world", "max_tokens": 6, "n": 3,
                                              "temperature": 0.9}).json()
    assert [c["index"] for c in r["choices"]] == [0, 1, 2]
    assert 3 <= r["usage"]["completion_tokens"] <= 18
    body = {"prompt": "hello world", "max_tokens": 12, "stream": True, "stop": stop}
    with client.stream("POST", "/v1/completions", json=body) as s:
        text = "".join(json.loads(line[6:])["choices"][0]["text"] for line in s.iter_lines()
                       if line.startswith("data: {"))
    assert stop not in text and full.startswith(text)
    assert client.post("/v1/completions", json={"prompt": "x", "stop": ["a"] * 5}).status_code == 400
    assert client.post("/v1/completions", json={"prompt": "x", "n": 9}).status_code == 400
    assert client.post("/v1/completions", json={"prompt": "x", "n": 2, "stream": True}).status_code == 400
    chat = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                     "max_tokens": 5, "n": 2}).json()
    assert len(chat["choices"]) == 2
