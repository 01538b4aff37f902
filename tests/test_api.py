"""HTTP surfaces on CPU with the tiny model: native NDJSON generate, OpenAI completions and
chat (plain and SSE), Anthropic messages, health/models/metrics, error shapes."""
import json

import pytest
import torch

pytest.importorskip("fastapi")
from fastapi.testclient import TestClient  # noqa: E402

from syntropy_b200.api import build_app  # noqa: E402
from syntropy_b200.models.config import get_config  # noqa: E402
from syntropy_b200.models.transformer import prepare_weights  # noqa: E402
from syntropy_b200.runtime.async_engine import AsyncEngine  # noqa: E402
from syntropy_b200.runtime.engine import LLMEngine  # noqa: E402
from syntropy_b200.runtime.runner import ModelRunner  # noqa: E402
from syntropy_b200.text.tokenizer import ByteTokenizer  # noqa: E402


@pytest.fixture(scope="module")
def client():
    cfg = get_config("tiny-llama")
    mw = prepare_weights(cfg, "cpu", seed=0)
    aeng = AsyncEngine(LLMEngine(ModelRunner(mw, max_batch=4, max_seq_len=256)))
    app = build_app(aeng, ByteTokenizer(cfg.vocab), model_id="tiny")
    with TestClient(app) as c:
        yield c
    aeng.close()


def test_health_models_version(client):
    assert client.get("/healthz").json()["status"] == "ok"
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
    assert "version" in client.get("/v1/syntropy/version").json()


def test_native_generate_ndjson(client):
    r = client.post("/v1/syntropy/generate", json={"model": "tiny", "tokens": [5, 6, 7, 8],
                                                   "sampling": {"max_tokens": 5}, "return_tokens": True})
    lines = [json.loads(x) for x in r.text.strip().splitlines()]
    assert lines[0]["event"] == "started" and lines[-1]["event"] == "done"
    toks = [t for x in lines if x["event"] == "text" for t in x["tokens"]]
    assert len(toks) == 5 and lines[-1]["usage"]["completion_tokens"] == 5
    assert [x["id"].split(":")[1] for x in lines] == [str(i) for i in range(len(lines))]


def test_native_generate_range_check(client):
    r = client.post("/v1/syntropy/generate", json={"model": "tiny", "tokens": [1, 99999]})
    assert r.status_code == 400 and r.json()["error"]["type"] == "token_id_out_of_range"
    r = client.post("/v1/syntropy/generate", json={"model": "tiny", "tokens": [1], "bogus": 1})
    assert r.status_code == 400


def test_openai_completions_and_chat(client):
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": "hello", "max_tokens": 4, "temperature": 0})
    j = r.json()
    assert j["object"] == "text_completion" and j["usage"]["completion_tokens"] == 4
    r = client.post("/v1/chat/completions", json={"model": "tiny", "messages": [{"role": "user", "content": "hi"}],
                                                  "max_tokens": 3, "temperature": 0})
    j = r.json()
    assert j["choices"][0]["message"]["role"] == "assistant" and j["usage"]["completion_tokens"] == 3
    r = client.post("/v1/chat/completions", json={"model": "tiny", "messages": [{"role": "user", "content": "hi"}],
                                                  "max_tokens": 3, "stream": True, "temperature": 0.7, "seed": 1})
    events = [x for x in r.text.split("\n\n") if x.startswith("data: ")]
    assert events[-1] == "data: [DONE]"
    assert json.loads(events[-2][6:])["choices"][0]["finish_reason"] == "length"


def test_anthropic_messages(client):
    r = client.post("/v1/messages", json={"model": "tiny", "max_tokens": 3,
                                          "messages": [{"role": "user", "content": "hi"}]})
    j = r.json()
    assert j["type"] == "message" and j["usage"]["output_tokens"] == 3 and j["stop_reason"] == "max_tokens"
    r = client.post("/v1/messages", json={"model": "tiny", "messages": [{"role": "user", "content": "x"}]})
    assert r.status_code == 400
    r = client.post("/v1/messages", json={"model": "tiny", "max_tokens": 2, "stream": True,
                                          "messages": [{"role": "user", "content": "hi"}]})
    kinds = [x.split("\n")[0] for x in r.text.strip().split("\n\n")]
    assert kinds[0] == "event: message_start" and kinds[-1] == "event: message_stop"


def test_metrics_exposed(client):
    client.post("/v1/completions", json={"model": "tiny", "prompt": [1, 2, 3], "max_tokens": 2})
    m = client.get("/metrics").text
    assert "syntropy_requests_total" in m and "syntropy_generated_tokens_total" in m
    # engine state after each step, as gauges
    for g in ("running_sequences", "waiting_sequences", "kv_pages_free", "kv_swapped_out_total",
              "kv_host_swap_bytes"):
        assert f"# TYPE syntropy_{g} gauge" in m, g


def test_constrained_requests(client):
    """OpenAI guided_choice and response_format json_object; native constraint field."""
    r = client.post("/v1/completions", json={"model": "tiny", "prompt": "answer:", "max_tokens": 8,
                                             "temperature": 0, "guided_choice": ["red", "green"]})
    assert r.status_code == 200, r.text
    assert r.json()["choices"][0]["text"] in ("red", "green")
    r = client.post("/v1/chat/completions", json={"model": "tiny", "max_tokens": 12, "temperature": 0,
                                                  "response_format": {"type": "json_object"},
                                                  "messages": [{"role": "user", "content": "json please"}]})
    assert r.status_code == 200, r.text
    text = r.json()["choices"][0]["message"]["content"]
    assert text.lstrip().startswith("{")
    r = client.post("/v1/syntropy/generate", json={"prompt": "x", "sampling": {"max_tokens": 6},
                                                   "constraint": {"choices": ["ab", "cd"]}})
    assert r.status_code == 200, r.text


def test_openai_logprobs(client):
    """Chat `logprobs` / `top_logprobs` and completions `logprobs: n`: one record per emitted
    token; greedy tokens are their own top alternative; log-probabilities are <= 0."""
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4,
                                                  "temperature": 0, "logprobs": True, "top_logprobs": 2,
                                                  "ignore_eos": True}).json()
    content = r["choices"][0]["logprobs"]["content"]
    assert len(content) == r["usage"]["completion_tokens"] == 4
    for c in content:
        assert c["logprob"] <= 0 and len(c["top_logprobs"]) == 2
        assert c["top_logprobs"][0]["token"] == c["token"]
        assert abs(c["top_logprobs"][0]["logprob"] - c["logprob"]) < 1e-6
    r = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 3, "temperature": 0, "logprobs": 1,
                                             "ignore_eos": True}).json()
    lp = r["choices"][0]["logprobs"]
    assert len(lp["tokens"]) == len(lp["token_logprobs"]) == len(lp["top_logprobs"]) == 3
    r = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 2, "temperature": 0}).json()
    assert "logprobs" not in r["choices"][0]


def test_oversized_logprobs_rejected_and_server_keeps_serving(client):
    """A logprobs count beyond the cap (20) or the vocabulary is a 400 for that request only;
    the engine keeps serving the next one."""
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 2,
                                                  "logprobs": True, "top_logprobs": 5000})
    assert r.status_code == 400, r.text
    r = client.post("/v1/completions", json={"prompt": "abc", "max_tokens": 2, "logprobs": 21})
    assert r.status_code == 400, r.text
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 3,
                                                  "temperature": 0, "ignore_eos": True, "logprobs": True,
                                                  "top_logprobs": 20})
    assert r.status_code == 200, r.text
    assert all(len(c["top_logprobs"]) == 20 for c in r.json()["choices"][0]["logprobs"]["content"])


def test_streamed_logprobs(client):
    """With stream=true every token chunk carries its logprobs record."""
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 3,
                                                  "temperature": 0, "logprobs": True, "top_logprobs": 1,
                                                  "ignore_eos": True, "stream": True})
    assert r.status_code == 200
    chunks = [json.loads(line[6:]) for line in r.text.splitlines() if line.startswith("data: {")]
    recs = [c["choices"][0]["logprobs"]["content"] for c in chunks if "logprobs" in c["choices"][0]]
    assert sum(len(x) for x in recs) == 3
    for x in recs:
        for c in x:
            assert c["logprob"] <= 0 and c["top_logprobs"][0]["token"] == c["token"]
