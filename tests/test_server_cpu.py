"""The OpenAI-compatible server (nanoquant_b200/server.py) without a GPU: a stand-in engine and
tokenizer behind the real app; endpoints, bearer-token check and request validation follow the
reference's server (src/nanoquant/openai_server.py:168-373)."""
import argparse

import pytest
import torch

from nanoquant_b200 import server

fastapi_testclient = pytest.importorskip("fastapi.testclient")


class Tok:
    eos_token_id = 0

    def apply_chat_template(self, messages, tokenize=True, add_generation_prompt=True, **kw):
        text = " ".join(m["content"] for m in messages)
        return [1 + (ord(c) % 200) for c in text]

    def decode(self, ids, skip_special_tokens=False):
        return "".join(chr(65 + i % 26) for i in ids)


class Engine:
    def __init__(self):
        self.calls = []

    def generate(self, ids, max_new, temperature, top_p, top_k, seed):
        self.calls.append((len(ids), max_new, temperature, top_p, top_k, seed))
        return list(range(3, 3 + max_new))


def client():
    args = argparse.Namespace(api_key="k", model_name="m", device="cuda:0", dtype="float16", max_tokens=16)
    eng = Engine()
    return fastapi_testclient.TestClient(server.create_app(args, engine=eng, tokenizer=Tok())), eng


def test_auth_models_health():
    c, _ = client()
    assert c.get("/v1/models").status_code == 401
    assert c.get("/v1/models", headers={"Authorization": "Bearer wrong"}).status_code == 401
    h = {"Authorization": "Bearer k"}
    assert c.get("/v1/models", headers=h).json()["data"][0]["id"] == "m"
    assert c.get("/health", headers=h).json()["status"] == "ok"


def test_chat_completion_and_validation():
    c, eng = client()
    h = {"Authorization": "Bearer k"}
    body = {"messages": [{"role": "user", "content": "hello"}], "max_tokens": 4, "temperature": 0, "seed": 3}
    r = c.post("/v1/chat/completions", headers=h, json=body)
    assert r.status_code == 200, r.text
    j = r.json()
    assert j["object"] == "chat.completion" and j["choices"][0]["finish_reason"] == "length"
    assert j["usage"] == {"prompt_tokens": 5, "completion_tokens": 4, "total_tokens": 9}
    assert eng.calls[-1] == (5, 4, 0.0, 0.95, 20, 3)
    for bad, msg in (({"stream": True}, "Streaming"), ({"n": 2}, "n=1"), ({"max_tokens": 0}, "max_tokens"),
                     ({"max_tokens": 17}, "max_tokens"), ({"stop": ["x"]}, "stop strings"),
                     ({"temperature": -1}, "temperature"), ({"top_p": 0}, "top_p"), ({"tools": 1}, "tools")):
        r = c.post("/v1/chat/completions", headers=h, json={**body, **bad})
        assert r.status_code == 400 and msg in r.json()["detail"], (bad, r.text)
    assert c.post("/v1/chat/completions", headers=h, json={"messages": []}).status_code == 400


def test_sample_respects_top_k_and_top_p():
    logits = torch.tensor([5.0, 4.0, 1.0, 0.0, -3.0])
    g = torch.Generator().manual_seed(0)
    assert {server.sample(logits, 1.0, 2, g) for _ in range(50)} <= {0, 1}
    assert {server.sample(logits, 0.5, 0, g) for _ in range(50)} == {0}
