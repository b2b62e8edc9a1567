"""Cross-node worker routes of the HTTP API on CPU: tensors over JSON, two nodes' layer
ranges composed over /api/worker/forward_layers give the single model's logits,
/api/distributed/generate with a stage server generates the single model's tokens, and
/api/swarm/awaken sends Wake-on-LAN magic packets."""
import os
import socket

import pytest
import torch
from fastapi.testclient import TestClient

from vramancer_b200.cluster import worker_api
from vramancer_b200.cluster.stage_server import StageServer
from vramancer_b200.engine.engine import SamplingParams
from vramancer_b200.llm import LLM
from vramancer_b200.models.config import get_config
from vramancer_b200.serving.api import create_app


@pytest.fixture(scope="module")
def client():
    os.environ["VRM_API_TOKEN"] = "testtoken"
    os.environ["VRM_DISABLE_RATE_LIMIT"] = "1"
    app = create_app(None)
    with TestClient(app) as c:
        c.headers.update({"Authorization": "Bearer testtoken"})
        yield c
    app.state.node_worker.close()


def test_tensor_codec():
    for t in (torch.randn(3, 5), torch.randn(2, 4).bfloat16(), torch.arange(7, dtype=torch.int32)):
        assert torch.equal(worker_api.decode_tensor(worker_api.encode_tensor(t)), t)
    with pytest.raises(ValueError):
        worker_api.decode_tensor({"dtype": "float32", "shape": [4], "data": "AAAA"})


def test_forward_layers_compose_to_the_full_model(client):
    cfg = get_config("tiny-qwen2")
    ids = [5, 9, 2, 77, 31, 8]
    full = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", use_cuda_graph=False, max_batch=1,
               max_model_len=64, kv_pages=8, seed=4)
    from vramancer_b200.engine.runner import PrefillItem
    # the whole sequence in page 0 of the single model's pool
    item = PrefillItem(token_ids=ids, start_pos=0, slots=list(range(len(ids))), block_table=[0],
                       context_len=len(ids), want_logits=True)
    want = full.runner.prefill_logits([item])[-1].float()

    assert client.get("/api/worker/model_info").json() == {"loaded": False}
    split = cfg.num_layers // 2
    r = client.post("/api/worker/load_partial", json={"model": "tiny-qwen2", "start_layer": 0, "end_layer": split,
                                                      "seed": 4})
    assert r.status_code == 200 and r.json()["end_layer"] == split
    h = client.post("/api/worker/forward_layers", json={"input_ids": ids}).json()
    assert h["kind"] == "hidden"
    r = client.post("/api/worker/load_partial", json={"model": "tiny-qwen2", "start_layer": split, "seed": 4})
    assert r.json()["has_head"] is True
    out = client.post("/api/worker/forward_layers", json={"hidden": h["output"]}).json()
    assert out["kind"] == "logits"
    got = worker_api.decode_tensor(out["output"]).float()[-1]
    assert torch.allclose(got, want, atol=1e-4, rtol=1e-4)
    assert client.post("/api/worker/forward_layers", json={"hidden": {"dtype": "float32", "shape": [2, 3],
                                                                      "data": ""}}).status_code == 400


def test_distributed_generate_matches_single_model(client):
    cfg = get_config("tiny-qwen2")
    split = cfg.num_layers // 2
    prompts = [[3, 1, 4, 1, 5, 9, 2, 6], list(range(20, 45))]
    ref = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", use_cuda_graph=False, max_batch=4,
              max_model_len=128, kv_pages=64, seed=5)
    want = [o.output_ids for o in ref.generate(prompts, SamplingParams(max_tokens=6))]
    srv = StageServer(cfg, split, cfg.num_layers, port=0, num_pages=64, seed=5, key=b"k").start()
    try:
        r = client.post("/api/distributed/generate", json={
            "model": "tiny-qwen2", "prompts": prompts, "max_tokens": 6, "split": split, "seed": 5, "key": "k",
            "num_pages": 64, "workers": [{"host": "127.0.0.1", "port": srv.port}]})
        assert r.status_code == 200, r.text
        assert r.json()["outputs"] == want
        bad = client.post("/api/distributed/generate", json={
            "model": "tiny-qwen2", "prompts": prompts, "max_tokens": 2, "split": split - 1, "seed": 5, "key": "k",
            "workers": [{"host": "127.0.0.1", "port": srv.port}]})
        assert bad.status_code == 400
    finally:
        srv.close()


def test_swarm_awaken_sends_magic_packets(client):
    rx = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
    rx.bind(("127.0.0.1", 0))
    rx.settimeout(5)
    port = rx.getsockname()[1]
    r = client.post("/api/swarm/awaken", json={"macs": ["aa:bb:cc:dd:ee:01"], "broadcast": "127.0.0.1",
                                               "port": port})
    assert r.json() == {"sent": 1}
    data, _ = rx.recvfrom(256)
    rx.close()
    assert data == b"\xff" * 6 + bytes.fromhex("aabbccddee01") * 16
    assert client.post("/api/swarm/awaken", json={"macs": ["nope"]}).status_code == 400
