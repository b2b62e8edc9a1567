"""Backend factory and the non-native backends (CPU)."""
import json
import os
import threading
from http.server import BaseHTTPRequestHandler, HTTPServer

import pytest
import torch

from vramancer_b200.backends import (HuggingFaceBackend, LlamaCppBackend, NativeBackend, OllamaBackend,
                                     select_backend)


def test_auto_selection(tmp_path):
    assert isinstance(select_backend("tiny-qwen2"), NativeBackend)
    assert isinstance(select_backend("model.Q4_K_M.gguf"), LlamaCppBackend)
    d = tmp_path / "neox"
    d.mkdir()
    (d / "config.json").write_text(json.dumps({"model_type": "gpt_neox_unknown_arch"}))
    assert isinstance(select_backend(str(d)), HuggingFaceBackend)
    with pytest.raises(ValueError):
        select_backend("x", backend="nope")


def test_native_backend_generates_cpu():
    be = select_backend("tiny-qwen2", backend="native").load_model("tiny-qwen2", device="cpu", max_batch=2,
                                                                    max_model_len=64, kv_pages=32)
    try:
        ids = be.generate_ids([1, 2, 3], max_new_tokens=4)
        assert len(ids) == 4
        assert be.infer(torch.tensor([[1, 2, 3]])).shape[-1] == be.pipe.llm.cfg.vocab_size
    finally:
        be.unload()


def test_huggingface_backend_from_config_cpu():
    from transformers import Qwen2Config
    cfg = Qwen2Config(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, vocab_size=300)
    be = HuggingFaceBackend(device="cpu").load_model(None, config=cfg)
    out = be.generate_ids([5, 6, 7], max_new_tokens=5, min_new_tokens=5)
    assert len(out) == 5
    assert be.infer(torch.tensor([[5, 6, 7]])).shape == (1, 3, 300)


def test_llamacpp_backend_reports_missing_package():
    with pytest.raises(ImportError):
        LlamaCppBackend().load_model("x.gguf")


def test_ollama_backend_against_a_local_server():
    class H(BaseHTTPRequestHandler):
        def do_POST(self):
            body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
            out = json.dumps({"response": f"echo:{body['prompt']}:{body['options']['num_predict']}"}).encode()
            self.send_response(200)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(out)))
            self.end_headers()
            self.wfile.write(out)

        def log_message(self, *a):
            pass

    srv = HTTPServer(("127.0.0.1", 0), H)
    th = threading.Thread(target=srv.serve_forever, daemon=True)
    th.start()
    try:
        be = OllamaBackend(host=f"127.0.0.1:{srv.server_address[1]}").load_model("llama3")
        assert be.generate("hi", max_new_tokens=7) == "echo:hi:7"
    finally:
        srv.shutdown()
