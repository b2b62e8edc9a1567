"""Cross-node pipeline parallelism over signed TCP frames: a local stage plus a remote
stage server (CPU, localhost) generate token-for-token like the single-device model."""
import torch

from vramancer_b200.cluster.stage_server import RemoteStage, StageServer
from vramancer_b200.engine.engine import LLMEngine, SamplingParams
from vramancer_b200.engine.runner import ModelRunner
from vramancer_b200.kv.paged import PagedKVCacheManager
from vramancer_b200.kv.pool import KVPool, KVPoolSpec
from vramancer_b200.llm import LLM
from vramancer_b200.models.config import get_config
from vramancer_b200.models.transformer import DecoderModel
from vramancer_b200.models.weights import random_weights
from vramancer_b200.parallel.pipeline import LocalPipeline


def test_remote_stage_matches_single_device():
    cfg = get_config("tiny-qwen2")
    split = cfg.num_layers // 2
    pages = 64
    prompts = [[3, 1, 4, 1, 5, 9, 2, 6], list(range(20, 60))]
    sp = SamplingParams(max_tokens=6)
    ref = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", use_cuda_graph=False, max_batch=4,
              max_model_len=128, kv_pages=pages, seed=5)
    want = [o.output_ids for o in ref.generate(prompts, sp)]

    srv = StageServer(cfg, split, cfg.num_layers, port=0, num_pages=pages, seed=5, key=b"k").start()
    try:
        w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=5, layers=range(0, split), embed=True,
                           head=False)
        m0 = DecoderModel(cfg, w, device="cpu", dtype=torch.float32, first_layer=0, last_layer=split)
        p0 = KVPool(KVPoolSpec(pages, split, m0.kvh, cfg.head_dim, dtype=torch.float32), torch.device("cpu"))
        remote = RemoteStage("127.0.0.1", srv.port, key=b"k")
        assert (remote.first_layer, remote.last_layer) == (split, cfg.num_layers)
        pipe = LocalPipeline([(m0, p0), (remote, None)])
        kv = PagedKVCacheManager(pages)
        eng = LLMEngine(ModelRunner(pipe, None, max_batch=4, max_model_len=128, use_cuda_graph=False), kv)
        got = [o.output_ids for o in eng.generate(prompts, sp)]
        assert got == want
        assert srv.requests > 0
        remote.shutdown_server()
    finally:
        srv.close()
