"""Scheduler, layer streaming, profiler, auto-detect, telemetry, persistence (CPU)."""
import torch

from vramancer_b200.engine.engine import SamplingParams
from vramancer_b200.parallel.scheduler import Scheduler


def _sched():
    return Scheduler(gpus=[{"id": 0, "name": "B200", "total_mb": 1000.0, "free_mb": 1000.0},
                           {"id": 1, "name": "B200", "total_mb": 1000.0, "free_mb": 600.0}], reserve_frac=0.1)


def test_scheduler_blocks_and_kv_reservations():
    s = _sched()
    b = s.allocate_block(300)
    assert b.gpu_id == 0                                   # most usable memory
    s.reserve_kv_cache(0, 400)
    b2 = s.allocate_block(300)
    assert b2.gpu_id == 1
    assert s.total_allocated_mb() == 600 and s.kv_cache_reserved_mb(0) == 400
    s.migrate_block(b, 1) if s.usable_mb(1) >= 300 else None
    try:
        s.allocate_block(10_000)
        raise AssertionError("expected MemoryError")
    except MemoryError:
        pass
    s.release_block(b2)
    s.release_kv_cache(0, 400)
    assert s.kv_cache_reserved_mb() == 0
    assert Scheduler.predict_next_layers([3, 5], 8, 3) == [6, 7, 0]
    mb = Scheduler.estimate_kv_cache_mb(48, 8, 128, 32, 1024)
    assert abs(mb - 2 * 48 * 8 * 128 * 32 * 1024 * 2 / 2**20) < 1e-6


def test_streamed_model_matches_resident():
    from vramancer_b200.llm import LLM
    kw = dict(device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", use_cuda_graph=False, max_batch=2,
              max_model_len=64, kv_pages=32, seed=9)
    prompts = [[1, 2, 3, 4, 5, 6], list(range(30, 50))]
    sp = SamplingParams(max_tokens=5)
    want = [o.output_ids for o in LLM("tiny-qwen2", **kw).generate(prompts, sp)]
    llm = LLM("tiny-qwen2", stream_layers=1, **kw)
    got = [o.output_ids for o in llm.generate(prompts, sp)]
    assert got == want
    st = llm.model.streamer.stats()
    assert st["loads"] > 0 and st["resident"] <= 1


def test_autodetect_telemetry_persistence(tmp_path):
    from vramancer_b200.utils import autodetect, persistence, telemetry
    assert autodetect.recommend_quantization(vram_gb=24, params_b=14) in ("nvfp4", "fp8")
    assert autodetect.recommend_quantization(vram_gb=180, params_b=14) == "none"
    assert autodetect.recommend_backend("x.gguf") == "llamacpp"
    assert autodetect.should_disable_p2p({"virtualized": True, "hypervisor": "kvm"}) is True
    rec = telemetry.NodeTelemetry(node_id=7, gpu_util=0.5, vram_used_gb=100.25, vram_total_gb=180.0,
                                  tok_s=1234.5, temp_c=61, power_w=700)
    raw = rec.pack()
    assert len(raw) == 24 and telemetry.NodeTelemetry.unpack(raw).node_id == 7
    back = telemetry.NodeTelemetry.unpack(raw)
    assert abs(back.tok_s - 1234.5) < 1 and back.temp_c == 61
    db = persistence.WorkflowStore(str(tmp_path / "wf.sqlite"))
    wid = db.create("summarise", {"steps": 2})
    db.update(wid, status="done", result={"ok": True})
    assert db.get(wid)["status"] == "done" and db.get(wid)["result"] == {"ok": True}
    assert [w["id"] for w in db.list()] == [wid]


def test_layer_profiler_cpu():
    from vramancer_b200.llm import LLM
    from vramancer_b200.utils.profiler import LayerProfiler
    llm = LLM("tiny-qwen2", device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", use_cuda_graph=False,
              max_batch=2, max_model_len=64, kv_pages=32)
    prof = LayerProfiler().profile_model(llm, tokens=8)
    assert len(prof) == llm.cfg.num_layers and all(p.time_ms >= 0 and p.params > 0 for p in prof)
    plan = LayerProfiler().plan(prof, [1.0, 1.0])
    assert sum(len(r) for r in plan.layer_ranges) == llm.cfg.num_layers
