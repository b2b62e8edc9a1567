"""VRAMancer-B200: a B200-native (sm_100a) multi-GPU LLM inference framework.

Public API (the reference's names where they exist):
    patch / unpatch / is_patched / compute_max_memory    drop-in for HF from_pretrained
    InferencePipeline, get_pipeline, reset_pipeline      conductor
    LLM, SamplingParams                                  one-call engine construction
    LLMEngine (ContinuousBatcher)                        continuous batching over paged KV
    PagedKVCacheManager, KVPool                          paged KV
    split_model_into_blocks, auto_configure              placement
    TurboEngine, MultiGPUTurboEngine,                    engine object over a loaded HF model
    SpeculativeTurboEngine, create_turbo_engine          (or preset / checkpoint directory)
"""
__version__ = "0.1.0"

_LAZY = {
    "patch": ("dropin", "patch"), "unpatch": ("dropin", "unpatch"), "is_patched": ("dropin", "is_patched"),
    "compute_max_memory": ("parallel.placement", "compute_max_memory"),
    "InferencePipeline": ("pipeline", "InferencePipeline"), "get_pipeline": ("pipeline", "get_pipeline"),
    "reset_pipeline": ("pipeline", "reset_pipeline"),
    "LLM": ("llm", "LLM"), "SamplingParams": ("engine.engine", "SamplingParams"),
    "LLMEngine": ("engine.engine", "LLMEngine"), "ContinuousBatcher": ("engine.engine", "LLMEngine"),
    "PagedKVCacheManager": ("kv.paged", "PagedKVCacheManager"), "KVPool": ("kv.pool", "KVPool"),
    "split_model_into_blocks": ("parallel.placement", "split_model_into_blocks"),
    "auto_configure": ("parallel.placement", "auto_configure"),
    "VRAMLendingPool": ("kv.lending", "VRAMLendingPool"),
    "KVCacheCompressor": ("kv.turboquant", "KVCacheCompressor"),
    "TurboQuantCache": ("kv.turboquant", "TurboQuantCache"),
    "DirectFP4Linear": ("quant.nvfp4", "DirectFP4Linear"),
    "apply_tensor_parallel": ("parallel.tensor_parallel", "apply_tensor_parallel"),
    "TurboEngine": ("engine.turbo", "TurboEngine"), "MultiGPUTurboEngine": ("engine.turbo", "MultiGPUTurboEngine"),
    "SpeculativeTurboEngine": ("engine.turbo", "SpeculativeTurboEngine"),
    "create_turbo_engine": ("engine.turbo", "create_turbo_engine"),
    "weights_from_state_dict": ("models.weights", "weights_from_state_dict"),
}


def __getattr__(name):
    if name in _LAZY:
        import importlib
        mod, attr = _LAZY[name]
        return getattr(importlib.import_module(f".{mod}", __name__), attr)
    raise AttributeError(name)


__all__ = sorted(_LAZY)
