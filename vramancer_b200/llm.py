"""`LLM`: one-call construction of the serving stack on one device.

    llm = LLM("qwen2.5-14b")                     # preset, random-init weights
    llm = LLM("/models/Qwen2.5-14B-Instruct")    # HF checkpoint directory
    outs = llm.generate([[1, 2, 3]], SamplingParams(max_tokens=32))

Builds the weights (HF safetensors, NVFP4 checkpoint or random N(0, 0.02)), the paged
KV pool sized from the free memory left after the weights, the block manager, the
model runner (CUDA-graph decode) and the continuous-batching engine.

With `kv_lender=d` (or a `lending_pool`), KV pages beyond the local pool are borrowed
from GPU d's memory (kv/overflow.py) and read in place by the attention kernels, so a
sequence may grow past the local pool; the memory returns to the lender when its pages
are freed or reclaimed.

With `fold_norms=True` (the default; dense RMSNorm models with bf16 weights on one
GPU) the input and post-attention RMSNorm weights are multiplied into the columns of
`qkv_w` / `gate_up_w` in place, so small decode batches run the norms inside the
GEMMs.  `llm.weights` then holds the folded matrices (each marked with the norm weight
it carries, `_vrm_norm_w`); pass `fold_norms=False` to keep checkpoint tensors as
loaded.
"""
from __future__ import annotations

import os
from typing import List, Optional, Sequence, Union

import torch

from .engine.engine import LLMEngine, Request, SamplingParams
from .engine.runner import ModelRunner
from .kv.paged import PagedKVCacheManager
from .kv.pool import KVPool, KVPoolSpec, kv_dtype_from_str
from .models.config import ModelConfig, get_config
from .models.transformer import DecoderModel
from .models.weights import load_safetensors, random_weights


def _moe_graph_safe() -> bool:
    """True when MoE layers run on the device-scheduled grouped GEMM (no host sync)."""
    from .parallel import moe
    return getattr(moe, "DEVICE_MOE", False)


def _is_checkpoint_dir(p: str) -> bool:
    return os.path.isdir(p) and any(f.endswith(".safetensors") for f in os.listdir(p))


class LLM:
    def __init__(self, model: Union[str, ModelConfig] = "qwen2.5-14b", *, device: str = "cuda",
                 dtype: torch.dtype = torch.bfloat16, kv_cache_dtype: str = "bf16", max_batch: int = 64,
                 max_model_len: int = 4096, kv_pages: Optional[int] = None, gpu_memory_utilization: float = 0.9,
                 seed: int = 0, use_cuda_graph: bool = True, enable_prefix_cache: bool = True,
                 max_prefill_tokens: int = 8192, eos_token_id: Optional[int] = None, weights=None,
                 num_layers: Optional[int] = None, tp=None, quantization: Optional[str] = None,
                 spec_num_draft: int = 0, spec_ngram: int = 3, kv_offload_pages: int = 0, hierarchy=None,
                 stream_layers: int = 0, ep=None, fold_norms: bool = True, pp_grid=None,
                 prefill_microbatches: int = 0, decode_microbatches: int = 1, kv_lender: Optional[int] = None,
                 kv_borrow_pages: int = 0, lending_pool=None):
        if isinstance(model, ModelConfig):
            cfg = model
        else:
            cfg = get_config(model)
        if num_layers is not None:
            cfg = cfg.with_(num_layers=num_layers)
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.type == "cuda":
            if self.device.index is None:         # "cuda" = the current device
                self.device = torch.device("cuda", torch.cuda.current_device())
            torch.cuda.set_device(self.device)
        self.tp = tp
        tp_rank, tp_size = (tp.rank, tp.size) if tp is not None else (0, 1)
        # expert parallelism: `ep` is an ExpertParallel (or True to build one over the
        # default process group); experts are sharded, everything else is replicated
        if ep is True:
            from .parallel.expert_parallel import ExpertParallel
            ep = ExpertParallel(cfg, device=self.device)
        if ep is not None and tp is not None and tp.size > 1:
            raise ValueError("expert parallelism runs with data-parallel attention (tp must be 1)")
        self.ep = ep
        ep_rank, ep_size = (ep.rank, ep.world) if ep is not None else (0, 1)
        # pipeline x tensor parallelism (parallel/pp.py): this rank's stage only
        self.pp_grid = pp_grid
        part = {}
        if pp_grid is not None:
            first, last = pp_grid.layers(cfg.num_layers)
            part = dict(layers=range(first, last), embed=pp_grid.is_first, head=pp_grid.is_last)
        if weights is None:
            if isinstance(model, str) and _is_checkpoint_dir(model):
                weights = load_safetensors(model, cfg, device=self.device, dtype=dtype, tp_rank=tp_rank,
                                           tp_size=tp_size, ep_rank=ep_rank, ep_size=ep_size, **part)
            else:
                # streamed layers live in host memory: build them there
                wdev = torch.device("cpu") if stream_layers > 0 else self.device
                weights = random_weights(cfg, device=wdev, dtype=dtype, seed=seed, tp_rank=tp_rank,
                                         tp_size=tp_size, ep_rank=ep_rank, ep_size=ep_size, **part)
        self.quantization = (quantization or "").lower() or None
        if self.quantization == "nvfp4":
            from .quant.nvfp4 import quantize_model_weights
            weights = quantize_model_weights(weights, cfg)
        elif self.quantization == "fp8":
            from .quant.fp8 import quantize_model_weights as fp8_quantize
            weights = fp8_quantize(weights, cfg)
        elif self.quantization not in (None, "none", "bf16"):
            raise ValueError(f"unsupported quantization {quantization!r} (nvfp4, fp8 or none)")
        self.weights = weights
        if cfg.is_moe and not _moe_graph_safe():
            # the host-driven expert loop reads routing counts back: no graph capture
            use_cuda_graph = False
        if stream_layers > 0:
            # layer weights stay in pinned host memory, `stream_layers` layers resident
            from .engine.streaming import StreamedDecoderModel
            self.model = StreamedDecoderModel(cfg, weights, budget_layers=stream_layers, device=self.device,
                                              dtype=dtype, tp=tp)
            use_cuda_graph = False
        elif pp_grid is not None:
            from .parallel.pp import PPStageModel
            self.model = PPStageModel(cfg, weights, pp_grid, device=self.device, dtype=dtype, tp=tp,
                                      prefill_microbatches=prefill_microbatches,
                                      decode_microbatches=decode_microbatches)
        else:
            self.model = DecoderModel(cfg, weights, device=self.device, dtype=dtype, tp=tp, ep=ep)
            if (fold_norms and self.quantization is None and ep is None
                    and (tp is None or tp.size == 1 or getattr(tp, "fused_ar", None) is not None)
                    and os.environ.get("VRM_FOLD_NORM", "1") != "0"):
                # small decode batches run the RMSNorms inside the GEMMs (weights folded in place)
                self.model.fold_norms()
        kvd = kv_dtype_from_str(kv_cache_dtype)
        if kv_pages is None:
            kv_pages = self._pages_from_memory(cfg, kvd, gpu_memory_utilization, max_batch, max_model_len)
        spec = KVPoolSpec(kv_pages, self._kv_layers(), self.model.kvh, cfg.head_dim, dtype=kvd)
        if kv_lender is not None or lending_pool is not None:
            # VRAM lending: pages beyond the local pool are borrowed from another GPU's
            # memory and read in place by the kernels (kv/overflow.py)
            from .kv.overflow import ExtensiblePagePool
            self.pool = ExtensiblePagePool(spec, self.device, kv_lender, kv_borrow_pages or kv_pages,
                                           lending_pool=lending_pool)
        else:
            self.pool = KVPool(spec, self.device)
        self.offload = None
        if kv_offload_pages > 0 and enable_prefix_cache:
            # evicted prefix pages go to pinned host memory (and on to NVMe through `hierarchy`)
            from .kv.offload import KVOffloader
            self.offload = KVOffloader([self.pool.cache], kv_offload_pages, hierarchy=hierarchy)
        self.kv = PagedKVCacheManager(kv_pages, spec.page_size, enable_prefix_cache=enable_prefix_cache,
                                      offload=self.offload)
        if hasattr(self.pool, "attach"):
            self.pool.attach(self.kv)
        self.runner = ModelRunner(self.model, self.pool, max_batch=max_batch, max_model_len=max_model_len,
                                  use_cuda_graph=use_cuda_graph, seed=seed)
        ep_sync = None
        if ep is not None:
            import torch.distributed as dist

            from .engine.engine import EPSync
            grp = None
            if dist.is_initialized() and dist.get_backend() != "gloo":
                grp = dist.new_group(backend="gloo")      # host-side step agreement
            ep_sync = EPSync(self.kv, group=grp)
            max_prefill_tokens = min(max_prefill_tokens, getattr(ep, "max_tokens", max_prefill_tokens))
        self.engine = LLMEngine(self.runner, self.kv, max_prefill_tokens=max_prefill_tokens,
                                eos_token_id=eos_token_id, spec_num_draft=spec_num_draft, spec_ngram=spec_ngram,
                                ep_sync=ep_sync)
        if ep is not None and self.runner.use_graph:
            # a lazy capture runs an eager warm-up pass, which would unpair the ranks' MoE
            # calls mid-run: every rank captures every bucket now, in the same order
            self.runner.capture_all()

    def _kv_layers(self) -> int:
        """Layers whose KV this rank holds (a pipeline stage holds its own layers')."""
        return self.model.num_local_layers if self.pp_grid is not None else self.cfg.num_layers

    def _pages_from_memory(self, cfg, kvd, util, max_batch, max_model_len) -> int:
        need = max_batch * ((max_model_len + 15) // 16) + 16
        if self.device.type != "cuda":
            return min(need, 4096)
        free, total = torch.cuda.mem_get_info(self.device)
        budget = int(free - (1 - util) * total) - (2 << 30)   # keep ~2 GiB for activations/graphs
        per = KVPoolSpec(1, self._kv_layers(), self.model.kvh, cfg.head_dim, dtype=kvd).bytes_per_page
        return max(16, min(need * 2, budget // per))

    # ------------------------------------------------------------------ API
    @classmethod
    def from_local_pipeline(cls, cfg: ModelConfig, blocks, *, num_pages: int, max_batch: int = 64,
                            max_model_len: int = 4096, dtype: torch.dtype = torch.bfloat16, kv_dtype=None,
                            weights=None, transfer=None, eos_token_id: Optional[int] = None) -> "LLM":
        """An LLM over an in-process layer pipeline: one stage (layers, KV pool) per block
        of `blocks` (parallel.placement.Block: start, end, device), activations moved
        between the stages' devices by `transfer(tensor, device)` (a peer copy by
        default).  Decode runs eagerly (no CUDA graph across devices)."""
        from .parallel.pipeline import LocalPipeline, build_local_pipeline
        pipe = build_local_pipeline(cfg, blocks, num_pages=num_pages, dtype=dtype, kv_dtype=kv_dtype or dtype,
                                    weights=weights)
        if transfer is not None:
            pipe = LocalPipeline(pipe.stages, transfer=transfer)
        llm = cls.__new__(cls)
        llm.cfg, llm.device, llm.model, llm.pool = cfg, pipe.device, pipe, None
        llm.tp, llm.pp_grid, llm.quantization, llm.offload = None, None, None, None
        llm.weights = weights
        llm.kv = PagedKVCacheManager(num_pages)
        llm.runner = ModelRunner(pipe, None, max_batch=max_batch, max_model_len=max_model_len, use_cuda_graph=False)
        llm.engine = LLMEngine(llm.runner, llm.kv, eos_token_id=eos_token_id)
        return llm

    def generate(self, prompts: Sequence[Sequence[int]], params: Optional[SamplingParams] = None) -> List[Request]:
        return self.engine.generate(prompts, params)

    def warmup(self, batch_sizes: Optional[Sequence[int]] = None) -> None:
        """Captures the decode graphs ahead of time."""
        self.runner.capture_all(batch_sizes)

    def stats(self):
        d = dict(self.engine.stats)
        d.update({f"kv_{k}": v for k, v in self.kv.stats().items()})
        return d
