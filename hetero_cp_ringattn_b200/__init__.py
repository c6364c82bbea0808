"""hetero_cp_ringattn_b200: a B200-native heterogeneous context-parallel inference framework.

A coordinator splits a prompt into uneven, capacity-weighted per-rank sequence chunks; every
rank (one process per GPU) holds a full Llama/Qwen2 replica and keeps only its own shard of the
KV cache. Prefill attention is blockwise online-softmax ring attention: each rank's projection
epilogue (or push kernel) stores its K/V rows once into every rank's staging buffer over NVLink,
and the tcgen05 attention kernel reads them from local memory. Decode attention computes per-rank
partial (O, LSE) over the local shard and combines them across ranks with peer stores.

Sub-packages:
  models/    Llama/Qwen2 engine (LlamaCPEngine), HF safetensors weights, sampling, fp32 oracle
  ops/       Python front-ends of the sm_100a kernels (+ fp32/fp64 reference oracles)
  parallel/  capacity chunking, ring layouts, KV-growth schedule (bindings of the host library)
  kv/        paged, position-tagged KV arena bookkeeping
  serve/     control protocol, coordinator, scheduler, worker loop, HTTP API
  utils/     perf JSONL, CUDA-event timing, clock sampling
Native code: `_C` (sm_100a kernels + the domain runtime), `_host` (C++ host runtime library).

Common entry points are importable from the package root:

    from hetero_cp_ringattn_b200 import LlamaCPEngine, ModelWeights, PreparedWeights, preset
"""

__version__ = "0.1.0"

_EXPORTS = {
    "LlamaCPEngine": ("models.llama", "LlamaCPEngine"),
    "ModelWeights": ("models.weights", "ModelWeights"),
    "PreparedWeights": ("models.weights", "PreparedWeights"),
    "ModelConfig": ("config", "ModelConfig"),
    "EnvConfig": ("config", "EnvConfig"),
    "preset": ("config", "preset"),
    "RingStrategy": ("parallel.strategy", "RingStrategy"),
    "Coordinator": ("serve.coordinator", "Coordinator"),
    "CoordinatorArgs": ("serve.coordinator", "CoordinatorArgs"),
}

__all__ = sorted(_EXPORTS) + ["__version__"]


def __getattr__(name):
    # imported on first use, so `import hetero_cp_ringattn_b200` stays cheap
    if name in _EXPORTS:
        import importlib
        mod, attr = _EXPORTS[name]
        return getattr(importlib.import_module(f"{__name__}.{mod}"), attr)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
