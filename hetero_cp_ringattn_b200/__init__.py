"""hetero_cp_ringattn_b200: a B200-native heterogeneous context-parallel inference framework.

A coordinator splits a prompt into uneven, capacity-weighted per-rank sequence chunks; every
rank (one process per GPU) holds a full Llama/Qwen2 replica and keeps only its own shard of the
KV cache. Prefill attention is blockwise online-softmax ring attention whose peer-KV rotation
runs over NVLink from inside the attention kernel; decode attention computes per-rank partial
(O, LSE) over the local shard and combines them across ranks with peer stores.

Sub-packages:
  models/    Llama/Qwen2 decoder, HF safetensors weights, sampling, generators
  ops/       Python front-ends of the sm_100a kernels (+ fp32/fp64 reference oracles)
  parallel/  capacity chunking, ring strategies, KV assignee schedule, peer memory, ring/decode
  kv/        paged, position-tagged KV arena
  serve/     control protocol, coordinator, scheduler, worker loop, HTTP API
  utils/     perf JSONL, CUDA-event timing, clock sampling
"""

__version__ = "0.1.0"
