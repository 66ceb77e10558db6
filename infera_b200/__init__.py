"""infera_b200: a Blackwell-native distributed-inference orchestrator.

Layers (bottom up):
  ops/, csrc/      sm_100a kernels (tcgen05/TMEM/TMA) behind a C ABI
  models/          decoder models built from those ops (Llama-style GQA,
                   DeepSeek-V3-style MLA + MoE)
  engine/          paged-KV serving engine: block manager with prefix cache,
                   continuous-batching scheduler, CUDA-graph decode, KV events,
                   KV tiering, worker HTTP server and lifecycle
  parallel/        tensor / expert parallel groups and the fused
                   compute+collective kernels over NVLink peer memory
  kv/, kvd/        KV index and event plane; the KV tier daemon
  router/, server/ KV-aware router and the OpenAI/Anthropic front door
  native/          C++ router data plane
"""

__version__ = "0.1.0"
