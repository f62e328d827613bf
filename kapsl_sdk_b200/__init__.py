"""kapsl_sdk_b200: a B200-native (sm_100a) LLM inference runtime with the
capabilities and wire surface of kapsl-runtime / kapsl-sdk.

Layers (bottom-up): ``ops`` (sm_100a kernels), ``parallel`` (NCCL + NVLink
peer-memory collectives, TP/EP/PP), ``models`` (Llama/Qwen2/Mixtral),
``llm`` (paged-KV continuous-batching engine), ``runtime`` (request
scheduling, replicas, registry, packages), ``server`` (UDS/TCP/SHM wire
servers), ``monitor`` (Prometheus metrics).
"""
__version__ = "0.1.0"
