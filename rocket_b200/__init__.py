"""rocket_b200: a B200-native (sm_100a) MoE LLM inference engine.

Layers: config (fuel/booster/rocket/engine YAML) -> fuel (NVFP4 codec,
safetensors) -> ops (tcgen05/TMA kernels) -> models (GPU executor + CPU oracle)
-> engine (continuous batching, paged KV, CUDA graphs) -> parallel (NCCL +
fused NVLink collectives).
"""
__version__ = "0.1.0"
