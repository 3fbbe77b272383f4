"""sparkpipe_rs_b200 — a B200-native (sm_100a) MLA-MoE LLM serving engine.

Layers (top to bottom):
  serving/   HTTP gateway + SSE, OpenAI/Anthropic compat, service runtime, engine pump
  core/      C++ serving runtime bindings: KV arena, prefix cache, scheduler, work control, ...
  parallel/  process groups, data/expert/tensor/pipeline parallel plumbing, fused collectives
  models/    model contracts and configs, weights, the fp32 oracle, the kernel-backed model
  ops/       Python entry points of the hand-written sm_100a CUDA kernels
  utils/     timing, clocks, misc helpers
"""
__version__ = "0.1.0"
