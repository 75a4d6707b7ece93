"""B200-native (sm_100a) CUDA engine for the H2 engine's Qwen2 Q4_0 token loop.

Public surface (mirrors the reference engine, h2-own-inference-engine/engine/):
  gguf      parse_gguf / qwen2_config (gguf.js) and a GGUF writer for seeded models
  backend   create_cuda(...) -> backend object with the shape of createCPU's (cpu.js:52-68)
  llm       LLM.load / feed / generate_ids / reset (llm.js)
  synth     seeded benchmark models
The CUDA library itself is csrc/ -> libh2cuda.so, declared in include/h2cuda.h.
"""
__all__ = ["gguf", "synth"]
