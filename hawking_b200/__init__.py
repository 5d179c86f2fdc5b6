"""hawking_b200: a B200-native LLM inference engine.

Layers (top to bottom): ``serve`` (OpenAI HTTP server, C++), ``engine`` (paged KV, scheduler,
sampling, speculative decode), ``models`` (Llama/Qwen/Mixtral/Qwen3-Next/DeepSeek forwards in
PyTorch over our kernels), ``parallel`` (TP/EP over NCCL plus in-kernel NVLink collectives),
``ops`` (sm_100a CUDA kernels), ``formats`` (GGUF, .gravity, HGRAV* codecs).
"""
__version__ = "0.1.0"
