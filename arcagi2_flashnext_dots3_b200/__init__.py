"""B200-native (sm_100a) serving and repair-training framework for low-bit MoE LLMs.

Same capabilities as notnitsuj/arcagi2_flashnext_dots3 (Flash-Next-shaped hybrid GDN/sparse-attention MoE and
Dots3-shaped MLA MoE with packed 2/3/4-bit GPTQ experts), rebuilt around hand-written tcgen05/TMA kernels and
in-kernel NVLink collectives. Subpackages:

* ``formats``  checkpoint formats (planar low-bit experts, routers, keep sets, deltas) and runtime layouts
* ``ops``      kernel entry points (CUDA on GPU tensors, torch reference on CPU tensors)
* ``models``   model definitions (Flash-Next-shaped, Dots3-shaped, dense fp32 oracles)
* ``parallel`` process groups, symmetric peer memory, fused compute+collective kernels, NCCL baseline
* ``engine``   paged KV, scheduler, CUDA-graph runner, speculative decoding, sessions, public LLM API
* ``server``   HTTP API (completions + session routes)
* ``training`` low-bit student autograd, RL repair step, gradient overlap, delta export
* ``agent``    ARC solver harness (sandbox, grid library, voting, deadlines)
* ``launch``   launchers, packaging, preflight
* ``utils``    logging, tracing, step logs, timing
"""
__version__ = "0.1.0"
