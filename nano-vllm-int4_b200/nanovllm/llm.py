"""``LLM``: the user-facing entry point (the reference's ``nanovllm/llm.py``):
``LLM(model, w4a4_checkpoint=..., use_w4a16=..., tensor_parallel_size=...)``
then ``generate(prompts, SamplingParams(...))``."""
from nanovllm.engine.llm_engine import LLMEngine


class LLM(LLMEngine):
    pass
