"""B200 (sm_100a) implementation of Nano-vLLM-INT4's quantized-linear path.

Drop-in module paths of the reference:
  nanovllm.kernels.rht_a4_tilelang      rht_quant_pack, Config, best_config, compile_kernel
  nanovllm.kernels.w4a4_grouped_kernel  w4a4_grouped_gemm, GroupedConfig, best_grouped_config,
                                        compile_grouped_gemm (+ w4a4_group_dots diagnostic)
  nanovllm.layers.linear_w4a4           W4A4Linear (+ tensor-parallel variants)
  nanovllm.layers.linear_w4a16          W4A16Linear
  nanovllm.utils.loader_w4a4            load_w4a4_model
  nanovllm.LLM, nanovllm.SamplingParams  the engine (Qwen3; W4A4, W4A16 or BF16 linears;
                                        tensor parallelism one process per GPU)
All kernels live in the C-ABI library _lib/libnv4.so (see include/nv4.h).
"""
__version__ = "0.1.0"


def __getattr__(name):
    # `from nanovllm import LLM, SamplingParams` as in the reference, loaded on
    # first use (the engine pulls in transformers)
    if name == "LLM":
        from nanovllm.llm import LLM
        return LLM
    if name == "SamplingParams":
        from nanovllm.sampling_params import SamplingParams
        return SamplingParams
    raise AttributeError(name)
