"""B200-native (sm_100a) gpt-oss mixture-of-experts layer.

A drop-in for the MoE layer that hareramray/BlockStreamer runs
(``block_streamer.gptoss.MXFP4Experts`` inside transformers' ``GptOssMLP``):
same module API and parameter names, with the router, dispatch, MXFP4 expert
projections, SwiGLU and weighted combine running as hand-written CUDA kernels
behind a C ABI (``include/bs_moe.h``, ``libbs_moe.so``).

Submodules:
  ``gptoss``           drop-in modules and functions (the reference's API)
  ``kernels``          torch wrappers over the C ABI
  ``expert_parallel``  expert-parallel layer over torch.distributed (NCCL)
  ``synthetic``        seeded synthetic layers/tokens for tests and benchmarks
  ``build``            in-tree build of the library
"""

from .gptoss import (B200GptOssMLP, B200GptOssMoEBlock, B200MXFP4Experts, dequantize_expert,
                     install_b200_experts, install_b200_mlp, mxfp4_matmul)

__all__ = ["B200GptOssMLP", "B200GptOssMoEBlock", "B200MXFP4Experts", "dequantize_expert",
           "install_b200_experts", "install_b200_mlp", "mxfp4_matmul"]
