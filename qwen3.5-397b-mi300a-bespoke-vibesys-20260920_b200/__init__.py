"""qwen35_b200: a B200-native serving engine for the Qwen3.5-MoE hybrid architecture.

Layers (top to bottom):

* ``serving``  - HTTP server, continuous-batching scheduler, prefix/session cache, paged
  block pool, prompt cache, CUDA-graph runners.
* ``parallel`` - tensor/expert-parallel plan, SPMD command protocol, NCCL/gloo process group,
  symmetric peer memory and the fused collective kernels' host side.
* ``models``   - config, weight loading / random init, the Qwen3.5-MoE runtime and the MTP
  draft layer.
* ``ops``      - Python entry points of the sm_100a CUDA kernels (``csrc/``), each with a
  plain PyTorch statement of the same math used on CPU and as the test oracle.
* ``utils``    - safetensors IO, MXFP4 codec, telemetry, flags.
"""
