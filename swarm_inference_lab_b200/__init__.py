"""swarm-inference-lab for B200: a Blackwell-native distributed inference runtime.

Layers (bottom up): ``ops`` (hand-written sm_100a kernels), ``models``
(decoder families and the PyTorch oracle), ``engine`` (paged KV cache,
continuous batching, CUDA-graph decode), ``parallel`` (tensor / expert /
pipeline parallel over NCCL and NVLink peer memory), ``protocol`` and
``transport`` (the SWRING01 stage ring), ``runtime`` (persistent stage
owners), ``coordinator`` / ``planner`` / ``cluster`` (control plane) and
``cli`` (the ``swarm`` command).
"""
__version__ = "0.1.0"
