"""specgrove_b200 — B200-native (sm_100a) packed tree-verification step.

The compute path is the C-ABI library ``libspecgrove_b200.so`` (hand-written
CUDA for sm_100a, declared in ``include/specgrove_b200.h``) driven from Python
through ctypes; PyTorch only provides device memory, streams and
``torch.distributed``.  Submodules:

  sampling   tree-sampling acceptance (reference verifier API + packed batch)
  arena      persistent per-request KV arena and accepted-path commit
  workloads  seeded synthetic inputs with the benchmark shapes
  build      nvcc build of the library
"""

__version__ = "0.1.0"
