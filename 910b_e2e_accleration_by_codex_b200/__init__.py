"""B200 (sm_100a) GatedDeltaNet hot path: CUDA kernels behind a C ABI, torch drop-ins for the
reference's plug-in points, and a slot-indexed continuous-batching engine.

Submodules:
  ops     torch-facing operators (reference signatures and slot-indexed forms)
  patch   patch_model(): installs the operators on HF Qwen3.5 modules
  engine  CBEngine: slot engine with CUDA-graph decode
  tp      tensor-parallel sharding and TPEngine
  build   nvcc build of libgdn_b200.so
"""
__version__ = "0.1.0"
