"""orcaml_b200 -- a B200 (sm_100a) CUDA backend for Orca's FP32 MLP
data-parallel training path.

  backend.CudaBackend      the reference's Backend trait over liborca_cuda.so
  mlp.MlpTrainer           fused device-resident training step
  distributed              NCCL gradient exchange with the reference's DDP surface
  synthetic                seeded inputs/weights with the benchmark configs' shapes

The compute path is liborca_cuda.so only; importing a submodule that needs it
raises if the library has not been built (python -m orcaml_b200.build).
"""
__version__ = "0.1.0"
