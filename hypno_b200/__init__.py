"""hypno_b200 — an sm_100a (B200) backend for hypno's Q4_0 inference path.

The compute lives in libhypno_cuda.so (CUDA kernels + C ABI, see
include/hypno_cuda.h).  This package is the host-side mirror of the reference
engine's interfaces:
    hypno_b200.ops         ops.rs / quant.rs entry points
    hypno_b200.engine      HypnoModel, FlatKVCache, batch_forward, model_forward
    hypno_b200.hypno_file  the .hypno container
    hypno_b200.tp          tensor-parallel shard plan and communicator setup
    hypno_b200.serve       continuous batching for the serve path (serve.rs)
    hypno_b200.convert     safetensors -> .hypno with Q4_0 packed on the GPU
                           (sft_convert.rs)
    hypno_b200.synth       seeded synthetic models for the benchmark configs
    hypno_b200.build       nvcc build of the shared library
"""
__version__ = "0.1.0"
