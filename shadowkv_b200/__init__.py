"""shadowkv_b200: ShadowKV's sparse decode-attention step, hand-written for B200 (sm_100a).

Modules
-------
shadowkv   drop-in for the reference's ``kernels.shadowkv`` extension (12 bindings)
tensor_op  the reference's decode-path helpers of models/tensor_op.py
kvcache    ``ShadowKVCache_CPU`` (reference path and fused slot-stable path)
attention  ``ShadowAttention.decode`` / ``decode_fused``
decode     torch wrappers of the fused ``skv_decode_*`` C ABI (``step``: the one-call step)
graph      ``DecodeGraph``: the decode step of every layer captured as one CUDA graph
sharding   batch / KV-head partition across GPUs (head ranges; NCCL all-gather helper)
peer       kv-head outputs exchanged by the attention kernel over NVLink peer memory
workload   seeded synthetic workloads with the benchmark shapes
build      nvcc build of ``libshadowkv_b200.so``

The compute path is the CUDA library only; importing a module that needs it
raises if ``libshadowkv_b200.so`` has not been built.
"""

__version__ = "1.0.0"


def library_path() -> str:
    from ._lib import LIB_PATH
    return LIB_PATH
