"""B200-native paged-attention hot path for the continuous-batching LLM server.

The package directory name is not a Python identifier, so it is imported under the alias
``llm_serving_b200`` (see ``load_package`` in ``__graft_entry__.py`` at the repository root).

Submodules:
  _native            ctypes binding of the C-ABI library libb200paged.so (include/b200_paged.h)
  paged_ops          torch-tensor front end of the C ABI (decode, prefill, cache writes, copies)
  llm_allocator_cpp  drop-in for the reference's pybind module of the same name
  block_manager      device-resident FIFO block pool and per-sequence block tables
  kv_cache           paged KV store on the device (reshape_and_cache, slot mapping, block tables,
                     prefix sharing, swap space)
  step_context       per-step ragged metadata built on the device
  attention_backends drop-in for app/model/attention_backends.py (NativePagedBackend)
  paged_attention    the per-layer attention hook (app/model/paged_attention.py)
  engine             continuous-batching engine: scheduler, CUDA-graph decode steps
  model              random-init Llama-style decoder, tensor parallel by KV head
  workloads          seeded synthetic batches and request streams for the BASELINE configurations
"""
from . import workloads  # noqa: F401
