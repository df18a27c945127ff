"""B200-native paged-attention hot path for the continuous-batching LLM server.

The package directory name is not a Python identifier, so it is imported under the alias
``llm_serving_b200`` (see ``load_package`` in ``__graft_entry__.py`` at the repository root).

Submodules:
  _native            ctypes binding of the C-ABI library libb200paged.so (include/b200_paged.h)
  llm_allocator_cpp  drop-in for the reference's pybind module of the same name
  block_manager      device-resident FIFO block pool and per-sequence block tables
  kv_cache           paged KV store on the device (reshape_and_cache, slot mapping, block tables)
  step_context       per-step ragged metadata built on the device
  attention_backends drop-in for app/model/attention_backends.py (NativePagedBackend)
  workloads          seeded synthetic batches for the BASELINE configurations
"""
from . import workloads  # noqa: F401
