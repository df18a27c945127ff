"""Import the reference's own Python engine (app/, staged unmodified into oracle/_ref/app by
`make -C oracle ref`) with its `import llm_allocator_cpp` bound to a module chosen by the caller:
this package's drop-in module (host allocator mirror + the B200 kernels behind the binding's
names) or the reference's compiled binding.  Test infrastructure only."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_APP_PARENT = os.path.join(ROOT, "oracle", "_ref")


def staged() -> bool:
    return os.path.isfile(os.path.join(REF_APP_PARENT, "app", "engine", "llm_engine.py"))


def torch_compat():
    """The reference pins torch 2.13 (requirements.txt:65); its CudaKVCacheStrategy enters
    torch.cuda._device_ctx(index) (app/memory/strategies.py:112,118), a private helper this
    image's torch 2.11 does not have.  torch.cuda.device(index) is the same context manager (the
    device is current inside the block), so it stands in for it; nothing else is changed."""
    import torch
    if not hasattr(torch.cuda, "_device_ctx"):
        torch.cuda._device_ctx = torch.cuda.device


def import_reference_app(binding):
    """Make `import llm_allocator_cpp` resolve to `binding`, put the staged tree first on the
    path and import the engine's modules.  One binding per process: the reference modules keep
    the module object they imported."""
    current = sys.modules.get("llm_allocator_cpp")
    if current is not None and current is not binding:
        raise RuntimeError("the reference app was already imported with another binding")
    sys.modules["llm_allocator_cpp"] = binding
    torch_compat()
    if REF_APP_PARENT not in sys.path:
        sys.path.insert(0, REF_APP_PARENT)
    import app.engine.llm_engine as llm_engine
    import app.memory.manager as manager
    import app.model.attention_backends as backends
    import app.model.paged_attention as paged_attention
    import app.scheduler.scheduler as scheduler
    return {"LLMEngine": llm_engine.LLMEngine, "PagedKVCacheManager": manager.PagedKVCacheManager,
            "Scheduler": scheduler.Scheduler, "backends": backends,
            "paged_attention": paged_attention}
