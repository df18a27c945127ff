"""The reference-facing boundary on the GPU, exercised the way the reference's own code calls it:

* the C symbol ``paged_attention`` itself (csrc/include/paged_kernels.h:22-34 signature: no
  status code, a scratch pointer that is not used, a stream), called through ctypes on config 1;
* the drop-in ``llm_allocator_cpp.paged_attention`` (the binding of csrc/src/bindings.cpp:10-76),
  which must hand back a numpy array (1, Nq, Hq, D) whether its inputs are numpy arrays or CUDA
  tensors, so that the reference's unchanged caller NativePagedBackend.attend
  (app/model/attention_backends.py:108-117) can run ``torch.from_numpy(output)`` on it.

Tolerance: fp32 within 1e-5 relative (max |diff| / max |ref|) of the reference's output."""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import max_rel

pytestmark = pytest.mark.gpu

FP32_REL = 1e-5


def test_c_symbol_paged_attention_config1(pkg, golden):
    """Config 1 through the void ``paged_attention`` symbol with device pointers."""
    from config1_inputs import config1_inputs
    from llm_serving_b200 import _native as N
    b, q, kc, vc, gs, mask = config1_inputs()
    dev = torch.device("cuda")
    tq, tk, tv = (torch.from_numpy(x).to(dev) for x in (q, kc, vc))
    tgs, tm = torch.from_numpy(gs).to(dev), torch.from_numpy(mask).to(dev)
    out = torch.full((1, q.shape[2], q.shape[1], q.shape[3]), float("nan"), device=dev)
    dims = N.PagedAttentionDims(q.shape[1], q.shape[2], q.shape[3], kc.shape[0], kc.shape[1],
                                kc.shape[2], kc.shape[3], gs.shape[0])
    lib = ctypes.CDLL(N.LIB_PATH)
    fn = lib.paged_attention
    fn.restype = None
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                   N.PagedAttentionDims, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    stream = torch.cuda.current_stream(dev)
    fn(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), 0, dims, tgs.data_ptr(), tm.data_ptr(),
       ctypes.c_float(b.scale), out.data_ptr(), None, ctypes.c_void_p(stream.cuda_stream))
    stream.synchronize()
    assert max_rel(out.cpu().numpy(), golden["config1_out"]) <= FP32_REL


def test_binding_returns_numpy_for_host_and_device_inputs(pkg, golden):
    from config1_inputs import config1_inputs
    from llm_serving_b200 import llm_allocator_cpp as la
    b, q, kc, vc, gs, mask = config1_inputs()
    ref = golden["config1_out"]
    # host numpy inputs, as the reference's own tests would pass them
    out_np = la.paged_attention(q, kc, vc, 0, gs, mask, b.scale)
    assert isinstance(out_np, np.ndarray) and out_np.dtype == np.float32
    assert out_np.shape == (1, q.shape[2], q.shape[1], q.shape[3])
    assert max_rel(out_np, ref) <= FP32_REL
    # CUDA tensors, as NativePagedBackend.attend passes them when the model is on the GPU; the
    # caller's next line is torch.from_numpy(output).to(query.device)
    dev = torch.device("cuda")
    query = torch.from_numpy(q).to(dev)
    args = [query] + [torch.from_numpy(x).to(dev) for x in (kc, vc)]
    out = la.paged_attention(*args, 0, torch.from_numpy(gs).to(dev),
                             torch.from_numpy(mask).to(dev), b.scale)
    assert isinstance(out, np.ndarray)
    back = torch.from_numpy(out).to(query.device)
    assert back.is_cuda and back.shape == (1, q.shape[2], q.shape[1], q.shape[3])
    assert max_rel(back.cpu().numpy(), ref) <= FP32_REL
    # host torch tensors (the binding's force-cast also accepts them)
    out_t = la.paged_attention(torch.from_numpy(q), torch.from_numpy(kc), torch.from_numpy(vc), 0,
                               torch.from_numpy(gs), torch.from_numpy(mask), b.scale)
    assert max_rel(out_t, ref) <= FP32_REL


def test_binding_errors_match_the_reference(pkg):
    """Validation order and messages of bindings.cpp:25-48 (RuntimeError), and the fp32-only
    cache rule for device caches."""
    from llm_serving_b200 import llm_allocator_cpp as la
    dev = torch.device("cuda")
    q = torch.zeros((1, 4, 2, 64), device=dev)
    kc = torch.zeros((2, 8, 16, 2, 64), device=dev)
    gs = torch.zeros(5, dtype=torch.int32, device=dev)
    m = torch.ones((1, 1, 2, 5), dtype=torch.uint8, device=dev)
    with pytest.raises(RuntimeError, match="query must be 4-D"):
        la.paged_attention(q[0], kc, kc, 0, gs, m, 1.0)
    with pytest.raises(RuntimeError, match="key_cache must be 5-D"):
        la.paged_attention(q, kc[0], kc[0], 0, gs, m, 1.0)
    with pytest.raises(RuntimeError, match="gather_slots must be 1-D"):
        la.paged_attention(q, kc, kc, 0, gs[None], m, 1.0)
    with pytest.raises(RuntimeError, match="attention_mask must be 4-D"):
        la.paged_attention(q, kc, kc, 0, gs, m[0], 1.0)
    with pytest.raises(RuntimeError, match="multiple of num_kv_heads"):
        la.paged_attention(torch.zeros((1, 3, 2, 64), device=dev), kc, kc, 0, gs, m, 1.0)
    with pytest.raises(RuntimeError, match="layer_idx out of range"):
        la.paged_attention(q, kc, kc, 2, gs, m, 1.0)
    with pytest.raises(TypeError, match="float32"):
        la.paged_attention(q, kc.to(torch.bfloat16), kc.to(torch.bfloat16), 0, gs, m, 1.0)
