"""The allocation-free INT8 norm producer, h3b_norm_pad_quant_noalloc.

It exists for callers that cannot allocate device memory at the call site (a host that gives the
library only its input and output buffers from a pre-sized pool, with no allocator or spare
workspace to pass): its scratch is a static 4 MiB device array inside the library.  This test
calls it through the C ABI twice in a row, on two different shapes, and checks each result against
the workspace entry point h3b_norm_pad_quant on the same inputs (same kernels, so the INT8 values
and the scale must be identical), then checks that an over-large shape is refused.  It is
collected last so that a failure here does not stop the rest of the GPU suite.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

CL3 = torch.channels_last_3d


def _inputs(shape, seed):
    g = torch.Generator().manual_seed(seed)
    b, c, d, h, w = shape
    x = torch.randn(shape, generator=g).half().cuda().contiguous(memory_format=CL3)
    gamma = torch.randn(c, generator=g).half().cuda()
    beta = torch.randn(c, generator=g).half().cuda()
    pre = torch.randn(c, generator=g).half().cuda()
    return x, gamma, beta, pre


def _outputs(shape):
    b, c, d, h, w = shape
    q = torch.empty((b, c, d + 2, h + 2, w + 2), dtype=torch.int8, device="cuda", memory_format=CL3)
    s = torch.empty((), dtype=torch.float32, device="cuda")
    return q, s


def test_noalloc_producer_matches_workspace_producer_twice(cuda_lib):
    from h3vae_b200 import _lib
    lib = cuda_lib
    stream = torch.cuda.current_stream().cuda_stream
    for shape, seed in (((1, 128, 5, 32, 48), 11), ((2, 256, 3, 16, 24), 12)):
        x, gamma, beta, pre = _inputs(shape, seed)
        b, c, d, h, w = shape
        # existing entry point, caller-provided workspace
        ws_bytes = lib.h3b_norm_workspace_size(b, c, d, h, w)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        q_ref, s_ref = _outputs(shape)
        _lib.check(lib.h3b_norm_pad_quant(x.data_ptr(), b, c, d, h, w, pre.data_ptr(), gamma.data_ptr(),
                                          beta.data_ptr(), ctypes.c_float(1e-6), q_ref.data_ptr(), s_ref.data_ptr(),
                                          ws.data_ptr(), ws_bytes, stream))
        # allocation-free entry point
        q, s = _outputs(shape)
        _lib.check(lib.h3b_norm_pad_quant_noalloc(x.data_ptr(), b, c, d, h, w, pre.data_ptr(), gamma.data_ptr(),
                                                  beta.data_ptr(), ctypes.c_float(1e-6), q.data_ptr(), s.data_ptr(),
                                                  stream))
        torch.cuda.synchronize()
        assert torch.equal(s, s_ref), (float(s), float(s_ref))
        assert torch.equal(q, q_ref)
    assert _lib.device_error() == 0


def test_noalloc_producer_rejects_shapes_beyond_its_scratch(cuda_lib):
    from h3vae_b200 import _lib
    lib = cuda_lib
    b, c, d, h, w = 64, 128, 17, 256, 256   # needs far more than the 4 MiB static scratch
    assert lib.h3b_norm_workspace_size(b, c, d, h, w) > (4 << 20)
    rc = lib.h3b_norm_pad_quant_noalloc(None, b, c, d, h, w, None, None, None, ctypes.c_float(1e-6), None, None,
                                        torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.H3B_EUNSUPPORTED
    assert "static buffer" in _lib.last_error()
