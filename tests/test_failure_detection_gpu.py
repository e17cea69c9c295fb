"""Device-side failure detection without a GPU fault: every spin-wait in the library is bounded and
reports through the device error word.  The probe entry point runs the kernels' own bounded mbarrier
wait on a barrier that nothing arrives at, with a short poll limit; the wait must run out, set the
barrier-timeout bit, come back as a negative status, and leave the context usable (a conv run
afterwards is bit-exact).  Nothing traps and nothing waits without a bound."""
import numpy as np
import pytest
import torch

from oracle import h3vae_oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_runs_out_and_reports(cuda_lib):
    from h3vae_b200 import _lib
    from h3vae_b200 import kernels as K
    assert _lib.device_error(clear=True) == 0
    stream = torch.cuda.current_stream().cuda_stream
    assert cuda_lib.h3b_probe_wait_timeout(0, stream) == _lib.H3B_EINVAL        # limit out of range
    rc = cuda_lib.h3b_probe_wait_timeout(1024, stream)
    assert rc == _lib.H3B_EDEVICE, (rc, _lib.last_error())
    assert "bounded wait expired after 1024 polls" in _lib.last_error()
    bits = _lib.device_error(clear=True)
    assert bits & 1, bits                                                        # kErrBarrierTimeout
    assert _lib.device_error(clear=True) == 0

    # the context still answers: an INT8 conv afterwards is bit-exact
    rng = np.random.default_rng(3)
    qx = rng.integers(-127, 128, size=(1, 128, 5, 10, 18), dtype=np.int8)
    qx[:, :, :2] = 0
    qw = rng.integers(-127, 128, size=(128, 27 * 128), dtype=np.int8)
    ws = (rng.random(128, dtype=np.float32) * 1e-3 + 1e-4).astype(np.float32)
    acc = torch.empty((1, 128, 3, 8, 16), dtype=torch.int32, device="cuda", memory_format=torch.channels_last_3d)
    K.conv3d_i8(torch.from_numpy(qx).cuda().contiguous(memory_format=torch.channels_last_3d),
                torch.tensor(0.01, device="cuda"), torch.from_numpy(qw).cuda(), torch.from_numpy(ws).cuda(), None,
                (3, 3, 3), causal_zero_frames=2, acc_out=acc)
    assert np.array_equal(acc.cpu().numpy(), O.conv3d_int_acc(qx, qw, (3, 3, 3)))
    assert _lib.device_error(clear=True) == 0
