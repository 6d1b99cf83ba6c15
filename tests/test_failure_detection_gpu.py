"""Failure detection without a GPU fault: every barrier wait in the tensor-core kernels is bounded, and a
wait that runs out records a code in the device status word and lets the kernel return, so the host sees
an error status instead of a hung GPU.

The test makes one wait run out on purpose through the library's test hook (jx_gemm_wait_test): the GEMM
kernel runs with its TMA loads withheld and a short wait budget, so the MMA thread's wait for the first
operand stage is a barrier that nothing completes. Nothing faults, traps or spins without a limit."""
import time

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_status_and_context_stays_usable():
    from midstream_llm_b200 import _lib, ops
    torch.cuda.set_device(0)
    _lib.device_status(clear=True)
    g = torch.Generator(device="cuda").manual_seed(3)
    A = (torch.randn(128, 64, device="cuda", generator=g) * 0.5).half()
    B = (torch.randn(256, 64, device="cuda", generator=g) * 0.5).half()
    C = torch.full((128, 256), 7.0, device="cuda", dtype=torch.float16)
    t0 = time.perf_counter()
    _lib.call("jx_gemm_wait_test", A.data_ptr(), B.data_ptr(), C.data_ptr(), 100_000,
              torch.cuda.current_stream().cuda_stream)
    status = _lib.device_status(clear=True)  # synchronises the device
    elapsed = time.perf_counter() - t0
    assert status == 102, status  # the MMA thread's operand wait gave up
    assert elapsed < 5.0, elapsed  # the kernel returned after its short budget
    assert bool((C == 7.0).all())  # the abandoned tile wrote nothing
    # The context is intact: the next ordinary call works and leaves the status clear.
    out = ops.gemm_f16(A, B)
    assert rel_err(out, A.float() @ B.float().T) < 2e-3
    assert _lib.device_status(clear=True) == 0


def test_wait_test_hook_rejects_unbounded_budget():
    from midstream_llm_b200 import _lib
    x = torch.zeros(256, 256, device="cuda", dtype=torch.float16)
    with pytest.raises(_lib.JxError, match="wait budget"):
        _lib.call("jx_gemm_wait_test", x.data_ptr(), x.data_ptr(), x.data_ptr(), 0,
                  torch.cuda.current_stream().cuda_stream)
